// bst_halo.cu — Z-slab ghost planes across GPUs: the NCCL exchange, the overlapped slab sweep,
// and the peer-memory slab sweep whose boundary launches store straight into the neighbours'
// ghost planes over NVLink.
//
// NCCL is bound at run time with dlopen (as crates/basalto-communication/src/nccl.rs:43-85
// does), preferring the copy already loaded in the process (torch's), so a process never
// mixes two NCCL builds.  Communicators are created non-blocking and polled with a host
// timeout; on timeout they are aborted and an error is returned instead of hanging.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>  // types and enums only; every call goes through the dlopen'd table

#include <algorithm>
#include <chrono>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "bst_internal.h"
#include "bst_kernels.cuh"

namespace bst {

struct NcclApi {
  void* lib = nullptr;
  decltype(&ncclGetUniqueId) GetUniqueId = nullptr;
  decltype(&ncclCommInitRankConfig) CommInitRankConfig = nullptr;
  decltype(&ncclCommGetAsyncError) CommGetAsyncError = nullptr;
  decltype(&ncclCommAbort) CommAbort = nullptr;
  decltype(&ncclCommDestroy) CommDestroy = nullptr;
  decltype(&ncclCommFinalize) CommFinalize = nullptr;
  decltype(&ncclSend) Send = nullptr;
  decltype(&ncclRecv) Recv = nullptr;
  decltype(&ncclGroupStart) GroupStart = nullptr;
  decltype(&ncclGroupEnd) GroupEnd = nullptr;
  decltype(&ncclGetErrorString) GetErrorString = nullptr;
  decltype(&ncclGetVersion) GetVersion = nullptr;
  std::string load_error;
};

static NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    const char* env = std::getenv("BASALTO_NCCL_LIB");
    void* h = nullptr;
    if (env && *env) h = dlopen(env, RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // already in the process
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      const char* e = dlerror();
      api.load_error = e ? e : "dlopen(libnccl.so.2) failed";
      return;
    }
    api.lib = h;
#define BST_SYM(field, name) api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, name))
    BST_SYM(GetUniqueId, "ncclGetUniqueId");
    BST_SYM(CommInitRankConfig, "ncclCommInitRankConfig");
    BST_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
    BST_SYM(CommAbort, "ncclCommAbort");
    BST_SYM(CommDestroy, "ncclCommDestroy");
    BST_SYM(CommFinalize, "ncclCommFinalize");
    BST_SYM(Send, "ncclSend");
    BST_SYM(Recv, "ncclRecv");
    BST_SYM(GroupStart, "ncclGroupStart");
    BST_SYM(GroupEnd, "ncclGroupEnd");
    BST_SYM(GetErrorString, "ncclGetErrorString");
    BST_SYM(GetVersion, "ncclGetVersion");
#undef BST_SYM
    if (!api.GetUniqueId || !api.CommInitRankConfig || !api.CommGetAsyncError || !api.CommAbort ||
        !api.CommDestroy || !api.Send || !api.Recv || !api.GroupStart || !api.GroupEnd)
      api.load_error = "libnccl.so.2 lacks a required symbol";
  });
  return api;
}

static int nccl_ready() {
  NcclApi& a = nccl();
  if (!a.load_error.empty()) return fail(BST_ERR_NCCL, "NCCL unavailable: " + a.load_error);
  return BST_OK;
}

static int nccl_fail(ncclResult_t r, const char* what) {
  NcclApi& a = nccl();
  return fail(BST_ERR_NCCL, std::string(what) + ": " + (a.GetErrorString ? a.GetErrorString(r) : "error"));
}

}  // namespace bst

using namespace bst;

struct bst_comm {
  ncclComm_t comm = nullptr;
  int nranks = 0, rank = 0, device = 0;
  double timeout_s = 60.0;
  cudaStream_t comm_stream = nullptr;
  cudaEvent_t ev_bnd = nullptr, ev_comm = nullptr;
  // Deep-halo passes: boundary launches on a high-priority stream, concurrent with the
  // interior launch of the same pass.
  cudaStream_t bnd_stream = nullptr;
  cudaEvent_t ev_b[2] = {nullptr, nullptr}, ev_int = nullptr;
  // Copy transport: the upper side's boundary launch and copy get a stream pair of their own
  // (created on first use), so both sides' rows and copies proceed in parallel.
  cudaStream_t bnd2_stream = nullptr, comm2_stream = nullptr;
  cudaEvent_t ev_w = nullptr, ev_b2 = nullptr, ev_comm2 = nullptr;
  // Optional per-pass timing (bst_comm_profile_begin/end): six timing events per pass —
  // boundary start/end, exchange start/end, interior start/end.
  std::vector<cudaEvent_t> prof;
  int prof_cap = 0, prof_used = 0;
  // Peer-memory slabs (bst_comm_register_slab / bst_slab_sweeps_p2p).
  struct PeerSlab {
    char* local = nullptr;  // this rank's buffer (plane 0 = the first lower ghost plane)
    int64_t n_local = 0, plane = 0;
    int32_t ghost = 0, es = 0;
    char* lo = nullptr;  // rank-1's buffer registered in the same slot (peer mapping), or null
    char* hi = nullptr;  // rank+1's
    int64_t n_lo = 0, n_hi = 0;  // their owned planes
    int32_t g_lo = 0, g_hi = 0;  // their ghost depths
  };
  std::vector<PeerSlab> slabs;
  // flags[0]: last pass whose planes rank-1 stored here; flags[1]: the same for rank+1;
  // flags[2], flags[3]: completion counters of this rank's lower / upper boundary launches.
  unsigned long long* flags = nullptr;
  unsigned long long* flag_lo_remote = nullptr;  // rank-1's flags[1]
  unsigned long long* flag_hi_remote = nullptr;  // rank+1's flags[0]
  unsigned long long seq = 0;                     // peer passes issued so far
  void* xfer = nullptr;                           // device staging for the setup messages
  struct Mapping {
    int peer;
    cudaIpcMemHandle_t handle;
    char* base;
  };
  std::vector<Mapping> mappings;  // opened peer allocations (closed on destroy)
};

namespace bst {
// Poll a non-blocking communicator until its pending operation leaves ncclInProgress.
static int wait_comm(bst_comm* c, const char* what) {
  NcclApi& a = nccl();
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t st = ncclInProgress;
    ncclResult_t r = a.CommGetAsyncError(c->comm, &st);
    if (r != ncclSuccess) return nccl_fail(r, what);
    if (st == ncclSuccess) return BST_OK;
    if (st != ncclInProgress) return nccl_fail(st, what);
    const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el > c->timeout_s) return fail(BST_ERR_TIMEOUT, std::string(what) + ": timed out");
    // An enqueue normally completes within microseconds: poll tightly first (a sleep costs
    // ~100 us of scheduler latency per exchange), then back off so a stuck peer does not
    // burn a core until the timeout.
    if (el < 2e-3) std::this_thread::yield();
    else std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}
// Poll a stream until its work is done, bounded by the communicator's timeout (a neighbour that
// never joins the NCCL group must not hang the caller).
static int wait_stream_bounded(bst_comm* c, cudaStream_t st, const char* what) {
  NcclApi& a = nccl();
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t e = cudaStreamQuery(st);
    if (e == cudaSuccess) return BST_OK;
    if (e != cudaErrorNotReady) return cuda_fail(e, what);
    ncclResult_t st_nccl = ncclSuccess;
    if (a.CommGetAsyncError(c->comm, &st_nccl) == ncclSuccess && st_nccl != ncclSuccess && st_nccl != ncclInProgress)
      return nccl_fail(st_nccl, what);
    const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el > c->timeout_s) return fail(BST_ERR_TIMEOUT, std::string(what) + ": timed out");
    std::this_thread::sleep_for(std::chrono::microseconds(el < 2e-3 ? 5 : 100));
  }
}

// What a rank tells its neighbours about one registered buffer.
struct PeerMsg {
  cudaIpcMemHandle_t handle;
  uint64_t offset;   // the buffer's start inside that allocation
  int64_t n_local;   // owned planes
  int64_t plane;     // elements per plane
  int32_t ghost;     // ghost planes per side
  int32_t es;        // element size
};
static_assert(sizeof(PeerMsg) <= 256, "one staging slot per message");

// Send `mine` to rank-1 and rank+1 and receive theirs (zeroed where there is no neighbour).
static int swap_with_neighbours(bst_comm* c, const PeerMsg& mine, PeerMsg* from_lo, PeerMsg* from_hi) {
  std::memset(from_lo, 0, sizeof *from_lo);
  std::memset(from_hi, 0, sizeof *from_hi);
  if (c->nranks == 1) return BST_OK;
  char* x = static_cast<char*>(c->xfer);
  BST_CUDA(cudaMemcpy(x, &mine, sizeof mine, cudaMemcpyHostToDevice));
  NcclApi& a = nccl();
  ncclResult_t r = a.GroupStart();
  if (r != ncclSuccess) return nccl_fail(r, "ncclGroupStart");
  ncclResult_t e[4] = {ncclSuccess, ncclSuccess, ncclSuccess, ncclSuccess};
  if (c->rank > 0) {
    e[0] = a.Send(x, sizeof(PeerMsg), ncclUint8, c->rank - 1, c->comm, c->comm_stream);
    e[1] = a.Recv(x + 256, sizeof(PeerMsg), ncclUint8, c->rank - 1, c->comm, c->comm_stream);
  }
  if (c->rank < c->nranks - 1) {
    e[2] = a.Send(x, sizeof(PeerMsg), ncclUint8, c->rank + 1, c->comm, c->comm_stream);
    e[3] = a.Recv(x + 512, sizeof(PeerMsg), ncclUint8, c->rank + 1, c->comm, c->comm_stream);
  }
  r = a.GroupEnd();
  for (ncclResult_t v : e)
    if (v != ncclSuccess && v != ncclInProgress) return nccl_fail(v, "ncclSend/ncclRecv (peer setup)");
  if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(r, "ncclGroupEnd (peer setup)");
  int rc = wait_comm(c, "peer setup enqueue");
  if (rc) return rc;
  rc = wait_stream_bounded(c, c->comm_stream, "peer setup exchange");
  if (rc) return rc;
  if (c->rank > 0) BST_CUDA(cudaMemcpy(from_lo, x + 256, sizeof *from_lo, cudaMemcpyDeviceToHost));
  if (c->rank < c->nranks - 1) BST_CUDA(cudaMemcpy(from_hi, x + 512, sizeof *from_hi, cudaMemcpyDeviceToHost));
  return BST_OK;
}

// This rank's message for the allocation holding `p`.
static int describe(const void* p, PeerMsg* m) {
  static PFN_cuMemGetAddressRange_v3020 range = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
  });
  if (!range) return fail(BST_ERR_CUDA, "cuMemGetAddressRange entry point unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(p)) != CUDA_SUCCESS)
    return fail(BST_ERR_INVALID, "the slab buffer is not CUDA device memory");
  BST_CUDA(cudaIpcGetMemHandle(&m->handle, reinterpret_cast<void*>(base)));
  m->offset = uint64_t(reinterpret_cast<uintptr_t>(p) - uintptr_t(base));
  return BST_OK;
}

// The neighbour's buffer described by `m`, mapped into this process (each allocation once).
static int map_peer(bst_comm* c, int peer, const PeerMsg& m, char** out) {
  for (const auto& mp : c->mappings)
    if (mp.peer == peer && std::memcmp(&mp.handle, &m.handle, sizeof m.handle) == 0) {
      *out = mp.base + m.offset;
      return BST_OK;
    }
  void* base = nullptr;
  BST_CUDA(cudaIpcOpenMemHandle(&base, m.handle, cudaIpcMemLazyEnablePeerAccess));
  c->mappings.push_back(bst_comm::Mapping{peer, m.handle, static_cast<char*>(base)});
  *out = static_cast<char*>(base) + m.offset;
  return BST_OK;
}

// First use: the flag words, exchanged with the neighbours like a slab.
static int ensure_flags(bst_comm* c) {
  if (c->flags) return BST_OK;
  BST_CUDA(cudaMalloc(&c->xfer, 1024));
  void* f = nullptr;
  BST_CUDA(cudaMalloc(&f, 256));
  BST_CUDA(cudaMemset(f, 0, 256));
  c->flags = static_cast<unsigned long long*>(f);
  PeerMsg mine{}, lo{}, hi{};
  int rc = describe(c->flags, &mine);
  if (rc) return rc;
  rc = swap_with_neighbours(c, mine, &lo, &hi);
  if (rc) return rc;
  char* p = nullptr;
  if (c->rank > 0) {
    if ((rc = map_peer(c, c->rank - 1, lo, &p))) return rc;
    c->flag_lo_remote = reinterpret_cast<unsigned long long*>(p) + 1;  // rank-1 hears from its upper neighbour
  }
  if (c->rank < c->nranks - 1) {
    if ((rc = map_peer(c, c->rank + 1, hi, &p))) return rc;
    c->flag_hi_remote = reinterpret_cast<unsigned long long*>(p) + 0;  // rank+1 hears from its lower neighbour
  }
  return BST_OK;
}

}  // namespace bst

static void release_profile(bst_comm* c) {
  for (cudaEvent_t ev : c->prof)
    if (ev) cudaEventDestroy(ev);
  c->prof.clear();
  c->prof_cap = c->prof_used = 0;
}

// Records timing event `which` (0..5) of the next profiled pass on `st` (no-op when off).
static cudaError_t prof_mark(bst_comm* c, int which, cudaStream_t st) {
  if (c->prof_used >= c->prof_cap) return cudaSuccess;
  return cudaEventRecord(c->prof[size_t(c->prof_used) * 6 + which], st);
}

static void release_peers(bst_comm* c) {
  for (auto& m : c->mappings) cudaIpcCloseMemHandle(m.base);
  c->mappings.clear();
  c->slabs.clear();
  if (c->flags) cudaFree(c->flags);
  if (c->xfer) cudaFree(c->xfer);
  c->flags = nullptr;
  c->xfer = nullptr;
  c->flag_lo_remote = c->flag_hi_remote = nullptr;
}

static void release_cuda(bst_comm* c) {
  release_profile(c);
  release_peers(c);
  if (c->ev_bnd) cudaEventDestroy(c->ev_bnd);
  if (c->ev_comm) cudaEventDestroy(c->ev_comm);
  for (cudaEvent_t& ev : c->ev_b)
    if (ev) cudaEventDestroy(ev);
  if (c->ev_int) cudaEventDestroy(c->ev_int);
  if (c->comm_stream) cudaStreamDestroy(c->comm_stream);
  if (c->bnd_stream) cudaStreamDestroy(c->bnd_stream);
  for (cudaEvent_t ev : {c->ev_w, c->ev_b2, c->ev_comm2})
    if (ev) cudaEventDestroy(ev);
  if (c->bnd2_stream) cudaStreamDestroy(c->bnd2_stream);
  if (c->comm2_stream) cudaStreamDestroy(c->comm2_stream);
}

static int ensure_copy_streams(bst_comm* c) {
  if (c->comm2_stream) return BST_OK;
  int least = 0, greatest = 0;
  BST_CUDA(cudaDeviceGetStreamPriorityRange(&least, &greatest));
  BST_CUDA(cudaStreamCreateWithPriority(&c->bnd2_stream, cudaStreamNonBlocking, greatest));
  for (cudaEvent_t* ev : {&c->ev_w, &c->ev_b2, &c->ev_comm2})
    BST_CUDA(cudaEventCreateWithFlags(ev, cudaEventDisableTiming));
  BST_CUDA(cudaStreamCreateWithFlags(&c->comm2_stream, cudaStreamNonBlocking));
  return BST_OK;
}

extern "C" {

int bst_nccl_get_unique_id(uint8_t id_out[128]) {
  clear_error();
  if (!id_out) return fail(BST_ERR_INVALID, "null output");
  int rc = nccl_ready();
  if (rc) return rc;
  ncclUniqueId id;
  ncclResult_t r = nccl().GetUniqueId(&id);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  static_assert(sizeof(id) == 128, "ncclUniqueId is 128 bytes");
  std::memcpy(id_out, &id, 128);
  return BST_OK;
}

int bst_comm_create(const uint8_t id[128], int32_t nranks, int32_t rank, int32_t device, double timeout_s,
                    bst_comm** out) {
  clear_error();
  if (!id || !out) return fail(BST_ERR_INVALID, "null argument");
  if (nranks < 1 || rank < 0 || rank >= nranks) return fail(BST_ERR_INVALID, "bad rank/nranks");
  int rc = nccl_ready();
  if (rc) return rc;
  BST_CUDA(cudaSetDevice(device));
  auto* c = new bst_comm();
  c->nranks = nranks;
  c->rank = rank;
  c->device = device;
  c->timeout_s = timeout_s > 0 ? timeout_s : 60.0;
  ncclUniqueId uid;
  std::memcpy(&uid, id, 128);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = nccl().CommInitRankConfig(&c->comm, nranks, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    delete c;
    return nccl_fail(r, "ncclCommInitRankConfig");
  }
  rc = wait_comm(c, "NCCL communicator bootstrap");
  if (rc) {
    const std::string msg = bst_last_error();
    if (c->comm) nccl().CommAbort(c->comm);
    delete c;
    return fail(rc, msg);
  }
  cudaError_t e = cudaStreamCreateWithFlags(&c->comm_stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->ev_bnd, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->ev_comm, cudaEventDisableTiming);
  int prio_least = 0, prio_greatest = 0;
  if (e == cudaSuccess) e = cudaDeviceGetStreamPriorityRange(&prio_least, &prio_greatest);
  if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&c->bnd_stream, cudaStreamNonBlocking, prio_greatest);
  for (int i = 0; i < 2 && e == cudaSuccess; ++i) e = cudaEventCreateWithFlags(&c->ev_b[i], cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->ev_int, cudaEventDisableTiming);
  if (e != cudaSuccess) {
    nccl().CommAbort(c->comm);
    release_cuda(c);
    delete c;
    return cuda_fail(e, "comm stream/events");
  }
  *out = c;
  return BST_OK;
}


int bst_comm_destroy(bst_comm* c) {
  clear_error();
  if (!c) return BST_OK;
  int rc = BST_OK;
  if (c->comm) {
    cudaSetDevice(c->device);
    if (c->comm_stream) cudaStreamSynchronize(c->comm_stream);
    if (c->bnd_stream) cudaStreamSynchronize(c->bnd_stream);
    if (nccl().CommFinalize) {
      ncclResult_t r = nccl().CommFinalize(c->comm);
      if (r == ncclSuccess || r == ncclInProgress) rc = wait_comm(c, "ncclCommFinalize");
      else rc = nccl_fail(r, "ncclCommFinalize");
    }
    if (rc == BST_OK) {
      ncclResult_t r = nccl().CommDestroy(c->comm);
      if (r != ncclSuccess) rc = nccl_fail(r, "ncclCommDestroy");
    } else {
      nccl().CommAbort(c->comm);
    }
  }
  release_cuda(c);
  delete c;
  return rc;
}

int bst_comm_abort(bst_comm* c) {
  clear_error();
  if (!c) return BST_OK;
  if (c->comm) nccl().CommAbort(c->comm);
  release_cuda(c);
  delete c;
  return BST_OK;
}

int bst_comm_rank(const bst_comm* c) { return c ? c->rank : -1; }
int bst_comm_size(const bst_comm* c) { return c ? c->nranks : -1; }

static int halo_enqueue(bst_comm* c, void* slab, int32_t dtype, int64_t plane_elems, int64_t n_local,
                        int32_t ghost, cudaStream_t st) {
  if (c->nranks == 1 || ghost == 0) return BST_OK;
  const size_t es = dtype == BST_F64 ? 8 : 4;
  const ncclDataType_t nt = dtype == BST_F64 ? ncclFloat64 : ncclFloat32;
  const size_t count = size_t(ghost) * size_t(plane_elems);
  char* base = static_cast<char*>(slab);
  char* lo_ghost = base;
  char* lo_owned = base + size_t(ghost) * plane_elems * es;
  char* hi_owned = base + size_t(n_local) * plane_elems * es;
  char* hi_ghost = base + size_t(n_local + ghost) * plane_elems * es;
  NcclApi& a = nccl();
  ncclResult_t r = a.GroupStart();
  if (r != ncclSuccess) return nccl_fail(r, "ncclGroupStart");
  ncclResult_t e1 = ncclSuccess, e2 = ncclSuccess, e3 = ncclSuccess, e4 = ncclSuccess;
  if (c->rank > 0) {
    e1 = a.Send(lo_owned, count, nt, c->rank - 1, c->comm, st);
    e2 = a.Recv(lo_ghost, count, nt, c->rank - 1, c->comm, st);
  }
  if (c->rank < c->nranks - 1) {
    e3 = a.Send(hi_owned, count, nt, c->rank + 1, c->comm, st);
    e4 = a.Recv(hi_ghost, count, nt, c->rank + 1, c->comm, st);
  }
  r = a.GroupEnd();
  for (ncclResult_t e : {e1, e2, e3, e4})
    if (e != ncclSuccess && e != ncclInProgress) return nccl_fail(e, "ncclSend/ncclRecv");
  if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(r, "ncclGroupEnd");
  return wait_comm(c, "halo exchange enqueue");
}

int bst_halo_exchange(bst_comm* c, void* slab, int32_t dtype, int64_t plane_elems, int64_t n_local, int32_t ghost,
                      void* stream) {
  clear_error();
  if (!c || !slab) return fail(BST_ERR_INVALID, "null argument");
  if (dtype != BST_F32 && dtype != BST_F64) return fail(BST_ERR_UNSUPPORTED, "dtype must be float32 or float64");
  if (plane_elems <= 0 || ghost < 0 || n_local < ghost) return fail(BST_ERR_INVALID, "slab must own at least `ghost` planes");
  return halo_enqueue(c, slab, dtype, plane_elems, n_local, ghost, static_cast<cudaStream_t>(stream));
}

// Canonical form of a slab program: axis 0 widened by `ghost` planes on each side, output
// plane o reading input plane o + ghost + dm.
static int slab_canon(const bst_program* prog, int32_t ndim, const int64_t* local_shape, int32_t ghost, Canon* k,
                      int64_t s[3], int64_t* plane) {
  int rc = canonicalize(prog, ndim, local_shape, k);
  if (rc) return rc;
  if (k->boundary != BST_BOUNDARY_ZERO) return fail(BST_ERR_INVALID, "slab sweeps need a same-size program");
  const int64_t nl = local_shape[0];
  *plane = 1;
  for (int i = 1; i < ndim; ++i) *plane *= local_shape[i];
  k->n[0] = nl + 2 * int64_t(ghost);
  k->org[0] = ghost;
  k->no[0] = nl;
  int64_t st_t[3];
  int64_t acc = 1;
  for (int i = ndim - 1; i >= 0; --i) {
    st_t[i] = acc;
    acc *= (i == 0 ? nl + 2 * int64_t(ghost) : local_shape[i]);
  }
  logical_strides(ndim, st_t, s);
  return BST_OK;
}

int bst_slab_ghost_depth(const bst_program* prog, int32_t dtype, int32_t ndim, const int64_t* local_shape,
                         int32_t* ghost_out) {
  clear_error();
  if (!prog || !local_shape || !ghost_out) return fail(BST_ERR_INVALID, "null argument");
  if (dtype != BST_F32 && dtype != BST_F64) return fail(BST_ERR_UNSUPPORTED, "dtype must be float32 or float64");
  if (ndim < 2) return fail(BST_ERR_INVALID, "slabs split axis 0 of a 2-D or 3-D grid");
  Canon k;
  int64_t s[3], plane = 0;
  int rc = canonicalize(prog, ndim, local_shape, &k);
  if (rc) return rc;
  const int R = k.R[0];
  // Probe the fused kernel's limit on the widest layout it could use (16-byte aligned buffers).
  rc = slab_canon(prog, ndim, local_shape, R * 8, &k, s, &plane);
  if (rc) return rc;
  const int kmax = R > 0 ? tb_max_sweeps(k, dtype, nullptr, s, nullptr, s) : 1;
  *ghost_out = R * (kmax > 1 ? kmax : 1);
  return BST_OK;
}

}  // extern "C"

namespace bst {

// Copy-engine transport kernels.  The wait is one thread polling this GPU's flags for the
// neighbours' previous pass (bounded, like the peer-store kernel's); the set is one thread
// storing this pass's sequence number into the neighbours' flags after the copies ahead of it
// on the same stream have completed.
__global__ void slab_flags_wait_kernel(const unsigned long long* f_lo, const unsigned long long* f_hi,
                                       unsigned long long v, unsigned* err) {
  if (threadIdx.x != 0) return;
  if (f_lo) peer_wait(f_lo, v, err);
  if (f_hi) peer_wait(f_hi, v, err);
}

__global__ void slab_flags_set_kernel(unsigned long long* r_lo, unsigned long long* r_hi, unsigned long long v) {
  if (threadIdx.x != 0) return;
  __threadfence_system();
  if (r_lo) asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(r_lo), "l"(v) : "memory");
  if (r_hi) asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(r_hi), "l"(v) : "memory");
}

enum class SlabTransport { kNccl, kCopy };

// Overlapped slab passes (boundary rows, ghost transfer, interior rows) for both transports.
static int slab_passes(bst_comm* c, const bst_program* prog, int32_t dtype, int32_t ndim, const int64_t* local_shape,
                       int32_t ghost, void* a, void* b, int32_t nsteps, void* stream, SlabTransport tr) {
  if (!c || !prog || !local_shape || !a || !b) return fail(BST_ERR_INVALID, "null argument");
  if (a == b) return fail(BST_ERR_INVALID, "ping-pong slabs must differ");
  if (nsteps < 0) return fail(BST_ERR_INVALID, "negative step count");
  if (dtype != BST_F32 && dtype != BST_F64) return fail(BST_ERR_UNSUPPORTED, "dtype must be float32 or float64");
  if (ndim < 2) return fail(BST_ERR_INVALID, "slabs split axis 0 of a 2-D or 3-D grid");
  if (ghost < 0 || ghost > (1 << 20)) return fail(BST_ERR_INVALID, "ghost depth out of range");
  Canon k_canon;
  int64_t s[3], plane = 0;
  int rc = slab_canon(prog, ndim, local_shape, ghost, &k_canon, s, &plane);
  if (rc) return rc;
  const int R = k_canon.R[0];
  const int64_t nl = local_shape[0];
  if (ghost < R) return fail(BST_ERR_INVALID, "ghost depth is below the program's axis-0 radius");
  // Sweeps fused per exchange: bounded by the kernel and by the ghost depth (k*R planes).
  int kmax = 1;
  if (R > 0 && ghost >= 2 * R) {
    const int kt = tb_max_sweeps(k_canon, dtype, a, s, b, s, true);  // the caller chose the ghost depth
    kmax = kt < ghost / R ? kt : ghost / R;
  }
  const std::vector<int> plan = fuse_plan(nsteps, kmax);
  int kbig = 1;
  for (int kk : plan) kbig = kk > kbig ? kk : kbig;
  if (int64_t(kbig) * R > ghost) return fail(BST_ERR_INVALID, "fused sweeps read beyond the ghost planes");
  // Every pass refreshes all `ghost` planes per side, so the result's ghosts are complete and a
  // later call may fuse as deeply as the ghost depth allows, whatever this call fused.
  const int64_t gx = ghost;
  if (c->nranks > 1 && nl < gx) return fail(BST_ERR_INVALID, "each rank must own at least `ghost` planes");
  const size_t es = dtype == BST_F64 ? 8 : 4;
  // Intermediate levels are real data everywhere except beyond the global ends.
  const int64_t big = int64_t(1) << 40;
  const int64_t row_lo = c->rank == 0 ? 0 : -big;
  const int64_t row_hi = c->rank == c->nranks - 1 ? nl : big;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  BST_CUDA(cudaSetDevice(c->device));
  char* src = static_cast<char*>(a);
  char* dst = static_cast<char*>(b);
  const size_t ghost_bytes = size_t(ghost) * plane * es;
  const bool copy = tr == SlabTransport::kCopy && c->nranks > 1 && gx > 0;
  const bool has_lo = c->rank > 0, has_hi = c->rank < c->nranks - 1;
  // Copy transport: both buffers are registered slabs (the neighbours' mappings of the same
  // slot are where this rank's boundary planes go).
  const bst_comm::PeerSlab* reg[2] = {nullptr, nullptr};
  if (copy) {
    void* bufs[2] = {a, b};
    for (int i = 0; i < 2; ++i) {
      for (const auto& ps : c->slabs)
        if (ps.local == bufs[i] && ps.n_local == nl && ps.plane == plane && ps.ghost == ghost && size_t(ps.es) == es)
          reg[i] = &ps;
      if (!reg[i] && (i == 1 ? nsteps >= 1 : nsteps >= 2))
        return fail(BST_ERR_INVALID, "bst_slab_sweeps_copy: every buffer it writes must be registered with "
                                     "bst_comm_register_slab (same geometry)");
    }
    if (!c->flags) return fail(BST_ERR_INVALID, "bst_slab_sweeps_copy: no slab is registered on this communicator");
  }
  unsigned* err = copy ? device_error_word() : nullptr;
  if (copy && !err) return fail(BST_ERR_CUDA, "device error word unavailable");
  const int64_t lo_end = std::min<int64_t>(gx, nl);
  const int64_t hi_begin = std::max<int64_t>(nl - gx, lo_end);
  // Per pass k (src -> dst): the boundary rows run on the high-priority boundary stream,
  // concurrently with the interior rows on `st`; both read src and write disjoint rows of dst.
  //   boundary k  waits for interior k-1 (ev_int) and exchange k-1 (ev_comm: src's ghosts);
  //   exchange k  (comm stream) waits for boundary k;
  //   interior k  waits for boundary k-1 (ev_b[(k-1) % 2]; its rows are inside what interior k reads).
  // Events are waited on before they are re-recorded, so every wait sees the intended pass.
  // Copy transport, per pass k with sequence number q: the boundary stream first waits (bounded,
  // on the GPU) until both neighbours have raised their flags to q - 1, i.e. their copies of
  // pass k-1 into src's ghost planes have landed and they are done reading the ghost planes
  // that this pass's copies overwrite; after the boundary rows, the comm stream copies the
  // first / last `ghost` owned planes into the neighbours' ghost planes with the copy engines
  // (no SMs) and raises the neighbours' flags to q; the interior rows wait for the boundary
  // rows, so the copies overlap the interior launch, which holds every SM.
  const bool exchange = c->nranks > 1 && gx > 0;
  BST_CUDA(cudaEventRecord(c->ev_int, st));  // src (with its ghosts) is ready on the caller's stream
  int k = 0;
  int cur = 0;  // index of src in {a, b}
  if (copy && (rc = ensure_copy_streams(c))) return rc;
  for (int kk : plan) {
    void* out = dst + ghost_bytes;
    if (copy) {
      // Copy-transport pass: lower side on (bnd, comm), upper side on (bnd2, comm2).
      const unsigned long long q = ++c->seq;
      const bst_comm::PeerSlab* dr = reg[1 - cur];
      const size_t pb = size_t(plane) * es;
      if (k > 0) BST_CUDA(cudaStreamWaitEvent(c->bnd_stream, c->ev_comm, 0));  // own copies out of dst
      slab_flags_wait_kernel<<<1, 32, 0, c->bnd_stream>>>(has_lo ? c->flags + 0 : nullptr,
                                                          has_hi ? c->flags + 1 : nullptr, q - 1, err);
      BST_CUDA(cudaGetLastError());
      BST_CUDA(cudaStreamWaitEvent(c->bnd_stream, c->ev_int, 0));
      BST_CUDA(cudaEventRecord(c->ev_w, c->bnd_stream));
      BST_CUDA(cudaStreamWaitEvent(c->bnd2_stream, c->ev_w, 0));
      BST_CUDA(prof_mark(c, 0, c->bnd_stream));
      if (kk == 1 && hi_begin < nl && nl - hi_begin == lo_end) {
        // single sweep: both boundary ranges in one launch (one ramp, fuller waves)
        rc = launch_sweep(k_canon, dtype, src, s, out, s, 0, lo_end, c->bnd_stream, nullptr, hi_begin, nl);
        if (rc) return rc;
        BST_CUDA(cudaEventRecord(c->ev_b[k % 2], c->bnd_stream));
        BST_CUDA(cudaEventRecord(c->ev_b2, c->bnd_stream));
      } else {
        rc = launch_fused(k_canon, dtype, src, s, out, s, kk, 0, lo_end, row_lo, row_hi, c->bnd_stream);
        if (rc) return rc;
        BST_CUDA(cudaEventRecord(c->ev_b[k % 2], c->bnd_stream));
        if (hi_begin < nl) {
          rc = launch_fused(k_canon, dtype, src, s, out, s, kk, hi_begin, nl, row_lo, row_hi, c->bnd2_stream);
          if (rc) return rc;
        }
        BST_CUDA(cudaEventRecord(c->ev_b2, c->bnd2_stream));
      }
      BST_CUDA(cudaStreamWaitEvent(c->bnd_stream, c->ev_b2, 0));  // boundary end mark covers both sides
      BST_CUDA(prof_mark(c, 1, c->bnd_stream));
      // owned planes [nl - gx, nl) -> rank+1's lower ghost planes, then its flag
      BST_CUDA(cudaStreamWaitEvent(c->comm2_stream, c->ev_b2, 0));
      if (has_hi) {
        BST_CUDA(cudaMemcpyAsync(dr->hi + size_t(dr->g_hi - gx) * pb, dst + ghost_bytes + size_t(nl - gx) * pb,
                                 size_t(gx) * pb, cudaMemcpyDeviceToDevice, c->comm2_stream));
        slab_flags_set_kernel<<<1, 32, 0, c->comm2_stream>>>(nullptr, c->flag_hi_remote, q);
        BST_CUDA(cudaGetLastError());
      }
      BST_CUDA(cudaEventRecord(c->ev_comm2, c->comm2_stream));
      // owned planes [0, gx) -> rank-1's upper ghost planes, then its flag
      BST_CUDA(cudaStreamWaitEvent(c->comm_stream, c->ev_b[k % 2], 0));
      BST_CUDA(prof_mark(c, 2, c->comm_stream));
      if (has_lo) {
        BST_CUDA(cudaMemcpyAsync(dr->lo + size_t(dr->g_lo + dr->n_lo) * pb, dst + ghost_bytes, size_t(gx) * pb,
                                 cudaMemcpyDeviceToDevice, c->comm_stream));
        slab_flags_set_kernel<<<1, 32, 0, c->comm_stream>>>(c->flag_lo_remote, nullptr, q);
        BST_CUDA(cudaGetLastError());
      }
      BST_CUDA(cudaStreamWaitEvent(c->comm_stream, c->ev_comm2, 0));  // ev_comm covers both sides
      BST_CUDA(prof_mark(c, 3, c->comm_stream));
      BST_CUDA(cudaEventRecord(c->ev_comm, c->comm_stream));
      // interior rows after both sides' boundary rows
      BST_CUDA(cudaStreamWaitEvent(st, c->ev_b[k % 2], 0));
      BST_CUDA(cudaStreamWaitEvent(st, c->ev_b2, 0));
    } else {
      BST_CUDA(cudaStreamWaitEvent(c->bnd_stream, c->ev_int, 0));
      if (k > 0 && exchange) BST_CUDA(cudaStreamWaitEvent(c->bnd_stream, c->ev_comm, 0));
      BST_CUDA(prof_mark(c, 0, c->bnd_stream));
      rc = launch_fused(k_canon, dtype, src, s, out, s, kk, 0, lo_end, row_lo, row_hi, c->bnd_stream);
      if (!rc && hi_begin < nl)
        rc = launch_fused(k_canon, dtype, src, s, out, s, kk, hi_begin, nl, row_lo, row_hi, c->bnd_stream);
      if (rc) return rc;
      BST_CUDA(prof_mark(c, 1, c->bnd_stream));
      BST_CUDA(cudaEventRecord(c->ev_b[k % 2], c->bnd_stream));
      if (exchange) {
        BST_CUDA(cudaStreamWaitEvent(c->comm_stream, c->ev_b[k % 2], 0));
        BST_CUDA(prof_mark(c, 2, c->comm_stream));
        rc = halo_enqueue(c, dst, dtype, plane, nl, int32_t(gx), c->comm_stream);
        if (rc) return rc;
        BST_CUDA(prof_mark(c, 3, c->comm_stream));
        BST_CUDA(cudaEventRecord(c->ev_comm, c->comm_stream));
      }
      if (k > 0) BST_CUDA(cudaStreamWaitEvent(st, c->ev_b[(k - 1) % 2], 0));
    }
    BST_CUDA(prof_mark(c, 4, st));
    if (lo_end < hi_begin) {
      rc = launch_fused(k_canon, dtype, src, s, out, s, kk, lo_end, hi_begin, row_lo, row_hi, st);
      if (rc) return rc;
    }
    BST_CUDA(prof_mark(c, 5, st));
    if (c->prof_used < c->prof_cap) {
      if (!exchange) {  // no exchange: a zero-length exchange interval at the boundary's end
        BST_CUDA(cudaEventRecord(c->prof[size_t(c->prof_used) * 6 + 2], c->bnd_stream));
        BST_CUDA(cudaEventRecord(c->prof[size_t(c->prof_used) * 6 + 3], c->bnd_stream));
      }
      ++c->prof_used;
    }
    BST_CUDA(cudaEventRecord(c->ev_int, st));
    std::swap(src, dst);
    cur = 1 - cur;
    ++k;
  }
  if (k > 0 && copy) BST_CUDA(cudaStreamWaitEvent(st, c->ev_b2, 0));
  if (k > 0) {
    BST_CUDA(cudaStreamWaitEvent(st, c->ev_b[(k - 1) % 2], 0));
    if (exchange) BST_CUDA(cudaStreamWaitEvent(st, c->ev_comm, 0));
  }
  return BST_OK;
}

}  // namespace bst

extern "C" {

int bst_slab_sweeps_deep(bst_comm* c, const bst_program* prog, int32_t dtype, int32_t ndim,
                         const int64_t* local_shape, int32_t ghost, void* a, void* b, int32_t nsteps, void* stream) {
  clear_error();
  return slab_passes(c, prog, dtype, ndim, local_shape, ghost, a, b, nsteps, stream, SlabTransport::kNccl);
}

int bst_slab_sweeps_copy(bst_comm* c, const bst_program* prog, int32_t dtype, int32_t ndim,
                         const int64_t* local_shape, int32_t ghost, void* a, void* b, int32_t nsteps, void* stream) {
  clear_error();
  return slab_passes(c, prog, dtype, ndim, local_shape, ghost, a, b, nsteps, stream, SlabTransport::kCopy);
}

int bst_comm_profile_begin(bst_comm* c, int32_t max_passes) {
  clear_error();
  if (!c) return fail(BST_ERR_INVALID, "null communicator");
  if (max_passes < 1 || max_passes > (1 << 16)) return fail(BST_ERR_INVALID, "max_passes must be in 1..65536");
  BST_CUDA(cudaSetDevice(c->device));
  release_profile(c);
  c->prof.assign(size_t(max_passes) * 6, nullptr);
  for (cudaEvent_t& ev : c->prof) {
    cudaError_t e = cudaEventCreate(&ev);
    if (e != cudaSuccess) {
      release_profile(c);
      return cuda_fail(e, "profiling events");
    }
  }
  c->prof_cap = max_passes;
  c->prof_used = 0;
  return BST_OK;
}

int bst_comm_profile_end(bst_comm* c, double out[6]) {
  clear_error();
  if (!c || !out) return fail(BST_ERR_INVALID, "null argument");
  for (int i = 0; i < 6; ++i) out[i] = 0.0;
  if (c->prof_cap == 0) return fail(BST_ERR_INVALID, "profiling was not started");
  BST_CUDA(cudaSetDevice(c->device));
  int rc = BST_OK;
  for (int p = 0; p < c->prof_used && rc == BST_OK; ++p) {
    cudaEvent_t* e = &c->prof[size_t(p) * 6];
    float t_b = 0, t_x = 0, t_i = 0, t_end_i = 0, t_end_x = 0;
    cudaError_t err = cudaEventSynchronize(e[5]);
    if (err == cudaSuccess) err = cudaEventSynchronize(e[3]);
    if (err == cudaSuccess) err = cudaEventElapsedTime(&t_b, e[0], e[1]);
    if (err == cudaSuccess) err = cudaEventElapsedTime(&t_x, e[2], e[3]);
    if (err == cudaSuccess) err = cudaEventElapsedTime(&t_i, e[4], e[5]);
    if (err == cudaSuccess) err = cudaEventElapsedTime(&t_end_i, e[0], e[5]);
    if (err == cudaSuccess) err = cudaEventElapsedTime(&t_end_x, e[0], e[3]);
    if (err != cudaSuccess) {
      rc = cuda_fail(err, "reading the profiling events");
      break;
    }
    out[0] += t_b;
    out[1] += t_x;
    out[2] += t_i;
    out[3] += t_end_i > t_end_x ? t_end_i : t_end_x;  // pass span: boundary start to last end
    out[5] += t_end_x - t_end_i > 0 ? t_end_x - t_end_i : 0;  // exchange left over after the interior
  }
  out[4] = double(c->prof_used);
  release_profile(c);
  return rc;
}

int bst_comm_register_slab(bst_comm* c, void* buf, int32_t dtype, int64_t plane_elems, int64_t n_local,
                           int32_t ghost) {
  clear_error();
  if (!c || !buf) return fail(BST_ERR_INVALID, "null argument");
  if (dtype != BST_F32 && dtype != BST_F64) return fail(BST_ERR_UNSUPPORTED, "dtype must be float32 or float64");
  if (plane_elems <= 0 || n_local <= 0 || ghost < 0) return fail(BST_ERR_INVALID, "bad slab geometry");
  BST_CUDA(cudaSetDevice(c->device));
  int rc = ensure_flags(c);
  if (rc) return rc;
  PeerMsg mine{}, lo{}, hi{};
  if ((rc = describe(buf, &mine))) return rc;
  mine.n_local = n_local;
  mine.plane = plane_elems;
  mine.ghost = ghost;
  mine.es = dtype == BST_F64 ? 8 : 4;
  if ((rc = swap_with_neighbours(c, mine, &lo, &hi))) return rc;
  bst_comm::PeerSlab ps;
  ps.local = static_cast<char*>(buf);
  ps.n_local = n_local;
  ps.plane = plane_elems;
  ps.ghost = ghost;
  ps.es = mine.es;
  for (int side = 0; side < 2; ++side) {
    const bool has = side == 0 ? c->rank > 0 : c->rank < c->nranks - 1;
    if (!has) continue;
    const PeerMsg& m = side == 0 ? lo : hi;
    if (m.plane != plane_elems || m.es != mine.es || m.ghost != ghost)
      return fail(BST_ERR_INVALID, "neighbouring slabs registered in the same slot differ in plane size, dtype or "
                                   "ghost depth (register the buffers in the same order on every rank)");
    char* p = nullptr;
    if ((rc = map_peer(c, side == 0 ? c->rank - 1 : c->rank + 1, m, &p))) return rc;
    if (side == 0) {
      ps.lo = p;
      ps.n_lo = m.n_local;
      ps.g_lo = m.ghost;
    } else {
      ps.hi = p;
      ps.n_hi = m.n_local;
      ps.g_hi = m.ghost;
    }
  }
  c->slabs.push_back(ps);
  return BST_OK;
}

int bst_slab_sweeps_p2p(bst_comm* c, const bst_program* prog, int32_t dtype, int32_t ndim, const int64_t* local_shape,
                        int32_t ghost, void* a, void* b, int32_t nsteps, void* stream) {
  clear_error();
  if (!c || !prog || !local_shape || !a || !b) return fail(BST_ERR_INVALID, "null argument");
  if (a == b) return fail(BST_ERR_INVALID, "ping-pong slabs must differ");
  if (nsteps < 0) return fail(BST_ERR_INVALID, "negative step count");
  if (dtype != BST_F32 && dtype != BST_F64) return fail(BST_ERR_UNSUPPORTED, "dtype must be float32 or float64");
  if (ndim < 2 || ndim > 3) return fail(BST_ERR_INVALID, "slabs split axis 0 of a 2-D or 3-D grid");
  Canon k_canon;
  int64_t s[3], plane = 0;
  int rc = slab_canon(prog, ndim, local_shape, ghost, &k_canon, s, &plane);
  if (rc) return rc;
  const int R = k_canon.R[0];
  const int64_t nl = local_shape[0];
  const int64_t G = ghost;
  if (ghost < R || ghost < 1) return fail(BST_ERR_INVALID, "ghost depth is below the program's axis-0 radius");
  if (nl < 2 * G) return fail(BST_ERR_INVALID, "each rank must own at least 2 x ghost planes");
  const size_t es = dtype == BST_F64 ? 8 : 4;
  // Both buffers receive boundary planes from the neighbours, so both must be registered slabs.
  const bst_comm::PeerSlab* reg[2] = {nullptr, nullptr};
  void* bufs[2] = {a, b};
  for (int i = 0; i < 2; ++i) {
    for (const auto& ps : c->slabs)
      if (ps.local == bufs[i] && ps.n_local == nl && ps.plane == plane && ps.ghost == ghost && size_t(ps.es) == es)
        reg[i] = &ps;
    const bool written = i == 1 ? nsteps >= 1 : nsteps >= 2;  // pass k writes bufs[(k + 1) % 2]
    if (!reg[i] && c->nranks > 1 && written)
      return fail(BST_ERR_INVALID, "bst_slab_sweeps_p2p: every buffer it writes must be registered with "
                                   "bst_comm_register_slab (same geometry)");
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  BST_CUDA(cudaSetDevice(c->device));
  const size_t ghost_bytes = size_t(G) * plane * es;
  const bool lo = c->nranks > 1 && c->rank > 0, hi = c->nranks > 1 && c->rank < c->nranks - 1;
  int cur = 0;  // index of src in bufs
  for (int k = 0; k < nsteps; ++k) {
    char* src = static_cast<char*>(bufs[cur]);
    char* dst = static_cast<char*>(bufs[1 - cur]);
    const bst_comm::PeerSlab* dreg = reg[1 - cur];
    void* out = dst + ghost_bytes;
    // One launch per sweep.  Items holding the first / last G owned planes also store them
    // into the neighbours' ghost planes and raise their flags when all such items are done;
    // items reading ghost planes first wait for the neighbours' previous sweep.
    PeerStore pe{};
    pe.seq = ++c->seq;
    pe.wait_value = pe.seq - 1;
    pe.done = c->flags + 2;
    pe.lo_end = 0;
    pe.hi_begin = int(nl);
    if (lo) {  // owned plane m (< G) -> rank-1's upper ghost plane g_lo + n_lo + m
      pe.delta_lo = (long long)(intptr_t(dreg->lo) - intptr_t(dst)) +
                    (long long)(dreg->g_lo + dreg->n_lo - G) * (long long)(plane * es);
      pe.lo_end = int(G);
      pe.wait_lo = c->flags + 0;
      pe.flag_lo = c->flag_lo_remote;
    }
    if (hi) {  // owned plane m (>= nl - G) -> rank+1's lower ghost plane m - (nl - G)
      pe.delta_hi = (long long)(intptr_t(dreg->hi) - intptr_t(dst)) - (long long)nl * (long long)(plane * es);
      pe.hi_begin = int(nl - G);
      pe.wait_hi = c->flags + 1;
      pe.flag_hi = c->flag_hi_remote;
    }
    const bool prof = c->prof_used < c->prof_cap;
    if (prof)  // the whole sweep is one launch: boundary and exchange ride inside it
      for (int i = 0; i < 6; ++i)
        if (i != 5) BST_CUDA(cudaEventRecord(c->prof[size_t(c->prof_used) * 6 + i], st));
    rc = launch_sweep(k_canon, dtype, src, s, out, s, 0, nl, st, (lo || hi) ? &pe : nullptr);
    if (rc) return rc;
    if (prof) {
      BST_CUDA(cudaEventRecord(c->prof[size_t(c->prof_used) * 6 + 5], st));
      ++c->prof_used;
    }
    cur = 1 - cur;
  }
  return BST_OK;
}

int bst_slab_sweeps(bst_comm* c, const bst_program* prog, int32_t dtype, int32_t ndim, const int64_t* local_shape,
                    void* a, void* b, int32_t nsteps, void* stream) {
  clear_error();
  if (!prog || !local_shape) return fail(BST_ERR_INVALID, "null argument");
  if (ndim < 2 || ndim > 3) return fail(BST_ERR_INVALID, "slabs split axis 0 of a 2-D or 3-D grid");
  Canon k;
  const int rc = canonicalize(prog, ndim, local_shape, &k);
  if (rc) return rc;
  return bst_slab_sweeps_deep(c, prog, dtype, ndim, local_shape, k.R[0], a, b, nsteps, stream);
}

}  // extern "C"
