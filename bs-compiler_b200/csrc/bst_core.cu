// bst_core.cu — C-ABI core: errors, program canonicalisation, sweeps, device queries.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

#include "bst_internal.h"
#include "bst_plan.h"

namespace bst {

// ---- errors ---------------------------------------------------------------------
static thread_local std::string t_last_error;
std::atomic<uint64_t> g_launches{0};

void set_error(const std::string& msg) { t_last_error = msg; }
void clear_error() { t_last_error.clear(); }
int fail(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}
int cuda_fail(cudaError_t e, const char* what) {
  t_last_error = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
  return e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver ? BST_ERR_NO_DEVICE : BST_ERR_CUDA;
}

// ---- device helpers -------------------------------------------------------------
int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = v > 0 ? v : 148;
  }
  return cache[dev];
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int occupancy(const void* fn, int threads, int smem) {
  static std::mutex mu;
  static std::unordered_map<std::string, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  char key[96];
  std::snprintf(key, sizeof key, "%p/%d/%d/%d", fn, threads, smem, dev);
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int n = 0;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, threads, smem) != cudaSuccess) return 0;
  cache[key] = n;
  return n;
}

unsigned* device_error_word() {
  static std::mutex mu;
  static unsigned* words[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (!words[dev]) {
    void* p = nullptr;
    if (cudaMalloc(&p, 256) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, 256) != cudaSuccess) return nullptr;
    words[dev] = static_cast<unsigned*>(p);
  }
  return words[dev];
}

// Runtime-table programs resident on each device (launch_direct_table).  Keyed by the
// table's bytes: FNV-1a digest first, then a full comparison.
const void* cached_device_table(const void* blob, size_t bytes) {
  struct Entry {
    std::vector<unsigned char> host;
    void* dev;
  };
  static std::mutex mu;
  static std::unordered_map<uint64_t, std::vector<Entry>> cache[64];
  static int count[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  const unsigned char* b = static_cast<const unsigned char*>(blob);
  uint64_t h = 1469598103934665603ull;
  for (size_t i = 0; i < bytes; ++i) h = (h ^ b[i]) * 1099511628211ull;
  std::lock_guard<std::mutex> lk(mu);
  auto& bucket = cache[dev][h];
  for (const Entry& e : bucket)
    if (e.host.size() == bytes && std::memcmp(e.host.data(), b, bytes) == 0) return e.dev;
  if (count[dev] >= kTableCacheMax) return nullptr;
  void* d = nullptr;
  if (cudaMalloc(&d, bytes) != cudaSuccess) return nullptr;
  // Synchronous copy: the entry is complete before any stream can launch with it.
  if (cudaMemcpy(d, b, bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaFree(d);
    return nullptr;
  }
  bucket.push_back(Entry{std::vector<unsigned char>(b, b + bytes), d});
  ++count[dev];
  return d;
}

int check_device_error(cudaStream_t st) {
  unsigned* w = device_error_word();
  if (!w) return fail(BST_ERR_CUDA, "device error word unavailable");
  unsigned h = 0;
  BST_CUDA(cudaMemcpyAsync(&h, w, sizeof h, cudaMemcpyDeviceToHost, st));
  BST_CUDA(cudaStreamSynchronize(st));
  if (h != 0) {
    BST_CUDA(cudaMemsetAsync(w, 0, sizeof h, st));
    BST_CUDA(cudaStreamSynchronize(st));
    std::string what;
    if (h & 1u) what += "a TMA stage that never landed";
    if (h & 2u) what += std::string(what.empty() ? "" : " and ") + "a neighbour's ghost planes that never arrived";
    if (what.empty()) what = "an unknown wait";
    return fail(BST_ERR_TIMEOUT, "a kernel gave up waiting for " + what + " (error bits " + std::to_string(h) + ")");
  }
  return BST_OK;
}

// ---- programs ---------------------------------------------------------------------
static void to_logical(int ndim, const int32_t o[3], Tap* t) {
  if (ndim == 1) *t = Tap{0, 0, o[0]};
  else if (ndim == 2) *t = Tap{o[0], 0, o[1]};
  else *t = Tap{o[0], o[1], o[2]};
}
static void extents_logical(int ndim, const int64_t* s, int64_t out[3]) {
  if (ndim == 1) { out[0] = 1; out[1] = 1; out[2] = s[0]; }
  else if (ndim == 2) { out[0] = s[0]; out[1] = 1; out[2] = s[1]; }
  else { out[0] = s[0]; out[1] = s[1]; out[2] = s[2]; }
}

void logical_strides(int ndim, const int64_t* st, int64_t out[3]) {
  if (ndim == 1) { out[0] = st[0]; out[1] = st[0]; out[2] = st[0]; }
  else if (ndim == 2) { out[0] = st[0]; out[1] = st[0]; out[2] = st[1]; }
  else { out[0] = st[0]; out[1] = st[1]; out[2] = st[2]; }
}

int canonicalize(const bst_program* p, int ndim, const int64_t* shape, Canon* c) {
  if (!p) return fail(BST_ERR_INVALID, "null program");
  if (ndim < 1 || ndim > 3) return fail(BST_ERR_INVALID, "only 1-D, 2-D and 3-D grids are supported (ndim=" + std::to_string(ndim) + ")");
  if (p->ndim != ndim) return fail(BST_ERR_INVALID, "program ndim does not match the grid");
  if (p->ntaps < 1 || p->ntaps > BST_MAX_TAPS) return fail(BST_ERR_INVALID, "ntaps out of range");
  if (p->nterms < 1 || p->nterms > BST_MAX_TERMS) return fail(BST_ERR_INVALID, "nterms out of range");
  if (p->boundary != BST_BOUNDARY_ZERO && p->boundary != BST_BOUNDARY_VALID)
    return fail(BST_ERR_INVALID, "unknown boundary mode");
  for (int i = 0; i < ndim; ++i)
    if (shape[i] <= 0) return fail(BST_ERR_INVALID, "non-positive extent");
  int next = 0;
  for (int g = 0; g < p->nterms; ++g) {
    if (p->term_first[g] != next || p->term_count[g] < 1)
      return fail(BST_ERR_INVALID, "terms must partition the taps in order");
    if (p->term_op[g] < BST_TERM_SUM || p->term_op[g] > BST_TERM_DIV)
      return fail(BST_ERR_INVALID, "unknown term operator");
    next += p->term_count[g];
  }
  if (next != p->ntaps) return fail(BST_ERR_INVALID, "terms must cover every tap");

  Canon k;
  k.ndim = ndim;
  k.boundary = p->boundary;
  k.init_zero = p->init_zero ? 1 : 0;
  if (p->flags & ~int32_t(BST_PROGRAM_CONTRACT)) return fail(BST_ERR_INVALID, "unknown program flags");
  k.contract = (p->flags & BST_PROGRAM_CONTRACT) ? 1 : 0;
  k.ntaps = p->ntaps;
  k.nterms = p->nterms;
  k.taps.resize(p->ntaps);
  k.terms.resize(p->nterms);
  k.scale.resize(p->nterms);
  for (int g = 0; g < p->nterms; ++g) {
    k.terms[g] = Term{p->term_first[g], p->term_count[g], p->term_op[g]};
    k.scale[g] = p->term_scale[g];
  }
  for (int i = 0; i < p->ntaps; ++i) {
    for (int a = ndim; a < 3; ++a)
      if (p->tap[i][a] != 0) return fail(BST_ERR_INVALID, "tap offset on an axis beyond ndim");
    for (int a = 0; a < ndim; ++a)
      if (p->tap[i][a] < -64 || p->tap[i][a] > 64) return fail(BST_ERR_UNSUPPORTED, "tap offset beyond +-64");
    to_logical(ndim, p->tap[i], &k.taps[i]);
  }
  extents_logical(ndim, shape, k.n);
  if (p->boundary == BST_BOUNDARY_ZERO) {
    for (int a = 0; a < 3; ++a) k.no[a] = k.n[a];
  } else {
    int64_t outs[3];
    for (int a = 0; a < ndim; ++a) {
      outs[a] = p->out_shape[a];
      if (outs[a] <= 0) return fail(BST_ERR_INVALID, "valid-region output extent must be positive");
    }
    extents_logical(ndim, outs, k.no);
    // Taps are relative to the output index and must stay inside the input.
    for (int a = 0; a < 3; ++a) {
      int lo = 1 << 30, hi = -(1 << 30);
      for (int i = 0; i < k.ntaps; ++i) {
        const int v = a == 0 ? k.taps[i].dm : (a == 1 ? k.taps[i].dy : k.taps[i].dx);
        lo = std::min(lo, v);
        hi = std::max(hi, v);
      }
      if (lo < 0 || k.no[a] - 1 + hi > k.n[a] - 1)
        return fail(BST_ERR_INVALID, "valid-region taps read outside the input");
      const int o = (lo + hi) >= 0 ? (lo + hi) / 2 : -((-(lo + hi) + 1) / 2);
      k.org[a] = o;
      for (int i = 0; i < k.ntaps; ++i) {
        if (a == 0) k.taps[i].dm -= o;
        else if (a == 1) k.taps[i].dy -= o;
        else k.taps[i].dx -= o;
      }
    }
  }
  for (int i = 0; i < k.ntaps; ++i) {
    k.R[0] = std::max(k.R[0], std::abs(k.taps[i].dm));
    k.R[1] = std::max(k.R[1], std::abs(k.taps[i].dy));
    k.R[2] = std::max(k.R[2], std::abs(k.taps[i].dx));
  }
  *c = std::move(k);
  return BST_OK;
}

struct LaunchReq;
template <typename T>
int dispatch_sweep(const LaunchReq& r);
int dispatch_f32(const Canon& c, const void* x, const int64_t xs[3], void* y, const int64_t ys[3],
                 int64_t m_lo, int64_t m_hi, cudaStream_t st, const PeerStore* peer, int64_t m2_lo, int64_t m2_hi);
int dispatch_f64(const Canon& c, const void* x, const int64_t xs[3], void* y, const int64_t ys[3],
                 int64_t m_lo, int64_t m_hi, cudaStream_t st, const PeerStore* peer, int64_t m2_lo, int64_t m2_hi);
int tb_max_f32(const Canon& c, const void* x, const int64_t xs[3], void* y, const int64_t ys[3], bool capability);
int tb_max_f64(const Canon& c, const void* x, const int64_t xs[3], void* y, const int64_t ys[3], bool capability);
int dispatch_tb_f32(const Canon& c, const void* x, const int64_t xs[3], void* y, const int64_t ys[3], int k,
                    int64_t m_lo, int64_t m_hi, int64_t row_lo, int64_t row_hi, cudaStream_t st);
int dispatch_tb_f64(const Canon& c, const void* x, const int64_t xs[3], void* y, const int64_t ys[3], int k,
                    int64_t m_lo, int64_t m_hi, int64_t row_lo, int64_t row_hi, cudaStream_t st);

int launch_sweep(const Canon& c, int dtype, const void* x, const int64_t xs[3], void* y,
                 const int64_t ys[3], int64_t m_lo, int64_t m_hi, cudaStream_t st, const PeerStore* peer,
                 int64_t m2_lo, int64_t m2_hi) {
  if (dtype == BST_F32) return dispatch_f32(c, x, xs, y, ys, m_lo, m_hi, st, peer, m2_lo, m2_hi);
  if (dtype == BST_F64) return dispatch_f64(c, x, xs, y, ys, m_lo, m_hi, st, peer, m2_lo, m2_hi);
  return fail(BST_ERR_UNSUPPORTED, "dtype must be float32 or float64");
}

Schedule march_schedule() {
  static const Schedule s = [] {
    const char* e = std::getenv("BST_MARCH_SCHEDULE");
    if (e && std::strcmp(e, "balanced") == 0) return Schedule::kBalanced;
    if (e && std::strcmp(e, "lockstep") == 0) return Schedule::kLockstep;
    return Schedule::kItems;
  }();
  return s;
}

int tb_max_sweeps(const Canon& c, int dtype, const void* x, const int64_t xs[3], void* y, const int64_t ys[3],
                  bool capability) {
  if (dtype == BST_F32) return tb_max_f32(c, x, xs, y, ys, capability);
  if (dtype == BST_F64) return tb_max_f64(c, x, xs, y, ys, capability);
  return 1;
}

int launch_fused(const Canon& c, int dtype, const void* x, const int64_t xs[3], void* y, const int64_t ys[3],
                 int k, int64_t m_lo, int64_t m_hi, int64_t row_lo, int64_t row_hi, cudaStream_t st) {
  if (k == 1) return launch_sweep(c, dtype, x, xs, y, ys, m_lo, m_hi, st);
  if (dtype == BST_F32) return dispatch_tb_f32(c, x, xs, y, ys, k, m_lo, m_hi, row_lo, row_hi, st);
  if (dtype == BST_F64) return dispatch_tb_f64(c, x, xs, y, ys, k, m_lo, m_hi, row_lo, row_hi, st);
  return fail(BST_ERR_UNSUPPORTED, "dtype must be float32 or float64");
}

std::vector<int> fuse_plan(int nsteps, int kmax) {
  std::vector<int> ks;
  if (kmax < 2 || nsteps < 2) {
    ks.assign(size_t(nsteps > 0 ? nsteps : 0), 1);
    return ks;
  }
  // Fewest launches of at most kmax sweeps, one more if their count has the wrong parity;
  // the sweeps are then spread evenly (larger launches first), so no launch is left with a
  // single sweep when n >= 2 x launches.
  int launches = (nsteps + kmax - 1) / kmax;
  if ((launches & 1) != (nsteps & 1)) ++launches;
  const int base = nsteps / launches, rem = nsteps % launches;
  for (int i = 0; i < launches; ++i) ks.push_back(base + (i < rem ? 1 : 0));
  return ks;
}

static void contiguous_strides(int ndim, const int64_t* shape, int64_t* st) {
  int64_t s = 1;
  for (int i = ndim - 1; i >= 0; --i) {
    st[i] = s;
    s *= shape[i];
  }
}

static int64_t span_elems(int ndim, const int64_t* shape, const int64_t* st, int64_t* lo_out) {
  int64_t lo = 0, hi = 0;
  for (int i = 0; i < ndim; ++i) {
    const int64_t e = (shape[i] - 1) * st[i];
    if (e < 0) lo += e;
    else hi += e;
  }
  *lo_out = lo;
  return hi - lo + 1;
}

static int elem_size(int dtype) { return dtype == BST_F64 ? 8 : 4; }

}  // namespace bst

using namespace bst;

extern "C" {

int bst_abi_version(void) { return BST_ABI_VERSION; }
const char* bst_last_error(void) { return t_last_error.c_str(); }
uint64_t bst_launch_count(void) { return g_launches.load(); }

int bst_device_error_check(void* stream) {
  clear_error();
  return check_device_error(static_cast<cudaStream_t>(stream));
}

int32_t bst_extract_radius(const char* op) {
  // "_r<k>": the text after the first "_r" must parse as an unsigned integer
  // (interceptor.rs:197-200 uses split("_r").nth(1).parse::<usize>()).
  if (!op) return 1;
  const char* pos = std::strstr(op, "_r");
  if (pos) {
    const char* s = pos + 2;
    const char* e = std::strstr(s, "_r");  // nth(1) ends at the next "_r"
    const size_t len = e ? size_t(e - s) : std::strlen(s);
    if (len > 0 && len < 20) {
      bool digits = true;
      for (size_t i = 0; i < len; ++i) digits = digits && (s[i] >= '0' && s[i] <= '9');
      if (digits) {
        long long v = 0;
        for (size_t i = 0; i < len; ++i) v = v * 10 + (s[i] - '0');
        if (v <= INT32_MAX) return int32_t(v);
      }
    }
  }
  if (std::strstr(op, "order_8")) return 4;
  if (std::strstr(op, "order_12")) return 6;
  return 1;
}

int bst_program_box(int32_t ndim, int32_t radius, const double* coeffs, int64_t ncoeffs, bst_program* out) {
  clear_error();
  if (!out) return fail(BST_ERR_INVALID, "null output program");
  if (ndim < 1 || ndim > 3) return fail(BST_ERR_INVALID, "only 1-D, 2-D and 3-D boxes");
  if (radius < 0) return fail(BST_ERR_INVALID, "negative radius");
  int64_t w = 2 * int64_t(radius) + 1, n = 1;
  for (int i = 0; i < ndim; ++i) n *= w;
  if (n > BST_MAX_TAPS || n > BST_MAX_TERMS)
    return fail(BST_ERR_UNSUPPORTED, "box of " + std::to_string(n) + " taps exceeds the program limit of " +
                                         std::to_string(BST_MAX_TAPS) + " taps");
  if (coeffs && ncoeffs != n)
    return fail(BST_ERR_INVALID, "expected " + std::to_string(n) + " coefficients, got " + std::to_string(ncoeffs));
  std::memset(out, 0, sizeof *out);
  out->ndim = ndim;
  out->ntaps = int32_t(n);
  out->nterms = int32_t(n);
  out->init_zero = 1;  // sum = 0.0; sum += v*c  (executor.rs:217-224)
  out->boundary = BST_BOUNDARY_ZERO;
  const double iso = 1.0 / double(n);  // flir_builder.rs:62-64
  for (int64_t k = 0; k < n; ++k) {
    int64_t r = k;
    int32_t o[3] = {0, 0, 0};
    for (int a = ndim - 1; a >= 0; --a) {
      o[a] = int32_t(r % w) - radius;
      r /= w;
    }
    for (int a = 0; a < 3; ++a) out->tap[k][a] = o[a];
    out->term_first[k] = int32_t(k);
    out->term_count[k] = 1;
    out->term_op[k] = BST_TERM_MUL;
    out->term_scale[k] = coeffs ? coeffs[k] : iso;
  }
  return BST_OK;
}

int bst_stencil_apply(const bst_program* prog, int32_t dtype, int32_t ndim, const int64_t* shape,
                      const int64_t* x_strides, const void* x, const int64_t* y_strides, void* y,
                      void* stream) {
  clear_error();
  if (!shape || !prog) return fail(BST_ERR_INVALID, "null shape or program");
  if (dtype != BST_F32 && dtype != BST_F64) return fail(BST_ERR_UNSUPPORTED, "dtype must be float32 or float64");
  if (ndim < 1 || ndim > 3) return fail(BST_ERR_INVALID, "only 1-D, 2-D and 3-D grids are supported");
  // An empty input or output grid is a no-op (empty tensors may carry null pointers).
  for (int i = 0; i < ndim; ++i) {
    if (shape[i] < 0) return fail(BST_ERR_INVALID, "negative extent");
    if (shape[i] == 0) return BST_OK;
    if (prog->boundary == BST_BOUNDARY_VALID && prog->out_shape[i] == 0) return BST_OK;
  }
  if (!x || !y) return fail(BST_ERR_INVALID, "null device pointer");
  Canon c;
  int rc = canonicalize(prog, ndim, shape, &c);
  if (rc) return rc;
  int64_t xs_t[3], ys_t[3], oshape[3];
  for (int i = 0; i < ndim; ++i)
    oshape[i] = prog->boundary == BST_BOUNDARY_VALID ? prog->out_shape[i] : shape[i];
  if (x_strides) std::copy(x_strides, x_strides + ndim, xs_t);
  else contiguous_strides(ndim, shape, xs_t);
  if (y_strides) std::copy(y_strides, y_strides + ndim, ys_t);
  else contiguous_strides(ndim, oshape, ys_t);
  // Reject overlapping input/output (the sweep is out of place).
  const int es = elem_size(dtype);
  int64_t xlo, ylo;
  const int64_t xspan = span_elems(ndim, shape, xs_t, &xlo), yspan = span_elems(ndim, oshape, ys_t, &ylo);
  const char* xb = static_cast<const char*>(x) + xlo * es;
  const char* yb = static_cast<const char*>(y) + ylo * es;
  if (xb < yb + yspan * es && yb < xb + xspan * es) return fail(BST_ERR_INVALID, "input and output overlap");
  int64_t xs[3], ys[3];
  logical_strides(ndim, xs_t, xs);
  logical_strides(ndim, ys_t, ys);
  return launch_sweep(c, dtype, x, xs, y, ys, 0, c.no[0], static_cast<cudaStream_t>(stream));
}

int bst_stencil_sweeps(const bst_program* prog, int32_t dtype, int32_t ndim, const int64_t* shape, void* a,
                       void* b, int32_t nsteps, void* stream) {
  return bst_stencil_sweeps_fused(prog, dtype, ndim, shape, a, b, nsteps, 0, stream);
}

int bst_stencil_sweeps_fused(const bst_program* prog, int32_t dtype, int32_t ndim, const int64_t* shape, void* a,
                             void* b, int32_t nsteps, int32_t max_fused, void* stream) {
  clear_error();
  if (max_fused < 0) return fail(BST_ERR_INVALID, "negative max_fused");
  if (!shape) return fail(BST_ERR_INVALID, "null shape");
  if (!a || !b) return fail(BST_ERR_INVALID, "null device pointer");
  if (a == b) return fail(BST_ERR_INVALID, "ping-pong buffers must differ");
  if (nsteps < 0) return fail(BST_ERR_INVALID, "negative step count");
  if (dtype != BST_F32 && dtype != BST_F64) return fail(BST_ERR_UNSUPPORTED, "dtype must be float32 or float64");
  Canon c;
  int rc = canonicalize(prog, ndim, shape, &c);
  if (rc) return rc;
  if (c.boundary != BST_BOUNDARY_ZERO) return fail(BST_ERR_INVALID, "multi-step sweeps need a same-size (ZERO boundary) program");
  int64_t st_t[3], s[3];
  contiguous_strides(ndim, shape, st_t);
  logical_strides(ndim, st_t, s);
  // Fuse up to kmax sweeps per launch (temporal blocking) where a kernel exists; keep the
  // number of launches of the same parity as nsteps so the result lands in the buffer the
  // contract names.
  int kmax = tb_max_sweeps(c, dtype, a, s, b, s, max_fused > 0);
  if (max_fused > 0 && kmax > max_fused) kmax = max_fused;
  void* src = a;
  void* dst = b;
  for (int k : fuse_plan(nsteps, kmax)) {
    rc = launch_fused(c, dtype, src, s, dst, s, k, 0, c.no[0], 0, c.no[0], static_cast<cudaStream_t>(stream));
    if (rc) return rc;
    std::swap(src, dst);
  }
  return BST_OK;
}

int bst_march_item_plan(int64_t tiles, int64_t planes, int32_t rb, int32_t overhead, int64_t resident,
                        int64_t out[5]) {
  clear_error();
  if (!out) return fail(BST_ERR_INVALID, "null output");
  if (tiles < 1 || planes < 1 || rb < 1 || overhead < 0 || resident < 1)
    return fail(BST_ERR_INVALID, "tiles, planes, rb and resident must be positive, overhead non-negative");
  const ItemPlan p = choose_item_plan(tiles, planes, rb, overhead, resident);
  out[0] = p.tiles1;
  out[1] = p.chunk1;
  out[2] = p.n1;
  out[3] = p.chunk2;
  out[4] = p.n2;
  return BST_OK;
}

int bst_device_caps_query(int32_t device, bst_device_caps* out) {
  clear_error();
  if (!out) return fail(BST_ERR_INVALID, "null output");
  cudaDeviceProp p;
  BST_CUDA(cudaGetDeviceProperties(&p, device));
  std::memset(out, 0, sizeof *out);
  out->compute_capability_major = p.major;
  out->compute_capability_minor = p.minor;
  out->max_threads_per_block = p.maxThreadsPerBlock;
  out->max_shared_memory_per_block = p.sharedMemPerBlock;
  out->max_registers_per_block = p.regsPerBlock;
  out->warp_size = p.warpSize;
  out->multi_processor_count = p.multiProcessorCount;
  std::snprintf(out->name, sizeof out->name, "%s", p.name);
  std::snprintf(out->arch, sizeof out->arch, "sm_%d%d", p.major, p.minor);
  int drv = 0;
  cudaDriverGetVersion(&drv);
  out->driver_version = drv;
  fill_driver_string(out);
  return BST_OK;
}

}  // extern "C"
