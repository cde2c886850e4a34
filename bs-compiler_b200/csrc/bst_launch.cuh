// bst_launch.cuh — typed launchers for one catalog shape (included by the per-dtype
// instantiation units).
#pragma once
#include <cudaTypedefs.h>

#include <algorithm>
#include <climits>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "bst_internal.h"
#include "bst_kernels.cuh"
#include "bst_plan.h"

namespace bst {

struct LaunchReq {
  const Canon* c;
  const void* x;
  int64_t xs[3];
  void* y;
  int64_t ys[3];
  int64_t m_lo, m_hi;
  cudaStream_t st;
  // Temporally blocked launches: rows (output coordinates) whose intermediate levels are
  // computed; outside it they are ghost cells.  Default: the grid's own rows.
  int64_t row_lo = 0, row_hi = -1;
  // Slab boundary launches: also store into a neighbouring GPU's ghost planes (TMA march only).
  const PeerStore* peer = nullptr;
  // A second range of output planes [m2_lo, m2_hi) in the same request (slab boundary rows):
  // one launch on the TMA march kernel, two launches elsewhere.
  int64_t m2_lo = 0, m2_hi = 0;
};

inline bool two_ranges(const LaunchReq& r) { return r.m2_hi > r.m2_lo; }

// Runs a two-range request as two launches of `launch`.
template <class F>
int each_range(const LaunchReq& r, F&& launch) {
  LaunchReq a = r;
  a.m2_lo = a.m2_hi = 0;
  if (int rc = launch(a)) return rc;
  LaunchReq b = a;
  b.m_lo = r.m2_lo;
  b.m_hi = r.m2_hi;
  return launch(b);
}

inline int peer_unsupported(const LaunchReq& r, const char* kernel) {
  if (!r.peer) return BST_OK;
  return fail(BST_ERR_UNSUPPORTED, std::string("peer-memory boundary stores need the TMA march kernel; this request "
                                               "runs ") + kernel);
}

template <typename T, int N>
Coefs<T, N> make_coefs(const Canon& c) {
  Coefs<T, N> k{};
  for (int g = 0; g < c.nterms && g < N; ++g) {
    k.scale[g] = T(c.scale[g]);
    // div_by's reciprocal: fp32 divisors with |d| in [2^-60, 2^60] (0 = plain IEEE division)
    const float d = float(c.scale[g]);
    const float ad = d < 0.f ? -d : d;
    if (sizeof(T) == 4 && c.terms[g].op == kDiv && ad >= 0x1p-60f && ad <= 0x1p60f) k.rcp[g] = T(1.0f / d);
  }
  k.init_zero = c.init_zero;
  k.negzero = T(-0.0);
  return k;
}

inline GridDesc make_grid(const LaunchReq& r) {
  GridDesc g{};
  for (int i = 0; i < 3; ++i) {
    g.n[i] = r.c->n[i];
    g.s[i] = r.xs[i];
    g.no[i] = r.c->no[i];
    g.so[i] = r.ys[i];
    g.org[i] = r.c->org[i];
  }
  g.m_lo = r.m_lo;
  g.m_hi = r.m_hi;
  return g;
}

int sm_count();
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// ---- direct ---------------------------------------------------------------------
template <typename T, class S>
int launch_direct(const LaunchReq& r) {
  if (two_ranges(r)) return each_range(r, [](const LaunchReq& q) { return launch_direct<T, S>(q); });
  if (int rc = peer_unsupported(r, "the direct kernel")) return rc;
  const GridDesc g = make_grid(r);
  const long long total = (r.m_hi - r.m_lo) * g.no[1] * g.no[2];
  if (total <= 0) return BST_OK;
  long long blocks = (total + 255) / 256;
  const long long cap = (long long)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  direct_kernel<T, S><<<unsigned(blocks), 256, 0, r.st>>>(static_cast<const T*>(r.x),
                                                         static_cast<T*>(r.y), g, make_coefs<T, S::NTERMS>(*r.c));
  BST_CUDA(cudaGetLastError());
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return BST_OK;
}

template <typename T>
int launch_direct_table(const LaunchReq& r) {
  if (two_ranges(r)) return each_range(r, [](const LaunchReq& q) { return launch_direct_table<T>(q); });
  if (int rc = peer_unsupported(r, "the runtime-table kernel")) return rc;
  const Canon& c = *r.c;
  const GridDesc g = make_grid(r);
  const long long total = (r.m_hi - r.m_lo) * g.no[1] * g.no[2];
  if (total <= 0) return BST_OK;
  // The table and scales travel in one device buffer.
  struct Blob {
    TableProgram p;
    T scale[kMaxTerms];
  };
  std::vector<unsigned char> host(sizeof(Blob), 0);
  Blob* h = reinterpret_cast<Blob*>(host.data());
  h->p.ntaps = c.ntaps;
  h->p.nterms = c.nterms;
  h->p.init_zero = c.init_zero;
  for (int i = 0; i < c.ntaps; ++i) {
    h->p.tap[i][0] = short(c.taps[i].dm);
    h->p.tap[i][1] = short(c.taps[i].dy);
    h->p.tap[i][2] = short(c.taps[i].dx);
  }
  for (int i = 0; i < c.nterms; ++i) {
    h->p.term_first[i] = short(c.terms[i].first);
    h->p.term_count[i] = short(c.terms[i].count);
    h->p.term_op[i] = (unsigned char)c.terms[i].op;
    h->scale[i] = T(c.scale[i]);
  }
  long long blocks = (total + 255) / 256;
  const long long cap = (long long)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  const Blob* cached = static_cast<const Blob*>(cached_device_table(host.data(), host.size()));
  if (cached) {
    direct_table_kernel<T><<<unsigned(blocks), 256, 0, r.st>>>(
        static_cast<const T*>(r.x), static_cast<T*>(r.y), g, &cached->p,
        TableCoefs<T>{cached->scale, c.init_zero, c.contract});
    BST_CUDA(cudaGetLastError());
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return BST_OK;
  }
  // Cache full: a stream-ordered buffer for this call only.
  void* d = nullptr;
  BST_CUDA(cudaMallocAsync(&d, sizeof(Blob), r.st));
  cudaError_t e = cudaMemcpyAsync(d, h, sizeof(Blob), cudaMemcpyHostToDevice, r.st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(r.st);  // host staging buffer dies on return
  if (e != cudaSuccess) {
    cudaFreeAsync(d, r.st);
    return cuda_fail(e, "upload of the stencil table");
  }
  const Blob* db = static_cast<const Blob*>(d);
  direct_table_kernel<T><<<unsigned(blocks), 256, 0, r.st>>>(
      static_cast<const T*>(r.x), static_cast<T*>(r.y), g, &db->p, TableCoefs<T>{db->scale, c.init_zero, c.contract});
  e = cudaGetLastError();
  cudaFreeAsync(d, r.st);
  if (e != cudaSuccess) return cuda_fail(e, "direct_table_kernel launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return BST_OK;
}

// ---- 1-D line ---------------------------------------------------------------------
int occupancy(const void* fn, int threads, int smem);  // resident CTAs per SM (cached)

template <typename T, class S, int ORG>
int launch_line(const LaunchReq& r) {
  if (two_ranges(r)) return each_range(r, [](const LaunchReq& q) { return launch_line<T, S, ORG>(q); });
  if (int rc = peer_unsupported(r, "the 1-D line kernel")) return rc;
  constexpr int V = Vec16<T>::N;
  LineArgs a{r.c->n[2], r.c->no[2]};
  const long long nvec = (a.n_out + V - 1) / V;
  if (nvec <= 0) return BST_OK;
  const long long per_block = 256LL * LINE_U;  // vectors one block covers per chunk round
  long long blocks = (nvec + per_block - 1) / per_block;
  // One wave of resident blocks; later chunks go round the grid.
  const int occ = occupancy(reinterpret_cast<const void*>(line_kernel<T, S, ORG>), 256, 0);
  const long long cap = (long long)sm_count() * (occ > 0 ? occ : 1);
  if (blocks > cap) blocks = cap;
  line_kernel<T, S, ORG><<<unsigned(blocks), 256, 0, r.st>>>(
      static_cast<const T*>(r.x), static_cast<T*>(r.y), a, make_coefs<T, S::NTERMS>(*r.c));
  BST_CUDA(cudaGetLastError());
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return BST_OK;
}

// ---- TMA march ----------------------------------------------------------------------
template <typename T>
constexpr CUtensorMapDataType tma_dtype() {
  return sizeof(T) == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT64;
}

// L2 sector promotion of the march kernel's plane loads (BST_TMA_PROMO: 0 none, 1 64 B,
// 2 128 B, 3 256 B).
#ifndef BST_TMA_PROMO
#define BST_TMA_PROMO 3
#endif
inline CUtensorMapL2promotion march_l2_promotion() {
  switch (BST_TMA_PROMO) {
    case 0: return CU_TENSOR_MAP_L2_PROMOTION_NONE;
    case 1: return CU_TENSOR_MAP_L2_PROMOTION_L2_64B;
    case 2: return CU_TENSOR_MAP_L2_PROMOTION_L2_128B;
    default: return CU_TENSOR_MAP_L2_PROMOTION_L2_256B;
  }
}

// Whether the request meets TMA's rules for this configuration.
template <typename T, class C>
bool march_eligible(const LaunchReq& r) {
  const Canon& c = *r.c;
  constexpr int E = sizeof(T);
  if (reinterpret_cast<uintptr_t>(r.x) % 16 != 0) return false;
  if (r.xs[2] != 1) return false;
  if ((r.xs[1] * E) % 16 != 0 || (r.xs[0] * E) % 16 != 0) return false;
  if (r.xs[0] <= 0 || r.xs[1] <= 0) return false;
  for (int i = 0; i < 3; ++i)
    if (c.n[i] >= (int64_t(1) << 31) || c.no[i] >= (int64_t(1) << 31)) return false;
  // The tile's first loaded column and every thread's vector sit on 16-byte boundaries.
  if (((c.org[2] - C::XC) % C::VX + C::VX) % C::VX != 0) return false;
  if (c.R[0] > C::RM || c.R[1] > C::RY || c.R[2] > C::RX) return false;
  return true;
}

struct OccKey {
  const void* fn;
  int smem;
  bool operator==(const OccKey& o) const { return fn == o.fn && smem == o.smem; }
};
struct OccHash {
  size_t operator()(const OccKey& k) const { return std::hash<const void*>()(k.fn) ^ size_t(k.smem); }
};
int occupancy(const void* fn, int threads, int smem);

template <typename T, class C>
int launch_march(const LaunchReq& r) {
  // Two ranges in one launch: equal lengths, the second above the first, no peer stores.
  const bool pair = two_ranges(r);
  if (pair && (r.peer || r.m_hi - r.m_lo != r.m2_hi - r.m2_lo || r.m2_lo < r.m_hi))
    return each_range(r, [](const LaunchReq& q) { return launch_march<T, C>(q); });
  const Canon& c = *r.c;
  constexpr int E = sizeof(T);
  const long long nm = (r.m_hi - r.m_lo) * (pair ? 2 : 1);  // a pair: both ranges, stacked
  if (nm <= 0) return BST_OK;
  CUtensorMap map;
  const cuuint64_t dims[3] = {cuuint64_t(c.n[2]), cuuint64_t(c.n[1]), cuuint64_t(c.n[0])};
  // Stride of the unit Y axis of a 2-D grid is irrelevant but must be legal.
  const int64_t sy = c.n[1] == 1 ? r.xs[0] : r.xs[1];
  const cuuint64_t strides[2] = {cuuint64_t(sy * E), cuuint64_t(r.xs[0] * E)};
  const cuuint32_t box[3] = {cuuint32_t(C::TXL), cuuint32_t(C::TYL), cuuint32_t(C::RB)};
  const cuuint32_t estr[3] = {1, 1, 1};
  auto enc = tensor_map_encoder();
  if (!enc) return fail(BST_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  CUresult cr = enc(&map, tma_dtype<T>(), 3, const_cast<void*>(r.x), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                    march_l2_promotion(), CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return fail(BST_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(int(cr)) + ")");

  auto kern = r.peer ? march_tma_kernel<T, C, true> : march_tma_kernel<T, C, false>;

  MarchArgs a{};
  a.g = make_grid(r);
  a.gap_at = LLONG_MAX;
  if (pair) {  // planes [m_lo, m_lo + 2L) of the launch: the upper half is [m2_lo, m2_hi)
    const long long len = r.m_hi - r.m_lo;
    a.g.m_hi = r.m_lo + 2 * len;
    a.gap_at = r.m_lo + len;
    a.gap = r.m2_lo - (r.m_lo + len);
  }
  a.tiles_x = int((c.no[2] + C::TX - 1) / C::TX);
  a.tiles_y = int((c.no[1] + C::TY - 1) / C::TY);
  const int occ = occupancy(reinterpret_cast<const void*>(kern), C::THREADS, C::SMEM);
  if (occ <= 0) return fail(BST_ERR_CUDA, "march kernel does not fit on an SM");
  const long long resident = (long long)occ * sm_count();
  const long long tiles = (long long)a.tiles_x * a.tiles_y;
  a.nm = nm;
  long long grid = 0;
  // Peer-store sweeps count their boundary items, so they use the item schedule; a pair of
  // ranges is one chunk per range and tile column.
  switch (r.peer || pair ? Schedule::kItems : march_schedule()) {
    case Schedule::kBalanced:
      a.balanced = 1;
      a.work = tiles * nm;
      grid = a.work < resident ? a.work : resident;
      break;
    case Schedule::kLockstep:
      if (tiles <= resident) {  // one wave: every tile column in floor(resident / tiles) chunks
        long long s = resident / tiles;
        if (s > nm) s = nm;
        a.chunk = (nm + s - 1) / s;
        a.work = tiles * ((nm + a.chunk - 1) / a.chunk);
        grid = a.work;
        break;
      }
      [[fallthrough]];
    default: {
      const int overhead = 2 * C::RM + 2 * C::RB + 8;
      if (pair) {
        a.chunk = r.m_hi - r.m_lo;
        a.work = tiles * 2;
      } else if (r.peer) {  // one band: the peer logic counts items per chunk row
        int chunk = 0;
        long long nchunks = 1;
        choose_chunks(tiles, nm, C::RB, overhead, resident, &chunk, &nchunks);
        a.chunk = chunk;
        a.work = tiles * nchunks;
      } else {
        const ItemPlan p = choose_item_plan(tiles, nm, C::RB, overhead, resident);
        a.chunk = p.chunk1;
        a.chunk2 = p.chunk2;
        a.tiles1 = p.tiles1;
        a.work1 = p.tiles1 * p.n1;
        a.work = a.work1 + (tiles - p.tiles1) * p.n2;
      }
      grid = a.work < resident ? a.work : resident;
    }
  }
  if (a.tiles1 == 0) {  // one band
    a.tiles1 = tiles;
    a.work1 = a.work;
    a.chunk2 = a.chunk;
  }
  a.err = device_error_word();
  if (!a.err) return fail(BST_ERR_CUDA, "device error word unavailable");
  a.vec_store = (reinterpret_cast<uintptr_t>(r.y) % 16 == 0 && r.ys[2] == 1 && (r.ys[1] * E) % 16 == 0 &&
                 (r.ys[0] * E) % 16 == 0)
                    ? 1
                    : 0;
  if (r.peer) {
    a.peer = *r.peer;
    if (a.peer.delta_lo % 16 != 0 || a.peer.delta_hi % 16 != 0) a.vec_store = 0;  // remote rows aligned too
    // The lower and upper boundary chunks run first (their planes reach the neighbours early,
    // and the neighbours' next launch reads them without waiting).  Count the items storing to
    // each side.
    const long long nchunks = a.work / tiles;
    long long lo = 0, hi = 0;
    for (long long ci = 0; ci < nchunks; ++ci) {
      const long long b = r.m_lo + ci * a.chunk, e = b + a.chunk < r.m_hi ? b + a.chunk : r.m_hi;
      if (b < (long long)a.peer.lo_end) ++lo;
      if (e > (long long)a.peer.hi_begin) ++hi;
    }
    a.peer.items_lo = lo * tiles;
    a.peer.items_hi = hi * tiles;
    if (a.peer.flag_lo && a.peer.items_lo == 0) return fail(BST_ERR_INVALID, "no item stores to the lower neighbour");
    if (a.peer.flag_hi && a.peer.items_hi == 0) return fail(BST_ERR_INVALID, "no item stores to the upper neighbour");
  }
  dim3 block(C::THREADS);
  kern<<<unsigned(grid), block, C::SMEM, r.st>>>(map, static_cast<T*>(r.y), a,
                                                  make_coefs<T, C::shape::NTERMS>(c));
  BST_CUDA(cudaGetLastError());
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return BST_OK;
}

}  // namespace bst
