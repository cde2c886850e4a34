// bst_catalog.cuh — the compiled shape catalog and the per-dtype dispatcher.
//
// A request is matched against the catalog by its canonical tap/term structure.  A
// match runs that shape's specialised kernel (TMA march for 2-D/3-D when the layout
// meets TMA's 16-byte rules, the vector line kernel for 1-D, else the direct kernel);
// anything else runs the runtime-table direct kernel.  Every path computes the same
// operations in the same order, so the choice never changes a result bit.
#pragma once
#include "bst_launch.cuh"
#include "bst_tb2d.cuh"
#include "bst_tb3d.cuh"

namespace bst {

template <class S>
bool shape_matches(const Canon& c) {
  if (c.ntaps != S::NTAPS || c.nterms != S::NTERMS) return false;
  for (int g = 0; g < c.nterms; ++g) {
    const Term& a = c.terms[g];
    const Term& b = S::tbl.terms[g];
    if (a.first != b.first || a.count != b.count || a.op != b.op) return false;
    for (int k = 0; k < a.count; ++k) {
      const Tap& u = c.taps[a.first + k];
      // The first two taps of a term commute ((u+v) == (v+u) in IEEE arithmetic).
      int kk = k;
      if (a.count >= 2 && k < 2) {
        const Tap& s0 = S::tbl.taps[b.first + k];
        if (!(u.dm == s0.dm && u.dy == s0.dy && u.dx == s0.dx)) kk = 1 - k;
      }
      const Tap& v = S::tbl.taps[b.first + kk];
      if (u.dm != v.dm || u.dy != v.dy || u.dx != v.dx) return false;
    }
  }
  return true;
}

template <typename T, int R>
constexpr int xhalo() {
  return round_up_c(R, 16 / int(sizeof(T)));
}

// Try the TMA march configuration C, else the direct kernel of its shape.
template <typename T, class C>
int run_march_or_direct(const LaunchReq& r) {
  if (march_eligible<T, C>(r)) return launch_march<T, C>(r);
  return launch_direct<T, typename C::shape>(r);
}

template <typename T, class S>
int run_line(const LaunchReq& r) {
  const Canon& c = *r.c;
  const bool aligned = reinterpret_cast<uintptr_t>(r.x) % 16 == 0 &&
                       reinterpret_cast<uintptr_t>(r.y) % 16 == 0 && r.xs[2] == 1 && r.ys[2] == 1;
  if (aligned && c.R[2] <= S::RX) {
    if (c.org[2] == 0) return launch_line<T, S, 0>(r);
    if (c.org[2] == S::RX) return launch_line<T, S, S::RX>(r);
  }
  return launch_direct<T, S>(r);
}

// Tile configurations.  A tile row is one warp of 16-byte vectors: 128 fp32 or 64 fp64
// columns.  2-D grids march along rows with one-warp CTAs (many resident per SM);
// 3-D tiles stack PY-row groups of warps and march along Z.  The defaults below were chosen
// by measurement on B200 (rows per tile, rows per thread, prefetch stages).
#ifndef BST_2D_RB
#define BST_2D_RB 4
#endif
#ifndef BST_2D_NSX
#define BST_2D_NSX 4
#endif
#ifndef BST_HEAT_TY
#define BST_HEAT_TY 64
#endif
#ifndef BST_HEAT_PY
#define BST_HEAT_PY 2
#endif
#ifndef BST_HEAT_NSX
#define BST_HEAT_NSX 2
#endif
#ifndef BST_BOX_TY
#define BST_BOX_TY 8
#endif
#ifndef BST_BOX_PY
#define BST_BOX_PY 2
#endif
#ifndef BST_BOX_NSX
#define BST_BOX_NSX 3
#endif
#ifndef BST_STAR_TY
#define BST_STAR_TY 8
#endif
#ifndef BST_STAR_PY
#define BST_STAR_PY 2
#endif
#ifndef BST_STAR_NSX
#define BST_STAR_NSX 3
#endif
// x-halo source per family (measured): shuffles for radius-1 stars, shared-memory vectors
// for boxes and the radius-4 star.
#ifndef BST_2D_HALO_LDS
#define BST_2D_HALO_LDS 0
#endif
#ifndef BST_HEAT_HALO_LDS
#define BST_HEAT_HALO_LDS 0
#endif
#ifndef BST_BOX_HALO_LDS
#define BST_BOX_HALO_LDS 1
#endif
#ifndef BST_STAR_HALO_LDS
#define BST_STAR_HALO_LDS 1
#endif
template <typename T>
constexpr int kRowCols = 32 * (16 / int(sizeof(T)));
template <typename T, class S>
using Cfg2D = MarchCfg<T, S, kRowCols<T>, 1, 1, BST_2D_RB, BST_2D_NSX, bool(BST_2D_HALO_LDS)>;
template <typename T, class S, int TY, int PY, int NSX, bool HALO = false>
using Cfg3D = MarchCfg<T, S, kRowCols<T>, TY, PY, 1, NSX, HALO>;
#ifndef BST_HEAT_RB
#define BST_HEAT_RB 1
#endif
template <typename T, class S>
using CfgHeat = MarchCfg<T, S, kRowCols<T>, BST_HEAT_TY, BST_HEAT_PY, BST_HEAT_RB, BST_HEAT_NSX, bool(BST_HEAT_HALO_LDS)>;
template <typename T, class S>
using CfgBox = Cfg3D<T, S, BST_BOX_TY, BST_BOX_PY, BST_BOX_NSX, bool(BST_BOX_HALO_LDS)>;
#ifndef BST_STAR_WINDOW
#define BST_STAR_WINDOW 1
#endif
#ifndef BST_STAR_RB
#define BST_STAR_RB 2  // two planes per stage: half the per-group bookkeeping per plane
#endif
#ifndef BST_STAR_PAIR
#define BST_STAR_PAIR 1  // fp32 points two at a time (paired add / fma instructions, exact)
#endif
#ifndef BST_STAR_MINB
#define BST_STAR_MINB 1  // CTAs per SM the register allocation must allow
#endif
#ifndef BST_STAR_CIRC
#define BST_STAR_CIRC 0  // circular register window (one group body per phase, no register moves)
#endif
#ifndef BST_STAR_INTERLEAVE
#define BST_STAR_INTERLEAVE 0  // 1: a plane's point pairs fold term by term together; 2: all planes of a group do
#endif
#ifndef BST_STAR_VXB
#define BST_STAR_VXB 16  // fp32 lane vector bytes: 8 = two x points per lane (half the window registers)
#endif
template <typename T>
constexpr int kStarVXB = sizeof(T) == 4 ? BST_STAR_VXB : 16;
template <typename T, class S>
using CfgStar = MarchCfg<T, S, 32 * kStarVXB<T> / int(sizeof(T)), BST_STAR_TY, BST_STAR_PY, BST_STAR_RB, BST_STAR_NSX,
                         bool(BST_STAR_HALO_LDS), false, bool(BST_STAR_WINDOW), BST_STAR_MINB, bool(BST_STAR_PAIR),
                         bool(BST_STAR_CIRC), BST_STAR_INTERLEAVE, kStarVXB<T>>;
// Boxes in ascending order stream: each input plane is applied to every output it touches as
// it arrives (stream_mode in bst_kernels.cuh); descending boxes keep the per-output gather.
#ifndef BST_BOXS_TY
#define BST_BOXS_TY 32
#endif
#ifndef BST_BOXS_PY
#define BST_BOXS_PY 2
#endif
#ifndef BST_BOXS_NSX
#define BST_BOXS_NSX 2
#endif
#ifndef BST_BOX_STREAM
#define BST_BOX_STREAM 1
#endif
#ifndef BST_BOXS_RB
#define BST_BOXS_RB 2
#endif
#ifndef BST_BOXS_MINB
#define BST_BOXS_MINB 2  // 2 CTAs per SM: the fused fold would otherwise take 76 registers
#endif
#ifndef BST_BOXS_PAIR
#define BST_BOXS_PAIR 0  // fp32 points two at a time (paired add / fma instructions, exact)
#endif
template <typename T, class S>
using CfgBoxS = MarchCfg<T, S, kRowCols<T>, BST_BOXS_TY, BST_BOXS_PY, BST_BOXS_RB, BST_BOXS_NSX, bool(BST_BOX_HALO_LDS),
                         bool(BST_BOX_STREAM), true, BST_BOXS_MINB, bool(BST_BOXS_PAIR)>;

// Whether BST_PROGRAM_CONTRACT changes this program's arithmetic: some multiplied term after
// the first (only those fold as fma).
inline bool contract_applies(const Canon& c) {
  if (!c.contract) return false;
  for (int g = 1; g < c.nterms; ++g)
    if (c.terms[g].op == kMul) return true;
  return false;
}

// Contracted programs: the 3-D catalog shapes have fused instantiations; others run the
// runtime-table kernel, which honours the flag too.
template <typename T>
int dispatch_contracted(const LaunchReq& r) {
  const Canon& c = *r.c;
  if (c.ndim == 3) {
    if (shape_matches<Heat3D>(c)) return run_march_or_direct<T, CfgHeat<T, Contracted<Heat3D>>>(r);
    if (shape_matches<Box<1, 7, false>>(c))
      return run_march_or_direct<T, CfgBoxS<T, Contracted<Box<1, 7, false>>>>(r);
    if (shape_matches<StarPair3D<4>>(c)) return run_march_or_direct<T, CfgStar<T, Contracted<StarPair3D<4>>>>(r);
    if (shape_matches<WStar7>(c)) return run_march_or_direct<T, CfgHeat<T, Contracted<WStar7>>>(r);
    if (shape_matches<Box<1, 7, true>>(c)) return run_march_or_direct<T, CfgBox<T, Contracted<Box<1, 7, true>>>>(r);
  }
  return launch_direct_table<T>(r);
}

template <typename T>
int dispatch_sweep(const LaunchReq& r) {
  const Canon& c = *r.c;
  if (contract_applies(c)) return dispatch_contracted<T>(r);
  if (c.ndim == 1) {
    if (shape_matches<Mean3Line>(c)) return run_line<T, Mean3Line>(r);
    if (shape_matches<Box<1, 1, false>>(c)) return run_line<T, Box<1, 1, false>>(r);
    if (shape_matches<Box<2, 1, false>>(c)) return run_line<T, Box<2, 1, false>>(r);
    if (shape_matches<Box<3, 1, false>>(c)) return run_line<T, Box<3, 1, false>>(r);
    if (shape_matches<Box<4, 1, false>>(c)) return run_line<T, Box<4, 1, false>>(r);
    if (shape_matches<Box<1, 1, true>>(c)) return run_line<T, Box<1, 1, true>>(r);
    return launch_direct_table<T>(r);
  }
  if (c.ndim == 2) {
    if (shape_matches<Jacobi2D>(c)) return run_march_or_direct<T, Cfg2D<T, Jacobi2D>>(r);
    if (shape_matches<Box<1, 5, false>>(c)) return run_march_or_direct<T, Cfg2D<T, Box<1, 5, false>>>(r);
    if (shape_matches<Box<2, 5, false>>(c)) return run_march_or_direct<T, Cfg2D<T, Box<2, 5, false>>>(r);
    if (shape_matches<Box<3, 5, false>>(c)) return run_march_or_direct<T, Cfg2D<T, Box<3, 5, false>>>(r);
    if (shape_matches<Box<4, 5, false>>(c)) return run_march_or_direct<T, Cfg2D<T, Box<4, 5, false>>>(r);
    if (shape_matches<Box<1, 5, true>>(c)) return run_march_or_direct<T, Cfg2D<T, Box<1, 5, true>>>(r);
    return launch_direct_table<T>(r);
  }
  // ndim == 3
  if (shape_matches<Heat3D>(c)) return run_march_or_direct<T, CfgHeat<T, Heat3D>>(r);
  if (shape_matches<Box<1, 7, false>>(c)) return run_march_or_direct<T, CfgBoxS<T, Box<1, 7, false>>>(r);
  if (shape_matches<StarPair3D<4>>(c)) return run_march_or_direct<T, CfgStar<T, StarPair3D<4>>>(r);
  if (shape_matches<WStar7>(c)) return run_march_or_direct<T, CfgHeat<T, WStar7>>(r);
  if (shape_matches<Box<2, 7, false>>(c))
    return run_march_or_direct<T, Cfg3D<T, Box<2, 7, false>, 4, 1, 2, bool(BST_BOX_HALO_LDS)>>(r);
  if (shape_matches<Box<1, 7, true>>(c)) return run_march_or_direct<T, CfgBox<T, Box<1, 7, true>>>(r);
  return launch_direct_table<T>(r);
}

// ---- temporally blocked multi-sweep (2-D window shapes) -------------------------------
template <typename T, class C>
bool tb_eligible(const LaunchReq& r) {
  const Canon& c = *r.c;
  constexpr int E = sizeof(T);
  if (c.ndim != 2 || c.boundary != BST_BOUNDARY_ZERO || c.org[2] != 0) return false;
  if (c.no[0] >= (int64_t(1) << 30)) return false;
  if (reinterpret_cast<uintptr_t>(r.x) % 16 != 0 || r.xs[2] != 1 || (r.xs[0] * E) % 16 != 0) return false;
  if (c.n[0] >= (int64_t(1) << 31) || c.n[2] >= (int64_t(1) << 31)) return false;
  if (c.R[0] > C::R || c.R[2] > C::RX) return false;
  return true;
}

template <typename T, class C>
int launch_tb2d(const LaunchReq& r) {
  if (int rc = peer_unsupported(r, "the temporally blocked kernel")) return rc;
  const Canon& c = *r.c;
  constexpr int E = sizeof(T);
  const long long nm = r.m_hi - r.m_lo;
  if (nm <= 0) return BST_OK;
  CUtensorMap map;
  const cuuint64_t dims[3] = {cuuint64_t(c.n[2]), 1, cuuint64_t(c.n[0])};
  const cuuint64_t strides[2] = {cuuint64_t(r.xs[0] * E), cuuint64_t(r.xs[0] * E)};
  const cuuint32_t box[3] = {cuuint32_t(C::TXL), 1, cuuint32_t(C::RB)};
  const cuuint32_t estr[3] = {1, 1, 1};
  auto enc = tensor_map_encoder();
  if (!enc) return fail(BST_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  CUresult cr = enc(&map, tma_dtype<T>(), 3, const_cast<void*>(r.x), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return fail(BST_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(int(cr)) + ")");
  auto kern = march_tb2d_kernel<T, C>;
  TbArgs a{};
  a.g = make_grid(r);
  a.tiles_x = int((c.no[2] + C::TXO - 1) / C::TXO);
  const int occ = occupancy(reinterpret_cast<const void*>(kern), C::THREADS, C::SMEM);
  if (occ <= 0) return fail(BST_ERR_CUDA, "temporally blocked kernel does not fit on an SM");
  const long long resident = (long long)occ * sm_count();
  long long nchunks = 1;
  choose_chunks(a.tiles_x, nm, 1, 2 * C::K * C::R + C::RB + 8, resident, &a.chunk, &nchunks);
  a.n_items = (long long)a.tiles_x * nchunks;
  a.err = device_error_word();
  if (!a.err) return fail(BST_ERR_CUDA, "device error word unavailable");
  a.vec_store = (reinterpret_cast<uintptr_t>(r.y) % 16 == 0 && r.ys[2] == 1 && (r.ys[0] * E) % 16 == 0) ? 1 : 0;
  const int64_t big = int64_t(1) << 30;
  const int64_t lo = r.row_hi < r.row_lo ? 0 : r.row_lo, hi = r.row_hi < r.row_lo ? c.no[0] : r.row_hi;
  a.row_lo = int(lo < -big ? -big : lo);
  a.row_hi = int(hi > big ? big : hi);
  const long long grid = a.n_items < resident ? a.n_items : resident;
  kern<<<unsigned(grid), C::THREADS, C::SMEM, r.st>>>(map, static_cast<T*>(r.y), a,
                                                      make_coefs<T, C::shape::NTERMS>(c));
  BST_CUDA(cudaGetLastError());
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return BST_OK;
}

// ---- temporally blocked multi-sweep (3-D seven-point shapes) ----------------------------
template <typename T, class C>
bool tb3_eligible(const LaunchReq& r) {
  const Canon& c = *r.c;
  constexpr int E = sizeof(T);
  if (c.ndim != 3 || c.boundary != BST_BOUNDARY_ZERO) return false;
  if (c.org[1] != 0 || c.org[2] != 0) return false;
  if (reinterpret_cast<uintptr_t>(r.x) % 16 != 0 || r.xs[2] != 1 || (r.xs[1] * E) % 16 != 0 ||
      (r.xs[0] * E) % 16 != 0)
    return false;
  for (int i = 0; i < 3; ++i)
    if (c.n[i] >= (int64_t(1) << 30) || c.no[i] >= (int64_t(1) << 30)) return false;
  if (c.R[0] > 1 || c.R[1] > 1 || c.R[2] > 1) return false;
  return true;
}

template <typename T, class C>
int launch_tb3d(const LaunchReq& r) {
  if (int rc = peer_unsupported(r, "the temporally blocked kernel")) return rc;
  const Canon& c = *r.c;
  constexpr int E = sizeof(T);
  const long long nm = r.m_hi - r.m_lo;
  if (nm <= 0) return BST_OK;
  CUtensorMap map;
  const cuuint64_t dims[3] = {cuuint64_t(c.n[2]), cuuint64_t(c.n[1]), cuuint64_t(c.n[0])};
  const cuuint64_t strides[2] = {cuuint64_t(r.xs[1] * E), cuuint64_t(r.xs[0] * E)};
  const cuuint32_t box[3] = {cuuint32_t(C::TXL), cuuint32_t(C::TYL), 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  auto enc = tensor_map_encoder();
  if (!enc) return fail(BST_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  CUresult cr = enc(&map, tma_dtype<T>(), 3, const_cast<void*>(r.x), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, march_l2_promotion(),
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return fail(BST_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(int(cr)) + ")");
  auto kern = march_tb3d_kernel<T, C>;
  Tb3Args a{};
  a.g = make_grid(r);
  a.tiles_x = int((c.no[2] + C::TXO - 1) / C::TXO);
  a.tiles_y = int((c.no[1] + C::TYO - 1) / C::TYO);
  const int occ = occupancy(reinterpret_cast<const void*>(kern), C::THREADS, C::SMEM);
  if (occ <= 0) return fail(BST_ERR_CUDA, "3-D temporally blocked kernel does not fit on an SM");
  const long long resident = (long long)occ * sm_count();
  const long long tiles = (long long)a.tiles_x * a.tiles_y;
  long long nchunks = 1;
  choose_chunks(tiles, nm, 1, 2 * C::K * C::R + 8, resident, &a.chunk, &nchunks);
  a.n_items = tiles * nchunks;
  a.err = device_error_word();
  if (!a.err) return fail(BST_ERR_CUDA, "device error word unavailable");
  a.vec_store = (reinterpret_cast<uintptr_t>(r.y) % 16 == 0 && r.ys[2] == 1 && (r.ys[1] * E) % 16 == 0 &&
                 (r.ys[0] * E) % 16 == 0)
                    ? 1
                    : 0;
  const int64_t big = int64_t(1) << 30;
  const int64_t lo = r.row_hi < r.row_lo ? 0 : r.row_lo, hi = r.row_hi < r.row_lo ? c.no[0] : r.row_hi;
  a.row_lo = int(lo < -big ? -big : lo);
  a.row_hi = int(hi > big ? big : hi);
  const long long grid = a.n_items < resident ? a.n_items : resident;
  kern<<<unsigned(grid), C::THREADS, C::SMEM, r.st>>>(map, static_cast<T*>(r.y), a,
                                                      make_coefs<T, C::shape::NTERMS>(c));
  BST_CUDA(cudaGetLastError());
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return BST_OK;
}

#ifndef BST_TB3_ROWS
#define BST_TB3_ROWS 16  // tile rows = warps per CTA (16: 538 Gpts/s, 24: 449, 32: 504 on heat-7 512^3, 2 sweeps)
#endif
#ifndef BST_TB3_NSX
#define BST_TB3_NSX 6  // prefetch depth (planes); measured 489 -> 504 Gpts/s from 2 to 6 (heat-7 512^3)
#endif
#ifndef BST_TB3_KMAX
#define BST_TB3_KMAX 2  // sweeps fused per 3-D launch at most (fp32 seven-point shapes)
#endif
template <typename T, class S, int K>
using CfgTb3 = Tb3Cfg<T, S, K, BST_TB3_ROWS, BST_TB3_NSX>;

#ifndef BST_TB_RB
#define BST_TB_RB 6  // a multiple of the window (2R+1 = 3): one group body, no phase dispatch
#endif
#ifndef BST_TB_NSX
#define BST_TB_NSX 1
#endif
template <typename T, class S, int K>
using CfgTb = TbCfg<T, S, K, BST_TB_RB, BST_TB_NSX>;

// Sweeps fused per launch at most (fp32: 2..5; fp64 keeps 3, the most its x-halo allows).
#ifndef BST_TB_KMAX_F32
#define BST_TB_KMAX_F32 4
#endif

// Largest number of sweeps one temporally blocked launch can fuse for this request (1 = none).
// capability = false: only where fusing is the faster choice — the 3-D kernel (bit-identical,
// but measured slower than single sweeps of the 94 %-of-HBM march kernel) runs only when a
// caller asks for fused sweeps (bst_stencil_sweeps_fused, or slabs with deeper ghosts).
template <typename T>
int tb_max_sweeps(const LaunchReq& r, bool capability) {
  if (shape_matches<Jacobi2D>(*r.c) && tb_eligible<T, CfgTb<T, Jacobi2D, 2>>(r))
    return sizeof(T) == 4 ? BST_TB_KMAX_F32 : 3;
  if constexpr (sizeof(T) == 4) {
    if (capability && !contract_applies(*r.c) && shape_matches<Heat3D>(*r.c) &&
        tb3_eligible<T, CfgTb3<T, Heat3D, 2>>(r))
      return BST_TB3_KMAX;
  }
  return 1;
}

// k sweeps (2 <= k <= tb_max_sweeps) in one launch.
template <typename T>
int dispatch_tb(const LaunchReq& r, int k) {
  if (shape_matches<Jacobi2D>(*r.c)) {
    switch (k) {
      case 2: return launch_tb2d<T, CfgTb<T, Jacobi2D, 2>>(r);
      case 3: return launch_tb2d<T, CfgTb<T, Jacobi2D, 3>>(r);
      case 4:
        if constexpr (sizeof(T) == 4) return launch_tb2d<T, CfgTb<T, Jacobi2D, 4>>(r);
        break;
      case 5:
        if constexpr (sizeof(T) == 4) return launch_tb2d<T, CfgTb<T, Jacobi2D, 5>>(r);
        break;
      default:
        break;
    }
  }
  if constexpr (sizeof(T) == 4) {
    if (!contract_applies(*r.c) && shape_matches<Heat3D>(*r.c)) {
      switch (k) {
        case 2: return launch_tb3d<T, CfgTb3<T, Heat3D, 2>>(r);
#if BST_TB3_KMAX >= 3
        case 3: return launch_tb3d<T, CfgTb3<T, Heat3D, 3>>(r);
#endif
#if BST_TB3_KMAX >= 4
        case 4: return launch_tb3d<T, CfgTb3<T, Heat3D, 4>>(r);
#endif
        default: break;
      }
    }
  }
  return fail(BST_ERR_UNSUPPORTED, "no temporally blocked kernel for this request");
}

}  // namespace bst
