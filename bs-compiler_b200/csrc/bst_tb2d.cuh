// bst_tb2d.cuh — temporally blocked 2-D march: K sweeps of a 2-D window stencil per launch.
//
// A multi-sweep run of a 2-D stencil reads and writes the whole grid once per sweep.  This
// kernel keeps K successive sweeps in flight inside one pass over the grid, so HBM is read
// and written once per K sweeps.  The arithmetic is unchanged (every level performs the
// same separately rounded operations in the same order), so the result is bit-identical
// to K single sweeps.
//
//  * Rows (the marching axis): one warp marches down a column strip.  Level 0 is the input
//    (a register window of 2R+1 row vectors fed by TMA, as in march_tma_kernel); level l
//    computes row i - l*R from level l-1's window and pushes it into its own window.  Level
//    K is stored.  An item of output rows [mb, me) reads input rows [mb-K*R, me+K*R): the
//    K*R halo rows on each side are recomputed by the neighbouring items.
//  * Columns: the warp's 32 lanes own 128 (fp32) / 64 (fp64) columns, but only the central
//    30 lanes' columns are stored.  Level l's values near the warp edges have no neighbour
//    lane to take their x-halo from; the error moves inward by R columns per level and never
//    reaches the stored columns while (K-1)*R <= one lane's width.
//  * Dirichlet-0: level values outside the grid (rows or columns) are ghost cells of the
//    next level and are forced to zero, exactly as a sweep reads zeros outside the grid.
#pragma once
#include "bst_kernels.cuh"

namespace bst {

template <typename T, class S, int K_, int RB_, int NSX_>
struct TbCfg {
  using shape = S;
  static constexpr int K = K_;
  static constexpr int VX = 16 / int(sizeof(T));
  static constexpr int R = S::RM;                       // row radius
  static constexpr int RX = S::RX;                      // column radius
  static constexpr int HL = 1;                          // overlap lanes at each warp edge
  static constexpr int TXO = (32 - 2 * HL) * VX;        // stored columns per tile
  static constexpr int HXI = ((RX + VX - 1) / VX) * VX; // loaded columns beyond the warp
  static constexpr int TXL = 32 * VX + 2 * HXI;         // loaded columns per row
  static constexpr int RB = RB_;                        // rows per stage
  static constexpr int PLANE = TXL;
  static constexpr int STAGE_BYTES = round_up_c(PLANE * RB * int(sizeof(T)), 128);
  static constexpr int STAGE = STAGE_BYTES / int(sizeof(T));
  static constexpr int B = (R + RB - 1) / RB;            // earlier stages a group still reads
  // A group waits for its own stage before the barrier and refills after it, so that
  // stage must have been issued by the previous group: NS >= B + 2.
  static constexpr int NS = (B + 2 > B + 1 + NSX_) ? B + 2 : B + 1 + NSX_;
  static constexpr int SMEM = NS * STAGE_BYTES + 128;
  static constexpr int SEGW = VX + 2 * HXI;
  static constexpr int THREADS = 32;
  static_assert(window_mode<S>() && S::RY == 0, "2-D window shapes only");
  static_assert((K - 1) * RX <= HL * VX, "stored columns stay valid through K levels");
  static_assert(TXL <= 256 && RB <= 256, "TMA box extent");
  static_assert(NS >= B + 2, "every stage is issued before a group waits on it");
};

struct TbArgs {
  GridDesc g;
  int tiles_x, chunk;
  long long n_items;
  unsigned* err;
  int vec_store;
  int row_lo, row_hi;  // output-coordinate rows whose level values are computed; others are ghosts (0)
};

// Level windows are circular: a level that has been pushed c times keeps its logical row k
// (0 = oldest of the 2R+1) in physical slot (c + k) mod W, so a push writes one slot and no
// register moves.  Every push count is a compile-time function of the step's phase.
template <typename T, class C, int V, int PH>  // PH = pushes of the window so far, mod W
struct TbFetch {
  const T (&w)[2 * C::R + 1][C::VX];
  const T (&seg)[C::SEGW];
  template <int dm, int dy, int dx>
  __device__ __forceinline__ T get() const {
    if constexpr (dm != 0) return w[(PH + C::R + dm) % (2 * C::R + 1)][V];
    else return seg[C::HXI + V + dx];
  }
};

// x-halo of one level's centre row: own vector plus neighbour lanes' elements; at level 0
// the warp's edge lanes read the loaded halo columns from shared memory.
template <typename T, class C, bool LEVEL0>
__device__ __forceinline__ void tb_segment(T (&seg)[C::SEGW], const T (&own)[C::VX], const T* row, int lane) {
#pragma unroll
  for (int e = 0; e < C::VX; ++e) seg[C::HXI + e] = own[e];
#pragma unroll
  for (int e = -C::RX; e < 0; ++e) {
    const int d = (-e + C::VX - 1) / C::VX;
    T v = __shfl_up_sync(0xffffffffu, own[e + d * C::VX], d);
    if (LEVEL0 && lane < d) v = row[e];
    seg[C::HXI + e] = v;
  }
#pragma unroll
  for (int e = C::VX; e < C::VX + C::RX; ++e) {
    const int d = e / C::VX;
    T v = __shfl_down_sync(0xffffffffu, own[e - d * C::VX], d);
    if (LEVEL0 && lane >= 32 - d) v = row[e];
    seg[C::HXI + e] = v;
  }
}

template <typename T, class C, int PH, int... Vs>
__device__ __forceinline__ void tb_eval(const T (&w)[2 * C::R + 1][C::VX], const T (&seg)[C::SEGW],
                                        const Coefs<T, C::shape::NTERMS>& c, T (&res)[C::VX],
                                        std::integer_sequence<int, Vs...>) {
  ((res[Vs] = eval_shape<typename C::shape, T>(TbFetch<T, C, Vs, PH>{w, seg}, c)), ...);
}

// Per-item constants of a tile (rows in output coordinates, 32-bit).
struct TbTile {
  int L0;            // row of the item's first input row
  int mb, me;        // stored output rows
  int row_lo, row_hi;  // level values outside [row_lo, row_hi) are ghost cells (0)
  bool rows_safe;    // every row this item touches lies inside [row_lo, row_hi)
  int cmask;         // bit e: this lane's column e lies inside the grid
  bool edge;         // the warp's columns reach outside the grid
  bool store_lane;   // this lane's columns are stored
  int c0;            // first column of this lane
};

// Levels L..K for input row i.  Q0 = (pushes of level 0 so far, this step's included) mod W;
// window l >= 1 has then been pushed Q0 - 2R times (mod W) when it is read, and this step's
// row of level l goes to slot (Q0 - 1 - 2R) mod W.  `dst` = the store address of level K's
// row for this lane.
template <typename T, class C, int L, int Q0>
__device__ __forceinline__ void tb_levels(T (&win)[C::K][2 * C::R + 1][C::VX], const T* edge_row, int lane,
                                          const TbTile& t, int i, const Coefs<T, C::shape::NTERMS>& coef,
                                          const GridDesc& g, T* dst, int vec_store) {
  if constexpr (L <= C::K) {
    constexpr int W = 2 * C::R + 1;
    constexpr int PH = L == 1 ? Q0 % W : ((Q0 - 2 * C::R) % W + W) % W;  // pushes of window L-1, mod W
    T seg[C::SEGW];
    tb_segment<T, C, L == 1>(seg, win[L - 1][(PH + C::R) % W], edge_row, lane);
    T res[C::VX];
    tb_eval<T, C, PH>(win[L - 1], seg, coef, res, std::make_integer_sequence<int, C::VX>{});
    const int row = i - L * C::R;  // row this level computed
    if constexpr (L < C::K) {
      // Ghost cells of level L+1 are zero: rows outside [row_lo, row_hi) (warp-uniform, only
      // checked in items that reach them) and columns outside the grid (edge tiles only).
      if (!t.rows_safe && (row < t.row_lo || row >= t.row_hi)) {
#pragma unroll
        for (int e = 0; e < C::VX; ++e) res[e] = T(0);
      } else if (t.edge) {
#pragma unroll
        for (int e = 0; e < C::VX; ++e)
          if (!((t.cmask >> e) & 1)) res[e] = T(0);
      }
      constexpr int SLOT = ((Q0 - 1 - 2 * C::R) % W + W) % W;
#pragma unroll
      for (int e = 0; e < C::VX; ++e) win[L][SLOT][e] = res[e];
      tb_levels<T, C, L + 1, Q0>(win, edge_row, lane, t, i, coef, g, dst, vec_store);
    } else {
      if (row >= t.mb && row < t.me && t.store_lane) {
        if (vec_store && t.c0 + C::VX <= g.no[2]) {
          using VT = typename Vec16<T>::type;
          VT q;
          T* e = reinterpret_cast<T*>(&q);
#pragma unroll
          for (int v = 0; v < C::VX; ++v) e[v] = res[v];
          *reinterpret_cast<VT*>(dst) = q;
        } else {
#pragma unroll
          for (int v = 0; v < C::VX; ++v)
            if (t.c0 + v < g.no[2]) dst[(long long)v * g.so[2]] = res[v];
        }
      }
    }
  }
}

// Step P of a group whose first input row has phase GP = (grp * RB) mod W.  FIRST: the item's
// first group (level 0's window still filling); FULL: every step of the group is in range.
template <typename T, class C, int GP, bool FIRST, bool FULL, int P>
__device__ __forceinline__ void tb_step(T (&win)[C::K][2 * C::R + 1][C::VX], const T* const* sb, int lane,
                                        const TbTile& t, int grp, int total, const Coefs<T, C::shape::NTERMS>& coef,
                                        const GridDesc& g, T* dst_grp, int vec_store) {
  constexpr int W = 2 * C::R + 1;
  const int s = grp * C::RB + P;  // input row relative to L0
  if constexpr (!FULL) {
    if (s >= total) return;
  }
  const int col = C::HXI + lane * C::VX;
  // Leading input row into level 0's window: push number s goes to slot s mod W.
  lds_vec<T, C::VX>(sb[C::B] + P * C::PLANE + col, win[0][(GP + P) % W]);
  if constexpr (FIRST) {
    if (s < 2 * C::R) return;  // level 0's window is still filling
  }
  // Level 0's centre row (s - R) for the warp-edge x-halo; stage offset is compile-time.
  constexpr int REL = P - C::R;  // relative to this group's first row
  constexpr int SK = REL >= 0 ? REL / C::RB : -((-REL + C::RB - 1) / C::RB);
  constexpr int OFF = REL - SK * C::RB;
  const T* edge_row = sb[C::B + SK] + OFF * C::PLANE + col;
  tb_levels<T, C, 1, (GP + P + 1) % W>(win, edge_row, lane, t, t.L0 + s, coef, g, dst_grp + P * g.so[0],
                                       vec_store);
}

template <typename T, class C, int GP, bool FIRST, bool FULL, int... Ps>
__device__ __forceinline__ void tb_group(T (&win)[C::K][2 * C::R + 1][C::VX], const T* const* sb, int lane,
                                         const TbTile& t, int grp, int total, const Coefs<T, C::shape::NTERMS>& coef,
                                         const GridDesc& g, T* dst_grp, int vec_store, std::integer_sequence<int, Ps...>) {
  (tb_step<T, C, GP, FIRST, FULL, Ps>(win, sb, lane, t, grp, total, coef, g, dst_grp, vec_store), ...);
}

template <typename T, class C, int GP>
__device__ __forceinline__ void tb_group_any(T (&win)[C::K][2 * C::R + 1][C::VX], const T* const* sb, int lane,
                                             const TbTile& t, int grp, int total,
                                             const Coefs<T, C::shape::NTERMS>& coef, const GridDesc& g, T* dst_grp,
                                             int vec_store) {
  using Seq = std::make_integer_sequence<int, C::RB>;
  if (grp == 0) tb_group<T, C, GP, true, false>(win, sb, lane, t, grp, total, coef, g, dst_grp, vec_store, Seq{});
  else if ((grp + 1) * C::RB <= total)
    tb_group<T, C, GP, false, true>(win, sb, lane, t, grp, total, coef, g, dst_grp, vec_store, Seq{});
  else tb_group<T, C, GP, false, false>(win, sb, lane, t, grp, total, coef, g, dst_grp, vec_store, Seq{});
}

// Dispatch the group body on its phase (grp * RB) mod W (compile-time slot arithmetic).
template <typename T, class C, int... GPs>
__device__ __forceinline__ void tb_group_phase(int phase, T (&win)[C::K][2 * C::R + 1][C::VX], const T* const* sb,
                                               int lane, const TbTile& t, int grp, int total,
                                               const Coefs<T, C::shape::NTERMS>& coef, const GridDesc& g,
                                               T* dst_grp, int vec_store, std::integer_sequence<int, GPs...>) {
  ((phase == GPs ? tb_group_any<T, C, GPs>(win, sb, lane, t, grp, total, coef, g, dst_grp, vec_store) : void()),
   ...);
}

template <typename T, class C>
__global__ void __launch_bounds__(32)
    march_tb2d_kernel(const __grid_constant__ CUtensorMap tmap, T* __restrict__ out, const TbArgs a,
                      const Coefs<T, C::shape::NTERMS> coef) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t bars[C::NS];
  T* ring = reinterpret_cast<T*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int lane = threadIdx.x;
  const bool leader = lane == 0;
  if (leader) {
    for (int i = 0; i < C::NS; ++i) mbar_init(&bars[i], 1);
    mbar_fence_init();
  }
  __syncthreads();
  const GridDesc& g = a.g;
  unsigned q_base = 0;
  int n_issued = 0, n_waited = 0;
  bool failed = false;
  T win[C::K][2 * C::R + 1][C::VX];

  for (long long item = blockIdx.x; item < a.n_items; item += gridDim.x) {
    const int tile_x = int(item % a.tiles_x);
    const int chunk = int(item / a.tiles_x);
    const int x0 = tile_x * C::TXO;
    TbTile t;
    t.mb = int(g.m_lo + (long long)chunk * a.chunk);
    t.me = (t.mb + a.chunk < g.m_hi) ? t.mb + a.chunk : int(g.m_hi);
    t.L0 = t.mb - C::K * C::R;
    t.row_lo = a.row_lo;
    t.row_hi = a.row_hi;
    const int total = (t.me - t.mb) + 2 * C::K * C::R;  // input rows of the item
    t.rows_safe = t.L0 >= t.row_lo && t.L0 + total <= t.row_hi;
    t.c0 = x0 - C::HL * C::VX + lane * C::VX;
    t.cmask = 0;
#pragma unroll
    for (int e = 0; e < C::VX; ++e)
      if (t.c0 + e >= 0 && t.c0 + e < g.no[2]) t.cmask |= 1 << e;
    t.edge = (x0 - C::HL * C::VX < 0) || (x0 - C::HL * C::VX + 32 * C::VX > g.no[2]);
    t.store_lane = lane >= C::HL && lane < 32 - C::HL && t.c0 < g.no[2];
    const int ngroups = (total + C::RB - 1) / C::RB;
    const int qt = ngroups;
    const int cx = x0 - C::HL * C::VX - C::HXI;
    const int L0 = t.L0 + g.org[0];  // input-buffer row of the first input row
    // Store address of level K's row for step s = 0 (row L0 - K*R), this lane's columns.
    T* const out0 = out + (long long)(t.L0 - C::K * C::R) * g.so[0] + (long long)t.c0 * g.so[2];
    auto issue = [&](int q) {
      const unsigned slot = (q_base + unsigned(q)) % C::NS;
      mbar_expect_tx(&bars[slot], unsigned(C::PLANE * C::RB * sizeof(T)));
      tma_load_3d(ring + size_t(slot) * C::STAGE, &tmap, &bars[slot], cx, 0, L0 + q * C::RB);
    };
    __syncthreads();
    n_issued = qt < C::NS ? qt : C::NS;
    n_waited = 0;
    if (leader) {
      fence_proxy_async_smem();
      for (int q = 0; q < n_issued; ++q) issue(q);
    }
#pragma unroll
    for (int l = 0; l < C::K; ++l)
#pragma unroll
      for (int k = 0; k < 2 * C::R + 1; ++k)
#pragma unroll
        for (int e = 0; e < C::VX; ++e) win[l][k][e] = T(0);

    for (int grp = 0; grp < ngroups; ++grp) {
      for (; n_waited <= grp; ++n_waited) {
        const unsigned gq = q_base + unsigned(n_waited);
        if (!failed && !mbar_wait_bounded(&bars[gq % C::NS], (gq / C::NS) & 1u)) failed = true;
      }
      if (__syncthreads_or(failed)) {
        failed = true;
        break;
      }
      if (grp >= 1) {
        const int lim = grp - C::B + C::NS;  // stages before grp - B are retired
        const int target = qt < lim ? qt : lim;
        if (n_issued < target) {
          if (leader) {
            fence_proxy_async_smem();
            for (int q = n_issued; q < target; ++q) issue(q);
          }
          n_issued = target;
        }
      }
      const T* sb[C::B + 1];  // stages grp-B .. grp (earlier ones only for the edge halo rows)
#pragma unroll
      for (int k = 0; k <= C::B; ++k) {
        const int q = grp - C::B + k;
        sb[k] = ring + size_t((q_base + unsigned(q < 0 ? 0 : q)) % C::NS) * C::STAGE;
      }
      constexpr int W = 2 * C::R + 1;
      T* dst_grp = out0 + (long long)grp * C::RB * g.so[0];
      if constexpr (C::RB % W == 0)  // every group starts at phase 0: one body
        tb_group_any<T, C, 0>(win, sb, lane, t, grp, total, coef, g, dst_grp, a.vec_store);
      else
        tb_group_phase<T, C>((grp * C::RB) % W, win, sb, lane, t, grp, total, coef, g, dst_grp, a.vec_store,
                             std::make_integer_sequence<int, W>{});
    }
    if (failed) break;
    q_base += unsigned(qt);
  }

  if (failed) {
    if (leader) {
      atomicOr(a.err, kErrTmaTimeout);
      for (int q = n_waited; q < n_issued; ++q) {
        const unsigned gq = q_base + unsigned(q);
        const uint64_t t0 = global_ns();
        while (!mbar_try_wait(&bars[gq % C::NS], (gq / C::NS) & 1u) && global_ns() - t0 < 200000000ull) {
        }
      }
    }
    __syncthreads();
  }
}

}  // namespace bst
