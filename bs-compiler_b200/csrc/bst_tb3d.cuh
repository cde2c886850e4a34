// bst_tb3d.cuh — temporally blocked 3-D march: K sweeps of a 3-D seven-point stencil per launch.
//
// A multi-sweep run of a 3-D stencil reads and writes the whole grid once per sweep; for the
// seven-point heat step that traffic is the bound (one sweep runs at ~94 % of HBM).  This kernel
// keeps K successive sweeps in flight in one pass, so HBM is read and written once per K sweeps.
// Every level performs the same separately rounded operations in the same order as a single
// sweep, so the result is bit-identical to K launches.
//
//  * A CTA owns a tile of TYL rows x 128 columns (fp32) of every plane and marches along Z;
//    warp w holds row w, lane j the 16-byte vector of columns 4j..4j+3.  Level 0 (the input)
//    arrives plane by plane through TMA into a ring; level l computes plane s - l at step s from
//    level l-1's planes s-l-1 .. s-l+1.
//  * Neighbours: along Z from each level's 3-plane register window; along X from the own
//    vector and the neighbouring lanes (shuffles; level 0's warp-edge lanes read the loaded
//    halo columns); along Y from other warps: level 0's rows come from the TMA ring, level l's
//    (1 <= l < K) from a double-buffered shared-memory plane that level l writes at step s and
//    level l+1 reads at step s+1, one CTA barrier per step in between.
//  * Valid region: level l is exact on rows [l, TYL-l) and on lanes whose columns stay within
//    K-1 of the warp's loaded edge, so a tile stores rows [K, TYL-K) and lanes 1..30; tiles
//    overlap accordingly.  Level values outside the grid (rows, columns, or planes outside
//    [row_lo, row_hi)) are forced to zero, exactly as one sweep reads zeros there.
//  * Planes: an item of output planes [mb, me) reads input planes [mb-K, me+K).
#pragma once
#include "bst_kernels.cuh"

namespace bst {

template <typename T, class S, int K_, int TYL_, int NSX_>
struct Tb3Cfg {
  using shape = S;
  static constexpr int K = K_;
  static constexpr int R = 1;
  static constexpr int VX = 16 / int(sizeof(T));
  static constexpr int HL = 1;                        // overlap lanes at each warp edge
  static constexpr int TXO = (32 - 2 * HL) * VX;      // stored columns per tile
  static constexpr int HXI = VX;                      // loaded columns beyond the warp, each side
  static constexpr int TXL = 32 * VX + 2 * HXI;       // loaded columns per row
  static constexpr int TYL = TYL_;                    // loaded rows per tile = warps per CTA
  static constexpr int TYO = TYL - 2 * K * R;         // stored rows per tile
  static constexpr int PLANE = TXL * TYL;
  static constexpr int STAGE_BYTES = round_up_c(PLANE * int(sizeof(T)), 128);
  static constexpr int STAGE = STAGE_BYTES / int(sizeof(T));
  // Step s reads stages s (level 0's new plane) and s-1 (its y-neighbours for level 1); a step
  // waits before its barrier and refills after it, so a stage must be issued a step before it
  // is waited on: NS >= 3.
  static constexpr int NS = 2 + NSX_;
  static constexpr int SROW = 32 * VX;                // one row of an exchange plane
  static constexpr int SPLANE = SROW * TYL;
  static constexpr int XBYTES = (K > 1 ? K - 1 : 0) * 2 * SPLANE * int(sizeof(T));
  static constexpr int SMEM = NS * STAGE_BYTES + XBYTES + 128;
  static constexpr int THREADS = 32 * TYL;
  static_assert(window_mode<S>() && S::RM == 1 && S::RY == 1 && S::RX == 1, "radius-1 3-D window shapes");
  static_assert(K >= 1 && (K - 1) * R <= HL * VX, "stored columns stay valid through K levels");
  static_assert(TXL <= 256 && TYL <= 32 && TYO >= 1, "TMA box extent / CTA size");
  static_assert(NS >= 3, "every stage is issued a step before it is waited on");
};

struct Tb3Args {
  GridDesc g;
  int tiles_x, tiles_y;
  int chunk;
  long long n_items;
  unsigned* err;
  int vec_store;
  int row_lo, row_hi;  // planes (output coordinates) whose level values are computed; others are ghosts (0)
};

// Taps of point V of a level: Z from the window (slots 0, 1, 2 = planes p-1, p, p+1), Y from the
// neighbouring rows' vectors, X from the segment (own vector with one element each side).
template <typename T, class C, int V>
struct Tb3Fetch {
  const T (&w)[3][C::VX];
  const T (&ym)[C::VX];
  const T (&yp)[C::VX];
  const T (&seg)[C::VX + 2];
  template <int dm, int dy, int dx>
  __device__ __forceinline__ T get() const {
    if constexpr (dm != 0) return w[1 + dm][V];
    else if constexpr (dy < 0) return ym[V];
    else if constexpr (dy > 0) return yp[V];
    else return seg[1 + V + dx];
  }
};

template <typename T, class C, int... Vs>
__device__ __forceinline__ void tb3_eval(const T (&w)[3][C::VX], const T (&ym)[C::VX], const T (&yp)[C::VX],
                                         const T (&seg)[C::VX + 2], const Coefs<T, C::shape::NTERMS>& c,
                                         T (&res)[C::VX], std::integer_sequence<int, Vs...>) {
  ((res[Vs] = eval_shape<typename C::shape, T>(Tb3Fetch<T, C, Vs>{w, ym, yp, seg}, c)), ...);
}

// Per-item constants (32-bit coordinates: plane, row and column indices of the output grid).
struct Tb3Tile {
  int L0;              // output-coordinate plane of the item's step 0
  int mb, me;          // stored output planes
  int row_lo, row_hi;  // level values outside these planes are ghosts (0)
  int y;               // this warp's row
  bool row_in;         // that row lies inside the grid
  bool row_store;      // that row is stored (inside the tile's stored rows and the grid)
  int cmask;           // bit e: this lane's column e lies inside the grid
  bool store_lane;     // this lane's columns are stored
  int c0;              // first column of this lane
};

// Level L (1..K) at step s: computes plane s - L from level L-1's window (and its y-rows), then
// either feeds level L+1 (window + exchange plane) or, at L == K, stores.
template <typename T, class C, int L>
__device__ __forceinline__ void tb3_level(T (&win)[C::K][3][C::VX], T* xbuf, const T* ring_prev,
                                          int warp, int lane, const Tb3Tile& t, int s,
                                          const Coefs<T, C::shape::NTERMS>& coef, const GridDesc& g, T* dst,
                                          int vec_store) {
  if constexpr (L <= C::K) {
    if (s >= 2 * L) {
      const int ym_w = warp > 0 ? warp - 1 : 0, yp_w = warp < C::TYL - 1 ? warp + 1 : C::TYL - 1;
      T ym[C::VX], yp[C::VX], seg[C::VX + 2];
      const T(&w)[3][C::VX] = win[L - 1];
      if constexpr (L == 1) {  // level 0's plane s-1: rows from the TMA ring
        const T* base = ring_prev + C::HXI + lane * C::VX;
        lds_vec<T, C::VX>(base + ym_w * C::TXL, ym);
        lds_vec<T, C::VX>(base + yp_w * C::TXL, yp);
      } else {  // level L-1's plane s-L: rows from its exchange plane (slot (s-L) & 1)
        const T* xp = xbuf + (size_t((L - 2) * 2 + ((s - L) & 1)) * C::SPLANE) + lane * C::VX;
        lds_vec<T, C::VX>(xp + ym_w * C::SROW, ym);
        lds_vec<T, C::VX>(xp + yp_w * C::SROW, yp);
      }
#pragma unroll
      for (int e = 0; e < C::VX; ++e) seg[1 + e] = w[1][e];
      T left = __shfl_up_sync(0xffffffffu, w[1][C::VX - 1], 1);
      T right = __shfl_down_sync(0xffffffffu, w[1][0], 1);
      if constexpr (L == 1) {  // the warp's edge lanes read level 0's loaded halo columns
        const T* row = ring_prev + warp * C::TXL + C::HXI + lane * C::VX;
        if (lane == 0) left = row[-1];
        if (lane == 31) right = row[C::VX];
      }
      seg[0] = left;
      seg[C::VX + 1] = right;
      T res[C::VX];
      tb3_eval<T, C>(w, ym, yp, seg, coef, res, std::make_integer_sequence<int, C::VX>{});
      const int plane = t.L0 + s - L;  // output-coordinate plane this level computed
      if constexpr (L < C::K) {
        // Ghost cells of level L+1 are zero: planes outside [row_lo, row_hi), rows and
        // columns outside the grid.
        if (plane < t.row_lo || plane >= t.row_hi || !t.row_in) {
#pragma unroll
          for (int e = 0; e < C::VX; ++e) res[e] = T(0);
        } else if (t.cmask != (1 << C::VX) - 1) {
#pragma unroll
          for (int e = 0; e < C::VX; ++e)
            if (!((t.cmask >> e) & 1)) res[e] = T(0);
        }
        T* xo = xbuf + (size_t((L - 1) * 2 + ((s - L) & 1)) * C::SPLANE) + warp * C::SROW + lane * C::VX;
        using VT = typename Vec16<T>::type;
        VT q;
        T* qe = reinterpret_cast<T*>(&q);
#pragma unroll
        for (int e = 0; e < C::VX; ++e) {
          qe[e] = res[e];
          win[L][2][e] = res[e];
        }
        *reinterpret_cast<VT*>(xo) = q;
        tb3_level<T, C, L + 1>(win, xbuf, ring_prev, warp, lane, t, s, coef, g, dst, vec_store);
      } else if (plane >= t.mb && plane < t.me && t.row_store && t.store_lane) {
        T* d = dst + (long long)plane * g.so[0];
        if (vec_store && t.c0 + C::VX <= g.no[2]) {
          using VT = typename Vec16<T>::type;
          VT q;
          T* qe = reinterpret_cast<T*>(&q);
#pragma unroll
          for (int v = 0; v < C::VX; ++v) qe[v] = res[v];
          *reinterpret_cast<VT*>(d) = q;
        } else {
#pragma unroll
          for (int v = 0; v < C::VX; ++v)
            if (t.c0 + v < g.no[2]) d[(long long)v * g.so[2]] = res[v];
        }
      }
    }
  }
}

template <typename T, class C>
__global__ void __launch_bounds__(C::THREADS, 1)
    march_tb3d_kernel(const __grid_constant__ CUtensorMap tmap, T* __restrict__ out, const Tb3Args a,
                      const Coefs<T, C::shape::NTERMS> coef) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t bars[C::NS];
  T* ring = reinterpret_cast<T*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  T* xbuf = ring + size_t(C::NS) * C::STAGE;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const bool leader = threadIdx.x == 0;
  if (leader) {
    for (int i = 0; i < C::NS; ++i) mbar_init(&bars[i], 1);
    mbar_fence_init();
  }
  __syncthreads();
  const GridDesc& g = a.g;
  unsigned q_base = 0;
  int n_issued = 0, n_waited = 0;
  bool failed = false;
  T win[C::K][3][C::VX];
  const long long tiles = (long long)a.tiles_x * a.tiles_y;

  for (long long item = blockIdx.x; item < a.n_items; item += gridDim.x) {
    const long long tile = item % tiles;
    const int chunk = int(item / tiles);
    const int tile_x = int(tile % a.tiles_x), tile_y = int(tile / a.tiles_x);
    const int x0 = tile_x * C::TXO, y0 = tile_y * C::TYO;
    Tb3Tile t;
    t.mb = int(g.m_lo + (long long)chunk * a.chunk);
    t.me = (t.mb + a.chunk < g.m_hi) ? t.mb + a.chunk : int(g.m_hi);
    t.L0 = t.mb - C::K * C::R;
    t.row_lo = a.row_lo;
    t.row_hi = a.row_hi;
    t.y = y0 - C::K * C::R + warp;
    t.row_in = t.y >= 0 && t.y < g.no[1];
    t.row_store = warp >= C::K * C::R && warp < C::TYL - C::K * C::R && t.y < g.no[1];
    t.c0 = x0 - C::HL * C::VX + lane * C::VX;
    t.cmask = 0;
#pragma unroll
    for (int e = 0; e < C::VX; ++e)
      if (t.c0 + e >= 0 && t.c0 + e < g.no[2]) t.cmask |= 1 << e;
    t.store_lane = lane >= C::HL && lane < 32 - C::HL && t.c0 < g.no[2];
    const int total = (t.me - t.mb) + 2 * C::K * C::R;  // steps (input planes) of the item
    const int cx = x0 - C::HL * C::VX - C::HXI + g.org[2];
    const int cy = y0 - C::K * C::R + g.org[1];
    const int cz = t.L0 + g.org[0];  // input-buffer plane of step 0
    T* const dst = out + (long long)t.y * g.so[1] + (long long)t.c0 * g.so[2];
    auto issue = [&](int q) {
      const unsigned slot = (q_base + unsigned(q)) % C::NS;
      mbar_expect_tx(&bars[slot], unsigned(C::PLANE * sizeof(T)));
      tma_load_3d(ring + size_t(slot) * C::STAGE, &tmap, &bars[slot], cx, cy, cz + q);
    };
    __syncthreads();  // the previous item is done with the ring and the exchange planes
    n_issued = total < C::NS ? total : C::NS;
    n_waited = 0;
    if (leader) {
      fence_proxy_async_smem();
      for (int q = 0; q < n_issued; ++q) issue(q);
    }
#pragma unroll
    for (int l = 0; l < C::K; ++l)
#pragma unroll
      for (int k = 0; k < 3; ++k)
#pragma unroll
        for (int e = 0; e < C::VX; ++e) win[l][k][e] = T(0);

    for (int s = 0; s < total; ++s) {
      for (; n_waited <= s; ++n_waited) {
        const unsigned gq = q_base + unsigned(n_waited);
        if (!failed && !mbar_wait_bounded(&bars[gq % C::NS], (gq / C::NS) & 1u)) failed = true;
      }
      // CTA-uniform; also orders step s-1's exchange-plane writes before this step's reads and
      // retires stage s-2 from every thread.
      if (__syncthreads_or(failed)) {
        failed = true;
        break;
      }
      if (s >= 1) {
        const int lim = s - 1 + C::NS;  // stages before s-1 are retired
        const int target = total < lim ? total : lim;
        if (n_issued < target) {
          if (leader) {
            fence_proxy_async_smem();
            for (int q = n_issued; q < target; ++q) issue(q);
          }
          n_issued = target;
        }
      }
      const T* cur = ring + size_t((q_base + unsigned(s)) % C::NS) * C::STAGE;
      const T* prev = ring + size_t((q_base + unsigned(s > 0 ? s - 1 : 0)) % C::NS) * C::STAGE;
      // Level 0's new plane into its window.
      lds_vec<T, C::VX>(cur + warp * C::TXL + C::HXI + lane * C::VX, win[0][2]);
      tb3_level<T, C, 1>(win, xbuf, prev, warp, lane, t, s, coef, g, dst, a.vec_store);
      // Every window moves one plane on.
#pragma unroll
      for (int l = 0; l < C::K; ++l)
#pragma unroll
        for (int e = 0; e < C::VX; ++e) {
          win[l][0][e] = win[l][1][e];
          win[l][1][e] = win[l][2][e];
        }
    }
    if (failed) break;
    q_base += unsigned(total);
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
