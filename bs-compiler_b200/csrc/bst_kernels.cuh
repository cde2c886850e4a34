// bst_kernels.cuh — the sm_100a stencil kernels.
//
//  * march_tma_kernel : 2-D/3-D sweep.  Each CTA owns a TX x TY tile of one M-chunk and
//    marches along M.  Input planes arrive by TMA (cp.async.bulk.tensor, no multicast)
//    into a ring of NS shared-memory stages of RB planes each, completion tracked by one
//    mbarrier per stage; TMA's out-of-bounds zero fill supplies the Dirichlet-0 ghost
//    cells, so the interior and the boundary run the same code.  Taps are read from the
//    ring at compile-time offsets; the result is stored with coalesced global stores.
//    Persistent: the grid is at most the resident CTA count; the work schedule (round-robin
//    items or contiguous balanced shares) is chosen per launch (MarchArgs).
//  * line_kernel      : 1-D sweep with 128-bit vector loads/stores and warp shuffles for
//    the neighbour elements held by adjacent lanes.
//  * direct_kernel    : any layout/stride (the fallback when TMA's 16-byte rules are not
//    met): one thread per output point, taps read through the read-only cache.
// Every kernel increments nothing and allocates nothing; waits on mbarriers are bounded
// and report through an error word instead of trapping.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <type_traits>
#include <utility>

#include "bst_shapes.cuh"

namespace bst {

// Error word bits written by kernels (host reads them back on request).
enum : unsigned { kErrTmaTimeout = 1u, kErrPeerTimeout = 2u };

constexpr int round_up_c(int v, int m) { return (v + m - 1) / m * m; }
constexpr int floor_div_c(int a, int b) { return a >= 0 ? a / b : -((-a + b - 1) / b); }

// ---------------------------------------------------------------------------------
// PTX helpers (mbarrier + TMA).  Hand-written inline PTX for sm_100a.
__device__ __forceinline__ unsigned smem_u32(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait: gives up after ~2 s of wall time and returns false.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, unsigned parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (unsigned it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0 && global_ns() - t0 > 2000000000ull) return false;
  }
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                            int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------------
// Register-blocked evaluation plan (compile time).
//
// Each thread owns VX consecutive x (one 16-byte vector) of PY consecutive rows of the tile
// and marches along M.  Two sources feed the taps:
//  * the M-window: when every tap off the current plane is a centre tap (dy = dx = 0, as in
//    the star stencils), the thread keeps the centre vectors of planes m-WM..m+WM in
//    registers and loads only the leading plane per step;
//  * row segments: every other (dm, row) the taps touch is loaded once per step as one
//    128-bit shared-memory vector per thread, its x-halo taken from neighbouring lanes by
//    warp shuffles (lanes at a row edge read the halo from shared memory instead).
struct SegRow {
  int dm, srow, lo, hi;  // plane offset, row relative to the thread's first row, element range
};
template <int N>
struct SegTable {
  SegRow r[N > 0 ? N : 1];
  int n;
};

template <class S>
constexpr bool window_mode() {
  for (int i = 0; i < S::NTAPS; ++i) {
    const Tap t = S::tbl.taps[i];
    if (t.dm != 0 && (t.dy != 0 || t.dx != 0)) return false;
  }
  return true;
}

template <class S, int PY, int VX, bool W = window_mode<S>()>
constexpr auto make_segs() {
  constexpr int NMAX = (2 * S::RM + 1) * (PY + 2 * S::RY);
  SegTable<NMAX> t{};
  t.n = 0;
  for (int j = 0; j < PY; ++j)
    for (int i = 0; i < S::NTAPS; ++i) {
      const Tap tp = S::tbl.taps[i];
      if (W && (tp.dm != 0 || (tp.dy == 0 && tp.dx == 0))) continue;  // from the window
      const int srow = j + tp.dy;
      int k = 0;
      while (k < t.n && !(t.r[k].dm == tp.dm && t.r[k].srow == srow)) ++k;
      if (k == t.n) {
        t.r[k] = SegRow{tp.dm, srow, tp.dx, VX - 1 + tp.dx};
        ++t.n;
      } else {
        t.r[k].lo = t.r[k].lo < tp.dx ? t.r[k].lo : tp.dx;
        t.r[k].hi = t.r[k].hi > VX - 1 + tp.dx ? t.r[k].hi : VX - 1 + tp.dx;
      }
    }
  return t;
}

template <class S>
constexpr int window_depth() {
  int w = 0;
  for (int i = 0; i < S::NTAPS; ++i) w = cmax(w, cabs(S::tbl.taps[i].dm));
  return window_mode<S>() ? w : 0;
}

// Streaming mode: every term reads a single plane offset dm, the fold visits the offsets in
// ascending order and starts at -RM (box stencils in slowest-axis-major order).  Input planes
// then arrive in fold order: when plane p arrives, output p+RM starts its fold with the
// dm = -RM terms, the outputs in between continue with their middle offsets, and output p-RM
// completes with dm = +RM.  Each input row is read from shared memory once per step instead
// of once per plane offset, and the result keeps the exact operation order.
template <class S>
constexpr bool stream_mode() {
  if (S::RM == 0 || window_mode<S>()) return false;
  int prev = -S::RM;
  if (S::tbl.taps[S::tbl.terms[0].first].dm != -S::RM) return false;
  for (int g = 0; g < S::NTERMS; ++g) {
    const Term t = S::tbl.terms[g];
    const int dm = S::tbl.taps[t.first].dm;
    for (int k = 1; k < t.count; ++k)
      if (S::tbl.taps[t.first + k].dm != dm) return false;
    if (dm < prev) return false;
    prev = dm;
  }
  return true;
}

// First term whose plane offset is >= dm (stream mode): offset dm's terms are
// [group_begin(dm), group_begin(dm + 1)).
template <class S>
constexpr int group_begin(int dm) {
  for (int g = 0; g < S::NTERMS; ++g)
    if (S::tbl.taps[S::tbl.terms[g].first].dm >= dm) return g;
  return S::NTERMS;
}

// Stream mode rows: the lead plane's rows -RY .. PY-1+RY, each with the full x-halo.
template <class S, int PY, int VX>
constexpr auto make_stream_segs() {
  SegTable<PY + 2 * S::RY> t{};
  t.n = PY + 2 * S::RY;
  for (int i = 0; i < t.n; ++i) t.r[i] = SegRow{S::RM, i - S::RY, -S::RX, VX - 1 + S::RX};
  return t;
}

template <bool STREAM, bool WINDOW, class S, int PY, int VX>
constexpr auto pick_segs() {
  if constexpr (STREAM) return make_stream_segs<S, PY, VX>();
  else return make_segs<S, PY, VX, WINDOW>();
}

// ---------------------------------------------------------------------------------
// March kernel configuration (compile time).
// HALO_LDS: a row's x-halo comes as whole neighbouring vectors from shared memory (one
// ld.shared.v4 each) instead of shuffles plus edge-lane loads; cheaper in issue slots for
// wide radii, dearer in shared-memory bandwidth.
// VXB_: bytes of one lane's vector of consecutive x points (16; 8 halves a lane's registers).
template <typename T, class S, int TX_, int TY_, int PY_, int RB_, int NSX_, bool HALO_LDS_ = false,
          bool STREAM_ = false, bool WINDOW_ = true, int MINB_ = 1, bool PAIR_ = false, bool CIRC_ = false,
          int INTERLEAVE_ = 0, int VXB_ = 16>
struct MarchCfg {
  using shape = S;
  static constexpr int MINB = MINB_;  // CTAs per SM the register allocation must allow
  static constexpr bool HALO_LDS = HALO_LDS_;
  static constexpr bool STREAM = STREAM_ && stream_mode<S>();
  static constexpr int VX = VXB_ / int(sizeof(T));  // elements per lane vector
  static constexpr int TX = TX_;                   // output columns per tile
  static constexpr int TY = TY_;                   // output rows per tile
  static constexpr int PY = PY_;                   // rows per thread
  static constexpr int RB = RB_;                   // planes per stage (power of two)
  static constexpr int RM = S::RM, RY = S::RY, RX = S::RX;
  static constexpr int LPR = TX / VX;              // lanes per tile row
  static constexpr int NRG = TY / PY;              // row groups
  static constexpr int THREADS = LPR * NRG;
  static constexpr int HX = ((RX + VX - 1) / VX) * VX;  // x halo, whole vectors
  static constexpr int XC = HX;                    // tile column of output x0 (16-byte aligned)
  static constexpr int TXL = TX + 2 * HX;          // loaded columns (<= 256)
  static constexpr int TYL = TY + 2 * RY;          // loaded rows
  static constexpr int PLANE = TXL * TYL;          // elements per plane tile
  static constexpr int STAGE_BYTES = round_up_c(PLANE * RB * int(sizeof(T)), 128);
  static constexpr int STAGE = STAGE_BYTES / int(sizeof(T));
  // Window mode (off-centre plane taps from a register window) where the shape allows it
  // and the configuration asks for it; otherwise every tap is read from the shared ring.
  static constexpr bool WINDOW = WINDOW_ && window_mode<S>();
  static constexpr int WM = WINDOW ? window_depth<S>() : 0;
  // Window slots: a group of RB plane steps reads planes g0-WM .. g0+RB-1+WM (g0 = the group's
  // first output plane), so the window holds 2WM+RB planes and shifts by RB once per group.
  static constexpr int WSLOTS = WINDOW ? 2 * WM + RB : 1;
  // Circular window: instead of shifting the window by RB registers per group, group g uses
  // the slots of phase g mod PHASES, so a plane stays in one register for its whole life and
  // the group body exists once per phase (PHASES copies of the code, no register moves).
  static constexpr bool CIRC = CIRC_ && WINDOW && WSLOTS % RB == 0;
  static constexpr int PHASES = CIRC ? WSLOTS / RB : 1;
  // Window register slot of relative slot `rel` (0 = the group's oldest plane) in phase ph.
  static constexpr int wslot(int ph, int rel) { return CIRC ? (ph * RB + rel) % WSLOTS : rel; }
  // fp32 points evaluated two at a time with paired instructions.
  static constexpr bool PAIR = PAIR_ && sizeof(T) == 4;
  // Paired folds: 1 = the thread's point pairs of a plane advance term by term together;
  // 2 = the pairs of all RB planes of a group do (each plane step gets its own row segments).
  static constexpr int INTERLEAVE = (PAIR && !STREAM) ? INTERLEAVE_ : 0;
  static constexpr int SEGBANKS = INTERLEAVE == 2 ? RB : 1;
  static constexpr int bank(int p) { return SEGBANKS > 1 ? p : 0; }
  // Stages read by group g (input planes g*RB + [0, RB-1+2RM] relative to the item's first
  // loaded plane): the window keeps planes behind the current one in registers, so in window
  // mode group g only reads from plane g*RB + RM on and earlier stages retire early.
  static constexpr int NEED = 1 + (RB - 1 + 2 * RM) / RB;  // stages of group 0 (incl. window fill)
  // First stage still read, minus g: stream mode reads only the lead plane (g*RB + P + 2RM),
  // window mode the centre plane on, otherwise every plane from g*RB on.
  static constexpr int FIRST_OFF = (STREAM ? 2 * RM : (WINDOW ? RM : 0)) / RB;
  static constexpr int SPAN = NEED - FIRST_OFF;            // stages one steady-state group reads
  // Ring depth.  A group waits before its barrier and refills after it, so every stage a
  // group waits for must have been issued one group earlier: NS >= NEED + 1 covers group 1
  // (from the initial fill) and every later group (from the previous group's refill).
  static constexpr int NS = NEED + 1 > SPAN + NSX_ ? NEED + 1 : SPAN + NSX_;
  static constexpr int SMEM = NS * STAGE_BYTES + 128;      // + alignment slack
  static constexpr auto SEGS = pick_segs<STREAM, WINDOW, S, PY, VX>();
  static constexpr int NSEG = SEGS.n;
  static constexpr int SEGW = VX + 2 * HX;
  static_assert(TXL <= 256 && TYL <= 256 && RB <= 256, "TMA box extent");
  static_assert(TX % VX == 0 && (LPR & (LPR - 1)) == 0 && LPR <= 32, "lanes per row: power of two <= 32");
  static_assert(TY % PY == 0 && THREADS % 32 == 0, "whole warps");
  static_assert((RB & (RB - 1)) == 0, "RB power of two");
  static_assert(RX <= 2 * VX, "x halo within two neighbouring lanes");
  static_assert(NS >= NEED + 1, "every stage is issued before a group waits on it");

  static constexpr int seg_index(int dm, int srow) {
    for (int k = 0; k < SEGS.n; ++k)
      if (SEGS.r[k].dm == dm && SEGS.r[k].srow == srow) return k;
    return -1;
  }
};

// Work of one launch: tiles_x * tiles_y tile columns of nm planes each.  Two schedules:
//  * items (balanced == 0): the columns are cut into chunks of `chunk` planes; item
//    i = tile + tiles * chunk_index, and CTAs take items round-robin.  CTAs running at the
//    same time hold adjacent tiles of the same planes, so x/y halo re-reads hit L2.
//  * balanced (balanced == 1): the work is linearised as w = tile * nm + plane, and CTA b
//    marches the contiguous range [b*W/G, (b+1)*W/G) as one or more segments.  Every CTA
//    finishes together and M-halo planes are re-read only at segment starts.
struct MarchArgs {
  GridDesc g;
  int tiles_x, tiles_y;
  long long nm;        // planes per tile column
  long long work;      // items (balanced == 0) or tiles * nm (balanced == 1)
  long long chunk;     // planes per item (balanced == 0)
  int balanced;
  unsigned* err;
  int vec_store;  // output rows are 16-byte aligned and contiguous in x
  PeerStore peer;  // slab sweeps with peer stores (the PEER kernel); the two boundary chunks then
                  // run first (chunk 0, the last chunk, then the interior chunks in order)
  // Item plan (balanced == 0) in two bands: items [0, work1) cover tile columns [0, tiles1) in
  // chunks of `chunk` planes, items [work1, work) the other columns in chunks of `chunk2`.
  long long work1;
  long long chunk2;
  long long tiles1;
  // Two plane ranges in one launch (item schedule): items whose first plane is at or above
  // gap_at are moved up by gap planes (LLONG_MAX: one range).
  long long gap_at;
  long long gap;
};

// Balanced contiguous range of CTA b among G CTAs over W units.
__device__ __forceinline__ void cta_range(long long W, long long b, long long G, long long* w0, long long* w1) {
  const long long base = W / G, rem = W % G;
  *w0 = b * base + (b < rem ? b : rem);
  *w1 = *w0 + base + (b < rem ? 1 : 0);
}

template <typename T>
struct Vec16;
template <>
struct Vec16<float> {
  using type = float4;
  static constexpr int N = 4;
};
template <>
struct Vec16<double> {
  using type = double2;
  static constexpr int N = 2;
};

// N consecutive elements of T moved by one 8- or 16-byte access.
template <typename T, int N>
struct VecN;
template <>
struct VecN<float, 4> {
  using type = float4;
};
template <>
struct VecN<float, 2> {
  using type = float2;
};
template <>
struct VecN<double, 2> {
  using type = double2;
};
template <>
struct VecN<double, 1> {
  using type = double;
};

// Per-thread register state of the march: window and row segments.
template <typename T, class C>
struct MarchRegs {
  T win[C::WSLOTS][C::PY][C::VX];
  T seg[C::SEGBANKS][C::NSEG > 0 ? C::NSEG : 1][C::SEGW];
  T acc[C::STREAM ? 2 * C::RM + 1 : 1][C::PY][C::VX];  // stream mode: outputs g .. g+2RM in flight
};

// Tap values of point (row J, element V) at plane step P of a group of window phase PH.
template <typename T, class C, int J, int V, int P = 0, int PH = 0>
struct PointFetch {
  const MarchRegs<T, C>& r;
  template <int dm, int dy, int dx>
  __device__ __forceinline__ T get() const {
    if constexpr (C::WINDOW && (dm != 0 || (dy == 0 && dx == 0))) {
      return r.win[C::wslot(PH, P + C::WM + dm)][J][V];
    } else if constexpr (C::STREAM) {  // every offset reads the current lead plane's rows
      constexpr int k = C::seg_index(C::RM, J + dy);
      static_assert(k >= 0, "tap without a row segment");
      return r.seg[C::bank(P)][k][C::HX + V + dx];
    } else {
      constexpr int k = C::seg_index(dm, J + dy);
      static_assert(k >= 0, "tap without a row segment");
      return r.seg[C::bank(P)][k][C::HX + V + dx];
    }
  }
};

template <typename T, int N>
__device__ __forceinline__ void lds_vec(const T* p, T (&v)[N]) {
  using VT = typename VecN<T, N>::type;
  const VT q = *reinterpret_cast<const VT*>(p);
  const T* e = reinterpret_cast<const T*>(&q);
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = e[i];
}

// Load row segment K for the plane whose tile starts at `pl` (dm already applied), at plane
// step P of a group.  `pl` points at the thread's first vector (row 0 of its rows) in the
// plane tile.
template <typename T, class C, int K, int P = 0, int PH = 0>
__device__ __forceinline__ void load_segment(MarchRegs<T, C>& r, const T* pl, int /*unused*/, int lane_x) {
  constexpr SegRow R = C::SEGS.r[K];
  const T* rowp = pl + R.srow * C::TXL;
  T own[C::VX];
  if constexpr (C::WINDOW && R.dm == 0 && R.srow >= 0 && R.srow < C::PY) {
#pragma unroll
    for (int e = 0; e < C::VX; ++e) own[e] = r.win[C::wslot(PH, P + C::WM)][R.srow][e];
  } else {
    lds_vec<T, C::VX>(rowp, own);
  }
#pragma unroll
  for (int e = 0; e < C::VX; ++e) r.seg[C::bank(P)][K][C::HX + e] = own[e];
  if constexpr (C::HALO_LDS) {
    // x-halo as whole neighbouring 16-byte vectors straight from the tile (it holds HX
    // loaded columns on each side): one ld.shared.v4 per vector instead of a shuffle and a
    // predicated edge load per element.
    constexpr int v_lo = floor_div_c(R.lo, C::VX), v_hi = floor_div_c(R.hi, C::VX);
#pragma unroll
    for (int vv = v_lo; vv <= v_hi; ++vv) {
      if (vv == 0) continue;
      T nb[C::VX];
      lds_vec<T, C::VX>(rowp + vv * C::VX, nb);
#pragma unroll
      for (int e = 0; e < C::VX; ++e)
        if (vv * C::VX + e >= R.lo && vv * C::VX + e <= R.hi) r.seg[C::bank(P)][K][C::HX + vv * C::VX + e] = nb[e];
    }
  } else {
    // x-halo from neighbouring lanes; the tile's edge lanes read shared memory.
#pragma unroll
    for (int e = R.lo; e < 0; ++e) {
      const int d = (-e + C::VX - 1) / C::VX;  // lanes to the left holding element e
      T v = __shfl_up_sync(0xffffffffu, own[e + d * C::VX], d, C::LPR);
      if (lane_x < d) v = rowp[e];
      r.seg[C::bank(P)][K][C::HX + e] = v;
    }
#pragma unroll
    for (int e = C::VX; e <= R.hi; ++e) {
      const int d = e / C::VX;  // lanes to the right holding element e
      T v = __shfl_down_sync(0xffffffffu, own[e - d * C::VX], d, C::LPR);
      if (lane_x >= C::LPR - d) v = rowp[e];
      r.seg[C::bank(P)][K][C::HX + e] = v;
    }
  }
}

// Tap values of the points (row J, elements V and V+1) as one pair (PAIR configurations).
template <class C, int J, int V, int P, int PH = 0>
struct PairFetch {
  const MarchRegs<float, C>& r;
  template <int dm, int dy, int dx>
  __device__ __forceinline__ float2 get() const {
    return make_float2(PointFetch<float, C, J, V, P, PH>{r}.template get<dm, dy, dx>(),
                       PointFetch<float, C, J, V + 1, P, PH>{r}.template get<dm, dy, dx>());
  }
};

// The coefficient set a configuration evaluates with: pairs of equal scales for PAIR.
template <typename T, class C>
using EvalCoefs = std::conditional_t<C::PAIR, Coefs<float2, C::shape::NTERMS>, Coefs<T, C::shape::NTERMS>>;

template <typename T, class C>
__device__ __forceinline__ EvalCoefs<T, C> eval_coefs(const Coefs<T, C::shape::NTERMS>& c) {
  if constexpr (C::PAIR) {
    Coefs<float2, C::shape::NTERMS> p;
#pragma unroll
    for (int g = 0; g < C::shape::NTERMS; ++g) {
      p.scale[g] = make_float2(c.scale[g], c.scale[g]);
      p.rcp[g] = make_float2(c.rcp[g], c.rcp[g]);
    }
    p.init_zero = c.init_zero;
    p.negzero = make_float2(c.negzero, c.negzero);
    return p;
  } else {
    return c;
  }
}

template <typename T, class C, int P, int PH, int J, int... Vs>
__device__ __forceinline__ void eval_row(const MarchRegs<T, C>& r, const EvalCoefs<T, C>& c, T (&res)[C::VX],
                                         std::integer_sequence<int, Vs...>) {
  if constexpr (C::PAIR) {
    static_assert(C::VX % 2 == 0, "whole pairs");
    (
        [&] {
          if constexpr (Vs % 2 == 0) {
            const float2 v = eval_shape<typename C::shape, float2>(PairFetch<C, J, Vs, P, PH>{r}, c);
            res[Vs] = v.x;
            res[Vs + 1] = v.y;
          }
        }(),
        ...);
  } else {
    ((res[Vs] = eval_shape<typename C::shape, T>(PointFetch<T, C, J, Vs, P, PH>{r}, c)), ...);
  }
}

// One row of VX outputs to `d` and, when pd != 0, also to the same position pd bytes away (a
// neighbouring GPU's ghost planes, through its peer mapping).  `interior`: the whole tile is
// inside the output and rows are 16-byte aligned (unchecked vector stores).
template <typename T, class C>
__device__ __forceinline__ void store_row(T* d, const T (&res)[C::VX], bool interior, bool row_ok, int cols_left,
                                          long long so2, long long pd) {
  using VT = typename VecN<T, C::VX>::type;
  if (interior) {
    VT q;
    T* e = reinterpret_cast<T*>(&q);
#pragma unroll
    for (int v = 0; v < C::VX; ++v) e[v] = res[v];
    *reinterpret_cast<VT*>(d) = q;
    if (pd) *reinterpret_cast<VT*>(reinterpret_cast<char*>(d) + pd) = q;
  } else if (row_ok) {
#pragma unroll
    for (int v = 0; v < C::VX; ++v)
      if (v < cols_left) {
        d[v * so2] = res[v];
        if (pd) *reinterpret_cast<T*>(reinterpret_cast<char*>(d + v * so2) + pd) = res[v];
      }
  }
}

// Interleaved paired evaluation (INTERLEAVE configurations): the thread's PY x VX/2 point
// pairs advance term by term together, so consecutive instructions belong to independent
// fold chains (each chain keeps its own exact order).
template <typename T, class C, int P, int PH, int G, int J, int... Qs>
__device__ __forceinline__ void fold_pairs_row(float2 (&a)[C::VX / 2], const MarchRegs<T, C>& r,
                                               const EvalCoefs<T, C>& c, std::integer_sequence<int, Qs...>) {
  using S = typename C::shape;
  if constexpr (G == 0) {
    ((a[Qs] = eval_term<S, 0, float2>(PairFetch<C, J, 2 * Qs, P, PH>{r}, c)), ...);
    if (c.init_zero) ((a[Qs] = add_rn(zero_of<float2>(), a[Qs])), ...);
  } else {
    ((a[Qs] = fold_term<S, G, float2>(a[Qs], PairFetch<C, J, 2 * Qs, P, PH>{r}, c)), ...);
  }
}
template <typename T, class C, int P, int PH, int G, int... Js>
__device__ __forceinline__ void fold_pairs_term(float2 (&a)[C::PY][C::VX / 2], const MarchRegs<T, C>& r,
                                                const EvalCoefs<T, C>& c, std::integer_sequence<int, Js...>) {
  (fold_pairs_row<T, C, P, PH, G, Js>(a[Js], r, c, std::make_integer_sequence<int, C::VX / 2>{}), ...);
}
template <typename T, class C, int P, int PH, int... Gs>
__device__ __forceinline__ void fold_pairs(float2 (&a)[C::PY][C::VX / 2], const MarchRegs<T, C>& r,
                                           const EvalCoefs<T, C>& c, std::integer_sequence<int, Gs...>) {
  (fold_pairs_term<T, C, P, PH, Gs>(a, r, c, std::make_integer_sequence<int, C::PY>{}), ...);
}

// Evaluate the PY x VX points of one plane step and store them.  `dst` points at the
// thread's first output of row 0 of this plane.
template <typename T, class C, int P, int PH, int... Js>
__device__ __forceinline__ void eval_store(const MarchRegs<T, C>& r, const EvalCoefs<T, C>& c,
                                           T* __restrict__ dst, long long so1, bool interior, int rows_left,
                                           int cols_left, long long so2, long long pd,
                                           std::integer_sequence<int, Js...>) {
  if constexpr (C::INTERLEAVE == 1) {
    float2 a[C::PY][C::VX / 2];
    fold_pairs<T, C, P, PH>(a, r, c, std::make_integer_sequence<int, C::shape::NTERMS>{});
    (
        [&] {
          T res[C::VX];
#pragma unroll
          for (int q = 0; q < C::VX / 2; ++q) {
            res[2 * q] = a[Js][q].x;
            res[2 * q + 1] = a[Js][q].y;
          }
          store_row<T, C>(dst + Js * so1, res, interior, Js < rows_left, cols_left, so2, pd);
        }(),
        ...);
  } else {
    (
        [&] {
          T res[C::VX];
          eval_row<T, C, P, PH, Js>(r, c, res, std::make_integer_sequence<int, C::VX>{});
          store_row<T, C>(dst + Js * so1, res, interior, Js < rows_left, cols_left, so2, pd);
        }(),
        ...);
  }
}

// Shared-memory tile of the input plane at offset REL from the group's first input plane.
template <typename T, class C, int REL>
__device__ __forceinline__ const T* stage_plane(const T* const* sb) {
  return sb[REL / C::RB] + (REL % C::RB) * C::PLANE;
}

template <typename T, class C, int P, int PH, int... Ks>
__device__ __forceinline__ void load_segments_at(MarchRegs<T, C>& r, const T* const* sb, int toff, int lane_x,
                                                 std::integer_sequence<int, Ks...>) {
  (load_segment<T, C, Ks, P, PH>(r, stage_plane<T, C, P + C::RM + C::SEGS.r[Ks].dm>(sb) + toff, 0, lane_x), ...);
}

// ---- stream mode -------------------------------------------------------------------
// Offset DM's terms for point (J, V) of accumulator slot K; START: DM = -RM, the fold begins
// (term 0, then the zero-start rule, exactly as eval_shape).
template <typename T, class C, int DM, bool START, int K, int J, int V>
__device__ __forceinline__ void stream_point(MarchRegs<T, C>& r, const EvalCoefs<T, C>& c) {
  using S = typename C::shape;
  constexpr int gb = group_begin<S>(DM), ge = group_begin<S>(DM + 1);
  if constexpr (C::PAIR) {  // points V and V + 1 in one pair (V even)
    const PairFetch<C, J, V, 0> f{r};
    float2 acc;
    if constexpr (START) {
      static_assert(gb == 0 && ge >= 1, "the fold starts with offset -RM");
      acc = eval_term<S, 0, float2>(f, c);
      if (c.init_zero) acc = add_rn(zero_of<float2>(), acc);
      acc = fold_range<S, float2, 1>(acc, f, c, std::make_integer_sequence<int, ge - 1>{});
    } else {
      acc = fold_range<S, float2, gb>(make_float2(r.acc[K][J][V], r.acc[K][J][V + 1]), f, c,
                                      std::make_integer_sequence<int, ge - gb>{});
    }
    r.acc[K][J][V] = acc.x;
    r.acc[K][J][V + 1] = acc.y;
  } else {
    const PointFetch<T, C, J, V> f{r};
    if constexpr (START) {
      static_assert(gb == 0 && ge >= 1, "the fold starts with offset -RM");
      T acc = eval_term<S, 0, T>(f, c);
      if (c.init_zero) acc = add_rn(T(0), acc);
      r.acc[K][J][V] = fold_range<S, T, 1>(acc, f, c, std::make_integer_sequence<int, ge - 1>{});
    } else {
      r.acc[K][J][V] = fold_range<S, T, gb>(r.acc[K][J][V], f, c, std::make_integer_sequence<int, ge - gb>{});
    }
  }
}

template <typename T, class C, int DM, bool START, int K, int J, int... Vs>
__device__ __forceinline__ void stream_row(MarchRegs<T, C>& r, const EvalCoefs<T, C>& c,
                                           std::integer_sequence<int, Vs...>) {
  if constexpr (C::PAIR)
    ((Vs % 2 == 0 ? stream_point<T, C, DM, START, K, J, Vs>(r, c) : void()), ...);
  else
    (stream_point<T, C, DM, START, K, J, Vs>(r, c), ...);
}

template <typename T, class C, int DM, bool START, int K, int... Js>
__device__ __forceinline__ void stream_slot(MarchRegs<T, C>& r, const EvalCoefs<T, C>& c,
                                            std::integer_sequence<int, Js...>) {
  (stream_row<T, C, DM, START, K, Js>(r, c, std::make_integer_sequence<int, C::VX>{}), ...);
}

// Steady step: the lead plane is offset RM - K of output slot K (slot 2RM starts, slot 0 ends).
template <typename T, class C, int... Ks>
__device__ __forceinline__ void stream_apply(MarchRegs<T, C>& r, const EvalCoefs<T, C>& c,
                                             std::integer_sequence<int, Ks...>) {
  (stream_slot<T, C, C::RM - Ks, Ks == 2 * C::RM, Ks>(r, c, std::make_integer_sequence<int, C::PY>{}), ...);
}

// Rows of relative input plane REL into the segment registers.
template <typename T, class C, int REL, int... Ks>
__device__ __forceinline__ void stream_rows(MarchRegs<T, C>& r, const T* const* sb, int toff, int lane_x,
                                            std::integer_sequence<int, Ks...>) {
  (load_segment<T, C, Ks>(r, stage_plane<T, C, REL>(sb) + toff, 0, lane_x), ...);
}

// Warm-up plane PL (< 2RM) of an item: it is offset PL - RM - K of output slot K <= PL.
template <typename T, class C, int PL, int... Ks>
__device__ __forceinline__ void stream_warm(MarchRegs<T, C>& r, const EvalCoefs<T, C>& c,
                                            std::integer_sequence<int, Ks...>) {
  (stream_slot<T, C, PL - C::RM - Ks, Ks == PL, Ks>(r, c, std::make_integer_sequence<int, C::PY>{}), ...);
}

template <typename T, class C, int... PLs>
__device__ __forceinline__ void stream_fill(MarchRegs<T, C>& r, const T* const* sb, int toff, int lane_x,
                                            const EvalCoefs<T, C>& c, std::integer_sequence<int, PLs...>) {
  ((stream_rows<T, C, PLs>(r, sb, toff, lane_x, std::make_integer_sequence<int, C::NSEG>{}),
    stream_warm<T, C, PLs>(r, c, std::make_integer_sequence<int, PLs + 1>{})),
   ...);
}

// Store the PY x VX completed points of slot 0 (same rules as eval_store).
template <typename T, class C, int... Js>
__device__ __forceinline__ void stream_store(const MarchRegs<T, C>& r, T* __restrict__ dst, long long so1,
                                             bool interior, int rows_left, int cols_left, long long so2, long long pd,
                                             std::integer_sequence<int, Js...>) {
  (store_row<T, C>(dst + Js * so1, r.acc[0][Js], interior, Js < rows_left, cols_left, so2, pd), ...);
}

// One plane step P (0..RB-1) of a group: window lead, segments, evaluate + store (the window
// shifts once per group, in group_steps).
template <typename T, class C, int P, int PH>
__device__ __forceinline__ void plane_step(MarchRegs<T, C>& r, const T* const* sb, int toff, int lane_x,
                                           const EvalCoefs<T, C>& coef, T* dst, long long so1,
                                           bool interior, int rows_left, int cols_left, long long so2, long long pd) {
  if constexpr (C::STREAM) {
    stream_rows<T, C, P + 2 * C::RM>(r, sb, toff, lane_x, std::make_integer_sequence<int, C::NSEG>{});
    stream_apply<T, C>(r, coef, std::make_integer_sequence<int, 2 * C::RM + 1>{});
    stream_store<T, C>(r, dst, so1, interior, rows_left, cols_left, so2, pd, std::make_integer_sequence<int, C::PY>{});
#pragma unroll
    for (int k = 0; k < 2 * C::RM; ++k)
#pragma unroll
      for (int j = 0; j < C::PY; ++j)
#pragma unroll
        for (int e = 0; e < C::VX; ++e) r.acc[k][j][e] = r.acc[k + 1][j][e];
  } else {
    if constexpr (C::WINDOW) {
      const T* pl = stage_plane<T, C, P + C::RM + C::WM>(sb) + toff;
#pragma unroll
      for (int j = 0; j < C::PY; ++j) lds_vec<T, C::VX>(pl + j * C::TXL, r.win[C::wslot(PH, P + 2 * C::WM)][j]);
    }
    if constexpr (C::NSEG > 0)
      load_segments_at<T, C, P, PH>(r, sb, toff, lane_x, std::make_integer_sequence<int, C::NSEG>{});
    eval_store<T, C, P, PH>(r, coef, dst, so1, interior, rows_left, cols_left, so2, pd,
                            std::make_integer_sequence<int, C::PY>{});
  }
}

// Term G of every point pair of every plane of a group (INTERLEAVE == 2).
template <typename T, class C, int PH, int G, int... Ps>
__device__ __forceinline__ void fold_group_term(float2 (&a)[C::RB][C::PY][C::VX / 2], const MarchRegs<T, C>& r,
                                                const EvalCoefs<T, C>& c) {
  (fold_pairs_term<T, C, Ps, PH, G>(a[Ps], r, c, std::make_integer_sequence<int, C::PY>{}), ...);
}
template <typename T, class C, int PH, int... Ps, int... Gs>
__device__ __forceinline__ void fold_group(float2 (&a)[C::RB][C::PY][C::VX / 2], const MarchRegs<T, C>& r,
                                           const EvalCoefs<T, C>& c, std::integer_sequence<int, Gs...>) {
  (fold_group_term<T, C, PH, Gs, Ps...>(a, r, c), ...);
}

// A finished item's output planes [m0, m1) of its tile, copied to the same place `delta` bytes
// away (a neighbouring GPU's ghost planes, through its peer mapping).  Called by the whole CTA
// after its stores; they are still in L2.  16-byte vectors where the rows allow.
template <typename T, class C>
__device__ __forceinline__ void peer_copy(T* out, const GridDesc& g, int x0, int y0, long long m0, long long m1,
                                          long long delta, bool vec) {
  __syncthreads();  // every thread's stores of the item are done
  const int rows = (int)(g.no[1] - y0 < C::TY ? g.no[1] - y0 : C::TY);
  const int cols = (int)(g.no[2] - x0 < C::TX ? g.no[2] - x0 : C::TX);
  if (m1 <= m0 || rows <= 0 || cols <= 0) return;
  if (vec && cols == C::TX) {
    using VT = typename VecN<T, C::VX>::type;
    constexpr int NV = C::TX / C::VX;
    const long long total = (m1 - m0) * rows * NV;
    for (long long i = threadIdx.x; i < total; i += C::THREADS) {
      const int v = int(i % NV);
      const long long r = i / NV;
      const int y = int(r % rows);
      const long long m = m0 + r / rows;
      const T* src = out + m * g.so[0] + (long long)(y0 + y) * g.so[1] + (long long)(x0 + v * C::VX) * g.so[2];
      const VT q = *reinterpret_cast<const VT*>(src);
      *reinterpret_cast<VT*>(reinterpret_cast<char*>(const_cast<T*>(src)) + delta) = q;
    }
  } else {
    const long long total = (m1 - m0) * rows * cols;
    for (long long i = threadIdx.x; i < total; i += C::THREADS) {
      const int x = int(i % cols);
      const long long r = i / cols;
      const int y = int(r % rows);
      const long long m = m0 + r / rows;
      T* src = out + m * g.so[0] + (long long)(y0 + y) * g.so[1] + (long long)(x0 + x) * g.so[2];
      *reinterpret_cast<T*>(reinterpret_cast<char*>(src) + delta) = *src;
    }
  }
}

template <typename T, class C, bool PEER, int PH, int... Ps>
__device__ __forceinline__ void group_steps(MarchRegs<T, C>& r, const T* const* sb, int toff, int lane_x,
                                            const EvalCoefs<T, C>& coef, T* dst0, long long so0,
                                            long long so1, bool interior, int rows_left, int cols_left,
                                            long long so2, const PeerStore& pe, int m0, int planes,
                                            std::integer_sequence<int, Ps...>) {
  if constexpr (C::INTERLEAVE == 2) {
    // Every plane of the group at once: leads and row segments first, then all point pairs of
    // all planes fold term by term, then the stores (planes beyond the chunk end are computed
    // from shared memory the ring holds anyway, and not stored).
    (
        [&] {
          const T* pl = stage_plane<T, C, Ps + C::RM + C::WM>(sb) + toff;
#pragma unroll
          for (int j = 0; j < C::PY; ++j) lds_vec<T, C::VX>(pl + j * C::TXL, r.win[C::wslot(PH, Ps + 2 * C::WM)][j]);
          if constexpr (C::NSEG > 0)
            load_segments_at<T, C, Ps, PH>(r, sb, toff, lane_x, std::make_integer_sequence<int, C::NSEG>{});
        }(),
        ...);
    float2 a[C::RB][C::PY][C::VX / 2];
    fold_group<T, C, PH, Ps...>(a, r, coef, std::make_integer_sequence<int, C::shape::NTERMS>{});
    (
        [&] {
          if (Ps < planes) {
            const long long pd = 0ll;
#pragma unroll
            for (int j = 0; j < C::PY; ++j) {
              T res[C::VX];
#pragma unroll
              for (int q = 0; q < C::VX / 2; ++q) {
                res[2 * q] = a[Ps][j][q].x;
                res[2 * q + 1] = a[Ps][j][q].y;
              }
              store_row<T, C>(dst0 + Ps * so0 + j * so1, res, interior, j < rows_left, cols_left, so2, pd);
            }
          }
        }(),
        ...);
  } else {
    // Planes beyond the chunk end (last group only) are skipped; the check is warp-uniform.
    ((Ps < planes ? plane_step<T, C, Ps, PH>(r, sb, toff, lane_x, coef, dst0 + Ps * so0, so1, interior, rows_left,
                                             cols_left, so2, 0ll)
                  : void()),
     ...);
  }
  if constexpr (C::WINDOW && !C::CIRC) {  // next group: its planes g0+RB-WM .. are slots RB ..
#pragma unroll
    for (int k = 0; k < 2 * C::WM; ++k)
#pragma unroll
      for (int j = 0; j < C::PY; ++j)
#pragma unroll
        for (int e = 0; e < C::VX; ++e) r.win[k][j][e] = r.win[k + C::RB][j][e];
  }
}

// The group body of window phase ph (compile-time dispatch over the PHASES bodies).
template <typename T, class C, bool PEER, int... PHs>
__device__ __forceinline__ void run_group(int ph, MarchRegs<T, C>& r, const T* const* sb, int toff, int lane_x,
                                          const EvalCoefs<T, C>& coef, T* dst0, long long so0, long long so1,
                                          bool interior, int rows_left, int cols_left, long long so2,
                                          const PeerStore& pe, int m0, int planes,
                                          std::integer_sequence<int, PHs...>) {
  ((ph == PHs ? group_steps<T, C, PEER, PHs>(r, sb, toff, lane_x, coef, dst0, so0, so1, interior, rows_left, cols_left,
                                       so2, pe, m0, planes, std::make_integer_sequence<int, C::RB>{})
              : void()),
   ...);
}

// An item that stored into a neighbour's ghost planes is done: every thread's stores are made
// visible system-wide, and the item that completes the side's count sets the neighbour's
// sequence flag (the neighbour reads it before its next pass touches those planes).  Called by
// the whole CTA.
__device__ __forceinline__ void peer_item_done(unsigned long long* done, long long items, unsigned long long* flag,
                                               unsigned long long seq) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned long long n = atomicAdd(done, 1ull) + 1ull;
    if (n == (unsigned long long)items) {
      atomicExch(done, 0ull);  // every item of this side has counted: reset for the next pass
      __threadfence_system();
      asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(flag), "l"(seq) : "memory");
    }
  }
}

// Bounded wait (about 2 s, one thread) until a neighbour's flag in this GPU's memory reaches v;
// on expiry the error word gets kErrPeerTimeout.  The proxy fence lets the TMA loads that follow
// see the planes the neighbour stored.
__device__ __forceinline__ void peer_wait(const unsigned long long* f, unsigned long long v, unsigned* err) {
  unsigned long long x;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(x) : "l"(f) : "memory");
  if (x < v) {
    const uint64_t t0 = global_ns();
    for (;;) {
      __nanosleep(128);
      asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(x) : "l"(f) : "memory");
      if (x >= v) break;
      if (global_ns() - t0 > 2000000000ull) {
        atomicOr(err, kErrPeerTimeout);
        break;
      }
    }
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// PEER: the Z-slab sweep whose boundary planes also go to the neighbouring GPUs (a.peer);
// ordinary launches are compiled without that logic.
// End of an item of a peer-store sweep: its boundary planes to the neighbours, then the item is
// counted.
template <typename T, class C>
__device__ __forceinline__ void peer_item_end(const MarchArgs* a, T* out, const int* peer_tile) {
  __syncthreads();
  const int imb = peer_tile[0], ime = peer_tile[1], ix0 = peer_tile[2], iy0 = peer_tile[3];
  const PeerStore& p = a->peer;
  if (p.flag_lo && imb < p.lo_end) {
    peer_copy<T, C>(out, a->g, ix0, iy0, imb, ime < p.lo_end ? ime : p.lo_end, p.delta_lo, a->vec_store != 0);
    peer_item_done(p.done + 0, p.items_lo, p.flag_lo, p.seq);
  }
  if (p.flag_hi && ime > p.hi_begin) {
    peer_copy<T, C>(out, a->g, ix0, iy0, imb > p.hi_begin ? imb : p.hi_begin, ime, p.delta_hi, a->vec_store != 0);
    peer_item_done(p.done + 1, p.items_hi, p.flag_hi, p.seq);
  }
}

// The PEER variant is compiled for one CTA per SM: its end-of-item work needs a few registers
// more, which a two-CTA bound of 64 would have to spill.
template <typename T, class C, bool PEER = false>
__global__ void __launch_bounds__(C::THREADS, PEER ? 1 : C::MINB)
    march_tma_kernel(const __grid_constant__ CUtensorMap tmap, T* __restrict__ out,
                     const __grid_constant__ MarchArgs a, const Coefs<T, C::shape::NTERMS> coef) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t bars[C::NS];
  __shared__ int peer_tile[5];  // PEER: item mb, me, x0, y0, first stage reaching the upper ghosts
  T* ring = reinterpret_cast<T*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));

  const int t = threadIdx.x;
  const int lane_x = t % C::LPR;
  const int rg = t / C::LPR;
  const int row0 = rg * C::PY;  // first tile row of this thread
  const bool leader = (t == 0);
  // Offset of the thread's first vector inside a plane tile.
  const int toff = (row0 + C::RY) * C::TXL + C::XC + lane_x * C::VX;
  if (leader) {
    for (int i = 0; i < C::NS; ++i) mbar_init(&bars[i], 1);
    mbar_fence_init();
  }
  __syncthreads();

  const GridDesc& g = a.g;
  unsigned q_base = 0;     // stages issued by this CTA before the current item
  int n_issued = 0;        // stages of the current item issued so far
  int n_waited = 0;        // stages of the current item waited on so far
  bool failed = false;
  MarchRegs<T, C> r;
  const EvalCoefs<T, C> ecoef = eval_coefs<T, C>(coef);

  const long long tiles = (long long)a.tiles_x * a.tiles_y;
  long long w_beg, w_end;
  if (a.balanced) {
    cta_range(a.work, blockIdx.x, gridDim.x, &w_beg, &w_end);
  } else {
    w_beg = blockIdx.x;
    w_end = a.work;
  }
  for (long long w = w_beg; w < w_end;) {
    long long tile, mb, me;
    if (a.balanced) {
      tile = w / a.nm;
      const long long seg_end = (tile + 1) * a.nm < w_end ? (tile + 1) * a.nm : w_end;
      mb = g.m_lo + (w - tile * a.nm);
      me = g.m_lo + (seg_end - tile * a.nm);
      w = seg_end;
    } else {
      long long ci, chunk = a.chunk;
      if (w < a.work1) {
        tile = w % a.tiles1;
        ci = w / a.tiles1;
      } else {  // second band
        const long long v = w - a.work1, tb = tiles - a.tiles1;
        tile = a.tiles1 + v % tb;
        ci = v / tb;
        chunk = a.chunk2;
      }
      // PEER (one band): boundary chunks first, so their planes reach the neighbours early in
      // the launch and the neighbours' next launch finds them there without waiting.
      const long long nch = a.work / tiles;
      const long long c_idx = !PEER || ci == 0 ? ci : (ci == 1 ? nch - 1 : ci - 1);
      mb = g.m_lo + c_idx * chunk;
      me = mb + chunk < g.m_hi ? mb + chunk : g.m_hi;
      if (mb >= a.gap_at) {
        mb += a.gap;
        me += a.gap;
      }
      w += gridDim.x;
    }
    const int tile_x = int(tile % a.tiles_x);
    const int tile_y = int(tile / a.tiles_x);
    const int x0 = tile_x * C::TX, y0 = tile_y * C::TY;
    const int ngroups = int((me - mb + C::RB - 1) / C::RB);
    const int qt = ngroups - 1 + C::NEED;  // stages this item loads

    // TMA coordinates of stage q: the tile's loaded window, planes L0 + q*RB ...
    const int cx = x0 + g.org[2] - C::XC;
    const int cy = y0 + g.org[1] - C::RY;
    const int L0 = int(mb + g.org[0] - C::RM);
    // Output addressing of this thread for the item.
    const int xo = x0 + lane_x * C::VX, yo = y0 + row0;
    const int rows_left = int(g.no[1] - yo);
    const int cols_left = int(g.no[2] - xo);
    const bool interior = a.vec_store && x0 + C::TX <= g.no[2] && y0 + C::TY <= g.no[1];
    T* out_item = out + mb * g.so[0] + (long long)yo * g.so[1] + (long long)xo * g.so[2];

    // Peer-store sweeps: the first stage reaching the upper ghost planes (stage pq_hi on) waits
    // for the upper neighbour, so that wait falls at the end of the item; the lower ghost planes
    // are read from the start.  The item's coordinates for its end-of-item work are parked in
    // shared memory, not kept in registers across the item.
    auto issue = [&](int q) {
      if constexpr (PEER) {
        if (q >= peer_tile[4]) {
          peer_wait(a.peer.wait_hi, a.peer.wait_value, a.err);
          peer_tile[4] = 1 << 30;
        }
      }
      const unsigned slot = (q_base + unsigned(q)) % C::NS;
      mbar_expect_tx(&bars[slot], unsigned(C::PLANE * C::RB * sizeof(T)));
      tma_load_3d(ring + size_t(slot) * C::STAGE, &tmap, &bars[slot], cx, cy, L0 + q * C::RB);
    };
    __syncthreads();  // the previous item's last group is done with the ring
    n_issued = qt < C::NS ? qt : C::NS;
    n_waited = 0;
    if (leader) {
      if constexpr (PEER) {
        peer_tile[0] = int(mb);
        peer_tile[1] = int(me);
        peer_tile[2] = x0;
        peer_tile[3] = y0;
        // stage q reaches the upper ghosts when mb - RM + (q + 1) * RB - 1 >= n
        peer_tile[4] = a.peer.wait_hi ? int(floor_div_c(int(g.no[0]) - int(mb) + C::RM - C::RB + 1 + C::RB - 1, C::RB))
                                      : (1 << 30);
      }
      if (PEER && a.peer.wait_lo && mb - C::RM < 0) peer_wait(a.peer.wait_lo, a.peer.wait_value, a.err);
      fence_proxy_async_smem();
      for (int q = 0; q < n_issued; ++q) issue(q);
    }

    for (int grp = 0; grp < ngroups; ++grp) {
      // Wait (bounded) for the stages this group reads that were not waited on yet.
      const int q_last = grp + C::NEED - 1;
      for (; n_waited <= q_last; ++n_waited) {
        const unsigned gq = q_base + unsigned(n_waited);
        if (!failed && !mbar_wait_bounded(&bars[gq % C::NS], (gq / C::NS) & 1u)) failed = true;
      }
      // CTA-uniform decision; this barrier also retires group grp-1 from every thread.
      if (__syncthreads_or(failed)) {
        failed = true;
        break;
      }
      if (grp >= 1) {
        // Stages before FIRST(grp) are retired: refill the ring up to FIRST(grp) + NS.
        const int lim = grp + C::FIRST_OFF + C::NS;
        const int target = qt < lim ? qt : lim;
        if (n_issued < target) {
          if (leader) {
            fence_proxy_async_smem();
            for (int q = n_issued; q < target; ++q) issue(q);
          }
          n_issued = target;
        }
      }
      // Stage tiles read by this group.
      const T* sb[C::NEED];
      {
        unsigned slot = (q_base + unsigned(grp)) % C::NS;
#pragma unroll
        for (int k = 0; k < C::NEED; ++k) {
          sb[k] = ring + size_t(slot) * C::STAGE;
          slot = slot + 1 == unsigned(C::NS) ? 0u : slot + 1;
        }
      }
      if constexpr (C::WINDOW) {
        if (grp == 0) {  // fill the window with planes mb-WM .. mb+WM-1
#pragma unroll
          for (int k = 0; k < 2 * C::WM; ++k) {
            const int rel = C::RM - C::WM + k;
            const T* pl = sb[rel / C::RB] + (rel % C::RB) * C::PLANE + toff;
#pragma unroll
            for (int j = 0; j < C::PY; ++j) lds_vec<T, C::VX>(pl + j * C::TXL, r.win[k][j]);
          }
        }
      }
      if constexpr (C::STREAM) {
        if (grp == 0)  // planes mb-RM .. mb+RM-1 start outputs mb .. mb+2RM-1
          stream_fill<T, C>(r, sb, toff, lane_x, ecoef, std::make_integer_sequence<int, 2 * C::RM>{});
      }
      const long long m_grp = (long long)grp * C::RB;
      const int planes = int(me - mb - m_grp);
      run_group<T, C, PEER>(grp % C::PHASES, r, sb, toff, lane_x, ecoef, out_item + m_grp * g.so[0], g.so[0], g.so[1],
                      interior, rows_left, cols_left, g.so[2], a.peer, int(mb + m_grp), planes,
                      std::make_integer_sequence<int, C::PHASES>{});
    }
    if (failed) break;
    q_base += unsigned(qt);
    if constexpr (PEER) peer_item_end<T, C>(&a, out, peer_tile);
  }

  if (failed) {
    if (leader) {
      atomicOr(a.err, kErrTmaTimeout);
      // Let copies already in flight land before the CTA's shared memory is released.
      for (int q = n_waited; q < n_issued; ++q) {
        const unsigned gq = q_base + unsigned(q);
        const uint64_t t0 = global_ns();
        while (!mbar_try_wait(&bars[gq % C::NS], (gq / C::NS) & 1u) &&
               global_ns() - t0 < 200000000ull) {
        }
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------------
// Direct kernel: any strides, one output point per thread, zero outside the input.
template <typename T>
struct GlobalFetch {
  const T* __restrict__ x;
  long long m, y, xx;  // input coordinate of the output point (before the tap)
  const GridDesc* g;
  __device__ __forceinline__ T at(int dm, int dy, int dx) const {
    const long long a = m + dm, b = y + dy, c = xx + dx;
    if (a < 0 || a >= g->n[0] || b < 0 || b >= g->n[1] || c < 0 || c >= g->n[2]) return T(0);
    return __ldg(x + a * g->s[0] + b * g->s[1] + c * g->s[2]);
  }
  template <int dm, int dy, int dx>
  __device__ __forceinline__ T get() const {
    return at(dm, dy, dx);
  }
};

template <typename T, class S>
__global__ void __launch_bounds__(256)
    direct_kernel(const T* __restrict__ x, T* __restrict__ out, const GridDesc g,
                  const Coefs<T, S::NTERMS> coef) {
  const long long nm = g.m_hi - g.m_lo;
  const long long total = nm * g.no[1] * g.no[2];
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long xo = i % g.no[2];
    const long long r = i / g.no[2];
    const long long yo = r % g.no[1];
    const long long mo = g.m_lo + r / g.no[1];
    GlobalFetch<T> f{x, mo + g.org[0], yo + g.org[1], xo + g.org[2], &g};
    out[mo * g.so[0] + yo * g.so[1] + xo * g.so[2]] = eval_shape<S, T>(f, coef);
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
    direct_table_kernel(const T* __restrict__ x, T* __restrict__ out, const GridDesc g,
                        const TableProgram* __restrict__ prog, const TableCoefs<T> coef) {
  const long long nm = g.m_hi - g.m_lo;
  const long long total = nm * g.no[1] * g.no[2];
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long xo = i % g.no[2];
    const long long r = i / g.no[2];
    const long long yo = r % g.no[1];
    const long long mo = g.m_lo + r / g.no[1];
    GlobalFetch<T> f{x, mo + g.org[0], yo + g.org[1], xo + g.org[2], &g};
    out[mo * g.so[0] + yo * g.so[1] + xo * g.so[2]] = eval_table<T>(f, *prog, coef);
  }
}

// ---------------------------------------------------------------------------------
// 1-D line kernel.  Each thread owns V = 16/sizeof(T) consecutive outputs; its input
// window is gathered from its own 16-byte vector and its neighbours' through shuffles.

template <typename T>
__device__ __forceinline__ void load_vec(const T* p, T* dst) {
  using V = typename Vec16<T>::type;
  const V q = __ldg(reinterpret_cast<const V*>(p));
  const T* e = reinterpret_cast<const T*>(&q);
#pragma unroll
  for (int i = 0; i < Vec16<T>::N; ++i) dst[i] = e[i];
}

struct LineArgs {
  long long n_in, n_out;  // input / output lengths
};

template <typename T>
struct WinFetch {
  const T* w;
  template <int dm, int dy, int dx>
  __device__ __forceinline__ T get() const {
    return w[dx];
  }
};

// Vectors per lane and warp chunk: a warp owns LINE_U * 32 consecutive output vectors and
// issues all their loads before it computes, so each thread keeps LINE_U 16-byte loads in
// flight (one was too few to cover HBM latency at full occupancy).
constexpr int LINE_U = 4;

// ORG: input index = output index + ORG + tap (0 for same-size, R for valid region).
template <typename T, class S, int ORG>
__global__ void __launch_bounds__(256)
    line_kernel(const T* __restrict__ x, T* __restrict__ y, const LineArgs a,
                const Coefs<T, S::NTERMS> coef) {
  constexpr int V = Vec16<T>::N;
  constexpr int U = LINE_U;
  constexpr int R = S::RX;
  constexpr int LW = (R + V - 1) / V;  // neighbour vectors needed on each side (org in [0, R])
  constexpr int LWR = (2 * R + V - 1) / V;
  constexpr int W = V * (1 + LW + LWR);   // window elements, window[0] = x[i0 - LW*V]
  const int lane = threadIdx.x & 31;
  const long long nvec_out = (a.n_out + V - 1) / V;
  // Warp chunks of U*32 vectors, warp-strided over the grid; all lanes of a warp iterate
  // together (shuffles), so the loop bound is warp-uniform.
  const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long ch = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; ch * U * 32 < nvec_out;
       ch += nwarps) {
    // Own vectors of the input: x[i0 .. i0+V) (aligned: x base 16-byte aligned, i0 % V == 0).
    T own[U][V];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const long long i0 = ((ch * U + u) * 32 + lane) * V;
      if (i0 + V <= a.n_in) {
        load_vec<T>(x + i0, own[u]);
      } else {
#pragma unroll
        for (int j = 0; j < V; ++j) own[u][j] = (i0 + j < a.n_in) ? x[i0 + j] : T(0);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const long long v_idx = (ch * U + u) * 32 + lane;  // this lane's output vector
      const long long i0 = v_idx * V;                    // first output index
      T win[W];
#pragma unroll
      for (int j = 0; j < V; ++j) win[LW * V + j] = own[u][j];
      // Neighbour vectors at lane offsets -LW..-1 and +1..+LWR; lanes past the warp's edge
      // read them from memory (cached: the warp's own neighbouring loads).
#pragma unroll
      for (int l = -LW; l <= LWR; ++l) {
        if (l == 0) continue;
        const int src = lane + l;
        T nb[V];
#pragma unroll
        for (int j = 0; j < V; ++j) nb[j] = __shfl_sync(0xffffffffu, own[u][j], src & 31);
        if (src < 0 || src > 31) {
          const long long b = i0 + (long long)l * V;
          if (b >= 0 && b + V <= a.n_in) {
            load_vec<T>(x + b, nb);
          } else {
#pragma unroll
            for (int j = 0; j < V; ++j) nb[j] = (b + j >= 0 && b + j < a.n_in) ? x[b + j] : T(0);
          }
        }
#pragma unroll
        for (int j = 0; j < V; ++j) win[(LW + l) * V + j] = nb[j];
      }
      if (v_idx < nvec_out) {
        T res[V];
#pragma unroll
        for (int j = 0; j < V; ++j) {
          // Window index of input (output index + ORG) for this output; taps add dx.
          WinFetch<T> f{win + LW * V + j + ORG};
          res[j] = eval_shape<S, T>(f, coef);
        }
        if (i0 + V <= a.n_out) {
          using VT = typename Vec16<T>::type;
          VT q;
          T* e = reinterpret_cast<T*>(&q);
#pragma unroll
          for (int j = 0; j < V; ++j) e[j] = res[j];
          *reinterpret_cast<VT*>(y + i0) = q;
        } else {
#pragma unroll
          for (int j = 0; j < V; ++j)
            if (i0 + j < a.n_out) y[i0 + j] = res[j];
        }
      }
    }
  }
}

}  // namespace bst
