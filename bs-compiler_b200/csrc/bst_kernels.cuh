// bst_kernels.cuh — the sm_100a stencil kernels.
//
//  * march_tma_kernel : 2-D/3-D sweep.  Each CTA owns a TX x TY tile of one M-chunk and
//    marches along M.  Input planes arrive by TMA (cp.async.bulk.tensor, no multicast)
//    into a ring of NS shared-memory stages of RB planes each, completion tracked by one
//    mbarrier per stage; TMA's out-of-bounds zero fill supplies the Dirichlet-0 ghost
//    cells, so the interior and the boundary run the same code.  Taps are read from the
//    ring at compile-time offsets; the result is stored with coalesced global stores.
//    Persistent: the grid is sized to the SM count and CTAs stride over work items.
//  * line_kernel      : 1-D sweep with 128-bit vector loads/stores and warp shuffles for
//    the neighbour elements held by adjacent lanes.
//  * direct_kernel    : any layout/stride (the fallback when TMA's 16-byte rules are not
//    met): one thread per output point, taps read through the read-only cache.
// Every kernel increments nothing and allocates nothing; waits on mbarriers are bounded
// and report through an error word instead of trapping.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include "bst_shapes.cuh"

namespace bst {

// Error word bits written by kernels (host reads them back on request).
enum : unsigned { kErrTmaTimeout = 1u };

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
// March kernel configuration (compile time).
template <typename T, class S, int TX_, int TY_, int NTY_, int RB_, int NSX_, int XC_>
struct MarchCfg {
  using shape = S;
  static constexpr int TX = TX_;    // output columns per tile (= threads in x)
  static constexpr int TY = TY_;    // output rows per tile
  static constexpr int NTY = NTY_;  // thread rows
  static constexpr int RB = RB_;    // planes per stage (power of two)
  static constexpr int RM = S::RM, RY = S::RY, RX = S::RX;
  static constexpr int V16 = 16 / int(sizeof(T));  // elements per 16 bytes
  static constexpr int XC = XC_;                   // tile column of output x0
  static constexpr int TXL = round_up_c(XC + TX + RX, V16);  // loaded columns (<= 256)
  static constexpr int TYL = TY + 2 * RY;                     // loaded rows
  static constexpr int PLANE = TXL * TYL;                     // elements per plane tile
  static constexpr int STAGE_BYTES = round_up_c(PLANE * RB * int(sizeof(T)), 128);
  static constexpr int STAGE = STAGE_BYTES / int(sizeof(T));
  static constexpr int NEED = 1 + (RB - 1 + 2 * RM) / RB;  // stages one group reads
  static constexpr int NS = NEED + NSX_;                   // ring depth (NSX = prefetch)
  static constexpr int THREADS = TX * NTY;
  static constexpr int ROWS = RB * TY;                // (plane,row) pairs per group
  static constexpr int PER_THREAD = ROWS / NTY;       // points per thread per group
  static constexpr int SMEM = NS * STAGE_BYTES + 128; // + alignment slack
  static_assert(TXL <= 256 && TYL <= 256 && RB <= 256, "TMA box extent");
  static_assert(ROWS % NTY == 0, "thread rows must divide the group");
  static_assert(XC >= RX, "halo column");
  static_assert((RB & (RB - 1)) == 0, "RB power of two");
};

struct MarchArgs {
  GridDesc g;
  int tiles_x, tiles_y, chunk, n_chunks;
  long long n_items;
  unsigned* err;
};

template <typename T, int RM, int TXL>
struct RingFetch {
  const T* pl[2 * RM + 1];
  int off;
  template <int dm, int dy, int dx>
  __device__ __forceinline__ T get() const {
    return pl[dm + RM][off + dy * TXL + dx];
  }
};

template <typename T, class C>
__global__ void __launch_bounds__(C::THREADS)
    march_tma_kernel(const __grid_constant__ CUtensorMap tmap, T* __restrict__ out,
                     const MarchArgs a, const Coefs<T, C::shape::NTERMS> coef) {
  using S = typename C::shape;
  extern __shared__ unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t bars[C::NS];
  T* ring = reinterpret_cast<T*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));

  const int tx = threadIdx.x, ty = threadIdx.y;
  const bool leader = (tx == 0 && ty == 0);
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

  for (long long item = blockIdx.x; item < a.n_items; item += gridDim.x) {
    const int tile_x = int(item % a.tiles_x);
    const long long rest = item / a.tiles_x;
    const int tile_y = int(rest % a.tiles_y);
    const int chunk = int(rest / a.tiles_y);
    const int x0 = tile_x * C::TX, y0 = tile_y * C::TY;
    const long long mb = g.m_lo + (long long)chunk * a.chunk;
    const long long me = (mb + a.chunk < g.m_hi) ? mb + a.chunk : g.m_hi;
    const int ngroups = int((me - mb + C::RB - 1) / C::RB);
    const int qt = ngroups - 1 + C::NEED;  // stages this item loads

    // TMA coordinates of stage q: the tile's loaded window, planes L0 + q*RB ...
    const int cx = x0 + g.org[2] - C::XC;
    const int cy = y0 + g.org[1] - C::RY;
    const int L0 = int(mb + g.org[0] - C::RM);

    auto issue = [&](int q) {
      const unsigned slot = (q_base + unsigned(q)) % C::NS;
      mbar_expect_tx(&bars[slot], unsigned(C::PLANE * C::RB * sizeof(T)));
      tma_load_3d(ring + size_t(slot) * C::STAGE, &tmap, &bars[slot], cx, cy, L0 + q * C::RB);
    };
    __syncthreads();  // the previous item's last group is done with the ring
    n_issued = qt < C::NS ? qt : C::NS;
    n_waited = 0;
    if (leader) {
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
      if (grp >= 1 && grp - 1 + C::NS < qt) {
        if (leader) {
          fence_proxy_async_smem();
          issue(grp - 1 + C::NS);
        }
        ++n_issued;
      }

      const long long m_grp = mb + (long long)grp * C::RB;
#pragma unroll
      for (int k = 0; k < C::PER_THREAD; ++k) {
        const int w = ty + k * C::NTY;
        const int p = w / C::TY;
        const int yl = w % C::TY;
        const long long mo = m_grp + p;
        const int yo = y0 + yl, xo = x0 + tx;
        RingFetch<T, C::RM, C::TXL> f;
#pragma unroll
        for (int d = 0; d < 2 * C::RM + 1; ++d) {
          const int rel = grp * C::RB + p + d;  // input plane relative to L0
          const unsigned slot = (q_base + unsigned(rel / C::RB)) % C::NS;
          f.pl[d] = ring + size_t(slot) * C::STAGE + size_t(rel % C::RB) * C::PLANE;
        }
        f.off = (yl + C::RY) * C::TXL + C::XC + tx;
        const T v = eval_shape<S, T>(f, coef);
        if (mo < me && yo < g.no[1] && xo < g.no[2])
          out[mo * g.so[0] + (long long)yo * g.so[1] + (long long)xo * g.so[2]] = v;
      }
    }
    if (failed) break;
    q_base += unsigned(qt);
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

template <typename T, int N>
struct VecRegs {
  T v[N];
};

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

// ORG: input index = output index + ORG + tap (0 for same-size, R for valid region).
template <typename T, class S, int ORG>
__global__ void __launch_bounds__(256)
    line_kernel(const T* __restrict__ x, T* __restrict__ y, const LineArgs a,
                const Coefs<T, S::NTERMS> coef) {
  constexpr int V = Vec16<T>::N;
  constexpr int R = S::RX;
  constexpr int LW = (R + V - 1) / V;  // neighbour vectors needed on each side (org in [0, R])
  constexpr int LWR = (2 * R + V - 1) / V;
  constexpr int W = V * (1 + LW + LWR);   // window elements, window[0] = x[i0 - LW*V]
  const int lane = threadIdx.x & 31;
  const long long nvec_out = (a.n_out + V - 1) / V;
  const long long stride = (long long)gridDim.x * blockDim.x;
  // All lanes of a warp iterate together (shuffles), so loop to a warp-uniform bound.
  const long long base = blockIdx.x * (long long)blockDim.x + (threadIdx.x & ~31);
  for (long long wv = base; wv < nvec_out; wv += stride) {
    const long long v_idx = wv + lane;  // this lane's output vector
    const long long i0 = v_idx * V;     // first output index
    T win[W];
    // Own vector of the input: x[i0 .. i0+V) (aligned: x base 16-byte aligned, i0 % V == 0).
    T own[V];
    const bool own_full = (i0 + V <= a.n_in);
    if (own_full) {
      load_vec<T>(x + i0, own);
    } else {
#pragma unroll
      for (int j = 0; j < V; ++j) own[j] = (i0 + j < a.n_in) ? x[i0 + j] : T(0);
    }
#pragma unroll
    for (int j = 0; j < V; ++j) win[LW * V + j] = own[j];
    // Neighbour vectors at lane offsets -LW..-1 and +1..+LWR.
#pragma unroll
    for (int l = -LW; l <= LWR; ++l) {
      if (l == 0) continue;
      const int src = lane + l;
      T nb[V];
#pragma unroll
      for (int j = 0; j < V; ++j) nb[j] = __shfl_sync(0xffffffffu, own[j], src & 31);
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
    if (v_idx >= nvec_out) continue;
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

}  // namespace bst
