// bst_noalloc.cu — bst_stencil_apply_noalloc: one stencil sweep that allocates nothing.
//
// Why it exists: some callers cannot allocate GPU memory while they run a sweep — code
// that must not enter the CUDA allocator (a real-time or embedded loop with a fixed memory
// budget, a host framework that owns every device byte through its own pool, a caller that
// must never block on cudaMalloc's implicit synchronisation).  The general entry point runs
// programs outside the compiled shape catalog through a runtime-table kernel whose table
// lives in a device buffer it allocates per call.  This variant keeps that table in a
// file-scope device array instead, so a call allocates no device memory and makes no
// allocating CUDA or library call.
//
// Limits and sharing:
//  * the table (taps, term descriptors and scales) must fit in kNoAllocTableBytes (32 KiB);
//    larger programs are rejected with BST_ERR_UNSUPPORTED and a message giving both sizes;
//  * every call, on every stream, writes the same array: two calls whose copies and kernels
//    overlap on the GPU race (use one stream, or order the calls).  Each call rewrites the
//    whole header and every entry the kernel reads, so nothing left by an earlier call is used;
//  * the first call on a device looks up the array's device address (cudaGetSymbolAddress)
//    with that device current; that first call should come before any stream capture begins.
// Every GPU that loads the library holds the 32 KiB array until the process exits.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "bst_internal.h"
#include "bst_kernels.cuh"

namespace bst {

int sm_count();  // bst_core.cu

constexpr int kNoAllocTableBytes = 32 * 1024;

// The only scratch memory of this entry point.
static __device__ __align__(256) unsigned char g_noalloc_table[kNoAllocTableBytes];

// Packed table layout (byte offsets, all from the array's start):
//   0                     int32 ntaps, nterms, init_zero, (unused)
//   16                    int16 tap[ntaps][3]                   (logical M, Y, X offsets)
//   tf = align4(..)       int16 term_first[nterms], int16 term_count[nterms]
//   to = tf + 4*nterms    uint8 term_op[nterms]
//   sc = align8(..)       T     scale[nterms]
struct NoAllocLayout {
  int taps, term_first, term_count, term_op, scale, bytes;
};

__host__ __device__ inline NoAllocLayout noalloc_layout(int ntaps, int nterms, int elem) {
  NoAllocLayout L;
  L.taps = 16;
  L.term_first = (L.taps + 6 * ntaps + 3) & ~3;
  L.term_count = L.term_first + 2 * nterms;
  L.term_op = L.term_count + 2 * nterms;
  L.scale = (L.term_op + nterms + 7) & ~7;
  L.bytes = L.scale + elem * nterms;
  return L;
}

template <typename T>
__global__ void __launch_bounds__(256)
    direct_table_noalloc_kernel(const T* __restrict__ x, T* __restrict__ out, const GridDesc g,
                                const unsigned char* __restrict__ table) {
  const int* hdr = reinterpret_cast<const int*>(table);
  const int ntaps = hdr[0], nterms = hdr[1], init_zero = hdr[2];
  const NoAllocLayout L = noalloc_layout(ntaps, nterms, int(sizeof(T)));
  const short* tap = reinterpret_cast<const short*>(table + L.taps);
  const short* tfirst = reinterpret_cast<const short*>(table + L.term_first);
  const short* tcount = reinterpret_cast<const short*>(table + L.term_count);
  const unsigned char* top = table + L.term_op;
  const T* scale = reinterpret_cast<const T*>(table + L.scale);
  const long long nm = g.m_hi - g.m_lo;
  const long long total = nm * g.no[1] * g.no[2];
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long xo = i % g.no[2];
    const long long r = i / g.no[2];
    const long long yo = r % g.no[1];
    const long long mo = g.m_lo + r / g.no[1];
    GlobalFetch<T> f{x, mo + g.org[0], yo + g.org[1], xo + g.org[2], &g};
    // Same fold as every other kernel: terms left to right, taps left to right.
    T acc = T(0);
    for (int t = 0; t < nterms; ++t) {
      const int first = tfirst[t];
      T s = f.at(tap[3 * first], tap[3 * first + 1], tap[3 * first + 2]);
      for (int k = 1; k < tcount[t]; ++k) {
        const int q = first + k;
        s = add_rn(s, f.at(tap[3 * q], tap[3 * q + 1], tap[3 * q + 2]));
      }
      const T v = apply_op<T>(top[t], scale[t], s);
      acc = t == 0 ? (init_zero ? add_rn(T(0), v) : v) : add_rn(acc, v);
    }
    out[mo * g.so[0] + yo * g.so[1] + xo * g.so[2]] = acc;
  }
}

// Device address of g_noalloc_table per device, looked up once with that device current.
static int noalloc_table_ptr(unsigned char** out) {
  static std::mutex mu;
  static unsigned char* ptrs[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(BST_ERR_UNSUPPORTED, "device index beyond 63");
  std::lock_guard<std::mutex> lk(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_table);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_table)");
    ptrs[dev] = static_cast<unsigned char*>(p);
  }
  *out = ptrs[dev];
  return BST_OK;
}

// Validate the program and pack it into `buf` (logical [M, Y, X] taps, centred for
// valid-region programs) without touching the heap.  Fills the launch geometry.
template <typename T>
static int noalloc_pack(const bst_program* p, int ndim, const int64_t* shape, unsigned char* buf, int* bytes,
                        GridDesc* g) {
  if (p->ndim != ndim) return fail(BST_ERR_INVALID, "program ndim does not match the grid");
  if (p->ntaps < 1 || p->ntaps > BST_MAX_TAPS) return fail(BST_ERR_INVALID, "ntaps out of range");
  if (p->nterms < 1 || p->nterms > BST_MAX_TERMS) return fail(BST_ERR_INVALID, "nterms out of range");
  if (p->boundary != BST_BOUNDARY_ZERO && p->boundary != BST_BOUNDARY_VALID)
    return fail(BST_ERR_INVALID, "unknown boundary mode");
  const NoAllocLayout L = noalloc_layout(p->ntaps, p->nterms, int(sizeof(T)));
  if (L.bytes > kNoAllocTableBytes)
    return fail(BST_ERR_UNSUPPORTED, "program table needs " + std::to_string(L.bytes) +
                                         " bytes; the allocation-free entry point holds at most " +
                                         std::to_string(kNoAllocTableBytes));
  int next = 0;
  for (int t = 0; t < p->nterms; ++t) {
    if (p->term_first[t] != next || p->term_count[t] < 1)
      return fail(BST_ERR_INVALID, "terms must partition the taps in order");
    if (p->term_op[t] < BST_TERM_SUM || p->term_op[t] > BST_TERM_DIV)
      return fail(BST_ERR_INVALID, "unknown term operator");
    next += p->term_count[t];
  }
  if (next != p->ntaps) return fail(BST_ERR_INVALID, "terms must cover every tap");
  // Logical axes [M, Y, X] of a 1-, 2- or 3-D grid (1-D: X only; 2-D: M and X).
  const int axis_of[3][3] = {{2, -1, -1}, {0, 2, -1}, {0, 1, 2}};
  int64_t n[3] = {1, 1, 1}, no[3] = {1, 1, 1};
  for (int a = 0; a < ndim; ++a) {
    n[axis_of[ndim - 1][a]] = shape[a];
    no[axis_of[ndim - 1][a]] = p->boundary == BST_BOUNDARY_VALID ? p->out_shape[a] : shape[a];
  }
  int lo[3] = {0, 0, 0}, hi[3] = {0, 0, 0};  // per logical axis: min / max tap offset
  for (int i = 0; i < p->ntaps; ++i)
    for (int a = 0; a < 3; ++a) {
      const int v = p->tap[i][a];
      if (a >= ndim && v != 0) return fail(BST_ERR_INVALID, "tap offset on an axis beyond ndim");
      if (v < -64 || v > 64) return fail(BST_ERR_UNSUPPORTED, "tap offset beyond +-64");
      if (a < ndim) {
        const int la = axis_of[ndim - 1][a];
        lo[la] = (i == 0 || v < lo[la]) ? v : lo[la];
        hi[la] = (i == 0 || v > hi[la]) ? v : hi[la];
      }
    }
  int org[3] = {0, 0, 0};
  if (p->boundary == BST_BOUNDARY_VALID) {
    for (int a = 0; a < 3; ++a) {
      if (no[a] <= 0) return fail(BST_ERR_INVALID, "valid-region output extent must be positive");
      const bool used = (a == 2) || (a == 0 && ndim >= 2) || (a == 1 && ndim == 3);
      if (!used) continue;
      if (lo[a] < 0 || no[a] - 1 + hi[a] > n[a] - 1) return fail(BST_ERR_INVALID, "valid-region taps read outside the input");
      const int s = lo[a] + hi[a];
      org[a] = s >= 0 ? s / 2 : -((-s + 1) / 2);
    }
  }
  int32_t* hdr = reinterpret_cast<int32_t*>(buf);
  hdr[0] = p->ntaps;
  hdr[1] = p->nterms;
  hdr[2] = p->init_zero ? 1 : 0;
  hdr[3] = 0;
  int16_t* tap = reinterpret_cast<int16_t*>(buf + L.taps);
  for (int i = 0; i < p->ntaps; ++i) {
    int16_t lt[3] = {0, 0, 0};
    for (int a = 0; a < ndim; ++a) {
      const int la = axis_of[ndim - 1][a];
      lt[la] = int16_t(p->tap[i][a] - org[la]);
    }
    tap[3 * i] = lt[0];
    tap[3 * i + 1] = lt[1];
    tap[3 * i + 2] = lt[2];
  }
  int16_t* tf = reinterpret_cast<int16_t*>(buf + L.term_first);
  int16_t* tc = reinterpret_cast<int16_t*>(buf + L.term_count);
  unsigned char* top = buf + L.term_op;
  T* sc = reinterpret_cast<T*>(buf + L.scale);
  for (int t = 0; t < p->nterms; ++t) {
    tf[t] = int16_t(p->term_first[t]);
    tc[t] = int16_t(p->term_count[t]);
    top[t] = (unsigned char)p->term_op[t];
    sc[t] = T(p->term_scale[t]);
  }
  *bytes = L.bytes;
  for (int a = 0; a < 3; ++a) {
    g->n[a] = n[a];
    g->no[a] = no[a];
    g->org[a] = org[a];
  }
  g->m_lo = 0;
  g->m_hi = no[0];
  return BST_OK;
}

template <typename T>
static int noalloc_apply(const bst_program* prog, int ndim, const int64_t* shape, const int64_t* xs_t, const void* x,
                         const int64_t* ys_t, void* y, cudaStream_t st) {
  alignas(16) unsigned char buf[kNoAllocTableBytes];  // host staging on the stack
  GridDesc g{};
  int bytes = 0;
  int rc = noalloc_pack<T>(prog, ndim, shape, buf, &bytes, &g);
  if (rc) return rc;
  int64_t xs[3], ys[3];
  logical_strides(ndim, xs_t, xs);
  logical_strides(ndim, ys_t, ys);
  for (int a = 0; a < 3; ++a) {
    g.s[a] = xs[a];
    g.so[a] = ys[a];
  }
  unsigned char* table = nullptr;
  rc = noalloc_table_ptr(&table);
  if (rc) return rc;
  // Pageable source: the call returns once the bytes are staged, and the copy is ordered
  // before the kernel on the same stream.
  cudaError_t e = cudaMemcpyAsync(table, buf, size_t(bytes), cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync to the stencil table array");
  const long long total = g.no[0] * g.no[1] * g.no[2];
  long long blocks = (total + 255) / 256;
  const long long cap = (long long)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  direct_table_noalloc_kernel<T><<<unsigned(blocks), 256, 0, st>>>(static_cast<const T*>(x), static_cast<T*>(y), g,
                                                                    table);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "direct_table_noalloc_kernel launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return BST_OK;
}

}  // namespace bst

using namespace bst;

extern "C" int bst_stencil_apply_noalloc(const bst_program* prog, int32_t dtype, int32_t ndim, const int64_t* shape,
                                         const int64_t* x_strides, const void* x, const int64_t* y_strides, void* y,
                                         void* stream) {
  clear_error();
  if (!shape || !prog) return fail(BST_ERR_INVALID, "null shape or program");
  if (dtype != BST_F32 && dtype != BST_F64) return fail(BST_ERR_UNSUPPORTED, "dtype must be float32 or float64");
  if (ndim < 1 || ndim > 3) return fail(BST_ERR_INVALID, "only 1-D, 2-D and 3-D grids are supported");
  if (prog->ndim != ndim) return fail(BST_ERR_INVALID, "program ndim does not match the grid");
  if (prog->flags != 0) return fail(BST_ERR_UNSUPPORTED, "program flags (fused multiply-add) are not supported here");
  int64_t oshape[3] = {0, 0, 0};
  for (int i = 0; i < ndim; ++i) {
    if (shape[i] < 0) return fail(BST_ERR_INVALID, "negative extent");
    oshape[i] = prog->boundary == BST_BOUNDARY_VALID ? prog->out_shape[i] : shape[i];
    if (shape[i] == 0 || oshape[i] == 0) return BST_OK;  // empty grid: nothing to do
  }
  if (!x || !y) return fail(BST_ERR_INVALID, "null device pointer");
  int64_t xs_t[3], ys_t[3];
  int64_t s = 1, so = 1;
  for (int i = ndim - 1; i >= 0; --i) {
    xs_t[i] = x_strides ? x_strides[i] : s;
    ys_t[i] = y_strides ? y_strides[i] : so;
    s *= shape[i];
    so *= oshape[i];
  }
  // The sweep is out of place: input and output must not overlap.
  const int64_t es = dtype == BST_F64 ? 8 : 4;
  int64_t xlo = 0, xhi = 0, ylo = 0, yhi = 0;
  for (int i = 0; i < ndim; ++i) {
    const int64_t ex = (shape[i] - 1) * xs_t[i], ey = (oshape[i] - 1) * ys_t[i];
    (ex < 0 ? xlo : xhi) += ex;
    (ey < 0 ? ylo : yhi) += ey;
  }
  const char* xb = static_cast<const char*>(x) + xlo * es;
  const char* yb = static_cast<const char*>(y) + ylo * es;
  if (xb < yb + (yhi - ylo + 1) * es && yb < xb + (xhi - xlo + 1) * es)
    return fail(BST_ERR_INVALID, "input and output overlap");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == BST_F32) return noalloc_apply<float>(prog, ndim, shape, xs_t, x, ys_t, y, st);
  return noalloc_apply<double>(prog, ndim, shape, xs_t, x, ys_t, y, st);
}
