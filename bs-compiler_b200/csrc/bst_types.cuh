// bst_types.cuh — shared device/host types for the stencil kernels.
//
// A grid is addressed as three logical axes [M, Y, X] (slowest to fastest):
//   1-D input [n]        -> [1, 1, n]
//   2-D input [ny, nx]   -> [ny, 1, nx]   (the row axis is the marching axis M)
//   3-D input [nz,ny,nx] -> [nz, ny, nx]  (Z is the marching axis M)
// so one kernel family covers 2-D and 3-D; tap offsets are remapped the same way.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace bst {

constexpr int kMaxTaps = 2304;
constexpr int kMaxTerms = 2304;

enum TermOp : int { kSum = 0, kMul = 1, kDiv = 2 };

struct Tap {
  int dm, dy, dx;
};
struct Term {
  int first, count, op;
};

// Geometry of one launch.  Input coordinate of a tap = output coordinate + org + tap.
struct GridDesc {
  int64_t n[3];      // input extents [M, Y, X]
  int64_t s[3];      // input strides (elements)
  int64_t no[3];     // output extents
  int64_t so[3];     // output strides (elements)
  int32_t org[3];    // output->input origin shift
  int32_t pad;
  int64_t m_lo, m_hi;  // output M range computed by this launch
};

// A Z-slab sweep whose boundary planes also go to the neighbouring GPUs (peer stores).
// Output planes [0, lo_end) are stored a second time delta_lo bytes away (the lower
// neighbour's upper ghost planes, through its peer mapping) and planes [hi_begin, n) delta_hi
// bytes away (the upper neighbour's lower ghost planes).  Before an item reads planes below 0
// (above n) it waits until *wait_lo (*wait_hi) >= wait_value: the neighbour's previous pass
// has stored them here and has finished reading the ghost planes this pass stores into.  When
// every item that stores to a side is done, the last one sets that neighbour's flag
// (*flag_lo / *flag_hi) to seq.  done[0] / done[1] count those items (zeroed; the last one
// resets its counter); items_lo / items_hi are their numbers, from the launcher's work plan.
struct PeerStore {
  long long delta_lo, delta_hi;
  int lo_end, hi_begin;  // output planes (a slab has < 2^31 planes)
  const unsigned long long* wait_lo;
  const unsigned long long* wait_hi;
  unsigned long long wait_value;
  unsigned long long* done;
  unsigned long long* flag_lo;
  unsigned long long* flag_hi;
  unsigned long long seq;
  long long items_lo, items_hi;
};

// Runtime scalars of a program (compile-time structure lives in the shape type);
// passed by value, sized exactly to the shape's term count.
template <typename T, int N>
struct Coefs {
  T scale[N];
  int init_zero;
  T negzero;  // -0.0, passed from the host so the compiler cannot fold it (product_rn)
};

// Runtime-table program for the generic kernels (lives in device memory).
struct TableProgram {
  int ntaps, nterms, init_zero, pad;
  short tap[kMaxTaps][3];
  short term_first[kMaxTerms], term_count[kMaxTerms];
  unsigned char term_op[kMaxTerms];
};
// Scales of a runtime-table program (device memory, element type T).
template <typename T>
struct TableCoefs {
  const T* scale;
  int init_zero;
  int contract;  // BST_PROGRAM_CONTRACT
};

// ---- correctly rounded scalar arithmetic, never contracted into FMA -------------
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ double add_rn(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ double mul_rn(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ float div_rn(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ double div_rn(double a, double b) { return __ddiv_rn(a, b); }
// a * b + c with one rounding (used only for BST_PROGRAM_CONTRACT programs).
__device__ __forceinline__ float fma_rn(float a, float b, float c) { return __fmaf_rn(a, b, c); }
__device__ __forceinline__ double fma_rn(double a, double b, double c) { return __fma_rn(a, b, c); }

// Two fp32 lanes per instruction (sm_100 paired add/fma .f32x2).  One paired add or fma rounds
// each component exactly as the scalar __fadd_rn / __fmaf_rn (checked on B200 over 2^24
// components, special values included).  A paired multiply, however, is fused by the compiler
// into a following paired add even when written with an explicit rounding mode, so products
// are formed as fma(a, b, -0.0) instead (product_rn): that is exactly round(a*b) for every
// input (a*b + (-0) == a*b, and +0 + -0 == +0), and an fma result cannot be fused further.
// The -0.0 arrives as a kernel argument, so the compiler cannot fold the fma back into a
// multiply.  There is no paired divide: its components divide separately.
__device__ __forceinline__ float2 add_rn(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 div_rn(float2 a, float2 b) {
  return make_float2(__fdiv_rn(a.x, b.x), __fdiv_rn(a.y, b.y));
}
__device__ __forceinline__ float2 fma_rn(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// scale * s rounded once and kept apart from any later addition.
__device__ __forceinline__ float product_rn(float a, float b, float) { return mul_rn(a, b); }
__device__ __forceinline__ double product_rn(double a, double b, double) { return mul_rn(a, b); }
__device__ __forceinline__ float2 product_rn(float2 a, float2 b, float2 negzero) { return __ffma2_rn(a, b, negzero); }

template <typename T>
__device__ __forceinline__ T zero_of() {
  return T(0);
}
template <>
__device__ __forceinline__ float2 zero_of<float2>() {
  return make_float2(0.f, 0.f);
}

template <typename T>
__device__ __forceinline__ T apply_op(int op, T scale, T s) {
  // torch: `c * t` and `t * c` are the same IEEE product; `t / c` is IEEE division.
  return op == kMul ? mul_rn(scale, s) : (op == kDiv ? div_rn(s, scale) : s);
}

}  // namespace bst
