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
  T rcp[N];   // fp32 division terms: RN(1 / scale) for div_by, 0 where the divisor is out of its range
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
// Correctly rounded x / d for an fp32 divisor fixed per launch, from y = RN(1/d) (host IEEE
// division), by two quotient corrections (P. Markstein, "Computation of elementary functions
// on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990; the correction theorem
// as proved in Cornea, Golliver and Markstein, ARITH-14, 1999):
//  * q0 = RN(x y) lies within 1.5 ulp of x/d, and q0 + r0 y, with r0 = RN(x - q0 d), differs
//    from x/d by (q0 - x/d)(1 - d y) plus r0's rounding, a few 2^-24 ulp, so q1 = RN(q0 + r0 y)
//    is a faithful (within 1 ulp) quotient;
//  * for a faithful q1 the remainder r1 = x - q1 d is exact in an fma, and with y within half an
//    ulp of 1/d the theorem gives RN(q1 + r1 y) = RN(x / d).
// Nothing under- or overflows while |x| and |d| lie in [2^-60, 2^60]; the host passes y = 0 for
// other divisors and other x (zeros, subnormals, infinities, NaN) take IEEE division.
__device__ __forceinline__ float div_by(float x, float d, float y) {
  const float ax = fabsf(x);
  if (y != 0.f && ax >= 0x1p-60f && ax <= 0x1p60f) {
    const float q0 = __fmul_rn(x, y);
    const float r0 = __fmaf_rn(-q0, d, x);
    const float q1 = __fmaf_rn(r0, y, q0);
    const float r1 = __fmaf_rn(-q1, d, x);
    return __fmaf_rn(r1, y, q1);
  }
  return __fdiv_rn(x, d);
}
__device__ __forceinline__ double div_by(double x, double d, double) { return __ddiv_rn(x, d); }
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
__device__ __forceinline__ float2 div_by(float2 a, float2 b, float2 y) {
  return make_float2(div_by(a.x, b.x, y.x), div_by(a.y, b.y, y.y));
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
