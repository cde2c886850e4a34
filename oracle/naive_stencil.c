/*
 * naive_stencil.c — C restatement of the reference's CPU stencil check.  TEST
 * INFRASTRUCTURE ONLY: loaded by tests/ (and bench.py's CPU-baseline leg) as the checker,
 * never by the product path.
 *
 * oracle_naive_box_f64 follows Executor::naive_stencil_cpu
 * (crates/basalto-tree/src/executor.rs:207-289): a same-size zero-padded box of radius r,
 * coefficient index running slowest-axis-major over offsets -r..r, accumulated in double as
 * `sum = 0.0; sum += val * coeff`.  One deliberate difference: the reference indexes as if
 * shape[0] were the fastest axis (executor.rs:227-283); here the grid is C-contiguous, as
 * torch hands it over, with shape[0] the slowest axis.
 *
 * oracle_program_{f32,f64} evaluate the generic program semantics (a left fold of terms,
 * each an optional scale applied to a left-to-right sum of taps) point by point in the
 * element type.  Build with -ffp-contract=off so no multiply-add is fused implicitly.
 * With `contract` set, every later multiplied term is folded as one fused multiply-add,
 * acc = fma(scale, sum, acc) (C99 fma: one rounding), which is how the reference's GPU
 * kernel accumulates `acc += x * c` once LLVM's NVPTX backend contracts it
 * (crates/basalto-core/src/ir/stencil_3d.rs:232-294, flir_builder.rs:118-149).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define OP_SUM 0
#define OP_MUL 1
#define OP_DIV 2

void oracle_naive_box_f64(const double* in, double* out, int ndim, const int64_t* shape, int radius,
                          const double* coeffs) {
  int64_t n[3] = {1, 1, 1};
  /* pad the shape to 3 axes on the slow side */
  for (int a = 0; a < ndim; ++a) n[3 - ndim + a] = shape[a];
  const int w = 2 * radius + 1;
  const int rz = ndim >= 3 ? radius : 0, ry = ndim >= 2 ? radius : 0, rx = radius;
  for (int64_t z = 0; z < n[0]; ++z)
    for (int64_t y = 0; y < n[1]; ++y)
      for (int64_t x = 0; x < n[2]; ++x) {
        double sum = 0.0;
        int idx = 0;
        for (int dz = -rz; dz <= rz; ++dz)
          for (int dy = -ry; dy <= ry; ++dy)
            for (int dx = -rx; dx <= rx; ++dx) {
              const int64_t iz = z + dz, iy = y + dy, ix = x + dx;
              double val = 0.0;
              if (!(iz < 0 || iz >= n[0] || iy < 0 || iy >= n[1] || ix < 0 || ix >= n[2]))
                val = in[(iz * n[1] + iy) * n[2] + ix];
              sum += val * coeffs[idx];
              idx++;
            }
        out[(z * n[1] + y) * n[2] + x] = sum;
      }
  (void)w;
}

#define DEFINE_PROGRAM(T, SUFFIX, FMA)                                                              \
  void oracle_program_##SUFFIX(const T* in, T* out, int ndim, const int64_t* shape, int boundary,  \
                               const int64_t* out_shape, int init_zero, int nterms, const int* op,  \
                               const double* scale, const int* count, const int* taps,              \
                               int contract) {                                                      \
    int64_t n[3] = {1, 1, 1}, no[3] = {1, 1, 1};                                                    \
    for (int a = 0; a < ndim; ++a) {                                                                \
      n[3 - ndim + a] = shape[a];                                                                   \
      no[3 - ndim + a] = boundary ? out_shape[a] : shape[a];                                        \
    }                                                                                               \
    for (int64_t z = 0; z < no[0]; ++z)                                                             \
      for (int64_t y = 0; y < no[1]; ++y)                                                           \
        for (int64_t x = 0; x < no[2]; ++x) {                                                       \
          T acc = (T)0;                                                                             \
          int k = 0;                                                                                \
          for (int g = 0; g < nterms; ++g) {                                                        \
            T s = (T)0;                                                                             \
            for (int j = 0; j < count[g]; ++j, ++k) {                                               \
              int64_t o[3] = {0, 0, 0};                                                             \
              for (int a = 0; a < ndim; ++a) o[3 - ndim + a] = taps[3 * k + a];                     \
              const int64_t iz = z + o[0], iy = y + o[1], ix = x + o[2];                            \
              T v = (T)0;                                                                           \
              if (!(iz < 0 || iz >= n[0] || iy < 0 || iy >= n[1] || ix < 0 || ix >= n[2]))          \
                v = in[(iz * n[1] + iy) * n[2] + ix];                                               \
              s = j == 0 ? v : (T)(s + v);                                                          \
            }                                                                                       \
            const T c = (T)scale[g];                                                                \
            const T t = op[g] == OP_MUL ? (T)(c * s) : (op[g] == OP_DIV ? (T)(s / c) : s);          \
            if (g == 0) acc = init_zero ? (T)((T)0 + t) : t;                                        \
            else if (contract && op[g] == OP_MUL) acc = FMA(c, s, acc);                             \
            else acc = (T)(acc + t);                                                                \
          }                                                                                         \
          out[(z * no[1] + y) * no[2] + x] = acc;                                                   \
        }                                                                                           \
  }

DEFINE_PROGRAM(float, f32, fmaf)
DEFINE_PROGRAM(double, f64, fma)
