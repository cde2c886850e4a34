// bst_shapes.cuh — compile-time stencil shapes and the exact-order evaluator.
//
// A shape fixes the tap offsets, the grouping of taps into terms and each term's
// operator at compile time; the scales (coefficients) stay runtime values.  The
// evaluator folds terms and taps strictly left to right with separately rounded
// operations, so a shape written in the order of an eager-torch expression reproduces
// that expression bit for bit.  Offsets are in logical [M, Y, X] space (see
// bst_types.cuh: a 2-D [y, x] tap (a, b) is (a, 0, b) here, a 1-D tap (a) is (0, 0, a)).
#pragma once
#include <type_traits>
#include <utility>
#include "bst_types.cuh"

namespace bst {

template <int NT, int NG>
struct ShapeTable {
  Tap taps[NT];
  Term terms[NG];
};

constexpr int cabs(int v) { return v < 0 ? -v : v; }
constexpr int cmax(int a, int b) { return a > b ? a : b; }
constexpr int ipow(int b, int e) { return e == 0 ? 1 : b * ipow(b, e - 1); }

template <int NT, int NG>
constexpr int radius_of(const ShapeTable<NT, NG>& t, int axis) {
  int r = 0;
  for (int i = 0; i < NT; ++i) {
    int v = axis == 0 ? t.taps[i].dm : (axis == 1 ? t.taps[i].dy : t.taps[i].dx);
    r = cmax(r, cabs(v));
  }
  return r;
}

// Base that derives radii and counts from a table.
template <class Derived, int NT, int NG>
struct ShapeBase {
  static constexpr int NTAPS = NT;
  static constexpr int NTERMS = NG;
};

// The same shape evaluated with BST_PROGRAM_CONTRACT: every multiplied term after the first
// folds as one fused multiply-add, acc = fma(scale, sum, acc).  Plain shapes round every
// operation separately.
template <class S>
struct Contracted : S {
  static constexpr bool CONTRACT = true;
};
template <class S, class = void>
struct contract_of : std::false_type {};
template <class S>
struct contract_of<S, std::void_t<decltype(S::CONTRACT)>> : std::bool_constant<S::CONTRACT> {};

#define BST_SHAPE_RADII(NAME)                               \
  static constexpr int RM = radius_of(NAME::tbl, 0);        \
  static constexpr int RY = radius_of(NAME::tbl, 1);        \
  static constexpr int RX = radius_of(NAME::tbl, 2);

// ---------------------------------------------------------------------------------
// 2-D five-point Jacobi, Dirichlet-0:  0.25 * (u[y-1] + u[y+1] + u[x-1] + u[x+1])
struct Jacobi2D : ShapeBase<Jacobi2D, 4, 1> {
  static constexpr ShapeTable<4, 1> tbl = {
      {{-1, 0, 0}, {1, 0, 0}, {0, 0, -1}, {0, 0, 1}},
      {{0, 4, kMul}}};
  BST_SHAPE_RADII(Jacobi2D)
};

// 3-D seven-point heat step:  c0 * u + c1 * (u[z-1]+u[z+1]+u[y-1]+u[y+1]+u[x-1]+u[x+1])
struct Heat3D : ShapeBase<Heat3D, 7, 2> {
  static constexpr ShapeTable<7, 2> tbl = {
      {{0, 0, 0}, {-1, 0, 0}, {1, 0, 0}, {0, -1, 0}, {0, 1, 0}, {0, 0, -1}, {0, 0, 1}},
      {{0, 1, kMul}, {1, 6, kMul}}};
  BST_SHAPE_RADII(Heat3D)
};

// 3-D seven-point with one weight per tap (c*u + w*u[z-1] + ...), tap order
// centre, z-1, z+1, y-1, y+1, x-1, x+1 (the reference's report stencils).
struct WStar7 : ShapeBase<WStar7, 7, 7> {
  static constexpr ShapeTable<7, 7> tbl = {
      {{0, 0, 0}, {-1, 0, 0}, {1, 0, 0}, {0, -1, 0}, {0, 1, 0}, {0, 0, -1}, {0, 0, 1}},
      {{0, 1, kMul}, {1, 1, kMul}, {2, 1, kMul}, {3, 1, kMul}, {4, 1, kMul}, {5, 1, kMul},
       {6, 1, kMul}}};
  BST_SHAPE_RADII(WStar7)
};

// Box of radius R over the axes in AXES (bit 0 = X, 1 = Y, 2 = M), one weighted term
// per tap, offsets ascending slowest-axis-major (DESC: the reverse order, as a
// roll-based accumulation produces).
template <int R, int AXES, bool DESC>
constexpr auto make_box() {
  constexpr int nm = (AXES & 4) ? 2 * R + 1 : 1;
  constexpr int ny = (AXES & 2) ? 2 * R + 1 : 1;
  constexpr int nx = (AXES & 1) ? 2 * R + 1 : 1;
  constexpr int N = nm * ny * nx;
  ShapeTable<N, N> t{};
  int k = 0;
  for (int a = 0; a < nm; ++a)
    for (int b = 0; b < ny; ++b)
      for (int c = 0; c < nx; ++c) {
        int idx = DESC ? (N - 1 - k) : k;
        t.taps[idx] = Tap{(AXES & 4) ? a - R : 0, (AXES & 2) ? b - R : 0, (AXES & 1) ? c - R : 0};
        t.terms[idx] = Term{idx, 1, kMul};
        ++k;
      }
  return t;
}

template <int R, int AXES, bool DESC>
struct Box {
  static constexpr auto tbl = make_box<R, AXES, DESC>();
  static constexpr int NTAPS = sizeof(tbl.taps) / sizeof(Tap);
  static constexpr int NTERMS = sizeof(tbl.terms) / sizeof(Term);
  BST_SHAPE_RADII(Box)
};

// Star of radius R in 3-D: c0*u, then for k = 1..R and axis M, Y, X in turn
// c_k * (u[+k] + u[-k]).  (Addition is commutative, so the pair order is immaterial.)
template <int R>
constexpr auto make_star3() {
  ShapeTable<1 + 6 * R, 1 + 3 * R> t{};
  t.taps[0] = Tap{0, 0, 0};
  t.terms[0] = Term{0, 1, kMul};
  int tp = 1, tm = 1;
  for (int k = 1; k <= R; ++k)
    for (int ax = 0; ax < 3; ++ax) {
      t.taps[tp] = Tap{ax == 0 ? k : 0, ax == 1 ? k : 0, ax == 2 ? k : 0};
      t.taps[tp + 1] = Tap{ax == 0 ? -k : 0, ax == 1 ? -k : 0, ax == 2 ? -k : 0};
      t.terms[tm] = Term{tp, 2, kMul};
      tp += 2;
      ++tm;
    }
  return t;
}
template <int R>
struct StarPair3D {
  static constexpr auto tbl = make_star3<R>();
  static constexpr int NTAPS = 1 + 6 * R;
  static constexpr int NTERMS = 1 + 3 * R;
  BST_SHAPE_RADII(StarPair3D)
};

// 1-D three-point mean (x[i-1] + x[i] + x[i+1]) / c, the reference README example.
struct Mean3Line {
  static constexpr ShapeTable<3, 1> tbl = {{{0, 0, -1}, {0, 0, 0}, {0, 0, 1}}, {{0, 3, kDiv}}};
  static constexpr int NTAPS = 3, NTERMS = 1;
  BST_SHAPE_RADII(Mean3Line)
};

#undef BST_SHAPE_RADII

// ---------------------------------------------------------------------------------
// Exact-order evaluation.  F provides `template <int dm, int dy, int dx> T get() const`.
template <class S, int G, class T, class F, int... Ks>
__device__ __forceinline__ T term_sum(const F& f, std::integer_sequence<int, Ks...>) {
  constexpr Tap t0 = S::tbl.taps[S::tbl.terms[G].first];
  T s = f.template get<t0.dm, t0.dy, t0.dx>();
  ((s = add_rn(s, f.template get<S::tbl.taps[S::tbl.terms[G].first + Ks + 1].dm,
                                 S::tbl.taps[S::tbl.terms[G].first + Ks + 1].dy,
                                 S::tbl.taps[S::tbl.terms[G].first + Ks + 1].dx>())),
   ...);
  return s;
}

template <class S, int G, class T, class F>
__device__ __forceinline__ T eval_term(const F& f, const Coefs<T, S::NTERMS>& c) {
  constexpr int cnt = S::tbl.terms[G].count;
  T s = term_sum<S, G, T>(f, std::make_integer_sequence<int, cnt - 1>{});
  constexpr int op = S::tbl.terms[G].op;
  if constexpr (op == kMul) return product_rn(c.scale[G], s, c.negzero);
  else if constexpr (op == kDiv) return div_by(s, c.scale[G], c.rcp[G]);
  else return s;
}

// acc + term G: separately rounded, or (contracted shapes, multiplied terms) one fma.
template <class S, int G, class T, class F>
__device__ __forceinline__ T fold_term(T acc, const F& f, const Coefs<T, S::NTERMS>& c) {
  if constexpr (contract_of<S>::value && S::tbl.terms[G].op == kMul) {
    constexpr int cnt = S::tbl.terms[G].count;
    return fma_rn(c.scale[G], term_sum<S, G, T>(f, std::make_integer_sequence<int, cnt - 1>{}), acc);
  } else {
    return add_rn(acc, eval_term<S, G, T>(f, c));
  }
}

template <class S, class T, class F, int... Gs>
__device__ __forceinline__ T fold_terms(T acc, const F& f, const Coefs<T, S::NTERMS>& c,
                                        std::integer_sequence<int, Gs...>) {
  ((acc = fold_term<S, Gs + 1, T>(acc, f, c)), ...);
  return acc;
}

// Terms G0 .. G0 + sizeof(Is) - 1 folded into acc (continuing a fold).
template <class S, class T, int G0, class F, int... Is>
__device__ __forceinline__ T fold_range(T acc, const F& f, const Coefs<T, S::NTERMS>& c,
                                        std::integer_sequence<int, Is...>) {
  ((acc = fold_term<S, G0 + Is, T>(acc, f, c)), ...);
  return acc;
}

template <class S, class T, class F>
__device__ __forceinline__ T eval_shape(const F& f, const Coefs<T, S::NTERMS>& c) {
  T acc = eval_term<S, 0, T>(f, c);
  if (c.init_zero) acc = add_rn(zero_of<T>(), acc);
  return fold_terms<S, T>(acc, f, c, std::make_integer_sequence<int, S::NTERMS - 1>{});
}

// Runtime-table evaluation (generic programs).  F provides `T at(int dm, int dy, int dx)`.
template <class T, class F>
__device__ __forceinline__ T eval_table(const F& f, const TableProgram& p, const TableCoefs<T>& c) {
  T acc = T(0);
  for (int g = 0; g < p.nterms; ++g) {
    const int first = p.term_first[g];
    T s = f.at(p.tap[first][0], p.tap[first][1], p.tap[first][2]);
    for (int k = 1; k < p.term_count[g]; ++k)
      s = add_rn(s, f.at(p.tap[first + k][0], p.tap[first + k][1], p.tap[first + k][2]));
    if (g > 0 && c.contract && p.term_op[g] == kMul) {
      acc = fma_rn(c.scale[g], s, acc);
      continue;
    }
    const T t = apply_op<T>(p.term_op[g], c.scale[g], s);
    if (g == 0) acc = c.init_zero ? add_rn(T(0), t) : t;
    else acc = add_rn(acc, t);
  }
  return acc;
}

}  // namespace bst
