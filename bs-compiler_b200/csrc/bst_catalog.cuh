// bst_catalog.cuh — the compiled shape catalog and the per-dtype dispatcher.
//
// A request is matched against the catalog by its canonical tap/term structure.  A
// match runs that shape's specialised kernel (TMA march for 2-D/3-D when the layout
// meets TMA's 16-byte rules, the vector line kernel for 1-D, else the direct kernel);
// anything else runs the runtime-table direct kernel.  Every path computes the same
// operations in the same order, so the choice never changes a result bit.
#pragma once
#include "bst_launch.cuh"

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
#define BST_HEAT_TY 16
#endif
#ifndef BST_HEAT_PY
#define BST_HEAT_PY 4
#endif
#ifndef BST_HEAT_NSX
#define BST_HEAT_NSX 3
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
#define BST_STAR_TY 16
#endif
#ifndef BST_STAR_PY
#define BST_STAR_PY 2
#endif
#ifndef BST_STAR_NSX
#define BST_STAR_NSX 4
#endif
template <typename T>
constexpr int kRowCols = 32 * (16 / int(sizeof(T)));
template <typename T, class S>
using Cfg2D = MarchCfg<T, S, kRowCols<T>, 1, 1, BST_2D_RB, BST_2D_NSX>;
template <typename T, class S, int TY, int PY, int NSX>
using Cfg3D = MarchCfg<T, S, kRowCols<T>, TY, PY, 1, NSX>;
template <typename T, class S>
using CfgHeat = Cfg3D<T, S, BST_HEAT_TY, BST_HEAT_PY, BST_HEAT_NSX>;
template <typename T, class S>
using CfgBox = Cfg3D<T, S, BST_BOX_TY, BST_BOX_PY, BST_BOX_NSX>;
template <typename T, class S>
using CfgStar = Cfg3D<T, S, BST_STAR_TY, BST_STAR_PY, BST_STAR_NSX>;

template <typename T>
int dispatch_sweep(const LaunchReq& r) {
  const Canon& c = *r.c;
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
  if (shape_matches<Box<1, 7, false>>(c)) return run_march_or_direct<T, CfgBox<T, Box<1, 7, false>>>(r);
  if (shape_matches<StarPair3D<4>>(c)) return run_march_or_direct<T, CfgStar<T, StarPair3D<4>>>(r);
  if (shape_matches<WStar7>(c)) return run_march_or_direct<T, CfgHeat<T, WStar7>>(r);
  if (shape_matches<Box<2, 7, false>>(c)) return run_march_or_direct<T, Cfg3D<T, Box<2, 7, false>, 4, 1, 2>>(r);
  if (shape_matches<Box<1, 7, true>>(c)) return run_march_or_direct<T, CfgBox<T, Box<1, 7, true>>>(r);
  return launch_direct_table<T>(r);
}

}  // namespace bst
