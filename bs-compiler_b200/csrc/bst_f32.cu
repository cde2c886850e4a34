// bst_f32.cu — float32 instantiations of the shape catalog.
#include "bst_catalog.cuh"

namespace bst {
int dispatch_f32(const Canon& c, const void* x, const int64_t xs[3], void* y, const int64_t ys[3],
                 int64_t m_lo, int64_t m_hi, cudaStream_t st, const PeerStore* peer, int64_t m2_lo, int64_t m2_hi) {
  LaunchReq r{&c, x, {xs[0], xs[1], xs[2]}, y, {ys[0], ys[1], ys[2]}, m_lo, m_hi, st};
  r.peer = peer;
  r.m2_lo = m2_lo;
  r.m2_hi = m2_hi;
  return dispatch_sweep<float>(r);
}
int tb_max_f32(const Canon& c, const void* x, const int64_t xs[3], void* y, const int64_t ys[3], bool capability) {
  LaunchReq r{&c, x, {xs[0], xs[1], xs[2]}, y, {ys[0], ys[1], ys[2]}, 0, c.no[0], nullptr};
  return tb_max_sweeps<float>(r, capability);
}
int dispatch_tb_f32(const Canon& c, const void* x, const int64_t xs[3], void* y, const int64_t ys[3], int k,
                    int64_t m_lo, int64_t m_hi, int64_t row_lo, int64_t row_hi, cudaStream_t st) {
  LaunchReq r{&c, x, {xs[0], xs[1], xs[2]}, y, {ys[0], ys[1], ys[2]}, m_lo, m_hi, st, row_lo, row_hi};
  return dispatch_tb<float>(r, k);
}
}  // namespace bst
