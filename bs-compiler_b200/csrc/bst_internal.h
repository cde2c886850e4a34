// bst_internal.h — host-side internals shared by the C-ABI translation units.
#pragma once
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <string>
#include <vector>

#include "../../include/basalto_b200.h"
#include "bst_types.cuh"

namespace bst {

// ---- error reporting --------------------------------------------------------------
void set_error(const std::string& msg);
void clear_error();
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);
#define BST_CUDA(call)                                  \
  do {                                                  \
    cudaError_t e_ = (call);                            \
    if (e_ != cudaSuccess) return ::bst::cuda_fail(e_, #call); \
  } while (0)

extern std::atomic<uint64_t> g_launches;

// ---- canonical program in logical [M, Y, X] space ----------------------------------
struct Canon {
  int ndim = 0;
  int boundary = BST_BOUNDARY_ZERO;
  int init_zero = 0;
  int contract = 0;  // BST_PROGRAM_CONTRACT
  int ntaps = 0, nterms = 0;
  std::vector<Tap> taps;       // centred offsets (input = output + org + tap)
  std::vector<Term> terms;
  std::vector<double> scale;
  int R[3] = {0, 0, 0};    // per logical axis: max |tap|
  int org[3] = {0, 0, 0};  // output -> input origin shift
  int64_t n[3] = {1, 1, 1};   // input extents
  int64_t no[3] = {1, 1, 1};  // output extents
};

// Validate `p` against an input of `shape` (ndim entries) and fill `c`.
int canonicalize(const bst_program* p, int ndim, const int64_t* shape, Canon* c);

// Logical strides [M, Y, X] from torch-order strides (elements).
void logical_strides(int ndim, const int64_t* strides, int64_t out[3]);

// Launch one sweep.  x/y strides are logical [M,Y,X]; m range is in output planes.  `peer`:
// also store every output into a neighbouring GPU's memory (TMA march kernels only).
// [m2_lo, m2_hi): a second range of output planes (the upper slab boundary rows), in the same
// launch where the kernel allows (TMA march, ranges of equal length), else a second launch.
int launch_sweep(const Canon& c, int dtype, const void* x, const int64_t xs[3], void* y,
                 const int64_t ys[3], int64_t m_lo, int64_t m_hi, cudaStream_t st,
                 const PeerStore* peer = nullptr, int64_t m2_lo = 0, int64_t m2_hi = 0);

// Temporal blocking.  tb_max_sweeps: most sweeps one launch can fuse for this request
// (1 = no fused kernel).  launch_fused: k sweeps of output planes [m_lo, m_hi) in one launch
// (k == 1 is launch_sweep); intermediate values of planes outside [row_lo, row_hi) (output
// coordinates) are forced to zero, as a single sweep reads zeros outside the grid.
// capability: the kernel's limit; otherwise the default (fusing only where it is faster).
int tb_max_sweeps(const Canon& c, int dtype, const void* x, const int64_t xs[3], void* y, const int64_t ys[3],
                  bool capability = false);
int launch_fused(const Canon& c, int dtype, const void* x, const int64_t xs[3], void* y, const int64_t ys[3],
                 int k, int64_t m_lo, int64_t m_hi, int64_t row_lo, int64_t row_hi, cudaStream_t st);
// Sweeps per launch for nsteps ping-pong sweeps, at most kmax per launch, with a launch
// count of the same parity as nsteps (so the result lands where a per-sweep ping-pong would).
std::vector<int> fuse_plan(int nsteps, int kmax);

// Work schedule of the march kernel (MarchArgs).  BST_MARCH_SCHEDULE = items | lockstep |
// balanced selects one for tuning runs; the default is the measured best.
enum class Schedule { kItems, kLockstep, kBalanced };
Schedule march_schedule();

// Device copies of runtime-table programs, uploaded once per device and shared by every later
// call that carries the same table bytes: the repeat path makes no allocation, no copy and no
// host synchronisation.  A miss allocates and copies synchronously (once per program); the
// entries live until the process exits, at most kTableCacheMax per device.  Returns nullptr
// when the cache is full or the upload failed (the caller then uploads for one call).
constexpr int kTableCacheMax = 256;
const void* cached_device_table(const void* blob, size_t bytes);

// vendor ("nvidia") and driver (the NVRM version field of /proc/driver/nvidia/version, as
// crates/basalto-common/src/hardware.rs:154-159 reads it; "unknown" without it).
void fill_driver_string(bst_device_caps* c);

// Device error word (kernels OR bits into it); allocated once per device.
unsigned* device_error_word();
// Reads and clears the calling device's error word (synchronizes the stream).
int check_device_error(cudaStream_t st);

}  // namespace bst
