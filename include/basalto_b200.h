/*
 * basalto_b200.h — C ABI of the B200-native Basalto stencil hot path.
 *
 * Plain C: pointers, sizes and status codes only; no torch or C++ types cross this
 * boundary.  Device pointers are raw CUDA device addresses in the caller's current
 * context (the primary context, as torch uses); `stream` is a cudaStream_t passed
 * as void* (NULL = the legacy default stream).  All entry points return a
 * bst_status; on failure bst_last_error() gives a per-thread message.
 *
 * Layout convention: shapes and strides are given in torch order (shape[0] is the
 * slowest axis of a C-contiguous tensor), strides in ELEMENTS, as the reference's
 * Python layer passes them (python/basalto/compiler.py:79,82).
 *
 * Each declaration names the reference interface it replaces (paths relative to the
 * reference project root).
 */
#ifndef BASALTO_B200_H
#define BASALTO_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BST_ABI_VERSION 1

#if defined(__GNUC__)
#define BST_API __attribute__((visibility("default")))
#else
#define BST_API
#endif

/* ---- status codes -------------------------------------------------------------- */
typedef enum bst_status {
  BST_OK = 0,
  BST_ERR_INVALID = 1,      /* bad argument: rank, shape/strides mismatch, null pointer */
  BST_ERR_UNSUPPORTED = 2,  /* well-formed request outside what this build implements */
  BST_ERR_CUDA = 3,         /* a CUDA runtime/driver call failed */
  BST_ERR_NCCL = 4,         /* an NCCL call failed or NCCL could not be loaded */
  BST_ERR_TIMEOUT = 5,      /* a bounded host-side wait ran out (NCCL bootstrap / exchange) */
  BST_ERR_NO_DEVICE = 6     /* no CUDA device visible */
} bst_status;

/* ---- element types ------------------------------------------------------------- */
typedef enum bst_dtype { BST_F32 = 0, BST_F64 = 1 } bst_dtype;

/* ---- stencil program ("grouped linear stencil") ---------------------------------
 * out(p) = fold+( term_0, term_1, ..., term_{nterms-1} )       left fold: ((t0+t1)+t2)+...
 *          (with init_zero: ((0 + t0) + t1) + ..., as `torch.zeros_like(x); y += ...`)
 * term_g = scale_g (op) ( x(p+o_a) + x(p+o_b) + ... )            taps term_first..+term_count-1,
 *                                                                summed left to right
 * op: BST_TERM_SUM (no scale), BST_TERM_MUL (scale*sum), BST_TERM_DIV (sum/scale).
 * Every add/mul/div is rounded separately in the element type (IEEE RN, no FMA), so a
 * program written in the same order as an eager-torch expression reproduces it bit for bit.
 *
 * boundary BST_BOUNDARY_ZERO : output shape == input shape; reads outside the grid are 0
 *                              (Dirichlet-0 ghosts; crates/basalto-core/src/ir/common.rs:49-63,
 *                              crates/basalto-tree/src/executor.rs:222,240-244,270-277).
 * boundary BST_BOUNDARY_VALID: output shape = out_shape (taps are relative to the output
 *                              index and must stay inside the input; slice-style stencils).
 * Tap offsets are given per axis in shape order (axis 0 = slowest).
 * The reference's per-call FLIR module (crates/basalto-core/src/flir_builder.rs:24-90:
 * radius, coeffs, tiles, strides) is replaced by this descriptor. */
#define BST_MAX_TAPS 2304   /* >= 13^3: the 3-D box of radius 6 ("order_12") */
#define BST_MAX_TERMS 2304
enum { BST_TERM_SUM = 0, BST_TERM_MUL = 1, BST_TERM_DIV = 2 };
enum { BST_BOUNDARY_ZERO = 0, BST_BOUNDARY_VALID = 1 };
/* BST_PROGRAM_CONTRACT: fold every multiplied term after the first as one fused multiply-add,
 * acc = fma(scale, sum, acc) — the arithmetic of the reference's GPU kernel, whose
 * `acc += x * c` (crates/basalto-core/src/ir/stencil_3d.rs:232-294) LLVM's NVPTX backend
 * contracts into fma.  Without it (default) results are bit-identical to eager torch; with
 * it they differ from eager torch by rounding only (one rounding per term instead of two)
 * and are bit-identical to a C fma() restatement.  Not accepted by
 * bst_stencil_apply_noalloc. */
enum { BST_PROGRAM_CONTRACT = 1 };

typedef struct bst_program {
  int32_t ndim;       /* 1..3 */
  int32_t ntaps;      /* 1..BST_MAX_TAPS */
  int32_t nterms;     /* 1..BST_MAX_TERMS */
  int32_t init_zero;  /* 1: fold starts from +0.0 */
  int32_t boundary;   /* BST_BOUNDARY_* */
  int32_t flags;      /* BST_PROGRAM_* bits; 0 = every operation rounded separately */
  int64_t out_shape[3];                 /* VALID only: output extents (shape order) */
  int32_t tap[BST_MAX_TAPS][3];         /* offsets, shape order; unused axes 0 */
  int32_t term_first[BST_MAX_TERMS];
  int32_t term_count[BST_MAX_TERMS];
  int32_t term_op[BST_MAX_TERMS];
  double term_scale[BST_MAX_TERMS];     /* rounded to the element type before use */
} bst_program;

/* ---- library ------------------------------------------------------------------- */
BST_API int bst_abi_version(void);
/* Last error message of the calling thread ("" when none). */
BST_API const char* bst_last_error(void);
/* Number of kernels this library has launched in this process (all devices). */
BST_API uint64_t bst_launch_count(void);
/* Synchronizes `stream`, then reads and clears the current device's kernel error word:
 * BST_ERR_TIMEOUT if a kernel gave up a bounded wait (a TMA stage that never landed) since
 * the last check.  No reference counterpart (the reference's launch has no device-side
 * waits; crates/basalto-target-nvidia/src/runtime.rs:161-194 only checks cuLaunchKernel). */
BST_API int bst_device_error_check(void* stream);

/* Build the program the reference generates for op "stencil[_r<k>|order_8|order_12]":
 * a (2r+1)^ndim zero-padded box with isotropic weights 1/(2r+1)^ndim (or `coeffs`, in
 * slowest-axis-major order), accumulated from 0 in ascending offset order.
 * Replaces crates/basalto-core/src/flir_builder.rs:58-65 (coefficients) together with
 * the generators' tap order crates/basalto-core/src/ir/stencil_{1d,2d,3d}.rs
 * (stencil_3d.rs:236-294) and the CPU check crates/basalto-tree/src/executor.rs:207-289. */
BST_API int bst_program_box(int32_t ndim, int32_t radius, const double* coeffs, int64_t ncoeffs,
                    bst_program* out);

/* Radius encoded in an op name: "_r<k>" -> k, "order_8" -> 4, "order_12" -> 6, else 1.
 * Replaces crates/basalto-tree/src/interceptor.rs:196-205 (extract_radius). */
BST_API int32_t bst_extract_radius(const char* op);

/* One sweep y = S(x) on the current device.  shape/strides: ndim entries (strides in
 * elements; NULL = C-contiguous).  For BST_BOUNDARY_VALID the output shape is
 * prog->out_shape.  x and y must not overlap.
 * Replaces the stencil path of crates/basalto-tree/src/interceptor.rs:316-491 ->
 * crates/basalto-tree/src/executor.rs:586-707 (execute_flir_kernel) ->
 * crates/basalto-target-nvidia/src/runtime.rs:161-194,235-250 (module load + launch). */
BST_API int bst_stencil_apply(const bst_program* prog, int32_t dtype, int32_t ndim, const int64_t* shape,
                      const int64_t* x_strides, const void* x, const int64_t* y_strides, void* y,
                      void* stream);

/* One sweep y = S(x), same arguments and result as bst_stencil_apply, for callers that
 * cannot allocate GPU memory during the call (a fixed-budget real-time loop, a host
 * framework that owns every device byte through its own pool, code that must not hit
 * cudaMalloc's implicit synchronisation).  No counterpart in the reference.
 * It always runs the runtime-table kernel, with the program table in a fixed 32 KiB device
 * array compiled into the library instead of a per-call device buffer: it makes no
 * cudaMalloc/cudaFree or other allocating call.  Programs whose packed table (16 + 6*ntaps
 * + 5*nterms + elem*nterms bytes, aligned) exceeds 32 KiB return BST_ERR_UNSUPPORTED.
 * The array is shared by every call on the device: calls whose work overlaps on the GPU
 * (different streams, unordered) race; each call rewrites all the table it uses.  The first
 * call on a device looks up the array's device address (set-up); make that first call before
 * any stream capture begins. */
BST_API int bst_stencil_apply_noalloc(const bst_program* prog, int32_t dtype, int32_t ndim,
                                      const int64_t* shape, const int64_t* x_strides, const void* x,
                                      const int64_t* y_strides, void* y, void* stream);

/* nsteps sweeps ping-ponging between two C-contiguous same-shape buffers (ZERO boundary
 * programs only): step 1 reads a and writes b, step 2 reads b and writes a, ...; the
 * result is in b when nsteps is odd, in a when even.  The reference runs one sweep per
 * Python call (report/scripts/multi_gpu_halo.py:74-78); this is the same loop without
 * the per-step host round trip. */
BST_API int bst_stencil_sweeps(const bst_program* prog, int32_t dtype, int32_t ndim, const int64_t* shape,
                       void* a, void* b, int32_t nsteps, void* stream);

/* bst_stencil_sweeps with a caller-chosen limit of sweeps per launch: max_fused = 0 is the
 * library's choice (bst_stencil_sweeps: fuse only where a fused launch is faster), k > 0 fuses
 * up to k sweeps wherever a temporally blocked kernel exists — including the 3-D seven-point
 * heat step, whose kernel is bit-identical to single sweeps but measured slower than them on
 * B200 (it is offered for callers that are bound by HBM traffic elsewhere, e.g. sharing it).
 * Same ping-pong contract as bst_stencil_sweeps.  No reference counterpart (the reference runs
 * one sweep per call). */
BST_API int bst_stencil_sweeps_fused(const bst_program* prog, int32_t dtype, int32_t ndim, const int64_t* shape,
                                     void* a, void* b, int32_t nsteps, int32_t max_fused, void* stream);

/* ---- device identity (crates/basalto-common/src/hardware.rs:8-16,19-57,70-86) ---- */
typedef struct bst_device_caps {
  int32_t compute_capability_major;
  int32_t compute_capability_minor;
  int32_t max_threads_per_block;
  uint64_t max_shared_memory_per_block;
  int32_t max_registers_per_block;
  int32_t warp_size;
  int32_t multi_processor_count;
  char name[96];
  char vendor[16];     /* "nvidia" */
  char arch[16];       /* "sm_100" */
  char driver[32];     /* NVRM version from /proc/driver/nvidia/version, else "unknown" */
  int32_t driver_version;  /* cudaDriverGetVersion */
} bst_device_caps;
BST_API int bst_device_caps_query(int32_t device, bst_device_caps* out);

/* ---- kernel/plan cache key (crates/basalto-core/src/hasher.rs:53-128) ------------
 * Fixed-width little-endian serialization of op[32], dtype[16], shape (u64 count +
 * u64 each), strides (u64 count + i64 each), radius u64, the matmul flag byte (0),
 * vendor[16], arch[16], driver[32] and the 7 capability fields (caps NULL: 56 zero
 * bytes, as hasher.rs:116-118), then `extra` bytes (this build appends a digest of an
 * explicit program or custom coefficients, which the reference key omits), hashed with
 * keyed BLAKE3 (32-byte key; NULL key = all zeros).  hex_out receives 64 hex chars + NUL. */
BST_API int bst_cache_key(const char* op, const char* dtype, int32_t ndim, const int64_t* shape,
                  const int64_t* strides, int64_t radius, const bst_device_caps* caps,
                  const uint8_t* extra, int64_t extra_len, const uint8_t* key32, char* hex_out);
/* Keyed (key32 != NULL) or plain BLAKE3 of `data`, 32-byte digest into out32. */
BST_API int bst_blake3(const uint8_t* data, int64_t len, const uint8_t* key32, uint8_t* out32);

/* ---- interceptor (crates/basalto-tree/src/interceptor.rs:39-194,226-524) --------- */
typedef struct bst_interceptor bst_interceptor;
/* interceptor.rs:50-194 (BasaltoInterceptor::new) / interceptor.rs:536-541 (PyO3 #[new]) */
BST_API int bst_interceptor_create(bst_interceptor** out);
BST_API void bst_interceptor_destroy(bst_interceptor* h);
/* interceptor.rs:226-237 (compile_and_execute) with the PyO3 argument list of
 * interceptor.rs:543-554 plus: optional custom coefficients (the Rust-only
 * `custom_coeffs`), an optional explicit program (NULL = the op's isotropic box) and
 * the stream.  dtype accepts "float32"/"f32"/"float64"/"f64".  Returns BST_ERR_INVALID
 * for rank > 3, shape/strides length mismatch or null x/y (interceptor.rs:316-324), and
 * BST_ERR_UNSUPPORTED for "matmul*" ops.  When stream is NULL the call is synchronous,
 * as the reference's launch is (crates/basalto-target-nvidia/src/runtime.rs:187); to queue on
 * the legacy default stream without waiting, pass CUDA's handle for it, cudaStreamLegacy. */
BST_API int bst_interceptor_compile_and_execute(bst_interceptor* h, const char* op, const char* dtype,
                                        int32_t ndim, const int64_t* shape, const int64_t* strides,
                                        const char* job_id, uint64_t device_ptr_x,
                                        uint64_t device_ptr_y, uint64_t device_ptr_z,
                                        const double* custom_coeffs, int64_t ncoeffs,
                                        const bst_program* program, void* stream);
/* Plans resident in the interceptor's LRU (crates/basalto-tree/src/local_cache.rs:46-68). */
BST_API int64_t bst_interceptor_cache_size(const bst_interceptor* h);
BST_API int64_t bst_interceptor_cache_hits(const bst_interceptor* h);
/* Last cache key computed by this interceptor (64 hex chars + NUL into hex_out). */
BST_API int bst_interceptor_last_key(const bst_interceptor* h, char* hex_out);

/* ---- multi-GPU: Z-slab halo exchange over NCCL ------------------------------------
 * crates/basalto-communication/src/nccl.rs:21-169 (NcclRuntime, dlopen'd NCCL) and
 * crates/basalto-communication/src/halo_exchange.rs:6-164 (HaloExchanger).
 * NCCL is loaded with dlopen at first use (the copy already in the process if any). */
typedef struct bst_comm bst_comm;
BST_API int bst_nccl_get_unique_id(uint8_t id_out[128]);
/* Non-blocking init (ncclCommInitRankConfig, blocking=0) polled until ready or until
 * timeout_s; on timeout the communicator is aborted and BST_ERR_TIMEOUT returned. */
BST_API int bst_comm_create(const uint8_t id[128], int32_t nranks, int32_t rank, int32_t device,
                    double timeout_s, bst_comm** out);
BST_API int bst_comm_destroy(bst_comm* c);
BST_API int bst_comm_abort(bst_comm* c);
BST_API int bst_comm_rank(const bst_comm* c);
BST_API int bst_comm_size(const bst_comm* c);

/* Exchange ghost planes of a Z-slab laid out as [ghost planes][n_local owned][ghost]:
 * the first `ghost` owned planes go to rank-1's upper ghost, the last `ghost` owned
 * planes to rank+1's lower ghost; ghosts are received from rank-1 / rank+1.  Ranks 0
 * and nranks-1 keep their outer ghost (non-periodic, Dirichlet-0 global ends) — the
 * reference instead wraps periodically and receives over owned data
 * (halo_exchange.rs:111-164).  One NCCL group on `stream`.
 * plane_elems = product of the non-slab extents.  Replaces
 * halo_exchange.rs:64-91 (exchange_halo_3d) + :93-164 (exchange_halo_nccl). */
BST_API int bst_halo_exchange(bst_comm* c, void* slab, int32_t dtype, int64_t plane_elems,
                      int64_t n_local, int32_t ghost, void* stream);

/* nsteps sweeps of a ZERO-boundary program over a Z-slab pair (a, b), each laid out
 * [ghost][n_local][ghost] along axis 0 with ghost = the program's axis-0 radius and the
 * global ends' outer ghosts zero.  Per step: boundary planes -> event -> halo exchange on
 * an internal comm stream, overlapped with the interior planes on `stream`.
 * Precondition: a's ghost planes hold the neighbours' planes of the input (call
 * bst_halo_exchange(a) first, or zero them for a single rank).  Result in b when nsteps
 * is odd, in a when even, with valid ghosts.  Replaces the serial exchange-then-launch
 * of crates/basalto-tree/src/executor.rs:91-119. */
BST_API int bst_slab_sweeps(bst_comm* c, const bst_program* prog, int32_t dtype, int32_t ndim,
                    const int64_t* local_shape, void* a, void* b, int32_t nsteps, void* stream);

/* Deep halos.  bst_slab_sweeps_deep is bst_slab_sweeps on slabs with `ghost` planes per side
 * (ghost >= the axis-0 radius R).  Where a temporally blocked kernel exists for the program
 * it fuses k <= min(kernel limit, ghost / R) sweeps per launch and exchanges k*R planes once
 * per k sweeps (boundary planes first, interior overlapped), so a run of n sweeps makes about
 * n/k exchanges instead of n.  Same result-buffer contract (b when nsteps is odd, a when even)
 * and the same bits as n single sweeps.  Every pass refreshes all `ghost` planes per side, so
 * the result's ghosts are complete and a later call may fuse as deeply as `ghost` allows
 * (a 1-sweep call followed by an n-sweep call equals one (n+1)-sweep call).  Each rank must
 * own at least `ghost` planes.
 * bst_slab_ghost_depth reports the depth that allows the most fusion for this program and
 * local shape (R when nothing fuses).  Replaces the per-step exchange of
 * crates/basalto-tree/src/executor.rs:91-119 (one exchange per kernel launch). */
BST_API int bst_slab_ghost_depth(const bst_program* prog, int32_t dtype, int32_t ndim, const int64_t* local_shape,
                                 int32_t* ghost_out);
BST_API int bst_slab_sweeps_deep(bst_comm* c, const bst_program* prog, int32_t dtype, int32_t ndim,
                                 const int64_t* local_shape, int32_t ghost, void* a, void* b, int32_t nsteps,
                                 void* stream);

/* ---- peer-memory slabs: the ghost exchange fused into the boundary sweep ----------
 * bst_comm_register_slab registers one slab buffer ([ghost][n_local][ghost] planes of
 * plane_elems elements along axis 0) for peer stores.  It is collective: every rank calls it
 * for its own buffer, in the same order, so that slot i on one rank and slot i on its
 * neighbours name the same logical buffer; neighbours then map each other's slot-i buffers over
 * NVLink (CUDA IPC).  The buffer must be CUDA device memory that stays allocated while the
 * communicator lives.  (The reference exchanges through NCCL or host staging before each
 * launch, crates/basalto-communication/src/halo_exchange.rs:93-322.)
 *
 * bst_slab_sweeps_p2p: nsteps sweeps over (a, b) like bst_slab_sweeps, without NCCL and
 * without an exchange step: each sweep is ONE launch on `stream`.  The launch's work items that
 * hold the first / last `ghost` owned planes, once their outputs are written, copy those planes
 * of their tile through the peer mapping over NVLink into the neighbours' ghost planes; when
 * every such item of a side is done, the last one raises that neighbour's sequence flag.  Items that read
 * ghost planes first wait (one thread, bounded at about 2 s; a timeout sets the error bit
 * bst_device_error_check reports) until the neighbour's flag shows its previous sweep, which
 * both delivered those planes and finished reading the ghost planes this sweep overwrites.
 * The two boundary chunks run first, so their planes reach the neighbours early and the
 * neighbours' next sweep normally finds its flags already set.
 * Every buffer a sweep writes (b, and a when nsteps >= 2) must be registered with this
 * geometry; a's ghost planes must hold the neighbours' planes of the input (for example after
 * bst_halo_exchange).  Each rank must own at least 2 x ghost planes; ghost >= the axis-0
 * radius; the program must run on the TMA march kernel (2-D/3-D catalog shapes).  Result in b
 * when nsteps is odd, in a when even, ghosts complete.  All ranks must issue the same
 * sequence of these calls. */
BST_API int bst_comm_register_slab(bst_comm* c, void* buf, int32_t dtype, int64_t plane_elems, int64_t n_local,
                                   int32_t ghost);
BST_API int bst_slab_sweeps_p2p(bst_comm* c, const bst_program* prog, int32_t dtype, int32_t ndim,
                                const int64_t* local_shape, int32_t ghost, void* a, void* b, int32_t nsteps,
                                void* stream);

/* bst_slab_sweeps_copy: bst_slab_sweeps_deep (same passes, fusion, contract and ghost depth)
 * with the ghost planes moved by the GPUs' copy engines over NVLink instead of NCCL, on slabs
 * registered with bst_comm_register_slab (a and b, as for bst_slab_sweeps_p2p).  Per pass:
 * the boundary rows run first, after a one-thread wait (bounded at about 2 s; a timeout sets
 * the error bit bst_device_error_check reports) for both neighbours' flags to show their
 * previous pass; then cudaMemcpyAsync copies the first / last `ghost` owned planes into the
 * neighbours' ghost planes (through the peer mappings) and a one-thread kernel raises the
 * neighbours' flags, while the interior rows compute on every SM (the copy engines need none).
 * All ranks must issue the same sequence of slab calls on the communicator. */
BST_API int bst_slab_sweeps_copy(bst_comm* c, const bst_program* prog, int32_t dtype, int32_t ndim,
                                 const int64_t* local_shape, int32_t ghost, void* a, void* b, int32_t nsteps,
                                 void* stream);

/* Per-pass timing of the slab sweeps (diagnostics).  After bst_comm_profile_begin, the next
 * max_passes passes of bst_slab_sweeps_deep / _copy / _p2p on this communicator record CUDA timing events
 * around their boundary launches, their ghost exchange and their interior launch.
 * bst_comm_profile_end waits for those events and returns, summed over the recorded passes:
 * out[0] boundary-launch ms, out[1] exchange ms, out[2] interior-launch ms, out[3] pass span ms
 * (boundary start to the later of interior end and exchange end), out[4] passes recorded,
 * out[5] ms by which exchanges outlasted their interior launch (exposed exchange time).
 * The reference times whole launches only (crates/basalto-tree/src/executor.rs:107-124). */
BST_API int bst_comm_profile_begin(bst_comm* c, int32_t max_passes);
BST_API int bst_comm_profile_end(bst_comm* c, double out[6]);

/* The march kernel's work plan for a launch of `tiles` tile columns of `planes` output planes
 * on `resident` persistent CTAs (diagnostics; host only): out[0] tile columns in the first
 * band, out[1] its chunk length in planes, out[2] its chunks per column, out[3] and out[4] the
 * same for the other columns.  Chunks are whole multiples of rb planes (the last one of a
 * column may be shorter); overhead is the per-item ramp, in planes, of the launch model that
 * picks the plan.  One band when out[0] == tiles. */
BST_API int bst_march_item_plan(int64_t tiles, int64_t planes, int32_t rb, int32_t overhead, int64_t resident,
                                int64_t out[5]);

#ifdef __cplusplus
}
#endif
#endif /* BASALTO_B200_H */
