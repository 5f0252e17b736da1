/*
 * cresso_b200.h - C ABI of the B200-native CRESSO5 optimizer step.
 *
 * This library replaces the reference's PyTorch-extension boundary
 * (cresso_cuda_ext.py JIT loader + cresso_cuda/cresso_cuda.cpp pybind module,
 * 19 entries at cresso_cuda.cpp:170-196) with plain C entry points:
 *   - raw device pointers, plain integer / double sizes, a cudaStream_t;
 *   - every entry returns an int status (0 = ok, else a CRESSO_E* code) and
 *     never throws or aborts; the message of the last failure on the calling
 *     thread is read with cresso_last_error();
 *   - the library allocates no device memory for the optimizer step: the
 *     caller provides workspaces whose sizes are queried first;
 *   - all GPU work is stream-ordered on the given stream, with no implicit
 *     device synchronisation.
 *
 * All structs below contain only 8-byte fields (int64_t / double / pointers
 * stored as uint64_t) so that they have the same layout from C, ctypes and
 * numpy.  cresso_abi_layout() reports their sizes for a load-time check.
 */
#ifndef CRESSO_B200_H
#define CRESSO_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CRESSO_API __attribute__((visibility("default")))
#else
#define CRESSO_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef void* cresso_stream_t; /* a cudaStream_t; NULL = legacy default stream */

enum {
    CRESSO_OK = 0,
    CRESSO_EINVAL = 1,       /* bad argument (shape, pointer, size, value)      */
    CRESSO_EUNSUPPORTED = 2, /* valid for the reference, not on this CUDA path  */
    CRESSO_ECUDA = 3,        /* a CUDA runtime call or kernel launch failed     */
    CRESSO_ESCRATCH = 4      /* caller workspace smaller than the queried size  */
};

enum { CRESSO_MAX_NDIM = 8, CRESSO_MAX_RANK = 16 };

/* Hyper-parameters of one parameter group.  Mirrors the `defaults` dict of
 * CRESSO5.__init__ (reference cresso_v5.py:760-818); integer options are
 * stored as doubles.  Keys that only steer host routing (min_spectral_size,
 * thin_matrix_*, micro_field_max_size) are not read by the kernels. */
typedef struct cresso_hparams {
    double lr, weight_decay, energy_power, dt, impulse_friction, contact_gain, restoring, cubic;
    double metric_dt, metric_friction, metric_coupling, local_sharpness;
    double instant_metric_coupling, instant_metric_power, root_channel_mix, echo_mix, transport_mix;
    double hash_decay, hash_impulse_decay, hash_metric_coupling, hash_drive_mix;
    double direct_force_mix, residual_feedback_mix, reservoir_decay, refractory_decay, refractory_gain;
    double confidence_decay, confidence_gain, surprise_gain, surprise_decay, prediction_mix, novelty_mix;
    double warmup_steps, surprise_brake, target_update_rms, min_gain, max_gain, drive_clip, spike_mix;
    double eps, maximize, rank, max_frequency, hash_bins, hash_tables, hard_channel_min_size;
    double thin_matrix_hard_cutoff;
    double micro_decay, micro_impulse_decay, micro_drive_mix; /* micro-field route */
} cresso_hparams;

/* One parameter tensor handed to a group step.  `shape` is the GLOBAL shape.
 * A row-sharded 2-D tensor passes its local row block [row0, row0+rows);
 * a sharded 1-D tensor passes its element range [col0, col0+cols).  An
 * unsharded tensor passes row0 = col0 = 0 and the full extents.
 * State pointers point at the reference state tensors (cresso_v5.py:857-891)
 * owned by the caller and are updated in place. */
typedef struct cresso_tensor_desc {
    int64_t ndim;
    int64_t shape[CRESSO_MAX_NDIM];
    int64_t row0, rows, col0, cols;
    int64_t step; /* state["step"] after the increment of this step (1-based) */
    uint64_t param, grad;           /* dtype below, contiguous, local block        */
    uint64_t shape_ws;              /* cresso_shape_workspace_init() output       */
    uint64_t hash_cache;            /* cresso_hash_cache_init() output or 0        */
    int64_t hash_cache_n;           /* flat indices covered by hash_cache          */
    /* spectral route state (float32): */
    uint64_t omega, q_cos, q_sin, p_cos, p_sin, metric_cos, metric_sin, metric_p_cos, metric_p_sin;
    uint64_t calcium_cos, calcium_sin, mode_confidence, hash_energy, hash_impulse, hash_refractory;
    /* common 0-d state (float32): */
    uint64_t force_rms, drive_energy, surprise, action;
    /* scalar route 0-d state (float32): */
    uint64_t q, impulse, metric_q, metric_impulse;
    /* element type of param and grad (CRESSO_DTYPE_*); the work and the state are
     * float32 for float32 / float16 / bfloat16 parameters, and a float16 / bfloat16
     * parameter receives the update rounded to its type first, as
     * param.add_(update.to(param.dtype)) does (cresso_v5.py:119-124, 1353, 1582).
     * float64 parameters work in float64 and their state pointers point at
     * float64 values (spectral route: cresso_spectral64_run). */
    int64_t dtype;
    /* micro-field route state: float32 fields of the parameter's shape */
    uint64_t micro_energy, micro_impulse, micro_refractory;
} cresso_tensor_desc;

enum { CRESSO_DTYPE_F32 = 0, CRESSO_DTYPE_F16 = 1, CRESSO_DTYPE_BF16 = 2, CRESSO_DTYPE_F64 = 3 };

/* ---------------------------------------------------------------- info --- */

CRESSO_API const char* cresso_version(void);
/* Architecture the kernels were compiled for ("sm_100a"). */
CRESSO_API const char* cresso_arch(void);
/* Copies the last error message of this thread into buf (NUL-terminated);
 * returns its full length. */
CRESSO_API int cresso_last_error(char* buf, size_t n);
/* out[0] = sizeof(cresso_hparams), out[1] = sizeof(cresso_tensor_desc),
 * out[2] = CRESSO_MAX_NDIM, out[3] = CRESSO_MAX_RANK. */
CRESSO_API int cresso_abi_layout(int64_t* out, int n);
/* Number of kernels this library has launched in the process so far (all
 * devices and threads); lets a caller count the GPU launches of a region. */
CRESSO_API int64_t cresso_launch_count(void);

/* ------------------------------------------------------------ hash ops --- */

/* idx[i] = hash(offset + i) mod bins for table `salt`, int64.  Restates the
 * coordinate hash _hash_index_tensor (cresso_v5.py:495-516); the reference
 * CUDA computes the same value inline (cresso_cuda_kernel.cu:184-201). */
CRESSO_API int cresso_hash_index(int64_t offset, int64_t n, int64_t bins, int64_t salt, int64_t* idx,
                      cresso_stream_t stream);

/* out[b] = mean of x over the elements hashed to bin b (0 for empty bins).
 * Replaces ops.hash_reduce_mean (cresso_cuda.cpp:186, kernel cu:1222-1253). */
CRESSO_API int cresso_hash_reduce_mean(const float* x, int64_t n, int64_t bins, int64_t salt, float* out,
                            cresso_stream_t stream);

/* out[i] = values[hash(i) mod bins].  Replaces ops.hash_gather
 * (cresso_cuda.cpp:187, kernel cu:1255-1276). */
CRESSO_API int cresso_hash_gather(const float* values, int64_t bins, int64_t n, int64_t salt, float* out,
                       cresso_stream_t stream);

/* Per-process bin-index cache for `tables` salted tables over flat indices
 * [0, n): uint8 per index when bins <= 256, else uint16, table t at [t * n].
 * With two tables of at most 64 bins a joint section follows at byte offset
 * align_up(2 n, 256): one uint16 b0 + 64 b1 per index (read by the kernels of
 * the full-tile tensor class).  Shared by every tensor with the same (bins,
 * tables).  Replaces the per-kernel hash recomputation of the reference
 * (cu:189-201 called from K11-K17). */
CRESSO_API int cresso_hash_cache_bytes(int64_t n, int64_t bins, int64_t tables, int64_t* bytes);
CRESSO_API int cresso_hash_cache_init(int64_t n, int64_t bins, int64_t tables, void* cache, cresso_stream_t stream);

/* ----------------------------------------------------------- basis ops --- */

/* Per-shape workspace: separable axis tables of the spectral carriers, their
 * normalisation stats, the carrier Gram matrix and the hash bin counts.
 * Replaces basis_axis_cache + basis_stats_with_cache (cresso_cuda.cpp:171-173,
 * cu:842-932) and the transient per-step _CudaBasisCache (cresso_v5.py:100-107,
 * 380-415); the caller keeps it across steps (never in state_dict).
 * freqs: host int64 [rank][ndim] = state["freqs"].  bins / tables = 0 skips
 * the counts.  Supports ndim 1..CRESSO_MAX_NDIM (a tensor of rank n >= 2 is
 * laid out as (product of its n - 1 leading axes) x (last axis)), rank
 * 1..CRESSO_MAX_RANK. */
CRESSO_API int cresso_shape_workspace_bytes(int64_t ndim, const int64_t* shape, int64_t rank, int64_t bins,
                                 int64_t tables, int64_t* bytes);
CRESSO_API int cresso_shape_workspace_init(int64_t ndim, const int64_t* shape, int64_t rank, const int64_t* freqs,
                                int64_t bins, int64_t tables, void* ws, cresso_stream_t stream);

/* out_cos[r] = mean(x * cos_r), out_sin[r] = mean(x * sin_r) over the whole
 * tensor.  Replaces ops.basis_project* (cresso_cuda.cpp:174-176, cu:934-1089);
 * matches _project (cresso_v5.py:351-359). */
CRESSO_API int cresso_basis_project(const float* x, const void* ws, float* out_cos, float* out_sin,
                         cresso_stream_t stream);

/* out = shrink * sum_r g_r (c_r cos_r + s_r sin_r); gates may be NULL (g = 1).
 * Replaces ops.basis_reconstruct* (cresso_cuda.cpp:177-185, cu:1091-1220);
 * matches _reconstruct (cresso_v5.py:362-376). */
CRESSO_API int cresso_basis_reconstruct(const float* coef_cos, const float* coef_sin, const float* gates,
                             const void* ws, float* out, cresso_stream_t stream);

/* Stateless axial metric of a 1-D or 2-D field (cresso_v5.py:243-262).
 * Replaces ops.instant_axis_metric_2d (cresso_cuda.cpp:190, cu:1766-1827). */
CRESSO_API int cresso_instant_axis_metric(const float* rel, int64_t ndim, const int64_t* shape, double power,
                               double coupling, double eps, float* out, cresso_stream_t stream);

/* ---------------------------------------------------- spectral route ---- */

/* Fused CRESSO5 step of n spectral-route tensors (cresso_v5.py:945-1353),
 * replacing the 13 reference call sites into the extension inside
 * _spectral_step (metric/confidence/contact/drive updates, hash metric and
 * impulse, projections and reconstructions; cresso_cuda.cpp:171-194).
 *
 * The step is a sequence of CRESSO_SPECTRAL_STAGES kernel stages:
 *    0 upload plan | 1 pass P1  2 reduce 1 | 3 finalize 1  4 pass P2  5 reduce 2 |
 *    6 finalize 2  7 pass P3  8 reduce 3 | 9 finalize 3  10 pass P4  11 reduce 4 |
 *   12 finalize 4  13 pass P5
 * P1 force energy; P2 density, hash bins, projection, axis sums; P3 tangent,
 * prediction error, port; P4 drive statistics; P5 parameter update.
 * Reduction vector k (k = 1..4, float64) is complete after stage 3k-1.  A
 * single GPU runs stages [0, 14) in one call.  A row-sharded run calls
 * [0,3) [3,6) [6,9) [9,12) [12,14) and SUM-all-reduces reduction vector k
 * across ranks between the k-th and (k+1)-th call.
 *
 * layout[0]  = scratch bytes needed
 * layout[1+2(k-1)], layout[2+2(k-1)] (k = 1..4) = byte offset in the scratch
 *              and length in doubles of reduction vector k.
 * Written only when layout_len is large enough (no counterpart in the reference):
 * layout[9]  = byte offset of an int32 status word in the scratch, zeroed by
 *              stage 0 and set nonzero by a kernel whose bounded wait for its
 *              tensor-core products gave up (the step's results are then invalid);
 * layout[10] = rows per item of the 256-column tiles;
 * layout[11] = bit p set when pass Pp of the full-tile tensors runs on the
 *              tcgen05 tensor cores (p = 3, 4, 5). */
enum { CRESSO_SPECTRAL_STAGES = 14 };

/* Self-test of the bounded in-kernel wait that guards the tensor-core passes
 * (no counterpart in the reference): one block waits on an mbarrier that
 * completes only if `arrive` is nonzero, for at most limit_ns (<= 2 s), then
 * stores 1 in the device int32 *status_word if the wait ran out, else 0.  It
 * shows on a live GPU that a wait which nothing satisfies ends with an error
 * status the host reads, and the context stays usable. */
CRESSO_API int cresso_selftest_bounded_wait(int64_t limit_ns, int64_t arrive, void* status_word,
                                            cresso_stream_t stream);
CRESSO_API int cresso_spectral_layout(const cresso_tensor_desc* descs, int64_t n, const cresso_hparams* hp,
                           int64_t num_sms, int64_t* layout, int64_t layout_len);
CRESSO_API int cresso_spectral_run(const cresso_tensor_desc* descs, int64_t n, const cresso_hparams* hp, void* scratch,
                        int64_t scratch_bytes, int64_t stage_begin, int64_t stage_end, int64_t num_sms,
                        cresso_stream_t stream);
/* cresso_spectral_run reporting device-side failures into a caller-owned
 * int32 device word (no counterpart in the reference, whose kernels have no
 * in-kernel waits).  Kernels OR failure bits into *status_word and nothing
 * in the library clears it: bit 0 (1) = a bounded wait inside a pass kernel
 * gave up and that group's results and state of this step are invalid; bit 1
 * (2) = after such a give-up the in-flight tensor-core work did not finish
 * within its bound either, so later steps in this process are not to be
 * trusted.  The caller zeroes the word once, keeps it across steps and groups,
 * and reads it asynchronously (e.g. copied to pinned host memory after the
 * step).  status_word = NULL is cresso_spectral_run (the scratch word of
 * layout[9], cleared by stage 0). */
CRESSO_API int cresso_spectral_run_status(const cresso_tensor_desc* descs, int64_t n, const cresso_hparams* hp,
                                          void* scratch, int64_t scratch_bytes, int64_t stage_begin,
                                          int64_t stage_end, int64_t num_sms, void* status_word,
                                          cresso_stream_t stream);
/* Stream-ordered copy of a device status word into host memory the device can
 * write (pinned host memory under unified addressing), by a one-thread kernel
 * rather than a copy engine, so that it never waits behind the caller's own
 * host-device transfers (no counterpart in the reference). */
CRESSO_API int cresso_status_copy(const void* status_word, void* host_word, cresso_stream_t stream);

/* Copies n_segments byte ranges in one launch.  `table` is device memory of
 * n_segments rows of three uint64 values: source address, destination
 * address, byte count (ranges must not overlap).  No counterpart in the
 * reference, which has no multi-GPU path: the row-sharded optimizer packs the
 * parameters and floating-point state of the tensors it steps whole (one
 * owner rank each) into one byte buffer before an all-gather, and unpacks
 * the gathered buffer into every rank's tensors, with one launch each instead
 * of one copy per tensor. */
CRESSO_API int cresso_copy_segments(const uint64_t* table, int64_t n_segments, cresso_stream_t stream);

/* Float64 parameters on the spectral route (cresso_v5.py:945-1353 with the
 * float64 work and state of cresso_v5.py:119-124), and float32 / float16 /
 * bfloat16 parameters when rank > CRESSO_MAX_RANK (rank up to 4096, the bound of
 * the reference's CUDA contact kernel, cresso_cuda_kernel.cu:1937; the
 * reference's PyTorch path takes any rank).  The shape
 * workspace holds float64 axis tables and the carrier stats built from them;
 * state pointers of the descriptors point at float64 values for float64
 * parameters and at float32 values otherwise, `shape_ws` at this workspace.
 * The step runs the same five passes as cresso_spectral_run in float64
 * arithmetic, a group of tensors at a time (above rank 64 the reconstructions
 * loop over the modes and the projections run in chunks of 16 modes, with the
 * port field stored between them); a 16-bit parameter receives the update rounded
 * to its type, as in cresso_spectral_run.  Tensors are whole (not sharded),
 * hash_bins * hash_tables <= 2048. */
CRESSO_API int cresso_shape_workspace64_bytes(int64_t ndim, const int64_t* shape, int64_t rank, int64_t* bytes);
CRESSO_API int cresso_shape_workspace64_init(int64_t ndim, const int64_t* shape, int64_t rank, const int64_t* freqs,
                                             void* ws, cresso_stream_t stream);
CRESSO_API int cresso_spectral64_scratch_bytes(const cresso_tensor_desc* descs, int64_t n, const cresso_hparams* hp,
                                               int64_t* bytes);
CRESSO_API int cresso_spectral64_run(const cresso_tensor_desc* descs, int64_t n, const cresso_hparams* hp,
                                     void* scratch, int64_t scratch_bytes, cresso_stream_t stream);

/* ------------------------------------------------------ scalar route ---- */

/* Fused scalar-route step of n small / LoRA-thin tensors
 * (cresso_v5.py:1434-1582), one thread block per tensor, all tensors in one
 * launch.  Replaces ops.scalar_update_2d (cresso_cuda.cpp:195,
 * cu:3225-3605), and also covers 0-d, 1-d and N-d (N <= 8) tensors that the
 * reference sends to its PyTorch path.  Tensors are never sharded. */
CRESSO_API int cresso_scalar_scratch_bytes(const cresso_tensor_desc* descs, int64_t n, int64_t* bytes);
CRESSO_API int cresso_scalar_run(const cresso_tensor_desc* descs, int64_t n, const cresso_hparams* hp, void* scratch,
                      int64_t scratch_bytes, cresso_stream_t stream);

/* ------------------------------------------------------- micro route ---- */

/* Fused micro-field step of n small tensors (cresso_v5.py:1355-1432, the
 * route of every tensor with 0 < numel <= micro_field_max_size and rank >= 1):
 * per-element energy / impulse / refractory fields (micro_* in the
 * descriptor), one thread block per tensor, all tensors in one launch.  The
 * reference has this route on its PyTorch path only.  Tensors are never
 * sharded. */
CRESSO_API int cresso_micro_scratch_bytes(const cresso_tensor_desc* descs, int64_t n, int64_t* bytes);
CRESSO_API int cresso_micro_run(const cresso_tensor_desc* descs, int64_t n, const cresso_hparams* hp, void* scratch,
                                int64_t scratch_bytes, cresso_stream_t stream);

/* ---------------------------------------------- allocation-free entry ---- */

/* Size of the library's built-in device scratch array (8 MiB). */
#define CRESSO_NOALLOC_SCRATCH_BYTES (8u << 20)

/* cresso_scalar_run without caller scratch.  This entry point has no
 * counterpart in the reference.  It is for callers that cannot allocate
 * device memory themselves: hosts whose device memory is owned by another
 * allocator (a framework's caching allocator or a pool reserved at start-up
 * that forbids raw cudaMalloc later) and thin FFI hosts that have no device
 * allocator of their own.  It calls no cudaMalloc / cudaFree or any
 * allocating routine; its scratch is a file-scope device array of
 * CRESSO_NOALLOC_SCRATCH_BYTES that every GPU loading the library holds until
 * the process exits.  Tensor lists whose scratch (cresso_scalar_scratch_bytes)
 * exceeds that size are rejected with CRESSO_ESCRATCH: split them over several
 * calls.  Every call looks up the array's device address in the current
 * context (cudaGetSymbolAddress, with the target device current); the first
 * call on a device also loads the library's module there, so make that first
 * call before any stream capture.  All calls share the one array, so calls that may overlap
 * on the GPU (other streams, other host threads, same device) race: order
 * them on one stream or serialise them. */
CRESSO_API int cresso_scalar_run_noalloc(const cresso_tensor_desc* descs, int64_t n, const cresso_hparams* hp,
                                         cresso_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* CRESSO_B200_H */
