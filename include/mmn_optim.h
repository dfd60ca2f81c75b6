/*
 * mmn_optim.h — C ABI of the B200-native MagicMindNet optimizer step.
 *
 * This is the boundary a rewritten `mmn-cuda` crate binds with `extern "C"`.
 * Every entry point replaces one item of the reference's Rust API
 * (crates/mmn-optim/src/lib.rs unless stated) and keeps its argument meaning:
 * `param` is updated in place, `grad` is read, optimizer state lives with the
 * handle (on the GPU) keyed by the caller's id exactly like the reference's
 * HashMaps. The library owns device buffers; the caller owns host buffers.
 *
 * Conventions
 *   - Return 0 (MMN_OK) on success, a negative MMN_E_* code on failure;
 *     mmn_last_error() returns a message for the calling thread's last failure.
 *     Where the reference panics (shape mismatch, lib.rs:148,161 unwrap) these
 *     calls return MMN_E_SHAPE instead.
 *   - `mem` says where pointers live: MMN_MEM_HOST (pageable or pinned host
 *     memory; the call copies in, runs and copies out before returning) or
 *     MMN_MEM_DEVICE (device memory of the handle's GPU; work is enqueued on
 *     the handle's stream and the call returns without synchronising).
 *   - One handle is used by one thread at a time (the reference's `&mut self`).
 *   - No pointer argument carries a C++ or torch type; shapes are int64 arrays.
 */
#ifndef MMN_OPTIM_H
#define MMN_OPTIM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MMN_OPTIM_ABI_VERSION 3

/* status codes */
#define MMN_OK 0
#define MMN_E_INVALID (-1)   /* null pointer, bad enum, bad size */
#define MMN_E_SHAPE (-2)     /* shape differs from the state registered for the id */
#define MMN_E_CUDA (-3)      /* a CUDA runtime call failed */
#define MMN_E_NO_DEVICE (-4) /* cuda requested without a usable GPU (MmnError::cuda_missing) */
#define MMN_E_STATE (-5)     /* call out of order (e.g. step before finalize) */
#define MMN_E_OOM (-6)       /* device allocation failed */
#define MMN_E_TIMEOUT (-7)   /* a kernel gave up a bounded wait and reported it */
#define MMN_E_UNSUPPORTED (-8)

/* where a pointer lives */
#define MMN_MEM_HOST 0
#define MMN_MEM_DEVICE 1

/* element types */
#define MMN_DTYPE_F32 0
#define MMN_DTYPE_BF16 1

/* routing of one tensor (HybridOptimizer::classify_param, lib.rs:196-202) */
#define MMN_ROUTE_AUTO 0  /* the reference rule: 2-D with both dims > 1 -> Muon */
#define MMN_ROUTE_MUON 1
#define MMN_ROUTE_ADAMW 2

/* Newton-Schulz arithmetic */
#define MMN_NS_REFERENCE 0 /* lib.rs:112-120 rounding points; B = b*A + c*A2 kept exact */
#define MMN_NS_BF16 1      /* B rounded to bf16 before B*X (faster; looser tolerance) */
#define MMN_NS_TF32 2      /* the same recipe with tf32 rounding points in place of bf16
                              (X, A, A2 held as tf32 values in fp32 words, kind::tf32
                              tensor-core products, fp32 accumulate): about 8x closer to
                              exact Newton-Schulz, half the bf16 tensor rate. No
                              counterpart in the reference. */
#define MMN_NS_FP32 3      /* no rounding points: X, A, A2 kept as fp32 values (each as
                              hi + lo tf32 planes) and every product formed from three
                              tf32 MMAs (hi*hi + hi*lo + lo*hi), fp32 accumulate: fp32-
                              accurate Newton-Schulz at about a sixth of the bf16 rate.
                              No counterpart in the reference. */

/* AdamWConfig, lib.rs:6-11 (defaults lib.rs:13-21: 3e-4, (0.9, 0.95), 1e-8, 0.01) */
typedef struct {
    float lr;
    float beta1;
    float beta2;
    float eps;
    float weight_decay;
} mmn_adamw_config;

/* MuonConfig, lib.rs:63-69 (defaults lib.rs:71-80: 0.02, 0.95, true, 5) */
typedef struct {
    float lr;
    float momentum;
    int32_t nesterov;
    int32_t ns_steps;
} mmn_muon_config;

typedef struct mmn_adamw mmn_adamw_t;
typedef struct mmn_muon mmn_muon_t;
typedef struct mmn_hybrid mmn_hybrid_t;
typedef struct mmn_optim mmn_optim_t;

/* ------------------------------------------------------------ environment */

/* crates/mmn-cuda/src/lib.rs:5-12 is_available(): 1 when a CUDA device with
 * compute capability 10.0 (B200) is usable, else 0. */
int mmn_cuda_is_available(void);

/* crates/mmn-core/src/device.rs:29-37 Device::require_cuda_available_checked:
 * MMN_E_NO_DEVICE when cuda_requested and no usable device, else MMN_OK. */
int mmn_require_cuda(int cuda_requested);

/* Message for the calling thread's most recent failure ("" if none). */
const char *mmn_last_error(void);

/* MMN_OPTIM_ABI_VERSION of the loaded library. */
int mmn_abi_version(void);

/* Failure-detection self-test: one kernel waits on an mbarrier phase that
 * nothing completes, through the bounded wait every pipelined kernel uses,
 * with a limit of limit_ns (at most 2 s). Returns MMN_E_TIMEOUT when the wait
 * gave up and reported it (the expected outcome; the device stays usable),
 * MMN_OK if it did not time out. No counterpart in the reference. */
int mmn_selftest_bounded_wait(int device, uint64_t limit_ns);

/* AdamWConfig::default() / MuonConfig::default() (lib.rs:13-21, 71-80). */
mmn_adamw_config mmn_adamw_config_default(void);
mmn_muon_config mmn_muon_config_default(void);

/* ------------------------------------------------------------------ AdamW */

/* AdamW::new (lib.rs:32-39). `device` is the CUDA ordinal; `stream` a
 * cudaStream_t (NULL = the library's own stream for this handle). */
int mmn_adamw_create(const mmn_adamw_config *cfg, int device, void *stream, mmn_adamw_t **out);
int mmn_adamw_destroy(mmn_adamw_t *h);

/* AdamW::step_param (lib.rs:41-60): advances the per-instance step counter,
 * creates zero m/v for a new id, updates param in place. `shape`/`ndim`
 * describe param and grad (same shape). grad_divisor folds
 * GradAccumulator::averaged_grad (lib.rs:254-257); pass 1 for none. */
int mmn_adamw_step_param(mmn_adamw_t *h, uint64_t id, float *param, const float *grad,
                         const int64_t *shape, int ndim, float grad_divisor, int mem);

/* The instance step counter (lib.rs:26) — read or seed it. */
int mmn_adamw_get_step(const mmn_adamw_t *h, uint64_t *step);
int mmn_adamw_set_step(mmn_adamw_t *h, uint64_t step);

/* Copy the m or v state of an id (which = 0: m, 1: v) to or from `buf`
 * (numel floats, `mem` as above). Importing creates the id's state. */
int mmn_adamw_export_state(mmn_adamw_t *h, uint64_t id, int which, float *buf, int64_t numel,
                           int mem);
int mmn_adamw_import_state(mmn_adamw_t *h, uint64_t id, int which, const float *buf,
                           int64_t numel, int mem);

/* ------------------------------------------------------------------- Muon */

/* Muon::new (lib.rs:134-139) with the Newton-Schulz arithmetic mode. */
int mmn_muon_create(const mmn_muon_config *cfg, int ns_mode, int device, void *stream,
                    mmn_muon_t **out);
int mmn_muon_destroy(mmn_muon_t *h);

/* Muon::step_matrix (lib.rs:141-175) for a 2-D rows x cols param. */
int mmn_muon_step_matrix(mmn_muon_t *h, uint64_t id, float *param, const float *grad,
                         const int64_t *shape, int ndim, float grad_divisor, int mem);

/* Create the zero velocity of an id without stepping it (lib.rs:150-153 does
 * this lazily on the first step), so that state can be imported first. An id
 * already known with the same shape is left as it is; another shape returns
 * MMN_E_SHAPE. */
int mmn_muon_register(mmn_muon_t *h, uint64_t id, const int64_t *shape, int ndim);

/* Velocity state of an id (rows*cols floats). */
int mmn_muon_export_velocity(mmn_muon_t *h, uint64_t id, float *buf, int64_t numel, int mem);
int mmn_muon_import_velocity(mmn_muon_t *h, uint64_t id, const float *buf, int64_t numel,
                             int mem);

/* newton_schulz5 (lib.rs:83-126). A non-2-D input of len elements is
 * zero-padded row-major to side x side, side = ceil(sqrt(len)) (lib.rs:89-99);
 * `out` receives rows*cols (2-D) or side*side floats. `ns_mode` as above.
 * Synchronous for MMN_MEM_HOST; enqueued on `stream` for MMN_MEM_DEVICE. */
int mmn_newton_schulz5(const float *g, const int64_t *shape, int ndim, int steps, int ns_mode,
                       float *out, int device, void *stream, int mem);

/* newton_schulz5 that allocates no device memory. No counterpart in the
 * reference: it exists for callers that cannot call cudaMalloc (device memory
 * wholly owned by another framework's allocator or a fixed arena, hosts that
 * forbid allocation after start-up, or paths where cudaMalloc's implicit
 * device synchronisation is not acceptable). Same kernels and result as
 * mmn_newton_schulz5 on a rows x cols matrix; g and out are device pointers
 * (rows*cols floats) on `device`. Its scratch is one fixed 8.25 MiB array in
 * the library, held by every GPU that loads the library until exit, so the
 * size is limited to min(rows, cols) <= 1024 and rows*cols <= 1048576; larger
 * inputs, and MMN_NS_TF32 / MMN_NS_FP32, return MMN_E_UNSUPPORTED. The first
 * call on a device resolves that array's device address and should come
 * before any stream capture. All calls on a device share the array, so calls
 * that overlap on the GPU race. Work is enqueued on `stream` (NULL = legacy
 * default stream) and the call returns after it has finished; it waits for
 * that stream only, not for the whole device. */
int mmn_newton_schulz5_noalloc(const float *g, int64_t rows, int64_t cols, int steps,
                               int ns_mode, float *out, int device, void *stream);

/* One loop body of newton_schulz5 (lib.rs:113-119) on an n x m (n <= m)
 * matrix x whose values are bf16-representable (tf32-representable for
 * MMN_NS_TF32, any fp32 value for MMN_NS_FP32), divided by x_norm first
 * (x_norm = the Frobenius norm for the first iteration, 1 afterwards). Writes
 * A = bf16(x x^T), A2 = bf16(A A) (or, for MMN_NS_BF16, bf16(b*A + c*A2); tf32
 * in place of bf16 for MMN_NS_TF32, no rounding for MMN_NS_FP32), and the next
 * x; any output pointer may be NULL. Host memory, synchronous.
 * Exposes the three tensor-core products for per-iteration parity checks. */
int mmn_newton_schulz_iteration(const float *x, int64_t n, int64_t m, float x_norm, int ns_mode,
                                float *a_out, float *a2_out, float *x_next, int device);

/* ---------------------------------------------------------------- Hybrid */

/* HybridOptimizer::classify_param (lib.rs:196-202): MMN_ROUTE_MUON (Matrix)
 * or MMN_ROUTE_ADAMW (Other). */
int mmn_hybrid_classify_param(const int64_t *shape, int ndim);

/* HybridOptimizer::new (lib.rs:189-194). */
int mmn_hybrid_create(const mmn_muon_config *muon, const mmn_adamw_config *adamw, int ns_mode,
                      int device, void *stream, mmn_hybrid_t **out);
int mmn_hybrid_destroy(mmn_hybrid_t *h);

/* HybridOptimizer::step (lib.rs:204-209). `route` MMN_ROUTE_AUTO applies the
 * reference's shape rule; MMN_ROUTE_MUON / MMN_ROUTE_ADAMW override it (the
 * tagged policy that sends embeddings and lm_head to AdamW). */
int mmn_hybrid_step(mmn_hybrid_t *h, uint64_t id, float *param, const float *grad,
                    const int64_t *shape, int ndim, int route, float grad_divisor, int mem);

/* The AdamW and Muon members (HybridOptimizer.{adamw, muon}, lib.rs:183-186). */
mmn_adamw_t *mmn_hybrid_adamw(mmn_hybrid_t *h);
mmn_muon_t *mmn_hybrid_muon(mmn_hybrid_t *h);

/* ------------------------------------------- batched device-resident step */
/*
 * The whole model's optimizer step as one device-resident operation. It
 * replaces the per-tensor optim_step_weight calls of one training step
 * (crates/mmn-models/src/chatbot.rs:208-227, call order :1104-1196 and
 * :964-1075) and the optimizer construction in the trainer
 * (crates/mmn-train/src/lib.rs:367-378). Parameters are registered once in
 * the reference's call order; the AdamW step counter advances per AdamW
 * tensor in that order, exactly as the reference's per-call counter does.
 */
typedef struct {
    mmn_adamw_config adamw;
    mmn_muon_config muon;
    int32_t use_hybrid;       /* TrainConfig.optimizer == "hybrid" (crates/mmn-train/src/lib.rs:378);
                                 0 routes every tensor to AdamW, as the reference does
                                 for "adamw" and for the documented-but-unimplemented "muon" */
    int32_t ns_mode;          /* MMN_NS_* */
    int32_t fresh_state;      /* 1: m, v and velocity start at zero every step (the
                                 trainer never reuses ids, crates/mmn-train/src/lib.rs:380) */
    int32_t grad_dtype;       /* MMN_DTYPE_F32 or MMN_DTYPE_BF16 */
    int32_t bf16_param_shadow;/* 1: keep a bf16 copy of every param, refreshed each step */
    int32_t loss_scaling;     /* 1: grads are divided by a device loss scale, any
                                 non-finite grad skips the step and halves the scale */
    float loss_scale_init;    /* e.g. 65536 */
    int32_t growth_interval;  /* clean steps before the scale doubles (e.g. 2000) */
    int32_t rank;             /* shard of the step this process owns (0 .. world_size-1) */
    int32_t world_size;       /* 1 = unsharded */
    int32_t use_graph;        /* 1: capture the step in a CUDA graph at first use */
    int32_t reduce_grads;     /* 1: every rank holds its own local grads and
                                 mmn_optim_reduce_grads sums them across ranks before
                                 each step (data parallelism); the step then takes its
                                 skip decision from that call instead of scanning */
    int32_t scan_shard;       /* 1 (loss_scaling, world_size > 1, grads replicated): each
                                 rank scans only what it steps, in mmn_optim_scan_grads,
                                 and sets every rank's skip flag; the step does not scan */
} mmn_optim_config;

/* Defaults: AdamW/Muon defaults, hybrid, reference NS, persistent state, f32
 * grads, no shadow, no loss scaling, unsharded, graphs on. */
mmn_optim_config mmn_optim_config_default(void);

int mmn_optim_create(const mmn_optim_config *cfg, int device, void *stream, mmn_optim_t **out);
int mmn_optim_destroy(mmn_optim_t *h);

/* Register one parameter tensor (call order = optimizer call order). Returns
 * its slot index in *slot. ids must be distinct. */
int mmn_optim_add_param(mmn_optim_t *h, uint64_t id, const int64_t *shape, int ndim, int route,
                        int *slot);

/* Freeze the layout and allocate every device buffer. After a failed finalize
 * (e.g. MMN_E_OOM) the handle only accepts mmn_optim_destroy: further calls
 * return MMN_E_STATE. */
int mmn_optim_finalize(mmn_optim_t *h);

/* Device pointers of a slot's fp32 param, its grad (grad_dtype) and its bf16
 * shadow (NULL without one). Valid until destroy. */
int mmn_optim_slot_ptrs(mmn_optim_t *h, int slot, float **param, void **grad,
                        void **param_bf16);

/* Copy a slot's param in or out, or its grad in (`mem` as above; device
 * copies are enqueued on the handle's stream). */
int mmn_optim_set_param(mmn_optim_t *h, int slot, const float *src, int mem);
int mmn_optim_get_param(mmn_optim_t *h, int slot, float *dst, int mem);
int mmn_optim_set_grad(mmn_optim_t *h, int slot, const void *src, int mem);

/* Optimizer state of a slot: which = 0 m, 1 v (AdamW slots), 2 velocity (Muon). */
int mmn_optim_set_state(mmn_optim_t *h, int slot, int which, const float *src, int mem);
int mmn_optim_get_state(mmn_optim_t *h, int slot, int which, float *dst, int mem);

/* Seed / read the AdamW step counter (calls so far). */
int mmn_optim_set_adamw_step(mmn_optim_t *h, uint64_t step);
int mmn_optim_get_adamw_step(mmn_optim_t *h, uint64_t *step);

/* Enqueue one optimizer step over every slot this rank owns. grad_divisor is
 * GradAccumulator's micro-batch count (1 = none). Asynchronous. A handle made
 * with reduce_grads (scan_shard) returns MMN_E_STATE unless
 * mmn_optim_reduce_grads (mmn_optim_scan_grads) ran since its last step; the
 * same holds for mmn_optim_step_host. */
int mmn_optim_step(mmn_optim_t *h, float grad_divisor);

/* One step from host memory, the batched form of the reference's
 * optim_step_weight calls on host arrays (crates/mmn-models/src/chatbot.rs:208-227
 * calling HybridOptimizer::step, crates/mmn-optim/src/lib.rs:221-245).
 * grads[slot] (host, grad_dtype, numel elements) are copied in, the step runs,
 * and the updated fp32 params go to params[slot] (host); the device copy stays
 * the master. Either array may hold null entries (that slot's copy is skipped:
 * its grad is already on the device / its params are not read back). With
 * world_size > 1 a rank copies only what it steps (its Muon matrices and its
 * AdamW range; every grad when loss_scaling is on, for the non-finite scan).
 * The copies run on two copy streams in chunks, overlapped with the compute
 * and with each other; pinned (page-locked) host memory lets them overlap.
 * Synchronous: returns once params[] hold the step's result. */
int mmn_optim_step_host(mmn_optim_t *h, const void *const *grads, float *const *params,
                        float grad_divisor);

/* Wait for the handle's stream; reports MMN_E_TIMEOUT if a kernel gave up. */
int mmn_optim_sync(mmn_optim_t *h);

/* Loss-scaling state (after mmn_optim_sync): current scale, steps skipped. */
int mmn_optim_loss_scale(mmn_optim_t *h, float *scale, int64_t *skipped_steps);

/* The whole loss-scaling state, for checkpoints: scale, steps skipped so far
 * and clean steps since the scale last changed. Synchronous. */
int mmn_optim_get_loss_state(mmn_optim_t *h, float *scale, int64_t *skipped_steps,
                             int32_t *good_steps);
int mmn_optim_set_loss_state(mmn_optim_t *h, float scale, int64_t skipped_steps,
                             int32_t good_steps);

/* Sharding plan (world_size > 1). A Muon matrix is stepped whole by one rank,
 * chosen by longest-processing-time bin packing on its Newton-Schulz flops;
 * the flat AdamW arena is cut into world_size equal element ranges.
 * owner_rank is the Muon owner, or -1 for an AdamW slot (split by range). */
int mmn_optim_slot_owner(mmn_optim_t *h, int slot, int *owner_rank);

/* Where the params live for the post-step exchange. Each arena is
 * world_size equal regions of `*_region` elements; rank r steps region r of
 * both. An all-gather of region r from every rank into the same offsets
 * completes the step everywhere. With bf16_param_shadow the bf16 arenas (same
 * element layout) are the ones to gather. */
typedef struct {
    float *adamw_param;
    void *adamw_param_bf16;
    int64_t adamw_region;
    float *muon_param;
    void *muon_param_bf16;
    int64_t muon_region;
} mmn_optim_gather_layout;
int mmn_optim_get_gather_layout(mmn_optim_t *h, mmn_optim_gather_layout *out);

/* The layout and sharding plan mmn_optim_finalize uses, computed on the host
 * alone (no device): n tensors, `shapes` holds their dims back to back
 * (ndims[i] each), `routes` as for mmn_optim_add_param. Fills, per tensor, the
 * Muon owner rank (-1 for AdamW tensors, which are split by arena range) and
 * the element offset in its arena, plus both arenas' per-rank region sizes.
 * Every rank computes the same plan from the same inputs. */
int mmn_optim_plan(const int64_t *shapes, const int *ndims, const int *routes, int n,
                   int use_hybrid, int ns_steps, int world_size, int *owner, int64_t *offset,
                   int64_t *adamw_region, int64_t *muon_region);

/* Parameter exchange fused into the step (world_size > 1), in place of a
 * post-step all-gather. After mmn_optim_connect_peers the step pushes each
 * finished piece of this rank's regions into every peer's arena at the same
 * offset, over NVLink through CUDA IPC mappings, on transfer streams of its
 * own (one per peer): the AdamW range once its kernel ends, and the Newton-Schulz matrices in
 * chunks (runs of at most 16 matrices of one shape, largest first), each as
 * soon as its last iteration ends, so the copies overlap the chunks still
 * computing. fp32 params are sent, or only the bf16 copies when
 * bf16_param_shadow is on (the fp32 master then stays with its owner). Every
 * rank must finish its step before any rank reads parameters or starts the
 * next step: order the ranks after each mmn_optim_step (for example a
 * one-element all-reduce on the same stream).
 * mmn_optim_export_ipc writes this rank's MMN_IPC_BLOB_BYTES-byte blob;
 * mmn_optim_connect_peers takes the world_size blobs back to back in rank
 * order (exchanged by the caller, e.g. with an all-gather). */
#define MMN_IPC_BLOB_BYTES 512
int mmn_optim_export_ipc(mmn_optim_t *h, void *blob);
int mmn_optim_connect_peers(mmn_optim_t *h, const void *blobs);

/* Data-parallel grad reduction fused with the non-finite scan, over NVLink
 * (config.reduce_grads = 1, world_size > 1, after mmn_optim_connect_peers).
 * This is the all-reduce (or reduce-scatter) of the local grads that a
 * data-parallel trainer runs before the optimizer step; the reference trains
 * on one process and has none. Every rank holds its own local grads for every
 * slot; the call makes this rank's regions (its Muon matrices and its AdamW
 * range, all its step reads) hold the sum over ranks, accumulated in fp32 in
 * rank order 0, 1, ..., world_size-1 (bf16 grads: the fp32 sum rounded to bf16
 * once), by loading the peers' grads directly from their memory. Other regions
 * keep this rank's local grads. Averaging is the step's grad_divisor. With
 * loss_scaling, a non-finite sum anywhere sets every rank's skip flag, and the
 * next mmn_optim_step skips on every rank without a scan. The ranks must be
 * ordered before the call (every rank's grads final) and between the call and
 * mmn_optim_step (every rank's loads and flags done), e.g. with one-element
 * all-reduces on the same stream. Asynchronous. */
int mmn_optim_reduce_grads(mmn_optim_t *h);

/* Non-finite scan of this rank's part of the grads (config.scan_shard = 1,
 * after mmn_optim_connect_peers), the sharded form of the scan every rank
 * otherwise runs over every grad inside mmn_optim_step: a non-finite value in
 * this rank's Muon matrices or AdamW range sets every rank's skip flag
 * through peer memory, so each rank reads 1/world_size of the grads. `grads`
 * NULL: the grads are on the device; else host buffers per slot (NULL entries
 * skipped) of which this rank's parts are copied in first, and the call
 * returns once they have been read. Order the ranks between this call and the
 * step that uses the flag (e.g. a one-element all-reduce on the same stream),
 * as for mmn_optim_reduce_grads; with scan_shard, mmn_optim_step_host takes
 * null grads (they came in here). No counterpart in the reference. */
int mmn_optim_scan_grads(mmn_optim_t *h, const void *const *grads);

/* The reduction of mmn_optim_reduce_grads on buffers the caller owns, for a
 * trainer that keeps its grads outside a handle: dst[i] = src[0][i] +
 * src[1][i] + ... + src[nsrc-1][i] for i in [0, numel), accumulated in fp32 in
 * source order (MMN_DTYPE_BF16: bf16 inputs, the fp32 sum rounded to bf16
 * once), the same kernels and arithmetic as the handle's rank-ordered sum.
 * 2 <= nsrc <= 8. Every pointer is a 16-byte aligned device pointer. dst is
 * memory of `device`, and either equals one source (an in-place sum) or
 * overlaps none. A source is memory of `device` or of another GPU that
 * `device` can reach over NVLink (a peer allocation or a cudaIpcOpenMemHandle
 * mapping); the call enables peer access to that GPU first. When
 * nonfinite_flag (an int on `device`) is not NULL, a non-finite sum sets it to
 * 1; it is never cleared here. Enqueued on `stream` (NULL = legacy default
 * stream); returns without synchronising. The reference trains on one process
 * and has no counterpart; this is the data-parallel sum that runs before
 * crates/mmn-optim/src/lib.rs:41-60 / :141-175 on each rank. */
int mmn_grad_reduce(const void *const *src, int nsrc, void *dst, int64_t numel, int dtype,
                    int *nonfinite_flag, int device, void *stream);

/* The sharded non-finite scan of mmn_optim_scan_grads on a buffer the caller
 * owns: when any of grads[0, numel) (fp32, or bf16 for MMN_DTYPE_BF16) is Inf
 * or NaN, every flags[k] (k < nflags, 1 <= nflags <= 8) is set to 1; flags are
 * never cleared here. Each rank scans only its own part of the grads and
 * raises its peers' flags as well as its own, so the ranks reach one skip
 * decision while each reads 1/world_size of the grads. grads is a 16-byte
 * aligned device pointer on `device`; a flag is an int of `device` or of a
 * peer GPU that `device` can reach (peer access is enabled first). Enqueued on
 * `stream`; returns without synchronising. The reference checks no grads for
 * non-finite values and has no counterpart (the loss-scaled step skips on one,
 * see mmn_optim_step). */
int mmn_grad_nonfinite_scan(const void *grads, int64_t numel, int dtype, int *const *flags,
                            int nflags, int device, void *stream);

/* Parameter counts: total registered, stepped by AdamW, stepped by Muon. */
int mmn_optim_param_counts(mmn_optim_t *h, int64_t *total, int64_t *adamw, int64_t *muon);

/* Algorithmic Newton-Schulz flops of one step on this rank
 * (ns_steps * (4 n^2 m + 2 n^3) per owned matrix, n <= m). */
int mmn_optim_ns_flops(mmn_optim_t *h, double *flops);

/* Kernel launches one mmn_optim_step enqueues on this rank, and one
 * mmn_optim_reduce_grads or mmn_optim_scan_grads (0 unless reduce_grads or
 * scan_shard). */
int mmn_optim_kernel_launches(mmn_optim_t *h, int64_t *per_step, int64_t *per_reduce);

/* Per-step device-time breakdown in ms, averaged over the steps enqueued since
 * timing was (re-)enabled (each such step records CUDA events around its phases
 * and is launched without the CUDA graph): [0] AdamW kernel, [1] Muon
 * momentum+norm, [2] Newton-Schulz GEMMs, [3] Muon update, [4] whole step. */
int mmn_optim_enable_timing(mmn_optim_t *h, int enable);
int mmn_optim_last_timing(mmn_optim_t *h, float *ms5);

/* The same breakdown with the Muon momentum pass and the Frobenius norms apart:
 * [0] AdamW kernel, [1] Muon momentum, [2] Newton-Schulz input norms, [3]
 * Newton-Schulz GEMMs, [4] Muon update, [5] whole step. On host steps
 * (mmn_optim_step_host) no events are recorded. */
int mmn_optim_last_timing_ex(mmn_optim_t *h, float *ms6);

#ifdef __cplusplus
}
#endif
#endif /* MMN_OPTIM_H */
