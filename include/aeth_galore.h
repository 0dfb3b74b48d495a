/*
 * aeth_galore.h -- C ABI of the B200 (sm_100a) per-layer optimizer step.
 *
 * Every entry point takes plain device pointers and sizes and returns an int
 * status (except doublepass_galore_apply, whose reference signature is void):
 *     0                  success
 *    -1  AETH_ERR_ARG    bad dimensions / null pointer (the reference's -1)
 *    -2  AETH_ERR_SHAPE  shape mismatch (GaLoreError::Shape, galore/src/error.rs:10-29)
 *    -3  AETH_ERR_CONFIG configuration error (GaLoreError::Config)
 *    -4  AETH_ERR_UNSUPPORTED  shape/alignment this build does not handle
 *    -5  AETH_ERR_NOT_FOUND    unknown parameter key
 *    -6  AETH_ERR_TIMEOUT      a bounded device-side wait gave up (kernel returned early)
 *    -7  AETH_ERR_LINALG       rank-deficient factorisation (GaLoreError::Linalg)
 *    >0  a cudaError_t value
 * No entry point aborts the process.  All work is enqueued on the caller's
 * stream; only functions documented as synchronous wait on it.
 *
 * Streams are passed as `aeth_stream_t` (void*), ABI-identical to the
 * reference's cudaStream_t / Rust `*mut c_void` (galore/src/kernels/mod.rs:10-50).
 * Reference paths below are relative to the reference project's aethelStream/.
 */
#ifndef AETH_GALORE_H
#define AETH_GALORE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* aeth_stream_t;

enum {
    AETH_OK = 0,
    AETH_ERR_ARG = -1,
    AETH_ERR_SHAPE = -2,
    AETH_ERR_CONFIG = -3,
    AETH_ERR_UNSUPPORTED = -4,
    AETH_ERR_NOT_FOUND = -5,
    AETH_ERR_TIMEOUT = -6,
    AETH_ERR_LINALG = -7,
};

typedef enum { AETH_DTYPE_F32 = 0, AETH_DTYPE_F16 = 1, AETH_DTYPE_BF16 = 2 } aeth_dtype;

/* ======================================================================
 * 1. Reference-compatible symbols (same names, signatures and status codes).
 * ====================================================================== */

/* Replaces galore/kernels/galore_project.cuh:19-29 (galore_project.cu:63-110).
 * R(r x r) = P^T G Q, all fp16 row-major device buffers; temp is the caller's
 * r x n fp16 scratch holding P^T G.  tcgen05 tensor cores, fp32 accumulation.
 * Returns 0, or -1 when m, n or r <= 0. */
int galore_project_forward(const void* G, const void* P, const void* Q, void* R, void* temp, int m, int n, int r,
                           aeth_stream_t stream);

/* Replaces galore/kernels/galore_project.cuh:40-50 (galore_project.cu:112-159).
 * G~(m x n) = P N Q^T; temp is the caller's m x r fp16 scratch holding P N. */
int galore_project_backward(const void* N, const void* P, const void* Q, void* G_tilde, void* temp, int m, int n,
                            int r, aeth_stream_t stream);

/* No counterpart in the reference.  galore_project_forward without the temp
 * argument, for callers that cannot allocate device memory where they call
 * this: code inside another framework's step whose device memory is all held
 * by that framework's caching allocator (a raw cudaMalloc there fails or
 * fragments the pool), or code that must not allocate once a run has started.
 * The r x n fp16 intermediate P^T G lives in a fixed 16 MiB array inside the
 * library (r * n <= 8,388,608), which every GPU that loads the library holds
 * until the process exits; no call allocates or frees anything.
 * Larger r * n returns AETH_ERR_UNSUPPORTED (-4) without touching the GPU.
 * The first call on a device looks up the array's device address (and sets up
 * the library's per-device error word there); make that first call before any
 * stream capture.  All calls on a device share the one array: calls whose
 * work overlaps on the GPU (different streams, or different host threads)
 * race on it and must be serialised by the caller.  The array's previous
 * contents never matter, since the intermediate is fully written before it is
 * read.  Otherwise identical to galore_project_forward (same status codes). */
int galore_project_forward_noalloc(const void* G, const void* P, const void* Q, void* R, int m, int n, int r,
                                   aeth_stream_t stream);

/* Replaces galore/kernels/quantize_state.cuh:12-18 (quantize_state.cu:61-86).
 * scale = max|x| / 127 (1.0 when max|x| == 0), q = clamp(round(x / scale), +-127)
 * with round half away from zero as in the live CPU path (galore/src/quantize.rs:17-26).
 * scale_out is a device float; no host synchronisation.  Returns -1 when n <= 0. */
int galore_quantize_absmax_f32_to_i8(const float* src, int8_t* dst, float* scale_out, int n_elements,
                                     aeth_stream_t stream);

/* Replaces galore/kernels/quantize_state.cuh:20-26 (quantize_state.cu:88-98): dst = q * scale. */
int galore_dequantize_i8_to_f32(const int8_t* src, float* dst, float scale, int n_elements, aeth_stream_t stream);

/* Replaces the stub doublepass/kernels/galore_apply.cuh:22-34 (galore_apply.cu:16-24).
 * Full-rank fused Adam on device buffers, legacy default stream:
 *   g = grad_lr * clip; m = b1 m + (1-b1) g; v = b2 v + (1-b2) g^2;
 *   param -= lr * m_hat / (sqrt(v_hat) + eps)
 * with m_hat = m / (1 - b1^step), v_hat = v / (1 - b2^step) for step >= 1 and
 * m_hat = m, v_hat = v for step <= 0 (galore/src/standard_adamw.rs:84-114).
 * void as in the reference; errors are readable with aeth_last_error(). */
void doublepass_galore_apply(float* param, const float* grad_lr, float* m, float* v, float clip_scale, float beta1,
                             float beta2, float eps, float lr, int n_elements, int step);

/* ======================================================================
 * 2. Optimizer handle: mirrors doublepass::OptimizerBackend
 *    (doublepass/src/lib.rs:62-107) as implemented by GaLoreOptimizer
 *    (galore/src/optimizer.rs:81-403), with device pointers and a stream.
 * ====================================================================== */

typedef enum {
    /* Reference semantics: two-sided R = P^T G Q (r x r), fp32 throughout,
     * per-tensor absmax INT8 m/v (galore/src/optimizer.rs:264-362). */
    AETH_MODE_REF = 0,
    /* B200 semantics: one-sided projection on the smaller dimension,
     * bf16 tensor-core GEMMs, blockwise INT8 m/v, fused NF4 weight write. */
    AETH_MODE_B200 = 1,
} aeth_mode;

typedef enum {
    AETH_CODEC_PER_TENSOR = 0,   /* galore/src/quantize.rs:4-34 */
    AETH_CODEC_BLOCK_LINEAR = 1, /* same formula per block of state_block elements */
    AETH_CODEC_BLOCK_DYNAMIC = 2 /* 8-bit dynamic map per block (Dettmers et al. 2021) */
} aeth_state_codec;

/* GaLoreConfig (galore/src/optimizer.rs:35-61) + AdamWConfig (adamw.rs:8-34)
 * + LayerRankConfig (layer_rank.rs:8-28) + TrainingPlan::max_grad_norm
 * (doublepass/src/plan.rs:197-243) + the B200-mode options. */
typedef struct {
    int mode;                 /* aeth_mode */
    int default_rank;         /* 16 */
    int attn_rank;            /* 32 */
    int mlp_rank;             /* 16 */
    int vector_rank;          /* 8 */
    uint64_t switch_interval; /* 200; 0 holds the projection constant */
    int oversampling;         /* 10 */
    float beta1, beta2, eps;  /* 0.9, 0.999, 1e-8 */
    float lr;                 /* 1e-3 */
    float weight_decay;       /* 0 */
    int scale_lr_by_rank;     /* 0 */
    float max_grad_norm;      /* 1.0 */
    int state_codec;          /* aeth_state_codec; REF mode requires PER_TENSOR */
    int state_block;          /* 2048 */
    int init_projectors;      /* 1: init_random_projection at create; 0: zero, set with aeth_galore_set_projector */
    int svd_refresh;          /* 1: capture gradients and refresh in notify_step as the reference; 0: fixed projectors */
    int power_iters;          /* 0 (the reference); > 0 adds subspace iterations to the refresh */
    int grad_dtype;           /* B200: the gradients' aeth_dtype (BF16).  F32 / F16 allocate the split
                                 path's buffers at create, so no step allocates */
    int ref_gemm;             /* REF: AETH_REF_GEMM_EXACT (the reference's loop order, bit for bit) or
                                 AETH_REF_GEMM_SPLIT3 (tensor cores, fp32 accuracy) */
} aeth_galore_config;

/* REF mode's projection and back-projection (galore/src/project.rs:33-58):
 *   EXACT:  CUDA-core GEMMs that sum each output in the reference's loop order
 *           with separately rounded multiply and add -- bit-identical results.
 *   SPLIT3: tcgen05 GEMMs; each fp32 operand is split exactly into three bf16
 *           terms and the six term products above 2^-24 are summed in fp32 --
 *           within about 1e-6 of the reference (its own rounding error), not
 *           bit-identical.  Parameters whose m, n or rank is not a multiple of
 *           8 stay on the EXACT path. */
enum { AETH_REF_GEMM_EXACT = 0, AETH_REF_GEMM_SPLIT3 = 1 };

typedef struct {
    uint32_t layer_idx;
    const char* name; /* d_wq, d_wk, d_wv, d_wo, d_wg, d_wu, d_wd, d_rms1_w, ... */
    int m, n;         /* weight is m x n row-major (out x in) */
    int rank;         /* 0: LayerRankConfig::rank_for_param (layer_rank.rs:32-40) */
} aeth_param_spec;

typedef struct {
    int m, n, rank;
    int side;               /* 0 two-sided (REF), 1 left P (m<n), 2 right Q (m>=n) */
    int64_t state_elems;    /* r*r (REF) or r*max(m,n) (B200) */
    int64_t state_blocks;   /* number of INT8 scales per moment */
    uint32_t layer_idx;
} aeth_param_info;

typedef enum {
    AETH_WEIGHT_NONE = 0, /* no in-place update: only delta_out (take_weight_delta) */
    AETH_WEIGHT_F32 = 1,  /* dense fp32 m x n, updated in place: w -= delta */
    AETH_WEIGHT_NF4 = 2,  /* NF4 (64-element blocks, fp32 absmax), dequant -> update -> requant in place */
} aeth_weight_kind;

typedef struct {
    int kind;         /* aeth_weight_kind */
    void* data;       /* F32: m*n floats; NF4: m*n/2 packed bytes (high nibble = even element) */
    float* absmax;    /* NF4: m*n/64 floats */
    float* delta_out; /* optional m*n fp32 delta (lr applied) = GaLoreOptimizer::take_weight_delta */
    float* prequant_out; /* optional m*n fp32 updated weight before NF4 requantisation (testing) */
} aeth_weight_ref;

typedef struct aeth_galore_ctx aeth_galore_ctx;

void aeth_galore_config_default(aeth_galore_config* cfg);

/* GaLoreOptimizer::new (optimizer.rs:81-133): registers the parameters,
 * allocates all per-parameter device state on `device`, initialises P/Q with
 * init_random_projection (seeds layer*17 and layer*31, optimizer.rs:419-448).
 * Synchronous. */
int aeth_galore_create(const aeth_galore_config* cfg, const aeth_param_spec* specs, int n_specs, int device,
                       aeth_galore_ctx** out);
int aeth_galore_destroy(aeth_galore_ctx* ctx);
/* Index of (layer_idx, name), or AETH_ERR_NOT_FOUND. */
int aeth_galore_find(const aeth_galore_ctx* ctx, uint32_t layer_idx, const char* name);
int aeth_galore_param_info(const aeth_galore_ctx* ctx, int idx, aeth_param_info* out);
int aeth_galore_num_params(const aeth_galore_ctx* ctx);

/* OptimizerBackend::project_and_accumulate (optimizer.rs:264-292):
 * accum += projection(grad).  grad is m*n device values of `grad_dtype`.
 * REF: F32, or BF16 / F16 widened exactly.  B200: BF16 goes to the tensor
 * cores as it is; F32 and F16 are never narrowed: each gradient is split
 * exactly into three (F32) or two (F16) bf16 terms, stacked along the
 * contraction and projected in one launch against the projector repeated
 * that many times (16-byte aligned gradient, n % 8 == 0).  The terms go
 * through one staging buffer of the optimizer (terms * m * n bf16 of the
 * largest such parameter), so F32 / F16 projections of one optimizer must be
 * issued on one stream.  The buffer is allocated at create when
 * config.grad_dtype declares F32 / F16; otherwise on the first such call,
 * which then synchronises the stream and is refused (AETH_ERR_UNSUPPORTED)
 * while the stream is being captured into a CUDA graph. */
int aeth_galore_project_accumulate(aeth_galore_ctx* ctx, int idx, const void* grad, int grad_dtype,
                                   aeth_stream_t stream);
/* OptimizerBackend::lowrank_grad_sqnorm (optimizer.rs:294-301): sum of squares
 * of the accumulator in f64.  The _device form writes it to a device double
 * without synchronising; the host form synchronises the stream. */
int aeth_galore_sqnorm_device(aeth_galore_ctx* ctx, int idx, double* out_dev, aeth_stream_t stream);
int aeth_galore_sqnorm(aeth_galore_ctx* ctx, int idx, double* out_host, aeth_stream_t stream);
/* Global clip of doublepass/src/hook.rs:139-203 on the device:
 * *clip_dev = min(1, max_norm / (sqrt(sum_i sq[i]) + 1e-6)) over n device doubles. */
int aeth_clip_coeff_device(const double* sq_dev, int n, float max_norm, float* clip_dev, double* gnorm_dev,
                           aeth_stream_t stream);
/* OptimizerBackend::apply_update (optimizer.rs:303-362) with the clip taken
 * from the host (clip) or from device memory (clip_dev, if not NULL). */
int aeth_galore_apply_update(aeth_galore_ctx* ctx, int idx, float clip, const float* clip_dev,
                             const aeth_weight_ref* w, aeth_stream_t stream);
/* OptimizerBackend::zero_accum (adamw.rs:107-109). */
int aeth_galore_zero_accum(aeth_galore_ctx* ctx, int idx, aeth_stream_t stream);
/* OptimizerBackend::notify_step (optimizer.rs:373-398): records the step,
 * then runs the pending subspace refreshes (process_pending_svd,
 * optimizer.rs:208-246).  With svd_refresh = 1, project_accumulate (and
 * aeth_galore_step) capture the full gradient of every parameter -- summed
 * over calls -- when step + 1 == 1 or should_switch_subspace(step + 1,
 * switch_interval) (optimizer.rs:264-292, randomized_svd.rs:273-276).  Each
 * captured parameter then gets new projectors from aeth_randomized_svd with
 * seed = step * 0x9E3779B9 (wrapping), its own rank and config.oversampling
 * (B200 mode keeps the projector of its side), and a reset Adam state; the
 * optimizer version goes up by one when all succeed.  The first failure is
 * returned and ends the refresh (later captures are dropped, as in the
 * reference).  notify_step uses the legacy default stream and waits for the
 * refresh; notify_step_async enqueues it on `stream` (it still waits once per
 * refreshed parameter for the factorisation status). */
int aeth_galore_notify_step(aeth_galore_ctx* ctx, uint64_t step);
int aeth_galore_notify_step_async(aeth_galore_ctx* ctx, uint64_t step, aeth_stream_t stream);
uint64_t aeth_galore_step_count(const aeth_galore_ctx* ctx);
/* optimizer_version (optimizer.rs:249-253): subspace refreshes completed. */
uint64_t aeth_galore_version(const aeth_galore_ctx* ctx);

/* optimizer_states.bin (galore/src/state_file.rs:1-580; flush_all_to_file,
 * optimizer.rs:180-192; GaLoreOptimizer::open, :135-176).  REF mode writes
 * and reads the reference's version 2 byte for byte: P and Q as FP16 through
 * galore's own conversion (project.rs:135-185), INT8 m/v, one scale each, the
 * Adam constants and the step count in the header; layers in parameter order.
 * Loading also reads version 1 files.  B200 mode writes version 3 (no
 * reference counterpart), which keeps the one-sided state losslessly: the bf16
 * projector of the parameter's side, INT8 m/v and their block scales.
 * load_state checks every layer's m, n and rank (and, for version 3, side,
 * codec, block and state size) against the context (AETH_ERR_SHAPE), installs
 * the state, zeroes the accumulators, and adopts the file's step count and
 * beta1, beta2, eps, as the reference's open does.  Both wait on `stream`.
 * Status: AETH_ERR_NOT_FOUND when the file cannot be opened, AETH_ERR_CONFIG
 * for I/O failures, a bad magic / version or a section outside the file.
 * load_state checks the whole file before it installs anything, so those
 * errors leave the optimizer unchanged; a CUDA error while the checked
 * sections are installed leaves its state undefined. */
int aeth_galore_save_state(aeth_galore_ctx* ctx, const char* path, aeth_stream_t stream);
int aeth_galore_load_state(aeth_galore_ctx* ctx, const char* path, aeth_stream_t stream);

/* Device randomized SVD, K8 (randomized_svd_projections, randomized_svd.rs:
 * 76-149; the reference's device entry point randomized_svd_on_device,
 * :282-298, routes to an unimplemented kernel).  g: m x n f32 row-major;
 * p_out (m x r) and q_out (n x r) f32 row-major, either may be NULL.
 * power_iters > 0 adds subspace iterations, a B200 extension (the reference
 * ignores its power_iters).  Returns AETH_ERR_CONFIG when rank == 0 or
 * rank + oversampling > min(m, n) (GaLoreError::Config) and AETH_ERR_LINALG
 * for a rank-deficient sketch (GaLoreError::Linalg).  Waits on `stream` once
 * to read the factorisation status. */
int aeth_randomized_svd(const float* g, int m, int n, int rank, int oversampling, int power_iters, uint64_t seed,
                        float* p_out, float* q_out, aeth_stream_t stream);
/* Two steps of it on their own.  aeth_rsvd_omega: `count` Gaussians of
 * Rng::new(seed).next_gaussian() in order (randomized_svd.rs:38-66), every
 * thread starting from the jumped-ahead xorshift64 state.  aeth_rsvd_jacobi:
 * jacobi_eigenvectors (randomized_svd.rs:210-271) on the n x n f32 matrix
 * `mat` (overwritten) with the eigenvector estimate in u (n x n). */
/* aeth_randomized_svd with a bf16 or f32 g (g_dtype) and, with fast != 0,
 * every product on the tensor cores over exact bf16 terms (fp32-accurate, not
 * the reference's summation order; a bf16 g is its own single term) when m, n,
 * rank and rank + oversampling are multiples of 8 -- otherwise, and with
 * fast == 0, the exact-order path of aeth_randomized_svd. */
int aeth_randomized_svd_ex(const void* g, int g_dtype, int m, int n, int rank, int oversampling, int power_iters,
                           uint64_t seed, int fast, float* p_out, float* q_out, aeth_stream_t stream);
int aeth_rsvd_omega(uint64_t seed, int64_t count, float* out, aeth_stream_t stream);
int aeth_rsvd_jacobi(float* mat, int n, float* u, aeth_stream_t stream);
/* Steps 2-5 of randomized_svd_projections (randomized_svd.rs:95-149) from the
 * caller's sketch omega (n x (rank + oversampling) f32 row-major, device
 * memory) instead of step 1's draw; no power iterations, as in the reference.
 * fast == 0 runs the exact-order path, whose products and Gram-Schmidt are the
 * reference's own loops: with the sketch the reference drew on the host (its
 * Box-Muller goes through the host libm's ln and cos), P and Q equal the
 * reference's bit for bit.  Statuses as aeth_randomized_svd_ex. */
int aeth_randomized_svd_sketch(const void* g, int g_dtype, int m, int n, int rank, int oversampling,
                               const float* omega, int fast, float* p_out, float* q_out, aeth_stream_t stream);

/* Whole-layer step of deferred_apply_with_clip (hook.rs:115-203) for a
 * single micro-batch: for each listed parameter project_and_accumulate, then
 * the exact global-norm clip on the device, then apply_update + zero_accum.
 * When `sq_hook` is set it is called between the sqnorm and apply phases with
 * the device array of per-parameter sqnorms (length n) so a multi-GPU caller
 * can all-reduce it in place on `stream`.
 * The call can be recorded into a CUDA graph (stream capture) and replayed
 * once per step: it neither synchronises nor allocates, and its counters live
 * on the device.  While capturing it records no phase events, and it returns
 * AETH_ERR_UNSUPPORTED when the subspace refresh is on, whose gradient capture
 * follows the host step count. */
typedef int (*aeth_sqnorm_hook)(double* sq_dev, int n, aeth_stream_t stream, void* user);
int aeth_galore_step(aeth_galore_ctx* ctx, int n, const int* idx, const void* const* grads, int grad_dtype,
                     const aeth_weight_ref* weights, aeth_sqnorm_hook sq_hook, void* hook_user, float* clip_dev_out,
                     aeth_stream_t stream);

/* The same step for a whole model whose gradients arrive layer by layer, as
 * doublepass's backward produces them: backward.rs:509-521 calls
 * project_and_accumulate for each layer's parameters as soon as that layer's
 * gradients exist, and the clip and the update then run once for the model
 * (deferred_apply_with_clip, hook.rs:115-203).  A full gradient set of a
 * 70B model (137 GB in bf16) is never resident at once; only the projected
 * accumulators are.
 *   aeth_galore_project_layer: project_and_accumulate for the n listed
 *     parameters (normally one layer's matrices), in grouped launches.  The
 *     gradient buffers can be refilled once the work this call enqueued on
 *     `stream` has run (record an event after it).
 *   aeth_galore_finish_step: the exact global-norm clip over the n listed
 *     parameters -- every parameter of the model that this GPU owns -- in one
 *     squared-norm launch (n <= 1024 with a clip group; the clip group
 *     exchanges the sum with the peer GPUs inside that launch), then Adam for
 *     all of them, then the back-projection with the weight write, zeroing
 *     the accumulators.  weights[i], sq_hook and clip_dev_out as in
 *     aeth_galore_step.
 * Calling project_layer for every layer and then finish_step gives the same
 * bits as aeth_galore_step over the same parameters.  Both record into a
 * CUDA graph under the conditions aeth_galore_step states. */
int aeth_galore_project_layer(aeth_galore_ctx* ctx, int n, const int* idx, const void* const* grads, int grad_dtype,
                              aeth_stream_t stream);
int aeth_galore_finish_step(aeth_galore_ctx* ctx, int n, const int* idx, const aeth_weight_ref* weights,
                            aeth_sqnorm_hook sq_hook, void* hook_user, float* clip_dev_out, aeth_stream_t stream);

/* The subspace refresh of a streamed step (B200 mode; no reference
 * counterpart as an entry point: the reference captures every parameter's
 * full gradient during project_and_accumulate and refreshes in notify_step,
 * optimizer.rs:208-246, 264-292, 373-398, which a 70B sweep cannot hold).
 * For each listed parameter, the randomized SVD of this gradient (rank,
 * config.oversampling and config.power_iters; seed (step + 1) * 0x9E3779B9,
 * the step notify_step will record) runs on the tensor cores right away and
 * its projector is kept aside; the next notify_step installs it and resets
 * the parameter's Adam state, as the reference's refresh does, and counts one
 * optimizer version.  The step's own back-projection still uses the old
 * projector.  Call it on refresh steps (step + 1 == 1 or a multiple of
 * switch_interval), with svd_refresh = 0, after or before project_layer for
 * the same gradients.  Allocates (workspace, and the pending projector on
 * first use) and waits on `stream` once per parameter for the factorisation
 * status; refused while the stream is being captured. */
int aeth_galore_refresh_layer(aeth_galore_ctx* ctx, int n, const int* idx, const void* const* grads, int grad_dtype,
                              aeth_stream_t stream);
/* The bf16 projector of a B200 parameter's side (rows x cols = s x rank,
 * row-major, device memory owned by the optimizer): for broadcasting a
 * refreshed projector from its owner (NCCL), read-only. */
int aeth_galore_projector_buffer(aeth_galore_ctx* ctx, int idx, void** proj_bf16, int* rows, int* cols);

/* Per-phase device timing of the step (no reference counterpart).  While
 * enabled, every B200-mode aeth_galore_step, project_layer and finish_step
 * call records CUDA events on its stream at the phase boundaries: projection
 * | squared norms and clip | Adam | back-projection with the weight write.
 * aeth_galore_phase_times waits for the recorded calls, adds their elapsed
 * milliseconds per phase into ms_out[0..3], stores the number of completed
 * steps (aeth_galore_step and finish_step calls) in *steps and forgets them. */
int aeth_galore_set_phase_timing(aeth_galore_ctx* ctx, int enable);
int aeth_galore_phase_times(aeth_galore_ctx* ctx, double ms_out[4], int* steps);

/* Global clip over a group of GPUs through peer memory (B200 mode; replaces
 * the f64 all-reduce of hook.rs:149-186, no reference counterpart as an
 * API).  Each rank's aeth_galore_step then computes its local sum of squared
 * norms, writes it into a slot on every other rank's GPU (NVLink stores),
 * waits for theirs and forms the clip from the total added in rank order, so
 * every rank gets the same bits, all inside the one squared-norm launch.
 *   aeth_galore_clip_handle allocates this context's slots for a group of
 *   `world` GPUs (zeroed) and writes their 64-byte CUDA IPC handle;
 *   aeth_galore_set_clip_group opens the other ranks' handles (`handles`:
 *   world x 64 bytes in rank order) and zeroes the own slots.  world == 1
 *   leaves the group.  After every rank's set_clip_group returned, the ranks
 *   must meet at a host barrier before the first step; after that, every rank
 *   calls aeth_galore_step the same number of times, without a hook.
 *   aeth_galore_set_clip_group_ptrs takes the slot pointers directly (own
 *   slots at `rank`, from aeth_galore_clip_slots), for callers that map the
 *   peer memory themselves.
 * Each wait is bounded by timeout_ns (0: two seconds).  When a peer's sum
 * does not arrive, the step uses clip 0 (this step's gradients are dropped,
 * the moments decay), AETH_DEVERR_TIMEOUT_PEER is set in the device error
 * word, and the ranks' optimizer states may differ: the caller restores them
 * from the last saved state. */
int aeth_galore_clip_handle(aeth_galore_ctx* ctx, int world, void* handle_out);
int aeth_galore_set_clip_group(aeth_galore_ctx* ctx, int rank, int world, const void* handles, uint64_t timeout_ns);
int aeth_galore_set_clip_group_ptrs(aeth_galore_ctx* ctx, int rank, int world, void* const* slots,
                                    uint64_t timeout_ns);
int aeth_galore_clip_slots(aeth_galore_ctx* ctx, void** slots_out);

/* Projector access.  REF: P (m x r) and Q (n x r).  B200: only the projector
 * of the chosen side (P for m < n, Q for m >= n; the other pointer is ignored).
 * fp32 device buffers.  set_projector resets the Adam state, as the subspace
 * switch does (optimizer.rs:236-238). */
int aeth_galore_set_projector(aeth_galore_ctx* ctx, int idx, const float* P, const float* Q, aeth_stream_t stream);
int aeth_galore_get_projector(aeth_galore_ctx* ctx, int idx, float* P, float* Q, aeth_stream_t stream);
/* State access (device buffers): m8, v8 (state_elems), scales (state_blocks). */
int aeth_galore_get_state(aeth_galore_ctx* ctx, int idx, int8_t* m8, int8_t* v8, float* m_scales, float* v_scales,
                          aeth_stream_t stream);
int aeth_galore_set_state(aeth_galore_ctx* ctx, int idx, const int8_t* m8, const int8_t* v8, const float* m_scales,
                          const float* v_scales, aeth_stream_t stream);
int aeth_galore_get_accum(aeth_galore_ctx* ctx, int idx, float* accum, aeth_stream_t stream);

/* ======================================================================
 * 3. Stand-alone kernels of the path.
 * ====================================================================== */

/* NF4 dequantise (shard_engine/src/nf4.rs:37-83, quantizer.py:55-75): out[i] =
 * CODES[nib(i)] * absmax[i / block]; out_dtype F32 (the exact product), F16
 * (RNE, as nf4.rs:78) or BF16 (RNE). */
int aeth_nf4_dequant(const uint8_t* packed, const float* absmax, int64_t n, int block, void* out, int out_dtype,
                     aeth_stream_t stream);
/* NF4 quantise (quantizer.py:21-53), bit-exact: absmax per block (raw),
 * argmin over the 16 codes of x / max(absmax, 1e-8), first index on ties.
 * x is F32, F16 or BF16.  Trailing elements of the last block are treated as 0. */
int aeth_nf4_quant(const void* x, int x_dtype, int64_t n, int block, uint8_t* packed, float* absmax,
                   aeth_stream_t stream);

/* INT8 state codecs.  PER_TENSOR: scales[0]; BLOCK_*: one scale per block.
 * is_signed selects the signed or unsigned dynamic map. */
int aeth_int8_quantize(const float* x, int64_t n, int codec, int block, int is_signed, int8_t* q, float* scales,
                       aeth_stream_t stream);
int aeth_int8_dequantize(const int8_t* q, const float* scales, int64_t n, int codec, int block, int is_signed,
                         float* out, aeth_stream_t stream);
/* The 256-entry dynamic map used by AETH_CODEC_BLOCK_DYNAMIC (host copy). */
int aeth_dynamic_map(int is_signed, float out[256]);
/* Self-checks with no reference counterpart.  Each runs float bit patterns
 * through a fast device path and the plain definition it replaces, on the
 * current device, and stores the number of disagreements in *mismatches
 * (synchronous):
 *   DMAP_SIGNED / DMAP_UNSIGNED: all 2^32 patterns through the bucket-table
 *     dynamic-map encoder of the Adam and LOMO kernels against the binary
 *     search over the map;
 *   ADAM_DIR: all 2^32 patterns; the bf16 Adam direction from approximate
 *     sqrt and reciprocal against IEEE sqrt and division (the pattern is v; m
 *     is hashed from it);
 *   NF4_CLASSIFY: for block absmax values 1, 0.37, 0.02, 3.3e-5, 1e-9 (below
 *     the 1e-8 clamp) and 7.7e30, every x with |x| <= absmax, both signs,
 *     through the fused epilogues' NF4 classifier (bucket shuffle, near-window
 *     repair) against the reference's argmin over IEEE x / absmax. */
enum {
    AETH_SELFCHECK_DMAP_SIGNED = 0,
    AETH_SELFCHECK_DMAP_UNSIGNED = 1,
    AETH_SELFCHECK_ADAM_DIR = 2,
    AETH_SELFCHECK_NF4_CLASSIFY = 3
};
int aeth_selfcheck(int which, unsigned long long* mismatches);

/* LOMO fused full-rank update over a flat NF4 tensor (Lv et al. 2023):
 * aeth_lomo_sqnorm adds sum(g^2) (f64) into *sq_dev; aeth_lomo_update reads
 * the global sum from sq_dev (after any cross-tensor / cross-rank reduction),
 * clips with min(1, max_norm / (sqrt(sq) + 1e-6)), updates the blockwise INT8
 * momentum m = beta m + g*clip, writes w = w - lr m and requantises w to NF4.
 * grad is bf16; n must be a multiple of 64 and of `block` / 64. */
int aeth_lomo_sqnorm(const void* grad_bf16, int64_t n, double* sq_dev, aeth_stream_t stream);

/* Streamed-weight decode, the step before the optimizer path in the streaming
 * pipeline (QuantizedDecoder, flowcast/src/decode.rs:63-104): quantised
 * weights to f16 with flowcast's own f32 -> f16 conversion (decode.rs:191-210:
 * mantissa truncation; +-0 below the normal range, +-inf above it).
 *   aeth_fc_decode_int8: out[i] = f16(src[i] * scales[ch]), ch = i / max(n /
 *     num_channels, 1) (0 when num_channels == 0), a channel at or past
 *     n_scales decoding with 1.0 (decode_int8_to_fp16).
 *   aeth_fc_decode_nf4: nbytes packed NF4 bytes, LOW nibble first, one absmax
 *     for the tensor -> 2 * nbytes f16 values (decode_int4_to_fp16).
 *     shard_engine's layout (high nibble first, 64-element blocks) is
 *     aeth_nf4_dequant's.
 * Device pointers: src 4-byte aligned, out 8-byte (INT8) or 16-byte (NF4)
 * aligned (AETH_ERR_UNSUPPORTED otherwise). */
int aeth_fc_decode_int8(const int8_t* src, int64_t n, const float* scales, int64_t n_scales, int num_channels,
                        uint16_t* out_f16, aeth_stream_t stream);
int aeth_fc_decode_nf4(const uint8_t* src, int64_t nbytes, float absmax, uint16_t* out_f16, aeth_stream_t stream);
/* The step after it: apply_galore_bf16_update (doublepass/src/precision.rs:
 * 184-217).  master[i] += delta[i], then stochastic rounding to bf16 with the
 * 16 bits drawn from the MMIX LCG for element i, in element order; master
 * keeps the widened bf16 value and bf16_out (optional) the bf16 bits.
 * *rng_state (host memory) is the state before element 0 and is advanced past
 * element n - 1 on return, as the sequential loop leaves it.  master and
 * delta 16-byte aligned, bf16_out 8-byte aligned. */
int aeth_bf16_sr_update(float* master, const float* delta, int64_t n, uint64_t* rng_state, uint16_t* bf16_out,
                        aeth_stream_t stream);
int aeth_lomo_update(const void* grad_bf16, int64_t n, const double* sq_dev, float max_norm, float lr, float beta,
                     int codec, int block, int8_t* mom8, float* mom_scales, uint8_t* w_packed, float* w_absmax,
                     float* prequant_out, aeth_stream_t stream);

/* ======================================================================
 * 4. Errors and build information.
 * ====================================================================== */
const char* aeth_status_string(int status);
/* Last error recorded on the calling thread (for void entry points). */
int aeth_last_error(void);
/* Reads and clears the device-side error word set by bounded waits on
 * `device` (synchronises the device).  Returns AETH_OK or AETH_ERR_TIMEOUT. */
int aeth_device_error(int device);
/* The same, returning the word's bits: which wait gave up. */
#define AETH_DEVERR_TIMEOUT_TMA 1u
#define AETH_DEVERR_TIMEOUT_MMA 2u
#define AETH_DEVERR_TIMEOUT_EPI 4u
#define AETH_DEVERR_BAD_ARG 8u
#define AETH_DEVERR_TIMEOUT_PEER 16u
int aeth_device_error_bits(int device, uint32_t* bits);
/* Library version string. */
const char* aeth_version(void);

#ifdef __cplusplus
}
#endif
#endif /* AETH_GALORE_H */
