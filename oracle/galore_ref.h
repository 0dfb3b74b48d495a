/*
 * galore_ref.h -- CPU oracle for the per-layer optimizer step.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing under aethelstream_b200/ links, loads or
 * calls this code; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline legs use it, and only as the checker or as the timed CPU baseline.
 *
 * Two groups of functions:
 *   ref_*  -- line-by-line restatements of the reference's CPU path (Rust
 *             `galore` crate, `shard_engine` NF4 code).  Same loop order, f32
 *             accumulation, no FMA contraction (the file is compiled with
 *             -ffp-contract=off, matching Rust, which never fuses a*b+c).
 *   b2_*   -- the B200 build's extended semantics (one-sided projection,
 *             2048-element blockwise INT8 state, NF4 requantisation of the
 *             updated weight, LOMO).  These have no reference implementation;
 *             they are written so that they reduce to the ref_* functions
 *             where the reference defines the behaviour (see each comment).
 *
 * Pinning: the NF4 functions are pinned bit-for-bit against fixtures made by
 * running the reference's own quantizer.py (tests/golden/make_golden.py).
 * The GaLore functions are pinned by re-running the reference test suite's
 * assertions (galore/tests/test_galore_projection_roundtrip.rs,
 * test_galore_quantize_roundtrip.rs and the crate's unit tests) on them; the
 * Rust crate cannot be compiled in this image, so no reference-generated
 * GaLore vectors exist.  The b2_* functions are parity-unpinned except where
 * they reduce to ref_* (block >= tensor, linear codec).
 */
#ifndef AETH_GALORE_REF_H
#define AETH_GALORE_REF_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- NF4 (shard_engine/src/nf4.rs, shard_engine/python/pipeline/quantizer.py) ---- */
extern const float REF_NF4_CODES[16];
void ref_nf4_quantize(const float* x, int64_t n, int block, uint8_t* packed, float* absmax);
void ref_nf4_dequant_f32(const uint8_t* packed, const float* absmax, int64_t n, int block, float* out);
void ref_nf4_dequant_f16(const uint8_t* packed, const float* absmax, int64_t n, int block, uint16_t* out);
uint16_t ref_f32_to_f16_rne(float x);
uint16_t ref_f32_to_bf16_rne(float x);
float ref_bf16_to_f32(uint16_t b);

/* ---- per-tensor absmax INT8 (galore/src/quantize.rs) ---- */
float ref_absmax_scale(const float* x, int64_t n);
float ref_quantize_absmax(const float* x, int64_t n, int8_t* q);
void ref_dequantize_absmax(const int8_t* q, float scale, int64_t n, float* out);

/* ---- projections (galore/src/project.rs) ---- */
void ref_matmul_f32(const float* a, const float* b, float* c, int m, int k, int n);
void ref_project_forward(const float* g, const float* p, const float* q, float* r_out, int m, int n, int r);
void ref_project_backward(const float* nm, const float* p, const float* q, float* g_out, int m, int n, int r);
double ref_projection_roundtrip_error(const float* g, const float* p, const float* q, int m, int n, int r);
/* Row-sampled variants used to time the reference loops on a bounded sample. */
void ref_project_forward_rows(const float* g, const float* p, const float* q, float* temp, int m, int n, int r,
                              int i0, int i1);
void ref_project_backward_rows(const float* temp_mr, const float* q, float* g_out, int m, int n, int r,
                               int i0, int i1);

/* ---- low-rank Adam (galore/src/adamw.rs) ---- */
void ref_adamw_inner_update(const float* accum, float* mom, float* var, int64_t n,
                            float b1, float b2, float eps, float* normalized);
float ref_effective_lr(float lr, int scale_by_rank, int rank);

/* One apply_update of GaLoreOptimizer (galore/src/optimizer.rs:303-362) for one
 * parameter.  State in/out: m8, v8 (r*r), *scale_m, *scale_v.  weight_delta: m*n. */
void ref_galore_apply_update(const float* grad_accum, const float* p, const float* q,
                             int8_t* m8, int8_t* v8, float* scale_m, float* scale_v,
                             int m, int n, int r, float clip,
                             float b1, float b2, float eps, float lr, int scale_by_rank,
                             float* normalized_out, float* weight_delta);

/* init_random_projection (galore/src/optimizer.rs:419-448) */
void ref_init_random_projection(int rows, int cols, uint32_t seed, float* out);
/* LayerRankConfig::rank_for_param (galore/src/layer_rank.rs:32-40) */
int ref_rank_for_param(const char* name, int m, int n, int default_rank, int attn_rank, int mlp_rank,
                       int vector_rank);
/* global clip coefficient (doublepass/src/hook.rs:184-187) */
float ref_clip_coeff(double gsq, float max_norm);
double ref_sqnorm_f64(const float* x, int64_t n);
/* should_switch_subspace (galore/src/randomized_svd.rs:273-276) */
int ref_should_switch(uint64_t step, uint64_t interval);
/* galore's half conversion for the state file (galore/src/project.rs:135-185). */
uint16_t ref_galore_f32_to_f16(float x);
float ref_galore_f16_to_f32(uint16_t h);
/* Randomized SVD refresh (galore/src/randomized_svd.rs:38-271). */
float ref_rsvd_gaussian(uint64_t* state);
void ref_rsvd_omega(uint64_t seed, int64_t count, float* out);
void ref_rsvd_jacobi(float* mat, int n, float* u);
int ref_randomized_svd(const float* g, int m, int n, int r, int oversampling, uint64_t seed, float* p_out,
                       float* q_out);
/* The same from a given n x (r + oversampling) row-major sketch omega. */
int ref_randomized_svd_sketch(const float* g, int m, int n, int r, int oversampling, const float* omega,
                              float* p_out, float* q_out);

/* StandardAdamW::apply_update (galore/src/standard_adamw.rs:84-114), plus the
 * bias-corrected form documented for doublepass_galore_apply's `step` argument
 * (doublepass/kernels/galore_apply.cuh:22-34).  step <= 0: no bias correction. */
void ref_full_adam_apply(float* param, const float* grad, float* m, float* v, int64_t n,
                         float clip, float b1, float b2, float eps, float lr, int step);

/* ---- B200-mode extensions (parity unpinned unless noted) ---- */
enum { B2_CODEC_LINEAR = 0, B2_CODEC_DYNAMIC = 1 };
void b2_dynamic_map(int is_signed, float out[256]);
void b2_block_quantize(const float* x, int64_t n, int block, int codec, int is_signed, int8_t* q, float* scales);
void b2_block_dequantize(const int8_t* q, const float* scales, int64_t n, int block, int codec, int is_signed,
                         float* out);
int b2_side_is_right(int m, int n);
/* R (l x r, row-major) += contraction of g (m x n) with proj (s x r) over the small dim. */
void b2_project_accumulate(const float* g, const float* proj, float* racc, int m, int n, int r);
/* Adam on the l x r state; writes the bf16-rounded N (as float values). */
void b2_adam_state(const float* racc, int8_t* m8, int8_t* v8, float* mscale, float* vscale, int64_t count,
                   int block, int codec, float clip, float b1, float b2, float eps, float* n_bf16_out);
/* Weight update + NF4 requant from the (bf16) N and projector. */
void b2_apply_weight(const float* n_bf16, const float* proj, int m, int n, int r,
                     const uint8_t* w_packed, const float* w_absmax, float lr, float wd,
                     uint8_t* w_packed_out, float* w_absmax_out, float* w_prequant_out, float* dw_out);
/* NF4 requantisation of already-updated fp32 values (used to pin the GPU's
 * requant bit-for-bit on the GPU's own pre-quant values). */
void b2_nf4_requant(const float* w, int64_t n, uint8_t* packed, float* absmax);

/* ---- Streamed-weight decode (flowcast) and the BF16 stochastic-rounding write-back ---- */
/* flowcast/src/decode.rs:191-210: f32 -> f16 by exponent rebias and mantissa
 * truncation; exponents below the f16 normal range give +-0, above it +-inf;
 * NaN keeps the quiet bit only. */
uint16_t fc_f32_to_f16(float v);
/* decode.rs:63-86: out[i] = f16(i8 * scale[i / (n / num_channels)]); a
 * channel without a scale (index >= n_scales) uses 1.0. */
void fc_decode_int8_to_f16(const int8_t* src, int64_t n, const float* scales, int64_t n_scales, int num_channels,
                           uint16_t* out);
/* decode.rs:88-104: two codes per byte, LOW nibble first, per-tensor absmax. */
void fc_decode_int4_to_f16(const uint8_t* src, int64_t nbytes, float absmax, uint16_t* out);
/* doublepass/src/precision.rs:212-217: Knuth MMIX LCG; returns bits 33-48. */
uint16_t dp_lcg_next(uint64_t* state);
/* precision.rs:124-136 */
uint16_t dp_stochastic_round_to_bf16(float v, uint16_t rand_bits);
/* precision.rs:184-202: master += delta, then stochastic rounding to bf16
 * with one LCG draw per element in order; master holds the widened value. */
void dp_apply_galore_bf16_update(float* master, const float* delta, int64_t n, uint64_t* rng);

/* LOMO fused full-rank SGD with INT8 momentum and NF4 requantisation. */
double b2_lomo_sqnorm_bf16(const uint16_t* g, int64_t n);
void b2_lomo_update(const uint16_t* g, int64_t n, float clip, float beta, float lr, int block, int codec,
                    int8_t* mom8, float* mom_scales, const uint8_t* w_packed, const float* w_absmax,
                    uint8_t* w_packed_out, float* w_absmax_out, float* w_prequant_out);

#ifdef __cplusplus
}
#endif

/* ---- the galore tests' toy transformer (doublepass_toy.c; test infrastructure) ---- */
int64_t toy_layer_size(int d, int ff);
void toy_init_layer(int d, int ff, int layer, float* w);
void toy_lm_head(int vocab, int d, float* out);
void toy_inputs(int d, int seq, int batch, float* out);
void toy_labels(int seq, int batch, int vocab, uint32_t* out);
float toy_step(int d, int h, int ff, int seq, int bsz, int nl, const float* weights, const float* x_in,
               const float* lm_head, int vocab, int chunk_size, const uint32_t* labels, float* grads);
#endif
