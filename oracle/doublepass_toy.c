/* doublepass_toy.c -- TEST INFRASTRUCTURE (not product code).
 *
 * A restatement, in f32 and in the reference's own loop order, of the small
 * transformer that the galore crate's tests train to exercise the optimizer:
 *   doublepass/src/forward.rs:160-270  single_layer_forward (pre-norm block:
 *       RMSNorm, Q/K/V, softmax attention without a mask, Wo, residual,
 *       RMSNorm, SwiGLU MLP, residual), :64-108 the weight formula;
 *   doublepass/src/math.rs:9-99         matmul_tb, add_vecs, rms_norm_fwd,
 *       softmax_rows, silu_f, silu_grad_f;
 *   doublepass/src/loss.rs:83-377        streaming_cut_ce (online softmax over
 *       vocabulary chunks, mean cross entropy, gradient of the hidden state);
 *   doublepass/src/backward.rs:48-382   single_layer_backward;
 *   galore/tests/common/mod.rs:52-71    make_lm_head, make_inputs, make_labels.
 * Compiled with -ffp-contract=off like galore_ref.c: Rust never fuses a*b+c.
 * Rust's f32 sums (`iter().sum()`, `+=` loops) add left to right; its f32
 * exp/ln/sin/sqrt are the C library's expf/logf/sinf/sqrtf. With these, the
 * per-step losses and gradients equal the reference's bit for bit, which the
 * tests check against the loss curves the reference's own test suite wrote
 * (the JSON files in galore/pyref).
 *
 * Weight layout of one layer (floats, in this order): rms1_w d, wq d*d,
 * wk d*d, wv d*d, wo d*d, rms2_w d, wg ff*d, wu ff*d, wd d*ff -- the
 * reference's BlockWeights fields, each row-major as stored there.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "galore_ref.h"

static int64_t toy_layer_floats(int d, int ff) { return 2 * (int64_t)d + 4 * (int64_t)d * d + 3 * (int64_t)ff * d; }

int64_t toy_layer_size(int d, int ff) { return toy_layer_floats(d, ff); }

/* BlockWeights::from_formula_layered (forward.rs:87-107): sin in f64, cast. */
void toy_init_layer(int d, int ff, int layer, float* w) {
    const double off = (double)layer * 100.0;
    const int64_t sizes[9] = {d, (int64_t)d * d, (int64_t)d * d, (int64_t)d * d, (int64_t)d * d, d,
                              (int64_t)ff * d, (int64_t)ff * d, (int64_t)d * ff};
    for (int t = 0; t < 9; ++t) {
        const double base = (double)t;
        for (int64_t i = 0; i < sizes[t]; ++i) *w++ = (float)(sin((double)i * 0.137 + base + off) * 0.1);
    }
}

/* make_lm_head, make_inputs, make_labels (galore/tests/common/mod.rs:52-71). */
void toy_lm_head(int vocab, int d, float* out) {
    for (int64_t i = 0; i < (int64_t)vocab * d; ++i) {
        const float x = (float)i * 0.001f - 0.5f;
        out[i] = sinf(x) * 0.05f;
    }
}
void toy_inputs(int d, int seq, int batch, float* out) {
    for (int64_t i = 0; i < (int64_t)seq * batch * d; ++i) out[i] = sinf((float)i * 0.013f) * 0.1f;
}
void toy_labels(int seq, int batch, int vocab, uint32_t* out) {
    for (int i = 0; i < seq * batch; ++i) out[i] = ((uint32_t)i * 7u + 3u) % (uint32_t)vocab;
}

/* ---- math.rs ---- */
static void matmul_tb(const float* a, const float* b, int m, int k, int n, float* c) {
    for (int i = 0; i < m; ++i)
        for (int j = 0; j < n; ++j) {
            float s = 0.0f;
            for (int l = 0; l < k; ++l) s += a[i * k + l] * b[j * k + l];
            c[i * n + j] = s;
        }
}

static void rms_norm_fwd(const float* x, const float* w, int bs, int d, float* y, float* x_hat, float* rms) {
    const float eps = 1e-6f;
    for (int b = 0; b < bs; ++b) {
        float ss = 0.0f;
        for (int i = 0; i < d; ++i) ss += x[b * d + i] * x[b * d + i];
        const float mean_sq = ss / (float)d;
        rms[b] = sqrtf(mean_sq + eps);
        for (int i = 0; i < d; ++i) {
            x_hat[b * d + i] = x[b * d + i] / rms[b];
            y[b * d + i] = x_hat[b * d + i] * w[i];
        }
    }
}

static float silu_f(float x) { return x / (1.0f + expf(-x)); }
static float silu_grad_f(float x) {
    const float sigma = 1.0f / (1.0f + expf(-x));
    return sigma * (1.0f + x * (1.0f - sigma));
}

/* Activations of one layer (SingleLayerFwdOut, forward.rs:110-157). */
typedef struct {
    float *x_in, *rms1, *x_norm1, *h1, *q_heads, *k_heads, *v_heads, *attn_weights, *attn_out, *x2, *rms2, *x_norm2,
        *h2, *gate, *up, *silu_gate, *hidden, *output;
} toy_act;

static float* falloc(int64_t n) { return (float*)calloc((size_t)(n > 0 ? n : 1), sizeof(float)); }

static void act_alloc(toy_act* a, int bs, int d, int ff, int bh, int s, int dh) {
    a->x_in = falloc((int64_t)bs * d); a->rms1 = falloc(bs); a->x_norm1 = falloc((int64_t)bs * d);
    a->h1 = falloc((int64_t)bs * d); a->q_heads = falloc((int64_t)bh * s * dh); a->k_heads = falloc((int64_t)bh * s * dh);
    a->v_heads = falloc((int64_t)bh * s * dh); a->attn_weights = falloc((int64_t)bh * s * s);
    a->attn_out = falloc((int64_t)bs * d); a->x2 = falloc((int64_t)bs * d); a->rms2 = falloc(bs);
    a->x_norm2 = falloc((int64_t)bs * d); a->h2 = falloc((int64_t)bs * d); a->gate = falloc((int64_t)bs * ff);
    a->up = falloc((int64_t)bs * ff); a->silu_gate = falloc((int64_t)bs * ff); a->hidden = falloc((int64_t)bs * ff);
    a->output = falloc((int64_t)bs * d);
}
static void act_free(toy_act* a) {
    float** f[] = {&a->x_in, &a->rms1, &a->x_norm1, &a->h1, &a->q_heads, &a->k_heads, &a->v_heads, &a->attn_weights,
                   &a->attn_out, &a->x2, &a->rms2, &a->x_norm2, &a->h2, &a->gate, &a->up, &a->silu_gate, &a->hidden,
                   &a->output};
    for (size_t i = 0; i < sizeof(f) / sizeof(f[0]); ++i) free(*f[i]);
}

/* single_layer_forward (forward.rs:160-270); w: one layer's weights. */
static void layer_forward(const float* w, const float* input, int bsz, int seq, int d, int h, int ff, toy_act* a,
                          float* tmp_flat, float* tmp_scores) {
    const int bs = bsz * seq, dh = d / h, bh = bsz * h, s = seq;
    const float *rms1_w = w, *wq = rms1_w + d, *wk = wq + d * d, *wv = wk + d * d, *wo = wv + d * d,
                *rms2_w = wo + d * d, *wg = rms2_w + d, *wu = wg + ff * d, *wd = wu + ff * d;
    memcpy(a->x_in, input, sizeof(float) * (size_t)bs * d);
    rms_norm_fwd(input, rms1_w, bs, d, a->h1, a->x_norm1, a->rms1);
    float* heads[3] = {a->q_heads, a->k_heads, a->v_heads};
    const float* mats[3] = {wq, wk, wv};
    for (int t3 = 0; t3 < 3; ++t3) {
        matmul_tb(a->h1, mats[t3], bs, d, d, tmp_flat);
        for (int b = 0; b < bsz; ++b)
            for (int hh = 0; hh < h; ++hh)
                for (int ss = 0; ss < s; ++ss)
                    for (int t = 0; t < dh; ++t)
                        heads[t3][((b * h + hh) * s + ss) * dh + t] = tmp_flat[(b * s + ss) * d + hh * dh + t];
    }
    const float scale = sqrtf((float)dh);
    for (int bi = 0; bi < bh; ++bi)
        for (int s1 = 0; s1 < s; ++s1)
            for (int s2 = 0; s2 < s; ++s2) {
                float dot = 0.0f;
                for (int t = 0; t < dh; ++t) dot += a->q_heads[bi * s * dh + s1 * dh + t] * a->k_heads[bi * s * dh + s2 * dh + t];
                tmp_scores[bi * s * s + s1 * s + s2] = dot / scale;
            }
    /* softmax_rows (math.rs:56-84) */
    for (int r = 0; r < bh * s; ++r) {
        const float* row = tmp_scores + r * s;
        float mx = -INFINITY;
        for (int c = 0; c < s; ++c) mx = fmaxf(mx, row[c]);
        float sum = 0.0f;
        for (int c = 0; c < s; ++c) {
            a->attn_weights[r * s + c] = expf(row[c] - mx);
            sum += a->attn_weights[r * s + c];
        }
        for (int c = 0; c < s; ++c) a->attn_weights[r * s + c] = a->attn_weights[r * s + c] / sum;
    }
    float* aoh = tmp_flat;  /* attn_out_heads, bh*s*dh == bs*d */
    for (int bi = 0; bi < bh; ++bi)
        for (int s1 = 0; s1 < s; ++s1)
            for (int t = 0; t < dh; ++t) {
                float v = 0.0f;
                for (int s2 = 0; s2 < s; ++s2) v += a->attn_weights[bi * s * s + s1 * s + s2] * a->v_heads[bi * s * dh + s2 * dh + t];
                aoh[bi * s * dh + s1 * dh + t] = v;
            }
    for (int b = 0; b < bsz; ++b)
        for (int hh = 0; hh < h; ++hh)
            for (int ss = 0; ss < s; ++ss)
                for (int t = 0; t < dh; ++t) a->attn_out[(b * s + ss) * d + hh * dh + t] = aoh[((b * h + hh) * s + ss) * dh + t];
    matmul_tb(a->attn_out, wo, bs, d, d, tmp_flat);  /* out_proj; dropout p = 0 */
    for (int i = 0; i < bs * d; ++i) a->x2[i] = input[i] + tmp_flat[i];
    rms_norm_fwd(a->x2, rms2_w, bs, d, a->h2, a->x_norm2, a->rms2);
    matmul_tb(a->h2, wg, bs, d, ff, a->gate);
    matmul_tb(a->h2, wu, bs, d, ff, a->up);
    for (int i = 0; i < bs * ff; ++i) {
        a->silu_gate[i] = silu_f(a->gate[i]);
        a->hidden[i] = a->silu_gate[i] * a->up[i];
    }
    matmul_tb(a->hidden, wd, bs, ff, d, tmp_flat);  /* mlp_out */
    for (int i = 0; i < bs * d; ++i) a->output[i] = a->x2[i] + tmp_flat[i];
}

/* single_layer_backward (backward.rs:48-382): gradients into g (same layout as
 * the weights), upstream gradient in `up_in`, input gradient into `d_input`. */
static void layer_backward(const float* w, const toy_act* a, const float* up_in, int bsz, int seq, int d, int h, int ff,
                           float* g, float* d_input) {
    const int bs = bsz * seq, dh = d / h, bh = bsz * h, s = seq;
    const float *rms1_w = w, *wq = rms1_w + d, *wk = wq + d * d, *wv = wk + d * d, *wo = wv + d * d,
                *rms2_w = wo + d * d, *wg = rms2_w + d, *wu = wg + ff * d, *wd = wu + ff * d;
    float *d_rms1_w = g, *d_wq = d_rms1_w + d, *d_wk = d_wq + d * d, *d_wv = d_wk + d * d, *d_wo = d_wv + d * d,
          *d_rms2_w = d_wo + d * d, *d_wg = d_rms2_w + d, *d_wu = d_wg + ff * d, *d_wd = d_wu + ff * d;
    memset(g, 0, sizeof(float) * (size_t)toy_layer_floats(d, ff));
    float* d_x2 = falloc((int64_t)bs * d);
    memcpy(d_x2, up_in, sizeof(float) * (size_t)bs * d);
    const float* d_mlp_out = up_in;
    float* d_hidden = falloc((int64_t)bs * ff);
    for (int i = 0; i < bs; ++i)
        for (int j = 0; j < ff; ++j)
            for (int k = 0; k < d; ++k) d_hidden[i * ff + j] += d_mlp_out[i * d + k] * wd[k * ff + j];
    for (int k = 0; k < d; ++k)
        for (int j = 0; j < ff; ++j)
            for (int i = 0; i < bs; ++i) d_wd[k * ff + j] += d_mlp_out[i * d + k] * a->hidden[i * ff + j];
    float* d_gate = falloc((int64_t)bs * ff);
    float* d_up = falloc((int64_t)bs * ff);
    for (int i = 0; i < bs * ff; ++i) {
        const float d_silu_gate = d_hidden[i] * a->up[i];
        d_up[i] = d_hidden[i] * a->silu_gate[i];
        d_gate[i] = d_silu_gate * silu_grad_f(a->gate[i]);
    }
    float* d_h2 = falloc((int64_t)bs * d);
    for (int i = 0; i < bs; ++i)
        for (int j = 0; j < ff; ++j)
            for (int k = 0; k < d; ++k) {
                d_h2[i * d + k] += d_gate[i * ff + j] * wg[j * d + k];
                d_wg[j * d + k] += d_gate[i * ff + j] * a->h2[i * d + k];
                d_h2[i * d + k] += d_up[i * ff + j] * wu[j * d + k];
                d_wu[j * d + k] += d_up[i * ff + j] * a->h2[i * d + k];
            }
    const float eps = 1e-6f;
    float* dxn = falloc(d);
    for (int b = 0; b < bs; ++b) {
        for (int i = 0; i < d; ++i) d_rms2_w[i] += d_h2[b * d + i] * a->x_norm2[b * d + i];
        for (int i = 0; i < d; ++i) dxn[i] = d_h2[b * d + i] * rms2_w[i];
        float dot = 0.0f;
        for (int i = 0; i < d; ++i) dot += dxn[i] * a->x_norm2[b * d + i];
        dot = dot / (float)d;
        for (int i = 0; i < d; ++i) {
            const float rpe = fmaxf(a->rms2[b], eps);
            d_x2[b * d + i] += (dxn[i] - a->x_norm2[b * d + i] * dot) / rpe;
        }
    }
    const float* d_out_proj = d_x2;
    float* d_attn_out = falloc((int64_t)bs * d);
    for (int i = 0; i < bs; ++i)
        for (int j = 0; j < d; ++j)
            for (int k = 0; k < d; ++k) {
                d_attn_out[i * d + k] += d_out_proj[i * d + j] * wo[j * d + k];
                d_wo[j * d + k] += d_out_proj[i * d + j] * a->attn_out[i * d + k];
            }
    float* daoh = falloc((int64_t)bh * s * dh);
    for (int b = 0; b < bsz; ++b)
        for (int hh = 0; hh < h; ++hh)
            for (int ss = 0; ss < s; ++ss)
                for (int t = 0; t < dh; ++t) daoh[((b * h + hh) * s + ss) * dh + t] = d_attn_out[(b * s + ss) * d + hh * dh + t];
    float* d_v_heads = falloc((int64_t)bh * s * dh);
    for (int bi = 0; bi < bh; ++bi)
        for (int s2 = 0; s2 < s; ++s2)
            for (int t = 0; t < dh; ++t)
                for (int s1 = 0; s1 < s; ++s1)
                    d_v_heads[bi * s * dh + s2 * dh + t] +=
                        a->attn_weights[bi * s * s + s1 * s + s2] * daoh[bi * s * dh + s1 * dh + t];
    float* d_logits = falloc((int64_t)bh * s * s);
    for (int bi = 0; bi < bh; ++bi)
        for (int s1 = 0; s1 < s; ++s1)
            for (int s2 = 0; s2 < s; ++s2)
                for (int t = 0; t < dh; ++t)
                    d_logits[bi * s * s + s1 * s + s2] += daoh[bi * s * dh + s1 * dh + t] * a->v_heads[bi * s * dh + s2 * dh + t];
    float* d_scores = falloc((int64_t)bh * s * s);
    for (int bi = 0; bi < bh; ++bi)
        for (int s1 = 0; s1 < s; ++s1) {
            float dot = 0.0f;
            for (int s2 = 0; s2 < s; ++s2) dot += d_logits[bi * s * s + s1 * s + s2] * a->attn_weights[bi * s * s + s1 * s + s2];
            for (int s2 = 0; s2 < s; ++s2)
                d_scores[bi * s * s + s1 * s + s2] =
                    a->attn_weights[bi * s * s + s1 * s + s2] * (d_logits[bi * s * s + s1 * s + s2] - dot);
        }
    const float scale = sqrtf((float)dh);
    for (int i = 0; i < bh * s * s; ++i) d_scores[i] /= scale;
    float* d_q_heads = falloc((int64_t)bh * s * dh);
    float* d_k_heads = falloc((int64_t)bh * s * dh);
    for (int bi = 0; bi < bh; ++bi)
        for (int s1 = 0; s1 < s; ++s1)
            for (int t = 0; t < dh; ++t)
                for (int s2 = 0; s2 < s; ++s2) {
                    d_q_heads[bi * s * dh + s1 * dh + t] += d_scores[bi * s * s + s1 * s + s2] * a->k_heads[bi * s * dh + s2 * dh + t];
                    d_k_heads[bi * s * dh + s2 * dh + t] += d_scores[bi * s * s + s1 * s + s2] * a->q_heads[bi * s * dh + s1 * dh + t];
                }
    float* flat[3];
    const float* hsrc[3] = {d_q_heads, d_k_heads, d_v_heads};
    for (int t3 = 0; t3 < 3; ++t3) {
        flat[t3] = falloc((int64_t)bs * d);
        for (int b = 0; b < bsz; ++b)
            for (int hh = 0; hh < h; ++hh)
                for (int ss = 0; ss < s; ++ss)
                    for (int t = 0; t < dh; ++t) flat[t3][(b * s + ss) * d + hh * dh + t] = hsrc[t3][((b * h + hh) * s + ss) * dh + t];
    }
    float* d_h1 = falloc((int64_t)bs * d);
    for (int i = 0; i < bs; ++i)
        for (int j = 0; j < d; ++j)
            for (int k = 0; k < d; ++k) {
                d_h1[i * d + k] += flat[0][i * d + j] * wq[j * d + k];
                d_wq[j * d + k] += flat[0][i * d + j] * a->h1[i * d + k];
                d_h1[i * d + k] += flat[1][i * d + j] * wk[j * d + k];
                d_wk[j * d + k] += flat[1][i * d + j] * a->h1[i * d + k];
                d_h1[i * d + k] += flat[2][i * d + j] * wv[j * d + k];
                d_wv[j * d + k] += flat[2][i * d + j] * a->h1[i * d + k];
            }
    for (int b = 0; b < bs; ++b)
        for (int i = 0; i < d; ++i) d_rms1_w[i] += d_h1[b * d + i] * a->x_norm1[b * d + i];
    for (int b = 0; b < bs; ++b) {
        const float r1e = fmaxf(a->rms1[b], eps);
        float dot = 0.0f;
        for (int i = 0; i < d; ++i) dot += (d_h1[b * d + i] * rms1_w[i]) * a->x_norm1[b * d + i];
        dot = dot / (float)d;
        for (int i = 0; i < d; ++i) {
            const float dn = d_h1[b * d + i] * rms1_w[i];
            const float from_attn = (dn - a->x_norm1[b * d + i] * dot) / r1e;
            d_input[b * d + i] = d_x2[b * d + i] + from_attn;
        }
    }
    free(d_x2); free(d_hidden); free(d_gate); free(d_up); free(d_h2); free(dxn); free(d_attn_out); free(daoh);
    free(d_v_heads); free(d_logits); free(d_scores); free(d_q_heads); free(d_k_heads); free(d_h1);
    for (int t3 = 0; t3 < 3; ++t3) free(flat[t3]);
}

/* One training step's loss and parameter gradients (train_step.rs:59-147 with
 * one micro-batch): full forward, streaming_cut_ce with one vocabulary chunk of
 * chunk_size (loss.rs:83-249, the loss added as (-label + ln sum) + max per
 * token, then divided by the token count), then the layers' backward from the
 * last to the first.  weights / grads: nl consecutive layer blocks. */
float toy_step(int d, int h, int ff, int seq, int bsz, int nl, const float* weights, const float* x_in,
               const float* lm_head, int vocab, int chunk_size, const uint32_t* labels, float* grads) {
    const int bs = bsz * seq, dh = d / h, bh = bsz * h, s = seq;
    const int64_t lf = toy_layer_floats(d, ff);
    toy_act* acts = (toy_act*)calloc((size_t)nl, sizeof(toy_act));
    float* tmp_flat = falloc((int64_t)bs * (d > ff ? d : ff));
    float* tmp_scores = falloc((int64_t)bh * s * s);
    const float* in = x_in;
    for (int l = 0; l < nl; ++l) {
        act_alloc(&acts[l], bs, d, ff, bh, s, dh);
        layer_forward(weights + l * lf, in, bsz, seq, d, h, ff, &acts[l], tmp_flat, tmp_scores);
        in = acts[l].output;
    }
    const float* hidden = in;
    /* streaming_cut_ce */
    float* run_max = falloc(bs);
    float* run_sumexp = falloc(bs);
    float* label_logit = falloc(bs);
    for (int i = 0; i < bs; ++i) run_max[i] = -INFINITY;
    const int cmax = chunk_size < vocab ? chunk_size : vocab;
    float* logits = falloc((int64_t)bs * cmax);
    for (int v0 = 0; v0 < vocab; v0 += cmax) {
        const int c = cmax < vocab - v0 ? cmax : vocab - v0;
        const float* wch = lm_head + (int64_t)v0 * d;
        for (int i = 0; i < bs; ++i)
            for (int k = 0; k < c; ++k) {
                float dot = 0.0f;
                for (int j = 0; j < d; ++j) dot += hidden[i * d + j] * wch[k * d + j];
                logits[i * c + k] = dot;
            }
        for (int i = 0; i < bs; ++i) {
            float cm = -INFINITY;
            for (int k = 0; k < c; ++k) cm = fmaxf(cm, logits[i * c + k]);
            const float nm = fmaxf(run_max[i], cm);
            run_sumexp[i] *= expf(run_max[i] - nm);
            for (int k = 0; k < c; ++k) run_sumexp[i] += expf(logits[i * c + k] - nm);
            run_max[i] = nm;
        }
        for (int i = 0; i < bs; ++i)
            if ((int)labels[i] >= v0 && (int)labels[i] < v0 + c) label_logit[i] = logits[i * c + (labels[i] - v0)];
    }
    float loss = 0.0f;
    for (int i = 0; i < bs; ++i) loss += -label_logit[i] + logf(run_sumexp[i]) + run_max[i];
    loss /= (float)bs;
    float* gh = falloc((int64_t)bs * d);
    for (int v0 = 0; v0 < vocab; v0 += cmax) {
        const int c = cmax < vocab - v0 ? cmax : vocab - v0;
        const float* wch = lm_head + (int64_t)v0 * d;
        for (int i = 0; i < bs; ++i)
            for (int k = 0; k < c; ++k) {
                float dot = 0.0f;
                for (int j = 0; j < d; ++j) dot += hidden[i * d + j] * wch[k * d + j];
                logits[i * c + k] = dot;
            }
        for (int i = 0; i < bs; ++i)
            for (int k = 0; k < c; ++k) {
                float factor = expf(logits[i * c + k] - run_max[i]) / run_sumexp[i];
                if (v0 + k == (int)labels[i]) factor -= 1.0f;
                for (int j = 0; j < d; ++j) gh[i * d + j] += factor * wch[k * d + j];
            }
    }
    const float inv_bs = 1.0f / (float)bs;
    for (int i = 0; i < bs * d; ++i) gh[i] *= inv_bs;
    /* backward, last layer first */
    float* up = gh;
    float* d_in = falloc((int64_t)bs * d);
    for (int l = nl - 1; l >= 0; --l) {
        layer_backward(weights + l * lf, &acts[l], up, bsz, seq, d, h, ff, grads + l * lf, d_in);
        memcpy(up, d_in, sizeof(float) * (size_t)bs * d);
    }
    for (int l = 0; l < nl; ++l) act_free(&acts[l]);
    free(acts); free(tmp_flat); free(tmp_scores); free(run_max); free(run_sumexp); free(label_logit); free(logits);
    free(gh); free(d_in);
    return loss;
}
