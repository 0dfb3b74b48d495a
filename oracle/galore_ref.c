/*
 * galore_ref.c -- CPU oracle for the per-layer optimizer step (TEST
 * INFRASTRUCTURE ONLY; see galore_ref.h for what is pinned and how).
 *
 * Build with -ffp-contract=off: the reference is Rust, which never contracts
 * a*b+c into an FMA, so every product and sum below rounds separately, in the
 * same order as the Rust source it cites.  File paths are relative to the
 * reference project's aethelStream/ directory.
 */
#include "galore_ref.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* shard_engine/src/nf4.rs:6-23 (identical values in quantizer.py:5-10). */
const float REF_NF4_CODES[16] = {
    -1.0f,        -0.6961928f, -0.52507305f, -0.3949175f, -0.28444138f, -0.18477343f,
    -0.09105004f, 0.0f,        0.0795803f,   0.1609302f,  0.2461123f,   0.33791524f,
    0.44070983f,  0.562617f,   0.72295684f,  1.0f,
};

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* IEEE binary32 -> binary16, round to nearest even.  This is what `half`
 * 2.7.1's f16::from_f32 (nf4.rs:78) and torch's .to(float16)
 * (quantizer.py:75) both do. */
uint16_t ref_f32_to_f16_rne(float f) {
    uint32_t x = f2u(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xffu;
    uint32_t mant = x & 0x7fffffu;
    if (exp == 0xffu) return (uint16_t)(sign | 0x7c00u | (mant ? (0x200u | (mant >> 13)) : 0u));
    int e = (int)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        uint32_t m = mant | 0x800000u;
        int shift = 14 - e;
        uint32_t h = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = sign | ((uint32_t)e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)h;
}

uint16_t ref_f32_to_bf16_rne(float f) {
    uint32_t x = f2u(f);
    if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
    x += 0x7fffu + ((x >> 16) & 1u);
    return (uint16_t)(x >> 16);
}

float ref_bf16_to_f32(uint16_t b) { return u2f((uint32_t)b << 16); }

/* ---------------------------------------------------------------------------
 * NF4 quantise: shard_engine/python/pipeline/quantizer.py:21-53.
 *   pad to the block size with zeros; absmax = max|x| per block (stored raw);
 *   xn = x / clamp(absmax, 1e-8); idx = argmin_c |xn - CODES[c]| (first index
 *   wins ties, as torch.argmin); packed byte k = idx[2k] << 4 | idx[2k+1].
 * ------------------------------------------------------------------------- */
static inline int nf4_argmin(float xn) {
    int best = 0;
    float bd = fabsf(xn - REF_NF4_CODES[0]);
    for (int c = 1; c < 16; ++c) {
        float d = fabsf(xn - REF_NF4_CODES[c]);
        if (d < bd) { bd = d; best = c; }
    }
    return best;
}

void ref_nf4_quantize(const float* x, int64_t n, int block, uint8_t* packed, float* absmax) {
    int64_t nblocks = (n + block - 1) / block;
    for (int64_t b = 0; b < nblocks; ++b) {
        int64_t s = b * block;
        /* blocks.abs().max(dim=1) propagates a NaN; clamp(min=1e-8) keeps it, so
         * every element of such a block gets code 0 (argmin over NaN distances) */
        float amax = 0.0f;
        int has_nan = 0;
        for (int i = 0; i < block; ++i) {
            float v = (s + i < n) ? x[s + i] : 0.0f;
            float a = fabsf(v);
            if (a != a) has_nan = 1;
            else if (a > amax) amax = a;
        }
        if (has_nan) amax = NAN;
        absmax[b] = amax;
        float safe = amax < 1e-8f ? 1e-8f : amax;
        for (int i = 0; i < block && s + i < n; ++i) {
            int64_t e = s + i;
            int idx = nf4_argmin(x[e] / safe);
            if ((e & 1) == 0) packed[e >> 1] = (uint8_t)(idx << 4);
            else packed[e >> 1] |= (uint8_t)idx;
        }
    }
}

/* NF4 dequantise to the fp32 product CODES[idx] * absmax[block]
 * (quantizer.py:73-74 before the cast; nf4.rs:76-77).  High nibble is the even
 * element (nf4.rs:66-74). */
void ref_nf4_dequant_f32(const uint8_t* packed, const float* absmax, int64_t n, int block, float* out) {
    for (int64_t e = 0; e < n; ++e) {
        uint8_t byte = packed[e >> 1];
        int nib = (e & 1) == 0 ? (byte >> 4) & 0xf : byte & 0xf;
        out[e] = REF_NF4_CODES[nib] * absmax[e / block];
    }
}

/* nf4.rs:37-83 (dequant_nf4_into) with the f16 RNE cast of nf4.rs:78. */
void ref_nf4_dequant_f16(const uint8_t* packed, const float* absmax, int64_t n, int block, uint16_t* out) {
    for (int64_t e = 0; e < n; ++e) {
        uint8_t byte = packed[e >> 1];
        int nib = (e & 1) == 0 ? (byte >> 4) & 0xf : byte & 0xf;
        out[e] = ref_f32_to_f16_rne(REF_NF4_CODES[nib] * absmax[e / block]);
    }
}

/* ---------------------------------------------------------------------------
 * Per-tensor absmax INT8: galore/src/quantize.rs:4-34.
 * ------------------------------------------------------------------------- */
float ref_absmax_scale(const float* x, int64_t n) {
    float m = 0.0f;
    for (int64_t i = 0; i < n; ++i) m = fmaxf(m, fabsf(x[i]));   /* fold(0.0, acc.max(v.abs())) */
    return m <= 0.0f ? 1.0f : m / 127.0f;
}

float ref_quantize_absmax(const float* x, int64_t n, int8_t* q) {
    float scale = ref_absmax_scale(x, n);
    float inv = scale > 0.0f ? 1.0f / scale : 0.0f;
    for (int64_t i = 0; i < n; ++i) {
        float v = roundf(x[i] * inv);              /* f32::round: half away from zero */
        if (v < -127.0f) v = -127.0f;
        if (v > 127.0f) v = 127.0f;
        q[i] = (int8_t)v;
    }
    return scale;
}

void ref_dequantize_absmax(const int8_t* q, float scale, int64_t n, float* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = (float)q[i] * scale;
}

/* ---------------------------------------------------------------------------
 * Projections: galore/src/project.rs:6-58 (same loop order, f32 sums).
 * ------------------------------------------------------------------------- */
void ref_matmul_f32(const float* a, const float* b, float* c, int m, int k, int n) {
    for (int i = 0; i < m; ++i)
        for (int j = 0; j < n; ++j) {
            float sum = 0.0f;
            for (int p = 0; p < k; ++p) sum += a[(int64_t)i * k + p] * b[(int64_t)p * n + j];
            c[(int64_t)i * n + j] = sum;
        }
}

/* project.rs:33-47: Temp = P^T G (r x n), then R = Temp Q (r x r). */
void ref_project_forward(const float* g, const float* p, const float* q, float* r_out, int m, int n, int r) {
    float* temp = (float*)calloc((size_t)r * n, sizeof(float));
    ref_project_forward_rows(g, p, q, temp, m, n, r, 0, r);
    ref_matmul_f32(temp, q, r_out, r, n, r);
    free(temp);
}

void ref_project_forward_rows(const float* g, const float* p, const float* q, float* temp, int m, int n, int r,
                              int i0, int i1) {
    (void)q;
    for (int i = i0; i < i1; ++i)
        for (int j = 0; j < n; ++j) {
            float sum = 0.0f;
            for (int k = 0; k < m; ++k) sum += p[(int64_t)k * r + i] * g[(int64_t)k * n + j];
            temp[(int64_t)i * n + j] = sum;
        }
}

/* project.rs:50-58: Temp = P N (m x r), then G~ = Temp Q^T (m x n). */
void ref_project_backward(const float* nm, const float* p, const float* q, float* g_out, int m, int n, int r) {
    float* temp = (float*)calloc((size_t)m * r, sizeof(float));
    ref_matmul_f32(p, nm, temp, m, r, r);
    ref_project_backward_rows(temp, q, g_out, m, n, r, 0, m);
    free(temp);
}

void ref_project_backward_rows(const float* temp, const float* q, float* g_out, int m, int n, int r, int i0,
                               int i1) {
    (void)m;
    float* qt = (float*)malloc((size_t)r * n * sizeof(float));
    for (int i = 0; i < n; ++i)                                   /* transpose_f32(q, qt, n, r) */
        for (int j = 0; j < r; ++j) qt[(int64_t)j * n + i] = q[(int64_t)i * r + j];
    for (int i = i0; i < i1; ++i)
        for (int j = 0; j < n; ++j) {
            float sum = 0.0f;
            for (int k = 0; k < r; ++k) sum += temp[(int64_t)i * r + k] * qt[(int64_t)k * n + j];
            g_out[(int64_t)i * n + j] = sum;
        }
    free(qt);
}

/* project.rs:61-80 */
double ref_projection_roundtrip_error(const float* g, const float* p, const float* q, int m, int n, int r) {
    float* compact = (float*)calloc((size_t)r * r, sizeof(float));
    float* recon = (float*)calloc((size_t)m * n, sizeof(float));
    ref_project_forward(g, p, q, compact, m, n, r);
    ref_project_backward(compact, p, q, recon, m, n, r);
    double diff = 0.0, orig = 0.0;
    for (int64_t i = 0; i < (int64_t)m * n; ++i) {
        double d = (double)(g[i] - recon[i]);
        diff += d * d;
        orig += (double)g[i] * (double)g[i];
    }
    free(compact);
    free(recon);
    return orig <= 1e-30 ? 0.0 : sqrt(diff / orig);
}

/* ---------------------------------------------------------------------------
 * Low-rank Adam: galore/src/adamw.rs:37-43, 116-135 (no bias correction).
 * ------------------------------------------------------------------------- */
void ref_adamw_inner_update(const float* accum, float* mom, float* var, int64_t n, float b1, float b2, float eps,
                            float* normalized) {
    for (int64_t i = 0; i < n; ++i) {
        float g = accum[i];
        mom[i] = b1 * mom[i] + (1.0f - b1) * g;
        var[i] = b2 * var[i] + (1.0f - b2) * g * g;
    }
    for (int64_t i = 0; i < n; ++i) normalized[i] = mom[i] / (sqrtf(var[i]) + eps);
}

float ref_effective_lr(float lr, int scale_by_rank, int rank) {
    if (!scale_by_rank) return lr;
    return lr / (float)(rank < 1 ? 1 : rank);
}

/* galore/src/optimizer.rs:303-362 (apply_update for one parameter). */
void ref_galore_apply_update(const float* grad_accum, const float* p, const float* q, int8_t* m8, int8_t* v8,
                             float* scale_m, float* scale_v, int m, int n, int r, float clip, float b1, float b2,
                             float eps, float lr, int scale_by_rank, float* normalized_out, float* weight_delta) {
    int64_t rr = (int64_t)r * r;
    float* mom = (float*)malloc(rr * sizeof(float));
    float* var = (float*)malloc(rr * sizeof(float));
    float* acc = (float*)malloc(rr * sizeof(float));
    float* nrm = (float*)malloc(rr * sizeof(float));
    ref_dequantize_absmax(m8, *scale_m, rr, mom);                 /* dequantize_from_ram (adamw.rs:79-82) */
    ref_dequantize_absmax(v8, *scale_v, rr, var);
    for (int64_t i = 0; i < rr; ++i) acc[i] = clip != 1.0f ? grad_accum[i] * clip : grad_accum[i];
    ref_adamw_inner_update(acc, mom, var, rr, b1, b2, eps, nrm);
    ref_project_backward(nrm, p, q, weight_delta, m, n, r);
    float lre = ref_effective_lr(lr, scale_by_rank, r);
    for (int64_t i = 0; i < (int64_t)m * n; ++i) weight_delta[i] *= lre;
    *scale_m = ref_quantize_absmax(mom, rr, m8);                  /* quantize_to_ram (adamw.rs:85-88) */
    *scale_v = ref_quantize_absmax(var, rr, v8);
    if (normalized_out) memcpy(normalized_out, nrm, rr * sizeof(float));
    free(mom); free(var); free(acc); free(nrm);
}

/* galore/src/optimizer.rs:419-448 */
void ref_init_random_projection(int rows, int cols, uint32_t seed, float* data) {
    uint64_t s = (uint64_t)seed + 1;
    for (int64_t i = 0; i < (int64_t)rows * cols; ++i) {
        s ^= s << 13;
        s ^= s >> 7;
        s ^= s << 17;
        data[i] = ((float)(s >> 40) / (float)(1u << 24)) - 0.5f;
    }
    for (int j = 0; j < cols; ++j) {
        for (int i = 0; i < j; ++i) {
            float dot = 0.0f;
            for (int row = 0; row < rows; ++row) dot += data[(int64_t)row * cols + i] * data[(int64_t)row * cols + j];
            for (int row = 0; row < rows; ++row) data[(int64_t)row * cols + j] -= dot * data[(int64_t)row * cols + i];
        }
        float norm = 0.0f;
        for (int row = 0; row < rows; ++row) norm += data[(int64_t)row * cols + j] * data[(int64_t)row * cols + j];
        norm = sqrtf(fmaxf(norm, 1e-12f));
        for (int row = 0; row < rows; ++row) data[(int64_t)row * cols + j] /= norm;
    }
}

/* galore/src/layer_rank.rs:32-40 */
int ref_rank_for_param(const char* name, int m, int n, int default_rank, int attn_rank, int mlp_rank,
                       int vector_rank) {
    int base = default_rank;
    if (!strcmp(name, "d_wq") || !strcmp(name, "d_wk") || !strcmp(name, "d_wv") || !strcmp(name, "d_wo"))
        base = attn_rank;
    else if (!strcmp(name, "d_wg") || !strcmp(name, "d_wu") || !strcmp(name, "d_wd"))
        base = mlp_rank;
    else if (!strcmp(name, "d_rms1_w") || !strcmp(name, "d_rms2_w"))
        base = vector_rank;
    int mm = m < 1 ? 1 : m, nn = n < 1 ? 1 : n;
    int v = base < mm ? base : mm;
    v = v < nn ? v : nn;
    return v < 1 ? 1 : v;
}

/* doublepass/src/hook.rs:184-187: min(1, (max_norm / (gnorm + 1e-6)) as f32). */
float ref_clip_coeff(double gsq, float max_norm) {
    double gnorm = sqrt(gsq);
    float c = (float)((double)max_norm / (gnorm + 1e-6));
    return c < 1.0f ? c : 1.0f;
}

/* galore/src/adamw.rs:99-104 */
double ref_sqnorm_f64(const float* x, int64_t n) {
    double s = 0.0;
    for (int64_t i = 0; i < n; ++i) s += (double)x[i] * (double)x[i];
    return s;
}

int ref_should_switch(uint64_t step, uint64_t interval) {
    return interval > 0 && step > 0 && (step % interval) == 0;
}

/* galore's own half conversion (galore/src/project.rs:135-185), used by the
 * state file for P and Q: add half an ulp and truncate, carry ORed into the
 * exponent, NaN payload truncated. */
uint16_t ref_galore_f32_to_f16(float x) {
    uint32_t bits = f2u(x);
    uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
    int exp = (int)((bits >> 23) & 0xffu);
    uint32_t frac = bits & 0x7fffffu;
    if (exp == 0xff) return (uint16_t)(sign | 0x7c00u | ((frac >> 13) & 0x3ffu));
    int new_exp = exp - 127 + 15;
    if (new_exp >= 0x1f) return (uint16_t)(sign | 0x7c00u);
    if (new_exp <= 0) {
        if (new_exp < -10) return sign;
        uint32_t mant = (frac | 0x800000u) >> (1 - new_exp);
        return (uint16_t)(sign | (uint16_t)((mant + 0x1000u) >> 13));
    }
    return (uint16_t)(sign | (uint16_t)(new_exp << 10) | (uint16_t)((frac + 0x1000u) >> 13));
}

float ref_galore_f16_to_f32(uint16_t h) {
    uint32_t sign = h & 0x8000u, exp = (h >> 10) & 0x1fu, frac = h & 0x3ffu, bits;
    if (exp == 0) {
        if (frac == 0) {
            bits = sign << 16;
        } else {
            uint32_t e = 0;
            while ((frac & 0x400u) == 0) { frac <<= 1; e++; }
            frac &= 0x3ffu;
            bits = (sign << 16) | ((127 - 15 - e) << 23) | (frac << 13);
        }
    } else if (exp == 0x1f) {
        bits = (sign << 16) | 0x7f800000u | (frac << 13);
    } else {
        bits = (sign << 16) | ((exp + 127 - 15) << 23) | (frac << 13);
    }
    return u2f(bits);
}

/* ---------------------------------------------------------------------------
 * Randomized SVD subspace refresh (galore/src/randomized_svd.rs:38-271).
 * ------------------------------------------------------------------------- */

/* Rng (randomized_svd.rs:38-66): xorshift64 from max(seed, 1); a uniform is
 * (x >> 40) / 2^24; a Gaussian is Box-Muller over two uniforms with the
 * first clamped to 1e-7. */
static uint64_t rsvd_next_u64(uint64_t* s) {
    uint64_t x = *s;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    *s = x;
    return x;
}
static float rsvd_next_f32(uint64_t* s) { return (float)(rsvd_next_u64(s) >> 40) / (float)(1u << 24); }
float ref_rsvd_gaussian(uint64_t* state) {
    float u1 = fmaxf(rsvd_next_f32(state), 1e-7f);
    float u2 = rsvd_next_f32(state);
    const float two_pi = 2.0f * 3.14159265358979323846f;
    return sqrtf(-2.0f * logf(u1)) * cosf(two_pi * u2);
}

void ref_rsvd_omega(uint64_t seed, int64_t count, float* out) {
    uint64_t s = seed > 1 ? seed : 1;
    for (int64_t i = 0; i < count; ++i) out[i] = ref_rsvd_gaussian(&s);
}

/* qr_columns (randomized_svd.rs:160-185): modified Gram-Schmidt on the
 * columns of a row-major m x k matrix; -1 on a column norm below 1e-12. */
static int rsvd_mgs(float* q, int m, int k, int fail_on_small) {
    for (int j = 0; j < k; ++j) {
        for (int i = 0; i < j; ++i) {
            float dot = 0.0f;
            for (int row = 0; row < m; ++row) dot += q[(int64_t)row * k + i] * q[(int64_t)row * k + j];
            for (int row = 0; row < m; ++row) q[(int64_t)row * k + j] -= dot * q[(int64_t)row * k + i];
        }
        float norm = 0.0f;
        for (int row = 0; row < m; ++row) norm += q[(int64_t)row * k + j] * q[(int64_t)row * k + j];
        if (fail_on_small) {
            norm = sqrtf(norm);
            if (norm < 1e-12f) return -1;
        } else {
            /* orthonormalize_columns (randomized_svd.rs:187-207) */
            norm = sqrtf(fmaxf(norm, 1e-12f));
        }
        for (int row = 0; row < m; ++row) q[(int64_t)row * k + j] /= norm;
    }
    return 0;
}

/* jacobi_eigenvectors (randomized_svd.rs:210-271): at most 50 single
 * rotations, each on the largest off-diagonal |a_pq| (first in row-major
 * order), stopping below 1e-10.  The rotation loop runs in place over k, so
 * for k = p and k = q it reads values written earlier in the same loop. */
void ref_rsvd_jacobi(float* mat, int n, float* u) {
    for (int i = 0; i < n * n; ++i) u[i] = 0.0f;
    for (int i = 0; i < n; ++i) u[i * n + i] = 1.0f;
    for (int it = 0; it < 50; ++it) {
        float max_off = 0.0f;
        int p = 0, q = 1;
        for (int i = 0; i < n; ++i)
            for (int j = i + 1; j < n; ++j) {
                float v = fabsf(mat[i * n + j]);
                if (v > max_off) { max_off = v; p = i; q = j; }
            }
        if (max_off < 1e-10f) break;
        float app = mat[p * n + p], aqq = mat[q * n + q], apq = mat[p * n + q];
        float tau = (aqq - app) / (2.0f * apq);
        float t = tau >= 0.0f ? 1.0f / (tau + sqrtf(1.0f + tau * tau)) : -1.0f / (-tau + sqrtf(1.0f + tau * tau));
        float c = 1.0f / sqrtf(1.0f + t * t);
        float s = t * c;
        for (int k = 0; k < n; ++k) {
            float mkp = mat[k * n + p], mkq = mat[k * n + q];
            mat[k * n + p] = c * mkp - s * mkq;
            mat[p * n + k] = mat[k * n + p];
            mat[k * n + q] = s * mkp + c * mkq;
            mat[q * n + k] = mat[k * n + q];
        }
        mat[p * n + q] = 0.0f;
        mat[q * n + p] = 0.0f;
        for (int k = 0; k < n; ++k) {
            float ukp = u[k * n + p], ukq = u[k * n + q];
            u[k * n + p] = c * ukp - s * ukq;
            u[k * n + q] = s * ukp + c * ukq;
        }
    }
}

/* randomized_svd_projections (randomized_svd.rs:76-149).  Returns 0, -2 for
 * an invalid rank / oversampling (GaLoreError::Config) or -3 for a rank
 * deficient sketch (GaLoreError::Linalg).  p_out: m x r, q_out: n x r. */
int ref_randomized_svd(const float* g, int m, int n, int r, int oversampling, uint64_t seed, float* p_out,
                       float* q_out) {
    const int l = r + oversampling;
    if (r == 0 || l > (n < m ? n : m)) return -2;
    float* omega = (float*)malloc(sizeof(float) * (size_t)n * l);
    ref_rsvd_omega(seed, (int64_t)n * l, omega);
    const int st = ref_randomized_svd_sketch(g, m, n, r, oversampling, omega, p_out, q_out);
    free(omega);
    return st;
}

/* Steps 2-5 of randomized_svd_projections (randomized_svd.rs:95-149) from a
 * given n x l sketch omega (step 1's draw). */
int ref_randomized_svd_sketch(const float* g, int m, int n, int r, int oversampling, const float* omega,
                              float* p_out, float* q_out) {
    const int l = r + oversampling;
    if (r == 0 || l > (n < m ? n : m)) return -2;
    float* y = (float*)malloc(sizeof(float) * (size_t)m * l);
    float* qt = (float*)malloc(sizeof(float) * (size_t)l * m);
    float* b = (float*)malloc(sizeof(float) * (size_t)l * n);
    float* bt = (float*)malloc(sizeof(float) * (size_t)n * l);
    float* bbt = (float*)malloc(sizeof(float) * (size_t)l * l);
    float* u = (float*)malloc(sizeof(float) * (size_t)l * l);
    int st = 0;
    ref_matmul_f32(g, omega, y, m, n, l);
    if (rsvd_mgs(y, m, l, 1) != 0) { st = -3; goto done; }
    for (int i = 0; i < m; ++i)
        for (int j = 0; j < l; ++j) qt[(int64_t)j * m + i] = y[(int64_t)i * l + j];
    ref_matmul_f32(qt, g, b, l, m, n);
    for (int i = 0; i < l; ++i)
        for (int j = 0; j < n; ++j) bt[(int64_t)j * l + i] = b[(int64_t)i * n + j];
    ref_matmul_f32(b, bt, bbt, l, n, l);
    ref_rsvd_jacobi(bbt, l, u);
    for (int i = 0; i < m; ++i)
        for (int j = 0; j < r; ++j) {
            float sum = 0.0f;
            for (int k = 0; k < l; ++k) sum += y[(int64_t)i * l + k] * u[k * l + j];
            p_out[(int64_t)i * r + j] = sum;
        }
    for (int i = 0; i < n; ++i)
        for (int j = 0; j < r; ++j) {
            float sum = 0.0f;
            for (int k = 0; k < l; ++k) sum += b[(int64_t)k * n + i] * u[k * l + j];
            q_out[(int64_t)i * r + j] = sum;
        }
    rsvd_mgs(q_out, n, r, 0);
done:
    free(y); free(qt); free(b); free(bt); free(bbt); free(u);
    return st;
}

/* galore/src/standard_adamw.rs:84-114; with step >= 1 the moments are bias
 * corrected by the host-computed factors 1 - beta^step. */
void ref_full_adam_apply(float* param, const float* grad, float* m, float* v, int64_t n, float clip, float b1,
                         float b2, float eps, float lr, int step) {
    float bc1 = 1.0f, bc2 = 1.0f;
    if (step >= 1) {
        bc1 = (float)(1.0 - pow((double)b1, (double)step));
        bc2 = (float)(1.0 - pow((double)b2, (double)step));
    }
    for (int64_t i = 0; i < n; ++i) {
        float gs = grad[i] * clip;
        m[i] = b1 * m[i] + (1.0f - b1) * gs;
        v[i] = b2 * v[i] + (1.0f - b2) * gs * gs;
        float mh = m[i], vh = v[i];
        if (step >= 1) { mh = mh / bc1; vh = vh / bc2; }
        float d = lr * mh / (sqrtf(vh) + eps);
        param[i] -= d;
    }
}

/* ---------------------------------------------------------------------------
 * B200-mode extensions.
 * ------------------------------------------------------------------------- */

/* 256-entry 8-bit "dynamic" map in the style of Dettmers et al. 2021
 * (8-bit Optimizers via Block-wise Quantization, dynamic tree quantisation):
 * after the optional sign bit, E leading zero bits select the decade 10^-E,
 * the first one bit is an indicator, and the remaining F bits are a linear
 * fraction whose 2^F levels are the centres of equal bins over [0.1, 1].
 * Signed: E = 0..6, F = 6 - E (127 magnitudes per sign) plus 0 and +1.0.
 * Unsigned: E = 0..6, F = 7 - E (254 magnitudes) plus 0 and 1.0.
 * The table is sorted ascending; a stored code is an index into it. */
static int cmp_float(const void* a, const void* b) {
    float x = *(const float*)a, y = *(const float*)b;
    return (x > y) - (x < y);
}

void b2_dynamic_map(int is_signed, float out[256]) {
    static const double decade[7] = {1.0, 1e-1, 1e-2, 1e-3, 1e-4, 1e-5, 1e-6};
    int k = 0;
    for (int e = 0; e < 7; ++e) {
        int fbits = (is_signed ? 6 : 7) - e;
        int levels = 1 << fbits;
        for (int j = 0; j < levels; ++j) {
            double f = 0.1 + 0.9 * ((double)j + 0.5) / (double)levels;
            out[k++] = (float)(decade[e] * f);
            if (is_signed) out[k++] = (float)(-decade[e] * f);
        }
    }
    out[k++] = 0.0f;
    out[k++] = 1.0f;
    qsort(out, 256, sizeof(float), cmp_float);
}

static int dmap_nearest(const float* map, float xn) {
    int lo = 0, hi = 256;
    while (lo < hi) {
        int mid = (lo + hi) >> 1;
        if (map[mid] < xn) lo = mid + 1; else hi = mid;
    }
    if (lo == 0) return 0;
    if (lo == 256) return 255;
    float dl = fabsf(xn - map[lo - 1]);
    float dh = fabsf(xn - map[lo]);
    return dh < dl ? lo : lo - 1;
}

/* Blockwise INT8 codec over contiguous blocks of `block` elements (the last
 * block may be partial).  LINEAR: per-block copy of quantize.rs:4-26, so with
 * block >= n it is bit-identical to ref_quantize_absmax.  DYNAMIC: the block's
 * raw absmax is the scale; codes index b2_dynamic_map; nearest entry of
 * x * (1 / absmax) (one fp32 reciprocal per block), lower index on ties. */
void b2_block_quantize(const float* x, int64_t n, int block, int codec, int is_signed, int8_t* q, float* scales) {
    float map[256];
    if (codec == B2_CODEC_DYNAMIC) b2_dynamic_map(is_signed, map);
    int64_t nb = (n + block - 1) / block;
    for (int64_t b = 0; b < nb; ++b) {
        int64_t s = b * block, e = s + block < n ? s + block : n;
        if (codec == B2_CODEC_LINEAR) {
            scales[b] = ref_quantize_absmax(x + s, e - s, q + s);
        } else {
            float amax = 0.0f;
            for (int64_t i = s; i < e; ++i) amax = fmaxf(amax, fabsf(x[i]));
            scales[b] = amax;
            const float inv = amax > 0.0f ? 1.0f / amax : 0.0f;  /* one reciprocal per block */
            for (int64_t i = s; i < e; ++i) {
                float xn = x[i] * inv;
                q[i] = (int8_t)(uint8_t)dmap_nearest(map, xn);
            }
        }
    }
}

void b2_block_dequantize(const int8_t* q, const float* scales, int64_t n, int block, int codec, int is_signed,
                         float* out) {
    float map[256];
    if (codec == B2_CODEC_DYNAMIC) b2_dynamic_map(is_signed, map);
    for (int64_t i = 0; i < n; ++i) {
        float s = scales[i / block];
        out[i] = codec == B2_CODEC_LINEAR ? (float)q[i] * s : map[(uint8_t)q[i]] * s;
    }
}

/* One-sided GaLore (Zhao et al. 2024): project on the smaller dimension.
 * m >= n: right projector Q (n x r), R = G Q (m x r).
 * m <  n: left projector P (m x r), R^T = G^T P (n x r).
 * Either way the state is l x r row-major with l = max(m, n). */
int b2_side_is_right(int m, int n) { return m >= n; }

void b2_project_accumulate(const float* g, const float* proj, float* racc, int m, int n, int r) {
    double* acc = (double*)calloc((size_t)r, sizeof(double));
    if (b2_side_is_right(m, n)) {
        for (int i = 0; i < m; ++i) {
            memset(acc, 0, r * sizeof(double));
            for (int j = 0; j < n; ++j) {
                double gv = g[(int64_t)i * n + j];
                const float* qrow = proj + (int64_t)j * r;
                for (int c = 0; c < r; ++c) acc[c] += gv * (double)qrow[c];
            }
            for (int c = 0; c < r; ++c) racc[(int64_t)i * r + c] = racc[(int64_t)i * r + c] + (float)acc[c];
        }
    } else {
        double* full = (double*)calloc((size_t)n * r, sizeof(double));
        for (int i = 0; i < m; ++i) {
            const float* prow = proj + (int64_t)i * r;
            for (int j = 0; j < n; ++j) {
                double gv = g[(int64_t)i * n + j];
                double* dst = full + (int64_t)j * r;
                for (int c = 0; c < r; ++c) dst[c] += gv * (double)prow[c];
            }
        }
        for (int64_t e = 0; e < (int64_t)n * r; ++e) racc[e] = racc[e] + (float)full[e];
        free(full);
    }
    free(acc);
}

/* Adam over the l x r state with blockwise INT8 m/v.  Same arithmetic as
 * adamw.rs:116-135 per element; g = R * clip (optimizer.rs:318-322).  With the
 * LINEAR codec and block >= count this is ref_galore_apply_update's state
 * update exactly. */
void b2_adam_state(const float* racc, int8_t* m8, int8_t* v8, float* mscale, float* vscale, int64_t count, int block,
                   int codec, float clip, float b1, float b2, float eps, float* n_bf16_out) {
    float* mom = (float*)malloc(count * sizeof(float));
    float* var = (float*)malloc(count * sizeof(float));
    b2_block_dequantize(m8, mscale, count, block, codec, 1, mom);
    b2_block_dequantize(v8, vscale, count, block, codec, 0, var);
    for (int64_t i = 0; i < count; ++i) {
        float g = racc[i] * clip;
        mom[i] = b1 * mom[i] + (1.0f - b1) * g;
        var[i] = b2 * var[i] + (1.0f - b2) * g * g;
        float nv = mom[i] / (sqrtf(var[i]) + eps);
        if (n_bf16_out) n_bf16_out[i] = ref_bf16_to_f32(ref_f32_to_bf16_rne(nv));
    }
    b2_block_quantize(mom, count, block, codec, 1, m8, mscale);
    b2_block_quantize(var, count, block, codec, 0, v8, vscale);
    free(mom);
    free(var);
}

void b2_nf4_requant(const float* w, int64_t n, uint8_t* packed, float* absmax) {
    ref_nf4_quantize(w, n, 64, packed, absmax);
}

/* dW = P N^T (left) or N Q^T (right), accumulated in double; w' = w - lr*dW
 * (two roundings, as weight_delta *= lr then w -= d in optimizer.rs:337-340
 * and tests/common/mod.rs:106-111), optional decoupled decay of
 * adamw.rs:194-202, then NF4 requantisation (quantizer.py:21-53). */
void b2_apply_weight(const float* n_bf16, const float* proj, int m, int n, int r, const uint8_t* w_packed,
                     const float* w_absmax, float lr, float wd, uint8_t* w_packed_out, float* w_absmax_out,
                     float* w_prequant_out, float* dw_out) {
    int64_t mn = (int64_t)m * n;
    float* w = (float*)malloc(mn * sizeof(float));
    ref_nf4_dequant_f32(w_packed, w_absmax, mn, 64, w);
    int right = b2_side_is_right(m, n);
    for (int i = 0; i < m; ++i)
        for (int j = 0; j < n; ++j) {
            const float* a = right ? n_bf16 + (int64_t)i * r : proj + (int64_t)i * r;
            const float* b = right ? proj + (int64_t)j * r : n_bf16 + (int64_t)j * r;
            double s = 0.0;
            for (int c = 0; c < r; ++c) s += (double)a[c] * (double)b[c];
            float d = (float)s;
            if (dw_out) dw_out[(int64_t)i * n + j] = d;
            float t = lr * d;
            float wv = w[(int64_t)i * n + j] - t;
            if (wd > 0.0f) wv = wv * (1.0f - lr * wd);
            w[(int64_t)i * n + j] = wv;
        }
    if (w_prequant_out) memcpy(w_prequant_out, w, mn * sizeof(float));
    ref_nf4_quantize(w, mn, 64, w_packed_out, w_absmax_out);
    free(w);
}

/* LOMO (Lv et al. 2023) fused full-rank step over a flat NF4 tensor.  Pass 1:
 * squared norm of the bf16 gradient (f64).  Pass 2: g' = g * clip; momentum
 * m = beta * m + g' (SGD momentum without dampening) kept in blockwise INT8;
 * w' = w - lr * m; NF4 requantisation.  There is no LOMO code in the
 * reference; the full-rank SGD step w -= lr * g of
 * doublepass/tests/test_resume.rs:138-152 is the beta = 0 case. */
double b2_lomo_sqnorm_bf16(const uint16_t* g, int64_t n) {
    double s = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        double v = ref_bf16_to_f32(g[i]);
        s += v * v;
    }
    return s;
}

void b2_lomo_update(const uint16_t* g, int64_t n, float clip, float beta, float lr, int block, int codec,
                    int8_t* mom8, float* mom_scales, const uint8_t* w_packed, const float* w_absmax,
                    uint8_t* w_packed_out, float* w_absmax_out, float* w_prequant_out) {
    float* mom = (float*)malloc(n * sizeof(float));
    float* w = (float*)malloc(n * sizeof(float));
    b2_block_dequantize(mom8, mom_scales, n, block, codec, 1, mom);
    ref_nf4_dequant_f32(w_packed, w_absmax, n, 64, w);
    for (int64_t i = 0; i < n; ++i) {
        float gs = ref_bf16_to_f32(g[i]) * clip;
        mom[i] = beta * mom[i] + gs;
        float t = lr * mom[i];
        w[i] = w[i] - t;
    }
    if (w_prequant_out) memcpy(w_prequant_out, w, n * sizeof(float));
    b2_block_quantize(mom, n, block, codec, 1, mom8, mom_scales);
    ref_nf4_quantize(w, n, 64, w_packed_out, w_absmax_out);
    free(mom);
    free(w);
}

/* ---------------------------------------------------------------------------
 * Streamed-weight decode (flowcast/src/decode.rs) and the BF16
 * stochastic-rounding write-back (doublepass/src/precision.rs), restated.
 * ------------------------------------------------------------------------- */
uint16_t fc_f32_to_f16(float v) {
    /* decode.rs:191-210 */
    uint32_t bits = f2u(v);
    uint16_t sign = (uint16_t)(bits >> 31);
    int32_t exp = (int32_t)((bits >> 23) & 0xFF);
    uint32_t mant = bits & 0x7FFFFF;
    if (exp == 0xFF) return (uint16_t)((sign << 15) | 0x7C00 | (mant != 0 ? 0x0200 : 0));
    int32_t exp16 = exp - 127 + 15;
    if (exp16 <= 0) return (uint16_t)(sign << 15);
    if (exp16 >= 31) return (uint16_t)((sign << 15) | 0x7C00);
    return (uint16_t)((sign << 15) | ((uint16_t)exp16 << 10) | (uint16_t)(mant >> 13));
}

void fc_decode_int8_to_f16(const int8_t* src, int64_t n, const float* scales, int64_t n_scales, int num_channels,
                           uint16_t* out) {
    /* decode.rs:63-86: channel = i / max(n / num_channels, 1) (0 when num_channels == 0);
     * scale_per_channel.get(channel) or 1.0 */
    int64_t per = num_channels > 0 ? n / num_channels : n;
    if (per < 1) per = 1;
    for (int64_t i = 0; i < n; ++i) {
        int64_t ch = num_channels > 0 ? i / per : 0;
        float s = ch < n_scales ? scales[ch] : 1.0f;
        out[i] = fc_f32_to_f16((float)src[i] * s);
    }
}

void fc_decode_int4_to_f16(const uint8_t* src, int64_t nbytes, float absmax, uint16_t* out) {
    /* decode.rs:88-104: low nibble first */
    for (int64_t k = 0; k < nbytes; ++k) {
        out[2 * k] = fc_f32_to_f16(REF_NF4_CODES[src[k] & 0x0F] * absmax);
        out[2 * k + 1] = fc_f32_to_f16(REF_NF4_CODES[(src[k] >> 4) & 0x0F] * absmax);
    }
}

uint16_t dp_lcg_next(uint64_t* state) {
    *state = *state * 6364136223846793005ull + 1442695040888963407ull;
    return (uint16_t)((*state >> 33) & 0xFFFF);
}

uint16_t dp_stochastic_round_to_bf16(float v, uint16_t rand_bits) {
    uint32_t bits = f2u(v);
    uint16_t low16 = (uint16_t)(bits & 0xFFFF), high16 = (uint16_t)(bits >> 16);
    if (low16 > rand_bits) return high16 == 0xFFFF ? high16 : (uint16_t)(high16 + 1); /* saturating_add */
    return high16;
}

void dp_apply_galore_bf16_update(float* master, const float* delta, int64_t n, uint64_t* rng) {
    for (int64_t i = 0; i < n; ++i) {
        master[i] += delta[i];
        uint16_t r = dp_lcg_next(rng);
        master[i] = u2f((uint32_t)dp_stochastic_round_to_bf16(master[i], r) << 16);
    }
}
