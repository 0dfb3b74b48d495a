// small_rank.cuh -- B200-mode projection and weight write for the shapes the
// TMA-fed tensor-core kernels cannot describe: a rank that is not a multiple
// of 8 or a side that is not a multiple of 8 elements (a TMA row pitch must be
// a multiple of 16 bytes).  The case that matters is a layer's RMS-norm
// weights d_rms1_w / d_rms2_w: 1 x d vectors whose rank LayerRankConfig clamps
// to 1 (galore/src/layer_rank.rs:32-40; galore/tests/common/mod.rs:73-89),
// stepped with the layer's matrices (doublepass/src/backward.rs:512-520).
// These tensors are tiny (d elements), so plain CUDA-core kernels with f64
// accumulation of exact products serve them; the definitions are the same as
// the tensor-core path's (one-sided projection on the smaller dimension,
// bf16 projector, bf16 Adam direction N).
#pragma once
#include "common.cuh"
#include "nf4.cuh"

namespace aeth {

// R += projection(G), R l x r row-major.  right (m >= n): R[i][c] += sum_j
// G[i][j] Q[j][c] (proj = Q, n x r); left: R[j][c] += sum_i G[i][j] P[i][c]
// (proj = P, m x r).  One thread per element of R; the gradient (any dtype,
// widened exactly) times the bf16 projector is exact in f64.
__global__ void small_project_kernel(const void* __restrict__ g, int dtype, int m, int n, int r, int right,
                                     const uint16_t* __restrict__ proj, float* __restrict__ racc) {
    const int64_t l = right ? m : n;
    const int K = right ? n : m;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < l * r; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = t / r;
        const int c = (int)(t % r);
        double s = 0.0;
        for (int k = 0; k < K; ++k) {
            const int64_t gi = right ? row * n + k : (int64_t)k * n + row;
            s += (double)load_as_f32(g, gi, dtype) * (double)bf16_bits_to_f32(proj[(int64_t)k * r + c]);
        }
        racc[t] = __fadd_rn(racc[t], (float)s);
    }
}

// The weight write for those shapes.  dW[i][j] = sum_c X[i][c] Y[j][c] (X =
// N, Y = Q on the right side; X = P, Y = N on the left; both bf16, r columns),
// w' = w - fl(lr dW), then w' *= (1 - lr wd) with decay; kind NF4 requantises
// each 64-element block exactly as the reference's quantiser
// (quantizer.py:21-53: NaN-propagating block absmax, IEEE x / max(absmax,
// 1e-8), first index on ties), one warp per block (lane: elements 2 lane,
// 2 lane + 1, one packed byte).  kind F32 updates the dense weight in place;
// kind NONE only writes delta_out = fl(lr dW).
__global__ void small_apply_kernel(const uint16_t* __restrict__ X, const uint16_t* __restrict__ Y, int m, int n,
                                   int r, float lr, float decay_mul, int has_decay, int kind, void* __restrict__ wdata,
                                   float* __restrict__ wabsmax, float* __restrict__ prequant,
                                   float* __restrict__ delta_out) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int64_t nblocks = (int64_t)m * n / 64;  // m n % 64 == 0; blocks run over the flattened weight
    for (int64_t b = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); b < nblocks; b += warps) {
        const int64_t e0 = b * 64 + 2 * lane;
        float w[2];
        uint8_t* wp = static_cast<uint8_t*>(wdata);
        if (kind == AETH_WEIGHT_NF4) {
            const uint32_t byte = wp[e0 / 2];
            const float am = wabsmax[b];
            w[0] = __fmul_rn(c_nf4_codes[byte >> 4], am);
            w[1] = __fmul_rn(c_nf4_codes[byte & 15], am);
        } else if (kind == AETH_WEIGHT_F32) {
            w[0] = static_cast<float*>(wdata)[e0];
            w[1] = static_cast<float*>(wdata)[e0 + 1];
        } else {
            w[0] = w[1] = 0.0f;
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int64_t i = (e0 + h) / n, j = (e0 + h) % n;
            double s = 0.0;
            for (int c = 0; c < r; ++c)
                s += (double)bf16_bits_to_f32(X[i * r + c]) * (double)bf16_bits_to_f32(Y[j * r + c]);
            const float t = __fmul_rn(lr, (float)s);
            if (delta_out) delta_out[e0 + h] = t;
            float wv = __fsub_rn(w[h], t);
            if (has_decay) wv = __fmul_rn(wv, decay_mul);
            w[h] = wv;
            if (prequant) prequant[e0 + h] = wv;
        }
        if (kind == AETH_WEIGHT_F32) {
            static_cast<float*>(wdata)[e0] = w[0];
            static_cast<float*>(wdata)[e0 + 1] = w[1];
        } else if (kind == AETH_WEIGHT_NF4) {
            float a = fmax_nan(fabsf(w[0]), fabsf(w[1]));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) a = fmax_nan(a, __shfl_xor_sync(0xffffffffu, a, o));
            const float safe = nf4_safe(a);
            const uint32_t c0 = nf4_code_exact(w[0], safe), c1 = nf4_code_exact(w[1], safe);
            wp[e0 / 2] = (uint8_t)((c0 << 4) | c1);
            if (lane == 0) wabsmax[b] = nf4_store_amax(a);
        }
    }
}

}  // namespace aeth
