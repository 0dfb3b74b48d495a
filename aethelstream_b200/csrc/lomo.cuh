// lomo.cuh -- LOMO fused full-rank update (K7) over a flat NF4 tensor.
//
// Pass 1 (lomo_sqnorm_kernel): sum of squares of the bf16 gradient in f64.
// Pass 2 (lomo_update_kernel): clip from the (reduced) sum, INT8 blockwise
// momentum m = beta * m + g * clip, w = w - lr * m, NF4 requantisation -- one
// HBM pass: bf16 g (2 B), NF4 w read + write (2 x 0.5625 B), INT8 m read +
// write (2 B) per element.
#pragma once
#include "codec.cuh"
#include "nf4.cuh"

namespace aeth {

__global__ void __launch_bounds__(256) lomo_sqnorm_kernel(const uint16_t* __restrict__ g, int64_t n,
                                                          double* __restrict__ sq_out) {
    __shared__ double red[8];
    double s = 0.0;
    const int64_t n8 = n / 8;
    for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < n8; c += (int64_t)gridDim.x * blockDim.x) {
        uint4 u = __ldg(reinterpret_cast<const uint4*>(g) + c);
        uint32_t w[4] = {u.x, u.y, u.z, u.w};
        double dpart = 0.0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            double lo = (double)bf16_bits_to_f32((uint16_t)(w[k] & 0xffffu));
            double hi = (double)bf16_bits_to_f32((uint16_t)(w[k] >> 16));
            dpart += lo * lo + hi * hi;
        }
        s += dpart;
    }
    for (int64_t i = n8 * 8 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        double v = (double)bf16_bits_to_f32(g[i]);
        s += v * v;
    }
    s = warp_sum_d(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
        atomicAdd(sq_out, t);
    }
}

// One CTA of 256 threads per momentum block of 2048 elements; thread t owns 8
// consecutive elements, so 8 consecutive threads form one NF4 block of 64.
__global__ void __launch_bounds__(256) lomo_update_kernel(const uint16_t* __restrict__ g, int64_t n,
                                                          const double* __restrict__ sq, float max_norm, float lr,
                                                          float beta, int codec, int8_t* __restrict__ mom8,
                                                          float* __restrict__ mom_scales, uint8_t* __restrict__ wp,
                                                          float* __restrict__ wa, float* __restrict__ prequant) {
    __shared__ Nf4Tables tab;
    __shared__ float dm[256];
    __shared__ uint2 dlut[kDmapLutEntries];
    __shared__ float red[8];
    nf4_tables_init(&tab, threadIdx.x, blockDim.x);
    if (codec == AETH_CODEC_BLOCK_DYNAMIC) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) dm[i] = c_dmap_signed[i];
        for (int i = threadIdx.x; i < kDmapLutEntries; i += blockDim.x) dlut[i] = g_dmap_lut[0][i];
    }
    __syncthreads();
    double gnorm = sqrt(*sq);
    float clip = (float)((double)max_norm / (gnorm + 1e-6));
    clip = clip < 1.0f ? clip : 1.0f;
    const int64_t n_blocks = n / 2048;
    for (int64_t b = blockIdx.x; b < n_blocks; b += gridDim.x) {
        const int64_t e0 = b * 2048 + threadIdx.x * 8;
        const float ms = mom_scales[b];
        uint4 gu = __ldg(reinterpret_cast<const uint4*>(g + e0));
        uint2 mq = *reinterpret_cast<const uint2*>(mom8 + e0);
        uint32_t wq = *reinterpret_cast<const uint32_t*>(wp + e0 / 2);
        float wamax = wa[e0 / 64];
        float w[8], mo[8];
        nf4_dequant_word(wq, wamax, tab.byte_lut, w);
        uint32_t gw[4] = {gu.x, gu.y, gu.z, gu.w};
        uint32_t mw[2] = {mq.x, mq.y};
        float am = 0.0f, aw = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            uint16_t gb = (uint16_t)((gw[k >> 1] >> (16 * (k & 1))) & 0xffffu);
            float gs = __fmul_rn(bf16_bits_to_f32(gb), clip);
            int8_t q = (int8_t)((mw[k >> 2] >> (8 * (k & 3))) & 0xffu);
            float m0 = codec == AETH_CODEC_BLOCK_LINEAR ? __fmul_rn((float)q, ms) : __fmul_rn(dm[(uint8_t)q], ms);
            mo[k] = __fadd_rn(__fmul_rn(beta, m0), gs);
            w[k] = __fsub_rn(w[k], __fmul_rn(lr, mo[k]));
            am = fmaxf(am, fabsf(mo[k]));
            aw = fmax_nan(aw, fabsf(w[k]));
        }
        // NF4 block absmax across the 8 lanes owning this 64-element block.
        aw = fmax_nan(aw, __shfl_xor_sync(0xffffffffu, aw, 1));
        aw = fmax_nan(aw, __shfl_xor_sync(0xffffffffu, aw, 2));
        aw = fmax_nan(aw, __shfl_xor_sync(0xffffffffu, aw, 4));
        uint32_t pk[1];
        nf4_quant_regs<8>(w, aw, tab.bucket, pk);
        *reinterpret_cast<uint32_t*>(wp + e0 / 2) = pk[0];
        if ((threadIdx.x & 7) == 0) wa[e0 / 64] = nf4_store_amax(aw);
        if (prequant) {
            *reinterpret_cast<float4*>(prequant + e0) = make_float4(w[0], w[1], w[2], w[3]);
            *reinterpret_cast<float4*>(prequant + e0 + 4) = make_float4(w[4], w[5], w[6], w[7]);
        }
        // Momentum block absmax across the CTA.
        am = warp_max(am);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = am;
        __syncthreads();
        float bm = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) bm = fmaxf(bm, red[i]);
        uint32_t out[2] = {0u, 0u};
        if (codec == AETH_CODEC_BLOCK_LINEAR) {
            float nsm = lin_scale_from_absmax(bm), inv = lin_inv(nsm);
#pragma unroll
            for (int k = 0; k < 8; ++k) out[k >> 2] |= ((uint32_t)(uint8_t)lin_encode(mo[k], inv)) << (8 * (k & 3));
            if (threadIdx.x == 0) mom_scales[b] = nsm;
        } else {
            const float inv = dyn_inv(bm);
#pragma unroll
            for (int k = 0; k < 8; ++k)
                out[k >> 2] |= dmap_encode_lut<true>(dlut, dm, dyn_xn(mo[k], inv)) << (8 * (k & 3));
            if (threadIdx.x == 0) mom_scales[b] = bm;
        }
        *reinterpret_cast<uint2*>(mom8 + e0) = make_uint2(out[0], out[1]);
        __syncthreads();
    }
}

}  // namespace aeth
