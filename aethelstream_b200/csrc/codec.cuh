// codec.cuh -- INT8 optimizer-state codecs (K3).
//
// PER_TENSOR  galore/src/quantize.rs:4-34: scale = max|x|/127 (1.0 when the
//             max is 0), q = clamp(round(x * (1/scale)), +-127), round half away
//             from zero; dequant x = q * scale.
// BLOCK_LINEAR  the same formula per contiguous block of `block` elements.
// BLOCK_DYNAMIC per-block raw absmax; code = index of the nearest entry of a
//             sorted 256-entry dynamic map to x * (1 / absmax) (one reciprocal
//             per block; lower index on ties).
#pragma once
#include "common.cuh"

namespace aeth {

// Sorted dynamic maps (signed for first moments, unsigned for second
// moments), uploaded once per device by codec_maps_ensure().
__constant__ float c_dmap_signed[256];
__constant__ float c_dmap_unsigned[256];

// Same construction as the oracle's b2_dynamic_map (see aeth_dynamic_map).
int build_dynamic_map(int is_signed, float out[256]);

inline bool g_maps_uploaded[kMaxDevices] = {};

inline int codec_maps_ensure() {
    int dev = 0;
    AETH_TRY(current_device(&dev));
    if (dev < 0 || dev >= kMaxDevices) return set_err(AETH_ERR_UNSUPPORTED);
    if (!g_maps_uploaded[dev]) {
        float s[256], u[256];
        build_dynamic_map(1, s);
        build_dynamic_map(0, u);
        AETH_CUDA(cudaMemcpyToSymbol(c_dmap_signed, s, sizeof(s)));
        AETH_CUDA(cudaMemcpyToSymbol(c_dmap_unsigned, u, sizeof(u)));
        g_maps_uploaded[dev] = true;
    }
    return AETH_OK;
}

// Linear INT8 encode with the reference's rounding (half away from zero).
__device__ __forceinline__ int8_t lin_encode(float x, float inv) {
    float q = roundf(__fmul_rn(x, inv));
    q = fminf(fmaxf(q, -127.0f), 127.0f);
    return (int8_t)(int)q;
}

__device__ __forceinline__ float lin_scale_from_absmax(float amax) {
    return amax <= 0.0f ? 1.0f : __fdiv_rn(amax, 127.0f);
}

__device__ __forceinline__ float lin_inv(float scale) { return scale > 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f; }

// Nearest entry of a sorted 256-entry map held in shared memory.
__device__ __forceinline__ uint32_t dmap_encode(const float* __restrict__ map, float xn) {
    int lo = 0;
#pragma unroll
    for (int step = 128; step > 0; step >>= 1)
        if (map[lo + step - 1] < xn) lo += step;
    // lo = number of entries < xn (lower_bound), in [0, 256]
    if (lo == 0) return 0u;
    if (lo == 256) return 255u;
    float dl = fabsf(__fsub_rn(xn, map[lo - 1]));
    float dh = fabsf(__fsub_rn(xn, map[lo]));
    return dh < dl ? (uint32_t)lo : (uint32_t)(lo - 1);
}

// Dynamic codec normalisation: xn = x * (1 / absmax), one reciprocal per block.
__device__ __forceinline__ float dyn_inv(float amax) { return amax > 0.0f ? __frcp_rn(amax) : 0.0f; }
__device__ __forceinline__ float dyn_xn(float x, float inv) { return __fmul_rn(x, inv); }

// ---------------------------------------------------------------------------
// Per-tensor codec: absmax reduction into a device float (atomicMax on the
// non-negative bit pattern), then encode.  galore_quantize_absmax_f32_to_i8
// keeps the absmax in *scale_out, encodes, then finalises *scale_out.
// ---------------------------------------------------------------------------
__global__ void absmax_reduce_kernel(const float* __restrict__ x, int64_t n, float* __restrict__ amax_out) {
    float a = 0.0f;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        a = fmaxf(a, fabsf(x[i]));
    a = warp_max(a);
    __shared__ float red[32];
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = a;
    __syncthreads();
    if (threadIdx.x < 32) {
        float b = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
        b = warp_max(b);
        if (threadIdx.x == 0) atomic_max_nonneg(amax_out, b);
    }
}

__global__ void per_tensor_encode_kernel(const float* __restrict__ x, int64_t n, const float* __restrict__ amax_in,
                                         int8_t* __restrict__ q) {
    float scale = lin_scale_from_absmax(*amax_in);
    float inv = lin_inv(scale);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        q[i] = lin_encode(x[i], inv);
}

__global__ void per_tensor_finalize_kernel(float* __restrict__ scale_io) {
    *scale_io = lin_scale_from_absmax(*scale_io);
}

__global__ void dequant_linear_kernel(const int8_t* __restrict__ q, const float* __restrict__ scales, float scale_arg,
                                      int64_t n, int block, float* __restrict__ out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float s = scales ? scales[block > 0 ? i / block : 0] : scale_arg;
        out[i] = __fmul_rn((float)q[i], s);
    }
}

__global__ void dequant_dynamic_kernel(const int8_t* __restrict__ q, const float* __restrict__ scales, int64_t n,
                                       int block, int is_signed, float* __restrict__ out) {
    __shared__ float map[256];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) map[i] = is_signed ? c_dmap_signed[i] : c_dmap_unsigned[i];
    __syncthreads();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = __fmul_rn(map[(uint8_t)q[i]], scales[i / block]);
}

// Blockwise encode: one CTA per block (any block size), two passes over the
// block (absmax, then encode).
__global__ void block_encode_kernel(const float* __restrict__ x, int64_t n, int block, int codec, int is_signed,
                                    int8_t* __restrict__ q, float* __restrict__ scales) {
    __shared__ float map[256];
    __shared__ float red[32];
    if (codec == AETH_CODEC_BLOCK_DYNAMIC) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) map[i] = is_signed ? c_dmap_signed[i] : c_dmap_unsigned[i];
    }
    const int64_t n_blocks = (n + block - 1) / block;
    for (int64_t b = blockIdx.x; b < n_blocks; b += gridDim.x) {
        int64_t s = b * block, e = s + block < n ? s + block : n;
        float a = 0.0f;
        for (int64_t i = s + threadIdx.x; i < e; i += blockDim.x) a = fmaxf(a, fabsf(x[i]));
        a = warp_max(a);
        __syncthreads();
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = a;
        __syncthreads();
        float amax = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) amax = fmaxf(amax, red[w]);
        if (codec == AETH_CODEC_BLOCK_LINEAR) {
            float scale = lin_scale_from_absmax(amax), inv = lin_inv(scale);
            for (int64_t i = s + threadIdx.x; i < e; i += blockDim.x) q[i] = lin_encode(x[i], inv);
            if (threadIdx.x == 0) scales[b] = scale;
        } else {
            const float inv = dyn_inv(amax);
            for (int64_t i = s + threadIdx.x; i < e; i += blockDim.x)
                q[i] = (int8_t)(uint8_t)dmap_encode(map, dyn_xn(x[i], inv));
            if (threadIdx.x == 0) scales[b] = amax;
        }
    }
}

}  // namespace aeth
