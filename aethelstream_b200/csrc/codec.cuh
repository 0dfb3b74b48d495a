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

// ---------------------------------------------------------------------------
// Bucket tables for a fast dynamic-map encode that always returns what the
// binary search (dmap_encode) returns.
//
// The encode is a step function of the magnitude a = |xn|: the code changes
// only at the decision points between neighbouring map entries, each within
// 1.5 ulp of the real midpoint of the two entries (the binary search's two
// distances each carry at most half an ulp of error, plus the rounding of the
// midpoint to float).  A magnitude selects bucket b = (bits(a) >> 17) -
// (103 << 6), clamped to [0, kDmapLutN]: 64 buckets per octave over
// [2^-24, 2), bucket 0 also taking everything below 2^-24, and a last entry
// for a >= 2, infinities and NaN.  An entry is {threshold bits, code below}:
// the float bits of the one decision threshold within 56 bit steps of the
// bucket (several midpoints of the map fall exactly on bucket edges), or
// kDmapNoThr, which no magnitude reaches; code = below + [bits(a) >=
// threshold].  The binary search handles magnitudes within kDmapGuard bit
// steps of the threshold and entries flagged kDmapSearch: buckets with two
// thresholds near them and the last entry.
//
// Table 0 covers the signed map's non-negative half (indices 127..255); the
// map is symmetric about index 127 except for the extra entry 1.0 at 255, so a
// negative xn encodes as 254 - code(|xn|) (0 for codes 254 and 255).  Table 1
// covers the unsigned map, whose entry 0 is 0.0 and nearest to every negative
// xn.  Exact ties (xn on a real midpoint) always lie in the guard band, where
// the binary search applies its own tie rule.
// ---------------------------------------------------------------------------
constexpr int kDmapLutExpLo = 103;                     // 2^-24
constexpr int kDmapLutN = (128 - kDmapLutExpLo) << 6;  // 1600 buckets
constexpr int kDmapLutEntries = kDmapLutN + 1;         // + the entry for a >= 2, inf, NaN
constexpr uint32_t kDmapGuard = 8;                     // bit steps (ulp) around a threshold
constexpr uint32_t kDmapReach = 56;                    // thresholds this far outside a bucket count
constexpr uint32_t kDmapNoThr = 0xc0000000u;           // above every magnitude, far from all of them
constexpr uint32_t kDmapSearch = 0x100u;               // in the code word: always search
__device__ uint2 g_dmap_lut[2][kDmapLutEntries];

inline void build_dmap_lut(const float map[256], int is_signed, uint2* out) {
    std::vector<std::pair<double, int>> M;  // entries ascending by magnitude, with their codes
    for (int i = is_signed ? 127 : 0; i < 256; ++i) M.push_back({(double)map[i], i});
    auto bits_of = [](double v) {
        const float f = (float)v;
        uint32_t u;
        memcpy(&u, &f, 4);
        return u;
    };
    for (int b = 0; b < kDmapLutN; ++b) {
        const uint32_t lo_bits = (uint32_t)(b + (kDmapLutExpLo << 6)) << 17;
        const uint32_t hi_bits = lo_bits + (1u << 17);
        // midpoints (as floats) within kDmapReach bit steps of the bucket;
        // bucket 0 also holds everything below 2^-24
        const uint32_t ext_lo = b == 0 ? 0u : lo_bits - kDmapReach, ext_hi = hi_bits + kDmapReach;
        int nmid = 0, kmid = -1;
        for (size_t k = 0; k + 1 < M.size(); ++k) {
            const uint32_t tb = bits_of(0.5 * (M[k].first + M[k + 1].first));
            if (tb >= ext_lo && tb < ext_hi) { ++nmid; kmid = (int)k; }
        }
        if (nmid == 0) {
            float lof;
            memcpy(&lof, &lo_bits, 4);
            const double lo = b == 0 ? 0.0 : (double)lof;
            size_t k = 0;  // the nearest entry is the same over the whole bucket
            while (k + 1 < M.size() && 0.5 * (M[k].first + M[k + 1].first) < lo) ++k;
            out[b] = make_uint2(kDmapNoThr, (uint32_t)M[k].second);
        } else if (nmid == 1 && b > 0) {
            out[b] = make_uint2(bits_of(0.5 * (M[kmid].first + M[kmid + 1].first)), (uint32_t)M[kmid].second);
        } else {
            out[b] = make_uint2(kDmapNoThr, kDmapSearch);
        }
    }
    out[kDmapLutN] = make_uint2(kDmapNoThr, kDmapSearch);
}

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
        static uint2 lut[2][kDmapLutEntries];
        build_dmap_lut(s, 1, lut[0]);
        build_dmap_lut(u, 0, lut[1]);
        AETH_CUDA(cudaMemcpyToSymbol(g_dmap_lut, lut, sizeof(lut)));
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

// The binary search as an out-of-line call for the rare cases of the bucket
// encoder, so that the compiler branches around it instead of evaluating it
// for every element under a predicate.
__device__ __noinline__ uint32_t dmap_encode_rare(const float* map, float xn) { return dmap_encode(map, xn); }

// Bucket-table encode (tables built by build_dmap_lut); `lut` is table 0 for
// the signed map and table 1 for the unsigned one, `map` the sorted map for
// the rare binary-search cases.  Returns dmap_encode(map, xn) for every xn.
template <bool SIGNED>
__device__ __forceinline__ uint32_t dmap_encode_lut(const uint2* __restrict__ lut, const float* __restrict__ map,
                                                    float xn) {
    const uint32_t ab = __float_as_uint(xn) & 0x7fffffffu;
    const int b = min(max((int)(ab >> 17) - (kDmapLutExpLo << 6), 0), kDmapLutN);
    const uint2 e = lut[b];
    uint32_t code = e.y + (ab >= e.x ? 1u : 0u);
    // signed: mirror image; unsigned: every negative value is nearest to entry 0 (= 0)
    if (xn < 0.0f) code = SIGNED ? (uint32_t)max(254 - (int)code, 0) : 0u;
    if (e.y > 0xffu || ab - e.x + kDmapGuard < 2u * kDmapGuard) code = dmap_encode_rare(map, xn);
    return code;
}

// Every float bit pattern through dmap_encode_lut and dmap_encode; counts
// disagreements (a self-check of the bucket tables, run by the test suite).
__global__ void dmap_selfcheck_kernel(int is_signed, unsigned long long* __restrict__ mismatches) {
    __shared__ float map[256];
    __shared__ uint2 lut[kDmapLutEntries];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) map[i] = is_signed ? c_dmap_signed[i] : c_dmap_unsigned[i];
    for (int i = threadIdx.x; i < kDmapLutEntries; i += blockDim.x) lut[i] = g_dmap_lut[is_signed ? 0 : 1][i];
    __syncthreads();
    unsigned long long bad = 0;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < (1ull << 32); i += stride) {
        const float x = __uint_as_float((uint32_t)i);
        const uint32_t want = dmap_encode(map, x);
        const uint32_t got = is_signed ? dmap_encode_lut<true>(lut, map, x) : dmap_encode_lut<false>(lut, map, x);
        bad += got != want;
    }
    bad = warp_sum_u64(bad);
    if ((threadIdx.x & 31) == 0 && bad) atomicAdd(mismatches, bad);
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
