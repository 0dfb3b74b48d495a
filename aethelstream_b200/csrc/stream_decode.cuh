// stream_decode.cuh -- the steps on either side of the optimizer path in the
// streaming pipeline: flowcast's decode of quantised weights to f16
// (flowcast/src/decode.rs:63-104,191-210) and the BF16 stochastic-rounding
// write-back of the master weights (doublepass/src/precision.rs:124-217).
//
// Decode: HBM-bound at 3 (INT8) or 2.5 (NF4) bytes per element; each warp
// moves whole contiguous spans per load and store instruction.  The f16 conversion is flowcast's own: exponent
// rebias and mantissa truncation, +-0 below the normal range, +-inf above it.
// flowcast packs NF4 with the LOW nibble first and one absmax per tensor
// (shard_engine's format, high nibble first with 64-element blocks, is
// aeth_nf4_dequant's).
//
// Write-back: master += delta, then stochastic rounding to bf16 with 16 random
// bits per element from a 64-bit LCG advanced once per element in order.  The
// LCG is affine (x -> A x + C mod 2^64), so k steps are one affine map
// (A^k, C (A^k - 1) / (A - 1)); maps for 2^j steps sit in constant memory, and
// each thread starts from the state of its first element, as the sequential
// loop would reach it, then steps forward.  The results are the reference's bit
// for bit.
#pragma once
#include "nf4.cuh"

namespace aeth {

// precision.rs:212-217
constexpr uint64_t kLcgA = 6364136223846793005ull;
constexpr uint64_t kLcgC = 1442695040888963407ull;

struct Affine64 {
    uint64_t a, c;
};

// (second after first): x -> s.a (f.a x + f.c) + s.c
__host__ __device__ inline Affine64 affine_then(Affine64 first, Affine64 second) {
    return Affine64{second.a * first.a, second.a * first.c + second.c};
}

__constant__ Affine64 c_lcg_pow2[64];  // the map of 2^j LCG steps

inline void lcg_pow2_host(Affine64 out[64]) {
    Affine64 m{kLcgA, kLcgC};
    for (int j = 0; j < 64; ++j) {
        out[j] = m;
        m = affine_then(m, m);
    }
}

// The map of k steps, from the 2^j maps (host or constant-memory table).
__host__ __device__ inline Affine64 lcg_jump(uint64_t k, const Affine64* pow2) {
    Affine64 r{1ull, 0ull};
    for (int j = 0; k != 0; ++j, k >>= 1)
        if (k & 1ull) r = affine_then(r, pow2[j]);
    return r;
}

// The NaN an x86-64 scalar SSE operation returns, which is what the reference
// (host code) produces: the first NaN operand, quieted, else the default NaN
// 0xFFC00000 of an invalid operation (inf - inf, 0 x inf).  The device's own
// NaN is 0x7FFFFFFF; its sign and low bits would decide the f16 sign and the
// stochastic rounding differently.
__device__ __forceinline__ float x86_nan(float a, float b) {
    const uint32_t ua = __float_as_uint(a), ub = __float_as_uint(b);
    if ((ua & 0x7fffffffu) > 0x7f800000u) return __uint_as_float(ua | 0x00400000u);
    if ((ub & 0x7fffffffu) > 0x7f800000u) return __uint_as_float(ub | 0x00400000u);
    return __uint_as_float(0xffc00000u);
}
__device__ __forceinline__ float x86_mul(float a, float b) {
    const float p = __fmul_rn(a, b);
    return p != p ? x86_nan(a, b) : p;
}
__device__ __forceinline__ float x86_add(float a, float b) {
    const float s = __fadd_rn(a, b);
    return s != s ? x86_nan(a, b) : s;
}

// decode.rs:191-210, without branches: on |bits| the rebiased exponent and
// truncated mantissa are (|bits| >> 13) - (112 << 10) for exponents 113..142;
// below (f16 exponent <= 0) the result is +-0, above it +-inf, and NaN keeps
// only the quiet bit (0x7E00).
__device__ __forceinline__ uint16_t fc_f32_to_f16(float v) {
    const uint32_t bits = __float_as_uint(v);
    const uint32_t mag = bits & 0x7fffffffu;
    uint32_t h = (mag >> 13) - (112u << 10);
    h = mag < 0x38800000u ? 0u : h;
    h = mag >= 0x47800000u ? (mag > 0x7f800000u ? 0x7e00u : 0x7c00u) : h;
    return (uint16_t)(((bits >> 16) & 0x8000u) | h);
}

__device__ __forceinline__ uint32_t fc_pack2(float lo, float hi) {
    return (uint32_t)fc_f32_to_f16(lo) | ((uint32_t)fc_f32_to_f16(hi) << 16);
}

// Both decoders give each warp 128 consecutive 32-bit input words per
// iteration: lane l reads words l, 32 + l, 64 + l and 96 + l (128 contiguous
// bytes per load instruction) and writes each word's f16 values to the
// matching place, so every store instruction of the warp covers one
// contiguous span of whole sectors.  (A lane writing its own contiguous 64
// bytes as four 16-byte stores leaves half-written sectors per instruction,
// which ran at half the bandwidth.)
constexpr int kDecodeWords = 128;  // input words per warp and iteration

// decode.rs:63-86: out[i] = f16(i8 * scale[ch]), ch = i / per (per = max(n / channels, 1);
// 0 without channels), a channel at or past n_scales decoding with 1.0.  The
// channel comes from a double-precision reciprocal of per (exact for element
// indices below 2^53 after a one-step correction), once per word; a word
// inside one channel with a finite scale multiplies without NaN handling.
__device__ __forceinline__ int64_t fc_channel(int64_t e, int64_t per, double inv_per) {
    int64_t c = (int64_t)((double)e * inv_per);
    if (c * per > e) --c;
    else if ((c + 1) * per <= e) ++c;
    return c;
}

// The signed byte k of w as a float, exactly, without a conversion instruction:
// 1.5 * 2^23 + b has b in its low mantissa bits; subtracting 1.5 * 2^23 is exact.
__device__ __forceinline__ float fc_byte_f32(uint32_t w, int k) {
    const int32_t b = (int32_t)(w << (24 - 8 * k)) >> 24;
    return __fsub_rn(__int_as_float(0x4B400000 + b), 12582912.0f);
}

__device__ __forceinline__ uint2 fc_int8_word(uint32_t w, int64_t e0, const float* __restrict__ scales,
                                              int64_t n_scales, int64_t per, double inv_per, int has_channels) {
    float s0 = n_scales > 0 ? scales[0] : 1.0f;
    int64_t next = INT64_MAX;
    if (has_channels) {
        const int64_t ch = fc_channel(e0, per, inv_per);
        s0 = ch < n_scales ? scales[ch] : 1.0f;
        next = (ch + 1) * per;
    } else {
        s0 = n_scales > 0 ? scales[0] : 1.0f;
    }
    float v[4];
    if (e0 + 3 < next && fabsf(s0) <= 3.402823466e38f) {
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = __fmul_rn(fc_byte_f32(w, k), s0);
    } else {  // a channel boundary inside the word, or an infinite or NaN scale
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            float s = s0;
            if (e0 + k >= next) {
                const int64_t c = fc_channel(e0 + k, per, inv_per);
                s = c < n_scales ? scales[c] : 1.0f;
            }
            v[k] = x86_mul(fc_byte_f32(w, k), s);
        }
    }
    return make_uint2(fc_pack2(v[0], v[1]), fc_pack2(v[2], v[3]));
}

// A CTA's 8 warps cover 1024 consecutive words (4096 elements) per iteration.
// When a channel spans at least that many elements, the span meets at most two
// channels, and the 256 possible products of each are tabulated as f16 in
// shared memory first: one table lookup per element.  Otherwise every word
// computes its products.
constexpr int kDecodeSpan = 8 * kDecodeWords * 4;  // elements per CTA iteration

__global__ void __launch_bounds__(256) fc_decode_int8_kernel(const int8_t* __restrict__ src, int64_t n,
                                                             const float* __restrict__ scales, int64_t n_scales,
                                                             int64_t per, double inv_per, int has_channels,
                                                             uint16_t* __restrict__ out) {
    __shared__ uint16_t tab[2][256];
    const uint32_t* src32 = reinterpret_cast<const uint32_t*>(src);
    const int64_t nw = n / 4;  // whole words
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const bool tabulate = !has_channels || per >= kDecodeSpan;
    for (int64_t base = (int64_t)blockIdx.x * kDecodeSpan; base < nw * 4; base += (int64_t)gridDim.x * kDecodeSpan) {
        const int64_t w0 = base / 4 + warp * kDecodeWords;
        uint32_t q[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            const int64_t wi = w0 + h * 32 + lane;
            q[h] = wi < nw ? __ldcs(src32 + wi) : 0u;
        }
        if (tabulate) {
            // the span's channels: ch_a from its first element, ch_a + 1 from `split` on
            const int64_t ch_a = has_channels ? fc_channel(base, per, inv_per) : 0;
            const int64_t split = has_channels ? (ch_a + 1) * per : INT64_MAX;
            __syncthreads();  // the previous iteration's lookups are done
            {
                const int t = threadIdx.x;  // 256 threads: one byte value each
                const float b = fc_byte_f32((uint32_t)t, 0);
                const float sa = ch_a < n_scales ? scales[ch_a] : 1.0f;
                const float sb = ch_a + 1 < n_scales ? scales[ch_a + 1] : 1.0f;
                tab[0][t] = fc_f32_to_f16(x86_mul(b, sa));
                tab[1][t] = fc_f32_to_f16(x86_mul(b, has_channels ? sb : sa));
            }
            __syncthreads();
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                const int64_t wi = w0 + h * 32 + lane;
                if (wi < nw) {
                    const int64_t e0 = wi * 4;
                    uint32_t o[4];
#pragma unroll
                    for (int k = 0; k < 4; ++k) o[k] = tab[e0 + k >= split][(q[h] >> (8 * k)) & 0xffu];
                    __stcs(reinterpret_cast<uint2*>(out) + wi, make_uint2(o[0] | (o[1] << 16), o[2] | (o[3] << 16)));
                }
            }
        } else {
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                const int64_t wi = w0 + h * 32 + lane;
                if (wi < nw)
                    __stcs(reinterpret_cast<uint2*>(out) + wi,
                           fc_int8_word(q[h], wi * 4, scales, n_scales, per, inv_per, has_channels));
            }
        }
    }
    // ragged tail (n % 4 elements)
    for (int64_t e = nw * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t ch = has_channels ? fc_channel(e, per, inv_per) : 0;
        out[e] = fc_f32_to_f16(x86_mul((float)src[e], ch < n_scales ? scales[ch] : 1.0f));
    }
}

// decode.rs:88-104: byte k -> elements 2k (low nibble) and 2k + 1 (high nibble).
// The 16 decoded values depend only on the code, so a 256-entry table holds
// the f16 pair of every byte: one lookup per two elements.
__global__ void __launch_bounds__(256) fc_decode_nf4_kernel(const uint8_t* __restrict__ src, int64_t nbytes,
                                                            float absmax, uint16_t* __restrict__ out) {
    __shared__ uint32_t pair[256];
    for (int b = threadIdx.x; b < 256; b += blockDim.x)
        pair[b] = fc_pack2(x86_mul(c_nf4_codes[b & 15], absmax), x86_mul(c_nf4_codes[b >> 4], absmax));
    __syncthreads();
    const uint32_t* src32 = reinterpret_cast<const uint32_t*>(src);
    const int64_t nw = nbytes / 4;
    const int lane = threadIdx.x & 31;
    const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t w0 = ((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5) * kDecodeWords; w0 < nw;
         w0 += warps * kDecodeWords) {
        uint32_t q[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            const int64_t wi = w0 + h * 32 + lane;
            q[h] = wi < nw ? __ldcs(src32 + wi) : 0u;
        }
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            const int64_t wi = w0 + h * 32 + lane;
            if (wi < nw)
                __stcs(reinterpret_cast<uint4*>(out) + wi,
                       make_uint4(pair[q[h] & 0xffu], pair[(q[h] >> 8) & 0xffu], pair[(q[h] >> 16) & 0xffu],
                                  pair[q[h] >> 24]));
        }
    }
    for (int64_t k = nw * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < nbytes;
         k += (int64_t)gridDim.x * blockDim.x)
        reinterpret_cast<uint32_t*>(out)[k] = pair[src[k]];
}

// precision.rs:124-136: round up when the discarded 16 bits exceed the random
// ones; saturating at 0xFFFF.
__device__ __forceinline__ uint32_t sr_bf16(float v, uint32_t rand16) {
    const uint32_t bits = __float_as_uint(v);
    const uint32_t hi = bits >> 16;
    return ((bits & 0xffffu) > rand16 && hi != 0xffffu) ? hi + 1u : hi;
}

// precision.rs:184-202 over 4 consecutive elements per thread and iteration.
// x0 is the LCG state before element 0; element i draws from the state after
// i + 1 steps.  `step` is the map of 4 x (threads in the grid) steps.
__global__ void __launch_bounds__(256) bf16_sr_update_kernel(float* __restrict__ master,
                                                             const float* __restrict__ delta, int64_t n, uint64_t x0,
                                                             Affine64 step, uint16_t* __restrict__ bf16_out) {
    const int64_t gtid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t stride4 = (int64_t)gridDim.x * blockDim.x * 4;
    const Affine64 start = lcg_jump((uint64_t)(gtid * 4 + 1), c_lcg_pow2);
    uint64_t xf = start.a * x0 + start.c;  // state drawn by this thread's first element
    for (int64_t e0 = gtid * 4; e0 < n; e0 += stride4) {
        uint64_t x = xf;
        if (e0 + 4 <= n) {
            float4 m = *reinterpret_cast<const float4*>(master + e0);
            const float4 d = __ldcs(reinterpret_cast<const float4*>(delta + e0));
            float v[4] = {x86_add(m.x, d.x), x86_add(m.y, d.y), x86_add(m.z, d.z), x86_add(m.w, d.w)};
            uint32_t b[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                b[k] = sr_bf16(v[k], (uint32_t)(x >> 33) & 0xffffu);
                x = kLcgA * x + kLcgC;
            }
            *reinterpret_cast<float4*>(master + e0) = make_float4(__uint_as_float(b[0] << 16), __uint_as_float(b[1] << 16),
                                                                  __uint_as_float(b[2] << 16), __uint_as_float(b[3] << 16));
            if (bf16_out)
                *reinterpret_cast<uint2*>(bf16_out + e0) = make_uint2(b[0] | (b[1] << 16), b[2] | (b[3] << 16));
        } else {
            for (int64_t e = e0; e < n; ++e) {
                const uint32_t bb = sr_bf16(x86_add(master[e], delta[e]), (uint32_t)(x >> 33) & 0xffffu);
                x = kLcgA * x + kLcgC;
                master[e] = __uint_as_float(bb << 16);
                if (bf16_out) bf16_out[e] = (uint16_t)bb;
            }
        }
        xf = step.a * xf + step.c;
    }
}

}  // namespace aeth
