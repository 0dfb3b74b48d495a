// nf4.cuh -- NF4 (4-bit NormalFloat, 64-element blocks, fp32 absmax)
// dequantisation and bit-exact requantisation.
//
// Format (shard_engine/src/nf4.rs:6-83, shard_engine/python/pipeline/quantizer.py:21-75):
//   w[i] = CODES[nib(i)] * absmax[i / 64], nib(i) = high nibble of byte i/2 for even i.
// Quantisation: absmax = max|x| per block (stored raw); xn = x / max(absmax, 1e-8);
// code = argmin_c |xn - CODES[c]| with the first index winning ties (torch.argmin).
//
// The quantiser here is bit-exact with that definition while avoiding a
// division and a 16-way search per element: xn is approximated as x * (1/absmax)
// and classified with a 33-bucket table (bucket width 1/16 is narrower than the
// smallest gap between decision midpoints, 0.080, so a bucket holds at most one
// midpoint).  Any element whose approximation lies within 1e-6 of a midpoint --
// far wider than the few-ulp band in which the approximation or the fp32
// distance rounding could change the answer -- sends its block through the
// exact path (IEEE division and the full 16-code argmin).
#pragma once
#include "common.cuh"

namespace aeth {

__constant__ float c_nf4_codes[16] = {
    -1.0f,        -0.6961928f, -0.52507305f, -0.3949175f, -0.28444138f, -0.18477343f,
    -0.09105004f, 0.0f,        0.0795803f,   0.1609302f,  0.2461123f,   0.33791524f,
    0.44070983f,  0.562617f,   0.72295684f,  1.0f,
};

constexpr float kNf4NearWindow = 1e-6f;

// The block scale as the reference forms it (quantizer.py:35-36): absmax =
// max|x| is NaN when the block holds a NaN (torch's max propagates it), and
// clamp(min=1e-8) keeps a NaN.  Every element of such a block then gets code
// 0 (argmin over NaN distances), and +-inf / inf gives NaN as well.
__device__ __forceinline__ float fmax_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float nf4_safe(float amax) { return amax < 1e-8f ? 1e-8f : amax; }
// The stored absmax of a NaN block: the quiet NaN the reference's max returns
// for an input NaN (0x7fc00000), whatever NaN the device arithmetic produced.
__device__ __forceinline__ float nf4_store_amax(float amax) {
    return amax != amax ? __uint_as_float(0x7fc00000u) : amax;
}

struct Nf4Tables {
    float2 byte_lut[256];  // (CODES[byte >> 4], CODES[byte & 15])
    // {midpoint threshold or +inf, lower code index as int bits}; entries 33..63
    // are reached only by a NaN xn (index bits & 63) and send it to the exact path
    float2 bucket[64];
};

// Fill the shared tables; call with all threads of the CTA, then __syncthreads().
__device__ __forceinline__ void nf4_tables_init(Nf4Tables* t, int tid, int nthreads) {
    for (int i = tid; i < 256; i += nthreads)
        t->byte_lut[i] = make_float2(c_nf4_codes[i >> 4], c_nf4_codes[i & 15]);
    for (int b = 33 + tid; b < 64; b += nthreads) t->bucket[b] = make_float2(__int_as_float(0x7fc00000), 0.0f);
    for (int b = tid; b < 33; b += nthreads) {
        // bucket b holds xn with rint(16 xn) + 16 == b, i.e. [(b-16.5)/16, (b-15.5)/16)
        float lo = ((float)b - 16.5f) * 0.0625f, hi = ((float)b - 15.5f) * 0.0625f;
        int below = 0;
        float thr = __int_as_float(0x7f800000);  // +inf: no midpoint in this bucket
        int code = 0;
        for (int k = 0; k < 15; ++k) {
            float mid = (c_nf4_codes[k] + c_nf4_codes[k + 1]) * 0.5f;
            if (mid < lo) below = k + 1;
            else if (mid < hi) { thr = mid; code = k; }
        }
        if (thr == __int_as_float(0x7f800000)) code = below;
        t->bucket[b] = make_float2(thr, __int_as_float(code));
    }
}

// Exact reference decision for one element (quantizer.py:29-35).  Not
// inlined: it runs only for elements next to a decision boundary, and
// keeping it out of line keeps the unrolled fast path small.
__device__ __noinline__ uint32_t nf4_code_exact(float x, float safe) {
    float xn = __fdiv_rn(x, safe);
    uint32_t best = 0;
    float bd = fabsf(__fsub_rn(xn, c_nf4_codes[0]));
#pragma unroll
    for (int c = 1; c < 16; ++c) {
        float d = fabsf(__fsub_rn(xn, c_nf4_codes[c]));
        if (d < bd) { bd = d; best = (uint32_t)c; }
    }
    return best;
}

// Quantise N values (N a multiple of 8, all in one NF4 block with absmax
// `amax`) held in registers.  Output: N/8 words, each packing 8 codes in
// memory byte order (byte k = code[2k] << 4 | code[2k+1]).
template <int N>
__device__ __forceinline__ void nf4_quant_regs(const float (&v)[N], float amax, const float2* __restrict__ bucket,
                                               uint32_t (&packed)[N / 8]) {
    const float safe = nf4_safe(amax);
    const float inv = __frcp_rn(safe);
    uint32_t near[N / 8];
#pragma unroll
    for (int w = 0; w < N / 8; ++w) {
        uint32_t word = 0, nb = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float xn = __fmul_rn(v[w * 8 + j], inv);
            float t = __fmaf_rn(xn, 16.0f, 12582928.0f);  // 1.5*2^23 + 16: low bits = rint(16 xn) + 16
            float2 e = bucket[__float_as_int(t) & 63];
            float d = __fsub_rn(xn, e.x);
            uint32_t code = (uint32_t)__float_as_int(e.y) + (d > 0.0f ? 1u : 0u);
            nb |= (fabsf(d) >= kNf4NearWindow ? 0u : 1u) << j;  // NaN: exact path
            word |= code << (8 * (j >> 1) + ((j & 1) ? 0 : 4));
        }
        packed[w] = word;
        near[w] = nb;
    }
    // Rare: redo the elements next to a boundary with the exact definition.
#pragma unroll
    for (int w = 0; w < N / 8; ++w) {
        if (near[w]) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (near[w] & (1u << j)) {
                    const uint32_t sh = 8 * (j >> 1) + ((j & 1) ? 0 : 4);
                    packed[w] = (packed[w] & ~(0xfu << sh)) | (nf4_code_exact(v[w * 8 + j], safe) << sh);
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Tables for the fused epilogues.  byte_rep: the 256-entry byte table
// (CODES[byte >> 4], CODES[byte & 15]) in 16 copies, entry b of copy c at
// byte offset 128 b + 8 c, so the 16 lanes of a half-warp (copy = lane % 16;
// an 8-byte load is served per half-warp) read 16 different bank pairs
// whatever their bytes: one lookup costs the minimum two wavefronts per warp.
// One byte permute and a shift form the offset (nf4_dequant_word_s).
//
// Buckets: bucket b = rint(14 xn) + 14 (0..28; width 1/14 is narrower than the
// smallest gap between midpoints, 0.085, and every midpoint lies at least
// 3.4e-3 inside its bucket), read from the float bits of t = fma(x, 14 inv,
// 1.5*2^23 + 14) as bits(t) - 0x4B400000.  29 entries fit one warp: lane b
// holds entry b in a register and the fast path fetches entries with one
// shuffle; bucket32 keeps the same entries in shared memory for the
// divergent rare path.  Entry b = the NEGATED midpoint threshold of bucket b
// with (lower code + 1) stored in its low 4 mantissa bits (nf4_bucket32_entry),
// so the signed distance to the threshold is one fused multiply-add, inv x +
// entry; the perturbation (< 16 ulp, < 1e-6 absolute) is covered by the wider
// near-window kNf4NearWindow32.
// Window budget: the stored threshold moves by at most 15 ulp of the largest
// midpoint (0.8615: 8.9e-7); x * rcp(absmax) is within 2 ulp of x / absmax
// (2.4e-7); the fp32 midpoint and the reference's rounded distances add under
// 5e-8.  Total 1.2e-6, so 1.5e-6 leaves a quarter in reserve.  A near element
// is always near its own bucket's threshold (the 3.4e-3 margin).
// ---------------------------------------------------------------------------
constexpr float kNf4NearWindow32 = 1.5e-6f;
constexpr float kNf4BucketScale = 14.0f;
constexpr float kNf4BucketMagic = 12582926.0f;  // 1.5 * 2^23 + 14

struct Nf4Tables32 {
    float2 byte_rep[256 * 16];
    uint32_t bucket32[32];  // entries 0..28 used; 29..31 hold the top code, as the lanes do
};

// Entry of bucket b: with a midpoint between codes k and k + 1 inside,
// -midpoint with k + 1 in the low 4 bits; without one, +2.0 (the distance
// xn + 2 is positive for every |xn| <= 1 + 2^-20, so nothing is subtracted and
// no element is near) with the bucket's code itself.  Either way the low
// nibble is what the positive-distance case keeps, and it is at least 1
// wherever a negative distance subtracts 1.
__device__ __forceinline__ uint32_t nf4_bucket32_entry(int b) {
    const float lo = ((float)b - 14.5f) / kNf4BucketScale, hi = ((float)b - 13.5f) / kNf4BucketScale;
    int below = 0, code = -1;
    float thr = 0.0f;
    for (int k = 0; k < 15; ++k) {
        const float mid = (c_nf4_codes[k] + c_nf4_codes[k + 1]) * 0.5f;
        if (mid < lo) below = k + 1;
        else if (mid < hi) { thr = mid; code = k; }
    }
    if (code < 0) return __float_as_uint(2.0f) | (uint32_t)below;
    return (__float_as_uint(-thr) & ~15u) | (uint32_t)(code + 1);
}

__device__ __forceinline__ void nf4_tables32_init(Nf4Tables32* t, int tid, int nthreads) {
    for (int i = tid; i < 256 * 16; i += nthreads)  // entry i >> 4, copy i & 15
        t->byte_rep[i] = make_float2(c_nf4_codes[i >> 8], c_nf4_codes[(i >> 4) & 15]);
    for (int b = tid; b < 32; b += nthreads) t->bucket32[b] = nf4_bucket32_entry(b);
}


// Exact decisions for 8 elements (rare path; kept out of line).
__device__ __noinline__ uint32_t nf4_exact_word8(float a0, float a1, float a2, float a3, float a4, float a5, float a6,
                                                 float a7, float safe) {
    const float a[8] = {a0, a1, a2, a3, a4, a5, a6, a7};
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) word |= nf4_code_exact(a[j], safe) << (8 * (j >> 1) + ((j & 1) ? 0 : 4));
    return word;
}


// Rare-path repair of one fast-classified word: elements within the near
// window of their bucket's threshold (the lower code k = low bits - 1 of the
// entry) get the reference's decision between codes k and k + 1 from the
// IEEE quotient x / safe -- the other 14 codes are at least 0.03 further away
// -- with the lower code winning a tie, as torch.argmin does.
__device__ __noinline__ uint32_t nf4_fix_word8(uint32_t word, float a0, float a1, float a2, float a3, float a4,
                                               float a5, float a6, float a7, float inv, float safe,
                                               uint32_t bucket_bias) {
    const float a[8] = {a0, a1, a2, a3, a4, a5, a6, a7};
    const float invs = inv * kNf4BucketScale;
#pragma unroll 1
    for (int j = 0; j < 8; ++j) {
        // the fast classifier's bucket and distance, bit for bit (nf4_fast_word8_s)
        const float t = __fmaf_rn(a[j], invs, kNf4BucketMagic);
        uint32_t e;
        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(e) : "r"(bucket_bias + (__float_as_uint(t) << 2)));
        const float d = __fmaf_rn(a[j], inv, __uint_as_float(e));
        if (fabsf(d) < kNf4NearWindow32) {
            const uint32_t k = (e & 15u) - 1u;
            const float xe = __fdiv_rn(a[j], safe);
            const float dlo = fabsf(__fsub_rn(xe, c_nf4_codes[k])), dhi = fabsf(__fsub_rn(xe, c_nf4_codes[k + 1]));
            const uint32_t code = dhi < dlo ? k + 1 : k;
            const uint32_t sh = 8 * (j >> 1) + ((j & 1) ? 0 : 4);
            word = (word & ~(0xfu << sh)) | (code << sh);
        }
    }
    return word;
}

// bucket_bias: shared address of bucket32[0] minus (0x4B400000 << 2) modulo
// 2^32, so the entry of value t = fma(x, 14 inv, 1.5*2^23 + 14) sits at
// bucket_bias + (bits(t) << 2).  Only finite |xn| <= 1 + 2^-20 may be looked
// up there: callers decide elements of blocks holding a non-finite value on
// the exact path.
__device__ __forceinline__ uint32_t nf4_bucket_bias(const Nf4Tables32* t) {
    return smem_u32_addr(t->bucket32) - (0x4B400000u << 2);
}


// 8 values -> one packed word, two elements per step through the packed
// f32x2 instructions.  Byte k of the word = code[2k] << 4 | code[2k+1].  The
// signed distance d = xn + (-threshold) gives code = (lower + 1) - [d < 0];
// d == 0 lies in the near band.  Packing: the entries' low nibbles (lower + 1,
// 1..15) are funnel-shifted in from the top, one instruction per element, in
// the order 1,0,3,2,5,4,7,6 that puts element j at its nibble; the signs of
// the eight distances are gathered as bytes (prmt sign fill) and subtracted
// at the nibbles' low bits, which cannot borrow since every nibble is >= 1.
// Both the bucket index and the distance are single fused multiply-adds of the
// unscaled value: t = rn(fl(14 inv) w + 1.5*2^23 + 14) and d = rn(inv w -
// threshold).  The exact product moves d by under an ulp of xn from the
// separately rounded xn + entry, far inside kNf4NearWindow32, whose elements
// are decided again exactly; a bucket index that rounding moves across a
// bucket edge still classifies correctly, since every midpoint lies at least
// 3.4e-3 inside its bucket.  The entry comes from lane bits(t) mod 32 of the
// warp (lane_entry = bucket32[lane]): all 32 lanes must call this together.
// A non-finite value reads some lane's entry and gives a meaningless code,
// which callers replace on the exact path (their near flag is forced).
__device__ __forceinline__ uint32_t nf4_fast_word8_s(const float* w, float inv, uint32_t lane_entry, float& mind) {
    const float2 inv2 = make_float2(inv, inv);
    const float invs1 = inv * kNf4BucketScale;
    const float2 invs = make_float2(invs1, invs1), kbias = make_float2(kNf4BucketMagic, kNf4BucketMagic);
    uint32_t e[8], sg[8];
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        const float2 x = make_float2(w[2 * s], w[2 * s + 1]);
        const float2 t = fma2_rn(x, invs, kbias);  // low bits: rint(14 xn) + 14
        e[2 * s] = __shfl_sync(0xffffffffu, lane_entry, (int)__float_as_uint(t.x));
        e[2 * s + 1] = __shfl_sync(0xffffffffu, lane_entry, (int)__float_as_uint(t.y));
        const float2 d = fma2_rn(x, inv2, make_float2(__uint_as_float(e[2 * s]), __uint_as_float(e[2 * s + 1])));
        sg[2 * s] = __float_as_uint(d.x);
        sg[2 * s + 1] = __float_as_uint(d.y);
        mind = fmin3(mind, fabsf(d.x), fabsf(d.y));
    }
    uint32_t word = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        word = __funnelshift_r(word, e[2 * k + 1], 4);
        word = __funnelshift_r(word, e[2 * k], 4);
    }
    // sign bytes (0xff for d < 0) of the odd and the even elements, byte k for pair k
    const uint32_t odd = prmt(prmt(sg[1], sg[3], 0xFBu), prmt(sg[5], sg[7], 0xFBu), 0x5410u);
    const uint32_t even = prmt(prmt(sg[0], sg[2], 0xFBu), prmt(sg[4], sg[6], 0xFBu), 0x5410u);
    return word - (odd & 0x01010101u) - (even & 0x10101010u);
}

// Self-check of the classifier as the fused epilogues run it (fast word, then
// the near-window repair of flagged words) against nf4_code_exact, for one
// block scale: every magnitude bit pattern 0 .. bits(amax), each with both
// signs, eight values (four magnitudes) per word.  The loop trip count is the
// same for every lane (the classifier shuffles across the warp); words past
// the end repeat the top magnitude and are not counted.
__global__ void nf4_classify_selfcheck_kernel(float amax, unsigned long long* __restrict__ mismatches) {
    __shared__ uint32_t bucket32[32];
    if (threadIdx.x < 32) bucket32[threadIdx.x] = nf4_bucket32_entry((int)threadIdx.x);
    __syncthreads();
    const uint32_t lane_entry = bucket32[threadIdx.x & 31];
    const uint32_t bias = smem_u32_addr(bucket32) - (0x4B400000u << 2);
    const float safe = nf4_safe(amax), inv = __frcp_rn(safe);
    const uint32_t top = __float_as_uint(amax);
    const uint64_t nwords = ((uint64_t)top + 4) / 4;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t iters = (nwords + stride - 1) / stride;
    unsigned long long bad = 0;
    for (uint64_t it = 0; it < iters; ++it) {
        const uint64_t wi = it * stride + blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
        float w[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint64_t u = wi * 4 + j;
            w[2 * j] = __uint_as_float(u < top ? (uint32_t)u : top);
            w[2 * j + 1] = -w[2 * j];
        }
        float mind = 1.0f;
        uint32_t word = nf4_fast_word8_s(w, inv, lane_entry, mind);
        if (mind < kNf4NearWindow32)
            word = nf4_fix_word8(word, w[0], w[1], w[2], w[3], w[4], w[5], w[6], w[7], inv, safe, bias);
        if (wi < nwords) {
#pragma unroll 1
            for (int j = 0; j < 8; ++j) {
                const uint32_t got = (word >> (8 * (j >> 1) + ((j & 1) ? 0 : 4))) & 15u;
                bad += got != nf4_code_exact(w[j], safe);
            }
        }
    }
    bad = warp_sum_u64(bad);
    if ((threadIdx.x & 31) == 0 && bad) atomicAdd(mismatches, bad);
}

// Shared address of the replicated byte table, and this lane's copy offset
// before the final halving ((lane % 16) * 16, below 256: one byte).
__device__ __forceinline__ uint32_t nf4_byte_rep_base(const Nf4Tables32* t) { return smem_u32_addr(t->byte_rep); }
__device__ __forceinline__ uint32_t nf4_byte_rep_lane(int lane) { return (uint32_t)(lane & 15) * 16u; }

// Dequantise one packed word (8 elements) with this lane's copy of a
// replicated byte table; one packed multiply per byte.  One byte permute
// forms 256 byte + lane_off (byte 0 = the lane offset, byte 1 = byte k of the
// word, bytes 2 and 3 = the lane offset's zero byte 1): the offset itself for
// a table with a 256-byte entry stride (STRIDE128 = false: LOMO's, lane_off =
// 8 x copy), half of it for Nf4Tables32's 128-byte stride (lane_off = 16 x
// copy, nf4_byte_rep_lane).
template <bool STRIDE128 = false>
__device__ __forceinline__ void nf4_dequant_word_s(uint32_t word, float amax, uint32_t rep_base, uint32_t lane_off,
                                                   float* out8) {
    const float2 a2 = make_float2(amax, amax);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        float2 c;
        const uint32_t off = prmt(word, lane_off, 0x5504u | ((uint32_t)k << 4));
        asm("ld.shared.v2.f32 {%0, %1}, [%2];"
            : "=f"(c.x), "=f"(c.y)
            : "r"(rep_base + (STRIDE128 ? off >> 1 : off)));
        const float2 p = mul2_rn(c, a2);
        out8[2 * k] = p.x;
        out8[2 * k + 1] = p.y;
    }
}

// Dequantise 8 codes packed in one little-endian word into fp32 products.
__device__ __forceinline__ void nf4_dequant_word(uint32_t word, float amax, const float2* __restrict__ lut,
                                                 float* out8) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        float2 c = lut[(word >> (8 * k)) & 0xffu];
        out8[2 * k] = __fmul_rn(c.x, amax);
        out8[2 * k + 1] = __fmul_rn(c.y, amax);
    }
}

// ---------------------------------------------------------------------------
// Stand-alone dequantisation (K1).  Fast kernel: block == 64, n % 32 == 0,
// 16-byte aligned packed; each thread expands 16 bytes (32 elements).
// ---------------------------------------------------------------------------
template <typename OutT>
__device__ __forceinline__ void store_vals(OutT* out, int64_t base, const float* v, int cnt);

template <>
__device__ __forceinline__ void store_vals<float>(float* out, int64_t base, const float* v, int cnt) {
#pragma unroll
    for (int i = 0; i < 32; i += 4)
        *reinterpret_cast<float4*>(out + base + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    (void)cnt;
}

template <>
__device__ __forceinline__ void store_vals<__half>(__half* out, int64_t base, const float* v, int cnt) {
#pragma unroll
    for (int i = 0; i < 32; i += 8) {
        uint4 u;
        __half2 h0 = __floats2half2_rn(v[i], v[i + 1]), h1 = __floats2half2_rn(v[i + 2], v[i + 3]);
        __half2 h2 = __floats2half2_rn(v[i + 4], v[i + 5]), h3 = __floats2half2_rn(v[i + 6], v[i + 7]);
        u.x = *reinterpret_cast<uint32_t*>(&h0);
        u.y = *reinterpret_cast<uint32_t*>(&h1);
        u.z = *reinterpret_cast<uint32_t*>(&h2);
        u.w = *reinterpret_cast<uint32_t*>(&h3);
        *reinterpret_cast<uint4*>(out + base + i) = u;
    }
    (void)cnt;
}

template <>
__device__ __forceinline__ void store_vals<__nv_bfloat16>(__nv_bfloat16* out, int64_t base, const float* v, int cnt) {
#pragma unroll
    for (int i = 0; i < 32; i += 8) {
        uint4 u;
        __nv_bfloat162 h0 = __floats2bfloat162_rn(v[i], v[i + 1]), h1 = __floats2bfloat162_rn(v[i + 2], v[i + 3]);
        __nv_bfloat162 h2 = __floats2bfloat162_rn(v[i + 4], v[i + 5]), h3 = __floats2bfloat162_rn(v[i + 6], v[i + 7]);
        u.x = *reinterpret_cast<uint32_t*>(&h0);
        u.y = *reinterpret_cast<uint32_t*>(&h1);
        u.z = *reinterpret_cast<uint32_t*>(&h2);
        u.w = *reinterpret_cast<uint32_t*>(&h3);
        *reinterpret_cast<uint4*>(out + base + i) = u;
    }
    (void)cnt;
}

template <typename OutT>
__global__ void __launch_bounds__(256) nf4_dequant64_kernel(const uint8_t* __restrict__ packed,
                                                            const float* __restrict__ absmax, int64_t n_chunks,
                                                            OutT* __restrict__ out) {
    __shared__ float2 lut[256];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) lut[i] = make_float2(c_nf4_codes[i >> 4], c_nf4_codes[i & 15]);
    __syncthreads();
    for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < n_chunks; c += (int64_t)gridDim.x * blockDim.x) {
        uint4 w = __ldg(reinterpret_cast<const uint4*>(packed) + c);
        float amax = __ldg(absmax + (c >> 1));  // 32 elements per chunk, 64 per block
        float v[32];
        nf4_dequant_word(w.x, amax, lut, v);
        nf4_dequant_word(w.y, amax, lut, v + 8);
        nf4_dequant_word(w.z, amax, lut, v + 16);
        nf4_dequant_word(w.w, amax, lut, v + 24);
        store_vals<OutT>(out, c * 32, v, 32);
    }
}

// Generic dequantisation: any block size, any n, any alignment.
__global__ void nf4_dequant_generic_kernel(const uint8_t* __restrict__ packed, const float* __restrict__ absmax,
                                           int64_t n, int block, void* __restrict__ out, int out_dtype) {
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        uint8_t byte = packed[e >> 1];
        int nib = (e & 1) == 0 ? (byte >> 4) & 15 : byte & 15;
        float v = __fmul_rn(c_nf4_codes[nib], absmax[e / block]);
        if (out_dtype == AETH_DTYPE_F32) static_cast<float*>(out)[e] = v;
        else if (out_dtype == AETH_DTYPE_F16) static_cast<__half*>(out)[e] = __float2half_rn(v);
        else static_cast<__nv_bfloat16*>(out)[e] = __float2bfloat16_rn(v);
    }
}

// ---------------------------------------------------------------------------
// Stand-alone quantisation (K2).  Fast kernel: block == 64, n % 64 == 0;
// 4 threads per block, 16 elements each, absmax by two xor-shuffles.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) nf4_quant64_kernel(const void* __restrict__ x, int x_dtype, int64_t n_blocks,
                                                          uint8_t* __restrict__ packed, float* __restrict__ absmax) {
    __shared__ Nf4Tables tab;
    nf4_tables_init(&tab, threadIdx.x, blockDim.x);
    __syncthreads();
    const int64_t n_quads = n_blocks * 4;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    // The loop trip count is identical for the 4 lanes of a block (n_quads is a
    // multiple of 4 and the stride a multiple of 32), so the shuffles below see
    // all their partners.
    for (int64_t qd0 = blockIdx.x * (int64_t)blockDim.x + (threadIdx.x & ~31); qd0 < n_quads; qd0 += stride) {
        int64_t qd = qd0 + (threadIdx.x & 31);
        bool active = qd < n_quads;
        float v[16];
        int64_t e0 = qd * 16;
        if (active) {
            if (x_dtype == AETH_DTYPE_F32) {
                const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(x) + e0);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    float4 f = __ldg(p + i);
                    v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
                }
            } else {
                const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + e0);
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    uint4 u = __ldg(p + i);
                    uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        uint16_t lo = (uint16_t)(w[k] & 0xffffu), hi = (uint16_t)(w[k] >> 16);
                        if (x_dtype == AETH_DTYPE_BF16) {
                            v[8 * i + 2 * k] = bf16_bits_to_f32(lo);
                            v[8 * i + 2 * k + 1] = bf16_bits_to_f32(hi);
                        } else {
                            v[8 * i + 2 * k] = __half2float(__ushort_as_half(lo));
                            v[8 * i + 2 * k + 1] = __half2float(__ushort_as_half(hi));
                        }
                    }
                }
            }
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = 0.0f;
        }
        float a = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i) a = fmax_nan(a, fabsf(v[i]));
        a = fmax_nan(a, __shfl_xor_sync(0xffffffffu, a, 1));
        a = fmax_nan(a, __shfl_xor_sync(0xffffffffu, a, 2));
        if (active) {
            uint32_t pk[2];
            nf4_quant_regs<16>(v, a, tab.bucket, pk);
            *reinterpret_cast<uint2*>(packed + e0 / 2) = make_uint2(pk[0], pk[1]);
            if ((qd & 3) == 0) absmax[qd >> 2] = nf4_store_amax(a);
        }
    }
}

// Generic quantisation, pass 1: absmax per block (one warp per block).
__global__ void nf4_absmax_generic_kernel(const void* __restrict__ x, int x_dtype, int64_t n, int block,
                                          int64_t n_blocks, float* __restrict__ absmax) {
    int lane = threadIdx.x & 31;
    int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t b = warp; b < n_blocks; b += nwarps) {
        float a = 0.0f;
        for (int64_t i = lane; i < block; i += 32) {
            int64_t e = b * block + i;
            if (e < n) a = fmax_nan(a, fabsf(load_as_f32(x, e, x_dtype)));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a = fmax_nan(a, __shfl_xor_sync(0xffffffffu, a, o));
        if (lane == 0) absmax[b] = nf4_store_amax(a);
    }
}

// Generic quantisation, pass 2: one thread per packed byte.
__global__ void nf4_pack_generic_kernel(const void* __restrict__ x, int x_dtype, int64_t n, int block,
                                        const float* __restrict__ absmax, uint8_t* __restrict__ packed) {
    int64_t nbytes = (n + 1) / 2;
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < nbytes; k += (int64_t)gridDim.x * blockDim.x) {
        int64_t e0 = 2 * k, e1 = 2 * k + 1;
        uint32_t c0 = nf4_code_exact(load_as_f32(x, e0, x_dtype), nf4_safe(absmax[e0 / block]));
        // quantizer.py:37-39: an odd element count is padded with code 0.
        uint32_t c1 = e1 < n ? nf4_code_exact(load_as_f32(x, e1, x_dtype), nf4_safe(absmax[e1 / block])) : 0u;
        packed[k] = (uint8_t)((c0 << 4) | c1);
    }
}

}  // namespace aeth
