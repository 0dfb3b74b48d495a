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
// For x of one sign the binary search's code is a non-decreasing step
// function of the key bits(|x|) (x >= 0) or ~bits(|x|) (x < 0): between two
// neighbouring map entries it compares two rounded distances, one shrinking
// and one growing with x, so its decision flips exactly once, at a float that
// the host finds by bisection over the search itself -- ties and rounding
// included.  A magnitude selects bucket b = (bits(|x|) >> S) - 103 P, clamped
// to [0, N]: P buckets per octave over [2^-24, 2) (P = 64, S = 17 for the
// signed map; P = 128, S = 16 for the unsigned map, whose entries near 1 lie
// closer than 1/64 of an octave), bucket 0 also taking everything below
// 2^-24, and a last entry for |x| >= 2, infinities and NaN.  An entry is {threshold key, code below}: code = below +
// [key >= threshold], exact for every key of the bucket.  Buckets where the
// code changes more than once, and the last entry, are flagged kDmapSearch
// and sent to the binary search.
//
// The signed map's table has a half per sign (negative keys at offset
// kDmapLutEntries); the unsigned map's has only the non-negative half, and a
// negative x (never an Adam v) takes the search.  With these resolutions no
// bucket of either map holds two code changes, so only |x| >= 2, infinities
// and NaN (and a negative unsigned x) search.  aeth_selfcheck runs every float
// bit pattern through both paths.
// ---------------------------------------------------------------------------
constexpr int kDmapLutExpLo = 103;                      // 2^-24
constexpr int kDmapLutLog2P = 6;                        // signed map: 64 buckets per octave
constexpr int kDmapLutULog2P = 7;                       // unsigned map: 128 buckets per octave
constexpr int kDmapLutN = (128 - kDmapLutExpLo) << kDmapLutLog2P;     // 1600 buckets
constexpr int kDmapLutEntries = kDmapLutN + 1;                        // + the entry for |x| >= 2, inf, NaN
constexpr int kDmapLutUN = (128 - kDmapLutExpLo) << kDmapLutULog2P;   // 3200 buckets
constexpr int kDmapLutUEntries = kDmapLutUN + 1;
constexpr uint32_t kDmapSearch = 0x100u;                // in the code word: always search
__device__ uint2 g_dmap_lut_s[2 * kDmapLutEntries];    // signed map: x >= 0, then x < 0
__device__ uint2 g_dmap_lut_u[kDmapLutUEntries];       // unsigned map: x >= 0
__device__ uint32_t g_dmap_lut4_s[2 * kDmapLutEntries];  // the same, packed to 4 bytes (build_dmap_lut4)
__device__ uint32_t g_dmap_lut4_u[kDmapLutUEntries];

// The binary search on the host (dmap_encode's arithmetic: IEEE single
// subtraction and comparison).
inline uint32_t host_dmap_encode(const float* map, float x) {
    int lo = 0;
    for (int step = 128; step > 0; step >>= 1)
        if (map[lo + step - 1] < x) lo += step;
    if (lo == 0) return 0u;
    if (lo == 256) return 255u;
    const float dl = fabsf(x - map[lo - 1]), dh = fabsf(x - map[lo]);
    return dh < dl ? (uint32_t)lo : (uint32_t)(lo - 1);
}

// halves = 2 for the signed map (out: 2 * (nb + 1)), 1 for the unsigned one;
// 2^log2p buckets per octave, nb = 25 * 2^log2p buckets and the last entry.
inline void build_dmap_lut(const float map[256], int halves, int log2p, uint2* out) {
    const int nb = (128 - kDmapLutExpLo) << log2p, sh = 23 - log2p;
    for (int h = 0; h < halves; ++h) {
        uint2* o = out + h * (nb + 1);
        auto code_of = [&](uint32_t key) {
            const uint32_t bits = h ? (~key | 0x80000000u) : key;  // x of this half with that key
            float x;
            memcpy(&x, &bits, 4);
            return host_dmap_encode(map, x);
        };
        for (int b = 0; b < nb; ++b) {
            const uint32_t lo_ab = b == 0 ? 0u : (uint32_t)(b + (kDmapLutExpLo << log2p)) << sh;
            const uint32_t hi_ab = ((uint32_t)(b + 1 + (kDmapLutExpLo << log2p)) << sh) - 1u;
            const uint32_t kmin = h ? ~hi_ab : lo_ab, kmax = h ? ~lo_ab : hi_ab;
            const uint32_t cmin = code_of(kmin), cmax = code_of(kmax);
            if (cmin == cmax) {  // one code throughout: a threshold no key of the bucket misses or reaches
                if (cmin >= 1) o[b] = make_uint2(kmin, cmin - 1);
                else if (kmax != 0xffffffffu) o[b] = make_uint2(kmax + 1u, 0u);
                else o[b] = make_uint2(0xffffffffu, kDmapSearch);
            } else if (cmax == cmin + 1) {  // one flip: the first key with the upper code
                uint32_t lo = kmin, hi = kmax;
                while (hi - lo > 1u) {
                    const uint32_t mid = lo + (hi - lo) / 2u;
                    if (code_of(mid) == cmin) lo = mid;
                    else hi = mid;
                }
                o[b] = make_uint2(hi, cmin);
            } else {
                o[b] = make_uint2(0xffffffffu, kDmapSearch);
            }
        }
        o[nb] = make_uint2(0xffffffffu, kDmapSearch);
    }
}

// The 4-byte form of a bucket table for the flag-free encode (dmap_enc4_*):
// entry = t << 8 | code below, t = the threshold key's offset from the
// bucket's first key (0: every key of the bucket reaches it; 2^(23 - log2p):
// none does).  A bucket then spans 2^(23 - log2p) keys, bucket 0 included,
// because the flag-free encode raises magnitudes below 2^-24 to 2^-24; the
// offset of a key is its low 23 - log2p bits (keys ~bits(|x|) for x < 0
// count down from the bucket's largest magnitude, so the same holds).
// Entries only reachable outside that domain (|x| >= 2) are never used.
inline void build_dmap_lut4(const uint2* lut8, int halves, int log2p, uint32_t* out) {
    const int nb = (128 - kDmapLutExpLo) << log2p, sh = 23 - log2p;
    const uint32_t span = 1u << sh;
    for (int h = 0; h < halves; ++h) {
        for (int b = 0; b <= nb; ++b) {
            const uint2 e = lut8[h * (nb + 1) + b];
            const uint32_t lo_ab = (uint32_t)(b + (kDmapLutExpLo << log2p)) << sh, hi_ab = lo_ab + span - 1u;
            const uint32_t first = h ? ~hi_ab : lo_ab;
            uint32_t t = span;
            if (b < nb && !(e.y & kDmapSearch)) t = e.x <= first ? 0u : (e.x - first >= span ? span : e.x - first);
            out[h * (nb + 1) + b] = (t << 8) | (e.y & 0xffu);
        }
    }
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
        static uint2 lut_s[2 * kDmapLutEntries], lut_u[kDmapLutUEntries];
        build_dmap_lut(s, 2, kDmapLutLog2P, lut_s);
        build_dmap_lut(u, 1, kDmapLutULog2P, lut_u);
        AETH_CUDA(cudaMemcpyToSymbol(g_dmap_lut_s, lut_s, sizeof(lut_s)));
        AETH_CUDA(cudaMemcpyToSymbol(g_dmap_lut_u, lut_u, sizeof(lut_u)));
        static uint32_t lut4_s[2 * kDmapLutEntries], lut4_u[kDmapLutUEntries];
        build_dmap_lut4(lut_s, 2, kDmapLutLog2P, lut4_s);
        build_dmap_lut4(lut_u, 1, kDmapLutULog2P, lut4_u);
        AETH_CUDA(cudaMemcpyToSymbol(g_dmap_lut4_s, lut4_s, sizeof(lut4_s)));
        AETH_CUDA(cudaMemcpyToSymbol(g_dmap_lut4_u, lut4_u, sizeof(lut4_u)));
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

// Bucket-table encode without a branch (tables built by build_dmap_lut): `lut`
// is the signed map's table (both halves) for SIGNED, else the unsigned map's.
// Returns dmap_encode(map, xn) unless the bucket is flagged for the search (or,
// unsigned, xn is negative): then the result is meaningless and `flags` gets
// a bit above 0xff.  Callers OR the flags of several elements and search once.
template <bool SIGNED>
__device__ __forceinline__ uint32_t dmap_encode_lut_flag(const uint2* __restrict__ lut, float xn, uint32_t& flags) {
    const uint32_t bits = __float_as_uint(xn);
    const uint32_t ab = bits & 0x7fffffffu;
    constexpr int kLog2P = SIGNED ? kDmapLutLog2P : kDmapLutULog2P;
    constexpr int kN = SIGNED ? kDmapLutN : kDmapLutUN;
    const int b = min(max((int)(ab >> (23 - kLog2P)) - (kDmapLutExpLo << kLog2P), 0), kN);
    if (SIGNED) {
        const uint32_t neg = (uint32_t)((int32_t)bits >> 31);  // all ones for x < 0
        const uint2 e = lut[b + (neg & (uint32_t)kDmapLutEntries)];
        flags |= e.y;
        return e.y + ((ab ^ neg) >= e.x ? 1u : 0u);
    } else {
        const uint2 e = lut[b];
        flags |= e.y | ((bits >> 31) << 8);
        return e.y + (ab >= e.x ? 1u : 0u);
    }
}

// The same with the search taken for a flagged element: dmap_encode(map, xn)
// for every xn (`map` is the sorted map).
template <bool SIGNED>
__device__ __forceinline__ uint32_t dmap_encode_lut(const uint2* __restrict__ lut, const float* __restrict__ map,
                                                    float xn) {
    uint32_t flags = 0;
    const uint32_t code = dmap_encode_lut_flag<SIGNED>(lut, xn, flags);
    if (flags > 0xffu) return dmap_encode_rare(map, xn);
    return code;
}

// Flag-free bucket encodes for a block whose normalised values are all
// finite, |xn| <= 1 + 2^-22 (x = xn * (1 / absmax) of a finite absmax): no
// bucket in that range holds two code changes or needs the search, so the
// entry carries no flag and the index needs no upper clamp.  A magnitude
// below 2^-24 is raised to 2^-24: every key of bucket 0 has the code of 0.0 in
// both maps (their smallest non-zero entries are above 1.6e-7), so the raised
// key encodes the same.  The tables are the 4-byte ones (build_dmap_lut4):
// code = below + [key offset >= t], in the low byte of the result (the byte
// never carries: a bucket whose compare can add one has a code above it).
// The bucket index is a multiply-high by a power of two known only at run
// time (m15 = 2^15: bits >> 17, m16 = 2^16: bits >> 16, m1 = 2: the sign bit),
// which issues on the FMA pipe rather than as a shift on the integer pipe.
// lut_adj is the table's shared address minus 4 x the first bucket's index
// (kDmapLutExpLo << log2 P).
// The compare offset >= t is done as 256 offset + 255 >= t << 8 | below (m8 =
// 256 at run time: a multiply-add instead of a shift of the entry).
__device__ __forceinline__ uint32_t dmap_enc4_s(uint32_t lut_adj, float xn, uint32_t m1, uint32_t m8, uint32_t m15) {
    const uint32_t xb = __float_as_uint(xn);
    const uint32_t km = __float_as_uint(fmaxf(fabsf(xn), 0x1p-24f));
    const uint32_t neg = (uint32_t)((int32_t)xb >> 31);
    const uint32_t idx = __umulhi(km, m15) + __umulhi(xb, m1) * (uint32_t)kDmapLutEntries;
    const uint32_t e = lds_u32(lut_adj + idx * 4u);
    return e + (((km ^ neg) & 0x1ffffu) * m8 + 255u >= e ? 1u : 0u);
}

__device__ __forceinline__ uint32_t dmap_enc4_u(uint32_t lut_adj, float xn, uint32_t m8, uint32_t m16) {
    const uint32_t k = __float_as_uint(fmaxf(xn, 0x1p-24f));
    const uint32_t e = lds_u32(lut_adj + __umulhi(k, m16) * 4u);
    return e + ((k & 0xffffu) * m8 + 255u >= e ? 1u : 0u);
}

// Every float bit pattern through dmap_encode_lut and dmap_encode; counts
// disagreements (a self-check of the bucket tables, run by the test suite).
// Patterns with |x| <= 1 + 2^-22 (signed map) or 0 <= x <= 1 + 2^-22
// (unsigned map; -0.0 included) also go through the flag-free encode.
__global__ void dmap_selfcheck_kernel(int is_signed, unsigned long long* __restrict__ mismatches, uint32_t one) {
    __shared__ float map[256];
    __shared__ uint2 lut[2 * kDmapLutEntries];
    __shared__ uint32_t lut4[2 * kDmapLutEntries];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) map[i] = is_signed ? c_dmap_signed[i] : c_dmap_unsigned[i];
    static_assert(kDmapLutUEntries <= 2 * kDmapLutEntries, "the unsigned table must fit the signed one's space");
    for (int i = threadIdx.x; i < (is_signed ? 2 * kDmapLutEntries : kDmapLutUEntries); i += blockDim.x) {
        lut[i] = is_signed ? g_dmap_lut_s[i] : g_dmap_lut_u[i];
        lut4[i] = is_signed ? g_dmap_lut4_s[i] : g_dmap_lut4_u[i];
    }
    __syncthreads();
    const uint32_t adj = smem_u32_addr(lut4) - (uint32_t)(kDmapLutExpLo << (is_signed ? kDmapLutLog2P : kDmapLutULog2P)) * 4u;
    const uint32_t m1 = one << 1, m8 = one << 8, m15 = one << 15, m16 = one << 16;
    const uint32_t top = __float_as_uint(1.0f) + 2u;  // bits of 1 + 2^-22
    unsigned long long bad = 0;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < (1ull << 32); i += stride) {
        const float x = __uint_as_float((uint32_t)i);
        const uint32_t want = dmap_encode(map, x);
        const uint32_t got = is_signed ? dmap_encode_lut<true>(lut, map, x) : dmap_encode_lut<false>(lut, map, x);
        bad += got != want;
        const uint32_t ab = (uint32_t)i & 0x7fffffffu;
        if (is_signed && ab <= top) bad += (dmap_enc4_s(adj, x, m1, m8, m15) & 0xffu) != want;
        if (!is_signed && ((uint32_t)i <= top || (uint32_t)i == 0x80000000u))
            bad += (dmap_enc4_u(adj, x, m8, m16) & 0xffu) != want;
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
