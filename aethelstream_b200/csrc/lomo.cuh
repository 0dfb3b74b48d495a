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

// Shared tables of the update kernel.  rep: 256 entries of 256 bytes; entry b
// holds the NF4 byte table's pair (CODES[b >> 4], CODES[b & 15]) in 16 copies
// at 8 c (c = lane % 16) and, for the dynamic codec, map entry b in 32 copies
// at 128 + 4 lane -- so one byte permute forms either offset from the packed
// code word and the lane (nf4_dequant_word_s), and no lookup of a warp meets a
// bank conflict whatever the codes.  bucket32: the 29-bucket classifier of the
// fused apply epilogue (requant); dm and dlut4: the signed map (for the rare
// binary search) and its 4-byte bucket table (the flag-free encode of finite
// blocks, dmap_enc4_s).
constexpr int kLomoGroups = 5;  // independent 128-thread groups per CTA
constexpr int kLomoThreads = 128 * kLomoGroups;
struct LomoTables {
    uint8_t rep[256 * 256];
    uint32_t bucket32[32];
    float dm[256];
    uint32_t dlut4[2 * kDmapLutEntries];
};
constexpr int kLomoSmem = (int)sizeof(LomoTables);

// A CTA is kLomoGroups independent groups of 128 threads that share one copy
// of the tables.  A group takes one momentum block of 2048 elements per
// iteration and synchronises on its own named barrier; thread t of the group
// owns 16 consecutive elements, so 4 consecutive threads form one NF4 block of
// 64 and each warp a quarter of the momentum block.  The next block's
// gradient, momentum and weight words are loaded while the current one is
// processed.  Element pairs go through the packed f32x2 multiply; sums that
// must round twice add with scalar adds (a packed add of fresh products would
// be fused).
template <int CODEC>
__global__ void __launch_bounds__(kLomoThreads, 1)
    lomo_update_kernel(const uint16_t* __restrict__ g, int64_t n, const double* __restrict__ sq, float max_norm,
                       float lr, float beta, int8_t* __restrict__ mom8, float* __restrict__ mom_scales,
                       uint8_t* __restrict__ wp, float* __restrict__ wa, float* __restrict__ prequant, uint32_t one) {
    extern __shared__ __align__(16) uint8_t lomo_smem[];
    LomoTables& tab = *reinterpret_cast<LomoTables*>(lomo_smem);
    __shared__ uint32_t red[kLomoGroups][2][4];  // NaN-propagating momentum maxima (bits), by block parity
    __shared__ uint32_t red2[kLomoGroups][4];    // NaN-ignoring maxima of a block holding NaN or inf
    for (int i = threadIdx.x; i < 256 * 16; i += blockDim.x) {
        const int b = i >> 4;
        *reinterpret_cast<float2*>(tab.rep + b * 256 + (i & 15) * 8) =
            make_float2(c_nf4_codes[b >> 4], c_nf4_codes[b & 15]);
    }
    if (CODEC == AETH_CODEC_BLOCK_DYNAMIC) {
        for (int i = threadIdx.x; i < 256 * 32; i += blockDim.x)
            *reinterpret_cast<float*>(tab.rep + (i >> 5) * 256 + 128 + (i & 31) * 4) = c_dmap_signed[i >> 5];
        for (int i = threadIdx.x; i < 256; i += blockDim.x) tab.dm[i] = c_dmap_signed[i];
        for (int i = threadIdx.x; i < 2 * kDmapLutEntries; i += blockDim.x) tab.dlut4[i] = g_dmap_lut4_s[i];
    }
    for (int b = threadIdx.x; b < 32; b += blockDim.x) tab.bucket32[b] = nf4_bucket32_entry(b);
    __syncthreads();
    const int group = threadIdx.x >> 7, tid = threadIdx.x & 127;
    const int lane = tid & 31, warp = tid >> 5;
    const uint32_t bucket_bias = smem_u32_addr(tab.bucket32) - (0x4B400000u << 2);
    const uint32_t bucket_lane = tab.bucket32[lane];
    const uint32_t rep_base = smem_u32_addr(tab.rep);
    const uint32_t byte_lane = (uint32_t)(lane & 15) * 8u, map_lane = 128u + (uint32_t)lane * 4u;
    const double gnorm = sqrt(*sq);
    float clip = (float)((double)max_norm / (gnorm + 1e-6));
    clip = clip < 1.0f ? clip : 1.0f;
    const float2 clip2 = make_float2(clip, clip), beta2 = make_float2(beta, beta), nlr2 = make_float2(-lr, -lr);
    const int64_t n_blocks = n / 2048;
    const int64_t vgrid = (int64_t)gridDim.x * kLomoGroups;
    int64_t b = (int64_t)blockIdx.x * kLomoGroups + group;
    uint4 g0 = make_uint4(0u, 0u, 0u, 0u), g1 = g0, mq = g0;
    uint2 wq = make_uint2(0u, 0u);
    float ms = 0.0f, wamax = 0.0f;
    auto fetch = [&](int64_t blk) {
        const int64_t e = blk * 2048 + tid * 16;
        g0 = __ldcs(reinterpret_cast<const uint4*>(g + e));
        g1 = __ldcs(reinterpret_cast<const uint4*>(g + e + 8));
        mq = *reinterpret_cast<const uint4*>(mom8 + e);
        wq = *reinterpret_cast<const uint2*>(wp + e / 2);
        wamax = wa[e / 64];
        ms = mom_scales[blk];
    };
    if (b < n_blocks) fetch(b);
    for (int it = 0; b < n_blocks; b += vgrid, ++it) {
        const int64_t e0 = b * 2048 + tid * 16;
        float w[16], mo[16];
        // NF4 dequant (byte table), gradient, momentum decode
        nf4_dequant_word_s(wq.x, wamax, rep_base, byte_lane, w);
        nf4_dequant_word_s(wq.y, wamax, rep_base, byte_lane, w + 8);
        const uint32_t gw[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        const uint32_t mw[4] = {mq.x, mq.y, mq.z, mq.w};
        const float cur_ms = ms;
        if (b + vgrid < n_blocks) fetch(b + vgrid);
        const float2 ms2 = make_float2(cur_ms, cur_ms);
        float am = 0.0f, aw = 0.0f;
#pragma unroll
        for (int k = 0; k < 16; k += 2) {
            const uint32_t gp = gw[k >> 1];
            const float2 gg = mul2_rn(make_float2(__uint_as_float(gp << 16), __uint_as_float(gp & 0xffff0000u)), clip2);
            const uint32_t mword = mw[k >> 2];
            const int sh = 8 * (k & 3);
            float2 m0;
            if (CODEC == AETH_CODEC_BLOCK_DYNAMIC) {
                // map entries of code bytes k % 4 and k % 4 + 1 of the word, this lane's copy
                const uint32_t kb = (uint32_t)(k & 3);
                float m_lo, m_hi;
                asm("ld.shared.f32 %0, [%1];" : "=f"(m_lo) : "r"(rep_base + prmt(mword, map_lane, 0x5504u | (kb << 4))));
                asm("ld.shared.f32 %0, [%1];"
                    : "=f"(m_hi)
                    : "r"(rep_base + prmt(mword, map_lane, 0x5504u | ((kb + 1u) << 4))));
                m0 = make_float2(m_lo, m_hi);
            } else {
                m0 = make_float2((float)(int8_t)(mword >> sh), (float)(int8_t)(mword >> (sh + 8)));
            }
            m0 = mul2_rn(m0, ms2);
            // m = fl(fl(beta m) + g clip); w = fl(w - fl(lr m))
            const float2 mm = add2_sep(mul2_rn(beta2, m0), gg);
            const float2 ww = add2_sep(make_float2(w[k], w[k + 1]), mul2_rn(mm, nlr2));
            mo[k] = mm.x;
            mo[k + 1] = mm.y;
            w[k] = ww.x;
            w[k + 1] = ww.y;
            am = fmax3_nan(am, fabsf(mm.x), fabsf(mm.y));
            aw = fmax3_nan(aw, fabsf(ww.x), fabsf(ww.y));
        }
        // NF4 block absmax over the 4 threads of the block (NaN-propagating, as the reference's max)
        aw = fmax_nan(aw, __shfl_xor_sync(0xffffffffu, aw, 1));
        aw = fmax_nan(aw, __shfl_xor_sync(0xffffffffu, aw, 2));
        const bool bad = !(aw <= 3.402823466e38f);
        const float safe = nf4_safe(aw), inv = __frcp_rn(safe);
        uint32_t pk0 = 0u, pk1 = 0u;
        float mind = 1.0f;
        pk0 = nf4_fast_word8_s(w, inv, bucket_lane, mind);  // all lanes: entries come by shuffle
        pk1 = nf4_fast_word8_s(w + 8, inv, bucket_lane, mind);
        if (bad) mind = 0.0f;
        if (mind < kNf4NearWindow32) {  // rare: exact decisions next to a boundary, or a non-finite block
            if (bad) {
                pk0 = nf4_exact_word8(w[0], w[1], w[2], w[3], w[4], w[5], w[6], w[7], safe);
                pk1 = nf4_exact_word8(w[8], w[9], w[10], w[11], w[12], w[13], w[14], w[15], safe);
            } else {
                pk0 = nf4_fix_word8(pk0, w[0], w[1], w[2], w[3], w[4], w[5], w[6], w[7], inv, safe, bucket_bias);
                pk1 = nf4_fix_word8(pk1, w[8], w[9], w[10], w[11], w[12], w[13], w[14], w[15], inv, safe,
                                    bucket_bias);
            }
        }
        *reinterpret_cast<uint2*>(wp + e0 / 2) = make_uint2(pk0, pk1);
        if ((tid & 3) == 0) wa[e0 / 64] = nf4_store_amax(aw);
        if (prequant) {
#pragma unroll
            for (int k = 0; k < 16; k += 4)
                *reinterpret_cast<float4*>(prequant + e0 + k) = make_float4(w[k], w[k + 1], w[k + 2], w[k + 3]);
        }
        // momentum block maxima over the group, NaN-propagating (canonical NaN orders
        // above +inf as unsigned bits; double-buffered slots: one barrier per block)
        const uint32_t amb = __reduce_max_sync(0xffffffffu, __float_as_uint(am));
        uint32_t* rs = red[group][it & 1];
        if (lane == 0) rs[warp] = amb;
        asm volatile("bar.sync %0, 128;" ::"r"(1 + group) : "memory");
        const uint32_t bmb = max(max(rs[0], rs[1]), max(rs[2], rs[3]));
        float bm = __uint_as_float(bmb);
        // finite and 0 or normal: every normalised value lies within 1 + 2^-23 (group-uniform)
        const bool finite = bmb < 0x7f800000u && (bmb == 0u || bmb >= 0x00800000u);
        if (!finite) {  // rare: the maximum again, ignoring NaN, as the reference's max does
            float a2 = 0.0f;
#pragma unroll
            for (int k = 0; k < 16; k += 2) a2 = fmax3(a2, fabsf(mo[k]), fabsf(mo[k + 1]));
            a2 = warp_max_nonneg(a2);
            if (lane == 0) red2[group][warp] = __float_as_uint(a2);
            asm volatile("bar.sync %0, 128;" ::"r"(1 + group) : "memory");
            bm = __uint_as_float(max(max(red2[group][0], red2[group][1]), max(red2[group][2], red2[group][3])));
        }
        uint32_t out[4] = {0u, 0u, 0u, 0u};
        if (CODEC == AETH_CODEC_BLOCK_LINEAR) {
            const float nsm = lin_scale_from_absmax(bm), linv = lin_inv(nsm);
#pragma unroll
            for (int k = 0; k < 16; ++k) out[k >> 2] |= ((uint32_t)(uint8_t)lin_encode(mo[k], linv)) << (8 * (k & 3));
            if (tid == 0) mom_scales[b] = nsm;
        } else {
            const float dinv = dyn_inv(bm);
            if (finite) {
                const float2 dinv2 = make_float2(dinv, dinv);
                const uint32_t m1 = one << 1, m8 = one << 8, m15 = one << 15;
                const uint32_t lut_adj = smem_u32_addr(tab.dlut4) - (uint32_t)(kDmapLutExpLo << kDmapLutLog2P) * 4u;
                uint32_t hp[8];  // codes of element pairs in bytes 0 and 1
#pragma unroll
                for (int k = 0; k < 16; k += 2) {
                    const float2 x2 = mul2_rn(make_float2(mo[k], mo[k + 1]), dinv2);
                    hp[k >> 1] = prmt(dmap_enc4_s(lut_adj, x2.x, m1, m8, m15), dmap_enc4_s(lut_adj, x2.y, m1, m8, m15),
                                      0x3340u);
                }
#pragma unroll
                for (int w4 = 0; w4 < 4; ++w4) out[w4] = prmt(hp[2 * w4], hp[2 * w4 + 1], 0x5410u);
            } else {
#pragma unroll
                for (int k = 0; k < 16; ++k)
                    out[k >> 2] |= dmap_encode_rare(tab.dm, __fmul_rn(mo[k], dinv)) << (8 * (k & 3));
            }
            if (tid == 0) mom_scales[b] = bm;
        }
        *reinterpret_cast<uint4*>(mom8 + e0) = make_uint4(out[0], out[1], out[2], out[3]);
    }
}

}  // namespace aeth
