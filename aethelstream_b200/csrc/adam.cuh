// adam.cuh -- low-rank Adam (K5), squared norms, the global clip and the
// full-rank fused Adam of doublepass_galore_apply.
#pragma once
#include "codec.cuh"
#include "common.cuh"

namespace aeth {

// ---------------------------------------------------------------------------
// REF mode: one parameter's r x r Adam step with per-tensor absmax INT8 state,
// bit-exact with galore/src/optimizer.rs:314-351 + adamw.rs:79-88,116-135 +
// quantize.rs:4-26.  One CTA; two passes separated by the absmax reduction.
//   mom/var: fp32 working buffers (the Rust struct's momentum/variance Vecs).
//   m_scale, v_scale: one device float each (in/out).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) ref_adam_kernel(const float* __restrict__ accum, int8_t* __restrict__ m8,
                                                        int8_t* __restrict__ v8, float* __restrict__ m_scale,
                                                        float* __restrict__ v_scale, float* __restrict__ mom,
                                                        float* __restrict__ var, float* __restrict__ normalized,
                                                        int64_t n, float clip_host, const float* __restrict__ clip_dev,
                                                        float b1, float b2, float eps) {
    __shared__ float red_m[32], red_v[32];
    __shared__ float s_scales[2];
    const float clip = clip_dev ? *clip_dev : clip_host;
    const float sm = *m_scale, sv = *v_scale;
    const float omb1 = __fsub_rn(1.0f, b1), omb2 = __fsub_rn(1.0f, b2);
    float am = 0.0f, av = 0.0f;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        float mo = __fmul_rn((float)m8[i], sm);
        float va = __fmul_rn((float)v8[i], sv);
        float g = accum[i];
        if (clip != 1.0f) g = __fmul_rn(g, clip);
        mo = __fadd_rn(__fmul_rn(b1, mo), __fmul_rn(omb1, g));
        va = __fadd_rn(__fmul_rn(b2, va), __fmul_rn(__fmul_rn(omb2, g), g));
        normalized[i] = __fdiv_rn(mo, __fadd_rn(__fsqrt_rn(va), eps));
        mom[i] = mo;
        var[i] = va;
        am = fmaxf(am, fabsf(mo));
        av = fmaxf(av, fabsf(va));
    }
    am = warp_max(am);
    av = warp_max(av);
    if ((threadIdx.x & 31) == 0) { red_m[threadIdx.x >> 5] = am; red_v[threadIdx.x >> 5] = av; }
    __syncthreads();
    if (threadIdx.x == 0) {
        float a = 0.0f, b = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) { a = fmaxf(a, red_m[w]); b = fmaxf(b, red_v[w]); }
        s_scales[0] = lin_scale_from_absmax(a);
        s_scales[1] = lin_scale_from_absmax(b);
    }
    __syncthreads();
    const float nsm = s_scales[0], nsv = s_scales[1];
    const float im = lin_inv(nsm), iv = lin_inv(nsv);
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        m8[i] = lin_encode(mom[i], im);
        v8[i] = lin_encode(var[i], iv);
    }
    if (threadIdx.x == 0) { *m_scale = nsm; *v_scale = nsv; }
}

// ---------------------------------------------------------------------------
// B200 mode: Adam over the l x r state with blockwise INT8 m/v.  One CTA per
// state block (grid-stride over blocks).  Pass 1 updates and tracks the block
// absmax and writes N (bf16); pass 2 recomputes the same values (bit-identical)
// and encodes them with the new block scales.  Optionally zeroes the
// accumulator (the fused zero_accum of a whole-layer step).
// ---------------------------------------------------------------------------
struct AdamB2Args {
    const float* accum;
    int8_t* m8;
    int8_t* v8;
    float* m_scales;
    float* v_scales;
    uint16_t* n_out;  // bf16 N, same l x r layout
    int64_t count;
    int block;
    int codec;        // AETH_CODEC_BLOCK_LINEAR / AETH_CODEC_BLOCK_DYNAMIC
    float clip_host;
    const float* clip_dev;
    float b1, b2, eps;
    int zero_accum;
};

__device__ __forceinline__ void b2_adam_elem(float g_raw, float clip, int8_t qm, int8_t qv, float sm, float sv,
                                             int codec, const float* dm, const float* du, float b1, float omb1,
                                             float b2, float omb2, float& mo, float& va) {
    float g = clip != 1.0f ? __fmul_rn(g_raw, clip) : g_raw;
    float m0, v0;
    if (codec == AETH_CODEC_BLOCK_LINEAR) {
        m0 = __fmul_rn((float)qm, sm);
        v0 = __fmul_rn((float)qv, sv);
    } else {
        m0 = __fmul_rn(dm[(uint8_t)qm], sm);
        v0 = __fmul_rn(du[(uint8_t)qv], sv);
    }
    mo = __fadd_rn(__fmul_rn(b1, m0), __fmul_rn(omb1, g));
    va = __fadd_rn(__fmul_rn(b2, v0), __fmul_rn(__fmul_rn(omb2, g), g));
}

__global__ void __launch_bounds__(256) b2_adam_kernel(AdamB2Args a) {
    __shared__ float dm[256], du[256];
    __shared__ float red_m[8], red_v[8];
    if (a.codec == AETH_CODEC_BLOCK_DYNAMIC) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) { dm[i] = c_dmap_signed[i]; du[i] = c_dmap_unsigned[i]; }
    }
    const float clip = a.clip_dev ? *a.clip_dev : a.clip_host;
    const float omb1 = __fsub_rn(1.0f, a.b1), omb2 = __fsub_rn(1.0f, a.b2);
    const int64_t n_blocks = (a.count + a.block - 1) / a.block;
    __syncthreads();
    for (int64_t b = blockIdx.x; b < n_blocks; b += gridDim.x) {
        const int64_t s = b * a.block, e = s + a.block < a.count ? s + a.block : a.count;
        const float sm = a.m_scales[b], sv = a.v_scales[b];
        float am = 0.0f, av = 0.0f;
        for (int64_t i = s + threadIdx.x; i < e; i += blockDim.x) {
            float mo, va;
            b2_adam_elem(a.accum[i], clip, a.m8[i], a.v8[i], sm, sv, a.codec, dm, du, a.b1, omb1, a.b2, omb2, mo, va);
            float nv = __fdiv_rn(mo, __fadd_rn(__fsqrt_rn(va), a.eps));
            a.n_out[i] = f32_to_bf16_bits(nv);
            am = fmaxf(am, fabsf(mo));
            av = fmaxf(av, fabsf(va));
        }
        am = warp_max(am);
        av = warp_max(av);
        if ((threadIdx.x & 31) == 0) { red_m[threadIdx.x >> 5] = am; red_v[threadIdx.x >> 5] = av; }
        __syncthreads();
        float bm = 0.0f, bv = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) { bm = fmaxf(bm, red_m[w]); bv = fmaxf(bv, red_v[w]); }
        float nsm, nsv, im = 0.0f, iv = 0.0f;
        if (a.codec == AETH_CODEC_BLOCK_LINEAR) {
            nsm = lin_scale_from_absmax(bm); nsv = lin_scale_from_absmax(bv);
            im = lin_inv(nsm); iv = lin_inv(nsv);
        } else {
            nsm = bm; nsv = bv;
        }
        // Every thread has read the old scales and the block's old codes for
        // its own elements; pass 2 touches only the same elements.
        for (int64_t i = s + threadIdx.x; i < e; i += blockDim.x) {
            float mo, va;
            b2_adam_elem(a.accum[i], clip, a.m8[i], a.v8[i], sm, sv, a.codec, dm, du, a.b1, omb1, a.b2, omb2, mo, va);
            if (a.codec == AETH_CODEC_BLOCK_LINEAR) {
                a.m8[i] = lin_encode(mo, im);
                a.v8[i] = lin_encode(va, iv);
            } else {
                a.m8[i] = (int8_t)(uint8_t)dmap_encode(dm, dyn_xn(mo, dyn_inv(nsm)));
                a.v8[i] = (int8_t)(uint8_t)dmap_encode(du, dyn_xn(va, dyn_inv(nsv)));
            }
            if (a.zero_accum) const_cast<float*>(a.accum)[i] = 0.0f;
        }
        __syncthreads();
        if (threadIdx.x == 0) { a.m_scales[b] = nsm; a.v_scales[b] = nsv; }
    }
}

// ---------------------------------------------------------------------------
// B200 mode, grouped: the Adam step of every parameter of a layer in one
// persistent launch.  State blocks of 2048 elements, one per 256-thread group
// iteration; thread t owns elements [8t, 8t+8) of the block, so the update,
// the block absmax and the encode run from registers in a single HBM pass:
// read R (4 B) + m, v codes (2 B), write m, v codes (2 B) + N bf16 (2 B)
// [+ zero R (4 B)] per element.  b2_adam_group_kernel runs the linear codec,
// b2_adam_dyn_kernel the dynamic map.  Element pairs go through the packed
// f32x2 helpers (mul2_rn, add2_sep), which round every lane like the scalar
// __fmul_rn / __fadd_rn.
// ---------------------------------------------------------------------------
constexpr int kAdamGroupMax = 16;

struct AdamGroupArgs {
    const float* accum[kAdamGroupMax];
    int8_t* m8[kAdamGroupMax];
    int8_t* v8[kAdamGroupMax];
    float* ms[kAdamGroupMax];
    float* vs[kAdamGroupMax];
    uint16_t* nout[kAdamGroupMax];
    int64_t count[kAdamGroupMax];
    int block_begin[kAdamGroupMax + 1];
    int np;
    int codec;
    float clip_host;
    const float* clip_dev;
    float b1, b2, eps;
    int zero_accum;
    unsigned int* work;  // [next block, CTAs done], zero between launches
    uint32_t one;        // 1 (b2_adam_dyn_kernel's run-time multipliers)
};

// ---------------------------------------------------------------------------
// Adam direction in bf16: bf16(fl(mo / fl(fl(sqrt(va)) + eps))) (adamw.rs:
// 129-131 followed by the bf16 store of N).  Fast path: hardware sqrt and
// reciprocal approximations, q' = fl(mo * rcp(fl(sqrt'(va) + eps))), within
// about ten ulp of the correctly rounded quotient q (a few ulp for each
// approximation, half an ulp per rounding).  bf16 rounding of q' and of q
// agree unless the low 16 bits of q' lie within kAdamDirGuard of the tie
// 0x8000, so those -- and tiny, infinite or NaN values -- are recomputed
// with IEEE sqrt and division.  aeth_selfcheck(AETH_SELFCHECK_ADAM_DIR)
// compares the two paths over every float bit pattern of va.
// ---------------------------------------------------------------------------
constexpr uint32_t kAdamDirGuard = 32;  // ulp, about three times the error bound

__device__ __forceinline__ float adam_dir_exact(float mo, float va, float eps) {
    return __fdiv_rn(mo, __fadd_rn(__fsqrt_rn(va), eps));
}

// Out of line, so the fast path branches around it rather than evaluating
// IEEE sqrt and division for every element under a predicate.
__device__ __noinline__ float adam_dir_exact_rare(float mo, float va, float eps) { return adam_dir_exact(mo, va, eps); }

// The .ftz forms are single hardware instructions.  They flush subnormals: a
// subnormal v has a square root below 1.1e-19, under half an ulp of any
// eps >= 1e-10 (callers use the fast path only then), so d is the same either
// way and at least eps; q is formed by an ordinary multiply.  Returns q and
// sets `flag` where the exact path is needed: q within the guard of a bf16
// tie; q nonzero below 2^-100, infinite or NaN (a NaN v or a NaN / infinite m
// gives a NaN q); or v with its sign bit set (a negative subnormal v flushes
// to -0 where IEEE sqrt gives NaN; -0 itself gives the same either way).
// Callers OR the flags of several elements and branch once.
__device__ __forceinline__ float adam_dir_q(float mo, float va, float eps, uint32_t& flag) {  // flag: 0 or 1
    float s, r;
    asm("sqrt.approx.ftz.f32 %0, %1;" : "=f"(s) : "f"(va));
    const float d = __fadd_rn(s, eps);
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d));
    const float q = __fmul_rn(mo, r);
    const uint32_t qb = __float_as_uint(q), mag = qb & 0x7fffffffu;
    const bool near_tie = ((qb & 0xffffu) + kAdamDirGuard - 0x8000u) < 2u * kAdamDirGuard;
    // mag in [1, 2^-100) wraps to the top of the range, [inf, NaN] lands just above 0x72000000
    const bool odd = (mag - 0x0d800000u) >= 0x72000000u && mag != 0u;
    flag = (uint32_t)(near_tie || odd) | (__float_as_uint(va) >> 31);
    return q;
}

__device__ __forceinline__ float adam_dir_fast(float mo, float va, float eps) {
    uint32_t flag = 0;
    const float q = adam_dir_q(mo, va, eps, flag);
    return flag ? adam_dir_exact_rare(mo, va, eps) : q;
}

// adam_dir_q's approximate quotient with its checks folded into two running
// minima over a thread's elements instead of a flag per element:
//   tie_min  = min of (bits(q) << 16) + ((kAdamDirGuard - 0x8000) << 16): below
//              2 kAdamDirGuard << 16 exactly when some q's low 16 bits lie within
//              the guard of the bf16 tie;
//   tiny_min = min of 2 bits(q) - 2: below (27 << 24) - 2 exactly when some q is
//              non-zero with magnitude below 2^-100 (q = 0 maps to the top).
// m16 = 2^16 and m2 = 2 at run time (multiply-adds on the FMA pipe).
__device__ __forceinline__ float adam_dir_q_raw(float mo, float va, float eps, uint32_t m16, uint32_t m2,
                                                uint32_t& tie_min, uint32_t& tiny_min) {
    float s, r;
    asm("sqrt.approx.ftz.f32 %0, %1;" : "=f"(s) : "f"(va));
    const float d = __fadd_rn(s, eps);
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d));
    const float q = __fmul_rn(mo, r);
    const uint32_t qb = __float_as_uint(q);
    tie_min = min(tie_min, qb * m16 + ((kAdamDirGuard - 0x8000u) << 16));
    tiny_min = min(tiny_min, qb * m2 - 2u);
    return q;
}

// True when none of a thread's approximate quotients needs the IEEE path,
// given the two minima of adam_dir_q_raw and the thread's NaN-propagating
// maxima of |mo| and |va| and minimum of va: then no element would carry
// adam_dir_q's flag.  A q near a bf16 tie or tiny and non-zero shows in the
// minima; an infinite or NaN q needs |mo| >= 2^90 (|q| <= |mo| / eps and
// eps >= 1e-10), a NaN or infinite mo, or a NaN va; a negative va shows in
// vmin (-0 passes, as adam_dir_q lets it).  A thread that fails re-checks
// each element with adam_dir_q, so the results equal the per-element flags'.
__device__ __forceinline__ bool adam_dir_fast_thread_ok(uint32_t tie_min, uint32_t tiny_min, float am, float av,
                                                        float vmin) {
    return tie_min >= (2u * kAdamDirGuard << 16) && tiny_min >= (27u << 24) - 2u &&
           __float_as_uint(am) < 0x5c800000u && __float_as_uint(av) < 0x7f800000u && !(vmin < 0.0f);
}

// Every float bit pattern as va, with mo drawn from [-0.5, 0.5) by a hash of
// the pattern and eps = 1e-8: counts bf16 disagreements of the two paths.
// The same patterns in groups of 8 consecutive ones through the per-thread
// folded checks (adam_dir_q_raw, adam_dir_fast_thread_ok, then each element's
// own check when the group fails), with mo also scaled by 2^s, s = 4 (g mod 61)
// - 120 for group g, so groups with huge, tiny, infinite or zero quotients
// occur too.
__global__ void adam_dir_selfcheck_kernel(unsigned long long* __restrict__ mismatches) {
    unsigned long long bad = 0;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    auto differ = [](uint16_t f, uint16_t e) {  // NaN results may differ in payload only
        return f != e && !((f & 0x7fffu) > 0x7f80u && (e & 0x7fffu) > 0x7f80u);
    };
    const uint32_t m16 = 1u << 16, m2 = 2u;
    for (uint64_t g = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; g < (1ull << 29); g += stride) {
        const float scale = ldexpf(1.0f, 4 * (int)(g % 61) - 120);
        float mo[8], va[8], nq[8];
        uint32_t tie_min = 0xffffffffu, tiny_min = 0xffffffffu;
        float am = 0.0f, av = 0.0f, vmin = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t i = (uint32_t)(g * 8 + j);
            va[j] = __uint_as_float(i);
            const float m = (float)((i * 2654435761u) >> 8) * 0x1p-24f - 0.5f;
            bad += differ(f32_to_bf16_bits(adam_dir_fast(m, va[j], 1e-8f)),
                          f32_to_bf16_bits(adam_dir_exact(m, va[j], 1e-8f)));
            mo[j] = __fmul_rn(m, scale);
            nq[j] = adam_dir_q_raw(mo[j], va[j], 1e-8f, m16, m2, tie_min, tiny_min);
            am = fmax3_nan(am, fabsf(mo[j]), fabsf(mo[j]));
            av = fmax3_nan(av, fabsf(va[j]), fabsf(va[j]));
            vmin = fminf(vmin, va[j]);
        }
        const bool ok = adam_dir_fast_thread_ok(tie_min, tiny_min, am, av, vmin);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            uint32_t f = 0;
            if (!ok) adam_dir_q(mo[j], va[j], 1e-8f, f);
            const float q = f ? adam_dir_exact(mo[j], va[j], 1e-8f) : nq[j];
            bad += differ(f32_to_bf16_bits(q), f32_to_bf16_bits(adam_dir_exact(mo[j], va[j], 1e-8f)));
        }
    }
    bad = warp_sum_u64(bad);
    if ((threadIdx.x & 31) == 0 && bad) atomicAdd(mismatches, bad);
}

// Linear codec.  A CTA of 512 threads is two independent 256-thread halves,
// each taking its own blocks and synchronising through its own named barrier,
// so two CTAs (32 warps) fit an SM.
__global__ void __launch_bounds__(512, 2) b2_adam_group_kernel(const __grid_constant__ AdamGroupArgs a) {
    __shared__ float red_m[2][2][8], red_v[2][2][8];  // [half][block parity][warp]: one barrier per block
    const int half = threadIdx.x >> 8, tid = threadIdx.x & 255;
    const int lane = tid & 31, warp = tid >> 5;
    const int vcta = blockIdx.x * 2 + half, vgrid = gridDim.x * 2;
    const float clip = a.clip_dev ? *a.clip_dev : a.clip_host;
    const float omb1 = __fsub_rn(1.0f, a.b1), omb2 = __fsub_rn(1.0f, a.b2);
    const float2 b1x2 = make_float2(a.b1, a.b1), b2x2 = make_float2(a.b2, a.b2);
    const float2 omb1x2 = make_float2(omb1, omb1), omb2x2 = make_float2(omb2, omb2);
    const float2 clipx2 = make_float2(clip, clip);
    const bool fast_dir = a.eps >= 1e-10f;  // the error bound and the flush-to-zero argument need it
    const int total = a.block_begin[a.np];
    // Blocks: the first 2 * gridDim.x by half index, the rest handed out by a device
    // counter (even finish times).  Each block's inputs are loaded one
    // iteration ahead, during the previous block's encode.
    __shared__ int s_next[2][2];
    int it = 0;
    int gb = vcta;
    int p = 0, b = 0;
    int64_t e0 = 0;
    bool valid = false;
    float sm = 0.0f, sv = 0.0f;
    float4 g0 = make_float4(0.f, 0.f, 0.f, 0.f), g1 = g0;
    uint2 qm = make_uint2(0u, 0u), qv = qm;
    // A half's blocks come in increasing order (its first by index, then from
    // the counter, offset by the grid), so the owning parameter only moves
    // forward: the search continues from the current one.
    auto fetch = [&](int blk) {
#pragma unroll 1
        while (p + 1 < a.np && blk >= a.block_begin[p + 1]) ++p;
        b = blk - a.block_begin[p];
        e0 = (int64_t)b * 2048 + tid * 8;
        valid = e0 < a.count[p];  // counts are multiples of 8
        sm = a.ms[p][b];
        sv = a.vs[p][b];
        if (valid) {
            g0 = *reinterpret_cast<const float4*>(a.accum[p] + e0);
            g1 = *reinterpret_cast<const float4*>(a.accum[p] + e0 + 4);
            qm = *reinterpret_cast<const uint2*>(a.m8[p] + e0);
            qv = *reinterpret_cast<const uint2*>(a.v8[p] + e0);
        }
    };
    if (gb < total) fetch(gb);
    while (gb < total) {
        const int par = it & 1;
        if (tid == 0) s_next[half][par] = (int)atomicAdd(a.work, 1u) + vgrid;
        float mo[8], va[8];
        float am = 0.0f, av = 0.0f;
        if (valid) {
            const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
            const float2 smx2 = make_float2(sm, sm), svx2 = make_float2(sv, sv);
            float nq[8];
            uint32_t dmask = fast_dir ? 0u : 0xffu;  // elements whose quotient needs the IEEE path
#pragma unroll
            for (int k = 0; k < 8; k += 2) {
                const uint32_t wm = k < 4 ? qm.x : qm.y, wv = k < 4 ? qv.x : qv.y;
                const uint32_t cm0 = (wm >> (8 * (k & 3))) & 0xffu, cm1 = (wm >> (8 * (k & 3) + 8)) & 0xffu;
                const uint32_t cv0 = (wv >> (8 * (k & 3))) & 0xffu, cv1 = (wv >> (8 * (k & 3) + 8)) & 0xffu;
                float2 m0 = make_float2((float)(int8_t)cm0, (float)(int8_t)cm1);
                float2 v0 = make_float2((float)(int8_t)cv0, (float)(int8_t)cv1);
                m0 = mul2_rn(m0, smx2);
                v0 = mul2_rn(v0, svx2);
                float2 gg = make_float2(g[k], g[k + 1]);
                if (clip != 1.0f) gg = mul2_rn(gg, clipx2);
                // products paired, sums scalar (a packed add of fresh products would be fused)
                const float2 mo2 = add2_sep(mul2_rn(b1x2, m0), mul2_rn(omb1x2, gg));
                const float2 va2 = add2_sep(mul2_rn(b2x2, v0), mul2_rn(mul2_rn(omb2x2, gg), gg));
                mo[k] = mo2.x;
                mo[k + 1] = mo2.y;
                va[k] = va2.x;
                va[k + 1] = va2.y;
                // N is stored in bf16, so the approximate quotient serves where its
                // bf16 rounding provably matches (for eps >= 1e-10, see adam_dir_q).
                uint32_t f0, f1;
                nq[k] = adam_dir_q(mo2.x, va2.x, a.eps, f0);
                nq[k + 1] = adam_dir_q(mo2.y, va2.y, a.eps, f1);
                dmask |= (f0 | (f1 << 1)) << k;
                am = fmax3(am, fabsf(mo2.x), fabsf(mo2.y));
                av = fmax3(av, fabsf(va2.x), fabsf(va2.y));
            }
            if (dmask) {  // rare (or eps < 1e-10): the flagged quotients the IEEE way
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    if (dmask & (1u << k)) nq[k] = adam_dir_exact_rare(mo[k], va[k], a.eps);
            }
            uint32_t nb[4];
#pragma unroll
            for (int k = 0; k < 8; k += 2) {
                const __nv_bfloat162 nn = __floats2bfloat162_rn(nq[k], nq[k + 1]);  // .x = nq[k] in the low half
                nb[k >> 1] = *reinterpret_cast<const uint32_t*>(&nn);
            }
            *reinterpret_cast<uint4*>(a.nout[p] + e0) = make_uint4(nb[0], nb[1], nb[2], nb[3]);
        }
        am = warp_max_nonneg(am);  // fmax3 from 0 ignores NaN: am, av >= 0 and not NaN
        av = warp_max_nonneg(av);
        if (lane == 0) { red_m[half][par][warp] = am; red_v[half][par][warp] = av; }
        // this half's 256 threads; the slots of this parity are rewritten two blocks later
        if (half)  // constant barrier ids (warp-uniform branch)
            asm volatile("bar.sync 2, 256;" ::: "memory");
        else
            asm volatile("bar.sync 1, 256;" ::: "memory");
        float bm = 0.0f, bv = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; ++w) { bm = fmaxf(bm, red_m[half][par][w]); bv = fmaxf(bv, red_v[half][par][w]); }
        const int next = s_next[half][par];
        ++it;
        // this block's coordinates, then the next block's inputs
        const int cp = p, cb = b;
        const int64_t ce0 = e0;
        const bool cvalid = valid;
        if (next < total) fetch(next);
        float nsm, nsv;
        if (cvalid) {
            uint32_t om[2] = {0u, 0u}, ov[2] = {0u, 0u};
            nsm = lin_scale_from_absmax(bm);
            nsv = lin_scale_from_absmax(bv);
            const float im = lin_inv(nsm), iv = lin_inv(nsv);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                om[k >> 2] |= ((uint32_t)(uint8_t)lin_encode(mo[k], im)) << (8 * (k & 3));
                ov[k >> 2] |= ((uint32_t)(uint8_t)lin_encode(va[k], iv)) << (8 * (k & 3));
            }
            *reinterpret_cast<uint2*>(a.m8[cp] + ce0) = make_uint2(om[0], om[1]);
            *reinterpret_cast<uint2*>(a.v8[cp] + ce0) = make_uint2(ov[0], ov[1]);
            if (a.zero_accum) {
                float* z = const_cast<float*>(a.accum[cp]) + ce0;
                *reinterpret_cast<float4*>(z) = make_float4(0.f, 0.f, 0.f, 0.f);
                *reinterpret_cast<float4*>(z + 4) = make_float4(0.f, 0.f, 0.f, 0.f);
            }
            if (tid == 0) { a.ms[cp][cb] = nsm; a.vs[cp][cb] = nsv; }
        }
        gb = next;
    }
    // The last half out resets the counters for the next launch.
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(a.work + 1, 1u) == (unsigned)vgrid - 1u) {
            a.work[0] = 0u;
            a.work[1] = 0u;
        }
    }
}

// ---------------------------------------------------------------------------
// B200 mode, dynamic codec: the grouped Adam with its CUDA-core work laid out
// for the sm_100 pipes.  The integer/logic pipe issues at half the FMA pipe's
// rate and was the busiest one (mostly the encode's index arithmetic), so:
//   * a 1024-thread CTA is four independent 256-thread groups, each taking
//     whole 2048-element blocks (8 elements per thread) from the device
//     counter, all four sharing one copy of the tables; one CTA per SM;
//   * decode: both maps in one 64 KB table whose row c holds 32 copies of
//     the signed map's entry c, then 32 of the unsigned map's (256 bytes), so
//     one byte permute of the packed codes forms a lane's bank-private offset
//     c * 256 + 4 lane (+ 128 for v);
//   * the block maxima are reduced NaN-propagating (a redux over the bit
//     patterns); a block whose maxima are finite encodes every value with the
//     flag-free bucket lookup (dmap_enc4_*, 4-byte entries: a warp's 32
//     lookups are one 128-byte wavefront when they hit distinct banks), the
//     rare other blocks reduce
//     again ignoring NaN, as the reference's max does, and encode by the
//     binary search -- the same codes and scales as b2_adam_group_kernel;
//   * the group's eight warp maxima are combined by one redux per warp.
// ---------------------------------------------------------------------------
constexpr int kAdamDynThreads = 1024;
constexpr int kAdamDynDecBytes = 256 * 256;
constexpr int kAdamDynSmem2 = kAdamDynDecBytes + (2 * kDmapLutEntries + kDmapLutUEntries) * 4 + 2 * 256 * 4;

// Barrier `id` (1..4) of one 256-thread group (group-uniform id).
__device__ __forceinline__ void group_bar(int id) { asm volatile("bar.sync %0, 256;" ::"r"(id) : "memory"); }

__device__ __forceinline__ float lds_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
    return v;
}

__global__ void __launch_bounds__(kAdamDynThreads, 1) b2_adam_dyn_kernel(const __grid_constant__ AdamGroupArgs a) {
    extern __shared__ __align__(16) uint8_t adam_smem[];
    float* dec = reinterpret_cast<float*>(adam_smem);
    uint32_t* lut_s = reinterpret_cast<uint32_t*>(adam_smem + kAdamDynDecBytes);
    uint32_t* lut_u = lut_s + 2 * kDmapLutEntries;
    float* map_s = reinterpret_cast<float*>(lut_u + kDmapLutUEntries);
    float* map_u = map_s + 256;
    __shared__ uint32_t red[4][2][2][8];  // [group][block parity][m, v][warp]: NaN-propagating maxima (bits)
    __shared__ uint32_t red2[4][2][8];    // [group][m, v][warp]: NaN-ignoring maxima (rare blocks)
    __shared__ int s_next[4][2];
    const int grp = threadIdx.x >> 8, tid = threadIdx.x & 255;
    const int lane = tid & 31, warp = tid >> 5;
    const int vcta = blockIdx.x * 4 + grp, vgrid = gridDim.x * 4;
    for (int i = threadIdx.x; i < 256 * 64; i += blockDim.x)
        dec[i] = (i & 63) < 32 ? c_dmap_signed[i >> 6] : c_dmap_unsigned[i >> 6];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
        map_s[i] = c_dmap_signed[i];
        map_u[i] = c_dmap_unsigned[i];
    }
    for (int i = threadIdx.x; i < 2 * kDmapLutEntries; i += blockDim.x) lut_s[i] = g_dmap_lut4_s[i];
    for (int i = threadIdx.x; i < kDmapLutUEntries; i += blockDim.x) lut_u[i] = g_dmap_lut4_u[i];
    __syncthreads();
    // run-time powers of two: the products below stay multiplies (FMA pipe)
    const uint32_t one = a.one;
    const uint32_t m1 = one << 1, m8 = one << 8, m15 = one << 15, m16 = one << 16;
    const uint32_t dec_base = smem_u32_addr(dec), off_m = (uint32_t)lane * 4u, off_v = off_m + 128u;
    const uint32_t lut_s_adj = smem_u32_addr(lut_s) - (uint32_t)(kDmapLutExpLo << kDmapLutLog2P) * 4u;
    const uint32_t lut_u_adj = smem_u32_addr(lut_u) - (uint32_t)(kDmapLutExpLo << kDmapLutULog2P) * 4u;
    const float clip = a.clip_dev ? *a.clip_dev : a.clip_host;
    const float omb1 = __fsub_rn(1.0f, a.b1), omb2 = __fsub_rn(1.0f, a.b2);
    const float2 b1x2 = make_float2(a.b1, a.b1), b2x2 = make_float2(a.b2, a.b2);
    const float2 omb1x2 = make_float2(omb1, omb1), omb2x2 = make_float2(omb2, omb2);
    const float2 clipx2 = make_float2(clip, clip);
    const bool fast_dir = a.eps >= 1e-10f;  // the error bound and the flush-to-zero argument need it
    const int total = a.block_begin[a.np];
    int it = 0;
    int gb = vcta;
    int p = 0, b = 0;
    int64_t e0 = 0;
    bool valid = false;
    float sm = 0.0f, sv = 0.0f;
    float4 g0 = make_float4(0.f, 0.f, 0.f, 0.f), g1 = g0;
    uint2 qm = make_uint2(0u, 0u), qv = qm;
    // a group's blocks come in increasing order, so the owning parameter only moves forward
    auto fetch = [&](int blk) {
#pragma unroll 1
        while (p + 1 < a.np && blk >= a.block_begin[p + 1]) ++p;
        b = blk - a.block_begin[p];
        e0 = (int64_t)b * 2048 + tid * 8;
        valid = e0 < a.count[p];  // counts are multiples of 8
        sm = a.ms[p][b];
        sv = a.vs[p][b];
        if (valid) {
            g0 = *reinterpret_cast<const float4*>(a.accum[p] + e0);
            g1 = *reinterpret_cast<const float4*>(a.accum[p] + e0 + 4);
            qm = *reinterpret_cast<const uint2*>(a.m8[p] + e0);
            qv = *reinterpret_cast<const uint2*>(a.v8[p] + e0);
        }
    };
    if (gb < total) fetch(gb);
    while (gb < total) {
        const int par = it & 1;
        if (tid == 0) s_next[grp][par] = (int)atomicAdd(a.work, 1u) + vgrid;
        float mo[8], va[8];
        float am = 0.0f, av = 0.0f;
        if (valid) {
            const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
            const float2 smx2 = make_float2(sm, sm), svx2 = make_float2(sv, sv);
            float nq[8];
            // the approximate quotients' checks, folded per thread (adam_dir_fast_thread_ok)
            uint32_t tie_min = 0xffffffffu, tiny_min = 0xffffffffu;
            float vmin = 0.0f;
#pragma unroll
            for (int k = 0; k < 8; k += 2) {
                const uint32_t wm = k < 4 ? qm.x : qm.y, wv = k < 4 ? qv.x : qv.y;
                const uint32_t s0 = 0x5504u | ((uint32_t)(k & 3) << 4), s1 = s0 + 0x10u;  // byte k & 3, (k & 3) + 1
                float2 m0 = make_float2(lds_f32(dec_base + prmt(wm, off_m, s0)), lds_f32(dec_base + prmt(wm, off_m, s1)));
                float2 v0 = make_float2(lds_f32(dec_base + prmt(wv, off_v, s0)), lds_f32(dec_base + prmt(wv, off_v, s1)));
                m0 = mul2_rn(m0, smx2);
                v0 = mul2_rn(v0, svx2);
                float2 gg = make_float2(g[k], g[k + 1]);
                if (clip != 1.0f) gg = mul2_rn(gg, clipx2);
                // products paired, sums scalar (a packed add of fresh products would be fused)
                const float2 mo2 = add2_sep(mul2_rn(b1x2, m0), mul2_rn(omb1x2, gg));
                const float2 va2 = add2_sep(mul2_rn(b2x2, v0), mul2_rn(mul2_rn(omb2x2, gg), gg));
                mo[k] = mo2.x;
                mo[k + 1] = mo2.y;
                va[k] = va2.x;
                va[k + 1] = va2.y;
                nq[k] = adam_dir_q_raw(mo2.x, va2.x, a.eps, m16, m1, tie_min, tiny_min);
                nq[k + 1] = adam_dir_q_raw(mo2.y, va2.y, a.eps, m16, m1, tie_min, tiny_min);
                am = fmax3_nan(am, fabsf(mo2.x), fabsf(mo2.y));
                av = fmax3_nan(av, fabsf(va2.x), fabsf(va2.y));
                vmin = fmin3(vmin, va2.x, va2.y);
            }
            if (!fast_dir || !adam_dir_fast_thread_ok(tie_min, tiny_min, am, av, vmin)) {
                // rare (or eps < 1e-10): each element's own check, the flagged ones the IEEE way
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    uint32_t f;
                    adam_dir_q(mo[k], va[k], a.eps, f);
                    if (f || !fast_dir) nq[k] = adam_dir_exact_rare(mo[k], va[k], a.eps);
                }
            }
            uint32_t nb[4];
#pragma unroll
            for (int k = 0; k < 8; k += 2) {
                const __nv_bfloat162 nn = __floats2bfloat162_rn(nq[k], nq[k + 1]);  // .x = nq[k] in the low half
                nb[k >> 1] = *reinterpret_cast<const uint32_t*>(&nn);
            }
            *reinterpret_cast<uint4*>(a.nout[p] + e0) = make_uint4(nb[0], nb[1], nb[2], nb[3]);
        }
        // non-negative or NaN (canonical 0x7fffffff): NaN-propagating maxima as unsigned bit patterns
        const uint32_t amb = __reduce_max_sync(0xffffffffu, __float_as_uint(am));
        const uint32_t avb = __reduce_max_sync(0xffffffffu, __float_as_uint(av));
        if (lane == 0) { red[grp][par][0][warp] = amb; red[grp][par][1][warp] = avb; }
        group_bar(1 + grp);  // this group's 256 threads; the parity's slots are rewritten two blocks later
        const uint32_t bmb = __reduce_max_sync(0xffffffffu, lane < 8 ? red[grp][par][0][lane] : 0u);
        const uint32_t bvb = __reduce_max_sync(0xffffffffu, lane < 8 ? red[grp][par][1][lane] : 0u);
        const int next = s_next[grp][par];
        ++it;
        const int cp = p, cb = b;
        const int64_t ce0 = e0;
        const bool cvalid = valid;
        if (next < total) fetch(next);
        // group-uniform: finite maxima that are 0 or normal, so 1 / max is finite
        // and every normalised value lies within 1 + 2^-23
        const bool finite = bmb < 0x7f800000u && bvb < 0x7f800000u && (bmb == 0u || bmb >= 0x00800000u) &&
                            (bvb == 0u || bvb >= 0x00800000u);
        float nsm = __uint_as_float(bmb), nsv = __uint_as_float(bvb);
        if (!finite) {
            // rare: a NaN or an infinity in the block -- the maxima again, ignoring NaN
            float am2 = 0.0f, av2 = 0.0f;
            if (cvalid) {
#pragma unroll
                for (int k = 0; k < 8; k += 2) {
                    am2 = fmax3(am2, fabsf(mo[k]), fabsf(mo[k + 1]));
                    av2 = fmax3(av2, fabsf(va[k]), fabsf(va[k + 1]));
                }
            }
            am2 = warp_max_nonneg(am2);
            av2 = warp_max_nonneg(av2);
            if (lane == 0) { red2[grp][0][warp] = __float_as_uint(am2); red2[grp][1][warp] = __float_as_uint(av2); }
            group_bar(1 + grp);
            nsm = __uint_as_float(__reduce_max_sync(0xffffffffu, lane < 8 ? red2[grp][0][lane] : 0u));
            nsv = __uint_as_float(__reduce_max_sync(0xffffffffu, lane < 8 ? red2[grp][1][lane] : 0u));
        }
        if (cvalid) {
            const float im = dyn_inv(nsm), iv = dyn_inv(nsv);
            uint32_t om[2] = {0u, 0u}, ov[2] = {0u, 0u};
            if (finite) {
                const float2 imx2 = make_float2(im, im), ivx2 = make_float2(iv, iv);
                uint32_t hm[4], hv[4];  // codes of element pairs in bytes 0 and 1
#pragma unroll
                for (int k = 0; k < 8; k += 2) {
                    const float2 m2 = mul2_rn(make_float2(mo[k], mo[k + 1]), imx2);  // dyn_xn, paired
                    const float2 v2 = mul2_rn(make_float2(va[k], va[k + 1]), ivx2);
                    hm[k >> 1] = prmt(dmap_enc4_s(lut_s_adj, m2.x, m1, m8, m15), dmap_enc4_s(lut_s_adj, m2.y, m1, m8, m15),
                                      0x3340u);
                    hv[k >> 1] = prmt(dmap_enc4_u(lut_u_adj, v2.x, m8, m16), dmap_enc4_u(lut_u_adj, v2.y, m8, m16), 0x3340u);
                }
                om[0] = prmt(hm[0], hm[1], 0x5410u);
                om[1] = prmt(hm[2], hm[3], 0x5410u);
                ov[0] = prmt(hv[0], hv[1], 0x5410u);
                ov[1] = prmt(hv[2], hv[3], 0x5410u);
            } else {
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    om[k >> 2] |= dmap_encode_rare(map_s, __fmul_rn(mo[k], im)) << (8 * (k & 3));
                    ov[k >> 2] |= dmap_encode_rare(map_u, __fmul_rn(va[k], iv)) << (8 * (k & 3));
                }
            }
            *reinterpret_cast<uint2*>(a.m8[cp] + ce0) = make_uint2(om[0], om[1]);
            *reinterpret_cast<uint2*>(a.v8[cp] + ce0) = make_uint2(ov[0], ov[1]);
            if (a.zero_accum) {
                float* z = const_cast<float*>(a.accum[cp]) + ce0;
                *reinterpret_cast<float4*>(z) = make_float4(0.f, 0.f, 0.f, 0.f);
                *reinterpret_cast<float4*>(z + 4) = make_float4(0.f, 0.f, 0.f, 0.f);
            }
            if (tid == 0) { a.ms[cp][cb] = nsm; a.vs[cp][cb] = nsv; }
        }
        gb = next;
    }
    // The last group out resets the counters for the next launch.
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(a.work + 1, 1u) == (unsigned)vgrid - 1u) {
            a.work[0] = 0u;
            a.work[1] = 0u;
        }
    }
}

// ---------------------------------------------------------------------------
// Squared Frobenius norm in f64 (adamw.rs:99-104).  Deterministic: fixed grid
// of partial sums, then an ordered final sum.
// ---------------------------------------------------------------------------
constexpr int kSqPartials = 256;

__global__ void __launch_bounds__(256) sqnorm_partial_kernel(const float* __restrict__ x, int64_t n,
                                                             double* __restrict__ partials) {
    __shared__ double red[8];
    double s = 0.0;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        double v = (double)x[i];
        s += v * v;
    }
    s = warp_sum_d(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
        partials[blockIdx.x] = t;
    }
}

__global__ void sqnorm_final_kernel(const double* __restrict__ partials, int np, double* __restrict__ out) {
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        double t = 0.0;
        for (int i = 0; i < np; ++i) t += partials[i];
        *out = t;
    }
}

// hook.rs:184-187: clip = min(1, (max_norm / (sqrt(sum) + 1e-6)) as f32).
__global__ void clip_coeff_kernel(const double* __restrict__ sq, int n, float max_norm, float* __restrict__ clip_out,
                                  double* __restrict__ gnorm_out) {
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        double t = 0.0;
        for (int i = 0; i < n; ++i) t += sq[i];
        double gnorm = sqrt(t);
        float c = (float)((double)max_norm / (gnorm + 1e-6));
        *clip_out = c < 1.0f ? c : 1.0f;
        if (gnorm_out) *gnorm_out = gnorm;
    }
}

// ---------------------------------------------------------------------------
// Full-rank fused Adam (doublepass_galore_apply; StandardAdamW arithmetic of
// standard_adamw.rs:84-114 with optional bias correction).
// ---------------------------------------------------------------------------
__global__ void full_adam_kernel(float* __restrict__ param, const float* __restrict__ grad, float* __restrict__ m,
                                 float* __restrict__ v, int64_t n, float clip, float b1, float b2, float eps, float lr,
                                 int bias_correct, float bc1, float bc2) {
    const float omb1 = __fsub_rn(1.0f, b1), omb2 = __fsub_rn(1.0f, b2);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float gs = __fmul_rn(grad[i], clip);
        float mo = __fadd_rn(__fmul_rn(b1, m[i]), __fmul_rn(omb1, gs));
        float va = __fadd_rn(__fmul_rn(b2, v[i]), __fmul_rn(__fmul_rn(omb2, gs), gs));
        m[i] = mo;
        v[i] = va;
        float mh = mo, vh = va;
        if (bias_correct) { mh = __fdiv_rn(mh, bc1); vh = __fdiv_rn(vh, bc2); }
        float d = __fdiv_rn(__fmul_rn(lr, mh), __fadd_rn(__fsqrt_rn(vh), eps));
        param[i] = __fsub_rn(param[i], d);
    }
}

}  // namespace aeth
