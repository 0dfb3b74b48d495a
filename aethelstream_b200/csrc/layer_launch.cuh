// layer_launch.cuh -- host launchers for the grouped (whole-layer) kernels:
// projection (K4), squared norms, back-projection + NF4 write (K6).
#pragma once
#include <vector>

#include "adam.cuh"
#include "apply_tc.cuh"
#include "gemm_tc.cuh"
#include "proj_tc.cuh"

namespace aeth {

// ---------------------------------------------------------------------------
// K4
// ---------------------------------------------------------------------------
struct ProjJob {
    const void* grad;       // bf16 m x n
    const uint16_t* projT;  // bf16 r x s (s = min(m, n))
    float* racc;            // fp32 l x r
    int m, n;
    int ldr = 0;            // row stride of racc in floats (0: r); a column slice of a wider R
};

template <int BN>
int proj_grouped_launch_bn(const ProjJob* jobs, int nj, int r, cudaStream_t st) {
    // As many 32-48 KB operand stages as shared memory holds: more bytes in flight per SM.
    constexpr int STAGES = BN <= 128 ? 6 : 4;
    using L = ProjLayout<BN, STAGES>;
    static_assert(1024 + L::kTotal <= 227 * 1024, "projection kernel shared memory above the per-CTA limit");
    DeviceRuntime* rt = nullptr;
    AETH_TRY(runtime_for_current(&rt));
    ProjArgs a;
    memset(&a, 0, sizeof(a));
    a.nprob = nj;
    a.r = r;
    a.idesc_k = idesc_f16(128, BN, true, false, false);
    a.idesc_mn = idesc_f16(128, BN, true, true, false);
    // Split-K depth: the persistent CTAs take units round-robin, so the launch
    // lasts about ceil(units / SMs) units of (k-blocks + epilogue) each.  Pick
    // the k-blocks per unit (at least 8) that minimises that, counting an
    // epilogue as 2 k-blocks of work.
    int kb_target = 8;
    {
        int64_t best = -1;
        for (int kt = 8; kt <= 64; ++kt) {
            int64_t units_k = 0, per_unit = 0;
            for (int i = 0; i < nj; ++i) {
                const int l = std::max(jobs[i].m, jobs[i].n), s = std::min(jobs[i].m, jobs[i].n);
                const int kbt = (s + 63) / 64;
                int sp = (kbt + kt - 1) / kt;
                const int kpu = (kbt + sp - 1) / sp;
                sp = (kbt + kpu - 1) / kpu;
                units_k += (int64_t)((l + 127) / 128) * sp;
                per_unit = std::max<int64_t>(per_unit, kpu);
            }
            const int64_t span = (units_k + num_sms() - 1) / num_sms() * (per_unit + 2);
            if (best < 0 || span < best) { best = span; kb_target = kt; }
        }
    }
    int units = 0;
    for (int i = 0; i < nj; ++i) {
        const ProjJob& j = jobs[i];
        ProjProblem& p = a.p[i];
        const bool right = j.m >= j.n;
        const int l = right ? j.m : j.n, s = right ? j.n : j.m;
        if (right) AETH_TRY(make_tmap_16b(&p.tmA, j.grad, (uint64_t)j.n, (uint64_t)j.m, j.n, 64, 128, true));
        else AETH_TRY(make_tmap_16b(&p.tmA, j.grad, (uint64_t)j.n, (uint64_t)j.m, j.n, 64, 64, true));
        AETH_TRY(make_tmap_16b(&p.tmB, j.projT, (uint64_t)s, (uint64_t)r, s, 64, BN, true));
        AETH_TRY(make_tmap_2d(&p.tmC, j.racc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)r, (uint64_t)l,
                              j.ldr > 0 ? j.ldr : r, 32, 128, CU_TENSOR_MAP_SWIZZLE_128B));
        p.a_mn = right ? 0 : 1;
        p.kb_total = (s + 63) / 64;
        p.splits = (p.kb_total + kb_target - 1) / kb_target;
        p.kb_per_unit = (p.kb_total + p.splits - 1) / p.splits;
        p.splits = (p.kb_total + p.kb_per_unit - 1) / p.kb_per_unit;
        p.unit_begin = units;
        units += ((l + 127) / 128) * p.splits;
    }
    a.total_units = units;
    const int smem = 1024 + L::kTotal;
    auto kern = proj_grouped_kernel<BN, STAGES>;
    static bool attr_set[kMaxDevices] = {};
    int dev = 0;
    AETH_TRY(current_device(&dev));
    if (!attr_set[dev]) {
        AETH_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        attr_set[dev] = true;
    }
    const int grid = std::min(num_sms(), units);
    kern<<<grid, 192, smem, st>>>(a, rt->err_word);
    AETH_LAUNCH_CHECK();
    return AETH_OK;
}

// Projects and accumulates every job; jobs must share the rank r.  Ranks
// above 256 (one MMA's N) run as column slices of at most 256 of R, each a
// launch over its rows of projT: R[:, c0:c1] += G Q[:, c0:c1].  The gradient
// is read once per slice.
inline int proj_grouped_launch(const ProjJob* jobs, int nj, int r, cudaStream_t st) {
    if (r <= 0 || r > 1024 || r % 8 != 0) return AETH_ERR_UNSUPPORTED;
    if (r > 256) {
        if (r % 64 != 0) return AETH_ERR_UNSUPPORTED;
        for (int c0 = 0; c0 < r; c0 += 256) {
            const int w = std::min(256, r - c0);
            std::vector<ProjJob> slice(jobs, jobs + nj);
            for (ProjJob& j : slice) {
                const int s = std::min(j.m, j.n);
                j.projT += (size_t)c0 * s;
                j.racc += c0;
                j.ldr = r;
            }
            AETH_TRY(proj_grouped_launch(slice.data(), nj, w, st));
        }
        return AETH_OK;
    }
    for (int off = 0; off < nj; off += kProjMaxProblems) {
        const int cnt = std::min(kProjMaxProblems, nj - off);
        if (r <= 64) AETH_TRY(proj_grouped_launch_bn<64>(jobs + off, cnt, r, st));
        else if (r <= 128) AETH_TRY(proj_grouped_launch_bn<128>(jobs + off, cnt, r, st));
        else AETH_TRY(proj_grouped_launch_bn<256>(jobs + off, cnt, r, st));
    }
    return AETH_OK;
}

// out[i] = sum of squares of xs[i] (f64).  With clip_out (np <= kSqGroupMax)
// the same launch also writes the global clip coefficient for max_norm.
// With a clip group of several GPUs the clip is computed from the sum over
// the whole group (clip_group_total); the device epoch advances once per launch.
// Arguments of one squared-norm launch over cnt accumulators (cnt <=
// kSqGroupMax); returns the chunks per accumulator, or a negative status.
inline int sq_fill_args(const float* const* xs, const int64_t* ns, int cnt, double* out, double* partials,
                        unsigned int* ticket, float max_norm, float* clip_out, double* gnorm_out,
                        const ClipGroup* group, uint32_t* err, SqGroupArgs* a) {
    memset(a, 0, sizeof(*a));
    int64_t largest = 0;
    for (int i = 0; i < cnt; ++i) {
        a->x[i] = xs[i];
        a->n[i] = ns[i];
        largest = std::max(largest, a->n[i]);
        if ((reinterpret_cast<uintptr_t>(a->x[i]) & 15) != 0) return AETH_ERR_UNSUPPORTED;
    }
    a->np = cnt;
    a->max_norm = max_norm;
    a->clip_out = clip_out;
    a->gnorm_out = gnorm_out;
    a->out = out;
    a->partials = partials;
    a->ticket = ticket;
    a->world = 1;
    a->err = err;
    a->timeout_ns = 0;
    if (group && group->world > 1) {
        a->rank = group->rank;
        a->world = group->world;
        for (int p = 0; p < group->world; ++p) a->slots[p] = group->slots[p];
        a->epoch = group->epoch;
        a->timeout_ns = group->timeout_ns;
    }
    return sq_chunks_for(largest);
}

inline int sqnorm_group(const float* const* xs, const int64_t* ns, int np, double* out, double* partials,
                        unsigned int* ticket, float max_norm, float* clip_out, double* gnorm_out, cudaStream_t st,
                        ClipGroup* group = nullptr) {
    if (clip_out && np > kSqGroupMax) return AETH_ERR_UNSUPPORTED;
    if (group && group->world > 1 && !clip_out) return AETH_ERR_ARG;
    DeviceRuntime* rt = nullptr;
    AETH_TRY(runtime_for_current(&rt));
    for (int off = 0; off < np; off += kSqGroupMax) {
        const int cnt = std::min(kSqGroupMax, np - off);
        SqGroupArgs a;
        const int chunks = sq_fill_args(xs + off, ns + off, cnt, out + off, partials, ticket, max_norm, clip_out,
                                        gnorm_out, group, rt->err_word, &a);
        if (chunks < 0) return chunks;
        sqnorm_group_kernel<<<dim3(chunks, cnt), 256, 0, st>>>(a);
        AETH_LAUNCH_CHECK();
    }
    return AETH_OK;
}

// ---------------------------------------------------------------------------
// K6
// ---------------------------------------------------------------------------
struct ApplyJob {
    const uint16_t* X;  // m x r bf16
    const uint16_t* Y;  // n x r bf16
    uint8_t* wp;        // m x n/2
    float* wa;          // m x n/64
    int m, n;
    float lr, decay_mul;
    int has_decay;
    float* prequant;
    float* delta;
};

// The grouped kernel needs n % 256 == 0 (absmax rows a multiple of 16 bytes)
// and r % 8 == 0; the rank is the MMAs' K, taken 64 at a time.
inline bool apply_grouped_supported(int m, int n, int r) {
    return m > 0 && n > 0 && n % 256 == 0 && r > 0 && r % 8 == 0 && r <= 1024;
}

inline int apply_grouped_launch(const ApplyJob* jobs, int nj, int r, cudaStream_t st) {
    // Two operand stages: up to r = 256 a unit's MMAs take a fraction of its
    // epilogue, and the freed 48 KB hold the replicated byte table; larger
    // ranks stream more k-blocks through the same two stages.
    constexpr int STAGES = 2;
    using L = ApplyLayout<STAGES>;
    static_assert(1024 + L::kTotal <= 227 * 1024, "apply kernel shared memory above the per-CTA limit");
    DeviceRuntime* rt = nullptr;
    AETH_TRY(runtime_for_current(&rt));
    for (int off = 0; off < nj; off += kApplyMaxProblems) {
        const int cnt = std::min(kApplyMaxProblems, nj - off);
        ApplyArgs a;
        memset(&a, 0, sizeof(a));
        a.nprob = cnt;
        a.kb = (r + 63) / 64;
        a.idesc = idesc_f16(128, kApplyBN, true, false, false);
        int units = 0;
        for (int i = 0; i < cnt; ++i) {
            const ApplyJob& j = jobs[off + i];
            if (!apply_grouped_supported(j.m, j.n, r)) return AETH_ERR_UNSUPPORTED;
            ApplyProblem& p = a.p[i];
            AETH_TRY(make_tmap_16b(&p.tmX, j.X, (uint64_t)r, (uint64_t)j.m, r, 64, 128, true));
            AETH_TRY(make_tmap_16b(&p.tmY, j.Y, (uint64_t)r, (uint64_t)j.n, r, 64, kApplyBN, true));
            AETH_TRY(make_tmap_2d(&p.tmW, j.wp, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)(j.n / 2), (uint64_t)j.m,
                                  j.n / 2, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B));
            AETH_TRY(make_tmap_2d(&p.tmS, j.wa, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)(j.n / 64), (uint64_t)j.m,
                                  j.n / 64, 4, 128, CU_TENSOR_MAP_SWIZZLE_NONE));
            AETH_TRY(make_tmap_2d(&p.tmWq, j.wp, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)(j.n / 2), (uint64_t)j.m,
                                  j.n / 2, 128, 32, CU_TENSOR_MAP_SWIZZLE_128B));
            AETH_TRY(make_tmap_2d(&p.tmSq, j.wa, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)(j.n / 64), (uint64_t)j.m,
                                  j.n / 64, 4, 32, CU_TENSOR_MAP_SWIZZLE_NONE));
            p.prequant_out = j.prequant;
            p.delta_out = j.delta;
            p.m = j.m;
            p.n = j.n;
            p.n_tiles = (j.n + kApplyBN - 1) / kApplyBN;
            p.unit_begin = units;
            p.lr = j.lr;
            p.decay_mul = j.decay_mul;
            p.has_decay = j.has_decay;
            units += ((j.m + 127) / 128) * p.n_tiles;
        }
        a.total_units = units;
        const int smem = 1024 + L::kTotal;
        auto kern = apply_grouped_kernel<STAGES>;
        static bool attr_set[kMaxDevices] = {};
        int dev = 0;
        AETH_TRY(current_device(&dev));
        if (!attr_set[dev]) {
            AETH_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
            attr_set[dev] = true;
        }
        const int grid = std::min(num_sms(), units);
        kern<<<grid, kApplyThreads, smem, st>>>(a, rt->err_word);
        AETH_LAUNCH_CHECK();
    }
    return AETH_OK;
}

}  // namespace aeth
