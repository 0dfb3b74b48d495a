// aeth_galore.cu -- libaeth_galore: the C ABI of include/aeth_galore.h.
//
// One translation unit (the kernels live in the included .cuh files) so the
// __constant__ tables exist once per library.  Reference paths are relative
// to the reference project's aethelStream/ directory.
#include <math.h>
#include <string.h>

#include <algorithm>
#include <array>
#include <mutex>
#include <string>
#include <vector>

#include "adam.cuh"
#include "codec.cuh"
#include "common.cuh"
#include "gemm_simt.cuh"
#include "gemm_tc.cuh"
#include "layer_launch.cuh"
#include "small_rank.cuh"
#include "split_gemm.cuh"
#include "lomo.cuh"
#include "nf4.cuh"
#include "rsvd.cuh"
#include "state_file.h"
#include "stream_decode.cuh"

using namespace aeth;

// ===========================================================================
// Host helpers
// ===========================================================================
namespace aeth {

// Dynamic 8-bit map (Dettmers et al. 2021 dynamic tree quantisation): after
// the optional sign bit, E = 0..6 leading zero bits select the decade 10^-E,
// an indicator bit follows, and the remaining F bits (6-E signed, 7-E
// unsigned) index the centres of 2^F equal bins over [0.1, 1].  Plus 0 and 1.
// Sorted ascending; a code is an index into the table.
int build_dynamic_map(int is_signed, float out[256]) {
    static const double decade[7] = {1.0, 1e-1, 1e-2, 1e-3, 1e-4, 1e-5, 1e-6};
    std::vector<float> v;
    v.reserve(256);
    for (int e = 0; e < 7; ++e) {
        int fbits = (is_signed ? 6 : 7) - e;
        int levels = 1 << fbits;
        for (int j = 0; j < levels; ++j) {
            double f = 0.1 + 0.9 * ((double)j + 0.5) / (double)levels;
            v.push_back((float)(decade[e] * f));
            if (is_signed) v.push_back((float)(-decade[e] * f));
        }
    }
    v.push_back(0.0f);
    v.push_back(1.0f);
    if (v.size() != 256) return AETH_ERR_CONFIG;
    std::sort(v.begin(), v.end());
    memcpy(out, v.data(), sizeof(float) * 256);
    return AETH_OK;
}

// init_random_projection (galore/src/optimizer.rs:419-448): xorshift64
// uniforms in [-0.5, 0.5) then modified Gram-Schmidt in f32.  One-time
// initialisation at create(); the step path never calls it.
static void init_random_projection_host(int rows, int cols, uint32_t seed, float* data) {
    uint64_t s = (uint64_t)seed + 1;
    for (int64_t i = 0; i < (int64_t)rows * cols; ++i) {
        s ^= s << 13;
        s ^= s >> 7;
        s ^= s << 17;
        data[i] = ((float)(s >> 40) / (float)(1u << 24)) - 0.5f;
    }
    for (int j = 0; j < cols; ++j) {
        for (int i = 0; i < j; ++i) {
            float dot = 0.0f;
            for (int r = 0; r < rows; ++r) {
                volatile float prod = data[(int64_t)r * cols + i] * data[(int64_t)r * cols + j];
                dot = dot + prod;
            }
            for (int r = 0; r < rows; ++r) {
                volatile float prod = dot * data[(int64_t)r * cols + i];
                data[(int64_t)r * cols + j] = data[(int64_t)r * cols + j] - prod;
            }
        }
        float norm = 0.0f;
        for (int r = 0; r < rows; ++r) {
            volatile float prod = data[(int64_t)r * cols + j] * data[(int64_t)r * cols + j];
            norm = norm + prod;
        }
        norm = sqrtf(fmaxf(norm, 1e-12f));
        for (int r = 0; r < rows; ++r) data[(int64_t)r * cols + j] /= norm;
    }
}

// LayerRankConfig::rank_for_param (galore/src/layer_rank.rs:32-40).
static int rank_for_param(const aeth_galore_config& c, const char* name, int m, int n) {
    int base = c.default_rank;
    std::string s = name ? name : "";
    if (s == "d_wq" || s == "d_wk" || s == "d_wv" || s == "d_wo") base = c.attn_rank;
    else if (s == "d_wg" || s == "d_wu" || s == "d_wd") base = c.mlp_rank;
    else if (s == "d_rms1_w" || s == "d_rms2_w") base = c.vector_rank;
    int mm = m < 1 ? 1 : m, nn = n < 1 ? 1 : n;
    int v = base < mm ? base : mm;
    v = v < nn ? v : nn;
    return v < 1 ? 1 : v;
}

static uint16_t host_f32_to_bf16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
    x += 0x7fffu + ((x >> 16) & 1u);
    return (uint16_t)(x >> 16);
}

// Projector conversion: fp32 s x r -> bf16 proj (s x r) and projT (r x s).
__global__ void proj_to_bf16_kernel(const float* __restrict__ p, int s, int r, uint16_t* __restrict__ proj,
                                    uint16_t* __restrict__ projT) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (int64_t)s * r; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t row = i / r, col = i % r;
        uint16_t b = f32_to_bf16_bits(p[i]);
        proj[i] = b;
        projT[col * s + row] = b;
    }
}

__global__ void bf16_to_f32_kernel(const uint16_t* __restrict__ x, int64_t n, float* __restrict__ y) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = bf16_bits_to_f32(x[i]);
}

__global__ void to_bf16_kernel(const void* __restrict__ x, int dtype, int64_t n, uint16_t* __restrict__ y) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = f32_to_bf16_bits(load_as_f32(x, i, dtype));
}

// Exact bf16 split of an fp32 or f16 gradient for the tensor-core projection:
// x = hi + lo (+ lo2), each term bf16 (RNE of the remainder so far), so the
// terms hold all 24 (fp32) or 11 (f16) significant bits and their products
// with the bf16 projector are exact.  The terms are stacked along the
// contraction dimension -- right side (m >= n, contraction over columns):
// row i of the output is [hi(i, :) | lo(i, :) | lo2(i, :)] (m x nsplit*n);
// left side (contraction over rows): the m x n blocks hi, lo, lo2 one below
// the other (nsplit*m x n) -- so one projection with the contraction
// nsplit times longer, against the projector repeated nsplit times, adds the
// terms' contributions.  A non-finite x keeps only hi (inf / NaN as in the
// bf16 path).  Eight elements per thread, 16-byte stores.
__global__ void grad_split_kernel(const void* __restrict__ g, int dtype, int64_t m, int64_t n, int nsplit, int right,
                                  uint16_t* __restrict__ out) {
    const int64_t total8 = m * n / 8;
    for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < total8; v += (int64_t)gridDim.x * blockDim.x) {
        const int64_t e0 = v * 8;
        float x[8];
        if (dtype == AETH_DTYPE_F32) {
            const float4 a = reinterpret_cast<const float4*>(g)[2 * v];
            const float4 b = reinterpret_cast<const float4*>(g)[2 * v + 1];
            x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
        } else {
            const uint4 a = reinterpret_cast<const uint4*>(g)[v];
            const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                x[2 * k] = __half2float(__ushort_as_half((unsigned short)(w[k] & 0xffffu)));
                x[2 * k + 1] = __half2float(__ushort_as_half((unsigned short)(w[k] >> 16)));
            }
        }
        const int64_t i = e0 / n, j = e0 % n;  // n % 8 == 0: the 8 elements share a row
#pragma unroll 1
        for (int t = 0; t < nsplit; ++t) {
            uint32_t packed[4];
#pragma unroll
            for (int k = 0; k < 8; k += 2) {
                uint16_t b[2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const float r = x[k + h];
                    const uint16_t q = f32_to_bf16_bits(r);
                    const bool finite = fabsf(r) <= 3.402823466e38f;
                    b[h] = (t == 0 || finite) ? q : (uint16_t)0;
                    x[k + h] = finite ? __fsub_rn(r, bf16_bits_to_f32(q)) : 0.0f;  // exact remainder
                }
                packed[k / 2] = (uint32_t)b[0] | ((uint32_t)b[1] << 16);
            }
            const int64_t o = right ? (i * nsplit + t) * n + j : ((int64_t)t * m + i) * n + j;
            *reinterpret_cast<uint4*>(out + o) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
        }
    }
}

__global__ void fill_f32_kernel(float* __restrict__ x, int64_t n, float v) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) x[i] = v;
}

// Dense delta applied to an NF4 weight (REF mode with an NF4 weight):
// w = dequant(w) - delta, requantised.  One thread per 64-element block.
__global__ void nf4_apply_delta_kernel(uint8_t* __restrict__ wp, float* __restrict__ wa, const float* __restrict__ delta,
                                       int64_t n_blocks, float* __restrict__ prequant) {
    __shared__ Nf4Tables tab;
    nf4_tables_init(&tab, threadIdx.x, blockDim.x);
    __syncthreads();
    for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < n_blocks; b += (int64_t)gridDim.x * blockDim.x) {
        uint8_t* p = wp + b * 32;
        uint32_t q[8];
        for (int k = 0; k < 8; ++k) q[k] = reinterpret_cast<uint32_t*>(p)[k];
        float w[64];
        float am0 = wa[b];
        for (int k = 0; k < 8; ++k) nf4_dequant_word(q[k], am0, tab.byte_lut, w + 8 * k);
        float amax = 0.0f;
        for (int i = 0; i < 64; ++i) {
            w[i] = __fsub_rn(w[i], delta[b * 64 + i]);
            amax = fmax_nan(amax, fabsf(w[i]));  // a NaN weight makes the block's absmax NaN, as the reference's max
            if (prequant) prequant[b * 64 + i] = w[i];
        }
        uint32_t pk[8];
        nf4_quant_regs<64>(w, amax, tab.bucket, pk);
        for (int k = 0; k < 8; ++k) reinterpret_cast<uint32_t*>(p)[k] = pk[k];
        wa[b] = nf4_store_amax(amax);
    }
}

// Generic f16/bf16/f32 GEMM for shapes TMA cannot describe (unaligned row
// pitch): one thread per output, fp32 accumulation in increasing k.
__global__ void simt_gemm_any_kernel(const void* A, int adt, int64_t sai, int64_t sak, const void* B, int bdt,
                                     int64_t sbk, int64_t sbj, void* C, int cdt, int64_t ldc, int M, int N, int K) {
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < (int64_t)M * N; t += (int64_t)gridDim.x * blockDim.x) {
        int i = (int)(t / N), j = (int)(t % N);
        float s = 0.0f;
        for (int k = 0; k < K; ++k)
            s = __fadd_rn(s, __fmul_rn(load_as_f32(A, i * sai + k * sak, adt), load_as_f32(B, k * sbk + j * sbj, bdt)));
        int64_t o = (int64_t)i * ldc + j;
        if (cdt == AETH_DTYPE_F32) static_cast<float*>(C)[o] = s;
        else if (cdt == AETH_DTYPE_F16) static_cast<__half*>(C)[o] = __float2half_rn(s);
        else static_cast<__nv_bfloat16*>(C)[o] = __float2bfloat16_rn(s);
    }
}

// ---------------------------------------------------------------------------
// tcgen05 GEMM dispatch on (A major, B major, N width).
// ---------------------------------------------------------------------------
template <bool A_MN, bool B_MN, class Epi>
static int tc_gemm(TcOperand A, TcOperand B, int M, int N, int K, bool bf16, const Epi& epi, cudaStream_t st) {
    if (N <= 64) return tc_gemm_launch<64, 4, A_MN, B_MN>(A, B, M, N, K, bf16, epi, st);
    if (N <= 128) return tc_gemm_launch<128, 4, A_MN, B_MN>(A, B, M, N, K, bf16, epi, st);
    return tc_gemm_launch<256, 4, A_MN, B_MN>(A, B, M, N, K, bf16, epi, st);
}

}  // namespace aeth

// ===========================================================================
// Context
// ===========================================================================
struct Param {
    uint32_t layer = 0;
    std::string name;
    int m = 0, n = 0, r = 0;
    int side = 0;  // 0 two-sided (REF), 1 left, 2 right
    int64_t state_elems = 0, state_blocks = 0;
    // REF
    float* P = nullptr;
    float* Q = nullptr;
    float* mom = nullptr;
    float* var = nullptr;
    float* normalized = nullptr;
    float* temp = nullptr;
    float* gtmp = nullptr;
    float* dtmp = nullptr;
    // shared
    float* accum = nullptr;
    int8_t* m8 = nullptr;
    int8_t* v8 = nullptr;
    float* mscale = nullptr;
    float* vscale = nullptr;
    // B200
    uint16_t* proj = nullptr;
    uint16_t* projT = nullptr;
    uint16_t* nbuf = nullptr;
    // fp32 / f16 gradients: projT repeated ksplit times along the contraction
    // (r x ksplit*s), matching the stacked bf16 terms of grad_split_kernel
    uint16_t* projTk = nullptr;
    int ksplit = 0;
    // subspace refresh: full gradient captured at refresh steps (m x n f32, lazy)
    float* capture = nullptr;
    bool captured = false;
    // streamed refresh (aeth_galore_refresh_layer): the new bf16 projector of
    // the parameter's side, installed by the next notify_step
    uint16_t* pend_proj = nullptr;
    uint16_t* pend_projT = nullptr;
    bool pending = false;
};

struct aeth_galore_ctx {
    aeth_galore_config cfg;
    int device = 0;
    uint64_t step = 0;
    std::vector<Param> params;
    double* sq_slots = nullptr;  // one per parameter
    double* sq_step = nullptr;   // contiguous slots for aeth_galore_step
    double* partials = nullptr;  // kSqPartials
    float* clip_dev = nullptr;
    double* gnorm_dev = nullptr;
    unsigned int* sq_ticket = nullptr;  // sqnorm_group's completion counter, zero between launches
    unsigned int* work = nullptr;       // b2_adam_group_kernel's block counters, zero between launches
    uint64_t* clip_epoch = nullptr;     // clip group's exchange counter (device; zeroed on joining)
    uint64_t version = 0;               // completed subspace refreshes (optimizer_version)
    // stacked bf16 terms of one fp32 / f16 gradient (grad_split_kernel), shared
    // by the parameters: their projections run one after another on the stream
    uint16_t* gsplit = nullptr;
    int64_t gsplit_elems = 0;
    // REF mode on the tensor cores (config.ref_gemm): the bf16 terms of one
    // product's operands, shared by the parameters (one stream)
    uint16_t* rsplit = nullptr;
    // global clip over several GPUs through peer memory (aeth_galore_set_clip_group)
    ClipGroup group;
    PeerSlot* own_slots = nullptr;      // 2 x world entries, cudaMalloc'd (exported by IPC handle)
    int own_slots_world = 0;
    std::vector<void*> peer_maps;       // IPC mappings of the other ranks' slots
    std::vector<cudaStream_t> side_streams;  // aeth_galore_refresh_layer's concurrent refreshes
    std::vector<void*> allocs;
    // aeth_galore_set_phase_timing: events at the phase boundaries of every
    // step, projection and finishing call
    bool phase_timing = false;
    struct PhaseRecord {
        std::vector<cudaEvent_t> ev;  // boundaries; interval k belongs to phase[k]
        std::vector<int> phase;
        int steps = 0;                // 1 for a call that ends a step
    };
    std::vector<PhaseRecord> phase_pending;
    std::vector<cudaEvent_t> event_pool;
};

namespace {

// Phase-boundary events of one call (aeth_galore_step, project_layer or
// finish_step); the events go back to the pool unless the call finished and
// committed them.
struct PhaseMarks {
    aeth_galore_ctx* c = nullptr;
    aeth_galore_ctx::PhaseRecord rec;
    bool committed = false;
    int begin(aeth_galore_ctx* ctx) {
        if (ctx->phase_timing) c = ctx;
        return AETH_OK;
    }
    // A boundary; the interval that it closes (if any) counts for `phase`,
    // the one it opens for the phase given to the next mark.
    int mark(cudaStream_t st, int phase_after) {
        if (!c) return AETH_OK;
        cudaEvent_t e = nullptr;
        if (c->event_pool.empty()) {
            AETH_CUDA(cudaEventCreate(&e));
        } else {
            e = c->event_pool.back();
            c->event_pool.pop_back();
        }
        rec.ev.push_back(e);
        rec.phase.push_back(phase_after);
        AETH_CUDA(cudaEventRecord(e, st));
        return AETH_OK;
    }
    void commit(int steps) {
        if (c) {
            rec.steps = steps;
            c->phase_pending.push_back(std::move(rec));
        }
        committed = true;
    }
    ~PhaseMarks() {
        if (c && !committed)
            for (cudaEvent_t e : rec.ev) c->event_pool.push_back(e);
    }
};

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

template <class T>
int ctx_alloc(aeth_galore_ctx* c, T** p, int64_t count) {
    void* v = nullptr;
    if (count <= 0) count = 1;
    AETH_CUDA(cudaMalloc(&v, (size_t)count * sizeof(T)));
    c->allocs.push_back(v);
    *p = static_cast<T*>(v);
    return AETH_OK;
}

// Frees a buffer that ctx_alloc made.
void ctx_free(aeth_galore_ctx* c, void* p) {
    if (!p) return;
    auto it = std::find(c->allocs.begin(), c->allocs.end(), p);
    if (it != c->allocs.end()) c->allocs.erase(it);
    cudaFree(p);
}

int reset_state(aeth_galore_ctx* c, Param& p, cudaStream_t st) {
    AETH_CUDA(cudaMemsetAsync(p.m8, 0, p.state_elems, st));
    AETH_CUDA(cudaMemsetAsync(p.v8, 0, p.state_elems, st));
    AETH_CUDA(cudaMemsetAsync(p.accum, 0, p.state_elems * sizeof(float), st));
    // LowRankAdamState::new + quantize_to_ram (adamw.rs:65-76): scale 1.0.
    float init = c->cfg.state_codec == AETH_CODEC_BLOCK_DYNAMIC ? 0.0f : 1.0f;
    fill_f32_kernel<<<grid_for(p.state_blocks, 256), 256, 0, st>>>(p.mscale, p.state_blocks, init);
    fill_f32_kernel<<<grid_for(p.state_blocks, 256), 256, 0, st>>>(p.vscale, p.state_blocks, init);
    AETH_LAUNCH_CHECK();
    return AETH_OK;
}

int check_idx(const aeth_galore_ctx* c, int idx) {
    if (!c) return AETH_ERR_ARG;
    if (idx < 0 || idx >= (int)c->params.size()) return AETH_ERR_NOT_FOUND;
    return AETH_OK;
}

int sqnorm_into(aeth_galore_ctx* c, Param& p, double* out_dev, cudaStream_t st) {
    sqnorm_partial_kernel<<<kSqPartials, 256, 0, st>>>(p.accum, p.state_elems, c->partials);
    sqnorm_final_kernel<<<1, 32, 0, st>>>(c->partials, kSqPartials, out_dev);
    AETH_LAUNCH_CHECK();
    return AETH_OK;
}

// ---- REF mode -------------------------------------------------------------
// Whether REF mode's products of this parameter run on the tensor cores
// (config.ref_gemm; every pitch a multiple of 8 elements for TMA).
bool ref_split(const aeth_galore_ctx* c, const Param& p) {
    return c->cfg.ref_gemm == AETH_REF_GEMM_SPLIT3 && p.r % 8 == 0 && p.m % 8 == 0 && p.n % 8 == 0;
}

// dW = fl(lr D) elementwise (optimizer.rs:337-340, weight_delta *= lr); with
// w: w = fl(w - dW); delta_out and scaled_out (either may be null) get dW.
__global__ void ref_delta_apply_kernel(const float* __restrict__ d, int64_t n, float lr, float* __restrict__ w,
                                       float* __restrict__ delta_out, float* __restrict__ scaled_out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float dw = __fmul_rn(d[i], lr);
        if (w) w[i] = __fsub_rn(w[i], dw);
        if (delta_out) delta_out[i] = dw;
        if (scaled_out) scaled_out[i] = dw;
    }
}

int ref_project_accumulate(aeth_galore_ctx* c, Param& p, const void* grad, int dtype, cudaStream_t st) {
    const float* g = static_cast<const float*>(grad);
    if (dtype != AETH_DTYPE_F32) {
        to_f32_kernel<<<grid_for((int64_t)p.m * p.n, 256), 256, 0, st>>>(grad, dtype, (int64_t)p.m * p.n, p.gtmp);
        AETH_LAUNCH_CHECK();
        g = p.gtmp;
    }
    const int m = p.m, n = p.n, r = p.r;
    if (ref_split(c, p)) {
        // Temp(r x n) = P^T G: A = P^T (P read MN-major), B = G (MN-major), K = m
        AETH_TRY(split3_gemm(F32Op{p.P, m, r, true}, F32Op{g, m, n, true}, p.temp, n, r, n, m, false, c->rsplit, st));
        // R += Temp Q: A = Temp (K-major), B = Q (MN-major), K = n
        return split3_gemm(F32Op{p.temp, r, n, false}, F32Op{p.Q, n, r, true}, p.accum, r, r, r, n, true, c->rsplit,
                           st);
    }
    // project.rs:36-46: Temp(r x n) = P^T G, sum over k of p[k*r+i] * g[k*n+j].
    AETH_TRY(simt_gemm_exact(p.P, 1, r, g, n, 1, p.temp, n, r, n, m, SIMT_STORE, 1.0f, nullptr, st));
    // project.rs:46 + adamw.rs:91-96: accum += Temp Q.
    AETH_TRY(simt_gemm_exact(p.temp, n, 1, p.Q, r, 1, p.accum, r, r, r, n, SIMT_ACCUM, 1.0f, nullptr, st));
    return AETH_OK;
}

int ref_apply(aeth_galore_ctx* c, Param& p, float clip, const float* clip_dev, const aeth_weight_ref* w,
              cudaStream_t st) {
    const aeth_galore_config& cfg = c->cfg;
    const int m = p.m, n = p.n, r = p.r;
    ref_adam_kernel<<<1, 1024, 0, st>>>(p.accum, p.m8, p.v8, p.mscale, p.vscale, p.mom, p.var, p.normalized,
                                        (int64_t)r * r, clip, clip_dev, cfg.beta1, cfg.beta2, cfg.eps);
    AETH_LAUNCH_CHECK();
    const float lr = cfg.scale_lr_by_rank ? cfg.lr / (float)(r < 1 ? 1 : r) : cfg.lr;  // adamw.rs:37-43
    const int kind = w ? w->kind : AETH_WEIGHT_NONE;
    if (ref_split(c, p)) {
        // project.rs:50-58 on the tensor cores: Temp(m x r) = P N (A = P K-major,
        // B = N MN-major, K = r); D(m x n) = Temp Q^T (B(k, j) = Q[j][k]: K-major,
        // K = r) into dtmp; then dW = lr D and the weight write elementwise.
        AETH_TRY(split3_gemm(F32Op{p.P, m, r, false}, F32Op{p.normalized, r, r, true}, p.temp, r, m, r, r, false,
                             c->rsplit, st));
        AETH_TRY(split3_gemm(F32Op{p.temp, m, r, false}, F32Op{p.Q, n, r, false}, p.dtmp, n, m, n, r, false,
                             c->rsplit, st));
        const int64_t mn = (int64_t)m * n;
        float* wf = kind == AETH_WEIGHT_F32 ? static_cast<float*>(w->data) : nullptr;
        float* delta = w ? w->delta_out : nullptr;
        ref_delta_apply_kernel<<<grid_for(mn, 256), 256, 0, st>>>(p.dtmp, mn, lr, wf, delta,
                                                                 kind == AETH_WEIGHT_NF4 ? p.dtmp : nullptr);
        AETH_LAUNCH_CHECK();
        if (kind == AETH_WEIGHT_NF4) {
            if (mn % 64 != 0) return AETH_ERR_SHAPE;
            nf4_apply_delta_kernel<<<grid_for(mn / 64, 128), 128, 0, st>>>(static_cast<uint8_t*>(w->data), w->absmax,
                                                                          p.dtmp, mn / 64, w->prequant_out);
            AETH_LAUNCH_CHECK();
        }
        return AETH_OK;
    }
    // project.rs:50-58: Temp(m x r) = P N; dW = Temp Q^T; dW *= lr.
    AETH_TRY(simt_gemm_exact(p.P, r, 1, p.normalized, r, 1, p.temp, r, m, r, r, SIMT_STORE, 1.0f, nullptr, st));
    if (kind == AETH_WEIGHT_F32) {
        AETH_TRY(simt_gemm_exact(p.temp, r, 1, p.Q, 1, r, static_cast<float*>(w->data), n, m, n, r, SIMT_SUB_SCALED,
                                 lr, w->delta_out, st));
    } else {
        float* dst = (kind == AETH_WEIGHT_NF4) ? p.dtmp : (w ? w->delta_out : nullptr);
        if (kind == AETH_WEIGHT_NF4 && w->delta_out) dst = w->delta_out;
        if (dst) AETH_TRY(simt_gemm_exact(p.temp, r, 1, p.Q, 1, r, dst, n, m, n, r, SIMT_SCALE, lr, nullptr, st));
        if (kind == AETH_WEIGHT_NF4) {
            if (((int64_t)m * n) % 64 != 0) return AETH_ERR_SHAPE;
            int64_t nb = (int64_t)m * n / 64;
            nf4_apply_delta_kernel<<<grid_for(nb, 128), 128, 0, st>>>(static_cast<uint8_t*>(w->data), w->absmax, dst,
                                                                    nb, w->prequant_out);
            AETH_LAUNCH_CHECK();
        }
    }
    return AETH_OK;
}

// ---- B200 mode ------------------------------------------------------------
// Number of exact bf16 terms of a gradient dtype (fp32: 24 significant bits
// in three terms of 8; f16: 11 bits in two).
int grad_terms(int dtype) { return dtype == AETH_DTYPE_F32 ? 3 : dtype == AETH_DTYPE_F16 ? 2 : 1; }

// projTk = projT repeated p.ksplit times along the contraction.
int sync_projk(Param& p, cudaStream_t st) {
    if (!p.projTk) return AETH_OK;
    const size_t s = (size_t)(p.side == 1 ? p.m : p.n);
    for (int t = 0; t < p.ksplit; ++t)
        AETH_CUDA(cudaMemcpy2DAsync(p.projTk + t * s, (size_t)p.ksplit * s * 2, p.projT, s * 2, s * 2, (size_t)p.r,
                                    cudaMemcpyDeviceToDevice, st));
    return AETH_OK;
}

// Buffers of the split path for `terms` bf16 terms: allocated at create when
// the configuration declares an fp32 / f16 gradient, else on first use
// (never while the stream is being captured into a graph).
int ensure_split(aeth_galore_ctx* c, Param& p, int terms, cudaStream_t st) {
    const int64_t need = (int64_t)terms * p.m * p.n;
    const bool have = p.projTk && p.ksplit >= terms && c->gsplit && c->gsplit_elems >= need;
    if (have) return AETH_OK;
    bool capturing = false;
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    AETH_CUDA(cudaStreamIsCapturing(st, &cap));
    capturing = cap != cudaStreamCaptureStatusNone;
    if (capturing) return AETH_ERR_UNSUPPORTED;
    AETH_CUDA(cudaStreamSynchronize(st));  // a smaller buffer may still be in use
    if (!c->gsplit || c->gsplit_elems < need) {
        ctx_free(c, c->gsplit);
        c->gsplit = nullptr;
        c->gsplit_elems = 0;
        AETH_TRY(ctx_alloc(c, &c->gsplit, need));
        c->gsplit_elems = need;
    }
    if (!p.projTk || p.ksplit < terms) {
        ctx_free(c, p.projTk);
        p.projTk = nullptr;
        p.ksplit = 0;
        const int64_t s = p.side == 1 ? p.m : p.n;
        AETH_TRY(ctx_alloc(c, &p.projTk, (int64_t)terms * s * p.r));
        p.ksplit = terms;
        AETH_TRY(sync_projk(p, st));
    }
    return AETH_OK;
}

// The projection job of one gradient: a bf16 gradient as it is; an fp32 or
// f16 gradient as its exact bf16 terms stacked along the contraction
// (grad_split_kernel), against the repeated projector.  No narrowing.
int b2_grad_job(aeth_galore_ctx* c, Param& p, const void* grad, int dtype, cudaStream_t st, ProjJob* job) {
    *job = ProjJob{grad, p.projT, p.accum, p.m, p.n};
    if (dtype == AETH_DTYPE_BF16) return AETH_OK;
    if (dtype != AETH_DTYPE_F32 && dtype != AETH_DTYPE_F16) return AETH_ERR_ARG;
    const int terms = grad_terms(dtype);
    const int64_t mn = (int64_t)p.m * p.n;
    if (p.n % 8 != 0) return AETH_ERR_UNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(grad) & 15) != 0) return AETH_ERR_UNSUPPORTED;
    AETH_TRY(ensure_split(c, p, terms, st));
    grad_split_kernel<<<grid_for(mn / 8, 256), 256, 0, st>>>(grad, dtype, p.m, p.n, terms, p.side == 2 ? 1 : 0,
                                                           c->gsplit);
    AETH_LAUNCH_CHECK();
    // projTk holds p.ksplit >= terms copies; the first `terms` are read
    *job = ProjJob{c->gsplit, p.projTk, p.accum, p.m, p.n};
    job->ksplit = terms;
    job->projk_ld = p.ksplit;
    return AETH_OK;
}

// One-CTA-per-tile tcgen05 projection, for shapes the grouped kernel does not
// take.  With k terms (the split path) the contraction is k times longer.
int b2_project_tile(Param& p, const ProjJob& j, cudaStream_t st) {
    const int m = p.m, n = p.n, r = p.r;
    const int k = j.ksplit, kl = j.projk_ld;
    EpiAccum epi{p.accum, r};
    if (p.side == 2) {
        // R(m x r) += G Q : A = G (K-major, ld k n), B(k,j) = Q[k][j] = projT[j*n + k] (K-major, ld kl n)
        return tc_gemm<false, false>(TcOperand{j.grad, k * n}, TcOperand{j.projT, kl * n}, m, r, k * n, true, epi, st);
    }
    // R^T(n x r) += G^T P : A(i,k) = G[k*n + i] (MN-major, ld n), B(k,j) = P[k][j] = projT[j*m + k] (K-major, ld kl m)
    return tc_gemm<true, false>(TcOperand{j.grad, n}, TcOperand{j.projT, kl * m}, n, r, k * m, true, epi, st);
}

// Whether the TMA-fed tensor-core kernels can describe this parameter: every
// row pitch of the gradient, the projector and the l x r state a multiple of
// 16 bytes.  Otherwise (the rank-1 RMS-norm vectors) small_rank.cuh serves it.
bool b2_tma_shape(const Param& p) { return p.r % 8 == 0 && p.m % 8 == 0 && p.n % 8 == 0; }

int b2_project_small(Param& p, const void* grad, int dtype, cudaStream_t st) {
    const int64_t cnt = (int64_t)std::max(p.m, p.n) * p.r;
    small_project_kernel<<<grid_for(cnt, 128), 128, 0, st>>>(grad, dtype, p.m, p.n, p.r, p.side == 2 ? 1 : 0, p.proj,
                                                            p.accum);
    AETH_LAUNCH_CHECK();
    return AETH_OK;
}

int b2_project_accumulate(aeth_galore_ctx* c, Param& p, const void* grad, int dtype, cudaStream_t st) {
    if (!b2_tma_shape(p) || (reinterpret_cast<uintptr_t>(grad) & 15) != 0) return b2_project_small(p, grad, dtype, st);
    ProjJob j;
    AETH_TRY(b2_grad_job(c, p, grad, dtype, st, &j));
    int s = proj_grouped_launch(&j, 1, p.r, st);
    return s == AETH_ERR_UNSUPPORTED ? b2_project_tile(p, j, st) : s;
}

float b2_lr(const aeth_galore_config& cfg, int r) {
    return cfg.scale_lr_by_rank ? cfg.lr / (float)(r < 1 ? 1 : r) : cfg.lr;  // adamw.rs:37-43
}

// K5: Adam on the state, N (bf16) out, optionally zeroing the accumulator.
int b2_adam(aeth_galore_ctx* c, Param& p, float clip, const float* clip_dev, int zero_accum, cudaStream_t st) {
    const aeth_galore_config& cfg = c->cfg;
    AETH_TRY(codec_maps_ensure());
    AdamB2Args a;
    a.accum = p.accum;
    a.m8 = p.m8;
    a.v8 = p.v8;
    a.m_scales = p.mscale;
    a.v_scales = p.vscale;
    a.n_out = p.nbuf;
    a.count = p.state_elems;
    a.block = cfg.state_block;
    a.codec = cfg.state_codec;
    a.clip_host = clip;
    a.clip_dev = clip_dev;
    a.b1 = cfg.beta1;
    a.b2 = cfg.beta2;
    a.eps = cfg.eps;
    a.zero_accum = zero_accum;
    b2_adam_kernel<<<grid_for(p.state_blocks, 1, 148 * 8), 256, 0, st>>>(a);
    AETH_LAUNCH_CHECK();
    return AETH_OK;
}

// K5 for several parameters in one persistent launch (2048-element blocks).
int b2_adam_group(aeth_galore_ctx* c, Param* const* ps, int np, float clip, const float* clip_dev, int zero_accum,
                  cudaStream_t st) {
    const aeth_galore_config& cfg = c->cfg;
    if (cfg.state_block != 2048) {
        for (int i = 0; i < np; ++i) AETH_TRY(b2_adam(c, *ps[i], clip, clip_dev, zero_accum, st));
        return AETH_OK;
    }
    AETH_TRY(codec_maps_ensure());
    {
        // a state whose size is not a multiple of 8 goes through the per-parameter kernel
        std::vector<Param*> grouped;
        for (int i = 0; i < np; ++i) {
            if (ps[i]->state_elems % 8 != 0) AETH_TRY(b2_adam(c, *ps[i], clip, clip_dev, zero_accum, st));
            else grouped.push_back(ps[i]);
        }
        if ((int)grouped.size() != np) {
            if (grouped.empty()) return AETH_OK;
            return b2_adam_group(c, grouped.data(), (int)grouped.size(), clip, clip_dev, zero_accum, st);
        }
    }
    const bool dyn = cfg.state_codec == AETH_CODEC_BLOCK_DYNAMIC;
    // 91 KB of tables per 1024-thread CTA, one CTA (32 warps) per SM
    static_assert(kAdamDynSmem2 + 1024 <= 227 * 1024, "the dynamic-codec Adam tables must fit one CTA");
    static bool attr_set[kMaxDevices] = {};
    int dev = 0;
    AETH_TRY(current_device(&dev));
    if (dyn && !attr_set[dev]) {
        AETH_CUDA(cudaFuncSetAttribute(b2_adam_dyn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAdamDynSmem2));
        attr_set[dev] = true;
    }
    for (int off = 0; off < np; off += kAdamGroupMax) {
        const int cnt = std::min(kAdamGroupMax, np - off);
        AdamGroupArgs a;
        memset(&a, 0, sizeof(a));
        int blocks = 0;
        for (int i = 0; i < cnt; ++i) {
            Param& p = *ps[off + i];
            if (p.state_elems % 8 != 0) return AETH_ERR_UNSUPPORTED;  // filtered out by the caller
            a.accum[i] = p.accum;
            a.m8[i] = p.m8;
            a.v8[i] = p.v8;
            a.ms[i] = p.mscale;
            a.vs[i] = p.vscale;
            a.nout[i] = p.nbuf;
            a.count[i] = p.state_elems;
            a.block_begin[i] = blocks;
            blocks += (int)p.state_blocks;
        }
        a.block_begin[cnt] = blocks;
        a.np = cnt;
        a.codec = cfg.state_codec;
        a.clip_host = clip;
        a.clip_dev = clip_dev;
        a.b1 = cfg.beta1;
        a.b2 = cfg.beta2;
        a.eps = cfg.eps;
        a.zero_accum = zero_accum;
        a.work = c->work;
        a.one = 1u;
        // dynamic codec: 1024-thread CTAs of four 256-thread groups, one per SM;
        // linear: 512-thread CTAs of two groups, two per SM; each group one block at a time
        if (dyn)
            b2_adam_dyn_kernel<<<std::min((blocks + 3) / 4, num_sms()), kAdamDynThreads, kAdamDynSmem2, st>>>(a);
        else
            b2_adam_group_kernel<<<std::min((blocks + 1) / 2, num_sms() * 2), 512, 0, st>>>(a);
        AETH_LAUNCH_CHECK();
    }
    return AETH_OK;
}

// K6 job for an NF4 weight, when the grouped kernel takes the shape.
bool b2_apply_job(const aeth_galore_config& cfg, const Param& p, const aeth_weight_ref* w, ApplyJob* j) {
    if (!w || w->kind != AETH_WEIGHT_NF4 || !apply_grouped_supported(p.m, p.n, p.r)) return false;
    const float lr = b2_lr(cfg, p.r);
    j->X = p.side == 2 ? p.nbuf : p.proj;
    j->Y = p.side == 2 ? p.proj : p.nbuf;
    j->wp = static_cast<uint8_t*>(w->data);
    j->wa = w->absmax;
    j->m = p.m;
    j->n = p.n;
    j->lr = lr;
    j->decay_mul = 1.0f - lr * cfg.weight_decay;
    j->has_decay = cfg.weight_decay > 0.0f;
    j->prequant = w->prequant_out;
    j->delta = w->delta_out;
    return (reinterpret_cast<uintptr_t>(w->data) & 15) == 0 && (reinterpret_cast<uintptr_t>(w->absmax) & 15) == 0;
}

int b2_weight_tile(aeth_galore_ctx* c, Param& p, const aeth_weight_ref* w, cudaStream_t st);

// K6: back-projection and weight write for one parameter.
int b2_weight(aeth_galore_ctx* c, Param& p, const aeth_weight_ref* w, cudaStream_t st) {
    ApplyJob job;
    if (b2_apply_job(c->cfg, p, w, &job)) return apply_grouped_launch(&job, 1, p.r, st);
    return b2_weight_tile(c, p, w, st);
}

int b2_apply(aeth_galore_ctx* c, Param& p, float clip, const float* clip_dev, const aeth_weight_ref* w,
             int zero_accum, cudaStream_t st) {
    Param* pp = &p;
    AETH_TRY(b2_adam_group(c, &pp, 1, clip, clip_dev, zero_accum, st));
    return b2_weight(c, p, w, st);
}

// One-CTA-per-tile back-projection with the generic epilogues (NF4 shapes the
// grouped kernel does not take, dense fp32 weights, delta-only output).
int b2_weight_tile(aeth_galore_ctx* c, Param& p, const aeth_weight_ref* w, cudaStream_t st) {
    const aeth_galore_config& cfg = c->cfg;
    const int m = p.m, n = p.n, r = p.r;
    const float lr = b2_lr(cfg, r);
    const int has_decay = cfg.weight_decay > 0.0f;
    const float decay_mul = 1.0f - lr * cfg.weight_decay;
    if (!b2_tma_shape(p)) {
        const int kind = w ? w->kind : AETH_WEIGHT_NONE;
        if (((int64_t)m * n) % 64 != 0) return AETH_ERR_UNSUPPORTED;
        if (kind == AETH_WEIGHT_NONE && !(w && w->delta_out)) return AETH_OK;
        const uint16_t* X = p.side == 2 ? p.nbuf : p.proj;
        const uint16_t* Y = p.side == 2 ? p.proj : p.nbuf;
        const int64_t blocks = (int64_t)m * n / 64;
        small_apply_kernel<<<grid_for(blocks * 32, 256), 256, 0, st>>>(
            X, Y, m, n, r, lr, decay_mul, has_decay, kind, w ? w->data : nullptr, w ? w->absmax : nullptr,
            w ? w->prequant_out : nullptr, w ? w->delta_out : nullptr);
        AETH_LAUNCH_CHECK();
        return AETH_OK;
    }
    // dW = X Y^T with X (m x r), Y (n x r), both K-major.
    TcOperand X = p.side == 2 ? TcOperand{p.nbuf, r} : TcOperand{p.proj, r};
    TcOperand Y = p.side == 2 ? TcOperand{p.proj, r} : TcOperand{p.nbuf, r};
    const int kind = w ? w->kind : AETH_WEIGHT_NONE;
    if (kind == AETH_WEIGHT_NF4) {
        if (n % 64 != 0) return AETH_ERR_UNSUPPORTED;
        EpiNf4Update e{static_cast<uint8_t*>(w->data), w->absmax, n, lr, decay_mul, has_decay, w->delta_out,
                       w->prequant_out};
        return tc_gemm_launch<256, 2, false, false>(X, Y, m, n, r, true, e, st);
    }
    if (kind == AETH_WEIGHT_F32) {
        EpiF32Update e{static_cast<float*>(w->data), n, lr, decay_mul, has_decay, w->delta_out};
        return tc_gemm_launch<256, 2, false, false>(X, Y, m, n, r, true, e, st);
    }
    if (w && w->delta_out) {
        // take_weight_delta semantics: delta = lr * dW (fp32).
        EpiStore s{w->delta_out, n, AETH_DTYPE_F32, lr};
        return tc_gemm_launch<256, 2, false, false>(X, Y, m, n, r, true, s, st);
    }
    return AETH_OK;
}

// ---------------------------------------------------------------------------
// Subspace refresh (optimizer.rs:208-246, 264-292, 373-398).
// ---------------------------------------------------------------------------
__global__ void capture_grad_kernel(const void* __restrict__ g, int dtype, int64_t n, float* __restrict__ cap,
                                    int first) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float v = load_as_f32(g, i, dtype);
        cap[i] = first ? v : __fadd_rn(cap[i], v);  // or_insert(grad.to_vec()) / and_modify(+=)
    }
}

// project_and_accumulate's capture (optimizer.rs:266-286): at step + 1 == 1
// or should_switch_subspace(step + 1, switch_interval), sum the full gradient.
int capture_if_due(aeth_galore_ctx* c, Param& p, const void* grad, int dtype, cudaStream_t st) {
    if (!c->cfg.svd_refresh) return AETH_OK;
    const uint64_t this_step = c->step + 1;
    const uint64_t every = c->cfg.switch_interval;
    if (!(this_step == 1 || (every > 0 && this_step % every == 0))) return AETH_OK;
    const int64_t n = (int64_t)p.m * p.n;
    if (!p.capture) AETH_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&p.capture), n * sizeof(float), st));
    capture_grad_kernel<<<grid_for(n, 256), 256, 0, st>>>(grad, dtype, n, p.capture, p.captured ? 0 : 1);
    AETH_LAUNCH_CHECK();
    p.captured = true;
    return AETH_OK;
}

void drop_capture(Param& p, cudaStream_t st) {
    if (p.capture) cudaFreeAsync(p.capture, st);
    p.capture = nullptr;
    p.captured = false;
}

// New projectors for one captured parameter, then the Adam state reset
// (optimizer.rs:229-240).  The projectors change only on success.
int refresh_param(aeth_galore_ctx* c, Param& p, uint64_t seed, cudaStream_t st) {
    const bool ref = c->cfg.mode == AETH_MODE_REF;
    const bool want_p = ref || p.side == 1, want_q = ref || p.side == 2;
    float* tp = nullptr;
    float* tq = nullptr;
    int status = AETH_OK;
    cudaError_t e = cudaSuccess;
    if (want_p) e = cudaMallocAsync(reinterpret_cast<void**>(&tp), sizeof(float) * (size_t)p.m * p.r, st);
    if (e == cudaSuccess && want_q)
        e = cudaMallocAsync(reinterpret_cast<void**>(&tq), sizeof(float) * (size_t)p.n * p.r, st);
    if (e != cudaSuccess) status = (int)e;
    // REF mode with the exact GEMMs keeps the reference's f32 loop order;
    // otherwise the products run on the tensor cores
    const bool fast = !ref || c->cfg.ref_gemm == AETH_REF_GEMM_SPLIT3;
    if (status == AETH_OK)
        status = rsvd_device(p.capture, false, p.m, p.n, p.r, c->cfg.oversampling, c->cfg.power_iters, seed, fast,
                             tp, tq, st);
    if (status == AETH_OK) {
        if (ref) {
            e = cudaMemcpyAsync(p.P, tp, sizeof(float) * (size_t)p.m * p.r, cudaMemcpyDeviceToDevice, st);
            if (e == cudaSuccess)
                e = cudaMemcpyAsync(p.Q, tq, sizeof(float) * (size_t)p.n * p.r, cudaMemcpyDeviceToDevice, st);
            if (e != cudaSuccess) status = (int)e;
        } else {
            const int s_dim = p.side == 1 ? p.m : p.n;
            proj_to_bf16_kernel<<<grid_for((int64_t)s_dim * p.r, 256), 256, 0, st>>>(p.side == 1 ? tp : tq, s_dim,
                                                                                     p.r, p.proj, p.projT);
            e = cudaGetLastError();
            if (e != cudaSuccess) status = (int)e;
            if (status == AETH_OK) status = sync_projk(p, st);
        }
        if (status == AETH_OK) status = reset_state(c, p, st);
    }
    if (tp) cudaFreeAsync(tp, st);
    if (tq) cudaFreeAsync(tq, st);
    drop_capture(p, st);
    return status;
}

// New projector of one B200 parameter from this step's gradient, kept aside
// (pend_proj / pend_projT) until notify_step installs it: the step's own
// back-projection still uses the projector its accumulator was projected
// with, as the reference's refresh in notify_step after the update does
// (optimizer.rs:208-246, 373-398).  Seed of the step in progress.  Enqueued
// on `st` without waiting; *status_dev becomes 1 for a rank-deficient sketch.
// pend_proj / pend_projT must be allocated.
int refresh_enqueue(aeth_galore_ctx* c, Param& p, const void* grad, int dtype, int* status_dev, cudaStream_t st) {
    const int s_dim = p.side == 1 ? p.m : p.n;
    const size_t pe = (size_t)s_dim * p.r;
    const uint64_t seed = (c->step + 1) * 0x9E3779B9ull;  // the step notify_step will record
    float* tproj = nullptr;
    float* gf = nullptr;
    const int64_t mn = (int64_t)p.m * p.n;
    AETH_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&tproj), sizeof(float) * pe, st));
    int status = AETH_OK;
    const void* g = grad;
    if (dtype == AETH_DTYPE_F16) {  // widened exactly; the refresh reads bf16 or fp32
        cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&gf), sizeof(float) * (size_t)mn, st);
        if (e != cudaSuccess) status = (int)e;
        else {
            to_f32_kernel<<<grid_for(mn, 256), 256, 0, st>>>(grad, dtype, mn, gf);
            g = gf;
        }
    }
    if (status == AETH_OK)
        status = rsvd_launch(g, dtype == AETH_DTYPE_BF16, p.m, p.n, p.r, c->cfg.oversampling, c->cfg.power_iters,
                             seed, true, p.side == 1 ? tproj : nullptr, p.side == 2 ? tproj : nullptr, status_dev, st);
    if (status == AETH_OK) {
        proj_to_bf16_kernel<<<grid_for((int64_t)pe, 256), 256, 0, st>>>(tproj, s_dim, p.r, p.pend_proj,
                                                                       p.pend_projT);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) status = (int)e;
    }
    cudaFreeAsync(tproj, st);
    if (gf) cudaFreeAsync(gf, st);
    return status;
}

// Installs the pending projectors (stable buffers, so recorded graphs stay
// valid) and resets their Adam state.  Returns whether any was installed.
int install_pending(aeth_galore_ctx* c, cudaStream_t st, bool* any) {
    *any = false;
    for (Param& p : c->params) {
        if (!p.pending) continue;
        const size_t bytes = sizeof(uint16_t) * (size_t)(p.side == 1 ? p.m : p.n) * p.r;
        AETH_CUDA(cudaMemcpyAsync(p.proj, p.pend_proj, bytes, cudaMemcpyDeviceToDevice, st));
        AETH_CUDA(cudaMemcpyAsync(p.projT, p.pend_projT, bytes, cudaMemcpyDeviceToDevice, st));
        AETH_TRY(sync_projk(p, st));
        AETH_TRY(reset_state(c, p, st));
        p.pending = false;
        *any = true;
    }
    return AETH_OK;
}

int notify_step_on(aeth_galore_ctx* c, uint64_t step, cudaStream_t st) {
    c->step = step;
    bool installed = false;
    AETH_TRY(install_pending(c, st, &installed));
    bool any = false;
    for (Param& p : c->params) any = any || p.captured;
    if (!any) {
        if (installed) ++c->version;
        return AETH_OK;
    }
    const uint64_t seed = step * 0x9E3779B9ull;  // wrapping_mul (optimizer.rs:216-221)
    int status = AETH_OK;
    for (Param& p : c->params) {
        if (!p.captured) continue;
        if (status == AETH_OK) status = refresh_param(c, p, seed, st);
        else drop_capture(p, st);  // the reference drops the remaining jobs after an error
    }
    if (status == AETH_OK) ++c->version;
    return status;
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

const char* aeth_version(void) { return "aeth_galore 0.1 (sm_100a)"; }

const char* aeth_status_string(int st) {
    switch (st) {
        case AETH_OK: return "ok";
        case AETH_ERR_ARG: return "invalid argument";
        case AETH_ERR_SHAPE: return "shape mismatch";
        case AETH_ERR_CONFIG: return "configuration error";
        case AETH_ERR_UNSUPPORTED: return "unsupported shape or alignment";
        case AETH_ERR_NOT_FOUND: return "unknown parameter";
        case AETH_ERR_TIMEOUT: return "device wait timed out";
        case AETH_ERR_LINALG: return "rank-deficient factorisation";
        default: return st > 0 ? cudaGetErrorString((cudaError_t)st) : "unknown error";
    }
}

int aeth_last_error(void) { return tl_last_error; }

int aeth_device_error_bits(int device, uint32_t* bits) {
    if (!bits) return set_err(AETH_ERR_ARG);
    DeviceGuard g(device);
    DeviceRuntime* rt = nullptr;
    AETH_TRY(runtime_for_current(&rt));
    AETH_CUDA(cudaDeviceSynchronize());
    uint32_t v = 0;
    AETH_CUDA(cudaMemcpy(&v, rt->err_word, sizeof(v), cudaMemcpyDeviceToHost));
    AETH_CUDA(cudaMemset(rt->err_word, 0, sizeof(uint32_t)));
    *bits = v;
    return AETH_OK;
}

int aeth_device_error(int device) {
    uint32_t v = 0;
    AETH_TRY(aeth_device_error_bits(device, &v));
    return v ? AETH_ERR_TIMEOUT : AETH_OK;
}

int aeth_dynamic_map(int is_signed, float out[256]) {
    if (!out) return AETH_ERR_ARG;
    return build_dynamic_map(is_signed, out);
}

int aeth_selfcheck(int which, unsigned long long* mismatches) {
    if (!mismatches || which < AETH_SELFCHECK_DMAP_SIGNED || which > AETH_SELFCHECK_NF4_CLASSIFY)
        return set_err(AETH_ERR_ARG);
    AETH_TRY(codec_maps_ensure());
    unsigned long long* d = nullptr;
    AETH_CUDA(cudaMalloc(&d, sizeof(*d)));
    cudaError_t e = cudaMemset(d, 0, sizeof(*d));
    if (e == cudaSuccess) {
        if (which == AETH_SELFCHECK_NF4_CLASSIFY) {
            const float amaxes[] = {1.0f, 0.37f, 0.02f, 3.3e-5f, 1e-9f, 7.7e30f};
            for (float amax : amaxes) nf4_classify_selfcheck_kernel<<<num_sms() * 8, 256>>>(amax, d);
        } else if (which == AETH_SELFCHECK_ADAM_DIR)
            adam_dir_selfcheck_kernel<<<num_sms() * 8, 256>>>(d);
        else
            dmap_selfcheck_kernel<<<num_sms() * 8, 256>>>(which == AETH_SELFCHECK_DMAP_SIGNED ? 1 : 0, d, 1u);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpy(mismatches, d, sizeof(*d), cudaMemcpyDeviceToHost);
    cudaFree(d);
    AETH_CUDA(e);
    return AETH_OK;
}

// ---------------------------------------------------------------------------
// Reference-compatible symbols
// ---------------------------------------------------------------------------
int galore_project_forward(const void* G, const void* P, const void* Q, void* R, void* temp, int m, int n, int r,
                           aeth_stream_t stream) {
    if (m <= 0 || n <= 0 || r <= 0) return set_err(AETH_ERR_ARG);
    if (!G || !P || !Q || !R || !temp) return set_err(AETH_ERR_ARG);
    cudaStream_t st = to_stream(stream);
    // Temp(r x n) = P^T G: A(i,k) = P[k*r + i] (MN-major), B(k,j) = G[k*n + j] (MN-major)
    EpiStore e1{temp, n, AETH_DTYPE_F16, 1.0f};
    int s1 = tc_gemm<true, true>(TcOperand{P, r}, TcOperand{G, n}, r, n, m, false, e1, st);
    if (s1 == AETH_ERR_UNSUPPORTED) {
        simt_gemm_any_kernel<<<grid_for((int64_t)r * n, 256), 256, 0, st>>>(P, AETH_DTYPE_F16, 1, r, G, AETH_DTYPE_F16,
                                                                          n, 1, temp, AETH_DTYPE_F16, n, r, n, m);
        AETH_LAUNCH_CHECK();
    } else if (s1 != AETH_OK) {
        return set_err(s1);
    }
    // R(r x r) = Temp Q: A = Temp (K-major, ld n), B(k,j) = Q[k*r + j] (MN-major, ld r)
    EpiStore e2{R, r, AETH_DTYPE_F16, 1.0f};
    int s2 = tc_gemm<false, true>(TcOperand{temp, n}, TcOperand{Q, r}, r, r, n, false, e2, st);
    if (s2 == AETH_ERR_UNSUPPORTED) {
        simt_gemm_any_kernel<<<grid_for((int64_t)r * r, 256), 256, 0, st>>>(temp, AETH_DTYPE_F16, n, 1, Q,
                                                                          AETH_DTYPE_F16, r, 1, R, AETH_DTYPE_F16, r, r,
                                                                          r, n);
        AETH_LAUNCH_CHECK();
    } else if (s2 != AETH_OK) {
        return set_err(s2);
    }
    return AETH_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free variant of galore_project_forward.
//
// For callers that cannot allocate device memory at the point of the call:
// for example code running inside another framework's step whose device
// memory is all reserved by that framework's caching allocator (a raw
// cudaMalloc there fails or fragments the pool), or code that must not
// allocate once a run has started.  The r x n fp16 intermediate P^T G lives
// in g_noalloc_temp below, a fixed array every device that loads this library
// holds until the process exits.  Device code may name the array; host code
// must use the address from cudaGetSymbolAddress (the host-side symbol is a
// stand-in, not a device address).
// ---------------------------------------------------------------------------
namespace {

constexpr int64_t kNoAllocTempElems = 8 * 1024 * 1024;  // 16 MiB of fp16: r * n <= 8,388,608

static __device__ __align__(256) __half g_noalloc_temp[kNoAllocTempElems];
// Error word for the bounded waits of the tcgen05 kernels, so the first call
// on a device needs no cudaMalloc either.
static __device__ __align__(16) uint32_t g_noalloc_err_word;

struct NoAllocDevice {
    void* temp = nullptr;
    bool ready = false;
};
NoAllocDevice g_noalloc[kMaxDevices];

// Once per device, with that device current: device addresses of the static
// arrays.  If the library's per-device runtime is not set up yet, its error
// word becomes g_noalloc_err_word (zero-initialised at module load), so no
// later step on this path allocates.
int noalloc_setup(void** temp) {
    int dev = 0;
    AETH_TRY(current_device(&dev));
    if (dev < 0 || dev >= kMaxDevices) return AETH_ERR_UNSUPPORTED;
    // g_rt_mu also guards runtime_for_current's first use, so the error word
    // is chosen exactly once per device whichever path comes first.
    std::lock_guard<std::mutex> lock(g_rt_mu);
    NoAllocDevice& d = g_noalloc[dev];
    if (!d.ready) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_temp);
        if (e != cudaSuccess) return (int)e;
        if (!g_rt[dev].init.load(std::memory_order_relaxed)) {
            void* w = nullptr;
            e = cudaGetSymbolAddress(&w, g_noalloc_err_word);
            if (e != cudaSuccess) return (int)e;
            g_rt[dev].err_word = static_cast<uint32_t*>(w);
            g_rt[dev].init.store(true, std::memory_order_release);
        }
        d.temp = p;
        d.ready = true;
    }
    *temp = d.temp;
    return AETH_OK;
}

}  // namespace

extern "C" {

int galore_project_forward_noalloc(const void* G, const void* P, const void* Q, void* R, int m, int n, int r,
                                   aeth_stream_t stream) {
    if (m <= 0 || n <= 0 || r <= 0) return set_err(AETH_ERR_ARG);
    if (!G || !P || !Q || !R) return set_err(AETH_ERR_ARG);
    if ((int64_t)r * n > kNoAllocTempElems) return set_err(AETH_ERR_UNSUPPORTED);  // r * n above the fixed scratch
    void* temp = nullptr;
    int st = noalloc_setup(&temp);
    if (st != AETH_OK) return set_err(st);
    // Every element of the r x n intermediate is written before it is read,
    // so the array's previous contents never matter.
    return galore_project_forward(G, P, Q, R, temp, m, n, r, stream);
}

int galore_project_backward(const void* N, const void* P, const void* Q, void* G_tilde, void* temp, int m, int n,
                            int r, aeth_stream_t stream) {
    if (m <= 0 || n <= 0 || r <= 0) return set_err(AETH_ERR_ARG);
    if (!N || !P || !Q || !G_tilde || !temp) return set_err(AETH_ERR_ARG);
    cudaStream_t st = to_stream(stream);
    // Temp(m x r) = P N: A = P (K-major, ld r), B(k,j) = N[k*r + j] (MN-major, ld r)
    EpiStore e1{temp, r, AETH_DTYPE_F16, 1.0f};
    int s1 = tc_gemm<false, true>(TcOperand{P, r}, TcOperand{N, r}, m, r, r, false, e1, st);
    if (s1 == AETH_ERR_UNSUPPORTED) {
        simt_gemm_any_kernel<<<grid_for((int64_t)m * r, 256), 256, 0, st>>>(P, AETH_DTYPE_F16, r, 1, N, AETH_DTYPE_F16,
                                                                          r, 1, temp, AETH_DTYPE_F16, r, m, r, r);
        AETH_LAUNCH_CHECK();
    } else if (s1 != AETH_OK) {
        return set_err(s1);
    }
    // G~(m x n) = Temp Q^T: A = Temp (K-major, ld r), B(k,j) = Q[j*r + k] (K-major, ld r)
    EpiStore e2{G_tilde, n, AETH_DTYPE_F16, 1.0f};
    int s2 = tc_gemm<false, false>(TcOperand{temp, r}, TcOperand{Q, r}, m, n, r, false, e2, st);
    if (s2 == AETH_ERR_UNSUPPORTED) {
        simt_gemm_any_kernel<<<grid_for((int64_t)m * n, 256), 256, 0, st>>>(temp, AETH_DTYPE_F16, r, 1, Q,
                                                                          AETH_DTYPE_F16, 1, r, G_tilde, AETH_DTYPE_F16,
                                                                          n, m, n, r);
        AETH_LAUNCH_CHECK();
    } else if (s2 != AETH_OK) {
        return set_err(s2);
    }
    return AETH_OK;
}

int galore_quantize_absmax_f32_to_i8(const float* src, int8_t* dst, float* scale_out, int n_elements,
                                     aeth_stream_t stream) {
    if (n_elements <= 0 || !src || !dst || !scale_out) return set_err(AETH_ERR_ARG);
    cudaStream_t st = to_stream(stream);
    AETH_CUDA(cudaMemsetAsync(scale_out, 0, sizeof(float), st));
    absmax_reduce_kernel<<<grid_for(n_elements, 256, 148 * 4), 256, 0, st>>>(src, n_elements, scale_out);
    per_tensor_encode_kernel<<<grid_for(n_elements, 256), 256, 0, st>>>(src, n_elements, scale_out, dst);
    per_tensor_finalize_kernel<<<1, 1, 0, st>>>(scale_out);
    AETH_LAUNCH_CHECK();
    return AETH_OK;
}

int galore_dequantize_i8_to_f32(const int8_t* src, float* dst, float scale, int n_elements, aeth_stream_t stream) {
    if (n_elements <= 0 || !src || !dst) return set_err(AETH_ERR_ARG);
    cudaStream_t st = to_stream(stream);
    dequant_linear_kernel<<<grid_for(n_elements, 256), 256, 0, st>>>(src, nullptr, scale, n_elements, 0, dst);
    AETH_LAUNCH_CHECK();
    return AETH_OK;
}

void doublepass_galore_apply(float* param, const float* grad_lr, float* m, float* v, float clip_scale, float beta1,
                             float beta2, float eps, float lr, int n_elements, int step) {
    tl_last_error = AETH_OK;
    if (n_elements <= 0 || !param || !grad_lr || !m || !v) {
        set_err(AETH_ERR_ARG);
        return;
    }
    float bc1 = 1.0f, bc2 = 1.0f;
    if (step >= 1) {
        bc1 = (float)(1.0 - pow((double)beta1, (double)step));
        bc2 = (float)(1.0 - pow((double)beta2, (double)step));
    }
    full_adam_kernel<<<grid_for(n_elements, 256), 256, 0, 0>>>(param, grad_lr, m, v, n_elements, clip_scale, beta1,
                                                               beta2, eps, lr, step >= 1 ? 1 : 0, bc1, bc2);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) set_err((int)e);
}

// ---------------------------------------------------------------------------
// Optimizer handle
// ---------------------------------------------------------------------------
void aeth_galore_config_default(aeth_galore_config* c) {
    if (!c) return;
    memset(c, 0, sizeof(*c));
    c->mode = AETH_MODE_REF;
    c->default_rank = 16;   // GaLoreConfig::default rank (optimizer.rs:49-60)
    c->attn_rank = 32;      // LayerRankConfig::default (layer_rank.rs:19-27)
    c->mlp_rank = 16;
    c->vector_rank = 8;
    c->switch_interval = 200;
    c->oversampling = 10;
    c->beta1 = 0.9f;        // AdamWConfig::default (adamw.rs:23-33)
    c->beta2 = 0.999f;
    c->eps = 1e-8f;
    c->lr = 1e-3f;
    c->weight_decay = 0.0f;
    c->scale_lr_by_rank = 0;
    c->max_grad_norm = 1.0f;  // TrainingPlan (doublepass/src/plan.rs)
    c->state_codec = AETH_CODEC_PER_TENSOR;
    c->state_block = 2048;
    c->init_projectors = 1;
    c->svd_refresh = 1;  // the reference captures at step 1 and every switch_interval steps
    c->power_iters = 0;  // RandomizedSvdConfig::default (randomized_svd.rs:19-28), never used by the reference
    c->grad_dtype = AETH_DTYPE_BF16;
    c->ref_gemm = AETH_REF_GEMM_EXACT;
}

int aeth_galore_destroy(aeth_galore_ctx* ctx) {
    if (!ctx) return AETH_ERR_ARG;
    DeviceGuard g(ctx->device);
    cudaDeviceSynchronize();
    for (auto& rec : ctx->phase_pending)
        for (cudaEvent_t e : rec.ev) cudaEventDestroy(e);
    for (cudaEvent_t e : ctx->event_pool) cudaEventDestroy(e);
    for (void* p : ctx->allocs) cudaFree(p);
    for (Param& p : ctx->params)
        if (p.capture) cudaFree(p.capture);
    for (void* m : ctx->peer_maps) cudaIpcCloseMemHandle(m);
    for (cudaStream_t s : ctx->side_streams) cudaStreamDestroy(s);
    if (ctx->own_slots) cudaFree(ctx->own_slots);
    delete ctx;
    return AETH_OK;
}

int aeth_galore_create(const aeth_galore_config* cfg, const aeth_param_spec* specs, int n_specs, int device,
                       aeth_galore_ctx** out) {
    if (!cfg || !out || n_specs < 0 || (n_specs > 0 && !specs)) return set_err(AETH_ERR_ARG);
    *out = nullptr;
    if (cfg->mode != AETH_MODE_REF && cfg->mode != AETH_MODE_B200) return set_err(AETH_ERR_CONFIG);
    if (cfg->mode == AETH_MODE_REF && cfg->state_codec != AETH_CODEC_PER_TENSOR) return set_err(AETH_ERR_CONFIG);
    if (cfg->mode == AETH_MODE_B200 &&
        (cfg->state_codec == AETH_CODEC_PER_TENSOR || cfg->state_block <= 0))
        return set_err(AETH_ERR_CONFIG);
    if (cfg->grad_dtype != AETH_DTYPE_F32 && cfg->grad_dtype != AETH_DTYPE_F16 && cfg->grad_dtype != AETH_DTYPE_BF16)
        return set_err(AETH_ERR_CONFIG);
    if (cfg->ref_gemm != AETH_REF_GEMM_EXACT && cfg->ref_gemm != AETH_REF_GEMM_SPLIT3) return set_err(AETH_ERR_CONFIG);
    DeviceGuard g(device);
    aeth_galore_ctx* c = new aeth_galore_ctx();
    c->cfg = *cfg;
    c->device = device;
    auto fail = [&](int st) {
        aeth_galore_destroy(c);
        return set_err(st);
    };
    int st = AETH_OK;
    if ((st = codec_maps_ensure()) != AETH_OK) return fail(st);
    c->params.resize(n_specs);
    int64_t split_need = 0;
    for (int i = 0; i < n_specs; ++i) {
        const aeth_param_spec& s = specs[i];
        if (s.m <= 0 || s.n <= 0) return fail(AETH_ERR_SHAPE);
        for (int j = 0; j < i; ++j)
            if (specs[j].layer_idx == s.layer_idx && std::string(specs[j].name ? specs[j].name : "") == (s.name ? s.name : ""))
                return fail(AETH_ERR_CONFIG);
        Param& p = c->params[i];
        p.layer = s.layer_idx;
        p.name = s.name ? s.name : "";
        p.m = s.m;
        p.n = s.n;
        p.r = s.rank > 0 ? s.rank : rank_for_param(*cfg, s.name, s.m, s.n);
        if (p.r > (s.m < s.n ? s.m : s.n)) return fail(AETH_ERR_CONFIG);
        const int m = p.m, n = p.n, r = p.r;
        if (cfg->mode == AETH_MODE_REF) {
            p.side = 0;
            p.state_elems = (int64_t)r * r;
            p.state_blocks = 1;
            if ((st = ctx_alloc(c, &p.P, (int64_t)m * r)) || (st = ctx_alloc(c, &p.Q, (int64_t)n * r)) ||
                (st = ctx_alloc(c, &p.mom, (int64_t)r * r)) || (st = ctx_alloc(c, &p.var, (int64_t)r * r)) ||
                (st = ctx_alloc(c, &p.normalized, (int64_t)r * r)) ||
                (st = ctx_alloc(c, &p.temp, std::max((int64_t)r * n, (int64_t)m * r))) ||
                (st = ctx_alloc(c, &p.gtmp, (int64_t)m * n)) || (st = ctx_alloc(c, &p.dtmp, (int64_t)m * n)))
                return fail(st);
        } else {
            p.side = m >= n ? 2 : 1;
            const int64_t l = m >= n ? m : n;
            const int s_dim = m >= n ? n : m;
            p.state_elems = l * r;
            p.state_blocks = (p.state_elems + cfg->state_block - 1) / cfg->state_block;
            if ((st = ctx_alloc(c, &p.proj, (int64_t)s_dim * r)) || (st = ctx_alloc(c, &p.projT, (int64_t)s_dim * r)) ||
                (st = ctx_alloc(c, &p.nbuf, p.state_elems)))
                return fail(st);
        }
        if ((st = ctx_alloc(c, &p.accum, p.state_elems)) || (st = ctx_alloc(c, &p.m8, p.state_elems)) ||
            (st = ctx_alloc(c, &p.v8, p.state_elems)) || (st = ctx_alloc(c, &p.mscale, p.state_blocks)) ||
            (st = ctx_alloc(c, &p.vscale, p.state_blocks)))
            return fail(st);
        if ((st = reset_state(c, p, 0)) != AETH_OK) return fail(st);
        // Projector initialisation (optimizer.rs:98-100): P from seed layer*17, Q from layer*31.
        const bool want_p = cfg->mode == AETH_MODE_REF || p.side == 1;
        const bool want_q = cfg->mode == AETH_MODE_REF || p.side == 2;
        std::vector<float> hp, hq;
        if (cfg->init_projectors) {
            if (want_p) { hp.resize((size_t)m * r); init_random_projection_host(m, r, p.layer * 17u, hp.data()); }
            if (want_q) { hq.resize((size_t)n * r); init_random_projection_host(n, r, p.layer * 31u, hq.data()); }
        } else {
            if (want_p) hp.assign((size_t)m * r, 0.0f);
            if (want_q) hq.assign((size_t)n * r, 0.0f);
        }
        if (cfg->mode == AETH_MODE_REF) {
            if (cudaMemcpy(p.P, hp.data(), hp.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
                cudaMemcpy(p.Q, hq.data(), hq.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
                return fail(AETH_ERR_CONFIG);
        } else {
            const std::vector<float>& src = p.side == 1 ? hp : hq;
            const int s_dim = p.side == 1 ? m : n;
            std::vector<uint16_t> b(src.size()), bt(src.size());
            for (int row = 0; row < s_dim; ++row)
                for (int col = 0; col < r; ++col) {
                    uint16_t v = host_f32_to_bf16(src[(size_t)row * r + col]);
                    b[(size_t)row * r + col] = v;
                    bt[(size_t)col * s_dim + row] = v;
                }
            if (cudaMemcpy(p.proj, b.data(), b.size() * 2, cudaMemcpyHostToDevice) != cudaSuccess ||
                cudaMemcpy(p.projT, bt.data(), bt.size() * 2, cudaMemcpyHostToDevice) != cudaSuccess)
                return fail(AETH_ERR_CONFIG);
            // a declared fp32 / f16 gradient: the split path's buffers now, so
            // no step allocates (and every step can be captured into a graph)
            const int terms = grad_terms(cfg->grad_dtype);
            if (terms > 1) {
                if ((st = ctx_alloc(c, &p.projTk, (int64_t)terms * s_dim * r)) != AETH_OK) return fail(st);
                p.ksplit = terms;
                if ((st = sync_projk(p, 0)) != AETH_OK) return fail(st);
                split_need = std::max(split_need, (int64_t)terms * m * n);
            }
        }
    }
    if ((st = ctx_alloc(c, &c->sq_slots, n_specs)) || (st = ctx_alloc(c, &c->sq_step, n_specs)) ||
        (st = ctx_alloc(c, &c->partials, std::max(kSqPartials, kSqPartialSlots))) ||
        (st = ctx_alloc(c, &c->clip_dev, 1)) ||
        (st = ctx_alloc(c, &c->gnorm_dev, 1)) || (st = ctx_alloc(c, &c->sq_ticket, 1)) ||
        (st = ctx_alloc(c, &c->work, 2)) || (st = ctx_alloc(c, &c->clip_epoch, 1)))
        return fail(st);
    if (split_need > 0) {
        if ((st = ctx_alloc(c, &c->gsplit, split_need)) != AETH_OK) return fail(st);
        c->gsplit_elems = split_need;
    }
    if (cfg->mode == AETH_MODE_REF && cfg->ref_gemm == AETH_REF_GEMM_SPLIT3) {
        // three terms of each operand of the largest product, P^T G (r m + m n)
        int64_t need = 0;
        for (const Param& p : c->params)
            need = std::max(need, 3 * ((int64_t)p.r * std::max(p.m, p.n) + (int64_t)p.m * p.n + (int64_t)p.r * p.r));
        if ((st = ctx_alloc(c, &c->rsplit, need)) != AETH_OK) return fail(st);
    }
    if (cudaMemset(c->sq_ticket, 0, sizeof(unsigned int)) != cudaSuccess ||
        cudaMemset(c->work, 0, 2 * sizeof(unsigned int)) != cudaSuccess)
        return fail(AETH_ERR_CONFIG);
    if (cudaDeviceSynchronize() != cudaSuccess) return fail(AETH_ERR_CONFIG);
    *out = c;
    return AETH_OK;
}

int aeth_galore_num_params(const aeth_galore_ctx* ctx) { return ctx ? (int)ctx->params.size() : AETH_ERR_ARG; }

int aeth_galore_find(const aeth_galore_ctx* ctx, uint32_t layer_idx, const char* name) {
    if (!ctx || !name) return AETH_ERR_ARG;
    for (size_t i = 0; i < ctx->params.size(); ++i)
        if (ctx->params[i].layer == layer_idx && ctx->params[i].name == name) return (int)i;
    return AETH_ERR_NOT_FOUND;
}

int aeth_galore_param_info(const aeth_galore_ctx* ctx, int idx, aeth_param_info* out) {
    AETH_TRY(check_idx(ctx, idx));
    if (!out) return AETH_ERR_ARG;
    const Param& p = ctx->params[idx];
    out->m = p.m;
    out->n = p.n;
    out->rank = p.r;
    out->side = p.side;
    out->state_elems = p.state_elems;
    out->state_blocks = p.state_blocks;
    out->layer_idx = p.layer;
    return AETH_OK;
}

int aeth_galore_project_accumulate(aeth_galore_ctx* ctx, int idx, const void* grad, int grad_dtype,
                                   aeth_stream_t stream) {
    AETH_TRY(check_idx(ctx, idx));
    if (!grad) return set_err(AETH_ERR_ARG);
    DeviceGuard g(ctx->device);
    Param& p = ctx->params[idx];
    cudaStream_t st = to_stream(stream);
    AETH_TRY(set_err(capture_if_due(ctx, p, grad, grad_dtype, st)));
    if (ctx->cfg.mode == AETH_MODE_REF) return set_err(ref_project_accumulate(ctx, p, grad, grad_dtype, st));
    return set_err(b2_project_accumulate(ctx, p, grad, grad_dtype, st));
}

int aeth_galore_sqnorm_device(aeth_galore_ctx* ctx, int idx, double* out_dev, aeth_stream_t stream) {
    AETH_TRY(check_idx(ctx, idx));
    DeviceGuard g(ctx->device);
    Param& p = ctx->params[idx];
    return set_err(sqnorm_into(ctx, p, out_dev ? out_dev : ctx->sq_slots + idx, to_stream(stream)));
}

int aeth_galore_sqnorm(aeth_galore_ctx* ctx, int idx, double* out_host, aeth_stream_t stream) {
    AETH_TRY(check_idx(ctx, idx));
    if (!out_host) return set_err(AETH_ERR_ARG);
    DeviceGuard g(ctx->device);
    cudaStream_t st = to_stream(stream);
    AETH_TRY(sqnorm_into(ctx, ctx->params[idx], ctx->sq_slots + idx, st));
    AETH_CUDA(cudaMemcpyAsync(out_host, ctx->sq_slots + idx, sizeof(double), cudaMemcpyDeviceToHost, st));
    AETH_CUDA(cudaStreamSynchronize(st));
    return AETH_OK;
}

int aeth_clip_coeff_device(const double* sq_dev, int n, float max_norm, float* clip_dev, double* gnorm_dev,
                           aeth_stream_t stream) {
    if (!sq_dev || n <= 0 || !clip_dev) return set_err(AETH_ERR_ARG);
    clip_coeff_kernel<<<1, 32, 0, to_stream(stream)>>>(sq_dev, n, max_norm, clip_dev, gnorm_dev);
    AETH_LAUNCH_CHECK();
    return AETH_OK;
}

int aeth_galore_apply_update(aeth_galore_ctx* ctx, int idx, float clip, const float* clip_dev,
                             const aeth_weight_ref* w, aeth_stream_t stream) {
    AETH_TRY(check_idx(ctx, idx));
    DeviceGuard g(ctx->device);
    Param& p = ctx->params[idx];
    cudaStream_t st = to_stream(stream);
    if (w && w->kind != AETH_WEIGHT_NONE && !w->data) return set_err(AETH_ERR_ARG);
    if (w && w->kind == AETH_WEIGHT_NF4 && !w->absmax) return set_err(AETH_ERR_ARG);
    if (ctx->cfg.mode == AETH_MODE_REF) return set_err(ref_apply(ctx, p, clip, clip_dev, w, st));
    return set_err(b2_apply(ctx, p, clip, clip_dev, w, 0, st));
}

int aeth_galore_zero_accum(aeth_galore_ctx* ctx, int idx, aeth_stream_t stream) {
    AETH_TRY(check_idx(ctx, idx));
    DeviceGuard g(ctx->device);
    Param& p = ctx->params[idx];
    AETH_CUDA(cudaMemsetAsync(p.accum, 0, p.state_elems * sizeof(float), to_stream(stream)));
    return AETH_OK;
}

int aeth_galore_notify_step(aeth_galore_ctx* ctx, uint64_t step) {
    if (!ctx) return set_err(AETH_ERR_ARG);
    DeviceGuard g(ctx->device);
    AETH_TRY(set_err(notify_step_on(ctx, step, cudaStreamLegacy)));
    AETH_CUDA(cudaStreamSynchronize(cudaStreamLegacy));
    return AETH_OK;
}

int aeth_galore_notify_step_async(aeth_galore_ctx* ctx, uint64_t step, aeth_stream_t stream) {
    if (!ctx) return set_err(AETH_ERR_ARG);
    DeviceGuard g(ctx->device);
    return set_err(notify_step_on(ctx, step, to_stream(stream)));
}

uint64_t aeth_galore_version(const aeth_galore_ctx* ctx) { return ctx ? ctx->version : 0; }

}  // extern "C"

// ---------------------------------------------------------------------------
// optimizer_states.bin (state_file.h): REF mode writes and reads version 2
// byte for byte as the reference; B200 mode writes version 3.
// ---------------------------------------------------------------------------
namespace {

template <class T>
int d2h(std::vector<T>& h, const void* d, size_t count, cudaStream_t st) {
    h.resize(count);
    AETH_CUDA(cudaMemcpyAsync(h.data(), d, count * sizeof(T), cudaMemcpyDeviceToHost, st));
    return AETH_OK;
}

struct FileCloser {
    FILE* f = nullptr;
    ~FileCloser() {
        if (f) fclose(f);
    }
};

}  // namespace

extern "C" {

int aeth_galore_save_state(aeth_galore_ctx* ctx, const char* path, aeth_stream_t stream) {
    if (!ctx || !path) return set_err(AETH_ERR_ARG);
    DeviceGuard g(ctx->device);
    cudaStream_t st = to_stream(stream);
    const bool ref = ctx->cfg.mode == AETH_MODE_REF;
    const uint32_t nl = (uint32_t)ctx->params.size();
    StateHeader h;
    h.version = ref ? 2 : 3;
    h.num_layers = nl;
    h.rank = nl ? (uint32_t)ctx->params[0].r : 16u;
    h.beta1 = ctx->cfg.beta1;
    h.beta2 = ctx->cfg.beta2;
    h.eps = ctx->cfg.eps;
    h.step_count = ctx->step;
    const uint32_t dsz = ref ? kStateDescV2 : kStateDescV3;
    std::vector<StateDesc> descs(nl);
    uint64_t off = kStateHeaderSize + (uint64_t)nl * dsz;
    for (uint32_t i = 0; i < nl; ++i) {
        const Param& p = ctx->params[i];
        StateDesc& d = descs[i];
        d.m = (uint32_t)p.m;
        d.n = (uint32_t)p.n;
        d.rank = (uint32_t)p.r;
        d.side = (uint32_t)p.side;
        d.codec = (uint32_t)ctx->cfg.state_codec;
        d.block = (uint32_t)ctx->cfg.state_block;
        d.state_elems = (uint64_t)p.state_elems;
        d.byte_offset = off;
        const uint64_t s = p.side == 1 ? p.m : p.n;
        off += ref ? state_section_v2(p.m, p.n, p.r) : state_section_v3(s, p.r, p.state_elems, p.state_blocks);
    }
    h.total_size = off;
    std::vector<uint8_t> head(kStateHeaderSize + (size_t)nl * dsz, 0);
    encode_state_header(h, head);
    for (uint32_t i = 0; i < nl; ++i) {
        const size_t b = kStateHeaderSize + (size_t)i * dsz;
        const StateDesc& d = descs[i];
        if (ref) {
            put_le(head, b, d.m);
            put_le(head, b + 4, d.n);
            put_le(head, b + 8, d.rank);
            put_le(head, b + 12, d.byte_offset);
        } else {
            put_le(head, b, d.m);
            put_le(head, b + 4, d.n);
            put_le(head, b + 8, d.rank);
            put_le(head, b + 12, d.side);
            put_le(head, b + 16, d.codec);
            put_le(head, b + 20, d.block);
            put_le(head, b + 24, d.state_elems);
            put_le(head, b + 32, d.byte_offset);
        }
    }
    FileCloser fc;
    fc.f = fopen(path, "wb");
    if (!fc.f) return set_err(AETH_ERR_CONFIG);
    if (fwrite(head.data(), 1, head.size(), fc.f) != head.size()) return set_err(AETH_ERR_CONFIG);
    std::vector<float> pf, qf, ms, vs;
    std::vector<uint16_t> pb;
    std::vector<int8_t> m8, v8;
    for (uint32_t i = 0; i < nl; ++i) {
        const Param& p = ctx->params[i];
        std::vector<uint8_t> sec;
        if (ref) {
            AETH_TRY(d2h(pf, p.P, (size_t)p.m * p.r, st));
            AETH_TRY(d2h(qf, p.Q, (size_t)p.n * p.r, st));
        } else {
            AETH_TRY(d2h(pb, p.proj, (size_t)(p.side == 1 ? p.m : p.n) * p.r, st));
        }
        AETH_TRY(d2h(m8, p.m8, (size_t)p.state_elems, st));
        AETH_TRY(d2h(v8, p.v8, (size_t)p.state_elems, st));
        AETH_TRY(d2h(ms, p.mscale, (size_t)p.state_blocks, st));
        AETH_TRY(d2h(vs, p.vscale, (size_t)p.state_blocks, st));
        AETH_CUDA(cudaStreamSynchronize(st));
        if (ref) {
            // P f16, Q f16, momentum, variance, scale_m, scale_v (state_file.rs:484-527)
            std::vector<uint16_t> ph(pf.size()), qh(qf.size());
            for (size_t k = 0; k < pf.size(); ++k) ph[k] = galore_f32_to_f16(pf[k]);
            for (size_t k = 0; k < qf.size(); ++k) qh[k] = galore_f32_to_f16(qf[k]);
            bool ok = fwrite(ph.data(), 2, ph.size(), fc.f) == ph.size() && fwrite(qh.data(), 2, qh.size(), fc.f) == qh.size();
            ok = ok && fwrite(m8.data(), 1, m8.size(), fc.f) == m8.size() && fwrite(v8.data(), 1, v8.size(), fc.f) == v8.size();
            ok = ok && fwrite(ms.data(), 4, 1, fc.f) == 1 && fwrite(vs.data(), 4, 1, fc.f) == 1;
            if (!ok) return set_err(AETH_ERR_CONFIG);
        } else {
            bool ok = fwrite(pb.data(), 2, pb.size(), fc.f) == pb.size();
            ok = ok && fwrite(m8.data(), 1, m8.size(), fc.f) == m8.size() && fwrite(v8.data(), 1, v8.size(), fc.f) == v8.size();
            ok = ok && fwrite(ms.data(), 4, ms.size(), fc.f) == ms.size() && fwrite(vs.data(), 4, vs.size(), fc.f) == vs.size();
            if (!ok) return set_err(AETH_ERR_CONFIG);
        }
    }
    if (fflush(fc.f) != 0) return set_err(AETH_ERR_CONFIG);
    return AETH_OK;
}

int aeth_galore_load_state(aeth_galore_ctx* ctx, const char* path, aeth_stream_t stream) {
    if (!ctx || !path) return set_err(AETH_ERR_ARG);
    DeviceGuard g(ctx->device);
    cudaStream_t st = to_stream(stream);
    const bool ref = ctx->cfg.mode == AETH_MODE_REF;
    std::vector<uint8_t> buf;
    {
        FileCloser fc;
        fc.f = fopen(path, "rb");
        if (!fc.f) return set_err(AETH_ERR_NOT_FOUND);
        if (fseek(fc.f, 0, SEEK_END) != 0) return set_err(AETH_ERR_CONFIG);
        const long len = ftell(fc.f);
        if (len < (long)kStateHeaderSize || fseek(fc.f, 0, SEEK_SET) != 0) return set_err(AETH_ERR_CONFIG);
        buf.resize((size_t)len);
        if (fread(buf.data(), 1, buf.size(), fc.f) != buf.size()) return set_err(AETH_ERR_CONFIG);
    }
    const StateHeader h = decode_state_header(buf.data());
    // version 1 files (16-byte descriptors, no hyperparameters) read as the reference does
    const bool v1 = h.version < 2;
    if (h.magic != kStateMagic || (ref ? h.version > 2 : h.version != 3)) return set_err(AETH_ERR_CONFIG);
    const uint32_t nl = (uint32_t)ctx->params.size();
    if (h.num_layers != nl) return set_err(AETH_ERR_SHAPE);
    const uint32_t dsz = ref ? (v1 ? 16u : kStateDescV2) : kStateDescV3;
    if (buf.size() < kStateHeaderSize + (size_t)nl * dsz) return set_err(AETH_ERR_CONFIG);
    std::vector<StateDesc> descs(nl);
    for (uint32_t i = 0; i < nl; ++i) {
        const uint8_t* b = buf.data() + kStateHeaderSize + (size_t)i * dsz;
        StateDesc& d = descs[i];
        d.m = get_le<uint32_t>(b);
        d.n = get_le<uint32_t>(b + 4);
        if (ref) {
            d.rank = v1 ? h.rank : get_le<uint32_t>(b + 8);
            d.byte_offset = get_le<uint64_t>(b + (v1 ? 8 : 12));
        } else {
            d.rank = get_le<uint32_t>(b + 8);
            d.side = get_le<uint32_t>(b + 12);
            d.codec = get_le<uint32_t>(b + 16);
            d.block = get_le<uint32_t>(b + 20);
            d.state_elems = get_le<uint64_t>(b + 24);
            d.byte_offset = get_le<uint64_t>(b + 32);
        }
        const Param& p = ctx->params[i];
        if (d.m != (uint32_t)p.m || d.n != (uint32_t)p.n || d.rank != (uint32_t)p.r) return set_err(AETH_ERR_SHAPE);
        if (!ref && (d.side != (uint32_t)p.side || d.codec != (uint32_t)ctx->cfg.state_codec ||
                     d.block != (uint32_t)ctx->cfg.state_block || d.state_elems != (uint64_t)p.state_elems))
            return set_err(AETH_ERR_SHAPE);
        const uint64_t s = p.side == 1 ? p.m : p.n;
        const uint64_t need = ref ? state_section_v2(p.m, p.n, p.r) : state_section_v3(s, p.r, p.state_elems, p.state_blocks);
        // written so that a byte_offset near 2^64 cannot wrap the sum
        if (d.byte_offset > buf.size() || need > buf.size() - d.byte_offset) return set_err(AETH_ERR_CONFIG);
    }
    // Every descriptor is checked above, before anything is installed, so a
    // malformed file leaves the optimizer as it was.  The sections are then
    // installed layer by layer straight into the live state; a CUDA error
    // during that loop leaves the optimizer state undefined (reload a good
    // file or recreate the optimizer).
    for (uint32_t i = 0; i < nl; ++i) {
        Param& p = ctx->params[i];
        const uint8_t* b = buf.data() + descs[i].byte_offset;
        const size_t elems = (size_t)p.state_elems, blocks = (size_t)p.state_blocks;
        if (ref) {
            std::vector<float> pf((size_t)p.m * p.r), qf((size_t)p.n * p.r);
            for (size_t k = 0; k < pf.size(); ++k) pf[k] = galore_f16_to_f32(get_le<uint16_t>(b + 2 * k));
            b += 2 * pf.size();
            for (size_t k = 0; k < qf.size(); ++k) qf[k] = galore_f16_to_f32(get_le<uint16_t>(b + 2 * k));
            b += 2 * qf.size();
            AETH_CUDA(cudaMemcpyAsync(p.P, pf.data(), pf.size() * 4, cudaMemcpyHostToDevice, st));
            AETH_CUDA(cudaMemcpyAsync(p.Q, qf.data(), qf.size() * 4, cudaMemcpyHostToDevice, st));
            AETH_CUDA(cudaStreamSynchronize(st));  // the host vectors go out of scope
        } else {
            const int s_dim = p.side == 1 ? p.m : p.n;
            std::vector<float> pf((size_t)s_dim * p.r);
            for (size_t k = 0; k < pf.size(); ++k) pf[k] = bf16_bits_to_f32_host(get_le<uint16_t>(b + 2 * k));
            b += 2 * pf.size();
            float* tmp = nullptr;
            AETH_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&tmp), pf.size() * 4, st));
            cudaError_t e = cudaMemcpyAsync(tmp, pf.data(), pf.size() * 4, cudaMemcpyHostToDevice, st);
            if (e == cudaSuccess) {
                proj_to_bf16_kernel<<<grid_for((int64_t)s_dim * p.r, 256), 256, 0, st>>>(tmp, s_dim, p.r, p.proj,
                                                                                          p.projT);
                e = cudaGetLastError();
                if (e == cudaSuccess && sync_projk(p, st) != AETH_OK) e = cudaGetLastError();
            }
            cudaFreeAsync(tmp, st);
            if (e == cudaSuccess) e = cudaStreamSynchronize(st);
            AETH_CUDA(e);
        }
        AETH_CUDA(cudaMemcpyAsync(p.m8, b, elems, cudaMemcpyHostToDevice, st));
        AETH_CUDA(cudaMemcpyAsync(p.v8, b + elems, elems, cudaMemcpyHostToDevice, st));
        AETH_CUDA(cudaMemcpyAsync(p.mscale, b + 2 * elems, blocks * 4, cudaMemcpyHostToDevice, st));
        AETH_CUDA(cudaMemcpyAsync(p.vscale, b + 2 * elems + blocks * 4, blocks * 4, cudaMemcpyHostToDevice, st));
        AETH_CUDA(cudaMemsetAsync(p.accum, 0, (size_t)p.state_elems * sizeof(float), st));  // new grad_accum
        drop_capture(p, st);
    }
    AETH_CUDA(cudaStreamSynchronize(st));  // buf is read by the copies above
    // OptimizerStateFile::open adopts the header's step and Adam constants
    // (optimizer.rs:136-143); version 1 files carry neither.
    ctx->step = v1 ? 0 : h.step_count;
    if (!v1) {
        ctx->cfg.beta1 = h.beta1;
        ctx->cfg.beta2 = h.beta2;
        ctx->cfg.eps = h.eps;
    }
    return AETH_OK;
}

int aeth_randomized_svd(const float* g, int m, int n, int rank, int oversampling, int power_iters, uint64_t seed,
                        float* p_out, float* q_out, aeth_stream_t stream) {
    if (!g || m <= 0 || n <= 0) return set_err(AETH_ERR_ARG);
    return set_err(
        rsvd_device(g, false, m, n, rank, oversampling, power_iters, seed, false, p_out, q_out, to_stream(stream)));
}

int aeth_randomized_svd_ex(const void* g, int g_dtype, int m, int n, int rank, int oversampling, int power_iters,
                           uint64_t seed, int fast, float* p_out, float* q_out, aeth_stream_t stream) {
    if (!g || m <= 0 || n <= 0) return set_err(AETH_ERR_ARG);
    if (g_dtype != AETH_DTYPE_F32 && g_dtype != AETH_DTYPE_BF16) return set_err(AETH_ERR_ARG);
    return set_err(rsvd_device(g, g_dtype == AETH_DTYPE_BF16, m, n, rank, oversampling, power_iters, seed, fast != 0,
                               p_out, q_out, to_stream(stream)));
}

int aeth_randomized_svd_sketch(const void* g, int g_dtype, int m, int n, int rank, int oversampling,
                               const float* omega, int fast, float* p_out, float* q_out, aeth_stream_t stream) {
    if (!g || !omega || m <= 0 || n <= 0) return set_err(AETH_ERR_ARG);
    if (g_dtype != AETH_DTYPE_F32 && g_dtype != AETH_DTYPE_BF16) return set_err(AETH_ERR_ARG);
    return set_err(rsvd_device(g, g_dtype == AETH_DTYPE_BF16, m, n, rank, oversampling, 0, 1, fast != 0, p_out,
                               q_out, to_stream(stream), omega));
}

int aeth_rsvd_omega(uint64_t seed, int64_t count, float* out, aeth_stream_t stream) {
    if (!out || count <= 0) return set_err(AETH_ERR_ARG);
    cudaStream_t st = to_stream(stream);
    uint64_t* jump = nullptr;
    AETH_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&jump), sizeof(uint64_t) * 64 * kOmegaLevels, st));
    cudaError_t e = cudaMemcpyAsync(jump, omega_jump_host(), sizeof(Gf2Mat64) * kOmegaLevels, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) {
        const int64_t chunks = (count + kOmegaChunk - 1) / kOmegaChunk;
        rsvd_omega_kernel<<<(unsigned)((chunks + 255) / 256), 256, 0, st>>>(jump, seed > 1 ? seed : 1, count, out);
        e = cudaGetLastError();
    }
    cudaFreeAsync(jump, st);
    AETH_CUDA(e);
    return AETH_OK;
}

int aeth_rsvd_jacobi(float* mat, int n, float* u, aeth_stream_t stream) {
    if (!mat || !u || n < 1) return set_err(AETH_ERR_ARG);
    if (n > kJacobiMaxN) return set_err(AETH_ERR_UNSUPPORTED);
    jacobi50_kernel<<<1, 1024, 0, to_stream(stream)>>>(mat, n, u);
    AETH_CUDA(cudaGetLastError());
    return AETH_OK;
}

uint64_t aeth_galore_step_count(const aeth_galore_ctx* ctx) { return ctx ? ctx->step : 0; }

}  // extern "C"

namespace {

// Concurrent refreshes of aeth_galore_refresh_layer.
constexpr int kRefreshStreams = 8;

// Phase ids of aeth_galore_phase_times.
enum { PH_PROJ = 0, PH_NORM = 1, PH_ADAM = 2, PH_APPLY = 3 };

int check_list(const aeth_galore_ctx* ctx, int n, const int* idx) {
    if (!ctx || n <= 0 || !idx) return AETH_ERR_ARG;
    if (n > (int)ctx->params.size()) return AETH_ERR_ARG;
    for (int i = 0; i < n; ++i) AETH_TRY(check_idx(ctx, idx[i]));
    return AETH_OK;
}

int stream_capturing(cudaStream_t st, bool* capturing) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    AETH_CUDA(cudaStreamIsCapturing(st, &cap));
    *capturing = cap != cudaStreamCaptureStatusNone;
    return AETH_OK;
}

// project_and_accumulate for every listed parameter (backward.rs:509-521).
// B200 mode: grouped launches, one per rank value (column slices of 256 above
// rank 256), the per-tile kernel for shapes the grouped kernel does not take.
int project_group(aeth_galore_ctx* ctx, int n, const int* idx, const void* const* grads, int grad_dtype,
                  cudaStream_t st) {
    for (int i = 0; i < n; ++i) AETH_TRY(capture_if_due(ctx, ctx->params[idx[i]], grads[i], grad_dtype, st));
    if (ctx->cfg.mode == AETH_MODE_REF) {
        for (int i = 0; i < n; ++i) AETH_TRY(ref_project_accumulate(ctx, ctx->params[idx[i]], grads[i], grad_dtype, st));
        return AETH_OK;
    }
    if (grad_dtype != AETH_DTYPE_BF16) {
        // fp32 / f16: each gradient's bf16 terms go through the one staging
        // buffer, so the parameters are projected one after another
        for (int i = 0; i < n; ++i)
            AETH_TRY(b2_project_accumulate(ctx, ctx->params[idx[i]], grads[i], grad_dtype, st));
        return AETH_OK;
    }
    std::vector<ProjJob> jobs;
    std::vector<int> ranks;
    std::vector<char> small(n, 0);
    for (int i = 0; i < n; ++i) {
        Param& p = ctx->params[idx[i]];
        small[i] = !b2_tma_shape(p) || (reinterpret_cast<uintptr_t>(grads[i]) & 15) != 0;
        if (small[i]) {
            AETH_TRY(b2_project_small(p, grads[i], grad_dtype, st));
        } else if (std::find(ranks.begin(), ranks.end(), p.r) == ranks.end()) {
            ranks.push_back(p.r);
        }
        jobs.push_back(ProjJob{grads[i], p.projT, p.accum, p.m, p.n});
    }
    for (int r : ranks) {
        std::vector<ProjJob> grp;
        std::vector<int> members;
        for (int i = 0; i < n; ++i)
            if (!small[i] && ctx->params[idx[i]].r == r) { grp.push_back(jobs[i]); members.push_back(i); }
        int s = proj_grouped_launch(grp.data(), (int)grp.size(), r, st);
        if (s == AETH_ERR_UNSUPPORTED) {
            for (int i : members) AETH_TRY(b2_project_tile(ctx->params[idx[i]], jobs[i], st));
        } else if (s != AETH_OK) {
            return s;
        }
    }
    return AETH_OK;
}

// The rest of deferred_apply_with_clip (hook.rs:139-203) for the listed
// parameters: squared norms and the exact global clip, then apply_update and
// zero_accum for each.  Marks the phase boundaries in pm.
int finish_group(aeth_galore_ctx* ctx, int n, const int* idx, const aeth_weight_ref* weights, aeth_sqnorm_hook sq_hook,
                 void* hook_user, float* clip, aeth_stream_t stream, PhaseMarks& pm) {
    cudaStream_t st = to_stream(stream);
    if (ctx->cfg.mode == AETH_MODE_REF) {
        // A6 pass 1: squared norms (hook.rs:149-182).
        for (int i = 0; i < n; ++i) AETH_TRY(sqnorm_into(ctx, ctx->params[idx[i]], ctx->sq_step + i, st));
        if (sq_hook) AETH_TRY(sq_hook(ctx->sq_step, n, stream, hook_user));
        clip_coeff_kernel<<<1, 32, 0, st>>>(ctx->sq_step, n, ctx->cfg.max_grad_norm, clip, ctx->gnorm_dev);
        AETH_LAUNCH_CHECK();
        AETH_TRY(pm.mark(st, PH_APPLY));
        // A6 pass 2: apply_update + zero_accum (hook.rs:190-194).
        for (int i = 0; i < n; ++i) {
            Param& p = ctx->params[idx[i]];
            AETH_TRY(ref_apply(ctx, p, 1.0f, clip, weights ? &weights[i] : nullptr, st));
            AETH_CUDA(cudaMemsetAsync(p.accum, 0, p.state_elems * sizeof(float), st));
        }
        return AETH_OK;
    }
    std::vector<const float*> xs(n);
    std::vector<int64_t> ns(n);
    for (int i = 0; i < n; ++i) { xs[i] = ctx->params[idx[i]].accum; ns[i] = ctx->params[idx[i]].state_elems; }
    // Without a hook the norms and the clip coefficient come from one launch.
    // With a clip group the same launch also exchanges the sum with the peers.
    const bool grouped = ctx->group.world > 1;
    if (grouped && sq_hook) return AETH_ERR_ARG;
    if (grouped && n > kSqGroupMax) return AETH_ERR_UNSUPPORTED;
    const bool fuse_clip = !sq_hook && n <= kSqGroupMax;
    AETH_TRY(sqnorm_group(xs.data(), ns.data(), n, ctx->sq_step, ctx->partials, ctx->sq_ticket,
                          ctx->cfg.max_grad_norm, fuse_clip ? clip : nullptr, fuse_clip ? ctx->gnorm_dev : nullptr,
                          st, grouped ? &ctx->group : nullptr));
    if (!fuse_clip) {
        if (sq_hook) AETH_TRY(sq_hook(ctx->sq_step, n, stream, hook_user));
        clip_coeff_kernel<<<1, 32, 0, st>>>(ctx->sq_step, n, ctx->cfg.max_grad_norm, clip, ctx->gnorm_dev);
        AETH_LAUNCH_CHECK();
    }
    AETH_TRY(pm.mark(st, PH_ADAM));
    {
        std::vector<Param*> ps(n);
        for (int i = 0; i < n; ++i) ps[i] = &ctx->params[idx[i]];
        AETH_TRY(b2_adam_group(ctx, ps.data(), n, 1.0f, clip, 1, st));
    }
    AETH_TRY(pm.mark(st, PH_APPLY));
    std::vector<int> ranks;
    for (int i = 0; i < n; ++i)
        if (std::find(ranks.begin(), ranks.end(), ctx->params[idx[i]].r) == ranks.end())
            ranks.push_back(ctx->params[idx[i]].r);
    for (int r : ranks) {
        std::vector<ApplyJob> grp;
        for (int i = 0; i < n; ++i) {
            Param& p = ctx->params[idx[i]];
            if (p.r != r) continue;
            const aeth_weight_ref* w = weights ? &weights[i] : nullptr;
            ApplyJob job;
            if (b2_apply_job(ctx->cfg, p, w, &job)) grp.push_back(job);
            else AETH_TRY(b2_weight_tile(ctx, p, w, st));
        }
        if (!grp.empty()) AETH_TRY(apply_grouped_launch(grp.data(), (int)grp.size(), r, st));
    }
    return AETH_OK;
}

int check_weights(int n, const aeth_weight_ref* weights) {
    if (!weights) return AETH_OK;
    for (int i = 0; i < n; ++i) {
        const aeth_weight_ref& w = weights[i];
        if (w.kind != AETH_WEIGHT_NONE && !w.data) return AETH_ERR_ARG;
        if (w.kind == AETH_WEIGHT_NF4 && !w.absmax) return AETH_ERR_ARG;
    }
    return AETH_OK;
}

}  // namespace

extern "C" {

int aeth_galore_step(aeth_galore_ctx* ctx, int n, const int* idx, const void* const* grads, int grad_dtype,
                     const aeth_weight_ref* weights, aeth_sqnorm_hook sq_hook, void* hook_user, float* clip_dev_out,
                     aeth_stream_t stream) {
    AETH_TRY(set_err(check_list(ctx, n, idx)));
    if (!grads) return set_err(AETH_ERR_ARG);
    AETH_TRY(set_err(check_weights(n, weights)));
    DeviceGuard g(ctx->device);
    cudaStream_t st = to_stream(stream);
    float* clip = clip_dev_out ? clip_dev_out : ctx->clip_dev;
    // Under CUDA graph capture the step records only kernels: no phase events,
    // and no gradient capture for a subspace refresh, whose schedule depends on
    // the host step count that a replayed graph cannot follow.
    bool capturing = false;
    AETH_TRY(set_err(stream_capturing(st, &capturing)));
    if (capturing && ctx->cfg.svd_refresh) return set_err(AETH_ERR_UNSUPPORTED);
    PhaseMarks pm;
    if (!capturing) AETH_TRY(pm.begin(ctx));
    AETH_TRY(pm.mark(st, PH_PROJ));
    AETH_TRY(set_err(project_group(ctx, n, idx, grads, grad_dtype, st)));
    AETH_TRY(pm.mark(st, PH_NORM));
    AETH_TRY(set_err(finish_group(ctx, n, idx, weights, sq_hook, hook_user, clip, stream, pm)));
    AETH_TRY(pm.mark(st, -1));
    pm.commit(1);
    return AETH_OK;
}

int aeth_galore_project_layer(aeth_galore_ctx* ctx, int n, const int* idx, const void* const* grads,
                              int grad_dtype, aeth_stream_t stream) {
    AETH_TRY(set_err(check_list(ctx, n, idx)));
    if (!grads) return set_err(AETH_ERR_ARG);
    for (int i = 0; i < n; ++i)
        if (!grads[i]) return set_err(AETH_ERR_ARG);
    DeviceGuard g(ctx->device);
    cudaStream_t st = to_stream(stream);
    bool capturing = false;
    AETH_TRY(set_err(stream_capturing(st, &capturing)));
    if (capturing && ctx->cfg.svd_refresh) return set_err(AETH_ERR_UNSUPPORTED);
    PhaseMarks pm;
    if (!capturing) AETH_TRY(pm.begin(ctx));
    AETH_TRY(pm.mark(st, PH_PROJ));
    AETH_TRY(set_err(project_group(ctx, n, idx, grads, grad_dtype, st)));
    AETH_TRY(pm.mark(st, -1));
    pm.commit(0);
    return AETH_OK;
}

int aeth_galore_refresh_layer(aeth_galore_ctx* ctx, int n, const int* idx, const void* const* grads,
                              int grad_dtype, aeth_stream_t stream) {
    AETH_TRY(set_err(check_list(ctx, n, idx)));
    if (!grads) return set_err(AETH_ERR_ARG);
    if (ctx->cfg.mode != AETH_MODE_B200) return set_err(AETH_ERR_CONFIG);
    if (grad_dtype != AETH_DTYPE_F32 && grad_dtype != AETH_DTYPE_F16 && grad_dtype != AETH_DTYPE_BF16)
        return set_err(AETH_ERR_ARG);
    for (int i = 0; i < n; ++i)
        if (!grads[i]) return set_err(AETH_ERR_ARG);
    DeviceGuard g(ctx->device);
    cudaStream_t st = to_stream(stream);
    bool capturing = false;
    AETH_TRY(set_err(stream_capturing(st, &capturing)));
    if (capturing) return set_err(AETH_ERR_UNSUPPORTED);
    for (int i = 0; i < n; ++i) {
        Param& p = ctx->params[idx[i]];
        if (!p.pend_proj) {
            const int64_t pe = (int64_t)(p.side == 1 ? p.m : p.n) * p.r;
            AETH_TRY(set_err(ctx_alloc(ctx, &p.pend_proj, pe)));
            AETH_TRY(set_err(ctx_alloc(ctx, &p.pend_projT, pe)));
        }
    }
    // The parameters' refreshes run concurrently on the optimizer's side
    // streams (their factorisations are one-CTA kernels that overlap the
    // others' GEMMs), forked from and joined back into `stream`; one wait at
    // the end reads every status.
    if (ctx->side_streams.empty()) {
        for (int k = 0; k < kRefreshStreams; ++k) {
            cudaStream_t s = nullptr;
            AETH_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
            ctx->side_streams.push_back(s);
        }
    }
    int* flags = nullptr;
    AETH_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&flags), sizeof(int) * (size_t)n, st));
    int status = AETH_OK;
    cudaEvent_t fork = nullptr;
    std::vector<cudaEvent_t> joins;
    cudaError_t e = cudaMemsetAsync(flags, 0, sizeof(int) * (size_t)n, st);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&fork, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventRecord(fork, st);
    if (e != cudaSuccess) status = (int)e;
    const int nside = std::min<int>(kRefreshStreams, n);
    for (int k = 0; k < nside && status == AETH_OK; ++k) {
        e = cudaStreamWaitEvent(ctx->side_streams[k], fork, 0);
        if (e != cudaSuccess) status = (int)e;
    }
    for (int i = 0; i < n && status == AETH_OK; ++i)
        status = refresh_enqueue(ctx, ctx->params[idx[i]], grads[i], grad_dtype, flags + i,
                                 ctx->side_streams[i % nside]);
    for (int k = 0; k < nside; ++k) {
        cudaEvent_t j = nullptr;
        if (cudaEventCreateWithFlags(&j, cudaEventDisableTiming) != cudaSuccess) continue;
        cudaEventRecord(j, ctx->side_streams[k]);
        cudaStreamWaitEvent(st, j, 0);
        joins.push_back(j);
    }
    std::vector<int> h((size_t)n, 0);
    e = cudaMemcpyAsync(h.data(), flags, sizeof(int) * (size_t)n, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (status == AETH_OK && e != cudaSuccess) status = (int)e;
    cudaFreeAsync(flags, st);
    if (fork) cudaEventDestroy(fork);
    for (cudaEvent_t j : joins) cudaEventDestroy(j);
    if (status != AETH_OK) return set_err(status);
    for (int i = 0; i < n; ++i) {
        if (h[i]) status = AETH_ERR_LINALG;  // the reference drops such a refresh with an error
        else ctx->params[idx[i]].pending = true;
    }
    return set_err(status);
}

int aeth_galore_projector_buffer(aeth_galore_ctx* ctx, int idx, void** proj_bf16, int* rows, int* cols) {
    AETH_TRY(check_idx(ctx, idx));
    if (!proj_bf16 || ctx->cfg.mode != AETH_MODE_B200) return set_err(AETH_ERR_ARG);
    const Param& p = ctx->params[idx];
    *proj_bf16 = p.proj;
    if (rows) *rows = p.side == 1 ? p.m : p.n;
    if (cols) *cols = p.r;
    return AETH_OK;
}

int aeth_galore_finish_step(aeth_galore_ctx* ctx, int n, const int* idx, const aeth_weight_ref* weights,
                            aeth_sqnorm_hook sq_hook, void* hook_user, float* clip_dev_out, aeth_stream_t stream) {
    AETH_TRY(set_err(check_list(ctx, n, idx)));
    AETH_TRY(set_err(check_weights(n, weights)));
    DeviceGuard g(ctx->device);
    cudaStream_t st = to_stream(stream);
    float* clip = clip_dev_out ? clip_dev_out : ctx->clip_dev;
    bool capturing = false;
    AETH_TRY(set_err(stream_capturing(st, &capturing)));
    PhaseMarks pm;
    if (!capturing) AETH_TRY(pm.begin(ctx));
    AETH_TRY(pm.mark(st, PH_NORM));
    AETH_TRY(set_err(finish_group(ctx, n, idx, weights, sq_hook, hook_user, clip, stream, pm)));
    AETH_TRY(pm.mark(st, -1));
    pm.commit(1);
    return AETH_OK;
}

int aeth_galore_clip_handle(aeth_galore_ctx* ctx, int world, void* handle_out) {
    if (!ctx || !handle_out || world < 1 || world > kClipGroupMax) return set_err(AETH_ERR_ARG);
    DeviceGuard g(ctx->device);
    if (ctx->own_slots && ctx->own_slots_world != world) {
        if (ctx->group.world > 1) return set_err(AETH_ERR_CONFIG);  // in use
        cudaFree(ctx->own_slots);
        ctx->own_slots = nullptr;
    }
    if (!ctx->own_slots) {
        const size_t bytes = sizeof(PeerSlot) * 2 * (size_t)world;
        AETH_CUDA(cudaMalloc(reinterpret_cast<void**>(&ctx->own_slots), bytes));
        ctx->own_slots_world = world;
        AETH_CUDA(cudaMemset(ctx->own_slots, 0, bytes));
        AETH_CUDA(cudaDeviceSynchronize());
    }
    cudaIpcMemHandle_t h;
    AETH_CUDA(cudaIpcGetMemHandle(&h, ctx->own_slots));
    memcpy(handle_out, &h, sizeof(h));
    return AETH_OK;
}

int aeth_galore_set_clip_group(aeth_galore_ctx* ctx, int rank, int world, const void* handles, uint64_t timeout_ns) {
    if (!ctx || world < 1 || world > kClipGroupMax || rank < 0 || rank >= world) return set_err(AETH_ERR_ARG);
    if (ctx->cfg.mode != AETH_MODE_B200) return set_err(AETH_ERR_UNSUPPORTED);
    DeviceGuard g(ctx->device);
    for (void* m : ctx->peer_maps) cudaIpcCloseMemHandle(m);
    for (cudaStream_t s : ctx->side_streams) cudaStreamDestroy(s);
    ctx->peer_maps.clear();
    ctx->group = ClipGroup();
    if (world == 1) return AETH_OK;
    if (!handles || !ctx->own_slots || ctx->own_slots_world != world) return set_err(AETH_ERR_CONFIG);
    // fresh slots: epochs restart at 1 (the ranks meet at a barrier after this)
    AETH_CUDA(cudaMemset(ctx->own_slots, 0, sizeof(PeerSlot) * 2 * (size_t)world));
    AETH_CUDA(cudaMemset(ctx->clip_epoch, 0, sizeof(uint64_t)));
    AETH_CUDA(cudaDeviceSynchronize());
    ClipGroup grp;
    grp.rank = rank;
    grp.world = world;
    grp.epoch = ctx->clip_epoch;
    grp.timeout_ns = timeout_ns ? timeout_ns : kWaitLimitNs;
    for (int p = 0; p < world; ++p) {
        if (p == rank) {
            grp.slots[p] = ctx->own_slots;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)p * sizeof(h), sizeof(h));
        void* ptr = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (void* m : ctx->peer_maps) cudaIpcCloseMemHandle(m);
    for (cudaStream_t s : ctx->side_streams) cudaStreamDestroy(s);
            ctx->peer_maps.clear();
            return set_err((int)e);
        }
        ctx->peer_maps.push_back(ptr);
        grp.slots[p] = static_cast<PeerSlot*>(ptr);
    }
    ctx->group = grp;
    return AETH_OK;
}

int aeth_galore_set_clip_group_ptrs(aeth_galore_ctx* ctx, int rank, int world, void* const* slots,
                                    uint64_t timeout_ns) {
    if (!ctx || world < 2 || world > kClipGroupMax || rank < 0 || rank >= world || !slots) return set_err(AETH_ERR_ARG);
    if (ctx->cfg.mode != AETH_MODE_B200) return set_err(AETH_ERR_UNSUPPORTED);
    if (!ctx->own_slots || ctx->own_slots_world != world || slots[rank] != ctx->own_slots)
        return set_err(AETH_ERR_CONFIG);
    for (int p = 0; p < world; ++p)
        if (!slots[p]) return set_err(AETH_ERR_ARG);
    DeviceGuard g(ctx->device);
    for (void* m : ctx->peer_maps) cudaIpcCloseMemHandle(m);
    for (cudaStream_t s : ctx->side_streams) cudaStreamDestroy(s);
    ctx->peer_maps.clear();
    ctx->group = ClipGroup();
    AETH_CUDA(cudaMemset(ctx->own_slots, 0, sizeof(PeerSlot) * 2 * (size_t)world));
    AETH_CUDA(cudaMemset(ctx->clip_epoch, 0, sizeof(uint64_t)));
    AETH_CUDA(cudaDeviceSynchronize());
    ClipGroup grp;
    grp.rank = rank;
    grp.world = world;
    grp.epoch = ctx->clip_epoch;
    grp.timeout_ns = timeout_ns ? timeout_ns : kWaitLimitNs;
    for (int p = 0; p < world; ++p) grp.slots[p] = static_cast<PeerSlot*>(slots[p]);
    ctx->group = grp;
    return AETH_OK;
}

int aeth_galore_clip_slots(aeth_galore_ctx* ctx, void** slots_out) {
    if (!ctx || !slots_out) return set_err(AETH_ERR_ARG);
    *slots_out = ctx->own_slots;
    return ctx->own_slots ? AETH_OK : set_err(AETH_ERR_CONFIG);
}

int aeth_galore_set_phase_timing(aeth_galore_ctx* ctx, int enable) {
    if (!ctx) return set_err(AETH_ERR_ARG);
    ctx->phase_timing = enable != 0;
    return AETH_OK;
}

int aeth_galore_phase_times(aeth_galore_ctx* ctx, double ms_out[4], int* steps) {
    if (!ctx || !ms_out) return set_err(AETH_ERR_ARG);
    DeviceGuard g(ctx->device);
    for (int k = 0; k < 4; ++k) ms_out[k] = 0.0;
    int done = 0;
    int status = AETH_OK;
    for (auto& rec : ctx->phase_pending) {
        if (status == AETH_OK && !rec.ev.empty()) {
            cudaError_t e = cudaEventSynchronize(rec.ev.back());
            for (size_t k = 0; k + 1 < rec.ev.size() && e == cudaSuccess; ++k) {
                float ms = 0.0f;
                e = cudaEventElapsedTime(&ms, rec.ev[k], rec.ev[k + 1]);
                if (rec.phase[k] >= 0 && rec.phase[k] < 4) ms_out[rec.phase[k]] += ms;
            }
            if (e != cudaSuccess) status = set_err((int)e);
            else done += rec.steps;
        }
        for (cudaEvent_t e : rec.ev) ctx->event_pool.push_back(e);
    }
    ctx->phase_pending.clear();
    if (steps) *steps = done;
    return status;
}

int aeth_galore_set_projector(aeth_galore_ctx* ctx, int idx, const float* P, const float* Q, aeth_stream_t stream) {
    AETH_TRY(check_idx(ctx, idx));
    DeviceGuard g(ctx->device);
    Param& p = ctx->params[idx];
    cudaStream_t st = to_stream(stream);
    if (ctx->cfg.mode == AETH_MODE_REF) {
        if (!P || !Q) return set_err(AETH_ERR_ARG);
        AETH_CUDA(cudaMemcpyAsync(p.P, P, (size_t)p.m * p.r * 4, cudaMemcpyDeviceToDevice, st));
        AETH_CUDA(cudaMemcpyAsync(p.Q, Q, (size_t)p.n * p.r * 4, cudaMemcpyDeviceToDevice, st));
    } else {
        const float* src = p.side == 1 ? P : Q;
        if (!src) return set_err(AETH_ERR_ARG);
        const int s_dim = p.side == 1 ? p.m : p.n;
        proj_to_bf16_kernel<<<grid_for((int64_t)s_dim * p.r, 256), 256, 0, st>>>(src, s_dim, p.r, p.proj, p.projT);
        AETH_LAUNCH_CHECK();
        AETH_TRY(set_err(sync_projk(p, st)));
    }
    // Subspace switch resets the Adam state (optimizer.rs:236-238).
    return set_err(reset_state(ctx, p, st));
}

int aeth_galore_get_projector(aeth_galore_ctx* ctx, int idx, float* P, float* Q, aeth_stream_t stream) {
    AETH_TRY(check_idx(ctx, idx));
    DeviceGuard g(ctx->device);
    Param& p = ctx->params[idx];
    cudaStream_t st = to_stream(stream);
    if (ctx->cfg.mode == AETH_MODE_REF) {
        if (P) AETH_CUDA(cudaMemcpyAsync(P, p.P, (size_t)p.m * p.r * 4, cudaMemcpyDeviceToDevice, st));
        if (Q) AETH_CUDA(cudaMemcpyAsync(Q, p.Q, (size_t)p.n * p.r * 4, cudaMemcpyDeviceToDevice, st));
    } else {
        float* dst = p.side == 1 ? P : Q;
        const int s_dim = p.side == 1 ? p.m : p.n;
        if (dst) {
            bf16_to_f32_kernel<<<grid_for((int64_t)s_dim * p.r, 256), 256, 0, st>>>(p.proj, (int64_t)s_dim * p.r, dst);
            AETH_LAUNCH_CHECK();
        }
    }
    return AETH_OK;
}

int aeth_galore_get_state(aeth_galore_ctx* ctx, int idx, int8_t* m8, int8_t* v8, float* m_scales, float* v_scales,
                          aeth_stream_t stream) {
    AETH_TRY(check_idx(ctx, idx));
    DeviceGuard g(ctx->device);
    Param& p = ctx->params[idx];
    cudaStream_t st = to_stream(stream);
    if (m8) AETH_CUDA(cudaMemcpyAsync(m8, p.m8, p.state_elems, cudaMemcpyDeviceToDevice, st));
    if (v8) AETH_CUDA(cudaMemcpyAsync(v8, p.v8, p.state_elems, cudaMemcpyDeviceToDevice, st));
    if (m_scales) AETH_CUDA(cudaMemcpyAsync(m_scales, p.mscale, p.state_blocks * 4, cudaMemcpyDeviceToDevice, st));
    if (v_scales) AETH_CUDA(cudaMemcpyAsync(v_scales, p.vscale, p.state_blocks * 4, cudaMemcpyDeviceToDevice, st));
    return AETH_OK;
}

int aeth_galore_set_state(aeth_galore_ctx* ctx, int idx, const int8_t* m8, const int8_t* v8, const float* m_scales,
                          const float* v_scales, aeth_stream_t stream) {
    AETH_TRY(check_idx(ctx, idx));
    DeviceGuard g(ctx->device);
    Param& p = ctx->params[idx];
    cudaStream_t st = to_stream(stream);
    if (m8) AETH_CUDA(cudaMemcpyAsync(p.m8, m8, p.state_elems, cudaMemcpyDeviceToDevice, st));
    if (v8) AETH_CUDA(cudaMemcpyAsync(p.v8, v8, p.state_elems, cudaMemcpyDeviceToDevice, st));
    if (m_scales) AETH_CUDA(cudaMemcpyAsync(p.mscale, m_scales, p.state_blocks * 4, cudaMemcpyDeviceToDevice, st));
    if (v_scales) AETH_CUDA(cudaMemcpyAsync(p.vscale, v_scales, p.state_blocks * 4, cudaMemcpyDeviceToDevice, st));
    return AETH_OK;
}

int aeth_galore_get_accum(aeth_galore_ctx* ctx, int idx, float* accum, aeth_stream_t stream) {
    AETH_TRY(check_idx(ctx, idx));
    if (!accum) return set_err(AETH_ERR_ARG);
    DeviceGuard g(ctx->device);
    Param& p = ctx->params[idx];
    AETH_CUDA(cudaMemcpyAsync(accum, p.accum, p.state_elems * 4, cudaMemcpyDeviceToDevice, to_stream(stream)));
    return AETH_OK;
}

// ---------------------------------------------------------------------------
// Stand-alone kernels
// ---------------------------------------------------------------------------
int aeth_nf4_dequant(const uint8_t* packed, const float* absmax, int64_t n, int block, void* out, int out_dtype,
                     aeth_stream_t stream) {
    if (!packed || !absmax || !out || n <= 0 || block <= 0) return set_err(AETH_ERR_ARG);
    if (out_dtype < AETH_DTYPE_F32 || out_dtype > AETH_DTYPE_BF16) return set_err(AETH_ERR_ARG);
    cudaStream_t st = to_stream(stream);
    const bool aligned = (reinterpret_cast<uintptr_t>(packed) & 15) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0;
    if (block == 64 && n % 32 == 0 && aligned) {
        int64_t chunks = n / 32;
        int grid = grid_for(chunks, 256, 148 * 8);
        if (out_dtype == AETH_DTYPE_F32)
            nf4_dequant64_kernel<float><<<grid, 256, 0, st>>>(packed, absmax, chunks, static_cast<float*>(out));
        else if (out_dtype == AETH_DTYPE_F16)
            nf4_dequant64_kernel<__half><<<grid, 256, 0, st>>>(packed, absmax, chunks, static_cast<__half*>(out));
        else
            nf4_dequant64_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(packed, absmax, chunks,
                                                                      static_cast<__nv_bfloat16*>(out));
    } else {
        nf4_dequant_generic_kernel<<<grid_for(n, 256), 256, 0, st>>>(packed, absmax, n, block, out, out_dtype);
    }
    AETH_LAUNCH_CHECK();
    return AETH_OK;
}

int aeth_nf4_quant(const void* x, int x_dtype, int64_t n, int block, uint8_t* packed, float* absmax,
                   aeth_stream_t stream) {
    if (!x || !packed || !absmax || n <= 0 || block <= 0) return set_err(AETH_ERR_ARG);
    if (x_dtype < AETH_DTYPE_F32 || x_dtype > AETH_DTYPE_BF16) return set_err(AETH_ERR_ARG);
    cudaStream_t st = to_stream(stream);
    const bool aligned = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(packed) & 7) == 0;
    if (block == 64 && n % 64 == 0 && aligned) {
        int64_t nb = n / 64;
        nf4_quant64_kernel<<<grid_for(nb * 4, 256, 148 * 8), 256, 0, st>>>(x, x_dtype, nb, packed, absmax);
    } else {
        int64_t nb = (n + block - 1) / block;
        nf4_absmax_generic_kernel<<<grid_for(nb * 32, 256), 256, 0, st>>>(x, x_dtype, n, block, nb, absmax);
        nf4_pack_generic_kernel<<<grid_for((n + 1) / 2, 256), 256, 0, st>>>(x, x_dtype, n, block, absmax, packed);
    }
    AETH_LAUNCH_CHECK();
    return AETH_OK;
}

int aeth_int8_quantize(const float* x, int64_t n, int codec, int block, int is_signed, int8_t* q, float* scales,
                       aeth_stream_t stream) {
    if (!x || !q || !scales || n <= 0) return set_err(AETH_ERR_ARG);
    cudaStream_t st = to_stream(stream);
    AETH_TRY(codec_maps_ensure());
    if (codec == AETH_CODEC_PER_TENSOR) {
        AETH_CUDA(cudaMemsetAsync(scales, 0, sizeof(float), st));
        absmax_reduce_kernel<<<grid_for(n, 256, 148 * 4), 256, 0, st>>>(x, n, scales);
        per_tensor_encode_kernel<<<grid_for(n, 256), 256, 0, st>>>(x, n, scales, q);
        per_tensor_finalize_kernel<<<1, 1, 0, st>>>(scales);
    } else if (codec == AETH_CODEC_BLOCK_LINEAR || codec == AETH_CODEC_BLOCK_DYNAMIC) {
        if (block <= 0) return set_err(AETH_ERR_ARG);
        int64_t nb = (n + block - 1) / block;
        block_encode_kernel<<<grid_for(nb, 1, 148 * 8), 256, 0, st>>>(x, n, block, codec, is_signed, q, scales);
    } else {
        return set_err(AETH_ERR_ARG);
    }
    AETH_LAUNCH_CHECK();
    return AETH_OK;
}

int aeth_int8_dequantize(const int8_t* q, const float* scales, int64_t n, int codec, int block, int is_signed,
                         float* out, aeth_stream_t stream) {
    if (!q || !scales || !out || n <= 0) return set_err(AETH_ERR_ARG);
    cudaStream_t st = to_stream(stream);
    AETH_TRY(codec_maps_ensure());
    if (codec == AETH_CODEC_PER_TENSOR) {
        dequant_linear_kernel<<<grid_for(n, 256), 256, 0, st>>>(q, scales, 0.0f, n, 0, out);
    } else if (codec == AETH_CODEC_BLOCK_LINEAR) {
        if (block <= 0) return set_err(AETH_ERR_ARG);
        dequant_linear_kernel<<<grid_for(n, 256), 256, 0, st>>>(q, scales, 0.0f, n, block, out);
    } else if (codec == AETH_CODEC_BLOCK_DYNAMIC) {
        if (block <= 0) return set_err(AETH_ERR_ARG);
        dequant_dynamic_kernel<<<grid_for(n, 256), 256, 0, st>>>(q, scales, n, block, is_signed, out);
    } else {
        return set_err(AETH_ERR_ARG);
    }
    AETH_LAUNCH_CHECK();
    return AETH_OK;
}

int aeth_fc_decode_int8(const int8_t* src, int64_t n, const float* scales, int64_t n_scales, int num_channels,
                        uint16_t* out_f16, aeth_stream_t stream) {
    if (!src || !out_f16 || n < 0 || n_scales < 0 || num_channels < 0 || (n_scales > 0 && !scales))
        return set_err(AETH_ERR_ARG);
    if (n == 0) return AETH_OK;
    if ((reinterpret_cast<uintptr_t>(src) & 3) || (reinterpret_cast<uintptr_t>(out_f16) & 7))
        return set_err(AETH_ERR_UNSUPPORTED);
    const int64_t per = num_channels > 0 ? std::max<int64_t>(n / num_channels, 1) : n;
    // 8 warps per CTA, 128 words (512 elements) per warp and iteration; the
    // kernel's shared table needs exactly 256 threads
    fc_decode_int8_kernel<<<grid_for((n + kDecodeSpan - 1) / kDecodeSpan, 1, num_sms() * 8), 256, 0,
                            to_stream(stream)>>>(
        src, n, scales, n_scales, per, 1.0 / (double)per, num_channels > 0 ? 1 : 0, out_f16);
    AETH_LAUNCH_CHECK();
    return AETH_OK;
}

int aeth_fc_decode_nf4(const uint8_t* src, int64_t nbytes, float absmax, uint16_t* out_f16, aeth_stream_t stream) {
    if (!src || !out_f16 || nbytes < 0) return set_err(AETH_ERR_ARG);
    if (nbytes == 0) return AETH_OK;
    if ((reinterpret_cast<uintptr_t>(src) & 3) || (reinterpret_cast<uintptr_t>(out_f16) & 15))
        return set_err(AETH_ERR_UNSUPPORTED);
    fc_decode_nf4_kernel<<<grid_for((nbytes + 4095) / 4096, 1, num_sms() * 8), 256, 0, to_stream(stream)>>>(
        src, nbytes, absmax, out_f16);
    AETH_LAUNCH_CHECK();
    return AETH_OK;
}

int aeth_bf16_sr_update(float* master, const float* delta, int64_t n, uint64_t* rng_state, uint16_t* bf16_out,
                        aeth_stream_t stream) {
    if (!master || !delta || !rng_state || n < 0) return set_err(AETH_ERR_ARG);
    if (n == 0) return AETH_OK;
    if ((reinterpret_cast<uintptr_t>(master) & 15) || (reinterpret_cast<uintptr_t>(delta) & 15) ||
        (bf16_out && (reinterpret_cast<uintptr_t>(bf16_out) & 7)))
        return set_err(AETH_ERR_UNSUPPORTED);
    static Affine64 pow2[64];
    static bool pow2_init = false;
    static bool uploaded[kMaxDevices] = {};
    if (!pow2_init) {
        lcg_pow2_host(pow2);
        pow2_init = true;
    }
    int dev = 0;
    AETH_TRY(current_device(&dev));
    if (dev < 0 || dev >= kMaxDevices) return set_err(AETH_ERR_UNSUPPORTED);
    if (!uploaded[dev]) {
        AETH_CUDA(cudaMemcpyToSymbol(c_lcg_pow2, pow2, sizeof(pow2)));
        uploaded[dev] = true;
    }
    const int grid = grid_for((n + 3) / 4, 256, num_sms() * 8);
    const Affine64 step = lcg_jump((uint64_t)grid * 256 * 4, pow2);
    bf16_sr_update_kernel<<<grid, 256, 0, to_stream(stream)>>>(master, delta, n, *rng_state, step, bf16_out);
    AETH_LAUNCH_CHECK();
    // the state after n draws, as the sequential loop leaves it
    const Affine64 all = lcg_jump((uint64_t)n, pow2);
    *rng_state = all.a * *rng_state + all.c;
    return AETH_OK;
}

int aeth_lomo_sqnorm(const void* grad_bf16, int64_t n, double* sq_dev, aeth_stream_t stream) {
    if (!grad_bf16 || !sq_dev || n <= 0) return set_err(AETH_ERR_ARG);
    if ((reinterpret_cast<uintptr_t>(grad_bf16) & 15) != 0) return set_err(AETH_ERR_UNSUPPORTED);
    lomo_sqnorm_kernel<<<grid_for(n / 8 + 1, 256, 148 * 4), 256, 0, to_stream(stream)>>>(
        static_cast<const uint16_t*>(grad_bf16), n, sq_dev);
    AETH_LAUNCH_CHECK();
    return AETH_OK;
}

int aeth_lomo_update(const void* grad_bf16, int64_t n, const double* sq_dev, float max_norm, float lr, float beta,
                     int codec, int block, int8_t* mom8, float* mom_scales, uint8_t* w_packed, float* w_absmax,
                     float* prequant_out, aeth_stream_t stream) {
    if (!grad_bf16 || !sq_dev || !mom8 || !mom_scales || !w_packed || !w_absmax || n <= 0) return set_err(AETH_ERR_ARG);
    if (block != 2048 || n % 2048 != 0) return set_err(AETH_ERR_UNSUPPORTED);
    if (codec != AETH_CODEC_BLOCK_LINEAR && codec != AETH_CODEC_BLOCK_DYNAMIC) return set_err(AETH_ERR_ARG);
    if ((reinterpret_cast<uintptr_t>(grad_bf16) & 15) || (reinterpret_cast<uintptr_t>(mom8) & 7) ||
        (reinterpret_cast<uintptr_t>(w_packed) & 3))
        return set_err(AETH_ERR_UNSUPPORTED);
    AETH_TRY(codec_maps_ensure());
    if ((reinterpret_cast<uintptr_t>(mom8) & 15) || (reinterpret_cast<uintptr_t>(w_packed) & 7) ||
        (prequant_out && (reinterpret_cast<uintptr_t>(prequant_out) & 15)))
        return set_err(AETH_ERR_UNSUPPORTED);
    // one resident wave: the kernel strides over the blocks and prefetches the next one
    const int64_t nb = n / 2048;
    const uint16_t* gb = static_cast<const uint16_t*>(grad_bf16);
    auto kern = codec == AETH_CODEC_BLOCK_DYNAMIC ? lomo_update_kernel<AETH_CODEC_BLOCK_DYNAMIC>
                                                  : lomo_update_kernel<AETH_CODEC_BLOCK_LINEAR>;
    static bool attr_set[2][kMaxDevices] = {};
    int dev = 0;
    AETH_TRY(current_device(&dev));
    const int ci = codec == AETH_CODEC_BLOCK_DYNAMIC ? 1 : 0;
    if (!attr_set[ci][dev]) {
        AETH_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kLomoSmem));
        attr_set[ci][dev] = true;
    }
    int per_sm = 0;
    AETH_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kLomoThreads, kLomoSmem));
    // each CTA runs kLomoGroups independent 128-thread groups, one block each at a time
    const int grid = (int)std::min<int64_t>((nb + kLomoGroups - 1) / kLomoGroups,
                                            (int64_t)num_sms() * std::max(per_sm, 1));
    kern<<<grid, kLomoThreads, kLomoSmem, to_stream(stream)>>>(gb, n, sq_dev, max_norm, lr, beta, mom8, mom_scales,
                                                               w_packed, w_absmax, prequant_out, 1u);
    AETH_LAUNCH_CHECK();
    return AETH_OK;
}

}  // extern "C"
