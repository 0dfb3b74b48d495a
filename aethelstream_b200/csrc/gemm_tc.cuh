// gemm_tc.cuh -- TMA-fed tcgen05 GEMM, D(128 x BN tile) = A(M x K) B(K x N),
// f16/bf16 operands, fp32 accumulation in TMEM, pluggable epilogue.
//
// One CTA per output tile, 6 warps:
//   warp 0      TMEM allocation + TMA producer (one elected lane)
//   warp 1      UMMA issuer (one elected lane): 4 x (M128, N=BN, K16) per stage
//   warps 2..5  epilogue: warp w reads TMEM lanes 32*(w%4)..+31 (one output row
//               per thread) in 64-column chunks via tcgen05.ld
// Pipeline: STAGES smem slots, `full` barriers completed by TMA transaction
// bytes, `empty` barriers completed by tcgen05.commit once the UMMAs that read
// the slot finished.  Every wait is bounded (mbar_wait).
//
// Operand majors (template flags):
//   A K-major:  A(i,k) = a[i*lda + k]       A MN-major: A(i,k) = a[k*lda + i]
//   B K-major:  B(k,j) = b[j*ldb + k]       B MN-major: B(k,j) = b[k*ldb + j]
#pragma once
#include <cudaTypedefs.h>

#include "nf4.cuh"
#include "umma.cuh"

namespace aeth {

constexpr int kBM = 128, kBK = 64;

// ---------------------------------------------------------------------------
// Epilogues.  apply() receives one output row's 64 consecutive columns.
// ---------------------------------------------------------------------------
struct EpiStore {  // C = D * alpha, converted to dtype (f32 / f16 / bf16)
    void* C;
    int64_t ldc;
    int dtype;
    float alpha;
    struct Shared { int unused; };
    __device__ void init_shared(Shared*, int, int) const {}
    __device__ __forceinline__ void apply(Shared*, int row, int col, const float (&vin)[64], int M, int N) const {
        if (row >= M) return;
        float v[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) v[i] = __fmul_rn(vin[i], alpha);
        const int64_t base = (int64_t)row * ldc + col;
        const bool full = col + 64 <= N && (ldc % 8) == 0;
        if (dtype == AETH_DTYPE_F32) {
            float* c = static_cast<float*>(C) + base;
            if (full) {
#pragma unroll
                for (int i = 0; i < 64; i += 4) *reinterpret_cast<float4*>(c + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
            } else {
#pragma unroll
                for (int i = 0; i < 64; ++i)
                    if (col + i < N) c[i] = v[i];
            }
        } else {
            uint16_t* c = static_cast<uint16_t*>(C) + base;
            if (full) {
#pragma unroll
                for (int i = 0; i < 64; i += 8) {
                    uint32_t w[4];
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        uint16_t lo, hi;
                        if (dtype == AETH_DTYPE_F16) {
                            lo = __half_as_ushort(__float2half_rn(v[i + 2 * k]));
                            hi = __half_as_ushort(__float2half_rn(v[i + 2 * k + 1]));
                        } else {
                            lo = f32_to_bf16_bits(v[i + 2 * k]);
                            hi = f32_to_bf16_bits(v[i + 2 * k + 1]);
                        }
                        w[k] = (uint32_t)lo | ((uint32_t)hi << 16);
                    }
                    *reinterpret_cast<uint4*>(c + i) = make_uint4(w[0], w[1], w[2], w[3]);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 64; ++i)
                    if (col + i < N)
                        c[i] = dtype == AETH_DTYPE_F16 ? __half_as_ushort(__float2half_rn(v[i])) : f32_to_bf16_bits(v[i]);
            }
        }
    }
};

struct EpiAccum {  // C(f32) = C + D   (R accumulation, adamw.rs:91-96)
    float* C;
    int64_t ldc;
    struct Shared { int unused; };
    __device__ void init_shared(Shared*, int, int) const {}
    __device__ __forceinline__ void apply(Shared*, int row, int col, const float (&v)[64], int M, int N) const {
        if (row >= M) return;
        float* c = C + (int64_t)row * ldc + col;
        if (col + 64 <= N && (ldc % 4) == 0) {
#pragma unroll
            for (int i = 0; i < 64; i += 4) {
                float4 o = *reinterpret_cast<float4*>(c + i);
                o.x = __fadd_rn(o.x, v[i]);
                o.y = __fadd_rn(o.y, v[i + 1]);
                o.z = __fadd_rn(o.z, v[i + 2]);
                o.w = __fadd_rn(o.w, v[i + 3]);
                *reinterpret_cast<float4*>(c + i) = o;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 64; ++i)
                if (col + i < N) c[i] = __fadd_rn(c[i], v[i]);
        }
    }
};

// Dense fp32 weight: w = w - lr * D (two roundings), optional decay and delta.
struct EpiF32Update {
    float* w;
    int64_t ldw;
    float lr, decay_mul;
    int has_decay;
    float* delta_out;
    struct Shared { int unused; };
    __device__ void init_shared(Shared*, int, int) const {}
    __device__ __forceinline__ void apply(Shared*, int row, int col, const float (&v)[64], int M, int N) const {
        if (row >= M) return;
#pragma unroll
        for (int i = 0; i < 64; ++i) {
            if (col + i >= N) continue;
            int64_t o = (int64_t)row * ldw + col + i;
            float d = __fmul_rn(v[i], lr);
            if (delta_out) delta_out[o] = d;
            float x = __fsub_rn(w[o], d);
            if (has_decay) x = __fmul_rn(x, decay_mul);
            w[o] = x;
        }
    }
};

// NF4 weight (K6 epilogue): dequantise the 64-element block, w -= lr * dW,
// optional decoupled decay, requantise bit-exactly, store codes + absmax.
struct EpiNf4Update {
    uint8_t* wp;
    float* wa;
    int64_t n;  // weight row length (multiple of 64)
    float lr, decay_mul;
    int has_decay;
    float* delta_out;
    float* prequant_out;
    struct Shared { Nf4Tables tab; };
    __device__ void init_shared(Shared* s, int tid, int nt) const { nf4_tables_init(&s->tab, tid, nt); }
    __device__ __forceinline__ void apply(Shared* s, int row, int col, const float (&v)[64], int M, int N) const {
        if (row >= M || col >= N) return;
        uint8_t* p = wp + (int64_t)row * (n / 2) + col / 2;
        float* ap = wa + (int64_t)row * (n / 64) + col / 64;
        const uint4 q0 = *reinterpret_cast<const uint4*>(p);
        const uint4 q1 = *reinterpret_cast<const uint4*>(p + 16);
        const float amax_old = *ap;
        float w[64];
        nf4_dequant_word(q0.x, amax_old, s->tab.byte_lut, w);
        nf4_dequant_word(q0.y, amax_old, s->tab.byte_lut, w + 8);
        nf4_dequant_word(q0.z, amax_old, s->tab.byte_lut, w + 16);
        nf4_dequant_word(q0.w, amax_old, s->tab.byte_lut, w + 24);
        nf4_dequant_word(q1.x, amax_old, s->tab.byte_lut, w + 32);
        nf4_dequant_word(q1.y, amax_old, s->tab.byte_lut, w + 40);
        nf4_dequant_word(q1.z, amax_old, s->tab.byte_lut, w + 48);
        nf4_dequant_word(q1.w, amax_old, s->tab.byte_lut, w + 56);
        const int64_t o = (int64_t)row * n + col;
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 64; ++i) {
            float d = __fmul_rn(v[i], lr);
            float x = __fsub_rn(w[i], d);
            if (has_decay) x = __fmul_rn(x, decay_mul);
            w[i] = x;
            amax = fmax_nan(amax, fabsf(x));
        }
        if (delta_out) {
#pragma unroll
            for (int i = 0; i < 64; i += 4)
                *reinterpret_cast<float4*>(delta_out + o + i) =
                    make_float4(__fmul_rn(v[i], lr), __fmul_rn(v[i + 1], lr), __fmul_rn(v[i + 2], lr), __fmul_rn(v[i + 3], lr));
        }
        if (prequant_out) {
#pragma unroll
            for (int i = 0; i < 64; i += 4)
                *reinterpret_cast<float4*>(prequant_out + o + i) = make_float4(w[i], w[i + 1], w[i + 2], w[i + 3]);
        }
        uint32_t pk[8];
        nf4_quant_regs<64>(w, amax, s->tab.bucket, pk);
        *reinterpret_cast<uint4*>(p) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        *reinterpret_cast<uint4*>(p + 16) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        *ap = nf4_store_amax(amax);
    }
};

// ---------------------------------------------------------------------------
// Kernel
// ---------------------------------------------------------------------------
template <int BN, int STAGES>
struct TcLayout {
    static constexpr int kABytes = kBM * kBK * 2;  // 16 KB
    static constexpr int kBBytes = BN * kBK * 2;
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kOperandBytes = STAGES * kStageBytes;
    static constexpr int kBarrierBytes = 256;
    // TMEM is allocated in powers of two of at least 32 columns
    static constexpr int kTmemCols = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : BN <= 256 ? 256 : 512;
};

template <int BN, int STAGES, bool A_MN, bool B_MN, class Epi>
__global__ void __launch_bounds__(192, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N,
                   int K, uint32_t idesc, Epi epi, uint32_t* err) {
    using L = TcLayout<BN, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);  // stays a shared pointer
    uint8_t* sA = base;
    uint8_t* sB = base + STAGES * L::kABytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(base + L::kOperandBytes);
    uint64_t* empty = full + STAGES;
    uint64_t* accf = empty + STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accf + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    typename Epi::Shared* eshared = reinterpret_cast<typename Epi::Shared*>(base + L::kOperandBytes + L::kBarrierBytes);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * BN;
    const int nk = (K + kBK - 1) / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        mbar_init(accf, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 0) { tmem_alloc(tmem_slot, L::kTmemCols); tmem_relinquish(); }
    epi.init_shared(eshared, threadIdx.x, blockDim.x);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            tma_prefetch_desc(&tmA);
            tma_prefetch_desc(&tmB);
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % STAGES;
                const uint32_t ph = (uint32_t)(kb / STAGES) & 1u;
                if (!mbar_wait(&empty[s], ph ^ 1u, abort, err, DEVERR_TIMEOUT_TMA)) break;
                mbar_arrive_expect_tx(&full[s], L::kStageBytes);
                const int k0 = kb * kBK;
                uint8_t* a = sA + s * L::kABytes;
                uint8_t* b = sB + s * L::kBBytes;
                if (A_MN) {
                    tma_load_2d(a, &tmA, &full[s], m0, k0);
                    tma_load_2d(a + 8192, &tmA, &full[s], m0 + 64, k0);
                } else {
                    tma_load_2d(a, &tmA, &full[s], k0, m0);
                }
                if (B_MN) {
#pragma unroll
                    for (int c = 0; c < BN / 64; ++c) tma_load_2d(b + c * 8192, &tmB, &full[s], n0 + 64 * c, k0);
                } else {
                    tma_load_2d(b, &tmB, &full[s], k0, n0);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % STAGES;
                const uint32_t ph = (uint32_t)(kb / STAGES) & 1u;
                if (!mbar_wait(&full[s], ph, abort, err, DEVERR_TIMEOUT_MMA)) break;
                tc_fence_after();
                const uint32_t a_addr = smem_u32(sA + s * L::kABytes);
                const uint32_t b_addr = smem_u32(sB + s * L::kBBytes);
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk) {
                    const uint64_t ad = A_MN ? sdesc_sw128(a_addr + kk * 2048, 8192, 1024)
                                             : sdesc_sw128(a_addr + kk * 32, 16, 1024);
                    const uint64_t bd = B_MN ? sdesc_sw128(b_addr + kk * 2048, 8192, 1024)
                                             : sdesc_sw128(b_addr + kk * 32, 16, 1024);
                    umma_f16_ss(tmem, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
                }
                umma_commit(&empty[s]);
            }
            umma_commit(accf);
        }
    } else {
        const int q = warp & 3;
        if (mbar_wait(accf, 0, abort, err, DEVERR_TIMEOUT_EPI) && !*abort) {
            tc_fence_after();
            const int row = m0 + q * 32 + lane;
#pragma unroll 1
            for (int c = 0; c < BN; c += 64) {
                float v[64];
                tmem_ld32<0>(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c, v);
                tmem_ld32<32>(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(c + 32), v);
                tmem_wait_ld();
                epi.apply(eshared, row, n0 + c, v, M, N);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, L::kTmemCols);
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
struct TcOperand {
    const void* ptr;
    int64_t ld;  // row pitch in elements
};

inline PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 2-D tensor map over a row-major matrix: `inner` contiguous elements per row,
// `outer` rows, row pitch `ld` elements of `esize` bytes.  Returns
// AETH_ERR_UNSUPPORTED when TMA cannot describe it (base not 16-byte aligned,
// pitch not a multiple of 16 bytes).
inline int make_tmap_2d(CUtensorMap* map, const void* ptr, CUtensorMapDataType dt, int esize, uint64_t inner,
                        uint64_t outer, int64_t ld, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
    auto enc = tmap_encoder();
    if (!enc) return AETH_ERR_UNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) != 0 || ((ld * esize) % 16) != 0) return AETH_ERR_UNSUPPORTED;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * esize)};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? AETH_OK : AETH_ERR_UNSUPPORTED;
}

// Tensor map over 16-bit (f16 / bf16) operands with the 128-byte swizzle the
// UMMA descriptors expect.
inline int make_tmap_16b(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, int64_t ld,
                         uint32_t box_inner, uint32_t box_outer, bool bf16) {
    return make_tmap_2d(map, ptr, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, inner,
                        outer, ld, box_inner, box_outer, CU_TENSOR_MAP_SWIZZLE_128B);
}

inline int num_sms() {
    static int n[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
    if (!n[dev] && cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) n[dev] = 148;
    return n[dev];
}

template <int BN, int STAGES, bool A_MN, bool B_MN, class Epi>
int tc_gemm_launch(TcOperand A, TcOperand B, int M, int N, int K, bool bf16, const Epi& epi, cudaStream_t st) {
    if (M <= 0 || N <= 0 || K <= 0) return AETH_ERR_ARG;
    DeviceRuntime* rt = nullptr;
    AETH_TRY(runtime_for_current(&rt));
    CUtensorMap ta, tb;
    if (A_MN) AETH_TRY(make_tmap_16b(&ta, A.ptr, (uint64_t)M, (uint64_t)K, A.ld, 64, 64, bf16));
    else AETH_TRY(make_tmap_16b(&ta, A.ptr, (uint64_t)K, (uint64_t)M, A.ld, 64, kBM, bf16));
    if (B_MN) AETH_TRY(make_tmap_16b(&tb, B.ptr, (uint64_t)N, (uint64_t)K, B.ld, 64, 64, bf16));
    else AETH_TRY(make_tmap_16b(&tb, B.ptr, (uint64_t)K, (uint64_t)N, B.ld, 64, BN, bf16));
    using L = TcLayout<BN, STAGES>;
    const int smem = 1024 + L::kOperandBytes + L::kBarrierBytes + (int)sizeof(typename Epi::Shared);
    auto kern = tc_gemm_kernel<BN, STAGES, A_MN, B_MN, Epi>;
    static bool attr_set[kMaxDevices] = {};
    int dev = 0;
    AETH_TRY(current_device(&dev));
    if (!attr_set[dev]) {
        AETH_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        attr_set[dev] = true;
    }
    dim3 grid((N + BN - 1) / BN, (M + kBM - 1) / kBM);
    kern<<<grid, 192, smem, st>>>(ta, tb, M, N, K, idesc_f16(kBM, BN, bf16, A_MN, B_MN), epi, rt->err_word);
    AETH_LAUNCH_CHECK();
    return AETH_OK;
}

}  // namespace aeth
