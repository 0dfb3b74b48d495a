// split_gemm.cuh -- fp32 products on the bf16 tensor cores without fp32
// rounding loss, for REF mode (the reference's fp32 GaLore projections,
// galore/src/project.rs:33-58).
//
// Each fp32 operand x is split into three bf16 terms, x = x0 + x1 + x2, each
// the round-to-nearest of the remainder so far; the terms carry all 24
// significant bits (barring underflow of the smallest term), and every
// product of two bf16 terms is exact in the tensor core's fp32 accumulator.
// A B = sum over the term pairs (i, j) of A_i B_j; the six pairs with
// i + j <= 2 are computed (the dropped ones are below 2^-24 relative), the
// smallest first, each a tcgen05 GEMM whose fp32 result is added into C.
// The result agrees with the reference's sequential fp32 loops to about the
// accuracy of those loops themselves (their own rounding error), not bit for
// bit; the exact-order CUDA-core GEMM (gemm_simt.cuh) stays the bit-exact path.
#pragma once
#include "gemm_tc.cuh"

namespace aeth {

// dst[t * count + i] = term t of src[i] (t < 3), bf16 bits.  A non-finite
// value keeps only term 0.
__global__ void split3_terms_kernel(const float* __restrict__ src, int64_t count, uint16_t* __restrict__ dst) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
        float r = src[i];
        const bool finite = fabsf(r) <= 3.402823466e38f;
#pragma unroll
        for (int t = 0; t < 3; ++t) {
            const uint16_t q = f32_to_bf16_bits(r);
            dst[t * count + i] = (t == 0 || finite) ? q : (uint16_t)0;
            r = finite ? __fsub_rn(r, bf16_bits_to_f32(q)) : 0.0f;
        }
    }
}

// One operand of split3_gemm: the fp32 matrix as stored (row-major, `rows` x
// `cols`, pitch `cols`) and whether the GEMM reads it K-major (A: rows = M,
// cols = K; B: rows = N, cols = K) or MN-major (A: rows = K, cols = M; B:
// rows = K, cols = N).
struct F32Op {
    const float* p;
    int rows, cols;
    bool mn_major;
};

template <bool A_MN, bool B_MN, class Epi>
int split3_gemm_pass(const uint16_t* a, int64_t lda, const uint16_t* b, int64_t ldb, int M, int N, int K,
                     const Epi& epi, cudaStream_t st) {
    TcOperand A{a, lda}, B{b, ldb};
    if (N <= 64) return tc_gemm_launch<64, 4, A_MN, B_MN>(A, B, M, N, K, true, epi, st);
    if (N <= 128) return tc_gemm_launch<128, 4, A_MN, B_MN>(A, B, M, N, K, true, epi, st);
    return tc_gemm_launch<256, 4, A_MN, B_MN>(A, B, M, N, K, true, epi, st);
}

template <bool A_MN, bool B_MN>
int split3_gemm_t(const uint16_t* at, int64_t acount, int64_t lda, const uint16_t* bt, int64_t bcount, int64_t ldb,
                  float* C, int64_t ldc, int M, int N, int K, bool accumulate, cudaStream_t st) {
    // term pairs, smallest contribution first; the first pass stores unless accumulating
    static const int pairs[6][2] = {{2, 0}, {1, 1}, {0, 2}, {1, 0}, {0, 1}, {0, 0}};
    for (int p = 0; p < 6; ++p) {
        const uint16_t* a = at + pairs[p][0] * acount;
        const uint16_t* b = bt + pairs[p][1] * bcount;
        if (p == 0 && !accumulate) {
            EpiStore e{C, ldc, AETH_DTYPE_F32, 1.0f};
            AETH_TRY((split3_gemm_pass<A_MN, B_MN>(a, lda, b, ldb, M, N, K, e, st)));
        } else {
            EpiAccum e{C, ldc};
            AETH_TRY((split3_gemm_pass<A_MN, B_MN>(a, lda, b, ldb, M, N, K, e, st)));
        }
    }
    return AETH_OK;
}

// C (M x N fp32, pitch ldc) = A B, or C += A B with `accumulate`.  `scratch`
// holds 3 (M K + K N) bf16 values.  Every pitch must be a multiple of 8
// elements (TMA), else AETH_ERR_UNSUPPORTED.
inline int split3_gemm(F32Op A, F32Op B, float* C, int64_t ldc, int M, int N, int K, bool accumulate,
                       uint16_t* scratch, cudaStream_t st) {
    const int64_t acount = (int64_t)A.rows * A.cols, bcount = (int64_t)B.rows * B.cols;
    if (A.cols % 8 != 0 || B.cols % 8 != 0) return AETH_ERR_UNSUPPORTED;
    uint16_t* at = scratch;
    uint16_t* bt = scratch + 3 * acount;
    split3_terms_kernel<<<grid_for(acount, 256), 256, 0, st>>>(A.p, acount, at);
    split3_terms_kernel<<<grid_for(bcount, 256), 256, 0, st>>>(B.p, bcount, bt);
    AETH_LAUNCH_CHECK();
    if (A.mn_major && B.mn_major)
        return split3_gemm_t<true, true>(at, acount, A.cols, bt, bcount, B.cols, C, ldc, M, N, K, accumulate, st);
    if (A.mn_major)
        return split3_gemm_t<true, false>(at, acount, A.cols, bt, bcount, B.cols, C, ldc, M, N, K, accumulate, st);
    if (B.mn_major)
        return split3_gemm_t<false, true>(at, acount, A.cols, bt, bcount, B.cols, C, ldc, M, N, K, accumulate, st);
    return split3_gemm_t<false, false>(at, acount, A.cols, bt, bcount, B.cols, C, ldc, M, N, K, accumulate, st);
}

}  // namespace aeth
