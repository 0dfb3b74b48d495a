// split_gemm.cuh -- fp32 products on the bf16 tensor cores without fp32
// rounding loss: REF mode's projections (galore/src/project.rs:33-58) and the
// randomized-SVD refresh's sketches (galore/src/randomized_svd.rs:76-149).
//
// Each fp32 operand x is split into three bf16 terms, x = x0 + x1 + x2, each
// the round-to-nearest of the remainder so far; the terms carry all 24
// significant bits (barring underflow of the smallest term), and every
// product of two bf16 terms is exact in the tensor core's fp32 accumulator.
// A bf16 operand is its own single term.  A B = sum over the term pairs (i, j)
// of A_i B_j; the pairs with i + j <= 2 are computed (the dropped ones are
// below 2^-24 relative), the smallest first, each a tcgen05 GEMM whose fp32
// result is added into C.  The result agrees with a sequential fp32 loop to
// about that loop's own rounding error, not bit for bit; the exact-order
// CUDA-core GEMM (gemm_simt.cuh) stays the bit-exact path.
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

inline int split3_terms(const float* src, int64_t count, uint16_t* dst, cudaStream_t st) {
    split3_terms_kernel<<<grid_for(count, 256), 256, 0, st>>>(src, count, dst);
    AETH_LAUNCH_CHECK();
    return AETH_OK;
}

// A GEMM operand as bf16 term matrices: `nterms` (1 or 3) matrices of `count`
// elements each, consecutive in memory, pitch `ld`; read K-major (A: M x K
// rows x cols; B: N x K) or MN-major (A: K x M; B: K x N).
struct TermOp {
    const uint16_t* terms;
    int nterms;
    int64_t count;
    int64_t ld;
    bool mn_major;
};

template <int BN, bool A_MN, bool B_MN, class Epi>
int terms_pass_bn(const uint16_t* a, int64_t lda, const uint16_t* b, int64_t ldb, int M, int N, int K, const Epi& epi,
                  cudaStream_t st) {
    return tc_gemm_launch<BN, 4, A_MN, B_MN>(TcOperand{a, lda}, TcOperand{b, ldb}, M, N, K, true, epi, st);
}

// The output tile width with the least padding of N (64, 128, 192 or 256
// columns; 192 suits N = r + p = 520, three tiles where 256 needs three
// mostly empty ones too).
inline int terms_tile_n(int N) {
    int best = 64;
    int64_t best_cols = -1;
    for (int bn : {256, 192, 128, 64}) {
        const int64_t cols = (int64_t)((N + bn - 1) / bn) * bn;
        if (best_cols < 0 || cols < best_cols) { best_cols = cols; best = bn; }
    }
    return best;
}

template <bool A_MN, bool B_MN, class Epi>
int terms_pass(const uint16_t* a, int64_t lda, const uint16_t* b, int64_t ldb, int M, int N, int K, const Epi& epi,
               cudaStream_t st) {
    switch (terms_tile_n(N)) {
        case 64: return terms_pass_bn<64, A_MN, B_MN>(a, lda, b, ldb, M, N, K, epi, st);
        case 128: return terms_pass_bn<128, A_MN, B_MN>(a, lda, b, ldb, M, N, K, epi, st);
        case 192: return terms_pass_bn<192, A_MN, B_MN>(a, lda, b, ldb, M, N, K, epi, st);
        default: return terms_pass_bn<256, A_MN, B_MN>(a, lda, b, ldb, M, N, K, epi, st);
    }
}

template <bool A_MN, bool B_MN>
int terms_gemm_t(const TermOp& A, const TermOp& B, float* C, int64_t ldc, int M, int N, int K, bool accumulate,
                 cudaStream_t st) {
    // term pairs, smallest contribution first; the first pass stores unless accumulating
    static const int pairs[6][2] = {{2, 0}, {1, 1}, {0, 2}, {1, 0}, {0, 1}, {0, 0}};
    bool first = !accumulate;
    for (const auto& pr : pairs) {
        if (pr[0] >= A.nterms || pr[1] >= B.nterms) continue;
        const uint16_t* a = A.terms + pr[0] * A.count;
        const uint16_t* b = B.terms + pr[1] * B.count;
        if (first) {
            EpiStore e{C, ldc, AETH_DTYPE_F32, 1.0f};
            AETH_TRY((terms_pass<A_MN, B_MN>(a, A.ld, b, B.ld, M, N, K, e, st)));
            first = false;
        } else {
            EpiAccum e{C, ldc};
            AETH_TRY((terms_pass<A_MN, B_MN>(a, A.ld, b, B.ld, M, N, K, e, st)));
        }
    }
    return AETH_OK;
}

// C (M x N fp32, pitch ldc) = A B, or C += A B with `accumulate`.  Every pitch
// must be a multiple of 8 elements (TMA), else AETH_ERR_UNSUPPORTED.
inline int terms_gemm(const TermOp& A, const TermOp& B, float* C, int64_t ldc, int M, int N, int K, bool accumulate,
                      cudaStream_t st) {
    if (A.ld % 8 != 0 || B.ld % 8 != 0) return AETH_ERR_UNSUPPORTED;
    if (A.mn_major && B.mn_major) return terms_gemm_t<true, true>(A, B, C, ldc, M, N, K, accumulate, st);
    if (A.mn_major) return terms_gemm_t<true, false>(A, B, C, ldc, M, N, K, accumulate, st);
    if (B.mn_major) return terms_gemm_t<false, true>(A, B, C, ldc, M, N, K, accumulate, st);
    return terms_gemm_t<false, false>(A, B, C, ldc, M, N, K, accumulate, st);
}

// One fp32 operand of split3_gemm: the matrix as stored (row-major, `rows` x
// `cols`, pitch `cols`) and whether the GEMM reads it K-major (A: rows = M,
// cols = K; B: rows = N, cols = K) or MN-major (A: rows = K, cols = M; B:
// rows = K, cols = N).
struct F32Op {
    const float* p;
    int rows, cols;
    bool mn_major;
};

// C (M x N fp32, pitch ldc) = A B (or += with `accumulate`) for fp32 A and B,
// both split into three terms.  `scratch` holds 3 (M K + K N) bf16 values.
inline int split3_gemm(F32Op A, F32Op B, float* C, int64_t ldc, int M, int N, int K, bool accumulate,
                       uint16_t* scratch, cudaStream_t st) {
    const int64_t acount = (int64_t)A.rows * A.cols, bcount = (int64_t)B.rows * B.cols;
    if (A.cols % 8 != 0 || B.cols % 8 != 0) return AETH_ERR_UNSUPPORTED;
    uint16_t* at = scratch;
    uint16_t* bt = scratch + 3 * acount;
    AETH_TRY(split3_terms(A.p, acount, at, st));
    AETH_TRY(split3_terms(B.p, bcount, bt, st));
    return terms_gemm(TermOp{at, 3, acount, A.cols, A.mn_major}, TermOp{bt, 3, bcount, B.cols, B.mn_major}, C, ldc, M,
                      N, K, accumulate, st);
}

}  // namespace aeth
