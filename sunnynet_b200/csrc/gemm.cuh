// Dense contractions of the token loop: C[m][n] = epi( sum_k A'[m][k] * W'[n][k] ).
//
//   A' = A, or a row LayerNorm of A applied while staging it:
//        ((A[m][k] - mu[m]) * rs[m]) * g[k] + c[k]
//   W' = W (fp32 / fp16) or (float)Wq (int8; the per-row scale multiplies the
//        finished dot product)
//   epi: none | softwedge z*(1 + 0.5a/(1+|z|)) | residual acc + (p*S + F + X)
//
// Both operands are K-major ((out,in) row-major weights, one activation row
// per sequence). Two kernels: a weight-streaming GEMV for M <= 8 rows (the
// bandwidth-bound decode at small batch; the A rows sit in shared memory and
// every warp streams whole weight rows with 16-byte loads), and a register-
// tiled SIMT GEMM for larger M.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace sn {

// kEpiAdd: C = C + acc (accumulate into the output, e.g. x += W y)
enum Epi : int {
    kEpiNone = 0,
    kEpiWedge = 1,
    kEpiResid = 2,
    kEpiAdd = 3,
    kEpiRelu2 = 4,
    kEpiTanh = 5,
    kEpiSigmoid = 6
};
enum WType : int { kWF32 = 0, kWI8 = 1, kWF16 = 2 };

struct GemmArgs {
    int M = 0, N = 0, K = 0;
    const float* A = nullptr;
    long long lda = 0;
    const void* W = nullptr;
    long long ldw = 0;
    const float* wscale = nullptr;  // int8: per output row n
    float* C = nullptr;
    long long ldc = 0;
    // optional row-LN prologue on A: statistics given (mu, rs), or computed in
    // the kernel from the staged rows (ln_inline, small-batch row path only)
    const float* mu = nullptr;
    const float* rs = nullptr;
    const float* g = nullptr;
    const float* c = nullptr;
    int ln_inline = 0;
    float ln_eps = 0.0f;
    // epilogue
    int epi = kEpiNone;
    float p = 0.0f;
    const float* S = nullptr;
    long long lds = 0;
    const float* F = nullptr;
    long long ldf = 0;
    const float* X = nullptr;
    long long ldx = 0;
    // tensor-core path only: also store the result as bf16 hi/lo planes
    // (ld = ldc), the input format of a following tensor-core contraction
    void* Ch = nullptr;
    void* Cl = nullptr;
    // tensor-core path only: > 0 keeps the grid within this many CTAs where a
    // tile width allows it (a contraction that runs beside another stream's
    // kernels leaves them the rest of the SMs)
    int max_ctas = 0;
};

struct TcWeights;

// Runs on the tensor cores when `tc` is given and the shape suits them
// (tc_gemm.cu), else on the SIMT kernels. pdl: the SIMT tiled kernel is
// launched with programmatic serialization (the small-batch row kernel
// always is).
int launch_gemm(const GemmArgs& a, int wtype, cudaStream_t st, const TcWeights* tc = nullptr,
                bool pdl = false);

// A' element (row-LN prologue when mu is set)
__device__ __forceinline__ float gemm_a_eff(const GemmArgs& a, int m, int k, float v) {
    if (a.mu) v = __fmul_rn(__fmul_rn(v - a.mu[m], a.rs[m]), a.g[k]) + a.c[k];
    return v;
}

// epilogue of one output element
__device__ __forceinline__ float gemm_epilogue(const GemmArgs& a, int m, int n, float acc) {
    if (a.wscale) acc = acc * a.wscale[n];
    switch (a.epi) {
        case kEpiWedge: return acc * (1.0f + 0.5f * a.p / (1.0f + fabsf(acc)));
        case kEpiResid:
            return acc + (a.p * a.S[m * a.lds + n] + a.F[m * a.ldf + n] + a.X[m * a.ldx + n]);
        case kEpiAdd: return a.C[m * a.ldc + n] + acc;
        case kEpiRelu2: {
            const float t = acc > 0.0f ? acc : 0.0f;
            return t * t;
        }
        case kEpiTanh: return tanhf(acc);
        case kEpiSigmoid: return 1.0f / (1.0f + expf(-acc));
        default: return acc;
    }
}

}  // namespace sn
