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
    // optional row-LN prologue on A
    const float* mu = nullptr;
    const float* rs = nullptr;
    const float* g = nullptr;
    const float* c = nullptr;
    // epilogue
    int epi = kEpiNone;
    float p = 0.0f;
    const float* S = nullptr;
    long long lds = 0;
    const float* F = nullptr;
    long long ldf = 0;
    const float* X = nullptr;
    long long ldx = 0;
};

int launch_gemm(const GemmArgs& a, int wtype, cudaStream_t st);

}  // namespace sn
