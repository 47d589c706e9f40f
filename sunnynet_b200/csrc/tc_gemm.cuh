// Tensor-core (tcgen05 / TMEM) contraction for the batched token loop.
//
// C[m][n] = epi( sum_k A'[m][k] * W[n][k] ) exactly like gemm.cuh, with A' the
// fp32 activations (optionally row-LayerNormed on load) and W the weights,
// computed to ~fp32 accuracy with a bf16x3 split: A' = Ah + Al, W = Wh + Wl
// (bf16 each) and D = Ah*Wh + Ah*Wl + Al*Wh accumulated in fp32 in TMEM
// (relative error ~2^-16 per product). INT8 weights are exact in bf16, so
// they need no Wl and only two MMAs; their per-row scale multiplies the result.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "gemm.cuh"

namespace sn {

// Weights prepared for the tensor-core path: bf16 planes (N,K) K-major plus
// one TMA descriptor per plane and tile width.
struct TcWeights {
    int N = 0, K = 0;
    bool int8 = false;                 // hi holds the exact int8 codes; no lo plane
    __nv_bfloat16* hi = nullptr;
    __nv_bfloat16* lo = nullptr;
    CUtensorMap tm_hi[3];              // box rows 32 / 64 / 128
    CUtensorMap tm_lo[3];
    bool ready = false;
};

// Split device weights (fp32 / fp16 (out,in) or int8 codes) into bf16 planes
// (allocated with cudaMalloc into *allocs owner) and build the TMA maps.
// wtype: kWF32, kWF16, kWI8.
int tc_prepare(TcWeights* tw, const void* W, int wtype, int N, int K, void* (*alloc)(size_t, void*),
               void* owner);

// Reserve the bf16 activation planes the tensor-core path splits A into, for
// every contraction with this K and up to `rows` rows. Must run outside CUDA
// graph capture (it may allocate); the planes are shared by all contractions
// with the same K, which run in stream order.
int tc_reserve(int K, long long rows);

// True when the tensor-core path supports this problem (planes reserved).
bool tc_usable(const GemmArgs& a, const TcWeights* tw);

int launch_tc_gemm(const GemmArgs& a, const TcWeights& tw, cudaStream_t st);

}  // namespace sn
