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
    // INT8: bf16 planes of the codes (hi, exact; no lo), or, with the
    // runtime's int8_mainloop setting at preparation, the codes themselves
    // (q8, (N,K) bytes, 16-byte aligned), converted to bf16 in the
    // contraction's main loop
    bool int8 = false;
    const int8_t* q8 = nullptr;
    __nv_bfloat16* hi = nullptr;
    __nv_bfloat16* lo = nullptr;
    CUtensorMap tm_hi[5];              // box rows 32 / 64 / 128 / 256 / 192
    CUtensorMap tm_lo[5];
    bool ready = false;
};

// Split device weights (fp32 / fp16 (out,in); INT8 codes into one exact
// plane) into bf16 planes (allocated through `alloc` for `owner`) and build
// the TMA maps; with the int8_mainloop setting INT8 codes are used in place
// (copied only to reach 16-byte alignment). wtype: kWF32, kWF16, kWI8.
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

// bf16 activation planes A' = hi + lo, (rows, K) with rows `ld` elements
// apart, and their TMA maps (box 64 x 128, SWIZZLE_128B). The kernel that
// produces a contraction's input writes them directly (store_split), so the
// contraction needs no split launch of its own.
struct TcAct {
    int K = 0;
    long long rows = 0, ld = 0;
    __nv_bfloat16* hi = nullptr;
    __nv_bfloat16* lo = nullptr;
    CUtensorMap tm_hi, tm_lo;
    bool ready = false;
};

// Allocate (rows, K) planes, ld = K. K % 8 == 0 (16-byte TMA row stride).
int tc_act_alloc(TcAct* p, int K, long long rows, void* (*alloc)(size_t, void*), void* owner);
// View of `rows` rows of K elements starting `off` elements into base's
// planes, `ld` elements apart (off and ld multiples of 8).
int tc_act_view(TcAct* v, const TcAct& base, long long off, long long rows, long long ld, int K);
// Split fp32 rows (rows, K) with row stride lda into dst's planes (ld = K).
int launch_split_rows(const float* A, long long rows, int K, long long lda, const TcAct& dst,
                      cudaStream_t st);
// The contraction with A' read from planes already written (a.A, a.mu are not
// read; the epilogue operands and a.Ch / a.Cl are as for launch_tc_gemm).
// pdl: launched with programmatic serialization: its barrier setup, TMEM
// allocation and first weight tiles overlap the previous kernel's tail.
int launch_tc_gemm_act(const GemmArgs& a, const TcWeights& tw, const TcAct& act, cudaStream_t st,
                       bool pdl = false);

// hi = bf16(v), lo = bf16(v - hi): the split every plane writer uses
__device__ __forceinline__ void store_split(__nv_bfloat16* hi, __nv_bfloat16* lo, long long i,
                                            float v) {
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    hi[i] = h;
    lo[i] = __float2bfloat16_rn(v - __bfloat162float(h));
}

// The same split for four consecutive elements (i a multiple of 4, planes
// 8-byte aligned): one 8-byte store per plane.
__device__ __forceinline__ void store_split4(__nv_bfloat16* hi, __nv_bfloat16* lo, long long i,
                                             float4 v) {
    const float x[4] = {v.x, v.y, v.z, v.w};
    __align__(8) __nv_bfloat16 h[4], l[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        h[k] = __float2bfloat16_rn(x[k]);
        l[k] = __float2bfloat16_rn(x[k] - __bfloat162float(h[k]));
    }
    *reinterpret_cast<uint2*>(hi + i) = *reinterpret_cast<const uint2*>(h);
    *reinterpret_cast<uint2*>(lo + i) = *reinterpret_cast<const uint2*>(l);
}

}  // namespace sn
