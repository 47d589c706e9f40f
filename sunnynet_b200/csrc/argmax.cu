// Greedy next token for a batch of logit rows: the largest logit, the lowest
// id among equal ones, NaN never chosen (a row of NaN yields 0x7fffffff).
//
// A row of a large vocabulary (32K-65K logits) read by one CTA is a long
// serial scan; here every row is cut into kArgChunks slices read by separate
// CTAs (B x kArgChunks CTAs), each writing its best (value, id), and one warp
// per row then combines the slices in order. No atomics: the result does not
// depend on scheduling.
#include <cuda_runtime.h>

#include <cmath>

#include "kernels.cuh"
#include "ptx.cuh"
#include "runtime.cuh"

namespace sn {
namespace {

__device__ __forceinline__ void keep_better(float& bv, int& bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
    }
}

__global__ void __launch_bounds__(256)
    argmax_part_kernel(int V, const float* __restrict__ lg, float2* __restrict__ part) {
    __shared__ float sv[8];
    __shared__ int si[8];
    const int c = blockIdx.x, row = blockIdx.y;
    pdl_trigger();
    const long long lo = (long long)V * c / kArgChunks, hi = (long long)V * (c + 1) / kArgChunks;
    const float* r = lg + (size_t)row * V;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (long long i = lo + threadIdx.x; i < hi; i += blockDim.x) keep_better(bv, bi, r[i], (int)i);
    for (int o = 16; o; o >>= 1)
        keep_better(bv, bi, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o));
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        sv[w] = bv;
        si[w] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 1; k < (int)(blockDim.x >> 5); ++k) keep_better(bv, bi, sv[k], si[k]);
        part[(size_t)row * kArgChunks + c] = make_float2(bv, __int_as_float(bi));
    }
}

__global__ void argmax_final_kernel(const float2* __restrict__ part, int32_t* __restrict__ out) {
    const int row = blockIdx.x, lane = threadIdx.x;
    pdl_wait();  // the partials of argmax_part_kernel (programmatic launch)
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int c = lane; c < kArgChunks; c += 32) {
        const float2 p = part[(size_t)row * kArgChunks + c];
        keep_better(bv, bi, p.x, __float_as_int(p.y));
    }
    for (int o = 16; o; o >>= 1)
        keep_better(bv, bi, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o));
    if (lane == 0) out[row] = bi;
}

}  // namespace

int launch_argmax(const float* lg, int B, int V, float2* part, int32_t* out, cudaStream_t st) {
    if (B <= 0) return SN_OK;
    if (B > 65535) return fail(SN_E_INVAL, "argmax: %d rows exceed 65535", B);
    argmax_part_kernel<<<dim3(kArgChunks, B), 256, 0, st>>>(V, lg, part);
    SN_TRY(cuda_check(cudaGetLastError(), "argmax launch"));
    return cuda_check(launch_pdl(argmax_final_kernel, dim3(B), dim3(32), 0, st,
                                 (const float2*)part, out),
                      "argmax launch");
}

}  // namespace sn
