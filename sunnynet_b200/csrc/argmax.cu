// Greedy next token for a batch of logit rows: the largest logit, the lowest
// id among equal ones, NaN never chosen (a row of NaN yields 0x7fffffff).
//
// Every row is cut into nch slices read by separate CTAs (B x nch CTAs),
// each writing its best (value, id), and one warp per row then combines the
// slices. nch is chosen so the CTAs cover the SMs twice: 32 slices for a
// single row (a 32K-65K vocabulary read by one CTA would be a long serial
// scan), one CTA per row once there are ~300 rows. Rows whose length and
// base allow it are read with 16-byte loads. No atomics: the result does not
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
    argmax_part_kernel(int V, const float* __restrict__ lg, float2* __restrict__ part, int nch,
                       int vec) {
    __shared__ float sv[8];
    __shared__ int si[8];
    const int c = blockIdx.x, row = blockIdx.y;
    pdl_trigger();
    const float* r = lg + (size_t)row * V;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    if (vec) {  // V % 4 == 0, 16-byte rows: slices of whole float4
        const long long n4 = V / 4;
        const long long lo = n4 * c / nch, hi = n4 * (c + 1) / nch;
        const float4* r4 = reinterpret_cast<const float4*>(r);
        for (long long i = lo + threadIdx.x; i < hi; i += blockDim.x) {
            const float4 v = r4[i];
            const int j = (int)(4 * i);
            keep_better(bv, bi, v.x, j);
            keep_better(bv, bi, v.y, j + 1);
            keep_better(bv, bi, v.z, j + 2);
            keep_better(bv, bi, v.w, j + 3);
        }
    } else {
        const long long lo = (long long)V * c / nch, hi = (long long)V * (c + 1) / nch;
        for (long long i = lo + threadIdx.x; i < hi; i += blockDim.x)
            keep_better(bv, bi, r[i], (int)i);
    }
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
        part[(size_t)row * nch + c] = make_float2(bv, __int_as_float(bi));
    }
}

__global__ void argmax_final_kernel(const float2* __restrict__ part, int32_t* __restrict__ out,
                                    int nch) {
    const int row = blockIdx.x, lane = threadIdx.x;
    pdl_wait();  // the partials of argmax_part_kernel (programmatic launch)
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int c = lane; c < nch; c += 32) {
        const float2 p = part[(size_t)row * nch + c];
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
    const long long want = 2ll * rt().num_sms;  // CTAs to cover the SMs twice
    int nch = (int)((want + B - 1) / B);
    nch = nch < 1 ? 1 : (nch > kArgChunks ? kArgChunks : nch);
    const int vec = V % 4 == 0 && ((uintptr_t)lg & 15) == 0;
    argmax_part_kernel<<<dim3(nch, B), 256, 0, st>>>(V, lg, part, nch, vec);
    SN_TRY(cuda_check(cudaGetLastError(), "argmax launch"));
    return cuda_check(launch_pdl(argmax_final_kernel, dim3(B), dim3(32), 0, st,
                                 (const float2*)part, out, nch),
                      "argmax launch");
}

}  // namespace sn
