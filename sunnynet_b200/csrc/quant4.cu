// Group-symmetric INT4 weights and the W4A8 GEMV on sm_100a.
//
// Reference: sunnynet/runtime/quant.c (sn_quant_i4 34-65, sn_dequant_i4 67-87,
// sn_gemv_i4 89-154, sn_gemv_f32 156-172).
//
// W4A8 semantics, reproduced bit for bit: the activation is quantised per
// block (sc = amax/127, 1 if zero; q = rint(x/sc) clamped to +-127), each
// (row, block) integer dot sum_k q_w[k]*q_x[k] is exact (dp4a on nibble bytes,
// integer shuffles), and the row accumulates acc = acc + (s_w*s_x)*(float)(dot
// - 8*sum q_x) block by block in block order with round-to-nearest mul/add and
// no contraction -- the reference's ISO-C evaluation order.
//
// Memory layout: codes (out, in/2) row-major, byte k of a group = value k
// (low nibble) | value k+block/2 (high nibble); scales (out, in/block) fp32
// or fp16. A warp owns one output row per pass and streams it with 16-byte
// loads; 16 code bytes = 32 weights = one dp4a pair per 4 bytes.
#include <algorithm>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "kernels.cuh"
#include "ptx.cuh"
#include "quant.h"
#include "runtime.cuh"
#include "w4a8_rows.cuh"

namespace sn {
namespace {

// ------------------------------------------------------------ quantisers
// One warp per (row, group).
__global__ void quant_i4_kernel(const float* __restrict__ x, uint8_t* __restrict__ q,
                                void* __restrict__ scale, int rows, int N, int block, int fp16) {
    const int nb = N / block, half = block / 2;
    const long long wid = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (wid >= (long long)rows * nb) return;
    const int r = (int)(wid / nb), b = (int)(wid % nb);
    const float* xb = x + (size_t)r * N + (size_t)b * block;
    float m = 0.0f;
    for (int i = lane; i < block; i += 32) m = fmaxf(m, fabsf(xb[i]));
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float sc = m > 0.0f ? __fdiv_rn(m, 7.0f) : 1.0f;
    if (fp16) {
        __half h = __float2half_rn(sc);
        if ((__half_as_ushort(h) & 0x7fffu) == 0) h = __ushort_as_half((unsigned short)1);
        sc = __half2float(h);
        if (lane == 0) reinterpret_cast<__half*>(scale)[wid] = h;
    } else if (lane == 0) {
        reinterpret_cast<float*>(scale)[wid] = sc;
    }
    const float inv = __fdiv_rn(1.0f, sc);
    uint8_t* qb = q + (size_t)r * (N / 2) + (size_t)b * half;
    for (int k = lane; k < half; k += 32) {
        int lo = __float2int_rn(__fmul_rn(xb[k], inv));
        int hi = __float2int_rn(__fmul_rn(xb[half + k], inv));
        lo = min(max(lo, -8), 7);
        hi = min(max(hi, -8), 7);
        qb[k] = (uint8_t)((lo + 8) | ((hi + 8) << 4));
    }
}

__global__ void dequant_i4_kernel(const uint8_t* __restrict__ q, const void* __restrict__ scale,
                                  float* __restrict__ x, long long total_bytes, int N, int block,
                                  int fp16) {
    const int half = block / 2, nb = N / block, rb = N / 2;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total_bytes;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / rb;
        const int j = (int)(i - r * rb);
        const int b = j / half, k = j % half;
        const float sc = load_scale(scale, (size_t)r * nb + b, fp16);
        const uint8_t v = q[i];
        float* xr = x + (size_t)r * N + (size_t)b * block;
        xr[k] = __fmul_rn((float)((int)(v & 0x0F) - 8), sc);
        xr[half + k] = __fmul_rn((float)((int)(v >> 4) - 8), sc);
    }
}

template <bool FP16S, int NCH>
__global__ void __launch_bounds__(256, NCH == 1 ? 4 : 2)
    w4a8_kernel(float* __restrict__ Y, const float* __restrict__ X, const uint8_t* __restrict__ Wq,
                const void* __restrict__ scale, int nseq, int in, int out, int block, int epi) {
    w4a8_rows<FP16S, NCH>(Y, X, Wq, scale, nseq, in, out, block, epi,
                          blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5),
                          gridDim.x * (blockDim.x >> 5));
}

// Up to 8 contractions sharing the input width, block and scale type in one
// launch (the first-stage projections of an RWKV-7 layer at small batch):
// CTAs [cta0[p], cta0[p+1]) take problem p's rows, quantising only its input.
struct W4SimtGroup {
    float* Y[kW4MaxProblems];
    const float* X[kW4MaxProblems];
    const uint8_t* Wq[kW4MaxProblems];
    const void* scale[kW4MaxProblems];
    int N[kW4MaxProblems];
    int epi[kW4MaxProblems];
    int cta0[kW4MaxProblems + 1];
    int np;
};

template <bool FP16S, int NCH>
__global__ void __launch_bounds__(256, NCH == 1 ? 4 : 2)
    w4a8_group_kernel(const __grid_constant__ W4SimtGroup g, int nseq, int in, int block) {
    int p = 0;
    while (p + 1 < g.np && (int)blockIdx.x >= g.cta0[p + 1]) ++p;
    const int local = (int)blockIdx.x - g.cta0[p], nct = g.cta0[p + 1] - g.cta0[p];
    w4a8_rows<FP16S, NCH>(g.Y[p], g.X[p], g.Wq[p], g.scale[p], nseq, in, g.N[p], block, g.epi[p],
                          local * (blockDim.x >> 5) + (threadIdx.x >> 5), nct * (blockDim.x >> 5));
}

// General path (any even block dividing in): one lane per (row, block) dot,
// then the same ordered accumulation. Slower; used for odd block sizes.
template <bool FP16S>
__global__ void w4a8_generic_kernel(float* __restrict__ Y, const float* __restrict__ X,
                                    const uint8_t* __restrict__ Wq, const void* __restrict__ scale,
                                    int nseq, int in, int out, int block, int epi) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int nb = in / block, half = block / 2;
    const int seq0 = blockIdx.y * kMaxSeqTile;
    const int ns = min(kMaxSeqTile, nseq - seq0);
    int8_t* xq = reinterpret_cast<int8_t*>(smem);
    float* xs = reinterpret_cast<float*>(smem + (size_t)kMaxSeqTile * in);
    int* xsum = reinterpret_cast<int*>(xs + kMaxSeqTile * nb);
    pdl_trigger();
    pdl_wait();
    quant_act_smem(X + (size_t)seq0 * in, ns, in, block, nb, xq, xs, xsum);
    __syncthreads();
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < out * ns;
         idx += gridDim.x * blockDim.x) {
        const int row = idx / ns, s = idx % ns;
        const uint8_t* wr = Wq + (size_t)row * (in / 2);
        float acc = 0.0f;
        for (int b = 0; b < nb; ++b) {
            int d = 0;
            const int8_t* xl = xq + (size_t)s * in + b * block;
            for (int k = 0; k < half; ++k) {
                const uint8_t v = wr[b * half + k];
                d += (int)(v & 0x0F) * xl[k] + (int)(v >> 4) * xl[half + k];
            }
            const float sw = load_scale(scale, (size_t)row * nb + b, FP16S);
            acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(sw, xs[s * nb + b]),
                                           (float)(d - 8 * xsum[s * nb + b])));
        }
        w4_store(Y + (size_t)(seq0 + s) * out + row, acc, epi);
    }
}

// fp32 GEMV y = W(out,in) x: warp per row, float4 streaming.
__global__ void gemv_f32_kernel(float* __restrict__ y, const float* __restrict__ x,
                                const float* __restrict__ W, int in, int out, int vec) {
    const int lane = threadIdx.x & 31;
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int nw = gridDim.x * (blockDim.x >> 5);
    for (int row = gw; row < out; row += nw) {
        const float* wr = W + (size_t)row * in;
        float acc = 0.0f;
        if (vec) {
            for (int i = lane * 4; i < in; i += 128) {
                const float4 w = __ldg(reinterpret_cast<const float4*>(wr + i));
                const float4 v = *reinterpret_cast<const float4*>(x + i);
                acc = fmaf(w.x, v.x, acc);
                acc = fmaf(w.y, v.y, acc);
                acc = fmaf(w.z, v.z, acc);
                acc = fmaf(w.w, v.w, acc);
            }
        } else {
            for (int i = lane; i < in; i += 32) acc = fmaf(wr[i], x[i], acc);
        }
        for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) y[row] = acc;
    }
}

}  // namespace

// Device-pointer W4A8 GEMV/GEMM (Y (nseq,out), X (nseq,in)), used by the ABI
// and by the RWKV-7 model.
int launch_w4a8(float* Y, const float* X, const uint8_t* Wq, const void* scale, int nseq, int in,
                int out, int block, bool fp16, cudaStream_t st, int epi, bool pdl) {
    if (w4a8_tc_ok(nseq, in, out, block, Wq) && w4a8_tc_ready(nseq, in, block))
        return launch_w4a8_tc(Y, X, Wq, scale, nseq, in, out, block, fp16, epi, st, pdl);
    const int nb = in / block;
    const size_t smem = (size_t)kMaxSeqTile * in + (size_t)kMaxSeqTile * nb * 8 + 16;
    if (smem > 200 * 1024) return fail(SN_E_INVAL, "gemv_i4: in=%d too large", in);
    // whole 16-byte chunks per block half, and chunk groups that tile a warp
    const bool pow2 = block == 32 || block == 64 || block == 128 || block == 256;
    const bool fast = pow2 && in % 32 == 0 && in <= 4096 && ((uintptr_t)Wq % 16 == 0);
    const int nch = in <= 1024 ? 1 : (in <= 2048 ? 2 : 4);
    const int seq_tiles = (nseq + kMaxSeqTile - 1) / kMaxSeqTile;
    const int warps_needed = out;
    int ctas = (warps_needed + 7) / 8;
    const int cap = 8 * rt().num_sms;  // 8 CTAs of 256 threads fit on an SM
    if (ctas > cap) ctas = cap;
    dim3 grid(ctas, seq_tiles);
    if (fast) {
        auto k = nch == 1 ? (fp16 ? w4a8_kernel<true, 1> : w4a8_kernel<false, 1>)
                 : nch == 2 ? (fp16 ? w4a8_kernel<true, 2> : w4a8_kernel<false, 2>)
                            : (fp16 ? w4a8_kernel<true, 4> : w4a8_kernel<false, 4>);
        if (smem > 48 * 1024)
            SN_TRY(cuda_check(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)smem), "w4a8 smem"));
        return cuda_check(launch_pdl_if(pdl, k, grid, dim3(256), smem, st, Y, X, Wq, scale, nseq,
                                        in, out, block, epi),
                          "w4a8 launch");
    } else {
        auto k = fp16 ? w4a8_generic_kernel<true> : w4a8_generic_kernel<false>;
        if (smem > 48 * 1024)
            SN_TRY(cuda_check(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)smem), "w4a8 smem"));
        return cuda_check(launch_pdl_if(pdl, k, grid, dim3(256), smem, st, Y, X, Wq, scale, nseq,
                                        in, out, block, epi),
                          "w4a8 launch");
    }
}

int launch_w4a8_group(const W4Problem* pr, int np, int nseq, int in, int block, bool fp16,
                      cudaStream_t st, bool pdl) {
    if (np < 1 || np > kW4MaxProblems) return fail(SN_E_INVAL, "w4a8 group: %d problems", np);
    if (nseq > kMaxSeqTile)  // one sequence tile per CTA in the grouped form
        return fail(SN_E_INVAL, "w4a8 group: %d sequences (at most %d)", nseq, kMaxSeqTile);
    const bool pow2 = block == 32 || block == 64 || block == 128 || block == 256;
    if (!pow2 || in % 32 != 0 || in > 4096 || in % block != 0)
        return fail(SN_E_INVAL, "w4a8 group: unsupported in=%d block=%d", in, block);
    W4SimtGroup g;
    g.np = np;
    g.cta0[0] = 0;
    long long rows = 0;
    for (int i = 0; i < np; ++i) rows += pr[i].N;
    const int budget = 8 * rt().num_sms;  // CTAs, shared out by rows
    for (int i = 0; i < np; ++i) {
        if ((uintptr_t)pr[i].Wq % 16) return fail(SN_E_INVAL, "w4a8 group: unaligned codes");
        g.Y[i] = pr[i].Y;
        g.X[i] = pr[i].X;
        g.Wq[i] = pr[i].Wq;
        g.scale[i] = pr[i].scale;
        g.N[i] = pr[i].N;
        g.epi[i] = pr[i].epi;
        int c = (int)((long long)budget * pr[i].N / rows);
        c = std::max(1, std::min(c, (pr[i].N + 7) / 8));
        g.cta0[i + 1] = g.cta0[i] + c;
    }
    const int nb = in / block;
    const size_t smem = (size_t)kMaxSeqTile * in + (size_t)kMaxSeqTile * nb * 8 + 16;
    const int nch = in <= 1024 ? 1 : (in <= 2048 ? 2 : 4);
    auto k = nch == 1 ? (fp16 ? w4a8_group_kernel<true, 1> : w4a8_group_kernel<false, 1>)
             : nch == 2 ? (fp16 ? w4a8_group_kernel<true, 2> : w4a8_group_kernel<false, 2>)
                        : (fp16 ? w4a8_group_kernel<true, 4> : w4a8_group_kernel<false, 4>);
    if (smem > 48 * 1024)
        SN_TRY(cuda_check(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)smem),
                          "w4a8 group smem"));
    return cuda_check(launch_pdl_if(pdl, k, dim3(g.cta0[np]), dim3(256), smem, st, g, nseq, in,
                                    block),
                      "w4a8 group launch");
}

int launch_gemv_f32(float* y, const float* x, const float* W, int in, int out, cudaStream_t st) {
    const bool vec = in % 4 == 0 && (uintptr_t)W % 16 == 0 && (uintptr_t)x % 16 == 0;
    int ctas = (out + 7) / 8;
    if (ctas > 8 * rt().num_sms) ctas = 8 * rt().num_sms;
    gemv_f32_kernel<<<ctas, 256, 0, st>>>(y, x, W, in, out, vec ? 1 : 0);
    return cuda_check(cudaGetLastError(), "gemv_f32 launch");
}

int launch_quant_i4(const float* x, uint8_t* q, void* scale, int rows, int N, int block,
                    bool fp16, cudaStream_t st) {
    const long long warps = (long long)rows * (N / block);
    const long long ctas = (warps + 7) / 8;
    quant_i4_kernel<<<(unsigned)ctas, 256, 0, st>>>(x, q, scale, rows, N, block, fp16 ? 1 : 0);
    return cuda_check(cudaGetLastError(), "quant_i4 launch");
}

}  // namespace sn

using namespace sn;

namespace {

bool i4_shape_ok(int rows, int N, int block) {
    return rows > 0 && N > 0 && block > 0 && block % 2 == 0 && N % block == 0;
}

int do_quant_i4(const float* x, uint8_t* q, void* scale, int rows, int N, int block, int fp16) {
    if (block <= 0) block = SN_I4_BLOCK;
    if (!x || !q || !scale || !i4_shape_ok(rows, N, block))
        return fail(SN_E_INVAL, "quant_i4: bad arguments (rows=%d N=%d block=%d)", rows, N, block);
    SN_TRY(ensure_init());
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    const size_t ns = (size_t)rows * (N / block) * (fp16 ? 2 : 4);
    Arr X, Q, S;
    SN_TRY(stage_in(x, (size_t)rows * N * 4, 0, &X));
    SN_TRY(stage_out(q, (size_t)rows * (N / 2), 1, &Q));
    SN_TRY(stage_out(scale, ns, 2, &S));
    SN_TRY(launch_quant_i4((const float*)X.dev, (uint8_t*)Q.dev, S.dev, rows, N, block, fp16 != 0,
                           stream()));
    SN_TRY(copy_back(Q));
    SN_TRY(copy_back(S));
    return finish(Q.host || S.host || X.dev != x);
}

int do_dequant_i4(const uint8_t* q, const void* scale, float* x, int rows, int N, int block,
                  int fp16) {
    if (block <= 0) block = SN_I4_BLOCK;
    if (!x || !q || !scale || !i4_shape_ok(rows, N, block))
        return fail(SN_E_INVAL, "dequant_i4: bad arguments");
    SN_TRY(ensure_init());
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    const size_t ns = (size_t)rows * (N / block) * (fp16 ? 2 : 4);
    Arr Q, S, X;
    SN_TRY(stage_in(q, (size_t)rows * (N / 2), 0, &Q));
    SN_TRY(stage_in(scale, ns, 1, &S));
    SN_TRY(stage_out(x, (size_t)rows * N * 4, 2, &X));
    const long long total = (long long)rows * (N / 2);
    const int blocks = grid_blocks(total);
    dequant_i4_kernel<<<blocks, 256, 0, stream()>>>((const uint8_t*)Q.dev, S.dev, (float*)X.dev,
                                                    total, N, block, fp16);
    SN_TRY(cuda_check(cudaGetLastError(), "dequant_i4 launch"));
    SN_TRY(copy_back(X));
    return finish(X.host || Q.dev != q || S.dev != scale);
}

int do_gemm_i4(float* Y, const float* X, const uint8_t* Wq, const void* scale, int B, int in,
               int out, int block, int fp16) {
    if (block <= 0) block = SN_I4_BLOCK;
    if (!Y || !X || !Wq || !scale || B <= 0 || out <= 0 || !i4_shape_ok(out, in, block))
        return fail(SN_E_INVAL, "gemv_i4: in %% block != 0 or bad arguments (in=%d block=%d)", in,
                    block);
    if (block > 256)
        return fail(SN_E_INVAL, "gemv_i4: block > 256 overflows the reference's 16-bit lane sums");
    SN_TRY(ensure_init());
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    const size_t ns = (size_t)out * (in / block) * (fp16 ? 2 : 4);
    Arr Xa, Q, S, Ya;
    SN_TRY(stage_in(X, (size_t)B * in * 4, 0, &Xa));
    SN_TRY(stage_in(Wq, (size_t)out * (in / 2), 1, &Q));
    SN_TRY(stage_in(scale, ns, 2, &S));
    SN_TRY(stage_out(Y, (size_t)B * out * 4, 3, &Ya));
    if (w4a8_tc_ok(B, in, out, block, Q.dev)) SN_TRY(w4a8_tc_reserve(B, in, block));
    SN_TRY(launch_w4a8((float*)Ya.dev, (const float*)Xa.dev, (const uint8_t*)Q.dev, S.dev, B, in,
                       out, block, fp16 != 0, stream(), kW4Store));
    SN_TRY(copy_back(Ya));
    return finish(Ya.host || Xa.dev != X || Q.dev != Wq || S.dev != scale);
}

int do_gemv_f32(float* y, const float* x, const float* W, int in, int out) {
    if (!y || !x || !W || in <= 0 || out <= 0) return fail(SN_E_INVAL, "gemv_f32: bad arguments");
    SN_TRY(ensure_init());
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    Arr Xa, Wa, Ya;
    SN_TRY(stage_in(x, (size_t)in * 4, 0, &Xa));
    SN_TRY(stage_in(W, (size_t)in * out * 4, 1, &Wa));
    SN_TRY(stage_out(y, (size_t)out * 4, 2, &Ya));
    SN_TRY(launch_gemv_f32((float*)Ya.dev, (const float*)Xa.dev, (const float*)Wa.dev, in, out,
                           stream()));
    SN_TRY(copy_back(Ya));
    return finish(Ya.host || Xa.dev != x || Wa.dev != W);
}

}  // namespace

extern "C" {

sn_status sn_abi_quant_i4(const float* x, uint8_t* q, void* scale, int32_t rows, int32_t N,
                          int32_t block, int32_t scale_fp16) {
    return do_quant_i4(x, q, scale, rows, N, block, scale_fp16);
}

sn_status sn_abi_dequant_i4(const uint8_t* q, const void* scale, float* x, int32_t rows,
                            int32_t N, int32_t block, int32_t scale_fp16) {
    return do_dequant_i4(q, scale, x, rows, N, block, scale_fp16);
}

sn_status sn_abi_gemv_i4(float* y, const float* x, const uint8_t* Wq, const void* scale,
                         int32_t in, int32_t out, int32_t block, int32_t scale_fp16) {
    return do_gemm_i4(y, x, Wq, scale, 1, in, out, block, scale_fp16);
}

sn_status sn_abi_gemm_i4(float* Y, const float* X, const uint8_t* Wq, const void* scale,
                         int32_t B, int32_t in, int32_t out, int32_t block, int32_t scale_fp16) {
    return do_gemm_i4(Y, X, Wq, scale, B, in, out, block, scale_fp16);
}

void sn_quant_i4(const float* x, unsigned char* q, float* scale, int rows, int N, int block) {
    do_quant_i4(x, q, scale, rows, N, block, 0);
}

void sn_dequant_i4(const unsigned char* q, const float* scale, float* x, int rows, int N,
                   int block) {
    do_dequant_i4(q, scale, x, rows, N, block, 0);
}

void sn_gemv_i4(float* y, const float* x, const unsigned char* Wq, const float* scale, int in,
                int out, int block) {
    do_gemm_i4(y, x, Wq, scale, 1, in, out, block, 0);
}

void sn_gemv_f32(float* y, const float* x, const float* W, int in, int out) {
    do_gemv_f32(y, x, W, in, out);
}

}  // extern "C"
