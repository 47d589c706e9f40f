// SIMT implementations of the contractions declared in gemm.cuh.
#include "gemm.cuh"
#include "ptx.cuh"
#include "runtime.cuh"
#include "tc_gemm.cuh"

namespace sn {
namespace {

template <int WT>
__device__ __forceinline__ float wload(const void* W, long long i) {
    if (WT == kWF32) return reinterpret_cast<const float*>(W)[i];
    if (WT == kWI8) return (float)reinterpret_cast<const int8_t*>(W)[i];
    return __half2float(reinterpret_cast<const __half*>(W)[i]);
}

__device__ __forceinline__ float a_eff(const GemmArgs& a, int m, int k, float v) {
    return gemm_a_eff(a, m, k, v);
}

__device__ __forceinline__ float epilogue(const GemmArgs& a, int m, int n, float acc) {
    return gemm_epilogue(a, m, n, acc);
}

// ---------------------------------------------------------------- GEMV (M <= 8)
constexpr int kGemvRows = 8;

template <int WT>
__global__ void __launch_bounds__(256) gemv_rows_kernel(GemmArgs a) {
    extern __shared__ __align__(16) float sA[];  // [M][K], then mean[M], rstd[M]
    const int M = a.M, K = a.K;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nw = gridDim.x * (blockDim.x >> 5);
    pdl_trigger();
    {   // this warp's weight rows do not depend on the previous kernel: pull them
        // into L2 while it finishes (launched with programmatic serialization)
        const int wb = WT == kWF32 ? 4 : (WT == kWI8 ? 1 : 2);
        const long long rowbytes = (long long)K * wb;
        for (int n = blockIdx.x * (blockDim.x >> 5) + warp; n < a.N; n += nw) {
            const char* row = reinterpret_cast<const char*>(a.W) + (long long)n * a.ldw * wb;
            for (long long off = (long long)lane * 128; off < rowbytes; off += 32 * 128)
                prefetch_l2(row + off);
        }
    }
    pdl_wait();
    float* st_mu = sA + M * K;
    float* st_rs = st_mu + M;
    for (int i = threadIdx.x; i < M * K; i += blockDim.x) {
        const int m = i / K, k = i - m * K;
        const float v = a.A[m * a.lda + k];
        sA[i] = a.ln_inline ? v : a_eff(a, m, k, v);
    }
    __syncthreads();
    if (a.ln_inline) {  // two-pass row statistics, one warp per row (M <= 8)
        if (warp < M) {
            const float* r = sA + warp * K;
            float s = 0.0f;
            for (int k = lane; k < K; k += 32) s += r[k];
            for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            const float mean = s / (float)K;
            float v = 0.0f;
            for (int k = lane; k < K; k += 32) {
                const float d = r[k] - mean;
                v += d * d;
            }
            for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) {
                st_mu[warp] = mean;
                st_rs[warp] = 1.0f / sqrtf(v / (float)K + a.ln_eps);
            }
        }
        __syncthreads();
        for (int i = threadIdx.x; i < M * K; i += blockDim.x) {
            const int m = i / K, k = i - m * K;
            sA[i] = __fmul_rn(__fmul_rn(sA[i] - st_mu[m], st_rs[m]), a.g[k]) + a.c[k];
        }
        __syncthreads();
    }
    const bool vec = (WT == kWF32 ? K % 4 == 0 : (WT == kWI8 ? K % 16 == 0 : K % 8 == 0)) &&
                     (a.ldw % (WT == kWF32 ? 4 : (WT == kWI8 ? 16 : 8)) == 0);
    for (int n = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); n < a.N; n += nw) {
        float acc[kGemvRows];
#pragma unroll
        for (int m = 0; m < kGemvRows; ++m) acc[m] = 0.0f;
        if (WT == kWF32 && vec) {
            const float4* w4 = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.W) +
                                                               n * a.ldw);
            for (int k4 = lane; k4 < K / 4; k4 += 32) {
                const float4 w = __ldg(w4 + k4);
#pragma unroll
                for (int m = 0; m < kGemvRows; ++m) {
                    if (m < M) {
                        const float4 x = *reinterpret_cast<const float4*>(sA + m * K + 4 * k4);
                        acc[m] = fmaf(w.x, x.x, acc[m]);
                        acc[m] = fmaf(w.y, x.y, acc[m]);
                        acc[m] = fmaf(w.z, x.z, acc[m]);
                        acc[m] = fmaf(w.w, x.w, acc[m]);
                    }
                }
            }
        } else if (WT == kWI8 && vec) {
            const int4* w16 = reinterpret_cast<const int4*>(reinterpret_cast<const int8_t*>(a.W) +
                                                            n * a.ldw);
            for (int k16 = lane; k16 < K / 16; k16 += 32) {
                const int4 w = __ldg(w16 + k16);
                const int8_t* wb = reinterpret_cast<const int8_t*>(&w);
#pragma unroll
                for (int m = 0; m < kGemvRows; ++m) {
                    if (m < M) {
                        const float* x = sA + m * K + 16 * k16;
#pragma unroll
                        for (int j = 0; j < 16; ++j) acc[m] = fmaf((float)wb[j], x[j], acc[m]);
                    }
                }
            }
        } else {
            for (int k = lane; k < K; k += 32) {
                const float w = wload<WT>(a.W, n * a.ldw + k);
#pragma unroll
                for (int m = 0; m < kGemvRows; ++m)
                    if (m < M) acc[m] = fmaf(w, sA[m * K + k], acc[m]);
            }
        }
#pragma unroll
        for (int m = 0; m < kGemvRows; ++m) {
            if (m < M) {
                float v = acc[m];
                for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                if (lane == 0) a.C[m * a.ldc + n] = epilogue(a, m, n, v);
            }
        }
    }
}

// ------------------------------------------------------------ tiled SIMT GEMM
constexpr int BM = 64, BN = 64, BK = 16;

template <int WT>
__global__ void __launch_bounds__(256) gemm_tiled_kernel(GemmArgs a) {
    __shared__ __align__(16) float As[2][BK][BM + 4];
    __shared__ __align__(16) float Ws[2][BK][BN + 4];
    const int tid = threadIdx.x;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int tx = tid % 16, ty = tid / 16;
    pdl_trigger();
    pdl_wait();  // no-op unless launched with programmatic serialization
    float acc[4][4] = {};
    // staging: each thread loads 4 A and 4 W elements per BK slab
    float ra[4], rw[4];
    auto load = [&](int k0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int e = tid + i * 256;  // 0..1023 over (row, k) of a 64x16 tile
            const int r = e / BK, k = e % BK;
            const int m = m0 + r, n = n0 + r, kk = k0 + k;
            ra[i] = (m < a.M && kk < a.K) ? a_eff(a, m, kk, a.A[m * a.lda + kk]) : 0.0f;
            rw[i] = (n < a.N && kk < a.K) ? wload<WT>(a.W, n * a.ldw + kk) : 0.0f;
        }
    };
    auto store = [&](int buf) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int e = tid + i * 256;
            const int r = e / BK, k = e % BK;
            As[buf][k][r] = ra[i];
            Ws[buf][k][r] = rw[i];
        }
    };
    const int nk = (a.K + BK - 1) / BK;
    load(0);
    store(0);
    __syncthreads();
    for (int kt = 0; kt < nk; ++kt) {
        const int buf = kt & 1;
        if (kt + 1 < nk) load((kt + 1) * BK);
#pragma unroll
        for (int k = 0; k < BK; ++k) {
            const float4 av = *reinterpret_cast<const float4*>(&As[buf][k][ty * 4]);
            const float4 wv = *reinterpret_cast<const float4*>(&Ws[buf][k][tx * 4]);
            const float am[4] = {av.x, av.y, av.z, av.w};
            const float wn[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(am[i], wn[j], acc[i][j]);
        }
        if (kt + 1 < nk) store(buf ^ 1);
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + ty * 4 + i;
        if (m >= a.M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + tx * 4 + j;
            if (n < a.N) a.C[m * a.ldc + n] = epilogue(a, m, n, acc[i][j]);
        }
    }
}

template <int WT>
int launch_wt(const GemmArgs& a, cudaStream_t st, bool pdl) {
    if (a.M <= kGemvRows) {
        const size_t smem = ((size_t)a.M * a.K + 2 * kGemvRows) * sizeof(float);
        if (smem > 200 * 1024) return fail(SN_E_INVAL, "gemm: K=%d too large for the row path", a.K);
        static int attr_set = 0;
        if (!attr_set) {
            SN_TRY(cuda_check(cudaFuncSetAttribute(gemv_rows_kernel<WT>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   200 * 1024),
                              "gemv smem"));
            attr_set = 1;
        }
        int ctas = (a.N + 7) / 8;
        const int cap = 2 * rt().num_sms;
        if (ctas > cap) ctas = cap;
        SN_TRY(cuda_check(launch_pdl(gemv_rows_kernel<WT>, dim3(ctas), dim3(256), smem, st, a),
                          "gemv launch"));
    } else {
        if (a.ln_inline) return fail(SN_E_INVAL, "gemm: in-kernel LN statistics need M <= 8");
        dim3 grid((a.N + BN - 1) / BN, (a.M + BM - 1) / BM);
        SN_TRY(cuda_check(launch_pdl_if(pdl, gemm_tiled_kernel<WT>, grid, dim3(256), 0, st, a),
                          "gemm launch"));
    }
    return cuda_check(cudaGetLastError(), "gemm launch");
}

}  // namespace

int launch_gemm(const GemmArgs& a, int wtype, cudaStream_t st, const TcWeights* tc, bool pdl) {
    if (a.M <= 0 || a.N <= 0 || a.K <= 0) return SN_OK;
    if (tc && tc_usable(a, tc)) return launch_tc_gemm(a, *tc, st);
    switch (wtype) {
        case kWI8: return launch_wt<kWI8>(a, st, pdl);
        case kWF16: return launch_wt<kWF16>(a, st, pdl);
        default: return launch_wt<kWF32>(a, st, pdl);
    }
}

}  // namespace sn
