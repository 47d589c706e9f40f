// tcgen05 / TMEM contraction for the batched token loop (see tc_gemm.cuh).
//
// One CTA computes a 128 x BN tile of C with the whole K loop, through an
// S-deep shared-memory ring of K-slabs of 64 (one 128-byte swizzle row of bf16):
//   warps 0-3  A producers: thread t owns row m0+t, loads 64 fp32 of it,
//              applies the row-LN prologue, splits into bf16 hi/lo and stores
//              both in the SWIZZLE_128B K-major layout the MMA descriptor
//              expects (16-byte chunk c of row r at r*128 + ((c ^ r%8) * 16)
//              inside its 1024-byte 8-row atom); then the epilogue
//   warp 4     W producer: TMA 2-D tile loads of the hi/lo weight planes
//              (SWIZZLE_128B, no multicast) signalled through complete_tx
//   warp 5     TMEM allocation and the single MMA-issuing thread:
//              tcgen05.mma.cta_group::1.kind::f16, M=128, N=BN, K=16, three
//              products per K step (Ah*Wh, Ah*Wl, Al*Wh; two for INT8),
//              tcgen05.commit frees a stage / signals the accumulator
// Epilogue: tcgen05.ld 32x32b (warp w reads TMEM lanes 32w..32w+31 = its
// rows) into registers, the shared gemm_epilogue, 16-byte global stores.
// Every mbarrier wait is bounded; a role that gives up sets the error word,
// drains its own in-flight TMA/MMA work and the CTA frees its TMEM.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdio>

#include "ptx.cuh"
#include "runtime.cuh"
#include "tc_gemm.cuh"

namespace sn {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // bf16 per slab row = 128 bytes
constexpr int kThreads = 192;

template <int BN>
struct TcCfg {
    static constexpr int A_BYTES = BM * 128;
    static constexpr int W_BYTES = BN * 128;
    static constexpr int STAGE = 2 * A_BYTES + 2 * W_BYTES;
    static constexpr int S = BN == 128 ? 3 : (BN == 64 ? 4 : 5);
    static constexpr int SMEM = S * STAGE + 1024 + 256;
};

__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu)  // start address
           | ((uint64_t)1u << 16)               // leading byte offset (16 B, unused for SW128 K-major)
           | ((uint64_t)64u << 32)              // stride byte offset: 1024 B between 8-row atoms
           | ((uint64_t)1u << 46)               // descriptor version (sm_100)
           | ((uint64_t)2u << 61);              // SWIZZLE_128B
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, int x, int y,
                                            uint64_t* mbar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
        "%3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(tm), "r"(x), "r"(y), "r"(smem_u32(mbar))
        : "memory");
}

__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                       uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* b) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(b))
        : "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
        "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
        "%30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);  // .x = a (low half), .y = b
    return *reinterpret_cast<const uint32_t*>(&h);
}

template <int BN, bool I8>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmh, const __grid_constant__ CUtensorMap tml,
                   GemmArgs a, int* err) {
    using C = TcCfg<BN>;
    constexpr int S = C::S;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* sb = smem_raw + (((raw + 1023u) & ~1023u) - raw);  // 1024-B aligned ring
    uint64_t* a_full = reinterpret_cast<uint64_t*>(sb + S * C::STAGE);
    uint64_t* w_full = a_full + S;
    uint64_t* empty = w_full + S;
    uint64_t* acc_full = empty + S;
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(acc_full + 1);
    volatile int* give_up = reinterpret_cast<volatile int*>(acc_full + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int nk = (a.K + BK - 1) / BK;
    auto stage_ptr = [&](int s, int part) -> uint8_t* {  // 0 Ah, 1 Al, 2 Wh, 3 Wl
        return sb + s * C::STAGE +
               (part < 2 ? part * C::A_BYTES : 2 * C::A_BYTES + (part - 2) * C::W_BYTES);
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&a_full[s], 128);
            mbar_init(&w_full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(acc_full, 1);
        *give_up = 0;
        fence_mbar_init();
    }
    if (warp == 5) {  // TMEM accumulator: BN fp32 columns x 128 lanes
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32((const void*)tmem_slot)),
                     "r"((uint32_t)BN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp < 4) {  // ------------------------------------------ A producers
        const int t = threadIdx.x;
        const int m = m0 + t;
        const bool live = m < a.M;
        const float mu = (live && a.mu) ? a.mu[m] : 0.0f;
        const float rs = (live && a.mu) ? a.rs[m] : 0.0f;
        const float* arow = a.A + (long long)(live ? m : 0) * a.lda;
        const uint32_t r8 = t & 7;
        const uint32_t row_off = (t >> 3) * 1024 + r8 * 128;
        // the next slab's 64 values are loaded while this one is converted
        float4 nx[16];
        auto load_slab = [&](int kt) {
#pragma unroll
            for (int q = 0; q < 16; ++q) {
                const int k = kt * BK + 4 * q;
                nx[q] = (live && k < a.K) ? *reinterpret_cast<const float4*>(arow + k)
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        };
        load_slab(0);
        for (int kt = 0; kt < nk; ++kt) {
            const int s = kt % S;
            float4 cur[16];
#pragma unroll
            for (int q = 0; q < 16; ++q) cur[q] = nx[q];
            if (kt + 1 < nk) load_slab(kt + 1);
            if (kt >= S && !mbar_wait(&empty[s], ((kt / S) - 1) & 1, err)) {
                *give_up = 1;
                break;
            }
            const int k0 = kt * BK;
            uint8_t* ah = stage_ptr(s, 0) + row_off;
            uint8_t* al = stage_ptr(s, 1) + row_off;
#pragma unroll
            for (int c = 0; c < 8; ++c) {  // 8 values per 16-byte chunk
                const int k = k0 + 8 * c;
                float v[8] = {cur[2 * c].x,     cur[2 * c].y,     cur[2 * c].z,
                              cur[2 * c].w,     cur[2 * c + 1].x, cur[2 * c + 1].y,
                              cur[2 * c + 1].z, cur[2 * c + 1].w};
                if (a.mu && live && k < a.K) {  // K % 8 == 0: a chunk is all in or all out
                    const float4 g0 = __ldg(reinterpret_cast<const float4*>(a.g + k));
                    const float4 g1 = __ldg(reinterpret_cast<const float4*>(a.g + k + 4));
                    const float4 c0 = __ldg(reinterpret_cast<const float4*>(a.c + k));
                    const float4 c1 = __ldg(reinterpret_cast<const float4*>(a.c + k + 4));
                    const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
                    const float cc[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        v[j] = __fmul_rn(__fmul_rn(v[j] - mu, rs), gg[j]) + cc[j];
                }
                float lo[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float h = __bfloat162float(__float2bfloat16_rn(v[j]));
                    lo[j] = v[j] - h;
                }
                const uint32_t sw = ((uint32_t)c ^ r8) * 16;
                *reinterpret_cast<uint4*>(ah + sw) =
                    make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]),
                               pack_bf16(v[6], v[7]));
                *reinterpret_cast<uint4*>(al + sw) =
                    make_uint4(pack_bf16(lo[0], lo[1]), pack_bf16(lo[2], lo[3]),
                               pack_bf16(lo[4], lo[5]), pack_bf16(lo[6], lo[7]));
            }
            fence_proxy_async();  // generic-proxy smem writes -> visible to the tensor core
            mbar_arrive(&a_full[s]);
        }
    } else if (warp == 4) {  // ----------------------------------- W producer
        if (lane == 0) {
            int issued = 0;
            for (int kt = 0; kt < nk; ++kt) {
                const int s = kt % S;
                if (*give_up) break;
                if (kt >= S && !mbar_wait(&empty[s], ((kt / S) - 1) & 1, err)) {
                    *give_up = 1;
                    break;
                }
                mbar_expect_tx(&w_full[s], I8 ? C::W_BYTES : 2 * C::W_BYTES);
                tma_load_2d(stage_ptr(s, 2), &tmh, kt * BK, n0, &w_full[s]);
                if (!I8) tma_load_2d(stage_ptr(s, 3), &tml, kt * BK, n0, &w_full[s]);
                issued = kt + 1;
            }
            // never leave with a tile load in flight: wait for the last use of each stage
            for (int kt = issued - S < 0 ? 0 : issued - S; kt < issued; ++kt)
                mbar_wait(&w_full[kt % S], (kt / S) & 1, err);
        }
    } else {  // ----------------------------------------------- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = (1u << 4)                    // D: f32
                                   | (1u << 7) | (1u << 10)     // A, B: bf16
                                   | ((uint32_t)(BN >> 3) << 17)  // N
                                   | ((uint32_t)(BM >> 4) << 24);  // M
            for (int kt = 0; kt < nk; ++kt) {
                const int s = kt % S;
                if (!mbar_wait(&a_full[s], (kt / S) & 1, err) ||
                    !mbar_wait(&w_full[s], (kt / S) & 1, err)) {
                    *give_up = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t ah = smem_u32(stage_ptr(s, 0)), al = smem_u32(stage_ptr(s, 1));
                const uint32_t wh = smem_u32(stage_ptr(s, 2)), wl = smem_u32(stage_ptr(s, 3));
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk) {
                    const uint32_t off = kk * 32;  // 16 bf16 along K inside the swizzle row
                    const uint32_t acc = (kt > 0 || kk > 0) ? 1u : 0u;
                    tc_mma(tmem, sw128_desc(ah + off), sw128_desc(wh + off), idesc, acc);
                    if (!I8) tc_mma(tmem, sw128_desc(ah + off), sw128_desc(wl + off), idesc, 1u);
                    tc_mma(tmem, sw128_desc(al + off), sw128_desc(wh + off), idesc, 1u);
                }
                tc_commit(&empty[s]);  // stage reusable once these MMAs have read it
            }
            tc_commit(acc_full);  // accumulator complete (or: no MMA left in flight)
        }
    }

    // ------------------------------------------------------------- epilogue
    if (warp < 4) {
        const bool ok = mbar_wait(acc_full, 0, err);
        tc_fence_after();
        if (ok && !*give_up) {
            // 32x32 blocks go through shared memory (the idle ring) so that a
            // warp touches one 128-byte row segment per global access
            float* stg = reinterpret_cast<float*>(sb) + warp * (32 * 33);
#pragma unroll 1
            for (int j0 = 0; j0 < BN; j0 += 32) {
                float v[32];
                tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)j0, v);
#pragma unroll
                for (int j = 0; j < 32; ++j) stg[lane * 33 + j] = v[j];
                __syncwarp();
                const int n = n0 + j0 + lane;
#pragma unroll 4
                for (int r = 0; r < 32; ++r) {
                    const int mm = m0 + warp * 32 + r;
                    if (mm < a.M && n < a.N)
                        a.C[(long long)mm * a.ldc + n] = gemm_epilogue(a, mm, n, stg[r * 33 + lane]);
                }
                __syncwarp();
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"((uint32_t)BN)
                     : "memory");
    }
}

__global__ void split_bf16_kernel(const void* __restrict__ W, int wtype, long long n,
                                  __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        float v;
        if (wtype == kWI8) v = (float)reinterpret_cast<const int8_t*>(W)[i];
        else if (wtype == kWF16) v = __half2float(reinterpret_cast<const __half*>(W)[i]);
        else v = reinterpret_cast<const float*>(W)[i];
        const __nv_bfloat16 h = __float2bfloat16_rn(v);
        hi[i] = h;
        if (lo) lo[i] = __float2bfloat16_rn(v - __bfloat162float(h));
    }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point, so the
// library has no link-time dependency on libcuda (it loads on GPU-less hosts).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
        else
            cudaGetLastError();
    }
    return fn;
}

int encode_map(CUtensorMap* tm, const void* base, int N, int K, int box_rows) {
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)N};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(SN_E_DEVICE, "cuTensorMapEncodeTiled entry point unavailable");
    const CUresult r = enc(
        tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? SN_OK : fail(SN_E_DEVICE, "cuTensorMapEncodeTiled failed (%d)", (int)r);
}

template <int BN, bool I8>
int launch_bn(const GemmArgs& a, const TcWeights& tw, cudaStream_t st) {
    using C = TcCfg<BN>;
    static bool attr = false;
    auto k = tc_gemm_kernel<BN, I8>;
    if (!attr) {
        SN_TRY(cuda_check(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               C::SMEM),
                          "tc smem"));
        attr = true;
    }
    const int bi = BN == 32 ? 0 : (BN == 64 ? 1 : 2);
    dim3 grid((a.N + BN - 1) / BN, (a.M + BM - 1) / BM);
    k<<<grid, kThreads, C::SMEM, st>>>(tw.tm_hi[bi], tw.tm_lo[bi], a, rt().d_err);
    return cuda_check(cudaGetLastError(), "tc_gemm launch");
}

}  // namespace

int tc_prepare(TcWeights* tw, const void* W, int wtype, int N, int K,
               void* (*alloc)(size_t, void*), void* owner) {
    tw->N = N;
    tw->K = K;
    tw->int8 = wtype == kWI8;
    tw->ready = false;
    if (K % 8 != 0) return SN_OK;  // TMA row stride must be a multiple of 16 bytes
    const size_t n = (size_t)N * K;
    tw->hi = (__nv_bfloat16*)alloc(n * 2, owner);
    tw->lo = tw->int8 ? nullptr : (__nv_bfloat16*)alloc(n * 2, owner);
    if (!tw->hi || (!tw->int8 && !tw->lo)) return fail(SN_E_NOMEM, "tc weight planes");
    split_bf16_kernel<<<grid_blocks((long long)n), 256>>>(W, wtype, (long long)n, tw->hi, tw->lo);
    SN_TRY(cuda_check(cudaGetLastError(), "split launch"));
    const int rows[3] = {32, 64, 128};
    for (int i = 0; i < 3; ++i) {
        SN_TRY(encode_map(&tw->tm_hi[i], tw->hi, N, K, rows[i]));
        SN_TRY(encode_map(&tw->tm_lo[i], tw->int8 ? tw->hi : tw->lo, N, K, rows[i]));
    }
    tw->ready = true;
    return SN_OK;
}

bool tc_usable(const GemmArgs& a, const TcWeights* tw) {
    static int disabled = -1;
    if (disabled < 0) {
        const char* e = getenv("SN_DISABLE_TC");
        disabled = e && atoi(e) ? 1 : 0;
    }
    return !disabled && tw && tw->ready && a.M >= 16 && a.K == tw->K && a.N == tw->N &&
           a.K % 8 == 0 && a.lda % 4 == 0 && ((uintptr_t)a.A % 16) == 0;
}

int launch_tc_gemm(const GemmArgs& a, const TcWeights& tw, cudaStream_t st) {
    // widest tile that still gives about a wave of CTAs
    const long long mt = (a.M + BM - 1) / BM;
    const long long sms = rt().num_sms;
    int bn = 32;
    if (mt * ((a.N + 127) / 128) >= sms * 3 / 4) bn = 128;
    else if (mt * ((a.N + 63) / 64) >= sms * 3 / 4) bn = 64;
    if (tw.int8) {
        if (bn == 128) return launch_bn<128, true>(a, tw, st);
        if (bn == 64) return launch_bn<64, true>(a, tw, st);
        return launch_bn<32, true>(a, tw, st);
    }
    if (bn == 128) return launch_bn<128, false>(a, tw, st);
    if (bn == 64) return launch_bn<64, false>(a, tw, st);
    return launch_bn<32, false>(a, tw, st);
}

}  // namespace sn
