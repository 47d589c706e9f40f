// Batched W4A8 contraction on the tensor cores: tcgen05.mma kind::i8 with
// int32 accumulators in TMEM, bit-identical to the reference GEMV.
//
// Reference: sunnynet/runtime/quant.c (sn_gemv_i4 89-154). For a sequence row
// m and an output row n, with q the unsigned 4-bit weight codes, xq the int8
// activation codes of the row's block quantisation (sc = amax/127, 1 if zero;
// xq = rint(x/sc) clamped to +-127) and xsum their per-block sums:
//   acc = 0; for each block b in order:
//       acc = acc + (s_w[n][b]*s_x[m][b]) * (float)(dot_b - 8*xsum[m][b])
// with dot_b = sum over the block of q*xq (exact integer). The integer dots
// are what the tensor cores compute exactly; the block-ordered fp32
// accumulation stays in the epilogue with round-to-nearest mul/add, so every
// output equals the SIMT GEMV's (and the reference's) bit for bit.
//
// Two launches per contraction:
//   quant_rows_kernel  activation rows -> codes (M,K) int8 + per-block scale
//                      and code sum (a warp per (row, block), the reference's
//                      arithmetic), once per contraction
//   w4a8_tc_kernel     one CTA per 128 sequences x BN output rows; K walks in
//                      128-byte slabs through an S-deep shared-memory ring
//     warp 0     TMA: activation codes (SWIZZLE_128B box 128x128) and the
//                packed nibble rows (box 64 B x BN), one complete_tx barrier
//     warps 6-9  dequant in the mainloop: unpack each slab's nibbles to u8
//                codes in the 128-byte swizzled K-major layout the MMA reads
//                (byte k of a block holds codes k and k+block/2), then a proxy
//                fence and an arrive
//     warp 1     TMEM (2 x BN int32 columns); one thread issues block/32
//                MMAs (M=128, N=BN, K=32; A s8, B u8) per quantisation block
//                into one of two accumulator slots, commits the slot
//     warps 2-5  per block: tcgen05.ld the slot (warp w reads TMEM lanes of
//                quarter w%4 = its 32 sequences), release it, accumulate in
//                block order in registers; finally the epilogue and stores
// Every wait is bounded; a role that gives up records the error and leaves
// its loop, the MMA issuer waits for its own MMAs, the TMA issuer for its own
// loads, and the CTA frees its TMEM.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "kernels.cuh"
#include "runtime.cuh"
#include "tcgen05.cuh"

namespace sn {
namespace {

constexpr int kBM = 128;
constexpr int kSlab = 128;  // K bytes (= int8 codes) per stage
constexpr int kW4Threads = 320;
constexpr int kW4Stages = 4;

template <int BN>
struct W4Cfg {
    static constexpr int A_BYTES = kBM * kSlab;  // activation codes, swizzled
    static constexpr int U_BYTES = BN * kSlab;   // unpacked weight codes, swizzled
    static constexpr int P_BYTES = BN * kSlab / 2;  // packed nibbles as loaded
    static constexpr int STAGE = A_BYTES + U_BYTES + P_BYTES;  // multiple of 1024
};

__device__ __forceinline__ float load_scale_w(const void* s, size_t i, bool fp16) {
    return fp16 ? __half2float(reinterpret_cast<const __half*>(s)[i])
                : reinterpret_cast<const float*>(s)[i];
}

__device__ __forceinline__ void w4_apply(float* y, float v, int epi) {
    switch (epi) {
        case kW4Add: *y = *y + v; break;
        case kW4Relu2: {
            const float t = v > 0.0f ? v : 0.0f;
            *y = t * t;
        } break;
        case kW4Tanh: *y = tanhf(v); break;
        case kW4Sigmoid: *y = 1.0f / (1.0f + expf(-v)); break;
        default: *y = v;
    }
}

// Warp per (row, block): the reference's activation quantisation.
__global__ void quant_rows_kernel(const float* __restrict__ X, int M, int K, int block,
                                  int8_t* __restrict__ codes, float* __restrict__ sx,
                                  int* __restrict__ xsum) {
    const int nb = K / block;
    const int lane = threadIdx.x & 31;
    const long long w = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5);
    if (w >= (long long)M * nb) return;
    const int m = (int)(w / nb), b = (int)(w % nb);
    const float* xb = X + (size_t)m * K + (size_t)b * block;
    float mx = 0.0f;
    for (int i = lane; i < block; i += 32) mx = fmaxf(mx, fabsf(xb[i]));
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float sc = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 1.0f;
    const float inv = __fdiv_rn(1.0f, sc);
    int sum = 0;
    for (int i = lane; i < block; i += 32) {
        int t = __float2int_rn(__fmul_rn(xb[i], inv));
        t = min(max(t, -127), 127);
        codes[(size_t)m * K + (size_t)b * block + i] = (int8_t)t;
        sum += t;
    }
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) {
        sx[(size_t)m * nb + b] = sc;
        xsum[(size_t)m * nb + b] = sum;
    }
}

template <int BN, bool FP16S>
__global__ void __launch_bounds__(kW4Threads, 1)
    w4a8_tc_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmw,
                   float* __restrict__ Y, const void* __restrict__ scale,
                   const float* __restrict__ sxg, const int* __restrict__ xsg, int M, int N, int K,
                   int block, int epi, int* err) {
    using C = W4Cfg<BN>;
    constexpr int S = kW4Stages;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* ring = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    const int nb = K / block, nslab = K / kSlab, bps = kSlab / block, mpb = block / 32;
    float* sw_s = reinterpret_cast<float*>(ring + S * C::STAGE);  // [BN][nb]
    float* sx_s = sw_s + BN * nb;                                 // [128][nb]
    int* xs_s = reinterpret_cast<int*>(sx_s + kBM * nb);          // [128][nb]
    uint64_t* full = reinterpret_cast<uint64_t*>(xs_s + kBM * nb + ((BN * nb) & 1));
    uint64_t* wready = full + S;
    uint64_t* empty = wready + S;
    uint64_t* accf = empty + S;  // [2]
    uint64_t* acce = accf + 2;   // [2]
    uint64_t* done = acce + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* give_up = reinterpret_cast<volatile int*>(tmem_slot + 1);
    auto sA = [&](int s) { return ring + s * C::STAGE; };
    auto sU = [&](int s) { return ring + s * C::STAGE + C::A_BYTES; };
    auto sP = [&](int s) { return ring + s * C::STAGE + C::A_BYTES + C::U_BYTES; };

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * BN;
    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&wready[s], 128);
            mbar_init(&empty[s], 1);
        }
        for (int j = 0; j < 2; ++j) {
            mbar_init(&accf[j], 1);
            mbar_init(&acce[j], 128);
        }
        mbar_init(done, 1);
        *give_up = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, 2 * BN);
    for (int i = tid; i < BN * nb; i += kW4Threads) {
        const int j = i / nb, b = i - j * nb, n = n0 + j;
        sw_s[i] = n < N ? load_scale_w(scale, (size_t)n * nb + b, FP16S) : 0.0f;
    }
    for (int i = tid; i < kBM * nb; i += kW4Threads) {
        const int r = i / nb, m = m0 + r;
        sx_s[i] = m < M ? sxg[(size_t)m0 * nb + i] : 0.0f;
        xs_s[i] = m < M ? xsg[(size_t)m0 * nb + i] : 0;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {  // --------------------------------------------------- TMA
        if (lane == 0) {
            int issued = 0;
            for (int s = 0; s < nslab; ++s) {
                const int st = s % S;
                if (*give_up) break;
                if (s >= S && !mbar_wait(&empty[st], ((s / S) - 1) & 1, err)) {
                    *give_up = 1;
                    break;
                }
                mbar_expect_tx(&full[st], C::A_BYTES + C::P_BYTES);
                tma_load_2d(sA(st), &tma, s * kSlab, m0, &full[st]);
                tma_load_2d(sP(st), &tmw, s * (kSlab / 2), n0, &full[st]);
                issued = s + 1;
            }
            for (int s = issued - S < 0 ? 0 : issued - S; s < issued; ++s)
                mbar_wait(&full[s % S], (s / S) & 1, err);  // no load left in flight
        }
    } else if (warp >= 6) {  // ----------------------------------- unpack nibbles
        const int ut = tid - 192, half = block / 2;
        for (int s = 0; s < nslab; ++s) {
            const int st = s % S;
            if (*give_up) break;
            if (!mbar_wait(&full[st], (s / S) & 1, err)) {
                *give_up = 1;
                break;
            }
            const uint8_t* P = sP(st);
            uint8_t* U = sU(st);
            for (int c = ut; c < BN * 4; c += 128) {
                const int row = c >> 2, pb = (c & 3) * 16;  // 16 packed bytes of this row
                const int bb = pb / half, j0 = pb - bb * half;
                const uint4 w = *reinterpret_cast<const uint4*>(P + row * (kSlab / 2) + pb);
                const uint4 lo = make_uint4(w.x & 0x0F0F0F0Fu, w.y & 0x0F0F0F0Fu,
                                            w.z & 0x0F0F0F0Fu, w.w & 0x0F0F0F0Fu);
                const uint4 hi = make_uint4((w.x >> 4) & 0x0F0F0F0Fu, (w.y >> 4) & 0x0F0F0F0Fu,
                                            (w.z >> 4) & 0x0F0F0F0Fu, (w.w >> 4) & 0x0F0F0F0Fu);
                const int clo = bb * block + j0, chi = clo + half;  // 16-code chunks
                *reinterpret_cast<uint4*>(U + row * kSlab + (((clo >> 4) ^ (row & 7)) << 4)) = lo;
                *reinterpret_cast<uint4*>(U + row * kSlab + (((chi >> 4) ^ (row & 7)) << 4)) = hi;
            }
            fence_proxy_async_smem();  // the MMA reads U through the async proxy
            mbar_arrive(&wready[st]);
        }
    } else if (warp == 1) {  // --------------------------------------------- MMA
        if (lane == 0) {
            const uint32_t idesc = (2u << 4)                        // D: s32
                                   | (1u << 7)                      // A: s8
                                   | (0u << 10)                     // B: u8
                                   | ((uint32_t)(BN >> 3) << 17)    // N
                                   | ((uint32_t)(kBM >> 4) << 24);  // M
            int b = 0;
            bool ok = true;
            for (int s = 0; s < nslab && ok; ++s) {
                const int st = s % S;
                if (!mbar_wait(&wready[st], (s / S) & 1, err)) {
                    *give_up = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t aa = smem_u32(sA(st)), ua = smem_u32(sU(st));
                for (int bb = 0; bb < bps; ++bb, ++b) {
                    const int slot = b & 1;
                    if (b >= 2 && !mbar_wait(&acce[slot], ((b >> 1) - 1) & 1, err)) {
                        *give_up = 1;
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    for (int kk = 0; kk < mpb; ++kk) {
                        const uint32_t off = (uint32_t)(bb * block + kk * 32);
                        tc_mma_i8(tmem + (uint32_t)(slot * BN), sw128_desc(aa + off),
                                  sw128_desc(ua + off), idesc, kk > 0 ? 1u : 0u);
                    }
                    tc_commit(&accf[slot]);
                }
                tc_commit(&empty[st]);
            }
            tc_commit(done);
            mbar_wait(done, 0, err);  // every MMA issued here has completed
        }
    } else {  // ----------------------------------------------- epilogue, warps 2-5
        const int q = warp & 3, r = q * 32 + lane, m = m0 + r;
        float acc[BN];
#pragma unroll
        for (int j = 0; j < BN; ++j) acc[j] = 0.0f;
        bool ok = true;
        for (int b = 0; b < nb; ++b) {
            const int slot = b & 1;
            if (*give_up || !mbar_wait(&accf[slot], (b >> 1) & 1, err)) {
                *give_up = 1;
                ok = false;
                break;
            }
            tc_fence_after();
            const float xs = sx_s[r * nb + b];
            const int x8 = 8 * xs_s[r * nb + b];
#pragma unroll
            for (int j0 = 0; j0 < BN; j0 += 32) {
                uint32_t d[32];
                tmem_ld32_u(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(slot * BN + j0), d);
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const float f = (float)((int)d[j] - x8);
                    acc[j0 + j] = __fadd_rn(acc[j0 + j],
                                            __fmul_rn(__fmul_rn(sw_s[(j0 + j) * nb + b], xs), f));
                }
            }
            tc_fence_before();
            mbar_arrive(&acce[slot]);
        }
        if (ok && m < M) {
            float* yr = Y + (size_t)m * N;
#pragma unroll
            for (int j = 0; j < BN; ++j)
                if (n0 + j < N) w4_apply(yr + n0 + j, acc[j], epi);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * BN);
    }
}

// Workspace for the activation codes of one contraction (reused in stream
// order). Grown outside graph capture only; a superseded buffer stays
// allocated because captured graphs may still reference it.
struct W4Work {
    void* p = nullptr;
    size_t cap = 0;
};
W4Work& w4_work() {
    static W4Work w;
    return w;
}

size_t w4_work_bytes(int M, int K, int block) {
    const size_t nb = (size_t)(K / block);
    return (((size_t)M * K + 255) / 256) * 256 + (size_t)M * nb * 8;
}

template <int BN, bool FP16S>
int launch_bn(const CUtensorMap& ta, const CUtensorMap& tw, float* Y, const void* scale,
              const float* sx, const int* xs, int M, int N, int K, int block, int epi,
              cudaStream_t st) {
    using C = W4Cfg<BN>;
    const int nb = K / block;
    const size_t smem = 1024 + (size_t)kW4Stages * C::STAGE + 4ull * (BN * nb + 2 * kBM * nb) +
                        8 + 8ull * (3 * kW4Stages + 5) + 16;
    static int attr = 0;
    if (!attr) {
        SN_TRY(cuda_check(cudaFuncSetAttribute(w4a8_tc_kernel<BN, FP16S>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               200 * 1024),
                          "w4a8_tc smem attr"));
        attr = 1;
    }
    if (smem > 200 * 1024) return fail(SN_E_INVAL, "w4a8_tc: K=%d needs too much shared memory", K);
    const dim3 grid((N + BN - 1) / BN, (M + kBM - 1) / kBM);
    w4a8_tc_kernel<BN, FP16S><<<grid, kW4Threads, smem, st>>>(ta, tw, Y, scale, sx, xs, M, N, K,
                                                              block, epi, rt().d_err);
    return cuda_check(cudaGetLastError(), "w4a8_tc launch");
}

}  // namespace

bool w4a8_tc_ok(int M, int K, int N, int block, const void* Wq) {
    return M >= 16 && N >= 32 && K % kSlab == 0 && (block == 32 || block == 64 || block == 128) &&
           (uintptr_t)Wq % 16 == 0 && !getenv("SN_DISABLE_TC");
}

bool w4a8_tc_ready(int M, int K, int block) {
    return w4_work().cap >= w4_work_bytes(M, K, block);
}

int w4a8_tc_reserve(int M, int K, int block) {
    W4Work& w = w4_work();
    const size_t need = w4_work_bytes(M, K, block);
    if (w.cap >= need) return SN_OK;
    void* p = nullptr;
    if (cudaMalloc(&p, need) != cudaSuccess) {
        cudaGetLastError();
        return fail(SN_E_NOMEM, "w4a8_tc: %zu bytes of activation codes", need);
    }
    w.p = p;  // the previous buffer is kept: captured graphs may still use it
    w.cap = need;
    return SN_OK;
}

int launch_w4a8_tc(float* Y, const float* X, const uint8_t* Wq, const void* scale, int M, int K,
                   int N, int block, bool fp16, int epi, cudaStream_t st) {
    W4Work& w = w4_work();
    if (w.cap < w4_work_bytes(M, K, block))
        return fail(SN_E_INVAL, "w4a8_tc: activation workspace not reserved");
    const int nb = K / block;
    int8_t* codes = static_cast<int8_t*>(w.p);
    float* sx = reinterpret_cast<float*>(static_cast<char*>(w.p) + (((size_t)M * K + 255) / 256) * 256);
    int* xs = reinterpret_cast<int*>(sx + (size_t)M * nb);
    {
        const long long warps = (long long)M * nb;
        quant_rows_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(X, M, K, block, codes, sx, xs);
        SN_TRY(cuda_check(cudaGetLastError(), "w4a8_tc quant launch"));
    }
    const int mt = (M + kBM - 1) / kBM;
    const int BN = (long long)((N + 63) / 64) * mt >= rt().num_sms ? 64 : 32;
    CUtensorMap ta, tw;
    SN_TRY(encode_tiled(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, codes, K, M, K, kSlab, kBM,
                        CU_TENSOR_MAP_SWIZZLE_128B));
    SN_TRY(encode_tiled(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, Wq, K / 2, N, K / 2, kSlab / 2, BN,
                        CU_TENSOR_MAP_SWIZZLE_NONE));
    if (BN == 64)
        return fp16 ? launch_bn<64, true>(ta, tw, Y, scale, sx, xs, M, N, K, block, epi, st)
                    : launch_bn<64, false>(ta, tw, Y, scale, sx, xs, M, N, K, block, epi, st);
    return fp16 ? launch_bn<32, true>(ta, tw, Y, scale, sx, xs, M, N, K, block, epi, st)
                : launch_bn<32, false>(ta, tw, Y, scale, sx, xs, M, N, K, block, epi, st);
}

}  // namespace sn
