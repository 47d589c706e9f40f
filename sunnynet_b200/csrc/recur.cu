// Generic first-order recurrence and INT8 quantisation on sm_100a.
//
// Reference: sunnynet/runtime/recur.c (sn_recur_scan 13-48, sn_recur_step
// 109-131, sn_quant_i8 134-161, sn_dequant_i8 163-178).
//
// Bit-exactness. The reference vectorises 8 channels with an FMA,
// s = fma(a, s, b) with b = (1-a)*u rounded separately, and runs the N%8
// remainder channels through scalar ISO-C code without contraction
// (s = a*s + b, two roundings). The kernels below apply the same per-channel
// rule with explicit __fmaf_rn / __fmul_rn / __fadd_rn, so every output is
// bit-identical to the reference.
//
// Scan layout. One CTA owns CW adjacent channels of one sequence and walks T
// in chunks of TC rows through an S-deep shared-memory ring:
//   warp 0  loader   cp.async 16B (or 4B) copies of a and b/u rows -> ring
//   warp 1  helper   gated form: b = (1-a)*u in place (same rounding as ref)
//   warp 2  chain    lane = channel, s = fma(a,s,b) per row, result over b
//   warp 3  storer   coalesced row stores of the results
// Stages are handed on with mbarriers (full -> ready -> done -> empty); every
// wait is bounded and records an error instead of hanging. The sequential
// chain is the only serial part: ~one dependent FFMA per row.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "kernels.cuh"
#include "ptx.cuh"
#include "recur.h"
#include "runtime.cuh"
#include "tc_gemm.cuh"
#include "tcgen05.cuh"

namespace sn {
namespace {

constexpr int kTC = 128;  // rows per chunk

template <int CW>
struct ScanCfg {
    static constexpr int S = CW == 8 ? 12 : (CW == 16 ? 7 : 4);  // ring depth (~100-128 KB)
    // a launch uses min(S, chunks) stages: short sequences keep more CTAs per SM
    static size_t smem(int stages) {
        return 2ull * stages * kTC * CW * sizeof(float) + 4ull * stages * 8;
    }
};

__device__ __forceinline__ float rec_fused(float a, float s, float b) { return __fmaf_rn(a, s, b); }
__device__ __forceinline__ float rec_split(float a, float s, float b) {
    return __fadd_rn(__fmul_rn(a, s), b);
}

// The serial part: kTC rows of one channel (stride CW in shared memory),
// s = fma(a, s, b), result written over b. The next 16 rows are loaded into
// registers before the current 16 are chained, so the only dependency left
// per row is the FMA itself (restrict: the a and b tiles never alias).
template <int CW>
__device__ __forceinline__ float chain_chunk(const float* __restrict__ pa, float* __restrict__ pb,
                                             float s) {
    constexpr int G = 16;
    float ca[G], cb[G];
#pragma unroll
    for (int j = 0; j < G; ++j) {
        ca[j] = pa[j * CW];
        cb[j] = pb[j * CW];
    }
#pragma unroll
    for (int g = 0; g < kTC / G; ++g) {
        float na[G], nb[G];
        if (g + 1 < kTC / G) {
#pragma unroll
            for (int j = 0; j < G; ++j) {
                na[j] = pa[((g + 1) * G + j) * CW];
                nb[j] = pb[((g + 1) * G + j) * CW];
            }
        }
#pragma unroll
        for (int j = 0; j < G; ++j) {
            s = rec_fused(ca[j], s, cb[j]);
            pb[(g * G + j) * CW] = s;
        }
        if (g + 1 < kTC / G) {
#pragma unroll
            for (int j = 0; j < G; ++j) {
                ca[j] = na[j];
                cb[j] = nb[j];
            }
        }
    }
    return s;
}

template <int CW>
__global__ void __launch_bounds__(128)
    scan_exact_kernel(const float* __restrict__ a, const float* __restrict__ b,
                      const float* s0, float* __restrict__ out, float* send, int T, int N,
                      int nv, int gated, int vec, long long s0_ld, long long send_ld,
                      __nv_bfloat16* __restrict__ ph, __nv_bfloat16* __restrict__ pl,
                      int* err) {
    constexpr int TILE = kTC * CW;
    const int S = min(ScanCfg<CW>::S, (T + kTC - 1) / kTC);  // stages of this launch
    extern __shared__ __align__(128) unsigned char smem_raw[];
    float* sa = reinterpret_cast<float*>(smem_raw);
    float* sb = sa + S * TILE;
    uint64_t* full = reinterpret_cast<uint64_t*>(sb + S * TILE);
    uint64_t* ready = full + S;
    uint64_t* done = ready + S;
    uint64_t* empty = done + S;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bb = blockIdx.y;
    const int d0 = blockIdx.x * CW;
    const size_t base = (size_t)bb * T * N;
    const int nch = (T + kTC - 1) / kTC;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 32);
            mbar_init(&ready[i], 32);
            mbar_init(&done[i], 32);
            mbar_init(&empty[i], 32);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == 0) {  // ---------------------------------------------- loader
        for (int c = 0; c < nch; ++c) {
            const int st = c % S;
            if (c >= S && !__all_sync(~0u, mbar_wait(&empty[st], ((c / S) - 1) & 1, err))) break;
            const int t0 = c * kTC;
            float* da = sa + st * TILE;
            float* db = sb + st * TILE;
            if (vec) {
                constexpr int Q = CW / 4;
#pragma unroll 4
                for (int i = lane; i < kTC * Q; i += 32) {
                    const int r = i / Q, q = i % Q;
                    const int t = t0 + r, d = d0 + 4 * q;
                    const bool ok = t < T && d < N;
                    const size_t off = ok ? base + (size_t)t * N + d : 0;
                    cp_async16(da + r * CW + 4 * q, a + off, ok ? 16u : 0u);
                    cp_async16(db + r * CW + 4 * q, b + off, ok ? 16u : 0u);
                }
            } else {
                for (int i = lane; i < TILE; i += 32) {
                    const int r = i / CW, ch = i % CW;
                    const int t = t0 + r, d = d0 + ch;
                    const bool ok = t < T && d < N;
                    const size_t off = ok ? base + (size_t)t * N + d : 0;
                    cp_async4(da + i, a + off, ok ? 4u : 0u);
                    cp_async4(db + i, b + off, ok ? 4u : 0u);
                }
            }
            cp_async_arrive(&full[st]);
        }
        cp_async_wait_all();
    } else if (warp == 1) {  // --------------------------------------- helper
        for (int c = 0; c < nch; ++c) {
            const int st = c % S;
            if (!__all_sync(~0u, mbar_wait(&full[st], (c / S) & 1, err))) break;
            if (gated) {
                float4* da = reinterpret_cast<float4*>(sa + st * TILE);
                float4* db = reinterpret_cast<float4*>(sb + st * TILE);
#pragma unroll 4
                for (int i = lane; i < TILE / 4; i += 32) {
                    const float4 x = da[i];
                    float4 u = db[i];
                    u.x = __fmul_rn(__fsub_rn(1.0f, x.x), u.x);
                    u.y = __fmul_rn(__fsub_rn(1.0f, x.y), u.y);
                    u.z = __fmul_rn(__fsub_rn(1.0f, x.z), u.z);
                    u.w = __fmul_rn(__fsub_rn(1.0f, x.w), u.w);
                    db[i] = u;
                }
            }
            mbar_arrive(&ready[st]);
        }
    } else if (warp == 2) {  // ---------------------------------------- chain
        const int d = d0 + lane;
        const bool live = lane < CW && d < N;
        float s = live ? s0[(size_t)bb * s0_ld + d] : 0.0f;
        // the state entering each position, as bf16 planes: row 0 is s0 (rows
        // t >= 1 are out row t - 1, written by the storer)
        if (ph && live) store_split(ph, pl, base + d, s);
        const bool all_fused = d0 + CW <= nv;
        const bool fused = d < nv;
        for (int c = 0; c < nch; ++c) {
            const int st = c % S;
            if (!__all_sync(~0u, mbar_wait(&ready[st], (c / S) & 1, err))) {
                s = __int_as_float(0x7fc00000);  // the final state is unknown
                break;
            }
            const int rows = min(kTC, T - c * kTC);
            if (lane < CW) {
                const float* pa = sa + st * TILE + lane;
                float* pb = sb + st * TILE + lane;
                if (all_fused && rows == kTC) {
                    s = chain_chunk<CW>(pa, pb, s);
                } else {
                    for (int r = 0; r < rows; ++r) {
                        const float av = pa[r * CW], bv = pb[r * CW];
                        s = fused ? rec_fused(av, s, bv) : rec_split(av, s, bv);
                        pb[r * CW] = s;
                    }
                }
            }
            mbar_arrive(&done[st]);
        }
        if (live) send[(size_t)bb * send_ld + d] = s;
    } else {  // ------------------------------------------------------ storer
        for (int c = 0; c < nch; ++c) {
            const int st = c % S;
            if (!__all_sync(~0u, mbar_wait(&done[st], (c / S) & 1, err))) break;
            const int t0 = c * kTC;
            const int rows = min(kTC, T - t0);
            const float* db = sb + st * TILE;
            if (vec) {
                constexpr int Q = CW / 4;
                for (int i = lane; i < rows * Q; i += 32) {
                    const int r = i / Q, q = i % Q;
                    const int d = d0 + 4 * q;
                    if (d < N) {
                        const float4 v = *reinterpret_cast<const float4*>(db + r * CW + 4 * q);
                        const size_t o = base + (size_t)(t0 + r) * N + d;
                        *reinterpret_cast<float4*>(out + o) = v;
                        if (ph && t0 + r + 1 < T) {  // the state entering position t + 1
                            const float x[4] = {v.x, v.y, v.z, v.w};
                            __nv_bfloat16 h[4], l[4];
#pragma unroll
                            for (int j = 0; j < 4; ++j) {  // store_split's rounding
                                h[j] = __float2bfloat16_rn(x[j]);
                                l[j] = __float2bfloat16_rn(x[j] - __bfloat162float(h[j]));
                            }
                            *reinterpret_cast<uint2*>(ph + o + N) = *reinterpret_cast<const uint2*>(h);
                            *reinterpret_cast<uint2*>(pl + o + N) = *reinterpret_cast<const uint2*>(l);
                        }
                    }
                }
            } else {
                for (int i = lane; i < rows * CW; i += 32) {
                    const int r = i / CW, ch = i % CW;
                    const int d = d0 + ch;
                    if (d < N) {
                        const size_t o = base + (size_t)(t0 + r) * N + d;
                        out[o] = db[i];
                        if (ph && t0 + r + 1 < T) store_split(ph, pl, o + N, db[i]);
                    }
                }
            }
            __syncwarp();
            mbar_arrive(&empty[st]);
        }
    }
}

template <int CW>
int launch_scan_cw(const float* a, const float* b, const float* s0, float* out, float* send,
                   int B, int T, int N, int gated, int vec, long long s0_ld, long long send_ld,
                   __nv_bfloat16* ph, __nv_bfloat16* pl, cudaStream_t st, int nv) {
    static bool attr = false;
    const int nch = (T + kTC - 1) / kTC;
    const size_t smem = ScanCfg<CW>::smem(nch < ScanCfg<CW>::S ? nch : ScanCfg<CW>::S);
    if (!attr) {  // the largest ring this kernel can take
        SN_TRY(cuda_check(cudaFuncSetAttribute(scan_exact_kernel<CW>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)ScanCfg<CW>::smem(ScanCfg<CW>::S)),
                          "scan smem attr"));
        attr = true;
    }
    dim3 grid((N + CW - 1) / CW, B);
    scan_exact_kernel<CW><<<grid, 128, smem, st>>>(a, b, s0, out, send, T, N, nv, gated,
                                                   vec, s0_ld, send_ld, ph, pl, rt().d_err);
    return cuda_check(cudaGetLastError(), "scan launch");
}

// Channels per CTA: enough CTAs to cover the SMs, wide rows when there are
// plenty. SN_SCAN_CW (8/16/32) overrides, for tuning sweeps.
int pick_cw(int B, int N) {
    static int forced = -1;
    if (forced < 0) {
        const char* e = getenv("SN_SCAN_CW");
        forced = e ? atoi(e) : 0;
    }
    if (forced == 8 || forced == 16 || forced == 32) return forced;
    const long long sms = rt().num_sms;
    if ((long long)B * ((N + 31) / 32) >= 2 * sms) return 32;
    if ((long long)B * ((N + 15) / 16) >= sms) return 16;
    return 8;
}

// ------------------------------------------------------- reverse pass (bwd)
// sn_recur_bwd (reference recur.c:51-107). Per channel, from t = T-1 down to
// 0: g = dout_t + g, then da_t = g*(s_{t-1} - u_t) and db_t = g*(1 - a_t) for
// the gated form (da_t = g*s_{t-1}, db_t = g for the FMA form), then
// g = g*a_t; s_{-1} = s0 and ds0 = g after t = 0. The reference rounds every
// operation separately, in its AVX2 lanes and in its N%8 scalar tail alike,
// so one rule with explicit round-to-nearest operations is bit-exact for
// every channel.
//
// Layout: one CTA owns CW adjacent channels of one sequence and walks T
// backwards in chunks of kBT rows through an S-deep ring of four row tiles
// (a, b/u, the state entering each row, dout):
//   warp 0     loader    cp.async of the four tiles; the state entering row t
//                        is out row t-1, or s0 for t = 0
//   warp 1     chain     lane = channel: g = dout + g, written over dout; g *= a
//   warps 2-3  epilogue  da, db from g, a, b and the entering state; row stores
// Stages are handed on with mbarriers (full: loader -> chain, done: chain ->
// epilogue, empty: epilogue -> loader); every wait is bounded and a warp that
// gives up leaves its loop (the chain then reports ds0 as NaN).
constexpr int kBT = 64;  // rows per chunk of the reverse walk

template <int CW>
struct BwdCfg {
    static constexpr int S = CW == 8 ? 12 : (CW == 16 ? 6 : 4);  // ring depth (~96-128 KB)
    static size_t smem(int stages) {
        return 4ull * stages * kBT * CW * sizeof(float) + 3ull * stages * 8;
    }
};

// kBT rows of one channel (stride CW), walked from the last row down: g =
// dout + g written over dout, g *= a. The next 16 rows are read into
// registers before the current 16 are chained.
template <int CW>
__device__ __forceinline__ float bwd_chain(const float* __restrict__ pa, float* __restrict__ pg,
                                           float g) {
    constexpr int G = 16, NG = kBT / G;
    float ca[G], cg[G];
#pragma unroll
    for (int j = 0; j < G; ++j) {
        ca[j] = pa[((NG - 1) * G + j) * CW];
        cg[j] = pg[((NG - 1) * G + j) * CW];
    }
#pragma unroll
    for (int gi = NG - 1; gi >= 0; --gi) {
        float na[G], ng[G];
        if (gi > 0) {
#pragma unroll
            for (int j = 0; j < G; ++j) {
                na[j] = pa[((gi - 1) * G + j) * CW];
                ng[j] = pg[((gi - 1) * G + j) * CW];
            }
        }
#pragma unroll
        for (int j = G - 1; j >= 0; --j) {
            g = __fadd_rn(cg[j], g);
            pg[(gi * G + j) * CW] = g;
            g = __fmul_rn(g, ca[j]);
        }
        if (gi > 0) {
#pragma unroll
            for (int j = 0; j < G; ++j) {
                ca[j] = na[j];
                cg[j] = ng[j];
            }
        }
    }
    return g;
}

__device__ __forceinline__ void bwd_grads(float g, float av, float bv, float sp, int gated,
                                          float* x, float* y) {
    if (gated) {
        *x = __fmul_rn(g, __fsub_rn(sp, bv));
        *y = __fmul_rn(g, __fsub_rn(1.0f, av));
    } else {
        *x = __fmul_rn(g, sp);
        *y = g;
    }
}

template <int CW>
__global__ void __launch_bounds__(128)
    scan_bwd_kernel(const float* __restrict__ a, const float* __restrict__ b,
                    const float* __restrict__ s0, const float* __restrict__ out,
                    const float* __restrict__ dout, float* __restrict__ da,
                    float* __restrict__ db, float* __restrict__ ds0, int T, int N, int gated,
                    int vec, int* err) {
    constexpr int TILE = kBT * CW;
    const int nch = (T + kBT - 1) / kBT;
    const int S = min(BwdCfg<CW>::S, nch);  // stages of this launch
    extern __shared__ __align__(128) unsigned char smem_raw[];
    float* ta = reinterpret_cast<float*>(smem_raw);  // [S][TILE] a
    float* tb = ta + S * TILE;                       // b (u when gated)
    float* tp = tb + S * TILE;                       // the state entering each row
    float* tg = tp + S * TILE;                       // dout, then g
    uint64_t* full = reinterpret_cast<uint64_t*>(tg + S * TILE);
    uint64_t* done = full + S;
    uint64_t* empty = done + S;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bb = blockIdx.y, d0 = blockIdx.x * CW;
    const size_t base = (size_t)bb * T * N;
    const float* s0b = s0 + (size_t)bb * N;
    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 32);
            mbar_init(&done[i], 32);
            mbar_init(&empty[i], 64);
        }
        fence_mbar_init();
    }
    __syncthreads();

    // step k of the walk handles chunk nch-1-k of the sequence, in stage k % S
    if (warp == 0) {  // ---------------------------------------------- loader
        for (int k = 0; k < nch; ++k) {
            const int st = k % S;
            if (k >= S && !__all_sync(~0u, mbar_wait(&empty[st], ((k / S) - 1) & 1, err))) break;
            const int t0 = (nch - 1 - k) * kBT;
            float* pa = ta + st * TILE;
            float* pb = tb + st * TILE;
            float* pp = tp + st * TILE;
            float* pg = tg + st * TILE;
            if (vec) {
                constexpr int Q = CW / 4;
#pragma unroll 2
                for (int i = lane; i < kBT * Q; i += 32) {
                    const int r = i / Q, q = i % Q;
                    const int t = t0 + r, d = d0 + 4 * q;
                    const bool ok = t < T && d < N;
                    const size_t off = ok ? base + (size_t)t * N + d : 0;
                    const float* ps = !ok ? a : (t > 0 ? out + off - N : s0b + d);
                    const uint32_t n = ok ? 16u : 0u;
                    cp_async16(pa + r * CW + 4 * q, a + off, n);
                    cp_async16(pb + r * CW + 4 * q, b + off, n);
                    cp_async16(pp + r * CW + 4 * q, ps, n);
                    cp_async16(pg + r * CW + 4 * q, dout + off, n);
                }
            } else {
                for (int i = lane; i < TILE; i += 32) {
                    const int r = i / CW, ch = i % CW;
                    const int t = t0 + r, d = d0 + ch;
                    const bool ok = t < T && d < N;
                    const size_t off = ok ? base + (size_t)t * N + d : 0;
                    const float* ps = !ok ? a : (t > 0 ? out + off - N : s0b + d);
                    const uint32_t n = ok ? 4u : 0u;
                    cp_async4(pa + i, a + off, n);
                    cp_async4(pb + i, b + off, n);
                    cp_async4(pp + i, ps, n);
                    cp_async4(pg + i, dout + off, n);
                }
            }
            cp_async_arrive(&full[st]);
        }
        cp_async_wait_all();
    } else if (warp == 1) {  // ---------------------------------------- chain
        const int d = d0 + lane;
        float g = 0.0f;
        for (int k = 0; k < nch; ++k) {
            const int st = k % S;
            if (!__all_sync(~0u, mbar_wait(&full[st], (k / S) & 1, err))) {
                g = __int_as_float(0x7fc00000);  // the gradient of s0 is unknown
                break;
            }
            const int rows = min(kBT, T - (nch - 1 - k) * kBT);
            if (lane < CW) {
                const float* pa = ta + st * TILE + lane;
                float* pg = tg + st * TILE + lane;
                if (rows == kBT) {
                    g = bwd_chain<CW>(pa, pg, g);
                } else {
                    for (int r = rows - 1; r >= 0; --r) {
                        g = __fadd_rn(pg[r * CW], g);
                        pg[r * CW] = g;
                        g = __fmul_rn(g, pa[r * CW]);
                    }
                }
            }
            mbar_arrive(&done[st]);
        }
        if (lane < CW && d < N) ds0[(size_t)bb * N + d] = g;
    } else {  // ------------------------------------------------------ epilogue
        const int e = threadIdx.x - 64;
        for (int k = 0; k < nch; ++k) {
            const int st = k % S;
            if (!__all_sync(~0u, mbar_wait(&done[st], (k / S) & 1, err))) break;
            const int t0 = (nch - 1 - k) * kBT;
            const int rows = min(kBT, T - t0);
            const float* pa = ta + st * TILE;
            const float* pb = tb + st * TILE;
            const float* pp = tp + st * TILE;
            const float* pg = tg + st * TILE;
            if (vec) {
                constexpr int Q = CW / 4;
                for (int i = e; i < rows * Q; i += 64) {
                    const int r = i / Q, q = i % Q;
                    const int d = d0 + 4 * q;
                    if (d >= N) continue;
                    const int j = r * CW + 4 * q;
                    const float4 G4 = *reinterpret_cast<const float4*>(pg + j);
                    const float4 A4 = *reinterpret_cast<const float4*>(pa + j);
                    const float4 B4 = *reinterpret_cast<const float4*>(pb + j);
                    const float4 P4 = *reinterpret_cast<const float4*>(pp + j);
                    float4 X, Y;
                    bwd_grads(G4.x, A4.x, B4.x, P4.x, gated, &X.x, &Y.x);
                    bwd_grads(G4.y, A4.y, B4.y, P4.y, gated, &X.y, &Y.y);
                    bwd_grads(G4.z, A4.z, B4.z, P4.z, gated, &X.z, &Y.z);
                    bwd_grads(G4.w, A4.w, B4.w, P4.w, gated, &X.w, &Y.w);
                    const size_t o = base + (size_t)(t0 + r) * N + d;
                    *reinterpret_cast<float4*>(da + o) = X;
                    *reinterpret_cast<float4*>(db + o) = Y;
                }
            } else {
                for (int i = e; i < rows * CW; i += 64) {
                    const int r = i / CW, ch = i % CW;
                    const int d = d0 + ch;
                    if (d >= N) continue;
                    float x, y;
                    bwd_grads(pg[i], pa[i], pb[i], pp[i], gated, &x, &y);
                    const size_t o = base + (size_t)(t0 + r) * N + d;
                    da[o] = x;
                    db[o] = y;
                }
            }
            mbar_arrive(&empty[st]);
        }
    }
}

template <int CW>
int launch_bwd_cw(const float* a, const float* b, const float* s0, const float* out,
                  const float* dout, float* da, float* db, float* ds0, int B, int T, int N,
                  int gated, int vec, cudaStream_t st) {
    static const cudaError_t attr_rc = cudaFuncSetAttribute(  // the largest ring, once
        scan_bwd_kernel<CW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
        (int)BwdCfg<CW>::smem(BwdCfg<CW>::S));
    SN_TRY(cuda_check(attr_rc, "scan bwd smem attr"));
    const int nch = (T + kBT - 1) / kBT;
    const size_t smem = BwdCfg<CW>::smem(nch < BwdCfg<CW>::S ? nch : BwdCfg<CW>::S);
    dim3 grid((N + CW - 1) / CW, B);
    scan_bwd_kernel<CW><<<grid, 128, smem, st>>>(a, b, s0, out, dout, da, db, ds0, T, N, gated,
                                                 vec, rt().d_err);
    return cuda_check(cudaGetLastError(), "scan bwd launch");
}

}  // namespace

// Device-pointer scan used by the ABI entry points and by the model code.
int launch_scan(const float* a, const float* b, const float* s0, float* out, float* send, int B,
                int T, int N, int gated, cudaStream_t st) {
    return launch_scan_strided(a, b, s0, N, out, send, N, B, T, N, gated, nullptr, nullptr, st);
}

int launch_scan_strided(const float* a, const float* b, const float* s0, long long s0_ld,
                        float* out, float* send, long long send_ld, int B, int T, int N,
                        int gated, __nv_bfloat16* ph, __nv_bfloat16* pl, cudaStream_t st,
                        int nv) {
    if (B > 65535) return fail(SN_E_INVAL, "recur_scan: B=%d exceeds 65535", B);
    if (nv < 0) nv = N - N % 8;
    // (plane stores are 8-byte vectors of four channels on the vector path)
    const bool vec = N % 4 == 0 && ((uintptr_t)a % 16 == 0) && ((uintptr_t)b % 16 == 0) &&
                     ((uintptr_t)out % 16 == 0) &&
                     (!ph || ((uintptr_t)ph % 8 == 0 && (uintptr_t)pl % 8 == 0));
    switch (pick_cw(B, N)) {
        case 32: return launch_scan_cw<32>(a, b, s0, out, send, B, T, N, gated, vec, s0_ld, send_ld, ph, pl, st, nv);
        case 16: return launch_scan_cw<16>(a, b, s0, out, send, B, T, N, gated, vec, s0_ld, send_ld, ph, pl, st, nv);
        default: return launch_scan_cw<8>(a, b, s0, out, send, B, T, N, gated, vec, s0_ld, send_ld, ph, pl, st, nv);
    }
}

// Reverse pass of the scan on device arrays (sn_recur_bwd).
int launch_scan_bwd(const float* a, const float* b, const float* s0, const float* out,
                    const float* dout, float* da, float* db, float* ds0, int B, int T, int N,
                    int gated, cudaStream_t st) {
    if (B > 65535) return fail(SN_E_INVAL, "recur_bwd: B=%d exceeds 65535", B);
    auto al = [](const void* p) { return (uintptr_t)p % 16 == 0; };
    const int vec = N % 4 == 0 && al(a) && al(b) && al(s0) && al(out) && al(dout) && al(da) &&
                    al(db);
    switch (pick_cw(B, N)) {
        case 32: return launch_bwd_cw<32>(a, b, s0, out, dout, da, db, ds0, B, T, N, gated, vec, st);
        case 16: return launch_bwd_cw<16>(a, b, s0, out, dout, da, db, ds0, B, T, N, gated, vec, st);
        default: return launch_bwd_cw<8>(a, b, s0, out, dout, da, db, ds0, B, T, N, gated, vec, st);
    }
}

// ------------------------------------------------------- chunked scan (mode 1)
// The recurrence is an affine map per row, s -> a*s + b, and affine maps
// compose associatively: (A1,B1) then (A2,B2) is (A2*A1, A2*B1 + B2). Mode 1
// cuts T into chunks of L rows and runs three kernels:
//   agg    thread per (seq, chunk, channel): the chunk's composed map (A, B),
//          B chained from 0 with the reference's per-row rule
//   carry  per (seq, channel), over chunks: carry_c = A_c*carry_{c-1} + B_c,
//          a two-level pass (32 warps split the chunks, a shuffle scan of
//          the 32 warp totals, then each warp re-applies its chunks); the
//          state entering chunk c replaces A_c in the record
//   apply  same threads as agg: re-run the chunk's rows from its carry with
//          the reference rule, write every row; the last chunk writes send
// Rows are read twice, the second time mostly from L2 (the agg pass just
// pulled them in). Only the carry entering each chunk is composed, so the
// outputs differ from the sequential scan by rounding of that composition
// (a few ulp of the state per chunk boundary), not bit for bit.
// Record layout: agg[(seq*nch + c)*N + n] = float2 (A or carry, B).
// The agg and apply kernels stage their tile (rows of the CTA's channels, a
// and b) in shared memory, by TMA for full 128-channel tiles (two buffers in
// flight, results stored back by bulk copies) and by cp.async otherwise, so
// a CTA has whole rounds of rows in flight instead of a few rows per thread.
namespace {

constexpr int kSub = 32;        // rows staged per round
constexpr int kScanTile = 128;  // channels per CTA: a 32 KB tile, 7 CTAs per SM

__device__ __forceinline__ float gate_b(float av, float uv, int gated) {
    return gated ? __fmul_rn(__fsub_rn(1.0f, av), uv) : uv;
}

// rows x tpb floats of a and b, starting at element off0 (row stride N,
// channel n0 of the tile at column 0) -> sa, sb (row stride tpb). Channels
// >= N are zero-filled. vec: 16-byte copies (N % 4 == 0, 16-byte bases).
__device__ __forceinline__ void stage_rows(float* sa, float* sb, const float* a, const float* b,
                                           size_t off0, int rows, int N, int n0, int tpb,
                                           bool vec) {
    if (vec) {
        const int q4 = tpb >> 2;
        for (int i = threadIdx.x; i < rows * q4; i += blockDim.x) {
            const int r = i / q4, q = i - r * q4;
            const bool ok = n0 + 4 * q < N;
            const size_t g = ok ? off0 + (size_t)r * N + 4 * q : 0;
            cp_async16(sa + r * tpb + 4 * q, a + g, ok ? 16u : 0u);
            cp_async16(sb + r * tpb + 4 * q, b + g, ok ? 16u : 0u);
        }
    } else {
        for (int i = threadIdx.x; i < rows * tpb; i += blockDim.x) {
            const int r = i / tpb, ch = i - r * tpb;
            const bool ok = n0 + ch < N;
            const size_t g = ok ? off0 + (size_t)r * N + ch : 0;
            cp_async4(sa + i, a + g, ok ? 4u : 0u);
            cp_async4(sb + i, b + g, ok ? 4u : 0u);
        }
    }
    cp_async_wait_all();
    __syncthreads();
}

// Full 128-channel tiles are staged by TMA instead: boxes of 8 rows x 128
// channels of a and b (tensor maps over the (B*T, N) arrays; rows or
// channels past the end read as zero), issued by one thread. Rows past the
// chunk's end (up to 7) are loaded and not used.
constexpr int kBoxRows = 8;

// Full 128-channel tiles by TMA run as a two-buffer pipeline: rounds of
// kRound rows (a then b), round k in buffer k & 1 with its own mbarrier, so
// round k + 1 lands while round k is consumed; the apply kernel writes its
// results over the consumed a rows and stores each row by one bulk copy.
// Both buffers together take the same 32 KB as the kSub staging area.
constexpr int kRound = 16;
constexpr int kBufF = 2 * kRound * kScanTile;  // floats per buffer
static_assert(2 * kBufF == 2 * kSub * kScanTile, "pipeline buffers share the staging area");

// One thread: issue round rows [row0, row0 + min(kRound, left)) of tile n0
// into buffer `buf`, completing on `bar`.
__device__ __forceinline__ void issue_round(float* buf, const CUtensorMap* ta,
                                            const CUtensorMap* tb, int row0, int left, int n0,
                                            uint64_t* bar) {
    fence_proxy_async_smem();  // the generic accesses of the buffer's last round come first
    const int nbox = ((left < kRound ? left : kRound) + kBoxRows - 1) / kBoxRows;
    mbar_expect_tx(bar, (uint32_t)(2 * nbox * kBoxRows * kScanTile * sizeof(float)));
    for (int i = 0; i < nbox; ++i) {
        tma_load_2d(buf + i * kBoxRows * kScanTile, ta, n0, row0 + i * kBoxRows, bar);
        tma_load_2d(buf + kRound * kScanTile + i * kBoxRows * kScanTile, tb, n0,
                    row0 + i * kBoxRows, bar);
    }
}

// Wait for round k (buffer k & 1) of the two-buffer TMA pipeline. The
// outcome is the same for every thread of the CTA: when any thread's bounded
// wait gave up, thread 0 first waits (bounded again) for the rounds still in
// flight into this CTA's shared memory, rounds k and k + 1, so no copy lands
// after the CTA has left; then all threads return true together.
__device__ __forceinline__ bool round_gave_up(uint64_t* bars, int k, int nr, int* err) {
    const bool bad = !mbar_wait(&bars[k & 1], (uint32_t)((k >> 1) & 1), err);
    if (!__syncthreads_or(bad)) return false;
    if (threadIdx.x == 0) {
        mbar_wait(&bars[k & 1], (uint32_t)((k >> 1) & 1), nullptr);
        if (k + 1 < nr) mbar_wait(&bars[(k + 1) & 1], (uint32_t)(((k + 1) >> 1) & 1), nullptr);
    }
    __syncthreads();
    return true;
}

__global__ void __launch_bounds__(256)
    scan_agg_kernel(const float* __restrict__ a, const float* __restrict__ b,
                    float2* __restrict__ agg, int T, int N, int nv, int L, int nch, int gated,
                    int vec, const __grid_constant__ CUtensorMap ta,
                    const __grid_constant__ CUtensorMap tb, int tma, int* err) {
    extern __shared__ __align__(16) unsigned char stile_raw[];
    __shared__ __align__(8) uint64_t bars[2];
    pdl_trigger();
    const int tpb = blockDim.x;
    // 128-byte aligned staging area (TMA destinations)
    float* stile = reinterpret_cast<float*>(
        stile_raw + (((smem_u32(stile_raw) + 127u) & ~127u) - smem_u32(stile_raw)));
    float* sa = stile;
    float* sb = stile + kSub * tpb;
    const int n0 = blockIdx.x * tpb, n = n0 + threadIdx.x;
    const int c = blockIdx.y, sq = blockIdx.z;
    const int t0 = c * L, rows = min(L, T - t0);
    const bool fused = n < nv;
    float A = 1.0f, Bc = 0.0f;
    if (tma) {
        const int nr = (rows + kRound - 1) / kRound;
        if (threadIdx.x == 0) {
            mbar_init(&bars[0], 1);
            mbar_init(&bars[1], 1);
            fence_mbar_init();
            for (int k = 0; k < 2 && k < nr; ++k)
                issue_round(stile + k * kBufF, &ta, &tb, sq * T + t0 + k * kRound,
                            rows - k * kRound, n0, &bars[k]);
        }
        __syncthreads();  // barriers initialised before anyone waits
        for (int k = 0; k < nr; ++k) {
            const int j = k & 1;
            if (round_gave_up(bars, k, nr, err)) {  // the chunk's map is unknown
                A = Bc = __int_as_float(0x7fc00000);
                break;
            }
            const float* ra = stile + j * kBufF;
            const float* rb = ra + kRound * kScanTile;
            const int rs = min(kRound, rows - k * kRound);
            for (int r = 0; r < rs; ++r) {
                const float av = ra[r * kScanTile + threadIdx.x];
                const float bv = gate_b(av, rb[r * kScanTile + threadIdx.x], gated);
                Bc = fused ? rec_fused(av, Bc, bv) : rec_split(av, Bc, bv);
                A = __fmul_rn(A, av);
            }
            __syncthreads();  // buffer j consumed
            if (threadIdx.x == 0 && k + 2 < nr)
                issue_round(stile + j * kBufF, &ta, &tb, sq * T + t0 + (k + 2) * kRound,
                            rows - (k + 2) * kRound, n0, &bars[j]);
        }
    } else {
        for (int r0 = 0; r0 < rows; r0 += kSub) {
            const int rs = min(kSub, rows - r0);
            if (r0) __syncthreads();  // the previous round is consumed
            stage_rows(sa, sb, a, b, ((size_t)sq * T + t0 + r0) * N + n0, rs, N, n0, tpb,
                       vec != 0);
            for (int r = 0; r < rs; ++r) {
                const float av = sa[r * tpb + threadIdx.x];
                const float bv = gate_b(av, sb[r * tpb + threadIdx.x], gated);
                Bc = fused ? rec_fused(av, Bc, bv) : rec_split(av, Bc, bv);
                A = __fmul_rn(A, av);
            }
        }
    }
    if (n < N) agg[((size_t)sq * nch + c) * N + n] = make_float2(A, Bc);
}

// Block: 32 channels x kCarryWarps (= 32) warps; warp w owns chunks
// [w*per, (w+1)*per). Each warp composes its chunks' maps (records read
// kCarryBatch at a time into registers, one L2 round trip per batch, and kept
// there when per <= kCarryBatch); the 32 warp totals of a channel are then
// scanned by one warp with shuffles (log2(32) compositions instead of a
// serial walk), and each warp re-applies its chunks from the carry entering
// them.
constexpr int kCarryWarps = 32;
constexpr int kCarryBatch = 8;

// (A1, B1) then (A2, B2): s -> A2*(A1*s + B1) + B2
__device__ __forceinline__ float2 compose(float2 first, float2 then) {
    return make_float2(__fmul_rn(then.x, first.x), __fmaf_rn(then.x, first.y, then.y));
}

__global__ void __launch_bounds__(kCarryWarps * 32)
    scan_carry_kernel(const float* __restrict__ s0, float2* __restrict__ agg, int N, int nch) {
    static_assert(kCarryWarps == 32, "one warp scans the warp totals");
    __shared__ float2 wtot[kCarryWarps][33];  // [warp][channel]: totals, then carries in
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int n = blockIdx.x * 32 + lane, sq = blockIdx.y;
    const bool live = n < N;
    const int per = (nch + kCarryWarps - 1) / kCarryWarps;
    const int c0 = min(nch, w * per), c1 = min(nch, c0 + per);
    float2* rec = agg + (size_t)sq * nch * N + n;
    const bool keep = per <= kCarryBatch;  // one batch: the records stay in registers
    float2 m[kCarryBatch];
    float A = 1.0f, Bc = 0.0f;  // composition of this warp's chunks
    for (int cb = c0; cb < c1; cb += kCarryBatch) {
#pragma unroll
        for (int j = 0; j < kCarryBatch; ++j)
            if (live && cb + j < c1) m[j] = ld_cg(rec + (size_t)(cb + j) * N);
#pragma unroll
        for (int j = 0; j < kCarryBatch; ++j) {
            if (live && cb + j < c1) {
                Bc = __fmaf_rn(m[j].x, Bc, m[j].y);
                A = __fmul_rn(m[j].x, A);
            }
        }
    }
    wtot[w][lane] = make_float2(A, Bc);
    __syncthreads();
    {   // warp v: exclusive scan over the warps' totals of channel v (lane = warp)
        const int v = w;
        float2 t = wtot[lane][v];
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const float2 e = make_float2(__shfl_up_sync(~0u, t.x, off), __shfl_up_sync(~0u, t.y, off));
            if (lane >= off) t = compose(e, t);
        }
        float2 ex = make_float2(__shfl_up_sync(~0u, t.x, 1), __shfl_up_sync(~0u, t.y, 1));
        if (lane == 0) ex = make_float2(1.0f, 0.0f);
        __syncthreads();  // every total read before the carries overwrite them
        wtot[lane][v] = ex;
    }
    __syncthreads();
    const float2 ex = wtot[w][lane];
    float s = live ? __fmaf_rn(ex.x, s0[(size_t)sq * N + n], ex.y) : 0.0f;
    for (int cb = c0; cb < c1; cb += kCarryBatch) {
        if (!keep) {
#pragma unroll
            for (int j = 0; j < kCarryBatch; ++j)
                if (live && cb + j < c1) m[j] = ld_cg(rec + (size_t)(cb + j) * N);
        }
#pragma unroll
        for (int j = 0; j < kCarryBatch; ++j) {
            if (live && cb + j < c1) {
                rec[(size_t)(cb + j) * N].x = s;
                s = __fmaf_rn(m[j].x, s, m[j].y);
            }
        }
    }
}

__global__ void __launch_bounds__(256)
    scan_apply_kernel(const float* __restrict__ a, const float* __restrict__ b,
                      const float2* __restrict__ agg, float* __restrict__ out,
                      float* __restrict__ send, int T, int N, int nv, int L, int nch, int gated,
                      int vec, const __grid_constant__ CUtensorMap ta,
                      const __grid_constant__ CUtensorMap tb, int tma, int* err) {
    extern __shared__ __align__(16) unsigned char stile_raw[];
    __shared__ __align__(8) uint64_t bars[2];
    const int tpb = blockDim.x;
    // 128-byte aligned staging area (TMA destinations)
    float* stile = reinterpret_cast<float*>(
        stile_raw + (((smem_u32(stile_raw) + 127u) & ~127u) - smem_u32(stile_raw)));
    float* sa = stile;
    float* sb = stile + kSub * tpb;
    const int n0 = blockIdx.x * tpb, n = n0 + threadIdx.x;
    const int c = blockIdx.y, sq = blockIdx.z;
    const int t0 = c * L, rows = min(L, T - t0);
    const bool fused = n < nv;
    const size_t base = ((size_t)sq * T + t0) * N;
    float s = 0.0f;
    if (tma) {
        const int nr = (rows + kRound - 1) / kRound;
        // results go back over the consumed a rows, out by one bulk copy per row
        const bool bulk_out = (reinterpret_cast<uintptr_t>(out) & 15) == 0;
        const int nval = N - n0 < kScanTile ? N - n0 : kScanTile;  // channels of this tile
        // a and b were complete before the agg kernel started: stage the first
        // rounds while the carry kernel still runs, then wait for the carries
        if (threadIdx.x == 0) {
            mbar_init(&bars[0], 1);
            mbar_init(&bars[1], 1);
            fence_mbar_init();
            for (int k = 0; k < 2 && k < nr; ++k)
                issue_round(stile + k * kBufF, &ta, &tb, sq * T + t0 + k * kRound,
                            rows - k * kRound, n0, &bars[k]);
        }
        __syncthreads();  // barriers initialised before anyone waits
        pdl_wait();
        s = n < N ? ld_cg(&agg[((size_t)sq * nch + c) * N + n]).x : 0.0f;
        for (int k = 0; k < nr; ++k) {
            const int j = k & 1;
            if (round_gave_up(bars, k, nr, err)) {
                // rows from this round on stay uncomputed: mark them NaN
                s = __int_as_float(0x7fc00000);
                if (n < N)
                    for (int r = k * kRound; r < rows; ++r) out[base + (size_t)r * N + n] = s;
                break;
            }
            float* ra = stile + j * kBufF;
            const float* rb = ra + kRound * kScanTile;
            const int rs = min(kRound, rows - k * kRound);
            const size_t rbase = base + (size_t)(k * kRound) * N;
            for (int r = 0; r < rs; ++r) {
                const float av = ra[r * kScanTile + threadIdx.x];
                const float bv = gate_b(av, rb[r * kScanTile + threadIdx.x], gated);
                s = fused ? rec_fused(av, s, bv) : rec_split(av, s, bv);
                if (bulk_out) ra[r * kScanTile + threadIdx.x] = s;
                else if (n < N) __stcs(out + rbase + (size_t)r * N + n, s);
            }
            if (bulk_out) {
                fence_proxy_async_smem();
                __syncthreads();  // the round's rows are complete
                if (threadIdx.x < rs) {
                    bulk_s2g(out + rbase + (size_t)threadIdx.x * N + n0,
                             ra + threadIdx.x * kScanTile, (uint32_t)nval * 4u);
                    bulk_commit();
                    bulk_wait_read_all();  // the buffer is reloaded below
                }
            }
            __syncthreads();  // buffer j consumed
            if (threadIdx.x == 0 && k + 2 < nr)
                issue_round(stile + j * kBufF, &ta, &tb, sq * T + t0 + (k + 2) * kRound,
                            rows - (k + 2) * kRound, n0, &bars[j]);
        }
    } else {
        stage_rows(sa, sb, a, b, base + n0, min(kSub, rows), N, n0, tpb, vec != 0);
        pdl_wait();
        s = n < N ? ld_cg(&agg[((size_t)sq * nch + c) * N + n]).x : 0.0f;
        for (int r0 = 0; r0 < rows; r0 += kSub) {
            const int rs = min(kSub, rows - r0);
            if (r0) {
                __syncthreads();
                stage_rows(sa, sb, a, b, base + (size_t)r0 * N + n0, rs, N, n0, tpb, vec != 0);
            }
            for (int r = 0; r < rs; ++r) {
                const float av = sa[r * tpb + threadIdx.x];
                const float bv = gate_b(av, sb[r * tpb + threadIdx.x], gated);
                s = fused ? rec_fused(av, s, bv) : rec_split(av, s, bv);
                if (n < N) __stcs(out + base + (size_t)(r0 + r) * N + n, s);
            }
        }
    }
    if (c == nch - 1 && n < N) send[(size_t)sq * N + n] = s;
}

}  // namespace

// Chunk length for mode 1: the shortest (>= 16 rows) whose (seq, chunk,
// channel tile) CTAs all fit in one wave at the agg / apply kernels' real
// occupancy (a second, partial wave would cost as much as the first), then
// longer until the records fit in `max_records` (<= 0: no limit). Returns 0
// when even one chunk per sequence does not fit.
int scan_chunk_rows(int B, int T, int N, int num_sms, long long max_records) {
    const int tpb = N >= kScanTile ? kScanTile : ((N + 31) / 32) * 32;
    const long long tiles = (long long)B * ((N + tpb - 1) / tpb);
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, scan_agg_kernel, tpb,
                                                      2ull * kSub * tpb * sizeof(float) + 128) !=
            cudaSuccess ||
        occ < 1) {
        cudaGetLastError();
        occ = 6;
    }
    const long long slots = (long long)num_sms * occ;
    long long L = ((long long)T * tiles + slots - 1) / slots;
    L = (L + kBoxRows - 1) / kBoxRows * kBoxRows;  // whole TMA boxes
    if (L < 16) L = 16;
    if (max_records > 0) {
        while ((long long)B * N * ((T + L - 1) / L) > max_records) {
            if (L >= T) return 0;
            L = L > T / 2 ? T : 2 * L;
        }
    }
    return (int)(L < T ? L : T);
}

long long scan_chunk_records(int B, int T, int N, int L) {
    return (long long)B * N * ((T + L - 1) / L);
}

int launch_scan_chunked(const float* a, const float* b, const float* s0, float* out,
                        float* send, int B, int T, int N, int gated, int L, float2* agg,
                        cudaStream_t st, bool prof_scopes, int* err) {
    if (!err) err = rt().d_err;
    if (B > 65535) return fail(SN_E_INVAL, "recur_scan: B=%d exceeds 65535", B);
    if (L <= 0 || L > T) return fail(SN_E_INVAL, "recur_scan: bad chunk length %d", L);
    const int nch = (T + L - 1) / L;
    if (nch > 65535) return fail(SN_E_INVAL, "recur_scan: %d chunks exceed 65535", nch);
    const int nv = N - N % 8;
    const int tpb = N >= kScanTile ? kScanTile : ((N + 31) / 32) * 32;
    const dim3 grid((N + tpb - 1) / tpb, nch, B);
    const size_t smem = 2ull * kSub * tpb * sizeof(float) + 128;  // + alignment slack
    const int vec = N % 4 == 0 && (uintptr_t)a % 16 == 0 && (uintptr_t)b % 16 == 0;
    // TMA staging for full 128-channel tiles (16-byte rows and bases)
    CUtensorMap ta, tb;
    memset(&ta, 0, sizeof ta);
    memset(&tb, 0, sizeof tb);
    int tma = vec && tpb == kScanTile && !getenv("SN_SCAN_NO_TMA");
    if (tma) {
        tma = encode_tiled(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a, N, (long long)B * T,
                           (long long)N * 4, kScanTile, kBoxRows, CU_TENSOR_MAP_SWIZZLE_NONE) ==
                  SN_OK &&
              encode_tiled(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, b, N, (long long)B * T,
                           (long long)N * 4, kScanTile, kBoxRows, CU_TENSOR_MAP_SWIZZLE_NONE) ==
                  SN_OK;
    }
    static const cudaError_t attr_rc = [] {  // once per process (thread-safe init)
        const int mx = (int)(2ull * kSub * kScanTile * sizeof(float) + 128);
        cudaError_t e = cudaFuncSetAttribute(scan_agg_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(scan_apply_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
        return e;
    }();
    SN_TRY(cuda_check(attr_rc, "scan smem attribute"));
    {
        ProfScope ps(prof_scopes ? "scan_agg" : nullptr, st);
        scan_agg_kernel<<<grid, tpb, smem, st>>>(a, b, agg, T, N, nv, L, nch, gated, vec, ta, tb,
                                                 tma, err);
        SN_TRY(cuda_check(cudaGetLastError(), "scan agg launch"));
    }
    {
        ProfScope ps(prof_scopes ? "scan_carry" : nullptr, st);
        SN_TRY(cuda_check(launch_pdl(scan_carry_kernel, dim3((N + 31) / 32, B),
                                     dim3(kCarryWarps * 32), 0, st, s0, agg, N, nch),
                          "scan carry launch"));
    }
    {
        ProfScope ps(prof_scopes ? "scan_apply" : nullptr, st);
        SN_TRY(cuda_check(launch_pdl(scan_apply_kernel, grid, dim3(tpb), smem, st, a, b,
                                     (const float2*)agg, out, send, T, N, nv, L, nch, gated,
                                     vec, ta, tb, tma, err),
                          "scan apply launch"));
    }
    return SN_OK;
}

// ------------------------------------------------------------------- step
__global__ void step_kernel(const float* __restrict__ a, const float* __restrict__ b,
                            float* __restrict__ s, long long total, int N, int nv, int gated) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const float av = a[i];
        const float bv = gated ? __fmul_rn(__fsub_rn(1.0f, av), b[i]) : b[i];
        const int d = (int)(i % N);
        s[i] = d < nv ? rec_fused(av, s[i], bv) : rec_split(av, s[i], bv);
    }
}

int launch_step(const float* a, const float* b, float* s, int B, int N, int gated,
                cudaStream_t st) {
    const long long total = (long long)B * N;
    const int blocks = grid_blocks(total);
    step_kernel<<<blocks, 256, 0, st>>>(a, b, s, total, N, N - N % 8, gated);
    return cuda_check(cudaGetLastError(), "step launch");
}

// ------------------------------------------------------------- INT8 quant
// One CTA per (row, block): amax by max-reduction (exact), then the reference
// arithmetic: sc = amax/127 (1 if amax == 0), inv = 1/sc, q = rint(x*inv).
__global__ void quant_i8_kernel(const float* __restrict__ x, int8_t* __restrict__ q,
                                float* __restrict__ scale, int N, int block, int nb) {
    const int k = blockIdx.x, row = blockIdx.y;
    const int lo = k * block, hi = min(N, lo + block);
    const float* xr = x + (size_t)row * N;
    float m = 0.0f;
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) m = fmaxf(m, fabsf(xr[i]));
    __shared__ float red[32];
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (threadIdx.x == 0) red[0] = m;
    }
    __syncthreads();
    const float amax = red[0];
    const float sc = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
    const float inv = __fdiv_rn(1.0f, sc);
    if (threadIdx.x == 0) scale[(size_t)row * nb + k] = sc;
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        float t = rintf(__fmul_rn(xr[i], inv));
        t = fminf(fmaxf(t, -127.0f), 127.0f);
        q[(size_t)row * N + i] = (int8_t)(int)t;
    }
}

__global__ void dequant_i8_kernel(const int8_t* __restrict__ q, const float* __restrict__ scale,
                                  float* __restrict__ x, long long total, int N, int block,
                                  int nb) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long row = i / N;
        const int col = (int)(i - row * N);
        x[i] = __fmul_rn((float)q[i], scale[row * nb + col / block]);
    }
}

}  // namespace sn

using namespace sn;

// ======================================================== C-ABI entry points
namespace {

int do_scan(const float* a, const float* b, const float* s0, float* out, float* send, int B,
            int T, int N, int gated) {
    if (!a || !b || !s0 || !out || !send || B <= 0 || T <= 0 || N <= 0)
        return fail(SN_E_INVAL, "recur_scan: null pointer or non-positive dimension");
    SN_TRY(ensure_init());
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    const size_t big = (size_t)B * T * N * sizeof(float), small = (size_t)B * N * sizeof(float);
    Arr A, Bv, S0, O, SE;
    SN_TRY(stage_in(a, big, 0, &A));
    SN_TRY(stage_in(b, big, 1, &Bv));
    SN_TRY(stage_in(s0, small, 2, &S0));
    SN_TRY(stage_out(out, big, 3, &O));
    SN_TRY(stage_out(send, small, 4, &SE));
    if (rt().scan_mode == 1) {
        const int L = scan_chunk_rows(B, T, N, rt().num_sms, 0);
        const size_t rb = (size_t)scan_chunk_records(B, T, N, L) * sizeof(float2);
        void* agg = scratch(10, rb);
        if (!agg) return fail(SN_E_NOMEM, "recur_scan: %zu bytes of chunk records", rb);
        SN_TRY(launch_scan_chunked((const float*)A.dev, (const float*)Bv.dev,
                                   (const float*)S0.dev, (float*)O.dev, (float*)SE.dev, B, T, N,
                                   gated ? 1 : 0, L, (float2*)agg, stream()));
    } else {
        SN_TRY(launch_scan((const float*)A.dev, (const float*)Bv.dev, (const float*)S0.dev,
                           (float*)O.dev, (float*)SE.dev, B, T, N, gated ? 1 : 0, stream()));
    }
    SN_TRY(copy_back(O));
    SN_TRY(copy_back(SE));
    return finish(O.host || SE.host || A.dev != a || Bv.dev != b || S0.dev != s0);
}

int do_bwd(const float* a, const float* b, const float* s0, const float* out, const float* dout,
           float* da, float* db, float* ds0, int B, int T, int N, int gated) {
    if (!a || !b || !s0 || !out || !dout || !da || !db || !ds0 || B <= 0 || T <= 0 || N <= 0)
        return fail(SN_E_INVAL, "recur_bwd: null pointer or non-positive dimension");
    SN_TRY(ensure_init());
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    const size_t big = (size_t)B * T * N * sizeof(float), small = (size_t)B * N * sizeof(float);
    Arr A, Bv, S0, O, DO, DA, DB, D0;
    SN_TRY(stage_in(a, big, 0, &A));
    SN_TRY(stage_in(b, big, 1, &Bv));
    SN_TRY(stage_in(s0, small, 2, &S0));
    SN_TRY(stage_in(out, big, 3, &O));
    SN_TRY(stage_in(dout, big, 4, &DO));
    SN_TRY(stage_out(da, big, 5, &DA));
    SN_TRY(stage_out(db, big, 6, &DB));
    SN_TRY(stage_out(ds0, small, 7, &D0));
    SN_TRY(launch_scan_bwd((const float*)A.dev, (const float*)Bv.dev, (const float*)S0.dev,
                           (const float*)O.dev, (const float*)DO.dev, (float*)DA.dev,
                           (float*)DB.dev, (float*)D0.dev, B, T, N, gated ? 1 : 0, stream()));
    SN_TRY(copy_back(DA));
    SN_TRY(copy_back(DB));
    SN_TRY(copy_back(D0));
    return finish(DA.host || DB.host || D0.host || A.dev != a || Bv.dev != b || S0.dev != s0 ||
                  O.dev != out || DO.dev != dout);
}

int do_step(const float* a, const float* b, float* s, int B, int N, int gated) {
    if (!a || !b || !s || B <= 0 || N <= 0)
        return fail(SN_E_INVAL, "recur_step: null pointer or non-positive dimension");
    SN_TRY(ensure_init());
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    const size_t n = (size_t)B * N * sizeof(float);
    Arr A, Bv, Sx;
    SN_TRY(stage_in(a, n, 0, &A));
    SN_TRY(stage_in(b, n, 1, &Bv));
    SN_TRY(stage_inout(s, n, 2, &Sx));
    SN_TRY(launch_step((const float*)A.dev, (const float*)Bv.dev, (float*)Sx.dev, B, N,
                       gated ? 1 : 0, stream()));
    SN_TRY(copy_back(Sx));
    return finish(Sx.host || A.dev != a || Bv.dev != b);
}

int do_quant_i8(const float* x, int8_t* q, float* scale, int B, int N, int block) {
    if (!x || !q || !scale || B <= 0 || N <= 0)
        return fail(SN_E_INVAL, "quant_i8: null pointer or non-positive dimension");
    SN_TRY(ensure_init());
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    if (block <= 0) block = N;
    const int nb = (N + block - 1) / block;
    Arr X, Q, SC;
    SN_TRY(stage_in(x, (size_t)B * N * 4, 0, &X));
    SN_TRY(stage_out(q, (size_t)B * N, 1, &Q));
    SN_TRY(stage_out(scale, (size_t)B * nb * 4, 2, &SC));
    if (B > 65535) return fail(SN_E_INVAL, "quant_i8: B > 65535 rows");
    quant_i8_kernel<<<dim3(nb, B), 256, 0, stream()>>>((const float*)X.dev, (int8_t*)Q.dev,
                                                      (float*)SC.dev, N, block, nb);
    SN_TRY(cuda_check(cudaGetLastError(), "quant_i8 launch"));
    SN_TRY(copy_back(Q));
    SN_TRY(copy_back(SC));
    return finish(Q.host || SC.host || X.dev != x);
}

int do_dequant_i8(const int8_t* q, const float* scale, float* x, int B, int N, int block) {
    if (!x || !q || !scale || B <= 0 || N <= 0)
        return fail(SN_E_INVAL, "dequant_i8: null pointer or non-positive dimension");
    SN_TRY(ensure_init());
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    if (block <= 0) block = N;
    const int nb = (N + block - 1) / block;
    Arr Q, SC, X;
    SN_TRY(stage_in(q, (size_t)B * N, 0, &Q));
    SN_TRY(stage_in(scale, (size_t)B * nb * 4, 1, &SC));
    SN_TRY(stage_out(x, (size_t)B * N * 4, 2, &X));
    const long long total = (long long)B * N;
    const int blocks = grid_blocks(total);
    dequant_i8_kernel<<<blocks, 256, 0, stream()>>>((const int8_t*)Q.dev, (const float*)SC.dev,
                                                    (float*)X.dev, total, N, block, nb);
    SN_TRY(cuda_check(cudaGetLastError(), "dequant_i8 launch"));
    SN_TRY(copy_back(X));
    return finish(X.host || Q.dev != q || SC.dev != scale);
}

}  // namespace

extern "C" {

sn_status sn_abi_recur_scan(const float* a, const float* b, const float* s0, float* out,
                            float* send, int32_t B, int32_t T, int32_t N, int32_t gated) {
    return do_scan(a, b, s0, out, send, B, T, N, gated);
}

sn_status sn_abi_recur_bwd(const float* a, const float* b, const float* s0, const float* out,
                           const float* dout, float* da, float* db, float* ds0, int32_t B,
                           int32_t T, int32_t N, int32_t gated) {
    return do_bwd(a, b, s0, out, dout, da, db, ds0, B, T, N, gated);
}

sn_status sn_abi_recur_step(const float* a, const float* b, float* s, int32_t B, int32_t N,
                            int32_t gated) {
    return do_step(a, b, s, B, N, gated);
}

sn_status sn_abi_quant_i8(const float* x, int8_t* q, float* scale, int32_t B, int32_t N,
                          int32_t block) {
    return do_quant_i8(x, q, scale, B, N, block);
}

sn_status sn_abi_dequant_i8(const int8_t* q, const float* scale, float* x, int32_t B, int32_t N,
                            int32_t block) {
    return do_dequant_i8(q, scale, x, B, N, block);
}

// Internal symbol set (recur.h): same work, void returns like the reference;
// failures are reported through sn_abi_last_error.
void sn_recur_scan(const float* a, const float* b, const float* s0, float* out, float* send, int B,
                   int T, int N, int gated) {
    do_scan(a, b, s0, out, send, B, T, N, gated);
}

void sn_recur_step(const float* a, const float* b, float* s, int B, int N, int gated) {
    do_step(a, b, s, B, N, gated);
}

void sn_recur_bwd(const float* a, const float* b, const float* s0, const float* out,
                  const float* dout, float* da, float* db, float* ds0, int B, int T, int N,
                  int gated) {
    do_bwd(a, b, s0, out, dout, da, db, ds0, B, T, N, gated);
}

void sn_quant_i8(const float* x, signed char* q, float* scale, int B, int N, int block) {
    do_quant_i8(x, (int8_t*)q, scale, B, N, block);
}

void sn_dequant_i8(const signed char* q, const float* scale, float* x, int B, int N, int block) {
    do_dequant_i8((const int8_t*)q, scale, x, B, N, block);
}

}  // extern "C"
