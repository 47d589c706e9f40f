// tcgen05 / TMEM contraction for the batched token loop (see tc_gemm.cuh).
//
// Two launches per contraction:
//   split_act_kernel  A' (fp32 activations, row-LN prologue applied) -> bf16
//                     planes Ah, Al (M,K) with A' = Ah + Al to ~16 bits; once
//                     per GEMM instead of once per N-tile
//   tc_gemm_kernel    one CTA per 128 x BN tile of C, whole K loop through an
//                     S-deep ring of 64-wide K slabs (one 128-byte swizzle row):
//     warp 0  one thread issues the TMA 2-D tile loads of Ah, Al, Wh, Wl
//             (SWIZZLE_128B, no multicast), one complete_tx barrier per stage
//     warp 1  TMEM allocation; one thread issues tcgen05.mma.cta_group::1
//             .kind::f16 (M=128, N=BN, K=16): Ah*Wh + Ah*Wl + Al*Wh per K step
//             (two products for INT8 weights, exact in bf16), tcgen05.commit
//             frees the stage / signals the accumulator
//     warps 2.. epilogue: tcgen05.ld 32x32b (warp w reads TMEM lanes of
//             quarter w%4), each thread finishing its own output row (wide
//             tiles: four warp groups share the 32-column blocks) in a staged
//             tile (residual operands loaded into it under the main loop),
//             which all epilogue threads then store with coalesced 16-byte
//             stores; unaligned shapes stage 32x32 blocks so each global
//             access is one 128-byte row segment; same arithmetic as
//             gemm_epilogue
// Every mbarrier wait is bounded; a role that gives up records the error,
// drains its own in-flight TMA/MMA work, and the CTA frees its TMEM.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <map>
#include <vector>

#include "ptx.cuh"
#include "runtime.cuh"
#include "tc_gemm.cuh"
#include "tcgen05.cuh"

namespace sn {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // bf16 per slab row = 128 bytes
// Epilogue warps: group 0 (warps 2-5, one per TMEM lane quarter) runs every
// epilogue; in the thread-per-row epilogues of wide tiles (BN > 32) four
// groups share the 32-column blocks, so the latency chains of several warps
// (IEEE divides, tanh, exp) interleave on each scheduler. 32-column tiles
// launch group 0 alone.
template <int BN>
struct TcEpi {
    static constexpr int GROUPS = BN > 32 ? 4 : 1;
    static constexpr int THREADS = 64 + 128 * GROUPS;
};
// INT8 codes converted in the main loop (CV) add converter warps after the
// epilogue warps: one warp group, two for tiles of 128 columns and more
template <int BN, bool CV>
struct TcThreads {
    static constexpr int CONV = CV ? (BN >= 128 ? 256 : 128) : 0;
    static constexpr int N = TcEpi<BN>::THREADS + CONV;
};

// Residual / accumulate tiles of 64 or 128 columns stage their whole operand
// tile ([BM][BN + 4] fp32): under the main loop, next to the ring, where that
// leaves the ring three stages at least; else in the drained ring after it.
template <int BN, bool LOADS>
struct TcStage {
    static constexpr bool ON = LOADS && BN > 32 && BN <= 128;
};

template <int BN, bool I8, bool LOADS = false>
struct TcCfg {
    static constexpr int A_BYTES = BM * 128;
    static constexpr int W_BYTES = BN * 128;
    // a stage: the A hi / lo slabs and the weight slab, bf16 hi and lo (INT8
    // weights: the one bf16 slab the converter warps write)
    static constexpr int STAGE = 2 * A_BYTES + (I8 ? 1 : 2) * W_BYTES;
    // epilogue operands loaded under the main loop: [4 warps][32][33] floats
    // (32x32 blocks), or the staged operand tile
    static constexpr int PRE_BLOCKS = 4 * 32 * 33 * 4;
    static constexpr int TILE = BM * (BN + 4) * 4;
    static constexpr int FIXED = 1024 + 256 + BN * 4;  // alignment slack, barriers, scales
    static constexpr bool EARLY =
        TcStage<BN, LOADS>::ON &&
        (227 * 1024 - (TILE > PRE_BLOCKS ? TILE : PRE_BLOCKS) - FIXED) / STAGE >= 3;
    static constexpr int PRE = EARLY && TILE > PRE_BLOCKS ? TILE : PRE_BLOCKS;
    // as many stages as fit the 227 KB of shared memory next to the operand
    // area, 1 KB of alignment slack, 256 B of barriers and BN column scales
    static constexpr int S_FIT = (227 * 1024 - PRE - FIXED) / STAGE;
    static constexpr int S = S_FIT > 6 ? 6 : S_FIT;
    static_assert(S >= 2, "two ring stages at least");
    // late staging fetches the S, F and X rows by bulk copies into the
    // drained ring and the operand area that follows it where the three fit
    // (LATE3), else p*S + F + X into the ring with 16-byte loads
    static constexpr bool LATE3 = 3 * TILE <= S * STAGE + PRE;
    static_assert(EARLY || !TcStage<BN, LOADS>::ON || TILE <= S * STAGE, "late operand tile fits");
    // after the 256 bytes of barriers: the tile's per-column weight scales
    static constexpr int SMEM = S * STAGE + PRE + 1024 + 256 + BN * 4;
};

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);  // .x = a (low half), .y = b
    return *reinterpret_cast<const uint32_t*>(&h);
}

// A' -> (Ah, Al), 8 elements (one 16-byte chunk of each plane) per thread-step.
__global__ void split_act_kernel(GemmArgs a, __nv_bfloat16* __restrict__ hi,
                                 __nv_bfloat16* __restrict__ lo) {
    const int cpr = a.K / 8;
    const long long total = (long long)a.M * cpr;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int m = (int)(i / cpr), k = (int)(i % cpr) * 8;
        const float* src = a.A + (long long)m * a.lda + k;
        const float4 x0 = *reinterpret_cast<const float4*>(src);
        const float4 x1 = *reinterpret_cast<const float4*>(src + 4);
        float v[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        if (a.mu) {
            const float mu = a.mu[m], rs = a.rs[m];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = __fmul_rn(__fmul_rn(v[j] - mu, rs), a.g[k + j]) + a.c[k + j];
        }
        float l[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) l[j] = v[j] - __bfloat162float(__float2bfloat16_rn(v[j]));
        const long long o = (long long)m * a.K + k;
        *reinterpret_cast<uint4*>(hi + o) = make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]),
                                                       pack_bf16(v[4], v[5]), pack_bf16(v[6], v[7]));
        *reinterpret_cast<uint4*>(lo + o) = make_uint4(pack_bf16(l[0], l[1]), pack_bf16(l[2], l[3]),
                                                       pack_bf16(l[4], l[5]), pack_bf16(l[6], l[7]));
    }
}

// 32 rows [mr0, mr0 + 32) of output column n from a staged 32x32 block
// (row r at stg[r * 33 + lane]) with the element-wise epilogue EPI (the
// kinds that read nothing but the accumulator), same arithmetic as
// gemm_epilogue; optionally also the bf16 planes of the result.
template <int EPI>
__device__ __forceinline__ void tc_rows(const GemmArgs& a, int mr0, int n, bool nok, float ws,
                                        const float* stg, int lane) {
    if (!nok) return;
#pragma unroll 4  // compact: this runs once per launch, from a cold instruction cache
    for (int r = 0; r < 32; ++r) {
        const int mm = mr0 + r;
        if (mm >= a.M) continue;
        float acc = stg[r * 33 + lane];
        if (a.wscale) acc = acc * ws;
        float y;
        if (EPI == kEpiWedge) y = acc * (1.0f + 0.5f * a.p / (1.0f + fabsf(acc)));
        else if (EPI == kEpiRelu2) {
            const float t = acc > 0.0f ? acc : 0.0f;
            y = t * t;
        } else if (EPI == kEpiTanh) y = tanhf(acc);
        else if (EPI == kEpiSigmoid) y = 1.0f / (1.0f + expf(-acc));
        else y = acc;
        const long long o = (long long)mm * a.ldc + n;
        a.C[o] = y;
        if (a.Ch) store_split((__nv_bfloat16*)a.Ch, (__nv_bfloat16*)a.Cl, o, y);
    }
}

// gemm_epilogue with the kind fixed at compile time (same arithmetic).
template <int EPI>
__device__ __forceinline__ float epi_elem(const GemmArgs& a, int m, int n, float acc) {
    if (a.wscale) acc = acc * a.wscale[n];
    if (EPI == kEpiWedge) return acc * (1.0f + 0.5f * a.p / (1.0f + fabsf(acc)));
    if (EPI == kEpiResid)
        return acc + (a.p * a.S[m * a.lds + n] + a.F[m * a.ldf + n] + a.X[m * a.ldx + n]);
    if (EPI == kEpiAdd) return a.C[m * a.ldc + n] + acc;
    if (EPI == kEpiRelu2) {
        const float t = acc > 0.0f ? acc : 0.0f;
        return t * t;
    }
    if (EPI == kEpiTanh) return tanhf(acc);
    if (EPI == kEpiSigmoid) return 1.0f / (1.0f + expf(-acc));
    return acc;
}

// The residual (p*S + F + X) or accumulate (C) operand of output (mm, n),
// 0 outside the matrix.
__device__ __forceinline__ float tc_operand(const GemmArgs& a, long long mm, int n) {
    if (mm >= a.M || n >= a.N) return 0.0f;
    return a.epi == kEpiResid ? a.p * a.S[mm * a.lds + n] + a.F[mm * a.ldf + n] + a.X[mm * a.ldx + n]
                              : a.C[mm * a.ldc + n];
}

// Rows [mr0, mr0 + 32) of column n's operand into pre_w[r * 33 + lane]. Loads
// through GemmArgs' pointers may alias the generic shared-memory pointer, so
// the compiler keeps each load after the previous store; sixteen rows are
// loaded into registers before any is stored, so their round trips overlap.
__device__ __forceinline__ void tc_block_operands(const GemmArgs& a, long long mr0, int n,
                                                  float* pre_w, int lane) {
#pragma unroll 1
    for (int r0 = 0; r0 < 32; r0 += 16) {
        float t[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) t[i] = tc_operand(a, mr0 + r0 + i, n);
#pragma unroll
        for (int i = 0; i < 16; ++i) pre_w[(r0 + i) * 33 + lane] = t[i];
    }
}

// L2 prefetch hints for row mm's operand segment [n0, min(n0 + BN, N)): one
// bulk prefetch per segment when rows are 16-byte aligned, else one hint per
// 128-byte line, every address inside the matrix. Issued by the idle epilogue
// threads under the main loop, so the epilogue's reads hit L2.
template <int BN>
__device__ __forceinline__ void tc_prefetch_row(const GemmArgs& a, long long mm, int n0, bool bulk) {
    if (mm >= a.M || n0 >= a.N) return;
    const int nl = (a.N - n0 < BN ? a.N - n0 : BN) - 1;  // last column offset
    const float* rows[3];
    int nr = 0;
    if (a.epi == kEpiResid) {
        rows[nr++] = a.S + mm * a.lds + n0;
        rows[nr++] = a.F + mm * a.ldf + n0;
        rows[nr++] = a.X + mm * a.ldx + n0;
    } else {
        rows[nr++] = a.C + mm * a.ldc + n0;
    }
    for (int i = 0; i < nr; ++i) {
        if (bulk) {
            bulk_prefetch_l2(rows[i], (uint32_t)(nl + 1) * 4u);
        } else {
            for (int c = 0; c < nl; c += 32) prefetch_l2(rows[i] + c);
            prefetch_l2(rows[i] + nl);
        }
    }
}

// True when every operand row segment of the epilogue can move as one bulk
// copy: 16-byte aligned bases, leading dimensions and widths (N % 4 == 0).
__device__ __forceinline__ bool tc_rows_aligned(const GemmArgs& a) {
    auto al = [](const float* p, long long ld) {
        return (reinterpret_cast<uintptr_t>(p) & 15) == 0 && (ld & 3) == 0;
    };
    if ((a.N & 3) != 0) return false;
    return a.epi == kEpiResid ? al(a.S, a.lds) && al(a.F, a.ldf) && al(a.X, a.ldx) : al(a.C, a.ldc);
}

// The operand tile of a residual (p*S + F + X) or accumulate (C) epilogue:
// rows [0, nr) x columns [0, nc) of the tile at (m0, n0) into `ra` as
// [BM][BN + 4] fp32, run under the main loop. 16-byte loads spread over all
// nt epilogue threads (consecutive threads on consecutive 16 bytes of a row),
// four per thread in flight before their shared-memory stores. Same
// arithmetic as tc_operand; nc % 4 == 0 and 16-byte aligned rows.
template <int BN>
__device__ __forceinline__ void tc_stage_operands(const GemmArgs& a, int m0, int n0, int nr,
                                                  int nc, float* ra, int et, int nt) {
    constexpr int RS = BN + 4, U = 4;
    const int c4 = nc >> 2, total = nr * c4;
    const bool resid = a.epi == kEpiResid;
#pragma unroll 1
    for (int i0 = et; i0 < total; i0 += U * nt) {
        float4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = i0 + u * nt;
            v[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (i < total) {
                const int r = nc == BN ? i / (BN / 4) : i / c4;
                const long long mm = m0 + r;
                const int n = n0 + ((i - r * c4) << 2);
                if (resid) {
                    const float4 sv = *reinterpret_cast<const float4*>(a.S + mm * a.lds + n);
                    const float4 fv = *reinterpret_cast<const float4*>(a.F + mm * a.ldf + n);
                    const float4 xv = *reinterpret_cast<const float4*>(a.X + mm * a.ldx + n);
                    v[u] = make_float4(a.p * sv.x + fv.x + xv.x, a.p * sv.y + fv.y + xv.y,
                                       a.p * sv.z + fv.z + xv.z, a.p * sv.w + fv.w + xv.w);
                } else {
                    v[u] = *reinterpret_cast<const float4*>(a.C + mm * a.ldc + n);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = i0 + u * nt;
            if (i < total) {
                const int r = nc == BN ? i / (BN / 4) : i / c4;
                *reinterpret_cast<float4*>(ra + r * RS + ((i - r * c4) << 2)) = v[u];
            }
        }
    }
}

// Rows [0, nr) x columns [0, nc) of a finished tile, staged in shared memory
// as [BM][BN + 4] fp32 at `src`, to C[m0 + r][n0 + c]: 16-byte stores over
// all nt epilogue threads, consecutive threads on consecutive 16 bytes of a
// row (nc % 4 == 0, C rows 16-byte aligned).
template <int BN>
__device__ __forceinline__ void tc_store_tile(float* C, long long ldc, int m0, int n0, int nr,
                                              int nc, const float* src, int et, int nt) {
    constexpr int RS = BN + 4;
    const int c4 = nc >> 2, total = nr * c4;
#pragma unroll 4
    for (int i = et; i < total; i += nt) {
        const int r = nc == BN ? i / (BN / 4) : i / c4;
        const int c = (i - r * c4) << 2;
        *reinterpret_cast<float4*>(C + (long long)(m0 + r) * ldc + n0 + c) =
            *reinterpret_cast<const float4*>(src + r * RS + c);
    }
}

// The same for one bf16 plane of the result, staged as [BM][BN + 8] at `src`:
// 16-byte stores of 8 elements (nc % 8 == 0, plane rows 16-byte aligned).
template <int BN>
__device__ __forceinline__ void tc_store_plane(__nv_bfloat16* P, long long ldc, int m0, int n0,
                                               int nr, int nc, const __nv_bfloat16* src, int et,
                                               int nt) {
    constexpr int RSH = BN + 8;
    const int c8 = nc >> 3, total = nr * c8;
#pragma unroll 4
    for (int i = et; i < total; i += nt) {
        const int r = nc == BN ? i / (BN / 8) : i / c8;
        const int c = (i - r * c8) << 3;
        *reinterpret_cast<uint4*>(P + (long long)(m0 + r) * ldc + n0 + c) =
            *reinterpret_cast<const uint4*>(src + r * RSH + c);
    }
}

// Thread-per-row epilogue of the accumulator-only kinds, one 32-column
// block: v = 32 accumulator columns of this thread's row (as tcgen05.ld
// hands them), ws = their weight scales (shared memory), the result into the
// staged fp32 row `out` (16-byte aligned) and, with planes, the bf16 rows
// hi / lo. Same arithmetic as tc_rows.
template <int EPI>
__device__ __forceinline__ void tc_row_block(const GemmArgs& a, const float* v, const float* ws,
                                             float* out, __nv_bfloat16* hi, __nv_bfloat16* lo) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
        float y[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float acc = v[j + i];
            if (a.wscale) acc = acc * ws[j + i];
            if (EPI == kEpiWedge) {
                y[i] = acc * (1.0f + 0.5f * a.p / (1.0f + fabsf(acc)));
            } else if (EPI == kEpiRelu2) {
                const float t = acc > 0.0f ? acc : 0.0f;
                y[i] = t * t;
            } else if (EPI == kEpiTanh) {
                y[i] = tanhf(acc);
            } else if (EPI == kEpiSigmoid) {
                y[i] = 1.0f / (1.0f + expf(-acc));
            } else {
                y[i] = acc;
            }
        }
        *reinterpret_cast<float4*>(out + j) = make_float4(y[0], y[1], y[2], y[3]);
        if (hi) {
            __nv_bfloat16 h[4], l[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {  // store_split's rounding
                h[i] = __float2bfloat16_rn(y[i]);
                l[i] = __float2bfloat16_rn(y[i] - __bfloat162float(h[i]));
            }
            *reinterpret_cast<uint2*>(hi + j) = *reinterpret_cast<const uint2*>(h);
            *reinterpret_cast<uint2*>(lo + j) = *reinterpret_cast<const uint2*>(l);
        }
    }
}

// Epilogue code runs once per launch, mostly from a cold instruction cache:
// its loops keep small bodies (a few elements per iteration, enough loads in
// flight) instead of being unrolled whole.
//
// Split K, owner side, in groups of 4 consecutive outputs of a row (16-byte
// loads and stores; the host splits K only when every operand allows that).
// The owner's ng = rows * BN / 4 groups are spread over the nt epilogue
// threads (et = 0..nt-1), row-major. tc_own_operands stages each group's
// residual / accumulate operands in shared memory before the accumulator is
// ready; tc_reduce sums the ks partial rows of the cluster in rank order
// (partials at [row][BN+4] in each CTA), then applies the epilogue.
template <int BN>
__device__ __forceinline__ void tc_own_operands(const GemmArgs& a, int mr0, int n0, int ng, int et,
                                                int nt, float4* pre) {
#pragma unroll 2
    for (int g = et; g < ng; g += nt) {
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        const long long mm = mr0 + (4 * g) / BN;
        const int n = n0 + (4 * g) % BN;
        if (mm < a.M && n < a.N) {
            if (a.epi == kEpiResid) {
                const float4 sv = *reinterpret_cast<const float4*>(a.S + mm * a.lds + n);
                const float4 fv = *reinterpret_cast<const float4*>(a.F + mm * a.ldf + n);
                const float4 xv = *reinterpret_cast<const float4*>(a.X + mm * a.ldx + n);
                v = make_float4(a.p * sv.x + fv.x + xv.x, a.p * sv.y + fv.y + xv.y,
                                a.p * sv.z + fv.z + xv.z, a.p * sv.w + fv.w + xv.w);
            } else {
                v = *reinterpret_cast<const float4*>(a.C + mm * a.ldc + n);
            }
        }
        pre[g] = v;
    }
}

template <int EPI, int BN>
__device__ __forceinline__ void tc_reduce(const GemmArgs& a, const float* part, int ks, int rows,
                                          int r0, int m0, int n0, int et, int nt,
                                          const float4* pre) {
    const int ng = rows * BN / 4;
#pragma unroll 2
    for (int g = et; g < ng; g += nt) {
        const int r = (4 * g) / BN, c = (4 * g) % BN;
        const float* src = part + (r0 + r) * (BN + 4) + c;
        float4 x = ld_dsmem_f32x4(src, 0);
        for (int p = 1; p < ks; ++p) {
            const float4 t = ld_dsmem_f32x4(src, (uint32_t)p);
            x.x += t.x;
            x.y += t.y;
            x.z += t.z;
            x.w += t.w;
        }
        const long long mm = m0 + r0 + r;
        const int n = n0 + c;
        if (mm >= a.M || n >= a.N) continue;  // N % 4 == 0: a group is all in or all out
        float y[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if (EPI == kEpiResid || EPI == kEpiAdd) {
                const float4 pv = pre[g];
                const float pi = i == 0 ? pv.x : (i == 1 ? pv.y : (i == 2 ? pv.z : pv.w));
                float xi = y[i];
                if (a.wscale) xi = xi * a.wscale[n + i];
                y[i] = EPI == kEpiResid ? xi + pi : pi + xi;
            } else {
                y[i] = epi_elem<EPI>(a, (int)mm, n + i, y[i]);
            }
        }
        const long long o = mm * a.ldc + n;
        *reinterpret_cast<float4*>(a.C + o) = make_float4(y[0], y[1], y[2], y[3]);
        if (a.Ch) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
                store_split((__nv_bfloat16*)a.Ch, (__nv_bfloat16*)a.Cl, o + i, y[i]);
        }
    }
}

// LOADS: the epilogue reads more than the accumulator (residual / accumulate
// kinds); those operands are then all loaded before any result is stored.
template <int BN, bool I8, bool LOADS, bool CV>
__global__ void __launch_bounds__(TcThreads<BN, CV>::N, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tah, const __grid_constant__ CUtensorMap tal,
                   const __grid_constant__ CUtensorMap twh, const __grid_constant__ CUtensorMap twl,
                   GemmArgs a, int* err) {
    using C = TcCfg<BN, I8, LOADS>;
    constexpr int S = C::S;
    constexpr int kEpiGroups = TcEpi<BN>::GROUPS;
    // TMEM is allocated in powers of two columns (a 192-wide tile takes 256)
    constexpr uint32_t kTmemCols = BN <= 32 ? 32u : (BN <= 64 ? 64u : (BN <= 128 ? 128u : 256u));
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* sb = smem_raw + (((raw + 1023u) & ~1023u) - raw);  // 1024-B aligned ring
    float* pre_all = reinterpret_cast<float*>(sb + S * C::STAGE);
    uint64_t* full = reinterpret_cast<uint64_t*>(sb + S * C::STAGE + C::PRE);
    uint64_t* empty = full + S;
    uint64_t* conv = empty + S;  // INT8: a stage's weight slab converted to bf16
    uint64_t* acc_full = conv + S;
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(acc_full + 1);
    volatile int* give_up = reinterpret_cast<volatile int*>(acc_full + 2);
    uint64_t* op_full = acc_full + 3;  // [4]: a quarter's operand rows landed (late staging)
    float* wsc = reinterpret_cast<float*>(sb + S * C::STAGE + C::PRE + 256);  // [BN]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // split K: a cluster of ks CTAs along x shares one output tile, CTA kz of
    // it takes K slabs [k0, k0 + nk) (ks = 1 without a cluster launch)
    const int ks = (int)cluster_size(), kz = (int)cluster_rank();
    const int m0 = blockIdx.y * BM, n0 = (blockIdx.x / ks) * BN;
    const int nkt = (a.K + BK - 1) / BK;
    const int k0 = kz * nkt / ks, nk = (kz + 1) * nkt / ks - k0;
    // INT8 weights: codes converted to bf16 in the main loop by the converter
    // warps (CV), or bf16 code planes loaded by TMA like other weights
    constexpr bool cv = I8 && CV;
    pdl_trigger();  // the next kernel may start its own prologue
    auto stage_ptr = [&](int s, int part) -> uint8_t* {  // 0 Ah, 1 Al, 2 Wh, 3 Wl
        return sb + s * C::STAGE +
               (part < 2 ? part * C::A_BYTES : 2 * C::A_BYTES + (part - 2) * C::W_BYTES);
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            mbar_init(&conv[s], TcThreads<BN, CV>::CONV > 0 ? TcThreads<BN, CV>::CONV : 1);
        }
        mbar_init(acc_full, 1);
        for (int q = 0; q < 4; ++q) mbar_init(&op_full[q], 1);
        *give_up = 0;
        fence_mbar_init();
    }
    if (warp == 1) {  // TMEM accumulator: BN fp32 columns x 128 lanes
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32((const void*)tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {  // --------------------------------------------- TMA producer
        if (lane == 0) {
            // descriptors into the cache before the first copies (the A maps'
            // first use comes after the wait for the previous kernel)
            prefetch_tmap(&tah);
            prefetch_tmap(&tal);
            // INT8 codes converted in the main loop (cv) are not loaded by TMA:
            // the converter warps write the weight slab
            auto load_w = [&](int s, int kt) {
                if (cv) return;
                tma_load_2d(stage_ptr(s, 2), &twh, (k0 + kt) * BK, n0, &full[s]);
                if (!I8) tma_load_2d(stage_ptr(s, 3), &twl, (k0 + kt) * BK, n0, &full[s]);
            };
            if (!cv) {
                prefetch_tmap(&twh);
                if (!I8) prefetch_tmap(&twl);
            }
            const uint32_t bytes = 2 * C::A_BYTES + (cv ? 0 : (I8 ? 1 : 2) * C::W_BYTES);
            // the weight tiles of the first S stages do not depend on the
            // previous kernel: in flight before waiting for it (programmatic
            // launch; pdl_wait is a no-op otherwise)
            const int pre = nk < S ? nk : S;
            for (int kt = 0; kt < pre; ++kt) {
                mbar_expect_tx(&full[kt], bytes);
                load_w(kt, kt);
            }
            pdl_wait();
            int issued = 0;
            for (int kt = 0; kt < nk; ++kt) {
                const int s = kt % S;
                if (kt >= pre) {  // stages of the first round are never abandoned half-loaded
                    if (*give_up) break;
                    if (!mbar_wait(&empty[s], ((kt / S) - 1) & 1, err)) {
                        *give_up = 1;
                        break;
                    }
                    mbar_expect_tx(&full[s], bytes);
                    load_w(s, kt);
                }
                tma_load_2d(stage_ptr(s, 0), &tah, (k0 + kt) * BK, m0, &full[s]);
                tma_load_2d(stage_ptr(s, 1), &tal, (k0 + kt) * BK, m0, &full[s]);
                issued = kt + 1;
            }
            // never leave with a tile load in flight: wait for the last use of each stage
            for (int kt = issued - S < 0 ? 0 : issued - S; kt < issued; ++kt)
                mbar_wait(&full[kt % S], (kt / S) & 1, err);
        }
    } else if (warp == 1) {  // ---------------------------------------- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = (1u << 4)                      // D: f32
                                   | (1u << 7) | (1u << 10)       // A, B: bf16
                                   | ((uint32_t)(BN >> 3) << 17)  // N
                                   | ((uint32_t)(BM >> 4) << 24); // M
            for (int kt = 0; kt < nk; ++kt) {
                const int s = kt % S;
                if (!mbar_wait(&full[s], (kt / S) & 1, err) ||
                    (cv && !mbar_wait(&conv[s], (kt / S) & 1, err))) {
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
            tc_commit(acc_full);  // accumulator complete (or: nothing left in flight)
        }
    } else if (cv && warp >= 2 + 4 * kEpiGroups) {  // ------------- INT8 converter
        if (!cv) {
            // bf16 code planes: nothing to convert
        } else {
        // Each K slab's BN x 64 weight codes, read from global memory (L2) a
        // few slabs ahead into registers, become the stage's bf16 slab the
        // MMAs read, in the layout a SWIZZLE_128B load would write: row n in
        // 8-row atoms of 1024 B, its 16-byte chunk c at position c ^ (n % 8).
        // A code q is exact in bf16: the fp32 bit pattern 0x4B0000(q ^ 0x80)
        // is 2^23 + 128 + q, so one subtraction gives q and its upper 16 bits
        // are bf16(q). A thread takes 32 codes (row i / 2, half i % 2) per
        // pass; codes past N or K read as zero. The weights do not depend on
        // the previous kernel: no wait for it.
        constexpr int NC = TcThreads<BN, CV>::CONV > 0 ? TcThreads<BN, CV>::CONV : 128;
        constexpr int PER = (2 * BN + NC - 1) / NC;  // row halves per thread per slab
        constexpr int DEPTH = 3;                      // slabs in flight per thread
        const int ct = threadIdx.x - (64 + 128 * kEpiGroups);
        const int8_t* q8 = reinterpret_cast<const int8_t*>(a.W);
        uint4 buf[DEPTH][PER][2];
        auto load = [&](int kt, uint4 (&b)[PER][2]) {
#pragma unroll
            for (int p = 0; p < PER; ++p) {
                const int i = ct + p * NC, n = i >> 1, h = i & 1;
                const int row = n0 + n, k = (k0 + kt) * BK + h * 32;
                const int8_t* src = q8 + (long long)row * a.ldw + k;
                const bool rok = i < 2 * BN && row < a.N && kt < nk;
                b[p][0] = rok && k < a.K ? __ldg(reinterpret_cast<const uint4*>(src))
                                         : make_uint4(0, 0, 0, 0);
                b[p][1] = rok && k + 16 < a.K ? __ldg(reinterpret_cast<const uint4*>(src + 16))
                                              : make_uint4(0, 0, 0, 0);
            }
        };
#pragma unroll
        for (int d = 0; d < DEPTH; ++d) load(d, buf[d]);
        bool stop = false;
        for (int kt0 = 0; kt0 < nk && !stop; kt0 += DEPTH) {
#pragma unroll
            for (int d = 0; d < DEPTH; ++d) {
                const int kt = kt0 + d, s = kt % S;
                if (kt >= nk || stop) break;
                if (*give_up ||
                    (kt >= S && !mbar_wait(&empty[s], ((kt / S) - 1) & 1, err))) {
                    *give_up = 1;
                    stop = true;
                    break;
                }
                uint8_t* dst = stage_ptr(s, 2);
#pragma unroll
                for (int p = 0; p < PER; ++p) {
                    const int i = ct + p * NC, n = i >> 1, h = i & 1;
                    if (i >= 2 * BN) continue;
                    const uint32_t* qw = reinterpret_cast<const uint32_t*>(buf[d][p]);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {  // chunk 4h + j: codes 8j .. 8j + 7 of the half
                        uint32_t o[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const uint32_t u = qw[2 * j + (e >> 1)] ^ 0x80808080u;  // q + 128
                            const int b0 = (e & 1) * 2;  // bytes b0, b0 + 1 of the word
                            const float f0 =
                                __int_as_float((int)__byte_perm(u, 0x4B000000u, 0x7540u + b0)) -
                                8388736.0f;
                            const float f1 =
                                __int_as_float((int)__byte_perm(u, 0x4B000000u, 0x7541u + b0)) -
                                8388736.0f;
                            o[e] = __byte_perm(__float_as_uint(f0), __float_as_uint(f1), 0x7632u);
                        }
                        *reinterpret_cast<uint4*>(dst + (n >> 3) * 1024 + (n & 7) * 128 +
                                                  ((((4 * h + j) ^ (n & 7))) << 4)) =
                            make_uint4(o[0], o[1], o[2], o[3]);
                    }
                }
                fence_proxy_async_smem();  // the slab, for the tensor cores
                mbar_arrive(&conv[s]);
                load(kt + DEPTH, buf[d]);
            }
        }
        }
    } else {  // ------------------------------------------------ epilogue (warps 2..)
        const int q = warp & 3;         // TMEM lane quarter this warp may read
        const int g = (warp - 2) >> 2;  // column group
        const int et = threadIdx.x - 64;
        pdl_wait();  // the epilogue reads (and overwrites) the previous kernels' outputs
        if (ks > 1) {
            // split K: CTA kz owns rows [kz*rows, (kz+1)*rows) of the tile; its
            // residual / accumulate operands are loaded now, under the main loop
            // (every epilogue thread)
            const int rows = BM / ks;
            if (LOADS)
                tc_own_operands<BN>(a, m0 + kz * rows, n0, rows * BN / 4, et, 128 * kEpiGroups,
                                    reinterpret_cast<float4*>(pre_all));
            const bool ok = mbar_wait(acc_full, 0, err);
            tc_fence_after();
            if (ok && !*give_up) {
                // this CTA's partial rows into its own shared memory (the
                // drained ring), [128][BN+4]; the owners read them below. The
                // groups share the 32-column blocks.
                float4* part = reinterpret_cast<float4*>(reinterpret_cast<float*>(sb) +
                                                         (q * 32 + lane) * (BN + 4));
#pragma unroll 1
                for (int j0 = g * 32; j0 < BN; j0 += 32 * kEpiGroups) {
                    float v[32];
                    tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)j0, v);
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        part[(j0 + j) / 4] = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                }
            }
        } else {
            // this warp's operands of a 32x32 block, [row][33] in shared memory
            // (group 0)
            float* pre_w = pre_all + ((warp - 2) & 3) * (32 * 33);
            // Wide residual / accumulate tiles with 16-byte aligned rows stage
            // their operand tile (p*S + F + X, or C) in its own area `ra` under
            // the main loop, 16-byte loads spread over every epilogue thread;
            // each thread then finishes its own row in place (the 32
            // accumulator columns tcgen05.ld hands it, conflict-free float4
            // accesses) and all of them store the tile with coalesced 16-byte
            // stores. Wide accumulator-only tiles do the same with their rows
            // staged in the drained ring (and the bf16 planes after them).
            constexpr int RS = BN + 4;  // padded row stride: 16-byte bank groups differ per row
            constexpr bool kStage = TcStage<BN, LOADS>::ON;
            constexpr int kEt = 128 * kEpiGroups;  // epilogue threads
            const bool out_al = (reinterpret_cast<uintptr_t>(a.C) & 15) == 0 && (a.ldc & 3) == 0 &&
                                (a.N & 3) == 0;
            const bool staged = kStage && tc_rows_aligned(a) && a.Ch == nullptr && out_al;
            constexpr int RSH = BN + 8;
            constexpr bool kPlanesFit = BM * RS * 4 + 2 * BM * RSH * 2 <= S * C::STAGE;
            const bool planes_al = a.Ch != nullptr && kPlanesFit &&
                                   (reinterpret_cast<uintptr_t>(a.Ch) & 15) == 0 &&
                                   (reinterpret_cast<uintptr_t>(a.Cl) & 15) == 0 &&
                                   (a.ldc & 7) == 0 && (a.N & 7) == 0;
            const bool rows = !LOADS && BN > 32 && out_al && (a.Ch == nullptr || planes_al);
            const int nc = a.N - n0 < BN ? a.N - n0 : BN;  // this tile's columns
            const int nr = a.M - m0 < BM ? a.M - m0 : BM;  // and rows inside the matrix
            // [BM][RS]: the staged operand tile, then the results (late
            // staging: in the drained ring, loaded once the accumulator is ready)
            constexpr bool kEarly = C::EARLY;
            float* ra = kEarly ? pre_all : reinterpret_cast<float*>(sb);
            if (LOADS && BN == 32 && g == 0)  // the only block's operands, under the main loop
                tc_block_operands(a, m0 + q * 32, n0 + lane, pre_w, lane);
            if (kStage && (!staged || !kEarly) && g == 0)  // operands into L2 meanwhile
                tc_prefetch_row<BN>(a, m0 + et, n0, staged);
            if (staged && kEarly) tc_stage_operands<BN>(a, m0, n0, nr, nc, ra, et, kEt);
            if (a.wscale)  // the tile's column scales, read from shared memory below
                for (int c = et; c < BN; c += kEt) wsc[c] = n0 + c < a.N ? a.wscale[n0 + c] : 1.0f;
            named_bar_sync(1, kEt);  // every epilogue warp: ra and wsc complete
            bool ok = mbar_wait(acc_full, 0, err);
            tc_fence_after();
            const int row = q * 32 + lane;  // TMEM lane = tile row of this thread
            // a quarter's 32 rows are stored by its four warps (one per group,
            // named barrier 2 + q) as soon as they are finished
            const int eq = g * 32 + lane, nq = nr - q * 32 < 0 ? 0 : (nr - q * 32 < 32 ? nr - q * 32 : 32);
            // Rows of 128 columns and more leave by one bulk copy per row (the
            // copy engine moves them faster than the warps' stores); narrower
            // ones by the quarter's coalesced stores.
            constexpr bool kBulkRows = BN >= 128;
            auto store_rows = [&](const float* fq, const __nv_bfloat16* hq, const __nv_bfloat16* lq) {
                if (kBulkRows) fence_proxy_async_smem();  // the rows, for the copy engine
                named_bar_sync(2 + q, 128);  // this quarter's rows finished
                if (!ok || *give_up) return;
                if (kBulkRows) {
                    if (g == 0 && lane < nq) {
                        const long long o = (long long)(m0 + row) * a.ldc + n0;
                        bulk_s2g(a.C + o, fq + lane * RS, nc * 4);
                        if (hq) {
                            bulk_s2g(reinterpret_cast<__nv_bfloat16*>(a.Ch) + o, hq + lane * RSH, nc * 2);
                            bulk_s2g(reinterpret_cast<__nv_bfloat16*>(a.Cl) + o, lq + lane * RSH, nc * 2);
                        }
                        bulk_commit();
                        bulk_wait_read_all();  // the rows stay valid until read
                    }
                } else {
                    tc_store_tile<BN>(a.C, a.ldc, m0 + q * 32, n0, nq, nc, fq, eq, 128);
                    if (hq) {
                        tc_store_plane<BN>(reinterpret_cast<__nv_bfloat16*>(a.Ch), a.ldc, m0 + q * 32, n0,
                                           nq, nc, hq, eq, 128);
                        tc_store_plane<BN>(reinterpret_cast<__nv_bfloat16*>(a.Cl), a.ldc, m0 + q * 32, n0,
                                           nq, nc, lq, eq, 128);
                    }
                }
            };
            if (staged) {
                const bool resid = a.epi == kEpiResid;
                if (!kEarly && !C::LATE3) {
                    // every MMA has completed, so the ring is free: the operand
                    // tile p*S + F + X (or C) by every epilogue thread
                    if (ok && !*give_up) tc_stage_operands<BN>(a, m0, n0, nr, nc, ra, et, kEt);
                    named_bar_sync(1, kEt);
                } else if (!kEarly) {
                    // every MMA has completed, so the ring is free: the quarter's
                    // operand rows by bulk copies (group 0, a row per thread)
                    if (g == 0 && ok && !*give_up) {
                        if (lane == 0)
                            mbar_expect_tx(&op_full[q], (uint32_t)(nq * nc * 4 * (resid ? 3 : 1)));
                        __syncwarp();
                        if (lane < nq) {
                            float* orow = ra + row * RS;
                            const long long mm = m0 + row;
                            if (resid) {
                                bulk_g2s(orow, a.S + mm * a.lds + n0, nc * 4, &op_full[q]);
                                bulk_g2s(orow + BM * RS, a.F + mm * a.ldf + n0, nc * 4, &op_full[q]);
                                bulk_g2s(orow + 2 * BM * RS, a.X + mm * a.ldx + n0, nc * 4, &op_full[q]);
                            } else {
                                bulk_g2s(orow, a.C + mm * a.ldc + n0, nc * 4, &op_full[q]);
                            }
                        }
                    }
                    if (ok && !*give_up) ok = mbar_wait(&op_full[q], 0, err);
                }
                float* orow = ra + row * RS;
#pragma unroll 1
                for (int j0 = g * 32; ok && !*give_up && j0 < BN; j0 += 32 * kEpiGroups) {
                    float v[32];
                    tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)j0, v);
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        float4* o = reinterpret_cast<float4*>(orow + j0 + j);
                        float y[4] = {v[j], v[j + 1], v[j + 2], v[j + 3]};
                        float rv[4];
                        if (kEarly || !C::LATE3 || !resid) {  // the staged operand (p*S + F + X, or C)
                            const float4 r4 = o[0];
                            rv[0] = r4.x, rv[1] = r4.y, rv[2] = r4.z, rv[3] = r4.w;
                        } else {  // late staging: S, F and X rows as fetched
                            const float4 s4 = o[0], f4 = o[BM * RS / 4], x4 = o[2 * BM * RS / 4];
                            rv[0] = a.p * s4.x + f4.x + x4.x;
                            rv[1] = a.p * s4.y + f4.y + x4.y;
                            rv[2] = a.p * s4.z + f4.z + x4.z;
                            rv[3] = a.p * s4.w + f4.w + x4.w;
                        }
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            if (a.wscale) y[i] = y[i] * wsc[j0 + j + i];
                            // same arithmetic as tc_operand and the staged block path
                            y[i] = resid ? y[i] + rv[i] : rv[i] + y[i];
                        }
                        o[0] = make_float4(y[0], y[1], y[2], y[3]);
                    }
                }
                store_rows(ra + q * 32 * RS, nullptr, nullptr);
            } else if (rows) {
                float* orow = reinterpret_cast<float*>(sb) + row * RS;
                __nv_bfloat16* hrow =
                    a.Ch ? reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<float*>(sb) + BM * RS) +
                               row * RSH
                         : nullptr;
                __nv_bfloat16* lrow = a.Ch ? hrow + BM * RSH : nullptr;
#pragma unroll 1
                for (int j0 = g * 32; ok && !*give_up && j0 < BN; j0 += 32 * kEpiGroups) {
                    float v[32];
                    tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)j0, v);
                    __nv_bfloat16* h = hrow ? hrow + j0 : nullptr;
                    __nv_bfloat16* l = lrow ? lrow + j0 : nullptr;
                    float* out = orow + j0;
                    switch (a.epi) {
                        case kEpiWedge: tc_row_block<kEpiWedge>(a, v, wsc + j0, out, h, l); break;
                        case kEpiRelu2: tc_row_block<kEpiRelu2>(a, v, wsc + j0, out, h, l); break;
                        case kEpiTanh: tc_row_block<kEpiTanh>(a, v, wsc + j0, out, h, l); break;
                        case kEpiSigmoid: tc_row_block<kEpiSigmoid>(a, v, wsc + j0, out, h, l); break;
                        default: tc_row_block<kEpiNone>(a, v, wsc + j0, out, h, l);
                    }
                }
                const __nv_bfloat16* hs =
                    reinterpret_cast<const __nv_bfloat16*>(reinterpret_cast<float*>(sb) + BM * RS) +
                    q * 32 * RSH;
                store_rows(reinterpret_cast<float*>(sb) + q * 32 * RS, a.Ch ? hs : nullptr,
                           a.Ch ? hs + BM * RSH : nullptr);
            } else if (g == 0 && ok && !*give_up) {
                // 32x32 blocks go through shared memory (the drained ring) so that a
                // warp touches one 128-byte row segment per global access
                float* stg = reinterpret_cast<float*>(sb) + (warp - 2) * (32 * 33);
#pragma unroll 1
                for (int j0 = 0; j0 < BN; j0 += 32) {
                    float v[32];
                    tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)j0, v);
#pragma unroll
                    for (int j = 0; j < 32; ++j) stg[lane * 33 + j] = v[j];
                    __syncwarp();
                    const int n = n0 + j0 + lane;
                    const bool nok = n < a.N;
                    if (!LOADS) {
                        // the epilogue kind is chosen once per block, not per element
                        const float ws = a.wscale && nok ? a.wscale[n] : 1.0f;
                        const int mr0 = m0 + q * 32;
                        switch (a.epi) {
                            case kEpiWedge: tc_rows<kEpiWedge>(a, mr0, n, nok, ws, stg, lane); break;
                            case kEpiRelu2: tc_rows<kEpiRelu2>(a, mr0, n, nok, ws, stg, lane); break;
                            case kEpiTanh: tc_rows<kEpiTanh>(a, mr0, n, nok, ws, stg, lane); break;
                            case kEpiSigmoid: tc_rows<kEpiSigmoid>(a, mr0, n, nok, ws, stg, lane); break;
                            default: tc_rows<kEpiNone>(a, mr0, n, nok, ws, stg, lane);
                        }
                    } else {
                        if (BN > 32)  // wider tiles: this block's operands now
                            tc_block_operands(a, m0 + q * 32, n, pre_w, lane);
                        const float ws = a.wscale && nok ? a.wscale[n] : 1.0f;
#pragma unroll 4
                        for (int r = 0; r < 32; ++r) {
                            const long long mr = m0 + q * 32 + r;
                            if (mr < a.M && nok) {
                                float acc = stg[r * 33 + lane];
                                if (a.wscale) acc = acc * ws;
                                const float pr = pre_w[r * 33 + lane];
                                const float y = a.epi == kEpiResid ? acc + pr : pr + acc;
                                a.C[mr * a.ldc + n] = y;
                                if (a.Ch)
                                    store_split((__nv_bfloat16*)a.Ch, (__nv_bfloat16*)a.Cl,
                                                mr * a.ldc + n, y);
                            }
                        }
                    }
                    __syncwarp();
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTmemCols)
                     : "memory");
    }
    if (ks > 1) {
        // every thread of the cluster reaches both barriers (all waits above
        // are bounded). CTA kz finishes rows [kz*rows, (kz+1)*rows) of the
        // tile, summing the cluster's partials in rank order (results do not
        // depend on timing); no CTA leaves while its partials may be read.
        cluster_sync();
        if (warp >= 2 && warp < 2 + 4 * kEpiGroups) {  // every epilogue thread
            const int et = threadIdx.x - 64, nt = 128 * kEpiGroups, rows = BM / ks, r0 = kz * rows;
            const float* part = reinterpret_cast<const float*>(sb);
            switch (a.epi) {
                case kEpiWedge: tc_reduce<kEpiWedge, BN>(a, part, ks, rows, r0, m0, n0, et, nt, reinterpret_cast<const float4*>(pre_all)); break;
                case kEpiResid: tc_reduce<kEpiResid, BN>(a, part, ks, rows, r0, m0, n0, et, nt, reinterpret_cast<const float4*>(pre_all)); break;
                case kEpiAdd: tc_reduce<kEpiAdd, BN>(a, part, ks, rows, r0, m0, n0, et, nt, reinterpret_cast<const float4*>(pre_all)); break;
                case kEpiRelu2: tc_reduce<kEpiRelu2, BN>(a, part, ks, rows, r0, m0, n0, et, nt, reinterpret_cast<const float4*>(pre_all)); break;
                case kEpiTanh: tc_reduce<kEpiTanh, BN>(a, part, ks, rows, r0, m0, n0, et, nt, reinterpret_cast<const float4*>(pre_all)); break;
                case kEpiSigmoid: tc_reduce<kEpiSigmoid, BN>(a, part, ks, rows, r0, m0, n0, et, nt, reinterpret_cast<const float4*>(pre_all)); break;
                default: tc_reduce<kEpiNone, BN>(a, part, ks, rows, r0, m0, n0, et, nt, reinterpret_cast<const float4*>(pre_all));
            }
        }
        cluster_sync();
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

// bf16 (rows, K) K-major plane, box = 64 x box_rows, SWIZZLE_128B
int encode_map(CUtensorMap* tm, const void* base, long long rows, int K, int box_rows) {
    return encode_tiled(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, K, rows, (long long)K * 2, BK,
                        box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
}

// Activation planes per K, reused by every contraction with that K (they run
// in stream order). Grown only outside graph capture; superseded planes stay
// allocated because captured graphs may still reference them.
struct ActPlanes {
    long long cap = 0;
    __nv_bfloat16 *hi = nullptr, *lo = nullptr;
    CUtensorMap tm_hi, tm_lo;
};
std::map<int, ActPlanes>& act_cache() {
    static std::map<int, ActPlanes> c;
    return c;
}

template <int BN, bool I8, bool LOADS, bool CV = false>
int launch_bn(const GemmArgs& a, const TcWeights& tw, const CUtensorMap& tah,
              const CUtensorMap& tal, cudaStream_t st, bool pdl, int ks) {
    using C = TcCfg<BN, I8, LOADS>;
    static bool attr = false;
    auto k = tc_gemm_kernel<BN, I8, LOADS, CV>;
    if (!attr) {
        SN_TRY(cuda_check(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               C::SMEM),
                          "tc smem"));
        attr = true;
    }
    const int bi = BN == 32 ? 0 : (BN == 64 ? 1 : (BN == 128 ? 2 : (BN == 256 ? 3 : 4)));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(((a.N + BN - 1) / BN) * ks), (unsigned)((a.M + BM - 1) / BM));
    cfg.blockDim = dim3(TcThreads<BN, CV>::N);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute la[2];
    int na = 0;
    if (pdl) {
        la[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        la[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (ks > 1) {  // split K over a cluster of ks CTAs along x
        la[na].id = cudaLaunchAttributeClusterDimension;
        la[na].val.clusterDim.x = (unsigned)ks;
        la[na].val.clusterDim.y = 1;
        la[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = la;
    cfg.numAttrs = na;
    GemmArgs ka = a;
    if (CV) {  // the converter warps read the (16-byte aligned) codes
        ka.W = tw.q8;
        ka.ldw = tw.K;
    }
    return cuda_check(cudaLaunchKernelEx(&cfg, k, tah, tal, tw.tm_hi[bi], tw.tm_lo[bi], ka,
                                         rt().d_err),
                      "tc_gemm launch");
}

}  // namespace

// 2-D tensor map: `rows` rows of `inner` elements, `row_bytes` apart, box
// box_inner x box_rows, out-of-range elements read as zero.
int encode_tiled(CUtensorMap* tm, CUtensorMapDataType type, const void* base, long long inner,
                 long long rows, long long row_bytes, int box_inner, int box_rows,
                 CUtensorMapSwizzle swz) {
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(SN_E_DEVICE, "cuTensorMapEncodeTiled entry point unavailable");
    const CUresult r = enc(tm, type, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? SN_OK : fail(SN_E_DEVICE, "cuTensorMapEncodeTiled failed (%d)", (int)r);
}

int tc_reserve(int K, long long rows) {
    if (K % 8 != 0 || rows <= 0) return SN_OK;
    ActPlanes& p = act_cache()[K];
    if (p.cap >= rows) return SN_OK;
    long long cap = 128;
    while (cap < rows) cap *= 2;
    void *hi = nullptr, *lo = nullptr;
    if (cudaMalloc(&hi, (size_t)cap * K * 2) != cudaSuccess ||
        cudaMalloc(&lo, (size_t)cap * K * 2) != cudaSuccess) {
        cudaGetLastError();
        if (hi) cudaFree(hi);
        return fail(SN_E_NOMEM, "activation planes (%lld x %d)", cap, K);
    }
    ActPlanes np;
    np.cap = cap;
    np.hi = (__nv_bfloat16*)hi;
    np.lo = (__nv_bfloat16*)lo;
    SN_TRY(encode_map(&np.tm_hi, np.hi, cap, K, BM));
    SN_TRY(encode_map(&np.tm_lo, np.lo, cap, K, BM));
    p = np;  // the old planes (if any) stay allocated for graphs that captured them
    return SN_OK;
}

int tc_prepare(TcWeights* tw, const void* W, int wtype, int N, int K,
               void* (*alloc)(size_t, void*), void* owner) {
    tw->N = N;
    tw->K = K;
    tw->int8 = wtype == kWI8;
    tw->ready = false;
    const int rows[5] = {32, 64, 128, 256, 192};  // weight tile heights (BN)
    if (tw->int8 && rt().int8_mainloop) {
        // the codes stay as they are: the contraction's converter warps read
        // each K slab's codes and write its bf16 slab (rows of K bytes, 16-byte
        // aligned: K % 16 == 0)
        if (K % 16 != 0) return SN_OK;
        const int8_t* q = reinterpret_cast<const int8_t*>(W);
        if ((uintptr_t)q % 16 != 0) {  // a 16-byte aligned copy
            int8_t* c = (int8_t*)alloc((size_t)N * K, owner);
            if (!c) return fail(SN_E_NOMEM, "tc int8 weights");
            SN_TRY(cuda_check(cudaMemcpy(c, q, (size_t)N * K, cudaMemcpyDeviceToDevice),
                              "tc int8 copy"));
            q = c;
        }
        tw->q8 = q;
        // valid maps for the kernel's parameters (not used for the weights)
        for (int i = 0; i < 5; ++i) {
            SN_TRY(encode_tiled(&tw->tm_lo[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, q, K, N, K, BK,
                                rows[i], CU_TENSOR_MAP_SWIZZLE_NONE));
            tw->tm_hi[i] = tw->tm_lo[i];
        }
        tw->ready = true;
        return SN_OK;
    }
    if (tw->int8) {  // bf16 code planes (exact), loaded by TMA; no lo plane
        if (K % 8 != 0) return SN_OK;
        const size_t n = (size_t)N * K;
        tw->hi = (__nv_bfloat16*)alloc(n * 2, owner);
        if (!tw->hi) return fail(SN_E_NOMEM, "tc weight planes");
        split_bf16_kernel<<<grid_blocks((long long)n), 256>>>(W, wtype, (long long)n, tw->hi,
                                                              nullptr);
        SN_TRY(cuda_check(cudaGetLastError(), "split launch"));
        for (int i = 0; i < 5; ++i) {
            SN_TRY(encode_map(&tw->tm_hi[i], tw->hi, N, K, rows[i]));
            tw->tm_lo[i] = tw->tm_hi[i];
        }
        tw->ready = true;
        return SN_OK;
    }
    if (K % 8 != 0) return SN_OK;  // TMA row stride must be a multiple of 16 bytes
    const size_t n = (size_t)N * K;
    tw->hi = (__nv_bfloat16*)alloc(n * 2, owner);
    tw->lo = (__nv_bfloat16*)alloc(n * 2, owner);
    if (!tw->hi || !tw->lo) return fail(SN_E_NOMEM, "tc weight planes");
    split_bf16_kernel<<<grid_blocks((long long)n), 256>>>(W, wtype, (long long)n, tw->hi, tw->lo);
    SN_TRY(cuda_check(cudaGetLastError(), "split launch"));
    for (int i = 0; i < 5; ++i) {
        SN_TRY(encode_map(&tw->tm_hi[i], tw->hi, N, K, rows[i]));
        SN_TRY(encode_map(&tw->tm_lo[i], tw->lo, N, K, rows[i]));
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
    if (disabled || !tw || !tw->ready || a.M < 16 || a.K != tw->K || a.N != tw->N ||
        a.K % 8 != 0 || a.lda % 4 != 0 || ((uintptr_t)a.A % 16) != 0)
        return false;
    auto it = act_cache().find(a.K);
    return it != act_cache().end() && it->second.cap >= a.M;  // planes reserved up front
}

namespace {

// Whether K may split ks ways for a tile width (host side): each CTA's
// partial tile [BM][BN + 4] fp32 must fit its drained ring and, for residual /
// accumulate kinds, the owner's operand rows ([BM / ks][BN] fp32) the operand
// area next to it.
template <int B, bool I, bool L>
bool split_fits_cfg(int ks) {
    using C = TcCfg<B, I, L>;
    return BM % ks == 0 && BM * (B + 4) * 4 <= C::S * C::STAGE && (!L || (BM / ks) * B * 4 <= C::PRE);
}
bool split_fits(int b, bool i8, bool ld, int ks) {
#define SN_FIT(B)                                                                        \
    if (b == B)                                                                          \
        return i8 ? (ld ? split_fits_cfg<B, true, true>(ks) : split_fits_cfg<B, true, false>(ks)) \
                  : (ld ? split_fits_cfg<B, false, true>(ks) : split_fits_cfg<B, false, false>(ks));
    SN_FIT(32)
    SN_FIT(64)
    SN_FIT(128)
    SN_FIT(192)
    SN_FIT(256)
#undef SN_FIT
    return false;
}

// Tile width BN and K split ks from a cost model of this kernel, per CTA in
// SM cycles, fitted to launches timed back to back on B200 decode and prefill
// shapes: ~10400 of launch, first-slab latency and epilogue, then per K slab
// the slower of its TMA bytes at ~92 B/cycle (2 x 128 x 128 B of A planes +
// 128 B per weight row and plane) and its MMAs (two or three per 16-wide K
// step; one M=128 tcgen05.mma of N columns takes max(90, 0.63 N) cycles, so
// narrow tiles are issue-bound), and 4500 + 22 per column for a split's
// cluster reduction and co-scheduling (a cluster waits for SMs of one GPC to
// be free together, which the step's overlapping kernels make costly); times
// the number of waves. Split K needs a
// 16-byte-friendly epilogue, partial and operand tiles that fit shared memory
// (split_fits) and >= 8 K slabs (two per CTA at least).
int launch_tiles(const GemmArgs& a, const TcWeights& tw, const CUtensorMap& tah,
                 const CUtensorMap& tal, cudaStream_t st, bool pdl) {
    const long long mt = (a.M + BM - 1) / BM;
    const long long sms = rt().num_sms;
    const int nkt = (a.K + BK - 1) / BK;
    auto al16 = [](const void* p, long long ld) {
        return p == nullptr || ((uintptr_t)p % 16 == 0 && ld % 4 == 0);
    };
    bool vec = a.N % 4 == 0 && al16(a.C, a.ldc) &&
               (a.Ch == nullptr || ((uintptr_t)a.Ch % 8 == 0 && (uintptr_t)a.Cl % 8 == 0));
    if (a.epi == kEpiResid) vec = vec && al16(a.S, a.lds) && al16(a.F, a.ldf) && al16(a.X, a.ldx);
    const bool may_split = vec && nkt >= 8 && !getenv("SN_TC_NO_SPLITK");
    const bool ld = a.epi == kEpiResid || a.epi == kEpiAdd;
    // residual / accumulate tiles of 64 or 128 columns stage their operand
    // tile under the main loop when rows are 16-byte aligned and no bf16
    // planes are written; otherwise wide tiles load them block by block after
    // the main loop, which the model does not see: those keep BN = 32 unless
    // that leaves most SMs idle
    const bool staged = ld && vec && a.Ch == nullptr;
    const int bld = mt * ((a.N + 255) / 256) >= sms * 3 / 4   ? 256
                    : mt * ((a.N + 127) / 128) >= sms * 3 / 4 ? 128
                    : mt * ((a.N + 63) / 64) >= sms * 3 / 4   ? 64
                                                              : 32;
    int bn = 32, ks = 1;
    double best = 1e300;
    for (int pass = a.max_ctas > 0 ? 0 : 1; pass < 2 && best == 1e300; ++pass)
    for (int b : {32, 64, 128, 192, 256}) {
        if (ld && (staged ? b > 128 : b != bld)) continue;
        // 192-wide tiles: two ring stages, and neither residual operands nor
        // the bf16 planes of the result fit the drained ring for their epilogue
        if (b == 192 && (ld || a.Ch != nullptr || tw.int8)) continue;
        const long long tiles = mt * ((a.N + b - 1) / b);
        const double bytes = 2.0 * BM * 128 + (tw.q8 ? 0.5 : (tw.int8 ? 1.0 : 2.0)) * b * 128;
        const double mma = 0.63 * b > 90.0 ? 0.63 * b : 90.0;
        const double slab = bytes / 92.0 > (tw.int8 ? 8 : 12) * mma ? bytes / 92.0
                                                                    : (tw.int8 ? 8 : 12) * mma;
        for (int k = 1; k <= 8; k *= 2) {
            if (k > 1 && (!may_split || !split_fits(b, tw.int8, ld, k) || nkt < 2 * k ||
                          tiles * k > sms))
                continue;
            if (pass == 0 && tiles * k > a.max_ctas) continue;  // within the CTA cap first
            const long long waves = (tiles * k + sms - 1) / sms;
            const double t = (double)waves * (10400.0 + ((nkt + k - 1) / k) * slab +
                                              (k > 1 ? 4500.0 + 22.0 * b : 0.0));
            if (t < best * 0.98) {  // a wider or more split choice must win clearly
                best = t;
                bn = b;
                ks = k;
            }
        }
    }
    // SN_TC_FORCE_BN (32/64/128/192/256): a test hook that overrides the
    // model's width, unsplit, wherever that width is allowed for the shape
    if (const char* fb = getenv("SN_TC_FORCE_BN")) {
        const int b = atoi(fb);
        const bool ok = (b == 32 || b == 64 || b == 128 || b == 192 || b == 256) &&
                        (!ld || (staged ? b <= 128 : b == bld)) &&
                        !(b == 192 && (ld || a.Ch != nullptr || tw.int8));
        if (ok) {
            bn = b;
            ks = 1;
            // SN_TC_FORCE_KS (2/4/8) with it: that K split where it is allowed
            if (const char* fk = getenv("SN_TC_FORCE_KS")) {
                const int k = atoi(fk);
                if ((k == 2 || k == 4 || k == 8) && may_split && split_fits(b, tw.int8, ld, k) &&
                    nkt >= 2 * k)
                    ks = k;
            }
        }
    }
#define SN_TC_BN(I8, LD, CV)                                                                  \
    return bn == 256   ? launch_bn<256, I8, LD, CV>(a, tw, tah, tal, st, pdl, ks)              \
           : bn == 192 ? launch_bn<192, I8, LD, CV>(a, tw, tah, tal, st, pdl, ks)              \
           : bn == 128 ? launch_bn<128, I8, LD, CV>(a, tw, tah, tal, st, pdl, ks)              \
                       : (bn == 64 ? launch_bn<64, I8, LD, CV>(a, tw, tah, tal, st, pdl, ks)   \
                                   : launch_bn<32, I8, LD, CV>(a, tw, tah, tal, st, pdl, ks))
    if (tw.int8 && tw.q8) {  // codes converted in the main loop
        if (ld) SN_TC_BN(true, true, true);
        SN_TC_BN(true, false, true);
    }
    if (tw.int8) {
        if (ld) SN_TC_BN(true, true, false);
        SN_TC_BN(true, false, false);
    }
    if (ld) SN_TC_BN(false, true, false);
    SN_TC_BN(false, false, false);
#undef SN_TC_BN
}

}  // namespace

int launch_tc_gemm(const GemmArgs& a, const TcWeights& tw, cudaStream_t st) {
    const ActPlanes& ap = act_cache()[a.K];
    split_act_kernel<<<grid_blocks((long long)a.M * (a.K / 8), 256, 8), 256, 0, st>>>(a, ap.hi,
                                                                                     ap.lo);
    SN_TRY(cuda_check(cudaGetLastError(), "split_act launch"));
    return launch_tiles(a, tw, ap.tm_hi, ap.tm_lo, st, false);
}

int tc_act_alloc(TcAct* p, int K, long long rows, void* (*alloc)(size_t, void*), void* owner) {
    *p = TcAct{};
    if (K % 8 != 0 || rows <= 0) return fail(SN_E_INVAL, "tc planes: K %% 8 or rows");
    p->hi = (__nv_bfloat16*)alloc((size_t)rows * K * 2, owner);
    p->lo = (__nv_bfloat16*)alloc((size_t)rows * K * 2, owner);
    if (!p->hi || !p->lo) return fail(SN_E_NOMEM, "tc planes (%lld x %d)", rows, K);
    return tc_act_view(p, *p, 0, rows, K, K);
}

int tc_act_view(TcAct* v, const TcAct& base, long long off, long long rows, long long ld, int K) {
    if (off % 8 || ld % 8 || K % 8 || rows <= 0) return fail(SN_E_INVAL, "tc plane view");
    TcAct t;
    t.K = K;
    t.rows = rows;
    t.ld = ld;
    t.hi = base.hi + off;
    t.lo = base.lo + off;
    SN_TRY(encode_tiled(&t.tm_hi, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, t.hi, K, rows, ld * 2, BK, BM,
                        CU_TENSOR_MAP_SWIZZLE_128B));
    SN_TRY(encode_tiled(&t.tm_lo, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, t.lo, K, rows, ld * 2, BK, BM,
                        CU_TENSOR_MAP_SWIZZLE_128B));
    t.ready = true;
    *v = t;
    return SN_OK;
}

int launch_split_rows(const float* A, long long rows, int K, long long lda, const TcAct& dst,
                      cudaStream_t st) {
    if (!dst.ready || dst.K != K || dst.ld != K || rows > dst.rows || K % 8 || lda % 4 ||
        (uintptr_t)A % 16)
        return fail(SN_E_INVAL, "split_rows: planes do not fit");
    GemmArgs g;
    g.M = (int)rows;
    g.K = K;
    g.A = A;
    g.lda = lda;
    split_act_kernel<<<grid_blocks(rows * (K / 8), 256, 8), 256, 0, st>>>(g, dst.hi, dst.lo);
    return cuda_check(cudaGetLastError(), "split_rows launch");
}

int launch_tc_gemm_act(const GemmArgs& a, const TcWeights& tw, const TcAct& act, cudaStream_t st,
                       bool pdl) {
    if (!tw.ready || !act.ready || a.K != tw.K || a.N != tw.N || a.K != act.K || a.M > act.rows ||
        a.M <= 0)
        return fail(SN_E_INVAL, "tc_gemm_act: shape does not match the planes / weights");
    return launch_tiles(a, tw, act.tm_hi, act.tm_lo, st, pdl);
}

}  // namespace sn
