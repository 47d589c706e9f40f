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
// Two launches per group of contractions (up to kW4MaxGroup problems sharing
// M, K, the block size and the scale type, e.g. the seven projections of an
// RWKV-7 layer's input mixes):
//   quant_rows_kernel  activation rows -> codes (M,K) int8 + per-block scale
//                      and code sum (a warp per (input, row, block), the
//                      reference's arithmetic), once per distinct input
//   w4a8_tc_kernel     persistent, one CTA per SM over the tiles (problem,
//                      128 sequences, BN output rows), the problem found from
//                      a prefix of tile counts; K walks in 128-byte slabs
//                      through an S-deep shared-memory ring that, like the two
//                      accumulator slots, carries over from tile to tile
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
//                block order in registers (the block's scales brought in by
//                cp.async a few blocks ahead); per tile the epilogue, rows
//                staged in shared memory so each store is one coalesced row
//                segment
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

constexpr int kW4MaxGroup = 8;
constexpr int kScD = 4;  // blocks of scales in flight ahead of the epilogue

// One launch's problems: tensor maps of each problem's activation codes and
// packed weights, outputs, scales, activation block scales and code sums.
struct W4Group {
    CUtensorMap ta[kW4MaxGroup];
    CUtensorMap tw[kW4MaxGroup];
    float* Y[kW4MaxGroup];
    const void* scale[kW4MaxGroup];
    const float* sx[kW4MaxGroup];
    const int* xs[kW4MaxGroup];
    int N[kW4MaxGroup];
    int epi[kW4MaxGroup];
    int tile0[kW4MaxGroup + 1];  // first CTA of each problem; tile0[np] = grid size
    int np;
};

// The distinct inputs of a group, quantised into consecutive planes.
struct W4QGroup {
    const float* X[kW4MaxGroup];
    int n;
};

__device__ __forceinline__ float load_scale_w(const void* s, size_t i, bool fp16) {
    return fp16 ? __half2float(reinterpret_cast<const __half*>(s)[i])
                : reinterpret_cast<const float*>(s)[i];
}

// Rows [mrow0, mrow0 + 32) x columns [n0, n0 + BN) of one tile from the
// warp's staging area to Y with epilogue EPI; lane j stores columns j, j+32,
// so each row is one coalesced segment.
template <int BN, int EPI>
__device__ __forceinline__ void w4_store_rows(float* __restrict__ Y, int N, int M, int mrow0,
                                              int n0, const float* stg, int lane) {
#pragma unroll
    for (int jj = 0; jj < BN / 32; ++jj) {
        const int j = jj * 32 + lane, n = n0 + j;
        if (n >= N) continue;
        // compact loop (runs once per tile, from a cold instruction cache);
        // kW4Add reads 8 rows' old values before storing any of them
#pragma unroll 1
        for (int r0 = 0; r0 < 32; r0 += 8) {
            float old[8];
            if (EPI == kW4Add) {
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    old[q] = mrow0 + r0 + q < M ? Y[(size_t)(mrow0 + r0 + q) * N + n] : 0.0f;
            }
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const int rr = r0 + q;
                if (mrow0 + rr >= M) continue;
                const float v = stg[rr * (BN + 1) + j];
                float* y = Y + (size_t)(mrow0 + rr) * N + n;
                if (EPI == kW4Add) {
                    *y = old[q] + v;
                    } else if (EPI == kW4Relu2) {
                    const float t = v > 0.0f ? v : 0.0f;
                    *y = t * t;
                } else if (EPI == kW4Tanh) {
                    *y = tanhf(v);
                } else if (EPI == kW4Sigmoid) {
                    *y = 1.0f / (1.0f + expf(-v));
                } else {
                    *y = v;
                }
            }
        }
    }
}

// Warp per (input, row, block): the reference's activation quantisation.
// Input u's codes go to plane u of codes / sx / xsum.
__global__ void quant_rows_kernel(const __grid_constant__ W4QGroup q, int M, int K, int block,
                                  int8_t* __restrict__ codes, float* __restrict__ sx,
                                  int* __restrict__ xsum) {
    const int nb = K / block;
    const int lane = threadIdx.x & 31;
    pdl_trigger();
    pdl_wait();  // no-op unless launched with programmatic serialization
    const long long w = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5);
    if (w >= (long long)q.n * M * nb) return;
    const int u = (int)(w / ((long long)M * nb));
    const long long wr = w - (long long)u * M * nb;
    const int m0 = (int)(wr / nb), b = (int)(wr % nb);
    const int m = u * M + m0;  // row of the plane-stacked outputs
    const float* xb = q.X[u] + (size_t)m0 * K + (size_t)b * block;
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

// Per-problem tables of a launch, copied from the parameters into shared
// memory once (indexing the parameter arrays by a run-time problem number
// costs a memory round trip each time).
struct W4Tables {
    int tile0[kW4MaxGroup + 1];
    int N[kW4MaxGroup];
    int epi[kW4MaxGroup];
    float* Y[kW4MaxGroup];
    const void* scale[kW4MaxGroup];
    const float* sx[kW4MaxGroup];
    const int* xs[kW4MaxGroup];
    int np;
};

// Problem, first sequence and first output row of tile t of a group.
template <int BN>
__device__ __forceinline__ void w4_tile(const W4Tables& g, int t, int& pi, int& m0, int& n0) {
    pi = 0;
    while (pi + 1 < g.np && t >= g.tile0[pi + 1]) ++pi;
    const int ntn = (g.N[pi] + BN - 1) / BN, local = t - g.tile0[pi];
    m0 = (local / ntn) * kBM;
    n0 = (local % ntn) * BN;
}

// Persistent: CTA c takes tiles c, c + gridDim.x, ... and every role walks
// the same sequence of (tile, slab) and (tile, block) steps, so the ring and
// the two accumulator slots carry over tile boundaries (the loads and MMAs
// of the next tile overlap the epilogue of the last).
template <int BN, bool FP16S>
__global__ void __launch_bounds__(kW4Threads, 1)
    w4a8_tc_kernel(const __grid_constant__ W4Group g, int M, int K, int block, int* err) {
    using C = W4Cfg<BN>;
    constexpr int S = kW4Stages;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* ring = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    const int nb = K / block, nslab = K / kSlab, bps = kSlab / block, mpb = block / 32;
    const int ntiles = g.tile0[g.np];
    float* stg_all = reinterpret_cast<float*>(ring + S * C::STAGE);  // [4][32][BN+1]
    // per epilogue warp: kScD slots of [32 sx][32 xsum][BN weight-scale words]
    uint32_t* scr_all = reinterpret_cast<uint32_t*>(stg_all + 4 * 32 * (BN + 1));
    uint64_t* full = reinterpret_cast<uint64_t*>(scr_all + 4 * kScD * (64 + BN));
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
    pdl_trigger();  // the next kernel may start its own prologue
    __shared__ W4Tables gt;
#pragma unroll
    for (int i = 0; i < kW4MaxGroup; ++i) {  // constant indices: parameter-bank loads
        if (tid == i) {
            gt.tile0[i] = g.tile0[i];
            gt.N[i] = g.N[i];
            gt.epi[i] = g.epi[i];
            gt.Y[i] = g.Y[i];
            gt.scale[i] = g.scale[i];
            gt.sx[i] = g.sx[i];
            gt.xs[i] = g.xs[i];
        }
    }
    if (tid == kW4MaxGroup) {
        gt.tile0[kW4MaxGroup] = g.tile0[kW4MaxGroup];
        gt.np = g.np;
    }
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
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {  // --------------------------------------------------- TMA
        if (lane == 0) {
            // the packed weights of the first tile's first S slabs do not depend
            // on the previous kernel (the activation quantisation): in flight
            // before waiting for it
            const int pre = nslab < S ? nslab : S;
            if ((int)blockIdx.x < ntiles) {
                int pi, m0, n0;
                w4_tile<BN>(gt, blockIdx.x, pi, m0, n0);
                prefetch_tmap(&g.ta[pi]);  // first used after the wait below
                prefetch_tmap(&g.tw[pi]);
                for (int s = 0; s < pre; ++s) {
                    mbar_expect_tx(&full[s], C::A_BYTES + C::P_BYTES);
                    tma_load_2d(sP(s), &g.tw[pi], s * (kSlab / 2), n0, &full[s]);
                }
            }
            pdl_wait();
            int gs = 0, issued = 0;
            bool run = true;
            for (int t = blockIdx.x; t < ntiles && run; t += gridDim.x) {
                int pi, m0, n0;
                w4_tile<BN>(gt, t, pi, m0, n0);
                for (int s = 0; s < nslab; ++s, ++gs) {
                    const int st = gs % S;
                    if (gs >= pre) {  // first-round stages are never abandoned half-loaded
                        if (*give_up || !mbar_wait(&empty[st], ((gs / S) - 1) & 1, err)) {
                            *give_up = 1;
                            run = false;
                            break;
                        }
                        mbar_expect_tx(&full[st], C::A_BYTES + C::P_BYTES);
                        tma_load_2d(sP(st), &g.tw[pi], s * (kSlab / 2), n0, &full[st]);
                    }
                    tma_load_2d(sA(st), &g.ta[pi], s * kSlab, m0, &full[st]);
                    issued = gs + 1;
                }
            }
            for (int x = issued - S < 0 ? 0 : issued - S; x < issued; ++x)
                mbar_wait(&full[x % S], (x / S) & 1, err);  // no load left in flight
        }
    } else if (warp >= 6) {  // ----------------------------------- unpack nibbles
        const int ut = tid - 192, half = block / 2;
        const int total = ((ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x) * nslab;
        for (int gs = 0; gs < total; ++gs) {
            const int st = gs % S;
            if (*give_up) break;
            if (!mbar_wait(&full[st], (gs / S) & 1, err)) {
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
            const int total =
                ((ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x) * nslab;
            int b = 0;
            bool ok = true;
            for (int gs = 0; gs < total && ok; ++gs) {
                const int st = gs % S;
                if (!mbar_wait(&wready[st], (gs / S) & 1, err)) {
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
        // warp w reads TMEM lanes of quarter w%4: sequences m0 + 32*(w%4) + lane.
        // The scales of block k (activation scale and code sum of the lane's
        // row, weight scale of each output row of the tile) arrive by cp.async
        // in a ring of kScD blocks, issued kScD blocks ahead of their use.
        const int q = warp & 3, wi = warp - 2;
        pdl_wait();  // scales and (kW4Add) outputs come from earlier kernels
        float* stg = stg_all + wi * 32 * (BN + 1);
        uint32_t* scr = scr_all + wi * kScD * (64 + BN);
        int b = 0;  // block counter across tiles (accumulator slot b & 1)
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
            int pi, m0, n0;
            w4_tile<BN>(gt, t, pi, m0, n0);
            const int N = gt.N[pi], mrow0 = m0 + q * 32, m = mrow0 + lane;
            const bool mok = m < M;
            const float* sxr = gt.sx[pi] + (size_t)(mok ? m : 0) * nb;
            const int* xsr = gt.xs[pi] + (size_t)(mok ? m : 0) * nb;
            const char* scale = static_cast<const char*>(gt.scale[pi]);
            auto issue = [&](int k) {  // block k's scales into slot k % kScD
                uint32_t* sl = scr + (k % kScD) * (64 + BN);
                cp_async4(sl + lane, sxr + k, mok ? 4u : 0u);
                cp_async4(sl + 32 + lane, xsr + k, mok ? 4u : 0u);
#pragma unroll
                for (int jj = 0; jj < BN / 32; ++jj) {
                    const int n = n0 + jj * 32 + lane;
                    const size_t e = (size_t)(n < N ? n : 0) * nb + k;
                    // fp16: the aligned 4-byte word holding the element
                    const char* src = FP16S ? reinterpret_cast<const char*>(
                                                  reinterpret_cast<uintptr_t>(scale + 2 * e) & ~(uintptr_t)3)
                                            : scale + 4 * e;
                    cp_async4(sl + 64 + jj * 32 + lane, src, n < N ? 4u : 0u);
                }
            };
#pragma unroll
            for (int p = 0; p < kScD; ++p) {
                if (p < nb) issue(p);
                cp_async_commit();
            }
            float acc[BN];
#pragma unroll
            for (int j = 0; j < BN; ++j) acc[j] = 0.0f;
            bool ok = true;
            // block k of the tile from TMEM values d (block counter bb): the
            // reference's ordered accumulation, then the slot is released
            // block k's weight scales, as they arrived (fp16 in the aligned
            // word that holds it, or fp32) -> fp32 in place: lane j converts
            // column j once, instead of every lane converting every column
            auto decode = [&](int k) {
                uint32_t* sl = scr + (k % kScD) * (64 + BN);
#pragma unroll
                for (int jj = 0; jj < BN / 32; ++jj) {
                    const int j = jj * 32 + lane;
                    if (FP16S) {
                        const uint32_t wd = sl[64 + j];
                        const uintptr_t ea =
                            reinterpret_cast<uintptr_t>(scale + 2 * ((size_t)(n0 + j) * nb + k));
                        sl[64 + j] = __float_as_uint(__half2float(__ushort_as_half(
                            (unsigned short)((ea & 2) ? (wd >> 16) : (wd & 0xFFFFu)))));
                    }
                }
                __syncwarp();
            };
            auto consume = [&](const uint32_t* d, int k, int bb, int j0) {
                const uint32_t* sl = scr + (k % kScD) * (64 + BN);
                const float xs = __uint_as_float(sl[lane]);
                const int x8 = 8 * (int)sl[32 + lane];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const float w = __uint_as_float(sl[64 + j0 + j]);  // same address in every lane
                    const float f = (float)((int)d[j] - x8);
                    acc[j0 + j] = __fadd_rn(acc[j0 + j], __fmul_rn(__fmul_rn(w, xs), f));
                }
            };
            auto wait_acc = [&](int bb) -> bool {  // one decision per warp
                bool w = !*give_up && mbar_wait(&accf[bb & 1], (bb >> 1) & 1, err);
                w = __all_sync(0xffffffffu, w);
                if (!w) *give_up = 1;
                return w;
            };
            auto release = [&](int k, int bb) {  // slot and scale ring entry done
                tc_fence_before();
                mbar_arrive(&acce[bb & 1]);
                __syncwarp();  // every lane is done with the ring slot before it is refilled
                if (k + kScD < nb) issue(k + kScD);
                cp_async_commit();
            };
            const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
            if (BN == 32) {
                // pipelined: block k+1's TMEM load is in flight while block k
                // is applied (two register buffers, alternating)
                uint32_t dA[32], dB[32];
                int k = 0;
                ok = wait_acc(b);
                if (ok) {
                    tc_fence_after();
                    tmem_ld32_issue(trow + (uint32_t)((b & 1) * BN), dA);
                    tmem_wait32(dA);
                }
                while (ok && k < nb) {
                    bool more = k + 1 < nb;
                    if (more) {
                        ok = wait_acc(b + 1);
                        if (ok) {
                            tc_fence_after();
                            tmem_ld32_issue(trow + (uint32_t)(((b + 1) & 1) * BN), dB);
                        }
                    }
                    cp_async_wait_group<kScD - 1>();  // block k's scales have landed
                    __syncwarp();
                    decode(k);
                    consume(dA, k, b, 0);
                    release(k, b);
                    ++k;
                    ++b;
                    if (!ok || !more) break;
                    tmem_wait32(dB);
                    more = k + 1 < nb;
                    if (more) {
                        ok = wait_acc(b + 1);
                        if (ok) {
                            tc_fence_after();
                            tmem_ld32_issue(trow + (uint32_t)(((b + 1) & 1) * BN), dA);
                        }
                    }
                    cp_async_wait_group<kScD - 1>();
                    __syncwarp();
                    decode(k);
                    consume(dB, k, b, 0);
                    release(k, b);
                    ++k;
                    ++b;
                    if (!ok || !more) break;
                    tmem_wait32(dA);
                }
                if (!ok) b += nb - k;  // keep the slot counter in step with the MMA side
            } else {
                for (int k = 0; k < nb; ++k, ++b) {
                    cp_async_wait_group<kScD - 1>();  // block k's group has landed
                    __syncwarp();
                    decode(k);
                    ok = wait_acc(b);
                    if (!ok) break;
                    tc_fence_after();
#pragma unroll
                    for (int j0 = 0; j0 < BN; j0 += 32) {
                        uint32_t d[32];
                        tmem_ld32_u(trow + (uint32_t)((b & 1) * BN + j0), d);
                        consume(d, k, b, j0);
                    }
                    release(k, b);
                }
            }
            cp_async_wait_all();
            if (!ok) break;
            // rows through shared memory: one coalesced segment per stored row
#pragma unroll
            for (int j = 0; j < BN; ++j) stg[lane * (BN + 1) + j] = acc[j];
            __syncwarp();
            float* __restrict__ Y = gt.Y[pi];
            switch (gt.epi[pi]) {
                case kW4Add: w4_store_rows<BN, kW4Add>(Y, N, M, mrow0, n0, stg, lane); break;
                case kW4Relu2: w4_store_rows<BN, kW4Relu2>(Y, N, M, mrow0, n0, stg, lane); break;
                case kW4Tanh: w4_store_rows<BN, kW4Tanh>(Y, N, M, mrow0, n0, stg, lane); break;
                case kW4Sigmoid: w4_store_rows<BN, kW4Sigmoid>(Y, N, M, mrow0, n0, stg, lane); break;
                default: w4_store_rows<BN, kW4Store>(Y, N, M, mrow0, n0, stg, lane);
            }
            __syncwarp();
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * BN);
    }
}

// Workspace for the activation codes of one launch (reused in stream order).
// Grown outside graph capture only; a superseded buffer stays allocated
// because captured graphs may still reference it.
struct W4Work {
    void* p = nullptr;
    size_t cap = 0;
};
W4Work& w4_work() {
    static W4Work w;
    return w;
}

size_t w4_codes_bytes(int planes, int M, int K) {
    return (((size_t)planes * M * K + 255) / 256) * 256;
}
size_t w4_work_bytes(int M, int K, int block, int planes) {
    return w4_codes_bytes(planes, M, K) + (size_t)planes * M * (K / block) * 8;
}

template <int BN, bool FP16S>
int launch_bn(const W4Group& g, int M, int K, int block, cudaStream_t st) {
    // always a programmatic launch: it follows its own quantisation kernel
    using C = W4Cfg<BN>;
    const size_t smem = 1024 + (size_t)kW4Stages * C::STAGE + 4ull * 4 * 32 * (BN + 1) +
                        4ull * 4 * kScD * (64 + BN) + 8ull * (3 * kW4Stages + 5) + 16;
    static int attr = 0;
    if (!attr) {
        SN_TRY(cuda_check(cudaFuncSetAttribute(w4a8_tc_kernel<BN, FP16S>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               200 * 1024),
                          "w4a8_tc smem attr"));
        attr = 1;
    }
    if (smem > 200 * 1024) return fail(SN_E_INVAL, "w4a8_tc: BN=%d needs too much shared memory", BN);
    const int ctas = g.tile0[g.np] < rt().num_sms ? g.tile0[g.np] : rt().num_sms;  // persistent
    return cuda_check(launch_pdl(w4a8_tc_kernel<BN, FP16S>, dim3(ctas), dim3(kW4Threads), smem, st,
                                 g, M, K, block, rt().d_err),
                      "w4a8_tc launch");
}

}  // namespace

bool w4a8_tc_ok(int M, int K, int N, int block, const void* Wq) {
    return M >= 16 && N >= 32 && K % kSlab == 0 && (block == 32 || block == 64 || block == 128) &&
           (uintptr_t)Wq % 16 == 0 && !getenv("SN_DISABLE_TC");
}

bool w4a8_tc_ready(int M, int K, int block, int planes) {
    if (block <= 0 || M <= 0 || planes <= 0) return false;
    return w4_work().cap >= w4_work_bytes(M, K, block, planes);
}

int w4a8_tc_reserve(int M, int K, int block, int planes) {
    if (block <= 0 || M <= 0 || planes <= 0) return fail(SN_E_INVAL, "w4a8_tc: bad reserve shape");
    W4Work& w = w4_work();
    const size_t need = w4_work_bytes(M, K, block, planes);
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

int launch_w4a8_tc_group(const W4Problem* pr, int np, int M, int K, int block, bool fp16,
                         cudaStream_t st, bool pdl) {
    if (np < 1 || np > kW4MaxGroup) return fail(SN_E_INVAL, "w4a8_tc: %d problems in a group", np);
    // distinct inputs, each quantised once
    W4QGroup q;
    q.n = 0;
    int plane[kW4MaxGroup];
    for (int i = 0; i < np; ++i) {
        int u = 0;
        while (u < q.n && q.X[u] != pr[i].X) ++u;
        if (u == q.n) q.X[q.n++] = pr[i].X;
        plane[i] = u;
    }
    W4Work& w = w4_work();
    if (w.cap < w4_work_bytes(M, K, block, q.n))
        return fail(SN_E_INVAL, "w4a8_tc: activation workspace not reserved");
    const int nb = K / block;
    int8_t* codes = static_cast<int8_t*>(w.p);
    float* sx = reinterpret_cast<float*>(static_cast<char*>(w.p) + w4_codes_bytes(q.n, M, K));
    int* xs = reinterpret_cast<int*>(sx + (size_t)q.n * M * nb);
    {
        const long long warps = (long long)q.n * M * nb;
        SN_TRY(cuda_check(launch_pdl_if(pdl, quant_rows_kernel, dim3((unsigned)((warps + 7) / 8)),
                                        dim3(256), 0, st, q, M, K, block, codes, sx, xs),
                          "w4a8_tc quant launch"));
    }
    const int mt = (M + kBM - 1) / kBM;
    long long tiles64 = 0;
    for (int i = 0; i < np; ++i) tiles64 += (long long)((pr[i].N + 63) / 64) * mt;
    const int BN = tiles64 >= rt().num_sms ? 64 : 32;
    W4Group g;
    g.np = np;
    g.tile0[0] = 0;
    for (int i = 0; i < np; ++i) {
        const int u = plane[i];
        SN_TRY(encode_tiled(&g.ta[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, codes + (size_t)u * M * K, K,
                            M, K, kSlab, kBM, CU_TENSOR_MAP_SWIZZLE_128B));
        SN_TRY(encode_tiled(&g.tw[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, pr[i].Wq, K / 2, pr[i].N,
                            K / 2, kSlab / 2, BN, CU_TENSOR_MAP_SWIZZLE_NONE));
        g.Y[i] = pr[i].Y;
        g.scale[i] = pr[i].scale;
        g.sx[i] = sx + (size_t)u * M * nb;
        g.xs[i] = xs + (size_t)u * M * nb;
        g.N[i] = pr[i].N;
        g.epi[i] = pr[i].epi;
        g.tile0[i + 1] = g.tile0[i] + ((pr[i].N + BN - 1) / BN) * mt;
    }
    if (BN == 64)
        return fp16 ? launch_bn<64, true>(g, M, K, block, st) : launch_bn<64, false>(g, M, K, block, st);
    return fp16 ? launch_bn<32, true>(g, M, K, block, st) : launch_bn<32, false>(g, M, K, block, st);
}

int launch_w4a8_tc(float* Y, const float* X, const uint8_t* Wq, const void* scale, int M, int K,
                   int N, int block, bool fp16, int epi, cudaStream_t st, bool pdl) {
    const W4Problem p{Y, X, Wq, scale, N, epi};
    return launch_w4a8_tc_group(&p, 1, M, K, block, fp16, st, pdl);
}

}  // namespace sn
