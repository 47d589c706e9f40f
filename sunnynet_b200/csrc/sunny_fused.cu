// Fused small-batch SunnyNet decode step (see sunny_fused.cuh).
//
// Reference arithmetic: sunnynet/runtime/sunnynet.c (sn_step: LN, depthwise
// taps, readout V/U, gated competition and state update, Wz with softwedge,
// LN + Wc with the residual s*b_gain + Ws s_prev + x, final LN, tied head).
// The per-element formulas are those of the multi-kernel step in sunny.cu;
// the summation order of the dot products and of the causal taps differs
// (fp32 tolerance).
//
// Why one kernel. At B <= 8 every contraction is a GEMV of a few hundred KB
// to a few MB: a launch costs more than its data. Launched as ~40 dependent
// kernels the step is latency-bound (~4-5 us per kernel). Here one CTA per
// SM runs the whole step; a layer is four phases separated by grid barriers:
//   P1  every CTA recomputes LN(x) and the causal taps for the batch in
//       shared memory (a few KB from L2), then its slice of the V rows
//       (v = V at) and of the Ws rows (sfb = Ws s_prev)
//   P2  its slice of the competition groups: the 2G rows of U of each group
//       spread over the CTA's warps, then the gate and the state update for
//       the groups' channels from shared memory; CTA 0 also writes the ring
//       row of the taps (every CTA read the ring in P1)
//   P3  its slice of Wz (z = softwedge(Wz u))
//   P4  LN statistics of z (redundantly per CTA), its slice of Wc with the
//       residual epilogue into x
// and the head is one more phase. Each CTA owns contiguous row ranges, so
// its weights for a phase are one or two contiguous byte ranges: thread 0
// prefetches them into L2 (cp.async.bulk.prefetch) kPrefetchAhead phases
// before they are read, and the HBM stream runs under the barrier chain.
// Within a phase a warp takes two weight rows at a time so their loads
// overlap; loads that do not depend on the phase's dot products (ring rows,
// residual terms) are issued with the phase inputs.
//
// Barriers. The launch is cooperative (all CTAs co-resident). Barrier k of a
// launch: thread 0 adds 1 to a monotonic counter with red.release (after
// bar.sync, so the release covers the whole CTA's writes) and polls it,
// relaxed, until it reaches (k+1)*CTAs, then fences (acquire). The counter
// is zeroed before each launch. Data written by other CTAs is read with
// ld.global.cg (L2), never through L1 or the read-only path. Every wait is
// bounded (~2^31 cycles): on give-up the CTA sets the abort word and the
// device error word, and all CTAs leave at their next barrier. In profile
// mode thread 0 of every CTA records %globaltimer at each phase end and
// barrier exit (FusedArgs::trace).
#include <cuda_fp16.h>

#include "gemm.cuh"
#include "ptx.cuh"
#include "runtime.cuh"
#include "sunny_fused.cuh"

namespace sn {
namespace {

constexpr int kWarps = kFusedThreads / 32;
constexpr int kPrefetchAhead = 4;  // phases (one layer)
constexpr unsigned kPrefetchChunk = 1u << 16;

__device__ __forceinline__ void bulk_prefetch_l2(const void* p, unsigned bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ unsigned ld_relaxed_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_gpu() {
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
}

__device__ __forceinline__ float sigm(float x) { return 1.0f / (1.0f + expf(-x)); }

__device__ __forceinline__ float warp_sum(float v) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Barrier k of this launch; false when the step is being abandoned.
__device__ bool grid_sync(unsigned* bar, unsigned k, int* err) {
    __shared__ int ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        int res = 1;
        const unsigned target = (k + 1) * gridDim.x;
        red_release_add(bar, 1u);
        const long long t0 = clock64();
        unsigned it = 0;
        while (ld_relaxed_u32(bar) < target) {
            if ((++it & 63u) == 0) {
                if (ld_relaxed_u32(bar + kBarAbort)) {
                    res = 0;
                    break;
                }
                if (clock64() - t0 > (1ll << 31)) {
                    atomicExch(bar + kBarAbort, 1u);
                    atomicExch(err, kErrWaitTimeout);
                    res = 0;
                    break;
                }
            }
        }
        fence_acq_rel_gpu();
        ok = res;
    }
    __syncthreads();
    return ok != 0;
}

__device__ __forceinline__ void trace_mark(const FusedArgs& a, int e) {
    if (a.trace && threadIdx.x == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        a.trace[(size_t)blockIdx.x * a.trace_slots + e] = t;
    }
}

__device__ __forceinline__ int slice_lo(int total, int part, int parts) {
    return (int)((long long)total * part / parts);
}

template <int WT>
struct WBytes {
    static constexpr int v = WT == kWF32 ? 4 : (WT == kWI8 ? 1 : 2);
};

// Per-lane partial dot products of NR weight rows (K-major, ldw = K) with
// the B rows of X (shared memory, row stride K); the loads of the NR rows are
// issued together. The caller reduces over lanes.
template <int WT, int NR>
__device__ __forceinline__ void rows_dot(const void* W, const int (&n)[NR], int K, const float* X,
                                         int B, float (&acc)[NR][kFusedMaxB]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int r = 0; r < NR; ++r)
#pragma unroll
        for (int m = 0; m < kFusedMaxB; ++m) acc[r][m] = 0.0f;
    if (WT == kWF32) {
        const float4* w4[NR];
#pragma unroll
        for (int r = 0; r < NR; ++r)
            w4[r] = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(W) +
                                                    (size_t)n[r] * K);
#pragma unroll 2
        for (int k4 = lane; k4 < K / 4; k4 += 32) {
            float4 w[NR];
#pragma unroll
            for (int r = 0; r < NR; ++r) w[r] = __ldg(w4[r] + k4);
#pragma unroll
            for (int m = 0; m < kFusedMaxB; ++m) {
                if (m < B) {
                    const float4 x = *reinterpret_cast<const float4*>(X + m * K + 4 * k4);
#pragma unroll
                    for (int r = 0; r < NR; ++r) {
                        acc[r][m] = fmaf(w[r].x, x.x, acc[r][m]);
                        acc[r][m] = fmaf(w[r].y, x.y, acc[r][m]);
                        acc[r][m] = fmaf(w[r].z, x.z, acc[r][m]);
                        acc[r][m] = fmaf(w[r].w, x.w, acc[r][m]);
                    }
                }
            }
        }
    } else if (WT == kWI8) {
        const int4* w16[NR];
#pragma unroll
        for (int r = 0; r < NR; ++r)
            w16[r] = reinterpret_cast<const int4*>(reinterpret_cast<const int8_t*>(W) +
                                                   (size_t)n[r] * K);
        for (int k16 = lane; k16 < K / 16; k16 += 32) {
            int4 w[NR];
#pragma unroll
            for (int r = 0; r < NR; ++r) w[r] = __ldg(w16[r] + k16);
#pragma unroll
            for (int m = 0; m < kFusedMaxB; ++m) {
                if (m < B) {
                    const float* x = X + m * K + 16 * k16;
#pragma unroll
                    for (int r = 0; r < NR; ++r) {
                        const int8_t* wb = reinterpret_cast<const int8_t*>(&w[r]);
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            acc[r][m] = fmaf((float)wb[j], x[j], acc[r][m]);
                    }
                }
            }
        }
    } else {
        const int4* w8[NR];
#pragma unroll
        for (int r = 0; r < NR; ++r)
            w8[r] = reinterpret_cast<const int4*>(reinterpret_cast<const __half*>(W) +
                                                  (size_t)n[r] * K);
        for (int k8 = lane; k8 < K / 8; k8 += 32) {
            int4 w[NR];
#pragma unroll
            for (int r = 0; r < NR; ++r) w[r] = __ldg(w8[r] + k8);
#pragma unroll
            for (int m = 0; m < kFusedMaxB; ++m) {
                if (m < B) {
                    const float* x = X + m * K + 8 * k8;
#pragma unroll
                    for (int r = 0; r < NR; ++r) {
                        const __half* wh = reinterpret_cast<const __half*>(&w[r]);
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            acc[r][m] = fmaf(__half2float(wh[j]), x[j], acc[r][m]);
                    }
                }
            }
        }
    }
}

// `count` rows of W (row index map(i), i < count) with the B inputs in X,
// two rows per warp pass. pre(n) is issued before the dot (per lane, lane =
// sequence) and its value handed to emit(i, n, dot, pre) on lanes < B.
template <int WT, class Map, class Pre, class Emit>
__device__ __forceinline__ void rows_loop(const void* W, const float* ws, int count, Map map,
                                          int K, const float* X, int B, Pre pre, Emit emit) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int i = warp;
    for (; i + kWarps < count; i += 2 * kWarps) {
        const int n[2] = {map(i), map(i + kWarps)};
        const float p0 = pre(n[0]), p1 = pre(n[1]);
        float acc[2][kFusedMaxB];
        rows_dot<WT, 2>(W, n, K, X, B, acc);
        float o0 = 0.0f, o1 = 0.0f;
#pragma unroll
        for (int m = 0; m < kFusedMaxB; ++m) {
            if (m < B) {
                const float v0 = warp_sum(acc[0][m]), v1 = warp_sum(acc[1][m]);
                if (lane == m) {
                    o0 = v0;
                    o1 = v1;
                }
            }
        }
        if (ws) {
            o0 *= __ldg(ws + n[0]);
            o1 *= __ldg(ws + n[1]);
        }
        if (lane < B) {
            emit(i, n[0], o0, p0);
            emit(i + kWarps, n[1], o1, p1);
        }
    }
    if (i < count) {
        const int n[1] = {map(i)};
        const float p0 = pre(n[0]);
        float acc[1][kFusedMaxB];
        rows_dot<WT, 1>(W, n, K, X, B, acc);
        float o0 = 0.0f;
#pragma unroll
        for (int m = 0; m < kFusedMaxB; ++m) {
            if (m < B) {
                const float v0 = warp_sum(acc[0][m]);
                if (lane == m) o0 = v0;
            }
        }
        if (ws) o0 *= __ldg(ws + n[0]);
        if (lane < B) emit(i, n[0], o0, p0);
    }
}

// Two-pass mean / rstd of B rows of length n in shared memory (warp m < B).
__device__ __forceinline__ void row_stats(const float* X, int n, int B, float eps, float* stat) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp < B) {
        const float* r = X + warp * n;
        float s = 0.0f;
        for (int k = lane; k < n; k += 32) s += r[k];
        const float mean = warp_sum(s) / (float)n;
        float v = 0.0f;
        for (int k = lane; k < n; k += 32) {
            const float d = r[k] - mean;
            v += d * d;
        }
        v = warp_sum(v);
        if (lane == 0) {
            stat[warp] = mean;
            stat[kFusedMaxB + warp] = 1.0f / sqrtf(v / (float)n + eps);
        }
    }
}

template <int WT>
__device__ void prefetch_phase(const FusedArgs& a, int p) {
    if (!a.bulk_prefetch || threadIdx.x != 0 || p > 4 * a.L) return;
    if (p == 4 * a.L && !a.with_head) return;
    constexpr int wb = WBytes<WT>::v;
    const int cta = blockIdx.x, nct = gridDim.x;
    const char* ptr[2] = {nullptr, nullptr};
    long long bytes[2] = {0, 0};
    if (p == 4 * a.L) {
        const int r0 = slice_lo(a.vocab, cta, nct), r1 = slice_lo(a.vocab, cta + 1, nct);
        ptr[0] = reinterpret_cast<const char*>(a.head) + (size_t)r0 * a.D * wb;
        bytes[0] = (long long)(r1 - r0) * a.D * wb;
    } else {
        const FusedLayer& y = a.layers[p / 4];
        const int D = a.D, R = a.R, I = a.I;
        switch (p % 4) {
            case 0: {
                const int r0 = slice_lo(R + D, cta, nct), r1 = slice_lo(R + D, cta + 1, nct);
                const int v0 = min(r0, R), v1 = min(r1, R);
                ptr[0] = reinterpret_cast<const char*>(y.V) + (size_t)v0 * D * wb;
                bytes[0] = (long long)(v1 - v0) * D * wb;
                const int s0 = max(r0, R) - R, s1 = max(r1, R) - R;
                ptr[1] = reinterpret_cast<const char*>(y.Ws) + (size_t)s0 * D * wb;
                bytes[1] = (long long)(s1 - s0) * D * wb;
                break;
            }
            case 1: {
                const int NG = D / a.G;
                const int g0 = slice_lo(NG, cta, nct), g1 = slice_lo(NG, cta + 1, nct);
                ptr[0] = reinterpret_cast<const char*>(y.U) + (size_t)g0 * a.G * R * wb;
                bytes[0] = (long long)(g1 - g0) * a.G * R * wb;
                ptr[1] = reinterpret_cast<const char*>(y.U) + (size_t)(D + g0 * a.G) * R * wb;
                bytes[1] = bytes[0];
                break;
            }
            case 2: {
                const int r0 = slice_lo(I, cta, nct), r1 = slice_lo(I, cta + 1, nct);
                ptr[0] = reinterpret_cast<const char*>(y.Wz) + (size_t)r0 * D * wb;
                bytes[0] = (long long)(r1 - r0) * D * wb;
                break;
            }
            default: {
                const int r0 = slice_lo(D, cta, nct), r1 = slice_lo(D, cta + 1, nct);
                ptr[0] = reinterpret_cast<const char*>(y.Wc) + (size_t)r0 * I * wb;
                bytes[0] = (long long)(r1 - r0) * I * wb;
                break;
            }
        }
    }
    for (int i = 0; i < 2; ++i)
        for (long long o = 0; o < bytes[i]; o += kPrefetchChunk) {
            const long long n = bytes[i] - o < kPrefetchChunk ? bytes[i] - o : kPrefetchChunk;
            bulk_prefetch_l2(ptr[i] + o, (unsigned)n);
        }
}

// Shared-memory layout of the fused step (floats), shared by host and device.
struct FusedSmem {
    int A, Rr, S, Q, stat, pos, total;
    __host__ __device__ FusedSmem(const FusedArgs& a, int ctas) {
        const int maxK = max(a.D, max(a.I, a.R));
        const int NG = a.D / a.G;
        const int groups = (NG + ctas - 1) / ctas;  // most groups a CTA owns
        A = 0;                                      // [B][K] inputs of the phase's rows
        Rr = A + a.B * maxK;                        // [B][D] normalised x (ring row)
        S = Rr + a.B * a.D;                         // [B][D] state before the update
        Q = S + a.B * a.D;                          // [groups][2G][8] U outputs (P2)
        stat = Q + groups * 2 * a.G * kFusedMaxB;   // mean[8], rstd[8]
        pos = stat + 2 * kFusedMaxB;                // [B][L] ring positions at step start
        total = pos + a.B * a.L;
    }
};

template <int WT>
__global__ void __launch_bounds__(kFusedThreads, 1) sunny_fused_kernel(FusedArgs a) {
    extern __shared__ __align__(16) float sm[];
    const int B = a.B, D = a.D, I = a.I, R = a.R, L = a.L, G = a.G, KH = a.KH, Kc = a.K;
    const int cta = blockIdx.x, nct = gridDim.x;
    const FusedSmem lay(a, nct);
    float* bufA = sm + lay.A;
    float* bufR = sm + lay.Rr;
    float* bufS = sm + lay.S;
    float* gq = sm + lay.Q;
    float* stat = sm + lay.stat;
    int* spos = reinterpret_cast<int*>(sm + lay.pos);
    const int tid = threadIdx.x;
    unsigned nbar = 0;
    auto none = [](int) { return 0.0f; };

    trace_mark(a, 0);
    for (int p = 0; p < kPrefetchAhead; ++p) prefetch_phase<WT>(a, p);
    for (int i = tid; i < B * L; i += kFusedThreads) spos[i] = __ldcg(a.pos + i);
    __syncthreads();

    for (int l = 0; l < L; ++l) {
        const FusedLayer& y = a.layers[l];
        // ------------------------------------------------ P1: LN, taps, V, Ws
        for (int i = tid; i < B * D; i += kFusedThreads) {
            const int b = i / D, d = i - b * D;
            float xv;
            if (l == 0) {
                int t = a.tok[b];
                if (t < 0 || t >= a.vocab) {  // never read outside the table; report instead
                    if (d == 0) atomicExch(a.err, kErrBadIndex);
                    t = 0;
                }
                xv = a.embed[(size_t)t * D + d];
                if (cta == 0) a.x[i] = xv;
            } else {
                xv = __ldcg(a.x + i);
            }
            bufR[i] = xv;
            bufS[i] = __ldcg(a.s + ((size_t)b * L + l) * D + d);
            if (Kc > 1) {  // the ring part of the causal taps (no LN needed)
                const int p = spos[b * L + l];
                const float* hb = a.hist + ((size_t)b * L + l) * KH * D;
                float part = 0.0f;
                for (int k = 0; k < Kc - 1; ++k) {
                    const int slot = ((p - 1 - k) % KH + KH) % KH;
                    part += __ldcg(hb + (size_t)slot * D + d) * y.dw[(size_t)(Kc - 2 - k) * D + d];
                }
                bufA[i] = part;
            }
        }
        __syncthreads();
        row_stats(bufR, D, B, a.eps, stat);
        __syncthreads();
        for (int i = tid; i < B * D; i += kFusedThreads) {
            const int b = i / D, d = i - b * D;
            const float r = (bufR[i] - stat[b]) * stat[kFusedMaxB + b] * y.ni_g[d] + y.ni_c[d];
            bufR[i] = r;
            bufA[i] = Kc > 1 ? r + (r * y.dw[(size_t)(Kc - 1) * D + d] + bufA[i]) : r;
        }
        __syncthreads();
        {
            const int r0 = slice_lo(R + D, cta, nct), r1 = slice_lo(R + D, cta + 1, nct);
            const int v0 = min(r0, R), v1 = min(r1, R);
            const int w0 = max(r0, R) - R, w1 = max(r1, R) - R;
            rows_loop<WT>(y.V, y.sV, v1 - v0, [=](int i) { return v0 + i; }, D, bufA, B, none,
                          [&](int, int n, float v, float) { a.v[(threadIdx.x & 31) * R + n] = v; });
            rows_loop<WT>(y.Ws, y.sWs, w1 - w0, [=](int i) { return w0 + i; }, D, bufS, B, none,
                          [&](int, int n, float v, float) {
                              a.sfb[(threadIdx.x & 31) * D + n] = v;
                          });
        }
        trace_mark(a, 1 + 8 * l);
        prefetch_phase<WT>(a, 4 * l + kPrefetchAhead);
        if (!grid_sync(a.bar, nbar++, a.err)) return;
        trace_mark(a, 2 + 8 * l);

        // ------------------------------------ P2: U, competition, state update
        for (int i = tid; i < B * R; i += kFusedThreads) bufA[i] = __ldcg(a.v + i);
        if (cta == 0 && Kc > 1) {
            for (int i = tid; i < B * D; i += kFusedThreads) {
                const int b = i / D, d = i - b * D;
                const int p = spos[b * L + l];
                a.hist[(((size_t)b * L + l) * KH + ((p % KH) + KH) % KH) * D + d] = bufR[i];
            }
            if (tid < B) a.pos[tid * L + l] = spos[tid * L + l] + 1;
        }
        __syncthreads();
        {
            const int NG = D / G;
            const int g0 = slice_lo(NG, cta, nct), g1 = slice_lo(NG, cta + 1, nct);
            const int twoG = 2 * G;
            rows_loop<WT>(
                y.U, y.sU, (g1 - g0) * twoG,
                [=](int i) {
                    const int grp = g0 + i / twoG, j = i - (i / twoG) * twoG;
                    return j < G ? grp * G + j : D + grp * G + (j - G);
                },
                R, bufA, B, none,
                [&](int i, int, float v, float) { gq[i * kFusedMaxB + (threadIdx.x & 31)] = v; });
            __syncthreads();
            for (int t = tid; t < (g1 - g0) * G * B; t += kFusedThreads) {
                const int m = t % B, gj = t / B;
                const int gi = gj / G, j = gj - gi * G;
                const int d = (g0 + gi) * G + j;
                const float* q = gq + gi * twoG * kFusedMaxB;
                const float g0v = q[(G + j) * kFusedMaxB + m];
                const float g1v = q[(G + (j + 1) % G) * kFusedMaxB + m];
                const float g2v = q[(G + (j + 2) % G) * kFusedMaxB + m];
                const float uu = q[j * kFusedMaxB + m] * (sigm(g0v - g1v) * sigm(g0v - g2v));
                float pg = 1.0f - y.delta[d] * (1.0f - sigm(g0v));
                if (a.clamp && pg < a.p_floor) pg = a.p_floor;
                a.s[((size_t)m * L + l) * D + d] = pg * bufS[m * D + d] + (1.0f - pg) * uu;
                a.u[m * D + d] = uu;
            }
        }
        trace_mark(a, 3 + 8 * l);
        prefetch_phase<WT>(a, 4 * l + 1 + kPrefetchAhead);
        if (!grid_sync(a.bar, nbar++, a.err)) return;
        trace_mark(a, 4 + 8 * l);

        // ------------------------------------------------------------ P3: Wz
        for (int i = tid; i < B * D; i += kFusedThreads) bufA[i] = __ldcg(a.u + i);
        __syncthreads();
        {
            const int r0 = slice_lo(I, cta, nct), r1 = slice_lo(I, cta + 1, nct);
            const float at = y.a_tanh;
            rows_loop<WT>(y.Wz, y.sWz, r1 - r0, [=](int i) { return r0 + i; }, D, bufA, B, none,
                          [&](int, int n, float acc, float) {
                              a.z[(threadIdx.x & 31) * I + n] =
                                  acc * (1.0f + 0.5f * at / (1.0f + fabsf(acc)));
                          });
        }
        trace_mark(a, 5 + 8 * l);
        prefetch_phase<WT>(a, 4 * l + 2 + kPrefetchAhead);
        if (!grid_sync(a.bar, nbar++, a.err)) return;
        trace_mark(a, 6 + 8 * l);

        // ---------------------------------------------- P4: LN(z), Wc, residual
        for (int i = tid; i < B * I; i += kFusedThreads) bufA[i] = __ldcg(a.z + i);
        __syncthreads();
        row_stats(bufA, I, B, a.eps, stat);
        __syncthreads();
        for (int i = tid; i < B * I; i += kFusedThreads) {
            const int b = i / I, k = i - b * I;
            bufA[i] = __fmul_rn(__fmul_rn(bufA[i] - stat[b], stat[kFusedMaxB + b]), y.nm_g[k]) +
                      y.nm_c[k];
        }
        __syncthreads();
        {
            const int r0 = slice_lo(D, cta, nct), r1 = slice_lo(D, cta + 1, nct);
            const float bg = y.b_gain;
            const int Bq = B;
            // the residual terms do not depend on the dot: issue them first
            auto resid = [&](int n) {
                const int m = threadIdx.x & 31;
                if (m >= Bq) return 0.0f;
                const size_t o = (size_t)m * D + n;
                return bg * __ldcg(a.s + ((size_t)m * L + l) * D + n) + __ldcg(a.sfb + o) +
                       __ldcg(a.x + o);
            };
            rows_loop<WT>(y.Wc, y.sWc, r1 - r0, [=](int i) { return r0 + i; }, I, bufA, B, resid,
                          [&](int, int n, float acc, float rsd) {
                              a.x[(size_t)(threadIdx.x & 31) * D + n] = acc + rsd;
                          });
        }
        trace_mark(a, 7 + 8 * l);
        prefetch_phase<WT>(a, 4 * l + 3 + kPrefetchAhead);
        if (l + 1 < L || a.with_head) {
            if (!grid_sync(a.bar, nbar++, a.err)) return;
            trace_mark(a, 8 + 8 * l);
        }
    }
    if (!a.with_head) return;

    // --------------------------------------------------- head: LN(x), logits
    for (int i = tid; i < B * D; i += kFusedThreads) bufA[i] = __ldcg(a.x + i);
    __syncthreads();
    row_stats(bufA, D, B, a.eps, stat);
    __syncthreads();
    for (int i = tid; i < B * D; i += kFusedThreads) {
        const int b = i / D, k = i - b * D;
        bufA[i] = __fmul_rn(__fmul_rn(bufA[i] - stat[b], stat[kFusedMaxB + b]), a.no_g[k]) +
                  a.no_c[k];
    }
    __syncthreads();
    {
        const int r0 = slice_lo(a.vocab, cta, nct), r1 = slice_lo(a.vocab, cta + 1, nct);
        const int V = a.vocab;
        rows_loop<WT>(a.head, a.shead, r1 - r0, [=](int i) { return r0 + i; }, D, bufA, B, none,
                      [&](int, int n, float v, float) {
                          a.logits[(size_t)(threadIdx.x & 31) * V + n] = v;
                      });
    }
    trace_mark(a, 1 + 8 * L);
}

template <int WT>
int launch_wt(const FusedArgs& a, size_t smem, cudaStream_t st) {
    static int ok = -1;
    if (ok < 0) {
        SN_TRY(cuda_check(cudaFuncSetAttribute(sunny_fused_kernel<WT>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               200 * 1024),
                          "fused smem attr"));
        int per_sm = 0;
        SN_TRY(cuda_check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                              &per_sm, sunny_fused_kernel<WT>, kFusedThreads, 200 * 1024),
                          "fused occupancy"));
        ok = per_sm >= 1 ? 1 : 0;
    }
    if (!ok) return fail(SN_E_UNSUPPORTED, "fused step: no CTA fits on an SM");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.ctas);
    cfg.blockDim = dim3(kFusedThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_check(cudaLaunchKernelEx(&cfg, sunny_fused_kernel<WT>, a), "fused step launch");
}

}  // namespace

size_t fused_smem_bytes(const FusedArgs& a) {
    if (a.B < 1 || a.B > kFusedMaxB || a.G < 1 || a.G > kFusedMaxG || a.D % a.G) return 0;
    if (a.ctas < 1) return 0;
    const int wb = a.wtype == kWF32 ? 4 : (a.wtype == kWI8 ? 16 : 8);  // K multiple for 16 B
    if (a.D % wb || a.I % wb || a.R % wb) return 0;
    const size_t bytes = (size_t)FusedSmem(a, a.ctas).total * sizeof(float);
    return bytes <= 200 * 1024 ? bytes : 0;
}

int launch_sunny_fused(const FusedArgs& a, cudaStream_t st) {
    const size_t smem = fused_smem_bytes(a);
    if (!smem) return fail(SN_E_INVAL, "fused step: shapes unsupported");
    SN_TRY(cuda_check(cudaMemsetAsync(a.bar, 0, kBarWords * sizeof(unsigned), st),
                      "barrier reset"));
    switch (a.wtype) {
        case kWI8: return launch_wt<kWI8>(a, smem, st);
        case kWF16: return launch_wt<kWF16>(a, smem, st);
        default: return launch_wt<kWF32>(a, smem, st);
    }
}

}  // namespace sn
