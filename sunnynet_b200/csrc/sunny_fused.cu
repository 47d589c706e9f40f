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
// its weights for a phase are one or two contiguous byte ranges. Staged
// variant (the slices fit two shared-memory buffers): at the start of phase
// p thread 0 bulk-copies phase p+1's ranges into the buffer phase p-1 used
// (cp.async.bulk, completion on that buffer's mbarrier), so each phase finds
// its weights on chip and the HBM stream runs under the barrier chain; the
// head (largest slice) is read from global memory behind an L2 prefetch
// issued a layer ahead. Unstaged variant: every phase reads global memory
// behind cp.async.bulk.prefetch.L2 hints issued kPrefetchAhead phases ahead.
// Within a phase a warp takes two weight rows at a time so their loads
// overlap; loads that do not depend on the phase's dot products (ring rows,
// residual terms) are issued with the phase inputs.
//
// Barriers. The launch is cooperative (all CTAs co-resident). Barrier k of a
// launch: thread 0 adds 1 to a monotonic counter with red.release (after
// bar.sync, so the release covers the whole CTA's writes) and polls it with
// acquire loads until it reaches (k+1)*CTAs. The counter
// is zeroed before each launch. Data written by other CTAs is read with
// ld.global.cg (L2), never through L1 or the read-only path. Every wait is
// bounded (~2^31 cycles): on give-up the CTA sets the abort word and the
// device error word, and all CTAs leave at their next barrier. In profile
// mode thread 0 of every CTA records %globaltimer at each phase end and
// barrier exit (FusedArgs::trace).
#include <cuda_fp16.h>

#include <algorithm>

#include "gemm.cuh"
#include "ptx.cuh"
#include "runtime.cuh"
#include "sunny_fused.cuh"
#include "grid_sync.cuh"

namespace sn {
namespace {

constexpr int kWarps = kFusedThreads / 32;
constexpr int kPrefetchAhead = 4;  // phases (one layer)
constexpr unsigned kPrefetchChunk = 1u << 16;

__device__ __forceinline__ void bulk_prefetch_l2(const void* p, unsigned bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ float sigm(float x) { return 1.0f / (1.0f + expf(-x)); }

__device__ __forceinline__ float warp_sum(float v) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Profile mode: %globaltimer (shared time base, ~1 us ticks) and clock64
// (this SM's cycles, fine-grained) at mark e of this CTA.
__device__ __forceinline__ void trace_mark(const FusedArgs& a, int e) {
    if (a.trace && threadIdx.x == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        unsigned long long* row = a.trace + (size_t)blockIdx.x * 2 * a.trace_slots;
        row[e] = t;
        row[a.trace_slots + e] = (unsigned long long)clock64();
    }
}

__device__ __forceinline__ int slice_lo(int total, int part, int parts) {
    return (int)((long long)total * part / parts);
}

template <int WT>
struct WBytes {
    static constexpr int v = WT == kWF32 ? 4 : (WT == kWI8 ? 1 : 2);
};

// Per-lane partial dot products of NR weight rows (row r starts at rp[r]:
// global memory, or this CTA's staged copy in shared memory when S) with the
// B rows of X (shared memory, row stride K); the loads of the NR rows are
// issued together. The caller reduces over lanes.
template <int WT, int NR, bool S, int MB>
__device__ __forceinline__ void rows_dot(const char* const (&rp)[NR], int K, const float* X,
                                         int B, float (&acc)[NR][MB]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int r = 0; r < NR; ++r)
#pragma unroll
        for (int m = 0; m < MB; ++m) acc[r][m] = 0.0f;
    if (WT == kWF32) {
#pragma unroll 2
        for (int k4 = lane; k4 < K / 4; k4 += 32) {
            float4 w[NR];
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                const float4* p = reinterpret_cast<const float4*>(rp[r]) + k4;
                w[r] = S ? *p : __ldg(p);
            }
#pragma unroll
            for (int m = 0; m < MB; ++m) {
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
    } else {
        constexpr int E = WT == kWI8 ? 16 : 8;  // weights per 16-byte load
        for (int kv = lane; kv < K / E; kv += 32) {
            int4 w[NR];
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                const int4* p = reinterpret_cast<const int4*>(rp[r]) + kv;
                w[r] = S ? *p : __ldg(p);
            }
#pragma unroll
            for (int m = 0; m < MB; ++m) {
                if (m < B) {
                    const float* x = X + m * K + E * kv;
#pragma unroll
                    for (int r = 0; r < NR; ++r) {
                        if (WT == kWI8) {
                            const int8_t* wb = reinterpret_cast<const int8_t*>(&w[r]);
#pragma unroll
                            for (int j = 0; j < 16; ++j)
                                acc[r][m] = fmaf((float)wb[j], x[j], acc[r][m]);
                        } else {
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
}

// `count` rows (global row index map(i), data at rowp(i, n)) with the B
// inputs in X, two rows per warp pass. pre(n) is issued before the dot (per
// lane, lane = sequence) and its value handed to emit(i, n, dot, pre) on
// lanes < B. ws: per-row scales of int8 weights (or null).
template <int WT, bool S, int MB, class Map, class RowP, class Pre, class Emit>
__device__ __forceinline__ void rows_loop(const float* ws, int count, Map map, RowP rowp, int K,
                                          const float* X, int B, Pre pre, Emit emit) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int i = warp;
    for (; i + kWarps < count; i += 2 * kWarps) {
        const int n0 = map(i), n1 = map(i + kWarps);
        const char* rp[2] = {rowp(i, n0), rowp(i + kWarps, n1)};
        const float p0 = pre(n0), p1 = pre(n1);
        float acc[2][MB];
        rows_dot<WT, 2, S, MB>(rp, K, X, B, acc);
        float o0 = 0.0f, o1 = 0.0f;
#pragma unroll
        for (int m = 0; m < MB; ++m) {
            if (m < B) {
                const float v0 = warp_sum(acc[0][m]), v1 = warp_sum(acc[1][m]);
                if (lane == m) {
                    o0 = v0;
                    o1 = v1;
                }
            }
        }
        if (ws) {
            o0 *= __ldg(ws + n0);
            o1 *= __ldg(ws + n1);
        }
        if (lane < B) {
            emit(i, n0, o0, p0);
            emit(i + kWarps, n1, o1, p1);
        }
    }
    if (i < count) {
        const int n0 = map(i);
        const char* rp[1] = {rowp(i, n0)};
        const float p0 = pre(n0);
        float acc[1][MB];
        rows_dot<WT, 1, S, MB>(rp, K, X, B, acc);
        float o0 = 0.0f;
#pragma unroll
        for (int m = 0; m < MB; ++m) {
            if (m < B) {
                const float v0 = warp_sum(acc[0][m]);
                if (lane == m) o0 = v0;
            }
        }
        if (ws) o0 *= __ldg(ws + n0);
        if (lane < B) emit(i, n0, o0, p0);
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

// This CTA's weight bytes of phase p (4l+k for layer l, 4L for the head): up
// to two contiguous ranges, in the order the phase's rows are staged.
//   P1: V rows then Ws rows of the CTA's slice of R+D;  P2: the u rows then
//   the gate rows of U for its groups;  P3: Wz rows;  P4: Wc rows;  head rows.
template <int WT>
__device__ void phase_ranges(const FusedArgs& a, const FusedLayer* layers, int p,
                             const char* (&ptr)[2],
                             long long (&bytes)[2]) {
    constexpr int wb = WBytes<WT>::v;
    const int cta = blockIdx.x, nct = gridDim.x;
    ptr[0] = ptr[1] = nullptr;
    bytes[0] = bytes[1] = 0;
    if (p >= 4 * a.L) {
        const int r0 = slice_lo(a.vocab, cta, nct), r1 = slice_lo(a.vocab, cta + 1, nct);
        ptr[0] = reinterpret_cast<const char*>(a.head) + (size_t)r0 * a.D * wb;
        bytes[0] = (long long)(r1 - r0) * a.D * wb;
        return;
    }
    const FusedLayer& y = layers[p / 4];
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

// L2 prefetch hint for phase p's ranges (thread 0).
template <int WT>
__device__ void prefetch_phase(const FusedArgs& a, const FusedLayer* layers, int p) {
    // the head (p == 4L) is staged / prefetched by the kernel at the last layer
    if (!a.bulk_prefetch || threadIdx.x != 0 || p >= 4 * a.L) return;
    const char* ptr[2];
    long long bytes[2];
    phase_ranges<WT>(a, layers, p, ptr, bytes);
    for (int i = 0; i < 2; ++i)
        for (long long o = 0; o < bytes[i]; o += kPrefetchChunk) {
            const long long n = bytes[i] - o < kPrefetchChunk ? bytes[i] - o : kPrefetchChunk;
            bulk_prefetch_l2(ptr[i] + o, (unsigned)n);
        }
}

// Copy phase p's ranges into `buf` (back to back), completing on `mb`
// (thread 0). Every thread's reads of `buf` from its previous use finished
// before the grid barrier that precedes this call.
template <int WT>
__device__ void stage_phase(const FusedArgs& a, const FusedLayer* layers, int p, char* buf,
                            uint64_t* mb) {
    if (threadIdx.x != 0) return;
    const char* ptr[2];
    long long bytes[2];
    phase_ranges<WT>(a, layers, p, ptr, bytes);
    fence_proxy_async_smem();
    mbar_expect_tx(mb, (uint32_t)(bytes[0] + bytes[1]));
    long long off = 0;
    for (int i = 0; i < 2; ++i)
        for (long long o = 0; o < bytes[i]; o += kPrefetchChunk) {
            const long long n = bytes[i] - o < kPrefetchChunk ? bytes[i] - o : kPrefetchChunk;
            bulk_g2s(buf + off, ptr[i] + o, (uint32_t)n, mb);
            off += n;
        }
}

// Shared-memory layout of the fused step, shared by host and device: float
// offsets, then (staged variant) two weight buffers and their mbarriers.
struct FusedSmem {
    int A, Rr, S, Q, stat, pos, par, desc, wbuf, hbuf, mbar, total;  // in floats
    __host__ __device__ FusedSmem(const FusedArgs& a, int ctas) {
        const int maxK = max(a.D, max(a.I, a.R));
        const int NG = a.D / a.G;
        const int groups = (NG + ctas - 1) / ctas;  // most groups a CTA owns
        A = 0;                                      // [B][K] inputs of the phase's rows
        Rr = A + a.B * maxK;                        // [B][D] normalised x (ring row)
        S = Rr + a.B * a.D;                         // [B][D] state before the update
        Q = S + a.B * a.D;  // [groups][2G][8] U outputs (P2), then argmax scratch (head)
        stat = Q + max(groups * 2 * a.G * kFusedMaxB, 2 * kWarps * kFusedMaxB);  // mean, rstd
        pos = stat + 2 * kFusedMaxB;                // [B][L] ring positions, [8] tokens
        par = pos + a.B * a.L + kFusedMaxB;         // the phase's per-channel parameters
        desc = (par + max(3 * a.D, max(2 * a.I, groups * a.G)) + 1) / 2 * 2;  // 8-byte aligned
        wbuf = (desc + a.L * (int)(sizeof(FusedLayer) / 4) + 31) / 32 * 32;  // 128-byte aligned
        hbuf = wbuf + 2 * (a.stage_bytes / 4);      // staged head rows
        mbar = hbuf + a.head_stage_bytes / 4;       // 3 x uint64
        total = mbar + 6;
    }
};

template <int WT, bool STAGE, int MB>
__global__ void __launch_bounds__(kFusedThreads, 1) sunny_fused_kernel(FusedArgs a) {
    extern __shared__ __align__(128) float sm[];
    constexpr int wb = WBytes<WT>::v;
    // MB: compile-time bound of the batch (1: the single-sequence variant)
    const int B = MB == 1 ? 1 : a.B, D = a.D, I = a.I, R = a.R, L = a.L, G = a.G, KH = a.KH,
              Kc = a.K;
    const int cta = blockIdx.x, nct = gridDim.x;
    const FusedSmem lay(a, nct);
    float* bufA = sm + lay.A;
    float* bufR = sm + lay.Rr;
    float* bufS = sm + lay.S;
    float* gq = sm + lay.Q;
    float* stat = sm + lay.stat;
    int* spos = reinterpret_cast<int*>(sm + lay.pos);
    int* stok = spos + B * L;
    float* par = sm + lay.par;
    const FusedLayer* sdesc = reinterpret_cast<const FusedLayer*>(sm + lay.desc);
    char* wbuf = reinterpret_cast<char*>(sm + lay.wbuf);
    char* hbuf = reinterpret_cast<char*>(sm + lay.hbuf);
    uint64_t* mb = reinterpret_cast<uint64_t*>(sm + lay.mbar);  // [0,1] layer, [2] head
    const int tid = threadIdx.x;
    unsigned nbar = 0;
    auto none = [](int) { return 0.0f; };
    const int hr0 = slice_lo(a.vocab, cta, nct), hr1 = slice_lo(a.vocab, cta + 1, nct);
    const int hs = min(hr1 - hr0, a.head_stage_bytes / (D * wb));  // staged head rows

    // profile mode: mark j of phase p (see FusedArgs::trace)
    auto TM = [&](int p, int j) { trace_mark(a, 1 + 8 * p + j); };
    trace_mark(a, 0);
    if (tid == 0) {
        mbar_init(&mb[0], 1);
        mbar_init(&mb[1], 1);
        mbar_init(&mb[2], 1);
        fence_mbar_init();
    }
    {   // layer descriptors into shared memory (read at every parameter access)
        const unsigned* src = reinterpret_cast<const unsigned*>(a.layers);
        unsigned* dst = reinterpret_cast<unsigned*>(sm + lay.desc);
        for (int w = tid; w < L * (int)(sizeof(FusedLayer) / 4); w += kFusedThreads)
            dst[w] = __ldg(src + w);
    }
    for (int i = tid; i < B * L; i += kFusedThreads) spos[i] = ld_cg(a.pos + i);
    if (tid < B) {
        int t = a.tok[tid];
        if (t < 0 || t >= a.vocab) {  // never read outside the table; report instead
            atomicExch(a.err, kErrBadIndex);
            t = 0;
        }
        stok[tid] = t;
    }
    __syncthreads();
    if (tid == 0 && a.bulk_prefetch) {
        // the small per-layer vectors, the recurrent state and the ring rows
        // are read once per step, each right when a phase needs it: pull them
        // all into L2 now, each range by one CTA
        int idx = 0;
        auto pf = [&](const void* p, long long bytes) {
            if (idx++ % nct != cta) return;
            for (long long o = 0; o < bytes; o += kPrefetchChunk)
                bulk_prefetch_l2(static_cast<const char*>(p) + o,
                                 (unsigned)(bytes - o < kPrefetchChunk ? bytes - o : kPrefetchChunk));
        };
        for (int l = 0; l < L; ++l) {
            const FusedLayer& y = sdesc[l];
            pf(y.ni_g, D * 4ll);
            pf(y.ni_c, D * 4ll);
            pf(y.nm_g, I * 4ll);
            pf(y.nm_c, I * 4ll);
            pf(y.dw, (long long)Kc * D * 4);
            pf(y.delta, D * 4ll);
        }
        pf(a.no_g, D * 4ll);
        pf(a.no_c, D * 4ll);
        for (int b = 0; b < B; ++b) {
            pf(a.s + (size_t)b * L * D, (long long)L * D * 4);
            if (Kc > 1) pf(a.hist + (size_t)b * L * KH * D, (long long)L * KH * D * 4);
        }
    }
    if (STAGE) {
        stage_phase<WT>(a, sdesc, 0, wbuf, &mb[0]);
        stage_phase<WT>(a, sdesc, 1, wbuf + a.stage_bytes, &mb[1]);
    } else {
        for (int p = 0; p < kPrefetchAhead; ++p) prefetch_phase<WT>(a, sdesc, p);
    }

    // start of phase p (after its barrier): stage p+1 / prefetch ahead; at
    // the last layer also the head: its first hs rows into hbuf, the rest as
    // an L2 hint. Before its rows: wait for the staged weights of p.
    auto phase_begin = [&](int p) {
        if (STAGE && p >= 1 && p + 1 < 4 * L)
            stage_phase<WT>(a, sdesc, p + 1, wbuf + ((p + 1) & 1) * a.stage_bytes, &mb[(p + 1) & 1]);
        if (p == 4 * L - 4 && a.with_head && tid == 0) {
            const char* h = reinterpret_cast<const char*>(a.head) + (size_t)hr0 * D * wb;
            const long long sb = (long long)hs * D * wb;
            const long long rest = (long long)(hr1 - hr0) * D * wb - sb;
            fence_proxy_async_smem();
            mbar_expect_tx(&mb[2], (uint32_t)sb);
            for (long long o = 0; o < sb; o += kPrefetchChunk)
                bulk_g2s(hbuf + o, h + o, (uint32_t)(sb - o < kPrefetchChunk ? sb - o : kPrefetchChunk),
                         &mb[2]);
            if (a.bulk_prefetch)
                for (long long o = 0; o < rest; o += kPrefetchChunk)
                    bulk_prefetch_l2(h + sb + o,
                                     (unsigned)(rest - o < kPrefetchChunk ? rest - o : kPrefetchChunk));
        }
    };
    auto weights_ready = [&](int p) -> bool {
        if (!STAGE) return true;
        if (mbar_wait(&mb[p & 1], (p >> 1) & 1, a.err)) return true;
        if (tid == 0) atomicExch(a.bar + kBarAbort, 1u);  // others leave at their barrier
        return false;
    };
    auto wrow = [&](int p, long long off) -> const char* {  // staged row of phase p
        return wbuf + (p & 1) * a.stage_bytes + off;
    };

    for (int l = 0; l < L; ++l) {
        const FusedLayer& y = sdesc[l];
        // ------------------------------------------------ P1: LN, taps, V, Ws
        const int p1 = 4 * l;
        phase_begin(p1);
        for (int i = tid; i < B * D; i += kFusedThreads) {
            // every global load of the element first, then the shared stores:
            // a load placed after a store through a generic pointer waits for
            // it, which would serialise the round trips
            const int b = i / D, d = i - b * D;
            const float xv = l == 0 ? a.embed[(size_t)stok[b] * D + d] : ld_cg(a.x + i);
            const float sv = ld_cg(a.s + ((size_t)b * L + l) * D + d);
            float g = 0.0f, c = 0.0f, wl = 0.0f;
            if (b == 0) {  // this layer's LN parameters and newest tap weight
                g = y.ni_g[d];
                c = y.ni_c[d];
                wl = Kc > 1 ? y.dw[(size_t)(Kc - 1) * D + d] : 0.0f;
            }
            float hv[kFusedMaxTaps], wv[kFusedMaxTaps];  // the ring part of the taps
            const int p = spos[b * L + l];
            const float* hb = a.hist + ((size_t)b * L + l) * KH * D;
#pragma unroll
            for (int k = 0; k < kFusedMaxTaps; ++k) {
                if (k < Kc - 1) {
                    const int slot = ((p - 1 - k) % KH + KH) % KH;
                    hv[k] = ld_cg(hb + (size_t)slot * D + d);
                    wv[k] = y.dw[(size_t)(Kc - 2 - k) * D + d];
                }
            }
            float part = 0.0f;
#pragma unroll
            for (int k = 0; k < kFusedMaxTaps; ++k)
                if (k < Kc - 1) part += hv[k] * wv[k];
            if (l == 0 && cta == 0) a.x[i] = xv;
            bufR[i] = xv;
            bufS[i] = sv;
            if (b == 0) {
                par[d] = g;
                par[D + d] = c;
                par[2 * D + d] = wl;
            }
            bufA[i] = part;
        }
        __syncthreads();
        TM(4 * l, 0);
        row_stats(bufR, D, B, a.eps, stat);
        __syncthreads();
        TM(4 * l, 1);
        for (int i = tid; i < B * D; i += kFusedThreads) {
            const int b = i / D, d = i - b * D;
            const float r = (bufR[i] - stat[b]) * stat[kFusedMaxB + b] * par[d] + par[D + d];
            bufR[i] = r;
            bufA[i] = Kc > 1 ? r + (r * par[2 * D + d] + bufA[i]) : r;
        }
        __syncthreads();
        TM(4 * l, 2);
        if (!weights_ready(p1)) return;
        TM(4 * l, 3);
        {
            const int r0 = slice_lo(R + D, cta, nct), r1 = slice_lo(R + D, cta + 1, nct);
            const int v0 = min(r0, R), v1 = min(r1, R);
            const int w0 = max(r0, R) - R, w1 = max(r1, R) - R;
            const long long vbytes = (long long)(v1 - v0) * D * wb;
            rows_loop<WT, STAGE, MB>(
                y.sV, v1 - v0, [=](int i) { return v0 + i; },
                [&](int i, int n) {
                    return STAGE ? wrow(p1, (long long)i * D * wb)
                                 : reinterpret_cast<const char*>(y.V) + (size_t)n * D * wb;
                },
                D, bufA, B, none,
                [&](int, int n, float v, float) { a.v[(threadIdx.x & 31) * R + n] = v; });
            rows_loop<WT, STAGE, MB>(
                y.sWs, w1 - w0, [=](int i) { return w0 + i; },
                [&](int i, int n) {
                    return STAGE ? wrow(p1, vbytes + (long long)i * D * wb)
                                 : reinterpret_cast<const char*>(y.Ws) + (size_t)n * D * wb;
                },
                D, bufS, B, none,
                [&](int, int n, float v, float) { a.sfb[(threadIdx.x & 31) * D + n] = v; });
        }
        TM(4 * l, 4);
        if (!STAGE) prefetch_phase<WT>(a, sdesc, p1 + kPrefetchAhead);
        if (!grid_sync(a.bar, nbar++, a.err)) return;
        TM(4 * l, 5);

        // ------------------------------------ P2: U, competition, state update
        const int p2 = p1 + 1;
        phase_begin(p2);
        {   // v, and the decay gains of this CTA's competition groups
            const int NG = D / G;
            const int c0 = slice_lo(NG, cta, nct) * G, c1 = slice_lo(NG, cta + 1, nct) * G;
            const int n = max(B * R, c1 - c0);
            for (int i = tid; i < n; i += kFusedThreads) {
                const float vv = i < B * R ? ld_cg(a.v + i) : 0.0f;
                const float dl = i < c1 - c0 ? y.delta[c0 + i] : 0.0f;
                if (i < B * R) bufA[i] = vv;
                if (i < c1 - c0) par[i] = dl;
            }
        }
        if (cta == 0 && Kc > 1) {
            for (int i = tid; i < B * D; i += kFusedThreads) {
                const int b = i / D, d = i - b * D;
                const int p = spos[b * L + l];
                a.hist[(((size_t)b * L + l) * KH + ((p % KH) + KH) % KH) * D + d] = bufR[i];
            }
            if (tid < B) a.pos[tid * L + l] = spos[tid * L + l] + 1;
        }
        __syncthreads();
        TM(4 * l + 1, 0);
        TM(4 * l + 1, 1);
        TM(4 * l + 1, 2);
        if (!weights_ready(p2)) return;
        TM(4 * l + 1, 3);
        {
            const int NG = D / G;
            const int g0 = slice_lo(NG, cta, nct), g1 = slice_lo(NG, cta + 1, nct);
            const int twoG = 2 * G;
            const long long ubytes = (long long)(g1 - g0) * G * R * wb;  // the u rows
            rows_loop<WT, STAGE, MB>(
                y.sU, (g1 - g0) * twoG,
                [=](int i) {
                    const int grp = g0 + i / twoG, j = i - (i / twoG) * twoG;
                    return j < G ? grp * G + j : D + grp * G + (j - G);
                },
                [&](int i, int n) {
                    if (!STAGE) return reinterpret_cast<const char*>(y.U) + (size_t)n * R * wb;
                    const int gi = i / twoG, j = i - gi * twoG;
                    const long long row = (long long)gi * G + (j < G ? j : j - G);
                    return wrow(p2, (j < G ? 0 : ubytes) + row * R * wb);
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
                float pg = 1.0f - par[gi * G + j] * (1.0f - sigm(g0v));
                if (a.clamp && pg < a.p_floor) pg = a.p_floor;
                a.s[((size_t)m * L + l) * D + d] = pg * bufS[m * D + d] + (1.0f - pg) * uu;
                a.u[m * D + d] = uu;
            }
        }
        TM(4 * l + 1, 4);
        if (!STAGE) prefetch_phase<WT>(a, sdesc, p2 + kPrefetchAhead);
        if (!grid_sync(a.bar, nbar++, a.err)) return;
        TM(4 * l + 1, 5);

        // ------------------------------------------------------------ P3: Wz
        const int p3 = p2 + 1;
        phase_begin(p3);
        for (int i = tid; i < B * D; i += kFusedThreads) bufA[i] = ld_cg(a.u + i);
        __syncthreads();
        TM(4 * l + 2, 0);
        TM(4 * l + 2, 1);
        TM(4 * l + 2, 2);
        if (!weights_ready(p3)) return;
        TM(4 * l + 2, 3);
        {
            const int r0 = slice_lo(I, cta, nct), r1 = slice_lo(I, cta + 1, nct);
            const float at = y.a_tanh;
            rows_loop<WT, STAGE, MB>(
                y.sWz, r1 - r0, [=](int i) { return r0 + i; },
                [&](int i, int n) {
                    return STAGE ? wrow(p3, (long long)i * D * wb)
                                 : reinterpret_cast<const char*>(y.Wz) + (size_t)n * D * wb;
                },
                D, bufA, B, none,
                [&](int, int n, float acc, float) {
                    a.z[(threadIdx.x & 31) * I + n] =
                        acc * (1.0f + 0.5f * at / (1.0f + fabsf(acc)));
                });
        }
        TM(4 * l + 2, 4);
        if (!STAGE) prefetch_phase<WT>(a, sdesc, p3 + kPrefetchAhead);
        if (!grid_sync(a.bar, nbar++, a.err)) return;
        TM(4 * l + 2, 5);

        // ---------------------------------------------- P4: LN(z), Wc, residual
        const int p4 = p3 + 1;
        phase_begin(p4);
        for (int i = tid; i < B * I; i += kFusedThreads) {
            const float zv = ld_cg(a.z + i);
            float g = 0.0f, c = 0.0f;
            if (i < I) {
                g = y.nm_g[i];
                c = y.nm_c[i];
            }
            bufA[i] = zv;
            if (i < I) {
                par[i] = g;
                par[I + i] = c;
            }
        }
        __syncthreads();
        TM(4 * l + 3, 0);
        row_stats(bufA, I, B, a.eps, stat);
        __syncthreads();
        TM(4 * l + 3, 1);
        for (int i = tid; i < B * I; i += kFusedThreads) {
            const int b = i / I, k = i - b * I;
            bufA[i] = __fmul_rn(__fmul_rn(bufA[i] - stat[b], stat[kFusedMaxB + b]), par[k]) +
                      par[I + k];
        }
        __syncthreads();
        TM(4 * l + 3, 2);
        if (!weights_ready(p4)) return;
        TM(4 * l + 3, 3);
        {
            const int r0 = slice_lo(D, cta, nct), r1 = slice_lo(D, cta + 1, nct);
            const float bg = y.b_gain;
            const int Bq = B;
            // the residual terms do not depend on the dot: issue them first
            auto resid = [&](int n) {
                const int m = threadIdx.x & 31;
                if (m >= Bq) return 0.0f;
                const size_t o = (size_t)m * D + n;
                return bg * ld_cg(a.s + ((size_t)m * L + l) * D + n) + ld_cg(a.sfb + o) +
                       ld_cg(a.x + o);
            };
            rows_loop<WT, STAGE, MB>(
                y.sWc, r1 - r0, [=](int i) { return r0 + i; },
                [&](int i, int n) {
                    return STAGE ? wrow(p4, (long long)i * I * wb)
                                 : reinterpret_cast<const char*>(y.Wc) + (size_t)n * I * wb;
                },
                I, bufA, B, resid,
                [&](int, int n, float acc, float rsd) {
                    a.x[(size_t)(threadIdx.x & 31) * D + n] = acc + rsd;
                });
        }
        TM(4 * l + 3, 4);
        if (!STAGE) prefetch_phase<WT>(a, sdesc, p4 + kPrefetchAhead);
        if (l + 1 < L || a.with_head) {
            if (!grid_sync(a.bar, nbar++, a.err)) return;
            TM(4 * l + 3, 5);
        }
    }
    if (!a.with_head) return;

    // ------------------------------------------- head: LN(x), logits, argmax
    for (int i = tid; i < B * D; i += kFusedThreads) {
        const float xv = ld_cg(a.x + i);
        float g = 0.0f, c = 0.0f;
        if (i < D) {
            g = a.no_g[i];
            c = a.no_c[i];
        }
        bufA[i] = xv;
        if (i < D) {
            par[i] = g;
            par[D + i] = c;
        }
    }
    __syncthreads();
    row_stats(bufA, D, B, a.eps, stat);
    __syncthreads();
    for (int i = tid; i < B * D; i += kFusedThreads) {
        const int b = i / D, k = i - b * D;
        bufA[i] = __fmul_rn(__fmul_rn(bufA[i] - stat[b], stat[kFusedMaxB + b]), par[k]) +
                  par[D + k];
    }
    __syncthreads();
    {
        const int V = a.vocab;
        float bv = -INFINITY;  // this lane's (sequence's) best logit and its row
        int bi = 0x7fffffff;
        auto emit = [&](int, int n, float v, float) {
            if (a.logits) a.logits[(size_t)(threadIdx.x & 31) * V + n] = v;
            if (v > bv || (v == bv && n < bi)) {  // NaN never wins, lowest id on ties
                bv = v;
                bi = n;
            }
        };
        TM(4 * L, 0);
        TM(4 * L, 1);
        TM(4 * L, 2);
        if (hs > 0) {
            if (!(mbar_wait(&mb[2], 0, a.err))) {
                if (tid == 0) atomicExch(a.bar + kBarAbort, 1u);
                return;
            }
            TM(4 * L, 3);
            rows_loop<WT, true, MB>(
                a.shead, hs, [=](int i) { return hr0 + i; },
                [&](int i, int) -> const char* { return hbuf + (size_t)i * D * wb; }, D, bufA, B,
                none, emit);
        }
        if (hs == 0) TM(4 * L, 3);
        rows_loop<WT, false, MB>(
            a.shead, hr1 - hr0 - hs, [=](int i) { return hr0 + hs + i; },
            [&](int, int n) { return reinterpret_cast<const char*>(a.head) + (size_t)n * D * wb; },
            D, bufA, B, none, emit);
        if (a.next) {  // CTA best per sequence, then a packed atomic max across CTAs
            float* wv = gq;  // [warps][8] (P2 scratch is free now)
            int* wi = reinterpret_cast<int*>(gq + kWarps * kFusedMaxB);
            const int warp = tid >> 5, lane = tid & 31;
            if (lane < kFusedMaxB) {
                wv[warp * kFusedMaxB + lane] = bv;
                wi[warp * kFusedMaxB + lane] = bi;
            }
            __syncthreads();
            unsigned long long* slot = reinterpret_cast<unsigned long long*>(a.bar + kBarAmax);
            if (tid < B) {
                float v = -INFINITY;
                int ix = 0x7fffffff;
                for (int w = 0; w < kWarps; ++w) {
                    const float wvv = wv[w * kFusedMaxB + tid];
                    const int wii = wi[w * kFusedMaxB + tid];
                    if (wvv > v || (wvv == v && wii < ix)) {
                        v = wvv;
                        ix = wii;
                    }
                }
                if (ix != 0x7fffffff) {  // ordered float bits above, lowest id wins ties
                    const unsigned f = __float_as_uint(v);
                    const unsigned key = (f & 0x80000000u) ? ~f : (f | 0x80000000u);
                    atomicMax(slot + tid, ((unsigned long long)key << 32) | (0xffffffffu - ix));
                }
            }
            __syncthreads();
            if (tid == 0) {  // the last CTA through here decodes the winners
                __threadfence();
                const unsigned done = atomicAdd(a.bar + kBarDone, 1u);
                if (done == gridDim.x - 1) {
                    __threadfence();
                    for (int m = 0; m < B; ++m) {
                        const unsigned long long k = atomicAdd(slot + m, 0ull);
                        a.next[m] = k ? (int)(0xffffffffu - (unsigned)(k & 0xffffffffu))
                                      : 0x7fffffff;  // every logit NaN
                    }
                }
            }
        }
    }
    TM(4 * L, 4);
}

template <int WT, bool STAGE, int MB>
int launch_wt(const FusedArgs& a, size_t smem, cudaStream_t st) {
    static int ok = -1;
    if (ok < 0) {
        SN_TRY(cuda_check(cudaFuncSetAttribute(sunny_fused_kernel<WT, STAGE, MB>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               kFusedMaxSmem),
                          "fused smem attr"));
        int per_sm = 0;
        SN_TRY(cuda_check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                              &per_sm, sunny_fused_kernel<WT, STAGE, MB>, kFusedThreads,
                              kFusedMaxSmem),
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
    return cuda_check(cudaLaunchKernelEx(&cfg, sunny_fused_kernel<WT, STAGE, MB>, a),
                      "fused step launch");
}

// Largest per-CTA weight slice of any layer phase (bytes), for staging.
long long max_phase_slice(const FusedArgs& a) {
    const int wb = a.wtype == kWF32 ? 4 : (a.wtype == kWI8 ? 1 : 2);
    auto up = [&](long long n) { return (n + a.ctas - 1) / a.ctas; };
    const long long NG = a.D / a.G;
    long long m = up((long long)a.R + a.D) * a.D;
    m = std::max(m, up(NG) * 2 * a.G * a.R);
    m = std::max(m, up(a.I) * a.D);
    m = std::max(m, up(a.D) * a.I);
    return (m * wb + 127) / 128 * 128;
}

}  // namespace

size_t fused_smem_bytes(const FusedArgs& a) {
    if (a.B < 1 || a.B > kFusedMaxB || a.G < 1 || a.G > kFusedMaxG || a.D % a.G) return 0;
    if (a.K < 1 || a.K - 1 > kFusedMaxTaps) return 0;
    if (a.ctas < 1) return 0;
    const int wb = a.wtype == kWF32 ? 4 : (a.wtype == kWI8 ? 16 : 8);  // K multiple for 16 B
    if (a.D % wb || a.I % wb || a.R % wb) return 0;
    const size_t bytes = (size_t)FusedSmem(a, a.ctas).total * sizeof(float);
    return bytes <= (size_t)kFusedMaxSmem ? bytes : 0;
}

size_t fused_plan(FusedArgs* a, bool stage) {
    a->stage_bytes = 0;
    a->head_stage_bytes = 0;
    if (!fused_smem_bytes(*a)) return 0;
    if (stage) {
        a->stage_bytes = (int)max_phase_slice(*a);
        if (!fused_smem_bytes(*a)) a->stage_bytes = 0;
        // the rest of the shared memory holds the first rows of the head slice
        const long long row = (long long)a->D * (a->wtype == kWF32 ? 4 : (a->wtype == kWI8 ? 1 : 2));
        const long long rows = (a->vocab + a->ctas - 1) / a->ctas;
        const long long room = (long long)kFusedMaxSmem - (long long)fused_smem_bytes(*a);
        const long long fit = room > 0 ? room / row : 0;
        a->head_stage_bytes = (int)((fit < rows ? fit : rows) * row);
    }
    return fused_smem_bytes(*a);
}

int launch_sunny_fused(const FusedArgs& a, cudaStream_t st) {
    const size_t smem = fused_smem_bytes(a);
    if (!smem) return fail(SN_E_INVAL, "fused step: shapes unsupported");
    SN_TRY(cuda_check(cudaMemsetAsync(a.bar, 0, kBarWords * sizeof(unsigned), st),
                      "barrier reset"));
    const bool stage = a.stage_bytes > 0, one = a.B == 1;
#define SN_FUSED_LAUNCH(WT)                                                    \
    return stage ? (one ? launch_wt<WT, true, 1>(a, smem, st)                  \
                        : launch_wt<WT, true, kFusedMaxB>(a, smem, st))        \
                 : (one ? launch_wt<WT, false, 1>(a, smem, st)                 \
                        : launch_wt<WT, false, kFusedMaxB>(a, smem, st))
    switch (a.wtype) {
        case kWI8: SN_FUSED_LAUNCH(kWI8);
        case kWF16: SN_FUSED_LAUNCH(kWF16);
        default: SN_FUSED_LAUNCH(kWF32);
    }
#undef SN_FUSED_LAUNCH
}

}  // namespace sn

// ------------------------------------------------- failure-path self-test
// One CTA waits on something nothing will ever complete, through the same
// bounded waits the step kernels use: kind 0 an mbarrier phase no thread
// arrives on, kind 1 a grid barrier (grid_sync) whose arrival target one CTA
// can never reach, kind 2 the same barrier in its two halves (grid_arrive,
// then grid_wait, as the fused RWKV-7 step uses it). The wait gives up after `limit` cycles, records
// kErrWaitTimeout in the error word and the kernel returns, so the host sees
// SN_E_DEVICE and the context stays usable. Nothing is in flight when it
// gives up: no copies, no TMEM.
namespace sn {
namespace {

__device__ unsigned g_selftest_bar[kBarWords];

__global__ void wait_selftest_kernel(int kind, long long limit, int* err) {
    __shared__ __align__(8) uint64_t mb;
    if (kind == 0) {
        if (threadIdx.x == 0) {
            mbar_init(&mb, 1);
            fence_mbar_init();
        }
        __syncthreads();
        mbar_wait_for(&mb, 0, err, limit);  // phase 0 never completes
    } else {
        if (threadIdx.x == 0) {
            g_selftest_bar[0] = 0u;
            g_selftest_bar[kBarAbort] = 0u;
            __threadfence();
        }
        // barrier 3 of a one-CTA grid wants 4 arrivals; only 1 comes
        if (kind == 1) {
            grid_sync(g_selftest_bar, 3u, err, limit);
        } else {
            grid_arrive(g_selftest_bar);
            grid_wait(g_selftest_bar, 3u, err, limit);
        }
    }
}

}  // namespace
}  // namespace sn

extern "C" sn_status sn_abi_cuda_wait_selftest(int32_t kind, int64_t cycles) {
    using namespace sn;
    if (kind < 0 || kind > 2) return fail(SN_E_INVAL, "wait_selftest: kind must be 0, 1 or 2");
    if (cycles < 1 || cycles > kWaitCycles)
        return fail(SN_E_INVAL, "wait_selftest: cycles must be in [1, 2^31]");
    SN_TRY(ensure_init());
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    wait_selftest_kernel<<<1, 32, 0, stream()>>>(kind, (long long)cycles, rt().d_err);
    return finish(true);
}
