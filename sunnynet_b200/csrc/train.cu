// The reference's kernels module (sunnynet/kernels: scan_avx2.c, core_avx2.c,
// step_avx2.c) on sm_100a, under its exported names so its ctypes loader
// (kernels/__init__.py load_kernel) binds this library unchanged:
//
//   scan_f32 / scan_bwd_f32   the gated scan and its reverse pass with the
//                             gate p and the input nu (s = p*s + (1-p)*nu):
//                             the exact scan kernels of recur.cu, bit-exact
//   core_fwd_f32              competition gate + decay gate + scan over T
//   core_bwd_f32              its reverse pass (gradients of q, delta, s0)
//   step_core_f32             one decode step of core_fwd
//   dw_step_f32               one step of the depthwise causal taps, bit-exact
//
// core_* and step_core: one thread per channel, walking T in order (forward)
// or reverse (backward); the competition needs e = exp(-gate) of channels
// i+1 and i+2 of the same group of 8 (and the backward pass a1, a2 of i-1
// and i-2): those come from the neighbouring lanes by warp shuffles within
// 8-lane segments, so a CTA is a whole number of groups. Channels past the
// last full group are left untouched, as the reference's 8-lane loops leave
// them. Every operation is rounded as the reference rounds it (explicit
// fma where it uses _mm256_fmadd_ps, correctly rounded division) except
// exp, which is CUDA's expf rather than the host libm's: results agree to a
// few ulp, not bit for bit. Loads of the next rows are issued before the
// current row is chained, so the serial dependency per row is the state
// update alone.
#include <cuda_runtime.h>

#include "kernels.cuh"
#include "runtime.cuh"

namespace sn {
namespace {

constexpr int kCoreThreads = 128;  // 16 groups of 8 channels per CTA
constexpr int kRows = 8;           // rows loaded ahead of the chain

// v of lane (lane & ~7) | ((lane + k) & 7): the k-th next channel of this
// lane's group of 8, wrapping (torch.roll within the group).
__device__ __forceinline__ float grp(float v, int k) {
    const int lane = threadIdx.x & 31;
    return __shfl_sync(0xffffffffu, v, (lane & ~7) | ((lane + k) & 7));
}

struct Gates {
    float sig, s1, s2;
};

// sigma(g), sigma(g_i - g_{i+1}) and sigma(g_i - g_{i+2}) in the reference's
// ratio form: e = exp(-g), sigma(g_i - g_j) = 1 / (1 + e_i / e_j).
__device__ __forceinline__ Gates gates(float gate) {
    const float e = expf(0.0f - gate);
    const float e1 = grp(e, 1), e2 = grp(e, 2);
    Gates r;
    r.sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
    r.s1 = __fdiv_rn(1.0f, __fadd_rn(1.0f, __fdiv_rn(e, e1)));
    r.s2 = __fdiv_rn(1.0f, __fadd_rn(1.0f, __fdiv_rn(e, e2)));
    return r;
}

// core_avx2.c:34-79
__global__ void __launch_bounds__(kCoreThreads)
    core_fwd_kernel(const float* __restrict__ q, const float* __restrict__ delta,
                    const float* __restrict__ s0, float* __restrict__ states,
                    float* __restrict__ uo, float* __restrict__ po, int T, int D, int DV) {
    const int d = blockIdx.x * kCoreThreads + threadIdx.x;
    const int b = blockIdx.y;
    const bool live = d < DV;  // groups are whole: a group is live or not as a unit
    const int dc = live ? d : 0;
    const float dl = delta[dc];
    const float base = __fsub_rn(1.0f, dl);
    float s = live ? s0[(size_t)b * D + dc] : 0.0f;
    const float* qb = q + (size_t)b * T * 2 * D + dc;
    const size_t ob = (size_t)b * T * D + dc;
    for (int t0 = 0; t0 < T; t0 += kRows) {
        float ur[kRows], gt[kRows];
#pragma unroll
        for (int j = 0; j < kRows; ++j) {
            const bool ok = t0 + j < T;
            ur[j] = ok ? qb[(size_t)(t0 + j) * 2 * D] : 0.0f;
            gt[j] = ok ? qb[(size_t)(t0 + j) * 2 * D + D] : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < kRows; ++j) {
            const Gates g = gates(gt[j]);  // every lane takes part in the shuffles
            const float w = __fmul_rn(g.s1, g.s2);
            const float u = __fmul_rn(ur[j], w);
            const float p = __fmaf_rn(dl, g.sig, base);
            s = __fmaf_rn(p, s, __fmul_rn(__fsub_rn(1.0f, p), u));
            if (live && t0 + j < T) {
                const size_t o = ob + (size_t)(t0 + j) * D;
                states[o] = s;
                uo[o] = u;
                po[o] = p;
            }
        }
    }
}

// core_avx2.c:84-148. ddelta += the sum over this sequence's rows (atomic
// across sequences, as the reference's OpenMP atomics).
__global__ void __launch_bounds__(kCoreThreads)
    core_bwd_kernel(const float* __restrict__ q, const float* __restrict__ delta,
                    const float* __restrict__ s0, const float* __restrict__ states,
                    const float* __restrict__ uo, const float* __restrict__ po,
                    const float* __restrict__ dstate, const float* __restrict__ du_in,
                    float* __restrict__ dq, float* __restrict__ ddelta, float* __restrict__ ds0,
                    int T, int D, int DV) {
    const int d = blockIdx.x * kCoreThreads + threadIdx.x;
    const int b = blockIdx.y;
    const bool live = d < DV;
    const int dc = live ? d : 0;
    const float dl = delta[dc];
    const float s0v = s0[(size_t)b * D + dc];
    const float* qb = q + (size_t)b * T * 2 * D + dc;
    float* dqb = dq + (size_t)b * T * 2 * D + dc;
    const size_t ob = (size_t)b * T * D + dc;
    float ds = 0.0f, dacc = 0.0f;
    for (int t1 = T - 1; t1 >= 0; t1 -= kRows) {
        float gds[kRows], u[kRows], p[kRows], sp[kRows], din[kRows], ur[kRows], gt[kRows];
#pragma unroll
        for (int j = 0; j < kRows; ++j) {  // rows t1, t1-1, ...
            const int t = t1 - j;
            const bool ok = t >= 0;
            const size_t o = ob + (size_t)(ok ? t : 0) * D;
            gds[j] = ok ? dstate[o] : 0.0f;
            u[j] = ok ? uo[o] : 0.0f;
            p[j] = ok ? po[o] : 0.0f;
            sp[j] = ok ? (t > 0 ? states[o - D] : s0v) : 0.0f;
            din[j] = ok ? du_in[o] : 0.0f;
            ur[j] = ok ? qb[(size_t)t * 2 * D] : 0.0f;
            gt[j] = ok ? qb[(size_t)t * 2 * D + D] : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < kRows; ++j) {
            const int t = t1 - j;
            const bool ok = t >= 0;
            float dp = 0.0f, du = 0.0f;
            if (ok) {
                ds = __fadd_rn(ds, gds[j]);
                dp = __fmul_rn(ds, __fsub_rn(sp[j], u[j]));
                du = __fmaf_rn(ds, __fsub_rn(1.0f, p[j]), din[j]);
                ds = __fmul_rn(ds, p[j]);
            }
            const Gates g = gates(gt[j]);
            const float w = __fmul_rn(g.s1, g.s2);
            const float dur = __fmul_rn(du, w);
            const float dw = __fmul_rn(du, ur[j]);
            const float ds1 = __fmul_rn(dw, g.s2), ds2 = __fmul_rn(dw, g.s1);
            const float a1 = __fmul_rn(ds1, __fmul_rn(g.s1, __fsub_rn(1.0f, g.s1)));
            const float a2 = __fmul_rn(ds2, __fmul_rn(g.s2, __fsub_rn(1.0f, g.s2)));
            float dg = __fadd_rn(a1, a2);
            dg = __fsub_rn(dg, grp(a1, -1));
            dg = __fsub_rn(dg, grp(a2, -2));
            dg = __fmaf_rn(__fmul_rn(dp, dl), __fmul_rn(g.sig, __fsub_rn(1.0f, g.sig)), dg);
            if (ok) {
                dacc = __fmaf_rn(dp, __fsub_rn(g.sig, 1.0f), dacc);
                if (live) {
                    dqb[(size_t)t * 2 * D] = dur;
                    dqb[(size_t)t * 2 * D + D] = dg;
                }
            }
        }
    }
    if (live) {
        ds0[(size_t)b * D + d] = ds;
        atomicAdd(ddelta + d, dacc);
    }
}

// step_avx2.c:54-86: one row per sequence, grid-stride over (sequence, group).
__global__ void __launch_bounds__(kCoreThreads)
    step_core_kernel(const float* __restrict__ q, const float* __restrict__ delta,
                     const float* __restrict__ s, float* __restrict__ s_new,
                     float* __restrict__ uo, int B, int D, int DV) {
    const long long total = (long long)B * DV;
    for (long long i0 = (long long)blockIdx.x * kCoreThreads; i0 < total;
         i0 += (long long)gridDim.x * kCoreThreads) {
        const long long i = i0 + threadIdx.x;  // groups never straddle rows: DV % 8 == 0
        const bool live = i < total;
        const int b = live ? (int)(i / DV) : 0, d = live ? (int)(i % DV) : 0;
        const float* qb = q + (size_t)b * 2 * D;
        const Gates g = gates(live ? qb[D + d] : 0.0f);
        if (live) {
            const float u = __fmul_rn(qb[d], __fmul_rn(g.s1, g.s2));
            const float dl = delta[d];
            const float p = __fmaf_rn(dl, g.sig, __fsub_rn(1.0f, dl));
            const size_t o = (size_t)b * D + d;
            uo[o] = u;
            s_new[o] = __fmaf_rn(p, s[o], __fmul_rn(__fsub_rn(1.0f, p), u));
        }
    }
}

// step_avx2.c:24-50: FMA chain on the 8-wide lanes, separate multiply and
// add on the D % 8 tail (as the reference build compiles its scalar loop).
__global__ void dw_step_kernel(const float* __restrict__ x, const float* __restrict__ hist,
                               const float* __restrict__ w, float* __restrict__ acc, int B,
                               int D, int taps) {
    const int k = taps - 1, DV = D & ~7;
    const long long total = (long long)B * D;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int b = (int)(i / D), d = (int)(i % D);
        float a = __fmul_rn(x[i], w[(size_t)(taps - 1) * D + d]);
        for (int j = 0; j < k; ++j) {
            const float hv = hist[((size_t)b * k + j) * D + d];
            const float wv = w[(size_t)(taps - 2 - j) * D + d];
            a = d < DV ? __fmaf_rn(hv, wv, a) : __fadd_rn(a, __fmul_rn(hv, wv));
        }
        acc[i] = a;
    }
}

bool dims_ok(int B, int T, int D) { return B > 0 && T > 0 && D > 0 && B <= 65535; }

}  // namespace
}  // namespace sn

using namespace sn;

extern "C" {

// scan_avx2.c:12-45 (p, nu, s0 -> out, send): the gated scan with a = p,
// u = nu, every channel on the 8-lane FMA rule (the reference build
// contracts its scalar tail to the same form).
void scan_f32(const float* p, const float* nu, const float* s0, float* out, float* send, int B,
              int T, int N) {
    if (!p || !nu || !s0 || !out || !send || !dims_ok(B, T, N)) {
        fail(SN_E_INVAL, "scan_f32: null pointer or bad dimension");
        return;
    }
    if (ensure_init() != SN_OK) return;
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    const size_t big = (size_t)B * T * N * 4, small = (size_t)B * N * 4;
    Arr P, U, S0, O, SE;
    if (stage_in(p, big, 0, &P) || stage_in(nu, big, 1, &U) || stage_in(s0, small, 2, &S0) ||
        stage_out(out, big, 3, &O) || stage_out(send, small, 4, &SE))
        return;
    if (launch_scan_strided((const float*)P.dev, (const float*)U.dev, (const float*)S0.dev, N,
                            (float*)O.dev, (float*)SE.dev, N, B, T, N, 1, nullptr, nullptr,
                            stream(), N) != SN_OK)
        return;
    if (copy_back(O) || copy_back(SE)) return;
    finish(true);
}

// scan_avx2.c:50-95: dp = ds*(s_prev - nu), dnu = ds*(1 - p) (recur_bwd's
// gated form).
void scan_bwd_f32(const float* p, const float* nu, const float* s0, const float* out,
                  const float* dout, float* dp, float* dnu, float* ds0, int B, int T, int N) {
    if (!p || !nu || !s0 || !out || !dout || !dp || !dnu || !ds0 || !dims_ok(B, T, N)) {
        fail(SN_E_INVAL, "scan_bwd_f32: null pointer or bad dimension");
        return;
    }
    if (ensure_init() != SN_OK) return;
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    const size_t big = (size_t)B * T * N * 4, small = (size_t)B * N * 4;
    Arr P, U, S0, O, DO, DP, DN, D0;
    if (stage_in(p, big, 0, &P) || stage_in(nu, big, 1, &U) || stage_in(s0, small, 2, &S0) ||
        stage_in(out, big, 3, &O) || stage_in(dout, big, 4, &DO) ||
        stage_out(dp, big, 5, &DP) || stage_out(dnu, big, 6, &DN) ||
        stage_out(ds0, small, 7, &D0))
        return;
    if (launch_scan_bwd((const float*)P.dev, (const float*)U.dev, (const float*)S0.dev,
                        (const float*)O.dev, (const float*)DO.dev, (float*)DP.dev,
                        (float*)DN.dev, (float*)D0.dev, B, T, N, 1, stream()) != SN_OK)
        return;
    if (copy_back(DP) || copy_back(DN) || copy_back(D0)) return;
    finish(true);
}

void core_fwd_f32(const float* q, const float* delta, const float* s0, float* states, float* uo,
                  float* po, int B, int T, int D) {
    if (!q || !delta || !s0 || !states || !uo || !po || !dims_ok(B, T, D)) {
        fail(SN_E_INVAL, "core_fwd_f32: null pointer or bad dimension");
        return;
    }
    if (ensure_init() != SN_OK) return;
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    const size_t bq = (size_t)B * T * 2 * D * 4, bo = (size_t)B * T * D * 4;
    // with a partial group the untouched channels of host outputs keep the
    // caller's values: stage those outputs in as well as out
    auto out = D % 8 ? stage_inout : stage_out;
    Arr Q, DL, S0, ST, UO, PO;
    if (stage_in(q, bq, 0, &Q) || stage_in(delta, (size_t)D * 4, 1, &DL) ||
        stage_in(s0, (size_t)B * D * 4, 2, &S0) || out(states, bo, 3, &ST) ||
        out(uo, bo, 4, &UO) || out(po, bo, 5, &PO))
        return;
    const int DV = D & ~7;
    if (DV > 0) {
        core_fwd_kernel<<<dim3((DV + kCoreThreads - 1) / kCoreThreads, B), kCoreThreads, 0,
                          stream()>>>((const float*)Q.dev, (const float*)DL.dev,
                                      (const float*)S0.dev, (float*)ST.dev, (float*)UO.dev,
                                      (float*)PO.dev, T, D, DV);
        if (cuda_check(cudaGetLastError(), "core_fwd launch") != SN_OK) return;
    }
    if (copy_back(ST) || copy_back(UO) || copy_back(PO)) return;
    finish(true);
}

void core_bwd_f32(const float* q, const float* delta, const float* s0, const float* states,
                  const float* uo, const float* po, const float* dstate, const float* du_in,
                  float* dq, float* ddelta, float* ds0, int B, int T, int D) {
    if (!q || !delta || !s0 || !states || !uo || !po || !dstate || !du_in || !dq || !ddelta ||
        !ds0 || !dims_ok(B, T, D)) {
        fail(SN_E_INVAL, "core_bwd_f32: null pointer or bad dimension");
        return;
    }
    if (ensure_init() != SN_OK) return;
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    const size_t bq = (size_t)B * T * 2 * D * 4, bo = (size_t)B * T * D * 4;
    Arr Q, DL, S0, ST, UO, PO, DS, DU, DQ, DD, D0;
    if (stage_in(q, bq, 0, &Q) || stage_in(delta, (size_t)D * 4, 1, &DL) ||
        stage_in(s0, (size_t)B * D * 4, 2, &S0) || stage_in(states, bo, 3, &ST) ||
        stage_in(uo, bo, 4, &UO) || stage_in(po, bo, 5, &PO) || stage_in(dstate, bo, 6, &DS) ||
        stage_in(du_in, bo, 7, &DU) || (D % 8 ? stage_inout : stage_out)(dq, bq, 8, &DQ) ||
        stage_inout(ddelta, (size_t)D * 4, 9, &DD) ||
        (D % 8 ? stage_inout : stage_out)(ds0, (size_t)B * D * 4, 10, &D0))
        return;
    const int DV = D & ~7;
    if (DV > 0) {
        core_bwd_kernel<<<dim3((DV + kCoreThreads - 1) / kCoreThreads, B), kCoreThreads, 0,
                          stream()>>>(
            (const float*)Q.dev, (const float*)DL.dev, (const float*)S0.dev,
            (const float*)ST.dev, (const float*)UO.dev, (const float*)PO.dev,
            (const float*)DS.dev, (const float*)DU.dev, (float*)DQ.dev, (float*)DD.dev,
            (float*)D0.dev, T, D, DV);
        if (cuda_check(cudaGetLastError(), "core_bwd launch") != SN_OK) return;
    }
    if (copy_back(DQ) || copy_back(DD) || copy_back(D0)) return;
    finish(true);
}

void step_core_f32(const float* q, const float* delta, const float* s, float* s_new, float* uo,
                   int B, int D) {
    if (!q || !delta || !s || !s_new || !uo || B <= 0 || D <= 0) {
        fail(SN_E_INVAL, "step_core_f32: null pointer or bad dimension");
        return;
    }
    if (ensure_init() != SN_OK) return;
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    const size_t bs = (size_t)B * D * 4;
    auto out = D % 8 ? stage_inout : stage_out;  // keep untouched channels of host outputs
    Arr Q, DL, S, SN_, UO;
    if (stage_in(q, 2 * bs, 0, &Q) || stage_in(delta, (size_t)D * 4, 1, &DL) ||
        stage_in(s, bs, 2, &S) || out(s_new, bs, 3, &SN_) || out(uo, bs, 4, &UO))
        return;
    const int DV = D & ~7;
    if (DV > 0) {
        step_core_kernel<<<grid_blocks((long long)B * DV, kCoreThreads), kCoreThreads, 0,
                           stream()>>>((const float*)Q.dev, (const float*)DL.dev,
                                       (const float*)S.dev, (float*)SN_.dev, (float*)UO.dev, B,
                                       D, DV);
        if (cuda_check(cudaGetLastError(), "step_core launch") != SN_OK) return;
    }
    if (copy_back(SN_) || copy_back(UO)) return;
    finish(true);
}

void dw_step_f32(const float* x, const float* hist, const float* w, float* acc, int B, int D,
                 int taps) {
    if (!x || !w || !acc || B <= 0 || D <= 0 || taps < 1 || (taps > 1 && !hist)) {
        fail(SN_E_INVAL, "dw_step_f32: null pointer or bad dimension");
        return;
    }
    if (ensure_init() != SN_OK) return;
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    const size_t bs = (size_t)B * D * 4;
    Arr X, H, W, A;
    if (stage_in(x, bs, 0, &X) || stage_in(w, (size_t)taps * D * 4, 2, &W) ||
        stage_out(acc, bs, 3, &A))
        return;
    H.dev = nullptr;
    if (taps > 1 && stage_in(hist, bs * (taps - 1), 1, &H)) return;
    dw_step_kernel<<<grid_blocks((long long)B * D), 256, 0, stream()>>>(
        (const float*)X.dev, (const float*)H.dev, (const float*)W.dev, (float*)A.dev, B, D,
        taps);
    if (cuda_check(cudaGetLastError(), "dw_step launch") != SN_OK) return;
    if (copy_back(A)) return;
    finish(true);
}

}  // extern "C"
