// RWKV-7 whole-model decode on sm_100a.
//
// Reference: sunnynet/runtime/rwkv7.c (head_step 143-189, rk_layer 191-320,
// sn_rk_step 349-360, sn_rk_prefill 362-364, sn_rk_dbg 366-374, sn_rk_load
// 415-508) and the numpy oracle RWKV7.step (runtime/rwkv7.py:123-211).
//
// Per layer and step, for B sequences:
//   tmix_prep   xn = LN(x); d = shift0 - xn; six lerps; shift0 <- xn
//   GEMVs       r, k, v, tanh(W1 xw), A1 xa, V1 xv, sigmoid(G1 xg)
//   GEMVs       W2, A2, V2, G2 on the LoRA intermediates
//   mix         w = exp(-sig(.)/sqrt(e)), v-first mix, a = sig(.), kk, k
//   heads       per (sequence, head) CTA: the 64x64 state in place,
//               S <- S*diag(w) - (S kk^)(kk^ a)^T + v k^T, y = S r, then the
//               per-head group norm, the r.k bonus and the g gate
//   GEMV        x += Wo y
//   cmix_prep   xn2 = LN(x); xk = lerp(xn2, shift1); shift1 <- xn2
//   GEMVs       relu(Wk xk)^2, then x += Wv (.)
// then the final LN and the LM head. INT4 matrices run the W4A8 GEMV of
// quant4.cu (bit-identical to the reference's sn_gemv_i4); fp32 matrices the
// fp32 contraction of gemm.cu. The step is captured into a CUDA graph per B.
//
// HBM layout: INT4 codes (out,in/2) + scales (out,in/block) fp32 or fp16;
// fp32 matrices transposed at load to (out,in); state S [seq][L][NH][HS][HS]
// (row i = value dim), token shift [seq][L][2][D].
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <vector>

#include "gemm.cuh"
#include "grid_sync.cuh"
#include "kernels.cuh"
#include "ptx.cuh"
#include "runtime.cuh"
#include "rwkv7.h"
#include "sn_abi.h"
#include "w4a8_rows.cuh"

namespace sn {
namespace {

constexpr int32_t kKRWK = 0x4B57524B;
constexpr float kInvSqrtE = 0.6065306597126334f;  // rwkv7.c:33
constexpr float kEpsGroup = 6.4e-4f;               // rwkv7.c:34

__device__ __forceinline__ float sigm(float x) { return 1.0f / (1.0f + expf(-x)); }

__device__ float block_sum(float v, float* red) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    v = l < nw ? red[l] : 0.0f;
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// LN of one row held in `xr` (two-pass, as rwkv7.c:128-140); returns mean/rstd.
__device__ void row_stats(const float* xr, int n, float eps, float* red, float* mean,
                          float* rstd) {
    float s = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s += xr[i];
    const float m = block_sum(s, red) / (float)n;
    float v = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float d = xr[i] - m;
        v += d * d;
    }
    *mean = m;
    *rstd = 1.0f / sqrtf(block_sum(v, red) / (float)n + eps);
}

// x = LN(embed[tok]) (rwkv7.c:352-353)
__global__ void rk_embed_kernel(int D, const int32_t* __restrict__ tok, int vocab,
                                int* __restrict__ err, const float* __restrict__ embed,
                                const float* __restrict__ w, const float* __restrict__ b,
                                float* __restrict__ x, float eps) {
    __shared__ float red[32];
    pdl_trigger();
    int t = tok[blockIdx.x];
    if (t < 0 || t >= vocab) {  // never read outside the table; report instead
        if (threadIdx.x == 0) atomicExch(err, kErrBadIndex);
        t = 0;
    }
    const float* e = embed + (size_t)t * D;
    float mean, rstd;
    row_stats(e, D, eps, red, &mean, &rstd);
    for (int i = threadIdx.x; i < D; i += blockDim.x)
        x[(size_t)blockIdx.x * D + i] = (e[i] - mean) * rstd * w[i] + b[i];
}

// time-mix prologue (rwkv7.c:213-226); lerps written as 6 (rows,D) planes.
// Rows are T consecutive tokens of each sequence (T = 1 for a decode step).
// The token before row t is row t-1 of the same sequence, whose normalised
// input is recomputed here (the same arithmetic that row computes for
// itself), or the shift state for t = 0. With T = 1 the shift state is
// updated in place; with T > 1 the caller copies the last row's xn into it
// after this kernel (other rows still read the old value here).
__global__ void rk_tmix_prep_kernel(int D, int B, const float* __restrict__ x,
                                    float* __restrict__ shift, long long shift_stride,
                                    const float* __restrict__ w, const float* __restrict__ b,
                                    const float* __restrict__ lerp, float* __restrict__ xn_out,
                                    float* __restrict__ planes, float eps, int T) {
    __shared__ float red[32];
    pdl_trigger();
    pdl_wait();  // no-op unless launched with programmatic serialization
    const int s = blockIdx.x, seq = s / T, t = s - seq * T;
    const float* xr = x + (size_t)s * D;
    float* sh = shift + seq * shift_stride;
    float mean, rstd, pmean = 0.0f, prstd = 0.0f;
    row_stats(xr, D, eps, red, &mean, &rstd);
    if (t > 0) row_stats(xr - D, D, eps, red, &pmean, &prstd);
    const size_t plane = (size_t)B * D;
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
        const float xn = (xr[i] - mean) * rstd * w[i] + b[i];
        const float prev = t > 0 ? (xr[i - D] - pmean) * prstd * w[i] + b[i] : sh[i];
        const float d = prev - xn;
        float* o = planes + (size_t)s * D + i;
#pragma unroll
        for (int j = 0; j < 6; ++j) o[j * plane] = xn + lerp[j * D + i] * d;
        if (T == 1) sh[i] = xn;
        xn_out[(size_t)s * D + i] = xn;
    }
}

// w, v-first mix, a, kk, k (rwkv7.c:232-264); one thread per (seq, channel)
__global__ void rk_mix_kernel(int B, int D, int first, const float* __restrict__ dw,
                              const float* __restrict__ w0, const float* __restrict__ dv,
                              const float* __restrict__ v0, const float* __restrict__ da,
                              const float* __restrict__ a0, const float* __restrict__ kkw,
                              const float* __restrict__ kaw, float* __restrict__ ww,
                              float* __restrict__ v, float* __restrict__ vfirst,
                              float* __restrict__ a, float* __restrict__ k,
                              float* __restrict__ kk) {
    pdl_trigger();
    pdl_wait();  // no-op unless launched with programmatic serialization
    const long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (idx >= (long long)B * D) return;
    const int i = (int)(idx % D);
    ww[idx] = expf(-sigm(dw[idx] + w0[i]) * kInvSqrtE);
    if (first) {
        vfirst[idx] = v[idx];
    } else {
        const float vv = v[idx];
        v[idx] = vv + (vfirst[idx] - vv) * sigm(dv[idx] + v0[i]);
    }
    const float aa = sigm(da[idx] + a0[i]);
    a[idx] = aa;
    const float kv = k[idx];
    kk[idx] = kv * kkw[i];
    k[idx] = kv + kv * (aa - 1.0f) * kaw[i];
}

// rk_mix_kernel with the LoRA second stages folded in, for fp32 w2 / a2 / v2
// (rank Rw, Ra, Rv <= kLoraMax): dw = w2 lo_w, da = a2 lo_a, dv = v2 lo_v
// (first: no dv) per (sequence, channel), each a sequential fmaf over the
// rank, then the mix. CTA = 32 channels x 8 sequences (warp w: sequence
// by*8 + w, lane: channel bx*32 + lane); the 32 channels' weight rows are
// staged transposed in shared memory ([k][33]), the 8 sequences' LoRA
// vectors after them.
constexpr int kLoraMax = 128;
__global__ void __launch_bounds__(256)
    rk_lora_mix_kernel(int B, int D, int first, int Rw, int Ra, int Rv,
                       const float* __restrict__ w2, const float* __restrict__ a2,
                       const float* __restrict__ v2, const float* __restrict__ lo_w,
                       const float* __restrict__ lo_a, const float* __restrict__ lo_v,
                       const float* __restrict__ w0, const float* __restrict__ v0,
                       const float* __restrict__ a0, const float* __restrict__ kkw,
                       const float* __restrict__ kaw, float* __restrict__ ww,
                       float* __restrict__ v, float* __restrict__ vfirst, float* __restrict__ a,
                       float* __restrict__ k, float* __restrict__ kk) {
    extern __shared__ float sm[];
    pdl_trigger();
    pdl_wait();  // no-op unless launched with programmatic serialization
    const int rv = first ? 0 : Rv, R = Rw + Ra + rv;
    float* wt = sm;                 // [R][33]: rows of w2, then a2, then v2
    float* lo = sm + R * 33;        // [8][R]
    const int d0 = blockIdx.x * 32, b0 = blockIdx.y * 8;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // staged with cp.async: every thread's copies are in flight at once (a
    // load-then-store loop would wait a memory round trip per element)
    for (int i = tid; i < 32 * R; i += 256) {
        const int c = i / R, kk_ = i % R, d = d0 + c < D ? d0 + c : 0;
        const float* src = kk_ < Rw        ? w2 + (size_t)d * Rw + kk_
                           : kk_ < Rw + Ra ? a2 + (size_t)d * Ra + (kk_ - Rw)
                                           : v2 + (size_t)d * Rv + (kk_ - Rw - Ra);
        cp_async4(wt + kk_ * 33 + c, src, d0 + c < D ? 4u : 0u);
    }
    for (int i = tid; i < 8 * R; i += 256) {
        const int j = i / R, kk_ = i % R, b = b0 + j < B ? b0 + j : 0;
        const float* src = kk_ < Rw        ? lo_w + (size_t)b * Rw + kk_
                           : kk_ < Rw + Ra ? lo_a + (size_t)b * Ra + (kk_ - Rw)
                                           : lo_v + (size_t)b * Rv + (kk_ - Rw - Ra);
        cp_async4(lo + j * R + kk_, src, b0 + j < B ? 4u : 0u);
    }
    cp_async_wait_all();
    __syncthreads();
    const int b = b0 + warp, i = d0 + lane;
    if (b >= B || i >= D) return;
    const float* lb = lo + warp * R;
    float dw = 0.0f, da = 0.0f, dv = 0.0f;
    for (int q = 0; q < Rw; ++q) dw = fmaf(lb[q], wt[q * 33 + lane], dw);
    for (int q = Rw; q < Rw + Ra; ++q) da = fmaf(lb[q], wt[q * 33 + lane], da);
    for (int q = Rw + Ra; q < R; ++q) dv = fmaf(lb[q], wt[q * 33 + lane], dv);
    const size_t idx = (size_t)b * D + i;
    ww[idx] = expf(-sigm(dw + w0[i]) * kInvSqrtE);
    if (first) {
        vfirst[idx] = v[idx];
    } else {
        const float vv = v[idx];
        v[idx] = vv + (vfirst[idx] - vv) * sigm(dv + v0[i]);
    }
    const float aa = sigm(da + a0[i]);
    a[idx] = aa;
    const float kv = k[idx];
    kk[idx] = kv * kkw[i];
    k[idx] = kv + kv * (aa - 1.0f) * kaw[i];
}

// One CTA (8 warps) per (sequence, head): the matrix-state update of
// rwkv7.c:143-189 followed by group norm + bonus + gate (rwkv7.c:268-289).
// A warp owns state rows i = warp, warp+8, ...; a lane owns VPL columns.
// One CTA per (sequence, head) walks that sequence's T consecutive rows in
// order (T = 1 for a decode step, the prompt chunk in a prefill); heads up to
// 128 wide keep the state in registers across the rows.
// CG: the step's vectors are read through L2 (ld.global.cg), for a caller in
// which other CTAs of the same launch wrote them (the fused decode step).
struct RkNoPre {
    __device__ bool operator()() const { return true; }
};

// NOG: y is left ungated (the caller multiplies by g, the same single
// rounding); pre() runs after the state rows are requested and before the
// head's vectors are read (the fused step computes them there), and returns
// false, the same in every thread, to leave the state untouched.
template <int VPL, bool CG, bool NOG = false, class Pre = RkNoPre>
__device__ __forceinline__ void rk_heads_body(int h, int b, int NH, int L, int layer, int D,
                                              float* __restrict__ S, const float* ww,
                                              const float* k, const float* v, const float* a,
                                              const float* kk, const float* r, const float* g,
                                              const float* __restrict__ rk,
                                              const float* __restrict__ lnw,
                                              const float* __restrict__ lnb, float* y, int T,
                                              float* kn, float* yv, float* red, Pre pre = Pre()) {
    auto ld = [](const float* p) { return CG ? __ldcg(p) : *p; };
    constexpr int HS = VPL * 32;
    // warp w owns state rows w, w+8, ...; for heads up to 128 wide all of
    // them are loaded at once, before anything else, so the state costs one
    // memory round trip per warp instead of one per row
    constexpr int RPW = HS / 8;
    constexpr bool PRE = VPL <= 4;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* Sh = S + (((size_t)b * L + layer) * NH + h) * HS * HS;
    float spre[PRE ? RPW : 1][VPL];
    if (PRE) {
#pragma unroll
        for (int q = 0; q < (PRE ? RPW : 1); ++q)
#pragma unroll
            for (int t = 0; t < VPL; ++t) spre[q][t] = Sh[(size_t)(warp + 8 * q) * HS + lane + 32 * t];
    }
    if (!pre()) return;
    for (int step = 0; step < T; ++step) {
        const size_t o = ((size_t)b * T + step) * D + (size_t)h * HS;
        // kk normalised with floor 1e-12 (rwkv7.c:162-165)
        float ss = 0.0f;
        for (int j = threadIdx.x; j < HS; j += blockDim.x) ss += ld(&kk[o + j]) * ld(&kk[o + j]);
        float nrm = sqrtf(block_sum(ss, red));
        if (!(nrm > 1e-12f)) nrm = 1e-12f;
        const float inv = 1.0f / nrm;
        for (int j = threadIdx.x; j < HS; j += blockDim.x) kn[j] = ld(&kk[o + j]) * inv;
        __syncthreads();
        float wj[VPL], kj[VPL], rj[VPL], knj[VPL], kaj[VPL];
#pragma unroll
        for (int t = 0; t < VPL; ++t) {
            const int j = lane + 32 * t;
            wj[t] = ld(&ww[o + j]);
            kj[t] = ld(&k[o + j]);
            rj[t] = ld(&r[o + j]);
            knj[t] = kn[j];
            kaj[t] = __fmul_rn(kn[j], ld(&a[o + j]));
        }
#pragma unroll(PRE ? RPW : 1)
        for (int q = 0; q < RPW; ++q) {
            const int i = warp + 8 * q;
            float* row = Sh + (size_t)i * HS;
            float sv[VPL];
            float p = 0.0f;
#pragma unroll
            for (int t = 0; t < VPL; ++t) {
                sv[t] = PRE ? spre[PRE ? q : 0][t] : row[lane + 32 * t];
                p = fmaf(sv[t], knj[t], p);
            }
            for (int off = 16; off; off >>= 1) p += __shfl_xor_sync(0xffffffffu, p, off);
            const float vi = ld(&v[o + i]);
            float yacc = 0.0f;
#pragma unroll
            for (int t = 0; t < VPL; ++t) {
                const float ns =
                    __fmaf_rn(sv[t], wj[t], __fsub_rn(__fmul_rn(vi, kj[t]), __fmul_rn(p, kaj[t])));
                if (PRE)
                    spre[PRE ? q : 0][t] = ns;
                else
                    row[lane + 32 * t] = ns;
                yacc = fmaf(ns, rj[t], yacc);
            }
            for (int off = 16; off; off >>= 1) yacc += __shfl_xor_sync(0xffffffffu, yacc, off);
            if (lane == 0) yv[i] = yacc;
        }
        __syncthreads();
        // group norm over the head, r.k bonus, gate
        float m = 0.0f;
        for (int j = threadIdx.x; j < HS; j += blockDim.x) m += yv[j];
        const float mean = block_sum(m, red) / (float)HS;
        float var = 0.0f, dot = 0.0f;
        for (int j = threadIdx.x; j < HS; j += blockDim.x) {
            const float t = yv[j] - mean;
            var += t * t;
            dot += ld(&r[o + j]) * ld(&k[o + j]) * rk[h * HS + j];
        }
        const float rstd = 1.0f / sqrtf(block_sum(var, red) / (float)HS + kEpsGroup);
        dot = block_sum(dot, red);
        for (int j = threadIdx.x; j < HS; j += blockDim.x) {
            const float nv = (yv[j] - mean) * rstd * lnw[h * HS + j] + lnb[h * HS + j];
            if (NOG)
                y[o + j] = nv + dot * ld(&v[o + j]);
            else
                y[o + j] = (nv + dot * ld(&v[o + j])) * ld(&g[o + j]);
        }
        __syncthreads();  // kn and yv are rewritten by the next row
    }
    if (PRE) {
#pragma unroll
        for (int q = 0; q < (PRE ? RPW : 1); ++q)
#pragma unroll
            for (int t = 0; t < VPL; ++t) Sh[(size_t)(warp + 8 * q) * HS + lane + 32 * t] = spre[q][t];
    }
}


template <int VPL>
__global__ void __launch_bounds__(256)
    rk_heads_kernel(int NH, int L, int layer, int D, float* __restrict__ S,
                    const float* __restrict__ ww, const float* __restrict__ k,
                    const float* __restrict__ v, const float* __restrict__ a,
                    const float* __restrict__ kk, const float* __restrict__ r,
                    const float* __restrict__ g, const float* __restrict__ rk,
                    const float* __restrict__ lnw, const float* __restrict__ lnb,
                    float* __restrict__ y, int T) {
    __shared__ float kn[VPL * 32], yv[VPL * 32], red[32];
    pdl_trigger();
    pdl_wait();  // no-op unless launched with programmatic serialization
    rk_heads_body<VPL, false>((int)blockIdx.x % NH, (int)blockIdx.x / NH, NH, L, layer, D, S, ww,
                              k, v, a, kk, r, g, rk, lnw, lnb, y, T, kn, yv, red);
}

// channel-mix prologue (rwkv7.c:295-297); rows and the shift state as in
// rk_tmix_prep_kernel (xn2_out: every row's normalised input, for the
// caller's copy of the last row into the shift state when T > 1).
__global__ void rk_cmix_prep_kernel(int D, const float* __restrict__ x, float* __restrict__ shift,
                                    long long shift_stride, const float* __restrict__ w,
                                    const float* __restrict__ b, const float* __restrict__ lerp,
                                    float* __restrict__ xk, float eps, int T,
                                    float* __restrict__ xn2_out) {
    __shared__ float red[32];
    pdl_trigger();
    pdl_wait();  // no-op unless launched with programmatic serialization
    const int s = blockIdx.x, seq = s / T, t = s - seq * T;
    const float* xr = x + (size_t)s * D;
    float* sh = shift + seq * shift_stride + D;
    float mean, rstd, pmean = 0.0f, prstd = 0.0f;
    row_stats(xr, D, eps, red, &mean, &rstd);
    if (t > 0) row_stats(xr - D, D, eps, red, &pmean, &prstd);
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
        const float xn2 = (xr[i] - mean) * rstd * w[i] + b[i];
        const float prev = t > 0 ? (xr[i - D] - pmean) * prstd * w[i] + b[i] : sh[i];
        xk[(size_t)s * D + i] = xn2 + lerp[i] * (prev - xn2);
        if (T == 1) sh[i] = xn2;
        if (xn2_out) xn2_out[(size_t)s * D + i] = xn2;
    }
}

// y = LN(x) per row (final norm); input rows ldx floats apart
__global__ void rk_ln_kernel(int D, const float* __restrict__ x, const float* __restrict__ w,
                             const float* __restrict__ b, float* __restrict__ y, float eps,
                             long long ldx) {
    __shared__ float red[32];
    pdl_trigger();
    pdl_wait();  // no-op unless launched with programmatic serialization
    const float* xr = x + (size_t)blockIdx.x * ldx;
    float mean, rstd;
    row_stats(xr, D, eps, red, &mean, &rstd);
    for (int i = threadIdx.x; i < D; i += blockDim.x)
        y[(size_t)blockIdx.x * D + i] = (xr[i] - mean) * rstd * w[i] + b[i];
}


__global__ void rk_transpose_kernel(const float* __restrict__ src, float* __restrict__ dst, int in,
                                    int out) {
    __shared__ float t[32][33];
    const int bx = blockIdx.x * 32, by = blockIdx.y * 32;
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int i = by + j, o = bx + threadIdx.x;
        if (i < in && o < out) t[j][threadIdx.x] = src[(size_t)i * out + o];
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int o = bx + j, i = by + threadIdx.x;
        if (i < in && o < out) dst[(size_t)o * in + i] = t[threadIdx.x][j];
    }
}

}  // namespace

struct RkMat {
    int q4 = 0, in = 0, out = 0, block = 0;
    bool fp16 = false;
    float* w = nullptr;  // fp32 (out,in)
    uint8_t* q = nullptr;
    void* scale = nullptr;
};

struct RkLayer {
    float *ln1w, *ln1b, *ln2w, *ln2b, *lerp;
    RkMat rw, kw, vw, ow, w1, w2, a1, a2, v1, v2, g1, g2, cmk, cmv;
    float *w0, *a0, *v0, *kkw, *kaw, *rkw, *lnxw, *lnxb, *cmk_lerp;
    int Rw, Ra, Rv, Rg;
};

// Row buffers of one pass over the layers: a decode step's B rows, or a
// prefill chunk's B sequences x T tokens.
struct RkBufs {
    int rows = 0;
    int32_t* tok = nullptr;
    float *x = nullptr, *xn = nullptr, *planes = nullptr, *r = nullptr, *k = nullptr,
          *v = nullptr, *a = nullptr, *g = nullptr, *kk = nullptr, *ww = nullptr, *y = nullptr,
          *xk2 = nullptr, *lo_w = nullptr, *lo_a = nullptr, *lo_v = nullptr, *lo_g = nullptr,
          *dw = nullptr, *da = nullptr, *dv = nullptr, *ck = nullptr, *vfirst = nullptr,
          *xf = nullptr, *logits = nullptr;
};

// The fused B = 1 decode step's tables (its kernel is below).
struct RkFMat {
    const uint8_t* q;
    const void* scale;
    int in, out;
};

struct RkFLayer {
    const float *ln1w, *ln1b, *ln2w, *ln2b, *lerp, *cmk_lerp;
    RkFMat rw, kw, vw, w1, a1, g1, v1, g2, ow, cmk, cmv;
    const float *w2, *a2, *v2;  // fp32 LoRA second stages (D, rank)
    int Rw, Ra, Rv;
    const float *w0, *a0, *v0, *kkw, *kaw, *rkw, *lnxw, *lnxb;
};

struct RkFArgs {
    const RkFLayer* layers;
    int L, D, NH, F, block, with_head;
    float eps;
    const int32_t* tok;
    int vocab;
    int* err;
    const float *embed, *en_w, *en_b, *on_w, *on_b;
    RkFMat head;
    float *S, *shift;  // sequence 0's state and shift rows
    float *x, *r, *k, *v, *a, *g, *kk, *ww, *y, *ck, *lo_w, *lo_a, *lo_v, *lo_g, *vfirst;
    float *logits, *xn, *xn2;
    unsigned* bar;
    int part0[8], part1[8];  // phase A: first CTA of each problem (layer 0: 6, later: 7), then the grid size
    size_t qbytes;           // W4A8 quantisation area at the start of shared memory
};


struct RwkvModel {
    int vocab = 0, D = 0, HS = 0, NH = 0, F = 0, L = 0, nseq = 0, q4 = 0, group = 64;
    float eps = 1e-5f;
    std::vector<RkLayer> ly;
    float *en_w = nullptr, *en_b = nullptr, *on_w = nullptr, *on_b = nullptr, *embed = nullptr;
    RkMat head;
    float *S = nullptr, *shift = nullptr;
    int32_t *tok = nullptr, *next = nullptr;
    float *x = nullptr, *xn = nullptr, *planes = nullptr, *r = nullptr, *k = nullptr, *v = nullptr;
    float *a = nullptr, *g = nullptr, *kk = nullptr, *ww = nullptr, *y = nullptr, *xk2 = nullptr;
    float *lo_w = nullptr, *lo_a = nullptr, *lo_v = nullptr, *lo_g = nullptr;
    float *dw = nullptr, *da = nullptr, *dv = nullptr, *ck = nullptr, *vfirst = nullptr;
    float *logits = nullptr, *xf = nullptr;
    float2* apart = nullptr;  // argmax partials (B x kArgChunks)
    RkBufs pre;                // prefill workspace (allocated on first use)
    std::vector<void*> pre_allocs;
    int rmax = 0;              // widest LoRA rank
    std::vector<void*> allocs;
    std::map<std::pair<int, int>, cudaGraphExec_t> graphs;
    std::map<std::pair<int, int>, ProfGraph> pgraphs;  // instrumented (profile mode 2)
    cudaStream_t cap = nullptr;
    bool ready = false;
    // fused B = 1 decode step: -1 not tried yet, 0 not applicable, 1 set up
    int fused = -1, fctas = 0;
    RkFLayer* flayers = nullptr;
    unsigned* fbar = nullptr;
    float* xn2 = nullptr;

    ~RwkvModel() {
        for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
        if (cap) cudaStreamDestroy(cap);
        for (void* p : allocs) cudaFree(p);
        for (void* p : pre_allocs) cudaFree(p);
    }
    template <class T>
    T* dalloc(size_t n) {
        void* p = nullptr;
        if (cudaMalloc(&p, (n ? n : 1) * sizeof(T)) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        allocs.push_back(p);
        return (T*)p;
    }
};

namespace {

// Parses the tagged tensor stream of a KRWK file held in host memory.
struct RkParser {
    RwkvModel* m;
    const unsigned char* p;
    const unsigned char* end;
    int version;
    bool ok = true;
    float* tmp = nullptr;
    size_t tmp_n = 0;

    const unsigned char* take(size_t n) {
        if (!ok || (size_t)(end - p) < n) {
            ok = false;
            return nullptr;
        }
        const unsigned char* r = p;
        p += n;
        return r;
    }
    int i32() {
        const unsigned char* q = take(4);
        int v = 0;
        if (q) memcpy(&v, q, 4);
        return v;
    }
    template <class T>
    T* upload(const void* src, size_t n) {
        T* d = m->dalloc<T>(n);
        if (!d || cudaMemcpy(d, src, n * sizeof(T), cudaMemcpyHostToDevice) != cudaSuccess) {
            ok = false;
            return nullptr;
        }
        return d;
    }
    float* vec(size_t n) {  // rwkv7.c:404-409
        if (i32() != 0) ok = false;
        const unsigned char* q = take(n * 4);
        return q ? upload<float>(q, n) : nullptr;
    }
    void mat(RkMat* M, int in, int out) {  // rwkv7.c:380-402 (+ tag 2)
        const int tag = i32();
        M->in = in;
        M->out = out;
        if (!ok) return;
        if (tag == 0) {
            const size_t n = (size_t)in * out;
            const unsigned char* q = take(n * 4);
            if (!q) return;
            if (tmp_n < n) {
                if (tmp) cudaFree(tmp);
                tmp = nullptr;
                if (cudaMalloc(&tmp, n * 4) != cudaSuccess) {
                    cudaGetLastError();
                    ok = false;
                    return;
                }
                tmp_n = n;
            }
            cudaMemcpy(tmp, q, n * 4, cudaMemcpyHostToDevice);
            M->w = m->dalloc<float>(n);
            if (!M->w) {
                ok = false;
                return;
            }
            dim3 grid((out + 31) / 32, (in + 31) / 32);
            rk_transpose_kernel<<<grid, dim3(32, 8)>>>(tmp, M->w, in, out);
        } else if (tag == 1 || (tag == 2 && version == 4)) {
            const int blk = tag == 1 ? 64 : m->group;
            if (blk <= 0 || in % blk) {
                ok = false;
                return;
            }
            const size_t qb = (size_t)out * (in / 2), ns = (size_t)out * (in / blk);
            const unsigned char* q = take(qb);
            const unsigned char* s = take(ns * (tag == 1 ? 4 : 2));
            if (!q || !s) return;
            M->q4 = 1;
            M->block = blk;
            M->fp16 = tag == 2;
            M->q = upload<uint8_t>(q, qb);
            M->scale = tag == 1 ? (void*)upload<float>(s, ns) : (void*)upload<__half>(s, ns);
        } else {
            ok = false;
        }
    }
};

// Activation workspace of the tensor-core W4A8 path for contractions of
// `rows` rows (allocates: call outside any stream capture).
int reserve_tc(RwkvModel* m, int rows) {
    auto reserve = [&](const RkMat& M) -> int {
        if (!M.q4 || !w4a8_tc_ok(rows, M.in, M.out, M.block, M.q)) return SN_OK;
        return w4a8_tc_reserve(rows, M.in, M.block);
    };
    for (const RkLayer& y : m->ly)
        for (const RkMat* M : {&y.rw, &y.kw, &y.vw, &y.ow, &y.w1, &y.w2, &y.a1, &y.a2, &y.v1,
                               &y.v2, &y.g1, &y.g2, &y.cmk, &y.cmv})
            SN_TRY(reserve(*M));
    SN_TRY(reserve(m->head));
    if (!m->ly.empty()) {  // the grouped first-stage projections: six input planes
        const RkMat& r0 = m->ly[0].rw;
        if (r0.q4 && w4a8_tc_ok(rows, r0.in, r0.out, r0.block, r0.q))
            SN_TRY(w4a8_tc_reserve(rows, r0.in, r0.block, 6));
    }
    return SN_OK;
}

// The decode step's row buffers (nseq rows).
RkBufs step_bufs(RwkvModel* m) {
    RkBufs w;
    w.rows = m->nseq;
    w.tok = m->tok; w.x = m->x; w.xn = m->xn; w.planes = m->planes;
    w.r = m->r; w.k = m->k; w.v = m->v; w.a = m->a; w.g = m->g; w.kk = m->kk; w.ww = m->ww;
    w.y = m->y; w.xk2 = m->xk2; w.lo_w = m->lo_w; w.lo_a = m->lo_a; w.lo_v = m->lo_v;
    w.lo_g = m->lo_g; w.dw = m->dw; w.da = m->da; w.dv = m->dv; w.ck = m->ck;
    w.vfirst = m->vfirst; w.xf = m->xf; w.logits = m->logits;
    return w;
}

// Prefill workspace of at least `rows` rows (prompt chunks of all sequences
// at once); the final norm and the head only ever see nseq rows.
int ensure_pre(RwkvModel* m, int rows) {
    if (m->pre.rows >= rows) return SN_OK;
    cudaStreamSynchronize(stream());
    for (void* p : m->pre_allocs) cudaFree(p);
    m->pre_allocs.clear();
    m->pre = RkBufs{};
    bool ok = true;
    auto al = [&](size_t n) -> float* {
        void* p = nullptr;
        if (cudaMalloc(&p, (n ? n : 1) * sizeof(float)) != cudaSuccess) {
            cudaGetLastError();
            ok = false;
            return nullptr;
        }
        m->pre_allocs.push_back(p);
        return (float*)p;
    };
    const size_t R = (size_t)rows, D = m->D, S = m->nseq;
    RkBufs w;
    w.rows = rows;
    w.tok = (int32_t*)al(R);
    w.x = al(R * D); w.xn = al(R * D); w.planes = al(6 * R * D);
    w.r = al(R * D); w.k = al(R * D); w.v = al(R * D); w.a = al(R * D); w.g = al(R * D);
    w.kk = al(R * D); w.ww = al(R * D); w.y = al(R * D); w.xk2 = al(R * D);
    w.lo_w = al(R * m->rmax); w.lo_a = al(R * m->rmax); w.lo_v = al(R * m->rmax);
    w.lo_g = al(R * m->rmax); w.dw = al(R * D); w.da = al(R * D); w.dv = al(R * D);
    w.ck = al(R * m->F); w.vfirst = al(R * D);
    w.xf = al(S * D); w.logits = al(S * m->vocab);
    if (!ok) return fail(SN_E_NOMEM, "rwkv7 prefill workspace of %d rows", rows);
    SN_TRY(reserve_tc(m, rows));
    m->pre = w;
    return SN_OK;
}

int load_rwkv(RwkvModel* m, const char* path, int nseq) {
    FILE* f = fopen(path, "rb");
    if (!f) return fail(SN_E_IO, "cannot open %s", path);
    fseek(f, 0, SEEK_END);
    const long n = ftell(f);
    fseek(f, 0, SEEK_SET);
    if (n < 48) {
        fclose(f);
        return fail(SN_E_FORMAT, "%s: truncated", path);
    }
    std::vector<unsigned char> buf((size_t)n);
    const size_t got = fread(buf.data(), 1, (size_t)n, f);
    fclose(f);
    if (got != (size_t)n) return fail(SN_E_IO, "%s: short read", path);
    int32_t h[10];
    memcpy(h, buf.data(), 40);
    if (h[0] != kKRWK || (h[1] != 3 && h[1] != 4))
        return fail(SN_E_FORMAT, "%s: bad magic/version", path);
    SN_TRY(ensure_init());
    RkParser P{m, buf.data() + 40, buf.data() + buf.size(), h[1]};
    m->L = h[2]; m->D = h[3]; m->HS = h[4]; m->NH = h[5]; m->F = h[6]; m->vocab = h[8];
    m->q4 = h[9];
    m->nseq = nseq;
    const unsigned char* pe = P.take(4);
    if (pe) memcpy(&m->eps, pe, 4);
    if (h[1] == 4) m->group = P.i32();
    const int L = m->L, D = m->D;
    if (!P.ok || L <= 0 || D <= 0 || m->vocab <= 0 || m->F <= 0 || m->NH * m->HS != D ||
        !(m->HS == 32 || m->HS == 64 || m->HS == 128 || m->HS == 256))
        return fail(SN_E_FORMAT, "%s: unsupported dims", path);
    m->ly.resize(L);
    int rmax = 0;
    for (int l = 0; l < L; ++l) {
        RkLayer& A = m->ly[l];
        A.Rw = P.i32(); A.Ra = P.i32(); A.Rv = P.i32(); A.Rg = P.i32();
        rmax = std::max(std::max(rmax, std::max(A.Rw, A.Ra)), std::max(A.Rv, A.Rg));
    }
    m->rmax = rmax;
    for (int l = 0; l < L && P.ok; ++l) {
        RkLayer& A = m->ly[l];
        A.ln1w = P.vec(D); A.ln1b = P.vec(D); A.ln2w = P.vec(D); A.ln2b = P.vec(D);
        A.lerp = P.vec((size_t)6 * D);
        P.mat(&A.rw, D, D); P.mat(&A.kw, D, D); P.mat(&A.vw, D, D); P.mat(&A.ow, D, D);
        P.mat(&A.w1, D, A.Rw); P.mat(&A.w2, A.Rw, D);
        P.mat(&A.a1, D, A.Ra); P.mat(&A.a2, A.Ra, D);
        P.mat(&A.v1, D, A.Rv); P.mat(&A.v2, A.Rv, D);
        P.mat(&A.g1, D, A.Rg); P.mat(&A.g2, A.Rg, D);
        A.w0 = P.vec(D); A.a0 = P.vec(D); A.v0 = P.vec(D);
        A.kkw = P.vec(D); A.kaw = P.vec(D); A.rkw = P.vec(D);
        A.lnxw = P.vec(D); A.lnxb = P.vec(D);
        P.mat(&A.cmk, D, m->F); P.mat(&A.cmv, m->F, D);
        A.cmk_lerp = P.vec(D);
    }
    if (P.ok) {
        m->en_w = P.vec(D); m->en_b = P.vec(D); m->on_w = P.vec(D); m->on_b = P.vec(D);
        m->embed = P.vec((size_t)m->vocab * D);
        P.mat(&m->head, D, m->vocab);
    }
    if (P.tmp) cudaFree(P.tmp);
    if (!P.ok) return fail(SN_E_FORMAT, "%s: malformed tensor stream", path);
    const size_t B = (size_t)nseq;
    m->S = m->dalloc<float>(B * L * m->NH * m->HS * m->HS);
    m->shift = m->dalloc<float>(B * L * 2 * D);
    m->tok = m->dalloc<int32_t>(B);
    m->next = m->dalloc<int32_t>(B);
    m->x = m->dalloc<float>(B * D); m->xn = m->dalloc<float>(B * D);
    m->planes = m->dalloc<float>(6 * B * D);
    m->r = m->dalloc<float>(B * D); m->k = m->dalloc<float>(B * D); m->v = m->dalloc<float>(B * D);
    m->a = m->dalloc<float>(B * D); m->g = m->dalloc<float>(B * D); m->kk = m->dalloc<float>(B * D);
    m->ww = m->dalloc<float>(B * D); m->y = m->dalloc<float>(B * D); m->xk2 = m->dalloc<float>(B * D);
    m->lo_w = m->dalloc<float>(B * rmax); m->lo_a = m->dalloc<float>(B * rmax);
    m->lo_v = m->dalloc<float>(B * rmax); m->lo_g = m->dalloc<float>(B * rmax);
    m->dw = m->dalloc<float>(B * D); m->da = m->dalloc<float>(B * D); m->dv = m->dalloc<float>(B * D);
    m->ck = m->dalloc<float>(B * m->F); m->vfirst = m->dalloc<float>(B * D);
    m->xf = m->dalloc<float>(B * D);
    m->logits = m->dalloc<float>(B * m->vocab);
    m->apart = m->dalloc<float2>(B * kArgChunks);
    if (!m->logits || !m->xf || !m->apart) return fail(SN_E_NOMEM, "device allocation failed");
    cudaMemset(m->S, 0, B * L * m->NH * m->HS * m->HS * 4);
    cudaMemset(m->shift, 0, B * L * 2 * D * 4);
    SN_TRY(cuda_check(cudaStreamCreateWithFlags(&m->cap, cudaStreamNonBlocking), "stream"));
    SN_TRY(reserve_tc(m, nseq));  // before any capture
    SN_TRY(cuda_check(cudaDeviceSynchronize(), "rwkv load"));
    m->ready = true;
    return SN_OK;
}

// y (B,out) [epi]= M x (B,in)
// Launched with programmatic serialization: inside the step every contraction
// follows another kernel of the same stream.
int mat_mul(const RkMat& M, float* y, const float* x, int B, int epi, cudaStream_t st) {
    ProfScope ps(M.q4 ? "w4a8_gemv" : "gemm_f32", st);
    if (M.q4) {
        static const int map[] = {kW4Store, kW4Add, kW4Relu2, kW4Tanh, kW4Sigmoid};
        return launch_w4a8(y, x, M.q, M.scale, B, M.in, M.out, M.block, M.fp16, st, map[epi],
                           true);
    }
    GemmArgs g;
    g.M = B; g.N = M.out; g.K = M.in;
    g.A = x; g.lda = M.in;
    g.W = M.w; g.ldw = M.in;
    g.C = y; g.ldc = M.out;
    static const int emap[] = {kEpiNone, kEpiAdd, kEpiRelu2, kEpiTanh, kEpiSigmoid};
    g.epi = emap[epi];
    return launch_gemm(g, kWF32, st, nullptr, true);
}

enum { E_STORE = 0, E_ADD = 1, E_RELU2 = 2, E_TANH = 3, E_SIG = 4 };

// ------------------------------------------------- fused decode step (B = 1)
// One sequence's decode step in one cooperative launch (one CTA of 256
// threads per SM) instead of ~90 dependent launches of small kernels. Each
// layer is five phases separated by grid barriers (grid_sync.cuh):
//   A  every CTA: x (the embedding, or the residual stream through L2),
//      LN1 and the time-mix lerp of its problem's plane; its share of the
//      rows of one first-stage projection (r, k, v, w1, a1, g1, v1: the CTAs
//      are partitioned over the problems in proportion to their rows)
//   BC CTA h < NH, for head h's 64 channels: the LoRA second stages and the
//      mix (the w, a and v sums on three thread groups, each the same
//      sequential fmaf over its rank as rk_lora_mix_kernel; the rows staged
//      by cp.async during A), then the head's matrix-state step
//      (rk_heads_body, output left ungated); the other CTAs meanwhile take
//      the g2 rows, and the last one writes A's normalised input into the
//      time-mix shift state (every CTA read the old one in A)
//   D  ow rows over every warp (x += Wo (y g), the gate applied as the rows'
//      input is staged: the heads kernel's one rounding of the product)
//   E  every CTA: LN2 and the channel-mix lerp; its share of the cmk rows
//   F  cmv rows (x += Wv relu(.)^2); CTA 0 updates the channel-mix shift
// then the final LN and the head rows over every warp. Every per-element
// formula, reduction partition (256-thread CTAs) and W4A8 row is the
// multi-kernel path's, so the two produce identical results. Vectors other
// CTAs wrote in this launch are read through L2 (ld.global.cg). Each phase's
// input row is staged after its first weight rows are requested.
constexpr int kRkFusedThreads = 256;

// dst[0, n) = src[0, n) (times gate[0, n) when given, one rounding) through
// L2: another CTA wrote it in this launch. A thread's 16-byte loads are all
// issued before its stores. src, gate and dst are 16-byte aligned.
__device__ __forceinline__ const float* rk_stage(float* dst, const float* src, int n,
                                                 const float* gate = nullptr) {
    const int n4 = n >> 2, nt = blockDim.x;
    const float4* s4 = reinterpret_cast<const float4*>(src);
    const float4* g4 = reinterpret_cast<const float4*>(gate);
    float4* d4 = reinterpret_cast<float4*>(dst);
    for (int i0 = threadIdx.x; i0 < n4; i0 += 4 * nt) {
        float4 t[4], u[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int i = i0 + k * nt;
            if (i < n4) {
                t[k] = __ldcg(s4 + i);
                if (gate) u[k] = __ldcg(g4 + i);
            }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int i = i0 + k * nt;
            if (i < n4) {
                if (gate) {
                    t[k].x = __fmul_rn(t[k].x, u[k].x);
                    t[k].y = __fmul_rn(t[k].y, u[k].y);
                    t[k].z = __fmul_rn(t[k].z, u[k].z);
                    t[k].w = __fmul_rn(t[k].w, u[k].w);
                }
                d4[i] = t[k];
            }
        }
    }
    for (int i = 4 * n4 + threadIdx.x; i < n; i += nt)
        dst[i] = gate ? __fmul_rn(__ldcg(src + i), __ldcg(gate + i)) : __ldcg(src + i);
    __syncthreads();
    return dst;
}

// Rows gw, gw + nw, ... of one W4A8 contraction of a single activation row;
// pro() stages the row once the first weight rows are in flight.
template <bool FP16S, int NCH, class Pro>
__device__ __forceinline__ void rk_rows(const RkFMat& M, float* Y, int epi, int block, int gw,
                                        int nw, unsigned char* sm, Pro pro) {
    w4a8_rows_p<FP16S, NCH, 1>(Y, M.q, M.scale, 1, 0, M.in, M.out, block, epi, gw, nw, sm, pro);
    __syncthreads();  // the quantisation area is reused by the next contraction
}

template <bool FP16S, int NCHD, int NCHF>
__global__ void __launch_bounds__(kRkFusedThreads, 1) rk_fused_kernel(const __grid_constant__ RkFArgs a) {
    extern __shared__ __align__(16) unsigned char rk_sm[];
    unsigned char* sm = rk_sm;
    __shared__ float red[32], kn[64], yv[64];
    __shared__ float dlo[3][64];  // the head's LoRA second-stage sums (w, a, v)
    const int cta = blockIdx.x, nct = gridDim.x, tid = threadIdx.x, warp = tid >> 5;
    const int D = a.D, gw = cta * (kRkFusedThreads / 32) + warp, nw = nct * (kRkFusedThreads / 32);
    float* xr = reinterpret_cast<float*>(sm + a.qbytes);  // [max(D, F)]: the phase's input row
    float* mix = xr + (a.F > D ? a.F : D);                // [D]: a lerped plane
    float* lov = mix + D;                                 // LoRA vectors (Rw + Ra + Rv, rg)
    float* lrows = lov + 3 * kLoraMax + D;                // [64][Rw + Ra + Rv + 4]: BC rows
    float* cst = lrows + 64 * (3 * kLoraMax + 4);         // [4][D]: A's or E's constants
    // the layer tables (weight and vector addresses), copied once: every phase
    // starts by reading them, and from shared memory that costs no round trip
    RkFLayer* ltab = reinterpret_cast<RkFLayer*>(cst + 4 * D);
    __shared__ __align__(16) float hc[5][64];             // the head's w0, a0, v0, kkw, kaw
    unsigned nbar = 0;
    {
        static_assert(sizeof(RkFLayer) % 8 == 0, "layer table rows are copied in 8-byte words");
        const int nwd = a.L * (int)(sizeof(RkFLayer) / 8);
        const unsigned long long* src = reinterpret_cast<const unsigned long long*>(a.layers);
        unsigned long long* dst = reinterpret_cast<unsigned long long*>(ltab);
        for (int i = tid; i < nwd; i += kRkFusedThreads) dst[i] = src[i];
    }
    // the embedding row, LN'd (every CTA; CTA 0 also stores the residual stream)
    {
        int t = a.tok[0];
        if (t < 0 || t >= a.vocab) {  // never read outside the table; report instead
            if (tid == 0 && cta == 0) atomicExch(a.err, kErrBadIndex);
            t = 0;
        }
        const float* e = a.embed + (size_t)t * D;
        float mean, rstd;
        row_stats(e, D, a.eps, red, &mean, &rstd);
        for (int i = tid; i < D; i += kRkFusedThreads) {
            const float xv = (e[i] - mean) * rstd * a.en_w[i] + a.en_b[i];
            xr[i] = xv;
            if (cta == 0) a.x[i] = xv;
        }
        __syncthreads();
    }
    // A CTA arrives at the grid barrier that opens a phase as soon as its
    // part of the previous one is written, then requests the phase's weight
    // rows (rk_rows calls its prologue, which waits at the barrier, once they
    // are in flight) and copies the per-channel constants it needs to shared
    // memory: after the barrier, only the vectors other CTAs just wrote cost
    // a round trip. When a barrier gives up (an error is recorded), the phase
    // under way finishes its in-bounds arithmetic on whatever it reads,
    // writes no recurrent state, and the kernel returns.
    bool ok = true;
    auto arrive = [&] { grid_arrive(a.bar); };
    auto sync = [&] { ok = ok && grid_wait(a.bar, nbar++, a.err); };
    auto consts = [&](const float* c0, const float* c1, const float* c2, const float* c3) {
        const float* src[4] = {c0, c1, c2, c3};
        const int n4 = D / 4;
        for (int e = tid; e < 4 * n4; e += kRkFusedThreads) {
            const int v = e / n4, q = (e - v * n4) * 4;
            cp_async16(cst + v * D + q, src[v] + q, 16u);
        }
    };
    for (int l = 0; l < a.L; ++l) {
        const RkFLayer& Y = ltab[l];
        float* sh = a.shift + (size_t)l * 2 * D;
        const int Rw = Y.Rw, Ra = Y.Ra, Rv = l > 0 ? Y.Rv : 0, R = Rw + Ra + Rv;
        // ------------------------------------------------------------- A
        if (l > 0) arrive();
        if (cta < a.NH) {  // head h's 64 channels' LoRA rows (w2, a2, v2) and constants
            // rows of R + 4 floats: 16-byte aligned (ranks % 4 == 0), and
            // consecutive channels' float4 reads fall on different bank groups
            const int c0 = cta * 64, RS = R + 4, R4 = R / 4;
            for (int e = tid; e < 64 * R4; e += kRkFusedThreads) {
                const int t = e / R4, q = (e - t * R4) * 4, i = c0 + t;
                const float* src = q < Rw        ? Y.w2 + (size_t)i * Rw + q
                                   : q < Rw + Ra ? Y.a2 + (size_t)i * Ra + (q - Rw)
                                                 : Y.v2 + (size_t)i * Y.Rv + (q - Rw - Ra);
                cp_async16(lrows + t * RS + q, src, 16u);
            }
            if (tid < 80) {
                const float* hsrc[5] = {Y.w0, Y.a0, Y.v0, Y.kkw, Y.kaw};
                cp_async16(&hc[tid >> 4][(tid & 15) * 4], hsrc[tid >> 4] + c0 + (tid & 15) * 4,
                           16u);
            }
        }
        {
            const int* part = l == 0 ? a.part0 : a.part1;
            const int np = l == 0 ? 6 : 7;
            int p = 0;
            while (p + 1 < np && cta >= part[p + 1]) ++p;
            const RkFMat* mats[7] = {&Y.rw, &Y.kw, &Y.vw, &Y.w1, &Y.a1, &Y.g1, &Y.v1};
            float* outs[7] = {a.r, a.k, a.v, a.lo_w, a.lo_a, a.lo_g, a.lo_v};
            const int plane[7] = {0, 2, 3, 1, 4, 5, 3};  // r, k, v <- xr, xk, xv; w1, a1, g1, v1
            const int epis[7] = {kW4Store, kW4Store, kW4Store, kW4Tanh, kW4Store, kW4Sigmoid,
                                 kW4Store};
            // the time-mix shift row: this layer's BC phase rewrites it, after this read
            consts(sh, Y.ln1w, Y.ln1b, Y.lerp + (size_t)plane[p] * D);
            const int c0 = part[p], c1 = part[p + 1];
            rk_rows<FP16S, NCHD>(
                *mats[p], outs[p], epis[p], a.block, (cta - c0) * (kRkFusedThreads / 32) + warp,
                (c1 - c0) * (kRkFusedThreads / 32), sm, [&] {
                    if (l > 0) {
                        sync();
                        rk_stage(xr, a.x, D);
                    }
                    cp_async_wait_all();  // the constants (and a head's LoRA rows)
                    __syncthreads();
                    float mean, rstd;
                    row_stats(xr, D, a.eps, red, &mean, &rstd);
                    for (int i = tid; i < D; i += kRkFusedThreads) {
                        const float xn = (xr[i] - mean) * rstd * cst[D + i] + cst[2 * D + i];
                        const float d = cst[i] - xn;
                        mix[i] = xn + cst[3 * D + i] * d;
                        if (cta == 0) a.xn[i] = xn;
                    }
                    __syncthreads();
                    return static_cast<const float*>(mix);
                });
        }
        if (!ok) return;
        // ------------------------------------------------------------ BC
        arrive();
        if (cta < a.NH) {
            const int c0 = cta * 64;
            rk_heads_body<2, true, true>(
                cta, 0, a.NH, a.L, l, D, a.S, a.ww, a.k, a.v, a.a, a.kk, a.r, a.g, Y.rkw, Y.lnxw,
                Y.lnxb, a.y, 1, kn, yv, red, [&] {  // once the state rows are requested
                    sync();
                    float* lw = lov;
                    float* la = lw + Rw;
                    float* lv = la + Ra;
                    for (int i = tid; i < Rw; i += kRkFusedThreads) lw[i] = __ldcg(a.lo_w + i);
                    for (int i = tid; i < Ra; i += kRkFusedThreads) la[i] = __ldcg(a.lo_a + i);
                    for (int i = tid; i < Rv; i += kRkFusedThreads) lv[i] = __ldcg(a.lo_v + i);
                    __syncthreads();
                    if (tid < 192) {  // w, a, v sums of channel c0 + t on three groups
                        const int t = tid & 63, which = tid >> 6;
                        const int q0 = which == 0 ? 0 : which == 1 ? Rw : Rw + Ra;
                        const int n = which == 0 ? Rw : which == 1 ? Ra : Rv;
                        const float* lo = lw + q0;
                        const float* wr = lrows + t * (R + 4) + q0;
                        float acc = 0.0f;
                        for (int q = 0; q < n; q += 4) {  // sequential in q, four per load
                            const float4 w4 = *reinterpret_cast<const float4*>(wr + q);
                            acc = fmaf(lo[q], w4.x, acc);
                            acc = fmaf(lo[q + 1], w4.y, acc);
                            acc = fmaf(lo[q + 2], w4.z, acc);
                            acc = fmaf(lo[q + 3], w4.w, acc);
                        }
                        dlo[which][t] = acc;
                    }
                    __syncthreads();
                    if (tid < 64) {  // the LoRA mix of channel c0 + tid
                        const int i = c0 + tid;
                        a.ww[i] = expf(-sigm(dlo[0][tid] + hc[0][tid]) * kInvSqrtE);
                        if (l == 0) {
                            a.vfirst[i] = __ldcg(a.v + i);
                        } else {
                            const float vv = __ldcg(a.v + i);
                            a.v[i] = vv + (__ldcg(a.vfirst + i) - vv) * sigm(dlo[2][tid] + hc[2][tid]);
                        }
                        const float aa = sigm(dlo[1][tid] + hc[1][tid]);
                        a.a[i] = aa;
                        const float kv = __ldcg(a.k + i);
                        a.kk[i] = kv * hc[3][tid];
                        a.k[i] = kv + kv * (aa - 1.0f) * hc[4][tid];
                    }
                    __syncthreads();  // the head's vectors are written (read back through L2)
                    return ok;
                });
        } else {
            rk_rows<FP16S, NCHD>(Y.g2, a.g, kW4Store, a.block,
                                 (cta - a.NH) * (kRkFusedThreads / 32) + warp,
                                 (nct - a.NH) * (kRkFusedThreads / 32), sm, [&] {
                                     sync();
                                     if (ok && cta == nct - 1)  // the time-mix shift: A read the old one
                                         for (int i = tid; i < D; i += kRkFusedThreads)
                                             sh[i] = __ldcg(a.xn + i);
                                     return rk_stage(lov, a.lo_g, Y.g2.in);
                                 });
        }
        if (!ok) return;
        // ------------------------------------------------------------- D
        arrive();
        rk_rows<FP16S, NCHD>(Y.ow, a.x, kW4Add, a.block, gw, nw, sm, [&] {
            sync();
            return rk_stage(mix, a.y, D, a.g);
        });
        if (!ok) return;
        // ------------------------------------------------------------- E
        arrive();
        // the channel-mix shift row: F rewrites it, after this read
        consts(sh + D, Y.ln2w, Y.ln2b, Y.cmk_lerp);
        rk_rows<FP16S, NCHD>(Y.cmk, a.ck, kW4Relu2, a.block, gw, nw, sm, [&] {
            sync();
            rk_stage(xr, a.x, D);
            cp_async_wait_all();
            __syncthreads();
            float mean, rstd;
            row_stats(xr, D, a.eps, red, &mean, &rstd);
            for (int i = tid; i < D; i += kRkFusedThreads) {
                const float xn2 = (xr[i] - mean) * rstd * cst[D + i] + cst[2 * D + i];
                mix[i] = xn2 + cst[3 * D + i] * (cst[i] - xn2);
                if (cta == 0) a.xn2[i] = xn2;
            }
            __syncthreads();
            return static_cast<const float*>(mix);
        });
        if (!ok) return;
        // ------------------------------------------------------------- F
        arrive();
        rk_rows<FP16S, NCHF>(Y.cmv, a.x, kW4Add, a.block, gw, nw, sm, [&] {
            sync();
            if (ok && cta == 0)  // the channel-mix shift: E read the old one
                for (int i = tid; i < D; i += kRkFusedThreads) sh[D + i] = __ldcg(a.xn2 + i);
            return rk_stage(xr, a.ck, a.F);
        });
        if (!ok) return;
    }
    if (a.with_head) {  // final LN (rk_ln_kernel's arithmetic), then the head rows
        arrive();
        rk_rows<FP16S, NCHD>(a.head, a.logits, kW4Store, a.block, gw, nw, sm, [&] {
            sync();
            rk_stage(xr, a.x, D);
            float mean, rstd;
            row_stats(xr, D, a.eps, red, &mean, &rstd);
            for (int i = tid; i < D; i += kRkFusedThreads)
                mix[i] = (xr[i] - mean) * rstd * a.on_w[i] + a.on_b[i];
            __syncthreads();
            return static_cast<const float*>(mix);
        });
    }
}

// The fused step applies to one sequence of a model whose every contraction
// is W4A8 (one block size and scale type), with fp32 LoRA second stages of
// rank <= kLoraMax, 64-wide heads, and widths the SIMT rows take.
bool rk_fused_shape_ok(const RwkvModel* m) {
    if (!m->q4 || m->HS != 64 || m->D % 32 || m->D > 2048 || m->F % 32 || m->F > 4096)
        return false;
    const int blk = m->head.block;
    const bool f16 = m->head.fp16;
    if (!(blk == 32 || blk == 64 || blk == 128 || blk == 256)) return false;
    auto q4 = [&](const RkMat& M, int in) {
        return M.q4 && M.block == blk && M.fp16 == f16 && M.in == in && M.in % 32 == 0 &&
               M.in % blk == 0 && (uintptr_t)M.q % 16 == 0;
    };
    if (!q4(m->head, m->D) || m->head.out != m->vocab) return false;
    for (int l = 0; l < m->L; ++l) {
        const RkLayer& A = m->ly[l];
        if (!q4(A.rw, m->D) || !q4(A.kw, m->D) || !q4(A.vw, m->D) || !q4(A.w1, m->D) ||
            !q4(A.a1, m->D) || !q4(A.g1, m->D) || (l > 0 && !q4(A.v1, m->D)) ||
            !q4(A.g2, A.g2.in) || A.g2.in > m->D || A.g2.out != m->D || !q4(A.ow, m->D) ||
            !q4(A.cmk, m->D) || !q4(A.cmv, m->F))
            return false;
        if (A.w2.q4 || A.a2.q4 || (l > 0 && A.v2.q4) || A.w2.in > kLoraMax ||
            A.a2.in > kLoraMax || A.v2.in > kLoraMax || A.w2.in % 4 || A.a2.in % 4 ||
            A.v2.in % 4 || (uintptr_t)A.w2.w % 16 || (uintptr_t)A.a2.w % 16 ||
            (l > 0 && (uintptr_t)A.v2.w % 16))
            return false;
    }
    return true;
}

RkFMat fmat(const RkMat& M) { return RkFMat{M.q, M.scale, M.in, M.out}; }

// First CTA of each of np problems (np + 1 entries, the last = ctas): CTAs
// first .. ctas - 1 in proportion to the problems' rows, at least one each.
void rk_partition(const int* rows, int np, int first, int ctas, int* part) {
    const int avail = ctas - first;
    long long tot = 0;
    for (int p = 0; p < np; ++p) tot += rows[p];
    int n[8], used = 0;
    for (int p = 0; p < np; ++p) {
        n[p] = std::max(1, (int)((long long)avail * rows[p] / tot));
        used += n[p];
    }
    while (used > avail) {  // take back from the largest
        int b = 0;
        for (int p = 1; p < np; ++p) if (n[p] > n[b]) b = p;
        --n[b];
        --used;
    }
    for (int p = 0; used < avail; p = (p + 1) % np, ++used) ++n[p];
    part[0] = first;
    for (int p = 0; p < np; ++p) part[p + 1] = part[p] + n[p];
}

// The fused step's kernel instance, shared-memory size and W4A8 area.
struct RkFusedCfg {
    void (*kern)(RkFArgs) = nullptr;
    size_t smem = 0, qbytes = 0;
};
RkFusedCfg rk_fused_cfg(const RwkvModel* m) {
    const int D = m->D;
    const int nchd = D <= 1024 ? 1 : 2, nchf = m->F <= 1024 ? 1 : (m->F <= 2048 ? 2 : 4);
    const bool f16 = m->head.fp16;
    auto kern = [&]() -> void (*)(RkFArgs) {
#define RKF(F16, A, B) if (f16 == F16 && nchd == A && nchf == B) return rk_fused_kernel<F16, A, B>;
        RKF(false, 1, 1) RKF(false, 1, 2) RKF(false, 1, 4) RKF(false, 2, 2) RKF(false, 2, 4)
        RKF(true, 1, 1) RKF(true, 1, 2) RKF(true, 1, 4) RKF(true, 2, 2) RKF(true, 2, 4)
#undef RKF
        return nullptr;
    }();
    RkFusedCfg c;
    c.kern = kern;
    const int maxin = std::max(D, m->F);
    const int blk = m->head.block > 0 ? m->head.block : 32;
    c.qbytes = ((size_t)kMaxSeqTile * maxin + (size_t)kMaxSeqTile * (maxin / blk) * 8 + 15) / 16 * 16;
    c.smem = c.qbytes + ((size_t)maxin + D + 3 * kLoraMax + D + (size_t)64 * (3 * kLoraMax + 4) + (size_t)4 * D) *
                            sizeof(float) +
             (size_t)m->L * sizeof(RkFLayer);
    return c;
}

// Check the model and build the fused step's device tables, once per model
// and outside any stream capture (it allocates and copies): m->fused becomes
// 1, or 0 when the model or the device does not take the fused step.
int rk_fused_setup(RwkvModel* m) {
    if (m->fused >= 0) return SN_OK;
    m->fused = 0;
    const RkFusedCfg c = rk_fused_cfg(m);
    auto kern = c.kern;
    const size_t smem = c.smem;
    {
        // the heads' CTAs and at least as many again for the g2 rows
        if (!kern || !rk_fused_shape_ok(m) || smem > 200 * 1024 || rt().num_sms < 2 * m->NH)
            return SN_OK;
        SN_TRY(cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)smem),
                          "rwkv fused smem"));
        int per_sm = 0;
        SN_TRY(cuda_check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                              &per_sm, kern, kRkFusedThreads, smem),
                          "rwkv fused occupancy"));
        if (per_sm < 1) return SN_OK;
        std::vector<RkFLayer> h(m->L);
        for (int l = 0; l < m->L; ++l) {
            const RkLayer& A = m->ly[l];
            RkFLayer& f = h[l];
            f.ln1w = A.ln1w; f.ln1b = A.ln1b; f.ln2w = A.ln2w; f.ln2b = A.ln2b;
            f.lerp = A.lerp; f.cmk_lerp = A.cmk_lerp;
            f.rw = fmat(A.rw); f.kw = fmat(A.kw); f.vw = fmat(A.vw); f.w1 = fmat(A.w1);
            f.a1 = fmat(A.a1); f.g1 = fmat(A.g1); f.v1 = fmat(A.v1); f.g2 = fmat(A.g2);
            f.ow = fmat(A.ow); f.cmk = fmat(A.cmk); f.cmv = fmat(A.cmv);
            f.w2 = A.w2.w; f.a2 = A.a2.w; f.v2 = A.v2.w;
            f.Rw = A.w2.in; f.Ra = A.a2.in; f.Rv = A.v2.in;
            f.w0 = A.w0; f.a0 = A.a0; f.v0 = A.v0; f.kkw = A.kkw; f.kaw = A.kaw;
            f.rkw = A.rkw; f.lnxw = A.lnxw; f.lnxb = A.lnxb;
        }
        m->flayers = m->dalloc<RkFLayer>(m->L);
        m->fbar = m->dalloc<unsigned>(64);
        m->xn2 = m->dalloc<float>(m->D);
        if (!m->flayers || !m->fbar || !m->xn2) return fail(SN_E_NOMEM, "rwkv fused tables");
        SN_TRY(cuda_check(cudaMemcpy(m->flayers, h.data(), h.size() * sizeof(RkFLayer),
                                     cudaMemcpyHostToDevice),
                          "rwkv fused tables"));
        m->fctas = rt().num_sms;
        m->fused = 1;
    }
    return SN_OK;
}

// Launch the fused step (set up first: rk_fused_setup); SN_E_UNSUPPORTED when
// the model or the device does not take it (the caller then runs the chain).
int rk_fused_launch(RwkvModel* m, const RkBufs& w, bool head, cudaStream_t st) {
    SN_TRY(rk_fused_setup(m));
    if (m->fused != 1) return SN_E_UNSUPPORTED;
    const RkFusedCfg c = rk_fused_cfg(m);
    auto kern = c.kern;
    const size_t smem = c.smem, qbytes = c.qbytes;
    const int D = m->D;
    RkFArgs a{};
    a.layers = m->flayers;
    a.L = m->L; a.D = D; a.NH = m->NH; a.F = m->F; a.block = m->head.block;
    a.with_head = head ? 1 : 0;
    a.eps = m->eps;
    a.tok = w.tok; a.vocab = m->vocab; a.err = rt().d_err;
    a.embed = m->embed; a.en_w = m->en_w; a.en_b = m->en_b; a.on_w = m->on_w; a.on_b = m->on_b;
    a.head = fmat(m->head);
    a.S = m->S; a.shift = m->shift;
    a.x = w.x; a.r = w.r; a.k = w.k; a.v = w.v; a.a = w.a; a.g = w.g; a.kk = w.kk; a.ww = w.ww;
    a.y = w.y; a.ck = w.ck; a.lo_w = w.lo_w; a.lo_a = w.lo_a; a.lo_v = w.lo_v; a.lo_g = w.lo_g;
    a.vfirst = w.vfirst; a.logits = w.logits; a.xn = w.xn; a.xn2 = m->xn2;
    a.bar = m->fbar;
    {
        const RkLayer& A = m->ly[m->L > 1 ? 1 : 0];
        const int rows[7] = {A.rw.out, A.kw.out, A.vw.out, A.w1.out, A.a1.out, A.g1.out, A.v1.out};
        rk_partition(rows, 6, 0, m->fctas, a.part0);
        rk_partition(rows, 7, 0, m->fctas, a.part1);
    }
    a.qbytes = qbytes;
    SN_TRY(cuda_check(cudaMemsetAsync(m->fbar, 0, 64 * sizeof(unsigned), st), "rwkv fused reset"));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)m->fctas);
    cfg.blockDim = dim3(kRkFusedThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_check(cudaLaunchKernelEx(&cfg, kern, a), "rwkv fused step launch");
}

// trace (device, (B, L+1, D)) or nullptr: the residual stream entering each
// layer and leaving the last one, copied out after the embedding and after
// every layer (a debugging view of the same kernels, used without a graph).
// A pass over `nb` sequences of T tokens each (rows = nb * T, sequence-major;
// T = 1 is a decode step): every contraction and elementwise kernel runs over
// all rows at once, the token shift reads the previous row of the same
// sequence, the matrix-state recurrence walks each sequence's rows in order.
// With T > 1 the shift states are set from each sequence's last row after
// the kernels that read them, and the head (when asked) runs on the last row
// of each sequence only.
int enqueue_rk(RwkvModel* m, const RkBufs& w, int nb, int T, bool head, cudaStream_t st,
               int last_layer = -1, float* trace = nullptr) {
    const int D = m->D;
    // one sequence's decode step: the fused persistent kernel where it applies
    // (SN_RK_UNFUSED=1 keeps the kernel chain, for comparisons)
    if (nb == 1 && T == 1 && last_layer < 0 && !trace && !getenv("SN_RK_UNFUSED")) {
        ProfScope ps("rk_fused", st);
        const int rc = rk_fused_launch(m, w, head, st);
        if (rc != SN_E_UNSUPPORTED) return rc;
    }
    const int B = nb * T;  // rows
    const size_t plane = (size_t)B * D;
    // the shift state of layer l, slot j, from the last row of each sequence
    auto shift_from_last = [&](int l, int j, const float* src) {
        return cuda_check(cudaMemcpy2DAsync(m->shift + ((size_t)l * 2 + j) * D,
                                            (size_t)m->L * 2 * D * 4, src + (size_t)(T - 1) * D,
                                            (size_t)T * D * 4, (size_t)D * 4, (size_t)nb,
                                            cudaMemcpyDeviceToDevice, st),
                          "shift update");
    };
    const long long sh_stride = (long long)m->L * 2 * D;
    auto trace_x = [&](int j) {
        return cuda_check(cudaMemcpy2DAsync(trace + (size_t)j * D, (size_t)(m->L + 1) * D * 4,
                                            w.x, (size_t)D * 4, (size_t)D * 4, (size_t)B,
                                            cudaMemcpyDeviceToDevice, st),
                          "trace copy");
    };
    rk_embed_kernel<<<B, 256, 0, st>>>(D, w.tok, m->vocab, rt().d_err, m->embed, m->en_w,
                                       m->en_b, w.x, m->eps);
    if (trace) SN_TRY(trace_x(0));
    const int nl = last_layer >= 0 ? last_layer + 1 : m->L;
    const unsigned ew = (unsigned)((plane + 255) / 256);
    for (int l = 0; l < nl; ++l) {
        const RkLayer& A = m->ly[l];
        float* sh = m->shift + (size_t)l * 2 * D;
        // every kernel after the embedding follows another one on this stream:
        // programmatic launches (each waits before touching its inputs)
        SN_TRY(cuda_check(launch_pdl(rk_tmix_prep_kernel, dim3(B), dim3(256), 0, st, D, B,
                                     (const float*)w.x, sh, sh_stride, (const float*)A.ln1w,
                                     (const float*)A.ln1b, (const float*)A.lerp, w.xn, w.planes,
                                     m->eps, T),
                          "tmix launch"));
        if (T > 1) SN_TRY(shift_from_last(l, 0, w.xn));
        const float *xr = w.planes, *xw = xr + plane, *xk = xw + plane, *xv = xk + plane,
                    *xa = xv + plane, *xg = xa + plane;
        {   // first-stage projections of the input mixes (v1 from layer 1 on):
            // one grouped tensor-core launch when every matrix qualifies
            const RkMat* gm[7] = {&A.rw, &A.kw, &A.vw, &A.w1, &A.a1, &A.g1, &A.v1};
            float* gy[7] = {w.r, w.k, w.v, w.lo_w, w.lo_a, w.lo_g, w.lo_v};
            const float* gx[7] = {xr, xk, xv, xw, xa, xg, xv};
            const int ge[7] = {E_STORE, E_STORE, E_STORE, E_TANH, E_STORE, E_SIG, E_STORE};
            const int ng = l > 0 ? 7 : 6;
            bool grouped = gm[0]->q4 && w4a8_tc_ready(B, D, gm[0]->block, 6);
            for (int i = 0; i < ng && grouped; ++i)
                grouped = gm[i]->q4 && gm[i]->in == D && gm[i]->block == gm[0]->block &&
                          gm[i]->fp16 == gm[0]->fp16 &&
                          w4a8_tc_ok(B, gm[i]->in, gm[i]->out, gm[i]->block, gm[i]->q);
            // small batches: the same group on the SIMT kernel
            bool small = !grouped && B <= 8 && gm[0]->q4;
            for (int i = 0; i < ng && small; ++i)
                small = gm[i]->q4 && gm[i]->in == D && gm[i]->block == gm[0]->block &&
                        gm[i]->fp16 == gm[0]->fp16 && (uintptr_t)gm[i]->q % 16 == 0;
            small = small && D % 32 == 0 && D <= 4096 &&
                    (gm[0]->block == 32 || gm[0]->block == 64 || gm[0]->block == 128 ||
                     gm[0]->block == 256);
            if (grouped || small) {
                static const int map[] = {kW4Store, kW4Add, kW4Relu2, kW4Tanh, kW4Sigmoid};
                W4Problem pr[7];
                for (int i = 0; i < ng; ++i)
                    pr[i] = W4Problem{gy[i], gx[i], gm[i]->q, gm[i]->scale, gm[i]->out, map[ge[i]]};
                ProfScope ps("w4a8_group", st);
                if (grouped)
                    SN_TRY(launch_w4a8_tc_group(pr, ng, B, D, gm[0]->block, gm[0]->fp16, st, true));
                else
                    SN_TRY(launch_w4a8_group(pr, ng, B, D, gm[0]->block, gm[0]->fp16, st, true));
            } else {
                for (int i = 0; i < ng; ++i) SN_TRY(mat_mul(*gm[i], gy[i], gx[i], B, ge[i], st));
            }
        }
        SN_TRY(mat_mul(A.g2, w.g, w.lo_g, B, E_STORE, st));
        // fp32 LoRA second stages (ranks below a quantisation block stay fp32)
        // are folded into the mix kernel
        const int R = A.w2.in + A.a2.in + (l > 0 ? A.v2.in : 0);
        const size_t smem = ((size_t)R * 33 + 8 * R) * 4;
        const bool fold = !A.w2.q4 && !A.a2.q4 && (l == 0 || !A.v2.q4) && A.w2.in <= kLoraMax &&
                          A.a2.in <= kLoraMax && A.v2.in <= kLoraMax && smem <= 48 * 1024;
        if (fold) {
            ProfScope ps("rk_lora_mix", st);
            SN_TRY(cuda_check(
                launch_pdl(rk_lora_mix_kernel, dim3((unsigned)((D + 31) / 32), (unsigned)((B + 7) / 8)),
                           dim3(256), smem, st, B, D, l == 0 ? 1 : 0, A.w2.in, A.a2.in, A.v2.in,
                           (const float*)A.w2.w, (const float*)A.a2.w, (const float*)A.v2.w,
                           (const float*)w.lo_w, (const float*)w.lo_a, (const float*)w.lo_v,
                           (const float*)A.w0, (const float*)A.v0, (const float*)A.a0,
                           (const float*)A.kkw, (const float*)A.kaw, w.ww, w.v, w.vfirst, w.a,
                           w.k, w.kk),
                "lora mix launch"));
        } else {
            SN_TRY(mat_mul(A.w2, w.dw, w.lo_w, B, E_STORE, st));
            if (l > 0) SN_TRY(mat_mul(A.v2, w.dv, w.lo_v, B, E_STORE, st));
            SN_TRY(mat_mul(A.a2, w.da, w.lo_a, B, E_STORE, st));
            SN_TRY(cuda_check(launch_pdl(rk_mix_kernel, dim3(ew), dim3(256), 0, st, B, D,
                                         l == 0 ? 1 : 0, (const float*)w.dw, (const float*)A.w0,
                                         (const float*)w.dv, (const float*)A.v0,
                                         (const float*)w.da, (const float*)A.a0,
                                         (const float*)A.kkw, (const float*)A.kaw, w.ww, w.v,
                                         w.vfirst, w.a, w.k, w.kk),
                              "mix launch"));
        }
        {
            const dim3 grid((unsigned)(nb * m->NH));
            ProfScope ps_heads("rk_heads", st);
            cudaError_t e;
            switch (m->HS) {
#define RK_HEADS(V)                                                                                \
    e = launch_pdl(rk_heads_kernel<V>, grid, dim3(256), 0, st, m->NH, m->L, l, D, m->S,            \
                   (const float*)w.ww, (const float*)w.k, (const float*)w.v, (const float*)w.a, \
                   (const float*)w.kk, (const float*)w.r, (const float*)w.g,                    \
                   (const float*)A.rkw, (const float*)A.lnxw, (const float*)A.lnxb, w.y, T);      \
    break;
                case 32: RK_HEADS(1)
                case 64: RK_HEADS(2)
                case 128: RK_HEADS(4)
                default: RK_HEADS(8)
#undef RK_HEADS
            }
            SN_TRY(cuda_check(e, "heads launch"));
        }
        SN_TRY(mat_mul(A.ow, w.x, w.y, B, E_ADD, st));
        SN_TRY(cuda_check(launch_pdl(rk_cmix_prep_kernel, dim3(B), dim3(256), 0, st, D,
                                     (const float*)w.x, sh, sh_stride, (const float*)A.ln2w,
                                     (const float*)A.ln2b, (const float*)A.cmk_lerp, w.xk2,
                                     m->eps, T, T > 1 ? w.xn : (float*)nullptr),
                          "cmix launch"));
        if (T > 1) SN_TRY(shift_from_last(l, 1, w.xn));
        SN_TRY(mat_mul(A.cmk, w.ck, w.xk2, B, E_RELU2, st));
        SN_TRY(mat_mul(A.cmv, w.x, w.ck, B, E_ADD, st));
        if (trace) SN_TRY(trace_x(l + 1));
    }
    if (last_layer < 0 && head) {  // the last row of each sequence
        SN_TRY(cuda_check(launch_pdl(rk_ln_kernel, dim3(nb), dim3(256), 0, st, D,
                                     (const float*)(w.x + (size_t)(T - 1) * D),
                                     (const float*)m->on_w, (const float*)m->on_b, w.xf, m->eps,
                                     (long long)T * D),
                          "ln launch"));
        SN_TRY(mat_mul(m->head, w.logits, w.xf, nb, E_STORE, st));
    }
    return cuda_check(cudaGetLastError(), "rwkv step launch");
}

int rk_run(RwkvModel* m, int B, bool head, float* trace = nullptr) {
    auto key = std::make_pair(B, head ? 1 : 0);
    if (B == 1) SN_TRY(rk_fused_setup(m));  // allocates: before any capture
    if (prof_graph() && !trace)  // the step's graph with event nodes around each family
        return prof_graph_run(&m->pgraphs[key], m->cap, stream(),
                              [&](cudaStream_t cs) {
                                  return enqueue_rk(m, step_bufs(m), B, 1, head, cs);
                              });
    if (prof_on() || trace)  // bracket kernels / copy out the trace: no graph
        return enqueue_rk(m, step_bufs(m), B, 1, head, stream(), -1, trace);
    auto it = m->graphs.find(key);
    if (it == m->graphs.end()) {
        cudaGraph_t g = nullptr;
        SN_TRY(cuda_check(cudaStreamBeginCapture(m->cap, cudaStreamCaptureModeThreadLocal),
                          "begin capture"));
        const int rc = enqueue_rk(m, step_bufs(m), B, 1, head, m->cap);
        const cudaError_t e = cudaStreamEndCapture(m->cap, &g);
        if (rc != SN_OK) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        SN_TRY(cuda_check(e, "end capture"));
        cudaGraphExec_t ex = nullptr;
        const cudaError_t e2 = cudaGraphInstantiate(&ex, g, 0);
        cudaGraphDestroy(g);
        SN_TRY(cuda_check(e2, "graph instantiate"));
        it = m->graphs.emplace(key, ex).first;
    }
    return cuda_check(cudaGraphLaunch(it->second, stream()), "graph launch");
}

int rk_step(RwkvModel* m, const int32_t* tokens, int B, float* logits, int32_t* next,
            float* xs = nullptr) {
    if (!m || !m->ready || !tokens || B <= 0 || B > m->nseq)
        return fail(SN_E_INVAL, "rwkv7_step: bad handle, tokens or B");
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    cudaStream_t st = stream();
    const bool tdev = is_device_ptr(tokens);
    SN_TRY(cuda_check(cudaMemcpyAsync(m->tok, tokens, (size_t)B * 4,
                                      tdev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, st),
                      "tokens"));
    Arr XS;
    if (xs) SN_TRY(stage_out(xs, (size_t)B * (m->L + 1) * m->D * 4, 11, &XS));
    SN_TRY(rk_run(m, B, logits || next, xs ? (float*)XS.dev : nullptr));
    bool host = !tdev;
    if (xs) {
        SN_TRY(copy_back(XS));
        host |= XS.host != nullptr;
    }
    if (logits) {
        const bool dev = is_device_ptr(logits);
        host |= !dev;
        SN_TRY(cuda_check(cudaMemcpyAsync(logits, m->logits, (size_t)B * m->vocab * 4,
                                          dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost,
                                          st),
                          "logits"));
    }
    if (next) {
        SN_TRY(launch_argmax(m->logits, B, m->vocab, m->apart, m->next, st));
        const bool dev = is_device_ptr(next);
        host |= !dev;
        SN_TRY(cuda_check(cudaMemcpyAsync(next, m->next, (size_t)B * 4,
                                          dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost,
                                          st),
                          "next"));
    }
    return finish(host);
}

// Prompt of T tokens for each of nb sequences (tokens (nb, T) row-major, host
// or device) -> logits (nb, vocab) of each sequence's last token (NULL: state
// only). Replaces the reference's token-by-token loop (rwkv7.c:362-364) with
// layer-major passes over chunks of the prompt: every contraction over all
// nb x Tc rows of a chunk at once, the recurrence T-serial per (sequence,
// head), the state carried from chunk to chunk.
constexpr int kPrefillRows = 8192;  // rows per pass (bounds the workspace)

int rk_prefill(RwkvModel* m, const int32_t* tokens, int nb, int T, float* logits) {
    if (!m || !m->ready || !tokens || nb <= 0 || T <= 0 || nb > m->nseq)
        return fail(SN_E_INVAL, "rwkv7_prefill: bad handle, tokens or shape");
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    cudaStream_t st = stream();
    int cap = std::max(kPrefillRows, m->nseq);
    if (const char* e = getenv("SN_RK_PREFILL_ROWS"))  // test hook: smaller passes
        cap = std::max(1, atoi(e));
    const int Tc = std::max(1, std::min(T, cap / nb));
    SN_TRY(ensure_pre(m, nb * Tc));
    const bool tdev = is_device_ptr(tokens);
    for (int t0 = 0; t0 < T; t0 += Tc) {
        const int tc = std::min(Tc, T - t0);
        SN_TRY(cuda_check(cudaMemcpy2DAsync(m->pre.tok, (size_t)tc * 4, tokens + t0,
                                            (size_t)T * 4, (size_t)tc * 4, (size_t)nb,
                                            tdev ? cudaMemcpyDeviceToDevice
                                                 : cudaMemcpyHostToDevice,
                                            st),
                          "prefill tokens"));
        SN_TRY(enqueue_rk(m, m->pre, nb, tc, logits != nullptr && t0 + tc >= T, st));
    }
    bool host = !tdev;
    if (logits) {
        const bool dev = is_device_ptr(logits);
        host |= !dev;
        SN_TRY(cuda_check(cudaMemcpyAsync(logits, m->pre.logits, (size_t)nb * m->vocab * 4,
                                          dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost,
                                          st),
                          "logits"));
    }
    return finish(host);
}

int rk_reset(RwkvModel* m) {
    if (!m || !m->ready) return fail(SN_E_INVAL, "rwkv7_reset: bad handle");
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    const size_t B = (size_t)m->nseq;
    cudaStream_t st = stream();
    cudaMemsetAsync(m->S, 0, B * m->L * m->NH * m->HS * m->HS * 4, st);
    cudaMemsetAsync(m->shift, 0, B * m->L * 2 * m->D * 4, st);
    return finish(false);
}

}  // namespace
}  // namespace sn

using namespace sn;

struct SnAbiRwkv7 {
    std::unique_ptr<RwkvModel> m;
};
struct SnRWKV7 {
    std::unique_ptr<RwkvModel> m;
};

namespace {
std::unique_ptr<RwkvModel> open_rwkv(const char* path, int nseq) {
    if (!path || nseq <= 0) {
        fail(SN_E_INVAL, "rwkv7 load: null path or nseq <= 0");
        return nullptr;
    }
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    auto m = std::make_unique<RwkvModel>();
    if (load_rwkv(m.get(), path, nseq) != SN_OK) return nullptr;
    return m;
}
}  // namespace

extern "C" {

SnAbiRwkv7* sn_abi_rwkv7_load(const char* blob_path) {
    auto m = open_rwkv(blob_path, 1);
    return m ? new SnAbiRwkv7{std::move(m)} : nullptr;
}

SnAbiRwkv7* sn_abi_rwkv7_load_batch(const char* blob_path, int32_t nseq) {
    auto m = open_rwkv(blob_path, nseq);
    return m ? new SnAbiRwkv7{std::move(m)} : nullptr;
}

int32_t sn_abi_rwkv7_vocab(const SnAbiRwkv7* m) { return m ? m->m->vocab : 0; }

sn_status sn_abi_rwkv7_step(SnAbiRwkv7* m, int32_t token, float* logits) {
    if (!m || !logits || token < 0) return SN_E_INVAL;
    if (token >= m->m->vocab) return fail(SN_E_INVAL, "token %d out of range", token);
    return rk_step(m->m.get(), &token, 1, logits, nullptr);
}

sn_status sn_abi_rwkv7_prefill(SnAbiRwkv7* m, const int32_t* tokens, int32_t n, float* logits) {
    if (!m || !tokens || !logits || n <= 0) return SN_E_INVAL;
    if (!is_device_ptr(tokens))  // host ids are checked here (device ids on the device)
        for (int i = 0; i < n; ++i)
            if (tokens[i] < 0 || tokens[i] >= m->m->vocab) return SN_E_INVAL;
    return rk_prefill(m->m.get(), tokens, 1, n, logits);
}

sn_status sn_abi_rwkv7_prefill_batch(SnAbiRwkv7* m, const int32_t* tokens, int32_t B, int32_t T,
                                     float* logits) {
    if (!m) return SN_E_INVAL;
    return rk_prefill(m->m.get(), tokens, B, T, logits);
}

sn_status sn_abi_rwkv7_reset(SnAbiRwkv7* m) { return m ? rk_reset(m->m.get()) : SN_E_INVAL; }

void sn_abi_rwkv7_free(SnAbiRwkv7* m) {
    if (!m) return;
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    cudaDeviceSynchronize();
    delete m;
}

sn_status sn_abi_rwkv7_step_batch(SnAbiRwkv7* m, const int32_t* tokens, int32_t B,
                                  float* logits) {
    return m ? rk_step(m->m.get(), tokens, B, logits, nullptr) : SN_E_INVAL;
}

sn_status sn_abi_rwkv7_step_argmax(SnAbiRwkv7* m, const int32_t* tokens, int32_t B,
                                   int32_t* next) {
    if (!m || !next) return SN_E_INVAL;
    return rk_step(m->m.get(), tokens, B, nullptr, next);
}

sn_status sn_abi_rwkv7_step_trace(SnAbiRwkv7* m, const int32_t* tokens, int32_t B,
                                  float* logits, float* xs) {
    if (!m || !xs) return fail(SN_E_INVAL, "rwkv7_step_trace: null handle or trace");
    return rk_step(m->m.get(), tokens, B, logits, nullptr, xs);
}

sn_status sn_abi_rwkv7_get_state(SnAbiRwkv7* m, int32_t B, float* S, float* shift) {
    if (!m || !S || !shift || B <= 0 || B > m->m->nseq) return SN_E_INVAL;
    RwkvModel* r = m->m.get();
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    const size_t ns = (size_t)B * r->L * r->NH * r->HS * r->HS * 4;
    const size_t nh = (size_t)B * r->L * 2 * r->D * 4;
    const bool d1 = is_device_ptr(S), d2 = is_device_ptr(shift);
    cudaStream_t st = stream();
    SN_TRY(cuda_check(cudaMemcpyAsync(S, r->S, ns, d1 ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, st), "S"));
    SN_TRY(cuda_check(cudaMemcpyAsync(shift, r->shift, nh, d2 ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, st), "shift"));
    return finish(true);
}

int32_t sn_abi_rwkv7_dims(const SnAbiRwkv7* m, int32_t* d) {
    if (!m || !d) return SN_E_INVAL;
    const RwkvModel* r = m->m.get();
    const int32_t v[8] = {r->vocab, r->D, r->HS, r->NH, r->F, r->L, r->q4, r->group};
    memcpy(d, v, sizeof v);
    return SN_OK;
}

// ---------------------------------------------------- reference rwkv7.h symbol set
SnRWKV7* sn_rk_load(const char* path) {
    auto m = open_rwkv(path, 1);
    return m ? new SnRWKV7{std::move(m)} : nullptr;
}

void sn_rk_free(SnRWKV7* m) {
    if (!m) return;
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    cudaDeviceSynchronize();
    delete m;
}

void sn_rk_reset(SnRWKV7* m) {
    if (m) rk_reset(m->m.get());
}

void sn_rk_step(SnRWKV7* m, int token, float* logits) {
    if (!m) return;
    const int32_t t = token;
    rk_step(m->m.get(), &t, 1, logits, nullptr);
}

void sn_rk_prefill(SnRWKV7* m, const int* tokens, int n, float* logits) {
    if (!m || !tokens || n <= 0) return;
    rk_prefill(m->m.get(), (const int32_t*)tokens, 1, n, logits);
}

void sn_rk_dbg(SnRWKV7* m, int token, int layer, float* out) {
    if (!m || !out || layer < 0 || layer >= m->m->L) return;
    RwkvModel* r = m->m.get();
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    cudaStream_t st = stream();
    const int32_t t = token;
    cudaMemcpyAsync(r->tok, &t, 4, cudaMemcpyHostToDevice, st);
    if (enqueue_rk(r, step_bufs(r), 1, 1, false, st, layer) != SN_OK) return;
    // xn, r, k, v, a, g, ww, y, x (rwkv7.c:322-333)
    const float* parts[9] = {r->xn, r->r, r->k, r->v, r->a, r->g, r->ww, r->y, r->x};
    Arr o;
    if (stage_out(out, (size_t)9 * r->D * 4, 7, &o) != SN_OK) return;
    for (int i = 0; i < 9; ++i)
        cudaMemcpyAsync((char*)o.dev + (size_t)i * r->D * 4, parts[i], (size_t)r->D * 4,
                        cudaMemcpyDeviceToDevice, st);
    copy_back(o);
    finish(true);
}

int sn_rk_vocab(const SnRWKV7* m) { return m ? m->m->vocab : 0; }
int sn_rk_ready(const SnRWKV7* m) { return m && m->m->ready ? 1 : 0; }

}  // extern "C"
