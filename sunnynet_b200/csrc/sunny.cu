// SunnyNet whole-model decode on sm_100a.
//
// Reference: sunnynet/runtime/sunnynet.c (sn_load 358-454, layer_step 212-291,
// sn_step 321-334, sn_prefill 347-349, sn_reset 296-303, sn_dbg_layer 336-345)
// and the batched oracle SunnyNet.forward_step (model.py:113-124,
// layers.py:287-326).
//
// Per layer and step, for the B sequences of a batch (rows of every matrix
// below are sequences):
//   prep        raw = LN(x); at = raw + sum_k w_k*{raw, hist}; hist ring <- raw
//   GEMM Ws     sfb = s_old Ws^T                    (reads the previous state)
//   GEMM V      v = at V^T
//   GEMM U      q = v U^T
//   gate        u = q[:D]*sig(g_i-g_{i+1})*sig(g_i-g_{i+2}) in groups of G,
//               p = 1 - delta(1-sig(g)), s = p*s + (1-p)*u   (state in place)
//   GEMM Wz     z = u Wz^T, softwedge epilogue
//   stats       per-row mean / rstd of z
//   GEMM Wc     out = LN(z) Wc^T + (b_gain*s + sfb + x)   (LN applied on load)
// then stats + LM head with the final LN applied on load. The whole step is
// captured once per batch size into a CUDA graph and replayed.
//
// HBM layout: weights (out,in) row-major (fp32, fp16 or int8 + fp32 row
// scale); state s [seq][L][D]; conv history as a ring [seq][L][K-1][D] with a
// per-sequence write position (newest at slot (pos-1) mod (K-1)), so a step
// writes one history row instead of shifting K-1 of them.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <vector>

#include "gemm.cuh"
#include "kernels.cuh"
#include "ptx.cuh"
#include "runtime.cuh"
#include "sn_abi.h"
#include "sunny_fused.cuh"
#include "sunnynet.h"
#include "tc_gemm.cuh"

namespace sn {
namespace {

constexpr int32_t kUSNN = 0x4E4E5355;
constexpr int32_t kUSNQ = 0x514E5355;

__device__ __forceinline__ float sigm(float x) { return 1.0f / (1.0f + expf(-x)); }

// Block-wide sum (blockDim.x multiple of 32, <= 1024).
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

// One CTA per sequence: x (layer 0: embedding row), LN, causal taps, ring write.
__global__ void prep_kernel(int D, int K, int KH, int layer, int L, const int32_t* __restrict__ tok,
                            int vocab, int* __restrict__ err,
                            const float* __restrict__ embed, float* __restrict__ x,
                            float* __restrict__ raw_out, float* __restrict__ at,
                            float* __restrict__ hist, int32_t* __restrict__ pos,
                            const float* __restrict__ g, const float* __restrict__ c,
                            const float* __restrict__ dw, float eps,
                            __nv_bfloat16* __restrict__ ath = nullptr,
                            __nv_bfloat16* __restrict__ atl = nullptr) {
    __shared__ float red[32];
    pdl_trigger();  // the next GEMV may start prefetching its weights
    pdl_wait();     // no-op unless launched with programmatic serialization
    const int b = blockIdx.x;
    // ring position of this (sequence, layer); every thread reads it before the
    // block-wide barriers below, thread 0 advances it at the end
    const int p = pos[b * L + layer];
    float* xr = x + (size_t)b * D;
    if (layer == 0) {
        int t = tok[b];
        if (t < 0 || t >= vocab) {  // never read outside the table; report instead
            if (threadIdx.x == 0) atomicExch(err, kErrBadIndex);
            t = 0;
        }
        const float* e = embed + (size_t)t * D;
        for (int i = threadIdx.x; i < D; i += blockDim.x) xr[i] = e[i];
        __syncthreads();
    }
    float s = 0.0f;
    for (int i = threadIdx.x; i < D; i += blockDim.x) s += xr[i];
    const float mean = block_sum(s, red) / (float)D;
    float v = 0.0f;
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
        const float d = xr[i] - mean;
        v += d * d;
    }
    const float rstd = 1.0f / sqrtf(block_sum(v, red) / (float)D + eps);
    float* hb = hist + ((size_t)b * L + layer) * KH * D;
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
        const float r = (xr[i] - mean) * rstd * g[i] + c[i];
        float a = r;
        if (K > 1) {
            float acc = r * dw[(size_t)(K - 1) * D + i];
            for (int k = 0; k < K - 1; ++k) {
                const int slot = ((p - 1 - k) % KH + KH) % KH;
                acc += hb[(size_t)slot * D + i] * dw[(size_t)(K - 2 - k) * D + i];
            }
            a = r + acc;
            hb[(size_t)(((p % KH) + KH) % KH) * D + i] = r;
        }
        at[(size_t)b * D + i] = a;
        if (ath) store_split(ath, atl, (long long)b * D + i, a);
        if (raw_out) raw_out[(size_t)b * D + i] = r;
    }
    if (threadIdx.x == 0) pos[b * L + layer] = p + 1;
}

// Gated competition + decay gate + state update, one thread per (seq, channel).
__global__ void gate_kernel(int B, int D, int G, int L, int layer, const float* __restrict__ q,
                            const float* __restrict__ delta, float* __restrict__ s,
                            float* __restrict__ u, float* __restrict__ gate_out, int clamp,
                            float p_floor, __nv_bfloat16* __restrict__ uh = nullptr,
                            __nv_bfloat16* __restrict__ ul = nullptr) {
    pdl_trigger();
    pdl_wait();
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= (long long)B * D) return;
    const int b = (int)(i / D), d = (int)(i % D);
    const float* qb = q + (size_t)b * 2 * D;
    const int base = (d / G) * G, off = d - base;
    const float g0 = qb[D + d];
    const float g1 = qb[D + base + (off + 1) % G];
    const float g2 = qb[D + base + (off + 2) % G];
    const float uu = qb[d] * (sigm(g0 - g1) * sigm(g0 - g2));
    float p = 1.0f - delta[d] * (1.0f - sigm(g0));
    if (clamp && p < p_floor) p = p_floor;
    float* sp = s + ((size_t)b * L + layer) * D + d;
    *sp = p * *sp + (1.0f - p) * uu;
    u[i] = uu;
    if (uh) store_split(uh, ul, i, uu);
    if (gate_out) gate_out[i] = g0;
}

// Two-pass row mean / rstd.
__global__ void rowstats_kernel(int n, const float* __restrict__ X, long long ldx,
                                float* __restrict__ mu, float* __restrict__ rs, float eps) {
    __shared__ float red[32];
    const float* xr = X + blockIdx.x * ldx;
    float s = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s += xr[i];
    const float mean = block_sum(s, red) / (float)n;
    float v = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float d = xr[i] - mean;
        v += d * d;
    }
    const float r = 1.0f / sqrtf(block_sum(v, red) / (float)n + eps);
    if (threadIdx.x == 0) {
        mu[blockIdx.x] = mean;
        rs[blockIdx.x] = r;
    }
}

// Row LN written straight into bf16 planes: the statistics as rowstats_kernel
// computes them, then ((x - mu) * rs) * g + c per element (the order the
// contraction prologue uses), one CTA per row.
__global__ void ln_split_kernel(int n, const float* __restrict__ X, long long ldx,
                                const float* __restrict__ g, const float* __restrict__ c,
                                __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo,
                                float eps) {
    __shared__ float red[32];
    pdl_trigger();
    pdl_wait();
    const float* xr = X + blockIdx.x * ldx;
    float s = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s += xr[i];
    const float mean = block_sum(s, red) / (float)n;
    float v = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float d = xr[i] - mean;
        v += d * d;
    }
    const float r = 1.0f / sqrtf(block_sum(v, red) / (float)n + eps);
    const long long o = (long long)blockIdx.x * n;
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        store_split(hi, lo, o + i, __fmul_rn(__fmul_rn(xr[i] - mean, r), g[i]) + c[i]);
}


// ------------------------------------- row kernels: one float4 per thread
// One CTA per row of n floats (n % 4 == 0, 16-byte aligned rows), n / 4
// threads rounded up to whole warps, each thread holding one float4 of the
// row in registers: every load of a row is issued at once, the statistics
// are warp sums combined through shared memory, and B rows give B CTAs. The
// launchers below pick these whenever the shape allows, for every path alike
// (the step, the split-launch step, the fused B <= 8 step's fallback,
// prefill), so paths that must agree bit for bit compute their statistics the
// same way.
constexpr int kRowMaxThreads = 1024;  // rows up to 4096 floats

__device__ __forceinline__ float warp_allsum(float v) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }

// sum over the CTA (whole warps), returned to every thread
__device__ __forceinline__ float cta_allsum(float v, float* red) {
    v = warp_allsum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();  // red is free (a previous reduction has been read)
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = l < nw ? red[l] : 0.0f;
    return warp_allsum(t);
}

// mean and 1/sqrt(var + eps) of the row whose float4 `v` this thread holds
// (`live`: the thread's columns are inside the row)
__device__ __forceinline__ void cta_row_stats(float4 v, bool live, int n, float eps, float* red,
                                              float* mean, float* rstd) {
    const float s = live ? (v.x + v.y) + (v.z + v.w) : 0.0f;
    const float mu = cta_allsum(s, red) / (float)n;
    float q = 0.0f;
    if (live) {
        const float a = v.x - mu, b = v.y - mu, c = v.z - mu, d = v.w - mu;
        q = (a * a + b * b) + (c * c + d * d);
    }
    *mean = mu;
    *rstd = 1.0f / sqrtf(cta_allsum(q, red) / (float)n + eps);
}

// prep_kernel's work (LN, causal taps, ring write), one float4 per thread
__global__ void __launch_bounds__(kRowMaxThreads)
    prep_vec_kernel(int D, int K, int KH, int layer, int L, const int32_t* __restrict__ tok,
                    int vocab, int* __restrict__ err, const float* __restrict__ embed,
                    float* __restrict__ x, float* __restrict__ raw_out, float* __restrict__ at,
                    float* __restrict__ hist, int32_t* __restrict__ pos,
                    const float* __restrict__ g, const float* __restrict__ c,
                    const float* __restrict__ dw, float eps, __nv_bfloat16* __restrict__ ath,
                    __nv_bfloat16* __restrict__ atl) {
    __shared__ float red[32];
    pdl_trigger();
    const int b = blockIdx.x;
    const int col = 4 * threadIdx.x;
    const bool live = col < D;
    // Before waiting for the previous kernel: everything this kernel reads
    // that no kernel of the current step writes before it (the ring position
    // and history rows of this layer, written only by this layer's prep of
    // earlier steps; the parameters; the token and its embedding row).
    const int p = pos[b * L + layer];
    float* xr = x + (size_t)b * D;
    const float* src = xr;
    if (layer == 0) {
        int t = tok[b];
        if (t < 0 || t >= vocab) {  // never read outside the table; report instead
            if (threadIdx.x == 0) atomicExch(err, kErrBadIndex);
            t = 0;
        }
        src = embed + (size_t)t * D;
    }
    float* hb = hist + ((size_t)b * L + layer) * KH * D;
    float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f), gg = v, cc = v, wl = v;
    float4 hv[3], wv[3];
    const int kk = K - 1 < 3 ? K - 1 : 3;  // history rows held in registers
    if (live) {  // every load of this thread's columns, issued together
        gg = ld4(g + col);
        cc = ld4(c + col);
        if (K > 1) wl = ld4(dw + (size_t)(K - 1) * D + col);
#pragma unroll
        for (int j = 0; j < 3; ++j)
            if (j < kk) {
                const int slot = ((p - 1 - j) % KH + KH) % KH;
                hv[j] = ld4(hb + (size_t)slot * D + col);
                wv[j] = ld4(dw + (size_t)(K - 2 - j) * D + col);
            }
        if (layer == 0) v = ld4(src + col);
    }
    pdl_wait();  // x: the previous layer's output
    if (live) {
        if (layer > 0) v = ld4(src + col);
        else st4(xr + col, v);
    }
    float mean, rstd;
    cta_row_stats(v, live, D, eps, red, &mean, &rstd);
    if (!live) return;
    const float r[4] = {(v.x - mean) * rstd * gg.x + cc.x, (v.y - mean) * rstd * gg.y + cc.y,
                        (v.z - mean) * rstd * gg.z + cc.z, (v.w - mean) * rstd * gg.w + cc.w};
    float a[4] = {r[0], r[1], r[2], r[3]};
    if (K > 1) {
        float acc[4] = {r[0] * wl.x, r[1] * wl.y, r[2] * wl.z, r[3] * wl.w};
        for (int j = 0; j < K - 1; ++j) {
            float4 h, w;
            if (j < 3) {
                h = hv[j < 3 ? j : 0];
                w = wv[j < 3 ? j : 0];
            } else {  // taps beyond the registers: load in order
                const int slot = ((p - 1 - j) % KH + KH) % KH;
                h = ld4(hb + (size_t)slot * D + col);
                w = ld4(dw + (size_t)(K - 2 - j) * D + col);
            }
            acc[0] += h.x * w.x;
            acc[1] += h.y * w.y;
            acc[2] += h.z * w.z;
            acc[3] += h.w * w.w;
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) a[e] = r[e] + acc[e];
        st4(hb + (size_t)(((p % KH) + KH) % KH) * D + col, make_float4(r[0], r[1], r[2], r[3]));
    }
    const float4 av = make_float4(a[0], a[1], a[2], a[3]);
    st4(at + (size_t)b * D + col, av);
    if (ath) store_split4(ath, atl, (long long)b * D + col, av);
    if (raw_out) st4(raw_out + (size_t)b * D + col, make_float4(r[0], r[1], r[2], r[3]));
    if (threadIdx.x == 0) pos[b * L + layer] = p + 1;
}

// rowstats_kernel's work, one float4 per thread
__global__ void __launch_bounds__(kRowMaxThreads)
    rowstats_vec_kernel(int n, const float* __restrict__ X, long long ldx,
                        float* __restrict__ mu, float* __restrict__ rs, float eps) {
    __shared__ float red[32];
    pdl_trigger();
    pdl_wait();
    const int col = 4 * threadIdx.x;
    const bool live = col < n;
    const float4 v = live ? ld4(X + (size_t)blockIdx.x * ldx + col)
                          : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    float mean, rstd;
    cta_row_stats(v, live, n, eps, red, &mean, &rstd);
    if (threadIdx.x == 0) {
        mu[blockIdx.x] = mean;
        rs[blockIdx.x] = rstd;
    }
}

// ln_split_kernel's work, one float4 per thread: the statistics as
// rowstats_vec_kernel, then ((x - mu) * rs) * g + c per element
__global__ void __launch_bounds__(kRowMaxThreads)
    ln_split_vec_kernel(int n, const float* __restrict__ X, long long ldx,
                        const float* __restrict__ g, const float* __restrict__ c,
                        __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo,
                        float eps) {
    __shared__ float red[32];
    pdl_trigger();
    const int col = 4 * threadIdx.x;
    const bool live = col < n;
    float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f), gg = v, cc = v;
    if (live) {  // the parameters before waiting for X's producer
        gg = ld4(g + col);
        cc = ld4(c + col);
    }
    pdl_wait();
    if (live) v = ld4(X + (size_t)blockIdx.x * ldx + col);
    float mean, rstd;
    cta_row_stats(v, live, n, eps, red, &mean, &rstd);
    if (!live) return;
    const float4 y = make_float4(__fmul_rn(__fmul_rn(v.x - mean, rstd), gg.x) + cc.x,
                                 __fmul_rn(__fmul_rn(v.y - mean, rstd), gg.y) + cc.y,
                                 __fmul_rn(__fmul_rn(v.z - mean, rstd), gg.z) + cc.z,
                                 __fmul_rn(__fmul_rn(v.w - mean, rstd), gg.w) + cc.w);
    store_split4(hi, lo, (long long)blockIdx.x * n + col, y);
}

// gate_kernel's work for groups of 8 channels, one thread per (sequence,
// group): every element's arithmetic exactly as gate_kernel writes it
__global__ void __launch_bounds__(256)
    gate8_kernel(int B, int D, int L, int layer, const float* __restrict__ q,
                 const float* __restrict__ delta, float* __restrict__ s, float* __restrict__ u,
                 float* __restrict__ gate_out, int clamp, float p_floor,
                 __nv_bfloat16* __restrict__ uh, __nv_bfloat16* __restrict__ ul) {
    pdl_trigger();
    const int ng = D >> 3;
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    const bool live = i < (long long)B * ng;
    const int b = live ? (int)(i / ng) : 0, d0 = live ? (int)(i - (long long)b * ng) * 8 : 0;
    const float* qb = q + (size_t)b * 2 * D;
    float* sp = s + ((size_t)b * L + layer) * D + d0;
    // before waiting for U: delta, and this layer's state (written only by
    // this layer's gate, in earlier steps)
    float4 e0, e1, s0, s1;
    if (live) {
        e0 = ld4(delta + d0), e1 = ld4(delta + d0 + 4);
        s0 = ld4(sp), s1 = ld4(sp + 4);
    }
    pdl_wait();
    if (!live) return;
    const float4 a0 = ld4(qb + d0), a1 = ld4(qb + d0 + 4);
    const float4 g0 = ld4(qb + D + d0), g1 = ld4(qb + D + d0 + 4);
    const float ur[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    const float gt[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
    const float dl[8] = {e0.x, e0.y, e0.z, e0.w, e1.x, e1.y, e1.z, e1.w};
    const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    float uo[8], so[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const float gk = gt[k], gk1 = gt[(k + 1) & 7], gk2 = gt[(k + 2) & 7];
        const float uu = ur[k] * (sigm(gk - gk1) * sigm(gk - gk2));
        float p = 1.0f - dl[k] * (1.0f - sigm(gk));
        if (clamp && p < p_floor) p = p_floor;
        so[k] = p * sv[k] + (1.0f - p) * uu;
        uo[k] = uu;
    }
    st4(sp, make_float4(so[0], so[1], so[2], so[3]));
    st4(sp + 4, make_float4(so[4], so[5], so[6], so[7]));
    const size_t o = (size_t)b * D + d0;
    const float4 u0 = make_float4(uo[0], uo[1], uo[2], uo[3]);
    const float4 u1 = make_float4(uo[4], uo[5], uo[6], uo[7]);
    st4(u + o, u0);
    st4(u + o + 4, u1);
    if (uh) {
        store_split4(uh, ul, (long long)o, u0);
        store_split4(uh, ul, (long long)o + 4, u1);
    }
    if (gate_out) {
        st4(gate_out + o, g0);
        st4(gate_out + o + 4, g1);
    }
}

bool al16(const void* p) { return ((uintptr_t)p & 15) == 0; }
bool al8(const void* p) { return ((uintptr_t)p & 7) == 0; }

// threads of a row kernel for a row of n floats (0: the float4 kernels do not apply)
int row_threads(int n) {
    if (n <= 0 || n % 4 || n / 4 > kRowMaxThreads) return 0;
    return (n / 4 + 31) / 32 * 32;
}

// LN + causal taps + ring write of layer `layer` for B sequences (`pdl`:
// launched with programmatic serialization after the previous kernel).
int launch_prep(bool pdl, cudaStream_t st, int B, int D, int K, int KH, int layer, int L,
                const int32_t* tok, int vocab, const float* embed, float* x, float* raw_out,
                float* at, float* hist, int32_t* pos, const float* g, const float* c,
                const float* dw, float eps, __nv_bfloat16* ath, __nv_bfloat16* atl) {
    const int nt = row_threads(D);
    const bool vec = nt && al16(x) && al16(at) && al16(hist) && al16(embed) && al16(g) &&
                     al16(c) && al16(dw) && (!raw_out || al16(raw_out)) &&
                     (!ath || (al8(ath) && al8(atl)));
    if (vec)
        return cuda_check(launch_pdl_if(pdl, prep_vec_kernel, dim3(B), dim3(nt), 0, st, D, K, KH,
                                        layer, L, tok, vocab, rt().d_err, embed, x, raw_out, at,
                                        hist, pos, g, c, dw, eps, ath, atl),
                          "prep launch");
    return cuda_check(launch_pdl_if(pdl, prep_kernel, dim3(B), dim3(256), 0, st, D, K, KH, layer,
                                    L, tok, vocab, rt().d_err, embed, x, raw_out, at, hist, pos,
                                    g, c, dw, eps, ath, atl),
                      "prep launch");
}

// competition gate + decay gate + state update of layer `layer`
int launch_gate(bool pdl, cudaStream_t st, int B, int D, int G, int L, int layer, const float* q,
                const float* delta, float* s, float* u, float* gate_out, int clamp, float p_floor,
                __nv_bfloat16* uh, __nv_bfloat16* ul) {
    const bool g8 = G == 8 && D % 8 == 0 && al16(q) && al16(delta) && al16(s) && al16(u) &&
                    (!gate_out || al16(gate_out)) && (!uh || (al8(uh) && al8(ul)));
    if (g8)
        return cuda_check(launch_pdl_if(pdl, gate8_kernel,
                                        dim3((unsigned)(((long long)B * (D / 8) + 255) / 256)),
                                        dim3(256), 0, st, B, D, L, layer, q, delta, s, u, gate_out,
                                        clamp, p_floor, uh, ul),
                          "gate launch");
    return cuda_check(launch_pdl_if(pdl, gate_kernel,
                                    dim3((unsigned)(((long long)B * D + 255) / 256)), dim3(256), 0,
                                    st, B, D, G, L, layer, q, delta, s, u, gate_out, clamp,
                                    p_floor, uh, ul),
                      "gate launch");
}

bool rows_ok(int n, const float* X, long long ldx) { return row_threads(n) && al16(X) && ldx % 4 == 0; }

// row mean / rstd of `rows` rows of n floats, ldx apart
int launch_rowstats(bool pdl, cudaStream_t st, int rows, int n, const float* X, long long ldx,
                    float* mu, float* rs, float eps) {
    if (rows_ok(n, X, ldx))
        return cuda_check(launch_pdl_if(pdl, rowstats_vec_kernel, dim3((unsigned)rows),
                                        dim3(row_threads(n)), 0, st, n, X, ldx, mu, rs, eps),
                          "rowstats launch");
    return cuda_check(launch_pdl_if(pdl, rowstats_kernel, dim3((unsigned)rows), dim3(256), 0, st,
                                    n, X, ldx, mu, rs, eps),
                      "rowstats launch");
}

// row LN written as the bf16 planes of the next contraction's input
int launch_ln_split(bool pdl, cudaStream_t st, int rows, int n, const float* X, long long ldx,
                    const float* g, const float* c, __nv_bfloat16* hi, __nv_bfloat16* lo,
                    float eps) {
    if (rows_ok(n, X, ldx) && al16(g) && al16(c) && al8(hi) && al8(lo))
        return cuda_check(launch_pdl_if(pdl, ln_split_vec_kernel, dim3((unsigned)rows),
                                        dim3(row_threads(n)), 0, st, n, X, ldx, g, c, hi, lo, eps),
                          "ln_split launch");
    return cuda_check(launch_pdl_if(pdl, ln_split_kernel, dim3((unsigned)rows), dim3(256), 0, st,
                                    n, X, ldx, g, c, hi, lo, eps),
                      "ln_split launch");
}

// y = LN(z) materialised (debug dumps only).
__global__ void apply_ln_kernel(int n, const float* __restrict__ z, const float* __restrict__ mu,
                                const float* __restrict__ rs, const float* __restrict__ g,
                                const float* __restrict__ c, float* __restrict__ y) {
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        y[(size_t)blockIdx.x * n + i] = (z[(size_t)blockIdx.x * n + i] - mu[blockIdx.x]) *
                                            rs[blockIdx.x] * g[i] + c[i];
}


// (in,out) -> (out,in)
__global__ void transpose_kernel(const float* __restrict__ src, float* __restrict__ dst, int in,
                                 int out) {
    __shared__ float t[32][33];
    const int bx = blockIdx.x * 32, by = blockIdx.y * 32;  // bx over out, by over in
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

__global__ void f32_to_f16_kernel(const float* __restrict__ s, __half* __restrict__ d, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        d[i] = __float2half_rn(s[i]);
}

// ---------------------------------------------------------- chunked prefill
// x[m] = embed[tok[m]] for the M = B*Tc rows of a chunk.
__global__ void gather_embed_kernel(int D, int vocab, int* __restrict__ err,
                                    const int32_t* __restrict__ tok,
                                    const float* __restrict__ embed, float* __restrict__ x) {
    int t = tok[blockIdx.x];
    if (t < 0 || t >= vocab) {
        if (threadIdx.x == 0) atomicExch(err, kErrBadIndex);
        t = 0;
    }
    const float* e = embed + (size_t)t * D;
    float* xr = x + (size_t)blockIdx.x * D;
    for (int i = threadIdx.x; i < D; i += blockDim.x) xr[i] = e[i];
}

// Y[m] = LN(X[m]) per row
__global__ void ln_rows_kernel(int n, const float* __restrict__ X, float* __restrict__ Y,
                               const float* __restrict__ g, const float* __restrict__ c,
                               float eps) {
    __shared__ float red[32];
    const float* xr = X + (size_t)blockIdx.x * n;
    float s = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s += xr[i];
    const float mean = block_sum(s, red) / (float)n;
    float v = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float d = xr[i] - mean;
        v += d * d;
    }
    const float rstd = 1.0f / sqrtf(block_sum(v, red) / (float)n + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        Y[(size_t)blockIdx.x * n + i] = (xr[i] - mean) * rstd * g[i] + c[i];
}

// Causal taps over a chunk: position t of sequence b reads raw rows t-1..t-K+1
// of the chunk, or the history ring for the ones before the chunk.
// With hi / lo, the taps are written only as the bf16 planes of the next
// contraction's input (the values split_act_kernel would make from at).
__global__ void conv_chunk_kernel(int B, int Tc, int D, int K, int KH, int L, int layer,
                                  const float* __restrict__ raw, const float* __restrict__ hist,
                                  const int32_t* __restrict__ pos, const float* __restrict__ dw,
                                  float* __restrict__ at, __nv_bfloat16* __restrict__ hi = nullptr,
                                  __nv_bfloat16* __restrict__ lo = nullptr) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= (long long)B * Tc * D) return;
    const int d = (int)(i % D);
    const long long m = i / D;
    const int t = (int)(m % Tc), b = (int)(m / Tc);
    const float r = raw[i];
    float a = r;
    if (K > 1) {
        const int p = pos[b * L + layer];
        const float* hb = hist + ((size_t)b * L + layer) * KH * D;
        float acc = r * dw[(size_t)(K - 1) * D + d];
        for (int k = 0; k < K - 1; ++k) {
            const int tt = t - 1 - k;
            const float hv = tt >= 0 ? raw[(m - 1 - k) * D + d]
                                     : hb[(size_t)(((p + tt) % KH + KH) % KH) * D + d];
            acc += hv * dw[(size_t)(K - 2 - k) * D + d];
        }
        a = r + acc;
    }
    if (hi) store_split(hi, lo, i, a);
    else at[i] = a;
}

// ring_update_kernel with float4 copies (D % 4 == 0, 16-byte aligned rows),
// launched with enough threads that each copies about one vector.
__global__ void ring_update4_kernel(int Tc, int D, int KH, int L, int layer,
                                    const float* __restrict__ raw, float* __restrict__ hist,
                                    int32_t* __restrict__ pos) {
    const int b = blockIdx.x;
    const int p = pos[b * L + layer];
    __syncthreads();
    float* hb = hist + ((size_t)b * L + layer) * KH * D;
    const int first = Tc > KH ? Tc - KH : 0, D4 = D >> 2;
    for (int i = threadIdx.x; i < (Tc - first) * D4; i += blockDim.x) {
        const int t = first + i / D4, d = (i % D4) * 4;
        *reinterpret_cast<float4*>(hb + (size_t)(((p + t) % KH + KH) % KH) * D + d) =
            *reinterpret_cast<const float4*>(raw + ((size_t)b * Tc + t) * D + d);
    }
    __syncthreads();
    if (threadIdx.x == 0) pos[b * L + layer] = p + Tc;
}

// conv_chunk_kernel for four consecutive channels per thread (D % 4 == 0,
// 16-byte aligned rows), writing the taps only as bf16 planes; the same
// arithmetic per channel.
__global__ void conv_chunk4_kernel(int B, int Tc, int D, int K, int KH, int L, int layer,
                                   const float* __restrict__ raw, const float* __restrict__ hist,
                                   const int32_t* __restrict__ pos, const float* __restrict__ dw,
                                   __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo) {
    const int D4 = D >> 2;
    const long long i4 = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i4 >= (long long)B * Tc * D4) return;
    const int d = (int)(i4 % D4) * 4;
    const long long m = i4 / D4;
    const int t = (int)(m % Tc), b = (int)(m / Tc);
    const float4 r4 = *reinterpret_cast<const float4*>(raw + m * D + d);
    const float r[4] = {r4.x, r4.y, r4.z, r4.w};
    float a[4] = {r[0], r[1], r[2], r[3]};
    if (K > 1) {
        const int p = pos[b * L + layer];
        const float* hb = hist + ((size_t)b * L + layer) * KH * D;
        const float4 w4 = *reinterpret_cast<const float4*>(dw + (size_t)(K - 1) * D + d);
        const float w[4] = {w4.x, w4.y, w4.z, w4.w};
        float acc[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[j] = r[j] * w[j];
        for (int k = 0; k < K - 1; ++k) {
            const int tt = t - 1 - k;
            const float* src = tt >= 0 ? raw + (m - 1 - k) * D + d
                                       : hb + (size_t)(((p + tt) % KH + KH) % KH) * D + d;
            const float4 h4 = *reinterpret_cast<const float4*>(src);
            const float4 k4 = *reinterpret_cast<const float4*>(dw + (size_t)(K - 2 - k) * D + d);
            const float hv[4] = {h4.x, h4.y, h4.z, h4.w}, wk[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[j] += hv[j] * wk[j];
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) a[j] = r[j] + acc[j];
    }
    __nv_bfloat16 h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {  // store_split's rounding
        h[j] = __float2bfloat16_rn(a[j]);
        l[j] = __float2bfloat16_rn(a[j] - __bfloat162float(h[j]));
    }
    *reinterpret_cast<uint2*>(hi + m * D + d) = *reinterpret_cast<const uint2*>(h);
    *reinterpret_cast<uint2*>(lo + m * D + d) = *reinterpret_cast<const uint2*>(l);
}

// After the taps of a chunk: the last K-1 raw rows of each sequence enter the
// ring and the position advances by Tc. One CTA per sequence.
__global__ void ring_update_kernel(int Tc, int D, int KH, int L, int layer,
                                   const float* __restrict__ raw, float* __restrict__ hist,
                                   int32_t* __restrict__ pos) {
    const int b = blockIdx.x;
    const int p = pos[b * L + layer];
    __syncthreads();
    float* hb = hist + ((size_t)b * L + layer) * KH * D;
    const int first = Tc > KH ? Tc - KH : 0;
    for (int i = threadIdx.x; i < (Tc - first) * D; i += blockDim.x) {
        const int t = first + i / D, d = i % D;
        hb[(size_t)(((p + t) % KH + KH) % KH) * D + d] = raw[((size_t)b * Tc + t) * D + d];
    }
    __syncthreads();
    if (threadIdx.x == 0) pos[b * L + layer] = p + Tc;
}

// u = compete(q), p = decay gate (the scan's a), one thread per (row, channel)
// (with uh / ul also the bf16 planes of u, the input of the Wz contraction)
__global__ void gate_chunk_kernel(long long M, int D, int G, const float* __restrict__ q,
                                  const float* __restrict__ delta, float* __restrict__ u,
                                  float* __restrict__ pa, int clamp, float p_floor,
                                  __nv_bfloat16* __restrict__ uh = nullptr,
                                  __nv_bfloat16* __restrict__ ul = nullptr) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= M * D) return;
    const long long m = i / D;
    const int d = (int)(i % D);
    const float* qb = q + m * 2 * D;
    const int base = (d / G) * G, off = d - base;
    const float g0 = qb[D + d];
    const float g1 = qb[D + base + (off + 1) % G];
    const float g2 = qb[D + base + (off + 2) % G];
    const float uu = qb[d] * (sigm(g0 - g1) * sigm(g0 - g2));
    u[i] = uu;
    if (uh) store_split(uh, ul, i, uu);
    float p = 1.0f - delta[d] * (1.0f - sigm(g0));
    if (clamp && p < p_floor) p = p_floor;
    pa[i] = p;
}

// gate_chunk_kernel with one thread per competition group of G channels
// (G = 4 or 8, D % G == 0, 16-byte aligned rows): the group's u and gate
// inputs read as float4s, u, p and u's bf16 planes written as vectors; the
// same arithmetic per channel.
template <int G>
__global__ void gate_group_kernel(long long M, int D, const float* __restrict__ q,
                                  const float* __restrict__ delta, float* __restrict__ u,
                                  float* __restrict__ pa, int clamp, float p_floor,
                                  __nv_bfloat16* __restrict__ uh, __nv_bfloat16* __restrict__ ul) {
    const int ng = D / G;
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= M * ng) return;
    const long long m = i / ng;
    const int base = (int)(i % ng) * G;
    const float* qb = q + m * 2 * D;
    float qv[G], gq[G], dl[G];
#pragma unroll
    for (int j = 0; j < G; j += 4) {
        const float4 a = *reinterpret_cast<const float4*>(qb + base + j);
        const float4 g = *reinterpret_cast<const float4*>(qb + D + base + j);
        const float4 e = *reinterpret_cast<const float4*>(delta + base + j);
        qv[j] = a.x, qv[j + 1] = a.y, qv[j + 2] = a.z, qv[j + 3] = a.w;
        gq[j] = g.x, gq[j + 1] = g.y, gq[j + 2] = g.z, gq[j + 3] = g.w;
        dl[j] = e.x, dl[j + 1] = e.y, dl[j + 2] = e.z, dl[j + 3] = e.w;
    }
    float uu[G], pp[G];
#pragma unroll
    for (int off = 0; off < G; ++off) {
        const float g0 = gq[off], g1 = gq[(off + 1) % G], g2 = gq[(off + 2) % G];
        uu[off] = qv[off] * (sigm(g0 - g1) * sigm(g0 - g2));
        float p = 1.0f - dl[off] * (1.0f - sigm(g0));
        if (clamp && p < p_floor) p = p_floor;
        pp[off] = p;
    }
    const long long o = m * D + base;
#pragma unroll
    for (int j = 0; j < G; j += 4) {
        *reinterpret_cast<float4*>(u + o + j) = make_float4(uu[j], uu[j + 1], uu[j + 2], uu[j + 3]);
        *reinterpret_cast<float4*>(pa + o + j) = make_float4(pp[j], pp[j + 1], pp[j + 2], pp[j + 3]);
    }
    if (uh) {
        __nv_bfloat16 h[G], l[G];
#pragma unroll
        for (int j = 0; j < G; ++j) {  // store_split's rounding
            h[j] = __float2bfloat16_rn(uu[j]);
            l[j] = __float2bfloat16_rn(uu[j] - __bfloat162float(h[j]));
        }
#pragma unroll
        for (int j = 0; j < G; j += 4) {
            *reinterpret_cast<uint2*>(uh + o + j) = *reinterpret_cast<const uint2*>(h + j);
            *reinterpret_cast<uint2*>(ul + o + j) = *reinterpret_cast<const uint2*>(l + j);
        }
    }
}

// prev[b][t] = state before position t: s_in for t = 0, else states[b][t-1]
__global__ void prev_kernel(int Tc, int D, long long total, const float* __restrict__ s0,
                            const float* __restrict__ st, float* __restrict__ prev) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= total) return;
    const int d = (int)(i % D);
    const long long m = i / D;
    const int t = (int)(m % Tc);
    const long long b = m / Tc;
    prev[i] = t == 0 ? s0[b * D + d] : st[i - D];
}

// state export / import: ring <-> newest-first history
__global__ void hist_io_kernel(int B, int L, int KH, int D, float* ring, float* flat,
                               int32_t* pos, int to_flat) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    const long long total = (long long)B * L * KH * D;
    if (i >= total) return;
    const int d = (int)(i % D);
    const int k = (int)((i / D) % KH);
    const long long bl = i / ((long long)KH * D);
    const int p = to_flat ? pos[bl] : 0;  // pos is [seq][layer], bl = seq*L + layer
    const int slot = ((p - 1 - k) % KH + KH) % KH;
    float* r = ring + (bl * KH + slot) * D + d;
    if (to_flat) flat[i] = *r;
    else *r = flat[i];
}

}  // namespace

struct SunnyLayer {
    float *ni_g, *ni_c, *nm_g, *nm_c, *dw, *delta;
    void *V, *U, *Wz, *Wc, *Ws;
    float *sV, *sU, *sWz, *sWc, *sWs;  // int8 row scales
    float a_tanh, b_gain;
    TcWeights tV, tU, tWz, tWc, tWs;   // bf16 planes + TMA maps for the batched path
};

struct SunnyModel {
    int vocab = 0, D = 0, I = 0, R = 0, K = 0, L = 0, G = 0, clamp = 0, nseq = 0, KH = 1;
    int wtype = kWF32;
    float eps = 0, p_floor = 0;
    std::vector<SunnyLayer> ly;
    float *no_g = nullptr, *no_c = nullptr, *embed = nullptr;
    void* head = nullptr;
    float* shead = nullptr;
    TcWeights thead;
    std::vector<void*> allocs;
    // state
    float* s = nullptr;
    float* hist = nullptr;
    int32_t* pos = nullptr;
    // activations (nseq rows)
    int32_t* tok = nullptr;
    int32_t* next = nullptr;
    float *x = nullptr, *at = nullptr, *raw = nullptr, *v = nullptr, *q = nullptr, *u = nullptr;
    float *gate = nullptr, *sfb = nullptr, *z = nullptr, *mu = nullptr, *rs = nullptr;
    float *logits = nullptr, *yn = nullptr;
    float2* apart = nullptr;  // argmax partials (B x kArgChunks)
    // tensor-core step (B >= 16): bf16 planes of each contraction's input,
    // the per-layer state feedback sfb of all layers, and the side stream the
    // feedback contractions run on (with its fork / join events)
    bool tc_step = false;
    TcAct p_at, p_v, p_u, p_z, p_x, p_s;
    std::vector<TcAct> p_sl;  // layer l's rows of p_s
    float* sfb_all = nullptr;  // [L][nseq][D]
    cudaStream_t side = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_split = nullptr;
    std::vector<cudaEvent_t> ev_ws;
    std::map<std::pair<int, int>, cudaGraphExec_t> graphs;  // (B, with head) -> graph
    // chunked prefill: buffers of B*Tc rows, one graph per (B, Tc, head)
    long long crows = 0;
    int cseqs = 0;
    int32_t* ctok = nullptr;
    float *cx = nullptr, *craw = nullptr, *cat = nullptr, *cv = nullptr, *cq = nullptr;
    float *cu = nullptr, *cp = nullptr, *cst = nullptr, *cprev = nullptr, *csfb = nullptr;
    float *cz = nullptr, *cmu = nullptr, *crs = nullptr, *cs0 = nullptr, *csend = nullptr;
    // tensor-core prefill: each contraction's input written as bf16 planes by
    // its producer (taps, V's epilogue, the gate, the state shift, the LN of z)
    bool c_tc = false;
    TcAct c_at, c_v, c_u, c_prev, c_z;
    std::map<std::pair<long long, int>, cudaGraphExec_t> cgraphs;  // (B*65536+Tc, head)
    std::map<std::pair<long long, int>, ProfGraph> pgraphs;  // instrumented (profile mode 2)
    cudaStream_t cap = nullptr;
    // fused small-batch step (sunny_fused.cu): per-layer descriptors on the
    // device, barrier words, and the arguments common to every launch
    FusedLayer* dlayers = nullptr;
    unsigned* fbar = nullptr;
    unsigned long long* ftrace = nullptr;  // profile mode: phase timestamps
    FusedArgs fbase;
    bool ready = false;

    ~SunnyModel() {
        for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
        for (auto& kv : cgraphs) cudaGraphExecDestroy(kv.second);
        if (cap) cudaStreamDestroy(cap);
        if (side) cudaStreamDestroy(side);
        if (ev_fork) cudaEventDestroy(ev_fork);
        if (ev_split) cudaEventDestroy(ev_split);
        for (cudaEvent_t e : ev_ws) cudaEventDestroy(e);
        for (void* p : allocs) cudaFree(p);
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

struct BlobReader {
    FILE* f = nullptr;
    bool ok = true;
    explicit BlobReader(const char* path) : f(fopen(path, "rb")) { ok = f != nullptr; }
    ~BlobReader() {
        if (f) fclose(f);
    }
    bool read(void* dst, size_t n) {
        if (ok && fread(dst, 1, n, f) != n) ok = false;
        return ok;
    }
};

// Upload helpers (host staging buffer reused).
struct Uploader {
    SunnyModel* m;
    BlobReader* br;
    std::vector<unsigned char> host;
    float* tmp = nullptr;  // device scratch for transposes
    size_t tmp_n = 0;
    int rc = SN_OK;

    float* vec(size_t n) {
        float* d = m->dalloc<float>(n);
        host.resize(n * 4);
        if (!d) {
            rc = SN_E_NOMEM;
            return nullptr;
        }
        if (!br->read(host.data(), n * 4)) {
            rc = SN_E_IO;
            return nullptr;
        }
        if (cudaMemcpy(d, host.data(), n * 4, cudaMemcpyHostToDevice) != cudaSuccess) rc = SN_E_DEVICE;
        return d;
    }

    // fp32 (in,out) block -> (out,in) fp32 or fp16 on device
    void* mat_f32(int in, int out, bool half) {
        const size_t n = (size_t)in * out;
        if (tmp_n < n) {
            if (tmp) cudaFree(tmp);
            if (cudaMalloc(&tmp, n * 4) != cudaSuccess) {
                cudaGetLastError();
                rc = SN_E_NOMEM;
                tmp = nullptr;
                tmp_n = 0;
                return nullptr;
            }
            tmp_n = n;
        }
        host.resize(n * 4);
        if (!br->read(host.data(), n * 4)) {
            rc = SN_E_IO;
            return nullptr;
        }
        if (cudaMemcpy(tmp, host.data(), n * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
            rc = SN_E_DEVICE;
            return nullptr;
        }
        float* d = m->dalloc<float>(n);
        if (!d) {
            rc = SN_E_NOMEM;
            return nullptr;
        }
        dim3 grid((out + 31) / 32, (in + 31) / 32);
        transpose_kernel<<<grid, dim3(32, 8)>>>(tmp, d, in, out);
        if (!half) return d;
        __half* h = m->dalloc<__half>(n);
        if (!h) {
            rc = SN_E_NOMEM;
            return nullptr;
        }
        f32_to_f16_kernel<<<grid_blocks((long long)n), 256>>>(d, h, (long long)n);
        return h;
    }

    // int8 (out,in) codes + fp32 row scales
    void* mat_i8(int in, int out, float** scale) {
        const size_t n = (size_t)in * out;
        int8_t* d = m->dalloc<int8_t>(n);
        if (!d) {
            rc = SN_E_NOMEM;
            return nullptr;
        }
        host.resize(n);
        if (!br->read(host.data(), n)) {
            rc = SN_E_IO;
            return nullptr;
        }
        if (cudaMemcpy(d, host.data(), n, cudaMemcpyHostToDevice) != cudaSuccess) rc = SN_E_DEVICE;
        *scale = vec((size_t)out);
        return d;
    }
};

int load_model(SunnyModel* m, const char* path, int nseq, bool half, const int* want) {
    BlobReader br(path);
    if (!br.ok) return fail(SN_E_IO, "cannot open %s", path);
    int32_t h[12];
    if (!br.read(h, 40)) return fail(SN_E_FORMAT, "%s: truncated header", path);
    bool quant = false;
    int vocab, D, I, R, K, L, G, tied, clamp;
    if (h[0] == kUSNN) {
        vocab = h[1]; D = h[2]; I = h[3]; R = h[4]; K = h[5]; L = h[6]; G = h[7]; tied = h[8];
        clamp = h[9];
    } else if (h[0] == kUSNQ) {
        if (!br.read(h + 10, 8) || h[1] != 1 || h[11] != 8)
            return fail(SN_E_FORMAT, "%s: unsupported USNQ version", path);
        quant = true;
        vocab = h[2]; D = h[3]; I = h[4]; R = h[5]; K = h[6]; L = h[7]; G = h[8]; tied = h[9];
        clamp = h[10];
    } else {
        return fail(SN_E_FORMAT, "%s: bad magic 0x%08x", path, (unsigned)h[0]);
    }
    if (want) {  // sn_load: caller dims must match the header (sunnynet.c:363-368)
        const int got[8] = {vocab, D, I, R, K, L, G, tied};
        for (int i = 0; i < 8; ++i)
            if (got[i] != want[i]) return fail(SN_E_FORMAT, "%s: header/dims mismatch", path);
    }
    if (vocab <= 0 || D <= 0 || I <= 0 || R <= 0 || K <= 0 || L <= 0 || G < 3 || D % G)
        return fail(SN_E_FORMAT, "%s: invalid dims", path);
    if (half && quant) return fail(SN_E_UNSUPPORTED, "fp16 load of an INT8 blob");
    SN_TRY(ensure_init());
    m->vocab = vocab; m->D = D; m->I = I; m->R = R; m->K = K; m->L = L; m->G = G;
    m->clamp = clamp; m->nseq = nseq; m->KH = K > 1 ? K - 1 : 1;
    m->wtype = quant ? kWI8 : (half ? kWF16 : kWF32);
    Uploader up{m, &br};
    m->ly.resize(L);
    for (int l = 0; l < L && up.rc == SN_OK; ++l) {
        SunnyLayer& y = m->ly[l];
        memset(&y, 0, sizeof y);
        y.ni_g = up.vec(D); y.ni_c = up.vec(D); y.nm_g = up.vec(I); y.nm_c = up.vec(I);
        y.dw = up.vec((size_t)K * D);
        if (quant) {
            y.V = up.mat_i8(D, R, &y.sV);
            y.U = up.mat_i8(R, 2 * D, &y.sU);
            y.Wz = up.mat_i8(D, I, &y.sWz);
            y.Wc = up.mat_i8(I, D, &y.sWc);
            y.Ws = up.mat_i8(D, D, &y.sWs);
        } else {
            y.V = up.mat_f32(D, R, half);
            y.U = up.mat_f32(R, 2 * D, half);
            y.Wz = up.mat_f32(D, I, half);
            y.Wc = up.mat_f32(I, D, half);
            y.Ws = up.mat_f32(D, D, half);
        }
        y.delta = up.vec(D);
        float sc2[2];
        if (!br.read(sc2, 8)) up.rc = SN_E_IO;
        y.a_tanh = sc2[0];
        y.b_gain = sc2[1];
    }
    float ep[2] = {0, 0};
    if (up.rc == SN_OK && !br.read(ep, 8)) up.rc = SN_E_IO;
    if (up.rc == SN_OK) {
        m->no_g = up.vec(D);
        m->no_c = up.vec(D);
        m->embed = up.vec((size_t)vocab * D);
        m->head = quant ? up.mat_i8(D, vocab, &m->shead) : up.mat_f32(D, vocab, half);
    }
    if (up.tmp) cudaFree(up.tmp);
    if (up.rc != SN_OK) return fail(up.rc == SN_E_IO ? SN_E_FORMAT : up.rc, "%s: load failed", path);
    if (!getenv("SN_DISABLE_TC")) {  // bf16 hi/lo planes for the tensor-core path (B >= 16)
        auto al = [](size_t n, void* o) -> void* { return ((SunnyModel*)o)->dalloc<uint8_t>(n); };
        for (int l = 0; l < L; ++l) {
            SunnyLayer& y = m->ly[l];
            SN_TRY(tc_prepare(&y.tV, y.V, m->wtype, R, D, al, m));
            SN_TRY(tc_prepare(&y.tU, y.U, m->wtype, 2 * D, R, al, m));
            SN_TRY(tc_prepare(&y.tWz, y.Wz, m->wtype, I, D, al, m));
            SN_TRY(tc_prepare(&y.tWc, y.Wc, m->wtype, D, I, al, m));
            SN_TRY(tc_prepare(&y.tWs, y.Ws, m->wtype, D, D, al, m));
        }
        SN_TRY(tc_prepare(&m->thead, m->head, m->wtype, vocab, D, al, m));
        if (nseq >= 16) {
            SN_TRY(tc_reserve(D, nseq));
            SN_TRY(tc_reserve(R, nseq));
            SN_TRY(tc_reserve(I, nseq));
        }
    }
    m->eps = ep[0];
    m->p_floor = ep[1];
    const size_t n = (size_t)nseq;
    m->s = m->dalloc<float>(n * L * D);
    m->hist = m->dalloc<float>(n * L * m->KH * D);
    m->pos = m->dalloc<int32_t>(n * L);
    m->tok = m->dalloc<int32_t>(n);
    m->next = m->dalloc<int32_t>(n);
    m->x = m->dalloc<float>(n * D);
    m->at = m->dalloc<float>(n * D);
    m->raw = m->dalloc<float>(n * D);
    m->v = m->dalloc<float>(n * R);
    m->q = m->dalloc<float>(n * 2 * D);
    m->u = m->dalloc<float>(n * D);
    m->gate = m->dalloc<float>(n * D);
    m->sfb = m->dalloc<float>(n * D);
    m->z = m->dalloc<float>(n * I);
    m->yn = m->dalloc<float>(n * I);
    m->mu = m->dalloc<float>(n);
    m->rs = m->dalloc<float>(n);
    m->logits = m->dalloc<float>(n * vocab);
    m->apart = m->dalloc<float2>(n * kArgChunks);
    if (!m->logits || !m->rs || !m->apart) return fail(SN_E_NOMEM, "device allocation failed");
    SN_TRY(cuda_check(cudaStreamCreateWithFlags(&m->cap, cudaStreamNonBlocking), "stream"));
    bool tc_all = nseq >= 16 && m->thead.ready && D % 8 == 0 && R % 8 == 0 && I % 8 == 0;
    for (int l = 0; l < L && tc_all; ++l) {
        const SunnyLayer& y = m->ly[l];
        tc_all = y.tV.ready && y.tU.ready && y.tWz.ready && y.tWc.ready && y.tWs.ready;
    }
    if (tc_all) {
        auto al = [](size_t nb, void* o) -> void* { return ((SunnyModel*)o)->dalloc<uint8_t>(nb); };
        SN_TRY(tc_act_alloc(&m->p_at, D, nseq, al, m));
        SN_TRY(tc_act_alloc(&m->p_v, R, nseq, al, m));
        SN_TRY(tc_act_alloc(&m->p_u, D, nseq, al, m));
        SN_TRY(tc_act_alloc(&m->p_z, I, nseq, al, m));
        SN_TRY(tc_act_alloc(&m->p_x, D, nseq, al, m));
        SN_TRY(tc_act_alloc(&m->p_s, D, n * L, al, m));
        m->p_sl.resize(L);
        for (int l = 0; l < L; ++l)
            SN_TRY(tc_act_view(&m->p_sl[l], m->p_s, (long long)l * D, nseq, (long long)L * D, D));
        m->sfb_all = m->dalloc<float>(n * L * D);
        if (!m->sfb_all) return fail(SN_E_NOMEM, "device allocation failed");
        // the feedback contractions' side stream at the lowest priority, the
        // captured layer chain at the highest: where both have CTAs waiting,
        // the chain's go first
        int lo = 0, hi = 0;
        SN_TRY(cuda_check(cudaDeviceGetStreamPriorityRange(&lo, &hi), "priorities"));
        SN_TRY(cuda_check(cudaStreamCreateWithPriority(&m->side, cudaStreamNonBlocking, lo),
                          "stream"));
        SN_TRY(cuda_check(cudaStreamDestroy(m->cap), "stream"));
        m->cap = nullptr;
        SN_TRY(cuda_check(cudaStreamCreateWithPriority(&m->cap, cudaStreamNonBlocking, hi),
                          "stream"));
        SN_TRY(cuda_check(cudaEventCreateWithFlags(&m->ev_fork, cudaEventDisableTiming), "event"));
        SN_TRY(cuda_check(cudaEventCreateWithFlags(&m->ev_split, cudaEventDisableTiming), "event"));
        m->ev_ws.assign(L, nullptr);
        for (int l = 0; l < L; ++l)
            SN_TRY(cuda_check(cudaEventCreateWithFlags(&m->ev_ws[l], cudaEventDisableTiming),
                              "event"));
        m->tc_step = !getenv("SN_TC_SPLIT_STEP");
    }
    cudaMemset(m->s, 0, n * L * D * 4);
    cudaMemset(m->hist, 0, n * L * m->KH * D * 4);
    cudaMemset(m->pos, 0, n * L * 4);
    {   // fused small-batch step: layer descriptors and barrier words
        std::vector<FusedLayer> fl(L);
        for (int l = 0; l < L; ++l) {
            const SunnyLayer& y = m->ly[l];
            fl[l] = FusedLayer{y.ni_g, y.ni_c, y.nm_g, y.nm_c, y.dw, y.delta, y.V, y.U, y.Wz,
                               y.Wc, y.Ws, y.sV, y.sU, y.sWz, y.sWc, y.sWs, y.a_tanh, y.b_gain};
        }
        m->dlayers = m->dalloc<FusedLayer>(L);
        m->fbar = m->dalloc<unsigned>(kBarWords);
        m->ftrace = m->dalloc<unsigned long long>((size_t)rt().num_sms * 2 * (32 * L + 9));
        if (!m->dlayers || !m->fbar || !m->ftrace)
            return fail(SN_E_NOMEM, "device allocation failed");
        SN_TRY(cuda_check(cudaMemcpy(m->dlayers, fl.data(), L * sizeof(FusedLayer),
                                     cudaMemcpyHostToDevice),
                          "layer descriptors"));
        FusedArgs& f = m->fbase;
        f.D = D; f.I = I; f.R = R; f.K = m->K; f.KH = m->KH; f.L = L; f.G = m->G;
        f.vocab = vocab; f.clamp = m->clamp; f.wtype = m->wtype;
        f.ctas = rt().num_sms;
        f.bulk_prefetch = getenv("SN_FUSED_NO_PREFETCH") ? 0 : 1;
        f.eps = m->eps; f.p_floor = m->p_floor;
        f.layers = m->dlayers;
        f.no_g = m->no_g; f.no_c = m->no_c; f.embed = m->embed;
        f.head = m->head; f.shead = m->shead;
        f.s = m->s; f.hist = m->hist; f.pos = m->pos; f.tok = m->tok;
        f.x = m->x; f.v = m->v; f.u = m->u; f.sfb = m->sfb; f.z = m->z;
        f.logits = m->logits;
        f.bar = m->fbar;
        f.err = rt().d_err;
    }
    SN_TRY(cuda_check(cudaDeviceSynchronize(), "load"));
    m->ready = true;
    return SN_OK;
}

GemmArgs gemm(int M, int N, int K, const float* A, const void* W, const float* ws, float* C) {
    GemmArgs g;
    g.M = M; g.N = N; g.K = K;
    g.A = A; g.lda = K;
    g.W = W; g.ldw = K; g.wscale = ws;
    g.C = C; g.ldc = N;
    return g;
}

// Enqueue one decode step for sequences [0,B) (tokens already in m->tok).
// last_layer >= 0 stops after that layer and fills the debug buffers.
int enqueue_step(SunnyModel* m, int B, bool with_head, cudaStream_t st, int last_layer = -1) {
    const int D = m->D, I = m->I, R = m->R;
    const int nl = last_layer >= 0 ? last_layer + 1 : m->L;
    const bool dbg = last_layer >= 0;
    for (int l = 0; l < nl; ++l) {
        const SunnyLayer& y = m->ly[l];
        const bool this_dbg = dbg && l == last_layer;
        {
            ProfScope ps("prep_ln_taps", st);
            SN_TRY(launch_prep(false, st, B, D, m->K, m->KH, l, m->L, m->tok, m->vocab, m->embed,
                               m->x, this_dbg ? m->raw : nullptr, m->at, m->hist, m->pos,
                               y.ni_g, y.ni_c, y.dw, m->eps, nullptr, nullptr));
        }
        // feedback reads the previous state: before the gate kernel updates it
        GemmArgs gs = gemm(B, D, D, m->s + (size_t)l * D, y.Ws, y.sWs, m->sfb);
        gs.lda = (long long)m->L * D;
        {
            ProfScope ps("gemm_Ws", st);
            SN_TRY(launch_gemm(gs, m->wtype, st, &y.tWs));
        }
        {
            ProfScope ps("gemm_V", st);
            SN_TRY(launch_gemm(gemm(B, R, D, m->at, y.V, y.sV, m->v), m->wtype, st, &y.tV));
        }
        {
            ProfScope ps("gemm_U", st);
            SN_TRY(launch_gemm(gemm(B, 2 * D, R, m->v, y.U, y.sU, m->q), m->wtype, st, &y.tU));
        }
        {
            ProfScope ps("gate_state", st);
            SN_TRY(launch_gate(false, st, B, D, m->G, m->L, l, m->q, y.delta, m->s, m->u,
                               this_dbg ? m->gate : nullptr, m->clamp, m->p_floor, nullptr,
                               nullptr));
        }
        GemmArgs gz = gemm(B, I, D, m->u, y.Wz, y.sWz, m->z);
        gz.epi = kEpiWedge;
        gz.p = y.a_tanh;
        {
            ProfScope ps("gemm_Wz", st);
            SN_TRY(launch_gemm(gz, m->wtype, st, &y.tWz));
        }
        // small batches compute the LN statistics inside the GEMV (one launch less)
        const bool inline_ln = B <= 8 && !this_dbg;
        if (!inline_ln) {
            ProfScope ps("rowstats", st);
            SN_TRY(launch_rowstats(false, st, B, I, m->z, I, m->mu, m->rs, m->eps));
        }
        if (this_dbg)
            apply_ln_kernel<<<B, 256, 0, st>>>(I, m->z, m->mu, m->rs, y.nm_g, y.nm_c, m->yn);
        GemmArgs gc = gemm(B, D, I, m->z, y.Wc, y.sWc, m->x);
        gc.g = y.nm_g; gc.c = y.nm_c;
        if (inline_ln) {
            gc.ln_inline = 1;
            gc.ln_eps = m->eps;
        } else {
            gc.mu = m->mu; gc.rs = m->rs;
        }
        gc.epi = kEpiResid;
        gc.p = y.b_gain;
        gc.S = m->s + (size_t)l * D;
        gc.lds = (long long)m->L * D;
        gc.F = m->sfb; gc.ldf = D;
        gc.X = m->x; gc.ldx = D;
        {
            ProfScope ps("gemm_Wc", st);
            SN_TRY(launch_gemm(gc, m->wtype, st, &y.tWc));
        }
    }
    if (dbg) return cuda_check(cudaGetLastError(), "dbg step");
    if (with_head) {
        if (B > 8) {
            ProfScope ps("rowstats", st);
            SN_TRY(launch_rowstats(false, st, B, D, m->x, D, m->mu, m->rs, m->eps));
        }
        GemmArgs gh = gemm(B, m->vocab, D, m->x, m->head, m->shead, m->logits);
        gh.g = m->no_g; gh.c = m->no_c;
        if (B <= 8) {
            gh.ln_inline = 1;
            gh.ln_eps = m->eps;
        } else {
            gh.mu = m->mu; gh.rs = m->rs;
        }
        ProfScope ps("gemm_head", st);
        SN_TRY(launch_gemm(gh, m->wtype, st, &m->thead));
    }
    return cuda_check(cudaGetLastError(), "step launch");
}

// The batched step on the tensor cores (B >= 16, model->tc_step). Same
// arithmetic as enqueue_step, arranged for the tensor-core contractions:
//  - each contraction's input is written as bf16 planes by the kernel that
//    produces it (prep: at; V epilogue: v; gate: u; ln_split: LN(z) and the
//    final LN(x)), so no contraction needs a split launch of its own;
//  - the feedback contractions sfb_l = s_l(old) Ws_l^T read only the state
//    left by the previous step, so all L of them run on a side stream (after
//    one split of the whole state) while the layer chain runs; gate_0 waits
//    for that split (the gates overwrite the state) and Wc_l for sfb_l.
// With side == st (profile mode) everything runs in order on one stream.
int enqueue_step_tc(SunnyModel* m, int B, bool with_head, cudaStream_t st, cudaStream_t side) {
    const int D = m->D, I = m->I, R = m->R, L = m->L;
    const size_t n = (size_t)m->nseq;
    const bool fork = side != st;
    if (fork) {
        SN_TRY(cuda_check(cudaEventRecord(m->ev_fork, st), "fork"));
        SN_TRY(cuda_check(cudaStreamWaitEvent(side, m->ev_fork, 0), "fork"));
    }
    {
        ProfScope ps("split_state", side);
        SN_TRY(launch_split_rows(m->s, (long long)B * L, D, D, m->p_s, side));
    }
    if (fork) SN_TRY(cuda_check(cudaEventRecord(m->ev_split, side), "split event"));
    for (int l = 0; l < L; ++l) {
        const SunnyLayer& y = m->ly[l];
        GemmArgs gs = gemm(B, D, D, m->s + (size_t)l * D, y.Ws, y.sWs, m->sfb_all + l * n * D);
        gs.lda = (long long)L * D;
        // a sixth of the SMs: the layer chain's contractions keep the rest
        gs.max_ctas = rt().num_sms / 6;
        {
            ProfScope ps("gemm_Ws", side);
            SN_TRY(launch_tc_gemm_act(gs, y.tWs, m->p_sl[l], side));
        }
        if (fork) SN_TRY(cuda_check(cudaEventRecord(m->ev_ws[l], side), "Ws event"));
    }
    for (int l = 0; l < L; ++l) {
        const SunnyLayer& y = m->ly[l];
        {
            ProfScope ps("prep_ln_taps", st);
            // layers > 0 follow Wc of the previous layer on this stream
            SN_TRY(launch_prep(l > 0, st, B, D, m->K, m->KH, l, L, m->tok, m->vocab, m->embed,
                               m->x, nullptr, m->at, m->hist, m->pos, y.ni_g, y.ni_c, y.dw,
                               m->eps, m->p_at.hi, m->p_at.lo));
        }
        {
            GemmArgs gv = gemm(B, R, D, m->at, y.V, y.sV, m->v);
            gv.Ch = m->p_v.hi;
            gv.Cl = m->p_v.lo;
            ProfScope ps("gemm_V", st);
            SN_TRY(launch_tc_gemm_act(gv, y.tV, m->p_at, st, true));
        }
        {
            ProfScope ps("gemm_U", st);
            SN_TRY(launch_tc_gemm_act(gemm(B, 2 * D, R, m->v, y.U, y.sU, m->q), y.tU, m->p_v, st,
                                      true));
        }
        if (l == 0 && fork) SN_TRY(cuda_check(cudaStreamWaitEvent(st, m->ev_split, 0), "join"));
        {
            ProfScope ps("gate_state", st);
            // after the join (layer 0) a plain launch; later layers follow U directly
            SN_TRY(launch_gate(l > 0 || !fork, st, B, D, m->G, L, l, m->q, y.delta, m->s, m->u,
                               nullptr, m->clamp, m->p_floor, m->p_u.hi, m->p_u.lo));
        }
        {
            GemmArgs gz = gemm(B, I, D, m->u, y.Wz, y.sWz, m->z);
            gz.epi = kEpiWedge;
            gz.p = y.a_tanh;
            ProfScope ps("gemm_Wz", st);
            SN_TRY(launch_tc_gemm_act(gz, y.tWz, m->p_u, st, true));
        }
        {
            ProfScope ps("rowstats", st);
            SN_TRY(launch_ln_split(true, st, B, I, m->z, I, y.nm_g, y.nm_c, m->p_z.hi, m->p_z.lo,
                                   m->eps));
        }
        if (fork) SN_TRY(cuda_check(cudaStreamWaitEvent(st, m->ev_ws[l], 0), "join"));
        GemmArgs gc = gemm(B, D, I, m->z, y.Wc, y.sWc, m->x);
        gc.epi = kEpiResid;
        gc.p = y.b_gain;
        gc.S = m->s + (size_t)l * D;
        gc.lds = (long long)L * D;
        gc.F = m->sfb_all + l * n * D;
        gc.ldf = D;
        gc.X = m->x;
        gc.ldx = D;
        {
            ProfScope ps("gemm_Wc", st);  // after the join with sfb_l: a plain launch
            SN_TRY(launch_tc_gemm_act(gc, y.tWc, m->p_z, st, !fork));
        }
    }
    if (with_head) {
        {
            ProfScope ps("rowstats", st);
            SN_TRY(launch_ln_split(true, st, B, D, m->x, D, m->no_g, m->no_c, m->p_x.hi,
                                   m->p_x.lo, m->eps));
        }
        ProfScope ps("gemm_head", st);
        SN_TRY(launch_tc_gemm_act(gemm(B, m->vocab, D, m->x, m->head, m->shead, m->logits),
                                  m->thead, m->p_x, st, true));
    }
    return cuda_check(cudaGetLastError(), "tc step launch");
}

// Profile mode: per-phase times of one fused step from its device timestamps
// (slot 1+8p+j of phase p: j = 0 loads done, 1 row statistics done, 2 inputs
// ready, 3 weights ready, 4 rows done, 5 barrier passed). A part's time is the
// slowest CTA's span in its own clock64 cycles; a barrier's is (last CTA out)
// - (last CTA in) on %globaltimer.
int fused_trace_report(SunnyModel* m, const FusedArgs& fa, cudaStream_t st) {
    const int n = rt().num_sms, S = fa.trace_slots, L = m->L;
    std::vector<unsigned long long> t((size_t)n * 2 * S);  // [cta][globaltimer S | clock64 S]
    SN_TRY(cuda_check(cudaMemcpyAsync(t.data(), fa.trace, t.size() * sizeof(t[0]),
                                      cudaMemcpyDeviceToHost, st),
                      "fused trace"));
    SN_TRY(cuda_check(cudaStreamSynchronize(st), "fused trace"));
    int khz = 0;  // SM clock for the cycle spans
    cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, rt().device);
    const double ms_per_cycle = khz > 0 ? 1.0 / khz : 0.0;
    auto last = [&](int e) {
        unsigned long long v = 0;
        for (int c = 0; c < n; ++c) {
            const unsigned long long x = t[(size_t)c * 2 * S + e];
            v = x > v ? x : v;
        }
        return v;
    };
    auto span = [&](int e0, int e1) {  // slowest CTA, in its own cycles
        long long w = 0;
        for (int c = 0; c < n; ++c) {
            const unsigned long long* ck = &t[(size_t)c * 2 * S + S];
            const long long d = (long long)(ck[e1] - ck[e0]);
            w = d > w ? d : w;
        }
        return w * ms_per_cycle;
    };
    static const char* names[5] = {"P1_ln_taps_V_Ws", "P2_U_gate_state", "P3_Wz",
                                   "P4_lnz_Wc_resid", "head"};
    double bar_ns = 0.0;
    int nbar = 0;
    static const char* parts[5] = {"loads", "stats", "ln", "wait_w", "rows"};
    for (int p = 0; p <= 4 * L; ++p) {
        if (p == 4 * L && !fa.with_head) break;
        const int k = p == 4 * L ? 4 : p % 4;
        int prev = p == 0 ? 0 : 1 + 8 * (p - 1) + 5;  // start: previous barrier passed
        for (int j = 0; j < 5; ++j) {
            const int e = 1 + 8 * p + j;
            char name[64];
            snprintf(name, sizeof name, "fused:%s.%s", names[k], parts[j]);
            prof_add(name, 1, span(prev, e));
            prev = e;
        }
        if (p < 4 * L && (p + 1 < 4 * L || fa.with_head)) {
            bar_ns += (double)(last(1 + 8 * p + 5) - last(1 + 8 * p + 4));
            ++nbar;
        }
    }
    prof_add("fused:barriers", nbar, bar_ns * 1e-6);
    return SN_OK;
}

// Replay (capturing on first use) the graph of a B-sequence step.
int run_step(SunnyModel* m, int B, bool with_head) {
    cudaStream_t st = stream();
    const bool tc = m->tc_step && B >= 16;
    if (prof_graph())  // the step's graph with event nodes around each family
        return prof_graph_run(&m->pgraphs[std::make_pair((long long)B, with_head ? 1 : 0)],
                              m->cap, st, [&](cudaStream_t cs) {
                                  return tc ? enqueue_step_tc(m, B, with_head, cs, m->side)
                                            : enqueue_step(m, B, with_head, cs);
                              });
    if (prof_on())  // bracket kernels, no graph
        return tc ? enqueue_step_tc(m, B, with_head, st, st) : enqueue_step(m, B, with_head, st);
    auto key = std::make_pair(B, with_head ? 1 : 0);
    auto it = m->graphs.find(key);
    if (it == m->graphs.end()) {
        cudaGraph_t g = nullptr;
        SN_TRY(cuda_check(cudaStreamBeginCapture(m->cap, cudaStreamCaptureModeThreadLocal),
                          "begin capture"));
        const int rc = tc ? enqueue_step_tc(m, B, with_head, m->cap, m->side)
                          : enqueue_step(m, B, with_head, m->cap);
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
    return cuda_check(cudaGraphLaunch(it->second, st), "graph launch");
}

// ------------------------------------------------------------ chunked prefill
int ensure_chunk_bufs(SunnyModel* m, int B, int Tc) {
    const long long rows = (long long)B * Tc;
    if (rows <= m->crows && B <= m->cseqs) return SN_OK;
    const size_t D = m->D, I = m->I, R = m->R, n = (size_t)rows;
    m->ctok = m->dalloc<int32_t>(n);
    m->cx = m->dalloc<float>(n * D);
    m->craw = m->dalloc<float>(n * D);
    m->cat = m->dalloc<float>(n * D);
    m->cv = m->dalloc<float>(n * R);
    m->cq = m->dalloc<float>(n * 2 * D);
    m->cu = m->dalloc<float>(n * D);
    m->cp = m->dalloc<float>(n * D);
    m->cst = m->dalloc<float>(n * D);
    m->cprev = m->dalloc<float>(n * D);
    m->csfb = m->dalloc<float>(n * D);
    m->cz = m->dalloc<float>(n * I);
    m->cmu = m->dalloc<float>(n);
    m->crs = m->dalloc<float>(n);
    m->cs0 = m->dalloc<float>((size_t)B * D);
    m->csend = m->dalloc<float>((size_t)B * D);
    if (!m->csend || !m->cs0 || !m->crs || !m->cz)
        return fail(SN_E_NOMEM, "prefill buffers for %lld rows", rows);
    if (!getenv("SN_DISABLE_TC") && rows >= 16) {
        SN_TRY(tc_reserve(m->D, rows));
        SN_TRY(tc_reserve(m->R, rows));
        SN_TRY(tc_reserve(m->I, rows));
    }
    bool tc = !getenv("SN_DISABLE_TC") && rows >= 16 && D % 8 == 0 && R % 8 == 0 && I % 8 == 0;
    for (int l = 0; l < m->L && tc; ++l) {
        const SunnyLayer& y = m->ly[l];
        tc = y.tV.ready && y.tU.ready && y.tWz.ready && y.tWc.ready && y.tWs.ready;
    }
    m->c_tc = false;
    if (tc) {
        auto al = [](size_t nb, void* o) -> void* { return ((SunnyModel*)o)->dalloc<uint8_t>(nb); };
        SN_TRY(tc_act_alloc(&m->c_at, (int)D, rows, al, m));
        SN_TRY(tc_act_alloc(&m->c_v, (int)R, rows, al, m));
        SN_TRY(tc_act_alloc(&m->c_u, (int)D, rows, al, m));
        SN_TRY(tc_act_alloc(&m->c_prev, (int)D, rows, al, m));
        SN_TRY(tc_act_alloc(&m->c_z, (int)I, rows, al, m));
        m->c_tc = true;
    }
    m->crows = rows;
    m->cseqs = B;
    for (auto& kv : m->cgraphs) cudaGraphExecDestroy(kv.second);  // captured old pointers
    m->cgraphs.clear();
    m->pgraphs.clear();
    return SN_OK;
}

// One chunk of Tc tokens for sequences [0,B) (ids already in m->ctok, row b*Tc+t):
// every contraction runs over M = B*Tc rows, the recurrence as the scan.
int enqueue_chunk(SunnyModel* m, int B, int Tc, bool head, cudaStream_t st) {
    const int D = m->D, I = m->I, R = m->R, L = m->L;
    const long long M = (long long)B * Tc;
    const unsigned eb = (unsigned)((M * D + 255) / 256);
    // producer-written planes (the contraction dispatch uses SIMT below 16 rows)
    const bool ctc = m->c_tc && M >= 16;
    {
        ProfScope ps("prefill_rows", st);
        gather_embed_kernel<<<(unsigned)M, 256, 0, st>>>(D, m->vocab, rt().d_err, m->ctok,
                                                         m->embed, m->cx);
    }
    for (int l = 0; l < L; ++l) {
        const SunnyLayer& y = m->ly[l];
        {
            ProfScope ps("prefill_rows", st);
            ln_rows_kernel<<<(unsigned)M, 256, 0, st>>>(D, m->cx, m->craw, y.ni_g, y.ni_c, m->eps);
            const bool al16 = (uintptr_t)y.dw % 16 == 0 && (uintptr_t)m->hist % 16 == 0 &&
                              (uintptr_t)m->craw % 16 == 0;
            if (ctc && al16)  // four channels per thread (planes: D % 8 == 0)
                conv_chunk4_kernel<<<(unsigned)((M * D / 4 + 255) / 256), 256, 0, st>>>(
                    B, Tc, D, m->K, m->KH, L, l, m->craw, m->hist, m->pos, y.dw, m->c_at.hi,
                    m->c_at.lo);
            else
                conv_chunk_kernel<<<eb, 256, 0, st>>>(B, Tc, D, m->K, m->KH, L, l, m->craw,
                                                     m->hist, m->pos, y.dw, m->cat,
                                                     ctc ? m->c_at.hi : nullptr,
                                                     ctc ? m->c_at.lo : nullptr);
            if (m->K > 1 && al16 && D % 4 == 0) {
                const int v = (Tc < m->KH ? Tc : m->KH) * D / 4;
                const int th = v < 1024 ? (v + 31) / 32 * 32 : 1024;
                ring_update4_kernel<<<B, th, 0, st>>>(Tc, D, m->KH, L, l, m->craw, m->hist,
                                                      m->pos);
            } else if (m->K > 1) {
                ring_update_kernel<<<B, 256, 0, st>>>(Tc, D, m->KH, L, l, m->craw, m->hist,
                                                      m->pos);
            }
        }
        if (ctc) {  // inputs as producer-written planes; V writes U's
            GemmArgs gv = gemm((int)M, R, D, m->cat, y.V, y.sV, m->cv);
            gv.Ch = m->c_v.hi;
            gv.Cl = m->c_v.lo;
            {
                ProfScope ps("gemm_V", st);
                SN_TRY(launch_tc_gemm_act(gv, y.tV, m->c_at, st));
            }
            ProfScope ps("gemm_U", st);
            SN_TRY(launch_tc_gemm_act(gemm((int)M, 2 * D, R, m->cv, y.U, y.sU, m->cq), y.tU,
                                      m->c_v, st));
        } else {
            {
                ProfScope ps("gemm_V", st);
                SN_TRY(launch_gemm(gemm((int)M, R, D, m->cat, y.V, y.sV, m->cv), m->wtype, st,
                                   &y.tV));
            }
            ProfScope ps("gemm_U", st);
            SN_TRY(launch_gemm(gemm((int)M, 2 * D, R, m->cv, y.U, y.sU, m->cq), m->wtype, st,
                               &y.tU));
        }
        {
            ProfScope ps("prefill_scan", st);
            __nv_bfloat16* uh = ctc ? m->c_u.hi : nullptr;
            __nv_bfloat16* ul = ctc ? m->c_u.lo : nullptr;
            const bool gvec = D % 8 == 0 && (uintptr_t)y.delta % 16 == 0 &&
                              (uintptr_t)m->cq % 16 == 0 && (uintptr_t)m->cu % 16 == 0 &&
                              (uintptr_t)m->cp % 16 == 0;
            const unsigned gb = (unsigned)((M * D / 8 + 255) / 256);
            if (gvec && m->G == 8)
                gate_group_kernel<8><<<gb, 256, 0, st>>>(M, D, m->cq, y.delta, m->cu, m->cp,
                                                         m->clamp, m->p_floor, uh, ul);
            else if (gvec && m->G == 4)
                gate_group_kernel<4><<<2 * gb, 256, 0, st>>>(M, D, m->cq, y.delta, m->cu, m->cp,
                                                             m->clamp, m->p_floor, uh, ul);
            else
                gate_chunk_kernel<<<eb, 256, 0, st>>>(M, D, m->G, m->cq, y.delta, m->cu, m->cp,
                                                      m->clamp, m->p_floor, uh, ul);
            if (ctc) {
                // the layer's state rows read and written in place, the state
                // entering each position written as Ws's input planes
                float* sl = m->s + (size_t)l * D;
                SN_TRY(launch_scan_strided(m->cp, m->cu, sl, (long long)L * D, m->cst, sl,
                                           (long long)L * D, B, Tc, D, 1, m->c_prev.hi,
                                           m->c_prev.lo, st));
            } else {
                SN_TRY(cuda_check(cudaMemcpy2DAsync(m->cs0, (size_t)D * 4, m->s + (size_t)l * D,
                                                    (size_t)L * D * 4, (size_t)D * 4, B,
                                                    cudaMemcpyDeviceToDevice, st),
                                  "s0"));
                SN_TRY(launch_scan(m->cp, m->cu, m->cs0, m->cst, m->csend, B, Tc, D, 1, st));
                SN_TRY(cuda_check(cudaMemcpy2DAsync(m->s + (size_t)l * D, (size_t)L * D * 4,
                                                    m->csend, (size_t)D * 4, (size_t)D * 4, B,
                                                    cudaMemcpyDeviceToDevice, st),
                                  "send"));
                prev_kernel<<<eb, 256, 0, st>>>(Tc, D, M * D, m->cs0, m->cst, m->cprev);
            }
        }
        {
            ProfScope ps("gemm_Ws", st);
            const GemmArgs gs = gemm((int)M, D, D, m->cprev, y.Ws, y.sWs, m->csfb);
            if (ctc) SN_TRY(launch_tc_gemm_act(gs, y.tWs, m->c_prev, st));
            else SN_TRY(launch_gemm(gs, m->wtype, st, &y.tWs));
        }
        GemmArgs gz = gemm((int)M, I, D, m->cu, y.Wz, y.sWz, m->cz);
        gz.epi = kEpiWedge;
        gz.p = y.a_tanh;
        {
            ProfScope ps("gemm_Wz", st);
            if (ctc) SN_TRY(launch_tc_gemm_act(gz, y.tWz, m->c_u, st));
            else SN_TRY(launch_gemm(gz, m->wtype, st, &y.tWz));
        }
        if (ctc) {  // LN(z) straight into Wc's input planes
            ProfScope ps("rowstats", st);
            SN_TRY(launch_ln_split(false, st, (int)M, I, m->cz, I, y.nm_g, y.nm_c, m->c_z.hi,
                                   m->c_z.lo, m->eps));
        } else {
            ProfScope ps("rowstats", st);
            SN_TRY(launch_rowstats(false, st, (int)M, I, m->cz, I, m->cmu, m->crs, m->eps));
        }
        GemmArgs gc = gemm((int)M, D, I, m->cz, y.Wc, y.sWc, m->cx);
        if (!ctc) {
            gc.mu = m->cmu; gc.rs = m->crs; gc.g = y.nm_g; gc.c = y.nm_c;
        }
        gc.epi = kEpiResid;
        gc.p = y.b_gain;
        gc.S = m->cst; gc.lds = D;
        gc.F = m->csfb; gc.ldf = D;
        gc.X = m->cx; gc.ldx = D;
        {
            ProfScope ps("gemm_Wc", st);
            if (ctc) SN_TRY(launch_tc_gemm_act(gc, y.tWc, m->c_z, st));
            else SN_TRY(launch_gemm(gc, m->wtype, st, &y.tWc));
        }
    }
    if (head) {  // logits of each sequence's last position only
        const float* last = m->cx + (size_t)(Tc - 1) * D;
        SN_TRY(launch_rowstats(false, st, B, D, last, (long long)Tc * D, m->cmu, m->crs, m->eps));
        GemmArgs gh = gemm(B, m->vocab, D, last, m->head, m->shead, m->logits);
        gh.lda = (long long)Tc * D;
        gh.mu = m->cmu; gh.rs = m->crs; gh.g = m->no_g; gh.c = m->no_c;
        ProfScope ps("gemm_head", st);
        SN_TRY(launch_gemm(gh, m->wtype, st, &m->thead));
    }
    return cuda_check(cudaGetLastError(), "prefill chunk launch");
}

int run_chunk(SunnyModel* m, int B, int Tc, bool head) {
    cudaStream_t st = stream();
    auto key = std::make_pair((long long)B * 65536 + Tc, head ? 1 : 0);
    if (prof_graph())
        return prof_graph_run(&m->pgraphs[std::make_pair(-key.first, key.second)], m->cap, st,
                              [&](cudaStream_t cs) { return enqueue_chunk(m, B, Tc, head, cs); });
    if (prof_on()) return enqueue_chunk(m, B, Tc, head, st);
    auto it = m->cgraphs.find(key);
    if (it == m->cgraphs.end()) {
        cudaGraph_t g = nullptr;
        SN_TRY(cuda_check(cudaStreamBeginCapture(m->cap, cudaStreamCaptureModeThreadLocal),
                          "begin capture"));
        const int rc = enqueue_chunk(m, B, Tc, head, m->cap);
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
        it = m->cgraphs.emplace(key, ex).first;
    }
    return cuda_check(cudaGraphLaunch(it->second, st), "graph launch");
}

// tokens (B,T) row-major; the carried state is the handle's own
int sunny_prefill(SunnyModel* m, const int32_t* tokens, int B, int T, int chunk, float* logits) {
    if (!m || !m->ready || !tokens || B <= 0 || T <= 0 || B > m->nseq || chunk <= 0)
        return fail(SN_E_INVAL, "sunny_prefill: bad arguments");
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    const int Tc = chunk < T ? chunk : T;
    SN_TRY(ensure_chunk_bufs(m, B, Tc));
    cudaStream_t st = stream();
    const bool tdev = is_device_ptr(tokens);
    for (int c0 = 0; c0 < T; c0 += Tc) {
        const int tc = Tc < T - c0 ? Tc : T - c0;
        const bool last = c0 + tc >= T;
        SN_TRY(cuda_check(cudaMemcpy2DAsync(m->ctok, (size_t)tc * 4, tokens + c0, (size_t)T * 4,
                                            (size_t)tc * 4, B,
                                            tdev ? cudaMemcpyDeviceToDevice
                                                 : cudaMemcpyHostToDevice,
                                            st),
                          "prefill tokens"));
        SN_TRY(run_chunk(m, B, tc, last && logits != nullptr));
    }
    bool host = !tdev;
    if (logits) {
        const bool dev = is_device_ptr(logits);
        host |= !dev;
        SN_TRY(cuda_check(cudaMemcpyAsync(logits, m->logits, (size_t)B * m->vocab * 4,
                                          dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost,
                                          st),
                          "logits"));
    }
    return finish(host);
}

int sunny_step(SunnyModel* m, const int32_t* tokens, int B, float* logits, int32_t* next) {
    if (!m || !m->ready || !tokens || B <= 0 || B > m->nseq)
        return fail(SN_E_INVAL, "sunny_step: bad handle, tokens or B");
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    cudaStream_t st = stream();
    const bool tok_dev = is_device_ptr(tokens);
    const bool head = logits != nullptr || next != nullptr;
    if (B <= kFusedMaxB && !getenv("SN_DISABLE_FUSED")) {
        // one persistent kernel per step; it reads the caller's device tokens
        // and writes device logits / next tokens (greedy argmax fused) in place
        FusedArgs fa = m->fbase;
        fa.B = B;
        fa.with_head = head ? 1 : 0;
        if (fused_plan(&fa, !getenv("SN_FUSED_NO_STAGE"))) {
            if (!tok_dev)
                SN_TRY(cuda_check(cudaMemcpyAsync(m->tok, tokens, (size_t)B * 4,
                                                  cudaMemcpyHostToDevice, st),
                                  "tokens"));
            const bool lg_dev = logits && is_device_ptr(logits);
            const bool nx_dev = next && is_device_ptr(next);
            fa.tok = tok_dev ? tokens : m->tok;
            fa.logits = logits ? (lg_dev ? logits : m->logits) : nullptr;
            fa.next = next ? (nx_dev ? next : m->next) : nullptr;
            if (prof_on()) {
                fa.trace = m->ftrace;
                fa.trace_slots = 32 * m->L + 9;
                {
                    ProfScope ps("fused_step", st);
                    SN_TRY(launch_sunny_fused(fa, st));
                }
                SN_TRY(fused_trace_report(m, fa, st));
            } else {
                SN_TRY(launch_sunny_fused(fa, st));
            }
            if (logits && !lg_dev)
                SN_TRY(cuda_check(cudaMemcpyAsync(logits, m->logits, (size_t)B * m->vocab * 4,
                                                  cudaMemcpyDeviceToHost, st),
                                  "logits"));
            if (next && !nx_dev)
                SN_TRY(cuda_check(cudaMemcpyAsync(next, m->next, (size_t)B * 4,
                                                  cudaMemcpyDeviceToHost, st),
                                  "next"));
            return finish(!tok_dev || (logits && !lg_dev) || (next && !nx_dev));
        }
    }
    SN_TRY(cuda_check(cudaMemcpyAsync(m->tok, tokens, (size_t)B * 4,
                                      tok_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                                      st),
                      "tokens"));
    SN_TRY(run_step(m, B, head));
    bool host = !tok_dev;
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

// Zero the state of sequences [seq0, seq0 + n) (all of them by default).
int sunny_reset(SunnyModel* m, int seq0 = 0, int n = -1) {
    if (!m || !m->ready) return fail(SN_E_INVAL, "sunny_reset: bad handle");
    if (n < 0) n = m->nseq - seq0;
    if (seq0 < 0 || n <= 0 || seq0 + n > m->nseq)
        return fail(SN_E_INVAL, "sunny_reset: sequences [%d, %d) outside [0, %d)", seq0,
                    seq0 + n, m->nseq);
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    cudaStream_t st = stream();
    const size_t a = (size_t)seq0, k = (size_t)n;
    cudaMemsetAsync(m->s + a * m->L * m->D, 0, k * m->L * m->D * 4, st);
    cudaMemsetAsync(m->hist + a * m->L * m->KH * m->D, 0, k * m->L * m->KH * m->D * 4, st);
    cudaMemsetAsync(m->pos + a * m->L, 0, k * m->L * 4, st);
    return finish(false);
}

// State of sequences [seq0, seq0 + B): s (B,L,D) and hist (B,L,K-1,D), newest
// history row first, out of (get) or into the handle's ring buffers.
int sunny_state_io(SunnyModel* m, int seq0, int B, float* s, float* hist, bool get) {
    if (!m || !m->ready || seq0 < 0 || B <= 0 || seq0 + B > m->nseq || !s || !hist)
        return fail(SN_E_INVAL, "sunny state: bad arguments");
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    cudaStream_t st = stream();
    const size_t ns = (size_t)B * m->L * m->D * 4, nh = (size_t)B * m->L * m->KH * m->D * 4;
    float* ms = m->s + (size_t)seq0 * m->L * m->D;
    float* mh = m->hist + (size_t)seq0 * m->L * m->KH * m->D;
    int32_t* mp = m->pos + (size_t)seq0 * m->L;
    Arr S, H;
    if (get) {
        SN_TRY(stage_out(s, ns, 5, &S));
        SN_TRY(stage_out(hist, nh, 6, &H));
        SN_TRY(cuda_check(cudaMemcpyAsync(S.dev, ms, ns, cudaMemcpyDeviceToDevice, st), "s"));
    } else {
        SN_TRY(stage_in(s, ns, 5, &S));
        SN_TRY(stage_in(hist, nh, 6, &H));
        SN_TRY(cuda_check(cudaMemcpyAsync(ms, S.dev, ns, cudaMemcpyDeviceToDevice, st), "s"));
        cudaMemsetAsync(mp, 0, (size_t)B * m->L * 4, st);
    }
    const long long total = (long long)B * m->L * m->KH * m->D;
    hist_io_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(
        B, m->L, m->KH, m->D, mh, (float*)H.dev, mp, get ? 1 : 0);
    SN_TRY(cuda_check(cudaGetLastError(), "hist io"));
    if (get) {
        SN_TRY(copy_back(S));
        SN_TRY(copy_back(H));
    }
    return finish(true);
}

}  // namespace
}  // namespace sn

using namespace sn;

struct SnAbiSunny {
    std::unique_ptr<SunnyModel> m;
};
struct SnModel {
    std::unique_ptr<SunnyModel> m;
};

namespace {
SnAbiSunny* open_sunny(const char* path, int nseq, bool half, const int* want) {
    if (!path || nseq <= 0) {
        fail(SN_E_INVAL, "sunny load: null path or nseq <= 0");
        return nullptr;
    }
    auto h = new SnAbiSunny{std::make_unique<SunnyModel>()};
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    if (load_model(h->m.get(), path, nseq, half, want) != SN_OK) {
        delete h;
        return nullptr;
    }
    return h;
}
}  // namespace

extern "C" {

SnAbiSunny* sn_abi_sunny_load(const char* blob_path, int32_t nseq) {
    return open_sunny(blob_path, nseq, false, nullptr);
}

void sn_abi_sunny_free(SnAbiSunny* m) {
    if (!m) return;
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    cudaDeviceSynchronize();
    delete m;
}

sn_status sn_abi_sunny_reset(SnAbiSunny* m) { return m ? sunny_reset(m->m.get()) : SN_E_INVAL; }

int32_t sn_abi_sunny_vocab(const SnAbiSunny* m) { return m ? m->m->vocab : 0; }

int32_t sn_abi_sunny_dims(const SnAbiSunny* m, int32_t* d) {
    if (!m || !d) return SN_E_INVAL;
    const SunnyModel* s = m->m.get();
    const int32_t v[8] = {s->vocab, s->D, s->I, s->R, s->K, s->L, s->G, s->wtype};
    memcpy(d, v, sizeof v);
    return SN_OK;
}

sn_status sn_abi_sunny_step(SnAbiSunny* m, const int32_t* tokens, int32_t B, float* logits) {
    if (!m) return SN_E_INVAL;
    return sunny_step(m->m.get(), tokens, B, logits, nullptr);
}

sn_status sn_abi_sunny_step_argmax(SnAbiSunny* m, const int32_t* tokens, int32_t B,
                                   int32_t* next) {
    if (!m || !next) return SN_E_INVAL;
    return sunny_step(m->m.get(), tokens, B, nullptr, next);
}

sn_status sn_abi_sunny_prefill(SnAbiSunny* m, const int32_t* tokens, int32_t B, int32_t T,
                               float* logits) {
    if (!m) return SN_E_INVAL;
    return sunny_prefill(m->m.get(), tokens, B, T, 256, logits);
}

sn_status sn_abi_sunny_prefill_chunked(SnAbiSunny* m, const int32_t* tokens, int32_t B, int32_t T,
                                       int32_t chunk, float* logits) {
    if (!m) return SN_E_INVAL;
    return sunny_prefill(m->m.get(), tokens, B, T, chunk, logits);
}

sn_status sn_abi_sunny_get_state(SnAbiSunny* m, int32_t B, float* s, float* hist) {
    return m ? sunny_state_io(m->m.get(), 0, B, s, hist, true) : SN_E_INVAL;
}

sn_status sn_abi_sunny_get_state_at(SnAbiSunny* m, int32_t seq0, int32_t n, float* s,
                                    float* hist) {
    return m ? sunny_state_io(m->m.get(), seq0, n, s, hist, true) : SN_E_INVAL;
}

sn_status sn_abi_sunny_set_state_at(SnAbiSunny* m, int32_t seq0, int32_t n, const float* s,
                                    const float* hist) {
    return m ? sunny_state_io(m->m.get(), seq0, n, (float*)s, (float*)hist, false) : SN_E_INVAL;
}

sn_status sn_abi_sunny_reset_at(SnAbiSunny* m, int32_t seq0, int32_t n) {
    return m ? sunny_reset(m->m.get(), seq0, n) : SN_E_INVAL;
}

sn_status sn_abi_sunny_set_state(SnAbiSunny* m, int32_t B, const float* s, const float* hist) {
    return m ? sunny_state_io(m->m.get(), 0, B, (float*)s, (float*)hist, false) : SN_E_INVAL;
}

// ---------------------------------------------- reference sunnynet.h symbol set
SnModel* sn_load(const char* path, int vocab, int dim, int inner, int rank, int taps, int layers,
                 int group, int tied) {
    const int want[8] = {vocab, dim, inner, rank, taps, layers, group, tied};
    SnAbiSunny* h = open_sunny(path, 1, false, want);
    if (!h) return nullptr;
    SnModel* m = new SnModel{std::move(h->m)};
    delete h;
    return m;
}

SnModel* sn_load_h(const char* path, int vocab, int dim, int inner, int rank, int taps,
                   int layers, int group, int tied) {
    const int want[8] = {vocab, dim, inner, rank, taps, layers, group, tied};
    SnAbiSunny* h = open_sunny(path, 1, true, want);
    if (!h) return nullptr;
    SnModel* m = new SnModel{std::move(h->m)};
    delete h;
    return m;
}

void sn_free(SnModel* m) {
    if (!m) return;
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    cudaDeviceSynchronize();
    delete m;
}

void sn_reset(SnModel* m) {
    if (m) sunny_reset(m->m.get());
}

void sn_step(SnModel* m, int token, float* logits) {
    if (!m) return;
    const int32_t t = token;
    sunny_step(m->m.get(), &t, 1, logits, nullptr);
}

// sunnynet.c:347-349 feeds the tokens one by one; the result (state and the
// last token's logits) is the same when the prompt runs as 256-token chunks.
void sn_prefill(SnModel* m, const int* tokens, int n, float* logits) {
    if (!m || !tokens || n <= 0) return;
    sunny_prefill(m->m.get(), (const int32_t*)tokens, 1, n, 256, logits);
}

int sn_vocab(const SnModel* m) { return m ? m->m->vocab : 0; }

int sn_ready(const SnModel* m) { return m && m->m->ready ? 1 : 0; }

void sn_dbg_layer(SnModel* m, int token, int layer, float* dbg) {
    if (!m || !dbg || layer < 0 || layer >= m->m->L) return;
    SunnyModel* s = m->m.get();
    std::lock_guard<std::recursive_mutex> lk(rt().mu);
    cudaStream_t st = stream();
    const int32_t t = token;
    cudaMemcpyAsync(s->tok, &t, 4, cudaMemcpyHostToDevice, st);
    if (enqueue_step(s, 1, false, st, layer) != SN_OK) return;
    const int D = s->D, I = s->I, R = s->R;
    // raw, at, v, gate, u, s, zn, yn, sfb, out (sunnynet.c:278-290)
    struct Part {
        const float* p;
        int n;
    } parts[10] = {{s->raw, D}, {s->at, D}, {s->v, R}, {s->gate, D}, {s->u, D},
                   {s->s + (size_t)layer * D, D}, {s->z, I}, {s->yn, I}, {s->sfb, D}, {s->x, D}};
    Arr out;
    const size_t total = (size_t)(7 * D + R + 2 * I) * 4;
    if (stage_out(dbg, total, 7, &out) != SN_OK) return;
    size_t off = 0;
    for (auto& pt : parts) {
        cudaMemcpyAsync((char*)out.dev + off, pt.p, (size_t)pt.n * 4, cudaMemcpyDeviceToDevice, st);
        off += (size_t)pt.n * 4;
    }
    copy_back(out);
    finish(true);
}

}  // extern "C"
