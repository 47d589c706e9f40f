/* CPU oracle for the SunnyNet token loop -- TEST INFRASTRUCTURE ONLY.
 *
 * Restates the reference runtime's arithmetic (CodeDoes/SunnyNet,
 * sunnynet/runtime/{recur,quant,sunnynet,rwkv7}.c) in plain scalar C. The
 * reference is compiled as ISO C11 (no FP contraction) with explicit AVX2 FMA
 * intrinsics; this file reproduces the same rounding sequence with fmaf()
 * where the reference fuses and separate mul/add where it does not, and the
 * same reduction trees for its horizontal sums, so its results are
 * bit-identical to the reference build. See sn_oracle.h for who may use it.
 */
#include "sn_oracle.h"

#include <math.h>
#include <omp.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ fp16 */
static uint16_t f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u, ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 rounds to inf */
    if (ax < 0x38800000u) {                                   /* below 2^-14: subnormal */
        float af;
        memcpy(&af, &ax, 4);
        return (uint16_t)(sign | (uint32_t)nearbyintf(af * 16777216.0f));
    }
    uint32_t h = ((((ax >> 23) - 127u + 15u) << 10) | ((ax & 0x7fffffu) >> 13));
    const uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
}

static float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    uint32_t x;
    if (e == 0) {
        float f = (float)m * 5.9604644775390625e-8f; /* m * 2^-24, exact */
        memcpy(&x, &f, 4);
        x |= sign;
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e - 15u + 127u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

/* ------------------------------------------------------- shared helpers */
/* 1/(1+exp(-x)) as sunnynet.c:247 / rwkv7.c:118 */
static float sig(float x) { return 1.0f / (1.0f + expf(-x)); }

/* Horizontal sum of 8 lanes the way the reference's SSE hadd tree does it
 * (quant.c:156-172, rwkv7.c:109-116): ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7)). */
static float hsum8_tree(const float* l) {
    const float c0 = l[0] + l[4], c1 = l[1] + l[5], c2 = l[2] + l[6], c3 = l[3] + l[7];
    return (c0 + c1) + (c2 + c3);
}

/* Row dot product as the SunnyNet GEMV (sunnynet.c:123-138): 8 interleaved FMA
 * accumulators, then a left-to-right sum of the 8 lanes, then a scalar tail. */
static float dot_sunny(const float* w, const float* x, int n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int i = 0;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; ++l) acc[l] = fmaf(w[i + l], x[i + l], acc[l]);
    float s = acc[0];
    for (int l = 1; l < 8; ++l) s = s + acc[l];
    for (; i < n; ++i) s = s + w[i] * x[i];
    return s;
}

/* y[out] = W(out,in) x, SunnyNet order. `par`: rows spread over the OpenMP
 * threads (each row's sum is unchanged, so the result is the same). */
static void gemv_sunny_p(float* y, const float* x, const float* W, int in, int out, int par) {
#pragma omp parallel for schedule(static) if (par)
    for (int j = 0; j < out; ++j) y[j] = dot_sunny(W + (size_t)j * in, x, in);
}

static void gemv_sunny(float* y, const float* x, const float* W, int in, int out) {
    gemv_sunny_p(y, x, W, in, out, 0);
}

/* Two-pass layernorm with sequential sums (sunnynet.c:198-210, rwkv7.c:128-140). */
static void layernorm(float* y, const float* x, const float* g, const float* c, int n,
                      float eps) {
    float sum = 0.0f;
    for (int i = 0; i < n; ++i) sum = sum + x[i];
    const float mean = sum / (float)n;
    float vs = 0.0f;
    for (int i = 0; i < n; ++i) {
        const float d = x[i] - mean;
        vs = vs + d * d;
    }
    const float rstd = 1.0f / sqrtf(vs / (float)n + eps);
    for (int i = 0; i < n; ++i) y[i] = (x[i] - mean) * rstd * g[i] + c[i];
}

/* ------------------------------------------------------ recurrence (recur.c) */
/* recur.c:13-48. The reference vectorises 8 channels at a time with an FMA and
 * handles the N%8 remainder in scalar code without contraction, so the last
 * N%8 channels use mul+add instead of fma. */
void or_recur_scan(const float* a, const float* b, const float* s0, float* out,
                   float* send, int B, int T, int N, int gated) {
    const int nv = N - N % 8;
#pragma omp parallel for schedule(static)
    for (int bb = 0; bb < B; ++bb) {
        const size_t base = (size_t)bb * T * N;
        for (int d = 0; d < N; ++d) {
            float s = s0[(size_t)bb * N + d];
            for (int t = 0; t < T; ++t) {
                const size_t o = base + (size_t)t * N + d;
                const float av = a[o];
                const float bv = gated ? (1.0f - av) * b[o] : b[o];
                s = (d < nv) ? fmaf(av, s, bv) : av * s + bv;
                out[o] = s;
            }
            send[(size_t)bb * N + d] = s;
        }
    }
}

/* recur.c:51-107: reverse-time pass of the scan. Per channel, from t = T-1
 * down to 0: g = dout_t + g (one rounding), da_t = g*(s_{t-1} - u_t) and
 * db_t = g*(1 - a_t) for the gated form (da_t = g*s_{t-1}, db_t = g for the
 * FMA form), then g = g*a_t. s_{-1} = s0; ds0 = g after t = 0. No FMA appears
 * in either of the reference's paths (AVX2 lanes and the N%8 tail), so one
 * rule serves every channel. */
void or_recur_bwd(const float* a, const float* b, const float* s0, const float* out,
                  const float* dout, float* da, float* db, float* ds0, int B, int T, int N,
                  int gated) {
#pragma omp parallel for schedule(static)
    for (int bb = 0; bb < B; ++bb) {
        const size_t base = (size_t)bb * T * N;
        for (int d = 0; d < N; ++d) {
            float g = 0.0f;
            for (int t = T - 1; t >= 0; --t) {
                const size_t o = base + (size_t)t * N + d;
                g = dout[o] + g;
                const float av = a[o];
                const float sp = t > 0 ? out[o - N] : s0[(size_t)bb * N + d];
                if (gated) {
                    const float diff = sp - b[o];
                    const float oma = 1.0f - av;
                    da[o] = g * diff;
                    db[o] = g * oma;
                } else {
                    da[o] = g * sp;
                    db[o] = g;
                }
                g = g * av;
            }
            ds0[(size_t)bb * N + d] = g;
        }
    }
}

/* recur.c:109-131, same fused/unfused split as the scan. */
void or_recur_step(const float* a, const float* b, float* s, int B, int N, int gated) {
    const int nv = N - N % 8;
    for (int bb = 0; bb < B; ++bb)
        for (int d = 0; d < N; ++d) {
            const size_t o = (size_t)bb * N + d;
            const float av = a[o];
            const float bv = gated ? (1.0f - av) * b[o] : b[o];
            s[o] = (d < nv) ? fmaf(av, s[o], bv) : av * s[o] + bv;
        }
}

/* recur.c:134-161: symmetric per-block INT8, sc = amax/127 (1 if amax == 0). */
void or_quant_i8(const float* x, int8_t* q, float* scale, int B, int N, int block) {
    if (block <= 0) block = N;
    const int nb = (N + block - 1) / block;
    for (int bb = 0; bb < B; ++bb)
        for (int k = 0; k < nb; ++k) {
            const int lo = k * block, hi = (k + 1) * block < N ? (k + 1) * block : N;
            const float* xb = x + (size_t)bb * N;
            float amax = 0.0f;
            for (int i = lo; i < hi; ++i) {
                const float v = fabsf(xb[i]);
                if (v > amax) amax = v;
            }
            const float sc = amax > 0.0f ? amax / 127.0f : 1.0f;
            const float inv = 1.0f / sc;
            scale[(size_t)bb * nb + k] = sc;
            for (int i = lo; i < hi; ++i) {
                float t = nearbyintf(xb[i] * inv);
                if (t > 127.0f) t = 127.0f;
                if (t < -127.0f) t = -127.0f;
                q[(size_t)bb * N + i] = (int8_t)t;
            }
        }
}

/* recur.c:163-178 */
void or_dequant_i8(const int8_t* q, const float* scale, float* x, int B, int N, int block) {
    if (block <= 0) block = N;
    const int nb = (N + block - 1) / block;
    for (int bb = 0; bb < B; ++bb)
        for (int i = 0; i < N; ++i)
            x[(size_t)bb * N + i] = (float)q[(size_t)bb * N + i] * scale[(size_t)bb * nb + i / block];
}

/* ----------------------------------------------------------- INT4 (quant.c) */
static float scale_at(const void* scale, size_t i, int fp16) {
    return fp16 ? f16_to_f32(((const uint16_t*)scale)[i]) : ((const float*)scale)[i];
}

/* quant.c:34-65. With fp16 scales (the group-128 format) the stored scale is
 * fp16(amax/7) and the codes are computed against that stored value. */
void or_quant_i4(const float* x, uint8_t* q, void* scale, int rows, int N, int block,
                 int scale_fp16) {
    if (block <= 0) block = 64;
    const int nb = N / block, half = block / 2;
    for (int r = 0; r < rows; ++r)
        for (int b = 0; b < nb; ++b) {
            const float* xb = x + (size_t)r * N + (size_t)b * block;
            float amax = 0.0f;
            for (int i = 0; i < block; ++i) {
                const float v = fabsf(xb[i]);
                if (v > amax) amax = v;
            }
            float sc = amax > 0.0f ? amax / 7.0f : 1.0f;
            if (scale_fp16) {
                uint16_t h = f32_to_f16(sc);
                if ((h & 0x7fffu) == 0) h = 1; /* keep a usable, non-zero step */
                ((uint16_t*)scale)[(size_t)r * nb + b] = h;
                sc = f16_to_f32(h);
            } else {
                ((float*)scale)[(size_t)r * nb + b] = sc;
            }
            const float inv = 1.0f / sc;
            uint8_t* qb = q + (size_t)r * (N / 2) + (size_t)b * half;
            for (int k = 0; k < half; ++k) {
                int lo = (int)nearbyintf(xb[k] * inv);
                int hi = (int)nearbyintf(xb[half + k] * inv);
                lo = lo < -8 ? -8 : (lo > 7 ? 7 : lo);
                hi = hi < -8 ? -8 : (hi > 7 ? 7 : hi);
                qb[k] = (uint8_t)((lo + 8) | ((hi + 8) << 4));
            }
        }
}

/* quant.c:67-87 */
void or_dequant_i4(const uint8_t* q, const void* scale, float* x, int rows, int N,
                   int block, int scale_fp16) {
    if (block <= 0) block = 64;
    const int nb = N / block, half = block / 2;
    for (int r = 0; r < rows; ++r)
        for (int b = 0; b < nb; ++b) {
            const float sc = scale_at(scale, (size_t)r * nb + b, scale_fp16);
            const uint8_t* qb = q + (size_t)r * (N / 2) + (size_t)b * half;
            float* xr = x + (size_t)r * N + (size_t)b * block;
            for (int k = 0; k < half; ++k) {
                xr[k] = (float)((int)(qb[k] & 0x0F) - 8) * sc;
                xr[half + k] = (float)((int)(qb[k] >> 4) - 8) * sc;
            }
        }
}

/* quant.c:89-154, the W4A8 GEMV: per-block INT8 activation quantisation, exact
 * integer block dot products, then acc += (s_w*s_x)*(float)(dot) block by
 * block. Returns -1 for shapes the reference only handles through its
 * fp32-reinterpretation fallback (in % block != 0), or that overflow its
 * 16-bit lane sums (block > 256). */
int or_gemv_i4(float* y, const float* x, const uint8_t* Wq, const void* scale, int in,
               int out, int block, int scale_fp16) {
    if (block <= 0) block = 64;
    if (in % block || block % 2 || block > 256) return -1;
    const int nb = in / block, half = block / 2;
    int8_t* xq = (int8_t*)malloc((size_t)in);
    float* xs = (float*)malloc(sizeof(float) * (size_t)nb);
    int* xsum = (int*)malloc(sizeof(int) * (size_t)nb);
    if (!xq || !xs || !xsum) { free(xq); free(xs); free(xsum); return -2; }
    for (int b = 0; b < nb; ++b) {
        const float* xb = x + (size_t)b * block;
        float amax = 0.0f;
        for (int i = 0; i < block; ++i) {
            const float v = fabsf(xb[i]);
            if (v > amax) amax = v;
        }
        const float sc = amax > 0.0f ? amax / 127.0f : 1.0f;
        const float inv = 1.0f / sc;
        xs[b] = sc;
        int sum = 0;
        for (int i = 0; i < block; ++i) {
            int t = (int)nearbyintf(xb[i] * inv);
            t = t > 127 ? 127 : (t < -127 ? -127 : t);
            xq[b * block + i] = (int8_t)t;
            sum += t;
        }
        xsum[b] = sum;
    }
#pragma omp parallel for schedule(static) if (out >= 512)
    for (int o = 0; o < out; ++o) {
        const uint8_t* row = Wq + (size_t)o * (in / 2);
        float acc = 0.0f;
        for (int b = 0; b < nb; ++b) {
            const uint8_t* wb = row + (size_t)b * half;
            const int8_t* xl = xq + b * block;
            int s = 0;
            for (int k = 0; k < half; ++k)
                s += (int)(wb[k] & 0x0F) * (int)xl[k] + (int)(wb[k] >> 4) * (int)xl[half + k];
            const float sw = scale_at(scale, (size_t)o * nb + b, scale_fp16);
            acc = acc + sw * xs[b] * (float)(s - 8 * xsum[b]);
        }
        y[o] = acc;
    }
    free(xq);
    free(xs);
    free(xsum);
    return 0;
}

/* quant.c:156-172: fp32 reference GEMV, SSE-tree horizontal sum. */
void or_gemv_f32(float* y, const float* x, const float* W, int in, int out) {
    for (int o = 0; o < out; ++o) {
        const float* row = W + (size_t)o * in;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        int i = 0;
        for (; i + 8 <= in; i += 8)
            for (int l = 0; l < 8; ++l) acc[l] = fmaf(row[i + l], x[i + l], acc[l]);
        float s = hsum8_tree(acc);
        for (; i < in; ++i) s = s + row[i] * x[i];
        y[o] = s;
    }
}

/* =================================================== SunnyNet whole model */
#define USNN_MAGIC 0x4E4E5355 /* fp32 blob, release.py:93-141 */
#define USNQ_MAGIC 0x514E5355 /* INT8 per-output-row blob (this project's format) */

typedef struct {
    float *ni_g, *ni_c, *nm_g, *nm_c, *dw; /* dw (K,D) */
    float *V, *U, *Wz, *Wc, *Ws;           /* (out,in) row-major */
    float* delta;
    float a_tanh, b_gain;
} OrLayer;

struct OrSunny {
    int vocab, D, I, R, K, L, G, clamp, nseq;
    float eps, p_floor;
    OrLayer* ly;
    float *no_g, *no_c, *embed, *head; /* head (vocab,D) */
    float* s;                          /* (nseq,L,D) */
    float* hist;                       /* (nseq,L,KH,D), KH = max(K-1,1) */
    float** blocks;
    int nblocks;
    int row_par; /* GEMV rows over threads (set while sequences run one at a time) */
};

static float* sn_alloc(OrSunny* m, size_t n) {
    float* p = (float*)calloc(n ? n : 1, sizeof(float));
    if (!p) return NULL;
    m->blocks[m->nblocks++] = p;
    return p;
}

static int rd(FILE* f, void* dst, size_t bytes) { return fread(dst, 1, bytes, f) == bytes; }

/* (in,out) stored block -> (out,in) row-major, as the reference loader flips it
 * (sunnynet.c:428-445). */
static int rd_flip(FILE* f, float* dst, int in, int out) {
    const size_t n = (size_t)in * out;
    float* tmp = (float*)malloc(sizeof(float) * n);
    if (!tmp) return 0;
    if (!rd(f, tmp, sizeof(float) * n)) { free(tmp); return 0; }
    for (int i = 0; i < in; ++i)
        for (int j = 0; j < out; ++j) dst[(size_t)j * in + i] = tmp[(size_t)i * out + j];
    free(tmp);
    return 1;
}

/* INT8 (out,in) codes + fp32 per-row scale -> fp32, (float)q*sc (recur.c:163-178). */
static int rd_q8(FILE* f, float* dst, int in, int out) {
    const size_t n = (size_t)in * out;
    int8_t* q = (int8_t*)malloc(n);
    float* sc = (float*)malloc(sizeof(float) * (size_t)out);
    int ok = q && sc && rd(f, q, n) && rd(f, sc, sizeof(float) * (size_t)out);
    if (ok)
        for (int j = 0; j < out; ++j)
            for (int i = 0; i < in; ++i)
                dst[(size_t)j * in + i] = (float)q[(size_t)j * in + i] * sc[j];
    free(q);
    free(sc);
    return ok;
}

OrSunny* or_sn_load(const char* path, int nseq) {
    if (nseq <= 0) return NULL;
    FILE* f = fopen(path, "rb");
    if (!f) return NULL;
    int32_t h[12];
    if (!rd(f, h, 4 * 10)) { fclose(f); return NULL; }
    int quant = 0;
    int vocab, D, I, R, K, L, G, clamp;
    if (h[0] == USNN_MAGIC) {
        vocab = h[1]; D = h[2]; I = h[3]; R = h[4]; K = h[5]; L = h[6]; G = h[7]; clamp = h[9];
    } else if (h[0] == USNQ_MAGIC) {
        if (!rd(f, h + 10, 4 * 2) || h[1] != 1 || h[11] != 8) { fclose(f); return NULL; }
        quant = 1;
        vocab = h[2]; D = h[3]; I = h[4]; R = h[5]; K = h[6]; L = h[7]; G = h[8]; clamp = h[10];
    } else {
        fclose(f);
        return NULL;
    }
    if (vocab <= 0 || D <= 0 || I <= 0 || R <= 0 || K <= 0 || L <= 0 || G < 3 || D % G) {
        fclose(f);
        return NULL;
    }
    OrSunny* m = (OrSunny*)calloc(1, sizeof(OrSunny));
    m->blocks = (float**)calloc((size_t)L * 16 + 16, sizeof(float*));
    m->ly = (OrLayer*)calloc((size_t)L, sizeof(OrLayer));
    m->vocab = vocab; m->D = D; m->I = I; m->R = R; m->K = K; m->L = L; m->G = G;
    m->clamp = clamp; m->nseq = nseq;
    int ok = 1;
    for (int l = 0; l < L && ok; ++l) {
        OrLayer* y = &m->ly[l];
        y->ni_g = sn_alloc(m, D); y->ni_c = sn_alloc(m, D);
        y->nm_g = sn_alloc(m, I); y->nm_c = sn_alloc(m, I);
        y->dw = sn_alloc(m, (size_t)K * D);
        y->V = sn_alloc(m, (size_t)R * D); y->U = sn_alloc(m, (size_t)2 * D * R);
        y->Wz = sn_alloc(m, (size_t)I * D); y->Wc = sn_alloc(m, (size_t)D * I);
        y->Ws = sn_alloc(m, (size_t)D * D); y->delta = sn_alloc(m, D);
        ok = rd(f, y->ni_g, 4 * (size_t)D) && rd(f, y->ni_c, 4 * (size_t)D) &&
             rd(f, y->nm_g, 4 * (size_t)I) && rd(f, y->nm_c, 4 * (size_t)I) &&
             rd(f, y->dw, 4 * (size_t)K * D);
        if (!ok) break;
        if (quant)
            ok = rd_q8(f, y->V, D, R) && rd_q8(f, y->U, R, 2 * D) && rd_q8(f, y->Wz, D, I) &&
                 rd_q8(f, y->Wc, I, D) && rd_q8(f, y->Ws, D, D);
        else
            ok = rd_flip(f, y->V, D, R) && rd_flip(f, y->U, R, 2 * D) &&
                 rd_flip(f, y->Wz, D, I) && rd_flip(f, y->Wc, I, D) && rd_flip(f, y->Ws, D, D);
        float sc2[2];
        ok = ok && rd(f, y->delta, 4 * (size_t)D) && rd(f, sc2, 8);
        y->a_tanh = sc2[0];
        y->b_gain = sc2[1];
    }
    float ep[2];
    m->no_g = sn_alloc(m, D);
    m->no_c = sn_alloc(m, D);
    m->embed = sn_alloc(m, (size_t)vocab * D);
    m->head = sn_alloc(m, (size_t)vocab * D);
    ok = ok && rd(f, ep, 8) && rd(f, m->no_g, 4 * (size_t)D) && rd(f, m->no_c, 4 * (size_t)D) &&
         rd(f, m->embed, 4 * (size_t)vocab * D);
    if (ok) ok = quant ? rd_q8(f, m->head, D, vocab) : rd_flip(f, m->head, D, vocab);
    fclose(f);
    m->eps = ep[0];
    m->p_floor = ep[1];
    const int KH = K > 1 ? K - 1 : 1;
    m->s = sn_alloc(m, (size_t)nseq * L * D);
    m->hist = sn_alloc(m, (size_t)nseq * L * KH * D);
    if (!ok || !m->s || !m->hist) { or_sn_free(m); return NULL; }
    return m;
}

void or_sn_free(OrSunny* m) {
    if (!m) return;
    for (int i = 0; i < m->nblocks; ++i) free(m->blocks[i]);
    free(m->blocks);
    free(m->ly);
    free(m);
}

void or_sn_reset(OrSunny* m) {
    const int KH = m->K > 1 ? m->K - 1 : 1;
    memset(m->s, 0, sizeof(float) * (size_t)m->nseq * m->L * m->D);
    memset(m->hist, 0, sizeof(float) * (size_t)m->nseq * m->L * KH * m->D);
}

int or_sn_vocab(const OrSunny* m) { return m ? m->vocab : 0; }

/* One layer for one sequence (sunnynet.c:212-291). sc holds 3D+R+2D+2D+2I+D floats. */
static void sn_layer(const OrSunny* m, const OrLayer* L, float* s, float* hist,
                     const float* x, float* out, float* sc, float* dbg) {
    const int D = m->D, I = m->I, R = m->R, K = m->K, G = m->G;
    float *raw = sc, *at = raw + D, *v = at + D, *q = v + R, *u = q + 2 * D, *gate = u + D;
    float *zn = gate + D, *yn = zn + I, *sfb = yn + I;
    layernorm(raw, x, L->ni_g, L->ni_c, D, m->eps);
    if (K > 1) {
        for (int i = 0; i < D; ++i) {
            float acc = raw[i] * L->dw[(size_t)(K - 1) * D + i];
            for (int k = 0; k < K - 1; ++k)
                acc = acc + hist[(size_t)k * D + i] * L->dw[(size_t)(K - 2 - k) * D + i];
            at[i] = raw[i] + acc;
        }
        for (int k = K - 2; k >= 1; --k)
            memcpy(hist + (size_t)k * D, hist + (size_t)(k - 1) * D, sizeof(float) * D);
        memcpy(hist, raw, sizeof(float) * D);
    } else {
        memcpy(at, raw, sizeof(float) * D);
    }
    const int par = m->row_par;
    gemv_sunny_p(v, at, L->V, D, R, par);
    gemv_sunny_p(q, v, L->U, R, 2 * D, par);
    memcpy(gate, q + D, sizeof(float) * D);
    for (int i = 0; i < D; ++i) {
        const int base = (i / G) * G, off = i - base;
        u[i] = q[i] * (sig(gate[i] - gate[base + (off + 1) % G]) *
                       sig(gate[i] - gate[base + (off + 2) % G]));
    }
    gemv_sunny_p(sfb, s, L->Ws, D, D, par); /* feedback reads the previous state */
    for (int i = 0; i < D; ++i) {
        float p = 1.0f - L->delta[i] * (1.0f - sig(gate[i]));
        if (m->clamp && p < m->p_floor) p = m->p_floor;
        s[i] = p * s[i] + (1.0f - p) * u[i];
    }
    gemv_sunny_p(zn, u, L->Wz, D, I, par);
    for (int i = 0; i < I; ++i) zn[i] = zn[i] * (1.0f + 0.5f * L->a_tanh / (1.0f + fabsf(zn[i])));
    layernorm(yn, zn, L->nm_g, L->nm_c, I, m->eps);
    gemv_sunny_p(out, yn, L->Wc, I, D, par);
    for (int i = 0; i < D; ++i) out[i] = out[i] + (L->b_gain * s[i] + sfb[i] + x[i]);
    if (dbg) {
        float* t = dbg;
        memcpy(t, raw, 4 * (size_t)D); t += D;
        memcpy(t, at, 4 * (size_t)D); t += D;
        memcpy(t, v, 4 * (size_t)R); t += R;
        memcpy(t, gate, 4 * (size_t)D); t += D;
        memcpy(t, u, 4 * (size_t)D); t += D;
        memcpy(t, s, 4 * (size_t)D); t += D;
        memcpy(t, zn, 4 * (size_t)I); t += I;
        memcpy(t, yn, 4 * (size_t)I); t += I;
        memcpy(t, sfb, 4 * (size_t)D); t += D;
        memcpy(t, out, 4 * (size_t)D);
    }
}

static size_t sn_scratch(const OrSunny* m) {
    return (size_t)3 * m->D + m->R + 4 * (size_t)m->D + 2 * (size_t)m->I + m->D + 3 * (size_t)m->D;
}

/* sunnynet.c:321-334 for sequence `seq`; stops after `last_layer` when >= 0. */
static void sn_seq(OrSunny* m, int seq, int token, float* logits, int last_layer, float* dbg,
                   float* sc) {
    const int D = m->D, KH = m->K > 1 ? m->K - 1 : 1;
    float *x = sc + sn_scratch(m) - 3 * (size_t)D, *lout = x + D, *nrm = lout + D;
    memcpy(x, m->embed + (size_t)token * D, sizeof(float) * D);
    const int nl = last_layer >= 0 ? last_layer + 1 : m->L;
    for (int l = 0; l < nl; ++l) {
        float* s = m->s + ((size_t)seq * m->L + l) * D;
        float* hist = m->hist + ((size_t)seq * m->L + l) * KH * D;
        sn_layer(m, &m->ly[l], s, hist, x, lout, sc, l == last_layer ? dbg : NULL);
        memcpy(x, lout, sizeof(float) * D);
    }
    if (last_layer >= 0 || !logits) return;
    layernorm(nrm, x, m->no_g, m->no_c, D, m->eps);
    gemv_sunny_p(logits, nrm, m->head, D, m->vocab, m->row_par);
}

/* Sequences in parallel when there are at least as many as threads; else one
 * at a time with each GEMV's rows spread over the threads. Either way every
 * value is computed by the same sequence of operations. */
void or_sn_step(OrSunny* m, const int32_t* tokens, float* logits) {
    if (m->nseq >= omp_get_max_threads()) {
#pragma omp parallel for schedule(static)
        for (int i = 0; i < m->nseq; ++i) {
            float* sc = (float*)malloc(sizeof(float) * sn_scratch(m));
            sn_seq(m, i, tokens[i], logits ? logits + (size_t)i * m->vocab : NULL, -1, NULL, sc);
            free(sc);
        }
        return;
    }
    float* sc = (float*)malloc(sizeof(float) * sn_scratch(m));
    m->row_par = 1;
    for (int i = 0; i < m->nseq; ++i)
        sn_seq(m, i, tokens[i], logits ? logits + (size_t)i * m->vocab : NULL, -1, NULL, sc);
    m->row_par = 0;
    free(sc);
}

void or_sn_dbg_layer(OrSunny* m, int token, int layer, float* dbg) {
    float* sc = (float*)malloc(sizeof(float) * sn_scratch(m));
    sn_seq(m, 0, token, NULL, layer, dbg, sc);
    free(sc);
}

void or_sn_get_state(const OrSunny* m, int seq, float* s, float* hist) {
    const int KH = m->K > 1 ? m->K - 1 : 1;
    memcpy(s, m->s + (size_t)seq * m->L * m->D, sizeof(float) * (size_t)m->L * m->D);
    memcpy(hist, m->hist + (size_t)seq * m->L * KH * m->D,
           sizeof(float) * (size_t)m->L * KH * m->D);
}

void or_sn_set_state(OrSunny* m, int seq, const float* s, const float* hist) {
    const int KH = m->K > 1 ? m->K - 1 : 1;
    memcpy(m->s + (size_t)seq * m->L * m->D, s, sizeof(float) * (size_t)m->L * m->D);
    memcpy(m->hist + (size_t)seq * m->L * KH * m->D, hist,
           sizeof(float) * (size_t)m->L * KH * m->D);
}

/* ====================================================== RWKV-7 whole model */
#define KRWK_MAGIC 0x4B57524B

typedef struct {
    int q4, in, out, block;
    float* w;      /* fp32 (in,out) */
    uint8_t* q;    /* INT4 (out,in/2) */
    float* scale;  /* (out,in/block), fp16 scales widened exactly */
} OrMat;

typedef struct {
    float *ln1w, *ln1b, *ln2w, *ln2b, *lerp;
    OrMat rw, kw, vw, ow, w1, w2, a1, a2, v1, v2, g1, g2, cmk, cmv;
    float *w0, *a0, *v0, *kk_w, *ka_w, *rk_w, *lnx_w, *lnx_b, *cmk_lerp;
    int Rw, Ra, Rv, Rg;
} OrRkLayer;

struct OrRwkv {
    int vocab, D, HS, NH, F, L, nseq;
    float eps;
    OrRkLayer* ly;
    float *en_w, *en_b, *on_w, *on_b, *embed;
    OrMat head;
    float* S;     /* (nseq,L,NH,HS,HS) */
    float* shift; /* (nseq,L,2,D) */
    unsigned char* buf;
};

typedef struct {
    const unsigned char *p, *end;
    int ok;
} Cur;

static const void* take(Cur* c, size_t n) {
    if (!c->ok || (size_t)(c->end - c->p) < n) { c->ok = 0; return NULL; }
    const void* r = c->p;
    c->p += n;
    return r;
}

static int take_i32(Cur* c) {
    const void* p = take(c, 4);
    int v = 0;
    if (p) memcpy(&v, p, 4);
    return v;
}

/* Tensors are copied out of the file buffer so every array is aligned. */
static float* take_vec(Cur* c, size_t n) {
    if (take_i32(c) != 0) c->ok = 0;
    const void* p = take(c, 4 * n);
    if (!p) return NULL;
    float* r = (float*)malloc(4 * n);
    memcpy(r, p, 4 * n);
    return r;
}

/* rwkv7.c:380-402 (tag 0 fp32 (in,out), tag 1 INT4 block 64 fp32 scales) plus
 * tag 2: INT4 group `group` with fp16 scales (this project's v4 format). */
static void take_mat(Cur* c, OrMat* M, int in, int out, int group) {
    const int tag = take_i32(c);
    memset(M, 0, sizeof(*M));
    M->in = in;
    M->out = out;
    if (tag == 0) {
        const void* p = take(c, (size_t)4 * in * out);
        if (!p) return;
        M->w = (float*)malloc((size_t)4 * in * out);
        memcpy(M->w, p, (size_t)4 * in * out);
    } else if (tag == 1 || tag == 2) {
        const int blk = tag == 1 ? 64 : group;
        if (blk <= 0 || in % blk) { c->ok = 0; return; }
        const size_t qb = (size_t)out * (in / 2), ns = (size_t)out * (in / blk);
        const void* q = take(c, qb);
        const void* s = take(c, ns * (tag == 1 ? 4 : 2));
        if (!q || !s) return;
        M->q4 = 1;
        M->block = blk;
        M->q = (uint8_t*)malloc(qb);
        memcpy(M->q, q, qb);
        M->scale = (float*)malloc(4 * ns);
        for (size_t i = 0; i < ns; ++i) M->scale[i] = scale_at(s, i, tag == 2);
    } else {
        c->ok = 0;
    }
}

static void free_mat(OrMat* M) {
    free(M->w);
    free(M->q);
    free(M->scale);
}

/* y = M x: fp32 (in,out) GEMV of rwkv7.c:89-121 or the W4A8 GEMV. */
static void mat_mul(float* y, const float* x, const OrMat* M) {
    if (M->q4) {
        or_gemv_i4(y, x, M->q, M->scale, M->in, M->out, M->block, 0);
        return;
    }
    const int in = M->in, out = M->out, ov = out - out % 8;
    for (int j = 0; j < out; ++j) {
        float acc = 0.0f;
        if (j < ov)
            for (int i = 0; i < in; ++i) acc = fmaf(x[i], M->w[(size_t)i * out + j], acc);
        else
            for (int i = 0; i < in; ++i) acc = acc + x[i] * M->w[(size_t)i * out + j];
        y[j] = acc;
    }
}

OrRwkv* or_rk_load(const char* path, int nseq) {
    if (nseq <= 0) return NULL;
    FILE* f = fopen(path, "rb");
    if (!f) return NULL;
    fseek(f, 0, SEEK_END);
    const long n = ftell(f);
    fseek(f, 0, SEEK_SET);
    unsigned char* buf = (unsigned char*)malloc((size_t)n);
    if (!buf || fread(buf, 1, (size_t)n, f) != (size_t)n) { free(buf); fclose(f); return NULL; }
    fclose(f);
    Cur c = {buf, buf + n, 1};
    int32_t h[10];
    for (int i = 0; i < 10; ++i) h[i] = take_i32(&c);
    if (!c.ok || h[0] != KRWK_MAGIC || (h[1] != 3 && h[1] != 4)) { free(buf); return NULL; }
    OrRwkv* m = (OrRwkv*)calloc(1, sizeof(OrRwkv));
    m->L = h[2]; m->D = h[3]; m->HS = h[4]; m->NH = h[5]; m->F = h[6]; m->vocab = h[8];
    m->nseq = nseq;
    m->buf = buf;
    const void* pe = take(&c, 4);
    if (pe) memcpy(&m->eps, pe, 4);
    const int group = h[1] == 4 ? take_i32(&c) : 64;
    const int L = m->L, D = m->D;
    if (!c.ok || L <= 0 || D <= 0 || m->HS <= 0 || m->HS % 8 || m->NH * m->HS != D) {
        free(buf);
        free(m);
        return NULL;
    }
    m->ly = (OrRkLayer*)calloc((size_t)L, sizeof(OrRkLayer));
    for (int l = 0; l < L; ++l) {
        OrRkLayer* A = &m->ly[l];
        A->Rw = take_i32(&c); A->Ra = take_i32(&c); A->Rv = take_i32(&c); A->Rg = take_i32(&c);
    }
    for (int l = 0; l < L && c.ok; ++l) {
        OrRkLayer* A = &m->ly[l];
        A->ln1w = take_vec(&c, D); A->ln1b = take_vec(&c, D);
        A->ln2w = take_vec(&c, D); A->ln2b = take_vec(&c, D);
        A->lerp = take_vec(&c, (size_t)6 * D);
        take_mat(&c, &A->rw, D, D, group); take_mat(&c, &A->kw, D, D, group);
        take_mat(&c, &A->vw, D, D, group); take_mat(&c, &A->ow, D, D, group);
        take_mat(&c, &A->w1, D, A->Rw, group); take_mat(&c, &A->w2, A->Rw, D, group);
        take_mat(&c, &A->a1, D, A->Ra, group); take_mat(&c, &A->a2, A->Ra, D, group);
        take_mat(&c, &A->v1, D, A->Rv, group); take_mat(&c, &A->v2, A->Rv, D, group);
        take_mat(&c, &A->g1, D, A->Rg, group); take_mat(&c, &A->g2, A->Rg, D, group);
        A->w0 = take_vec(&c, D); A->a0 = take_vec(&c, D); A->v0 = take_vec(&c, D);
        A->kk_w = take_vec(&c, D); A->ka_w = take_vec(&c, D); A->rk_w = take_vec(&c, D);
        A->lnx_w = take_vec(&c, D); A->lnx_b = take_vec(&c, D);
        take_mat(&c, &A->cmk, D, m->F, group); take_mat(&c, &A->cmv, m->F, D, group);
        A->cmk_lerp = take_vec(&c, D);
    }
    m->en_w = take_vec(&c, D); m->en_b = take_vec(&c, D);
    m->on_w = take_vec(&c, D); m->on_b = take_vec(&c, D);
    m->embed = take_vec(&c, (size_t)m->vocab * D);
    take_mat(&c, &m->head, D, m->vocab, group);
    m->S = (float*)calloc((size_t)nseq * L * m->NH * m->HS * m->HS, sizeof(float));
    m->shift = (float*)calloc((size_t)nseq * L * 2 * D, sizeof(float));
    if (!c.ok || !m->S || !m->shift) { or_rk_free(m); return NULL; }
    return m;
}

void or_rk_free(OrRwkv* m) {
    if (!m) return;
    if (m->ly)
        for (int l = 0; l < m->L; ++l) {
            OrRkLayer* A = &m->ly[l];
            float* v[] = {A->ln1w, A->ln1b, A->ln2w, A->ln2b, A->lerp, A->w0, A->a0, A->v0,
                          A->kk_w, A->ka_w, A->rk_w, A->lnx_w, A->lnx_b, A->cmk_lerp};
            for (size_t i = 0; i < sizeof(v) / sizeof(v[0]); ++i) free(v[i]);
            OrMat* mm[] = {&A->rw, &A->kw, &A->vw, &A->ow, &A->w1, &A->w2, &A->a1,
                           &A->a2, &A->v1, &A->v2, &A->g1, &A->g2, &A->cmk, &A->cmv};
            for (size_t i = 0; i < sizeof(mm) / sizeof(mm[0]); ++i) free_mat(mm[i]);
        }
    free(m->ly);
    free(m->en_w); free(m->en_b); free(m->on_w); free(m->on_b); free(m->embed);
    free_mat(&m->head);
    free(m->S);
    free(m->shift);
    free(m->buf);
    free(m);
}

void or_rk_reset(OrRwkv* m) {
    memset(m->S, 0, sizeof(float) * (size_t)m->nseq * m->L * m->NH * m->HS * m->HS);
    memset(m->shift, 0, sizeof(float) * (size_t)m->nseq * m->L * 2 * m->D);
}

int or_rk_vocab(const OrRwkv* m) { return m ? m->vocab : 0; }

/* rwkv7.c:143-189: per head, normalise kk, then per state row i
 *   proj = S_i . kk^ ; S_i <- S_i*w + (v_i k - proj (kk^ a)) ; y_i = S_i . r */
static void rk_heads(int HS, int NH, float* S, const float* w, const float* k, const float* v,
                     const float* a, const float* kk, const float* r, float* y) {
    float kn[512];
    for (int h = 0; h < NH; ++h) {
        float* Sh = S + (size_t)h * HS * HS;
        const int o = h * HS;
        float l8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int j = 0; j < HS; j += 8)
            for (int l = 0; l < 8; ++l) l8[l] = fmaf(kk[o + j + l], kk[o + j + l], l8[l]);
        float nrm = sqrtf(hsum8_tree(l8));
        if (!(nrm > 1e-12f)) nrm = 1e-12f;
        const float inv = 1.0f / nrm;
        for (int j = 0; j < HS; ++j) kn[j] = kk[o + j] * inv;
        for (int i = 0; i < HS; ++i) {
            float* row = Sh + (size_t)i * HS;
            float p8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int j = 0; j < HS; j += 8)
                for (int l = 0; l < 8; ++l) p8[l] = fmaf(row[j + l], kn[j + l], p8[l]);
            const float pv = hsum8_tree(p8), vi = v[o + i];
            float y8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int j = 0; j < HS; j += 8)
                for (int l = 0; l < 8; ++l) {
                    const int jj = j + l;
                    const float kka = kn[jj] * a[o + jj];
                    const float vk = vi * k[o + jj];
                    const float ns = fmaf(row[jj], w[o + jj], vk - pv * kka);
                    row[jj] = ns;
                    y8[l] = fmaf(ns, r[o + jj], y8[l]);
                }
            y[o + i] = hsum8_tree(y8);
        }
    }
}

#define RK_INV_SQRT_E 0.6065306597126334f /* rwkv7.c:33 */
#define RK_EPS_GROUP 6.4e-4f               /* rwkv7.c:34 */

/* rwkv7.c:191-320, one layer for one sequence. */
static void rk_layer(const OrRwkv* m, const OrRkLayer* A, int first, float* S, float* shift,
                     float* x, float* vfirst, float* sc, float* dbg) {
    const int D = m->D, HS = m->HS, NH = m->NH, F = m->F;
    float *xn = sc, *dd = xn + D, *xr = dd + D, *xw = xr + D, *xk = xw + D, *xv = xk + D;
    float *xa = xv + D, *xg = xa + D, *r = xg + D, *k = r + D, *v = k + D, *a = v + D;
    float *g = a + D, *kk = g + D, *ww = kk + D, *y = ww + D, *xn2 = y + D, *xk2 = xn2 + D;
    float *lo = xk2 + D, *ck = lo + 512, *cksq = ck + F;
    layernorm(xn, x, A->ln1w, A->ln1b, D, m->eps);
    for (int i = 0; i < D; ++i) dd[i] = shift[i] - xn[i];
    const float* lp = A->lerp;
    for (int i = 0; i < D; ++i) {
        const float d = dd[i];
        xr[i] = xn[i] + lp[i] * d;
        xw[i] = xn[i] + lp[D + i] * d;
        xk[i] = xn[i] + lp[2 * D + i] * d;
        xv[i] = xn[i] + lp[3 * D + i] * d;
        xa[i] = xn[i] + lp[4 * D + i] * d;
        xg[i] = xn[i] + lp[5 * D + i] * d;
    }
    mat_mul(r, xr, &A->rw);
    mat_mul(k, xk, &A->kw);
    mat_mul(v, xv, &A->vw);
    mat_mul(lo, xw, &A->w1);
    for (int i = 0; i < A->Rw; ++i) lo[i] = tanhf(lo[i]);
    mat_mul(dd, lo, &A->w2);
    for (int i = 0; i < D; ++i) ww[i] = expf(-sig(dd[i] + A->w0[i]) * RK_INV_SQRT_E);
    if (first) {
        memcpy(vfirst, v, sizeof(float) * D);
    } else {
        mat_mul(lo, xv, &A->v1);
        mat_mul(dd, lo, &A->v2);
        for (int i = 0; i < D; ++i) v[i] = v[i] + (vfirst[i] - v[i]) * sig(dd[i] + A->v0[i]);
    }
    mat_mul(lo, xa, &A->a1);
    mat_mul(dd, lo, &A->a2);
    for (int i = 0; i < D; ++i) a[i] = sig(dd[i] + A->a0[i]);
    mat_mul(lo, xg, &A->g1);
    for (int i = 0; i < A->Rg; ++i) lo[i] = sig(lo[i]);
    mat_mul(g, lo, &A->g2);
    for (int i = 0; i < D; ++i) {
        kk[i] = k[i] * A->kk_w[i];
        k[i] = k[i] + k[i] * (a[i] - 1.0f) * A->ka_w[i];
    }
    rk_heads(HS, NH, S, ww, k, v, a, kk, r, y);
    for (int h = 0; h < NH; ++h) {
        float *yh = y + h * HS;
        const int o = h * HS;
        float mean = 0.0f;
        for (int i = 0; i < HS; ++i) mean = mean + yh[i];
        mean = mean / (float)HS;
        float var = 0.0f;
        for (int i = 0; i < HS; ++i) {
            const float t = yh[i] - mean;
            var = var + t * t;
        }
        const float rstd = 1.0f / sqrtf(var / (float)HS + RK_EPS_GROUP);
        float dot = 0.0f;
        for (int i = 0; i < HS; ++i) dot = dot + r[o + i] * k[o + i] * A->rk_w[o + i];
        for (int i = 0; i < HS; ++i) {
            const float nv = (yh[i] - mean) * rstd * A->lnx_w[o + i] + A->lnx_b[o + i];
            yh[i] = (nv + dot * v[o + i]) * g[o + i];
        }
    }
    mat_mul(dd, y, &A->ow);
    for (int i = 0; i < D; ++i) x[i] = x[i] + dd[i];
    memcpy(shift, xn, sizeof(float) * D);
    layernorm(xn2, x, A->ln2w, A->ln2b, D, m->eps);
    for (int i = 0; i < D; ++i) xk2[i] = xn2[i] + A->cmk_lerp[i] * (shift[D + i] - xn2[i]);
    mat_mul(ck, xk2, &A->cmk);
    for (int i = 0; i < F; ++i) {
        const float t = ck[i] > 0.0f ? ck[i] : 0.0f;
        cksq[i] = t * t;
    }
    mat_mul(dd, cksq, &A->cmv);
    for (int i = 0; i < D; ++i) x[i] = x[i] + dd[i];
    memcpy(shift + D, xn2, sizeof(float) * D);
    if (dbg) {
        const float* src[9] = {xn, r, k, v, a, g, ww, y, x};
        for (int i = 0; i < 9; ++i) memcpy(dbg + (size_t)i * D, src[i], sizeof(float) * D);
    }
}

static size_t rk_scratch(const OrRwkv* m) { return (size_t)21 * m->D + 512 + 2 * (size_t)m->F; }

/* rwkv7.c:349-360 for one sequence. */
static void rk_seq(OrRwkv* m, int seq, int token, float* logits, int last_layer, float* dbg,
                   float* sc) {
    const int D = m->D, L = m->L;
    float *x = sc + rk_scratch(m) - 3 * (size_t)D, *nrm = x + D, *vfirst = nrm + D;
    memcpy(x, m->embed + (size_t)token * D, sizeof(float) * D);
    layernorm(x, x, m->en_w, m->en_b, D, m->eps);
    const int nl = last_layer >= 0 ? last_layer + 1 : L;
    const size_t sz = (size_t)m->NH * m->HS * m->HS;
    for (int l = 0; l < nl; ++l)
        rk_layer(m, &m->ly[l], l == 0, m->S + ((size_t)seq * L + l) * sz,
                 m->shift + ((size_t)seq * L + l) * 2 * D, x, vfirst, sc,
                 l == last_layer ? dbg : NULL);
    if (last_layer >= 0 || !logits) return;
    layernorm(nrm, x, m->on_w, m->on_b, D, m->eps);
    mat_mul(logits, nrm, &m->head);
}

void or_rk_step(OrRwkv* m, const int32_t* tokens, float* logits) {
#pragma omp parallel for schedule(static)
    for (int i = 0; i < m->nseq; ++i) {
        float* sc = (float*)malloc(sizeof(float) * rk_scratch(m));
        rk_seq(m, i, tokens[i], logits ? logits + (size_t)i * m->vocab : NULL, -1, NULL, sc);
        free(sc);
    }
}

void or_rk_dbg(OrRwkv* m, int token, int layer, float* out) {
    float* sc = (float*)malloc(sizeof(float) * rk_scratch(m));
    rk_seq(m, 0, token, NULL, layer, out, sc);
    free(sc);
}

void or_rk_set_state(OrRwkv* m, int seq, const float* S, const float* shift) {
    const size_t sz = (size_t)m->L * m->NH * m->HS * m->HS;
    memcpy(m->S + (size_t)seq * sz, S, sizeof(float) * sz);
    memcpy(m->shift + (size_t)seq * m->L * 2 * m->D, shift, sizeof(float) * (size_t)m->L * 2 * m->D);
}

/* One step in which layer l of sequence i starts from xs_in[i][l] (the input
 * another implementation fed that layer) instead of this oracle's own layer
 * l-1 output: xs_out[i][0] = the embedding row after its norm, xs_out[i][l+1]
 * = layer l applied to xs_in[i][l] (states updated as in a normal step; the
 * v-first vector comes from layer 0 applied to xs_in[i][0]); logits from the
 * final norm and head applied to xs_in[i][L]. xs_* are (nseq, L+1, D). */
void or_rk_step_forced(OrRwkv* m, const int32_t* tokens, const float* xs_in, float* xs_out,
                       float* logits) {
    const int D = m->D, L = m->L;
    const size_t sz = (size_t)m->NH * m->HS * m->HS;
#pragma omp parallel for schedule(static)
    for (int i = 0; i < m->nseq; ++i) {
        float* sc = (float*)malloc(sizeof(float) * rk_scratch(m));
        float *x = sc + rk_scratch(m) - 3 * (size_t)D, *nrm = x + D, *vfirst = nrm + D;
        const float* in = xs_in + (size_t)i * (L + 1) * D;
        float* out = xs_out + (size_t)i * (L + 1) * D;
        memcpy(x, m->embed + (size_t)tokens[i] * D, sizeof(float) * D);
        layernorm(out, x, m->en_w, m->en_b, D, m->eps);
        for (int l = 0; l < L; ++l) {
            memcpy(x, in + (size_t)l * D, sizeof(float) * D);
            rk_layer(m, &m->ly[l], l == 0, m->S + ((size_t)i * L + l) * sz,
                     m->shift + ((size_t)i * L + l) * 2 * D, x, vfirst, sc, NULL);
            memcpy(out + (size_t)(l + 1) * D, x, sizeof(float) * D);
        }
        if (logits) {
            layernorm(nrm, in + (size_t)L * D, m->on_w, m->on_b, D, m->eps);
            mat_mul(logits + (size_t)i * m->vocab, nrm, &m->head);
        }
        free(sc);
    }
}

void or_rk_get_state(const OrRwkv* m, int seq, float* S, float* shift) {
    const size_t sz = (size_t)m->L * m->NH * m->HS * m->HS;
    memcpy(S, m->S + (size_t)seq * sz, sizeof(float) * sz);
    memcpy(shift, m->shift + (size_t)seq * m->L * 2 * m->D, sizeof(float) * (size_t)m->L * 2 * m->D);
}

/* ------------------------------------------- kernels module (sunnynet/kernels)
 * Restatements of the reference's AVX2 training/step kernels, one lane at a
 * time in the same operation order. These files are compiled as GNU C (no
 * -std=c11, kernels/__init__.py:24-36), which would allow the compiler to
 * contract the N % 8 scalar tails into FMAs; the reference build leaves them
 * as separate multiply and add, which these restatements follow and the
 * tests check against the reference library built with its own flags. */

/* core_avx2.c:17-18 lane rolls within a group of 8: v[i+1], v[i+2], v[i-1], v[i-2] */
#define GRP(i, k) (((i) & ~7) + ((((i) & 7) + (k) + 8) & 7))

/* core_avx2.c:34-79: q (B,T,2D) = [u_raw | gate], delta (D), s0 (B,D) ->
 * states, u, p (B,T,D). Groups of 8 channels (D % 8 channels are not written). */
void or_core_fwd(const float* q, const float* delta, const float* s0, float* states, float* uo,
                 float* po, int B, int T, int D) {
    const int DV = D & ~7;
#pragma omp parallel for schedule(static)
    for (int b = 0; b < B; ++b) {
        float* s = (float*)malloc(sizeof(float) * (DV > 0 ? DV : 1));
        float* e = (float*)malloc(sizeof(float) * (DV > 0 ? DV : 1));
        for (int d = 0; d < DV; ++d) s[d] = s0[(size_t)b * D + d];
        for (int t = 0; t < T; ++t) {
            const float* qt = q + ((size_t)b * T + t) * 2 * D;
            const size_t o = ((size_t)b * T + t) * D;
            for (int d = 0; d < DV; ++d) e[d] = expf(0.0f - qt[D + d]);
            for (int d = 0; d < DV; ++d) {
                const float sig = 1.0f / (1.0f + e[d]);
                const float s1 = 1.0f / (1.0f + e[d] / e[GRP(d, 1)]);
                const float s2 = 1.0f / (1.0f + e[d] / e[GRP(d, 2)]);
                const float w = s1 * s2;
                const float u = qt[d] * w;
                const float p = fmaf(delta[d], sig, 1.0f - delta[d]);
                s[d] = fmaf(p, s[d], (1.0f - p) * u);
                states[o + d] = s[d];
                uo[o + d] = u;
                po[o + d] = p;
            }
        }
        free(s);
        free(e);
    }
}

/* core_avx2.c:84-148: reverse pass. ddelta is accumulated (+=) over the
 * sequences in order b = 0, 1, ... (the reference adds them with OpenMP
 * atomics in whatever order its threads finish). */
void or_core_bwd(const float* q, const float* delta, const float* s0, const float* states,
                 const float* uo, const float* po, const float* dstate, const float* du_in,
                 float* dq, float* ddelta, float* ds0, int B, int T, int D) {
    const int DV = D & ~7;
    float* acc = (float*)calloc((size_t)B * (DV > 0 ? DV : 1), sizeof(float));
#pragma omp parallel for schedule(static)
    for (int b = 0; b < B; ++b) {
        const size_t n = DV > 0 ? DV : 1;
        float* ds = (float*)calloc(n, sizeof(float));
        float* e = (float*)malloc(sizeof(float) * n);
        float* a1 = (float*)malloc(sizeof(float) * n);
        float* a2 = (float*)malloc(sizeof(float) * n);
        float* dp = (float*)malloc(sizeof(float) * n);
        float* sg = (float*)malloc(sizeof(float) * n);
        float* dacc = acc + (size_t)b * n;
        for (int t = T - 1; t >= 0; --t) {
            const size_t qo = ((size_t)b * T + t) * 2 * D;
            const size_t o = ((size_t)b * T + t) * D;
            for (int d = 0; d < DV; ++d) e[d] = expf(0.0f - q[qo + D + d]);
            for (int d = 0; d < DV; ++d) {
                ds[d] = ds[d] + dstate[o + d];
                const float u = uo[o + d], p = po[o + d];
                const float sprev = t > 0 ? states[o - D + d] : s0[(size_t)b * D + d];
                dp[d] = ds[d] * (sprev - u);
                const float du = fmaf(ds[d], 1.0f - p, du_in[o + d]);
                ds[d] = ds[d] * p;
                const float ur = q[qo + d];
                const float sig = 1.0f / (1.0f + e[d]);
                const float s1 = 1.0f / (1.0f + e[d] / e[GRP(d, 1)]);
                const float s2 = 1.0f / (1.0f + e[d] / e[GRP(d, 2)]);
                const float w = s1 * s2;
                dq[qo + d] = du * w;
                const float dw = du * ur;
                const float ds1 = dw * s2, ds2 = dw * s1;
                a1[d] = ds1 * (s1 * (1.0f - s1));
                a2[d] = ds2 * (s2 * (1.0f - s2));
                sg[d] = sig;
            }
            for (int d = 0; d < DV; ++d) {
                float dg = a1[d] + a2[d];
                dg = dg - a1[GRP(d, -1)];
                dg = dg - a2[GRP(d, -2)];
                dg = fmaf(dp[d] * delta[d], sg[d] * (1.0f - sg[d]), dg);
                dacc[d] = fmaf(dp[d], sg[d] - 1.0f, dacc[d]);
                dq[qo + D + d] = dg;
            }
        }
        for (int d = 0; d < DV; ++d) ds0[(size_t)b * D + d] = ds[d];
        free(ds); free(e); free(a1); free(a2); free(dp); free(sg);
    }
    for (int b = 0; b < B; ++b)
        for (int d = 0; d < DV; ++d) ddelta[d] = ddelta[d] + acc[(size_t)b * DV + d];
    free(acc);
}

/* step_avx2.c:54-86: one step of core_fwd: q (B,2D), s (B,D) -> s_new, u (B,D). */
void or_step_core(const float* q, const float* delta, const float* s, float* s_new, float* uo,
                  int B, int D) {
    const int DV = D & ~7;
    float* e = (float*)malloc(sizeof(float) * (DV > 0 ? DV : 1));
    for (int b = 0; b < B; ++b) {
        const float* qb = q + (size_t)b * 2 * D;
        for (int d = 0; d < DV; ++d) e[d] = expf(0.0f - qb[D + d]);
        for (int d = 0; d < DV; ++d) {
            const float sig = 1.0f / (1.0f + e[d]);
            const float s1 = 1.0f / (1.0f + e[d] / e[GRP(d, 1)]);
            const float s2 = 1.0f / (1.0f + e[d] / e[GRP(d, 2)]);
            const float u = qb[d] * (s1 * s2);
            const float p = fmaf(delta[d], sig, 1.0f - delta[d]);
            uo[(size_t)b * D + d] = u;
            s_new[(size_t)b * D + d] = fmaf(p, s[(size_t)b * D + d], (1.0f - p) * u);
        }
    }
    free(e);
}

/* step_avx2.c:24-50: acc = w[K-1]*x + sum_j w[K-2-j]*hist[j]: an FMA chain
 * on the 8-wide lanes, separate multiply and add on the D % 8 tail (the
 * reference build leaves that scalar loop uncontracted; pinned by test). */
void or_dw_step(const float* x, const float* hist, const float* w, float* acc, int B, int D,
                int taps) {
    const int k = taps - 1, DV = D & ~7;
    for (int b = 0; b < B; ++b)
        for (int d = 0; d < D; ++d) {
            float a = x[(size_t)b * D + d] * w[(size_t)(taps - 1) * D + d];
            for (int j = 0; j < k; ++j) {
                const float hv = hist[((size_t)b * k + j) * D + d];
                const float wv = w[(size_t)(taps - 2 - j) * D + d];
                if (d < DV) {
                    a = fmaf(hv, wv, a);
                } else {
                    const float m = hv * wv;
                    a = a + m;
                }
            }
            acc[(size_t)b * D + d] = a;
        }
}
/* scan_avx2.c:12-45 scan_f32: the gated scan with (a, u) = (p, nu); the
 * reference build contracts its N % 8 tail to fma(p, s, (1-p)*nu), the lane
 * rule, so every channel follows it. */
void or_scan_f32(const float* p, const float* nu, const float* s0, float* out, float* send,
                 int B, int T, int N) {
#pragma omp parallel for schedule(static)
    for (int bb = 0; bb < B; ++bb)
        for (int d = 0; d < N; ++d) {
            float s = s0[(size_t)bb * N + d];
            for (int t = 0; t < T; ++t) {
                const size_t o = ((size_t)bb * T + t) * N + d;
                s = fmaf(p[o], s, (1.0f - p[o]) * nu[o]);
                out[o] = s;
            }
            send[(size_t)bb * N + d] = s;
        }
}
#undef GRP
