// The SIMT W4A8 contraction rows (sn_gemv_i4 semantics, bit for bit), shared
// by the launch-per-contraction kernels (quant4.cu) and the fused RWKV-7
// decode step (rwkv7.cu).
//
// Reference: sunnynet/runtime/quant.c (sn_gemv_i4 89-154). The activation is
// quantised per block (sc = amax/127, 1 if zero; q = rint(x/sc) clamped to
// +-127), each (row, block) integer dot sum_k q_w[k]*q_x[k] is exact (dp4a on
// nibble bytes, integer shuffles), and the row accumulates
// acc = acc + (s_w*s_x)*(float)(dot - 8*sum q_x) block by block in block
// order with round-to-nearest mul/add and no contraction.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.cuh"
#include "ptx.cuh"

namespace sn {
namespace {

__device__ __forceinline__ float load_scale(const void* s, size_t i, bool fp16) {
    return fp16 ? __half2float(reinterpret_cast<const __half*>(s)[i])
                : reinterpret_cast<const float*>(s)[i];
}

// ------------------------------------------------------- activation quant
// Quantise NB activation rows (in floats each) into shared memory:
// xq[NB][in] int8, xs[NB][nb] scale, xsum[NB][nb] integer sums. Warp per block.
__device__ void quant_act_smem(const float* __restrict__ X, int nseq, int in, int block, int nb,
                               int8_t* xq, float* xs, int* xsum) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int w = warp; w < nseq * nb; w += nw) {
        const int s = w / nb, b = w % nb;
        const float* xb = X + (size_t)s * in + (size_t)b * block;
        float m = 0.0f;
        for (int i = lane; i < block; i += 32) m = fmaxf(m, fabsf(xb[i]));
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const float sc = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;
        const float inv = __fdiv_rn(1.0f, sc);
        int sum = 0;
        for (int i = lane; i < block; i += 32) {
            int t = __float2int_rn(__fmul_rn(xb[i], inv));
            t = min(max(t, -127), 127);
            xq[(size_t)s * in + (size_t)b * block + i] = (int8_t)t;
            sum += t;
        }
        for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) {
            xs[s * nb + b] = sc;
            xsum[s * nb + b] = sum;
        }
    }
}

// The same quantisation with one thread per 16 consecutive activations
// (four 16-byte loads, one 16-byte store of codes) and the block's
// block/16 threads combining its max and code sum by shuffles. Max and integer
// sums are exact in any order, so the codes, scales and sums are those of
// quant_act_smem. Needs block a power of two in [32, 512], in % block == 0
// and X 16-byte aligned.
__device__ void quant_act_smem16(const float* __restrict__ X, int nseq, int in, int block,
                                 int8_t* xq, float* xs, int* xsum) {
    const int L = block >> 4;  // threads per block, a power of two dividing 32
    const int lane = threadIdx.x & 31, ngr = nseq * (in >> 4);
    for (int base = threadIdx.x & ~31; base < ngr; base += blockDim.x) {
        const int g = base + lane;  // groups of a block never straddle g == ngr
        const bool live = g < ngr;
        float x[16];
        float m = 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            float4 t = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (live) t = reinterpret_cast<const float4*>(X)[(size_t)g * 4 + k];
            x[4 * k] = t.x;
            x[4 * k + 1] = t.y;
            x[4 * k + 2] = t.z;
            x[4 * k + 3] = t.w;
        }
#pragma unroll
        for (int k = 0; k < 16; ++k) m = fmaxf(m, fabsf(x[k]));
        for (int o = 1; o < L; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const float sc = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;
        const float inv = __fdiv_rn(1.0f, sc);
        int sum = 0;
        unsigned w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            unsigned packed = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                int t = __float2int_rn(__fmul_rn(x[4 * k + j], inv));
                t = min(max(t, -127), 127);
                sum += t;
                packed |= (unsigned)(t & 0xff) << (8 * j);
            }
            w[k] = packed;
        }
        if (live) reinterpret_cast<uint4*>(xq)[g] = make_uint4(w[0], w[1], w[2], w[3]);
        for (int o = 1; o < L; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (live && (lane & (L - 1)) == 0) {
            xs[g / L] = sc;  // block index s * nb + b = element index / block
            xsum[g / L] = sum;
        }
    }
}

__device__ __forceinline__ int dot16(uint4 w, const int8_t* xlo, const int8_t* xhi) {
    const int4 a = *reinterpret_cast<const int4*>(xlo);
    const int4 c = *reinterpret_cast<const int4*>(xhi);
    int d = 0;
    d = __dp4a((int)(w.x & 0x0F0F0F0Fu), a.x, d);
    d = __dp4a((int)((w.x >> 4) & 0x0F0F0F0Fu), c.x, d);
    d = __dp4a((int)(w.y & 0x0F0F0F0Fu), a.y, d);
    d = __dp4a((int)((w.y >> 4) & 0x0F0F0F0Fu), c.y, d);
    d = __dp4a((int)(w.z & 0x0F0F0F0Fu), a.z, d);
    d = __dp4a((int)((w.z >> 4) & 0x0F0F0F0Fu), c.z, d);
    d = __dp4a((int)(w.w & 0x0F0F0F0Fu), a.w, d);
    d = __dp4a((int)((w.w >> 4) & 0x0F0F0F0Fu), c.w, d);
    return d;
}

constexpr int kMaxSeqTile = 8;

// Output epilogues (the RWKV-7 layer fuses these into its GEMVs):
// store | accumulate into Y (x += W y, rwkv7.c:292,306) | relu^2 | tanh | sigmoid
__device__ __forceinline__ void w4_store(float* y, float v, int epi) {
    switch (epi) {
        case kW4Add: *y = __ldcg(y) + v; break;  // L2: other CTAs may have written it
        case kW4Relu2: {
            const float t = v > 0.0f ? v : 0.0f;
            *y = t * t;
        } break;
        case kW4Tanh: *y = tanhf(v); break;
        case kW4Sigmoid: *y = 1.0f / (1.0f + expf(-v)); break;
        default: *y = v;
    }
}

// Fast path: block % 32 == 0 (whole 16-byte chunks per block half), in % 32 == 0,
// in <= 1024 * NCH (a 16-byte chunk holds 32 codes; NCH chunk passes of 32
// lanes per row). A warp takes kW4Rows output rows at a time
// (rows gw, gw + nw, ...): the 16-byte weight chunks and block scales of all
// of them are loaded before any is used, and the first group's before the
// activations are quantised (they do not depend on the previous kernel), so
// the weight stream has several rows in flight per warp. NS sequences share
// each weight load. The per-row arithmetic is the reference's, in its order.
constexpr int kW4Rows = 4;
//
// w4a8_rows_p: rows gw, gw + nw, ... of the contraction for the ns <= NSX
// (<= 8) activation rows from seq0 on, with the quantised activations in
// `smem` ([kMaxSeqTile][in] codes, then scales and code sums). `pro` runs
// after the first rows' weights are requested and returns the activation rows
// (ns x in floats, global or shared memory): it performs whatever wait they
// need. With NSX == 1 each lane keeps its row-invariant operands (its 32
// activation codes, the block's scale and 8 x code sum) in registers, so a
// row costs its weight chunk's dot products, the block combination and one
// store: the same operations on the same values, in the same order.
template <bool FP16S, int NCH, int NSX = kMaxSeqTile, class Pro>
__device__ __forceinline__ void w4a8_rows_p(float* __restrict__ Y, const uint8_t* __restrict__ Wq,
                                            const void* __restrict__ scale, int ns, int seq0,
                                            int in, int out, int block, int epi, int gw, int nw,
                                            unsigned char* smem, Pro pro) {
    const int nb = in / block, half = block / 2, cpb = half / 16, cpr = in / 32;
    const int nch = (cpr + 31) / 32;  // chunk passes per row (<= NCH)
    int8_t* xq = reinterpret_cast<int8_t*>(smem);
    float* xs = reinterpret_cast<float*>(smem + (size_t)kMaxSeqTile * in);
    int* xsum = reinterpret_cast<int*>(xs + kMaxSeqTile * nb);
    const int lane = threadIdx.x & 31;
    // Weight chunks and the raw bits of their block scales: predicated loads
    // into zeroed registers, nothing that waits for the data until it is used,
    // so a warp's requests all leave before its first use.
    uint4 wr[kW4Rows][NCH];
    unsigned swr[kW4Rows][NCH];
    auto load_rows = [&](int row0) {  // rows row0 + i*nw, i < kW4Rows
#pragma unroll
        for (int i = 0; i < kW4Rows; ++i) {
            const int row = row0 + i * nw;
#pragma unroll
            for (int c = 0; c < NCH; ++c) {
                const int ci = c * 32 + lane;
                const bool live = c < nch && ci < cpr && row < out;
                wr[i][c] = make_uint4(0, 0, 0, 0);
                swr[i][c] = 0u;
                if (live) {
                    wr[i][c] = __ldg(reinterpret_cast<const uint4*>(Wq + (size_t)row * (in / 2)) + ci);
                    const size_t si = (size_t)row * nb + ci / cpb;
                    swr[i][c] = FP16S ? (unsigned)__ldg(reinterpret_cast<const unsigned short*>(scale) + si)
                                      : __ldg(reinterpret_cast<const unsigned*>(scale) + si);
                }
            }
        }
    };
    auto scale_of = [](unsigned raw) {
        return FP16S ? __half2float(__ushort_as_half((unsigned short)raw)) : __uint_as_float(raw);
    };
    load_rows(gw);
    const float* X = pro();
    if (((uintptr_t)X & 15) == 0 && block >= 32 && block <= 512 && (block & (block - 1)) == 0)
        quant_act_smem16(X, ns, in, block, xq, xs, xsum);
    else
        quant_act_smem(X, ns, in, block, nb, xq, xs, xsum);
    __syncthreads();

    if constexpr (NSX == 1) {
        int4 xlo[NCH], xhi[NCH];
        float xsc[NCH];
        int xs8[NCH], nbk[NCH];
        bool lv[NCH];
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
            const int ci = c * 32 + lane;
            lv[c] = c < nch && ci < cpr;
            const int b = lv[c] ? ci / cpb : 0;
            const int j = (ci % cpb) * 16;
            xlo[c] = make_int4(0, 0, 0, 0);
            xhi[c] = make_int4(0, 0, 0, 0);
            xsc[c] = 0.0f;
            xs8[c] = 0;
            if (lv[c]) {
                xlo[c] = *reinterpret_cast<const int4*>(xq + b * block + j);
                xhi[c] = *reinterpret_cast<const int4*>(xq + b * block + half + j);
                xsc[c] = xs[b];
                xs8[c] = 8 * xsum[b];
            }
            nbk[c] = c < nch ? min(32, cpr - c * 32) / cpb : 0;  // whole blocks in the pass
        }
        // A row's block sum for chunk pass c: integer dot products over the
        // block's cpb (1, 2, 4 or 8) lanes, then the block term.
        auto term = [&](const uint4& w, unsigned sraw, int c) {
            int d = 0;  // dot16's order: (low, high) nibbles of each word
            d = __dp4a((int)(w.x & 0x0F0F0F0Fu), xlo[c].x, d);
            d = __dp4a((int)((w.x >> 4) & 0x0F0F0F0Fu), xhi[c].x, d);
            d = __dp4a((int)(w.y & 0x0F0F0F0Fu), xlo[c].y, d);
            d = __dp4a((int)((w.y >> 4) & 0x0F0F0F0Fu), xhi[c].y, d);
            d = __dp4a((int)(w.z & 0x0F0F0F0Fu), xlo[c].z, d);
            d = __dp4a((int)((w.z >> 4) & 0x0F0F0F0Fu), xhi[c].z, d);
            d = __dp4a((int)(w.w & 0x0F0F0F0Fu), xlo[c].w, d);
            d = __dp4a((int)((w.w >> 4) & 0x0F0F0F0Fu), xhi[c].w, d);
            if (!lv[c]) d = 0;
            int t = __shfl_xor_sync(0xffffffffu, d, 1);
            d += cpb > 1 ? t : 0;
            t = __shfl_xor_sync(0xffffffffu, d, 2);
            d += cpb > 2 ? t : 0;
            t = __shfl_xor_sync(0xffffffffu, d, 4);
            d += cpb > 4 ? t : 0;
            return lv[c] ? __fmul_rn(__fmul_rn(scale_of(sraw), xsc[c]), (float)(d - xs8[c])) : 0.0f;
        };
        for (int row0 = gw; row0 < out; row0 += kW4Rows * nw) {
            if (row0 + (kW4Rows - 1) * nw < out) {
                // a full group: its rows side by side, so their dot products,
                // block terms and in-order block sums interleave
                float acc[kW4Rows];
#pragma unroll
                for (int i = 0; i < kW4Rows; ++i) acc[i] = 0.0f;
#pragma unroll
                for (int c = 0; c < NCH; ++c) {
                    if (c >= nch) break;
                    float fb[kW4Rows];
#pragma unroll
                    for (int i = 0; i < kW4Rows; ++i) fb[i] = term(wr[i][c], swr[i][c], c);
                    for (int k = 0; k < nbk[c]; ++k) {
#pragma unroll
                        for (int i = 0; i < kW4Rows; ++i)
                            acc[i] = __fadd_rn(acc[i], __shfl_sync(0xffffffffu, fb[i], k * cpb));
                    }
                }
                if (lane == 0 && ns > 0) {
#pragma unroll
                    for (int i = 0; i < kW4Rows; ++i)
                        w4_store(Y + (size_t)seq0 * out + row0 + i * nw, acc[i], epi);
                }
            } else {
#pragma unroll
                for (int i = 0; i < kW4Rows; ++i) {  // the last, partial group: row by row
                    const int row = row0 + i * nw;
                    if (row >= out) break;
                    float acc = 0.0f;
#pragma unroll
                    for (int c = 0; c < NCH; ++c) {
                        if (c >= nch) break;
                        const float fb = term(wr[i][c], swr[i][c], c);
#pragma unroll 4
                        for (int k = 0; k < nbk[c]; ++k)
                            acc = __fadd_rn(acc, __shfl_sync(0xffffffffu, fb, k * cpb));
                    }
                    if (lane == 0 && ns > 0) w4_store(Y + (size_t)seq0 * out + row, acc, epi);
                }
            }
            if (row0 + kW4Rows * nw < out) load_rows(row0 + kW4Rows * nw);
        }
        return;
    }

    for (int row0 = gw; row0 < out; row0 += kW4Rows * nw) {
#pragma unroll
        for (int i = 0; i < kW4Rows; ++i) {
            const int row = row0 + i * nw;
            if (row >= out) break;
            float acc[kMaxSeqTile];
#pragma unroll
            for (int s = 0; s < kMaxSeqTile; ++s) acc[s] = 0.0f;
#pragma unroll
            for (int c = 0; c < NCH; ++c) {
                if (c >= nch) break;
                const int c0 = c * 32, ci = c0 + lane;
                const bool live = ci < cpr;
                const uint4 w = wr[i][c];
                const int b = live ? ci / cpb : 0;
                const int j = (ci % cpb) * 16;
                const int nblk = min(32, cpr - c0) / cpb;  // whole blocks in this pass
#pragma unroll
                for (int s = 0; s < kMaxSeqTile; ++s) {
                    if (s >= ns) break;
                    int d = live ? dot16(w, xq + (size_t)s * in + b * block + j,
                                         xq + (size_t)s * in + b * block + half + j)
                                 : 0;
                    for (int o = 1; o < cpb; o <<= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
                    // every lane of block b's group forms the block's term; the
                    // terms are then added in block order (same value in every lane)
                    const float fb =
                        live ? __fmul_rn(__fmul_rn(scale_of(swr[i][c]), xs[s * nb + b]),
                                         (float)(d - 8 * xsum[s * nb + b]))
                             : 0.0f;
#pragma unroll 4
                    for (int k = 0; k < nblk; ++k)
                        acc[s] = __fadd_rn(acc[s], __shfl_sync(0xffffffffu, fb, k * cpb));
                }
            }
            if (lane < ns) {
                float v = acc[0];
#pragma unroll
                for (int s = 1; s < kMaxSeqTile; ++s)
                    if (lane == s) v = acc[s];
                w4_store(Y + (size_t)(seq0 + lane) * out + row, v, epi);
            }
        }
        if (row0 + kW4Rows * nw < out) load_rows(row0 + kW4Rows * nw);
    }
}


// The launch-per-contraction form: sequence tile blockIdx.y, activations
// read after the programmatic wait for the previous kernel.
template <bool FP16S, int NCH>
__device__ __forceinline__ void w4a8_rows(float* __restrict__ Y, const float* __restrict__ X,
                                          const uint8_t* __restrict__ Wq,
                                          const void* __restrict__ scale, int nseq, int in,
                                          int out, int block, int epi, int gw, int nw) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int seq0 = blockIdx.y * kMaxSeqTile;
    const int ns = min(kMaxSeqTile, nseq - seq0);
    pdl_trigger();
    w4a8_rows_p<FP16S, NCH>(Y, Wq, scale, ns, seq0, in, out, block, epi, gw, nw, smem, [&] {
        pdl_wait();  // no-op unless launched with programmatic serialization
        return X + (size_t)seq0 * in;
    });
}

constexpr int kW4MaxProblems = 8;

}  // namespace
}  // namespace sn
