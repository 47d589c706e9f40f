/* Group-symmetric INT4 weights and the W4A8 GEMV, internal symbol set of the
 * reference's sunnynet/runtime/quant.h:20-30 (same signatures, fp32 scales,
 * (out,in) row-major codes, byte k of a group = value k | value k+block/2 << 4).
 * Array arguments may be host or device pointers (see sn_abi.h). */
#ifndef SN_QUANT_H
#define SN_QUANT_H

#ifdef __cplusplus
extern "C" {
#endif

#define SN_I4_BLOCK 64

/* quant.h:20-23 */
void sn_quant_i4(const float* x, unsigned char* q, float* scale, int rows, int N, int block);
void sn_dequant_i4(const unsigned char* q, const float* scale, float* x, int rows, int N,
                   int block);
/* quant.h:26-27. in % block != 0 (where the reference reinterprets the INT4
 * bytes as fp32, quant.c:92) leaves y untouched and records SN_E_INVAL. */
void sn_gemv_i4(float* y, const float* x, const unsigned char* Wq, const float* scale,
                int in, int out, int block);
/* quant.h:30 */
void sn_gemv_f32(float* y, const float* x, const float* W, int in, int out);

#ifdef __cplusplus
}
#endif
#endif
