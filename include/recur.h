/* Generic first-order recurrence, internal symbol set of the reference's
 * sunnynet/runtime/recur.h:18-41, same signatures and semantics, computed on a
 * B200. Array arguments may be host or device pointers (see sn_abi.h).
 *
 *   s_t = a_t * s_{t-1} + b_t              (gated == 0)
 *   s_t = a_t * s_{t-1} + (1 - a_t) * u_t  (gated == 1, b holds u)
 */
#ifndef SN_RECUR_H
#define SN_RECUR_H

#ifdef __cplusplus
extern "C" {
#endif

#define SN_FMA   0
#define SN_GATED 1

void sn_set_threads(int n);                 /* recur.h:21 (and sunnynet.h:43) */
int  sn_threads(void);                      /* recur.h:22 */

/* recur.h:26-27; a, b, out (B,T,N); s0, send (B,N). Bit-identical to the reference. */
void sn_recur_scan(const float* a, const float* b, const float* s0,
                   float* out, float* send, int B, int T, int N, int gated);
/* recur.h:27-30: reverse pass over the scan's outputs. a, b, out, dout, da,
 * db (B,T,N); s0, ds0 (B,N). With gated == 1, b holds u and da/db are the
 * gradients w.r.t. a and u: da = ds*(s_prev - u), db = ds*(1 - a).
 * Bit-identical to the reference (recur.c:51-107). */
void sn_recur_bwd(const float* a, const float* b, const float* s0,
                  const float* out, const float* dout,
                  float* da, float* db, float* ds0,
                  int B, int T, int N, int gated);
/* recur.h:36: one step, s updated in place. */
void sn_recur_step(const float* a, const float* b, float* s, int B, int N, int gated);
/* recur.h:40-43: symmetric per-block INT8, block <= 0 = whole row. */
void sn_quant_i8(const float* x, signed char* q, float* scale, int B, int N, int block);
void sn_dequant_i8(const signed char* q, const float* scale, float* x, int B, int N, int block);

#ifdef __cplusplus
}
#endif
#endif
