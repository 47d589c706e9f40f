/* RWKV-7 whole-model decode, internal symbol set of the reference's
 * sunnynet/runtime/rwkv7.h:16-28, same signatures. Loads KRWK v3 blobs (fp32
 * or INT4 block 64) and this project's KRWK v4 (INT4 group G, fp16 scales). */
#ifndef SN_RWKV7_H
#define SN_RWKV7_H

#ifdef __cplusplus
extern "C" {
#endif

typedef struct SnRWKV7 SnRWKV7;

SnRWKV7* sn_rk_load(const char* path);                          /* rwkv7.h:16 */
void sn_rk_free(SnRWKV7* m);                                    /* rwkv7.h:17 */
void sn_rk_reset(SnRWKV7* m);                                   /* rwkv7.h:18 */
void sn_rk_step(SnRWKV7* m, int token, float* logits);          /* rwkv7.h:21 */
void sn_rk_prefill(SnRWKV7* m, const int* tokens, int n, float* logits); /* :22 */
/* rwkv7.h:25: xn, r, k, v, a, g, ww, y, x_out of `layer`, each (D,) */
void sn_rk_dbg(SnRWKV7* m, int token, int layer, float* out);
int  sn_rk_vocab(const SnRWKV7* m);                             /* rwkv7.h:27 */
int  sn_rk_ready(const SnRWKV7* m);                             /* rwkv7.h:28 */

#ifdef __cplusplus
}
#endif
#endif
