/* SunnyNet whole-model decode, internal symbol set of the reference's
 * sunnynet/runtime/sunnynet.h:22-47 (B=1 handle), same signatures. The handle
 * keeps weights and state in HBM; logits is a caller buffer of >= vocab floats
 * (host or device). See sn_abi.h for the batched, stable-ABI handle. */
#ifndef SN_MODEL_H
#define SN_MODEL_H

#ifdef __cplusplus
extern "C" {
#endif

typedef struct SnModel SnModel;

/* sunnynet.h:22-23: NULL on any failure or header/dims mismatch */
SnModel* sn_load(const char* path, int vocab, int dim, int inner, int rank,
                 int taps, int layers, int group, int tied);
/* sunnynet.h:27-28: fp16 GEMV weights + head */
SnModel* sn_load_h(const char* path, int vocab, int dim, int inner, int rank,
                   int taps, int layers, int group, int tied);
void sn_free(SnModel* m);                                      /* sunnynet.h:30 */
void sn_reset(SnModel* m);                                     /* sunnynet.h:31 */
void sn_step(SnModel* m, int token, float* logits);           /* sunnynet.h:34 */
void sn_prefill(SnModel* m, const int* tokens, int n, float* logits); /* :37 */
int  sn_vocab(const SnModel* m);                               /* sunnynet.h:39 */
int  sn_ready(const SnModel* m);                               /* sunnynet.h:40 */
int  sn_get_threads(void);                                     /* sunnynet.h:44 */
int  sn_recommended_threads(void);                             /* sunnynet.h:47 */
/* sunnynet.c:336-345: runs layers 0..layer for `token` and dumps
 * raw,at,v,gate,u,s,zn,yn,sfb,out of `layer` (7D+R+2I floats). */
void sn_dbg_layer(SnModel* m, int token, int layer, float* dbg);

#ifdef __cplusplus
}
#endif
#endif
