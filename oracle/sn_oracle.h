/* CPU oracle for the SunnyNet token loop -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference runtime's arithmetic, written so that
 * every rounding step happens in the same order as the reference (which is
 * built as ISO C11, i.e. without FP contraction, plus explicit FMA intrinsics).
 * It is pinned bit-for-bit against the reference runtime compiled from its own
 * sources (oracle/_ref) and against committed golden vectors (tests/golden).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may
 * load this library, and only as the checker / the timed CPU baseline. The
 * product (sunnynet_b200/) never calls it.
 */
#ifndef SN_ORACLE_H
#define SN_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- generic recurrence (reference sunnynet/runtime/recur.c) ---- */
void or_recur_scan(const float* a, const float* b, const float* s0, float* out,
                   float* send, int B, int T, int N, int gated);
/* reverse pass: a, b/u, out, dout, da, db (B,T,N); s0, ds0 (B,N) */
void or_recur_bwd(const float* a, const float* b, const float* s0, const float* out,
                  const float* dout, float* da, float* db, float* ds0, int B, int T, int N,
                  int gated);
void or_recur_step(const float* a, const float* b, float* s, int B, int N, int gated);
void or_quant_i8(const float* x, int8_t* q, float* scale, int B, int N, int block);
void or_dequant_i8(const int8_t* q, const float* scale, float* x, int B, int N, int block);

/* ---- INT4 (reference sunnynet/runtime/quant.c); scale_fp16 selects fp16 scales ---- */
void or_quant_i4(const float* x, uint8_t* q, void* scale, int rows, int N, int block,
                 int scale_fp16);
void or_dequant_i4(const uint8_t* q, const void* scale, float* x, int rows, int N,
                   int block, int scale_fp16);
int  or_gemv_i4(float* y, const float* x, const uint8_t* Wq, const void* scale, int in,
                int out, int block, int scale_fp16);
void or_gemv_f32(float* y, const float* x, const float* W, int in, int out);

/* ---- SunnyNet whole model (reference sunnynet/runtime/sunnynet.c) ----
 * Loads USNN (fp32) or USNQ (INT8 per-output-row) blobs; nseq independent
 * sequences, each with its own state. */
typedef struct OrSunny OrSunny;
OrSunny* or_sn_load(const char* path, int nseq);
void or_sn_free(OrSunny* m);
void or_sn_reset(OrSunny* m);
int  or_sn_vocab(const OrSunny* m);
/* tokens[nseq] -> logits[nseq][vocab] (NULL skips the head). */
void or_sn_step(OrSunny* m, const int32_t* tokens, float* logits);
/* dump raw,at,v,gate,u,s,zn,yn,sfb,out of `layer` for sequence 0 (as sn_dbg_layer). */
void or_sn_dbg_layer(OrSunny* m, int token, int layer, float* dbg);
/* state of sequence i: s (L,D), hist (L,K-1,D). */
void or_sn_get_state(const OrSunny* m, int seq, float* s, float* hist);
void or_sn_set_state(OrSunny* m, int seq, const float* s, const float* hist);

/* ---- RWKV-7 whole model (reference sunnynet/runtime/rwkv7.c) ----
 * Loads KRWK v3 (fp32 / INT4 block 64 fp32 scales) and v4 (INT4 group G, fp16 scales). */
typedef struct OrRwkv OrRwkv;
OrRwkv* or_rk_load(const char* path, int nseq);
void or_rk_free(OrRwkv* m);
void or_rk_reset(OrRwkv* m);
int  or_rk_vocab(const OrRwkv* m);
void or_rk_step(OrRwkv* m, const int32_t* tokens, float* logits);
void or_rk_dbg(OrRwkv* m, int token, int layer, float* out);
/* state of sequence i: S (L,NH,HS,HS), shift (L,2,D). */
void or_rk_get_state(const OrRwkv* m, int seq, float* S, float* shift);
void or_rk_set_state(OrRwkv* m, int seq, const float* S, const float* shift);
/* one step with every layer fed the given input: xs_in, xs_out (nseq, L+1, D) */
void or_rk_step_forced(OrRwkv* m, const int32_t* tokens, const float* xs_in, float* xs_out,
                       float* logits);

/* ---- kernels module (reference sunnynet/kernels/{core,step}_avx2.c) ---- */
void or_core_fwd(const float* q, const float* delta, const float* s0, float* states, float* u,
                 float* p, int B, int T, int D);
void or_core_bwd(const float* q, const float* delta, const float* s0, const float* states,
                 const float* u, const float* p, const float* dstate, const float* du_in,
                 float* dq, float* ddelta, float* ds0, int B, int T, int D);
void or_step_core(const float* q, const float* delta, const float* s, float* s_new, float* u,
                  int B, int D);
void or_dw_step(const float* x, const float* hist, const float* w, float* acc, int B, int D,
                int taps);
void or_scan_f32(const float* p, const float* nu, const float* s0, float* out, float* send,
                 int B, int T, int N);

#ifdef __cplusplus
}
#endif
#endif
