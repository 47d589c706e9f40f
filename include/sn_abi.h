/* SunnyNet stable C ABI -- B200 (sm_100a) implementation.
 *
 * Drop-in for the reference's sunnynet/runtime/sn_abi.h:20-101: every symbol,
 * signature, status code and capability bit of ABI 1.0 is kept, so a caller
 * built against the reference header links against libsunnynet_cuda.so
 * unchanged. ABI 1.1 adds functions behind new capability bits (a MINOR bump,
 * docs/ABI.md:6-17): unknown bits must be ignored by callers, old callers keep
 * working.
 *
 * Pointers. Every array argument may be host memory or CUDA device memory
 * (the library tells them apart through unified virtual addressing). Host
 * arrays are staged through device memory and the call returns when the
 * results are back in them, exactly like the reference. When all array
 * arguments of a call are device pointers and async mode is on
 * (sn_abi_cuda_set_async), the call only enqueues work on the library stream.
 */
#ifndef SN_ABI_H
#define SN_ABI_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SN_ABI_VERSION_MAJOR 1
#define SN_ABI_VERSION_MINOR 1
#define SN_ABI_VERSION_PATCH 0

#define SN_ABI_VERSION \
    ((SN_ABI_VERSION_MAJOR << 16) | (SN_ABI_VERSION_MINOR << 8) | SN_ABI_VERSION_PATCH)

/* ABI 1.0 capability bits (reference sn_abi.h:34-38) */
#define SN_CAP_RECUR_SCAN   (1u << 0)
#define SN_CAP_RECUR_STEP   (1u << 1)
#define SN_CAP_QUANT_I8     (1u << 2)
#define SN_CAP_RWKV7        (1u << 3)
#define SN_CAP_THREADS      (1u << 4)
/* ABI 1.1 additions */
#define SN_CAP_CUDA         (1u << 5)  /* device pointers, stream, async mode */
#define SN_CAP_QUANT_I4     (1u << 6)  /* sn_abi_quant_i4 / dequant_i4 / gemv_i4 */
#define SN_CAP_SUNNY        (1u << 7)  /* sn_abi_sunny_* whole-model handle */
#define SN_CAP_BATCH        (1u << 8)  /* batched steps + state export/import */
#define SN_CAP_RECUR_BWD    (1u << 9)  /* sn_abi_recur_bwd */

/* Status codes (reference sn_abi.h:41-46, docs/ABI.md:55-68) */
#define SN_OK              0
#define SN_E_INVAL        -1
#define SN_E_NOMEM        -2
#define SN_E_IO           -3
#define SN_E_FORMAT       -4
#define SN_E_UNSUPPORTED  -5
#define SN_E_DEVICE       -6  /* ABI 1.1: CUDA error or a bounded device wait gave up */

typedef int32_t sn_status;

/* ------------------------------------------------ ABI 1.0 (reference sn_abi.h) */
int32_t   sn_abi_version(void);                                   /* sn_abi.h:52 */
uint32_t  sn_abi_caps(void);                                      /* sn_abi.h:55 */
sn_status sn_abi_check(int32_t caller_major);                     /* sn_abi.h:58 */
int32_t   sn_abi_version_string(char* buf, int32_t buflen);       /* sn_abi.h:62 */
int32_t   sn_abi_backend_string(char* buf, int32_t buflen);       /* sn_abi.h:65, "cuda" */
sn_status sn_abi_set_threads(int32_t n);                          /* sn_abi.h:68 */
int32_t   sn_abi_get_threads(void);                               /* sn_abi.h:69 */

/* s = a*s + b (gated: b = (1-a)*u); a, b, s (B,N). sn_abi.h:74-75 */
sn_status sn_abi_recur_step(const float* a, const float* b, float* s,
                            int32_t B, int32_t N, int32_t gated);
/* a, b, out (B,T,N); s0, send (B,N). sn_abi.h:78-80. Bit-identical to the
 * reference AVX2 kernel. */
sn_status sn_abi_recur_scan(const float* a, const float* b, const float* s0,
                            float* out, float* send,
                            int32_t B, int32_t T, int32_t N, int32_t gated);
/* No counterpart in the reference. The chunked scan (the arithmetic of scan
 * mode 1, within a few ulp per chunk boundary of the bit-exact scan) for
 * callers that cannot allocate device memory: a process whose device memory
 * belongs to its own pool allocator, a loop that must not stall on the
 * device synchronisation cudaMalloc/cudaFree imply, a fixed memory budget.
 * It calls no allocator: its temporary records live in a fixed 2 MiB array
 * of the library's device image, held by every GPU that loads the library
 * until exit. Every array must be memory of the current device (or managed
 * memory); the work is enqueued on `cuda_stream` (NULL = legacy default
 * stream) and the call returns without synchronising. Rejects B*N > 262144
 * with SN_E_INVAL. The first call on a device looks up the array's device
 * address (make it before any stream capture). Calls that overlap on the GPU
 * share the array and race: order them on one stream. Nothing in the array
 * needs to start at zero. A device wait that gives up (a GPU stalled for
 * about a second) cannot change the returned status; it leaves the affected
 * rows and final states NaN instead, so check `send` when that matters. */
sn_status sn_abi_recur_scan_noalloc(const float* a, const float* b, const float* s0,
                                    float* out, float* send,
                                    int32_t B, int32_t T, int32_t N, int32_t gated,
                                    void* cuda_stream);
/* ABI 1.1 (SN_CAP_RECUR_BWD): the stable, status-returning face of the
 * reference's internal sn_recur_bwd (recur.h:27-30, recur.c:51-107), the
 * reverse pass over the scan's outputs. a, b, out, dout, da, db (B,T,N); s0,
 * ds0 (B,N); gated == 1: b holds u, da = ds*(s_prev - u), db = ds*(1 - a).
 * Bit-identical to the reference. */
sn_status sn_abi_recur_bwd(const float* a, const float* b, const float* s0,
                           const float* out, const float* dout,
                           float* da, float* db, float* ds0,
                           int32_t B, int32_t T, int32_t N, int32_t gated);
/* symmetric per-block INT8; block <= 0 means one block per row. sn_abi.h:83-86 */
sn_status sn_abi_quant_i8(const float* x, int8_t* q, float* scale,
                          int32_t B, int32_t N, int32_t block);
sn_status sn_abi_dequant_i8(const int8_t* q, const float* scale, float* x,
                            int32_t B, int32_t N, int32_t block);

typedef struct SnAbiRwkv7 SnAbiRwkv7;                             /* sn_abi.h:90 */
SnAbiRwkv7* sn_abi_rwkv7_load(const char* blob_path);             /* sn_abi.h:92 */
sn_status   sn_abi_rwkv7_step(SnAbiRwkv7* m, int32_t token, float* logits);   /* :95 */
sn_status   sn_abi_rwkv7_prefill(SnAbiRwkv7* m, const int32_t* tokens,
                                 int32_t n, float* logits);      /* sn_abi.h:96-97 */
sn_status   sn_abi_rwkv7_reset(SnAbiRwkv7* m);                    /* sn_abi.h:98 */
void        sn_abi_rwkv7_free(SnAbiRwkv7* m);                     /* sn_abi.h:99 */
int32_t     sn_abi_rwkv7_vocab(const SnAbiRwkv7* m);              /* sn_abi.h:100 */

/* ------------------------------------------------------- ABI 1.1 additions */
/* No reference counterpart: CUDA execution control (SN_CAP_CUDA). */
/* Stream for all later work. NULL selects the legacy default stream; until the
 * first call the library uses a stream of its own. */
sn_status sn_abi_cuda_set_stream(void* cuda_stream);
sn_status sn_abi_cuda_set_async(int32_t on);          /* device-pointer calls only enqueue */
sn_status sn_abi_cuda_synchronize(void);              /* waits; reports deferred errors */
int32_t   sn_abi_last_error(char* buf, int32_t buflen); /* message of the last failure */
void      sn_abi_clear_error(void);                    /* empties it (this thread) */
int32_t   sn_abi_cuda_scan_mode(int32_t mode);        /* 0 exact (default), 1 chunked; returns old */
/* INT8 weights of models loaded afterwards, batched (tensor-core) path: 1 keeps
 * the codes (1 byte per weight) and converts each K slab to bf16 inside the
 * contraction's main loop; 0 (default) expands them once at load to bf16 code
 * planes (2 bytes per weight, faster on this build's B200 measurements).
 * Results are identical. Returns the old setting. */
int32_t   sn_abi_cuda_int8_mainloop(int32_t on);
/* Kernel-family timing with CUDA events (1 = start and clear, 0 = stop). While
 * on, model steps run without their CUDA graph so each kernel can be bracketed. */
sn_status sn_abi_cuda_profile(int32_t on);
/* JSON {"family": [launches, total_ms], ...}; returns the length incl. NUL. */
int32_t   sn_abi_cuda_profile_report(char* buf, int32_t buflen);
/* Failure-path test hook (no reference counterpart). Runs one CTA that waits,
 * through the library's bounded device waits, on something that never
 * completes: kind 0 an mbarrier phase, kind 1 a grid barrier like the fused
 * decode step's, kind 2 the same barrier split into its arrive and wait
 * halves (the fused RWKV-7 step's form). After `cycles` SM cycles (1 .. 2^31; the step kernels use
 * 2^31) the wait gives up and the kernel returns. Returns SN_E_DEVICE when
 * the give-up was reported, as every model call does after a device wait
 * times out; the library stays usable afterwards. */
sn_status sn_abi_cuda_wait_selftest(int32_t kind, int64_t cycles);

/* INT4 (SN_CAP_QUANT_I4), the stable-ABI face of the reference's internal
 * quant.h:20-27. scale_fp16 != 0 selects fp16 scales (group formats). */
sn_status sn_abi_quant_i4(const float* x, uint8_t* q, void* scale, int32_t rows,
                          int32_t N, int32_t block, int32_t scale_fp16);
sn_status sn_abi_dequant_i4(const uint8_t* q, const void* scale, float* x, int32_t rows,
                            int32_t N, int32_t block, int32_t scale_fp16);
/* y[out] = Wq(out,in) x with the W4A8 semantics of quant.c:89-154 (bit-identical). */
sn_status sn_abi_gemv_i4(float* y, const float* x, const uint8_t* Wq, const void* scale,
                         int32_t in, int32_t out, int32_t block, int32_t scale_fp16);
/* batched W4A8: Y[B][out] = rows of X[B][in] each through the same semantics */
sn_status sn_abi_gemm_i4(float* Y, const float* X, const uint8_t* Wq, const void* scale,
                         int32_t B, int32_t in, int32_t out, int32_t block, int32_t scale_fp16);

/* SunnyNet whole model (SN_CAP_SUNNY). The reference exposes this only through
 * its internal sunnynet.h:22-47; here it gets a stable handle that owns `nseq`
 * independent sequences. Loads USNN (fp32) or USNQ (INT8 per-row) blobs. */
typedef struct SnAbiSunny SnAbiSunny;
SnAbiSunny* sn_abi_sunny_load(const char* blob_path, int32_t nseq);
void        sn_abi_sunny_free(SnAbiSunny* m);
sn_status   sn_abi_sunny_reset(SnAbiSunny* m);
int32_t     sn_abi_sunny_vocab(const SnAbiSunny* m);
int32_t     sn_abi_sunny_dims(const SnAbiSunny* m, int32_t* dims8); /* vocab,D,I,R,K,L,G,quant */
/* one token per sequence for the first B sequences: tokens[B] -> logits[B][vocab]
 * (logits may be NULL to skip the LM head). */
sn_status   sn_abi_sunny_step(SnAbiSunny* m, const int32_t* tokens, int32_t B, float* logits);
/* greedy: next[B] = argmax of the step's logits (ties -> lowest id) */
sn_status   sn_abi_sunny_step_argmax(SnAbiSunny* m, const int32_t* tokens, int32_t B,
                                     int32_t* next);
/* feed tokens (B,T) row-major; logits of the last position -> logits[B][vocab]
 * (NULL skips the head). Runs as 256-token chunks: the contractions over all
 * B*chunk rows at once, the recurrence as a scan carrying only the state. */
sn_status   sn_abi_sunny_prefill(SnAbiSunny* m, const int32_t* tokens, int32_t B, int32_t T,
                                 float* logits);
sn_status   sn_abi_sunny_prefill_chunked(SnAbiSunny* m, const int32_t* tokens, int32_t B,
                                         int32_t T, int32_t chunk, float* logits);
/* state of sequences [0,B): s (B,L,D), hist (B,L,K-1,D), hist[.,.,0] newest */
sn_status   sn_abi_sunny_get_state(SnAbiSunny* m, int32_t B, float* s, float* hist);
sn_status   sn_abi_sunny_set_state(SnAbiSunny* m, int32_t B, const float* s, const float* hist);
/* No reference counterpart (serving with continuous batching): the same for
 * sequences [seq0, seq0 + n) of the handle, and a reset of just those. */
sn_status   sn_abi_sunny_get_state_at(SnAbiSunny* m, int32_t seq0, int32_t n, float* s,
                                      float* hist);
sn_status   sn_abi_sunny_set_state_at(SnAbiSunny* m, int32_t seq0, int32_t n, const float* s,
                                      const float* hist);
sn_status   sn_abi_sunny_reset_at(SnAbiSunny* m, int32_t seq0, int32_t n);

/* RWKV-7 batched (SN_CAP_BATCH): a handle owning nseq sequences. */
SnAbiRwkv7* sn_abi_rwkv7_load_batch(const char* blob_path, int32_t nseq);
sn_status   sn_abi_rwkv7_step_batch(SnAbiRwkv7* m, const int32_t* tokens, int32_t B,
                                    float* logits);
sn_status   sn_abi_rwkv7_step_argmax(SnAbiRwkv7* m, const int32_t* tokens, int32_t B,
                                     int32_t* next);
/* No reference counterpart: a debugging view of one batched step. The same
 * kernels run (without the step's CUDA graph) and the residual stream is
 * copied out as it enters each layer and leaves the last one: xs (B, L+1, D),
 * host or device. logits (B, vocab) may be NULL. Lets a checker run any
 * single layer from exactly this step's input. */
sn_status   sn_abi_rwkv7_step_trace(SnAbiRwkv7* m, const int32_t* tokens, int32_t B,
                                    float* logits, float* xs);
/* Prompt of T tokens for each of the first B sequences (tokens (B,T) row-major)
 * -> logits (B, vocab) of each sequence's last token (NULL: state only). The
 * reference feeds a prompt token by token (rwkv7.c:362-364); here each layer
 * runs over all prompt rows at once and only the matrix-state recurrence
 * walks the tokens in order; results match stepping within fp32 rounding. */
sn_status   sn_abi_rwkv7_prefill_batch(SnAbiRwkv7* m, const int32_t* tokens, int32_t B,
                                       int32_t T, float* logits);
/* S (B,L,NH,HS,HS), shift (B,L,2,D) */
sn_status   sn_abi_rwkv7_get_state(SnAbiRwkv7* m, int32_t B, float* S, float* shift);
int32_t     sn_abi_rwkv7_dims(const SnAbiRwkv7* m, int32_t* dims8); /* vocab,D,HS,NH,F,L,q4,group */

#ifdef __cplusplus
}
#endif
#endif /* SN_ABI_H */
