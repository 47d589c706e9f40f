/* The reference's kernels module (sunnynet/kernels/scan_avx2.c, core_avx2.c,
 * step_avx2.c; loaded by kernels/__init__.py load_kernel, which sets the
 * argtypes of exactly these names), computed on a B200. Same names,
 * signatures and array layouts; every array may be host or device memory
 * (see sn_abi.h). The functions return nothing, as the reference's do;
 * failures are reported through sn_abi_last_error.
 *
 * Numerics: scan_f32, scan_bwd_f32 and dw_step_f32 are bit-identical to the
 * reference build. core_fwd_f32, core_bwd_f32 and step_core_f32 round every
 * operation as the reference does except exp (CUDA expf instead of the host
 * libm): a few ulp apart. D % 8 channels are left untouched by the core
 * functions, as the reference's 8-lane loops leave them.
 */
#ifndef SN_KERNELS_H
#define SN_KERNELS_H

#ifdef __cplusplus
extern "C" {
#endif

/* scan_avx2.c:12-45: s_t = p_t*s_{t-1} + (1-p_t)*nu_t; p, nu, out (B,T,N);
 * s0, send (B,N). */
void scan_f32(const float* p, const float* nu, const float* s0, float* out, float* send,
              int B, int T, int N);
/* scan_avx2.c:50-95: dp = ds*(s_prev - nu), dnu = ds*(1 - p), ds0 (B,N). */
void scan_bwd_f32(const float* p, const float* nu, const float* s0, const float* out,
                  const float* dout, float* dp, float* dnu, float* ds0, int B, int T, int N);
/* core_avx2.c:34-79: q (B,T,2D) = [u_raw | gate], delta (D), s0 (B,D) ->
 * states, u, p (B,T,D): competition within groups of 8, decay gate, scan. */
void core_fwd_f32(const float* q, const float* delta, const float* s0, float* states,
                  float* u, float* p, int B, int T, int D);
/* core_avx2.c:84-148: dq (B,T,2D), ds0 (B,D); ddelta (D) is accumulated (+=). */
void core_bwd_f32(const float* q, const float* delta, const float* s0, const float* states,
                  const float* u, const float* p, const float* dstate, const float* du_in,
                  float* dq, float* ddelta, float* ds0, int B, int T, int D);
/* step_avx2.c:54-86: one step: q (B,2D), s (B,D) -> s_new, u (B,D). */
void step_core_f32(const float* q, const float* delta, const float* s, float* s_new,
                   float* u, int B, int D);
/* step_avx2.c:24-50: acc (B,D) = w[K-1]*x + sum_j w[K-2-j]*hist[:,j];
 * x (B,D), hist (B,K-1,D), w (K,D). */
void dw_step_f32(const float* x, const float* hist, const float* w, float* acc, int B, int D,
                 int taps);

#ifdef __cplusplus
}
#endif
#endif /* SN_KERNELS_H */
