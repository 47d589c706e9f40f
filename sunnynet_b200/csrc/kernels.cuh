// Device-pointer launchers shared between translation units. All take device
// pointers, enqueue on `st` and return an sn_status.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace sn {

// W4A8 output epilogues
enum W4Epi : int { kW4Store = 0, kW4Add = 1, kW4Relu2 = 2, kW4Tanh = 3, kW4Sigmoid = 4 };

int launch_scan(const float* a, const float* b, const float* s0, float* out, float* send, int B,
                int T, int N, int gated, cudaStream_t st);
// The same scan with the entering / leaving states at row strides s0_ld /
// send_ld (a layer's rows of a [seq][layer][N] state array), optionally also
// writing the state entering each position as bf16 planes ph / pl (row t:
// s0 for t = 0, out row t - 1 after), the input of a following contraction.
// nv: channels [0, nv) use the reference's 8-lane FMA rule, [nv, N) its
// scalar rule (separate multiply and add); < 0 = N - N % 8, as recur.c.
int launch_scan_strided(const float* a, const float* b, const float* s0, long long s0_ld,
                        float* out, float* send, long long send_ld, int B, int T, int N,
                        int gated, __nv_bfloat16* ph, __nv_bfloat16* pl, cudaStream_t st,
                        int nv = -1);
// Reverse pass of the scan (sn_recur_bwd) on device arrays.
int launch_scan_bwd(const float* a, const float* b, const float* s0, const float* out,
                    const float* dout, float* da, float* db, float* ds0, int B, int T, int N,
                    int gated, cudaStream_t st);
int launch_step(const float* a, const float* b, float* s, int B, int N, int gated,
                cudaStream_t st);
// Scan mode 1 (chunked in T): chunk length for the shape (0 when even one
// chunk per sequence needs more than `max_records`; <= 0 means no limit),
// the float2 records it needs, and the three-kernel scan itself. The records
// need no initial contents: every record is written before it is read within
// the same call. prof_scopes=false keeps the profiler's events out. `err`:
// the device error word a bounded wait that gives up sets (nullptr: the
// runtime's mapped word). A CTA whose wait gave up leaves its uncomputed
// outputs NaN (its chunk record, or its chunk's rows and final state), so the
// failure also shows in the results.
int scan_chunk_rows(int B, int T, int N, int num_sms, long long max_records);
long long scan_chunk_records(int B, int T, int N, int L);
int launch_scan_chunked(const float* a, const float* b, const float* s0, float* out,
                        float* send, int B, int T, int N, int gated, int L, float2* agg,
                        cudaStream_t st, bool prof_scopes = true, int* err = nullptr);
// Y (nseq,out) = W4A8(X (nseq,in)) with codes (out,in/2) and scales (out,in/block).
// pdl: launched with programmatic serialization (the kernels wait for the
// previous one before reading their input; weights may be fetched earlier).
int launch_w4a8(float* Y, const float* X, const uint8_t* Wq, const void* scale, int nseq, int in,
                int out, int block, bool fp16, cudaStream_t st, int epi, bool pdl = false);
// The same contraction on the tensor cores (w4a8_tc.cu) for M >= 16 sequences,
// K % 128 == 0, block in {32, 64, 128}: bit-identical results. Its activation
// workspace is reserved outside graph capture (w4a8_tc_reserve) before use.
// `planes`: distinct activation inputs one launch quantises (a group).
bool w4a8_tc_ok(int M, int K, int N, int block, const void* Wq);
bool w4a8_tc_ready(int M, int K, int block, int planes = 1);
int w4a8_tc_reserve(int M, int K, int block, int planes = 1);
int launch_w4a8_tc(float* Y, const float* X, const uint8_t* Wq, const void* scale, int M, int K,
                   int N, int block, bool fp16, int epi, cudaStream_t st, bool pdl = false);
// Up to 8 such contractions sharing M, K, block and scale type in one launch
// (plus one quantisation launch over their distinct inputs).
struct W4Problem {
    float* Y;
    const float* X;
    const uint8_t* Wq;
    const void* scale;
    int N;
    int epi;
};
int launch_w4a8_tc_group(const W4Problem* pr, int np, int M, int K, int block, bool fp16,
                         cudaStream_t st, bool pdl = false);
// The same group on the SIMT W4A8 kernel, for nseq <= 8 (quant4.cu): one
// launch, each CTA on one problem's rows.
int launch_w4a8_group(const W4Problem* pr, int np, int nseq, int in, int block, bool fp16,
                      cudaStream_t st, bool pdl = false);
int launch_gemv_f32(float* y, const float* x, const float* W, int in, int out, cudaStream_t st);
// out[b] = argmax of logits row b (lowest id on ties, NaN never chosen);
// part holds B * kArgChunks float2 of scratch (argmax.cu).
constexpr int kArgChunks = 32;
int launch_argmax(const float* lg, int B, int V, float2* part, int32_t* out, cudaStream_t st);
int launch_quant_i4(const float* x, uint8_t* q, void* scale, int rows, int N, int block,
                    bool fp16, cudaStream_t st);

}  // namespace sn
