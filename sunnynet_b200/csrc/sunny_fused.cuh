// One SunnyNet decode step for a small batch (B <= 8) as a single persistent
// kernel: one CTA per SM, grid barriers between the dependent phases of a
// layer, weights pulled into L2 ahead of the phase that reads them.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace sn {

constexpr int kFusedMaxB = 8;
constexpr int kFusedThreads = 512;
constexpr int kFusedMaxG = 16;
constexpr int kFusedMaxTaps = 8;  // ring taps (conv kernel - 1)
constexpr int kFusedMaxSmem = 200 * 1024;  // dynamic shared memory cap

// Per-layer weights (device pointers), copied to device memory once at load.
struct FusedLayer {
    const float *ni_g, *ni_c, *nm_g, *nm_c, *dw, *delta;
    const void *V, *U, *Wz, *Wc, *Ws;
    const float *sV, *sU, *sWz, *sWc, *sWs;  // int8 row scales (null otherwise)
    float a_tanh, b_gain;
};

struct FusedArgs {
    int B = 0, D = 0, I = 0, R = 0, K = 0, KH = 1, L = 0, G = 0, vocab = 0, clamp = 0;
    int wtype = 0;  // WType of gemm.cuh
    int ctas = 0;   // grid size (one CTA per SM)
    int with_head = 1;
    int bulk_prefetch = 0;  // every weight row slice is 16-byte aligned and sized
    // bytes of each of the two shared-memory buffers a CTA stages its next
    // phase's weight slice in (fused_stage_bytes), or 0: read weights from
    // global memory behind an L2 prefetch hint
    int stage_bytes = 0;
    // bytes of the CTA's head rows staged in shared memory a layer ahead
    // (whole rows; the rest is read from global memory), or 0
    int head_stage_bytes = 0;
    float eps = 0, p_floor = 0;
    const FusedLayer* layers = nullptr;
    const float *no_g = nullptr, *no_c = nullptr, *embed = nullptr;
    const void* head = nullptr;
    const float* shead = nullptr;
    // state and activations ([seq] rows, as in the multi-kernel step)
    float* s = nullptr;
    float* hist = nullptr;
    int32_t* pos = nullptr;
    const int32_t* tok = nullptr;
    float *x = nullptr, *v = nullptr, *u = nullptr, *sfb = nullptr, *z = nullptr;
    float* logits = nullptr;  // [B][vocab], or null: logits not stored
    int32_t* next = nullptr;  // greedy next token per sequence (argmax), or null
    // step words, kBarWords unsigned zeroed before every launch: [0] barrier
    // arrivals (monotonic within a launch), [kBarAbort] abort flag,
    // [kBarDone] CTAs finished with the head, [kBarAmax..] per-sequence packed
    // argmax (8 x u64); each group on its own 128-byte line
    unsigned* bar = nullptr;
    int* err = nullptr;
    // profiling only, per CTA: slot 0 at the start, then for phase p (4l+k,
    // head 4L) slot 1+8p+j at j = 0 loads done, 1 row statistics done, 2
    // inputs ready, 3 weights ready, 4 rows done, 5 barrier passed;
    // [cta][%globaltimer x trace_slots | clock64 x trace_slots],
    // trace_slots = 32L + 9; or null
    unsigned long long* trace = nullptr;
    int trace_slots = 0;
};

constexpr int kBarAbort = 32, kBarDone = 64, kBarAmax = 96, kBarWords = 128;
static_assert(kBarAbort == 32, "the abort word grid_sync.cuh polls (kGridAbortWord)");

// Dynamic shared memory the fused step needs (0 when the shapes do not fit).
size_t fused_smem_bytes(const FusedArgs& a);
// Fill in a->stage_bytes and a->head_stage_bytes (stage: shared-memory
// staging of the weights where it fits) and return the dynamic shared memory
// the launch needs, or 0 when the fused step does not take these shapes.
size_t fused_plan(FusedArgs* a, bool stage);
// Enqueue the fused step (cooperative launch, one CTA per SM). The barrier
// words are reset on `st` first.
int launch_sunny_fused(const FusedArgs& a, cudaStream_t st);

}  // namespace sn
