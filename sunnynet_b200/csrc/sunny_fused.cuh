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
    float* logits = nullptr;
    // barrier words: [0] arrivals (monotonic within a launch), [kBarAbort]
    // abort flag on its own 128-byte line; kBarWords unsigned, zeroed before
    // every launch
    unsigned* bar = nullptr;
    int* err = nullptr;
    // profiling only: %globaltimer per CTA at each phase end and barrier exit
    // ([cta][trace_slots], trace_slots = 8L + 2), or null
    unsigned long long* trace = nullptr;
    int trace_slots = 0;
};

constexpr int kBarAbort = 32, kBarWords = 64;

// Dynamic shared memory the fused step needs (0 when the shapes do not fit).
size_t fused_smem_bytes(const FusedArgs& a);
// Enqueue the fused step (cooperative launch, one CTA per SM). The barrier
// words are reset on `st` first.
int launch_sunny_fused(const FusedArgs& a, cudaStream_t st);

}  // namespace sn
