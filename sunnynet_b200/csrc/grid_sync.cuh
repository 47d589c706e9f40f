// Grid-wide barrier of a cooperative launch (every CTA co-resident): a
// monotonic arrival counter in global memory, zeroed before each launch.
// Barrier k: thread 0 adds 1 with red.release (after bar.sync, so the release
// covers the whole CTA's writes) and polls with acquire loads until the
// counter reaches (k+1)*CTAs (the passing read synchronizes with every add). Word kGridAbortWord of the same array is
// the abort flag. Data other CTAs wrote is read through L2 (ld.global.cg),
// never through L1 or the read-only path.
#pragma once
#include <cuda_runtime.h>

#include "ptx.cuh"
#include "runtime.cuh"

namespace sn {

constexpr int kGridAbortWord = 32;

namespace {

__device__ __forceinline__ unsigned ld_relaxed_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Barrier k of this launch; false when the step is being abandoned. A CTA
// gives up after `limit` SM cycles (default about a second), raises the
// abort flag so the others leave at their barrier too, and records
// kErrWaitTimeout in the error word.
__device__ bool grid_sync(unsigned* bar, unsigned k, int* err, long long limit = kWaitCycles) {
    __shared__ int ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        int res = 1;
        const unsigned target = (k + 1) * gridDim.x;
        red_release_add(bar, 1u);
        const long long t0 = clock64();
        unsigned it = 0;
        while (ld_acquire_u32(bar) < target) {  // the read that passes is the acquire
            if ((++it & 63u) == 0) {
                if (ld_relaxed_u32(bar + kGridAbortWord)) {
                    res = 0;
                    break;
                }
                if (clock64() - t0 > limit) {
                    atomicExch(bar + kGridAbortWord, 1u);
                    atomicExch(err, kErrWaitTimeout);
                    res = 0;
                    break;
                }
            }
        }
        ok = res;
    }
    __syncthreads();
    return ok != 0;
}

// The two halves of grid_sync, for a CTA that has work to issue while it
// waits: grid_arrive after the CTA's writes for barrier k (bar.sync, then
// thread 0's release add), grid_wait to pass barrier k. Loads issued between
// the two are not ordered by the barrier (they must not read what another CTA
// writes before it), and the release does not wait for them. The wait ends
// with an acquire load of the counter, which synchronizes with every CTA's
// release add.
__device__ __forceinline__ void grid_arrive(unsigned* bar) {
    __syncthreads();
    if (threadIdx.x == 0) red_release_add(bar, 1u);
}
__device__ bool grid_wait(unsigned* bar, unsigned k, int* err, long long limit = kWaitCycles) {
    __shared__ int ok;
    if (threadIdx.x == 0) {
        int res = 1;
        const unsigned target = (k + 1) * gridDim.x;
        const long long t0 = clock64();
        unsigned it = 0;
        while (ld_acquire_u32(bar) < target) {  // the read that passes is the acquire
            if ((++it & 63u) == 0) {
                if (ld_relaxed_u32(bar + kGridAbortWord)) {
                    res = 0;
                    break;
                }
                if (clock64() - t0 > limit) {
                    atomicExch(bar + kGridAbortWord, 1u);
                    atomicExch(err, kErrWaitTimeout);
                    res = 0;
                    break;
                }
            }
        }
        ok = res;
    }
    __syncthreads();
    return ok != 0;
}

}  // namespace
}  // namespace sn
