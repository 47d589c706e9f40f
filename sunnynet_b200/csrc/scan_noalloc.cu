// sn_abi_recur_scan_noalloc: the chunked gated/FMA scan (scan mode 1) for
// callers that cannot allocate device memory.
//
// Who needs it. The regular entry point sn_abi_recur_scan keeps its chunk
// records in library scratch that grows with cudaMalloc (and frees the old
// buffer with cudaFree, which synchronises the device). Some callers cannot
// let that happen: a process whose device memory is owned by its own pool
// allocator (a serving engine that reserves nearly all HBM at start-up and
// hands out slices), a latency-critical loop in which an implicit device
// synchronisation would stall other streams, or an embedding under a fixed
// memory budget. This entry point takes device pointers for every input and
// output and an explicit stream, and finds its temporary memory in one
// fixed-size array that is part of the library's device image.
//
// The fixed array. kRecords float2 records (2 MiB) in a file-scope
// `static __device__` array. It is created when the CUDA driver loads this
// part of the library on a GPU and is held by every GPU that loads it until
// the process exits. One record is needed per (sequence, time chunk,
// channel); chunks grow up to the full length T, so a call fits whenever
// B*N <= kRecords (262,144 channels across all sequences) and is rejected
// with SN_E_INVAL beyond that.
//
// Set-up. Host code cannot use the array's name as a device address (the
// name is a host-side stand-in; a kernel given it would fault, or read host
// memory on a system where the GPU can reach it). The first call on each
// device therefore looks the address up with cudaGetSymbolAddress, with that
// device current, and caches it; that first call may also make the driver
// load this module. Make the first call on each device before any stream
// capture begins.
//
// Contents and concurrency. Every call shares the array and it keeps the
// last call's contents. Nothing in it has to start at zero: each call writes
// every record it uses before reading it. Calls whose kernels overlap on the
// GPU (issued on different streams, or from several threads without
// ordering) use the same records and corrupt each other's results; issue
// them on one stream, or order them with events.
//
// Results. The arithmetic is that of scan mode 1 of sn_abi_recur_scan: per
// chunk, the affine maps of the rows are composed into the carry entering
// the chunk, and the rows are re-run from it with the reference's per-row
// rule. Outputs differ from the sequential (mode 0, bit-exact) scan by a few
// ulp of the state per chunk boundary.
//
// Device-side failures. The kernels' waits on their shared-memory copies are
// bounded (about a second). A wait can only give up on a GPU that stalls that
// long, and this call has returned SN_OK by then: its status is decided when
// the work is enqueued. So a give-up is reported in the results: the CTA
// waits for its copies still in flight, marks what it leaves uncomputed as NaN
// (its chunk's summary, which turns every later row and final state of those
// channels NaN, or its chunk's remaining rows and final state) and returns.
// It also sets a second fixed device word of this file (g_noalloc_err), never
// the library's shared error word, so no later call of the regular entry
// points reports a failure that was not theirs. The word is not cleared and
// nothing reads it back: a NaN in `send` is the signal a caller checks.
//
// Devices. Every array must be memory of the current device (or managed
// memory): an array of another GPU would make the kernels read that GPU's
// memory across NVLink, or fault without peer access.
#include <cuda_runtime.h>

#include <mutex>

#include "kernels.cuh"
#include "runtime.cuh"
#include "sn_abi.h"

namespace sn {
namespace {

constexpr long long kRecords = 1ll << 18;  // float2 records: 2 MiB
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float2 g_scan_records[kRecords];
static __device__ int g_noalloc_err;

struct DeviceSlot {
    float2* records = nullptr;  // device address of g_scan_records on this device
    int* err = nullptr;         // device address of g_noalloc_err on this device
    int num_sms = 0;
};
DeviceSlot g_slots[kMaxDevices];
std::mutex g_setup_mu;

// Once per device, with `dev` current: the array's device address and the
// facts the launch needs. Nothing here allocates.
int setup_device(int dev, DeviceSlot** out) {
    std::lock_guard<std::mutex> lk(g_setup_mu);
    DeviceSlot& s = g_slots[dev];
    if (!s.records) {
        int major = 0, sms = 0;
        SN_TRY(cuda_check(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev),
                          "recur_scan_noalloc: device attribute"));
        SN_TRY(cuda_check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev),
                          "recur_scan_noalloc: device attribute"));
        if (major < 10)
            return fail(SN_E_UNSUPPORTED, "recur_scan_noalloc: device %d is sm_%d0; this build "
                        "targets sm_100a", dev, major);
        void* p = nullptr;
        void* e = nullptr;
        SN_TRY(cuda_check(cudaGetSymbolAddress(&p, g_scan_records),
                          "recur_scan_noalloc: cudaGetSymbolAddress of the fixed scratch"));
        SN_TRY(cuda_check(cudaGetSymbolAddress(&e, g_noalloc_err),
                          "recur_scan_noalloc: cudaGetSymbolAddress of the error word"));
        s.num_sms = sms;
        s.err = static_cast<int*>(e);
        s.records = static_cast<float2*>(p);
    }
    *out = &s;
    return SN_OK;
}

// Memory the kernels on device `dev` may read and write directly: that
// device's own allocations, or managed memory.
bool on_device(const void* p, int dev) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return at.type == cudaMemoryTypeManaged ||
           (at.type == cudaMemoryTypeDevice && at.device == dev);
}

}  // namespace
}  // namespace sn

using namespace sn;

extern "C" sn_status sn_abi_recur_scan_noalloc(const float* a, const float* b, const float* s0,
                                               float* out, float* send, int32_t B, int32_t T,
                                               int32_t N, int32_t gated, void* cuda_stream) {
    if (!a || !b || !s0 || !out || !send || B <= 0 || T <= 0 || N <= 0)
        return fail(SN_E_INVAL, "recur_scan_noalloc: null pointer or non-positive dimension");
    if ((long long)B * N > kRecords)
        return fail(SN_E_INVAL,
                    "recur_scan_noalloc: B*N = %lld channels exceed the fixed scratch of %lld "
                    "records (2 MiB); use sn_abi_recur_scan",
                    (long long)B * N, kRecords);
    int dev = 0;
    SN_TRY(cuda_check(cudaGetDevice(&dev), "recur_scan_noalloc: cudaGetDevice"));
    if (dev < 0 || dev >= kMaxDevices)
        return fail(SN_E_UNSUPPORTED, "recur_scan_noalloc: device ordinal %d", dev);
    DeviceSlot* slot = nullptr;
    SN_TRY(setup_device(dev, &slot));
    if (!on_device(a, dev) || !on_device(b, dev) || !on_device(s0, dev) ||
        !on_device(out, dev) || !on_device(send, dev))
        return fail(SN_E_INVAL, "recur_scan_noalloc: every array must be device memory of the "
                    "current device %d (host arrays would need staging buffers, i.e. an "
                    "allocation; another GPU's arrays would be read across NVLink)", dev);
    const int L = scan_chunk_rows(B, T, N, slot->num_sms, kRecords);
    if (L <= 0)
        return fail(SN_E_INVAL, "recur_scan_noalloc: shape does not fit the fixed scratch");
    return launch_scan_chunked(a, b, s0, out, send, B, T, N, gated ? 1 : 0, L, slot->records,
                               static_cast<cudaStream_t>(cuda_stream), false, slot->err);
}
