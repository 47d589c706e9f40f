// Library runtime: one CUDA context per process, one stream, staging of host
// arrays, error reporting. Every C-ABI entry point goes through here.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <functional>
#include <mutex>

#include "sn_abi.h"

namespace sn {

struct Runtime {
    std::recursive_mutex mu;
    bool inited = false;
    int device = -1;
    int num_sms = 148;
    cudaStream_t own = nullptr;   // library-owned stream, used until a caller picks one
    cudaStream_t user = nullptr;  // caller stream (sn_abi_cuda_set_stream; NULL = legacy default)
    bool has_user = false;
    bool async = false;
    int threads = 1;
    int scan_mode = 0;
    int int8_mainloop = 0;  // INT8 contractions convert codes in the main loop
    volatile int* h_err = nullptr;  // mapped pinned word written by device waits
    int* d_err = nullptr;           // device alias of h_err
    void* slot[12] = {};
    size_t cap[12] = {};
};

Runtime& rt();
int ensure_init();                     // SN_OK or SN_E_DEVICE
cudaStream_t stream();
int fail(int code, const char* fmt, ...);
int cuda_check(cudaError_t e, const char* where);
bool is_device_ptr(const void* p);
void* scratch(int slot, size_t bytes);  // device scratch, grows; nullptr on OOM
int finish(bool host_involved);        // sync when needed, surface device errors

// Device view of a caller array. Host arrays are copied into a scratch slot
// (inputs) or computed there and copied back by finish_out (outputs).
struct Arr {
    void* dev = nullptr;
    void* host = nullptr;  // non-null when the caller passed host memory
    size_t bytes = 0;
};
int stage_in(const void* p, size_t bytes, int slot, Arr* a);
int stage_out(void* p, size_t bytes, int slot, Arr* a);
int stage_inout(void* p, size_t bytes, int slot, Arr* a);
int copy_back(const Arr& a);

// Blocks of `threads` covering `total` items, at most `per_sm` blocks per SM
// (grid-stride kernels loop over the rest).
inline int grid_blocks(long long total, int threads = 256, int per_sm = 8) {
    const long long b = (total + threads - 1) / threads;
    const long long cap = (long long)per_sm * rt().num_sms;
    return (int)(b < 1 ? 1 : (b < cap ? b : cap));
}

// Kernel-family timing with CUDA events on the launching stream, between
// sn_abi_cuda_profile(1 or 2) and sn_abi_cuda_profile(0).
//   mode 1: model steps run without their CUDA graph, every kernel family
//           bracketed by events (serialised: each launch waits for the last)
//   mode 2: model steps replay an instrumented copy of their graph: the same
//           nodes, streams and dependencies plus event-record nodes around
//           each family, read after every replay (in-graph durations)
// Work that is not graphed is bracketed directly in both modes.
bool prof_on();      // ProfScopes record (mode 1 outside captures; mode 2 always)
bool prof_graph();   // mode 2
void prof_begin(const char* family, cudaStream_t st);
void prof_end(cudaStream_t st);

// Mode 2: an instrumented graph of one step shape, captured on first use in a
// profiling session (and again after the session restarts), replayed, its
// family events read once the replay is done.
struct ProfGraph {
    cudaGraphExec_t ex = nullptr;
    size_t i0 = 0, i1 = 0;  // its records in the session's list
    unsigned epoch = 0;
    ProfGraph() = default;
    ProfGraph(const ProfGraph&) = delete;
    ProfGraph& operator=(const ProfGraph&) = delete;
    ~ProfGraph() {
        if (ex) cudaGraphExecDestroy(ex);
    }
};
// Capture `enqueue(cap)` when needed, replay on `st`, wait, add the families'
// in-graph times to the report.
int prof_graph_run(ProfGraph* pg, cudaStream_t cap, cudaStream_t st,
                   const std::function<int(cudaStream_t)>& enqueue);
// Add a family measured another way (e.g. device timestamps) to the report.
void prof_add(const char* family, int launches, double ms);

struct ProfScope {
    cudaStream_t st;
    bool on;
    // family == nullptr: no scope
    ProfScope(const char* family, cudaStream_t s) : st(s), on(family && prof_on()) {
        if (on) prof_begin(family, st);
    }
    ~ProfScope() {
        if (on) prof_end(st);
    }
};

// Launch with programmatic stream serialization (the kernel may start while
// the previous one finishes; it must call pdl_wait before reading its inputs).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// launch_pdl when `pdl`, else a plain launch of the same kernel.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_if(bool pdl, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Error codes written into the device error word.
enum DevErr : int { kErrNone = 0, kErrWaitTimeout = 1, kErrBadIndex = 2 };

}  // namespace sn

#define SN_TRY(expr)                 \
    do {                             \
        int _rc = (expr);            \
        if (_rc != SN_OK) return _rc; \
    } while (0)
