// Library runtime implementation (see runtime.cuh).
#include "runtime.cuh"

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

namespace sn {

static thread_local char g_last_err[512];

Runtime& rt() {
    static Runtime r;
    return r;
}

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_err, sizeof g_last_err, fmt, ap);
    va_end(ap);
    return code;
}

int cuda_check(cudaError_t e, const char* where) {
    if (e == cudaSuccess) return SN_OK;
    cudaGetLastError();
    return fail(SN_E_DEVICE, "%s: %s", where, cudaGetErrorString(e));
}

int ensure_init() {
    Runtime& r = rt();
    if (r.inited) return SN_OK;
    std::lock_guard<std::recursive_mutex> lk(r.mu);
    if (r.inited) return SN_OK;
    int dev = 0;
    SN_TRY(cuda_check(cudaGetDevice(&dev), "cudaGetDevice"));
    cudaDeviceProp p;
    SN_TRY(cuda_check(cudaGetDeviceProperties(&p, dev), "cudaGetDeviceProperties"));
    if (p.major < 10)
        return fail(SN_E_UNSUPPORTED, "device %s is sm_%d%d; this build targets sm_100a", p.name,
                    p.major, p.minor);
    r.device = dev;
    r.num_sms = p.multiProcessorCount;
    SN_TRY(cuda_check(cudaStreamCreateWithFlags(&r.own, cudaStreamNonBlocking), "stream"));
    int* h = nullptr;
    SN_TRY(cuda_check(cudaHostAlloc((void**)&h, 64, cudaHostAllocMapped), "cudaHostAlloc"));
    memset(h, 0, 64);
    r.h_err = h;
    SN_TRY(cuda_check(cudaHostGetDevicePointer((void**)&r.d_err, h, 0), "mapped err"));
    r.inited = true;
    return SN_OK;
}

cudaStream_t stream() {
    Runtime& r = rt();
    return r.has_user ? r.user : r.own;
}

bool is_device_ptr(const void* p) {
    if (!p) return false;
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
}

void* scratch(int slot, size_t bytes) {
    Runtime& r = rt();
    if (bytes == 0) bytes = 16;
    if (r.cap[slot] >= bytes) return r.slot[slot];
    if (r.slot[slot]) {
        cudaStreamSynchronize(stream());
        cudaFree(r.slot[slot]);
        r.slot[slot] = nullptr;
        r.cap[slot] = 0;
    }
    size_t want = bytes + bytes / 4;
    void* p = nullptr;
    if (cudaMalloc(&p, want) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    r.slot[slot] = p;
    r.cap[slot] = want;
    return p;
}

int stage_in(const void* p, size_t bytes, int slot, Arr* a) {
    a->bytes = bytes;
    if (is_device_ptr(p)) {
        a->dev = const_cast<void*>(p);
        a->host = nullptr;
        return SN_OK;
    }
    void* d = scratch(slot, bytes);
    if (!d) return fail(SN_E_NOMEM, "device staging of %zu bytes failed", bytes);
    SN_TRY(cuda_check(cudaMemcpyAsync(d, p, bytes, cudaMemcpyHostToDevice, stream()), "H2D"));
    a->dev = d;
    a->host = nullptr;  // inputs never copy back
    return SN_OK;
}

int stage_out(void* p, size_t bytes, int slot, Arr* a) {
    a->bytes = bytes;
    if (is_device_ptr(p)) {
        a->dev = p;
        a->host = nullptr;
        return SN_OK;
    }
    void* d = scratch(slot, bytes);
    if (!d) return fail(SN_E_NOMEM, "device staging of %zu bytes failed", bytes);
    a->dev = d;
    a->host = p;
    return SN_OK;
}

int stage_inout(void* p, size_t bytes, int slot, Arr* a) {
    SN_TRY(stage_out(p, bytes, slot, a));
    if (a->host)
        SN_TRY(cuda_check(cudaMemcpyAsync(a->dev, p, bytes, cudaMemcpyHostToDevice, stream()),
                          "H2D"));
    return SN_OK;
}

int copy_back(const Arr& a) {
    if (!a.host) return SN_OK;
    return cuda_check(cudaMemcpyAsync(a.host, a.dev, a.bytes, cudaMemcpyDeviceToHost, stream()),
                      "D2H");
}

int finish(bool host_involved) {
    Runtime& r = rt();
    SN_TRY(cuda_check(cudaGetLastError(), "kernel launch"));
    if (host_involved || !r.async) {
        SN_TRY(cuda_check(cudaStreamSynchronize(stream()), "cudaStreamSynchronize"));
        int e = r.h_err[0];
        if (e != kErrNone) {
            r.h_err[0] = kErrNone;
            return fail(SN_E_DEVICE, "device-side check failed (code %d)", e);
        }
    }
    return SN_OK;
}

// ----------------------------------------------------------------- profiler
namespace {
struct ProfRec {
    std::string family;
    cudaEvent_t a, b;
    bool graph;  // recorded by a graph's event nodes: read per replay, not here
};
struct Prof {
    int mode = 0;
    unsigned epoch = 0;  // bumped when a session starts: instrumented graphs recapture
    std::vector<ProfRec> recs;
    std::vector<cudaEvent_t> pool;
    std::string open;
    cudaEvent_t open_ev = nullptr;
    std::map<std::string, std::pair<int, double>> extra;  // prof_add (device timestamps)
};
Prof& prof() {
    static Prof p;
    return p;
}
cudaEvent_t take_event() {
    Prof& p = prof();
    if (!p.pool.empty()) {
        cudaEvent_t e = p.pool.back();
        p.pool.pop_back();
        return e;
    }
    cudaEvent_t e;
    cudaEventCreate(&e);
    return e;
}
}  // namespace

namespace {
bool capturing(cudaStream_t st) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cs) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return cs == cudaStreamCaptureStatusActive;
}
// inside a capture the record becomes an event-record node of the graph
void record(cudaEvent_t e, cudaStream_t st) {
    if (capturing(st))
        cudaEventRecordWithFlags(e, st, cudaEventRecordExternal);
    else
        cudaEventRecord(e, st);
}
}  // namespace

bool prof_on() {
    const Prof& p = prof();
    if (p.mode == 2) return true;
    if (p.mode != 1) return false;
    return !capturing(stream());
}

bool prof_graph() { return prof().mode == 2; }

void prof_begin(const char* family, cudaStream_t st) {
    Prof& p = prof();
    p.open = family;
    p.open_ev = take_event();
    record(p.open_ev, st);
}

void prof_end(cudaStream_t st) {
    Prof& p = prof();
    cudaEvent_t e = take_event();
    record(e, st);
    p.recs.push_back({p.open, p.open_ev, e, capturing(st)});
}

int prof_graph_run(ProfGraph* pg, cudaStream_t cap, cudaStream_t st,
                   const std::function<int(cudaStream_t)>& enqueue) {
    Prof& p = prof();
    if (!pg->ex || pg->epoch != p.epoch) {
        if (pg->ex) cudaGraphExecDestroy(pg->ex);
        pg->ex = nullptr;
        cudaGraph_t g = nullptr;
        SN_TRY(cuda_check(cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal),
                          "begin capture (profiled)"));
        const size_t i0 = p.recs.size();
        const int rc = enqueue(cap);
        const cudaError_t e = cudaStreamEndCapture(cap, &g);
        if (rc != SN_OK) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        SN_TRY(cuda_check(e, "end capture (profiled)"));
        const cudaError_t e2 = cudaGraphInstantiate(&pg->ex, g, 0);
        cudaGraphDestroy(g);
        SN_TRY(cuda_check(e2, "graph instantiate (profiled)"));
        pg->i0 = i0;
        pg->i1 = p.recs.size();
        pg->epoch = p.epoch;
    }
    SN_TRY(cuda_check(cudaGraphLaunch(pg->ex, st), "graph launch (profiled)"));
    SN_TRY(cuda_check(cudaStreamSynchronize(st), "profiled replay"));
    for (size_t i = pg->i0; i < pg->i1 && i < p.recs.size(); ++i) {
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, p.recs[i].a, p.recs[i].b) != cudaSuccess) {
            cudaGetLastError();
            continue;
        }
        auto& a = p.extra[p.recs[i].family];
        a.first += 1;
        a.second += ms;
    }
    return SN_OK;
}

void prof_add(const char* family, int launches, double ms) {
    auto& a = prof().extra[family];
    a.first += launches;
    a.second += ms;
}

}  // namespace sn

using namespace sn;

extern "C" {

// Start (1: ungraphed, 2: instrumented graphs) / stop (0) kernel-family
// timing. Starting clears earlier records.
sn_status sn_abi_cuda_profile(int32_t on) {
    SN_TRY(ensure_init());
    if (on < 0 || on > 2) return fail(SN_E_INVAL, "cuda_profile: mode must be 0, 1 or 2");
    Prof& p = prof();
    if (on) {
        cudaStreamSynchronize(stream());
        for (auto& r : p.recs) {
            p.pool.push_back(r.a);
            p.pool.push_back(r.b);
        }
        p.recs.clear();
        p.extra.clear();
        ++p.epoch;
    }
    p.mode = on;
    return SN_OK;
}

// JSON object {"family": [launches, total_ms], ...} of the records so far.
int32_t sn_abi_cuda_profile_report(char* buf, int32_t buflen) {
    Prof& p = prof();
    cudaStreamSynchronize(stream());
    std::map<std::string, std::pair<int, double>> agg;
    for (auto& r : p.recs) {
        if (r.graph) continue;  // read per replay into `extra`
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, r.a, r.b) != cudaSuccess) cudaGetLastError();
        auto& a = agg[r.family];
        a.first += 1;
        a.second += ms;
    }
    for (auto& kv : p.extra) {
        auto& a = agg[kv.first];
        a.first += kv.second.first;
        a.second += kv.second.second;
    }
    std::string s = "{";
    for (auto& kv : agg) {
        char tmp[256];
        snprintf(tmp, sizeof tmp, "%s\"%s\": [%d, %.6f]", s.size() > 1 ? ", " : "",
                 kv.first.c_str(), kv.second.first, kv.second.second);
        s += tmp;
    }
    s += "}";
    const int32_t need = (int32_t)s.size() + 1;
    if (buf && buflen >= need) memcpy(buf, s.c_str(), (size_t)need);
    return need;
}

void sn_abi_clear_error(void) { g_last_err[0] = '\0'; }

int32_t sn_abi_last_error(char* buf, int32_t buflen) {
    int32_t need = (int32_t)strlen(g_last_err) + 1;
    if (buf && buflen >= need) memcpy(buf, g_last_err, (size_t)need);
    return need;
}

sn_status sn_abi_cuda_set_stream(void* s) {
    SN_TRY(ensure_init());
    rt().user = (cudaStream_t)s;
    rt().has_user = true;
    return SN_OK;
}

sn_status sn_abi_cuda_set_async(int32_t on) {
    SN_TRY(ensure_init());
    rt().async = on != 0;
    return SN_OK;
}

sn_status sn_abi_cuda_synchronize(void) {
    SN_TRY(ensure_init());
    return finish(true);
}

int32_t sn_abi_cuda_scan_mode(int32_t mode) {
    int32_t old = rt().scan_mode;
    if (mode == 0 || mode == 1) rt().scan_mode = mode;
    return old;
}

int32_t sn_abi_cuda_int8_mainloop(int32_t on) {
    int32_t old = rt().int8_mainloop;
    if (on == 0 || on == 1) rt().int8_mainloop = on;
    return old;
}

}  // extern "C"
