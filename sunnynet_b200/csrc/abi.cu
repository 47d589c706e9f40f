// Stable-ABI bookkeeping: version, capability bits, strings, thread knob.
// Reference: sunnynet/runtime/sn_abi.c:17-49 (same contract), docs/ABI.md.
#include <cstring>
#include <fstream>
#include <set>
#include <string>
#include <utility>

#include "runtime.cuh"
#include "sn_abi.h"

using namespace sn;

namespace {

int32_t copy_str(const char* src, char* buf, int32_t buflen) {
    const int32_t need = (int32_t)strlen(src) + 1;
    if (buf == nullptr || buflen < need) return need;
    memcpy(buf, src, (size_t)need);
    return need;
}

}  // namespace

extern "C" {

int32_t sn_abi_version(void) { return SN_ABI_VERSION; }

uint32_t sn_abi_caps(void) {
    return SN_CAP_RECUR_SCAN | SN_CAP_RECUR_STEP | SN_CAP_QUANT_I8 | SN_CAP_RWKV7 |
           SN_CAP_THREADS | SN_CAP_CUDA | SN_CAP_QUANT_I4 | SN_CAP_SUNNY | SN_CAP_BATCH |
           SN_CAP_RECUR_BWD;
}

sn_status sn_abi_check(int32_t caller_major) {
    return caller_major == SN_ABI_VERSION_MAJOR ? SN_OK : SN_E_UNSUPPORTED;
}

int32_t sn_abi_version_string(char* buf, int32_t buflen) { return copy_str("1.1.0", buf, buflen); }

int32_t sn_abi_backend_string(char* buf, int32_t buflen) { return copy_str("cuda", buf, buflen); }

// The GPU backend has no thread pool; the knob keeps the reference contract
// (n <= 0 -> SN_E_INVAL, value is remembered and reported back).
sn_status sn_abi_set_threads(int32_t n) {
    if (n <= 0) return SN_E_INVAL;
    rt().threads = n;
    return SN_OK;
}

int32_t sn_abi_get_threads(void) { return rt().threads; }

// recur.h:21-22 / sunnynet.h:43-47
void sn_set_threads(int n) {
    if (n > 0) rt().threads = n;
}
int sn_threads(void) { return rt().threads; }
int sn_get_threads(void) { return rt().threads; }

// Physical cores of the host, as sunnynet.c:40-79 (kept for callers that size
// host-side work with it).
int sn_recommended_threads(void) {
    std::ifstream f("/proc/cpuinfo");
    if (!f) return 0;
    std::set<std::pair<int, int>> cores;
    std::string line;
    int phys = -1, core = -1;
    auto flush = [&] {
        if (core >= 0) cores.insert({phys, core});
        phys = core = -1;
    };
    while (std::getline(f, line)) {
        if (line.empty()) {
            flush();
            continue;
        }
        const auto c = line.find(':');
        if (c == std::string::npos) continue;
        const std::string k = line.substr(0, line.find_last_not_of(" \t", c - 1) + 1);
        if (k == "physical id") phys = std::atoi(line.c_str() + c + 1);
        if (k == "core id") core = std::atoi(line.c_str() + c + 1);
    }
    flush();
    return cores.empty() ? 0 : (int)cores.size();
}

}  // extern "C"
