// Per-device set-up caches for the launchers. A process may drive several GPUs (one trainer per device, or the
// allocation-free entry on whichever device is current), so an SM count or a kernel's dynamic shared-memory
// opt-in (cudaFuncSetAttribute acts on the current device's context) is kept per device ordinal, never once per
// process. Both are safe to call from several host threads.
#include "kernels.h"

#include <map>
#include <mutex>
#include <utility>

namespace ntcb {

thread_local cudaError_t* g_soft_error = nullptr;

namespace {
std::mutex g_mu;
std::map<int, int> g_nsm;                                   // device -> SM count
std::map<std::pair<int, const void*>, int> g_smem;          // (device, kernel) -> dynamic shared memory opted in
}  // namespace

int device_sm_count() {
    int dev = 0;
    NTCB_CHECK(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(g_mu);
    auto it = g_nsm.find(dev);
    if (it != g_nsm.end()) return it->second;
    int n = 0;
    NTCB_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
    g_nsm[dev] = n;
    return n;
}

void ensure_dynamic_smem(const void* kernel, int bytes) {
    int dev = 0;
    NTCB_CHECK(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(g_mu);
    int& have = g_smem[{dev, kernel}];
    if (have >= bytes) return;
    NTCB_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    have = bytes;
}

}  // namespace ntcb
