// dlopen binding of the five NCCL calls the library's multi-GPU iteration uses (declarations from nccl.h).
#include "nccl_link.h"

#include <dlfcn.h>
#include <nccl.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

namespace ntcb::nccl {

namespace {

struct Api {
    bool tried = false, ok = false;
    std::string why;
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) comm_init_rank = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
    decltype(&ncclGetVersion) get_version = nullptr;
};

std::mutex g_mu;
Api g_api;

template <class F>
bool sym(void* h, const char* name, F& out, std::string& why) {
    out = reinterpret_cast<F>(dlsym(h, name));
    if (!out) { why = std::string("libnccl.so.2 has no ") + name; return false; }
    return true;
}

const Api& api() {
    std::lock_guard<std::mutex> lk(g_mu);
    Api& a = g_api;
    if (a.tried) return a;
    a.tried = true;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) { a.why = std::string("cannot load libnccl.so.2: ") + dlerror(); return a; }
    a.ok = sym(h, "ncclGetUniqueId", a.get_unique_id, a.why) && sym(h, "ncclCommInitRank", a.comm_init_rank, a.why) &&
           sym(h, "ncclCommDestroy", a.comm_destroy, a.why) && sym(h, "ncclAllGather", a.all_gather, a.why) &&
           sym(h, "ncclGetErrorString", a.error_string, a.why) && sym(h, "ncclGetVersion", a.get_version, a.why);
    return a;
}

}  // namespace

bool unique_id(unsigned char* id, std::string& why) {
    static_assert(sizeof(ncclUniqueId) == kUniqueIdBytes, "NCCL unique id size");
    const Api& a = api();
    if (!a.ok) { why = a.why; return false; }
    ncclUniqueId u;
    const ncclResult_t r = a.get_unique_id(&u);
    if (r != ncclSuccess) { why = std::string("ncclGetUniqueId: ") + a.error_string(r); return false; }
    std::memcpy(id, &u, sizeof(u));
    return true;
}

void* comm_init(const unsigned char* id, int world, int rank, std::string& why) {
    const Api& a = api();
    if (!a.ok) { why = a.why; return nullptr; }
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof(u));
    ncclComm_t c = nullptr;
    const ncclResult_t r = a.comm_init_rank(&c, world, u, rank);
    if (r != ncclSuccess) { why = std::string("ncclCommInitRank: ") + a.error_string(r); return nullptr; }
    return c;
}

void comm_destroy(void* comm) {
    const Api& a = api();
    if (a.ok && comm) a.comm_destroy(static_cast<ncclComm_t>(comm));
}

void all_gather_inplace(void* comm, void* buf, size_t bytes, int rank, cudaStream_t s) {
    const Api& a = api();
    char* b = static_cast<char*>(buf);
    const ncclResult_t r = a.all_gather(b + (size_t)rank * bytes, b, bytes, ncclUint8, static_cast<ncclComm_t>(comm), s);
    if (r != ncclSuccess) {
        fprintf(stderr, "ntc_b200: ncclAllGather failed: %s\n", a.error_string(r));
        exit(1);
    }
}

int version() {
    const Api& a = api();
    int v = 0;
    if (a.ok) a.get_version(&v);
    return v;
}

}  // namespace ntcb::nccl
