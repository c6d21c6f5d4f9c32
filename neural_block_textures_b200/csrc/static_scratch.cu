// ES fitness evaluation that allocates no memory: ntcb_es_fitness_noalloc (include/ntc_b200.h).
//
// Who needs it: callers that cannot allocate device memory on the path where they evaluate a population —
// a host engine whose memory budget is fixed after start-up and that forbids allocations on the frame
// path, a process running under an allocator that has no room left by design, or a plugin that may only
// use memory handed to it. cudaMalloc can also block and synchronise the device, which such callers cannot
// afford. This entry point computes the same per-pair fitness as the trainer's population evaluation
// (the kernels of kernels_mlp.cu), with all of its working memory in one file-scope device array.
//
// The array, g_fitness_scratch, is NTCB_STATIC_SCRATCH_BYTES (16 MiB) on every GPU that loads the library,
// held until the process exits. Host code cannot use its name as a device address (in host code it names a
// host-side stand-in), so the first call on each device, with that device current, asks the runtime for the
// device address (cudaGetSymbolAddress) and keeps it; later calls on that device reuse it. That first call
// may load the module, so make it before any stream capture begins. The kept address belongs to the device's
// current context: after a cudaDeviceReset the module may load at another address, so do not call this entry
// again in a process that has reset the device. Within one process every call on a device shares the array,
// which keeps the last call's contents: calls that overlap in time (for example from several host threads)
// race on it and must be serialised by the caller; each process has its own copy. No region needs clearing
// between calls: every value a kernel reads is written earlier in the same call.
//
// Errors come back to the caller, never as a process exit: a bad argument or a request above the maximum is
// refused before the GPU is touched, and a CUDA failure inside the call (a copy, a launch) makes it return 0 with
// the runtime's message. A CUDA error the caller left pending before the call is reported the same way (and left
// pending), since the call could not tell its own launch errors from it.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "../../include/ntc_b200.h"
#include "kernels.h"

namespace {

constexpr size_t kScratchBytes = NTCB_STATIC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_fitness_scratch[kScratchBytes];

std::mutex g_setup_mutex;
unsigned char* g_scratch_addr[kMaxDevices] = {};

size_t align256(size_t n) { return (n + 255) / 256 * 256; }

void set_reason(char* why, size_t cap, const char* msg) {
    if (why && cap) { strncpy(why, msg, cap - 1); why[cap - 1] = 0; }
}

// Minibatch rows [M][n] (the features / targets of loss_subset's pixels) -> [n][mstride], the layout the
// population kernel reads with coalesced loads.
__global__ void k_rows_to_cols(const float* __restrict__ src, int M, int n, int mstride, float* __restrict__ dst) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)M * n) return;
    const int s = (int)(i / n), c = (int)(i % n);
    dst[(long long)c * mstride + s] = src[i];
}

}  // namespace

extern "C" int ntcb_es_fitness_noalloc(const ntcb_model_desc* d, int it, float sigma, int pair_begin, int npairs,
                                       const float* w, const float* feat, const float* tgt, int M, double* fit,
                                       char* why, size_t why_cap) {
    using namespace ntcb;
    // ---- validate before touching the GPU
    if (!d || !w || !feat || !tgt || !fit) { set_reason(why, why_cap, "null pointer argument"); return 0; }
    if (M < 1 || npairs < 1 || pair_begin < 0) { set_reason(why, why_cap, "need M >= 1, npairs >= 1, pair_begin >= 0"); return 0; }
    if (d->nin < 1 || d->nin > kMaxIn || d->nout < 1 || d->nout > kMaxOut || d->nhidden < 0 || d->nhidden > kMaxHidden) {
        set_reason(why, why_cap, "model outside the envelope (nin <= 64, nout <= 12, <= 8 hidden layers)"); return 0;
    }
    long long P = 0;
    {
        int ncur = d->nin;
        for (int l = 0; l < d->nhidden; l++) {
            if (d->hidden[l] < 1 || d->hidden[l] > kMaxWidth) { set_reason(why, why_cap, "hidden width outside 1..64"); return 0; }
            P += (long long)d->hidden[l] * ncur + d->hidden[l];
            ncur = d->hidden[l];
        }
        P += (long long)d->nout * ncur + d->nout;
    }
    if (P * 4 > 48 * 1024) { set_reason(why, why_cap, "MLP above 12288 weights"); return 0; }
    DevModel m;
    memset(&m, 0, sizeof(m));
    m.nin = d->nin; m.nout = d->nout; m.nhidden = d->nhidden;
    for (int l = 0; l < d->nhidden; l++) m.hidden[l] = d->hidden[l];
    m.leak = d->leak; m.clamp_out = d->clamp_out ? 1 : 0;
    for (int c = 0; c < kMaxOut; c++) m.cw[c] = c < d->nout ? d->cw[c] : 0.0f;
    m.wsum = d->wsum; m.P = (int)P;
    const int shape = shape_id(m);
    const int rows = pop_chunk_rows(shape);
    const int passes = (M + rows - 1) / rows;
    const int chunk = rows * std::max(1, (passes + 3) / 4);
    const int chunks = pop_chunks(M, chunk);
    const int mstride = (M + 31) / 32 * 32;
    const size_t o_w = 0;
    const size_t o_frows = o_w + align256((size_t)P * 4);
    const size_t o_trows = o_frows + align256((size_t)M * d->nin * 4);
    const size_t o_feat = o_trows + align256((size_t)M * d->nout * 4);
    const size_t o_tgt = o_feat + align256((size_t)d->nin * mstride * 4);
    const size_t o_eps = o_tgt + align256((size_t)d->nout * mstride * 4);
    const size_t o_part = o_eps + align256((size_t)npairs * P * 4);
    const size_t o_fit = o_part + align256((size_t)npairs * 2 * chunks * 8);
    const size_t need = o_fit + align256((size_t)npairs * 2 * 8);
    if (need > kScratchBytes) {
        char msg[200];
        snprintf(msg, sizeof(msg), "npairs %d x %lld weights with M %d needs %zu bytes of scratch, above the %zu-byte static maximum",
                 npairs, P, M, need, kScratchBytes);
        set_reason(why, why_cap, msg);
        return 0;
    }
    // ---- a CUDA error pending from the caller's earlier work: report it, leave it pending
    {
        const cudaError_t pending = cudaPeekAtLastError();
        if (pending != cudaSuccess) {
            char msg[200];
            snprintf(msg, sizeof(msg), "a CUDA error was pending before the call: %s", cudaGetErrorString(pending));
            set_reason(why, why_cap, msg);
            return 0;
        }
    }
    // ---- once per device: the device address of the static array
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) { set_reason(why, why_cap, "no usable CUDA device"); return 0; }
    unsigned char* base = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_setup_mutex);
        if (!g_scratch_addr[dev]) {
            void* p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g_fitness_scratch);
            if (e != cudaSuccess || !p) {
                cudaGetLastError();
                char msg[200];
                snprintf(msg, sizeof(msg), "cudaGetSymbolAddress of the static scratch failed: %s", cudaGetErrorString(e));
                set_reason(why, why_cap, msg);
                return 0;
            }
            g_scratch_addr[dev] = static_cast<unsigned char*>(p);
        }
        base = g_scratch_addr[dev];
    }
    float* sw = reinterpret_cast<float*>(base + o_w);
    float* frows = reinterpret_cast<float*>(base + o_frows);
    float* trows = reinterpret_cast<float*>(base + o_trows);
    float* feat_t = reinterpret_cast<float*>(base + o_feat);
    float* tgt_t = reinterpret_cast<float*>(base + o_tgt);
    float* eps = reinterpret_cast<float*>(base + o_eps);
    double* part = reinterpret_cast<double*>(base + o_part);
    double* sfit = reinterpret_cast<double*>(base + o_fit);
    // ---- inputs in, kernels, output out (legacy default stream; the copies are synchronous). Inside the scope every
    // CUDA failure, here or in the launchers, is recorded instead of ending the process; the first one is returned.
    SoftErrorScope soft;
    auto failed = [&](const char* where) {
        if (soft.err == cudaSuccess) return false;
        cudaGetLastError();   // clear a launch error this call made (a sticky error stays with the context)
        char msg[240];
        snprintf(msg, sizeof(msg), "CUDA error during %s: %s", where, cudaGetErrorString(soft.err));
        set_reason(why, why_cap, msg);
        return true;
    };
    NTCB_CHECK(cudaMemcpy(sw, w, (size_t)P * 4, cudaMemcpyHostToDevice));
    NTCB_CHECK(cudaMemcpy(frows, feat, (size_t)M * d->nin * 4, cudaMemcpyHostToDevice));
    NTCB_CHECK(cudaMemcpy(trows, tgt, (size_t)M * d->nout * 4, cudaMemcpyHostToDevice));
    if (failed("the input copies")) return 0;
    k_rows_to_cols<<<(unsigned)(((long long)M * d->nin + 255) / 256), 256>>>(frows, M, d->nin, mstride, feat_t);
    NTCB_CHECK(cudaGetLastError());
    k_rows_to_cols<<<(unsigned)(((long long)M * d->nout + 255) / 256), 256>>>(trows, M, d->nout, mstride, tgt_t);
    NTCB_CHECK(cudaGetLastError());
    if (failed("the row transposes")) return 0;
    if (sigma != 0.0f) launch_mlp_noise(nullptr, d->seed, it, pair_begin, npairs, (int)P, eps);
    if (failed("the noise launch")) return 0;
    PopArgs a{};
    a.mode = 0; a.it = it; a.sigma = sigma; a.fd_h = 0.0f; a.cand_begin = pair_begin; a.ncand = npairs;
    a.M = M; a.mstride = mstride; a.chunk = chunk;
    a.w0 = sw; a.eps = eps; a.feat_t = feat_t; a.tgt_t = tgt_t; a.part = part;
    launch_pop_eval(nullptr, shape, m, a);
    if (failed("the population launch")) return 0;
    launch_pop_finish(nullptr, part, npairs, chunks, 3.0 * (double)d->wsum * M, sfit);
    if (failed("the fitness launch")) return 0;
    NTCB_CHECK(cudaMemcpy(fit, sfit, (size_t)npairs * 2 * 8, cudaMemcpyDeviceToHost));
    if (failed("the kernels or the result copy")) return 0;
    return 1;
}
