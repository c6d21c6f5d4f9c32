// Host orchestration of the B200 ES training backend: device state, the training steps, the flat
// C ABI (include/ntc_b200.h) and the drop-in C++ class ntc_cuda::Trainer (include/ntc_cuda.h).
//
// One Engine (= ntc_cuda::Trainer::Impl) owns every device buffer of one model on one GPU and
// launches all of its kernels on one stream. Public calls follow the reference's contract
// (cuda/ntc_cuda.cu:699-1179): host buffers are consumed or filled before the call returns, runtime
// failures print and exit(1), init() reports unsupported models with false + a reason.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/ntc_b200.h"
#include "../../include/ntc_cuda.h"
#include "kernels.h"
#include "kernels_snap.h"
#include "nccl_link.h"
#include "p2p_exchange.h"

// The C description structs are the C++ ones byte for byte (main.cpp fills the C++ ones; FFI callers the C ones).
static_assert(sizeof(ntcb_level_desc) == sizeof(ntc_cuda::LevelDesc), "LevelDesc layout");
static_assert(offsetof(ntcb_level_desc, off) == offsetof(ntc_cuda::LevelDesc, off), "LevelDesc layout");
static_assert(offsetof(ntcb_level_desc, nearest) == offsetof(ntc_cuda::LevelDesc, nearest), "LevelDesc layout");
static_assert(sizeof(ntcb_model_desc) == sizeof(ntc_cuda::ModelDesc), "ModelDesc layout");
#define NTCB_SAME_OFFSET(F) static_assert(offsetof(ntcb_model_desc, F) == offsetof(ntc_cuda::ModelDesc, F), "ModelDesc." #F);
NTCB_SAME_OFFSET(W) NTCB_SAME_OFFSET(T) NTCB_SAME_OFFSET(nlev) NTCB_SAME_OFFSET(lv) NTCB_SAME_OFFSET(npos) NTCB_SAME_OFFSET(pos)
NTCB_SAME_OFFSET(nin) NTCB_SAME_OFFSET(nout) NTCB_SAME_OFFSET(nhidden) NTCB_SAME_OFFSET(hidden) NTCB_SAME_OFFSET(leak)
NTCB_SAME_OFFSET(clamp_out) NTCB_SAME_OFFSET(cw) NTCB_SAME_OFFSET(wsum) NTCB_SAME_OFFSET(qat_bits) NTCB_SAME_OFFSET(qat)
NTCB_SAME_OFFSET(qat_grid) NTCB_SAME_OFFSET(qes_bits) NTCB_SAME_OFFSET(dct) NTCB_SAME_OFFSET(dct_C) NTCB_SAME_OFFSET(dct_N)
NTCB_SAME_OFFSET(dct_dc_step) NTCB_SAME_OFFSET(dct_q) NTCB_SAME_OFFSET(dct_basis) NTCB_SAME_OFFSET(dct_zigzag)
NTCB_SAME_OFFSET(max_pairs) NTCB_SAME_OFFSET(max_batch) NTCB_SAME_OFFSET(seed)
#undef NTCB_SAME_OFFSET
static_assert(sizeof(ntcb_qes_desc) == sizeof(ntc_cuda::QesDesc), "QesDesc layout");
static_assert(sizeof(ntcb_dct_desc) == sizeof(ntc_cuda::DctDesc), "DctDesc layout");
static_assert(sizeof(ntcb::QesTables) == sizeof(ntc_cuda::QesDesc), "QesTables mirrors QesDesc");

namespace ntc_cuda {

struct Trainer::Impl {
    ModelDesc d{};
    ntcb::DevModel dm{};
    int shape = 0;
    int P = 0;
    long long nz = 0, npix = 0, n0 = 0;
    int device = -1;
    cudaStream_t own_stream = nullptr, stream = nullptr;
    bool ready = false;

    // latent
    float *z = nullptr, *zgrad = nullptr, *zm = nullptr, *zv = nullptr, *ztmp = nullptr, *zq = nullptr, *zdec = nullptr;
    float* qgrid = nullptr;
    ntcb::QesTables* qes_dev = nullptr;
    bool qes = false;
    float* lat_eps = nullptr; long long lat_eps_cap = 0;   // [K][nz]
    float* dpix = nullptr; long long dpix_cap = 0;         // [K][npix]
    std::vector<int*> lvl_xr, lvl_yr;                      // per level footprint ranges (device)
    int qat_cw = 0, qat_ch = 0;                            // level-0 cell size in pixels when every footprint is a whole cell
    int* ranges = nullptr;
    // DCT
    bool dct = false, dct_live = false, rate_es = false, rate_trunc = false;
    long long dct_n = 0;
    ntcb::DctTables dtab{};
    int16_t* dsym = nullptr; uint8_t* dcode = nullptr; int* dsteps = nullptr; float* dlam = nullptr;
    int32_t* dbits = nullptr; int32_t* ddbits = nullptr; long long ddbits_cap = 0; int* dcnt = nullptr;
    int dct_evals = 0, dct_last_K = 0; float rate_scale = 0.0f;
    // MLP
    float *w = nullptr, *wgrad = nullptr, *wm = nullptr, *wv = nullptr;
    float *tgt = nullptr, *img = nullptr;
    int* bidx = nullptr; float *feat_t = nullptr, *tgt_t = nullptr; int Mcap = 0, mstride = 0;
    float* mlp_eps = nullptr; int pairs_cap = 0;
    double* part = nullptr; long long part_cap = 0;
    double *fit = nullptr, *dl = nullptr, *lsum = nullptr, *hh = nullptr;
    double* fit_stats = nullptr;
    // ES evaluations (MLP pairs and the latent pass): true (default) = the tensor-core kernels (3xTF32) where the
    // shape has them; false = the packed-FP32 kernels, bit-identical per unit to the reference backend. FD always
    // uses the latter.
    bool tensor_pop = true;
    int* tc_err = nullptr;   // device flag the tensor-core kernel sets when an MMA completion wait times out
    float* gpart = nullptr; long long gpart_cap = 0;
    char* xbuf = nullptr; long long xbuf_cap = 0;   // exchange blocks of the native sharded iteration ([rank][block])
    // peer-memory exchange of the native sharded iteration (ntcb_p2p_export / ntcb_p2p_import)
    ntcb::P2PArgs p2p{};
    char* p2p_buf = nullptr;   // this rank's exchange buffer (flags, counters, staging)
    bool p2p_ready = false;
    uint32_t p2p_epoch = 0;
    uint32_t p2p_poll_limit = ntcb::kP2PPollLimit;   // polls of one staged line before an exchange wait fails
    float* qat_grid = nullptr; int* qat_bits = nullptr;
    // progress-print statistics: the last set_qes description (host copy) and a device scratch buffer
    ntc_cuda::QesDesc qes_host{};
    char* stats_buf = nullptr; size_t stats_cap = 0;
    double* hstage = nullptr; size_t hstage_cap = 0;   // pinned host staging of the statistics reads (doubles)
    // counters
    int mlp_t = 0, lat_t = 0, lat_step_no = 0;
    int last_N = 0, last_M = 0, last_pairs = 0; bool last_fd = false;
    // pairs whose dl / lsum (read only by mlp_stats and debug_last_dl) are still to be reduced from fit: the sharded
    // ES step defers that launch until one of them asks
    mutable int dl_pending = 0;
    long long launches = 0;
    // timing
    bool timing = false;
    std::string timing_only;   // non-empty: only this kernel class is timed (the others launch without events)
    struct Pending { std::string cls; cudaEvent_t a, b; };
    std::vector<Pending> pending;
    std::map<std::string, std::pair<double, int>> totals;
    // banner
    std::string dev_name; int sm_major = 0, sm_minor = 0, sms = 0, rt_ver = 0;
};

}  // namespace ntc_cuda

using Impl = ntc_cuda::Trainer::Impl;

namespace {

void die(const char* msg) { fprintf(stderr, "ntc_b200: %s\n", msg); exit(1); }

template <class T>
T* dalloc(size_t n) {
    T* p = nullptr;
    NTCB_CHECK(cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)));
    return p;
}
template <class T>
void dfree(T*& p) { if (p) { cudaFree(p); p = nullptr; } }

// Records CUDA events around one launch of kernel class `cls` when timing is on.
template <class F>
void timed(Impl& I, const char* cls, int nlaunch, F&& launch) {
    if (!I.timing || (!I.timing_only.empty() && I.timing_only != cls)) { launch(); I.launches += nlaunch; return; }
    Impl::Pending p{cls, nullptr, nullptr};
    NTCB_CHECK(cudaEventCreate(&p.a)); NTCB_CHECK(cudaEventCreate(&p.b));
    NTCB_CHECK(cudaEventRecord(p.a, I.stream));
    launch();
    NTCB_CHECK(cudaEventRecord(p.b, I.stream));
    I.pending.push_back(p);
    I.launches += nlaunch;
}
void flush_timing(Impl& I) {
    if (I.pending.empty()) return;
    NTCB_CHECK(cudaStreamSynchronize(I.stream));
    for (auto& p : I.pending) {
        float ms = 0.0f;
        NTCB_CHECK(cudaEventElapsedTime(&ms, p.a, p.b));
        auto& t = I.totals[p.cls];
        t.first += ms; t.second += 1;
        cudaEventDestroy(p.a); cudaEventDestroy(p.b);
    }
    I.pending.clear();
}

// After a stream synchronisation: a tensor-core CTA whose MMA completion wait timed out has flagged it (and
// left its partial sums unwritten); that is a runtime failure like any CUDA error.
void check_tc_err(const Impl& I) {
    if (!I.tc_err) return;
    int e = 0;
    NTCB_CHECK(cudaMemcpy(&e, I.tc_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (e) {
        fprintf(stderr, e == 2 ? "ntc_b200: a peer exchange timed out waiting for another rank\n"
                               : "ntc_b200: a tensor-core population CTA timed out waiting for its MMAs\n");
        exit(1);
    }
}

void sync(Impl& I) {
    NTCB_CHECK(cudaStreamSynchronize(I.stream));
    check_tc_err(I);
}
void set_device(Impl& I) { if (I.device >= 0) NTCB_CHECK(cudaSetDevice(I.device)); }

// Footprint rectangles of every texel of a level (per texel column [xb, xe), per texel row [yb, ye)):
// nearest levels use the cell rule of qat_search (main.cpp:2095-2096); bilinear levels the rule of the
// latent scatter (main.cpp:2015-2024): a pixel feeds texel tx if its clamped tap x0 == tx, or x1 == tx
// with x1 != x0. The pixels of a texel form one contiguous range per axis; init() verifies that.
bool axis_ranges(int npx, int ntex, bool nearest, std::vector<int>& lo, std::vector<int>& hi) {
    lo.assign(ntex, npx); hi.assign(ntex, 0);
    std::vector<int> count(ntex, 0);
    for (int px = 0; px < npx; px++) {
        const float u = ((float)px + 0.5f) / (float)npx;
        int t0, t1;
        if (nearest) {
            const float x = u * (float)ntex;
            t0 = t1 = std::max(0, std::min(ntex - 1, (int)std::floor(x)));
        } else {
            const float x = std::fmaf(u, (float)ntex, -0.5f);
            const int x0 = (int)std::floor(x);
            t0 = std::max(0, std::min(ntex - 1, x0));
            t1 = std::max(0, std::min(ntex - 1, x0 + 1));
        }
        lo[t0] = std::min(lo[t0], px); hi[t0] = std::max(hi[t0], px + 1); count[t0]++;
        if (t1 != t0) { lo[t1] = std::min(lo[t1], px); hi[t1] = std::max(hi[t1], px + 1); count[t1]++; }
    }
    for (int t = 0; t < ntex; t++)
        if (count[t] && hi[t] - lo[t] != count[t]) return false;
    return true;
}

void ensure_part(Impl& I, long long need) {
    if (need <= I.part_cap) return;
    dfree(I.part);
    I.part = dalloc<double>((size_t)need);
    I.part_cap = need;
}
void ensure_lat(Impl& I, int K) {
    if ((long long)K * I.nz > I.lat_eps_cap) {
        dfree(I.lat_eps);
        I.lat_eps_cap = (long long)K * I.nz;
        I.lat_eps = dalloc<float>((size_t)I.lat_eps_cap);
        NTCB_CHECK(cudaMemsetAsync(I.lat_eps, 0, (size_t)I.lat_eps_cap * sizeof(float), I.stream));
    }
    if ((long long)K * I.npix > I.dpix_cap) {
        dfree(I.dpix);
        I.dpix_cap = (long long)K * I.npix;
        I.dpix = dalloc<float>((size_t)I.dpix_cap);
    }
    if (I.dct && (long long)K * I.dct_n > I.ddbits_cap) {
        dfree(I.ddbits);
        I.ddbits_cap = (long long)K * I.dct_n;
        I.ddbits = dalloc<int32_t>((size_t)I.ddbits_cap);
        NTCB_CHECK(cudaMemsetAsync(I.ddbits, 0, (size_t)I.ddbits_cap * sizeof(int32_t), I.stream));
    }
}
void ensure_xbuf(Impl& I, long long bytes) {
    if (bytes <= I.xbuf_cap) return;
    dfree(I.xbuf);
    I.xbuf = dalloc<char>((size_t)bytes);
    I.xbuf_cap = bytes;
}
void ensure_gpart(Impl& I, long long need) {
    if (need <= I.gpart_cap) return;
    dfree(I.gpart);
    I.gpart = dalloc<float>((size_t)need);
    I.gpart_cap = need;
}

// Rows of the minibatch one population CTA covers: a multiple of the CTA's pass, about M / 4 so that the
// grid has ~4 CTAs per candidate pair (a short last wave).
int pop_chunk(const Impl& I, int M) {
    const int rows = ntcb::pop_chunk_rows(I.shape);
    if (const char* e = getenv("NTCB_POP_CHUNK")) { const int c = atoi(e); if (c >= rows && c % rows == 0) return c; }
    const int passes = (M + rows - 1) / rows;
    return rows * std::max(1, (passes + 3) / 4);
}

void adam_coeffs(int t, float& c1, float& c2) {
    c1 = 1.0f - powf(0.9f, (float)t);
    c2 = 1.0f - powf(0.999f, (float)t);
}

// The snapped decode copy (cuda/ntc_cuda.cu:920-932): --qes grid snap (a plain copy for levels without
// bits), then the DCT snap of level 0 once live, or the pre-start clamp.
void snap_latent_impl(Impl& I) {
    if (!I.qes && !I.dct) return;
    timed(I, "snap", 1, [&] { ntcb::launch_qes_snap(I.stream, I.dm, I.qes_dev, I.z, I.zq, I.qgrid, I.nz); });
    if (I.dct) {
        if (I.dct_live) {
            if (I.rate_es || I.rate_trunc) NTCB_CHECK(cudaMemsetAsync(I.dcnt, 0, 2 * sizeof(int), I.stream));
            timed(I, "dct_snap", 1, [&] {
                ntcb::launch_dct_snap(I.stream, I.dm, I.dtab, I.z, I.zq, I.dsym, I.dcode, I.dsteps, I.dlam, I.dbits, I.dcnt);
            });
        } else {
            timed(I, "snap", 1, [&] { ntcb::launch_dct_clamp0(I.stream, I.z, I.zq, I.dm.lv[0].off, I.n0); });
        }
    }
}

void free_all(Impl& I) {
    dfree(I.z); dfree(I.zgrad); dfree(I.zm); dfree(I.zv); dfree(I.ztmp); dfree(I.zq); dfree(I.qgrid); dfree(I.qes_dev);
    dfree(I.lat_eps); dfree(I.dpix); dfree(I.ranges);
    dfree(I.dsym); dfree(I.dcode); dfree(I.dsteps); dfree(I.dlam); dfree(I.dbits); dfree(I.ddbits); dfree(I.dcnt);
    dfree(I.w); dfree(I.wgrad); dfree(I.wm); dfree(I.wv); dfree(I.tgt); dfree(I.img);
    dfree(I.bidx); dfree(I.feat_t); dfree(I.tgt_t); dfree(I.mlp_eps); dfree(I.part);
    dfree(I.fit); dfree(I.dl); dfree(I.lsum); dfree(I.hh); dfree(I.fit_stats); dfree(I.gpart); dfree(I.xbuf); I.xbuf_cap = 0; dfree(I.tc_err);
    dfree(I.qat_grid); dfree(I.qat_bits); dfree(I.stats_buf); I.stats_cap = 0;
    if (I.hstage) { cudaFreeHost(I.hstage); I.hstage = nullptr; I.hstage_cap = 0; }
    if (I.p2p_ready)
        for (int q = 0; q < I.p2p.world; q++)
            if (q != I.p2p.rank && I.p2p.base[q]) cudaIpcCloseMemHandle(I.p2p.base[q]);
    I.p2p = ntcb::P2PArgs{}; I.p2p_ready = false;
    dfree(I.p2p_buf);
    for (auto& p : I.pending) { cudaEventDestroy(p.a); cudaEventDestroy(p.b); }
    I.pending.clear();
    if (I.own_stream) { cudaStreamDestroy(I.own_stream); I.own_stream = nullptr; }
}

bool init_impl(Impl& I, const ntc_cuda::ModelDesc& d, const float* z, const float* p, const float* target, std::string& why) {
    using namespace ntcb;
    I.d = d;
    // The reference's envelope (cuda/ntc_cuda.cu:751-785), kept so that the same models are accepted.
    int need = d.nin;
    for (int l = 0; l < d.nhidden; l++) need = std::max(need, d.hidden[l]);
    if (need > kMaxWidth) { why = "the B200 backend supports at most 64 units per layer (input and hidden)"; return false; }
    if (d.nhidden < 0 || d.nhidden > kMaxHidden) { why = "too many hidden layers"; return false; }
    if (d.nout < 1 || d.nout > kMaxOut) { why = "too many MLP outputs"; return false; }
    if (d.nlev < 1 || d.nlev > kMaxLevels) { why = "bad level count"; return false; }
    if (d.lv[0].C > kMaxCh) { why = "the B200 backend supports at most 16 level-0 channels"; return false; }
    if (d.npos < 0 || d.npos > kMaxPos) { why = "too many positional features"; return false; }
    I.qes = false;
    for (int l = 0; l < d.nlev; l++)
        if (d.qes_bits[l] > 0) {
            I.qes = true;
            if (d.qes_bits[l] < 2 || d.qes_bits[l] > 12) { why = "--qes bits out of range"; return false; }
            if (d.lv[l].C > 64) { why = "the B200 backend supports at most 64 channels on a --qes level"; return false; }
        }
    I.dct = d.dct != 0; I.dct_live = false;
    if (I.dct) {
        if (d.dct_N != 8) { why = "--dct-q: the B200 backend supports --dct-block 8 only"; return false; }
        if (d.dct_C < 1 || d.dct_C > 4 || d.dct_C != d.lv[0].C) { why = "--dct-q: level 0 must have 1..4 channels (= dct_C)"; return false; }
        if (!d.lv[0].nearest || d.lv[0].W != d.W || d.lv[0].H != d.H || d.W % 8 != 0 || d.H % 8 != 0) {
            why = "--dct-q: level 0 must be a full-resolution nearest level with a size that is a multiple of 8"; return false;
        }
        if (!d.dct_basis) { why = "--dct-q needs the host basis table"; return false; }
        if (!d.dct_zigzag) { why = "--dct-q needs the host zigzag table"; return false; }
        if (d.dct_dc_step < 1 || d.dct_dc_step > 64) { why = "--dct-q: DC step out of range"; return false; }
    }
    if ((long long)d.W * d.H >= (1ll << 28)) { why = "the B200 backend supports images below 2^28 pixels"; return false; }
    if (d.W < 1 || d.H < 1) { why = "empty image"; return false; }
    if (d.max_pairs < 1 || d.max_batch < 1) { why = "bad pair / batch counts"; return false; }
    {
        int ncur = d.nin; long long n = 0;
        for (int l = 0; l < d.nhidden; l++) { n += (long long)d.hidden[l] * ncur + d.hidden[l]; ncur = d.hidden[l]; }
        n += (long long)d.nout * ncur + d.nout;
        if (n * 4 > 48 * 1024) { why = "the B200 backend supports MLPs up to 12288 weights"; return false; }
        I.P = (int)n;
    }
    int nin_check = 0;
    for (int l = 0; l < d.nlev; l++) nin_check += d.lv[l].C;
    nin_check += 2 * d.npos;
    if (nin_check != d.nin) { why = "nin does not match the level channels plus the positional features"; return false; }
    for (int q = 0; q < d.npos; q++)
        if (d.pos[q].kind == ntc_cuda::PK_LV1LOCAL && d.nlev < 2) { why = "lv1local needs a second level"; return false; }
    if (d.qat > 0) {
        if (!d.lv[0].nearest) { why = "--qat needs nearest sampling on level 0"; return false; }
        if (!d.qat_grid) { why = "--qat needs the host grid table"; return false; }
        for (int c = 0; c < d.lv[0].C; c++)
            if (d.qat_bits[c] < 1 || d.qat_bits[c] > 8) { why = "--qat bits out of range"; return false; }
    }

    if (cudaGetDevice(&I.device) != cudaSuccess) { why = "no CUDA device"; return false; }
    cudaDeviceProp prop;
    NTCB_CHECK(cudaGetDeviceProperties(&prop, I.device));
    I.dev_name = prop.name; I.sm_major = prop.major; I.sm_minor = prop.minor; I.sms = prop.multiProcessorCount;
    NTCB_CHECK(cudaRuntimeGetVersion(&I.rt_ver));
    if (prop.major != 10) { why = "libntc_b200 is built for sm_100a (B200) only; this device is sm_" + std::to_string(prop.major * 10 + prop.minor); return false; }
    NTCB_CHECK(cudaStreamCreateWithFlags(&I.own_stream, cudaStreamNonBlocking));
    I.stream = I.own_stream;

    // device model
    DevModel& m = I.dm;
    memset(&m, 0, sizeof(m));
    m.W = d.W; m.H = d.H; m.nlev = d.nlev;
    I.nz = 0;
    for (int l = 0; l < d.nlev; l++) {
        m.lv[l].W = d.lv[l].W; m.lv[l].H = d.lv[l].H; m.lv[l].C = d.lv[l].C; m.lv[l].nearest = d.lv[l].nearest ? 1 : 0;
        m.lv[l].off = (long long)d.lv[l].off;
        I.nz = std::max<long long>(I.nz, (long long)d.lv[l].off + (long long)d.lv[l].W * d.lv[l].H * d.lv[l].C);
    }
    m.npos = d.npos;
    for (int q = 0; q < d.npos; q++) m.pos_kind[q] = d.pos[q].kind;
    m.nin = d.nin; m.nout = d.nout; m.nhidden = d.nhidden;
    for (int l = 0; l < d.nhidden; l++) m.hidden[l] = d.hidden[l];
    m.leak = d.leak; m.clamp_out = d.clamp_out ? 1 : 0;
    for (int c = 0; c < kMaxOut; c++) m.cw[c] = c < d.nout ? d.cw[c] : 0.0f;
    m.wsum = d.wsum; m.P = I.P;
    I.shape = shape_id(m);
    if (const char* e = getenv("NTCB_FORCE_GENERIC")) if (atoi(e)) I.shape = 0;
    I.npix = (long long)d.W * d.H;
    I.n0 = (long long)d.lv[0].W * d.lv[0].H * d.lv[0].C;

    // footprint ranges per level
    {
        std::vector<int> all;
        std::vector<size_t> offs;
        for (int l = 0; l < d.nlev; l++) {
            std::vector<int> xb, xe, yb, ye;
            const bool nr = d.lv[l].nearest;
            if (!axis_ranges(d.W, d.lv[l].W, nr, xb, xe) || !axis_ranges(d.H, d.lv[l].H, nr, yb, ye)) {
                why = "a texel footprint is not contiguous (unsupported level geometry)"; free_all(I); return false;
            }
            if (l == 0 && nr && d.W % d.lv[0].W == 0 && d.H % d.lv[0].H == 0) {
                // uniform cells: texel t covers pixels [t r, (t + 1) r) on both axes (the tensor-core selector search)
                const int rx = d.W / d.lv[0].W, ry = d.H / d.lv[0].H;
                bool uniform = true;
                for (int t = 0; t < d.lv[0].W; t++) uniform = uniform && xb[t] == t * rx && xe[t] == (t + 1) * rx;
                for (int t = 0; t < d.lv[0].H; t++) uniform = uniform && yb[t] == t * ry && ye[t] == (t + 1) * ry;
                if (uniform) { I.qat_cw = rx; I.qat_ch = ry; }
            }
            offs.push_back(all.size());
            all.insert(all.end(), xb.begin(), xb.end()); all.insert(all.end(), xe.begin(), xe.end());
            offs.push_back(all.size());
            all.insert(all.end(), yb.begin(), yb.end()); all.insert(all.end(), ye.begin(), ye.end());
        }
        I.ranges = dalloc<int>(all.size());
        NTCB_CHECK(cudaMemcpy(I.ranges, all.data(), all.size() * sizeof(int), cudaMemcpyHostToDevice));
        I.lvl_xr.clear(); I.lvl_yr.clear();
        for (int l = 0; l < d.nlev; l++) { I.lvl_xr.push_back(I.ranges + offs[2 * l]); I.lvl_yr.push_back(I.ranges + offs[2 * l + 1]); }
    }

    // buffers
    I.z = dalloc<float>(I.nz); I.zgrad = dalloc<float>(I.nz); I.zm = dalloc<float>(I.nz); I.zv = dalloc<float>(I.nz);
    I.ztmp = dalloc<float>(I.nz);
    NTCB_CHECK(cudaMemset(I.zm, 0, I.nz * sizeof(float))); NTCB_CHECK(cudaMemset(I.zv, 0, I.nz * sizeof(float)));
    NTCB_CHECK(cudaMemset(I.zgrad, 0, I.nz * sizeof(float)));
    if (I.qes || I.dct) {
        I.zq = dalloc<float>(I.nz);
        I.qes_dev = dalloc<QesTables>(1);
        NTCB_CHECK(cudaMemset(I.qes_dev, 0, sizeof(QesTables)));
        QesTables qt; memset(&qt, 0, sizeof(qt));
        for (int l = 0; l < d.nlev; l++) qt.bits[l] = d.qes_bits[l];
        NTCB_CHECK(cudaMemcpy(I.qes_dev, &qt, sizeof(qt), cudaMemcpyHostToDevice));
        if (I.qes) {
            const size_t ng = (size_t)kMaxLevels * 64 * 4096;
            I.qgrid = dalloc<float>(ng);
            NTCB_CHECK(cudaMemset(I.qgrid, 0, ng * sizeof(float)));
        }
        if (I.dct) {
            I.dct_n = (long long)(d.W / 8) * (d.H / 8) * d.dct_C;
            I.dsym = dalloc<int16_t>((size_t)I.dct_n * 64); I.dcode = dalloc<uint8_t>((size_t)I.dct_n);
            I.dsteps = dalloc<int>((size_t)d.dct_C * 16 * 64); I.dlam = dalloc<float>(16);
            I.dbits = dalloc<int32_t>((size_t)I.dct_n); I.dcnt = dalloc<int>(3);
            NTCB_CHECK(cudaMemset(I.dsym, 0, (size_t)I.dct_n * 64 * sizeof(int16_t)));
            NTCB_CHECK(cudaMemset(I.dcode, 0, (size_t)I.dct_n));
            NTCB_CHECK(cudaMemset(I.dsteps, 0, (size_t)d.dct_C * 16 * 64 * sizeof(int)));
            NTCB_CHECK(cudaMemset(I.dlam, 0, 16 * sizeof(float)));
            NTCB_CHECK(cudaMemset(I.dbits, 0, (size_t)I.dct_n * sizeof(int32_t)));
            NTCB_CHECK(cudaMemset(I.dcnt, 0, 3 * sizeof(int)));
            DctTables& T = I.dtab;
            memset(&T, 0, sizeof(T));
            T.C = d.dct_C; T.BW = d.W / 8; T.BH = d.H / 8; T.dc_step = d.dct_dc_step; T.deadzone = 1; T.lo_w16 = 16; T.rate_on = 0;
            memcpy(T.basis, d.dct_basis, 64 * sizeof(float));
            memcpy(T.zigzag, d.dct_zigzag, 64 * sizeof(int));
        }
        I.zdec = I.zq;
    } else {
        I.zdec = I.z;
    }
    I.w = dalloc<float>(I.P); I.wgrad = dalloc<float>(I.P); I.wm = dalloc<float>(I.P); I.wv = dalloc<float>(I.P);
    NTCB_CHECK(cudaMemset(I.wm, 0, I.P * sizeof(float))); NTCB_CHECK(cudaMemset(I.wv, 0, I.P * sizeof(float)));
    NTCB_CHECK(cudaMemset(I.wgrad, 0, I.P * sizeof(float)));
    I.tgt = dalloc<float>((size_t)I.npix * d.nout); I.img = dalloc<float>((size_t)I.npix * d.nout);
    I.Mcap = d.max_batch;
    I.mstride = (I.Mcap + 31) / 32 * 32;
    I.bidx = dalloc<int>(I.Mcap);
    NTCB_CHECK(cudaMemset(I.bidx, 0, I.Mcap * sizeof(int)));
    I.feat_t = dalloc<float>((size_t)d.nin * I.mstride);
    I.tgt_t = dalloc<float>((size_t)d.nout * I.mstride);
    I.pairs_cap = d.max_pairs;
    I.mlp_eps = dalloc<float>((size_t)I.pairs_cap * I.P);
    const int cands = std::max(I.pairs_cap, I.P);
    I.fit = dalloc<double>(2 * (size_t)cands);
    I.dl = dalloc<double>(cands); I.lsum = dalloc<double>(cands); I.hh = dalloc<double>(I.P);
    NTCB_CHECK(cudaMemset(I.dl, 0, cands * sizeof(double))); NTCB_CHECK(cudaMemset(I.lsum, 0, cands * sizeof(double)));
    NTCB_CHECK(cudaMemset(I.fit, 0, 2 * cands * sizeof(double)));
    I.fit_stats = dalloc<double>(2);
    I.tc_err = dalloc<int>(1);
    NTCB_CHECK(cudaMemset(I.tc_err, 0, sizeof(int)));
    if (const char* e = getenv("NTCB_POP_KERNEL")) I.tensor_pop = strcmp(e, "ffma") != 0;
    ensure_part(I, (long long)cands * 2 * 8);
    ensure_gpart(I, (long long)((I.pairs_cap + 63) / 64 + 1) * I.P);
    if (d.qat > 0) {
        I.qat_grid = dalloc<float>(9 * 257);
        NTCB_CHECK(cudaMemcpy(I.qat_grid, d.qat_grid, 9 * 257 * sizeof(float), cudaMemcpyHostToDevice));
        I.qat_bits = dalloc<int>(kMaxCh);
        NTCB_CHECK(cudaMemcpy(I.qat_bits, d.qat_bits, kMaxCh * sizeof(int), cudaMemcpyHostToDevice));
    }
    NTCB_CHECK(cudaMemcpy(I.tgt, target, (size_t)I.npix * d.nout * sizeof(float), cudaMemcpyHostToDevice));
    NTCB_CHECK(cudaDeviceSynchronize());
    I.ready = true;
    return true;
}

void require_ready(const Impl& I) { if (!I.ready) die("trainer used before a successful init"); }

void upload_model_impl(Impl& I, const float* z, const float* p) {
    require_ready(I); set_device(I);
    NTCB_CHECK(cudaMemcpyAsync(I.z, z, I.nz * sizeof(float), cudaMemcpyHostToDevice, I.stream));
    NTCB_CHECK(cudaMemcpyAsync(I.w, p, I.P * sizeof(float), cudaMemcpyHostToDevice, I.stream));
    snap_latent_impl(I);
    sync(I);
}

void download_model_impl(Impl& I, float* z, float* p) {
    require_ready(I); set_device(I);
    NTCB_CHECK(cudaMemcpyAsync(z, I.z, I.nz * sizeof(float), cudaMemcpyDeviceToHost, I.stream));
    NTCB_CHECK(cudaMemcpyAsync(p, I.w, I.P * sizeof(float), cudaMemcpyDeviceToHost, I.stream));
    sync(I);
}

void draw_batch(Impl& I, int it, int M) {
    timed(I, "batch", 1, [&] { ntcb::launch_batch(I.stream, I.dm, I.d.seed, it, M, I.mstride, I.zdec, I.tgt, I.bidx, I.feat_t, I.tgt_t); });
    I.last_M = M;
}

// Evaluates the ES pairs [p0, p1) of step `it` on the current minibatch (with `draw`, the minibatch of step `it`
// is drawn first, in the noise kernel's launch); writes (lp, lm) per pair to fit, and with `reduce` (the whole
// population on this trainer) dl and lsum as well.
void es_eval_pairs(Impl& I, int it, float sigma, int M, int p0, int p1, double* fit, bool reduce = false, bool draw = false) {
    const int n = p1 - p0;
    if (draw) {
        timed(I, "batch", 1, [&] {
            ntcb::launch_batch_noise(I.stream, I.dm, I.d.seed, it, M, I.mstride, I.zdec, I.tgt, I.bidx, I.feat_t, I.tgt_t, p0, std::max(n, 0),
                                     I.P, I.mlp_eps);
        });
        I.last_M = M;
    }
    if (n <= 0) return;
    if (!draw) timed(I, "noise", 1, [&] { ntcb::launch_mlp_noise(I.stream, I.d.seed, it, p0, n, I.P, I.mlp_eps); });
    ntcb::PopArgs a{};
    a.mode = 0; a.it = it; a.sigma = sigma; a.fd_h = 0.0f; a.cand_begin = p0; a.ncand = n;
    a.M = M; a.mstride = I.mstride; a.chunk = pop_chunk(I, M);
    a.w0 = I.w; a.eps = I.mlp_eps; a.feat_t = I.feat_t; a.tgt_t = I.tgt_t; a.tc_err = I.tc_err;
    const int chunks = ntcb::pop_chunks(M, a.chunk);
    ensure_part(I, (long long)n * 2 * chunks);
    a.part = I.part;
    timed(I, "mlp_eval", 1, [&] {
        if (!(I.tensor_pop && ntcb::launch_pop_eval_tc(I.stream, I.shape, I.dm, a))) ntcb::launch_pop_eval(I.stream, I.shape, I.dm, a);
    });
    timed(I, "mlp_finish", 1, [&] {
        ntcb::launch_pop_finish(I.stream, I.part, n, chunks, 3.0 * (double)I.d.wsum * M, fit, reduce ? I.dl : nullptr,
                                reduce ? I.lsum : nullptr);
    });
}

// ES gradient from the fitness of all N pairs (pair order) and the Adam step on the weights.
// Pairs per ES gradient segment: partial sums over consecutive pairs, summed in segment order (one segment,
// the reference's serial order, for small populations).
int es_seglen(int N) { return N <= 256 ? N : 64; }

void es_apply(Impl& I, int it, float sigma, float lr, int N, const double* fit_all, bool regenerate_noise, bool reduced = false) {
    if (regenerate_noise) timed(I, "noise", 1, [&] { ntcb::launch_mlp_noise(I.stream, I.d.seed, it, 0, N, I.P, I.mlp_eps); });
    if (!reduced) timed(I, "mlp_finish", 1, [&] { ntcb::launch_es_reduce(I.stream, fit_all, N, I.dl, I.lsum); });
    const float scale = 1.0f / (2.0f * (float)N * sigma);
    const int seglen = es_seglen(N);
    const int nseg = (N + seglen - 1) / seglen;
    ensure_gpart(I, (long long)nseg * I.P);
    timed(I, "mlp_grad", 2, [&] {
        ntcb::launch_es_grad_partial(I.stream, I.dl, I.mlp_eps, N, I.P, scale, seglen, I.gpart);
        I.mlp_t++;
        float c1, c2; adam_coeffs(I.mlp_t, c1, c2);
        ntcb::launch_es_grad_adam(I.stream, I.gpart, nseg, I.P, I.wgrad, I.w, I.wm, I.wv, lr, c1, c2);
    });
    I.last_N = N; I.last_fd = false; I.last_pairs = N; I.dl_pending = 0;
}

// The deferred dl / lsum reduction of a sharded ES step (k_es_reduce over the gathered fitness in fit).
void ensure_dl(const Impl& I) {
    if (I.dl_pending <= 0) return;
    ntcb::launch_es_reduce(I.stream, I.fit, I.dl_pending, I.dl, I.lsum);
    I.dl_pending = 0;
}

void mlp_step_impl(Impl& I, int it, float sigma, float lr, int N, int M) {
    require_ready(I); set_device(I);
    if (N > I.pairs_cap || M > I.Mcap || N < 1 || M < 1) {
        fprintf(stderr, "ntc_b200: MLP step with %d pairs / %d pixels exceeds the buffers sized at init (%d / %d)\n", N, M, I.pairs_cap, I.Mcap);
        exit(1);
    }
    es_eval_pairs(I, it, sigma, M, 0, N, I.fit, true, true);
    es_apply(I, it, sigma, lr, N, I.fit, false, true);
}

// FD candidates [j0, j1) of step `it` on a fresh minibatch: the unperturbed stats pair into fit_stats
// (cuda/ntc_cuda.cu:1059-1068), then (lp, lm) of every weight j in the range (both signs in one CTA) into fit.
void fd_eval_part(Impl& I, int it, float h, int M, int j0, int j1, double* fit) {
    draw_batch(I, it, M);
    const int nw = std::max(0, j1 - j0);
    // one launch: the unperturbed stats pair first, then weights j0 .. j1 - 1 at w_j +- h; on the tensor-core kernel
    // unless the exact kernels are selected (the +- candidates of a weight differ in that weight only, so their
    // 3xTF32 rounding is nearly the same on both sides and cancels in the difference)
    ntcb::PopArgs a{};
    a.mode = 1; a.it = it; a.sigma = 0.0f; a.fd_h = h; a.cand_begin = j0; a.ncand = nw + 1; a.stats_first = 1;
    a.M = M; a.mstride = I.mstride; a.chunk = pop_chunk(I, M);
    a.w0 = I.w; a.eps = I.mlp_eps; a.feat_t = I.feat_t; a.tgt_t = I.tgt_t; a.tc_err = I.tc_err;
    const int chunks = ntcb::pop_chunks(M, a.chunk);
    ensure_part(I, (long long)(nw + 1) * 2 * chunks);
    a.part = I.part;
    const double norm = 3.0 * (double)I.d.wsum * M;
    timed(I, "fd_eval", 1, [&] {
        if (!(I.tensor_pop && ntcb::launch_pop_eval_tc(I.stream, I.shape, I.dm, a))) ntcb::launch_pop_eval(I.stream, I.shape, I.dm, a);
    });
    timed(I, "mlp_finish", nw > 0 ? 2 : 1, [&] {
        ntcb::launch_pop_finish(I.stream, I.part, 1, chunks, norm, I.fit_stats);
        if (nw > 0) ntcb::launch_pop_finish(I.stream, I.part + 2LL * chunks, nw, chunks, norm, fit);
    });
}

// FD gradient from the (lp, lm) of all P weights (weight order; I.fit unless given) and the Adam step.
void fd_apply(Impl& I, float h, float lr, const double* fit = nullptr) {
    timed(I, "mlp_finish", 1, [&] { ntcb::launch_fd_reduce(I.stream, fit ? fit : I.fit, I.w, h, I.P, I.dl, I.hh); });
    timed(I, "mlp_grad", 1, [&] {
        I.mlp_t++;
        float c1, c2; adam_coeffs(I.mlp_t, c1, c2);
        ntcb::launch_fd_grad_adam(I.stream, I.dl, I.hh, I.P, I.wgrad, I.w, I.wm, I.wv, lr, c1, c2);
    });
    I.last_N = I.P; I.last_fd = true; I.last_pairs = 0; I.dl_pending = 0;
}

void mlp_step_fd_impl(Impl& I, int it, float h, float lr, int M) {
    require_ready(I); set_device(I);
    if (M > I.Mcap || M < 1) {
        fprintf(stderr, "ntc_b200: FD step with %d pixels exceeds the buffers sized at init (%d)\n", M, I.Mcap);
        exit(1);
    }
    fd_eval_part(I, it, h, M, 0, I.P, I.fit);
    fd_apply(I, h, lr);
}

// Pinned host doubles for the statistics reads (a pageable destination costs a staged copy per call).
double* ensure_hstage(Impl& I, size_t n) {
    if (n > I.hstage_cap) {
        if (I.hstage) cudaFreeHost(I.hstage);
        I.hstage = nullptr; I.hstage_cap = 0;
        NTCB_CHECK(cudaMallocHost(&I.hstage, n * sizeof(double)));
        I.hstage_cap = n;
    }
    return I.hstage;
}

void mlp_stats_impl(Impl& I, double& batch_loss, double& diff_std) {
    require_ready(I); set_device(I);
    if (I.last_N == 0) { batch_loss = 0; diff_std = 0; return; }
    if (!I.last_fd) {
        ensure_dl(I);
        double* dl = ensure_hstage(I, 2 * (size_t)I.last_N);
        double* ls = dl + I.last_N;
        NTCB_CHECK(cudaMemcpyAsync(dl, I.dl, I.last_N * sizeof(double), cudaMemcpyDeviceToHost, I.stream));
        NTCB_CHECK(cudaMemcpyAsync(ls, I.lsum, I.last_N * sizeof(double), cudaMemcpyDeviceToHost, I.stream));
        sync(I);
        double mean = 0, mean2 = 0, lmean = 0;
        for (int i = 0; i < I.last_N; i++) { mean += dl[i]; mean2 += dl[i] * dl[i]; lmean += ls[i]; }
        mean /= I.last_N; mean2 /= I.last_N; lmean /= I.last_N;
        diff_std = std::sqrt(std::max(0.0, mean2 - mean * mean));
        batch_loss = lmean;
    } else {
        double* dl = ensure_hstage(I, (size_t)I.P + 2);
        double* l0 = dl + I.P;
        NTCB_CHECK(cudaMemcpyAsync(dl, I.dl, I.P * sizeof(double), cudaMemcpyDeviceToHost, I.stream));
        NTCB_CHECK(cudaMemcpyAsync(l0, I.fit_stats, 2 * sizeof(double), cudaMemcpyDeviceToHost, I.stream));
        sync(I);
        double ss = 0;
        for (int j = 0; j < I.P; j++) ss += dl[j] * dl[j];
        diff_std = std::sqrt(ss / I.P);
        batch_loss = 0.5 * (l0[0] + l0[1]);
    }
}

unsigned lat_mask(const Impl& I) {
    const bool qat = I.d.qat > 0;
    unsigned mask = 0;
    for (int l = 0; l < I.d.nlev; l++) if (!(qat && l == 0)) mask |= 1u << l;
    return mask;
}

// The first half of a latent ES step: the noise of every ES-trained texel for the K pairs of this step, and
// the per-pixel loss differences of pixels [p_begin, p_end) written into dpix ([K][W H]).
// Pixels [p_begin, p_end) of all K pairs; pair k's value of pixel p goes to dpix[k * pstride + p - p_begin].
// eps_lo / eps_hi >= 0: the pass reads the noise of flat latent elements [eps_lo, eps_hi) only, and only those are
// generated (a rank's pixel rows of the texel-row split).
void lat_eval_part(Impl& I, float sigma, int K, long long p_begin, long long p_end, float* dpix, long long pstride, long long eps_lo = -1,
                   long long eps_hi = -1) {
    const unsigned mask = lat_mask(I);
    if (!mask) return;
    ensure_lat(I, K);
    int nact = 0;
    for (int l = 0; l < I.d.nlev; l++) if (mask & (1u << l)) nact++;
    const int step = I.lat_step_no;
    timed(I, "lat_noise", eps_lo >= 0 ? 1 : nact, [&] {
        if (eps_lo >= 0) ntcb::launch_lat_noise_range(I.stream, I.d.seed, step, K, eps_lo, eps_hi, I.nz, I.lat_eps);
        else ntcb::launch_lat_noise(I.stream, I.d.seed, step, K, I.dm, mask, I.nz, I.lat_eps);
    });
    const float inv_px = 1.0f / (3.0f * I.d.wsum * (float)I.d.W * (float)I.d.H);
    timed(I, "lat_eval", 1, [&] {
        if (!(I.tensor_pop && ntcb::launch_lat_eval_tc(I.stream, I.shape, I.dm, I.w, I.zdec, I.lat_eps, I.nz, I.tgt, K, mask, sigma,
                                                       inv_px, dpix, p_begin, p_end, pstride, I.tc_err)))
            ntcb::launch_lat_eval(I.stream, I.shape, I.dm, I.w, I.zdec, I.lat_eps, I.nz, I.tgt, K, mask, sigma, inv_px, dpix, p_begin, p_end,
                                  pstride);
    });
}

// The second half: the DCT rate pass, the footprint gathers of every pixel's dpix, Adam, the snap.
// dpix in blocks of rows_per_block image rows, each [K][rows_per_block * W] (one block of H rows: [K][W * H]).
void lat_apply_part(Impl& I, float sigma, float lr, int K, const float* dpix, int rows_per_block) {
    const unsigned mask = lat_mask(I);
    const bool rate = I.dct_live && I.rate_es;
    if (rate) NTCB_CHECK(cudaMemsetAsync(I.dcnt + 2, 0, sizeof(int), I.stream));
    I.dct_evals = rate ? (int)(I.dct_n * K) : 0;
    if (mask) {
        ntcb::RateTerm rt{nullptr, 0.0f, 0, 0};
        if (rate) {
            timed(I, "dct_rate", 1, [&] {
                ntcb::launch_dct_rate_pairs(I.stream, I.dm, I.dtab, K, sigma, I.z, I.lat_eps, I.nz, I.dcode, I.dsteps, I.dlam, I.ddbits, I.dcnt + 2);
            });
            rt.dbits = I.ddbits; rt.rate_scale = I.rate_scale; rt.BW = I.dtab.BW; rt.C = I.dtab.C;
            I.dct_last_K = K;
        }
        const float scale = 1.0f / (2.0f * (float)K * sigma);
        // Adam runs inside each ES-trained level's gather; a level that is never ES-trained (the --qat level) has a
        // zero gradient and zero moments, which leave it unchanged, so skipping it there is exact.
        I.lat_t++;
        float c1, c2; adam_coeffs(I.lat_t, c1, c2);
        const ntcb::LatAdam adam{I.z, I.zm, I.zv, lr, c1, c2};
        for (int l = 0; l < I.d.nlev; l++) {
            if (!(mask & (1u << l))) continue;
            const ntcb::RateTerm r = (l == 0) ? rt : ntcb::RateTerm{nullptr, 0.0f, 0, 0};
            timed(I, "lat_gather", 1, [&] {
                ntcb::launch_lat_gather(I.stream, I.dm, l, I.lvl_xr[l], I.lvl_yr[l], dpix, I.lat_eps, I.nz, K, scale, r, I.zgrad, rows_per_block,
                                        0, I.d.lv[l].H, 0, adam);
            });
        }
    } else {
        I.lat_t++;
    }
    snap_latent_impl(I);
    I.lat_step_no++;
}

// Texel-row sharding of the latent step: with one ES-trained level and no qes / DCT snap (so the decode
// buffer is the latent itself), rank r of G owns texel rows [ta, tb) = [r LH / G, (r + 1) LH / G) of that level
// and evaluates the pixel rows [pa, pb) their footprints cover (its own rows plus a halo); it gathers and
// Adam-updates only its texels, and the ranks exchange the updated level instead of the per-pixel planes.
bool lat_rows_plan(const Impl& I, int world, int rank, int& lvl, int& ta, int& tb, int& pa, int& pb) {
    const unsigned mask = lat_mask(I);
    if (!mask || (mask & (mask - 1)) || I.qes || I.dct || world < 1 || rank < 0 || rank >= world) return false;
    lvl = 0;
    while (!(mask & (1u << lvl))) lvl++;
    const auto& L = I.d.lv[lvl];
    if (L.H % world) return false;
    ta = rank * (L.H / world); tb = ta + L.H / world;
    std::vector<int> yb, ye;
    if (!axis_ranges(I.d.H, L.H, L.nearest, yb, ye)) return false;
    pa = I.d.H; pb = 0;
    for (int t = ta; t < tb; t++) { pa = std::min(pa, yb[t]); pb = std::max(pb, ye[t]); }
    return pb > pa;
}

void lat_step_impl(Impl& I, int it, float sigma, float lr, int K) {
    (void)it;
    require_ready(I); set_device(I);
    if (K < 1) die("lat_step needs K >= 1 pairs");
    if (lat_mask(I)) {
        ensure_lat(I, K);
        lat_eval_part(I, sigma, K, 0, I.npix, I.dpix, I.npix);
    }
    lat_apply_part(I, sigma, lr, K, I.dpix, I.d.H);
}

// Level-0 texels [t_begin, t_end) (row-major over the level) searched in place on the decode buffer.
void qat_rows_part(Impl& I, long long t_begin, long long t_end) {
    if (I.d.qat <= 0) die("qat_search without --qat in the model description");
    timed(I, "qat", 1, [&] {
        int max_bits = 0, min_bits = 64;
        for (int c = 0; c < I.d.lv[0].C; c++) { max_bits = std::max(max_bits, I.d.qat_bits[c]); min_bits = std::min(min_bits, I.d.qat_bits[c]); }
        const bool tc = I.tensor_pop && I.qat_cw > 0 && min_bits == max_bits &&
                        ntcb::launch_qat_tc(I.stream, I.shape, I.dm, I.w, I.zdec, I.tgt, I.qat_grid, max_bits, I.qat_cw, I.qat_ch, t_begin,
                                            t_end, I.tc_err);
        if (!tc)
            ntcb::launch_qat(I.stream, I.shape, I.dm, I.w, I.zdec, I.tgt, I.lvl_xr[0], I.lvl_yr[0], I.qat_grid, I.qat_bits, t_begin, t_end,
                             max_bits);
    });
}
void qat_copy_back(Impl& I) {
    if (I.zdec != I.z)
        NTCB_CHECK(cudaMemcpyAsync(I.z + I.dm.lv[0].off, I.zdec + I.dm.lv[0].off, I.n0 * sizeof(float), cudaMemcpyDeviceToDevice, I.stream));
}

void qat_search_impl(Impl& I) {
    require_ready(I); set_device(I);
    qat_rows_part(I, 0, (long long)I.d.lv[0].W * I.d.lv[0].H);
    qat_copy_back(I);
}

void decode_full_impl(Impl& I, const float* z_host, float* img) {
    require_ready(I); set_device(I);
    const float* src = I.zdec;
    if (z_host) {
        NTCB_CHECK(cudaMemcpyAsync(I.ztmp, z_host, I.nz * sizeof(float), cudaMemcpyHostToDevice, I.stream));
        src = I.ztmp;
    }
    timed(I, "decode", 1, [&] { ntcb::launch_decode(I.stream, I.shape, I.dm, I.w, src, I.img); });
    NTCB_CHECK(cudaMemcpyAsync(img, I.img, (size_t)I.npix * I.d.nout * sizeof(float), cudaMemcpyDeviceToHost, I.stream));
    sync(I);
}

void set_qes_impl(Impl& I, const ntc_cuda::QesDesc& q, const float* grid, size_t grid_n) {
    require_ready(I); set_device(I);
    if (!I.qes) die("set_qes without a --qes level in the model description");
    if (grid_n > (size_t)ntcb::kMaxLevels * 64 * 4096) die("--qes grid table too large");
    NTCB_CHECK(cudaMemcpyAsync(I.qes_dev, &q, sizeof(q), cudaMemcpyHostToDevice, I.stream));
    I.qes_host = q;
    if (grid_n) NTCB_CHECK(cudaMemcpyAsync(I.qgrid, grid, grid_n * sizeof(float), cudaMemcpyHostToDevice, I.stream));
    snap_latent_impl(I);
    sync(I);
}

void set_dct_impl(Impl& I, const ntc_cuda::DctDesc& d, const uint8_t* code, const int16_t* sym, const int* step) {
    require_ready(I); set_device(I);
    if (!I.dct) die("set_dct without --dct-q in the model description");
    if (d.C != I.d.dct_C || (long long)d.BW * d.BH * d.C != I.dct_n || d.N != 8) die("set_dct description mismatch");
    ntcb::DctTables& T = I.dtab;
    T.C = d.C; T.BW = d.BW; T.BH = d.BH; T.dc_step = d.dc_step; T.deadzone = d.deadzone; T.lo_w16 = d.lo_w16;
    T.rate_on = (d.rate_es || d.rate_trunc) ? 1 : 0;
    I.rate_es = d.rate_es != 0; I.rate_trunc = d.rate_trunc != 0; I.rate_scale = d.rate_scale;
    NTCB_CHECK(cudaMemcpyAsync(I.dlam, d.lam_t16, 16 * sizeof(float), cudaMemcpyHostToDevice, I.stream));
    NTCB_CHECK(cudaMemcpyAsync(I.dsteps, step, (size_t)d.C * 16 * 64 * sizeof(int), cudaMemcpyHostToDevice, I.stream));
    NTCB_CHECK(cudaMemcpyAsync(I.dcode, code, (size_t)I.dct_n, cudaMemcpyHostToDevice, I.stream));
    NTCB_CHECK(cudaMemcpyAsync(I.dsym, sym, (size_t)I.dct_n * 64 * sizeof(int16_t), cudaMemcpyHostToDevice, I.stream));
    I.dct_live = true;
    timed(I, "dct_recon", 1, [&] { ntcb::launch_dct_recon(I.stream, I.dm, I.dtab, I.dsym, I.dcode, I.dsteps, I.zq, I.dbits); });
    sync(I);
}

void download_dct_rate_impl(Impl& I, int32_t* bits, int32_t* dbl, int* ntrunc, int* nz_before, int* hits, int* evals) {
    require_ready(I); set_device(I);
    if (!I.dct) return;
    if (bits) NTCB_CHECK(cudaMemcpyAsync(bits, I.dbits, (size_t)I.dct_n * sizeof(int32_t), cudaMemcpyDeviceToHost, I.stream));
    if (dbl) {
        if (I.ddbits && I.dct_last_K > 0)
            NTCB_CHECK(cudaMemcpyAsync(dbl, I.ddbits + (long long)(I.dct_last_K - 1) * I.dct_n, (size_t)I.dct_n * sizeof(int32_t),
                                       cudaMemcpyDeviceToHost, I.stream));
        else memset(dbl, 0, (size_t)I.dct_n * sizeof(int32_t));
    }
    int cnt[3];
    NTCB_CHECK(cudaMemcpyAsync(cnt, I.dcnt, 3 * sizeof(int), cudaMemcpyDeviceToHost, I.stream));
    sync(I);
    if (ntrunc) *ntrunc = cnt[0];
    if (nz_before) *nz_before = cnt[1];
    if (hits) *hits = cnt[2];
    if (evals) *evals = I.dct_evals;
}


void shadow_pull_impl(Impl& I, size_t off, size_t n, float f) {
    require_ready(I); set_device(I);
    if (!I.zq || n == 0) return;
    if ((long long)(off + n) > I.nz) die("shadow_pull range outside the latent");
    timed(I, "snap", 1, [&] { ntcb::launch_shadow_pull(I.stream, I.z, I.zq, (long long)off, (long long)n, f); });
    snap_latent_impl(I);
}
void download_zq_impl(Impl& I, float* zq) {
    require_ready(I); set_device(I);
    NTCB_CHECK(cudaMemcpyAsync(zq, I.zdec, I.nz * sizeof(float), cudaMemcpyDeviceToHost, I.stream));
    sync(I);
}
void download_dct_impl(Impl& I, int16_t* sym, uint8_t* code) {
    require_ready(I); set_device(I);
    if (!I.dct) return;
    NTCB_CHECK(cudaMemcpyAsync(sym, I.dsym, (size_t)I.dct_n * 64 * sizeof(int16_t), cudaMemcpyDeviceToHost, I.stream));
    NTCB_CHECK(cudaMemcpyAsync(code, I.dcode, (size_t)I.dct_n, cudaMemcpyDeviceToHost, I.stream));
    sync(I);
}
void reset_mlp_adam_impl(Impl& I) {
    require_ready(I); set_device(I);
    NTCB_CHECK(cudaMemsetAsync(I.wm, 0, I.P * sizeof(float), I.stream));
    NTCB_CHECK(cudaMemsetAsync(I.wv, 0, I.P * sizeof(float), I.stream));
    I.mlp_t = 0;
}

std::string banner_impl(const Impl& I) {
    char buf[320];
    snprintf(buf, sizeof(buf), "%s (sm_%d%d, %d SMs), CUDA runtime %d.%d, B200 backend (libntc_b200), MLP kernels %s",
             I.dev_name.c_str(), I.sm_major, I.sm_minor, I.sms, I.rt_ver / 1000, (I.rt_ver % 1000) / 10,
             I.shape ? "register-tiled fixed shape" : "runtime-shaped");
    return buf;
}

template <class T>
size_t copy_out(const Impl& I, const T* dev, size_t count, T* out, size_t cap) {
    const size_t n = std::min(count, cap);
    if (n && out) {
        NTCB_CHECK(cudaMemcpyAsync(out, dev, n * sizeof(T), cudaMemcpyDeviceToHost, I.stream));
        NTCB_CHECK(cudaStreamSynchronize(I.stream));
        check_tc_err(I);
    }
    return count;
}

// ---------------------------------------------------------------------- population sharding (one rank's part)
// Size of a rank's ES block for pairs [p0, p1): 2 doubles per pair + P floats per gradient segment, padded to a
// multiple of 16 bytes (the blocks sit back to back in the exchange buffer, and each block's fitness doubles must
// stay 8-byte aligned whatever P is); -1 when the range is not aligned to the segments (or the population is one
// segment).
long long es_part_bytes(const Impl& I, int N, int n) { return 4LL * (n / es_seglen(N)) * I.P; }
long long es_block_bytes(const Impl& I, int N, int p0, int p1) {
    const int seglen = es_seglen(N), n = p1 - p0;
    if (!I.ready || N <= 256 || n <= 0 || p0 % seglen || n % seglen) return -1;
    return (16LL * n + es_part_bytes(I, N, n) + 15) / 16 * 16;
}

// Pairs [p0, p1) of step `it`: minibatch, noise, population, and this rank's block = [fitness | segment sums].
void shard_mlp_eval_grad_impl(Impl& I, int it, float sigma, int N, int M, int p0, int p1, void* block) {
    const int n = p1 - p0, seglen = es_seglen(N);
    double* fit = static_cast<double*>(block);
    float* part = reinterpret_cast<float*>(static_cast<char*>(block) + 16LL * n);
    // minibatch and this rank's pairs' noise (one launch), fitness with the loss differences (one launch), and the
    // gradient segments of these pairs
    es_eval_pairs(I, it, sigma, M, p0, p1, fit, true, true);
    const float scale = 1.0f / (2.0f * (float)N * sigma);
    timed(I, "mlp_grad", 1, [&] { ntcb::launch_es_grad_partial(I.stream, I.dl, I.mlp_eps, n, I.P, scale, seglen, part); });
}

// All ranks' blocks ([rank][block], rank order = pair order) -> the fitness of all N pairs, the segment sums in
// order, the ES gradient and Adam.
void shard_mlp_apply_grad_impl(Impl& I, float lr, int N, const void* blocks, int world) {
    const int n = N / world, seglen = es_seglen(N);
    const long long bytes = es_block_bytes(I, N, 0, n);
    const size_t fit_bytes = 16 * (size_t)n;
    const char* src = static_cast<const char*>(blocks);
    // [rank][fitness | partials | pad] -> fitness of all N pairs in pair order (kept for the statistics); the
    // partials are summed in segment order straight from the blocks
    NTCB_CHECK(cudaMemcpy2DAsync(I.fit, fit_bytes, src, (size_t)bytes, fit_bytes, world, cudaMemcpyDeviceToDevice, I.stream));
    timed(I, "mlp_grad", 1, [&] {
        I.mlp_t++;
        float c1, c2; adam_coeffs(I.mlp_t, c1, c2);
        ntcb::launch_es_grad_adam_ranks(I.stream, reinterpret_cast<const float*>(src + fit_bytes), bytes / 4, world, n / seglen, I.P,
                                        I.wgrad, I.w, I.wm, I.wv, lr, c1, c2);
    });
    I.last_N = N; I.last_fd = false; I.last_pairs = N;
    I.dl_pending = N;   // dl / lsum of all N pairs from I.fit when mlp_stats / debug_last_dl ask
}

// Texel-row latent step of one rank (plan from lat_rows_plan): pixel rows [pa, pb) of all K pairs, gathers and
// Adam of texel rows [ta, tb) of level lvl, in place in the latent. Returns the float offset of those rows.
long long shard_lat_rows_impl(Impl& I, float sigma, float lr, int K, int lvl, int ta, int tb, int pa, int pb) {
    const auto& L = I.d.lv[lvl];
    ensure_lat(I, K);
    const long long W = I.d.W;
    // the texel rows that pixel rows [pa, pb) sample (a superset of [ta, tb), whose gathers read the same noise): the
    // only noise this rank's pass and gathers read
    std::vector<int> yb, ye;
    axis_ranges(I.d.H, L.H, L.nearest, yb, ye);
    int na = L.H, nb = 0;
    for (int t = 0; t < L.H; t++)
        if (yb[t] < pb && ye[t] > pa) { na = std::min(na, t); nb = std::max(nb, t + 1); }
    na = std::min(na, ta); nb = std::max(nb, tb);
    const long long row = (long long)L.W * L.C;
    lat_eval_part(I, sigma, K, (long long)pa * W, (long long)pb * W, I.dpix, (long long)(pb - pa) * W, (long long)L.off + na * row,
                  (long long)L.off + nb * row);
    const long long off = (long long)L.off + (long long)ta * L.W * L.C;
    const float scale = 1.0f / (2.0f * (float)K * sigma);
    I.lat_t++;
    float c1, c2; adam_coeffs(I.lat_t, c1, c2);
    timed(I, "lat_gather", 1, [&] {
        ntcb::launch_lat_gather(I.stream, I.dm, lvl, I.lvl_xr[lvl], I.lvl_yr[lvl], I.dpix, I.lat_eps, I.nz, K, scale,
                                ntcb::RateTerm{nullptr, 0.0f, 0, 0}, I.zgrad, pb - pa, ta, tb, pa, ntcb::LatAdam{I.z, I.zm, I.zv, lr, c1, c2});
    });
    I.lat_step_no++;
    return off;
}

}  // namespace

// ====================================================================== C ABI
struct ntcb_trainer { Impl impl; };

extern "C" {

ntcb_trainer* ntcb_create(void) { return new ntcb_trainer(); }
void ntcb_destroy(ntcb_trainer* t) {
    if (!t) return;
    if (t->impl.ready || t->impl.own_stream) { set_device(t->impl); flush_timing(t->impl); free_all(t->impl); }
    delete t;
}
int ntcb_init(ntcb_trainer* t, const ntcb_model_desc* d, const float* z, const float* p, const float* target, char* why, size_t why_cap) {
    std::string reason;
    if (t->impl.ready) { reason = "trainer already initialised"; }
    else if (init_impl(t->impl, *reinterpret_cast<const ntc_cuda::ModelDesc*>(d), z, p, target, reason)) {
        upload_model_impl(t->impl, z, p);
        return 1;
    }
    if (why && why_cap) { strncpy(why, reason.c_str(), why_cap - 1); why[why_cap - 1] = 0; }
    return 0;
}
size_t ntcb_banner(const ntcb_trainer* t, char* buf, size_t cap) {
    const std::string b = banner_impl(t->impl);
    if (buf && cap) { strncpy(buf, b.c_str(), cap - 1); buf[cap - 1] = 0; }
    return b.size();
}
void ntcb_upload_model(ntcb_trainer* t, const float* z, const float* p) { upload_model_impl(t->impl, z, p); }
void ntcb_download_model(ntcb_trainer* t, float* z, float* p) { download_model_impl(t->impl, z, p); }
void ntcb_set_qes(ntcb_trainer* t, const ntcb_qes_desc* q, const float* grid, size_t grid_n) {
    set_qes_impl(t->impl, *reinterpret_cast<const ntc_cuda::QesDesc*>(q), grid, grid_n);
}
void ntcb_snap_latent(ntcb_trainer* t) { require_ready(t->impl); set_device(t->impl); snap_latent_impl(t->impl); sync(t->impl); }
void ntcb_shadow_pull(ntcb_trainer* t, size_t off, size_t n, float f) { shadow_pull_impl(t->impl, off, n, f); }
void ntcb_download_zq(ntcb_trainer* t, float* zq) { download_zq_impl(t->impl, zq); }
void ntcb_set_dct(ntcb_trainer* t, const ntcb_dct_desc* d, const uint8_t* code, const int16_t* sym, const int* step) {
    set_dct_impl(t->impl, *reinterpret_cast<const ntc_cuda::DctDesc*>(d), code, sym, step);
}
void ntcb_download_dct(ntcb_trainer* t, int16_t* sym, uint8_t* code) { download_dct_impl(t->impl, sym, code); }
void ntcb_download_dct_rate(ntcb_trainer* t, int32_t* bits, int32_t* dbl, int* ntrunc, int* nz_before, int* hits, int* evals) {
    download_dct_rate_impl(t->impl, bits, dbl, ntrunc, nz_before, hits, evals);
}
void ntcb_mlp_step(ntcb_trainer* t, int it, float sigma, float lr, int N, int M) { mlp_step_impl(t->impl, it, sigma, lr, N, M); }
void ntcb_mlp_step_fd(ntcb_trainer* t, int it, float h, float lr, int M) { mlp_step_fd_impl(t->impl, it, h, lr, M); }
void ntcb_reset_mlp_adam(ntcb_trainer* t) { reset_mlp_adam_impl(t->impl); }
void ntcb_mlp_stats(ntcb_trainer* t, double* batch_loss, double* diff_std) {
    double a = 0, b = 0;
    mlp_stats_impl(t->impl, a, b);
    if (batch_loss) *batch_loss = a;
    if (diff_std) *diff_std = b;
}
void ntcb_lat_step(ntcb_trainer* t, int it, float sigma, float lr, int K) { lat_step_impl(t->impl, it, sigma, lr, K); }
void ntcb_qat_search(ntcb_trainer* t) { qat_search_impl(t->impl); }
void ntcb_decode_full(ntcb_trainer* t, const float* z_host, float* img) { decode_full_impl(t->impl, z_host, img); }
size_t ntcb_debug_last_batch(const ntcb_trainer* t, int* out, size_t cap) {
    const Impl& I = t->impl;
    if (!I.ready) return 0;
    return copy_out(I, I.bidx, (size_t)I.last_M, out, cap);
}
size_t ntcb_debug_last_dl(const ntcb_trainer* t, double* out, size_t cap) {
    const Impl& I = t->impl;
    if (!I.ready) return 0;
    if (!I.last_fd) ensure_dl(I);
    return copy_out(I, I.dl, (size_t)I.last_N, out, cap);
}
size_t ntcb_debug_last_zgrad(const ntcb_trainer* t, float* out, size_t cap) {
    const Impl& I = t->impl;
    if (!I.ready) return 0;
    return copy_out(I, I.zgrad, (size_t)I.nz, out, cap);
}
size_t ntcb_debug_last_fitness(const ntcb_trainer* t, double* lp, double* lm, size_t cap) {
    const Impl& I = t->impl;
    if (!I.ready) return 0;
    const size_t n = (size_t)I.last_pairs;
    std::vector<double> f(2 * n);
    copy_out(I, I.fit, 2 * n, f.data(), 2 * n);
    for (size_t i = 0; i < std::min(n, cap); i++) { if (lp) lp[i] = f[2 * i]; if (lm) lm[i] = f[2 * i + 1]; }
    return n;
}
void ntcb_set_stream(ntcb_trainer* t, void* stream) {
    Impl& I = t->impl;
    I.stream = stream ? (cudaStream_t)stream : I.own_stream;
}
void ntcb_kernel_timing(ntcb_trainer* t, int enable) {
    Impl& I = t->impl;
    flush_timing(I);
    I.timing = enable != 0;
}
void ntcb_kernel_timing_only(ntcb_trainer* t, const char* kernel) {
    Impl& I = t->impl;
    flush_timing(I);
    I.timing_only = kernel ? kernel : "";
}
void ntcb_kernel_time(ntcb_trainer* t, const char* kernel, double* total_ms, int* launches) {
    Impl& I = t->impl;
    flush_timing(I);
    auto it = I.totals.find(kernel ? kernel : "");
    if (it == I.totals.end()) { if (total_ms) *total_ms = 0.0; if (launches) *launches = 0; return; }
    if (total_ms) *total_ms = it->second.first;
    if (launches) *launches = it->second.second;
    I.totals.erase(it);
}
long long ntcb_launch_count(const ntcb_trainer* t) { return t->impl.launches; }
// The progress print's statistics (main.cpp:4155-4205) on the device; see ntcb_print_stats. The host part
// below is bitrate_stats' arithmetic (main.cpp:2272-2352) on the device's exact histograms, term for term.
// The bit simulator's totals from the token statistics of k_dct_tokens (dct_analyze, main.cpp:1080-1160): every
// token is charged its symbol's code length -log2(count / total) under the order-0 model (raw, |q|, DC residual,
// scale code) or the context model (run and |q| given the zigzag position of the previous nonzero), so each class
// sums to count x code length over its histogram; one bit per sign; raw fixed lengths dc_raw_bits per block, 7 + 8
// + 1 per nonzero, 7 per EOB, 4 per scale code; a 96-bit header per channel. The progress print has no context
// statistics for the code plane and charges its order-0 figure in the context total too.
static void dct_sim_totals(const int* hist, int C, double nb, int dc_step, double& raw, double& h0, double& ctx, double& header) {
    auto cl0 = [](double cnt, double tot) { return cnt > 0 && tot > 0 ? -std::log2(cnt / tot) : 0.0; };
    auto ent = [&](const int* h, int n, double tot) {
        double e = 0;
        for (int k = 0; k < n; k++) if (h[k]) e += (double)h[k] * cl0(h[k], tot);
        return e;
    };
    int dc_raw_bits = 0;
    { const int lvl = 512 / std::max(1, dc_step) + 1; while ((1 << dc_raw_bits) < lvl) dc_raw_bits++; }
    raw = h0 = ctx = header = 0;
    for (int c = 0; c < C; c++) {
        const int* H = hist + (long long)c * ntcb::kDctHistInts;
        const double nrun = H[ntcb::kDctCounts], neob = H[ntcb::kDctCounts + 1];
        const double dc = ent(H + ntcb::kDctDcres, 4097, nb);
        const double code = ent(H + ntcb::kDctCode, 16, nb);
        const double run0 = ent(H + ntcb::kDctRun, 65, nrun + neob), mag0 = ent(H + ntcb::kDctMag, 257, nrun);
        double runc = 0, magc = 0;
        for (int prev = 0; prev < 64; prev++) {
            const int* cr = H + ntcb::kDctCtxRun + prev * 65;
            const int* cm = H + ntcb::kDctCtxMag + prev * 257;
            double tr = 0, tm = 0;
            for (int r = 0; r < 65; r++) tr += cr[r];
            for (int m = 0; m < 257; m++) tm += cm[m];
            runc += ent(cr, 65, tr);
            magc += ent(cm, 257, tm);
        }
        raw += nb * dc_raw_bits + 16.0 * nrun + 7.0 * neob + 4.0 * nb + 96.0;
        h0 += dc + run0 + mag0 + nrun + code + 96.0;
        ctx += dc + runc + magc + nrun + code + 96.0;
        header += 96.0;
    }
}

static int print_stats_impl(Impl& I, const int* level_bits, int ew, int eh, float* zq_out, ntcb_progress_stats* out) {
    using namespace ntcb;
    require_ready(I); set_device(I);
    const ntc_cuda::ModelDesc& d = I.d;
    const int nl = d.nlev, nb = lat_moment_blocks();
    struct Plan { int mode, hstride; bool dct; int bits[kMaxCh]; long long hist_at, mm_at; };
    std::vector<Plan> plan(nl);
    long long ints = 0;
    for (int l = 0; l < nl; l++) {
        Plan& q = plan[l];
        const int C = d.lv[l].C;
        const bool fixed = l == 0 && d.qat > 0;
        const bool qes = I.qes && I.qes_host.live && I.qes_host.bits[l] > 0;
        q.dct = l == 0 && I.dct_live;
        q.mode = fixed ? 1 : (qes ? 2 : 0);
        q.hstride = 1;
        for (int c = 0; c < C; c++) {
            q.bits[c] = fixed ? d.qat_bits[c] : (qes ? I.qes_host.bits[l] : (level_bits ? level_bits[l] : 8));
            if (!q.dct && (q.bits[c] < 1 || q.bits[c] > 16)) return -1;
            q.hstride = std::max(q.hstride, 1 << std::min(16, std::max(0, q.bits[c])));
        }
        q.mm_at = ints; ints += 2 * C;
        q.hist_at = ints; ints += q.dct ? (long long)C * kDctHistInts : 2LL * C * q.hstride;
    }
    // scratch: [ints] int32, then sse 2 x kMaxOut / 3 u64, the off-grid count u64, moments nl x 3 nb f64
    const size_t o_sse = ((size_t)ints * 4 + 15) / 16 * 16;
    const size_t o_cnt = o_sse + 2 * (kMaxOut / 3) * 8;
    const size_t o_mom = o_cnt + 8;
    const size_t bytes = o_mom + (size_t)nl * 3 * nb * 8;
    if (bytes > I.stats_cap) { dfree(I.stats_buf); I.stats_buf = dalloc<char>(bytes); I.stats_cap = bytes; }
    int* ibuf = reinterpret_cast<int*>(I.stats_buf);
    auto* sse = reinterpret_cast<unsigned long long*>(I.stats_buf + o_sse);
    auto* cnt = reinterpret_cast<unsigned long long*>(I.stats_buf + o_cnt);
    auto* mom = reinterpret_cast<double*>(I.stats_buf + o_mom);
    float* zq = I.ztmp;

    timed(I, "print_stats", 0, [&] {
        for (int l = 0; l < nl; l++) {
            const Plan& q = plan[l];
            const auto& L = d.lv[l];
            const long long ntex = (long long)L.W * L.H, off = I.dm.lv[l].off;
            if (q.dct) {
                NTCB_CHECK(cudaMemcpyAsync(zq + off, I.zdec + off, (size_t)ntex * L.C * sizeof(float), cudaMemcpyDeviceToDevice, I.stream));
                NTCB_CHECK(cudaMemsetAsync(ibuf + q.hist_at, 0, (size_t)L.C * kDctHistInts * sizeof(int), I.stream));
                launch_dct_tokens(I.stream, I.dtab, I.dsym, I.dcode, ibuf + q.hist_at);
                I.launches += 1;
            } else {
                if (q.mode == 0) { launch_level_minmax(I.stream, I.z + off, ntex, L.C, ibuf + q.mm_at); I.launches += 2; }
                LevelQuantArgs a{};
                a.z = I.z + off; a.zd = I.zdec + off; a.zq = zq + off;
                a.W = L.W; a.H = L.H; a.C = L.C; a.mode = q.mode;
                for (int c = 0; c < L.C; c++) {
                    a.bits[c] = q.bits[c];
                    if (q.mode == 2) { a.lo[c] = I.qes_host.lo[l][c]; a.range[c] = I.qes_host.range[l][c]; }
                }
                a.minmax = ibuf + q.mm_at;
                a.dpcm = l > 0 ? 1 : 0;
                a.hist = ibuf + q.hist_at; a.rhist = a.hist + (long long)L.C * q.hstride; a.hstride = q.hstride;
                launch_level_quant(I.stream, a);
                I.launches += 1;
            }
            launch_lat_moments(I.stream, I.z + off, ntex * L.C, mom + (size_t)l * 3 * nb);
            I.launches += 1;
        }
        if (d.qat > 0) { launch_qat_offgrid(I.stream, I.z, I.n0, d.lv[0].C, I.qat_bits, I.qat_grid, cnt); I.launches += 1; }
        else NTCB_CHECK(cudaMemsetAsync(cnt, 0, 8, I.stream));
        if (ew <= 0 || ew > d.W) ew = d.W;
        if (eh <= 0 || eh > d.H) eh = d.H;
        launch_decode(I.stream, I.shape, I.dm, I.w, I.zdec, I.img);
        launch_mse8(I.stream, I.tgt, I.img, d.W, ew, eh, d.nout, sse);
        launch_decode(I.stream, I.shape, I.dm, I.w, zq, I.img);
        launch_mse8(I.stream, I.tgt, I.img, d.W, ew, eh, d.nout, sse + kMaxOut / 3);
        I.launches += 4;
    });
    std::vector<char> h(bytes);
    NTCB_CHECK(cudaMemcpyAsync(h.data(), I.stats_buf, bytes, cudaMemcpyDeviceToHost, I.stream));
    if (zq_out) NTCB_CHECK(cudaMemcpyAsync(zq_out, zq, (size_t)I.nz * sizeof(float), cudaMemcpyDeviceToHost, I.stream));
    sync(I);
    const int* hi = reinterpret_cast<const int*>(h.data());
    const auto* hsse = reinterpret_cast<const unsigned long long*>(h.data() + o_sse);
    const auto* hcnt = reinterpret_cast<const unsigned long long*>(h.data() + o_cnt);
    const auto* hmom = reinterpret_cast<const double*>(h.data() + o_mom);

    ntcb_progress_stats s;
    memset(&s, 0, sizeof(s));
    // mse_of (main.cpp:1779-1787)
    const int T = d.nout / 3;
    const double npe = (double)ew * eh;
    for (int k = 0; k < 2; k++) {
        double* tex = k ? s.mse_q_tex : s.mse_tex;
        double ws = 0.0;
        for (int t = 0; t < T; t++) {
            const double e = (double)hsse[k * (kMaxOut / 3) + t];
            tex[t] = e / (3.0 * npe);
            ws += (double)d.cw[3 * t] * e;
        }
        (k ? s.mse_q : s.mse) = ws / (3.0 * d.wsum * npe);
    }
    // bitrate_stats (main.cpp:2272-2352), progress-print form
    const double npix = (double)d.W * d.H;
    s.bits_mlp = I.P * 16.0;
    s.bpp_fp32 = ((double)I.nz * 32.0 + I.P * 32.0) / npix;
    double ent_bits = 0, header_bits = 0, raw_bits = 0, ctx_bits = 0, est_bits = 0;
    for (int l = 0; l < nl; l++) {
        const Plan& q = plan[l];
        const auto& L = d.lv[l];
        const double ntex = (double)L.W * L.H;
        if (q.dct) {
            // a live DCT-coded level 0: its bit simulator's totals (dct_analyze as the progress print runs it, with the
            // order-0 figure of the code plane in place of its context figure), as bitrate_stats adds them
            // (main.cpp:2294-2301)
            double raw = 0, h0 = 0, ctx = 0, hdr = 0;
            dct_sim_totals(hi + q.hist_at, L.C, (double)L.W / 8 * (L.H / 8), I.dtab.dc_step, raw, h0, ctx, hdr);
            raw_bits += raw - hdr; ent_bits += h0 - hdr; ctx_bits += ctx - hdr; est_bits += h0 - hdr;
            s.bpp_ctx_level0 += (ctx - hdr) / npix;
            header_bits += hdr;
            s.level0_dct = 1;
            s.dct_bits_raw = raw; s.dct_bits_h0 = h0; s.dct_bits_ctx = ctx; s.dct_bits_header = hdr;
            continue;
        }
        const bool fixed = q.mode == 1, qes = q.mode == 2;
        if (!fixed && !qes) raw_bits += (double)((long long)L.W * L.H * L.C) * (double)q.bits[0];
        for (int c = 0; c < L.C; c++) {
            const int levels = (1 << q.bits[c]) - 1;
            if (fixed || qes) raw_bits += ntex * (double)q.bits[c];
            const int* hist = hi + q.hist_at + (long long)c * q.hstride;
            const int* rh = hi + q.hist_at + (long long)(L.C + c) * q.hstride;
            double h0 = 0;
            for (int qv = 0; qv <= levels; qv++)
                if (hist[qv]) h0 -= hist[qv] * std::log2(hist[qv] / ntex);
            ent_bits += h0;
            if (l == 0) { ctx_bits += h0; s.bpp_ctx_level0 += h0 / npix; }
            else ctx_bits += h0;
            if (l == 0) est_bits += h0;
            else {
                double hr = 0;
                for (int qv = 0; qv <= levels; qv++) if (rh[qv]) hr -= rh[qv] * std::log2(rh[qv] / ntex);
                est_bits += hr;
            }
        }
        if (!fixed) header_bits += L.C * 2 * 32.0;
    }
    s.bpp_q8 = (raw_bits + header_bits + s.bits_mlp) / npix;
    s.bpp_q8_ent = (ent_bits + header_bits + s.bits_mlp) / npix;
    s.bpp_q8_ctx = (ctx_bits + header_bits + s.bits_mlp) / npix;
    s.bpp_est = (est_bits + header_bits + s.bits_mlp) / npix;
    s.bits_raw_latent = raw_bits; s.bits_header = header_bits;
    // latent_stats (main.cpp:2212-2217), block partials summed in block order
    for (int l = 0; l < nl; l++) {
        const double* m = hmom + (size_t)l * 3 * nb;
        double sum = 0, s2 = 0, mx = 0;
        for (int b = 0; b < nb; b++) { sum += m[3 * b]; s2 += m[3 * b + 1]; mx = std::max(mx, m[3 * b + 2]); }
        const double n = (double)((long long)d.lv[l].W * d.lv[l].H * d.lv[l].C);
        s.lat_mean[l] = (float)(sum / n);
        s.lat_sd[l] = (float)std::sqrt(std::max(0.0, s2 / n - (sum / n) * (sum / n)));
        s.lat_max[l] = (float)mx;
    }
    s.qat_off_grid = (long long)*hcnt;
    if (out) *out = s;
    return 0;
}

static size_t dct_probe_impl(Impl& I, uint8_t* codes, float* gains, size_t cap) {
    require_ready(I); set_device(I);
    const int BW = I.d.W / 8, BH = I.d.H / 8, C = I.d.lv[0].C;
    const size_t n = (size_t)BW * BH * C;
    if ((!codes && !gains) || n == 0) return n;
    uint8_t* dc = dalloc<uint8_t>(n);
    float* dg = dalloc<float>(n);
    timed(I, "dct_probe", 1, [&] { ntcb::launch_dct_probe(I.stream, I.dm, I.w, I.zdec, BW, BH, C, dc, dg); });
    const size_t k = std::min(n, cap);
    if (codes) NTCB_CHECK(cudaMemcpyAsync(codes, dc, k, cudaMemcpyDeviceToHost, I.stream));
    if (gains) NTCB_CHECK(cudaMemcpyAsync(gains, dg, k * sizeof(float), cudaMemcpyDeviceToHost, I.stream));
    sync(I);
    dfree(dc); dfree(dg);
    return n;
}
size_t ntcb_dct_probe(ntcb_trainer* t, uint8_t* codes, float* gains, size_t cap) { return dct_probe_impl(t->impl, codes, gains, cap); }
int ntcb_shard_lat_plan(const ntcb_trainer* t, int world, int rank, long long* plan) {
    const Impl& I = t->impl;
    int lvl, ta, tb, pa, pb;
    if (!I.ready || !lat_rows_plan(I, world, rank, lvl, ta, tb, pa, pb)) return 0;
    if (plan) {
        plan[0] = lvl; plan[1] = ta; plan[2] = tb; plan[3] = pa; plan[4] = pb;
        plan[5] = (long long)(tb - ta) * I.d.lv[lvl].W * I.d.lv[lvl].C;
    }
    return 1;
}
void ntcb_shard_lat_step_rows(ntcb_trainer* t, int it, float sigma, float lr, int K, int world, int rank, float* zblock_dev) {
    (void)it;
    Impl& I = t->impl;
    require_ready(I); set_device(I);
    int lvl, ta, tb, pa, pb;
    if (K < 1 || !lat_rows_plan(I, world, rank, lvl, ta, tb, pa, pb)) die("shard_lat_step_rows: the texel-row plan does not apply");
    const long long off = shard_lat_rows_impl(I, sigma, lr, K, lvl, ta, tb, pa, pb);
    const long long n = (long long)(tb - ta) * I.d.lv[lvl].W * I.d.lv[lvl].C;
    NTCB_CHECK(cudaMemcpyAsync(zblock_dev, I.z + off, n * sizeof(float), cudaMemcpyDeviceToDevice, I.stream));
}
void ntcb_shard_lat_install(ntcb_trainer* t, int level, const float* level_dev) {
    Impl& I = t->impl;
    require_ready(I); set_device(I);
    if (level < 0 || level >= I.d.nlev) die("shard_lat_install: bad level");
    const auto& L = I.d.lv[level];
    NTCB_CHECK(cudaMemcpyAsync(I.z + L.off, level_dev, (size_t)L.W * L.H * L.C * sizeof(float), cudaMemcpyDeviceToDevice, I.stream));
}
size_t ntcb_cpp_dct_probe(void* cpp_trainer, uint8_t* codes, float* gains, size_t cap) {
    return dct_probe_impl(*static_cast<ntc_cuda::Trainer*>(cpp_trainer)->im, codes, gains, cap);
}
int ntcb_print_stats(ntcb_trainer* t, const int* level_bits, int eval_w, int eval_h, float* zq, ntcb_progress_stats* out) {
    return print_stats_impl(t->impl, level_bits, eval_w, eval_h, zq, out);
}
int ntcb_cpp_print_stats(void* cpp_trainer, const int* level_bits, int eval_w, int eval_h, float* zq, ntcb_progress_stats* out) {
    return print_stats_impl(*static_cast<ntc_cuda::Trainer*>(cpp_trainer)->im, level_bits, eval_w, eval_h, zq, out);
}
void ntcb_set_pop_kernel(ntcb_trainer* t, int tensor) { t->impl.tensor_pop = tensor != 0; }
int ntcb_pop_kernel(const ntcb_trainer* t) { return (t->impl.tensor_pop && t->impl.shape != 0) ? 1 : 0; }
int ntcb_footprint_ranges(int npx, int ntex, int nearest, int* lo, int* hi) {
    std::vector<int> l, h;
    const bool ok = axis_ranges(npx, ntex, nearest != 0, l, h);
    for (int t = 0; t < ntex; t++) { lo[t] = l[t]; hi[t] = h[t]; }
    return ok ? 1 : 0;
}
double ntcb_fp32_peak_tflops(void) {
    int dev = 0; cudaDeviceProp prop;
    NTCB_CHECK(cudaGetDevice(&dev));
    NTCB_CHECK(cudaGetDeviceProperties(&prop, dev));
    return ntcb::measure_ffma_tflops(prop.multiProcessorCount);
}
void ntcb_noise_fill(uint64_t seed, uint32_t stream, uint32_t step, uint32_t pair, uint64_t index0, size_t n,
                     float* gauss_host, uint32_t* u32_host) {
    if (n == 0) return;
    float* g = dalloc<float>(n);
    uint32_t* u = dalloc<uint32_t>(n);
    ntcb::launch_noise_fill(nullptr, seed, stream, step, pair, index0, (long long)n, g, u);
    if (gauss_host) NTCB_CHECK(cudaMemcpy(gauss_host, g, n * sizeof(float), cudaMemcpyDeviceToHost));
    if (u32_host) NTCB_CHECK(cudaMemcpy(u32_host, u, n * sizeof(uint32_t), cudaMemcpyDeviceToHost));
    NTCB_CHECK(cudaDeviceSynchronize());
    dfree(g); dfree(u);
}

void ntcb_shard_mlp_eval(ntcb_trainer* t, int it, float sigma, int N, int M, int pair_begin, int pair_end, double* fit_dev) {
    Impl& I = t->impl;
    require_ready(I); set_device(I);
    if (pair_begin < 0 || pair_end > N || pair_begin > pair_end || N > I.pairs_cap || M > I.Mcap || M < 1)
        die("shard_mlp_eval: pair range or sizes outside the buffers sized at init");
    es_eval_pairs(I, it, sigma, M, pair_begin, pair_end, fit_dev, false, true);
}
void ntcb_shard_lat_eval(ntcb_trainer* t, float sigma, int K, int row_begin, int row_end, float* block_dev) {
    Impl& I = t->impl;
    require_ready(I); set_device(I);
    if (K < 1 || row_begin < 0 || row_end > I.d.H || row_begin > row_end) die("shard_lat_eval: bad pair count or row range");
    lat_eval_part(I, sigma, K, (long long)row_begin * I.d.W, (long long)row_end * I.d.W, block_dev, (long long)(row_end - row_begin) * I.d.W);
}
void ntcb_shard_lat_apply(ntcb_trainer* t, int it, float sigma, float lr, int K, const float* blocks_dev, int rows_per_block) {
    (void)it;
    Impl& I = t->impl;
    require_ready(I); set_device(I);
    if (K < 1) die("shard_lat_apply needs K >= 1 pairs");
    if (rows_per_block < 1 || I.d.H % rows_per_block) die("shard_lat_apply: rows_per_block must divide the image height");
    if (lat_mask(I)) ensure_lat(I, K);
    lat_apply_part(I, sigma, lr, K, blocks_dev, rows_per_block);
}
void ntcb_shard_qat(ntcb_trainer* t, int trow_begin, int trow_end, float* level0_dev) {
    Impl& I = t->impl;
    require_ready(I); set_device(I);
    const int LW = I.d.lv[0].W, LH = I.d.lv[0].H, LC = I.d.lv[0].C;
    if (trow_begin < 0 || trow_end > LH || trow_begin > trow_end) die("shard_qat: bad texel row range");
    qat_rows_part(I, (long long)trow_begin * LW, (long long)trow_end * LW);
    const long long off = (long long)trow_begin * LW * LC, n = (long long)(trow_end - trow_begin) * LW * LC;
    if (n > 0)
        NTCB_CHECK(cudaMemcpyAsync(level0_dev + off, I.zdec + I.dm.lv[0].off + off, n * sizeof(float), cudaMemcpyDeviceToDevice, I.stream));
}
void ntcb_shard_qat_apply(ntcb_trainer* t, const float* level0_all_dev) {
    Impl& I = t->impl;
    require_ready(I); set_device(I);
    NTCB_CHECK(cudaMemcpyAsync(I.zdec + I.dm.lv[0].off, level0_all_dev, I.n0 * sizeof(float), cudaMemcpyDeviceToDevice, I.stream));
    qat_copy_back(I);
}
void ntcb_shard_fd_eval(ntcb_trainer* t, int it, float h, int M, int j_begin, int j_end, double* fit_dev) {
    Impl& I = t->impl;
    require_ready(I); set_device(I);
    if (j_begin < 0 || j_end > I.P || j_begin > j_end || M > I.Mcap || M < 1)
        die("shard_fd_eval: weight range or batch size outside the buffers sized at init");
    fd_eval_part(I, it, h, M, j_begin, j_end, fit_dev);
}
void ntcb_shard_fd_apply(ntcb_trainer* t, float h, float lr, const double* fit_all_dev) {
    Impl& I = t->impl;
    require_ready(I); set_device(I);
    NTCB_CHECK(cudaMemcpyAsync(I.fit, fit_all_dev, 2 * (size_t)I.P * sizeof(double), cudaMemcpyDeviceToDevice, I.stream));
    fd_apply(I, h, lr);
}
long long ntcb_shard_es_block_bytes(const ntcb_trainer* t, int N, int pair_begin, int pair_end) {
    return es_block_bytes(t->impl, N, pair_begin, pair_end);
}
void ntcb_shard_mlp_eval_grad(ntcb_trainer* t, int it, float sigma, int N, int M, int pair_begin, int pair_end, void* block_dev) {
    Impl& I = t->impl;
    require_ready(I); set_device(I);
    if (es_block_bytes(I, N, pair_begin, pair_end) < 0 || N > I.pairs_cap || M > I.Mcap || M < 1)
        die("shard_mlp_eval_grad: pair range not aligned to gradient segments, or sizes outside the buffers sized at init");
    shard_mlp_eval_grad_impl(I, it, sigma, N, M, pair_begin, pair_end, block_dev);
}
void ntcb_shard_mlp_apply_grad(ntcb_trainer* t, int it, float sigma, float lr, int N, int M, const void* blocks_dev, int world) {
    (void)it; (void)sigma; (void)M;
    Impl& I = t->impl;
    require_ready(I); set_device(I);
    if (world < 1 || N % world || N > I.pairs_cap) die("shard_mlp_apply_grad: N must split evenly over the ranks and fit the buffers");
    if (es_block_bytes(I, N, 0, N / world) < 0) die("shard_mlp_apply_grad: the ranks' pair ranges are not aligned to gradient segments");
    shard_mlp_apply_grad_impl(I, lr, N, blocks_dev, world);
}
void ntcb_shard_mlp_apply(ntcb_trainer* t, int it, float sigma, float lr, int N, int M, const double* fit_all_dev) {
    Impl& I = t->impl;
    require_ready(I); set_device(I);
    if (N > I.pairs_cap || N < 1) die("shard_mlp_apply: N outside the buffers sized at init");
    (void)M;
    NTCB_CHECK(cudaMemcpyAsync(I.fit, fit_all_dev, 2 * (size_t)N * sizeof(double), cudaMemcpyDeviceToDevice, I.stream));
    es_apply(I, it, sigma, lr, N, I.fit, true);
}

// ---------------------------------------------------------------------- native sharded iteration (NCCL)
struct ntcb_comm { void* nc = nullptr; int world = 1, rank = 0, device = -1; };

static void set_why(char* why, size_t cap, const std::string& r) {
    if (why && cap) { strncpy(why, r.c_str(), cap - 1); why[cap - 1] = 0; }
}
int ntcb_comm_unique_id(unsigned char* id, char* why, size_t why_cap) {
    std::string r;
    if (!id) { set_why(why, why_cap, "null id buffer"); return 0; }
    if (!ntcb::nccl::unique_id(id, r)) { set_why(why, why_cap, r); return 0; }
    return 1;
}
ntcb_comm* ntcb_comm_create(const unsigned char* id, int world, int rank, char* why, size_t why_cap) {
    if (!id || world < 1 || rank < 0 || rank >= world) { set_why(why, why_cap, "bad id, world size or rank"); return nullptr; }
    int dev = -1;
    NTCB_CHECK(cudaGetDevice(&dev));
    std::string r;
    void* nc = ntcb::nccl::comm_init(id, world, rank, r);
    if (!nc) { set_why(why, why_cap, r); return nullptr; }
    ntcb_comm* c = new ntcb_comm();
    c->nc = nc; c->world = world; c->rank = rank; c->device = dev;
    return c;
}
void ntcb_comm_destroy(ntcb_comm* c) {
    if (!c) return;
    int prev = -1;
    NTCB_CHECK(cudaGetDevice(&prev));
    NTCB_CHECK(cudaSetDevice(c->device));
    ntcb::nccl::comm_destroy(c->nc);
    NTCB_CHECK(cudaSetDevice(prev));
    delete c;
}
int ntcb_nccl_version(void) { return ntcb::nccl::version(); }

// Which exchange each phase of ntcb_shard_iteration uses for this model and world size (0 = refused, reason in
// why): mlp 1 = segment blocks (fitness + ES gradient segments), 2 = fitness only (every rank regenerates all
// noise for the gradient); latent 1 = texel rows (the updated level), 2 = pixel rows (the K loss-difference
// planes); FD and selector search have one form each.
static int iteration_plan(const Impl& I, int world, int rank, int mlp_mode, int N, int M, int K, int qat, int& mlp_x, int& lat_x,
                          std::string& why) {
    mlp_x = 0; lat_x = 0;
    if (!I.ready) { why = "trainer not initialised"; return 0; }
    if (world < 1 || rank < 0 || rank >= world) { why = "bad world size or rank"; return 0; }
    if (mlp_mode < 0 || mlp_mode > 2) { why = "mlp mode must be 0 (none), 1 (ES) or 2 (FD)"; return 0; }
    if (mlp_mode != 0 && (M < 1 || M > I.Mcap)) { why = "minibatch outside the buffers sized at init"; return 0; }
    if (mlp_mode == 1) {
        if (N < 1 || N > I.pairs_cap || N % world) { why = "the ES pairs must split evenly over the ranks and fit the buffers sized at init"; return 0; }
        mlp_x = es_block_bytes(I, N, rank * (N / world), (rank + 1) * (N / world)) > 0 ? 1 : 2;
    }
    if (K > 0 && lat_mask(I)) {
        int lvl, ta, tb, pa, pb;
        if (lat_rows_plan(I, world, rank, lvl, ta, tb, pa, pb)) lat_x = 1;
        else if (I.d.H % world == 0) lat_x = 2;
        else { why = "the image height does not split evenly over the ranks"; return 0; }
    }
    if (qat) {
        if (I.d.qat <= 0) { why = "selector search requested for a model without --qat"; return 0; }
        if (I.d.lv[0].H % world) { why = "the level-0 rows do not split evenly over the ranks"; return 0; }
    }
    return 1;
}

int ntcb_shard_iteration_plan(const ntcb_trainer* t, int world, int rank, int mlp_mode, int N, int M, int K, int qat, int* mlp_exchange,
                              int* lat_exchange, char* why, size_t why_cap) {
    int mx = 0, lx = 0;
    std::string r;
    const int ok = iteration_plan(t->impl, world, rank, mlp_mode, N, M, K, qat, mx, lx, r);
    if (mlp_exchange) *mlp_exchange = mx;
    if (lat_exchange) *lat_exchange = lx;
    if (!ok) set_why(why, why_cap, r);
    return ok;
}

// Largest block one rank contributes to any exchange of ntcb_shard_iteration for (world, N, K) and both MLP modes.
static size_t max_exchange_block(const Impl& I, int world, int rank, int N, int K, int qat, int mx, int lx) {
    size_t cap = 0;
    const int n = N / world;
    cap = std::max(cap, mx == 1 ? (size_t)es_block_bytes(I, N, rank * n, (rank + 1) * n) : 16 * (size_t)n);
    cap = std::max(cap, 2 * (size_t)((I.P + world - 1) / world) * sizeof(double));
    if (lx == 1) {
        int lvl, ta, tb, pa, pb;
        lat_rows_plan(I, world, rank, lvl, ta, tb, pa, pb);
        cap = std::max(cap, (size_t)(tb - ta) * I.d.lv[lvl].W * I.d.lv[lvl].C * sizeof(float));
    } else if (lx == 2) {
        cap = std::max(cap, (size_t)K * (I.d.H / world) * I.d.W * sizeof(float));
    }
    if (qat) cap = std::max(cap, (size_t)(I.d.lv[0].H / world) * I.d.lv[0].W * I.d.lv[0].C * sizeof(float));
    return (cap + 255) / 256 * 256;
}

int ntcb_p2p_export(ntcb_trainer* t, int world, int rank, int N, int K, int qat, unsigned char* handle, char* why, size_t why_cap) {
    Impl& I = t->impl;
    std::string r;
    int mx = 0, lx = 0;
    if (!I.ready) { set_why(why, why_cap, "trainer not initialised"); return 0; }
    set_device(I);
    if (world < 1 || world > ntcb::kP2PMaxRanks) { set_why(why, why_cap, "peer exchange supports 1-8 ranks"); return 0; }
    if (!iteration_plan(I, world, rank, 1, N, 1, K, qat, mx, lx, r)) { set_why(why, why_cap, r); return 0; }
    if (I.p2p_buf) { set_why(why, why_cap, "peer exchange already set up for this trainer"); return 0; }
    const size_t cap = (ntcb::p2p_stage_bytes(max_exchange_block(I, world, rank, N, K, qat, mx, lx)) + 255) / 256 * 256;
    if (cap / 16 * (size_t)std::max(1, world - 1) >= (1ull << 31)) {   // the exchange kernel indexes (peer, line) tasks in 32 bits
        set_why(why, why_cap, "exchange blocks too large for the peer exchange (use the NCCL exchange)");
        return 0;
    }
    const size_t total = ntcb::kP2PHeader + 2 * (size_t)world * cap;
    I.p2p_buf = dalloc<char>(total);
    NTCB_CHECK(cudaMemset(I.p2p_buf, 0, total));
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, I.p2p_buf) != cudaSuccess) {
        cudaGetLastError();
        dfree(I.p2p_buf);
        set_why(why, why_cap, "cudaIpcGetMemHandle failed");
        return 0;
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    memcpy(handle, &h, sizeof(h));
    I.p2p = ntcb::P2PArgs{};
    I.p2p.world = world; I.p2p.rank = rank; I.p2p.cap = cap;
    I.p2p.base[rank] = I.p2p_buf;
    return 1;
}

int ntcb_p2p_import(ntcb_trainer* t, const unsigned char* handles, int world, int rank, char* why, size_t why_cap) {
    Impl& I = t->impl;
    if (!I.p2p_buf || I.p2p.world != world || I.p2p.rank != rank || I.p2p_ready) {
        set_why(why, why_cap, "ntcb_p2p_export with the same world size and rank must come first, once");
        return 0;
    }
    set_device(I);
    for (int q = 0; q < world; q++) {
        if (q == rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, handles + 64 * (size_t)q, sizeof(h));
        void* p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            cudaGetLastError();
            for (int j = 0; j < q; j++) if (j != rank && I.p2p.base[j]) { cudaIpcCloseMemHandle(I.p2p.base[j]); I.p2p.base[j] = nullptr; }
            set_why(why, why_cap, std::string("cudaIpcOpenMemHandle failed for rank ") + std::to_string(q) + ": " + cudaGetErrorString(e));
            return 0;
        }
        I.p2p.base[q] = static_cast<char*>(p);
    }
    I.p2p_ready = true;
    I.p2p_epoch = 0;
    return 1;
}

void ntcb_p2p_set_poll_limit(ntcb_trainer* t, unsigned polls) {
    t->impl.p2p_poll_limit = polls ? polls : ntcb::kP2PPollLimit;
}

int ntcb_p2p_barrier(ntcb_trainer* t, unsigned polls) {
    Impl& I = t->impl;
    require_ready(I); set_device(I);
    if (!I.p2p_ready) die("p2p_barrier: no peer exchange set up (ntcb_p2p_export / ntcb_p2p_import)");
    // one 4-byte token per rank, all-gathered through the staging into this rank's header slots
    char* slots = I.p2p_buf;
    static_assert(ntcb::kP2PHeader >= 4 * ntcb::kP2PMaxRanks, "barrier token slots");
    const uint32_t token = I.p2p_epoch + 1;
    NTCB_CHECK(cudaMemcpyAsync(slots + 4 * (size_t)I.p2p.rank, &token, 4, cudaMemcpyHostToDevice, I.stream));
    I.p2p_epoch++;
    ntcb::launch_p2p_allgather(I.stream, I.p2p, slots, 4, I.p2p_epoch, polls ? polls : I.p2p_poll_limit, I.tc_err);
    NTCB_CHECK(cudaStreamSynchronize(I.stream));
    int e = 0;
    NTCB_CHECK(cudaMemcpy(&e, I.tc_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (e) NTCB_CHECK(cudaMemset(I.tc_err, 0, sizeof(int)));
    return e;
}

void ntcb_p2p_release(ntcb_trainer* t) {
    Impl& I = t->impl;
    if (!I.p2p_ready) return;
    set_device(I);
    NTCB_CHECK(cudaStreamSynchronize(I.stream));
    for (int q = 0; q < I.p2p.world; q++)
        if (q != I.p2p.rank && I.p2p.base[q]) { cudaIpcCloseMemHandle(I.p2p.base[q]); I.p2p.base[q] = nullptr; }
    I.p2p_ready = false;
}

void ntcb_shard_iteration(ntcb_trainer* t, ntcb_comm* c, int it, int mlp_mode, float mlp_sigma, float mlp_lr, int N, int M, int K,
                          float lat_sigma, float lat_lr, int qat) {
    Impl& I = t->impl;
    require_ready(I); set_device(I);
    if (!c || c->device != I.device) die("shard_iteration: no communicator, or one made on another device");
    const int G = c->world, r = c->rank;
    int mx = 0, lx = 0;
    std::string why;
    if (!iteration_plan(I, G, r, mlp_mode, N, M, K, qat, mx, lx, why)) die(("shard_iteration: " + why).c_str());
    const bool p2p = I.p2p_ready && I.p2p.world == G && I.p2p.rank == r;
    auto gather = [&](void* buf, size_t bytes) {
        if (p2p) {
            if (bytes % 4 || ntcb::p2p_stage_bytes(bytes) > I.p2p.cap)
                die("shard_iteration: an exchange block does not fit the peer buffers set up for it");
            I.p2p_epoch++;
            timed(I, "exchange", 1, [&] { ntcb::launch_p2p_allgather(I.stream, I.p2p, buf, bytes, I.p2p_epoch, I.p2p_poll_limit, I.tc_err); });
        } else {
            timed(I, "exchange", 0, [&] { ntcb::nccl::all_gather_inplace(c->nc, buf, bytes, r, I.stream); });
        }
    };
    // MLP step (mlp_step / mlp_step_fd)
    if (mlp_mode == 1) {
        const int n = N / G, p0 = r * n;
        if (mx == 1) {
            const long long block = es_block_bytes(I, N, p0, p0 + n);
            ensure_xbuf(I, block * G);
            shard_mlp_eval_grad_impl(I, it, mlp_sigma, N, M, p0, p0 + n, I.xbuf + (long long)r * block);
            gather(I.xbuf, (size_t)block);
            shard_mlp_apply_grad_impl(I, mlp_lr, N, I.xbuf, G);
        } else {
            const size_t bytes = 16 * (size_t)n;
            ensure_xbuf(I, (long long)bytes * G);
            es_eval_pairs(I, it, mlp_sigma, M, p0, p0 + n, reinterpret_cast<double*>(I.xbuf + (size_t)r * bytes), false, true);
            gather(I.xbuf, bytes);
            es_apply(I, it, mlp_sigma, mlp_lr, N, reinterpret_cast<const double*>(I.xbuf), true);
        }
    } else if (mlp_mode == 2) {
        const int B = (I.P + G - 1) / G, j0 = std::min(r * B, I.P), j1 = std::min((r + 1) * B, I.P);
        const size_t bytes = 2 * (size_t)B * sizeof(double);
        ensure_xbuf(I, (long long)bytes * G);
        fd_eval_part(I, it, mlp_sigma, M, j0, j1, reinterpret_cast<double*>(I.xbuf + (size_t)r * bytes));
        gather(I.xbuf, bytes);
        fd_apply(I, mlp_sigma, mlp_lr, reinterpret_cast<const double*>(I.xbuf));
    }
    // latent ES step (lat_step)
    if (lx == 1) {
        int lvl, ta, tb, pa, pb;
        lat_rows_plan(I, G, r, lvl, ta, tb, pa, pb);
        shard_lat_rows_impl(I, lat_sigma, lat_lr, K, lvl, ta, tb, pa, pb);
        const auto& L = I.d.lv[lvl];
        gather(I.z + L.off, (size_t)(tb - ta) * L.W * L.C * sizeof(float));
    } else if (lx == 2) {
        const int rows = I.d.H / G;
        const long long plane = (long long)rows * I.d.W;
        ensure_lat(I, K);
        lat_eval_part(I, lat_sigma, K, (long long)r * plane, (long long)(r + 1) * plane, I.dpix + (long long)r * K * plane, plane);
        gather(I.dpix, (size_t)K * plane * sizeof(float));
        lat_apply_part(I, lat_sigma, lat_lr, K, I.dpix, rows);
    }
    // selector search (qat_search)
    if (qat) {
        const long long LW = I.d.lv[0].W, LC = I.d.lv[0].C, rows = I.d.lv[0].H / G;
        qat_rows_part(I, r * rows * LW, (r + 1) * rows * LW);
        // the searched rows travel as one-byte grid indices (exact both ways), blocks padded to whole 4-byte words
        const long long n = rows * LW * LC;
        const size_t blk = ((size_t)n + 3) / 4 * 4;
        ensure_xbuf(I, (long long)blk * G);
        float* z0 = I.zdec + I.dm.lv[0].off;
        uint8_t* xb = reinterpret_cast<uint8_t*>(I.xbuf);
        ntcb::launch_qat_pack(I.stream, z0 + r * n, n, (int)LC, I.qat_bits, xb + (size_t)r * blk);
        gather(I.xbuf, blk);
        ntcb::launch_qat_unpack(I.stream, xb, (long long)blk, n, G, (int)LC, I.qat_bits, I.qat_grid, z0);
        qat_copy_back(I);
    }
}

}  // extern "C"

// ====================================================================== drop-in C++ class
namespace ntc_cuda {

Trainer::Trainer() : im(new Impl) {}
Trainer::~Trainer() {
    if (im->ready || im->own_stream) { set_device(*im); flush_timing(*im); free_all(*im); }
    delete im;
}
bool Trainer::init(const ModelDesc& d, const float* z, const float* p, const float* target, std::string& why) {
    if (im->ready) { why = "trainer already initialised"; return false; }
    if (!init_impl(*im, d, z, p, target, why)) return false;
    upload_model_impl(*im, z, p);
    return true;
}
std::string Trainer::banner() const { return banner_impl(*im); }
void Trainer::upload_model(const float* z, const float* p) { upload_model_impl(*im, z, p); }
void Trainer::download_model(float* z, float* p) { download_model_impl(*im, z, p); }
void Trainer::set_qes(const QesDesc& q, const float* grid, size_t grid_n) { set_qes_impl(*im, q, grid, grid_n); }
void Trainer::snap_latent() { require_ready(*im); set_device(*im); snap_latent_impl(*im); sync(*im); }
void Trainer::shadow_pull(size_t off, size_t n, float f) { shadow_pull_impl(*im, off, n, f); }
void Trainer::download_zq(float* zq) { download_zq_impl(*im, zq); }
void Trainer::set_dct(const DctDesc& d, const uint8_t* code, const int16_t* sym, const int* step) { set_dct_impl(*im, d, code, sym, step); }
void Trainer::download_dct(int16_t* sym, uint8_t* code) { download_dct_impl(*im, sym, code); }
void Trainer::download_dct_rate(int32_t* bits, int32_t* dbl, int* ntrunc, int* nz_before, int* hits, int* evals) {
    download_dct_rate_impl(*im, bits, dbl, ntrunc, nz_before, hits, evals);
}
void Trainer::mlp_step(int it, float sigma, float lr, int N, int M) { mlp_step_impl(*im, it, sigma, lr, N, M); }
void Trainer::mlp_step_fd(int it, float h, float lr, int M) { mlp_step_fd_impl(*im, it, h, lr, M); }
void Trainer::reset_mlp_adam() { reset_mlp_adam_impl(*im); }
void Trainer::mlp_stats(double& batch_loss, double& diff_std) { mlp_stats_impl(*im, batch_loss, diff_std); }
void Trainer::lat_step(int it, float sigma, float lr, int K) { lat_step_impl(*im, it, sigma, lr, K); }
void Trainer::qat_search() { qat_search_impl(*im); }
void Trainer::decode_full(const float* z_host, float* img) { decode_full_impl(*im, z_host, img); }
void Trainer::debug_last_batch(std::vector<int>& bidx) const {
    bidx.resize(im->last_M);
    if (im->ready) copy_out(*im, im->bidx, bidx.size(), bidx.data(), bidx.size());
}
void Trainer::debug_last_dl(std::vector<double>& dl) const {
    dl.resize(im->last_N);
    if (im->ready && !im->last_fd) ensure_dl(*im);
    if (im->ready) copy_out(*im, im->dl, dl.size(), dl.data(), dl.size());
}
void Trainer::debug_last_zgrad(std::vector<float>& g) const {
    g.resize(im->nz);
    if (im->ready) copy_out(*im, im->zgrad, g.size(), g.data(), g.size());
}

}  // namespace ntc_cuda
