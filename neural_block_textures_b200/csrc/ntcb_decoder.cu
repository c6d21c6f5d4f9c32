// Decoder of .ntcb containers on the device: the inference-side neighbour of the trainer (the reference's
// ntc_decode.cpp is its SSE4.1 CPU counterpart). The host parser (ntcb_format.cpp) validates the file and
// parses the DCT tokens and fp16 weights; the whole file is uploaded once and every fixed-width grid index is
// unpacked by its own thread straight from the bit stream; a DCT-coded level 0 is reconstructed by the
// trainer's own strict-FP kernel; the image is decoded by the trainer's decode kernels and quantized to RGB8
// as the reference writes PNGs (lround(clamp(v, 0, 1) * 255), one RGB plane per texture, cropped to the
// source size).
#include "kernels.h"
#include "kernels_snap.h"
#include "ntcb_format.h"
#include "quant.cuh"
#include "../../include/ntc_b200.h"

#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

namespace ntcb {

namespace {

inline unsigned blocks_for(long long n, int tpb) { return (unsigned)((n + tpb - 1) / tpb); }

// One grid level's unpack: index k of (texel t, channel c) sits at bit `chan_bit[c] + t bits[c]` of the body.
struct UnpackArgs {
    const uint8_t* body;          // the level's section body (device copy of the file, padded by 8 bytes)
    float* z;                     // the level's latent [W * H][C]
    long long ntex;
    int C, mode;
    long long chan_bit[kMaxCh];
    int bits[kMaxCh];
    const float* table;           // mode 0 / 1: [C][2] (lo, range); mode 2: [C][256] palette
};

__global__ void k_ntcb_unpack(UnpackArgs a) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= a.ntex * a.C) return;
    const int c = (int)(i / a.ntex);
    const long long t = i - (long long)c * a.ntex;
    const int b = a.bits[c];
    const unsigned long long bit = (unsigned long long)a.chan_bit[c] + (unsigned long long)t * (unsigned long long)b;
    const uint8_t* p = a.body + (bit >> 3);
    const uint32_t w = (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
    const int k = (int)((w >> (bit & 7)) & ((1u << b) - 1u));
    float v;
    if (a.mode == 2) v = a.table[c * 256 + k];
    else v = q8_value_dev(k, a.table[2 * c], a.table[2 * c + 1], (1 << b) - 1);   // lo + k / levels * range, strict
    a.z[t * a.C + c] = v;
}

// RGB8 of the crop: out[t][y][x][3] = lround(clamp(img, 0, 1) * 255) of texture t's three outputs.
__global__ void k_ntcb_rgb8(const float* __restrict__ img, int W, int nout, int cw, int ch, uint8_t* __restrict__ out) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long npx = (long long)cw * ch;
    if (i >= npx * (nout / 3)) return;
    const int t = (int)(i / npx);
    const long long q = i - (long long)t * npx;
    const int y = (int)(q / cw), x = (int)(q - (long long)y * cw);
    const float* s = img + ((long long)y * W + x) * nout + 3 * t;
    uint8_t* d = out + i * 3;
#pragma unroll
    for (int c = 0; c < 3; c++) d[c] = (uint8_t)lroundf(fminf(1.0f, fmaxf(0.0f, s[c])) * 255.0f);
}

void fill_info(const NtcbFile& f, long long nz, ntcb_container_desc* info) {
    memset(info, 0, sizeof(*info));
    info->version = f.version; info->img_w = f.img_w; info->img_h = f.img_h; info->src_w = f.src_w; info->src_h = f.src_h;
    info->T = f.T; info->nlevels = f.nlevels; info->nin = f.nin; info->nout = f.nout; info->nhidden = f.nhidden;
    for (int l = 0; l < f.nhidden && l < NTCB_MAX_HIDDEN; l++) info->hidden[l] = f.hidden[(size_t)l];
    info->leak = f.leak; info->clamp_out = f.clamp;
    for (int l = 0; l < f.nlevels; l++) {
        const NtcbLevelRec& L = f.lv[(size_t)l];
        info->lv_W[l] = L.W; info->lv_H[l] = L.H; info->lv_C[l] = L.C; info->lv_nearest[l] = L.nearest; info->lv_mode[l] = L.mode;
        info->lv_bits[l] = L.bits.empty() ? 0 : L.bits[0];
    }
    info->npos = (int)f.pos_kinds.size();
    for (size_t q = 0; q < f.pos_kinds.size() && q < NTCB_MAX_POS; q++) info->pos_kind[q] = f.pos_kinds[q];
    info->nz = nz;
    info->nweights = (long long)f.weights.size();
}

void set_err(const std::string& e, char* err, size_t cap) {
    if (err && cap) { const size_t k = std::min(cap - 1, e.size()); memcpy(err, e.data(), k); err[k] = 0; }
}

long long latent_size(const NtcbFile& f) {
    long long nz = 0;
    for (const NtcbLevelRec& L : f.lv) nz += (long long)L.W * L.H * L.C;
    return nz;
}

}  // namespace
}  // namespace ntcb

struct ntcb_decoder {
    ntcb::NtcbFile f;
    ntcb::DevModel dm{};
    int shape = 0;
    long long nz = 0;
    cudaStream_t stream = nullptr;
    uint8_t* bytes = nullptr;
    float *z = nullptr, *w = nullptr, *img = nullptr, *tables = nullptr;
    int16_t* sym = nullptr; uint8_t* code = nullptr; int* steps = nullptr;
    uint8_t* rgb = nullptr; size_t rgb_cap = 0;
};

namespace {

template <class T>
T* dev_alloc(size_t n) {
    T* p = nullptr;
    NTCB_CHECK(cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)));
    return p;
}
template <class T>
void dev_free(T*& p) { if (p) { cudaFree(p); p = nullptr; } }

void release(ntcb_decoder* d) {
    dev_free(d->bytes); dev_free(d->z); dev_free(d->w); dev_free(d->img); dev_free(d->tables);
    dev_free(d->sym); dev_free(d->code); dev_free(d->steps); dev_free(d->rgb);
    if (d->stream) { cudaStreamDestroy(d->stream); d->stream = nullptr; }
}

}  // namespace

extern "C" {

int ntcb_container_info(const uint8_t* bytes, size_t n, ntcb_container_desc* info, char* err, size_t err_cap) {
    ntcb::NtcbFile f;
    std::string e;
    if (!bytes || !ntcb::ntcb_parse(bytes, n, f, e)) { ntcb::set_err(bytes ? e : "null buffer", err, err_cap); return -1; }
    if (info) ntcb::fill_info(f, ntcb::latent_size(f), info);
    ntcb::set_err("", err, err_cap);
    return 0;
}

void ntcb_dct_tables(int q, int dc_step, float* basis, int* zigzag, int* steps) {
    if (basis) ntcb::dct_basis(basis);
    if (zigzag) ntcb::dct_zigzag(zigzag);
    if (steps) ntcb::dct_steps(q, dc_step, steps);
}

ntcb_decoder* ntcb_decoder_open(const uint8_t* bytes, size_t n, char* err, size_t err_cap) {
    using namespace ntcb;
    auto* d = new ntcb_decoder();
    std::string e;
    if (!bytes || !ntcb_parse(bytes, n, d->f, e)) { set_err(bytes ? e : "null buffer", err, err_cap); delete d; return nullptr; }
    const NtcbFile& f = d->f;
    int dev = 0;
    cudaDeviceProp prop;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaGetDeviceProperties(&prop, dev) != cudaSuccess) { set_err("no CUDA device", err, err_cap); delete d; return nullptr; }
    if (prop.major != 10) { set_err("libntc_b200 is built for sm_100a (B200) only", err, err_cap); delete d; return nullptr; }
    if ((long long)f.img_w * f.img_h >= (1ll << 28)) { set_err("the device decoder takes images below 2^28 pixels", err, err_cap); delete d; return nullptr; }
    for (const NtcbLevelRec& L : f.lv) if (L.C > kMaxCh) { set_err("the device decoder takes at most 16 channels per level", err, err_cap); delete d; return nullptr; }
    if ((long long)f.weights.size() * 4 > 48 * 1024) { set_err("the device decoder takes MLPs up to 12288 weights", err, err_cap); delete d; return nullptr; }

    // the device model of the container (decode size = the header's image size)
    DevModel& m = d->dm;
    memset(&m, 0, sizeof(m));
    m.W = f.img_w; m.H = f.img_h; m.nlev = f.nlevels;
    long long off = 0;
    for (int l = 0; l < f.nlevels; l++) {
        const NtcbLevelRec& L = f.lv[(size_t)l];
        m.lv[l].W = L.W; m.lv[l].H = L.H; m.lv[l].C = L.C; m.lv[l].nearest = L.nearest; m.lv[l].off = off;
        off += (long long)L.W * L.H * L.C;
    }
    d->nz = off;
    m.npos = (int)f.pos_kinds.size();
    for (int q = 0; q < m.npos; q++) m.pos_kind[q] = f.pos_kinds[(size_t)q];
    m.nin = f.nin; m.nout = f.nout; m.nhidden = f.nhidden;
    for (int l = 0; l < f.nhidden; l++) m.hidden[l] = f.hidden[(size_t)l];
    m.leak = f.leak; m.clamp_out = f.clamp;
    for (int c = 0; c < kMaxOut; c++) m.cw[c] = c < f.nout ? 1.0f : 0.0f;
    m.wsum = (float)f.T; m.P = (int)f.weights.size();
    d->shape = shape_id(m);

    NTCB_CHECK(cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking));
    cudaStream_t s = d->stream;
    d->bytes = dev_alloc<uint8_t>(n + 8);
    NTCB_CHECK(cudaMemsetAsync(d->bytes + n, 0, 8, s));
    NTCB_CHECK(cudaMemcpyAsync(d->bytes, bytes, n, cudaMemcpyHostToDevice, s));
    d->z = dev_alloc<float>((size_t)d->nz);
    d->w = dev_alloc<float>(f.weights.size());
    NTCB_CHECK(cudaMemcpyAsync(d->w, f.weights.data(), f.weights.size() * sizeof(float), cudaMemcpyHostToDevice, s));
    d->img = dev_alloc<float>((size_t)f.img_w * f.img_h * f.nout);

    // per-level tables, then the unpack / reconstruction launches
    std::vector<float> tab;
    std::vector<size_t> tab_at((size_t)f.nlevels, 0);
    for (int l = 0; l < f.nlevels; l++) {
        const NtcbLevelRec& L = f.lv[(size_t)l];
        tab_at[(size_t)l] = tab.size();
        if (L.mode == 0 || L.mode == 1) {
            for (int c = 0; c < L.C; c++) {
                const float lo = L.lo[(size_t)c], hi = L.hi[(size_t)c];
                const float r = hi - lo;
                tab.push_back(lo);
                tab.push_back(r < 1e-6f ? 1e-6f : r);   // range = max(hi - lo, 1e-6f)
            }
        } else if (L.mode == 2) {
            for (int c = 0; c < L.C; c++)
                for (int k = 0; k < 256; k++) tab.push_back(k < (int)L.palette[(size_t)c].size() ? L.palette[(size_t)c][(size_t)k] : 0.0f);
        }
    }
    d->tables = dev_alloc<float>(tab.size());
    if (!tab.empty()) NTCB_CHECK(cudaMemcpyAsync(d->tables, tab.data(), tab.size() * sizeof(float), cudaMemcpyHostToDevice, s));
    for (int l = 0; l < f.nlevels; l++) {
        const NtcbLevelRec& L = f.lv[(size_t)l];
        if (L.mode == 3) {
            DctTables T{};
            T.C = L.C; T.BW = L.W / 8; T.BH = L.H / 8; T.dc_step = L.dc_step; T.deadzone = L.deadzone; T.lo_w16 = 0; T.rate_on = 0;
            dct_basis(T.basis);
            dct_zigzag(T.zigzag);
            std::vector<int> st((size_t)L.C * 16 * 64);
            for (int c = 0; c < L.C; c++) dct_steps(L.q[(size_t)c], L.dc_step, st.data() + (size_t)c * 16 * 64);
            d->sym = dev_alloc<int16_t>(L.sym.size());
            d->code = dev_alloc<uint8_t>(L.code.size());
            d->steps = dev_alloc<int>(st.size());
            NTCB_CHECK(cudaMemcpyAsync(d->sym, L.sym.data(), L.sym.size() * sizeof(int16_t), cudaMemcpyHostToDevice, s));
            NTCB_CHECK(cudaMemcpyAsync(d->code, L.code.data(), L.code.size(), cudaMemcpyHostToDevice, s));
            NTCB_CHECK(cudaMemcpyAsync(d->steps, st.data(), st.size() * sizeof(int), cudaMemcpyHostToDevice, s));
            launch_dct_recon(s, m, T, d->sym, d->code, d->steps, d->z, nullptr);
            continue;
        }
        UnpackArgs a{};
        a.body = d->bytes + L.body;
        a.z = d->z + m.lv[l].off;
        a.ntex = (long long)L.W * L.H;
        a.C = L.C; a.mode = L.mode;
        for (int c = 0; c < L.C; c++) { a.chan_bit[c] = (long long)L.chan_bit[(size_t)c]; a.bits[c] = L.bits[(size_t)c]; }
        a.table = d->tables + tab_at[(size_t)l];
        k_ntcb_unpack<<<blocks_for(a.ntex * a.C, 256), 256, 0, s>>>(a);
        NTCB_CHECK(cudaGetLastError());
    }
    NTCB_CHECK(cudaStreamSynchronize(s));
    set_err("", err, err_cap);
    return d;
}

void ntcb_decoder_get_info(const ntcb_decoder* d, ntcb_container_desc* info) {
    if (d && info) ntcb::fill_info(d->f, d->nz, info);
}

void ntcb_decoder_model(ntcb_decoder* d, float* z, float* w) {
    if (!d) return;
    if (z) NTCB_CHECK(cudaMemcpyAsync(z, d->z, (size_t)d->nz * sizeof(float), cudaMemcpyDeviceToHost, d->stream));
    if (w) memcpy(w, d->f.weights.data(), d->f.weights.size() * sizeof(float));
    NTCB_CHECK(cudaStreamSynchronize(d->stream));
}

int ntcb_decoder_rgb8_device(ntcb_decoder* d, int crop_w, int crop_h, uint8_t* out_dev, void* stream) {
    if (!d || !out_dev) return -1;
    const ntcb::NtcbFile& f = d->f;
    const int cw = crop_w > 0 ? crop_w : f.src_w, ch = crop_h > 0 ? crop_h : f.src_h;
    if (cw > f.img_w || ch > f.img_h) return -1;
    cudaStream_t s = stream ? (cudaStream_t)stream : d->stream;
    ntcb::launch_decode(s, d->shape, d->dm, d->w, d->z, d->img);
    const long long n = (long long)cw * ch * f.T;
    ntcb::k_ntcb_rgb8<<<ntcb::blocks_for(n, 256), 256, 0, s>>>(d->img, f.img_w, f.nout, cw, ch, out_dev);
    NTCB_CHECK(cudaGetLastError());
    return 0;
}

size_t ntcb_decoder_rgb8(ntcb_decoder* d, int crop_w, int crop_h, uint8_t* out, size_t cap) {
    if (!d) return 0;
    const ntcb::NtcbFile& f = d->f;
    const int cw = crop_w > 0 ? crop_w : f.src_w, ch = crop_h > 0 ? crop_h : f.src_h;
    if (cw > f.img_w || ch > f.img_h) return 0;
    const size_t bytes = (size_t)cw * ch * 3 * f.T;
    if (!out) return bytes;
    if (bytes > d->rgb_cap) { dev_free(d->rgb); d->rgb = dev_alloc<uint8_t>(bytes); d->rgb_cap = bytes; }
    if (ntcb_decoder_rgb8_device(d, cw, ch, d->rgb, nullptr) != 0) return 0;
    NTCB_CHECK(cudaMemcpyAsync(out, d->rgb, std::min(cap, bytes), cudaMemcpyDeviceToHost, d->stream));
    NTCB_CHECK(cudaStreamSynchronize(d->stream));
    return bytes;
}

void ntcb_decoder_close(ntcb_decoder* d) {
    if (!d) return;
    if (d->stream) cudaStreamSynchronize(d->stream);
    release(d);
    delete d;
}

}  // extern "C"
