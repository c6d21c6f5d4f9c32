// Device-side model description and the per-pixel decode geometry of the ES training backend.
//
// The model travels to every kernel as a by-value kernel parameter (DevModel, a few hundred bytes
// in the constant bank), not as __constant__ globals: one process can hold several trainers
// (tests, one per GPU) without them overwriting each other's descriptors.
//
// Geometry and features restate the reference's CPU decoder (main.cpp) operation by operation so
// that the decoded values agree with it to float rounding; each function cites what it follows.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

namespace ntcb {

constexpr int kMaxLevels = 3;
constexpr int kMaxPos = 16;
constexpr int kMaxOut = 12;
constexpr int kMaxHidden = 8;
constexpr int kMaxCh = 16;
constexpr int kMaxIn = 64;      // widest MLP input / hidden layer the backend accepts (as the reference's v1 envelope)
constexpr int kMaxWidth = 64;

// A failing CUDA call prints and exits the process, as the reference backend does (cuda/ntc_cuda.cu:55-56), unless the
// calling host thread has installed a soft-error slot (SoftErrorScope): then the first failure is recorded there and
// the call returns, so an entry point that reports errors to its caller can check the slot and return.
extern thread_local cudaError_t* g_soft_error;
struct SoftErrorScope {
    cudaError_t err = cudaSuccess;
    cudaError_t* prev;
    SoftErrorScope() : prev(g_soft_error) { g_soft_error = &err; }
    ~SoftErrorScope() { g_soft_error = prev; }
    SoftErrorScope(const SoftErrorScope&) = delete;
    SoftErrorScope& operator=(const SoftErrorScope&) = delete;
};
#define NTCB_CHECK(x) do { cudaError_t e_ = (x); if (e_ != cudaSuccess) { \
    if (::ntcb::g_soft_error) { if (*::ntcb::g_soft_error == cudaSuccess) *::ntcb::g_soft_error = e_; } else { \
    fprintf(stderr, "ntc_b200: CUDA error %s at %s:%d: %s\n", #x, __FILE__, __LINE__, cudaGetErrorString(e_)); exit(1); } } } while (0)

struct DevLevel {
    int W, H, C, nearest;
    long long off;               // float offset of the level in the flat latent
};

struct DevModel {
    int W, H;                    // image size
    int nlev;
    DevLevel lv[kMaxLevels];
    int npos;
    int pos_kind[kMaxPos];       // 0 = uv, 1 = lv1local (main.cpp PosKind order)
    int nin, nout, nhidden;
    int hidden[kMaxHidden];
    float leak;
    int clamp_out;
    float cw[kMaxOut];
    float wsum;
    int P;                       // MLP weight count
};

// One bilinear / nearest tap: clamped texel indices and the cell offsets (main.cpp:507-531 BilinearTap).
struct Tap { int x0, x1, y0, y1; float fx, fy; };

// bilinear_tap (main.cpp:512-531): nearest levels read the texel whose cell holds (u, v) and report the
// offset inside the cell; bilinear levels blend the four texels around (u W - 0.5, v H - 0.5), clamped.
__device__ __forceinline__ Tap level_tap(const DevLevel& L, float u, float v) {
    Tap t;
    if (L.nearest) {
        const float x = u * (float)L.W, y = v * (float)L.H;
        const int ix = (int)floorf(x), iy = (int)floorf(y);
        t.fx = x - (float)ix; t.fy = y - (float)iy;
        t.x0 = t.x1 = max(0, min(L.W - 1, ix));
        t.y0 = t.y1 = max(0, min(L.H - 1, iy));
        return t;
    }
    // u W - 0.5 as one fused multiply-add: the form the reference's compilers emit for this expression
    // (nvcc's default contraction; g++ -ffast-math with FMA). It is written explicitly so that the texel
    // footprints the host precomputes (engine.cu axis_ranges) use the same rounding.
    const float x = fmaf(u, (float)L.W, -0.5f), y = fmaf(v, (float)L.H, -0.5f);
    const int x0 = (int)floorf(x), y0 = (int)floorf(y);
    t.fx = x - (float)x0; t.fy = y - (float)y0;
    t.x0 = max(0, min(L.W - 1, x0)); t.x1 = max(0, min(L.W - 1, x0 + 1));
    t.y0 = max(0, min(L.H - 1, y0)); t.y1 = max(0, min(L.H - 1, y0 + 1));
    return t;
}

// The four bilinear weights in the reference's expression order (main.cpp:543-544).
struct TapW { float w00, w10, w01, w11; };
__device__ __forceinline__ TapW tap_weights(const Tap& t) {
    TapW w;
    w.w00 = (1.0f - t.fx) * (1.0f - t.fy); w.w10 = t.fx * (1.0f - t.fy);
    w.w01 = (1.0f - t.fx) * t.fy;          w.w11 = t.fx * t.fy;
    return w;
}
// w00 a + w10 b + w01 c + w11 d, left to right (main.cpp:545-546), each add fused with the product
// that follows it (the contracted form of the expression).
__device__ __forceinline__ float blend4(const TapW& w, float a, float b, float c, float d) {
    return fmaf(w.w11, d, fmaf(w.w01, c, fmaf(w.w10, b, w.w00 * a)));
}

// sample_latent (main.cpp:533-547) for one level; zl points at the level's first float.
__device__ __forceinline__ void sample_level(const DevLevel& L, const float* __restrict__ zl, const Tap& t, float* out) {
    if (L.nearest) {
        const float* a = zl + ((long long)t.y0 * L.W + t.x0) * L.C;
        for (int k = 0; k < L.C; k++) out[k] = a[k];
        return;
    }
    const float* a = zl + ((long long)t.y0 * L.W + t.x0) * L.C;
    const float* b = zl + ((long long)t.y0 * L.W + t.x1) * L.C;
    const float* c = zl + ((long long)t.y1 * L.W + t.x0) * L.C;
    const float* d = zl + ((long long)t.y1 * L.W + t.x1) * L.C;
    const TapW w = tap_weights(t);
    for (int k = 0; k < L.C; k++) out[k] = blend4(w, a[k], b[k], c[k], d[k]);
}

// Pixel centre in [0,1]^2 (main.cpp:1688).
__device__ __forceinline__ float pix_u(const DevModel& m, int px) { return ((float)px + 0.5f) / (float)m.W; }
__device__ __forceinline__ float pix_v(const DevModel& m, int py) { return ((float)py + 0.5f) / (float)m.H; }

// PosEnc::encode (main.cpp:1593-1608): uv -> (2u-1, 2v-1); lv1local -> level 1's cell offset mapped to [-1,1].
__device__ __forceinline__ int pos_encode(const DevModel& m, float u, float v, const Tap& t1, float* f) {
    int k = 0;
    for (int q = 0; q < m.npos; q++) {
        if (m.pos_kind[q] == 0) { f[k++] = u * 2.0f - 1.0f; f[k++] = v * 2.0f - 1.0f; }
        else { f[k++] = t1.fx * 2.0f - 1.0f; f[k++] = t1.fy * 2.0f - 1.0f; }
    }
    return k;
}

// Decoder::features (main.cpp:1687-1702): level 0's sample, the other levels' samples, the positional
// inputs. z is the flat latent (level offsets from the model).
__device__ __forceinline__ void pixel_features(const DevModel& m, const float* __restrict__ z, int px, int py, float* f) {
    const float u = pix_u(m, px), v = pix_v(m, py);
    Tap t1 = {0, 0, 0, 0, 0.0f, 0.0f};
    int k = 0;
    for (int l = 0; l < m.nlev; l++) {
        const DevLevel& L = m.lv[l];
        const Tap t = level_tap(L, u, v);
        if (l == 1) t1 = t;
        sample_level(L, z + L.off, t, f + k);
        k += L.C;
    }
    pos_encode(m, u, v, t1, f + k);
}

// The leaky ReLU (activate, main.cpp:560).
__device__ __forceinline__ float leaky(float x, float leak) { return x > 0.0f ? x : leak * x; }
// The output unit (main.cpp:624-625): clamp(s + 0.5) with --clamp, else the logistic sigmoid
// 1 / (1 + expf(-s)). The IEEE quotient 1 / x is the correctly rounded reciprocal, which __frcp_rn
// computes without the general division path: the same value.
__device__ __forceinline__ float out_act(float s, int clamp_out) {
    return clamp_out ? fminf(1.0f, fmaxf(0.0f, s + 0.5f)) : __frcp_rn(1.0f + expf(-s));
}

}  // namespace ntcb
