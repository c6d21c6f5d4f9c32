// Perturbed decoder features for the latent ES pass (shared by the packed-FP32 and tensor-core kernels).
#pragma once
#include "device_model.cuh"

namespace ntcb {

// Features of one pixel with the active levels perturbed by sign * sg * eps (pair k). The reference
// perturbs the latent texel by texel, zp = zb + sg eps (fma), and samples the perturbed latent
// (LatentTrainer::step, main.cpp:1997-2007); the same is done here per tap.
__device__ __forceinline__ void perturbed_features(const DevModel& m, const float* __restrict__ z, const float* __restrict__ ek,
                                                   unsigned active, float sgn_sg, int px, int py, float* f) {
    const float u = pix_u(m, px), v = pix_v(m, py);
    Tap t1 = {0, 0, 0, 0, 0.0f, 0.0f};
    int slot = 0;
    for (int l = 0; l < m.nlev; l++) {
        const DevLevel& L = m.lv[l];
        const Tap t = level_tap(L, u, v);
        if (l == 1) t1 = t;
        const float* zl = z + L.off;
        if (!(active & (1u << l))) {
            sample_level(L, zl, t, f + slot);
        } else {
            const float* el = ek + L.off;
            const long long ia = ((long long)t.y0 * L.W + t.x0) * L.C;
            if (L.nearest) {
                for (int c = 0; c < L.C; c++) f[slot + c] = fmaf(sgn_sg, el[ia + c], zl[ia + c]);
            } else {
                const long long ib = ((long long)t.y0 * L.W + t.x1) * L.C;
                const long long ic = ((long long)t.y1 * L.W + t.x0) * L.C;
                const long long id = ((long long)t.y1 * L.W + t.x1) * L.C;
                const TapW w = tap_weights(t);
                for (int c = 0; c < L.C; c++)
                    f[slot + c] = blend4(w, fmaf(sgn_sg, el[ia + c], zl[ia + c]), fmaf(sgn_sg, el[ib + c], zl[ib + c]),
                                         fmaf(sgn_sg, el[ic + c], zl[ic + c]), fmaf(sgn_sg, el[id + c], zl[id + c]));
            }
        }
        slot += L.C;
    }
    pos_encode(m, u, v, t1, f + slot);
}

// The + and - features of one pixel for pair k in one pass (taps, latent and noise loads shared).
__device__ __forceinline__ void perturbed_features_pm(const DevModel& m, const float* __restrict__ z, const float* __restrict__ ek,
                                                      unsigned active, float sg, int px, int py, float* fp, float* fm) {
    const float u = pix_u(m, px), v = pix_v(m, py);
    Tap t1 = {0, 0, 0, 0, 0.0f, 0.0f};
    int slot = 0;
    for (int l = 0; l < m.nlev; l++) {
        const DevLevel& L = m.lv[l];
        const Tap t = level_tap(L, u, v);
        if (l == 1) t1 = t;
        const float* zl = z + L.off;
        if (!(active & (1u << l))) {
            sample_level(L, zl, t, fp + slot);
            for (int c = 0; c < L.C; c++) fm[slot + c] = fp[slot + c];
        } else {
            const float* el = ek + L.off;
            const long long ia = ((long long)t.y0 * L.W + t.x0) * L.C;
            if (L.nearest) {
                for (int c = 0; c < L.C; c++) {
                    const float e = el[ia + c], zz = zl[ia + c];
                    fp[slot + c] = fmaf(sg, e, zz); fm[slot + c] = fmaf(-sg, e, zz);
                }
            } else {
                const long long ib = ((long long)t.y0 * L.W + t.x1) * L.C;
                const long long ic = ((long long)t.y1 * L.W + t.x0) * L.C;
                const long long id = ((long long)t.y1 * L.W + t.x1) * L.C;
                const TapW w = tap_weights(t);
                for (int c = 0; c < L.C; c++) {
                    const float ea = el[ia + c], eb = el[ib + c], ec = el[ic + c], ed = el[id + c];
                    const float za = zl[ia + c], zb = zl[ib + c], zc = zl[ic + c], zd = zl[id + c];
                    fp[slot + c] = blend4(w, fmaf(sg, ea, za), fmaf(sg, eb, zb), fmaf(sg, ec, zc), fmaf(sg, ed, zd));
                    fm[slot + c] = blend4(w, fmaf(-sg, ea, za), fmaf(-sg, eb, zb), fmaf(-sg, ec, zc), fmaf(-sg, ed, zd));
                }
            }
        }
        slot += L.C;
    }
    pos_encode(m, u, v, t1, fp + slot);
    for (int q = slot; q < m.nin; q++) fm[q] = fp[q];
}

}  // namespace ntcb
