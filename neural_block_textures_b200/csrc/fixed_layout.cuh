// Compile-time level layouts for the fixed MLP shapes.
//
// The runtime feature gather (pixel_features, perturbed_features_pm) walks the model's levels with runtime channel
// counts, so its output array is indexed at runtime and lives in local memory. For the layouts the benchmark shapes
// use — level 0 with C0 channels, an optional level 1 with C1 channels, one uv position pair — the same features are
// gathered here with every index known at compile time, so they stay in registers. A kernel instantiated with a
// layout runs only for a model that matches it exactly (Layout::matches, checked by the launcher); any other model
// inside the envelope takes the runtime path. Geometry (W, H, offsets, nearest or bilinear) stays runtime. The
// arithmetic is the runtime path's, operation by operation (taps, the bilinear blend order, the perturbation fma,
// 2u - 1), so both paths produce the same bits.
#pragma once
#include "device_model.cuh"

namespace ntcb {

template <int NLEV_, int C0_, int C1_>
struct Layout {
    static constexpr int NLEV = NLEV_, C0 = C0_, C1 = C1_, NIN = C0 + C1 + 2;
    static_assert(NLEV == 1 || NLEV == 2, "one or two levels");
    static_assert(NLEV == 2 || C1 == 0, "one level has no C1");
    // Exact match of the model's level channels and positional inputs; level offsets aligned to the vector loads.
    static bool matches(const DevModel& m) {
        if (m.nlev != NLEV || m.nin != NIN || m.npos != 1 || m.pos_kind[0] != 0 || m.lv[0].C != C0) return false;
        if (NLEV == 2 && m.lv[1].C != C1) return false;
        long long nz = 0;
        for (int l = 0; l < m.nlev; l++) nz += (long long)m.lv[l].W * m.lv[l].H * m.lv[l].C;
        for (int l = 0; l < NLEV; l++) {
            const int C = l == 0 ? C0 : C1;
            // vector loads of the latent and of the latent noise rows (pair k starts at k * nz floats)
            if ((C == 2 || C == 4) && (m.lv[l].off % C != 0 || nz % C != 0)) return false;
        }
        return true;
    }
};

// The layout a fixed shape is compiled for (the benchmark configurations): 5 inputs = 1-channel level 0 + 2-channel
// level 1 (configs 2 and 4), 6 = one 4-channel level (config 1), 8 = 2-channel level 0 + 4-channel level 1 (configs 3, 5).
template <int NIN> struct LayoutForNin { using type = void; };
template <> struct LayoutForNin<5> { using type = Layout<2, 1, 2>; };
template <> struct LayoutForNin<6> { using type = Layout<1, 4, 0>; };
template <> struct LayoutForNin<8> { using type = Layout<2, 2, 4>; };

// C consecutive floats of one texel (vector loads for 2 and 4 channels: the texel starts at a multiple of C floats).
// Plain loads, not the read-only path: the selector search rewrites level 0 while it reads it.
template <int C>
__device__ __forceinline__ void load_texel(const float* p, float (&v)[C]) {
    if constexpr (C == 4) {
        const float4 q = *reinterpret_cast<const float4*>(p);
        v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
    } else if constexpr (C == 2) {
        const float2 q = *reinterpret_cast<const float2*>(p);
        v[0] = q.x; v[1] = q.y;
    } else {
#pragma unroll
        for (int c = 0; c < C; c++) v[c] = p[c];
    }
}

// sample_level with a compile-time channel count; out[0 .. C).
template <int C>
__device__ __forceinline__ void sample_level_c(const DevLevel& L, const float* zl, const Tap& t, float* out) {
    float a[C];
    load_texel<C>(zl + ((long long)t.y0 * L.W + t.x0) * C, a);
    if (L.nearest) {
#pragma unroll
        for (int k = 0; k < C; k++) out[k] = a[k];
        return;
    }
    float b[C], c[C], d[C];
    load_texel<C>(zl + ((long long)t.y0 * L.W + t.x1) * C, b);
    load_texel<C>(zl + ((long long)t.y1 * L.W + t.x0) * C, c);
    load_texel<C>(zl + ((long long)t.y1 * L.W + t.x1) * C, d);
    const TapW w = tap_weights(t);
#pragma unroll
    for (int k = 0; k < C; k++) out[k] = blend4(w, a[k], b[k], c[k], d[k]);
}

// pixel_features for layout LY: [level 0 | level 1 | 2u - 1, 2v - 1].
template <class LY>
__device__ __forceinline__ void layout_features(const DevModel& m, const float* z, int px, int py, float (&f)[LY::NIN]) {
    const float u = pix_u(m, px), v = pix_v(m, py);
    sample_level_c<LY::C0>(m.lv[0], z + m.lv[0].off, level_tap(m.lv[0], u, v), f);
    if constexpr (LY::NLEV == 2) sample_level_c<LY::C1>(m.lv[1], z + m.lv[1].off, level_tap(m.lv[1], u, v), f + LY::C0);
    f[LY::C0 + LY::C1] = u * 2.0f - 1.0f;
    f[LY::C0 + LY::C1 + 1] = v * 2.0f - 1.0f;
}

// One level of perturbed_features_pm with a compile-time channel count: + and - features of the level's taps, the
// level perturbed by +-sg eps when it is active, sampled plain otherwise.
template <int C>
__device__ __forceinline__ void perturbed_level_pm(const DevLevel& L, const float* __restrict__ zl, const float* __restrict__ el,
                                                   bool active, float sg, const Tap& t, float* fp, float* fm) {
    if (!active) {
        sample_level_c<C>(L, zl, t, fp);
#pragma unroll
        for (int c = 0; c < C; c++) fm[c] = fp[c];
        return;
    }
    const long long ia = ((long long)t.y0 * L.W + t.x0) * C;
    float za[C], ea[C];
    load_texel<C>(zl + ia, za);
    load_texel<C>(el + ia, ea);
    if (L.nearest) {
#pragma unroll
        for (int c = 0; c < C; c++) { fp[c] = fmaf(sg, ea[c], za[c]); fm[c] = fmaf(-sg, ea[c], za[c]); }
        return;
    }
    const long long ib = ((long long)t.y0 * L.W + t.x1) * C;
    const long long ic = ((long long)t.y1 * L.W + t.x0) * C;
    const long long id = ((long long)t.y1 * L.W + t.x1) * C;
    float zb[C], zc[C], zd[C], eb[C], ec[C], ed[C];
    load_texel<C>(zl + ib, zb); load_texel<C>(el + ib, eb);
    load_texel<C>(zl + ic, zc); load_texel<C>(el + ic, ec);
    load_texel<C>(zl + id, zd); load_texel<C>(el + id, ed);
    const TapW w = tap_weights(t);
#pragma unroll
    for (int c = 0; c < C; c++) {
        fp[c] = blend4(w, fmaf(sg, ea[c], za[c]), fmaf(sg, eb[c], zb[c]), fmaf(sg, ec[c], zc[c]), fmaf(sg, ed[c], zd[c]));
        fm[c] = blend4(w, fmaf(-sg, ea[c], za[c]), fmaf(-sg, eb[c], zb[c]), fmaf(-sg, ec[c], zc[c]), fmaf(-sg, ed[c], zd[c]));
    }
}

// perturbed_features_pm for layout LY (ek = pair k's noise over the flat latent).
template <class LY>
__device__ __forceinline__ void layout_features_pm(const DevModel& m, const float* __restrict__ z, const float* __restrict__ ek,
                                                   unsigned active, float sg, int px, int py, float (&fp)[LY::NIN],
                                                   float (&fm)[LY::NIN]) {
    const float u = pix_u(m, px), v = pix_v(m, py);
    perturbed_level_pm<LY::C0>(m.lv[0], z + m.lv[0].off, ek + m.lv[0].off, (active & 1u) != 0, sg, level_tap(m.lv[0], u, v), fp, fm);
    if constexpr (LY::NLEV == 2)
        perturbed_level_pm<LY::C1>(m.lv[1], z + m.lv[1].off, ek + m.lv[1].off, (active & 2u) != 0, sg, level_tap(m.lv[1], u, v),
                                   fp + LY::C0, fm + LY::C0);
    constexpr int q = LY::C0 + LY::C1;
    fp[q] = fm[q] = u * 2.0f - 1.0f;
    fp[q + 1] = fm[q + 1] = v * 2.0f - 1.0f;
}

}  // namespace ntcb
