// Device helpers shared by the population kernels (packed-FP32 and tensor-core variants).
#pragma once
#include "kernels.h"

namespace ntcb {

// Fixed-order CTA sum of doubles: warp shuffle tree, then the warp totals in index order (thread 0).
template <int TPB>
__device__ __forceinline__ double cta_sum(double v, double* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    double r = 0.0;
    if (threadIdx.x == 0)
        for (int i = 0; i < TPB / 32; i++) r += red[i];
    return r;   // valid in thread 0
}

// The perturbed weight of slot k for sign +/- : ES w0 +- sigma eps with each perturbed weight rounded once,
// fma(+-sigma, eps, w0) (MlpTrainer::step, main.cpp:1856); FD: w0 except weight j at the float-realised
// w0[j] + h / w0[j] - h (main.cpp:1906-1910).
// Candidate index of launch slot i (perturbed_weight's `cand`: an ES pair, an FD weight, or -1 = unperturbed).
__device__ __forceinline__ int pop_cand(const PopArgs& a, int i) {
    return a.stats_first ? (i == 0 ? -1 : a.cand_begin + i - 1) : a.cand_begin + i;
}

// Weight k of the pair's two sets from its base value w0 and, for an ES pair, its noise *ek (nullptr otherwise).
__device__ __forceinline__ void perturbed_weight_of(const PopArgs& a, float w0, const float* ek, int k, int cand, float& wp, float& wm) {
    wp = w0; wm = w0;
    if (ek) { wp = fmaf(a.sigma, *ek, w0); wm = fmaf(-a.sigma, *ek, w0); }
    else if (a.mode == 1 && k == cand) { wp = w0 + a.fd_h; wm = w0 - a.fd_h; }
}
__device__ __forceinline__ void perturbed_weight(const PopArgs& a, const float* e, int k, int cand, float& wp, float& wm) {
    perturbed_weight_of(a, a.w0[k], e ? e + k : nullptr, k, cand, wp, wm);
}

}  // namespace ntcb
