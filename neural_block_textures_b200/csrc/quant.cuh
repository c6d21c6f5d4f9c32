// Grid-index and grid-value functions of the reference's latent quantizers, on the device.
//
// q8_index / q8_value / qes_index sit in the reference's strict floating-point region (STRICT_FP_BEGIN,
// main.cpp:446-482): every operation below is an explicit round-to-nearest intrinsic so that nvcc cannot
// contract or reorder it. qat_index is outside that region; its expression has no product-plus-sum to fuse.
#pragma once

namespace ntcb {

// qat_index (main.cpp:2060-2064): the grid index of a --qat value, lround((v + 1) / 2 * levels), clamped.
__device__ __forceinline__ int qat_index(float v, int bits) {
    const int levels = (1 << bits) - 1;
    const int k = (int)lroundf((v + 1.0f) * 0.5f * (float)levels);
    return max(0, min(levels, k));
}

// qes_index (main.cpp:448-453): round-half-even of ((v - lo) / range) * levels, clamped in float.
__device__ __forceinline__ int qes_index_dev(float v, float lo, float range, int levels) {
    const float r = rintf(__fmul_rn(__fdiv_rn(__fsub_rn(v, lo), range), (float)levels));
    return r <= 0.0f ? 0 : (r >= (float)levels ? levels : (int)r);
}

// q8_index (main.cpp:478-481): the post-hoc index lround((z - lo) / range * levels), clamped.
__device__ __forceinline__ int q8_index_dev(float z, float lo, float range, int levels) {
    const int qi = (int)lroundf(__fmul_rn(__fdiv_rn(__fsub_rn(z, lo), range), (float)levels));
    return max(0, min(levels, qi));
}
// q8_value (main.cpp:482): lo + k / levels * range, the value both container readers reconstruct.
__device__ __forceinline__ float q8_value_dev(int k, float lo, float range, int levels) {
    return __fadd_rn(lo, __fmul_rn(__fdiv_rn((float)k, (float)levels), range));
}

}  // namespace ntcb
