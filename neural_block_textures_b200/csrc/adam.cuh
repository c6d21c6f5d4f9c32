// The Adam update shared by the weight and latent kernels.
#pragma once

namespace ntcb {

// Adam::step (main.cpp:1797-1809): theta -= lr * (m / c1) / (sqrt(v / c2) + eps), c1 / c2 computed on the host.
__device__ __forceinline__ void adam_update(float& theta, float g, float& m, float& v, float lr, float c1, float c2) {
    const float b1 = 0.9f, b2 = 0.999f, eps = 1e-8f;
    m = b1 * m + (1.0f - b1) * g;
    v = b2 * v + (1.0f - b2) * g * g;
    const float mh = m / c1, vh = v / c2;
    theta -= lr * mh / (sqrtf(vh) + eps);
}

}  // namespace ntcb
