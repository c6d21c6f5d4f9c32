// Counter-based noise, usable on host and device.
//
// The reference keys every perturbation and minibatch draw on (seed, stream, step, pair, index)
// through the splitmix64 output function (Steele, Lea and Flood, "Fast splittable pseudorandom
// number generators", OOPSLA 2014) applied twice, and turns a 64-bit draw into a standard normal
// with the cosine branch of Box-Muller (cuda/ntc_noise.h:20-47). The streams, the key layout, the
// 24-bit uniform split and the expression sqrtf(-2 logf(u1)) * cosf(2 pi u2) must stay exactly the
// same for the draws to be bit-identical with the reference's device noise; they are restated here.
// CUDA's own logf / cosf / sqrtf are called (the library is built without fast-math), which is what
// makes the device values equal to the reference backend's bit for bit; against a CPU C library
// they agree to an ulp or two, the same statement the reference makes.
#pragma once
#include <stdint.h>
#include <math.h>

#ifdef __CUDACC__
#define NTCB_HD __host__ __device__ __forceinline__
#else
#define NTCB_HD static inline
#endif

namespace ntcb {

enum NoiseStream : uint32_t { kStreamLatent = 1, kStreamMlp = 2, kStreamBatchPix = 3, kStreamBatchTex = 4 };

constexpr uint64_t kGolden64 = 0x9E3779B97F4A7C15ull;

// splitmix64 output function.
NTCB_HD uint64_t mix64(uint64_t x) {
    x += kGolden64;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

// The per-(seed, stream, step, pair) key; the draw for `index` is mix64(key + index * golden).
NTCB_HD uint64_t stream_key(uint64_t seed, uint32_t stream, uint32_t step, uint32_t pair) {
    return mix64(seed ^ ((uint64_t)stream << 56) ^ ((uint64_t)step << 32) ^ (uint64_t)pair);
}
NTCB_HD uint64_t draw64(uint64_t key, uint64_t index) { return mix64(key + index * kGolden64); }

// High 32 bits of a draw; and the multiply-high map of a 32-bit draw onto [0, n).
NTCB_HD uint32_t draw_u32(uint64_t key, uint64_t index) { return (uint32_t)(draw64(key, index) >> 32); }
NTCB_HD uint32_t uniform_below(uint32_t u, uint32_t n) { return (uint32_t)(((uint64_t)u * (uint64_t)n) >> 32); }

// Standard normal from a 64-bit draw: u1 = (top 24 bits + 1) / 2^24 in (0, 1], u2 = low 24 bits / 2^24.
NTCB_HD float gauss_of(uint64_t h) {
    const float u1 = (float)((h >> 40) + 1ull) * (1.0f / 16777216.0f);
    const float u2 = (float)(h & 0xFFFFFFull) * (1.0f / 16777216.0f);
    return sqrtf(-2.0f * logf(u1)) * cosf(6.283185307179586f * u2);
}
NTCB_HD float gauss_at(uint64_t key, uint64_t index) { return gauss_of(draw64(key, index)); }

}  // namespace ntcb
