// Register-tiled MLP forward on the packed FP32 pipe, for the population kernels.
//
// The reference evaluates one pixel per thread and reads every weight from shared memory once per
// FFMA (cuda/ntc_cuda.cu:164-194, loops predicated to a 32/64 maximum width). Here a thread owns R2 row
// pairs (two pixels, or two candidates of one pixel, per pair) whose activations live in registers as
// float2 (.x = first row, .y = second row). sm_100's FFMA2 (__ffma2_rn) performs two independent
// round-to-nearest FMAs per instruction, so every value is bit-identical to a scalar FMA chain while the
// FMA issue count halves. Weight sets are stored in shared memory with every weight duplicated, {w, w},
// so one broadcast LDS.128 delivers two weight pairs with no register moves. The hidden layer 2 ->
// output layer product is streamed: hidden unit j is computed, activated and immediately folded into
// the output accumulators, so only the layer-1 activations and the outputs are register-resident.
//
// Evaluation order per unit is the reference's (mlp_forward, main.cpp:603-627): s = bias, then
// s += w[i] * a[i] for i ascending (one FMA each), so every unit's value is the same FMA chain the
// reference CUDA backend computes. The output layer's chain over hidden units j also starts from its
// bias and runs j ascending, exactly as a separate pass would.
//
// Shared-memory layout of one weight set for a FixedShape, in floats before the duplication (each slot
// then occupies two floats, so every offset doubles):
//   W0T [NIN][H1]   layer-1 weights transposed (column i of W0 contiguous)
//   b0  [H1]
//   W1  [H2][H1]    layer-2 weights, row j contiguous
//   b1  [H2]
//   W2T [H2][NOUTP] output weights transposed, NOUT padded to a multiple of 4
//   b2  [NOUTP]
// slot(k) maps the reference's flat parameter index k (per layer W[out][in] row-major, then b[out])
// to this layout.
#pragma once
#include "device_model.cuh"

namespace ntcb {

template <int NIN_, int H1_, int H2_, int NOUT_>
struct FixedShape {
    static constexpr bool kFixed = true;
    static constexpr int NIN = NIN_, H1 = H1_, H2 = H2_, NOUT = NOUT_;
    static constexpr int NOUTP = (NOUT + 3) / 4 * 4;
    static constexpr int oW0T = 0;
    static constexpr int oB0 = oW0T + NIN * H1;
    static constexpr int oW1 = oB0 + H1;
    static constexpr int oB1 = oW1 + H2 * H1;
    static constexpr int oW2T = (oB1 + H2 + 3) / 4 * 4;
    static constexpr int oB2 = oW2T + H2 * NOUTP;
    static constexpr int SIZE = (oB2 + NOUTP + 3) / 4 * 4;   // slots per set (2 * SIZE floats in shared memory)
    static constexpr int P = H1 * NIN + H1 + H2 * H1 + H2 + NOUT * H2 + NOUT;
    // Register bound of the population kernel: 4 resident CTAs of 128 threads (128 registers) when the
    // tile fits without spilling, 2 otherwise (the 12-output material shape).
    static constexpr int kPopMinBlocks = NOUT <= 3 ? 4 : 2;
    static_assert(H1 % 4 == 0 && H2 % 4 == 0, "hidden widths of a fixed shape are multiples of 4");

    __host__ __device__ static int slot(int k) {
        if (k < H1 * NIN) { const int j = k / NIN, i = k - j * NIN; return oW0T + i * H1 + j; }
        k -= H1 * NIN;
        if (k < H1) return oB0 + k;
        k -= H1;
        if (k < H2 * H1) return oW1 + k;
        k -= H2 * H1;
        if (k < H2) return oB1 + k;
        k -= H2;
        if (k < NOUT * H2) { const int o = k / H2, j = k - o * H2; return oW2T + j * NOUTP + o; }
        k -= NOUT * H2;
        return oB2 + k;
    }
    // The compiled kernels form the leaky ReLU as max(x, leak x), which equals the reference's select
    // (x > 0 ? x : leak x) for 0 <= leak <= 1 only; other slopes run the runtime-shaped kernels.
    static bool matches(const DevModel& m) {
        return m.nin == NIN && m.nhidden == 2 && m.hidden[0] == H1 && m.hidden[1] == H2 && m.nout == NOUT &&
               m.leak >= 0.0f && m.leak <= 1.0f;
    }
};

// Runtime-shaped fallback: the reference's flat layout, one row per thread, exact loop bounds.
struct GenericShape {
    static constexpr bool kFixed = false;
};

__device__ __forceinline__ float4 lds4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }

__device__ __forceinline__ float2 leaky2(float2 s, float leak) {
    // For 0 <= leak <= 1 (the only slopes FixedShape::matches admits), max(x, leak x) equals
    // (x > 0 ? x : leak x) for every float, signed zeros and NaN included.
    const float2 t = __fmul2_rn(s, f2(leak));
    return make_float2(fmaxf(s.x, t.x), fmaxf(s.y, t.y));
}

// Stage the flat weights wg (reference layout) into shared memory as one duplicated FixedShape set.
template <class S>
__device__ __forceinline__ void load_weights_x2(const float* __restrict__ wg, int P, float* ws) {
    for (int k = threadIdx.x; k < 2 * S::SIZE; k += blockDim.x) ws[k] = 0.0f;
    __syncthreads();
    for (int k = threadIdx.x; k < P; k += blockDim.x) {
        const float v = wg[k];
        *reinterpret_cast<float2*>(ws + 2 * S::slot(k)) = make_float2(v, v);
    }
    __syncthreads();
}

// Forward of R2 row pairs through one duplicated weight set `w` (shared memory). x: inputs, o: outputs.
template <class S, int R2>
__device__ __forceinline__ void fixed_forward_x2(const float* __restrict__ w, const float2 (&x)[R2][S::NIN],
                                                 float2 (&o)[R2][S::NOUT], float leak, int clamp_out) {
    float2 a[R2][S::H1];
#pragma unroll
    for (int j = 0; j < S::H1; j += 2) {
        const float4 b = lds4(w + 2 * (S::oB0 + j));
#pragma unroll
        for (int q = 0; q < R2; q++) { a[q][j] = make_float2(b.x, b.y); a[q][j + 1] = make_float2(b.z, b.w); }
    }
#pragma unroll
    for (int i = 0; i < S::NIN; i++) {
#pragma unroll
        for (int j = 0; j < S::H1; j += 2) {
            const float4 c = lds4(w + 2 * (S::oW0T + i * S::H1 + j));
            const float2 c0 = make_float2(c.x, c.y), c1 = make_float2(c.z, c.w);
#pragma unroll
            for (int q = 0; q < R2; q++) {
                a[q][j] = __ffma2_rn(c0, x[q][i], a[q][j]);
                a[q][j + 1] = __ffma2_rn(c1, x[q][i], a[q][j + 1]);
            }
        }
    }
#pragma unroll
    for (int q = 0; q < R2; q++)
#pragma unroll
        for (int j = 0; j < S::H1; j++) a[q][j] = leaky2(a[q][j], leak);

#pragma unroll
    for (int q = 0; q < R2; q++)
#pragma unroll
        for (int k = 0; k < S::NOUT; k++) o[q][k] = f2(w[2 * (S::oB2 + k)]);

#pragma unroll 2
    for (int j = 0; j < S::H2; j++) {
        float2 s[R2];
        const float bj = w[2 * (S::oB1 + j)];
#pragma unroll
        for (int q = 0; q < R2; q++) s[q] = f2(bj);
        const float* wr = w + 2 * (S::oW1 + j * S::H1);
#pragma unroll
        for (int i = 0; i < S::H1; i += 2) {
            const float4 c = lds4(wr + 2 * i);
            const float2 c0 = make_float2(c.x, c.y), c1 = make_float2(c.z, c.w);
#pragma unroll
            for (int q = 0; q < R2; q++) {
                s[q] = __ffma2_rn(c0, a[q][i], s[q]);
                s[q] = __ffma2_rn(c1, a[q][i + 1], s[q]);
            }
        }
        float2 wo[S::NOUTP];
#pragma unroll
        for (int k = 0; k < S::NOUTP; k += 2) {
            const float4 c = lds4(w + 2 * (S::oW2T + j * S::NOUTP + k));
            wo[k] = make_float2(c.x, c.y); wo[k + 1] = make_float2(c.z, c.w);
        }
#pragma unroll
        for (int q = 0; q < R2; q++) {
            const float2 h = leaky2(s[q], leak);
#pragma unroll
            for (int k = 0; k < S::NOUT; k++) o[q][k] = __ffma2_rn(wo[k], h, o[q][k]);
        }
    }
#pragma unroll
    for (int q = 0; q < R2; q++)
#pragma unroll
        for (int k = 0; k < S::NOUT; k++) o[q][k] = make_float2(out_act(o[q][k].x, clamp_out), out_act(o[q][k].y, clamp_out));
}

// Forward of one row through the reference's flat layout with the model's runtime widths
// (mlp_forward, main.cpp:603-627). `in` holds nin floats; out receives nout floats.
__device__ __forceinline__ void generic_forward(const DevModel& m, const float* __restrict__ w, const float* in, float* out) {
    float bufA[kMaxWidth], bufB[kMaxWidth];
    const float* cur = in;
    float* nxt = bufA;
    int ncur = m.nin;
    const float* p = w;
    for (int l = 0; l < m.nhidden; l++) {
        const int nh = m.hidden[l];
        const float* b = p + nh * ncur;
        for (int j = 0; j < nh; j++) {
            float s = b[j];
            const float* wr = p + j * ncur;
            for (int i = 0; i < ncur; i++) s = fmaf(wr[i], cur[i], s);
            nxt[j] = leaky(s, m.leak);
        }
        p = b + nh;
        cur = nxt; ncur = nh;
        nxt = (nxt == bufA) ? bufB : bufA;
    }
    const float* b = p + m.nout * ncur;
    for (int j = 0; j < m.nout; j++) {
        float s = b[j];
        const float* wr = p + j * ncur;
        for (int i = 0; i < ncur; i++) s = fmaf(wr[i], cur[i], s);
        out[j] = out_act(s, m.clamp_out);
    }
}

// Per-pixel weighted squared error, one channel term at a time.
// Double accumulation (loss_subset, main.cpp:1746): each term cw[c] * (d * d) is a float product.
__device__ __forceinline__ double pixel_err_d(const DevModel& m, const float* o, const float* t) {
    double s = 0.0;
    for (int c = 0; c < m.nout; c++) { const float d = o[c] - t[c]; s += (double)(m.cw[c] * (d * d)); }
    return s;
}
// Float accumulation (decode_err, main.cpp:1731).
__device__ __forceinline__ float pixel_err_f(const DevModel& m, const float* o, const float* t) {
    float e = 0.0f;
    for (int c = 0; c < m.nout; c++) { const float d = o[c] - t[c]; e += m.cw[c] * (d * d); }
    return e;
}

}  // namespace ntcb
