// Population evaluation on the 5th-generation tensor core (tcgen05, kind::tf32, 3xTF32 products).
//
// The reference evaluates one pixel per thread on the FP32 pipe (k_mlp_es_eval, cuda/ntc_cuda.cu:270-291;
// mlp_forward, main.cpp:603-627). Here one CTA of 128 threads owns one antithetic candidate pair and a
// chunk of minibatch rows, and each 128-row tile of each sign goes through
//
//   D1 = X  W0^T      X  = [features | 1 | 0 pad]  (K1 = NIN + 1 rounded up to 8; b0 folded in as a column)
//   D2 = H1 W1^T      H1 = leaky(D1)               (K2 = H1 width)
//   o  = b2 + W2 H2   H2 = leaky(D2 + b1)          3 outputs: packed FP32 in registers (a 16-wide MMA would be
//                                                  mostly padding); 12 outputs: one more MMA layer into D3
//
// Row r of a tile is TMEM lane r, so thread t (warp w = t / 32) owns row t: it loads its accumulator row
// from TMEM, applies bias / activation, and stores the next layer's A operand back to TMEM (A-from-TMEM
// MMAs). The B operands (both signs' W0 | b0 and W1) sit in shared memory, K-major without swizzle.
// One warp per stream issues the MMAs: the converged warp elects one lane, which issues all of a layer's MMAs
// (compile-time TMEM / shared addresses, unrolled) and commits them to an mbarrier.
//
// Schedule per stream (u = tile x sign): L1(u) issued -> wait, load, activation, store H -> L2(u) issued ->
// wait, load D2 -> L1(u + 1) issued (the next tile's features were prefetched one tile ahead), together with
// the output-layer MMAs of u when those run on the tensor core -> the output layer / error of u finish on the
// CUDA cores while the tensor core works on L1(u + 1). A kernel that allocates TMEM is held to one resident
// CTA per SM, so the overlap comes from four independent 128-thread streams inside each CTA (below).
//
// Precision: every tensor product is formed as 3xTF32, a b = a_hi b_hi + a_hi b_lo + a_lo b_hi with x_hi the
// top 19 bits of x and x_lo = x - x_hi (exact), accumulated in FP32 by the tensor core. The dropped a_lo b_lo
// term and the TF32 truncation of the lo parts leave a relative error near 2^-21 per product: FP32-level, but
// not the bit pattern of the reference's sequential FMA chain. The output sigmoid uses the fast exponential.
// Fitness agrees with the exact kernels to ~1e-6 relative (the pinned tolerance is 1e-5). FD candidates (mode 1:
// the stats pair and weight j at +-h) run on this kernel too unless the exact mode is selected; the packed-FP32
// kernel stays available for bit-exact runs (ntcb_set_pop_kernel).
//
// Every mbarrier wait is bounded: on time-out the CTA records an error flag, stops issuing, gives the
// outstanding MMAs one more bounded wait and still frees its TMEM.
#include "kernels.h"
#include "mlp_tile.cuh"
#include "pop_common.cuh"
#include "tc.cuh"
#include "latent_features.cuh"
#include "fixed_layout.cuh"
#include "quant.cuh"

#include <algorithm>
#include <type_traits>

namespace ntcb {

namespace {

constexpr int kTcRows = 128;                  // rows per tile (= TMEM lanes = threads of one stream)
constexpr int kTmemCols = 512;                // TMEM columns of an SM, all allocated by the one resident CTA
constexpr uint32_t kTcWaitPolls = 4000;       // mbarrier polls (<= 1 ms each) before a wait is declared failed

__host__ __device__ constexpr int round_up(int x, int m) { return (x + m - 1) / m * m; }

// Canonical no-swizzle K-major float offset of element (n, k) of an [N][K] B operand: 8-row x 4-float core
// matrices, K chunks 32 floats apart (LBO = 128 B), 8-row groups K * 8 floats apart (SBO = 32 K bytes).
__host__ __device__ constexpr int kmajor(int n, int k, int K) { return (n >> 3) * (K * 8) + (k >> 2) * 32 + (n & 7) * 4 + (k & 3); }

template <class S>
struct TcShape {
    // Layer-1 bias: a column of X (X = [features | 1 | 0 pad]) when the features leave padding in their 8-wide K step,
    // otherwise (8 features) a K step of its own against the constant block (below), which keeps X at 8 columns.
    static constexpr bool XB = S::NIN % 8 != 0;
    static constexpr int K1 = round_up(S::NIN + (XB ? 1 : 0), 8);
    static constexpr int N1 = round_up(S::H1, 16);
    static constexpr int K2 = S::H1;
    static constexpr int K3 = S::H2;
    static constexpr int N3 = round_up(S::NOUT, 16);
    static constexpr int NOUTP = round_up(S::NOUT, 4);
    // The output layer runs on the tensor core for wide outputs (12: measured 1.33 vs 1.52 ms at config 3)
    // and on the FP32 pipe for 3 outputs (0.86 vs 1.03 ms at config 2), where 16-wide MMAs are mostly padding.
    static constexpr bool L3TC = S::NOUT > 4;
    // FP32 output layer: layer 2 also produces W2 h2 (the output layer's linear part) in NLIN extra accumulator columns.
    static constexpr int NLIN = L3TC ? 0 : S::NOUT;
    static constexpr int N2 = round_up(S::H2 + NLIN, 16);
    static constexpr int D2COLS = round_up(S::H2 + NLIN, 4);   // accumulator columns the layer-2 epilogue loads
    static constexpr int P = S::H1 * S::NIN + S::H1 + S::H2 * S::H1 + S::H2 + S::NOUT * S::H2 + S::NOUT;
    static_assert(S::H1 % 8 == 0 && S::H2 % 8 == 0, "hidden widths must be multiples of 8");
    static_assert(N1 <= 32 && N2 <= 32 && N3 <= 16, "accumulators wider than their reserved TMEM columns");
    // shared memory, floats, per weight set (sign)
    static constexpr int oB1h = 0, oB1l = oB1h + N1 * K1;           // layer 1: [W0 | b0] (W0 alone without XB)
    static constexpr int oB2h = oB1l + N1 * K1, oB2l = oB2h + N2 * K2;   // layer 2, H step: c1 W1 (+ W2 c1 W1 rows)
    static constexpr int oB2xh = oB2l + N2 * K2, oB2xl = oB2xh + N2 * K1;   // layer 2, X step: leak W1 [W0 | b0] (+ W2 rows)
    static constexpr int ob1 = oB2xl + N2 * K1;                     // b1 [H2]
    static constexpr int oW2 = round_up(ob1 + S::H2, 4);            // FP32 output layer: c1 W2 [NOUT][H2], row-major
    static constexpr int ob2 = oW2 + S::NOUT * S::H2;               // b2 [NOUTP]
    static_assert(S::H2 % 4 == 0, "output-layer rows are read as float4");
    static constexpr int oB3h = round_up(ob2 + NOUTP, 4), oB3l = oB3h + N3 * K3;   // W2 as an MMA B operand
    // b1 as an extra K step of layer 2: B block [N2][8] K-major with b1 (and W2 b1) in k = 0 (hi / lo), against a
    // constant A block (column 0 = 1, columns 1-7 = 0) that every stream of the CTA shares
    static constexpr int oBbh = oB3l + N3 * K3, oBbl = oBbh + N2 * 8;
    static constexpr int oB0h = oBbl + N2 * 8, oB0l = oB0h + N1 * 8;   // layer-1 bias step without XB: b0 in k = 0
    static constexpr int oRaw = oB0l + N1 * 8;                      // the set's flat weights (staging input)
    static constexpr int SIGN = round_up(oRaw + P, 32);
    // TMEM columns of one stream: D (layers 1 and 2), D3 (tensor output layer only), X and H as A operands, each
    // split into hi / lo and interleaved by 8-column K steps ([hi 8 | lo 8] per step)
    static constexpr int cD = 0, cD3 = 32, cX = L3TC ? 48 : 32, cH = cX + 2 * K1;
    static constexpr int COLS = cH + 2 * K2;
    // Layer 1 accumulates into the H columns (N1 <= 2 K2), which its epilogue overwrites row by row with the split
    // activations: layer 1 of the next unit then never waits for the threads to finish reading the layer-2
    // accumulator D. With the tensor-core output layer, whose MMAs read H while the next layer 1 runs, it uses D.
    static constexpr int cL1 = L3TC ? cD : cH;
    static_assert(L3TC || N1 <= 2 * K2, "the layer-1 accumulator fits the H columns");
    // Streams per CTA: as many as the SM's TMEM holds, up to 5 (640 threads leave 102 registers per thread: enough for
    // up to 6 features, and for 8 with the FP32 3-output layer; the 12-output shape keeps 4). Measured: 2 streams cost
    // +33 % over 4.
    static constexpr int STREAMS = (kTmemCols / COLS >= 5 && (S::NIN <= 6 || S::NOUT <= 4)) ? 5 : 4;
    static constexpr int TPB = kTcRows * STREAMS;
    static_assert(STREAMS * COLS <= kTmemCols, "TMEM columns");
    static_assert(STREAMS * 2 * SIGN * 4 + 1024 <= 227 * 1024, "the population kernel's two weight sets per stream fit shared memory");
    // Layer-2 bias (and, without XB, the layer-1 bias) on the tensor core when the streams leave 8 TMEM columns for the
    // constant block; otherwise b1 is added in the epilogue.
    static constexpr bool B1TC = STREAMS * COLS + 8 <= kTmemCols;
    static_assert(L3TC || B1TC, "the FP32 output layer's linear part needs the layer-2 bias on the tensor core");
    static_assert(XB || B1TC, "the layer-1 bias step needs the constant block");
    static constexpr int cOne = STREAMS * COLS;   // the constant block's first column (from the CTA's TMEM base)
};

// ---- weight staging: leaky ReLU folded into the operands
// For any slope l, leaky(x) = l x + c1 (x + |x|) with c1 = (1 - l) / 2, and x + |x| = 2 relu(x) exactly, which is
// one add with an absolute-value operand on the FP32 pipe (no multiply, no ALU max). So
//   h2 = W1 leaky(h1) + b1 = (c1 W1) (h1 + |h1|) + (l W1 W0) x + (l W1 b0 + b1)        (h1 = W0 x + b0)
// layer 2 takes A = split(h1 + |h1|) against B = c1 W1 (the H step) plus A = X against B = l W1 [W0 | b0] (one more
// 8-wide K step on the features already in TMEM), and for the FP32 output layer
//   out = b2 + W2 leaky(h2) = b2 + l (W2 h2) + (c1 W2) (h2 + |h2|)
// where W2 h2 comes out of layer 2 itself: B rows H2 .. H2 + NOUT hold W2 times the rows above them (W2 c1 W1,
// W2 l W1 [W0 | b0], W2 b1), filling the accumulator's padding columns.
template <class S>
__device__ __forceinline__ void put_split(float* sw, int oh, int ol, int idx, float w) {
    const float hi = tc::tf32_hi(w);
    sw[oh + idx] = hi;
    sw[ol + idx] = w - hi;
}

// Row j < H2 of the layer-2 bias step: b1 (+ l W1 b0 when b0 is not a column of X).
template <class S>
__device__ __forceinline__ float bias2_row(const float* W1, const float* b0, const float* b1, float leak, int j) {
    if constexpr (TcShape<S>::XB) {
        return b1[j];
    } else {
        float v = 0.0f;
        for (int q = 0; q < S::H1; q++) v = fmaf(W1[j * S::H1 + q], b0[q], v);
        return fmaf(leak, v, b1[j]);
    }
}

// Phase A of staging one weight set from its flat weights at sw + oRaw (the reference layout, main.cpp:549-599):
// every derived value that needs only the flat weights. Threads tid, tid + nthr, ... of the set's staging group.
template <class S>
__device__ __forceinline__ void stage_set_a(float* sw, float leak, int tid, int nthr) {
    using T = TcShape<S>;
    const float* W0 = sw + T::oRaw;
    const float* b0 = W0 + S::H1 * S::NIN;
    const float* W1 = b0 + S::H1;
    const float* b1 = W1 + S::H2 * S::H1;
    const float* W2 = b1 + S::H2;
    const float* b2 = W2 + S::NOUT * S::H2;
    const float c1 = 0.5f * (1.0f - leak);
    constexpr int XC = S::NIN + (T::XB ? 1 : 0);   // X columns with weights: the features (and the bias column)
    constexpr int nB1 = S::H1 * XC, nB0 = T::XB ? 0 : S::H1, nB2 = (S::H2 + T::NLIN) * S::H1, nB2x = S::H2 * XC;
    constexpr int nBb = T::B1TC ? S::H2 + T::NLIN : 0, nW2 = S::NOUT * S::H2, nb = S::H2 + S::NOUT;
    constexpr int total = nB1 + nB0 + nB2 + nB2x + nBb + nW2 + nb;
    for (int e = tid; e < total; e += nthr) {
        int k = e;
        if (k < nB1) {                        // layer 1: [W0 | b0], or W0
            const int j = k / XC, i = k - j * XC;
            put_split<S>(sw, T::oB1h, T::oB1l, kmajor(j, i, T::K1), i < S::NIN ? W0[j * S::NIN + i] : b0[j]);
            continue;
        }
        k -= nB1;
        if (k < nB0) {                        // layer-1 bias step: b0
            put_split<S>(sw, T::oB0h, T::oB0l, kmajor(k, 0, 8), b0[k]);
            continue;
        }
        k -= nB0;
        if (k < nB2) {                        // layer 2, H step: c1 W1, then the output rows W2 (c1 W1)
            const int j = k / S::H1, i = k - j * S::H1;
            float v;
            if (j < S::H2) {
                v = c1 * W1[j * S::H1 + i];
            } else {
                const int c = j - S::H2;
                v = 0.0f;
                for (int q = 0; q < S::H2; q++) v = fmaf(W2[c * S::H2 + q], c1 * W1[q * S::H1 + i], v);
            }
            put_split<S>(sw, T::oB2h, T::oB2l, kmajor(j, i, T::K2), v);
            continue;
        }
        k -= nB2;
        if (k < nB2x) {                       // layer 2, X step: l W1 [W0 | b0], or l W1 W0
            const int j = k / XC, i = k - j * XC;
            float v = 0.0f;
            for (int q = 0; q < S::H1; q++) v = fmaf(W1[j * S::H1 + q], i < S::NIN ? W0[q * S::NIN + i] : b0[q], v);
            put_split<S>(sw, T::oB2xh, T::oB2xl, kmajor(j, i, T::K1), leak * v);
            continue;
        }
        k -= nB2x;
        if (k < nBb) {                        // layer-2 bias step: its rows (W2 times them: phase B)
            if (k < S::H2) put_split<S>(sw, T::oBbh, T::oBbl, kmajor(k, 0, 8), bias2_row<S>(W1, b0, b1, leak, k));
            continue;
        }
        k -= nBb;
        if (k < nW2) {                        // output layer: c1 W2 (FP32 pipe), or W2 as an MMA operand and as floats
            if constexpr (T::L3TC) {
                const int o = k / S::H2, j = k - o * S::H2;
                put_split<S>(sw, T::oB3h, T::oB3l, kmajor(o, j, T::K3), W2[k]);
                sw[T::oW2 + k] = W2[k];
            } else {
                sw[T::oW2 + k] = c1 * W2[k];
            }
            continue;
        }
        k -= nW2;
        if (k < S::H2) sw[T::ob1 + k] = b1[k];
        else sw[T::ob2 + k - S::H2] = b2[k - S::H2];
    }
}

// Phase B: the output rows of the X step, W2 (l W1 [W0 | b0]), and of the bias step, W2 (b1 + ...), from phase A's
// values (hi + lo = the exact float), so no thread of phase A runs a product of two 24-long sums.
template <class S>
__device__ __forceinline__ void stage_set_b(float* sw, int tid, int nthr) {
    using T = TcShape<S>;
    const float* W2 = sw + T::oRaw + S::H1 * S::NIN + S::H1 + S::H2 * S::H1 + S::H2;
    constexpr int XC = S::NIN + (T::XB ? 1 : 0);
    constexpr int nx = T::NLIN * XC, nb = T::B1TC ? T::NLIN : 0;
    for (int e = tid; e < nx + nb; e += nthr) {
        if (e < nx) {
            const int c = e / XC, i = e - c * XC;
            float v = 0.0f;
            for (int q = 0; q < S::H2; q++) {
                const int at = kmajor(q, i, T::K1);
                v = fmaf(W2[c * S::H2 + q], sw[T::oB2xh + at] + sw[T::oB2xl + at], v);
            }
            put_split<S>(sw, T::oB2xh, T::oB2xl, kmajor(S::H2 + c, i, T::K1), v);
        } else {
            const int c = e - nx;
            float v = 0.0f;
            for (int q = 0; q < S::H2; q++) {
                const int at = kmajor(q, 0, 8);
                v = fmaf(W2[c * S::H2 + q], sw[T::oBbh + at] + sw[T::oBbl + at], v);
            }
            put_split<S>(sw, T::oBbh, T::oBbl, kmajor(S::H2 + c, 0, 8), v);
        }
    }
}

__device__ __forceinline__ bool elect_one() {
    uint32_t p = 0;
    asm volatile("{\n\t.reg .pred P1;\n\telect.sync _|P1, 0xffffffff;\n\tselp.b32 %0, 1, 0, P1;\n\t}" : "=r"(p));
    return p != 0;
}

__device__ __forceinline__ float rcp_approx(float x) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}
// Leaky ReLU of a pair; for 0 <= leak <= 1 (the only slopes the compiled shapes admit) max(x, leak x)
// equals the reference's select for every float.
__device__ __forceinline__ float2 leaky_pair(float2 x, float leak) {
    const float2 t = __fmul2_rn(x, make_float2(leak, leak));
    return make_float2(fmaxf(x.x, t.x), fmaxf(x.y, t.y));
}

// Split N (multiple of 8) values into hi / lo and store them as an interleaved A operand from TMEM column c:
// K step q / 8 occupies columns [c + 2q, c + 2q + 16) = [hi of v[q .. q + 8) | lo of v[q .. q + 8)].
template <int N>
__device__ __forceinline__ void store_split(uint32_t trow, int c, const float* v) {
#pragma unroll
    for (int q = 0; q < N; q += 8) {
        float hl[16];
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
            const float2 x = make_float2(v[q + j], v[q + j + 1]);
            const float2 h = make_float2(tc::tf32_hi(x.x), tc::tf32_hi(x.y));
            const float2 l = __ffma2_rn(h, make_float2(-1.0f, -1.0f), x);   // x - hi, exact
            hl[j] = h.x; hl[j + 1] = h.y; hl[8 + j] = l.x; hl[8 + j + 1] = l.y;
        }
        tc::st_x8p(trow + c + 2 * q, hl);          // two 8-column stores: one 16-column store spills registers
        tc::st_x8p(trow + c + 2 * q + 8, hl + 8);
    }
}
// N (multiple of 4) accumulator columns from TMEM column c into v, in as few loads as the widths allow.
template <int N>
__device__ __forceinline__ void load_acc(uint32_t trow, int c, float* v) {
    static_assert(N % 4 == 0, "accumulator columns in fours");
#pragma unroll
    for (int q = 0; q + 16 <= N; q += 16) tc::ld_x16p(trow + c + q, v + q);
    constexpr int r = N / 16 * 16;
    if constexpr (N % 16 >= 8) tc::ld_x8p(trow + c + r, v + r);
    if constexpr (N % 8 == 4) tc::ld_x4p(trow + c + N - 4, v + N - 4);
}

// Output layer + weighted squared error of one row on the FP32 pipe, from the layer-2 accumulator row h: h[0 .. H2)
// = h2 (b1 included), h[H2 + c] = (W2 h2)_c. out_c = b2_c + l (W2 h2)_c + sum_j (c1 W2)_cj (h2_j + |h2_j|) (the folded
// leaky ReLU: one add per hidden unit), hidden units in pairs, two partial sums per output, float error sum.
// Shapes whose population kernel runs the output layer on the tensor core (L3TC) have no W2 h2 columns: there the
// FP32 form (the latent pass) applies the leaky ReLU to h2 as written (adding b1 when the tensor core has not), with
// the plain W2.
template <class S, bool CLAMP>
__device__ __forceinline__ float out_layer_error(const DevModel& m, const float* ws, const float* h, const float* t,
                                                 float leak) {
    using T = TcShape<S>;
    float2 acc[S::NOUT];
#pragma unroll
    for (int c = 0; c < S::NOUT; c++) acc[c] = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int j = 0; j < S::H2; j += 4) {
        float2 r0, r1;
        if constexpr (T::L3TC) {
            r0 = make_float2(h[j], h[j + 1]);
            r1 = make_float2(h[j + 2], h[j + 3]);
            if constexpr (!T::B1TC) {
                const float4 b = *reinterpret_cast<const float4*>(ws + T::ob1 + j);
                r0 = __fadd2_rn(r0, make_float2(b.x, b.y));
                r1 = __fadd2_rn(r1, make_float2(b.z, b.w));
            }
            r0 = leaky_pair(r0, leak);
            r1 = leaky_pair(r1, leak);
        } else {
            r0 = make_float2(h[j] + fabsf(h[j]), h[j + 1] + fabsf(h[j + 1]));
            r1 = make_float2(h[j + 2] + fabsf(h[j + 2]), h[j + 3] + fabsf(h[j + 3]));
        }
#pragma unroll
        for (int c = 0; c < S::NOUT; c++) {
            const float4 w = *reinterpret_cast<const float4*>(ws + T::oW2 + c * S::H2 + j);
            acc[c] = __ffma2_rn(make_float2(w.x, w.y), r0, acc[c]);
            acc[c] = __ffma2_rn(make_float2(w.z, w.w), r1, acc[c]);
        }
    }
    float e = 0.0f;
#pragma unroll
    for (int c = 0; c < S::NOUT; c++) {
        float sum = ws[T::ob2 + c] + (acc[c].x + acc[c].y);
        if constexpr (!T::L3TC) sum = fmaf(leak, h[S::H2 + c], sum);
        const float o = CLAMP ? fminf(fmaxf(sum, 0.0f), 1.0f) : rcp_approx(1.0f + __expf(-sum));
        const float d = o - t[c];
        e = fmaf(m.cw[c], d * d, e);
    }
    return e;
}
// The layer-1 epilogue's operand for layer 2: h1 + |h1| (= 2 relu(h1)), in place.
template <int N>
__device__ __forceinline__ void relu2(float* h) {
#pragma unroll
    for (int j = 0; j < N; j++) h[j] = h[j] + fabsf(h[j]);
}

// The issuing warp (converged; one elected lane issues): D = A B^T over K as 3xTF32 (lo*hi, hi*lo, hi*hi per 8-wide K
// step), then commit. a: the
// interleaved A operand in TMEM (K step s: hi at a + 16 s, lo at a + 16 s + 8); b_hi4 / b_lo4: the B operands' shared
// addresses shifted right by 4 (hoisted; each descriptor is then one add).
template <int K, int N>
__device__ __forceinline__ void issue3(uint32_t d, uint32_t a, uint32_t b_hi4, uint32_t b_lo4, uint64_t* bar) {
    constexpr uint32_t id = tc::idesc_tf32(kTcRows, N);
    constexpr uint32_t sbo = (uint32_t)K * 32u;
    tc::fence_after_sync();
    if (elect_one()) {
#pragma unroll
        for (int s = 0; s < K / 8; s++) {
            tc::mma_tf32_ts(d, a + 16 * s + 8, tc::sdesc_s4(b_hi4 + 16 * s, 128, sbo), id, s > 0 ? 1u : 0u);
            tc::mma_tf32_ts(d, a + 16 * s, tc::sdesc_s4(b_lo4 + 16 * s, 128, sbo), id, 1u);
            tc::mma_tf32_ts(d, a + 16 * s, tc::sdesc_s4(b_hi4 + 16 * s, 128, sbo), id, 1u);
        }
        tc::commit(bar);
    }
    __syncwarp();
}

// Layer 2: the 3xTF32 product of the H step over K (A = split(h1 + |h1|)), then the X step over KX (A = the features,
// B = l W1 [W0 | b0]), then with B1TC D += 1 * b1_lo + 1 * b1_hi from the constant A block `one` (its lo part is
// zero), then commit.
template <int K, int KX, int N, bool BIAS>
__device__ __forceinline__ void issue_l2(uint32_t d, uint32_t a, uint32_t b_hi4, uint32_t b_lo4, uint32_t ax, uint32_t bx_hi4,
                                         uint32_t bx_lo4, uint32_t one, uint32_t bb_hi4, uint32_t bb_lo4, uint64_t* bar) {
    constexpr uint32_t id = tc::idesc_tf32(kTcRows, N);
    constexpr uint32_t sbo = (uint32_t)K * 32u, sbox = (uint32_t)KX * 32u;
    tc::fence_after_sync();
    if (elect_one()) {
#pragma unroll
        for (int s = 0; s < K / 8; s++) {
            tc::mma_tf32_ts(d, a + 16 * s + 8, tc::sdesc_s4(b_hi4 + 16 * s, 128, sbo), id, s > 0 ? 1u : 0u);
            tc::mma_tf32_ts(d, a + 16 * s, tc::sdesc_s4(b_lo4 + 16 * s, 128, sbo), id, 1u);
            tc::mma_tf32_ts(d, a + 16 * s, tc::sdesc_s4(b_hi4 + 16 * s, 128, sbo), id, 1u);
        }
#pragma unroll
        for (int s = 0; s < KX / 8; s++) {
            tc::mma_tf32_ts(d, ax + 16 * s + 8, tc::sdesc_s4(bx_hi4 + 16 * s, 128, sbox), id, 1u);
            tc::mma_tf32_ts(d, ax + 16 * s, tc::sdesc_s4(bx_lo4 + 16 * s, 128, sbox), id, 1u);
            tc::mma_tf32_ts(d, ax + 16 * s, tc::sdesc_s4(bx_hi4 + 16 * s, 128, sbox), id, 1u);
        }
        if constexpr (BIAS) {
            tc::mma_tf32_ts(d, one, tc::sdesc_s4(bb_lo4, 128, 256), id, 1u);
            tc::mma_tf32_ts(d, one, tc::sdesc_s4(bb_hi4, 128, 256), id, 1u);
        }
        tc::commit(bar);
    }
    __syncwarp();
}

// Byte offset / 16 of a float offset into a weight set (every B operand block starts on a 16-byte boundary).
template <int FLOATS>
constexpr uint32_t s4() { static_assert(FLOATS % 4 == 0, "B operand blocks are 16-byte aligned"); return (uint32_t)FLOATS / 4; }

// Layer 1 of unit (A = X of the stream, B = the sign's W0 | b0 block); sb4 = the sign's weight set address >> 4.
template <class T>
__device__ __forceinline__ void issue_layer1(uint32_t tbase, uint32_t tb, uint32_t sb4, uint64_t* bar) {
    if constexpr (T::XB)
        issue3<T::K1, T::N1>(tb + T::cL1, tb + T::cX, sb4 + s4<T::oB1h>(), sb4 + s4<T::oB1l>(), bar);
    else   // the features over K1, then b0 against the constant block
        issue_l2<T::K1, 0, T::N1, true>(tb + T::cL1, tb + T::cX, sb4 + s4<T::oB1h>(), sb4 + s4<T::oB1l>(), 0, 0, 0, tbase + T::cOne,
                                        sb4 + s4<T::oB0h>(), sb4 + s4<T::oB0l>(), bar);
}
// Layer 2 of unit (A = H and X of the stream, B = the sign's H-step, X-step and bias blocks).
template <class T>
__device__ __forceinline__ void issue_layer2(uint32_t tbase, uint32_t tb, uint32_t sb4, uint64_t* bar) {
    issue_l2<T::K2, T::K1, T::N2, T::B1TC>(tb + T::cD, tb + T::cH, sb4 + s4<T::oB2h>(), sb4 + s4<T::oB2l>(), tb + T::cX,
                                            sb4 + s4<T::oB2xh>(), sb4 + s4<T::oB2xl>(), tbase + T::cOne, sb4 + s4<T::oBbh>(),
                                            sb4 + s4<T::oBbl>(), bar);
}

// The constant A block of the layer-2 bias step: TMEM column cOne = 1, cOne + 1 .. + 7 = 0 on all 128 lanes,
// written by the 128 threads of stream 0 (thread t of warp w reaches lane 32 w + t).
template <class T>
__device__ __forceinline__ void init_one_block(uint32_t tbase, int g, int warp) {
    if constexpr (T::B1TC) {
        if (g == 0) {
            const float v[8] = {1.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
            tc::st_x8(tbase + T::cOne + ((uint32_t)(warp * 32) << 16), v);
            tc::wait_st();
        }
    }
}

// Named barrier over the 128 threads of one stream (ids 1..STREAMS; 0 is __syncthreads), AND-reducing v.
__device__ __forceinline__ bool stream_sync_and(int id, bool v) {
    uint32_t r;
    asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, %2, 128, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
                 : "=r"(r) : "r"((uint32_t)v), "r"(id) : "memory");
    return r != 0;
}
__device__ __forceinline__ void stream_sync(int id) { asm volatile("bar.sync %0, 128;" ::"r"(id) : "memory"); }

// Fixed-order sum over one stream's 128 threads (warp trees, then the 4 warp totals in order); valid in its thread 0.
__device__ __forceinline__ double stream_sum(double v, double* red4, int id) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
    const int lane = threadIdx.x & 31, w = (threadIdx.x >> 5) & 3;
    stream_sync(id);
    if (lane == 0) red4[w] = v;
    stream_sync(id);
    return red4[0] + red4[1] + red4[2] + red4[3];
}

// One CTA per SM (a kernel that allocates TMEM is held to one resident CTA per SM), four streams of 128
// threads. Stream g owns TMEM columns [128 g, 128 g + 128), one mbarrier, one named barrier and one pair of
// weight sets, and works through a contiguous range of the (pair, chunk) items, so consecutive items
// mostly share a pair and its weights are staged once. The streams interleave on the SM: one stream's
// element-wise work overlaps the others' MMAs.
template <class S, bool L3TC, bool CLAMP>
__global__ void __launch_bounds__(TcShape<S>::TPB, 1) k_pop_eval_tc(DevModel m, PopArgs a, int chunks) {
    using T = TcShape<S>;
    constexpr int NS = T::STREAMS;
    extern __shared__ __align__(1024) float dyn[];   // [NS][2][T::SIGN]
    __shared__ __align__(8) uint64_t bars[NS];
    __shared__ __align__(8) uint64_t bars1[NS];   // layer-1 commits (separate: see below)
    __shared__ __align__(8) uint64_t bars3[NS];   // output-layer commits
    __shared__ uint32_t tbase;
    __shared__ double red[NS][4];
    const int g = threadIdx.x >> 7, tid = threadIdx.x & 127, warp = tid >> 5;
    // The warp that issues a stream's MMAs: local warp g % 4, i.e. global warp 4 g + g % 4, so the streams'
    // issue work spreads over the SM's four schedulers (warp w runs on scheduler w % 4) instead of all
    // landing on scheduler 0.
    const int issuer = g & 3;
    const int bar_id = 1 + g;
    float* sw = dyn + g * 2 * T::SIGN;
    uint64_t* bar = &bars[g];
    // Layer 1, layer 2 and the tensor-core output layer commit to three mbarriers. On one mbarrier two commits could
    // both complete before a slow thread polls for the first (sign 1's layer 1 goes out as soon as the issuing warp has
    // seen layer 2 complete, with no stream barrier in between; the output-layer MMAs and the next layer 1 go out back
    // to back), leaving the barrier at the parity that thread waits for: it would then wait for a phase nobody
    // completes. On its own barrier each kind's next commit needs every thread past a stream barrier it reaches only
    // after waiting for the previous one, so commits and waits alternate on each.
    uint64_t* bar1 = &bars1[g];
    uint64_t* bar3 = &bars3[g];

    if (threadIdx.x < 32) tc::tmem_alloc(&tbase, kTmemCols);
    if (tid == 0) { tc::mbar_init(bar, 1); tc::mbar_init(bar1, 1); tc::mbar_init(bar3, 1); tc::mbar_init_fence(); }
    for (int i = threadIdx.x; i < NS * 2 * T::SIGN; i += T::TPB) dyn[i] = 0.0f;   // padding stays zero
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    init_one_block<T>(tbase, g, warp);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();

    const uint32_t tb = tbase + (uint32_t)(T::COLS * g);
    const uint32_t trow = tb + ((uint32_t)(warp * 32) << 16);
    const uint32_t sb0 = tc::smem_addr(sw) >> 4, sb1 = sb0 + s4<T::SIGN>();   // the signs' weight sets, address >> 4
    const float leak = m.leak;
    uint32_t waited = 0, waited1 = 0, waited3 = 0;   // completed phases this thread has observed on bar / bar1 / bar3
    bool ok = true;

    auto wait_mma = [&]() {
        const bool done = tc::mbar_wait_bounded(bar, waited & 1u, kTcWaitPolls);
        if (done) waited++;
        ok = ok && done;
        tc::fence_after_sync();
    };
    auto wait_mma1 = [&]() {
        const bool done = tc::mbar_wait_bounded(bar1, waited1 & 1u, kTcWaitPolls);
        if (done) waited1++;
        ok = ok && done;
        tc::fence_after_sync();
    };
    auto wait_mma3 = [&]() {
        const bool done = tc::mbar_wait_bounded(bar3, waited3 & 1u, kTcWaitPolls);
        if (done) waited3++;
        ok = ok && done;
        tc::fence_after_sync();
    };
    float xr[S::NIN];      // features of the next tile (prefetched one tile ahead)
    auto load_x = [&](int base) {
        const int s = min(base + tid, a.M - 1);
#pragma unroll
        for (int i = 0; i < S::NIN; i++) xr[i] = __ldg(a.feat_t + (long long)i * a.mstride + s);
    };
    auto store_x = [&]() {
        float x[T::K1];
#pragma unroll
        for (int i = 0; i < T::K1; i++) x[i] = i < S::NIN ? xr[i] : (i == S::NIN ? 1.0f : 0.0f);
        store_split<T::K1>(trow, T::cX, x);
    };
    const long long items = (long long)a.ncand * chunks;
    const long long nstreams = (long long)gridDim.x * T::STREAMS, gs = (long long)blockIdx.x * T::STREAMS + g;
    const long long i0 = gs * items / nstreams, i1 = (gs + 1) * items / nstreams;
    int cur = -1;
#pragma unroll 1
    for (long long item = i0; item < i1 && ok; item++) {
        const int pl = (int)(item / chunks), chunk = (int)(item - (long long)pl * chunks);
        if (pl != cur) {
            // stage both perturbed weight sets of this pair (the previous pair's MMAs have all completed)
            const int cand = pop_cand(a, pl);
            const float* e = (a.mode == 0 && a.sigma != 0.0f) ? a.eps + (long long)pl * m.P : nullptr;
            constexpr int PER = (T::P + kTcRows - 1) / kTcRows, BATCH = 4;   // weights per thread, loaded 4 at a time
#pragma unroll 1
            for (int u0 = 0; u0 < PER; u0 += BATCH) {
                float w0r[BATCH], er[BATCH];
#pragma unroll
                for (int u = 0; u < BATCH; u++) {
                    const int k = tid + (u0 + u) * kTcRows;
                    w0r[u] = k < T::P ? a.w0[k] : 0.0f;
                    er[u] = (e && k < T::P) ? e[k] : 0.0f;
                }
#pragma unroll
                for (int u = 0; u < BATCH; u++) {
                    const int k = tid + (u0 + u) * kTcRows;
                    if (k < T::P) {
                        float wp, wm;
                        perturbed_weight_of(a, w0r[u], e ? &er[u] : nullptr, k, cand, wp, wm);
                        sw[T::oRaw + k] = wp;
                        sw[T::SIGN + T::oRaw + k] = wm;
                    }
                }
            }
            stream_sync(bar_id);
            stage_set_a<S>(sw, leak, tid, kTcRows);
            stage_set_a<S>(sw + T::SIGN, leak, tid, kTcRows);
            stream_sync(bar_id);
            stage_set_b<S>(sw, tid, kTcRows);
            stage_set_b<S>(sw + T::SIGN, tid, kTcRows);
            tc::fence_proxy_async_smem();
            cur = pl;
        }
        const int row0 = chunk * a.chunk;
        const int row1 = min(a.M, row0 + a.chunk);
        double acc_p = 0.0, acc_m = 0.0;

        // prologue: first tile's features to TMEM, the next tile's prefetched, L1 of (first tile, +) issued
        load_x(row0);
        store_x();
        load_x(row0 + kTcRows);
        tc::wait_st();
        tc::fence_before_sync();
        stream_sync(bar_id);
        if (warp == issuer) issue_layer1<T>(tbase, tb, sb0, bar1);

#pragma unroll 1
        for (int base = row0; base < row1; base += kTcRows) {
            const int row = base + tid;
            const bool valid = row < row1;
            const bool more = base + kTcRows < row1;
            float t[S::NOUT];
            {
                const int s = min(row, a.M - 1);
#pragma unroll
                for (int c = 0; c < S::NOUT; c++) t[c] = __ldg(a.tgt_t + (long long)c * a.mstride + s);
            }
#pragma unroll
            for (int sg = 0; sg < 2; sg++) {
                const uint32_t sb = sg ? sb1 : sb0;
                const float* ws = sw + sg * T::SIGN;
                float h[S::H1 > T::D2COLS ? S::H1 : T::D2COLS];
                // layer 1 result -> H (h1 + |h1|, the folded leaky ReLU)
                wait_mma1();
                load_acc<S::H1>(trow, T::cL1, h);
                tc::wait_ld();
                relu2<S::H1>(h);
                store_split<T::K2>(trow, T::cH, h);
                tc::wait_st();
                tc::fence_before_sync();
                ok = stream_sync_and(bar_id, ok);
                if (!ok) break;
                if (warp == issuer) issue_layer2<T>(tbase, tb, sb, bar);
                // layer 2 result -> registers (with the FP32 output layer: h2 and W2 h2)
                wait_mma();
                if constexpr (!L3TC) {
                    // sign 1 of this tile: the same features, and its layer 1 accumulates into the H columns, which
                    // layer 2 has finished reading; issued at once, no stream barrier, overlapping this unit's loads
                    // and output layer (the issuing warp's lanes agree on the wait's outcome first)
                    if (sg == 0 && warp == issuer && __all_sync(0xffffffffu, ok)) issue_layer1<T>(tbase, tb, sb1, bar1);
                }
                load_acc<L3TC ? S::H2 : T::D2COLS>(trow, T::cD, h);
                tc::wait_ld();
                // next unit's layer 1: the other sign of this tile, or the next tile's + sign
                const bool next = sg == 0 || more;
                if constexpr (L3TC) {
                    // H2 = leaky(D2 + b1) -> TMEM; output-layer MMAs (into D3) and the next unit's layer 1
                    // (into D) go out together as two commits
#pragma unroll
                    for (int j = 0; j < S::H2; j += 4) {
                        float2 h0 = make_float2(h[j], h[j + 1]), h1 = make_float2(h[j + 2], h[j + 3]);
                        if constexpr (!T::B1TC) {
                            const float4 b = *reinterpret_cast<const float4*>(ws + T::ob1 + j);
                            h0 = __fadd2_rn(h0, make_float2(b.x, b.y));
                            h1 = __fadd2_rn(h1, make_float2(b.z, b.w));
                        }
                        h0 = leaky_pair(h0, leak);
                        h1 = leaky_pair(h1, leak);
                        h[j] = h0.x; h[j + 1] = h0.y; h[j + 2] = h1.x; h[j + 3] = h1.y;
                    }
                    store_split<T::K3>(trow, T::cH, h);
                    if (sg == 1 && more) { store_x(); load_x(base + 2 * kTcRows); }
                    tc::wait_st();
                    tc::fence_before_sync();
                    ok = stream_sync_and(bar_id, ok);
                    if (!ok) break;
                    if (warp == issuer) {
                        issue3<T::K3, T::N3>(tb + T::cD3, tb + T::cH, sb + s4<T::oB3h>(), sb + s4<T::oB3l>(), bar3);
                        if (next) issue_layer1<T>(tbase, tb, sg ? sb0 : sb1, bar1);
                    }
                    wait_mma3();
                    float o[T::NOUTP];
#pragma unroll
                    for (int q = 0; q < T::NOUTP; q += 4) tc::ld_x4p(trow + T::cD3 + q, o + q);
                    tc::wait_ld();
                    float e = 0.0f;
#pragma unroll
                    for (int c = 0; c < S::NOUT; c++) {
                        const float sum = o[c] + ws[T::ob2 + c];
                        const float d = (CLAMP ? fminf(fmaxf(sum, 0.0f), 1.0f) : rcp_approx(1.0f + __expf(-sum))) - t[c];
                        e = fmaf(m.cw[c], d * d, e);
                    }
                    if (valid) { if (sg == 0) acc_p += (double)e; else acc_m += (double)e; }
                } else {
                    if (sg == 1) {
                        // the next tile's features into X (free since layer 2 finished), then its + sign's layer 1
                        if (more) {
                            store_x();
                            load_x(base + 2 * kTcRows);
                            tc::wait_st();
                        }
                        tc::fence_before_sync();
                        ok = stream_sync_and(bar_id, ok);
                        if (!ok) break;
                        if (more && warp == issuer) issue_layer1<T>(tbase, tb, sb0, bar1);
                    }
                    // output layer and error of this unit, overlapping the tensor core's next layer 1
                    double e = 0.0;
                    if constexpr (!L3TC) e = valid ? (double)out_layer_error<S, CLAMP>(m, ws, h, t, leak) : 0.0;
                    if (sg == 0) acc_p += e; else acc_m += e;
                }
            }
            if (!ok) break;
        }
        if (!ok) break;
        const double sp = stream_sum(acc_p, red[g], bar_id);
        const double sm = stream_sum(acc_m, red[g], bar_id);
        if (tid == 0) {
            double* dst = a.part + (long long)pl * 2 * chunks;
            dst[chunk] = sp;
            dst[chunks + chunk] = sm;
        }
    }
    if (!ok) {
        // A wait timed out: flag it, give the outstanding MMAs one more bounded wait, then free TMEM.
        if (tid == 0) atomicExch(a.tc_err, 1);
        tc::mbar_wait_bounded(bar, waited & 1u, kTcWaitPolls);
        tc::mbar_wait_bounded(bar1, waited1 & 1u, kTcWaitPolls);
        if (L3TC) tc::mbar_wait_bounded(bar3, waited3 & 1u, kTcWaitPolls);
    }
    tc::fence_before_sync();
    __syncthreads();
    if (threadIdx.x < 32) { tc::fence_after_sync(); tc::tmem_dealloc(tbase, kTmemCols); }
}

template <class S>
void launch_tc(cudaStream_t s, const DevModel& m, const PopArgs& a) {
    using T = TcShape<S>;
    const int chunks = pop_chunks(a.M, a.chunk);
    const size_t smem = (size_t)T::STREAMS * 2 * T::SIGN * sizeof(float);
    constexpr bool kL3TC = T::L3TC;
    const int nsm = device_sm_count();
    const long long items = (long long)a.ncand * chunks;
    const int grid = (int)std::min<long long>(nsm, (items + T::STREAMS - 1) / T::STREAMS);
    if (m.clamp_out) {
        ensure_dynamic_smem((const void*)k_pop_eval_tc<S, kL3TC, true>, (int)smem);
        k_pop_eval_tc<S, kL3TC, true><<<grid, T::TPB, smem, s>>>(m, a, chunks);
    } else {
        ensure_dynamic_smem((const void*)k_pop_eval_tc<S, kL3TC, false>, (int)smem);
        k_pop_eval_tc<S, kL3TC, false><<<grid, T::TPB, smem, s>>>(m, a, chunks);
    }
}

// ---------------------------------------------------------------------------------------------------------
// Latent ES pass on the tensor core: every pixel of [p_begin, p_end) decoded with the active latent levels
// perturbed by +sigma eps_k and by -sigma eps_k for each of the K pairs, dpix[k][p] = (e+ - e-) inv_px with
// e the weighted squared error summed in float (decode_err, main.cpp:1722-1735; LatentTrainer::step,
// main.cpp:1990-2015). The reference launches one kernel per pair (k_lat_pair, cuda/ntc_cuda.cu:358-409).
//
// Same machinery as the population kernel with one weight set shared by all rows: an item is (pair k,
// 128-pixel tile), its two units are the + and - decodes of the tile (X = the +/- perturbed features, which
// share their taps and are gathered together, one item ahead, while the layer-2 MMAs of the current item
// run). The output layer runs on the FP32 pipe.
template <class S, class LY, bool CLAMP>
__global__ void __launch_bounds__(TcShape<S>::TPB, 1) k_lat_eval_tc(DevModel m, const float* __restrict__ wg, const float* __restrict__ z,
                                                         const float* __restrict__ eps, long long nz, const float* __restrict__ tgt,
                                                         int K, unsigned active, float sg, float inv_px, float* __restrict__ dpix,
                                                         long long p_begin, long long p_end, long long pstride,
                                                         int* __restrict__ err) {
    using T = TcShape<S>;
    extern __shared__ __align__(1024) float sw[];   // one weight set [T::SIGN]
    __shared__ __align__(8) uint64_t bars[T::STREAMS];
    __shared__ uint32_t tbase;
    const int g = threadIdx.x >> 7, tid = threadIdx.x & 127, warp = tid >> 5;
    // The warp that issues a stream's MMAs: local warp g % 4, i.e. global warp 4 g + g % 4, so the streams'
    // issue work spreads over the SM's four schedulers (warp w runs on scheduler w % 4) instead of all
    // landing on scheduler 0.
    const int issuer = g & 3;
    const int bar_id = 1 + g;
    uint64_t* bar = &bars[g];

    if (threadIdx.x < 32) tc::tmem_alloc(&tbase, kTmemCols);
    if (tid == 0) { tc::mbar_init(bar, 1); tc::mbar_init_fence(); }
    for (int i = threadIdx.x; i < T::SIGN; i += T::TPB) sw[i] = 0.0f;
    __syncthreads();
    for (int k = threadIdx.x; k < T::P; k += T::TPB) sw[T::oRaw + k] = wg[k];
    __syncthreads();
    stage_set_a<S>(sw, m.leak, threadIdx.x, T::TPB);
    __syncthreads();
    stage_set_b<S>(sw, threadIdx.x, T::TPB);
    tc::fence_proxy_async_smem();
    init_one_block<T>(tbase, g, warp);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();

    const uint32_t tb = tbase + (uint32_t)(T::COLS * g);
    const uint32_t trow = tb + ((uint32_t)(warp * 32) << 16);
    const uint32_t sb = tc::smem_addr(sw) >> 4;   // the weight set's address >> 4
    const float leak = m.leak;
    uint32_t waited = 0;
    bool ok = true;
    auto wait_mma = [&]() {
        const bool done = tc::mbar_wait_bounded(bar, waited & 1u, kTcWaitPolls);
        if (done) waited++;
        ok = ok && done;
        tc::fence_after_sync();
    };

    const long long npix = (long long)m.W * m.H;
    const long long ntiles = (p_end - p_begin + kTcRows - 1) / kTcRows;
    const long long items = (long long)K * ntiles;
    const long long nstreams = (long long)gridDim.x * T::STREAMS, gs = (long long)blockIdx.x * T::STREAMS + g;
    const long long i0 = gs * items / nstreams, i1 = (gs + 1) * items / nstreams;

    // +/- features and targets of this thread's pixel in an item
    float fp[S::NIN], fm[S::NIN], t[S::NOUT];
    auto gather = [&](long long item, float (&xp)[S::NIN], float (&xm)[S::NIN], float (&tt)[S::NOUT]) {
        const int k = (int)(item / ntiles);
        const long long p = p_begin + (item - (long long)k * ntiles) * kTcRows + tid;
        const long long pc = p < p_end ? p : p_end - 1;
        if constexpr (std::is_void_v<LY>) {
            float a[kMaxIn], b[kMaxIn];
            perturbed_features_pm(m, z, eps + (long long)k * nz, active, sg, (int)(pc % m.W), (int)(pc / m.W), a, b);
#pragma unroll
            for (int i = 0; i < S::NIN; i++) { xp[i] = a[i]; xm[i] = b[i]; }
        } else {
            layout_features_pm<LY>(m, z, eps + (long long)k * nz, active, sg, (int)(pc % m.W), (int)(pc / m.W), xp, xm);
        }
#pragma unroll
        for (int c = 0; c < S::NOUT; c++) tt[c] = __ldg(tgt + pc * S::NOUT + c);
    };
    auto store_x = [&](const float (&x)[S::NIN]) {
        float v[T::K1];
#pragma unroll
        for (int i = 0; i < T::K1; i++) v[i] = i < S::NIN ? x[i] : (i == S::NIN ? 1.0f : 0.0f);
        store_split<T::K1>(trow, T::cX, v);
    };
    // layer-1 result -> H in TMEM, then layer 2 issued
    auto layer1_to_layer2 = [&]() {
        float h[S::H1];
        wait_mma();
        load_acc<S::H1>(trow, T::cL1, h);
        tc::wait_ld();
        relu2<S::H1>(h);
        store_split<T::K2>(trow, T::cH, h);
        tc::wait_st();
        tc::fence_before_sync();
        ok = stream_sync_and(bar_id, ok);
        if (ok && warp == issuer) issue_layer2<T>(tbase, tb, sb, bar);
    };

    if (i0 < i1) {
        gather(i0, fp, fm, t);
        store_x(fp);
        tc::wait_st();
        tc::fence_before_sync();
        stream_sync(bar_id);
        if (warp == issuer) issue_layer1<T>(tbase, tb, sb, bar);
    }
#pragma unroll 1
    for (long long item = i0; item < i1 && ok; item++) {
        const bool more = item + 1 < i1;
        float h[T::L3TC ? S::H2 : T::D2COLS];
        float np[S::NIN], nm[S::NIN], nt[S::NOUT];
        // + unit
        layer1_to_layer2();
        if (!ok) break;
        if (more) gather(item + 1, np, nm, nt);    // overlaps the layer-2 MMAs
        wait_mma();
        load_acc<T::L3TC ? S::H2 : T::D2COLS>(trow, T::cD, h);
        tc::wait_ld();
        store_x(fm);
        tc::wait_st();
        tc::fence_before_sync();
        ok = stream_sync_and(bar_id, ok);
        if (!ok) break;
        if (warp == issuer) issue_layer1<T>(tbase, tb, sb, bar);
        const float ep = out_layer_error<S, CLAMP>(m, sw, h, t, leak);
        // - unit
        layer1_to_layer2();
        if (!ok) break;
        wait_mma();
        load_acc<T::L3TC ? S::H2 : T::D2COLS>(trow, T::cD, h);
        tc::wait_ld();
        if (more) { store_x(np); tc::wait_st(); }
        tc::fence_before_sync();
        ok = stream_sync_and(bar_id, ok);
        if (!ok) break;
        if (more && warp == issuer) issue_layer1<T>(tbase, tb, sb, bar);
        const float em = out_layer_error<S, CLAMP>(m, sw, h, t, leak);
        {
            const int k = (int)(item / ntiles);
            const long long p = p_begin + (item - (long long)k * ntiles) * kTcRows + tid;
            if (p < p_end) dpix[(long long)k * pstride + (p - p_begin)] = (ep - em) * inv_px;
        }
#pragma unroll
        for (int i = 0; i < S::NIN; i++) { fp[i] = np[i]; fm[i] = nm[i]; }
#pragma unroll
        for (int c = 0; c < S::NOUT; c++) t[c] = nt[c];
    }
    if (!ok) {
        if (tid == 0) atomicExch(err, 1);
        tc::mbar_wait_bounded(bar, waited & 1u, kTcWaitPolls);
    }
    tc::fence_before_sync();
    __syncthreads();
    if (threadIdx.x < 32) { tc::fence_after_sync(); tc::tmem_dealloc(tbase, kTmemCols); }
}

// ---------------------------------------------------------------------------------------------------------
// --qat selector search on the tensor core (qat_search, main.cpp:2088-2139; the reference's k_qat_search,
// cuda/ntc_cuda.cu:451-492). For level-0 cells of cw x ch pixels (the image a whole multiple of the level, so every
// texel's footprint is its cell) and n = 2^bits candidates per channel, one texel's candidates x pixels are
// rpt = n cw ch consecutive rows of a 128-row tile (rpt a power of two <= 32, so one warp holds a texel), and a tile
// covers 128 / rpt texels. Per channel, in order: every row decodes its pixel with the channel set to its candidate
// (the MMA pipeline of the latent pass, one weight set), each candidate's cell loss is its pixels' errors summed in
// raster order in double by warp shuffles, and the reference's rule (the current value first, a strictly smaller
// loss wins, in index order) picks the value that is installed before the next channel is searched. The cell losses
// carry the 3xTF32 rounding (~1e-6 relative), so near-ties can resolve differently from the exact kernel; the
// reference's own harness accepts exactly that (main.cpp:3136-3146: differing texels within 1e-4 of each other, the
// searched image's loss within 1e-6).
template <class S, class LY, bool CLAMP>
__global__ void __launch_bounds__(TcShape<S>::TPB, 1) k_qat_tc(DevModel m, const float* __restrict__ wg, float* z,
                                                               const float* __restrict__ tgt, const float* __restrict__ grid,
                                                               int bits, int cw, int ch, long long t_begin, long long t_end,
                                                               int* __restrict__ err) {
    using T = TcShape<S>;
    extern __shared__ __align__(1024) float sw[];   // one weight set [T::SIGN]
    __shared__ __align__(8) uint64_t bars[T::STREAMS];
    __shared__ uint32_t tbase;
    const int g = threadIdx.x >> 7, tid = threadIdx.x & 127, warp = tid >> 5, lane = threadIdx.x & 31;
    const int issuer = g & 3;
    const int bar_id = 1 + g;
    uint64_t* bar = &bars[g];

    if (threadIdx.x < 32) tc::tmem_alloc(&tbase, kTmemCols);
    if (tid == 0) { tc::mbar_init(bar, 1); tc::mbar_init_fence(); }
    for (int i = threadIdx.x; i < T::SIGN; i += T::TPB) sw[i] = 0.0f;
    __syncthreads();
    for (int k = threadIdx.x; k < T::P; k += T::TPB) sw[T::oRaw + k] = wg[k];
    __syncthreads();
    stage_set_a<S>(sw, m.leak, threadIdx.x, T::TPB);
    __syncthreads();
    stage_set_b<S>(sw, threadIdx.x, T::TPB);
    tc::fence_proxy_async_smem();
    init_one_block<T>(tbase, g, warp);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();

    const uint32_t tb = tbase + (uint32_t)(T::COLS * g);
    const uint32_t trow = tb + ((uint32_t)(warp * 32) << 16);
    const uint32_t sb = tc::smem_addr(sw) >> 4;
    const float leak = m.leak;
    uint32_t waited = 0;
    bool ok = true;
    auto wait_mma = [&]() {
        const bool done = tc::mbar_wait_bounded(bar, waited & 1u, kTcWaitPolls);
        if (done) waited++;
        ok = ok && done;
        tc::fence_after_sync();
    };

    const DevLevel& L0 = m.lv[0];
    const int n = 1 << bits, cellpix = cw * ch, rpt = n * cellpix, tpt = kTcRows / rpt;
    const int slot = tid / rpt, local = tid - slot * rpt, k = local / cellpix, pi = local - k * cellpix;
    const int group = lane & ~(rpt - 1);        // first lane of this texel's rows
    const float* gv = grid + bits * 257;
    const long long ntiles = (t_end - t_begin + tpt - 1) / tpt;
    const long long nstreams = (long long)gridDim.x * T::STREAMS, gs = (long long)blockIdx.x * T::STREAMS + g;
    const long long i0 = gs * ntiles / nstreams, i1 = (gs + 1) * ntiles / nstreams;

#pragma unroll 1
    for (long long tile = i0; tile < i1 && ok; tile++) {
        const long long t = t_begin + tile * tpt + slot;
        const bool live = t < t_end;
        const long long tcl = live ? t : t_end - 1;   // rows past the end shadow the last texel and install nothing
        const int tx = (int)(tcl % L0.W), ty = (int)(tcl / L0.W);
        const int px = tx * cw + pi % cw, py = ty * ch + pi / cw;
        float* zt = z + L0.off + tcl * L0.C;
        float tt[S::NOUT];
#pragma unroll
        for (int c = 0; c < S::NOUT; c++) tt[c] = __ldg(tgt + ((long long)py * m.W + px) * S::NOUT + c);
        // the row's features; only level 0 changes between channels (the winners installed so far), so with a second
        // level its features and the position are gathered once per tile
        float fb[S::NIN];
        Tap tap0{};
        if constexpr (LY::NLEV == 2) {
            layout_features<LY>(m, z, px, py, fb);
            tap0 = level_tap(L0, pix_u(m, px), pix_v(m, py));
        }
#pragma unroll 1
        for (int c = 0; c < LY::C0; c++) {
            // X = this row's features with channel c set to candidate k
            {
                float f[S::NIN];
                if constexpr (LY::NLEV == 2) {
#pragma unroll
                    for (int i = 0; i < S::NIN; i++) f[i] = fb[i];
                    if (c > 0) sample_level_c<LY::C0>(L0, z + L0.off, tap0, f);
                } else {
                    layout_features<LY>(m, z, px, py, f);
                }
#pragma unroll
                for (int i = 0; i < LY::C0; i++) if (i == c) f[i] = gv[k];
                float x[T::K1];
#pragma unroll
                for (int i = 0; i < T::K1; i++) x[i] = i < S::NIN ? f[i] : (i == S::NIN ? 1.0f : 0.0f);
                store_split<T::K1>(trow, T::cX, x);
            }
            tc::wait_st();
            tc::fence_before_sync();
            ok = stream_sync_and(bar_id, ok);
            if (!ok) break;
            if (warp == issuer) issue_layer1<T>(tbase, tb, sb, bar);
            float h[S::H1 > T::D2COLS ? S::H1 : T::D2COLS];
            wait_mma();
            load_acc<S::H1>(trow, T::cL1, h);
            tc::wait_ld();
            relu2<S::H1>(h);
            store_split<T::K2>(trow, T::cH, h);
            tc::wait_st();
            tc::fence_before_sync();
            ok = stream_sync_and(bar_id, ok);
            if (!ok) break;
            if (warp == issuer) issue_layer2<T>(tbase, tb, sb, bar);
            wait_mma();
            load_acc<T::L3TC ? S::H2 : T::D2COLS>(trow, T::cD, h);
            tc::wait_ld();
            const float e = out_layer_error<S, CLAMP>(m, sw, h, tt, leak);
            // candidate k's cell loss: its pixels' errors in raster order (rows pi = 0, 1, ...), in double
            double loss = (double)e;
            for (int j = 1; j < cellpix; j++) loss += (double)__shfl_down_sync(0xffffffffu, e, j);
            // the reference's choice: the smallest loss among k != cur (ties to the smaller k) wins if below loss[cur]
            const int cur = qat_index(zt[c], bits);
            const double lcur = __shfl_sync(0xffffffffu, loss, group + cur * cellpix);
            const bool cand = pi == 0 && k != cur;
            double best = cand ? loss : 0.0;
            int bk = cand ? k : n;
            for (int o = cellpix; o < rpt; o <<= 1) {
                const double ob = __shfl_xor_sync(0xffffffffu, best, o);
                const int okk = __shfl_xor_sync(0xffffffffu, bk, o);
                if (okk < n && (bk >= n || ob < best || (ob == best && okk < bk))) { best = ob; bk = okk; }
            }
            const int win = (bk < n && best < lcur) ? bk : cur;
            __syncwarp();
            if (live && local == 0) zt[c] = gv[win];
            __syncwarp();
        }
    }
    if (!ok) {
        if (tid == 0) atomicExch(err, 1);
        tc::mbar_wait_bounded(bar, waited & 1u, kTcWaitPolls);
    }
    tc::fence_before_sync();
    __syncthreads();
    if (threadIdx.x < 32) { tc::fence_after_sync(); tc::tmem_dealloc(tbase, kTmemCols); }
}

template <class S>
bool launch_qat_tc_shape(cudaStream_t s, const DevModel& m, const float* w, float* zdec, const float* tgt, const float* qgrid,
                         int bits, int cw, int ch, long long t_begin, long long t_end, int* err) {
    using T = TcShape<S>;
    using LY = typename LayoutForNin<S::NIN>::type;
    if constexpr (std::is_void_v<LY>) {
        return false;
    } else {
        if (!LY::matches(m) || !m.lv[0].nearest) return false;
        const int rpt = (1 << bits) * cw * ch;
        if (bits < 1 || cw < 1 || ch < 1 || rpt > 32 || (rpt & (rpt - 1)) != 0) return false;
        const size_t smem = (size_t)T::SIGN * sizeof(float);
        const int tpt = kTcRows / rpt;
        const long long ntiles = (t_end - t_begin + tpt - 1) / tpt;
        const int blocks = (int)std::min<long long>(device_sm_count(), (ntiles + T::STREAMS - 1) / T::STREAMS);
        auto go = [&](auto kernel) {
            ensure_dynamic_smem((const void*)kernel, (int)smem);
            kernel<<<blocks, T::TPB, smem, s>>>(m, w, zdec, tgt, qgrid, bits, cw, ch, t_begin, t_end, err);
        };
        if (m.clamp_out) go(k_qat_tc<S, LY, true>); else go(k_qat_tc<S, LY, false>);
        return true;
    }
}

template <class S>
void launch_lat_tc(cudaStream_t s, const DevModel& m, const float* w, const float* zdec, const float* eps, long long nz,
                   const float* tgt, int K, unsigned active, float sg, float inv_px, float* dpix, long long p_begin,
                   long long p_end, long long pstride, int* err) {
    using T = TcShape<S>;
    const size_t smem = (size_t)T::SIGN * sizeof(float);
    using LY = typename LayoutForNin<S::NIN>::type;
    const int nsm = device_sm_count();
    const long long items = (long long)K * ((p_end - p_begin + kTcRows - 1) / kTcRows);
    const int grid = (int)std::min<long long>(nsm, (items + T::STREAMS - 1) / T::STREAMS);
    auto go = [&](auto kernel) {
        ensure_dynamic_smem((const void*)kernel, (int)smem);
        kernel<<<grid, T::TPB, smem, s>>>(m, w, zdec, eps, nz, tgt, K, active, sg, inv_px, dpix, p_begin, p_end, pstride, err);
    };
    if constexpr (!std::is_void_v<LY>) {
        if (LY::matches(m)) {
            if (m.clamp_out) go(k_lat_eval_tc<S, LY, true>); else go(k_lat_eval_tc<S, LY, false>);
            return;
        }
    }
    if (m.clamp_out) go(k_lat_eval_tc<S, void, true>); else go(k_lat_eval_tc<S, void, false>);
}

}  // namespace

int pop_tc_rows() { return kTcRows; }

bool launch_pop_eval_tc(cudaStream_t s, int shape, const DevModel& m, const PopArgs& a) {
    if (a.ncand <= 0) return true;
    if (a.chunk % kTcRows != 0 || a.tc_err == nullptr) return false;
    switch (shape) {
#define NTCB_CASE(ID, NIN, H1, H2, NOUT) case ID: launch_tc<FixedShape<NIN, H1, H2, NOUT>>(s, m, a); break;
        NTCB_FIXED_SHAPES(NTCB_CASE)
#undef NTCB_CASE
        default: return false;
    }
    NTCB_CHECK(cudaGetLastError());
    return true;
}

bool launch_qat_tc(cudaStream_t s, int shape, const DevModel& m, const float* w, float* zdec, const float* tgt, const float* grid,
                   int bits, int cw, int ch, long long t_begin, long long t_end, int* err) {
    if (t_end <= t_begin) return true;
    if (err == nullptr) return false;
    bool done = false;
    switch (shape) {
#define NTCB_CASE(ID, NIN, H1, H2, NOUT) case ID: done = launch_qat_tc_shape<FixedShape<NIN, H1, H2, NOUT>>(s, m, w, zdec, tgt, grid, bits, cw, ch, t_begin, t_end, err); break;
        NTCB_FIXED_SHAPES(NTCB_CASE)
#undef NTCB_CASE
        default: return false;
    }
    if (done) NTCB_CHECK(cudaGetLastError());
    return done;
}

bool launch_lat_eval_tc(cudaStream_t s, int shape, const DevModel& m, const float* w, const float* zdec, const float* eps,
                        long long nz, const float* tgt, int K, unsigned active_mask, float sg, float inv_px, float* dpix,
                        long long p_begin, long long p_end, long long pstride, int* err) {
    if (p_end <= p_begin || K <= 0) return true;
    if (err == nullptr) return false;
    switch (shape) {
#define NTCB_CASE(ID, NIN, H1, H2, NOUT) case ID: launch_lat_tc<FixedShape<NIN, H1, H2, NOUT>>(s, m, w, zdec, eps, nz, tgt, K, active_mask, sg, inv_px, dpix, p_begin, p_end, pstride, err); break;
        NTCB_FIXED_SHAPES(NTCB_CASE)
#undef NTCB_CASE
        default: return false;
    }
    NTCB_CHECK(cudaGetLastError());
    return true;
}

}  // namespace ntcb
