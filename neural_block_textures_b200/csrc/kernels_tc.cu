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
// Warp 0 issues the MMAs converged, one elected lane per instruction, with compile-time TMEM / shared
// addresses (a divergent single-thread issue loop costs ~4x more per MMA), and commits them to an mbarrier.
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
    static constexpr int K1 = round_up(S::NIN + 1, 8);
    static constexpr int N1 = round_up(S::H1, 16);
    static constexpr int K2 = S::H1;
    static constexpr int N2 = round_up(S::H2, 16);
    static constexpr int K3 = S::H2;
    static constexpr int N3 = round_up(S::NOUT, 16);
    static constexpr int NOUTP = round_up(S::NOUT, 4);
    static_assert(S::H1 % 8 == 0 && S::H2 % 8 == 0, "hidden widths must be multiples of 8");
    static_assert(N1 <= 32 && N2 <= 32 && N3 <= 16, "accumulators wider than their reserved TMEM columns");
    // shared memory, floats, per sign
    static constexpr int oB1h = 0, oB1l = oB1h + N1 * K1;
    static constexpr int oB2h = oB1l + N1 * K1, oB2l = oB2h + N2 * K2;
    static constexpr int ob1 = oB2l + N2 * K2;                 // b1 [H2]
    static constexpr int oW2 = round_up(ob1 + S::H2, 4);      // W2 [NOUT][H2], the reference's row-major order
    static constexpr int ob2 = oW2 + S::NOUT * S::H2;         // b2 [NOUTP]
    static_assert(S::H2 % 4 == 0, "output-layer rows are read as float4");
    static constexpr int oB3h = round_up(ob2 + NOUTP, 4), oB3l = oB3h + N3 * K3;   // W2 as an MMA B operand
    // b1 as an extra K step of layer 2: B block [N2][8] K-major with b1 in k = 0 (hi / lo), against a constant
    // A block (column 0 = 1, columns 1-7 = 0) that every stream of the CTA shares
    static constexpr int oBbh = oB3l + N3 * K3, oBbl = oBbh + N2 * 8;
    static constexpr int SIGN = round_up(oBbl + N2 * 8, 32);
    // TMEM columns: D (layers 1 and 2), D3 (output layer), X hi / lo, H hi / lo
    // The output layer runs on the tensor core for wide outputs (12: measured 1.33 vs 1.52 ms at config 3)
    // and on the FP32 pipe for 3 outputs (0.86 vs 1.03 ms at config 2), where 16-wide MMAs are mostly padding.
    static constexpr bool L3TC = S::NOUT > 4;
    // TMEM columns of one stream: D (layers 1 and 2), D3 (tensor output layer only), X and H as A operands, each
    // split into hi / lo and interleaved by 8-column K steps ([hi 8 | lo 8] per step: one 16-column store per step)
    static constexpr int cD = 0, cD3 = 32, cX = L3TC ? 48 : 32, cH = cX + 2 * K1;
    static constexpr int COLS = cH + 2 * K2;
    // Streams per CTA: as many as the SM's TMEM holds, up to 5 (640 threads leave 102 registers per thread;
    // 4 streams is the floor the kernels were tuned at). Measured: 2 streams cost +33 % over 4.
    static constexpr int STREAMS = kTmemCols / COLS >= 5 ? 5 : 4;
    static constexpr int TPB = kTcRows * STREAMS;
    static_assert(STREAMS * COLS <= kTmemCols, "TMEM columns");
    // Layer-2 bias on the tensor core when the streams leave 8 TMEM columns for the constant block (every 3-output
    // shape); otherwise (12 outputs: all 512 columns in use) it is added in the epilogue.
    static constexpr bool B1TC = !L3TC && STREAMS * COLS + 8 <= kTmemCols;
    static constexpr int cOne = STREAMS * COLS;   // the constant block's first column (from the CTA's TMEM base)

    // Writes flat reference weight k (value w) to every place a kernel variant reads it from: MMA B operands
    // as hi / lo, biases and the row-major output layer as plain floats.
    __device__ static void store(float* sw, int k, float w) {
        const float hi = tc::tf32_hi(w), lo = w - hi;
        if (k < S::H1 * S::NIN) { const int j = k / S::NIN, i = k - j * S::NIN; sw[oB1h + kmajor(j, i, K1)] = hi; sw[oB1l + kmajor(j, i, K1)] = lo; return; }
        k -= S::H1 * S::NIN;
        if (k < S::H1) { sw[oB1h + kmajor(k, S::NIN, K1)] = hi; sw[oB1l + kmajor(k, S::NIN, K1)] = lo; return; }
        k -= S::H1;
        if (k < S::H2 * S::H1) { const int j = k / S::H1, i = k - j * S::H1; sw[oB2h + kmajor(j, i, K2)] = hi; sw[oB2l + kmajor(j, i, K2)] = lo; return; }
        k -= S::H2 * S::H1;
        if (k < S::H2) { sw[ob1 + k] = w; sw[oBbh + kmajor(k, 0, 8)] = hi; sw[oBbl + kmajor(k, 0, 8)] = lo; return; }
        k -= S::H2;
        if (k < S::NOUT * S::H2) {
            const int o = k / S::H2, j = k - o * S::H2;
            sw[oW2 + k] = w; sw[oB3h + kmajor(o, j, K3)] = hi; sw[oB3l + kmajor(o, j, K3)] = lo;
            return;
        }
        k -= S::NOUT * S::H2;
        sw[ob2 + k] = w;
    }
};

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
__device__ __forceinline__ float out_act_fast(float s, int clamp_out) {
    return clamp_out ? fminf(fmaxf(s, 0.0f), 1.0f) : rcp_approx(1.0f + __expf(-s));
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
// N (multiple of 8) accumulator columns from TMEM column c into v, in as few loads as the widths allow.
template <int N>
__device__ __forceinline__ void load_acc(uint32_t trow, int c, float* v) {
#pragma unroll
    for (int q = 0; q + 16 <= N; q += 16) tc::ld_x16p(trow + c + q, v + q);
    if constexpr (N % 16 != 0) tc::ld_x8p(trow + c + (N / 16) * 16, v + (N / 16) * 16);
}

// Output layer + weighted squared error of one row on the FP32 pipe, from the layer-2 accumulator row h
// (b1 not yet added): hidden units in pairs (packed bias, activation and products), two partial sums per
// output, float error sum over the channels.
template <class S>
__device__ __forceinline__ float out_layer_error(const DevModel& m, const float* ws, const float* h, const float* t,
                                                 float leak) {
    using T = TcShape<S>;
    float2 acc[S::NOUT];
#pragma unroll
    for (int c = 0; c < S::NOUT; c++) acc[c] = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int j = 0; j < S::H2; j += 4) {
        float2 h0, h1;
        if constexpr (T::B1TC) {   // b1 already in the accumulator
            h0 = leaky_pair(make_float2(h[j], h[j + 1]), leak);
            h1 = leaky_pair(make_float2(h[j + 2], h[j + 3]), leak);
        } else {
            const float4 b = *reinterpret_cast<const float4*>(ws + T::ob1 + j);
            h0 = leaky_pair(__fadd2_rn(make_float2(h[j], h[j + 1]), make_float2(b.x, b.y)), leak);
            h1 = leaky_pair(__fadd2_rn(make_float2(h[j + 2], h[j + 3]), make_float2(b.z, b.w)), leak);
        }
#pragma unroll
        for (int c = 0; c < S::NOUT; c++) {
            const float4 w = *reinterpret_cast<const float4*>(ws + T::oW2 + c * S::H2 + j);
            acc[c] = __ffma2_rn(make_float2(w.x, w.y), h0, acc[c]);
            acc[c] = __ffma2_rn(make_float2(w.z, w.w), h1, acc[c]);
        }
    }
    float e = 0.0f;
#pragma unroll
    for (int c = 0; c < S::NOUT; c++) {
        const float d = out_act_fast(ws[T::ob2 + c] + (acc[c].x + acc[c].y), m.clamp_out) - t[c];
        e = fmaf(m.cw[c], d * d, e);
    }
    return e;
}

// Warp 0 (converged): D = A B^T over K as 3xTF32 (lo*hi, hi*lo, hi*hi per 8-wide K step), then commit. a: the
// interleaved A operand in TMEM (K step s: hi at a + 16 s, lo at a + 16 s + 8); b_hi4 / b_lo4: the B operands' shared
// addresses shifted right by 4 (hoisted; each descriptor is then one add).
template <int K, int N>
__device__ __forceinline__ void issue3(uint32_t d, uint32_t a, uint32_t b_hi4, uint32_t b_lo4, uint64_t* bar) {
    constexpr uint32_t id = tc::idesc_tf32(kTcRows, N);
    constexpr uint32_t sbo = (uint32_t)K * 32u;
    tc::fence_after_sync();
#pragma unroll
    for (int s = 0; s < K / 8; s++) {
        if (elect_one()) tc::mma_tf32_ts(d, a + 16 * s + 8, tc::sdesc_s4(b_hi4 + 16 * s, 128, sbo), id, s > 0 ? 1u : 0u);
        if (elect_one()) tc::mma_tf32_ts(d, a + 16 * s, tc::sdesc_s4(b_lo4 + 16 * s, 128, sbo), id, 1u);
        if (elect_one()) tc::mma_tf32_ts(d, a + 16 * s, tc::sdesc_s4(b_hi4 + 16 * s, 128, sbo), id, 1u);
    }
    if (elect_one()) tc::commit(bar);
    __syncwarp();
}

// Layer 2 of a shape with B1TC: the 3xTF32 product over K, then D += 1 * b1_lo + 1 * b1_hi from the constant A
// block `one` (its lo part is zero), then commit.
template <int K, int N>
__device__ __forceinline__ void issue3_bias(uint32_t d, uint32_t a, uint32_t b_hi4, uint32_t b_lo4, uint32_t one, uint32_t bb_hi4,
                                            uint32_t bb_lo4, uint64_t* bar) {
    constexpr uint32_t id = tc::idesc_tf32(kTcRows, N);
    constexpr uint32_t sbo = (uint32_t)K * 32u;
    tc::fence_after_sync();
#pragma unroll
    for (int s = 0; s < K / 8; s++) {
        if (elect_one()) tc::mma_tf32_ts(d, a + 16 * s + 8, tc::sdesc_s4(b_hi4 + 16 * s, 128, sbo), id, s > 0 ? 1u : 0u);
        if (elect_one()) tc::mma_tf32_ts(d, a + 16 * s, tc::sdesc_s4(b_lo4 + 16 * s, 128, sbo), id, 1u);
        if (elect_one()) tc::mma_tf32_ts(d, a + 16 * s, tc::sdesc_s4(b_hi4 + 16 * s, 128, sbo), id, 1u);
    }
    if (elect_one()) tc::mma_tf32_ts(d, one, tc::sdesc_s4(bb_lo4, 128, 256), id, 1u);
    if (elect_one()) tc::mma_tf32_ts(d, one, tc::sdesc_s4(bb_hi4, 128, 256), id, 1u);
    if (elect_one()) tc::commit(bar);
    __syncwarp();
}

// Byte offset / 16 of a float offset into a weight set (every B operand block starts on a 16-byte boundary).
template <int FLOATS>
constexpr uint32_t s4() { static_assert(FLOATS % 4 == 0, "B operand blocks are 16-byte aligned"); return (uint32_t)FLOATS / 4; }

// Layer 1 of unit (A = X of the stream, B = the sign's W0 | b0 block); sb4 = the sign's weight set address >> 4.
template <class T>
__device__ __forceinline__ void issue_layer1(uint32_t tb, uint32_t sb4, uint64_t* bar) {
    issue3<T::K1, T::N1>(tb + T::cD, tb + T::cX, sb4 + s4<T::oB1h>(), sb4 + s4<T::oB1l>(), bar);
}
// Layer 2 of unit (A = H of the stream, B = the sign's W1 and b1 blocks).
template <class T>
__device__ __forceinline__ void issue_layer2(uint32_t tbase, uint32_t tb, uint32_t sb4, uint64_t* bar) {
    if constexpr (T::B1TC)
        issue3_bias<T::K2, T::N2>(tb + T::cD, tb + T::cH, sb4 + s4<T::oB2h>(), sb4 + s4<T::oB2l>(), tbase + T::cOne,
                                  sb4 + s4<T::oBbh>(), sb4 + s4<T::oBbl>(), bar);
    else
        issue3<T::K2, T::N2>(tb + T::cD, tb + T::cH, sb4 + s4<T::oB2h>(), sb4 + s4<T::oB2l>(), bar);
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
template <class S, bool L3TC>
__global__ void __launch_bounds__(TcShape<S>::TPB, 1) k_pop_eval_tc(DevModel m, PopArgs a, int chunks) {
    using T = TcShape<S>;
    constexpr int NS = T::STREAMS;
    extern __shared__ __align__(1024) float dyn[];   // [NS][2][T::SIGN]
    __shared__ __align__(8) uint64_t bars[NS];
    __shared__ __align__(8) uint64_t bars3[NS];   // output-layer commits (separate: see below)
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
    // The output-layer MMAs and the next unit's layer 1 are committed back to back. On one mbarrier both
    // phases could complete before a thread polls, leaving the barrier at the parity it waits for (it would
    // then wait for a phase nobody completes); with their own barrier, commits and waits alternate on each.
    uint64_t* bar3 = &bars3[g];

    if (threadIdx.x < 32) tc::tmem_alloc(&tbase, kTmemCols);
    if (tid == 0) { tc::mbar_init(bar, 1); tc::mbar_init(bar3, 1); tc::mbar_init_fence(); }
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
    uint32_t waited = 0, waited3 = 0;   // completed phases this thread has observed on bar / bar3
    bool ok = true;

    auto wait_mma = [&]() {
        const bool done = tc::mbar_wait_bounded(bar, waited & 1u, kTcWaitPolls);
        if (done) waited++;
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
            for (int k = tid; k < m.P; k += kTcRows) {
                float wp, wm;
                perturbed_weight(a, e, k, cand, wp, wm);
                T::store(sw, k, wp);
                T::store(sw + T::SIGN, k, wm);
            }
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
        if (warp == issuer) issue_layer1<T>(tb, sb0, bar);

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
                float h[S::H1 > S::H2 ? S::H1 : S::H2];
                // layer 1 result -> H
                wait_mma();
                load_acc<S::H1>(trow, T::cD, h);
                tc::wait_ld();
#pragma unroll
                for (int j = 0; j < S::H1; j += 2) {
                    const float2 v = leaky_pair(make_float2(h[j], h[j + 1]), leak);
                    h[j] = v.x; h[j + 1] = v.y;
                }
                store_split<T::K2>(trow, T::cH, h);
                tc::wait_st();
                tc::fence_before_sync();
                ok = stream_sync_and(bar_id, ok);
                if (!ok) break;
                if (warp == issuer) issue_layer2<T>(tbase, tb, sb, bar);
                // layer 2 result -> registers
                wait_mma();
                load_acc<S::H2>(trow, T::cD, h);
                tc::wait_ld();
                // next unit's layer 1: the other sign of this tile, or the next tile's + sign
                const bool next = sg == 0 || more;
                if constexpr (L3TC) {
                    // H2 = leaky(D2 + b1) -> TMEM; output-layer MMAs (into D3) and the next unit's layer 1
                    // (into D) go out together as two commits
#pragma unroll
                    for (int j = 0; j < S::H2; j += 4) {
                        const float4 b = *reinterpret_cast<const float4*>(ws + T::ob1 + j);
                        const float2 h0 = leaky_pair(__fadd2_rn(make_float2(h[j], h[j + 1]), make_float2(b.x, b.y)), leak);
                        const float2 h1 = leaky_pair(__fadd2_rn(make_float2(h[j + 2], h[j + 3]), make_float2(b.z, b.w)), leak);
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
                        if (next) issue_layer1<T>(tb, sg ? sb0 : sb1, bar);
                    }
                    wait_mma3();
                    float o[T::NOUTP];
#pragma unroll
                    for (int q = 0; q < T::NOUTP; q += 4) tc::ld_x4p(trow + T::cD3 + q, o + q);
                    tc::wait_ld();
                    float e = 0.0f;
#pragma unroll
                    for (int c = 0; c < S::NOUT; c++) {
                        const float d = out_act_fast(o[c] + ws[T::ob2 + c], m.clamp_out) - t[c];
                        e = fmaf(m.cw[c], d * d, e);
                    }
                    if (valid) { if (sg == 0) acc_p += (double)e; else acc_m += (double)e; }
                } else {
                    if (sg == 1 && more) {
                        store_x();
                        load_x(base + 2 * kTcRows);
                        tc::wait_st();
                    }
                    tc::fence_before_sync();
                    ok = stream_sync_and(bar_id, ok);
                    if (!ok) break;
                    if (next && warp == issuer) issue_layer1<T>(tb, sg ? sb0 : sb1, bar);
                    // output layer and error of this unit, overlapping the tensor core's next layer 1
                    const double e = valid ? (double)out_layer_error<S>(m, ws, h, t, leak) : 0.0;
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
    ensure_dynamic_smem((const void*)k_pop_eval_tc<S, kL3TC>, (int)smem);
    const long long items = (long long)a.ncand * chunks;
    const int grid = (int)std::min<long long>(nsm, (items + T::STREAMS - 1) / T::STREAMS);
    k_pop_eval_tc<S, kL3TC><<<grid, T::TPB, smem, s>>>(m, a, chunks);
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
template <class S, class LY>
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
    for (int k = threadIdx.x; k < m.P; k += T::TPB) T::store(sw, k, wg[k]);
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
        load_acc<S::H1>(trow, T::cD, h);
        tc::wait_ld();
#pragma unroll
        for (int j = 0; j < S::H1; j += 2) {
            const float2 v = leaky_pair(make_float2(h[j], h[j + 1]), leak);
            h[j] = v.x; h[j + 1] = v.y;
        }
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
        if (warp == issuer) issue_layer1<T>(tb, sb, bar);
    }
#pragma unroll 1
    for (long long item = i0; item < i1 && ok; item++) {
        const bool more = item + 1 < i1;
        float h[S::H2];
        float np[S::NIN], nm[S::NIN], nt[S::NOUT];
        // + unit
        layer1_to_layer2();
        if (!ok) break;
        if (more) gather(item + 1, np, nm, nt);    // overlaps the layer-2 MMAs
        wait_mma();
        load_acc<S::H2>(trow, T::cD, h);
        tc::wait_ld();
        store_x(fm);
        tc::wait_st();
        tc::fence_before_sync();
        ok = stream_sync_and(bar_id, ok);
        if (!ok) break;
        if (warp == issuer) issue_layer1<T>(tb, sb, bar);
        const float ep = out_layer_error<S>(m, sw, h, t, leak);
        // - unit
        layer1_to_layer2();
        if (!ok) break;
        wait_mma();
        load_acc<S::H2>(trow, T::cD, h);
        tc::wait_ld();
        if (more) { store_x(np); tc::wait_st(); }
        tc::fence_before_sync();
        ok = stream_sync_and(bar_id, ok);
        if (!ok) break;
        if (more && warp == issuer) issue_layer1<T>(tb, sb, bar);
        const float em = out_layer_error<S>(m, sw, h, t, leak);
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
    if constexpr (!std::is_void_v<LY>) {
        if (LY::matches(m)) {
            ensure_dynamic_smem((const void*)k_lat_eval_tc<S, LY>, (int)smem);
            k_lat_eval_tc<S, LY><<<grid, T::TPB, smem, s>>>(m, w, zdec, eps, nz, tgt, K, active, sg, inv_px, dpix, p_begin, p_end, pstride, err);
            return;
        }
    }
    ensure_dynamic_smem((const void*)k_lat_eval_tc<S, void>, (int)smem);
    k_lat_eval_tc<S, void><<<grid, T::TPB, smem, s>>>(m, w, zdec, eps, nz, tgt, K, active, sg, inv_px, dpix, p_begin, p_end, pstride, err);
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
