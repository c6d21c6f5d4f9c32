// Latent ES (all K antithetic pairs in one pass over the image), the footprint gather of the latent
// gradient, and the exhaustive per-texel selector search of --qat.
#include "adam.cuh"
#include "kernels.h"
#include "mlp_tile.cuh"
#include "fixed_layout.cuh"
#include "latent_features.cuh"
#include "noise.cuh"

#include <type_traits>
#include "quant.cuh"

namespace ntcb {

namespace {
constexpr int kLatTPB = 128;
constexpr int kLatPairs = 2;            // pairs per thread: rows = 2 pairs x 2 signs
constexpr int kQatTPB = 128;
inline unsigned blocks_for(long long n, int tpb) { return (unsigned)((n + tpb - 1) / tpb); }
}  // namespace

// eps[k][i] = gauss(seed, latent stream, step, k, i) for every flat index i of every ES-perturbed level
// (LatentTrainer::step, main.cpp:1990-2001: one epsilon over the flat vector, keyed by the flat index).
__global__ void k_lat_noise(uint64_t seed, int step, int K, long long lo, long long hi, long long nz, float* __restrict__ eps) {
    const int k = blockIdx.y;
    const uint64_t key = stream_key(seed, kStreamLatent, (uint32_t)step, (uint32_t)k);
    for (long long i = lo + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < hi; i += (long long)gridDim.x * blockDim.x)
        eps[(long long)k * nz + i] = gauss_at(key, (uint64_t)i);
}

void launch_lat_noise_range(cudaStream_t s, uint64_t seed, int step, int K, long long lo, long long hi, long long nz, float* eps) {
    if (hi <= lo) return;
    dim3 grid((unsigned)std::min<long long>(blocks_for(hi - lo, 256), 4096), (unsigned)K);
    k_lat_noise<<<grid, 256, 0, s>>>(seed, step, K, lo, hi, nz, eps);
    NTCB_CHECK(cudaGetLastError());
}
void launch_lat_noise(cudaStream_t s, uint64_t seed, int step, int K, const DevModel& m, unsigned active_mask, long long nz, float* eps) {
    for (int l = 0; l < m.nlev; l++) {
        if (!(active_mask & (1u << l))) continue;
        const long long lo = m.lv[l].off, n = (long long)m.lv[l].W * m.lv[l].H * m.lv[l].C;
        launch_lat_noise_range(s, seed, step, K, lo, lo + n, nz, eps);
    }
}

// One thread per (pixel, group of kLatPairs pairs): the 2 x kLatPairs perturbed decodes of the pixel run
// as one register tile on the packed FP32 pipe, each latent pair's (+, -) decodes forming one row pair;
// dpix[k][p] = (e+ - e-) * inv_px with the float per-pixel error of decode_err (main.cpp:1722-1735, 2015).
// The reference launches one kernel per pair and regenerates the noise of every tap
// (cuda/ntc_cuda.cu:358-409, 1124-1144).
template <class S, int TPB, class LY>
__global__ void __launch_bounds__(TPB) k_lat_eval_fixed(DevModel m, const float* __restrict__ wg, const float* __restrict__ z,
                                                        const float* __restrict__ eps, long long nz, const float* __restrict__ tgt,
                                                        int K, unsigned active, float sg, float inv_px, float* __restrict__ dpix,
                                                        long long p_begin, long long p_end, long long pstride) {
    constexpr int R2 = kLatPairs;
    extern __shared__ __align__(16) float ws[];
    load_weights_x2<S>(wg, m.P, ws);
    const long long p = p_begin + (long long)blockIdx.x * TPB + threadIdx.x;
    const long long pc = p < p_end ? p : p_end - 1;
    const int px = (int)(pc % m.W), py = (int)(pc / m.W);
    const int k0 = blockIdx.y * kLatPairs;
    float2 x[R2][S::NIN];
#pragma unroll
    for (int q = 0; q < R2; q++) {
        const int k = min(k0 + q, K - 1);
        if constexpr (std::is_void_v<LY>) {
            float fp[kMaxIn], fm[kMaxIn];
            perturbed_features_pm(m, z, eps + (long long)k * nz, active, sg, px, py, fp, fm);
#pragma unroll
            for (int i = 0; i < S::NIN; i++) x[q][i] = make_float2(fp[i], fm[i]);
        } else {
            float fp[S::NIN], fm[S::NIN];
            layout_features_pm<LY>(m, z, eps + (long long)k * nz, active, sg, px, py, fp, fm);
#pragma unroll
            for (int i = 0; i < S::NIN; i++) x[q][i] = make_float2(fp[i], fm[i]);
        }
    }
    float2 o[R2][S::NOUT];
    fixed_forward_x2<S, R2>(ws, x, o, m.leak, m.clamp_out);
    if (p >= p_end) return;
    const float* t = tgt + pc * S::NOUT;
    float tv[S::NOUT];
#pragma unroll
    for (int c = 0; c < S::NOUT; c++) tv[c] = t[c];
#pragma unroll
    for (int q = 0; q < R2; q++) {
        const int k = k0 + q;
        float ep = 0.0f, em = 0.0f;
#pragma unroll
        for (int c = 0; c < S::NOUT; c++) {
            const float dp = o[q][c].x - tv[c], dm = o[q][c].y - tv[c];
            ep += m.cw[c] * (dp * dp);
            em += m.cw[c] * (dm * dm);
        }
        if (k < K) dpix[(long long)k * pstride + (p - p_begin)] = (ep - em) * inv_px;
    }
}

__global__ void k_lat_eval_generic(DevModel m, const float* __restrict__ wg, const float* __restrict__ z, const float* __restrict__ eps,
                                   long long nz, const float* __restrict__ tgt, int K, unsigned active, float sg, float inv_px,
                                   float* __restrict__ dpix, long long p_begin, long long p_end, long long pstride) {
    extern __shared__ __align__(16) float ws[];
    for (int k = threadIdx.x; k < m.P; k += blockDim.x) ws[k] = wg[k];
    __syncthreads();
    const long long p = p_begin + (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const int k = blockIdx.y;
    if (p >= p_end) return;
    const int px = (int)(p % m.W), py = (int)(p / m.W);
    float f[kMaxIn], o[kMaxOut];
    const float* t = tgt + p * m.nout;
    perturbed_features(m, z, eps + (long long)k * nz, active, sg, px, py, f);
    generic_forward(m, ws, f, o);
    const float ep = pixel_err_f(m, o, t);
    perturbed_features(m, z, eps + (long long)k * nz, active, -sg, px, py, f);
    generic_forward(m, ws, f, o);
    const float em = pixel_err_f(m, o, t);
    dpix[(long long)k * pstride + (p - p_begin)] = (ep - em) * inv_px;
}

template <class S>
void launch_lat_fixed(cudaStream_t s, const DevModel& m, const float* w, const float* zdec, const float* eps, long long nz,
                      const float* tgt, int K, unsigned active_mask, float sg, float inv_px, float* dpix, long long p_begin,
                      long long p_end, long long pstride) {
    using LY = typename LayoutForNin<S::NIN>::type;
    dim3 grid(blocks_for(p_end - p_begin, kLatTPB), (unsigned)((K + kLatPairs - 1) / kLatPairs));
    const size_t smem = 2 * S::SIZE * sizeof(float);
    if constexpr (!std::is_void_v<LY>) {
        if (LY::matches(m)) {
            k_lat_eval_fixed<S, kLatTPB, LY><<<grid, kLatTPB, smem, s>>>(m, w, zdec, eps, nz, tgt, K, active_mask, sg, inv_px, dpix,
                                                                         p_begin, p_end, pstride);
            return;
        }
    }
    k_lat_eval_fixed<S, kLatTPB, void><<<grid, kLatTPB, smem, s>>>(m, w, zdec, eps, nz, tgt, K, active_mask, sg, inv_px, dpix,
                                                                   p_begin, p_end, pstride);
}

void launch_lat_eval(cudaStream_t s, int shape, const DevModel& m, const float* w, const float* zdec, const float* eps,
                     long long nz, const float* tgt, int K, unsigned active_mask, float sg, float inv_px, float* dpix,
                     long long p_begin, long long p_end, long long pstride) {
    const long long n = p_end - p_begin;
    if (n <= 0) return;
    switch (shape) {
#define NTCB_CASE(ID, NIN, H1, H2, NOUT) case ID: launch_lat_fixed<FixedShape<NIN, H1, H2, NOUT>>(s, m, w, zdec, eps, nz, tgt, K, \
        active_mask, sg, inv_px, dpix, p_begin, p_end, pstride); break;
        NTCB_FIXED_SHAPES(NTCB_CASE)
#undef NTCB_CASE
        default: {
            dim3 grid(blocks_for(n, 128), (unsigned)K);
            k_lat_eval_generic<<<grid, 128, m.P * sizeof(float), s>>>(m, w, zdec, eps, nz, tgt, K, active_mask, sg, inv_px, dpix, p_begin, p_end, pstride);
        }
    }
    NTCB_CHECK(cudaGetLastError());
}

// Footprint attribution in gather form (LatentTrainer::step, main.cpp:2009-2036): texel t of level l sums
// dpix over the pixels whose tap reads it — a rectangle [xr[tx], xr[W+tx]) x [yr[ty], yr[H+ty]) precomputed
// on the host with the reference's distinct-texel rule — in raster order, which is the order the
// reference's scatter adds them in; then grad[t, c] += (d * scale) * eps[k][t, c], pairs in order. When
// the DCT rate term is on (level 0), pair k's rate contribution follows its mse contribution
// (dct_rate_pass, main.cpp:1935-1958).
// Up to 32 texels per CTA (fewer for many pairs, to fit the sums in 48 KB of shared memory): first one thread
// per (texel, pair) sums that pair's dpix over the texel's footprint in
// raster order (each sum stays one sequential float chain, so the values are unchanged), then one thread per
// texel applies the pairs' updates in pair order. The footprint sums are latency-bound loads, so spreading
// them over the pairs' threads is what sets the speed.
__global__ void k_lat_gather(DevModel m, int level, const int* __restrict__ xr, const int* __restrict__ yr, const float* __restrict__ dpix,
                             const float* __restrict__ eps, long long nz, int K, float scale, RateTerm rate, float* __restrict__ grad,
                             int rpb, int ty0, int ty1, int row_base, int tpc, LatAdam adam) {
    extern __shared__ float dsum[];   // [tpc][K]
    const DevLevel& L = m.lv[level];
    const long long t0 = (long long)ty0 * L.W + (long long)blockIdx.x * tpc;
    const long long t_end = (long long)ty1 * L.W;
    const long long plane = (long long)rpb * m.W, block = (long long)K * plane;
    for (int j = threadIdx.x; j < tpc * K; j += blockDim.x) {
        const int tl = j % tpc, k = j / tpc;
        const long long t = t0 + tl;
        if (t >= t_end) continue;
        const int tx = (int)(t % L.W), ty = (int)(t / L.W);
        const int x0 = xr[tx], x1 = xr[L.W + tx], y0 = yr[ty], y1 = yr[L.H + ty];
        float d = 0.0f;
        for (int py = y0; py < y1; py++) {
            const int pr = py - row_base;
            const float* row = dpix + (pr / rpb) * block + k * plane + (long long)(pr % rpb) * m.W;
            int px = x0;
            // up to 16 values of the row loaded together, then added in raster order (the same float chain)
            for (; px < x1; px += 16) {
                float v[16];
#pragma unroll
                for (int j = 0; j < 16; j++) v[j] = px + j < x1 ? row[px + j] : 0.0f;
#pragma unroll
                for (int j = 0; j < 16; j++)
                    if (px + j < x1) d += v[j];
            }
        }
        dsum[tl * K + k] = d;
    }
    __syncthreads();
    const long long t = t0 + threadIdx.x;
    if ((int)threadIdx.x >= tpc || t >= t_end) return;
    const int tx = (int)(t % L.W), ty = (int)(t / L.W);
    const long long base = L.off + t * L.C;
    const long long b = (long long)(ty / 8) * rate.BW + tx / 8;
    // per channel: the pairs' terms in pair order (mse term, then its rate term), from zero — the chain the
    // reference's scatter forms on a zeroed gradient — then Adam on the texel
    for (int c = 0; c < L.C; c++) {
        float g = 0.0f;
        for (int k = 0; k < K; k++) {
            const float e = eps[(long long)k * nz + base + c];
            g = fmaf(dsum[threadIdx.x * K + k] * scale, e, g);
            if (rate.dbits) {
                const int* db = rate.dbits + (long long)k * ((long long)(m.H / 8) * rate.BW * rate.C);
                g = fmaf(rate.rate_scale * (float)db[b * rate.C + c] * scale, e, g);
            }
        }
        grad[base + c] = g;
        float th = adam.z[base + c], mm = adam.m[base + c], vv = adam.v[base + c];
        adam_update(th, g, mm, vv, adam.lr, adam.c1, adam.c2);
        adam.z[base + c] = th; adam.m[base + c] = mm; adam.v[base + c] = vv;
    }
}

void launch_lat_gather(cudaStream_t s, const DevModel& m, int level, const int* xr, const int* yr, const float* dpix,
                       const float* eps, long long nz, int K, float scale, const RateTerm& rate, float* grad,
                       int rows_per_block, int ty0, int ty1, int row_base, const LatAdam& adam) {
    const long long ntx = (long long)m.lv[level].W * (ty1 - ty0);
    if (ntx <= 0) return;
    const int tpc = std::max(1, std::min(32, 12288 / std::max(1, K)));
    k_lat_gather<<<blocks_for(ntx, tpc), 128, (size_t)tpc * K * sizeof(float), s>>>(
        m, level, xr, yr, dpix, eps, nz, K, scale, rate, grad, rows_per_block, ty0, ty1, row_base, tpc, adam);
    NTCB_CHECK(cudaGetLastError());
}

// ------------------------------------------------------------------ --qat selector search
// qat_search (main.cpp:2088-2139) for the fixed shapes: G consecutive lanes of a warp share one level-0
// texel; lane gi evaluates the candidate pairs gi, gi + G, ... (grid values 2q and 2q + 1 as one packed-FP32
// row pair). A candidate's cell loss is accumulated in double over the texel's pixels in raster order by
// one lane, as the reference does. Channels run in order and the winner is installed before the next
// channel. The reference's choice (best = loss[current]; for every other value k in order: if loss[k] <
// best take it) equals: the smallest k != current attaining the minimum of the other losses, if that
// minimum is below loss[current]; the lanes combine their (loss, k) with that rule by shuffles.
template <class S, int TPB, int G, int R2, class LY>
__global__ void __launch_bounds__(TPB, 3) k_qat_fixed(DevModel m, const float* __restrict__ wg, float* __restrict__ z,
                                                   const float* __restrict__ tgt, const int* __restrict__ xr,
                                                   const int* __restrict__ yr, const float* __restrict__ grid,
                                                   const int* __restrict__ bits_c, long long t_begin, long long t_end) {
    static_assert(G == 1 || G == 2 || G == 4 || G == 8, "lanes per texel");
    extern __shared__ __align__(16) float ws[];
    load_weights_x2<S>(wg, m.P, ws);
    const DevLevel& L = m.lv[0];
    const long long gt = (long long)blockIdx.x * TPB + threadIdx.x;
    const int gi = (int)(gt % G);
    const long long t = t_begin + gt / G;
    const bool live = t < t_end;
    const long long tc = live ? t : t_end - 1;            // dead lanes shadow a live texel and write nothing
    const int tx = (int)(tc % L.W), ty = (int)(tc / L.W);
    const int x0 = xr[tx], x1 = xr[L.W + tx], y0 = yr[ty], y1 = yr[L.H + ty];
    float* zt = z + L.off + tc * L.C;
    const unsigned gmask = (G == 1) ? 0xffffffffu : (((1u << G) - 1u) << ((threadIdx.x & 31) & ~(G - 1)));
    for (int c = 0; c < L.C; c++) {
        const int bits = bits_c[c], n = 1 << bits;
        const float* gv = grid + bits * 257;
        const int cur = qat_index(zt[c], bits);
        double cur_loss = 0.0, best = 0.0;
        int best_k = -1;
        for (int q = gi; 2 * R2 * q < n; q += G) {
            double acc[2 * R2];
#pragma unroll
            for (int r = 0; r < 2 * R2; r++) acc[r] = 0.0;
#pragma unroll 1
            for (int py = y0; py < y1; py++)
#pragma unroll 1
                for (int px = x0; px < x1; px++) {
                    // keeps the weight loads of the forward inside the loop (hoisted, they exhaust the registers)
                    asm volatile("" ::: "memory");
                    float f[S::NIN];
                    if constexpr (std::is_void_v<LY>) {
                        float fr[kMaxIn];
                        pixel_features(m, z, px, py, fr);
#pragma unroll
                        for (int i = 0; i < S::NIN; i++) f[i] = fr[i];
                    } else {
                        layout_features<LY>(m, z, px, py, f);   // registers: the layout is known at compile time
                    }
                    float2 x[R2][S::NIN];
#pragma unroll
                    for (int h = 0; h < R2; h++) {
                        const float va = gv[min(2 * R2 * q + 2 * h, n - 1)], vb = gv[min(2 * R2 * q + 2 * h + 1, n - 1)];
#pragma unroll
                        for (int i = 0; i < S::NIN; i++) x[h][i] = (i == c) ? make_float2(va, vb) : make_float2(f[i], f[i]);
                    }
                    float2 o[R2][S::NOUT];
                    fixed_forward_x2<S, R2>(ws, x, o, m.leak, m.clamp_out);
                    const float* tp = tgt + ((long long)py * m.W + px) * S::NOUT;
#pragma unroll
                    for (int h = 0; h < R2; h++)
#pragma unroll
                        for (int k = 0; k < S::NOUT; k++) {
                            const float da = o[h][k].x - tp[k], db = o[h][k].y - tp[k];
                            acc[2 * h] += (double)(m.cw[k] * (da * da));
                            acc[2 * h + 1] += (double)(m.cw[k] * (db * db));
                        }
                }
#pragma unroll
            for (int r = 0; r < 2 * R2; r++) {
                const int k = 2 * R2 * q + r;
                if (k >= n) continue;
                const double lk = acc[r];
                if (k == cur) cur_loss = lk;
                else if (best_k < 0 || lk < best) { best = lk; best_k = k; }
            }
        }
        if (G > 1) {
            // combine: smaller loss wins, equal losses go to the smaller index (the first in scan order)
#pragma unroll
            for (int o = 1; o < G; o <<= 1) {
                const double ob = __shfl_xor_sync(gmask, best, o);
                const int ok = __shfl_xor_sync(gmask, best_k, o);
                if (ok >= 0 && (best_k < 0 || ob < best || (ob == best && ok < best_k))) { best = ob; best_k = ok; }
            }
            const int owner = (cur / (2 * R2)) % G;
            cur_loss = __shfl_sync(gmask, cur_loss, ((threadIdx.x & 31) & ~(G - 1)) + owner);
        }
        const float win = gv[(best_k >= 0 && best < cur_loss) ? best_k : cur];
        if (live && gi == 0) zt[c] = win;
        __syncwarp(gmask);
    }
}

__global__ void k_qat_generic(DevModel m, const float* __restrict__ wg, float* __restrict__ z, const float* __restrict__ tgt,
                              const int* __restrict__ xr, const int* __restrict__ yr, const float* __restrict__ grid,
                              const int* __restrict__ bits_c, long long t_begin, long long t_end) {
    extern __shared__ __align__(16) float ws[];
    for (int k = threadIdx.x; k < m.P; k += blockDim.x) ws[k] = wg[k];
    __syncthreads();
    const DevLevel& L = m.lv[0];
    const long long t = t_begin + (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= t_end) return;
    const int tx = (int)(t % L.W), ty = (int)(t / L.W);
    const int x0 = xr[tx], x1 = xr[L.W + tx], y0 = yr[ty], y1 = yr[L.H + ty];
    if (x0 >= x1 || y0 >= y1) return;
    float* zt = z + L.off + t * L.C;
    for (int c = 0; c < L.C; c++) {
        const int bits = bits_c[c], levels = (1 << bits) - 1;
        const float* gv = grid + bits * 257;
        auto cell_loss = [&](float val) {
            double sum = 0.0;
            for (int py = y0; py < y1; py++)
                for (int px = x0; px < x1; px++) {
                    float f[kMaxIn], o[kMaxOut];
                    pixel_features(m, z, px, py, f);
                    f[c] = val;
                    generic_forward(m, ws, f, o);
                    sum += pixel_err_d(m, o, tgt + ((long long)py * m.W + px) * m.nout);
                }
            return sum;
        };
        int best_k = qat_index(zt[c], bits);
        double best = cell_loss(gv[best_k]);
        for (int k = 0; k <= levels; k++) {
            if (k == best_k) continue;
            const double sk = cell_loss(gv[k]);
            if (sk < best) { best = sk; best_k = k; }
        }
        zt[c] = gv[best_k];
    }
}

// The selector search's exchange carries level 0 as grid indices, one byte per value: every value of a searched row
// is a grid value of its channel (qat_index recovers its index exactly and the grid table gives the value back), a
// quarter of the float bytes on the wire.
__global__ void k_qat_pack(const float* __restrict__ z0, long long n, int C, const int* __restrict__ bits, uint8_t* __restrict__ out) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = (uint8_t)qat_index(z0[i], bits[(int)(i % C)]);
}
__global__ void k_qat_unpack(const uint8_t* __restrict__ in, long long blk, long long n, int world, int C, const int* __restrict__ bits,
                             const float* __restrict__ grid, float* __restrict__ z0) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * world) return;
    const long long q = i / n, j = i - q * n;
    z0[i] = grid[bits[(int)(j % C)] * 257 + in[q * blk + j]];
}
void launch_qat_pack(cudaStream_t s, const float* z0, long long n, int C, const int* bits, uint8_t* out) {
    if (n <= 0) return;
    k_qat_pack<<<blocks_for(n, 256), 256, 0, s>>>(z0, n, C, bits, out);
    NTCB_CHECK(cudaGetLastError());
}
void launch_qat_unpack(cudaStream_t s, const uint8_t* in, long long blk, long long n, int world, int C, const int* bits,
                       const float* grid, float* z0) {
    if (n <= 0) return;
    k_qat_unpack<<<blocks_for(n * world, 256), 256, 0, s>>>(in, blk, n, world, C, bits, grid, z0);
    NTCB_CHECK(cudaGetLastError());
}

template <class S, int G, int R2>
void launch_qat_fixed(cudaStream_t s, const DevModel& m, const float* w, float* zdec, const float* tgt, const int* xr0,
                      const int* yr0, const float* grid, const int* bits, long long t_begin, long long t_end) {
    using LY = typename LayoutForNin<S::NIN>::type;
    const long long lanes = (t_end - t_begin) * G;
    const size_t smem = 2 * S::SIZE * sizeof(float);
    if constexpr (!std::is_void_v<LY>) {
        if (LY::matches(m)) {
            k_qat_fixed<S, kQatTPB, G, R2, LY><<<blocks_for(lanes, kQatTPB), kQatTPB, smem, s>>>(m, w, zdec, tgt, xr0, yr0, grid, bits,
                                                                                                t_begin, t_end);
            return;
        }
    }
    k_qat_fixed<S, kQatTPB, G, R2, void><<<blocks_for(lanes, kQatTPB), kQatTPB, smem, s>>>(m, w, zdec, tgt, xr0, yr0, grid, bits,
                                                                                          t_begin, t_end);
}

void launch_qat(cudaStream_t s, int shape, const DevModel& m, const float* w, float* zdec, const float* tgt,
                const int* xr0, const int* yr0, const float* grid, const int* bits, long long t_begin, long long t_end,
                int max_bits) {
    const long long ntx = t_end - t_begin;
    if (ntx <= 0) return;
    // 3 outputs: one lane per texel with 4 candidates per tile (measured 1.72 ms at config 5 against 1.92 ms
    // for 2 lanes x 2); 12 outputs: the wider output layer leaves room for one candidate pair per lane and up
    // to 4 lanes per texel (0.19 ms against 0.27 ms at config 3).
    const int G = max_bits <= 1 ? 1 : (max_bits == 2 ? 2 : 4);
    switch (shape) {
#define NTCB_CASE(ID, NIN, H1, H2, NOUT) case ID: { using S = FixedShape<NIN, H1, H2, NOUT>; \
        if constexpr (NOUT <= 4) launch_qat_fixed<S, 1, 2>(s, m, w, zdec, tgt, xr0, yr0, grid, bits, t_begin, t_end); \
        else if (G == 1) launch_qat_fixed<S, 1, 1>(s, m, w, zdec, tgt, xr0, yr0, grid, bits, t_begin, t_end); \
        else if (G == 2) launch_qat_fixed<S, 2, 1>(s, m, w, zdec, tgt, xr0, yr0, grid, bits, t_begin, t_end); \
        else launch_qat_fixed<S, 4, 1>(s, m, w, zdec, tgt, xr0, yr0, grid, bits, t_begin, t_end); \
        break; }
        NTCB_FIXED_SHAPES(NTCB_CASE)
#undef NTCB_CASE
        default: k_qat_generic<<<blocks_for(ntx, 128), 128, m.P * sizeof(float), s>>>(m, w, zdec, tgt, xr0, yr0, grid, bits, t_begin, t_end);
    }
    NTCB_CHECK(cudaGetLastError());
}

}  // namespace ntcb
