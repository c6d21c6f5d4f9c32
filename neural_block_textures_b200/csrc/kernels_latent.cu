// Latent ES (all K antithetic pairs in one pass over the image), the footprint gather of the latent
// gradient, and the exhaustive per-texel selector search of --qat.
#include "kernels.h"
#include "mlp_tile.cuh"
#include "latent_features.cuh"
#include "noise.cuh"

namespace ntcb {

namespace {
constexpr int kLatTPB = 128;
constexpr int kLatPairs = 2;            // pairs per thread: rows = 2 pairs x 2 signs
constexpr int kQatTPB = 128;
constexpr int kQatRows = 4;             // candidate values per forward tile
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

void launch_lat_noise(cudaStream_t s, uint64_t seed, int step, int K, const DevModel& m, unsigned active_mask, long long nz, float* eps) {
    for (int l = 0; l < m.nlev; l++) {
        if (!(active_mask & (1u << l))) continue;
        const long long lo = m.lv[l].off, n = (long long)m.lv[l].W * m.lv[l].H * m.lv[l].C;
        dim3 grid((unsigned)std::min<long long>(blocks_for(n, 256), 4096), (unsigned)K);
        k_lat_noise<<<grid, 256, 0, s>>>(seed, step, K, lo, lo + n, nz, eps);
        NTCB_CHECK(cudaGetLastError());
    }
}

// One thread per (pixel, group of kLatPairs pairs): the 2 x kLatPairs perturbed decodes of the pixel run
// as one register tile on the packed FP32 pipe, each latent pair's (+, -) decodes forming one row pair;
// dpix[k][p] = (e+ - e-) * inv_px with the float per-pixel error of decode_err (main.cpp:1722-1735, 2015).
// The reference launches one kernel per pair and regenerates the noise of every tap
// (cuda/ntc_cuda.cu:358-409, 1124-1144).
template <class S, int TPB>
__global__ void __launch_bounds__(TPB) k_lat_eval_fixed(DevModel m, const float* __restrict__ wg, const float* __restrict__ z,
                                                        const float* __restrict__ eps, long long nz, const float* __restrict__ tgt,
                                                        int K, unsigned active, float sg, float inv_px, float* __restrict__ dpix,
                                                        long long p_begin, long long p_end) {
    constexpr int R2 = kLatPairs;
    extern __shared__ __align__(16) float ws[];
    load_weights_x2<S>(wg, m.P, ws);
    const long long npix = (long long)m.W * m.H;
    const long long p = p_begin + (long long)blockIdx.x * TPB + threadIdx.x;
    const long long pc = p < p_end ? p : p_end - 1;
    const int px = (int)(pc % m.W), py = (int)(pc / m.W);
    const int k0 = blockIdx.y * kLatPairs;
    float2 x[R2][S::NIN];
#pragma unroll
    for (int q = 0; q < R2; q++) {
        const int k = min(k0 + q, K - 1);
        float fp[kMaxIn], fm[kMaxIn];
        perturbed_features_pm(m, z, eps + (long long)k * nz, active, sg, px, py, fp, fm);
#pragma unroll
        for (int i = 0; i < S::NIN; i++) x[q][i] = make_float2(fp[i], fm[i]);
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
        if (k < K) dpix[(long long)k * npix + p] = (ep - em) * inv_px;
    }
}

__global__ void k_lat_eval_generic(DevModel m, const float* __restrict__ wg, const float* __restrict__ z, const float* __restrict__ eps,
                                   long long nz, const float* __restrict__ tgt, int K, unsigned active, float sg, float inv_px,
                                   float* __restrict__ dpix, long long p_begin, long long p_end) {
    extern __shared__ __align__(16) float ws[];
    for (int k = threadIdx.x; k < m.P; k += blockDim.x) ws[k] = wg[k];
    __syncthreads();
    const long long npix = (long long)m.W * m.H;
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
    dpix[(long long)k * npix + p] = (ep - em) * inv_px;
}

void launch_lat_eval(cudaStream_t s, int shape, const DevModel& m, const float* w, const float* zdec, const float* eps,
                     long long nz, const float* tgt, int K, unsigned active_mask, float sg, float inv_px, float* dpix,
                     long long p_begin, long long p_end) {
    const long long n = p_end - p_begin;
    if (n <= 0) return;
    switch (shape) {
#define NTCB_CASE(ID, NIN, H1, H2, NOUT) case ID: { using S = FixedShape<NIN, H1, H2, NOUT>; \
        dim3 grid(blocks_for(n, kLatTPB), (unsigned)((K + kLatPairs - 1) / kLatPairs)); \
        k_lat_eval_fixed<S, kLatTPB><<<grid, kLatTPB, 2 * S::SIZE * sizeof(float), s>>>(m, w, zdec, eps, nz, tgt, K, active_mask, sg, inv_px, dpix, \
                                                                                     p_begin, p_end); break; }
        NTCB_FIXED_SHAPES(NTCB_CASE)
#undef NTCB_CASE
        default: {
            dim3 grid(blocks_for(n, 128), (unsigned)K);
            k_lat_eval_generic<<<grid, 128, m.P * sizeof(float), s>>>(m, w, zdec, eps, nz, tgt, K, active_mask, sg, inv_px, dpix, p_begin, p_end);
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
__global__ void k_lat_gather(DevModel m, int level, const int* __restrict__ xr, const int* __restrict__ yr, const float* __restrict__ dpix,
                             const float* __restrict__ eps, long long nz, int K, float scale, RateTerm rate, float* __restrict__ grad) {
    const DevLevel& L = m.lv[level];
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (long long)L.W * L.H) return;
    const int tx = (int)(t % L.W), ty = (int)(t / L.W);
    const int x0 = xr[tx], x1 = xr[L.W + tx], y0 = yr[ty], y1 = yr[L.H + ty];
    const long long npix = (long long)m.W * m.H;
    const long long base = L.off + t * L.C;
    for (int k = 0; k < K; k++) {
        float d = 0.0f;
        const float* dp = dpix + (long long)k * npix;
        for (int py = y0; py < y1; py++)
            for (int px = x0; px < x1; px++) d += dp[(long long)py * m.W + px];
        const float w = d * scale;
        const float* ek = eps + (long long)k * nz;
        for (int c = 0; c < L.C; c++) grad[base + c] = fmaf(w, ek[base + c], grad[base + c]);
        if (rate.dbits) {
            const long long b = (long long)(ty / 8) * rate.BW + tx / 8;
            const int* db = rate.dbits + (long long)k * ((long long)(m.H / 8) * rate.BW * rate.C);
            for (int c = 0; c < L.C; c++)
                grad[base + c] = fmaf(rate.rate_scale * (float)db[b * rate.C + c] * scale, ek[base + c], grad[base + c]);
        }
    }
}

void launch_lat_gather(cudaStream_t s, const DevModel& m, int level, const int* xr, const int* yr, const float* dpix,
                       const float* eps, long long nz, int K, float scale, const RateTerm& rate, float* grad) {
    const long long ntx = (long long)m.lv[level].W * m.lv[level].H;
    k_lat_gather<<<blocks_for(ntx, 128), 128, 0, s>>>(m, level, xr, yr, dpix, eps, nz, K, scale, rate, grad);
    NTCB_CHECK(cudaGetLastError());
}

// ------------------------------------------------------------------ --qat selector search
// qat_index (main.cpp:2060-2064): the grid index of an on-grid value, lround((v + 1) / 2 * levels), clamped.
__device__ __forceinline__ int qat_index(float v, int bits) {
    const int levels = (1 << bits) - 1;
    const int k = (int)lroundf((v + 1.0f) * 0.5f * (float)levels);
    return max(0, min(levels, k));
}

// qat_search (main.cpp:2088-2139), one thread per level-0 texel: channels in order; for channel c every grid
// value's cell loss (double, pixels in raster order) is computed — kQatRows candidates per forward tile —
// then the reference's rule picks the winner: the current value first, any other value only if strictly
// lower. The winner is written in place before the next channel is searched.
// The rule is applied as the losses stream in: the first strict minimum over the other grid values (index
// order), which wins only if it is below the current value's loss — the same choice as the reference's scan
// (best = loss[current]; for k != current in order: if loss[k] < best take it), with no per-value array.
template <class S, int TPB>
__global__ void __launch_bounds__(TPB) k_qat_fixed(DevModel m, const float* __restrict__ wg, float* __restrict__ z,
                                                   const float* __restrict__ tgt, const int* __restrict__ xr,
                                                   const int* __restrict__ yr, const float* __restrict__ grid,
                                                   const int* __restrict__ bits_c, long long t_begin, long long t_end) {
    constexpr int R = kQatRows, R2 = kQatRows / 2;
    extern __shared__ __align__(16) float ws[];
    load_weights_x2<S>(wg, m.P, ws);
    const DevLevel& L = m.lv[0];
    const long long t = t_begin + (long long)blockIdx.x * TPB + threadIdx.x;
    if (t >= t_end) return;   // no barrier below
    const int tx = (int)(t % L.W), ty = (int)(t / L.W);
    const int x0 = xr[tx], x1 = xr[L.W + tx], y0 = yr[ty], y1 = yr[L.H + ty];
    if (x0 >= x1 || y0 >= y1) return;
    float* zt = z + L.off + t * L.C;
    for (int c = 0; c < L.C; c++) {
        const int bits = bits_c[c], n = 1 << bits;
        const float* gv = grid + bits * 257;
        const int cur = qat_index(zt[c], bits);
        double cur_loss = 0.0, other = 0.0;
        int other_k = -1;
        for (int kg = 0; kg < n; kg += R) {
            double acc[R];
#pragma unroll
            for (int r = 0; r < R; r++) acc[r] = 0.0;
            for (int py = y0; py < y1; py++)
                for (int px = x0; px < x1; px++) {
                    float f[kMaxIn];
                    pixel_features(m, z, px, py, f);
                    float2 x[R2][S::NIN];
#pragma unroll
                    for (int h = 0; h < R2; h++) {
                        const float va = gv[min(kg + 2 * h, n - 1)], vb = gv[min(kg + 2 * h + 1, n - 1)];
#pragma unroll
                        for (int i = 0; i < S::NIN; i++) x[h][i] = (i == c) ? make_float2(va, vb) : make_float2(f[i], f[i]);
                    }
                    float2 o[R2][S::NOUT];
                    fixed_forward_x2<S, R2>(ws, x, o, m.leak, m.clamp_out);
                    const float* tp = tgt + ((long long)py * m.W + px) * S::NOUT;
#pragma unroll
                    for (int h = 0; h < R2; h++)
#pragma unroll
                        for (int q = 0; q < S::NOUT; q++) {
                            const float da = o[h][q].x - tp[q], db = o[h][q].y - tp[q];
                            acc[2 * h] += (double)(m.cw[q] * (da * da));
                            acc[2 * h + 1] += (double)(m.cw[q] * (db * db));
                        }
                }
#pragma unroll
            for (int r = 0; r < R; r++) {
                const int k = kg + r;
                if (k >= n) continue;
                if (k == cur) cur_loss = acc[r];
                else if (other_k < 0 || acc[r] < other) { other = acc[r]; other_k = k; }
            }
        }
        zt[c] = gv[(other_k >= 0 && other < cur_loss) ? other_k : cur];
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

void launch_qat(cudaStream_t s, int shape, const DevModel& m, const float* w, float* zdec, const float* tgt,
                const int* xr0, const int* yr0, const float* grid, const int* bits, long long t_begin, long long t_end) {
    const long long ntx = t_end - t_begin;
    if (ntx <= 0) return;
    switch (shape) {
#define NTCB_CASE(ID, NIN, H1, H2, NOUT) case ID: { using S = FixedShape<NIN, H1, H2, NOUT>; \
        k_qat_fixed<S, kQatTPB><<<blocks_for(ntx, kQatTPB), kQatTPB, 2 * S::SIZE * sizeof(float), s>>>(m, w, zdec, tgt, xr0, yr0, grid, bits, \
                                                                                                      t_begin, t_end); break; }
        NTCB_FIXED_SHAPES(NTCB_CASE)
#undef NTCB_CASE
        default: k_qat_generic<<<blocks_for(ntx, 128), 128, m.P * sizeof(float), s>>>(m, w, zdec, tgt, xr0, yr0, grid, bits, t_begin, t_end);
    }
    NTCB_CHECK(cudaGetLastError());
}

}  // namespace ntcb
