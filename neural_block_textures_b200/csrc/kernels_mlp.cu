// MLP population kernels: minibatch draw, ES noise, population evaluation (ES pairs and FD
// candidates), fitness reduction, ES gradient + Adam, full-image decode.
#include "adam.cuh"
#include "kernels.h"
#include "mlp_tile.cuh"
#include "noise.cuh"
#include "pop_common.cuh"

namespace ntcb {

namespace {

constexpr int kPopTPB = 128;   // threads per population CTA
constexpr int kPopRows = 4;    // rows (pixels) per thread in the fixed-shape population kernel
constexpr int kDecTPB = 128;
constexpr int kDecRows = 4;

inline unsigned blocks_for(long long n, int tpb) { return (unsigned)((n + tpb - 1) / tpb); }

}  // namespace

int shape_id(const DevModel& m) {
#define NTCB_MATCH(ID, NIN, H1, H2, NOUT) if (FixedShape<NIN, H1, H2, NOUT>::matches(m)) return ID;
    NTCB_FIXED_SHAPES(NTCB_MATCH)
#undef NTCB_MATCH
    return 0;
}

int pop_chunk_rows(int shape) { return shape ? kPopTPB * kPopRows : kPopTPB; }
int pop_chunks(int M, int chunk) { return (M + chunk - 1) / chunk; }

// ------------------------------------------------------------------ minibatch
// MlpTrainer::draw_batch (main.cpp:1825-1833, hash branch) + the feature / target rows the population
// kernel reads: slot s draws pixel uniform_below(u32(seed, batch stream, it, 0, s), W H). Features and
// targets are stored transposed ([feature][slot]) so that a warp's loads of one feature are coalesced.
__device__ __forceinline__ void batch_slot(const DevModel& m, uint64_t seed, int it, int s, int mstride, const float* __restrict__ zdec,
                                           const float* __restrict__ tgt, int* __restrict__ bidx, float* __restrict__ feat_t,
                                           float* __restrict__ tgt_t) {
    const uint64_t key = stream_key(seed, kStreamBatchPix, (uint32_t)it, 0);
    const int idx = (int)uniform_below(draw_u32(key, (uint64_t)s), (uint32_t)(m.W * m.H));
    bidx[s] = idx;
    float f[kMaxIn];
    pixel_features(m, zdec, idx % m.W, idx / m.W, f);
    for (int i = 0; i < m.nin; i++) feat_t[(long long)i * mstride + s] = f[i];
    const float* t = tgt + (long long)idx * m.nout;
    for (int c = 0; c < m.nout; c++) tgt_t[(long long)c * mstride + s] = t[c];
}
__global__ void k_batch(DevModel m, uint64_t seed, int it, int M, int mstride, const float* __restrict__ zdec,
                        const float* __restrict__ tgt, int* __restrict__ bidx, float* __restrict__ feat_t,
                        float* __restrict__ tgt_t) {
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s < M) batch_slot(m, seed, it, s, mstride, zdec, tgt, bidx, feat_t, tgt_t);
}

void launch_batch(cudaStream_t s, const DevModel& m, uint64_t seed, int it, int M, int mstride, const float* zdec,
                  const float* tgt, int* bidx, float* feat_t, float* tgt_t) {
    k_batch<<<blocks_for(M, 128), 128, 0, s>>>(m, seed, it, M, mstride, zdec, tgt, bidx, feat_t, tgt_t);
    NTCB_CHECK(cudaGetLastError());
}

// ------------------------------------------------------------------ ES noise
// eps[i][k] = gauss(seed, MLP stream, it, pair_begin + i, k): every pair's perturbation, generated once
// per step and read by both the population kernel and the gradient (the reference regenerates it in
// each of its per-chunk CTAs and again per weight in the gradient).
// One CTA row per pair (blockIdx.y), the block sized to P rounded up to a warp so few threads idle.
__global__ void k_mlp_noise(uint64_t seed, int it, int pair_begin, int npairs, int P, float* __restrict__ eps) {
    const int i = blockIdx.y;
    const uint64_t key = stream_key(seed, kStreamMlp, (uint32_t)it, (uint32_t)(pair_begin + i));
    for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < P; k += gridDim.x * blockDim.x)
        eps[(long long)i * P + k] = gauss_at(key, (uint64_t)k);
}

__global__ void k_noise_fill(uint64_t seed, uint32_t stream, uint32_t step, uint32_t pair, uint64_t index0, long long n,
                             float* __restrict__ gauss, uint32_t* __restrict__ u32) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint64_t key = stream_key(seed, stream, step, pair);
    gauss[i] = gauss_at(key, index0 + (uint64_t)i);
    u32[i] = draw_u32(key, index0 + (uint64_t)i);
}
void launch_noise_fill(cudaStream_t s, uint64_t seed, uint32_t stream, uint32_t step, uint32_t pair, uint64_t index0, long long n,
                       float* gauss, uint32_t* u32) {
    k_noise_fill<<<blocks_for(n, 256), 256, 0, s>>>(seed, stream, step, pair, index0, n, gauss, u32);
    NTCB_CHECK(cudaGetLastError());
}

// The minibatch of step `it` and the ES noise of its pairs [pair_begin, pair_begin + npairs) in one launch: the
// first blocks draw the minibatch slots, the rest fill eps row by row (kBatchNoiseTPB weights per block).
constexpr int kBatchNoiseTPB = 128;
__global__ void __launch_bounds__(kBatchNoiseTPB) k_batch_noise(DevModel m, uint64_t seed, int it, int M, int mstride,
                                                                const float* __restrict__ zdec, const float* __restrict__ tgt,
                                                                int* __restrict__ bidx, float* __restrict__ feat_t,
                                                                float* __restrict__ tgt_t, int batch_blocks, int pair_begin, int P,
                                                                int row_blocks, float* __restrict__ eps) {
    if ((int)blockIdx.x < batch_blocks) {
        const int s = blockIdx.x * kBatchNoiseTPB + threadIdx.x;
        if (s < M) batch_slot(m, seed, it, s, mstride, zdec, tgt, bidx, feat_t, tgt_t);
        return;
    }
    const int b = blockIdx.x - batch_blocks, i = b / row_blocks;
    const int k = (b - i * row_blocks) * kBatchNoiseTPB + threadIdx.x;
    if (k >= P) return;
    const uint64_t key = stream_key(seed, kStreamMlp, (uint32_t)it, (uint32_t)(pair_begin + i));
    eps[(long long)i * P + k] = gauss_at(key, (uint64_t)k);
}
void launch_batch_noise(cudaStream_t s, const DevModel& m, uint64_t seed, int it, int M, int mstride, const float* zdec,
                        const float* tgt, int* bidx, float* feat_t, float* tgt_t, int pair_begin, int npairs, int P, float* eps) {
    const int batch_blocks = (int)blocks_for(M, kBatchNoiseTPB), row_blocks = (int)blocks_for(P, kBatchNoiseTPB);
    const long long blocks = batch_blocks + (long long)row_blocks * std::max(0, npairs);
    k_batch_noise<<<(unsigned)blocks, kBatchNoiseTPB, 0, s>>>(m, seed, it, M, mstride, zdec, tgt, bidx, feat_t, tgt_t, batch_blocks,
                                                             pair_begin, P, row_blocks, eps);
    NTCB_CHECK(cudaGetLastError());
}

void launch_mlp_noise(cudaStream_t s, uint64_t seed, int it, int pair_begin, int npairs, int P, float* eps) {
    if (npairs <= 0) return;
    const int tpb = std::min(1024, (P + 31) / 32 * 32);
    dim3 grid(blocks_for(P, tpb), (unsigned)npairs);
    k_mlp_noise<<<grid, tpb, 0, s>>>(seed, it, pair_begin, npairs, P, eps);
    NTCB_CHECK(cudaGetLastError());
}

// ------------------------------------------------------------------ population evaluation
// Runtime-shaped kernels: both weight sets in the reference's flat layout.
__device__ __forceinline__ void build_weight_pair_flat(const DevModel& m, const PopArgs& a, int cand, float* ws) {
    const float* e = (a.mode == 0 && a.sigma != 0.0f) ? a.eps + (long long)(cand - a.cand_begin) * m.P : nullptr;
    for (int k = threadIdx.x; k < m.P; k += blockDim.x) perturbed_weight(a, e, k, cand, ws[k], ws[m.P + k]);
    __syncthreads();
}

// One CTA per (candidate pair, batch chunk): the + and - weight sets are evaluated over the chunk's
// minibatch rows on the packed FP32 pipe (R2 row pairs per thread per pass, weight sets stored duplicated:
// {w, w} per slot, 2 * S::SIZE floats per set); the per-row weighted squared errors are accumulated in
// double (loss_subset, main.cpp:1739-1750) and reduced in a fixed order into part[cand][sign][chunk].
template <class S>
__device__ __forceinline__ void build_weight_pair_x2(const DevModel& m, const PopArgs& a, int cand, float* ws) {
    constexpr int kSet = 2 * S::SIZE;
    const float* e = (a.mode == 0 && a.sigma != 0.0f) ? a.eps + (long long)(cand - a.cand_begin) * m.P : nullptr;
    for (int k = threadIdx.x; k < 2 * kSet; k += blockDim.x) ws[k] = 0.0f;
    __syncthreads();
    for (int k = threadIdx.x; k < m.P; k += blockDim.x) {
        float wp, wm;
        perturbed_weight(a, e, k, cand, wp, wm);
        const int sl = 2 * S::slot(k);
        *reinterpret_cast<float2*>(ws + sl) = make_float2(wp, wp);
        *reinterpret_cast<float2*>(ws + kSet + sl) = make_float2(wm, wm);
    }
    __syncthreads();
}

template <class S, int TPB, int R2>
__global__ void __launch_bounds__(TPB, S::kPopMinBlocks) k_pop_eval_x2(DevModel m, PopArgs a, int chunks) {
    extern __shared__ __align__(16) float ws[];
    __shared__ double red[TPB / 32];
    constexpr int R = 2 * R2;
    const int cand = pop_cand(a, blockIdx.x);
    const int chunk = blockIdx.y;
    build_weight_pair_x2<S>(m, a, cand, ws);
    const int row0 = chunk * a.chunk;
    const int row1 = min(a.M, row0 + a.chunk);
    double acc[2] = {0.0, 0.0};
#pragma unroll 1
    for (int sg = 0; sg < 2; sg++) {
        const float* w = ws + sg * 2 * S::SIZE;
#pragma unroll 1
        for (int base = row0; base < row1; base += TPB * R) {
            float2 x[R2][S::NIN];
            int rows[R];
#pragma unroll
            for (int r = 0; r < R; r++) rows[r] = base + r * TPB + threadIdx.x;
#pragma unroll
            for (int q = 0; q < R2; q++) {
                const int s0 = min(rows[2 * q], a.M - 1), s1 = min(rows[2 * q + 1], a.M - 1);
#pragma unroll
                for (int i = 0; i < S::NIN; i++)
                    x[q][i] = make_float2(__ldg(a.feat_t + (long long)i * a.mstride + s0), __ldg(a.feat_t + (long long)i * a.mstride + s1));
            }
            float2 o[R2][S::NOUT];
            fixed_forward_x2<S, R2>(w, x, o, m.leak, m.clamp_out);
#pragma unroll
            for (int q = 0; q < R2; q++) {
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const int s = rows[2 * q + h];
                    if (s < row1) {
                        double e = 0.0;
#pragma unroll
                        for (int c = 0; c < S::NOUT; c++) {
                            const float ov = h ? o[q][c].y : o[q][c].x;
                            const float d = ov - __ldg(a.tgt_t + (long long)c * a.mstride + s);
                            e += (double)(m.cw[c] * (d * d));
                        }
                        acc[sg] += e;
                    }
                }
            }
        }
    }
    const double sp = cta_sum<TPB>(acc[0], red);
    const double sm = cta_sum<TPB>(acc[1], red);
    if (threadIdx.x == 0) {
        double* dst = a.part + (long long)blockIdx.x * 2 * chunks;
        dst[chunk] = sp;
        dst[chunks + chunk] = sm;
    }
}

// Runtime-shaped variant: one row per thread through the flat layout.
template <int TPB>
__global__ void __launch_bounds__(TPB) k_pop_eval_generic(DevModel m, PopArgs a, int chunks) {
    extern __shared__ __align__(16) float ws[];
    __shared__ double red[TPB / 32];
    const int cand = pop_cand(a, blockIdx.x);
    const int chunk = blockIdx.y;
    build_weight_pair_flat(m, a, cand, ws);
    const int row0 = chunk * a.chunk;
    const int row1 = min(a.M, row0 + a.chunk);
    double acc[2] = {0.0, 0.0};
    for (int sg = 0; sg < 2; sg++) {
        const float* w = ws + sg * m.P;
        for (int s = row0 + threadIdx.x; s < row1; s += TPB) {
            float f[kMaxIn], o[kMaxOut], t[kMaxOut];
            for (int i = 0; i < m.nin; i++) f[i] = a.feat_t[(long long)i * a.mstride + s];
            for (int c = 0; c < m.nout; c++) t[c] = a.tgt_t[(long long)c * a.mstride + s];
            generic_forward(m, w, f, o);
            acc[sg] += pixel_err_d(m, o, t);
        }
    }
    const double sp = cta_sum<TPB>(acc[0], red);
    const double sm = cta_sum<TPB>(acc[1], red);
    if (threadIdx.x == 0) {
        double* dst = a.part + (long long)blockIdx.x * 2 * chunks;
        dst[chunk] = sp;
        dst[chunks + chunk] = sm;
    }
}

template <class S>
static void launch_pop_fixed(cudaStream_t s, const DevModel& m, const PopArgs& a) {
    const int chunks = pop_chunks(a.M, a.chunk);
    dim3 grid((unsigned)a.ncand, (unsigned)chunks);
    k_pop_eval_x2<S, kPopTPB, kPopRows / 2><<<grid, kPopTPB, 4 * S::SIZE * sizeof(float), s>>>(m, a, chunks);
}

void launch_pop_eval(cudaStream_t s, int shape, const DevModel& m, const PopArgs& a) {
    if (a.ncand <= 0) return;
    switch (shape) {
#define NTCB_CASE(ID, NIN, H1, H2, NOUT) case ID: launch_pop_fixed<FixedShape<NIN, H1, H2, NOUT>>(s, m, a); break;
        NTCB_FIXED_SHAPES(NTCB_CASE)
#undef NTCB_CASE
        default: {
            const int chunks = pop_chunks(a.M, a.chunk);
            dim3 grid((unsigned)a.ncand, (unsigned)chunks);
            const size_t smem = 2 * (size_t)m.P * sizeof(float);
            // two weight sets of up to 12288 floats: above the 48 KB default
            ensure_dynamic_smem((const void*)k_pop_eval_generic<kPopTPB>, 2 * 12288 * 4);
            k_pop_eval_generic<kPopTPB><<<grid, kPopTPB, smem, s>>>(m, a, chunks);
        }
    }
    NTCB_CHECK(cudaGetLastError());
}

// fit[2i] = (sum over chunks of the + partials) / norm, fit[2i+1] likewise for - (k_mlp_es_finish's order).
// With dl / lsum given (a population evaluated whole on one trainer) the ES reduction of k_es_reduce is
// applied to the same values in the same launch.
__global__ void k_pop_finish(const double* __restrict__ part, int ncand, int chunks, double norm, double* __restrict__ fit,
                             double* __restrict__ dl, double* __restrict__ lsum) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= ncand) return;
    double lp = 0.0, lm = 0.0;
    const double* p = part + (long long)i * 2 * chunks;
    for (int j = 0; j < chunks; j++) { lp += p[j]; lm += p[chunks + j]; }
    lp /= norm;
    lm /= norm;
    fit[2 * i] = lp;
    fit[2 * i + 1] = lm;
    if (dl) {
        dl[i] = lp - lm;
        lsum[i] = 0.5 * (lp + lm);
    }
}
void launch_pop_finish(cudaStream_t s, const double* part, int ncand, int chunks, double norm, double* fit, double* dl,
                       double* lsum) {
    if (ncand <= 0) return;
    k_pop_finish<<<blocks_for(ncand, 128), 128, 0, s>>>(part, ncand, chunks, norm, fit, dl, lsum);
    NTCB_CHECK(cudaGetLastError());
}

// dl[i] = lp - lm, lsum[i] = (lp + lm) / 2 (MlpTrainer::step, main.cpp:1859).
__global__ void k_es_reduce(const double* __restrict__ fit, int N, double* __restrict__ dl, double* __restrict__ lsum) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= N) return;
    const double lp = fit[2 * i], lm = fit[2 * i + 1];
    dl[i] = lp - lm;
    lsum[i] = 0.5 * (lp + lm);
}
void launch_es_reduce(cudaStream_t s, const double* fit, int N, double* dl, double* lsum) {
    k_es_reduce<<<blocks_for(N, 128), 128, 0, s>>>(fit, N, dl, lsum);
    NTCB_CHECK(cudaGetLastError());
}

// dl[j] = lp - lm and the realised step hh[j] = (double)(w0 + h) - (double)(w0 - h) (main.cpp:1912-1915).
__global__ void k_fd_reduce(const double* __restrict__ fit, const float* __restrict__ w0, float h, int P,
                            double* __restrict__ dl, double* __restrict__ hh) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= P) return;
    dl[j] = fit[2 * j] - fit[2 * j + 1];
    const float wp = w0[j] + h, wm = w0[j] - h;
    hh[j] = (double)wp - (double)wm;
}
void launch_fd_reduce(cudaStream_t s, const double* fit, const float* w0, float h, int P, double* dl, double* hh) {
    k_fd_reduce<<<blocks_for(P, 128), 128, 0, s>>>(fit, w0, h, P, dl, hh);
    NTCB_CHECK(cudaGetLastError());
}

// ------------------------------------------------------------------ ES gradient + Adam
// g_k = sum_i ((float)dl_i * scale) * eps_ik (MlpTrainer::step, main.cpp:1867-1873), one FMA per pair in
// pair order inside a segment of `seglen` pairs; the segment partials are summed in segment order by
// k_es_grad_adam. With a single segment this is the reference's serial order exactly.
__global__ void k_es_grad_partial(const double* __restrict__ dl, const float* __restrict__ eps, int N, int P, float scale,
                                  int seglen, float* __restrict__ gpart) {
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    const int seg = blockIdx.y;
    if (k >= P) return;
    const int i0 = seg * seglen, i1 = min(N, i0 + seglen);
    float g = 0.0f;
    int i = i0;
    // 32 pairs' loads issued together (the kernel is bound by loads in flight, not by its FMAs), then their FMAs in
    // pair order: the same chain as one pair at a time
    constexpr int U = 32;
    for (; i + U <= i1; i += U) {
        float e[U];
#pragma unroll
        for (int j = 0; j < U; j++) e[j] = __ldg(eps + (long long)(i + j) * P + k);
#pragma unroll
        for (int j = 0; j < U; j++) g = fmaf((float)__ldg(dl + i + j) * scale, e[j], g);
    }
    for (; i < i1; i++) g = fmaf((float)dl[i] * scale, __ldg(eps + (long long)i * P + k), g);
    gpart[(long long)seg * P + k] = g;
}
void launch_es_grad_partial(cudaStream_t s, const double* dl, const float* eps, int N, int P, float scale, int seglen, float* gpart) {
    const int nseg = (N + seglen - 1) / seglen;
    dim3 grid(blocks_for(P, 128), (unsigned)nseg);
    k_es_grad_partial<<<grid, 128, 0, s>>>(dl, eps, N, P, scale, seglen, gpart);
    NTCB_CHECK(cudaGetLastError());
}

// One thread per weight adds the segment sums from segment 0 in order, as single floats (32 segments' loads issued
// together, then their adds): the order of the single-GPU sum whatever the layout. Segment s lives at part + s * P
// (one gathered array) or, with RANKS, at part + r * rank_stride + t * P for s = r * segs + t (the ranks' exchange
// blocks read in place).
template <bool RANKS>
__device__ __forceinline__ const float* seg_at(const float* pk, int s, long long rank_stride, int segs, int P) {
    if constexpr (RANKS) {
        const int r = s / segs;
        return pk + r * rank_stride + (long long)(s - r * segs) * P;
    } else {
        return pk + (long long)s * P;
    }
}
template <bool RANKS>
__global__ void k_es_grad_adam(const float* __restrict__ part, long long rank_stride, int segs, int nseg, int P, float* __restrict__ grad,
                               float* __restrict__ theta, float* __restrict__ m, float* __restrict__ v, float lr, float c1, float c2) {
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= P) return;
    const float* pk = part + k;
    float g = pk[0];
    int sg = 1;
    constexpr int U = 32;
    for (; sg + U <= nseg; sg += U) {   // 32 segments' loads together, summed in segment order
        float e[U];
#pragma unroll
        for (int j = 0; j < U; j++) e[j] = *seg_at<RANKS>(pk, sg + j, rank_stride, segs, P);
#pragma unroll
        for (int j = 0; j < U; j++) g += e[j];
    }
    for (; sg < nseg; sg++) g += *seg_at<RANKS>(pk, sg, rank_stride, segs, P);
    grad[k] = g;
    float th = theta[k], mm = m[k], vv = v[k];
    adam_update(th, g, mm, vv, lr, c1, c2);
    theta[k] = th; m[k] = mm; v[k] = vv;
}
void launch_es_grad_adam(cudaStream_t s, const float* gpart, int nseg, int P, float* grad, float* theta, float* m, float* v,
                         float lr, float c1, float c2) {
    k_es_grad_adam<false><<<blocks_for(P, 64), 64, 0, s>>>(gpart, 0, nseg, nseg, P, grad, theta, m, v, lr, c1, c2);
    NTCB_CHECK(cudaGetLastError());
}
void launch_es_grad_adam_ranks(cudaStream_t s, const float* part, long long rank_stride, int world, int segs, int P, float* grad,
                               float* theta, float* m, float* v, float lr, float c1, float c2) {
    k_es_grad_adam<true><<<blocks_for(P, 64), 64, 0, s>>>(part, rank_stride, segs, world * segs, P, grad, theta, m, v, lr, c1, c2);
    NTCB_CHECK(cudaGetLastError());
}

// FD: grad_j = (float)(dl_j / hh_j) (main.cpp:1917), then Adam.
__global__ void k_fd_grad_adam(const double* __restrict__ dl, const double* __restrict__ hh, int P, float* __restrict__ grad,
                               float* __restrict__ theta, float* __restrict__ m, float* __restrict__ v, float lr, float c1, float c2) {
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= P) return;
    const float g = (float)(dl[k] / hh[k]);
    grad[k] = g;
    float th = theta[k], mm = m[k], vv = v[k];
    adam_update(th, g, mm, vv, lr, c1, c2);
    theta[k] = th; m[k] = mm; v[k] = vv;
}
void launch_fd_grad_adam(cudaStream_t s, const double* dl, const double* hh, int P, float* grad, float* theta, float* m, float* v,
                         float lr, float c1, float c2) {
    k_fd_grad_adam<<<blocks_for(P, 256), 256, 0, s>>>(dl, hh, P, grad, theta, m, v, lr, c1, c2);
    NTCB_CHECK(cudaGetLastError());
}

// ------------------------------------------------------------------ full-image decode
// Decoder::decode_full (main.cpp:1712-1718): every pixel's features and MLP outputs, interleaved.
template <class S, int TPB, int R>
__global__ void __launch_bounds__(TPB) k_decode_fixed(DevModel m, const float* __restrict__ wg, const float* __restrict__ z,
                                                      float* __restrict__ img) {
    constexpr int R2 = R / 2;
    extern __shared__ __align__(16) float ws[];
    load_weights_x2<S>(wg, m.P, ws);
    const long long npix = (long long)m.W * m.H;
    const long long base = (long long)blockIdx.x * TPB * R;
    float2 x[R2][S::NIN];
#pragma unroll
    for (int h = 0; h < R2; h++) {
        long long pa = base + (2 * h) * TPB + threadIdx.x, pb = base + (2 * h + 1) * TPB + threadIdx.x;
        if (pa >= npix) pa = npix - 1;
        if (pb >= npix) pb = npix - 1;
        float fa[kMaxIn], fb[kMaxIn];
        pixel_features(m, z, (int)(pa % m.W), (int)(pa / m.W), fa);
        pixel_features(m, z, (int)(pb % m.W), (int)(pb / m.W), fb);
#pragma unroll
        for (int i = 0; i < S::NIN; i++) x[h][i] = make_float2(fa[i], fb[i]);
    }
    float2 o[R2][S::NOUT];
    fixed_forward_x2<S, R2>(ws, x, o, m.leak, m.clamp_out);
#pragma unroll
    for (int h = 0; h < R2; h++) {
        const long long pa = base + (2 * h) * TPB + threadIdx.x, pb = base + (2 * h + 1) * TPB + threadIdx.x;
        if (pa < npix)
#pragma unroll
            for (int c = 0; c < S::NOUT; c++) img[pa * S::NOUT + c] = o[h][c].x;
        if (pb < npix)
#pragma unroll
            for (int c = 0; c < S::NOUT; c++) img[pb * S::NOUT + c] = o[h][c].y;
    }
}

__global__ void k_decode_generic(DevModel m, const float* __restrict__ wg, const float* __restrict__ z, float* __restrict__ img) {
    extern __shared__ __align__(16) float ws[];
    for (int k = threadIdx.x; k < m.P; k += blockDim.x) ws[k] = wg[k];
    __syncthreads();
    const long long p = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= (long long)m.W * m.H) return;
    float f[kMaxIn], o[kMaxOut];
    pixel_features(m, z, (int)(p % m.W), (int)(p / m.W), f);
    generic_forward(m, ws, f, o);
    for (int c = 0; c < m.nout; c++) img[p * m.nout + c] = o[c];
}

void launch_decode(cudaStream_t s, int shape, const DevModel& m, const float* w, const float* z, float* img) {
    const long long npix = (long long)m.W * m.H;
    switch (shape) {
#define NTCB_CASE(ID, NIN, H1, H2, NOUT) case ID: { using S = FixedShape<NIN, H1, H2, NOUT>; \
        k_decode_fixed<S, kDecTPB, kDecRows><<<blocks_for(npix, kDecTPB * kDecRows), kDecTPB, 2 * S::SIZE * sizeof(float), s>>>(m, w, z, img); break; }
        NTCB_FIXED_SHAPES(NTCB_CASE)
#undef NTCB_CASE
        default: k_decode_generic<<<blocks_for(npix, 128), 128, m.P * sizeof(float), s>>>(m, w, z, img);
    }
    NTCB_CHECK(cudaGetLastError());
}

// ------------------------------------------------------------------ DCT sensitivity probe
// dct_probe_codes (main.cpp:1002-1030), one thread per (8x8 block, level-0 channel): at the 4 pixels
// (8 bx + {2, 5}, 8 by + {2, 5}) the features of the decode buffer with channel c set to -1, -0.5, 0, 0.5, 1
// go through the MLP; each of the 4 segments contributes g^2 with g = (255 / 16) sqrt(sum_o cw[o] d_o^2 / wsum)
// in double; the block gain is sqrt(sum / 16) and the code lround(log2(gain / floor) / 0.6) clamped to
// [0, 15] (dct_code_of_gain, main.cpp:981-985). The reference runs it on the host between steps; it is an
// estimate there too (its comment: a CPU and a --cuda run may differ on a code boundary).
__global__ void k_dct_probe(DevModel m, const float* __restrict__ wg, const float* __restrict__ z, int BW, int BH, int C,
                            uint8_t* __restrict__ code, float* __restrict__ gain) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)BW * BH * C) return;
    const int c = (int)(i % C);
    const long long b = i / C;
    const int bx = (int)(b % BW), by = (int)(b / BW);
    const int P[2] = {2, 5};
    const float SJ[5] = {-1.0f, -0.5f, 0.0f, 0.5f, 1.0f};
    double acc = 0.0;
    for (int qy = 0; qy < 2; qy++)
        for (int qx = 0; qx < 2; qx++) {
            float f[kMaxIn], out[5][kMaxOut];
            pixel_features(m, z, bx * 8 + P[qx], by * 8 + P[qy], f);
            for (int j = 0; j < 5; j++) { f[c] = SJ[j]; generic_forward(m, wg, f, out[j]); }
            for (int j = 0; j < 4; j++) {
                double ss = 0.0;
                for (int o = 0; o < m.nout; o++) {
                    const double d = (double)out[j + 1][o] - (double)out[j][o];
                    ss += (double)m.cw[o] * d * d;
                }
                const double g = (255.0 / 16.0) * sqrt(ss / (double)m.wsum);
                acc += g * g;
            }
        }
    const double gb = sqrt(acc / 16.0);
    const double floor_g = 14.0 / 64.0;
    const double gg = gb > floor_g ? gb : floor_g;
    const long long k = llround(log2(gg / floor_g) / 0.6);
    code[i] = (uint8_t)(k < 0 ? 0 : (k > 15 ? 15 : k));
    if (gain) gain[i] = (float)gb;
}
void launch_dct_probe(cudaStream_t s, const DevModel& m, const float* w, const float* z, int BW, int BH, int C, uint8_t* code, float* gain) {
    const long long n = (long long)BW * BH * C;
    if (n <= 0) return;
    k_dct_probe<<<blocks_for(n, 128), 128, 0, s>>>(m, w, z, BW, BH, C, code, gain);
    NTCB_CHECK(cudaGetLastError());
}

}  // namespace ntcb

namespace ntcb {
// FP32 FMA throughput probe: every thread runs 8 independent FMA chains (the FMA latency hidden by ILP
// and by 8 warps per scheduler); the result is stored so the chains are live. Measures the FFMA peak
// the population kernel is bounded by (the driver's measured peaks cover HBM and bf16 tensor only).
__global__ void __launch_bounds__(256) k_ffma_peak(float* out, int iters, float a, float b) {
    float x[8];
#pragma unroll
    for (int j = 0; j < 8; j++) x[j] = (float)(threadIdx.x + j) * 1e-3f;
    for (int i = 0; i < iters; i++) {
#pragma unroll
        for (int j = 0; j < 8; j++) x[j] = fmaf(x[j], a, b);
    }
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; j++) s += x[j];
    if (s == 12345.678f) out[threadIdx.x] = s;   // never true for the inputs used; keeps the chains live
}
double measure_ffma_tflops(int sms) {
    float* out = nullptr;
    NTCB_CHECK(cudaMalloc(&out, 256 * sizeof(float)));
    const int blocks = sms * 8, iters = 1 << 16;
    cudaEvent_t e0, e1;
    NTCB_CHECK(cudaEventCreate(&e0)); NTCB_CHECK(cudaEventCreate(&e1));
    k_ffma_peak<<<blocks, 256>>>(out, 256, 0.999f, 1e-4f);   // warm up
    NTCB_CHECK(cudaEventRecord(e0));
    k_ffma_peak<<<blocks, 256>>>(out, iters, 0.999f, 1e-4f);
    NTCB_CHECK(cudaEventRecord(e1));
    NTCB_CHECK(cudaEventSynchronize(e1));
    float ms = 0.0f;
    NTCB_CHECK(cudaEventElapsedTime(&ms, e0, e1));
    cudaEventDestroy(e0); cudaEventDestroy(e1); cudaFree(out);
    const double flops = 2.0 * 8.0 * (double)iters * blocks * 256;
    return flops / (ms * 1e-3) / 1e12;
}
}  // namespace ntcb
