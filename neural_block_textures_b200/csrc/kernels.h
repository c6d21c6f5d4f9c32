// Host-side launchers of the backend's kernels. Every launcher takes the trainer's stream and the
// by-value model description; the shape id selects a compile-time-shaped instantiation
// (shape_id() == 0 selects the runtime-shaped fallback).
#pragma once
#include "device_model.cuh"

namespace ntcb {

// The compile-time MLP shapes (nin, hidden1, hidden2, nout) with specialised kernels. Every other
// shape inside the envelope runs the runtime-shaped kernels.
#define NTCB_FIXED_SHAPES(X) \
    X(1, 5, 24, 24, 3)       \
    X(2, 6, 24, 24, 3)       \
    X(3, 8, 24, 24, 3)       \
    X(4, 8, 24, 24, 12)

int shape_id(const DevModel& m);
double measure_ffma_tflops(int sms);   // FP32 FMA peak of the current device, TFLOP/s

// Per-device launch set-up (device_cache.cu): the current device's SM count, and a kernel's dynamic shared-memory
// opt-in, each made once per device ordinal (thread-safe).
int device_sm_count();
void ensure_dynamic_smem(const void* kernel, int bytes);

// ---- MLP population (kernels_mlp.cu) ----
struct PopArgs {
    int mode;                  // 0 = ES pairs (w0 +- sigma eps), 1 = FD (w0 with weight j at +- h)
    int it;                    // iteration (noise step)
    float sigma;               // ES sigma (0: the unperturbed weights, no noise read)
    float fd_h;                // FD step
    int cand_begin, ncand;     // ES: global pair index range; FD: weight index range
    int stats_first;           // FD: candidate 0 is the unperturbed pair (the step's statistics), candidate i >= 1 weight
                               // cand_begin + i - 1
    int M, mstride;            // minibatch size and the row stride of feat_t / tgt_t
    int chunk;                 // rows per CTA along the batch (multiple of the tile rows)
    const float* w0;           // base weights (flat reference layout)
    const float* eps;          // ES noise [ncand][P] (row = pair - cand_begin)
    const float* feat_t;       // [nin][mstride]
    const float* tgt_t;        // [nout][mstride]
    double* part;              // [ncand][2][chunks] per-CTA partial sums
    int* tc_err;               // tensor-core kernel: set to 1 when an MMA completion wait timed out
};
int pop_chunks(int M, int chunk);
int pop_chunk_rows(int shape);                 // rows one CTA pass covers (chunk granularity)
void launch_batch(cudaStream_t s, const DevModel& m, uint64_t seed, int it, int M, int mstride, const float* zdec,
                  const float* tgt, int* bidx, float* feat_t, float* tgt_t);
void launch_noise_fill(cudaStream_t s, uint64_t seed, uint32_t stream, uint32_t step, uint32_t pair, uint64_t index0, long long n,
                       float* gauss, uint32_t* u32);
void launch_mlp_noise(cudaStream_t s, uint64_t seed, int it, int pair_begin, int npairs, int P, float* eps);
// launch_batch and launch_mlp_noise (pairs [pair_begin, pair_begin + npairs)) in one launch.
void launch_batch_noise(cudaStream_t s, const DevModel& m, uint64_t seed, int it, int M, int mstride, const float* zdec,
                        const float* tgt, int* bidx, float* feat_t, float* tgt_t, int pair_begin, int npairs, int P, float* eps);
void launch_pop_eval(cudaStream_t s, int shape, const DevModel& m, const PopArgs& a);
// Tensor-core (tcgen05, 3xTF32) population evaluation for the fixed shapes; false when the shape or the
// chunk size (a multiple of pop_tc_rows()) does not fit it, in which case nothing was launched.
bool launch_pop_eval_tc(cudaStream_t s, int shape, const DevModel& m, const PopArgs& a);
int pop_tc_rows();
// Tensor-core latent ES pass (same contract as launch_lat_eval) for the fixed shapes; false when the shape has
// no tensor kernel (nothing launched). err: device flag set when an MMA completion wait timed out.
bool launch_lat_eval_tc(cudaStream_t s, int shape, const DevModel& m, const float* w, const float* zdec, const float* eps,
                        long long nz, const float* tgt, int K, unsigned active_mask, float sg, float inv_px, float* dpix,
                        long long p_begin, long long p_end, long long pstride, int* err);
// Sum the chunk partials of every candidate in order, normalise, and write (lp, lm) pairs to fit[2*i], fit[2*i+1];
// with dl / lsum non-null also dl[i] = lp - lm and lsum[i] = (lp + lm) / 2 (launch_es_reduce's values).
void launch_pop_finish(cudaStream_t s, const double* part, int ncand, int chunks, double norm, double* fit,
                       double* dl = nullptr, double* lsum = nullptr);
// ES: dl, lsum from the fitness of all N pairs; FD: dl, hh.
void launch_es_reduce(cudaStream_t s, const double* fit, int N, double* dl, double* lsum);
void launch_fd_reduce(cudaStream_t s, const double* fit, const float* w0, float h, int P, double* dl, double* hh);
// ES gradient partials over pair segments: gpart[seg][k] = sum_{i in seg} ((float)dl[i] * scale) * eps[i][k].
void launch_es_grad_partial(cudaStream_t s, const double* dl, const float* eps, int N, int P, float scale, int seglen, float* gpart);
// grad[k] = sum_seg gpart[seg][k] (fixed order), then Adam on (theta, m, v).
void launch_es_grad_adam(cudaStream_t s, const float* gpart, int nseg, int P, float* grad, float* theta, float* m, float* v,
                         float lr, float c1, float c2);
// The same from the ranks' exchange blocks in place: rank r's segs segment sums start at part + r * rank_stride floats.
void launch_es_grad_adam_ranks(cudaStream_t s, const float* part, long long rank_stride, int world, int segs, int P, float* grad,
                               float* theta, float* m, float* v, float lr, float c1, float c2);
void launch_fd_grad_adam(cudaStream_t s, const double* dl, const double* hh, int P, float* grad, float* theta, float* m, float* v,
                         float lr, float c1, float c2);
void launch_decode(cudaStream_t s, int shape, const DevModel& m, const float* w, const float* z, float* img);
// DCT sensitivity probe (codes [BW * BH][C], gains optional) of the MLP w on the decode buffer z.
void launch_dct_probe(cudaStream_t s, const DevModel& m, const float* w, const float* z, int BW, int BH, int C, uint8_t* code, float* gain);

// ---- latent ES and selector search (kernels_latent.cu) ----
void launch_lat_noise(cudaStream_t s, uint64_t seed, int step, int K, const DevModel& m, unsigned active_mask, long long nz, float* eps);
// The same noise for the flat latent elements [lo, hi) only (each value depends on its index alone).
void launch_lat_noise_range(cudaStream_t s, uint64_t seed, int step, int K, long long lo, long long hi, long long nz, float* eps);
void launch_lat_eval(cudaStream_t s, int shape, const DevModel& m, const float* w, const float* zdec, const float* eps,
                     long long nz, const float* tgt, int K, unsigned active_mask, float sg, float inv_px, float* dpix,
                     long long p_begin, long long p_end, long long pstride);
// (pixels [p_begin, p_end) of every pair; pair k's value of pixel p goes to dpix[k * pstride + p - p_begin])
struct RateTerm {              // DCT rate term of the latent gradient (level 0), null dbits = off
    const int* dbits;          // [K][nblk * C]
    float rate_scale;
    int BW, C;
};
struct LatAdam {              // Adam on the texels a gather produces (latent, moments, host bias corrections)
    float *z, *m, *v;
    float lr, c1, c2;
};
// Texel rows [ty0, ty1) of the level. dpix: blocks of rows_per_block image rows starting at image row row_base,
// each block [K][rows_per_block * W] (one block from row 0 = the plain [K][W * H]). Writes the texels' gradient
// to grad (not accumulated) and applies the Adam step to them.
void launch_lat_gather(cudaStream_t s, const DevModel& m, int level, const int* xr, const int* yr, const float* dpix,
                       const float* eps, long long nz, int K, float scale, const RateTerm& rate, float* grad,
                       int rows_per_block, int ty0, int ty1, int row_base, const LatAdam& adam);
// Level-0 values of n consecutive floats (C channels) as one-byte grid indices, and back: world blocks of blk bytes,
// block q holding values [q n, (q + 1) n) (the sharded selector search's exchange).
void launch_qat_pack(cudaStream_t s, const float* z0, long long n, int C, const int* bits, uint8_t* out);
void launch_qat_unpack(cudaStream_t s, const uint8_t* in, long long blk, long long n, int world, int C, const int* bits,
                       const float* grid, float* z0);
// Tensor-core selector search (one bit depth for every level-0 channel, uniform cw x ch pixel cells, the fixed shapes
// with their compile-time level layout, (2^bits) cw ch <= 32 rows per texel); false when it does not apply (nothing
// launched). err: device flag set when an MMA completion wait timed out.
bool launch_qat_tc(cudaStream_t s, int shape, const DevModel& m, const float* w, float* zdec, const float* tgt, const float* grid,
                   int bits, int cw, int ch, long long t_begin, long long t_end, int* err);
void launch_qat(cudaStream_t s, int shape, const DevModel& m, const float* w, float* zdec, const float* tgt,
                const int* xr0, const int* yr0, const float* grid, const int* bits, long long t_begin, long long t_end,
                int max_bits);

// ---- progress-print statistics (kernels_stats.cu) ----
// Channel min / max of a level [ntex][C] as order-preserving int keys, mm[2 c] / mm[2 c + 1].
void launch_level_minmax(cudaStream_t s, const float* z, long long ntex, int C, int* mm);
struct LevelQuantArgs {
    const float* z;            // training latent of the level [W * H][C]
    const float* zd;           // decode buffer of the level
    float* zq;                 // out: the quantized copy
    int W, H, C;
    int mode;                  // 0 post-hoc min / max grid, 1 --qat grid (zq = z), 2 --qes grid (zq = zd)
    int bits[kMaxCh];          // depth per channel
    float lo[kMaxCh], range[kMaxCh];   // mode 2: the fitted --qes table
    const int* minmax;         // mode 0: launch_level_minmax's keys
    int dpcm;                  // also the DPCM residual histogram
    int *hist, *rhist;         // [C][hstride] each
    int hstride;
};
void launch_level_quant(cudaStream_t s, const LevelQuantArgs& a);
// Integer 8-bit squared error per texture (sse[kMaxOut / 3]) of images a, b ([H][W][nc]) over ew x eh.
void launch_mse8(cudaStream_t s, const float* a, const float* b, int W, int ew, int eh, int nc, unsigned long long* sse);
int lat_moment_blocks();
// Per-block (sum, sum of squares, max |v|) of n values, part[3 * lat_moment_blocks()].
void launch_lat_moments(cudaStream_t s, const float* z, long long n, double* part);
void launch_qat_offgrid(cudaStream_t s, const float* z, long long n, int C, const int* bits, const float* grid,
                        unsigned long long* count);
// Token statistics of a DCT-coded level 0 for the bit simulator (dct_analyze, main.cpp:1080-1160): per channel,
// kDctHistInts ints at hist + c * kDctHistInts (zeroed by the caller): the run histogram (run 64 = EOB), the |q|
// histogram (|q| > 256 folded into 256), the run and |q| histograms per context (the zigzag position of the
// previous nonzero), the DC-residual histogram (DC minus the left block's, the upper block's in the first column,
// 0 for the first block; offset 2048, clamped to 0..4096), the scale-code histogram, then the counts of nonzero
// tokens, of EOBs and of magnitudes above 256.
constexpr int kDctRun = 0, kDctMag = kDctRun + 65, kDctCtxRun = kDctMag + 257, kDctCtxMag = kDctCtxRun + 64 * 65,
              kDctDcres = kDctCtxMag + 64 * 257, kDctCode = kDctDcres + 4097, kDctCounts = kDctCode + 16,
              kDctHistInts = kDctCounts + 3;
struct DctTables;
void launch_dct_tokens(cudaStream_t s, const DctTables& T, const int16_t* sym, const uint8_t* code, int* hist);

}  // namespace ntcb
