/* libntc_b200.so: flat C ABI of the B200 ES training backend for neural_block_textures.
 *
 * Every entry point mirrors one member of the reference backend's C++ class
 * ntc_cuda::Trainer (cuda/ntc_cuda.h:78-132, cited per function) with plain pointers and
 * sizes, so that any FFI (ctypes, cgo, JNI) can drive the same engine that the C++ class in
 * ntc_cuda.h exposes to main.cpp. The description structs have exactly the layout of
 * ntc_cuda::LevelDesc / ModelDesc / QesDesc / DctDesc (static_assert-ed in the library).
 *
 * Conventions (as the reference): host buffers are read or written synchronously inside the call
 * and never retained; ntcb_init reports an unsupported model by returning 0 and writing a reason;
 * every later runtime failure (a CUDA error, a size above what init sized) prints a message to
 * stderr and exits the process, because the reference's caller has no error path.
 * The ntcb_shard_* / ntcb_set_stream / ntcb_kernel_time entries are additions with no member
 * counterpart (multi-GPU population sharding and measurement); they are marked as such. */
#ifndef NTC_B200_H
#define NTC_B200_H
#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NTCB_MAX_LEVELS 3
#define NTCB_MAX_POS 16
#define NTCB_MAX_OUT 12
#define NTCB_MAX_HIDDEN 8
#define NTCB_MAX_CH 16
#define NTCB_MAX_QES_CH 64
#define NTCB_MAX_DCT_CH 4

/* = ntc_cuda::LevelDesc (cuda/ntc_cuda.h:25) */
typedef struct ntcb_level_desc { int W, H, C; size_t off; bool nearest; } ntcb_level_desc;
/* = ntc_cuda::PosDesc (cuda/ntc_cuda.h:26) */
typedef struct ntcb_pos_desc { int kind; } ntcb_pos_desc;
/* = ntc_cuda::ModelDesc (cuda/ntc_cuda.h:29-52) */
typedef struct ntcb_model_desc {
    int W, H, T;
    int nlev; ntcb_level_desc lv[NTCB_MAX_LEVELS];
    int npos; ntcb_pos_desc pos[NTCB_MAX_POS];
    int nin, nout;
    int nhidden; int hidden[NTCB_MAX_HIDDEN];
    float leak;
    bool clamp_out;
    float cw[NTCB_MAX_OUT];
    float wsum;
    int qat_bits[NTCB_MAX_CH];
    int qat;
    const float* qat_grid;
    int qes_bits[NTCB_MAX_LEVELS];
    int dct, dct_C, dct_N, dct_dc_step;
    int dct_q[NTCB_MAX_DCT_CH];
    const float* dct_basis;
    const int* dct_zigzag;
    int max_pairs, max_batch;
    uint64_t seed;
} ntcb_model_desc;
/* = ntc_cuda::QesDesc (cuda/ntc_cuda.h:58-64) */
typedef struct ntcb_qes_desc {
    int bits[NTCB_MAX_LEVELS];
    int live, frozen;
    float lo[NTCB_MAX_LEVELS][NTCB_MAX_QES_CH], hi[NTCB_MAX_LEVELS][NTCB_MAX_QES_CH], range[NTCB_MAX_LEVELS][NTCB_MAX_QES_CH];
    int grid_off[NTCB_MAX_LEVELS][NTCB_MAX_QES_CH];
} ntcb_qes_desc;
/* = ntc_cuda::DctDesc (cuda/ntc_cuda.h:69-76) */
typedef struct ntcb_dct_desc {
    int live, C, BW, BH, N, dc_step;
    int rate_es, rate_trunc; float rate_scale; float lam_t16[16];
    int lo_w16;
    int deadzone;
} ntcb_dct_desc;

typedef struct ntcb_trainer ntcb_trainer;

/* Trainer::Trainer() (cuda/ntc_cuda.h:80): an uninitialised trainer; touches no GPU. */
ntcb_trainer* ntcb_create(void);
/* Trainer::~Trainer() (cuda/ntc_cuda.h:81): frees every device buffer. */
void ntcb_destroy(ntcb_trainer* t);
/* Trainer::init (cuda/ntc_cuda.h:85): allocates device state on the current CUDA device and uploads
 * z (the flat latent), p (the flat MLP) and target (W*H*nout floats in [0,1], interleaved).
 * Returns 1 on success; 0 with a NUL-terminated reason in why[0..why_cap) otherwise. */
int ntcb_init(ntcb_trainer* t, const ntcb_model_desc* d, const float* z, const float* p, const float* target,
              char* why, size_t why_cap);
/* Trainer::banner (cuda/ntc_cuda.h:86): device / runtime line; returns the full length. */
size_t ntcb_banner(const ntcb_trainer* t, char* buf, size_t cap);
/* Trainer::upload_model (cuda/ntc_cuda.h:88): replaces shadow latent and weights, re-snaps the decode copy. */
void ntcb_upload_model(ntcb_trainer* t, const float* z, const float* p);
/* Trainer::download_model (cuda/ntc_cuda.h:89): the fp32 shadow latent and the weights. */
void ntcb_download_model(ntcb_trainer* t, float* z, float* p);
/* Trainer::set_qes (cuda/ntc_cuda.h:93): host-fitted --qes ranges and grid table (grid_n floats), then snap. */
void ntcb_set_qes(ntcb_trainer* t, const ntcb_qes_desc* q, const float* grid, size_t grid_n);
/* Trainer::snap_latent (cuda/ntc_cuda.h:94): rebuild the decode copy from the shadow. */
void ntcb_snap_latent(ntcb_trainer* t);
/* Trainer::shadow_pull (cuda/ntc_cuda.h:95): z[off..off+n) += f * (zq - z), then snap. */
void ntcb_shadow_pull(ntcb_trainer* t, size_t off, size_t n, float f);
/* Trainer::download_zq (cuda/ntc_cuda.h:96): the decode buffer (the shadow when nothing is snapped). */
void ntcb_download_zq(ntcb_trainer* t, float* zq);
/* Trainer::set_dct (cuda/ntc_cuda.h:100): description, scale codes, symbols, step tables; rebuilds level 0 of the copy. */
void ntcb_set_dct(ntcb_trainer* t, const ntcb_dct_desc* d, const uint8_t* code, const int16_t* sym, const int* step);
/* Trainer::download_dct (cuda/ntc_cuda.h:101) */
void ntcb_download_dct(ntcb_trainer* t, int16_t* sym, uint8_t* code);
/* Trainer::download_dct_rate (cuda/ntc_cuda.h:105): every pointer may be NULL. */
void ntcb_download_dct_rate(ntcb_trainer* t, int32_t* bits, int32_t* dbits_last_pair, int* ntrunc, int* nz_before,
                            int* hits, int* evals);
/* Trainer::mlp_step (cuda/ntc_cuda.h:109): one antithetic ES step on the MLP, N pairs, M-pixel minibatch. */
void ntcb_mlp_step(ntcb_trainer* t, int it, float sigma, float lr, int N, int M);
/* Trainer::mlp_step_fd (cuda/ntc_cuda.h:111): one central-difference step on the MLP. */
void ntcb_mlp_step_fd(ntcb_trainer* t, int it, float h, float lr, int M);
/* Trainer::reset_mlp_adam (cuda/ntc_cuda.h:112) */
void ntcb_reset_mlp_adam(ntcb_trainer* t);
/* Trainer::mlp_stats (cuda/ntc_cuda.h:114): mean batch loss and dstd (ES) or fd-rms (FD) of the last step. */
void ntcb_mlp_stats(ntcb_trainer* t, double* batch_loss, double* diff_std);
/* Trainer::lat_step (cuda/ntc_cuda.h:117): one latent ES step with K pairs. */
void ntcb_lat_step(ntcb_trainer* t, int it, float sigma, float lr, int K);
/* Trainer::qat_search (cuda/ntc_cuda.h:119): exhaustive per-texel selector search on level 0. */
void ntcb_qat_search(ntcb_trainer* t);
/* Trainer::decode_full (cuda/ntc_cuda.h:122): z_host NULL decodes the device latent; img gets W*H*nout floats. */
void ntcb_decode_full(ntcb_trainer* t, const float* z_host, float* img);
/* Trainer::debug_last_batch (cuda/ntc_cuda.h:126): minibatch pixel indices of the last MLP step.
 * Writes min(cap, count) entries; returns count. */
size_t ntcb_debug_last_batch(const ntcb_trainer* t, int* out, size_t cap);
/* Trainer::debug_last_dl (cuda/ntc_cuda.h:127): per-pair (ES) or per-weight (FD) loss differences. */
size_t ntcb_debug_last_dl(const ntcb_trainer* t, double* out, size_t cap);
/* Trainer::debug_last_zgrad (cuda/ntc_cuda.h:128): the latent ES gradient of the last lat_step (before Adam). */
size_t ntcb_debug_last_zgrad(const ntcb_trainer* t, float* out, size_t cap);

/* ---- additions (no ntc_cuda::Trainer counterpart) ---- */
/* Per-candidate fitness of the last ES step: lp[i] = L(w + sigma eps_i), lm[i] = L(w - sigma eps_i) for the
 * pairs this trainer evaluated (normalised like loss_subset). Returns the pair count. */
size_t ntcb_debug_last_fitness(const ntcb_trainer* t, double* lp, double* lm, size_t cap);
/* Launch every subsequent kernel of this trainer on `stream` (a cudaStream_t; NULL restores the trainer's own). */
void ntcb_set_stream(ntcb_trainer* t, void* stream);
/* Kernel timing with CUDA events on the trainer's stream: enable, then read the summed device time and the launch
 * count of one kernel class since the last read ("mlp_eval", "lat_eval", "lat_gather", "qat", "mlp_grad", "decode",
 * "noise", "batch", "fd_eval"). Reading synchronises the stream. */
void ntcb_kernel_timing(ntcb_trainer* t, int enable);
/* While timing is enabled, time only kernel class `kernel` (NULL or "": every class). Every timed launch costs two
 * event records and the host calls that create them; timing one class keeps a measured loop close to untimed. */
void ntcb_kernel_timing_only(ntcb_trainer* t, const char* kernel);
void ntcb_kernel_time(ntcb_trainer* t, const char* kernel, double* total_ms, int* launches);
/* Fills n draws of the counter-based noise on the current CUDA device (no trainer needed): gauss_host[i] and
 * u32_host[i] for index index0 + i of (seed, stream, step, pair); either pointer may be NULL. For tests. */
void ntcb_noise_fill(uint64_t seed, uint32_t stream, uint32_t step, uint32_t pair, uint64_t index0, size_t n,
                     float* gauss_host, uint32_t* u32_host);
/* No counterpart in the reference. The per-pair ES fitness of mlp_step (L(w + sigma eps_i), L(w - sigma eps_i)
 * for pairs pair_begin .. pair_begin + npairs - 1 of iteration `it`, hash noise keyed by d->seed, normalised
 * like loss_subset) for callers that cannot allocate device memory where they run — a host engine whose device
 * memory is fixed after start-up, or a plugin that may only use memory it is handed; cudaMalloc can also block
 * and synchronise the device. It allocates nothing: its scratch is one file-scope device array of
 * NTCB_STATIC_SCRATCH_BYTES per GPU, held until exit. Inputs are host arrays: w (the flat MLP), feat (M rows of
 * d->nin features, the minibatch pixels' MLP inputs), tgt (M rows of d->nout targets); fit receives 2 * npairs
 * doubles (L+, L- per pair). Returns 1, or 0 with a reason in why when the sizes need more than the static
 * maximum, the model is outside the envelope, a CUDA error was already pending, or a CUDA call inside it failed
 * (it never exits the process). The first call on a device looks up the array's device address (make it before
 * any stream capture; not valid across a cudaDeviceReset). Calls in one process share the array: concurrent calls
 * race and must be serialised by the caller. Synchronous on the legacy default stream. */
#define NTCB_STATIC_SCRATCH_BYTES ((size_t)16 << 20)
int ntcb_es_fitness_noalloc(const ntcb_model_desc* d, int it, float sigma, int pair_begin, int npairs,
                            const float* w, const float* feat, const float* tgt, int M, double* fit,
                            char* why, size_t why_cap);
/* Host-only: the per-texel pixel range [lo[t], hi[t]) along one axis of a level with ntex texels over npx
 * pixels, with the nearest-cell rule or the bilinear distinct-texel rule the latent gradient gathers with.
 * Returns 1 when every texel's pixels form one contiguous range (the gather's precondition), else 0. */
int ntcb_footprint_ranges(int npx, int ntex, int nearest, int* lo, int* hi);
/* Measured FP32 FMA throughput of the current device in TFLOP/s (the roofline of the population kernels). */
double ntcb_fp32_peak_tflops(void);
/* The DCT scale-code sensitivity probe (dct_probe_codes, main.cpp:1002-1030) on the device, for the current MLP
 * and decode buffer: one code per (8x8 block of the image, level-0 channel), [block raster][channel], and the
 * block gains. Fills min(n, cap) entries of codes / gains (host buffers, either may be null) and returns n =
 * (W / 8) * (H / 8) * C. Replaces the host probe of the --dct-q switch and refits (main.cpp:4110-4120), which
 * would otherwise download the model and decode on the host. Not strict FP, like the host probe: codes can
 * differ from a host run where a gain lies on a code boundary. No counterpart in the reference. */
size_t ntcb_dct_probe(ntcb_trainer* t, uint8_t* codes, float* gains, size_t cap);
/* The same for a drop-in C++ trainer: cpp_trainer points at an initialised ntc_cuda::Trainer. */
size_t ntcb_cpp_dct_probe(void* cpp_trainer, uint8_t* codes, float* gains, size_t cap);

#define NTCB_MAX_T (NTCB_MAX_OUT / 3)
/* The figures of the reference trainer's progress print (main.cpp:4155-4205), computed on the device. */
typedef struct ntcb_progress_stats {
    /* mse_of (main.cpp:1764-1788) of the decode of the current latent, and of the decode of the quantized copy
       (the print's recon and recon_q): weighted, and per texture */
    double mse, mse_tex[NTCB_MAX_T];
    double mse_q, mse_q_tex[NTCB_MAX_T];
    /* bitrate_stats (main.cpp:2272-2352) as the progress print calls it: the order-0 entropy of level 0 stands
       in for its context-model figure (g_ctx_stats off), so bpp_q8_ctx and bpp_ctx_level0 carry that */
    double bpp_fp32, bpp_q8, bpp_q8_ent, bpp_q8_ctx, bpp_ctx_level0, bpp_est, bits_mlp, bits_raw_latent, bits_header;
    /* latent_stats (main.cpp:2212-2217) of each level's training values */
    float lat_mean[NTCB_MAX_LEVELS], lat_sd[NTCB_MAX_LEVELS], lat_max[NTCB_MAX_LEVELS];
    /* --qat: level-0 training values off their channel's grid (main.cpp:4196-4200); 0 without --qat */
    long long qat_off_grid;
    /* 1 when level 0 is DCT-coded and live (set_dct): its quantized copy is the snapped plane and its bits are its
       bit simulator's (dct_analyze, main.cpp:1080, run on the device's symbols as the progress print runs it),
       added to the figures above as bitrate_stats does at main.cpp:2294-2301 */
    int level0_dct;
    /* the bit simulator's totals for that level (bits, all channels): raw, order-0, context, and the header part
       each includes; 0 without a live DCT level */
    double dct_bits_raw, dct_bits_h0, dct_bits_ctx, dct_bits_header;
} ntcb_progress_stats;
/* The progress print's statistics for the current model (main.cpp:4155-4205) without downloading it:
 * level_bits[l] = the post-hoc depth of each continuous level (bitrate_stats' lbits, main.cpp:2288; ignored for
 * the --qat level 0 and for live --qes levels, whose depths the trainer holds), eval_w x eval_h = the evaluation
 * extent of mse_of (0 = the whole image). zq (host, nz floats, may be null) receives the quantized copy
 * bitrate_stats returns (zpost). Returns 0, or -1 when a depth is outside 1..16. Leaves the model unchanged; uses
 * the decode buffer of decode_full. No counterpart in the reference, whose print downloads the model and runs
 * these on the host. */
int ntcb_print_stats(ntcb_trainer* t, const int* level_bits, int eval_w, int eval_h, float* zq, ntcb_progress_stats* out);
/* The same for a drop-in C++ trainer: cpp_trainer points at an initialised ntc_cuda::Trainer. */
int ntcb_cpp_print_stats(void* cpp_trainer, const int* level_bits, int eval_w, int eval_h, float* zq, ntcb_progress_stats* out);

/* ---- .ntcb containers (the reference's --write-ntcb output, layout versions 1 and 2) decoded on the device: the
 * inference-side neighbour of the trainer, replacing the reference's CPU decoder ntc_decode.cpp for this format. */
typedef struct ntcb_container_desc {
    int version, img_w, img_h, src_w, src_h, T, nlevels;
    int nin, nout, nhidden; int hidden[NTCB_MAX_HIDDEN];
    float leak; int clamp_out;
    int lv_W[NTCB_MAX_LEVELS], lv_H[NTCB_MAX_LEVELS], lv_C[NTCB_MAX_LEVELS], lv_nearest[NTCB_MAX_LEVELS];
    int lv_mode[NTCB_MAX_LEVELS];   /* 0 post-hoc grid, 1 --qes grid, 2 --qat palette, 3 DCT symbols */
    int lv_bits[NTCB_MAX_LEVELS];   /* index depth of channel 0 (0 for DCT) */
    int npos; int pos_kind[NTCB_MAX_POS];
    long long nz, nweights;
} ntcb_container_desc;
typedef struct ntcb_decoder ntcb_decoder;
/* Parse and validate a container on the host (no GPU needed): every header field and range, the file length and
 * hash, each section header, sync marker and length, the DCT token stream and the fp16 weights (the refusals of
 * ntcb_read_header / ntcb_restore, main.cpp:2521-2629 and 2762-2855). Returns 0, or -1 with the first problem in
 * err (err_cap bytes, may be null). */
int ntcb_container_info(const uint8_t* bytes, size_t n, ntcb_container_desc* info, char* err, size_t err_cap);
/* Parse, upload and reconstruct the latent of a container on the current device (grid indices unpacked by the
 * device, a DCT-coded level 0 reconstructed from its symbols). Null with the reason in err on refusal. */
ntcb_decoder* ntcb_decoder_open(const uint8_t* bytes, size_t n, char* err, size_t err_cap);
void ntcb_decoder_get_info(const ntcb_decoder* d, ntcb_container_desc* info);
/* The reconstructed latent (nz floats) and the weights (nweights floats, the fp16 values) on the host; either may be null. */
void ntcb_decoder_model(ntcb_decoder* d, float* z, float* w);
/* Decode the image and quantize it as the reference writes its PNGs (lround(clamp(v, 0, 1) * 255)): out receives T
 * planes [crop_h][crop_w][3] (texture-major), the top-left crop (0 = the header's source size). Returns the byte
 * count (out may be null to ask for it), 0 on a bad crop. */
size_t ntcb_decoder_rgb8(ntcb_decoder* d, int crop_w, int crop_h, uint8_t* out, size_t cap);
/* The same into device memory on `stream` (null = the decoder's own), without synchronising. Returns 0 or -1. */
int ntcb_decoder_rgb8_device(ntcb_decoder* d, int crop_w, int crop_h, uint8_t* out_dev, void* stream);
void ntcb_decoder_close(ntcb_decoder* d);
/* The DCT tables the reconstruction uses, from their definitions: basis [64], zigzag [64] and the 16 step tables
 * [16][64] of one channel at quality q (dct_build_steps, main.cpp:747-781); any pointer may be null. */
void ntcb_dct_tables(int q, int dc_step, float* basis, int* zigzag, int* steps);
/* Number of kernels this trainer has launched since creation. */
long long ntcb_launch_count(const ntcb_trainer* t);
/* Which kernels evaluate the ES decodes (mlp_step / ntcb_shard_mlp_eval pairs and the lat_step pass). tensor = 1
 * (the default): tcgen05 MMAs with 3xTF32 products, FP32-level accuracy (fitness within ~1e-6 relative of the
 * exact kernels); tensor = 0: the packed-FP32 kernels, bit-identical per unit to the reference CUDA backend
 * (cuda/ntc_cuda.cu:164-194). The FD step and the selector search always use the exact kernels, and
 * runtime-shaped models (no fixed-shape kernel) always do too. The environment variable NTCB_POP_KERNEL=ffma
 * selects 0 at init for callers of the C++ Trainer. No counterpart in the reference. */
void ntcb_set_pop_kernel(ntcb_trainer* t, int tensor);
/* 1 when ES pairs currently run on the tensor-core kernel, else 0. */
int ntcb_pop_kernel(const ntcb_trainer* t);

/* Population sharding over G ranks (one process and one GPU per rank). A rank evaluates only the pairs
 * [pair_begin, pair_end) of an N-pair ES step, regenerating their noise from the counter, and writes the
 * per-pair fitness (lp, lm) as 2 doubles per pair into fit_dev (a DEVICE buffer of 2 * (pair_end - pair_begin)
 * doubles, on this trainer's stream). After the caller all-gathers every rank's slice into a device buffer of
 * 2 * N doubles (rank order = pair order), ntcb_shard_mlp_apply turns it into the ES gradient and the Adam
 * step; every rank computes the identical update, so the replicas stay bit-identical. */
void ntcb_shard_mlp_eval(ntcb_trainer* t, int it, float sigma, int N, int M, int pair_begin, int pair_end, double* fit_dev);
void ntcb_shard_mlp_apply(ntcb_trainer* t, int it, float sigma, float lr, int N, int M, const double* fit_all_dev);
/* The same step with the ES gradient sharded too (no rank regenerates other ranks' noise). A rank's pair range
 * must start and end on a gradient segment (64 pairs; N > 256); ntcb_shard_es_block_bytes returns the size of
 * its exchange block in bytes, or -1 when the range does not qualify (then use the pair above). The block is
 * [2 * n doubles: (L+, L-) per pair][n / 64 * P floats: the rank's gradient segment sums][zero to 12 bytes of
 * padding to a multiple of 16 bytes]. After the caller
 * all-gathers every rank's block (rank order = pair order, equal n), ntcb_shard_mlp_apply_grad sums all
 * segments in order and runs Adam: the same update, bit for bit, as the single-GPU step. */
long long ntcb_shard_es_block_bytes(const ntcb_trainer* t, int N, int pair_begin, int pair_end);
void ntcb_shard_mlp_eval_grad(ntcb_trainer* t, int it, float sigma, int N, int M, int pair_begin, int pair_end, void* block_dev);
void ntcb_shard_mlp_apply_grad(ntcb_trainer* t, int it, float sigma, float lr, int N, int M, const void* blocks_dev, int world);
/* The FD step (mlp_step_fd) sharded by weight: a rank draws the step's minibatch, evaluates the unperturbed
 * stats pair and the central differences of weights [j_begin, j_end), and writes their (lp, lm) as 2 doubles per
 * weight into fit_dev (DEVICE, 2 * (j_end - j_begin) doubles). After the caller gathers all P weights' pairs in
 * weight order into a device buffer of 2 * P doubles, ntcb_shard_fd_apply runs the FD gradient and Adam
 * identically on every rank. */
void ntcb_shard_fd_eval(ntcb_trainer* t, int it, float h, int M, int j_begin, int j_end, double* fit_dev);
void ntcb_shard_fd_apply(ntcb_trainer* t, float h, float lr, const double* fit_all_dev);
/* The latent ES step sharded by pixel rows: a rank writes the per-pixel loss differences of image rows
 * [row_begin, row_end) for all K pairs into block_dev, a DEVICE buffer laid out [K][(row_end - row_begin) * W].
 * After the caller all-gathers the ranks' blocks (rank order = row order, equal blocks of rows_per_block rows,
 * so one collective carries all K planes), ntcb_shard_lat_apply runs the footprint gathers, Adam and the snap
 * identically on every rank. */
void ntcb_shard_lat_eval(ntcb_trainer* t, float sigma, int K, int row_begin, int row_end, float* block_dev);
void ntcb_shard_lat_apply(ntcb_trainer* t, int it, float sigma, float lr, int K, const float* blocks_dev, int rows_per_block);
/* The latent ES step sharded by texel rows (one ES-trained level, no qes / DCT snap; ntcb_shard_lat_plan
 * returns 0 otherwise, and the pixel-row pair above applies). plan receives {level, ta, tb, pa, pb, n}: rank
 * `rank` of `world` owns texel rows [ta, tb) of the level, evaluates pixel rows [pa, pb) (its footprints: own
 * rows plus a halo), gathers and Adam-updates only its texels, and ntcb_shard_lat_step_rows copies its n updated
 * latent floats (rows [ta, tb), contiguous) into zblock_dev. After the caller all-gathers the blocks (rank order
 * = row order) into the whole level, ntcb_shard_lat_install writes it on every rank. The latent is then
 * bit-identical to the single-GPU step; each rank keeps the Adam moments of its own rows only. */
int ntcb_shard_lat_plan(const ntcb_trainer* t, int world, int rank, long long* plan);
void ntcb_shard_lat_step_rows(ntcb_trainer* t, int it, float sigma, float lr, int K, int world, int rank, float* zblock_dev);
void ntcb_shard_lat_install(ntcb_trainer* t, int level, const float* level_dev);
/* The selector search sharded by level-0 texel rows: a rank searches rows [trow_begin, trow_end) and copies
 * their level-0 values into level0_dev (a DEVICE buffer of the level's W * H * C floats, rows contiguous);
 * after the caller's all-gather, ntcb_shard_qat_apply installs the full level 0 on every rank. */
void ntcb_shard_qat(ntcb_trainer* t, int trow_begin, int trow_end, float* level0_dev);
void ntcb_shard_qat_apply(ntcb_trainer* t, const float* level0_all_dev);

/* Native sharded iteration (addition; no counterpart in the reference, whose backend runs on one GPU).
 * One call runs the body of the reference trainer's CUDA loop (main.cpp:4121-4137: mlp_step or mlp_step_fd,
 * lat_step, qat_search) over `world` ranks, one process and one GPU per rank, with the library's own NCCL
 * communicator: the same per-rank work as the ntcb_shard_* pairs above, each exchange an in-place NCCL
 * all-gather on the trainer's stream into the trainer's own buffers (the ES blocks, the updated latent level
 * or the loss-difference planes, level 0), so nothing crosses the host. The ranks end bit-identical to one GPU
 * running the plain steps.
 *
 * NCCL is loaded with dlopen("libnccl.so.2") on first use. Rank 0 makes an id with ntcb_comm_unique_id and
 * hands its NTCB_COMM_ID_BYTES bytes to the other ranks (any host channel); every rank then calls
 * ntcb_comm_create with the device of its trainer current. Both return 0 / NULL with a reason on failure.
 * NCCL errors inside an iteration print and exit the process, like every other runtime failure. */
#define NTCB_COMM_ID_BYTES 128
typedef struct ntcb_comm ntcb_comm;
int ntcb_comm_unique_id(unsigned char* id, char* why, size_t why_cap);
ntcb_comm* ntcb_comm_create(const unsigned char* id, int world, int rank, char* why, size_t why_cap);
void ntcb_comm_destroy(ntcb_comm* c);
int ntcb_nccl_version(void);
/* Whether ntcb_shard_iteration applies (1) or not (0, reason in why), and which exchange it uses:
 * *mlp_exchange 1 = per-rank blocks of fitness + ES gradient segments (each rank's pair range a whole number of
 * 64-pair segments, N > 256), 2 = fitness only (every rank regenerates all N pairs' noise for the gradient);
 * *lat_exchange 1 = texel rows (ntcb_shard_lat_plan applies), 2 = pixel rows (the image height splits evenly),
 * 0 = no latent step. mlp_mode: 0 none, 1 ES (mlp_step), 2 FD (mlp_step_fd). K = 0 skips the latent step, which
 * is also skipped when no level is ES-trained (--qat with one level); qat != 0 runs the selector search. */
int ntcb_shard_iteration_plan(const ntcb_trainer* t, int world, int rank, int mlp_mode, int N, int M, int K, int qat,
                              int* mlp_exchange, int* lat_exchange, char* why, size_t why_cap);
/* One iteration: mlp_mode 1 = mlp_step(it, mlp_sigma, mlp_lr, N, M), 2 = mlp_step_fd(it, h = mlp_sigma, mlp_lr, M);
 * then lat_step(it, lat_sigma, lat_lr, K) and qat_search() as above. The communicator's device must be the
 * trainer's. Asynchronous on the trainer's stream like the single-GPU steps. */
void ntcb_shard_iteration(ntcb_trainer* t, ntcb_comm* c, int it, int mlp_mode, float mlp_sigma, float mlp_lr, int N, int M, int K,
                          float lat_sigma, float lat_lr, int qat);
/* Peer-memory exchanges for ntcb_shard_iteration (addition): instead of NCCL, each exchange is one kernel that writes
 * this rank's block into every peer's staging buffer over NVLink as 16-byte lines that carry the exchange's epoch
 * beside the data (no separate flag or fence), waits (bounded, a few seconds) until every peer's lines carry the
 * epoch and copies the staged words into place. Set-up: every rank calls
 * ntcb_p2p_export for the (world, N, K, qat) it will iterate with, which allocates its exchange buffer and writes the
 * buffer's CUDA IPC handle (NTCB_P2P_HANDLE_BYTES bytes); the caller gathers the handles of all ranks in rank order
 * (any host channel) and every rank calls ntcb_p2p_import. Both return 0 with a reason on failure (then the
 * iteration keeps using NCCL). A wait that runs out makes the next synchronising call print and exit. The ranks
 * must all have finished their last iteration (a barrier) before any of them destroys its trainer. */
#define NTCB_P2P_HANDLE_BYTES 64
int ntcb_p2p_export(ntcb_trainer* t, int world, int rank, int N, int K, int qat, unsigned char* handle, char* why, size_t why_cap);
int ntcb_p2p_import(ntcb_trainer* t, const unsigned char* handles, int world, int rank, char* why, size_t why_cap);
/* Unmaps the peers' exchange buffers after this rank's stream has drained (the iteration falls back to NCCL). Call it
 * on every rank, then a barrier, before any rank destroys its trainer: a buffer is freed only when no peer maps it. */
void ntcb_p2p_release(ntcb_trainer* t);
/* Bounded-wait control of the peer exchanges (addition; the reference has no multi-GPU path and exits on any runtime
 * failure, cuda/ntc_cuda.cu:55-56). ntcb_p2p_set_poll_limit: how many times an exchange polls one staged line of a
 * peer before it gives up (0 restores the default, 2^22 polls: a few seconds); a wait that runs out sets the
 * trainer's device error word to 2 and the next synchronising call prints and exits. ntcb_p2p_barrier: every rank
 * pushes a token to every peer and waits for all peers' tokens through the same staging, with `polls` as the limit (0:
 * the trainer's limit); it synchronises the trainer's stream and returns the device error word instead of exiting
 * (0 = every peer arrived, 2 = a peer did not arrive in time, 1 = an earlier tensor-core wait had timed out), then
 * clears it. Every rank must call it at the same point of its sequence of exchanges. After a non-zero return the
 * ranks' exchange epochs disagree: release the peer exchange (ntcb_p2p_release) and set it up again before the next
 * sharded iteration. */
void ntcb_p2p_set_poll_limit(ntcb_trainer* t, unsigned polls);
int ntcb_p2p_barrier(ntcb_trainer* t, unsigned polls);

#ifdef __cplusplus
}
#endif
#endif /* NTC_B200_H */
