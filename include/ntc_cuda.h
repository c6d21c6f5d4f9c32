// The training-backend interface of neural_block_textures' trainer (main.cpp), implemented by
// libntc_b200.so. This header declares the same types, field order and member functions as the
// reference's cuda/ntc_cuda.h (lines cited per item), so main.cpp — which fills the description
// structs by field name and calls the Trainer methods — links against this library unchanged
// (same mangled names, same struct layouts; tests/test_abi.py checks the layouts against the
// reference header). Host code only: no CUDA types appear here.
//
// Ownership and errors follow the reference: the Trainer owns every device buffer; host pointers are
// read or written synchronously inside each call and never retained; init() reports an unsupported
// model with false + a reason; any later runtime failure prints a message and exits the process.
#pragma once
#include <stdint.h>
#include <string>
#include <vector>

namespace ntc_cuda {

// Envelope constants (cuda/ntc_cuda.h:14-20).
static const int MAX_LEVELS = 3;     // latent levels
static const int MAX_POS = 16;       // positional feature generators
static const int MAX_OUT = 12;       // MLP outputs: 3 RGB channels x up to 4 textures
static const int MAX_HIDDEN = 8;     // hidden layers
static const int MAX_CH = 16;        // level-0 channels with their own --qat depth
static const int MAX_QES_CH = 64;    // channels of a --qes level
static const int MAX_DCT_CH = 4;     // channels of a DCT-coded level 0

// Positional feature kinds, numbered as main.cpp's PosKind (cuda/ntc_cuda.h:23).
enum PosKindDev { PK_UV, PK_LV1LOCAL };

// One latent level: W x H texels of C channels at float offset `off` of the flat latent, sampled
// bilinearly or (nearest) as a block per texel (cuda/ntc_cuda.h:25).
struct LevelDesc { int W = 0, H = 0, C = 0; size_t off = 0; bool nearest = false; };
struct PosDesc { int kind = 0; };   // cuda/ntc_cuda.h:26

// The model handed to init() (cuda/ntc_cuda.h:29-52).
struct ModelDesc {
    int W = 0, H = 0;                // image size in pixels
    int T = 1;                       // textures of the material (nout = 3T)
    int nlev = 0; LevelDesc lv[MAX_LEVELS];
    int npos = 0; PosDesc pos[MAX_POS];
    int nin = 0, nout = 3;           // MLP input / output widths
    int nhidden = 0; int hidden[MAX_HIDDEN];
    float leak = 0.01f;              // negative slope of the leaky-ReLU hidden activation
    bool clamp_out = false;          // clamp(s + 0.5) output instead of the sigmoid
    float cw[MAX_OUT];               // loss weight per output channel
    float wsum = 1.0f;               // sum of the per-texture weights (loss divisor 3 * wsum)
    int qat_bits[MAX_CH];            // --qat depth per level-0 channel (0 = off)
    int qat = 0;                     // largest --qat depth (0 = off)
    const float* qat_grid = nullptr; // the host's 9 x 257 grid table, copied at init
    int qes_bits[MAX_LEVELS] = { 0, 0, 0 };   // --qes depth per level (0 = continuous)
    int dct = 0, dct_C = 0, dct_N = 8, dct_dc_step = 4;   // DCT-coded level 0 (dct != 0)
    int dct_q[MAX_DCT_CH] = { 0, 0, 0, 0 };               // per-channel quality (informational)
    const float* dct_basis = nullptr;                     // the host's 8 x 8 basis, copied at init
    const int* dct_zigzag = nullptr;                      // zigzag position -> natural index, copied
    int max_pairs = 64;              // largest N mlp_step will see (sizes per-pair buffers)
    int max_batch = 4096;            // largest minibatch M (sizes per-slot buffers)
    uint64_t seed = 1;               // key of every noise draw
};

// --qes tables computed on the host (cuda/ntc_cuda.h:58-64).
struct QesDesc {
    int bits[MAX_LEVELS];
    int live;
    int frozen;
    float lo[MAX_LEVELS][MAX_QES_CH], hi[MAX_LEVELS][MAX_QES_CH], range[MAX_LEVELS][MAX_QES_CH];
    int grid_off[MAX_LEVELS][MAX_QES_CH];
};

// DCT-coded level-0 description uploaded by set_dct (cuda/ntc_cuda.h:69-76).
struct DctDesc {
    int live, C, BW, BH, N, dc_step;
    int rate_es, rate_trunc; float rate_scale; float lam_t16[16];
    int lo_w16;
    int deadzone;
};

// The backend (cuda/ntc_cuda.h:78-132). Every method mirrors the reference method of the same name.
class Trainer {
public:
    Trainer();
    ~Trainer();
    bool init(const ModelDesc& d, const float* z, const float* p, const float* target, std::string& why);
    std::string banner() const;

    void upload_model(const float* z, const float* p);
    void download_model(float* z, float* p);
    void set_qes(const QesDesc& q, const float* grid, size_t grid_n);
    void snap_latent();
    void shadow_pull(size_t off, size_t n, float f);
    void download_zq(float* zq);
    void set_dct(const DctDesc& d, const uint8_t* code, const int16_t* sym, const int* step);
    void download_dct(int16_t* sym, uint8_t* code);
    void download_dct_rate(int32_t* bits, int32_t* dbits_last_pair, int* ntrunc, int* nz_before, int* hits, int* evals);

    void mlp_step(int it, float sigma, float lr, int N, int M);
    void mlp_step_fd(int it, float h, float lr, int M);
    void reset_mlp_adam();
    void mlp_stats(double& batch_loss, double& diff_std);

    void lat_step(int it, float sigma, float lr, int K);
    void qat_search();
    void decode_full(const float* z_host, float* img);

    void debug_last_batch(std::vector<int>& bidx) const;
    void debug_last_dl(std::vector<double>& dl) const;
    void debug_last_zgrad(std::vector<float>& g) const;

    struct Impl;
    Impl* im;
};

}  // namespace ntc_cuda
