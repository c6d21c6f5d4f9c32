/* Test infrastructure (oracle), not product code: a plain-C restatement of the reference trainer's
 * CPU path (main.cpp), used only by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg
 * as the checker. Pinned against the reference's own outputs by tests/test_oracle_pin.py (golden
 * vectors recorded from the reference main.cpp through oracle/ref_shim.cpp).
 *
 * Floating point: compiled with -ffp-contract=off; where the reference's builds fuse a multiply-add
 * (nvcc by default, g++ -ffast-math with FMA) the oracle writes fmaf() explicitly at the same place,
 * so features and every MLP unit before its activation follow one fixed rounding sequence. */
#ifndef NTC_ORACLE_H
#define NTC_ORACLE_H
#include <stddef.h>
#include <stdint.h>

typedef struct { int W, H, C, nearest; long long off; } or_level;
typedef struct {
    int W, H, nlev;
    or_level lv[3];
    int npos;
    int pos_kind[16];
    int nin, nout, nhidden;
    int hidden[8];
    float leak;
    int clamp_out;
    float cw[12];
    float wsum;
    int P;
} or_model;

uint64_t or_mix64(uint64_t x);
uint32_t or_noise_u32(uint64_t seed, uint32_t stream, uint32_t step, uint32_t pair, uint64_t index);
float or_gauss(uint64_t seed, uint32_t stream, uint32_t step, uint32_t pair, uint64_t index);
void or_gauss_block(uint64_t seed, uint32_t stream, uint32_t step, uint32_t pair, uint64_t index0, size_t n, float* out);

void or_features(const or_model* m, const float* z, int px, int py, float* f);
void or_mlp_forward(const or_model* m, const float* p, const float* in, float* out);
void or_decode_full(const or_model* m, const float* p, const float* z, float* img);
void or_decode_err(const or_model* m, const float* p, const float* z, const float* tgt, float* err);
double or_loss_subset(const or_model* m, const float* p, const float* z, const float* tgt, const int* idx, int n);
void or_draw_batch(uint64_t seed, int it, int M, int npix, int* out);
void or_es_fitness(const or_model* m, const float* p, const float* z, const float* tgt, uint64_t seed, int it, float sigma,
                   int pair0, int npairs, const int* idx, int M, double* lp, double* lm);
void or_es_grad(const or_model* m, uint64_t seed, int it, float sigma, int N, const double* dl, float* grad);
void or_adam(float* theta, const float* g, float* mm, float* vv, size_t n, float lr, int t);
void or_fd_dl(const or_model* m, const float* p, const float* z, const float* tgt, const int* idx, int M, float h,
              const int* js, int nj, double* dl, double* hh);
void or_lat_grad(const or_model* m, const float* p, const float* zdec, const float* tgt, uint64_t seed, int step, int K,
                 float sigma, unsigned active_mask, float* grad);
void or_qat_search(const or_model* m, const float* p, float* z, const float* tgt, const int* bits, const float* grid);
int or_qes_index(float v, float lo, float range, int levels);

/* DCT-coded level 0 (main.cpp:783-977). basis[64], zigzag[64], steps [C][16][64]. */
typedef struct { int C, BW, BH, dc_step, deadzone, lo_w16; float basis[64]; int zigzag[64]; } or_dct;
void or_dct_fwd8(const or_dct* T, const float* w, float* C);
void or_dct_inv8(const or_dct* T, const float* C, float* w);
int or_dct_quantize_block(const or_dct* T, const float* Cf, const int* st, float lam16, int with_bits, int16_t* sym, int* ntrunc, int* nz_before);
int or_dct_block_bits(const or_dct* T, const int16_t* sym);
void or_dct_snap_level0(const or_dct* T, const or_model* m, float* z, float* zq, int16_t* sym, const uint8_t* code, const int* steps,
                        const float* lam_t16, int32_t* bits, int* ntrunc, int* nz_before);
void or_dct_recon_level0(const or_dct* T, const or_model* m, float* zq, const int16_t* sym, const uint8_t* code, const int* steps);
int or_dct_rate_block(const or_dct* T, const or_model* m, long long b, int c, const float* z, const float* eps, float sg, float sign,
                      const uint8_t* code, const int* steps, const float* lam_t16);

#endif
