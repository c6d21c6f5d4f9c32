// Test infrastructure (oracle), not product code.
//
// Compiles the reference trainer main.cpp UNMODIFIED (it is #included from the read-only
// reference tree by oracle/Makefile, with its CLI entry point renamed) and exposes its CPU
// training path through a small extern "C" surface, so that
//   * tests/golden/make_golden.py can record golden input/output vectors produced by the
//     reference's own code (Decoder::features / loss_subset / decode_full, MlpTrainer::step and
//     step_fd, LatentTrainer::step, qat_search, qes_snap_level, the DCT snap), and
//   * bench.py --impl reference can time the reference's own OpenMP CPU iteration
//     (MlpTrainer::step + LatentTrainer::step + qat_search, main.cpp:4121-4148) on the host.
// Nothing here is reachable from the product library.
#define main ntc_reference_cli_main
#include "main.cpp"
#undef main

#include <memory>

namespace {

struct RefSession {
    Options o;
    Decoder D;
    Image target;
    MlpTrainer mt;
    LatentTrainer lt;
    std::mt19937 rng;
};

}  // namespace

extern "C" {

// ntc_noise.h draws (the reference's counter-based generator, compiled by the host compiler).
uint32_t ref_noise_u32(uint64_t seed, uint32_t stream, uint32_t step, uint32_t pair, uint64_t index) {
    return ntc_noise_u32(seed, stream, step, pair, index);
}
float ref_noise_gauss(uint64_t seed, uint32_t stream, uint32_t step, uint32_t pair, uint64_t index) {
    return ntc_gauss(seed, stream, step, pair, index);
}
void ref_noise_gauss_block(uint64_t seed, uint32_t stream, uint32_t step, uint32_t pair, uint64_t index0, size_t n, float* out) {
    for (size_t i = 0; i < n; i++) out[i] = ntc_gauss(seed, stream, step, pair, index0 + i);
}

void ref_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#endif
}
int ref_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

// Build a session the way main() does (main.cpp:3478-3565), except that z and p are supplied by
// the caller (so both backends start from identical bytes). lv_* hold nlev entries; qat_ch holds
// lv_C[0] entries when qat > 0. weights holds T per-texture loss weights.
void* ref_session_new(int W, int H, int T, const float* target_rgb, const float* weights,
                      int nlev, const int* lv_W, const int* lv_H, const int* lv_C, const int* lv_nearest,
                      int nhidden, const int* hidden, const char* pos, float leak, int clamp_out,
                      int qat, const int* qat_ch, unsigned seed) {
    auto* s = new RefSession();
    Options& o = s->o;
    o.seed = seed;
    o.rng_hash = true;
    o.hidden.assign(hidden, hidden + nhidden);
    o.leak = leak;
    o.pos = pos;
    o.clamp_out = clamp_out != 0;
    o.qat = qat;
    if (qat > 0) o.qat_ch.assign(qat_ch, qat_ch + lv_C[0]);
    o.weights.assign(weights, weights + T);
    float wsum = 0.0f;
    for (int t = 0; t < T; t++) wsum += o.weights[t];
    o.LW = lv_W[0]; o.LH = lv_H[0]; o.LC = lv_C[0];
    if (nlev > 1) { o.LW2 = lv_W[1]; o.LH2 = lv_H[1]; o.LC2 = lv_C[1]; }
    if (nlev > 2) { o.LW3 = lv_W[2]; o.LH3 = lv_H[2]; o.LC3 = lv_C[2]; }
    s->target.w = W; s->target.h = H; s->target.nc = 3 * T;
    s->target.rgb.assign(target_rgb, target_rgb + (size_t)W * H * 3 * T);
    s->rng.seed(seed);
    Decoder& D = s->D;
    D.opt = &s->o;
    if (!D.pos.parse(o.pos)) { delete s; return nullptr; }
    D.W = W; D.H = H;
    for (int l = 0; l < nlev; l++) D.lat.add(lv_W[l], lv_H[l], lv_C[l], lv_nearest[l] != 0);
    D.qat_bits = o.qat;
    D.qat_ch = o.qat_ch;
    if (o.qat > 0) qat_init_grid();
    D.qes.assign(nlev, QesLevel());
    D.mlp.nout = 3 * T;
    D.mlp.init(D.nin(), o.hidden, s->rng);
    D.mlp.leak = o.leak;
    D.wsum = wsum;
    D.cw.resize(D.mlp.nout);
    for (int c = 0; c < D.mlp.nout; c++) D.cw[c] = o.weights[c / 3];
    s->mt.init(D.mlp.size());
    s->lt.init(D.lat.size());
    return s;
}
void ref_session_free(void* h) { delete static_cast<RefSession*>(h); }

void ref_sizes(void* h, size_t* nz, size_t* P, int* nin, int* nout) {
    auto* s = static_cast<RefSession*>(h);
    *nz = s->D.lat.size(); *P = s->D.mlp.size(); *nin = s->D.nin(); *nout = s->D.mlp.nout;
}
void ref_set_model(void* h, const float* z, const float* p) {
    auto* s = static_cast<RefSession*>(h);
    std::copy(z, z + s->D.lat.size(), s->D.lat.z.begin());
    std::copy(p, p + s->D.mlp.size(), s->D.mlp.p.begin());
    s->D.qes_refresh();
}
void ref_get_model(void* h, float* z, float* p) {
    auto* s = static_cast<RefSession*>(h);
    std::copy(s->D.lat.z.begin(), s->D.lat.z.end(), z);
    std::copy(s->D.mlp.p.begin(), s->D.mlp.p.end(), p);
}
// The reference's MLP initialiser (MLP::init, main.cpp:586-599) and latent draw (main.cpp:3539-3543)
// from std::mt19937(seed): lets tests start both backends from the reference's own initial state.
void ref_init_like_cli(void* h, float lat_init) {
    auto* s = static_cast<RefSession*>(h);
    std::mt19937 rng(s->o.seed);
    std::normal_distribution<float> N(0.0f, lat_init);
    for (auto& z : s->D.lat.z) z = N(rng);
    if (s->o.qat > 0) qat_snap_level0(s->D.lat, s->o.qat_ch);
    s->D.mlp.init(s->D.nin(), s->o.hidden, rng);
}
void ref_qat_grid(float* out /* 9 * 257 */) { qat_init_grid(); memcpy(out, QAT_GRID, sizeof(QAT_GRID)); }

// Decoder::features (main.cpp:1687-1702) on a caller latent.
void ref_features(void* h, const float* z, int px, int py, float* f) {
    static_cast<RefSession*>(h)->D.features(z, px, py, f);
}
// Decoder::decode_full (main.cpp:1712-1718): z == NULL decodes the session's decode buffer.
void ref_decode_full(void* h, const float* p, const float* z, float* img) {
    auto* s = static_cast<RefSession*>(h);
    Image out;
    s->D.decode_full(p ? p : s->D.mlp.p.data(), z ? z : s->D.zdec(), out);
    std::copy(out.rgb.begin(), out.rgb.end(), img);
}
// Decoder::decode_err (main.cpp:1722-1735).
void ref_decode_err(void* h, const float* p, const float* z, float* err) {
    auto* s = static_cast<RefSession*>(h);
    std::vector<float> e;
    s->D.decode_err(p ? p : s->D.mlp.p.data(), z ? z : s->D.zdec(), s->target, e);
    std::copy(e.begin(), e.end(), err);
}
// Decoder::loss_subset (main.cpp:1739-1750) on the session's decode buffer.
double ref_loss_subset(void* h, const float* p, const int* idx, int n) {
    auto* s = static_cast<RefSession*>(h);
    std::vector<int> v(idx, idx + n);
    return s->D.loss_subset(p, s->D.zdec(), s->target, v);
}
// MlpTrainer::step (main.cpp:1836-1876) with --rng hash at iteration `it`; returns the mean batch loss.
double ref_mlp_step(void* h, int it, int N, int M, float sigma, float lr, double* diff_std) {
    auto* s = static_cast<RefSession*>(h);
    s->o.mlp_pairs = N; s->o.mlp_batch = M; s->o.mlp_sigma = sigma; s->o.mlp_lr = lr;
    s->mt.cur_it = it;
    double ds = 0;
    const double l = s->mt.step(s->D, s->target, s->rng, s->o, ds);
    if (diff_std) *diff_std = ds;
    return l;
}
// MlpTrainer::step_fd (main.cpp:1890-1920); returns the unperturbed batch loss.
double ref_mlp_step_fd(void* h, int it, int M, float fd_h, float lr, double* fd_rms) {
    auto* s = static_cast<RefSession*>(h);
    s->o.mlp_batch = M; s->o.mlp_fd_h = fd_h; s->o.mlp_lr = lr;
    s->mt.cur_it = it;
    double ds = 0;
    const double l = s->mt.step_fd(s->D, s->target, s->rng, s->o, ds);
    if (fd_rms) *fd_rms = ds;
    return l;
}
// Per-pair losses L(p + sigma eps_i), L(p - sigma eps_i) on a given minibatch with hash noise, computed the way
// --cuda-check's host side does (main.cpp:3008-3013), in the reference's own compiled code.
void ref_es_fitness(void* h, int it, float sigma, int pair0, int npairs, const int* idx, int M, double* lp, double* lm) {
    auto* s = static_cast<RefSession*>(h);
    const size_t P = s->D.mlp.size();
    std::vector<int> b(idx, idx + M);
    std::vector<float> pp(P), pm(P);
    for (int i = 0; i < npairs; i++) {
        for (size_t k = 0; k < P; k++) {
            const float e = ntc_gauss(s->o.seed, NS_MLP, it, pair0 + i, k);
            pp[k] = s->D.mlp.p[k] + sigma * e; pm[k] = s->D.mlp.p[k] - sigma * e;
        }
        lp[i] = s->D.loss_subset(pp.data(), s->D.zdec(), s->target, b);
        lm[i] = s->D.loss_subset(pm.data(), s->D.zdec(), s->target, b);
    }
}
// Central differences of the weights js on a given minibatch (main.cpp:3024-3033).
void ref_fd_dl(void* h, float fd_h, const int* idx, int M, const int* js, int nj, double* dl) {
    auto* s = static_cast<RefSession*>(h);
    std::vector<int> b(idx, idx + M);
    std::vector<float> pw(s->D.mlp.p);
    for (int q = 0; q < nj; q++) {
        const size_t j = (size_t)js[q];
        const float orig = pw[j], wp = orig + fd_h, wm = orig - fd_h;
        pw[j] = wp; const double lp = s->D.loss_subset(pw.data(), s->D.zdec(), s->target, b);
        pw[j] = wm; const double lm = s->D.loss_subset(pw.data(), s->D.zdec(), s->target, b);
        pw[j] = orig;
        dl[q] = lp - lm;
    }
}
void ref_mlp_reset_adam(void* h) { auto* s = static_cast<RefSession*>(h); s->mt.adam.init(s->D.mlp.size()); }
void ref_last_batch(void* h, int* out) { auto* s = static_cast<RefSession*>(h); std::copy(s->mt.batch.begin(), s->mt.batch.end(), out); }
void ref_mlp_grad(void* h, float* out) { auto* s = static_cast<RefSession*>(h); std::copy(s->mt.grad.begin(), s->mt.grad.end(), out); }
// LatentTrainer::step (main.cpp:1973-2043) with --rng hash; the gradient before Adam is copied out.
void ref_lat_step(void* h, int K, float sigma, float lr, float* grad_out) {
    auto* s = static_cast<RefSession*>(h);
    s->o.lat_pairs = K; s->o.lat_sigma = sigma; s->o.lat_lr = lr;
    s->lt.step(s->D, s->target, s->rng, s->o);
    if (grad_out) std::copy(s->lt.grad.begin(), s->lt.grad.end(), grad_out);
}
int ref_lat_step_no(void* h) { return static_cast<RefSession*>(h)->lt.step_no; }
void ref_set_lat_step_no(void* h, int n) { static_cast<RefSession*>(h)->lt.step_no = n; }
// qat_search (main.cpp:2088-2139).
void ref_qat_search(void* h) { auto* s = static_cast<RefSession*>(h); qat_search(s->D, s->target, s->o.qat_ch); }
void ref_qat_levels_index(float v, int bits, int* out) { *out = qat_index(v, bits); }

// One training iteration of the reference CPU path, as main() runs it (main.cpp:4121-4148) for the
// configurations timed by bench.py: ES (or FD) MLP step, latent ES step (skipped with --qat and a
// single level), selector search when --qat is on.
void ref_iteration(void* h, int it, int N, int M, float mlp_sigma, float mlp_lr, int fd, float fd_h,
                   int K, float lat_sigma, float lat_lr) {
    auto* s = static_cast<RefSession*>(h);
    s->o.mlp_pairs = N; s->o.mlp_batch = M; s->o.mlp_sigma = mlp_sigma; s->o.mlp_lr = mlp_lr;
    s->o.mlp_fd_h = fd_h; s->o.lat_pairs = K; s->o.lat_sigma = lat_sigma; s->o.lat_lr = lat_lr;
    s->mt.cur_it = it;
    double ds = 0;
    if (fd) s->mt.step_fd(s->D, s->target, s->rng, s->o, ds); else s->mt.step(s->D, s->target, s->rng, s->o, ds);
    if (!(s->o.qat > 0 && s->D.lat.lv.size() == 1)) s->lt.step(s->D, s->target, s->rng, s->o);
    if (s->o.qat > 0) qat_search(s->D, s->target, s->o.qat_ch);
}

// Reported image error of a decode (mse_of + psnr_of, main.cpp:1764-1790) against the session target.
double ref_psnr_of_decode(void* h, const float* img) {
    auto* s = static_cast<RefSession*>(h);
    Image a; a.w = s->D.W; a.h = s->D.H; a.nc = s->D.mlp.nout;
    a.rgb.assign(img, img + (size_t)a.w * a.h * a.nc);
    return psnr_of(mse_of(s->target, a, s->o.weights, s->D.wsum).weighted);
}

// ---- the progress print's statistics (main.cpp:4155-4205) ----
// bitrate_stats (main.cpp:2272-2352) as the print calls it (g_ctx_stats off) on the session's model. out receives
// bpp_fp32, bpp_q8, bpp_q8_ent, bpp_q8_ctx, bpp_ctx_level0, bpp_est, bits_mlp, bits_raw_latent, bits_header; zq the
// returned quantized copy (nz floats).
void ref_bitrate_stats(void* h, int qbits, double* out, float* zq) {
    auto* s = static_cast<RefSession*>(h);
    std::vector<float> zpost;
    g_ctx_stats = false;
    const BitrateStats b = bitrate_stats(s->D, qbits, zpost);
    g_ctx_stats = true;
    const double v[9] = { b.bpp_fp32, b.bpp_q8, b.bpp_q8_ent, b.bpp_q8_ctx, b.bpp_ctx_level0, b.bpp_est, b.bits_mlp,
                          b.bits_raw_latent, b.bits_header };
    std::copy(v, v + 9, out);
    if (zq) std::copy(zpost.begin(), zpost.end(), zq);
}
// mse_of (main.cpp:1764-1788) of an image shaped like the target, over the extent ew x eh (0 = whole image);
// tex receives the per-texture figures. Returns the weighted one.
double ref_mse_of(void* h, const float* img, int ew, int eh, double* tex) {
    auto* s = static_cast<RefSession*>(h);
    Image a; a.w = s->D.W; a.h = s->D.H; a.nc = s->D.mlp.nout;
    a.rgb.assign(img, img + (size_t)a.w * a.h * a.nc);
    const Mse m = mse_of(s->target, a, s->o.weights, s->D.wsum, ew, eh);
    if (tex) for (int t = 0; t < a.nc / 3; t++) tex[t] = m.tex[t];
    return m.weighted;
}
// latent_stats (main.cpp:2212-2217) of level l's training values: msm = mean, sd, max |v|.
void ref_latent_stats(void* h, int l, float* msm) {
    auto* s = static_cast<RefSession*>(h);
    latent_stats(s->D.lat.lv[l], s->D.lat.level(l), msm[0], msm[1], msm[2]);
}

// ---- --qes (QES region, main.cpp:414-496) ----
int ref_qes_index(float v, float lo, float range, int levels) { return qes_index(v, lo, range, levels); }
// Fit the ranges of level `l` at `bits` from the shadow, freeze them and snap every level (Decoder::qes_fit_all).
void ref_qes_fit_level(void* h, int l, int bits) {
    auto* s = static_cast<RefSession*>(h);
    s->D.qes[l].bits = bits;
    s->D.qes_on = true;
    s->D.qes_fit_all();
}
void ref_qes_tables(void* h, int l, float* lo, float* hi, float* range, float* grid) {
    auto* s = static_cast<RefSession*>(h);
    const QesLevel& Q = s->D.qes[l];
    std::copy(Q.lo.begin(), Q.lo.end(), lo); std::copy(Q.hi.begin(), Q.hi.end(), hi);
    std::copy(Q.range.begin(), Q.range.end(), range); std::copy(Q.grid.begin(), Q.grid.end(), grid);
}
void ref_qes_refresh(void* h) { static_cast<RefSession*>(h)->D.qes_refresh(); }
void ref_get_zdec(void* h, float* out) {
    auto* s = static_cast<RefSession*>(h);
    std::copy(s->D.zdec(), s->D.zdec() + s->D.lat.size(), out);
}

// ---- DCT region (main.cpp:629-1045) ----
void ref_dct_tables(float* basis /* 64 */, int* zigzag /* 64 */, float* ak /* 16 */) {
    dct_init_tables();
    memcpy(basis, DCT_BASIS, sizeof(DCT_BASIS)); memcpy(zigzag, DCT_ZIGZAG, sizeof(DCT_ZIGZAG)); memcpy(ak, DCT_AK, sizeof(DCT_AK));
}
void ref_dct_build_steps(int q, int dc_step, int* out /* 16 * 64 */) { dct_init_tables(); dct_build_steps(q, 8, dc_step, out); }
void ref_dct_fwd8(const float* w, float* C) { dct_init_tables(); dct_fwd8(w, C); }
void ref_dct_inv8(const float* C, float* w) { dct_init_tables(); dct_inv8(C, w); }
int ref_dct_quantize_block(const float* Cf, const int* st, int dc_step, float lam16, int lo16, int dz, int with_bits,
                           int16_t* sym, int* ntrunc, int* nz_before) {
    dct_init_tables();
    return dct_quantize_block(Cf, st, dc_step, lam16, lo16, dz != 0, with_bits != 0, sym, ntrunc, nz_before);
}
int ref_dct_block_bits(const int16_t* sym, int lo16) { dct_init_tables(); return dct_block_bits(sym, lo16); }
double ref_dct_gain_of_code(int k) { return dct_gain_of_code(k); }
float ref_dct_quality_scale(int q) { return dct_quality_scale(q); }
// Turn on a DCT-coded level 0 the way main() does (main.cpp:3521-3538) with `lambda` already resolved.
void ref_dct_enable(void* h, const int* q, int dc_step, int deadzone, float lambda, int rate_es, int rate_trunc, float lambda_lo) {
    auto* s = static_cast<RefSession*>(h);
    Decoder& D = s->D;
    dct_init_tables();
    D.dct.on = true; D.dct.N = 8; D.dct.dc_step = dc_step; D.dct.C = D.lat.lv[0].C;
    D.dct.deadzone = deadzone != 0;
    D.dct.q.assign(q, q + D.dct.C);
    D.dct.BW = D.W / 8; D.dct.BH = D.H / 8;
    D.dct.sym.assign(D.dct.nblk() * D.dct.C * DCT_NN, 0);
    D.dct.code.assign(D.dct.nblk() * D.dct.C, 0);
    D.dct.step.assign((size_t)D.dct.C * 16 * DCT_NN, 0);
    for (int c = 0; c < D.dct.C; c++) dct_build_steps(D.dct.q[c], D.dct.N, D.dct.dc_step, &D.dct.step[(size_t)c * 16 * DCT_NN]);
    D.dct.lambda = lambda; D.dct.rate_es = rate_es != 0; D.dct.rate_trunc = rate_trunc != 0;
    D.dct.lo_w16 = std::min(16, std::max(0, (int)lround(lambda_lo * 16.0f)));
    for (int k = 0; k < 16; k++) D.dct.lam_t16[k] = D.dct.rate_trunc ? (float)((double)lambda / (dct_gain_of_code(k) * dct_gain_of_code(k) * 16.0)) : 0.0f;
    D.dct.bits.assign(D.dct.nblk() * D.dct.C, 0);
}
// Decoder::dct_fit_all (probe + go live + snap).
void ref_dct_fit(void* h, int it) { static_cast<RefSession*>(h)->D.dct_fit_all(it); }
void ref_dct_state(void* h, int16_t* sym, uint8_t* code, int* step, int32_t* bits, float* lam_t16, int* lo_w16,
                   size_t* last_trunc, size_t* last_nz_before, size_t* rate_hits) {
    auto* s = static_cast<RefSession*>(h);
    const DctLevel& Q = s->D.dct;
    if (sym) std::copy(Q.sym.begin(), Q.sym.end(), sym);
    if (code) std::copy(Q.code.begin(), Q.code.end(), code);
    if (step) std::copy(Q.step.begin(), Q.step.end(), step);
    if (bits) std::copy(Q.bits.begin(), Q.bits.end(), bits);
    if (lam_t16) for (int k = 0; k < 16; k++) lam_t16[k] = Q.lam_t16[k];
    if (lo_w16) *lo_w16 = Q.lo_w16;
    if (last_trunc) *last_trunc = Q.last_truncated;
    if (last_nz_before) *last_nz_before = Q.last_nz_before;
    if (rate_hits) *rate_hits = Q.rate_hits;
}
// dct_analyze (main.cpp:1080) of the session's DCT level as the progress print runs it (g_ctx_stats off):
// out = {raw_total, h0_total, ctx_total, header}.
void ref_dct_analyze(void* h, double* out) {
    auto* s = static_cast<RefSession*>(h);
    const bool keep = g_ctx_stats;
    g_ctx_stats = false;
    const DctStats S = dct_analyze(s->D.dct);
    g_ctx_stats = keep;
    out[0] = S.raw_total; out[1] = S.h0_total; out[2] = S.ctx_total; out[3] = S.header;
}
// Replaces the session's DCT symbols and scale codes (sizes as ref_dct_state's).
void ref_dct_set_symbols(void* h, const int16_t* sym, const uint8_t* code) {
    auto* s = static_cast<RefSession*>(h);
    DctLevel& Q = s->D.dct;
    std::copy(sym, sym + Q.sym.size(), Q.sym.begin());
    std::copy(code, code + Q.code.size(), Q.code.begin());
}
// The --dct-shadow-pull step on the host (main.cpp:4139-4146).
void ref_dct_shadow_pull(void* h, float f) {
    auto* s = static_cast<RefSession*>(h);
    const size_t o0 = s->D.lat.lv[0].off, n0 = s->D.lat.lv[0].size();
    for (size_t i = 0; i < n0; i++) s->D.lat.z[o0 + i] += f * (s->D.zq[o0 + i] - s->D.lat.z[o0 + i]);
    s->D.qes_refresh();
}

}  // extern "C"
