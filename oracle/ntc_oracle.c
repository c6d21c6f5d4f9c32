/* Test infrastructure (oracle), not product code. See ntc_oracle.h. Every function cites the reference
 * code it restates (main.cpp = the reference trainer, cuda/ntc_noise.h = its counter-based noise). */
#include "ntc_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ---- noise (cuda/ntc_noise.h:20-47): splitmix64 output function twice, Box-Muller cosine branch */
uint64_t or_mix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}
static uint64_t key_of(uint64_t seed, uint32_t stream, uint32_t step, uint32_t pair) {
    return or_mix64(seed ^ ((uint64_t)stream << 56) ^ ((uint64_t)step << 32) ^ (uint64_t)pair);
}
static uint64_t draw64(uint64_t key, uint64_t index) { return or_mix64(key + index * 0x9E3779B97F4A7C15ull); }
uint32_t or_noise_u32(uint64_t seed, uint32_t stream, uint32_t step, uint32_t pair, uint64_t index) {
    return (uint32_t)(draw64(key_of(seed, stream, step, pair), index) >> 32);
}
static float gauss_of(uint64_t h) {
    const float u1 = (float)((h >> 40) + 1ull) * (1.0f / 16777216.0f);
    const float u2 = (float)(h & 0xFFFFFFull) * (1.0f / 16777216.0f);
    return sqrtf(-2.0f * logf(u1)) * cosf(6.283185307179586f * u2);
}
float or_gauss(uint64_t seed, uint32_t stream, uint32_t step, uint32_t pair, uint64_t index) {
    return gauss_of(draw64(key_of(seed, stream, step, pair), index));
}
void or_gauss_block(uint64_t seed, uint32_t stream, uint32_t step, uint32_t pair, uint64_t index0, size_t n, float* out) {
    const uint64_t k = key_of(seed, stream, step, pair);
    for (size_t i = 0; i < n; i++) out[i] = gauss_of(draw64(k, index0 + i));
}
static uint32_t uniform_below(uint32_t u, uint32_t n) { return (uint32_t)(((uint64_t)u * (uint64_t)n) >> 32); }

/* ---- geometry (main.cpp:507-547) */
typedef struct { int x0, x1, y0, y1; float fx, fy; } tap_t;
static int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }
static tap_t tap(const or_level* L, float u, float v) {
    tap_t t;
    if (L->nearest) {
        const float x = u * (float)L->W, y = v * (float)L->H;
        const int ix = (int)floorf(x), iy = (int)floorf(y);
        t.fx = x - (float)ix; t.fy = y - (float)iy;
        t.x0 = t.x1 = clampi(ix, 0, L->W - 1);
        t.y0 = t.y1 = clampi(iy, 0, L->H - 1);
        return t;
    }
    const float x = fmaf(u, (float)L->W, -0.5f), y = fmaf(v, (float)L->H, -0.5f);
    const int x0 = (int)floorf(x), y0 = (int)floorf(y);
    t.fx = x - (float)x0; t.fy = y - (float)y0;
    t.x0 = clampi(x0, 0, L->W - 1); t.x1 = clampi(x0 + 1, 0, L->W - 1);
    t.y0 = clampi(y0, 0, L->H - 1); t.y1 = clampi(y0 + 1, 0, L->H - 1);
    return t;
}
static void sample(const or_level* L, const float* zl, const tap_t* t, float* out) {
    const float* a = zl + ((long long)t->y0 * L->W + t->x0) * L->C;
    if (L->nearest) { for (int k = 0; k < L->C; k++) out[k] = a[k]; return; }
    const float* b = zl + ((long long)t->y0 * L->W + t->x1) * L->C;
    const float* c = zl + ((long long)t->y1 * L->W + t->x0) * L->C;
    const float* d = zl + ((long long)t->y1 * L->W + t->x1) * L->C;
    const float w00 = (1.0f - t->fx) * (1.0f - t->fy), w10 = t->fx * (1.0f - t->fy);
    const float w01 = (1.0f - t->fx) * t->fy, w11 = t->fx * t->fy;
    for (int k = 0; k < L->C; k++) out[k] = fmaf(w11, d[k], fmaf(w01, c[k], fmaf(w10, b[k], w00 * a[k])));
}
/* Decoder::features (main.cpp:1687-1702) + PosEnc::encode (main.cpp:1593-1608). */
void or_features(const or_model* m, const float* z, int px, int py, float* f) {
    const float u = ((float)px + 0.5f) / (float)m->W, v = ((float)py + 0.5f) / (float)m->H;
    tap_t t1 = {0, 0, 0, 0, 0.0f, 0.0f};
    int k = 0;
    for (int l = 0; l < m->nlev; l++) {
        const tap_t t = tap(&m->lv[l], u, v);
        if (l == 1) t1 = t;
        sample(&m->lv[l], z + m->lv[l].off, &t, f + k);
        k += m->lv[l].C;
    }
    for (int q = 0; q < m->npos; q++) {
        if (m->pos_kind[q] == 0) { f[k++] = u * 2.0f - 1.0f; f[k++] = v * 2.0f - 1.0f; }
        else { f[k++] = t1.fx * 2.0f - 1.0f; f[k++] = t1.fy * 2.0f - 1.0f; }
    }
}

/* ---- MLP (main.cpp:560, 603-627): s = b; s += w[i] * a[i] (fused), leaky hidden, sigmoid or clamp output */
void or_mlp_forward(const or_model* m, const float* p, const float* in, float* out) {
    float A[128], B[128];
    const float* cur = in;
    float* nxt = A;
    int ncur = m->nin;
    for (int l = 0; l < m->nhidden; l++) {
        const int nh = m->hidden[l];
        const float* b = p + nh * ncur;
        for (int j = 0; j < nh; j++) {
            float s = b[j];
            const float* w = p + j * ncur;
            for (int i = 0; i < ncur; i++) s = fmaf(w[i], cur[i], s);
            nxt[j] = s > 0.0f ? s : m->leak * s;
        }
        p = b + nh;
        cur = nxt; ncur = nh;
        nxt = (nxt == A) ? B : A;
    }
    const float* b = p + m->nout * ncur;
    for (int j = 0; j < m->nout; j++) {
        float s = b[j];
        const float* w = p + j * ncur;
        for (int i = 0; i < ncur; i++) s = fmaf(w[i], cur[i], s);
        if (m->clamp_out) { float v = s + 0.5f; out[j] = v > 1.0f ? 1.0f : (v < 0.0f ? 0.0f : v); }
        else out[j] = 1.0f / (1.0f + expf(-s));
    }
}

/* Decoder::decode_full (main.cpp:1712-1718). */
void or_decode_full(const or_model* m, const float* p, const float* z, float* img) {
    float f[128];
    for (int y = 0; y < m->H; y++)
        for (int x = 0; x < m->W; x++) {
            or_features(m, z, x, y, f);
            or_mlp_forward(m, p, f, img + ((long long)y * m->W + x) * m->nout);
        }
}
/* Decoder::decode_err (main.cpp:1722-1735): float per-pixel error, each term fused into the sum. */
void or_decode_err(const or_model* m, const float* p, const float* z, const float* tgt, float* err) {
    float f[128], o[12];
    for (int y = 0; y < m->H; y++)
        for (int x = 0; x < m->W; x++) {
            const long long i = (long long)y * m->W + x;
            or_features(m, z, x, y, f);
            or_mlp_forward(m, p, f, o);
            float e = 0.0f;
            for (int c = 0; c < m->nout; c++) { const float d = o[c] - tgt[i * m->nout + c]; e = fmaf(m->cw[c], d * d, e); }
            err[i] = e;
        }
}
/* Decoder::loss_subset (main.cpp:1739-1750): double sum of float terms cw[c] * (d * d), / (3 wsum |idx|). */
double or_loss_subset(const or_model* m, const float* p, const float* z, const float* tgt, const int* idx, int n) {
    float f[128], o[12];
    double s = 0.0;
    for (int k = 0; k < n; k++) {
        const int i = idx[k];
        or_features(m, z, i % m->W, i / m->W, f);
        or_mlp_forward(m, p, f, o);
        for (int c = 0; c < m->nout; c++) { const float d = o[c] - tgt[(long long)i * m->nout + c]; s += (double)(m->cw[c] * (d * d)); }
    }
    return s / (3.0 * (double)m->wsum * (double)n);
}

/* MlpTrainer::draw_batch, hash branch (main.cpp:1825-1829). */
void or_draw_batch(uint64_t seed, int it, int M, int npix, int* out) {
    for (int s = 0; s < M; s++) out[s] = (int)uniform_below(or_noise_u32(seed, 3, (uint32_t)it, 0, (uint64_t)s), (uint32_t)npix);
}

/* The per-pair losses of MlpTrainer::step (main.cpp:1850-1861): w +- sigma eps_i, each rounded once (fused). */
void or_es_fitness(const or_model* m, const float* p, const float* z, const float* tgt, uint64_t seed, int it, float sigma,
                   int pair0, int npairs, const int* idx, int M, double* lp, double* lm) {
    float* e = (float*)malloc(sizeof(float) * m->P);
    float* pp = (float*)malloc(sizeof(float) * m->P);
    float* pm = (float*)malloc(sizeof(float) * m->P);
    for (int i = 0; i < npairs; i++) {
        or_gauss_block(seed, 2, (uint32_t)it, (uint32_t)(pair0 + i), 0, (size_t)m->P, e);
        for (int k = 0; k < m->P; k++) { pp[k] = fmaf(sigma, e[k], p[k]); pm[k] = fmaf(-sigma, e[k], p[k]); }
        lp[i] = or_loss_subset(m, pp, z, tgt, idx, M);
        lm[i] = or_loss_subset(m, pm, z, tgt, idx, M);
    }
    free(e); free(pp); free(pm);
}
/* The ES gradient (main.cpp:1867-1873): g_k = sum_i ((float)dl_i * scale) eps_ik, pairs in order, fused. */
void or_es_grad(const or_model* m, uint64_t seed, int it, float sigma, int N, const double* dl, float* grad) {
    float* e = (float*)malloc(sizeof(float) * m->P);
    const float scale = 1.0f / (2.0f * (float)N * sigma);
    for (int k = 0; k < m->P; k++) grad[k] = 0.0f;
    for (int i = 0; i < N; i++) {
        const float w = (float)dl[i] * scale;
        or_gauss_block(seed, 2, (uint32_t)it, (uint32_t)i, 0, (size_t)m->P, e);
        for (int k = 0; k < m->P; k++) grad[k] = fmaf(w, e[k], grad[k]);
    }
    free(e);
}
/* Adam::step (main.cpp:1797-1809) with the step counter t already incremented. */
void or_adam(float* theta, const float* g, float* mm, float* vv, size_t n, float lr, int t) {
    const float b1 = 0.9f, b2 = 0.999f, eps = 1e-8f;
    const float c1 = 1.0f - powf(b1, (float)t), c2 = 1.0f - powf(b2, (float)t);
    for (size_t i = 0; i < n; i++) {
        mm[i] = b1 * mm[i] + (1.0f - b1) * g[i];
        vv[i] = b2 * vv[i] + (1.0f - b2) * g[i] * g[i];
        const float mh = mm[i] / c1, vh = vv[i] / c2;
        theta[i] -= lr * mh / (sqrtf(vh) + eps);
    }
}
/* MlpTrainer::step_fd (main.cpp:1900-1915) for the weights js[0..nj). */
void or_fd_dl(const or_model* m, const float* p, const float* z, const float* tgt, const int* idx, int M, float h,
              const int* js, int nj, double* dl, double* hh) {
    float* pw = (float*)malloc(sizeof(float) * m->P);
    memcpy(pw, p, sizeof(float) * m->P);
    for (int q = 0; q < nj; q++) {
        const int j = js[q];
        const float orig = pw[j], wp = orig + h, wm = orig - h;
        pw[j] = wp; const double lp = or_loss_subset(m, pw, z, tgt, idx, M);
        pw[j] = wm; const double lm = or_loss_subset(m, pw, z, tgt, idx, M);
        pw[j] = orig;
        dl[q] = lp - lm;
        hh[q] = (double)wp - (double)wm;
    }
    free(pw);
}

/* LatentTrainer::step with --rng hash, up to the gradient (main.cpp:1973-2036): K antithetic pairs, every
 * active level perturbed at once, per-pixel error differences scattered to the distinct texels of each
 * active level's tap in raster order, grad += (dtex * scale) * eps (fused). */
void or_lat_grad(const or_model* m, const float* p, const float* zdec, const float* tgt, uint64_t seed, int step, int K,
                 float sigma, unsigned active_mask, float* grad) {
    long long nz = 0;
    for (int l = 0; l < m->nlev; l++) {
        const long long e = m->lv[l].off + (long long)m->lv[l].W * m->lv[l].H * m->lv[l].C;
        if (e > nz) nz = e;
    }
    const long long npix = (long long)m->W * m->H;
    float* eps = (float*)malloc(sizeof(float) * nz);
    float* zp = (float*)malloc(sizeof(float) * nz);
    float* zm = (float*)malloc(sizeof(float) * nz);
    float* ep = (float*)malloc(sizeof(float) * npix);
    float* em = (float*)malloc(sizeof(float) * npix);
    long long maxtex = 0;
    for (int l = 0; l < m->nlev; l++) if ((long long)m->lv[l].W * m->lv[l].H > maxtex) maxtex = (long long)m->lv[l].W * m->lv[l].H;
    float* dtex = (float*)malloc(sizeof(float) * maxtex);
    const float inv_px = 1.0f / (3.0f * m->wsum * (float)m->W * (float)m->H);
    for (long long i = 0; i < nz; i++) grad[i] = 0.0f;
    for (int k = 0; k < K; k++) {
        for (int l = 0; l < m->nlev; l++) {
            const or_level* L = &m->lv[l];
            const long long n = (long long)L->W * L->H * L->C;
            for (long long i = L->off; i < L->off + n; i++) {
                if (active_mask & (1u << l)) {
                    eps[i] = or_gauss(seed, 1, (uint32_t)step, (uint32_t)k, (uint64_t)i);
                    zp[i] = fmaf(sigma, eps[i], zdec[i]);
                    zm[i] = fmaf(-sigma, eps[i], zdec[i]);
                } else { eps[i] = 0.0f; zp[i] = zdec[i]; zm[i] = zdec[i]; }
            }
        }
        or_decode_err(m, p, zp, tgt, ep);
        or_decode_err(m, p, zm, tgt, em);
        for (int l = 0; l < m->nlev; l++) {
            if (!(active_mask & (1u << l))) continue;
            const or_level* L = &m->lv[l];
            const float scale = 1.0f / (2.0f * (float)K * sigma);
            const long long ntex = (long long)L->W * L->H;
            for (long long t = 0; t < ntex; t++) dtex[t] = 0.0f;
            for (int py = 0; py < m->H; py++) {
                const float v = ((float)py + 0.5f) / (float)m->H;
                for (int px = 0; px < m->W; px++) {
                    const float u = ((float)px + 0.5f) / (float)m->W;
                    const float d = (ep[(long long)py * m->W + px] - em[(long long)py * m->W + px]) * inv_px;
                    const tap_t t = tap(L, u, v);
                    dtex[(long long)t.y0 * L->W + t.x0] += d;
                    if (t.x1 != t.x0) dtex[(long long)t.y0 * L->W + t.x1] += d;
                    if (t.y1 != t.y0) {
                        dtex[(long long)t.y1 * L->W + t.x0] += d;
                        if (t.x1 != t.x0) dtex[(long long)t.y1 * L->W + t.x1] += d;
                    }
                }
            }
            for (long long t = 0; t < ntex; t++) {
                const float w = dtex[t] * scale;
                const long long base = L->off + t * L->C;
                for (int c = 0; c < L->C; c++) grad[base + c] = fmaf(w, eps[base + c], grad[base + c]);
            }
        }
    }
    free(eps); free(zp); free(zm); free(ep); free(em); free(dtex);
}

/* qat_index (main.cpp:2060-2064) and qat_search (main.cpp:2088-2139) on the decode buffer z (in place). */
static int qat_index(float v, int bits) {
    const int levels = (1 << bits) - 1;
    const int k = (int)lroundf((v + 1.0f) * 0.5f * (float)levels);
    return k < 0 ? 0 : (k > levels ? levels : k);
}
void or_qat_search(const or_model* m, const float* p, float* z, const float* tgt, const int* bits, const float* grid) {
    const or_level* L = &m->lv[0];
    int* xb = (int*)malloc(sizeof(int) * L->W); int* xe = (int*)malloc(sizeof(int) * L->W);
    int* yb = (int*)malloc(sizeof(int) * L->H); int* ye = (int*)malloc(sizeof(int) * L->H);
    for (int t = 0; t < L->W; t++) { xb[t] = m->W; xe[t] = 0; }
    for (int t = 0; t < L->H; t++) { yb[t] = m->H; ye[t] = 0; }
    for (int px = 0; px < m->W; px++) { const int t = tap(L, ((float)px + 0.5f) / (float)m->W, 0.5f).x0; if (px < xb[t]) xb[t] = px; if (px + 1 > xe[t]) xe[t] = px + 1; }
    for (int py = 0; py < m->H; py++) { const int t = tap(L, 0.5f, ((float)py + 0.5f) / (float)m->H).y0; if (py < yb[t]) yb[t] = py; if (py + 1 > ye[t]) ye[t] = py + 1; }
    float f[128], o[12];
    for (int ty = 0; ty < L->H; ty++)
        for (int tx = 0; tx < L->W; tx++) {
            const int x0 = xb[tx], x1 = xe[tx], y0 = yb[ty], y1 = ye[ty];
            if (x0 >= x1 || y0 >= y1) continue;
            float* zt = z + L->off + ((long long)ty * L->W + tx) * L->C;
            for (int c = 0; c < L->C; c++) {
                const int b = bits[c], levels = (1 << b) - 1;
                double best = 0.0; int best_k = qat_index(zt[c], b);
                for (int pass = 0; pass <= levels + 1; pass++) {
                    const int k = pass == 0 ? best_k : pass - 1;
                    if (pass > 0 && k == best_k) continue;
                    if (k > levels) break;
                    const float val = grid[b * 257 + k];
                    double sum = 0.0;
                    for (int py = y0; py < y1; py++)
                        for (int px = x0; px < x1; px++) {
                            or_features(m, z, px, py, f);
                            f[c] = val;
                            or_mlp_forward(m, p, f, o);
                            const float* tp = tgt + ((long long)py * m->W + px) * m->nout;
                            for (int q = 0; q < m->nout; q++) { const float d = o[q] - tp[q]; sum += (double)(m->cw[q] * (d * d)); }
                        }
                    if (pass == 0) best = sum;
                    else if (sum < best) { best = sum; best_k = k; }
                }
                zt[c] = grid[b * 257 + best_k];
            }
        }
    free(xb); free(xe); free(yb); free(ye);
}

/* qes_index (main.cpp:448-453), strict float. */
int or_qes_index(float v, float lo, float range, int levels) {
    const float r = nearbyintf(((v - lo) / range) * (float)levels);
    return r <= 0.0f ? 0 : (r >= (float)levels ? levels : (int)r);
}

/* ---- DCT (main.cpp:783-977), strict float */
static float dclamp(float v, float lo, float hi) { if (!(v >= lo)) return lo; if (v > hi) return hi; return v; }
void or_dct_fwd8(const or_dct* T, const float* w, float* C) {
    float t[64];
    for (int x = 0; x < 8; x++)
        for (int v = 0; v < 8; v++) { float s = 0.0f; for (int y = 0; y < 8; y++) s += w[x * 8 + y] * T->basis[v * 8 + y]; t[x * 8 + v] = s; }
    for (int u = 0; u < 8; u++)
        for (int v = 0; v < 8; v++) { float s = 0.0f; for (int x = 0; x < 8; x++) s += t[x * 8 + v] * T->basis[u * 8 + x]; C[u * 8 + v] = s; }
}
void or_dct_inv8(const or_dct* T, const float* C, float* w) {
    float t[64];
    for (int x = 0; x < 8; x++)
        for (int v = 0; v < 8; v++) { float s = 0.0f; for (int u = 0; u < 8; u++) s += T->basis[u * 8 + x] * C[u * 8 + v]; t[x * 8 + v] = s; }
    for (int x = 0; x < 8; x++)
        for (int y = 0; y < 8; y++) { float s = 0.0f; for (int v = 0; v < 8; v++) s += T->basis[v * 8 + y] * t[x * 8 + v]; w[x * 8 + y] = s; }
}
static int first_order(int u, int v) { return (u == 1 && v == 0) || (u == 0 && v == 1); }
static int quant_dc(float d, int S) { return (int)dclamp(nearbyintf(d / (float)S), -1024.0f, 1024.0f); }
static float dequant_dc(int q, int S) { return (float)q * (float)S; }
static int quant_ac(float d, int L, int u, int v, int dz) {
    if (!dz || first_order(u, v)) return (int)dclamp(roundf(d / (float)L), -1024.0f, 1024.0f);
    const float s = fabsf(d), tau = 0.5f * (float)L;
    if (s <= tau) return 0;
    const float qf = (s - tau) / (float)L;
    const int q = (int)dclamp(floorf(qf + 0.5f), 0.0f, 1024.0f);
    return d < 0.0f ? -q : q;
}
static float dequant_ac(int q, int L, int u, int v, int dz) {
    if (!dz || first_order(u, v)) return (float)q * (float)L;
    if (q == 0) return 0.0f;
    const float tau = 0.5f * (float)L;
    const float mag = tau + (float)abs(q) * (float)L;
    return q < 0 ? -mag : mag;
}
static int floor_log2(unsigned v) { int k = 0; while (v >>= 1) k++; return k; }
static int c_run(int r) { return 16 * (2 * floor_log2((unsigned)(r + 1)) + 1); }
static int c_mag(int mm) { return 16 * (2 * floor_log2((unsigned)mm) + 1); }
static int lo_weight(int tok, int p, int lo16) { return p <= 2 ? (tok * lo16 + 8) >> 4 : tok; }
static int mini(int a, int b) { return a < b ? a : b; }
int or_dct_block_bits(const or_dct* T, const int16_t* sym) {
    int bits = 0, run = 0, lnz = 0;
    for (int p = 1; p < 64; p++) {
        const int q = sym[T->zigzag[p]];
        if (q == 0) { run++; continue; }
        bits += lo_weight(c_run(run) + c_mag(mini(256, abs(q))) + 16, p, T->lo_w16);
        lnz = p; run = 0;
    }
    if (lnz < 63) bits += 32;
    return bits;
}
static int truncate_block(const or_dct* T, const float* Cf, const int* st, float lam16, int16_t* sym) {
    int ntrunc = 0, next = 64;
    for (int p = 63; p >= 1; p--) {
        const int k = T->zigzag[p], q = sym[k];
        if (q == 0) continue;
        int prev = 0;
        for (int j = p - 1; j >= 1; j--) if (sym[T->zigzag[j]] != 0) { prev = j; break; }
        const int r1 = p - prev - 1;
        const int token = lo_weight(c_run(r1) + c_mag(mini(256, abs(q))) + 16, p, T->lo_w16);
        const int saved = next == 64 ? token - (p == 63 ? 32 : 0) : token + c_run(next - p - 1) - c_run(next - p - 1 + r1 + 1);
        const float v = dequant_ac(q, st[k], k / 8, k % 8, T->deadzone), c = Cf[k];
        const float dD = c * c - (c - v) * (c - v);
        if (dD < lam16 * (float)saved) { sym[k] = 0; ntrunc++; }
        else next = p;
    }
    return ntrunc;
}
int or_dct_quantize_block(const or_dct* T, const float* Cf, const int* st, float lam16, int with_bits, int16_t* sym, int* ntrunc, int* nz_before) {
    for (int k = 0; k < 64; k++) sym[k] = (int16_t)(k == 0 ? quant_dc(Cf[0], T->dc_step) : quant_ac(Cf[k], st[k], k / 8, k % 8, T->deadzone));
    int nt = 0, nz = 0;
    if (lam16 > 0.0f) {
        for (int k = 1; k < 64; k++) if (sym[k] != 0) nz++;
        nt = truncate_block(T, Cf, st, lam16, sym);
    }
    if (ntrunc) *ntrunc = nt;
    if (nz_before) *nz_before = nz;
    return with_bits ? or_dct_block_bits(T, sym) : 0;
}
static void recon_block(const or_dct* T, const or_model* m, long long i, float* zq, const int16_t* sym, const uint8_t* code, const int* steps) {
    const long long b = i / T->C; const int c = (int)(i % T->C);
    const int bx = (int)(b % T->BW), by = (int)(b / T->BW);
    const or_level* L0 = &m->lv[0];
    const int* st = steps + ((long long)c * 16 + code[i]) * 64;
    const int16_t* sy = sym + i * 64;
    float Cf[64], w[64];
    for (int k = 0; k < 64; k++) Cf[k] = k == 0 ? dequant_dc(sy[0], T->dc_step) : dequant_ac(sy[k], st[k], k / 8, k % 8, T->deadzone);
    or_dct_inv8(T, Cf, w);
    for (int y = 0; y < 8; y++)
        for (int x = 0; x < 8; x++) {
            const long long idx = L0->off + ((long long)(by * 8 + y) * L0->W + (bx * 8 + x)) * L0->C + c;
            zq[idx] = dclamp(w[y * 8 + x] / 32.0f - 1.0f, -1.0f, 1.0f);
        }
}
void or_dct_snap_level0(const or_dct* T, const or_model* m, float* z, float* zq, int16_t* sym, const uint8_t* code, const int* steps,
                        const float* lam_t16, int32_t* bits, int* ntrunc, int* nz_before) {
    const long long n = (long long)T->BW * T->BH * T->C;
    const or_level* L0 = &m->lv[0];
    int nt_all = 0, nz_all = 0;
    for (long long i = 0; i < n; i++) {
        const long long b = i / T->C; const int c = (int)(i % T->C);
        const int bx = (int)(b % T->BW), by = (int)(b / T->BW);
        float w[64], Cf[64];
        for (int y = 0; y < 8; y++)
            for (int x = 0; x < 8; x++) {
                const long long idx = L0->off + ((long long)(by * 8 + y) * L0->W + (bx * 8 + x)) * L0->C + c;
                const float s = dclamp(z[idx], -1.0f, 1.0f);
                z[idx] = s;
                w[y * 8 + x] = (s + 1.0f) * 32.0f;
            }
        or_dct_fwd8(T, w, Cf);
        const int cd = code[i];
        int nt = 0, nz = 0;
        or_dct_quantize_block(T, Cf, steps + ((long long)c * 16 + cd) * 64, lam_t16[cd], 0, sym + i * 64, &nt, &nz);
        if (bits) bits[i] = or_dct_block_bits(T, sym + i * 64);
        nt_all += nt; nz_all += nz;
        recon_block(T, m, i, zq, sym, code, steps);
    }
    if (ntrunc) *ntrunc = nt_all;
    if (nz_before) *nz_before = nz_all;
}
void or_dct_recon_level0(const or_dct* T, const or_model* m, float* zq, const int16_t* sym, const uint8_t* code, const int* steps) {
    const long long n = (long long)T->BW * T->BH * T->C;
    for (long long i = 0; i < n; i++) recon_block(T, m, i, zq, sym, code, steps);
}
/* dct_rate_block (main.cpp:884-897): proxy bits of snap(clamp(z + sign (sg eps))) for (block b, channel c);
 * z and eps are flat-latent pointers (level 0 at its offset). */
int or_dct_rate_block(const or_dct* T, const or_model* m, long long b, int c, const float* z, const float* eps, float sg, float sign,
                      const uint8_t* code, const int* steps, const float* lam_t16) {
    const or_level* L0 = &m->lv[0];
    float w[64], Cf[64]; int16_t sym[64];
    const int bx = (int)(b % T->BW), by = (int)(b / T->BW);
    for (int y = 0; y < 8; y++)
        for (int x = 0; x < 8; x++) {
            const long long i = L0->off + ((long long)(by * 8 + y) * L0->W + (bx * 8 + x)) * L0->C + c;
            const float s = dclamp(z[i] + sign * (sg * eps[i]), -1.0f, 1.0f);
            w[y * 8 + x] = (s + 1.0f) * 32.0f;
        }
    or_dct_fwd8(T, w, Cf);
    const int cd = code[b * T->C + c];
    return or_dct_quantize_block(T, Cf, steps + ((long long)c * 16 + cd) * 64, lam_t16[cd], 1, sym, NULL, NULL);
}
