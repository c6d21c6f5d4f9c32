// The snapped decode copy: the --qes grid snap, the DCT-coded level 0 (clamp, snap, reconstruction,
// the --dct-lambda rate pair) and the --dct-shadow-pull step.
//
// The reference computes these in strict floating point on the host (STRICT_FP_BEGIN in main.cpp: no
// contraction, no reassociation) and checks the device results bit for bit, so every product, sum
// and quotient below is an explicit round-to-nearest intrinsic (__fmul_rn, __fadd_rn, __fsub_rn,
// __fdiv_rn) that nvcc cannot fuse; tables (grid values, DCT basis, step tables) are the host's bit
// patterns, copied.
#include "kernels_snap.h"
#include "noise.cuh"
#include "quant.cuh"

namespace ntcb {

namespace {
inline unsigned blocks_for(long long n, int tpb) { return (unsigned)((n + tpb - 1) / tpb); }
}

// ------------------------------------------------------------------ --qes
// qes_snap_level over every level (main.cpp:485-496; copies for levels without --qes bits), with the
// frozen clamp of the shadow written back.
__global__ void k_qes_snap(DevModel m, const QesTables* __restrict__ q, float* __restrict__ z, float* __restrict__ zq,
                           const float* __restrict__ grid, long long nz) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nz) return;
    int l = 0;
    for (int j = 1; j < m.nlev; j++) if (i >= m.lv[j].off) l = j;
    const int bits = q->live ? q->bits[l] : 0;
    float v = z[i];
    if (bits == 0) { zq[i] = v; return; }
    const int c = (int)((i - m.lv[l].off) % m.lv[l].C);
    const float lo = q->lo[l][c], hi = q->hi[l][c], range = q->range[l][c];
    if (q->frozen) { v = (v < lo) ? lo : v; v = (hi < v) ? hi : v; z[i] = v; }
    const int levels = (1 << bits) - 1;
    zq[i] = grid[q->grid_off[l][c] + qes_index_dev(v, lo, range, levels)];
}

void launch_qes_snap(cudaStream_t s, const DevModel& m, const QesTables* q, float* z, float* zq, const float* grid, long long nz) {
    k_qes_snap<<<blocks_for(nz, 256), 256, 0, s>>>(m, q, z, zq, grid, nz);
    NTCB_CHECK(cudaGetLastError());
}

// ------------------------------------------------------------------ DCT level 0
// dct_clampf (main.cpp:798): NaN maps to lo.
__device__ __forceinline__ float dclamp(float v, float lo, float hi) { if (!(v >= lo)) return lo; if (v > hi) return hi; return v; }

// dct_fwd8 / dct_inv8 (main.cpp:783-796): sequential float sums from 0, inner index ascending.
__device__ __forceinline__ void fwd8(const DctTables& T, const float* w, float* C) {
    float t[64];
    for (int x = 0; x < 8; x++)
        for (int v = 0; v < 8; v++) {
            float s = 0.0f;
            for (int y = 0; y < 8; y++) s = __fadd_rn(s, __fmul_rn(w[x * 8 + y], T.basis[v * 8 + y]));
            t[x * 8 + v] = s;
        }
    for (int u = 0; u < 8; u++)
        for (int v = 0; v < 8; v++) {
            float s = 0.0f;
            for (int x = 0; x < 8; x++) s = __fadd_rn(s, __fmul_rn(t[x * 8 + v], T.basis[u * 8 + x]));
            C[u * 8 + v] = s;
        }
}
__device__ __forceinline__ void inv8(const DctTables& T, const float* C, float* w) {
    float t[64];
    for (int x = 0; x < 8; x++)
        for (int v = 0; v < 8; v++) {
            float s = 0.0f;
            for (int u = 0; u < 8; u++) s = __fadd_rn(s, __fmul_rn(T.basis[u * 8 + x], C[u * 8 + v]));
            t[x * 8 + v] = s;
        }
    for (int x = 0; x < 8; x++)
        for (int y = 0; y < 8; y++) {
            float s = 0.0f;
            for (int v = 0; v < 8; v++) s = __fadd_rn(s, __fmul_rn(T.basis[v * 8 + y], t[x * 8 + v]));
            w[x * 8 + y] = s;
        }
}

// Quantizers (main.cpp:800-821): DC uniform round-half-even; AC plain roundf (half away from zero) for
// the first-order pair or without the dead zone, else the dead-zone rule; dequantizers likewise.
__device__ __forceinline__ bool first_order(int u, int v) { return (u == 1 && v == 0) || (u == 0 && v == 1); }
__device__ __forceinline__ int quant_dc(float d, int S) { return (int)dclamp(rintf(__fdiv_rn(d, (float)S)), -1024.0f, 1024.0f); }
__device__ __forceinline__ float dequant_dc(int q, int S) { return __fmul_rn((float)q, (float)S); }
__device__ __forceinline__ int quant_ac(float d, int L, int u, int v, int dz) {
    if (!dz || first_order(u, v)) return (int)dclamp(roundf(__fdiv_rn(d, (float)L)), -1024.0f, 1024.0f);
    const float s = fabsf(d), tau = __fmul_rn(0.5f, (float)L);
    if (s <= tau) return 0;
    const float qf = __fdiv_rn(__fsub_rn(s, tau), (float)L);
    const int q = (int)dclamp(floorf(__fadd_rn(qf, 0.5f)), 0.0f, 1024.0f);
    return d < 0.0f ? -q : q;
}
__device__ __forceinline__ float dequant_ac(int q, int L, int u, int v, int dz) {
    if (!dz || first_order(u, v)) return __fmul_rn((float)q, (float)L);
    if (q == 0) return 0.0f;
    const float tau = __fmul_rn(0.5f, (float)L);
    const float mag = __fadd_rn(tau, __fmul_rn((float)abs(q), (float)L));
    return q < 0 ? -mag : mag;
}

// The integer token cost model in 1/16 bit (main.cpp:829-848): Exp-Golomb lengths of run + 1 and |q|
// (capped at 256), one bit per sign, two per EOB; the first-order pair weighted lo_w16 / 16.
__device__ __forceinline__ int floor_log2(unsigned v) { int k = 0; while (v >>= 1) k++; return k; }
__device__ __forceinline__ int c_run(int r) { return 16 * (2 * floor_log2((unsigned)(r + 1)) + 1); }
__device__ __forceinline__ int c_mag(int mm) { return 16 * (2 * floor_log2((unsigned)mm) + 1); }
__device__ __forceinline__ int lo_weight(int tok, int p, int lo16) { return p <= 2 ? (tok * lo16 + 8) >> 4 : tok; }
__device__ int block_bits(const DctTables& T, const int16_t* sym) {
    int bits = 0, run = 0, lnz = 0;
    for (int p = 1; p < 64; p++) {
        const int q = sym[T.zigzag[p]];
        if (q == 0) { run++; continue; }
        bits += lo_weight(c_run(run) + c_mag(min(256, abs(q))) + 16, p, T.lo_w16);
        lnz = p; run = 0;
    }
    if (lnz < 63) bits += 32;
    return bits;
}
// dct_truncate_block (main.cpp:850-869): from zigzag 63 down, zero every nonzero AC whose distortion
// increase is below lam16 times its token saving.
__device__ int truncate_block(const DctTables& T, const float* Cf, const int* st, float lam16, int16_t* sym) {
    int ntrunc = 0, next = 64;
    for (int p = 63; p >= 1; p--) {
        const int k = T.zigzag[p], q = sym[k];
        if (q == 0) continue;
        int prev = 0;
        for (int j = p - 1; j >= 1; j--) if (sym[T.zigzag[j]] != 0) { prev = j; break; }
        const int r1 = p - prev - 1;
        const int token = lo_weight(c_run(r1) + c_mag(min(256, abs(q))) + 16, p, T.lo_w16);
        const int saved = next == 64 ? token - (p == 63 ? 32 : 0) : token + c_run(next - p - 1) - c_run(next - p - 1 + r1 + 1);
        const float v = dequant_ac(q, st[k], k / 8, k % 8, T.deadzone), c = Cf[k];
        const float dD = __fsub_rn(__fmul_rn(c, c), __fmul_rn(__fsub_rn(c, v), __fsub_rn(c, v)));
        if (dD < __fmul_rn(lam16, (float)saved)) { sym[k] = 0; ntrunc++; }
        else next = p;
    }
    return ntrunc;
}
// dct_quantize_block (main.cpp:871-882).
__device__ int quantize_block(const DctTables& T, const float* Cf, const int* st, float lam16, bool with_bits, int16_t* sym,
                              int* ntrunc, int* nz_before) {
    for (int k = 0; k < 64; k++) sym[k] = (int16_t)(k == 0 ? quant_dc(Cf[0], T.dc_step) : quant_ac(Cf[k], st[k], k / 8, k % 8, T.deadzone));
    int nt = 0, nz = 0;
    if (lam16 > 0.0f) {
        for (int k = 1; k < 64; k++) if (sym[k] != 0) nz++;
        nt = truncate_block(T, Cf, st, lam16, sym);
    }
    *ntrunc = nt; *nz_before = nz;
    return with_bits ? block_bits(T, sym) : 0;
}
// dct_recon_block (main.cpp:899-916) for (block, channel) i: dequantize, inverse DCT, zq = clamp(w / 32 - 1).
__device__ void recon_block(const DevModel& m, const DctTables& T, long long i, const int16_t* __restrict__ sym,
                            const uint8_t* __restrict__ code, const int* __restrict__ steps, float* __restrict__ zq) {
    const long long b = i / T.C; const int c = (int)(i % T.C);
    const int bx = (int)(b % T.BW), by = (int)(b / T.BW);
    const DevLevel& L0 = m.lv[0];
    const int* st = steps + ((long long)c * 16 + min((int)code[i], 15)) * 64;
    const int16_t* sy = sym + i * 64;
    float Cf[64], w[64];
    for (int k = 0; k < 64; k++) Cf[k] = k == 0 ? dequant_dc(sy[0], T.dc_step) : dequant_ac(sy[k], st[k], k / 8, k % 8, T.deadzone);
    inv8(T, Cf, w);
    for (int y = 0; y < 8; y++)
        for (int x = 0; x < 8; x++) {
            const long long idx = L0.off + (((long long)(by * 8 + y) * L0.W + (bx * 8 + x)) * L0.C + c);
            zq[idx] = dclamp(__fsub_rn(__fdiv_rn(w[y * 8 + x], 32.0f), 1.0f), -1.0f, 1.0f);
        }
}

// dct_clamp_level0 (main.cpp:974-977) applied to the shadow, and the clamped value copied into the decode buffer.
__global__ void k_dct_clamp0(float* __restrict__ z, float* __restrict__ zq, long long off, long long n0) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n0) return;
    const float v = dclamp(z[off + i], -1.0f, 1.0f);
    z[off + i] = v; zq[off + i] = v;
}
void launch_dct_clamp0(cudaStream_t s, float* z, float* zq, long long off, long long n0) {
    k_dct_clamp0<<<blocks_for(n0, 256), 256, 0, s>>>(z, zq, off, n0);
    NTCB_CHECK(cudaGetLastError());
}

// dct_snap_block (main.cpp:918-934), one thread per (block, channel): clamp the 64 shadow values in place,
// w = (s + 1) * 32, forward DCT, quantize (+ truncation), store the symbols, reconstruct into zq. cnt[0] /
// cnt[1] accumulate the truncation count and the pre-truncation nonzero ACs (integer adds).
__global__ void k_dct_snap(DevModel m, DctTables T, float* __restrict__ z, float* __restrict__ zq, int16_t* __restrict__ sym,
                           const uint8_t* __restrict__ code, const int* __restrict__ steps, const float* __restrict__ lam_t16,
                           int32_t* __restrict__ bits, int* __restrict__ cnt) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)T.BW * T.BH * T.C) return;
    const long long b = i / T.C; const int c = (int)(i % T.C);
    const int bx = (int)(b % T.BW), by = (int)(b / T.BW);
    const DevLevel& L0 = m.lv[0];
    float w[64], Cf[64];
    for (int y = 0; y < 8; y++)
        for (int x = 0; x < 8; x++) {
            const long long idx = L0.off + (((long long)(by * 8 + y) * L0.W + (bx * 8 + x)) * L0.C + c);
            const float sv = dclamp(z[idx], -1.0f, 1.0f);
            z[idx] = sv;
            w[y * 8 + x] = __fmul_rn(__fadd_rn(sv, 1.0f), 32.0f);
        }
    fwd8(T, w, Cf);
    const int cd = min((int)code[i], 15);
    int16_t* sy = sym + i * 64;
    int nt = 0, nz = 0;
    quantize_block(T, Cf, steps + ((long long)c * 16 + cd) * 64, lam_t16[cd], false, sy, &nt, &nz);
    if (T.rate_on) {
        bits[i] = block_bits(T, sy);
        if (nt) atomicAdd(cnt, nt);
        if (nz) atomicAdd(cnt + 1, nz);
    }
    recon_block(m, T, i, sym, code, steps, zq);
}
void launch_dct_snap(cudaStream_t s, const DevModel& m, const DctTables& T, float* z, float* zq, int16_t* sym, const uint8_t* code,
                     const int* steps, const float* lam_t16, int32_t* bits, int* cnt) {
    const long long n = (long long)T.BW * T.BH * T.C;
    k_dct_snap<<<blocks_for(n, 128), 128, 0, s>>>(m, T, z, zq, sym, code, steps, lam_t16, bits, cnt);
    NTCB_CHECK(cudaGetLastError());
}

// dct_recon_level0 (main.cpp:959-972) from uploaded symbols; with the rate term on, also the proxy bits.
__global__ void k_dct_recon(DevModel m, DctTables T, const int16_t* __restrict__ sym, const uint8_t* __restrict__ code,
                            const int* __restrict__ steps, float* __restrict__ zq, int32_t* __restrict__ bits) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)T.BW * T.BH * T.C) return;
    if (T.rate_on) bits[i] = block_bits(T, sym + i * 64);
    recon_block(m, T, i, sym, code, steps, zq);
}
void launch_dct_recon(cudaStream_t s, const DevModel& m, const DctTables& T, const int16_t* sym, const uint8_t* code,
                      const int* steps, float* zq, int32_t* bits) {
    const long long n = (long long)T.BW * T.BH * T.C;
    k_dct_recon<<<blocks_for(n, 128), 128, 0, s>>>(m, T, sym, code, steps, zq, bits);
    NTCB_CHECK(cudaGetLastError());
}

// --dct-lambda part A (dct_rate_block twice, main.cpp:884-897 and 1944): for every (block, channel) and every
// pair k, the proxy bits of snap(clamp(z +- sg eps_k)) on the shadow; dbits[k][i] = bits+ - bits-, hits counts
// the nonzero differences. eps is the latent noise buffer (eps[k][flat index]).
__global__ void k_dct_rate_pairs(DevModel m, DctTables T, float sg, const float* __restrict__ z, const float* __restrict__ eps,
                                 long long nz, const uint8_t* __restrict__ code, const int* __restrict__ steps,
                                 const float* __restrict__ lam_t16, int32_t* __restrict__ dbits, int* __restrict__ hits) {
    const long long n = (long long)T.BW * T.BH * T.C;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const int k = blockIdx.y;
    if (i >= n) return;
    const long long b = i / T.C; const int c = (int)(i % T.C);
    const int bx = (int)(b % T.BW), by = (int)(b / T.BW);
    const DevLevel& L0 = m.lv[0];
    const int cd = min((int)code[i], 15);
    const int* st = steps + ((long long)c * 16 + cd) * 64;
    const float* ek = eps + (long long)k * nz;
    float w[64], Cf[64]; int16_t sy[64];
    int bb[2];
    for (int sgn = 0; sgn < 2; sgn++) {
        for (int y = 0; y < 8; y++)
            for (int x = 0; x < 8; x++) {
                const long long idx = L0.off + (((long long)(by * 8 + y) * L0.W + (bx * 8 + x)) * L0.C + c);
                const float d = __fmul_rn(sg, ek[idx]);
                const float sv = dclamp(sgn == 0 ? __fadd_rn(z[idx], d) : __fsub_rn(z[idx], d), -1.0f, 1.0f);
                w[y * 8 + x] = __fmul_rn(__fadd_rn(sv, 1.0f), 32.0f);
            }
        fwd8(T, w, Cf);
        int nt, nzb;
        bb[sgn] = quantize_block(T, Cf, st, lam_t16[cd], true, sy, &nt, &nzb);
    }
    dbits[(long long)k * n + i] = bb[0] - bb[1];
    if (bb[0] != bb[1]) atomicAdd(hits, 1);
}
void launch_dct_rate_pairs(cudaStream_t s, const DevModel& m, const DctTables& T, int K, float sg, const float* z, const float* eps,
                           long long nz, const uint8_t* code, const int* steps, const float* lam_t16, int32_t* dbits, int* hits) {
    const long long n = (long long)T.BW * T.BH * T.C;
    dim3 grid(blocks_for(n, 128), (unsigned)K);
    k_dct_rate_pairs<<<grid, 128, 0, s>>>(m, T, sg, z, eps, nz, code, steps, lam_t16, dbits, hits);
    NTCB_CHECK(cudaGetLastError());
}

// --dct-shadow-pull (main.cpp:4142-4146): z += f * (zq - z) on [off, off + n).
__global__ void k_shadow_pull(float* __restrict__ z, const float* __restrict__ zq, long long off, long long n, float f) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) z[off + i] += f * (zq[off + i] - z[off + i]);
}
void launch_shadow_pull(cudaStream_t s, float* z, const float* zq, long long off, long long n, float f) {
    k_shadow_pull<<<blocks_for(n, 256), 256, 0, s>>>(z, zq, off, n, f);
    NTCB_CHECK(cudaGetLastError());
}

}  // namespace ntcb
