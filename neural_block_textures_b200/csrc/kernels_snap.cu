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
__device__ __forceinline__ int floor_log2(unsigned v) { return v ? 31 - __clz(v) : 0; }
__device__ __forceinline__ int c_run(int r) { return 16 * (2 * floor_log2((unsigned)(r + 1)) + 1); }
__device__ __forceinline__ int c_mag(int mm) { return 16 * (2 * floor_log2((unsigned)mm) + 1); }
__device__ __forceinline__ int lo_weight(int tok, int p, int lo16) { return p <= 2 ? (tok * lo16 + 8) >> 4 : tok; }
// The token cost of a nonzero q at zigzag position p after a run of r zeros.
__device__ __forceinline__ int token_cost(const DctTables& T, int r, int q, int p) {
    return lo_weight(c_run(r) + c_mag(min(256, abs(q))) + 16, p, T.lo_w16);
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

// ---- one (block, channel) per group of eight lanes: lane l owns row l (or column l) of the 8 x 8 block in the DCT
// passes, the quantizers and the reconstruction; every value is the reference's own sequence of strict operations
// (each sum from 0 with its inner index ascending), so symbols, plane and rate integers are those of the host code.
// The truncation decisions, sequential in zigzag order, run on the group's lane 0 over the block's nonzero ACs only
// (a 64-bit zigzag mask gathered from the lanes). Shared layout per group: 8 x 8 float tiles with rows 9 words apart
// and groups 184 words apart (= 24 mod 32), so a warp's row and column accesses hit 32 distinct banks.
constexpr int kDctLanes = 8;
constexpr int kDctGroups = 32;                       // groups per CTA (256 threads)
constexpr int kRow = 9;                              // tile row stride (words)
struct alignas(16) DctGroupMem {
    float a[8 * kRow], b[8 * kRow];                  // inputs / row pass / dequantized values; coefficients
    int16_t sym[64];                                 // symbols, natural order (row l at [8 l, 8 l + 8): one 16-byte row)
    float pad[8];
};
static_assert(sizeof(DctGroupMem) == 184 * 4 && sizeof(DctGroupMem) % 16 == 0 && (sizeof(DctGroupMem) / 4) % 32 == 24, "group layout");
struct DctCtaMem { DctGroupMem g[kDctGroups]; float basis[64]; int zz[64]; };
__device__ __forceinline__ int tix(int k) { return (k >> 3) * kRow + (k & 7); }

// The per-CTA copies of the basis and the zigzag order (lane-dependent indices read them from shared memory).
__device__ __forceinline__ void dct_tables_to_shared(const DctTables& T, DctCtaMem& sm) {
    if (threadIdx.x < 64) { sm.basis[threadIdx.x] = T.basis[threadIdx.x]; sm.zz[threadIdx.x] = T.zigzag[threadIdx.x]; }
    __syncthreads();
}

// dct_fwd8 (main.cpp:783-789): C = fwd8(w), w in g.a, C into g.b; g.a is overwritten with the row pass. Lane l: row l
// of the row pass (t[l][v] = sum_y w[l][y] B[v][y]), column l of the column pass (C[u][l] = sum_x t[x][l] B[u][x]).
__device__ __forceinline__ void fwd8_group(const DctTables& T, DctGroupMem& g, int l) {
    float t[8];
#pragma unroll
    for (int v = 0; v < 8; v++) {
        float s = 0.0f;
#pragma unroll
        for (int y = 0; y < 8; y++) s = __fadd_rn(s, __fmul_rn(g.a[l * kRow + y], T.basis[v * 8 + y]));
        t[v] = s;
    }
#pragma unroll
    for (int v = 0; v < 8; v++) g.a[l * kRow + v] = t[v];    // row l is read by lane l alone above
    __syncwarp();
#pragma unroll
    for (int u = 0; u < 8; u++) {
        float s = 0.0f;
#pragma unroll
        for (int x = 0; x < 8; x++) s = __fadd_rn(s, __fmul_rn(g.a[x * kRow + l], T.basis[u * 8 + x]));
        g.b[u * kRow + l] = s;
    }
    __syncwarp();
}

// The zigzag mask of the block's nonzero ACs (bit p for zigzag position p >= 1), on every lane of the group: lane l
// looks at positions 8 l .. 8 l + 7, and three shuffles gather the bytes. With dd, lane l also stores, for each of
// its nonzero positions, the distortion increase of zeroing it (c^2 - (c - v)^2 with v the dequantized value, the
// reference's strict expression) in g.a at the position's slot. All 32 lanes of the warp call it together.
__device__ __forceinline__ unsigned long long group_mask(const DctTables& T, const DctCtaMem& sm, DctGroupMem& g, const int* st, bool dd,
                                                         int l) {
    unsigned mine = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int p = l * 8 + j;
        const int k = sm.zz[p];
        const int q = g.sym[k];
        if (p != 0 && q != 0) {
            mine |= 1u << j;
            if (dd) {
                const float v = dequant_ac(q, st[k], k >> 3, k & 7, T.deadzone), c = g.b[tix(k)];
                g.a[l * kRow + j] = __fsub_rn(__fmul_rn(c, c), __fmul_rn(__fsub_rn(c, v), __fsub_rn(c, v)));
            }
        }
    }
    unsigned long long mask = (unsigned long long)mine << (8 * l);
#pragma unroll
    for (int off = 1; off < kDctLanes; off <<= 1) mask |= __shfl_xor_sync(0xffffffffu, mask, off, kDctLanes);
    return mask;
}
// dct_block_bits (main.cpp:829-848) from the nonzero mask: nonzeros ascending with the zero runs between them, and two
// bits of EOB unless zigzag position 63 holds a nonzero.
__device__ __forceinline__ int mask_bits(const DctTables& T, const DctCtaMem& sm, const DctGroupMem& g, unsigned long long m) {
    int bits = 0, prevp = 0;
    for (; m; m &= m - 1) {
        const int p = __ffsll((long long)m) - 1;
        bits += token_cost(T, p - prevp - 1, g.sym[sm.zz[p]], p);
        prevp = p;
    }
    return prevp < 63 ? bits + 32 : bits;
}

// dct_quantize_block (main.cpp:871-882) with dct_truncate_block (main.cpp:850-869): g.sym = quantize(C in g.b), row l
// per lane; with lam16 > 0, lane 0 walks the nonzero ACs from zigzag 63 down: the nearest nonzero below p is the
// original one (positions below p are not visited yet), the nearest kept one above is the walk's state, and a nonzero
// is zeroed when its distortion increase is below lam16 times its token saving. Lane 0 returns the proxy bits of the
// result (when with_bits) and sets the truncation and pre-truncation nonzero counts.
__device__ __forceinline__ int quantize_group(const DctTables& T, const DctCtaMem& sm, DctGroupMem& g, const int* st, float lam16,
                                              bool with_bits, int l, int* ntrunc, int* nz_before) {
#pragma unroll
    for (int v = 0; v < 8; v++) {
        const int k = l * 8 + v;
        g.sym[k] = (int16_t)(k == 0 ? quant_dc(g.b[0], T.dc_step) : quant_ac(g.b[l * kRow + v], st[k], l, v, T.deadzone));
    }
    __syncwarp();
    const bool trunc = lam16 > 0.0f;
    // the four groups of a warp may hold blocks of different scale codes (lam16 differs): the mask's shuffles run on
    // every lane whenever any group needs them
    const bool need = __any_sync(0xffffffffu, trunc || with_bits);
    const unsigned long long mask = need ? group_mask(T, sm, g, st, trunc, l) : 0ull;
    __syncwarp();
    int bits = 0, nt = 0, nz = 0;
    if (l == 0) {
        unsigned long long fin = mask;
        if (trunc) {
            nz = __popcll(mask);
            int next = 64;
            unsigned long long m = mask;
            while (m) {
                const int p = 63 - __clzll(m);
                m &= ~(1ull << p);                               // m: the original nonzeros below p
                const int prev = m ? 63 - __clzll(m) : 0;
                const int k = sm.zz[p];
                const int r1 = p - prev - 1;
                const int token = token_cost(T, r1, g.sym[k], p);
                const int saved = next == 64 ? token - (p == 63 ? 32 : 0) : token + c_run(next - p - 1) - c_run(next - p - 1 + r1 + 1);
                if (g.a[tix(p)] < __fmul_rn(lam16, (float)saved)) { g.sym[k] = 0; fin &= ~(1ull << p); nt++; }
                else next = p;
            }
        }
        if (with_bits) bits = mask_bits(T, sm, g, fin);
    }
    __syncwarp();
    *ntrunc = nt; *nz_before = nz;
    return bits;
}

// dct_recon_block (main.cpp:899-916) with dct_inv8 (main.cpp:790-796): dequantize g.sym (steps st) into g.a, then lane
// l computes row l of the inverse (t[v] = sum_u B[u][l] C[u][v], w[l][y] = sum_v B[v][y] t[v]) and writes
// zq = clamp(w / 32 - 1) for pixel row by * 8 + l of block (bx, by), channel c.
__device__ __forceinline__ void recon_group(const DevModel& m, const DctTables& T, const DctCtaMem& sm, DctGroupMem& g, const int* st,
                                            int bx, int by, int c, int l, bool live, float* __restrict__ zq) {
#pragma unroll
    for (int v = 0; v < 8; v++) {
        const int k = l * 8 + v;
        g.a[l * kRow + v] = k == 0 ? dequant_dc(g.sym[0], T.dc_step) : dequant_ac(g.sym[k], st[k], l, v, T.deadzone);
    }
    __syncwarp();
    float t[8];
#pragma unroll
    for (int v = 0; v < 8; v++) {
        float s = 0.0f;
#pragma unroll
        for (int u = 0; u < 8; u++) s = __fadd_rn(s, __fmul_rn(sm.basis[u * 8 + l], g.a[u * kRow + v]));
        t[v] = s;
    }
    const DevLevel& L0 = m.lv[0];
#pragma unroll
    for (int y = 0; y < 8; y++) {
        float s = 0.0f;
#pragma unroll
        for (int v = 0; v < 8; v++) s = __fadd_rn(s, __fmul_rn(T.basis[v * 8 + y], t[v]));
        const long long idx = L0.off + (((long long)(by * 8 + l) * L0.W + (bx * 8 + y)) * L0.C + c);
        if (live) zq[idx] = dclamp(__fsub_rn(__fdiv_rn(s, 32.0f), 1.0f), -1.0f, 1.0f);
    }
    __syncwarp();
}

// dct_snap_block (main.cpp:918-934) per (block, channel): clamp the 64 shadow values in place, w = (s + 1) * 32,
// forward DCT, quantize (+ truncation), store the symbols, reconstruct into zq. cnt[0] / cnt[1] accumulate the
// truncation count and the pre-truncation nonzero ACs (integer adds).
__global__ void __launch_bounds__(kDctGroups * kDctLanes) k_dct_snap(DevModel m, DctTables T, float* __restrict__ z, float* __restrict__ zq,
                                                                      int16_t* __restrict__ sym, const uint8_t* __restrict__ code,
                                                                      const int* __restrict__ steps, const float* __restrict__ lam_t16,
                                                                      int32_t* __restrict__ bits, int* __restrict__ cnt) {
    __shared__ DctCtaMem sm;
    dct_tables_to_shared(T, sm);
    const int gi = threadIdx.x / kDctLanes, l = threadIdx.x % kDctLanes;
    DctGroupMem& g = sm.g[gi];
    const long long n = (long long)T.BW * T.BH * T.C;
    const long long i0 = (long long)blockIdx.x * kDctGroups + gi;
    const bool live = i0 < n;
    const long long i = live ? i0 : n - 1;     // dead groups shadow the last block and write nothing
    const long long b = i / T.C; const int c = (int)(i % T.C);
    const int bx = (int)(b % T.BW), by = (int)(b / T.BW);
    const DevLevel& L0 = m.lv[0];
#pragma unroll
    for (int x = 0; x < 8; x++) {
        const long long idx = L0.off + (((long long)(by * 8 + l) * L0.W + (bx * 8 + x)) * L0.C + c);
        const float sv = dclamp(z[idx], -1.0f, 1.0f);
        if (live) z[idx] = sv;
        g.a[l * kRow + x] = __fmul_rn(__fadd_rn(sv, 1.0f), 32.0f);
    }
    __syncwarp();
    fwd8_group(T, g, l);
    const int cd = min((int)code[i], 15);
    const int* st = steps + ((long long)c * 16 + cd) * 64;
    int nt = 0, nz = 0;
    const int bb = quantize_group(T, sm, g, st, lam_t16[cd], T.rate_on != 0, l, &nt, &nz);
    if (live) {
        reinterpret_cast<int4*>(sym + i * 64)[l] = reinterpret_cast<const int4*>(g.sym)[l];   // row l: 8 symbols, 16 bytes
        if (l == 0 && T.rate_on) {
            bits[i] = bb;
            if (nt) atomicAdd(cnt, nt);
            if (nz) atomicAdd(cnt + 1, nz);
        }
    }
    recon_group(m, T, sm, g, st, bx, by, c, l, live, zq);
}
void launch_dct_snap(cudaStream_t s, const DevModel& m, const DctTables& T, float* z, float* zq, int16_t* sym, const uint8_t* code,
                     const int* steps, const float* lam_t16, int32_t* bits, int* cnt) {
    const long long n = (long long)T.BW * T.BH * T.C;
    k_dct_snap<<<blocks_for(n, kDctGroups), kDctGroups * kDctLanes, 0, s>>>(m, T, z, zq, sym, code, steps, lam_t16, bits, cnt);
    NTCB_CHECK(cudaGetLastError());
}

// dct_recon_level0 (main.cpp:959-972) from uploaded symbols; with the rate term on, also the proxy bits.
__global__ void __launch_bounds__(kDctGroups * kDctLanes) k_dct_recon(DevModel m, DctTables T, const int16_t* __restrict__ sym,
                                                                       const uint8_t* __restrict__ code, const int* __restrict__ steps,
                                                                       float* __restrict__ zq, int32_t* __restrict__ bits) {
    __shared__ DctCtaMem sm;
    dct_tables_to_shared(T, sm);
    const int gi = threadIdx.x / kDctLanes, l = threadIdx.x % kDctLanes;
    DctGroupMem& g = sm.g[gi];
    const long long n = (long long)T.BW * T.BH * T.C;
    const long long i0 = (long long)blockIdx.x * kDctGroups + gi;
    const bool live = i0 < n;
    const long long i = live ? i0 : n - 1;
    const long long b = i / T.C; const int c = (int)(i % T.C);
    const int bx = (int)(b % T.BW), by = (int)(b / T.BW);
    reinterpret_cast<int4*>(g.sym)[l] = reinterpret_cast<const int4*>(sym + i * 64)[l];
    __syncwarp();
    const int* st = steps + ((long long)c * 16 + min((int)code[i], 15)) * 64;
    if (T.rate_on) {
        const unsigned long long mask = group_mask(T, sm, g, st, false, l);
        if (l == 0 && live) bits[i] = mask_bits(T, sm, g, mask);
    }
    recon_group(m, T, sm, g, st, bx, by, c, l, live, zq);
}
void launch_dct_recon(cudaStream_t s, const DevModel& m, const DctTables& T, const int16_t* sym, const uint8_t* code,
                      const int* steps, float* zq, int32_t* bits) {
    const long long n = (long long)T.BW * T.BH * T.C;
    k_dct_recon<<<blocks_for(n, kDctGroups), kDctGroups * kDctLanes, 0, s>>>(m, T, sym, code, steps, zq, bits);
    NTCB_CHECK(cudaGetLastError());
}

// --dct-lambda part A (dct_rate_block twice, main.cpp:884-897 and 1944): for every (block, channel) and every
// pair k, the proxy bits of snap(clamp(z +- sg eps_k)) on the shadow; dbits[k][i] = bits+ - bits-, hits counts
// the nonzero differences. eps is the latent noise buffer (eps[k][flat index]).
__global__ void __launch_bounds__(kDctGroups * kDctLanes) k_dct_rate_pairs(DevModel m, DctTables T, float sg, const float* __restrict__ z,
                                                                            const float* __restrict__ eps, long long nz,
                                                                            const uint8_t* __restrict__ code, const int* __restrict__ steps,
                                                                            const float* __restrict__ lam_t16, int32_t* __restrict__ dbits,
                                                                            int* __restrict__ hits) {
    __shared__ DctCtaMem sm;
    dct_tables_to_shared(T, sm);
    const int gi = threadIdx.x / kDctLanes, l = threadIdx.x % kDctLanes;
    DctGroupMem& g = sm.g[gi];
    const long long n = (long long)T.BW * T.BH * T.C;
    const long long i0 = (long long)blockIdx.x * kDctGroups + gi;
    const bool live = i0 < n;
    const long long i = live ? i0 : n - 1;
    const int k = blockIdx.y;
    const long long b = i / T.C; const int c = (int)(i % T.C);
    const int bx = (int)(b % T.BW), by = (int)(b / T.BW);
    const DevLevel& L0 = m.lv[0];
    const int cd = min((int)code[i], 15);
    const int* st = steps + ((long long)c * 16 + cd) * 64;
    const float* ek = eps + (long long)k * nz;
    int bplus = 0, bminus = 0;
#pragma unroll 1
    for (int sgn = 0; sgn < 2; sgn++) {
#pragma unroll
        for (int x = 0; x < 8; x++) {
            const long long idx = L0.off + (((long long)(by * 8 + l) * L0.W + (bx * 8 + x)) * L0.C + c);
            const float d = __fmul_rn(sg, ek[idx]);
            const float sv = dclamp(sgn == 0 ? __fadd_rn(z[idx], d) : __fsub_rn(z[idx], d), -1.0f, 1.0f);
            g.a[l * kRow + x] = __fmul_rn(__fadd_rn(sv, 1.0f), 32.0f);
        }
        __syncwarp();
        fwd8_group(T, g, l);
        int nt, nzb;
        const int bb = quantize_group(T, sm, g, st, lam_t16[cd], true, l, &nt, &nzb);
        if (sgn == 0) bplus = bb; else bminus = bb;
    }
    if (live && l == 0) {
        dbits[(long long)k * n + i] = bplus - bminus;
        if (bplus != bminus) atomicAdd(hits, 1);
    }
}
void launch_dct_rate_pairs(cudaStream_t s, const DevModel& m, const DctTables& T, int K, float sg, const float* z, const float* eps,
                           long long nz, const uint8_t* code, const int* steps, const float* lam_t16, int32_t* dbits, int* hits) {
    const long long n = (long long)T.BW * T.BH * T.C;
    dim3 grid(blocks_for(n, kDctGroups), (unsigned)K);
    k_dct_rate_pairs<<<grid, kDctGroups * kDctLanes, 0, s>>>(m, T, sg, z, eps, nz, code, steps, lam_t16, dbits, hits);
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
