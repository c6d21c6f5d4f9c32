// The statistics of the reference trainer's progress print (main.cpp:4155-4205) on the device: the
// bitrate estimate of the quantized latent (bitrate_stats, main.cpp:2272-2352, in its progress-print form
// without the context-model hashing), the 8-bit image error of a decode (mse_of, main.cpp:1764-1788), the
// latent moments (latent_stats, main.cpp:2212-2217) and the --qat off-grid count. The reference downloads
// the model and runs these on the host at every print; here only histograms and sums leave the device.
//
// Everything that decides a bit is exact: channel min / max (order-free), grid indices and quantized values
// (the strict-FP quantizers of quant.cuh), integer histograms, and integer squared-error sums. The double
// moment sums are reduced per block in a fixed order and finished on the host in block order.
#include "kernels.h"
#include "kernels_snap.h"
#include "quant.cuh"

namespace ntcb {

namespace {

inline unsigned blocks_for(long long n, int tpb) { return (unsigned)((n + tpb - 1) / tpb); }

// Order-preserving int key of a float (signed compare of keys = float compare; -0 keys below +0, which no
// result depends on: both give the same range and quantized values).
__device__ __forceinline__ int fkey(float f) {
    const int i = __float_as_int(f);
    return i >= 0 ? i : i ^ 0x7FFFFFFF;
}
__device__ __forceinline__ float fkey_value(int k) { return __int_as_float(k >= 0 ? k : k ^ 0x7FFFFFFF); }

}  // namespace

// ------------------------------------------------------------------ channel min / max of a level
// lo = min(1e30, z...), hi = max(-1e30, z...) per channel over the level's texels (bitrate_stats' scan,
// main.cpp:2305); NaN never compares below or above, so it is skipped as on the host.
__global__ void k_level_minmax(const float* __restrict__ z, long long ntex, int C, int* __restrict__ mm) {
    __shared__ int slo[kMaxCh], shi[kMaxCh];
    if (threadIdx.x < C) { slo[threadIdx.x] = fkey(1e30f); shi[threadIdx.x] = fkey(-1e30f); }
    __syncthreads();
    for (int c = 0; c < C; c++) {
        int lo = fkey(1e30f), hi = fkey(-1e30f);
        for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < ntex; t += (long long)gridDim.x * blockDim.x) {
            const float v = z[t * C + c];
            if (v == v) { lo = min(lo, fkey(v)); hi = max(hi, fkey(v)); }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
            hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
        }
        if ((threadIdx.x & 31) == 0) { atomicMin(&slo[c], lo); atomicMax(&shi[c], hi); }
    }
    __syncthreads();
    if (threadIdx.x < C) { atomicMin(&mm[2 * threadIdx.x], slo[threadIdx.x]); atomicMax(&mm[2 * threadIdx.x + 1], shi[threadIdx.x]); }
}

__global__ void k_minmax_init(int* mm, int C) {
    const int c = threadIdx.x;
    if (c < C) { mm[2 * c] = fkey(1e30f); mm[2 * c + 1] = fkey(-1e30f); }
}

void launch_level_minmax(cudaStream_t s, const float* z, long long ntex, int C, int* mm) {
    k_minmax_init<<<1, 32, 0, s>>>(mm, C);
    NTCB_CHECK(cudaGetLastError());
    if (ntex <= 0) return;
    const unsigned blocks = (unsigned)std::min<long long>(blocks_for(ntex, 256), 148 * 4);
    k_level_minmax<<<blocks, 256, 0, s>>>(z, ntex, C, mm);
    NTCB_CHECK(cudaGetLastError());
}

// ------------------------------------------------------------------ grid indices, quantized copy, histograms
// One thread per texel, channels in turn (bitrate_stats' per-channel loop, main.cpp:2300-2340):
//   mode 0  post-hoc grid: lo / hi from the min / max keys, range = max(hi - lo, 1e-6), q8_index / q8_value;
//   mode 1  --qat level 0: qat_index of the training value, which is also the returned value;
//   mode 2  --qes level: qes_index on its fitted table, the returned value is the snapped decode value.
// hist[c][qi] counts the indices; with dpcm, rhist[c][(cur - pred) & levels] counts the residuals of the
// predictor floor((left + up) / 2) (left alone on the first row, up alone on the first column, 0 at the origin).
__device__ __forceinline__ int level_index(const LevelQuantArgs& a, int c, float v, float lo, float range, int levels) {
    if (a.mode == 1) return qat_index(v, a.bits[c]);
    if (a.mode == 2) return qes_index_dev(v, lo, range, levels);
    return q8_index_dev(v, lo, range, levels);
}

__global__ void k_level_quant(LevelQuantArgs a, int use_smem) {
    extern __shared__ int sh[];   // [2][C][hstride] when use_smem
    const long long ntex = (long long)a.W * a.H;
    const int hs = a.hstride, C = a.C;
    int* hist = a.hist;
    int* rhist = a.rhist;
    if (use_smem) {
        for (int i = threadIdx.x; i < 2 * C * hs; i += blockDim.x) sh[i] = 0;
        __syncthreads();
        hist = sh;
        rhist = sh + C * hs;
    }
    for (int c = 0; c < C; c++) {
        const int levels = (1 << a.bits[c]) - 1;
        float lo = a.lo[c], range = a.range[c];
        if (a.mode == 0) {
            lo = fkey_value(a.minmax[2 * c]);
            const float hi = fkey_value(a.minmax[2 * c + 1]);
            range = fmaxf(__fsub_rn(hi, lo), 1e-6f);
        }
        for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < ntex; t += (long long)gridDim.x * blockDim.x) {
            const long long i = t * C + c;
            const float v = a.z[i];
            const int qi = level_index(a, c, v, lo, range, levels);
            a.zq[i] = a.mode == 0 ? q8_value_dev(qi, lo, range, levels) : (a.mode == 1 ? v : a.zd[i]);
            atomicAdd(&hist[c * hs + qi], 1);
            if (a.dpcm) {
                const int x = (int)(t % a.W), y = (int)(t / a.W);
                const int lf = x ? level_index(a, c, a.z[i - C], lo, range, levels) : -1;
                const int up = y ? level_index(a, c, a.z[i - (long long)a.W * C], lo, range, levels) : -1;
                const int pred = (lf >= 0 && up >= 0) ? (lf + up) / 2 : (lf >= 0 ? lf : (up >= 0 ? up : 0));
                atomicAdd(&rhist[c * hs + ((qi - pred) & levels)], 1);
            }
        }
    }
    if (use_smem) {
        __syncthreads();
        for (int i = threadIdx.x; i < C * hs; i += blockDim.x) {
            if (sh[i]) atomicAdd(&a.hist[i], sh[i]);
            if (a.dpcm && sh[C * hs + i]) atomicAdd(&a.rhist[i], sh[C * hs + i]);
        }
    }
}

void launch_level_quant(cudaStream_t s, const LevelQuantArgs& a) {
    const long long ntex = (long long)a.W * a.H;
    NTCB_CHECK(cudaMemsetAsync(a.hist, 0, (size_t)a.C * a.hstride * sizeof(int), s));
    NTCB_CHECK(cudaMemsetAsync(a.rhist, 0, (size_t)a.C * a.hstride * sizeof(int), s));
    if (ntex <= 0) return;
    const size_t smem = (size_t)2 * a.C * a.hstride * sizeof(int);
    const int use_smem = smem <= 48 * 1024 ? 1 : 0;
    const unsigned blocks = (unsigned)std::min<long long>(blocks_for(ntex, 256), 148 * 4);
    k_level_quant<<<blocks, 256, use_smem ? smem : 0, s>>>(a, use_smem);
    NTCB_CHECK(cudaGetLastError());
}

// ------------------------------------------------------------------ 8-bit image error
// mse_of (main.cpp:1764-1788): both images rounded as save_png does, lround(clamp(x, 0, 1) * 255), and the
// integer squared differences summed per texture over the evaluation extent ew x eh (row stride W pixels).
__global__ void k_mse8(const float* __restrict__ a, const float* __restrict__ b, int W, int ew, int eh, int nc,
                       unsigned long long* __restrict__ sse) {
    const int T = nc / 3;
    unsigned long long acc[kMaxOut / 3];
#pragma unroll
    for (int t = 0; t < kMaxOut / 3; t++) acc[t] = 0ull;
    const long long n = (long long)ew * eh;
    for (long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x; q < n; q += (long long)gridDim.x * blockDim.x) {
        const long long p = (q / ew) * W + (q % ew);
        const float* x = a + p * nc;
        const float* y = b + p * nc;
#pragma unroll
        for (int t = 0; t < kMaxOut / 3; t++) {
            if (t >= T) break;
            unsigned s = 0;
#pragma unroll
            for (int c = 0; c < 3; c++) {
                const int xi = (int)lroundf(fminf(1.0f, fmaxf(0.0f, x[3 * t + c])) * 255.0f);
                const int yi = (int)lroundf(fminf(1.0f, fmaxf(0.0f, y[3 * t + c])) * 255.0f);
                const int d = xi - yi;
                s += (unsigned)(d * d);
            }
            acc[t] += s;
        }
    }
#pragma unroll
    for (int t = 0; t < kMaxOut / 3; t++) {
        if (t >= T) break;
        unsigned long long v = acc[t];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if ((threadIdx.x & 31) == 0 && v) atomicAdd(&sse[t], v);
    }
}

void launch_mse8(cudaStream_t s, const float* a, const float* b, int W, int ew, int eh, int nc, unsigned long long* sse) {
    NTCB_CHECK(cudaMemsetAsync(sse, 0, (size_t)(kMaxOut / 3) * sizeof(unsigned long long), s));
    const long long n = (long long)ew * eh;
    if (n <= 0) return;
    const unsigned blocks = (unsigned)std::min<long long>(blocks_for(n, 256), 148 * 8);
    k_mse8<<<blocks, 256, 0, s>>>(a, b, W, ew, eh, nc, sse);
    NTCB_CHECK(cudaGetLastError());
}

// ------------------------------------------------------------------ latent moments
// latent_stats (main.cpp:2212-2217): sum and sum of squares in double, max |v|, over one level. Block b writes
// part[3 b .. 3 b + 2] = (sum, sum of squares, max |v| as a double); a fixed grid and a fixed in-block tree
// make the result the same on every run.
constexpr int kMomentBlocks = 148 * 2;
__global__ void k_lat_moments(const float* __restrict__ z, long long n, double* __restrict__ part) {
    __shared__ double rs[8], rs2[8];
    __shared__ float rmx[8];
    double s = 0.0, s2 = 0.0;
    float mx = 0.0f;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float v = z[i];
        s += (double)v;
        s2 += (double)v * (double)v;
        mx = fmaxf(mx, fabsf(v));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        s += __shfl_down_sync(0xffffffffu, s, o);
        s2 += __shfl_down_sync(0xffffffffu, s2, o);
        mx = fmaxf(mx, __shfl_down_sync(0xffffffffu, mx, o));
    }
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) { rs[w] = s; rs2[w] = s2; rmx[w] = mx; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int j = 1; j < (int)(blockDim.x >> 5); j++) { s += rs[j]; s2 += rs2[j]; mx = fmaxf(mx, rmx[j]); }
        part[3 * blockIdx.x] = s;
        part[3 * blockIdx.x + 1] = s2;
        part[3 * blockIdx.x + 2] = (double)mx;
    }
}

int lat_moment_blocks() { return kMomentBlocks; }

void launch_lat_moments(cudaStream_t s, const float* z, long long n, double* part) {
    k_lat_moments<<<kMomentBlocks, 256, 0, s>>>(z, n, part);
    NTCB_CHECK(cudaGetLastError());
}

// ------------------------------------------------------------------ --qat off-grid count
// The print's invariant check (main.cpp:4196-4200): level-0 values whose grid snap qat_value(qat_index(v))
// differs from the value. grid = the 9 x 257 --qat table, bits[c] per channel.
__global__ void k_qat_offgrid(const float* __restrict__ z, long long n, int C, const int* __restrict__ bits,
                              const float* __restrict__ grid, unsigned long long* __restrict__ count) {
    unsigned long long k = 0;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float v = z[i];
        const int b = bits[i % C];
        k += grid[b * 257 + qat_index(v, b)] != v ? 1ull : 0ull;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) k += __shfl_xor_sync(0xffffffffu, k, o);
    if ((threadIdx.x & 31) == 0 && k) atomicAdd(count, k);
}

void launch_qat_offgrid(cudaStream_t s, const float* z, long long n, int C, const int* bits, const float* grid,
                        unsigned long long* count) {
    NTCB_CHECK(cudaMemsetAsync(count, 0, sizeof(unsigned long long), s));
    if (n <= 0) return;
    const unsigned blocks = (unsigned)std::min<long long>(blocks_for(n, 256), 148 * 4);
    k_qat_offgrid<<<blocks, 256, 0, s>>>(z, n, C, bits, grid, count);
    NTCB_CHECK(cudaGetLastError());
}

// One thread per (block, channel): the block's DC residual and scale code, then its ACs in zigzag order as
// (run, |q|) tokens with the zigzag position of the previous nonzero as context, and an EOB unless the last
// nonzero sits at position 63 (the walk of dct_analyze's first pass, main.cpp:1100-1119). The small tables are
// counted in shared memory and added to the channel's histograms once per CTA; the context tables, which are
// sparse, take global atomics directly.
__global__ void k_dct_tokens(DctTables T, const int16_t* __restrict__ sym, const uint8_t* __restrict__ code, int* __restrict__ hist) {
    constexpr int kSmall = 65 + 257;               // run, mag: the global offsets of these equal the shared ones
    constexpr int kShared = kSmall + 4097 + 16;    // + dcres, code (contiguous in both layouts)
    __shared__ int sh[kShared];
    __shared__ int cnt[3];
    const int c = blockIdx.y;
    for (int i = threadIdx.x; i < kShared; i += blockDim.x) sh[i] = 0;
    if (threadIdx.x < 3) cnt[threadIdx.x] = 0;
    __syncthreads();
    int* H = hist + (long long)c * kDctHistInts;
    const long long nb = (long long)T.BW * T.BH;
    const long long b = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    int nrun = 0, neob = 0, nover = 0;
    if (b < nb) {
        const int16_t* s = sym + (b * T.C + c) * 64;
        const int bx = (int)(b % T.BW), by = (int)(b / T.BW);
        const int pred = bx > 0 ? sym[((b - 1) * T.C + c) * 64] : (by > 0 ? sym[((b - T.BW) * T.C + c) * 64] : 0);
        atomicAdd(&sh[kSmall + max(0, min(4096, (int)s[0] - pred + 2048))], 1);
        atomicAdd(&sh[kSmall + 4097 + min((int)code[b * T.C + c], 15)], 1);
        int run = 0, prev = 0, lnz = 0;
        for (int p = 1; p < 64; p++) {
            const int q = s[T.zigzag[p]];
            if (q == 0) { run++; continue; }
            const int aq = abs(q), mag = min(256, aq);
            if (aq > 256) nover++;
            atomicAdd(&sh[kDctRun + run], 1);
            atomicAdd(&sh[kDctMag + mag], 1);
            atomicAdd(&H[kDctCtxRun + prev * 65 + run], 1);
            atomicAdd(&H[kDctCtxMag + prev * 257 + mag], 1);
            nrun++; lnz = p; prev = p; run = 0;
        }
        if (lnz < 63) {
            atomicAdd(&sh[kDctRun + 64], 1);
            atomicAdd(&H[kDctCtxRun + prev * 65 + 64], 1);
            neob++;
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        nrun += __shfl_down_sync(0xffffffffu, nrun, o);
        neob += __shfl_down_sync(0xffffffffu, neob, o);
        nover += __shfl_down_sync(0xffffffffu, nover, o);
    }
    if ((threadIdx.x & 31) == 0) { atomicAdd(&cnt[0], nrun); atomicAdd(&cnt[1], neob); atomicAdd(&cnt[2], nover); }
    __syncthreads();
    for (int i = threadIdx.x; i < kShared; i += blockDim.x) {
        const int v = sh[i];
        if (v) atomicAdd(&H[i < kSmall ? i : kDctDcres + (i - kSmall)], v);
    }
    if (threadIdx.x < 3 && cnt[threadIdx.x]) atomicAdd(&H[kDctCounts + threadIdx.x], cnt[threadIdx.x]);
}

void launch_dct_tokens(cudaStream_t s, const DctTables& T, const int16_t* sym, const uint8_t* code, int* hist) {
    const long long nb = (long long)T.BW * T.BH;
    if (nb <= 0 || T.C <= 0) return;
    dim3 grid((unsigned)((nb + 255) / 256), (unsigned)T.C);
    k_dct_tokens<<<grid, 256, 0, s>>>(T, sym, code, hist);
    NTCB_CHECK(cudaGetLastError());
}

}  // namespace ntcb
