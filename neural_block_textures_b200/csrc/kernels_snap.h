// Launchers of the snapped-decode-copy kernels (kernels_snap.cu).
#pragma once
#include "device_model.cuh"

namespace ntcb {

// --qes tables in device memory (layout of ntc_cuda::QesDesc).
struct QesTables {
    int bits[kMaxLevels];
    int live, frozen;
    float lo[kMaxLevels][64], hi[kMaxLevels][64], range[kMaxLevels][64];
    int grid_off[kMaxLevels][64];
};

// DCT-coded level-0 parameters passed by value (the basis and zigzag are the host's tables).
struct DctTables {
    int C, BW, BH, dc_step, deadzone, lo_w16, rate_on;
    float basis[64];
    int zigzag[64];
};

void launch_qes_snap(cudaStream_t s, const DevModel& m, const QesTables* q, float* z, float* zq, const float* grid, long long nz);
void launch_dct_clamp0(cudaStream_t s, float* z, float* zq, long long off, long long n0);
void launch_dct_snap(cudaStream_t s, const DevModel& m, const DctTables& T, float* z, float* zq, int16_t* sym, const uint8_t* code,
                     const int* steps, const float* lam_t16, int32_t* bits, int* cnt);
void launch_dct_recon(cudaStream_t s, const DevModel& m, const DctTables& T, const int16_t* sym, const uint8_t* code,
                      const int* steps, float* zq, int32_t* bits);
void launch_dct_rate_pairs(cudaStream_t s, const DevModel& m, const DctTables& T, int K, float sg, const float* z, const float* eps,
                           long long nz, const uint8_t* code, const int* steps, const float* lam_t16, int32_t* dbits, int* hits);
void launch_shadow_pull(cudaStream_t s, float* z, const float* zq, long long off, long long n, float f);

}  // namespace ntcb
