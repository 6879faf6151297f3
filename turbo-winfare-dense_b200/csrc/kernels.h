// Host-side launchers of the device kernels (internal to the library).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

// ---- repack.cu
size_t g4b_qmat_bytes(int N, int K);
cudaError_t g4b_repack(const uint32_t* W, const uint16_t* S, const uint16_t* B, int N, int K, void* out,
                       cudaStream_t st);

// ---- rowops.cu
// x fp32 [M][ldx] (K used columns) -> B fragments for a K-column GEMM input (K padded to 128).
cudaError_t g4b_bfrag_from_f32(const float* x, int ldx, int M, int K, void* bfrag, cudaStream_t st, bool pdl);
