#pragma once
#include <cstdint>
#include <cuda_runtime.h>

// Fills a local [rows][K] INT4 G64 block (W [rows][K/8], S/B [rows][K/64]) whose rows are
// global rows row0.. and whose columns start at global column col0 of a Kg-wide matrix.
cudaError_t g4b_synth_qblock(uint32_t* W, uint16_t* S, uint16_t* B, int rows, int K, long long row0, int col0,
                             int Kg, uint64_t seed, uint64_t tensor, bool centered, cudaStream_t st);
// bf16 norm weights 1 + N(0, 0.05).
cudaError_t g4b_synth_norm(uint16_t* out, int n, uint64_t seed, uint64_t tensor, cudaStream_t st);
