// Dense bf16 GEMM on tcgen05 (k3_gemm.cu): shared declarations.
#pragma once

#include "k3_bs.cuh"

namespace k3 {

// X rows (bf16, row stride ldx) TMA can address: K a multiple of 64, 16-byte strides and bases.
bool gemm_bf16_ok(int64_t K, const void* w, int64_t ldw, const void* x, int64_t ldx);

// out[m][n] (+)= sum_k (xh[m][k] (+ xl[m][k])) * w[n][k], fp32 accumulation; xl may be null.
int launch_gemm_bf16(const uint16_t* xh, const uint16_t* xl, int64_t ldx, int64_t M, int64_t K, const uint16_t* w,
                     int64_t ldw, int64_t N, float* out, int64_t ldo, int accumulate, int* status, cudaStream_t s);

}  // namespace k3
