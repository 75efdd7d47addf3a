// Expert-parallel front end: plans from explicit pairs, x conversion for any token count.
#pragma once

#include "k3_moe.cuh"

namespace k3 {

constexpr int kMaxPairCandidates = 1024;

struct PairsArgs {
    const int32_t* slot;          // [n_in] pool slot per candidate pair, < 0 = skip
    const int32_t* tok;           // [n_in] token row
    const float* w;               // [n_in] routing weight
    int n_in;
    int num_slots;
    int T;                        // token rows
    Plan* plan;
    unsigned* cntA;               // arrival counters of the two launches, zeroed here
    int64_t n_cntA;
    unsigned* cntB;
    int64_t n_cntB;
};

int launch_plan_from_pairs(const PairsArgs& a, cudaStream_t s);
int launch_convert_tokens(const void* x, int x_dtype, int64_t T, int64_t K, uint8_t* xp, uint8_t* xsf,
                          cudaStream_t s);

}  // namespace k3
