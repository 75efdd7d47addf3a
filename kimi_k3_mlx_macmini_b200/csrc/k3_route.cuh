// Fused decode front end for the TMA path: router logits, x conversion, top-k + plan.
#pragma once

#include "k3_bs.cuh"
#include "k3_plan.cuh"

namespace k3 {

struct RouteArgs {
    const void* x;                 // router input [M][H]
    int x_dtype;
    int M;
    int64_t H;
    // expert input [M][He] for the E2M1 pieces (block-scaled path); null: x itself. A
    // latent MoE routes on the hidden state and runs its experts on the latent one.
    const void* xe;
    int xe_dtype;
    int64_t He;
    const uint16_t* W;             // router weight, bf16 bits [E][H]
    int64_t E;
    float* logit_part;             // [KQ][M][E] slice partials
    float* logits;                 // [M][E]
    unsigned* done;                // arrival counters [1 + row blocks] and the piece-task counter,
                                   // zeroed before each launch
    __half* xq_hi;                 // blocked x pieces [H/32][8][32]
    __half* xq_lo;                 // null for bf16 x
    float* xq_ts;                  // [8][H/512]
    // block-scaled path: x as E2M1 pieces [8M][H/2] and their per-row scales [8M][H/32]
    // (replaces xq_* when non-null)
    uint8_t* xp;
    uint8_t* xsf;
    // plan_args.keys / .scores [M][E]: written by the row blocks' finishing CTAs (the
    // top-k keys order_key(sigmoid(logit) + bias) and the sigmoid scores), read by the
    // CTA that runs the top-k
    PlanArgs plan_args;
    Plan* plan;
};

// Requirements: H % 512 == 0, H / kq % 512 == 0, M <= 8, E <= 1024.
int launch_route_fused(const RouteArgs& a, int kq, cudaStream_t s);

}  // namespace k3
