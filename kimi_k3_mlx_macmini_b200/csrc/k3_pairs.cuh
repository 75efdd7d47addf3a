// Expert-parallel front end: plans from explicit pairs, x conversion for any token count.
#pragma once

#include "k3_moe.cuh"

namespace k3 {

constexpr int kMaxPairCandidates = 1024;

struct PairsArgs {
    const int32_t* slot;          // [n_in] pool slot per candidate pair, < 0 = skip
    const int32_t* tok;           // [n_in] token row
    const float* w;               // [n_in] routing weight
    // or, with slot == nullptr, candidates from a routing result: candidate i < T*rk is
    // (expert idx[t][j] - expert_lo when in [0, n_local), token t, weight rw[t][j]) with
    // i = t*rk + j and rows rstride elements apart; the next shared_n candidates are
    // (shared_slot, shared_t0 + j, 1)
    const int32_t* ridx;
    const float* rw;
    int rk, rstride, expert_lo, n_local, shared_slot, shared_t0, shared_n;
    int n_in;
    int num_slots;
    int T;                        // token rows
    Plan* plan;
    unsigned* cntA;               // arrival counters of the two launches, zeroed here
    int64_t n_cntA;
    unsigned* cntB;
    int64_t n_cntB;
};

// Candidate i of a PairsArgs: its pool slot (-1 = skip), token row and weight.
__device__ __forceinline__ void pair_candidate(const PairsArgs& a, int i, int& slot, int& tok, float& w) {
    if (a.slot) {
        slot = a.slot[i];
        tok = a.tok[i];
        w = a.w[i];
    } else if (i < a.T * a.rk) {
        const int t = i / a.rk, j = i - t * a.rk;
        const int e = a.ridx[int64_t(t) * a.rstride + j] - a.expert_lo;
        slot = (e >= 0 && e < a.n_local) ? e : -1;
        tok = t;
        w = a.rw[int64_t(t) * a.rstride + j];
    } else {
        slot = a.shared_slot;
        tok = a.shared_t0 + (i - a.T * a.rk);
        w = 1.0f;
    }
    if (slot < 0 || slot >= a.num_slots || tok < 0 || tok >= a.T) slot = -1;
}

// Tokens to convert to E2M1 pieces alongside the plan (xp == nullptr: none).
struct ConvertArgs {
    const void* x;
    int x_dtype;
    int64_t T, K;
    uint8_t* xp;
    uint8_t* xsf;
};
// One launch: CTA 0 builds the plan from the candidates, CTAs 1.. convert the tokens.
int launch_plan_from_pairs(const PairsArgs& a, const ConvertArgs& conv, cudaStream_t s);
int launch_convert_tokens(const void* x, int x_dtype, int64_t T, int64_t K, uint8_t* xp, uint8_t* xsf,
                          cudaStream_t s);

}  // namespace k3
