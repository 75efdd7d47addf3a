// Decode-path data structures shared by the router, plan and grouped-matvec kernels.
#pragma once

#include "k3_common.cuh"

namespace k3 {

constexpr int kMaxTok = 8;                       // decode tokens = mma n8 columns
constexpr int kMaxTopK = 16;
constexpr int kMaxExperts = 1024;
constexpr int kMaxActive = kMaxTok * kMaxTopK + 1;
constexpr int kMaxPairs = kMaxTok * kMaxTopK + kMaxTok;

// Routing plan of one decode call: the active experts in ascending id order (the
// reference's `for e in sorted(...)`, moe.py:120 / k3ref/layers.py:252) and, per
// expert, its (token, weight) pairs in ascending token order. The shared expert, when
// present, is the last active expert with every token at weight 1.
struct Plan {
    int n_active;
    int n_pairs;
    int M;
    int status;
    int expert[kMaxActive];
    int pair_start[kMaxActive + 1];
    int pair_tok[kMaxPairs];
    float pair_w[kMaxPairs];
};

// Grouped-matvec tiling (see k3_moe.cu for the mainloop).
constexpr int kWarps = 8;          // warps per CTA; every warp runs its own items
constexpr int kTiles = 4;          // m16 row tiles per item -> 64 weight rows
constexpr int kItemRows = 16 * kTiles;
constexpr int kStageK = 128;       // k per pipeline stage: 64 packed bytes per row
constexpr int kStages = 3;         // cp.async ring depth per warp

struct Stage {
    uint8_t w[kTiles][16][64];     // packed rows, 16-byte chunks XOR-swizzled
    uint8_t s[kTiles][16][4];      // E8M0 scales of the stage's 4 groups per row
    __half bh[kMaxTok][kStageK];   // B operand hi pieces, per column (swizzled chunks)
    __half bl[kMaxTok][kStageK];   // B operand lo pieces (fp32 sources only)
    float ts[4][kMaxTok];          // B group scale 2**e, [group][column]
};
static_assert(sizeof(Stage) % 16 == 0, "stage must keep 16-byte alignment");
constexpr size_t kSmemPerWarp = sizeof(Stage) * kStages;
constexpr size_t kSmemBytes = kSmemPerWarp * kWarps;

// Workspace layout of the decode calls; every region is 256-byte aligned.
struct DecodeLayout {
    int64_t M, H, I, E, U, P;      // tokens, hidden, inter, experts, max active, max pairs
    int CA, CB;                    // k-chunks of the gate/up and down phases
    size_t plan, logits, route_idx, route_w, xq_hi, xq_lo, xq_ts, act_hi, act_lo, act_ts, partA, cntA, partB,
        cntB, total;
};

}  // namespace k3
