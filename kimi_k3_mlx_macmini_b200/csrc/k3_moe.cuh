// Decode-path data structures shared by the router, plan and grouped-matvec kernels.
#pragma once

#include "k3_common.cuh"

namespace k3 {

constexpr int kMaxTok = 8;                       // decode tokens = mma n8 columns
constexpr int kMaxTopK = 16;
constexpr int kMaxExperts = 1024;
// Routing plans hold at most this many expert items and (token, expert) pairs: a decode
// call (8 tokens x top-16 + shared) and the expert-parallel local calls (pairs routed to
// one rank's experts) both fit.
constexpr int kMaxActive = 256;
constexpr int kMaxPairs = 256;
static_assert(kMaxActive >= kMaxTok * kMaxTopK + 1 && kMaxPairs >= kMaxTok * kMaxTopK + kMaxTok,
              "plan capacity below one decode call");

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
// Pipeline stage of one warp: 64 packed bytes (128 k) of each of its 64 weight rows,
// their scales, and the B operand pieces of the same k range. HILO stages also carry
// the lo pieces of fp32 activations; bf16 activations need only the hi piece, which
// leaves room for a deeper ring.
template <bool HILO>
struct StageT {
    uint8_t w[kTiles][16][64];                         // packed rows, XOR-swizzled chunks
    uint8_t s[kTiles][16][4];                          // E8M0 scales of the 4 groups per row
    __half bh[kMaxTok][kStageK];                       // B hi pieces (swizzled chunks)
    __half bl[HILO ? kMaxTok : 1][HILO ? kStageK : 8]; // B lo pieces
    float ts[4][kMaxTok];                              // B group scale 2**e, [group][column]
};
static_assert(sizeof(StageT<true>) % 16 == 0 && sizeof(StageT<false>) % 16 == 0,
              "stages must keep 16-byte alignment");
template <bool HILO>
constexpr int stages_for() { return HILO ? 3 : 4; }
template <bool HILO>
constexpr size_t smem_bytes_for() { return sizeof(StageT<HILO>) * stages_for<HILO>() * kWarps; }
static_assert(smem_bytes_for<true>() <= 227 * 1024 && smem_bytes_for<false>() <= 227 * 1024,
              "ring exceeds shared memory");

// Workspace layout of the decode calls; every region is 256-byte aligned.
struct DecodeLayout {
    int64_t M, H, I, E, U, P;      // tokens, hidden, inter, experts, max active, max pairs
    int CA, CB;                    // k-chunks of the gate/up and down phases
    bool tma;                      // TMA-fed kernels over contiguous expert pools
    bool bs;                       // ... on the block-scaled (kind::mxf4) tensor-core path
    int64_t ppad, tspad;           // column strides of the blocked activation buffers
    int KQ;                        // router k-slices (fused router)
    size_t y_pair;                 // block-scaled path: one output row per pair
    size_t plan, logits, logit_part, route_done, route_idx, route_w, xq_hi, xq_lo, xq_ts, act_hi, act_lo, act_ts, partA, cntA, partB,
        cntB, total;
    size_t route_keys, route_scores;   // fused router: top-k keys and sigmoid scores [M][E]
};

}  // namespace k3
