// TMA-fed grouped MXFP4 matvec (decode path, sm_100a): shared declarations.
#pragma once

#include <cuda.h>

#include "k3_moe.cuh"

namespace k3 {

// A CTA has 8 consumer warps and 1 producer warp. An item is 128 weight rows (phase
// gate/up: 64 gate + 64 up rows of one expert; projections: 128 rows) x one k-chunk.
// The producer thread streams the item through a ring of CTA-wide stages with TMA
// (cp.async.bulk.tensor): per stage 512 k = 256 packed bytes per row (two 128-byte
// swizzled boxes), the 16 scale bytes per row, and the B operand pieces of those k.
constexpr int kTWarps = 8;
constexpr int kTThreads = (kTWarps + 1) * 32;
constexpr int kTStageK = 512;
constexpr int kTGroups = kTStageK / 32;      // 16 scale groups per stage
constexpr int kTRows = 128;
// A key is shared by at most one segment per CTA; grids never exceed this many CTAs.
constexpr int kTMaxSegments = 512;

template <bool HILO, bool GROUP_TS>
struct alignas(1024) TStage {
    uint8_t w[2][kTRows][128];                             // SW128 boxes: k bytes [0,128), [128,256)
    uint8_t s[kTRows][kTGroups];                           // E8M0 scales
    __half bh[kTGroups][kMaxTok][32];                      // B hi: [group][column][32 k]
    __half bl[HILO ? kTGroups : 1][kMaxTok][32];           // B lo
    float ts[GROUP_TS ? kTGroups : 1][kMaxTok];            // B group scales [group][column]
};

template <bool HILO>
constexpr int tstages() { return HILO ? 4 : 5; }

constexpr size_t kTEpilogueBytes = sizeof(float) * kMaxTok * kTRows;   // [column][row]

template <bool HILO, bool GROUP_TS>
constexpr size_t tsmem_bytes() {
    return sizeof(TStage<HILO, GROUP_TS>) * tstages<HILO>() + kTEpilogueBytes +
           1024 /*align*/ + 256 /*barriers*/;
}
static_assert(tsmem_bytes<false, false>() <= 227 * 1024 && tsmem_bytes<true, true>() <= 227 * 1024,
              "TMA ring exceeds shared memory");

// Tensor maps of one launch: weights/scales of the first (gate, or the only) and second
// (up) projection as 3-D [slot][row][k] views, the B pieces as 3-D [group][column][32]
// views, and the B group scales as a 2-D [group][column] view. Every map's innermost
// coordinate is a multiple of 16 bytes (TMA requirement): byte offsets of 256, scale
// groups of 16, element 0 of a 32-element block, column indices of 8 floats.
struct TMaps {
    CUtensorMap wA, sA, wB, sB, bh, bl, bts;
};

// Everything a launch needs besides the maps.
//
// Work is split into items; consecutive items that write the same outputs share a
// "key" (gate/up: one expert's 64-row block; projection: one 128-row block of y, over
// all experts and k-chunks). Each CTA owns one contiguous range of items, accumulates a
// key in registers while its items continue, and flushes it when the key changes: a
// key that lies wholly inside the CTA is finished in place; a key shared by several
// CTAs goes through per-segment partial sums that the last CTA to arrive reduces.
struct TArgs {
    const Plan* plan;
    int matvec;              // one plain matrix (slot 0): plan = tokens, B = x rows
    int64_t K;               // reduction length
    int64_t rows;            // rows of one projection
    int C;                   // k-chunks per (expert, row block)
    int* status;
    float* part;             // segment partial sums [key][maxseg][8 columns][128 rows]
    unsigned* cnt;           // arrival counter per key
    int maxseg;
    // gate/up epilogue: activation pieces per (active expert, token) in the blocked
    // layout [group][expert * 8 + token][32] plus scales [group][expert * 8 + token]
    __half* act_hi;
    __half* act_lo;
    float* act_ts;
    int64_t act_rows;        // rows of the blocked act tensors (active experts x 8)
    int act_groups;          // I / 32
    int act_kind;
    float beta, lbeta;
    const float* bts_tok;    // scales of x per (token, 512-k block): [8][K/512] (gate/up, matvec)
    // projection epilogue
    void* y;
    int y_dtype;
};

// Host: CUtensorMap encoding through the driver entry point (no libcuda link).
int encode_map(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* base,
               const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
               CUtensorMapSwizzle swizzle);

// Launches (defined in k3_tma.cu).
int launch_tma_gateup(const TMaps& maps, const TArgs& a, bool hilo, int grid, cudaStream_t s);
int launch_tma_proj(const TMaps& maps, const TArgs& a, bool hilo, bool group_ts, int grid,
                    cudaStream_t s);

}  // namespace k3
