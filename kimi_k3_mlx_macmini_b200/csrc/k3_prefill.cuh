// Prefill path (many tokens per call) on the block-scaled tensor cores: shared
// declarations.
//
// A call routes T tokens, groups the (token, expert) pairs by expert -- experts ascending,
// tokens ascending within an expert, the shared expert last (the order of the reference's
// `for e in sorted(...)` loop, air_llm/models/kimi_k3/moe.py:120) -- and cuts each
// expert's pairs into chunks of at most kPN tokens. One grouped GEMM per phase then runs
// over items = (chunk, weight row block):
//
//   gate/up: D_g, D_u [128 rows of I][chunk tokens] = W1/W3 rows x (x pieces)^T, then
//            act = phi(D_g, D_u) * routing weight, split into E2M1 pieces for the down
//            phase;
//   down:    D [2 x 128 rows of H][chunk tokens] = W2 rows x (act pieces)^T, reduce-added
//            into y[token] (fp32 adds in the L2; the order of the adds is not fixed).
//
// The activations enter the kind::mxf4 MMA as E2M1 pieces with one E8M0 scale per (piece,
// 32-block); the pieces of one value accumulate into the same TMEM column (one MMA per
// piece, accumulate on), so a chunk of n tokens takes n TMEM columns. bf16 tokens and the
// activations take kPPieces pieces (bf16's 8 significant bits fit in them); fp32 tokens
// take kPPiecesF32, which keeps the split error near 2e-6 of the value.
//
// Two pieces are stacked along N in one MMA (B rows [piece][token]); the two TMEM columns
// of a token are added in the epilogue. A tcgen05 MMA costs about the same per
// instruction for any N up to 256, so the stacking halves the tensor time; the price is
// a single-buffered accumulator (2 x 208 columns), drained quickly by the epilogue.
//
// Token operands live in "images": for every (chunk, 256-k step, piece pair) one
// contiguous block holding the scale chunks of the block's rows followed by its 2 n8 rows
// of 128 packed bytes, already in the 128-byte-swizzled order the tensor core reads
// (16-byte unit u of row r at position u ^ (r & 7)). One bulk copy moves a block into a
// shared-memory slot. The gate/up image is built from the token pieces by a permute
// kernel; the down image is written by the gate/up epilogue.
#pragma once

#include <cuda.h>

#include "k3_bs.cuh"

namespace k3 {

constexpr int kPPieces = 4;           // E2M1 pieces per activation value (bf16 tokens, act)
constexpr int kPPiecesF32 = 6;        // pieces per fp32 token value (gate/up input)
constexpr int kPStack = 2;            // pieces stacked along N in one MMA (B rows = piece-major)
constexpr int kPN = 104;              // tokens per chunk (MMA N = kPStack x rows <= 208)
constexpr int kPASlots = 3;           // weight ring: two 128-row tiles x 256 k per slot
constexpr int kPBSlots = 3;           // token ring: one image block (two pieces) per slot
constexpr int kPEpiWarps = 4;
constexpr int kPThreads = (3 + kPEpiWarps) * 32;   // A producer, MMA, 4 epilogue, B producer
constexpr int kPPlanBlock = 256;      // candidates per plan block
constexpr int kPMaxSlots = kMaxExperts + 1;
constexpr int kPImgSf = 4 * kBChunk;  // scale bytes at the head of an image block:
                                      // [k-half h][row set (rows 0-127, 128-255)][512]

// TMEM columns: two accumulators of kPStack * kPN columns (single buffer), then the scale
// slots (A: two tiles x two k-halves x 4 columns; B: two k-halves x two row sets x 4).
constexpr int kPAccCols = kPStack * kPN;
constexpr int kPSfaCol = 2 * kPAccCols;             // kPASlots x 16 columns
constexpr int kPSfbCol = kPSfaCol + 16 * kPASlots;  // kPBSlots x 16 columns
static_assert(kPSfbCol + 16 * kPBSlots <= 512, "prefill TMEM plan exceeds 512 columns");
static_assert(kPN % 8 == 0 && kPStack * kPN <= 256, "MMA N must be a multiple of 8, <= 256");

struct alignas(1024) PASlot {
    uint8_t a[2][kBRows][128];        // two weight tiles (gate + up, or two down row blocks), SW128
    uint8_t sfa[2][2 * kBChunk];      // their scale chunks (256 k)
};
struct alignas(1024) PBSlot {
    uint8_t sfb[kPImgSf];             // one image block: scale chunks, then
    uint8_t b[kPStack * kPN][128];    // rows [piece][token] of two pieces (256 k), SW128
};
constexpr size_t psmem_bytes() {
    return sizeof(PASlot) * kPASlots + sizeof(PBSlot) * kPBSlots + 1024 /*align*/ + 256 /*barriers*/;
}
static_assert(psmem_bytes() + 2048 <= 227 * 1024, "prefill ring exceeds shared memory");
// Gate/up epilogue staging per CTA: [token][gate | up][128 rows] fp32.
constexpr size_t kPSlabBytes = sizeof(float) * kPN * 2 * kBRows;

// Byte offset of the image block (chunk c, k-step s, piece pair pp) of an image with
// `pairs` piece pairs: blocks are ordered [chunk][step][pair], a block of a chunk with n8
// rows per piece holds kPImgSf + 128 * kPStack * n8 bytes, and n8p[c] = sum of n8 over the
// chunks before c. Row r of a block is (piece pp*kPStack + r / n8, token r % n8).
__host__ __device__ __forceinline__ int64_t img_block(const int* n8p, int c, int nst, int s, int pp, int n8,
                                                      int pairs) {
    return int64_t(pairs) * nst * (int64_t(kPImgSf) * c + 128 * kPStack * int64_t(n8p[c])) +
           int64_t(s * pairs + pp) * (kPImgSf + 128 * kPStack * n8);
}
// Offset inside a block of the scale byte of (row r, k-block j of the block's 256 k).
__host__ __device__ __forceinline__ int img_sf(int r, int j) {
    return (j >> 2) * 2 * kBChunk + (r >> 7) * kBChunk + sf_chunk_offset(r & 127, j & 3);
}

// Device-side routing plan of one prefill call (all arrays in the workspace).
struct PrefillHeader {
    int status;
    int n_pairs;
    int n_chunks;
    int pad;
};
struct PrefillPlan {
    PrefillHeader* hdr;
    int* blk_cnt;        // [nblk][NS] per-block slot counts, then per-block bases
    int* off;            // [NS + 1] first pair of each slot
    int* ch_first;       // [NS + 1] first chunk of each slot
    int* pair_tok;       // [NP] token row of each pair (grouped order)
    float* pair_w;       // [NP] its routing weight
    int* pair_cj;        // [NP] (chunk << 8) | row in the chunk
    int* ch_slot;        // [NC] chunk -> slot
    int* ch_p0;          // [NC] first pair of the chunk
    int* ch_n;           // [NC] pairs in the chunk (1..kPN)
    int* ch_n8p;         // [NC + 1] exclusive prefix of the chunks' rows rounded up to 8
};

// Where the (slot, token, weight) candidates come from: either a routing result
// idx/w (rows rstride elements apart; candidate i < T*k, i = t*k + j, is (idx[t][j] -
// expert_lo when in [0, n_local), t, w[t][j]); the next shared_n candidates are
// (shared_slot, shared_t0 + j, 1)), or explicit pair arrays.
struct PrefillCand {
    const int32_t* idx;
    const float* w;
    int T, k, shared_slot;
    int rstride, expert_lo, n_local, shared_t0, shared_n;
    const int32_t* slot;
    const int32_t* tok;
    const float* pw;
    int n;
    int num_slots;
};

// Tensor maps: the two weight tile pools ([slot * rows/128][K/256][128][128] boxes).
struct PMaps {
    CUtensorMap a0, a1;
};

struct PArgs {
    PrefillPlan P;
    int64_t K;               // reduction length (H for gate/up, I for down)
    int64_t rows;            // rows of one projection (I for gate/up, H for down)
    int* status;
    const uint8_t* sfa0;     // scale-chunk pools [slot][rows/128][K/128][512]
    const uint8_t* sfa1;     // (gate/up: W3's; down: unused)
    int64_t sf_slot;         // bytes per slot of a scale-chunk pool
    int routed_slots;        // slots below this stream with an evict-first L2 policy
    const uint8_t* img;      // B image of this phase
    // gate/up epilogue -> the down phase's image, through a per-CTA staging slab
    uint8_t* img_out;
    float* slab;
    int act_kind;
    float beta, lbeta;
    // down epilogue: y [T][H] fp32 (reduce-add)
    float* y;
};

// Router logits [T][E] of bf16 x on the tensor cores (tcgen05 kind::f16, fp32
// accumulation of the exact bf16 products); router_gemm_ok tells whether it applies.
bool router_gemm_ok(int xdt, int64_t H, const void* x, const void* gate_w);
int launch_router_gemm(const void* x, int64_t T, int64_t H, const uint16_t* gate_w, int64_t E, float* logits,
                       int* status, cudaStream_t s);

}  // namespace k3
