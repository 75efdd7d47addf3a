// Block-scaled decode path on the 5th-generation tensor cores (tcgen05, sm_100a):
// shared declarations.
//
// The MXFP4 weights are consumed as stored: E2M1 codes straight from HBM (TMA, 128-byte
// swizzle) and their E8M0 scales, re-laid once into the tensor core's scale-chunk
// layout. The activations enter as E2M1 too: each value is split into kBPieces E2M1
// pieces with one E8M0 scale per (piece, 32-element block) -- piece p holds what pieces
// 0..p-1 left over, so their sum reproduces the value to ~2^-25 relative (the split is
// exact bookkeeping; only the final remainder is dropped). B row n = 8 * column + piece,
// and the pieces of one column are summed after the MMA.
#pragma once

#include <cuda.h>

#include "k3_moe.cuh"

namespace k3 {

constexpr int kBPieces = 8;                     // E2M1 pieces per activation value
constexpr int kBStageK = 256;                   // k per pipeline stage: 128 packed bytes a row
constexpr int kBRows = 128;                     // weight rows per MMA tile (M)
constexpr int kBChunk = 512;                    // scale chunk: 128 rows x 4 k-blocks of 32
constexpr int kBMaxN = kMaxTok * kBPieces;      // B rows of one MMA (64)
constexpr int kBEpiWarps = 4;                   // epilogue warps (one per TMEM lane quarter)
constexpr int kBThreads = (2 + kBEpiWarps) * 32;
constexpr int kBMaxSegments = 256;              // CTAs sharing one key (grid <= 256)

// Byte of the scale of (row n, k-block j) inside its 512-byte chunk: the chunk is the
// 32 x 16-byte matrix tcgen05.cp replicates to the four TMEM lane quarters, row n in
// lane n % 32, column n / 32, byte j.
__host__ __device__ __forceinline__ int sf_chunk_offset(int n, int j) {
    return (n & 31) * 16 + (n >> 5) * 4 + j;
}

// One pipeline stage. Gate/up: the 128-row gate tile and the 128-row up tile of one
// expert block share the B tile; down: one 128-row tile. SFRAW stages (weights with their
// scales as stored, row-major [rows][K/32]) also hold the TMA box of those scales: 16
// bytes (512 k) of each of the 128 rows, from which the MMA warp writes the stage's two
// scale chunks. SFBRAW stages (gate/up) do the same for the activation pieces: per pair
// the 16-byte (512 k) box of its token's 8 piece rows of the per-row scales [8T][K/32].
template <bool GATEUP>
struct alignas(1024) BStageBase {
    uint8_t a[GATEUP ? 2 : 1][kBRows][128];     // E2M1 weights, SW128
    uint8_t b[kBMaxN][128];                     // E2M1 activation pieces, SW128
    uint8_t sfa[GATEUP ? 2 : 1][2 * kBChunk];   // weight scales, two chunks (256 k)
    uint8_t sfb[2 * kBChunk];                   // piece scales, two chunks
};
template <bool GATEUP, bool SFRAW = false, bool SFBRAW = false>
struct alignas(1024) BStage : BStageBase<GATEUP> {};
template <bool GATEUP>
struct alignas(1024) BStage<GATEUP, true, false> : BStageBase<GATEUP> {
    uint8_t sfraw[kBRows][16];                  // row-major weight scale box (512 k)
};
template <>
struct alignas(1024) BStage<true, false, true> : BStageBase<true> {
    uint8_t sfbraw[kBMaxN][16];                 // per pair: its token's 8 piece-scale rows (512 k)
};
static_assert(sizeof(BStage<false>) == sizeof(BStageBase<false>) && sizeof(BStage<true>) == sizeof(BStageBase<true>),
              "the stored-layout stages carry no raw scale box");

template <bool GATEUP, bool SFRAW = false, bool SFBRAW = false>
constexpr int bstages() { return GATEUP ? 5 : (SFRAW ? 7 : 8); }
template <bool GATEUP>
constexpr uint32_t btmem_cols() { return GATEUP ? 512 : 256; }
template <bool GATEUP, bool SFRAW = false, bool SFBRAW = false>
constexpr size_t bsmem_bytes() {
    return sizeof(BStage<GATEUP, SFRAW, SFBRAW>) * bstages<GATEUP, SFRAW, SFBRAW>() + 1024 /*align*/ +
           256 /*barriers*/;
}
static_assert(bsmem_bytes<true>() + 4096 <= 227 * 1024 && bsmem_bytes<false>() + 4096 <= 227 * 1024 &&
                  bsmem_bytes<false, true>() + 4096 <= 227 * 1024 &&
                  bsmem_bytes<true, false, true>() + 5 * 1024 + 512 <= 227 * 1024,
              "block-scaled ring exceeds shared memory");

// Tensor maps: a0/a1 = packed weight pools, row-major [slot][rows][K/2] (box 128 B x 128
// rows) or tiled [slot * rows/128][K/256][128][128] (box = one contiguous tile);
// b = activation pieces, gate/up x [8T][K/2] (box 128 B x 8 rows: one token's pieces),
// down act [v][64][K/2] (box 128 B x 8 rows: one pair's pieces); sfa (SFRAW only) = the
// weight scales as stored, [slot * rows][K/32] (box 16 B x 128 rows); sfb (SFBRAW only) =
// the per-row scales of the x pieces [8T][K/32] (box 16 B x 8 rows: one token's pieces).
struct BMaps {
    CUtensorMap a0, a1, b, sfa, sfb;
};

struct BArgs {
    const Plan* plan;
    int64_t K;              // reduction length
    int64_t rows;           // rows of one projection (I for gate/up, H for down)
    int C;                  // k-chunks per (expert, row block)
    int* status;
    float* part;            // segment partials [key][maxseg][PW][128], PW = 16 | 8
    unsigned* cnt;          // arrival counter per key
    int maxseg;
    const uint8_t* sfa0;    // weight scale chunks of pool a0 [slot][rows/128][K/128][512]
    const uint8_t* sfa1;    // of pool a1 (gate/up)
    int tiled;              // a0/a1 are tile pools (4-D maps) rather than row-major pools
    int64_t sf_slot;        // bytes per slot of a scale-chunk pool
    const uint8_t* sfb;     // B scale chunks per expert item [v][K/128][512] (gate/up
                            // over the identity plan: x pieces, from launch_mv_prep; down:
                            // act pieces); unused by the raw-scale gate/up (maps.sfb)
    // gate/up epilogue: act pieces of expert v's pair i, piece p at row v*64 + 8i + p of
    // act_p [.][I/2]; their scale chunks act_sf [v][I/128][512]
    uint8_t* act_p;
    uint8_t* act_sf;
    int act_kind;
    float beta, lbeta;
    // down epilogue: one f32 output row per pair, y_pair [pairs][H] (bf16 when y_bf16)
    float* y_pair;
    int y_bf16;
    // > 0: the plan is the identity plan of identity_m tokens (items of 8 tokens of slot 0,
    // weight 1), built by each CTA itself; the weights and their scales are then requested
    // before the wait for the previous launch (which writes only the activation operand)
    int identity_m;
    // request the first stages' weights before waiting for the previous launch (the weights
    // and the plan never come from it): set for the down phase, whose CTAs start on the SMs
    // that the gate/up launch's early finishers leave. (Measured slower for the gate/up
    // phase when a short scale-gather launch preceded it.)
    int early_a;
    // the previous launch writes the plan (the gate/up launch with raw piece scales follows
    // the plan producer directly): every thread waits for it before copying the plan
    int plan_in_prev;
};

int launch_bs_gateup(const BMaps& maps, const BArgs& a, int grid, cudaStream_t s);
// The gate/up kernel reading the x pieces' per-row scales through maps.sfb (no scale
// gather launch before it); a.plan_in_prev must be set.
int launch_bs_gateup_rawsfb(const BMaps& maps, const BArgs& a, int grid, cudaStream_t s);
int launch_bs_down(const BMaps& maps, const BArgs& a, int grid, cudaStream_t s);
// The down-phase kernel over a weight matrix whose scales are row-major as stored
// (maps.sfa), for the single-matrix matvec.
int launch_bs_proj_rawsf(const BMaps& maps, const BArgs& a, int grid, cudaStream_t s);
// x [M][K] -> E2M1 pieces [8M][K/2] and their scale chunks for identity-plan items of 8
// tokens [M/8][K/128][512]; zeroes ncnt arrival counters and sets *status = K3_OK (the
// launch a projection with identity_m = M depends on).
int launch_mv_prep(const void* x, int xdt, int M, int64_t K, uint8_t* xp, uint8_t* sfb, unsigned* cnt, int ncnt,
                   int* status, cudaStream_t s);
// y[t] = sum over the pairs of token t, in plan order, of y_pair[pair] (weights are
// already applied); y [M][H] f32 or bf16.
int launch_combine(const Plan* plan, const float* y_pair, int64_t H, int M, void* y, int y_dtype,
                   cudaStream_t s);
// Scale re-layout [batch][rows][cols/32] -> [batch][rows/128][cols/128][512] chunks.
int launch_scales_tc(const uint8_t* in, int64_t rows, int64_t cols, int64_t batch, uint8_t* out,
                     cudaStream_t s);
// Packed-code re-layout [batch][rows][cols/2] -> [batch][rows/128][cols/256][128][128].
int launch_tiles(const uint8_t* in, int64_t rows, int64_t cols, int64_t batch, uint8_t* out,
                 cudaStream_t s);

// SwiGLU / situ activation of one (gate, up) pair (air_llm/models/kimi_k3/ops.py:17-28,
// 42-43): sigmoid(g) = 1 / (1 + exp(-g)). exp's argument is clamped at 80 so the
// denominator stays finite (below g = -80 sigmoid is under 2e-35 either way): a division
// by infinity would send the whole warp down the division's slow path.
__device__ __forceinline__ float act_value(int kind, float g, float u, float beta, float lbeta) {
    const float den = 1.0f + expf(-fmaxf(g, -80.0f));
    if (kind == K3_ACT_SITU) {
        const float a = beta * tanhf(g / beta) / den;
        const float v = lbeta > 0.0f ? lbeta * tanhf(u / lbeta) : u;
        return a * v;
    }
    return g / den * u;
}

// Max of a non-negative float over the warp (bit patterns of non-negative floats order
// like unsigned integers).
__device__ __forceinline__ float warp_max_nonneg(float v) {
    uint32_t r;
    asm volatile("redux.sync.max.u32 %0, %1, 0xffffffff;\n" : "=r"(r) : "r"(__float_as_uint(v)));
    return __uint_as_float(r);
}

// E8M0 byte of the smallest power of two S with m <= 6 S, for the non-negative block
// maximum m given as its bit pattern: the exponent field minus 2, plus one when the
// significand is above 1.5, clamped to 1..253 (zero and subnormal m give 1). The same byte
// as frexp(m) = f * 2^E -> E - 3 + (f > 0.75) + 127, read off the bits; NaN gives 1 and
// +inf 125 (frexp's exponent 0 for it). Selects only, no branch: the split's unrolled
// chains of independent values interleave across it.
__device__ __forceinline__ int e8m0_cover6(uint32_t mb) {
    int b = int(mb >> 23) - 2 + ((mb & 0x7fffffu) > 0x400000u ? 1 : 0);
    b = min(max(b, 1), 253);
    b = mb > 0x7f800000u ? 1 : b;                        // NaN
    return mb == 0x7f800000u ? 125 : b;                  // +inf
}

// E2M1 codes of two floats, round to nearest even with saturation at +-6 (the block scale
// keeps |value| <= 6): code of a in bits 0-3, of b in bits 4-7.
__device__ __forceinline__ uint32_t e2m1x2_codes(float a, float b) {
    uint32_t r;
    asm("{\n"
        ".reg .b8 c;\n"
        "cvt.rn.satfinite.e2m1x2.f32 c, %2, %1;\n"
        "cvt.u32.u8 %0, c;\n"
        "}\n"
        : "=r"(r) : "f"(a), "f"(b));
    return r;
}

// The values of two E2M1 codes packed as e2m1x2_codes returns them (exact in f16).
__device__ __forceinline__ float2 e2m1x2_values(uint32_t codes) {
    uint32_t h;
    asm("{\n"
        ".reg .b8 c;\n"
        "cvt.u8.u32 c, %1;\n"
        "cvt.rn.f16x2.e2m1x2 %0, c;\n"
        "}\n"
        : "=r"(h) : "r"(codes));
    return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

// Within each group of 8 lanes, lane j holds 8 nibbles (nibble p at bits 4p); returns the
// transpose: lane p of the group gets nibble p of every lane j of the group at bits 4j.
// Three butterfly stages: in stage d, the nibbles whose position and lane differ in bit d
// swap across lanes j and j ^ d.
__device__ __forceinline__ uint32_t transpose_nibbles8(uint32_t n, int lane) {
#pragma unroll
    for (int d = 1; d < 8; d <<= 1) {
        const uint32_t m = d == 1 ? 0xF0F0F0F0u : (d == 2 ? 0xFF00FF00u : 0xFFFF0000u);
        const uint32_t o = __shfl_xor_sync(0xffffffffu, n, d);
        n = (lane & d) ? ((n & m) | ((o & m) >> (4 * d))) : ((n & ~m) | ((o & ~m) << (4 * d)));
    }
    return n;
}

// Warp-wide: lane l holds element l of a 32-element block of NV values (independent
// chains, interleaved); splits each into NP (default kBPieces, at most 8) E2M1 pieces.
// Piece p of value i: its 16 packed bytes go to data[i] + p*row_stride (element 2j in the
// low nibble of byte j) and its E8M0 scale to sf[i][p*sf_stride]. Values with sf[i] ==
// nullptr are skipped. Both scale layouts in use are affine in p: natural per-row scales
// ([row][block], stride = blocks per row) and the tensor-core chunk
// (sf_chunk_offset(8*col + p, j), stride 16 since the 8 rows of one column share a
// 32-row group).
// Piece p: S = the smallest power of two with max|res| <= 6 S over the block (one warp
// reduction), codes = E2M1(res / S) rounded to nearest even, res -= value(codes) * S
// (exact: value * S is on res's grid). The hardware conversions give the codes and their
// values; every lane keeps its codes of all pieces in one word, and one nibble transpose
// per 8 lanes turns those into the pieces' packed rows, written once at the end. A
// negative value that rounds to zero gets code 0 (not -0), and NaN codes as 0.
template <int NV, int NP = kBPieces>
__device__ __forceinline__ void split_pieces_n(const float (&v)[NV], int lane, uint8_t* const (&data)[NV],
                                               int64_t row_stride, uint8_t* const (&sf)[NV], int64_t sf_stride) {
    static_assert(NP >= 1 && NP <= 8, "a lane keeps at most 8 pieces' codes in one word");
    float res[NV];
    uint32_t nib[NV];
    int sfv[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        res[i] = v[i];
        nib[i] = 0u;
        sfv[i] = 1;
    }
#pragma unroll
    for (int p = 0; p < NP; ++p) {
        float a[NV + 1], S[NV];
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int b = e8m0_cover6(__float_as_uint(warp_max_nonneg(fabsf(res[i]))));
            S[i] = __int_as_float(b << 23);
            const float t = res[i] * __int_as_float((254 - b) << 23);
            a[i] = t == t ? t : 0.0f;
            sfv[i] = lane == p ? b : sfv[i];
        }
        a[NV] = 0.0f;
#pragma unroll
        for (int i = 0; i < NV; i += 2) {
            const uint32_t c = e2m1x2_codes(a[i], a[i + 1]);
            const float2 q = e2m1x2_values(c);
            res[i] = fmaf(-q.x, S[i], res[i]);
            nib[i] |= (c & 0xFu) << (4 * p);
            if (i + 1 < NV) {
                res[i + 1] = fmaf(-q.y, S[i + 1], res[i + 1]);
                nib[i + 1] |= (c >> 4) << (4 * p);
            }
        }
    }
    const int p = lane & 7, g = lane >> 3;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        // -0 codes (a negative value rounded to zero) become 0
        const uint32_t t = nib[i] ^ 0x88888888u;
        const uint32_t nz = (t | (t >> 1) | (t >> 2) | (t >> 3)) & 0x11111111u;
        const uint32_t w = transpose_nibbles8(nib[i] & ~((~nz & 0x11111111u) << 3), lane);
        if (sf[i]) {
            if (p < NP) *reinterpret_cast<uint32_t*>(data[i] + p * row_stride + 4 * g) = w;
            if (lane < NP) sf[i][lane * sf_stride] = uint8_t(sfv[i]);
        }
    }
}

// One value per lane (see split_pieces_n).
__device__ __forceinline__ void split_pieces(float v, int lane, uint8_t* data, int64_t row_stride,
                                             uint8_t* sf, int64_t sf_stride) {
    const float vv[1] = {v};
    uint8_t* const dd[1] = {data};
    uint8_t* const ss[1] = {sf};
    split_pieces_n<1>(vv, lane, dd, row_stride, ss, sf_stride);
}

}  // namespace k3
