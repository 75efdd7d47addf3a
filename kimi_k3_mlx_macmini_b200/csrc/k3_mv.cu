// Single-matrix fused MXFP4 matvec (mxfp4_matvec_fused, air_llm/kernels/metal/mxfp4_matvec.py:75-96)
// on the block-scaled tensor cores, reading the weights and their scales as the
// reference stores them (packed [N][K/2], scales [N][K/32]; nothing is re-laid).
//
// Two launches per call (up to 256 tokens each):
//   mv_prep_kernel   x [M][K] -> E2M1 pieces [8M][K/2] (one warp per (token, 32-block),
//                    kBPieces pieces with one E8M0 scale each) and their scale chunks in
//                    the tensor core's layout [M/8][K/128][512]; zeroes the arrival
//                    counters of a fresh workspace;
//   bs_gemv_kernel<projection, stored scales>
//                    the identity plan (items of 8 tokens), weight tiles by TMA from the
//                    row-major packed matrix and 512-k boxes of its row-major scales, from
//                    which the MMA warp writes each stage's scale chunks; it is a
//                    programmatic dependent of the prep launch and requests the first
//                    stages' weights before waiting for it. Output rows are the tokens.
#include "k3_async.cuh"
#include "k3_bs.cuh"
#include "k3_tma.cuh"

namespace k3 {

namespace {

constexpr int64_t kMvTok = kMaxPairs;            // tokens per launch pair (identity-plan capacity)

struct MvLayout {
    int64_t U;          // items of 8 tokens
    int C;              // k-chunks per 128-row block
    size_t status, xp, sfb, part, cnt, total;
};

// k-split over 256-k stages: the one whose busiest CTA streams the fewest stages, the
// smallest such split (fewer partial sums to merge).
int mv_split(int64_t keys, int64_t K, int grid) {
    const int64_t nst = K / kBStageK;
    int best = 1;
    int64_t best_span = INT64_MAX;
    for (int64_t c = 1; c <= nst; ++c) {
        if (nst % c) continue;
        const int64_t items = keys * c;
        const int64_t span = (items + grid - 1) / grid * (nst / c);
        if (span < best_span) {
            best_span = span;
            best = int(c);
        }
    }
    return best;
}

MvLayout mv_layout(int64_t Mc, int64_t K, int64_t N, int sms) {
    MvLayout L{};
    L.U = (Mc + kMaxTok - 1) / kMaxTok;
    const int64_t keys = L.U * (N / kBRows);
    L.C = mv_split(keys, K, sms);
    size_t off = 0;
    auto carve = [&](size_t bytes) {
        const size_t o = off;
        off = align_up(off + bytes, 256);
        return o;
    };
    L.status = carve(sizeof(int));
    L.xp = carve(size_t(L.U) * kBMaxN * (K / 2));
    L.sfb = carve(size_t(L.U) * (K / 128) * kBChunk);
    L.part = carve(sizeof(float) * size_t(keys) * L.C * kMaxTok * kBRows);
    L.cnt = carve(sizeof(unsigned) * size_t(keys));
    L.total = off;
    return L;
}

// CTA 0: status word and arrival counters; CTAs 1..: one warp per (token, 32-block).
__global__ void __launch_bounds__(256) mv_prep_kernel(const void* __restrict__ x, int x_dtype, int M, int64_t K,
                                                      uint8_t* __restrict__ xp, uint8_t* __restrict__ sfb,
                                                      unsigned* __restrict__ cnt, int ncnt, int* status) {
    // the projection launch may start now: it streams weights until it waits for this one
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (blockIdx.x == 0) {
        if (threadIdx.x == 0) *status = K3_OK;
        for (int i = threadIdx.x; i < ncnt; i += blockDim.x) cnt[i] = 0u;
        return;
    }
    const uint32_t G = uint32_t(K / 32);                  // 32-bit: no 64-bit division per warp
    const uint32_t task = (blockIdx.x - 1) * (blockDim.x >> 5) + warp;
    if (task >= uint32_t(M) * G) return;
    const int64_t t = task / G, g = task - uint32_t(t) * G;
    const float v = load_as_f32(x, x_dtype, t * K + 32 * g + lane);
    // piece p of token t: row 8t + p of the pieces (pair t % 8 of item t / 8); its scale
    // at row 8 (t % 8) + p, k-block g % 4 of chunk g / 4 of the item (16 bytes per piece)
    uint8_t* sf = sfb + ((t / kMaxTok) * (K / 128) + g / 4) * kBChunk + sf_chunk_offset(kBPieces * int(t % kMaxTok), int(g % 4));
    split_pieces(v, lane, xp + int64_t(kBPieces) * t * (K / 2) + 16 * g, K / 2, sf, 16);
}

}  // namespace

int launch_mv_prep(const void* x, int xdt, int M, int64_t K, uint8_t* xp, uint8_t* sfb, unsigned* cnt, int ncnt,
                   int* status, cudaStream_t s) {
    const int64_t tasks = int64_t(M) * (K / 32);
    mv_prep_kernel<<<unsigned(1 + (tasks + 7) / 8), 256, 0, s>>>(x, xdt, M, K, xp, sfb, cnt, ncnt, status);
    K3_CHECK_LAUNCH("mv_prep_kernel");
    return K3_OK;
}

// Shapes the block-scaled projection takes: K a multiple of 512 (the scale boxes and
// their 16-byte row stride), N a multiple of 128, 16-byte aligned matrices.
bool matvec_bs_ok(int64_t K, int64_t N, const uint8_t* packed, const uint8_t* scales) {
    return K % 512 == 0 && N % kBRows == 0 && (reinterpret_cast<uintptr_t>(packed) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(scales) & 15) == 0 && K / 2 <= (int64_t(1) << 31) &&
           (N / kBRows) * (K / kBStageK) < 65536;     // the kernel's 32-bit item indices
}

size_t matvec_bs_workspace(int64_t M, int64_t K, int64_t N) {
    return mv_layout(std::min<int64_t>(M, kMvTok), K, N, num_sms()).total;
}

int matvec_bs(const void* x, int xdt, int64_t M, int64_t K, const uint8_t* packed, const uint8_t* scales,
              int64_t N, void* out, int odt, uint8_t* ws, cudaStream_t s) {
    const int sms = num_sms();
    const size_t esz = xdt == K3_BF16 ? 2 : 4, osz = odt == K3_BF16 ? 2 : 4;
    BMaps maps{};
    {   // the packed matrix [N][K/2] as a one-slot pool: box 128 bytes x 128 rows, 128-byte swizzle
        const uint64_t d[3] = {uint64_t(K / 2), uint64_t(N), 1};
        const uint64_t st[2] = {uint64_t(K / 2), uint64_t(N) * uint64_t(K / 2)};
        const uint32_t b[3] = {128, uint32_t(kBRows), 1};
        if (int rc = encode_map(&maps.a0, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, packed, d, st, b,
                                CU_TENSOR_MAP_SWIZZLE_128B))
            return rc;
    }
    {
        const uint64_t d[2] = {uint64_t(K / 32), uint64_t(N)};
        const uint64_t st[1] = {uint64_t(K / 32)};
        const uint32_t b[2] = {16, uint32_t(kBRows)};
        if (int rc = encode_map(&maps.sfa, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, scales, d, st, b,
                                CU_TENSOR_MAP_SWIZZLE_NONE))
            return rc;
    }
    for (int64_t m0 = 0; m0 < M; m0 += kMvTok) {
        const int64_t Mc = std::min<int64_t>(kMvTok, M - m0);
        const MvLayout L = mv_layout(Mc, K, N, sms);
        {
            const uint64_t d[3] = {uint64_t(K / 2), uint64_t(kBMaxN), uint64_t(L.U)};
            const uint64_t st[2] = {uint64_t(K / 2), uint64_t(kBMaxN) * uint64_t(K / 2)};
            const uint32_t b[3] = {128, uint32_t(kBPieces), 1};
            if (int rc = encode_map(&maps.b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, ws + L.xp, d, st, b,
                                    CU_TENSOR_MAP_SWIZZLE_128B))
                return rc;
        }
        const int64_t keys = L.U * (N / kBRows);
        prof_begin(K3_PROF_TOPK, s);
        const int prc = launch_mv_prep(static_cast<const uint8_t*>(x) + size_t(m0) * K * esz, xdt, int(Mc), K,
                                       ws + L.xp, ws + L.sfb, reinterpret_cast<unsigned*>(ws + L.cnt), int(keys),
                                       reinterpret_cast<int*>(ws + L.status), s);
        prof_end(K3_PROF_TOPK, s);
        if (prc) return prc;
        BArgs a{};
        a.plan = nullptr;
        a.K = K;
        a.rows = N;
        a.C = L.C;
        a.status = reinterpret_cast<int*>(ws + L.status);
        a.part = reinterpret_cast<float*>(ws + L.part);
        a.cnt = reinterpret_cast<unsigned*>(ws + L.cnt);
        a.maxseg = L.C;
        a.tiled = 0;
        a.sf_slot = 0;
        a.sfb = ws + L.sfb;
        a.y_pair = reinterpret_cast<float*>(static_cast<uint8_t*>(out) + size_t(m0) * N * osz);
        a.y_bf16 = odt == K3_BF16 ? 1 : 0;
        a.identity_m = int(Mc);
        prof_begin(K3_PROF_MATVEC, s);
        const int rc = launch_bs_proj_rawsf(maps, a, sms, s);
        prof_end(K3_PROF_MATVEC, s);
        if (rc) return rc;
    }
    return K3_OK;
}

}  // namespace k3
