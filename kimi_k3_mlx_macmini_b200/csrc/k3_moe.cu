// Decode path: router, routing plan, and the MXFP4 grouped matvec (sm_100a).
//
// Work decomposition. A warp-item is 64 weight rows (four m16 tiles) x one k-chunk of
// one expert projection. Each warp streams its items through a private 3-stage
// cp.async ring in shared memory (64 packed bytes = 128 k per row per stage),
// reads the tiles with ldmatrix so that the four lanes of a quad hold the same
// 32-element scale group, converts E2M1 -> f16 in hardware, and issues
// mma.m16n8k16 with the tokens (<= 8) as the n8 dimension. Every 32-element group
// is accumulated into a temporary and added to the fp32 accumulator with its exact
// scale 2**(s-127) * 2**e_col (E8M0 weight scale times the power-of-two scale of the
// activation piece), so weights are never rounded and activations keep ~22 bits.
// Partial sums of k-chunks meet in global scratch; the last warp to finish a row
// block (atomic counter) reduces them in a fixed order, so results are deterministic.
#include <algorithm>
#include <cstring>
#include <vector>

#include "k3_moe.cuh"
#include "k3_plan.cuh"
#include "k3_tma.cuh"
#include "k3_bs.cuh"
#include "k3_pairs.cuh"
#include "k3_prefill.cuh"
#include "k3_route.cuh"

namespace k3 {

// ================================================================== router

// logits[m][e] = sum_k x[m][k] * W[e][k] for m < Mc (<= 8): one warp per expert row,
// lanes walk 8-element chunks, fp32 fma in chunk order, then a xor-tree reduction.
// (Generic form for H % 64 != 0; router_logits_kernel below is the fast form.)
template <int XDT>
__global__ void __launch_bounds__(256) router_logits_rowwarp_kernel(const void* __restrict__ x, int Mc,
                                                            int64_t H,
                                                            const uint16_t* __restrict__ W,
                                                            int64_t E, float* __restrict__ logits) {
    const int64_t e = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (e >= E) return;
    const uint16_t* wr = W + e * H;
    float acc[kMaxTok];
#pragma unroll
    for (int m = 0; m < kMaxTok; ++m) acc[m] = 0.0f;
    for (int64_t k = int64_t(lane) * 8; k < H; k += 256) {
        const uint4 wv = __ldg(reinterpret_cast<const uint4*>(wr + k));
        float wf[8];
        const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            wf[2 * j] = __uint_as_float(ww[j] << 16);
            wf[2 * j + 1] = __uint_as_float(ww[j] & 0xffff0000u);
        }
#pragma unroll
        for (int m = 0; m < kMaxTok; ++m) {
            if (m < Mc) {
                float xf[8];
                if (XDT == K3_BF16) {
                    const uint4 xv = __ldg(reinterpret_cast<const uint4*>(
                        reinterpret_cast<const uint16_t*>(x) + m * H + k));
                    const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        xf[2 * j] = __uint_as_float(xw[j] << 16);
                        xf[2 * j + 1] = __uint_as_float(xw[j] & 0xffff0000u);
                    }
                } else {
                    const float4* xp =
                        reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + m * H + k);
                    const float4 a = __ldg(xp), b = __ldg(xp + 1);
                    xf[0] = a.x; xf[1] = a.y; xf[2] = a.z; xf[3] = a.w;
                    xf[4] = b.x; xf[5] = b.y; xf[6] = b.z; xf[7] = b.w;
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[m] = fmaf(xf[j], wf[j], acc[m]);
            }
        }
    }
#pragma unroll
    for (int m = 0; m < kMaxTok; ++m) {
        if (m < Mc) {
            const float s = warp_sum(acc[m]);
            if (lane == 0) logits[int64_t(m) * E + e] = s;
        }
    }
}

__device__ __forceinline__ void bf16x8_to_f32(const uint4 v, float (&f)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        f[2 * j] = __uint_as_float(w[j] << 16);
        f[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
    }
}

// logits[m][e] = sum_k x[m][k] * W[e][k], m < Mc (<= 8), H % 64 == 0. One CTA per
// kRouterRows expert rows; its 8 warps each take a contiguous eighth of k, lanes walk
// 8-element chunks of it (fp32 fma in k order), so every x chunk loaded is used by all
// rows of the CTA. Lane partials meet in a fixed butterfly reduce-scatter, warp
// partials in warp order: the result is deterministic.
constexpr int kRouterRows = 4;
template <int XDT>
__global__ void __launch_bounds__(256) router_logits_kernel(const void* __restrict__ x, int Mc,
                                                            int64_t H,
                                                            const uint16_t* __restrict__ W,
                                                            int64_t E, float* __restrict__ logits) {
    static_assert(kRouterRows * kMaxTok == 32, "one reduced value per lane");
    __shared__ float part[8][32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t e0 = int64_t(blockIdx.x) * kRouterRows;
    const int64_t slice = H / 8, kb = warp * slice;
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = 0.0f;
    for (int64_t k = kb + lane * 8; k < kb + slice; k += 256) {
        float wf[kRouterRows][8];
#pragma unroll
        for (int r = 0; r < kRouterRows; ++r) {
            if (e0 + r < E) {
                bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(W + (e0 + r) * H + k)), wf[r]);
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) wf[r][j] = 0.0f;
            }
        }
#pragma unroll
        for (int m = 0; m < kMaxTok; ++m) {
            if (m < Mc) {
                float xf[8];
                if (XDT == K3_BF16) {
                    bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(
                                      reinterpret_cast<const uint16_t*>(x) + m * H + k)), xf);
                } else {
                    const float4* xp =
                        reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + m * H + k);
                    const float4 a = __ldg(xp), b = __ldg(xp + 1);
                    xf[0] = a.x; xf[1] = a.y; xf[2] = a.z; xf[3] = a.w;
                    xf[4] = b.x; xf[5] = b.y; xf[6] = b.z; xf[7] = b.w;
                }
#pragma unroll
                for (int r = 0; r < kRouterRows; ++r)
#pragma unroll
                    for (int j = 0; j < 8; ++j) v[r * kMaxTok + m] = fmaf(xf[j], wf[r][j], v[r * kMaxTok + m]);
            }
        }
    }
    // butterfly reduce-scatter: after the step with offset o every lane keeps the half
    // of its values selected by its bit o; lane l ends with the sum of value index l
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        const bool upper = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < o; ++i) {
            const float send = upper ? v[i] : v[i + o];
            const float keep = upper ? v[i + o] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
    part[warp][lane] = v[0];
    __syncthreads();
    if (threadIdx.x < 32) {
        const int r = lane / kMaxTok, m = lane % kMaxTok;
        float sum = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; ++w) sum += part[w][lane];
        if (m < Mc && e0 + r < E) logits[int64_t(m) * E + e0 + r] = sum;
    }
}

__global__ void __launch_bounds__(256) topk_kernel(const float* __restrict__ logits, int M, int E,
                                                   const float* __restrict__ bias, int k, int renorm,
                                                   float scale, int32_t* __restrict__ idx,
                                                   float* __restrict__ w, float* __restrict__ raw,
                                                   float* __restrict__ cor, int* status) {
    const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (t >= M) return;
    topk_row(logits + int64_t(t) * E, bias, E, k, renorm, scale, idx + int64_t(t) * k,
             w + int64_t(t) * k, raw ? raw + int64_t(t) * E : nullptr,
             cor ? cor + int64_t(t) * E : nullptr, lane, status);
}

// ==================================================================== prep

struct PrepArgs {
    int mode;                      // 0: plan from idx/w (after a top-k when logits != null);
                                   // 1: identity plan (matvec)
    const float* logits;
    PlanArgs pl;
    // activation conversion (CTAs >= 1)
    const void* x;
    int x_dtype;
    int M;
    int64_t K;                     // x row length
    __half* xq_hi;
    __half* xq_lo;                 // null when the source is bf16 (hi is exact)
    float* xq_ts;
    int blocked;                   // blocked pieces with one exponent per (token, 512-k)
                                   // block, rows M..7 zeros (TMA kernels); else row-major
                                   // with one exponent per token (generic kernels)
    uint8_t* xp;                   // block-scaled path: E2M1 pieces [8M][K/2] + per-row
    uint8_t* xsf;                  // scales [8M][K/32] instead of the f16 pieces
};

__global__ void __launch_bounds__(256) prep_kernel(PrepArgs a) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (blockIdx.x > 0) {
        if (a.xp) {                        // one warp per (token, 32-block): the piece split is a
                                           // serial chain, so it is spread over many CTAs
            const uint32_t G = uint32_t(a.K / 32);            // 32-bit: no 64-bit division per warp
            const uint32_t task = (blockIdx.x - 1) * (blockDim.x >> 5) + warp;
            if (task < uint32_t(a.M) * G) {
                const int64_t t = task / G, g = task - uint32_t(t) * G;
                const float v = load_as_f32(a.x, a.x_dtype, t * a.K + 32 * g + lane);
                split_pieces(v, lane, a.xp + int64_t(kBPieces) * t * (a.K / 2) + 16 * g, a.K / 2,
                             a.xsf + int64_t(kBPieces) * t * G + g, G);
            }
            return;
        }
        if (a.blocked) {                   // CTA 1+kb: block kb of every token (warp t)
            const int64_t kb = blockIdx.x - 1;
            if (kb < a.K / 512)
                convert_block(a.x, a.x_dtype, a.M, a.K, warp, kb, a.xq_hi, a.xq_lo, a.xq_ts, lane);
            return;
        }
        // CTA 1+t: x[t][:] -> (hi, lo) f16 pieces of x * 2**-e, one exponent per token
        const int t = blockIdx.x - 1;
        if (t >= a.M) return;
        __shared__ float red[8];
        const int64_t base = int64_t(t) * a.K;
        float mx = 0.0f;
        for (int64_t i = threadIdx.x; i < a.K; i += blockDim.x)
            mx = fmaxf(mx, fabsf(load_as_f32(a.x, a.x_dtype, base + i)));
        mx = warp_max(mx);
        if (lane == 0) red[warp] = mx;
        __syncthreads();
        mx = red[0];
#pragma unroll
        for (int w = 1; w < 8; ++w) mx = fmaxf(mx, red[w]);
        const int e = f16_group_exponent(mx);
        const float sc = ldexpf(1.0f, -e);
        const bool normal_sc = isfinite(sc) && sc >= 1.17549435e-38f;
        for (int64_t i = threadIdx.x; i < a.K; i += blockDim.x) {
            const float v = load_as_f32(a.x, a.x_dtype, base + i);
            __half hi, lo;
            split_f16(normal_sc ? v * sc : ldexpf(v, -e), hi, lo);
            a.xq_hi[base + i] = hi;
            if (a.xq_lo) a.xq_lo[base + i] = lo;
        }
        if (threadIdx.x == 0) a.xq_ts[t] = ldexpf(1.0f, e);
        return;
    }
    if (a.mode == 1) identity_plan_cta(a.pl);
    else build_plan_cta(a.pl, a.logits, warp, lane);
}

// ========================================================== grouped matvec

struct GemvArgs {
    const Plan* plan;
    const k3_expert_ptrs* table;
    const uint8_t* mat_packed;     // PROJ over one plain matrix (matvec) instead of w2
    const uint8_t* mat_scales;
    int64_t K;                     // reduction length of this phase
    int64_t rows;                  // rows of one projection (I for gate/up, H or N for PROJ)
    int C;                         // k-chunks per row block
    int hilo;                      // B operand carries lo pieces
    const __half* bh;              // B pieces: row r at bh + r*K
    const __half* bl;
    const float* bts;              // B group scales: row r at bts + r*(K/32)
    float* part;                   // partial sums
    unsigned* cnt;                 // arrival counters
    int Pmax;                      // PROJ partial stride (pairs)
    // GATEUP epilogue
    __half* act_hi;
    __half* act_lo;
    float* act_ts;
    int act_kind;
    float beta, lbeta;
    // PROJ epilogue
    void* y;
    int y_dtype;
};

__device__ __forceinline__ float apply_act(int kind, float g, float u, float beta, float lbeta) {
    return act_value(kind, g, u, beta, lbeta);
}

// GATEUP: gate+up items with the activation epilogue; otherwise plain projection items
// with the combine epilogue. GROUP_TS: the B operand carries one power-of-two scale per
// (column, 32-group) -- applied per group -- instead of one per column (applied once).
template <bool GATEUP, bool GROUP_TS, bool HILO>
__global__ void __launch_bounds__(kWarps * 32, 1) gemv_kernel(GemvArgs a) {
    using Stage = StageT<HILO>;
    constexpr int kStages = stages_for<HILO>();
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    Stage* ring = reinterpret_cast<Stage*>(smem_raw + size_t(warp) * sizeof(Stage) * kStages);
    const Plan* P = a.plan;
    const int n_active = P->n_active;
    const int64_t nRb = GATEUP ? a.rows / 32 : a.rows / kItemRows;
    const int64_t n_items = int64_t(n_active) * nRb * a.C;
    const int64_t wstride = a.K / 2, sstride = a.K / 32;
    const int64_t kchunk = a.K / a.C;
    const int nst = int(kchunk / kStageK);
    const int g = lane >> 2, q = lane & 3;
    const int64_t total_warps = int64_t(gridDim.x) * kWarps;

    for (int64_t item = int64_t(blockIdx.x) * kWarps + warp; item < n_items; item += total_warps) {
        const int kc = int(item % a.C);
        const int64_t rest = item / a.C;
        const int rb = int(rest % nRb);
        const int u = int(rest / nRb);
        const int ps = P->pair_start[u];
        const int ncols = P->pair_start[u + 1] - ps;
        const int64_t k0 = int64_t(kc) * kchunk;

        const uint8_t* wp[kTiles];
        const uint8_t* sp[kTiles];
        if (GATEUP) {
            const k3_expert_ptrs ep = a.table[P->expert[u]];
#pragma unroll
            for (int t = 0; t < kTiles; ++t) {
                const int64_t r0 = int64_t(rb) * 32 + (t & 1) * 16;
                wp[t] = (t < 2 ? ep.w1_packed : ep.w3_packed) + r0 * wstride;
                sp[t] = (t < 2 ? ep.w1_scales : ep.w3_scales) + r0 * sstride;
            }
        } else {
            const uint8_t* W;
            const uint8_t* S;
            if (a.mat_packed) {
                W = a.mat_packed;
                S = a.mat_scales;
            } else {
                const k3_expert_ptrs ep = a.table[P->expert[u]];
                W = ep.w2_packed;
                S = ep.w2_scales;
            }
#pragma unroll
            for (int t = 0; t < kTiles; ++t) {
                const int64_t r0 = int64_t(rb) * kItemRows + t * 16;
                wp[t] = W + r0 * wstride;
                sp[t] = S + r0 * sstride;
            }
        }
        // B rows of this lane's copy chunks: column (lane>>4) + 2i, and ts column lane&7.
        const __half* bsrc[4];
        const __half* blsrc[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int j = (lane >> 4) + 2 * i;
            bsrc[i] = nullptr;
            blsrc[i] = nullptr;
            if (j < ncols) {
                const int64_t row = GATEUP ? P->pair_tok[ps + j] : ps + j;
                bsrc[i] = a.bh + row * a.K + k0 + (lane & 15) * 8;
                if (HILO) blsrc[i] = a.bl + row * a.K + k0 + (lane & 15) * 8;
            }
        }
        const float* tssrc = nullptr;
        if (GROUP_TS) {
            const int j = lane & 7;
            if (j < ncols) {
                const int64_t row = GATEUP ? P->pair_tok[ps + j] : ps + j;
                tssrc = a.bts + row * sstride + k0 / 32 + (lane >> 3);
            }
        }

        auto issue = [&](int s) {
            Stage& st = ring[s % kStages];
            const int64_t kb = (k0 + int64_t(s) * kStageK) / 2;     // packed byte offset
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int t = i >> 1, r = (lane >> 2) + 8 * (i & 1), cc = lane & 3;
                cp_async_16_cg(smem_u32(&st.w[t][r][(cc ^ ((r >> 1) & 3)) * 16]),
                               wp[t] + r * wstride + kb + cc * 16);
            }
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int c = lane + 32 * i, t = c >> 4, r = c & 15;
                cp_async_4(smem_u32(&st.s[t][r][0]), sp[t] + r * sstride + kb / 16);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int j = (lane >> 4) + 2 * i, ch = lane & 15;
                const int pc = (ch ^ ((j & 1) << 2)) * 8;
                if (bsrc[i]) cp_async_16_ca(smem_u32(&st.bh[j][pc]), bsrc[i] + s * kStageK);
                if (HILO && blsrc[i]) cp_async_16_ca(smem_u32(&st.bl[j][pc]), blsrc[i] + s * kStageK);
            }
            if (GROUP_TS) {
                if (tssrc) cp_async_4(smem_u32(&st.ts[lane >> 3][lane & 7]), tssrc + s * (kStageK / 32));
                else st.ts[lane >> 3][lane & 7] = 0.0f;
            }
        };

        float acc[kTiles][4];
#pragma unroll
        for (int t = 0; t < kTiles; ++t)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[t][i] = 0.0f;

#pragma unroll
        for (int s = 0; s < kStages - 1; ++s) {
            if (s < nst) issue(s);
            cp_async_commit();
        }
        for (int s = 0; s < nst; ++s) {
            if (s + kStages - 1 < nst) issue(s + kStages - 1);
            cp_async_commit();
            cp_async_wait<kStages - 1>();
            __syncwarp();
            const Stage& st = ring[s % kStages];
#pragma unroll
            for (int gp = 0; gp < 2; ++gp) {
                uint4 X[2], XL[2];
                float2 tsv[2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int G = 2 * gp + h;
                    const int pc = (((G * 4 + q) ^ ((g & 1) << 2))) * 8;
                    X[h] = make_uint4(0, 0, 0, 0);
                    XL[h] = make_uint4(0, 0, 0, 0);
                    if (g < ncols) {
                        X[h] = *reinterpret_cast<const uint4*>(&st.bh[g][pc]);
                        if (HILO) XL[h] = *reinterpret_cast<const uint4*>(&st.bl[g][pc]);
                    }
                    if (GROUP_TS) tsv[h] = *reinterpret_cast<const float2*>(&st.ts[G][2 * q]);
                    else tsv[h] = make_float2(1.0f, 1.0f);
                }
#pragma unroll
                for (int t = 0; t < kTiles; ++t) {
                    uint32_t R0, R1, R2, R3;
                    {
                        const int m = lane >> 3, r = (lane & 7) + 8 * (m & 1), cc = 2 * gp + (m >> 1);
                        ldmatrix_x4(smem_u32(&st.w[t][r][(cc ^ ((r >> 1) & 3)) * 16]), R0, R1, R2, R3);
                    }
                    const uint32_t swg = *reinterpret_cast<const uint32_t*>(&st.s[t][g][0]);
                    const uint32_t swg8 = *reinterpret_cast<const uint32_t*>(&st.s[t][g + 8][0]);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int G = 2 * gp + h;
                        uint32_t f0, f1, f2, f3, e0, e1, e2, e3;
                        e2m1x8_to_f16x8(h ? R2 : R0, f0, f1, f2, f3);
                        e2m1x8_to_f16x8(h ? R3 : R1, e0, e1, e2, e3);
                        float tmp[4];
                        mma_f16_16816_zc(tmp, f0, e0, f1, e1, X[h].x, X[h].y);
                        mma_f16_16816(tmp, f2, e2, f3, e3, X[h].z, X[h].w);
                        if (HILO) {
                            mma_f16_16816(tmp, f0, e0, f1, e1, XL[h].x, XL[h].y);
                            mma_f16_16816(tmp, f2, e2, f3, e3, XL[h].z, XL[h].w);
                        }
                        const float rs0 = e8m0_to_f32((swg >> (8 * G)) & 0xffu);
                        const float rs1 = e8m0_to_f32((swg8 >> (8 * G)) & 0xffu);
                        if (GROUP_TS) {
                            acc[t][0] = fmaf(rs0 * tsv[h].x, tmp[0], acc[t][0]);
                            acc[t][1] = fmaf(rs0 * tsv[h].y, tmp[1], acc[t][1]);
                            acc[t][2] = fmaf(rs1 * tsv[h].x, tmp[2], acc[t][2]);
                            acc[t][3] = fmaf(rs1 * tsv[h].y, tmp[3], acc[t][3]);
                        } else {
                            acc[t][0] = fmaf(rs0, tmp[0], acc[t][0]);
                            acc[t][1] = fmaf(rs0, tmp[1], acc[t][1]);
                            acc[t][2] = fmaf(rs1, tmp[2], acc[t][2]);
                            acc[t][3] = fmaf(rs1, tmp[3], acc[t][3]);
                        }
                    }
                }
            }
            __syncwarp();
        }

        if (!GROUP_TS) {                       // one scale per column: apply it once
            float c0s = 0.0f, c1s = 0.0f;
            const int c0 = 2 * q;
            if (c0 < ncols) c0s = a.bts[GATEUP ? P->pair_tok[ps + c0] : ps + c0];
            if (c0 + 1 < ncols) c1s = a.bts[GATEUP ? P->pair_tok[ps + c0 + 1] : ps + c0 + 1];
#pragma unroll
            for (int t = 0; t < kTiles; ++t) {
                acc[t][0] *= c0s;
                acc[t][1] *= c1s;
                acc[t][2] *= c0s;
                acc[t][3] *= c1s;
            }
        }

        // ---- partial sums to scratch, then the last arrival reduces them
        unsigned* counter;
        unsigned target;
        if (GATEUP) {
            float* base = a.part + (rest * a.C + kc) * (kMaxTok * kItemRows);
#pragma unroll
            for (int t = 0; t < kTiles; ++t) {
                const int r0 = t * 16 + g, c0 = 2 * q;
                if (c0 < ncols) {
                    base[c0 * kItemRows + r0] = acc[t][0];
                    base[c0 * kItemRows + r0 + 8] = acc[t][2];
                }
                if (c0 + 1 < ncols) {
                    base[(c0 + 1) * kItemRows + r0] = acc[t][1];
                    base[(c0 + 1) * kItemRows + r0 + 8] = acc[t][3];
                }
            }
            counter = a.cnt + rest;
            target = unsigned(a.C);
        } else {
#pragma unroll
            for (int t = 0; t < kTiles; ++t) {
                const int64_t r0 = int64_t(rb) * kItemRows + t * 16 + g;
                const int c0 = 2 * q;
                if (c0 < ncols) {
                    float* b = a.part + (int64_t(kc) * a.Pmax + ps + c0) * a.rows;
                    b[r0] = acc[t][0];
                    b[r0 + 8] = acc[t][2];
                }
                if (c0 + 1 < ncols) {
                    float* b = a.part + (int64_t(kc) * a.Pmax + ps + c0 + 1) * a.rows;
                    b[r0] = acc[t][1];
                    b[r0 + 8] = acc[t][3];
                }
            }
            counter = a.cnt + rb;
            target = unsigned(n_active) * unsigned(a.C);
        }
        __threadfence();
        __syncwarp();
        unsigned old = 0;
        if (lane == 0) old = atomicAdd(counter, 1u);
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old + 1 != target) continue;
        __threadfence();
        if (lane == 0) *counter = 0u;                  // ready for the next call

        if (GATEUP) {
            // lane = act row; gate rows are partial rows 0..31, up rows 32..63
            const int64_t I = a.rows;
            for (int j = 0; j < ncols; ++j) {
                float gs = 0.0f, us = 0.0f;
                for (int c = 0; c < a.C; ++c) {
                    const float* base = a.part + (rest * a.C + c) * (kMaxTok * kItemRows) + j * kItemRows;
                    gs += __ldcg(base + lane);
                    us += __ldcg(base + 32 + lane);
                }
                const int p = ps + j;
                const float v = apply_act(a.act_kind, gs, us, a.beta, a.lbeta) * P->pair_w[p];
                const int e = f16_group_exponent(warp_max(fabsf(v)));
                __half hi, lo;
                split_f16(ldexpf(v, -e), hi, lo);
                const int64_t o = int64_t(p) * I + int64_t(rb) * 32 + lane;
                a.act_hi[o] = hi;
                a.act_lo[o] = lo;
                if (lane == 0) a.act_ts[int64_t(p) * (I / 32) + rb] = ldexpf(1.0f, e);
            }
        } else {
            const int np = P->n_pairs, M = P->M;
            for (int t = 0; t < M; ++t) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int64_t row = int64_t(rb) * kItemRows + lane + 32 * h;
                    float yv = 0.0f;
                    for (int p = 0; p < np; ++p) {
                        if (P->pair_tok[p] != t) continue;
                        for (int c = 0; c < a.C; ++c)
                            yv += __ldcg(a.part + (int64_t(c) * a.Pmax + p) * a.rows + row);
                    }
                    store_from_f32(a.y, a.y_dtype, int64_t(t) * a.rows + row, yv);
                }
            }
        }
    }
}

// ================================================================== host side

namespace {

// Smallest k-split C (a divisor of K/128 leaving >= 2 stages per item) that gives at
// least `target` items; falls back to the largest allowed split.
int choose_split(int64_t base_items, int64_t K, int64_t target) {
    const int64_t nst = K / kStageK;
    int best = 1;
    for (int64_t c = 1; c <= nst; ++c) {
        if (nst % c) continue;
        if (nst / c < 2 && c > 1) break;
        best = int(c);
        if (base_items * c >= target) break;
    }
    return best;
}

template <bool G, bool T, bool H>
int set_smem(const char* what) {
    return cuda_check(cudaFuncSetAttribute(gemv_kernel<G, T, H>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           int(smem_bytes_for<H>())),
                      what);
}

OncePerContext g_smem_attr;
int configure_smem() {
    return g_smem_attr.run([] {
        if (int rc = set_smem<true, false, false>("cudaFuncSetAttribute(gemv gate/up bf16)")) return rc;
        if (int rc = set_smem<true, false, true>("cudaFuncSetAttribute(gemv gate/up f32)")) return rc;
        if (int rc = set_smem<false, true, true>("cudaFuncSetAttribute(gemv down)")) return rc;
        if (int rc = set_smem<false, false, false>("cudaFuncSetAttribute(gemv matvec bf16)")) return rc;
        return set_smem<false, false, true>("cudaFuncSetAttribute(gemv matvec f32)");
    });
}

size_t carve(size_t& off, size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 256);
    return o;
}

// k-split for the TMA kernels: the smallest divisor C of K/512 for which n_base*C items
// split into `grid` contiguous ranges keep the longest range within 5% of the mean
// (else the best balance found).
int choose_split_tma(int64_t n_base, int64_t K, int64_t grid) {
    const int64_t nst = K / kTStageK;
    int best = 1;
    double best_eff = -1.0;
    for (int64_t c = 1; c <= nst; ++c) {
        if (nst % c) continue;
        const int64_t n = n_base * c;
        const double eff = double(n) / double(((n + grid - 1) / grid) * grid);
        if (eff >= 0.95) return int(c);
        if (eff > best_eff + 1e-9) {
            best_eff = eff;
            best = int(c);
        }
    }
    return best;
}

bool pool_usable(const k3_moe_params& p) {
    const k3_expert_pool* pl = p.pool;
    return pl && pl->w1_packed && pl->w1_scales && pl->w3_packed && pl->w3_scales &&
           pl->w2_packed && pl->w2_scales && pl->num_slots >= p.num_experts + (p.has_shared ? 1 : 0) &&
           p.hidden % kTStageK == 0 && p.inter % kTStageK == 0;
}

// The block-scaled kernels read the re-laid scales and either the tiles or the row-major
// packed codes; a pool may carry the re-laid copies alone (a streamed staging pool).
bool pool_bs(const k3_moe_params& p) {
    const k3_expert_pool* pl = p.pool;
    if (!pl || !pl->w1_scales_tc || !pl->w3_scales_tc || !pl->w2_scales_tc) return false;
    const bool tiles = pl->w1_tiles && pl->w3_tiles && pl->w2_tiles;
    const bool packed = pl->w1_packed && pl->w3_packed && pl->w2_packed;
    return (tiles || packed) && pl->num_slots >= p.num_experts + (p.has_shared ? 1 : 0) &&
           p.hidden % kTStageK == 0 && p.inter % kTStageK == 0;
}

// k-split for the block-scaled kernels: as choose_split_tma, over 256-k stages.
int choose_split_bs(int64_t n_base, int64_t K, int64_t grid) {
    const int64_t nst = K / kBStageK;
    int best = 1;
    double best_eff = -1.0;
    for (int64_t c = 1; c <= nst; ++c) {
        if (nst % c) continue;
        const int64_t n = n_base * c;
        const double eff = double(n) / double(((n + grid - 1) / grid) * grid);
        if (eff >= 0.95) return int(c);
        if (eff > best_eff + 1e-9) {
            best_eff = eff;
            best = int(c);
        }
    }
    return best;
}

// H_router: width of the router input (the expert input's, p.hidden, unless the MoE is
// latent); it sets the router's k-slices.
DecodeLayout decode_layout(const k3_moe_params& p, int64_t M, int sms, int64_t H_router = 0) {
    if (H_router <= 0) H_router = p.hidden;
    DecodeLayout L{};
    L.M = M;
    L.H = p.hidden;
    L.I = p.inter;
    L.E = p.num_experts;
    L.U = std::min<int64_t>(p.num_experts, M * p.top_k) + (p.has_shared ? 1 : 0);
    L.P = M * p.top_k + (p.has_shared ? M : 0);
    L.bs = pool_bs(p);
    L.tma = L.bs || pool_usable(p);
    size_t off = 0;
    if (L.bs) {
        // keys: (128-row block, active expert) in both phases
        L.CA = choose_split_bs(L.U * (L.I / kBRows), L.H, sms);
        L.CB = choose_split_bs(L.U * (L.H / kBRows), L.I, sms);
        L.plan = carve(off, sizeof(Plan));
        L.logits = carve(off, sizeof(float) * M * L.E);
        L.route_idx = carve(off, sizeof(int32_t) * M * p.top_k);
        L.route_w = carve(off, sizeof(float) * M * p.top_k);
        L.xq_hi = carve(off, size_t(kBMaxN) * (L.H / 2));              // x pieces
        L.xq_ts = carve(off, size_t(kBMaxN) * (L.H / 32));              // their per-row scales
        L.KQ = 1;
        for (int64_t c = 1; c <= H_router / 512 && c <= 16; ++c) {  // router k-slices: >= one CTA per SM
            if ((H_router / 512) % c) continue;
            L.KQ = int(c);
            if (((L.E + 15) / 16) * c >= sms) break;
        }
        L.logit_part = carve(off, sizeof(float) * L.KQ * M * L.E);
        L.route_done = carve(off, sizeof(unsigned) * (2 + (L.E + 15) / 16));   // + piece-task counter
        L.route_keys = carve(off, sizeof(uint32_t) * M * L.E);
        L.route_scores = carve(off, sizeof(float) * M * L.E);
        L.act_hi = carve(off, size_t(L.U) * kBMaxN * (L.I / 2));        // act pieces
        L.act_ts = carve(off, size_t(L.U) * (L.I / 128) * kBChunk);
        L.partA = carve(off, sizeof(float) * L.U * (L.I / kBRows) * L.CA * 2 * kMaxTok * kBRows);
        L.cntA = carve(off, sizeof(unsigned) * L.U * (L.I / kBRows));
        L.partB = carve(off, sizeof(float) * L.U * (L.H / kBRows) * L.CB * kMaxTok * kBRows);
        L.cntB = carve(off, sizeof(unsigned) * L.U * (L.H / kBRows));
        L.y_pair = carve(off, sizeof(float) * L.P * L.H);              // one output row per pair
        L.total = off;
        return L;
    }
    if (L.tma) {
        // keys: gate/up = (active expert, 64-row block); down = 128-row block of y
        L.CA = choose_split_tma(L.U * (L.I / 64), L.H, sms);
        L.CB = choose_split_tma(L.U * (L.H / kTRows), L.I, sms);
        L.ppad = L.U * kMaxTok;             // rows of the token-space activation tensors
        L.tspad = L.I / 32;
        L.plan = carve(off, sizeof(Plan));
        L.logits = carve(off, sizeof(float) * M * L.E);
        L.route_idx = carve(off, sizeof(int32_t) * M * p.top_k);
        L.route_w = carve(off, sizeof(float) * M * p.top_k);
        L.xq_hi = carve(off, sizeof(__half) * kMaxTok * L.H);
        L.xq_lo = carve(off, sizeof(__half) * kMaxTok * L.H);
        L.xq_ts = carve(off, sizeof(float) * kMaxTok * (L.H / 512));
        L.KQ = 1;
        for (int64_t c = 1; c <= L.H / 512 && c <= 16; ++c) {  // router k-slices: >= one CTA per SM
            if ((L.H / 512) % c) continue;
            L.KQ = int(c);
            if (((L.E + 15) / 16) * c >= sms) break;
        }
        L.logit_part = carve(off, sizeof(float) * L.KQ * M * L.E);
        L.route_done = carve(off, sizeof(unsigned) * (2 + (L.E + 15) / 16));   // + piece-task counter
        L.route_keys = carve(off, sizeof(uint32_t) * M * L.E);
        L.route_scores = carve(off, sizeof(float) * M * L.E);
        L.act_hi = carve(off, sizeof(__half) * L.ppad * L.I);
        L.act_lo = carve(off, sizeof(__half) * L.ppad * L.I);
        L.act_ts = carve(off, sizeof(float) * L.ppad * L.tspad);
        L.partA = carve(off, sizeof(float) * L.U * (L.I / 64) * L.CA * kMaxTok * kTRows);
        L.cntA = carve(off, sizeof(unsigned) * L.U * (L.I / 64));
        L.partB = carve(off, sizeof(float) * (L.H / kTRows) * L.U * L.CB * kMaxTok * kTRows);
        L.cntB = carve(off, sizeof(unsigned) * (L.H / kTRows));
        L.total = off;
        return L;
    }
    const int64_t target = int64_t(sms) * kWarps * 4;
    L.CA = choose_split(L.U * (L.I / 32), L.H, target);
    L.CB = choose_split(L.U * (L.H / kItemRows), L.I, target);
    L.plan = carve(off, sizeof(Plan));
    L.logits = carve(off, sizeof(float) * M * L.E);
    L.route_idx = carve(off, sizeof(int32_t) * M * p.top_k);   // when the caller passes NULL
    L.route_w = carve(off, sizeof(float) * M * p.top_k);
    L.xq_hi = carve(off, sizeof(__half) * kMaxTok * L.H);
    L.xq_lo = carve(off, sizeof(__half) * kMaxTok * L.H);
    L.xq_ts = carve(off, sizeof(float) * kMaxTok);
    L.act_hi = carve(off, sizeof(__half) * L.P * L.I);
    L.act_lo = carve(off, sizeof(__half) * L.P * L.I);
    L.act_ts = carve(off, sizeof(float) * L.P * (L.I / 32));
    L.partA = carve(off, sizeof(float) * L.U * (L.I / 32) * L.CA * kMaxTok * kItemRows);
    L.cntA = carve(off, sizeof(unsigned) * L.U * (L.I / 32));
    L.partB = carve(off, sizeof(float) * L.CB * L.P * L.H);
    L.cntB = carve(off, sizeof(unsigned) * (L.H / kItemRows));
    L.total = off;
    return L;
}

int check_moe_params(const k3_moe_params* p, int64_t M) {
    if (!p) return fail(K3_ERR_INVALID, "k3_moe_params is NULL");
    if (M < 1 || M > kMaxTok) return fail(K3_ERR_UNSUPPORTED, "decode path takes 1..8 tokens, got M=" + std::to_string(M));
    if (p->hidden <= 0 || p->hidden % 128) return fail(K3_ERR_UNSUPPORTED, "hidden must be a positive multiple of 128");
    if (p->inter <= 0 || p->inter % 128) return fail(K3_ERR_UNSUPPORTED, "inter must be a positive multiple of 128");
    if (p->num_experts < 1 || p->num_experts > kMaxExperts) return fail(K3_ERR_UNSUPPORTED, "num_experts must be 1..1024");
    if (p->top_k < 1 || p->top_k > kMaxTopK || p->top_k > p->num_experts) return fail(K3_ERR_UNSUPPORTED, "top_k must be 1..min(16, E)");
    if (!p->experts) return fail(K3_ERR_INVALID, "expert table is NULL");
    if (p->activation != K3_ACT_SILU && p->activation != K3_ACT_SITU) return fail(K3_ERR_INVALID, "unknown activation");
    return K3_OK;
}

int check_ws(void* ws, size_t bytes, size_t need) {
    if (!ws) return fail(K3_ERR_WORKSPACE, "workspace is NULL");
    if (reinterpret_cast<uintptr_t>(ws) % 256) return fail(K3_ERR_WORKSPACE, "workspace must be 256-byte aligned");
    if (bytes < need) return fail(K3_ERR_WORKSPACE, "workspace too small: need " + std::to_string(need) + " bytes");
    return K3_OK;
}

int launch_router_logits(const void* x, int xdt, int Mc, int64_t H, const uint16_t* W, int64_t E,
                         float* logits, cudaStream_t s) {
    prof_begin(K3_PROF_ROUTER, s);
    if (H % 64 == 0) {
        const int blocks = int((E + kRouterRows - 1) / kRouterRows);
        if (xdt == K3_BF16)
            router_logits_kernel<K3_BF16><<<blocks, 256, 0, s>>>(x, Mc, H, W, E, logits);
        else
            router_logits_kernel<K3_F32><<<blocks, 256, 0, s>>>(x, Mc, H, W, E, logits);
    } else {
        const int blocks = int((E * 32 + 255) / 256);
        if (xdt == K3_BF16)
            router_logits_rowwarp_kernel<K3_BF16><<<blocks, 256, 0, s>>>(x, Mc, H, W, E, logits);
        else
            router_logits_rowwarp_kernel<K3_F32><<<blocks, 256, 0, s>>>(x, Mc, H, W, E, logits);
    }
    prof_end(K3_PROF_ROUTER, s);
    K3_CHECK_LAUNCH("router_logits_kernel");
    return K3_OK;
}

// Tensor maps over a [slots][rows][bytes] pool and its [slots][rows][cols/32] scales.
int pool_maps(CUtensorMap* wmap, CUtensorMap* smap, const uint8_t* packed, const uint8_t* scales,
              int64_t rows, int64_t cols, int64_t slots, uint32_t box_rows) {
    const uint64_t dp[3] = {uint64_t(cols / 2), uint64_t(rows), uint64_t(slots)};
    const uint64_t sp[2] = {uint64_t(cols / 2), uint64_t(rows * cols / 2)};
    const uint32_t bp[3] = {128, box_rows, 1};
    if (int rc = encode_map(wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, packed, dp, sp, bp,
                            CU_TENSOR_MAP_SWIZZLE_128B))
        return rc;
    const uint64_t ds[3] = {uint64_t(cols / 32), uint64_t(rows), uint64_t(slots)};
    const uint64_t ss[2] = {uint64_t(cols / 32), uint64_t(rows * cols / 32)};
    const uint32_t bs[3] = {uint32_t(kTGroups), box_rows, 1};
    return encode_map(smap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, scales, ds, ss, bs,
                      CU_TENSOR_MAP_SWIZZLE_NONE);
}

// Map over activation pieces in the blocked [k/32][column][32] layout.
int blocked_map(CUtensorMap* m, const __half* base, int64_t cols, int64_t K) {
    const uint64_t d[3] = {32, uint64_t(cols), uint64_t(K / 32)};
    const uint64_t st[2] = {64, uint64_t(cols) * 64};
    const uint32_t b[3] = {32, uint32_t(kMaxTok), uint32_t(kTGroups)};
    return encode_map(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, base, d, st, b,
                      CU_TENSOR_MAP_SWIZZLE_NONE);
}

int decode_tma(const k3_moe_params* p, const DecodeLayout& L, uint8_t* ws, bool x_hilo, void* y,
               int ydt, int sms, cudaStream_t s) {
    const k3_expert_pool& pl = *p->pool;
    Plan* plan = reinterpret_cast<Plan*>(ws + L.plan);
    __half* act_hi = reinterpret_cast<__half*>(ws + L.act_hi);
    __half* act_lo = reinterpret_cast<__half*>(ws + L.act_lo);
    float* act_ts = reinterpret_cast<float*>(ws + L.act_ts);

    TMaps ma{};
    if (int rc = pool_maps(&ma.wA, &ma.sA, pl.w1_packed, pl.w1_scales, L.I, L.H, pl.num_slots, 64)) return rc;
    if (int rc = pool_maps(&ma.wB, &ma.sB, pl.w3_packed, pl.w3_scales, L.I, L.H, pl.num_slots, 64)) return rc;
    if (int rc = blocked_map(&ma.bh, reinterpret_cast<__half*>(ws + L.xq_hi), kMaxTok, L.H)) return rc;
    if (x_hilo)
        if (int rc = blocked_map(&ma.bl, reinterpret_cast<__half*>(ws + L.xq_lo), kMaxTok, L.H)) return rc;
    TArgs ta{};
    ta.plan = plan;
    ta.K = L.H;
    ta.rows = L.I;
    ta.C = L.CA;
    ta.status = &plan->status;
    ta.part = reinterpret_cast<float*>(ws + L.partA);
    ta.cnt = reinterpret_cast<unsigned*>(ws + L.cntA);
    ta.maxseg = L.CA;
    ta.act_hi = act_hi;
    ta.act_lo = act_lo;
    ta.act_ts = act_ts;
    ta.act_rows = L.ppad;
    ta.act_groups = int(L.tspad);
    ta.act_kind = p->activation;
    ta.beta = p->situ_beta;
    ta.lbeta = p->situ_linear_beta;
    ta.bts_tok = reinterpret_cast<float*>(ws + L.xq_ts);
    prof_begin(K3_PROF_GATEUP, s);
    int rc = launch_tma_gateup(ma, ta, x_hilo, sms, s);
    prof_end(K3_PROF_GATEUP, s);
    if (rc) return rc;

    TMaps mb{};
    if (int rc2 = pool_maps(&mb.wA, &mb.sA, pl.w2_packed, pl.w2_scales, L.H, L.I, pl.num_slots, kTRows)) return rc2;
    if (int rc2 = blocked_map(&mb.bh, act_hi, L.ppad, L.I)) return rc2;
    if (int rc2 = blocked_map(&mb.bl, act_lo, L.ppad, L.I)) return rc2;
    {
        // [group][expert*8 + token] with the column innermost: x = 8u, a multiple of 8 floats
        const uint64_t d[2] = {uint64_t(L.ppad), uint64_t(L.tspad)};
        const uint64_t st[1] = {uint64_t(L.ppad) * 4};
        const uint32_t b[2] = {uint32_t(kMaxTok), uint32_t(kTGroups)};
        if (int rc2 = encode_map(&mb.bts, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, act_ts, d, st, b,
                                 CU_TENSOR_MAP_SWIZZLE_NONE))
            return rc2;
    }
    TArgs tb{};
    tb.plan = plan;
    tb.K = L.I;
    tb.rows = L.H;
    tb.C = L.CB;
    tb.status = &plan->status;
    tb.part = reinterpret_cast<float*>(ws + L.partB);
    tb.cnt = reinterpret_cast<unsigned*>(ws + L.cntB);
    tb.maxseg = int(L.U * L.CB);
    tb.y = y;
    tb.y_dtype = ydt;
    prof_begin(K3_PROF_DOWN, s);
    rc = launch_tma_proj(mb, tb, true, true, sms, s);
    prof_end(K3_PROF_DOWN, s);
    return rc;
}

// Map over a packed pool [slots][rows][cols/2]: 128-byte x 128-row boxes, 128-byte swizzle.
int packed_map(CUtensorMap* m, const uint8_t* packed, int64_t rows, int64_t cols, int64_t slots) {
    const uint64_t d[3] = {uint64_t(cols / 2), uint64_t(rows), uint64_t(slots)};
    const uint64_t st[2] = {uint64_t(cols / 2), uint64_t(rows * cols / 2)};
    const uint32_t b[3] = {128, uint32_t(kBRows), 1};
    return encode_map(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, packed, d, st, b, CU_TENSOR_MAP_SWIZZLE_128B);
}

// Map over a tile pool [slots * rows/128][cols/256][128][128]: one box = one tile.
int tiles_map(CUtensorMap* m, const uint8_t* tiles, int64_t rows, int64_t cols, int64_t slots) {
    const uint64_t d[4] = {128, 128, uint64_t(cols / 256), uint64_t(slots * (rows / 128))};
    const uint64_t st[3] = {128, 128 * 128, uint64_t(128 * 128) * uint64_t(cols / 256)};
    const uint32_t b[4] = {128, 128, 1, 1};
    return encode_map(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, tiles, d, st, b, CU_TENSOR_MAP_SWIZZLE_128B);
}

// Block-scaled gate/up + down launches (the plan and x pieces are already in `ws`).
int decode_bs(const k3_moe_params* p, const DecodeLayout& L, uint8_t* ws, int M, void* y, int ydt,
              int sms, cudaStream_t s) {
    const k3_expert_pool& pl = *p->pool;
    Plan* plan = reinterpret_cast<Plan*>(ws + L.plan);
    uint8_t* act_p = ws + L.act_hi;
    uint8_t* act_sf = ws + L.act_ts;

    const bool tiled = pl.w1_tiles && pl.w3_tiles && pl.w2_tiles;
    BMaps ma{};
    if (tiled) {
        if (int rc = tiles_map(&ma.a0, pl.w1_tiles, L.I, L.H, pl.num_slots)) return rc;
        if (int rc = tiles_map(&ma.a1, pl.w3_tiles, L.I, L.H, pl.num_slots)) return rc;
    } else {
        if (int rc = packed_map(&ma.a0, pl.w1_packed, L.I, L.H, pl.num_slots)) return rc;
        if (int rc = packed_map(&ma.a1, pl.w3_packed, L.I, L.H, pl.num_slots)) return rc;
    }
    {
        const uint64_t d[2] = {uint64_t(L.H / 2), uint64_t(kBPieces * M)};
        const uint64_t st[1] = {uint64_t(L.H / 2)};
        const uint32_t b[2] = {128, uint32_t(kBPieces)};                // one token's pieces
        if (int rc = encode_map(&ma.b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, ws + L.xq_hi, d, st, b,
                                CU_TENSOR_MAP_SWIZZLE_128B))
            return rc;
    }
    {   // the pieces' per-row scales [8M][H/32]: one token's 8 rows x 16 bytes (512 k) a box
        const uint64_t d[2] = {uint64_t(L.H / 32), uint64_t(kBPieces * M)};
        const uint64_t st[1] = {uint64_t(L.H / 32)};
        const uint32_t b[2] = {16, uint32_t(kBPieces)};
        if (int rc = encode_map(&ma.sfb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, ws + L.xq_ts, d, st, b,
                                CU_TENSOR_MAP_SWIZZLE_NONE))
            return rc;
    }
    BArgs ta{};
    ta.plan = plan;
    ta.K = L.H;
    ta.rows = L.I;
    ta.C = L.CA;
    ta.status = &plan->status;
    ta.part = reinterpret_cast<float*>(ws + L.partA);
    ta.cnt = reinterpret_cast<unsigned*>(ws + L.cntA);
    ta.maxseg = L.CA;
    ta.sfa0 = pl.w1_scales_tc;
    ta.sfa1 = pl.w3_scales_tc;
    ta.tiled = tiled ? 1 : 0;
    ta.sf_slot = (L.I / 128) * (L.H / 128) * kBChunk;
    ta.act_p = act_p;
    ta.act_sf = act_sf;
    ta.act_kind = p->activation;
    ta.beta = p->situ_beta;
    ta.lbeta = p->situ_linear_beta;
    // the gate/up launch follows the plan producer (router, prep or pairs plan) directly:
    // it waits for it before copying the plan, and its producer loads each pair's piece
    // scales as stored, from which the MMA warp writes the scale chunks (no gather launch)
    ta.plan_in_prev = 1;
    prof_begin(K3_PROF_GATEUP, s);
    int rc = launch_bs_gateup_rawsfb(ma, ta, sms, s);
    prof_end(K3_PROF_GATEUP, s);
    if (rc) return rc;

    BMaps mb{};
    if (int rc2 = tiled ? tiles_map(&mb.a0, pl.w2_tiles, L.H, L.I, pl.num_slots)
                        : packed_map(&mb.a0, pl.w2_packed, L.H, L.I, pl.num_slots))
        return rc2;
    {
        const uint64_t d[3] = {uint64_t(L.I / 2), uint64_t(kBMaxN), uint64_t(L.U)};
        const uint64_t st[2] = {uint64_t(L.I / 2), uint64_t(kBMaxN) * uint64_t(L.I / 2)};
        const uint32_t b[3] = {128, uint32_t(kBPieces), 1};
        if (int rc2 = encode_map(&mb.b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, act_p, d, st, b,
                                 CU_TENSOR_MAP_SWIZZLE_128B))
            return rc2;
    }
    BArgs tb{};
    tb.plan = plan;
    tb.K = L.I;
    tb.rows = L.H;
    tb.C = L.CB;
    tb.status = &plan->status;
    tb.part = reinterpret_cast<float*>(ws + L.partB);
    tb.cnt = reinterpret_cast<unsigned*>(ws + L.cntB);
    tb.maxseg = L.CB;
    tb.sfa0 = pl.w2_scales_tc;
    tb.tiled = tiled ? 1 : 0;
    tb.sf_slot = (L.H / 128) * (L.I / 128) * kBChunk;
    tb.sfb = act_sf;
    tb.y_pair = reinterpret_cast<float*>(ws + L.y_pair);
    tb.early_a = 1;     // W2 tiles stream on the SMs the gate/up launch's early finishers free
    prof_begin(K3_PROF_DOWN, s);
    rc = launch_bs_down(mb, tb, sms, s);
    prof_end(K3_PROF_DOWN, s);
    if (rc) return rc;
    prof_begin(K3_PROF_OTHER, s);
    rc = launch_combine(plan, tb.y_pair, L.H, M, y, ydt, s);
    prof_end(K3_PROF_OTHER, s);
    return rc;
}

// One expert's SwiGLU FFN for M <= 8 tokens (LatentMoE.expert_forward, moe.py:90-103):
// three launches -- x pieces (launch_mv_prep), gate/up, down -- over the identity plan
// (one item of M tokens, weight 1), which both block-scaled launches build themselves, so
// neither waits for a plan and both request their first weight stages at once. The
// expert's pools are addressed as one-slot pools at its slot; the down launch writes the
// tokens' rows of y directly (the identity plan's pair t is token t), so no combine runs.
struct FfnLayout {
    int64_t U, keysA, keysB;
    int CA, CB;
    size_t status, xp, sfb, act_p, act_sf, partA, partB, cnt, total;
};

FfnLayout ffn_layout(const k3_moe_params& p, int64_t M, int sms) {
    FfnLayout L{};
    L.U = (M + kMaxTok - 1) / kMaxTok;
    L.keysA = L.U * (p.inter / kBRows);
    L.keysB = L.U * (p.hidden / kBRows);
    L.CA = choose_split_bs(L.keysA, p.hidden, sms);
    L.CB = choose_split_bs(L.keysB, p.inter, sms);
    size_t off = 0;
    L.status = carve(off, sizeof(int));
    L.xp = carve(off, size_t(L.U) * kBMaxN * (p.hidden / 2));
    L.sfb = carve(off, size_t(L.U) * (p.hidden / 128) * kBChunk);
    L.act_p = carve(off, size_t(L.U) * kBMaxN * (p.inter / 2));
    L.act_sf = carve(off, size_t(L.U) * (p.inter / 128) * kBChunk);
    L.partA = carve(off, sizeof(float) * size_t(L.keysA) * L.CA * 2 * kMaxTok * kBRows);
    L.partB = carve(off, sizeof(float) * size_t(L.keysB) * L.CB * kMaxTok * kBRows);
    L.cnt = carve(off, sizeof(unsigned) * size_t(L.keysA + L.keysB));   // gate/up keys, then down keys
    L.total = off;
    return L;
}

int expert_ffn_bs(const k3_moe_params* p, const void* x, int xdt, int64_t M, int64_t e, void* y, int ydt,
                  uint8_t* ws, const FfnLayout& L, cudaStream_t s) {
    int rc = configure_smem();
    if (rc) return rc;
    const int sms = num_sms();
    const k3_expert_pool& pl = *p->pool;
    const int64_t H = p->hidden, I = p->inter;
    const bool tiled = pl.w1_tiles && pl.w3_tiles && pl.w2_tiles;
    const size_t sfA = size_t(I / 128) * (H / 128) * kBChunk;     // scale-chunk bytes of one slot
    const size_t sfB = size_t(H / 128) * (I / 128) * kBChunk;
    const size_t codes = size_t(I) * (H / 2);                      // code bytes of one slot
    int* status = reinterpret_cast<int*>(ws + L.status);
    unsigned* cnt = reinterpret_cast<unsigned*>(ws + L.cnt);
    BMaps ma{};
    if (tiled) {
        if ((rc = tiles_map(&ma.a0, pl.w1_tiles + e * codes, I, H, 1))) return rc;
        if ((rc = tiles_map(&ma.a1, pl.w3_tiles + e * codes, I, H, 1))) return rc;
    } else {
        if ((rc = packed_map(&ma.a0, pl.w1_packed + e * codes, I, H, 1))) return rc;
        if ((rc = packed_map(&ma.a1, pl.w3_packed + e * codes, I, H, 1))) return rc;
    }
    {
        const uint64_t d[2] = {uint64_t(H / 2), uint64_t(kBPieces * M)};
        const uint64_t st[1] = {uint64_t(H / 2)};
        const uint32_t b[2] = {128, uint32_t(kBPieces)};                // one token's pieces
        if ((rc = encode_map(&ma.b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, ws + L.xp, d, st, b,
                             CU_TENSOR_MAP_SWIZZLE_128B)))
            return rc;
    }
    BMaps mb{};
    if ((rc = tiled ? tiles_map(&mb.a0, pl.w2_tiles + e * codes, H, I, 1)
                    : packed_map(&mb.a0, pl.w2_packed + e * codes, H, I, 1)))
        return rc;
    {
        const uint64_t d[3] = {uint64_t(I / 2), uint64_t(kBMaxN), uint64_t(L.U)};
        const uint64_t st[2] = {uint64_t(I / 2), uint64_t(kBMaxN) * uint64_t(I / 2)};
        const uint32_t b[3] = {128, uint32_t(kBPieces), 1};
        if ((rc = encode_map(&mb.b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, ws + L.act_p, d, st, b,
                             CU_TENSOR_MAP_SWIZZLE_128B)))
            return rc;
    }
    prof_begin(K3_PROF_TOPK, s);
    rc = launch_mv_prep(x, xdt, int(M), H, ws + L.xp, ws + L.sfb, cnt, int(L.keysA + L.keysB), status, s);
    prof_end(K3_PROF_TOPK, s);
    if (rc) return rc;

    BArgs ta{};
    ta.K = H;
    ta.rows = I;
    ta.C = L.CA;
    ta.status = status;
    ta.part = reinterpret_cast<float*>(ws + L.partA);
    ta.cnt = cnt;
    ta.maxseg = L.CA;
    ta.sfa0 = pl.w1_scales_tc + e * sfA;
    ta.sfa1 = pl.w3_scales_tc + e * sfA;
    ta.tiled = tiled ? 1 : 0;
    ta.sf_slot = int64_t(sfA);
    ta.sfb = ws + L.sfb;
    ta.act_p = ws + L.act_p;
    ta.act_sf = ws + L.act_sf;
    ta.act_kind = p->activation;
    ta.beta = p->situ_beta;
    ta.lbeta = p->situ_linear_beta;
    ta.identity_m = int(M);
    prof_begin(K3_PROF_GATEUP, s);
    rc = launch_bs_gateup(ma, ta, sms, s);
    prof_end(K3_PROF_GATEUP, s);
    if (rc) return rc;

    BArgs tb{};
    tb.K = I;
    tb.rows = H;
    tb.C = L.CB;
    tb.status = status;
    tb.part = reinterpret_cast<float*>(ws + L.partB);
    tb.cnt = cnt + L.keysA;
    tb.maxseg = L.CB;
    tb.sfa0 = pl.w2_scales_tc + e * sfB;
    tb.tiled = tiled ? 1 : 0;
    tb.sf_slot = int64_t(sfB);
    tb.sfb = ws + L.act_sf;
    tb.y_pair = static_cast<float*>(y);
    tb.y_bf16 = ydt == K3_BF16 ? 1 : 0;
    tb.identity_m = int(M);
    prof_begin(K3_PROF_DOWN, s);
    rc = launch_bs_down(mb, tb, sms, s);
    prof_end(K3_PROF_DOWN, s);
    return rc;
}

// Decode experts given routing; `logits` non-null also runs the top-k inside prep.
// xr (width Hr, dtype xrdt): a separate router input (latent MoE); null routes on x.
int decode_impl(const k3_moe_params* p, const void* x, int xdt, int64_t M,
                const uint16_t* gate_w, const float* bias, int32_t* idx, float* w, void* y,
                int ydt, uint8_t* ws, const DecodeLayout& L, cudaStream_t s, const void* xr = nullptr,
                int xrdt = K3_F32, int64_t Hr = 0) {
    int rc = configure_smem();
    if (rc) return rc;
    Plan* plan = reinterpret_cast<Plan*>(ws + L.plan);
    __half* xq_hi = reinterpret_cast<__half*>(ws + L.xq_hi);
    __half* xq_lo = reinterpret_cast<__half*>(ws + L.xq_lo);
    float* xq_ts = reinterpret_cast<float*>(ws + L.xq_ts);
    float* logits = reinterpret_cast<float*>(ws + L.logits);
    const bool x_hilo = (xdt == K3_F32);
    PlanArgs pl{};
    pl.bias = bias;
    pl.E = int(p->num_experts);
    pl.k = p->top_k;
    pl.renorm = p->renormalize;
    pl.scale = p->routed_scaling_factor;
    pl.idx = idx;
    pl.w = w;
    pl.has_shared = p->has_shared;
    pl.plan = plan;
    pl.cntA = reinterpret_cast<unsigned*>(ws + L.cntA);
    pl.cntB = reinterpret_cast<unsigned*>(ws + L.cntB);
    pl.n_cntA = L.bs ? L.U * (L.I / kBRows) : L.tma ? L.U * (L.I / 64) : L.U * (L.I / 32);
    pl.n_cntB = L.bs ? L.U * (L.H / kBRows) : L.tma ? L.H / kTRows : L.H / kItemRows;
    pl.M = int(M);
    const int sms = num_sms();

    if (L.tma && gate_w) {
        // one launch: router logits + x conversion + (last CTA) top-k and plan
        RouteArgs ra{};
        ra.x = xr ? xr : x;
        ra.x_dtype = xr ? xrdt : xdt;
        ra.M = int(M);
        ra.H = xr ? Hr : L.H;
        ra.xe = xr ? x : nullptr;
        ra.xe_dtype = xdt;
        ra.He = L.H;
        ra.W = gate_w;
        ra.E = L.E;
        ra.logit_part = reinterpret_cast<float*>(ws + L.logit_part);
        ra.logits = logits;
        pl.keys = reinterpret_cast<uint32_t*>(ws + L.route_keys);
        pl.scores = reinterpret_cast<float*>(ws + L.route_scores);
        ra.done = reinterpret_cast<unsigned*>(ws + L.route_done);
        ra.xq_hi = xq_hi;
        ra.xq_lo = x_hilo ? xq_lo : nullptr;
        ra.xq_ts = xq_ts;
        ra.xp = L.bs ? ws + L.xq_hi : nullptr;
        ra.xsf = L.bs ? ws + L.xq_ts : nullptr;
        ra.plan_args = pl;
        ra.plan = plan;
        if (int rc2 = cuda_check(cudaMemsetAsync(ra.done, 0, sizeof(unsigned) * (2 + (L.E + 15) / 16), s),
                                 "route counters"))
            return rc2;
        prof_begin(K3_PROF_ROUTER, s);
        rc = launch_route_fused(ra, L.KQ, s);
        prof_end(K3_PROF_ROUTER, s);
        if (rc) return rc;
        if (L.bs) return decode_bs(p, L, ws, int(M), y, ydt, sms, s);
        return decode_tma(p, L, ws, x_hilo, y, ydt, sms, s);
    }
    if (gate_w) {
        if (int rc2 = launch_router_logits(x, xdt, int(M), L.H, gate_w, L.E, logits, s)) return rc2;
    }
    PrepArgs pa{};
    pa.mode = 0;
    pa.logits = gate_w ? logits : nullptr;
    pa.pl = pl;
    pa.x = x;
    pa.x_dtype = xdt;
    pa.M = int(M);
    pa.K = L.H;
    pa.xq_hi = xq_hi;
    pa.xq_lo = x_hilo ? xq_lo : nullptr;
    pa.xq_ts = xq_ts;
    pa.blocked = L.tma ? 1 : 0;
    pa.xp = L.bs ? ws + L.xq_hi : nullptr;
    pa.xsf = L.bs ? ws + L.xq_ts : nullptr;
    prof_begin(K3_PROF_TOPK, s);
    const int prep_ctas = L.bs ? int((M * (L.H / 32) + 7) / 8) : L.tma ? int((L.H + 511) / 512) : int(M);
    prep_kernel<<<1 + prep_ctas, 256, 0, s>>>(pa);
    prof_end(K3_PROF_TOPK, s);
    K3_CHECK_LAUNCH("prep_kernel");
    if (L.bs) return decode_bs(p, L, ws, int(M), y, ydt, sms, s);

    if (L.tma) return decode_tma(p, L, ws, x_hilo, y, ydt, sms, s);
    GemvArgs ga{};
    ga.plan = plan;
    ga.table = p->experts;
    ga.K = L.H;
    ga.rows = L.I;
    ga.C = L.CA;
    ga.hilo = x_hilo ? 1 : 0;
    ga.bh = xq_hi;
    ga.bl = xq_lo;
    ga.bts = xq_ts;
    ga.part = reinterpret_cast<float*>(ws + L.partA);
    ga.cnt = reinterpret_cast<unsigned*>(ws + L.cntA);
    ga.act_hi = reinterpret_cast<__half*>(ws + L.act_hi);
    ga.act_lo = reinterpret_cast<__half*>(ws + L.act_lo);
    ga.act_ts = reinterpret_cast<float*>(ws + L.act_ts);
    ga.act_kind = p->activation;
    ga.beta = p->situ_beta;
    ga.lbeta = p->situ_linear_beta;
    prof_begin(K3_PROF_GATEUP, s);
    if (x_hilo)
        gemv_kernel<true, false, true><<<sms, kWarps * 32, smem_bytes_for<true>(), s>>>(ga);
    else
        gemv_kernel<true, false, false><<<sms, kWarps * 32, smem_bytes_for<false>(), s>>>(ga);
    prof_end(K3_PROF_GATEUP, s);
    K3_CHECK_LAUNCH("gemv_kernel<gate/up>");

    GemvArgs gb{};
    gb.plan = plan;
    gb.table = p->experts;
    gb.K = L.I;
    gb.rows = L.H;
    gb.C = L.CB;
    gb.hilo = 1;
    gb.bh = ga.act_hi;
    gb.bl = ga.act_lo;
    gb.bts = ga.act_ts;
    gb.part = reinterpret_cast<float*>(ws + L.partB);
    gb.cnt = reinterpret_cast<unsigned*>(ws + L.cntB);
    gb.Pmax = int(L.P);
    gb.y = y;
    gb.y_dtype = ydt;
    prof_begin(K3_PROF_DOWN, s);
    gemv_kernel<false, true, true><<<sms, kWarps * 32, smem_bytes_for<true>(), s>>>(gb);
    prof_end(K3_PROF_DOWN, s);
    K3_CHECK_LAUNCH("gemv_kernel<down>");
    return K3_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

// Matvec pieces (used by k3_capi.cu's k3_mxfp4_matvec fast path).
struct MatvecLayout {
    int C;
    bool tma;
    size_t plan, xq_hi, xq_lo, xq_ts, part, cnt, total;
};

MatvecLayout matvec_layout(int64_t M, int64_t K, int64_t N, int sms) {
    MatvecLayout L{};
    const int64_t Mc = std::min<int64_t>(M, kMaxTok);
    L.tma = (K % kTStageK == 0) && (N % kTRows == 0);
    L.C = L.tma ? choose_split_tma(N / kTRows, K, sms)
                : choose_split(N / kItemRows, K, int64_t(sms) * kWarps * 4);
    const int64_t xrows = L.tma ? kMaxTok : Mc;
    size_t off = 0;
    L.plan = carve(off, sizeof(Plan));
    L.xq_hi = carve(off, sizeof(__half) * xrows * K);
    L.xq_lo = carve(off, sizeof(__half) * xrows * K);
    L.xq_ts = carve(off, sizeof(float) * kMaxTok * (K / 512 > 0 ? K / 512 : 1));
    L.part = carve(off, L.tma ? sizeof(float) * (N / kTRows) * L.C * kMaxTok * kTRows
                              : sizeof(float) * L.C * Mc * N);
    L.cnt = carve(off, sizeof(unsigned) * (N / (L.tma ? kTRows : kItemRows)));
    L.total = off;
    return L;
}

bool matvec_fast_ok(int64_t K, int64_t N, const void* x, const uint8_t* packed,
                    const uint8_t* scales) {
    return K % 128 == 0 && N % kItemRows == 0 && aligned16(packed) &&
           (reinterpret_cast<uintptr_t>(scales) & 3) == 0 && x != nullptr;
}

int matvec_fast(const void* x, int xdt, int64_t M, int64_t K, const uint8_t* packed,
                const uint8_t* scales, int64_t N, void* out, int odt, uint8_t* ws,
                cudaStream_t s) {
    int rc = configure_smem();
    if (rc) return rc;
    const int sms = num_sms();
    const MatvecLayout L = matvec_layout(M, K, N, sms);
    const size_t esz = (xdt == K3_BF16 || xdt == K3_F16) ? 2 : 4;
    const size_t osz = (odt == K3_BF16 || odt == K3_F16) ? 2 : 4;
    const bool hilo = (xdt == K3_F32);
    for (int64_t m0 = 0; m0 < M; m0 += kMaxTok) {
        const int Mc = int(std::min<int64_t>(kMaxTok, M - m0));
        PrepArgs pa{};
        pa.mode = 1;
        pa.pl.plan = reinterpret_cast<Plan*>(ws + L.plan);
        pa.pl.cntB = reinterpret_cast<unsigned*>(ws + L.cnt);
        pa.pl.n_cntB = N / kItemRows;
        pa.pl.M = Mc;
        pa.x = static_cast<const uint8_t*>(x) + size_t(m0) * K * esz;
        pa.x_dtype = xdt;
        pa.M = Mc;
        pa.K = K;
        pa.xq_hi = reinterpret_cast<__half*>(ws + L.xq_hi);
        pa.xq_lo = hilo ? reinterpret_cast<__half*>(ws + L.xq_lo) : nullptr;
        pa.xq_ts = reinterpret_cast<float*>(ws + L.xq_ts);
        pa.blocked = L.tma ? 1 : 0;
        if (L.tma) pa.pl.n_cntB = N / kTRows;
        prof_begin(K3_PROF_TOPK, s);
        prep_kernel<<<1 + (L.tma ? int(K / 512) : Mc), 256, 0, s>>>(pa);
        prof_end(K3_PROF_TOPK, s);
        K3_CHECK_LAUNCH("prep_kernel(matvec)");
        if (L.tma) {
            TMaps mm{};
            if (int rc2 = pool_maps(&mm.wA, &mm.sA, packed, scales, N, K, 1, kTRows)) return rc2;
            if (int rc2 = blocked_map(&mm.bh, pa.xq_hi, kMaxTok, K)) return rc2;
            if (hilo)
                if (int rc2 = blocked_map(&mm.bl, reinterpret_cast<__half*>(ws + L.xq_lo), kMaxTok, K)) return rc2;
            TArgs ta{};
            ta.plan = pa.pl.plan;
            ta.matvec = 1;
            ta.K = K;
            ta.rows = N;
            ta.C = L.C;
            ta.part = reinterpret_cast<float*>(ws + L.part);
            ta.cnt = pa.pl.cntB;
            ta.maxseg = L.C;
            ta.status = &pa.pl.plan->status;
            ta.bts_tok = pa.xq_ts;
            ta.y = static_cast<uint8_t*>(out) + size_t(m0) * N * osz;
            ta.y_dtype = odt;
            prof_begin(K3_PROF_MATVEC, s);
            const int rc2 = launch_tma_proj(mm, ta, hilo, false, sms, s);
            prof_end(K3_PROF_MATVEC, s);
            if (rc2) return rc2;
            continue;
        }
        GemvArgs g{};
        g.plan = pa.pl.plan;
        g.mat_packed = packed;
        g.mat_scales = scales;
        g.K = K;
        g.rows = N;
        g.C = L.C;
        g.hilo = hilo ? 1 : 0;
        g.bh = pa.xq_hi;
        g.bl = reinterpret_cast<__half*>(ws + L.xq_lo);
        g.bts = pa.xq_ts;
        g.part = reinterpret_cast<float*>(ws + L.part);
        g.cnt = pa.pl.cntB;
        g.Pmax = Mc;
        g.y = static_cast<uint8_t*>(out) + size_t(m0) * N * osz;
        g.y_dtype = odt;
        prof_begin(K3_PROF_MATVEC, s);
        if (hilo)
            gemv_kernel<false, false, true><<<sms, kWarps * 32, smem_bytes_for<true>(), s>>>(g);
        else
            gemv_kernel<false, false, false><<<sms, kWarps * 32, smem_bytes_for<false>(), s>>>(g);
        prof_end(K3_PROF_MATVEC, s);
        K3_CHECK_LAUNCH("gemv_kernel<matvec>");
    }
    return K3_OK;
}

size_t matvec_fast_workspace(int64_t M, int64_t K, int64_t N) {
    return matvec_layout(M, K, N, num_sms()).total;
}

}  // namespace k3

using namespace k3;

// ================================================================ C ABI

// Above this many bf16 tokens the router logits run as a tensor-core GEMM.
constexpr int64_t kRouteGemmMinTokens = 64;

extern "C" K3_API size_t k3_moe_route_workspace(int64_t M, int64_t E) {
    return align_up(sizeof(float) * size_t(std::max<int64_t>(M, 1)) * size_t(std::max<int64_t>(E, 1)), 256) + 256;
}

extern "C" K3_API int k3_moe_route(const void* x, int x_dtype, int64_t M, int64_t H,
                                   const uint16_t* gate_w_bf16, const float* bias, int64_t E,
                                   int top_k, int renormalize, float routed_scaling_factor,
                                   int32_t* idx_out, float* weight_out, float* raw_out,
                                   float* corrected_out, void* workspace, size_t workspace_bytes,
                                   void* stream) {
    if (!x || !gate_w_bf16 || !idx_out || !weight_out) return fail(K3_ERR_INVALID, "k3_moe_route: NULL tensor");
    if (x_dtype != K3_F32 && x_dtype != K3_BF16) return fail(K3_ERR_INVALID, "k3_moe_route: x must be f32 or bf16");
    if (M < 1 || H < 8 || H % 8) return fail(K3_ERR_INVALID, "k3_moe_route: need M >= 1 and H % 8 == 0");
    if (E < 1 || E > kMaxExperts) return fail(K3_ERR_UNSUPPORTED, "k3_moe_route: E must be 1..1024");
    if (top_k < 1 || top_k > 32 || top_k > E) return fail(K3_ERR_UNSUPPORTED, "k3_moe_route: top_k must be 1..min(32, E)");
    if (!aligned16(x) || !aligned16(gate_w_bf16)) return fail(K3_ERR_INVALID, "k3_moe_route: x and gate_w must be 16-byte aligned");
    const size_t need = k3_moe_route_workspace(M, E);
    if (int rc = check_ws(workspace, workspace_bytes, need)) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float* logits = static_cast<float*>(workspace);
    int* status = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + need - 256);
    const size_t esz = x_dtype == K3_BF16 ? 2 : 4;
    if (int rc = cuda_check(cudaMemsetAsync(status, 0, sizeof(int), s), "cudaMemsetAsync")) return rc;
    if (M > kRouteGemmMinTokens && router_gemm_ok(x_dtype, H, x, gate_w_bf16)) {
        prof_begin(K3_PROF_ROUTER, s);
        const int rc = launch_router_gemm(x, M, H, gate_w_bf16, E, logits, status, s);
        prof_end(K3_PROF_ROUTER, s);
        if (rc) return rc;
    } else {
        for (int64_t m0 = 0; m0 < M; m0 += kMaxTok) {
            const int Mc = int(std::min<int64_t>(kMaxTok, M - m0));
            if (int rc = launch_router_logits(static_cast<const uint8_t*>(x) + size_t(m0) * H * esz,
                                              x_dtype, Mc, H, gate_w_bf16, E, logits + m0 * E, s))
                return rc;
        }
    }
    prof_begin(K3_PROF_TOPK, s);
    topk_kernel<<<int((M + 7) / 8), 256, 0, s>>>(logits, int(M), int(E), bias, top_k, renormalize,
                                                 routed_scaling_factor, idx_out, weight_out,
                                                 raw_out, corrected_out, status);
    prof_end(K3_PROF_TOPK, s);
    K3_CHECK_LAUNCH("topk_kernel");
    return K3_OK;
}

extern "C" K3_API size_t k3_moe_decode_workspace(const k3_moe_params* p, int64_t M) {
    if (check_moe_params(p, M) != K3_OK) return 0;
    return decode_layout(*p, M, num_sms()).total;
}

extern "C" K3_API int k3_moe_decode(const k3_moe_params* p, const void* x, int x_dtype, int64_t M,
                                    const uint16_t* gate_w_bf16, const float* bias, void* y_out,
                                    int y_dtype, int32_t* idx_out, float* weight_out,
                                    void* workspace, size_t workspace_bytes, void* stream) {
    if (int rc = check_moe_params(p, M)) return rc;
    if (!x || !gate_w_bf16 || !y_out) return fail(K3_ERR_INVALID, "k3_moe_decode: NULL tensor");
    if (x_dtype != K3_F32 && x_dtype != K3_BF16) return fail(K3_ERR_INVALID, "k3_moe_decode: x must be f32 or bf16");
    if (y_dtype != K3_F32 && y_dtype != K3_BF16) return fail(K3_ERR_INVALID, "k3_moe_decode: y must be f32 or bf16");
    if (!aligned16(x) || !aligned16(gate_w_bf16)) return fail(K3_ERR_INVALID, "k3_moe_decode: x and gate_w must be 16-byte aligned");
    const DecodeLayout L = decode_layout(*p, M, num_sms());
    if (int rc = check_ws(workspace, workspace_bytes, L.total)) return rc;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int32_t* idx = idx_out ? idx_out : reinterpret_cast<int32_t*>(ws + L.route_idx);
    float* w = weight_out ? weight_out : reinterpret_cast<float*>(ws + L.route_w);
    return decode_impl(p, x, x_dtype, M, gate_w_bf16, bias, idx, w, y_out, y_dtype, ws, L, s);
}

extern "C" K3_API size_t k3_moe_decode_latent_workspace(const k3_moe_params* p, int64_t M, int64_t H_router) {
    if (check_moe_params(p, M) != K3_OK || H_router < 512) return 0;
    return decode_layout(*p, M, num_sms(), H_router).total;
}

extern "C" K3_API int k3_moe_decode_latent(const k3_moe_params* p, const void* x_router, int xr_dtype,
                                           int64_t H_router, const void* x_expert, int xe_dtype, int64_t M,
                                           const uint16_t* gate_w_bf16, const float* bias, void* y_out,
                                           int y_dtype, int32_t* idx_out, float* weight_out, float* logits_out,
                                           void* workspace, size_t workspace_bytes, void* stream) {
    if (int rc = check_moe_params(p, M)) return rc;
    if (!x_router || !x_expert || !gate_w_bf16 || !y_out)
        return fail(K3_ERR_INVALID, "k3_moe_decode_latent: NULL tensor");
    if (xr_dtype != K3_F32 && xr_dtype != K3_BF16) return fail(K3_ERR_INVALID, "k3_moe_decode_latent: x_router must be f32 or bf16");
    if (xe_dtype != K3_F32 && xe_dtype != K3_BF16) return fail(K3_ERR_INVALID, "k3_moe_decode_latent: x_expert must be f32 or bf16");
    if (y_dtype != K3_F32 && y_dtype != K3_BF16) return fail(K3_ERR_INVALID, "k3_moe_decode_latent: y must be f32 or bf16");
    if (H_router < 512 || H_router % 512)
        return fail(K3_ERR_UNSUPPORTED, "k3_moe_decode_latent: the router width must be a multiple of 512");
    if (!pool_bs(*p))
        return fail(K3_ERR_UNSUPPORTED, "k3_moe_decode_latent needs the block-scaled expert pool (re-laid scales)");
    if (!aligned16(x_router) || !aligned16(gate_w_bf16))
        return fail(K3_ERR_INVALID, "k3_moe_decode_latent: x_router and gate_w must be 16-byte aligned");
    const DecodeLayout L = decode_layout(*p, M, num_sms(), H_router);
    if (int rc = check_ws(workspace, workspace_bytes, L.total)) return rc;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int32_t* idx = idx_out ? idx_out : reinterpret_cast<int32_t*>(ws + L.route_idx);
    float* w = weight_out ? weight_out : reinterpret_cast<float*>(ws + L.route_w);
    if (int rc = decode_impl(p, x_expert, xe_dtype, M, gate_w_bf16, bias, idx, w, y_out, y_dtype, ws, L, s, x_router,
                             xr_dtype, H_router))
        return rc;
    if (logits_out)
        return cuda_check(cudaMemcpyAsync(logits_out, ws + L.logits, sizeof(float) * M * p->num_experts,
                                          cudaMemcpyDeviceToDevice, s),
                          "cudaMemcpyAsync(logits)");
    return K3_OK;
}

extern "C" K3_API int k3_moe_experts_decode(const k3_moe_params* p, const void* x, int x_dtype,
                                            int64_t M, const int32_t* idx, const float* w,
                                            void* y_out, int y_dtype, void* workspace,
                                            size_t workspace_bytes, void* stream) {
    if (int rc = check_moe_params(p, M)) return rc;
    if (!x || !idx || !w || !y_out) return fail(K3_ERR_INVALID, "k3_moe_experts_decode: NULL tensor");
    if (x_dtype != K3_F32 && x_dtype != K3_BF16) return fail(K3_ERR_INVALID, "k3_moe_experts_decode: x must be f32 or bf16");
    if (y_dtype != K3_F32 && y_dtype != K3_BF16) return fail(K3_ERR_INVALID, "k3_moe_experts_decode: y must be f32 or bf16");
    const DecodeLayout L = decode_layout(*p, M, num_sms());
    if (int rc = check_ws(workspace, workspace_bytes, L.total)) return rc;
    return decode_impl(p, x, x_dtype, M, nullptr, nullptr, const_cast<int32_t*>(idx),
                       const_cast<float*>(w), y_out, y_dtype, static_cast<uint8_t*>(workspace), L,
                       static_cast<cudaStream_t>(stream));
}

extern "C" K3_API size_t k3_moe_expert_forward_workspace(const k3_moe_params* p, int64_t M) {
    if (!p || M < 1 || M > kMaxTok || p->hidden <= 0 || p->inter <= 0) return 0;
    return ffn_layout(*p, M, num_sms()).total;
}

extern "C" K3_API int k3_moe_expert_forward(const k3_moe_params* p, const void* x, int x_dtype, int64_t M,
                                            int64_t expert, void* y_out, int y_dtype, void* workspace,
                                            size_t workspace_bytes, void* stream) {
    if (!p) return fail(K3_ERR_INVALID, "k3_moe_expert_forward: params is NULL");
    if (M < 1 || M > kMaxTok) return fail(K3_ERR_UNSUPPORTED, "k3_moe_expert_forward takes 1..8 tokens, got M=" + std::to_string(M));
    if (!x || !y_out) return fail(K3_ERR_INVALID, "k3_moe_expert_forward: NULL tensor");
    if (x_dtype != K3_F32 && x_dtype != K3_BF16) return fail(K3_ERR_INVALID, "k3_moe_expert_forward: x must be f32 or bf16");
    if (y_dtype != K3_F32 && y_dtype != K3_BF16) return fail(K3_ERR_INVALID, "k3_moe_expert_forward: y must be f32 or bf16");
    if (p->activation != K3_ACT_SILU && p->activation != K3_ACT_SITU) return fail(K3_ERR_INVALID, "unknown activation");
    if (p->hidden % 512 || p->inter % 512)
        return fail(K3_ERR_UNSUPPORTED, "k3_moe_expert_forward: hidden and inter must be multiples of 512");
    if (!pool_bs(*p)) return fail(K3_ERR_UNSUPPORTED, "k3_moe_expert_forward needs the block-scaled expert pool");
    if (expert < 0 || expert >= p->pool->num_slots)
        return fail(K3_ERR_INVALID, "k3_moe_expert_forward: expert " + std::to_string(expert) + " is not a pool slot");
    const FfnLayout L = ffn_layout(*p, M, num_sms());
    if (int rc = check_ws(workspace, workspace_bytes, L.total)) return rc;
    return expert_ffn_bs(p, x, x_dtype, M, expert, y_out, y_dtype, static_cast<uint8_t*>(workspace), L,
                         static_cast<cudaStream_t>(stream));
}

// ------------------------------------------------------------ pairs (expert parallel)

namespace k3 {

// Router logits of any number of tokens on the CUDA cores (fp32 fma, 8 tokens a launch):
// the prefill path's route for f32 activations.
int launch_router_logits_rows(const void* x, int xdt, int64_t M, int64_t H, const uint16_t* W,
                              int64_t E, float* logits, cudaStream_t s) {
    const size_t esz = xdt == K3_BF16 ? 2 : 4;
    for (int64_t m0 = 0; m0 < M; m0 += kMaxTok) {
        const int Mc = int(std::min<int64_t>(kMaxTok, M - m0));
        if (int rc = launch_router_logits(static_cast<const uint8_t*>(x) + size_t(m0) * H * esz, xdt, Mc,
                                          H, W, E, logits + m0 * E, s))
            return rc;
    }
    return K3_OK;
}

// Sigmoid top-k of every row of logits [M][E] (one warp per row).
int launch_topk_rows(const float* logits, int64_t M, int64_t E, const float* bias, int k, int renorm,
                     float scale, int32_t* idx, float* w, int* status, cudaStream_t s) {
    topk_kernel<<<int((M + 7) / 8), 256, 0, s>>>(logits, int(M), int(E), bias, k, renorm, scale, idx, w,
                                                 nullptr, nullptr, status);
    K3_CHECK_LAUNCH("topk_kernel");
    return K3_OK;
}

// Workspace of a pairs call: T token rows, up to n_in candidate pairs.
DecodeLayout pairs_layout(const k3_moe_params& p, int64_t T, int64_t n_in, int sms) {
    DecodeLayout L{};
    L.M = T;
    L.H = p.hidden;
    L.I = p.inter;
    L.E = p.num_experts;
    L.U = std::min<int64_t>(n_in, kMaxActive);
    L.P = std::min<int64_t>(n_in, kMaxPairs);
    L.tma = L.bs = true;
    L.CA = choose_split_bs(L.U * (L.I / kBRows), L.H, sms);
    L.CB = choose_split_bs(L.U * (L.H / kBRows), L.I, sms);
    size_t off = 0;
    L.plan = carve(off, sizeof(Plan));
    L.xq_hi = carve(off, size_t(kBPieces) * T * (L.H / 2));
    L.xq_ts = carve(off, size_t(kBPieces) * T * (L.H / 32));
    L.act_hi = carve(off, size_t(L.U) * kBMaxN * (L.I / 2));
    L.act_ts = carve(off, size_t(L.U) * (L.I / 128) * kBChunk);
    L.partA = carve(off, sizeof(float) * L.U * (L.I / kBRows) * L.CA * 2 * kMaxTok * kBRows);
    L.cntA = carve(off, sizeof(unsigned) * L.U * (L.I / kBRows));
    L.partB = carve(off, sizeof(float) * L.U * (L.H / kBRows) * L.CB * kMaxTok * kBRows);
    L.cntB = carve(off, sizeof(unsigned) * L.U * (L.H / kBRows));
    L.y_pair = carve(off, sizeof(float) * L.P * L.H);
    L.total = off;
    return L;
}

}  // namespace k3

namespace k3 {

size_t pairs_decode_workspace(const k3_moe_params& p, int64_t T, int64_t n_in) {
    return pairs_layout(p, T, n_in, num_sms()).total;
}

// The decode kernels over the candidates of `cand` (explicit pairs or a routing result,
// cand.n_in of them): plan, x pieces, gate/up, down, ordered combine.
int pairs_decode_run(const k3_moe_params* p, const void* x, int x_dtype, int64_t T, const PairsArgs& cand,
                     void* y_out, int y_dtype, void* workspace, size_t workspace_bytes, cudaStream_t s) {
    if (cand.n_in < 1 || cand.n_in > kMaxPairCandidates)
        return fail(K3_ERR_UNSUPPORTED, "pairs decode: 1..1024 candidate pairs");
    if (!p->pool || !pool_bs(*p))
        return fail(K3_ERR_UNSUPPORTED, "pairs decode needs a block-scaled expert pool "
                                        "(re-laid scales and tiles; H, I multiples of 512)");
    const int sms = num_sms();
    const DecodeLayout L = pairs_layout(*p, T, cand.n_in, sms);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    if (int rc = check_ws(workspace, workspace_bytes, L.total)) return rc;
    if (int rc = configure_smem()) return rc;
    PairsArgs pa = cand;
    pa.num_slots = int(p->pool->num_slots);
    pa.T = int(T);
    pa.plan = reinterpret_cast<Plan*>(ws + L.plan);
    pa.cntA = reinterpret_cast<unsigned*>(ws + L.cntA);
    pa.n_cntA = L.U * (L.I / kBRows);
    pa.cntB = reinterpret_cast<unsigned*>(ws + L.cntB);
    pa.n_cntB = L.U * (L.H / kBRows);
    prof_begin(K3_PROF_TOPK, s);
    const ConvertArgs conv{x, x_dtype, T, L.H, ws + L.xq_hi, ws + L.xq_ts};
    if (int rc = launch_plan_from_pairs(pa, conv, s)) return rc;
    prof_end(K3_PROF_TOPK, s);
    return decode_bs(p, L, ws, int(T), y_out, y_dtype, sms, s);
}

}  // namespace k3

extern "C" K3_API size_t k3_moe_pairs_workspace(const k3_moe_params* p, int64_t T, int64_t n_pairs) {
    using namespace k3;
    if (!p || T < 1 || n_pairs < 1) return 0;
    return pairs_decode_workspace(*p, T, n_pairs);
}

extern "C" K3_API int k3_moe_pairs_decode(const k3_moe_params* p, const void* x, int x_dtype, int64_t T,
                                          const int32_t* pair_slot, const int32_t* pair_tok,
                                          const float* pair_w, int64_t n_pairs, void* y_out, int y_dtype,
                                          void* workspace, size_t workspace_bytes, void* stream) {
    using namespace k3;
    if (!p) return fail(K3_ERR_INVALID, "k3_moe_pairs_decode: params is NULL");
    if (!x || !pair_slot || !pair_tok || !pair_w || !y_out)
        return fail(K3_ERR_INVALID, "k3_moe_pairs_decode: NULL tensor");
    if (x_dtype != K3_F32 && x_dtype != K3_BF16) return fail(K3_ERR_INVALID, "x dtype must be f32 or bf16");
    if (y_dtype != K3_F32 && y_dtype != K3_BF16) return fail(K3_ERR_INVALID, "y dtype must be f32 or bf16");
    if (T < 1) return fail(K3_ERR_INVALID, "k3_moe_pairs_decode: T must be >= 1");
    if (n_pairs < 1 || n_pairs > kMaxPairCandidates)
        return fail(K3_ERR_UNSUPPORTED, "k3_moe_pairs_decode: 1..1024 candidate pairs");
    PairsArgs cand{};
    cand.slot = pair_slot;
    cand.tok = pair_tok;
    cand.w = pair_w;
    cand.n_in = int(n_pairs);
    return pairs_decode_run(p, x, x_dtype, T, cand, y_out, y_dtype, workspace, workspace_bytes,
                            static_cast<cudaStream_t>(stream));
}
