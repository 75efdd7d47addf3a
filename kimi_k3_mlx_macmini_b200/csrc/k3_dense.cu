// Dense bf16 matvecs of the Kimi-K3 MoE layer around the MXFP4 experts, for decode
// (M <= 8 tokens): the latent projections, the bf16 shared expert and the streamed
// lm_head argmax.
//
//   k3_dense_matvec, combine SUM:    out = sum over segments s of  X_s  W_s^T
//   k3_dense_matvec, combine ACT:    out = act(X W_gate^T, X W_up^T)
//   k3_lm_head_argmax:               argmax_n (h W^T)[n]
//
// W is bf16 [N][K] row-major (the checkpoint layout), X is f32 or bf16. A segment may
// RMS-normalise its input first (x -> norm_w * x * rsqrt(mean(x^2) + eps), the
// reference's `ops.rmsnorm`, air_llm/models/kimi_k3/ops.py:11-14), or read it as
// act(gate, up) from a [gate | up] row (the bf16 shared expert's activation feeding its
// down projection, moe.py:105-107). Products and sums are
// fp32, as in the reference, which computes these in fp32 on bf16 weights
// (air_llm/models/kimi_k3/moe.py:105-107, 116, 128-130; model.py:111-133).
//
// The matvecs are HBM-bound: every weight byte is read once. Work layout:
//
//   * a prep kernel stages each segment's input as fp32 in the order the matvec's lanes
//     read it (MT = M rounded up to 1, 2, 4 or 8; padded tokens and k beyond K are zero),
//     normalised or activated when the segment asks for it;
//   * the matvec kernel runs one CTA per SM. Units are (row block of 64 weight rows,
//     256-k step); a row block's units run over its segments' k in order. CTA b takes
//     the contiguous unit range [U b / G, U (b+1) / G), so every CTA streams the same
//     number of weight bytes. It is a programmatic dependent launch of the prep kernel:
//     its first weight tiles are requested before the prep kernel finishes. A producer
//     warp moves each unit into a 5-stage ring: the
//     64 x 256 weight tile (32 KB) as one TMA box, the 256 x MT input slice as one bulk
//     copy, both landing on the stage's mbarrier. Eight consumer warps own 8 rows of the
//     block each, lane l owns 8 k of the step; the fp32 products run as f32x2 FMAs, two
//     tokens (or, at MT = 1, two k) per instruction;
//   * at the end of a row block a warp reduces its lanes (recursive halving: lane l ends
//     with values 2l, 2l+1 of the warp's 8 x MT partial sums). A row block that lies
//     inside one CTA's range is finished at once. One that straddles CTAs is finished
//     by the last of its CTAs to arrive (a per-block counter): it adds the partial tiles
//     of all its CTAs in CTA order, so results do not depend on timing.
#include <cuda_bf16.h>

#include <algorithm>

#include "k3_async.cuh"
#include "k3_bs.cuh"
#include "k3_tma.cuh"

namespace k3 {

namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int check_ws(void* ws, size_t bytes, size_t need) {
    if (!ws) return fail(K3_ERR_WORKSPACE, "workspace is NULL");
    if (reinterpret_cast<uintptr_t>(ws) % 256) return fail(K3_ERR_WORKSPACE, "workspace must be 256-byte aligned");
    if (bytes < need) return fail(K3_ERR_WORKSPACE, "workspace too small: need " + std::to_string(need) + " bytes");
    return K3_OK;
}

constexpr int kDWarps = 8;                             // consumer warps
constexpr int kDThreads = (kDWarps + 1) * 32;          // + one producer warp
constexpr int kDRowsPerWarp = 8;
constexpr int kDBlockRows = kDWarps * kDRowsPerWarp;   // 64 weight rows per row block
constexpr int kDUnitK = 256;                           // k per unit: 32 lanes x 8
constexpr int kDStages = 5;
constexpr int kDMaxSeg = 2;

// combine modes: the two public ones, and the lm_head's argmax
enum { kCombineSum = K3_DENSE_SUM, kCombineAct = K3_DENSE_ACT, kCombineArgmax = 2 };

struct DenseSeg {
    int64_t K;
    int units;              // ceil(K / kDUnitK)
    const float* xt;        // staged input, [units][256 * MT] floats (see dense_prep_kernel)
};

struct DenseArgs {
    // weight tiles: SUM / ARGMAX one map per segment, box [64 rows][256 k]; ACT the gate
    // and up maps, box [32 rows][256 k]
    CUtensorMap map[kDMaxSeg];
    DenseSeg seg[kDMaxSeg];
    int nseg;
    int64_t N;              // output rows
    int M;
    int combine;
    int act_kind;
    float beta, lbeta;
    void* out;
    int out_dtype;
    int64_t ldo;
    int nblk;               // row blocks
    int ku;                 // units per row block (all segments)
    int64_t U;              // nblk * ku
    float* rec;             // [grid][2][kDBlockRows][MT] partial tiles
    int* cnt;               // [nblk] arrivals per straddling row block
    unsigned long long* key;   // argmax: (ordered value << 32) | ~index
    float* logits;          // argmax: optional [N] fp32 logits
    int* status;            // K3_ERR_TIMEOUT when a bounded wait gave up
};

// One stage: the weight tile [64 rows][256 k] bf16 as TMA writes it (row r at r * 512
// bytes), then the input slice of the unit (256 k x MT floats, laid out by the prep
// kernel so that each warp-wide read is contiguous across lanes).
template <int MT>
struct StageLayout {
    static constexpr int kWBytes = kDBlockRows * kDUnitK * 2;
    static constexpr int kXBytes = kDUnitK * MT * 4;
    static constexpr int kBytes = kWBytes + kXBytes;
};

template <int MT>
constexpr size_t dense_smem_bytes() {
    return size_t(StageLayout<MT>::kBytes) * kDStages + sizeof(float) * kDBlockRows * MT +
           2 * kDStages * sizeof(uint64_t) + 128;
}
static_assert(dense_smem_bytes<8>() <= 227 * 1024, "dense stages exceed shared memory");

// Position of input element (k, m) inside its unit's slice. Lane l of a warp owns k =
// 8 l + j (j < 8) of the unit. MT >= 2: vectors of V = min(MT, 4) tokens, ordered
// [j][token vector][lane][V]; MT == 1: pairs of k, ordered [j / 2][lane][2].
template <int MT>
__host__ __device__ __forceinline__ int xslot(int kk, int m) {
    const int l = kk >> 3, j = kk & 7;
    if constexpr (MT == 1) {
        return ((j >> 1) * 32 + l) * 2 + (j & 1);
    } else {
        constexpr int V = MT < 4 ? MT : 4;
        return ((j * (MT / V) + m / V) * 32 + l) * V + (m % V);
    }
}

// Monotone map of a float onto an unsigned key (larger value -> larger key).
__device__ __forceinline__ uint32_t ordered_key(float v) {
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Named barrier over the 256 consumer threads (the producer warp never joins it).
__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, %0;\n" ::"n"(kDWarps * 32) : "memory"); }

// acc[r][j]: MT >= 2 -> (token 2j, token 2j+1) of row r; MT == 1 -> (even k, odd k).
template <int MT>
struct Acc {
    static constexpr int kPairs = MT >= 2 ? MT / 2 : 1;
    float2 v[kDRowsPerWarp][kPairs];
};

template <int MT>
__device__ __forceinline__ void compute_unit(Acc<MT>& acc, const uint8_t* st, int warp, int lane) {
    using SL = StageLayout<MT>;
    uint4 w[kDRowsPerWarp];
#pragma unroll
    for (int r = 0; r < kDRowsPerWarp; ++r)
        w[r] = *reinterpret_cast<const uint4*>(st + (warp * kDRowsPerWarp + r) * kDUnitK * 2 + lane * 16);
    const float* xs = reinterpret_cast<const float*>(st + SL::kWBytes);
#pragma unroll
    for (int q = 0; q < 4; ++q) {                     // bf16 pair q: k = 2q, 2q+1 of the lane's 8
        if constexpr (MT == 1) {
            const float2 xp = *reinterpret_cast<const float2*>(xs + xslot<1>(8 * lane + 2 * q, 0));
#pragma unroll
            for (int r = 0; r < kDRowsPerWarp; ++r) {
                const uint32_t u = (&w[r].x)[q];
                const float2 wp = make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
                acc.v[r][0] = __ffma2_rn(wp, xp, acc.v[r][0]);
            }
        } else {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int kk = 8 * lane + 2 * q + h;
                float2 xp[MT / 2];
                if constexpr (MT >= 4) {
#pragma unroll
                    for (int g = 0; g < MT / 4; ++g) {
                        const float4 t = *reinterpret_cast<const float4*>(xs + xslot<MT>(kk, 4 * g));
                        xp[2 * g] = make_float2(t.x, t.y);
                        xp[2 * g + 1] = make_float2(t.z, t.w);
                    }
                } else {
                    xp[0] = *reinterpret_cast<const float2*>(xs + xslot<MT>(kk, 0));
                }
#pragma unroll
                for (int r = 0; r < kDRowsPerWarp; ++r) {
                    const uint32_t u = (&w[r].x)[q];
                    const float wv = __uint_as_float(h ? (u & 0xffff0000u) : (u << 16));
                    const float2 wp = make_float2(wv, wv);
#pragma unroll
                    for (int j = 0; j < MT / 2; ++j) acc.v[r][j] = __ffma2_rn(wp, xp[j], acc.v[r][j]);
                }
            }
        }
    }
}

// Sums the warp's 8 x MT partial sums over its 32 lanes and stores them into
// tile[warp*8 + r][m] (row-major [64][MT]).
template <int MT>
__device__ __forceinline__ void reduce_to_tile(Acc<MT>& acc, float* tile, int warp, int lane) {
    constexpr int V = kDRowsPerWarp * MT;
    float v[V];
#pragma unroll
    for (int r = 0; r < kDRowsPerWarp; ++r) {
        if constexpr (MT == 1) {
            v[r] = acc.v[r][0].x + acc.v[r][0].y;
        } else {
#pragma unroll
            for (int j = 0; j < MT / 2; ++j) {
                v[r * MT + 2 * j] = acc.v[r][j].x;
                v[r * MT + 2 * j + 1] = acc.v[r][j].y;
            }
        }
    }
    // recursive halving: at offset o the lanes with bit o set keep the upper half
    int n = V;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        if (n > 1) {
            const bool up = lane & o;
#pragma unroll
            for (int i = 0; i < V / 2; ++i) {
                if (i < n / 2) {
                    const float send = up ? v[i] : v[i + n / 2];
                    const float keep = up ? v[i + n / 2] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
                }
            }
            n >>= 1;
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
        }
    }
    // lane l now holds values [l * V / 32, ...) when V >= 32; with V < 32 the lanes of
    // each group of 32 / V hold value l / (32 / V)
    if constexpr (V >= 32) {
#pragma unroll
        for (int i = 0; i < V / 32; ++i) tile[warp * V + lane * (V / 32) + i] = v[i];
    } else {
        if (lane % (32 / V) == 0) tile[warp * V + lane / (32 / V)] = v[0];
    }
}

// Final combine of row block `blk` from its complete [64][MT] tile (consumer threads).
template <int MT>
__device__ void finish_block(const DenseArgs& a, int blk, const float* tile, unsigned long long* s_best) {
    const int tid = threadIdx.x;
    if (a.combine == kCombineAct) {
        for (int i = tid; i < (kDBlockRows / 2) * MT; i += kDWarps * 32) {
            const int m = i / (kDBlockRows / 2), r = i - m * (kDBlockRows / 2);
            const int64_t n = int64_t(blk) * (kDBlockRows / 2) + r;
            if (m < a.M && n < a.N)
                store_from_f32(a.out, a.out_dtype, m * a.ldo + n,
                               act_value(a.act_kind, tile[r * MT + m], tile[(r + kDBlockRows / 2) * MT + m], a.beta,
                                         a.lbeta));
        }
        return;
    }
    if (a.combine == kCombineArgmax) {
        // one token: the block's 64 logits; warp 0 finds the largest (lowest index on ties)
        if (tid < 32) {
            unsigned long long best = 0;
            for (int r = tid; r < kDBlockRows; r += 32) {
                const int64_t n = int64_t(blk) * kDBlockRows + r;
                if (n >= a.N) continue;
                const float v = tile[r * MT];
                if (a.logits) a.logits[n] = v;
                const unsigned long long k =
                    (static_cast<unsigned long long>(ordered_key(v)) << 32) | (0xffffffffu - uint32_t(n));
                best = k > best ? k : best;
            }
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) {
                const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
                best = other > best ? other : best;
            }
            if (tid == 0 && best > *s_best) *s_best = best;
        }
        return;
    }
    for (int i = tid; i < kDBlockRows * MT; i += kDWarps * 32) {
        const int m = i / kDBlockRows, r = i - m * kDBlockRows;
        const int64_t n = int64_t(blk) * kDBlockRows + r;
        if (m < a.M && n < a.N) store_from_f32(a.out, a.out_dtype, m * a.ldo + n, tile[r * MT + m]);
    }
}

__device__ __forceinline__ int64_t unit_cta(int64_t u, int64_t U, int G) { return ((u + 1) * G - 1) / U; }

template <int MT>
__global__ void __launch_bounds__(kDThreads, 1) dense_matvec_kernel(const __grid_constant__ DenseArgs a) {
    extern __shared__ __align__(1024) uint8_t dsm[];
    using SL = StageLayout<MT>;
    float* tile = reinterpret_cast<float*>(dsm + SL::kBytes * kDStages);
    uint64_t* full = reinterpret_cast<uint64_t*>(dsm + SL::kBytes * kDStages + sizeof(float) * kDBlockRows * MT);
    uint64_t* empty = full + kDStages;
    __shared__ int s_last;
    __shared__ volatile int s_abort;
    __shared__ unsigned long long s_best;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, b = blockIdx.x;
    const int64_t ub = a.U * b / G, ue = a.U * (b + 1) / G;
    if (threadIdx.x == 0) {
        s_best = 0;
        s_abort = 0;
        for (int i = 0; i < kDStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kDWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    __syncthreads();

    if (warp == kDWarps) {
        // ------------------------------------------------------------- producer
        if (lane == 0) {
            const bool act = a.combine == kCombineAct;
            // unit u -> (row block, segment, k step within the segment)
            auto locate = [&](int64_t u, int& blk, int& s, int& kstep) {
                blk = int(u / a.ku);
                kstep = int(u - int64_t(blk) * a.ku);
                s = 0;
                if (a.nseg > 1 && kstep >= a.seg[0].units) {
                    kstep -= a.seg[0].units;
                    s = 1;
                }
            };
            auto issue_w = [&](int64_t u, int st) {
                int blk, s, kstep;
                locate(u, blk, s, kstep);
                uint8_t* dst = dsm + SL::kBytes * st;
                mbar_expect_tx(&full[st], uint32_t(SL::kBytes));
                if (act) {
                    tma_2d(dst, &a.map[0], kstep * kDUnitK, blk * (kDBlockRows / 2), &full[st]);
                    tma_2d(dst + SL::kWBytes / 2, &a.map[1], kstep * kDUnitK, blk * (kDBlockRows / 2), &full[st]);
                } else {
                    tma_2d(dst, &a.map[s], kstep * kDUnitK, blk * kDBlockRows, &full[st]);
                }
            };
            auto issue_x = [&](int64_t u, int st) {
                int blk, s, kstep;
                locate(u, blk, s, kstep);
                bulk_g2s(dsm + SL::kBytes * st + SL::kWBytes, a.seg[s].xt + int64_t(kstep) * kDUnitK * MT,
                         uint32_t(SL::kXBytes), &full[st]);
            };
            // the weights do not depend on the prep kernel: the first stages' tiles are
            // requested before waiting for it (programmatic dependent launch)
            const int64_t pre = ue - ub < kDStages ? ue - ub : kDStages;
            for (int64_t i = 0; i < pre; ++i) issue_w(ub + i, int(i));
            asm volatile("griddepcontrol.wait;\n" ::: "memory");
            for (int64_t i = 0; i < pre; ++i) issue_x(ub + i, int(i));
            int64_t issued = pre;
            for (int64_t u = ub + pre; u < ue; ++u, ++issued) {
                const int j = int(u - ub), st = j % kDStages;
                if (!mbar_wait(&empty[st], ((j / kDStages) & 1) ^ 1, a.status, &s_abort)) {
                    s_abort = 1;
                    break;
                }
                issue_w(u, st);
                issue_x(u, st);
            }
            // copies in flight land before the CTA leaves: only the last kDStages units can
            // still be in flight, and their phases are each stage's latest (an older unit's
            // parity would alias a later phase of the same stage)
            for (int64_t i = issued > kDStages ? issued - kDStages : 0; i < issued; ++i) {
                const int j = int(i);
                if (!mbar_wait(&full[j % kDStages], (j / kDStages) & 1, a.status)) break;
            }
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    asm volatile("griddepcontrol.wait;\n" ::: "memory");   // counters, records, status: after prep
    Acc<MT> acc;
#pragma unroll
    for (int r = 0; r < kDRowsPerWarp; ++r)
#pragma unroll
        for (int j = 0; j < Acc<MT>::kPairs; ++j) acc.v[r][j] = make_float2(0.0f, 0.0f);

    int64_t run_start = ub;
    for (int64_t u = ub; u < ue; ++u) {
        const int j = int(u - ub), st = j % kDStages;
        // after a wait gives up the consumers keep stepping through the units without
        // computing, so that every warp reaches the same named barriers
        if (!s_abort && !mbar_wait(&full[st], (j / kDStages) & 1, a.status, &s_abort)) s_abort = 1;
        if (!s_abort) compute_unit<MT>(acc, dsm + SL::kBytes * st, warp, lane);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);

        const int blk = int(u / a.ku);
        const bool block_end = (u + 1) % a.ku == 0;
        if (!block_end && u + 1 < ue) continue;
        // ---- end of this CTA's run over row block blk
        reduce_to_tile<MT>(acc, tile, warp, lane);
#pragma unroll
        for (int r = 0; r < kDRowsPerWarp; ++r)
#pragma unroll
            for (int q = 0; q < Acc<MT>::kPairs; ++q) acc.v[r][q] = make_float2(0.0f, 0.0f);
        consumers_sync();
        const int64_t blk0 = int64_t(blk) * a.ku;
        const bool whole = run_start == blk0 && block_end;
        if (whole) {
            finish_block<MT>(a, blk, tile, &s_best);
        } else {
            // partial tile: slot 0 when this is the CTA's first run, else slot 1
            const int slot = run_start == ub ? 0 : 1;
            float* mine = a.rec + (int64_t(b) * 2 + slot) * kDBlockRows * MT;
            for (int i = threadIdx.x; i < kDBlockRows * MT; i += kDWarps * 32) mine[i] = tile[i];
            __threadfence();
            consumers_sync();
            const int c_lo = int(unit_cta(blk0, a.U, G)), c_hi = int(unit_cta(blk0 + a.ku - 1, a.U, G));
            if (threadIdx.x == 0) s_last = atomicAdd(&a.cnt[blk], 1) == c_hi - c_lo;
            consumers_sync();
            if (s_last) {
                __threadfence();
                for (int i = threadIdx.x; i < kDBlockRows * MT; i += kDWarps * 32) {
                    float v = 0.0f;
                    for (int c = c_lo; c <= c_hi; ++c) {
                        const int cs = (a.U * c / G) >= blk0 ? 0 : 1;   // c's first run is this block?
                        v += __ldcg(a.rec + (int64_t(c) * 2 + cs) * kDBlockRows * MT + i);
                    }
                    tile[i] = v;
                }
                consumers_sync();
                finish_block<MT>(a, blk, tile, &s_best);
            }
        }
        consumers_sync();
        run_start = u + 1;
    }
    if (a.combine == kCombineArgmax) {
        consumers_sync();
        if (threadIdx.x == 0 && s_best) atomicMax(a.key, s_best);
    }
}

// Stages every segment's input (blockIdx.y = segment, blockIdx.x = token slot < MT) in
// the unit layout of xslot(), RMS-normalised or formed as act(gate, up) when the segment
// asks for it; zeroes the row-block counters, the argmax key and the status word.
struct PrepArgs {
    const void* x[kDMaxSeg];
    int xdt[kDMaxSeg];
    int64_t ldx[kDMaxSeg];
    int64_t K[kDMaxSeg];
    int64_t Kp[kDMaxSeg];
    const float* norm_w[kDMaxSeg];
    float eps[kDMaxSeg];
    int act_in[kDMaxSeg];   // input row = [gate | up]; staged value act(gate, up)
    int act_kind;
    float beta, lbeta;
    float* xt[kDMaxSeg];
    int M, MT;
    int* cnt;
    int nblk;
    unsigned long long* key;
    int* status;
};

constexpr int kDPrepK = 1024;           // k per prep CTA

// grid (k chunks of kDPrepK, token slots MT, segments): one CTA writes one chunk of one
// token. With a norm weight every CTA of the token sums the whole row's squares itself.
template <int MT>
__global__ void __launch_bounds__(256) dense_prep_kernel(const __grid_constant__ PrepArgs p) {
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");   // the matvec may start now
    const int s = blockIdx.z, m = blockIdx.y;
    const int64_t k0 = int64_t(blockIdx.x) * kDPrepK;
    __shared__ float s_red[8];
    __shared__ float s_scale;
    if (s == 0 && m == 0 && blockIdx.x == 0) {
        for (int i = threadIdx.x; i < p.nblk; i += blockDim.x) p.cnt[i] = 0;
        if (threadIdx.x == 0) {
            *p.key = 0ull;
            *p.status = K3_OK;
        }
    }
    const int64_t K = p.K[s];
    if (k0 >= p.Kp[s]) return;
    float* xt = p.xt[s];
    const bool live = m < p.M;
    float scale = 1.0f;
    if (live && p.norm_w[s]) {
        // sixteen loads in flight per thread: one round trip for rows up to 4096 wide
        float ss[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int64_t k = threadIdx.x; k < K; k += 16 * blockDim.x) {
            float q[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int64_t kk = k + i * blockDim.x;
                q[i] = kk < K ? load_as_f32(p.x[s], p.xdt[s], m * p.ldx[s] + kk) : 0.0f;
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) ss[i & 3] = fmaf(q[i], q[i], ss[i & 3]);
        }
        float t = (ss[0] + ss[1]) + (ss[2] + ss[3]);
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = t;
        __syncthreads();
        if (threadIdx.x == 0) {
            float u = 0.0f;
            for (int i = 0; i < int(blockDim.x >> 5); ++i) u += s_red[i];
            s_scale = rsqrtf(u / float(K) + p.eps[s]);
        }
        __syncthreads();
        scale = s_scale;
    }
    float v[kDPrepK / 256];
#pragma unroll
    for (int i = 0; i < kDPrepK / 256; ++i) {
        const int64_t k = k0 + threadIdx.x + 256 * i;
        v[i] = 0.0f;
        if (live && k < K) {
            v[i] = load_as_f32(p.x[s], p.xdt[s], m * p.ldx[s] + k);
            if (p.act_in[s])
                v[i] = act_value(p.act_kind, v[i], load_as_f32(p.x[s], p.xdt[s], m * p.ldx[s] + K + k), p.beta,
                                 p.lbeta);
            else if (p.norm_w[s])
                v[i] = p.norm_w[s][k] * (v[i] * scale);
        }
    }
#pragma unroll
    for (int i = 0; i < kDPrepK / 256; ++i) {
        const int64_t k = k0 + threadIdx.x + 256 * i;
        if (k < p.Kp[s]) {
            const int64_t unit = k / kDUnitK;
            xt[unit * kDUnitK * MT + xslot<MT>(int(k - unit * kDUnitK), m)] = v[i];
        }
    }
}

__global__ void dense_argmax_finish_kernel(const unsigned long long* key, int32_t* idx, float* val) {
    const unsigned long long k = *key;
    *idx = k ? int32_t(0xffffffffu - uint32_t(k & 0xffffffffu)) : -1;
    *val = k ? key_value(uint32_t(k >> 32)) : -INFINITY;
}

int mt_of(int64_t M) { return M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8; }
int64_t units_of(int64_t K) { return (K + kDUnitK - 1) / kDUnitK; }

// Workspace: a 256-byte header (argmax key at 0, status word at 8), the staged inputs,
// the partial tiles and the row-block counters.
constexpr size_t kDKeyOff = 0, kDStatusOff = 8, kDHeader = 256;

struct DenseLayout {
    size_t xt[kDMaxSeg], rec, cnt, total;
};

DenseLayout dense_layout(int64_t M, int64_t nblk, int nseg, const int64_t* K) {
    DenseLayout L{};
    const int MT = mt_of(M);
    size_t off = kDHeader;
    for (int s = 0; s < kDMaxSeg; ++s) {
        L.xt[s] = off;
        if (s < nseg) off += align_up(sizeof(float) * size_t(units_of(K[s])) * kDUnitK * MT, 256);
    }
    L.rec = off;
    off += align_up(sizeof(float) * size_t(num_sms()) * 2 * kDBlockRows * MT, 256);
    L.cnt = off;
    off += align_up(sizeof(int) * size_t(std::max<int64_t>(nblk, 1)), 256);
    L.total = off;
    return L;
}

// Weight matrix W [rows][K] bf16 (row stride ldw elements) as a 2-D tensor map with
// boxes of [box_rows][256 k]; rows and k past the matrix read as zero.
int weight_map(CUtensorMap* m, const uint16_t* w, int64_t rows, int64_t K, int64_t ldw, int box_rows) {
    const uint64_t d[2] = {uint64_t(K), uint64_t(rows)};
    const uint64_t st[1] = {uint64_t(ldw) * 2};
    const uint32_t b[2] = {uint32_t(kDUnitK), uint32_t(box_rows)};
    return encode_map(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, w, d, st, b, CU_TENSOR_MAP_SWIZZLE_NONE);
}

template <int MT>
int launch_dense(const DenseArgs& a, cudaStream_t s) {
    static OncePerContext attr;
    const size_t smem = dense_smem_bytes<MT>();
    if (int rc = attr.run([&] {
            return cuda_check(cudaFuncSetAttribute(dense_matvec_kernel<MT>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
                              "cudaFuncSetAttribute(dense_matvec_kernel)");
        }))
        return rc;
    const int G = int(std::min<int64_t>(num_sms(), a.U));
    // programmatic dependent launch: the matvec starts streaming weights while the prep
    // kernel runs, and waits for it (griddepcontrol.wait) before touching its outputs
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(unsigned(G));
    cfg.blockDim = dim3(kDThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    if (int rc = cuda_check(cudaLaunchKernelEx(&cfg, dense_matvec_kernel<MT>, a), "dense_matvec_kernel")) return rc;
    return K3_OK;
}

template <int MT>
int launch_prep(const PrepArgs& p, int nx, cudaStream_t s) {
    int64_t kp = 0;
    for (int i = 0; i < nx; ++i) kp = std::max(kp, p.Kp[i]);
    dense_prep_kernel<MT><<<dim3(unsigned((kp + kDPrepK - 1) / kDPrepK), MT, nx), 256, 0, s>>>(p);
    K3_CHECK_LAUNCH("dense_prep_kernel");
    return K3_OK;
}

int check_seg(const k3_dense_seg& g, const char* who) {
    const std::string w(who);
    if (!g.w || !g.x) return fail(K3_ERR_INVALID, w + ": NULL weight or input");
    if (g.x_dtype != K3_F32 && g.x_dtype != K3_BF16) return fail(K3_ERR_INVALID, w + ": x must be f32 or bf16");
    if (g.K < 8 || g.K % 8) return fail(K3_ERR_INVALID, w + ": K must be a positive multiple of 8");
    if (g.ldw < g.K || g.ldw % 8) return fail(K3_ERR_INVALID, w + ": ldw must be >= K and a multiple of 8");
    if (g.ldx < g.K) return fail(K3_ERR_INVALID, w + ": ldx must be >= K");
    if (!aligned16(g.w)) return fail(K3_ERR_INVALID, w + ": weights must be 16-byte aligned");
    if (g.act_input) {
        if (g.ldx < 2 * g.K) return fail(K3_ERR_INVALID, w + ": an act_input row holds [gate | up]: ldx must be >= 2K");
        if (g.norm_w) return fail(K3_ERR_INVALID, w + ": act_input and norm_w exclude each other");
    }
    return K3_OK;
}

int dense_run(const k3_dense_seg* segs, int nseg, int64_t M, int64_t N, int combine, int act, float beta,
              float lbeta, void* out, int out_dtype, int64_t ldo, float* logits, void* ws, size_t ws_bytes,
              cudaStream_t s) {
    const int64_t nblk = combine == K3_DENSE_ACT ? (N + kDBlockRows / 2 - 1) / (kDBlockRows / 2)
                                                 : (N + kDBlockRows - 1) / kDBlockRows;
    int64_t K[kDMaxSeg] = {segs[0].K, nseg > 1 ? segs[1].K : 0};
    const DenseLayout L = dense_layout(M, nblk, combine == K3_DENSE_ACT ? 1 : nseg, K);
    if (int rc = check_ws(ws, ws_bytes, L.total)) return rc;
    uint8_t* w8 = static_cast<uint8_t*>(ws);
    const int MT = mt_of(M);
    const int nx = combine == K3_DENSE_ACT ? 1 : nseg;    // ACT: both matrices read segment 0's input

    DenseArgs a{};
    for (int i = 0; i < nseg; ++i) {
        const int box = combine == K3_DENSE_ACT ? kDBlockRows / 2 : kDBlockRows;
        if (int rc = weight_map(&a.map[i], segs[i].w, N, segs[i].K, segs[i].ldw, box)) return rc;
    }

    PrepArgs p{};
    for (int i = 0; i < nx; ++i) {
        p.x[i] = segs[i].x;
        p.xdt[i] = segs[i].x_dtype;
        p.ldx[i] = segs[i].ldx;
        p.K[i] = segs[i].K;
        p.Kp[i] = units_of(segs[i].K) * kDUnitK;
        p.norm_w[i] = segs[i].norm_w;
        p.eps[i] = segs[i].eps;
        p.act_in[i] = segs[i].act_input ? 1 : 0;
        p.xt[i] = reinterpret_cast<float*>(w8 + L.xt[i]);
    }
    p.act_kind = act;
    p.beta = beta;
    p.lbeta = lbeta;
    p.M = int(M);
    p.MT = MT;
    p.cnt = reinterpret_cast<int*>(w8 + L.cnt);
    p.nblk = int(nblk);
    p.key = reinterpret_cast<unsigned long long*>(w8 + kDKeyOff);
    p.status = reinterpret_cast<int*>(w8 + kDStatusOff);
    prof_begin(K3_PROF_DENSE, s);
    int rc = K3_OK;
    switch (MT) {
        case 1: rc = launch_prep<1>(p, nx, s); break;
        case 2: rc = launch_prep<2>(p, nx, s); break;
        case 4: rc = launch_prep<4>(p, nx, s); break;
        default: rc = launch_prep<8>(p, nx, s); break;
    }
    if (rc) return rc;

    for (int i = 0; i < nseg; ++i) {
        a.seg[i].K = segs[i].K;
        a.seg[i].units = int(units_of(segs[i].K));
        a.seg[i].xt = p.xt[combine == K3_DENSE_ACT ? 0 : i];
    }
    a.nseg = combine == K3_DENSE_ACT ? 1 : nseg;   // ACT runs the units of one k range
    a.N = N;
    a.M = int(M);
    a.combine = combine;
    a.act_kind = act;
    a.beta = beta;
    a.lbeta = lbeta;
    a.out = out;
    a.out_dtype = out_dtype;
    a.ldo = ldo;
    a.nblk = int(nblk);
    a.ku = a.seg[0].units + (a.nseg > 1 ? a.seg[1].units : 0);
    a.U = nblk * a.ku;
    a.rec = reinterpret_cast<float*>(w8 + L.rec);
    a.cnt = p.cnt;
    a.key = p.key;
    a.logits = logits;
    a.status = p.status;
    switch (MT) {
        case 1: rc = launch_dense<1>(a, s); break;
        case 2: rc = launch_dense<2>(a, s); break;
        case 4: rc = launch_dense<4>(a, s); break;
        default: rc = launch_dense<8>(a, s); break;
    }
    prof_end(K3_PROF_DENSE, s);
    return rc;
}

}  // namespace
}  // namespace k3

using namespace k3;

extern "C" K3_API size_t k3_dense_workspace(int64_t M, int64_t N, int nseg, int64_t K0, int64_t K1) {
    if (M < 1 || M > kMaxTok || N < 1 || nseg < 1 || nseg > kDMaxSeg) return 0;
    const int64_t K[kDMaxSeg] = {K0, K1};
    // the ACT layout (one input, twice the row blocks) is never larger than SUM's with nseg = 2
    const int64_t nblk = (N + kDBlockRows / 2 - 1) / (kDBlockRows / 2);
    return dense_layout(M, nblk, nseg, K).total;
}

extern "C" K3_API int k3_dense_matvec(const k3_dense_seg* segs, int nseg, int64_t M, int64_t N, int combine,
                                      int activation, float situ_beta, float situ_linear_beta, void* out,
                                      int out_dtype, int64_t ldo, void* workspace, size_t workspace_bytes,
                                      void* stream) {
    if (!segs || !out) return fail(K3_ERR_INVALID, "k3_dense_matvec: NULL segments or output");
    if (nseg < 1 || nseg > kDMaxSeg) return fail(K3_ERR_INVALID, "k3_dense_matvec: nseg must be 1 or 2");
    if (M < 1 || M > kMaxTok) return fail(K3_ERR_UNSUPPORTED, "k3_dense_matvec: M must be 1..8");
    if (N < 1 || N > (int64_t(1) << 31) - 64) return fail(K3_ERR_INVALID, "k3_dense_matvec: N out of range");
    if (combine != K3_DENSE_SUM && combine != K3_DENSE_ACT)
        return fail(K3_ERR_INVALID, "k3_dense_matvec: combine must be K3_DENSE_SUM or K3_DENSE_ACT");
    if (out_dtype != K3_F32 && out_dtype != K3_BF16) return fail(K3_ERR_INVALID, "k3_dense_matvec: out must be f32 or bf16");
    if (ldo < N) return fail(K3_ERR_INVALID, "k3_dense_matvec: ldo must be >= N");
    bool act_in = false;
    for (int i = 0; i < nseg; ++i) {
        if (int rc = check_seg(segs[i], "k3_dense_matvec")) return rc;
        act_in = act_in || segs[i].act_input;
    }
    if (act_in && combine != K3_DENSE_SUM)
        return fail(K3_ERR_INVALID, "k3_dense_matvec: act_input segments need K3_DENSE_SUM");
    if (act_in && activation != K3_ACT_SILU && activation != K3_ACT_SITU)
        return fail(K3_ERR_INVALID, "k3_dense_matvec: unknown activation");
    if (combine == K3_DENSE_ACT) {
        if (nseg != 2) return fail(K3_ERR_INVALID, "k3_dense_matvec: ACT needs two segments (gate, up)");
        if (segs[1].K != segs[0].K) return fail(K3_ERR_INVALID, "k3_dense_matvec: ACT segments need the same K");
        if (activation != K3_ACT_SILU && activation != K3_ACT_SITU)
            return fail(K3_ERR_INVALID, "k3_dense_matvec: unknown activation");
    }
    return dense_run(segs, nseg, M, N, combine, activation, situ_beta, situ_linear_beta, out, out_dtype, ldo, nullptr,
                     workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" K3_API size_t k3_lm_head_workspace(int64_t H, int64_t V) {
    if (H < 8 || V < 1) return 0;
    const int64_t K[kDMaxSeg] = {H, 0};
    return dense_layout(1, (V + kDBlockRows - 1) / kDBlockRows, 1, K).total;
}

extern "C" K3_API int k3_lm_head_argmax(const void* h, int h_dtype, int64_t H, const uint16_t* w, int64_t V,
                                        int32_t* idx_out, float* val_out, float* logits_out, void* workspace,
                                        size_t workspace_bytes, void* stream) {
    if (!h || !w || !idx_out || !val_out) return fail(K3_ERR_INVALID, "k3_lm_head_argmax: NULL tensor");
    if (V < 1 || V > (int64_t(1) << 31) - 64) return fail(K3_ERR_INVALID, "k3_lm_head_argmax: V out of range");
    k3_dense_seg g{};
    g.w = w;
    g.ldw = H;
    g.K = H;
    g.x = h;
    g.x_dtype = h_dtype;
    g.ldx = H;
    if (int rc = check_seg(g, "k3_lm_head_argmax")) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (int rc = dense_run(&g, 1, 1, V, kCombineArgmax, 0, 0.0f, 0.0f, nullptr, K3_F32, V, logits_out, workspace,
                           workspace_bytes, s))
        return rc;
    dense_argmax_finish_kernel<<<1, 1, 0, s>>>(
        reinterpret_cast<const unsigned long long*>(static_cast<uint8_t*>(workspace) + kDKeyOff), idx_out, val_out);
    K3_CHECK_LAUNCH("dense_argmax_finish_kernel");
    return K3_OK;
}

extern "C" K3_API int k3_dense_status(const void* workspace, void* stream) {
    if (!workspace) return fail(K3_ERR_INVALID, "k3_dense_status: workspace is NULL");
    int st = K3_OK;
    if (int rc = cuda_check(cudaMemcpyAsync(&st, static_cast<const uint8_t*>(workspace) + kDStatusOff, sizeof(int),
                                            cudaMemcpyDeviceToHost, static_cast<cudaStream_t>(stream)),
                            "cudaMemcpyAsync(status)"))
        return rc;
    if (int rc = cuda_check(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "cudaStreamSynchronize"))
        return rc;
    return st;
}
