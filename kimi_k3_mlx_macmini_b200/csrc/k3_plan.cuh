// Routing plan construction shared by the prep and fused-router kernels (device code
// included by each translation unit that launches them).
#pragma once

#include "k3_moe.cuh"

namespace k3 {

// Orderable 32-bit key of a float (unsigned order == float order; -0 keys as +0). NaN
// keys as 1, below every number (-inf keys as 0x007fffff), so a row is taken from its
// NaN entries (lowest index first, the call flagged invalid) only when it has fewer than
// k numbers; 0 marks retired and padding slots.
__device__ __forceinline__ uint32_t order_key(float f) {
    if (f != f) return 1u;
    const uint32_t b = __float_as_uint(f == 0.0f ? 0.0f : f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ uint32_t redux_max_u32(uint32_t v) {
    uint32_t r;
    asm volatile("redux.sync.max.u32 %0, %1, 0xffffffff;\n" : "=r"(r) : "r"(v));
    return r;
}
__device__ __forceinline__ uint32_t redux_min_u32(uint32_t v) {
    uint32_t r;
    asm volatile("redux.sync.min.u32 %0, %1, 0xffffffff;\n" : "=r"(r) : "r"(v));
    return r;
}

// Top-k of one token's row by one warp: raw = sigmoid(logit), corrected = raw + bias;
// k rounds of a warp argmax on (corrected desc, index asc); weights gathered from raw.
// Lane l holds entries l, l+32, ...; every load is issued up front (clamped index), and a
// round is a lane-local scan plus two warp reductions (max key, then lowest index).
__device__ inline void topk_row(const float* __restrict__ lrow, const float* __restrict__ bias, int E,
                                int k, int renorm, float scale, int32_t* __restrict__ idx_out,
                                float* __restrict__ w_out, float* __restrict__ raw_out,
                                float* __restrict__ cor_out, int lane, int* status) {
    const int ni = (E + 31) / 32;
    float raw[32];
    uint32_t key[32];
    float lv[32], bv[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const int e = min(lane + 32 * min(i, ni - 1), E - 1);
        lv[i] = __ldcg(lrow + e);                          // may come from other CTAs
        bv[i] = bias ? __ldg(bias + e) : 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        key[i] = 0u;
        raw[i] = 0.0f;
        if (i < ni) {
            const int e = lane + 32 * i;
            const float r = 1.0f / (1.0f + expf(-lv[i]));
            const float c = r + bv[i];
            if (e < E) {
                raw[i] = r;
                key[i] = order_key(c);
                if (raw_out) raw_out[e] = r;
                if (cor_out) cor_out[e] = c;
            }
        }
    }
    float wsum = 0.0f;
    for (int s = 0; s < k; ++s) {
        uint32_t best = 0u;
        int bi = 0;
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if (i < ni && key[i] > best) {                // strict: the lowest index wins ties
                best = key[i];
                bi = i;
            }
        const uint32_t kmax = redux_max_u32(best);
        const uint32_t cand = (best == kmax) ? uint32_t(lane + 32 * bi) : 0xffffffffu;
        uint32_t e = redux_min_u32(cand);
        if (kmax <= 1u) {                                  // only NaN (1) / exhausted (0) rows
            if (lane == 0) atomicExch(status, K3_ERR_INVALID);
            if (kmax == 0u) e = 0;
        }
        float mine = 0.0f;
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if (lane + 32 * i == int(e)) {
                mine = raw[i];
                key[i] = 0u;                               // retired
            }
        const float w = __shfl_sync(0xffffffffu, mine, int(e) & 31);
        wsum += w;
        if (lane == 0) {
            idx_out[s] = int32_t(e);
            w_out[s] = w;
        }
    }
    // w / (sum + 1e-20) then * scale, as moe.py:74-76 / k3ref/layers.py:221-224
    __syncwarp();
    if (lane < k) {
        const float w = w_out[lane];
        w_out[lane] = ((k > 1 && renorm) ? w / (wsum + 1e-20f) : w) * scale;
    }
    __syncwarp();
}

// One warp per token row from its precomputed keys (order_key(sigmoid(logit) + bias)) and
// sigmoid scores: lane l holds experts l, l+32, ... (NE = ceil(E/32) slots), loaded with
// one round trip; k rounds of argmax on (key desc, index asc) retire the winners and pick
// up their raw scores from the owning lane; the weights are those raw scores,
// renormalised (sum in selection order) and scaled as topk_row does. Results go to
// idx_out / w_out and to the CTA's shared copies si / sw.
template <int NE>
__device__ __noinline__ void topk_warp_regs(const uint32_t* __restrict__ krow, const float* __restrict__ srow,
                                            int E, int k, int renorm, float scale, int32_t* __restrict__ idx_out,
                                            float* __restrict__ w_out, int* si, float* sw, int lane, int* status) {
    float raw[NE];
    uint32_t key[NE];
#pragma unroll
    for (int i = 0; i < NE; ++i) {
        const int e = lane + 32 * i;
        key[i] = e < E ? __ldcg(krow + e) : 0u;               // written by other CTAs
        raw[i] = e < E ? __ldcg(srow + e) : 0.0f;
    }
    int mine = -1;
    float wmine = 0.0f;
#pragma unroll 1
    for (int s = 0; s < k; ++s) {
        uint32_t best = 0u;
        int bi = 0;
#pragma unroll
        for (int i = 0; i < NE; ++i)
            if (key[i] > best) {                              // strict: lowest index wins ties
                best = key[i];
                bi = i;
            }
        const uint32_t kmax = redux_max_u32(best);
        uint32_t e = redux_min_u32(best == kmax ? uint32_t(lane + 32 * bi) : 0xffffffffu);
        if (kmax <= 1u) {                                     // only NaN (1) / exhausted (0) rows
            if (lane == 0) atomicExch(status, K3_ERR_INVALID);
            if (kmax == 0u) e = 0;
        }
        float rw = 0.0f;
#pragma unroll
        for (int i = 0; i < NE; ++i)
            if (lane + 32 * i == int(e)) {
                key[i] = 0u;                                  // retired
                rw = raw[i];
            }
        const float w = __shfl_sync(0xffffffffu, rw, int(e) & 31);
        if (lane == s) {
            mine = int(e);
            wmine = w;
        }
    }
    float sum = 0.0f;
#pragma unroll 1
    for (int s = 0; s < k; ++s) sum += __shfl_sync(0xffffffffu, wmine, s);
    if (lane < k) {
        const float wo = ((k > 1 && renorm) ? wmine / (sum + 1e-20f) : wmine) * scale;
        idx_out[lane] = mine;
        w_out[lane] = wo;
        si[lane] = mine;
        sw[lane] = wo;
    }
}

// Top-k of one token row by one warp, from keys the CTA staged in shared memory (row[e] =
// order_key(sigmoid(logit) + bias), 1 for NaN) and the row's sigmoid scores srow. The selection is that of k rounds of argmax
// on (key desc, index asc), found without the rounds' serial chains: T, the k-th largest
// key, by a bitwise search on counts (keys >= candidate; lane l holds keys l, l+32, ... in
// NE registers, so each step is NE independent compares and one warp reduction, over only
// the bits below the common prefix of the row's largest and smallest key); then one pass in
// index order takes the keys above T and the lowest-index keys equal to T; then each winner's
// rank by counting. Weights are the winners' raw scores, renormalised (sum in rank order) and
// scaled as topk_row does; results go to idx_out / w_out and the shared copies si / sw. For wide routers (E > 512) this beats k argmax rounds over 24-32
// registers per lane; up to 512 experts the rounds are faster.
template <int NE>
__device__ __noinline__ void topk_warp_count(const uint32_t* row, const float* __restrict__ srow, int E, int k,
                                             int renorm, float scale, int32_t* __restrict__ idx_out,
                                             float* __restrict__ w_out, int* si, float* sw, int* cand_e,
                                             uint32_t* cand_k, int lane, int* status) {
    uint32_t key[NE];
    uint32_t hi = 0u, lo = 0xffffffffu;
#pragma unroll
    for (int s = 0; s < NE; ++s) {
        const int e = lane + 32 * s;
        key[s] = e < E ? row[e] : 0u;
        hi = max(hi, key[s]);
        lo = e < E ? min(lo, key[s]) : lo;
    }
    hi = redux_max_u32(hi);
    lo = redux_min_u32(lo);
    // every key shares hi's bits above the highest bit where hi and lo differ
    const uint32_t diff = hi ^ lo;
    const int nbits = diff ? 32 - __clz(int(diff)) : 0;
    uint32_t T = nbits == 32 ? 0u : (hi & ~((1u << nbits) - 1u));
    int n_gt = 0;
#pragma unroll 1
    for (int it = 0; it <= nbits; ++it) {
        // steps 0..nbits-1 try the next bit of T; the last counts the keys above T
        const uint32_t cand = it < nbits ? (T | (1u << (nbits - 1 - it))) : T + 1u;
        uint32_t c = 0;
#pragma unroll
        for (int s = 0; s < NE; ++s) c += key[s] >= cand ? 1u : 0u;
        c = __reduce_add_sync(0xffffffffu, c);
        if (it < nbits) {
            if (c >= uint32_t(k)) T = cand;
        } else {
            n_gt = int(c);
        }
    }
    if (T <= 1u && lane == 0) atomicExch(status, K3_ERR_INVALID);   // fewer than k non-NaN scores
    // the winners in index order: every key above T, then keys equal to T up to k
    const uint32_t lt = (1u << lane) - 1u;
    int taken = 0, quota = k - n_gt;
    uint32_t v = lane < E ? row[lane] : 0u;
#pragma unroll 1
    for (int e0 = 0; e0 < E && taken < k; e0 += 32) {
        const int e = e0 + lane;
        const uint32_t cur = v;
        v = e + 32 < E ? row[e + 32] : 0u;                       // next chunk in flight
        const bool eq = e < E && cur == T;
        const uint32_t be = __ballot_sync(0xffffffffu, eq);
        const bool take = (e < E && cur > T) || (eq && __popc(be & lt) < quota);
        const uint32_t bt = __ballot_sync(0xffffffffu, take);
        if (take) {
            const int at = taken + __popc(bt & lt);
            cand_e[at] = e;
            cand_k[at] = cur;
        }
        taken += __popc(bt);
        quota -= min(__popc(be), quota);
    }
    __syncwarp();
    // rank of each winner on (key desc, index asc), then the outputs in rank order
    const int ej = lane < k ? cand_e[lane] : 0;
    const uint32_t kj = lane < k ? cand_k[lane] : 0u;
    int rank = 0;
#pragma unroll 1
    for (int i = 0; i < k; ++i) {
        const uint32_t ki = __shfl_sync(0xffffffffu, kj, i);
        const int ei = __shfl_sync(0xffffffffu, ej, i);
        rank += (ki > kj || (ki == kj && ei < ej)) ? 1 : 0;
    }
    __syncwarp();
    if (lane < k) cand_e[rank] = ej;
    __syncwarp();
    const int mine = lane < k ? cand_e[lane] : 0;
    const float w = lane < k ? __ldcg(srow + mine) : 0.0f;
    float sum = 0.0f;
#pragma unroll 1
    for (int s = 0; s < k; ++s) sum += __shfl_sync(0xffffffffu, w, s);
    if (lane < k) {
        const float wo = ((k > 1 && renorm) ? w / (sum + 1e-20f) : w) * scale;
        idx_out[lane] = mine;
        w_out[lane] = wo;
        si[lane] = mine;
        sw[lane] = wo;
    }
}

// Whole-CTA top-k of M token rows (M <= 8) from precomputed keys and sigmoid scores
// ([M][E] each, written by other CTAs), warp t selecting token t's k experts into
// idx_out / w_out and the shared copies si / sw ([M][k]). Up to E = 512 the warp holds
// its row in registers and runs k argmax rounds; wider rows are first staged in s_key
// (M * E words of shared scratch; eight loads in flight per thread per pass) for the
// counting search.
__device__ inline void topk_cta(const uint32_t* __restrict__ keys, const float* __restrict__ scores, int M,
                                int E, int k, int renorm, float scale, int32_t* __restrict__ idx_out,
                                float* __restrict__ w_out, int* si, float* sw, uint32_t* s_key, int warp,
                                int lane, int* status) {
    __shared__ int cand_e[kMaxTok][kMaxTopK];
    __shared__ uint32_t cand_k[kMaxTok][kMaxTopK];
    if (E <= 512) {
        if (warp >= M) return;
        const uint32_t* krow = keys + int64_t(warp) * E;
        const float* srow = scores + int64_t(warp) * E;
        int32_t* io = idx_out + warp * k;
        float* wo = w_out + warp * k;
        int* sio = si + warp * k;
        float* swo = sw + warp * k;
        if (E <= 128) topk_warp_regs<4>(krow, srow, E, k, renorm, scale, io, wo, sio, swo, lane, status);
        else if (E <= 256) topk_warp_regs<8>(krow, srow, E, k, renorm, scale, io, wo, sio, swo, lane, status);
        else if (E <= 384) topk_warp_regs<12>(krow, srow, E, k, renorm, scale, io, wo, sio, swo, lane, status);
        else topk_warp_regs<16>(krow, srow, E, k, renorm, scale, io, wo, sio, swo, lane, status);
        return;
    }
#pragma unroll 1
    for (int i0 = threadIdx.x; i0 < M * E; i0 += 8 * blockDim.x) {
        uint32_t v[8];
#pragma unroll
        for (int h = 0; h < 8; ++h) v[h] = __ldcg(keys + min(i0 + h * int(blockDim.x), M * E - 1));
#pragma unroll
        for (int h = 0; h < 8; ++h) {
            const int i = i0 + h * int(blockDim.x);
            if (i < M * E) s_key[i] = v[h];
        }
    }
    __syncthreads();
    if (warp >= M) return;
    const uint32_t* row = s_key + warp * E;
    const float* srow = scores + int64_t(warp) * E;
    int32_t* io = idx_out + warp * k;
    float* wo = w_out + warp * k;
    int* sio = si + warp * k;
    float* swo = sw + warp * k;
    int* ce = cand_e[warp];
    uint32_t* ck = cand_k[warp];
    if (E <= 768) topk_warp_count<24>(row, srow, E, k, renorm, scale, io, wo, sio, swo, ce, ck, lane, status);
    else topk_warp_count<32>(row, srow, E, k, renorm, scale, io, wo, sio, swo, ce, ck, lane, status);
}

// The routing part of a decode call.
struct PlanArgs {
    const float* bias;
    // fused router only: the top-k keys and sigmoid scores [M][E] (see topk_cta)
    uint32_t* keys;
    float* scores;
    int E, k, renorm;
    float scale;
    int32_t* idx;                  // [M][k]: written here when logits are given, else read
    float* w;
    int has_shared;
    Plan* plan;
    unsigned* cntA;                // arrival counters of the two grouped-matvec launches,
    int64_t n_cntA;                // zeroed here
    unsigned* cntB;
    int64_t n_cntB;
    int M;
};

// Whole-CTA: zero the counters, run the top-k (warp t: token t; kSharedKeys: always,
// from a.keys / a.scores; otherwise when `logits` is given),
// then build the plan: active experts in ascending id order (moe.py:120), per expert its
// (token, weight) pairs in ascending token order, the shared expert last. Every routing
// entry finds its expert's slot and its rank among the same expert's earlier entries in
// parallel.
// kSharedKeys: the top-k runs topk_cta on the precomputed a.keys / a.scores (s_key: M * E
// words of shared scratch for wide routers) and leaves its results in shared memory as
// well; otherwise warp t runs topk_row on token t's logits. A compile-time choice, so a
// kernel carries the registers of only the form it uses.
template <bool kSharedKeys = false>
__device__ inline void build_plan_cta(const PlanArgs& a, const float* logits, int warp, int lane,
                                      uint32_t* s_key = nullptr) {
    Plan* P = a.plan;
    __shared__ uint32_t bitmap[kMaxExperts / 32];
    __shared__ int16_t pos_e[kMaxExperts];          // active index of expert e
    __shared__ int cnt[kMaxActive];
    __shared__ int start[kMaxActive + 1];
    __shared__ int n_routed;
    __shared__ int s_idx[kMaxTok * kMaxTopK];
    __shared__ float s_w[kMaxTok * kMaxTopK];
    if (threadIdx.x == 0) P->status = K3_OK;
    for (int64_t i = threadIdx.x; i < a.n_cntA; i += blockDim.x) a.cntA[i] = 0;
    for (int64_t i = threadIdx.x; i < a.n_cntB; i += blockDim.x) a.cntB[i] = 0;
    for (int i = threadIdx.x; i < kMaxExperts / 32; i += blockDim.x) bitmap[i] = 0;
    for (int i = threadIdx.x; i < kMaxActive; i += blockDim.x) cnt[i] = 0;
    __syncthreads();
    if constexpr (kSharedKeys) {
        topk_cta(a.keys, a.scores, a.M, a.E, a.k, a.renorm, a.scale, a.idx, a.w, s_idx, s_w, s_key, warp,
                 lane, &P->status);
    } else {
        if (logits && warp < a.M)
            topk_row(logits + int64_t(warp) * a.E, a.bias, a.E, a.k, a.renorm, a.scale,
                     a.idx + warp * a.k, a.w + warp * a.k, nullptr, nullptr, lane, &P->status);
    }
    __syncthreads();                               // top-k results visible
    const int nsel = a.M * a.k;
    for (int i = threadIdx.x; i < nsel; i += blockDim.x) {
        int e;
        if constexpr (kSharedKeys) {
            e = s_idx[i];                          // the top-k's shared copy
        } else {
            e = a.idx[i];
            s_idx[i] = e;
            s_w[i] = a.w[i];
        }
        if (e < 0 || e >= a.E)
            P->status = K3_ERR_INVALID;
        else
            atomicOr(&bitmap[e >> 5], 1u << (e & 31));
    }
    __syncthreads();
    if (warp == 0) {                               // ascending unique expert list
        int base = 0;
        for (int w0 = 0; w0 < kMaxExperts / 32; w0 += 32) {
            const uint32_t word = bitmap[w0 + lane];
            const int c = __popc(word);
            int incl = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            int pos = base + incl - c;
            uint32_t wv = word;
            while (wv) {
                const int b = __ffs(wv) - 1;
                wv &= wv - 1;
                const int e = (w0 + lane) * 32 + b;
                P->expert[pos] = e;
                pos_e[e] = int16_t(pos);
                ++pos;
            }
            base += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (lane == 0) n_routed = base;
    }
    __syncthreads();
    const int nr = n_routed;
    const int na = nr + (a.has_shared ? 1 : 0);
    // rank of each entry among the earlier entries of its expert (token-major order)
    int my_rank = 0, my_pos = 0;
    const int i_me = threadIdx.x;
    if (i_me < nsel) {
        const int e = s_idx[i_me];
        if (e >= 0 && e < a.E) {
            for (int j = 0; j < i_me; ++j) my_rank += (s_idx[j] == e);
            my_pos = pos_e[e];
            atomicAdd(&cnt[my_pos], 1);
        }
    }
    __syncthreads();
    if (warp == 0) {                               // pair offsets: exclusive scan of counts
        int base = 0;
        for (int u0 = 0; u0 < na + 1; u0 += 32) {
            const int u = u0 + lane;
            int c = 0;
            if (u < nr) {
                c = cnt[u];
                if (c > kMaxTok) {                 // a token listed the same expert twice
                    P->status = K3_ERR_INVALID;
                    c = kMaxTok;
                }
            } else if (u < na) {
                c = a.M;                           // shared expert: every token
            }
            int incl = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            if (u <= na) {
                start[u] = base + incl - c;
                P->pair_start[u] = base + incl - c;
            }
            base += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (lane == 0) {
            P->n_active = na;
            P->n_pairs = start[na];
            P->M = a.M;
            if (a.has_shared) P->expert[nr] = a.E;     // shared expert slot in the table
        }
    }
    __syncthreads();
    if (i_me < nsel) {
        const int e = s_idx[i_me];
        if (e >= 0 && e < a.E && my_rank < kMaxTok) {
            const int p = start[my_pos] + my_rank;
            P->pair_tok[p] = i_me / a.k;
            P->pair_w[p] = s_w[i_me];
        }
    }
    if (a.has_shared && int(threadIdx.x) < a.M) {
        const int p = start[nr] + threadIdx.x;
        P->pair_tok[p] = threadIdx.x;
        P->pair_w[p] = 1.0f;
    }
}

// Whole-CTA: the plan of a plain matvec -- one "expert", pairs = tokens, weights 1.
__device__ inline void identity_plan_cta(const PlanArgs& a) {
    Plan* P = a.plan;
    if (threadIdx.x == 0) P->status = K3_OK;
    for (int64_t i = threadIdx.x; i < a.n_cntA; i += blockDim.x) a.cntA[i] = 0;
    for (int64_t i = threadIdx.x; i < a.n_cntB; i += blockDim.x) a.cntB[i] = 0;
    if (threadIdx.x == 0) {
        P->M = a.M;
        P->n_active = 1;
        P->n_pairs = a.M;
        P->expert[0] = 0;
        P->pair_start[0] = 0;
        P->pair_start[1] = a.M;
    }
    for (int t = threadIdx.x; t < a.M; t += blockDim.x) {
        P->pair_tok[t] = t;
        P->pair_w[t] = 1.0f;
    }
}

// One warp: x[t][kb*512, +512) -> blocked f16 pieces [k/32][8][32] of x * 2**-e, one
// exponent per (token, 512-k block) stored in ts[t][kb]; rows t >= M become zeros.
__device__ inline void convert_block(const void* x, int x_dtype, int M, int64_t H, int t, int64_t kb,
                              __half* xq_hi, __half* xq_lo, float* xq_ts, int lane) {
    float v[16];
    float mx = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const int64_t k = kb * 512 + i * 32 + lane;
        v[i] = t < M ? load_as_f32(x, x_dtype, int64_t(t) * H + k) : 0.0f;
        mx = fmaxf(mx, fabsf(v[i]));
    }
    const int e = f16_group_exponent(warp_max(mx));
    const float sc = ldexpf(1.0f, -e);
    const bool normal_sc = isfinite(sc) && sc >= 1.17549435e-38f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        __half hi, lo;
        split_f16(normal_sc ? v[i] * sc : ldexpf(v[i], -e), hi, lo);
        const int64_t o = ((kb * 16 + i) * kMaxTok + t) * 32 + lane;
        xq_hi[o] = hi;
        if (xq_lo) xq_lo[o] = lo;
    }
    if (lane == 0) xq_ts[int64_t(t) * (H / 512) + kb] = ldexpf(1.0f, e);
}

}  // namespace k3
