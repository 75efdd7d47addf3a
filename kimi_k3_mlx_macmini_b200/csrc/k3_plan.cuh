// Routing plan construction shared by the prep and fused-router kernels (device code
// included by each translation unit that launches them).
#pragma once

#include "k3_moe.cuh"

namespace k3 {

// Top-k of one token's row by one warp: raw = sigmoid(logit), corrected = raw + bias;
// k rounds of a warp argmax on (corrected desc, index asc); weights gathered from raw.
__device__ inline void topk_row(const float* __restrict__ lrow, const float* __restrict__ bias, int E,
                         int k, int renorm, float scale, int32_t* __restrict__ idx_out,
                         float* __restrict__ w_out, float* __restrict__ raw_out,
                         float* __restrict__ cor_out, int lane, int* status) {
    float raw[32], cor[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const int e = lane + 32 * i;
        if (e < E) {
            const float l = __ldcg(lrow + e);      // may come from other CTAs of this launch
            const float r = 1.0f / (1.0f + expf(-l));
            const float c = r + (bias ? bias[e] : 0.0f);
            raw[i] = r;
            cor[i] = c;
            if (raw_out) raw_out[e] = r;
            if (cor_out) cor_out[e] = c;
        } else {
            raw[i] = 0.0f;
            cor[i] = -INFINITY;
        }
    }
    float wsel[kMaxTopK > 32 ? kMaxTopK : 32];
    int isel[kMaxTopK > 32 ? kMaxTopK : 32];
    for (int s = 0; s < 32; ++s) {
        if (s >= k) break;
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const int e = lane + 32 * i;
            if (e < E && (cor[i] > bv || (cor[i] == bv && e < bi))) {
                bv = cor[i];
                bi = e;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (bi >= E) {            // only NaN rows get here: report, pick a valid index
            if (lane == 0) atomicExch(status, K3_ERR_INVALID);
            bi = 0;
        }
        // the owner lane reads the raw score and retires the entry: a NaN never compares
        // greater or equal, so it cannot win again even when every other entry is -inf
        float mine = 0.0f;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            if (lane + 32 * i == bi) {
                mine = raw[i];
                cor[i] = __int_as_float(0x7fc00000u);
            }
        }
        wsel[s] = __shfl_sync(0xffffffffu, mine, bi & 31);
        isel[s] = bi;
    }
    // w / (sum + 1e-20) then * scale, as moe.py:74-76 / k3ref/layers.py:221-224
    float sum = 0.0f;
    for (int s = 0; s < k; ++s) sum += wsel[s];
    const float den = sum + 1e-20f;
    if (lane == 0) {
        for (int s = 0; s < k; ++s) {
            idx_out[s] = isel[s];
            w_out[s] = ((k > 1 && renorm) ? wsel[s] / den : wsel[s]) * scale;
        }
    }
}


// The routing part of a decode call.
struct PlanArgs {
    const float* bias;
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

// Whole-CTA: zero the counters, run the top-k when `logits` is given (warp t: token t),
// then build the plan: active experts in ascending id order (moe.py:120), per expert its
// (token, weight) pairs in ascending token order, the shared expert last.
__device__ inline void build_plan_cta(const PlanArgs& a, const float* logits, int warp, int lane) {
    Plan* P = a.plan;
    __shared__ uint32_t bitmap[kMaxExperts / 32];
    __shared__ int cnt[kMaxActive];
    __shared__ int n_routed;
    __shared__ int s_idx[kMaxTok * kMaxTopK];
    __shared__ float s_w[kMaxTok * kMaxTopK];
    if (threadIdx.x == 0) P->status = K3_OK;
    for (int64_t i = threadIdx.x; i < a.n_cntA; i += blockDim.x) a.cntA[i] = 0;
    for (int64_t i = threadIdx.x; i < a.n_cntB; i += blockDim.x) a.cntB[i] = 0;
    __syncthreads();
    if (logits && warp < a.M) {
        topk_row(logits + int64_t(warp) * a.E, a.bias, a.E, a.k, a.renorm, a.scale,
                 a.idx + warp * a.k, a.w + warp * a.k, nullptr, nullptr, lane, &P->status);
    }
    for (int i = threadIdx.x; i < kMaxExperts / 32; i += blockDim.x) bitmap[i] = 0;
    __syncthreads();                               // top-k results and zeroed bitmap visible
    const int nsel = a.M * a.k;
    for (int i = threadIdx.x; i < nsel; i += blockDim.x) {
        s_idx[i] = a.idx[i];
        s_w[i] = a.w[i];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < nsel; i += blockDim.x) {
        const int e = s_idx[i];
        if (e < 0 || e >= a.E) {
            P->status = K3_ERR_INVALID;
            continue;
        }
        atomicOr(&bitmap[e >> 5], 1u << (e & 31));
    }
    __syncthreads();
    if (warp == 0) {                               // ascending unique expert list
        const uint32_t word = bitmap[lane];
        const int c = __popc(word);
        int incl = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        int pos = incl - c;
        uint32_t wv = word;
        while (wv) {
            const int b = __ffs(wv) - 1;
            wv &= wv - 1;
            P->expert[pos++] = lane * 32 + b;
        }
        if (lane == 31) n_routed = incl;
    }
    __syncthreads();
    const int nr = n_routed;
    const int na = nr + (a.has_shared ? 1 : 0);
    for (int u = threadIdx.x; u < na; u += blockDim.x) {
        int c = 0;
        if (u < nr) {
            const int e = P->expert[u];
            for (int i = 0; i < nsel; ++i) c += (s_idx[i] == e);
            if (c > kMaxTok) {          // a token listed the same expert twice: invalid routing
                P->status = K3_ERR_INVALID;
                c = kMaxTok;
            }
        } else {
            c = a.M;
            P->expert[u] = a.E;                    // shared expert slot in the table
        }
        cnt[u] = c;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int s = 0;
        for (int u = 0; u < na; ++u) {
            P->pair_start[u] = s;
            s += cnt[u];
        }
        P->pair_start[na] = s;
        P->n_active = na;
        P->n_pairs = s;
        P->M = a.M;
    }
    __syncthreads();
    for (int u = threadIdx.x; u < na; u += blockDim.x) {
        int p = P->pair_start[u];
        if (u < nr) {
            const int e = P->expert[u];
            const int pend = P->pair_start[u + 1];
            for (int t = 0; t < a.M; ++t)
                for (int s = 0; s < a.k; ++s)
                    if (s_idx[t * a.k + s] == e && p < pend) {
                        P->pair_tok[p] = t;
                        P->pair_w[p] = s_w[t * a.k + s];
                        ++p;
                    }
        } else {
            for (int t = 0; t < a.M; ++t) {
                P->pair_tok[p] = t;
                P->pair_w[p] = 1.0f;
                ++p;
            }
        }
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
