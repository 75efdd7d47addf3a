// Routing plans from explicit (slot, token, weight) pairs, and x -> E2M1 pieces for any
// number of tokens: the front end of the expert-parallel local computation, where one
// rank runs its own experts over every pair that routes to them.
#include "k3_bs.cuh"
#include "k3_pairs.cuh"

namespace k3 {

// One CTA (256 threads). Candidates with slot outside [0, num_slots) or token outside
// [0, T) are skipped. Items: the used slots in ascending order, each split into chunks of
// at most 8 pairs; a slot's pairs keep their candidate order. Too many items or pairs for
// a plan set K3_ERR_UNSUPPORTED in plan->status (the surplus is dropped).
__device__ void convert_tokens_body(const void* x, int x_dtype, int64_t T, int64_t K, uint8_t* xp, uint8_t* xsf,
                                    int64_t first_warp, int64_t n_warps);

// CTA 0 builds the plan; CTAs 1.. convert the tokens to pieces (convert_tokens_body) at
// the same time, when conv.xp is set.
__global__ void __launch_bounds__(256) plan_from_pairs_kernel(PairsArgs a, ConvertArgs conv) {
    if (blockIdx.x > 0) {
        convert_tokens_body(conv.x, conv.x_dtype, conv.T, conv.K, conv.xp, conv.xsf,
                            int64_t(blockIdx.x - 1) * (blockDim.x >> 5), int64_t(gridDim.x - 1) * (blockDim.x >> 5));
        return;
    }
    constexpr int kMaxSlots = kMaxExperts + 1;
    __shared__ uint32_t bitmap[(kMaxSlots + 31) / 32];
    __shared__ int cnt_s[kMaxSlots];
    __shared__ int16_t pos_s[kMaxSlots];
    __shared__ int list[kMaxPairs];                    // used slots, ascending
    __shared__ int pbase[kMaxPairs + 1], ibase[kMaxPairs + 1];
    __shared__ int vidx[kMaxPairCandidates];           // valid candidates, in order
    __shared__ int vslot[kMaxPairCandidates];
    __shared__ int chunk_cnt[kMaxPairCandidates / 32];
    __shared__ int vrank[kMaxPairCandidates];          // rank among the earlier candidates of its slot
    __shared__ int run_s[kMaxSlots];                   // running count per slot (ranking pass)
    __shared__ int n_valid, n_used, n_items, n_pairs;
    Plan* P = a.plan;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) P->status = K3_OK;
    for (int64_t i = threadIdx.x; i < a.n_cntA; i += blockDim.x) a.cntA[i] = 0;
    for (int64_t i = threadIdx.x; i < a.n_cntB; i += blockDim.x) a.cntB[i] = 0;
    for (int i = threadIdx.x; i < (kMaxSlots + 31) / 32; i += blockDim.x) bitmap[i] = 0;
    for (int i = threadIdx.x; i < kMaxSlots; i += blockDim.x) {
        cnt_s[i] = 0;
        run_s[i] = 0;
    }
    __syncthreads();
    // validity and in-order compaction: ballots per 32 candidates, then a scan of chunk counts
    const int nin = a.n_in;
    bool vk[kMaxPairCandidates / 256];
#pragma unroll
    for (int h = 0; h < kMaxPairCandidates / 256; ++h) {
        const int i = h * 256 + threadIdx.x;
        bool ok = false;
        int sl = -1, t = 0;
        float wv = 0.0f;
        if (i < nin) {
            pair_candidate(a, i, sl, t, wv);
            ok = sl >= 0;
        }
        vk[h] = ok;
        const uint32_t bal = __ballot_sync(0xffffffffu, ok);
        if (lane == 0) chunk_cnt[h * 8 + warp] = __popc(bal);
    }
    __syncthreads();
    if (warp == 0) {
        int v = chunk_cnt[lane];
        int incl = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += u;
        }
        chunk_cnt[lane] = incl - v;                    // exclusive
        if (lane == 31) n_valid = incl;
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < kMaxPairCandidates / 256; ++h) {
        const int i = h * 256 + threadIdx.x;
        const uint32_t bal = __ballot_sync(0xffffffffu, vk[h]);
        if (vk[h]) {
            int sl, t;
            float wv;
            pair_candidate(a, i, sl, t, wv);
            const int pos = chunk_cnt[h * 8 + warp] + __popc(bal & ((1u << lane) - 1u));
            vidx[pos] = i;
            vslot[pos] = sl;
            atomicOr(&bitmap[sl >> 5], 1u << (sl & 31));
            atomicAdd(&cnt_s[sl], 1);
        }
    }
    __syncthreads();
    if (warp == 0) {                                   // used slots ascending, then offsets
        int base = 0;
        for (int w0 = 0; w0 < (kMaxSlots + 31) / 32; w0 += 32) {
            const uint32_t word = w0 + lane < (kMaxSlots + 31) / 32 ? bitmap[w0 + lane] : 0u;
            const int c = __popc(word);
            int incl = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int u = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += u;
            }
            int pos = base + incl - c;
            uint32_t wv = word;
            while (wv) {
                const int b = __ffs(wv) - 1;
                wv &= wv - 1;
                const int sl = (w0 + lane) * 32 + b;
                if (pos < kMaxPairs) list[pos] = sl;
                pos_s[sl] = int16_t(pos < kMaxPairs ? pos : kMaxPairs - 1);
                ++pos;
            }
            base += __shfl_sync(0xffffffffu, incl, 31);
        }
        const int nu = base < kMaxPairs ? base : kMaxPairs;
        int pb = 0, ib = 0;
        for (int j0 = 0; j0 < nu; j0 += 32) {
            const int j = j0 + lane;
            const int c = j < nu ? cnt_s[list[j]] : 0;
            const int it = (c + kBMaxN / kBPieces - 1) / (kBMaxN / kBPieces);
            int ic = c, ii = it;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int u = __shfl_up_sync(0xffffffffu, ic, o);
                const int w = __shfl_up_sync(0xffffffffu, ii, o);
                if (lane >= o) {
                    ic += u;
                    ii += w;
                }
            }
            if (j < nu) {
                pbase[j] = pb + ic - c;
                ibase[j] = ib + ii - it;
            }
            pb += __shfl_sync(0xffffffffu, ic, 31);
            ib += __shfl_sync(0xffffffffu, ii, 31);
        }
        if (lane == 0) {
            n_used = nu;
            n_pairs = pb;
            n_items = ib;
            pbase[nu] = pb;
            ibase[nu] = ib;
            if (base > kMaxPairs || pb > kMaxPairs || ib > kMaxActive) P->status = K3_ERR_UNSUPPORTED;
        }
    }
    __syncthreads();
    const int nitems = n_items < kMaxActive ? n_items : kMaxActive;
    const int npairs = n_pairs < kMaxPairs ? n_pairs : kMaxPairs;
    for (int j = threadIdx.x; j < n_used; j += blockDim.x) {
        const int c = cnt_s[list[j]];
        for (int q = 0; ibase[j] + q < nitems && 8 * q < c; ++q) {
            P->expert[ibase[j] + q] = list[j];
            P->pair_start[ibase[j] + q] = pbase[j] + 8 * q;
        }
    }
    const int nv = n_valid;
    if (warp == 0) {
        // ranks in candidate order, 32 candidates a step: lanes with the same slot find each
        // other (match.any), the last of a group advances that slot's running count
        for (int c0 = 0; c0 < nv; c0 += 32) {
            const int v = c0 + lane;
            const bool act = v < nv;
            const int sl = act ? vslot[v] : -1 - lane;
            const unsigned grp = __match_any_sync(0xffffffffu, sl);
            const int before = __popc(grp & ((1u << lane) - 1u));
            const int base = act ? run_s[sl] : 0;
            if (act) vrank[v] = base + before;
            __syncwarp();
            if (act && (grp >> lane) == 1u) run_s[sl] = base + before + 1;
            __syncwarp();
        }
    }
    __syncthreads();
    for (int v = threadIdx.x; v < nv; v += blockDim.x) {
        const int sl = vslot[v];
        const int rank = vrank[v];
        const int p = pbase[pos_s[sl]] + rank;
        if (p < npairs) {
            int s2, t;
            float wv;
            pair_candidate(a, vidx[v], s2, t, wv);
            P->pair_tok[p] = t;
            P->pair_w[p] = wv;
        }
    }
    if (threadIdx.x == 0) {
        P->pair_start[nitems] = npairs;
        P->n_active = nitems;
        P->n_pairs = npairs;
        P->M = a.T;
    }
}

int launch_plan_from_pairs(const PairsArgs& a, const ConvertArgs& conv, cudaStream_t s) {
    if (a.n_in > kMaxPairCandidates) return fail(K3_ERR_UNSUPPORTED, "more than 1024 pair candidates");
    const int64_t warps = conv.xp ? conv.T * (conv.K / 32) : 0;
    const int conv_blocks = int(std::min<int64_t>((warps + 7) / 8, int64_t(num_sms()) * 8));
    plan_from_pairs_kernel<<<1 + conv_blocks, 256, 0, s>>>(a, conv);
    K3_CHECK_LAUNCH("plan_from_pairs_kernel");
    return K3_OK;
}

// x [T][K] -> E2M1 pieces [8T][K/2] and per-row scales [8T][K/32]; one warp per
// (token, 32-element block), warps first_warp, first_warp + n_warps, ...
__device__ void convert_tokens_body(const void* x, int x_dtype, int64_t T, int64_t K, uint8_t* xp, uint8_t* xsf,
                                    int64_t first_warp, int64_t n_warps) {
    const int lane = threadIdx.x & 31;
    const uint32_t G = uint32_t(K / 32);                  // 32-bit: no 64-bit division per task
    for (uint32_t task = uint32_t(first_warp) + (threadIdx.x >> 5); task < uint32_t(T) * G; task += uint32_t(n_warps)) {
        const int64_t t = task / G, g = task - uint32_t(t) * G;
        const float v = load_as_f32(x, x_dtype, t * K + 32 * g + lane);
        split_pieces(v, lane, xp + kBPieces * t * (K / 2) + 16 * g, K / 2, xsf + kBPieces * t * G + g, G);
    }
}

__global__ void __launch_bounds__(256) convert_tokens_kernel(const void* x, int x_dtype, int64_t T, int64_t K,
                                                             uint8_t* xp, uint8_t* xsf) {
    convert_tokens_body(x, x_dtype, T, K, xp, xsf, int64_t(blockIdx.x) * (blockDim.x >> 5),
                        int64_t(gridDim.x) * (blockDim.x >> 5));
}

int launch_convert_tokens(const void* x, int x_dtype, int64_t T, int64_t K, uint8_t* xp, uint8_t* xsf,
                          cudaStream_t s) {
    const int64_t warps = T * (K / 32);
    const int blocks = int(std::min<int64_t>((warps + 7) / 8, int64_t(num_sms()) * 8));
    convert_tokens_kernel<<<blocks, 256, 0, s>>>(x, x_dtype, T, K, xp, xsf);
    K3_CHECK_LAUNCH("convert_tokens_kernel");
    return K3_OK;
}

}  // namespace k3
