// Counted all-to-all of an expert-parallel MoE step: the device side of the token
// exchange between ranks at prefill sizes.
//
// Rank r owns routed experts [r*E_loc, (r+1)*E_loc). A token goes to every rank that owns
// at least one of its top-k experts, once (not once per expert), and always to its own
// rank (which applies the shared expert to every one of its tokens). The send buffer is
// destination-major, tokens ascending within a destination, so after the all-to-all a
// rank's receive buffer is [rows from rank 0][rows from rank 1]..., and its own segment
// holds all of its tokens in order. The partial outputs come back through the reverse
// all-to-all into the send buffer's row order, and a token's result is the sum of its
// rows over destinations in ascending rank order (a fixed order: deterministic).
//
// The reference runs every expert in one process (air_llm/models/kimi_k3/moe.py:119-127:
// per-token gather, per-expert weighted scatter-add); this file is the exchange that
// splits that loop over ranks.
#include "k3_common.cuh"

namespace k3 {

constexpr int kA2AMaxWorld = 32;
constexpr int kA2AThreads = 1024;

// Destination mask of token t: bit d set when one of its experts lives on rank d, and
// always the own rank's bit. An expert id outside [0, E_loc * W) flags the call and is
// skipped.
__device__ __forceinline__ uint32_t dest_mask(const int32_t* __restrict__ idx, int rstride, int t, int k,
                                              int E_loc, int W, int rank, int* status) {
    uint32_t m = 1u << rank;
    const int32_t* row = idx + int64_t(t) * rstride;
    for (int j = 0; j < k; ++j) {
        const int e = __ldg(row + j);
        if (e >= 0 && e < E_loc * W)
            m |= 1u << (e / E_loc);
        else
            atomicExch(status, K3_ERR_INVALID);
    }
    return m;
}

// One CTA of 1024 threads. Pass 1 counts the rows per destination; pass 2 walks the
// tokens in chunks of 1024 (one per thread) and places each (token, destination) row with
// ballots and per-warp prefix counts, so rows keep ascending token order per destination.
// Outputs: counts[d] and offs[d] (exclusive prefix, int64 for the collective's split
// sizes), rows[offs[d] + i] = the i-th token sent to d, slot[t * W + d] = that row or -1.
__global__ void __launch_bounds__(kA2AThreads) a2a_plan_kernel(const int32_t* __restrict__ idx, int rstride, int M,
                                                              int k, int E_loc, int W, int rank,
                                                              int64_t* __restrict__ counts,
                                                              int64_t* __restrict__ offs,
                                                              int32_t* __restrict__ rows,
                                                              int32_t* __restrict__ slot, int* status) {
    __shared__ int s_total[kA2AMaxWorld];
    __shared__ int s_off[kA2AMaxWorld];
    __shared__ int s_base[kA2AMaxWorld];
    __shared__ int s_warp[kA2AThreads / 32][kA2AMaxWorld];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid < kA2AMaxWorld) {
        s_total[tid] = 0;
        s_base[tid] = 0;
    }
    __syncthreads();
    // pass 1: rows per destination
    int cnt[kA2AMaxWorld];
#pragma unroll
    for (int d = 0; d < kA2AMaxWorld; ++d) cnt[d] = 0;
    for (int t = tid; t < M; t += kA2AThreads) {
        const uint32_t m = dest_mask(idx, rstride, t, k, E_loc, W, rank, status);
#pragma unroll
        for (int d = 0; d < kA2AMaxWorld; ++d) cnt[d] += (m >> d) & 1u;
    }
#pragma unroll
    for (int d = 0; d < kA2AMaxWorld; ++d) {
        int v = cnt[d];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0 && d < W && v) atomicAdd(&s_total[d], v);
    }
    __syncthreads();
    if (tid == 0) {
        int64_t run = 0;
        for (int d = 0; d < W; ++d) {
            s_off[d] = int(run);
            counts[d] = s_total[d];
            offs[d] = run;
            run += s_total[d];
        }
    }
    __syncthreads();
    // pass 2: place the rows
    const uint32_t lt = (1u << lane) - 1u;
    for (int t0 = 0; t0 < M; t0 += kA2AThreads) {
        const int t = t0 + tid;
        const uint32_t m = t < M ? dest_mask(idx, rstride, t, k, E_loc, W, rank, status) : 0u;
        uint32_t bal[kA2AMaxWorld];
#pragma unroll
        for (int d = 0; d < kA2AMaxWorld; ++d) {
            bal[d] = d < W ? __ballot_sync(0xffffffffu, (m >> d) & 1u) : 0u;
            if (lane == 0 && d < W) s_warp[warp][d] = __popc(bal[d]);
        }
        __syncthreads();
        if (tid < W) {                                 // exclusive prefix over the warps
            int run = s_base[tid];
            for (int w = 0; w < kA2AThreads / 32; ++w) {
                const int v = s_warp[w][tid];
                s_warp[w][tid] = run;
                run += v;
            }
            s_base[tid] = run;
        }
        __syncthreads();
        if (t < M) {
#pragma unroll
            for (int d = 0; d < kA2AMaxWorld; ++d) {
                if (d >= W) break;
                int pos = -1;
                if ((m >> d) & 1u) {
                    pos = s_off[d] + s_warp[warp][d] + __popc(bal[d] & lt);
                    rows[pos] = t;
                }
                slot[int64_t(t) * W + d] = pos;
            }
        }
        __syncthreads();
    }
}

// dst[i] = src[rows[i]] for rows of `words` words (16-byte words when sizes and addresses
// allow, else 4-byte words); one CTA per row at a time. A row index outside [0, n_src)
// flags the call and leaves its destination row untouched.
template <typename V>
__global__ void __launch_bounds__(256) gather_rows_kernel(const V* __restrict__ src, int64_t n_src,
                                                         const int32_t* __restrict__ rows, int64_t n,
                                                         int64_t words, V* __restrict__ dst, int* status) {
    for (int64_t r = blockIdx.x; r < n; r += gridDim.x) {
        const int s = __ldg(rows + r);
        if (s < 0 || s >= n_src) {
            if (threadIdx.x == 0) atomicExch(status, K3_ERR_INVALID);
            continue;
        }
        const V* a = src + int64_t(s) * words;
        V* b = dst + r * words;
        for (int64_t c = threadIdx.x; c < words; c += blockDim.x) b[c] = __ldcs(a + c);
    }
}

// y[t] = base[t] + sum over d = 0..W-1 of (d == rank && own ? own[t] : part[slot[t][d]])
// (rows with slot -1 skipped), in that order, in fp32; one CTA per token row at a time,
// four columns per thread. base and own are optional [M][H] fp32 (NULL: absent).
template <typename OutT>
__global__ void __launch_bounds__(256) a2a_combine_kernel(const float* __restrict__ base,
                                                         const float* __restrict__ own, int rank,
                                                         const float* __restrict__ part, int64_t n_part,
                                                         const int32_t* __restrict__ slot, int M, int W,
                                                         int64_t H, OutT* __restrict__ y, int* status) {
    for (int t = blockIdx.x; t < M; t += gridDim.x) {
        const float* src[kA2AMaxWorld + 1];
        int nsrc = 0;
        if (base) src[nsrc++] = base + int64_t(t) * H;
        for (int d = 0; d < W; ++d) {
            const int s = __ldg(slot + int64_t(t) * W + d);
            if (s < 0) continue;
            if (d == rank && own) {
                src[nsrc++] = own + int64_t(t) * H;
                continue;
            }
            if (s >= n_part) {
                if (threadIdx.x == 0) atomicExch(status, K3_ERR_INVALID);
                continue;
            }
            src[nsrc++] = part + int64_t(s) * H;
        }
        for (int64_t c = int64_t(threadIdx.x) * 4; c < H; c += int64_t(blockDim.x) * 4) {
            float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            for (int j = 0; j < nsrc; ++j) {
                const float4 v = __ldcs(reinterpret_cast<const float4*>(src[j] + c));
                acc.x += v.x;
                acc.y += v.y;
                acc.z += v.z;
                acc.w += v.w;
            }
            if constexpr (sizeof(OutT) == 4) {
                *reinterpret_cast<float4*>(reinterpret_cast<float*>(y) + int64_t(t) * H + c) = acc;
            } else {
                __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
                uint2 u;
                u.x = *reinterpret_cast<uint32_t*>(&lo);
                u.y = *reinterpret_cast<uint32_t*>(&hi);
                *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(y) + int64_t(t) * H + c) = u;
            }
        }
    }
}

// One CTA per row, at most 8 per SM (grid-stride beyond).
static int grid_for(int64_t rows) {
    const int64_t cap = int64_t(num_sms()) * 8;
    return int(rows < 1 ? 1 : (rows > cap ? cap : rows));
}

}  // namespace k3

using namespace k3;

extern "C" K3_API int k3_ep_a2a_plan(const int32_t* idx, int64_t route_stride, int64_t M, int top_k,
                                     int experts_per_rank, int world, int rank, int64_t* send_counts,
                                     int64_t* send_offs, int32_t* send_rows, int32_t* tok_slot, int32_t* status,
                                     void* stream) {
    if (!idx || !send_counts || !send_offs || !send_rows || !tok_slot || !status)
        return fail(K3_ERR_INVALID, "k3_ep_a2a_plan: NULL pointer");
    if (M < 1 || M > (int64_t(1) << 24)) return fail(K3_ERR_INVALID, "k3_ep_a2a_plan: M must be 1..2^24");
    if (top_k < 1 || route_stride < top_k) return fail(K3_ERR_INVALID, "k3_ep_a2a_plan: route_stride < top_k");
    if (world < 1 || world > kA2AMaxWorld) return fail(K3_ERR_UNSUPPORTED, "k3_ep_a2a_plan: world must be 1..32");
    if (rank < 0 || rank >= world) return fail(K3_ERR_INVALID, "k3_ep_a2a_plan: rank outside [0, world)");
    if (experts_per_rank < 1 || int64_t(experts_per_rank) * world > (int64_t(1) << 30))
        return fail(K3_ERR_INVALID, "k3_ep_a2a_plan: experts_per_rank must be >= 1");
    if (M * world > (int64_t(1) << 31) - 1) return fail(K3_ERR_INVALID, "k3_ep_a2a_plan: M * world too large");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (int rc = cuda_check(cudaMemsetAsync(status, 0, sizeof(int32_t), s), "cudaMemsetAsync(status)")) return rc;
    prof_begin(K3_PROF_OTHER, s);
    a2a_plan_kernel<<<1, kA2AThreads, 0, s>>>(idx, int(route_stride), int(M), top_k, experts_per_rank, world, rank,
                                              send_counts, send_offs, send_rows, tok_slot, status);
    prof_end(K3_PROF_OTHER, s);
    K3_CHECK_LAUNCH("a2a_plan_kernel");
    return K3_OK;
}

extern "C" K3_API int k3_ep_gather_rows(const void* src, int64_t n_src, int64_t row_bytes, const int32_t* rows,
                                        int64_t n, void* dst, int32_t* status, void* stream) {
    if (!src || !rows || !dst || !status) return fail(K3_ERR_INVALID, "k3_ep_gather_rows: NULL pointer");
    if (n < 0 || n_src < 1 || row_bytes < 4 || (row_bytes & 3))
        return fail(K3_ERR_INVALID, "k3_ep_gather_rows: row_bytes must be a positive multiple of 4");
    if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 3)
        return fail(K3_ERR_INVALID, "k3_ep_gather_rows: src and dst must be 4-byte aligned");
    if (n == 0) return K3_OK;
    if (n > (int64_t(1) << 31) - 1) return fail(K3_ERR_INVALID, "k3_ep_gather_rows: too many rows");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (int rc = cuda_check(cudaMemsetAsync(status, 0, sizeof(int32_t), s), "cudaMemsetAsync(status)")) return rc;
    const bool wide = !(row_bytes & 15) && !((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15);
    prof_begin(K3_PROF_OTHER, s);
    if (wide) {
        const int64_t words = row_bytes / 16;
        gather_rows_kernel<uint4><<<grid_for(n), 256, 0, s>>>(static_cast<const uint4*>(src), n_src, rows, n,
                                                                     words, static_cast<uint4*>(dst), status);
    } else {
        const int64_t words = row_bytes / 4;
        gather_rows_kernel<uint32_t><<<grid_for(n), 256, 0, s>>>(static_cast<const uint32_t*>(src), n_src,
                                                                        rows, n, words, static_cast<uint32_t*>(dst),
                                                                        status);
    }
    prof_end(K3_PROF_OTHER, s);
    K3_CHECK_LAUNCH("gather_rows_kernel");
    return K3_OK;
}

extern "C" K3_API int k3_ep_a2a_combine(const float* base, const float* own, int rank, const float* part,
                                        int64_t n_part, const int32_t* tok_slot, int64_t M, int world, int64_t H,
                                        void* y_out, int y_dtype, int32_t* status, void* stream) {
    if (!tok_slot || !y_out || !status) return fail(K3_ERR_INVALID, "k3_ep_a2a_combine: NULL pointer");
    if (!part && n_part > 0) return fail(K3_ERR_INVALID, "k3_ep_a2a_combine: part is NULL");
    if (M < 1 || M > (int64_t(1) << 24)) return fail(K3_ERR_INVALID, "k3_ep_a2a_combine: M must be 1..2^24");
    if (world < 1 || world > kA2AMaxWorld) return fail(K3_ERR_UNSUPPORTED, "k3_ep_a2a_combine: world must be 1..32");
    if (rank < 0 || rank >= world) return fail(K3_ERR_INVALID, "k3_ep_a2a_combine: rank outside [0, world)");
    if (H < 4 || (H & 3)) return fail(K3_ERR_INVALID, "k3_ep_a2a_combine: H must be a positive multiple of 4");
    if (y_dtype != K3_F32 && y_dtype != K3_BF16) return fail(K3_ERR_INVALID, "k3_ep_a2a_combine: y must be f32 or bf16");
    if (n_part < 0) return fail(K3_ERR_INVALID, "k3_ep_a2a_combine: n_part < 0");
    const uintptr_t a = reinterpret_cast<uintptr_t>(part) | reinterpret_cast<uintptr_t>(base) |
                        reinterpret_cast<uintptr_t>(own);
    if ((a & 15) || (reinterpret_cast<uintptr_t>(y_out) & (y_dtype == K3_F32 ? 15 : 7)))
        return fail(K3_ERR_INVALID, "k3_ep_a2a_combine: base / own / part / y_out misaligned");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (int rc = cuda_check(cudaMemsetAsync(status, 0, sizeof(int32_t), s), "cudaMemsetAsync(status)")) return rc;
    const int g = grid_for(M);
    prof_begin(K3_PROF_OTHER, s);
    if (y_dtype == K3_F32)
        a2a_combine_kernel<float><<<g, 256, 0, s>>>(base, own, rank, part, n_part, tok_slot, int(M), world, H,
                                                    static_cast<float*>(y_out), status);
    else
        a2a_combine_kernel<__nv_bfloat16><<<g, 256, 0, s>>>(base, own, rank, part, n_part, tok_slot, int(M), world,
                                                            H, static_cast<__nv_bfloat16*>(y_out), status);
    prof_end(K3_PROF_OTHER, s);
    K3_CHECK_LAUNCH("a2a_combine_kernel");
    return K3_OK;
}
