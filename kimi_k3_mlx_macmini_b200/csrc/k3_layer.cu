// The MoE input of a Kimi-K3 decoder layer (air_llm/models/kimi_k3/layer.py:120-121):
//
//   x = rmsnorm(apply_attn_res(prefix_sum, block_residual, mlp_res_proj, mlp_res_norm),
//               post_attention_layernorm)
//
// apply_attn_res (ops.py:61-74) is a softmax over the block checkpoints plus the running
// sum: every vector v_b (b < B: block_residual[n][b], b = B: prefix_sum[n]) is scored by
// sum_h (v_b[h] * rsqrt(mean(v_b^2) + eps)) * res_norm[h] * res_proj[h], and the output
// is sum_b softmax(score)_b * v_b. One CTA per token: one pass over the B + 1 vectors
// for their sums of squares and score dots (registers, then a block reduction), the
// softmax, a second pass for the weighted sum (kept in shared memory) and its sum of
// squares, and a third that writes post_norm * (x * rsqrt(mean(x^2) + eps)).
#include <algorithm>

#include "k3_common.cuh"

namespace k3 {
namespace {

constexpr int kARThreads = 512;
constexpr int kARMaxVec = 17;          // up to 16 block checkpoints + the running sum

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();                     // red may still be read by a previous reduction
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.0f;
    for (int i = 0; i < kARThreads / 32; ++i) t += red[i];
    return t;
}

template <int NV>
__global__ void __launch_bounds__(kARThreads) attn_res_norm_kernel(const float* __restrict__ ps,
                                                                  const float* __restrict__ br, int nb, int64_t H,
                                                                  const float* __restrict__ proj,
                                                                  const float* __restrict__ rnorm,
                                                                  const float* __restrict__ pnorm, float eps,
                                                                  void* out, int out_dtype) {
    extern __shared__ float xs[];        // [H] the weighted sum
    __shared__ float red[kARThreads / 32];
    __shared__ float prob[kARMaxVec];
    const int64_t n = blockIdx.x;
    const int nv = nb + 1;
    auto vec = [&](int b) { return b < nb ? br + (n * nb + b) * H : ps + n * H; };

    float ss[NV], dot[NV];
#pragma unroll
    for (int b = 0; b < NV; ++b) ss[b] = dot[b] = 0.0f;
    for (int64_t h = threadIdx.x; h < H; h += kARThreads) {
        const float sw = rnorm[h] * proj[h];
#pragma unroll
        for (int b = 0; b < NV; ++b)
            if (b < nv) {
                const float v = vec(b)[h];
                ss[b] = fmaf(v, v, ss[b]);
                dot[b] = fmaf(v, sw, dot[b]);
            }
    }
    float score[NV];
#pragma unroll
    for (int b = 0; b < NV; ++b)
        if (b < nv) {
            const float s2 = block_sum(ss[b], red);
            const float d = block_sum(dot[b], red);
            score[b] = d * rsqrtf(s2 / float(H) + eps);
        }
    if (threadIdx.x == 0) {
        float mx = -INFINITY;
        for (int b = 0; b < nv; ++b) mx = fmaxf(mx, score[b]);
        float z = 0.0f;
        for (int b = 0; b < nv; ++b) z += (prob[b] = expf(score[b] - mx));
        for (int b = 0; b < nv; ++b) prob[b] /= z;
    }
    __syncthreads();
    float sx = 0.0f;
    for (int64_t h = threadIdx.x; h < H; h += kARThreads) {
        float x = 0.0f;
#pragma unroll
        for (int b = 0; b < NV; ++b)
            if (b < nv) x = fmaf(prob[b], vec(b)[h], x);
        xs[h] = x;
        sx = fmaf(x, x, sx);
    }
    const float r = rsqrtf(block_sum(sx, red) / float(H) + eps);
    for (int64_t h = threadIdx.x; h < H; h += kARThreads)
        store_from_f32(out, out_dtype, n * H + h, pnorm[h] * (xs[h] * r));
}

template <int NV>
void launch_ar(const float* ps, const float* br, int nb, int64_t N, int64_t H, const float* proj, const float* rn,
               const float* pn, float eps, void* out, int odt, cudaStream_t s) {
    attn_res_norm_kernel<NV><<<unsigned(N), kARThreads, sizeof(float) * size_t(H), s>>>(ps, br, nb, H, proj, rn, pn,
                                                                                        eps, out, odt);
}

}  // namespace
}  // namespace k3

using namespace k3;

extern "C" K3_API int k3_attn_res_norm(const float* prefix_sum, const float* block_residual, int64_t n_blocks,
                                       int64_t N, int64_t H, const float* res_proj, const float* res_norm,
                                       const float* post_norm, float eps, void* out, int out_dtype, void* stream) {
    if (!prefix_sum || !res_proj || !res_norm || !post_norm || !out)
        return fail(K3_ERR_INVALID, "k3_attn_res_norm: NULL tensor");
    if (n_blocks < 0 || n_blocks > kARMaxVec - 1)
        return fail(K3_ERR_UNSUPPORTED, "k3_attn_res_norm: at most 16 block checkpoints");
    if (n_blocks > 0 && !block_residual) return fail(K3_ERR_INVALID, "k3_attn_res_norm: block_residual is NULL");
    if (N < 1 || N > (int64_t(1) << 31) - 1) return fail(K3_ERR_INVALID, "k3_attn_res_norm: N out of range");
    if (H < 1 || H > 48 * 1024) return fail(K3_ERR_UNSUPPORTED, "k3_attn_res_norm: H must be 1..49152");
    if (out_dtype != K3_F32 && out_dtype != K3_BF16) return fail(K3_ERR_INVALID, "k3_attn_res_norm: out must be f32 or bf16");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t smem = sizeof(float) * size_t(H);
    if (smem > 48 * 1024) {
        static OncePerContext attr[2];
        const int i = n_blocks < 8 ? 0 : 1;
        if (int rc = attr[i].run([&] {
                return i == 0 ? cuda_check(cudaFuncSetAttribute(attn_res_norm_kernel<8>,
                                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                                48 * 1024 * 4),
                                           "cudaFuncSetAttribute(attn_res_norm)")
                              : cuda_check(cudaFuncSetAttribute(attn_res_norm_kernel<kARMaxVec>,
                                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                                48 * 1024 * 4),
                                           "cudaFuncSetAttribute(attn_res_norm)");
            }))
            return rc;
    }
    if (n_blocks < 8)
        launch_ar<8>(prefix_sum, block_residual, int(n_blocks), N, H, res_proj, res_norm, post_norm, eps, out,
                     out_dtype, s);
    else
        launch_ar<kARMaxVec>(prefix_sum, block_residual, int(n_blocks), N, H, res_proj, res_norm, post_norm, eps, out,
                             out_dtype, s);
    K3_CHECK_LAUNCH("attn_res_norm_kernel");
    return K3_OK;
}
