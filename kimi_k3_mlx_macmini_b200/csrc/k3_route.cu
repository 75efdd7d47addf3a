// Fused decode front end for the TMA path (sm_100a): router logits on tensor cores,
// x -> f16 pieces, and -- in the last CTA to finish -- top-k and the routing plan.
//
// Grid: ceil(E/16) row blocks x KQ k-slices (each slice a multiple of 512 k). A CTA
// computes the logits of its 16 expert rows over its k-slice with mma.m16n8k16 bf16
// (x bf16 is exact; fp32 x is split into bf16 hi + lo), its 8 warps taking equal parts
// of the slice and meeting in shared memory in warp order. Slice partials are summed
// in slice order by the last CTA of each row block to arrive, so the logits are
// deterministic; that CTA also turns its logits into the top-k's keys and sigmoid scores.
// The last row block to finish runs the top-k and builds the plan. The other CTAs
// split the expert input into E2M1 pieces (block-scaled path) or convert x to f16
// pieces.
#include "k3_route.cuh"

namespace k3 {

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// bf16 pair (hi, lo) of two floats: lo carries what bf16(v) drops.
__device__ __forceinline__ void split_bf16x2(float v0, float v1, uint32_t& hi, uint32_t& lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(v0, v1);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(v0 - hf.x, v1 - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

template <bool XF32>
__global__ void __launch_bounds__(256) route_fused_kernel(RouteArgs a) {
    __shared__ float red[8][16][kMaxTok];
    __shared__ int s_last;
    // the next launch (gate/up, a programmatic dependent that waits for this grid before
    // reading the plan) may be scheduled as soon as every CTA here is resident: its CTAs
    // set up on the SMs this grid's early finishers leave
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
    const int rb = blockIdx.x, kq = blockIdx.y;
    const int64_t slice = a.H / gridDim.y;
    const int64_t kw = slice / 8;                                 // k of one warp
    const int64_t k0 = int64_t(kq) * slice + int64_t(warp) * kw;
    const int64_t e0 = int64_t(rb) * 16 + g, e1 = e0 + 8;

    // ---- logits of 16 rows x 8 tokens over this warp's k range
    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int64_t k = k0; k < k0 + kw; k += 32) {
        const int64_t kk = k + 8 * q;
        uint4 w0 = make_uint4(0, 0, 0, 0), w1 = make_uint4(0, 0, 0, 0);
        if (e0 < a.E) w0 = __ldg(reinterpret_cast<const uint4*>(a.W + e0 * a.H + kk));
        if (e1 < a.E) w1 = __ldg(reinterpret_cast<const uint4*>(a.W + e1 * a.H + kk));
        uint32_t b[4] = {0, 0, 0, 0}, bl[4] = {0, 0, 0, 0};
        if (g < a.M) {
            if (XF32) {
                const float4* xp = reinterpret_cast<const float4*>(
                    reinterpret_cast<const float*>(a.x) + int64_t(g) * a.H + kk);
                const float4 x0 = __ldg(xp), x1 = __ldg(xp + 1);
                split_bf16x2(x0.x, x0.y, b[0], bl[0]);
                split_bf16x2(x0.z, x0.w, b[1], bl[1]);
                split_bf16x2(x1.x, x1.y, b[2], bl[2]);
                split_bf16x2(x1.z, x1.w, b[3], bl[3]);
            } else {
                const uint4 xv = __ldg(reinterpret_cast<const uint4*>(
                    reinterpret_cast<const uint16_t*>(a.x) + int64_t(g) * a.H + kk));
                b[0] = xv.x;
                b[1] = xv.y;
                b[2] = xv.z;
                b[3] = xv.w;
            }
        }
        // k-pair permutation shared by A and B: step 0 uses elements 8q..8q+3, step 1 8q+4..8q+7
        mma_bf16_16816(d, w0.x, w1.x, w0.y, w1.y, b[0], b[1]);
        mma_bf16_16816(d, w0.z, w1.z, w0.w, w1.w, b[2], b[3]);
        if (XF32) {
            mma_bf16_16816(d, w0.x, w1.x, w0.y, w1.y, bl[0], bl[1]);
            mma_bf16_16816(d, w0.z, w1.z, w0.w, w1.w, bl[2], bl[3]);
        }
    }
    red[warp][g][2 * q] = d[0];
    red[warp][g][2 * q + 1] = d[1];
    red[warp][g + 8][2 * q] = d[2];
    red[warp][g + 8][2 * q + 1] = d[3];

    // ---- expert input -> pieces, off the router's critical path: every CTA but the one that
    // ends up running the top-k and plan claims (token, 32-block) tasks in batches of 4 from
    // a counter after its last duty in the logits -> top-k chain (the next kernels read the
    // pieces only after this launch completes)
    auto do_pieces = [&]() {
        if (a.xp) {
            const void* xe = a.xe ? a.xe : a.x;
            const int xedt = a.xe ? a.xe_dtype : a.x_dtype;
            const int64_t He = a.xe ? a.He : a.H;
            const uint32_t ng = uint32_t(He / 32);
            const uint32_t ntask = uint32_t(a.M) * ng;
            unsigned* claim = a.done + 1 + gridDim.x;
            for (;;) {
                unsigned t0 = 0;
                if (lane == 0) t0 = atomicAdd(claim, 4u);
                t0 = __shfl_sync(0xffffffffu, t0, 0);
                if (t0 >= ntask) break;
                // the four claimed (token, 32-block) tasks split as four interleaved chains
                float v[4];
                uint8_t* d[4];
                uint8_t* sf[4];
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    const uint32_t task = min(t0 + uint32_t(h), ntask - 1u);
                    const uint32_t t = task / ng, g = task - t * ng;
                    v[h] = load_as_f32(xe, xedt, int64_t(t) * He + 32 * int64_t(g) + lane);
                    d[h] = a.xp + int64_t(kBPieces * t) * (He / 2) + 16 * int64_t(g);
                    sf[h] = t0 + uint32_t(h) < ntask ? a.xsf + int64_t(kBPieces * t) * ng + g : nullptr;
                }
                split_pieces_n<4>(v, lane, d, He / 2, sf, int64_t(ng));
            }
        } else {
            // ---- x -> f16 pieces: the CTAs of the first row blocks split the slice's 512-blocks
            const int64_t nb = slice / 512, b0 = int64_t(kq) * nb;
            for (int64_t j = rb; j < nb; j += gridDim.x)
                convert_block(a.x, a.x_dtype, a.M, a.H, warp, b0 + j, a.xq_hi, a.xq_lo, a.xq_ts, lane);
        }
    };
    __syncthreads();
    const int64_t n_rb = gridDim.x;
    if (threadIdx.x < 16 * kMaxTok) {
        const int r = threadIdx.x / kMaxTok, t = threadIdx.x % kMaxTok;
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; ++w) v += red[w][r][t];
        const int64_t e = int64_t(rb) * 16 + r;
        if (e < a.E && t < a.M) a.logit_part[(int64_t(kq) * a.M + t) * a.E + e] = v;
    }
    __threadfence();
    __syncthreads();
    // ---- the last slice CTA of this row block sums the slices (in slice order)
    if (threadIdx.x == 0) s_last = (atomicAdd(a.done + 1 + rb, 1u) + 1 == gridDim.y);
    __syncthreads();
    if (!s_last) {
        do_pieces();
        return;
    }
    __threadfence();
    if (threadIdx.x < 16 * kMaxTok) {
        const int r = threadIdx.x / kMaxTok, t = threadIdx.x % kMaxTok;
        const int64_t e = int64_t(rb) * 16 + r;
        if (e < a.E && t < a.M) {
            // every slice's partial in flight at once, summed in slice order
            constexpr int kMaxSlices = 16;
            float pv[kMaxSlices];
#pragma unroll
            for (int s = 0; s < kMaxSlices; ++s)
                pv[s] = s < int(gridDim.y) ? __ldcg(a.logit_part + (int64_t(s) * a.M + t) * a.E + e) : 0.0f;
            float v = 0.0f;
#pragma unroll
            for (int s = 0; s < kMaxSlices; ++s)
                if (s < int(gridDim.y)) v += pv[s];
            const int64_t o = int64_t(t) * a.E + e;
            a.logits[o] = v;
            // the top-k's inputs, here where 16 x M threads per row block compute them in
            // parallel instead of in the one CTA that runs the selection: raw = sigmoid,
            // key of raw + bias (moe.py:65-76)
            const float raw = 1.0f / (1.0f + expf(-v));
            const float* bias = a.plan_args.bias;
            a.plan_args.keys[o] = order_key(raw + (bias ? __ldg(bias + e) : 0.0f));
            a.plan_args.scores[o] = raw;
        }
    }
    __threadfence();
    __syncthreads();
    // ---- the last row block: top-k and plan
    if (threadIdx.x == 0) s_last = (atomicAdd(a.done, 1u) + 1 == unsigned(n_rb));
    __syncthreads();
    if (!s_last) {
        do_pieces();
        return;
    }
    __threadfence();
    extern __shared__ uint32_t s_key[];                      // M * E top-k keys
    build_plan_cta<true>(a.plan_args, nullptr, warp, lane, s_key);
    do_pieces();                                             // whatever the others left
}

int launch_route_fused(const RouteArgs& a, int kq, cudaStream_t s) {
    const dim3 grid(unsigned((a.E + 15) / 16), unsigned(kq));
    const size_t keys = sizeof(uint32_t) * size_t(a.M) * size_t(a.E);     // <= 32 KiB
    if (a.x_dtype == K3_F32)
        route_fused_kernel<true><<<grid, 256, keys, s>>>(a);
    else
        route_fused_kernel<false><<<grid, 256, keys, s>>>(a);
    K3_CHECK_LAUNCH("route_fused_kernel");
    return K3_OK;
}

}  // namespace k3
