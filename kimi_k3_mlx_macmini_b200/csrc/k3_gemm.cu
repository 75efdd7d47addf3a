// Dense GEMM on the 5th-generation tensor cores (tcgen05 kind::f16, sm_100a):
// out[m][n] (+)= sum_k X[m][k] * W[n][k] with bf16 W and bf16 X, fp32 accumulation in TMEM.
// fp32 X enters as two bf16 pieces (hi = bf16(x), lo = bf16(x - hi)), both multiplied by
// the same W tile into the same accumulator, which keeps ~16 significant bits of x.
//
// It serves two callers: the prefill router's logits (x bf16 [T][H] . W_gate [E][H]^T,
// one piece) and the dense projections of a Kimi-K3 layer above 8 tokens (latent
// down/up, shared expert; fp32 inputs, air_llm/models/kimi_k3/moe.py:105-131).
//
// One CTA per (128 rows of W, 96 rows of X) output tile; 6 warps: TMA producer (W tile and
// the X piece tiles per 64-k stage, 128-byte swizzle), MMA issuer (one elected lane, 4
// MMAs of k = 16 per stage and piece), 4 epilogue warps (TMEM lane quarter each). The k
// order is fixed, so results are deterministic; every wait is bounded.
#include "k3_async.cuh"
#include "k3_gemm.cuh"
#include "k3_tma.cuh"

namespace k3 {

namespace {

// Instruction descriptor of kind::f16: bf16 x bf16 -> fp32, M = 128, N = n, both K-major.
__device__ __forceinline__ uint32_t bf16_idesc(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(128 >> 4) << 24);
}
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

constexpr int kGN = 96;            // X rows per CTA (MMA N)
constexpr int kGThreads = 192;     // producer, MMA, 4 epilogue warps

template <bool XLO>
struct alignas(1024) GStage {
    uint8_t a[kBRows][128];        // 128 W rows x 64 k (bf16), SW128
    uint8_t b[XLO ? 2 : 1][kGN][128];  // X piece tiles: kGN rows x 64 k
};
template <bool XLO>
constexpr int gstages() { return XLO ? 5 : 6; }
template <bool XLO>
constexpr size_t gsmem_bytes() { return sizeof(GStage<XLO>) * gstages<XLO>() + 1024 + 256; }
static_assert(gsmem_bytes<true>() <= 227 * 1024 && gsmem_bytes<false>() <= 227 * 1024,
              "GEMM ring exceeds shared memory");

struct GArgs {
    int M, N;
    int64_t K;
    float* out;
    int64_t ldo;
    int accumulate;          // out += instead of out =
    int* status;
};

template <bool XLO>
__global__ void __launch_bounds__(kGThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                     const __grid_constant__ CUtensorMap xlmap, const GArgs g) {
    using St = GStage<XLO>;
    constexpr int S = gstages<XLO>();
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    St* ring = reinterpret_cast<St*>(base);
    uint64_t* full = reinterpret_cast<uint64_t*>(base + sizeof(St) * S);
    uint64_t* empty = full + S;
    uint64_t* accf = empty + S;
    uint64_t* drain = accf + 1;
    __shared__ uint32_t s_tmem;
    __shared__ volatile int s_abort;
    __shared__ volatile unsigned s_issued;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        prefetch_tensormap(&wmap);
        prefetch_tensormap(&xmap);
        if (XLO) prefetch_tensormap(&xlmap);
        s_abort = 0;
        s_issued = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accf, 1);
        mbar_init(drain, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (warp == 1) tmem_alloc(&s_tmem, 128);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = s_tmem;
    const int n0 = blockIdx.x * kBRows, m0 = blockIdx.y * kGN;
    const int nst = int(g.K / 64);

    if (warp == 0) {
        if (lane == 0) {
            for (int s = 0; s < nst; ++s) {
                const int si = s % S;
                if (!mbar_wait(&empty[si], ((s / S) & 1) ^ 1, g.status, &s_abort)) {
                    s_abort = 1;
                    break;
                }
                mbar_expect_tx(&full[si], uint32_t(sizeof(St)));
                tma_2d(&ring[si].a[0][0], &wmap, 64 * s, n0, &full[si]);
                tma_2d(&ring[si].b[0][0][0], &xmap, 64 * s, m0, &full[si]);
                if (XLO) tma_2d(&ring[si].b[XLO ? 1 : 0][0][0], &xlmap, 64 * s, m0, &full[si]);
                s_issued = unsigned(s + 1);
            }
        }
    } else if (warp == 1) {
        const uint32_t idesc = bf16_idesc(kGN);
        int s = 0;
        for (; s < nst; ++s) {
            const int si = s % S;
            if (!__all_sync(0xffffffffu, mbar_wait(&full[si], (s / S) & 1, g.status, &s_abort))) {
                s_abort = 1;
                break;
            }
            tc_fence_after();
            if (elect_one()) {
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint64_t ad = sw128_desc(&ring[si].a[0][0], 32 * kk);
                    mma_bf16(tm, ad, sw128_desc(&ring[si].b[0][0][0], 32 * kk), idesc, (s > 0 || kk > 0) ? 1u : 0u);
                    if (XLO) mma_bf16(tm, ad, sw128_desc(&ring[si].b[XLO ? 1 : 0][0][0], 32 * kk), idesc, 1u);
                }
                tc_commit(&empty[si]);
            }
            __syncwarp();
        }
        if (s == nst) {
            if (elect_one()) tc_commit(accf);
            __syncwarp();
        } else {
            // the producer's copies in flight land before the CTA leaves
            const unsigned issued = s_issued;
            for (unsigned k = unsigned(s); k < issued; ++k)
                if (!mbar_wait(&full[k % S], (k / S) & 1, g.status)) break;
        }
        if (elect_one()) tc_commit(drain);
        __syncwarp();
        mbar_wait(drain, 0, g.status);
    } else {
        const int q = warp & 3;
        if (__all_sync(0xffffffffu, mbar_wait(accf, 0, g.status, &s_abort))) {
            tc_fence_after();
            const int n = n0 + 32 * q + lane;
            const uint32_t taddr = tm + (uint32_t(32 * q) << 16);
#pragma unroll 1
            for (int j0 = 0; j0 < kGN; j0 += 16) {
                float v[16];
                tmem_ld16(taddr + j0, v);
#pragma unroll
                for (int jj = 0; jj < 16; ++jj) {
                    const int m = m0 + j0 + jj;
                    if (m < g.M && n < g.N) {
                        float* o = g.out + int64_t(m) * g.ldo + n;
                        *o = g.accumulate ? *o + v[jj] : v[jj];
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tm, 128);
    }
}

// x (f32 or bf16, row stride ldx) -> hi = bf16(x), lo = bf16(x - hi), both [M][K].
__global__ void __launch_bounds__(256) split_bf16_kernel(const void* __restrict__ x, int x_dtype, int64_t ldx,
                                                         int64_t M, int64_t K, __nv_bfloat16* __restrict__ hi,
                                                         __nv_bfloat16* __restrict__ lo) {
    const int64_t n = M * K;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t m = i / K, k = i - m * K;
        const float v = load_as_f32(x, x_dtype, m * ldx + k);
        const __nv_bfloat16 h = __float2bfloat16_rn(v);
        hi[i] = h;
        lo[i] = __float2bfloat16_rn(v - __bfloat162float(h));
    }
}

OncePerContext g_gemm_attr;

int map_rows(CUtensorMap* m, const void* base, int64_t rows, int64_t K, int64_t ld, int box_rows) {
    const uint64_t d[2] = {uint64_t(K), uint64_t(rows)};
    const uint64_t st[1] = {uint64_t(ld) * 2};
    const uint32_t b[2] = {64, uint32_t(box_rows)};
    return encode_map(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, d, st, b, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace

bool gemm_bf16_ok(int64_t K, const void* w, int64_t ldw, const void* x, int64_t ldx) {
    return K % 64 == 0 && K > 0 && ldw % 8 == 0 && ldx % 8 == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(x) & 15) == 0;
}

int launch_gemm_bf16(const uint16_t* xh, const uint16_t* xl, int64_t ldx, int64_t M, int64_t K, const uint16_t* w,
                     int64_t ldw, int64_t N, float* out, int64_t ldo, int accumulate, int* status, cudaStream_t s) {
    if (int rc = g_gemm_attr.run([] {
            if (int rc2 = cuda_check(cudaFuncSetAttribute(gemm_bf16_kernel<true>,
                                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                          int(gsmem_bytes<true>())),
                                     "cudaFuncSetAttribute(gemm_bf16 hi+lo)"))
                return rc2;
            return cuda_check(cudaFuncSetAttribute(gemm_bf16_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   int(gsmem_bytes<false>())),
                              "cudaFuncSetAttribute(gemm_bf16)");
        }))
        return rc;
    CUtensorMap wmap, xmap, xlmap;
    if (int rc = map_rows(&wmap, w, N, K, ldw, kBRows)) return rc;
    if (int rc = map_rows(&xmap, xh, M, K, ldx, kGN)) return rc;
    if (xl) {
        if (int rc = map_rows(&xlmap, xl, M, K, ldx, kGN)) return rc;
    } else {
        xlmap = xmap;
    }
    GArgs g{int(M), int(N), K, out, ldo, accumulate, status};
    const dim3 grid(unsigned((N + kBRows - 1) / kBRows), unsigned((M + kGN - 1) / kGN));
    if (xl)
        gemm_bf16_kernel<true><<<grid, kGThreads, gsmem_bytes<true>(), s>>>(wmap, xmap, xlmap, g);
    else
        gemm_bf16_kernel<false><<<grid, kGThreads, gsmem_bytes<false>(), s>>>(wmap, xmap, xlmap, g);
    K3_CHECK_LAUNCH("gemm_bf16_kernel");
    return K3_OK;
}

}  // namespace k3

using namespace k3;

extern "C" K3_API size_t k3_dense_gemm_workspace(int64_t M, int64_t K) {
    if (M < 1 || K < 1) return 0;
    return align_up(256 + 2 * size_t(M) * size_t(K) * 2, 256) + 256;
}

extern "C" K3_API int k3_dense_gemm(const void* x, int x_dtype, int64_t ldx, int64_t M, int64_t K, const uint16_t* w,
                                    int64_t ldw, int64_t N, float* out, int64_t ldo, int accumulate, void* workspace,
                                    size_t workspace_bytes, void* stream) {
    if (!x || !w || !out) return fail(K3_ERR_INVALID, "k3_dense_gemm: NULL tensor");
    if (x_dtype != K3_F32 && x_dtype != K3_BF16) return fail(K3_ERR_INVALID, "k3_dense_gemm: x must be f32 or bf16");
    if (M < 1 || N < 1 || K < 1 || ldx < K || ldw < K || ldo < N)
        return fail(K3_ERR_INVALID, "k3_dense_gemm: need M, N, K >= 1, ldx, ldw >= K and ldo >= N");
    if (K % 64 || ldw % 8 || (reinterpret_cast<uintptr_t>(w) & 15))
        return fail(K3_ERR_UNSUPPORTED, "k3_dense_gemm: K must be a multiple of 64 and W rows 16-byte aligned");
    if (M > (int64_t(1) << 31) - 1 || N > (int64_t(1) << 31) - 1)
        return fail(K3_ERR_UNSUPPORTED, "k3_dense_gemm: M and N must fit 31 bits");
    const size_t need = k3_dense_gemm_workspace(M, K);
    if (!workspace) return fail(K3_ERR_WORKSPACE, "k3_dense_gemm: workspace is NULL");
    if (reinterpret_cast<uintptr_t>(workspace) % 256) return fail(K3_ERR_WORKSPACE, "k3_dense_gemm: workspace must be 256-byte aligned");
    if (workspace_bytes < need) return fail(K3_ERR_WORKSPACE, "k3_dense_gemm: workspace too small: need " + std::to_string(need));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    int* status = reinterpret_cast<int*>(ws);
    if (int rc = cuda_check(cudaMemsetAsync(status, 0, sizeof(int), s), "k3_dense_gemm status")) return rc;
    const uint16_t* xh = static_cast<const uint16_t*>(x);
    const uint16_t* xl = nullptr;
    int64_t ld = ldx;
    if (x_dtype == K3_F32 || ldx % 8 || (reinterpret_cast<uintptr_t>(x) & 15)) {
        // fp32 rows (or bf16 rows TMA cannot address): hi and lo bf16 pieces, [M][K]
        __nv_bfloat16* hi = reinterpret_cast<__nv_bfloat16*>(ws + 256);
        __nv_bfloat16* lo = hi + M * K;
        const int blocks = int(std::min<int64_t>((M * K + 255) / 256, int64_t(num_sms()) * 8));
        split_bf16_kernel<<<blocks, 256, 0, s>>>(x, x_dtype, ldx, M, K, hi, lo);
        K3_CHECK_LAUNCH("split_bf16_kernel");
        xh = reinterpret_cast<const uint16_t*>(hi);
        xl = x_dtype == K3_F32 ? reinterpret_cast<const uint16_t*>(lo) : nullptr;
        ld = K;
    }
    prof_begin(K3_PROF_DENSE, s);
    const int rc = launch_gemm_bf16(xh, xl, ld, M, K, w, ldw, N, out, ldo, accumulate, status, s);
    prof_end(K3_PROF_DENSE, s);
    return rc;
}
