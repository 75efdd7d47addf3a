// MXFP4 codec kernels: full dequantisation (bit-exact), scale range reduction, and
// the generic CUDA-core matvec used for shapes the grouped-matvec path does not tile.
#include <algorithm>

#include "k3_common.cuh"

namespace k3 {

__constant__ float kE2M1[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};

// Exact 2**(b-127) for every byte, including the subnormal 2**-127 (b = 0) and
// +inf (b = 255) -- numpy's ldexp in the reference decoder (mxfp4.py:34).
__device__ __forceinline__ float e8m0_exact(uint32_t b) {
    return b == 0 ? __uint_as_float(0x00400000u) : __uint_as_float(b << 23);
}

__device__ __forceinline__ float e2m1_value(uint32_t code) {
    const float m = kE2M1[code & 7];
    return (code & 8) ? -m : m;
}

// One thread per packed byte pair (4 outputs); rows x cols/2 bytes in total.
template <int ODT>
__global__ void dequant_kernel(const uint8_t* __restrict__ packed, const uint8_t* __restrict__ scales,
                               int64_t rows, int64_t cols, void* __restrict__ out) {
    const int64_t half = cols / 2;
    const int64_t n = rows * half;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = i / half, cb = i % half;
        const uint32_t b = packed[i];
        const float s = e8m0_exact(scales[r * (cols / 32) + (2 * cb) / 32]);
        const float v0 = e2m1_value(b & 15) * s, v1 = e2m1_value(b >> 4) * s;
        const int64_t o = r * cols + 2 * cb;
        if (ODT == K3_BF16) {
            __nv_bfloat162 h;
            h.x = __float2bfloat16_rn(v0);
            h.y = __float2bfloat16_rn(v1);
            reinterpret_cast<__nv_bfloat162*>(out)[o / 2] = h;
        } else {
            reinterpret_cast<float2*>(out)[o / 2] = make_float2(v0, v1);
        }
    }
}

__global__ void minmax_kernel(const uint8_t* __restrict__ s, int64_t n, int32_t* out) {
    int lo = 255, hi = 0;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += int64_t(gridDim.x) * blockDim.x) {
        const int v = s[i];
        lo = min(lo, v);
        hi = max(hi, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
        hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
    if ((threadIdx.x & 31) == 0) {
        atomicMin(out, lo);
        atomicMax(out + 1, hi);
    }
}

__global__ void minmax_init_kernel(int32_t* out) {
    out[0] = 255;
    out[1] = 0;
}

// Generic matvec: one warp per (row n, chunk of 8 tokens); lanes walk the packed row,
// fp32 fma per element, xor-tree reduction. Any K % 32 == 0, any N, any M.
__global__ void __launch_bounds__(256) matvec_simple_kernel(const void* __restrict__ x, int xdt,
                                                            int64_t M, int64_t K,
                                                            const uint8_t* __restrict__ packed,
                                                            const uint8_t* __restrict__ scales,
                                                            int64_t N, void* __restrict__ out,
                                                            int odt) {
    const int64_t w = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t chunks = (M + 7) / 8;
    if (w >= N * chunks) return;
    const int64_t n = w / chunks, m0 = (w % chunks) * 8;
    const int mc = int((M - m0) < 8 ? (M - m0) : 8);
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const uint8_t* prow = packed + n * (K / 2);
    const uint8_t* srow = scales + n * (K / 32);
    for (int64_t kb = lane; kb < K / 2; kb += 32) {
        const uint32_t b = prow[kb];
        const float s = __uint_as_float(uint32_t(srow[(2 * kb) / 32]) << 23);
        const float v0 = e2m1_value(b & 15) * s, v1 = e2m1_value(b >> 4) * s;
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            if (m < mc) {
                const int64_t xi = (m0 + m) * K + 2 * kb;
                acc[m] = fmaf(load_as_f32(x, xdt, xi), v0, acc[m]);
                acc[m] = fmaf(load_as_f32(x, xdt, xi + 1), v1, acc[m]);
            }
        }
    }
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        if (m < mc) {
            const float v = warp_sum(acc[m]);
            if (lane == 0) store_from_f32(out, odt, (m0 + m) * N + n, v);
        }
    }
}

int launch_matvec_simple(const void* x, int xdt, int64_t M, int64_t K, const uint8_t* packed,
                         const uint8_t* scales, int64_t N, void* out, int odt, cudaStream_t s) {
    const int64_t warps = N * ((M + 7) / 8);
    const int64_t blocks = (warps * 32 + 255) / 256;
    if (blocks > 0x7fffffff) return fail(K3_ERR_UNSUPPORTED, "matvec too large for the generic kernel");
    prof_begin(K3_PROF_OTHER, s);
    matvec_simple_kernel<<<unsigned(blocks), 256, 0, s>>>(x, xdt, M, K, packed, scales, N, out, odt);
    prof_end(K3_PROF_OTHER, s);
    K3_CHECK_LAUNCH("matvec_simple_kernel");
    return K3_OK;
}

}  // namespace k3

using namespace k3;

extern "C" K3_API int k3_mxfp4_dequant(const uint8_t* packed, const uint8_t* scales, int64_t rows,
                                       int64_t cols, int group_size, void* out, int out_dtype,
                                       void* stream) {
    if (!packed || !scales || !out) return fail(K3_ERR_INVALID, "k3_mxfp4_dequant: NULL tensor");
    if (group_size != 32) return fail(K3_ERR_UNSUPPORTED, "k3_mxfp4_dequant: group_size must be 32");
    if (rows < 0 || cols < 0 || cols % 32) return fail(K3_ERR_INVALID, "k3_mxfp4_dequant: cols must be a multiple of 32");
    if (out_dtype != K3_F32 && out_dtype != K3_BF16) return fail(K3_ERR_INVALID, "k3_mxfp4_dequant: out must be f32 or bf16");
    if (rows == 0 || cols == 0) return K3_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t n = rows * cols / 2;
    const int blocks = int(std::min<int64_t>((n + 255) / 256, int64_t(num_sms()) * 16));
    prof_begin(K3_PROF_OTHER, s);
    if (out_dtype == K3_BF16)
        dequant_kernel<K3_BF16><<<blocks, 256, 0, s>>>(packed, scales, rows, cols, out);
    else
        dequant_kernel<K3_F32><<<blocks, 256, 0, s>>>(packed, scales, rows, cols, out);
    prof_end(K3_PROF_OTHER, s);
    K3_CHECK_LAUNCH("dequant_kernel");
    return K3_OK;
}

extern "C" K3_API int k3_mxfp4_scale_minmax(const uint8_t* scales, int64_t n, int32_t* minmax_out,
                                            void* stream) {
    if (!scales || !minmax_out) return fail(K3_ERR_INVALID, "k3_mxfp4_scale_minmax: NULL tensor");
    if (n < 1) return fail(K3_ERR_INVALID, "k3_mxfp4_scale_minmax: empty tensor");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    minmax_init_kernel<<<1, 1, 0, s>>>(minmax_out);
    K3_CHECK_LAUNCH("minmax_init_kernel");
    const int blocks = int(std::min<int64_t>((n + 255) / 256, int64_t(num_sms()) * 8));
    minmax_kernel<<<blocks, 256, 0, s>>>(scales, n, minmax_out);
    K3_CHECK_LAUNCH("minmax_kernel");
    return K3_OK;
}
