// Shared device/host helpers for the k3b200 library (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <string>
#include <utility>

#include "../../include/k3b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "k3b200 targets sm_100a (B200) only"
#endif

namespace k3 {

// ------------------------------------------------------------------ host errors

// Records `msg` as the calling thread's last error and returns `code`.
int fail(int code, const std::string& msg);
// Maps a CUDA error to K3_ERR_CUDA with context; K3_OK when e == cudaSuccess.
int cuda_check(cudaError_t e, const char* what);
int num_sms();
// Kernel timing diagnostics: no-ops unless k3_profile_enable(1) was called.
void prof_begin(int kind, cudaStream_t s);
void prof_end(int kind, cudaStream_t s);

#define K3_CHECK_LAUNCH(what)                                              \
    do {                                                                   \
        int _rc = ::k3::cuda_check(cudaGetLastError(), what);              \
        if (_rc != K3_OK) return _rc;                                      \
    } while (0)

constexpr int kMaxDevices = 64;

// The current device and the id of its current context. Function attributes and the
// device address of a __device__ array belong to a context: a cudaDeviceReset (or a
// primary context released and created again) gives the device a new context and a new
// id, and what was set up for the old one is gone. *ctx_id is 0 while the device has no
// context yet (nothing has run on it in this process).
int current_context(int* dev, unsigned long long* ctx_id);

// Runs a set-up step (cudaFuncSetAttribute and the like) once for every context it is
// called under: each device of a process that drives several GPUs, and again after a
// device's context was replaced. Thread-safe; a failed step is retried by the next call.
class OncePerContext {
public:
    template <class F>
    int run(F&& fn) {
        int dev = -1;
        unsigned long long id = 0;
        if (int rc = current_context(&dev, &id)) return rc;
        std::lock_guard<std::mutex> g(mu_);
        if (id != 0 && done_[dev] == id) return K3_OK;
        if (int rc = fn()) return rc;
        if (id == 0)                                  // fn() created the context
            if (int rc = current_context(&dev, &id)) return rc;
        done_[dev] = id;
        return K3_OK;
    }

private:
    std::mutex mu_;
    unsigned long long done_[kMaxDevices] = {};       // context id the step ran under
};

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Launches `kernel` as a programmatic dependent launch of the previous work on `s`: it
// may begin while that kernel finishes and must execute griddepcontrol.wait before it
// reads anything that kernel writes.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// -------------------------------------------------------------- device helpers

// E8M0 byte -> fp32 2**(b-127) by placing the byte in the exponent field. Exact for
// 1..254 (byte 0 gives +0, byte 255 +inf); the callers' host API rejects 0/255 ranges.
__device__ __forceinline__ float e8m0_to_f32(uint32_t b) { return __uint_as_float(b << 23); }

// Four bytes (eight E2M1 codes) -> four f16x2: byte j of w becomes register j, its low
// nibble (the even element) in the low half. Hardware conversion (sm_100a).
__device__ __forceinline__ void e2m1x8_to_f16x8(uint32_t w, uint32_t& d0, uint32_t& d1,
                                                uint32_t& d2, uint32_t& d3) {
    asm("{\n"
        " .reg .b8 b0, b1, b2, b3;\n"
        " mov.b32 {b0, b1, b2, b3}, %4;\n"
        " cvt.rn.f16x2.e2m1x2 %0, b0;\n"
        " cvt.rn.f16x2.e2m1x2 %1, b1;\n"
        " cvt.rn.f16x2.e2m1x2 %2, b2;\n"
        " cvt.rn.f16x2.e2m1x2 %3, b3;\n"
        "}\n"
        : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
        : "r"(w));
}

// D += A(16x16 f16, row) * B(16x8 f16, col), fp32 accumulate (PTX mma.m16n8k16).
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1,
                                              uint32_t a2, uint32_t a3, uint32_t b0,
                                              uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D = A * B with a zero accumulator input (starts a fresh partial sum without
// clearing registers first).
__device__ __forceinline__ void mma_f16_16816_zc(float (&d)[4], uint32_t a0, uint32_t a1,
                                                 uint32_t a2, uint32_t a3, uint32_t b0,
                                                 uint32_t b1) {
    const float z = 0.0f;
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                            uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte global->shared async copy, bypassing L1 (streamed weights).
__device__ __forceinline__ void cp_async_16_cg(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src));
}
// 16-byte copy through L1 (small, re-read operands).
__device__ __forceinline__ void cp_async_16_ca(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src));
}
__device__ __forceinline__ void cp_async_4(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(dst), "l"(src));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Power-of-two exponent that maps a group maximum `amax` into [2**14, 2**15): the
// f16 pieces of a group scaled by 2**-e keep 11 significant bits for every element
// within 2**28 of the maximum and cannot overflow (f16 max 65504).
__device__ __forceinline__ int f16_group_exponent(float amax) {
    if (!(amax > 0.0f) || !isfinite(amax)) return 0;
    int e;
    frexpf(amax, &e);          // amax = m * 2**e, m in [0.5, 1)
    return (e - 1) - 14;
}

// Splits v (already scaled into f16 range) into f16 hi + lo with hi + lo == v to ~22 bits.
__device__ __forceinline__ void split_f16(float v, __half& hi, __half& lo) {
    hi = __float2half_rn(v);
    lo = __float2half_rn(v - __half2float(hi));
}

__device__ __forceinline__ float load_as_f32(const void* p, int dtype, int64_t i) {
    if (dtype == K3_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    if (dtype == K3_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
    return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_from_f32(void* p, int dtype, int64_t i, float v) {
    if (dtype == K3_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
    else if (dtype == K3_F16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
    else reinterpret_cast<float*>(p)[i] = v;
}

}  // namespace k3
