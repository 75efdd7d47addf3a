// k3_mxfp4_matvec_noalloc: the fused MXFP4 matvec for callers that cannot allocate.
//
// Some hosts of this path hand it nothing but their own input and output buffers: an
// FFI binding of the three-argument mxfp4_matvec_fused whose device memory is owned by
// another allocator (a framework's caching allocator, or a fixed arena that holds the
// device's free memory). Such a caller cannot call cudaMalloc -- the allocation would
// go behind its allocator's back or fail against the arena, and cudaMalloc/cudaFree
// synchronise the device in the middle of a decode loop. This entry point therefore
// allocates nothing: its scratch is a file-scope device array that every GPU loading
// this library holds until the process exits.
#include <mutex>
#include <string>

#include "k3_common.cuh"

namespace k3 {

// defined in k3_moe.cu / k3_codec.cu
bool matvec_fast_ok(int64_t K, int64_t N, const void* x, const uint8_t* packed,
                    const uint8_t* scales);
size_t matvec_fast_workspace(int64_t M, int64_t K, int64_t N);
int matvec_fast(const void* x, int xdt, int64_t M, int64_t K, const uint8_t* packed,
                const uint8_t* scales, int64_t N, void* out, int odt, uint8_t* ws, cudaStream_t s);
int launch_matvec_simple(const void* x, int xdt, int64_t M, int64_t K, const uint8_t* packed,
                         const uint8_t* scales, int64_t N, void* out, int odt, cudaStream_t s);
// defined in k3_mv.cu
bool matvec_bs_ok(int64_t K, int64_t N, const uint8_t* packed, const uint8_t* scales);
size_t matvec_bs_workspace(int64_t M, int64_t K, int64_t N);
int matvec_bs(const void* x, int xdt, int64_t M, int64_t K, const uint8_t* packed, const uint8_t* scales,
              int64_t N, void* out, int odt, uint8_t* ws, cudaStream_t s);

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;   // 4 MiB per device

// The scratch of k3_mxfp4_matvec_noalloc. In host code this name is a host-side
// stand-in, not a device address: only the address from cudaGetSymbolAddress may be
// handed to a kernel.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};
unsigned long long g_scratch_ctx[kMaxDevices] = {};

// Device address of the scratch array in the current device's context. It is looked up
// once per context (with that device current) and cached; a device whose context was
// replaced since (cudaDeviceReset) gets a fresh lookup, since the array then lives at
// an address of the new context.
int scratch_address(void** out) {
    int dev = -1;
    unsigned long long ctx = 0;
    if (int rc = current_context(&dev, &ctx)) return rc;
    std::lock_guard<std::mutex> g(g_mu);
    if (ctx == 0 || g_scratch_ctx[dev] != ctx) {
        void* p = nullptr;
        if (int rc = cuda_check(cudaGetSymbolAddress(&p, g_noalloc_scratch),
                                "cudaGetSymbolAddress(no-alloc scratch)"))
            return rc;
        if (ctx == 0)                                  // the lookup created the context
            if (int rc = current_context(&dev, &ctx)) return rc;
        g_scratch_addr[dev] = p;
        g_scratch_ctx[dev] = ctx;
    }
    *out = g_scratch_addr[dev];
    return K3_OK;
}

}  // namespace
}  // namespace k3

using namespace k3;

extern "C" K3_API int k3_mxfp4_matvec_noalloc(const void* x, int x_dtype, int64_t M, int64_t K,
                                              const uint8_t* packed, const uint8_t* scales,
                                              int64_t N, void* out, int out_dtype, void* stream) {
    if (!x || !packed || !scales || !out) return fail(K3_ERR_INVALID, "k3_mxfp4_matvec_noalloc: NULL tensor");
    if (x_dtype != K3_F32 && x_dtype != K3_BF16) return fail(K3_ERR_INVALID, "k3_mxfp4_matvec_noalloc: x must be f32 or bf16");
    if (out_dtype != K3_F32 && out_dtype != K3_BF16) return fail(K3_ERR_INVALID, "k3_mxfp4_matvec_noalloc: out must be f32 or bf16");
    if (M < 1 || N < 1 || K < 32 || K % 32)
        return fail(K3_ERR_INVALID, "k3_mxfp4_matvec_noalloc: need M, N >= 1 and K a positive multiple of 32");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool bs = matvec_bs_ok(K, N, packed, scales);
    if (!bs && !matvec_fast_ok(K, N, x, packed, scales))  // the generic kernel needs no scratch
        return launch_matvec_simple(x, x_dtype, M, K, packed, scales, N, out, out_dtype, s);
    const size_t need = bs ? matvec_bs_workspace(M, K, N) : matvec_fast_workspace(M, K, N);
    if (need > kNoAllocScratchBytes)
        return fail(K3_ERR_INVALID, "k3_mxfp4_matvec_noalloc: M=" + std::to_string(M) + " K=" +
                                        std::to_string(K) + " N=" + std::to_string(N) + " needs " +
                                        std::to_string(need) + " bytes of scratch, above the " +
                                        std::to_string(kNoAllocScratchBytes) +
                                        "-byte no-alloc limit; use k3_mxfp4_matvec with a workspace");
    void* scratch = nullptr;
    if (int rc = scratch_address(&scratch)) return rc;
    // The prep kernel rewrites the converted x (and the plan) and zeroes the arrival
    // counters; every partial sum is written before it is read. Nothing of a previous
    // call's contents is used.
    if (bs)
        return matvec_bs(x, x_dtype, M, K, packed, scales, N, out, out_dtype, static_cast<uint8_t*>(scratch), s);
    return matvec_fast(x, x_dtype, M, K, packed, scales, N, out, out_dtype,
                       static_cast<uint8_t*>(scratch), s);
}
