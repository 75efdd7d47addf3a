// C-ABI plumbing: error state, device queries, and the fused-matvec entry point.
#include <algorithm>
#include <mutex>
#include <string>
#include <vector>

#include <cuda.h>

#include "k3_common.cuh"

namespace k3 {

namespace {
thread_local std::string g_last_error;
}

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int cuda_check(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return K3_OK;
    return fail(K3_ERR_CUDA, std::string(what) + ": " + cudaGetErrorName(e) + " (" +
                                 cudaGetErrorString(e) + ")");
}

namespace {
// Driver entry points for the context id, looked up through the runtime (the library
// links no driver library of its own).
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);
CtxGetCurrentFn g_ctx_get_current = nullptr;
CtxGetIdFn g_ctx_get_id = nullptr;
std::once_flag g_ctx_fns_once;
}  // namespace

int current_context(int* dev, unsigned long long* ctx_id) {
    *ctx_id = 0;
    if (int rc = cuda_check(cudaGetDevice(dev), "cudaGetDevice")) return rc;
    if (*dev < 0 || *dev >= kMaxDevices)
        return fail(K3_ERR_UNSUPPORTED, "device ordinal " + std::to_string(*dev) + " beyond " +
                                            std::to_string(kMaxDevices));
    std::call_once(g_ctx_fns_once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(f);
        f = nullptr;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_ctx_get_id = reinterpret_cast<CtxGetIdFn>(f);
    });
    if (!g_ctx_get_current || !g_ctx_get_id)
        return fail(K3_ERR_CUDA, "cuCtxGetCurrent/cuCtxGetId unavailable from the driver");
    CUcontext ctx = nullptr;
    if (g_ctx_get_current(&ctx) != CUDA_SUCCESS) return fail(K3_ERR_CUDA, "cuCtxGetCurrent failed");
    if (!ctx) return K3_OK;
    unsigned long long id = 0;
    if (g_ctx_get_id(ctx, &id) != CUDA_SUCCESS) return fail(K3_ERR_CUDA, "cuCtxGetId failed");
    *ctx_id = id + 1;                                 // 0 stays "no context"
    return K3_OK;
}

int num_sms() {
    static int cached[kMaxDevices] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
    if (!cached[dev]) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
            v = 148;
        cached[dev] = v;
    }
    return cached[dev];
}

namespace {
struct Mark {
    int kind;
    cudaEvent_t begin, end;
};
std::mutex g_prof_mu;
bool g_prof_on = false;
std::vector<Mark> g_marks;
std::vector<cudaEvent_t> g_free_events;

cudaEvent_t take_event() {
    if (!g_free_events.empty()) {
        cudaEvent_t e = g_free_events.back();
        g_free_events.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    return e;
}
}  // namespace

void prof_begin(int kind, cudaStream_t s) {
    std::lock_guard<std::mutex> g(g_prof_mu);
    if (!g_prof_on) return;
    cudaEvent_t e = take_event();
    if (!e) return;
    cudaEventRecord(e, s);
    g_marks.push_back({kind, e, nullptr});
}

void prof_end(int kind, cudaStream_t s) {
    std::lock_guard<std::mutex> g(g_prof_mu);
    if (!g_prof_on) return;
    for (auto it = g_marks.rbegin(); it != g_marks.rend(); ++it) {
        if (it->kind == kind && it->end == nullptr) {
            cudaEvent_t e = take_event();
            if (!e) return;
            cudaEventRecord(e, s);
            it->end = e;
            return;
        }
    }
}

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

}  // namespace k3

using namespace k3;

extern "C" K3_API int k3_abi_version(void) { return 3; }

extern "C" K3_API const char* k3_last_error(void) { return g_last_error.c_str(); }

extern "C" K3_API int k3_device_sms(void) { return num_sms(); }

extern "C" K3_API int k3_profile_enable(int on) {
    std::lock_guard<std::mutex> g(g_prof_mu);
    g_prof_on = on != 0;
    return K3_OK;
}

extern "C" K3_API int k3_profile_collect(double* ms_out, int64_t* launches_out, int n) {
    std::lock_guard<std::mutex> g(g_prof_mu);
    for (int i = 0; i < n; ++i) {
        if (ms_out) ms_out[i] = 0.0;
        if (launches_out) launches_out[i] = 0;
    }
    int rc = K3_OK;
    for (const Mark& m : g_marks) {
        if (m.end) {
            float ms = 0.0f;
            cudaError_t e = cudaEventSynchronize(m.end);
            if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, m.begin, m.end);
            if (e != cudaSuccess) rc = cuda_check(e, "k3_profile_collect");
            if (m.kind >= 0 && m.kind < n) {
                if (ms_out) ms_out[m.kind] += ms;
                if (launches_out) launches_out[m.kind] += 1;
            }
            g_free_events.push_back(m.end);
        }
        g_free_events.push_back(m.begin);
    }
    g_marks.clear();
    return rc;
}

extern "C" K3_API size_t k3_mxfp4_matvec_workspace(int64_t M, int64_t K, int64_t N) {
    if (M < 1 || K < 32 || N < 1) return 0;
    size_t need = 256;
    if (K % 128 == 0 && N % 64 == 0) need = std::max(need, matvec_fast_workspace(M, K, N));
    if (K % 512 == 0 && N % 128 == 0) need = std::max(need, matvec_bs_workspace(M, K, N));
    return need;
}

extern "C" K3_API int k3_mxfp4_matvec(const void* x, int x_dtype, int64_t M, int64_t K,
                                      const uint8_t* packed, const uint8_t* scales, int64_t N,
                                      void* out, int out_dtype, void* workspace,
                                      size_t workspace_bytes, void* stream) {
    if (!x || !packed || !scales || !out) return fail(K3_ERR_INVALID, "k3_mxfp4_matvec: NULL tensor");
    if (x_dtype != K3_F32 && x_dtype != K3_BF16) return fail(K3_ERR_INVALID, "k3_mxfp4_matvec: x must be f32 or bf16");
    if (out_dtype != K3_F32 && out_dtype != K3_BF16) return fail(K3_ERR_INVALID, "k3_mxfp4_matvec: out must be f32 or bf16");
    if (M < 1 || N < 1 || K < 32 || K % 32)
        return fail(K3_ERR_INVALID, "k3_mxfp4_matvec: need M, N >= 1 and K a positive multiple of 32 (K=" + std::to_string(K) + ")");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (matvec_bs_ok(K, N, packed, scales)) {           // block-scaled tensor cores (tcgen05)
        const size_t need = matvec_bs_workspace(M, K, N);
        if (!workspace) return fail(K3_ERR_WORKSPACE, "k3_mxfp4_matvec: workspace is NULL");
        if (reinterpret_cast<uintptr_t>(workspace) % 256) return fail(K3_ERR_WORKSPACE, "k3_mxfp4_matvec: workspace must be 256-byte aligned");
        if (workspace_bytes < need) return fail(K3_ERR_WORKSPACE, "k3_mxfp4_matvec: workspace too small: need " + std::to_string(need));
        return matvec_bs(x, x_dtype, M, K, packed, scales, N, out, out_dtype, static_cast<uint8_t*>(workspace), s);
    }
    if (matvec_fast_ok(K, N, x, packed, scales)) {
        const size_t need = matvec_fast_workspace(M, K, N);
        if (!workspace) return fail(K3_ERR_WORKSPACE, "k3_mxfp4_matvec: workspace is NULL");
        if (reinterpret_cast<uintptr_t>(workspace) % 256) return fail(K3_ERR_WORKSPACE, "k3_mxfp4_matvec: workspace must be 256-byte aligned");
        if (workspace_bytes < need) return fail(K3_ERR_WORKSPACE, "k3_mxfp4_matvec: workspace too small: need " + std::to_string(need));
        return matvec_fast(x, x_dtype, M, K, packed, scales, N, out, out_dtype,
                           static_cast<uint8_t*>(workspace), s);
    }
    return launch_matvec_simple(x, x_dtype, M, K, packed, scales, N, out, out_dtype, s);
}
