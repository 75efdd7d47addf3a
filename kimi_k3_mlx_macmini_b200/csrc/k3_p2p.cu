// Expert-parallel exchanges over NVLink peer memory: the all-gather of the tokens and
// their routing, and the reduce-scatter of the partial output rows, as plain kernels that
// store straight into the other ranks' exchange buffers (CUDA IPC mappings) and publish
// a flag per rank, instead of NCCL collectives.
//
// Every rank owns one exchange buffer (all ranks the same layout):
//   [header: per-rank gather / reduce flags, this rank's arrival counters]
//   [gather area 0: W slots][gather area 1: W slots][reduce area: W slots]
// All-gather: rank r copies its source(s) into slot r of every rank's gather areas, its
// CTAs fence (system scope) and arrive on its own counter, and the last one stores the
// operation's epoch into gflag[r] of every peer (release, system scope); CTA 0 then waits
// until every peer's gflag in its own header reaches that epoch. Reduce-scatter: rank r
// copies its chunk for rank d into slot r of d's reduce area, publishes the same way, and
// every CTA waits for the peers' flags and sums the W chunks of its own rows in rank order
// (its own chunk read from the source), fp32 -- a fixed order.
//
// Epochs need no reset: a launch always has kP2PGrid CTAs, so the n-th operation's
// arrivals take the counter from (n-1)*G to n*G and each CTA derives n from the value it
// saw. Every wait is bounded (2 s, then K3_ERR_TIMEOUT in *status and the kernel goes
// on). No TMA and no multicast: plain 16-byte loads and stores.
//
// Reuse of a slot is safe without double buffering: rank s writes rank r's gather slot for
// step n+1 only after its step-n reduce-scatter saw r's step-n partial rows, which r
// produced after reading step n's gathered rows; likewise for the reduce slots.
//
// The reference has one process and no exchange (air_llm/models/kimi_k3/moe.py:119-127).
#include <cuda.h>

#include <cstring>

#include "k3_async.cuh"

namespace k3 {

constexpr int kP2PMaxWorld = 32;
constexpr int kP2PGrid = 32;            // CTAs of every exchange launch (the epoch arithmetic relies on it)
constexpr int kP2PThreads = 256;
constexpr int64_t kP2PHeader = 1024;

struct P2PHeader {
    unsigned gflag[kP2PMaxWorld];       // stored by the peers
    unsigned rflag[kP2PMaxWorld];
    unsigned gcnt, rcnt;                // this rank's arrival counters
};
static_assert(sizeof(P2PHeader) <= kP2PHeader, "header");

struct P2PPeers {
    uint8_t* base[kP2PMaxWorld];
};

struct P2PLayout {
    int64_t g0, g1, red, total;
};

static int64_t round16(int64_t v) { return (v + 15) & ~int64_t(15); }

static P2PLayout p2p_layout(int W, int64_t gb, int64_t g2b, int64_t rb) {
    P2PLayout L;
    L.g0 = kP2PHeader;
    L.g1 = L.g0 + W * round16(gb);
    L.red = L.g1 + W * round16(g2b);
    L.total = L.red + W * round16(rb);
    return L;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Arrival of this CTA on `cnt` after its stores; returns the operation's epoch. The last
// CTA of the operation stores the epoch into flag slot `rank` of every peer's header.
__device__ unsigned p2p_arrive(unsigned* cnt, const P2PPeers& pe, int W, int rank, bool reduce) {
    __shared__ unsigned s_e;
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(cnt, 1u);
        const unsigned e = prev / kP2PGrid + 1u;
        if (prev % kP2PGrid == kP2PGrid - 1) {
            __threadfence_system();
            for (int d = 0; d < W; ++d) {
                if (d == rank) continue;
                P2PHeader* h = reinterpret_cast<P2PHeader*>(pe.base[d]);
                st_release_sys(reduce ? &h->rflag[rank] : &h->gflag[rank], e);
            }
        }
        s_e = e;
    }
    __syncthreads();
    return s_e;
}

// Threads 0..W-1 of the calling CTA wait until flag[t] of this rank's header reaches e
// (t != rank); bounded.
__device__ void p2p_wait(const unsigned* flag, int W, int rank, unsigned e, int* status) {
    const int t = threadIdx.x;
    if (t < W && t != rank) {
        const uint64_t t0 = global_ns();
        while (int(ld_acquire_sys(flag + t) - e) < 0) {
            if (global_ns() - t0 > kWaitLimitNs) {
                atomicExch(status, K3_ERR_TIMEOUT);
                break;
            }
            __nanosleep(64);
        }
    }
    __syncthreads();
}

// mode bit 0: put (copy + arrive + publish); bit 1: wait (CTA 0).
__global__ void __launch_bounds__(kP2PThreads) p2p_allgather_kernel(P2PPeers pe, int W, int rank, int64_t off0,
                                                                   int64_t off1, const uint4* __restrict__ s0,
                                                                   int n0, const uint4* __restrict__ s1, int n1,
                                                                   int mode, int* status) {
    P2PHeader* own = reinterpret_cast<P2PHeader*>(pe.base[rank]);
    unsigned e = 0;
    if (mode & 1) {
        const int units = n0 + n1;
        for (int d = 0; d < W; ++d) {
            uint4* d0 = reinterpret_cast<uint4*>(pe.base[d] + off0) + int64_t(rank) * n0;
            uint4* d1 = reinterpret_cast<uint4*>(pe.base[d] + off1) + int64_t(rank) * n1;
            for (int w = blockIdx.x * blockDim.x + threadIdx.x; w < units; w += gridDim.x * blockDim.x) {
                if (w < n0)
                    d0[w] = __ldg(s0 + w);
                else
                    d1[w - n0] = __ldg(s1 + (w - n0));
            }
        }
        e = p2p_arrive(&own->gcnt, pe, W, rank, false);
    } else {
        e = *reinterpret_cast<volatile unsigned*>(&own->gcnt) / kP2PGrid;
    }
    if ((mode & 2) && blockIdx.x == 0) p2p_wait(own->gflag, W, rank, e, status);
}

// mode bit 0: put (copy the chunks for the peers + arrive + publish); bit 1: wait and sum.
// src: W chunks of n floats (chunk d for rank d); out: n floats.
__global__ void __launch_bounds__(kP2PThreads) p2p_reduce_scatter_kernel(P2PPeers pe, int W, int rank,
                                                                        int64_t off_red,
                                                                        const float* __restrict__ src, int n,
                                                                        float* __restrict__ out, int mode,
                                                                        int* status) {
    P2PHeader* own = reinterpret_cast<P2PHeader*>(pe.base[rank]);
    const int q = n / 4;                                   // 16-byte words per chunk
    unsigned e = 0;
    if (mode & 1) {
        for (int d = 0; d < W; ++d) {
            if (d == rank) continue;
            const float4* a = reinterpret_cast<const float4*>(src + int64_t(d) * n);
            float4* b = reinterpret_cast<float4*>(pe.base[d] + off_red) + int64_t(rank) * q;
            for (int w = blockIdx.x * blockDim.x + threadIdx.x; w < q; w += gridDim.x * blockDim.x)
                b[w] = __ldg(a + w);
        }
        e = p2p_arrive(&own->rcnt, pe, W, rank, true);
    } else {
        e = *reinterpret_cast<volatile unsigned*>(&own->rcnt) / kP2PGrid;
    }
    if (!(mode & 2)) return;
    p2p_wait(own->rflag, W, rank, e, status);
    const float4* mine = reinterpret_cast<const float4*>(src + int64_t(rank) * n);
    const float4* red = reinterpret_cast<const float4*>(pe.base[rank] + off_red);
    for (int w = blockIdx.x * blockDim.x + threadIdx.x; w < q; w += gridDim.x * blockDim.x) {
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (int s = 0; s < W; ++s) {
            const float4 v = s == rank ? __ldg(mine + w) : __ldcg(red + int64_t(s) * q + w);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        reinterpret_cast<float4*>(out)[w] = acc;
    }
}

static int group_peers(const k3_p2p_group* g, P2PPeers* pe, const char* what) {
    if (!g) return fail(K3_ERR_INVALID, std::string(what) + ": group is NULL");
    if (g->world < 1 || g->world > kP2PMaxWorld) return fail(K3_ERR_UNSUPPORTED, std::string(what) + ": world must be 1..32");
    if (g->rank < 0 || g->rank >= g->world) return fail(K3_ERR_INVALID, std::string(what) + ": rank outside [0, world)");
    for (int d = 0; d < g->world; ++d) {
        if (!g->base[d] || (reinterpret_cast<uintptr_t>(g->base[d]) & 255))
            return fail(K3_ERR_INVALID, std::string(what) + ": a buffer base is NULL or not 256-byte aligned");
        pe->base[d] = static_cast<uint8_t*>(g->base[d]);
    }
    for (int d = g->world; d < kP2PMaxWorld; ++d) pe->base[d] = nullptr;
    return K3_OK;
}

using GetRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

static GetRangeFn get_range_fn() {
    static GetRangeFn fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &f, 12000, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<GetRangeFn>(f);
    }();
    return fn;
}

}  // namespace k3

using namespace k3;

extern "C" K3_API size_t k3_p2p_buffer_bytes(int world, int64_t gather_bytes, int64_t gather2_bytes,
                                             int64_t reduce_bytes) {
    if (world < 1 || world > kP2PMaxWorld || gather_bytes < 0 || gather2_bytes < 0 || reduce_bytes < 0) return 0;
    return size_t(p2p_layout(world, gather_bytes, gather2_bytes, reduce_bytes).total);
}

extern "C" K3_API int k3_p2p_area_offsets(int world, int64_t gather_bytes, int64_t gather2_bytes,
                                          int64_t reduce_bytes, int64_t* offsets_out) {
    if (!offsets_out) return fail(K3_ERR_INVALID, "k3_p2p_area_offsets: offsets_out is NULL");
    if (world < 1 || world > kP2PMaxWorld) return fail(K3_ERR_UNSUPPORTED, "k3_p2p_area_offsets: world must be 1..32");
    const P2PLayout L = p2p_layout(world, gather_bytes, gather2_bytes, reduce_bytes);
    offsets_out[0] = L.g0;
    offsets_out[1] = L.g1;
    offsets_out[2] = L.red;
    offsets_out[3] = L.total;
    return K3_OK;
}

extern "C" K3_API int k3_p2p_export(const void* ptr, uint8_t* handle_out, int64_t* offset_out) {
    if (!ptr || !handle_out || !offset_out) return fail(K3_ERR_INVALID, "k3_p2p_export: NULL pointer");
    GetRangeFn range = get_range_fn();
    if (!range) return fail(K3_ERR_CUDA, "k3_p2p_export: cuMemGetAddressRange is unavailable");
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
        return fail(K3_ERR_CUDA, "k3_p2p_export: cuMemGetAddressRange failed");
    cudaIpcMemHandle_t h;
    if (int rc = cuda_check(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)), "cudaIpcGetMemHandle")) return rc;
    static_assert(sizeof(h) == 64, "IPC handle size");
    memcpy(handle_out, &h, sizeof(h));
    *offset_out = int64_t(reinterpret_cast<CUdeviceptr>(ptr) - base);
    return K3_OK;
}

extern "C" K3_API int k3_p2p_open(const uint8_t* handle, int64_t offset, void** ptr_out) {
    if (!handle || !ptr_out || offset < 0) return fail(K3_ERR_INVALID, "k3_p2p_open: bad argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* base = nullptr;
    if (int rc = cuda_check(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle"))
        return rc;
    *ptr_out = static_cast<uint8_t*>(base) + offset;
    return K3_OK;
}

extern "C" K3_API int k3_p2p_close(void* ptr, int64_t offset) {
    if (!ptr || offset < 0) return fail(K3_ERR_INVALID, "k3_p2p_close: bad argument");
    return cuda_check(cudaIpcCloseMemHandle(static_cast<uint8_t*>(ptr) - offset), "cudaIpcCloseMemHandle");
}

extern "C" K3_API int k3_p2p_allgather(const k3_p2p_group* g, const void* src, int64_t bytes, const void* src2,
                                       int64_t bytes2, int mode, int32_t* status, void* stream) {
    P2PPeers pe;
    if (int rc = group_peers(g, &pe, "k3_p2p_allgather")) return rc;
    if (!status || mode < 1 || mode > 3) return fail(K3_ERR_INVALID, "k3_p2p_allgather: bad status or mode");
    if (bytes < 0 || bytes2 < 0 || (bytes & 15) || (bytes2 & 15) || bytes > g->gather_bytes ||
        bytes2 > g->gather2_bytes)
        return fail(K3_ERR_INVALID, "k3_p2p_allgather: sizes must be multiples of 16 within the slot capacities");
    if ((bytes && !src) || (bytes2 && !src2) ||
        ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(src2)) & 15))
        return fail(K3_ERR_INVALID, "k3_p2p_allgather: sources must be 16-byte aligned");
    if ((bytes + bytes2) / 16 > (int64_t(1) << 30)) return fail(K3_ERR_INVALID, "k3_p2p_allgather: too large");
    const P2PLayout L = p2p_layout(g->world, g->gather_bytes, g->gather2_bytes, g->reduce_bytes);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    prof_begin(K3_PROF_OTHER, s);
    p2p_allgather_kernel<<<kP2PGrid, kP2PThreads, 0, s>>>(pe, g->world, g->rank, L.g0, L.g1,
                                                           static_cast<const uint4*>(src), int(bytes / 16),
                                                           static_cast<const uint4*>(src2), int(bytes2 / 16), mode,
                                                           status);
    prof_end(K3_PROF_OTHER, s);
    K3_CHECK_LAUNCH("p2p_allgather_kernel");
    return K3_OK;
}

extern "C" K3_API int k3_p2p_reduce_scatter(const k3_p2p_group* g, const float* src, int64_t n, float* out,
                                            int mode, int32_t* status, void* stream) {
    P2PPeers pe;
    if (int rc = group_peers(g, &pe, "k3_p2p_reduce_scatter")) return rc;
    if (!status || mode < 1 || mode > 3) return fail(K3_ERR_INVALID, "k3_p2p_reduce_scatter: bad status or mode");
    if (!src || ((mode & 2) && !out)) return fail(K3_ERR_INVALID, "k3_p2p_reduce_scatter: NULL src or out");
    if (n < 4 || (n & 3) || n * 4 > g->reduce_bytes || n > (int64_t(1) << 30))
        return fail(K3_ERR_INVALID, "k3_p2p_reduce_scatter: n must be a multiple of 4 within the slot capacity");
    if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(out)) & 15)
        return fail(K3_ERR_INVALID, "k3_p2p_reduce_scatter: src and out must be 16-byte aligned");
    const P2PLayout L = p2p_layout(g->world, g->gather_bytes, g->gather2_bytes, g->reduce_bytes);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    prof_begin(K3_PROF_OTHER, s);
    p2p_reduce_scatter_kernel<<<kP2PGrid, kP2PThreads, 0, s>>>(pe, g->world, g->rank, L.red, src, int(n), out, mode,
                                                                status);
    prof_end(K3_PROF_OTHER, s);
    K3_CHECK_LAUNCH("p2p_reduce_scatter_kernel");
    return K3_OK;
}
