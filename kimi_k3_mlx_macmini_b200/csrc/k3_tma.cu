// TMA-fed grouped MXFP4 matvec (decode path, sm_100a).
//
// One producer thread per CTA streams weight tiles, their E8M0 scales and the B
// operand (activation pieces) into a ring of CTA-wide shared-memory stages with
// cp.async.bulk.tensor; each stage has a "full" mbarrier (transaction bytes) and an
// "empty" mbarrier (one arrival per consumer warp). Consumer warps read the swizzled
// weight tiles with ldmatrix so a quad holds one 32-element scale group, convert
// E2M1 -> f16 in hardware, issue mma.m16n8k16 (tokens or pairs as the n8 dimension) and
// add each group's partial sum to fp32 accumulators with its exact power-of-two scale.
// Partial sums of k-chunks meet in global scratch and the last CTA to finish a row
// block reduces them in a fixed order. Every wait is bounded (K3_ERR_TIMEOUT).
#include <cudaTypedefs.h>

#include <mutex>
#include <string>

#include "k3_async.cuh"
#include "k3_bs.cuh"
#include "k3_tma.cuh"

namespace k3 {

// ------------------------------------------------------------------- host maps

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
}  // namespace

int encode_map(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* base,
               const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
               CUtensorMapSwizzle swizzle) {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    if (!g_encode) return fail(K3_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t d[5], st[4];
    cuuint32_t b[5], es[5];
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        b[i] = box[i];
        es[i] = 1;
        if (i + 1 < rank) st[i] = strides_bytes[i];
    }
    const CUresult r = g_encode(m, dt, cuuint32_t(rank), const_cast<void*>(base), d, st, b, es,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(K3_ERR_INVALID, "cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
    return K3_OK;
}

// --------------------------------------------------------------- device helpers

__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;\n" ::"n"(kTWarps * 32) : "memory");
}

__device__ __forceinline__ float act_fn(int kind, float g, float u, float beta, float lbeta) {
    return act_value(kind, g, u, beta, lbeta);
}

// ---------------------------------------------------------------------- kernel

// CTA owning item i when n items are split into gridDim contiguous ranges
// [floor(b*n/g), floor((b+1)*n/g)).
__device__ __forceinline__ int64_t cta_of(int64_t i, int64_t n, int64_t g) {
    return ((i + 1) * g - 1) / n;
}

template <bool GATEUP, bool HILO, bool GROUP_TS>
__global__ void __launch_bounds__(kTThreads, 1)
    gemv_tma_kernel(const __grid_constant__ TMaps maps, const TArgs a) {
    using St = TStage<HILO, GROUP_TS>;
    constexpr int S = tstages<HILO>();
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    St* ring = reinterpret_cast<St*>(base);
    float* ebuf = reinterpret_cast<float*>(base + sizeof(St) * S);          // [8][128]
    uint64_t* full = reinterpret_cast<uint64_t*>(base + sizeof(St) * S + kTEpilogueBytes);
    uint64_t* empty = full + S;
    __shared__ int s_last;
    __shared__ int s_nseg;
    __shared__ int s_seg[kTMaxSegments];              // item offsets where key segments start
    __shared__ volatile int s_abort;                  // a consumer wait gave up
    __shared__ volatile unsigned s_issued;            // stages the producer has issued

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        s_abort = 0;
        s_issued = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kTWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    __syncthreads();

    const Plan* P = a.plan;
    const int n_active = P->n_active;
    const int M = P->M;
    const int64_t nRb = GATEUP ? a.rows / 64 : a.rows / kTRows;
    const int64_t ipk = GATEUP ? a.C : int64_t(n_active) * a.C;      // items per key
    const int64_t n_keys = GATEUP ? int64_t(n_active) * nRb : nRb;
    const int64_t n = n_keys * ipk;
    const int64_t grid = gridDim.x, b = blockIdx.x;
    const int64_t i0 = b * n / grid, i1 = (b + 1) * n / grid;
    const int64_t kchunk = a.K / a.C;
    const int nst = int(kchunk / kTStageK);

    if (warp == kTWarps) {
        // ------------------------------------------------------------ producer
        if (lane != 0) return;
        constexpr uint32_t kBytes = uint32_t(2 * kTRows * 128 + kTRows * kTGroups +
                                             kTGroups * kMaxTok * 32 * 2 * (HILO ? 2 : 1) +
                                             (GROUP_TS ? kTGroups * kMaxTok * 4 : 0));
        uint32_t gs = 0;
        for (int64_t i = i0; i < i1; ++i) {
            const int64_t key = i / ipk, j = i % ipk;
            const int u = GATEUP ? int(key / nRb) : int(j / a.C);
            const int rb = GATEUP ? int(key % nRb) : int(key);
            const int kc = int(GATEUP ? j : j % a.C);
            const int slot = a.matvec ? 0 : P->expert[u];
            const int brow = (GATEUP || a.matvec) ? 0 : u * kMaxTok;
            const int64_t k0 = int64_t(kc) * kchunk;
            for (int s = 0; s < nst; ++s, ++gs) {
                const int si = int(gs % S);
                if (!mbar_wait(&empty[si], ((gs / S) & 1) ^ 1, a.status)) return;
                St& st = ring[si];
                mbar_expect_tx(&full[si], kBytes);
                const int kb = int((k0 + int64_t(s) * kTStageK) / 2);
                const int kg = int((k0 + int64_t(s) * kTStageK) / 32);
                if (GATEUP) {
                    const int r0 = rb * 64;
                    tma_3d(&st.w[0][0][0], &maps.wA, kb, r0, slot, &full[si]);
                    tma_3d(&st.w[1][0][0], &maps.wA, kb + 128, r0, slot, &full[si]);
                    tma_3d(&st.w[0][64][0], &maps.wB, kb, r0, slot, &full[si]);
                    tma_3d(&st.w[1][64][0], &maps.wB, kb + 128, r0, slot, &full[si]);
                    tma_3d(&st.s[0][0], &maps.sA, kg, r0, slot, &full[si]);
                    tma_3d(&st.s[64][0], &maps.sB, kg, r0, slot, &full[si]);
                } else {
                    const int r0 = rb * kTRows;
                    tma_3d(&st.w[0][0][0], &maps.wA, kb, r0, slot, &full[si]);
                    tma_3d(&st.w[1][0][0], &maps.wA, kb + 128, r0, slot, &full[si]);
                    tma_3d(&st.s[0][0], &maps.sA, kg, r0, slot, &full[si]);
                }
                tma_3d(&st.bh[0][0][0], &maps.bh, 0, brow, kg, &full[si]);
                if (HILO) tma_3d(&st.bl[0][0][0], &maps.bl, 0, brow, kg, &full[si]);
                if (GROUP_TS) tma_2d(&st.ts[0][0], &maps.bts, brow, kg, &full[si]);
                s_issued = gs + 1;
            }
        }
        return;
    }

    // -------------------------------------------------------------- consumers
    // All consumer warps run the same sequence of named barriers, also after a
    // timed-out wait; the shared abort flag is read only after a barrier, so all warps
    // leave together.
    const int g = lane >> 2, q = lane & 3;
    const int tr = warp * 16;                         // this warp's 16 rows of the stage tile
    const int c0 = 2 * q, c1 = c0 + 1;                // this thread's accumulator columns
    const int ctid = int(threadIdx.x);                // 0..255
    uint32_t gs = 0;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const int64_t nkb = a.K / kTStageK;               // x scale blocks per token (!GROUP_TS)
    for (int64_t i = i0; i < i1; ++i) {
        const int64_t key = i / ipk, j = i % ipk;
        const int64_t kst0 = (GATEUP ? j : j % a.C) * nst;     // first 512-k block of the item
        for (int s = 0; s < nst; ++s, ++gs) {
            const int si = int(gs % S);
            if (s_abort || !mbar_wait(&full[si], (gs / S) & 1, a.status)) {
                s_abort = 1;
                break;
            }
            const St& st = ring[si];
            // !GROUP_TS: x has one scale per (token, stage); the stage's sums meet it once
            float sacc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            float* const dst = GROUP_TS ? acc : sacc;
            uint32_t sw0[4], sw8[4];                  // scale bytes of rows g, g+8 (16 groups)
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                sw0[k] = *reinterpret_cast<const uint32_t*>(&st.s[tr + g][4 * k]);
                sw8[k] = *reinterpret_cast<const uint32_t*>(&st.s[tr + g + 8][4 * k]);
            }
#pragma unroll
            for (int gp = 0; gp < kTGroups / 2; ++gp) {
                const int box = gp >> 2, gi = (2 * gp) & 7;
                uint32_t R0, R1, R2, R3;
                {
                    const int m = lane >> 3, r = tr + (lane & 7) + 8 * (m & 1);
                    const int c = gi + (m >> 1);
                    ldmatrix_x4(smem_u32(&st.w[box][r][(c ^ (r & 7)) << 4]), R0, R1, R2, R3);
                }
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int G = 2 * gp + h;
                    const uint4 X = *reinterpret_cast<const uint4*>(&st.bh[G][g][8 * q]);
                    uint32_t f0, f1, f2, f3, e0, e1, e2, e3;
                    e2m1x8_to_f16x8(h ? R2 : R0, f0, f1, f2, f3);
                    e2m1x8_to_f16x8(h ? R3 : R1, e0, e1, e2, e3);
                    float tmp[4];
                    mma_f16_16816_zc(tmp, f0, e0, f1, e1, X.x, X.y);
                    mma_f16_16816(tmp, f2, e2, f3, e3, X.z, X.w);
                    if (HILO) {
                        const uint4 XL = *reinterpret_cast<const uint4*>(&st.bl[G][g][8 * q]);
                        mma_f16_16816(tmp, f0, e0, f1, e1, XL.x, XL.y);
                        mma_f16_16816(tmp, f2, e2, f3, e3, XL.z, XL.w);
                    }
                    const int wi = G >> 2, sh = 8 * (G & 3);
                    const float rs0 = e8m0_to_f32((sw0[wi] >> sh) & 0xffu);
                    const float rs1 = e8m0_to_f32((sw8[wi] >> sh) & 0xffu);
                    if (GROUP_TS) {
                        const float2 tv = *reinterpret_cast<const float2*>(&st.ts[G][c0]);
                        dst[0] = fmaf(rs0 * tv.x, tmp[0], dst[0]);
                        dst[1] = fmaf(rs0 * tv.y, tmp[1], dst[1]);
                        dst[2] = fmaf(rs1 * tv.x, tmp[2], dst[2]);
                        dst[3] = fmaf(rs1 * tv.y, tmp[3], dst[3]);
                    } else {
                        dst[0] = fmaf(rs0, tmp[0], dst[0]);
                        dst[1] = fmaf(rs0, tmp[1], dst[1]);
                        dst[2] = fmaf(rs1, tmp[2], dst[2]);
                        dst[3] = fmaf(rs1, tmp[3], dst[3]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[si]);
            if (!GROUP_TS) {
                // rows M..7 of x are zeros with a finite scale
                const float t0 = __ldg(a.bts_tok + c0 * nkb + kst0 + s);
                const float t1 = __ldg(a.bts_tok + c1 * nkb + kst0 + s);
                acc[0] = fmaf(sacc[0], t0, acc[0]);
                acc[1] = fmaf(sacc[1], t1, acc[1]);
                acc[2] = fmaf(sacc[2], t0, acc[2]);
                acc[3] = fmaf(sacc[3], t1, acc[3]);
            }
        }
        if (!s_abort && i + 1 < i1 && (i + 1) / ipk == key) continue;   // key continues here

        // ---- flush the key
        const int64_t ks = key * ipk;                                // first item of the key
        const bool local = cta_of(ks, n, grid) == cta_of(ks + ipk - 1, n, grid);
        float* kpart = a.part + key * a.maxseg * (kMaxTok * kTRows);
        const int r = tr + g;                                        // stage-tile row
        if (local) {
            if (GATEUP) {
                ebuf[c0 * kTRows + r] = acc[0];
                ebuf[c1 * kTRows + r] = acc[1];
                ebuf[c0 * kTRows + r + 8] = acc[2];
                ebuf[c1 * kTRows + r + 8] = acc[3];
            } else {
                const int64_t row = key * kTRows + r;
                if (c0 < M) {
                    store_from_f32(a.y, a.y_dtype, int64_t(c0) * a.rows + row, acc[0]);
                    store_from_f32(a.y, a.y_dtype, int64_t(c0) * a.rows + row + 8, acc[2]);
                }
                if (c1 < M) {
                    store_from_f32(a.y, a.y_dtype, int64_t(c1) * a.rows + row, acc[1]);
                    store_from_f32(a.y, a.y_dtype, int64_t(c1) * a.rows + row + 8, acc[3]);
                }
            }
        } else {
            // segment slot = offset of this CTA's first item in the key
            const int64_t seg = (i0 > ks ? i0 : ks) - ks;
            float* sp = kpart + seg * (kMaxTok * kTRows);
            sp[c0 * kTRows + r] = acc[0];
            sp[c1 * kTRows + r] = acc[1];
            sp[c0 * kTRows + r + 8] = acc[2];
            sp[c1 * kTRows + r + 8] = acc[3];
            __threadfence();
        }
        acc[0] = acc[1] = acc[2] = acc[3] = 0.0f;
        if (!local && ctid == 0) {
            // the key's segments start where the owning CTA changes between items
            int ns = 0;
            for (int64_t jj = 0; jj < ipk && ns < kTMaxSegments; ++jj)
                if (jj == 0 || cta_of(ks + jj, n, grid) != cta_of(ks + jj - 1, n, grid)) s_seg[ns++] = int(jj);
            s_nseg = ns;
        }
        consumer_sync();
        if (ctid == 0)
            s_last = local || (!s_abort && atomicAdd(a.cnt + key, 1u) + 1 == unsigned(s_nseg));
        consumer_sync();
        if (s_abort) break;
        if (!s_last) continue;
        if (!local) __threadfence();

        // value of column c, stage-tile row rr of this key (summed over segments)
        auto val = [&](int c, int rr) -> float {
            if (local) return ebuf[c * kTRows + rr];
            float v = 0.0f;
            for (int sg = 0; sg < s_nseg; ++sg)
                v += __ldcg(kpart + int64_t(s_seg[sg]) * (kMaxTok * kTRows) + c * kTRows + rr);
            return v;
        };
        if (GATEUP) {
            // warp t: token t of this expert (zeros when t is not routed to it)
            const int u = int(key / nRb), rb = int(key % nRb);
            const int t = warp;
            float wgt = 0.0f;
            if (t < M)
                for (int p = P->pair_start[u]; p < P->pair_start[u + 1]; ++p)
                    if (P->pair_tok[p] == t) wgt = P->pair_w[p];
            const int64_t arow = int64_t(u) * kMaxTok + t;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int rr = half * 32 + lane;
                float v = 0.0f;
                if (wgt != 0.0f) v = act_fn(a.act_kind, val(t, rr), val(t, 64 + rr), a.beta, a.lbeta) * wgt;
                const int e = f16_group_exponent(warp_max(fabsf(v)));
                __half hi, lo;
                split_f16(ldexpf(v, -e), hi, lo);
                const int64_t G = int64_t(rb) * 2 + half;          // act group along I
                const int64_t o = (G * a.act_rows + arow) * 32 + lane;
                a.act_hi[o] = hi;
                a.act_lo[o] = lo;
                if (lane == 0) a.act_ts[G * a.act_rows + arow] = ldexpf(1.0f, e);
            }
        } else if (!local) {
            const int rr = ctid & (kTRows - 1);
            const int64_t row = key * kTRows + rr;
            for (int t = ctid >> 7; t < M; t += 2)
                store_from_f32(a.y, a.y_dtype, int64_t(t) * a.rows + row, val(t, rr));
        }
        if (!local && ctid == 0) a.cnt[key] = 0u;           // ready for the next call
        if (GATEUP) consumer_sync();                        // ebuf is reused by the next key
    }
    if (s_abort && ctid == 0) {
        // before leaving, wait (bounded) for the copies the producer already issued
        const unsigned issued = s_issued;
        for (unsigned k = gs; k < issued; ++k)
            if (!mbar_wait(&full[k % S], (k / S) & 1, a.status)) break;
    }
}

// ------------------------------------------------------------------ launches

template <bool G, bool H, bool T>
int launch_one(const TMaps& maps, const TArgs& a, int grid, cudaStream_t s, const char* what) {
    static OncePerContext attr;
    constexpr size_t smem = tsmem_bytes<H, T>();
    if (int rc = attr.run([&] {
            return cuda_check(cudaFuncSetAttribute(gemv_tma_kernel<G, H, T>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
                              what);
        }))
        return rc;
    gemv_tma_kernel<G, H, T><<<grid, kTThreads, smem, s>>>(maps, a);
    K3_CHECK_LAUNCH(what);
    return K3_OK;
}

int launch_tma_gateup(const TMaps& maps, const TArgs& a, bool hilo, int grid, cudaStream_t s) {
    return hilo ? launch_one<true, true, false>(maps, a, grid, s, "gemv_tma<gate/up f32>")
                : launch_one<true, false, false>(maps, a, grid, s, "gemv_tma<gate/up bf16>");
}

int launch_tma_proj(const TMaps& maps, const TArgs& a, bool hilo, bool group_ts, int grid,
                    cudaStream_t s) {
    if (group_ts) return launch_one<false, true, true>(maps, a, grid, s, "gemv_tma<down>");
    return hilo ? launch_one<false, true, false>(maps, a, grid, s, "gemv_tma<matvec f32>")
                : launch_one<false, false, false>(maps, a, grid, s, "gemv_tma<matvec bf16>");
}

}  // namespace k3
