// Block-scaled grouped MXFP4 matvec on tcgen05 (decode path, sm_100a).
//
// Roles per CTA (6 warps):
//   warp 0  producer: one thread streams each stage -- weight tiles (TMA, 128-byte
//           swizzle), their scale chunks and the B pieces' scale chunks (bulk copies),
//           the B piece tile (TMA) -- into a ring of shared-memory stages (full/empty
//           mbarriers, transaction-byte counted);
//   warp 1  MMA issuer: owns the TMEM allocation; one thread copies each stage's scale
//           chunks into TMEM (tcgen05.cp) and issues tcgen05.mma.kind::mxf4.block_scale
//           (M=128 weight rows, N = 8 pieces x columns, K=64) into a double-buffered TMEM
//           accumulator, then tcgen05.commit frees the stage and, at the end of an item,
//           hands the accumulator to the epilogue;
//   warps 2-5 epilogue: warp w reads TMEM lanes 32*(w%4).. (weight rows), sums the pieces
//           of each pair, accumulates the items of a key in registers and flushes it
//           (gate/up: activation x routing weight, split into the next launch's E2M1
//           pieces; down: one output row per pair), through per-segment partials when the
//           key spans CTAs.
//
// Work: key = (128-row block, expert item) for both phases, items = its k-chunks; each
// CTA owns a contiguous range of items. The B operand holds only the expert's (token,
// weight) pairs (8 piece rows per pair), so a call may carry any number of tokens; the
// down phase writes one output row per pair and the combine kernel sums a token's pairs.
// Every wait is bounded.
#include "k3_async.cuh"
#include "k3_bs.cuh"
#include "k3_tma.cuh"

namespace k3 {

namespace {

__device__ __forceinline__ void epi_sync() {
    asm volatile("bar.sync 1, %0;\n" ::"n"(kBEpiWarps * 32) : "memory");
}


// CTA owning item i of n items split over g CTAs in contiguous ranges [b n / g, (b+1) n / g)
// (32-bit: the host keeps n * g below 2^32)
__device__ __forceinline__ uint32_t owner_of(uint32_t i, uint32_t n, uint32_t g) {
    return ((i + 1) * g - 1) / n;
}

// sum of 8 consecutive values in a fixed order
__device__ __forceinline__ float sum8(const float* v) {
    return ((((((v[0] + v[1]) + v[2]) + v[3]) + v[4]) + v[5]) + v[6]) + v[7];
}

}  // namespace

// The last CTA of a split key sums the key's segment partials (each [PW][128] floats:
// per pair the gate or down value, then for gate/up the up value) in segment order into
// acc0 / acc1 for row r: G segments' values of the first NPM pairs in flight at once
// (np <= NPM; pairs past np read nothing and add zeros).
template <int G, int NPM, bool GATEUP>
__device__ __forceinline__ void sum_segments(const float* kpart, const int* segs, int nseg, int np, int r,
                                             float (&acc0)[kBMaxN / kBPieces], float (&acc1)[kBMaxN / kBPieces]) {
    constexpr int kMaxPr = kBMaxN / kBPieces;
    constexpr int kPW = GATEUP ? 2 * kMaxPr : kMaxPr;
    for (int sg0 = 0; sg0 < nseg; sg0 += G) {
        float x0[G][NPM], x1[G][NPM];
#pragma unroll
        for (int u = 0; u < G; ++u) {
            const float* sp = kpart + int64_t(segs[min(sg0 + u, nseg - 1)]) * (kPW * kBRows);
#pragma unroll
            for (int pi = 0; pi < NPM; ++pi) {
                const bool ok = sg0 + u < nseg && pi < np;
                x0[u][pi] = ok ? __ldcg(sp + pi * kBRows + r) : 0.0f;
                x1[u][pi] = (GATEUP && ok) ? __ldcg(sp + (kMaxPr + pi) * kBRows + r) : 0.0f;
            }
        }
#pragma unroll
        for (int u = 0; u < G; ++u) {
            if (sg0 + u >= nseg) break;
#pragma unroll
            for (int pi = 0; pi < NPM; ++pi) {
                acc0[pi] += x0[u][pi];
                if (GATEUP) acc1[pi] += x1[u][pi];
            }
        }
    }
}

template <bool GATEUP, bool SFRAW, bool SFBRAW>
__global__ void __launch_bounds__(kBThreads, 1)
    bs_gemv_kernel(const __grid_constant__ BMaps maps, const BArgs a) {
    static_assert(!(GATEUP && SFRAW), "row-major scales are read by the single-projection kernel only");
    static_assert(!SFBRAW || GATEUP, "raw piece scales are read by the gate/up kernel only");
    using St = BStage<GATEUP, SFRAW, SFBRAW>;
    constexpr int S = bstages<GATEUP, SFRAW, SFBRAW>();
    constexpr uint32_t kCols = btmem_cols<GATEUP>();
    constexpr int kAccW = GATEUP ? 128 : 64;               // TMEM columns per accumulator
    constexpr int kSf0 = 2 * kAccW;                        // first scale column
    constexpr int kSfW = GATEUP ? 24 : 16;                 // scale columns per stage
    constexpr int kMaxPr = kBMaxN / kBPieces;              // pairs per expert item (8)
    constexpr int kPW = GATEUP ? 2 * kMaxPr : kMaxPr;      // partial values per row
    static_assert(kSf0 + kSfW * S <= int(kCols), "TMEM plan exceeds the allocation");

    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    St* ring = reinterpret_cast<St*>(base);
    uint64_t* full = reinterpret_cast<uint64_t*>(base + sizeof(St) * S);
    uint64_t* empty = full + S;
    uint64_t* accf = empty + S;          // [2] accumulator ready (MMA -> epilogue)
    uint64_t* acce = accf + 2;           // [2] accumulator drained (epilogue -> MMA)
    uint64_t* drain = acce + 2;          // MMA teardown
    __shared__ uint32_t s_tmem;
    __shared__ Plan s_plan;                           // the routing plan, copied once
    __shared__ int s_last;
    __shared__ int s_nseg;
    __shared__ int s_seg[kBMaxSegments];
    __shared__ volatile int s_abort;
    __shared__ volatile unsigned s_issued;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        // the tensor-map descriptors are fetched while the prologue runs, not at the first
        // copy (about a microsecond each when cold)
        prefetch_tensormap(&maps.a0);
        if (GATEUP) prefetch_tensormap(&maps.a1);
        prefetch_tensormap(&maps.b);
        if (SFRAW) prefetch_tensormap(&maps.sfa);
        if (SFBRAW) prefetch_tensormap(&maps.sfb);
    }
    if (threadIdx.x == 0) {
        s_abort = 0;
        s_issued = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&accf[b], 1);
            mbar_init(&acce[b], kBEpiWarps);
        }
        mbar_init(drain, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    // the next launch (down, or the combine) may start its prologue (barriers, TMEM, plan
    // copy) now; it waits for this launch before reading anything it writes
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    if (warp == 1) tmem_alloc(&s_tmem, kCols);
    if (a.identity_m > 0) {
        // the identity plan (single-matrix matvec): items of 8 tokens, slot 0, weight 1
        const int Mi = a.identity_m, Vi = (Mi + kBMaxN / kBPieces - 1) / (kBMaxN / kBPieces);
        if (threadIdx.x == 0) {
            s_plan.n_active = Vi;
            s_plan.n_pairs = Mi;
            s_plan.M = Mi;
            s_plan.status = K3_OK;
        }
        for (int v = threadIdx.x; v <= Vi; v += blockDim.x) {
            if (v < Vi) s_plan.expert[v] = 0;
            s_plan.pair_start[v] = min(v * (kBMaxN / kBPieces), Mi);
        }
        for (int q = threadIdx.x; q < Mi; q += blockDim.x) {
            s_plan.pair_tok[q] = q;
            s_plan.pair_w[q] = 1.0f;
        }
    } else {
        // gate/up (plan_in_prev): the previous launch (router, prep or pairs plan) writes
        // the plan -- wait for it first. down: the plan is two launches old and was
        // complete when the previous launch (gate/up) started.
        if (a.plan_in_prev) asm volatile("griddepcontrol.wait;\n" ::: "memory");
        for (int i = threadIdx.x; i < int(sizeof(Plan) / 4); i += blockDim.x)
            reinterpret_cast<int*>(&s_plan)[i] = reinterpret_cast<const int*>(a.plan)[i];
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = s_tmem;

    // Keys: (128-row block rb, expert item v), key = rb * V + v (row-block major, so heavy
    // experts spread over CTAs); items = the key's C k-chunks.
    const Plan* P = &s_plan;
    // Item indices in 32-bit arithmetic (a 64-bit division by a runtime divisor is a long
    // dependent sequence, and the producer does four per item before its first request);
    // the host keeps (items) x (grid) below 2^32.
    const int V = P->n_active;
    const uint32_t uV = uint32_t(V);
    const uint32_t nRb = uint32_t(a.rows / kBRows);
    const uint32_t ipk = uint32_t(a.C);
    const uint32_t n = uV * nRb * ipk;
    const uint32_t grid = gridDim.x, bid = blockIdx.x;
    const uint32_t i0 = bid * n / grid, i1 = (bid + 1) * n / grid;
    const int64_t kchunk = a.K / a.C;
    const int nst = int(kchunk / kBStageK);
    const int64_t kcks = a.K / 128;                                   // scale chunks per row block

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const uint64_t stream_once = l2_evict_first();
            // what the stages of one item share (computed once per item: 64-bit divisions)
            struct Item {
                int v, rb, slot, ps, np, r0, tb;
                int64_t kbase;
                uint32_t bytes;
            };
            auto item_at = [&](uint32_t i) {
                Item it;
                const uint32_t key = i / ipk;
                it.v = int(key % uV);
                it.rb = int(key / uV);
                it.slot = P->expert[it.v];
                it.ps = P->pair_start[it.v];
                it.np = P->pair_start[it.v + 1] - it.ps;
                it.r0 = it.rb * kBRows;
                it.tb = it.slot * int(nRb) + it.rb;
                it.kbase = int64_t(i % ipk) * kchunk;
                it.bytes = uint32_t((GATEUP ? 2 : 1) * (kBRows * 128 + (SFRAW ? kBRows * 16 : 2 * kBChunk)) +
                                    it.np * kBPieces * 128 + (SFBRAW ? it.np * kBPieces * 16 : 2 * kBChunk));
                return it;
            };
            // the weight tiles and their scales of k-step s
            auto stage_a = [&](const Item& it, int s, int si) {
                St& st = ring[si];
                const int64_t k = it.kbase + int64_t(s) * kBStageK;
                const int64_t sfo = int64_t(it.slot) * a.sf_slot + (int64_t(it.rb) * kcks + k / 128) * kBChunk;
                if (a.tiled)
                    tma_4d_hint(&st.a[0][0][0], &maps.a0, 0, 0, int(k / kBStageK), it.tb, &full[si], stream_once);
                else
                    tma_3d_hint(&st.a[0][0][0], &maps.a0, int(k / 2), it.r0, it.slot, &full[si], stream_once);
                if constexpr (SFRAW)      // the 512-k scale box holding this stage's 256 k
                    tma_2d(&st.sfraw[0][0], &maps.sfa, int(k / 512) * 16, it.slot * int(a.rows) + it.r0, &full[si]);
                else
                    bulk_g2s_hint(&st.sfa[0][0], a.sfa0 + sfo, 2 * kBChunk, &full[si], stream_once);
                if (GATEUP) {
                    if (a.tiled)
                        tma_4d_hint(&st.a[GATEUP ? 1 : 0][0][0], &maps.a1, 0, 0, int(k / kBStageK), it.tb,
                                    &full[si], stream_once);
                    else
                        tma_3d_hint(&st.a[GATEUP ? 1 : 0][0][0], &maps.a1, int(k / 2), it.r0, it.slot, &full[si],
                                    stream_once);
                    bulk_g2s_hint(&st.sfa[GATEUP ? 1 : 0][0], a.sfa1 + sfo, 2 * kBChunk, &full[si], stream_once);
                }
            };
            // the activation pieces and their scale chunks of k-step s (written by the
            // previous launch)
            auto stage_b = [&](const Item& it, int s, int si) {
                St& st = ring[si];
                const int64_t k = it.kbase + int64_t(s) * kBStageK;
                if (GATEUP) {
                    for (int pi = 0; pi < it.np; ++pi) {    // one token's 8 piece rows per pair
                        const int row = kBPieces * P->pair_tok[it.ps + pi];
                        tma_2d(&st.b[kBPieces * pi][0], &maps.b, int(k / 2), row, &full[si]);
                        if constexpr (SFBRAW)                // and their scales' 512-k box
                            tma_2d(&st.sfbraw[kBPieces * pi][0], &maps.sfb, int(k / 512) * 16, row, &full[si]);
                    }
                } else {
                    for (int pi = 0; pi < it.np; ++pi)      // pair pi's 8 piece rows
                        tma_3d(&st.b[kBPieces * pi][0], &maps.b, int(k / 2), kBPieces * pi, it.v, &full[si]);
                }
                if constexpr (!SFBRAW)
                    bulk_g2s(&st.sfb[0], a.sfb + (int64_t(it.v) * kcks + k / 128) * kBChunk, 2 * kBChunk, &full[si]);
            };
            // Nothing of the weights comes from the previous launch: when allowed, request
            // the first stages' weight tiles and scales (the ring starts empty) before
            // waiting for it. (ie, se) is the first stage not yet requested.
            uint32_t ie = i0;
            int se = 0;
            uint32_t pre = 0;
            if (a.identity_m > 0 || a.early_a) {
                while (ie < i1 && pre < uint32_t(S)) {
                    const Item it = item_at(ie);
                    for (; se < nst && pre < uint32_t(S); ++se, ++pre) {
                        mbar_expect_tx(&full[pre], it.bytes);
                        stage_a(it, se, int(pre));
                    }
                    if (se == nst) {
                        se = 0;
                        ++ie;
                    }
                }
            }
            // The B operand (token or activation pieces and their scale chunks) comes from
            // the previous launch, which may still be running (programmatic dependent
            // launch): wait for it before the first request of it.
            asm volatile("griddepcontrol.wait;\n" ::: "memory");
            {
                uint32_t g = 0;
                for (uint32_t i = i0; g < pre; ++i) {
                    const Item it = item_at(i);
                    for (int s = 0; s < nst && g < pre; ++s, ++g) {
                        stage_b(it, s, int(g));
                        s_issued = g + 1;
                    }
                }
            }
            uint32_t gs = pre;
            for (uint32_t i = ie; i < i1 && !s_abort; ++i) {
                const Item it = item_at(i);
                for (int s = (i == ie ? se : 0); s < nst; ++s, ++gs) {
                    const int si = int(gs % S);
                    if (!mbar_wait(&empty[si], ((gs / S) & 1) ^ 1, a.status, &s_abort)) {
                        s_abort = 1;
                        break;
                    }
                    mbar_expect_tx(&full[si], it.bytes);
                    stage_a(it, s, si);
                    stage_b(it, s, si);
                    s_issued = gs + 1;
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA issuer
        // The whole warp runs the loop (warp-uniform descriptors); one elected lane issues.
        uint32_t gs = 0, ib = 0;
        for (uint32_t i = i0; i < i1 && !s_abort; ++i, ++ib) {
            const int v = int((i / ipk) % uV);
            const int np = P->pair_start[v + 1] - P->pair_start[v];
            const int nb = kBPieces * np;                                // MMA N
            // SFRAW: parity of the item's first 256-k step (which half of a 512-k scale box)
            const int half0 = (SFRAW || SFBRAW) ? int(((i % ipk) * uint32_t(nst)) & 1u) : 0;
            const uint32_t buf = ib & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&acce[buf], ((ib >> 1) & 1) ^ 1, a.status, &s_abort))) {
                s_abort = 1;
                break;
            }
            tc_fence_after();
            const uint32_t d0 = tm + buf * kAccW;                        // gate (or down)
            const uint32_t d1 = d0 + 64;                                 // up
            const uint32_t idesc0 = mxf4_idesc(nb, 0), idesc2 = mxf4_idesc(nb, 2);
            for (int s = 0; s < nst; ++s, ++gs) {
                const int si = int(gs % S);
                if (!__all_sync(0xffffffffu, mbar_wait(&full[si], (gs / S) & 1, a.status, &s_abort))) {
                    s_abort = 1;
                    break;
                }
                tc_fence_after();
                St& st = ring[si];
                if constexpr (SFRAW) {
                    // the stage's two scale chunks from its 8 bytes of every row of the raw
                    // box: lane l writes rows l + 32c, byte j of chunk h at l*16 + 4c + j
                    const int half = (half0 + s) & 1;
                    uint32_t w0[4], w1[4];
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const uint2 v2 = *reinterpret_cast<const uint2*>(&st.sfraw[32 * c + lane][8 * half]);
                        w0[c] = v2.x;
                        w1[c] = v2.y;
                    }
                    *reinterpret_cast<uint4*>(&st.sfa[0][16 * lane]) = make_uint4(w0[0], w0[1], w0[2], w0[3]);
                    *reinterpret_cast<uint4*>(&st.sfa[0][kBChunk + 16 * lane]) = make_uint4(w1[0], w1[1], w1[2], w1[3]);
                    // generic-proxy writes, read next by tcgen05.cp (async proxy)
                    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
                    __syncwarp();
                }
                if constexpr (SFBRAW) {
                    // the same for the piece scales: B row m (pair m / 8, piece m % 8), lane
                    // l takes rows l and l + 32, its 8 bytes of the stage's half of the box
                    const int half = (half0 + s) & 1;
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        const int m = lane + 32 * c;
                        if (m < nb) {
                            const uint2 v2 = *reinterpret_cast<const uint2*>(&st.sfbraw[m][8 * half]);
                            *reinterpret_cast<uint32_t*>(&st.sfb[sf_chunk_offset(m, 0)]) = v2.x;
                            *reinterpret_cast<uint32_t*>(&st.sfb[kBChunk + sf_chunk_offset(m, 0)]) = v2.y;
                        }
                    }
                    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
                    __syncwarp();
                }
                const uint32_t sf = tm + kSf0 + kSfW * si;
                const uint32_t sfa0 = sf, sfa1 = sf + 8, sfb = sf + (GATEUP ? 16 : 8);
                if (elect_one()) {
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        tc_cp_sf(sfa0 + 4 * c, sf_chunk_desc(&st.sfa[0][c * kBChunk]));
                        if (GATEUP) tc_cp_sf(sfa1 + 4 * c, sf_chunk_desc(&st.sfa[GATEUP ? 1 : 0][c * kBChunk]));
                        tc_cp_sf(sfb + 4 * c, sf_chunk_desc(&st.sfb[c * kBChunk]));
                    }
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint32_t id = 2 * (kk & 1), ch = 4 * (kk >> 1);
                        const uint32_t idesc = (kk & 1) ? idesc2 : idesc0;
                        const uint32_t acc = (s > 0 || kk > 0) ? 1u : 0u;
                        const uint64_t bd = sw128_desc(&st.b[0][0], 32 * kk);
                        mma_mxf4(d0, sw128_desc(&st.a[0][0][0], 32 * kk), bd, idesc, (sfa0 + ch) | (id << 30),
                                 (sfb + ch) | (id << 30), acc);
                        if (GATEUP)
                            mma_mxf4(d1, sw128_desc(&st.a[GATEUP ? 1 : 0][0][0], 32 * kk), bd, idesc,
                                     (sfa1 + ch) | (id << 30), (sfb + ch) | (id << 30), acc);
                    }
                    tc_commit(&empty[si]);
                }
                __syncwarp();
            }
            if (s_abort) break;
            if (elect_one()) tc_commit(&accf[buf]);
            __syncwarp();
        }
        if (s_abort) {
            // the producer's copies in flight land before the CTA leaves
            const unsigned issued = s_issued;
            for (unsigned k = gs; k < issued; ++k)
                if (!mbar_wait(&full[k % S], (k / S) & 1, a.status)) break;
        }
        // every tcgen05 operation of this warp completes before TMEM is released
        if (elect_one()) tc_commit(drain);
        __syncwarp();
        mbar_wait(drain, 0, a.status);
    } else {
        // ------------------------------------------------------------ epilogue
        const int q = warp & 3;                               // TMEM lane quarter
        const int r = 32 * q + lane;                          // weight row within the tile
        const int et = int(threadIdx.x) - 64;                 // 0..127
        const uint32_t lane_addr = uint32_t(32 * q) << 16;
        float acc0[kMaxPr], acc1[kMaxPr];                     // per pair: gate (or down), up
#pragma unroll
        for (int pi = 0; pi < kMaxPr; ++pi) acc0[pi] = acc1[pi] = 0.0f;
        uint32_t ib = 0;
        for (uint32_t i = i0; i < i1; ++i, ++ib) {
            const uint32_t key = i / ipk;
            const int v = int(key % uV), rb = int(key / uV);
            const int ps = P->pair_start[v], np = P->pair_start[v + 1] - ps;
            const uint32_t buf = ib & 1;
            const bool ok = mbar_wait(&accf[buf], (ib >> 1) & 1, a.status, &s_abort);
            if (ok) {
                tc_fence_after();
                const uint32_t d0 = tm + lane_addr + buf * kAccW;
#pragma unroll
                for (int c = 0; c < kMaxPr / 2; ++c) {
                    if (2 * c >= np) break;
                    float x[16];
                    tmem_ld16(d0 + 16 * c, x);
                    acc0[2 * c] += sum8(x);
                    acc0[2 * c + 1] += sum8(x + 8);               // past np: unused garbage
                    if (GATEUP) {
                        tmem_ld16(d0 + 64 + 16 * c, x);
                        acc1[2 * c] += sum8(x);
                        acc1[2 * c + 1] += sum8(x + 8);
                    }
                }
                tc_fence_before();
            } else {
                s_abort = 1;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&acce[buf]);
            // every epilogue warp reads the abort flag after the same barrier, so all leave
            // together when a wait gave up
            epi_sync();
            if (s_abort) break;
            if (i + 1 < i1 && (i + 1) / ipk == key) continue;

            // ---- flush the key
            const uint32_t ks = key * ipk;
            const bool local = ipk == 1 || (ks >= i0 && ks + ipk <= i1);
            float* kpart = a.part + int64_t(key) * a.maxseg * (kPW * kBRows);
            if (!local) {
                const int64_t seg = int64_t((i0 > ks ? i0 : ks) - ks);
                float* sp = kpart + seg * (kPW * kBRows);
#pragma unroll
                for (int pi = 0; pi < kMaxPr; ++pi) {
                    sp[pi * kBRows + r] = acc0[pi];
                    if (GATEUP) sp[(kMaxPr + pi) * kBRows + r] = acc1[pi];
                }
                __threadfence();
                if (et == 0) {
                    // the key's segments: one per CTA b owning items of it, starting at that
                    // CTA's first item (CTAs with empty ranges own nothing)
                    int ns = 0;
                    const uint32_t b0 = owner_of(ks, n, grid), b1 = owner_of(ks + ipk - 1, n, grid);
                    for (uint32_t cb = b0; cb <= b1 && ns < kBMaxSegments; ++cb) {
                        const uint32_t f0 = cb * n / grid, f1 = (cb + 1) * n / grid;
                        if (f1 > f0) s_seg[ns++] = int((f0 > ks ? f0 : ks) - ks);
                    }
                    s_nseg = ns;
                }
            }
            if (!local) {
                epi_sync();
                if (et == 0) s_last = !s_abort && atomicAdd(a.cnt + key, 1u) + 1 == unsigned(s_nseg);
                epi_sync();
                if (s_abort) break;
            }
            if (!local && !s_last) {
#pragma unroll
                for (int pi = 0; pi < kMaxPr; ++pi) acc0[pi] = acc1[pi] = 0.0f;
                continue;
            }
            if (!local) {
                __threadfence();
#pragma unroll
                for (int pi = 0; pi < kMaxPr; ++pi) acc0[pi] = acc1[pi] = 0.0f;
                // segment order: deterministic sums. Only the key's np pairs are read; in the
                // projection kernels, the fewer they are, the more segments' loads are in
                // flight at once (in gate/up the wider merge's registers cost more than its
                // round trips save: measured)
                const int nseg = s_nseg;
                if (GATEUP || np > 4) sum_segments<4, kMaxPr, GATEUP>(kpart, s_seg, nseg, np, r, acc0, acc1);
                else if (np <= 2) sum_segments<16, 2, GATEUP>(kpart, s_seg, nseg, np, r, acc0, acc1);
                else sum_segments<8, 4, GATEUP>(kpart, s_seg, nseg, np, r, acc0, acc1);
            }
            if (GATEUP) {
                // activation x routing weight per pair, split into the down kernel's pieces,
                // up to four pairs interleaved
                const int64_t rowb = a.rows / 2;                            // bytes per act row (I/2)
                uint8_t* sfc = a.act_sf + (int64_t(v) * (a.rows / 128) + rb) * kBChunk;
#pragma unroll 1
                for (int p0 = 0; p0 < np; p0 += 4) {
                    float xv[4];
                    uint8_t* d[4];
                    uint8_t* sf[4];
#pragma unroll
                    for (int h = 0; h < 4; ++h) {
                        const int pi = p0 + h;
                        float gv = 0.0f, uv = 0.0f;
#pragma unroll
                        for (int pp = 0; pp < kMaxPr; ++pp)
                            if (pp == pi) { gv = acc0[pp]; uv = acc1[pp]; }
                        xv[h] = pi < np ? act_value(a.act_kind, gv, uv, a.beta, a.lbeta) * P->pair_w[ps + pi] : 0.0f;
                        d[h] = a.act_p + (int64_t(v) * kBMaxN + kBPieces * pi) * rowb + (int64_t(rb) * kBRows + 32 * q) / 2;
                        sf[h] = pi < np ? sfc + sf_chunk_offset(kBPieces * pi, q) : nullptr;
                    }
                    // a single pair (every routed expert at M = 1): one chain, not four
                    // with three idle (the last item's split is the launch's tail)
                    if (np - p0 == 1) {
                        const float x1[1] = {xv[0]};
                        uint8_t* const d1[1] = {d[0]};
                        uint8_t* const s1[1] = {sf[0]};
                        split_pieces_n<1>(x1, lane, d1, rowb, s1, 16);
                    } else {
                        split_pieces_n<4>(xv, lane, d, rowb, sf, 16);
                    }
                }
            } else {
                // one output row per pair (the combine kernel sums a token's pairs)
                const int64_t row = int64_t(rb) * kBRows + r;
#pragma unroll
                for (int pi = 0; pi < kMaxPr; ++pi)
                    if (pi < np) {
                        if (a.y_bf16)
                            reinterpret_cast<__nv_bfloat16*>(a.y_pair)[int64_t(ps + pi) * a.rows + row] =
                                __float2bfloat16_rn(acc0[pi]);
                        else
                            a.y_pair[int64_t(ps + pi) * a.rows + row] = acc0[pi];
                    }
            }
            if (!local && et == 0) a.cnt[key] = 0u;        // ready for the next call
            if (!local) epi_sync();                          // s_seg is rewritten by the next key
#pragma unroll
            for (int pi = 0; pi < kMaxPr; ++pi) acc0[pi] = acc1[pi] = 0.0f;
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tm, kCols);
}

// ------------------------------------------------------------------- combine

// y[t][h] = sum of y_pair[p][h] over the pairs p of token t in plan order (experts
// ascending, the shared expert last), like the reference's per-expert y.at[ti].add
// loop (air_llm/models/kimi_k3/moe.py:120-131). Block (x, t): token t, 512 columns of h;
// warp 0 lists the token's pairs in order with ballots, every thread sums 4 columns.
__global__ void combine_kernel(const Plan* __restrict__ plan, const float* __restrict__ y_pair, int64_t H,
                               void* y, int y_dtype) {
    __shared__ int s_list[kMaxPairs];
    __shared__ int s_n;
    const int t = blockIdx.y;
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        const int np = plan->n_pairs;
        int cnt = 0;
        for (int p0 = 0; p0 < np; p0 += 32) {
            const int p = p0 + lane;
            const bool mine = p < np && plan->pair_tok[p] == t;
            const uint32_t bal = __ballot_sync(0xffffffffu, mine);
            if (mine) s_list[cnt + __popc(bal & ((1u << lane) - 1u))] = p;
            cnt += __popc(bal);
        }
        if (lane == 0) s_n = cnt;
    }
    __syncthreads();
    asm volatile("griddepcontrol.wait;\n" ::: "memory");     // y_pair comes from the down launch
    const int64_t h4 = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
    if (h4 >= H) return;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int j0 = 0; j0 < s_n; j0 += 8) {            // eight rows in flight, summed in order
        float4 v[8];
#pragma unroll
        for (int h = 0; h < 8; ++h)
            v[h] = j0 + h < s_n ? __ldcg(reinterpret_cast<const float4*>(y_pair + int64_t(s_list[j0 + h]) * H + h4))
                                : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
        for (int h = 0; h < 8; ++h) {
            if (j0 + h >= s_n) break;
            acc.x += v[h].x;
            acc.y += v[h].y;
            acc.z += v[h].z;
            acc.w += v[h].w;
        }
    }
    const int64_t o = int64_t(t) * H + h4;
    store_from_f32(y, y_dtype, o, acc.x);
    store_from_f32(y, y_dtype, o + 1, acc.y);
    store_from_f32(y, y_dtype, o + 2, acc.z);
    store_from_f32(y, y_dtype, o + 3, acc.w);
}

int launch_combine(const Plan* plan, const float* y_pair, int64_t H, int M, void* y, int y_dtype,
                   cudaStream_t s) {
    const dim3 grid(unsigned((H / 4 + 127) / 128), unsigned(M));
    return cuda_check(launch_pdl(combine_kernel, grid, dim3(128), 0, s, plan, y_pair, H, y, y_dtype), "combine_kernel");
}

// ---------------------------------------------------------------- scale layout

__global__ void scales_tc_kernel(const uint8_t* __restrict__ in, int64_t rows, int64_t cols,
                                 int64_t total_chunks, uint8_t* __restrict__ out) {
    // one thread per (chunk, row): 4 scale bytes
    const int64_t kc = cols / 128;                 // chunks per row block
    const int64_t g = cols / 32;                   // scale bytes per row
    for (int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < total_chunks * 128;
         idx += int64_t(gridDim.x) * blockDim.x) {
        const int64_t chunk = idx / 128;
        const int m = int(idx % 128);
        const int64_t c = chunk % kc;
        const int64_t rbk = chunk / kc;            // (batch, row block)
        const int64_t row = rbk * 128 + m;         // row in the flattened [batch*rows]
        const uint8_t* src = in + row * g + c * 4;
        uint8_t* dst = out + chunk * kBChunk;
#pragma unroll
        for (int j = 0; j < 4; ++j) dst[sf_chunk_offset(m, j)] = src[j];
    }
    (void)rows;
}

__global__ void tiles_kernel(const uint4* __restrict__ in, int64_t rows, int64_t cols, int64_t total,
                             uint4* __restrict__ out) {
    // one thread per 16 bytes of the output, in output order (coalesced writes)
    const int64_t rowb = cols / 32;                // 16-byte units per row
    const int64_t kt_n = cols / 256;               // tiles per row block
    for (int64_t o = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; o < total;
         o += int64_t(gridDim.x) * blockDim.x) {
        const int64_t c16 = o & 7;                 // 16-byte unit within the tile row
        const int64_t r = (o >> 3) & 127;          // row within the tile
        const int64_t t = o >> 10;                 // tile index (batch, row block, k tile)
        const int64_t kt = t % kt_n;
        const int64_t rbk = t / kt_n;              // (batch, row block) in [batch * rows/128]
        out[o] = in[(rbk * 128 + r) * rowb + kt * 8 + c16];
    }
    (void)rows;
}

int launch_tiles(const uint8_t* in, int64_t rows, int64_t cols, int64_t batch, uint8_t* out,
                 cudaStream_t s) {
    const int64_t total = batch * rows * cols / 32;          // 16-byte units
    const int blocks = int(std::min<int64_t>((total + 255) / 256, int64_t(num_sms()) * 32));
    tiles_kernel<<<blocks, 256, 0, s>>>(reinterpret_cast<const uint4*>(in), rows, cols, total,
                                        reinterpret_cast<uint4*>(out));
    K3_CHECK_LAUNCH("tiles_kernel");
    return K3_OK;
}

int launch_scales_tc(const uint8_t* in, int64_t rows, int64_t cols, int64_t batch, uint8_t* out,
                     cudaStream_t s) {
    const int64_t chunks = batch * (rows / 128) * (cols / 128);
    const int64_t threads = chunks * 128;
    const int blocks = int(std::min<int64_t>((threads + 255) / 256, int64_t(num_sms()) * 16));
    scales_tc_kernel<<<blocks, 256, 0, s>>>(in, rows, cols, chunks, out);
    K3_CHECK_LAUNCH("scales_tc_kernel");
    return K3_OK;
}

// ------------------------------------------------------------------ launches

template <bool G, bool SFRAW = false, bool SFBRAW = false>
int launch_bs(const BMaps& maps, const BArgs& a, int grid, cudaStream_t s, const char* what) {
    if (grid > kBMaxSegments) return fail(K3_ERR_UNSUPPORTED, "block-scaled grid above 256 CTAs");
    // item indices are 32-bit in the kernel: (items of at most kMaxActive experts) x grid
    if (uint64_t(kMaxActive) * uint64_t(a.rows / kBRows) * uint64_t(a.C) * uint64_t(grid) >= (uint64_t(1) << 32))
        return fail(K3_ERR_UNSUPPORTED, "block-scaled launch: too many items for 32-bit indices");
    static OncePerContext attr;
    constexpr size_t smem = bsmem_bytes<G, SFRAW, SFBRAW>();
    if (int rc = attr.run([&] {
            return cuda_check(cudaFuncSetAttribute(bs_gemv_kernel<G, SFRAW, SFBRAW>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
                              what);
        }))
        return rc;
    if (int rc = cuda_check(launch_pdl(bs_gemv_kernel<G, SFRAW, SFBRAW>, dim3(unsigned(grid)), dim3(kBThreads),
                                       smem, s, maps, a),
                            what))
        return rc;
    return K3_OK;
}

int launch_bs_gateup(const BMaps& maps, const BArgs& a, int grid, cudaStream_t s) {
    return launch_bs<true>(maps, a, grid, s, "bs_gemv<gate/up>");
}
int launch_bs_gateup_rawsfb(const BMaps& maps, const BArgs& a, int grid, cudaStream_t s) {
    if (!a.plan_in_prev) return fail(K3_ERR_INVALID, "bs_gemv<gate/up, raw piece scales>: plan_in_prev unset");
    return launch_bs<true, false, true>(maps, a, grid, s, "bs_gemv<gate/up, raw piece scales>");
}
int launch_bs_down(const BMaps& maps, const BArgs& a, int grid, cudaStream_t s) {
    return launch_bs<false>(maps, a, grid, s, "bs_gemv<down>");
}
int launch_bs_proj_rawsf(const BMaps& maps, const BArgs& a, int grid, cudaStream_t s) {
    return launch_bs<false, true>(maps, a, grid, s, "bs_gemv<projection, stored scales>");
}

}  // namespace k3

extern "C" K3_API int k3_mxfp4_scales_tc(const uint8_t* scales, int64_t rows, int64_t cols,
                                         int64_t batch, uint8_t* out, void* stream) {
    using namespace k3;
    if (!scales || !out) return fail(K3_ERR_INVALID, "k3_mxfp4_scales_tc: NULL tensor");
    if (rows < 128 || cols < 128 || batch < 1 || rows % 128 || cols % 128)
        return fail(K3_ERR_UNSUPPORTED, "k3_mxfp4_scales_tc: rows and cols must be positive multiples of 128");
    return launch_scales_tc(scales, rows, cols, batch, out, static_cast<cudaStream_t>(stream));
}

extern "C" K3_API int k3_mxfp4_tiles(const uint8_t* packed, int64_t rows, int64_t cols, int64_t batch,
                                     uint8_t* out, void* stream) {
    using namespace k3;
    if (!packed || !out) return fail(K3_ERR_INVALID, "k3_mxfp4_tiles: NULL tensor");
    if (rows < 128 || cols < 256 || batch < 1 || rows % 128 || cols % 256)
        return fail(K3_ERR_UNSUPPORTED, "k3_mxfp4_tiles: rows % 128 == 0 and cols % 256 == 0 required");
    if (reinterpret_cast<uintptr_t>(packed) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
        return fail(K3_ERR_INVALID, "k3_mxfp4_tiles: tensors must be 16-byte aligned");
    return launch_tiles(packed, rows, cols, batch, out, static_cast<cudaStream_t>(stream));
}
