// Prefill path (T tokens per call, T in the thousands) on the 5th-generation tensor cores:
// router GEMM, routing plan, activation pieces and the two block-scaled grouped GEMMs.
//
// The reference runs every routed expert of a layer over its token subset in a Python loop
// (air_llm/models/kimi_k3/moe.py:110-132, oracle k3ref/layers.py:241-261), one MXFP4
// matvec launch per projection; here one launch per phase covers every (expert, token)
// pair of the call:
//
//   gemm_bf16_kernel      logits [T][E] = x . W_g^T on tcgen05 kind::f16 (bf16 x bf16 ->
//                         fp32 in TMEM; k3_gemm.cu), then the shared sigmoid top-k kernel;
//   prefill_count/scan/place_kernel
//                         the pairs grouped by slot (experts ascending, shared last),
//                         candidates in order within a slot, cut into chunks of <= kPN
//                         pairs; per-CTA item ranges balanced by cost;
//   prefill_pieces_kernel x -> kPPieces E2M1 pieces [P][T][H/2] + E8M0 scales [P][T][H/32];
//   prefill_gemm_kernel   per item (chunk, 128-row block pair): weights by TMA from the
//                         tile pools, the chunk's token pieces gathered into the swizzled
//                         B tile by cp.async (gate/up) or TMA (down), kind::mxf4 MMAs into
//                         double-buffered TMEM accumulators, epilogue warps draining the
//                         other buffer.
#include "k3_async.cuh"
#include "k3_gemm.cuh"
#include "k3_pairs.cuh"
#include "k3_prefill.cuh"
#include "k3_tma.cuh"

namespace k3 {

int launch_router_logits_rows(const void* x, int xdt, int64_t M, int64_t H, const uint16_t* W,
                              int64_t E, float* logits, cudaStream_t s);
int launch_topk_rows(const float* logits, int64_t M, int64_t E, const float* bias, int k, int renorm,
                     float scale, int32_t* idx, float* w, int* status, cudaStream_t s);
bool router_gemm_ok(int xdt, int64_t H, const void* x, const void* gate_w);
int launch_router_gemm(const void* x, int64_t T, int64_t H, const uint16_t* gate_w, int64_t E, float* logits,
                       int* status, cudaStream_t s);

namespace {

// ------------------------------------------------------------------ primitives

// Four consecutive floats reduce-added at once (16-byte aligned).
__device__ __forceinline__ void red_add_v4(float* p, float4 v, uint64_t policy) {
    asm volatile("red.global.add.L2::cache_hint.v4.f32 [%0], {%1, %2, %3, %4}, %5;\n" ::"l"(p), "f"(v.x), "f"(v.y),
                 "f"(v.z), "f"(v.w), "l"(policy)
                 : "memory");
}
// Barrier of the four epilogue warps (named barrier 1).
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, %0;\n" ::"n"(kPEpiWarps * 32) : "memory"); }
__device__ __forceinline__ uint64_t l2_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;\n" : "=l"(p));
    return p;
}


// ------------------------------------------------------------------ routing plan

__device__ __forceinline__ void prefill_cand(const PrefillCand& c, int i, int& slot, int& tok, float& w) {
    if (c.slot) {
        slot = c.slot[i];
        tok = c.tok[i];
        w = c.pw[i];
        if (tok < 0 || tok >= c.T) slot = -1;
    } else if (i < c.T * c.k) {
        const int t = i / c.k, j = i - t * c.k;
        const int e = c.idx[int64_t(t) * c.rstride + j] - c.expert_lo;
        slot = (e >= 0 && e < c.n_local) ? e : -1;
        tok = t;
        w = c.w[int64_t(t) * c.rstride + j];
    } else {
        slot = c.shared_slot;
        tok = c.shared_t0 + (i - c.T * c.k);
        w = 1.0f;
    }
    if (slot < 0 || slot >= c.num_slots || tok < 0 || tok >= c.T) slot = -1;
}

// Candidates of this block as per-slot bit masks (bit = candidate index in the block).
__device__ __forceinline__ int build_masks(const PrefillCand& c, int n_cand, uint32_t* mask, int& tok,
                                           float& w) {
    const int NS = c.num_slots;
    for (int i = threadIdx.x; i < NS * 8; i += blockDim.x) mask[i] = 0;
    __syncthreads();
    const int i = blockIdx.x * kPPlanBlock + threadIdx.x;
    int sl = -1;
    tok = 0;
    w = 0.0f;
    if (i < n_cand) prefill_cand(c, i, sl, tok, w);
    if (sl >= 0) atomicOr(&mask[sl * 8 + (threadIdx.x >> 5)], 1u << (threadIdx.x & 31));
    __syncthreads();
    return sl;
}

__global__ void __launch_bounds__(kPPlanBlock) prefill_count_kernel(const __grid_constant__ PrefillCand c,
                                                                    int n_cand, int* blk_cnt) {
    extern __shared__ uint32_t mask[];
    int tok;
    float w;
    build_masks(c, n_cand, mask, tok, w);
    const int NS = c.num_slots;
    for (int s = threadIdx.x; s < NS; s += blockDim.x) {
        int n = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) n += __popc(mask[s * 8 + j]);
        blk_cnt[int64_t(blockIdx.x) * NS + s] = n;
    }
}

// Exclusive scan of v[0..n) into out[0..n] (out[n] = total) by one block; out may be v.
__device__ void block_exclusive_scan(const int* v, int n, int* out, int* s_warp) {
    const int per = (n + int(blockDim.x) - 1) / int(blockDim.x);
    const int b0 = int(threadIdx.x) * per;
    int sum = 0;
    for (int j = 0; j < per; ++j)
        if (b0 + j < n) sum += v[b0 + j];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    int x = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int wv = lane < nw ? s_warp[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, wv, o);
            if (lane >= o) wv += y;
        }
        s_warp[lane] = wv;
    }
    __syncthreads();
    int excl = x - sum + (warp > 0 ? s_warp[warp - 1] : 0);
    for (int j = 0; j < per; ++j)
        if (b0 + j < n) {
            const int val = v[b0 + j];
            out[b0 + j] = excl;
            excl += val;
        }
    if (threadIdx.x == blockDim.x - 1) out[n] = excl;
    __syncthreads();
}

// One warp per slot: the per-block counts of the slot -> per-block bases (exclusive
// scan over blocks); the slot's total count goes to cnt[s].
__global__ void __launch_bounds__(256) prefill_blkscan_kernel(int* blk_cnt, int nblk, int NS, int* cnt) {
    const int s = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (s >= NS) return;
    int carry = 0;
    for (int b0 = 0; b0 < nblk; b0 += 32) {
        const int b = b0 + lane;
        const int64_t o = int64_t(b) * NS + s;
        const int v = b < nblk ? blk_cnt[o] : 0;
        int x = v;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, d);
            if (lane >= d) x += y;
        }
        if (b < nblk) blk_cnt[o] = carry + x - v;
        carry += __shfl_sync(0xffffffffu, x, 31);
    }
    if (lane == 0) cnt[s] = carry;
}

// One block: per-slot counts (in P.off) -> pair offsets, chunks (a slot's n pairs split
// into ceil(n / kPN) chunks of near-equal size), the chunks' row prefix.
__global__ void __launch_bounds__(1024) prefill_scan_kernel(const __grid_constant__ PrefillPlan P, int NS,
                                                            int nc_max) {
    __shared__ int s_cnt[kPMaxSlots + 1];
    __shared__ int s_warp[32];
    for (int s = threadIdx.x; s < NS; s += blockDim.x) s_cnt[s] = P.off[s];
    __syncthreads();
    block_exclusive_scan(s_cnt, NS, P.off, s_warp);              // P.off[s] = first pair of s
    for (int s = threadIdx.x; s < NS; s += blockDim.x) s_cnt[s] = (s_cnt[s] + kPN - 1) / kPN;
    __syncthreads();
    block_exclusive_scan(s_cnt, NS, P.ch_first, s_warp);         // first chunk of s
    const int NC = P.ch_first[NS];
    if (threadIdx.x == 0) {
        P.hdr->n_pairs = P.off[NS];
        P.hdr->n_chunks = NC <= nc_max ? NC : nc_max;
        if (NC > nc_max) atomicExch(&P.hdr->status, K3_ERR_UNSUPPORTED);
    }
    for (int s = threadIdx.x; s < NS; s += blockDim.x) {
        const int n = P.off[s + 1] - P.off[s];
        const int c0 = P.ch_first[s], nc = P.ch_first[s + 1] - c0;
        if (nc == 0) continue;
        const int base = n / nc, rem = n % nc;
        int p = P.off[s];
        for (int j = 0; j < nc && c0 + j < nc_max; ++j) {
            const int sz = base + (j < rem ? 1 : 0);
            P.ch_slot[c0 + j] = s;
            P.ch_p0[c0 + j] = p;
            P.ch_n[c0 + j] = sz;
            P.ch_n8p[c0 + j] = (sz + 7) & ~7;
            p += sz;
        }
    }
    __syncthreads();
    block_exclusive_scan(P.ch_n8p, NC <= nc_max ? NC : nc_max, P.ch_n8p, s_warp);
}

// Each candidate's pair position (slot-grouped, candidate order within a slot) and its
// (chunk, row).
__global__ void __launch_bounds__(kPPlanBlock) prefill_place_kernel(const __grid_constant__ PrefillCand c,
                                                                    int n_cand,
                                                                    const __grid_constant__ PrefillPlan P) {
    extern __shared__ uint32_t mask[];
    int tok;
    float w;
    const int sl = build_masks(c, n_cand, mask, tok, w);
    if (sl < 0) return;
    const uint32_t* m = mask + sl * 8;
    const int wi = threadIdx.x >> 5;
    int rank = __popc(m[wi] & ((1u << (threadIdx.x & 31)) - 1u));
    for (int j = 0; j < wi; ++j) rank += __popc(m[j]);
    const int li = P.blk_cnt[int64_t(blockIdx.x) * c.num_slots + sl] + rank;   // index within the slot
    const int pos = P.off[sl] + li;
    const int n = P.off[sl + 1] - P.off[sl];
    const int nc = P.ch_first[sl + 1] - P.ch_first[sl];
    const int base = n / nc, rem = n % nc;
    int cl, row;
    if (li < rem * (base + 1)) {
        cl = li / (base + 1);
        row = li - cl * (base + 1);
    } else {
        const int l2 = li - rem * (base + 1);
        cl = rem + l2 / base;
        row = l2 - (l2 / base) * base;
    }
    P.pair_tok[pos] = tok;
    P.pair_w[pos] = w;
    P.pair_cj[pos] = ((P.ch_first[sl] + cl) << 8) | row;
}

// ------------------------------------------------------------------ activation pieces

// E2M1 pair (a -> high nibble, b -> low nibble), round to nearest even, saturating.
__device__ __forceinline__ uint32_t cvt_e2m1x2(float a, float b) {
    uint32_t r;
    asm("{\n .reg .b8 t;\n cvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n cvt.u32.u8 %0, t;\n}\n"
        : "=r"(r)
        : "f"(a), "f"(b));
    return r;
}
// The two values of an E2M1 pair (low nibble first).
__device__ __forceinline__ void e2m1x2_values(uint32_t byte, float& lo, float& hi) {
    uint32_t h2;
    asm("{\n .reg .b8 t;\n cvt.u8.u32 t, %1;\n cvt.rn.f16x2.e2m1x2 %0, t;\n}\n" : "=r"(h2) : "r"(byte));
    const __half2 v = *reinterpret_cast<const __half2*>(&h2);
    lo = __low2float(v);
    hi = __high2float(v);
}

// One 32-element block held by one thread -> NP E2M1 pieces: piece p's 16 packed bytes
// (element 2i in the low nibble of byte i) and E8M0 scale byte. Piece p holds what pieces
// 0..p-1 left over: scale = the smallest power of two S with max |remainder| <= 6 S,
// values rounded to the E2M1 grid (ties to even); the subtraction of each piece is exact.
template <int NP>
__device__ __forceinline__ void split_block32(float (&r)[32], uint4 (&data)[NP], uint32_t (&sf)[NP]) {
#pragma unroll
    for (int p = 0; p < NP; ++p) {
        uint32_t mb = 0;
#pragma unroll
        for (int i = 0; i < 32; ++i) mb = max(mb, __float_as_uint(r[i]) & 0x7fffffffu);
        int b = int(mb >> 23) - 2 + ((mb & 0x7fffffu) > 0x400000u ? 1 : 0);
        b = mb == 0 ? 1 : (b < 1 ? 1 : (b > 253 ? 253 : b));
        const float S = __uint_as_float(uint32_t(b) << 23);
        const float inv = __uint_as_float(uint32_t(254 - b) << 23);
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint32_t word = 0;
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                const int i = 8 * q + 2 * h;
                const uint32_t byte = cvt_e2m1x2(r[i + 1] * inv, r[i] * inv);
                float q0, q1;
                e2m1x2_values(byte, q0, q1);
                r[i] = fmaf(-q0, S, r[i]);
                r[i + 1] = fmaf(-q1, S, r[i + 1]);
                word |= byte << (8 * h);
            }
            w[q] = word;
        }
        data[p] = make_uint4(w[0], w[1], w[2], w[3]);
        sf[p] = uint32_t(b);
    }
}

// One thread per (token t, 32-block g): x[t][32g..32g+32) -> pieces at
// xp[(p*T + t)*(K/2) + 16g] and scales xsf[(p*T + t)*(K/32) + g].
template <int NP>
__global__ void __launch_bounds__(256) prefill_pieces_kernel(const void* __restrict__ x, int xdt, int T, int64_t K,
                                                             uint8_t* __restrict__ xp, uint8_t* __restrict__ xsf) {
    const int64_t G = K / 32;
    const int64_t id = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (id >= int64_t(T) * G) return;
    const int64_t t = id / G, g = id - t * G;
    float r[32];
    if (xdt == K3_BF16) {
        const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(x) + t * K + 32 * g);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint4 v = __ldg(src + q);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                r[8 * q + 2 * j] = __uint_as_float(w[j] << 16);
                r[8 * q + 2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
            }
        }
    } else {
        const float4* src = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + t * K + 32 * g);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float4 v = __ldg(src + q);
            r[4 * q] = v.x;
            r[4 * q + 1] = v.y;
            r[4 * q + 2] = v.z;
            r[4 * q + 3] = v.w;
        }
    }
    uint4 d[NP];
    uint32_t sf[NP];
    split_block32<NP>(r, d, sf);
#pragma unroll
    for (int p = 0; p < NP; ++p) {
        const int64_t row = int64_t(p) * T + t;
        *reinterpret_cast<uint4*>(xp + row * (K / 2) + 16 * g) = d[p];
        xsf[row * G + g] = uint8_t(sf[p]);
    }
}

// The gate/up image: one CTA per pair (grid = the candidate bound; CTAs past the plan's
// pair count leave at once), thread u per 16-byte unit of a row. For each of the np
// pieces a thread copies its unit into the pair's row of the image block (swizzled
// position); the lane owning unit 8s of a 256-k step also moves that step's 8 scale bytes
// as two 4-byte words (their chunk positions for k-blocks 0-3 and 4-7 are contiguous).
// Every thread of a CTA reads the same plan entries (one broadcast load each).
__global__ void __launch_bounds__(256) prefill_permute_kernel(const __grid_constant__ PrefillPlan P,
                                                              const uint8_t* __restrict__ xp,
                                                              const uint8_t* __restrict__ xsf, int T, int64_t K,
                                                              int np, uint8_t* __restrict__ img) {
    const int pos = blockIdx.x;
    if (pos >= P.hdr->n_pairs) return;
    const int U = int(K / 32);
    const int cj = P.pair_cj[pos];
    const int c = cj >> 8, j = cj & 255;
    const int n8 = (P.ch_n[c] + 7) & ~7;
    const int tok = P.pair_tok[pos];
    const int nst = int(K / kBStageK);
    const int pairs = np / kPStack;
    const int64_t cbase = img_block(P.ch_n8p, c, nst, 0, 0, n8, pairs);
    const int64_t bstride = kPImgSf + 128 * kPStack * int64_t(n8);
    for (int u = threadIdx.x; u < U; u += blockDim.x) {
        const int s = u >> 3, q = u & 7;
        for (int p = 0; p < np; ++p) {
            const int64_t row = int64_t(p) * T + tok;
            const uint4 v = __ldg(reinterpret_cast<const uint4*>(xp + row * (K / 2) + 16 * u));
            uint8_t* blk = img + cbase + int64_t(s * pairs + p / kPStack) * bstride;
            const int r = (p % kPStack) * n8 + j;                  // row in the stacked block
            *reinterpret_cast<uint4*>(blk + kPImgSf + r * 128 + ((q ^ (r & 7)) << 4)) = v;
            if (q == 0) {
                const uint2 sc = __ldg(reinterpret_cast<const uint2*>(xsf + row * U + 8 * s));
                *reinterpret_cast<uint32_t*>(blk + img_sf(r, 0)) = sc.x;
                *reinterpret_cast<uint32_t*>(blk + img_sf(r, 4)) = sc.y;
            }
        }
    }
}

__global__ void __launch_bounds__(256) f32_to_dtype_kernel(const float* __restrict__ in, int64_t n, void* out,
                                                           int dt) {
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        store_from_f32(out, dt, i, in[i]);
}

// ------------------------------------------------------------------ grouped GEMM

// Warp-wide: 32 consecutive 32-bit columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Items = (chunk c, row block r), r fastest; CTA b takes items b, b + grid, ... so the
// CTAs running at one time cover a few consecutive chunks and share their image blocks
// in the L2. PAIRS = piece pairs of this phase's token image (the down phase always has
// kPPieces / kPStack; the gate/up phase more for fp32 tokens).
template <bool GATEUP, int PAIRS>
__global__ void __launch_bounds__(kPThreads, 1)
    prefill_gemm_kernel(const __grid_constant__ PMaps maps, const __grid_constant__ PArgs a) {
    constexpr int kPairs = PAIRS;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    PASlot* aring = reinterpret_cast<PASlot*>(base);
    PBSlot* bring = reinterpret_cast<PBSlot*>(base + sizeof(PASlot) * kPASlots);
    uint64_t* afull = reinterpret_cast<uint64_t*>(base + sizeof(PASlot) * kPASlots + sizeof(PBSlot) * kPBSlots);
    uint64_t* aempty = afull + kPASlots;
    uint64_t* bfull = aempty + kPASlots;
    uint64_t* bempty = bfull + kPBSlots;
    uint64_t* accf = bempty + kPBSlots;   // accumulator ready (MMA -> epilogue)
    uint64_t* acce = accf + 1;            // accumulator drained (epilogue -> MMA)
    uint64_t* drain = acce + 1;
    __shared__ uint32_t s_tmem;
    __shared__ volatile int s_abort;
    __shared__ volatile int s_efail;      // written by epilogue warps only, read after epi_bar()
    __shared__ volatile unsigned s_aiss, s_biss;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        s_abort = 0;
        s_efail = 0;
        s_aiss = 0;
        s_biss = 0;
        for (int s = 0; s < kPASlots; ++s) {
            mbar_init(&afull[s], 1);
            mbar_init(&aempty[s], 1);
        }
        for (int s = 0; s < kPBSlots; ++s) {
            mbar_init(&bfull[s], 1);
            mbar_init(&bempty[s], 1);
        }
        mbar_init(accf, 1);
        mbar_init(acce, kPEpiWarps);
        mbar_init(drain, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (warp == 1) tmem_alloc(&s_tmem, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = s_tmem;

    const PrefillPlan& P = a.P;
    const int nrb = GATEUP ? int(a.rows / kBRows) : int(a.rows / (2 * kBRows));
    const int n_items = P.hdr->n_chunks * nrb;
    const int i0 = blockIdx.x, di = gridDim.x;
    const int nst = int(a.K / kBStageK);
    const int64_t kcks = a.K / 128;                    // scale chunks per weight row block
    const int64_t rbt = a.rows / kBRows;               // tile row blocks per slot

    if (warp == 0) {
        // ------------------------------------------------------- A producer (weights)
        if (lane == 0) {
            const uint64_t pol = l2_evict_first();
            uint32_t ga = 0;
            for (int i = i0; i < n_items && !s_abort; i += di) {
                const int c = i / nrb, rb = i - (i / nrb) * nrb;
                const int slot = P.ch_slot[c];
                const bool routed = slot < a.routed_slots;
                const int r0 = GATEUP ? rb : 2 * rb;                  // first tile row block
                const int tb0 = slot * int(rbt) + r0;
                const int tb1 = GATEUP ? tb0 : tb0 + 1;
                const uint8_t* sf0 = a.sfa0 + int64_t(slot) * a.sf_slot + int64_t(r0) * kcks * kBChunk;
                const uint8_t* sf1 = GATEUP ? a.sfa1 + int64_t(slot) * a.sf_slot + int64_t(r0) * kcks * kBChunk
                                            : sf0 + kcks * kBChunk;
                bool ok = true;
                for (int s = 0; s < nst; ++s, ++ga) {
                    const int si = int(ga % kPASlots);
                    if (!mbar_wait(&aempty[si], ((ga / kPASlots) & 1) ^ 1, a.status, &s_abort)) {
                        ok = false;
                        break;
                    }
                    PASlot& st = aring[si];
                    mbar_expect_tx(&afull[si], uint32_t(2 * kBRows * 128 + 4 * kBChunk));
                    if (routed) {
                        tma_4d_hint(&st.a[0][0][0], &maps.a0, 0, 0, s, tb0, &afull[si], pol);
                        tma_4d_hint(&st.a[1][0][0], &maps.a1, 0, 0, s, tb1, &afull[si], pol);
                        bulk_g2s_hint(&st.sfa[0][0], sf0 + int64_t(s) * 2 * kBChunk, 2 * kBChunk, &afull[si], pol);
                        bulk_g2s_hint(&st.sfa[1][0], sf1 + int64_t(s) * 2 * kBChunk, 2 * kBChunk, &afull[si], pol);
                    } else {     // the shared expert is re-read by every chunk: keep it in L2
                        tma_4d(&st.a[0][0][0], &maps.a0, 0, 0, s, tb0, &afull[si]);
                        tma_4d(&st.a[1][0][0], &maps.a1, 0, 0, s, tb1, &afull[si]);
                        bulk_g2s(&st.sfa[0][0], sf0 + int64_t(s) * 2 * kBChunk, 2 * kBChunk, &afull[si]);
                        bulk_g2s(&st.sfa[1][0], sf1 + int64_t(s) * 2 * kBChunk, 2 * kBChunk, &afull[si]);
                    }
                    s_aiss = ga + 1;
                }
                if (!ok) {
                    s_abort = 1;
                    break;
                }
            }
        }
    } else if (warp == 6) {
        // ------------------------------------------------- B producer (image blocks)
        if (lane == 0) {
            uint32_t gb = 0;
            bool ok = true;
            for (int i = i0; i < n_items && ok && !s_abort; i += di) {
                const int c = i / nrb;
                const int n8 = (P.ch_n[c] + 7) & ~7;
                const uint32_t bytes = uint32_t(kPImgSf + 128 * kPStack * n8);
                const uint8_t* cimg = a.img + img_block(P.ch_n8p, c, nst, 0, 0, n8, kPairs);
                for (int s = 0; s < nst && ok; ++s) {
                    for (int pp = 0; pp < kPairs; ++pp, ++gb) {
                        const int si = int(gb % kPBSlots);
                        if (!mbar_wait(&bempty[si], ((gb / kPBSlots) & 1) ^ 1, a.status, &s_abort)) {
                            ok = false;
                            break;
                        }
                        mbar_expect_tx(&bfull[si], bytes);
                        bulk_g2s(&bring[si].sfb[0], cimg + int64_t(s * kPairs + pp) * bytes, bytes, &bfull[si]);
                        s_biss = gb + 1;
                    }
                }
            }
            if (!ok) s_abort = 1;
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        uint32_t ga = 0, gb = 0, ib = 0;
        bool ok = true;
        const uint32_t d0 = tm, d1 = tm + kPAccCols;
        for (int i = i0; i < n_items && ok && !s_abort; i += di, ++ib) {
            const int c = i / nrb;
            const int n8 = (P.ch_n[c] + 7) & ~7;
            if (!__all_sync(0xffffffffu, mbar_wait(acce, (ib & 1) ^ 1, a.status, &s_abort))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t idesc0 = mxf4_idesc(kPStack * n8, 0), idesc2 = mxf4_idesc(kPStack * n8, 2);
            for (int s = 0; s < nst && ok; ++s, ++ga) {
                const int sa = int(ga % kPASlots);
                if (!__all_sync(0xffffffffu, mbar_wait(&afull[sa], (ga / kPASlots) & 1, a.status, &s_abort))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const PASlot& as = aring[sa];
                const uint32_t sfa = tm + kPSfaCol + 16 * sa;
                if (elect_one()) {
                    tc_cp_sf(sfa + 0, sf_chunk_desc(&as.sfa[0][0]));
                    tc_cp_sf(sfa + 4, sf_chunk_desc(&as.sfa[0][kBChunk]));
                    tc_cp_sf(sfa + 8, sf_chunk_desc(&as.sfa[1][0]));
                    tc_cp_sf(sfa + 12, sf_chunk_desc(&as.sfa[1][kBChunk]));
                }
                __syncwarp();
                for (int pp = 0; pp < kPairs; ++pp, ++gb) {
                    const int sb = int(gb % kPBSlots);
                    if (!__all_sync(0xffffffffu, mbar_wait(&bfull[sb], (gb / kPBSlots) & 1, a.status, &s_abort))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const PBSlot& bs = bring[sb];
                    const uint32_t sfb = tm + kPSfbCol + 16 * sb;   // [k-half][row set] x 4 columns
                    if (elect_one()) {
#pragma unroll
                        for (int h = 0; h < 2; ++h)
#pragma unroll
                            for (int rs = 0; rs < 2; ++rs)
                                tc_cp_sf(sfb + 8 * h + 4 * rs, sf_chunk_desc(&bs.sfb[(2 * h + rs) * kBChunk]));
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk) {
                            const uint32_t id = 2 * (kk & 1), h = kk >> 1;
                            const uint32_t idesc = (kk & 1) ? idesc2 : idesc0;
                            const uint32_t acc = (s > 0 || pp > 0 || kk > 0) ? 1u : 0u;
                            const uint64_t bd = sw128_desc(&bs.b[0][0], 32 * kk);
                            mma_mxf4(d0, sw128_desc(&as.a[0][0][0], 32 * kk), bd, idesc, (sfa + 4 * h) | (id << 30),
                                     (sfb + 8 * h) | (id << 30), acc);
                            mma_mxf4(d1, sw128_desc(&as.a[1][0][0], 32 * kk), bd, idesc,
                                     (sfa + 8 + 4 * h) | (id << 30), (sfb + 8 * h) | (id << 30), acc);
                        }
                        tc_commit(&bempty[sb]);
                    }
                    __syncwarp();
                }
                if (!ok) break;
                if (elect_one()) tc_commit(&aempty[sa]);
                __syncwarp();
            }
            if (!ok) break;
            if (elect_one()) tc_commit(accf);
            __syncwarp();
        }
        if (!ok || s_abort) {
            s_abort = 1;
            // the producers' copies in flight land before the CTA leaves
            const unsigned ai = s_aiss, bi = s_biss;
            for (unsigned k = ga; k < ai; ++k)
                if (!mbar_wait(&afull[k % kPASlots], (k / kPASlots) & 1, a.status)) break;
            for (unsigned k = gb; k < bi; ++k)
                if (!mbar_wait(&bfull[k % kPBSlots], (k / kPBSlots) & 1, a.status)) break;
        }
        // every tcgen05 operation of this warp completes before TMEM is released
        if (elect_one()) tc_commit(drain);
        __syncwarp();
        mbar_wait(drain, 0, a.status);
    } else {
        // -------------------------------------------------------------- epilogue
        const int q = warp & 3;                               // TMEM lane quarter
        const uint32_t lane_addr = uint32_t(32 * q) << 16;
        const uint32_t d0 = tm + lane_addr, d1 = d0 + kPAccCols;
        const uint64_t keep = l2_evict_last();
        float* const slab = a.slab + int64_t(blockIdx.x) * (kPN * 2 * kBRows);
        uint32_t ib = 0;
        for (int i = i0; i < n_items; i += di, ++ib) {
            const bool okw = __all_sync(0xffffffffu, mbar_wait(accf, ib & 1, a.status, &s_abort));
            if (GATEUP) {
                if (!okw) {
                    s_abort = 1;
                    break;
                }
            } else {
                // the four warps share the slab: they agree on failing, and none drains
                // into it before all have finished reading the previous item
                if (!okw && lane == 0) s_efail = 1;
                epi_bar();
                if (s_efail) {
                    s_abort = 1;
                    break;
                }
            }
            tc_fence_after();
            const int c = i / nrb, rb = i - (i / nrb) * nrb;
            const int n = P.ch_n[c], n8 = (n + 7) & ~7, p0 = P.ch_p0[c];
            if (GATEUP) {
                // drain: gate and up of rows rb*128 + 32q + lane (the two stacked piece
                // columns of a token added) -> the CTA's slab [token][gate|up][128 rows]
#pragma unroll 1
                for (int j0 = 0; j0 < n; j0 += 32) {
                    float va[32], vb[32];
                    tmem_ld32(d0 + j0, va);
                    tmem_ld32(d0 + n8 + j0, vb);
#pragma unroll
                    for (int cc = 0; cc < 32; ++cc)
                        if (j0 + cc < n) slab[(j0 + cc) * 2 * kBRows + 32 * q + lane] = va[cc] + vb[cc];
                    tmem_ld32(d1 + j0, va);
                    tmem_ld32(d1 + n8 + j0, vb);
#pragma unroll
                    for (int cc = 0; cc < 32; ++cc)
                        if (j0 + cc < n) slab[(j0 + cc) * 2 * kBRows + kBRows + 32 * q + lane] = va[cc] + vb[cc];
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(acce);             // the MMA may run the next item
                // act = phi(gate, up) * w, one token per lane: its 32 rows (one 32-block of
                // the down phase's k) split into pieces and written to the down image
                const int nst_dn = int(a.rows / kBStageK);
                const int unit = ((rb & 1) << 2) + q;                     // 16-byte unit of a row
#pragma unroll 1
                for (int j0 = 0; j0 < n; j0 += 32) {
                    const int j = j0 + lane;
                    if (j < n) {
                        const float4* gp = reinterpret_cast<const float4*>(slab + j * 2 * kBRows + 32 * q);
                        const float wt = P.pair_w[p0 + j];
                        float r[32];
#pragma unroll
                        for (int e4 = 0; e4 < 8; ++e4) {
                            const float4 g4 = gp[e4], u4 = gp[e4 + kBRows / 4];
                            r[4 * e4 + 0] = act_value(a.act_kind, g4.x, u4.x, a.beta, a.lbeta) * wt;
                            r[4 * e4 + 1] = act_value(a.act_kind, g4.y, u4.y, a.beta, a.lbeta) * wt;
                            r[4 * e4 + 2] = act_value(a.act_kind, g4.z, u4.z, a.beta, a.lbeta) * wt;
                            r[4 * e4 + 3] = act_value(a.act_kind, g4.w, u4.w, a.beta, a.lbeta) * wt;
                        }
                        uint4 dv[kPPieces];
                        uint32_t sv[kPPieces];
                        split_block32<kPPieces>(r, dv, sv);
#pragma unroll
                        for (int p = 0; p < kPPieces; ++p) {
                            uint8_t* blk = a.img_out + img_block(P.ch_n8p, c, nst_dn, rb >> 1, p / kPStack, n8,
                                                                 kPPieces / kPStack);
                            const int row = (p % kPStack) * n8 + j;
                            *reinterpret_cast<uint4*>(blk + kPImgSf + row * 128 + ((unit ^ (row & 7)) << 4)) = dv[p];
                            blk[img_sf(row, unit)] = uint8_t(sv[p]);
                        }
                    }
                }
                __syncwarp();
            } else {
                // drain: both row blocks (stacked piece columns added) -> the slab
                // [token][row block][128 rows]; then the reduce-adds into y run from the
                // slab while the MMA computes the next item
#pragma unroll 1
                for (int j0 = 0; j0 < n; j0 += 32) {
                    float va[32], vb[32];
                    tmem_ld32(d0 + j0, va);
                    tmem_ld32(d0 + n8 + j0, vb);
#pragma unroll
                    for (int cc = 0; cc < 32; ++cc)
                        if (j0 + cc < n) slab[(j0 + cc) * 2 * kBRows + 32 * q + lane] = va[cc] + vb[cc];
                    tmem_ld32(d1 + j0, va);
                    tmem_ld32(d1 + n8 + j0, vb);
#pragma unroll
                    for (int cc = 0; cc < 32; ++cc)
                        if (j0 + cc < n) slab[(j0 + cc) * 2 * kBRows + kBRows + 32 * q + lane] = va[cc] + vb[cc];
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(acce);             // the MMA may run the next item
                epi_bar();                                    // every warp's rows are in the slab
                const int64_t H = a.rows;
#pragma unroll 1
                for (int j = q; j < n; j += kPEpiWarps) {     // token j: 256 rows, 8 per lane
                    float* yr = a.y + int64_t(P.pair_tok[p0 + j]) * H + rb * 2 * kBRows + 4 * lane;
                    const float4* sp = reinterpret_cast<const float4*>(slab + j * 2 * kBRows) + lane;
                    red_add_v4(yr, sp[0], keep);
                    red_add_v4(yr + kBRows, sp[kBRows / 4], keep);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tm, 512);
    }
}

// ------------------------------------------------------------------ host side

OncePerContext g_prefill_attr;
int configure_prefill_once() {
    if (int rc = cuda_check(cudaFuncSetAttribute(prefill_gemm_kernel<true, kPPieces / kPStack>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, int(psmem_bytes())),
                            "cudaFuncSetAttribute(prefill gate/up)"))
        return rc;
    if (int rc = cuda_check(cudaFuncSetAttribute(prefill_gemm_kernel<true, kPPiecesF32 / kPStack>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, int(psmem_bytes())),
                            "cudaFuncSetAttribute(prefill gate/up, fp32 tokens)"))
        return rc;
    if (int rc = cuda_check(cudaFuncSetAttribute(prefill_gemm_kernel<false, kPPieces / kPStack>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, int(psmem_bytes())),
                            "cudaFuncSetAttribute(prefill down)"))
        return rc;
    return K3_OK;
}
int configure_prefill() { return g_prefill_attr.run(configure_prefill_once); }

size_t carve_p(size_t& off, size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 256);
    return o;
}

struct PrefillLayout {
    int64_t T, H, I, E, NS, n_cand, nc_max, nblk;
    int G;
    size_t hdr, logits, idx, w, blk, off, ch_first, pair_tok, pair_w, pair_cj, ch_slot, ch_p0, ch_n, ch_n8p;
    size_t xp, xsf, img_gu, img_dn, slab, y32, total;
};

// Bytes of an image of `pairs` piece pairs over nst k-steps: at most nc_max chunks and
// n_cand + 7 nc_max rows per piece.
size_t img_bytes(int pairs, int64_t nst, int64_t n_cand, int64_t nc_max) {
    return size_t(pairs) * size_t(nst) * (size_t(kPImgSf) * nc_max + 128 * kPStack * size_t(n_cand + 7 * nc_max));
}

PrefillLayout prefill_layout(const k3_moe_params& p, int64_t T, int64_t n_cand, int64_t num_slots, bool route) {
    PrefillLayout L{};
    L.T = T;
    L.H = p.hidden;
    L.I = p.inter;
    L.E = p.num_experts;
    L.NS = num_slots;
    L.n_cand = n_cand;
    L.nc_max = n_cand / kPN + num_slots + 1;
    L.nblk = (n_cand + kPPlanBlock - 1) / kPPlanBlock;
    L.G = num_sms();
    size_t off = 0;
    L.hdr = carve_p(off, sizeof(PrefillHeader));
    if (route) {
        L.logits = carve_p(off, sizeof(float) * T * L.E);
        L.idx = carve_p(off, sizeof(int32_t) * T * p.top_k);
        L.w = carve_p(off, sizeof(float) * T * p.top_k);
    }
    L.blk = carve_p(off, sizeof(int) * L.nblk * L.NS);
    L.off = carve_p(off, sizeof(int) * (L.NS + 1));
    L.ch_first = carve_p(off, sizeof(int) * (L.NS + 1));
    L.pair_tok = carve_p(off, sizeof(int) * n_cand);
    L.pair_w = carve_p(off, sizeof(float) * n_cand);
    L.pair_cj = carve_p(off, sizeof(int) * n_cand);
    L.ch_slot = carve_p(off, sizeof(int) * L.nc_max);
    L.ch_p0 = carve_p(off, sizeof(int) * L.nc_max);
    L.ch_n = carve_p(off, sizeof(int) * L.nc_max);
    L.ch_n8p = carve_p(off, sizeof(int) * (L.nc_max + 1));
    // token pieces and the gate/up image are sized for fp32 tokens (the larger case)
    L.xp = carve_p(off, size_t(kPPiecesF32) * T * (L.H / 2));
    L.xsf = carve_p(off, size_t(kPPiecesF32) * T * (L.H / 32));
    L.img_gu = carve_p(off, img_bytes(kPPiecesF32 / kPStack, L.H / kBStageK, n_cand, L.nc_max));
    L.img_dn = carve_p(off, img_bytes(kPPieces / kPStack, L.I / kBStageK, n_cand, L.nc_max));
    L.slab = carve_p(off, kPSlabBytes * size_t(L.G));
    L.y32 = carve_p(off, sizeof(float) * T * L.H);
    L.total = off;
    return L;
}

// Tile pool [slots * rows/128][cols/256][128][128]: one box = one contiguous tile.
int tile_pool_map(CUtensorMap* m, const uint8_t* tiles, int64_t rows, int64_t cols, int64_t slots) {
    const uint64_t d[4] = {128, 128, uint64_t(cols / 256), uint64_t(slots * (rows / 128))};
    const uint64_t st[3] = {128, 128 * 128, uint64_t(128 * 128) * uint64_t(cols / 256)};
    const uint32_t b[4] = {128, 128, 1, 1};
    return encode_map(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, tiles, d, st, b, CU_TENSOR_MAP_SWIZZLE_128B);
}

bool prefill_pool_ok(const k3_moe_params& p) {
    const k3_expert_pool* pl = p.pool;
    return pl && pl->w1_scales_tc && pl->w3_scales_tc && pl->w2_scales_tc && pl->w1_tiles && pl->w3_tiles &&
           pl->w2_tiles && p.hidden % 256 == 0 && p.inter % 256 == 0 && p.hidden >= 256 && p.inter >= 256;
}

int check_prefill(const k3_moe_params* p, const void* x, int xdt, int64_t T, const void* y, int ydt,
                  const char* what) {
    if (!p) return fail(K3_ERR_INVALID, std::string(what) + ": params is NULL");
    if (!x || !y) return fail(K3_ERR_INVALID, std::string(what) + ": NULL tensor");
    if (xdt != K3_F32 && xdt != K3_BF16) return fail(K3_ERR_INVALID, std::string(what) + ": x must be f32 or bf16");
    if (ydt != K3_F32 && ydt != K3_BF16) return fail(K3_ERR_INVALID, std::string(what) + ": y must be f32 or bf16");
    if (T < 1 || T > (int64_t(1) << 24)) return fail(K3_ERR_INVALID, std::string(what) + ": T must be 1..2^24");
    if (p->num_experts < 1 || p->num_experts > kMaxExperts)
        return fail(K3_ERR_UNSUPPORTED, std::string(what) + ": num_experts must be 1..1024");
    if (p->top_k < 1 || p->top_k > 32 || p->top_k > p->num_experts)
        return fail(K3_ERR_UNSUPPORTED, std::string(what) + ": top_k must be 1..min(32, E)");
    if (p->activation != K3_ACT_SILU && p->activation != K3_ACT_SITU)
        return fail(K3_ERR_INVALID, std::string(what) + ": unknown activation");
    if (!prefill_pool_ok(*p))
        return fail(K3_ERR_UNSUPPORTED, std::string(what) + " needs the block-scaled tile pool (re-laid scales "
                                                            "and tiles; H, I multiples of 256)");
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(y) & 15))
        return fail(K3_ERR_INVALID, std::string(what) + ": x and y must be 16-byte aligned");
    return K3_OK;
}

// Plan, pieces, image and both grouped GEMMs; y (f32 or bf16) = the sum over the candidates.
int prefill_run(const k3_moe_params* p, const void* x, int xdt, int64_t T, const PrefillCand& cand,
                void* y, int ydt, uint8_t* ws, const PrefillLayout& L, cudaStream_t s) {
    if (int rc = configure_prefill()) return rc;
    const k3_expert_pool& pl = *p->pool;
    PrefillPlan P{};
    P.hdr = reinterpret_cast<PrefillHeader*>(ws + L.hdr);
    P.blk_cnt = reinterpret_cast<int*>(ws + L.blk);
    P.off = reinterpret_cast<int*>(ws + L.off);
    P.ch_first = reinterpret_cast<int*>(ws + L.ch_first);
    P.pair_tok = reinterpret_cast<int*>(ws + L.pair_tok);
    P.pair_w = reinterpret_cast<float*>(ws + L.pair_w);
    P.pair_cj = reinterpret_cast<int*>(ws + L.pair_cj);
    P.ch_slot = reinterpret_cast<int*>(ws + L.ch_slot);
    P.ch_p0 = reinterpret_cast<int*>(ws + L.ch_p0);
    P.ch_n = reinterpret_cast<int*>(ws + L.ch_n);
    P.ch_n8p = reinterpret_cast<int*>(ws + L.ch_n8p);
    const int G = L.G;
    const int n_cand = int(L.n_cand);
    const int NS = int(L.NS);
    const size_t mask_bytes = sizeof(uint32_t) * 8 * size_t(NS);

    prof_begin(K3_PROF_TOPK, s);
    prefill_count_kernel<<<int(L.nblk), kPPlanBlock, mask_bytes, s>>>(cand, n_cand, P.blk_cnt);
    K3_CHECK_LAUNCH("prefill_count_kernel");
    prefill_blkscan_kernel<<<(NS + 7) / 8, 256, 0, s>>>(P.blk_cnt, int(L.nblk), NS, P.off);
    K3_CHECK_LAUNCH("prefill_blkscan_kernel");
    prefill_scan_kernel<<<1, 1024, 0, s>>>(P, NS, int(L.nc_max));
    K3_CHECK_LAUNCH("prefill_scan_kernel");
    prefill_place_kernel<<<int(L.nblk), kPPlanBlock, mask_bytes, s>>>(cand, n_cand, P);
    K3_CHECK_LAUNCH("prefill_place_kernel");
    {
        const int64_t n = T * (L.H / 32);
        if (xdt == K3_F32)
            prefill_pieces_kernel<kPPiecesF32>
                <<<int((n + 255) / 256), 256, 0, s>>>(x, xdt, int(T), L.H, ws + L.xp, ws + L.xsf);
        else
            prefill_pieces_kernel<kPPieces>
                <<<int((n + 255) / 256), 256, 0, s>>>(x, xdt, int(T), L.H, ws + L.xp, ws + L.xsf);
        K3_CHECK_LAUNCH("prefill_pieces_kernel");
        const int U = int(L.H / 32);                      // a multiple of 8 (H % 256 == 0)
        prefill_permute_kernel<<<n_cand, std::min(U, 256), 0, s>>>(
            P, ws + L.xp, ws + L.xsf, int(T), L.H, xdt == K3_F32 ? kPPiecesF32 : kPPieces, ws + L.img_gu);
        K3_CHECK_LAUNCH("prefill_permute_kernel");
    }
    prof_end(K3_PROF_TOPK, s);
    float* y32 = ydt == K3_F32 ? static_cast<float*>(y) : reinterpret_cast<float*>(ws + L.y32);
    if (int rc = cuda_check(cudaMemsetAsync(y32, 0, sizeof(float) * T * L.H, s), "cudaMemsetAsync(y)")) return rc;

    PArgs ga{};
    ga.P = P;
    ga.K = L.H;
    ga.rows = L.I;
    ga.status = &P.hdr->status;
    ga.sfa0 = pl.w1_scales_tc;
    ga.sfa1 = pl.w3_scales_tc;
    ga.sf_slot = (L.I / 128) * (L.H / 128) * kBChunk;
    ga.routed_slots = int(p->num_experts);
    ga.img = ws + L.img_gu;
    ga.img_out = ws + L.img_dn;
    ga.slab = reinterpret_cast<float*>(ws + L.slab);
    ga.act_kind = p->activation;
    ga.beta = p->situ_beta;
    ga.lbeta = p->situ_linear_beta;
    PMaps ma{};
    if (int rc = tile_pool_map(&ma.a0, pl.w1_tiles, L.I, L.H, pl.num_slots)) return rc;
    if (int rc = tile_pool_map(&ma.a1, pl.w3_tiles, L.I, L.H, pl.num_slots)) return rc;
    prof_begin(K3_PROF_GATEUP, s);
    if (xdt == K3_F32)
        prefill_gemm_kernel<true, kPPiecesF32 / kPStack><<<G, kPThreads, psmem_bytes(), s>>>(ma, ga);
    else
        prefill_gemm_kernel<true, kPPieces / kPStack><<<G, kPThreads, psmem_bytes(), s>>>(ma, ga);
    prof_end(K3_PROF_GATEUP, s);
    K3_CHECK_LAUNCH("prefill_gemm_kernel<gate/up>");

    PArgs da = ga;
    da.K = L.I;
    da.rows = L.H;
    da.sfa0 = pl.w2_scales_tc;
    da.sfa1 = nullptr;
    da.sf_slot = (L.H / 128) * (L.I / 128) * kBChunk;
    da.img = ws + L.img_dn;
    da.img_out = nullptr;
    da.slab = ga.slab;                   // the gate/up launch is done with it (same stream)
    da.y = y32;
    PMaps mb{};
    if (int rc = tile_pool_map(&mb.a0, pl.w2_tiles, L.H, L.I, pl.num_slots)) return rc;
    mb.a1 = mb.a0;
    prof_begin(K3_PROF_DOWN, s);
    prefill_gemm_kernel<false, kPPieces / kPStack><<<G, kPThreads, psmem_bytes(), s>>>(mb, da);
    prof_end(K3_PROF_DOWN, s);
    K3_CHECK_LAUNCH("prefill_gemm_kernel<down>");
    if (ydt != K3_F32) {
        prof_begin(K3_PROF_OTHER, s);
        f32_to_dtype_kernel<<<4 * G, 256, 0, s>>>(y32, T * L.H, y, ydt);
        prof_end(K3_PROF_OTHER, s);
        K3_CHECK_LAUNCH("f32_to_dtype_kernel");
    }
    return K3_OK;
}

int prefill_route(const k3_moe_params* p, const void* x, int xdt, int64_t T, const uint16_t* gate_w,
                  const float* bias, int32_t* idx, float* w, uint8_t* ws, const PrefillLayout& L, cudaStream_t s) {
    float* logits = reinterpret_cast<float*>(ws + L.logits);
    int* status = &reinterpret_cast<PrefillHeader*>(ws + L.hdr)->status;
    prof_begin(K3_PROF_ROUTER, s);
    if (router_gemm_ok(xdt, L.H, x, gate_w)) {
        if (int rc = launch_router_gemm(x, T, L.H, gate_w, L.E, logits, status, s)) return rc;
    } else {
        if (int rc = launch_router_logits_rows(x, xdt, T, L.H, gate_w, L.E, logits, s)) return rc;
    }
    prof_end(K3_PROF_ROUTER, s);
    prof_begin(K3_PROF_TOPK, s);
    const int rc = launch_topk_rows(logits, T, L.E, bias, p->top_k, p->renormalize, p->routed_scaling_factor, idx,
                                    w, status, s);
    prof_end(K3_PROF_TOPK, s);
    return rc;
}

int64_t routed_candidates(const k3_moe_params& p, int64_t T) {
    return T * p.top_k + (p.has_shared ? T : 0);
}

// Candidates of a whole layer's routing: every expert local, the shared expert (slot E)
// for every token.
PrefillCand routed_cand(const k3_moe_params& p, const int32_t* idx, const float* w, int64_t T, int ns) {
    PrefillCand c{};
    c.idx = idx;
    c.w = w;
    c.T = int(T);
    c.k = p.top_k;
    c.rstride = p.top_k;
    c.expert_lo = 0;
    c.n_local = int(p.num_experts);
    c.shared_slot = p.has_shared ? int(p.num_experts) : -1;
    c.shared_t0 = 0;
    c.shared_n = p.has_shared ? int(T) : 0;
    c.num_slots = ns;
    return c;
}

}  // namespace

bool router_gemm_ok(int xdt, int64_t H, const void* x, const void* gate_w) {
    return xdt == K3_BF16 && H % 64 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(gate_w) & 15) == 0;
}

int launch_router_gemm(const void* x, int64_t T, int64_t H, const uint16_t* gate_w, int64_t E, float* logits,
                       int* status, cudaStream_t s) {
    // logits [T][E] = x [T][H] . W_gate [E][H]^T: the dense tcgen05 GEMM, one bf16 piece
    return launch_gemm_bf16(static_cast<const uint16_t*>(x), nullptr, H, T, H, gate_w, H, E, logits, E, 0, status, s);
}

}  // namespace k3

using namespace k3;

extern "C" K3_API size_t k3_moe_prefill_workspace(const k3_moe_params* p, int64_t T) {
    if (!p || T < 1) return 0;
    const int64_t ns = p->num_experts + (p->has_shared ? 1 : 0);
    return prefill_layout(*p, T, routed_candidates(*p, T), ns, true).total;
}

extern "C" K3_API int k3_moe_prefill(const k3_moe_params* p, const void* x, int x_dtype, int64_t T,
                                     const uint16_t* gate_w_bf16, const float* bias, void* y_out, int y_dtype,
                                     int32_t* idx_out, float* weight_out, void* workspace, size_t workspace_bytes,
                                     void* stream) {
    if (int rc = check_prefill(p, x, x_dtype, T, y_out, y_dtype, "k3_moe_prefill")) return rc;
    if (!gate_w_bf16) return fail(K3_ERR_INVALID, "k3_moe_prefill: gate_w is NULL");
    if (p->pool->num_slots < p->num_experts + (p->has_shared ? 1 : 0))
        return fail(K3_ERR_INVALID, "k3_moe_prefill: the pool has fewer slots than experts");
    const int64_t ns = p->num_experts + (p->has_shared ? 1 : 0);
    const PrefillLayout L = prefill_layout(*p, T, routed_candidates(*p, T), ns, true);
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255))
        return fail(K3_ERR_WORKSPACE, "k3_moe_prefill: workspace must be non-NULL and 256-byte aligned");
    if (workspace_bytes < L.total)
        return fail(K3_ERR_WORKSPACE, "k3_moe_prefill: workspace too small: need " + std::to_string(L.total) + " bytes");
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (int rc = cuda_check(cudaMemsetAsync(ws + L.hdr, 0, sizeof(PrefillHeader), s), "cudaMemsetAsync(header)"))
        return rc;
    int32_t* idx = idx_out ? idx_out : reinterpret_cast<int32_t*>(ws + L.idx);
    float* w = weight_out ? weight_out : reinterpret_cast<float*>(ws + L.w);
    if (int rc = prefill_route(p, x, x_dtype, T, gate_w_bf16, bias, idx, w, ws, L, s)) return rc;
    return prefill_run(p, x, x_dtype, T, routed_cand(*p, idx, w, T, int(ns)), y_out, y_dtype, ws, L, s);
}

extern "C" K3_API int k3_moe_experts_prefill(const k3_moe_params* p, const void* x, int x_dtype, int64_t T,
                                             const int32_t* idx, const float* w, void* y_out, int y_dtype,
                                             void* workspace, size_t workspace_bytes, void* stream) {
    if (int rc = check_prefill(p, x, x_dtype, T, y_out, y_dtype, "k3_moe_experts_prefill")) return rc;
    if (!idx || !w) return fail(K3_ERR_INVALID, "k3_moe_experts_prefill: NULL routing");
    const int64_t ns = p->num_experts + (p->has_shared ? 1 : 0);
    if (p->pool->num_slots < ns) return fail(K3_ERR_INVALID, "k3_moe_experts_prefill: the pool has fewer slots than experts");
    const PrefillLayout L = prefill_layout(*p, T, routed_candidates(*p, T), ns, true);
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255))
        return fail(K3_ERR_WORKSPACE, "k3_moe_experts_prefill: workspace must be non-NULL and 256-byte aligned");
    if (workspace_bytes < L.total)
        return fail(K3_ERR_WORKSPACE,
                    "k3_moe_experts_prefill: workspace too small: need " + std::to_string(L.total) + " bytes");
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (int rc = cuda_check(cudaMemsetAsync(ws + L.hdr, 0, sizeof(PrefillHeader), s), "cudaMemsetAsync(header)"))
        return rc;
    return prefill_run(p, x, x_dtype, T, routed_cand(*p, idx, w, T, int(ns)), y_out, y_dtype, ws, L, s);
}

extern "C" K3_API size_t k3_moe_pairs_prefill_workspace(const k3_moe_params* p, int64_t T, int64_t n_pairs) {
    if (!p || !p->pool || T < 1 || n_pairs < 1) return 0;
    return prefill_layout(*p, T, n_pairs, p->pool->num_slots, false).total;
}

extern "C" K3_API int k3_moe_pairs_prefill(const k3_moe_params* p, const void* x, int x_dtype, int64_t T,
                                           const int32_t* pair_slot, const int32_t* pair_tok, const float* pair_w,
                                           int64_t n_pairs, void* y_out, int y_dtype, void* workspace,
                                           size_t workspace_bytes, void* stream) {
    if (int rc = check_prefill(p, x, x_dtype, T, y_out, y_dtype, "k3_moe_pairs_prefill")) return rc;
    if (!pair_slot || !pair_tok || !pair_w) return fail(K3_ERR_INVALID, "k3_moe_pairs_prefill: NULL pairs");
    if (n_pairs < 1 || n_pairs > (int64_t(1) << 28))
        return fail(K3_ERR_INVALID, "k3_moe_pairs_prefill: n_pairs must be 1..2^28");
    if (p->pool->num_slots < 1 || p->pool->num_slots > kPMaxSlots)
        return fail(K3_ERR_UNSUPPORTED, "k3_moe_pairs_prefill: the pool must have 1..1025 slots");
    const PrefillLayout L = prefill_layout(*p, T, n_pairs, p->pool->num_slots, false);
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255))
        return fail(K3_ERR_WORKSPACE, "k3_moe_pairs_prefill: workspace must be non-NULL and 256-byte aligned");
    if (workspace_bytes < L.total)
        return fail(K3_ERR_WORKSPACE,
                    "k3_moe_pairs_prefill: workspace too small: need " + std::to_string(L.total) + " bytes");
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (int rc = cuda_check(cudaMemsetAsync(ws + L.hdr, 0, sizeof(PrefillHeader), s), "cudaMemsetAsync(header)"))
        return rc;
    PrefillCand c{};
    c.slot = pair_slot;
    c.tok = pair_tok;
    c.pw = pair_w;
    c.n = int(n_pairs);
    c.T = int(T);
    c.shared_slot = -1;
    c.num_slots = int(p->pool->num_slots);
    return prefill_run(p, x, x_dtype, T, c, y_out, y_dtype, ws, L, s);
}

namespace k3 {
size_t pairs_decode_workspace(const k3_moe_params& p, int64_t T, int64_t n_in);
int pairs_decode_run(const k3_moe_params* p, const void* x, int x_dtype, int64_t T, const PairsArgs& cand,
                     void* y_out, int y_dtype, void* workspace, size_t workspace_bytes, cudaStream_t s);
}  // namespace k3

extern "C" K3_API size_t k3_moe_ep_local_workspace(const k3_moe_params* p, int64_t T, int64_t shared_n) {
    if (!p || !p->pool || T < 1 || shared_n < 0) return 0;
    const int64_t n = T * p->top_k + shared_n;
    if (n <= kMaxPairCandidates) return pairs_decode_workspace(*p, T, n);
    return prefill_layout(*p, T, n, p->pool->num_slots, false).total;
}

extern "C" K3_API int k3_moe_ep_local(const k3_moe_params* p, const void* x, int x_dtype, int64_t T,
                                      const int32_t* idx, const float* w, int64_t route_stride, int32_t expert_lo,
                                      int32_t shared_t0, int32_t shared_n, void* y_out, int y_dtype,
                                      void* workspace, size_t workspace_bytes, void* stream) {
    if (!p || !p->pool) return fail(K3_ERR_INVALID, "k3_moe_ep_local: params or pool is NULL");
    if (!x || !idx || !w || !y_out) return fail(K3_ERR_INVALID, "k3_moe_ep_local: NULL tensor");
    if (x_dtype != K3_F32 && x_dtype != K3_BF16) return fail(K3_ERR_INVALID, "k3_moe_ep_local: x must be f32 or bf16");
    if (y_dtype != K3_F32 && y_dtype != K3_BF16) return fail(K3_ERR_INVALID, "k3_moe_ep_local: y must be f32 or bf16");
    if (T < 1 || T > (int64_t(1) << 24)) return fail(K3_ERR_INVALID, "k3_moe_ep_local: T must be 1..2^24");
    if (p->top_k < 1 || route_stride < p->top_k) return fail(K3_ERR_INVALID, "k3_moe_ep_local: route_stride < top_k");
    if (shared_n < 0 || shared_t0 < 0 || int64_t(shared_t0) + shared_n > T)
        return fail(K3_ERR_INVALID, "k3_moe_ep_local: shared token range outside [0, T)");
    const int64_t n = T * p->top_k + shared_n;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int shared_slot = p->has_shared ? int(p->num_experts) : -1;
    if (n <= kMaxPairCandidates) {
        PairsArgs c{};
        c.ridx = idx;
        c.rw = w;
        c.rk = p->top_k;
        c.rstride = int(route_stride);
        c.expert_lo = expert_lo;
        c.n_local = int(p->num_experts);
        c.shared_slot = shared_slot;
        c.shared_t0 = shared_t0;
        c.shared_n = shared_n;
        c.n_in = int(n);
        return pairs_decode_run(p, x, x_dtype, T, c, y_out, y_dtype, workspace, workspace_bytes, s);
    }
    if (int rc = check_prefill(p, x, x_dtype, T, y_out, y_dtype, "k3_moe_ep_local")) return rc;
    if (p->pool->num_slots < 1 || p->pool->num_slots > kPMaxSlots)
        return fail(K3_ERR_UNSUPPORTED, "k3_moe_ep_local: the pool must have 1..1025 slots");
    const PrefillLayout L = prefill_layout(*p, T, n, p->pool->num_slots, false);
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255))
        return fail(K3_ERR_WORKSPACE, "k3_moe_ep_local: workspace must be non-NULL and 256-byte aligned");
    if (workspace_bytes < L.total)
        return fail(K3_ERR_WORKSPACE, "k3_moe_ep_local: workspace too small: need " + std::to_string(L.total) + " bytes");
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    if (int rc = cuda_check(cudaMemsetAsync(ws + L.hdr, 0, sizeof(PrefillHeader), s), "cudaMemsetAsync(header)"))
        return rc;
    PrefillCand c{};
    c.idx = idx;
    c.w = w;
    c.T = int(T);
    c.k = p->top_k;
    c.rstride = int(route_stride);
    c.expert_lo = expert_lo;
    c.n_local = int(p->num_experts);
    c.shared_slot = shared_slot;
    c.shared_t0 = shared_t0;
    c.shared_n = shared_n;
    c.num_slots = int(p->pool->num_slots);
    return prefill_run(p, x, x_dtype, T, c, y_out, y_dtype, ws, L, s);
}

extern "C" K3_API int k3_moe_prefill_status(const void* workspace, void* stream) {
    if (!workspace) return fail(K3_ERR_INVALID, "k3_moe_prefill_status: workspace is NULL");
    int st = 0;
    if (int rc = cuda_check(cudaMemcpyAsync(&st, workspace, sizeof(int), cudaMemcpyDeviceToHost,
                                            static_cast<cudaStream_t>(stream)),
                            "cudaMemcpyAsync(status)"))
        return rc;
    if (int rc = cuda_check(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "cudaStreamSynchronize"))
        return rc;
    return st;
}
