/*
 * k3b200 -- C ABI of the B200 (sm_100a) MXFP4 quantized-expert path.
 *
 * Drop-in for the hot path of sjdthree/kimi-k3-mlx-macmini: the fused MXFP4
 * dequant-matvec that runs every routed and shared expert projection, the sigmoid
 * top-k router, and the token->expert gather / weighted scatter-add around them.
 *
 * Conventions (every entry point):
 *  - Returns 0 (K3_OK) or a K3_ERR_* code; never aborts. k3_last_error() gives the
 *    message of the calling thread's last failure.
 *  - Tensor arguments are DEVICE pointers, row-major and contiguous, unless noted.
 *  - `stream` is a cudaStream_t (NULL = legacy default stream); all work is enqueued
 *    on it, nothing blocks the host.
 *  - Scratch ("workspace") is caller-owned device memory of at least the size the
 *    matching *_workspace() function returns, 256-byte aligned. Its contents need no
 *    initialisation and are not preserved between calls; calls that share one
 *    workspace must not overlap on the GPU.
 *
 * MXFP4 layout (the reference's, air_llm/models/kimi_k3/mxfp4.py:3-12): packed u8
 * [rows][cols/2], low nibble = even element; code bit 3 = sign, bits 0-2 index
 * {0,.5,1,1.5,2,3,4,6}; scales u8 [rows][cols/32], E8M0 value 2**(byte-127).
 */
#ifndef K3B200_H
#define K3B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define K3_API __attribute__((visibility("default")))
#else
#define K3_API
#endif

enum {
    K3_OK = 0,
    K3_ERR_INVALID = 1,      /* bad argument: shape, dtype, NULL pointer (reference: ValueError) */
    K3_ERR_UNSUPPORTED = 2,  /* valid request outside what this build implements */
    K3_ERR_CUDA = 3,         /* a CUDA runtime call failed */
    K3_ERR_WORKSPACE = 4,    /* workspace missing, too small or misaligned */
    K3_ERR_TIMEOUT = 5,      /* a bounded device-side wait gave up */
    K3_ERR_IO = 6            /* a file could not be opened or read (reference: OSError) */
};

enum { K3_F32 = 0, K3_BF16 = 1, K3_F16 = 2 };             /* element types */
enum { K3_ACT_SILU = 0, K3_ACT_SITU = 1 };                 /* expert activation */

/* 3: k3_dense_seg gained act_input. */
K3_API int k3_abi_version(void);
K3_API const char* k3_last_error(void);
/* Number of streaming multiprocessors of the current device (grid sizing / tests). */
K3_API int k3_device_sms(void);

/* Kernel timing diagnostics (no counterpart in the reference, which times with wall
 * clocks around mx.eval -- tools/profile_compute.py:26-33). While enabled, every kernel
 * launch of this library is bracketed by CUDA events on its launch stream;
 * k3_profile_collect waits for them and returns, per kernel kind, the summed device
 * milliseconds and the launch count since the previous collect. */
enum {
    K3_PROF_ROUTER = 0,      /* router logits GEMV                                */
    K3_PROF_TOPK = 1,        /* top-k / routing plan / activation conversion      */
    K3_PROF_GATEUP = 2,      /* grouped MXFP4 matvec: gate+up projections + act   */
    K3_PROF_DOWN = 3,        /* grouped MXFP4 matvec: down projection + combine   */
    K3_PROF_MATVEC = 4,      /* single-matrix MXFP4 matvec                        */
    K3_PROF_OTHER = 5,       /* codec and generic kernels                         */
    K3_PROF_DENSE = 6,       /* dense bf16 matvecs (latent, shared expert, lm_head) */
    K3_PROF_KINDS = 7
};
K3_API int k3_profile_enable(int on);
K3_API int k3_profile_collect(double* ms_out, int64_t* launches_out, int n);

/* ------------------------------------------------------------------ codec ----- */

/* Full dequantisation, bit-exact: out[r][c] = E2M1(code) * 2**(scale-127) as f32 or
 * bf16 (lossless for scale bytes 1..254 -- air_llm/models/kimi_k3/mxfp4.py:8-10).
 * Replaces decode_mxfp4_reference (air_llm/models/kimi_k3/mxfp4.py:26-36), the
 * k3ref decoder (k3ref/weights.py:29-37) and decode_mxfp4_mlx (mxfp4.py:68-81).
 * group_size must be 32. */
K3_API int k3_mxfp4_dequant(const uint8_t* packed, const uint8_t* scales, int64_t rows,
                            int64_t cols, int group_size, void* out, int out_dtype,
                            void* stream);

/* minmax_out (device int32[2]) <- {min, max} of n scale bytes. The reduction half of
 * assert_scales_representable (air_llm/models/kimi_k3/mxfp4.py:58-65); the caller
 * applies the 2..252 rule. */
/* Re-lays E8M0 scales [batch][rows][cols/32] (row-major, as stored) into the chunk
 * layout the block-scaled tensor-core MMA reads: [batch][rows/128][cols/128][512], where
 * the 512-byte chunk of (row block, 128-column block) holds the scale of row m and
 * 32-column block j at byte (m % 32) * 16 + (m / 32) * 4 + j. rows and cols must be
 * multiples of 128. No reference counterpart: a one-time preparation of an expert pool
 * (the reference reads scales row-major inside its Metal kernel,
 * air_llm/kernels/metal/mxfp4_matvec.py:29-63). */
K3_API int k3_mxfp4_scales_tc(const uint8_t* scales, int64_t rows, int64_t cols, int64_t batch,
                              uint8_t* out, void* stream);

/* Re-lays packed E2M1 codes [batch][rows][cols/2] into tiles [batch][rows/128][cols/256]
 * [128][128]: tile (row block, 256-column block) holds its 128 rows of 128 bytes
 * contiguously. rows % 128 == 0, cols % 256 == 0. No reference counterpart (one-time pool
 * preparation for the block-scaled decode kernels). */
K3_API int k3_mxfp4_tiles(const uint8_t* packed, int64_t rows, int64_t cols, int64_t batch,
                          uint8_t* out, void* stream);

K3_API int k3_mxfp4_scale_minmax(const uint8_t* scales, int64_t n, int32_t* minmax_out,
                                 void* stream);

/* ------------------------------------------------------------- fused matvec --- */

/* out[M][N] = x[M][K] . dequant(packed[N][K/2], scales[N][K/32])^T with fp32
 * accumulation; x is f32 or bf16, out f32 or bf16. Any M >= 1; K a multiple of 32.
 * Replaces mxfp4_matvec_fused (air_llm/kernels/metal/mxfp4_matvec.py:75-96) and its
 * MSL kernel (:29-63); K mismatch is the caller's ValueError (:85-86). */
K3_API size_t k3_mxfp4_matvec_workspace(int64_t M, int64_t K, int64_t N);
K3_API int k3_mxfp4_matvec(const void* x, int x_dtype, int64_t M, int64_t K,
                           const uint8_t* packed, const uint8_t* scales, int64_t N,
                           void* out, int out_dtype, void* workspace, size_t workspace_bytes,
                           void* stream);

/* k3_mxfp4_matvec for callers that cannot allocate device memory. No counterpart in the
 * reference (its mxfp4_matvec_fused gets its output from MLX's allocator).
 * Who needs it: a host that hands this path only its own input and output buffers --
 * e.g. an FFI binding of the three-argument mxfp4_matvec_fused inside a runtime whose
 * device memory belongs to another allocator (a caching allocator, or a fixed arena
 * holding the free memory) -- cannot call cudaMalloc: that memory would go behind its
 * allocator's back or not exist, and cudaMalloc/cudaFree synchronise the device.
 * This call allocates nothing. Its scratch is one file-scope device array of 4 MiB,
 * which every GPU that loads this library holds until the process exits; shapes that
 * need more scratch than that (see k3_mxfp4_matvec_workspace) return K3_ERR_INVALID.
 * The first call in a device's context looks the array's address up
 * (cudaGetSymbolAddress, with that device current) and keeps it for that context; a
 * cudaDeviceReset replaces the context, and the next call looks the address up again.
 * Make the first call on each device before any stream capture. Every call
 * shares the one array, so calls that overlap on the GPU (other streams, other host
 * threads) race; each call re-initialises what it reads from the array. Arguments and
 * results are those of k3_mxfp4_matvec. */
K3_API int k3_mxfp4_matvec_noalloc(const void* x, int x_dtype, int64_t M, int64_t K,
                                   const uint8_t* packed, const uint8_t* scales, int64_t N,
                                   void* out, int out_dtype, void* stream);

/* ------------------------------------------------------------------- router --- */

/* Sigmoid top-k router of LatentMoE.route (air_llm/models/kimi_k3/moe.py:65-76;
 * oracle k3ref/layers.py:214-224): logits = x_f32 . W_g^T (fp32), raw = sigmoid,
 * corrected = raw + bias (selection only), idx = top-k(corrected) in descending order
 * (ties: lower index), w = raw[idx], renormalised by sum + 1e-20 when top_k > 1 and
 * renormalize != 0, times routed_scaling_factor.
 * x [M][H] f32|bf16; gate_w bf16 bits [E][H]; bias f32 [E] or NULL (zeros);
 * idx_out int32 [M][top_k]; weight_out f32 [M][top_k]; raw/corrected f32 [M][E] or
 * NULL. Limits: E <= 1024, 1 <= top_k <= 32, H % 8 == 0. */
K3_API size_t k3_moe_route_workspace(int64_t M, int64_t E);
K3_API int k3_moe_route(const void* x, int x_dtype, int64_t M, int64_t H,
                        const uint16_t* gate_w_bf16, const float* bias, int64_t E, int top_k,
                        int renormalize, float routed_scaling_factor, int32_t* idx_out,
                        float* weight_out, float* raw_out, float* corrected_out,
                        void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------ MoE experts ----- */

/* One expert's three MXFP4 projections (device pointers), as expert_source returns
 * them (air_llm/models/kimi_k3/moe.py:79-88, loader.py:229-266): w1 = gate [I][H],
 * w3 = up [I][H], w2 = down [H][I]; each packed [rows][cols/2] + scales [rows][cols/32]. */
typedef struct k3_expert_ptrs {
    const uint8_t* w1_packed;
    const uint8_t* w1_scales;
    const uint8_t* w3_packed;
    const uint8_t* w3_scales;
    const uint8_t* w2_packed;
    const uint8_t* w2_scales;
} k3_expert_ptrs;

/* Optional contiguous expert pools (device pointers): slot e holds expert e, slot E the
 * shared expert. w1/w3 packed [slots][I][H/2], scales [slots][I][H/32]; w2 packed
 * [slots][H][I/2], scales [slots][H][I/32]. With a pool (and H, I multiples of 512) the
 * decode runs on the TMA-fed kernels; without one, on the pointer-table kernels. */
typedef struct k3_expert_pool {
    const uint8_t* w1_packed;
    const uint8_t* w1_scales;
    const uint8_t* w3_packed;
    const uint8_t* w3_scales;
    const uint8_t* w2_packed;
    const uint8_t* w2_scales;
    int64_t num_slots;
    /* Optional: the same scales re-laid by k3_mxfp4_scales_tc for the block-scaled
       tensor-core path ([slot][rows/128][cols/128][512]). All three non-NULL (and H, I
       multiples of 256) select that path; otherwise the f16 tensor-core path runs. */
    const uint8_t* w1_scales_tc;
    const uint8_t* w3_scales_tc;
    const uint8_t* w2_scales_tc;
    /* Optional, block-scaled path only: the packed codes re-laid by k3_mxfp4_tiles into
       contiguous 128-row x 128-byte tiles ([slot][rows/128][cols/256][128][128]) so every
       TMA box is one sequential 16 KiB read; NULL streams the row-major pools. */
    const uint8_t* w1_tiles;
    const uint8_t* w3_tiles;
    const uint8_t* w2_tiles;
} k3_expert_pool;

/* Static description of one MoE layer's expert set (host struct). */
typedef struct k3_moe_params {
    int64_t hidden;               /* H: w1/w3 input dim, w2 output dim               */
    int64_t inter;                /* I: expert intermediate size                     */
    int64_t num_experts;          /* E routed experts                                */
    int32_t top_k;                /* routed experts per token                        */
    int32_t renormalize;          /* moe_renormalize                                 */
    float routed_scaling_factor;
    int32_t has_shared;           /* 1: experts[E] is an MXFP4 shared expert applied
                                     to every token with weight 1                    */
    int32_t activation;           /* K3_ACT_SILU (silu(g)*u) or K3_ACT_SITU           */
    float situ_beta;              /* situ only (air_llm/models/kimi_k3/ops.py:17-28)  */
    float situ_linear_beta;       /* situ only; <= 0 means None                      */
    const k3_expert_ptrs* experts;/* DEVICE array [E + has_shared]                   */
    const k3_expert_pool* pool;   /* HOST pointer to pool descriptors, or NULL       */
} k3_moe_params;

/* Local expert computation of an expert-parallel MoE layer: T token rows x [T][H] and
 * n_pairs candidate (slot, token row, weight) pairs; candidates with slot < 0 (or out of
 * range) are skipped. y_out [T][H] (f32|bf16) receives, per token row, the sum over its
 * pairs of weight * expert(slot)(x[token]) in ascending slot order (rows without pairs
 * are zero). Needs the block-scaled pool (k3_expert_pool *_scales_tc and *_tiles).
 * Limits: n_pairs <= 1024 candidates; at most 256 of them valid and 256 expert items
 * (8 pairs each) per call, else the call's routing plan reports K3_ERR_UNSUPPORTED in
 * its status word. Replaces the per-expert loop of LatentMoE.__call__
 * (air_llm/models/kimi_k3/moe.py:110-132) for the experts one rank owns. */
K3_API size_t k3_moe_pairs_workspace(const k3_moe_params* p, int64_t T, int64_t n_pairs);
K3_API int k3_moe_pairs_decode(const k3_moe_params* p, const void* x, int x_dtype, int64_t T,
                               const int32_t* pair_slot, const int32_t* pair_tok,
                               const float* pair_w, int64_t n_pairs, void* y_out, int y_dtype,
                               void* workspace, size_t workspace_bytes, void* stream);

/* Decode (M <= 8 tokens) MoE block without the latent wrapper: route, then for every
 * routed expert y[t] += w[t,slot] * act(x W1^T, x W3^T) W2^T, summed in ascending
 * expert id, plus the shared expert. Replaces LatentMoE.__call__'s route + expert loop
 * + shared expert (air_llm/models/kimi_k3/moe.py:110-132; oracle k3ref/layers.py:
 * 241-261) for the BASELINE layer. y [M][H] f32|bf16; idx_out/weight_out as in
 * k3_moe_route (may be NULL). Limits: M <= 8, H % 128 == 0, I % 128 == 0, E <= 1024,
 * top_k <= 16. */
K3_API size_t k3_moe_decode_workspace(const k3_moe_params* p, int64_t M);
K3_API int k3_moe_decode(const k3_moe_params* p, const void* x, int x_dtype, int64_t M,
                         const uint16_t* gate_w_bf16, const float* bias, void* y_out,
                         int y_dtype, int32_t* idx_out, float* weight_out, void* workspace,
                         size_t workspace_bytes, void* stream);

/* Same expert computation with routing supplied (idx int32 [M][top_k], w f32
 * [M][top_k], e.g. from k3_moe_route): the expert loop of moe.py:115-127 + shared
 * expert (:131) alone. The input x here is the expert input h (latent or hidden). */
K3_API int k3_moe_experts_decode(const k3_moe_params* p, const void* x, int x_dtype, int64_t M,
                                 const int32_t* idx, const float* w, void* y_out, int y_dtype,
                                 void* workspace, size_t workspace_bytes, void* stream);

/* One expert's unweighted SwiGLU FFN: LatentMoE.expert_forward (air_llm/models/kimi_k3/
 * moe.py:90-103), y [M][H] = act(x W1^T, x W3^T) W2^T of pool slot `expert` (a routed
 * expert id, or num_experts for an MXFP4 shared expert). Three launches (x pieces,
 * gate/up, down) on the block-scaled pool; no routing plan. Limits: 1 <= M <= 8, H % 512
 * == 0, I % 512 == 0, a block-scaled pool (p->experts may be NULL). x f32|bf16, y
 * f32|bf16. */
K3_API size_t k3_moe_expert_forward_workspace(const k3_moe_params* p, int64_t M);
K3_API int k3_moe_expert_forward(const k3_moe_params* p, const void* x, int x_dtype, int64_t M,
                                 int64_t expert, void* y_out, int y_dtype, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------ prefill --- */

/* Prefill (any number of tokens T, meant for T in the hundreds to thousands) MoE block
 * without the latent wrapper: the same computation as k3_moe_decode -- route, every routed
 * expert y[t] += w[t,slot] * act(x W1^T, x W3^T) W2^T, plus the shared expert -- for the
 * BASELINE layer at prefill (replaces LatentMoE.__call__'s route + per-expert loop + shared
 * expert, air_llm/models/kimi_k3/moe.py:110-132; oracle k3ref/layers.py:241-261). The
 * pairs are grouped by expert and run as two block-scaled grouped GEMMs; the experts'
 * contributions to a token are added in fp32 in an order that is not fixed (results agree
 * with the ascending-expert sum to fp32 rounding). The activations enter the tensor cores
 * as 4 E2M1 pieces per value (relative error ~4e-5 on x, ~2e-4 on the activation).
 * Needs the block-scaled tile pool (k3_expert_pool *_scales_tc and *_tiles), H and I
 * multiples of 256, E <= 1024, top_k <= 32. x [T][H] f32|bf16 (bf16 routes on the tensor
 * cores); y [T][H] f32|bf16; idx_out/weight_out [T][top_k] may be NULL. */
K3_API size_t k3_moe_prefill_workspace(const k3_moe_params* p, int64_t T);
K3_API int k3_moe_prefill(const k3_moe_params* p, const void* x, int x_dtype, int64_t T,
                          const uint16_t* gate_w_bf16, const float* bias, void* y_out, int y_dtype,
                          int32_t* idx_out, float* weight_out, void* workspace,
                          size_t workspace_bytes, void* stream);

/* Same with the routing supplied (idx int32 [T][top_k], w f32 [T][top_k]; entries outside
 * [0, E) are skipped): the expert loop of moe.py:115-127 + shared expert (:131). Uses the
 * k3_moe_prefill_workspace size. */
K3_API int k3_moe_experts_prefill(const k3_moe_params* p, const void* x, int x_dtype, int64_t T,
                                  const int32_t* idx, const float* w, void* y_out, int y_dtype,
                                  void* workspace, size_t workspace_bytes, void* stream);

/* Prefill form of k3_moe_pairs_decode: n_pairs (slot, token row, weight) candidates, any
 * number; slots index the pool (candidates outside [0, num_slots) or with a token outside
 * [0, T) are skipped); y_out[t] = sum of weight * expert(slot)(x[t]) over t's candidates
 * (rows without any are zero). The expert-parallel prefill runs its local experts (and its
 * own tokens' shared expert) through this. */
K3_API size_t k3_moe_pairs_prefill_workspace(const k3_moe_params* p, int64_t T, int64_t n_pairs);
K3_API int k3_moe_pairs_prefill(const k3_moe_params* p, const void* x, int x_dtype, int64_t T,
                                const int32_t* pair_slot, const int32_t* pair_tok,
                                const float* pair_w, int64_t n_pairs, void* y_out, int y_dtype,
                                void* workspace, size_t workspace_bytes, void* stream);

/* Local expert computation of one expert-parallel rank, straight from the gathered
 * routing (no candidate arrays): x [T][H] holds every rank's tokens, idx/w the routing of
 * each token row (top_k entries per row, rows route_stride elements apart). This rank's
 * pool holds routed experts [expert_lo, expert_lo + num_experts) in slots 0.. and, with
 * has_shared, the shared expert in slot num_experts, applied to token rows
 * [shared_t0, shared_t0 + shared_n) with weight 1. y_out[t] = sum over t's local experts
 * of w * expert(x[t]) (+ shared), rows with none are zero. Up to 1024 candidates
 * (T * top_k + shared_n) run on the decode kernels, more on the prefill kernels. */
K3_API size_t k3_moe_ep_local_workspace(const k3_moe_params* p, int64_t T, int64_t shared_n);
K3_API int k3_moe_ep_local(const k3_moe_params* p, const void* x, int x_dtype, int64_t T,
                           const int32_t* idx, const float* w, int64_t route_stride, int32_t expert_lo,
                           int32_t shared_t0, int32_t shared_n, void* y_out, int y_dtype,
                           void* workspace, size_t workspace_bytes, void* stream);

/* Counted all-to-all token exchange of an expert-parallel step (prefill sizes). The
 * reference runs every routed expert in one process (air_llm/models/kimi_k3/moe.py:119-127:
 * per-expert gather of its tokens, weighted scatter-add of the outputs); these three calls
 * split that loop over ranks, rank d owning experts [d*experts_per_rank, (d+1)*experts_per_rank).
 *
 * k3_ep_a2a_plan: from this rank's routing idx [M][route_stride] (top_k ids per row), the
 * send plan: token t goes once to every rank owning one of its experts and always to its
 * own rank. send_counts[W] / send_offs[W] (int64: the collective's split sizes and their
 * exclusive prefix), send_rows[offs[d] + i] = the i-th token for rank d (ascending), and
 * tok_slot[t][W] = t's row in the send buffer for rank d, or -1. send_rows needs M*W
 * entries. *status (device int) becomes K3_ERR_INVALID for an expert id outside
 * [0, experts_per_rank * world) (the id is skipped). */
K3_API int k3_ep_a2a_plan(const int32_t* idx, int64_t route_stride, int64_t M, int top_k,
                          int experts_per_rank, int world, int rank, int64_t* send_counts,
                          int64_t* send_offs, int32_t* send_rows, int32_t* tok_slot, int32_t* status,
                          void* stream);
/* dst[i] = src[rows[i]] for n rows of row_bytes bytes (a multiple of 4; src and dst 4-byte
 * aligned): packs the send buffer (tokens and their routing rows). *status becomes
 * K3_ERR_INVALID for a row index outside [0, n_src). */
K3_API int k3_ep_gather_rows(const void* src, int64_t n_src, int64_t row_bytes, const int32_t* rows,
                             int64_t n, void* dst, int32_t* status, void* stream);
/* y_out[t] = base[t] + the sum over d = 0..world-1 of (d == rank and own given ? own[t] :
 * part[tok_slot[t][d]]) (rows with -1 skipped), in that order, in fp32: a token's shared
 * expert output (base), its own rank's partial row (own: the rank's own token rows, which
 * need not travel) and the partial rows the reverse all-to-all returned (part, in the send
 * buffer's layout). base and own are optional [M][H] (NULL: absent); part [n_part][H]
 * fp32; all 16-byte aligned, H % 4 == 0, y f32/bf16. */
K3_API int k3_ep_a2a_combine(const float* base, const float* own, int rank, const float* part,
                             int64_t n_part, const int32_t* tok_slot, int64_t M, int world, int64_t H,
                             void* y_out, int y_dtype, int32_t* status, void* stream);

/* Expert-parallel exchanges over NVLink peer memory (an alternative to the NCCL
 * all_gather / reduce_scatter of a decode step; the reference has one process and no
 * exchange: air_llm/models/kimi_k3/moe.py:119-127). Every rank owns one exchange buffer of
 * k3_p2p_buffer_bytes (zeroed before first use) and maps every peer's through CUDA IPC
 * (k3_p2p_export on the owner, k3_p2p_open on the others). Layout: a 1 KB header, then
 * gather areas 0 and 1 and the reduce area, world slots each (k3_p2p_area_offsets). Waits
 * are bounded (2 s, then K3_ERR_TIMEOUT in *status; the group must then be rebuilt). */
typedef struct {
    int32_t world, rank;
    int64_t gather_bytes, gather2_bytes, reduce_bytes;   /* slot capacities */
    void* base[32];        /* every rank's buffer as mapped in this process (own at [rank]) */
} k3_p2p_group;
K3_API size_t k3_p2p_buffer_bytes(int world, int64_t gather_bytes, int64_t gather2_bytes, int64_t reduce_bytes);
/* offsets_out[4]: gather area 0, gather area 1, reduce area, total bytes. */
K3_API int k3_p2p_area_offsets(int world, int64_t gather_bytes, int64_t gather2_bytes, int64_t reduce_bytes,
                               int64_t* offsets_out);
/* IPC handle (64 bytes) of the allocation holding ptr, and ptr's offset in it. */
K3_API int k3_p2p_export(const void* ptr, uint8_t* handle_out, int64_t* offset_out);
K3_API int k3_p2p_open(const uint8_t* handle, int64_t offset, void** ptr_out);
K3_API int k3_p2p_close(void* ptr, int64_t offset);
/* All-gather: src (bytes) and src2 (bytes2), multiples of 16, go to slot `rank` of gather
 * areas 0 and 1 of every rank (slot stride = this call's size, so each area holds the
 * world's rows contiguously); mode 1 = put and publish, 2 = wait for the peers, 3 = both. */
K3_API int k3_p2p_allgather(const k3_p2p_group* g, const void* src, int64_t bytes, const void* src2,
                            int64_t bytes2, int mode, int32_t* status, void* stream);
/* Reduce-scatter: src holds world chunks of n floats (chunk d for rank d); out[i] = sum over
 * ranks s ascending of rank s's chunk for this rank, fp32. Modes as for the all-gather
 * (2: wait and sum). */
K3_API int k3_p2p_reduce_scatter(const k3_p2p_group* g, const float* src, int64_t n, float* out, int mode,
                                 int32_t* status, void* stream);

/* Latent MoE decode (Kimi-K3, air_llm/models/kimi_k3/moe.py:110-127): the router reads
 * x_router [M][H_router] (the hidden state), the routed experts read x_expert [M][hidden]
 * (the latent state, p->hidden wide); y_out [M][hidden] = the weighted sum of the routed
 * experts (+ an MXFP4 shared expert when p->has_shared). One fused router launch (logits,
 * expert-input E2M1 pieces, top-k, plan) and the block-scaled expert kernels; needs the
 * block-scaled pool and H_router % 512 == 0. logits_out (optional, [M][E] fp32) receives
 * the router logits, from which RouterResult's raw / corrected scores follow. */
K3_API size_t k3_moe_decode_latent_workspace(const k3_moe_params* p, int64_t M, int64_t H_router);
K3_API int k3_moe_decode_latent(const k3_moe_params* p, const void* x_router, int xr_dtype, int64_t H_router,
                                const void* x_expert, int xe_dtype, int64_t M, const uint16_t* gate_w_bf16,
                                const float* bias, void* y_out, int y_dtype, int32_t* idx_out,
                                float* weight_out, float* logits_out, void* workspace,
                                size_t workspace_bytes, void* stream);

/* ------------------------------------------------- dense bf16 matvecs ----- */

/* The Kimi-K3 layer's dense bf16 parts around the MXFP4 experts, at decode (M <= 8
 * tokens): the latent projections `flat @ down.T` and `rmsnorm(y) @ up.T`
 * (air_llm/models/kimi_k3/moe.py:116, 128-129), the bf16 shared expert
 * `shared_forward` (moe.py:105-107) and the lm_head logits (model.py:111-133). fp32
 * products and sums over bf16 weights, as the reference computes them.
 *
 * One segment is out += X W^T with W bf16 [N][K] (row stride ldw elements, 16-byte
 * aligned, K and ldw multiples of 8) and X [M][K] f32 or bf16 (row stride ldx). With
 * norm_w set, X is first replaced by norm_w * X * rsqrt(mean(X^2) + eps) per row
 * (ops.rmsnorm, ops.py:11-14). With act_input set, each input row holds [gate | up]
 * (2K values, ldx >= 2K) and X = act(gate, up) with the call's activation, formed as the
 * input is staged (the bf16 shared expert's act(x Wg^T, x Wu^T), moe.py:105-107, fed to
 * its down projection); act_input excludes norm_w and K3_DENSE_ACT. */
typedef struct k3_dense_seg {
    const uint16_t* w;
    int64_t ldw;
    int64_t K;
    const void* x;
    int32_t x_dtype;
    int64_t ldx;
    const float* norm_w;
    float eps;
    int32_t act_input;
} k3_dense_seg;

enum {
    K3_DENSE_SUM = 0,   /* out = sum over the segments of X_s W_s^T                        */
    K3_DENSE_ACT = 1    /* two segments (gate, up) over segment 0's X: out = act(X Wg^T, X Wu^T) */
};

/* Workspace bytes for k3_dense_matvec with M tokens, N output rows and nseg segments of
 * K0 (and K1) columns. */
K3_API size_t k3_dense_workspace(int64_t M, int64_t N, int nseg, int64_t K0, int64_t K1);
/* out [M][N] (row stride ldo, f32 or bf16). `activation` (K3_ACT_SILU / K3_ACT_SITU,
 * situ_linear_beta <= 0 for none) is read for K3_DENSE_ACT and act_input segments only.
 * The result does not depend on timing: the split-k partial sums are added in a fixed
 * order. */
K3_API int k3_dense_matvec(const k3_dense_seg* segs, int nseg, int64_t M, int64_t N, int combine,
                           int activation, float situ_beta, float situ_linear_beta, void* out,
                           int out_dtype, int64_t ldo, void* workspace, size_t workspace_bytes,
                           void* stream);

/* The same dense projections for many tokens (a Kimi-K3 layer above 8 tokens: latent down
 * and up, shared expert -- air_llm/models/kimi_k3/moe.py:105-107,116,128-131, where MLX
 * multiplies the layer's bf16 weights with fp32 activations): out [M][N] (row stride ldo)
 * = X [M][K] . W [N][K]^T, or out += that when `accumulate` is set (a second segment into
 * the same output). W bf16 with row stride ldw; X f32 or bf16 with row stride ldx. fp32 X
 * enters the bf16 tensor cores (tcgen05 kind::f16) as two bf16 pieces (hi, lo) with fp32
 * accumulation (~16 significant bits of x); bf16 X is exact. K must be a multiple of 64
 * and W's rows 16-byte aligned. Deterministic (fixed k order). */
K3_API size_t k3_dense_gemm_workspace(int64_t M, int64_t K);
K3_API int k3_dense_gemm(const void* x, int x_dtype, int64_t ldx, int64_t M, int64_t K, const uint16_t* w,
                         int64_t ldw, int64_t N, float* out, int64_t ldo, int accumulate, void* workspace,
                         size_t workspace_bytes, void* stream);

/* Streamed lm_head argmax (`KimiK3.logits`, air_llm/models/kimi_k3/model.py:111-133): for
 * one hidden row h [H] (f32 or bf16) and W bf16 [V][H], idx_out = argmax_n h . W[n]
 * (lowest n on ties, as the reference's first-occurrence argmax over ascending chunks)
 * and val_out = that logit, both device scalars; logits_out (optional, [V] f32) receives
 * every logit. The reference's byte count is V * H * 2 by construction. */
K3_API size_t k3_lm_head_workspace(int64_t H, int64_t V);
/* Status of the last dense call on `workspace` (synchronises `stream`): K3_OK, or
 * K3_ERR_TIMEOUT when a kernel's bounded wait gave up. */
K3_API int k3_dense_status(const void* workspace, void* stream);
K3_API int k3_lm_head_argmax(const void* h, int h_dtype, int64_t H, const uint16_t* w, int64_t V,
                             int32_t* idx_out, float* val_out, float* logits_out, void* workspace,
                             size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------ caller step ----- */

/* The MoE input of a Kimi-K3 decoder layer (air_llm/models/kimi_k3/layer.py:120-121):
 * out [N][H] = post_norm * rmsnorm(apply_attn_res(prefix_sum, block_residual, res_proj,
 * res_norm)) — a softmax over the n_blocks checkpoints block_residual [N][n_blocks][H]
 * plus prefix_sum [N][H], each scored by its RMS-normalised dot with res_norm * res_proj
 * (ops.py:61-74). fp32 inputs and weights; out f32 or bf16; n_blocks <= 16. */
K3_API int k3_attn_res_norm(const float* prefix_sum, const float* block_residual, int64_t n_blocks, int64_t N,
                            int64_t H, const float* res_proj, const float* res_norm, const float* post_norm,
                            float eps, void* out, int out_dtype, void* stream);

/* ------------------------------------------------------ checkpoint reads ----- */

/* Byte ranges of one checkpoint file (manifest records: offset, nbytes —
 * tools/k3_manifest.py:97-156) into host memory with pread on `threads` threads.
 * Ranges adjacent in the file and in memory are read as one (the reference's one-read
 * packed + scale pair, air_llm/models/kimi_k3/loader.py:229-266). *bytes_read_out
 * (optional) = the bytes delivered. K3_ERR_IO on open/read failures, K3_ERR_INVALID for
 * ranges outside the file. */
K3_API int k3_file_read_ranges(const char* path, const int64_t* offsets, const int64_t* nbytes, int n,
                               void* const* dst, int threads, int64_t* bytes_read_out);
/* The same ranges into device memory through a caller-owned pinned staging buffer
 * (>= 8 KiB, used as two halves: the read of one half overlaps the host->device copy of
 * the other on `stream`). Returns after every copy has finished. */
K3_API int k3_file_read_to_device(const char* path, const int64_t* offsets, const int64_t* nbytes, int n,
                                  void* const* device_dst, void* pinned_staging, size_t staging_bytes,
                                  int threads, void* stream);

/* Device status word of the last prefill call on `workspace` (synchronises `stream`):
 * K3_OK, or K3_ERR_TIMEOUT when a kernel's bounded wait gave up. */
K3_API int k3_moe_prefill_status(const void* workspace, void* stream);

/* ------------------------------------------------------- failure detection ----- */

/* Self-test of the bounded device-side wait every pipelined kernel here uses (an
 * mbarrier wait that gives up after a time limit, writes K3_ERR_TIMEOUT into the call's
 * status word and returns, so the context stays usable). One CTA waits on a barrier whose
 * completion `mode` decides: 0 = nothing arrives, the wait runs out after limit_ns
 * (1e3..2e9); 1 = another warp arrives, the wait succeeds; 2 = another warp raises the
 * abort flag, the wait gives up without a timeout. result (device int32[3]) <- {status
 * word, 1 if the wait succeeded else 0, nanoseconds waited}. No reference counterpart:
 * the reference's guards are host-side (air_llm/models/kimi_k3/model.py:211-216,
 * loader.py:246-247) and it has no device waits. */
K3_API int k3_wait_selftest(int64_t limit_ns, int mode, int32_t* result, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* K3B200_H */
