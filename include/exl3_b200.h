/* C ABI of the B200 EXL3 trellis library (libexl3_b200.so).
 *
 * Plain device pointers, sizes and a CUDA stream (passed as void*, a cudaStream_t; NULL = legacy default stream).
 * Every entry point returns EXL3_OK or an error code and never throws; exl3_last_error() gives the text of the
 * calling thread's last failure. No entry point allocates device memory except where stated; scratch comes from
 * the caller as (workspace, ws_bytes) sized by the matching *_workspace_size function. All launches go on the
 * given stream, so calls are CUDA-graph capturable when the caller's buffers are fixed.
 *
 * Layouts (exllamav3 EXL3, unchanged): trellis = int16 [k/16][n/16][16*K] (a 16x16 tile of K-bit weights is
 * 8*K little-endian uint32 words); suh = fp16 [k]; svh = fp16 [n]; activations row-major [rows][k].
 * Reference interfaces are cited as paths inside horvay/b70-inference.
 */
#ifndef EXL3_B200_H
#define EXL3_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define EXL3_API __attribute__((visibility("default")))
#else
#define EXL3_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define EXL3_OK 0
#define EXL3_ERR_ARG 1          /* invalid argument (shape, pointer, alignment) */
#define EXL3_ERR_UNSUPPORTED 2  /* valid but not supported (codebook, K, size) */
#define EXL3_ERR_WORKSPACE 3    /* workspace missing or too small */
#define EXL3_ERR_CUDA 4         /* CUDA runtime error (launch, attribute) */
#define EXL3_ERR_TIMEOUT 5      /* a device-side wait gave up (recorded in the device status word) */

/* element types */
#define EXL3_F16 0
#define EXL3_BF16 1
#define EXL3_F32 2

/* router kinds */
#define EXL3_ROUTE_SIGMOID 0       /* noaux_tc sigmoid: glm/xpu/glm_xpu/ops.py:177-193 */
#define EXL3_ROUTE_SOFTMAX 1       /* Qwen-Next softmax: trellis-serve.patch:394-441 */
#define EXL3_ROUTE_SQRT_SOFTPLUS 2 /* DeepSeek-V4 sqrt(softplus): dsv41/xpu/csrc/dsv_moe_glue.sycl:155-193 */

/* One expert's three EXL3 matrices (device addresses). The shared expert is an ordinary entry.
 * trellis[0] = gate|up packed by exl3_pack_gateup, trellis[1] unused, trellis[2] = down packed by exl3_pack.
 * Replaces the int64 pointer tables of exllamav3's BC_BlockSparseMLP / exl3_mgemm
 * (glm/docs/ext-op-inventory.md:1018-1024,1104-1120) and the per-expert blob of
 * glm/xpu/csrc/exl3_moe.n128.sycl:3-13 (K may differ per matrix, as the DSV piece tables allow,
 * dsv41/xpu/csrc/dsv_moe.sycl:24-143). */
typedef struct exl3_expert {
    const void* trellis[3]; /* packed gate|up, (unused), packed down; gate/up k = hidden, n = interm */
    const void* suh[3];     /* fp16 [k] */
    const void* svh[3];     /* fp16 [n] */
    int32_t K[3];           /* bits per weight, 1..8 */
    int32_t pad;
} exl3_expert;

/* ---- library ---- */
EXL3_API int exl3_version(void);
EXL3_API const char* exl3_last_error(void);
/* Device status word (sticky EXL3_ERR_TIMEOUT from bounded device waits); reset != 0 clears it. Synchronous. */
EXL3_API int exl3_device_status(int reset);
/* Failure-path check of the bounded device waits: launches one thread that waits, with the library's wait and a
 * limit of limit_ns (0 < limit_ns <= 100 ms, the library's own limit), on an mbarrier that nothing completes. The
 * wait runs out, EXL3_ERR_TIMEOUT is recorded in the device status word and the kernel returns; the context stays
 * usable. Every kernel's waits (TMA stages, accumulator hand-offs, tensor-memory stages) use the same wait with the
 * 100 ms limit. No reference counterpart: the reference's SYCL kernels do not wait on one another. */
EXL3_API int exl3_wait_probe(uint64_t limit_ns, void* stream);
/* How long the decode GEMVs' finisher of a unit split over CTAs waits for the other contributors' partials before it
 * hands the unit to whichever contributor completes the count (0 <= wait_ns <= 100 ms; default 20 us). Results are
 * the same bits for any value (the partials are summed in CTA order on every path); 0 exercises the hand-off path
 * (tests). Applies to launches made after the call, on every device. No reference counterpart. */
EXL3_API int exl3_set_finisher_wait(uint64_t wait_ns);

/* ---- dequantisation ----
 * W_hat[:, n0 : n0 + n_slice] -> w (fp16 [k][n_slice], row stride ldw elements), Hadamard domain, no scales.
 * Replaces exl3_reconstruct (glm/xpu/csrc/exl3_ops.sycl:539-555) and exllamav3 reconstruct/reconstruct_slice
 * (glm/docs/ext-op-inventory.md:597-612). cb must be 2 (mul1). Bit-exact with the reference decode. */
EXL3_API int exl3_dequant(const void* trellis, int k, int n, int K, int cb, int n0, int n_slice, void* w, int ldw,
                 void* stream);

/* ---- Hadamard ----
 * Blockwise 128-point Hadamard, out = H(x [* pre]) * scale/sqrt(128) [* post] (pre wins if both given).
 * dtype: EXL3_F16 (in/out fp16, products rounded to fp16) or EXL3_F32. cols % 128 == 0. In place allowed.
 * Replaces had_r_128 (glm/xpu/glm_xpu/ops.py:132-142; glm/docs/ext-op-inventory.md:576-595) and the
 * exl3_had_in_rm / exl3_had_out_h ops (glm/xpu/csrc/exl3_ops.sycl:781-811). */
EXL3_API int exl3_had_r_128(const void* in, void* out, int dtype, int rows, int cols, const void* pre, const void* post,
                   float scale, void* stream);

/* ---- packed trellis layout ----
 * The GEMV kernels read weights column-block-major: for each 128-column block cb and tile-row r (16 input rows) the
 * 8 tiles of the block are contiguous, [n/128][k/16][8 tiles][8K words] (a fused gate|up pair: [I/128][H/16]
 * [8 gate tiles | 8 up tiles]), so that each CTA streams one contiguous slice with large TMA bulk copies. It is a
 * byte permutation of the exllamav3 layout, made once at load time, like the reference's expert blob packing
 * (pack_expert / planar4, glm/xpu/exl3xpu/moe_offload.py:68-94). out must not alias the input. */
EXL3_API int exl3_pack(const void* trellis, int k, int n, int K, void* out, void* stream);
EXL3_API int exl3_pack_gateup(const void* gate, const void* up, int H, int I, int Kg, int Ku, void* out,
                              void* stream);

/* ---- EXL3 linear, decode sizes ----
 * y[M][n] = Had(Had(x * suh) @ W_hat) * svh for M <= 16 rows (9..16 rows: every decoded weight fragment feeds two
 * MMAs, so the weights are decoded once per call; larger M: call per 16-row chunk, or use exl3_gemm_tc); x fp16 or
 * bf16 (x_dtype), y fp16/bf16/fp32 (y_dtype) with row strides ldx, ldy.
 * packed = the weights in the packed layout (exl3_pack). k % 128 == 0, n % 128 == 0, 1 <= K <= 8, cb == 2.
 * workspace >= exl3_gemv_workspace_size(M, k, n) bytes (rotated input rows, split-unit reduction state; calls that
 * share a workspace must be ordered on one stream). n_ctas = CTAs of the persistent launch (0 = one per SM).
 * Weights are decoded bit for bit up to the codebook's final fp16 affine, which is applied to the fp32-accumulated
 * dot product instead (the reference's fold form, glm/xpu/csrc/exl3_esimd.h:82-91: the product uses the unrounded
 * affine, within half an fp16 ulp of each weight); results are identical from call to call for one n_ctas.
 * Replaces exl3_gemm_small (glm/xpu/csrc/exl3_ops.sycl:258-321) / exllamav3 exl3_gemm
 * (glm/docs/ext-op-inventory.md:498-557) as called by BC_LinearEXL3.run (glm/xpu/glm_xpu/ops.py:60-80). */
EXL3_API size_t exl3_gemv_workspace_size(int M, int k, int n);
EXL3_API int exl3_gemv(const void* x, int x_dtype, int ldx, int M, const void* packed, const void* suh,
                       const void* svh, int k, int n, int K, int cb, void* y, int y_dtype, int ldy, void* workspace,
                       size_t ws_bytes, int n_ctas, void* stream);

/* ---- EXL3 linear, prefill sizes (tcgen05) ----
 * y[M][n] = Had(Had(x * suh) @ W_hat) * svh for any M, on the 5th-generation tensor cores: trellis tiles decoded to
 * the reference's fp16 weights bit for bit straight into tensor memory, tcgen05.mma.cta_group::2 kind::f16 (weights
 * from tensor memory, rotated activations from shared memory) with fp32 accumulation, 256 x 256 tiles per pair of
 * SMs. k % 128 == 0, n % 128 == 0, 1 <= K <= 8, cb == 2; packed = exl3_pack; suh, svh 8-byte aligned.
 * workspace >= exl3_gemm_tc_workspace_size(M, k) bytes, 256-byte aligned (the rotated input rows).
 * Replaces the reconstruct + GEMM linear for M > 128 (glm/xpu/csrc/exl3_ops.sycl:539-555,651-757) and exllamav3
 * exl3_gemm's large-M shapes (glm/docs/ext-op-inventory.md:498-557). */
EXL3_API size_t exl3_gemm_tc_workspace_size(int M, int k);
EXL3_API int exl3_gemm_tc(const void* x, int x_dtype, int ldx, int M, const void* packed, const void* suh,
                          const void* svh, int k, int n, int K, int cb, void* y, int y_dtype, int ldy,
                          void* workspace, size_t ws_bytes, void* stream);

/* No-allocation variant of exl3_gemv: same arguments minus the workspace and n_ctas; its scratch is a fixed
 * file-scope device array (1,845,248 bytes per device that loads the library: the rotated input rows and their
 * block sums, the split tickets and the partial slots, sized from the limits below), for callers that cannot
 * allocate device memory. Limits: M <= 8, k <= 32768, n <= 65536 (larger shapes return EXL3_ERR_UNSUPPORTED).
 * Calls on one device that may overlap race on the shared scratch: order them on one stream. Make the first call on
 * each device outside stream capture (it looks up the scratch's address). No reference counterpart. */
EXL3_API int exl3_gemv_noalloc(const void* x, int x_dtype, int ldx, int M, const void* packed, const void* suh,
                               const void* svh, int k, int n, int K, int cb, void* y, int y_dtype, int ldy,
                               void* stream);

/* ---- several EXL3 linears over pointer tables (exl3_mgemm) ----
 * Slot j (0 <= j < slots) uses matrix q = indices[j] (or j when indices is null); with min_index >= 0 only
 * q in [min_index, max_index) are kept, rebased to q - min_index; negative or out-of-range q skip the slot.
 *   C[j][m][n] = lin(A[a_batches == 1 ? 0 : j], matrix q)                 (weights null; skipped slots untouched)
 *   C[t][m][n] = sum over slots j of token t of weights[j] * lin(...)     (weights given; slots / num_tokens per
 *                                                                          token, summed in slot order in fp32)
 * A [a_batches][m][k] fp16/bf16 (row stride lda); trellis_ptrs / suh_ptrs / svh_ptrs: device arrays of n_mats device
 * addresses (trellis packed by exl3_pack; a zero suh entry means no input signs), K_per_mat device int32 [n_mats];
 * indices device int32 [slots] or null; weights device fp32 [slots] or null; C fp16/bf16/fp32 (row stride ldc).
 * k % 128 == 0, n % 128 == 0. Unweighted fp16 C follows the fp16 linear's rounding; weighted sums accumulate in
 * fp32 (the reference accumulates fp16 C with fp16 additions). workspace >= exl3_mgemm_workspace_size(...),
 * 256-byte aligned. Replaces exllamav3 exl3_mgemm (glm/docs/ext-op-inventory.md:664-688,1104-1120), without its
 * sliced mode (size_n_list / c_ptrs, used only by attention). */
EXL3_API size_t exl3_mgemm_workspace_size(int slots, int m, int k, int n, int n_mats);
EXL3_API int exl3_mgemm(const void* A, int a_dtype, int a_batches, int lda, int m, int k, int n,
                        const uint64_t* trellis_ptrs, const uint64_t* suh_ptrs, const uint64_t* svh_ptrs,
                        const int32_t* K_per_mat, int n_mats, const int32_t* indices, int slots, const float* weights,
                        int num_tokens, int min_index, int max_index, void* C, int c_dtype, int ldc, void* workspace,
                        size_t ws_bytes, void* stream);

/* ---- activation ----
 * z = fp16(min(silu(g), L) * clamp(u, -L, L)), L = act_limit (0 disables the clamps); fp32 math.
 * g, u, z fp16 [count]; z may alias u. Replaces silu_mul (glm/xpu/glm_xpu/ops.py:147-154). */
EXL3_API int exl3_silu_mul(const void* g, const void* u, void* z, int64_t count, float act_limit, void* stream);

/* ---- router ----
 * Top-k per row of logits fp32 [R][E] (row stride ld), E <= 1024, k <= 32.
 * score = sigmoid(l) | l (softmax kind) | sqrt(softplus(l)) (l > 20 -> l), evaluated in fp64 and rounded once;
 * key = score * mul + bias + res (each optional, fp32 [E]); res is the residency (locality) bias:
 * 0 resident, -margin slower tier, -inf unreadable, or +b on a resident subset.
 * picks: k argmax passes, ties to the lowest expert index; ids[r][j] = j-th best (int32, or int64 if ids64).
 * weights from the unbiased score: sigmoid / sqrt-softplus: w = s * scale / (sum + 1e-20);
 * softmax: w = p / (sum p + 1e-20) if renorm else p. want (optional) = top-k of score + bias.
 * Replaces routing_ds3_nogroup (glm/xpu/glm_xpu/ops.py:177-193) with the residency variant
 * (glm/xpu/glm_xpu/block_graphs.py:146-179), dsv_glue::moe_route (dsv41/xpu/csrc/dsv_moe_glue.sycl:426-440)
 * and fused_xpu.router (trellis-serve.patch:427-441). */
EXL3_API int exl3_route(const float* logits, int ld, int R, int E, int kind, int k, const float* bias, const float* res,
               const float* mul, float scale, int renorm, void* ids, int ids64, float* w, void* want,
               void* stream);

/* Router from the hidden states: logits[r][e] = fp16(hidden[r] . gate_t[e]) (fp32 FMA dot, rounded to fp16 as the
 * reference's routing GEMV does) computed in the same launch as the routing above (the CTA that finishes the logits
 * last routes every row). hidden fp16/bf16 [R][H] (row stride ldh), gate_t fp16 [E][H] (the router weight
 * transposed, as exllamav3's gate_t), R <= 64 (larger batches: a GEMM for the logits, then exl3_route).
 * logits_out (optional) receives the fp16 logits (the reference's `scores`). workspace >=
 * exl3_route_hidden_workspace_size(R, E), zeroed before its first use (each call leaves its ticket at zero).
 * Replaces routing_ds3_nogroup's routing GEMV + top-k (glm/docs/ext-op-inventory.md:958-1004) and the reference's
 * fused route (dsv41/xpu/csrc/dsv_moe_glue.sycl:442-520). */
EXL3_API size_t exl3_route_hidden_workspace_size(int R, int E);
EXL3_API int exl3_route_hidden(const void* hidden, int h_dtype, int ldh, int R, int H, const void* gate_t, int E,
                               int kind, int k, const float* bias, const float* res, const float* mul, float scale,
                               int renorm, void* ids, int ids64, float* w, void* want, void* logits_out,
                               void* workspace, size_t ws_bytes, void* stream);

/* The fused router above with a second router on the same hidden states: gate_t1 fp16 [E1][H] (the next layer's
 * router weight transposed) joins the same GEMV ([R][E + E1] logits in the workspace), and the next layer's picks
 * (ids1, w1; kind1, k1, bias1, mul1, scale1, renorm1 as for exl3_route; no residency bias) come out of the same
 * launch: the layer-ahead prediction the reference uses as a prefetch hint. workspace >=
 * exl3_route_hidden_workspace_size(R, E + E1). Replaces route_fused with w1 (dsv41/xpu/csrc/dsv_moe_glue.sycl:
 * 442-520) and the next-layer router call of glm/xpu/glm_xpu/moe_patch.py:74-84. */
EXL3_API int exl3_route_hidden_pair(const void* hidden, int h_dtype, int ldh, int R, int H, const void* gate_t, int E,
                                    int kind, int k, const float* bias, const float* res, const float* mul,
                                    float scale, int renorm, void* ids, int ids64, float* w, void* want,
                                    void* logits_out, const void* gate_t1, int E1, int kind1, int k1,
                                    const float* bias1, const float* mul1, float scale1, int renorm1, void* ids1,
                                    int ids1_64, float* w1, void* workspace, size_t ws_bytes, void* stream);

/* Router logits for any number of rows on the tensor cores: logits fp32 [R][E] (and logits_f16, optional) =
 * fp16(hidden [R][H] . gate_t [E][H]) with fp32 accumulation (bf16 hidden states are converted to fp16 on the way),
 * the fused router's rounding; then exl3_route selects. H % 32 == 0; hidden and gate_t 16-byte aligned, ldh % 8 == 0.
 * Replaces the routing GEMM of routing_ds3_nogroup at prefill sizes (glm/docs/ext-op-inventory.md:958-1004). */
EXL3_API int exl3_router_logits(const void* hidden, int h_dtype, int ldh, int R, int H, const void* gate_t, int E,
                                float* logits, void* logits_f16, void* stream);

/* ---- MoE decode ----
 * Routed MoE layer for decode batches: out[M][H] (fp32 or fp16) = sum_j w[m][j] * expert_{ids[m][j]}(x[m])
 * (+ expert E, the shared expert, with weight 1 when shared != 0), summed in slot order.
 * expert(x) = down(fp16(min(silu(gate(x)), L) * clamp(up(x), -L, L))), gate/up outputs rounded to fp16.
 * x fp16/bf16 [M][H] (row stride ldx); ids int32 [M][topk] (ids < 0 or >= E skipped); w fp32 [M][topk];
 * experts: device array of E (+1 shared) exl3_expert. H % 128 == 0, I % 128 == 0.
 * Each expert is read once per call whatever number of rows picked it (rows grouped 8 per work item).
 * n_ctas = CTAs of the persistent GEMV launches (0 = one per SM).
 * Replaces exl3xpu_moe::moe_forward (glm/xpu/csrc/exl3_moe.n128.sycl:1338-1439) and exllamav3
 * BC_BlockSparseMLP::run_bszN (glm/docs/ext-op-inventory.md:1030-1041). */
EXL3_API size_t exl3_moe_workspace_size(int M, int topk, int E, int H, int I, int shared);
EXL3_API int exl3_moe_decode(const void* x, int x_dtype, int ldx, int M, const int32_t* ids, const float* w, int topk,
                    const exl3_expert* experts, int E, int shared, int H, int I, float act_limit, void* out,
                    int out_dtype, void* workspace, size_t ws_bytes, int n_ctas, void* stream);

/* The phases of exl3_moe_decode as separate launches on one workspace, in order: exl3_moe_prepare (alignment of
 * pairs into per-expert items + the rotated gate/up input rows), exl3_moe_gateup (gate|up GEMVs + activation +
 * down-input rotation -> activation rows in the workspace), exl3_moe_down (down GEMVs x routing weight -> per-pair
 * rows), exl3_moe_combine (fixed-order sum into out). Same arguments and constraints as exl3_moe_decode.
 * Replace the reference's moe_align / GateUpKernel / DownKernel / CombineKernel launches
 * (glm/xpu/csrc/exl3_moe.n128.sycl:736-790,1418-1438). */
EXL3_API int exl3_moe_prepare(const void* x, int x_dtype, int ldx, int M, const int32_t* ids, const float* w,
                              int topk, const exl3_expert* experts, int E, int shared, int H, int I, void* workspace,
                              size_t ws_bytes, void* stream);
EXL3_API int exl3_moe_gateup(int M, int topk, const exl3_expert* experts, int E, int shared, int H, int I,
                             float act_limit, void* workspace, size_t ws_bytes, int n_ctas, void* stream);
EXL3_API int exl3_moe_down(int M, int topk, const exl3_expert* experts, int E, int shared, int H, int I,
                           void* workspace, size_t ws_bytes, int n_ctas, void* stream);
EXL3_API int exl3_moe_combine(int M, int topk, int E, int shared, int H, int I, void* out, int out_dtype,
                              void* workspace, size_t ws_bytes, void* stream);

/* ---- MoE prefill (tcgen05) ----
 * The routed MoE layer for prefill-sized batches, same contract as exl3_moe_decode (out = slot-order sum of the
 * picks' expert outputs + shared expert). Pairs are grouped per expert into items of <= 320 positions; gate, up and
 * down are grouped tcgen05 GEMMs (as exl3_gemm_tc: trellis decoded to bit-exact fp16 into tensor memory, fp32
 * accumulation), gate and up with fp16 outputs, then SiLU * clamp and the down input's rotation, down with the
 * routing weight; then the fixed-order combine. The experts' suh / svh vectors must be 8-byte aligned.
 * workspace >= exl3_moe_prefill_workspace_size(...), 256-byte aligned.
 * Replaces the reference's MoE prefill (GateUpDpasKernel / DownDpasKernel / moe_prefill,
 * glm/xpu/csrc/exl3_moe.n128.sycl:422-690,868-916) and dsv_xpu moe_prefill_grouped
 * (dsv41/xpu/dsv_xpu/moe.py:1383-1448). */
EXL3_API size_t exl3_moe_prefill_workspace_size(int M, int topk, int E, int H, int I, int shared);
EXL3_API int exl3_moe_prefill(const void* x, int x_dtype, int ldx, int M, const int32_t* ids, const float* w,
                              int topk, const exl3_expert* experts, int E, int shared, int H, int I, float act_limit,
                              void* out, int out_dtype, void* workspace, size_t ws_bytes, void* stream);

/* Alignment step on its own (debug / reuse): writes into the workspace the item table and the pair permutation, in
 * the layout documented in moe.cu. Replaces moe_align (glm/xpu/csrc/exl3_moe.n128.sycl:1442-1450). */
EXL3_API int exl3_moe_align(const int32_t* ids, const float* w, int M, int topk, int E, int shared, int chunk,
                   void* workspace, size_t ws_bytes, void* stream);

/* ---- expert-parallel exchange over peer memory ----
 * The dispatch and combine of an expert-parallel MoE layer (rank r holds experts [r E/W, (r+1) E/W)) as kernels that
 * write straight into the peers' memory over NVLink, in place of two all-to-all collectives per layer (the reference
 * runs on one GPU and has no exchange; it has no counterpart there). Every rank owns one
 * exchange buffer of exl3_ep_buffer_bytes(W, cap, H, topk) bytes, allocated by exl3_ep_buffer_create (cudaMalloc,
 * zeroed, exported as a 64-byte CUDA IPC handle that the caller passes to its peers, e.g. through torch.distributed)
 * and mapped on every peer with exl3_ep_buffer_open. peers = device array of W uint64 buffer addresses (this rank's
 * own at [rank]). Per call, on one stream, in the same order on every rank:
 *   exl3_ep_dispatch  rank r's rows x [B][H] (B <= cap), global ids int32 [B][topk] and weights [B][topk] into every
 *                     peer's receive region (picks rebased to that peer's experts, -1 for others; activations only
 *                     for rows with a pick there), then it waits for every peer's rows (bounded: 100 ms, then
 *                     EXL3_ERR_TIMEOUT in the device status word);
 *   (the caller runs its local experts on the W * cap received rows: recv_x / recv_ids / recv_w at the offsets
 *    exl3_ep_recv_offsets gives, producing part fp32 [W][cap][H])
 *   exl3_ep_combine   every received row that had a pick here goes back to its rank; waits for every peer's rows;
 *   exl3_ep_reduce    out[i] = sum over the ranks row i picked, in rank order, of their partial rows (+ shared[i]);
 *   exl3_ep_combine_reduce  the two steps above in one launch (every CTA waits for the peers' rows, then sums its
 *                     share of out): one kernel boundary less per layer, the same result bit for bit.
 * The calls count themselves on the device, so a captured sequence replays. exl3_ep_buffer_create allocates device
 * memory; no other entry point here does. */
EXL3_API size_t exl3_ep_buffer_bytes(int W, int cap, int H, int topk);
EXL3_API int exl3_ep_recv_offsets(int W, int cap, int H, int topk, size_t* recv_x, size_t* recv_ids, size_t* recv_w);
EXL3_API int exl3_ep_buffer_create(size_t bytes, void** ptr, void* ipc_handle);
EXL3_API int exl3_ep_buffer_open(const void* ipc_handle, void** peer_ptr);
EXL3_API int exl3_ep_buffer_close(void* peer_ptr);
EXL3_API int exl3_ep_buffer_free(void* ptr);
EXL3_API int exl3_ep_dispatch(const void* x, int x_dtype, int ldx, int B, const int32_t* ids, const float* w,
                              int topk, int E, int H, int W, int rank, int cap, const uint64_t* peers, void* local,
                              void* stream);
EXL3_API int exl3_ep_combine(const float* part, int topk, int E, int H, int W, int rank, int cap,
                             const uint64_t* peers, void* local, void* stream);
EXL3_API int exl3_ep_combine_reduce(const float* part, const int32_t* ids, int B, int topk, int E, int H, int W,
                                    int rank, int cap, const float* shared, const uint64_t* peers, void* local,
                                    float* out, void* stream);
EXL3_API int exl3_ep_reduce(const int32_t* ids, int B, int topk, int E, int H, int W, int rank, int cap,
                            const float* shared, void* local, float* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* EXL3_B200_H */
