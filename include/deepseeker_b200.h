/*
 * deepseeker_b200 -- C ABI of the B200 (sm_100a) routed-expert MoE hot path.
 *
 * Every entry point:
 *   - returns an int status (DS_OK = 0); the message of the last failure on
 *     the calling thread is available from ds_last_error_string();
 *   - takes DEVICE pointers for tensors (caller owns every buffer) unless the
 *     name says otherwise, plain integer sizes, and a cudaStream_t passed as
 *     `void* stream` (NULL = legacy default stream);
 *   - launches asynchronously on that stream and never synchronises it;
 *   - allocates nothing: scratch comes from a caller-provided workspace whose
 *     size a matching *_workspace_size() call reports (ds_moe_decode_noalloc
 *     uses a static device array instead).
 * The library is stateless and reentrant across distinct streams.
 *
 * Layout conventions (all row-major, K = input features contiguous):
 *   FP4  : packed [N, K/2] u8, two e2m1 codes per byte, LOW nibble = even
 *          element; scales [N, K/32] u8 (ue8m0: 2^(b-127), 0xFF = NaN).
 *   Q3   : words [N, K*3/32] u32, scales / biases [N, K/64] f16;
 *          w = f32(scale)*q + f32(bias).  One 64-element group = six
 *          little-endian u32 words: word w (0..3) holds the low two bits of
 *          elements 16w+i at bits [2i, 2i+2) (i = 0..15); word 4+h holds
 *          bit 2 of the codes: element 16(2h+v)+j at bit 8v+j and element
 *          16(2h+v)+8+j at bit 16+8v+j (v in {0,1}, j = 0..7).
 *   BF16 : [N, K] bf16.
 *   Expert banks stack E experts: [E, N, ...] with the per-expert layout above.
 */
#ifndef DEEPSEEKER_B200_H
#define DEEPSEEKER_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define DS_OK 0
#define DS_EINVAL 1   /* bad shape / dtype / argument                       */
#define DS_EALIGN 2   /* pointer not aligned as the call requires            */
#define DS_ERANGE 3   /* index out of range (host check or device guard)     */
#define DS_ECUDA 4    /* CUDA runtime error                                  */
#define DS_ETIMEOUT 5 /* a bounded device-side wait gave up                  */
#define DS_ENOTSUP 6  /* unsupported combination                            */

/* ---- element types ----------------------------------------------------- */
#define DS_F32 0
#define DS_BF16 1
#define DS_F16 2
#define DS_U8 3

/* ---- weight formats ---------------------------------------------------- */
#define DS_FMT_FP4 0
#define DS_FMT_Q3 1
#define DS_FMT_BF16 2

/* ---- routing kinds ----------------------------------------------------- */
#define DS_ROUTE_SOFTMAX 0      /* softmax over experts, top-k, renormalised  */
#define DS_ROUTE_SQRTSOFTPLUS 1 /* sqrt(softplus(s)), top-k of s+bias, *scale */
#define DS_ROUTE_SCORES 2       /* input already scores s: top-k of s+bias     */

/* Message of the last failed call on this thread ("" if none). */
const char* ds_last_error_string(void);

/* Library ABI version (major*10000 + minor*100 + patch). */
int ds_version(void);

/* ------------------------------------------------------------------------
 * FP4 e2m1 dequantisation, bit-exact with the reference table.
 * Replaces metal_fp4.metal_dequant / the three Metal kernels
 *   (reference: src/deepseeker/metal_fp4.py:28-66, 139-155) and
 *   mlx_weights.dequant_fp4_rowmajor (src/deepseeker/mlx_weights.py:148-166).
 * out[e] = FP4_TABLE[nibble(e)] * scale[e / 32] in f32 (round-to-nearest,
 * no flush-to-zero), then stored as f32 or bf16 (RNE).
 *   packed     : n_bytes u8 (n = 2*n_bytes elements)
 *   scales     : n_scales entries, f32 (scale_kind = DS_F32) or raw ue8m0
 *                bytes (scale_kind = DS_U8); n_scales must be ceil(n/32)
 *   out        : n elements of out_dtype (DS_F32 or DS_BF16)
 * ------------------------------------------------------------------------ */
int ds_fp4_dequant(const uint8_t* packed, int64_t n_bytes, const void* scales,
                   int scale_kind, int64_t n_scales, void* out, int out_dtype,
                   void* stream);

/* FP8 e4m3 with one ue8m0 scale per 32x32 block -> f32.
 * Replaces mlx_weights.dequant_fp8_block (src/deepseeker/mlx_weights.py:82-89).
 *   packed [rows, cols] u8, scales [rows/32, cols/32] u8, out [rows, cols] f32 */
int ds_fp8_block_dequant(const uint8_t* packed, int64_t rows, int64_t cols,
                         const uint8_t* scales, float* out, void* stream);

/* 3-bit affine (group 64) dequantisation: out = f32(scale)*q + f32(bias)
 * (multiply, then add: two roundings).  Replaces mx.dequantize(bits=3,
 * group_size=64) at src/deepseeker/mlx_forward.py:99-101 and
 * tests/test_q3.py:100-105.  cols % 64 == 0.
 *   words [rows, cols*3/32] u32, scales/biases [rows, cols/64] f16,
 *   out [rows, cols] of out_dtype (DS_F32 or DS_BF16) */
int ds_q3_dequant(const uint32_t* words, const uint16_t* scales,
                  const uint16_t* biases, int64_t rows, int64_t cols,
                  void* out, int out_dtype, void* stream);

/* 3-bit affine quantiser (builder rule: per-64 min/max, scale=(max-min)/7,
 * bias=min, both rounded to f16, q=clamp(rint((w-bias)/scale),0,7)).
 * Replaces mx.quantize(group_size=64, bits=3) in
 * scripts/requant_experts_3bit.py:69-83 (convert_tensor).
 *   w [rows, cols] f32 -> words [rows, cols*3/32], scales, biases [rows, cols/64] */
int ds_q3_quantize(const float* w, int64_t rows, int64_t cols, uint32_t* words,
                   uint16_t* scales, uint16_t* biases, void* stream);

/* FP4 quantiser for synthetic weights (builder rule: per-32 block
 * e = ceil(log2(amax/6)) clamped to [-127,127], RNE onto the e2m1 grid with
 * ties to the even code).  The reference consumes pre-quantised checkpoints
 * (no counterpart); used to build resident banks for tests and benches.
 *   w [rows, cols] f32 -> packed [rows, cols/2] u8, scales [rows, cols/32] u8 */
int ds_fp4_quantize(const float* w, int64_t rows, int64_t cols, uint8_t* packed,
                    uint8_t* scales, void* stream);

/* ------------------------------------------------------------------------
 * Router: per row, choose top_k experts and their gates.
 *   kind = DS_ROUTE_SOFTMAX: softmax over n_experts logits, top-k (ties to the
 *          lower id), gates renormalised to sum 1;
 *   kind = DS_ROUTE_SQRTSOFTPLUS: s = sqrt(softplus(logit)), top-k of s+bias,
 *          gates = s/(sum s + 1e-20) * route_scale
 *          (src/deepseeker/mlx_forward.py:62-81, sqrtsoftplus_scores/route_topk);
 *   kind = DS_ROUTE_SCORES: as SQRTSOFTPLUS with the input already the scores
 *          s (route_topk alone, mlx_forward.py:68-81).
 * Slots are written in descending selection-score order.
 *   logits [rows, n_experts] f32; bias [n_experts] f32 or NULL;
 *   ids [rows, top_k] i32; weights [rows, top_k] f32.  n_experts <= 1024,
 *   top_k <= 32. */
int ds_route_topk(const float* logits, const float* bias, int64_t rows,
                  int n_experts, int top_k, int kind, float route_scale,
                  int32_t* ids, float* weights, void* stream);

/* ------------------------------------------------------------------------
 * Expert banks and the fused routed-expert MoE layer.
 * ------------------------------------------------------------------------ */
typedef struct DsExpertBank {
  int32_t format;     /* DS_FMT_FP4, DS_FMT_Q3 or DS_FMT_BF16                 */
  int32_t n_experts;  /* E                                                    */
  int32_t rows;       /* N: output features                                  */
  int32_t cols;       /* K: input features                                   */
  const void* data;   /* FP4 [E,N,K/2] u8 | Q3 [E,N,K*3/32] u32 | BF16 [E,N,K] */
  const void* scales; /* FP4 [E,N,K/32] u8 | Q3 [E,N,K/64] f16 | BF16 NULL     */
  const void* biases; /* Q3 [E,N,K/64] f16 | otherwise NULL                   */
  const void* scales_tc; /* FP4 only, optional: the scales re-laid into tensor-
                            core atoms by ds_fp4_scale_atoms; when w1, w3 and w2
                            all carry them, ds_moe_decode runs its tcgen05
                            kernels.  NULL otherwise.                         */
} DsExpertBank;

typedef struct DsMoeDesc {
  int32_t hidden;       /* H                                                  */
  int32_t inter;        /* I (routed intermediate size)                       */
  int32_t n_experts;    /* E                                                  */
  int32_t top_k;        /* k                                                  */
  DsExpertBank w1;      /* gate: N = I, K = H                                 */
  DsExpertBank w3;      /* up  : N = I, K = H                                 */
  DsExpertBank w2;      /* down: N = H, K = I                                 */
  /* optional shared expert, BF16 (NULL pointers = none)                      */
  const void* shared_w1; /* [shared_inter, H] bf16                            */
  const void* shared_w3; /* [shared_inter, H] bf16                            */
  const void* shared_w2; /* [H, shared_inter] bf16                            */
  int32_t shared_inter;
  float swiglu_limit;    /* > 0: g = min(g, L), u = clip(u, -L, L); else none */
  int32_t route_before_down; /* 1: h *= gate before the down projection
                                (moe_layer, mlx_forward.py:404-405);
                                0: y *= gate after it (grouped.py:50-53)       */
  int32_t out_f32;       /* ds_moe_decode with bf16 x: 1 writes the layer
                            output in f32 without the final rounding (partial
                            sums that another rank adds to), 0 = x's dtype.
                            Served by FP4 banks with scale atoms, by one
                            token over FP4 banks with swiglu_limit > 0, and
                            by Q3 banks; DS_ENOTSUP otherwise.               */
} DsMoeDesc;

/* Workspace bytes ds_moe_decode needs for `tokens` rows.  The first 4096
 * bytes of a workspace are reserved (error word, control words of the
 * single-token kernel): zero them once before the first call with that
 * workspace (e.g. allocate it zero-filled); every call that completes leaves
 * the control words zero, so layers and token counts may share it.  After a
 * call that reported a bounded-wait timeout, zero it again. */
int ds_moe_decode_workspace_size(const DsMoeDesc* desc, int64_t tokens,
                                 size_t* bytes);

/* Fused routed-expert MoE layer for decode (tokens <= 8): for every distinct
 * routed expert e (ascending id), h = silu(min(x W1e^T, L)) * clip(x W3e^T, ±L)
 * (f32, weights dequantised in registers), scaled by the token's gate, then
 * out += h W2e^T; plus the shared expert (its output rounded to bf16 before
 * the add, as the reference does); out has the dtype of x.
 * Replaces moe_layer's expert loop + qmm + shared add
 *   (src/deepseeker/mlx_forward.py:84-103, 388-419;
 *    src/deepseeker/mlx_runner.py:776-781).
 *   x [tokens, H] of x_dtype (DS_BF16, or DS_F32 for the f32 oracle config);
 *   topk_ids [tokens, k] i32 (-1 = dropped slot); topk_w [tokens, k] f32;
 *   out [tokens, H] of x_dtype. */
int ds_moe_decode(const DsMoeDesc* desc, const void* x, int x_dtype, int64_t tokens,
                  const int32_t* topk_ids, const float* topk_w, void* out,
                  void* workspace, size_t workspace_bytes, void* stream);

/* Router + decode layer in one call: ds_route_topk(logits, route_bias, tokens,
 * n_experts, top_k, route_kind, route_scale) into topk_ids / topk_w (OUTPUTS
 * here, [tokens, k]), then ds_moe_decode with that routing.  Same results as
 * the two calls, bit for bit.  On the tcgen05 kernels (FP4 banks with scale
 * atoms, bf16 x) the routing is computed inside the decode's first kernel
 * (one launch fewer per layer); otherwise the router runs first.
 * Replaces route_topk + the moe_layer expert loop
 *   (src/deepseeker/mlx_forward.py:62-81, 388-419).
 *   logits [tokens, n_experts] f32, route_bias [n_experts] f32 or NULL;
 *   n_experts <= 1024, top_k <= 32; workspace as for ds_moe_decode. */
int ds_moe_decode_route(const DsMoeDesc* desc, const void* x, int x_dtype, int64_t tokens,
                        const float* logits, const float* route_bias, int route_kind,
                        float route_scale, int32_t* topk_ids, float* topk_w, void* out,
                        void* workspace, size_t workspace_bytes, void* stream);

/* One compressed matrix times a batch of activations: out[r, n] =
 * sum_k x[r, k] * W[n, k], W dequantised in registers (exactly: FP4 codes times
 * their ue8m0 scale; Q3 as f32(scale)*q + f32(bias)), f32 accumulate.
 * Replaces qmm (src/deepseeker/mlx_forward.py:84-103: mx.quantized_matmul with
 * mode="mxfp4", or bits=3 / group 64 with biases).
 *   w   : one matrix (n_experts = 1), DS_FMT_FP4 or DS_FMT_Q3, [N = rows, K = cols]
 *   x   : [rows, K] f32 (DS_F32) or bf16 (DS_BF16), 16-byte aligned
 *   out : [rows, N] f32.  K <= 6144 (eight x rows staged in shared memory). */
int ds_qmm(const DsExpertBank* w, const void* x, int x_dtype, int64_t rows, float* out, void* stream);

/* ---- host-fed decode steps: staging without the copy engines ------------ */

/* Device address of pinned host memory (cudaHostGetDevicePointer).  DS_EINVAL
 * when the memory is not pinned and mapped.  No reference counterpart: the
 * reference's MLX arrays live in unified memory. */
int ds_host_device_pointer(const void* host, void** device);

/* Copies n (1..4) byte ranges dst[k] <- src[k] in one kernel launch on
 * `stream`.  Pointers are device addresses (device memory, or pinned host
 * memory through ds_host_device_pointer), 16-byte aligned; bytes[k] is a
 * multiple of 16.  A host-fed decode step stages its inputs in and its
 * output out with it: a copy-engine transfer of a few kilobytes costs
 * several microseconds of latency on the step's critical path, this one
 * launch about as much as one.  No reference counterpart (see above). */
int ds_copy_ranges(int n, void* const* dst, const void* const* src, const size_t* bytes, void* stream);

/* ---- sort-and-pad of routed pairs by expert ---------------------------- */

/* Output capacities ds_moe_align needs for topk_ids [m, k] over n_experts:
 * sorted_cap = m*k + min(n_experts, m*k) * (block - 1), blocks_cap =
 * sorted_cap / block. */
int ds_moe_align_capacity(int64_t m, int k, int n_experts, int block,
                          int64_t* sorted_cap, int64_t* blocks_cap);

/* align_block_size on the device (src/deepseeker/moe_align.py:21-46):
 * flat positions of topk_ids [m, k] (i32, device) grouped by expert in
 * stable order, each expert's run padded with the sentinel m*k to a multiple
 * of block, experts in id order.  Writes sorted_ids (i32), expert_ids (i32,
 * one per block) and *n_pad (device i32, the padded length; -1 when an id is
 * outside [0, n_experts), in which case the other outputs are undefined).
 * n_experts <= 1024. */
int ds_moe_align(const int32_t* topk_ids, int64_t m, int k, int n_experts, int block,
                 int32_t* sorted_ids, int64_t sorted_cap, int32_t* expert_ids,
                 int64_t blocks_cap, int32_t* n_pad, void* stream);

/* ---- batched grouped expert FFN (FP4 banks, tcgen05) ------------------- */

/* FP4 bank scales [E, rows, cols/32] (ue8m0) -> tensor-core scale atoms
 * [E][rows/128][cols/128][512 B]: byte (r%32)*16 + (r/32)*4 + b of an atom is
 * the scale of row r, k-block b of that 128 x 128 tile.  rows and cols must be
 * multiples of 128; atoms holds E*rows*cols/32 bytes (the size of the scales).
 * Run once per resident bank; set DsExpertBank.scales_tc to the result. */
int ds_fp4_scale_atoms(const void* scales, int64_t n_experts, int rows, int cols, void* atoms,
                       void* stream);

/* Bytes of the re-laid-out block scales the grouped kernels read: W1 and W3
 * together (w13_bytes) and W2 (w2_bytes); same totals as the bank scales. */
int ds_grouped_scales_size(const DsMoeDesc* desc, size_t* w13_bytes, size_t* w2_bytes);

/* Re-lay the FP4 bank scales of desc (w1, w3, w2) into the tensor-core scale
 * atoms: for every 128 weight rows and 128-wide K chunk, 512 bytes where byte
 * (r%32)*16 + (r/32)*4 + b is the scale of row r, k-block b.  Run once per
 * resident bank (replaces no reference function: the reference reads the
 * checkpoint scales directly, mlx_weights.py:92-110). */
int ds_grouped_prepare_scales(const DsMoeDesc* desc, void* w13_sf, void* w2_sf, void* stream);

int ds_grouped_ffn_workspace_size(const DsMoeDesc* desc, int64_t tokens, size_t* bytes);

/* Routed-expert SwiGLU FFN for a batch of tokens (prefill / MTP verify):
 * pairs sorted by expert on the device, gate/up and down projections as
 * tcgen05 block-scaled MMAs, f32 accumulate, combine in top-k order.
 * Replaces grouped_swiglu and the moe_layer expert loop / banked gather
 * (src/deepseeker/grouped.py:34-56, src/deepseeker/mlx_forward.py:159-210,
 * 388-419).  FP4 banks: weights as e2m1 operands, activations as exact e4m3
 * pieces.  Q3 banks: the 3-bit codes become exact e4m3 operands in shared
 * memory and each 64-group's f16 scale and bias are applied after the MMA
 * (w13_sf / w2_sf unused, may be null).  Hidden and inter multiples of 128,
 * x bf16 [tokens, hidden], no shared expert (add it separately); topk_ids
 * [tokens, k] (-1 = dropped slot); out [tokens, hidden] of out_dtype (DS_BF16,
 * or DS_F32 for partial sums that are combined later, as the
 * expert-parallel path does).  desc->route_before_down selects where the
 * route weight is applied. */
int ds_grouped_ffn(const DsMoeDesc* desc, const void* w13_sf, const void* w2_sf,
                   const void* x, int x_dtype, int64_t tokens, const int32_t* topk_ids,
                   const float* topk_w, void* out, int out_dtype, void* workspace,
                   size_t workspace_bytes, void* stream);

/* FP4 throughput mode of the grouped FFN: FP4 banks with their scale atoms
 * (DsExpertBank.scales_tc, ds_fp4_scale_atoms) times activations rounded to
 * FP4 as well -- x and h become one e2m1 value per element with a per-32
 * ue8m0 scale that maps the block maximum into (3, 6] -- on tcgen05
 * kind::mxf4 MMAs (K = 64 per instruction, one MMA per weight byte instead of
 * one per activation piece).  The result carries the FP4 rounding of x and h
 * (relative L2 of order 0.1 against the exact layer); it equals, to f32
 * accumulation order, the layer evaluated on the FP4-rounded x and h.  No
 * reference counterpart: the reference's grouped path keeps f32 / bf16
 * activations (src/deepseeker/grouped.py:34-56).  Hidden and inter multiples
 * of 256; other arguments as ds_grouped_ffn. */
int ds_grouped_ffn_fp4_workspace_size(const DsMoeDesc* desc, int64_t tokens, size_t* bytes);
int ds_grouped_ffn_fp4(const DsMoeDesc* desc, const void* x, int x_dtype, int64_t tokens,
                       const int32_t* topk_ids, const float* topk_w, void* out, int out_dtype,
                       void* workspace, size_t workspace_bytes, void* stream);

/* ---- dense-weight pair FFN (grouped_swiglu / naive_swiglu with dense experts) */

int ds_dense_swiglu_workspace_size(int64_t n_pairs, int hidden, size_t* bytes);

/* y_p = w_p * (silu(x_r gate_e) * (x_r up_e)) down_e for every pair p = (r, e)
 * (f32; gate/up [E, H, I], down [E, I, H]; w_p = 1 when pair_weight is NULL;
 * swiglu_limit > 0 clamps as moe_layer does), then out[t] = sum of y_p over
 * the pairs row_ptr[t] .. row_ptr[t+1]-1 in that order
 * (src/deepseeker/grouped.py:34-81). */
int ds_dense_swiglu(const float* x, int64_t tokens, int hidden, int inter, int n_experts,
                    const float* gate, const float* up, const float* down, int64_t n_pairs,
                    const int32_t* pair_row, const int32_t* pair_expert, const float* pair_weight,
                    const int32_t* row_ptr, float swiglu_limit, float* out, void* workspace,
                    size_t workspace_bytes, void* stream);

/* ds_moe_decode without a workspace.  No counterpart in the reference (its
 * MLX runtime owns all scratch); added for callers that may not allocate
 * device memory at all while decoding, e.g. a serving loop whose device memory
 * is carved up once by its own pool.  Scratch comes from a static device array
 * of ds_moe_decode_noalloc_max_scratch() bytes (8 MiB) per device.
 *   - Kernels: exactly those ds_moe_decode runs when given a workspace of
 *     that size (the fastest path whose scratch fits: tcgen05 for FP4 banks
 *     with scale atoms, the single-token register-dequant kernel for one
 *     token over FP4 banks without them, the q3 kernels for Q3 banks, else
 *     the generic ones),
 *     so results equal ds_moe_decode's bit for bit whenever
 *     ds_moe_decode_workspace_size() <= the limit, and stay within the
 *     decode tolerance (rel-L2 <= 1e-3 of the f32 oracle) otherwise.
 *   - Limit: a layer whose generic-path scratch (4096 + (min(tokens*k, E) + 1)
 *     * tokens * max(inter, shared_inter) * 4 bytes, rounded up to 256) exceeds
 *     the array is rejected with DS_ERANGE.
 *   - The first call on each device resolves the array's address (setup,
 *     cudaGetSymbolAddress with that device current); make that first call
 *     before any stream capture and before any latency-sensitive phase.
 *   - Each call clears the array's 4096-byte reserved head (error word and
 *     control words) on `stream` (cudaMemsetAsync); nothing else has to start
 *     at zero.  ds_moe_decode_noalloc_status reads
 *     the word back: bit 0 = an expert id >= n_experts was skipped, bit 1 = a
 *     bounded device wait gave up (outputs of that call are then undefined).
 *   - All calls on one device share the array: two calls that may overlap
 *     (different streams, or host threads without ordering) race on it and
 *     corrupt each other's results.  Serialise them on one stream. */
size_t ds_moe_decode_noalloc_max_scratch(void);
int ds_moe_decode_noalloc(const DsMoeDesc* desc, const void* x, int x_dtype, int64_t tokens,
                          const int32_t* topk_ids, const float* topk_w, void* out,
                          void* stream);
/* Copy the no-allocation scratch's error word of the current device into *err
 * (host or device memory; one cudaMemcpyAsync on `stream`, read it after the
 * stream has finished).  No counterpart in the reference. */
int ds_moe_decode_noalloc_status(int32_t* err, void* stream);

/* ---------------------------------------------------------------------------
 * Expert-parallel decode over NVLink peer memory.
 *
 * Replaces, across G ranks (one process per GPU), the per-layer MoE call of a
 * decode step (src/deepseeker/mlx_runner.py:765-985 Runner.moe ->
 * src/deepseeker/mlx_forward.py:257-419 moe_layer).  Rank r holds experts
 * [first_expert, first_expert + desc->n_experts) of every layer and decodes
 * `rows` tokens per step; the token rows are exchanged and the partial
 * outputs summed by the library's own kernels through CUDA IPC mappings of
 * every rank's region (no collective library on the data path, so a step
 * captures into a CUDA graph).
 *
 * Setup, on every rank with its device current:
 *   ds_ep_create -> ds_ep_ipc_handle -> (exchange the world handles, e.g.
 *   torch.distributed.all_gather_object) -> ds_ep_connect(all handles, in
 *   rank order) -> a barrier, so that no rank writes into a peer before the
 *   peer has connected.
 * Step: every rank calls ds_ep_decode for the same layers in the same order
 * with the same `rows`.  Device waits give up after `timeout_ms`; the error
 * word then holds bit 2 (ds_ep_status), and later calls of that
 * communicator return without exchanging (outputs undefined).
 * Limits: world <= 8, world * max_rows <= 8; FP4 banks with scale atoms,
 * hidden and inter multiples of 1024 (the tcgen05 decode kernels), or Q3
 * banks, hidden and inter multiples of 128 (the CUDA-core q3 kernels). */
#define DS_EP_HANDLE_BYTES 64
typedef struct DsEp DsEp;
int ds_ep_create(int world, int rank, int max_rows, int hidden, int top_k, int timeout_ms, DsEp** ep);
size_t ds_ep_region_bytes(int world, int max_rows, int hidden, int top_k);
int ds_ep_ipc_handle(DsEp* ep, void* handle /* DS_EP_HANDLE_BYTES */);
int ds_ep_connect(DsEp* ep, const void* handles /* world * DS_EP_HANDLE_BYTES, rank order */);
/* Same as ds_ep_connect for communicators created by ONE process (one per
 * device, or several on one device: the single-device form exists to test
 * the bounded waits, since ranks sharing a GPU must not wait on each other).
 * all[world] in rank order, all[rank] == ep; peer access is enabled between
 * distinct devices. */
int ds_ep_connect_peers(DsEp* ep, DsEp* const* all);
int ds_ep_decode_workspace_size(DsEp* ep, const DsMoeDesc* desc, int64_t rows, size_t* bytes);
/* x [rows, hidden] bf16, topk_ids [rows, top_k] GLOBAL expert ids (-1 =
 * none), topk_w [rows, top_k] f32 -> out [rows, hidden] bf16: routed experts
 * of all ranks (route weight before the down projection) plus this layer's
 * shared expert (desc->shared_*, the full matrices on every rank: rank r
 * evaluates intermediate slice r of it for all ranks' rows when
 * shared_inter is a multiple of 256 * world, else all of it for its own
 * rows; its output is rounded to bf16 before it joins the routed sum). */
int ds_ep_decode(DsEp* ep, const DsMoeDesc* desc, int32_t first_expert, const void* x, int64_t rows,
                 const int32_t* topk_ids, const float* topk_w, void* out, void* workspace,
                 size_t workspace_bytes, void* stream);
int ds_ep_status(DsEp* ep, int32_t* err);
int ds_ep_destroy(DsEp* ep);

#ifdef __cplusplus
}
#endif

#endif /* DEEPSEEKER_B200_H */
