/* libmeep2b: B200 (sm_100a) kernels of the grouped MoE-LoRA expert layer, behind a plain C ABI.
 *
 * Every entry point takes device pointers, sizes and a CUDA stream (a cudaStream_t passed as void*), launches
 * asynchronously on that stream, allocates no device memory (buffers, including workspaces, come from the caller)
 * and returns a status: 0 on success, one of MEEP2B_ERR_* otherwise.  The Python host layer
 * (meepsquared_b200/_grouped.py, _moe.py, _fp8.py, _nf4.py) maps those statuses onto the reference's exceptions.
 *
 * Element types: "bf16" buffers hold IEEE bfloat16, "e4m3" buffers OCP FP8 E4M3 codes, one byte each.
 * Citations are file:line within thinkube/meepsquared (src/meepsquared/...).
 */
#ifndef MEEP2B_H
#define MEEP2B_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum meep2b_status {
  MEEP2B_OK = 0,
  MEEP2B_ERR_SHAPE = 1,       /* sizes that do not fit together: ValueError in the host layer */
  MEEP2B_ERR_DTYPE = 2,       /* an element type the entry point does not take: TypeError */
  MEEP2B_ERR_LAUNCH = 3,      /* a CUDA runtime or driver call failed: RuntimeError */
  MEEP2B_ERR_TIMEOUT = 4,     /* a bounded device-side wait ran out (see meep2b_device_error): RuntimeError */
  MEEP2B_ERR_UNSUPPORTED = 5, /* a combination the kernels do not implement: NotImplementedError */
  MEEP2B_ERR_ALIGN = 6,       /* a pointer or row stride that TMA cannot address (16-byte rule): ValueError */
  MEEP2B_ERR_DEVICE = 7       /* no compute capability 10.0 GPU: RuntimeError */
};

/* F32, BF16: plain types. Weight formats of meep2b_product.weight_dtype: BF16; E4M3 (codes converted exactly,
 * the per-expert `scale` applied in the epilogue); NF4 (packed codes with their block absmax); E4M3_BLOCKS (codes
 * with a grid of block scales). The last two take per-group multipliers (meep2b_quant_multipliers) in `wscale`. */
enum meep2b_dtype { MEEP2B_F32 = 0, MEEP2B_BF16 = 1, MEEP2B_E4M3 = 2, MEEP2B_NF4 = 3, MEEP2B_E4M3_BLOCKS = 4 };

enum meep2b_epilogue {
  MEEP2B_EPI_PLAIN = 0,   /* out = scale_e * (x W^T) + s (x A^T) B^T + bias_e                                   */
  MEEP2B_EPI_SWIGLU = 1,  /* gate_up forward: aux = pre-activation (rows, n), out = silu(gate) * up (rows, n/2)  */
  MEEP2B_EPI_DSWIGLU = 2  /* down backward: the product is dh (rows, n); aux = pre-activation (rows, 2n) read;
                             out = d(gate, up) (rows, 2n)                                                      */
};

/* ---------------------------------------------------------------------------------------------- library */

/* Version string of the library. */
const char* meep2b_version(void);
/* Message for a status code. */
const char* meep2b_status_string(int status);
/* MEEP2B_OK when `device` is a compute capability 10.0 GPU the kernels run on; replaces _grouped.available()
 * (_grouped.py:259-261) and the capability test of _grouped.wanted() (_grouped.py:57-67). */
int meep2b_device_ok(int device);
/* Reads and clears the device's error word, where a kernel records a bounded wait that ran out. Synchronous. */
int meep2b_device_error(int device, int* code);
/* Number of streaming multiprocessors of the device (the persistent kernels' grid). */
int meep2b_sm_count(int device, int* count);

/* ---------------------------------------------------------------------------------------------- routing */

/* Workspace bytes meep2b_route needs for `assignments` = tokens * top_k routed rows over `experts`. */
size_t meep2b_route_workspace_bytes(int64_t assignments, int32_t experts);

/* The permutation of _moe._routed_forward (_moe.py:77-86): a stable counting sort of the flat expert ids.
 * perm[i] = flat index of the i-th assignment in expert order (ties keep their flat order; ids >= experts, and
 * negative ids, are sentinels and sort last), expert_ids_g[i] = min(id, experts - 1), offsets[e] = inclusive
 * cumulative row count of experts 0..e (int32, sentinels not counted), inverse[perm[i]] = i (_moe.py:124-125).
 * expert_ids_g and inverse may be NULL. At most INT32_MAX assignments (positions and offsets are int32). */
int meep2b_route(const int64_t* expert_ids, int64_t assignments, int32_t experts, int64_t* perm,
                 int64_t* expert_ids_g, int32_t* offsets, int64_t* inverse, void* workspace,
                 size_t workspace_bytes, void* stream);

/* meep2b_route for callers that cannot allocate device memory; it has no counterpart in the reference. Some
 * callers own every device buffer and have no allocator to lend this library (an FFI caller outside PyTorch, a
 * serving process that reserves its device memory up front), or must not call cudaMalloc because it would
 * synchronise the device or break a memory budget; they cannot supply meep2b_route's workspace. This entry point
 * keeps the bucket-count table in a fixed 256 KB array of device memory that the library declares and that every
 * GPU loading the library holds until the process exits; it calls no cudaMalloc, cudaFree or other allocating
 * routine. Limit: ceil(assignments / 4096) * (experts + 1) <= 65536 (for example 262,144 assignments over up to
 * 1023 experts, or 1,048,576 over up to 255); larger requests return MEEP2B_ERR_SHAPE before any work. The first
 * call on a device looks up the array's device address with cudaGetSymbolAddress (with that device current), so
 * make that first call before any stream capture; later calls outside a capture look it up again (it can move
 * after cudaDeviceReset), calls on a capturing stream reuse the last lookup. All calls share the one array: calls
 * that overlap on the GPU (two streams, or two host threads on one device) race and must be serialised by the
 * caller. Outputs and arguments as meep2b_route; every table entry a call reads is written earlier in the same
 * call, so nothing from a previous call carries over. */
int meep2b_route_noalloc(const int64_t* expert_ids, int64_t assignments, int32_t experts, int64_t* perm,
                         int64_t* expert_ids_g, int32_t* offsets, int64_t* inverse, void* stream);

/* The router that feeds the routing (Transformers' Qwen3MoeTopKRouter.forward, after its linear layer): for each
 * token t, probs[t, :] = softmax(logits[t, :]) in float32 (logits (tokens, experts) F32 or BF16; probs may be
 * NULL), the top_k largest in descending order (a tie goes to the smaller expert index) as top_k_index[t, :]
 * (int64) and their probabilities, divided by their sum when norm_topk_prob, as top_k_weights[t, :] (float32);
 * then the routing permutation of meep2b_route over those ids, the router's pass doing the sort's histogram.
 * top_k <= 32 and <= experts; workspace as for meep2b_route. The reference takes the router's outputs as inputs
 * of the routed layer (_moe.py:70-87); this fuses the two steps. */
int meep2b_route_logits(const void* logits, int32_t logits_dtype, int64_t tokens, int32_t experts, int32_t top_k,
                        int32_t norm_topk_prob, float* probs, int64_t* top_k_index, float* top_k_weights,
                        int64_t* perm, int64_t* expert_ids_g, int32_t* offsets, int64_t* inverse, void* workspace,
                        size_t workspace_bytes, void* stream);

/* What the routed products need of the permutation without a gathered copy of the rows: per routed row i, the
 * token it reads, token_rows[i] = perm[i] / top_k (int32), and its routing weight weights_g[i] = weights[perm[i]]
 * as float32 (weights F32 or BF16; weights or weights_g may be NULL). */
int meep2b_routed_rows(const int64_t* perm, int64_t assignments, int32_t top_k, const void* weights,
                       int32_t weights_dtype, int32_t* token_rows, float* weights_g, void* stream);

/* The gather of _moe.py:80-81,87: selected[i] = hidden[perm[i] / top_k] (bf16 rows of hidden_dim), zero for the
 * sentinel rows i >= offsets[experts-1]; weights_g[i] = weights[perm[i]] (weights_dtype F32 or BF16, same type
 * out; both may be NULL). */
int meep2b_gather(const void* hidden, int64_t tokens, int64_t hidden_dim, int32_t top_k, const int64_t* perm,
                  const int32_t* offsets, int32_t experts, const void* weights, int32_t weights_dtype,
                  void* weights_g, void* selected, void* stream);

/* The weighted un-permute of _moe.py:123-126: out[t] = bf16(sum_j y[r] * w_g[r]), r = inverse[t*top_k + j],
 * the sum in float32 over j in order; rows r >= offsets[experts-1] (sentinels) count as zero. weights_g NULL
 * means weight 1 (the backward of the gather, _moe.py:80). */
int meep2b_unpermute(const void* y, const int64_t* inverse, const void* weights_g, int32_t weights_dtype,
                     const int32_t* offsets, int32_t experts, int64_t tokens, int32_t top_k, int64_t hidden_dim,
                     void* out, void* stream);

/* The same weighted un-permute over rows stored token-major (the down product's rows placed through the
 * permutation, meep2b_product.out_rows = perm): out[t] = bf16(sum_j y_tok[t*top_k + j] * w[t*top_k + j]), w the
 * routing weights in the router's (tokens, top_k) order (NULL: weight 1, the gather's backward), the sum in float32
 * over j in order, assignments whose inverse[t*top_k + j] >= offsets[experts-1] (sentinels, never stored) count as
 * zero. Reads each token's rows as one contiguous run: the forward combine of _moe.py:123-126. */
int meep2b_combine(const void* y_tok, const int64_t* inverse, const void* weights, int32_t weights_dtype,
                   const int32_t* offsets, int32_t experts, int64_t tokens, int32_t top_k, int64_t hidden_dim,
                   void* out, void* stream);

/* Backward of the un-permute (autograd of _moe.py:123-126): grad_y[i] = bf16(grad_out[perm[i]/top_k] * w_g[i]),
 * grad_weights[perm[i]] = sum_h grad_out[perm[i]/top_k][h] * y[i][h] (float32); sentinel rows give zeros. */
int meep2b_unpermute_backward(const void* grad_out, const void* y, const int64_t* perm, const void* weights_g,
                              int32_t weights_dtype, const int32_t* offsets, int32_t experts, int64_t assignments,
                              int32_t top_k, int64_t hidden_dim, void* grad_y, float* grad_weights, void* stream);

/* The routing weights' gradient when the un-permute's backward is folded into the down stack's input-gradient
 * product (meep2b_product.w_grad, per routed row and 96-column block <dh, h> = <g, y>): grad_weights[perm[i]] =
 * sum_{b < blocks} parts[i * ld + b], summed in order of b in float32, for the experts' rows i < offsets[experts-1],
 * and 0 for the sentinel rows. The weights' part of the backward of _moe.py:123-126 (weighted = out * w_g). */
int meep2b_weight_grad(const float* parts, int64_t ld, int32_t blocks, const int64_t* perm, int64_t assignments,
                       const int32_t* offsets, int32_t experts, float* grad_weights, void* stream);

/* ---------------------------------------------------------------------------------------------- tile map */

/* _grouped.tile_map (_grouped.py:88-103) on the device: tile_expert / tile_row get max_tiles(rows, experts,
 * block_m) = rows / block_m + experts entries (spares hold the last expert), *tiles the real count. */
int meep2b_tile_map(const int32_t* offsets, int32_t experts, int64_t rows, int32_t block_m, int32_t* tile_expert,
                    int32_t* tile_row, int32_t* tiles, void* stream);

/* ---------------------------------------------------------------------------------------------- grouped product */

/* One launch of the grouped product, the replacement of _grouped._launch (_grouped.py:313-345) and of
 * _grouped_gemm_kernel (_grouped.py:121-221): for each tile of 128 rows of one expert e, over the expert's rows
 *   acc  = x W_e^T           (tcgen05 MMA, float32 accumulator in tensor memory)
 *   low  = x P_e^T           (the rank-16 panel, in the same MMA: the panel rows ride along W's rows)
 *   acc += (s low / scale_e) U_e^T   (MMAs of depth 16; the panel as two bf16 planes, hi + lo)
 *   out  = epilogue(scale_e acc + bias_e)
 * Layouts (b_mn == 0, "K-major"): weight (experts, n, k), panel (experts, 16, k), up (experts, n, 16).
 *         (b_mn == 1, "MN-major"): weight (experts, k, n), panel (experts, k, 16),
 *                                  up (experts, 16, n).
 * The rank is padded to 16 with zeros (_grouped.py:275-282). x is (rows, k) with row stride ldx; rows of one
 * expert are contiguous, offsets[e] is the end of expert e's rows (int32, inclusive cumsum). tile_expert /
 * tile_row / tiles come from meep2b_tile_map with the product's block_m: 128 (one CTA per tile) or 256 (a CTA
 * pair per tile, tcgen05 cta_group::2, for b_mn == 0 only; each SM then stages half of the stack tile).
 * low (rows, 16) receives bf16(x P_e^T) when not NULL (kept for the backward pass, _grouped.py:212-214).
 * Quantised stacks (weight_dtype NF4, E4M3, E4M3_BLOCKS; block_m 128; k and n multiples of 64) are dequantised in
 * shared memory between the TMA load and the MMA, exactly as the reference dequantises them (_grouped.py:200-201
 * for E4M3; axolotl quantize.py:85-96 for NF4 and :131-157 for the block scales). weight then holds the codes of
 * the stored (experts, rows, cols) stack, cols contiguous (NF4: two codes a byte, the first in the high nibble);
 * wscale (NF4, E4M3_BLOCKS): the multiplier of each group of 64 consecutive weights, (experts, cols/64, rows)
 * float32, as meep2b_quant_multipliers prepares it once per frozen stack. */
typedef struct meep2b_product {
  const void* x;
  int64_t rows, k, ldx;
  const void* weight;
  int32_t weight_dtype; /* MEEP2B_BF16, MEEP2B_E4M3, MEEP2B_NF4 or MEEP2B_E4M3_BLOCKS */
  int32_t experts;
  int64_t n;
  int32_t b_mn;
  const float* scale;   /* (experts,) per-expert scale of the stack, or NULL */
  const void* panel;    /* NULL: no adapters */
  const void* up;
  float scaling;        /* s = alpha / r */
  const void* bias;     /* (experts, n) bf16 or NULL */
  const int32_t* offsets;
  const int32_t* tile_expert;
  const int32_t* tile_row;
  const int32_t* tiles;
  int64_t max_tiles;
  void* out;
  int64_t ldo;
  void* low;            /* (rows, 16) bf16 or NULL */
  int32_t epilogue;     /* enum meep2b_epilogue */
  void* aux;            /* SWIGLU: pre-activation out (rows, n); DSWIGLU: pre-activation in (rows, 2n) */
  int32_t sm_limit;     /* 0: one CTA per SM */
  int32_t block_m;      /* rows per tile: 128, or 256 for the CTA-pair kernel (bf16 stacks); 0 means 128 */
  const float* wscale;  /* NF4, E4M3_BLOCKS: per-group multipliers (experts, cols/64, rows); else NULL */
  /* The routed layer's fusions (bf16 stacks). x_rows: NULL, or row i of the product's input is row x_rows[i] of the
   * ldx-strided x, which has x_src_rows rows (the routed rows read from the token-major tensor: no gathered copy;
   * SWIGLU with b_mn == 0, and DSWIGLU with b_mn == 1). row_scale: NULL, or product row i is scaled by
   * row_scale[i] (the routing weight: the un-permute's backward folded into the down stack's input gradient), and
   * so is its stored panel. w_grad (DSWIGLU): NULL, or w_grad[i * w_ld + b] = sum over the columns j of block b of
   * 96 columns of dh[i, j] * h[i, j], the row's unscaled product dh and h = bf16(bf16(silu(gate)) * up), for rows i
   * of the experts' ranges (b < ceil(n / 96)): summed over b, the routing weight's gradient <g, y> (the caller sums
   * in a fixed order, so the result does not depend on the schedule). */
  const int32_t* x_rows;
  int64_t x_src_rows;
  const float* row_scale;
  float* w_grad;
  int64_t w_ld;
  /* out_rows (PLAIN epilogue, bf16 stacks): NULL, or product row i is stored at row out_rows[i] of out, e.g. the
   * routing permutation `perm` (the flat assignment token * top_k + j of each row), so that the rows land in
   * token-major order (tokens, top_k, n) and the un-permute becomes a streaming sum over each token's top_k
   * consecutive rows (meep2b_combine). The stored panel `low` stays at row i. */
  const int64_t* out_rows;
} meep2b_product;

int meep2b_grouped_product(const meep2b_product* p, void* stream);

/* ---------------------------------------------------------------------------------------------- FP8 products */

/* The activations of an FP8 product, quantised as the reference's X_FP8 path quantises each x tile
 * (_grouped.py:194-197), with tiles of 128 columns: for row r and block b of columns 128b..128b+127,
 * scales[b * ld_scales + r] = max(max |x[r, j]|, 1e-12) / 448 (float32) and codes[r * k + j] = e4m3(x[r, j] / that
 * scale), rounded to nearest even. x (rows, k) bf16 with row stride ldx (a multiple of 8); k a multiple of 16. */
int meep2b_fp8_rows_quantize(const void* x, int64_t rows, int64_t k, int64_t ldx, uint8_t* codes, float* scales,
                             int64_t ld_scales, void* stream);

/* One launch of the FP8 product, the reference's _grouped_gemm_kernel with W_FP8 and X_FP8 (_grouped.py:141-146,
 * 194-197, 202-219; selected by fp8_products, :70-80): for each tile of 128 rows of one expert e and 128 columns,
 *   acc  = sum over k-blocks b of (x8_b W8_{e,b}^T) * xscale[b, row] (* the stack's block scale)
 *          (tcgen05 kind::f8f6f4: e4m3 codes, float32 partial sums, one per 128-column k-block, promoted in registers)
 *   acc  = acc * scale_e + scaling * (low U_e^T) + bias_e,   out = bf16(acc)
 * x8 / xscale come from meep2b_fp8_rows_quantize (codes (rows, k), row stride k; scales (ceil(k/128), ld_xscale)).
 * weight: e4m3 codes, (experts, n, k) when b_mn == 0, (experts, k, n) when b_mn == 1. scale (experts,) or NULL.
 * wblock: NULL, or the stack's block scales: the partial sum of k-block b and column block c = col / 128 of expert e
 * is multiplied by wblock[e * wb_stride_e + (b / wb_div_k) * wb_stride_k + (c / wb_div_n) * wb_stride_n].
 * low (rows, 16) bf16: bf16(x A_e^T), the adapters' panel of the bf16 x (the reference multiplies the adapters with
 * the bf16 x tile, :141-146,203-213), or NULL without adapters; up (experts, n, 16) bf16, the rank padded with
 * zeros. offsets / tile_expert / tile_row / tiles / max_tiles as meep2b_product (block_m 128). k and n multiples
 * of 16; out (rows, n) bf16 with row stride ldo (a multiple of 8). */
typedef struct meep2b_product_f8 {
  const uint8_t* x8;
  int64_t rows, k;
  const float* xscale;
  int64_t ld_xscale;
  const uint8_t* weight;
  int32_t experts;
  int64_t n;
  int32_t b_mn;
  const float* scale;
  const float* wblock;
  int64_t wb_stride_e, wb_stride_k, wb_stride_n;
  int32_t wb_div_k, wb_div_n;
  const void* low;
  const void* up;
  float scaling;
  const void* bias;
  const int32_t* offsets;
  const int32_t* tile_expert;
  const int32_t* tile_row;
  const int32_t* tiles;
  int64_t max_tiles;
  void* out;
  int64_t ldo;
  int32_t sm_limit; /* 0: one CTA per SM */
} meep2b_product_f8;

int meep2b_grouped_product_f8(const meep2b_product_f8* p, void* stream);

/* ---------------------------------------------------------------------------------------------- SwiGLU gate */

/* Transformers' _default_apply_gate, which the reference's routed forward calls as experts._apply_gate
 * (_moe.py:119), for the layer's unfused form: h[r, j] = bf16(bf16(silu(g)) * u) with g = gate_up[r, j] and
 * u = gate_up[r, inter + j]; gate_up (rows, 2 inter) and h (rows, inter) bf16, contiguous; inter a multiple of 8.
 * The arithmetic of the fused products' SwiGLU epilogue. */
int meep2b_swiglu(const void* gate_up, int64_t rows, int64_t inter, void* h, void* stream);

/* Its backward: grad_gate_up[r, j] = bf16(dh u) sig(g) (1 + g (1 - sig(g))), grad_gate_up[r, inter + j] =
 * dh bf16(silu(g)) (dh = grad_h[r, j]), as the fused dSwiGLU epilogue. */
int meep2b_swiglu_backward(const void* gate_up, const void* grad_h, int64_t rows, int64_t inter, void* grad_gate_up,
                           void* stream);

/* _grouped._reduce / _grouped_reduce_kernel (_grouped.py:233-256,362-370): the adapters' gradients,
 * out[e, j, r] = bf16(scaling * sum over expert e's rows of g[row, j] * low[row, r]) for r < 16; g (rows, n) bf16
 * with row stride ldg, low (rows, 16) bf16, out (experts, n, 16) bf16 (out_layout 0) or (experts, 16, n) (out_layout
 * 1: a factor stored rank-major, as PEFT's lora_A is, takes its gradient in its own layout). */
int meep2b_grouped_reduce(const void* g, int64_t rows, int64_t n, int64_t ldg, const void* low,
                          const int32_t* offsets, int32_t experts, float scaling, void* out, int32_t out_layout,
                          void* stream);

/* The same reduction over rows gathered from a token-major tensor and weighted: out[e, j, r] = bf16(scaling * sum
 * over expert e's rows i of g[g_rows[i], j] * bf16(row_scale[i] * low[i, r])) (row_scale NULL: weight 1). Used
 * for the adapters of the gate/up stack (g = hidden, g_rows = the token of each routed row: no sorted copy) and of
 * the down stack (g = the layer's upstream gradient, row_scale = the routing weights: the un-permute's backward,
 * _moe.py:123-126, folded in). rows: the routed rows; g has ldg-strided rows indexed by g_rows. */
int meep2b_grouped_reduce_rows(const void* g, const int32_t* g_rows, const float* row_scale, int64_t rows,
                               int64_t n, int64_t ldg, const void* low, const int32_t* offsets, int32_t experts,
                               float scaling, void* out, int32_t out_layout, void* stream);

/* The gathered reduction of meep2b_grouped_reduce_rows (same result up to the order of float32 additions; bitwise
 * deterministic from call to call) for n = 768, 1536 or 2048 (MEEP2B_ERR_UNSUPPORTED otherwise): each CTA reads
 * whole rows, one bulk copy per row, over a chunk of up to meep2b_reduce_chunk_rows() rows of one expert, and
 * writes the chunk's float32 sums to `partial`; a second kernel adds each expert's chunks in order. The chunk map
 * (chunk_expert, chunk_row, chunks: device int32, max_chunks entries) is meep2b_tile_map's output for a tile height
 * of meep2b_reduce_chunk_rows(). partial: device float32 scratch of max_chunks x n x 16 entries (partial_bytes its
 * size; MEEP2B_ERR_SHAPE when smaller). */
int meep2b_grouped_reduce_rows_full(const void* g, const int32_t* g_rows, const float* row_scale, int64_t rows,
                                    int64_t n, int64_t ldg, const void* low, const int32_t* offsets, int32_t experts,
                                    float scaling, void* out, int32_t out_layout, const int32_t* chunk_expert,
                                    const int32_t* chunk_row, const int32_t* chunks, int64_t max_chunks,
                                    float* partial, size_t partial_bytes, void* stream);

/* Rows per chunk of meep2b_grouped_reduce_rows_full (the tile height of its chunk map). */
int meep2b_reduce_chunk_rows(void);

/* ---------------------------------------------------------------------------------------------- quantised stacks */

/* _fp8.quantize_stack (_fp8.py:122-128): scale[e] = max(amax_e, 1e-12) / 448, codes = e4m3(w / scale[e]) (round
 * to nearest even). w (experts, per_expert) in bf16 or f32. workspace: experts floats. */
int meep2b_fp8_stack_quantize(const void* w, int32_t dtype, int32_t experts, int64_t per_expert, uint8_t* codes,
                              float* scale, float* workspace, void* stream);
/* _fp8.dequantize_stack (_fp8.py:131-134, _grouped_scale_kernel :69-79): out = bf16(f32(codes) * scale[e]). */
int meep2b_fp8_stack_dequantize(const uint8_t* codes, const float* scale, int32_t experts, int64_t per_expert,
                                void* out, void* stream);
/* axolotl quantize.dequantize_fp8 (_vendor/axolotl/quantize.py:131-157), bf16 out, for `matrices` stacked
 * (rows, cols) matrices each with an (sr, sc) float32 scale grid: out = bf16(bf16(w) * bf16(scale)), blocks of
 * ceil(rows/sr) x ceil(cols/sc). */
int meep2b_fp8_block_dequantize(const uint8_t* codes, int64_t matrices, int64_t rows, int64_t cols,
                                const float* scale_inv, int32_t sr, int32_t sc, void* out, void* stream);
/* axolotl quantize.quantize_fp8 (quantize.py:238-263) with a 2-D scale grid, per stacked matrix:
 * scale = max(amax_block, 1e-12) / 448, codes = e4m3(clamp(w / scale, +-448)); w bf16 or f32. */
int meep2b_fp8_block_quantize(const void* w, int32_t dtype, int64_t matrices, int64_t rows, int64_t cols,
                              int32_t sr, int32_t sc, uint8_t* codes, float* scale_inv, void* stream);
/* The first stage of the NF4 dequantisation (axolotl quantize.py:74-83, bitsandbytes'
 * cdequantize_blockwise_fp32 then `+= offset`): absmax_out[i] = code2[absmax[i]] * absmax2[i / blocksize2] +
 * offset[0], two float32 roundings; count = number of 64-weight blocks. Its output is the `wscale` of an NF4
 * product (computed once per frozen stack). */
int meep2b_nf4_absmax(const uint8_t* absmax, const float* absmax2, const float* code2, const float* offset,
                      int32_t blocksize2, int64_t count, float* absmax_out, void* stream);
/* The multipliers of a quantised stack for meep2b_grouped_product, out (experts, cols/64, rows) float32, one per
 * group of 64 consecutive weights of each stored (rows, cols) matrix (cols a multiple of 64):
 *   MEEP2B_NF4:         src = the float32 absmax per 64-weight block in storage order (meep2b_nf4_absmax's output):
 *                       out[e][g][r] = src[(e * rows + r) * (cols / 64) + g];
 *   MEEP2B_E4M3_BLOCKS: src = the (experts, sr, sc) scales of dequantize_fp8 (quantize.py:131-157):
 *                       out[e][g][r] = bf16(src[e][r / br][64 g / bc]), br = ceil(rows/sr), bc = ceil(cols/sc)
 *                       (bc a multiple of 64: one scale per group). */
int meep2b_quant_multipliers(int32_t weight_dtype, const float* src, int32_t experts, int64_t rows, int64_t cols,
                             int32_t sr, int32_t sc, float* out, void* stream);
/* The NF4 double dequantisation of axolotl quantize._ctypes_nf4_dequant (quantize.py:52-101), which calls
 * bitsandbytes' cdequantize_blockwise_fp32 then `+= offset` then cdequantize_blockwise_bf16_nf4:
 * absmax_out[i] = code2[absmax[i]] * absmax2[i / blocksize2] + offset[0] (two float32 roundings);
 * out[j] = bf16(NF4[code_j] * absmax_out[j / blocksize]), two codes per byte, the first in the high nibble.
 * n = number of weights (even); absmax_out: n / blocksize floats (caller-provided workspace). */
int meep2b_nf4_dequantize(const uint8_t* packed, const uint8_t* absmax, const float* absmax2, const float* code2,
                          const float* offset, int32_t blocksize, int32_t blocksize2, int64_t n, float* absmax_out,
                          void* out, void* stream);

/* ------------------------------------------------------------------------------------------------ merged save */

/* _save._merged_stack (_save.py:79-95): out[e] = dtype(W_e + scaling * (lhs_e @ rhs_e)) for every expert, float32
 * arithmetic, the stack's own layout: W (experts, rows, cols) in f32, bf16 or e4m3 (then dequantised as
 * _fp8.dequantize_stack does for float32, f32(code) * scale[e]); lhs (experts, rows, rank) and rhs
 * (experts, rank, cols) float32, contiguous (rank <= 128), the factors of _moe._delta_factors (_moe.py:150-163),
 * or rank 0 and null factors for the stack alone (out = dtype(W_e)); out in f32 or bf16 (round to nearest even).
 * The rank products are summed in order, with fused multiply-adds. */
int meep2b_merge_stack(const void* weight, int32_t weight_dtype, const float* scale, const float* lhs,
                       const float* rhs, int32_t rank, float scaling, int64_t experts, int64_t rows, int64_t cols,
                       void* out, int32_t out_dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MEEP2B_H */
