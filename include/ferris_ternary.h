/*
 * ferris_ternary.h -- C ABI of libferris_ternary.so, the B200 (sm_100a) ternary
 * matmul hot path of FerrisRes.
 *
 * Conventions
 *   - Every entry point returns an int status (ft_status).  On failure the
 *     per-thread message is available from ft_last_error_string().  Nothing
 *     throws or aborts across this boundary.
 *   - Shapes follow the reference: a weight is [rows = out_features,
 *     cols = in_features] row-major ("row" = output channel); activations
 *     are [seq, cols]; outputs are [seq, rows].
 *   - Pointers documented as "device" are CUDA device pointers; "host" are
 *     ordinary host memory.  Device-pointer calls are asynchronous on the
 *     caller's stream (a cudaStream_t passed as void*, NULL = legacy default
 *     stream) and never synchronise.  Host-buffer calls are synchronous.
 *   - Reference interfaces replaced are cited as path:line within
 *     shift/FerrisRes v0.2.3.
 *
 * Status codes map onto FerrisResError (src/error.rs:3-36):
 *   1 Shape, 2 Gpu, 3 OOM, 4 Unsupported, 5 Timeout/Comm, 6 Device.
 */
#ifndef FERRIS_TERNARY_H
#define FERRIS_TERNARY_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

typedef enum ft_status {
  FT_OK = 0,
  FT_ERR_SHAPE = 1,       /* FerrisResError::Shape */
  FT_ERR_GPU = 2,         /* FerrisResError::Gpu */
  FT_ERR_OOM = 3,         /* FerrisResError::OOM */
  FT_ERR_UNSUPPORTED = 4, /* FerrisResError::Unsupported */
  FT_ERR_TIMEOUT = 5,     /* collective / wait timed out */
  FT_ERR_DEVICE = 6       /* FerrisResError::Device (bad device, no GPU) */
} ft_status;

typedef struct ft_ctx ft_ctx;       /* one CUDA device + workspace */
typedef struct ft_weight ft_weight; /* one dense ternary matrix resident in HBM */
typedef struct ft_moe ft_moe;       /* one ternary MoE FFN layer resident in HBM */
typedef struct ft_kv3 ft_kv3;       /* one layer's 3-bit KV cache resident in HBM */
typedef struct ft_kvp ft_kvp;       /* page pool of the paged 3-bit KV cache */

/* ---- library / context ------------------------------------------------ */
const char* ft_version(void);
const char* ft_last_error_string(void);
/* Number of CUDA kernels this library has launched in this process (a
 * diagnostic; launches replayed from a captured CUDA graph are not counted
 * again).  No reference counterpart. */
uint64_t ft_launch_counter(void);
/* Replaces TernaryMatMulOp::new(&Arc<Device>, &Arc<Queue>)
 * (src/compute/kernels/ternary_matmul.rs:84); the kernels are compiled ahead
 * of time, so creation only binds a device. */
int ft_ctx_create(int device, ft_ctx** out);
int ft_ctx_destroy(ft_ctx* ctx);
/* Synchronises the device and reports whether any kernel launched through
 * this context gave up a bounded internal wait (FT_ERR_TIMEOUT; the flag is
 * then cleared).  Kernels never spin unboundedly: a wait that exceeds 2 s
 * records its site here and the launch finishes with invalid results.
 * Note: a context's scratch is shared by its calls, so calls through one
 * context must be ordered (same stream, or synchronised). */
int ft_ctx_check(ft_ctx* ctx);

/* ---- dense weights ----------------------------------------------------- */
/* Upload from the reference host layout produced by pack_ternary
 * (src/model/ternary.rs:136-163): (rows*cols+3)/4 bytes, 4 codes per byte,
 * LSB first, code -1->0b00, 0->0b01, +1->0b10, 0b11->0.  row_scales: [rows]
 * host floats (the per-output-channel scale; pass the broadcast scalar for
 * the reference's single-alpha types, src/model/cpu_moe.rs:73-78).  The
 * matrix is repacked on the device into the tiled layout the kernels read. */
int ft_weight_upload_packed_u8(ft_ctx* ctx, const uint8_t* packed_host, int64_t rows,
                               int64_t cols, const float* row_scales_host, ft_weight** out);
/* Upload from the GPU layout of pack_ternary_u32 / the WGSL op
 * (src/model/ternary.rs:1317-1328, src/compute/kernels/ternary_matmul.rs:7-8):
 * rows * ceil(cols/16) u32 words, 16 codes per word, LSB first.  Replaces
 * GpuVramCache::upload (src/model/cpu_block_attn_res.rs:3072). */
int ft_weight_upload_packed_u32(ft_ctx* ctx, const uint32_t* words_host, int64_t rows,
                                int64_t cols, const float* row_scales_host, ft_weight** out);
/* Same layout already in device memory (e.g. a buffer the caller owns). */
int ft_weight_from_device_u32(ft_ctx* ctx, const uint32_t* words_dev, int64_t rows, int64_t cols,
                              const float* row_scales_dev, void* stream, ft_weight** out);
/* 2:4 sparse weights (every group of 4 codes along K holds exactly two +-1).
 * From the reference host type SparseTernaryMatrix (src/model/sparse_ternary.rs:52-70):
 * patterns = ceil(groups/2) bytes (3-bit pattern, even group in the low nibble),
 * signs = ceil(groups/4) bytes (2 bits per group, 1 = +1); groups = rows*cols/4,
 * cols % 4 == 0.  Stored on the device at 1.5 bits per weight, in the operand
 * form of the sparse tensor-core MMA (per group a 4-bit position nibble = the
 * 2:4 metadata, and one sign bit per nonzero), and usable with every
 * ft_ternary_matmul_* entry point. */
int ft_sparse_upload_host(ft_ctx* ctx, const uint8_t* patterns_host, const uint8_t* signs_host,
                          int64_t rows, int64_t cols, const float* row_scales_host,
                          ft_weight** out);
/* From the WGSL SparseTernaryMatMulOp layout (src/compute/kernels/sparse_ternary.rs:71-100):
 * rows * ceil(ceil(cols/4)/6) u32 words, 6 groups of 5 bits (3 pattern + 2 sign,
 * 1 = -1) per word. */
int ft_sparse_upload_wgsl(ft_ctx* ctx, const uint32_t* words_host, int64_t rows, int64_t cols,
                          const float* row_scales_host, ft_weight** out);
/* The codes of a resident weight (dense or 2:4) back as the reference pack_ternary
 * byte stream (src/model/ternary.rs:141-163): (rows*cols+3)/4 host bytes, padding
 * bits 0.  Synchronous.  For saving weights (the reference's TernaryExpert::to_fp32
 * path, src/model/cpu_moe.rs:64-66) and for checking device-side quantization. */
int ft_weight_export_packed_u8(ft_ctx* ctx, const ft_weight* w, uint8_t* packed_host);
int ft_weight_destroy(ft_weight* w);
int ft_weight_info(const ft_weight* w, int64_t* rows, int64_t* cols, int64_t* device_bytes);

/* Index-list form (ternary_sparse_indices, src/model/ternary.rs:681-707, used by
 * ternary_matmul_sparse_decode, :647-672): per row the columns holding +1 and
 * -1, as CSR host arrays (pos_off/neg_off [rows + 1], starting at 0; each
 * row's columns strictly increasing and the two lists disjoint, as
 * ternary_sparse_indices produces them; otherwise FT_ERR_SHAPE).  Stored as a
 * dense 2-bit weight (2 bits per weight beats a 32-bit index below ~94%
 * sparsity); ternary_matmul_sparse_decode is then ft_ternary_matmul_f32 with
 * seq 1 and the scale broadcast into row_scales_host. */
int ft_weight_upload_index_lists(ft_ctx* ctx, int64_t rows, int64_t cols, const int64_t* pos_off,
                                 const int64_t* pos_idx, const int64_t* neg_off,
                                 const int64_t* neg_idx, const float* row_scales_host,
                                 ft_weight** out);
/* fp32 weights quantized on the device: TernaryExpert::from_fp32
 * (src/model/cpu_moe.rs:33-37) = quantize_ternary (src/model/ternary.rs:31-57):
 * alpha = (sequential fp32 sum |w| / n) / 0.7978845608 (1 when not positive),
 * q = clamp(round_half_away(w * (1 / alpha)), -1, 1), NaN -> 0; every row
 * scale = alpha (returned in alpha_out when non-null).  w_host [rows, cols]. */
int ft_weight_quantize_f32(ft_ctx* ctx, const float* w_host, int64_t rows, int64_t cols,
                           float* alpha_out, ft_weight** out);
/* STE re-quantization in place (BitMoELayer::requantize_all, shared alpha,
 * src/training/bit_moe.rs:243-262): from a [rows, cols] fp32 (or bf16 bit
 * patterns when src_bf16) device matrix, n = v / alpha, q = +1 if n > 0.5, -1
 * if n < -0.5, else 0 (all 0 when alpha < 1e-10); every row scale = alpha.
 * Asynchronous on stream; the weight must not be in use by earlier work on
 * other streams. */
int ft_weight_requantize(ft_ctx* ctx, ft_weight* w, const void* src_dev, int src_bf16, float alpha,
                         void* stream);
/* The layer-shared alpha of BitMoELayer::recompute_alpha (src/training/bit_moe.rs:210-241):
 * mean |v| over n device buffers (counts[i] elements each, fp32 or bf16), summed in f64,
 * then (float)(sum / count).  A parallel f64 sum: it equals the reference's sequential one
 * whenever the f64 partial sums are exact (bf16 magnitudes within about 2^(44 - log2 n) of
 * each other).  Synchronous.  Leaves *alpha_out unchanged when the buffers hold no element,
 * as the reference keeps its previous alpha. */
int ft_shadow_alpha(ft_ctx* ctx, int n, const void* const* src_dev, const int64_t* counts,
                    int src_bf16, float* alpha_out);

/* ---- dense compute (device pointers, caller stream) -------------------- */
/* y[s, r] = row_scale[r] * sum_k W[r, k] * x[s, k], fp32 activations.
 * Replaces TernaryMatMulOp::dispatch (src/compute/kernels/ternary_matmul.rs:167-225)
 * for weights held as ft_weight.  Any seq >= 1 (decode GEMV and prefill GEMM).
 * Precision: the activations enter as 64-bit fixed point per token (exact for
 * every element within 2^38 of the token's largest finite |x|) and the sums are
 * exact integers, so each output is the correctly rounded value of the exact
 * sum times the row scale.  Non-finite activations follow the reference shader
 * (src/compute/kernels/ternary_matmul.rs:54-70): x[k] enters a row only where
 * its weight is nonzero, so a row meeting NaN or infinities of both signs is
 * NaN, one sign of infinity gives that infinity times the row scale. */
int ft_ternary_matmul_f32(ft_ctx* ctx, const ft_weight* w, int64_t seq, const float* x_dev,
                          float* y_dev, void* stream);
/* Same with bf16 activations (bit patterns as uint16). */
int ft_ternary_matmul_bf16(ft_ctx* ctx, const ft_weight* w, int64_t seq, const uint16_t* x_dev,
                           float* y_dev, void* stream);
/* Grouped form: n (1..64) independent matmuls with the same seq in one
 * persistent launch -- e.g. the q/k/v projections of a decode step, or the
 * gate and up projections of the experts a token selected (the reference runs
 * these as separate dispatches: src/model/cpu_block_attn_res.rs:2254-2316).
 * ws[i] : weight i; xs_dev[i] : [seq, ws[i].cols]; ys_dev[i] : [seq, ws[i].rows].
 * Entries that pass the same activation pointer share its preparation. */
int ft_ternary_matmul_f32_grouped(ft_ctx* ctx, int n, const ft_weight* const* ws, int64_t seq,
                                  const float* const* xs_dev, float* const* ys_dev, void* stream);
int ft_ternary_matmul_i8_grouped(ft_ctx* ctx, int n, const ft_weight* const* ws, int64_t seq,
                                 const int8_t* const* qs_dev, const float* const* sxs_dev,
                                 float* const* ys_dev, void* stream);
/* Allocation-free form of ft_ternary_matmul_f32 for decode-sized calls.  No
 * counterpart in the reference.  It is for callers that must not let a library
 * allocate device memory inside a call: a host that owns all device memory
 * itself (a serving engine with a fixed arena, or an FFI contract that forbids
 * hidden allocations on the hot path), or a real-time loop that cannot take
 * cudaMalloc's implicit device-wide synchronisation.  It calls no cudaMalloc or
 * cudaFree: its scratch is one ~2.6 MB array reserved in the library image on
 * every GPU that loads the library, held until the process exits.  Limits:
 * seq <= 4, w rows <= 16384, w cols <= 16384; larger shapes return
 * FT_ERR_UNSUPPORTED.  The context and weight are created beforehand as usual.
 * The first call on a device looks up the array's device address, so make
 * that first call before any stream capture.  All calls share the array (each
 * clears what must start at zero), so calls that overlap on the GPU -- other
 * streams, other host threads, other contexts on the same device -- race:
 * order them.  Its kernels record a bounded wait that gave up in an error word
 * inside the same array; the word keeps that report across later calls until
 * ft_ctx_check on a context that has used this entry point (on that device)
 * reads and clears it. */
int ft_ternary_matmul_f32_noalloc(ft_ctx* ctx, const ft_weight* w, int64_t seq, const float* x_dev,
                                  float* y_dev, void* stream);
/* ternary_matmul_blocked (src/model/ternary.rs:541-579): y[s, r] = row_scale[r] *
 * sum_b block_scales[b] * sum_{k in block b} W[r, k] x[s, k], block b = columns
 * [b * block_size, (b + 1) * block_size), block_scales_dev = ceil(cols / block_size)
 * device floats shared by every row (upload the weight with row scales 1 for the
 * reference's form).  The block scales are folded into the activations
 * (x' = scale * x) before the fixed-point image.  Non-finite inputs follow that
 * reference's products w * x: a zero weight meeting an infinity gives NaN too. */
int ft_ternary_matmul_blocked_f32(ft_ctx* ctx, const ft_weight* w, int64_t seq, const float* x_dev,
                                  const float* block_scales_dev, int64_t block_size, float* y_dev,
                                  void* stream);
/* Per-token absmax int8 quantizer: sx[s] = absmax/127 (1 when absmax == 0),
 * q = clamp(round_half_away(x * (127/absmax)), -127, 127).  No reference
 * counterpart (the reference has no int8 activation path); the formula is
 * pinned so the int8 matmul below is bit-exact against the reference's own
 * ternary_matmul run on the same int8 codes. */
int ft_quantize_absmax_i8_f32(ft_ctx* ctx, int64_t seq, int64_t cols, const float* x_dev,
                              int8_t* q_dev, float* sx_dev, void* stream);
int ft_quantize_absmax_i8_bf16(ft_ctx* ctx, int64_t seq, int64_t cols, const uint16_t* x_dev,
                               int8_t* q_dev, float* sx_dev, void* stream);
/* y[s, r] = ((float)acc[s, r] * sx[s]) * row_scale[r], acc = exact int32
 * sum_k W[r, k] * q[s, k].  Bit-exact against the reference ternary_matmul
 * (src/model/ternary.rs:292-328) fed the int8 codes as f32. */
int ft_ternary_matmul_i8(ft_ctx* ctx, const ft_weight* w, int64_t seq, const int8_t* q_dev,
                         const float* sx_dev, float* y_dev, void* stream);

/* Raw WGSL-op form: same arguments as TernaryMatMulOp::dispatch
 * (src/compute/kernels/ternary_matmul.rs:167-177): ternary = rows*ceil(in_cols/16)
 * u32 words in device memory, scales [out_rows], input [seq_len, in_cols],
 * output [seq_len, out_rows], all device pointers; sequential-in-K fp32 sum
 * then * scales[row], as the shader does. */
int ft_ternary_matmul_op_dispatch(ft_ctx* ctx, const uint32_t* ternary_dev,
                                  const float* scales_dev, const float* input_dev,
                                  float* output_dev, uint32_t seq_len, uint32_t in_cols,
                                  uint32_t out_rows, void* stream);

/* ---- host-buffer accelerator calls (synchronous) ----------------------- */
/* GpuMatmulAccelerator::gpu_ternary_matmul (src/model/gpu_forward.rs:1154-1237):
 * uploads weights, runs, reads back into output_host [seq_len*out_rows]. */
int ft_gpu_ternary_matmul(ft_ctx* ctx, const uint32_t* packed_weights_host,
                          const float* scales_host, const float* input_host, size_t seq_len,
                          size_t in_cols, size_t out_rows, float* output_host);
/* GpuMatmulAccelerator::gpu_sparse_ternary_matmul (src/model/gpu_forward.rs:1299-1327,
 * a stub returning zeros in the reference): WGSL-layout words, one global scale. */
int ft_gpu_sparse_ternary_matmul(ft_ctx* ctx, const uint32_t* sparse_words_host, float scale,
                                 const float* input_host, size_t seq_len, size_t in_cols,
                                 size_t out_rows, float* output_host);
/* GpuMatmulAccelerator::gpu_ternary_matmul_vram (src/model/gpu_forward.rs:1245-1297):
 * weights already resident (ft_weight); host activations [seq_len, in_cols] in,
 * host output [seq_len, out_rows] out.  in_cols / out_rows are the reference's
 * arguments: they must equal the weight's cols / rows (FT_ERR_SHAPE otherwise),
 * so a caller's slice lengths are checked at the boundary. */
int ft_gpu_ternary_matmul_vram(ft_ctx* ctx, const ft_weight* w, const float* input_host,
                               size_t seq_len, size_t in_cols, size_t out_rows,
                               float* output_host);

/* ---- MoE FFN layer: TernaryMoELayer (src/model/ternary_moe.rs:77-223) ------
 * router_host: [n_experts, hidden] fp32, row e = expert e (the layout
 * TernaryMoELayer::forward indexes, ternary_moe.rs:157).  Per expert e:
 * gate/up [inter, hidden] and down [hidden, inter] in the reference pack_ternary
 * byte layout with per-row scales.  top_k <= 8, n_experts <= 64, SwiGLU
 * (use_gelu = 0) or GeLU-tanh (use_gelu = 1).  For expert parallelism a rank
 * passes NULL gate/up/down pointers for the experts it does not hold; the
 * router is always complete. */
int ft_moe_create(ft_ctx* ctx, int64_t n_experts, int64_t hidden, int64_t inter, int top_k,
                  int use_gelu, const float* router_host, const uint8_t* const* gate_packed,
                  const float* const* gate_scales, const uint8_t* const* up_packed,
                  const float* const* up_scales, const uint8_t* const* down_packed,
                  const float* const* down_scales, ft_moe** out);
int ft_moe_destroy(ft_moe* m);
/* Whole layer on one GPU: y [T, hidden] fp32 from x [T, hidden] (fp32, or bf16
 * bit patterns when x_is_bf16).  probs_dev (optional, [T, n_experts]) receives
 * the router softmax.  Reads back the per-expert token counts once (a stream
 * synchronisation) to size the expert launches.  Replaces
 * TernaryMoELayer::forward (src/model/ternary_moe.rs:145). */
int ft_moe_forward(ft_ctx* ctx, ft_moe* m, int64_t T, const void* x_dev, int x_is_bf16,
                   float* y_dev, float* probs_dev, void* stream);
/* Same layer from fp32 expert matrices (the checkpoint's
 * layers.{i}.moe.expert.{e}.{gate,up,down}, src/model/checkpoint.rs:21-24, which
 * the reference re-quantizes at load, :387-400): each matrix is quantized on the
 * device as ft_weight_quantize_f32 does (its own absmean alpha as every row scale).
 * gate_f32/up_f32 [inter, hidden], down_f32 [hidden, inter], host; NULL gate for
 * experts held by another rank. */
int ft_moe_create_f32(ft_ctx* ctx, int64_t n_experts, int64_t hidden, int64_t inter, int top_k,
                      int use_gelu, const float* router_host, const float* const* gate_f32,
                      const float* const* up_f32, const float* const* down_f32, ft_moe** out);
/* Fused decode step for 1..8 tokens (tokens x top_k <= 16): the whole layer
 * (router, softmax top-k, gate/up, SwiGLU or GeLU, down, weighted combine) in
 * ONE cooperative kernel launch, with no host synchronisation (capturable in a
 * CUDA graph after a first call has sized the scratch).  Replaces the
 * reference's per-expert decode loop (src/model/cpu_block_attn_res.rs:2284-2316)
 * over TernaryMoELayer::forward (src/model/ternary_moe.rs:145-223).  y_dev
 * [T, hidden] fp32; topk_idx_dev / topk_w_dev [T, top_k] receive the routing;
 * probs_dev (optional) [T, n_experts].  Every expert must be on this device.
 * Router scores are fp32 dots in a different order than the reference's
 * sequential sum; expert activations use 4 fixed-point digits (the layer's
 * tolerance); non-finite activations are not propagated (use ft_moe_forward). */
int ft_moe_decode(ft_ctx* ctx, ft_moe* m, int64_t T, const void* x_dev, int x_is_bf16,
                  float* y_dev, int32_t* topk_idx_dev, float* topk_w_dev, float* probs_dev,
                  void* stream);
/* Same with host buffers (fp32), the reference's &[f32] -> Vec<f32> form. */
int ft_moe_forward_host(ft_ctx* ctx, ft_moe* m, const float* input_host, size_t seq,
                        float* output_host);
/* Stages, for expert-parallel hosts that exchange tokens between them:
 * route: top-k experts and gates per token ([T, top_k]) and per-expert counts
 * ([n_experts], zeroed first); probs_dev optional. */
int ft_moe_route(ft_ctx* ctx, ft_moe* m, int64_t T, const void* x_dev, int x_is_bf16,
                 int32_t* topk_idx_dev, float* topk_w_dev, float* probs_dev, int32_t* counts_dev,
                 void* stream);
/* Expert-major slots: offsets [n_experts + 1] (exclusive scan of counts), fill
 * [n_experts] scratch, slot_of [T*top_k] (slot of entry t*top_k + k), token_of
 * [T*top_k] (token of each slot). */
int ft_moe_dispatch_layout(ft_ctx* ctx, ft_moe* m, int64_t T, const int32_t* topk_idx_dev,
                           const int32_t* counts_dev, int32_t* offsets_dev, int32_t* fill_dev,
                           int32_t* slot_of_dev, int32_t* token_of_dev, void* stream);
/* out[r, :] = x[token_of[r], :] for r < n_rows (elem_bytes 2 or 4). */
int ft_moe_gather_rows(ft_ctx* ctx, const void* x_dev, int elem_bytes, int64_t H,
                       const int32_t* token_of_dev, int64_t n_rows, void* out_dev, void* stream);
/* Expert FFN (gate/up, activation, down) over rows stored in segments: segment
 * i holds seg_rows[i] consecutive rows for expert seg_expert[i] (host arrays,
 * at most 64 segments).  y_rows [sum rows, hidden] fp32. */
int ft_moe_expert_ffn(ft_ctx* ctx, ft_moe* m, int nseg, const int32_t* seg_expert_host,
                      const int64_t* seg_rows_host, const void* x_rows_dev, int x_is_bf16,
                      float* y_rows_dev, void* stream);
/* y[t] = sum_k w[t, k] * o[slot_of[t*top_k + k]] in top-k order (the
 * reference's accumulation order, ternary_moe.rs:217-221). */
int ft_moe_combine(ft_ctx* ctx, ft_moe* m, int64_t T, const float* o_rows_dev,
                   const int32_t* slot_of_dev, const float* topk_w_dev, float* y_dev, void* stream);

/* ---- 3-bit KV cache: TurboQuantKVCache (src/inference/turboquant_kv.rs:173-411)
 * One layer of the cache for `batch` sequences with kv_heads heads of head_dim
 * 128 (kv_dim = kv_heads * 128, quantisation group 128 = one head vector, the
 * reference's group_size 128).  max_seq is the initial capacity; an append past
 * it grows the cache (a reallocation, not allowed during stream capture), as
 * the reference's Vec storage grows.  Replaces TurboQuantKVCache::new (:211). */
int ft_kv3_create(ft_ctx* ctx, int64_t batch, int64_t kv_heads, int64_t head_dim,
                  int64_t max_seq, ft_kv3** out);
/* Same with a quantisation mode: 0 = the reference scheme above; 1 = "mode T"
 * (BASELINE's TurboQuant description: rotation + 3-bit codebook + fp32 norm;
 * the reference has no working implementation, src/compute/turboquant.rs:89-367,
 * so this mode's spec and oracle are this project's own): each vector is
 * rotated by H D / ||v|| (D = 128 signs drawn from SplitMix64(seed), H the
 * Walsh-Hadamard transform) and each coordinate y coded as
 * clamp(floor((y / 2.5 + 1) * 4), 0, 7), the nearest of the 8 uniform centroids on
 * [-1, 1] that the reference's compute_mse_centroids (:197-220) converges to; the
 * record's (min, max) holds -/+ ||v|| * 2.5 * 7/8 / sqrt(128).  append, get_range
 * (rotated back), flash decode (q rotated in, the output rotated back) and
 * export / append_packed (the stored rotated codes) work in both modes. */
int ft_kv3_create_mode(ft_ctx* ctx, int64_t batch, int64_t kv_heads, int64_t head_dim,
                       int64_t max_seq, int mode, uint64_t seed, ft_kv3** out);
/* Mode T: the 128 rotation signs (+-1) into signs_host. */
int ft_kv3_signs(const ft_kv3* c, float* signs_host);
int ft_kv3_destroy(ft_kv3* c);
/* Appends n_pos positions per sequence: k, v [batch, n_pos, kv_heads, 128]
 * fp32 (bf16 bit patterns when is_bf16), quantised exactly as append /
 * quantize_vector / quantize_3bit do (:240-266, :370-389, :83-107). */
int ft_kv3_append(ft_ctx* ctx, ft_kv3* c, int64_t n_pos, const void* k_dev, const void* v_dev,
                  int is_bf16, void* stream);
/* Appends positions already in the reference's stored form: codes
 * [batch, n_pos, kv_heads*48] bytes (pack_3bit of the kv_dim codes, :121-137)
 * and (min, max) [batch, n_pos, kv_heads, 2]. */
int ft_kv3_append_packed(ft_ctx* ctx, ft_kv3* c, int64_t n_pos, const uint8_t* k_codes_dev,
                         const float* k_minmax_dev, const uint8_t* v_codes_dev,
                         const float* v_minmax_dev, void* stream);
/* seq_len (:345) and the current capacity in positions. */
int ft_kv3_len(const ft_kv3* c, int64_t* len);
int ft_kv3_capacity(const ft_kv3* c, int64_t* cap);
/* Drops the n oldest positions (evict_oldest / evict_to, :308-328). */
int ft_kv3_evict_front(ft_kv3* c, int64_t n);
int ft_kv3_reset(ft_kv3* c); /* reset (:360) */
/* get_range (:271-291): dequantised K, V [batch, end-start, kv_heads, 128] fp32. */
int ft_kv3_get_range(ft_ctx* ctx, const ft_kv3* c, int64_t start, int64_t end, float* k_out_dev,
                     float* v_out_dev, void* stream);
/* Positions [start, end) in the reference's stored form (see append_packed). */
int ft_kv3_export_range(ft_ctx* ctx, const ft_kv3* c, int64_t start, int64_t end,
                        uint8_t* k_codes_dev, float* k_minmax_dev, uint8_t* v_codes_dev,
                        float* v_minmax_dev, void* stream);
/* Flash decode over the whole cache: out[b, h] = sum_s softmax_s(scale *
 * q[b, h] . K[b, s, h / (q_heads / kv_heads)]) V[b, s, ...] with q, out
 * [batch, q_heads, 128] fp32; scale <= 0 selects 1/sqrt(128).  The math of
 * flash_decode_ref (tests/kernel_tests.rs:1073-1110) on the dequantised cache
 * with the GQA head map of cpu_attention_raw (src/model/cpu_block_attn_res.rs:471-472). */
int ft_flash_decode_3bit(ft_ctx* ctx, ft_kv3* c, const float* q_dev, int64_t q_heads, float scale,
                         float* out_dev, void* stream);

/* ---- paged 3-bit KV cache: the GPU storage behind PagedAttention
 * (src/inference/paged_attention.rs).  The reference keeps only the metadata
 * there -- BlockAllocator (:44-150) hands out block ids, a BlockTable (:158-224)
 * per request and layer maps logical block j to a block id, fork_request
 * (:449-472) shares blocks by reference count -- and creates no GPU buffers.
 * An ft_kvp is that missing pool: block id P is page P, 32 positions of every
 * kv head in the ring cache's record format (same quantisation, both modes).
 * The calls below take the caller's tables as a device int32 array
 * [batch][table_stride] (row b = BlockTable::table() of sequence b, padded)
 * and read or write through them; the allocator, reference counts and
 * copy-on-write stay with the caller (the Python mirror in
 * ferrisres_b200/paged.py, or the reference's own manager).  Page ids and
 * positions read on the device are bounds-checked: a bad entry is skipped and
 * reported by ft_ctx_check as FT_ERR_SHAPE.  page_size must be 32 (the
 * reference's default is 16), head_dim 128.  mode / seed as ft_kv3_create_mode.
 * Replaces BlockAllocator::new's pool (:58) on the device side. */
int ft_kvp_create(ft_ctx* ctx, int64_t num_pages, int64_t kv_heads, int64_t head_dim,
                  int64_t page_size, int mode, uint64_t seed, ft_kvp** out);
int ft_kvp_destroy(ft_kvp* pool);
int ft_kvp_signs(const ft_kvp* pool, float* signs_host);
/* Writes n_pos positions of each of `batch` sequences: sequence b's at
 * positions start_pos[b] .. start_pos[b] + n_pos - 1 (start_pos int32 on the
 * device), through its table row.  k, v [batch, n_pos, kv_heads, 128] fp32
 * (bf16 bit patterns when is_bf16), quantised as ft_kv3_append.  The pages a
 * call writes must not be shared between its sequences (copy them first:
 * ft_kvp_copy_pages). */
int ft_kvp_append(ft_ctx* ctx, ft_kvp* pool, int64_t batch, int64_t n_pos,
                  const int32_t* tables_dev, int64_t table_stride, const int32_t* start_pos_dev,
                  const void* k_dev, const void* v_dev, int is_bf16, void* stream);
/* Same with positions already in the reference's stored form (see
 * ft_kv3_append_packed). */
int ft_kvp_append_packed(ft_ctx* ctx, ft_kvp* pool, int64_t batch, int64_t n_pos,
                         const int32_t* tables_dev, int64_t table_stride,
                         const int32_t* start_pos_dev, const uint8_t* k_codes_dev,
                         const float* k_minmax_dev, const uint8_t* v_codes_dev,
                         const float* v_minmax_dev, void* stream);
/* Copy-on-write: page dst[i] := page src[i] (host arrays of page ids), one
 * device copy each, on `stream`. */
int ft_kvp_copy_pages(ft_ctx* ctx, ft_kvp* pool, int64_t n, const int32_t* src_pages_host,
                      const int32_t* dst_pages_host, void* stream);
/* Positions [start, end) of every sequence through its table: dequantised
 * [batch, end-start, kv_heads, 128] fp32, or the reference's stored form. */
int ft_kvp_get_range(ft_ctx* ctx, const ft_kvp* pool, int64_t batch, const int32_t* tables_dev,
                     int64_t table_stride, int64_t start, int64_t end, float* k_out_dev,
                     float* v_out_dev, void* stream);
int ft_kvp_export_range(ft_ctx* ctx, const ft_kvp* pool, int64_t batch, const int32_t* tables_dev,
                        int64_t table_stride, int64_t start, int64_t end, uint8_t* k_codes_dev,
                        float* k_minmax_dev, uint8_t* v_codes_dev, float* v_minmax_dev,
                        void* stream);
/* Flash decode of `batch` sequences of ragged lengths seq_lens[b] (int32 on
 * the device, 0 <= seq_lens[b] <= max_seq_len; an empty sequence gives 0):
 * math, GQA map and output as ft_flash_decode_3bit. */
int ft_kvp_flash_decode(ft_ctx* ctx, ft_kvp* pool, int64_t batch, const int32_t* tables_dev,
                        int64_t table_stride, const int32_t* seq_lens_dev, int64_t max_seq_len,
                        const float* q_dev, int64_t q_heads, float scale, float* out_dev,
                        void* stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
#endif /* FERRIS_TERNARY_H */
