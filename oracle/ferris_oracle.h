/*
 * ferris_oracle.h -- CPU restatement of FerrisRes's ternary hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA path
 * of ferrisres_b200 is compared against, and the CPU baseline that bench.py
 * times beside it.  Nothing in the product (ferrisres_b200/, include/) links,
 * loads or calls it.
 *
 * Every function restates one function of the reference crate (shift/FerrisRes
 * v0.2.3, Rust) and cites the file:line it follows.  The reference cannot be
 * built in this image (no Rust toolchain, crate dependencies not vendored), so
 * the restatement is pinned against the reference's own unit-test known
 * answers, which tests/test_oracle_kats.py reproduces value for value.
 *
 * Summation order is the reference's (sequential over K, pos/neg split where
 * the reference splits), so float results match the reference bit for bit
 * wherever the reference's order is deterministic.
 */
#ifndef FERRIS_ORACLE_H
#define FERRIS_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- ternary codes: src/model/ternary.rs:134-179, :1317-1328 ------------ */
void fo_pack_ternary(const int8_t* values, size_t n, uint8_t* packed /* (n+3)/4 */);
void fo_unpack_ternary(const uint8_t* packed, size_t n, int8_t* values);
void fo_pack_ternary_u32(const uint8_t* packed_u8, size_t n_bytes, size_t total_values,
                         uint32_t* out /* (total_values+15)/16 */);
/* WGSL test packer: per-row ceil(cols/16) words, src/compute/kernels/ternary_matmul.rs:267-291 */
void fo_pack_ternary_rows_u32(const int8_t* values, size_t rows, size_t cols, uint32_t* out);

/* absmean quantizer src/model/ternary.rs:31-57; returns alpha */
float fo_quantize_ternary(const float* w, size_t n, int8_t* q);

/* ---- dense ternary matmuls ----------------------------------------------- */
/* src/model/ternary.rs:292-328 (pos/neg split, scalar scale) */
void fo_ternary_matmul(const int8_t* t, float scale, const float* x, size_t out_rows,
                       size_t in_cols, size_t seq, float* y);
/* src/model/ternary.rs:401-464 (flat packed indexing) */
void fo_ternary_matmul_packed(const uint8_t* packed, float scale, const float* x,
                              size_t out_rows, size_t in_cols, size_t seq, float* y);
/* src/model/ternary.rs:591-633 (8-way unrolled sequential) */
void fo_ternary_matmul_decode(const int8_t* t, float scale, const float* x, size_t out_rows,
                              size_t in_cols, float* y);
/* src/model/ternary.rs:541-579 (one scale per column block, shared by the rows) */
void fo_ternary_matmul_blocked(const int8_t* t, const float* scales, size_t block_size,
                               const float* x, size_t out_rows, size_t in_cols, size_t seq,
                               float* y);
/* src/model/ternary.rs:76-110 (flat blocks of block_size elements) */
void fo_quantize_ternary_blocked(const float* w, size_t n, size_t block_size, int8_t* q,
                                 float* scales);
/* src/model/ternary.rs:681-707 as CSR (offsets [out_rows + 1]) */
void fo_ternary_sparse_indices(const int8_t* t, size_t out_rows, size_t in_cols, int64_t* pos_off,
                               int64_t* pos_idx, int64_t* neg_off, int64_t* neg_idx);
/* src/model/ternary.rs:647-672 */
void fo_ternary_matmul_sparse_decode(const int64_t* pos_off, const int64_t* pos_idx,
                                     const int64_t* neg_off, const int64_t* neg_idx, float scale,
                                     const float* x, size_t out_rows, float* y);
/* src/training/bit_moe.rs:243-262 (STE requantize with a shared alpha; bf16 shadows) */
void fo_bitmoe_requantize(const uint16_t* shadow_bf16, size_t n, float alpha, int8_t* q);
/* src/training/bit_moe.rs:210-241 (sequential f64 mean of |shadow|); 0 when empty */
int fo_bitmoe_recompute_alpha(const uint16_t* const* shadows, const size_t* counts, size_t n,
                              float* alpha);
/* src/model/ternary.rs:471-529 restated with per-row scales (row_scales[r] in place of the
 * scalar, which is what gpu_packed() broadcasts, src/model/cpu_moe.rs:73-78).  Threads: the
 * reference's 32 row batches over `nthreads` workers (nthreads<=0: all cores). */
void fo_ternary_matmul_packed_parallel_rows(const uint8_t* packed, const float* row_scales,
                                            const float* x, size_t out_rows, size_t in_cols,
                                            float* y, int nthreads);
/* src/model/cpu_block_attn_res.rs:2373-2398 == WGSL ref src/compute/kernels/ternary_matmul.rs:233-265 */
void fo_gpu_ternary_mm_cpu(const uint32_t* packed, const float* scales, const float* x,
                           size_t seq, size_t in_cols, size_t out_rows, float* y);
/* src/model/ternary.rs:333-389 (parallel over tokens for seq>1), int8 codes fed as f32 */
void fo_ternary_matmul_parallel(const int8_t* t, float scale, const float* x, size_t out_rows,
                                size_t in_cols, size_t seq, float* y, int nthreads);

/* ---- int8 activation mode (pinned here; the reference has none) ---------- */
/* sx = absmax/127 (absmax==0 -> sx=1, q=0); q = clamp(round_half_away(x*(127/absmax)),-127,127) */
void fo_quantize_absmax_i8(const float* x, size_t seq, size_t cols, int8_t* q, float* sx);
/* y[m,n] = ((float)acc * sx[m]) * sw[n], acc = exact int32 sum; threaded over tokens */
void fo_ternary_matmul_i8(const int8_t* t, const int8_t* q, const float* sx, const float* sw,
                          size_t seq, size_t in_cols, size_t out_rows, float* y, int nthreads);
/* reference ternary_matmul (pos/neg split, f32) on int8 codes-as-f32, then the same epilogue */
void fo_ternary_matmul_i8_via_f32(const int8_t* t, const int8_t* q, const float* sx,
                                  const float* sw, size_t seq, size_t in_cols, size_t out_rows,
                                  float* y, int nthreads);

/* ---- 2:4 sparse (host layout) src/model/sparse_ternary.rs ---------------- */
/* from_ternary :78-150; patterns (ngroups+1)/2 bytes, signs (ngroups+3)/4 bytes */
void fo_sparse_from_ternary(const int8_t* t, size_t rows, size_t cols, uint8_t* patterns,
                            uint8_t* signs);
void fo_sparse_to_ternary(const uint8_t* patterns, const uint8_t* signs, size_t rows,
                          size_t cols, int8_t* t); /* :166-192 */
/* sparse_ternary_matmul :203-252, with per-row scales (row_scales==NULL -> scalar `scale`) */
void fo_sparse_ternary_matmul(const uint8_t* patterns, const uint8_t* signs, float scale,
                              const float* row_scales, size_t rows, size_t cols, const float* x,
                              size_t seq, float* y, int nthreads);
/* WGSL layout (5 bits/group, 6 groups/u32, sign 1 = -1): src/compute/kernels/sparse_ternary.rs:254-360 */
size_t fo_sparse_wgsl_words_per_row(size_t cols);
int fo_sparse_wgsl_pack(const int8_t* t, size_t rows, size_t cols, uint32_t* packed);
void fo_sparse_wgsl_ref(const uint32_t* packed, const float* scales, const float* x, size_t seq,
                        size_t cols, size_t rows, float* y);

/* ---- MoE layer: src/model/ternary_moe.rs:145-223 --------------------------
 * router [E, H] (row e = expert e), experts gate/up [F, H], down [H, F] as int8
 * ternary with per-row scales.  top-k by stable descending sort of softmax
 * probabilities; weights renormalised by their sum; SwiGLU x/(1+exp(-x)) * up.
 * Threaded over tokens (nthreads<=0: all cores).  route_out (optional) gets
 * the chosen experts [seq, top_k] and probs_out the softmax [seq, E]. */
void fo_moe_forward(const float* router, const int8_t* const* gate, const float* const* gate_s,
                    const int8_t* const* up, const float* const* up_s,
                    const int8_t* const* down, const float* const* down_s, size_t hidden,
                    size_t inter, size_t n_experts, size_t top_k, int use_gelu, const float* x,
                    size_t seq, float* y, int32_t* route_out, float* probs_out, int nthreads);

/* ---- TurboQuant 3-bit KV: src/inference/turboquant_kv.rs ---------------- */
void fo_pack_3bit(const uint8_t* codes, size_t n, uint8_t* packed /* 3*ceil(n/8) */);
void fo_unpack_3bit(const uint8_t* packed, size_t n, uint8_t* codes);
/* quantize_3bit :83-107; returns codes, *mn, *mx */
void fo_quantize_3bit(const float* v, size_t n, uint8_t* codes, float* mn, float* mx);
void fo_dequantize_3bit(const uint8_t* codes, size_t n, float mn, float mx, float* out);
/* append one position: quantize_vector + pack per group (:240-266, :370-389) */
void fo_kv_quantize_vector(const float* v, size_t kv_dim, size_t group, uint8_t* packed,
                           float* minmax /* [ngroups][2] */);
/* get_range dequant of one position (:271-291, :391-410) */
void fo_kv_dequantize_vector(const uint8_t* packed, const float* minmax, size_t kv_dim,
                             size_t group, float* out);

/* flash_decode_ref tests/kernel_tests.rs:1073-1110, generalised to GQA with the
 * kv-head map of src/model/cpu_block_attn_res.rs:471-472 (kv_h = h / (Hq/Hkv)).
 * q [B, Hq, d]; K, V [B, S, Hkv, d] f32; out [B, Hq, d]; scale = 1/sqrt(d). */
void fo_flash_decode_gqa(const float* q, const float* k, const float* v, size_t batch,
                         size_t seq, size_t hq, size_t hkv, size_t d, float* out, int nthreads);
/* Same over the reference 3-bit cache: K/V codes [B, S, Hkv, 3d/8] bytes, minmax
 * [B, S, Hkv, 2] (group = d), dequantised exactly as get_range does. */
void fo_flash_decode_3bit(const float* q, const uint8_t* kc, const float* kmm, const uint8_t* vc,
                          const float* vmm, size_t batch, size_t seq, size_t hq, size_t hkv,
                          size_t d, float* out, int nthreads);

int fo_num_threads(int requested);

/* 3-bit KV mode T (this project's spec; see ferris_oracle.c): one 128-vector ->
 * codes 0..7 and its norm; (min, max) of the shared record = -/+ norm * fo_kvt_mm_const() */
void fo_kvt_quantize(const float* v, const float* signs, uint8_t* codes, float* norm_out);
float fo_kvt_mm_const(void);
/* q' = H D q / sqrt(128) (inverse 0) or o = D H o' / sqrt(128) (inverse 1) */
void fo_kvt_rotate(const float* in, const float* signs, int inverse, float* out);
#ifdef __cplusplus
}
#endif
#endif
