//! Raw `extern "C"` bindings to libferris_ternary.so (declared in
//! include/ferris_ternary.h).  Every function returns an `ft_status` code
//! (`FT_OK` = 0); the message of a failure is `ft_last_error_string()`.
//! Device pointers are CUDA device addresses, streams are `cudaStream_t` as
//! `*mut c_void` (null = the legacy default stream).
#![allow(non_camel_case_types)]
use std::os::raw::{c_char, c_int, c_void};

#[repr(C)]
pub struct ft_ctx {
    _p: [u8; 0],
}
#[repr(C)]
pub struct ft_weight {
    _p: [u8; 0],
}
#[repr(C)]
pub struct ft_moe {
    _p: [u8; 0],
}
#[repr(C)]
pub struct ft_kv3 {
    _p: [u8; 0],
}
#[repr(C)]
pub struct ft_kvp {
    _p: [u8; 0],
}

/// Status codes (map onto FerrisResError, src/error.rs:3-36).
pub const FT_OK: c_int = 0;
pub const FT_ERR_SHAPE: c_int = 1;
pub const FT_ERR_GPU: c_int = 2;
pub const FT_ERR_OOM: c_int = 3;
pub const FT_ERR_UNSUPPORTED: c_int = 4;
pub const FT_ERR_TIMEOUT: c_int = 5;
pub const FT_ERR_DEVICE: c_int = 6;

extern "C" {
    pub fn ft_version() -> *const c_char;
    pub fn ft_last_error_string() -> *const c_char;
    pub fn ft_launch_counter() -> u64;
    pub fn ft_ctx_create(device: c_int, out: *mut *mut ft_ctx) -> c_int;
    pub fn ft_ctx_destroy(ctx: *mut ft_ctx) -> c_int;
    pub fn ft_ctx_check(ctx: *mut ft_ctx) -> c_int;
    pub fn ft_weight_upload_packed_u8(ctx: *mut ft_ctx, packed_host: *const u8, rows: i64, cols: i64, row_scales_host: *const f32, out: *mut *mut ft_weight) -> c_int;
    pub fn ft_weight_upload_packed_u32(ctx: *mut ft_ctx, words_host: *const u32, rows: i64, cols: i64, row_scales_host: *const f32, out: *mut *mut ft_weight) -> c_int;
    pub fn ft_weight_from_device_u32(ctx: *mut ft_ctx, words_dev: *const u32, rows: i64, cols: i64, row_scales_dev: *const f32, stream: *mut c_void, out: *mut *mut ft_weight) -> c_int;
    pub fn ft_sparse_upload_host(ctx: *mut ft_ctx, patterns_host: *const u8, signs_host: *const u8, rows: i64, cols: i64, row_scales_host: *const f32, out: *mut *mut ft_weight) -> c_int;
    pub fn ft_sparse_upload_wgsl(ctx: *mut ft_ctx, words_host: *const u32, rows: i64, cols: i64, row_scales_host: *const f32, out: *mut *mut ft_weight) -> c_int;
    pub fn ft_weight_export_packed_u8(ctx: *mut ft_ctx, w: *const ft_weight, packed_host: *mut u8) -> c_int;
    pub fn ft_weight_destroy(w: *mut ft_weight) -> c_int;
    pub fn ft_weight_info(w: *const ft_weight, rows: *mut i64, cols: *mut i64, device_bytes: *mut i64) -> c_int;
    pub fn ft_weight_upload_index_lists(ctx: *mut ft_ctx, rows: i64, cols: i64, pos_off: *const i64, pos_idx: *const i64, neg_off: *const i64, neg_idx: *const i64, row_scales_host: *const f32, out: *mut *mut ft_weight) -> c_int;
    pub fn ft_weight_quantize_f32(ctx: *mut ft_ctx, w_host: *const f32, rows: i64, cols: i64, alpha_out: *mut f32, out: *mut *mut ft_weight) -> c_int;
    pub fn ft_weight_requantize(ctx: *mut ft_ctx, w: *mut ft_weight, src_dev: *const c_void, src_bf16: c_int, alpha: f32, stream: *mut c_void) -> c_int;
    pub fn ft_shadow_alpha(ctx: *mut ft_ctx, n: c_int, src_dev: *const *const c_void, counts: *const i64, src_bf16: c_int, alpha_out: *mut f32) -> c_int;
    pub fn ft_ternary_matmul_f32(ctx: *mut ft_ctx, w: *const ft_weight, seq: i64, x_dev: *const f32, y_dev: *mut f32, stream: *mut c_void) -> c_int;
    pub fn ft_ternary_matmul_bf16(ctx: *mut ft_ctx, w: *const ft_weight, seq: i64, x_dev: *const u16, y_dev: *mut f32, stream: *mut c_void) -> c_int;
    pub fn ft_ternary_matmul_f32_grouped(ctx: *mut ft_ctx, n: c_int, ws: *const *const ft_weight, seq: i64, xs_dev: *const *const f32, ys_dev: *const *mut f32, stream: *mut c_void) -> c_int;
    pub fn ft_ternary_matmul_i8_grouped(ctx: *mut ft_ctx, n: c_int, ws: *const *const ft_weight, seq: i64, qs_dev: *const *const i8, sxs_dev: *const *const f32, ys_dev: *const *mut f32, stream: *mut c_void) -> c_int;
    pub fn ft_ternary_matmul_f32_noalloc(ctx: *mut ft_ctx, w: *const ft_weight, seq: i64, x_dev: *const f32, y_dev: *mut f32, stream: *mut c_void) -> c_int;
    pub fn ft_ternary_matmul_blocked_f32(ctx: *mut ft_ctx, w: *const ft_weight, seq: i64, x_dev: *const f32, block_scales_dev: *const f32, block_size: i64, y_dev: *mut f32, stream: *mut c_void) -> c_int;
    pub fn ft_quantize_absmax_i8_f32(ctx: *mut ft_ctx, seq: i64, cols: i64, x_dev: *const f32, q_dev: *mut i8, sx_dev: *mut f32, stream: *mut c_void) -> c_int;
    pub fn ft_quantize_absmax_i8_bf16(ctx: *mut ft_ctx, seq: i64, cols: i64, x_dev: *const u16, q_dev: *mut i8, sx_dev: *mut f32, stream: *mut c_void) -> c_int;
    pub fn ft_ternary_matmul_i8(ctx: *mut ft_ctx, w: *const ft_weight, seq: i64, q_dev: *const i8, sx_dev: *const f32, y_dev: *mut f32, stream: *mut c_void) -> c_int;
    pub fn ft_ternary_matmul_op_dispatch(ctx: *mut ft_ctx, ternary_dev: *const u32, scales_dev: *const f32, input_dev: *const f32, output_dev: *mut f32, seq_len: u32, in_cols: u32, out_rows: u32, stream: *mut c_void) -> c_int;
    pub fn ft_gpu_ternary_matmul(ctx: *mut ft_ctx, packed_weights_host: *const u32, scales_host: *const f32, input_host: *const f32, seq_len: usize, in_cols: usize, out_rows: usize, output_host: *mut f32) -> c_int;
    pub fn ft_gpu_sparse_ternary_matmul(ctx: *mut ft_ctx, sparse_words_host: *const u32, scale: f32, input_host: *const f32, seq_len: usize, in_cols: usize, out_rows: usize, output_host: *mut f32) -> c_int;
    pub fn ft_gpu_ternary_matmul_vram(ctx: *mut ft_ctx, w: *const ft_weight, input_host: *const f32, seq_len: usize, in_cols: usize, out_rows: usize, output_host: *mut f32) -> c_int;
    pub fn ft_moe_create(ctx: *mut ft_ctx, n_experts: i64, hidden: i64, inter: i64, top_k: c_int, use_gelu: c_int, router_host: *const f32, gate_packed: *const *const u8, gate_scales: *const *const f32, up_packed: *const *const u8, up_scales: *const *const f32, down_packed: *const *const u8, down_scales: *const *const f32, out: *mut *mut ft_moe) -> c_int;
    pub fn ft_moe_destroy(m: *mut ft_moe) -> c_int;
    pub fn ft_moe_forward(ctx: *mut ft_ctx, m: *mut ft_moe, T: i64, x_dev: *const c_void, x_is_bf16: c_int, y_dev: *mut f32, probs_dev: *mut f32, stream: *mut c_void) -> c_int;
    pub fn ft_moe_create_f32(ctx: *mut ft_ctx, n_experts: i64, hidden: i64, inter: i64, top_k: c_int, use_gelu: c_int, router_host: *const f32, gate_f32: *const *const f32, up_f32: *const *const f32, down_f32: *const *const f32, out: *mut *mut ft_moe) -> c_int;
    pub fn ft_moe_decode(ctx: *mut ft_ctx, m: *mut ft_moe, T: i64, x_dev: *const c_void, x_is_bf16: c_int, y_dev: *mut f32, topk_idx_dev: *mut i32, topk_w_dev: *mut f32, probs_dev: *mut f32, stream: *mut c_void) -> c_int;
    pub fn ft_moe_forward_host(ctx: *mut ft_ctx, m: *mut ft_moe, input_host: *const f32, seq: usize, output_host: *mut f32) -> c_int;
    pub fn ft_moe_route(ctx: *mut ft_ctx, m: *mut ft_moe, T: i64, x_dev: *const c_void, x_is_bf16: c_int, topk_idx_dev: *mut i32, topk_w_dev: *mut f32, probs_dev: *mut f32, counts_dev: *mut i32, stream: *mut c_void) -> c_int;
    pub fn ft_moe_dispatch_layout(ctx: *mut ft_ctx, m: *mut ft_moe, T: i64, topk_idx_dev: *const i32, counts_dev: *const i32, offsets_dev: *mut i32, fill_dev: *mut i32, slot_of_dev: *mut i32, token_of_dev: *mut i32, stream: *mut c_void) -> c_int;
    pub fn ft_moe_gather_rows(ctx: *mut ft_ctx, x_dev: *const c_void, elem_bytes: c_int, H: i64, token_of_dev: *const i32, n_rows: i64, out_dev: *mut c_void, stream: *mut c_void) -> c_int;
    pub fn ft_moe_expert_ffn(ctx: *mut ft_ctx, m: *mut ft_moe, nseg: c_int, seg_expert_host: *const i32, seg_rows_host: *const i64, x_rows_dev: *const c_void, x_is_bf16: c_int, y_rows_dev: *mut f32, stream: *mut c_void) -> c_int;
    pub fn ft_moe_combine(ctx: *mut ft_ctx, m: *mut ft_moe, T: i64, o_rows_dev: *const f32, slot_of_dev: *const i32, topk_w_dev: *const f32, y_dev: *mut f32, stream: *mut c_void) -> c_int;
    pub fn ft_kv3_create(ctx: *mut ft_ctx, batch: i64, kv_heads: i64, head_dim: i64, max_seq: i64, out: *mut *mut ft_kv3) -> c_int;
    pub fn ft_kv3_create_mode(ctx: *mut ft_ctx, batch: i64, kv_heads: i64, head_dim: i64, max_seq: i64, mode: c_int, seed: u64, out: *mut *mut ft_kv3) -> c_int;
    pub fn ft_kv3_signs(c: *const ft_kv3, signs_host: *mut f32) -> c_int;
    pub fn ft_kv3_destroy(c: *mut ft_kv3) -> c_int;
    pub fn ft_kv3_append(ctx: *mut ft_ctx, c: *mut ft_kv3, n_pos: i64, k_dev: *const c_void, v_dev: *const c_void, is_bf16: c_int, stream: *mut c_void) -> c_int;
    pub fn ft_kv3_append_packed(ctx: *mut ft_ctx, c: *mut ft_kv3, n_pos: i64, k_codes_dev: *const u8, k_minmax_dev: *const f32, v_codes_dev: *const u8, v_minmax_dev: *const f32, stream: *mut c_void) -> c_int;
    pub fn ft_kv3_len(c: *const ft_kv3, len: *mut i64) -> c_int;
    pub fn ft_kv3_capacity(c: *const ft_kv3, cap: *mut i64) -> c_int;
    pub fn ft_kv3_evict_front(c: *mut ft_kv3, n: i64) -> c_int;
    pub fn ft_kv3_reset(c: *mut ft_kv3) -> c_int;
    pub fn ft_kv3_get_range(ctx: *mut ft_ctx, c: *const ft_kv3, start: i64, end: i64, k_out_dev: *mut f32, v_out_dev: *mut f32, stream: *mut c_void) -> c_int;
    pub fn ft_kv3_export_range(ctx: *mut ft_ctx, c: *const ft_kv3, start: i64, end: i64, k_codes_dev: *mut u8, k_minmax_dev: *mut f32, v_codes_dev: *mut u8, v_minmax_dev: *mut f32, stream: *mut c_void) -> c_int;
    pub fn ft_flash_decode_3bit(ctx: *mut ft_ctx, c: *mut ft_kv3, q_dev: *const f32, q_heads: i64, scale: f32, out_dev: *mut f32, stream: *mut c_void) -> c_int;
    pub fn ft_kvp_create(ctx: *mut ft_ctx, num_pages: i64, kv_heads: i64, head_dim: i64, page_size: i64, mode: c_int, seed: u64, out: *mut *mut ft_kvp) -> c_int;
    pub fn ft_kvp_destroy(pool: *mut ft_kvp) -> c_int;
    pub fn ft_kvp_signs(pool: *const ft_kvp, signs_host: *mut f32) -> c_int;
    pub fn ft_kvp_append(ctx: *mut ft_ctx, pool: *mut ft_kvp, batch: i64, n_pos: i64, tables_dev: *const i32, table_stride: i64, start_pos_dev: *const i32, k_dev: *const c_void, v_dev: *const c_void, is_bf16: c_int, stream: *mut c_void) -> c_int;
    pub fn ft_kvp_append_packed(ctx: *mut ft_ctx, pool: *mut ft_kvp, batch: i64, n_pos: i64, tables_dev: *const i32, table_stride: i64, start_pos_dev: *const i32, k_codes_dev: *const u8, k_minmax_dev: *const f32, v_codes_dev: *const u8, v_minmax_dev: *const f32, stream: *mut c_void) -> c_int;
    pub fn ft_kvp_copy_pages(ctx: *mut ft_ctx, pool: *mut ft_kvp, n: i64, src_pages_host: *const i32, dst_pages_host: *const i32, stream: *mut c_void) -> c_int;
    pub fn ft_kvp_get_range(ctx: *mut ft_ctx, pool: *const ft_kvp, batch: i64, tables_dev: *const i32, table_stride: i64, start: i64, end: i64, k_out_dev: *mut f32, v_out_dev: *mut f32, stream: *mut c_void) -> c_int;
    pub fn ft_kvp_export_range(ctx: *mut ft_ctx, pool: *const ft_kvp, batch: i64, tables_dev: *const i32, table_stride: i64, start: i64, end: i64, k_codes_dev: *mut u8, k_minmax_dev: *mut f32, v_codes_dev: *mut u8, v_minmax_dev: *mut f32, stream: *mut c_void) -> c_int;
    pub fn ft_kvp_flash_decode(ctx: *mut ft_ctx, pool: *mut ft_kvp, batch: i64, tables_dev: *const i32, table_stride: i64, seq_lens_dev: *const i32, max_seq_len: i64, q_dev: *const f32, q_heads: i64, scale: f32, out_dev: *mut f32, stream: *mut c_void) -> c_int;
}
