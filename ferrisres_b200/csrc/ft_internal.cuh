// Internal definitions shared by the translation units of libferris_ternary.so.
//
// Device layout of a dense ternary weight ("tiled T128", lane-major blocks):
//   rows are grouped into tiles of 128 output channels, K into chunks of 128
//   codes.  Block (tile t, chunk c) is 4096 contiguous bytes at offset
//   (t * n_chunks + c) * 4096, arranged for the int8 MMA fragments of a warp:
//       [m-block mb in 0..7][lane L in 0..31][word i in 0..3]
//   with L = 4g + r.  Word i of lane (g, r) in m-block mb holds 16 codes:
//   byte b, bits 2j..2j+1 = code of
//       row 16*mb + g + 8*(i & 1),  K position 32*j + 16*(i >> 1) + 4*r + b,
//   i.e. code slot j belongs to k-step j of an m16n8k32 MMA and word i is
//   fragment register ai of it (a0/a1: rows g / g+8, k 4r..4r+3; a2/a3: the
//   same rows, k 16+4r..16+4r+3).  So the four words AND (3 << 2j) are the
//   A fragment of k-step j scaled by 4^j (one logic op per register; the
//   decode kernel divides the 4^j out of its per-k-step accumulators), and
//   (word >> 2j) & 0x03030303 are four unsigned bytes {0,1,2} = (w+1) at
//   K-consecutive positions (the tensor-core engine's TMEM operand).  A
//   row's 128 codes of a chunk are spread over the 4 lanes (g, 0..3) of its
//   m-block: 64 contiguous bytes.  Codes: 0 -> -1, 1 -> 0, 2 -> +1 (same as
//   the reference).  Padding rows and padding K positions hold code 1
//   (weight 0).
//
// Device layout of a 2:4 sparse weight (every group of 4 K positions holds
// exactly two +-1): the same tiles and chunks; block (t, c) is 3072 bytes,
// 8 m-blocks of 384 bytes each, in the operand form of the sparse tensor-core
// MMA (mma.sp m16n8k64 s8, ordered metadata): per m-block and k64 step s
// (chunk K 64s .. 64s+63, 16 groups j) lane L = 4g + t holds
//   * metadata: 8 nibbles, nibble i = (idx0 | idx1 << 2), the positions
//     inside group j = 8 * (t >> 1) + i of row 16*mb + g + 8 * (t & 1)
//     (idx0 < idx1) -- as uint2 (s = 0, 1) at byte 8L of the m-block record;
//   * signs: 16 bits, bit 4i + e = the sign (1 = -1) of compressed value e of
//     A register i, i.e. of nonzero (e & 1) of group 8 * (i >> 1) + 2t + (e >> 1)
//     of row g + 8 * (i & 1) -- as the low (s = 0) / high (s = 1) half of the
//     u32 at byte 256 + 4L.
// 1.5 bits per weight, the size of the reference's own packing (3-bit
// pattern in a nibble + 2 sign bits per group).  Padding rows and groups
// hold positions (0, 1) with signs +1: their products meet zero activations
// (K padding) or land in outputs that are never stored (row padding).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/ferris_ternary.h"

namespace ft {

constexpr int kTileRows = 128;  // output channels per tile
constexpr int kChunkK = 128;    // K codes per chunk
constexpr int kBlockBytes = kTileRows * kChunkK / 4;  // 4096 (dense 2-bit block)
// 2:4 sparse block: 8 m-blocks x 384 bytes (metadata + signs, see above).
constexpr int kSparseMbBytes = 384;
constexpr int kSparseBlockBytes = 8 * kSparseMbBytes;  // 3072
// reference pattern p (the two nonzero positions of a group, in order) ->
// metadata nibble idx0 | idx1 << 2: (0,1) (0,2) (0,3) (1,2) (1,3) (2,3)
__host__ __device__ constexpr uint32_t sparse_nibble(int p) {
  return (0xED9C84u >> (4 * p)) & 0xFu;
}

void set_error(const char* fmt, ...);
extern std::atomic<uint64_t> g_launches;  // kernels launched by this library
int fail(int status, const char* fmt, ...);

#define FT_CUDA(call)                                                                    \
  do {                                                                                   \
    cudaError_t e_ = (call);                                                             \
    if (e_ != cudaSuccess)                                                               \
      return ::ft::fail(e_ == cudaErrorMemoryAllocation ? FT_ERR_OOM : FT_ERR_GPU,       \
                        "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, \
                        __LINE__);                                                       \
  } while (0)

#define FT_CHECK(cond, status, ...)                 \
  do {                                              \
    if (!(cond)) return ::ft::fail(status, __VA_ARGS__); \
  } while (0)

// Kernel launch check: reports launch-configuration errors without syncing,
// and counts the launch.
#define FT_LAUNCH_CHECK()                                                                  \
  do {                                                                                     \
    ::ft::g_launches.fetch_add(1, std::memory_order_relaxed);                              \
    cudaError_t e_ = cudaGetLastError();                                                   \
    if (e_ != cudaSuccess)                                                                 \
      return ::ft::fail(FT_ERR_GPU, "kernel launch failed: %s (%s:%d)",                    \
                        cudaGetErrorString(e_), __FILE__, __LINE__);                        \
  } while (0)

inline int64_t round_up(int64_t a, int64_t b) { return (a + b - 1) / b * b; }
inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Fixed-point digits of an fp32/bf16 activation token: the kernels multiply
// the token by the power of two 2^sh that puts its largest finite |x| in
// [2^(8D-3), 2^(8D-2)) and split X = round(x * 2^sh) into D signed base-256
// digits (the top one within +-64).  D = 8 (the public fp32/bf16 entry points)
// represents every element within 2^38 of the token's absmax exactly, so the
// exact int32 digit sums give the correctly rounded dot product; D = 4 (the
// MoE expert GEMMs, tolerance 1e-4 of the output rms) rounds elements below
// absmax * 2^-6 to a quantum of absmax * 2^-30.
constexpr int kDigitsExact = 8;
constexpr int kDigitsMoE = 4;
// Non-finite activation positions remembered per token; a token with more is
// handled by scanning its whole row.
constexpr int kNfCap = 16;

#ifdef __CUDACC__
// sh such that 2^sh * a lies in [2^(8D-3), 2^(8D-2)) for a finite a > 0.
__device__ __forceinline__ int digit_shift(float a, int D) {
  const uint32_t ebits = __float_as_uint(a) >> 23;
  if (ebits != 0u) return (8 * D - 2) + 126 - (int)ebits;
  int ex = 0;
  frexpf(a, &ex);  // subnormal absmax
  return (8 * D - 2) - ex;
}

// Weight w in {-1, 0, +1} at (row R, column k) of a resident weight, read from
// its tiled layout (dense or 2:4, both described at the top of this file).  A
// slow scalar lookup for the non-finite activation path and the export.
__device__ __forceinline__ int weight_at(const uint8_t* codes, int format, int64_t n_chunks,
                                         int64_t R, int64_t k) {
  const int64_t t = R >> 7, c = k >> 7;
  const int r = (int)(R & 127), kk = (int)(k & 127);
  if (format == 0) {
    const uint8_t* blk = codes + (t * n_chunks + c) * kBlockBytes;
    const int mb = r >> 4, g = r & 7, ih = (r >> 3) & 1;
    const int j = kk >> 5, il = (kk >> 4) & 1, rr = (kk >> 2) & 3, b = kk & 3;
    const int byte = blk[(mb * 32 + 4 * g + rr) * 16 + (2 * il + ih) * 4 + b];
    return ((byte >> (2 * j)) & 3) - 1;
  }
  // 2:4: the metadata nibble of group j in k64 step s, then its sign bit
  const uint8_t* mbr = codes + (t * n_chunks + c) * kSparseBlockBytes + (r >> 4) * kSparseMbBytes;
  const int g = r & 7, h8 = (r >> 3) & 1, s = kk >> 6, j = (kk & 63) >> 2, e = kk & 3;
  const uint32_t meta = reinterpret_cast<const uint32_t*>(mbr)[2 * (4 * g + 2 * (j >> 3) + h8) + s];
  const uint32_t nib = (meta >> (4 * (j & 7))) & 0xFu;
  const int i0 = (int)(nib & 3u), i1 = (int)(nib >> 2);
  if (e != i0 && e != i1) return 0;
  const int pos = e == i0 ? 0 : 1;
  const uint32_t sg = reinterpret_cast<const uint32_t*>(mbr + 256)[4 * g + ((j & 7) >> 1)] >> (16 * s);
  const int bit = 4 * (2 * (j >> 3) + h8) + 2 * (j & 1) + pos;
  return ((sg >> bit) & 1u) ? -1 : 1;
}

// round(xs) as a 64-bit integer, |xs| < 2^63: integer-valued floats
// (|xs| >= 2^23) are read straight from their bits, smaller ones go through
// the 32-bit conversion.
__device__ __forceinline__ long long float_to_ll_exact(float xs) {
  const uint32_t b = __float_as_uint(xs);
  const int e = (int)((b >> 23) & 255u);
  if (e < 150) return (long long)__float2int_rn(xs);
  const unsigned long long m = (unsigned long long)((b & 0x7fffffu) | 0x800000u) << (e - 150);
  return (b >> 31) ? -(long long)m : (long long)m;
}

__device__ __forceinline__ bool is_nonfinite(float v) {
  return (__float_as_uint(v) & 0x7f800000u) == 0x7f800000u;
}

// The expert activation of the reference (ternary_moe.rs:199-209), act 1:
// SwiGLU silu(g) * u with silu(g) = g / (1 + e^-g); act 2: GeLU-tanh of g.
__device__ __forceinline__ float expert_act(float g, float u, int act) {
  if (act == 2) {
    const float ta = __fmul_rn(0.7978845608f,
                               __fadd_rn(g, __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, g), g), g)));
    return __fmul_rn(__fmul_rn(0.5f, g), __fadd_rn(1.0f, tanhf(ta)));
  }
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

// Output of row R for a token x_row [K] (fp32, or bf16 bit patterns when
// bf16) that holds non-finite elements.  The reference's per-row-scale
// matmuls (TernaryMatMulOp, src/compute/kernels/ternary_matmul.rs:54-70, and
// gpu_ternary_mm_cpu, src/model/cpu_block_attn_res.rs:2373-2398) add x[k] only
// where the weight is nonzero, in fp32: a row meeting a NaN, or infinities of
// both signs, ends NaN; one sign of infinity gives +-inf; then sum * scale.
// `pos` lists the token's non-finite positions (cnt of them; more than kNfCap:
// the whole row is scanned).  y_finite is returned when the row meets none.
//
// act != 0: x_row is a row of interleaved gate/up outputs and element k is
// expert_act(gate_k, up_k) (the MoE's fused activation operand).
//
// Column-block scales (ternary_matmul_blocked, src/model/ternary.rs:541-579:
// kscale != null, one scale per kblock columns): the kernels fold the scale
// into the activation, x' = kscale[k / kblock] * x, and that reference
// multiplies w * x in fp32, so a zero weight meeting an infinity gives NaN
// too (0 * inf).
// Kept out of line: it runs only for tokens with non-finite elements, and
// inlining its loops into the kernels' epilogues slows their common path.
static __device__ __noinline__ float nonfinite_row(float y_finite, const uint8_t* codes, int format,
                                               int64_t n_chunks, int64_t R, const void* x_row,
                                               bool bf16, int64_t K, const int* pos, int cnt,
                                               float scale, const float* kscale,
                                               int64_t kblock, int act = 0) {
  bool nan = false, pinf = false, ninf = false;
  const bool all = cnt > kNfCap;
  const int64_t n = all ? K : cnt;
  for (int64_t i = 0; i < n; ++i) {
    const int64_t k = all ? i : pos[i];
    float v;
    if (act) {  // x_row holds interleaved gate/up values (fp32)
      const float* gp = static_cast<const float*>(x_row) + 32 * (k >> 4) + (k & 15);
      v = expert_act(gp[0], gp[16], act);
    } else {
      v = bf16 ? __uint_as_float((uint32_t) static_cast<const uint16_t*>(x_row)[k] << 16)
               : static_cast<const float*>(x_row)[k];
    }
    if (kscale) v = __fmul_rn(v, kscale[k / kblock]);
    if (!is_nonfinite(v)) continue;
    const int w = weight_at(codes, format, n_chunks, R, k);
    if (w == 0) {
      if (kscale) nan = true;  // 0 * inf or 0 * NaN
      continue;
    }
    if (v != v) nan = true;
    else if ((v > 0.0f) == (w > 0)) pinf = true;
    else ninf = true;
  }
  if (nan || (pinf && ninf)) return __int_as_float(0x7fc00000);
  if (pinf) return __fmul_rn(__int_as_float(0x7f800000), scale);
  if (ninf) return __fmul_rn(__int_as_float(0xff800000), scale);
  return y_finite;
}
#endif

// Per-context device workspace (grown on demand, freed with the context).
struct Workspace {
  void* ptr = nullptr;
  size_t bytes = 0;
};

}  // namespace ft

struct ft_ctx {
  int device = 0;
  int num_sms = 0;
  ft::Workspace ws;
  cudaStream_t host_stream = nullptr;  // used by the synchronous host-buffer calls
  ft::Workspace io;                    // device staging for the host-buffer calls
  ft::Workspace hio;                   // pinned host staging for pageable host buffers
  void* hio_dev = nullptr;             // device mapping of hio.ptr (null if not mapped)
  ft::Workspace zs;                    // zero-initialised scratch (split-K sums, tickets)
  int* err_word = nullptr;             // device word set by a kernel whose bounded wait gave up
  int* na_err = nullptr;               // the allocation-free entry point's static error word,
                                       // once this context has used that entry point (sticky)
};

struct ft_weight {
  int device = 0;
  int format = 0;             // 0: dense 2-bit (T128 tiles), 1: 2:4 sparse (mma.sp operand form)
  int64_t rows = 0, cols = 0;
  int64_t n_tiles = 0, n_chunks = 0;
  uint8_t* codes = nullptr;   // n_tiles*n_chunks blocks of 4096 (dense) or 3072 (sparse) bytes
  float* row_scales = nullptr;  // [n_tiles*128], zero on padding rows
};

namespace ft {
// Ensures ctx->ws holds at least `bytes` (must not be called during stream
// capture; it may cudaMalloc).  Returns FT_OK or a status.
int workspace_reserve(ft_ctx* ctx, size_t bytes, cudaStream_t stream);
// Same for ctx->zs; new memory is zeroed on `stream`.  Kernels that use it
// leave it zeroed again when they finish.
int zero_scratch_reserve(ft_ctx* ctx, size_t bytes, cudaStream_t stream);

// Kernels launched by ft_api.cu (defined in ft_dense.cu).
int launch_repack_u8(const uint8_t* packed, int64_t rows, int64_t cols, ft_weight* w,
                     cudaStream_t s);
int launch_repack_u32(const uint32_t* words, int64_t rows, int64_t cols, ft_weight* w,
                      cudaStream_t s);
// 2:4 sparse repack from the reference host layout (patterns + signs) or from
// the WGSL layout (5-bit groups, 6 per u32).
int launch_repack_sparse_host(const uint8_t* patterns, const uint8_t* signs, int64_t rows,
                              int64_t cols, ft_weight* w, cudaStream_t s);
int launch_repack_sparse_wgsl(const uint32_t* words, int64_t rows, int64_t cols, ft_weight* w,
                              cudaStream_t s);
int launch_quantize_i8(const void* x, bool bf16, int64_t seq, int64_t cols, int8_t* q, float* sx,
                       cudaStream_t s);
// Quantizes a row-major [w->rows, w->cols] fp32/bf16 device matrix into w's
// codes with alpha = w->row_scales[row] (mode 0 absmean rule, 1 STE rule).
int launch_quantize_pack(const void* src, bool bf16, int mode, ft_weight* w, cudaStream_t s);
int launch_fill_scales(ft_weight* w, float alpha, cudaStream_t s);
// w's codes as the reference pack_ternary byte stream ((rows*cols+3)/4 bytes).
int launch_export_u8(const ft_weight* w, uint8_t* out, cudaStream_t s);
// *acc += sum |src[i]| in f64 (acc: device double).
int launch_abs_sum(const void* src, bool bf16, int64_t n, double* acc, cudaStream_t s);
// Absmean scale of quantize_ternary (src/model/ternary.rs:36-45): sequential
// fp32 sum of |w| in element order, (sum / n) / ABSMEAN_NORM, 1 when the sum
// is not positive.  Host code.
float host_absmean_alpha(const float* w, int64_t n);
int alloc_weight(ft_ctx* ctx, int64_t rows, int64_t cols, ft_weight** out, int format = 0);
// Tensor-core path (ft_tc.cu).  xkind: 0 f32, 1 bf16, 2 int8 codes (then sx
// is the per-token scale).
int launch_tc_matmul(ft_ctx* ctx, const ft_weight* w, int64_t seq, const void* x, int xkind,
                     const float* sx, float* y, cudaStream_t s);
// Group of up to 64 independent problems (same seq and activation kind) in
// one persistent launch; identical activation pointers share one operand.
// digits: fixed-point digits per fp32/bf16 token (kDigitsExact or kDigitsMoE;
// 0 = kDigitsExact); ignored for int8 codes.
// kscale/kblock (fp32/bf16 only): one scale per kblock columns, folded into
// the activations (the blocked matmul); applies to every problem of the group.
// act (fp32 only): the activations are the outputs of a gate/up weight with
// interleaved 16-row m-blocks, rows of ldx floats; the operand's element k is
// then expert_act(x[32 (k/16) + k%16], x[that + 16], act) (1 SwiGLU, 2 GeLU),
// so the MoE's activation needs no pass of its own.
int launch_tc_grouped(ft_ctx* ctx, int n, const ft_weight* const* ws, int64_t seq,
                      const void* const* xs, int xkind, const float* const* sxs, float* const* ys,
                      const int64_t* ldys, cudaStream_t s, const int64_t* seqs = nullptr,
                      int digits = 0, const float* kscale = nullptr, int64_t kblock = 1,
                      int act = 0, int64_t ldx = 0);
// Decode-shape kernel (ft_gemv.cu): dense problems whose activations fit 16
// operand columns; the kernel builds its activation operand itself.
constexpr int kGemvMaxSmem = 200 * 1024;
struct GvLaunchProblem {
  const uint8_t* codes;
  const float* row_scales;
  int64_t rows, n_chunks;
  const void* x;  // [seq, K] activations (f32, bf16 or int8 codes)
  int64_t K, seq;
  const float* sx;  // int8 mode: per-token scale
  float* y;
  int64_t ldy;
  const float* kscale = nullptr;  // fp32 mode: column-block scales (blocked matmul), or null
  int64_t kblock = 1;             // columns per block scale
  int act = 0;                    // x is interleaved gate/up rows (see launch_tc_grouped)
  int64_t ldx = 0;                // elements per activation row (0: K)
};
// Digits per fp32/bf16 token on the decode kernel for a requested count
// (8 when more than 4 are asked for, else 4); 1 for int8 codes.
int gemv_digits(int xkind, int digits);
bool gemv_fits(const ft_weight* w, int64_t seq, int xkind, int digits);
// All problems of one launch have the same weight format (sparse: 2:4).
int launch_gemv(ft_ctx* ctx, int nprob, const GvLaunchProblem* probs, int xkind, bool sparse,
                int digits, cudaStream_t s);
int launch_wgsl_op(const uint32_t* words, const float* scales, const float* x, float* y,
                   uint32_t seq, uint32_t in_cols, uint32_t out_rows, cudaStream_t s);
}  // namespace ft
