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
// 2:4 sparse block: each row's 32 groups of 4 codes as 5-bit group codes
// (pattern * 4 + signs, 24 = all-zero padding group), 20 bytes per row.
constexpr int kSparseBlockBytes = kTileRows * 20;      // 2560

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
  int format = 0;             // 0: dense 2-bit (T128 tiles), 1: 2:4 sparse (5-bit groups)
  int64_t rows = 0, cols = 0;
  int64_t n_tiles = 0, n_chunks = 0;
  uint8_t* codes = nullptr;   // n_tiles*n_chunks blocks of 4096 (dense) or 2560 (sparse) bytes
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
// Tensor-core path (ft_tc.cu).  xkind: 0 f32, 1 bf16, 2 int8 codes (then sx
// is the per-token scale).
int launch_tc_matmul(ft_ctx* ctx, const ft_weight* w, int64_t seq, const void* x, int xkind,
                     const float* sx, float* y, cudaStream_t s);
// Group of up to 64 independent problems (same seq and activation kind) in
// one persistent launch; identical activation pointers share one operand.
int launch_tc_grouped(ft_ctx* ctx, int n, const ft_weight* const* ws, int64_t seq,
                      const void* const* xs, int xkind, const float* const* sxs, float* const* ys,
                      const int64_t* ldys, cudaStream_t s, const int64_t* seqs = nullptr);
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
};
bool gemv_fits(const ft_weight* w, int64_t seq, int xkind);
// All problems of one launch have the same weight format (sparse: 2:4).
int launch_gemv(ft_ctx* ctx, int nprob, const GvLaunchProblem* probs, int xkind, bool sparse,
                cudaStream_t s);
int launch_wgsl_op(const uint32_t* words, const float* scales, const float* x, float* y,
                   uint32_t seq, uint32_t in_cols, uint32_t out_rows, cudaStream_t s);
}  // namespace ft
