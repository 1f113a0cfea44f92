// C ABI of libferris_ternary.so: context, errors, weight upload and the
// dense entry points.  Declarations and reference citations are in
// include/ferris_ternary.h.
#include <cstdlib>
#include <cstring>
#include <new>
#include <vector>

#include "ft_internal.cuh"

namespace ft {

static thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

int fail(int status, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

int workspace_reserve(ft_ctx* ctx, size_t bytes, cudaStream_t stream) {
  if (ctx->ws.bytes >= bytes) return FT_OK;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (stream != nullptr) cudaStreamIsCapturing(stream, &cs);
  FT_CHECK(cs == cudaStreamCaptureStatusNone, FT_ERR_UNSUPPORTED,
           "workspace must grow to %zu bytes but the stream is being captured; run the call "
           "once before capture",
           bytes);
  // Growing frees the old buffer: wait for work that may still read it.
  if (ctx->ws.ptr) {
    FT_CUDA(cudaDeviceSynchronize());
    FT_CUDA(cudaFree(ctx->ws.ptr));
    ctx->ws.ptr = nullptr;
    ctx->ws.bytes = 0;
  }
  size_t grow = bytes + bytes / 4 + (1 << 20);
  FT_CUDA(cudaMalloc(&ctx->ws.ptr, grow));
  ctx->ws.bytes = grow;
  return FT_OK;
}

int zero_scratch_reserve(ft_ctx* ctx, size_t bytes, cudaStream_t stream) {
  if (ctx->zs.bytes >= bytes) return FT_OK;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (stream != nullptr) cudaStreamIsCapturing(stream, &cs);
  FT_CHECK(cs == cudaStreamCaptureStatusNone, FT_ERR_UNSUPPORTED,
           "scratch must grow to %zu bytes but the stream is being captured; run the call "
           "once before capture",
           bytes);
  if (ctx->zs.ptr) {
    FT_CUDA(cudaDeviceSynchronize());
    FT_CUDA(cudaFree(ctx->zs.ptr));
    ctx->zs.ptr = nullptr;
    ctx->zs.bytes = 0;
  }
  size_t grow = bytes + bytes / 4 + (1 << 20);
  FT_CUDA(cudaMalloc(&ctx->zs.ptr, grow));
  ctx->zs.bytes = grow;
  FT_CUDA(cudaMemsetAsync(ctx->zs.ptr, 0, grow, stream));
  return FT_OK;
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

int alloc_weight(ft_ctx* ctx, int64_t rows, int64_t cols, ft_weight** out, int format) {
  FT_CHECK(ctx && out, FT_ERR_SHAPE, "null argument");
  FT_CHECK(rows > 0 && cols > 0, FT_ERR_SHAPE, "weight shape [%lld, %lld] must be positive",
           (long long)rows, (long long)cols);
  ft_weight* w = new (std::nothrow) ft_weight();
  FT_CHECK(w, FT_ERR_OOM, "host allocation failed");
  w->device = ctx->device;
  w->format = format;
  w->rows = rows;
  w->cols = cols;
  w->n_tiles = ceil_div(rows, kTileRows);
  w->n_chunks = ceil_div(cols, kChunkK);
  size_t code_bytes =
      (size_t)(w->n_tiles * w->n_chunks) * (format == 1 ? kSparseBlockBytes : kBlockBytes);
  size_t scale_bytes = (size_t)(w->n_tiles * kTileRows) * sizeof(float);
  cudaError_t e = cudaMalloc(&w->codes, code_bytes);
  if (e == cudaSuccess) e = cudaMalloc(&w->row_scales, scale_bytes);
  if (e != cudaSuccess) {
    if (w->codes) cudaFree(w->codes);
    delete w;
    return fail(e == cudaErrorMemoryAllocation ? FT_ERR_OOM : FT_ERR_GPU,
                "weight allocation (%zu bytes) failed: %s", code_bytes + scale_bytes,
                cudaGetErrorString(e));
  }
  *out = w;
  return FT_OK;
}

float host_absmean_alpha(const float* w, int64_t n) {
  // Iterator::sum over f32 is a sequential left fold; the compiler keeps this
  // order (no reassociation without fast-math).
  float sum_abs = 0.0f;
  for (int64_t i = 0; i < n; ++i) sum_abs += fabsf(w[i]);
  const float ABSMEAN_NORM = 0.7978845608f;  // src/model/ternary.rs:15
  return sum_abs > 0.0f ? (sum_abs / (float)n) / ABSMEAN_NORM : 1.0f;
}

static int finish_scales(ft_weight* w, const float* scales, bool host, cudaStream_t s) {
  size_t scale_bytes = (size_t)(w->n_tiles * kTileRows) * sizeof(float);
  FT_CUDA(cudaMemsetAsync(w->row_scales, 0, scale_bytes, s));
  FT_CUDA(cudaMemcpyAsync(w->row_scales, scales, (size_t)w->rows * sizeof(float),
                          host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice, s));
  return FT_OK;
}

}  // namespace ft

using namespace ft;

extern "C" {

const char* ft_version(void) { return "ferris-ternary-b200 0.1.0 (sm_100a)"; }

const char* ft_last_error_string(void) { return g_last_error.c_str(); }

uint64_t ft_launch_counter(void) { return g_launches.load(std::memory_order_relaxed); }

int ft_ctx_create(int device, ft_ctx** out) {
  FT_CHECK(out, FT_ERR_SHAPE, "null out pointer");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  FT_CHECK(e == cudaSuccess && n > 0, FT_ERR_DEVICE, "no CUDA device available (%s)",
           cudaGetErrorString(e));
  FT_CHECK(device >= 0 && device < n, FT_ERR_DEVICE, "device %d out of range [0, %d)", device, n);
  cudaDeviceProp prop;
  FT_CUDA(cudaGetDeviceProperties(&prop, device));
  FT_CHECK(prop.major == 10 && prop.minor == 0, FT_ERR_UNSUPPORTED,
           "device %d is sm_%d%d; this library is built for sm_100a (B200)", device, prop.major,
           prop.minor);
  DeviceGuard g(device);
  ft_ctx* c = new (std::nothrow) ft_ctx();
  FT_CHECK(c, FT_ERR_OOM, "host allocation failed");
  c->device = device;
  c->num_sms = prop.multiProcessorCount;
  cudaError_t se = cudaStreamCreateWithFlags(&c->host_stream, cudaStreamNonBlocking);
  if (se != cudaSuccess) {
    delete c;
    return fail(FT_ERR_GPU, "stream creation failed: %s", cudaGetErrorString(se));
  }
  se = cudaMalloc(&c->err_word, 256);
  if (se == cudaSuccess) se = cudaMemset(c->err_word, 0, 256);
  if (se != cudaSuccess) {
    cudaStreamDestroy(c->host_stream);
    if (c->err_word) cudaFree(c->err_word);
    delete c;
    return fail(FT_ERR_GPU, "error word allocation failed: %s", cudaGetErrorString(se));
  }
  *out = c;
  return FT_OK;
}

int ft_ctx_destroy(ft_ctx* ctx) {
  if (!ctx) return FT_OK;
  DeviceGuard g(ctx->device);
  cudaDeviceSynchronize();
  if (ctx->ws.ptr) cudaFree(ctx->ws.ptr);
  if (ctx->io.ptr) cudaFree(ctx->io.ptr);
  if (ctx->hio.ptr) cudaFreeHost(ctx->hio.ptr);
  if (ctx->zs.ptr) cudaFree(ctx->zs.ptr);
  if (ctx->err_word) cudaFree(ctx->err_word);
  if (ctx->host_stream) cudaStreamDestroy(ctx->host_stream);
  delete ctx;
  return FT_OK;
}

int ft_weight_upload_packed_u8(ft_ctx* ctx, const uint8_t* packed_host, int64_t rows,
                               int64_t cols, const float* row_scales_host, ft_weight** out) {
  FT_CHECK(packed_host && row_scales_host, FT_ERR_SHAPE, "null host buffer");
  DeviceGuard g(ctx ? ctx->device : 0);
  ft_weight* w = nullptr;
  int st = alloc_weight(ctx, rows, cols, &w);
  if (st != FT_OK) return st;
  size_t nbytes = (size_t)((rows * cols + 3) / 4);
  uint8_t* staging = nullptr;
  cudaStream_t s = ctx->host_stream;
  cudaError_t e = cudaMalloc(&staging, nbytes);
  if (e == cudaSuccess) e = cudaMemcpyAsync(staging, packed_host, nbytes, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) st = launch_repack_u8(staging, rows, cols, w, s);
  if (e == cudaSuccess && st == FT_OK) st = finish_scales(w, row_scales_host, true, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (staging) cudaFree(staging);
  if (e != cudaSuccess || st != FT_OK) {
    ft_weight_destroy(w);
    if (e != cudaSuccess) return fail(FT_ERR_GPU, "weight upload failed: %s", cudaGetErrorString(e));
    return st;
  }
  *out = w;
  return FT_OK;
}

int ft_weight_upload_packed_u32(ft_ctx* ctx, const uint32_t* words_host, int64_t rows,
                                int64_t cols, const float* row_scales_host, ft_weight** out) {
  FT_CHECK(words_host && row_scales_host, FT_ERR_SHAPE, "null host buffer");
  DeviceGuard g(ctx ? ctx->device : 0);
  ft_weight* w = nullptr;
  int st = alloc_weight(ctx, rows, cols, &w);
  if (st != FT_OK) return st;
  size_t nbytes = (size_t)rows * (size_t)ceil_div(cols, 16) * 4;
  uint32_t* staging = nullptr;
  cudaStream_t s = ctx->host_stream;
  cudaError_t e = cudaMalloc(&staging, nbytes);
  if (e == cudaSuccess) e = cudaMemcpyAsync(staging, words_host, nbytes, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) st = launch_repack_u32(staging, rows, cols, w, s);
  if (e == cudaSuccess && st == FT_OK) st = finish_scales(w, row_scales_host, true, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (staging) cudaFree(staging);
  if (e != cudaSuccess || st != FT_OK) {
    ft_weight_destroy(w);
    if (e != cudaSuccess) return fail(FT_ERR_GPU, "weight upload failed: %s", cudaGetErrorString(e));
    return st;
  }
  *out = w;
  return FT_OK;
}

int ft_weight_from_device_u32(ft_ctx* ctx, const uint32_t* words_dev, int64_t rows, int64_t cols,
                              const float* row_scales_dev, void* stream, ft_weight** out) {
  FT_CHECK(words_dev && row_scales_dev, FT_ERR_SHAPE, "null device buffer");
  DeviceGuard g(ctx ? ctx->device : 0);
  ft_weight* w = nullptr;
  int st = alloc_weight(ctx, rows, cols, &w);
  if (st != FT_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = launch_repack_u32(words_dev, rows, cols, w, s);
  if (st == FT_OK) st = finish_scales(w, row_scales_dev, false, s);
  if (st != FT_OK) {
    cudaStreamSynchronize(s);
    ft_weight_destroy(w);
    return st;
  }
  *out = w;
  return FT_OK;
}

int ft_sparse_upload_host(ft_ctx* ctx, const uint8_t* patterns_host, const uint8_t* signs_host,
                          int64_t rows, int64_t cols, const float* row_scales_host,
                          ft_weight** out) {
  FT_CHECK(patterns_host && signs_host && row_scales_host, FT_ERR_SHAPE, "null host buffer");
  FT_CHECK(cols > 0 && cols % 4 == 0, FT_ERR_SHAPE,
           "cols must be a positive multiple of 4 for 2:4 sparsity, got %lld", (long long)cols);
  DeviceGuard g(ctx ? ctx->device : 0);
  ft_weight* w = nullptr;
  int st = alloc_weight(ctx, rows, cols, &w, 1);
  if (st != FT_OK) return st;
  const size_t ng = (size_t)(rows * cols / 4);
  const size_t pb = (ng + 1) / 2, sb = (ng + 3) / 4;
  uint8_t* staging = nullptr;
  cudaStream_t s = ctx->host_stream;
  cudaError_t e = cudaMalloc(&staging, pb + sb);
  if (e == cudaSuccess) e = cudaMemcpyAsync(staging, patterns_host, pb, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(staging + pb, signs_host, sb, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) st = launch_repack_sparse_host(staging, staging + pb, rows, cols, w, s);
  if (e == cudaSuccess && st == FT_OK) st = finish_scales(w, row_scales_host, true, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (staging) cudaFree(staging);
  if (e != cudaSuccess || st != FT_OK) {
    ft_weight_destroy(w);
    if (e != cudaSuccess) return fail(FT_ERR_GPU, "sparse upload failed: %s", cudaGetErrorString(e));
    return st;
  }
  *out = w;
  return FT_OK;
}

int ft_sparse_upload_wgsl(ft_ctx* ctx, const uint32_t* words_host, int64_t rows, int64_t cols,
                          const float* row_scales_host, ft_weight** out) {
  FT_CHECK(words_host && row_scales_host, FT_ERR_SHAPE, "null host buffer");
  FT_CHECK(cols > 0 && cols % 4 == 0, FT_ERR_SHAPE,
           "cols must be a positive multiple of 4 for 2:4 sparsity, got %lld", (long long)cols);
  DeviceGuard g(ctx ? ctx->device : 0);
  ft_weight* w = nullptr;
  int st = alloc_weight(ctx, rows, cols, &w, 1);
  if (st != FT_OK) return st;
  const size_t nbytes = (size_t)rows * (size_t)ceil_div(cols / 4, 6) * 4;
  uint32_t* staging = nullptr;
  cudaStream_t s = ctx->host_stream;
  cudaError_t e = cudaMalloc(&staging, nbytes);
  if (e == cudaSuccess) e = cudaMemcpyAsync(staging, words_host, nbytes, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) st = launch_repack_sparse_wgsl(staging, rows, cols, w, s);
  if (e == cudaSuccess && st == FT_OK) st = finish_scales(w, row_scales_host, true, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (staging) cudaFree(staging);
  if (e != cudaSuccess || st != FT_OK) {
    ft_weight_destroy(w);
    if (e != cudaSuccess) return fail(FT_ERR_GPU, "sparse upload failed: %s", cudaGetErrorString(e));
    return st;
  }
  *out = w;
  return FT_OK;
}

int ft_gpu_sparse_ternary_matmul(ft_ctx* ctx, const uint32_t* sparse_words_host, float scale,
                                 const float* input_host, size_t seq_len, size_t in_cols,
                                 size_t out_rows, float* output_host) {
  FT_CHECK(ctx, FT_ERR_SHAPE, "null context");
  FT_CHECK(sparse_words_host && input_host && output_host, FT_ERR_SHAPE, "null host buffer");
  if (seq_len == 0 || out_rows == 0) return FT_OK;
  std::vector<float> scales(out_rows, scale);  // the reference passes one global scale
  ft_weight* w = nullptr;
  int st = ft_sparse_upload_wgsl(ctx, sparse_words_host, (int64_t)out_rows, (int64_t)in_cols,
                                 scales.data(), &w);
  if (st != FT_OK) return st;
  st = ft_gpu_ternary_matmul_vram(ctx, w, input_host, seq_len, in_cols, out_rows, output_host);
  ft_weight_destroy(w);
  return st;
}

int ft_weight_destroy(ft_weight* w) {
  if (!w) return FT_OK;
  DeviceGuard g(w->device);
  if (w->codes) cudaFree(w->codes);
  if (w->row_scales) cudaFree(w->row_scales);
  delete w;
  return FT_OK;
}

int ft_weight_info(const ft_weight* w, int64_t* rows, int64_t* cols, int64_t* device_bytes) {
  FT_CHECK(w, FT_ERR_SHAPE, "null weight");
  if (rows) *rows = w->rows;
  if (cols) *cols = w->cols;
  if (device_bytes)
    *device_bytes = w->n_tiles * w->n_chunks * (w->format == 1 ? kSparseBlockBytes : kBlockBytes) +
                    w->n_tiles * kTileRows * 4;
  return FT_OK;
}

int ft_ternary_matmul_f32(ft_ctx* ctx, const ft_weight* w, int64_t seq, const float* x_dev,
                          float* y_dev, void* stream) {
  FT_CHECK(ctx && w, FT_ERR_SHAPE, "null context or weight");
  FT_CHECK(seq >= 0, FT_ERR_SHAPE, "seq must be >= 0");
  FT_CHECK(seq == 0 || (x_dev && y_dev), FT_ERR_SHAPE, "null activation/output pointer");
  FT_CHECK(w->device == ctx->device, FT_ERR_DEVICE, "weight lives on device %d, context on %d",
           w->device, ctx->device);
  DeviceGuard g(ctx->device);
  return launch_tc_matmul(ctx, w, seq, x_dev, 0, nullptr, y_dev, static_cast<cudaStream_t>(stream));
}

int ft_ternary_matmul_bf16(ft_ctx* ctx, const ft_weight* w, int64_t seq, const uint16_t* x_dev,
                           float* y_dev, void* stream) {
  FT_CHECK(ctx && w, FT_ERR_SHAPE, "null context or weight");
  FT_CHECK(seq >= 0, FT_ERR_SHAPE, "seq must be >= 0");
  FT_CHECK(seq == 0 || (x_dev && y_dev), FT_ERR_SHAPE, "null activation/output pointer");
  FT_CHECK(w->device == ctx->device, FT_ERR_DEVICE, "weight lives on device %d, context on %d",
           w->device, ctx->device);
  DeviceGuard g(ctx->device);
  return launch_tc_matmul(ctx, w, seq, x_dev, 1, nullptr, y_dev, static_cast<cudaStream_t>(stream));
}

int ft_ternary_matmul_f32_grouped(ft_ctx* ctx, int n, const ft_weight* const* ws, int64_t seq,
                                  const float* const* xs_dev, float* const* ys_dev, void* stream) {
  FT_CHECK(ctx && ws && xs_dev && ys_dev, FT_ERR_SHAPE, "null argument");
  FT_CHECK(seq >= 0, FT_ERR_SHAPE, "seq must be >= 0");
  DeviceGuard g(ctx->device);
  return launch_tc_grouped(ctx, n, ws, seq, reinterpret_cast<const void* const*>(xs_dev), 0,
                           nullptr, ys_dev, nullptr, static_cast<cudaStream_t>(stream));
}

int ft_ternary_matmul_i8_grouped(ft_ctx* ctx, int n, const ft_weight* const* ws, int64_t seq,
                                 const int8_t* const* qs_dev, const float* const* sxs_dev,
                                 float* const* ys_dev, void* stream) {
  FT_CHECK(ctx && ws && qs_dev && sxs_dev && ys_dev, FT_ERR_SHAPE, "null argument");
  FT_CHECK(seq >= 0, FT_ERR_SHAPE, "seq must be >= 0");
  DeviceGuard g(ctx->device);
  return launch_tc_grouped(ctx, n, ws, seq, reinterpret_cast<const void* const*>(qs_dev), 2,
                           sxs_dev, ys_dev, nullptr, static_cast<cudaStream_t>(stream));
}

int ft_ctx_check(ft_ctx* ctx) {
  FT_CHECK(ctx, FT_ERR_SHAPE, "null context");
  DeviceGuard g(ctx->device);
  FT_CUDA(cudaDeviceSynchronize());
  int* words[2] = {ctx->err_word, ctx->na_err};
  for (int* wd : words) {
    if (!wd) continue;
    int code = 0;
    FT_CUDA(cudaMemcpy(&code, wd, sizeof(int), cudaMemcpyDeviceToHost));
    if (code != 0) {
      int zero = 0;
      FT_CUDA(cudaMemcpy(wd, &zero, sizeof(int), cudaMemcpyHostToDevice));
      if (code >= 1000)
        return fail(FT_ERR_SHAPE, "a kernel met an out-of-range page or position (site %d) "
                    "and skipped it; results of that launch are invalid", code);
      return fail(FT_ERR_TIMEOUT, "a kernel's bounded wait gave up (site %d); results of that "
                  "launch are invalid", code);
    }
  }
  return FT_OK;
}

int ft_quantize_absmax_i8_f32(ft_ctx* ctx, int64_t seq, int64_t cols, const float* x_dev,
                              int8_t* q_dev, float* sx_dev, void* stream) {
  FT_CHECK(ctx, FT_ERR_SHAPE, "null context");
  FT_CHECK(seq >= 0 && cols > 0, FT_ERR_SHAPE, "bad shape [%lld, %lld]", (long long)seq,
           (long long)cols);
  DeviceGuard g(ctx->device);
  return launch_quantize_i8(x_dev, false, seq, cols, q_dev, sx_dev, static_cast<cudaStream_t>(stream));
}

int ft_quantize_absmax_i8_bf16(ft_ctx* ctx, int64_t seq, int64_t cols, const uint16_t* x_dev,
                               int8_t* q_dev, float* sx_dev, void* stream) {
  FT_CHECK(ctx, FT_ERR_SHAPE, "null context");
  FT_CHECK(seq >= 0 && cols > 0, FT_ERR_SHAPE, "bad shape [%lld, %lld]", (long long)seq,
           (long long)cols);
  DeviceGuard g(ctx->device);
  return launch_quantize_i8(x_dev, true, seq, cols, q_dev, sx_dev, static_cast<cudaStream_t>(stream));
}

int ft_ternary_matmul_i8(ft_ctx* ctx, const ft_weight* w, int64_t seq, const int8_t* q_dev,
                         const float* sx_dev, float* y_dev, void* stream) {
  FT_CHECK(ctx && w, FT_ERR_SHAPE, "null context or weight");
  FT_CHECK(seq >= 0, FT_ERR_SHAPE, "seq must be >= 0");
  FT_CHECK(seq == 0 || (q_dev && sx_dev && y_dev), FT_ERR_SHAPE, "null activation/output pointer");
  FT_CHECK(w->device == ctx->device, FT_ERR_DEVICE, "weight lives on device %d, context on %d",
           w->device, ctx->device);
  DeviceGuard g(ctx->device);
  return launch_tc_matmul(ctx, w, seq, q_dev, 2, sx_dev, y_dev, static_cast<cudaStream_t>(stream));
}

int ft_ternary_matmul_op_dispatch(ft_ctx* ctx, const uint32_t* ternary_dev,
                                  const float* scales_dev, const float* input_dev,
                                  float* output_dev, uint32_t seq_len, uint32_t in_cols,
                                  uint32_t out_rows, void* stream) {
  FT_CHECK(ctx, FT_ERR_SHAPE, "null context");
  FT_CHECK(ternary_dev && scales_dev && input_dev && output_dev, FT_ERR_SHAPE, "null buffer");
  DeviceGuard g(ctx->device);
  return launch_wgsl_op(ternary_dev, scales_dev, input_dev, output_dev, seq_len, in_cols, out_rows,
                        static_cast<cudaStream_t>(stream));
}

int ft_gpu_ternary_matmul(ft_ctx* ctx, const uint32_t* packed_weights_host,
                          const float* scales_host, const float* input_host, size_t seq_len,
                          size_t in_cols, size_t out_rows, float* output_host) {
  FT_CHECK(ctx, FT_ERR_SHAPE, "null context");
  FT_CHECK(packed_weights_host && scales_host && input_host && output_host, FT_ERR_SHAPE,
           "null host buffer");
  if (seq_len == 0 || out_rows == 0) return FT_OK;
  ft_weight* w = nullptr;
  int st = ft_weight_upload_packed_u32(ctx, packed_weights_host, (int64_t)out_rows,
                                       (int64_t)in_cols, scales_host, &w);
  if (st != FT_OK) return st;
  st = ft_gpu_ternary_matmul_vram(ctx, w, input_host, seq_len, in_cols, out_rows, output_host);
  ft_weight_destroy(w);
  return st;
}

// Outputs up to this size are written by the kernel into mapped pinned memory.
constexpr size_t kDirectOutBytes = 256 * 1024;

int ft_gpu_ternary_matmul_vram(ft_ctx* ctx, const ft_weight* w, const float* input_host,
                               size_t seq_len, size_t in_cols, size_t out_rows,
                               float* output_host) {
  FT_CHECK(ctx && w, FT_ERR_SHAPE, "null context or weight");
  FT_CHECK(input_host && output_host, FT_ERR_SHAPE, "null host buffer");
  FT_CHECK((int64_t)in_cols == w->cols && (int64_t)out_rows == w->rows, FT_ERR_SHAPE,
           "in_cols x out_rows = %zu x %zu, the weight is [%lld, %lld]", in_cols, out_rows,
           (long long)w->rows, (long long)w->cols);
  if (seq_len == 0) return FT_OK;
  DeviceGuard g(ctx->device);
  cudaStream_t s = ctx->host_stream;
  const size_t in_raw = seq_len * (size_t)w->cols * sizeof(float);
  const size_t in_bytes = round_up(in_raw, 256);
  const size_t out_bytes = seq_len * (size_t)w->rows * sizeof(float);
  // Device staging is kept in the context and only grows (no per-call malloc).
  if (ctx->io.bytes < in_bytes + out_bytes) {
    FT_CUDA(cudaStreamSynchronize(s));
    if (ctx->io.ptr) FT_CUDA(cudaFree(ctx->io.ptr));
    ctx->io.ptr = nullptr;
    ctx->io.bytes = 0;
    FT_CUDA(cudaMalloc(&ctx->io.ptr, in_bytes + out_bytes));
    ctx->io.bytes = in_bytes + out_bytes;
  }
  // Pageable host buffers go through a pinned staging buffer of the context
  // (a host memcpy each way), so the copies stay asynchronous DMA transfers.
  cudaPointerAttributes ai, ao;
  const bool in_pinned = cudaPointerGetAttributes(&ai, input_host) == cudaSuccess &&
                         ai.type == cudaMemoryTypeHost;
  const bool out_pinned = cudaPointerGetAttributes(&ao, output_host) == cudaSuccess &&
                          ao.type == cudaMemoryTypeHost;
  cudaGetLastError();  // an unregistered pointer is not an error here
  const size_t need = (in_pinned ? 0 : in_bytes) + (out_pinned ? 0 : out_bytes);
  if (need > 0 && ctx->hio.bytes < need) {
    FT_CUDA(cudaStreamSynchronize(s));
    if (ctx->hio.ptr) FT_CUDA(cudaFreeHost(ctx->hio.ptr));
    ctx->hio.ptr = nullptr;
    ctx->hio_dev = nullptr;
    ctx->hio.bytes = 0;
    FT_CUDA(cudaHostAlloc(&ctx->hio.ptr, need, cudaHostAllocDefault));
    ctx->hio.bytes = need;
    if (cudaHostGetDevicePointer(&ctx->hio_dev, ctx->hio.ptr, 0) != cudaSuccess) {
      ctx->hio_dev = nullptr;
      cudaGetLastError();  // not mapped: outputs are copied back
    }
  }
  const float* src = input_host;
  if (!in_pinned) {
    std::memcpy(ctx->hio.ptr, input_host, in_raw);
    src = static_cast<const float*>(ctx->hio.ptr);
  }
  float* dst = out_pinned ? output_host
                          : reinterpret_cast<float*>(static_cast<char*>(ctx->hio.ptr) +
                                                     (in_pinned ? 0 : in_bytes));
  float* dx = static_cast<float*>(ctx->io.ptr);
  float* dy = reinterpret_cast<float*>(static_cast<char*>(ctx->io.ptr) + in_bytes);
  // A small output is written by the kernel straight into the pinned host
  // buffer through its device mapping: no device staging and no copy back.
  float* ky = dy;
  if (out_bytes <= kDirectOutBytes) {
    void* mapped = nullptr;
    if (out_pinned && dst == output_host) {
      mapped = ao.devicePointer;
    } else if (ctx->hio_dev) {
      mapped = static_cast<char*>(ctx->hio_dev) +
               (reinterpret_cast<char*>(dst) - static_cast<char*>(ctx->hio.ptr));
    }
    if (mapped) ky = static_cast<float*>(mapped);
  }
  FT_CUDA(cudaMemcpyAsync(dx, src, in_raw, cudaMemcpyHostToDevice, s));
  int st = launch_tc_matmul(ctx, w, (int64_t)seq_len, dx, 0, nullptr, ky, s);
  if (st != FT_OK) {
    cudaStreamSynchronize(s);
    return st;
  }
  if (ky == dy) FT_CUDA(cudaMemcpyAsync(dst, dy, out_bytes, cudaMemcpyDeviceToHost, s));
  FT_CUDA(cudaStreamSynchronize(s));
  if (!out_pinned) std::memcpy(output_host, dst, out_bytes);
  return FT_OK;
}

// ---- block-scale, index-list and fp32-ingestion entry points ------------

int ft_ternary_matmul_blocked_f32(ft_ctx* ctx, const ft_weight* w, int64_t seq, const float* x_dev,
                                  const float* block_scales_dev, int64_t block_size, float* y_dev,
                                  void* stream) {
  FT_CHECK(ctx && w, FT_ERR_SHAPE, "null context or weight");
  FT_CHECK(seq >= 0, FT_ERR_SHAPE, "seq must be >= 0");
  FT_CHECK(block_size >= 1, FT_ERR_SHAPE, "block_size must be >= 1");
  FT_CHECK(seq == 0 || (x_dev && y_dev && block_scales_dev), FT_ERR_SHAPE, "null pointer");
  FT_CHECK(w->device == ctx->device, FT_ERR_DEVICE, "weight lives on device %d, context on %d",
           w->device, ctx->device);
  if (seq == 0) return FT_OK;
  DeviceGuard g(ctx->device);
  const ft_weight* ws[1] = {w};
  const void* xs[1] = {x_dev};
  float* ys[1] = {y_dev};
  return launch_tc_grouped(ctx, 1, ws, seq, xs, 0, nullptr, ys, nullptr,
                           static_cast<cudaStream_t>(stream), nullptr, 0, block_scales_dev,
                           block_size);
}

int ft_weight_upload_index_lists(ft_ctx* ctx, int64_t rows, int64_t cols, const int64_t* pos_off,
                                 const int64_t* pos_idx, const int64_t* neg_off,
                                 const int64_t* neg_idx, const float* row_scales_host,
                                 ft_weight** out) {
  FT_CHECK(ctx && out && pos_off && neg_off && row_scales_host, FT_ERR_SHAPE, "null argument");
  FT_CHECK(rows > 0 && cols > 0, FT_ERR_SHAPE, "shape [%lld, %lld] must be positive",
           (long long)rows, (long long)cols);
  FT_CHECK(pos_off[0] == 0 && neg_off[0] == 0, FT_ERR_SHAPE, "offsets must start at 0");
  FT_CHECK((pos_off[rows] == 0 || pos_idx) && (neg_off[rows] == 0 || neg_idx), FT_ERR_SHAPE,
           "null index array");
  // The flat pack_ternary stream: all zero weights (code 1), then the lists'
  // columns set to +1 (code 2) or -1 (code 0).  Each row's lists must be
  // strictly increasing, in range, and disjoint (what ternary_sparse_indices
  // produces): a 2-bit code holds one weight per position.
  std::vector<uint8_t> packed((size_t)((rows * cols + 3) / 4), 0x55);
  for (int64_t r = 0; r < rows; ++r) {
    FT_CHECK(pos_off[r + 1] >= pos_off[r] && neg_off[r + 1] >= neg_off[r], FT_ERR_SHAPE,
             "row %lld: offsets decrease", (long long)r);
    for (int sign = 0; sign < 2; ++sign) {
      const int64_t* off = sign ? neg_off : pos_off;
      const int64_t* idx = sign ? neg_idx : pos_idx;
      int64_t last = -1;
      for (int64_t i = off[r]; i < off[r + 1]; ++i) {
        const int64_t j = idx[i];
        FT_CHECK(j > last && j < cols, FT_ERR_SHAPE,
                 "row %lld: column %lld out of range or out of order", (long long)r, (long long)j);
        last = j;
        const int64_t f = r * cols + j;
        uint8_t& byte = packed[(size_t)(f >> 2)];
        const int sh = (int)(f & 3) * 2;
        FT_CHECK(((byte >> sh) & 3) == 1, FT_ERR_SHAPE,
                 "row %lld: column %lld is in both the +1 and the -1 list", (long long)r,
                 (long long)j);
        byte = (uint8_t)((byte & ~(3 << sh)) | ((sign ? 0 : 2) << sh));
      }
    }
  }
  return ft_weight_upload_packed_u8(ctx, packed.data(), rows, cols, row_scales_host, out);
}

int ft_weight_quantize_f32(ft_ctx* ctx, const float* w_host, int64_t rows, int64_t cols,
                           float* alpha_out, ft_weight** out) {
  FT_CHECK(ctx && w_host && out, FT_ERR_SHAPE, "null argument");
  DeviceGuard g(ctx->device);
  ft_weight* w = nullptr;
  int st = alloc_weight(ctx, rows, cols, &w);
  if (st != FT_OK) return st;
  const float alpha = host_absmean_alpha(w_host, rows * cols);
  cudaStream_t s = ctx->host_stream;
  float* staging = nullptr;
  const size_t nbytes = (size_t)(rows * cols) * 4;
  cudaError_t e = cudaMalloc(&staging, nbytes);
  if (e == cudaSuccess) e = cudaMemcpyAsync(staging, w_host, nbytes, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) st = launch_fill_scales(w, alpha, s);
  if (e == cudaSuccess && st == FT_OK) st = launch_quantize_pack(staging, false, 0, w, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (staging) cudaFree(staging);
  if (e != cudaSuccess || st != FT_OK) {
    ft_weight_destroy(w);
    if (e != cudaSuccess) return fail(FT_ERR_GPU, "quantize upload failed: %s", cudaGetErrorString(e));
    return st;
  }
  if (alpha_out) *alpha_out = alpha;
  *out = w;
  return FT_OK;
}

int ft_weight_requantize(ft_ctx* ctx, ft_weight* w, const void* src_dev, int src_bf16, float alpha,
                         void* stream) {
  FT_CHECK(ctx && w && src_dev, FT_ERR_SHAPE, "null argument");
  FT_CHECK(w->format == 0, FT_ERR_UNSUPPORTED, "requantize needs a dense weight");
  FT_CHECK(w->device == ctx->device, FT_ERR_DEVICE, "weight lives on device %d, context on %d",
           w->device, ctx->device);
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int st = launch_fill_scales(w, alpha, s);
  if (st != FT_OK) return st;
  return launch_quantize_pack(src_dev, src_bf16 != 0, 1, w, s);
}

int ft_shadow_alpha(ft_ctx* ctx, int n, const void* const* src_dev, const int64_t* counts,
                    int src_bf16, float* alpha_out) {
  FT_CHECK(ctx && alpha_out && (n == 0 || (src_dev && counts)), FT_ERR_SHAPE, "null argument");
  FT_CHECK(n >= 0, FT_ERR_SHAPE, "negative buffer count");
  DeviceGuard g(ctx->device);
  int64_t total = 0;
  for (int i = 0; i < n; ++i) {
    FT_CHECK(counts[i] >= 0 && (counts[i] == 0 || src_dev[i]), FT_ERR_SHAPE, "bad buffer %d", i);
    total += counts[i];
  }
  if (total == 0) return FT_OK;  // the reference keeps the previous alpha
  cudaStream_t s = ctx->host_stream;
  double* acc = nullptr;
  FT_CUDA(cudaMalloc(&acc, sizeof(double)));
  cudaError_t e = cudaMemsetAsync(acc, 0, sizeof(double), s);
  int st = FT_OK;
  for (int i = 0; i < n && e == cudaSuccess && st == FT_OK; ++i)
    st = launch_abs_sum(src_dev[i], src_bf16 != 0, counts[i], acc, s);
  double sum = 0.0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&sum, acc, sizeof(double), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  cudaFree(acc);
  if (st != FT_OK) return st;
  FT_CHECK(e == cudaSuccess, FT_ERR_GPU, "abs-sum failed: %s", cudaGetErrorString(e));
  *alpha_out = (float)(sum / (double)total);
  return FT_OK;
}

int ft_weight_export_packed_u8(ft_ctx* ctx, const ft_weight* w, uint8_t* packed_host) {
  FT_CHECK(ctx && w && packed_host, FT_ERR_SHAPE, "null argument");
  FT_CHECK(w->device == ctx->device, FT_ERR_DEVICE, "weight lives on device %d, context on %d",
           w->device, ctx->device);
  DeviceGuard g(ctx->device);
  cudaStream_t s = ctx->host_stream;
  const size_t nbytes = (size_t)((w->rows * w->cols + 3) / 4);
  uint8_t* staging = nullptr;
  FT_CUDA(cudaMalloc(&staging, nbytes));
  int st = launch_export_u8(w, staging, s);
  cudaError_t e = cudaSuccess;
  if (st == FT_OK) e = cudaMemcpyAsync(packed_host, staging, nbytes, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  cudaFree(staging);
  if (st != FT_OK) return st;
  FT_CHECK(e == cudaSuccess, FT_ERR_GPU, "export failed: %s", cudaGetErrorString(e));
  return FT_OK;
}

}  // extern "C"
