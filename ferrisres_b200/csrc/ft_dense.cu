// Dense ternary kernels on CUDA cores: weight repack, int8 quantizer, the
// split-K fp32 / int8 matmuls over the tiled T128 layout, and the raw
// WGSL-layout op.  The tensor-core (tcgen05) path lives in ft_tc.cu.
#include "ft_internal.cuh"

namespace ft {
namespace {

// ---------------------------------------------------------------- repack --
// One thread per output u32 word of the tiled layout (see ft_internal.cuh).
template <bool kU32Src>
__global__ void repack_kernel(const void* __restrict__ src, int64_t rows, int64_t cols,
                              int64_t n_chunks, int64_t total_words, uint32_t* __restrict__ dst) {
  // one thread per output word; block = 1024 words = [m-block][lane][word i]
  int64_t gw = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gw >= total_words) return;
  int64_t block = gw >> 10;
  const int within = (int)(gw & 1023);
  const int mb = within >> 7, lane = (within >> 2) & 31, wi = within & 3;
  const int g = lane >> 2, r = lane & 3;
  int64_t tile = block / n_chunks, chunk = block % n_chunks;
  int64_t cp = (cols + 15) >> 4;
  uint32_t out = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      // code slot j of byte b = k-step j; the word picks the row half and k half
      const int64_t R = tile * kTileRows + 16 * mb + g + 8 * (wi & 1);
      const int64_t k = chunk * kChunkK + 32 * j + 16 * (wi >> 1) + 4 * r + b;
      uint32_t code = 1u;
      if (R < rows && k < cols) {
        if (kU32Src) {
          uint32_t word = static_cast<const uint32_t*>(src)[R * cp + (k >> 4)];
          code = (word >> ((k & 15) * 2)) & 3u;
        } else {
          int64_t idx = R * cols + k;  // flat pack_ternary stream
          uint8_t byte = static_cast<const uint8_t*>(src)[idx >> 2];
          code = (byte >> ((idx & 3) * 2)) & 3u;
        }
        if (code == 3u) code = 1u;  // 0b11 decodes to 0 in the reference
      }
      out |= code << (8 * b + 2 * j);
    }
  dst[gw] = out;
}

// -------------------------------------------------------- sparse repack --
// The metadata nibble and the two sign bits (1 = -1) of group kg (K / 4) of
// row R, read from a reference layout; padding (R >= rows or kg >= groups)
// gives positions (0, 1) and signs +1.
template <bool kWgsl>
__device__ __forceinline__ void ref_group(const uint8_t* pat, const uint8_t* sgn,
                                          const uint32_t* words, int64_t rows, int64_t gpr,
                                          int64_t R, int64_t kg, uint32_t& nib, uint32_t& s0,
                                          uint32_t& s1) {
  uint32_t p = 0, sb = 0;
  if (R < rows && kg < gpr) {
    if (kWgsl) {
      const int64_t wpr = (gpr + 5) / 6;
      const uint32_t v = (words[R * wpr + kg / 6] >> ((kg % 6) * 5)) & 31u;
      p = v & 7u;
      if (p > 5) p = 5;          // the WGSL shader clamps the pattern
      sb = (v >> 3) & 3u;        // 1 = negative
    } else {
      const int64_t gi = R * gpr + kg;  // flat group index of the host matrix
      p = (gi % 2 == 0) ? (pat[gi / 2] & 7u) : ((pat[gi / 2] >> 4) & 7u);
      if (p > 5) p = 0;          // to_ternary's fallback for an invalid pattern
      sb = (~(uint32_t)(sgn[gi / 4] >> ((gi % 4) * 2))) & 3u;  // host: 1 = positive
    }
  }
  nib = sparse_nibble((int)p);
  s0 = sb & 1u;
  s1 = (sb >> 1) & 1u;
}

// One thread per (tile, chunk, m-block, lane): that lane's metadata words and
// sign bits of the block (layout at the top of ft_internal.cuh).
template <bool kWgsl>
__global__ void repack_sparse_kernel(const uint8_t* __restrict__ pat, const uint8_t* __restrict__ sgn,
                                     const uint32_t* __restrict__ words, int64_t rows, int64_t cols,
                                     int64_t n_chunks, int64_t total, uint8_t* __restrict__ dst) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int L = (int)(idx & 31), mb = (int)((idx >> 5) & 7);
  const int64_t block = idx >> 8;
  const int64_t tile = block / n_chunks, chunk = block % n_chunks;
  const int g = L >> 2, t = L & 3;
  const int64_t gpr = cols / 4;  // groups per row (cols % 4 == 0)
  const int64_t r0 = tile * kTileRows + mb * 16 + g;
  uint32_t meta[2] = {0u, 0u}, signs = 0u;
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    const int64_t gb = chunk * 32 + 16 * s;  // first group of this k64 step
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      uint32_t nib, a, b;
      ref_group<kWgsl>(pat, sgn, words, rows, gpr, r0 + 8 * (t & 1), gb + 8 * (t >> 1) + i, nib, a, b);
      meta[s] |= nib << (4 * i);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t nib, a, b;
        ref_group<kWgsl>(pat, sgn, words, rows, gpr, r0 + 8 * (i & 1), gb + 8 * (i >> 1) + 2 * t + h,
                         nib, a, b);
        signs |= (a << (4 * i + 2 * h) | b << (4 * i + 2 * h + 1)) << (16 * s);
      }
  }
  uint8_t* rec = dst + block * kSparseBlockBytes + mb * kSparseMbBytes;
  reinterpret_cast<uint2*>(rec)[L] = make_uint2(meta[0], meta[1]);
  reinterpret_cast<uint32_t*>(rec + 256)[L] = signs;
}

// ------------------------------------------------------------- quantizer --
__device__ __forceinline__ float load_act(const void* x, bool bf16, int64_t i) {
  if (bf16) {
    uint32_t b = static_cast<const uint16_t*>(x)[i];
    return __uint_as_float(b << 16);
  }
  return static_cast<const float*>(x)[i];
}

__global__ void quantize_i8_kernel(const void* __restrict__ x, bool bf16, int64_t cols,
                                   int8_t* __restrict__ q, float* __restrict__ sx) {
  int64_t s = blockIdx.x;
  const int64_t off = s * cols;
  float amax = 0.0f;
  for (int64_t j = threadIdx.x; j < cols; j += blockDim.x) amax = fmaxf(amax, fabsf(load_act(x, bf16, off + j)));
  __shared__ float red[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  amax = red[0];
  if (amax == 0.0f) {
    for (int64_t j = threadIdx.x; j < cols; j += blockDim.x) q[off + j] = 0;
    if (threadIdx.x == 0) sx[s] = 1.0f;
    return;
  }
  const float inv = 127.0f / amax;  // IEEE division (no fast-math in this build)
  for (int64_t j = threadIdx.x; j < cols; j += blockDim.x) {
    float r = roundf(__fmul_rn(load_act(x, bf16, off + j), inv));
    r = fminf(fmaxf(r, -127.0f), 127.0f);
    q[off + j] = (int8_t)(int)r;
  }
  if (threadIdx.x == 0) sx[s] = __fdiv_rn(amax, 127.0f);
}

// Same arithmetic, 16-byte loads: a row of cols % (16 / element size) == 0 on
// 16-byte aligned rows.  The first kKeep loads of a thread stay in registers
// between the absmax and the rounding pass (all of them up to 8192 bf16 /
// 4096 f32 columns), later ones are read again.  Each thread then stores its
// codes as one 8-byte (bf16) or 4-byte (f32) word per load.
template <bool kBf16>
__global__ void quantize_i8_vec_kernel(const void* __restrict__ x, int64_t cols,
                                       int8_t* __restrict__ q, float* __restrict__ sx) {
  constexpr int V = kBf16 ? 8 : 4, kKeep = 4;
  const int64_t s = blockIdx.x;
  const uint4* xv =
      reinterpret_cast<const uint4*>(static_cast<const char*>(x) + s * cols * (kBf16 ? 2 : 4));
  const int64_t nv = cols / V;
  auto unpack = [](const uint4 u, float (&f)[V]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    if (kBf16) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        f[2 * e] = __uint_as_float(w[e] << 16);
        f[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
      }
    } else {
#pragma unroll
      for (int e = 0; e < V; ++e) f[e] = __uint_as_float(w[e]);
    }
  };
  uint4 keep[kKeep];
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < kKeep; ++i) {
    const int64_t j = threadIdx.x + (int64_t)i * blockDim.x;
    keep[i] = j < nv ? __ldg(xv + j) : make_uint4(0u, 0u, 0u, 0u);
  }
#pragma unroll
  for (int i = 0; i < kKeep; ++i) {
    float f[V];
    unpack(keep[i], f);
#pragma unroll
    for (int e = 0; e < V; ++e) amax = fmaxf(amax, fabsf(f[e]));
  }
  for (int64_t j = threadIdx.x + (int64_t)kKeep * blockDim.x; j < nv; j += blockDim.x) {
    float f[V];
    unpack(__ldg(xv + j), f);
#pragma unroll
    for (int e = 0; e < V; ++e) amax = fmaxf(amax, fabsf(f[e]));
  }
  __shared__ float red[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  amax = red[0];
  const bool zero = amax == 0.0f;
  const float inv = zero ? 0.0f : 127.0f / amax;  // IEEE division (no fast-math in this build)
  // codes of one load's elements (all zero for an all-zero row, as above)
  auto store = [&](const uint4 u, int8_t* qr, int64_t j) {
    float f[V];
    unpack(u, f);
    uint32_t w[2] = {0u, 0u};
#pragma unroll
    for (int g = 0; g < V / 4; ++g)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float r = roundf(__fmul_rn(f[4 * g + e], inv));
        r = fminf(fmaxf(r, -127.0f), 127.0f);
        w[g] |= zero ? 0u : (uint32_t)((int)r & 0xFF) << (8 * e);
      }
    if (kBf16) reinterpret_cast<uint2*>(qr)[j] = make_uint2(w[0], w[1]);
    else reinterpret_cast<uint32_t*>(qr)[j] = w[0];
  };
  int8_t* qr = q + s * cols;
#pragma unroll
  for (int i = 0; i < kKeep; ++i) {
    const int64_t j = threadIdx.x + (int64_t)i * blockDim.x;
    if (j < nv) store(keep[i], qr, j);
  }
  for (int64_t j = threadIdx.x + (int64_t)kKeep * blockDim.x; j < nv; j += blockDim.x)
    store(__ldg(xv + j), qr, j);
  if (threadIdx.x == 0) sx[s] = zero ? 1.0f : __fdiv_rn(amax, 127.0f);
}

// ------------------------------------------------------------ WGSL op ------
// One warp per (token, row) over the raw u32 layout; lanes take words
// round-robin, then a shuffle reduction; result * scales[row].
__global__ void wgsl_op_kernel(const uint32_t* __restrict__ words, const float* __restrict__ scales,
                               const float* __restrict__ x, float* __restrict__ y, uint32_t seq,
                               uint32_t in_cols, uint32_t out_rows) {
  int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  if (warp >= (int64_t)seq * out_rows) return;
  uint32_t s = (uint32_t)(warp / out_rows), row = (uint32_t)(warp % out_rows);
  uint32_t cp = (in_cols + 15) / 16;
  const uint32_t* wr = words + (int64_t)row * cp;
  const float* xr = x + (int64_t)s * in_cols;
  float sum = 0.0f;
  for (uint32_t p = lane; p < cp; p += 32) {
    uint32_t word = wr[p];
#pragma unroll
    for (uint32_t b = 0; b < 16; ++b) {
      uint32_t col = p * 16 + b;
      if (col >= in_cols) break;
      uint32_t code = (word >> (b * 2)) & 3u;
      float v = xr[col];
      if (code == 0u) sum -= v;
      else if (code == 2u) sum += v;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane == 0) y[(int64_t)s * out_rows + row] = sum * scales[row];
}

// ------------------------------------------------------- quantize + pack --
// One thread per output u32 word of the tiled layout: quantizes the word's 16
// source elements (fp32, or bf16 bit patterns) to codes.  alpha = row_alpha[R]:
//   mode 0, absmean (quantize_ternary, src/model/ternary.rs:31-57):
//     q = clamp(round_half_away(v * (1 / alpha)), -1, 1); NaN -> 0 (Rust's
//     `as i32` maps NaN to 0);
//   mode 1, STE requantize (BitMoELayer::requantize_all,
//     src/training/bit_moe.rs:243-262): n = v / alpha, q = +1 if n > 0.5,
//     -1 if n < -0.5, else 0; alpha < 1e-10 gives 0.
__global__ void quantize_pack_kernel(const void* __restrict__ src, int bf16, int64_t rows,
                                     int64_t cols, int64_t n_chunks, int64_t total_words,
                                     const float* __restrict__ row_alpha, int mode,
                                     uint32_t* __restrict__ dst) {
  const int64_t gw = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gw >= total_words) return;
  const int64_t block = gw >> 10;
  const int within = (int)(gw & 1023);
  const int mb = within >> 7, lane = (within >> 2) & 31, wi = within & 3;
  const int g = lane >> 2, r = lane & 3;
  const int64_t tile = block / n_chunks, chunk = block % n_chunks;
  const int64_t R = tile * kTileRows + 16 * mb + g + 8 * (wi & 1);
  float inv = 0.0f, alpha = 0.0f;
  if (R < rows) {
    alpha = row_alpha[R];
    inv = 1.0f / alpha;
  }
  uint32_t out = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int64_t k = chunk * kChunkK + 32 * j + 16 * (wi >> 1) + 4 * r + b;
      uint32_t code = 1u;
      if (R < rows && k < cols) {
        const int64_t i = R * cols + k;
        const float v = bf16 ? __uint_as_float((uint32_t) static_cast<const uint16_t*>(src)[i] << 16)
                             : static_cast<const float*>(src)[i];
        int q = 0;
        if (mode == 0) {
          const float rv = roundf(__fmul_rn(v, inv));
          q = rv != rv ? 0 : (rv >= 1.0f ? 1 : (rv <= -1.0f ? -1 : 0));
        } else if (!(alpha < 1e-10f)) {
          const float n = __fdiv_rn(v, alpha);
          q = n > 0.5f ? 1 : (n < -0.5f ? -1 : 0);
        }
        code = (uint32_t)(q + 1);
      }
      out |= code << (8 * b + 2 * j);
    }
  dst[gw] = out;
}

__global__ void fill_scales_kernel(float* __restrict__ dst, int64_t rows, int64_t padded,
                                   float alpha) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < padded) dst[i] = i < rows ? alpha : 0.0f;
}

// Sum of |v| over n elements (fp32 or bf16) in f64, added into *acc.
__global__ void abs_sum_kernel(const void* __restrict__ src, int bf16, int64_t n,
                               double* __restrict__ acc) {
  double part = 0.0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = bf16 ? __uint_as_float((uint32_t) static_cast<const uint16_t*>(src)[i] << 16)
                         : static_cast<const float*>(src)[i];
    part += (double)fabsf(v);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  __shared__ double red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = part;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    atomicAdd(acc, t);
  }
}

// One thread per byte of the reference pack_ternary stream (4 codes, LSB
// first): reads the codes back from the resident layout (dense or 2:4).
__global__ void export_u8_kernel(const uint8_t* __restrict__ codes, int format, int64_t rows,
                                 int64_t cols, int64_t n_chunks, int64_t nbytes,
                                 uint8_t* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nbytes) return;
  uint32_t b = 0;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int64_t f = 4 * i + e;
    if (f >= rows * cols) break;  // padding bits stay 0, as pack_ternary leaves them
    const int w = weight_at(codes, format, n_chunks, f / cols, f % cols);
    b |= (uint32_t)(w + 1) << (2 * e);
  }
  out[i] = (uint8_t)b;
}

}  // namespace

int launch_repack_u8(const uint8_t* packed, int64_t rows, int64_t cols, ft_weight* w,
                     cudaStream_t s) {
  int64_t total = w->n_tiles * w->n_chunks * (kBlockBytes / 4);
  repack_kernel<false><<<(unsigned)ceil_div(total, 256), 256, 0, s>>>(
      packed, rows, cols, w->n_chunks, total, reinterpret_cast<uint32_t*>(w->codes));
  FT_LAUNCH_CHECK();
  return FT_OK;
}

int launch_repack_u32(const uint32_t* words, int64_t rows, int64_t cols, ft_weight* w,
                      cudaStream_t s) {
  int64_t total = w->n_tiles * w->n_chunks * (kBlockBytes / 4);
  repack_kernel<true><<<(unsigned)ceil_div(total, 256), 256, 0, s>>>(
      words, rows, cols, w->n_chunks, total, reinterpret_cast<uint32_t*>(w->codes));
  FT_LAUNCH_CHECK();
  return FT_OK;
}

int launch_repack_sparse_host(const uint8_t* patterns, const uint8_t* signs, int64_t rows,
                              int64_t cols, ft_weight* w, cudaStream_t s) {
  int64_t total = w->n_tiles * w->n_chunks * 256;
  repack_sparse_kernel<false><<<(unsigned)ceil_div(total, 256), 256, 0, s>>>(
      patterns, signs, nullptr, rows, cols, w->n_chunks, total, w->codes);
  FT_LAUNCH_CHECK();
  return FT_OK;
}

int launch_repack_sparse_wgsl(const uint32_t* words, int64_t rows, int64_t cols, ft_weight* w,
                              cudaStream_t s) {
  int64_t total = w->n_tiles * w->n_chunks * 256;
  repack_sparse_kernel<true><<<(unsigned)ceil_div(total, 256), 256, 0, s>>>(
      nullptr, nullptr, words, rows, cols, w->n_chunks, total, w->codes);
  FT_LAUNCH_CHECK();
  return FT_OK;
}

int launch_quantize_i8(const void* x, bool bf16, int64_t seq, int64_t cols, int8_t* q, float* sx,
                       cudaStream_t s) {
  if (seq == 0) return FT_OK;
  const int V = bf16 ? 8 : 4;
  if (cols % V == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(q) & (bf16 ? 7 : 3)) == 0 && (cols * (bf16 ? 2 : 4)) % 16 == 0) {
    if (bf16) quantize_i8_vec_kernel<true><<<(unsigned)seq, 256, 0, s>>>(x, cols, q, sx);
    else quantize_i8_vec_kernel<false><<<(unsigned)seq, 256, 0, s>>>(x, cols, q, sx);
  } else {
    quantize_i8_kernel<<<(unsigned)seq, 256, 0, s>>>(x, bf16, cols, q, sx);
  }
  FT_LAUNCH_CHECK();
  return FT_OK;
}

int launch_wgsl_op(const uint32_t* words, const float* scales, const float* x, float* y,
                   uint32_t seq, uint32_t in_cols, uint32_t out_rows, cudaStream_t s) {
  int64_t warps = (int64_t)seq * out_rows;
  if (warps == 0) return FT_OK;
  wgsl_op_kernel<<<(unsigned)ceil_div(warps * 32, 256), 256, 0, s>>>(words, scales, x, y, seq,
                                                                    in_cols, out_rows);
  FT_LAUNCH_CHECK();
  return FT_OK;
}

int launch_quantize_pack(const void* src, bool bf16, int mode, ft_weight* w, cudaStream_t s) {
  const int64_t total = w->n_tiles * w->n_chunks * (kBlockBytes / 4);
  quantize_pack_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, s>>>(
      src, bf16 ? 1 : 0, w->rows, w->cols, w->n_chunks, total, w->row_scales, mode,
      reinterpret_cast<uint32_t*>(w->codes));
  FT_LAUNCH_CHECK();
  return FT_OK;
}

int launch_fill_scales(ft_weight* w, float alpha, cudaStream_t s) {
  const int64_t padded = w->n_tiles * kTileRows;
  fill_scales_kernel<<<(unsigned)ceil_div(padded, 256), 256, 0, s>>>(w->row_scales, w->rows, padded,
                                                                     alpha);
  FT_LAUNCH_CHECK();
  return FT_OK;
}

int launch_abs_sum(const void* src, bool bf16, int64_t n, double* acc, cudaStream_t s) {
  if (n <= 0) return FT_OK;
  int64_t blocks = ceil_div(n, 256 * 8);
  if (blocks > 1184) blocks = 1184;
  abs_sum_kernel<<<(unsigned)blocks, 256, 0, s>>>(src, bf16 ? 1 : 0, n, acc);
  FT_LAUNCH_CHECK();
  return FT_OK;
}

int launch_export_u8(const ft_weight* w, uint8_t* out, cudaStream_t s) {
  const int64_t nbytes = (w->rows * w->cols + 3) / 4;
  export_u8_kernel<<<(unsigned)ceil_div(nbytes, 256), 256, 0, s>>>(w->codes, w->format, w->rows,
                                                                   w->cols, w->n_chunks, nbytes, out);
  FT_LAUNCH_CHECK();
  return FT_OK;
}

}  // namespace ft
