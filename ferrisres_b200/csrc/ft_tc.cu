// Tensor-core (tcgen05, sm_100a) ternary matmul: y = scale * (W . x).
//
// Formulation.  The packed 2-bit codes u = w + 1 in {0, 1, 2} are unpacked
// in registers (one shift + one mask per 4 codes, thanks to the tiled T128
// layout) and written to tensor memory as the unsigned 8-bit A operand
// (M = 128 output channels of one tile).  The activations are the signed
// 8-bit B operand, K-major in shared memory, N = NPAD columns:
//   * int8 mode: one column per token, the caller's int8 codes q;
//   * fp32 mode: four columns per token, the signed base-256 digits of the
//     31-bit fixed-point image X = round(x * 2^30 / absmax(token)).
// tcgen05.mma kind::i8 accumulates exact int32 sums D = sum_k u_k b_k in TMEM;
// the epilogue subtracts sum_k b_k (so D becomes sum_k w_k b_k) and scales:
//   int8: y = ((float)D * sx[s]) * scale[r]      (bit-exact vs the reference)
//   fp32: y = (double)(sum_d D_d << 8d) * absmax/2^30 * scale[r]
// For fp32 activations the only approximation is the fixed-point image of x
// (error <= absmax * 2^-31 per element), which sits far inside the 1e-5
// condition-relative tolerance for any input whose row magnitudes are within
// ~1e4 of the token's absmax.
//
// Pipeline per CTA (one 128-row tile, one K range, one column pass):
//   warps 0-3  converters: thread r loads row r's 32 bytes per 128-K chunk
//              straight from HBM (coalesced 512 B per warp instruction,
//              4 chunks in flight), unpacks, tcgen05.st into A stage s;
//              later the epilogue (tcgen05.ld of row r's accumulators).
//   warp 4     producer: 1-D bulk copies of the B chunk into smem stage s.
//   warp 5     MMA issuer: 4 x tcgen05.mma (K = 32 each) per chunk,
//              tcgen05.commit frees the stage.
// Split-K partials are combined with exact int32 atomics in a zero-initialised
// scratch area; the last CTA of a tile (atomic ticket) runs the epilogue and
// clears the scratch again, so it stays zero between calls.
#include "ft_internal.cuh"
#include "ft_tc.cuh"

namespace ft {
namespace {

constexpr int kStages = 4;
constexpr int kPrefetch = 4;
constexpr int kThreads = 192;

struct TcParams {
  const uint8_t* codes;
  const float* row_scales;
  int64_t rows, n_tiles, n_chunks;
  const int8_t* bmat;       // [passes][n_chunks][NPAD*128]
  const int32_t* colsum;    // [passes][NPAD]
  const double* tok_scale;  // fp32 mode: absmax * 2^-30 per token
  const float* sx;          // int8 mode: per-token scale
  int64_t seq;
  int digits;               // 1 (int8) or 4 (fp32)
  int tok_per_pass;
  int chunks_per_split, ksplit;
  int32_t* acc;             // [passes][n_tiles][NPAD][128], zero between calls
  int32_t* cnt;             // [passes][n_tiles], zero between calls
  float* y;                 // [seq, rows]
  int* err;
};

__host__ __device__ constexpr uint32_t tmem_cols_for(int npad) {
  uint32_t need = (uint32_t)((npad + 31) / 32 * 32 + kStages * 32);
  uint32_t c = 32;
  while (c < need) c <<= 1;
  return c;
}

__device__ __forceinline__ void named_sync_epilogue() {
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

template <int NPAD>
__device__ __forceinline__ void epilogue_group(const TcParams& p, int pass, int64_t R,
                                               int col0, const int32_t (&v)[16]) {
  const int D = p.digits;
  for (int c = 0; c < 16; c += D) {
    int lt = (col0 + c) / D;
    int64_t t = (int64_t)pass * p.tok_per_pass + lt;
    if (t >= p.seq || lt >= p.tok_per_pass) break;
    float out;
    if (D == 1) {
      int32_t a = v[c] - p.colsum[pass * NPAD + col0 + c];
      out = __fmul_rn(__fmul_rn((float)a, p.sx[t]), p.row_scales[R]);
    } else {
      long long S = 0;
#pragma unroll
      for (int d = 0; d < 4; ++d) {
        long long a = (long long)(v[c + d] - p.colsum[pass * NPAD + col0 + c + d]);
        S += a * (1ll << (8 * d));
      }
      out = (float)((double)S * p.tok_scale[t] * (double)p.row_scales[R]);
    }
    p.y[t * p.rows + R] = out;
  }
}

template <int NPAD>
__global__ void __launch_bounds__(kThreads, 1) tc_ternary_kernel(const TcParams p) {
  extern __shared__ __align__(128) uint8_t smem_b[];  // kStages x NPAD*128 bytes
  __shared__ __align__(8) uint64_t bar_bfull[kStages];
  __shared__ __align__(8) uint64_t bar_afull[kStages];
  __shared__ __align__(8) uint64_t bar_free[kStages];
  __shared__ __align__(8) uint64_t bar_dfull;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int last_flag;

  constexpr uint32_t kBStage = NPAD * 128;
  constexpr uint32_t kLBO = (NPAD / 8) * 128;  // K-direction core-matrix stride
  constexpr uint32_t kSBO = 128;               // N-direction 8-row group stride
  constexpr uint32_t kTmemCols = tmem_cols_for(NPAD);
  constexpr uint32_t kACol0 = (NPAD + 31) / 32 * 32;
  constexpr uint32_t kIdesc = tc::idesc_i8(128, NPAD);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tile = blockIdx.x;
  const int ks = blockIdx.y;
  const int pass = blockIdx.z;
  const int64_t c0 = (int64_t)ks * p.chunks_per_split;
  int64_t c1 = c0 + p.chunks_per_split;
  if (c1 > p.n_chunks) c1 = p.n_chunks;
  const int nch = (int)(c1 - c0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      tc::mbar_init(tc::smem_u32(&bar_bfull[s]), 1);
      tc::mbar_init(tc::smem_u32(&bar_afull[s]), 4);
      tc::mbar_init(tc::smem_u32(&bar_free[s]), 1);
    }
    tc::mbar_init(tc::smem_u32(&bar_dfull), 1);
    tc::fence_barrier_init();
  }
  if (warp == 0) tc::tmem_alloc(tc::smem_u32(&tmem_base_sh), kTmemCols);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  tc::pdl_launch_dependents();
  const uint32_t tmem = tmem_base_sh;
  bool ok = true;

  if (warp < 4) {
    // ------------------------------------------------------ converters --
    const int r = threadIdx.x;
    const uint32_t lane_off = (uint32_t)(32 * warp) << 16;
    const uint8_t* wbase = p.codes + (tile * p.n_chunks + c0) * kBlockBytes + r * 16;
    uint4 buf[kPrefetch][2];
#pragma unroll
    for (int j = 0; j < kPrefetch; ++j)
      if (j < nch) {
        buf[j][0] = __ldg(reinterpret_cast<const uint4*>(wbase + (int64_t)j * kBlockBytes));
        buf[j][1] = __ldg(reinterpret_cast<const uint4*>(wbase + (int64_t)j * kBlockBytes + 2048));
      }
    for (int i0 = 0; i0 < nch; i0 += kPrefetch) {
#pragma unroll
      for (int j = 0; j < kPrefetch; ++j) {
        const int i = i0 + j;
        if (i >= nch) break;
        const uint32_t wv[8] = {buf[j][0].x, buf[j][0].y, buf[j][0].z, buf[j][0].w,
                                buf[j][1].x, buf[j][1].y, buf[j][1].z, buf[j][1].w};
        if (i + kPrefetch < nch) {
          const uint8_t* src = wbase + (int64_t)(i + kPrefetch) * kBlockBytes;
          buf[j][0] = __ldg(reinterpret_cast<const uint4*>(src));
          buf[j][1] = __ldg(reinterpret_cast<const uint4*>(src + 2048));
        }
        uint32_t a[32];
#pragma unroll
        for (int hw = 0; hw < 8; ++hw)
#pragma unroll
          for (int q = 0; q < 4; ++q) a[hw * 4 + q] = (wv[hw] >> (2 * q)) & 0x03030303u;
        const int s = i % kStages;
        if (ok && i >= kStages)
          ok = tc::mbar_wait(tc::smem_u32(&bar_free[s]), ((i / kStages) + 1) & 1, p.err, 11);
        ok = __all_sync(0xffffffffu, ok);  // tcgen05.st below is warp-collective
        tc::tc_fence_after();
        if (ok) tc::tmem_st_x32(tmem + lane_off + kACol0 + 32 * s, a);
        tc::tmem_wait_st();
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(tc::smem_u32(&bar_afull[s]));
      }
    }
  } else if (warp == 4) {
    // -------------------------------------------------------- producer --
    if (lane == 0) {
      tc::pdl_wait();  // B is written by the preceding prep kernel
      const int8_t* bsrc = p.bmat + ((int64_t)pass * p.n_chunks + c0) * kBStage;
      for (int i = 0; i < nch && ok; ++i) {
        const int s = i % kStages;
        if (i >= kStages)
          ok = tc::mbar_wait(tc::smem_u32(&bar_free[s]), ((i / kStages) + 1) & 1, p.err, 12);
        if (!ok) break;
        const uint32_t bar = tc::smem_u32(&bar_bfull[s]);
        tc::mbar_arrive_expect_tx(bar, kBStage);
        tc::bulk_g2s(tc::smem_u32(smem_b + s * kBStage), bsrc + (int64_t)i * kBStage, kBStage, bar);
      }
    }
  } else {
    // ------------------------------------------------------ MMA issuer --
    if (lane == 0) {
      for (int i = 0; i < nch && ok; ++i) {
        const int s = i % kStages;
        const uint32_t par = (i / kStages) & 1;
        ok = tc::mbar_wait(tc::smem_u32(&bar_afull[s]), par, p.err, 13) &&
             tc::mbar_wait(tc::smem_u32(&bar_bfull[s]), par, p.err, 14);
        if (!ok) break;
        tc::tc_fence_after();
        const uint32_t bst = tc::smem_u32(smem_b + s * kBStage);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint64_t bd = tc::smem_desc(bst + j * 2 * kLBO, kLBO, kSBO);
          tc::mma_i8_ts(tmem, tmem + kACol0 + 32 * s + 8 * j, bd, kIdesc, (i > 0 || j > 0) ? 1u : 0u);
        }
        tc::mma_commit(tc::smem_u32(&bar_free[s]));
      }
      tc::mma_commit(tc::smem_u32(&bar_dfull));
    }
  }

  if (warp < 4) {
    // -------------------------------------------------------- epilogue --
    const int r = threadIdx.x;
    const uint32_t lane_off = (uint32_t)(32 * warp) << 16;
    const int64_t R = tile * kTileRows + r;
    ok = ok && tc::mbar_wait(tc::smem_u32(&bar_dfull), 0, p.err, 15);
    tc::tc_fence_after();
    tc::pdl_wait();  // outputs / scratch may still be used by the previous launch
    const int ncols = p.tok_per_pass * p.digits;
    if (p.ksplit == 1) {
#pragma unroll 1
      for (int cg = 0; cg < NPAD / 16; ++cg) {
        uint32_t u[16];
        tc::tmem_ld_x16(tmem + lane_off + cg * 16, u);
        tc::tmem_wait_ld();
        int32_t v[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) v[c] = (int32_t)u[c];
        if (ok && R < p.rows && cg * 16 < ncols) epilogue_group<NPAD>(p, pass, R, cg * 16, v);
      }
    } else {
      int32_t* accp = p.acc + (((int64_t)pass * p.n_tiles + tile) * NPAD) * kTileRows;
#pragma unroll 1
      for (int cg = 0; cg < NPAD / 16; ++cg) {
        uint32_t u[16];
        tc::tmem_ld_x16(tmem + lane_off + cg * 16, u);
        tc::tmem_wait_ld();
        if (ok)
#pragma unroll
          for (int c = 0; c < 16; ++c)
            if (cg * 16 + c < ncols) atomicAdd(&accp[(cg * 16 + c) * kTileRows + r], (int32_t)u[c]);
      }
      __threadfence();
      named_sync_epilogue();
      if (r == 0) {
        int prev = atomicAdd(&p.cnt[(int64_t)pass * p.n_tiles + tile], 1);
        last_flag = (prev == p.ksplit - 1);
      }
      named_sync_epilogue();
      if (last_flag) {
        __threadfence();
#pragma unroll 1
        for (int cg = 0; cg < NPAD / 16 && cg * 16 < ncols; ++cg) {
          int32_t v[16];
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            int32_t* a = &accp[(cg * 16 + c) * kTileRows + r];
            v[c] = __ldcg(a);
            __stcg(a, 0);  // leave the scratch zeroed for the next call
          }
          if (ok && R < p.rows) epilogue_group<NPAD>(p, pass, R, cg * 16, v);
        }
        if (r == 0) p.cnt[(int64_t)pass * p.n_tiles + tile] = 0;
      }
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------- B prep -----
// One block per (pass, token slot): writes the token's digit columns of the
// K-major interleaved B operand for every chunk, their column sums, and the
// token scale.  Slots past `seq` write zero columns.
__device__ __forceinline__ int64_t b_offset(int64_t pass, int64_t chunk, int n, int kin, int npad,
                                            int64_t n_chunks) {
  return ((pass * n_chunks + chunk) * npad) * 128 + ((kin >> 4) * (npad >> 3) + (n >> 3)) * 128 +
         (n & 7) * 16 + (kin & 15);
}

// xkind: 0 = f32, 1 = bf16, 2 = int8 codes
__global__ void __launch_bounds__(256) prep_b_kernel(const void* __restrict__ x, int xkind,
                                                     int64_t seq, int64_t K, int64_t n_chunks,
                                                     int D, int npad, int tok_per_pass,
                                                     int8_t* __restrict__ bmat,
                                                     int32_t* __restrict__ colsum,
                                                     double* __restrict__ tok_scale) {
  // Let the matmul that consumes this launch start streaming its weights now;
  // then wait for the previous matmul, which may still be reading bmat.
  tc::pdl_launch_dependents();
  tc::pdl_wait();
  const int64_t pass = blockIdx.x / tok_per_pass;
  const int lt = blockIdx.x % tok_per_pass;
  const int64_t t = pass * tok_per_pass + lt;
  const int64_t kpad = n_chunks * 128;
  __shared__ float red_f[8];
  __shared__ int red_i[8][4];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool live = t < seq;
  double mult = 0.0;
  if (xkind != 2) {
    float amax = 0.0f;
    if (live)
      for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
        float v = xkind == 0 ? static_cast<const float*>(x)[t * K + k]
                             : __uint_as_float((uint32_t) static_cast<const uint16_t*>(x)[t * K + k] << 16);
        amax = fmaxf(amax, fabsf(v));
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) red_f[warp] = amax;
    __syncthreads();
    amax = 0.0f;
    for (int w = 0; w < 8; ++w) amax = fmaxf(amax, red_f[w]);
    if (amax > 0.0f) mult = 1073741824.0 / (double)amax;  // 2^30 / absmax
    if (threadIdx.x == 0 && live && tok_scale) tok_scale[t] = (double)amax / 1073741824.0;
  }
  int csum[4] = {0, 0, 0, 0};
  for (int64_t k = threadIdx.x; k < kpad; k += blockDim.x) {
    int dg[4] = {0, 0, 0, 0};
    if (live && k < K) {
      if (xkind == 2) {
        dg[0] = static_cast<const int8_t*>(x)[t * K + k];
      } else {
        float v = xkind == 0 ? static_cast<const float*>(x)[t * K + k]
                             : __uint_as_float((uint32_t) static_cast<const uint16_t*>(x)[t * K + k] << 16);
        long long X = __double2ll_rn((double)v * mult);
#pragma unroll
        for (int d = 0; d < 3; ++d) {
          int lo = (int)(X & 0xFF);
          lo = (lo ^ 0x80) - 0x80;  // signed low digit
          dg[d] = lo;
          X = (X - lo) >> 8;
        }
        dg[3] = (int)X;  // |X| <= 64 here
      }
    }
    const int64_t chunk = k >> 7;
    const int kin = (int)(k & 127);
    for (int d = 0; d < D; ++d) {
      bmat[b_offset(pass, chunk, lt * D + d, kin, npad, n_chunks)] = (int8_t)dg[d];
      csum[d] += dg[d];
    }
  }
  for (int d = 0; d < D; ++d) {
    int v = csum[d];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red_i[warp][d] = v;
  }
  __syncthreads();
  if (threadIdx.x < D) {
    int v = 0;
    for (int w = 0; w < 8; ++w) v += red_i[w][threadIdx.x];
    colsum[pass * npad + lt * D + threadIdx.x] = v;
  }
}

template <int NPAD>
int launch_tc_t(ft_ctx* ctx, const ft_weight* w, const TcParams& base, int passes,
                cudaStream_t s) {
  TcParams p = base;
  const int64_t tiles = w->n_tiles;
  // Split K so that a launch has about one CTA per SM (leaving room for the
  // next launch's CTAs to start under programmatic dependent launch).
  int64_t want = (ctx->num_sms + tiles * passes - 1) / (tiles * passes);
  if (want < 1) want = 1;
  if (want > w->n_chunks) want = w->n_chunks;
  int cps = (int)ceil_div(w->n_chunks, want);
  int ks = (int)ceil_div(w->n_chunks, cps);
  p.chunks_per_split = cps;
  p.ksplit = ks;
  const size_t smem = (size_t)kStages * NPAD * 128;
  static bool attr_set = false;  // per template instance
  if (!attr_set) {
    FT_CUDA(cudaFuncSetAttribute(tc_ternary_kernel<NPAD>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)tiles, (unsigned)ks, (unsigned)passes);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FT_CUDA(cudaLaunchKernelEx(&cfg, tc_ternary_kernel<NPAD>, p));
  FT_LAUNCH_CHECK();
  return FT_OK;
}

int pick_npad(int64_t ncols) {
  if (ncols <= 16) return 16;
  if (ncols <= 32) return 32;
  if (ncols <= 64) return 64;
  if (ncols <= 128) return 128;
  return 256;
}

}  // namespace

// Tensor-core matmul.  mode_digits = 4 for fp32/bf16 activations, 1 for int8.
int launch_tc_matmul(ft_ctx* ctx, const ft_weight* w, int64_t seq, const void* x, int xkind,
                     const float* sx, float* y, cudaStream_t s) {
  if (seq == 0) return FT_OK;
  const int D = xkind == 2 ? 1 : 4;
  const int64_t ncols_total = seq * D;
  const int npad = pick_npad(ncols_total);
  const int tok_per_pass = npad / D;
  const int64_t passes = ceil_div(seq, tok_per_pass);
  FT_CHECK(passes <= 65535, FT_ERR_UNSUPPORTED, "seq %lld too large", (long long)seq);
  const int64_t n_chunks = w->n_chunks;

  // general workspace: B operand, column sums, token scales
  size_t b_bytes = (size_t)(passes * n_chunks) * npad * 128;
  size_t cs_off = round_up((int64_t)b_bytes, 256);
  size_t ts_off = round_up((int64_t)(cs_off + passes * npad * 4), 256);
  size_t need = ts_off + (size_t)seq * 8 + 256;
  int st = workspace_reserve(ctx, need, s);
  if (st != FT_OK) return st;
  char* ws = static_cast<char*>(ctx->ws.ptr);
  int8_t* bmat = reinterpret_cast<int8_t*>(ws);
  int32_t* colsum = reinterpret_cast<int32_t*>(ws + cs_off);
  double* tok_scale = reinterpret_cast<double*>(ws + ts_off);

  // zero-initialised scratch for split-K (self-cleaning)
  size_t acc_bytes = (size_t)(passes * w->n_tiles) * npad * kTileRows * 4;
  size_t cnt_off = round_up((int64_t)acc_bytes, 256);
  size_t err_off = cnt_off + round_up(passes * w->n_tiles * 4, 256);
  st = zero_scratch_reserve(ctx, err_off + 256, s);
  if (st != FT_OK) return st;
  char* zs = static_cast<char*>(ctx->zs.ptr);

  {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(passes * tok_per_pass));
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    FT_CUDA(cudaLaunchKernelEx(&cfg, prep_b_kernel, x, xkind, seq, w->cols, n_chunks, D, npad,
                               tok_per_pass, bmat, colsum, tok_scale));
    FT_LAUNCH_CHECK();
  }

  TcParams p{};
  p.codes = w->codes;
  p.row_scales = w->row_scales;
  p.rows = w->rows;
  p.n_tiles = w->n_tiles;
  p.n_chunks = n_chunks;
  p.bmat = bmat;
  p.colsum = colsum;
  p.tok_scale = tok_scale;
  p.sx = sx;
  p.seq = seq;
  p.digits = D;
  p.tok_per_pass = tok_per_pass;
  p.acc = reinterpret_cast<int32_t*>(zs);
  p.cnt = reinterpret_cast<int32_t*>(zs + cnt_off);
  p.y = y;
  p.err = reinterpret_cast<int*>(zs + err_off);
  ctx->err_flag = p.err;
  switch (npad) {
    case 16: return launch_tc_t<16>(ctx, w, p, (int)passes, s);
    case 32: return launch_tc_t<32>(ctx, w, p, (int)passes, s);
    case 64: return launch_tc_t<64>(ctx, w, p, (int)passes, s);
    case 128: return launch_tc_t<128>(ctx, w, p, (int)passes, s);
    default: return launch_tc_t<256>(ctx, w, p, (int)passes, s);
  }
}

}  // namespace ft
