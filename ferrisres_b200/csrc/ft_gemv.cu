// Decode-shape ternary matmul (GEMV and small M): y = scale * (W . x) for a
// group of independent problems whose activations fit 16 operand columns
// (fp32/bf16: <= 4 tokens as 4 base-256 digits each; int8: <= 16 tokens).
//
// Same exact formulation as the tensor-core engine (ft_tc.cu): the A operand
// is the unsigned codes u = w + 1, the B operand the int8 activation columns
// (fp32/bf16: the signed base-256 digits of X = round(x * 2^30 / absmax(x)),
// int8: the caller's codes), int32 sums are exact, the epilogue subtracts the
// column sums and scales.  Here the MMAs are warp-level (mma.sync m16n8k32):
// every lane loads its 16 bytes of a 4 KB weight block straight from global
// memory with one coalesced 128-bit load (the lane-major block layout puts a
// warp's 512 bytes of an m-block contiguous), unpacks each word with one shift
// and one mask per fragment register, and issues 4 MMAs per n8 block.  The
// weight stream needs no shared memory staging, barriers or TMEM.
//
// prep_b_kernel (ft_tc.cu) writes the activation operand in this kernel's
// fragment order; the kernel is launched as its programmatic dependent, so
// each warp starts its weight stream before waiting for the prep, then the
// CTA copies its fragments into shared memory.
//
// Work: a CTA of 8 warps covers 8/S m-blocks (16 rows each) of one problem,
// each split S ways along K (S in {1, 2, 4, 8}, chosen so the launch has
// enough warps); the S partial sums of an m-block meet in shared memory.
#include "ft_internal.cuh"
#include "ft_tc.cuh"

namespace ft {
namespace {

constexpr int kGvWarps = 8;
constexpr int kGvMaxProblems = 64;
#ifndef FT_GV_DEPTH
#define FT_GV_DEPTH 6
#endif
#ifndef FT_GV_MIN_BLOCKS
#define FT_GV_MIN_BLOCKS 5
#endif
constexpr int kDepth = FT_GV_DEPTH;  // weight chunks in flight per warp (cp.async ring)
constexpr int kRingBytes = kGvWarps * kDepth * 512;

struct GvProblem {
  const uint4* codes;  // lane-major blocks, 256 uint4 per (tile, chunk)
  const float* row_scales;
  int64_t rows, n_tiles, n_chunks;
  const uint4* bfrag;       // [n_chunks][2][32 lanes][2 uint4] (prep_b_kernel)
  const int32_t* colsum;    // [16]
  const double* tok_scale;  // fp32 mode: absmax * 2^-30 per token
  const float* sx;          // int8 mode: per-token scale
  float* y;
  int64_t ldy, seq;
  int64_t cta_begin;  // first CTA of this problem
  int ksplit, cps;    // K splits, chunks per split
};

struct GvBatch {
  int nprob;
  int digits;  // 4 (fp32/bf16) or 1 (int8)
  int nb;      // n8 blocks of B (1 or 2)
  GvProblem p[kGvMaxProblems];
};

__device__ __forceinline__ void mma_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 16-byte asynchronous copy global -> shared (bypasses L1 and registers)
__device__ __forceinline__ void cp_async16(const void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   (uint32_t)__cvta_generic_to_shared(smem_dst)),
               "l"(gsrc)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// the 4 k-steps of one 128-K chunk against the 8 fragment words of one n8 block
__device__ __forceinline__ void chunk_mma(int (&acc)[4], const uint4 w, const uint4 b0,
                                          const uint4 b1) {
  const uint32_t wk[4] = {w.x, w.y, w.z, w.w};
  const uint32_t bw[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    const uint32_t a0 = wk[ks] & 0x03030303u;
    const uint32_t a1 = (wk[ks] >> 2) & 0x03030303u;
    const uint32_t a2 = (wk[ks] >> 4) & 0x03030303u;
    const uint32_t a3 = (wk[ks] >> 6) & 0x03030303u;
    mma_u8s8(acc, a0, a1, a2, a3, bw[2 * ks], bw[2 * ks + 1]);
  }
}

template <int NB>
__global__ void __launch_bounds__(kGvWarps * 32, FT_GV_MIN_BLOCKS) gemv_kernel(const __grid_constant__ GvBatch b) {
  // dynamic: [warp][kDepth][32 lanes] uint4 weight ring, then the B fragments
  // [n_chunks][NB][32 lanes][8 words]
  extern __shared__ __align__(16) uint4 dyn[];
  uint32_t* frag = reinterpret_cast<uint32_t*>(dyn + kRingBytes / 16);
  __shared__ int colsum[16];
  __shared__ double tok_scale[4];

  int pi = 0;
  while (pi + 1 < b.nprob && b.p[pi + 1].cta_begin <= (int64_t)blockIdx.x) ++pi;
  const GvProblem& p = b.p[pi];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, r = lane & 3;
  const int S = p.ksplit;
  const int64_t mblock = (blockIdx.x - p.cta_begin) * (kGvWarps / S) + warp / S;
  const int split = warp % S;
  const int64_t tile = mblock >> 3;
  const int mb = (int)(mblock & 7);
  const bool active = tile < p.n_tiles;
  int64_t c0 = (int64_t)split * p.cps, c1 = c0 + p.cps;
  if (c1 > p.n_chunks) c1 = p.n_chunks;
  if (!active) c1 = c0;

  // ---- start the weight stream: each lane copies (and later reads) only its
  // own 16 bytes of each chunk, so the ring needs no barriers
  const uint4* wp = p.codes + (tile * p.n_chunks) * 256 + mb * 32 + lane;
  uint4* ring = dyn + warp * (kDepth * 32) + lane;
#pragma unroll
  for (int d = 0; d < kDepth; ++d) {
    if (c0 + d < c1) cp_async16(ring + d * 32, wp + (c0 + d) * 256);
    cp_async_commit();  // one group per chunk slot, empty past the range
  }

  // ---- the activation operand, column sums and token scales of the prep
  tc::pdl_wait();
  const int D = b.digits;
  const int seq = (int)p.seq;
  {
    uint4* f4 = reinterpret_cast<uint4*>(frag);
    const int n16 = (int)(p.n_chunks * NB * 64);  // 16-byte pieces
    for (int i = tid; i < n16; i += blockDim.x) {
      const int64_t chunk = i / (NB * 64);
      const int rem = i % (NB * 64);  // (nb, lane, half)
      cp_async16(f4 + i, p.bfrag + chunk * 128 + rem);
    }
    cp_async_commit();
    if (tid < 16) colsum[tid] = p.colsum[tid];
    if (tid < 4 && D == 4) tok_scale[tid] = p.tok_scale[tid];
    // the weight ring's groups are older, so waiting for all is waiting for this one too
    cp_async_wait<0>();
  }
  __syncthreads();

  // ---- the weight stream against the fragments
  int acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
  const uint4* fq = reinterpret_cast<const uint4*>(frag);
  int slot = 0;
  for (int64_t ch = c0; ch < c1; ++ch) {
    cp_async_wait<kDepth - 1>();  // this lane's copy of chunk ch has landed
    const uint4 cur = ring[slot * 32];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      const uint4* f = fq + ((ch * NB + nb) * 32 + lane) * 2;
      chunk_mma(acc[nb], cur, f[0], f[1]);
    }
    // the MMAs consumed `cur`, so the slot can be refilled
    if (ch + kDepth < c1) cp_async16(ring + slot * 32, wp + (ch + kDepth) * 256);
    cp_async_commit();
    slot = slot + 1 == kDepth ? 0 : slot + 1;
  }
  cp_async_wait<0>();
  __syncthreads();  // the ring is reused for the split sums below

  // ---- combine the K splits of each m-block
  if (S > 1) {
    int(*red)[32][8] = reinterpret_cast<int(*)[32][8]>(dyn);  // [warp][lane][8], in the ring
#pragma unroll
    for (int nb = 0; nb < 2; ++nb)
#pragma unroll
      for (int i = 0; i < 4; ++i) red[warp][lane][nb * 4 + i] = acc[nb][i];
    __syncthreads();
    if (split != 0) return;
    for (int s = 1; s < S; ++s)
#pragma unroll
      for (int nb = 0; nb < 2; ++nb)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[nb][i] += red[warp + s][lane][nb * 4 + i];
  }
  if (!active) return;

  // ---- epilogue: acc[nb][0..1] = row g, columns 8nb + 2r, +1; [2..3] = row g + 8
  const int64_t R0 = tile * kTileRows + 16 * mb + g;
  if (D == 1) {
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int n = 8 * nb + 2 * r + (i & 1);
        const int64_t R = R0 + 8 * (i >> 1);
        if (n < seq && R < p.rows) {
          const int32_t a = acc[nb][i] - colsum[n];
          p.y[n * p.ldy + R] = __fmul_rn(__fmul_rn((float)a, p.sx[n]), p.row_scales[R]);
        }
      }
  } else {
    // token t = n / 4 lives in lanes r = 2(t%2) (digits 0, 1) and r + 1 (digits 2, 3)
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      const int hi0 = __shfl_xor_sync(0xffffffffu, acc[nb][0], 1);
      const int hi1 = __shfl_xor_sync(0xffffffffu, acc[nb][1], 1);
      const int hi2 = __shfl_xor_sync(0xffffffffu, acc[nb][2], 1);
      const int hi3 = __shfl_xor_sync(0xffffffffu, acc[nb][3], 1);
      if ((r & 1) == 0) {
        const int t = 2 * nb + (r >> 1);
        const int n0 = 4 * t;
        if (t < seq) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int64_t R = R0 + 8 * h;
            if (R >= p.rows) continue;
            const long long d0 = acc[nb][2 * h] - colsum[n0];
            const long long d1 = acc[nb][2 * h + 1] - colsum[n0 + 1];
            const long long d2 = (h ? hi2 : hi0) - colsum[n0 + 2];
            const long long d3 = (h ? hi3 : hi1) - colsum[n0 + 3];
            const long long S4 = d0 + d1 * 256 + d2 * 65536 + d3 * 16777216;
            p.y[t * p.ldy + R] = (float)((double)S4 * tok_scale[t] * (double)p.row_scales[R]);
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------- prep --
// Activation operand in fragment order for the kernel above, one CTA per
// (source, token slot): column n = slot*D + d of chunk c sits in lane
// 4(n%8) + r, word 2ks + kk of n8 block n/8 for K = c*128 + 32ks + 16kk + 4r
// .. +3.  fp32/bf16: the signed base-256 digits of X = round(x * 2^30 /
// absmax(x)) (|X| <= 2^30 fits 32 bits); int8: the caller's codes.  Slots
// past the token count write zeros.  Column sums and token scales as in
// prep_b_kernel.
struct FragSource {
  const void* x;
  uint32_t* frag;          // [n_chunks][2][32][8] words
  int32_t* colsum;         // [16]
  double* tok_scale;       // [4]
  int64_t K, n_chunks, seq;
};
constexpr int kMaxFragSources = 64;
constexpr int kPrepThreads = 512;
struct FragBatch {
  int nsrc, xkind, D, slots;  // token slots per source (8*nb / D)
  FragSource s[kMaxFragSources];
};

__device__ __forceinline__ float4 load_x4(const void* x, int xkind, int64_t row, int64_t k,
                                          int64_t K) {
  // elements k .. k+3 of row `row` (zero past K)
  float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  const int64_t i = row * K + k;
  if (xkind == 0) {
    const float* f = static_cast<const float*>(x);
    if (k + 3 < K && ((reinterpret_cast<uintptr_t>(f + i) & 15) == 0)) {
      v = __ldg(reinterpret_cast<const float4*>(f + i));
    } else {
      if (k < K) v.x = f[i];
      if (k + 1 < K) v.y = f[i + 1];
      if (k + 2 < K) v.z = f[i + 2];
      if (k + 3 < K) v.w = f[i + 3];
    }
  } else {
    const uint16_t* h = static_cast<const uint16_t*>(x);
    if (k < K) v.x = __uint_as_float((uint32_t)h[i] << 16);
    if (k + 1 < K) v.y = __uint_as_float((uint32_t)h[i + 1] << 16);
    if (k + 2 < K) v.z = __uint_as_float((uint32_t)h[i + 2] << 16);
    if (k + 3 < K) v.w = __uint_as_float((uint32_t)h[i + 3] << 16);
  }
  return v;
}

__global__ void __launch_bounds__(kPrepThreads) prep_frag_kernel(const __grid_constant__ FragBatch fb) {
  // let the matmul start streaming its weights, then wait for the producer of x
  tc::pdl_launch_dependents();
  tc::pdl_wait();
  const int si = blockIdx.x / fb.slots, t = blockIdx.x % fb.slots;
  const FragSource& src = fb.s[si];
  const int D = fb.D, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool live = t < src.seq;
  const int nquads = (int)(src.n_chunks * 32);
  constexpr int kQ = 4;  // quads per thread kept in registers (K <= 8192)
  __shared__ float red_f[kPrepThreads / 32];
  __shared__ int red_i[kPrepThreads / 32][4];
  uint32_t word[kQ][4];
  int cs[4] = {0, 0, 0, 0};
  if (D == 4) {
    float4 xv[kQ];
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < kQ; ++j) {
      const int qi = tid + j * kPrepThreads;
      xv[j] = live && qi < nquads ? load_x4(src.x, fb.xkind, t, 4 * (int64_t)qi, src.K)
                                  : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(xv[j].x), fabsf(xv[j].y)),
                               fmaxf(fabsf(xv[j].z), fabsf(xv[j].w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) red_f[warp] = amax;
    __syncthreads();
    amax = 0.0f;
#pragma unroll
    for (int w = 0; w < kPrepThreads / 32; ++w) amax = fmaxf(amax, red_f[w]);
    const double mult = amax > 0.0f ? 1073741824.0 / (double)amax : 0.0;  // 2^30 / absmax
    if (tid == 0 && live) src.tok_scale[t] = (double)amax / 1073741824.0;
#pragma unroll
    for (int j = 0; j < kQ; ++j) {
      const float e4[4] = {xv[j].x, xv[j].y, xv[j].z, xv[j].w};
      word[j][0] = word[j][1] = word[j][2] = word[j][3] = 0u;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int X = __double2int_rn((double)e4[e] * mult);
#pragma unroll
        for (int d = 0; d < 3; ++d) {
          const int lo = ((X & 0xFF) ^ 0x80) - 0x80;  // signed low digit
          word[j][d] |= (uint32_t)(lo & 0xFF) << (8 * e);
          cs[d] += lo;
          X = (X - lo) >> 8;
        }
        word[j][3] |= (uint32_t)(X & 0xFF) << (8 * e);  // |X| <= 65 here
        cs[3] += X;
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < kQ; ++j) {
      const int qi = tid + j * kPrepThreads;
      uint32_t wv = 0u;
      if (live && qi < nquads) {
        const int8_t* q = static_cast<const int8_t*>(src.x) + (int64_t)t * src.K;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int64_t k = 4 * (int64_t)qi + e;
          const int v = k < src.K ? q[k] : 0;
          wv |= (uint32_t)(v & 0xFF) << (8 * e);
          cs[0] += v;
        }
      }
      word[j][0] = wv;
    }
  }
#pragma unroll
  for (int j = 0; j < kQ; ++j) {
    const int qi = tid + j * kPrepThreads;
    if (qi >= nquads) break;
    const int64_t chunk = qi >> 5;
    const int kin = (qi & 31) * 4;
    const int rr = (kin >> 2) & 3, ks = kin >> 5, kk = (kin >> 4) & 1;
    for (int d = 0; d < D; ++d) {
      const int n = t * D + d;
      src.frag[((chunk * 2 + (n >> 3)) * 32 + 4 * (n & 7) + rr) * 8 + 2 * ks + kk] = word[j][d];
    }
  }
  // column sums
#pragma unroll
  for (int d = 0; d < 4; ++d) {
    int v = cs[d];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red_i[warp][d] = v;
  }
  __syncthreads();
  if (tid < D) {
    int v = 0;
#pragma unroll
    for (int w = 0; w < kPrepThreads / 32; ++w) v += red_i[w][tid];
    src.colsum[t * D + tid] = v;
  }
}

template <int NB>
int launch_nb(const GvBatch& batch, int64_t ctas, size_t smem, cudaStream_t s) {
  static int attr_smem = 0;  // per template instance
  if ((int)smem > attr_smem) {
    FT_CUDA(cudaFuncSetAttribute(gemv_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem));
    attr_smem = (int)smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctas);
  cfg.blockDim = dim3(kGvWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FT_CUDA(cudaLaunchKernelEx(&cfg, gemv_kernel<NB>, batch));
  FT_LAUNCH_CHECK();
  return FT_OK;
}

}  // namespace

bool gemv_fits(const ft_weight* w, int64_t seq, int xkind) {
  const int digits = xkind == 2 ? 1 : 4;
  const int64_t ncols = seq * digits;
  if (w->format != 0 || ncols > 16) return false;
  const int64_t nb = ncols > 8 ? 2 : 1;
  return kRingBytes + w->n_chunks * nb * 1024 <= kGemvMaxSmem;
}

int launch_gemv(ft_ctx* ctx, int nprob, const GvLaunchProblem* probs, int xkind,
                cudaStream_t s) {
  FT_CHECK(nprob > 0 && nprob <= kGvMaxProblems, FT_ERR_UNSUPPORTED, "bad GEMV group size");
  static thread_local GvBatch batch;
  batch.nprob = nprob;
  batch.digits = xkind == 2 ? 1 : 4;
  int64_t mblocks = 0, max_nch = 0, max_cols = 0;
  for (int i = 0; i < nprob; ++i) {
    mblocks += probs[i].n_tiles * 8;
    max_nch = probs[i].n_chunks > max_nch ? probs[i].n_chunks : max_nch;
    const int64_t nc = probs[i].seq * batch.digits;
    max_cols = nc > max_cols ? nc : max_cols;
  }
  batch.nb = max_cols > 8 ? 2 : 1;
  // K splits: enough warps for ~32 per SM, but a split keeps >= 8 chunks
  const int64_t want_warps = (int64_t)ctx->num_sms * 32;
  int64_t ctas = 0;
  for (int i = 0; i < nprob; ++i) {
    const GvLaunchProblem& q = probs[i];
    GvProblem& p = batch.p[i];
    int S = 1;
    while (S < 8 && mblocks * S < want_warps && q.n_chunks >= 8 * S) S *= 2;
    p.codes = reinterpret_cast<const uint4*>(q.codes);
    p.row_scales = q.row_scales;
    p.rows = q.rows;
    p.n_tiles = q.n_tiles;
    p.n_chunks = q.n_chunks;
    p.bfrag = reinterpret_cast<const uint4*>(q.bmat);
    p.colsum = q.colsum;
    p.tok_scale = q.tok_scale;
    p.sx = q.sx;
    p.y = q.y;
    p.ldy = q.ldy;
    p.seq = q.seq;
    p.ksplit = S;
    p.cps = (int)ceil_div(q.n_chunks, S);
    p.cta_begin = ctas;
    ctas += ceil_div(q.n_tiles * 8, kGvWarps / S);
  }
  FT_CHECK(ctas <= 0x7FFFFFFF, FT_ERR_UNSUPPORTED, "GEMV grid too large");
  const size_t smem = (size_t)kRingBytes + (size_t)max_nch * batch.nb * 1024;
  FT_CHECK(smem <= (size_t)kGemvMaxSmem, FT_ERR_UNSUPPORTED, "GEMV operand too large");
  static_assert(kRingBytes >= kGvWarps * 32 * 8 * 4, "split sums reuse the ring");
  return batch.nb == 1 ? launch_nb<1>(batch, ctas, smem, s) : launch_nb<2>(batch, ctas, smem, s);
}

int launch_gemv_prep(int nsrc, const GvPrepSource* srcs, int xkind, int nb, cudaStream_t s) {
  FT_CHECK(nsrc > 0 && nsrc <= kMaxFragSources, FT_ERR_UNSUPPORTED, "bad source count");
  static thread_local FragBatch fb;
  fb.nsrc = nsrc;
  fb.xkind = xkind;
  fb.D = xkind == 2 ? 1 : 4;
  fb.slots = 8 * nb / fb.D;
  for (int i = 0; i < nsrc; ++i) {
    FT_CHECK(srcs[i].n_chunks * 32 <= 4 * kPrepThreads, FT_ERR_UNSUPPORTED,
             "K too large for the decode prep");
    fb.s[i] = FragSource{srcs[i].x, reinterpret_cast<uint32_t*>(srcs[i].frag), srcs[i].colsum,
                         srcs[i].tok_scale, srcs[i].K, srcs[i].n_chunks, srcs[i].seq};
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(nsrc * fb.slots));
  cfg.blockDim = dim3(kPrepThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FT_CUDA(cudaLaunchKernelEx(&cfg, prep_frag_kernel, fb));
  FT_LAUNCH_CHECK();
  return FT_OK;
}

}  // namespace ft
