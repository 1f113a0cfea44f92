// Decode-shape ternary matmul (GEMV and small M): y = scale * (W . x) for a
// group of independent problems whose activations fit one 16-column operand
// (fp32/bf16: <= 4 tokens as 4 base-256 digits each; int8: <= 16 tokens).
//
// Same exact formulation as the tensor-core engine (ft_tc.cu): the A operand
// is the unsigned codes u = w + 1, the B operand the int8 activation columns
// written by prep_b_kernel, int32 sums are exact, the epilogue subtracts the
// column sums and scales.  Here the MMAs are warp-level (mma.sync m16n8k32):
// every lane loads its 16 bytes of a 4 KB weight block straight from global
// memory with one coalesced 128-bit load (the lane-major block layout puts a
// warp's 512 bytes of an m-block contiguous), unpacks each word with one shift
// and one mask per fragment register, and issues 4 MMAs per n-block.  The
// weight stream needs no shared memory, barriers or TMEM, so a decode GEMV
// runs at the memory system's pace.
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
constexpr int kNpad = 16;  // activation columns (two n8 blocks)
constexpr int kUnroll = 4;  // weight loads in flight per lane

struct GvProblem {
  const uint4* codes;  // lane-major blocks, 256 uint4 per (tile, chunk)
  const float* row_scales;
  int64_t rows, n_tiles, n_chunks;
  const int8_t* bmat;      // [n_chunks][kNpad * 128] (prep_b_kernel, one pass)
  const int32_t* colsum;   // [kNpad]
  const double* tok_scale; // fp32 mode: absmax * 2^-30 per token
  const float* sx;         // int8 mode: per-token scale
  float* y;
  int64_t ldy, seq;
  int64_t cta_begin;       // first CTA of this problem
  int ksplit, cps, nb;     // K splits, chunks per split, live n8 blocks (1 or 2)
};

struct GvBatch {
  int nprob;
  int digits;
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

__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// the 4 MMAs of one 128-K chunk for n8 blocks 0 .. NB-1
template <int NB>
__device__ __forceinline__ void chunk_mma(int (&acc)[2][4], const uint4 w, const int8_t* bchunk,
                                          int g, int r) {
  const uint32_t wk[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    const uint32_t a0 = wk[ks] & 0x03030303u;
    const uint32_t a1 = (wk[ks] >> 2) & 0x03030303u;
    const uint32_t a2 = (wk[ks] >> 4) & 0x03030303u;
    const uint32_t a3 = (wk[ks] >> 6) & 0x03030303u;
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      // B column n = g of n8 block nb; k 4r..4r+3 (k16 group 2ks) and 16+4r.. (2ks+1)
      const int8_t* bp = bchunk + ((2 * ks) * (kNpad / 8) + nb) * 128 + g * 16 + 4 * r;
      const uint32_t b0 = __ldg(reinterpret_cast<const uint32_t*>(bp));
      const uint32_t b1 = __ldg(reinterpret_cast<const uint32_t*>(bp + (kNpad / 8) * 128));
      mma_u8s8(acc[nb], a0, a1, a2, a3, b0, b1);
    }
  }
}

template <int NB>
__global__ void __launch_bounds__(kGvWarps * 32) gemv_kernel(const __grid_constant__ GvBatch b) {
  int pi = 0;
  while (pi + 1 < b.nprob && b.p[pi + 1].cta_begin <= (int64_t)blockIdx.x) ++pi;
  const GvProblem& p = b.p[pi];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
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

  int acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
  const uint4* wp = p.codes + (tile * p.n_chunks) * 256 + mb * 32 + lane;
  // the first weights do not depend on the previous launch: start them before
  // waiting for the prep kernel that writes the activation operand
  uint4 w[kUnroll];
#pragma unroll
  for (int u = 0; u < kUnroll; ++u)
    if (c0 + u < c1) w[u] = ldg_stream(wp + (c0 + u) * 256);
  tc::pdl_wait();
  for (int64_t c = c0; c < c1; c += kUnroll) {
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (c + u < c1) {
        const uint4 cur = w[u];
        if (c + u + kUnroll < c1) w[u] = ldg_stream(wp + (c + u + kUnroll) * 256);
        chunk_mma<NB>(acc, cur, p.bmat + (c + u) * (kNpad * 128), g, r);
      }
    }
  }

  // ---- combine the K splits of each m-block in shared memory
  __shared__ int red[kGvWarps][32][8];
  if (S > 1) {
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
  if (b.digits == 1) {
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int n = 8 * nb + 2 * r + (i & 1);
        const int64_t R = R0 + 8 * (i >> 1);
        if (n < p.seq && R < p.rows) {
          const int32_t a = acc[nb][i] - p.colsum[n];
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
        if (t < p.seq) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int64_t R = R0 + 8 * h;
            if (R >= p.rows) continue;
            const long long d0 = acc[nb][2 * h] - p.colsum[n0];
            const long long d1 = acc[nb][2 * h + 1] - p.colsum[n0 + 1];
            const long long d2 = (h ? hi2 : hi0) - p.colsum[n0 + 2];
            const long long d3 = (h ? hi3 : hi1) - p.colsum[n0 + 3];
            const long long S4 = d0 + d1 * 256 + d2 * 65536 + d3 * 16777216;
            p.y[t * p.ldy + R] =
                (float)((double)S4 * p.tok_scale[t] * (double)p.row_scales[R]);
          }
        }
      }
    }
  }
}

}  // namespace

// Launches the decode-shape kernel for problems whose prep output (npad 16,
// one pass) is ready in the workspace.  `probs` carries everything but the
// work split, which is chosen here.
int launch_gemv(ft_ctx* ctx, int nprob, const GvLaunchProblem* probs, int digits,
                cudaStream_t s) {
  FT_CHECK(nprob > 0 && nprob <= kGvMaxProblems, FT_ERR_UNSUPPORTED, "bad GEMV group size");
  static thread_local GvBatch batch;
  batch.nprob = nprob;
  batch.digits = digits;
  int64_t mblocks = 0;
  int nbmax = 1;
  for (int i = 0; i < nprob; ++i) mblocks += probs[i].n_tiles * 8;
  // K splits: enough warps for ~32 per SM, but a split keeps >= 2 chunks
  const int64_t want_warps = (int64_t)ctx->num_sms * 32;
  int64_t ctas = 0;
  for (int i = 0; i < nprob; ++i) {
    const GvLaunchProblem& q = probs[i];
    GvProblem& p = batch.p[i];
    int S = 1;
    while (S < 8 && mblocks * S < want_warps && q.n_chunks >= 4 * S) S *= 2;
    p.codes = reinterpret_cast<const uint4*>(q.codes);
    p.row_scales = q.row_scales;
    p.rows = q.rows;
    p.n_tiles = q.n_tiles;
    p.n_chunks = q.n_chunks;
    p.bmat = q.bmat;
    p.colsum = q.colsum;
    p.tok_scale = q.tok_scale;
    p.sx = q.sx;
    p.y = q.y;
    p.ldy = q.ldy;
    p.seq = q.seq;
    p.ksplit = S;
    p.cps = (int)ceil_div(q.n_chunks, S);
    p.nb = (int)((q.seq * digits + 7) / 8);
    if (p.nb > nbmax) nbmax = p.nb;
    p.cta_begin = ctas;
    ctas += ceil_div(q.n_tiles * 8, kGvWarps / S);
  }
  FT_CHECK(ctas <= 0x7FFFFFFF, FT_ERR_UNSUPPORTED, "GEMV grid too large");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctas);
  cfg.blockDim = dim3(kGvWarps * 32);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (nbmax == 1)
    FT_CUDA(cudaLaunchKernelEx(&cfg, gemv_kernel<1>, batch));
  else
    FT_CUDA(cudaLaunchKernelEx(&cfg, gemv_kernel<2>, batch));
  FT_LAUNCH_CHECK();
  return FT_OK;
}

}  // namespace ft
