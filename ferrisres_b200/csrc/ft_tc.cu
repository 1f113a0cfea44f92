// Tensor-core (tcgen05, sm_100a) ternary matmul: y = scale * (W . x), for a
// group of independent problems in one persistent launch.
//
// Formulation.  The packed 2-bit codes u = w + 1 in {0, 1, 2} are unpacked
// in registers (one shift + one mask per 4 codes, thanks to the lane-major
// T128 layout) and written to tensor memory as the 8-bit A operand (M = 128
// output channels of one tile).  The activations are the signed 8-bit B
// operand, K-major in shared memory, N = NPAD columns:
//   * int8 mode: one column per token, the caller's int8 codes q;
//   * fp32/bf16 mode: D columns per token (D = 8, or 4 for the MoE experts),
//     the signed base-256 digits of the fixed-point image X = round(x * 2^sh),
//     2^sh the power of two that puts the token's largest finite |x| in
//     [2^(8D-3), 2^(8D-2)).
// tcgen05.mma kind::i8 accumulates exact int32 sums D = sum_k u_k b_k in TMEM;
// the epilogue subtracts sum_k b_k (so D becomes sum_k w_k b_k) and scales:
//   int8: y = ((float)D * sx[s]) * scale[r]      (bit-exact vs the reference)
//   fp32: y = (double)(sum_d D_d * 256^d) * 2^-sh * scale[r]
// With D = 8 every element within 2^38 of the token's absmax is exact, so the
// result is the correctly rounded dot product.  Non-finite activations enter
// as 0; the prep kernel lists their positions per token (a negative token
// scale flags them) and the epilogue finishes the rows that meet them by the
// reference's rule (nonfinite_row, ft_internal.cuh).
//
// Work items.  A problem (one weight, its activations and output) is cut
// into items = (column pass, 128-row tile, K range).  The launch is persistent:
// CTA b takes items b, b + grid, b + 2*grid, ...  Warp roles (352 threads):
//   warp 4     weight producer: 1-D bulk copies of the 4 KB (tile, chunk)
//              blocks into a 16-deep smem ring (64 KB in flight per CTA),
//              running ahead across item boundaries.
//   warp 5     B producer: bulk copies of the B chunks into their own ring.
//   warps 0-3 (+ 11.. for further groups) converters, in groups of 4 warps
//              (one per TMEM sub-partition) taking alternate super-stages:
//              a warp reads its two m-blocks of the lane-major block as two
//              conflict-free 512-byte rows, unpacks each lane's 16 bytes and
//              writes them with one 16x128b tcgen05.st per m-block (the store
//              shape's lane/column map is the block's lane map).
//   warp 6     MMA issuer: 4 x tcgen05.mma (K = 32 each) per chunk into one of
//              two TMEM accumulators; tcgen05.commit frees stages / signals D.
//              Also owns the TMEM allocation.
//   warps 7-10 epilogue: tcgen05.ld of the finished accumulator, release it,
//              then scale and store (or add split-K partials).
// Split-K partials are combined with exact int32 atomics in a zero-initialised
// scratch area; the last CTA of a tile (atomic ticket) runs the final
// epilogue and clears the scratch again, so it stays zero between calls.
#include <cstring>
#include <type_traits>

#include "ft_internal.cuh"
#include "ft_tc.cuh"

namespace ft {
namespace {

#ifndef FT_TC_SA
#define FT_TC_SA 16
#endif
#ifndef FT_TC_BBUDGET
#define FT_TC_BBUDGET 98304
#endif
constexpr int kSK = 2;   // K chunks per super-stage: one barrier wait / commit per 8 KB of weights
constexpr int kWarpLoadA = 4, kWarpLoadB = 5, kWarpMma = 6;  // warps 0-3 convert, 7-10 epilogue
constexpr int kMaxProblems = 64;

struct TqProblem {
  const uint8_t* codes;
  const float* row_scales;
  int64_t rows, n_tiles, n_chunks;
  const int8_t* bmat;       // [passes][n_chunks][NPAD*128]
  const int32_t* colsum;    // [passes][NPAD]
  const double* tok_scale;  // fp32 mode: 2^-sh per token, negative when the token has
                            // non-finite elements
  const int32_t* nf;        // fp32 mode: per token [count, kNfCap positions]
  const void* x;            // fp32 mode: the activations (read by the non-finite fix-up)
  int64_t K;
  const float* kscale;      // fp32 mode: column-block scales folded into x, or null
  int64_t kblock;
  const float* sx;          // int8 mode: per-token scale
  float* y;                 // y[t * ldy + r]
  int64_t ldy;
  int64_t seq;
  int tok_per_pass, passes, ksplit, cps;
  int32_t* acc;             // [passes][n_tiles][NPAD][128], zero between calls
  int32_t* cnt;             // [passes][n_tiles], zero between calls
  int64_t item_begin;
  // activation rows: x + t * ldx (ldx = K, or the interleaved gate/up width
  // when act != 0: element k = act(gate_k, up_k), see act_operand)
  int64_t ldx;
  int act;
};

struct TqBatch {
  int nprob;
  int digits;
  int bf16;  // fp32 mode: activations are bf16 bit patterns
  int64_t total_items;
  int* err;
  // first item of each problem, contiguous (item decoding reads only this)
  int64_t item_begin[kMaxProblems + 1];
  TqProblem p[kMaxProblems];
};

struct Item {
  int prob;
  int pass;
  int64_t tile;
  int64_t c0;
  int nch;
};

__device__ __forceinline__ Item decode_item(const TqBatch& b, int64_t item) {
  // the last problem whose first item is <= item (binary search)
  int lo = 0, hi = b.nprob - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (b.item_begin[mid] <= item) lo = mid;
    else hi = mid - 1;
  }
  const int pi = lo;
  const TqProblem& p = b.p[pi];
  int64_t local = item - b.item_begin[pi];
  Item it;
  it.prob = pi;
  const int ks = (int)(local % p.ksplit);
  local /= p.ksplit;
  it.tile = local % p.n_tiles;
  it.pass = (int)(local / p.n_tiles);
  it.c0 = (int64_t)ks * p.cps;
  int64_t c1 = it.c0 + p.cps;
  if (c1 > p.n_chunks) c1 = p.n_chunks;
  it.nch = (int)(c1 - it.c0);
  return it;
}

// Walks the (item, chunk) sequence of this CTA.
struct Cursor {
  int64_t item;
  int chunk;
  Item it;
  __device__ __forceinline__ void start(const TqBatch& b) {
    item = blockIdx.x;
    chunk = 0;
    if (item < b.total_items) it = decode_item(b, item);
  }
  __device__ __forceinline__ bool valid(const TqBatch& b) const { return item < b.total_items; }
  // chunks in the super-stage that starts at `chunk` (never spans two items)
  __device__ __forceinline__ int ss_len() const {
    return it.nch - chunk < kSK ? it.nch - chunk : kSK;
  }
  __device__ __forceinline__ bool advance_ss(const TqBatch& b) {
    chunk += ss_len();
    if (chunk < it.nch) return false;
    chunk = 0;
    item += gridDim.x;
    if (item < b.total_items) it = decode_item(b, item);
    return true;
  }
};

__host__ __device__ constexpr int dbufs_for(int npad) { return npad <= 128 ? 2 : 1; }
__host__ __device__ constexpr uint32_t dstride_for(int npad) { return (uint32_t)((npad + 31) / 32 * 32); }
__host__ __device__ constexpr uint32_t acol0_for(int npad) { return dbufs_for(npad) * dstride_for(npad); }
// TMEM A super-stages (kSK*32 columns each) after the accumulators: within a
// 256-column allocation (two CTAs per SM) when at least two fit, else 512.
__host__ __device__ constexpr int ss_fit(int budget, int npad) {
  return (budget - (int)acol0_for(npad)) / (kSK * 32);
}
__host__ __device__ constexpr int a_ss_for(int npad) {
  return ss_fit(256, npad) >= 2 ? (ss_fit(256, npad) > 4 ? 4 : ss_fit(256, npad))
                                : (ss_fit(512, npad) > 4 ? 4 : ss_fit(512, npad));
}
__host__ __device__ constexpr uint32_t tmem_cols_for(int npad) {
  return acol0_for(npad) + a_ss_for(npad) * kSK * 32 <= 256 ? 256u : 512u;
}
// B-operand smem super-stages, between 2 and 8: within ~46 KB when two CTAs
// share an SM (256 TMEM columns each), else within ~96 KB.
__host__ __device__ constexpr int b_ss_raw(int npad) {
  return (tmem_cols_for(npad) <= 256 ? 47104 : FT_TC_BBUDGET) / (kSK * npad * 128);
}
__host__ __device__ constexpr int b_ss_for(int npad) {
  return b_ss_raw(npad) < 2 ? 2 : b_ss_raw(npad) > 8 ? 8 : b_ss_raw(npad);
}
// Per kernel instance: converter groups of 4 warps (one per TMEM
// sub-partition); group k converts super-stages k, k + G, k + 2G, ...  A
// group's pass over a super-stage is a long chain of waits and short
// latencies, so several groups work at once: three for the 2:4 kernel with
// 128-column passes (its thread-per-row expansion is the slowest role, 70 ->
// 61 us at cfg3 M=64), two otherwise.  A TMEM A stage is reused every SS
// super-stages, a weight slot every SA / kSK and a B stage every SBS: all
// three periods are multiples of G, so each stage and slot always returns to
// the same group, which waited on its previous phase.  (Parity waits tell
// only consecutive phases apart; with a stage shared between groups one could
// pass a wait a phase early: a 3-group build with 4 A stages did, and a
// 2-group build with 3 B stages relied on copies landing in issue order.)
template <int NPAD, bool kSparse>
struct TqCfg {
  static constexpr int G = (kSparse && NPAD == 128) ? 3 : 2;
  static constexpr int THREADS = (11 + 4 * (G - 1)) * 32;  // extra groups are warps 11..
  static constexpr int SA = FT_TC_SA / (kSK * G) * (kSK * G);  // ring of 4 KB weight blocks
  static constexpr int SS = a_ss_for(NPAD) / G * G;
  // B stages: b_ss_for's count rounded up to a multiple of G when that stays
  // within its budget (one CTA per SM: ~200 KB in all), else down
  static constexpr int SBS_UP = (b_ss_for(NPAD) + G - 1) / G * G;
  static constexpr int SBS =
      (tmem_cols_for(NPAD) > 256 && (size_t)SA * 4096 + (size_t)SBS_UP * kSK * NPAD * 128 <= 200 * 1024)
          ? SBS_UP
          : b_ss_for(NPAD) / G * G;
  static constexpr size_t SMEM = (size_t)SA * 4096 + (size_t)SBS * kSK * NPAD * 128;
  static_assert(SS >= G && SA >= kSK * G && SBS >= G, "each converter group needs its own stages");
  static_assert(SS % G == 0 && (SA / kSK) % G == 0 && SBS % G == 0,
                "stage periods must be multiples of G");
  static_assert(SMEM <= 220 * 1024, "shared memory");
};

__device__ __forceinline__ void named_sync_epilogue() {
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

// fp32 output of token t, row R from its digit-sum total S.
template <bool kSparse>
__device__ __forceinline__ float value_fp(const TqProblem& p, bool bf16, int64_t t, int64_t R,
                                          double S) {
  const double ts = p.tok_scale[t];
  float y = (float)(S * fabs(ts) * (double)p.row_scales[R]);
  if (ts < 0.0) {
    const int32_t* nf = p.nf + t * (kNfCap + 1);
    y = nonfinite_row(y, p.codes, kSparse ? 1 : 0, p.n_chunks, R,
                      static_cast<const char*>(p.x) + t * p.ldx * (bf16 ? 2 : 4), bf16, p.K, nf + 1,
                      nf[0], p.row_scales[R], p.kscale, p.kblock, p.act);
  }
  return y;
}

template <bool kSparse>
__device__ __forceinline__ void store_fp(const TqProblem& p, bool bf16, int64_t t, int64_t R,
                                         double S) {
  p.y[t * p.ldy + R] = value_fp<kSparse>(p, bf16, t, R, S);
}

template <int NPAD, bool kSparse>
__device__ __forceinline__ void epilogue_group(const TqProblem& p, int digits, bool bf16, int pass,
                                               int64_t R, int col0, const int32_t (&v)[16]) {
  if (digits == 8) {
#pragma unroll
    for (int c = 0; c < 16; c += 8) {
      const int lt = (col0 + c) >> 3;
      const int64_t t = (int64_t)pass * p.tok_per_pass + lt;
      if (t >= p.seq || lt >= p.tok_per_pass) break;
      double S = 0.0;
#pragma unroll
      for (int d = 0; d < 8; ++d)
        S += (double)(v[c + d] - p.colsum[pass * NPAD + col0 + c + d]) * (double)(1ll << (8 * d));
      store_fp<kSparse>(p, bf16, t, R, S);
    }
    return;
  }
  if (digits == 1) {
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      const int lt = col0 + c;
      const int64_t t = (int64_t)pass * p.tok_per_pass + lt;
      if (t >= p.seq || lt >= p.tok_per_pass) break;
      const int32_t a = v[c] - p.colsum[pass * NPAD + lt];
      p.y[t * p.ldy + R] = __fmul_rn(__fmul_rn((float)a, p.sx[t]), p.row_scales[R]);
    }
  } else {
#pragma unroll
    for (int c = 0; c < 16; c += 4) {
      const int lt = (col0 + c) >> 2;
      const int64_t t = (int64_t)pass * p.tok_per_pass + lt;
      if (t >= p.seq || lt >= p.tok_per_pass) break;
      long long S = 0;
#pragma unroll
      for (int d = 0; d < 4; ++d) {
        const long long a = (long long)(v[c + d] - p.colsum[pass * NPAD + col0 + c + d]);
        S += a * (1ll << (8 * d));
      }
      store_fp<kSparse>(p, bf16, t, R, (double)S);
    }
  }
}

template <int NPAD, bool kSparse>
__global__ void __launch_bounds__(TqCfg<NPAD, kSparse>::THREADS, 1)
    tq_grouped_kernel(const __grid_constant__ TqBatch b) {
  using Cfg = TqCfg<NPAD, kSparse>;
  constexpr int kSA = Cfg::SA, kConvGroups = Cfg::G;
  // weight block bytes in HBM and in the smem ring (2:4 blocks use the first 3072 bytes)
  constexpr uint32_t kBlk = kSparse ? kSparseBlockBytes : kBlockBytes;
  // 2:4 group (metadata nibble << 2 | the two sign bits) -> four unsigned
  // codes w + 1 (bytes in K order)
  __shared__ uint32_t s_lut[64];
  // dynamic smem: [kSA weight blocks of 4096 B][kSBS B super-stages of kSK*NPAD*128 B]
  extern __shared__ __align__(1024) uint8_t smem_dyn[];
  constexpr uint32_t kBStage = NPAD * 128;       // B bytes per chunk
  constexpr uint32_t kBSuper = kSK * kBStage;    // B bytes per super-stage
  constexpr int kSBS = Cfg::SBS;
  constexpr int kSS = Cfg::SS;
  uint8_t* const smem_a = smem_dyn;
  uint8_t* const smem_b = smem_dyn + kSA * kBlockBytes;
  __shared__ __align__(8) uint64_t bar_sa_full[kSA];    // weight block landed (tx)
  __shared__ __align__(8) uint64_t bar_sa_empty[kSA];   // converters done reading it (4)
  __shared__ __align__(8) uint64_t bar_sb_full[kSBS];   // B super-stage landed (tx)
  __shared__ __align__(8) uint64_t bar_sb_empty[kSBS];  // MMA done with it (commit)
  __shared__ __align__(8) uint64_t bar_afull[kSS];      // TMEM A super-stage written, B landed (4)
  __shared__ __align__(8) uint64_t bar_free[kSS];       // TMEM A super-stage consumed (commit)
  __shared__ __align__(8) uint64_t bar_dfull[2];
  __shared__ __align__(8) uint64_t bar_dfree[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ int last_flag;

  constexpr uint32_t kLBO = (NPAD / 8) * 128;  // K-direction core-matrix stride
  constexpr uint32_t kSBO = 128;               // N-direction 8-row group stride
  constexpr int kDBufs = dbufs_for(NPAD);
  constexpr uint32_t kDStride = dstride_for(NPAD);
  constexpr uint32_t kACol0 = acol0_for(NPAD);
  constexpr uint32_t kTmemCols = tmem_cols_for(NPAD);
  constexpr uint32_t kIdesc = tc::idesc_i8(128, NPAD);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (kSparse && threadIdx.x < 64) {
    const uint32_t c = threadIdx.x, i0 = (c >> 2) & 3u, i1 = c >> 4;
    uint32_t v = 0x01010101u;
    v ^= ((c & 1u) ? 1u : 3u) << (8 * i0);  // byte 1 -> 0 (w = -1) or 2 (w = +1)
    v ^= ((c & 2u) ? 1u : 3u) << (8 * i1);
    s_lut[c] = v;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSA; ++s) {
      tc::mbar_init(tc::smem_u32(&bar_sa_full[s]), 1);
      tc::mbar_init(tc::smem_u32(&bar_sa_empty[s]), 4);
    }
    for (int s = 0; s < kSBS; ++s) {
      tc::mbar_init(tc::smem_u32(&bar_sb_full[s]), 1);
      tc::mbar_init(tc::smem_u32(&bar_sb_empty[s]), 1);
    }
    for (int s = 0; s < kSS; ++s) {
      tc::mbar_init(tc::smem_u32(&bar_afull[s]), 4);
      tc::mbar_init(tc::smem_u32(&bar_free[s]), 1);
    }
    for (int d = 0; d < 2; ++d) {
      tc::mbar_init(tc::smem_u32(&bar_dfull[d]), 1);
      tc::mbar_init(tc::smem_u32(&bar_dfree[d]), 4);
    }
    tc::fence_barrier_init();
  }
  if (warp == kWarpMma) tc::tmem_alloc(tc::smem_u32(&tmem_base_sh), kTmemCols);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  tc::pdl_launch_dependents();
  const uint32_t tmem = tmem_base_sh;
  bool ok = true;

  if (warp < 4 || warp >= 11) {
    // ------------------------------------------------------ converters --
    const int cgroup = warp < 4 ? 0 : 1 + (warp - 11) / 4;
    const int sub = warp & 3;       // warp w may only touch TMEM lanes 32(w%4)..+31
    const int r = sub * 32 + lane;  // the tile row (TMEM lane) this thread converts
    const uint32_t lane_off = (uint32_t)(32 * sub) << 16;
    Cursor cs;
    cs.start(b);
    uint32_t gb = 0, gs = 0;  // weight-block and super-stage counters
    // this group's first super-stage
    for (int k = 0; k < cgroup && cs.valid(b); ++k) {
      gb += (uint32_t)cs.ss_len();
      ++gs;
      cs.advance_ss(b);
    }
    while (cs.valid(b)) {
      const int n = cs.ss_len();
      uint32_t wv[kSK][8];  // 2:4 sparse: row r's 4 metadata words and 4 sign words per chunk
      uint4 wd[kSK][2];     // dense: this lane's 16 bytes of m-blocks 2*sub and 2*sub+1
#pragma unroll
      for (int j = 0; j < kSK; ++j) {
        if (j < n) {
          const uint32_t sa = gb % kSA;
          ok = ok && tc::mbar_wait(tc::smem_u32(&bar_sa_full[sa]), (gb / kSA) & 1, b.err, 10);
          if (kSparse) {
            // row r's metadata (groups 0-7 and 8-15 of both k64 steps) and the
            // sign words of the 4 lanes holding its values
            const unsigned char* mbr = smem_a + sa * kBlockBytes + (r >> 4) * kSparseMbBytes;
            const uint32_t* mw = reinterpret_cast<const uint32_t*>(mbr);
            const uint32_t* sw = reinterpret_cast<const uint32_t*>(mbr + 256);
            const int g8 = r & 7, h8 = (r >> 3) & 1;
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              wv[j][2 * i] = ok ? mw[2 * (4 * g8 + 2 * i + h8)] : 0u;
              wv[j][2 * i + 1] = ok ? mw[2 * (4 * g8 + 2 * i + h8) + 1] : 0u;
            }
#pragma unroll
            for (int t2 = 0; t2 < 4; ++t2) wv[j][4 + t2] = ok ? sw[4 * g8 + t2] : 0u;
          } else {
            // the warp reads its two m-blocks as 2 x 512 contiguous bytes
            const uint4* blk = reinterpret_cast<const uint4*>(smem_a + sa * kBlockBytes);
#pragma unroll
            for (int m = 0; m < 2; ++m)
              wd[j][m] = ok ? blk[(2 * sub + m) * 32 + lane] : make_uint4(0, 0, 0, 0);
          }
          ++gb;
        }
      }
      const uint32_t s = gs % kSS;
      if (ok && gs >= (uint32_t)kSS)
        ok = tc::mbar_wait(tc::smem_u32(&bar_free[s]), ((gs / kSS) + 1) & 1, b.err, 11);
      ok = __all_sync(0xffffffffu, ok);  // tcgen05.st below is warp-collective
      tc::tc_fence_after();
#pragma unroll
      for (int j = 0; j < kSK; ++j) {
        if (j < n) {
          const uint32_t col = kACol0 + (s * kSK + j) * 32;
          if (kSparse) {
            const int h8 = (r >> 3) & 1;
#pragma unroll
            for (int h = 0; h < 2; ++h) {  // k64 step h: 16 groups = 16 TMEM columns
              uint32_t a[16];
#pragma unroll
              for (int gg = 0; gg < 16; ++gg) {  // group gg covers K 4gg..4gg+3
                const uint32_t meta = wv[j][2 * (gg >> 3) + h];
                const uint32_t nib = (meta >> (4 * (gg & 7))) & 0xFu;
                const uint32_t sgw = wv[j][4 + ((gg & 7) >> 1)] >> (16 * h);
                const uint32_t sb = (sgw >> (4 * (2 * (gg >> 3) + h8) + 2 * (gg & 1))) & 3u;
                a[gg] = s_lut[(nib << 2) | sb];
              }
              if (ok) tc::tmem_st_x16(tmem + lane_off + col + 16 * h, a);
            }
          } else {
            // Lane (g, r) of an m-block holds word i of k-step j's fragment:
            // row g + 8(i&1), TMEM column 8j + 4(i>>1) + r = the 16x128b
            // store's register 4j + i.  One store per m-block.
#pragma unroll
            for (int m = 0; m < 2; ++m) {
              const uint32_t w4[4] = {wd[j][m].x, wd[j][m].y, wd[j][m].z, wd[j][m].w};
              uint32_t a[16];
#pragma unroll
              for (int kj = 0; kj < 4; ++kj)
#pragma unroll
                for (int i = 0; i < 4; ++i) a[4 * kj + i] = (w4[i] >> (2 * kj)) & 0x03030303u;
              if (ok)
                tc::tmem_st_16x128b_x8(tmem + ((uint32_t)(32 * sub + 16 * m) << 16) + col, a);
            }
          }
        }
      }
      tc::tmem_wait_st();
      // Release the weight slots only now: the TMEM stores above consumed the
      // registers the shared loads filled, so those loads have completed and
      // the producer's next bulk copy cannot overwrite a slot still being read.
      __syncwarp();
      if (lane == 0)
        for (int j = 0; j < n; ++j)
          tc::mbar_arrive(tc::smem_u32(&bar_sa_empty[(gb - n + j) % kSA]));
      // The B super-stage is waited here too, so the MMA thread waits on one
      // barrier per super-stage.
      ok = ok && tc::mbar_wait(tc::smem_u32(&bar_sb_full[gs % kSBS]), (gs / kSBS) & 1, b.err, 18);
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(tc::smem_u32(&bar_afull[s]));
      ++gs;
      cs.advance_ss(b);
      // skip the other groups' super-stages
      for (int k = 1; k < kConvGroups && cs.valid(b); ++k) {
        gb += (uint32_t)cs.ss_len();
        ++gs;
        cs.advance_ss(b);
      }
    }
  } else if (warp == kWarpLoadA) {
    // ------------------------------------------- weight-block producer --
    // One super-stage (its one or two 4 KB blocks) per step: the whole warp
    // waits for the free slots, then an elect.sync lane issues the copies back
    // to back.  A wait issued right after a copy costs the copy's issue on
    // B200 (several hundred cycles with the activation copies in flight): a
    // wait-copy-wait-copy loop supplied one block per ~600 cycles, slower
    // than the MMAs consume them.
    {
      Cursor cs;
      cs.start(b);
      uint32_t gb = 0;
      while (cs.valid(b) && ok) {
        const TqProblem& p = b.p[cs.it.prob];
        const int n = cs.ss_len();
#pragma unroll
        for (int j = 0; j < kSK; ++j)
          if (j < n && gb + j >= (uint32_t)kSA)
            ok = ok && tc::mbar_wait(tc::smem_u32(&bar_sa_empty[(gb + j) % kSA]),
                                     (((gb + j) / kSA) + 1) & 1, b.err, 17);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        uint32_t leader;
        if (tc::elect_one(leader)) {
          const uint8_t* src = p.codes + (cs.it.tile * p.n_chunks + cs.it.c0 + cs.chunk) * kBlk;
#pragma unroll
          for (int j = 0; j < kSK; ++j) {
            if (j < n) {
              const uint32_t sa = (gb + j) % kSA;
              const uint32_t bar = tc::smem_u32(&bar_sa_full[sa]);
              tc::mbar_arrive_expect_tx(bar, kBlk);
              tc::bulk_g2s(tc::smem_u32(smem_a + sa * kBlockBytes), src + j * kBlk, kBlk, bar);
            }
          }
        }
        __syncwarp();
        gb += (uint32_t)n;
        cs.advance_ss(b);
      }
    }
  } else if (warp == kWarpLoadB) {
    // ------------------------------------------- B super-stage producer --
    // (same form as the weight producer)
    {
      tc::pdl_wait();  // B is written by the preceding prep kernel
      Cursor cs;
      cs.start(b);
      uint32_t gs = 0;
      while (cs.valid(b) && ok) {
        const TqProblem& p = b.p[cs.it.prob];
        const uint32_t n = (uint32_t)cs.ss_len();
        const uint32_t sb = gs % kSBS;
        if (gs >= (uint32_t)kSBS)
          ok = tc::mbar_wait(tc::smem_u32(&bar_sb_empty[sb]), ((gs / kSBS) + 1) & 1, b.err, 12);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        uint32_t leader;
        if (tc::elect_one(leader)) {
          const uint32_t bar = tc::smem_u32(&bar_sb_full[sb]);
          tc::mbar_arrive_expect_tx(bar, n * kBStage);
          // the super-stage's chunks are contiguous in the prepared operand
          const int8_t* src =
              p.bmat + ((int64_t)cs.it.pass * p.n_chunks + cs.it.c0 + cs.chunk) * kBStage;
          tc::bulk_g2s(tc::smem_u32(smem_b + sb * kBSuper), src, n * kBStage, bar);
        }
        __syncwarp();
        ++gs;
        cs.advance_ss(b);
      }
    }
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------ MMA issuer --
    // The whole warp runs the loop and waits on the barriers; one lane chosen
    // by elect.sync issues a super-stage's MMAs and commits.  Measured on B200
    // (M=128, N=128, kind::i8): issuing from a lone `lane == 0` thread that
    // waits between batches costs ~100 cycles per MMA, this form ~72 (64 with
    // no waits at all).  A super-stage is straight-line code; ring slots and
    // phases advance by counters.  tcgen05.commit tracks the MMAs of the lane
    // that executes it, so the MMAs and the commits that cover them are
    // issued in one elected block (elect.sync picks the same lane each time:
    // the lowest active one; a different lane is reported as an error).
    static_assert(kSK == 2, "the issue loop is written for two chunks per super-stage");
    {
      const uint64_t bdesc0 = tc::smem_desc(tc::smem_u32(smem_b), kLBO, kSBO);
      constexpr uint64_t kKStep = (uint64_t)((2 * kLBO) >> 4);  // descriptor step of K = 32
      constexpr uint64_t kBChunkDesc = (uint64_t)(kBStage >> 4);
      Cursor cs;
      cs.start(b);
      uint32_t s = 0, s_par = 0, sb = 0, ic = 0;
      while (cs.valid(b) && ok) {
        const uint32_t d = ic & (kDBufs - 1);
        if (ic >= (uint32_t)kDBufs)
          ok = tc::mbar_wait(tc::smem_u32(&bar_dfree[d]), ((ic / kDBufs) + 1) & 1, b.err, 13);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc::tc_fence_after();
        const uint32_t dcol = tmem + d * kDStride;
        uint32_t acc = 0u;  // the item's first MMA overwrites the accumulator
        bool item_done = false;
        while (!item_done) {
          const int n = cs.ss_len();
          const bool last = cs.chunk + n >= cs.it.nch;  // the item's last super-stage
          ok = tc::mbar_wait(tc::smem_u32(&bar_afull[s]), s_par, b.err, 14);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
          tc::tc_fence_after();
          uint32_t leader;
          if (tc::elect_one(leader)) {
            if (leader != 0u) atomicCAS(b.err, 0, 19);
            const uint64_t bd = bdesc0 + (uint64_t)((sb * kBSuper) >> 4);
            const uint32_t aa = tmem + kACol0 + s * (kSK * 32);
            tc::mma_i8_ts(dcol, aa, bd, kIdesc, acc);
            tc::mma_i8_ts(dcol, aa + 8, bd + kKStep, kIdesc, 1u);
            tc::mma_i8_ts(dcol, aa + 16, bd + 2 * kKStep, kIdesc, 1u);
            tc::mma_i8_ts(dcol, aa + 24, bd + 3 * kKStep, kIdesc, 1u);
            if (n > 1) {
              const uint64_t bd1 = bd + kBChunkDesc;
              tc::mma_i8_ts(dcol, aa + 32, bd1, kIdesc, 1u);
              tc::mma_i8_ts(dcol, aa + 40, bd1 + kKStep, kIdesc, 1u);
              tc::mma_i8_ts(dcol, aa + 48, bd1 + 2 * kKStep, kIdesc, 1u);
              tc::mma_i8_ts(dcol, aa + 56, bd1 + 3 * kKStep, kIdesc, 1u);
            }
            tc::mma_commit(tc::smem_u32(&bar_free[s]));
            tc::mma_commit(tc::smem_u32(&bar_sb_empty[sb]));
            if (last) tc::mma_commit(tc::smem_u32(&bar_dfull[d]));
          }
          __syncwarp();
          acc = 1u;
          if (++s == (uint32_t)kSS) {
            s = 0;
            s_par ^= 1u;
          }
          if (++sb == (uint32_t)kSBS) sb = 0;
          item_done = cs.advance_ss(b);
        }
        ++ic;
      }
    }
  } else {
    // -------------------------------------------------------- epilogue --
    // A warp may only touch the TMEM lanes of its sub-partition, warp id % 4.
    const int sub = warp & 3;
    const int r = sub * 32 + lane;
    const uint32_t lane_off = (uint32_t)(32 * sub) << 16;
    bool waited_pdl = false;
    int64_t item = blockIdx.x;
    uint32_t ic = 0;
    for (; item < b.total_items; item += gridDim.x, ++ic) {
      const Item it = decode_item(b, item);
      const TqProblem& p = b.p[it.prob];
      const uint32_t d = ic % kDBufs;
      ok = ok && tc::mbar_wait(tc::smem_u32(&bar_dfull[d]), (ic / kDBufs) & 1, b.err, 16);
      ok = __all_sync(0xffffffffu, ok);
      tc::tc_fence_after();
      if (!waited_pdl) {
        tc::pdl_wait();  // outputs / scratch may still be used by the previous launch
        waited_pdl = true;
      }
      const int64_t R = it.tile * kTileRows + r;
      const int ncols = p.tok_per_pass * b.digits;
      const uint32_t dcol = tmem + lane_off + d * kDStride;
      if (p.ksplit == 1) {
#pragma unroll 1
        for (int cg = 0; cg < NPAD / 16; ++cg) {
          uint32_t u[16];
          tc::tmem_ld_x16(dcol + cg * 16, u);
          tc::tmem_wait_ld();
          if (cg == NPAD / 16 - 1) {  // accumulator fully read: hand it back
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(tc::smem_u32(&bar_dfree[d]));
          }
          int32_t v[16];
#pragma unroll
          for (int c = 0; c < 16; ++c) v[c] = (int32_t)u[c];
          if (ok && R < p.rows && cg * 16 < ncols)
            epilogue_group<NPAD, kSparse>(p, b.digits, b.bf16 != 0, it.pass, R, cg * 16, v);
        }
      } else {
        int32_t* accp = p.acc + (((int64_t)it.pass * p.n_tiles + it.tile) * NPAD) * kTileRows;
#pragma unroll 1
        for (int cg = 0; cg < NPAD / 16; ++cg) {
          uint32_t u[16];
          tc::tmem_ld_x16(dcol + cg * 16, u);
          tc::tmem_wait_ld();
          if (cg == NPAD / 16 - 1) {
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(tc::smem_u32(&bar_dfree[d]));
          }
          if (ok)
#pragma unroll
            for (int c = 0; c < 16; ++c)
              if (cg * 16 + c < ncols) atomicAdd(&accp[(cg * 16 + c) * kTileRows + r], (int32_t)u[c]);
        }
        __threadfence();
        named_sync_epilogue();
        if (r == 0) {
          const int prev = atomicAdd(&p.cnt[(int64_t)it.pass * p.n_tiles + it.tile], 1);
          last_flag = (prev == p.ksplit - 1);
        }
        named_sync_epilogue();
        const bool last = last_flag;
        named_sync_epilogue();  // everyone has read last_flag before it is reused
        if (last) {
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
            if (ok && R < p.rows) epilogue_group<NPAD, kSparse>(p, b.digits, b.bf16 != 0, it.pass, R, cg * 16, v);
          }
          if (r == 0) p.cnt[(int64_t)it.pass * p.n_tiles + it.tile] = 0;
        }
      }
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------- B prep -----
// One warp per (source, pass, token slot): writes the token's digit columns
// of the K-major interleaved B operand for every chunk, their column sums,
// the token scale and its non-finite positions.  Slots past `seq` write zero
// columns.
struct PrepSource {
  const void* x;
  int64_t ldx;  // elements per activation row (K, or the gate/up width with act)
  int act;      // x holds interleaved gate/up rows: the operand is act(gate, up)
  const float* kscale;  // column-block scales folded into x, or null
  int64_t kblock;
  int8_t* bmat;
  int32_t* colsum;
  double* tok_scale;
  int32_t* nf;  // [seq][1 + kNfCap]
  int64_t seq, K, n_chunks;
  int passes;
};
constexpr int kMaxSources = 64;
struct PrepBatch {
  int nsrc;
  int xkind;  // 0 f32, 1 bf16, 2 int8 codes
  int D, npad, tok_per_pass;
  int64_t block_begin[kMaxSources + 1];  // first token slot of each source
  PrepSource s[kMaxSources];
};

__device__ __forceinline__ int64_t b_offset(int64_t pass, int64_t chunk, int n, int kin, int npad,
                                            int64_t n_chunks) {
  return ((pass * n_chunks + chunk) * npad) * 128 + ((kin >> 4) * (npad >> 3) + (n >> 3)) * 128 +
         (n & 7) * 16 + (kin & 15);
}

// DT: digits per token (1: int8 codes, 4 or 8), a template parameter so that
// the digit arrays stay in registers.
//
// W warps per (source, pass, token slot), 8 / W slots per block: W = 1 for
// launches of many slots (every reduction is a warp reduction), up to 8 (one
// block per slot) when there are few slots and long rows.  Thread tg of a
// slot's group holds elements S i + 8 tg .. +7 (S = 256 W; one 16-byte load of
// bf16 / int8, two of fp32, when aligned): the first stretches (2 for W = 1,
// one otherwise) stay in registers between the absmax, the non-finite count,
// the digit split and the column sums; the rest are read again (from cache),
// which keeps the warp-per-slot variant at three blocks per SM.  Each thread writes 8 bytes of
// each digit column's 16-byte operand row.
constexpr int kPrepThreads = 256, kPrepWarps = kPrepThreads / 32;

template <int DT, int W>
__global__ void __launch_bounds__(kPrepThreads, W == 1 ? 3 : 1) prep_b_kernel(const __grid_constant__ PrepBatch pb) {
  // Wait for the previous matmul, which may still be reading bmat.  A launch
  // of many slots releases the matmul that consumes it only at the end of
  // each block (that matmul's persistent CTAs, once resident, would leave
  // the remaining blocks a fraction of the SM's registers); a short one
  // releases it at once, so the matmul starts its weight stream meanwhile.
  if (W > 1) tc::pdl_launch_dependents();
  tc::pdl_wait();
  constexpr int kIt = W >= 2 ? 1 : 2, kS = 256 * W;  // register-cached stretches
  __shared__ float red_f[kPrepWarps];
  __shared__ int red_n[kPrepWarps];
  __shared__ int red_i[kPrepWarps][8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gw = warp % W, w0 = warp - gw;  // this warp's index in its slot group, and the first
  const int tg = 32 * gw + lane;
  const int64_t slot = (int64_t)blockIdx.x * (kPrepWarps / W) + warp / W;
  const bool have = slot < pb.block_begin[pb.nsrc];
  // the source holding this slot (binary search over the slot offsets)
  int lo = 0;
  if (have) {
    int hi = pb.nsrc - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (pb.block_begin[mid] <= slot) lo = mid;
      else hi = mid - 1;
    }
  }
  const PrepSource& src = pb.s[lo];
  const int64_t local = have ? slot - pb.block_begin[lo] : 0;
  const int64_t pass = local / pb.tok_per_pass;
  const int lt = (int)(local % pb.tok_per_pass);
  const int64_t t = pass * pb.tok_per_pass + lt;
  const int64_t K = src.K, kpad = src.n_chunks * 128;
  constexpr int D = DT;
  const int npad = pb.npad, xkind = pb.xkind;
  const float* kscale = src.kscale;
  const int64_t kblock = src.kblock;
  const void* xsrc = src.x;
  const bool live = have && t < src.seq;
  const int64_t nst = have ? (kpad + kS - 1) / kS : 0;  // stretches of this slot

  // the 8 elements at k0 .. k0+7 of this token (zero past K), as floats
  // (int8 codes: their integer values)
  auto load8 = [&](int64_t k0, float (&v)[8]) {
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = 0.0f;
    if (!live || k0 >= K) return;
    if (src.act) {
      // k0 .. k0+7 lie in one 16-wide group: gate row 32 (k0/16) + k0%16,
      // its up row 16 further
      const float* gp = static_cast<const float*>(xsrc) + t * src.ldx + 32 * (k0 >> 4) + (k0 & 15);
      if (k0 + 8 <= K && (reinterpret_cast<uintptr_t>(gp) & 15) == 0) {
        const float4 g0 = __ldg(reinterpret_cast<const float4*>(gp));
        const float4 g1 = __ldg(reinterpret_cast<const float4*>(gp) + 1);
        const float4 u0 = __ldg(reinterpret_cast<const float4*>(gp + 16));
        const float4 u1 = __ldg(reinterpret_cast<const float4*>(gp + 16) + 1);
        const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        const float u[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = expert_act(g[e], u[e], src.act);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (k0 + e < K) v[e] = expert_act(__ldg(gp + e), __ldg(gp + 16 + e), src.act);
      }
      return;
    }
    const int64_t i0 = t * src.ldx + k0;
    if (xkind == 2) {
      const int8_t* q = static_cast<const int8_t*>(xsrc) + i0;
      if (k0 + 8 <= K && (reinterpret_cast<uintptr_t>(q) & 7) == 0) {
        const uint2 u = __ldg(reinterpret_cast<const uint2*>(q));
        const uint32_t w2[2] = {u.x, u.y};
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = (float)(int8_t)(w2[e >> 2] >> (8 * (e & 3)));
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (k0 + e < K) v[e] = (float)q[e];
      }
      return;
    }
    if (xkind == 1) {
      const uint16_t* h = static_cast<const uint16_t*>(xsrc) + i0;
      if (k0 + 8 <= K && (reinterpret_cast<uintptr_t>(h) & 15) == 0) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(h));
        const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          v[2 * e] = __uint_as_float(w4[e] << 16);
          v[2 * e + 1] = __uint_as_float(w4[e] & 0xffff0000u);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (k0 + e < K) v[e] = __uint_as_float((uint32_t)h[e] << 16);
      }
    } else {
      const float* f = static_cast<const float*>(xsrc) + i0;
      if (k0 + 8 <= K && (reinterpret_cast<uintptr_t>(f) & 15) == 0) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(f));
        const float4 b = __ldg(reinterpret_cast<const float4*>(f) + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (k0 + e < K) v[e] = f[e];
      }
    }
    if (kscale) {
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (k0 + e < K) v[e] = __fmul_rn(v[e], kscale[(k0 + e) / kblock]);
    }
  };

  float xr[kIt][8];
  float f1 = 1.0f, f2 = 1.0f;
  if (D != 1) {
#pragma unroll
    for (int i = 0; i < kIt; ++i)
      if (i < nst) load8(kS * (int64_t)i + 8 * tg, xr[i]);
    // largest finite |x| and the non-finite count
    float amax = 0.0f;
    int nnf = 0;
    auto scan = [&](const float (&v)[8]) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const bool nf = is_nonfinite(v[e]);
        nnf += nf ? 1 : 0;
        amax = fmaxf(amax, nf ? 0.0f : fabsf(v[e]));
      }
    };
#pragma unroll
    for (int i = 0; i < kIt; ++i)
      if (i < nst) scan(xr[i]);
    for (int64_t i = kIt; i < nst; ++i) {
      float v[8];
      load8(kS * i + 8 * tg, v);
      scan(v);
    }
    int incl = nnf;  // inclusive scan of the non-finite counts over the warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    amax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(amax)));
    int before = incl - nnf, total = __shfl_sync(0xffffffffu, incl, 31);
    if (W > 1) {
      if (lane == 0) {
        red_f[warp] = amax;
        red_n[warp] = total;
      }
      __syncthreads();
      amax = 0.0f;
      total = 0;
#pragma unroll
      for (int w = 0; w < W; ++w) {
        amax = fmaxf(amax, red_f[w0 + w]);
        if (w < gw) before += red_n[w0 + w];
        total += red_n[w0 + w];
      }
    }
    const int sh = amax > 0.0f ? digit_shift(amax, D) : 0;
    const int s1 = sh > 127 ? 127 : (sh < -126 ? -126 : sh);
    f1 = __int_as_float((s1 + 127) << 23);
    f2 = __int_as_float((sh - s1 + 127) << 23);
    if (live) {
      int32_t* nf = src.nf + t * (kNfCap + 1);
      if (tg == 0) {
        // 2^-sh (1 for an all-zero token), negative when non-finite elements exist
        const double sc = amax > 0.0f ? __longlong_as_double((long long)(1023 - sh) << 52) : 1.0;
        src.tok_scale[t] = total ? -sc : sc;
        nf[0] = total;
      }
      if (nnf != 0 && total <= kNfCap) {
        // this thread's positions after those of the threads below it
        int slot_nf = before;
        for (int64_t i = 0; i < nst; ++i) {
          float v[8];
          load8(kS * i + 8 * tg, v);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (is_nonfinite(v[e])) nf[1 + slot_nf++] = (int32_t)(kS * i + 8 * tg + e);
        }
      }
    }
  }
  // digits of each element; one 8-byte word pair per digit column
  int csum[D];
#pragma unroll
  for (int d = 0; d < D; ++d) csum[d] = 0;
  // Byte permutes gather digit d of four elements (bytes of U0..U3) into one
  // word: [byte d of U0, U1, U2, U3].
  auto gather = [](uint32_t u0, uint32_t u1, uint32_t u2, uint32_t u3, uint32_t (&wd)[4]) {
    const uint32_t lo01 = __byte_perm(u0, u1, 0x5140), lo23 = __byte_perm(u2, u3, 0x5140);
    const uint32_t hi01 = __byte_perm(u0, u1, 0x7362), hi23 = __byte_perm(u2, u3, 0x7362);
    wd[0] = __byte_perm(lo01, lo23, 0x5410);
    wd[1] = __byte_perm(lo01, lo23, 0x7632);
    wd[2] = __byte_perm(hi01, hi23, 0x5410);
    wd[3] = __byte_perm(hi01, hi23, 0x7632);
  };
  auto emit = [&](int64_t k0, const float (&v)[8]) {
    if (k0 >= kpad) return;
    uint32_t w[D][2];
#pragma unroll
    for (int hq = 0; hq < 2; ++hq) {  // elements 4 hq .. 4 hq + 3
      if (D == 1) {
        uint32_t q = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) q |= (uint32_t)((int)v[4 * hq + e] & 0xFF) << (8 * e);
        w[0][hq] = q;
      } else {
        float xs[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float x = v[4 * hq + e];
          xs[e] = is_nonfinite(x) ? 0.0f : __fmul_rn(__fmul_rn(x, f1), f2);
        }
        if (D == 4) {
          // X = round(x * 2^sh), |X| < 2^30; U = X + 0x808080: its low three
          // bytes are the balanced low digits + 128, its top byte the top digit
          uint32_t wd[4];
          gather((uint32_t)__float2int_rn(xs[0]) + 0x808080u, (uint32_t)__float2int_rn(xs[1]) + 0x808080u,
                 (uint32_t)__float2int_rn(xs[2]) + 0x808080u, (uint32_t)__float2int_rn(xs[3]) + 0x808080u,
                 wd);
#pragma unroll
          for (int d = 0; d < 4; ++d) w[d < D ? d : 0][hq] = d < 3 ? wd[d] ^ 0x80808080u : wd[d];
        } else {
          // X = round(x * 2^sh), |X| < 2^62; U = X + 0x0080808080808080: bytes 0..6
          // are the balanced low digits + 128, byte 7 the top digit
          const unsigned long long b7 = 0x0080808080808080ull;
          unsigned long long U[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) U[e] = (unsigned long long)__float2ll_rn(xs[e]) + b7;
          uint32_t lo[4], hi[4];
          gather((uint32_t)U[0], (uint32_t)U[1], (uint32_t)U[2], (uint32_t)U[3], lo);
          gather((uint32_t)(U[0] >> 32), (uint32_t)(U[1] >> 32), (uint32_t)(U[2] >> 32),
                 (uint32_t)(U[3] >> 32), hi);
#pragma unroll
          for (int d = 0; d < 4; ++d) {
            w[d][hq] = lo[d] ^ 0x80808080u;
            w[(d + 4) < D ? d + 4 : 0][hq] = d < 3 ? hi[d] ^ 0x80808080u : hi[d];
          }
        }
      }
    }
    // column sums: signed bytes of each digit word
#pragma unroll
    for (int d = 0; d < D; ++d)
      csum[d] = __dp4a((int)w[d][1], 0x01010101, __dp4a((int)w[d][0], 0x01010101, csum[d]));
    const int64_t chunk = k0 >> 7;
    const int kin = (int)(k0 & 127);
#pragma unroll
    for (int d = 0; d < D; ++d)
      *reinterpret_cast<uint2*>(src.bmat + b_offset(pass, chunk, lt * D + d, kin & ~15, npad,
                                                    src.n_chunks) +
                                (kin & 8)) = make_uint2(w[d][0], w[d][1]);
  };
  if (D != 1) {
#pragma unroll
    for (int i = 0; i < kIt; ++i)
      if (i < nst) emit(kS * (int64_t)i + 8 * tg, xr[i]);
  }
  for (int64_t i = D != 1 ? kIt : 0; i < nst; ++i) {
    float v[8];
    load8(kS * i + 8 * tg, v);
    emit(kS * i + 8 * tg, v);
  }
#pragma unroll
  for (int d = 0; d < D; ++d) {
    const int v = __reduce_add_sync(0xffffffffu, (unsigned)csum[d]);
    if (W > 1) {
      if (lane == 0) red_i[warp][d] = v;
    } else if (have && lane == 0) {
      src.colsum[pass * npad + lt * D + d] = v;
    }
  }
  if (W > 1) {
    __syncthreads();
    if (have && gw == 0 && lane < D) {
      int v = 0;
#pragma unroll
      for (int w = 0; w < W; ++w) v += red_i[w0 + w][lane];
      src.colsum[pass * npad + lt * D + lane] = v;
    }
  }
  if (W == 1) tc::pdl_launch_dependents();
}

// int8 activations (D = 1): the operand is a re-layout of the codes.  A block
// takes 8 consecutive token slots of one (source, pass); lane (r, q) of warp w
// moves the 16 bytes of token r at K groups 4 (w + 8 i) + q, so every warp
// store writes four whole 128-byte core-matrix row groups (8 tokens x 16 bytes)
// and every load reads 64 contiguous bytes of a token row.  (The general
// kernel's 8-byte stores at the K-group stride took 6.9 us for cfg2's 2 MB.)
__global__ void __launch_bounds__(kPrepThreads) prep_i8_kernel(const __grid_constant__ PrepBatch pb) {
  tc::pdl_launch_dependents();
  tc::pdl_wait();  // the previous matmul may still be reading bmat
  __shared__ int red[kPrepWarps][8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane & 7, q = lane >> 3;
  const int64_t slot0 = (int64_t)blockIdx.x * 8;
  if (slot0 >= pb.block_begin[pb.nsrc]) return;  // uniform over the block
  int lo = 0, hi = pb.nsrc - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (pb.block_begin[mid] <= slot0) lo = mid;
    else hi = mid - 1;
  }
  const PrepSource& src = pb.s[lo];
  const int64_t local = slot0 - pb.block_begin[lo];
  const int64_t pass = local / pb.tok_per_pass;
  const int lt = (int)(local % pb.tok_per_pass) + r;
  const int64_t t = pass * pb.tok_per_pass + lt;
  const bool live = t < src.seq;
  const int64_t K = src.K, groups = src.n_chunks * 8;  // 16-byte K groups
  const int8_t* row = static_cast<const int8_t*>(src.x) + (live ? t : 0) * src.ldx;
  const bool fast = (K & 15) == 0 && (src.ldx & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(src.x) & 15) == 0;
  int cs = 0;
  // eight K groups per thread at a time, every load issued before any store
  constexpr int kStep = 4 * kPrepWarps, kU = 8;
  for (int64_t kb = 4 * warp + q; kb < groups; kb += kU * kStep) {
    uint4 v[kU];
#pragma unroll
    for (int i = 0; i < kU; ++i) {
      const int64_t k0 = 16 * (kb + i * kStep);
      v[i] = make_uint4(0u, 0u, 0u, 0u);
      if (live && k0 < K) {
        if (fast) {
          v[i] = __ldg(reinterpret_cast<const uint4*>(row + k0));
        } else {
          uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (k0 + e < K) w[e >> 2] |= (uint32_t)(row[k0 + e] & 0xFF) << (8 * (e & 3));
          v[i] = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < kU; ++i) {
      const int64_t kg = kb + i * kStep, k0 = 16 * kg;
      if (kg < groups) {
        cs = __dp4a((int)v[i].x, 0x01010101, cs);
        cs = __dp4a((int)v[i].y, 0x01010101, cs);
        cs = __dp4a((int)v[i].z, 0x01010101, cs);
        cs = __dp4a((int)v[i].w, 0x01010101, cs);
        *reinterpret_cast<uint4*>(src.bmat + b_offset(pass, k0 >> 7, lt, (int)(k0 & 127),
                                                      pb.npad, src.n_chunks)) = v[i];
      }
    }
  }
  // column sums of the 8 tokens: lanes r, r + 8, r + 16, r + 24 of every warp
  cs += __shfl_xor_sync(0xffffffffu, cs, 8);
  cs += __shfl_xor_sync(0xffffffffu, cs, 16);
  if (q == 0) red[warp][r] = cs;
  __syncthreads();
  if (threadIdx.x < 8) {  // lane r = threadIdx.x: lt is token r's slot
    int v = 0;
#pragma unroll
    for (int w = 0; w < kPrepWarps; ++w) v += red[w][threadIdx.x];
    src.colsum[pass * pb.npad + lt] = v;
  }
}

// slots -> warps per slot: many slots use one warp each, few slots (long
// rows, little parallelism) up to a block each
int prep_warps(int64_t slots) {
  return slots >= 4096 ? 1 : slots >= 2048 ? 2 : slots >= 1024 ? 4 : 8;
}

template <int DT>
cudaError_t launch_prep(const PrepBatch& pb, int64_t slots, cudaLaunchConfig_t cfg) {
  const int W = prep_warps(slots);
  cfg.gridDim = dim3((unsigned)ceil_div(slots * W, kPrepWarps));
  if (W == 1) return cudaLaunchKernelEx(&cfg, prep_b_kernel<DT, 1>, pb);
  if (W == 2) return cudaLaunchKernelEx(&cfg, prep_b_kernel<DT, 2>, pb);
  if (W == 4) return cudaLaunchKernelEx(&cfg, prep_b_kernel<DT, 4>, pb);
  return cudaLaunchKernelEx(&cfg, prep_b_kernel<DT, 8>, pb);
}

#ifndef FT_MAX_NPAD
#define FT_MAX_NPAD 128
#endif

// K splits of a launch of `tiles` (pass, tile) pairs whose longest weight has
// `chunks` K chunks.  Split-K partials are combined with int32 atomics, so a
// split pays 128 x npad atomics per item against the shorter per-CTA chunk
// chain it buys; the split with the least modelled time wins (fewer splits on
// near-ties).  The constants are measured on B200 with W[11008, 4096]: a CTA
// takes ~400 cycles per chunk at npad <= 64 and ~640 at npad 128 (MMA-bound),
// and the GPU completes ~100 int32 atomics per cycle.  With 86 tiles this
// picks no split: split 4-14 ways the same launch ran 1.6-2.5x slower.  A
// split must also beat the unsplit model by FT_TC_SPLIT_GAIN: the 2-way split
// the model chose at 16 columns (86 or 44 tiles) measured slower than none.
#ifndef FT_TC_SPLIT_GAIN
#define FT_TC_SPLIT_GAIN 0.7
#endif
int pick_ksplit(int64_t tiles, int64_t grid_target, int64_t chunks, int npad) {
  const double chunk_cycles = npad >= 128 ? 640.0 : 400.0, atomics_per_cycle = 100.0;
  double best = 0.0, unsplit = 0.0;
  int best_ks = 1;
  for (int ks = 1; ks <= 64 && ks <= chunks; ++ks) {
    const double t = (double)ceil_div(tiles * ks, grid_target) *
                         (double)ceil_div(chunks, (int64_t)ks) * chunk_cycles +
                     (ks > 1 ? (double)(tiles * ks) * 128.0 * npad / atomics_per_cycle : 0.0);
    if (ks == 1) unsplit = t;
    if (ks == 1 || (t < 0.97 * best && t < FT_TC_SPLIT_GAIN * unsplit)) {
      best = t;
      best_ks = ks;
    }
  }
  return best_ks;
}
// Column-pass width.  Wide problems use 128-column passes: two TMEM
// accumulators then fit, so a tile's epilogue overlaps the next tile's MMAs.
int pick_npad(int64_t ncols) {
  if (ncols <= 16) return 16;
  if (ncols <= 32) return 32;
  if (ncols <= 64) return 64;
  if (ncols <= 128 || FT_MAX_NPAD <= 128) return 128;
  return 256;
}

template <int NPAD, bool kSparse = false>
int launch_grouped_t(const TqBatch& batch, int64_t grid, cudaStream_t s) {
  const size_t smem = TqCfg<NPAD, kSparse>::SMEM;
  static bool attr_set = false;  // per template instance
  if (!attr_set) {
    FT_CUDA(cudaFuncSetAttribute(tq_grouped_kernel<NPAD, kSparse>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(TqCfg<NPAD, kSparse>::THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FT_CUDA(cudaLaunchKernelEx(&cfg, tq_grouped_kernel<NPAD, kSparse>, batch));
  FT_LAUNCH_CHECK();
  return FT_OK;
}

}  // namespace

// Grouped tensor-core matmul over up to 64 independent problems sharing the
// activation kind.  Problem i has seqs[i] tokens (or `seq` when seqs is null;
// problems with 0 tokens are skipped); activations xs[i] [seq_i, cols_i],
// output ys[i] rows of length ldys[i] (default rows_i).  Entries with the same
// activation pointer, K and seq share one prepared B operand.
int launch_tc_grouped(ft_ctx* ctx, int n, const ft_weight* const* ws, int64_t seq,
                      const void* const* xs, int xkind, const float* const* sxs, float* const* ys,
                      const int64_t* ldys, cudaStream_t s, const int64_t* seqs, int digits,
                      const float* kscale, int64_t kblock, int act, int64_t ldx) {
  FT_CHECK(n >= 1 && n <= kMaxProblems, FT_ERR_UNSUPPORTED, "group size %d not in [1, %d]", n,
           kMaxProblems);
  if (digits <= 0) digits = kDigitsExact;
  FT_CHECK(xkind == 2 || digits == kDigitsExact || digits == kDigitsMoE, FT_ERR_UNSUPPORTED,
           "unsupported digit count %d", digits);
  const int D = xkind == 2 ? 1 : digits;
  FT_CHECK(!act || (xkind == 0 && !kscale), FT_ERR_UNSUPPORTED,
           "the fused activation needs fp32 gate/up activations");
  FT_CHECK(!kscale || (xkind != 2 && kblock >= 1), FT_ERR_UNSUPPORTED,
           "column-block scales need fp32/bf16 activations and a block size >= 1");
  int64_t max_seq = 0;
  for (int i = 0; i < n; ++i) {
    const int64_t si = seqs ? seqs[i] : seq;
    FT_CHECK(si >= 0, FT_ERR_SHAPE, "negative seq in group entry %d", i);
    max_seq = si > max_seq ? si : max_seq;
  }
  if (max_seq == 0) return FT_OK;
  const int npad = pick_npad(max_seq * D);
  const int tok_per_pass = npad / D;
  FT_CHECK(ceil_div(max_seq, tok_per_pass) <= (1 << 20), FT_ERR_UNSUPPORTED, "seq %lld too large",
           (long long)max_seq);

  // live problems and their distinct activation sources (pointer, K, seq)
  int live[kMaxProblems];
  int nlive = 0;
  int src_of[kMaxProblems];
  int nsrc = 0;
  const void* src_x[kMaxSources];
  int64_t src_k[kMaxSources], src_seq[kMaxSources];
  for (int i = 0; i < n; ++i) {
    const int64_t si = seqs ? seqs[i] : seq;
    if (si == 0) continue;
    FT_CHECK(ws[i] && xs[i] && ys[i], FT_ERR_SHAPE, "null pointer in group entry %d", i);
    FT_CHECK(ws[i]->device == ctx->device, FT_ERR_DEVICE, "weight %d on another device", i);
    FT_CHECK(ws[i]->format == ws[0]->format, FT_ERR_UNSUPPORTED,
             "group mixes dense and 2:4 sparse weights (entry %d)", i);
    FT_CHECK(xkind != 2 || (sxs && sxs[i]), FT_ERR_SHAPE, "null sx in group entry %d", i);
    int j = 0;
    while (j < nsrc && !(src_x[j] == xs[i] && src_k[j] == ws[i]->cols && src_seq[j] == si)) ++j;
    if (j == nsrc) {
      FT_CHECK(nsrc < kMaxSources, FT_ERR_UNSUPPORTED, "more than %d distinct activations",
               kMaxSources);
      src_x[nsrc] = xs[i];
      src_k[nsrc] = ws[i]->cols;
      src_seq[nsrc] = si;
      ++nsrc;
    }
    src_of[nlive] = j;
    live[nlive++] = i;
  }

  // decode shapes run on the warp-level kernel (ft_gemv.cu), which builds its
  // activation operand itself
  bool gemv = true;
  for (int q = 0; q < nlive && gemv; ++q)
    gemv = gemv_fits(ws[live[q]], src_seq[src_of[q]], xkind, D);
  if (gemv) {
    GvLaunchProblem gp[kMaxProblems];
    for (int q = 0; q < nlive; ++q) {
      const int i = live[q];
      const ft_weight* w = ws[i];
      const int j = src_of[q];
      gp[q] = GvLaunchProblem{w->codes, w->row_scales, w->rows, w->n_chunks, src_x[j],
                              src_k[j], src_seq[j], sxs ? sxs[i] : nullptr, ys[i],
                              ldys ? ldys[i] : w->rows, kscale, kblock, act,
                              act ? ldx : src_k[j]};
    }
    return launch_gemv(ctx, nlive, gp, xkind, ws[live[0]]->format == 1, D, s);
  }

  // workspace: per source B operand, column sums, token scales, non-finite lists
  size_t off = 0;
  size_t b_off[kMaxSources], cs_off[kMaxSources], ts_off[kMaxSources], nf_off[kMaxSources];
  for (int j = 0; j < nsrc; ++j) {
    const int64_t nch = ceil_div(src_k[j], kChunkK);
    const int64_t passes = ceil_div(src_seq[j], tok_per_pass);
    b_off[j] = off;
    off = round_up((int64_t)(off + (size_t)(passes * nch) * npad * 128), 256);
    cs_off[j] = off;
    off = round_up((int64_t)(off + passes * npad * 4), 256);
    ts_off[j] = off;
    off = round_up((int64_t)(off + src_seq[j] * 8), 256);
    nf_off[j] = off;
    off = round_up((int64_t)(off + src_seq[j] * (kNfCap + 1) * 4), 256);
  }
  int st = workspace_reserve(ctx, off, s);
  if (st != FT_OK) return st;
  char* wsb = static_cast<char*>(ctx->ws.ptr);

  // work decomposition and zero-initialised split-K scratch
  // Two CTAs per SM when both fit in TMEM (each has its own MMA-issuing
  // thread, which is what limits a small-N launch); one otherwise.
  const int64_t grid_target = (int64_t)ctx->num_sms * (tmem_cols_for(npad) <= 256 ? 2 : 1);
  int64_t tiles_total = 0, max_chunks = 1;
  for (int q = 0; q < nlive; ++q) {
    tiles_total += ws[live[q]]->n_tiles * ceil_div(src_seq[src_of[q]], tok_per_pass);
    max_chunks = ws[live[q]]->n_chunks > max_chunks ? ws[live[q]]->n_chunks : max_chunks;
  }
  const int64_t ks_group = pick_ksplit(tiles_total, grid_target, max_chunks, npad);
  size_t zoff = 0;
  size_t acc_off[kMaxProblems], cnt_off[kMaxProblems];
  static thread_local TqBatch batch;  // host staging; the launch copies it as the parameter
  memset(&batch, 0, sizeof(batch));
  batch.nprob = nlive;
  batch.digits = D;
  batch.bf16 = xkind == 1;
  int64_t items = 0;
  for (int q = 0; q < nlive; ++q) {
    const int i = live[q];
    const ft_weight* w = ws[i];
    const int j = src_of[q];
    const int64_t passes = ceil_div(src_seq[j], tok_per_pass);
    TqProblem& p = batch.p[q];
    const int64_t want = ks_group < w->n_chunks ? ks_group : w->n_chunks;
    p.cps = (int)ceil_div(w->n_chunks, want);
    p.ksplit = (int)ceil_div(w->n_chunks, p.cps);
    p.codes = w->codes;
    p.row_scales = w->row_scales;
    p.rows = w->rows;
    p.n_tiles = w->n_tiles;
    p.n_chunks = w->n_chunks;
    p.bmat = reinterpret_cast<const int8_t*>(wsb + b_off[j]);
    p.colsum = reinterpret_cast<const int32_t*>(wsb + cs_off[j]);
    p.tok_scale = reinterpret_cast<const double*>(wsb + ts_off[j]);
    p.nf = reinterpret_cast<const int32_t*>(wsb + nf_off[j]);
    p.x = src_x[j];
    p.K = src_k[j];
    p.kscale = kscale;
    p.kblock = kblock;
    p.sx = sxs ? sxs[i] : nullptr;
    p.y = ys[i];
    p.ldy = ldys ? ldys[i] : w->rows;
    p.act = act;
    p.ldx = act ? ldx : src_k[j];
    p.seq = src_seq[j];
    p.tok_per_pass = tok_per_pass;
    p.passes = (int)passes;
    p.item_begin = items;
    batch.item_begin[q] = items;
    items += passes * w->n_tiles * p.ksplit;
    acc_off[q] = cnt_off[q] = 0;
    if (p.ksplit > 1) {
      acc_off[q] = zoff;
      zoff = round_up((int64_t)(zoff + (size_t)(passes * w->n_tiles) * npad * kTileRows * 4), 256);
      cnt_off[q] = zoff;
      zoff = round_up((int64_t)(zoff + passes * w->n_tiles * 4), 256);
    }
  }
  batch.total_items = items;
  batch.item_begin[nlive] = items;
  const size_t err_off = zoff;
  st = zero_scratch_reserve(ctx, err_off + 256, s);
  if (st != FT_OK) return st;
  char* zs = static_cast<char*>(ctx->zs.ptr);
  for (int q = 0; q < nlive; ++q)
    if (batch.p[q].ksplit > 1) {
      batch.p[q].acc = reinterpret_cast<int32_t*>(zs + acc_off[q]);
      batch.p[q].cnt = reinterpret_cast<int32_t*>(zs + cnt_off[q]);
    }
  batch.err = ctx->err_word;

  // prep launch: one block per source x pass x token slot of the operand
  {
    static thread_local PrepBatch pb;
    memset(&pb, 0, sizeof(pb));
    pb.nsrc = nsrc;
    pb.xkind = xkind;
    pb.D = D;
    pb.npad = npad;
    pb.tok_per_pass = tok_per_pass;
    int64_t blocks = 0;
    for (int j = 0; j < nsrc; ++j) {
      const int64_t passes = ceil_div(src_seq[j], tok_per_pass);
      pb.block_begin[j] = blocks;
      PrepSource& ps = pb.s[j];
      ps.x = src_x[j];
      ps.act = act;
      ps.ldx = act ? ldx : src_k[j];
      ps.kscale = kscale;
      ps.kblock = kblock;
      ps.bmat = reinterpret_cast<int8_t*>(wsb + b_off[j]);
      ps.colsum = reinterpret_cast<int32_t*>(wsb + cs_off[j]);
      ps.tok_scale = reinterpret_cast<double*>(wsb + ts_off[j]);
      ps.nf = reinterpret_cast<int32_t*>(wsb + nf_off[j]);
      ps.seq = src_seq[j];
      ps.K = src_k[j];
      ps.n_chunks = ceil_div(src_k[j], kChunkK);
      ps.passes = (int)passes;
      blocks += passes * tok_per_pass;
    }
    pb.block_begin[nsrc] = blocks;
    FT_CHECK(blocks <= 0x7FFFFFFF, FT_ERR_UNSUPPORTED, "too many prep blocks");
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(kPrepThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (D == 1) {  // int8 codes: tok_per_pass = npad, a multiple of 8 slots per (source, pass)
      cfg.gridDim = dim3((unsigned)(blocks / 8));
      FT_CUDA(cudaLaunchKernelEx(&cfg, prep_i8_kernel, pb));
    }
    else if (D == 4) FT_CUDA(launch_prep<4>(pb, blocks, cfg));
    else FT_CUDA(launch_prep<8>(pb, blocks, cfg));
    FT_LAUNCH_CHECK();
  }

  const int64_t grid = items < grid_target ? items : grid_target;
  if (ws[live[0]]->format == 1) {
    switch (npad) {
      case 16: return launch_grouped_t<16, true>(batch, grid, s);
      case 32: return launch_grouped_t<32, true>(batch, grid, s);
      case 64: return launch_grouped_t<64, true>(batch, grid, s);
      case 128: return launch_grouped_t<128, true>(batch, grid, s);
      default: return launch_grouped_t<256, true>(batch, grid, s);
    }
  }
  switch (npad) {
    case 16: return launch_grouped_t<16>(batch, grid, s);
    case 32: return launch_grouped_t<32>(batch, grid, s);
    case 64: return launch_grouped_t<64>(batch, grid, s);
    case 128: return launch_grouped_t<128>(batch, grid, s);
    default: return launch_grouped_t<256>(batch, grid, s);
  }
}

int launch_tc_matmul(ft_ctx* ctx, const ft_weight* w, int64_t seq, const void* x, int xkind,
                     const float* sx, float* y, cudaStream_t s) {
  const ft_weight* ws[1] = {w};
  const void* xs[1] = {x};
  const float* sxs[1] = {sx};
  float* ys[1] = {y};
  return launch_tc_grouped(ctx, 1, ws, seq, xs, xkind, xkind == 2 ? sxs : nullptr, ys, nullptr, s,
                           nullptr);
}

}  // namespace ft

// ---------------------------------------------------------------------------
// Allocation-free variant of the fp32 matmul, for decode-sized calls.
//
// Some callers cannot let a library allocate device memory during a call: a
// host that hands out all device memory itself (a serving engine with a fixed
// arena, or an FFI contract that forbids hidden allocations on the hot path),
// or a real-time loop that cannot take cudaMalloc's implicit device-wide
// synchronisation.  This entry point runs the same two kernels as
// ft_ternary_matmul_f32, but its scratch (activation operand, column sums,
// token scales, split-K sums and tickets, error word) lives in the
// file-scope array below, reserved in the library image on every GPU that
// loads the library and held until the process exits.
// ---------------------------------------------------------------------------
namespace ft {
namespace {
constexpr int64_t kNaMaxSeq = 4;  // tokens per call (8 digit columns each -> NPAD 32)
constexpr int64_t kNaMaxCols = 16384;
constexpr int64_t kNaMaxRows = 16384;
constexpr int kNaNpad = 32;
constexpr size_t kNaBOff = 0;
constexpr size_t kNaBBytes = (size_t)(kNaMaxCols / kChunkK) * kNaNpad * 128;        // 512 KiB
constexpr size_t kNaColsumOff = kNaBOff + kNaBBytes;                                  // 32 x int32
constexpr size_t kNaTokOff = kNaColsumOff + 256;                                      // 4 x double
constexpr size_t kNaNfOff = kNaTokOff + 256;                      // 4 x (1 + kNfCap) int32
constexpr size_t kNaAccOff = kNaNfOff + 512;
constexpr size_t kNaAccBytes = (size_t)(kNaMaxRows / kTileRows) * kNaNpad * kTileRows * 4;  // 2 MiB
constexpr size_t kNaCntOff = kNaAccOff + kNaAccBytes;
constexpr size_t kNaCntBytes = (size_t)(kNaMaxRows / kTileRows) * 4;
constexpr size_t kNaErrOff = kNaCntOff + (kNaCntBytes + 255) / 256 * 256;
constexpr size_t kNaBytes = kNaErrOff + 256;  // about 2.6 MB
static_assert(kNaMaxSeq * (1 + kNfCap) * 4 <= 512, "non-finite lists must fit their slot");
constexpr int kNaMaxDevices = 64;

static void* g_na_ptr[kNaMaxDevices];  // device address of g_noalloc_scratch, per device
}  // namespace

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNaBytes];

namespace {
// Looks up (once per device, with that device current) the device address of
// the scratch array; host code must never pass the symbol itself to a kernel.
int noalloc_scratch(int device, char** out) {
  FT_CHECK(device >= 0 && device < kNaMaxDevices, FT_ERR_DEVICE, "device %d not supported", device);
  if (g_na_ptr[device] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    FT_CHECK(e == cudaSuccess && p != nullptr, FT_ERR_GPU,
             "cudaGetSymbolAddress of the no-alloc scratch failed: %s", cudaGetErrorString(e));
    g_na_ptr[device] = p;
  }
  *out = static_cast<char*>(g_na_ptr[device]);
  return FT_OK;
}

int launch_tc_noalloc(ft_ctx* ctx, const ft_weight* w, int64_t seq, const float* x, float* y,
                      cudaStream_t s) {
  char* zs = nullptr;
  int st = noalloc_scratch(ctx->device, &zs);
  if (st != FT_OK) return st;

  const int D = kDigitsExact, npad = kNaNpad, tok_per_pass = npad / D;
  static thread_local TqBatch batch;
  memset(&batch, 0, sizeof(batch));
  batch.nprob = 1;
  batch.digits = D;
  batch.bf16 = 0;
  const int64_t grid_target = (int64_t)ctx->num_sms * (tmem_cols_for(npad) <= 256 ? 2 : 1);
  TqProblem& p = batch.p[0];
  const int64_t want = pick_ksplit(w->n_tiles, grid_target, w->n_chunks, npad);
  p.cps = (int)ceil_div(w->n_chunks, want);
  p.ksplit = (int)ceil_div(w->n_chunks, p.cps);
  p.codes = w->codes;
  p.row_scales = w->row_scales;
  p.rows = w->rows;
  p.n_tiles = w->n_tiles;
  p.n_chunks = w->n_chunks;
  p.bmat = reinterpret_cast<const int8_t*>(zs + kNaBOff);
  p.colsum = reinterpret_cast<const int32_t*>(zs + kNaColsumOff);
  p.tok_scale = reinterpret_cast<const double*>(zs + kNaTokOff);
  p.nf = reinterpret_cast<const int32_t*>(zs + kNaNfOff);
  p.x = x;
  p.ldx = w->cols;
  p.K = w->cols;
  p.kscale = nullptr;
  p.kblock = 1;
  p.sx = nullptr;
  p.y = y;
  p.ldy = w->rows;
  p.seq = seq;
  p.tok_per_pass = tok_per_pass;
  p.passes = 1;
  p.item_begin = 0;
  batch.item_begin[0] = 0;
  p.acc = reinterpret_cast<int32_t*>(zs + kNaAccOff);
  p.cnt = reinterpret_cast<int32_t*>(zs + kNaCntOff);
  batch.total_items = w->n_tiles * p.ksplit;
  batch.item_begin[1] = batch.total_items;
  // The split-K sums and tickets this call uses must start at zero (the kernel
  // leaves them zeroed, but a launch whose wait gave up may not have).  The
  // error word is not cleared here: it keeps a report until ft_ctx_check of a
  // context that used this entry point reads and clears it.
  if (p.ksplit > 1) {
    FT_CUDA(cudaMemsetAsync(zs + kNaAccOff, 0, (size_t)w->n_tiles * kNaNpad * kTileRows * 4, s));
    FT_CUDA(cudaMemsetAsync(zs + kNaCntOff, 0, (size_t)w->n_tiles * 4, s));
  }
  batch.err = reinterpret_cast<int*>(zs + kNaErrOff);
  ctx->na_err = batch.err;

  static thread_local PrepBatch pb;
  memset(&pb, 0, sizeof(pb));
  pb.nsrc = 1;
  pb.xkind = 0;
  pb.D = D;
  pb.npad = npad;
  pb.tok_per_pass = tok_per_pass;
  pb.block_begin[0] = 0;
  pb.block_begin[1] = tok_per_pass;
  PrepSource& ps = pb.s[0];
  ps.x = x;
  ps.ldx = w->cols;
  ps.kscale = nullptr;
  ps.kblock = 1;
  ps.bmat = reinterpret_cast<int8_t*>(zs + kNaBOff);
  ps.colsum = reinterpret_cast<int32_t*>(zs + kNaColsumOff);
  ps.tok_scale = reinterpret_cast<double*>(zs + kNaTokOff);
  ps.nf = reinterpret_cast<int32_t*>(zs + kNaNfOff);
  ps.seq = seq;
  ps.K = w->cols;
  ps.n_chunks = w->n_chunks;
  ps.passes = 1;
  prep_b_kernel<kDigitsExact, 8><<<tok_per_pass, kPrepThreads, 0, s>>>(pb);
  FT_LAUNCH_CHECK();
  const int64_t grid = batch.total_items < grid_target ? batch.total_items : grid_target;
  return launch_grouped_t<kNaNpad>(batch, grid, s);
}
}  // namespace
}  // namespace ft

extern "C" int ft_ternary_matmul_f32_noalloc(ft_ctx* ctx, const ft_weight* w, int64_t seq,
                                             const float* x_dev, float* y_dev, void* stream) {
  using namespace ft;
  FT_CHECK(ctx && w, FT_ERR_SHAPE, "null context or weight");
  FT_CHECK(seq >= 0, FT_ERR_SHAPE, "seq must be >= 0");
  FT_CHECK(seq == 0 || (x_dev && y_dev), FT_ERR_SHAPE, "null activation/output pointer");
  FT_CHECK(w->device == ctx->device, FT_ERR_DEVICE, "weight lives on device %d, context on %d",
           w->device, ctx->device);
  FT_CHECK(w->format == 0, FT_ERR_UNSUPPORTED, "the no-alloc matmul takes dense weights only");
  FT_CHECK(seq <= kNaMaxSeq && w->rows <= kNaMaxRows && w->cols <= kNaMaxCols,
           FT_ERR_UNSUPPORTED,
           "no-alloc matmul limits are seq <= %lld, rows <= %lld, cols <= %lld (got seq %lld, "
           "weight [%lld, %lld]); use ft_ternary_matmul_f32 for larger shapes",
           (long long)kNaMaxSeq, (long long)kNaMaxRows, (long long)kNaMaxCols, (long long)seq,
           (long long)w->rows, (long long)w->cols);
  if (seq == 0) return FT_OK;
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
  if (prev != ctx->device) FT_CUDA(cudaSetDevice(ctx->device));
  const int st = launch_tc_noalloc(ctx, w, seq, x_dev, y_dev, static_cast<cudaStream_t>(stream));
  if (prev >= 0 && prev != ctx->device) cudaSetDevice(prev);
  return st;
}
