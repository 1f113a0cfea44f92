// Decode-shape ternary matmul (GEMV and small M): y = scale * (W . x) for a
// group of independent problems whose activations fit 16 operand columns
// (fp32/bf16: <= 2 tokens as 8 base-256 digits each, or <= 4 tokens as 4
// digits; int8: <= 16 tokens).
//
// Same exact formulation as the tensor-core engine (ft_tc.cu): the A operand
// is the unsigned codes u = w + 1, the B operand the int8 activation columns
// (fp32/bf16: the signed base-256 digits of X = round(x * 2^s), 2^s the power
// of two that puts the token's largest finite |x| in [2^(8D-3), 2^(8D-2));
// int8: the caller's codes), int32 sums are exact, the epilogue subtracts the
// column sums and scales.  With D = 8 every element within 2^38 of the token's
// absmax is represented exactly, so the result is the correctly rounded dot
// product.  The MMAs are warp-level (mma.sync m16n8k32, u8 x s8).  Non-finite
// activations enter the digits as 0; their positions are kept per token and
// the rows that meet them are finished by the reference's rule (nonfinite_row).
//
// Weight stream: the lane-major block layout (ft_internal.cuh) gives every
// lane 16 contiguous bytes of an m-block per 128-K chunk, and code slot j of
// each byte belongs to k-step j, so the A fragment of k-step j is the loaded
// word AND (3 << 2j): one logic op per fragment register, no shifts.  The
// factor 4^j this leaves in the operand is divided out exactly at the end:
// each k-step has its own accumulator.  A unit is MB m-blocks (16 * MB
// rows) of one chunk, MB * 512 contiguous bytes, fetched by one bulk copy
// into the warp's ring (one mbarrier per slot, bounded waits); one read of
// the activation fragments feeds 4 * MB MMAs per operand block.
//
// Activation fragments are built by every CTA in its own shared memory (no
// separate prep launch): the token's x is loaded once, its absmax reduced
// over the CTA, then split into digits.
//
// Work split: a unit is (row-block of 16 * MB rows, chunk of 128 K).  Problems
// sharing an activation form a segment; a segment's units are split into
// row-block-aligned ranges, one per CTA, and a CTA's range is split evenly
// across its warps at unit granularity.  A row-block cut by a warp boundary
// is finished by the warp that holds its first chunk, which adds the other
// warps' partial sums from shared memory after the stream.
//
// Launch order: each CTA first lets the next launch start (programmatic
// dependent launch), starts its weight stream, and only then waits for the
// previous grid; activations, output and scales are touched after that wait.
// Weights must therefore not be written by the launch immediately before this
// one on the stream (uploads end with a copy or a synchronisation).
#include "ft_internal.cuh"
#include "ft_tc.cuh"

namespace ft {
namespace {

#ifndef FT_GV_WARPS
#define FT_GV_WARPS 8
#endif
// one n8 column block (<= 8 operand columns): units of FT_GV_MB1 m-blocks
#ifndef FT_GV_MB1
#define FT_GV_MB1 4
#endif
#ifndef FT_GV_DEPTH1
#define FT_GV_DEPTH1 5
#endif
// launches of <= 4 problems, one n8 block: units of 2 m-blocks, so a single
// GEMV spreads over more warps
#ifndef FT_GV_DEPTH1S
#define FT_GV_DEPTH1S 4
#endif
#ifndef FT_GV_CTAS1
#define FT_GV_CTAS1 2
#endif
// two n8 blocks: units of 2 m-blocks
#ifndef FT_GV_DEPTH2
#define FT_GV_DEPTH2 8
#endif
// int8 activations of more tokens go to the tensor-core engine: at 9-16
// tokens it measured 8.7-8.9 us per call on W[5632, 2048] and 13.5-13.7 us on
// W[11008, 4096] against 10.8-13.2 and 15.2-18.1 us here
#ifndef FT_GV_I8_MAX_TOKENS
#define FT_GV_I8_MAX_TOKENS 8
#endif
#ifndef FT_GV_GRID_SMALL
#define FT_GV_GRID_SMALL 1
#endif
#ifndef FT_GV_GRID_LARGE
#define FT_GV_GRID_LARGE 2
#endif
#ifndef FT_GV_SLEEP_NS
#define FT_GV_SLEEP_NS 1000  // suspend hint of the ring waits (woken when the copy lands)
#endif
constexpr int kW = FT_GV_WARPS;
constexpr int kThreads = kW * 32;
constexpr int kMaxProb = 64;

// Per operand width: m-blocks per unit (a unit is MB m-blocks x one 128-K
// chunk, MB * 512 contiguous bytes), ring depth in units, CTAs per SM.
template <int NB>
struct GvCfg;
template <>
struct GvCfg<1> {
  static constexpr int MB = FT_GV_MB1, DEPTH = FT_GV_DEPTH1, CTAS = FT_GV_CTAS1;
};
template <>
struct GvCfg<2> {
  static constexpr int MB = 2, DEPTH = FT_GV_DEPTH2, CTAS = 2;
};

// 2:4 sparse weights: an m-block of one chunk is the 384-byte metadata + sign
// record of the sparse MMA operand (ft_internal.cuh); the ring is deepened so
// that about as many bytes are in flight per warp as for dense units.
#ifndef FT_GV_SPDEPTH1
#define FT_GV_SPDEPTH1 5
#endif
#ifndef FT_GV_SPDEPTH2
#define FT_GV_SPDEPTH2 10
#endif
// m-blocks per unit; `small`: a launch of <= 4 problems
constexpr int unit_mb(int nb, bool sp, bool small) {
  return (small && nb == 1) ? 2 : (nb == 1 ? FT_GV_MB1 : 2);
}
template <int NB, bool SP, bool SMALL>
struct GvUnit {
  static constexpr int MB = unit_mb(NB, SP, SMALL);
  static constexpr int DEPTH = SP ? (NB == 1 ? FT_GV_SPDEPTH1 : FT_GV_SPDEPTH2)
                                  : (MB != GvCfg<NB>::MB ? FT_GV_DEPTH1S : GvCfg<NB>::DEPTH);
  static constexpr int MU = SP ? 24 : 32;    // uint4 per m-block of one chunk
  static constexpr uint32_t BYTES = MB * MU * 16;  // one unit
};

struct GvSeg {  // one activation source and the problems that read it
  const void* x;  // [seq, ldx]: f32, bf16 or int8 codes
  const float* kscale;  // column-block scales folded into x (blocked matmul), or null
  int64_t K, kblock;
  int64_t ldx;    // elements per activation row (K, or the gate/up width with act)
  int32_t act;    // x holds interleaved gate/up rows: element k = expert_act(gate_k, up_k)
  int32_t units;         // sum over its problems of row-blocks x chunks (< 2^31)
  int32_t q_cta, r_cta;  // units / n_cta, units % n_cta: CTA c starts near c*q + min(c, r)
  int32_t seq, n_chunks;
  int32_t prob_begin, prob_end;
  int32_t cta_begin, n_cta;
  int32_t upp;         // units per problem when all its problems share one shape, else 0
  int32_t unc, unrb;   // that shape's chunks and row-blocks
};

struct GvProb {
  const uint4* codes;
  const float* row_scales;
  const float* sx;  // int8 mode: per-token scale
  float* y;
  int64_t ldy, rows;
  int32_t unit_begin;  // first unit of this problem within its segment
  int32_t n_chunks, n_rb;
};

template <int NP>
struct GvParamsT {
  int nseg, nprob, xkind, D;
  int* err;  // device error word: a bounded wait that gave up records its site
  GvSeg g[NP];
  GvProb p[NP];
};
// Host staging and the large launch; calls of <= kSmallProb problems launch
// with a small parameter block (cheaper to launch).
using GvParams = GvParamsT<kMaxProb>;
constexpr int kSmallProb = 4;

__device__ __forceinline__ void mma_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Sparse MMA m16n8k64 (2:4 along K): A = the 16 x 32 compressed +-1 values,
// e = this lane's metadata word (selector 0: every lane contributes).
__device__ __forceinline__ void mma_sp_s8(int (&c)[4], const uint32_t (&a)[4], const uint4& b,
                                          uint32_t e) {
  asm volatile(
      "mma.sp::ordered_metadata.sync.aligned.m16n8k64.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9, %10, %11}, {%0, %1, %2, %3}, %12, 0x0;"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w),
        "r"(e));
}

// Four sign bits (bit e set = -1) -> the A register of four s8 values +-1:
// the bits spread to the low bit of each byte, then 0x01 ^ 0xFE per set bit.
__device__ __forceinline__ uint32_t sign_bytes(uint32_t bits) {
  const uint32_t spread = ((bits & 0xFu) * 0x00204081u) & 0x01010101u;
  return 0x01010101u ^ (spread * 0xFEu);
}

// Problem / row-block / chunk cursor over a segment's units.
struct Cursor {
  int p;
  int rb, c;
};

// Problem of segment s holding unit u: arithmetic when the segment's
// problems share one shape, else a scan of their first units.
template <class PT>
__device__ __forceinline__ int find_prob(const PT& P, const GvSeg& s, int u) {
  if (s.upp > 0) return s.prob_begin + (int)(u / s.upp);
  int pi = s.prob_begin;
  while (pi + 1 < s.prob_end && P.p[pi + 1].unit_begin <= u) ++pi;
  return pi;
}

template <class PT>
__device__ __forceinline__ Cursor cursor_at(const PT& P, const GvSeg& s, int u) {
  Cursor k;
  k.p = find_prob(P, s, u);
  if (s.upp > 0) {
    const int rel = u - (k.p - s.prob_begin) * s.upp;
    k.rb = rel / s.unc;
    k.c = rel - k.rb * s.unc;
  } else {
    const GvProb& q = P.p[k.p];
    const int rel = u - q.unit_begin;
    k.rb = rel / q.n_chunks;
    k.c = rel - k.rb * q.n_chunks;
  }
  return k;
}

// First unit of CTA `c` of a segment: c * q + min(c, r) (an even split of
// the units) rounded down to a row-block boundary; CTA c-1 computes the same
// value as its end.  32-bit arithmetic (segments have fewer than 2^31 units).
template <class PT>
__device__ __forceinline__ int cta_boundary(const PT& P, const GvSeg& s, int c) {
  if (c <= 0) return 0;
  if (c >= s.n_cta) return s.units;
  const int t = c * s.q_cta + (c < s.r_cta ? c : s.r_cta);
  if (s.upp > 0) {
    const int pbase = t / s.upp * s.upp;
    return pbase + (t - pbase) / s.unc * s.unc;
  }
  const GvProb& q = P.p[find_prob(P, s, t)];
  return q.unit_begin + (t - q.unit_begin) / q.n_chunks * q.n_chunks;
}

__device__ __forceinline__ float4 load_x4(const void* x, int xkind, int64_t row, int64_t k,
                                          int64_t K, int64_t ldx);

// load_x4 with the segment's column-block scales applied (x' = scale * x), or
// the activation of interleaved gate/up rows (S.act)
__device__ __forceinline__ float4 load_xs4(const GvSeg& S, int xkind, int64_t row, int64_t k) {
  if (S.act) {
    // k .. k+3 lie in one 16-wide group: gate row 32 (k/16) + k%16, up row 16 further
    float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const float* gp = static_cast<const float*>(S.x) + row * S.ldx + 32 * (k >> 4) + (k & 15);
    float* e = reinterpret_cast<float*>(&v);
    if (k + 4 <= S.K && (reinterpret_cast<uintptr_t>(gp) & 15) == 0) {
      const float4 g4 = __ldg(reinterpret_cast<const float4*>(gp));
      const float4 u4 = __ldg(reinterpret_cast<const float4*>(gp + 16));
      v = make_float4(expert_act(g4.x, u4.x, S.act), expert_act(g4.y, u4.y, S.act),
                      expert_act(g4.z, u4.z, S.act), expert_act(g4.w, u4.w, S.act));
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (k + i < S.K) e[i] = expert_act(__ldg(gp + i), __ldg(gp + 16 + i), S.act);
    }
    return v;
  }
  float4 v = load_x4(S.x, xkind, row, k, S.K, S.ldx);
  if (S.kscale) {
    float* e = reinterpret_cast<float*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (k + i < S.K) e[i] = __fmul_rn(e[i], S.kscale[(k + i) / S.kblock]);
  }
  return v;
}

__device__ __forceinline__ float4 load_x4(const void* x, int xkind, int64_t row, int64_t k,
                                          int64_t K, int64_t ldx) {
  // elements k .. k+3 of row `row` (rows of ldx elements; zero past K)
  float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  const int64_t i = row * ldx + k;
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

// Fragment word of (4 consecutive K at quad q, column n): chunk q/32, k-step
// j = (q%32)/8, half kk = (q%8)/4, lane 4*(n%8) + q%4; stored as
// [chunk][n/8][j/2][lane] uint4 holding words (b0, b1) of k-steps 2h, 2h+1.
// That uint4 is also the B operand (b0..b3) of the sparse m16n8k64 MMA over
// K 64h .. 64h+63 of the chunk, so dense and 2:4 weights share the layout.
__device__ __forceinline__ int frag_word(int q, int n, int nb) {
  const int c = q >> 5, j = (q >> 3) & 3, kk = (q >> 2) & 1, rr = q & 3;
  const int lane = 4 * (n & 7) + rr;
  return ((((c * nb + (n >> 3)) * 2 + (j >> 1)) * 32 + lane) << 2) + 2 * (j & 1) + kk;
}

// Weight-stream producer of one warp: walks the warp's units in order; the
// unit (row-block rb, chunk c) is the MB m-blocks (rb % (8/MB)) * MB .. +MB-1
// of block (rb / (8/MB), c), fetched with one bulk copy.  Offsets are in
// uint4 from the problem's codes; the step to the next unit is +256 (next
// chunk) within a row-block, then back to chunk 0 of the next row-block
// (same tile) or on to the next tile.  Every lane keeps the (uniform) state;
// lane 0 issues the copies.
struct Producer {
  const uint4* base;  // codes of the current problem
  uint32_t off;       // uint4 offset of the current unit
  int nc, nrb, rb, c, p;
};

template <int MB, bool SP, class PT>
__device__ __forceinline__ void prod_at(Producer& w, const PT& P, int p, int rb, int c) {
  constexpr int RPT = 8 / MB;  // row-blocks per tile
  constexpr int MU = SP ? 24 : 32, BU = SP ? 192 : 256;
  const GvProb& q = P.p[p];
  w.base = q.codes;
  w.nc = q.n_chunks;
  w.nrb = q.n_rb;
  w.p = p;
  w.rb = rb;
  w.c = c;
  w.off = (uint32_t)(((rb / RPT) * q.n_chunks + c) * BU + (rb % RPT) * (MB * MU));
}

template <int MB, bool SP, class PT>
__device__ __forceinline__ void prod_next(Producer& w, const PT& P) {
  constexpr int RPT = 8 / MB;
  constexpr uint32_t MU = SP ? 24 : 32, BU = SP ? 192 : 256;
  if (++w.c < w.nc) {
    w.off += BU;
  } else {
    w.c = 0;
    if (++w.rb < w.nrb)
      w.off += (w.rb % RPT) ? MB * MU - (uint32_t)(w.nc - 1) * BU : MB * MU;
    else if (w.p + 1 < P.nprob)
      prod_at<MB, SP>(w, P, w.p + 1, 0, 0);
  }
}

// lane 0: the current unit into ring slot `dst`, completion counted on `bar`;
// the weights are read once per launch, so they are marked evict-first in L2.
template <int MB, bool SP>
__device__ __forceinline__ void prod_copy(const Producer& w, uint32_t dst, uint32_t bar,
                                          uint64_t policy) {
  constexpr uint32_t bytes = MB * (SP ? (uint32_t)kSparseMbBytes : 512u);
  tc::mbar_arrive_expect_tx(bar, bytes);
  tc::bulk_g2s_hint(dst, w.base + w.off, bytes, bar, policy);
}

// Non-finite activations of the CTA's segment (shared memory): count and the
// first kNfCap positions per token, and what the fix-up needs to read weights.
struct GvNf {
  const int* cnt;             // [4]
  const int (*pos)[kNfCap];   // [4][kNfCap]
  const void* x;              // segment activations [seq, K]
  int64_t K;
  bool bf16;
  int format;
  const float* kscale;        // column-block scales, or null
  int64_t kblock;
  int64_t ldx;                // elements per activation row
  int act;                    // interleaved gate/up activations
};

// Output of one row-block (MB m-blocks) from its exact digit sums fin:
// fin[m][nb][e] = rows 16m + g (+8 for e >= 2), column 8nb + 2r + (e & 1).
template <int NB, int MB>
__device__ __forceinline__ void rowblock_store(const int (&fin)[MB][NB][4], const GvProb& q, int rb,
                                               int seq, int D, const int* colsum,
                                               const double* tok_scale, const GvNf& nf, int g,
                                               int r) {
  const int64_t rbase = (int64_t)rb * (16 * MB);
  auto finish = [&](int t, int64_t R, float y) {
    if (nf.cnt[t] != 0)
      y = nonfinite_row(y, reinterpret_cast<const uint8_t*>(q.codes), nf.format, q.n_chunks, R,
                        static_cast<const char*>(nf.x) + (int64_t)t * nf.ldx * (nf.bf16 ? 2 : 4),
                        nf.bf16, nf.K, nf.pos[t], nf.cnt[t], q.row_scales[R], nf.kscale,
                        nf.kblock, nf.act);
    q.y[t * q.ldy + R] = y;
  };
  if (D == 8) {
    // token t = nb: lane r holds digits 2r and 2r + 1 of both row halves
#pragma unroll
    for (int m = 0; m < MB; ++m)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        if (nb >= seq) continue;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int n0 = 8 * nb + 2 * r;
          double part = (double)(fin[m][nb][2 * h] - colsum[n0]) * (double)(1ll << (16 * r)) +
                        (double)(fin[m][nb][2 * h + 1] - colsum[n0 + 1]) *
                            (double)(1ll << (16 * r + 8));
          part += __shfl_xor_sync(0xffffffffu, part, 1);
          part += __shfl_xor_sync(0xffffffffu, part, 2);
          const int64_t R = rbase + 16 * m + g + 8 * h;
          if (r == 0 && R < q.rows)
            finish(nb, R, (float)(part * tok_scale[nb] * (double)q.row_scales[R]));
        }
      }
    return;
  }
  if (D == 1) {
#pragma unroll
    for (int m = 0; m < MB; ++m)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int col = 8 * nb + 2 * r + (e & 1);
          const int64_t R = rbase + 16 * m + g + 8 * (e >> 1);
          if (col < seq && R < q.rows)
            q.y[col * q.ldy + R] = __fmul_rn(
                __fmul_rn((float)(fin[m][nb][e] - colsum[col]), q.sx[col]), q.row_scales[R]);
        }
  } else {
    // token t = col / 4 lives in lanes r = 2(t%2) (digits 0, 1) and r + 1 (digits 2, 3)
#pragma unroll
    for (int m = 0; m < MB; ++m)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        int hi[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) hi[e] = __shfl_xor_sync(0xffffffffu, fin[m][nb][e], 1);
        const int t = 2 * nb + (r >> 1);
        if ((r & 1) == 0 && t < seq) {
          const int n0 = 4 * t;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int64_t R = rbase + 16 * m + g + 8 * h;
            if (R >= q.rows) continue;
            const long long d0 = fin[m][nb][2 * h] - colsum[n0];
            const long long d1 = fin[m][nb][2 * h + 1] - colsum[n0 + 1];
            const long long d2 = hi[2 * h] - colsum[n0 + 2];
            const long long d3 = hi[2 * h + 1] - colsum[n0 + 3];
            const long long s4 = d0 + d1 * 256 + d2 * 65536 + d3 * 16777216;
            finish(t, R, (float)((double)s4 * tok_scale[t] * (double)q.row_scales[R]));
          }
        }
      }
  }
}

// DT: digits per token (1: int8 codes; 4 or 8: fp32/bf16), a template
// parameter so that each instance carries only its own operand build.
template <int NB, int NP, bool SP, int DT>
__global__ void __launch_bounds__(kThreads, GvCfg<NB>::CTAS)
    gemv_kernel(const __grid_constant__ GvParamsT<NP> P) {
  using U = GvUnit<NB, SP, (NP <= kSmallProb)>;
  constexpr int MB = U::MB, kDepth = U::DEPTH;
  constexpr int kU4 = MB * U::MU;  // uint4 per unit
  constexpr int kRingBytes = kW * kDepth * (int)U::BYTES;
  extern __shared__ __align__(16) uint4 dyn[];
  // dynamic: weight ring | partial sums [warp][NB][MB][4][32] int | fragments
  uint4* ring = dyn;
  int* part = reinterpret_cast<int*>(dyn + kRingBytes / 16);
  uint32_t* frag = reinterpret_cast<uint32_t*>(part + kW * NB * MB * 128);
  __shared__ int colsum[16];
  __shared__ double tok_scale[4];
  __shared__ float red_f[kW][4];
  __shared__ int red_n[kW][4];
  __shared__ int nf_cnt[4];
  __shared__ int nf_pos[4][kNfCap];
  __shared__ int part_id[kW];
  __shared__ __align__(8) uint64_t full_bar[kW][kDepth];

  tc::pdl_launch_dependents();

  int si = 0;
  while (si + 1 < P.nseg && P.g[si + 1].cta_begin <= (int)blockIdx.x) ++si;
  const GvSeg& S = P.g[si];
  const int cta = (int)blockIdx.x - S.cta_begin;
  const int A = cta_boundary(P, S, cta), B = cta_boundary(P, S, cta + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, r = lane & 3;
  const int u0 = A + (int)((int64_t)(B - A) * warp / kW), u1 = A + (int)((int64_t)(B - A) * (warp + 1) / kW);
  const int n = (int)(u1 - u0);

  // ---- start the weight stream: per-warp ring of kDepth unit slots, one
  // mbarrier each (phase i / kDepth of slot i % kDepth = unit i landed)
  uint4* const myring = ring + warp * (kDepth * kU4);
  const uint32_t ring_s = tc::smem_u32(myring);
  const uint32_t bar_s = tc::smem_u32(&full_bar[warp][0]);
  const Cursor start = n > 0 ? cursor_at(P, S, u0) : Cursor{S.prob_begin, 0, 0};
  Producer pr;
  prod_at<MB, SP>(pr, P, start.p, start.rb, start.c);
  if (lane == 0) {
#pragma unroll
    for (int d = 0; d < kDepth; ++d) tc::mbar_init(bar_s + 8 * d, 1);
    tc::fence_barrier_init();
  }
  __syncwarp();
  const uint64_t l2_policy = tc::policy_evict_first();
  int issued = 0;
#pragma unroll
  for (int d = 0; d < kDepth; ++d) {
    if (issued < n) {
      if (lane == 0) prod_copy<MB, SP>(pr, ring_s + d * U::BYTES, bar_s + 8 * d, l2_policy);
      prod_next<MB, SP>(pr, P);
      ++issued;
    }
  }

  // ---- activation fragments of this CTA's segment (after the previous grid)
  tc::pdl_wait();
  constexpr int D = DT;
  const int seq = S.seq;
  const int nquad = S.n_chunks * 32;
  {
    // columns no token uses must read as zero
    if (D * seq < 8 * NB) {
      uint4* f4 = reinterpret_cast<uint4*>(frag);
      for (int i = tid; i < S.n_chunks * NB * 64; i += kThreads) f4[i] = make_uint4(0, 0, 0, 0);
    }
    if (tid < 16) colsum[tid] = 0;
    if (tid < 4) nf_cnt[tid] = 0;
    if (tid < kW) part_id[tid] = -1;
  }
  if (D == 1) __syncthreads();  // zero-fill above before the word stores below
  // One token at a time: its x quads stay in registers between the absmax
  // and the digit split (K up to 4 * kRQ * kThreads in one load).
  constexpr int kRQ = 4;
  // (int8 activations: four tokens per pass of this loop, see below)
  for (int t = 0; t < seq; t += (D == 1 ? 4 : 1)) {
    int cs[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const int ntok = D == 1 ? (seq - t < 4 ? seq - t : 4) : 1;
    if (D != 1) {
      float4 xr[kRQ];
      float am = 0.0f;
      int nnf = 0;  // this thread's non-finite elements
      auto scan = [&](float4& v) {
        float* e = reinterpret_cast<float*>(&v);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (is_nonfinite(e[i])) {
            ++nnf;
            e[i] = 0.0f;
          }
          am = fmaxf(am, fabsf(e[i]));
        }
      };
#pragma unroll
      for (int j = 0; j < kRQ; ++j) {
        const int q = tid + j * kThreads;
        xr[j] = q < nquad ? load_xs4(S, P.xkind, t, 4 * (int64_t)q)
                          : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        scan(xr[j]);
      }
      for (int q = tid + kRQ * kThreads; q < nquad; q += kThreads) {
        float4 v = load_xs4(S, P.xkind, t, 4 * (int64_t)q);
        scan(v);
      }
      // warp: absmax, and an exclusive scan of the non-finite counts (only
      // when the warp holds any)
      int nf_before = 0, nf_warp = 0;
      if (__any_sync(0xffffffffu, nnf != 0)) {
        int incl = nnf;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int v = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += v;
        }
        nf_before = incl - nnf;
        nf_warp = __shfl_sync(0xffffffffu, incl, 31);
      }
      // |x| >= 0 orders like its bit pattern: one warp-wide integer max
      am = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(am)));
      if (lane == 0) {
        red_f[warp][t] = am;
        red_n[warp][t] = nf_warp;
      }
      __syncthreads();
      float a = 0.0f;
      int nf_tot = 0;
#pragma unroll
      for (int w = 0; w < kW; ++w) {
        a = fmaxf(a, red_f[w][t]);
        if (w < warp) nf_before += red_n[w][t];
        nf_tot += red_n[w][t];
      }
      if (nf_tot != 0) {
        // record this thread's non-finite positions (in K order within the
        // thread; the fix-up does not depend on the order)
        if (tid == 0) nf_cnt[t] = nf_tot;
        if (nnf != 0 && nf_tot <= kNfCap) {
          int slot = nf_before;
          for (int q = tid; q < nquad; q += kThreads) {
            const float4 v = load_xs4(S, P.xkind, t, 4 * (int64_t)q);
            const float e4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
              if (is_nonfinite(e4[i])) nf_pos[t][slot++] = 4 * q + i;
          }
        }
      }
      const int sh = a > 0.0f ? digit_shift(a, D) : 0;
      if (tid == 0) tok_scale[t] = a > 0.0f ? __longlong_as_double((long long)(1023 - sh) << 52) : 0.0;
      const int s1 = sh > 127 ? 127 : (sh < -126 ? -126 : sh);
      const float f1 = __int_as_float((s1 + 127) << 23);
      const float f2 = __int_as_float((sh - s1 + 127) << 23);
      // Byte permutes gather digit d of four elements (bytes of U0..U3) into
      // one word: [byte d of U0, U1, U2, U3].
      auto gather = [](uint32_t u0, uint32_t u1, uint32_t u2, uint32_t u3, uint32_t (&wd)[4]) {
        const uint32_t lo01 = __byte_perm(u0, u1, 0x5140), lo23 = __byte_perm(u2, u3, 0x5140);
        const uint32_t hi01 = __byte_perm(u0, u1, 0x7362), hi23 = __byte_perm(u2, u3, 0x7362);
        wd[0] = __byte_perm(lo01, lo23, 0x5410);
        wd[1] = __byte_perm(lo01, lo23, 0x7632);
        wd[2] = __byte_perm(hi01, hi23, 0x5410);
        wd[3] = __byte_perm(hi01, hi23, 0x7632);
      };
      auto split = [&](float4 v, int q) {
        if (q >= kRQ * kThreads) {  // reloaded quads: non-finite -> 0
          if (is_nonfinite(v.x)) v.x = 0.0f;
          if (is_nonfinite(v.y)) v.y = 0.0f;
          if (is_nonfinite(v.z)) v.z = 0.0f;
          if (is_nonfinite(v.w)) v.w = 0.0f;
        }
        const int base = frag_word(q, D * t, NB);  // digit d: lane + 4d, word + 16d
        if (D == 4) {
          // X = round(x * 2^sh), |X| < 2^30.  With U = X + 0x808080 the low
          // three bytes of U are the low signed base-256 digits + 128 and the
          // top byte is the top digit (|.| <= 64); the XOR re-signs the low three.
          uint32_t wd[4];
          gather((uint32_t)__float2int_rn(__fmul_rn(__fmul_rn(v.x, f1), f2)) + 0x808080u,
                 (uint32_t)__float2int_rn(__fmul_rn(__fmul_rn(v.y, f1), f2)) + 0x808080u,
                 (uint32_t)__float2int_rn(__fmul_rn(__fmul_rn(v.z, f1), f2)) + 0x808080u,
                 (uint32_t)__float2int_rn(__fmul_rn(__fmul_rn(v.w, f1), f2)) + 0x808080u, wd);
          wd[0] ^= 0x80808080u;
          wd[1] ^= 0x80808080u;
          wd[2] ^= 0x80808080u;
#pragma unroll
          for (int d = 0; d < 4; ++d) {
            cs[d] = __dp4a((int)wd[d], 0x01010101, cs[d]);
            frag[base + 16 * d] = wd[d];
          }
        } else {
          // X = round(x * 2^sh), |X| < 2^62, U = X + 0x0080808080808080: bytes
          // 0..6 of U are the low digits + 128, byte 7 the top digit.
          const unsigned long long b7 = 0x0080808080808080ull;
          const unsigned long long U0 = (unsigned long long)__float2ll_rn(__fmul_rn(__fmul_rn(v.x, f1), f2)) + b7;
          const unsigned long long U1 = (unsigned long long)__float2ll_rn(__fmul_rn(__fmul_rn(v.y, f1), f2)) + b7;
          const unsigned long long U2 = (unsigned long long)__float2ll_rn(__fmul_rn(__fmul_rn(v.z, f1), f2)) + b7;
          const unsigned long long U3 = (unsigned long long)__float2ll_rn(__fmul_rn(__fmul_rn(v.w, f1), f2)) + b7;
          uint32_t lo[4], hi[4];
          gather((uint32_t)U0, (uint32_t)U1, (uint32_t)U2, (uint32_t)U3, lo);
          gather((uint32_t)(U0 >> 32), (uint32_t)(U1 >> 32), (uint32_t)(U2 >> 32),
                 (uint32_t)(U3 >> 32), hi);
#pragma unroll
          for (int d = 0; d < 4; ++d) {
            lo[d] ^= 0x80808080u;
            if (d < 3) hi[d] ^= 0x80808080u;
            cs[d] = __dp4a((int)lo[d], 0x01010101, cs[d]);
            cs[d + 4] = __dp4a((int)hi[d], 0x01010101, cs[d + 4]);
            frag[base + 16 * d] = lo[d];
            frag[base + 16 * (d + 4)] = hi[d];
          }
        }
      };
#pragma unroll
      for (int j = 0; j < kRQ; ++j) {
        const int q = tid + j * kThreads;
        if (q < nquad) split(xr[j], q);
      }
      for (int q = tid + kRQ * kThreads; q < nquad; q += kThreads)
        split(load_xs4(S, P.xkind, t, 4 * (int64_t)q), q);
    } else {
      // int8: tokens t..t+ntok-1 together, the 16 words of four tokens x four
      // quads loaded before any is used (a token at a time, each quad's load
      // latency was paid in turn: ~1 us per token at K = 4096)
      const int8_t* xq[4];
      bool fast = (S.K & 3) == 0 && (S.ldx & 3) == 0;
#pragma unroll
      for (int tt = 0; tt < 4; ++tt) {
        xq[tt] = static_cast<const int8_t*>(S.x) + (int64_t)(t + (tt < ntok ? tt : 0)) * S.ldx;
        fast = fast && (reinterpret_cast<uintptr_t>(xq[tt]) & 3) == 0;
      }
      for (int q0 = tid; q0 < nquad; q0 += 4 * kThreads) {
        uint32_t wv[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int tt = 0; tt < 4; ++tt) {
            const int q = q0 + j * kThreads;
            const int64_t k = 4 * (int64_t)q;
            uint32_t w = 0u;
            if (q < nquad && tt < ntok) {
              if (fast) {
                if (k < S.K) w = __ldg(reinterpret_cast<const uint32_t*>(xq[tt] + k));
              } else {
#pragma unroll
                for (int e = 0; e < 4; ++e)
                  if (k + e < S.K) w |= (uint32_t)(xq[tt][k + e] & 0xFF) << (8 * e);
              }
            }
            wv[j][tt] = w;
          }
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int tt = 0; tt < 4; ++tt) {
            const int q = q0 + j * kThreads;
            if (q < nquad && tt < ntok) {
              cs[tt] = __dp4a((int)wv[j][tt], 0x01010101, cs[tt]);
              frag[frag_word(q, t + tt, NB)] = wv[j][tt];
            }
          }
      }
    }
    // column sums: one warp-wide integer add per column, one shared atomic
    // per warp and column
    // (2:4 weights need none: their A operand is w itself, not w + 1)
    // (int8: column t + d is token t + d's single digit)
#pragma unroll
    for (int d = 0; d < 8; ++d) {
      if (d < (D == 1 ? ntok : D) && !SP) {
        const int v = __reduce_add_sync(0xffffffffu, cs[d]);
        if (lane == 0) atomicAdd(&colsum[t * D + d], v);
      }
    }
  }
  __syncthreads();
  const GvNf nfv{nf_cnt, nf_pos, S.x, S.K, P.xkind == 1, SP ? 1 : 0, S.kscale, S.kblock,
                 S.ldx, S.act};

  // ---- the weight stream against the fragments, one row-block segment at a time
  int acc[MB][NB][4][4];
#pragma unroll
  for (int m = 0; m < MB; ++m)
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int j = 0; j < 4; ++j)
        acc[m][nb][j][0] = acc[m][nb][j][1] = acc[m][nb][j][2] = acc[m][nb][j][3] = 0;
  const uint4* const fbase = reinterpret_cast<const uint4*>(frag) + lane;
  int slot = 0;
  uint32_t phase = 0;
  int consumed = 0;
  bool ok = true;
  int cp = start.p, crb = start.rb, c0 = start.c;
  int left = n;
  bool keep = false;  // the last row-block is unfinished and owned by this warp
  while (left > 0) {
    const int nc = P.p[cp].n_chunks;
    const int cnt = nc - c0 < left ? nc - c0 : left;
    const uint4* fp = fbase + c0 * (NB * 64);
    for (int k = 0; k < cnt; ++k) {
      ok = ok && tc::mbar_wait_sleep(bar_s + 8 * slot, phase, P.err, 60, FT_GV_SLEEP_NS);
      if (!ok) break;
      if constexpr (!SP) {
        uint4 w[MB];
#pragma unroll
        for (int m = 0; m < MB; ++m) w[m] = myring[slot * kU4 + m * 32 + lane];
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
          const uint4 blo = fp[nb * 64], bhi = fp[nb * 64 + 32];
          const uint32_t bj[4][2] = {{blo.x, blo.y}, {blo.z, blo.w}, {bhi.x, bhi.y}, {bhi.z, bhi.w}};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t M = 0x03030303u << (2 * j);
#pragma unroll
            for (int m = 0; m < MB; ++m)
              mma_u8s8(acc[m][nb][j], w[m].x & M, w[m].y & M, w[m].z & M, w[m].w & M, bj[j][0],
                       bj[j][1]);
          }
        }
      } else {
        // 2:4 sparse: per m-block and k64 step, this lane's metadata word and
        // 16 sign bits form the A operand of one sparse MMA per operand block
        // (A holds the weights +-1 themselves: no column-sum correction).
        const unsigned char* rec0 = reinterpret_cast<const unsigned char*>(myring + slot * kU4);
#pragma unroll
        for (int m = 0; m < MB; ++m) {
          const unsigned char* rec = rec0 + m * kSparseMbBytes;
          const uint2 meta = reinterpret_cast<const uint2*>(rec)[lane];
          const uint32_t sg = reinterpret_cast<const uint32_t*>(rec + 256)[lane];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t a[4] = {sign_bytes(sg >> (16 * h)), sign_bytes(sg >> (16 * h + 4)),
                                   sign_bytes(sg >> (16 * h + 8)), sign_bytes(sg >> (16 * h + 12))};
#pragma unroll
            for (int nb = 0; nb < NB; ++nb)
              mma_sp_s8(acc[m][nb][0], a, fp[nb * 64 + 32 * h], h ? meta.y : meta.x);
          }
        }
      }
      ++consumed;
      // every lane's reads of the slot are done (the MMAs took them): refill it
      __syncwarp();
      if (issued < n) {
        if (lane == 0) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          prod_copy<MB, SP>(pr, ring_s + slot * U::BYTES, bar_s + 8 * slot, l2_policy);
        }
        prod_next<MB, SP>(pr, P);
        ++issued;
      }
      if (++slot == kDepth) {
        slot = 0;
        phase ^= 1u;
      }
      fp += NB * 64;
    }
    if (!ok) break;
    left -= cnt;
    const bool ends = c0 + cnt == nc;  // this segment reaches the row-block's last chunk
    int fin[MB][NB][4];
#pragma unroll
    for (int m = 0; m < MB; ++m)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          fin[m][nb][e] = SP ? acc[m][nb][0][e]
                             : acc[m][nb][0][e] + (acc[m][nb][1][e] >> 2) +
                                   (acc[m][nb][2][e] >> 4) + (acc[m][nb][3][e] >> 6);
    if (c0 != 0) {
      // first row-block of this warp, begun by an earlier warp: hand it over
#pragma unroll
      for (int m = 0; m < MB; ++m)
#pragma unroll
        for (int nb = 0; nb < NB; ++nb)
#pragma unroll
          for (int e = 0; e < 4; ++e)
            part[(((warp * NB + nb) * MB + m) * 4 + e) * 32 + lane] = fin[m][nb][e];
      if (lane == 0) part_id[warp] = P.p[cp].unit_begin + crb * nc;
    } else if (ends) {
      rowblock_store<NB, MB>(fin, P.p[cp], crb, seq, D, colsum, tok_scale, nfv, g, r);
    } else {
      keep = true;  // finished after the stream, with the later warps' parts
      break;
    }
#pragma unroll
    for (int m = 0; m < MB; ++m)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          acc[m][nb][j][0] = acc[m][nb][j][1] = acc[m][nb][j][2] = acc[m][nb][j][3] = 0;
    c0 = 0;
    if (++crb == P.p[cp].n_rb) {
      crb = 0;
      ++cp;
    }
  }
  if (!ok) {
    // a wait gave up: let this warp's copies still in flight land before exiting
    for (; consumed < issued; ++consumed) {
      tc::mbar_wait(bar_s + 8 * slot, phase, P.err, 61);
      if (++slot == kDepth) {
        slot = 0;
        phase ^= 1u;
      }
    }
    keep = false;
  }
  __syncthreads();  // partial sums visible

  if (!keep) return;
  // ---- the row-block this warp began but did not finish: add the later warps' parts
  const GvProb& q = P.p[cp];
  const int id = q.unit_begin + crb * q.n_chunks;
  int fin[MB][NB][4];
#pragma unroll
  for (int m = 0; m < MB; ++m)
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e)
        fin[m][nb][e] = SP ? acc[m][nb][0][e]
                           : acc[m][nb][0][e] + (acc[m][nb][1][e] >> 2) + (acc[m][nb][2][e] >> 4) +
                                 (acc[m][nb][3][e] >> 6);
  for (int w = warp + 1; w < kW; ++w) {
    if (part_id[w] != id) continue;
#pragma unroll
    for (int m = 0; m < MB; ++m)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int e = 0; e < 4; ++e) fin[m][nb][e] += part[(((w * NB + nb) * MB + m) * 4 + e) * 32 + lane];
  }
  rowblock_store<NB, MB>(fin, q, crb, seq, D, colsum, tok_scale, nfv, g, r);
}

template <int NB, bool SP, bool SMALL>
size_t smem_for(int64_t max_chunks) {
  using U = GvUnit<NB, SP, SMALL>;
  return (size_t)kW * U::DEPTH * U::BYTES + (size_t)kW * NB * U::MB * 512 +
         (size_t)max_chunks * NB * 1024;
}

size_t smem_for(int nb, bool sp, bool small, int64_t max_chunks) {
  if (small) {
    if (sp) return nb == 1 ? smem_for<1, true, true>(max_chunks) : smem_for<2, true, true>(max_chunks);
    return nb == 1 ? smem_for<1, false, true>(max_chunks) : smem_for<2, false, true>(max_chunks);
  }
  if (sp) return nb == 1 ? smem_for<1, true, false>(max_chunks) : smem_for<2, true, false>(max_chunks);
  return nb == 1 ? smem_for<1, false, false>(max_chunks) : smem_for<2, false, false>(max_chunks);
}

template <int NB, int NP, bool SP, int DT>
int launch_nb(const GvParamsT<NP>& P, int64_t ctas, size_t smem, cudaStream_t s) {
  static int attr_smem = 0;  // per template instance
  if ((int)smem > attr_smem) {
    FT_CUDA(cudaFuncSetAttribute(gemv_kernel<NB, NP, SP, DT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem));
    attr_smem = (int)smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctas);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FT_CUDA(cudaLaunchKernelEx(&cfg, gemv_kernel<NB, NP, SP, DT>, P));
  FT_LAUNCH_CHECK();
  return FT_OK;
}

template <int NB, bool SP>
int launch_sized(const GvParams& P, int64_t ctas, size_t smem, cudaStream_t s) {
  if (P.nprob <= kSmallProb) {
    static thread_local GvParamsT<kSmallProb> Q;
    Q.nseg = P.nseg;
    Q.nprob = P.nprob;
    Q.xkind = P.xkind;
    Q.D = P.D;
    Q.err = P.err;
    for (int i = 0; i < P.nseg; ++i) Q.g[i] = P.g[i];
    for (int i = 0; i < P.nprob; ++i) Q.p[i] = P.p[i];
    return P.D == 1 ? launch_nb<NB, kSmallProb, SP, 1>(Q, ctas, smem, s)
         : P.D == 4 ? launch_nb<NB, kSmallProb, SP, 4>(Q, ctas, smem, s)
                    : launch_nb<NB, kSmallProb, SP, 8>(Q, ctas, smem, s);
  }
  return P.D == 1 ? launch_nb<NB, kMaxProb, SP, 1>(P, ctas, smem, s)
       : P.D == 4 ? launch_nb<NB, kMaxProb, SP, 4>(P, ctas, smem, s)
                  : launch_nb<NB, kMaxProb, SP, 8>(P, ctas, smem, s);
}

}  // namespace

int gemv_digits(int xkind, int digits) {
  return xkind == 2 ? 1 : (digits > 4 ? 8 : 4);
}

bool gemv_fits(const ft_weight* w, int64_t seq, int xkind, int digits) {
  const int64_t ncols = seq * gemv_digits(xkind, digits);
  // int32 bound: the k-step-3 accumulator grows by <= 128 * 128 * 32 per chunk
  if ((w->format != 0 && w->format != 1) || ncols > 16 || w->n_chunks > 2048) return false;
  if (xkind == 2 && ncols > FT_GV_I8_MAX_TOKENS) return false;
  const int nb = ncols > 8 ? 2 : 1;
  return smem_for(nb, w->format == 1, false, w->n_chunks) <= (size_t)kGemvMaxSmem &&
         smem_for(nb, w->format == 1, true, w->n_chunks) <= (size_t)kGemvMaxSmem;
}

int launch_gemv(ft_ctx* ctx, int nprob, const GvLaunchProblem* probs, int xkind, bool sparse,
                int digits, cudaStream_t s) {
  FT_CHECK(nprob > 0 && nprob <= kMaxProb, FT_ERR_UNSUPPORTED, "bad GEMV group size");
  static thread_local GvParams P;
  P.xkind = xkind;
  P.err = ctx->err_word;
  P.D = gemv_digits(xkind, digits);
  // segments: problems grouped by activation (pointer, K, seq), first-seen order
  int seg_of[kMaxProb];
  int nseg = 0;
  int64_t max_cols = 0, max_chunks = 0;
  for (int i = 0; i < nprob; ++i) {
    const GvLaunchProblem& q = probs[i];
    int j = 0;
    while (j < nseg && !(P.g[j].x == q.x && P.g[j].K == q.K && P.g[j].seq == q.seq &&
                         P.g[j].kscale == q.kscale && P.g[j].kblock == q.kblock &&
                         P.g[j].act == q.act))
      ++j;
    if (j == nseg) {
      P.g[j].x = q.x;
      P.g[j].K = q.K;
      P.g[j].act = q.act;
      P.g[j].ldx = q.ldx > 0 ? q.ldx : q.K;
      P.g[j].kscale = q.kscale;
      P.g[j].kblock = q.kblock;
      P.g[j].seq = (int32_t)q.seq;
      P.g[j].n_chunks = (int32_t)ceil_div(q.K, kChunkK);
      ++nseg;
    }
    seg_of[i] = j;
    max_cols = q.seq * P.D > max_cols ? q.seq * P.D : max_cols;
    max_chunks = q.n_chunks > max_chunks ? q.n_chunks : max_chunks;
  }
  P.nseg = nseg;
  P.nprob = nprob;
  const int nb = max_cols > 8 ? 2 : 1;
  const bool small = nprob <= kSmallProb;  // the kernel instance launch_sized picks
  const int mb = unit_mb(nb, sparse, small);  // m-blocks per unit
  int64_t total = 0;
  int np = 0;
  for (int j = 0; j < nseg; ++j) {
    GvSeg& g = P.g[j];
    g.prob_begin = np;
    int64_t units = 0;
    for (int i = 0; i < nprob; ++i) {
      if (seg_of[i] != j) continue;
      const GvLaunchProblem& q = probs[i];
      GvProb& p = P.p[np++];
      p.codes = reinterpret_cast<const uint4*>(q.codes);
      p.row_scales = q.row_scales;
      p.sx = q.sx;
      p.y = q.y;
      p.ldy = q.ldy;
      p.rows = q.rows;
      p.n_chunks = (int32_t)q.n_chunks;
      p.n_rb = (int32_t)ceil_div(q.rows, 16 * mb);
      p.unit_begin = (int32_t)units;
      units += (int64_t)p.n_rb * p.n_chunks;
    }
    g.prob_end = np;
    g.units = (int32_t)units;
    total += units;
    bool uni = true;
    for (int i = g.prob_begin + 1; i < g.prob_end && uni; ++i)
      uni = P.p[i].n_chunks == P.p[g.prob_begin].n_chunks && P.p[i].n_rb == P.p[g.prob_begin].n_rb;
    g.unc = P.p[g.prob_begin].n_chunks;
    g.unrb = P.p[g.prob_begin].n_rb;
    g.upp = uni ? g.unc * g.unrb : 0;
  }
  FT_CHECK(total < (int64_t)1 << 31, FT_ERR_UNSUPPORTED, "GEMV group too large");
  // CTAs per segment in proportion to its units, at least one, at most one
  // per row-block
  // CTAs per SM the grid targets: launches of <= kSmallProb problems and
  // larger ones separately (fewer than the SM can hold leaves room for the
  // next launch's CTAs to start streaming while this one finishes).
  const int per_sm = small ? FT_GV_GRID_SMALL : FT_GV_GRID_LARGE;
  const int64_t target = (int64_t)ctx->num_sms *
                         (per_sm < (nb == 1 ? GvCfg<1>::CTAS : GvCfg<2>::CTAS)
                              ? per_sm : (nb == 1 ? GvCfg<1>::CTAS : GvCfg<2>::CTAS));
  int64_t ctas = 0;
  for (int j = 0; j < nseg; ++j) {
    GvSeg& g = P.g[j];
    int64_t rbs = 0;
    for (int i = g.prob_begin; i < g.prob_end; ++i) rbs += P.p[i].n_rb;
    int64_t c = ((int64_t)g.units * target + total / 2) / total;
    if (c < 1) c = 1;
    if (c > rbs) c = rbs;
    g.cta_begin = (int32_t)ctas;
    g.n_cta = (int32_t)c;
    g.q_cta = (int32_t)(g.units / c);
    g.r_cta = (int32_t)(g.units % c);
    ctas += c;
  }
  const size_t smem = smem_for(nb, sparse, small, max_chunks);
  FT_CHECK(smem <= (size_t)kGemvMaxSmem, FT_ERR_UNSUPPORTED, "GEMV operand too large");
  if (sparse)
    return nb == 1 ? launch_sized<1, true>(P, ctas, smem, s) : launch_sized<2, true>(P, ctas, smem, s);
  return nb == 1 ? launch_sized<1, false>(P, ctas, smem, s) : launch_sized<2, false>(P, ctas, smem, s);
}

}  // namespace ft
