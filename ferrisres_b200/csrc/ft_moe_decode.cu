// Fused MoE decode step: the whole TernaryMoELayer::forward
// (src/model/ternary_moe.rs:145-223) for up to 8 tokens in ONE persistent
// cooperative kernel, with no host round trip (the reference's decode loop
// makes several per expert: src/model/cpu_block_attn_res.rs:2284-2316).
//
// Phases, separated by grid-wide barriers (bounded waits):
//   R  router partial scores: one warp per (expert, 256-wide K part) loads
//      that part of the router row once and dots it with every token (fp32,
//      8 products per lane in order, then a butterfly) -- barrier;
//   S  every CTA sums the parts in order and routes every token, one warp
//      each (softmax with the exponentials' sum in the reference's order,
//      stable descending top-k, renormalised gates) and builds the tokens'
//      int8-digit operand in shared memory;
//   G  gate||up: work units are (pair = token x chosen expert, 64-row block);
//      a CTA's 8 warps split the unit's 128-K chunks, each streams its chunks'
//      2-bit codes with 16-byte loads and runs mma.sync m16n8k32 (u8 codes AND
//      the slot mask x s8 digits, exact int32), the warps' sums meet in shared
//      memory and the unit's 64 outputs go to global scratch -- barrier;
//      CTAs without a G unit meanwhile pull the chosen experts' down
//      weights into L2 (bulk prefetch);
//   H  every CTA forms h = SwiGLU(gate, up) (or GeLU-tanh) of every pair and
//      its operand (all loads of a row issued before any arithmetic);
//   D  down projection, same scheme -- barrier;
//   C  y[t] = sum_k w[t,k] * o[t,k] in top-k order.
// Activations use 4 base-256 digits per token (the MoE's tolerance, 1e-4 of
// the output rms; see ft_internal.cuh), two tokens (or pairs) per n8 column
// block.  Non-finite activations enter as 0 (ft_moe_forward propagates them).
#include <cstring>

#include "ft_internal.cuh"
#include "ft_moe.cuh"
#include "ft_tc.cuh"

namespace ft {
namespace {

constexpr int kMdThreads = 256, kMdWarps = 8;
constexpr int kMdMaxTok = 8, kMdMaxPairs = 16;
constexpr int kMdRows = 64;  // rows per work unit (4 m-blocks of 16)

struct MdParams {
  int T, K, E, use_gelu, x_bf16;
  int nparts;  // 256-wide K parts of the router dot
  int x_vec;   // H % 8 == 0 and x 16-byte aligned: vector loads
  int64_t H, F;
  int64_t F2;             // rows of the interleaved gate/up weight (16-row gate/up m-blocks)
  int64_t nch_h, nch_f;   // 128-K chunks of H and of F
  const void* x;          // [T, H]
  const float* router;    // [E, H]
  const void* const* tab; // [4][E]: gate_up codes, gate_up scales, down codes, down scales
  float* logits;          // [T, E, nparts] partial router scores
  float* gu;              // [P, F2] interleaved gate/up rows
  float* o;               // [P, H]
  int32_t* topk_idx;      // [T, K] (output)
  float* topk_w;          // [T, K] (output)
  float* probs;           // [T, E] (optional output)
  float* y;               // [T, H] (output)
  unsigned* bar;          // grid barrier: arrival counter, zero at launch
  int* err;
};

__device__ __forceinline__ void mma_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Operand word of (4 consecutive K at quad q, column n) in the layout
// [chunk][n8 block][k-step pair][lane] uint4 (the decode GEMV's layout).
__device__ __forceinline__ int frag_word(int q, int n, int nb) {
  const int c = q >> 5, j = (q >> 3) & 3, kk = (q >> 2) & 1, rr = q & 3;
  const int lane = 4 * (n & 7) + rr;
  return ((((c * nb + (n >> 3)) * 2 + (j >> 1)) * 32 + lane) << 2) + 2 * (j & 1) + kk;
}

// Grid-wide barrier with a bounded wait: every CTA adds 1 to a counter that
// the launch starts at zero and waits until it reaches `target` (advanced by
// the grid size per barrier).  Returns false everywhere when the wait gave up
// (site recorded in *err).
__device__ bool grid_sync(unsigned* bar, unsigned& target, int* err, int site) {
  __syncthreads();
  int ok = 1;
  if (threadIdx.x == 0) {
    target += gridDim.x;
    __threadfence();
    atomicAdd(bar, 1u);
    const unsigned long long t0 = tc::globaltimer();
    for (unsigned it = 1; tc::ld_acquire_u32(bar) < target; ++it) {
      if ((it & 63u) == 0u && tc::globaltimer() - t0 > 2000000000ull) {
        atomicExch(err, site);
        ok = 0;
        break;
      }
    }
  }
  return __syncthreads_and(ok) != 0;
}

// The 4 digit words of a quad of 4 consecutive values (x already scaled by
// f1 * f2 when passed through digit_words).
__device__ __forceinline__ void digit_words(const float (&v)[4], float f1, float f2,
                                            uint32_t (&wd)[4]) {
  uint32_t u[4];
#pragma unroll
  for (int e = 0; e < 4; ++e)
    u[e] = (uint32_t)__float2int_rn(__fmul_rn(__fmul_rn(v[e], f1), f2)) + 0x808080u;
  const uint32_t lo01 = __byte_perm(u[0], u[1], 0x5140), lo23 = __byte_perm(u[2], u[3], 0x5140);
  const uint32_t hi01 = __byte_perm(u[0], u[1], 0x7362), hi23 = __byte_perm(u[2], u[3], 0x7362);
  wd[0] = __byte_perm(lo01, lo23, 0x5410) ^ 0x80808080u;
  wd[1] = __byte_perm(lo01, lo23, 0x7632) ^ 0x80808080u;
  wd[2] = __byte_perm(hi01, hi23, 0x5410) ^ 0x80808080u;
  wd[3] = __byte_perm(hi01, hi23, 0x7632);
}

// Digit operands of NR activation rows (row r = operand column block r:
// 4 digits at columns 4 * (r & 1) + d of n8 block r >> 1), with the column
// sums and each row's scale 2^-sh.  Rows are built G at a time (G the largest
// power of two <= min(NR, 8)) by 8 / G warps each.  A thread first issues
// every load of its first kRq quads (`fetch`: raw values; predicated, no
// load past the row), then transforms them (`xform`: raw -> fp32, applied
// again when the digits are written), so a row costs about one memory round
// trip; quads past kRq per thread are loaded again in a second pass.  colsum must be zero
// on entry.  Block-wide.
constexpr int kRq = 12;
template <class Fetch, class Xform>
__device__ void build_rows(int NR, Fetch fetch, Xform xform, int64_t n, int nchunks, int nb,
                           uint32_t* frag, int (*colsum)[4], double* tok_scale, float* red) {
  using Raw = decltype(fetch(0, (int64_t)0));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = NR >= 8 ? 8 : NR >= 4 ? 4 : NR >= 2 ? 2 : 1;
  const int wpp = kMdWarps / G, slot = warp / wpp, sub = warp % wpp;
  const int nthr = 32 * wpp, ts = sub * 32 + lane;
  const int nquad = nchunks * 32;
  auto value = [&](const Raw& raw, int64_t k) -> float {
    const float v = xform(raw);
    return (k >= n || is_nonfinite(v)) ? 0.0f : v;
  };
  for (int r0 = 0; r0 < NR; r0 += G) {
    const int r = r0 + slot;
    const bool live = r < NR;
    // predicated loads (no branch), so all of them are in flight together;
    // quads past the row are not loaded at all
    Raw raw[kRq][4];
#pragma unroll
    for (int i = 0; i < kRq; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int64_t k = 4 * (int64_t)(ts + nthr * i) + e;
        raw[i][e] = (live && k < n) ? fetch(r, k) : Raw{};
      }
    // each loaded value is transformed once (quads past the row are skipped)
    float v[kRq][4];
    float am = 0.0f;
#pragma unroll
    for (int i = 0; i < kRq; ++i) {
      const int q = ts + nthr * i;
#pragma unroll
      for (int e = 0; e < 4; ++e) v[i][e] = 0.0f;
      if (q < nquad) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          v[i][e] = value(raw[i][e], 4 * (int64_t)q + e);
          am = fmaxf(am, fabsf(v[i][e]));
        }
      }
    }
    for (int q = ts + nthr * kRq; live && q < nquad; q += nthr)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int64_t k = 4 * (int64_t)q + e;
        am = fmaxf(am, fabsf(value(k < n ? fetch(r, k) : Raw{}, k)));
      }
    am = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(am)));
    if (lane == 0) red[warp] = am;
    __syncthreads();
    float a = 0.0f;
    for (int w = slot * wpp; w < slot * wpp + wpp; ++w) a = fmaxf(a, red[w]);
    const int sh = a > 0.0f ? digit_shift(a, 4) : 0;
    const int s1 = sh > 127 ? 127 : (sh < -126 ? -126 : sh);
    const float f1 = __int_as_float((s1 + 127) << 23);
    const float f2 = __int_as_float((sh - s1 + 127) << 23);
    if (live) {
      int cs[4] = {0, 0, 0, 0};
      auto emit = [&](int q, const float (&x)[4]) {
        uint32_t wd[4];
        digit_words(x, f1, f2, wd);
        const int base = frag_word(q, 4 * r, nb);
#pragma unroll
        for (int d = 0; d < 4; ++d) {
          cs[d] = __dp4a((int)wd[d], 0x01010101, cs[d]);
          frag[base + 16 * d] = wd[d];
        }
      };
#pragma unroll
      for (int i = 0; i < kRq; ++i)
        if (ts + nthr * i < nquad) emit(ts + nthr * i, v[i]);
      for (int q = ts + nthr * kRq; q < nquad; q += nthr) {
        float x[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int64_t k = 4 * (int64_t)q + e;
          x[e] = value(k < n ? fetch(r, k) : Raw{}, k);
        }
        emit(q, x);
      }
#pragma unroll
      for (int d = 0; d < 4; ++d) {
        const int c = __reduce_add_sync(0xffffffffu, cs[d]);
        if (lane == 0) atomicAdd(&colsum[r][d], c);
      }
      if (ts == 0) tok_scale[r] = a > 0.0f ? __longlong_as_double((long long)(1023 - sh) << 52) : 0.0;
    }
    __syncthreads();  // red is reused by the next round
  }
}

// One work unit: rows [64 rb, 64 rb + 64) of a tiled weight (codes, nch
// chunks) against operand column block `col`; out[R] = scale[R] * (exact sum)
// for R < rows.  Block-wide (the 8 warps split the chunks).
__device__ void unit_matvec(const uint4* codes, const float* scale, int64_t rows, int64_t nch,
                            int64_t rb, int col, int nb, const uint4* frag4, const int (*colsum)[4],
                            const double* tok_scale, int* part, float* out) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t tile = rb >> 1;
  const int half = (int)(rb & 1);
  int acc[4][4][4];
#pragma unroll
  for (int m = 0; m < 4; ++m)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[m][j][0] = acc[m][j][1] = acc[m][j][2] = acc[m][j][3] = 0;
  for (int64_t c0 = warp; c0 < nch; c0 += 2 * kMdWarps) {
    // this warp's next two chunks: all eight 16-byte loads in flight together
    uint4 w[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int64_t c = c0 + (int64_t)i * kMdWarps;
#pragma unroll
      for (int m = 0; m < 4; ++m)
        w[i][m] = c < nch ? __ldg(codes + (tile * nch + c) * 256 + (4 * half + m) * 32 + lane)
                          : make_uint4(0x55555555u, 0x55555555u, 0x55555555u, 0x55555555u);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int64_t c = c0 + (int64_t)i * kMdWarps;
      if (c >= nch) break;
      const uint4* fp = frag4 + (c * nb + (col >> 1)) * 64 + lane;
      const uint4 blo = fp[0], bhi = fp[32];
      const uint32_t bj[4][2] = {{blo.x, blo.y}, {blo.z, blo.w}, {bhi.x, bhi.y}, {bhi.z, bhi.w}};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t M = 0x03030303u << (2 * j);
#pragma unroll
        for (int m = 0; m < 4; ++m)
          mma_u8s8(acc[m][j], w[i][m].x & M, w[i][m].y & M, w[i][m].z & M, w[i][m].w & M, bj[j][0],
                   bj[j][1]);
      }
    }
  }
  // exact per-row digit sums (the 4^j factors divided out), through shared memory
#pragma unroll
  for (int m = 0; m < 4; ++m)
#pragma unroll
    for (int e = 0; e < 4; ++e)
      part[((warp * 4 + m) * 4 + e) * 32 + lane] =
          acc[m][0][e] + (acc[m][1][e] >> 2) + (acc[m][2][e] >> 4) + (acc[m][3][e] >> 6);
  __syncthreads();
  if (tid < kMdRows) {
    const int m = tid >> 4, g = tid & 7, h = (tid >> 3) & 1;
    const int cb = 4 * (col & 1);
    long long S = 0;
#pragma unroll
    for (int d = 0; d < 4; ++d) {
      const int cc = cb + d, L = 4 * g + (cc >> 1), e = 2 * h + (cc & 1);
      int v = 0;
#pragma unroll
      for (int w = 0; w < kMdWarps; ++w) v += part[((w * 4 + m) * 4 + e) * 32 + L];
      S += (long long)(v - colsum[col][d]) * (1ll << (8 * d));
    }
    const int64_t R = rb * kMdRows + tid;
    if (R < rows) out[R] = (float)((double)S * tok_scale[col] * (double)scale[R]);
  }
  __syncthreads();  // part is reused by the next unit
}

__global__ void __launch_bounds__(kMdThreads, 1) moe_decode_kernel(const __grid_constant__ MdParams P) {
  extern __shared__ __align__(16) uint4 md_dyn[];
  __shared__ int colsum[kMdMaxPairs][4];
  __shared__ double tok_scale[kMdMaxPairs];
  __shared__ float red[kMdWarps];
  __shared__ float sc[kMdMaxTok][64];
  __shared__ int sel[kMdMaxTok * 8];
  __shared__ float wts[kMdMaxTok * 8];
  int* part = reinterpret_cast<int*>(md_dyn);  // [8 warps][4][4][32]
  uint32_t* frag = reinterpret_cast<uint32_t*>(part + kMdWarps * 4 * 4 * 32);
  const uint4* frag4 = reinterpret_cast<const uint4*>(frag);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int T = P.T, K = P.K, E = P.E, NP = T * K;
  const int64_t H = P.H, F = P.F, F2 = P.F2;
  unsigned target = 0;
  tc::pdl_wait();

  // ---- R: router partial scores, one warp per (expert, 256-wide K part)
  {
    const int np = P.nparts;
    const int gw = blockIdx.x * kMdWarps + warp, nw = gridDim.x * kMdWarps;
    for (int i = gw; i < E * np; i += nw) {
      const int e = i / np, part = i % np;
      const int64_t k0 = (int64_t)part * 256 + lane * 8;
      const bool full = P.x_vec && k0 + 8 <= H;
      const float* rr = P.router + (int64_t)e * H + k0;
      float r[8];
      if (full) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(rr));
        const float4 b = __ldg(reinterpret_cast<const float4*>(rr) + 1);
        r[0] = a.x; r[1] = a.y; r[2] = a.z; r[3] = a.w;
        r[4] = b.x; r[5] = b.y; r[6] = b.z; r[7] = b.w;
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) r[j] = k0 + j < H ? rr[j] : 0.0f;
      }
      for (int t = 0; t < T; ++t) {
        float xv[8];
        if (full && P.x_bf16) {
          const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(P.x) + t * H + k0);
          const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            xv[2 * j] = __uint_as_float(w4[j] << 16);
            xv[2 * j + 1] = __uint_as_float(w4[j] & 0xffff0000u);
          }
        } else if (full) {
          const float4* xp = reinterpret_cast<const float4*>(static_cast<const float*>(P.x) + t * H + k0);
          const float4 a = xp[0], b = xp[1];
          xv[0] = a.x; xv[1] = a.y; xv[2] = a.z; xv[3] = a.w;
          xv[4] = b.x; xv[5] = b.y; xv[6] = b.z; xv[7] = b.w;
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int64_t k = k0 + j;
            xv[j] = k >= H ? 0.0f
                  : P.x_bf16 ? __uint_as_float((uint32_t) static_cast<const uint16_t*>(P.x)[t * H + k] << 16)
                             : static_cast<const float*>(P.x)[t * H + k];
          }
        }
        float acc = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) acc = __fadd_rn(acc, __fmul_rn(xv[j], r[j]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
        if (lane == 0) P.logits[((int64_t)t * E + e) * np + part] = acc;
      }
    }
  }
  if (!grid_sync(P.bar, target, P.err, 101)) return;

  // ---- S: routing of every token (the reference's sequential softmax / top-k)
  for (int i = tid; i < T * E; i += kMdThreads) {
    const float* lp = P.logits + (int64_t)i * P.nparts;
    float v = 0.0f;
    for (int j = 0; j < P.nparts; ++j) v = __fadd_rn(v, __ldcg(lp + j));
    sc[i / E][i % E] = v;
  }
  if (tid < kMdMaxPairs * 4) colsum[tid >> 2][tid & 3] = 0;
  __syncthreads();
  // warp t routes token t: lanes hold experts lane and lane + 32 (E <= 64);
  // the max, the exponentials and the divisions are elementwise or exact, the
  // sum of the exponentials runs in the reference's order on lane 0, top-k
  // takes the largest probability, the lowest index among equals
  if (warp < T) {
    const int t = warp;
    float* s = sc[t];
    const bool h0 = lane < E, h1 = lane + 32 < E;
    const float v0 = h0 ? s[lane] : -INFINITY, v1 = h1 ? s[lane + 32] : -INFINITY;
    float mx = fmaxf(v0, v1);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float e0 = h0 ? expf(v0 - mx) : 0.0f, e1 = h1 ? expf(v1 - mx) : 0.0f;
    if (h0) s[lane] = e0;
    if (h1) s[lane + 32] = e1;
    __syncwarp();
    float se = 0.0f;
    if (lane == 0)
      for (int e = 0; e < E; ++e) se += s[e];
    se = __shfl_sync(0xffffffffu, se, 0);
    const float p0 = e0 / se, p1 = e1 / se;
    __syncwarp();
    if (h0) s[lane] = p0;
    if (h1) s[lane + 32] = p1;
    __syncwarp();
    uint64_t taken = 0;
    float wsum = 0.0f;
    for (int k = 0; k < K; ++k) {
      // candidates (valid, value, index); a beats b: valid first, then larger, then lower index
      bool bv = h0 && !((taken >> lane) & 1ull);
      float bp = p0;
      int bi = lane;
      if (h1 && !((taken >> (lane + 32)) & 1ull) && (!bv || p1 > bp)) {
        bv = true;
        bp = p1;
        bi = lane + 32;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const bool ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const float op = __shfl_xor_sync(0xffffffffu, bp, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov && (!bv || op > bp || (!(op < bp) && oi < bi))) {
          bv = ov;
          bp = op;
          bi = oi;
        }
      }
      taken |= 1ull << bi;
      if (lane == 0) {
        sel[t * K + k] = bi;
        wsum += s[bi];
      }
    }
    if (lane == 0)
      for (int k = 0; k < K; ++k) {
        const float p = s[sel[t * K + k]];
        wts[t * K + k] = wsum > 0.0f ? p / wsum : p;
      }
    __syncwarp();
    if (blockIdx.x == 0) {
      if (lane < K) {
        P.topk_idx[t * K + lane] = sel[t * K + lane];
        P.topk_w[t * K + lane] = wts[t * K + lane];
      }
      if (P.probs) {
        if (h0) P.probs[t * E + lane] = p0;
        if (h1) P.probs[t * E + lane + 32] = p1;
      }
    }
  }
  __syncthreads();
  // the tokens' operand: token t is column block t
  const int nbx = (T + 1) / 2;
  if (P.x_bf16) {
    const uint16_t* xb = static_cast<const uint16_t*>(P.x);
    build_rows(T, [&](int t, int64_t k) { return xb[t * H + k]; },
               [](uint16_t b) { return __uint_as_float((uint32_t)b << 16); }, H, (int)P.nch_h, nbx,
               frag, colsum, tok_scale, red);
  } else {
    const float* xf = static_cast<const float*>(P.x);
    build_rows(T, [&](int t, int64_t k) { return xf[t * H + k]; }, [](float v) { return v; }, H,
               (int)P.nch_h, nbx, frag, colsum, tok_scale, red);
  }

  // ---- G: gate||up of every (token, expert) pair
  const int64_t rb_gu = (F2 + kMdRows - 1) / kMdRows;
  if ((int64_t)blockIdx.x >= NP * rb_gu && tid == 0) {
    // no G unit here: pull the chosen experts' down weights into L2 for D
    const int64_t idle = gridDim.x - NP * rb_gu, me = blockIdx.x - NP * rb_gu;
    const int64_t bytes = ((H + 127) / 128) * P.nch_f * 4096;  // tiled codes of one down weight
    constexpr int64_t kPiece = 65536;
    const int64_t pieces = (bytes + kPiece - 1) / kPiece;
    for (int64_t j = me; j < NP * pieces; j += idle) {
      const int p = (int)(j / pieces);
      const int64_t off = (j % pieces) * kPiece;
      const int64_t sz = bytes - off < kPiece ? bytes - off : kPiece;
      tc::bulk_prefetch_l2(static_cast<const char*>(P.tab[2 * E + sel[p]]) + off, (uint32_t)sz);
    }
  }
  for (int64_t u = blockIdx.x; u < NP * rb_gu; u += gridDim.x) {
    const int p = (int)(u / rb_gu);
    const int64_t rb = u % rb_gu;
    const int e = sel[p];
    unit_matvec(static_cast<const uint4*>(P.tab[e]), static_cast<const float*>(P.tab[E + e]), F2,
                P.nch_h, rb, p / K, nbx, frag4, colsum, tok_scale, part, P.gu + (int64_t)p * F2);
  }
  if (!grid_sync(P.bar, target, P.err, 102)) return;

  // ---- H: h = act(gate, up) of every pair as column block p
  if (tid < kMdMaxPairs * 4) colsum[tid >> 2][tid & 3] = 0;
  __syncthreads();
  const int nbh = (NP + 1) / 2;
  {
    const float* gu = P.gu;
    // gate row j is interleaved row 32 (j / 16) + j % 16, its up row 16 further
    auto fetch = [&](int p, int64_t j) {
      const float* gp = gu + p * F2 + 32 * (j >> 4) + (j & 15);
      return make_float2(__ldcg(gp), __ldcg(gp + 16));
    };
    if (P.use_gelu) {
      build_rows(NP, fetch, [](float2 v) {
        const float g = v.x;
        const float ta = __fmul_rn(0.7978845608f,
                                   __fadd_rn(g, __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, g), g), g)));
        return __fmul_rn(__fmul_rn(0.5f, g), __fadd_rn(1.0f, tanhf(ta)));
      }, F, (int)P.nch_f, nbh, frag, colsum, tok_scale, red);
    } else {
      build_rows(NP, fetch, [](float2 v) {
        return __fmul_rn(__fdiv_rn(v.x, __fadd_rn(1.0f, expf(-v.x))), v.y);
      }, F, (int)P.nch_f, nbh, frag, colsum, tok_scale, red);
    }
  }
  __syncthreads();

  // ---- D: down projection of every pair
  const int64_t rb_d = (H + kMdRows - 1) / kMdRows;
  for (int64_t u = blockIdx.x; u < NP * rb_d; u += gridDim.x) {
    const int p = (int)(u / rb_d);
    const int64_t rb = u % rb_d;
    const int e = sel[p];
    unit_matvec(static_cast<const uint4*>(P.tab[2 * E + e]),
                static_cast<const float*>(P.tab[3 * E + e]), H, P.nch_f, rb, p, nbh, frag4, colsum,
                tok_scale, part, P.o + (int64_t)p * H);
  }
  if (!grid_sync(P.bar, target, P.err, 103)) return;

  // ---- C: y[t] = (0 + w_0 o_0) + w_1 o_1 ... in top-k order
  for (int64_t i = (int64_t)blockIdx.x * kMdThreads + tid; i < T * H;
       i += (int64_t)gridDim.x * kMdThreads) {
    const int t = (int)(i / H);
    const int64_t j = i % H;
    float acc = 0.0f;
    for (int k = 0; k < K; ++k)
      acc = __fadd_rn(acc, __fmul_rn(wts[t * K + k], __ldcg(P.o + (int64_t)(t * K + k) * H + j)));
    P.y[i] = acc;
  }
}

size_t md_smem(int64_t T, int K, int64_t nch_h, int64_t nch_f) {
  const int64_t nbx = (T + 1) / 2, nbh = (T * K + 1) / 2;
  const int64_t fragb = (nbx * nch_h > nbh * nch_f ? nbx * nch_h : nbh * nch_f) * 1024;
  return (size_t)kMdWarps * 4 * 4 * 32 * 4 + (size_t)fragb;
}

}  // namespace

int moe_decode(ft_ctx* ctx, ft_moe* m, int64_t T, const void* x, int bf16, float* y,
               int32_t* topk_idx, float* topk_w, float* probs, cudaStream_t s) {
  FT_CHECK(T >= 1 && T <= kMdMaxTok && T * m->top_k <= kMdMaxPairs, FT_ERR_UNSUPPORTED,
           "the fused decode takes 1..%d tokens with tokens x top_k <= %d (got %lld x %d)",
           kMdMaxTok, kMdMaxPairs, (long long)T, m->top_k);
  FT_CHECK(m->E <= 64 && m->dtab, FT_ERR_UNSUPPORTED, "layer has no decode tables");
  for (int64_t e = 0; e < m->E; ++e)
    FT_CHECK(m->gate_up[e] && m->down[e], FT_ERR_UNSUPPORTED,
             "the fused decode needs every expert on this device (expert %lld is not)", (long long)e);
  const int64_t nch_h = ceil_div(m->H, kChunkK), nch_f = ceil_div(m->F, kChunkK);
  const size_t smem = md_smem(T, m->top_k, nch_h, nch_f);
  FT_CHECK(smem <= 200 * 1024, FT_ERR_UNSUPPORTED, "layer too wide for the fused decode");
  const int64_t NP = T * m->top_k;
  // scratch: partial router scores | gu | o | barrier
  const int nparts = (int)ceil_div(m->H, 256);
  const size_t off_gu = round_up((int64_t)(T * m->E * nparts * 4), 256);
  const int64_t F2 = m->gate_up[0] ? m->gate_up[0]->rows : 32 * ceil_div(m->F, 16);
  const size_t off_o = off_gu + round_up(NP * F2 * 4, 256);
  const size_t off_bar = off_o + round_up(NP * m->H * 4, 256);
  const size_t need = off_bar + 256;
  if (m->dbuf.bytes < need) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (s != nullptr) cudaStreamIsCapturing(s, &cs);
    FT_CHECK(cs == cudaStreamCaptureStatusNone, FT_ERR_UNSUPPORTED,
             "decode scratch must grow to %zu bytes but the stream is being captured; run one "
             "call before capture", need);
    if (m->dbuf.ptr) {
      FT_CUDA(cudaDeviceSynchronize());
      FT_CUDA(cudaFree(m->dbuf.ptr));
      m->dbuf.ptr = nullptr;
      m->dbuf.bytes = 0;
    }
    FT_CUDA(cudaMalloc(&m->dbuf.ptr, need));
    m->dbuf.bytes = need;
  }
  char* b = static_cast<char*>(m->dbuf.ptr);
  FT_CUDA(cudaMemsetAsync(b + off_bar, 0, 8, s));
  MdParams P;
  memset(&P, 0, sizeof(P));
  P.T = (int)T;
  P.K = m->top_k;
  P.E = (int)m->E;
  P.use_gelu = m->use_gelu;
  P.x_bf16 = bf16;
  P.nparts = nparts;
  P.x_vec = (m->H % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) ? 1 : 0;
  P.H = m->H;
  P.F = m->F;
  P.F2 = F2;
  P.nch_h = nch_h;
  P.nch_f = nch_f;
  P.x = x;
  P.router = m->router;
  P.tab = m->dtab;
  P.logits = reinterpret_cast<float*>(b);
  P.gu = reinterpret_cast<float*>(b + off_gu);
  P.o = reinterpret_cast<float*>(b + off_o);
  P.topk_idx = topk_idx;
  P.topk_w = topk_w;
  P.probs = probs;
  P.y = y;
  P.bar = reinterpret_cast<unsigned*>(b + off_bar);
  P.err = ctx->err_word;
  static bool attr = false;
  if (!attr) {
    FT_CUDA(cudaFuncSetAttribute(moe_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 200 * 1024));
    attr = true;
  }
  // one CTA per SM: every CTA is resident (a cooperative launch guarantees
  // it), which the grid barriers need
  int per_sm = 0;
  FT_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, moe_decode_kernel, kMdThreads, smem));
  FT_CHECK(per_sm >= 1, FT_ERR_UNSUPPORTED, "fused decode does not fit an SM");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctx->num_sms);
  cfg.blockDim = dim3(kMdThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  FT_CUDA(cudaLaunchKernelEx(&cfg, moe_decode_kernel, P));
  FT_LAUNCH_CHECK();
  return FT_OK;
}

}  // namespace ft

extern "C" int ft_moe_decode(ft_ctx* ctx, ft_moe* m, int64_t T, const void* x_dev, int x_is_bf16,
                             float* y_dev, int32_t* topk_idx_dev, float* topk_w_dev,
                             float* probs_dev, void* stream) {
  using namespace ft;
  FT_CHECK(ctx && m && x_dev && y_dev && topk_idx_dev && topk_w_dev, FT_ERR_SHAPE, "null argument");
  FT_CHECK(m->device == ctx->device, FT_ERR_DEVICE, "layer lives on device %d, context on %d",
           m->device, ctx->device);
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
  if (prev != ctx->device) FT_CUDA(cudaSetDevice(ctx->device));
  const int st = moe_decode(ctx, m, T, x_dev, x_is_bf16, y_dev, topk_idx_dev, topk_w_dev, probs_dev,
                            static_cast<cudaStream_t>(stream));
  if (prev >= 0 && prev != ctx->device) cudaSetDevice(prev);
  return st;
}
