// Ternary MoE FFN layer (TernaryMoELayer::forward, src/model/ternary_moe.rs:145-223)
// on the B200 path:
//   router  : scores[t, e] = sum_j R[e, j] x[t, j]  (fp32, sequential in j, no FMA
//             contraction -- the reference loop's rounding), softmax, stable
//             descending top-k, gates renormalised by their sum;
//   dispatch: per-expert counts -> offsets -> expert-major slots (one slot per
//             (token, k)) -> gathered activation rows;
//   experts : one grouped tcgen05 launch for every expert's [gate; up]
//             projection, SwiGLU (or GeLU-tanh) on CUDA cores, one grouped launch
//             for the down projections;
//   combine : y[t] = (0 + w_0 * o_0) + w_1 * o_1 ... in top-k order, the
//             reference's accumulation order.
// The stages are exported separately so an expert-parallel host can put its
// all-to-all exchanges between them.
#include <cmath>
#include <cstring>
#include <vector>

#include "ft_internal.cuh"

#include "ft_moe.cuh"
#include "ft_tc.cuh"

namespace ft {
namespace {

constexpr int kRouterTok = 16;  // tokens per router block
constexpr int kRouterKc = 64;   // K chunk staged in shared memory
constexpr int kMaxExperts = 64;
constexpr int kRouterThreads = 256;
static_assert(kRouterTok * kRouterKc % kRouterThreads == 0 &&
                  kMaxExperts * kRouterKc % kRouterThreads == 0,
              "router chunk loads must split evenly over the block");

__device__ __forceinline__ float load_act(const void* x, int bf16, int64_t i) {
  return bf16 ? __uint_as_float((uint32_t) static_cast<const uint16_t*>(x)[i] << 16)
              : static_cast<const float*>(x)[i];
}

__device__ __forceinline__ void route_token(float* s, int E, int K, int64_t t,
                                            int32_t* __restrict__ topk_idx,
                                            float* __restrict__ topk_w,
                                            float* __restrict__ probs_out,
                                            int32_t* __restrict__ counts);

// One block = 16 tokens x all experts (E <= 64); thread t owns token t/16 and
// experts t%16 + 16m.  Then one thread per token does softmax and top-k in the
// reference's sequential order.
__global__ void __launch_bounds__(kRouterThreads) moe_router_kernel(
    const void* __restrict__ x, int bf16, int64_t T, int64_t H, int E, int K,
    const float* __restrict__ R, int32_t* __restrict__ topk_idx, float* __restrict__ topk_w,
    float* __restrict__ probs_out, int32_t* __restrict__ counts) {
  __shared__ float xs[kRouterTok][kRouterKc];
  __shared__ float rs[kRouterKc][kMaxExperts + 1];
  __shared__ float sc[kRouterTok][kMaxExperts];
  const int tt = threadIdx.x >> 4, el = threadIdx.x & 15;
  const int64_t t0 = (int64_t)blockIdx.x * kRouterTok;
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  // The next K chunk is loaded into registers while the current one is
  // computed (the loads are L2/HBM latency-bound otherwise).
  constexpr int kXL = kRouterTok * kRouterKc / kRouterThreads;   // x values per thread
  constexpr int kRL = kMaxExperts * kRouterKc / kRouterThreads;  // R values per thread
  float px[kXL], pr[kRL];
  auto fetch = [&](int64_t k0) {
#pragma unroll
    for (int j = 0; j < kXL; ++j) {
      const int i = threadIdx.x + j * kRouterThreads;
      const int a = i / kRouterKc, kk = i % kRouterKc;
      const int64_t t = t0 + a, k = k0 + kk;
      px[j] = (t < T && k < H) ? load_act(x, bf16, t * H + k) : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < kRL; ++j) {
      const int i = threadIdx.x + j * kRouterThreads;
      const int e = i / kRouterKc, kk = i % kRouterKc;
      const int64_t k = k0 + kk;
      pr[j] = (e < E && k < H) ? R[(int64_t)e * H + k] : 0.0f;
    }
  };
  fetch(0);
  for (int64_t k0 = 0; k0 < H; k0 += kRouterKc) {
    __syncthreads();  // the previous chunk is no longer read
#pragma unroll
    for (int j = 0; j < kXL; ++j) {
      const int i = threadIdx.x + j * kRouterThreads;
      xs[i / kRouterKc][i % kRouterKc] = px[j];
    }
#pragma unroll
    for (int j = 0; j < kRL; ++j) {
      const int i = threadIdx.x + j * kRouterThreads;
      rs[i % kRouterKc][i / kRouterKc] = pr[j];
    }
    __syncthreads();
    if (k0 + kRouterKc < H) fetch(k0 + kRouterKc);
    const int kn = (int)((H - k0) < kRouterKc ? (H - k0) : kRouterKc);
    for (int kk = 0; kk < kn; ++kk) {
      const float xv = xs[tt][kk];
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int e = el + 16 * m;
        if (e < E) acc[m] = __fadd_rn(acc[m], __fmul_rn(rs[kk][e], xv));
      }
    }
  }
#pragma unroll
  for (int m = 0; m < 4; ++m)
    if (el + 16 * m < E) sc[tt][el + 16 * m] = acc[m];
  __syncthreads();
  const int64_t t = t0 + tt;
  if (el != 0 || t >= T) return;
  route_token(sc[tt], E, K, t, topk_idx, topk_w, probs_out, counts);
}

// Softmax over the E scores of one token, then stable descending top-k with
// gates renormalised by their sum (TernaryMoELayer::forward,
// src/model/ternary_moe.rs:163-215), sequential in the reference's order.
__device__ __forceinline__ void route_token(float* s, int E, int K, int64_t t,
                                            int32_t* __restrict__ topk_idx,
                                            float* __restrict__ topk_w,
                                            float* __restrict__ probs_out,
                                            int32_t* __restrict__ counts) {
  float mx = -INFINITY;
  for (int e = 0; e < E; ++e) mx = fmaxf(mx, s[e]);
  float se = 0.0f;
  for (int e = 0; e < E; ++e) {
    s[e] = expf(s[e] - mx);
    se += s[e];
  }
  for (int e = 0; e < E; ++e) s[e] = s[e] / se;
  if (probs_out)
    for (int e = 0; e < E; ++e) probs_out[t * E + e] = s[e];
  uint64_t taken = 0;
  int idx[8];
  float wsum = 0.0f;
  for (int k = 0; k < K; ++k) {
    int best = -1;
    for (int e = 0; e < E; ++e)
      if (!((taken >> e) & 1ull) && (best < 0 || s[e] > s[best])) best = e;
    taken |= 1ull << best;
    idx[k] = best;
    wsum += s[best];
  }
  for (int k = 0; k < K; ++k) {
    topk_idx[t * K + k] = idx[k];
    topk_w[t * K + k] = wsum > 0.0f ? s[idx[k]] / wsum : s[idx[k]];
    atomicAdd(&counts[idx[k]], 1);
  }
}

// Router scores on the tensor cores.  x (fp32 or bf16) and the router (fp32)
// are sums of bf16 planes -- x = x0 + x1 + x2 exactly for fp32 (each plane the
// bf16 rounding of what the planes before it leave), one plane for bf16 x; the
// router planes are prepared at creation (one when the router is bf16-exact,
// as in BASELINE's bf16 router).  Products of bf16 planes are exact in fp32;
// mma.sync m16n8k16 accumulates them in fp32 over the plane pairs (i, j) with
// i + j <= 2 (the dropped pairs weigh below 2^-24 of the product), each 64-K
// chunk in its own fp32 MMA chain, the chunks summed in f64: the scores come
// out closer to the exact dot than the reference's sequential fp32 sum is.
// Block: 16 tokens x 64 experts, 4 warps (16 experts each); K in chunks of 64
// staged in shared memory (rows padded to 72 bf16: conflict-free fragment
// loads), the next chunk prefetched into registers while the tensor cores work
// on the current one.  Then one thread per token routes it.
constexpr int kRtTok = 16, kRtK = 64, kRtPad = 72, kRtThreads = 128;

__device__ __forceinline__ uint32_t bf16_rn_bits(float v) {
  uint32_t u = __float_as_uint(v);
  if ((u & 0x7f800000u) == 0x7f800000u) return u >> 16;  // inf / NaN: keep
  u += 0x7fffu + ((u >> 16) & 1u);
  return u >> 16;
}

__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(kRtThreads) moe_router_mma_kernel(
    const void* __restrict__ x, int bf16, int64_t T, int64_t H, int64_t Hpad, int E, int K,
    const uint16_t* __restrict__ Rp, int n_rplanes, int32_t* __restrict__ topk_idx,
    float* __restrict__ topk_w, float* __restrict__ probs_out, int32_t* __restrict__ counts) {
  // x planes; after the K loop the same bytes hold the scores
  __shared__ __align__(16) unsigned char xbuf[3 * kRtTok * kRtPad * 2];
  __shared__ __align__(16) uint16_t rs[3][kMaxExperts][kRtPad];
  static_assert(sizeof(float) * kRtTok * (kMaxExperts + 1) <= sizeof(xbuf), "scores alias x");
  auto xs = reinterpret_cast<uint16_t(*)[kRtTok][kRtPad]>(xbuf);
  auto sc = reinterpret_cast<float(*)[kMaxExperts + 1]>(xbuf);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int64_t t0 = (int64_t)blockIdx.x * kRtTok;
  const int nxp = bf16 ? 1 : 3;
  // this thread's share of a chunk: 8 consecutive k of token xa, and 16-byte
  // pieces of the router planes
  const int xa = tid >> 3, xk = 8 * (tid & 7);
  const bool xvec = (H & 7) == 0 &&
                    (reinterpret_cast<uintptr_t>(x) & 15) == 0;  // 16-byte aligned rows
  float xv[8];
  uint4 rv[3][4];
  auto fetch = [&](int64_t k0) {
    const int64_t t = t0 + xa, k = k0 + xk;
    if (t < T && xvec && k + 8 <= H) {
      if (bf16) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + t * H + k));
        const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          xv[2 * i] = __uint_as_float(w4[i] << 16);
          xv[2 * i + 1] = __uint_as_float(w4[i] & 0xffff0000u);
        }
      } else {
        const float4* f = reinterpret_cast<const float4*>(static_cast<const float*>(x) + t * H + k);
        const float4 a = __ldg(f), b = __ldg(f + 1);
        xv[0] = a.x; xv[1] = a.y; xv[2] = a.z; xv[3] = a.w;
        xv[4] = b.x; xv[5] = b.y; xv[6] = b.z; xv[7] = b.w;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) xv[e] = (t < T && k + e < H) ? load_act(x, bf16, t * H + k + e) : 0.0f;
    }
#pragma unroll
    for (int q = 0; q < 3; ++q)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int piece = tid + i * kRtThreads;  // 512 pieces of 8 bf16 per plane
        const int e = piece >> 3, kk = 8 * (piece & 7);
        rv[q][i] = (q < n_rplanes && e < E)
                       ? __ldg(reinterpret_cast<const uint4*>(Rp + ((int64_t)q * kMaxExperts + e) * Hpad + k0 + kk))
                       : make_uint4(0, 0, 0, 0);
      }
  };
  double acc[2][4];
#pragma unroll
  for (int n = 0; n < 2; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0;
  fetch(0);
  for (int64_t k0 = 0; k0 < Hpad; k0 += kRtK) {
    __syncthreads();  // the previous chunk is no longer read
    {
      // x split into planes (exact decomposition), 8 values -> 4 words per plane
      uint32_t pl[3][8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float r = xv[e];
#pragma unroll
        for (int q = 0; q < 3; ++q) {
          pl[q][e] = bf16_rn_bits(r);
          r = __fsub_rn(r, __uint_as_float(pl[q][e] << 16));
        }
      }
#pragma unroll
      for (int q = 0; q < 3; ++q)
        if (q < nxp)
          *reinterpret_cast<uint4*>(&xs[q][xa][xk]) =
              make_uint4(pl[q][0] | (pl[q][1] << 16), pl[q][2] | (pl[q][3] << 16),
                         pl[q][4] | (pl[q][5] << 16), pl[q][6] | (pl[q][7] << 16));
#pragma unroll
      for (int q = 0; q < 3; ++q)
        if (q < n_rplanes)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int piece = tid + i * kRtThreads;
            *reinterpret_cast<uint4*>(&rs[q][piece >> 3][8 * (piece & 7)]) = rv[q][i];
          }
    }
    __syncthreads();
    if (k0 + kRtK < Hpad) fetch(k0 + kRtK);  // in flight while the tensor cores work
    float part[2][4];
#pragma unroll
    for (int n = 0; n < 2; ++n) part[n][0] = part[n][1] = part[n][2] = part[n][3] = 0.0f;
#pragma unroll
    for (int ks = 0; ks < kRtK; ks += 16) {
      for (int i = 0; i < nxp; ++i) {
        const uint16_t* ar = &xs[i][0][0];
        const uint32_t a0 = *reinterpret_cast<const uint32_t*>(ar + g * kRtPad + ks + 2 * tq);
        const uint32_t a1 = *reinterpret_cast<const uint32_t*>(ar + (g + 8) * kRtPad + ks + 2 * tq);
        const uint32_t a2 = *reinterpret_cast<const uint32_t*>(ar + g * kRtPad + ks + 8 + 2 * tq);
        const uint32_t a3 = *reinterpret_cast<const uint32_t*>(ar + (g + 8) * kRtPad + ks + 8 + 2 * tq);
        for (int j = 0; j < n_rplanes && i + j <= 2; ++j) {
#pragma unroll
          for (int n = 0; n < 2; ++n) {
            const uint16_t* br = &rs[j][16 * warp + 8 * n + g][0];
            const uint32_t b0 = *reinterpret_cast<const uint32_t*>(br + ks + 2 * tq);
            const uint32_t b1 = *reinterpret_cast<const uint32_t*>(br + ks + 8 + 2 * tq);
            mma_bf16(part[n], a0, a1, a2, a3, b0, b1);
          }
        }
      }
    }
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[n][i] += (double)part[n][i];
  }
  __syncthreads();  // every warp is done reading x before the scores overwrite it
#pragma unroll
  for (int n = 0; n < 2; ++n) {
    const int e0 = 16 * warp + 8 * n + 2 * tq;
    sc[g][e0] = (float)acc[n][0];
    sc[g][e0 + 1] = (float)acc[n][1];
    sc[g + 8][e0] = (float)acc[n][2];
    sc[g + 8][e0 + 1] = (float)acc[n][3];
  }
  __syncthreads();
  const int64_t t = t0 + tid;
  if (tid < kRtTok && t < T) route_token(sc[tid], E, K, t, topk_idx, topk_w, probs_out, counts);
}

// bf16 activations against a one-plane (bf16-exact) router, the BASELINE's
// case: the chunks of x and of the router reach shared memory by cp.async,
// kRtStages - 1 chunks ahead of the one being multiplied (the plane kernel
// keeps one chunk in flight, and its K loop is load-latency-bound).  Same
// arithmetic: an fp32 MMA chain per 64-K chunk, chunks summed in f64.
constexpr int kRtStages = 4;
constexpr int kRtXsB = kRtTok * kRtPad * 2, kRtRsB = kMaxExperts * kRtPad * 2;
constexpr int kRtStB = kRtXsB + kRtRsB;
static_assert(kRtStages * kRtStB <= 48 * 1024, "router stages fit the default shared memory");

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(tc::smem_u32(dst)), "l"(src)
               : "memory");
}

__global__ void __launch_bounds__(kRtThreads) moe_router_bf16_kernel(
    const uint16_t* __restrict__ x, int64_t T, int64_t H, int64_t Hpad, int E, int K,
    const uint16_t* __restrict__ Rp, int32_t* __restrict__ topk_idx, float* __restrict__ topk_w,
    float* __restrict__ probs_out, int32_t* __restrict__ counts) {
  __shared__ __align__(16) unsigned char st[kRtStages * kRtStB];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int64_t t0 = (int64_t)blockIdx.x * kRtTok;
  const int nch = (int)(Hpad / kRtK);
  auto issue = [&](int c) {
    if (c < nch) {
      unsigned char* sb = st + (c % kRtStages) * kRtStB;
      const int64_t k0 = (int64_t)c * kRtK;
      {  // x: 16 tokens x 64 K = 128 pieces of 16 bytes, one per thread
        const int a = tid >> 3, kk = 8 * (tid & 7);
        const int64_t t = t0 + a, k = k0 + kk;
        uint16_t* dst = reinterpret_cast<uint16_t*>(sb) + a * kRtPad + kk;
        if (t < T && k + 8 <= H) cp_async16(dst, x + t * H + k);
        else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {  // router: 64 experts x 64 K = 512 pieces
        const int piece = tid + i * kRtThreads;
        const int e = piece >> 3, kk = 8 * (piece & 7);
        uint16_t* dst = reinterpret_cast<uint16_t*>(sb + kRtXsB) + e * kRtPad + kk;
        if (e < E) cp_async16(dst, Rp + (int64_t)e * Hpad + k0 + kk);
        else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");  // (possibly empty) group per chunk
  };
  for (int c = 0; c < kRtStages - 1; ++c) issue(c);
  double acc[2][4];
#pragma unroll
  for (int n = 0; n < 2; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0;
  for (int c = 0; c < nch; ++c) {
    asm volatile("cp.async.wait_group %0;" ::"n"(kRtStages - 2) : "memory");
    __syncthreads();  // chunk c is in; every thread is done with chunk c - 1
    issue(c + kRtStages - 1);  // into the stage chunk c - 1 used
    const unsigned char* sb = st + (c % kRtStages) * kRtStB;
    const uint16_t* xs = reinterpret_cast<const uint16_t*>(sb);
    const uint16_t* rs = reinterpret_cast<const uint16_t*>(sb + kRtXsB);
    float part[2][4];
#pragma unroll
    for (int n = 0; n < 2; ++n) part[n][0] = part[n][1] = part[n][2] = part[n][3] = 0.0f;
#pragma unroll
    for (int ks = 0; ks < kRtK; ks += 16) {
      const uint32_t a0 = *reinterpret_cast<const uint32_t*>(xs + g * kRtPad + ks + 2 * tq);
      const uint32_t a1 = *reinterpret_cast<const uint32_t*>(xs + (g + 8) * kRtPad + ks + 2 * tq);
      const uint32_t a2 = *reinterpret_cast<const uint32_t*>(xs + g * kRtPad + ks + 8 + 2 * tq);
      const uint32_t a3 = *reinterpret_cast<const uint32_t*>(xs + (g + 8) * kRtPad + ks + 8 + 2 * tq);
#pragma unroll
      for (int n = 0; n < 2; ++n) {
        const uint16_t* br = rs + (16 * warp + 8 * n + g) * kRtPad;
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(br + ks + 2 * tq);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(br + ks + 8 + 2 * tq);
        mma_bf16(part[n], a0, a1, a2, a3, b0, b1);
      }
    }
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[n][i] += (double)part[n][i];
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();  // every warp is done reading the stages before the scores overwrite them
  auto sc = reinterpret_cast<float(*)[kMaxExperts + 1]>(st);
#pragma unroll
  for (int n = 0; n < 2; ++n) {
    const int e0 = 16 * warp + 8 * n + 2 * tq;
    sc[g][e0] = (float)acc[n][0];
    sc[g][e0 + 1] = (float)acc[n][1];
    sc[g + 8][e0] = (float)acc[n][2];
    sc[g + 8][e0 + 1] = (float)acc[n][3];
  }
  __syncthreads();
  const int64_t t = t0 + tid;
  if (tid < kRtTok && t < T) route_token(sc[tid], E, K, t, topk_idx, topk_w, probs_out, counts);
}

__global__ void moe_offsets_kernel(const int32_t* __restrict__ counts, int E,
                                   int32_t* __restrict__ offsets, int32_t* __restrict__ fill) {
  if (threadIdx.x == 0) {
    int32_t o = 0;
    for (int e = 0; e < E; ++e) {
      offsets[e] = o;
      o += counts[e];
      fill[e] = 0;
    }
    offsets[E] = o;
  }
}

// slot_of[t*K+k] = expert-major slot of (t, k); token_of[slot] = t.
__global__ void moe_scatter_kernel(const int32_t* __restrict__ topk_idx, int64_t n_entries, int K,
                                   const int32_t* __restrict__ offsets, int32_t* __restrict__ fill,
                                   int32_t* __restrict__ slot_of, int32_t* __restrict__ token_of) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_entries) return;
  const int e = topk_idx[i];
  const int32_t slot = offsets[e] + atomicAdd(&fill[e], 1);
  slot_of[i] = slot;
  token_of[slot] = (int32_t)(i / K);
}

// xg[slot, :] = x[token_of[slot], :] (element type preserved)
__global__ void moe_gather_kernel(const void* __restrict__ x, int elem_bytes, int64_t H,
                                  const int32_t* __restrict__ token_of, int64_t n_slots,
                                  void* __restrict__ xg) {
  const int64_t row = blockIdx.x;
  if (row >= n_slots) return;
  const int64_t src = token_of[row];
  const int64_t nb = H * elem_bytes;
  const char* s = static_cast<const char*>(x) + src * nb;
  char* d = static_cast<char*>(xg) + row * nb;
  if ((nb & 15) == 0) {
    for (int64_t i = threadIdx.x * 16; i < nb; i += blockDim.x * 16)
      *reinterpret_cast<uint4*>(d + i) = *reinterpret_cast<const uint4*>(s + i);
  } else {
    for (int64_t i = threadIdx.x; i < nb; i += blockDim.x) d[i] = s[i];
  }
}

// The gate/up weight of an expert as one matrix with interleaved 16-row
// m-blocks: m-block 2b = gate rows 16b .. 16b+15, m-block 2b+1 = up rows
// 16b .. 16b+15 (2 * ceil(F/16) m-blocks; missing rows are weight 0, scale 0),
// so the engine's epilogue finds a gate row and its up row 16 lanes apart.
// One thread per uint4 of the stacked blocks (32 per m-block per chunk).
__global__ void interleave_gu_kernel(const uint4* __restrict__ gate, const uint4* __restrict__ up,
                                     const float* __restrict__ gs, const float* __restrict__ us,
                                     int64_t src_tiles, int64_t n_chunks, int64_t total,
                                     uint4* __restrict__ dst, float* __restrict__ dscale) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int lane = (int)(i & 31), M = (int)((i >> 5) & 7);
  const int64_t blk = i >> 8, T = blk / n_chunks, c = blk % n_chunks;
  const int64_t b = 4 * T + (M >> 1);  // source m-block
  const int64_t st = b >> 3;
  const uint4* src = (M & 1) ? up : gate;
  uint4 v = make_uint4(0x55555555u, 0x55555555u, 0x55555555u, 0x55555555u);  // code 1: w = 0
  if (st < src_tiles) v = src[((st * n_chunks + c) * 8 + (b & 7)) * 32 + lane];
  dst[i] = v;
  if (c == 0 && lane < 16) {
    const float* ss = (M & 1) ? us : gs;
    dscale[T * kTileRows + 16 * M + lane] = st < src_tiles ? ss[16 * b + lane] : 0.0f;
  }
}

// y[t, j] = sum_k w[t, k] * o[slot_of[t, k], j], accumulated from 0 in k order
// (grid: x over H in float4 pieces, y and z over tokens; K <= 8)
__global__ void moe_combine_kernel(const float* __restrict__ o, const int32_t* __restrict__ slot_of,
                                   const float* __restrict__ topk_w, int64_t T, int K, int64_t H,
                                   float* __restrict__ y) {
  const int64_t t = blockIdx.y + (int64_t)blockIdx.z * gridDim.y;
  if (t >= T) return;
  int64_t row[8];
  float w[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    row[k] = k < K ? (int64_t)slot_of[t * K + k] * H : 0;
    w[k] = k < K ? topk_w[t * K + k] : 0.0f;
  }
  const int64_t j0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if ((H & 3) == 0) {
    const int64_t j = 4 * j0;
    if (j >= H) return;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (k >= K) break;
      const float4 v = *reinterpret_cast<const float4*>(o + row[k] + j);
      acc.x = __fadd_rn(acc.x, __fmul_rn(w[k], v.x));
      acc.y = __fadd_rn(acc.y, __fmul_rn(w[k], v.y));
      acc.z = __fadd_rn(acc.z, __fmul_rn(w[k], v.z));
      acc.w = __fadd_rn(acc.w, __fmul_rn(w[k], v.w));
    }
    *reinterpret_cast<float4*>(y + t * H + j) = acc;
  } else {
    for (int64_t j = j0; j < H; j += (int64_t)gridDim.x * blockDim.x) {
      float acc = 0.0f;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (k >= K) break;
        acc = __fadd_rn(acc, __fmul_rn(w[k], o[row[k] + j]));
      }
      y[t * H + j] = acc;
    }
  }
}

// launch geometry of moe_combine_kernel
dim3 combine_grid(int64_t T, int64_t H) {
  const int64_t xs = (H & 3) == 0 ? ceil_div(H / 4, 256) : ceil_div(H, 256);
  const int64_t ys = T < 65535 ? T : 65535;
  return dim3((unsigned)(xs < 1 ? 1 : xs), (unsigned)(ys < 1 ? 1 : ys), (unsigned)ceil_div(T, ys < 1 ? 1 : ys));
}

int moe_reserve(ft_moe* m, size_t bytes, cudaStream_t s) {
  if (m->buf.bytes >= bytes) return FT_OK;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (s != nullptr) cudaStreamIsCapturing(s, &cs);
  FT_CHECK(cs == cudaStreamCaptureStatusNone, FT_ERR_UNSUPPORTED,
           "MoE buffers must grow but the stream is being captured");
  if (m->buf.ptr) {
    FT_CUDA(cudaDeviceSynchronize());
    FT_CUDA(cudaFree(m->buf.ptr));
    m->buf.ptr = nullptr;
    m->buf.bytes = 0;
  }
  const size_t grow = bytes + bytes / 8 + (1 << 20);
  FT_CUDA(cudaMalloc(&m->buf.ptr, grow));
  m->buf.bytes = grow;
  return FT_OK;
}

struct MoeBufs {
  int32_t* topk_idx;
  float* topk_w;
  int32_t* counts;
  int32_t* offsets;
  int32_t* fill;
  int32_t* slot_of;
  int32_t* token_of;
  void* xg;
  float* gu;  // gate/up outputs [n, interleaved rows]
  float* o;
};

// gate/up rows of the interleaved weight: 32 per 16 rows of F
int64_t gu_rows(int64_t F) { return 32 * ceil_div(F, 16); }

// Stacks separately uploaded gate and up weights ([F, H] each) into the
// interleaved gate/up weight; the two inputs are destroyed.
int stack_gate_up(ft_ctx* ctx, ft_weight* gate, ft_weight* up, cudaStream_t s, ft_weight** out) {
  *out = nullptr;
  ft_weight* w = nullptr;
  int st = alloc_weight(ctx, gu_rows(gate->rows), gate->cols, &w);
  if (st == FT_OK) {
    const int64_t total = w->n_tiles * w->n_chunks * 256;
    interleave_gu_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, s>>>(
        reinterpret_cast<const uint4*>(gate->codes), reinterpret_cast<const uint4*>(up->codes),
        gate->row_scales, up->row_scales, gate->n_tiles, w->n_chunks, total,
        reinterpret_cast<uint4*>(w->codes), w->row_scales);
    const cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) g_launches.fetch_add(1, std::memory_order_relaxed);
    const cudaError_t e2 = e == cudaSuccess ? cudaStreamSynchronize(s) : e;
    if (e2 != cudaSuccess) st = fail(FT_ERR_GPU, "gate/up stacking failed: %s", cudaGetErrorString(e2));
  }
  ft_weight_destroy(gate);
  ft_weight_destroy(up);
  if (st != FT_OK) {
    ft_weight_destroy(w);
    return st;
  }
  *out = w;
  return FT_OK;
}

// Layout of the forward intermediates for T tokens.
size_t moe_layout(const ft_moe* m, int64_t T, int x_bytes, char* base, MoeBufs* b) {
  const int64_t n = T * m->top_k;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    char* p = base ? base + off : nullptr;
    off = round_up((int64_t)(off + bytes), 256);
    return p;
  };
  b->topk_idx = reinterpret_cast<int32_t*>(take(n * 4));
  b->topk_w = reinterpret_cast<float*>(take(n * 4));
  b->counts = reinterpret_cast<int32_t*>(take((m->E + 1) * 4));
  b->offsets = reinterpret_cast<int32_t*>(take((m->E + 1) * 4));
  b->fill = reinterpret_cast<int32_t*>(take((m->E + 1) * 4));
  b->slot_of = reinterpret_cast<int32_t*>(take(n * 4));
  b->token_of = reinterpret_cast<int32_t*>(take(n * 4));
  b->xg = take((size_t)n * m->H * x_bytes);
  b->gu = reinterpret_cast<float*>(take((size_t)n * gu_rows(m->F) * 4));
  b->o = reinterpret_cast<float*>(take((size_t)n * m->H * 4));
  return off;
}

}  // namespace

int moe_route(ft_ctx* ctx, ft_moe* m, int64_t T, const void* x, int bf16, int32_t* topk_idx,
              float* topk_w, float* probs, int32_t* counts, cudaStream_t s) {
  FT_CUDA(cudaMemsetAsync(counts, 0, m->E * sizeof(int32_t), s));
  if (T == 0) return FT_OK;
  if (m->router_planes && bf16 && m->n_rplanes == 1 && m->H % 8 == 0 &&
      (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    moe_router_bf16_kernel<<<(unsigned)ceil_div(T, kRtTok), kRtThreads, 0, s>>>(
        static_cast<const uint16_t*>(x), T, m->H, m->Hpad, (int)m->E, m->top_k, m->router_planes,
        topk_idx, topk_w, probs, counts);
  } else if (m->router_planes) {
    moe_router_mma_kernel<<<(unsigned)ceil_div(T, kRtTok), kRtThreads, 0, s>>>(
        x, bf16, T, m->H, m->Hpad, (int)m->E, m->top_k, m->router_planes, m->n_rplanes, topk_idx,
        topk_w, probs, counts);
  } else {
    moe_router_kernel<<<(unsigned)ceil_div(T, kRouterTok), kRouterThreads, 0, s>>>(
        x, bf16, T, m->H, (int)m->E, m->top_k, m->router, topk_idx, topk_w, probs, counts);
  }
  FT_LAUNCH_CHECK();
  return FT_OK;
}

// Expert FFN over rows grouped in segments: segment i has seg_rows[i] rows for
// expert seg_expert[i], stored consecutively in x_rows / y_rows.
int moe_expert_segments(ft_ctx* ctx, ft_moe* m, int nseg, const int32_t* seg_expert,
                        const int64_t* seg_rows, const void* x_rows, int bf16, float* gu,
                        float* y_rows, cudaStream_t s) {
  FT_CHECK(nseg >= 0 && nseg <= 64, FT_ERR_UNSUPPORTED, "at most 64 segments per call");
  int64_t total = 0;
  std::vector<const ft_weight*> wgu(nseg), wd(nseg);
  std::vector<const void*> xs(nseg), gin(nseg);
  std::vector<float*> gout(nseg), ys(nseg);
  const int64_t F2 = gu_rows(m->F);
  const int xb = bf16 ? 2 : 4;
  for (int i = 0; i < nseg; ++i) {
    FT_CHECK(seg_expert[i] >= 0 && seg_expert[i] < m->E, FT_ERR_SHAPE, "segment %d: bad expert %d",
             i, seg_expert[i]);
    FT_CHECK(seg_rows[i] >= 0, FT_ERR_SHAPE, "segment %d: negative rows", i);
    FT_CHECK(m->gate_up[seg_expert[i]] && m->down[seg_expert[i]], FT_ERR_SHAPE,
             "segment %d: expert %d is not held by this layer", i, seg_expert[i]);
    wgu[i] = m->gate_up[seg_expert[i]];
    wd[i] = m->down[seg_expert[i]];
    xs[i] = static_cast<const char*>(x_rows) + total * m->H * xb;
    gout[i] = gu + total * F2;
    gin[i] = gout[i];
    ys[i] = y_rows + total * m->H;
    total += seg_rows[i];
  }
  if (total == 0) return FT_OK;
  // Expert GEMMs take kDigitsMoE fixed-point digits per token: the layer's
  // tolerance is 1e-4 of each output row's rms (ft_internal.cuh).  The down
  // GEMM builds its operand from the interleaved gate/up outputs, applying the
  // activation (SwiGLU, or GeLU) as it reads them: no pass of its own.
  int st = launch_tc_grouped(ctx, nseg, wgu.data(), 0, xs.data(), bf16 ? 1 : 0, nullptr,
                             gout.data(), nullptr, s, seg_rows, kDigitsMoE);
  if (st != FT_OK) return st;
  return launch_tc_grouped(ctx, nseg, wd.data(), 0, gin.data(), 0, nullptr, ys.data(), nullptr, s,
                           seg_rows, kDigitsMoE, nullptr, 1, m->use_gelu ? 2 : 1, F2);
}

// Router planes for moe_router_mma_kernel: router = p0 + p1 + p2 with each
// plane the bf16 rounding (to nearest even) of what the planes before it
// leave, which is exact for finite fp32 values; as few planes as the router
// needs (one for a bf16-exact router).  A router with non-finite values keeps
// the sequential kernel.
static uint16_t host_bf16_rn(float v, float* rest) {
  uint32_t u;
  memcpy(&u, &v, 4);
  u += 0x7fffu + ((u >> 16) & 1u);
  const uint16_t h = (uint16_t)(u >> 16);
  const uint32_t hb = (uint32_t)h << 16;
  float hv;
  memcpy(&hv, &hb, 4);
  *rest = v - hv;
  return h;
}

// Device tables of the experts' codes and row scales for the fused decode
// kernel: [gate_up codes][gate_up scales][down codes][down scales], E each.
int build_decode_tables(ft_moe* m) {
  std::vector<const void*> tab(4 * m->E, nullptr);
  for (int64_t e = 0; e < m->E; ++e) {
    if (m->gate_up[e]) {
      tab[e] = m->gate_up[e]->codes;
      tab[m->E + e] = m->gate_up[e]->row_scales;
    }
    if (m->down[e]) {
      tab[2 * m->E + e] = m->down[e]->codes;
      tab[3 * m->E + e] = m->down[e]->row_scales;
    }
  }
  FT_CUDA(cudaMalloc(&m->dtab, tab.size() * sizeof(void*)));
  FT_CUDA(cudaMemcpy(m->dtab, tab.data(), tab.size() * sizeof(void*), cudaMemcpyHostToDevice));
  return FT_OK;
}

int prepare_router_planes(ft_moe* m, const float* router_host) {
  const int64_t E = m->E, H = m->H;
  const int64_t Hpad = ceil_div(H, kRtK) * kRtK;
  std::vector<uint16_t> planes((size_t)3 * kMaxExperts * Hpad, 0);
  int need = 1;
  for (int64_t e = 0; e < E; ++e)
    for (int64_t k = 0; k < H; ++k) {
      float r = router_host[e * H + k];
      if (!std::isfinite(r)) return FT_OK;  // sequential router
      for (int q = 0; q < 3; ++q) {
        const uint16_t h = host_bf16_rn(r, &r);
        planes[((size_t)q * kMaxExperts + e) * Hpad + k] = h;
        if (h != 0 && q + 1 > need) need = q + 1;
      }
    }
  const size_t bytes = (size_t)need * kMaxExperts * Hpad * 2;
  FT_CUDA(cudaMalloc(&m->router_planes, bytes));
  FT_CUDA(cudaMemcpy(m->router_planes, planes.data(), bytes, cudaMemcpyHostToDevice));
  m->n_rplanes = need;
  m->Hpad = Hpad;
  return FT_OK;
}

}  // namespace ft

using namespace ft;

extern "C" {

int ft_moe_create(ft_ctx* ctx, int64_t n_experts, int64_t hidden, int64_t inter, int top_k,
                  int use_gelu, const float* router_host, const uint8_t* const* gate_packed,
                  const float* const* gate_scales, const uint8_t* const* up_packed,
                  const float* const* up_scales, const uint8_t* const* down_packed,
                  const float* const* down_scales, ft_moe** out) {
  FT_CHECK(ctx && out && router_host && gate_packed && gate_scales && up_packed && up_scales &&
               down_packed && down_scales,
           FT_ERR_SHAPE, "null argument");
  FT_CHECK(n_experts >= 1 && n_experts <= kMaxExperts, FT_ERR_UNSUPPORTED,
           "n_experts must be in [1, %d]", kMaxExperts);
  FT_CHECK(top_k >= 1 && top_k <= 8 && top_k <= n_experts, FT_ERR_UNSUPPORTED,
           "top_k must be in [1, min(8, n_experts)]");
  FT_CHECK(hidden > 0 && inter > 0 && (inter * hidden) % 4 == 0, FT_ERR_SHAPE,
           "hidden*inter must be a positive multiple of 4");
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != ctx->device) cudaSetDevice(ctx->device);
  ft_moe* m = new ft_moe();
  m->device = ctx->device;
  m->E = n_experts;
  m->H = hidden;
  m->F = inter;
  m->top_k = top_k;
  m->use_gelu = use_gelu;
  m->counts_host.assign(n_experts + 1, 0);
  int st = FT_OK;
  cudaError_t e = cudaMalloc(&m->router, (size_t)n_experts * hidden * 4);
  if (e == cudaSuccess)
    e = cudaMemcpy(m->router, router_host, (size_t)n_experts * hidden * 4, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) st = fail(FT_ERR_GPU, "router upload failed: %s", cudaGetErrorString(e));
  if (st == FT_OK) st = prepare_router_planes(m, router_host);
  for (int64_t x = 0; x < n_experts && st == FT_OK; ++x) {
    if (!gate_packed[x]) {  // expert held by another rank (expert parallelism)
      m->gate_up.push_back(nullptr);
      m->down.push_back(nullptr);
      continue;
    }
    FT_CHECK(up_packed[x] && down_packed[x] && gate_scales[x] && up_scales[x] && down_scales[x],
             FT_ERR_SHAPE, "expert %lld: gate given but up/down/scales missing", (long long)x);
    // gate and up uploaded separately, then interleaved by 16-row m-blocks
    ft_weight *wg = nullptr, *wu = nullptr, *w = nullptr;
    st = ft_weight_upload_packed_u8(ctx, gate_packed[x], inter, hidden, gate_scales[x], &wg);
    if (st == FT_OK) st = ft_weight_upload_packed_u8(ctx, up_packed[x], inter, hidden, up_scales[x], &wu);
    if (st == FT_OK) {
      st = stack_gate_up(ctx, wg, wu, ctx->host_stream, &w);
    } else {
      ft_weight_destroy(wg);
      ft_weight_destroy(wu);
    }
    if (st != FT_OK) break;
    m->gate_up.push_back(w);
    st = ft_weight_upload_packed_u8(ctx, down_packed[x], hidden, inter, down_scales[x], &w);
    if (st != FT_OK) break;
    m->down.push_back(w);
  }
  if (st == FT_OK) st = build_decode_tables(m);
  if (prev >= 0 && prev != ctx->device) cudaSetDevice(prev);
  if (st != FT_OK) {
    for (auto* w : m->gate_up) ft_weight_destroy(w);
    for (auto* w : m->down) ft_weight_destroy(w);
    if (m->router) cudaFree(m->router);
    if (m->router_planes) cudaFree(m->router_planes);
    if (m->dtab) cudaFree(m->dtab);
    delete m;
    return st;
  }
  *out = m;
  return FT_OK;
}

int ft_moe_create_f32(ft_ctx* ctx, int64_t n_experts, int64_t hidden, int64_t inter, int top_k,
                      int use_gelu, const float* router_host, const float* const* gate_f32,
                      const float* const* up_f32, const float* const* down_f32, ft_moe** out) {
  FT_CHECK(ctx && out && router_host && gate_f32 && up_f32 && down_f32, FT_ERR_SHAPE,
           "null argument");
  FT_CHECK(n_experts >= 1 && n_experts <= kMaxExperts, FT_ERR_UNSUPPORTED,
           "n_experts must be in [1, %d]", kMaxExperts);
  FT_CHECK(top_k >= 1 && top_k <= 8 && top_k <= n_experts, FT_ERR_UNSUPPORTED,
           "top_k must be in [1, min(8, n_experts)]");
  FT_CHECK(hidden > 0 && inter > 0, FT_ERR_SHAPE, "hidden and inter must be positive");
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != ctx->device) cudaSetDevice(ctx->device);
  ft_moe* m = new ft_moe();
  m->device = ctx->device;
  m->E = n_experts;
  m->H = hidden;
  m->F = inter;
  m->top_k = top_k;
  m->use_gelu = use_gelu;
  m->counts_host.assign(n_experts + 1, 0);
  int st = FT_OK;
  cudaStream_t s = ctx->host_stream;
  float* staging = nullptr;
  cudaError_t e = cudaMalloc(&m->router, (size_t)n_experts * hidden * 4);
  if (e == cudaSuccess)
    e = cudaMemcpy(m->router, router_host, (size_t)n_experts * hidden * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMalloc(&staging, (size_t)(inter * hidden) * 4);
  if (e != cudaSuccess) st = fail(FT_ERR_GPU, "MoE upload failed: %s", cudaGetErrorString(e));
  if (st == FT_OK) st = prepare_router_planes(m, router_host);
  const size_t mat = (size_t)(inter * hidden);
  for (int64_t x = 0; x < n_experts && st == FT_OK; ++x) {
    if (!gate_f32[x]) {  // expert held by another rank (expert parallelism)
      m->gate_up.push_back(nullptr);
      m->down.push_back(nullptr);
      continue;
    }
    if (!up_f32[x] || !down_f32[x]) {
      st = fail(FT_ERR_SHAPE, "expert %lld: gate given but up/down missing", (long long)x);
      break;
    }
    // TernaryExpert::from_fp32 (src/model/cpu_moe.rs:33-37) per matrix: the
    // absmean scale of quantize_ternary, then the rounding rule, here on the
    // device straight into the tiled layout; gate and up are then interleaved.
    const float ad = host_absmean_alpha(down_f32[x], (int64_t)mat);
    ft_weight* part[2] = {nullptr, nullptr};
    ft_weight* w = nullptr;
    for (int i = 0; i < 2 && st == FT_OK; ++i) {
      const float* src = i == 0 ? gate_f32[x] : up_f32[x];
      st = alloc_weight(ctx, inter, hidden, &part[i]);
      if (st != FT_OK) break;
      e = cudaMemcpyAsync(staging, src, mat * 4, cudaMemcpyHostToDevice, s);
      if (e == cudaSuccess) st = launch_fill_scales(part[i], host_absmean_alpha(src, (int64_t)mat), s);
      if (e == cudaSuccess && st == FT_OK) st = launch_quantize_pack(staging, false, 0, part[i], s);
      if (e == cudaSuccess) e = cudaStreamSynchronize(s);
      if (e != cudaSuccess && st == FT_OK)
        st = fail(FT_ERR_GPU, "expert upload failed: %s", cudaGetErrorString(e));
    }
    if (st == FT_OK) {
      st = stack_gate_up(ctx, part[0], part[1], s, &w);
    } else {
      ft_weight_destroy(part[0]);
      ft_weight_destroy(part[1]);
    }
    if (st != FT_OK) {
      m->gate_up.push_back(nullptr);
      m->down.push_back(nullptr);
      break;
    }
    m->gate_up.push_back(w);
    st = alloc_weight(ctx, hidden, inter, &w);
    if (st != FT_OK) {
      m->down.push_back(nullptr);
      break;
    }
    m->down.push_back(w);
    e = cudaMemcpyAsync(staging, down_f32[x], mat * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) st = launch_fill_scales(w, ad, s);
    if (e == cudaSuccess && st == FT_OK) st = launch_quantize_pack(staging, false, 0, w, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess && st == FT_OK)
      st = fail(FT_ERR_GPU, "expert upload failed: %s", cudaGetErrorString(e));
  }
  if (staging) cudaFree(staging);
  if (st == FT_OK) st = build_decode_tables(m);
  if (prev >= 0 && prev != ctx->device) cudaSetDevice(prev);
  if (st != FT_OK) {
    for (auto* w : m->gate_up) ft_weight_destroy(w);
    for (auto* w : m->down) ft_weight_destroy(w);
    if (m->router) cudaFree(m->router);
    if (m->router_planes) cudaFree(m->router_planes);
    if (m->dtab) cudaFree(m->dtab);
    delete m;
    return st;
  }
  *out = m;
  return FT_OK;
}

int ft_moe_destroy(ft_moe* m) {
  if (!m) return FT_OK;
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != m->device) cudaSetDevice(m->device);
  cudaDeviceSynchronize();
  for (auto* w : m->gate_up) ft_weight_destroy(w);
  for (auto* w : m->down) ft_weight_destroy(w);
  if (m->router) cudaFree(m->router);
  if (m->router_planes) cudaFree(m->router_planes);
  if (m->dtab) cudaFree(m->dtab);
  if (m->dbuf.ptr) cudaFree(m->dbuf.ptr);
  if (m->buf.ptr) cudaFree(m->buf.ptr);
  if (prev >= 0 && prev != m->device) cudaSetDevice(prev);
  delete m;
  return FT_OK;
}

int ft_moe_route(ft_ctx* ctx, ft_moe* m, int64_t T, const void* x_dev, int x_is_bf16,
                 int32_t* topk_idx_dev, float* topk_w_dev, float* probs_dev, int32_t* counts_dev,
                 void* stream) {
  FT_CHECK(ctx && m && counts_dev && (T == 0 || (x_dev && topk_idx_dev && topk_w_dev)),
           FT_ERR_SHAPE, "null argument");
  return moe_route(ctx, m, T, x_dev, x_is_bf16, topk_idx_dev, topk_w_dev, probs_dev, counts_dev,
                   static_cast<cudaStream_t>(stream));
}

int ft_moe_dispatch_layout(ft_ctx* ctx, ft_moe* m, int64_t T, const int32_t* topk_idx_dev,
                           const int32_t* counts_dev, int32_t* offsets_dev, int32_t* fill_dev,
                           int32_t* slot_of_dev, int32_t* token_of_dev, void* stream) {
  FT_CHECK(ctx && m && counts_dev && offsets_dev && fill_dev, FT_ERR_SHAPE, "null argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  moe_offsets_kernel<<<1, 32, 0, s>>>(counts_dev, (int)m->E, offsets_dev, fill_dev);
  FT_LAUNCH_CHECK();
  const int64_t n = T * m->top_k;
  if (n == 0) return FT_OK;
  moe_scatter_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(topk_idx_dev, n, m->top_k,
                                                                offsets_dev, fill_dev, slot_of_dev,
                                                                token_of_dev);
  FT_LAUNCH_CHECK();
  return FT_OK;
}

int ft_moe_gather_rows(ft_ctx* ctx, const void* x_dev, int elem_bytes, int64_t H,
                       const int32_t* token_of_dev, int64_t n_rows, void* out_dev, void* stream) {
  FT_CHECK(ctx && (n_rows == 0 || (x_dev && token_of_dev && out_dev)), FT_ERR_SHAPE,
           "null argument");
  FT_CHECK(elem_bytes == 2 || elem_bytes == 4, FT_ERR_SHAPE, "elem_bytes must be 2 or 4");
  if (n_rows == 0) return FT_OK;
  moe_gather_kernel<<<(unsigned)n_rows, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      x_dev, elem_bytes, H, token_of_dev, n_rows, out_dev);
  FT_LAUNCH_CHECK();
  return FT_OK;
}

int ft_moe_expert_ffn(ft_ctx* ctx, ft_moe* m, int nseg, const int32_t* seg_expert_host,
                      const int64_t* seg_rows_host, const void* x_rows_dev, int x_is_bf16,
                      float* y_rows_dev, void* stream) {
  FT_CHECK(ctx && m && (nseg == 0 || (seg_expert_host && seg_rows_host && x_rows_dev && y_rows_dev)),
           FT_ERR_SHAPE, "null argument");
  int64_t total = 0;
  for (int i = 0; i < nseg; ++i) total += seg_rows_host[i] > 0 ? seg_rows_host[i] : 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // gate/up scratch: the interleaved rows of F per token
  int st = moe_reserve(m, (size_t)total * gu_rows(m->F) * 4 + 512, s);
  if (st != FT_OK) return st;
  float* gu = static_cast<float*>(m->buf.ptr);
  return moe_expert_segments(ctx, m, nseg, seg_expert_host, seg_rows_host, x_rows_dev, x_is_bf16,
                             gu, y_rows_dev, s);
}

int ft_moe_combine(ft_ctx* ctx, ft_moe* m, int64_t T, const float* o_rows_dev,
                   const int32_t* slot_of_dev, const float* topk_w_dev, float* y_dev, void* stream) {
  FT_CHECK(ctx && m && (T == 0 || (o_rows_dev && slot_of_dev && topk_w_dev && y_dev)),
           FT_ERR_SHAPE, "null argument");
  if (T == 0) return FT_OK;
  moe_combine_kernel<<<combine_grid(T, m->H), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      o_rows_dev, slot_of_dev, topk_w_dev, T, m->top_k, m->H, y_dev);
  FT_LAUNCH_CHECK();
  return FT_OK;
}

int ft_moe_forward(ft_ctx* ctx, ft_moe* m, int64_t T, const void* x_dev, int x_is_bf16,
                   float* y_dev, float* probs_dev, void* stream) {
  FT_CHECK(ctx && m && (T == 0 || (x_dev && y_dev)), FT_ERR_SHAPE, "null argument");
  if (T == 0) return FT_OK;
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != ctx->device) FT_CUDA(cudaSetDevice(ctx->device));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int xb = x_is_bf16 ? 2 : 4;
  MoeBufs b;
  const size_t need = moe_layout(m, T, xb, nullptr, &b);
  int st = moe_reserve(m, need, s);
  if (st == FT_OK) {
    moe_layout(m, T, xb, static_cast<char*>(m->buf.ptr), &b);
    st = moe_route(ctx, m, T, x_dev, x_is_bf16, b.topk_idx, b.topk_w, probs_dev, b.counts, s);
  }
  if (st == FT_OK)
    st = ft_moe_dispatch_layout(ctx, m, T, b.topk_idx, b.counts, b.offsets, b.fill, b.slot_of,
                                b.token_of, s);
  if (st == FT_OK)
    st = ft_moe_gather_rows(ctx, x_dev, xb, m->H, b.token_of, T * m->top_k, b.xg, s);
  // The per-expert row counts size the grouped launches: one small read-back.
  if (st == FT_OK) {
    cudaError_t e = cudaMemcpyAsync(m->counts_host.data(), b.counts, m->E * 4,
                                    cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) st = fail(FT_ERR_GPU, "expert counts read-back failed: %s", cudaGetErrorString(e));
  }
  if (st == FT_OK) {
    std::vector<int32_t> ex(m->E);
    std::vector<int64_t> rows(m->E);
    for (int64_t e = 0; e < m->E; ++e) {
      ex[e] = (int32_t)e;
      rows[e] = m->counts_host[e];
    }
    st = moe_expert_segments(ctx, m, (int)m->E, ex.data(), rows.data(), b.xg, x_is_bf16, b.gu,
                             b.o, s);
  }
  if (st == FT_OK) st = ft_moe_combine(ctx, m, T, b.o, b.slot_of, b.topk_w, y_dev, s);
  if (prev >= 0 && prev != ctx->device) cudaSetDevice(prev);
  return st;
}

int ft_moe_forward_host(ft_ctx* ctx, ft_moe* m, const float* input_host, size_t seq,
                        float* output_host) {
  FT_CHECK(ctx && m && input_host && output_host, FT_ERR_SHAPE, "null argument");
  if (seq == 0) return FT_OK;
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != ctx->device) FT_CUDA(cudaSetDevice(ctx->device));
  cudaStream_t s = ctx->host_stream;
  const size_t in_b = seq * (size_t)m->H * 4;
  float* dx = nullptr;
  float* dy = nullptr;
  int st = FT_OK;
  cudaError_t e = cudaMalloc(&dx, in_b);
  if (e == cudaSuccess) e = cudaMalloc(&dy, in_b);
  if (e == cudaSuccess) e = cudaMemcpyAsync(dx, input_host, in_b, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) st = ft_moe_forward(ctx, m, (int64_t)seq, dx, 0, dy, nullptr, s);
  if (e == cudaSuccess && st == FT_OK)
    e = cudaMemcpyAsync(output_host, dy, in_b, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (dx) cudaFree(dx);
  if (dy) cudaFree(dy);
  if (prev >= 0 && prev != ctx->device) cudaSetDevice(prev);
  if (e != cudaSuccess) return fail(FT_ERR_GPU, "moe forward (host) failed: %s", cudaGetErrorString(e));
  return st;
}

}  // extern "C"
