// 3-bit KV cache (TurboQuantKVCache, src/inference/turboquant_kv.rs:173-411) and
// the split-S flash-decode that reads it (math of flash_decode_ref,
// tests/kernel_tests.rs:1073-1110, with the GQA head map kv_h = h / (Hq/Hkv) of
// src/model/cpu_block_attn_res.rs:471-472).
//
// Quantisation, per head vector of 128 values (the reference's group of 128 at
// kv_dim = Hkv * 128; turboquant_kv.rs:83-117): min, max, range = max - min,
// scale = 7 / range, code = clamp(round((v - min) * scale), 0, 7) (0 when
// range == 0); dequant = min + code * ((max - min) / 7).  The append kernel
// reproduces those roundings, so the stored codes and (min, max) equal the
// reference's bit for bit; the export kernel rebuilds the reference byte stream
// (8 codes -> 3 bytes, LSB first, :35-74) from them.
//
// Device layout.  Positions live in a ring of `cap` slots (cap a multiple of
// 32); logical position p of the cache is slot (head + p) % cap, so evicting
// the oldest positions only moves `head`.  Per (sequence, kv head) "row" the
// slots are grouped in blocks of 32, and each block is stored "lane-major":
// the 12 words that lane L = 4g + r (g = L/4, r = L%4) of a decode warp feeds
// into its tensor-core fragments are contiguous (48 bytes at L*48), so a lane
// reads them with three 128-bit shared loads.
// The unit of storage is a "triple": 3 words holding 8 quads Q = 0..7 of 4
// codes each, byte b of every word belonging to element b of each quad.
// Quads 0..5 are whole 3-bit fields (word Q/2, bits 8b + 3(Q%2) .. +2), so a
// quad becomes the 4 bytes of an int8 fragment register with one shift and
// one mask; quads 6 and 7 keep their low 2 bits in bits 8b+6..7 of word 0 and
// word 1 and their high bit in word 2 at bit 8b + Q.
//   K block (1536 B): slot s = g + 8e (e in 0..3) sits in lane group g; lane
//     4g + r, triple e holds slot s's codes of dims 4(r + 4Q) + b.
//   V block (1536 B): lane 4g + r, triple m (0..3) holds, for j = 0..3 and
//     a = 0..1, quad Q = 2j + a: the codes of dim 16(2m + j/2) + g + 8(j%2) at
//     slots r + 4a + 8b.
//   min/max: per block 32 float2 (K and V separately), slot s at (s%8)*4 + s/8.
// A block's K words, V words, K min/max and V min/max form one 3584-byte
// record, and consecutive blocks of a row are contiguous, so a tile of 4
// blocks is one bulk copy.
// 3 bits per code: 48 B of codes + 8 B of (min, max) per vector, the
// reference's footprint.
//
// Decode, per (sequence, kv head, group of <=4 q heads, split of the slots):
// four compute warps each take one 32-slot block of every 128-slot tile; a
// producer warp streams tiles into a 4-stage shared-memory ring with 1-D bulk
// copies.  Scores: mma.m16n8k32 with A = K codes (16 slots x 32 dims) and B =
// the q heads as 4 signed base-256 digits of round(q * 2^30 / absmax(q)),
// accumulated exactly in int32; q.k = min * sum(q) + (max-min)/7 * sum(q_i c_i).
// Online softmax in base 2.  P.V: mma.m16n8k32 with A = V codes (16 dims x 32
// slots) and B = the weights w = p * (max-min)/7 as 4 unsigned base-256 digits
// of round(w * 2^E); the digit sums stay exact in int32 and fold into fp32 only
// when the running max or the scale 2^E changes, and at the end.  The
// min * p term is a per-head scalar added to every dim.  Each split writes
// (m, l, numerator) partials; a combine kernel merges the splits.
//
// Mode T (ft_kv3_create_mode with mode 1; no working reference implementation,
// so parity is against this project's own oracle): each vector v is stored
// rotated, y = H D v / ||v|| (D = seeded +-1 signs, H the 128-point
// Walsh-Hadamard transform), coded as code = clamp(floor((y / 2.5 + 1) * 4), 0, 7)
// -- the nearest of the 8 uniform centroids (2i+1)/8 - 1 on [-1, 1] of y/2.5,
// the levels the reference's compute_mse_centroids (src/compute/turboquant.rs:
// 197-220) converges to -- and (min, max) = (-m, +m), m = ||v|| * 2.5 * 7/8 /
// sqrt(128).  In the rotated domain the vector is then affine in the code, so
// the same record and the same decode serve both modes: decode rotates q with
// H D / sqrt(128), and the split combine rotates the output back with
// D H / sqrt(128).
#include <cmath>
#include <cstring>
#include <vector>

#include "ft_internal.cuh"
#include "ft_tc.cuh"

struct ft_kv3 {
  int device = 0;
  int64_t batch = 0, kv_heads = 0, cap = 0;  // cap: slots per row, multiple of 32
  int64_t head = 0, len = 0;                   // ring start slot, live positions
  uint32_t* blocks = nullptr;  // [row][cap/32] block records
  ft::Workspace part;  // split partials
  int mode = 0;                // 0: the reference's min/max scheme, 1: mode T
  float* signs = nullptr;      // mode T: the 128 rotation signs (device)
  ft::Workspace rot;           // mode T: the rotated queries
};

// The page pool of the paged cache: page P holds 32 positions of every kv
// head, record (P, h) at (P * kv_heads + h) * 3584 bytes -- the ring's record,
// so the same kernels serve both.  The pool is storage only: which pages a
// sequence owns, and in which order, is the caller's block table.
struct ft_kvp {
  int device = 0;
  int64_t n_pages = 0, kv_heads = 0;
  uint32_t* blocks = nullptr;
  int mode = 0;
  float* signs = nullptr;
  ft::Workspace part, rot;
};

namespace ft {
namespace {

constexpr int kD = 128;                  // head dim = quantisation group
constexpr int kRec = 48;                 // bytes of codes per vector
constexpr int kBlk = 32;                 // slots per block
constexpr int kBlkWords = kBlk * kRec / 4;  // 384
constexpr int kBlkBytes = kBlk * kRec;   // 1536 (both K and V)
constexpr int kMmBlkBytes = kBlk * 8;    // 256
constexpr int kDecWarps = 4;             // compute warps = blocks per tile
#ifndef FT_KV_STAGES
#define FT_KV_STAGES 4
#endif
constexpr int kStages = FT_KV_STAGES;
constexpr int kRecBytes = 2 * kBlkBytes + 2 * kMmBlkBytes;  // 3584: K | V | K min/max | V min/max
constexpr int kRecWords = kRecBytes / 4;
constexpr int kRecV = kBlkWords, kRecKmm = 2 * kBlkWords, kRecVmm = 2 * kBlkWords + 2 * kBlk;
constexpr int kStageBytes = kDecWarps * kRecBytes;  // 14336
constexpr int kWsmBytes = kDecWarps * 4 * 4 * kBlk;      // [warp][digit][head][8 words]
constexpr int kQfBytes = 4 * 32 * 16;                    // q fragments [chunk][lane][16 B]
constexpr int kOsmBytes = kDecWarps * 4 * kD * 4;        // fp32 numerators [warp][head][128]
constexpr int kQdBytes = 4 * 4 * kD;  // q digits [head][digit][128], staged in the numerator area
constexpr int kOffW = kStages * kStageBytes;
constexpr int kOffQf = kOffW + kWsmBytes;
constexpr int kOffO = kOffQf + kQfBytes;
constexpr int kOffQinfo = kOffO + kOsmBytes;
constexpr int kOffBars = kOffQinfo + 64;
constexpr int kDecSmem = kOffBars + 16 * kStages;
constexpr int kPart = 2 + kD;  // partial record: m (log2 domain), l, numerator[128]
static_assert(kQdBytes <= kOsmBytes, "q digits are staged in the numerator area");
#ifndef FT_KV_MIN_BLOCKS
#define FT_KV_MIN_BLOCKS 3
#endif

__device__ __forceinline__ float load_act(const void* p, int64_t i, int bf16) {
  return bf16 ? __uint_as_float((uint32_t) static_cast<const uint16_t*>(p)[i] << 16)
              : static_cast<const float*>(p)[i];
}

// ---- layout maps (word indices within a 384-word block) ----
// triple base word and quad of K code (slot s, dim d) / V code (slot s, dim d)
__device__ __forceinline__ int k_triple(int s, int d) {
  return (4 * (s & 7) + ((d >> 2) & 3)) * 12 + 3 * (s >> 3);
}
__device__ __forceinline__ int k_quad(int d) { return d >> 4; }
__device__ __forceinline__ int k_elem(int s, int d) { return d & 3; }
__device__ __forceinline__ int v_triple(int s, int d) {
  return (4 * (d & 7) + (s & 3)) * 12 + 3 * (d >> 5);
}
__device__ __forceinline__ int v_quad(int s, int d) {
  return 2 * (2 * ((d >> 4) & 1) + ((d >> 3) & 1)) + ((s >> 2) & 1);
}
__device__ __forceinline__ int v_elem(int s) { return s >> 3; }
__device__ __forceinline__ int mm_index(int s) { return (s & 7) * 4 + (s >> 3); }

__device__ __forceinline__ uint32_t triple_get(const uint32_t* t, int Q, int b) {
  if (Q < 6) return (t[Q >> 1] >> (8 * b + 3 * (Q & 1))) & 7u;
  return ((t[Q - 6] >> (8 * b + 6)) & 3u) | (((t[2] >> (8 * b + Q)) & 1u) << 2);
}
// writes code c at (Q, b) of a shared-memory triple; concurrent writers touch
// disjoint bits
__device__ __forceinline__ void triple_put(uint32_t* t, int Q, int b, uint32_t c) {
  if (Q < 6) {
    const int sh = 8 * b + 3 * (Q & 1);
    atomicAnd(&t[Q >> 1], ~(7u << sh));
    atomicOr(&t[Q >> 1], c << sh);
  } else {
    atomicAnd(&t[Q - 6], ~(3u << (8 * b + 6)));
    atomicOr(&t[Q - 6], (c & 3u) << (8 * b + 6));
    atomicAnd(&t[2], ~(1u << (8 * b + Q)));
    atomicOr(&t[2], (c >> 2) << (8 * b + Q));
  }
}
__device__ __forceinline__ uint32_t k_code(const uint32_t* blk, int s, int d) {
  return triple_get(blk + k_triple(s, d), k_quad(d), k_elem(s, d));
}
__device__ __forceinline__ uint32_t v_code(const uint32_t* blk, int s, int d) {
  return triple_get(blk + v_triple(s, d), v_quad(s, d), v_elem(s));
}

// ---------------------------------------------------------------- append --
struct AppendParams {
  const void* k;  // kPacked: reference bytes [B][n][Hkv*48]; else values [B][n][Hkv][128]
  const void* v;
  const float* kmm_in;  // kPacked only: [B][n][Hkv][2]
  const float* vmm_in;
  int bf16;
  int64_t n_pos, Hkv, cap, nbc, s0;
  uint32_t* blocks;
  const float* signs;  // mode T rotation signs, or null (the reference's scheme)
  // paged pool (table != null): sequence b writes positions pos0[b] .. +n_pos,
  // logical block j of b lives in page table[b * tstride + j] (< n_pages)
  const int32_t* table;
  const int32_t* pos0;
  int64_t tstride, n_pages;
  int* err;
};

// A page index read from a caller's block table, checked: out-of-range
// entries are recorded in the error word (site `code`) and replaced by -1.
__device__ __forceinline__ int64_t checked_page(const int32_t* table, int64_t idx,
                                                int64_t n_pages, int* err, int code) {
  const int32_t pg = table[idx];
  if (pg < 0 || pg >= n_pages) {
    if (err) atomicCAS(err, 0, code);
    return -1;
  }
  return pg;
}

// Mode T constants: clip at 2.5 and the (min, max) factor 2.5 * 7/8 / sqrt(128).
constexpr float kTClip = 2.5f;
__device__ __forceinline__ float kvt_mm_const() {
  return __fdiv_rn(__fdiv_rn(__fmul_rn(kTClip, 7.0f), 8.0f), __fsqrt_rn(128.0f));
}

// In-place 128-point Walsh-Hadamard transform of y (shared), thread d = one
// element, butterflies h = 1, 2, ..., 64: y[j] = a + b, y[j + h] = a - b.
// Block-wide (128 threads).
__device__ __forceinline__ void fwht128(float* y, int d) {
  __syncthreads();  // the callers' writes of y are visible
#pragma unroll
  for (int h = 1; h < kD; h <<= 1) {
    const float a = y[d & ~h], b = y[d | h];
    __syncthreads();
    y[d] = (d & h) ? __fsub_rn(a, b) : __fadd_rn(a, b);
    __syncthreads();
  }
}

// Mode T code of element d of vector x (block-wide: every thread passes its
// element); returns the code and the vector's norm.
__device__ __forceinline__ uint32_t kvt_code(float x, float sign, int d, float* ybuf,
                                             float (*red)[4], int slot, float* norm_out) {
  const int warp = d >> 5, lane = d & 31;
  float sq = __fmul_rn(x, x);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, o));
  if (lane == 0) red[warp][slot] = sq;
  __syncthreads();
  const float n2 = __fadd_rn(__fadd_rn(__fadd_rn(red[0][slot], red[1][slot]), red[2][slot]),
                             red[3][slot]);
  const float norm = __fsqrt_rn(n2);
  ybuf[d] = norm > 0.0f ? __fmul_rn(__fdiv_rn(x, norm), sign) : 0.0f;
  fwht128(ybuf, d);
  const float c = floorf(__fmul_rn(__fadd_rn(__fdiv_rn(ybuf[d], kTClip), 1.0f), 4.0f));
  *norm_out = norm;
  return c <= 0.0f ? 0u : (c >= 7.0f ? 7u : (uint32_t)c);
}

// code idx of a reference LSB-first 3-bit stream (the next byte is read only
// when the code straddles it)
__device__ __forceinline__ uint32_t ref_stream_code(const uint8_t* bytes, int64_t idx) {
  const int64_t bit = 3 * idx;
  const int64_t by = bit >> 3;
  uint32_t w = bytes[by];
  if ((bit & 7) > 5) w |= (uint32_t)bytes[by + 1] << 8;
  return (w >> (bit & 7)) & 7u;
}

// One CTA per (32-slot block touched, row); thread = dim.  Quantises each new
// position of the block (or takes its codes from a reference byte stream),
// and rewrites the block's K and V words and min/max.
template <bool kPacked>
__global__ void __launch_bounds__(kD) kv3_append_kernel(AppendParams p) {
  const int64_t x = blockIdx.x, row = blockIdx.y;
  const int64_t b = row / p.Hkv, h = row % p.Hkv;
  const int d = threadIdx.x, warp = d >> 5, lane = d & 31;
  const int64_t s0 = p.table ? (int64_t)p.pos0[b] : p.s0;
  const int64_t off0 = s0 % kBlk;
  const int u_begin = x == 0 ? (int)off0 : 0;
  int64_t u_end64 = p.n_pos + off0 - x * kBlk;
  const int u_end = u_end64 > kBlk ? kBlk : (int)u_end64;
  if (u_begin >= u_end) return;  // paged: this sequence touches fewer blocks
  int64_t rec;                   // record index of the block
  if (p.table) {
    const int64_t lb = s0 / kBlk + x;
    if (s0 < 0 || lb >= p.tstride) {
      if (d == 0) atomicCAS(p.err, 0, 1001);
      return;
    }
    const int64_t pg = checked_page(p.table, b * p.tstride + lb, p.n_pages, p.err, 1002);
    if (pg < 0) return;
    rec = pg * p.Hkv + h;
  } else {
    rec = row * p.nbc + (s0 / kBlk + x) % p.nbc;
  }
  __shared__ float red[4][4];
  __shared__ uint32_t kw[kBlkWords], vw[kBlkWords];
  __shared__ float ybk[kD], ybv[kD];
  uint32_t* kg = p.blocks + rec * kRecWords;
  uint32_t* vg = kg + kRecV;
  float2* kmm = reinterpret_cast<float2*>(kg + kRecKmm);
  float2* vmm = reinterpret_cast<float2*>(kg + kRecVmm);
  for (int i = d; i < kBlkWords; i += kD) {
    kw[i] = kg[i];
    vw[i] = vg[i];
  }
  __syncthreads();
  for (int u = u_begin; u < u_end; ++u) {
    const int64_t pi = x * kBlk + u - off0;  // input position
    const int64_t vec = (b * p.n_pos + pi) * p.Hkv + h;
    uint32_t ck, cv;
    float kmin, kmax, vmin, vmax;
    if (kPacked) {
      const int64_t rowbytes = p.Hkv * kRec;
      const uint8_t* kb = static_cast<const uint8_t*>(p.k) + (b * p.n_pos + pi) * rowbytes;
      const uint8_t* vb = static_cast<const uint8_t*>(p.v) + (b * p.n_pos + pi) * rowbytes;
      ck = ref_stream_code(kb, h * kD + d);
      cv = ref_stream_code(vb, h * kD + d);
      kmin = p.kmm_in[vec * 2];
      kmax = p.kmm_in[vec * 2 + 1];
      vmin = p.vmm_in[vec * 2];
      vmax = p.vmm_in[vec * 2 + 1];
    } else if (p.signs) {
      // mode T: norm, signs, Walsh-Hadamard, uniform codebook
      const float xk = load_act(p.k, vec * kD + d, p.bf16);
      const float xv = load_act(p.v, vec * kD + d, p.bf16);
      const float sg = p.signs[d];
      float nk, nv;
      ck = kvt_code(xk, sg, d, ybk, red, 0, &nk);
      cv = kvt_code(xv, sg, d, ybv, red, 1, &nv);
      const float C = kvt_mm_const();
      kmax = __fmul_rn(C, nk);
      kmin = -kmax;
      vmax = __fmul_rn(C, nv);
      vmin = -vmax;
    } else {
      const float xk = load_act(p.k, vec * kD + d, p.bf16);
      const float xv = load_act(p.v, vec * kD + d, p.bf16);
      float a0 = xk, a1 = xk, a2 = xv, a3 = xv;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        a0 = fminf(a0, __shfl_xor_sync(0xffffffffu, a0, o));
        a1 = fmaxf(a1, __shfl_xor_sync(0xffffffffu, a1, o));
        a2 = fminf(a2, __shfl_xor_sync(0xffffffffu, a2, o));
        a3 = fmaxf(a3, __shfl_xor_sync(0xffffffffu, a3, o));
      }
      if (lane == 0) {
        red[warp][0] = a0;
        red[warp][1] = a1;
        red[warp][2] = a2;
        red[warp][3] = a3;
      }
      __syncthreads();
      kmin = fminf(fminf(red[0][0], red[1][0]), fminf(red[2][0], red[3][0]));
      kmax = fmaxf(fmaxf(red[0][1], red[1][1]), fmaxf(red[2][1], red[3][1]));
      vmin = fminf(fminf(red[0][2], red[1][2]), fminf(red[2][2], red[3][2]));
      vmax = fmaxf(fmaxf(red[0][3], red[1][3]), fmaxf(red[2][3], red[3][3]));
      // quantize_3bit (turboquant_kv.rs:83-107), same roundings
      const float kr = __fsub_rn(kmax, kmin), vr = __fsub_rn(vmax, vmin);
      ck = 0;
      if (kr > 0.0f) {
        const float q = roundf(__fmul_rn(__fsub_rn(xk, kmin), __fdiv_rn(7.0f, kr)));
        ck = q <= 0.0f ? 0u : (q >= 7.0f ? 7u : (uint32_t)q);
      }
      cv = 0;
      if (vr > 0.0f) {
        const float q = roundf(__fmul_rn(__fsub_rn(xv, vmin), __fdiv_rn(7.0f, vr)));
        cv = q <= 0.0f ? 0u : (q >= 7.0f ? 7u : (uint32_t)q);
      }
    }
    triple_put(kw + k_triple(u, d), k_quad(d), k_elem(u, d), ck);
    triple_put(vw + v_triple(u, d), v_quad(u, d), v_elem(u), cv);
    if (d == 0) kmm[mm_index(u)] = make_float2(kmin, kmax);
    if (d == 1) vmm[mm_index(u)] = make_float2(vmin, vmax);
    __syncthreads();  // red is reused by the next position
  }
  for (int i = d; i < kBlkWords; i += kD) {
    kg[i] = kw[i];
    vg[i] = vw[i];
  }
}

// ------------------------------------------------------- read-back kernels --
struct RangeParams {
  int64_t B, Hkv, cap, nbc, head, start, n;
  const uint32_t* blocks;
  const int32_t* table;  // paged pool: positions start + pos of sequence b through the table
  int64_t tstride, n_pages;
  int* err;
};

// The record holding position `pos` of the range for (b, h) and its slot in
// the block; null for a bad table entry (recorded in the error word).
__device__ __forceinline__ const uint32_t* range_record(const RangeParams& p, int64_t b,
                                                       int64_t h, int64_t pos, int* s) {
  if (p.table) {
    const int64_t lpos = p.start + pos;
    *s = (int)(lpos % kBlk);
    const int64_t pg = checked_page(p.table, b * p.tstride + lpos / kBlk, p.n_pages, p.err, 1003);
    return pg < 0 ? nullptr : p.blocks + (pg * p.Hkv + h) * kRecWords;
  }
  const int64_t slot = (p.head + p.start + pos) % p.cap;
  *s = (int)(slot % kBlk);
  return p.blocks + ((b * p.Hkv + h) * p.nbc + slot / kBlk) * kRecWords;
}

// get_range (turboquant_kv.rs:271-291): out [B][n][Hkv][128] f32, dequantised
// with the reference's roundings (dequantize_3bit :110-117).
// Mode T (signs != null): the rotated-domain values are rotated back,
// v = D H y / sqrt(128).
__global__ void kv3_dequant_kernel(RangeParams p, float* __restrict__ kout,
                                   float* __restrict__ vout, const float* __restrict__ signs) {
  const int64_t vec = blockIdx.x;  // (b, pos, h)
  const int d = threadIdx.x;
  const int64_t h = vec % p.Hkv;
  const int64_t pos = (vec / p.Hkv) % p.n;
  const int64_t b = vec / (p.Hkv * p.n);
  int s;
  const uint32_t* rec = range_record(p, b, h, pos, &s);
  if (!rec) {  // uniform over the block: no barrier is skipped by part of it
    kout[vec * kD + d] = 0.0f;
    vout[vec * kD + d] = 0.0f;
    return;
  }
  const uint32_t ck = k_code(rec, s, d);
  const uint32_t cv = v_code(rec + kRecV, s, d);
  const float2 km = reinterpret_cast<const float2*>(rec + kRecKmm)[mm_index(s)];
  const float2 vm = reinterpret_cast<const float2*>(rec + kRecVmm)[mm_index(s)];
  float kv, vv;
  if (km.y == km.x) {
    kv = km.x;
  } else {
    kv = __fadd_rn(km.x, __fmul_rn((float)ck, __fdiv_rn(__fsub_rn(km.y, km.x), 7.0f)));
  }
  if (vm.y == vm.x) {
    vv = vm.x;
  } else {
    vv = __fadd_rn(vm.x, __fmul_rn((float)cv, __fdiv_rn(__fsub_rn(vm.y, vm.x), 7.0f)));
  }
  if (signs) {
    __shared__ float yk[kD], yv[kD];
    yk[d] = kv;
    yv[d] = vv;
    fwht128(yk, d);
    fwht128(yv, d);
    const float sc = __fdiv_rn(1.0f, __fsqrt_rn(128.0f));
    kv = __fmul_rn(__fmul_rn(yk[d], sc), signs[d]);
    vv = __fmul_rn(__fmul_rn(yv[d], sc), signs[d]);
  }
  kout[vec * kD + d] = kv;
  vout[vec * kD + d] = vv;
}

// Mode T rotation of 128-vectors (one CTA each): out = H D in / sqrt(128)
// (forward) or D H in / sqrt(128) (inverse).
__global__ void kv3_rotate_kernel(const float* __restrict__ in, float* __restrict__ out,
                                  const float* __restrict__ signs, int inverse) {
  __shared__ float y[kD];
  const int64_t v = blockIdx.x;
  const int d = threadIdx.x;
  const float x = in[v * kD + d];
  y[d] = inverse ? x : __fmul_rn(x, signs[d]);
  fwht128(y, d);
  const float sc = __fdiv_rn(1.0f, __fsqrt_rn(128.0f));
  out[v * kD + d] = inverse ? __fmul_rn(__fmul_rn(y[d], sc), signs[d]) : __fmul_rn(y[d], sc);
}

// The reference's stored form: codes [B][n][Hkv*48] bytes (pack_3bit over the
// whole kv_dim vector) and (min, max) [B][n][Hkv][2].  Thread = 8 codes.
__global__ void kv3_export_kernel(RangeParams p, uint8_t* __restrict__ kbytes,
                                  float* __restrict__ kmm_out, uint8_t* __restrict__ vbytes,
                                  float* __restrict__ vmm_out) {
  const int64_t vec = blockIdx.x;  // (b, pos, h)
  const int m = threadIdx.x;       // 0..15: codes 8m..8m+7
  const int64_t h = vec % p.Hkv;
  const int64_t pos = (vec / p.Hkv) % p.n;
  const int64_t b = vec / (p.Hkv * p.n);
  int s;
  const uint32_t* kb = range_record(p, b, h, pos, &s);
  if (!kb) return;
  const uint32_t* vb = kb + kRecV;
  uint32_t kbits = 0, vbits = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    kbits |= k_code(kb, s, 8 * m + j) << (3 * j);
    vbits |= v_code(vb, s, 8 * m + j) << (3 * j);
  }
  const int64_t o = vec * kRec + 3 * m;  // [B][n][Hkv][48] == [B][n][Hkv*48]
  kbytes[o] = (uint8_t)(kbits & 0xFF);
  kbytes[o + 1] = (uint8_t)((kbits >> 8) & 0xFF);
  kbytes[o + 2] = (uint8_t)((kbits >> 16) & 0xFF);
  vbytes[o] = (uint8_t)(vbits & 0xFF);
  vbytes[o + 1] = (uint8_t)((vbits >> 8) & 0xFF);
  vbytes[o + 2] = (uint8_t)((vbits >> 16) & 0xFF);
  if (m == 0) {
    const float2 km = reinterpret_cast<const float2*>(kb + kRecKmm)[mm_index(s)];
    const float2 vm = reinterpret_cast<const float2*>(kb + kRecVmm)[mm_index(s)];
    kmm_out[vec * 2] = km.x;
    kmm_out[vec * 2 + 1] = km.y;
    vmm_out[vec * 2] = vm.x;
    vmm_out[vec * 2 + 1] = vm.y;
  }
}

// ---------------------------------------------------------------- decode --
struct DecodeParams {
  const float* q;  // [B][Hq][128]
  int64_t Hq, Hkv;
  int G, hgroups;  // q heads per kv head, CTAs (groups of <=4 q heads) per kv head
  int64_t nbc, head_off, head_blk, len;
  int64_t nlb;        // logical 32-slot blocks covering the live range
  int64_t tiles_per;  // 128-slot tiles per split
  float qk_log2;      // softmax scale * log2(e)
  const uint32_t* blocks;
  float* part;  // [B][Hq][nsplit][kPart]
  int* err;
  // paged pool (table != null): sequence b holds seq_lens[b] positions (at
  // most len), logical block j in page table[b * tstride + j] (< n_pages)
  const int32_t* table;
  const int32_t* seq_lens;
  int64_t tstride, n_pages;
};

__device__ __forceinline__ void mma_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_u8u8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// quad Q of a triple as the 4 bytes of an int8 fragment register
template <int Q>
__device__ __forceinline__ uint32_t tquad(uint32_t w0, uint32_t w1, uint32_t w2) {
  constexpr uint32_t M3 = 0x07070707u;
  if (Q == 0) return w0 & M3;
  if (Q == 1) return (w0 >> 3) & M3;
  if (Q == 2) return w1 & M3;
  if (Q == 3) return (w1 >> 3) & M3;
  if (Q == 4) return w2 & M3;
  if (Q == 5) return (w2 >> 3) & M3;
  if (Q == 6) return ((w0 >> 6) & 0x03030303u) | ((w2 >> 4) & 0x04040404u);
  return ((w1 >> 6) & 0x03030303u) | ((w2 >> 5) & 0x04040404u);
}

// exact for |d| < 2^22
__device__ __forceinline__ float small_int_to_float(int d) {
  return __int_as_float(0x4B400000 + d) - 12582912.0f;
}

__global__ void __launch_bounds__((kDecWarps + 1) * 32, FT_KV_MIN_BLOCKS)
    kv3_decode_kernel(const __grid_constant__ DecodeParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint32_t* wsm = reinterpret_cast<uint32_t*>(smem + kOffW);        // W digit words
  const uint4* qf = reinterpret_cast<const uint4*>(smem + kOffQf);   // q fragments
  float* osm = reinterpret_cast<float*>(smem + kOffO);               // fp32 numerators
  float* qinfo = reinterpret_cast<float*>(smem + kOffQinfo);         // qsum*, qscale*
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBars);
  const uint32_t full0 = tc::smem_u32(bars), empty0 = full0 + 8 * kStages;

  const int split = blockIdx.x;
  const int64_t kvh = blockIdx.y / p.hgroups;
  const int hg = blockIdx.y % p.hgroups;
  const int64_t b = blockIdx.z;
  const int64_t row = b * p.Hkv + kvh;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, r = lane & 3;
  int nheads = p.G - 4 * hg;
  if (nheads > 4) nheads = 4;
  const int64_t qh0 = kvh * p.G + 4 * hg;  // first q head of this CTA
  // live positions and logical blocks of this sequence
  int64_t len_b = p.len, nlb_b = p.nlb;
  if (p.table) {
    len_b = p.seq_lens[b];
    if (len_b < 0 || len_b > p.len) {
      if (tid == 0) atomicCAS(p.err, 0, 1004);
      len_b = len_b < 0 ? 0 : p.len;
    }
    nlb_b = (len_b + kBlk - 1) / kBlk;
  }

  const int64_t ntiles_all = (nlb_b + kDecWarps - 1) / kDecWarps;
  const int64_t t_begin = (int64_t)split * p.tiles_per;
  int64_t t_end = t_begin + p.tiles_per;
  if (t_end > ntiles_all) t_end = ntiles_all;
  const int ntiles = t_end > t_begin ? (int)(t_end - t_begin) : 0;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      tc::mbar_init(full0 + 8 * s, 1);
      tc::mbar_init(empty0 + 8 * s, kDecWarps);
    }
    tc::fence_barrier_init();
  }
  // q prep: warp w < 4 turns head w of the group (zeros past nheads) into
  // 4 signed base-256 digits of round(q * 2^30 / absmax), staged in the W area
  int8_t* qd = reinterpret_cast<int8_t*>(smem + kOffO);  // [head][digit][128], reused below
  if (warp < 4) {
    float qv[4];
    const bool valid = warp < nheads;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      qv[j] = valid ? p.q[((b * p.Hq) + qh0 + warp) * kD + 4 * lane + j] : 0.0f;
    float amax = fmaxf(fmaxf(fabsf(qv[0]), fabsf(qv[1])), fmaxf(fabsf(qv[2]), fabsf(qv[3])));
    float sum = (qv[0] + qv[1]) + (qv[2] + qv[3]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      sum += __shfl_xor_sync(0xffffffffu, sum, o);
    }
    const float mul = amax > 0.0f ? __fdiv_rn(1073741824.0f, amax) : 0.0f;  // 2^30 / amax
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int X = __float2int_rn(qv[j] * mul);
      const int dim = 4 * lane + j;
#pragma unroll
      for (int dg = 0; dg < 3; ++dg) {
        const int lo = ((X & 255) ^ 128) - 128;  // signed digit in [-128, 127]
        qd[(warp * 4 + dg) * kD + dim] = (int8_t)lo;
        X = (X - lo) >> 8;
      }
      qd[(warp * 4 + 3) * kD + dim] = (int8_t)X;  // |X| <= 65 here
    }
    if (lane == 0) {
      qinfo[warp] = sum * p.qk_log2;                                // sum(q) in score units
      qinfo[4 + warp] = amax * 9.313225746154785e-10f * p.qk_log2;  // amax / 2^30, same
    }
  }
  __syncthreads();
  // q B fragments, chunk c = ks (k-step of 32 dims): words {nb0 b0, nb0 b1, nb1 b0, nb1 b1};
  // column n = g <-> (head g/2, digit g%2 + 2*nb)
  if (warp < 4) {
    const int ks = warp;
    uint32_t w4[4];
#pragma unroll
    for (int nb = 0; nb < 2; ++nb) {
      const int8_t* src = qd + ((g >> 1) * 4 + (g & 1) + 2 * nb) * kD + 32 * ks + 4 * r;
      w4[2 * nb] = *reinterpret_cast<const uint32_t*>(src);
      w4[2 * nb + 1] = *reinterpret_cast<const uint32_t*>(src + 16);
    }
    reinterpret_cast<uint4*>(smem + kOffQf)[ks * 32 + lane] =
        make_uint4(w4[0], w4[1], w4[2], w4[3]);
  }
  __syncthreads();
  // the numerators start at zero (the q digits there are no longer needed)
  for (int i = tid; i < kDecWarps * 4 * kD; i += blockDim.x) osm[i] = 0.0f;
  __syncthreads();

  const uint32_t stage_base = tc::smem_u32(smem);
  if (warp == kDecWarps) {
    // ------------------------------------------------------ producer warp --
    if (lane == 0) {
      bool ok = true;
      int issued = 0;
      int64_t pb = (p.head_blk + t_begin * kDecWarps) % p.nbc;
      for (int it = 0; it < ntiles && ok; ++it) {
        const int s = it % kStages;
        if (it >= kStages)
          ok = tc::mbar_wait(empty0 + 8 * s, ((it / kStages) - 1) & 1, p.err, 31);
        if (!ok) break;
        const int64_t j0 = (t_begin + it) * kDecWarps;
        const int nb = nlb_b - j0 < kDecWarps ? (int)(nlb_b - j0) : kDecWarps;
        tc::mbar_arrive_expect_tx(full0 + 8 * s, nb * kRecBytes);
        const uint32_t sb = stage_base + s * kStageBytes;
        if (p.table) {
          // one record per page; a bad table entry reads page 0 (the launch
          // is reported invalid through the error word)
          for (int i = 0; i < nb; ++i) {
            int64_t pg = checked_page(p.table, b * p.tstride + j0 + i, p.n_pages, p.err, 1005);
            if (pg < 0) pg = 0;
            tc::bulk_g2s(sb + i * kRecBytes, p.blocks + (pg * p.Hkv + kvh) * kRecWords,
                         kRecBytes, full0 + 8 * s);
          }
        } else {
          // nb consecutive records from physical block pb, wrapping at most once
          const int n1 = pb + nb <= p.nbc ? nb : (int)(p.nbc - pb);
          tc::bulk_g2s(sb, p.blocks + (row * p.nbc + pb) * kRecWords, n1 * kRecBytes,
                       full0 + 8 * s);
          if (n1 < nb)
            tc::bulk_g2s(sb + n1 * kRecBytes, p.blocks + row * p.nbc * kRecWords,
                         (nb - n1) * kRecBytes, full0 + 8 * s);
          pb += nb;
          if (pb >= p.nbc) pb -= p.nbc;
        }
        ++issued;
      }
      // the copies of the last stages must land before the CTA may exit
      for (int it = issued - kStages < 0 ? 0 : issued - kStages; it < issued; ++it)
        tc::mbar_wait(full0 + 8 * (it % kStages), (it / kStages) & 1, p.err, 32);
    }
    return;
  }

  // -------------------------------------------------------- compute warps --
  const float qsum = qinfo[r], qscale = qinfo[4 + r];
  float m_run = -INFINITY, l_part = 0.0f, vmin_part = 0.0f;
  int pv[8][2][4];
#pragma unroll
  for (int mb = 0; mb < 8; ++mb)
#pragma unroll
    for (int nb = 0; nb < 2; ++nb)
#pragma unroll
      for (int c = 0; c < 4; ++c) pv[mb][nb][c] = 0;
  float wmul = 0.0f, wbound = 0.0f;  // W = p * vs * wmul, valid while vs < wbound
  uint32_t* my_w = wsm + warp * (4 * 4 * 8);
  float* my_o = osm + (warp * 4 + r) * kD;  // head r
  bool ok = true;

  // adds the digit sums times `inv` to the numerators and clears them; then
  // scales the numerators by alpha
  auto fold_scale = [&](float inv, float alpha) {
#pragma unroll
    for (int mb = 0; mb < 8; ++mb)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        // sum_j 256^j d_j in fp32 (relative error a few 2^-24)
        const float v = fmaf(fmaf(fmaf((float)pv[mb][1][2 * h + 1], 256.0f, (float)pv[mb][1][2 * h]),
                                  256.0f, (float)pv[mb][0][2 * h + 1]),
                             256.0f, (float)pv[mb][0][2 * h]);
        float* o = my_o + 16 * mb + g + 8 * h;
        *o = fmaf(v, inv, *o) * alpha;
      }
#pragma unroll
    for (int mb = 0; mb < 8; ++mb)
#pragma unroll
      for (int nb = 0; nb < 2; ++nb)
#pragma unroll
        for (int c = 0; c < 4; ++c) pv[mb][nb][c] = 0;
  };

  // 32-bit block arithmetic: the host keeps head_off + len below 2^31 - 64
  const int nlb32 = (int)nlb_b, hoff = p.table ? 0 : (int)p.head_off, len32 = (int)len_b;
  int j = (int)(t_begin * kDecWarps) + warp;  // logical block of this warp in tile `it`
  for (int it = 0; it < ntiles; ++it, j += kDecWarps) {
    const int s = it % kStages;
    if (ok) ok = tc::mbar_wait(full0 + 8 * s, (it / kStages) & 1, p.err, 33);
    if (ok && j < nlb32) {
      const uint8_t* sb = smem + s * kStageBytes + warp * kRecBytes;
      const uint4* kb4 = reinterpret_cast<const uint4*>(sb) + lane * 3;
      const uint4* vb4 = reinterpret_cast<const uint4*>(sb + 4 * kRecV) + lane * 3;
      const float4* km4 = reinterpret_cast<const float4*>(sb + 4 * kRecKmm) + g * 2;
      const float4* vm4 = reinterpret_cast<const float4*>(sb + 4 * kRecVmm) + g * 2;
      // live slots of this block: u in [lo_live, hi_live)
      const int base = j * kBlk - hoff;
      const int lo_live = base >= 0 ? 0 : -base;
      const int hl = len32 - base;
      const int hi_live = hl >= kBlk ? kBlk : hl;
      // ---- scores: this lane's slots u = g + 8e, e = 2*mb + h
      float s2[4], vsv[4], vmn[4];
      {
#pragma unroll
        for (int mb = 0; mb < 2; ++mb) {
          int acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
          // triples of slots e = 2mb (row g) and 2mb + 1 (row g + 8): words 6mb .. 6mb+5
          uint32_t kw0[2], kw1[2], kw2[2];
          const uint32_t* kwp = reinterpret_cast<const uint32_t*>(kb4) + 6 * mb;
          if (mb == 0) {
            const uint4 x = *reinterpret_cast<const uint4*>(kwp);
            const uint2 y = *reinterpret_cast<const uint2*>(kwp + 4);
            kw0[0] = x.x; kw1[0] = x.y; kw2[0] = x.z; kw0[1] = x.w; kw1[1] = y.x; kw2[1] = y.y;
          } else {
            const uint2 x = *reinterpret_cast<const uint2*>(kwp);
            const uint4 y = *reinterpret_cast<const uint4*>(kwp + 2);
            kw0[0] = x.x; kw1[0] = x.y; kw2[0] = y.x; kw0[1] = y.y; kw1[1] = y.z; kw2[1] = y.w;
          }
          const int ea = 0, eb = 1;
          // k-step ks covers quads 2ks (a0, a1) and 2ks + 1 (a2, a3)
#define FT_KSTEP(KS)                                                                      \
  {                                                                                       \
    const uint4 bq = qf[(KS) * 32 + lane];                                                \
    const uint32_t a0 = tquad<2 * (KS)>(kw0[ea], kw1[ea], kw2[ea]);                       \
    const uint32_t a1 = tquad<2 * (KS)>(kw0[eb], kw1[eb], kw2[eb]);                       \
    const uint32_t a2 = tquad<2 * (KS) + 1>(kw0[ea], kw1[ea], kw2[ea]);                   \
    const uint32_t a3 = tquad<2 * (KS) + 1>(kw0[eb], kw1[eb], kw2[eb]);                   \
    mma_u8s8(acc[0], a0, a1, a2, a3, bq.x, bq.y);                                         \
    mma_u8s8(acc[1], a0, a1, a2, a3, bq.z, bq.w);                                         \
  }
          FT_KSTEP(0) FT_KSTEP(1) FT_KSTEP(2) FT_KSTEP(3)
#undef FT_KSTEP
          const float4 kmA = km4[mb];  // (min, max) of slots e = 2mb, 2mb + 1
          const float4 vmA = vm4[mb];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int e = 2 * mb + h;
            const float S = fmaf(
                fmaf(fmaf(small_int_to_float(acc[1][2 * h + 1]), 256.0f,
                          small_int_to_float(acc[1][2 * h])),
                     256.0f, small_int_to_float(acc[0][2 * h + 1])),
                256.0f, small_int_to_float(acc[0][2 * h]));
            const float kmin = h ? kmA.z : kmA.x, kmax = h ? kmA.w : kmA.y;
            const float vmin = h ? vmA.z : vmA.x, vmax = h ? vmA.w : vmA.y;
            const float ksc = (kmax - kmin) * 0.14285714285714285f;
            s2[e] = fmaf(kmin, qsum, ksc * (S * qscale));
            vsv[e] = (vmax - vmin) * 0.14285714285714285f;
            vmn[e] = vmin;
          }
        }
      }
      if (lo_live > 0 || hi_live < kBlk) {  // a partial block (warp-uniform)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int u = g + 8 * e;
          if (u < lo_live || u >= hi_live) {
            s2[e] = -INFINITY;
            vsv[e] = 0.0f;
            vmn[e] = 0.0f;
          }
        }
      }
      // ---- online softmax (head r): max over the block's 32 slots
      float mt = fmaxf(fmaxf(s2[0], s2[1]), fmaxf(s2[2], s2[3]));
#pragma unroll
      for (int o2 = 4; o2 < 32; o2 <<= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o2));
      const float vloc = fmaxf(fmaxf(vsv[0], vsv[1]), fmaxf(vsv[2], vsv[3]));
      const bool rescale = __any_sync(0xffffffffu, vloc >= wbound && vloc > 0.0f);
      const float m_new = fmaxf(m_run, mt);
      if (m_new > m_run || rescale) {
        const float alpha = m_run == -INFINITY ? 0.0f : exp2f(m_run - m_new);
        if (wmul > 0.0f) fold_scale(1.0f / wmul, alpha);
        else {
#pragma unroll
          for (int mb = 0; mb < 8; ++mb)
#pragma unroll
            for (int h = 0; h < 2; ++h) my_o[16 * mb + g + 8 * h] *= alpha;
        }
        if (rescale) {
          float vsmax = vloc;
#pragma unroll
          for (int o2 = 1; o2 < 32; o2 <<= 1)
            vsmax = fmaxf(vsmax, __shfl_xor_sync(0xffffffffu, vsmax, o2));
          int e;
          frexpf(vsmax, &e);  // vsmax < 2^e
          wbound = ldexpf(1.0f, e);
          wmul = ldexpf(1.0f, 31 - e);
        }
        l_part *= alpha;
        vmin_part *= alpha;
        m_run = m_new;
      }
      // ---- probabilities -> W digit words: word (digit, head r, g) holds the
      // digit of the W of slots g + 8e as byte e
      uint32_t W[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float pr = s2[e] == -INFINITY ? 0.0f : exp2f(s2[e] - m_run);
        l_part += pr;
        vmin_part = fmaf(pr, vmn[e], vmin_part);
        W[e] = __float2uint_rn(pr * vsv[e] * wmul);
      }
      {
        const uint32_t t0 = __byte_perm(W[0], W[1], 0x5140), t1 = __byte_perm(W[2], W[3], 0x5140);
        const uint32_t t2 = __byte_perm(W[0], W[1], 0x7362), t3 = __byte_perm(W[2], W[3], 0x7362);
        my_w[0 * 32 + r * 8 + g] = __byte_perm(t0, t1, 0x5410);
        my_w[1 * 32 + r * 8 + g] = __byte_perm(t0, t1, 0x7632);
        my_w[2 * 32 + r * 8 + g] = __byte_perm(t2, t3, 0x5410);
        my_w[3 * 32 + r * 8 + g] = __byte_perm(t2, t3, 0x7632);
      }
      __syncwarp();
      // ---- P.V: B column n = g <-> (head g/2, digit g%2 + 2*nb); k = 4r + e <->
      // slot r + 8e (score lane g_s = r), k = 16 + 4r + e <-> slot r + 4 + 8e
      uint32_t bw[2][2];
#pragma unroll
      for (int nb = 0; nb < 2; ++nb) {
        const uint32_t* src = my_w + ((g & 1) + 2 * nb) * 32 + (g >> 1) * 8;
        bw[nb][0] = src[r];
        bw[nb][1] = src[r + 4];
      }
      {
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          // triple m: words 3m .. 3m+2, loaded in pairs of triples (uint4 + uint2
          // for m = 0, 1; uint2 + uint4 for m = 2, 3)
          const uint32_t* vwp = reinterpret_cast<const uint32_t*>(vb4) + 6 * (m >> 1);
          uint32_t t6[6];
          if ((m >> 1) == 0) {
            const uint4 x = *reinterpret_cast<const uint4*>(vwp);
            const uint2 y = *reinterpret_cast<const uint2*>(vwp + 4);
            t6[0] = x.x; t6[1] = x.y; t6[2] = x.z; t6[3] = x.w; t6[4] = y.x; t6[5] = y.y;
          } else {
            const uint2 x = *reinterpret_cast<const uint2*>(vwp);
            const uint4 y = *reinterpret_cast<const uint4*>(vwp + 2);
            t6[0] = x.x; t6[1] = x.y; t6[2] = y.x; t6[3] = y.y; t6[4] = y.z; t6[5] = y.w;
          }
          uint32_t vw0[4], vw1[4], vw2[4];
          vw0[m] = t6[3 * (m & 1)];
          vw1[m] = t6[3 * (m & 1) + 1];
          vw2[m] = t6[3 * (m & 1) + 2];
          // quad Q = 2j + a: dims j = 0, 1 are rows g, g+8 of mb = 2m, j = 2, 3 of
          // mb = 2m + 1; a = 0 is k 4r..4r+3, a = 1 is k 16+4r..
          uint32_t a0 = tquad<0>(vw0[m], vw1[m], vw2[m]);
          uint32_t a1 = tquad<2>(vw0[m], vw1[m], vw2[m]);
          uint32_t a2 = tquad<1>(vw0[m], vw1[m], vw2[m]);
          uint32_t a3 = tquad<3>(vw0[m], vw1[m], vw2[m]);
          mma_u8u8(pv[2 * m][0], a0, a1, a2, a3, bw[0][0], bw[0][1]);
          mma_u8u8(pv[2 * m][1], a0, a1, a2, a3, bw[1][0], bw[1][1]);
          a0 = tquad<4>(vw0[m], vw1[m], vw2[m]);
          a1 = tquad<6>(vw0[m], vw1[m], vw2[m]);
          a2 = tquad<5>(vw0[m], vw1[m], vw2[m]);
          a3 = tquad<7>(vw0[m], vw1[m], vw2[m]);
          mma_u8u8(pv[2 * m + 1][0], a0, a1, a2, a3, bw[0][0], bw[0][1]);
          mma_u8u8(pv[2 * m + 1][1], a0, a1, a2, a3, bw[1][0], bw[1][1]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(empty0 + 8 * s);
  }
  if (wmul > 0.0f) fold_scale(1.0f / wmul, 1.0f);
#pragma unroll
  for (int o2 = 4; o2 < 32; o2 <<= 1) {
    l_part += __shfl_xor_sync(0xffffffffu, l_part, o2);
    vmin_part += __shfl_xor_sync(0xffffffffu, vmin_part, o2);
  }
  // ---- combine the 4 warps through shared memory (the stage buffers are
  // free: every issued copy has been consumed)
  float* red = reinterpret_cast<float*>(smem);  // [warp][head][4]
  if (g == 0) {
    red[(warp * 4 + r) * 4 + 0] = m_run;
    red[(warp * 4 + r) * 4 + 1] = l_part;
    red[(warp * 4 + r) * 4 + 2] = vmin_part;
  }
  asm volatile("bar.sync 1, %0;" ::"r"(kDecWarps * 32) : "memory");
  {
    const int hh = warp;  // head written by this warp; dims 4*lane..4*lane+3
    if (hh < nheads) {
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kDecWarps; ++w) M = fmaxf(M, red[(w * 4 + hh) * 4]);
      float l = 0.0f, vm = 0.0f, num[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int w = 0; w < kDecWarps; ++w) {
        const float mw = red[(w * 4 + hh) * 4];
        const float f = mw == -INFINITY ? 0.0f : exp2f(mw - M);
        l = fmaf(f, red[(w * 4 + hh) * 4 + 1], l);
        vm = fmaf(f, red[(w * 4 + hh) * 4 + 2], vm);
        const float4 o4 = reinterpret_cast<const float4*>(osm + (w * 4 + hh) * kD)[lane];
        num[0] = fmaf(f, o4.x, num[0]);
        num[1] = fmaf(f, o4.y, num[1]);
        num[2] = fmaf(f, o4.z, num[2]);
        num[3] = fmaf(f, o4.w, num[3]);
      }
      const int nsplit = gridDim.x;
      float* pp = p.part + (((b * p.Hq) + qh0 + hh) * nsplit + split) * kPart;
      if (lane == 0) {
        pp[0] = M;
        pp[1] = l;
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) pp[2 + 4 * lane + k] = num[k] + vm;
    }
  }
}

// Merges the split partials of one (sequence, q head): thread = dim.
// Mode T (signs != null): the rotated-domain output is rotated back.
__global__ void kv3_combine_kernel(const float* __restrict__ part, int nsplit,
                                   float* __restrict__ out, const float* __restrict__ signs) {
  const int64_t bh = blockIdx.x;
  const int d = threadIdx.x;
  const float* pp = part + bh * nsplit * kPart;
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, pp[s * kPart]);
  float l = 0.0f, a = 0.0f;
  for (int s = 0; s < nsplit; ++s) {
    const float m = pp[s * kPart];
    if (m == -INFINITY) continue;
    const float f = exp2f(m - M);
    l = fmaf(pp[s * kPart + 1], f, l);
    a = fmaf(pp[s * kPart + 2 + d], f, a);
  }
  float r = l > 0.0f ? a / l : 0.0f;  // l == 0: an empty paged sequence
  if (signs) {
    __shared__ float y[kD];
    y[d] = r;
    fwht128(y, d);
    r = __fmul_rn(__fmul_rn(y[d], __fdiv_rn(1.0f, __fsqrt_rn(128.0f))), signs[d]);
  }
  out[bh * kD + d] = r;
}

// Opts the decode kernel into its dynamic shared memory (once per device) and
// returns its resident CTAs per SM.
int decode_occupancy(int device) {
  static int cached[64] = {0};
  if (device >= 0 && device < 64 && cached[device]) return cached[device];
  cudaFuncSetAttribute(kv3_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kDecSmem);
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kv3_decode_kernel,
                                                    (kDecWarps + 1) * 32, kDecSmem) != cudaSuccess ||
      occ < 1)
    occ = 1;
  if (device >= 0 && device < 64) cached[device] = occ;
  return occ;
}

// New ring of at least `need` slots; the live blocks are copied in logical
// order, so the new head is head % 32.
int grow(ft_kv3* c, int64_t need, cudaStream_t s) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (s) cudaStreamIsCapturing(s, &cs);
  FT_CHECK(cs == cudaStreamCaptureStatusNone, FT_ERR_UNSUPPORTED,
           "the 3-bit KV cache must grow but the stream is being captured");
  int64_t ncap = c->cap * 2;
  if (ncap < need + kBlk) ncap = need + kBlk;  // room for the head offset
  ncap = round_up(ncap, kBlk);
  const int64_t rows = c->batch * c->kv_heads, nbc = c->cap / kBlk, nnbc = ncap / kBlk;
  uint32_t* blocks = nullptr;
  cudaError_t e = cudaMalloc(&blocks, (size_t)(rows * nnbc) * kRecBytes);
  if (e == cudaSuccess) e = cudaMemsetAsync(blocks, 0, (size_t)(rows * nnbc) * kRecBytes, s);
  if (e != cudaSuccess) {
    cudaFree(blocks);
    return fail(e == cudaErrorMemoryAllocation ? FT_ERR_OOM : FT_ERR_GPU,
                "3-bit KV cache growth to %lld slots failed: %s", (long long)ncap,
                cudaGetErrorString(e));
  }
  const int64_t hb = c->head / kBlk;
  const int64_t nlb = c->len == 0 ? 0 : (c->head % kBlk + c->len + kBlk - 1) / kBlk;
  // runs of physical blocks: [hb, hb + n1) then [0, nlb - n1)
  const int64_t n1 = nlb < nbc - hb ? nlb : nbc - hb;
  const int64_t runs[2][3] = {{hb, 0, n1}, {0, n1, nlb - n1}};  // src block, dst block, count
  const size_t rb = (size_t)kRecBytes;
  for (const auto& run : runs) {
    if (run[2] <= 0) continue;
    FT_CUDA(cudaMemcpy2DAsync(reinterpret_cast<uint8_t*>(blocks) + run[1] * rb, nnbc * rb,
                              reinterpret_cast<uint8_t*>(c->blocks) + run[0] * rb, nbc * rb,
                              run[2] * rb, rows, cudaMemcpyDeviceToDevice, s));
  }
  FT_CUDA(cudaStreamSynchronize(s));
  cudaFree(c->blocks);
  c->blocks = blocks;
  c->cap = ncap;
  c->head = c->head % kBlk;
  return FT_OK;
}

class DeviceScope {
 public:
  explicit DeviceScope(int dev) : dev_(dev) {
    cudaGetDevice(&prev_);
    if (prev_ != dev) cudaSetDevice(dev);
  }
  ~DeviceScope() {
    if (prev_ >= 0 && prev_ != dev_) cudaSetDevice(prev_);
  }

 private:
  int dev_ = 0, prev_ = -1;
};

int append_common(ft_kv3* c, int64_t n_pos, const AppendParams& proto, bool packed,
                  cudaStream_t s) {
  FT_CHECK(n_pos >= 0, FT_ERR_SHAPE, "negative position count");
  if (n_pos == 0) return FT_OK;
  {
    // the new slots must fit the ring, and their blocks must be distinct (one
    // CTA per block): a range that wraps onto its own first block grows too
    const int64_t s0 = (c->head + c->len) % c->cap;
    const int64_t nblk = (s0 % kBlk + n_pos + kBlk - 1) / kBlk;
    if (c->len + n_pos > c->cap || nblk > c->cap / kBlk) {
      const int rc = grow(c, c->len + n_pos, s);
      if (rc != FT_OK) return rc;
    }
  }
  AppendParams p = proto;
  p.n_pos = n_pos;
  p.Hkv = c->kv_heads;
  p.cap = c->cap;
  p.nbc = c->cap / kBlk;
  p.s0 = (c->head + c->len) % c->cap;
  p.blocks = c->blocks;
  p.signs = packed ? nullptr : c->signs;
  const int64_t nblk = (p.s0 % kBlk + n_pos + kBlk - 1) / kBlk;
  // a block is touched by one CTA only: the new slots never wrap onto a block
  // that an earlier CTA of this launch also writes
  FT_CHECK(nblk <= p.nbc, FT_ERR_SHAPE, "append spans more blocks than the ring holds");
  dim3 grid((unsigned)nblk, (unsigned)(c->batch * c->kv_heads));
  if (packed)
    kv3_append_kernel<true><<<grid, kD, 0, s>>>(p);
  else
    kv3_append_kernel<false><<<grid, kD, 0, s>>>(p);
  FT_LAUNCH_CHECK();
  c->len += n_pos;
  return FT_OK;
}

// The 128 mode-T signs from SplitMix64(seed) (bit 63 of each draw set -> -1),
// uploaded to a new device array.
cudaError_t upload_signs(uint64_t seed, float** out) {
  std::vector<float> sg(kD);
  uint64_t z = seed;
  for (int i = 0; i < kD; ++i) {
    z += 0x9e3779b97f4a7c15ull;
    uint64_t r = z;
    r = (r ^ (r >> 30)) * 0xbf58476d1ce4e5b9ull;
    r = (r ^ (r >> 27)) * 0x94d049bb133111ebull;
    r ^= r >> 31;
    sg[i] = (r >> 63) ? -1.0f : 1.0f;
  }
  cudaError_t e = cudaMalloc(out, kD * sizeof(float));
  if (e == cudaSuccess) e = cudaMemcpy(*out, sg.data(), kD * sizeof(float), cudaMemcpyHostToDevice);
  return e;
}

RangeParams range_params(const ft_kv3* c, int64_t start, int64_t n) {
  RangeParams p{};
  p.B = c->batch;
  p.Hkv = c->kv_heads;
  p.cap = c->cap;
  p.nbc = c->cap / kBlk;
  p.head = c->head;
  p.start = start;
  p.n = n;
  p.blocks = c->blocks;
  return p;
}

}  // namespace
}  // namespace ft

using namespace ft;

extern "C" {

int ft_kv3_create(ft_ctx* ctx, int64_t batch, int64_t kv_heads, int64_t head_dim, int64_t max_seq,
                  ft_kv3** out) {
  FT_CHECK(ctx && out, FT_ERR_SHAPE, "null argument");
  FT_CHECK(head_dim == kD, FT_ERR_UNSUPPORTED,
           "head_dim must be %d (one quantisation group per head vector)", kD);
  FT_CHECK(batch > 0 && kv_heads > 0 && max_seq > 0, FT_ERR_SHAPE, "bad cache shape");
  DeviceScope scope(ctx->device);
  ft_kv3* c = new ft_kv3();
  c->device = ctx->device;
  c->batch = batch;
  c->kv_heads = kv_heads;
  c->cap = round_up(max_seq, kBlk);
  const size_t recs = (size_t)(batch * kv_heads * (c->cap / kBlk));
  cudaError_t e = cudaMalloc(&c->blocks, recs * kRecBytes);
  // blocks start zeroed (the decode reads whole blocks; slots outside the
  // live range get zero weight whatever they hold)
  if (e == cudaSuccess) e = cudaMemset(c->blocks, 0, recs * kRecBytes);
  if (e != cudaSuccess) {
    cudaFree(c->blocks);
    delete c;
    return fail(e == cudaErrorMemoryAllocation ? FT_ERR_OOM : FT_ERR_GPU,
                "3-bit KV cache allocation failed: %s", cudaGetErrorString(e));
  }
  *out = c;
  return FT_OK;
}

int ft_kv3_create_mode(ft_ctx* ctx, int64_t batch, int64_t kv_heads, int64_t head_dim,
                       int64_t max_seq, int mode, uint64_t seed, ft_kv3** out) {
  FT_CHECK(mode == 0 || mode == 1, FT_ERR_UNSUPPORTED, "mode must be 0 (reference) or 1 (T)");
  int st = ft_kv3_create(ctx, batch, kv_heads, head_dim, max_seq, out);
  if (st != FT_OK || mode == 0) return st;
  ft_kv3* c = *out;
  DeviceScope scope(c->device);
  cudaError_t e = upload_signs(seed, &c->signs);
  if (e != cudaSuccess) {
    ft_kv3_destroy(c);
    *out = nullptr;
    return fail(FT_ERR_GPU, "mode T setup failed: %s", cudaGetErrorString(e));
  }
  c->mode = 1;
  return FT_OK;
}

int ft_kv3_signs(const ft_kv3* c, float* signs_host) {
  FT_CHECK(c && signs_host, FT_ERR_SHAPE, "null argument");
  FT_CHECK(c->signs, FT_ERR_UNSUPPORTED, "the cache is not in mode T");
  DeviceScope scope(c->device);
  FT_CUDA(cudaMemcpy(signs_host, c->signs, kD * sizeof(float), cudaMemcpyDeviceToHost));
  return FT_OK;
}

int ft_kv3_destroy(ft_kv3* c) {
  if (!c) return FT_OK;
  DeviceScope scope(c->device);
  cudaDeviceSynchronize();
  cudaFree(c->blocks);
  if (c->part.ptr) cudaFree(c->part.ptr);
  if (c->signs) cudaFree(c->signs);
  if (c->rot.ptr) cudaFree(c->rot.ptr);
  delete c;
  return FT_OK;
}

int ft_kv3_append(ft_ctx* ctx, ft_kv3* c, int64_t n_pos, const void* k_dev, const void* v_dev,
                  int is_bf16, void* stream) {
  FT_CHECK(ctx && c && (n_pos == 0 || (k_dev && v_dev)), FT_ERR_SHAPE, "null argument");
  DeviceScope scope(c->device);
  AppendParams p{};
  p.k = k_dev;
  p.v = v_dev;
  p.bf16 = is_bf16 ? 1 : 0;
  return append_common(c, n_pos, p, false, static_cast<cudaStream_t>(stream));
}

int ft_kv3_append_packed(ft_ctx* ctx, ft_kv3* c, int64_t n_pos, const uint8_t* k_codes_dev,
                         const float* k_minmax_dev, const uint8_t* v_codes_dev,
                         const float* v_minmax_dev, void* stream) {
  FT_CHECK(ctx && c &&
               (n_pos == 0 || (k_codes_dev && k_minmax_dev && v_codes_dev && v_minmax_dev)),
           FT_ERR_SHAPE, "null argument");
  DeviceScope scope(c->device);
  AppendParams p{};
  p.k = k_codes_dev;
  p.v = v_codes_dev;
  p.kmm_in = k_minmax_dev;
  p.vmm_in = v_minmax_dev;
  return append_common(c, n_pos, p, true, static_cast<cudaStream_t>(stream));
}

int ft_kv3_len(const ft_kv3* c, int64_t* len) {
  FT_CHECK(c && len, FT_ERR_SHAPE, "null argument");
  *len = c->len;
  return FT_OK;
}

int ft_kv3_capacity(const ft_kv3* c, int64_t* cap) {
  FT_CHECK(c && cap, FT_ERR_SHAPE, "null argument");
  *cap = c->cap;
  return FT_OK;
}

int ft_kv3_evict_front(ft_kv3* c, int64_t n) {
  FT_CHECK(c, FT_ERR_SHAPE, "null argument");
  FT_CHECK(n >= 0, FT_ERR_SHAPE, "negative eviction count");
  if (n > c->len) n = c->len;
  c->head = (c->head + n) % c->cap;
  c->len -= n;
  return FT_OK;
}

int ft_kv3_reset(ft_kv3* c) {
  FT_CHECK(c, FT_ERR_SHAPE, "null argument");
  c->len = 0;
  c->head = 0;
  return FT_OK;
}

int ft_kv3_get_range(ft_ctx* ctx, const ft_kv3* c, int64_t start, int64_t end, float* k_out_dev,
                     float* v_out_dev, void* stream) {
  FT_CHECK(ctx && c && k_out_dev && v_out_dev, FT_ERR_SHAPE, "null argument");
  FT_CHECK(0 <= start && start <= end && end <= c->len, FT_ERR_SHAPE,
           "range [%lld, %lld) outside the cache length %lld", (long long)start, (long long)end,
           (long long)c->len);
  const int64_t n = end - start;
  if (n == 0) return FT_OK;
  DeviceScope scope(c->device);
  kv3_dequant_kernel<<<(unsigned)(c->batch * n * c->kv_heads), kD, 0,
                       static_cast<cudaStream_t>(stream)>>>(range_params(c, start, n), k_out_dev,
                                                            v_out_dev, c->signs);
  FT_LAUNCH_CHECK();
  return FT_OK;
}

int ft_kv3_export_range(ft_ctx* ctx, const ft_kv3* c, int64_t start, int64_t end,
                        uint8_t* k_codes_dev, float* k_minmax_dev, uint8_t* v_codes_dev,
                        float* v_minmax_dev, void* stream) {
  FT_CHECK(ctx && c && k_codes_dev && k_minmax_dev && v_codes_dev && v_minmax_dev, FT_ERR_SHAPE,
           "null argument");
  FT_CHECK(0 <= start && start <= end && end <= c->len, FT_ERR_SHAPE,
           "range [%lld, %lld) outside the cache length %lld", (long long)start, (long long)end,
           (long long)c->len);
  const int64_t n = end - start;
  if (n == 0) return FT_OK;
  DeviceScope scope(c->device);
  kv3_export_kernel<<<(unsigned)(c->batch * n * c->kv_heads), 16, 0,
                      static_cast<cudaStream_t>(stream)>>>(range_params(c, start, n), k_codes_dev,
                                                           k_minmax_dev, v_codes_dev,
                                                           v_minmax_dev);
  FT_LAUNCH_CHECK();
  return FT_OK;
}

}  // extern "C"

namespace ft {
namespace {

// Grows a workspace outside stream capture (a capture may only reuse it).
int ensure_ws(Workspace& w, size_t need, cudaStream_t s, const char* what) {
  if (w.bytes >= need) return FT_OK;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (s) cudaStreamIsCapturing(s, &cs);
  FT_CHECK(cs == cudaStreamCaptureStatusNone, FT_ERR_UNSUPPORTED,
           "the %s buffer must grow but the stream is being captured", what);
  if (w.ptr) {
    FT_CUDA(cudaStreamSynchronize(s));
    FT_CUDA(cudaFree(w.ptr));
    w.ptr = nullptr;
    w.bytes = 0;
  }
  FT_CUDA(cudaMalloc(&w.ptr, need));
  w.bytes = need;
  return FT_OK;
}

// Rotates q (mode T), picks the split of the slots, launches the decode and
// the combine.  p carries the cache geometry (ring or paged); p.len is the
// longest sequence.
int launch_decode(ft_ctx* ctx, DecodeParams p, int64_t batch, int64_t kv_heads, int64_t q_heads,
                  const float* signs, Workspace& part, Workspace& rot, const float* q_dev,
                  float scale, float* out_dev, cudaStream_t s) {
  p.q = q_dev;
  if (signs) {
    // mode T: attention runs in the rotated domain
    const int rc = ensure_ws(rot, (size_t)(batch * q_heads * kD) * 4, s, "rotated-query");
    if (rc != FT_OK) return rc;
    kv3_rotate_kernel<<<(unsigned)(batch * q_heads), kD, 0, s>>>(
        q_dev, static_cast<float*>(rot.ptr), signs, 0);
    FT_LAUNCH_CHECK();
    p.q = static_cast<const float*>(rot.ptr);
  }
  p.Hq = q_heads;
  p.Hkv = kv_heads;
  p.G = (int)(q_heads / kv_heads);
  p.hgroups = (p.G + 3) / 4;
  p.nlb = (p.head_off + p.len + kBlk - 1) / kBlk;
  const float sc = scale > 0.0f ? scale : 1.0f / sqrtf((float)kD);
  p.qk_log2 = sc * 1.4426950408889634f;
  p.err = ctx->err_word;
  // split choice: minimise waves x (tiles per CTA + per-CTA overhead); at most
  // 2^15 tiles (2^20 slots, 2^18 per warp) per CTA keeps every int32 digit sum
  // exact (7 * 255 * 2^18 < 2^31)
  const int64_t units = batch * kv_heads * p.hgroups;
  const int64_t ntiles = (p.nlb + kDecWarps - 1) / kDecWarps;
  const int64_t resident = (int64_t)decode_occupancy(ctx->device) * ctx->num_sms;
  int64_t best_cost = INT64_MAX, best_per = ntiles;
  for (int64_t sp = 1; sp <= 256 && sp <= ntiles; ++sp) {
    const int64_t per = ceil_div(ntiles, sp);
    if (per > 32768) continue;
    const int64_t nsp = ceil_div(ntiles, per);
    const int64_t waves = ceil_div(units * nsp, resident);
    const int64_t cost = waves * (per + 2);
    if (cost < best_cost) {
      best_cost = cost;
      best_per = per;
    }
  }
  FT_CHECK(best_per <= 32768, FT_ERR_UNSUPPORTED, "cache too long for one decode launch");
  p.tiles_per = best_per;
  const int64_t nsplit = ceil_div(ntiles, best_per);
  FT_CHECK(nsplit <= 65535 && kv_heads * p.hgroups <= 65535 && batch <= 65535,
           FT_ERR_UNSUPPORTED, "decode grid too large");
  const int rc = ensure_ws(part, (size_t)(batch * q_heads * nsplit * kPart) * 4, s,
                           "decode partials");
  if (rc != FT_OK) return rc;
  p.part = static_cast<float*>(part.ptr);
  dim3 grid((unsigned)nsplit, (unsigned)(kv_heads * p.hgroups), (unsigned)batch);
  kv3_decode_kernel<<<grid, (kDecWarps + 1) * 32, kDecSmem, s>>>(p);
  FT_LAUNCH_CHECK();
  kv3_combine_kernel<<<(unsigned)(batch * q_heads), kD, 0, s>>>(p.part, (int)nsplit, out_dev,
                                                                  signs);
  FT_LAUNCH_CHECK();
  return FT_OK;
}

}  // namespace
}  // namespace ft

extern "C" {

int ft_flash_decode_3bit(ft_ctx* ctx, ft_kv3* c, const float* q_dev, int64_t q_heads, float scale,
                         float* out_dev, void* stream) {
  FT_CHECK(ctx && c && q_dev && out_dev, FT_ERR_SHAPE, "null argument");
  FT_CHECK(q_heads > 0 && q_heads % c->kv_heads == 0, FT_ERR_SHAPE,
           "q_heads (%lld) must be a multiple of kv_heads (%lld)", (long long)q_heads,
           (long long)c->kv_heads);
  FT_CHECK(c->len > 0, FT_ERR_SHAPE, "flash decode over an empty cache");
  FT_CHECK(c->len + kBlk < (int64_t)INT32_MAX - 64, FT_ERR_UNSUPPORTED,
           "cache too long for the decode's 32-bit slot arithmetic");
  DeviceScope scope(c->device);
  DecodeParams p{};
  p.nbc = c->cap / kBlk;
  p.head_off = c->head % kBlk;
  p.head_blk = c->head / kBlk;
  p.len = c->len;
  p.blocks = c->blocks;
  return launch_decode(ctx, p, c->batch, c->kv_heads, q_heads, c->signs, c->part, c->rot, q_dev,
                       scale, out_dev, static_cast<cudaStream_t>(stream));
}

// ---- paged pool
int ft_kvp_create(ft_ctx* ctx, int64_t num_pages, int64_t kv_heads, int64_t head_dim,
                  int64_t page_size, int mode, uint64_t seed, ft_kvp** out) {
  FT_CHECK(ctx && out, FT_ERR_SHAPE, "null argument");
  *out = nullptr;
  FT_CHECK(head_dim == kD, FT_ERR_UNSUPPORTED, "head_dim %lld: only 128 is supported",
           (long long)head_dim);
  FT_CHECK(page_size == kBlk, FT_ERR_UNSUPPORTED, "page_size %lld: only %d is supported",
           (long long)page_size, kBlk);
  FT_CHECK(num_pages > 0 && num_pages < INT32_MAX && kv_heads > 0 && kv_heads <= 65535,
           FT_ERR_SHAPE, "bad pool shape (%lld pages, %lld kv heads)", (long long)num_pages,
           (long long)kv_heads);
  FT_CHECK(mode == 0 || mode == 1, FT_ERR_UNSUPPORTED, "mode must be 0 (reference) or 1 (T)");
  DeviceScope scope(ctx->device);
  ft_kvp* c = new ft_kvp();
  c->device = ctx->device;
  c->n_pages = num_pages;
  c->kv_heads = kv_heads;
  c->mode = mode;
  const size_t bytes = (size_t)(num_pages * kv_heads) * kRecBytes;
  cudaError_t e = cudaMalloc(&c->blocks, bytes);
  if (e == cudaSuccess) e = cudaMemset(c->blocks, 0, bytes);
  if (e == cudaSuccess && mode == 1) e = upload_signs(seed, &c->signs);
  if (e != cudaSuccess) {
    ft_kvp_destroy(c);
    return fail(e == cudaErrorMemoryAllocation ? FT_ERR_OOM : FT_ERR_GPU,
                "page pool of %lld pages failed: %s", (long long)num_pages, cudaGetErrorString(e));
  }
  *out = c;
  return FT_OK;
}

int ft_kvp_destroy(ft_kvp* c) {
  if (!c) return FT_OK;
  DeviceScope scope(c->device);
  cudaFree(c->blocks);
  if (c->signs) cudaFree(c->signs);
  if (c->part.ptr) cudaFree(c->part.ptr);
  if (c->rot.ptr) cudaFree(c->rot.ptr);
  delete c;
  return FT_OK;
}

int ft_kvp_signs(const ft_kvp* c, float* signs_host) {
  FT_CHECK(c && signs_host, FT_ERR_SHAPE, "null argument");
  FT_CHECK(c->signs, FT_ERR_UNSUPPORTED, "the pool is not in mode T");
  DeviceScope scope(c->device);
  FT_CUDA(cudaMemcpy(signs_host, c->signs, kD * sizeof(float), cudaMemcpyDeviceToHost));
  return FT_OK;
}

static int kvp_append(ft_ctx* ctx, ft_kvp* c, int64_t batch, int64_t n_pos,
                      const int32_t* tables_dev, int64_t table_stride,
                      const int32_t* start_pos_dev, AppendParams p, bool packed, void* stream) {
  FT_CHECK(ctx && c && tables_dev && start_pos_dev, FT_ERR_SHAPE, "null argument");
  FT_CHECK(batch >= 0 && batch <= 65535 && n_pos >= 0 && table_stride > 0, FT_ERR_SHAPE,
           "bad append shape (batch %lld, %lld positions, table stride %lld)", (long long)batch,
           (long long)n_pos, (long long)table_stride);
  if (batch == 0 || n_pos == 0) return FT_OK;
  FT_CHECK(n_pos <= table_stride * kBlk, FT_ERR_SHAPE,
           "%lld positions do not fit a block table of %lld pages", (long long)n_pos,
           (long long)table_stride);
  DeviceScope scope(c->device);
  p.n_pos = n_pos;
  p.Hkv = c->kv_heads;
  p.blocks = c->blocks;
  p.signs = packed ? nullptr : c->signs;
  p.table = tables_dev;
  p.pos0 = start_pos_dev;
  p.tstride = table_stride;
  p.n_pages = c->n_pages;
  p.err = ctx->err_word;
  const int64_t nblk = (kBlk - 1 + n_pos + kBlk - 1) / kBlk;  // most blocks one sequence touches
  dim3 grid((unsigned)nblk, (unsigned)(batch * c->kv_heads));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (packed)
    kv3_append_kernel<true><<<grid, kD, 0, s>>>(p);
  else
    kv3_append_kernel<false><<<grid, kD, 0, s>>>(p);
  FT_LAUNCH_CHECK();
  return FT_OK;
}

int ft_kvp_append(ft_ctx* ctx, ft_kvp* c, int64_t batch, int64_t n_pos, const int32_t* tables_dev,
                  int64_t table_stride, const int32_t* start_pos_dev, const void* k_dev,
                  const void* v_dev, int is_bf16, void* stream) {
  FT_CHECK(n_pos == 0 || batch == 0 || (k_dev && v_dev), FT_ERR_SHAPE, "null argument");
  AppendParams p{};
  p.k = k_dev;
  p.v = v_dev;
  p.bf16 = is_bf16 ? 1 : 0;
  return kvp_append(ctx, c, batch, n_pos, tables_dev, table_stride, start_pos_dev, p, false,
                    stream);
}

int ft_kvp_append_packed(ft_ctx* ctx, ft_kvp* c, int64_t batch, int64_t n_pos,
                         const int32_t* tables_dev, int64_t table_stride,
                         const int32_t* start_pos_dev, const uint8_t* k_codes_dev,
                         const float* k_minmax_dev, const uint8_t* v_codes_dev,
                         const float* v_minmax_dev, void* stream) {
  FT_CHECK(n_pos == 0 || batch == 0 ||
               (k_codes_dev && k_minmax_dev && v_codes_dev && v_minmax_dev),
           FT_ERR_SHAPE, "null argument");
  AppendParams p{};
  p.k = k_codes_dev;
  p.v = v_codes_dev;
  p.kmm_in = k_minmax_dev;
  p.vmm_in = v_minmax_dev;
  return kvp_append(ctx, c, batch, n_pos, tables_dev, table_stride, start_pos_dev, p, true,
                    stream);
}

int ft_kvp_copy_pages(ft_ctx* ctx, ft_kvp* c, int64_t n, const int32_t* src_pages_host,
                      const int32_t* dst_pages_host, void* stream) {
  FT_CHECK(ctx && c && (n == 0 || (src_pages_host && dst_pages_host)), FT_ERR_SHAPE,
           "null argument");
  const size_t pb = (size_t)c->kv_heads * kRecBytes;
  for (int64_t i = 0; i < n; ++i) {
    const int64_t a = src_pages_host[i], b = dst_pages_host[i];
    FT_CHECK(a >= 0 && a < c->n_pages && b >= 0 && b < c->n_pages, FT_ERR_SHAPE,
             "page copy %lld -> %lld outside the pool of %lld pages", (long long)a, (long long)b,
             (long long)c->n_pages);
  }
  DeviceScope scope(c->device);
  uint8_t* base = reinterpret_cast<uint8_t*>(c->blocks);
  for (int64_t i = 0; i < n; ++i) {
    if (src_pages_host[i] == dst_pages_host[i]) continue;
    FT_CUDA(cudaMemcpyAsync(base + dst_pages_host[i] * pb, base + src_pages_host[i] * pb, pb,
                            cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream)));
  }
  return FT_OK;
}

static int kvp_range(ft_ctx* ctx, const ft_kvp* c, int64_t batch, const int32_t* tables_dev,
                     int64_t table_stride, int64_t start, int64_t end, RangeParams* p) {
  FT_CHECK(ctx && c && tables_dev, FT_ERR_SHAPE, "null argument");
  FT_CHECK(batch >= 0 && table_stride > 0 && 0 <= start && start <= end &&
               end <= table_stride * kBlk,
           FT_ERR_SHAPE, "range [%lld, %lld) outside block tables of %lld pages",
           (long long)start, (long long)end, (long long)table_stride);
  *p = RangeParams{};
  p->B = batch;
  p->Hkv = c->kv_heads;
  p->cap = 1;
  p->nbc = 1;
  p->start = start;
  p->n = end - start;
  p->blocks = c->blocks;
  p->table = tables_dev;
  p->tstride = table_stride;
  p->n_pages = c->n_pages;
  p->err = ctx->err_word;
  return FT_OK;
}

int ft_kvp_get_range(ft_ctx* ctx, const ft_kvp* c, int64_t batch, const int32_t* tables_dev,
                     int64_t table_stride, int64_t start, int64_t end, float* k_out_dev,
                     float* v_out_dev, void* stream) {
  RangeParams p;
  const int rc = kvp_range(ctx, c, batch, tables_dev, table_stride, start, end, &p);
  if (rc != FT_OK) return rc;
  FT_CHECK(k_out_dev && v_out_dev, FT_ERR_SHAPE, "null argument");
  if (p.n == 0 || batch == 0) return FT_OK;
  DeviceScope scope(c->device);
  kv3_dequant_kernel<<<(unsigned)(batch * p.n * c->kv_heads), kD, 0,
                       static_cast<cudaStream_t>(stream)>>>(p, k_out_dev, v_out_dev, c->signs);
  FT_LAUNCH_CHECK();
  return FT_OK;
}

int ft_kvp_export_range(ft_ctx* ctx, const ft_kvp* c, int64_t batch, const int32_t* tables_dev,
                        int64_t table_stride, int64_t start, int64_t end, uint8_t* k_codes_dev,
                        float* k_minmax_dev, uint8_t* v_codes_dev, float* v_minmax_dev,
                        void* stream) {
  RangeParams p;
  const int rc = kvp_range(ctx, c, batch, tables_dev, table_stride, start, end, &p);
  if (rc != FT_OK) return rc;
  FT_CHECK(k_codes_dev && k_minmax_dev && v_codes_dev && v_minmax_dev, FT_ERR_SHAPE,
           "null argument");
  if (p.n == 0 || batch == 0) return FT_OK;
  DeviceScope scope(c->device);
  kv3_export_kernel<<<(unsigned)(batch * p.n * c->kv_heads), 16, 0,
                      static_cast<cudaStream_t>(stream)>>>(p, k_codes_dev, k_minmax_dev,
                                                           v_codes_dev, v_minmax_dev);
  FT_LAUNCH_CHECK();
  return FT_OK;
}

int ft_kvp_flash_decode(ft_ctx* ctx, ft_kvp* c, int64_t batch, const int32_t* tables_dev,
                        int64_t table_stride, const int32_t* seq_lens_dev, int64_t max_seq_len,
                        const float* q_dev, int64_t q_heads, float scale, float* out_dev,
                        void* stream) {
  FT_CHECK(ctx && c && tables_dev && seq_lens_dev && q_dev && out_dev, FT_ERR_SHAPE,
           "null argument");
  FT_CHECK(q_heads > 0 && q_heads % c->kv_heads == 0, FT_ERR_SHAPE,
           "q_heads (%lld) must be a multiple of kv_heads (%lld)", (long long)q_heads,
           (long long)c->kv_heads);
  FT_CHECK(batch > 0 && max_seq_len > 0 && table_stride > 0 &&
               max_seq_len <= table_stride * kBlk,
           FT_ERR_SHAPE, "bad decode shape (batch %lld, max_seq_len %lld, table stride %lld)",
           (long long)batch, (long long)max_seq_len, (long long)table_stride);
  FT_CHECK(max_seq_len + kBlk < (int64_t)INT32_MAX - 64, FT_ERR_UNSUPPORTED,
           "sequence too long for the decode's 32-bit slot arithmetic");
  DeviceScope scope(c->device);
  DecodeParams p{};
  p.nbc = 1;
  p.len = max_seq_len;
  p.blocks = c->blocks;
  p.table = tables_dev;
  p.seq_lens = seq_lens_dev;
  p.tstride = table_stride;
  p.n_pages = c->n_pages;
  return launch_decode(ctx, p, batch, c->kv_heads, q_heads, c->signs, c->part, c->rot, q_dev,
                       scale, out_dev, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
