/*
 * ferris_oracle.c -- CPU restatement of FerrisRes's ternary hot path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker and the timed CPU baseline); the
 * product never links it.  Compiled with -ffp-contract=off so that `a += b * c`
 * rounds twice, exactly as Rust (which never contracts to FMA) does.
 *
 * Reference: shift/FerrisRes v0.2.3.  Each function cites the file:line that it
 * restates.  Parity is pinned by tests/test_oracle_kats.py against the
 * reference's own unit-test known answers.
 */
#include "ferris_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ------------------------------------------------------------------------ */
/* tiny parallel-for: workers pull item indices from an atomic counter, like  */
/* rayon's par_chunks_mut work distribution (the order of items never changes */
/* any single item's arithmetic).                                             */
/* ------------------------------------------------------------------------ */
typedef void (*fo_item_fn)(void* ctx, size_t item);
typedef struct {
  fo_item_fn fn;
  void* ctx;
  size_t n;
  atomic_size_t next;
} fo_pool_job;

static void* fo_worker(void* p) {
  fo_pool_job* j = (fo_pool_job*)p;
  for (;;) {
    size_t i = atomic_fetch_add(&j->next, 1);
    if (i >= j->n) break;
    j->fn(j->ctx, i);
  }
  return NULL;
}

int fo_num_threads(int requested) {
  if (requested > 0) return requested;
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

/* Persistent worker threads (rayon's global pool is persistent too, so a timed
 * call pays no thread creation).  Workers sleep on a condition variable and
 * wake for each job; the calling thread works as well.  One job at a time. */
typedef struct {
  pthread_mutex_t mu;
  pthread_cond_t start, done;
  pthread_mutex_t call_mu; /* serialises callers from several host threads */
  int nworkers;            /* threads created so far */
  int want;                /* workers 0..want-1 take part in the current job */
  int finished;            /* of those, how many are done */
  unsigned gen;            /* job generation */
  fo_pool_job* job;
} fo_pool;

static fo_pool g_pool = {PTHREAD_MUTEX_INITIALIZER, PTHREAD_COND_INITIALIZER,
                         PTHREAD_COND_INITIALIZER, PTHREAD_MUTEX_INITIALIZER, 0, 0, 0, 0, NULL};

typedef struct {
  int id;
  unsigned born; /* generation before the first job this thread may take */
} fo_thread_arg;

static void* fo_pool_thread(void* arg) {
  const fo_thread_arg a = *(const fo_thread_arg*)arg;
  free(arg);
  const int id = a.id;
  unsigned seen = a.born;
  pthread_mutex_lock(&g_pool.mu);
  for (;;) {
    while (g_pool.gen == seen) pthread_cond_wait(&g_pool.start, &g_pool.mu);
    seen = g_pool.gen;
    if (id >= g_pool.want) continue;
    fo_pool_job* job = g_pool.job;
    pthread_mutex_unlock(&g_pool.mu);
    fo_worker(job);
    pthread_mutex_lock(&g_pool.mu);
    if (++g_pool.finished == g_pool.want) pthread_cond_signal(&g_pool.done);
  }
  return NULL;
}

static void fo_parallel_for(size_t n, int nthreads, fo_item_fn fn, void* ctx) {
  int t = fo_num_threads(nthreads);
  if ((size_t)t > n) t = (int)n;
  fo_pool_job job;
  job.fn = fn;
  job.ctx = ctx;
  job.n = n;
  atomic_init(&job.next, 0);
  if (t <= 1) {
    fo_worker(&job);
    return;
  }
  pthread_mutex_lock(&g_pool.call_mu);
  pthread_mutex_lock(&g_pool.mu);
  while (g_pool.nworkers < t - 1) {
    pthread_t th;
    fo_thread_arg* a = (fo_thread_arg*)malloc(sizeof(fo_thread_arg));
    if (!a) break;
    a->id = g_pool.nworkers;
    a->born = g_pool.gen;
    if (pthread_create(&th, NULL, fo_pool_thread, a) != 0) {
      free(a);
      break;
    }
    pthread_detach(th);
    ++g_pool.nworkers;
  }
  g_pool.want = g_pool.nworkers < t - 1 ? g_pool.nworkers : t - 1;
  g_pool.finished = 0;
  g_pool.job = &job;
  ++g_pool.gen;
  pthread_cond_broadcast(&g_pool.start);
  pthread_mutex_unlock(&g_pool.mu);
  fo_worker(&job);
  pthread_mutex_lock(&g_pool.mu);
  while (g_pool.finished < g_pool.want) pthread_cond_wait(&g_pool.done, &g_pool.mu);
  g_pool.job = NULL;
  pthread_mutex_unlock(&g_pool.mu);
  pthread_mutex_unlock(&g_pool.call_mu);
}

/* ------------------------------------------------------------------------ */
/* codes: src/model/ternary.rs:134-179                                      */
/* ------------------------------------------------------------------------ */
static const int8_t TERNARY_DECODE[4] = {-1, 0, 1, 0}; /* ternary.rs:138 */

void fo_pack_ternary(const int8_t* values, size_t n, uint8_t* packed) {
  size_t nb = (n + 3) / 4;
  memset(packed, 0, nb);
  for (size_t i = 0; i < n; ++i) {
    uint8_t code;
    switch (values[i]) { /* ternary.rs:149-154; out of range -> 0 */
      case -1: code = 0; break;
      case 1: code = 2; break;
      default: code = 1; break;
    }
    packed[i / 4] |= (uint8_t)(code << ((i % 4) * 2));
  }
}

void fo_unpack_ternary(const uint8_t* packed, size_t n, int8_t* values) {
  for (size_t i = 0; i < n; ++i) values[i] = TERNARY_DECODE[(packed[i / 4] >> ((i % 4) * 2)) & 3];
}

/* ternary.rs:1317-1328: missing bytes read as 0 */
void fo_pack_ternary_u32(const uint8_t* p, size_t n_bytes, size_t total_values, uint32_t* out) {
  size_t nw = (total_values + 15) / 16;
  for (size_t i = 0; i < nw; ++i) {
    uint32_t w = 0;
    for (int b = 0; b < 4; ++b) {
      size_t idx = i * 4 + (size_t)b;
      uint32_t v = idx < n_bytes ? p[idx] : 0u;
      w |= v << (8 * b);
    }
    out[i] = w;
  }
}

/* src/compute/kernels/ternary_matmul.rs:267-291 (WGSL test packer) */
void fo_pack_ternary_rows_u32(const int8_t* values, size_t rows, size_t cols, uint32_t* out) {
  size_t cp = (cols + 15) / 16;
  for (size_t r = 0; r < rows; ++r)
    for (size_t p = 0; p < cp; ++p) {
      uint32_t w = 0;
      for (size_t b = 0; b < 16; ++b) {
        size_t c = p * 16 + b;
        if (c >= cols) break;
        int8_t v = values[r * cols + c];
        uint32_t code = v == -1 ? 0u : v == 0 ? 1u : v == 1 ? 2u : 3u;
        w |= code << (b * 2);
      }
      out[r * cp + p] = w;
    }
}

/* Rust's `f32 as i32`: saturating, NaN -> 0 (C's cast is undefined there). */
static int fo_as_i32(float r) {
  if (r != r) return 0;
  if (r >= 2147483648.0f) return 2147483647;
  if (r <= -2147483648.0f) return (int)(-2147483647 - 1);
  return (int)r;
}

/* src/model/ternary.rs:31-57 */
float fo_quantize_ternary(const float* w, size_t n, int8_t* q) {
  if (n == 0) return 0.0f;
  float sum_abs = 0.0f;
  for (size_t i = 0; i < n; ++i) sum_abs += fabsf(w[i]);
  const float ABSMEAN_NORM = 0.7978845608f; /* ternary.rs:15 */
  float alpha = sum_abs > 0.0f ? (sum_abs / (float)n) / ABSMEAN_NORM : 1.0f;
  float inv = 1.0f / alpha;
  for (size_t i = 0; i < n; ++i) {
    float r = roundf(w[i] * inv); /* f32::round: half away from zero */
    int ri = fo_as_i32(r);         /* `as i32` */
    q[i] = (int8_t)(ri < -1 ? -1 : ri > 1 ? 1 : ri);
  }
  return alpha;
}

/* ------------------------------------------------------------------------ */
/* dense matmuls                                                            */
/* ------------------------------------------------------------------------ */
static float pos_neg_row(const int8_t* wrow, const float* x, size_t k) {
  /* ternary.rs:316-323: split positive / negative accumulators */
  float pos = 0.0f, neg = 0.0f;
  for (size_t j = 0; j < k; ++j) {
    int8_t w = wrow[j];
    float v = x[j];
    pos += w > 0 ? v : 0.0f;
    neg += w < 0 ? v : 0.0f;
  }
  return pos - neg;
}

void fo_ternary_matmul(const int8_t* t, float scale, const float* x, size_t out_rows,
                       size_t in_cols, size_t seq, float* y) {
  for (size_t s = 0; s < seq; ++s)
    for (size_t r = 0; r < out_rows; ++r)
      y[s * out_rows + r] = scale * pos_neg_row(t + r * in_cols, x + s * in_cols, in_cols);
}

/* src/model/ternary.rs:401-464.  Byte index is flat over the whole matrix
 * ((row_offset + q*4)/4); the remainder reads the low bits of the next byte,
 * exactly as the reference does. */
void fo_ternary_matmul_packed(const uint8_t* packed, float scale, const float* x,
                              size_t out_rows, size_t in_cols, size_t seq, float* y) {
  size_t full_quads = in_cols / 4, rem = in_cols % 4;
  for (size_t s = 0; s < seq; ++s) {
    const float* xr = x + s * in_cols;
    for (size_t r = 0; r < out_rows; ++r) {
      size_t row_offset = r * in_cols;
      float sum = 0.0f;
      for (size_t q = 0; q < full_quads; ++q) {
        uint8_t b = packed[(row_offset + q * 4) / 4];
        for (size_t bp = 0; bp < 4; ++bp) {
          float sg = (float)TERNARY_DECODE[(b >> (bp * 2)) & 3];
          sum += sg * xr[q * 4 + bp];
        }
      }
      if (rem > 0) {
        uint8_t b = packed[(row_offset + full_quads * 4) / 4];
        for (size_t bp = 0; bp < rem; ++bp) {
          float sg = (float)TERNARY_DECODE[(b >> (bp * 2)) & 3];
          sum += sg * xr[full_quads * 4 + bp];
        }
      }
      y[s * out_rows + r] = scale * sum;
    }
  }
}

/* src/model/ternary.rs:591-633 */
void fo_ternary_matmul_decode(const int8_t* t, float scale, const float* x, size_t out_rows,
                              size_t in_cols, float* y) {
  for (size_t r = 0; r < out_rows; ++r) {
    const int8_t* w = t + r * in_cols;
    float sum = 0.0f;
    size_t chunks = in_cols / 8;
    for (size_t c = 0; c < chunks; ++c) {
      size_t b = c * 8;
      for (size_t u = 0; u < 8; ++u) sum += (float)w[b + u] * x[b + u];
    }
    for (size_t j = chunks * 8; j < in_cols; ++j) sum += (float)w[j] * x[j];
    y[r] = scale * sum;
  }
}

/* src/model/ternary.rs:541-579: one scale per block of block_size columns,
 * shared by every row; per block an fp32 block_sum of w * x, then
 * sum += alpha * block_sum. */
void fo_ternary_matmul_blocked(const int8_t* t, const float* scales, size_t block_size,
                               const float* x, size_t out_rows, size_t in_cols, size_t seq,
                               float* y) {
  const size_t nb = (in_cols + block_size - 1) / block_size;
  for (size_t s = 0; s < seq; ++s) {
    const float* xr = x + s * in_cols;
    for (size_t r = 0; r < out_rows; ++r) {
      const int8_t* w = t + r * in_cols;
      float sum = 0.0f;
      for (size_t b = 0; b < nb; ++b) {
        const size_t c0 = b * block_size;
        size_t c1 = c0 + block_size;
        if (c1 > in_cols) c1 = in_cols;
        float block_sum = 0.0f;
        for (size_t j = c0; j < c1; ++j) block_sum += (float)w[j] * xr[j];
        sum += scales[b] * block_sum;
      }
      y[s * out_rows + r] = sum;
    }
  }
}

/* src/model/ternary.rs:76-110: flat blocks of block_size elements, absmean
 * alpha per block (sequential f32 sum of |w|), round half away, clamp. */
void fo_quantize_ternary_blocked(const float* w, size_t n, size_t block_size, int8_t* q,
                                 float* scales) {
  const float ABSMEAN_NORM = 0.7978845608f; /* ternary.rs:15 */
  const size_t nb = (n + block_size - 1) / block_size;
  for (size_t b = 0; b < nb; ++b) {
    const size_t s0 = b * block_size;
    size_t s1 = s0 + block_size;
    if (s1 > n) s1 = n;
    float sum_abs = 0.0f;
    for (size_t i = s0; i < s1; ++i) sum_abs += fabsf(w[i]);
    const float alpha = sum_abs > 0.0f ? (sum_abs / (float)(s1 - s0)) / ABSMEAN_NORM : 1.0f;
    scales[b] = alpha;
    const float inv = 1.0f / alpha;
    for (size_t i = s0; i < s1; ++i) {
      const int r = fo_as_i32(roundf(w[i] * inv));
      q[i] = (int8_t)(r < -1 ? -1 : r > 1 ? 1 : r);
    }
  }
}

/* src/model/ternary.rs:681-707: per row, the columns holding +1 and -1, in
 * column order.  Written as CSR: pos_off/neg_off [out_rows + 1], pos_idx /
 * neg_idx (capacity out_rows * in_cols each). */
void fo_ternary_sparse_indices(const int8_t* t, size_t out_rows, size_t in_cols, int64_t* pos_off,
                               int64_t* pos_idx, int64_t* neg_off, int64_t* neg_idx) {
  int64_t np = 0, nn = 0;
  for (size_t r = 0; r < out_rows; ++r) {
    pos_off[r] = np;
    neg_off[r] = nn;
    for (size_t j = 0; j < in_cols; ++j) {
      if (t[r * in_cols + j] == 1) pos_idx[np++] = (int64_t)j;
      else if (t[r * in_cols + j] == -1) neg_idx[nn++] = (int64_t)j;
    }
  }
  pos_off[out_rows] = np;
  neg_off[out_rows] = nn;
}

/* src/model/ternary.rs:647-672: sum += x[j] over the row's +1 list, then
 * sum -= x[j] over its -1 list, y = scale * sum. */
void fo_ternary_matmul_sparse_decode(const int64_t* pos_off, const int64_t* pos_idx,
                                     const int64_t* neg_off, const int64_t* neg_idx, float scale,
                                     const float* x, size_t out_rows, float* y) {
  for (size_t r = 0; r < out_rows; ++r) {
    float sum = 0.0f;
    for (int64_t i = pos_off[r]; i < pos_off[r + 1]; ++i) sum += x[pos_idx[i]];
    for (int64_t i = neg_off[r]; i < neg_off[r + 1]; ++i) sum -= x[neg_idx[i]];
    y[r] = scale * sum;
  }
}

/* src/training/bit_moe.rs:243-262 (ScaleSync::PerBlock): q = +1 if v / alpha > 0.5,
 * -1 if < -0.5, else 0; all 0 when alpha < 1e-10.  v: bf16 bit patterns. */
void fo_bitmoe_requantize(const uint16_t* shadow_bf16, size_t n, float alpha, int8_t* q) {
  for (size_t i = 0; i < n; ++i) {
    union {
      uint32_t u;
      float f;
    } c;
    c.u = (uint32_t)shadow_bf16[i] << 16;
    if (alpha < 1e-10f) {
      q[i] = 0;
      continue;
    }
    const float nv = c.f / alpha;
    q[i] = nv > 0.5f ? 1 : (nv < -0.5f ? -1 : 0);
  }
}

/* src/training/bit_moe.rs:210-241: total_abs += |v| as f64 over every shadow in
 * order, alpha = (total / count) as f32.  Returns 0 (alpha unchanged) when empty. */
int fo_bitmoe_recompute_alpha(const uint16_t* const* shadows, const size_t* counts, size_t n,
                              float* alpha) {
  double total = 0.0;
  size_t count = 0;
  for (size_t b = 0; b < n; ++b)
    for (size_t i = 0; i < counts[b]; ++i) {
      union {
        uint32_t u;
        float f;
      } c;
      c.u = (uint32_t)shadows[b][i] << 16;
      total += (double)fabsf(c.f);
      ++count;
    }
  if (count == 0) return 0;
  *alpha = (float)(total / (double)count);
  return 1;
}

/* src/model/ternary.rs:471-529, per-row scales */
typedef struct {
  const uint8_t* packed;
  const float* rs;
  const float* x;
  size_t out_rows, in_cols, batch;
  float* y;
} fo_pp_ctx;

static void fo_pp_item(void* vctx, size_t batch_idx) {
  fo_pp_ctx* c = (fo_pp_ctx*)vctx;
  size_t start = batch_idx * c->batch;
  size_t end = start + c->batch;
  if (end > c->out_rows) end = c->out_rows;
  size_t full_quads = c->in_cols / 4, rem = c->in_cols % 4;
  size_t row_bytes = (c->in_cols + 3) / 4;
  for (size_t row = start; row < end; ++row) {
    const uint8_t* p = c->packed + row * row_bytes;
    float sum = 0.0f;
    for (size_t q = 0; q < full_quads; ++q) {
      uint8_t b = p[q];
      float s0 = (float)TERNARY_DECODE[b & 3];
      float s1 = (float)TERNARY_DECODE[(b >> 2) & 3];
      float s2 = (float)TERNARY_DECODE[(b >> 4) & 3];
      float s3 = (float)TERNARY_DECODE[(b >> 6) & 3];
      const float* xb = c->x + q * 4;
      /* ternary.rs:511-514: one 4-term expression per byte, added to sum */
      sum += s0 * xb[0] + s1 * xb[1] + s2 * xb[2] + s3 * xb[3];
    }
    if (rem > 0) {
      uint8_t b = p[full_quads];
      for (size_t bp = 0; bp < rem; ++bp)
        sum += (float)TERNARY_DECODE[(b >> (bp * 2)) & 3] * c->x[full_quads * 4 + bp];
    }
    c->y[row] = c->rs[row] * sum;
  }
}

void fo_ternary_matmul_packed_parallel_rows(const uint8_t* packed, const float* row_scales,
                                            const float* x, size_t out_rows, size_t in_cols,
                                            float* y, int nthreads) {
  fo_pp_ctx c = {packed, row_scales, x, out_rows, in_cols, 0, y};
  c.batch = out_rows / 32 > 0 ? out_rows / 32 : 1; /* ternary.rs:481 */
  size_t nbatches = (out_rows + c.batch - 1) / c.batch;
  fo_parallel_for(nbatches, nthreads, fo_pp_item, &c);
}

void fo_gpu_ternary_mm_cpu(const uint32_t* packed, const float* scales, const float* x,
                           size_t seq, size_t in_cols, size_t out_rows, float* y) {
  size_t cp = (in_cols + 15) / 16;
  for (size_t t = 0; t < seq; ++t)
    for (size_t row = 0; row < out_rows; ++row) {
      float sum = 0.0f;
      for (size_t c = 0; c < cp; ++c) {
        uint32_t p = packed[row * cp + c];
        for (uint32_t bit = 0; bit < 16; ++bit) {
          size_t col = c * 16 + bit;
          if (col >= in_cols) break;
          uint32_t code = (p >> (bit * 2)) & 3u;
          float v = x[t * in_cols + col];
          if (code == 0) sum -= v;
          else if (code == 2) sum += v;
        }
      }
      y[t * out_rows + row] = sum * scales[row];
    }
}

/* src/model/ternary.rs:333-389 */
typedef struct {
  const int8_t* t;
  float scale;
  const float* x;
  size_t out_rows, in_cols, batch;
  float* y;
} fo_tp_ctx;

static void fo_tp_rows_item(void* v, size_t bi) {
  fo_tp_ctx* c = (fo_tp_ctx*)v;
  size_t s = bi * c->batch, e = s + c->batch;
  if (e > c->out_rows) e = c->out_rows;
  for (size_t r = s; r < e; ++r) c->y[r] = c->scale * pos_neg_row(c->t + r * c->in_cols, c->x, c->in_cols);
}

static void fo_tp_tok_item(void* v, size_t s) {
  fo_tp_ctx* c = (fo_tp_ctx*)v;
  const float* xr = c->x + s * c->in_cols;
  for (size_t r = 0; r < c->out_rows; ++r)
    c->y[s * c->out_rows + r] = c->scale * pos_neg_row(c->t + r * c->in_cols, xr, c->in_cols);
}

void fo_ternary_matmul_parallel(const int8_t* t, float scale, const float* x, size_t out_rows,
                                size_t in_cols, size_t seq, float* y, int nthreads) {
  fo_tp_ctx c = {t, scale, x, out_rows, in_cols, 0, y};
  if (seq <= 1) {
    c.batch = out_rows / 32 > 0 ? out_rows / 32 : 1;
    fo_parallel_for((out_rows + c.batch - 1) / c.batch, nthreads, fo_tp_rows_item, &c);
  } else {
    fo_parallel_for(seq, nthreads, fo_tp_tok_item, &c);
  }
}

/* ------------------------------------------------------------------------ */
/* int8 activation mode                                                     */
/* ------------------------------------------------------------------------ */
void fo_quantize_absmax_i8(const float* x, size_t seq, size_t cols, int8_t* q, float* sx) {
  for (size_t s = 0; s < seq; ++s) {
    const float* xr = x + s * cols;
    float amax = 0.0f;
    for (size_t j = 0; j < cols; ++j) {
      float a = fabsf(xr[j]);
      amax = a > amax ? a : amax;
    }
    if (amax == 0.0f) {
      sx[s] = 1.0f;
      memset(q + s * cols, 0, cols);
      continue;
    }
    sx[s] = amax / 127.0f;
    float inv = 127.0f / amax;
    for (size_t j = 0; j < cols; ++j) {
      float r = roundf(xr[j] * inv);
      r = r < -127.0f ? -127.0f : r > 127.0f ? 127.0f : r;
      q[s * cols + j] = (int8_t)r;
    }
  }
}

typedef struct {
  const int8_t* t;
  const int8_t* q;
  const float* sx;
  const float* sw;
  size_t in_cols, out_rows;
  float* y;
  int via_f32;
} fo_i8_ctx;

static void fo_i8_item(void* v, size_t s) {
  fo_i8_ctx* c = (fo_i8_ctx*)v;
  const int8_t* qr = c->q + s * c->in_cols;
  float* xf = NULL;
  if (c->via_f32) {
    xf = (float*)malloc(sizeof(float) * c->in_cols);
    for (size_t j = 0; j < c->in_cols; ++j) xf[j] = (float)qr[j];
  }
  for (size_t n = 0; n < c->out_rows; ++n) {
    const int8_t* w = c->t + n * c->in_cols;
    float accf;
    if (c->via_f32) {
      accf = 1.0f * pos_neg_row(w, xf, c->in_cols); /* exact: |sum| < 2^24 */
    } else {
      int32_t acc = 0;
      for (size_t j = 0; j < c->in_cols; ++j) acc += (int32_t)w[j] * (int32_t)qr[j];
      accf = (float)acc;
    }
    c->y[s * c->out_rows + n] = (accf * c->sx[s]) * c->sw[n];
  }
  free(xf);
}

void fo_ternary_matmul_i8(const int8_t* t, const int8_t* q, const float* sx, const float* sw,
                          size_t seq, size_t in_cols, size_t out_rows, float* y, int nthreads) {
  fo_i8_ctx c = {t, q, sx, sw, in_cols, out_rows, y, 0};
  fo_parallel_for(seq, nthreads, fo_i8_item, &c);
}

void fo_ternary_matmul_i8_via_f32(const int8_t* t, const int8_t* q, const float* sx,
                                  const float* sw, size_t seq, size_t in_cols, size_t out_rows,
                                  float* y, int nthreads) {
  fo_i8_ctx c = {t, q, sx, sw, in_cols, out_rows, y, 1};
  fo_parallel_for(seq, nthreads, fo_i8_item, &c);
}

/* ------------------------------------------------------------------------ */
/* 2:4 sparse, host layout: src/model/sparse_ternary.rs                     */
/* ------------------------------------------------------------------------ */
static const uint8_t SPARSE_PATTERN[6][2] = {{0, 1}, {0, 2}, {0, 3}, {1, 2}, {1, 3}, {2, 3}};

static int find_pattern(uint8_t p0, uint8_t p1) {
  for (int i = 0; i < 6; ++i)
    if (SPARSE_PATTERN[i][0] == p0 && SPARSE_PATTERN[i][1] == p1) return i;
  return -1;
}

/* sparse_ternary.rs:78-150 */
void fo_sparse_from_ternary(const int8_t* t, size_t rows, size_t cols, uint8_t* patterns,
                            uint8_t* signs) {
  size_t ng = rows * cols / 4;
  memset(patterns, 0, (ng + 1) / 2);
  memset(signs, 0, (ng + 3) / 4);
  for (size_t g = 0; g < ng; ++g) {
    const int8_t* v = t + g * 4;
    size_t idx[4] = {0, 1, 2, 3};
    /* stable sort by |v| descending (Rust slice::sort_by is stable) */
    for (int i = 1; i < 4; ++i) {
      size_t key = idx[i];
      int j = i - 1;
      while (j >= 0 && abs(v[idx[j]]) < abs(v[key])) {
        idx[j + 1] = idx[j];
        --j;
      }
      idx[j + 1] = key;
    }
    uint8_t pos0 = (uint8_t)idx[0];
    uint8_t pos1 = (v[idx[1]] != 0 || v[idx[0]] != 0) ? (uint8_t)idx[1] : 1u;
    uint8_t p0 = pos0 < pos1 ? pos0 : pos1, p1 = pos0 < pos1 ? pos1 : pos0;
    int pat = find_pattern(p0, p1);
    if (pat < 0) pat = 0; /* unreachable: reference `expect`s a valid pattern */
    if (g % 2 == 0) patterns[g / 2] |= (uint8_t)(pat & 7);
    else patterns[g / 2] |= (uint8_t)((pat & 7) << 4);
    uint8_t s0 = v[p0] >= 0 ? 1 : 0, s1 = v[p1] >= 0 ? 1 : 0;
    signs[g / 4] |= (uint8_t)((s0 | (s1 << 1)) << ((g % 4) * 2));
  }
}

/* sparse_ternary.rs:166-192 */
void fo_sparse_to_ternary(const uint8_t* patterns, const uint8_t* signs, size_t rows,
                          size_t cols, int8_t* t) {
  size_t ng = rows * cols / 4;
  memset(t, 0, rows * cols);
  for (size_t g = 0; g < ng; ++g) {
    int pat = g % 2 == 0 ? (patterns[g / 2] & 7) : ((patterns[g / 2] >> 4) & 7);
    if (pat >= 6) pat = 0;
    int sb = (signs[g / 4] >> ((g % 4) * 2)) & 3;
    t[g * 4 + SPARSE_PATTERN[pat][0]] = (sb & 1) ? 1 : -1;
    t[g * 4 + SPARSE_PATTERN[pat][1]] = (sb & 2) ? 1 : -1;
  }
}

typedef struct {
  const uint8_t* pat;
  const uint8_t* sg;
  float scale;
  const float* rs;
  size_t rows, cols;
  const float* x;
  float* y;
  size_t seq;
} fo_sp_ctx;

static float fo_sparse_row(const fo_sp_ctx* c, size_t r, const float* xr) {
  size_t ng = c->cols / 4;
  float sum = 0.0f;
  for (size_t g = 0; g < ng; ++g) {
    size_t gi = r * ng + g;
    int pat = gi % 2 == 0 ? (c->pat[gi / 2] & 7) : ((c->pat[gi / 2] >> 4) & 7);
    int sb = (c->sg[gi / 4] >> ((gi % 4) * 2)) & 3;
    float s0 = (sb & 1) ? 1.0f : -1.0f, s1 = (sb & 2) ? 1.0f : -1.0f;
    sum += s0 * xr[g * 4 + SPARSE_PATTERN[pat][0]];
    sum += s1 * xr[g * 4 + SPARSE_PATTERN[pat][1]];
  }
  return sum;
}

static void fo_sp_item(void* v, size_t item) {
  /* item = token*rows + row batch of 64 rows */
  fo_sp_ctx* c = (fo_sp_ctx*)v;
  size_t nb = (c->rows + 63) / 64;
  size_t s = item / nb, b = item % nb;
  size_t r0 = b * 64, r1 = r0 + 64 > c->rows ? c->rows : r0 + 64;
  const float* xr = c->x + s * c->cols;
  for (size_t r = r0; r < r1; ++r) {
    float sum = fo_sparse_row(c, r, xr);
    c->y[s * c->rows + r] = (c->rs ? c->rs[r] : c->scale) * sum;
  }
}

/* sparse_ternary.rs:203-252 */
void fo_sparse_ternary_matmul(const uint8_t* patterns, const uint8_t* signs, float scale,
                              const float* row_scales, size_t rows, size_t cols, const float* x,
                              size_t seq, float* y, int nthreads) {
  fo_sp_ctx c = {patterns, signs, scale, row_scales, rows, cols, x, y, seq};
  fo_parallel_for(seq * ((rows + 63) / 64), nthreads, fo_sp_item, &c);
}

size_t fo_sparse_wgsl_words_per_row(size_t cols) { return (((cols + 3) / 4) + 5) / 6; }

/* src/compute/kernels/sparse_ternary.rs:254-318; returns -1 when a group does
 * not hold exactly two nonzeros (the reference packer panics there). */
int fo_sparse_wgsl_pack(const int8_t* t, size_t rows, size_t cols, uint32_t* packed) {
  size_t gpr = (cols + 3) / 4, wpr = fo_sparse_wgsl_words_per_row(cols);
  memset(packed, 0, sizeof(uint32_t) * rows * wpr);
  for (size_t r = 0; r < rows; ++r)
    for (size_t g = 0; g < gpr; ++g) {
      int pos[2], val[2], nnz = 0;
      for (int i = 0; i < 4; ++i) {
        size_t col = g * 4 + (size_t)i;
        if (col < cols && t[r * cols + col] != 0) {
          if (nnz < 2) {
            pos[nnz] = i;
            val[nnz] = t[r * cols + col];
          }
          ++nnz;
        }
      }
      if (nnz != 2) return -1;
      int pat = find_pattern((uint8_t)pos[0], (uint8_t)pos[1]);
      uint32_t sgn = (uint32_t)(val[0] < 0) | ((uint32_t)(val[1] < 0) << 1);
      uint32_t gp = (uint32_t)pat | (sgn << 3);
      packed[r * wpr + g / 6] |= gp << ((g % 6) * 5);
    }
  return 0;
}

/* src/compute/kernels/sparse_ternary.rs:321-360 */
void fo_sparse_wgsl_ref(const uint32_t* packed, const float* scales, const float* x, size_t seq,
                        size_t cols, size_t rows, float* y) {
  size_t gpr = (cols + 3) / 4, wpr = fo_sparse_wgsl_words_per_row(cols);
  for (size_t s = 0; s < seq; ++s)
    for (size_t r = 0; r < rows; ++r) {
      float sum = 0.0f;
      for (size_t g = 0; g < gpr; ++g) {
        uint32_t gp = (packed[r * wpr + g / 6] >> ((g % 6) * 5)) & 0x1Fu;
        uint32_t pat = gp & 7u;
        if (pat > 5) pat = 5;
        uint32_t sg = (gp >> 3) & 3u;
        size_t ca = g * 4 + SPARSE_PATTERN[pat][0], cb = g * 4 + SPARSE_PATTERN[pat][1];
        float sa = (sg & 1u) ? -1.0f : 1.0f, sb = (sg & 2u) ? -1.0f : 1.0f;
        if (ca < cols) sum += sa * x[s * cols + ca];
        if (cb < cols) sum += sb * x[s * cols + cb];
      }
      y[s * rows + r] = sum * scales[r];
    }
}

/* ------------------------------------------------------------------------ */
/* MoE layer: src/model/ternary_moe.rs:145-223                              */
/* ------------------------------------------------------------------------ */
typedef struct {
  const float* router;
  const int8_t* const* gate;
  const float* const* gate_s;
  const int8_t* const* up;
  const float* const* up_s;
  const int8_t* const* down;
  const float* const* down_s;
  size_t hidden, inter, ne, top_k;
  int use_gelu;
  const float* x;
  float* y;
  int32_t* route;
  float* probs;
} fo_moe_ctx;

/* ternary_matmul_decode with per-row scales (ternary.rs:591-633) */
static void decode_rows(const int8_t* t, const float* rs, const float* x, size_t out_rows,
                        size_t in_cols, float* y) {
  for (size_t r = 0; r < out_rows; ++r) {
    const int8_t* w = t + r * in_cols;
    float sum = 0.0f;
    size_t chunks = in_cols / 8;
    for (size_t c = 0; c < chunks; ++c)
      for (size_t u = 0; u < 8; ++u) sum += (float)w[c * 8 + u] * x[c * 8 + u];
    for (size_t j = chunks * 8; j < in_cols; ++j) sum += (float)w[j] * x[j];
    y[r] = rs[r] * sum;
  }
}

static void fo_moe_item(void* v, size_t s) {
  fo_moe_ctx* c = (fo_moe_ctx*)v;
  size_t H = c->hidden, F = c->inter, E = c->ne;
  const float* xr = c->x + s * H;
  float* yr = c->y + s * H;
  float* scores = (float*)malloc(sizeof(float) * E);
  size_t* order = (size_t*)malloc(sizeof(size_t) * E);
  float* g = (float*)malloc(sizeof(float) * F);
  float* u = (float*)malloc(sizeof(float) * F);
  float* h = (float*)malloc(sizeof(float) * F);
  float* d = (float*)malloc(sizeof(float) * H);
  for (size_t j = 0; j < H; ++j) yr[j] = 0.0f;
  /* 1. router scores[e] = sum_j R[e*H+j] * x[j]  (ternary_moe.rs:153-160) */
  for (size_t e = 0; e < E; ++e) {
    float sum = 0.0f;
    for (size_t j = 0; j < H; ++j) sum += c->router[e * H + j] * xr[j];
    scores[e] = sum;
  }
  /* 2. softmax (:163-172) */
  float mx = -INFINITY;
  for (size_t e = 0; e < E; ++e) mx = fmaxf(mx, scores[e]);
  float se = 0.0f;
  for (size_t e = 0; e < E; ++e) {
    scores[e] = expf(scores[e] - mx);
    se += scores[e];
  }
  for (size_t e = 0; e < E; ++e) scores[e] /= se;
  if (c->probs) memcpy(c->probs + s * E, scores, sizeof(float) * E);
  /* 3. stable descending sort (:175-177) */
  for (size_t e = 0; e < E; ++e) order[e] = e;
  for (size_t i = 1; i < E; ++i) {
    size_t key = order[i];
    size_t j = i;
    while (j > 0 && scores[order[j - 1]] < scores[key]) {
      order[j] = order[j - 1];
      --j;
    }
    order[j] = key;
  }
  size_t K = c->top_k < E ? c->top_k : E;
  float wsum = 0.0f; /* (:180-183) */
  for (size_t k = 0; k < K; ++k) wsum += scores[order[k]];
  for (size_t k = 0; k < K; ++k) {
    size_t e = order[k];
    if (c->route) c->route[s * c->top_k + k] = (int32_t)e;
    decode_rows(c->gate[e], c->gate_s[e], xr, F, H, g);
    decode_rows(c->up[e], c->up_s[e], xr, F, H, u);
    for (size_t i = 0; i < F; ++i) {
      if (c->use_gelu) { /* (:199-204) */
        float xv = g[i];
        float ta = 0.7978845608f * (xv + 0.044715f * xv * xv * xv);
        h[i] = 0.5f * xv * (1.0f + tanhf(ta));
      } else { /* (:206-209) */
        float gv = g[i];
        float silu = gv / (1.0f + expf(-gv));
        h[i] = silu * u[i];
      }
    }
    decode_rows(c->down[e], c->down_s[e], h, H, F, d);
    float w = wsum > 0.0f ? scores[e] / wsum : scores[e]; /* (:218) */
    for (size_t j = 0; j < H; ++j) yr[j] += w * d[j];
  }
  free(scores); free(order); free(g); free(u); free(h); free(d);
}

void fo_moe_forward(const float* router, const int8_t* const* gate, const float* const* gate_s,
                    const int8_t* const* up, const float* const* up_s,
                    const int8_t* const* down, const float* const* down_s, size_t hidden,
                    size_t inter, size_t n_experts, size_t top_k, int use_gelu, const float* x,
                    size_t seq, float* y, int32_t* route_out, float* probs_out, int nthreads) {
  fo_moe_ctx c = {router, gate, gate_s, up, up_s, down, down_s, hidden, inter, n_experts, top_k,
                  use_gelu, x, y, route_out, probs_out};
  fo_parallel_for(seq, nthreads, fo_moe_item, &c);
}

/* ------------------------------------------------------------------------ */
/* TurboQuant 3-bit: src/inference/turboquant_kv.rs                         */
/* ------------------------------------------------------------------------ */
static void pack_3bit_8(const uint8_t* codes, uint8_t* p) { /* :35-54 */
  p[0] = p[1] = p[2] = 0;
  size_t bit = 0;
  for (int i = 0; i < 8; ++i) {
    uint8_t c3 = codes[i] & 7;
    size_t bi = bit / 8, sh = bit % 8;
    p[bi] |= (uint8_t)(c3 << sh);
    if (sh + 3 > 8) p[bi + 1] |= (uint8_t)(c3 >> (8 - sh));
    bit += 3;
  }
}

static void unpack_3bit_8(const uint8_t* p, uint8_t* codes) { /* :57-74 */
  size_t bit = 0;
  for (int i = 0; i < 8; ++i) {
    size_t bi = bit / 8, sh = bit % 8;
    uint8_t v = (uint8_t)((p[bi] >> sh) & 7);
    if (sh + 3 > 8) {
      size_t spill = sh + 3 - 8;
      v |= (uint8_t)((p[bi + 1] & ((1u << spill) - 1)) << (3 - spill));
    }
    codes[i] = v;
    bit += 3;
  }
}

void fo_pack_3bit(const uint8_t* codes, size_t n, uint8_t* packed) { /* :121-137 */
  size_t ng = (n + 7) / 8;
  for (size_t g = 0; g < ng; ++g) {
    uint8_t buf[8] = {0};
    for (size_t i = 0; i < 8 && g * 8 + i < n; ++i) buf[i] = codes[g * 8 + i];
    pack_3bit_8(buf, packed + g * 3);
  }
}

void fo_unpack_3bit(const uint8_t* packed, size_t n, uint8_t* codes) { /* :140-161 */
  size_t ng = (n + 7) / 8, out = 0;
  for (size_t g = 0; g < ng && out < n; ++g) {
    uint8_t buf[8];
    unpack_3bit_8(packed + g * 3, buf);
    for (int i = 0; i < 8 && out < n; ++i) codes[out++] = buf[i];
  }
}

void fo_quantize_3bit(const float* v, size_t n, uint8_t* codes, float* mn, float* mx) {
  if (n == 0) { *mn = 0.0f; *mx = 0.0f; return; }
  float lo = INFINITY, hi = -INFINITY;
  for (size_t i = 0; i < n; ++i) { lo = fminf(lo, v[i]); hi = fmaxf(hi, v[i]); }
  float range = hi - lo;
  float scale = range > 0.0f ? 7.0f / range : 0.0f;
  for (size_t i = 0; i < n; ++i) {
    if (range > 0.0f) {
      float r = roundf((v[i] - lo) * scale);
      uint32_t c = r <= 0.0f ? 0u : (uint32_t)r; /* `as u32` saturates at 0 */
      codes[i] = (uint8_t)(c > 7u ? 7u : c);
    } else {
      codes[i] = 0;
    }
  }
  *mn = lo;
  *mx = hi;
}

void fo_dequantize_3bit(const uint8_t* codes, size_t n, float mn, float mx, float* out) {
  if (mx == mn) { for (size_t i = 0; i < n; ++i) out[i] = mn; return; } /* :111-113 */
  float scale = (mx - mn) / 7.0f;
  for (size_t i = 0; i < n; ++i) out[i] = mn + (float)codes[i] * scale;
}

void fo_kv_quantize_vector(const float* v, size_t kv_dim, size_t group, uint8_t* packed,
                           float* minmax) {
  uint8_t* codes = (uint8_t*)malloc(kv_dim);
  size_t ng = (kv_dim + group - 1) / group;
  for (size_t g = 0; g < ng; ++g) {
    size_t s = g * group, e = s + group > kv_dim ? kv_dim : s + group;
    fo_quantize_3bit(v + s, e - s, codes + s, &minmax[2 * g], &minmax[2 * g + 1]);
  }
  fo_pack_3bit(codes, kv_dim, packed);
  free(codes);
}

void fo_kv_dequantize_vector(const uint8_t* packed, const float* minmax, size_t kv_dim,
                             size_t group, float* out) {
  uint8_t* codes = (uint8_t*)malloc(kv_dim);
  fo_unpack_3bit(packed, kv_dim, codes);
  size_t ng = (kv_dim + group - 1) / group;
  for (size_t g = 0; g < ng; ++g) {
    size_t s = g * group, e = s + group > kv_dim ? kv_dim : s + group;
    fo_dequantize_3bit(codes + s, e - s, minmax[2 * g], minmax[2 * g + 1], out + s);
  }
  free(codes);
}

/* ------------------------------------------------------------------------ */
/* flash decode: tests/kernel_tests.rs:1073-1110 + GQA map                  */
/* ------------------------------------------------------------------------ */
typedef struct {
  const float* q;
  const float* k;
  const float* v;
  const uint8_t* kc;
  const float* kmm;
  const uint8_t* vc;
  const float* vmm;
  size_t batch, seq, hq, hkv, d;
  float* out;
} fo_fd_ctx;

static void fd_load(const fo_fd_ctx* c, int is_v, size_t b, size_t s, size_t kvh, float* dst) {
  size_t off = ((b * c->seq + s) * c->hkv + kvh);
  if (c->kc) {
    const uint8_t* codes = (is_v ? c->vc : c->kc) + off * (c->d * 3 / 8);
    const float* mm = (is_v ? c->vmm : c->kmm) + off * 2;
    fo_kv_dequantize_vector(codes, mm, c->d, c->d, dst);
  } else {
    memcpy(dst, (is_v ? c->v : c->k) + off * c->d, sizeof(float) * c->d);
  }
}

static void fo_fd_item(void* vctx, size_t item) {
  fo_fd_ctx* c = (fo_fd_ctx*)vctx;
  size_t b = item / c->hq, h = item % c->hq;
  size_t kvh = h / (c->hq / c->hkv);
  size_t D = c->d;
  const float* q = c->q + (b * c->hq + h) * D;
  float scale = 1.0f / sqrtf((float)D);
  float* kv = (float*)malloc(sizeof(float) * D);
  float* acc = (float*)calloc(D, sizeof(float));
  float mx = -INFINITY;
  for (size_t s = 0; s < c->seq; ++s) { /* pass 1 */
    fd_load(c, 0, b, s, kvh, kv);
    float dot = 0.0f;
    for (size_t i = 0; i < D; ++i) dot += q[i] * kv[i];
    mx = fmaxf(mx, dot * scale);
  }
  float se = 0.0f;
  for (size_t s = 0; s < c->seq; ++s) { /* pass 2 */
    fd_load(c, 0, b, s, kvh, kv);
    float dot = 0.0f;
    for (size_t i = 0; i < D; ++i) dot += q[i] * kv[i];
    float w = expf(dot * scale - mx);
    se += w;
    fd_load(c, 1, b, s, kvh, kv);
    for (size_t i = 0; i < D; ++i) acc[i] += w * kv[i];
  }
  float inv = 1.0f / se;
  for (size_t i = 0; i < D; ++i) c->out[(b * c->hq + h) * D + i] = acc[i] * inv;
  free(kv);
  free(acc);
}

void fo_flash_decode_gqa(const float* q, const float* k, const float* v, size_t batch,
                         size_t seq, size_t hq, size_t hkv, size_t d, float* out, int nthreads) {
  fo_fd_ctx c = {q, k, v, NULL, NULL, NULL, NULL, batch, seq, hq, hkv, d, out};
  fo_parallel_for(batch * hq, nthreads, fo_fd_item, &c);
}

void fo_flash_decode_3bit(const float* q, const uint8_t* kc, const float* kmm, const uint8_t* vc,
                          const float* vmm, size_t batch, size_t seq, size_t hq, size_t hkv,
                          size_t d, float* out, int nthreads) {
  fo_fd_ctx c = {q, NULL, NULL, kc, kmm, vc, vmm, batch, seq, hq, hkv, d, out};
  fo_parallel_for(batch * hq, nthreads, fo_fd_item, &c);
}

/* ------------------------------------------------------------------------ */
/* 3-bit KV "mode T": rotation + uniform codebook + per-vector norm.        */
/* The reference has no working implementation of this scheme (its          */
/* TurboQuantEngine, src/compute/turboquant.rs:89-367, draws an unseeded     */
/* rotation and its WGSL does not compile); this is this project's spec:     */
/*   norm = ||v||_2 (fp32; squares summed as 4 warps of 32 lanes, each warp  */
/*          by the xor butterfly 16, 8, 4, 2, 1, then ((w0+w1)+w2)+w3)       */
/*   u    = v / norm, u_i *= sign_i (seeded +-1)                             */
/*   y    = H u (Walsh-Hadamard, butterflies h = 1, 2, ..., 64 in place:     */
/*          a = y[j], b = y[j+h]; y[j] = a + b; y[j+h] = a - b)              */
/*   z    = y / 2.5 (y_i ~ N(0, 1) for a random direction: clip at 2.5 sigma)*/
/*   code = clamp(floor((z + 1) * 4), 0, 7): the nearest of the 8 uniform    */
/*          centroids (2i+1)/8 - 1 on [-1, 1] (the centroids that            */
/*          compute_mse_centroids, turboquant.rs:197-220, converges to)      */
/* Dequantized, the rotated unit vector has coordinates                      */
/*   yhat_i = 2.5 * ((2 code_i + 1)/8 - 1) / sqrt(128)                       */
/* and v = norm * D H yhat / sqrt(128)... i.e. in the rotated domain the     */
/* vector is affine in the code: min + code * (max - min) / 7 with           */
/*   max = -min = norm * (2.5 * 7/8 / sqrt(128)).                            */
/* Attention in the rotated domain: q' = H D q / sqrt(128), o = D H o' /     */
/* sqrt(128).                                                                */
/* ------------------------------------------------------------------------ */
static const float FO_KVT_CLIP = 2.5f;

static void fo_fwht128(float* y) {
  for (int h = 1; h < 128; h <<= 1)
    for (int i = 0; i < 128; i += 2 * h)
      for (int j = i; j < i + h; ++j) {
        const float a = y[j], b = y[j + h];
        y[j] = a + b;
        y[j + h] = a - b;
      }
}

float fo_kvt_mm_const(void) { return (FO_KVT_CLIP * 7.0f / 8.0f) / sqrtf(128.0f); }

/* one 128-vector -> 128 codes (0..7) and its norm */
void fo_kvt_quantize(const float* v, const float* signs, uint8_t* codes, float* norm_out) {
  float sq[128];
  for (int i = 0; i < 128; ++i) sq[i] = v[i] * v[i];
  float wsum[4];
  for (int w = 0; w < 4; ++w) {
    float lanes[32];
    for (int l = 0; l < 32; ++l) lanes[l] = sq[32 * w + l];
    for (int o = 16; o > 0; o >>= 1) {
      float nl[32];
      for (int l = 0; l < 32; ++l) nl[l] = lanes[l] + lanes[l ^ o];
      memcpy(lanes, nl, sizeof(lanes));
    }
    wsum[w] = lanes[0];
  }
  const float n2 = ((wsum[0] + wsum[1]) + wsum[2]) + wsum[3];
  const float norm = sqrtf(n2);
  *norm_out = norm;
  float y[128];
  for (int i = 0; i < 128; ++i) y[i] = norm > 0.0f ? (v[i] / norm) * signs[i] : 0.0f;
  fo_fwht128(y);
  for (int i = 0; i < 128; ++i) {
    const float z = y[i] / FO_KVT_CLIP;
    const float c = floorf((z + 1.0f) * 4.0f);
    codes[i] = (uint8_t)(c <= 0.0f ? 0 : (c >= 7.0f ? 7 : (int)c));
  }
}

/* q' = H D q / sqrt(128) (inverse = 0) or o = D H o' / sqrt(128) (inverse = 1) */
void fo_kvt_rotate(const float* in, const float* signs, int inverse, float* out) {
  float y[128];
  for (int i = 0; i < 128; ++i) y[i] = inverse ? in[i] : in[i] * signs[i];
  fo_fwht128(y);
  const float s = 1.0f / sqrtf(128.0f);
  for (int i = 0; i < 128; ++i) out[i] = inverse ? (y[i] * s) * signs[i] : y[i] * s;
}
