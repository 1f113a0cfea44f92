/* A C program that drives libferris_ternary.so through its C ABI alone (no
 * Python, no CUDA headers): the calls a C or FFI host makes.  It uploads a
 * ternary weight in the reference's pack_ternary byte layout, runs the
 * host-buffer matmul (GpuMatmulAccelerator::gpu_ternary_matmul_vram form),
 * checks every output against a double-precision reference computed here
 * under the 1e-5-of-condition rule, reads the resident codes back, runs a
 * small MoE layer through ft_moe_forward_host, and checks that a bad shape is
 * refused with FT_ERR_SHAPE.  Prints "ok" and returns 0. */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "ferris_ternary.h"

static unsigned long long lcg = 88172645463325252ull;
static double urand(void) {
  lcg = lcg * 6364136223846793005ull + 1442695040888963407ull;
  return (double)(lcg >> 11) / 9007199254740992.0;
}

static int fail(const char* what, int st) {
  fprintf(stderr, "%s failed: status %d: %s\n", what, st, ft_last_error_string());
  return 1;
}

static void pack_ternary(const signed char* v, long n, unsigned char* out) {
  memset(out, 0, (size_t)((n + 3) / 4));
  for (long i = 0; i < n; ++i) {
    const unsigned code = v[i] == -1 ? 0u : v[i] == 1 ? 2u : 1u;
    out[i / 4] |= (unsigned char)(code << ((i % 4) * 2));
  }
}

int main(void) {
  printf("%s\n", ft_version());
  ft_ctx* ctx = NULL;
  int st = ft_ctx_create(0, &ctx);
  if (st) return fail("ft_ctx_create", st);

  /* dense matmul with host buffers */
  const long rows = 300, cols = 1000, seq = 3;
  signed char* t = malloc((size_t)(rows * cols));
  unsigned char* packed = malloc((size_t)((rows * cols + 3) / 4));
  float* rs = malloc(sizeof(float) * rows);
  float* x = malloc(sizeof(float) * seq * cols);
  float* y = malloc(sizeof(float) * seq * rows);
  for (long i = 0; i < rows * cols; ++i) t[i] = (signed char)((int)(urand() * 3.0) - 1);
  for (long r = 0; r < rows; ++r) rs[r] = (float)(0.01 + 0.09 * urand());
  for (long i = 0; i < seq * cols; ++i) x[i] = (float)(urand() * 2.0 - 1.0);
  pack_ternary(t, rows * cols, packed);
  ft_weight* w = NULL;
  st = ft_weight_upload_packed_u8(ctx, packed, rows, cols, rs, &w);
  if (st) return fail("ft_weight_upload_packed_u8", st);
  st = ft_gpu_ternary_matmul_vram(ctx, w, x, (size_t)seq, (size_t)cols, (size_t)rows, y);
  if (st) return fail("ft_gpu_ternary_matmul_vram", st);
  /* slice lengths that disagree with the weight are refused at the boundary */
  if (ft_gpu_ternary_matmul_vram(ctx, w, x, (size_t)seq, (size_t)cols, (size_t)rows + 1, y) !=
      FT_ERR_SHAPE)
    return fail("ft_gpu_ternary_matmul_vram accepted a wrong out_rows", -1);
  for (long s = 0; s < seq; ++s)
    for (long r = 0; r < rows; ++r) {
      double ref = 0.0, cond = 0.0;
      for (long k = 0; k < cols; ++k) {
        ref += (double)t[r * cols + k] * x[s * cols + k];
        cond += fabs((double)t[r * cols + k] * x[s * cols + k]);
      }
      ref *= rs[r];
      cond *= rs[r];
      if (fabs(y[s * rows + r] - ref) > 1e-5 * cond + 1e-30) {
        fprintf(stderr, "matmul mismatch at token %ld row %ld: %g vs %g\n", s, r,
                (double)y[s * rows + r], ref);
        return 1;
      }
    }

  /* the resident codes read back are the bytes that went in */
  unsigned char* back = malloc((size_t)((rows * cols + 3) / 4));
  st = ft_weight_export_packed_u8(ctx, w, back);
  if (st) return fail("ft_weight_export_packed_u8", st);
  if (memcmp(back, packed, (size_t)((rows * cols + 3) / 4)) != 0) {
    fprintf(stderr, "exported codes differ from the upload\n");
    return 1;
  }

  /* a weight shape the ABI must refuse */
  ft_weight* bad = NULL;
  st = ft_weight_upload_packed_u8(ctx, packed, 0, cols, rs, &bad);
  if (st != FT_ERR_SHAPE || bad != NULL) {
    fprintf(stderr, "zero-row weight not refused (status %d)\n", st);
    return 1;
  }

  /* a small MoE layer with host buffers: runs and gives finite outputs */
  const long E = 4, H = 64, F = 32, T = 5;
  float* router = malloc(sizeof(float) * E * H);
  for (long i = 0; i < E * H; ++i) router[i] = (float)(0.1 * (urand() - 0.5));
  const unsigned char* gp[4];
  const unsigned char* up[4];
  const unsigned char* dp[4];
  const float* gs[4];
  const float* us[4];
  const float* ds[4];
  signed char* tm = malloc((size_t)(F * H));
  for (long e = 0; e < E; ++e) {
    unsigned char* b[3];
    float* sc[3];
    for (int m = 0; m < 3; ++m) {
      for (long i = 0; i < F * H; ++i) tm[i] = (signed char)((int)(urand() * 3.0) - 1);
      b[m] = malloc((size_t)(F * H / 4));
      pack_ternary(tm, F * H, b[m]);
      const long n = m == 2 ? H : F;
      sc[m] = malloc(sizeof(float) * n);
      for (long i = 0; i < n; ++i) sc[m][i] = (float)(0.01 + 0.09 * urand());
    }
    gp[e] = b[0];
    up[e] = b[1];
    dp[e] = b[2];
    gs[e] = sc[0];
    us[e] = sc[1];
    ds[e] = sc[2];
  }
  ft_moe* moe = NULL;
  st = ft_moe_create(ctx, E, H, F, 2, 0, router, gp, gs, up, us, dp, ds, &moe);
  if (st) return fail("ft_moe_create", st);
  float* mx = malloc(sizeof(float) * T * H);
  float* my = malloc(sizeof(float) * T * H);
  for (long i = 0; i < T * H; ++i) mx[i] = (float)(urand() * 2.0 - 1.0);
  st = ft_moe_forward_host(ctx, moe, mx, (size_t)T, my);
  if (st) return fail("ft_moe_forward_host", st);
  double norm = 0.0;
  for (long i = 0; i < T * H; ++i) {
    if (!isfinite(my[i])) {
      fprintf(stderr, "non-finite MoE output\n");
      return 1;
    }
    norm += fabs(my[i]);
  }
  if (norm == 0.0) {
    fprintf(stderr, "MoE output is all zero\n");
    return 1;
  }
  st = ft_ctx_check(ctx);
  if (st) return fail("ft_ctx_check", st);
  ft_moe_destroy(moe);
  ft_weight_destroy(w);
  ft_ctx_destroy(ctx);
  printf("ok\n");
  return 0;
}
