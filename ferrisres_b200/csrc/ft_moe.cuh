// The resident MoE layer (shared by ft_moe.cu and ft_moe_decode.cu).
#pragma once

#include <vector>

#include "ft_internal.cuh"

struct ft_moe {
  int device = 0;
  int64_t E = 0, H = 0, F = 0;
  int top_k = 2;
  int use_gelu = 0;
  float* router = nullptr;  // [E, H] fp32 (row e = expert e)
  uint16_t* router_planes = nullptr;  // [n_rplanes][64][Hpad] bf16: router = sum of the planes
  int n_rplanes = 0;
  int64_t Hpad = 0;                   // H rounded up to the router kernel's K chunk
  std::vector<ft_weight*> gate_up;  // [2F, H] each: gate rows then up rows
  std::vector<ft_weight*> down;     // [H, F] each
  ft::Workspace buf;                // forward intermediates (grown on demand)
  std::vector<int32_t> counts_host;
  // device tables for the fused decode kernel: per expert the gate_up / down
  // codes and row scales (null for experts held by another rank)
  const void** dtab = nullptr;  // [4][E]
  ft::Workspace dbuf;           // decode scratch (grown on demand)
};

namespace ft {
// The fused decode step (ft_moe_decode.cu).
int moe_decode(ft_ctx* ctx, ft_moe* m, int64_t T, const void* x, int bf16, float* y,
               int32_t* topk_idx, float* topk_w, float* probs, cudaStream_t s);
}  // namespace ft
