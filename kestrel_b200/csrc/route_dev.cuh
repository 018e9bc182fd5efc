// Device pieces of the routing front shared by router.cu and the fused MoE
// decode kernel (moe_decode.cu): one output lane step of the router product
// and one token's softmax / top-k.
#pragma once

#include "common.cuh"

namespace kc {

constexpr int RT_MAXK = 64;  // largest top-k

// One 8-chunk step of output lane j's chain. GEMM: gemm_f32 lane chain (all
// chunks into a0) or, for m1, dot_f32 (even chunks a0, odd chunks a1); else
// quant::dot (separate multiply and add).
template <bool GEMM>
__device__ __forceinline__ void rl_step(float wv, float xv, bool odd, bool m1, float& a0, float& a1) {
  if (GEMM) {
    if (odd && m1) a1 = __fmaf_rn(wv, xv, a1);
    else a0 = __fmaf_rn(wv, xv, a0);
  } else {
    a0 = __fadd_rn(a0, __fmul_rn(wv, xv));
  }
}

// Transformer::route (transformer.rs:472-496): softmax with the sequential
// sum, stable descending order (ties to the lower index), top-k, optional
// renormalisation by the selection's sequential sum clamped at 2^-14, and
// optional weights_scale. One warp per token; p lives in shared memory.

// One token's routing by one warp: p [E] and the selection scratch (selw,
// seli: RT_MAXK each) in shared memory.
__device__ __forceinline__ void route_row(const float* __restrict__ row, int E, int k, int norm_topk, float weights_scale, float* p,
                          float* selw, int* seli, int lane, int* __restrict__ ids_out, float* __restrict__ w_out) {
  float m = -INFINITY;
  for (int e = lane; e < E; e += 32) m = fmaxf(m, row[e]);
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  for (int e = lane; e < E; e += 32) p[e] = exp_rn(__fsub_rn(row[e], m));
  __syncwarp();
  // Sequential sum (transformer.rs:481), loads batched ahead of the adds.
  float sum = -0.0f;
  if (lane == 0) {
    int e = 0;
    for (; e + 8 <= E; e += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = p[e + u];
#pragma unroll
      for (int u = 0; u < 8; ++u) sum = __fadd_rn(sum, v[u]);
    }
    for (; e < E; ++e) sum = __fadd_rn(sum, p[e]);
  }
  sum = __shfl_sync(0xffffffffu, sum, 0);
  for (int e = lane; e < E; e += 32) p[e] = __fdiv_rn(p[e], sum);
  __syncwarp();
  // Top-k by repeated arg-max (larger p first, ties to the lower index, which
  // is the first k of the reference's stable sort). Probabilities are >= 0, so
  // a taken entry is marked with -1 in shared memory.
  constexpr int NONE = 0x7fffffff;
  for (int r = 0; r < k; ++r) {
    float bp = 0.f;
    int bi = NONE;
    for (int e = lane; e < E; e += 32) {
      const float v = p[e];
      if (v < 0.f) continue;
      if (bi == NONE || v > bp) {  // e increases within a lane: ties keep the lower index
        bp = v;
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float op = __shfl_xor_sync(0xffffffffu, bp, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (oi != NONE && (bi == NONE || op > bp || (op == bp && oi < bi))) {
        bp = op;
        bi = oi;
      }
    }
    if (lane == 0) {
      seli[r] = bi;
      selw[r] = bp;
    }
    if (bi != NONE && lane == (bi & 31)) p[bi] = -1.f;
    __syncwarp();
  }
  if (lane == 0) {
    if (norm_topk) {
      float ss = -0.0f;
      for (int r = 0; r < k; ++r) ss = __fadd_rn(ss, selw[r]);
      ss = fmaxf(ss, 6.1035156e-5f);
      for (int r = 0; r < k; ++r) selw[r] = __fdiv_rn(selw[r], ss);
    }
    if (weights_scale != 0.f && weights_scale != 1.f)
      for (int r = 0; r < k; ++r) selw[r] = __fmul_rn(selw[r], weights_scale);
  }
  __syncwarp();
  for (int r = lane; r < k; r += 32) {
    ids_out[r] = seli[r];
    w_out[r] = selw[r];
  }
  __syncwarp();
}

}  // namespace kc
