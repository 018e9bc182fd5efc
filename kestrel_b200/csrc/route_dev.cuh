// Device pieces of the routing front (router.cu): one output lane step of the
// router product and one token's softmax / top-k.
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
// seli: RT_MAXK each) in shared memory. Lane l owns entries l, l + 32, ...
// The maximum and each arg-max of the top-k use warp reductions (redux.sync)
// on integer keys, so a round costs two reductions instead of a shuffle tree.

// Unsigned key with the order of the finite floats.
__device__ __forceinline__ uint32_t ord_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// Softmax of one token's logits into p (one warp).
__device__ __forceinline__ void route_probs(const float* __restrict__ row, int E, float* p, int lane) {
  // Maximum (its sign of zero does not matter: x - (+0) and x - (-0) agree,
  // and exp(+-0) = 1).
  uint32_t km = 0u;
  for (int e = lane; e < E; e += 32) {
    const float v = row[e];
    p[e] = v;
    km = max(km, ord_key(v));
  }
  const float m = key_float(__reduce_max_sync(0xffffffffu, km));
  for (int e = lane; e < E; e += 32) p[e] = exp_rn(__fsub_rn(p[e], m));
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
}

// Top-k of p (>= 0, so their bits order them; key = bits + 1, 0 = taken) by
// repeated arg-max: larger p first, ties to the lower index -- the first k of
// the reference's stable sort. k <= E, so a candidate always remains.
__device__ __forceinline__ void route_topk(int E, int k, float* p, float* selw, int* seli, int lane) {
  uint32_t lk = 0u;
  int li = 0;
  for (int e = lane; e < E; e += 32) {
    const uint32_t kk = __float_as_uint(p[e]) + 1u;
    if (kk > lk) {
      lk = kk;
      li = e;
    }
  }
  for (int r = 0; r < k; ++r) {
    const uint32_t mk = __reduce_max_sync(0xffffffffu, lk);
    const int bi = (int)__reduce_min_sync(0xffffffffu, lk == mk ? (uint32_t)li : 0xffffffffu);
    if (lane == (r & 31)) {
      seli[r] = bi;
      selw[r] = __uint_as_float(mk - 1u);
    }
    if (lane == (bi & 31)) {  // the winner's lane takes it and rescans its entries
      p[bi] = -1.f;
      lk = 0u;
      for (int e = lane; e < E; e += 32) {
        const float v = p[e];
        const uint32_t kk = v >= 0.f ? __float_as_uint(v) + 1u : 0u;
        if (kk > lk) {
          lk = kk;
          li = e;
        }
      }
    }
  }
  __syncwarp();
}

// Renormalisation by the selection's sequential sum clamped at 2^-14, then
// weights_scale; each selection's division is independent. selw keeps the
// final weights for the caller.
__device__ __forceinline__ void route_finish(int k, int norm_topk, float weights_scale, float* selw,
                                             const int* seli, int lane, int* __restrict__ ids_out,
                                             float* __restrict__ w_out) {
  float ss = 0.f;
  if (norm_topk) {
    if (lane == 0) {
      ss = -0.0f;
      for (int r = 0; r < k; ++r) ss = __fadd_rn(ss, selw[r]);
      ss = fmaxf(ss, 6.1035156e-5f);
    }
    ss = __shfl_sync(0xffffffffu, ss, 0);  // after lane 0's reads: selw may be overwritten
  }
  for (int r = lane; r < k; r += 32) {
    float v = selw[r];
    if (norm_topk) v = __fdiv_rn(v, ss);
    if (weights_scale != 0.f && weights_scale != 1.f) v = __fmul_rn(v, weights_scale);
    selw[r] = v;
    ids_out[r] = seli[r];
    w_out[r] = v;
  }
  __syncwarp();
}

__device__ __forceinline__ void route_row(const float* __restrict__ row, int E, int k, int norm_topk,
                                          float weights_scale, float* p, float* selw, int* seli, int lane,
                                          int* __restrict__ ids_out, float* __restrict__ w_out) {
  route_probs(row, E, p, lane);
  route_topk(E, k, p, selw, seli, lane);
  route_finish(k, norm_topk, weights_scale, selw, seli, lane, ids_out, w_out);
}

}  // namespace kc
