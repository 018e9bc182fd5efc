// Router logits, softmax/top-k routing, dispatch metadata (the permute) and
// the weighted combine (the un-permute).
#include <algorithm>

#include "common.cuh"
#include "decode.h"
#include "kernels.h"
#include "route_dev.cuh"

namespace kc {

// ---------------------------------------------------------------------------
// Router logits = quant::matmul of the F32 router [E, d] with h [n_tok, d]
// (crates/kestrel-engine/src/quant.rs:229-339), reproducing the reference's
// operation order exactly so that the top-k selection is bit-exact:
//   * n_tok < 4 (or d % 8 != 0): quant::dot (quant.rs:208-224) -- eight lane
//     accumulators, separate mul and add, lanes folded in order from -0.0, then
//     the scalar tail;
//   * n_tok >= 4: avx2::gemm_f32 (avx2.rs:230-286) on 48-row tiles: rows in the
//     tile's 3-row blocks and tokens in 4-token blocks use one 8-lane FMA chain
//     per output + hsum; the other outputs use dot_f32 (avx2.rs:289-308), whose
//     even 8-chunks feed acc0 and odd ones acc1, summed lane-wise before hsum.
// Thread layout: 8 threads (one per lane) per (expert row, token) output; a
// block computes RL_E rows x RL_T tokens. Weight and token rows are streamed
// through shared memory in K chunks of RL_KC floats with bulk copies
// (double-buffered), so every thread's chain reads shared memory only; each
// lane still visits its elements c = lane, lane+8, ... in increasing order.
constexpr int RT_WARPS = 4;      // route_kernel: tokens (warps) per CTA
constexpr int DP_THREADS = 1024; // dispatch: one block

__device__ void dispatch_block(const int* __restrict__ ids, const float* __restrict__ w, int n_tok, int k, int E,
                               const DispatchOut& o, uint32_t* dsm, bool rows);
__device__ void dispatch_small(const int* __restrict__ ids, const float* __restrict__ w, int n_tok, int k, int E,
                               const DispatchOut& o, uint32_t* dsm);

constexpr int RL_E = 8, RL_T = 4, RL_KC = 1024;
constexpr int RL_ROW = RL_KC + 8;  // padded shared row: the 4 expert rows a warp reads hit distinct banks
constexpr size_t rl_smem(int rt, int re) { return 2 * (size_t)(re + rt) * RL_ROW * sizeof(float); }

// RE expert rows x RT tokens per block. Decode-sized batches (n < 4) take one
// expert row per block, so that the router matrix is read by E blocks.
template <bool GEMM, int RT, int RE = RL_E>
__global__ void __launch_bounds__(RE * RT * 8) router_logits_kernel(const float* __restrict__ w, int64_t ws, int E,
                                                                    int d, const float* __restrict__ h, int n_tok,
                                                                    float* __restrict__ logits, int* status) {
  pdl_enter();
  extern __shared__ __align__(128) float rsm[];  // [2][RE + RT][RL_ROW]
  __shared__ __align__(8) uint64_t full[2];
  const int tid = threadIdx.x, j = tid & 7, grp = tid >> 3;
  const int er = grp % RE, tr = grp / RE;
  const int e0 = blockIdx.x * RE, s0 = blockIdx.y * RT;
  const int ne = min(RE, E - e0), nt = min(RT, n_tok - s0);
  const int erc = min(er, ne - 1), trc = min(tr, nt - 1);
  const int e = e0 + erc, s = s0 + trc;
  const bool valid = er < ne && tr < nt;
  const int n8 = d / 8 * 8;
  // gemm_f32 blocks rows in 3s inside 48-row tiles and tokens in 4s; the
  // outputs outside those blocks go through dot_f32 (m1).
  bool m1 = false;
  if (GEMM) {
    const int tile = e / 48, trows = min(48, E - tile * 48), rows3 = trows / 3 * 3;
    const bool row_blocked = (e - tile * 48) < rows3;
    m1 = !(row_blocked && s < n_tok / 4 * 4);
  }
  const int nchunk = (d + RL_KC - 1) / RL_KC;
  const bool bulk_ok = (d % 4) == 0 && (ws % 4) == 0 && ((uintptr_t)w & 15) == 0 &&
                       ((uintptr_t)h & 15) == 0;  // 16-byte aligned rows
  if (tid == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int c) {
    float* buf = rsm + (c & 1) * (RE + RT) * RL_ROW;
    const int k0 = c * RL_KC, kn = min(RL_KC, d - k0);
    const uint32_t rb = (uint32_t)kn * 4;
    mbar_expect_tx(&full[c & 1], rb * (ne + nt));
    for (int r = 0; r < ne; ++r) bulk_g2s(buf + r * RL_ROW, w + (int64_t)(e0 + r) * ws + k0, rb, &full[c & 1]);
    for (int r = 0; r < nt; ++r) bulk_g2s(buf + (RE + r) * RL_ROW, h + (int64_t)(s0 + r) * d + k0, rb, &full[c & 1]);
  };
  float a0 = 0.f, a1 = 0.f;
  if (bulk_ok) {
    if (tid == 0) {
      issue(0);
      if (nchunk > 1) issue(1);
    }
    for (int c = 0; c < nchunk; ++c) {
      mbar_wait(&full[c & 1], (c >> 1) & 1, status, W_ROUTER);
      const float* buf = rsm + (c & 1) * (RE + RT) * RL_ROW;
      const float* wr = buf + erc * RL_ROW + j;
      const float* xr = buf + (RE + trc) * RL_ROW + j;
      const int k0 = c * RL_KC, kn = min(RL_KC, n8 - k0);  // k0 is an even number of 8-chunks
      int cc = 0;
      for (; cc + 64 <= kn; cc += 64) {
        float wv[8], xv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          wv[u] = wr[cc + 8 * u];
          xv[u] = xr[cc + 8 * u];
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) rl_step<GEMM>(wv[u], xv[u], u & 1, m1, a0, a1);
      }
      for (; cc < kn; cc += 8) rl_step<GEMM>(wr[cc], xr[cc], (cc >> 3) & 1, m1, a0, a1);
      __syncthreads();  // everyone is done with this buffer
      if (tid == 0 && c + 2 < nchunk) issue(c + 2);
    }
  } else {
    // Rows not 16-byte aligned: read global memory directly.
    const float* wr = w + (int64_t)e * ws;
    const float* xr = h + (int64_t)s * d;
    for (int c = 0; c < n8; c += 8) rl_step<GEMM>(wr[c + j], xr[c + j], (c >> 3) & 1, m1, a0, a1);
  }
  float v;
  if (!GEMM) {
    // Sequential fold of the eight lanes from -0.0, then the tail.
    float sum = -0.0f;
#pragma unroll
    for (int l = 0; l < 8; ++l) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, a0, l, 8));
    for (int c = n8; c < d; ++c) sum = __fadd_rn(sum, __fmul_rn(w[(int64_t)e * ws + c], h[(int64_t)s * d + c]));
    v = sum;
  } else {
    v = hsum8_group(m1 ? __fadd_rn(a0, a1) : a0);
  }
  if (j == 0 && valid) logits[(int64_t)s * E + e] = v;
}

void launch_router_logits(const float* w, int64_t row_stride_floats, int E, int d, const float* h, int n_tok,
                          float* logits, int* status, cudaStream_t st, bool force_dot) {
  if (n_tok <= 0) return;
  static PerDeviceOnce attr_dot, attr_dot1;
  const size_t smem = rl_smem(RL_T, RL_E);
  smem_attr_once(attr_dot, router_logits_kernel<false, RL_T>, (int)smem);
  // quant::matmul's dispatch (quant.rs:241): the GEMM path needs >= 4 rows and
  // d % 8 == 0; otherwise quant::dot per output.
  if (!force_dot && n_tok >= 4 && d % 8 == 0) {
    // Two expert rows per block (four times the blocks of RL_E rows: the
    // router reads 1-4 MB, so more blocks in flight shorten the launch).
    static PerDeviceOnce attr_gemm2;
    const size_t smem2 = rl_smem(RL_T, 2);
    smem_attr_once(attr_gemm2, router_logits_kernel<true, RL_T, 2>, (int)smem2);
    dim3 grid(ceil_div(E, 2), ceil_div(n_tok, RL_T));
    launch_k(router_logits_kernel<true, RL_T, 2>, grid, 2 * RL_T * 8, smem2, st, w, row_stride_floats, E, d, h, n_tok,
             logits, status);
  } else if (n_tok < 4) {
    // One expert row and up to 4 tokens per block: E blocks.
    const size_t smem1 = rl_smem(RL_T, 1);
    smem_attr_once(attr_dot1, router_logits_kernel<false, RL_T, 1>, (int)smem1);
    launch_k(router_logits_kernel<false, RL_T, 1>, dim3(E, 1), RL_T * 8, smem1, st, w, row_stride_floats, E, d, h,
             n_tok, logits, status);
  } else {
    dim3 grid(ceil_div(E, RL_E), ceil_div(n_tok, RL_T));
    launch_k(router_logits_kernel<false, RL_T>, grid, RL_E * RL_T * 8, smem, st, w, row_stride_floats, E, d, h,
             n_tok, logits, status);
  }
}

// ---------------------------------------------------------------------------
// Transformer::route, one warp per token (route_row, route_dev.cuh).
__global__ void __launch_bounds__(RT_WARPS * 32) route_kernel(const float* __restrict__ logits, int n_tok, int E,
                                                               int k, int norm_topk, float weights_scale,
                                                               int* __restrict__ ids, float* __restrict__ wout,
                                                               const int* __restrict__ fail) {
  pdl_enter();
  extern __shared__ float sp[];  // [RT_WARPS][E] probabilities, then [RT_WARPS][RT_MAXK] selections
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int s = blockIdx.x * RT_WARPS + warp;
  if (s >= n_tok) return;
  // An earlier kernel of this call recorded a failure (a bounded wait that
  // expired): its logits are not trustworthy, so mark the selections invalid.
  if (fail && *(volatile const int*)fail != 0) {
    for (int i = lane; i < k; i += 32) {
      ids[(int64_t)s * k + i] = -1;
      wout[(int64_t)s * k + i] = 0.0f;
    }
    return;
  }
  float* p = sp + warp * E;
  float* selw = sp + RT_WARPS * E + warp * RT_MAXK;
  int* seli = reinterpret_cast<int*>(sp + RT_WARPS * (E + RT_MAXK)) + warp * RT_MAXK;
  route_row(logits + (int64_t)s * E, E, k, norm_topk, weights_scale, p, selw, seli, lane, ids + (int64_t)s * k,
            wout + (int64_t)s * k);
}

void launch_route(const float* logits, int n_tok, int E, int k, int norm_topk, float weights_scale, int* ids,
                  float* w, cudaStream_t st, const int* fail) {
  if (n_tok <= 0) return;
  size_t smem = (size_t)RT_WARPS * (E + 2 * RT_MAXK) * sizeof(float);
  launch_k(route_kernel, ceil_div(n_tok, RT_WARPS), RT_WARPS * 32, smem, st, logits, n_tok, E, k, norm_topk,
           weights_scale, ids, w, fail);
}

// ---------------------------------------------------------------------------
// Dispatch (the permute of transformer.rs:525-551 as metadata): slots are
// grouped by expert in ascending expert id, and within an expert by ascending
// token -- the order of the reference's BTreeMap<expert, Vec<(token, w)>>.
// One block of 1024 threads. Tokens are ranked inside each warp with a
// per-expert bitmask of the warp's tokens (popc of the lower lanes), and
// across warps and rounds with per-expert running bases.

// The dispatch metadata by one 1024-thread block; dsm: (64 E + 3 E + 1) words
// of shared memory.
// rows: every expert's rows go to the int8 list, in entries of at most three
// (list value e | part << 16: rows 3 part .. 3 part + 2 of expert e), and the
// tcgen05 list stays empty -- each row computed as a batch of one would be.
__device__ void dispatch_block(const int* __restrict__ ids, const float* __restrict__ w, int n_tok, int k, int E,
                               const DispatchOut& o, uint32_t* dsm, bool rows) {
  uint32_t* mask = dsm;                                // [32][E]
  int* pref = reinterpret_cast<int*>(dsm + 32 * E);    // [32][E]
  int* cnt = pref + 32 * E;                            // [E]
  int* base = cnt + E;                                 // [E]
  int* offs = base + E;                                // [E+1]
  __shared__ int4 wsum[32];
  const int tid = threadIdx.x, warp = tid / 32, lane = tid & 31;
  for (int e = tid; e < E; e += DP_THREADS) {
    cnt[e] = 0;
    base[e] = 0;
  }
  __syncthreads();
  const int64_t A = (int64_t)n_tok * k;
  for (int64_t i = tid; i < A; i += DP_THREADS) {
    const int e = ids[i];
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  // Block-wide exclusive scan over experts (thread e): slot offsets, positions
  // in the small (1..3 rows) and large (>= 4 rows) lists, and the large
  // experts' 128-slot tile prefix. The small list holds the 3-row experts,
  // then the 2-row, then the 1-row ones (ascending id within each): the
  // decode kernel's units of equal rows then share its groups. Counters
  // packed in 16-bit fields (E <= 1024): y = 3-row | 2-row << 16,
  // z = large | 1-row << 16.
  {
    const int e = tid;
    const int c = e < E ? cnt[e] : 0;
    // rows: z counts the expert's int8 entries instead (ceil(c / 3)).
    const int fl = !rows && c >= 4 ? 1 : 0, ft = fl ? (c + kMmaTileN - 1) / kMmaTileN : 0;
    const int fy = rows ? 0 : (c == 3 ? 1 : (c == 2 ? 1 << 16 : 0));
    const int fz = rows ? (c + 2) / 3 : fl | (c == 1 ? 1 << 16 : 0);
    int4 v = make_int4(c, fy, fz, ft);
#pragma unroll
    for (int sh = 1; sh < 32; sh <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, v.x, sh), y = __shfl_up_sync(0xffffffffu, v.y, sh);
      const int z = __shfl_up_sync(0xffffffffu, v.z, sh), t = __shfl_up_sync(0xffffffffu, v.w, sh);
      if (lane >= sh) {
        v.x += x;
        v.y += y;
        v.z += z;
        v.w += t;
      }
    }
    if (lane == 31) wsum[warp] = v;
    __syncthreads();
    if (warp == 0) {
      int4 u = wsum[lane];
#pragma unroll
      for (int sh = 1; sh < 32; sh <<= 1) {
        const int x = __shfl_up_sync(0xffffffffu, u.x, sh), y = __shfl_up_sync(0xffffffffu, u.y, sh);
        const int z = __shfl_up_sync(0xffffffffu, u.z, sh), t = __shfl_up_sync(0xffffffffu, u.w, sh);
        if (lane >= sh) {
          u.x += x;
          u.y += y;
          u.z += z;
          u.w += t;
        }
      }
      wsum[lane] = u;  // inclusive over warps
    }
    __syncthreads();
    const int4 wb = warp > 0 ? wsum[warp - 1] : make_int4(0, 0, 0, 0);
    const int4 ex = make_int4(wb.x + v.x - c, wb.y + v.y - fy, wb.z + v.z - fz, wb.w + v.w - ft);
    const int4 tot = wsum[31];
    const int n3 = tot.y & 0xFFFF, n2 = tot.y >> 16, n1 = tot.z >> 16, nl = rows ? 0 : tot.z & 0xFFFF;
    if (e < E) {
      offs[e] = ex.x;
      o.offsets[e] = ex.x;
      o.counts[e] = c;
      if (rows) {
        for (int p = 0; p < fz; ++p) o.small_list[ex.z + p] = e | (p << 16);
      } else {
        if (c == 3) o.small_list[ex.y & 0xFFFF] = e;
        if (c == 2) o.small_list[n3 + (ex.y >> 16)] = e;
        if (c == 1) o.small_list[n3 + n2 + (ex.z >> 16)] = e;
      }
      if (fl) {
        o.large_list[ex.z & 0xFFFF] = e;
        o.large_tt[ex.z & 0xFFFF] = ex.w;
      }
    }
    if (e == E - 1) {
      offs[E] = ex.x + c;
      o.offsets[E] = ex.x + c;
      o.n_lists[0] = rows ? tot.z : n3 + n2 + n1;
      o.n_lists[1] = nl;
      o.large_tt[nl] = rows ? 0 : tot.w;
    }
  }
  __syncthreads();
  const uint32_t lt = (1u << lane) - 1u;
  for (int r0 = 0; r0 < n_tok; r0 += DP_THREADS) {
    for (int i = tid; i < 32 * E; i += DP_THREADS) mask[i] = 0u;
    __syncthreads();
    const int s = r0 + tid;
    if (s < n_tok)
      for (int j = 0; j < k; ++j) {
        const int e = ids[(int64_t)s * k + j];
        if (e >= 0 && e < E) atomicOr(&mask[warp * E + e], 1u << lane);
      }
    __syncthreads();
    for (int e = tid; e < E; e += DP_THREADS) {
      int run = base[e];
      for (int wv = 0; wv < 32; ++wv) {
        pref[wv * E + e] = run;
        run += __popc(mask[wv * E + e]);
      }
      base[e] = run;
    }
    __syncthreads();
    if (s < n_tok)
      for (int j = 0; j < k; ++j) {
        int64_t i = (int64_t)s * k + j;
        int e = ids[i];
        if (e < 0 || e >= E) {
          o.tok_slot[i] = 0;
          continue;
        }
        int slot = offs[e] + pref[warp * E + e] + __popc(mask[warp * E + e] & lt);
        o.slot_tok[slot] = s;
        o.slot_w[slot] = w[i];
        o.tok_slot[i] = slot;
      }
    __syncthreads();
  }
}

// dispatch_block's metadata for batches of at most DS_MAXA selections (used
// for decode batches, where it is the faster of the two). An
// expert's slot offset is the number of selections with a smaller id, and
// its place in the int8 (1-3 rows) or tcgen05 (>= 4 rows) list is the number
// of listed experts below it (bitmasks), so thread e needs no block scan;
// a selection's slot adds the earlier tokens that chose the same expert.
constexpr int DS_MAXA = 256;
__device__ void dispatch_small(const int* __restrict__ ids, const float* __restrict__ w, int n_tok, int k, int E,
                               const DispatchOut& o, uint32_t* dsm) {
  int* ids_s = reinterpret_cast<int*>(dsm);        // [A]
  const int nw = (E + 31) / 32;
  uint32_t* small_m = dsm + DS_MAXA;               // [3][32]: experts with 1, 2, 3 rows
  uint32_t* large_m = small_m + 3 * 32;            // [nw] experts with >= 4 rows
  int* cnt_s = reinterpret_cast<int*>(large_m + 32);  // [E]
  const int tid = threadIdx.x, A = n_tok * k;
  for (int i = tid; i < nw; i += DP_THREADS) {
    small_m[i] = small_m[32 + i] = small_m[64 + i] = 0u;
    large_m[i] = 0u;
  }
  for (int i = tid; i < A; i += DP_THREADS) ids_s[i] = ids[i];
  __syncthreads();
  for (int e = tid; e < E; e += DP_THREADS) {
    int c = 0;
    for (int i = 0; i < A; ++i) c += ids_s[i] == e ? 1 : 0;
    cnt_s[e] = c;
    if (c >= 1 && c <= 3) atomicOr(&small_m[32 * (c - 1) + (e >> 5)], 1u << (e & 31));
    if (c >= 4) atomicOr(&large_m[e >> 5], 1u << (e & 31));
  }
  __syncthreads();
  // The small list: 3-row experts, then 2-row, then 1-row (ascending id
  // within each), so that the decode kernel's groups hold units of equal rows.
  int n_of[3] = {0, 0, 0};
  for (int q = 0; q < nw; ++q)
    for (int c = 0; c < 3; ++c) n_of[c] += __popc(small_m[32 * c + q]);
  for (int e = tid; e < E; e += DP_THREADS) {
    const int c = cnt_s[e];
    int less = 0;
    for (int i = 0; i < A; ++i) less += (ids_s[i] >= 0 && ids_s[i] < e) ? 1 : 0;
    o.counts[e] = c;
    o.offsets[e] = less;
    const uint32_t below = (1u << (e & 31)) - 1u;
    if (c >= 1 && c <= 3) {
      const uint32_t* m = small_m + 32 * (c - 1);
      int pos = __popc(m[e >> 5] & below) + (c < 3 ? n_of[2] : 0) + (c < 2 ? n_of[1] : 0);
      for (int q = 0; q < (e >> 5); ++q) pos += __popc(m[q]);
      o.small_list[pos] = e;
    } else if (c >= 4) {
      int pos = __popc(large_m[e >> 5] & below), tt = 0;
      for (int q = 0; q < (e >> 5); ++q) pos += __popc(large_m[q]);
      for (int e2 = 0; e2 < e; ++e2)
        if (cnt_s[e2] >= 4) tt += (cnt_s[e2] + kMmaTileN - 1) / kMmaTileN;
      o.large_list[pos] = e;
      o.large_tt[pos] = tt;
    }
  }
  if (tid == 0) {
    int n_valid = 0, n_small = 0, n_large = 0, tt = 0;
    for (int i = 0; i < A; ++i) n_valid += (ids_s[i] >= 0 && ids_s[i] < E) ? 1 : 0;
    n_small = n_of[0] + n_of[1] + n_of[2];
    for (int q = 0; q < nw; ++q) n_large += __popc(large_m[q]);
    for (int q = 0; q < nw; ++q)
      for (uint32_t m = large_m[q]; m; m &= m - 1u) {
        const int e = 32 * q + __ffs(m) - 1;
        tt += (cnt_s[e] + kMmaTileN - 1) / kMmaTileN;
      }
    o.offsets[E] = n_valid;
    o.n_lists[0] = n_small;
    o.n_lists[1] = n_large;
    o.large_tt[n_large] = tt;
  }
  for (int i = tid; i < A; i += DP_THREADS) {
    const int e = ids_s[i], s = i / k;
    if (e < 0 || e >= E) {
      o.tok_slot[i] = 0;
      continue;
    }
    int slot = 0;
    for (int i2 = 0; i2 < A; ++i2) {
      const int e2 = ids_s[i2];
      slot += ((e2 >= 0 && e2 < e) || (e2 == e && i2 / k < s)) ? 1 : 0;
    }
    o.slot_tok[slot] = s;
    o.slot_w[slot] = w[i];
    o.tok_slot[i] = slot;
  }
}

__global__ void __launch_bounds__(DP_THREADS) dispatch_kernel(const int* __restrict__ ids,
                                                               const float* __restrict__ w, int n_tok, int k, int E,
                                                               DispatchOut o, bool rows) {
  pdl_enter();
  extern __shared__ uint32_t dsm[];
  // Fewer than 4 tokens: no expert has more than 3 rows, so `rows` changes nothing.
  if (n_tok < 4 && n_tok * k <= DS_MAXA) dispatch_small(ids, w, n_tok, k, E, o, dsm);
  else dispatch_block(ids, w, n_tok, k, E, o, dsm, rows);
}

// Route + dispatch for batches of at most 32 tokens (one warp per token), and
// for decode batches (n_tok < 4; rec non-null) the Q8_K records of every
// slot's input row, in one 1024-thread block. Top-k: with at most one
// (token, expert) entry per thread, every entry's rank in its token's stable
// descending order is counted by its own thread (one parallel pass);
// otherwise each token's warp takes k arg-max rounds. With at most 32 tokens,
// each expert's choosers fit one 32-bit token mask (shared atomicOr), so:
// count = popc(mask); slot offsets, list positions and the tile prefix come
// from one warp's scan over the experts (into shared memory; all threads then
// store the metadata); a selection's slot is its expert's offset plus the
// earlier tokens in the mask. Slots are grouped by ascending expert id and
// ascending token within an expert, as dispatch_block orders them.
constexpr int RD_MAXT = DP_THREADS / 32;
// rec_bytes: the tokens' activation records (n_tok * d/256 * kRecK), held in
// shared memory between their quantisation and the copies to the slots.
static size_t rd_smem(int E, int k, size_t rec_bytes) {
  return ((size_t)RD_MAXT * (E + 2 * RT_MAXK) + 5 * (size_t)E + 5 + (size_t)RD_MAXT * k) * 4 + 16 + rec_bytes;
}

// Warp 0 of route_dispatch_kernel: from the experts' token masks, the slot
// offsets, each expert's place in the int8 or tcgen05 list, the tcgen05 tile
// prefix and the totals. Lane l takes experts [e0, e1) (contiguous) and the
// lanes' five partial counts (rows, int8-list entries by row count, tcgen05
// entries, tcgen05 token tiles) are scanned exclusively through shared
// memory (part_s, 5 x 32 ints) in five steps. The int8 list holds the 3-row
// experts, then the 2-row, then the 1-row ones (ascending id within each), so
// that the decode kernel's groups hold units of equal rows; the 3- and 2-row
// counts are packed as 3-row | 2-row << 16 (each at most E <= 1024). Not
// inlined: the kernel also runs it once on all-zero masks before it waits
// for the router, off the critical path. (A register scan with warp shuffles
// measured ~6,000 cycles here against ~1,000 for this one.)
__device__ __noinline__ void rd_scan(const uint32_t* mask_s, int E, bool rows, int* offs_s, int* pos_s, int* tt_s,
                                     int* tot_s, int* part_s, int lane) {
  const int C = (E + 31) / 32, e0 = min(E, lane * C), e1 = min(E, e0 + C);
  int v[5] = {0, 0, 0, 0, 0};  // rows, 3|2-row entries, 1-row (or rows-mode) entries, tcgen05 entries, tiles
  for (int e = e0; e < e1; ++e) {
    const int c = __popc(mask_s[e]);
    v[0] += c;
    if (rows) {
      v[2] += (c + 2) / 3;
      continue;
    }
    v[1] += c == 3 ? 1 : (c == 2 ? 1 << 16 : 0);
    v[2] += c == 1 ? 1 : 0;
    v[3] += c >= 4 ? 1 : 0;
    v[4] += c >= 4 ? (c + kMmaTileN - 1) / kMmaTileN : 0;
  }
  // Inclusive Kogge-Stone scan of the five values over the 32 lanes.
  int inc[5];
#pragma unroll
  for (int j = 0; j < 5; ++j) {
    inc[j] = v[j];
    part_s[j * 32 + lane] = v[j];
  }
  __syncwarp();
#pragma unroll
  for (int sh = 1; sh < 32; sh <<= 1) {
    int add[5];
#pragma unroll
    for (int j = 0; j < 5; ++j) add[j] = lane >= sh ? part_s[j * 32 + lane - sh] : 0;
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 5; ++j) {
      inc[j] += add[j];
      part_s[j * 32 + lane] = inc[j];
    }
    __syncwarp();
  }
  const int ts = part_s[1 * 32 + 31], n1 = part_s[2 * 32 + 31];
  const int n3 = ts & 0xFFFF, n2 = ts >> 16;
  int oc = inc[0] - v[0], os = inc[1] - v[1], ol = inc[3] - v[3], ot = inc[4] - v[4];
  int o3 = os & 0xFFFF, o2 = n3 + (os >> 16), o1 = n3 + n2 + (inc[2] - v[2]);
  for (int e = e0; e < e1; ++e) {
    const int c = __popc(mask_s[e]);
    offs_s[e] = oc;
    oc += c;
    if (rows) {
      pos_s[e] = o1;  // first of the expert's (c + 2) / 3 entries
      o1 += (c + 2) / 3;
    } else if (c == 3) {
      pos_s[e] = o3++;
    } else if (c == 2) {
      pos_s[e] = o2++;
    } else if (c == 1) {
      pos_s[e] = o1++;
    } else if (c >= 4) {
      pos_s[e] = ol++;
      tt_s[e] = ot;
      ot += (c + kMmaTileN - 1) / kMmaTileN;
    }
  }
  if (lane == 31) {
    offs_s[E] = oc;
    tot_s[0] = rows ? n1 : n3 + n2 + n1;
    tot_s[1] = ol;
    tot_s[2] = ot;
  }
}

__global__ void __launch_bounds__(DP_THREADS) route_dispatch_kernel(const float* __restrict__ logits, int n_tok,
                                                                     int E, int k, int norm_topk, float weights_scale,
                                                                     int* __restrict__ ids, float* __restrict__ w,
                                                                     DispatchOut o, const float* __restrict__ x,
                                                                     int d, uint8_t* __restrict__ rec, bool rows) {
  extern __shared__ __align__(16) uint32_t dsm[];
  __shared__ int part_s[5 * 32];                                  // rd_scan's partial counts
  const int SW = E + 2 * RT_MAXK;                                 // per-token scratch: p, selw, seli
  float* scratch = reinterpret_cast<float*>(dsm);                 // [RD_MAXT][SW]
  uint32_t* mask_s = dsm + RD_MAXT * SW;                          // [E] token mask per expert
  int* offs_s = reinterpret_cast<int*>(mask_s + E);               // [E + 1] slot offsets
  int* pos_s = offs_s + E + 1;                                    // [E] place in the int8 / tcgen05 list
  int* tt_s = pos_s + E;                                          // [E] tcgen05 tile prefix
  int* tot_s = tt_s + E;                                          // [4] int8 entries, tcgen05 entries, tiles
  int* slot_tok_s = tot_s + 4;                                    // [RD_MAXT * k]
  uint8_t* tokrec = reinterpret_cast<uint8_t*>(                   // [n_tok][d / 256] records
      (reinterpret_cast<uintptr_t>(slot_tok_s + RD_MAXT * k) + 15) & ~uintptr_t(15));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = d / 256;
  for (int e = threadIdx.x; e < E; e += DP_THREADS) mask_s[e] = 0u;
  __syncthreads();
  // Before the wait for the router (its logits are the only input written by
  // the previous kernel; x was complete before it started, and is read
  // through L2): the tokens' activation records, which do not depend on the
  // routing, into shared memory; and the dispatch scan once on the zero masks
  // (instruction-cache warm-up; its shared outputs are rewritten below).
  if (warp == 0) {
    rd_scan(mask_s, E, rows, offs_s, pos_s, tt_s, tot_s, part_s, lane);
  } else if (rec) {
    for (int task = warp - 1; task < n_tok * nb; task += DP_THREADS / 32 - 1) {
      const int t = task / nb, b = task - t * nb;
      const float4* xp = reinterpret_cast<const float4*>(x + (int64_t)t * d + b * 256 + lane * 8);
      const float4 a0 = __ldcg(xp), a1 = __ldcg(xp + 1);
      const float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      q8k_store_record(v, tokrec + (size_t)task * kRecK, lane);
    }
  }
  pdl_enter();
  float* p = scratch + warp * SW;
  float* selw = p + E;
  int* seli = reinterpret_cast<int*>(selw + RT_MAXK);
  if (n_tok * E <= DP_THREADS) {
    if (warp < n_tok) route_probs(logits + (int64_t)warp * E, E, p, lane);
    __syncthreads();
    const int i = threadIdx.x;
    if (i < n_tok * E) {
      const int t = i / E, e = i - t * E;
      const float* pt = scratch + t * SW;
      const float v = pt[e];
      int rank = 0;
      if ((E & 3) == 0) {
        for (int e2 = 0; e2 < E; e2 += 4) {
          const float4 q = *reinterpret_cast<const float4*>(pt + e2);
          rank += (q.x > v || (q.x == v && e2 < e)) ? 1 : 0;
          rank += (q.y > v || (q.y == v && e2 + 1 < e)) ? 1 : 0;
          rank += (q.z > v || (q.z == v && e2 + 2 < e)) ? 1 : 0;
          rank += (q.w > v || (q.w == v && e2 + 3 < e)) ? 1 : 0;
        }
      } else {
        for (int e2 = 0; e2 < E; ++e2) rank += (pt[e2] > v || (pt[e2] == v && e2 < e)) ? 1 : 0;
      }
      if (rank < k) {
        float* tw = scratch + t * SW + E;
        tw[rank] = v;
        reinterpret_cast<int*>(tw + RT_MAXK)[rank] = e;
        atomicOr(&mask_s[e], 1u << t);
      }
    }
    __syncthreads();
    if (warp < n_tok)
      route_finish(k, norm_topk, weights_scale, selw, seli, lane, ids + (int64_t)warp * k, w + (int64_t)warp * k);
  } else {
    __syncthreads();  // mask_s zeroed
    if (warp < n_tok) {
      route_row(logits + (int64_t)warp * E, E, k, norm_topk, weights_scale, p, selw, seli, lane,
                ids + (int64_t)warp * k, w + (int64_t)warp * k);
      for (int r = lane; r < k; r += 32) atomicOr(&mask_s[seli[r]], 1u << warp);
    }
  }
  __syncthreads();
  if (warp == 0) rd_scan(mask_s, E, rows, offs_s, pos_s, tt_s, tot_s, part_s, lane);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += DP_THREADS) {
    const int c = __popc(mask_s[e]);
    o.offsets[e] = offs_s[e];
    o.counts[e] = c;
    if (rows) {
      for (int p = 0; p < (c + 2) / 3; ++p) o.small_list[pos_s[e] + p] = e | (p << 16);
    } else if (c >= 1 && c <= 3) {
      o.small_list[pos_s[e]] = e;
    } else if (c >= 4) {
      o.large_list[pos_s[e]] = e;
      o.large_tt[pos_s[e]] = tt_s[e];
    }
  }
  if (threadIdx.x == DP_THREADS - 1) {
    o.offsets[E] = offs_s[E];
    o.n_lists[0] = tot_s[0];
    o.n_lists[1] = tot_s[1];
    o.large_tt[tot_s[1]] = tot_s[2];
  }
  const int A = n_tok * k;
  for (int i = threadIdx.x; i < A; i += DP_THREADS) {
    const int t = i / k, j = i - t * k;
    const float* tw = scratch + t * SW + E;  // token t's final weights (selw), then ids (seli)
    const int e = reinterpret_cast<const int*>(tw + RT_MAXK)[j];
    const int slot = offs_s[e] + __popc(mask_s[e] & ((1u << t) - 1u));
    o.slot_tok[slot] = t;
    o.slot_w[slot] = tw[j];
    o.tok_slot[i] = slot;
    slot_tok_s[slot] = t;
  }
  if (!rec) return;
  __syncthreads();
  // Each slot's records are its token's (16-byte copies from shared memory).
  constexpr int R16 = kRecK / 16;
  for (int i = threadIdx.x; i < A * nb * R16; i += DP_THREADS) {
    const int slot = i / (nb * R16), r = i - slot * nb * R16, b = r / R16, j = r - b * R16;
    const uint4 v = *reinterpret_cast<const uint4*>(tokrec + ((size_t)slot_tok_s[slot] * nb + b) * kRecK + 16 * j);
    *reinterpret_cast<uint4*>(rec + rec_index(b, slot, A) * kRecK + 16 * j) = v;
  }
}

bool route_dispatch_supported(int n_tok, int E, int k, int d, bool with_records) {
  const bool tok_ok = with_records ? (n_tok < 4 && d % 256 == 0) : n_tok <= RD_MAXT;
  return n_tok >= 1 && tok_ok && E >= 1 && E <= DP_THREADS && k >= 1 && k <= RT_MAXK && k <= E &&
         rd_smem(E, k, with_records ? (size_t)n_tok * (d / 256) * kRecK : 0) <= 200 * 1024;
}

void launch_route_dispatch(const float* logits, int n_tok, int E, int k, int norm_topk, float weights_scale, int* ids,
                           float* w, const DispatchOut& o, const float* x, int d, uint8_t* rec, cudaStream_t st,
                           bool rows) {
  static PerDeviceOnce attr;
  smem_attr_once(attr, route_dispatch_kernel, 200 * 1024);
  launch_k(route_dispatch_kernel, 1, DP_THREADS, rd_smem(E, k, rec ? (size_t)n_tok * (d / 256) * kRecK : 0), st,
           logits, n_tok, E, k, norm_topk, weights_scale,
           ids, w, o, x, d, rec, rows);
}

int launch_dispatch(const int* ids, const float* w, int n_tok, int k, int E, const DispatchOut& o, cudaStream_t st,
                    bool rows) {
  size_t smem = std::max((size_t)(64 * E + 3 * E + 1), (size_t)(DS_MAXA + 128 + E)) * 4;
  static PerDeviceOnce attr;
  smem_attr_once(attr, dispatch_kernel, 200 * 1024);
  if (smem > 200 * 1024 || E > DP_THREADS) return KC_ERR_SHAPE;
  launch_k(dispatch_kernel, 1, DP_THREADS, smem, st, ids, w, n_tok, k, E, o, rows);
  return KC_OK;
}

// One group (expert 0) holding rows 0..n-1: the metadata of a dense product.
// rows: groups g of rows 3g .. 3g + 2 instead (all on the int8 path; the
// product's matrix is shared by every group).
__global__ void dense_meta_kernel(int n, DispatchOut o, bool rows) {
  pdl_enter();
  if (rows) {
    const int ng = (n + 2) / 3;
    for (int g = 0; g < ng; ++g) {
      o.counts[g] = min(3, n - 3 * g);
      o.offsets[g] = 3 * g;
      o.small_list[g] = g;
    }
    o.offsets[ng] = n;
    o.n_lists[0] = ng;
    o.n_lists[1] = 0;
    o.large_tt[0] = 0;
    return;
  }
  o.counts[0] = n;
  o.offsets[0] = 0;
  o.offsets[1] = n;
  o.small_list[0] = 0;
  o.large_list[0] = 0;
  o.n_lists[0] = (n >= 1 && n <= 3) ? 1 : 0;
  o.n_lists[1] = n >= 4 ? 1 : 0;
  o.large_tt[0] = 0;
  o.large_tt[1] = n >= 4 ? (n + kMmaTileN - 1) / kMmaTileN : 0;
}

void launch_dense_meta(int n, const DispatchOut& o, cudaStream_t st, bool rows) {
  launch_k(dense_meta_kernel, 1, 1, 0, st, n, o, rows);
}

// ---------------------------------------------------------------------------
// Combine (transformer.rs:566-570): out[s] = sum over the token's experts in
// ascending expert id of w * y, each step a separate multiply and add, from
// +0.0. Block (token, column slice): CB_THREADS threads x 4 columns; every
// block orders its token's selections itself (k <= RT_MAXK <= CB_THREADS).
__global__ void combine_kernel(const float* __restrict__ y, const int* __restrict__ tok_slot,
                               const int* __restrict__ ids, const float* __restrict__ w, int k, int d,
                               float* __restrict__ out) {
  pdl_enter();
  __shared__ int ea[64], ss[64];
  __shared__ float sw[64];
  const int s = blockIdx.x;
  // Order the token's k selections by expert id: entry j goes to position
  // rank(j) = number of its selections with a smaller id (ids are distinct).
  const int t = threadIdx.x;
  int e = 0, slot = 0;
  float wj = 0.f;
  if (t < k) {
    e = ids[(int64_t)s * k + t];
    slot = tok_slot[(int64_t)s * k + t];
    wj = w[(int64_t)s * k + t];
    ea[t] = e;
  }
  __syncthreads();
  if (t < k) {
    int rank = 0;
    for (int i = 0; i < k; ++i) rank += (ea[i] < e || (ea[i] == e && i < t)) ? 1 : 0;
    ss[rank] = slot;
    sw[rank] = wj;
  }
  __syncthreads();
  const int c_end = min(d, (int)(blockIdx.y + 1) * 4 * (int)blockDim.x);
  for (int c = (int)blockIdx.y * 4 * blockDim.x + threadIdx.x * 4; c < c_end; c += blockDim.x * 4) {
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < k; ++j) {
      float4 v = *reinterpret_cast<const float4*>(y + (int64_t)ss[j] * d + c);
      float wj = sw[j];
      o.x = __fadd_rn(o.x, __fmul_rn(wj, v.x));
      o.y = __fadd_rn(o.y, __fmul_rn(wj, v.y));
      o.z = __fadd_rn(o.z, __fmul_rn(wj, v.z));
      o.w = __fadd_rn(o.w, __fmul_rn(wj, v.w));
    }
    *reinterpret_cast<float4*>(out + (int64_t)s * d + c) = o;
  }
}

constexpr int CB_THREADS = 64;
static_assert(RT_MAXK <= CB_THREADS, "one thread per selection");
void launch_combine(const float* y, const int* tok_slot, const int* ids, const float* w, int n_tok, int k, int d,
                    float* out, cudaStream_t st) {
  if (n_tok <= 0) return;
  // Column slices of 256 floats, so that a decode-sized batch spreads over
  // many SMs (the k rows each slice reads are its whole cost).
  launch_k(combine_kernel, dim3(n_tok, ceil_div(d, 4 * CB_THREADS)), CB_THREADS, 0, st, y, tok_slot, ids, w, k, d,
           out);
}

// ---------------------------------------------------------------------------
// Shared expert (qwen2moe, transformer.rs:577-585): gate = 1 / (1 + exp(-dot)),
// then out += gate * y elementwise (multiply, then add). One thread per 4
// floats.
__global__ void shared_add_kernel(const float* __restrict__ y, const float* __restrict__ logit, int n_tok, int d,
                                  float* __restrict__ out) {
  pdl_enter();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t per = d / 4;
  if (i >= (int64_t)n_tok * per) return;
  const int64_t s = i / per;
  const float g = logit ? __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_rn(-logit[s]))) : 1.0f;
  const float4 v = reinterpret_cast<const float4*>(y)[i];
  float4 o = reinterpret_cast<float4*>(out)[i];
  o.x = __fadd_rn(o.x, __fmul_rn(g, v.x));
  o.y = __fadd_rn(o.y, __fmul_rn(g, v.y));
  o.z = __fadd_rn(o.z, __fmul_rn(g, v.z));
  o.w = __fadd_rn(o.w, __fmul_rn(g, v.w));
  reinterpret_cast<float4*>(out)[i] = o;
}

void launch_shared_add(const float* y, const float* logit, int n_tok, int d, float* out, cudaStream_t st) {
  const int64_t n = (int64_t)n_tok * (d / 4);
  if (n <= 0) return;
  launch_k(shared_add_kernel, ceil_div(n, 256), 256, 0, st, y, logit, n_tok, d, out);
}

}  // namespace kc
