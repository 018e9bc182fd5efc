// Dense decode path kernels (model.h): embedding rows, residual add +
// RMSNorm, q/k post-processing with the f16 KV cache, causal GQA attention,
// argmax and the dense SwiGLU. Each follows the reference's operation order
// (transformer.rs:330-358, 375-467, 594-631) with separate multiplies and
// adds (the library is built with --fmad=false).
//
// Sums the reference folds sequentially (RMSNorm's sum of squares, the
// attention softmax denominator) are folded by one thread in the same order;
// only their independent terms are computed in parallel. exp is exp_rn
// (common.cuh).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "decode.h"
#include "model.h"

namespace kc {

__device__ __forceinline__ float h2f_at(const uint8_t* p) {
  return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

// scale_min_k4 (quant.rs:54-60).
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t* q, int& d, int& m) {
  if (j < 4) {
    d = q[j] & 63;
    m = q[j + 4] & 63;
  } else {
    d = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

// Element j of a GGUF row (dequant_row, quant.rs:63-205).
__device__ float dequant_elem(int t, const uint8_t* row, int j) {
  if (t == T_F32) return reinterpret_cast<const float*>(row)[j];
  if (t == T_Q8_0) {
    const uint8_t* blk = row + (j / 32) * 34;
    return __fmul_rn((float)(int8_t)blk[2 + j % 32], h2f_at(blk));
  }
  if (t == T_Q4_K) {
    const uint8_t* blk = row + (j / 256) * 144;
    const int r = j % 256, k = r / 64, l = r % 64, hi = l >= 32, ll = l % 32;
    int s, m;
    scale_min_k4(2 * k + hi, blk + 4, s, m);
    const float dl = __fmul_rn(h2f_at(blk), (float)s), ml = __fmul_rn(h2f_at(blk + 2), (float)m);
    const uint8_t q = blk[16 + 32 * k + ll];
    return __fsub_rn(__fmul_rn(dl, (float)(hi ? q >> 4 : q & 0xF)), ml);
  }
  if (t == T_Q6_K) {
    const uint8_t* blk = row + (j / 256) * 210;
    const int r = j % 256, h = r / 128, qr = (r % 128) / 32, l = r % 32, is = l / 16;
    const uint8_t* ql = blk + h * 64;
    const uint8_t* qh = blk + 128 + h * 32;
    const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192 + h * 8);
    const uint8_t lo = qr & 1 ? ql[l + 32] : ql[l];
    const int nib = qr >= 2 ? lo >> 4 : lo & 0xF;
    const int q = (nib | (((qh[l] >> (2 * qr)) & 3) << 4)) - 32;
    return __fmul_rn(__fmul_rn(h2f_at(blk + 208), (float)sc[is + 2 * qr]), (float)q);
  }
  return 0.f;
}

__global__ void embed_kernel(const uint8_t* __restrict__ E, int t, int64_t row_bytes, const uint32_t* __restrict__ tok,
                             int d, int n_vocab, float* __restrict__ x, int* status) {
  pdl_enter();
  const int s = blockIdx.x;
  const uint32_t id = tok[s];
  const bool ok = id < (uint32_t)n_vocab;
  if (!ok && threadIdx.x == 0) report(status, KC_ERR_ARG);
  const uint8_t* row = E + (int64_t)(ok ? id : 0) * row_bytes;
  for (int j = threadIdx.x; j < d; j += blockDim.x) x[(int64_t)s * d + j] = ok ? dequant_elem(t, row, j) : 0.f;
}

void launch_embed(const uint8_t* E, int t, int64_t row_bytes, const uint32_t* tok, int n, int d, int n_vocab,
                  float* x, int* status, cudaStream_t st) {
  if (n <= 0) return;
  launch_k(embed_kernel, n, 256, 0, st, E, t, row_bytes, tok, d, n_vocab, x, status);
}

// 1 / sqrt(sum / dim + eps) of the squares sq[0..dim) (16-byte aligned) folded
// in order from -0.0 (Rust's f32 Sum, transformer.rs:333) by one warp. For
// dim % 32 == 0 lane 0 runs the whole chain, reading the squares 32 at a time
// with the next 32 requested before the current ones are added, so the chain
// of dependent adds neither waits on a shared-memory load nor hands the sum
// from lane to lane. Otherwise, per pass of 1024 squares, lane l holds squares
// 32 l .. 32 l + 31 in registers and the running sum visits the lanes in order.
__device__ float rms_inv_warp(const float* sq, int dim, float eps, int lane) {
  float ss = -0.0f;
  if (dim % 32 == 0) {
    if (lane == 0) {
      const float4* q = reinterpret_cast<const float4*>(sq);
      float4 cur[8], nxt[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) cur[u] = q[u];
      for (int i = 0; i < dim / 4; i += 8) {
        if (i + 8 < dim / 4) {
#pragma unroll
          for (int u = 0; u < 8; ++u) nxt[u] = q[i + 8 + u];
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          ss = __fadd_rn(ss, cur[u].x);
          ss = __fadd_rn(ss, cur[u].y);
          ss = __fadd_rn(ss, cur[u].z);
          ss = __fadd_rn(ss, cur[u].w);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) cur[u] = nxt[u];
      }
    }
    ss = __shfl_sync(0xffffffffu, ss, 0);
    ss = __fdiv_rn(ss, (float)dim);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ss, eps)));
  }
  for (int base = 0; base < dim; base += 1024) {
    const int n = min(1024, dim - base);
    float v[32];
    const int l0 = lane * 32;
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      if (l0 + i + 3 < n) {
        const float4 q = *reinterpret_cast<const float4*>(sq + base + l0 + i);
        v[i] = q.x; v[i + 1] = q.y; v[i + 2] = q.z; v[i + 3] = q.w;
      } else {
#pragma unroll
        for (int u = 0; u < 4; ++u) v[i + u] = l0 + i + u < n ? sq[base + l0 + i + u] : 0.f;
      }
    }
    const int lanes = (n + 31) / 32;
    for (int l = 0; l < lanes; ++l) {
      if (lane == l) {
        const int cnt = min(32, n - l0);
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < cnt) ss = __fadd_rn(ss, v[i]);
      }
      ss = __shfl_sync(0xffffffffu, ss, l);
    }
  }
  ss = __fdiv_rn(ss, (float)dim);
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ss, eps)));
}

// One CTA per row: x += (y or the MoE combine of the row's token), then
// out = rmsnorm(x, w), and optionally the Q8_K records of out. The squares
// are formed in parallel; warp 0 folds them (rms_inv_warp). The combine is
// combine_kernel's arithmetic: the token's k selections ordered by expert id,
// c = 0; c += w * y in that order (transformer.rs:566-570), then x + c.
constexpr int NORM_THREADS = 256;
__global__ void __launch_bounds__(NORM_THREADS) add_rmsnorm_kernel(NormArgs a) {
  pdl_enter();
  extern __shared__ __align__(16) float sq[];
  __shared__ float r_s;
  __shared__ int c_slot[64];
  __shared__ float c_w[64];
  const int dim = a.dim, tid = threadIdx.x;
  float* xr = a.x + (int64_t)blockIdx.x * dim;
  if (a.cy) {
    const int t = a.tok0 + blockIdx.x;
    if (tid < a.k) {
      const int e = a.ids[(int64_t)t * a.k + tid];
      int rank = 0;
      for (int i = 0; i < a.k; ++i) {
        const int ei = a.ids[(int64_t)t * a.k + i];
        rank += (ei < e || (ei == e && i < tid)) ? 1 : 0;
      }
      c_slot[rank] = a.tok_slot[(int64_t)t * a.k + tid];
      c_w[rank] = a.cw[(int64_t)t * a.k + tid];
    }
    __syncthreads();
  }
  // Four consecutive elements per thread and step (dim % 4 == 0): 16-byte
  // loads, and the k expert rows of the combine loaded before they are added.
  for (int j = 4 * tid; j < dim; j += 4 * blockDim.x) {
    float4 v = *reinterpret_cast<const float4*>(xr + j);
    if (a.y) {
      const float4 y = *reinterpret_cast<const float4*>(a.y + (int64_t)blockIdx.x * dim + j);
      v = make_float4(__fadd_rn(v.x, y.x), __fadd_rn(v.y, y.y), __fadd_rn(v.z, y.z), __fadd_rn(v.w, y.w));
      *reinterpret_cast<float4*>(xr + j) = v;
    } else if (a.cy) {
      float4 c = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int i0 = 0; i0 < a.k; i0 += 8) {
        float4 yv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (i0 + i < a.k) yv[i] = *reinterpret_cast<const float4*>(a.cy + (int64_t)c_slot[i0 + i] * dim + j);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (i0 + i < a.k) {
            const float wv = c_w[i0 + i];
            c.x = __fadd_rn(c.x, __fmul_rn(wv, yv[i].x));
            c.y = __fadd_rn(c.y, __fmul_rn(wv, yv[i].y));
            c.z = __fadd_rn(c.z, __fmul_rn(wv, yv[i].z));
            c.w = __fadd_rn(c.w, __fmul_rn(wv, yv[i].w));
          }
      }
      v = make_float4(__fadd_rn(v.x, c.x), __fadd_rn(v.y, c.y), __fadd_rn(v.z, c.z), __fadd_rn(v.w, c.w));
      *reinterpret_cast<float4*>(xr + j) = v;
    }
    *reinterpret_cast<float4*>(sq + j) =
        make_float4(__fmul_rn(v.x, v.x), __fmul_rn(v.y, v.y), __fmul_rn(v.z, v.z), __fmul_rn(v.w, v.w));
  }
  __syncthreads();
  if (tid < 32) {
    const float r = rms_inv_warp(sq, dim, a.eps, tid);
    if (tid == 0) r_s = r;
  }
  __syncthreads();
  const float r = r_s;
  for (int j = 4 * tid; j < dim; j += 4 * blockDim.x) {
    const float4 xv = *reinterpret_cast<const float4*>(xr + j);
    const float4 wv = *reinterpret_cast<const float4*>(a.w + j);
    const float4 o = make_float4(__fmul_rn(__fmul_rn(xv.x, r), wv.x), __fmul_rn(__fmul_rn(xv.y, r), wv.y),
                                 __fmul_rn(__fmul_rn(xv.z, r), wv.z), __fmul_rn(__fmul_rn(xv.w, r), wv.w));
    if (a.out) *reinterpret_cast<float4*>(a.out + (int64_t)blockIdx.x * dim + j) = o;
    *reinterpret_cast<float4*>(sq + j) = o;
  }
  if (!a.rec) return;
  __syncthreads();
  const int warp = tid >> 5, lane = tid & 31;
  for (int b = warp; b < dim / 256; b += NORM_THREADS / 32) {
    float v[8];
    const float4 p0 = reinterpret_cast<const float4*>(sq + b * 256 + lane * 8)[0];
    const float4 p1 = reinterpret_cast<const float4*>(sq + b * 256 + lane * 8)[1];
    v[0] = p0.x; v[1] = p0.y; v[2] = p0.z; v[3] = p0.w; v[4] = p1.x; v[5] = p1.y; v[6] = p1.z; v[7] = p1.w;
    q8k_store_record(v, a.rec + rec_index(b, blockIdx.x, a.rec_slots) * kRecK, lane);
  }
}

void launch_add_rmsnorm(const NormArgs& a, int rows, cudaStream_t st) {
  if (rows <= 0) return;
  launch_k(add_rmsnorm_kernel, rows, NORM_THREADS, (size_t)a.dim * 4, st, a);
}

void launch_add_rmsnorm(float* x, const float* y, const float* w, int rows, int dim, float eps, float* out,
                        cudaStream_t st) {
  NormArgs a{};
  a.x = x;
  a.y = y;
  a.w = w;
  a.dim = dim;
  a.eps = eps;
  a.out = out;
  launch_add_rmsnorm(a, rows, st);
}

// One warp per (token, head); the head's hd values live in shared memory.
constexpr int QK_MAX_HD = 256;
__global__ void __launch_bounds__(32) qk_post_kernel(QkPostArgs a) {
  pdl_enter();
  __shared__ float v[QK_MAX_HD];
  __shared__ __align__(16) float sq[QK_MAX_HD];
  __shared__ float r_s;
  const int s = blockIdx.x, head = blockIdx.y, lane = threadIdx.x;
  const int hd = a.hd;
  const int kind = head < a.nh ? 0 : (head < a.nh + a.nkv ? 1 : 2);  // q, k, v
  const int hi = kind == 0 ? head : (kind == 1 ? head - a.nh : head - a.nh - a.nkv);
  const int width = (a.nh + 2 * a.nkv) * hd;
  const float* src = a.qkv + (int64_t)s * width + (int64_t)head * hd;
  const float* bias = kind == 0 ? a.bq : (kind == 1 ? a.bk : a.bv);
  for (int j = lane; j < hd; j += 32) v[j] = bias ? __fadd_rn(src[j], bias[hi * hd + j]) : src[j];
  __syncwarp();
  const float* nw = kind == 0 ? a.qn : (kind == 1 ? a.kn : nullptr);
  if (nw) {
    for (int j = lane; j < hd; j += 32) sq[j] = __fmul_rn(v[j], v[j]);
    __syncwarp();
    const float rr = rms_inv_warp(sq, hd, a.eps, lane);
    if (lane == 0) r_s = rr;
    __syncwarp();
    const float r = r_s;
    for (int j = lane; j < hd; j += 32) v[j] = __fmul_rn(__fmul_rn(v[j], r), nw[j]);
    __syncwarp();
  }
  const int pos = a.row_pos ? a.row_pos[s] : (a.pos_dev ? *a.pos_dev : a.pos0) + s;
  const int64_t seq_off = a.row_pos ? (int64_t)s * a.seq_stride : 0;
  if (kind < 2) {
    const int half = a.rd / 2;
    const float2* tab = a.rope + (int64_t)pos * half;
    for (int i = lane; i < half; i += 32) {
      const int ia = a.neox ? i : 2 * i, ib = a.neox ? i + half : 2 * i + 1;
      const float x0 = v[ia], x1 = v[ib];
      const float sn = tab[i].x, cs = tab[i].y;
      v[ia] = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
      v[ib] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
    }
    __syncwarp();
  }
  if (kind == 0) {
    float* q = a.q_out + ((int64_t)s * a.nh + hi) * hd;
    for (int j = lane; j < hd; j += 32) q[j] = v[j];
  } else {
    __half* c = (kind == 1 ? a.kc : a.vc) + seq_off + (int64_t)pos * a.nkv * hd + (int64_t)hi * hd;
    for (int j = lane; j < hd; j += 32) c[j] = __float2half_rn(v[j]);
  }
}

void launch_qk_post(const QkPostArgs& a, cudaStream_t st) {
  if (a.n <= 0) return;
  launch_k(qk_post_kernel, dim3(a.n, a.nh + 2 * a.nkv), 32, 0, st, a);
}

// One CTA per (query, head). K and V of the head's KV group are staged
// through shared memory in chunks of ATT_PC positions with 16-byte coalesced
// loads. Scores: quant::dot's eight accumulators per position (quant.rs:
// 208-224) -- thread (position, i) forms accumulator i over the 8-element
// chunks in order, and the position's first thread folds the eight from -0.0
// -- then * scale. The max is exact in any order; the exp'd scores are summed
// by one thread in position order from +0.0; each output element then
// accumulates (score * inv) * v over the positions in order.
constexpr int ATT_THREADS = 256;
constexpr int ATT_PC = 128;  // positions per staged chunk (two buffers)

// n_rows rows of hd halves (hd % 8 == 0: 16-byte pieces) into dst with
// asynchronous copies, committed as one group.
__device__ __forceinline__ void stage_rows_async(__half* dst, const __half* src, int n_rows, int hd,
                                                 int64_t row_stride, int tid) {
  const int per_row = hd / 8;
  for (int i = tid; i < n_rows * per_row; i += ATT_THREADS) {
    const int r = i / per_row, c = i - r * per_row;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst + (int64_t)r * hd + c * 8)),
                 "l"(src + r * row_stride + c * 8)
                 : "memory");
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// The chunk loop over positions 0 .. n_pos-1 of one cache (K or V) with two
// staging buffers of ATT_PC rows: chunk c + 1 is requested before chunk c is
// used, so the cache reads overlap the work on the previous chunk.
// body(p0, np, rows) gets the rows [np][hd] of positions p0 ...
template <class Body>
__device__ __forceinline__ void for_cache_chunks(__half* buf, const __half* base, int n_pos, int hd, int64_t kvw,
                                                 int tid, Body body) {
  const int n_chunks = (n_pos + ATT_PC - 1) / ATT_PC;
  __syncthreads();
  stage_rows_async(buf, base, min(ATT_PC, n_pos), hd, kvw, tid);
  for (int ci = 0; ci < n_chunks; ++ci) {
    const int p0 = ci * ATT_PC, np = min(ATT_PC, n_pos - p0);
    if (ci + 1 < n_chunks)
      stage_rows_async(buf + ((ci + 1) & 1) * ATT_PC * hd, base + (int64_t)(p0 + ATT_PC) * kvw,
                       min(ATT_PC, n_pos - p0 - ATT_PC), hd, kvw, tid);
    else
      asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 1;" ::: "memory");  // chunk c has landed
    __syncthreads();
    body(p0, np, buf + (ci & 1) * ATT_PC * hd);
    __syncthreads();
  }
}

__global__ void __launch_bounds__(ATT_THREADS) attention_kernel(const float* __restrict__ q,
                                                                const __half* __restrict__ kc,
                                                                const __half* __restrict__ vc, int nh, int nkv,
                                                                int hd, int pos0, const int* __restrict__ pos_dev,
                                                                float scale, float* __restrict__ out,
                                                                const int* __restrict__ row_pos, int64_t seq_stride) {
  pdl_enter();
  extern __shared__ __align__(16) float sm[];
  float* qs = sm;                                        // [hd]
  __half* ks = reinterpret_cast<__half*>(sm + hd);      // [2][ATT_PC][hd] (K, then V)
  float* sc = sm + hd + ATT_PC * hd;                     // [n_pos]
  __shared__ float red[ATT_THREADS / 32];
  __shared__ float inv_s;
  const int s = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, lane = tid & 31;
  const int kvh = h / (nh / nkv), kvw = nkv * hd;
  if (pos_dev) pos0 = *pos_dev;
  // Row s is query position pos0 + s of one sequence, or (row_pos) its own
  // sequence at position row_pos[s].
  const int n_pos = row_pos ? row_pos[s] + 1 : pos0 + s + 1;
  const int64_t seq_off = row_pos ? (int64_t)s * seq_stride : 0;
  for (int j = tid; j < hd; j += ATT_THREADS) qs[j] = q[((int64_t)s * nh + h) * hd + j];
  const __half* kbase = kc + seq_off + (int64_t)kvh * hd;
  const __half* vbase = vc + seq_off + (int64_t)kvh * hd;
  const int n8 = hd / 8;
  float mx = -INFINITY;
  for_cache_chunks(ks, kbase, n_pos, hd, kvw, tid, [&](int p0, int np, const __half* kch) {
    // Whole warps take part in every iteration (the shuffles below): the
    // bound is rounded up to 32 and positions past np compute nothing.
    const int tot = (np * 8 + 31) & ~31;
    for (int t = tid; t < tot; t += ATT_THREADS) {
      const int pp = t >> 3, i = t & 7;
      const bool valid = pp < np;
      const __half* kr = kch + (valid ? pp : 0) * hd;
      float acc = 0.f;
      if (valid)
        for (int m = 0; m < n8; ++m) acc = __fadd_rn(acc, __fmul_rn(qs[8 * m + i], __half2float(kr[8 * m + i])));
      // Fold the position's eight accumulators in order (8-lane groups are
      // aligned within the warp: t and tid share their low 3 bits).
      float d = -0.0f;
#pragma unroll
      for (int ii = 0; ii < 8; ++ii) d = __fadd_rn(d, __shfl_sync(0xffffffffu, acc, (lane & ~7) + ii));
      if (valid && i == 0) {
        for (int c = n8 * 8; c < hd; ++c) d = __fadd_rn(d, __fmul_rn(qs[c], __half2float(kr[c])));
        const float v = __fmul_rn(d, scale);
        sc[p0 + pp] = v;
        mx = fmaxf(mx, v);
      }
    }
  });
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[tid >> 5] = mx;
  __syncthreads();
  mx = red[0];
  for (int i = 1; i < ATT_THREADS / 32; ++i) mx = fmaxf(mx, red[i]);
  for (int p = tid; p < n_pos; p += ATT_THREADS) sc[p] = exp_rn(__fsub_rn(sc[p], mx));
  __syncthreads();
  if (tid == 0) {
    float sum = 0.0f;
    for (int p = 0; p < n_pos; ++p) sum = __fadd_rn(sum, sc[p]);
    inv_s = __fdiv_rn(1.0f, sum);
  }
  __syncthreads();
  const float inv = inv_s;
  float o = 0.0f;
  for_cache_chunks(ks, vbase, n_pos, hd, kvw, tid, [&](int p0, int np, const __half* vch) {
    if (tid < hd)
      for (int pp = 0; pp < np; ++pp)
        o = __fadd_rn(o, __fmul_rn(__fmul_rn(sc[p0 + pp], inv), __half2float(vch[pp * hd + tid])));
  });
  if (tid < hd) out[((int64_t)s * nh + h) * hd + tid] = o;
}

int attention_max_positions(int hd) { return 200 * 1024 / 4 - hd - ATT_PC * hd; }

void launch_attention(const float* q, const __half* kc, const __half* vc, int n, int nh, int nkv, int hd, int pos0,
                      const int* pos_dev, int max_pos, float scale, float* out, cudaStream_t st, const int* row_pos,
                      int64_t seq_stride) {
  if (n <= 0) return;
  // With the position on the device (graph replays, rows of sequences),
  // shared memory is sized for max_pos positions.
  const size_t smem = (size_t)(hd + ATT_PC * hd + (pos_dev || row_pos ? max_pos : pos0 + n)) * 4;
  static PerDeviceOnce attr;
  smem_attr_once(attr, attention_kernel, 200 * 1024);
  launch_k(attention_kernel, dim3(n, nh), ATT_THREADS, smem, st, q, kc, vc, nh, nkv, hd, pos0, pos_dev, scale, out,
           row_pos, seq_stride);
}

// One CTA: strided scans keep the first maximum of each thread, then a
// reduction that prefers the larger value and, on equal values, the lower
// index. A NaN never compares greater, so it is never chosen, except at
// index 0, where the reference's scan starts.
constexpr int AM_THREADS = 1024;
__global__ void __launch_bounds__(AM_THREADS) argmax_kernel(const float* __restrict__ l, int n, uint32_t* out) {
  pdl_enter();
  l += (int64_t)blockIdx.x * n;  // row blockIdx.x
  out += blockIdx.x;
  __shared__ float bv[AM_THREADS / 32];
  __shared__ int bi[AM_THREADS / 32];
  const int tid = threadIdx.x;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int i = tid; i < n; i += blockDim.x) {
    const float v = l[i];
    if (idx == 0x7fffffff ? !(v != v) : v > best) {
      best = v;
      idx = i;
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (oi != 0x7fffffff && (idx == 0x7fffffff || ov > best || (ov == best && oi < idx))) {
      best = ov;
      idx = oi;
    }
  }
  if ((tid & 31) == 0) {
    bv[tid >> 5] = best;
    bi[tid >> 5] = idx;
  }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < AM_THREADS / 32; ++w)
      if (bi[w] != 0x7fffffff && (idx == 0x7fffffff || bv[w] > best || (bv[w] == best && bi[w] < idx))) {
        best = bv[w];
        idx = bi[w];
      }
    const float l0 = l[0];
    *out = (l0 != l0 || idx == 0x7fffffff) ? 0u : (uint32_t)idx;
  }
}

void launch_argmax(const float* l, int n, uint32_t* out, cudaStream_t st, int rows) {
  launch_k(argmax_kernel, std::max(1, rows), AM_THREADS, 0, st, l, n, out);
}

__global__ void swiglu_kernel(float* __restrict__ g, const float* __restrict__ u, int64_t n) {
  pdl_enter();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float gv = g[i];
    g[i] = __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, exp_rn(-gv))), u[i]);
  }
}

void launch_swiglu(float* g, const float* u, int64_t n, cudaStream_t st) {
  if (n <= 0) return;
  launch_k(swiglu_kernel, (int)std::min<int64_t>(ceil_div(n, 256), 4 * 148), 256, 0, st, g, u, n);
}

}  // namespace kc

namespace kc {
// End of a graph-replayed decode step: append the step's argmax to the
// history and advance the step and position counters.
__global__ void advance_kernel(const uint32_t* next, uint32_t* hist, int* step, int* pos) {
  pdl_enter();
  hist[*step] = *next;
  *step += 1;
  *pos += 1;
}

void launch_advance(const uint32_t* next, uint32_t* hist, int* step, int* pos, cudaStream_t st) {
  launch_k(advance_kernel, 1, 1, 0, st, next, hist, step, pos);
}

__global__ void advance_rows_kernel(const uint32_t* next, uint32_t* hist, int64_t hist_stride, int n, int* step,
                                    int* pos) {
  pdl_enter();
  const int s = threadIdx.x;
  const int t = *step;
  __syncthreads();  // every thread has read the step before thread 0 moves it
  if (s < n) {
    hist[(int64_t)s * hist_stride + t] = next[s];
    pos[s] += 1;
  }
  if (s == 0) *step = t + 1;
}

void launch_advance_rows(const uint32_t* next, uint32_t* hist, int64_t hist_stride, int n, int* step, int* pos,
                         cudaStream_t st) {
  launch_k(advance_rows_kernel, 1, std::max(32, (n + 31) / 32 * 32), 0, st, next, hist, hist_stride, n, step, pos);
}
}  // namespace kc
