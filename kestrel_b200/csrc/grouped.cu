// Grouped quantized products over the routed experts (and the dense matvec).
//
// int8 path (experts with 1..3 rows; dense products with n < 4): the
// reference's Q8_K / Q8Row kernels (avx2.rs:49-58, 351-419), bit for bit.
// Weights stream HBM -> shared memory through a ring of bulk async copies
// (cp.async.bulk + mbarrier); one producer warp issues the copies, four
// consumer warps compute. Each weight row is owned by eight threads, thread j
// holding the j-th 32-bit lane of the reference's AVX2 accumulator: its
// integer sums are complete in-thread, its float FMA chain over superblocks
// runs in the reference's order, and the eight lanes are folded with hsum's
// addition tree. Work units (16 rows of one expert's matrix) are split evenly
// over a persistent grid.
//
// f32 path (experts with >= 4 rows): the reference dequantises exactly and
// runs an f32 GEMM (quant.rs:241-260); this kernel does the same arithmetic
// on CUDA cores (tolerance-checked, not bit-exact).
#include "common.cuh"
#include "kernels.h"

namespace kc {

constexpr int RT = 16;         // rows per work unit
constexpr int CONS_WARPS = 4;  // 8 threads per row
constexpr int I8_THREADS = 32 * (1 + CONS_WARPS);
constexpr int MAX_STAGES = 8;
constexpr int MAXS = 3;        // rows per expert on the int8 path

// Scale and min of Q4_K sub-block 2k+hi for a runtime k (scale_min_k4,
// quant.rs:54-60), from the three words holding the 12 packed bytes.
__device__ __forceinline__ void q4k_sm(int jj, uint32_t w0, uint32_t w1, uint32_t w2, int& s, int& m) {
  int sh = 8 * (jj & 3);
  uint32_t A = (w0 >> sh) & 0xFF, B = (w1 >> sh) & 0xFF, C = (w2 >> sh) & 0xFF;
  if (jj < 4) {
    s = A & 63;
    m = B & 63;
  } else {
    s = (C & 0xF) | ((A >> 6) << 4);
    m = (C >> 4) | ((B >> 6) << 4);
  }
}

__device__ __forceinline__ int sel4(int i, int a, int b, int c, int d) {
  return i == 0 ? a : i == 1 ? b : i == 2 ? c : d;
}
__device__ __forceinline__ int i8_of(uint32_t w, int byte) { return (int)(int8_t)((w >> (8 * byte)) & 0xFF); }

// One Q4_K row x up to MAXS Q8_K activation rows, lane j of the AVX2
// accumulator (avx2.rs:351-379). Returns hsum(acc) - summs in lane 0 of the
// 8-thread group.
template <int NS>
__device__ __forceinline__ void dot_row_q4k(const uint8_t* __restrict__ row, int nb, int j, int rot,
                                            const int8_t* const* xq, const float* const* xd,
                                            const int32_t* const* xs, float res[NS]) {
  float acc[NS], summs[NS];
#pragma unroll
  for (int s = 0; s < NS; ++s) acc[s] = summs[s] = 0.f;
  for (int b = 0; b < nb; ++b) {
    const uint8_t* blk = row + 144 * b;
    uint4 hdr = *reinterpret_cast<const uint4*>(blk);
    int sumi[NS];
#pragma unroll
    for (int s = 0; s < NS; ++s) sumi[s] = 0;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int k = (kk + rot) & 3;  // rotated to spread rows over smem banks
      uint32_t wq = *reinterpret_cast<const uint32_t*>(blk + 16 + 32 * k + 4 * j);
      int lo = (int)(wq & 0x0F0F0F0Fu), hi = (int)((wq >> 4) & 0x0F0F0F0Fu);
      int s0, m0, s1, m1;
      q4k_sm(2 * k, hdr.y, hdr.z, hdr.w, s0, m0);
      q4k_sm(2 * k + 1, hdr.y, hdr.z, hdr.w, s1, m1);
#pragma unroll
      for (int s = 0; s < NS; ++s) {
        const int8_t* xb = xq[s] + 256 * b + 64 * k + 4 * j;
        int xl = *reinterpret_cast<const int*>(xb), xh = *reinterpret_cast<const int*>(xb + 32);
        sumi[s] += s0 * dp4a(lo, xl, 0) + s1 * dp4a(hi, xh, 0);
      }
    }
    int sc[8], mn[8];
    q4k_scales(hdr.y, hdr.z, hdr.w, sc, mn);
    const float dw = h2f(hdr.x), dmw = h2f(hdr.x >> 16);
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      const int4* bs4 = reinterpret_cast<const int4*>(xs[s] + 16 * b);
      int4 p0 = bs4[0], p1 = bs4[1], p2 = bs4[2], p3 = bs4[3];
      int mins = mn[0] * (p0.x + p0.y) + mn[1] * (p0.z + p0.w) + mn[2] * (p1.x + p1.y) + mn[3] * (p1.z + p1.w) +
                 mn[4] * (p2.x + p2.y) + mn[5] * (p2.z + p2.w) + mn[6] * (p3.x + p3.y) + mn[7] * (p3.z + p3.w);
      float xdb = xd[s][b];
      float d = __fmul_rn(dw, xdb), dmin = __fmul_rn(dmw, xdb);
      acc[s] = __fmaf_rn((float)sumi[s], d, acc[s]);
      summs[s] = __fadd_rn(summs[s], __fmul_rn(dmin, (float)mins));
    }
    (void)sc;
  }
#pragma unroll
  for (int s = 0; s < NS; ++s) res[s] = __fsub_rn(hsum8_group(acc[s]), summs[s]);
}

// One Q6_K row (planar device layout) x up to MAXS Q8_K rows
// (avx2.rs:384-419). Lane j covers bytes 4j..4j+3 of each 32-element run;
// lanes 0-3 take the run's first sub-block scale, lanes 4-7 the second.
template <int NS>
__device__ __forceinline__ void dot_row_q6k(const uint8_t* __restrict__ row, int nb, int j, int rot,
                                            const int8_t* const* xq, const float* const* xd,
                                            const int32_t* const* xs, float res[NS]) {
  float acc[NS];
#pragma unroll
  for (int s = 0; s < NS; ++s) acc[s] = 0.f;
  const uint8_t* qlp = row;
  const uint8_t* qhp = row + 128 * nb;
  const uint8_t* scp = row + 192 * nb;
  const uint16_t* dp = reinterpret_cast<const uint16_t*>(row + 208 * nb);
  const int jh = j >> 2;  // which of the run's two sub-blocks
  for (int b = 0; b < nb; ++b) {
    uint4 scw = *reinterpret_cast<const uint4*>(scp + 16 * b);
    int sumi[NS];
#pragma unroll
    for (int s = 0; s < NS; ++s) sumi[s] = 0;
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      const int c = (cc + rot) & 3, h = c >> 1, hf = c & 1;
      uint32_t qlw = *reinterpret_cast<const uint32_t*>(qlp + 128 * b + 64 * h + 32 * hf + 4 * j);
      uint32_t qhw = *reinterpret_cast<const uint32_t*>(qhp + 64 * b + 32 * h + 4 * j);
#pragma unroll
      for (int nib = 0; nib < 2; ++nib) {
        const int ri = hf + 2 * nib;
        int qv = (int)(((qlw >> (4 * nib)) & 0x0F0F0F0Fu) | (((qhw >> (2 * ri)) & 0x03030303u) << 4));
        const int m = h * 8 + 2 * ri + jh;  // scale index 0..15
        int sw = sel4(m >> 2, (int)scw.x, (int)scw.y, (int)scw.z, (int)scw.w);
        int scale = i8_of((uint32_t)sw, m & 3);
#pragma unroll
        for (int s = 0; s < NS; ++s) {
          int xv = *reinterpret_cast<const int*>(xq[s] + 256 * b + 128 * h + 32 * ri + 4 * j);
          sumi[s] += scale * dp4a(qv, xv, 0);
        }
      }
    }
    const float dw = h2f(dp[b]);
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      const int4* bs4 = reinterpret_cast<const int4*>(xs[s] + 16 * b);
      int offs = 0;
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        int4 p = bs4[q4];
        uint32_t w = q4 == 0 ? scw.x : q4 == 1 ? scw.y : q4 == 2 ? scw.z : scw.w;
        offs += i8_of(w, 0) * p.x + i8_of(w, 1) * p.y + i8_of(w, 2) * p.z + i8_of(w, 3) * p.w;
      }
      float d = __fmul_rn(dw, xd[s][b]);
      acc[s] = __fmaf_rn((float)sumi[s], d, acc[s]);
      // avx2.rs:416: lane 0 gets (-32*d)*offs, lanes 1..7 get +0.0.
      acc[s] = __fadd_rn(acc[s], j == 0 ? __fmul_rn(__fmul_rn(-32.0f, d), (float)offs) : 0.0f);
    }
  }
#pragma unroll
  for (int s = 0; s < NS; ++s) res[s] = hsum8_group(acc[s]);
}

// One Q8_0 row (planar device layout) x up to MAXS Q8Row rows (avx2.rs:49-58).
template <int NS>
__device__ __forceinline__ void dot_row_q8_0(const uint8_t* __restrict__ row, int nb, int j,
                                             const int8_t* const* xq, const float* const* xd, float res[NS]) {
  float acc[NS];
#pragma unroll
  for (int s = 0; s < NS; ++s) acc[s] = 0.f;
  const uint16_t* dp = reinterpret_cast<const uint16_t*>(row + 32 * nb);
  for (int b = 0; b < nb; ++b) {
    int wv = *reinterpret_cast<const int*>(row + 32 * b + 4 * j);
    const float dw = h2f(dp[b]);
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      int xv = *reinterpret_cast<const int*>(xq[s] + 32 * b + 4 * j);
      int p = dp4a(wv, xv, 0);
      acc[s] = __fmaf_rn((float)p, __fmul_rn(dw, xd[s][b]), acc[s]);
    }
  }
#pragma unroll
  for (int s = 0; s < NS; ++s) res[s] = hsum8_group(acc[s]);
}

template <int T, int NS>
__device__ __forceinline__ void dot_row(const uint8_t* row, int cols, int j, int rot, const int8_t* const* xq,
                                        const float* const* xd, const int32_t* const* xs, float res[NS]) {
  if (T == T_Q4_K) dot_row_q4k<NS>(row, cols / 256, j, rot, xq, xd, xs, res);
  else if (T == T_Q6_K) dot_row_q6k<NS>(row, cols / 256, j, rot, xq, xd, xs, res);
  else dot_row_q8_0<NS>(row, cols / 32, j, xq, xd, res);
}

__device__ __forceinline__ float silu_mul(float g, float u) {
  // transformer.rs:558: g / (1 + exp(-g)) * u
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

template <int T, bool PAIR, int NS>
__device__ __forceinline__ void compute_rows(const GroupedArgs& a, const uint8_t* stage, int64_t mat_bytes, int q,
                                             int j, int r, int sbeg) {
  const int8_t* xq[NS];
  const float* xd[NS];
  const int32_t* xs[NS];
  const int blk = (T == T_Q8_0) ? 32 : 256;
#pragma unroll
  for (int s = 0; s < NS; ++s) {
    int slot = sbeg + s;
    int64_t ar = a.slot_src ? a.slot_src[slot] : slot;
    xq[s] = a.aq + ar * a.cols;
    xd[s] = a.ad + ar * (a.cols / blk);
    xs[s] = a.asum + ar * (a.cols / 16);
  }
  const int rot = q & 3;
  float g[NS], u[NS];
  dot_row<T, NS>(stage + q * a.row_stride, a.cols, j, rot, xq, xd, xs, g);
  if (PAIR) dot_row<T, NS>(stage + mat_bytes + q * a.row_stride, a.cols, j, rot, xq, xd, xs, u);
  if (j == 0 && r >= 0) {
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      float v = PAIR ? silu_mul(g[s], u[s]) : g[s];
      a.out[(int64_t)(sbeg + s) * a.out_stride + r] = v;
    }
  }
}

template <int T, bool PAIR>
__global__ void __launch_bounds__(I8_THREADS) grouped_int8_kernel(GroupedArgs a, int n_stages) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[MAX_STAGES], empty[MAX_STAGES];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_list = *a.n_list;
  const int tiles = (a.rows + RT - 1) / RT;
  const int64_t total = (int64_t)n_list * tiles;
  const int64_t beg = total * blockIdx.x / gridDim.x, end = total * (blockIdx.x + 1) / gridDim.x;
  if (beg >= end) return;
  const int64_t mat_bytes = (int64_t)RT * a.row_stride;
  const int64_t stage_bytes = mat_bytes * (PAIR ? 2 : 1);
  if (tid == 0) {
    for (int s = 0; s < n_stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], CONS_WARPS);
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int64_t u = beg; u < end; ++u, ++it) {
        const int st = it % n_stages;
        const uint32_t ph = (it / n_stages) & 1;
        if (it >= n_stages && !mbar_wait(&empty[st], ph ^ 1, a.status)) break;
        const int e = a.list[u / tiles];
        const int r0 = (int)(u % tiles) * RT, nr = min(RT, a.rows - r0);
        const uint32_t bytes = (uint32_t)(nr * a.row_stride);
        mbar_expect_tx(&full[st], bytes * (PAIR ? 2 : 1));
        const int64_t off = (int64_t)(e - a.expert_base) * a.expert_stride + (int64_t)r0 * a.row_stride;
        bulk_g2s(smem + st * stage_bytes, a.w0 + off, bytes, &full[st]);
        if (PAIR) bulk_g2s(smem + st * stage_bytes + mat_bytes, a.w1 + off, bytes, &full[st]);
      }
      // Do not leave while copies issued by this CTA may still land: wait for
      // the last use of every stage (bounded).
      for (int s = 0; s < n_stages && s < it; ++s) {
        int last = it - 1 - ((it - 1 - s) % n_stages);
        mbar_wait(&full[s], (last / n_stages) & 1, a.status);
      }
    }
    return;
  }
  const int c = tid - 32, q = c >> 3, j = c & 7;
  int it = 0;
  for (int64_t u = beg; u < end; ++u, ++it) {
    const int st = it % n_stages;
    const uint32_t ph = (it / n_stages) & 1;
    if (!mbar_wait(&full[st], ph, a.status)) return;
    const int e = a.list[u / tiles];
    const int r0 = (int)(u % tiles) * RT, nr = min(RT, a.rows - r0);
    const int sbeg = a.offsets[e], n = a.offsets[e + 1] - sbeg;
    const uint8_t* stage = smem + st * stage_bytes;
    // Every thread runs the row code (the lane folds are warp shuffles); rows
    // past the end of a partial tile recompute the tile's last row and do not
    // store.
    const int qq = min(q, nr - 1);
    const int r = q < nr ? r0 + q : -1;
    if (n == 1) compute_rows<T, PAIR, 1>(a, stage, mat_bytes, qq, j, r, sbeg);
    else if (n == 2) compute_rows<T, PAIR, 2>(a, stage, mat_bytes, qq, j, r, sbeg);
    else if (n == 3) compute_rows<T, PAIR, 3>(a, stage, mat_bytes, qq, j, r, sbeg);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }
}

template <int T, bool PAIR>
static int launch_i8_t(const GroupedArgs& a, int max_units, cudaStream_t st) {
  const int64_t stage_bytes = (int64_t)RT * a.row_stride * (PAIR ? 2 : 1);
  int n_stages = (int)std::min<int64_t>(MAX_STAGES, (200 * 1024) / stage_bytes);
  if (n_stages < 2) return KC_ERR_SHAPE;
  const size_t smem = (size_t)n_stages * stage_bytes;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(grouped_int8_kernel<T, PAIR>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    attr = true;
  }
  int grid = std::min(num_sms(), std::max(1, max_units));
  grouped_int8_kernel<T, PAIR><<<grid, I8_THREADS, smem, st>>>(a, n_stages);
  return KC_OK;
}

int launch_grouped_int8(const GroupedArgs& a, bool pair, int max_units, cudaStream_t st) {
  if (a.row_stride % 16 != 0) return KC_ERR_SHAPE;
  switch (a.type) {
    case T_Q4_K: return pair ? launch_i8_t<T_Q4_K, true>(a, max_units, st) : launch_i8_t<T_Q4_K, false>(a, max_units, st);
    case T_Q6_K: return pair ? launch_i8_t<T_Q6_K, true>(a, max_units, st) : launch_i8_t<T_Q6_K, false>(a, max_units, st);
    case T_Q8_0: return pair ? launch_i8_t<T_Q8_0, true>(a, max_units, st) : launch_i8_t<T_Q8_0, false>(a, max_units, st);
    default: return KC_ERR_TYPE;
  }
}

// ---------------------------------------------------------------------------
// f32 path: exact dequantisation (quant.rs:63-205 arithmetic) and f32 FMA
// products on CUDA cores. CTA tile: 64 weight rows x 32 slots, K chunks of 32.
constexpr int F_ROWS = 64, F_TOK = 32, F_K = 32, F_THREADS = 256;

template <int T>
__device__ __forceinline__ float dequant_elem(const uint8_t* __restrict__ row, int cols, int col) {
  if (T == T_Q4_K) {
    const int b = col >> 8, i = col & 255, k = i >> 6, hi = (i >> 5) & 1, l = i & 31;
    const uint8_t* blk = row + 144 * b;
    uint32_t w0 = *reinterpret_cast<const uint32_t*>(blk + 4), w1 = *reinterpret_cast<const uint32_t*>(blk + 8),
             w2 = *reinterpret_cast<const uint32_t*>(blk + 12);
    int s, m;
    q4k_sm(2 * k + hi, w0, w1, w2, s, m);
    uint32_t dd = *reinterpret_cast<const uint32_t*>(blk);
    float d1 = __fmul_rn(h2f(dd), (float)s), m1 = __fmul_rn(h2f(dd >> 16), (float)m);
    int qv = hi ? (blk[16 + 32 * k + l] >> 4) : (blk[16 + 32 * k + l] & 0xF);
    return __fsub_rn(__fmul_rn(d1, (float)qv), m1);
  } else if (T == T_Q6_K) {
    const int nb = cols >> 8, b = col >> 8, i = col & 255, h = i >> 7, r = (i >> 5) & 3, l = i & 31;
    int ql = row[128 * b + 64 * h + l + 32 * (r & 1)];
    int nib = (r >> 1) ? (ql >> 4) : (ql & 0xF);
    int qh = (row[128 * nb + 64 * b + 32 * h + l] >> (2 * r)) & 3;
    int qv = (nib | (qh << 4)) - 32;
    int sc = (int8_t)row[192 * nb + 16 * b + 8 * h + 2 * r + (l >> 4)];
    float d = h2f(*reinterpret_cast<const uint16_t*>(row + 208 * nb + 2 * b));
    return __fmul_rn(__fmul_rn(d, (float)sc), (float)qv);
  } else if (T == T_Q8_0) {
    const int nb = cols >> 5, b = col >> 5;
    float d = h2f(*reinterpret_cast<const uint16_t*>(row + 32 * nb + 2 * b));
    return __fmul_rn((float)(int8_t)row[col], d);
  } else {
    return reinterpret_cast<const float*>(row)[col];
  }
}

template <int T, bool PAIR>
__global__ void __launch_bounds__(F_THREADS) grouped_f32_kernel(GroupedArgs a) {
  __shared__ float Wg[F_ROWS][F_K + 1];
  __shared__ float Wu[PAIR ? F_ROWS : 1][F_K + 1];
  __shared__ float X[F_TOK][F_K + 1];
  const int i = blockIdx.y;
  if (i >= *a.n_list) return;
  const int e = a.list[i];
  const int sbeg = a.offsets[e], n = a.offsets[e + 1] - sbeg;
  const int t0 = blockIdx.z * F_TOK;
  if (t0 >= n) return;
  const int r0 = blockIdx.x * F_ROWS;
  const int tid = threadIdx.x;
  const int tr = (tid & 15) * 4, tt = (tid >> 4) * 2;  // 4 rows x 2 slots per thread
  float ag[4][2], au[4][2];
#pragma unroll
  for (int x = 0; x < 4; ++x)
#pragma unroll
    for (int y = 0; y < 2; ++y) ag[x][y] = au[x][y] = 0.f;
  const uint8_t* base0 = a.w0 + (int64_t)(e - a.expert_base) * a.expert_stride;
  const uint8_t* base1 = PAIR ? a.w1 + (int64_t)(e - a.expert_base) * a.expert_stride : nullptr;
  for (int k0 = 0; k0 < a.cols; k0 += F_K) {
    for (int idx = tid; idx < F_ROWS * F_K; idx += F_THREADS) {
      int rr = idx / F_K, kk = idx % F_K, r = r0 + rr;
      float vg = 0.f, vu = 0.f;
      if (r < a.rows) {
        vg = dequant_elem<T>(base0 + (int64_t)r * a.row_stride, a.cols, k0 + kk);
        if (PAIR) vu = dequant_elem<T>(base1 + (int64_t)r * a.row_stride, a.cols, k0 + kk);
      }
      Wg[rr][kk] = vg;
      if (PAIR) Wu[rr][kk] = vu;
    }
    for (int idx = tid; idx < F_TOK * F_K; idx += F_THREADS) {
      int ss = idx / F_K, kk = idx % F_K, t = t0 + ss;
      float v = 0.f;
      if (t < n) {
        int slot = sbeg + t;
        int64_t ar = a.slot_src ? a.slot_src[slot] : slot;
        v = a.af[ar * a.cols + k0 + kk];
      }
      X[ss][kk] = v;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < F_K; ++kk) {
      float xv0 = X[tt][kk], xv1 = X[tt + 1][kk];
#pragma unroll
      for (int x = 0; x < 4; ++x) {
        float wg = Wg[tr + x][kk];
        ag[x][0] = __fmaf_rn(wg, xv0, ag[x][0]);
        ag[x][1] = __fmaf_rn(wg, xv1, ag[x][1]);
        if (PAIR) {
          float wu = Wu[tr + x][kk];
          au[x][0] = __fmaf_rn(wu, xv0, au[x][0]);
          au[x][1] = __fmaf_rn(wu, xv1, au[x][1]);
        }
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int x = 0; x < 4; ++x)
#pragma unroll
    for (int y = 0; y < 2; ++y) {
      int r = r0 + tr + x, t = t0 + tt + y;
      if (r < a.rows && t < n) {
        float v = PAIR ? silu_mul(ag[x][y], au[x][y]) : ag[x][y];
        a.out[(int64_t)(sbeg + t) * a.out_stride + r] = v;
      }
    }
}

template <int T, bool PAIR>
static int launch_f32_t(const GroupedArgs& a, int max_experts, int max_rows, cudaStream_t st) {
  dim3 grid(ceil_div(a.rows, F_ROWS), max_experts, ceil_div(max_rows, F_TOK));
  grouped_f32_kernel<T, PAIR><<<grid, F_THREADS, 0, st>>>(a);
  return KC_OK;
}

int launch_grouped_f32(const GroupedArgs& a, bool pair, int max_experts, int max_rows_per_expert,
                       cudaStream_t st) {
  if (max_experts <= 0 || max_rows_per_expert <= 0) return KC_OK;
  if (a.cols % F_K) return KC_ERR_SHAPE;
  switch (a.type) {
    case T_Q4_K: return pair ? launch_f32_t<T_Q4_K, true>(a, max_experts, max_rows_per_expert, st)
                             : launch_f32_t<T_Q4_K, false>(a, max_experts, max_rows_per_expert, st);
    case T_Q6_K: return pair ? launch_f32_t<T_Q6_K, true>(a, max_experts, max_rows_per_expert, st)
                             : launch_f32_t<T_Q6_K, false>(a, max_experts, max_rows_per_expert, st);
    case T_Q8_0: return pair ? launch_f32_t<T_Q8_0, true>(a, max_experts, max_rows_per_expert, st)
                             : launch_f32_t<T_Q8_0, false>(a, max_experts, max_rows_per_expert, st);
    default: return KC_ERR_TYPE;
  }
}

}  // namespace kc
