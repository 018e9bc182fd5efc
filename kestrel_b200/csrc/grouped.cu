// f32 path of the grouped products (experts with >= 4 rows): the reference
// dequantises exactly and runs an f32 GEMM (quant.rs:241-260); this kernel
// does the same arithmetic on CUDA cores in the same order, bit for bit. It
// serves shapes the tensor-core kernel does not take and KC_OPT_F32_PREFILL.
#include "common.cuh"
#include "kernels.h"

namespace kc {

// Scale and min of Q4_K sub-block jj for a runtime jj (scale_min_k4,
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

// ---------------------------------------------------------------------------
// f32 path: exact dequantisation (quant.rs:63-205 arithmetic), then the
// reference's f32 GEMM operation order. CTA tile: F_RE weight rows x F_TE
// slots x 8 lanes; K chunks of F_KC elements.
constexpr int F_RE = 8, F_TE = 4, F_KC = 512, F_THREADS = F_RE * F_TE * 8;

// Element (r, col) of one expert matrix in the tiled device layout
// (common.cuh), dequantised with the reference's float operations
// (quant.rs:138-155 Q4_K, 180-201 Q6_K, 82-89 Q8_0).
template <int T>
__device__ __forceinline__ float dequant_elem(const uint8_t* __restrict__ mat, int cols, int r, int col) {
  const int rr = r % kTileRows;
  const uint8_t* tile = mat + (int64_t)(r / kTileRows) * tiled_tile_bytes(T, cols);
  if (T == T_Q4_K) {
    const int i = col & 255, k = i >> 6, hi = (i >> 5) & 1, l = i & 31;
    const uint8_t* sbt = tile + 4608 * (col >> 8);
    const uint8_t* hdr = sbt + 16 * rr;
    uint32_t w0 = *reinterpret_cast<const uint32_t*>(hdr + 4), w1 = *reinterpret_cast<const uint32_t*>(hdr + 8),
             w2 = *reinterpret_cast<const uint32_t*>(hdr + 12);
    int s, m;
    q4k_sm(2 * k + hi, w0, w1, w2, s, m);
    uint32_t dd = *reinterpret_cast<const uint32_t*>(hdr);
    float d1 = __fmul_rn(h2f(dd), (float)s), m1 = __fmul_rn(h2f(dd >> 16), (float)m);
    const int qb = 32 * k + l;  // byte of qs
    const int byte = sbt[kPlane + kPlane * (qb >> 4) + 16 * rr + (qb & 15)];
    const int qv = hi ? (byte >> 4) : (byte & 0xF);
    return __fsub_rn(__fmul_rn(d1, (float)qv), m1);
  } else if (T == T_Q6_K) {
    const int i = col & 255, h = i >> 7, r2 = (i >> 5) & 3, l = i & 31;
    const uint8_t* sbt = tile + 6720 * (col >> 8);
    const int lb = 64 * h + 32 * (r2 & 1) + l;  // byte of ql
    const int ql = sbt[kPlane * (lb >> 4) + 16 * rr + (lb & 15)];
    const int nib = (r2 >> 1) ? (ql >> 4) : (ql & 0xF);
    const int hb = 32 * h + l;  // byte of qh
    const int qh = (sbt[8 * kPlane + kPlane * (hb >> 4) + 16 * rr + (hb & 15)] >> (2 * r2)) & 3;
    const int qv = (nib | (qh << 4)) - 32;
    const int sc = (int8_t)sbt[12 * kPlane + 16 * rr + 8 * h + 2 * r2 + (l >> 4)];
    const float d = h2f(*reinterpret_cast<const uint16_t*>(sbt + 13 * kPlane + 2 * rr));
    return __fmul_rn(__fmul_rn(d, (float)sc), (float)qv);
  } else {
    const int cb = col >> 8, bl = (col & 255) >> 5, l = col & 31;
    const int nb32 = cols >> 5, nblk = min(8, nb32 - 8 * cb);
    const uint8_t* chunk = tile + 8704ll * cb;
    const float d = h2f(*reinterpret_cast<const uint16_t*>(chunk + 2 * kPlane * nblk + 16 * rr + 2 * bl));
    return __fmul_rn((float)(int8_t)chunk[kPlane * (2 * bl + (l >> 4)) + 16 * rr + (l & 15)], d);
  }
}

// One output (weight row r, slot s of an expert with n rows) is computed by 8
// threads, one per AVX2 lane, exactly as the reference's n >= 4 path does it
// (quant.rs:241-260 on 48-row tiles, avx2::gemm_f32 / dot_f32 avx2.rs:230-308):
//  * rows in a tile's 3-row blocks and slots in 4-slot blocks (s < n / 4 * 4):
//    one fused multiply-add chain per lane over the 8-element chunks, then
//    hsum;
//  * the other outputs (dot_f32): even chunks into a0, odd chunks into a1,
//    a0 + a1 lane-wise, then hsum.
// The weights are dequantised exactly into shared memory, K chunk by chunk;
// each lane visits its elements in increasing order, so the results are the
// reference's bit for bit. CTA: 8 rows x 4 slots x 8 lanes.
template <int T, bool PAIR>
__global__ void __launch_bounds__(F_THREADS) grouped_f32_kernel(GroupedArgs a) {
  pdl_enter();
  __shared__ float Wg[F_RE][F_KC + 4];
  __shared__ float Wu[PAIR ? F_RE : 1][F_KC + 4];
  __shared__ float X[F_TE][F_KC + 4];
  const int i = blockIdx.y;
  if (i >= *a.n_list) return;
  const int e = a.list[i];
  const int sbeg = a.offsets[e], n = a.offsets[e + 1] - sbeg;
  const int t0 = blockIdx.z * F_TE;
  if (t0 >= n) return;
  const int r0 = blockIdx.x * F_RE;
  const int tid = threadIdx.x, j = tid & 7, grp = tid >> 3;
  const int er = grp % F_RE, tr = grp / F_RE;
  const int r = r0 + er, t = t0 + tr;
  // quant.rs:243 tiles rows by 48; gemm_f32 blocks each tile's rows in 3s and
  // the slots in 4s.
  const int tile = r / 48, trows = min(48, a.rows - tile * 48);
  const bool m1 = !((r - tile * 48) < trows / 3 * 3 && t < n / 4 * 4);
  const int64_t epos = expert_pos(a.slot, e - a.expert_base);
  const uint8_t* base0 = a.w0 + epos * a.expert_stride;
  const uint8_t* base1 = PAIR ? a.w1 + epos * a.expert_stride : nullptr;
  float g0 = 0.f, g1 = 0.f, u0 = 0.f, u1 = 0.f;
  for (int k0 = 0; k0 < a.cols; k0 += F_KC) {
    const int kn = min(F_KC, a.cols - k0);
    for (int idx = tid; idx < F_RE * kn; idx += F_THREADS) {
      const int rr = idx / kn, kk = idx - rr * kn, row = r0 + rr;
      const bool ok = row < a.rows;
      Wg[rr][kk] = ok ? dequant_elem<T>(base0, a.cols, row, k0 + kk) : 0.f;
      if (PAIR) Wu[rr][kk] = ok ? dequant_elem<T>(base1, a.cols, row, k0 + kk) : 0.f;
    }
    for (int idx = tid; idx < F_TE * kn; idx += F_THREADS) {
      const int ss = idx / kn, kk = idx - ss * kn, tt = t0 + ss;
      float v = 0.f;
      if (tt < n) {
        const int slot = sbeg + tt;
        const int64_t ar = a.slot_src ? a.slot_src[slot] : slot;
        v = a.af[ar * a.cols + k0 + kk];
      }
      X[ss][kk] = v;
    }
    __syncthreads();
    for (int c = j; c < kn; c += 8) {
      const bool odd = (((k0 + c) >> 3) & 1) != 0;
      const float xv = X[tr][c];
      if (odd && m1) {
        g1 = __fmaf_rn(Wg[er][c], xv, g1);
        if (PAIR) u1 = __fmaf_rn(Wu[er][c], xv, u1);
      } else {
        g0 = __fmaf_rn(Wg[er][c], xv, g0);
        if (PAIR) u0 = __fmaf_rn(Wu[er][c], xv, u0);
      }
    }
    __syncthreads();
  }
  const float vg = hsum8_group(m1 ? __fadd_rn(g0, g1) : g0);
  const float vu = PAIR ? hsum8_group(m1 ? __fadd_rn(u0, u1) : u0) : 0.f;
  if (j == 0 && r < a.rows && t < n) {
    a.out[(int64_t)(sbeg + t) * a.out_stride + r] = vg;
    if (PAIR) a.out2[(int64_t)(sbeg + t) * a.out_stride + r] = vu;
  }
}

template <int T, bool PAIR>
static int launch_f32_t(const GroupedArgs& a, int max_experts, int max_rows, cudaStream_t st) {
  dim3 grid(ceil_div(a.rows, F_RE), max_experts, ceil_div(max_rows, F_TE));
  launch_k(grouped_f32_kernel<T, PAIR>, grid, F_THREADS, 0, st, a);
  return KC_OK;
}

int launch_grouped_f32(const GroupedArgs& a, bool pair, int max_experts, int max_rows_per_expert,
                       cudaStream_t st) {
  if (max_experts <= 0 || max_rows_per_expert <= 0) return KC_OK;
  if (a.cols % 32) return KC_ERR_SHAPE;
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
