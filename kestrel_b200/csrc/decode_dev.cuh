// Device building blocks of the decode-sized dequant-dot (decode.cu):
// work-unit geometry constants, shared-memory loads, the per-superblock
// integer kernels of the reference's Q4_K / Q6_K / Q8_0 x Q8_K / Q8 dot
// products, and one unit's consumer loop.
#pragma once

#include "common.cuh"
#include "decode.h"

namespace kc {

constexpr int DR = kTileRows;  // rows per unit
constexpr int DW = 8;          // units per group (one producer lane each)
constexpr int DC = 2 * DW;     // consumer warps
constexpr int DARR = 8;        // consumer arrivals that release a stage
constexpr int DTHREADS = 32 * (DC + 1);
constexpr int DMAX_STAGES = 64;
constexpr int DMAXS = 3;       // slots per unit (experts with 1..3 rows)
constexpr int DSMEM = 216 * 1024;
constexpr int DMAX_E = 1024;   // experts whose list / offsets are copied to shared memory

// ---------------------------------------------------------------------------
// Shared-memory loads by 32-bit shared-window address. Explicit ld.shared
// (volatile: kept in order with the mbarrier waits that guard the data).
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
// N consecutive 32-bit words (N = 4, 2, 1; address aligned to 4N bytes).
template <int N>
__device__ __forceinline__ void ldsw(uint32_t a, uint32_t (&w)[N]) {
  if constexpr (N == 4) {
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]) : "r"(a));
  } else if constexpr (N == 2) {
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(w[0]), "=r"(w[1]) : "r"(a));
  } else {
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(w[0]) : "r"(a));
  }
}
__device__ __forceinline__ float ldsf(uint32_t a) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t ldsu16(uint32_t a) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ int sbyte(uint32_t w, int i) { return (int)(int8_t)((w >> (8 * i)) & 0xFF); }
__device__ __forceinline__ int ubyte(uint32_t w, int i) { return (int)((w >> (8 * i)) & 0xFF); }
// dp2a: a = two int16, b = four int8; lo uses bytes 0-1 of b, hi bytes 2-3.
__device__ __forceinline__ int dp2a_lo(uint32_t a, uint32_t b, int c) { return __dp2a_lo((int)a, (int)b, c); }
__device__ __forceinline__ int dp2a_hi(uint32_t a, uint32_t b, int c) { return __dp2a_hi((int)a, (int)b, c); }

// The per-superblock kernels below compute, for one weight row, LPT of the
// reference's eight 32-bit AVX2 lanes: lanes l0 .. l0+LPT-1 (LPT = 4, 2 or 1;
// l0 a multiple of LPT). Lane j of a 32-byte vector is its word j, so the
// thread's lanes are words (l0 & 3) .. of the vector's 16-byte chunk l0 >> 2.
// acc[s][i] is lane l0 + i of slot s.

// One Q4_K superblock of row `row` (avx2.rs:351-379) against NS slots whose
// records start at xr (stride R).
template <int NS, int R, int LPT>
__device__ __forceinline__ void q4k_sb(uint32_t sbt, int row, int l0, uint32_t xr,
                                       float (&acc)[NS][LPT], float (&summs)[NS]) {
  const uint4 hdr = lds128(sbt + 16 * row);
  const float dw = h2f(hdr.x), dmw = h2f(hdr.x >> 16);
  // scale_min_k4 (quant.rs:54-60) for all eight sub-blocks, four per word.
  const uint32_t scA = hdr.y & 0x3F3F3F3Fu;
  const uint32_t scB = (hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u);
  const uint32_t mA = hdr.z & 0x3F3F3F3Fu;
  const uint32_t mB = ((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u);
  int sumi[NS][LPT];
#pragma unroll
  for (int s = 0; s < NS; ++s)
#pragma unroll
    for (int j = 0; j < LPT; ++j) sumi[s][j] = 0;
  // qs bytes 32k..32k+31 (sub-blocks 2k and 2k+1 in the low / high nibbles).
  const uint32_t qa = sbt + kPlane + kPlane * (l0 >> 2) + 16 * row + 4 * (l0 & 3);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    uint32_t qw[LPT];
    ldsw<LPT>(qa + 2 * kPlane * k, qw);
    int lo[LPT], hi[LPT];
#pragma unroll
    for (int j = 0; j < LPT; ++j) {
      lo[j] = (int)(qw[j] & 0x0F0F0F0Fu);
      hi[j] = (int)((qw[j] >> 4) & 0x0F0F0F0Fu);
    }
    const int slo = ubyte(k < 2 ? scA : scB, (2 * k) & 3), shi = ubyte(k < 2 ? scA : scB, (2 * k + 1) & 3);
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      const uint32_t x = xr + s * R + 64 * k + 4 * l0;
      uint32_t xl[LPT], xh[LPT];
      ldsw<LPT>(x, xl);
      ldsw<LPT>(x + 32, xh);
#pragma unroll
      for (int j = 0; j < LPT; ++j) {
        sumi[s][j] += slo * dp4a(lo[j], (int)xl[j], 0);
        sumi[s][j] += shi * dp4a(hi[j], (int)xh[j], 0);
      }
    }
  }
#pragma unroll
  for (int s = 0; s < NS; ++s) {
    const uint32_t x = xr + s * R;
    const float xd = ldsf(x + 304);
    const float d = __fmul_rn(dw, xd), dmin = __fmul_rn(dmw, xd);
#pragma unroll
    for (int j = 0; j < LPT; ++j) acc[s][j] = __fmaf_rn((float)sumi[s][j], d, acc[s][j]);
    // mins = sum over sub-blocks m[i] * (bsums[2i] + bsums[2i+1]) (one per row;
    // every thread of the row computes it, the lane-0 thread uses it)
    const uint4 bp = lds128(x + 288);
    const int mins = dp2a_lo(bp.x, mA, dp2a_hi(bp.y, mA, dp2a_lo(bp.z, mB, dp2a_hi(bp.w, mB, 0))));
    summs[s] = __fadd_rn(summs[s], __fmul_rn(dmin, (float)mins));
  }
}

// One Q6_K superblock (avx2.rs:384-419). Lanes 0-3 of a 32-run use its first
// 16-element scale, lanes 4-7 the second.
template <int NS, int R, int LPT>
__device__ __forceinline__ void q6k_sb(uint32_t sbt, int row, int l0, uint32_t xr, float (&acc)[NS][LPT]) {
  const float dw = h2f(ldsu16(sbt + 13 * kPlane + 2 * row));
  const uint4 scw = lds128(sbt + 12 * kPlane + 16 * row);
  const uint32_t sw[4] = {scw.x, scw.y, scw.z, scw.w};
  const int hf = l0 >> 2;  // which 16-byte chunk (and scale) of a 32-run
  const uint32_t wo = 16 * row + 4 * (l0 & 3);
  int sumi[NS][LPT];
#pragma unroll
  for (int s = 0; s < NS; ++s)
#pragma unroll
    for (int j = 0; j < LPT; ++j) sumi[s][j] = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t hw[LPT];
    ldsw<LPT>(sbt + 8 * kPlane + kPlane * (2 * h + hf) + wo, hw);
#pragma unroll
    for (int run = 0; run < 2; ++run) {
      uint32_t lw[LPT];
      ldsw<LPT>(sbt + kPlane * (4 * h + 2 * run + hf) + wo, lw);
#pragma unroll
      for (int nib = 0; nib < 2; ++nib) {
        const int ri = 2 * nib + run;
        int q6[LPT];
#pragma unroll
        for (int j = 0; j < LPT; ++j)
          q6[j] = (int)(((lw[j] >> (4 * nib)) & 0x0F0F0F0Fu) | (((hw[j] >> (2 * ri)) & 0x03030303u) << 4));
        const int si = 8 * h + 2 * ri;
        const uint32_t sa = sw[si >> 2], sb = sw[(si + 1) >> 2];
        const int sc = hf ? sbyte(sb, (si + 1) & 3) : sbyte(sa, si & 3);
#pragma unroll
        for (int s = 0; s < NS; ++s) {
          uint32_t xw[LPT];
          ldsw<LPT>(xr + s * R + 128 * h + 32 * ri + 4 * l0, xw);
#pragma unroll
          for (int j = 0; j < LPT; ++j) sumi[s][j] += sc * dp4a(q6[j], (int)xw[j], 0);
        }
      }
    }
  }
#pragma unroll
  for (int s = 0; s < NS; ++s) {
    const uint32_t x = xr + s * R;
    const float d = __fmul_rn(dw, ldsf(x + 304));
#pragma unroll
    for (int j = 0; j < LPT; ++j) acc[s][j] = __fmaf_rn((float)sumi[s][j], d, acc[s][j]);
    // offs = sum over the 16 sub-blocks sc[i] * bsums[i]
    const uint4 b0 = lds128(x + 256), b1 = lds128(x + 272);
    int offs = dp2a_lo(b0.x, sw[0], 0);
    offs = dp2a_hi(b0.y, sw[0], offs);
    offs = dp2a_lo(b0.z, sw[1], offs);
    offs = dp2a_hi(b0.w, sw[1], offs);
    offs = dp2a_lo(b1.x, sw[2], offs);
    offs = dp2a_hi(b1.y, sw[2], offs);
    offs = dp2a_lo(b1.z, sw[3], offs);
    offs = dp2a_hi(b1.w, sw[3], offs);
    // avx2.rs:416: lane 0 gets (-32*d)*offs, the other lanes +0.0.
    const float o = __fmul_rn(__fmul_rn(-32.0f, d), (float)offs);
    acc[s][0] = __fadd_rn(acc[s][0], l0 == 0 ? o : 0.0f);
#pragma unroll
    for (int j = 1; j < LPT; ++j) acc[s][j] = __fadd_rn(acc[s][j], 0.0f);
  }
}

// One chunk of up to 8 Q8_0 blocks (avx2.rs:49-58).
template <int NS, int R, int LPT>
__device__ __forceinline__ void q8_0_chunk(uint32_t cb, int nblk, int row, int l0, uint32_t xr,
                                           float (&acc)[NS][LPT]) {
  const uint32_t wo = kPlane * (l0 >> 2) + 16 * row + 4 * (l0 & 3);
#pragma unroll 1
  for (int bl = 0; bl < nblk; ++bl) {
    uint32_t ww[LPT];
    ldsw<LPT>(cb + 2 * kPlane * bl + wo, ww);
    const float dw = h2f(ldsu16(cb + 2 * kPlane * nblk + 16 * row + 2 * bl));
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      const uint32_t x = xr + s * R;
      uint32_t xw[LPT];
      ldsw<LPT>(x + 32 * bl + 4 * l0, xw);
      const float d = __fmul_rn(dw, ldsf(x + 256 + 4 * bl));
#pragma unroll
      for (int j = 0; j < LPT; ++j) acc[s][j] = __fmaf_rn((float)dp4a((int)ww[j], (int)xw[j], 0), d, acc[s][j]);
    }
  }
}

// hsum (avx2.rs:19-27): ((v0+v4)+(v2+v6)) + ((v1+v5)+(v3+v7)).
__device__ __forceinline__ float hsum8(const float (&v)[8]) {
  const float a = __fadd_rn(__fadd_rn(v[0], v[4]), __fadd_rn(v[2], v[6]));
  const float b = __fadd_rn(__fadd_rn(v[1], v[5]), __fadd_rn(v[3], v[7]));
  return __fadd_rn(a, b);
}

// ---------------------------------------------------------------------------
struct UnitMeta {
  int e, slot0, ns;
};

// Meta of list entry li from the shared copies of the list and offsets. An
// entry e | part << 16 holds rows DMAXS * part .. of expert e (part 0 unless
// the list was dispatched by rows).
__device__ __forceinline__ UnitMeta meta_at(const int* list_s, const int* off_s, int li) {
  UnitMeta m;
  const int v = list_s[li];
  m.e = v & 0xFFFF;
  m.slot0 = off_s[m.e] + DMAXS * (v >> 16);
  m.ns = max(1, min(DMAXS, off_s[m.e + 1] - m.slot0));
  return m;
}

// Position of unit u: list entry, matrix, 32-row tile.
struct UnitPos {
  int li, m, tile;
};
// tile_major (one matrix): the list entries of a tile are consecutive units,
// so entries sharing one matrix (a dense product by rows) read each tile
// close together in time, the later ones from L2.
__device__ __forceinline__ UnitPos unit_pos(int u, int tiles, int n_mat, bool tile_major = false, int n_list = 1) {
  UnitPos p;
  if (tile_major) {
    p.tile = u / n_list;
    p.li = u - p.tile * n_list;
    p.m = 0;
    return p;
  }
  const int q = u / tiles;
  p.tile = u - q * tiles;
  p.li = n_mat == 2 ? q >> 1 : q;
  p.m = n_mat == 2 ? q & 1 : 0;
  return p;
}

template <int T>
struct TypeR {
  static constexpr int R = T == T_Q8_0 ? kRecQ8 : kRecK;
};

// Threads per weight row for a group of wg units (1..DW): full and
// nearly full groups take two threads per row (DC = 2 * DW warps, two per
// unit); smaller groups spread each unit over more warps, so the tail of a
// CTA's range runs on all its warps.
__host__ __device__ constexpr int tpr_of(int wg) { return wg > DW / 2 ? 2 : (wg > DW / 4 ? 4 : 8); }
static_assert(DC == 2 * DW && DW % 4 == 0, "warp layout");

// One unit, all segments, on TPR threads per row. This warp holds rows
// `row` (one per lane / TPR) and lanes l0 = (lane % TPR) * LPT .. of each.
// The unit's stages are sid0, sid0 + wg, sid0 + 2 wg, ... (segment-major
// order of its group).
// Records of the stage: K-quant, slot s of superblock j at
// xr + (j / 2) * DMAXS * SR + (j % 2) * SBS + s * SR (pair blocks of DMAXS
// slots); Q8, chunk j at xr + j * SBS. The defaults (SR = R, SBS = DMAXS * R)
// make both superblock-major.
template <int T, int TPR, int NS, class Args, int SR = TypeR<T>::R, int SBS = DMAXS * TypeR<T>::R>
__device__ __forceinline__ void run_unit(const Args& a, const DecodeGeom& g, const uint8_t* ring,
                                         uint64_t* full, uint64_t* empty, int* rel, int n_stages, int sid0, int wg,
                                         int lane,
                                         int row, float* out, int r_out, bool& ok) {
  constexpr int R = TypeR<T>::R;
  constexpr int LPT = 8 / TPR;
  const int l0 = (lane % TPR) * LPT;
  float acc[NS][LPT], summs[NS];
#pragma unroll
  for (int s = 0; s < NS; ++s) {
    summs[s] = 0.f;
#pragma unroll
    for (int j = 0; j < LPT; ++j) acc[s][j] = 0.f;
  }
  // Stage number, ring slot and phase of the unit's segment 0; each later
  // segment is wg stages on (wg <= DW < n_stages).
  int sid = sid0, st = sid0 % n_stages;
  uint32_t ph = (uint32_t)((sid0 / n_stages) & 1);
  for (int seg = 0; seg < g.nseg; ++seg) {
    // A slot is used lap after lap by different warps, and bulk copies may land
    // out of order: before waiting on this lap's copy, wait until the slot's
    // previous lap has been released. Only then is the copy barrier known to be
    // in this lap's phase, so its parity test cannot alias an older phase. The
    // release is counted (rel), not tested by parity: a fast warp may arrive
    // here while the previous lap is not yet issued and the lap before it not
    // yet released, which a parity test would mistake for the release it wants.
    if (ok && sid >= n_stages && !count_wait(&rel[st], (sid / n_stages) * DARR, a.status, W_DEC_PREV)) ok = false;
    if (ok && !mbar_wait(&full[st], ph, a.status, W_DEC_FULL)) ok = false;
    if (ok) {
      const uint32_t sp = smem_u32(ring) + (uint32_t)(st * g.stage_bytes);
      const uint32_t xr = sp + (uint32_t)g.rec_off;
      const int sb0 = seg * g.ks;
      const int n = min(g.ks, g.nsb - sb0);
      for (int j = 0; j < n; ++j) {
        // K-quant records: pair block (j / 2) of the stage, record j % 2 of a slot.
        const uint32_t xj = xr + (j >> 1) * (DMAXS * SR) + (j & 1) * SBS;
        if (T == T_Q4_K) q4k_sb<NS, SR, LPT>(sp + 4608 * j, row, l0, xj, acc, summs);
        else if (T == T_Q6_K) q6k_sb<NS, SR, LPT>(sp + 6720 * j, row, l0, xj, acc);
        else q8_0_chunk<NS, SR, LPT>(sp + 8704 * j, min(8, g.nb32 - 8 * (sb0 + j)), row, l0, xr + j * SBS, acc);
      }
    }
    __syncwarp();
    // TPR warps hold the unit; each releases DARR / TPR of the slot's DARR arrivals.
    if (lane == 0) {
      mbar_arrive_cnt(&empty[st], DARR / TPR);  // for the producer
      count_add(&rel[st], DARR / TPR);          // for the next lap's consumers
    }
    sid += wg;
    st += wg;
    if (st >= n_stages) {
      st -= n_stages;
      ph ^= 1u;
    }
  }
  // Gather the row's eight lanes in its first thread, then hsum in the
  // reference's order.
#pragma unroll
  for (int s = 0; s < NS; ++s) {
    float v[8];
#pragma unroll
    for (int q = 0; q < TPR; ++q)
#pragma unroll
      for (int i = 0; i < LPT; ++i) v[q * LPT + i] = __shfl_sync(0xffffffffu, acc[s][i], (lane & ~(TPR - 1)) + q);
    float r = hsum8(v);
    if (T == T_Q4_K) r = __fsub_rn(r, summs[s]);
    if (l0 == 0 && r_out >= 0 && ok) out[(int64_t)s * a.out_stride + r_out] = r;
  }
}

template <int T, int TPR, int SR = TypeR<T>::R, int SBS = DMAXS * TypeR<T>::R, class Args>
__device__ __forceinline__ void run_unit_ns(int ns, const Args& a, const DecodeGeom& g, const uint8_t* ring,
                                            uint64_t* full, uint64_t* empty, int* rel, int n_stages, int sid0, int wg,
                                            int lane, int row, float* out, int r_out, bool& ok) {
  if (ns == 1) run_unit<T, TPR, 1, Args, SR, SBS>(a, g, ring, full, empty, rel, n_stages, sid0, wg, lane, row, out, r_out, ok);
  else if (ns == 2) run_unit<T, TPR, 2, Args, SR, SBS>(a, g, ring, full, empty, rel, n_stages, sid0, wg, lane, row, out, r_out, ok);
  else run_unit<T, TPR, 3, Args, SR, SBS>(a, g, ring, full, empty, rel, n_stages, sid0, wg, lane, row, out, r_out, ok);
}

}  // namespace kc
