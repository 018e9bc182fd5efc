// Decode-sized grouped dequant-dot: the reference's Q8_K / Q8Row integer
// kernels (crates/kestrel-engine/src/avx2.rs:49-58, 351-419) bit for bit, for
// experts with 1..3 routed rows and dense products with n < 4.
//
// Memory-bound design:
//  * Work unit = 16 rows of one expert matrix. A unit is streamed through one
//    or more pipeline stages (K segments of up to 8 superblocks). Activation
//    records (interleaved Q8_K: q[256] | bsums[16] | d per superblock) are
//    read through the read-only L1 path, where the few rows of an expert
//    stay hot; per-unit metadata (expert, slots, record rows) is loaded once
//    into shared memory.
//  * Weights are in the tiled device layout (common.cuh): a stage (16 rows x
//    2 superblocks, ~4.6-6.7 KB) is one contiguous range fetched by a single
//    cp.async.bulk into a ring of up to 48 stages tracked by mbarriers, so
//    ~170 KB per SM is in flight while consumers hold only the stages they
//    are computing; four consecutive rows read by a quarter warp fall on
//    distinct banks by construction.
//  * Six consumer pairs (2 warps, 64 threads) take units round-robin. Four
//    threads own a row: thread q holds lanes 2q and 2q+1 of the reference's
//    eight 32-bit AVX2 lanes. Integer sums are exact in any order; the float
//    FMA chain over superblocks runs in the reference's order inside each
//    thread, and the lanes are folded with hsum's tree via shuffles.
#include <algorithm>

#include "common.cuh"
#include "decode.h"
#include "kernels.h"

namespace kc {

constexpr int DR = 16;             // rows per unit
constexpr int DPAIRS = 6;          // consumer pairs
constexpr int DTHREADS = 32 + DPAIRS * 64;
constexpr int DMAX_STAGES = 48;
constexpr int DMAXS = 3;           // activation rows per unit

// ---------------------------------------------------------------------------
// Activation records. Q8_K (K-quant weights): per superblock 336 bytes =
// q[256] int8 | bsums[16] int32 | d f32 | pad. Q8 (Q8_0 weights): per chunk of
// 8 blocks 288 bytes = q[256] int8 | d[8] f32. Record stride = bytes per row.
__device__ __forceinline__ int64_t q8k_rec_stride(int64_t cols) { return cols / 256 * 336; }
__device__ __forceinline__ int64_t q8_rec_stride(int64_t cols) { return (cols / 32 + 7) / 8 * 288; }

// Q8KRow::quantize (qdot.rs:347-367) into records; optional SwiGLU first.
// One warp per (row, superblock): lane l owns elements 8l..8l+7.
__device__ __forceinline__ int i8_of4(uint32_t w, int b) { return (int)(int8_t)((w >> (8 * b)) & 0xFF); }

template <bool SWIGLU>
__global__ void q8k_records_kernel(const float* __restrict__ x, const float* __restrict__ u, int64_t n_rows,
                                   int64_t cols, uint8_t* __restrict__ rec, float* __restrict__ f32out,
                                   __half* __restrict__ f16out) {
  const int64_t nb = cols / 256;
  const int64_t gw = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (gw >= n_rows * nb) return;
  const int64_t r = gw / nb, b = gw % nb;
  const float* xp = x + r * cols + b * 256 + lane * 8;
  float v[8];
  {
    float4 a0 = reinterpret_cast<const float4*>(xp)[0], a1 = reinterpret_cast<const float4*>(xp)[1];
    v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w; v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
  }
  if (SWIGLU) {
    const float* up = u + r * cols + b * 256 + lane * 8;
    float4 b0 = reinterpret_cast<const float4*>(up)[0], b1 = reinterpret_cast<const float4*>(up)[1];
    float w[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i)  // transformer.rs:558: g / (1 + exp(-g)) * u
      v[i] = __fmul_rn(__fdiv_rn(v[i], __fadd_rn(1.0f, expf(-v[i]))), w[i]);
    if (f32out) {
      float4* o = reinterpret_cast<float4*>(f32out + r * cols + b * 256 + lane * 8);
      o[0] = make_float4(v[0], v[1], v[2], v[3]);
      o[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
    if (f16out) {
      __half2 h[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
      *reinterpret_cast<uint4*>(f16out + r * cols + b * 256 + lane * 8) = *reinterpret_cast<uint4*>(h);
    }
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float scale = __fdiv_rn(amax, 127.0f);
  const float inv = scale > 0.f ? __fdiv_rn(1.0f, scale) : 0.f;
  int s = 0;
  uint32_t packed[2] = {0, 0};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int qi = q8_round(__fmul_rn(v[i], inv));
    s += qi;
    packed[i / 4] |= (uint32_t)(qi & 0xFF) << (8 * (i % 4));
  }
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  uint8_t* rb = rec + r * q8k_rec_stride(cols) + b * 336;
  *reinterpret_cast<uint2*>(rb + lane * 8) = make_uint2(packed[0], packed[1]);
  if ((lane & 1) == 0) reinterpret_cast<int32_t*>(rb + 256)[lane / 2] = s;
  if (lane == 0) reinterpret_cast<float*>(rb + 320)[0] = scale;
}

// Q8Row::quantize (qdot.rs:29-49) into records; optional SwiGLU first. One
// warp per 32-block.
template <bool SWIGLU>
__global__ void q8_records_kernel(const float* __restrict__ x, const float* __restrict__ u, int64_t n_rows,
                                  int64_t cols, uint8_t* __restrict__ rec, float* __restrict__ f32out,
                                  __half* __restrict__ f16out) {
  const int64_t nb = cols / 32;
  const int64_t gw = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (gw >= n_rows * nb) return;
  const int64_t r = gw / nb, b = gw % nb;
  float v = x[r * cols + b * 32 + lane];
  if (SWIGLU) {
    v = __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, expf(-v))), u[r * cols + b * 32 + lane]);
    if (f32out) f32out[r * cols + b * 32 + lane] = v;
    if (f16out) f16out[r * cols + b * 32 + lane] = __float2half_rn(v);
  }
  float amax = fabsf(v);
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float scale = __fdiv_rn(amax, 127.0f);
  const float inv = scale > 0.f ? __fdiv_rn(1.0f, scale) : 0.f;
  const int qi = q8_round(__fmul_rn(v, inv));
  uint8_t* rb = rec + r * q8_rec_stride(cols) + (b / 8) * 288;
  rb[(b % 8) * 32 + lane] = (uint8_t)(int8_t)qi;
  if (lane == 0) reinterpret_cast<float*>(rb + 256)[b % 8] = scale;
}

void launch_act_records(bool kquant, const float* x, const float* u, int64_t n_rows, int64_t cols, uint8_t* rec,
                        float* f32out, __half* f16out, cudaStream_t st) {
  const int64_t warps = n_rows * (kquant ? cols / 256 : cols / 32);
  if (warps <= 0) return;
  const int grid = ceil_div(warps, 8);
  if (kquant) {
    if (u) q8k_records_kernel<true><<<grid, 256, 0, st>>>(x, u, n_rows, cols, rec, f32out, f16out);
    else q8k_records_kernel<false><<<grid, 256, 0, st>>>(x, u, n_rows, cols, rec, f32out, f16out);
  } else {
    if (u) q8_records_kernel<true><<<grid, 256, 0, st>>>(x, u, n_rows, cols, rec, f32out, f16out);
    else q8_records_kernel<false><<<grid, 256, 0, st>>>(x, u, n_rows, cols, rec, f32out, f16out);
  }
}

// ---------------------------------------------------------------------------
// Stage geometry: a stage is one 16-row tile x a segment of `ks` consecutive
// superblocks (Q8_0: chunks of 8 blocks), one contiguous range of the tiled
// device layout (common.cuh), fetched with a single bulk copy.
DecodeGeom decode_geom(int t, int64_t cols) {
  DecodeGeom g{};
  g.type = t;
  g.nb32 = t == T_Q8_0 ? (int)(cols / 32) : 0;
  g.nsb = tiled_nsb(t, cols);
  g.ks = std::min(g.nsb, t == T_Q8_0 ? 1 : 2);
  g.nseg = (g.nsb + g.ks - 1) / g.ks;
  g.tile_bytes = tiled_tile_bytes(t, cols);
  int mx = 0;
  for (int sg = 0; sg < g.nseg; ++sg) {
    const int a = sg * g.ks, b = std::min(g.nsb, a + g.ks);
    const int64_t end = b == g.nsb ? g.tile_bytes : tiled_sb_offset(t, cols, b);
    mx = std::max(mx, (int)(end - tiled_sb_offset(t, cols, a)));
  }
  g.stage_bytes = ((mx + 127) / 128) * 128;
  return g;
}

// hsum (avx2.rs:19-27) of the eight lanes held two per thread by four
// consecutive threads (thread q: lanes 2q, 2q+1). Valid in thread q == 0.
__device__ __forceinline__ float hsum8_quad(float a0, float a1) {
  a0 = __fadd_rn(a0, __shfl_down_sync(0xffffffffu, a0, 2, 4));  // v_i + v_{i+4}
  a1 = __fadd_rn(a1, __shfl_down_sync(0xffffffffu, a1, 2, 4));
  a0 = __fadd_rn(a0, __shfl_down_sync(0xffffffffu, a0, 1, 4));  // (t0 + t2), (t1 + t3)
  a1 = __fadd_rn(a1, __shfl_down_sync(0xffffffffu, a1, 1, 4));
  return __fadd_rn(a0, a1);
}
__device__ __forceinline__ int quad_sum(int v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1, 4);
  v += __shfl_xor_sync(0xffffffffu, v, 2, 4);
  return v;
}
__device__ __forceinline__ uint2 ldg2(const uint8_t* p) { return __ldg(reinterpret_cast<const uint2*>(p)); }
__device__ __forceinline__ int4 ldg4i(const uint8_t* p) { return __ldg(reinterpret_cast<const int4*>(p)); }
__device__ __forceinline__ float ldgf(const uint8_t* p) { return __ldg(reinterpret_cast<const float*>(p)); }

// Scale and min of Q4_K sub-block jj for a runtime jj (scale_min_k4,
// quant.rs:54-60), using shifts only.
__device__ __forceinline__ void q4k_sm_rt(int jj, uint32_t w0, uint32_t w1, uint32_t w2, int& s, int& m) {
  const int sh = 8 * (jj & 3);
  const uint32_t A = (w0 >> sh) & 0xFF, B = (w1 >> sh) & 0xFF, C = (w2 >> sh) & 0xFF;
  s = jj < 4 ? (int)(A & 63) : (int)((C & 0xF) | ((A >> 6) << 4));
  m = jj < 4 ? (int)(B & 63) : (int)((C >> 4) | ((B >> 6) << 4));
}

struct RowAcc {
  float a0[DMAXS], a1[DMAXS], summs[DMAXS];
};

// One superblock of a Q4_K row (avx2.rs:351-379), thread q of the row. xa[s]
// points at token s's activation record of this superblock.
template <int NS>
__device__ __forceinline__ void q4k_superblock(const uint8_t* __restrict__ sbt, int rr, const uint8_t* const* xa,
                                               int q, RowAcc& r) {
  const uint4 hdr = *reinterpret_cast<const uint4*>(sbt + 16 * rr);
  int sc[8], mn[8];
  q4k_scales(hdr.y, hdr.z, hdr.w, sc, mn);
  int lo[4][2], hi[4][2];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint2 w = *reinterpret_cast<const uint2*>(sbt + 256 + 512 * k + 32 * rr + 8 * q);
    lo[k][0] = (int)(w.x & 0x0F0F0F0Fu);
    hi[k][0] = (int)((w.x >> 4) & 0x0F0F0F0Fu);
    lo[k][1] = (int)(w.y & 0x0F0F0F0Fu);
    hi[k][1] = (int)((w.y >> 4) & 0x0F0F0F0Fu);
  }
  const float dw = h2f(hdr.x), dmw = h2f(hdr.x >> 16);
  // Sub-blocks 2q and 2q+1 of the min term (decoded with shifts: no indexed
  // register arrays), summed over the quad below.
  int mq0, mq1, dummy;
  q4k_sm_rt(2 * q, hdr.y, hdr.z, hdr.w, dummy, mq0);
  q4k_sm_rt(2 * q + 1, hdr.y, hdr.z, hdr.w, dummy, mq1);
#pragma unroll
  for (int s = 0; s < NS; ++s) {
    const uint8_t* x = xa[s];
    uint2 xl[4], xh[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      xl[k] = ldg2(x + 64 * k + 8 * q);
      xh[k] = ldg2(x + 64 * k + 32 + 8 * q);
    }
    const int4 bsq = ldg4i(x + 256 + 16 * q);  // bsums 4q..4q+3
    const float xd = ldgf(x + 320);
    int s0 = 0, s1 = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      s0 += sc[2 * k] * dp4a(lo[k][0], (int)xl[k].x, 0) + sc[2 * k + 1] * dp4a(hi[k][0], (int)xh[k].x, 0);
      s1 += sc[2 * k] * dp4a(lo[k][1], (int)xl[k].y, 0) + sc[2 * k + 1] * dp4a(hi[k][1], (int)xh[k].y, 0);
    }
    const int mins = quad_sum(mq0 * (bsq.x + bsq.y) + mq1 * (bsq.z + bsq.w));
    const float d = __fmul_rn(dw, xd), dmin = __fmul_rn(dmw, xd);
    r.a0[s] = __fmaf_rn((float)s0, d, r.a0[s]);
    r.a1[s] = __fmaf_rn((float)s1, d, r.a1[s]);
    r.summs[s] = __fadd_rn(r.summs[s], __fmul_rn(dmin, (float)mins));
  }
}

// One superblock of a planar Q6_K row segment (avx2.rs:384-419), thread q.
// Lanes 0-3 use the run's first sub-block scale, lanes 4-7 the second.
template <int NS>
__device__ __forceinline__ void q6k_superblock(const uint8_t* __restrict__ sbt, int rr, const uint8_t* const* xa,
                                               int q, RowAcc& r) {
  const uint4 scw = *reinterpret_cast<const uint4*>(sbt + 3072 + 16 * rr);
  const float dw = h2f(*reinterpret_cast<const uint16_t*>(sbt + 3328 + 2 * rr));
  uint2 ql[4], qh[2];
#pragma unroll
  for (int c = 0; c < 4; ++c) ql[c] = *reinterpret_cast<const uint2*>(sbt + 512 * c + 32 * rr + 8 * q);
#pragma unroll
  for (int h = 0; h < 2; ++h) qh[h] = *reinterpret_cast<const uint2*>(sbt + 2048 + 512 * h + 32 * rr + 8 * q);
  const int jh = q >> 1;
  const uint32_t sw[4] = {scw.x, scw.y, scw.z, scw.w};
  const uint32_t swq = (q & 2) ? ((q & 1) ? scw.w : scw.z) : ((q & 1) ? scw.y : scw.x);  // offsets m = 4q..4q+3
  int qv[8][2], scl[8];
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int ri = 0; ri < 4; ++ri) {
      const uint2 w = ql[2 * h + (ri & 1)];
      const int sh = 4 * (ri >> 1);
      qv[4 * h + ri][0] = (int)(((w.x >> sh) & 0x0F0F0F0Fu) | (((qh[h].x >> (2 * ri)) & 0x03030303u) << 4));
      qv[4 * h + ri][1] = (int)(((w.y >> sh) & 0x0F0F0F0Fu) | (((qh[h].y >> (2 * ri)) & 0x03030303u) << 4));
      const int m = 8 * h + 2 * ri;
      const int sc_lo = i8_of4(sw[m >> 2], m & 3), sc_hi = i8_of4(sw[(m + 1) >> 2], (m + 1) & 3);
      scl[4 * h + ri] = jh ? sc_hi : sc_lo;
    }
#pragma unroll
  for (int s = 0; s < NS; ++s) {
    const uint8_t* x = xa[s];
    int s0 = 0, s1 = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int ri = 0; ri < 4; ++ri) {
        const uint2 xv = ldg2(x + 128 * h + 32 * ri + 8 * q);
        s0 += scl[4 * h + ri] * dp4a(qv[4 * h + ri][0], (int)xv.x, 0);
        s1 += scl[4 * h + ri] * dp4a(qv[4 * h + ri][1], (int)xv.y, 0);
      }
    const int4 bsq = ldg4i(x + 256 + 16 * q);
    const int offs = quad_sum(i8_of4(swq, 0) * bsq.x + i8_of4(swq, 1) * bsq.y + i8_of4(swq, 2) * bsq.z +
                              i8_of4(swq, 3) * bsq.w);
    const float d = __fmul_rn(dw, ldgf(x + 320));
    r.a0[s] = __fmaf_rn((float)s0, d, r.a0[s]);
    r.a1[s] = __fmaf_rn((float)s1, d, r.a1[s]);
    // avx2.rs:416: lane 0 (thread 0's first lane) gets (-32*d)*offs, the
    // others +0.0.
    r.a0[s] = __fadd_rn(r.a0[s], q == 0 ? __fmul_rn(__fmul_rn(-32.0f, d), (float)offs) : 0.0f);
    r.a1[s] = __fadd_rn(r.a1[s], 0.0f);
  }
}

// One chunk of up to 8 Q8_0 blocks of a planar row segment (avx2.rs:49-58).
template <int NS>
__device__ __forceinline__ void q8_0_chunk(const uint8_t* __restrict__ cb, int nblk, int rr, const uint8_t* const* xa,
                                           int q, RowAcc& r) {
#pragma unroll 1
  for (int bl = 0; bl < nblk; ++bl) {
    const uint2 w = *reinterpret_cast<const uint2*>(cb + 512 * bl + 32 * rr + 8 * q);
    const float dw = h2f(*reinterpret_cast<const uint16_t*>(cb + 512 * nblk + 16 * rr + 2 * bl));
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      const uint2 x = ldg2(xa[s] + 32 * bl + 8 * q);
      const float sc = __fmul_rn(dw, ldgf(xa[s] + 256 + 4 * bl));
      r.a0[s] = __fmaf_rn((float)dp4a((int)w.x, (int)x.x, 0), sc, r.a0[s]);
      r.a1[s] = __fmaf_rn((float)dp4a((int)w.y, (int)x.y, 0), sc, r.a1[s]);
    }
  }
}

// Per-unit metadata, read by the producer and the consumers from shared
// memory (one table entry per expert of the CTA's unit range).
struct UnitMeta {
  int e, slot0, ns;
  int arow[DMAXS];
};
constexpr int DMETA = 96;

template <int T, int NS>
__device__ __forceinline__ void run_unit(const DecodeArgs& a, const DecodeGeom& g, uint8_t* smem, uint64_t* full,
                                         uint64_t* empty, int64_t stage0, int n_stages, int row, int q, int r_out,
                                         const UnitMeta& um, float* out, bool& ok) {
  RowAcc r;
#pragma unroll
  for (int s = 0; s < DMAXS; ++s) r.a0[s] = r.a1[s] = r.summs[s] = 0.f;
  const int rec = T == T_Q8_0 ? 288 : 336;
  for (int seg = 0; seg < g.nseg; ++seg) {
    const int64_t sid = stage0 + seg;
    const int st = (int)(sid % n_stages);
    const uint32_t ph = (uint32_t)((sid / n_stages) & 1);
    if (ok && !mbar_wait(&full[st], ph, a.status)) ok = false;
    if (ok) {
      const uint8_t* sp = smem + (int64_t)st * g.stage_bytes;
      const int sb0 = seg * g.ks;
      const int n = min(g.ks, g.nsb - sb0);
      for (int j = 0; j < n; ++j) {
        const uint8_t* xa[NS];
#pragma unroll
        for (int s = 0; s < NS; ++s) xa[s] = a.act + (int64_t)um.arow[s] * a.act_stride + (int64_t)rec * (sb0 + j);
        if (T == T_Q4_K) q4k_superblock<NS>(sp + 2304 * j, row, xa, q, r);
        else if (T == T_Q6_K) q6k_superblock<NS>(sp + 3360 * j, row, xa, q, r);
        else q8_0_chunk<NS>(sp + 4352 * j, min(8, g.nb32 - 8 * (sb0 + j)), row, xa, q, r);
      }
    }
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&empty[st]);
  }
#pragma unroll
  for (int s = 0; s < NS; ++s) {
    float v = hsum8_quad(r.a0[s], r.a1[s]);
    if (T == T_Q4_K) v = __fsub_rn(v, r.summs[s]);
    if (q == 0 && r_out >= 0 && ok) out[(int64_t)(um.slot0 + s) * a.out_stride + r_out] = v;
  }
}

__device__ __forceinline__ UnitMeta load_meta(const DecodeArgs& a, int li) {
  UnitMeta m;
  m.e = a.list[li];
  m.slot0 = a.offsets[m.e];
  m.ns = min(DMAXS, a.offsets[m.e + 1] - m.slot0);
#pragma unroll
  for (int s = 0; s < DMAXS; ++s) {
    const int slot = m.slot0 + min(s, m.ns - 1);
    m.arow[s] = a.slot_src ? a.slot_src[slot] : slot;
  }
  return m;
}

template <int T>
__global__ void __launch_bounds__(DTHREADS, 1) decode_kernel(DecodeArgs a, DecodeGeom g, int n_stages) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[DMAX_STAGES], empty[DMAX_STAGES];
  __shared__ UnitMeta meta[DMETA];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_list = *a.n_list;
  const int tiles = (int)(padded_rows(a.rows) / DR);
  const int per_expert = a.n_mat * tiles;
  const int64_t total = (int64_t)n_list * per_expert;
  const int64_t beg = total * blockIdx.x / gridDim.x, end = total * (blockIdx.x + 1) / gridDim.x;
  if (beg >= end) return;
  const int li0 = (int)(beg / per_expert);
  const int n_meta = min(DMETA, (int)((end - 1) / per_expert) - li0 + 1);
  for (int i = tid; i < n_meta; i += blockDim.x) meta[i] = load_meta(a, li0 + i);
  if (tid == 0) {
    for (int s = 0; s < n_stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 2);
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == 0) {
    // Producer: stages in unit order; unit u uses stages (u-beg)*nseg + seg.
    int64_t sid = 0;
    bool ok = true;
    for (int64_t u = beg; u < end && ok; ++u) {
      const int li = (int)(u / per_expert);
      const int m = (int)((u / tiles) % a.n_mat);
      const int r0 = (int)(u % tiles) * DR;
      const int e = li - li0 < DMETA ? meta[li - li0].e : a.list[li];
      const uint8_t* wb = (m == 0 ? a.w[0] : a.w[1]) + (int64_t)(e - a.expert_base) * a.expert_stride + (int64_t)(r0 / DR) * g.tile_bytes;
      for (int seg = 0; seg < g.nseg; ++seg, ++sid) {
        const int st = (int)(sid % n_stages);
        const uint32_t ph = (uint32_t)((sid / n_stages) & 1);
        if (sid >= n_stages && !mbar_wait(&empty[st], ph ^ 1, a.status)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          const int sb0 = seg * g.ks, sb1 = min(g.nsb, sb0 + g.ks);
          const int64_t off0 = tiled_sb_offset(g.type, a.cols, sb0);
          const int64_t off1 = sb1 == g.nsb ? g.tile_bytes : tiled_sb_offset(g.type, a.cols, sb1);
          const uint32_t bytes = (uint32_t)(off1 - off0);
          mbar_expect_tx(&full[st], bytes);
          bulk_g2s(smem + (int64_t)st * g.stage_bytes, wb + off0, bytes, &full[st]);
        }
        __syncwarp();
      }
    }
    // Keep the CTA alive until every issued copy has landed (bounded).
    if (lane == 0)
      for (int64_t k = (sid > n_stages ? sid - n_stages : 0); k < sid; ++k)
        mbar_wait(&full[k % n_stages], (uint32_t)((k / n_stages) & 1), a.status);
    return;
  }
  // Consumers: pair p = (warp-1)/2 takes units beg+p, beg+p+DPAIRS, ...
  const int p = (warp - 1) >> 1;
  const int t = tid - 32 - p * 64;  // 0..63
  const int row = t >> 2, q = t & 3;
  bool ok = true;
  for (int64_t u = beg + p; u < end; u += DPAIRS) {
    const int li = (int)(u / per_expert);
    const int m = (int)((u / tiles) % a.n_mat);
    const int r0 = (int)(u % tiles) * DR;
    const int nr = min(DR, a.rows - r0);
    const UnitMeta um = li - li0 < DMETA ? meta[li - li0] : load_meta(a, li);
    const int r_out = row < nr ? r0 + row : -1;  // padding rows (zeros) are computed, not stored
    const int64_t stage0 = (u - beg) * g.nseg;
    float* out = m == 0 ? a.out[0] : a.out[1];
    if (um.ns == 1) run_unit<T, 1>(a, g, smem, full, empty, stage0, n_stages, row, q, r_out, um, out, ok);
    else if (um.ns == 2) run_unit<T, 2>(a, g, smem, full, empty, stage0, n_stages, row, q, r_out, um, out, ok);
    else run_unit<T, 3>(a, g, smem, full, empty, stage0, n_stages, row, q, r_out, um, out, ok);
  }
}

template <int T>
static int launch_decode_t(const DecodeArgs& a, const DecodeGeom& g, int max_units, cudaStream_t st) {
  int n_stages = std::min(DMAX_STAGES, (int)((200 * 1024) / g.stage_bytes));
  if (n_stages < 2) return KC_ERR_SHAPE;
  const size_t smem = (size_t)n_stages * g.stage_bytes;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(decode_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    attr = true;
  }
  const int grid = std::min(num_sms(), std::max(1, max_units));
  decode_kernel<T><<<grid, DTHREADS, smem, st>>>(a, g, n_stages);
  return KC_OK;
}

int launch_decode(const DecodeArgs& a, int max_units, cudaStream_t st) {
  if (a.act_stride % 16 != 0) return KC_ERR_SHAPE;
  const DecodeGeom g = decode_geom(a.type, a.cols);
  switch (a.type) {
    case T_Q4_K: return launch_decode_t<T_Q4_K>(a, g, max_units, st);
    case T_Q6_K: return launch_decode_t<T_Q6_K>(a, g, max_units, st);
    case T_Q8_0: return launch_decode_t<T_Q8_0>(a, g, max_units, st);
    default: return KC_ERR_TYPE;
  }
}

}  // namespace kc
