// Grouped quantized GEMM on the 5th-generation tensor cores (tcgen05), for the
// experts with >= 4 routed rows and dense products with n >= 4 -- the rows the
// reference sends through its exact path: dequantise to f32, then an f32 GEMM
// (crates/kestrel-engine/src/quant.rs:241-260).
//
// Per work tile: one expert, 128 weight rows (the MMA's M) x up to 128 slots
// (N), all of K. Roles:
//   warp 0 (1 thread)  producer: bulk copies of the raw quantized superblock
//                      tiles (tiled device layout, >= 4.6 KB each) and TMA
//                      tensor loads of the f16 activation tile (128B swizzle).
//   warp 1             TMEM allocation; one thread issues
//                      tcgen05.mma.cta_group::1.kind::f16 into f32 TMEM
//                      accumulators (gate and up side by side) and commits to
//                      mbarriers.
//   warps 2-5          dequantisation (thread = weight row) with the
//                      reference's float operations, rounded once to f16 and
//                      written in the canonical K-major SWIZZLE_128B layout;
//                      then the epilogue (tcgen05.ld -> global).
// Operands are f16 (11-bit significand), accumulation f32: results match the
// reference's f32 path within the 1e-3 tolerance, not bit for bit.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "mma.h"

namespace kc {

constexpr int MM = 128;       // weight rows per tile
constexpr int MK = 64;        // K elements per operand stage (one 128B swizzle atom)
constexpr int MN = kMmaTileN; // slots per tile (N of the MMA: up to 256)
constexpr int M_DQW = 8;      // dequantisation + epilogue warps (two per row: one per 32-element half)
constexpr int M_THREADS = 64 + 32 * M_DQW;
constexpr int M_OPS_MAX = 6;  // operand stages: as many as shared memory holds, 2 .. 6
constexpr int M_RAWS = 2;     // raw superblock stages
constexpr int A_BYTES = MM * MK * 2;  // 16 KB
constexpr int B_BYTES = MN * MK * 2;  // 32 KB: the activation tile of 256 slots

__host__ __device__ constexpr int max_sbt_bytes(int t) { return t == T_Q4_K ? 4608 : t == T_Q6_K ? 6720 : 8704; }
constexpr int M_RT = MM / kTileRows;  // row tiles per M tile

// A work item is 128 weight rows (the MMA's M) of MI matrices x up to NT
// 256-slot tiles, MI * NT <= 2 accumulators side by side in TMEM:
//  * MI = 2, NT = 1: gate and up of one slot tile, which share its B tile;
//  * MI = 1, NT = 2: one matrix for two slot tiles, so that every weight
//    block is copied and dequantised once for up to 512 slots (prefill).
__host__ __device__ constexpr int mma_raw_bytes(int t, int mi) {
  return ((mi * M_RT * max_sbt_bytes(t) + 1023) / 1024) * 1024;
}
__host__ __device__ constexpr int mma_op_bytes(int mi, int nt) { return mi * A_BYTES + nt * B_BYTES; }
// Dynamic shared memory of a launch: 227 KB per block less the kernel's
// static arrays (~4.2 KB, mostly the list prefix pp_s).
constexpr int M_SMEM_CAP = 227 * 1024 - 5 * 1024;
__host__ __device__ constexpr bool mma_fits(int t, int mi, int nt, int ops) {
  return ops * mma_op_bytes(mi, nt) + M_RAWS * mma_raw_bytes(t, mi) + 1024 <= M_SMEM_CAP;
}
// Rows of the TMA box (and of the activation stage) for tiles of up to n
// slots: 16, 32, 64, 128 or 256.
__host__ __device__ inline int box_rows(int n) {
  return n <= 16 ? 16 : n <= 32 ? 32 : n <= 64 ? 64 : n <= 128 ? 128 : 256;
}
// Stage geometry of a launch whose tiles hold at most bn slots (0: 256): the
// activation part of an operand stage holds box_rows(bn) rows, and there are
// as many operand stages as the shared memory holds (2 .. M_OPS_MAX).
struct MmaSmem {
  int op_bytes, b_bytes, raw_bytes, ops, total;
};
__host__ __device__ inline MmaSmem mma_smem(int t, int mi, int nt, int bn) {
  MmaSmem s;
  s.b_bytes = box_rows(bn > 0 ? bn : MN) * MK * 2;
  s.op_bytes = mi * A_BYTES + nt * s.b_bytes;
  s.raw_bytes = mma_raw_bytes(t, mi);
  const int room = M_SMEM_CAP - 1024 - M_RAWS * s.raw_bytes;
  s.ops = room / s.op_bytes < 2 ? 2 : (room / s.op_bytes > M_OPS_MAX ? M_OPS_MAX : room / s.op_bytes);
  s.total = s.ops * s.op_bytes + M_RAWS * s.raw_bytes + 1024;  // + alignment slack
  return s;
}
constexpr int MMA_MAX_LIST = 1024;  // experts of one launch's tcgen05 list

// ---- tcgen05 / TMA helpers --------------------------------------------------
// Shared-memory matrix descriptor: K-major, 128B swizzle, 8-row groups 1024 B
// apart (SBO), version 1 (sm_100).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
// Instruction descriptor, kind::f16: A = B = f16, D = f32, both K-major.
__device__ __forceinline__ uint32_t f16_idesc(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(MM >> 4) << 24);
}
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float v[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// ---- dequantisation of one row's 64-element K chunk into the A tile ----------
// Raw superblocks and the A tile are addressed through the 32-bit shared
// window (explicit ld/st.shared). Pairs of elements go through the packed
// f32x2 instructions, which round each lane exactly as the scalar ones do.
__device__ __forceinline__ uint4 m_lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint16_t m_lds16(uint32_t a) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
// f16x2 of the two lanes (lane 0 in the low half), each rounded to nearest.
__device__ __forceinline__ uint32_t f2_h2(uint64_t v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// Exact floats 2^23 + byte i and 2^23 + byte i+1 of w: each byte is placed
// under the exponent of 2^23 (full-rate byte permutes).
__device__ __forceinline__ uint64_t bytes_f2(uint32_t w, int i) {
  return f2_pack(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u | (uint32_t)i)),
                 __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u | (uint32_t)(i + 1))));
}

// Element k of row m goes to byte (m/8)*1024 + (m%8)*128 + ((k/8 ^ m%8)*16) +
// (k%8)*2: the canonical K-major SWIZZLE_128B layout; h holds 8 elements.
__device__ __forceinline__ void put8(uint32_t A, int m, int c, const uint32_t h[4]) {
  const uint32_t a = A + (m >> 3) * 1024 + (m & 7) * 128 + ((c ^ (m & 7)) << 4);
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(h[0]), "r"(h[1]), "r"(h[2]), "r"(h[3])
               : "memory");
}

// Scale and min of Q4_K sub-block jj (scale_min_k4, quant.rs:54-60).
__device__ __forceinline__ void mma_q4k_sm(int jj, uint32_t w0, uint32_t w1, uint32_t w2, int& s, int& m) {
  const int sh = 8 * (jj & 3);
  const uint32_t A = (w0 >> sh) & 0xFF, B = (w1 >> sh) & 0xFF, C = (w2 >> sh) & 0xFF;
  if (jj < 4) {
    s = A & 63;
    m = B & 63;
  } else {
    s = (C & 0xF) | ((A >> 6) << 4);
    m = (C >> 4) | ((B >> 6) << 4);
  }
}

// Half `hf` (32 elements) of the 64-element K chunk kk of a row, per type.
// Q4_K (quant.rs:138-155): y = (d*sc)*q - dmin*m; half 0 = sub-block 2kk (low
// nibbles), half 1 = sub-block 2kk+1 (high nibbles). d*sc has at most 17
// significant bits (an f16 times a 6-bit scale), so (d*sc)*q (q < 16) is exact
// in f32 and one fma(d*sc, q, -dmin*m) rounds exactly as the reference's
// multiply then subtract. High nibbles are read in place as 16q with the
// scale d*sc/16 (a power-of-two step: the same exact product).
__device__ __forceinline__ void dq_q4k(uint32_t sbt, int rr, int kk, int hf, uint32_t A, int m) {
  const uint4 hdr = m_lds128(sbt + 16 * rr);
  const uint4 q0 = m_lds128(sbt + kPlane + kPlane * (2 * kk) + 16 * rr);
  const uint4 q1 = m_lds128(sbt + kPlane + kPlane * (2 * kk + 1) + 16 * rr);
  const float d = h2f(hdr.x), dmin = h2f(hdr.x >> 16);
  int sc, mn;
  mma_q4k_sm(2 * kk + hf, hdr.y, hdr.z, hdr.w, sc, mn);
  const float d1 = __fmul_rn(__fmul_rn(d, (float)sc), hf ? 0.0625f : 1.0f), m1 = __fmul_rn(dmin, (float)mn);
  const uint64_t dd = f2_pack(d1, d1), mm = f2_pack(-m1, -m1), bias = f2_pack(8388608.0f, 8388608.0f);
  const uint32_t mask = hf ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
  const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t h[4];
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      const uint32_t nw = qw[2 * c + h2] & mask;
#pragma unroll
      for (int p = 0; p < 2; ++p) h[2 * h2 + p] = f2_h2(f2_fma(dd, f2_sub(bytes_f2(nw, 2 * p), bias), mm));
    }
    put8(A, m, 4 * hf + c, h);
  }
}

// Q6_K (quant.rs:180-201): y = (d*sc)*(q-32).
__device__ __forceinline__ void dq_q6k(uint32_t sbt, int rr, int kk, int hf, uint32_t A, int m) {
  const int h = kk >> 1, nib = kk & 1, r2 = 2 * nib + hf;
  // ql bytes 64h + 32hf .. +31 = chunks 4h + 2hf (+1); qh bytes 32h .. +31 = chunks 2h (+1).
  const uint32_t qlp = sbt + kPlane * (4 * h + 2 * hf) + 16 * rr;
  const uint32_t qhp = sbt + 8 * kPlane + kPlane * (2 * h) + 16 * rr;
  const uint4 l0 = m_lds128(qlp), l1 = m_lds128(qlp + kPlane);
  const uint4 h0 = m_lds128(qhp), h1 = m_lds128(qhp + kPlane);
  const uint4 scw = m_lds128(sbt + 12 * kPlane + 16 * rr);
  const float d = h2f(m_lds16(sbt + 13 * kPlane + 2 * rr));
  const uint32_t lw[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
  const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
  const uint64_t bias = f2_pack(8388640.0f, 8388640.0f);  // 2^23 + 32: q - 32
#pragma unroll
  for (int c = 0; c < 4; ++c) {  // 8 elements l = 8c .. 8c+7
    const int si = 8 * h + 2 * r2 + (c >> 1);
    const uint32_t swd = (si >> 3) ? ((si >> 2) & 1 ? scw.w : scw.z) : ((si >> 2) & 1 ? scw.y : scw.x);
    const float dsc = __fmul_rn(d, (float)(int)(int8_t)((swd >> (8 * (si & 3))) & 0xFF));
    const uint64_t dd = f2_pack(dsc, dsc);
    uint32_t hv[4];
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      const int wi = 2 * c + h2;
      const uint32_t qv = ((lw[wi] >> (4 * nib)) & 0x0F0F0F0Fu) | (((hw[wi] >> (2 * r2)) & 0x03030303u) << 4);
#pragma unroll
      for (int p = 0; p < 2; ++p) hv[2 * h2 + p] = f2_h2(f2_mul(dd, f2_sub(bytes_f2(qv, 2 * p), bias)));
    }
    put8(A, m, 4 * hf + c, hv);
  }
}

// Q8_0 (quant.rs:82-89): y = q*d; half hf = block 2kk + hf of the chunk.
__device__ __forceinline__ void dq_q8_0(uint32_t cb, int nblk, int rr, int kk, int hf, uint32_t A, int m) {
  const int b = 2 * kk + hf;
  const uint4 q0 = m_lds128(cb + kPlane * (2 * b) + 16 * rr);
  const uint4 q1 = m_lds128(cb + kPlane * (2 * b + 1) + 16 * rr);
  const float d = h2f(m_lds16(cb + 2 * kPlane * nblk + 16 * rr + 2 * b));
  const uint64_t dd = f2_pack(d, d), bias = f2_pack(8388736.0f, 8388736.0f);  // 2^23 + 128
  const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t h[4];
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      const uint32_t uw = qw[2 * c + h2] ^ 0x80808080u;  // q + 128 per byte
#pragma unroll
      for (int p = 0; p < 2; ++p) h[2 * h2 + p] = f2_h2(f2_mul(f2_sub(bytes_f2(uw, 2 * p), bias), dd));
    }
    put8(A, m, 4 * hf + c, h);
  }
}

struct MmaMapsDev {
  CUtensorMap m[kMmaBoxes];
};
static_assert(sizeof(MmaMapsDev) == sizeof(MmaMaps), "tensor map block");
// The box (index, rows) for a tile of nt slots: the smallest of 16 .. 256 rows
// that holds round16(nt).
__device__ __forceinline__ int box_index(int nt) {
  const int n16 = (nt + 15) / 16;  // 1 .. 16
  return n16 <= 1 ? 0 : (n16 <= 2 ? 1 : (n16 <= 4 ? 2 : (n16 <= 8 ? 3 : 4)));
}

// ---- work tiles ---------------------------------------------------------------
// Item w of a launch (before the split): the first of its MI matrices
// m = (w % (NMAT / MI)) * MI, row tile rt, then the expert's group of up to
// NT slot tiles. pp_s: prefix over the list of each expert's groups.
struct Tile {
  int e, m, rt, slot0, t0, np;
  int nt[2];  // slots of tile p of the group (nt[1] = 0 when np == 1)
};
template <int NMAT, int MI, int NT>
__device__ __forceinline__ Tile tile_of(const MmaArgs& a, const int* pp_s, int w, int row_tiles, int n_large) {
  Tile t;
  constexpr int per = NMAT / MI;
  t.m = (w % per) * MI;
  w /= per;
  t.rt = w % row_tiles;
  const int pi = w / row_tiles;
  int lo = 0, hi = n_large - 1;  // last i with pp_s[i] <= pi
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (pp_s[mid] <= pi) lo = mid;
    else hi = mid - 1;
  }
  t.e = a.list[lo];
  t.slot0 = a.offsets[t.e];
  const int n = a.offsets[t.e + 1] - t.slot0;
  t.t0 = (pi - pp_s[lo]) * NT * MN;
  t.nt[0] = min(MN, n - t.t0);
  t.nt[1] = NT > 1 ? max(0, min(MN, n - t.t0 - MN)) : 0;
  t.np = t.nt[1] > 0 ? 2 : 1;
  return t;
}

// Named barrier among the dequantisation/epilogue warps only.
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, %0;" ::"r"(32 * M_DQW) : "memory"); }

// Work items: (item, split). With few items (decode-sized batches) the K range
// of each item is split over S work items so that more SMs stream weights;
// each writes f32 partial tiles and the last one to finish (a per-item
// counter) adds the S partials in split order and stores the result.
__device__ __forceinline__ int split_count(const MmaArgs& a, int total, int nsb) {
  if (!a.part || total <= 0) return 1;
  const int s = min(nsb, (int)gridDim.x / total);
  return s >= 2 ? s : 1;
}

// Position in the operand-stage ring (its size is a launch value): slot and
// phase parity advance with each stage instead of dividing every time.
struct OpRing {
  int it = 0, slot = 0, n;
  uint32_t ph = 0;
  __device__ explicit OpRing(int n_) : n(n_) {}
  __device__ void next() {
    ++it;
    if (++slot == n) {
      slot = 0;
      ph ^= 1u;
    }
  }
};

template <int T, int NMAT, int MI, int NT>
__global__ void __launch_bounds__(M_THREADS, 1) mma_grouped_kernel(const MmaArgs a,
                                                                     const __grid_constant__ MmaMapsDev maps) {
  static_assert(MI * NT <= 2 && NMAT % MI == 0, "at most two accumulators of 256 columns");
  static_assert(mma_fits(T, MI, NT, 2), "two operand stages of 256-slot tiles fit");
  pdl_enter();
  extern __shared__ uint8_t msm_raw[];
  __shared__ __align__(8) uint64_t raw_full[M_RAWS], raw_empty[M_RAWS], op_full[M_OPS_MAX], op_empty[M_OPS_MAX];
  __shared__ __align__(8) uint64_t acc_full, acc_empty;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int last_sh;
  __shared__ int pp_s[MMA_MAX_LIST + 1];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_large = min(*a.n_list, MMA_MAX_LIST);
  // Groups of up to NT slot tiles per expert, prefix over the list.
  if (warp == 0) {
    int run = 0;
    for (int base = 0; base < n_large; base += 32) {
      const int i = base + lane;
      int c = i < n_large ? (a.tt_prefix[i + 1] - a.tt_prefix[i] + NT - 1) / NT : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, c, o);
        if (lane >= o) c += v;
      }
      if (i < n_large) pp_s[i + 1] = run + c;
      run += __shfl_sync(0xffffffffu, c, 31);
    }
    if (lane == 0) pp_s[0] = 0;
  }
  __syncthreads();
  const int row_tiles = (a.rows + MM - 1) / MM;
  const int total = n_large > 0 ? pp_s[n_large] * row_tiles * (NMAT / MI) : 0;
  const int nkc = a.cols / MK;
  const int nsb = tiled_nsb(T, a.cols);
  const int S = split_count(a, total, nsb);
  const int items = total * S;
  if ((int)blockIdx.x >= items) return;
  const MmaSmem L = mma_smem(T, MI, NT, a.bn);
  const int M_OPS = L.ops;
  uint8_t* msm = msm_raw + ((1024 - (smem_u32(msm_raw) & 1023)) & 1023);
  uint8_t* ops = msm;
  uint8_t* raws = msm + M_OPS * L.op_bytes;
  const int64_t tile_bytes = tiled_tile_bytes(T, a.cols);
  const int prows = (int)padded_rows(a.rows);
  const uint32_t tcols = MI * NT * MN;  // 256 or 512 TMEM columns
  // K chunks [kc0, kc1) of split s: whole superblocks (4 chunks of 64).
  auto k_range = [&](int s, int& kc0, int& kc1) {
    kc0 = 4 * (s * nsb / S);
    kc1 = min(nkc, 4 * ((s + 1) * nsb / S));
  };

  if (tid == 0) {
    for (int i = 0; i < M_RAWS; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], M_DQW);
    }
    for (int i = 0; i < M_OPS; ++i) {
      mbar_init(&op_full[i], 1 + M_DQW);
      mbar_init(&op_empty[i], 1);
    }
    mbar_init(&acc_full, 1);
    mbar_init(&acc_empty, M_DQW);
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_sh)),
                 "r"(tcols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {
      int raw_it = 0;
      OpRing op(M_OPS);
      const uint64_t wpol = l2_evict_first();
      for (int w = blockIdx.x; w < items && ok; w += gridDim.x) {
        const Tile t = tile_of<NMAT, MI, NT>(a, pp_s, w / S, row_tiles, n_large);
        int kc0, kc1;
        k_range(w % S, kc0, kc1);
        const int n_rt = min(M_RT, (prows - MM * t.rt) / kTileRows);
        // Only the rows each tile uses: boxes of 16 .. 256 rows.
        int bx[2] = {box_index(t.nt[0]), t.np > 1 ? box_index(t.nt[1]) : 0};
        const uint32_t b_bytes = (uint32_t)(MK * 2 * ((16 << bx[0]) + (t.np > 1 ? (16 << bx[1]) : 0)));
        // A tile larger than the launch's bound (the host's promise) would
        // overrun its stage: report it and stop (the other roles' bounded
        // waits then end).
        if ((16 << bx[0]) * MK * 2 > L.b_bytes || (t.np > 1 && (16 << bx[1]) * MK * 2 > L.b_bytes)) {
          report(a.status, KC_ERR_SHAPE | (W_MMA_BOUND << 8));
          ok = false;
          break;
        }
        for (int kc = kc0; kc < kc1 && ok; ++kc) {
          const int sb = kc >> 2;
          if ((kc & 3) == 0) {
            const int r = raw_it % M_RAWS;
            if (raw_it >= M_RAWS && !mbar_wait(&raw_empty[r], ((raw_it / M_RAWS) & 1) ^ 1, a.status, W_MMA_RAW_EMPTY)) {
              ok = false;
              break;
            }
            const uint32_t sbytes = (uint32_t)tiled_sbt_bytes(T, a.cols, sb);
            mbar_expect_tx(&raw_full[r], sbytes * n_rt * MI);
            uint8_t* rbase = raws + r * L.raw_bytes;
#pragma unroll
            for (int mt = 0; mt < MI; ++mt) {
              const uint8_t* src = a.w[t.m + mt] + (int64_t)expert_pos(a.slot, t.e - a.expert_base) * a.expert_stride +
                                   (int64_t)(M_RT * t.rt) * tile_bytes + tiled_sb_offset(T, a.cols, sb);
              for (int x = 0; x < n_rt; ++x) {
                if (a.read_once)
                  bulk_g2s_hint(rbase + (mt * M_RT + x) * max_sbt_bytes(T), src + x * tile_bytes, sbytes,
                                &raw_full[r], wpol);
                else
                  bulk_g2s(rbase + (mt * M_RT + x) * max_sbt_bytes(T), src + x * tile_bytes, sbytes, &raw_full[r]);
              }
            }
            ++raw_it;
          }
          const int o = op.slot;
          if (op.it >= M_OPS && !mbar_wait(&op_empty[o], op.ph ^ 1u, a.status, W_MMA_OP_EMPTY_P)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&op_full[o], b_bytes);
          for (int p = 0; p < t.np; ++p)
            tma_load_2d(ops + o * L.op_bytes + MI * A_BYTES + p * L.b_bytes, &maps.m[bx[p]], kc * MK,
                        t.slot0 + t.t0 + p * MN, &op_full[o]);
          op.next();
        }
      }
      // Drain: every issued copy lands before the CTA may exit.
      const int op_it = op.it;
      for (int i = std::max(0, op_it - M_OPS); i < op_it; ++i)
        mbar_wait(&op_full[i % M_OPS], (i / M_OPS) & 1, a.status, W_MMA_DRAIN);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int tile_it = 0;
      OpRing op(M_OPS);
      for (int w = blockIdx.x; w < items && ok; w += gridDim.x, ++tile_it) {
        const Tile t = tile_of<NMAT, MI, NT>(a, pp_s, w / S, row_tiles, n_large);
        int kc0, kc1;
        k_range(w % S, kc0, kc1);
        uint32_t idesc[2];
#pragma unroll
        for (int p = 0; p < 2; ++p) idesc[p] = f16_idesc(((max(t.nt[p], 1) + 15) / 16) * 16);
        if (tile_it > 0 && !mbar_wait(&acc_empty, (tile_it - 1) & 1, a.status, W_MMA_ACC_EMPTY)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kc = kc0; kc < kc1; ++kc) {
          const int o = op.slot;
          if (!mbar_wait(&op_full[o], op.ph, a.status, W_MMA_OP_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(ops + o * L.op_bytes);
          const uint32_t sbb = sa + MI * A_BYTES;
#pragma unroll
          for (int k16 = 0; k16 < MK / 16; ++k16) {
            const uint32_t acc = (kc > kc0 || k16 > 0) ? 1u : 0u;
#pragma unroll
            for (int mt = 0; mt < MI; ++mt) {
              const uint64_t ad = sw128_desc(sa + mt * A_BYTES + 32 * k16);
#pragma unroll
              for (int p = 0; p < NT; ++p)
                if (p < t.np)
                  umma_f16(tmem + (mt * NT + p) * MN, ad, sw128_desc(sbb + p * L.b_bytes + 32 * k16), idesc[p], acc);
            }
          }
          umma_commit(&op_empty[o]);
          op.next();
        }
        if (!ok) break;
        umma_commit(&acc_full);
      }
      // Drain: the tensor core has finished with TMEM before it is freed.
      const int op_it = op.it;
      if (op_it > 0) mbar_wait(&op_empty[(op_it - 1) % M_OPS], ((op_it - 1) / M_OPS) & 1, a.status, W_MMA_TC_DRAIN);
    }
  } else {
    // Dequantisation warps: thread t holds weight row m = t % 128 of the tile
    // and half hf = t / 128 of each 64-element K chunk.
    const int t_dq = tid - 64, m = t_dq & (MM - 1), hf = t_dq >> 7;
    const int rt_local = m / kTileRows, rr = m % kTileRows;
    int raw_it = 0, tile_it = 0;
    OpRing op(M_OPS);
    // Every dequantisation warp runs every item (failed waits only skip the
    // work), so all of them reach the named barriers below equally often.
    for (int w = blockIdx.x; w < items; w += gridDim.x, ++tile_it) {
      const int tile = w / S, split = w % S;
      const Tile t = tile_of<NMAT, MI, NT>(a, pp_s, tile, row_tiles, n_large);
      int kc0, kc1;
      k_range(split, kc0, kc1);
      int r = 0;
      for (int kc = kc0; kc < kc1; ++kc) {
        const int sb = kc >> 2, kk = kc & 3;
        if (kk == 0) {
          r = raw_it % M_RAWS;
          if (ok && !mbar_wait(&raw_full[r], (raw_it / M_RAWS) & 1, a.status, W_MMA_RAW_FULL)) ok = false;
        }
        const int o = op.slot;
        if (ok && op.it >= M_OPS && !mbar_wait(&op_empty[o], op.ph ^ 1u, a.status, W_MMA_OP_EMPTY_D)) ok = false;
        if (ok) {
#pragma unroll
          for (int mt = 0; mt < MI; ++mt) {
            const uint32_t A = smem_u32(ops + o * L.op_bytes + mt * A_BYTES);
            const uint32_t sbt = smem_u32(raws + r * L.raw_bytes + (mt * M_RT + rt_local) * max_sbt_bytes(T));
            if (T == T_Q4_K) dq_q4k(sbt, rr, kk, hf, A, m);
            else if (T == T_Q6_K) dq_q6k(sbt, rr, kk, hf, A, m);
            else dq_q8_0(sbt, min(8, a.cols / 32 - 8 * sb), rr, kk, hf, A, m);
          }
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&op_full[o]);
        op.next();
        if (kk == 3 || kc == kc1 - 1) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&raw_empty[r]);
          ++raw_it;
        }
      }
      // Epilogue: rows of this warp's TMEM quadrant (warp % 4); the two warps
      // of a quadrant take alternate 16-column blocks of each slot tile.
      if (ok && !mbar_wait(&acc_full, tile_it & 1, a.status, W_MMA_ACC_FULL)) ok = false;
      tc_fence_after();
      const int quad = warp & 3, colh = (warp - 2) >> 2;
      const int rl = quad * 32 + lane;
      const int row = MM * t.rt + rl;
      if (ok) {
#pragma unroll
        for (int mt = 0; mt < MI; ++mt)
          for (int p = 0; p < t.np; ++p) {
            const int n = ((t.nt[p] + 15) / 16) * 16;
            float* outm = a.out[t.m + mt];
            for (int c0 = 16 * colh; c0 < n; c0 += 32) {
              float v[16];
              tmem_ld16(tmem + ((uint32_t)(quad * 32) << 16) + (mt * NT + p) * MN + c0, v);
              if (S == 1) {
                if (row < a.rows) {
#pragma unroll
                  for (int i = 0; i < 16; ++i)
                    if (c0 + i < t.nt[p]) outm[(int64_t)(t.slot0 + t.t0 + p * MN + c0 + i) * a.out_stride + row] = v[i];
                }
              } else {
                float* pp = a.part + (((int64_t)w * MI + mt) * NT + p) * (MM * MN);
#pragma unroll
                for (int i = 0; i < 16; ++i)
                  if (c0 + i < t.nt[p]) pp[(c0 + i) * MM + rl] = v[i];
              }
            }
          }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty);
      if (S > 1) {
        // Last split of this item adds the partials in split order.
        __threadfence();
        epi_sync();
        if (tid == 64) last_sh = atomicAdd(&a.tile_cnt[tile], 1) == S - 1 ? 1 : 0;
        epi_sync();
        if (last_sh) {
          __threadfence();
          if (ok && row < a.rows) {
#pragma unroll
            for (int mt = 0; mt < MI; ++mt)
              for (int p = 0; p < t.np; ++p)
                for (int c = colh; c < t.nt[p]; c += 2) {
                  float acc = 0.f;
                  for (int s2 = 0; s2 < S; ++s2)
                    acc = __fadd_rn(acc, __ldcg(a.part + (((int64_t)(tile * S + s2) * MI + mt) * NT + p) * (MM * MN) +
                                                 c * MM + rl));
                  a.out[t.m + mt][(int64_t)(t.slot0 + t.t0 + p * MN + c) * a.out_stride + row] = acc;
                }
          }
          if (tid == 64) a.tile_cnt[tile] = 0;  // ready for the next launch
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tcols));
}

// ---- host side ------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

static int make_tmap_f16(void* map_out, const void* ptr, int64_t rows, int64_t cols, int box_rows) {
  if (!g_encode) {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return KC_ERR_CUDA;
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  if (((uintptr_t)ptr & 15) || (cols * 2) % 16) return KC_ERR_SHAPE;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)std::max<int64_t>(rows, 1)};
  cuuint64_t strides[1] = {(cuuint64_t)(cols * 2)};
  cuuint32_t box[2] = {MK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(reinterpret_cast<CUtensorMap*>(map_out), CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                        const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? KC_OK : KC_ERR_CUDA;
}

int make_tmaps_f16(MmaMaps& maps, const void* ptr, int64_t rows, int64_t cols) {
  for (int i = 0; i < kMmaBoxes; ++i) {
    const int rc = make_tmap_f16(maps.m[i], ptr, rows, cols, 16 << i);
    if (rc != KC_OK) return rc;
  }
  return KC_OK;
}

bool mma_supported(int t, int64_t cols, int n_mat) {
  if (!(t == T_Q4_K || t == T_Q6_K || t == T_Q8_0) || cols % MK != 0) return false;
  return n_mat == 2 ? mma_fits(t, 2, 1, 2) : mma_fits(t, 1, 1, 2);
}

template <int T, int NMAT, int MI, int NT>
static int launch_t(const MmaArgs& a, const MmaMaps& maps, int max_tiles, cudaStream_t st, int max_ctas) {
  const MmaSmem L = mma_smem(T, MI, NT, a.bn);
  static PerDeviceOnce attr;
  // Every stage geometry stays within M_SMEM_CAP: the attribute is set once to that.
  if (smem_attr_once(attr, mma_grouped_kernel<T, NMAT, MI, NT>, M_SMEM_CAP) != cudaSuccess) return KC_ERR_CUDA;
  // With a split-K workspace every SM gets a CTA (the kernel splits K when the
  // batch has few tiles); otherwise one CTA per tile at most.
  const int cap = max_ctas > 0 ? std::min(max_ctas, num_sms()) : num_sms();
  const int grid = a.part ? cap : std::max(1, std::min(cap, max_tiles));
  launch_k(mma_grouped_kernel<T, NMAT, MI, NT>, grid, M_THREADS, (size_t)L.total, st, a,
           *reinterpret_cast<const MmaMapsDev*>(&maps));
  return KC_OK;
}

// Item shape per type and launch: gate/up pairs (MI = 2) unless a.wide asks
// for two slot tiles per weight block; single matrices two tiles wide when
// a.wide and shared memory allows.
template <int T>
static int launch_type(const MmaArgs& a, const MmaMaps& maps, int max_tiles, cudaStream_t st, int max_ctas) {
  if (a.n_mat == 2) {
    if constexpr (mma_fits(T, 1, 2, 2))
      if (a.wide) return launch_t<T, 2, 1, 2>(a, maps, max_tiles, st, max_ctas);
    if constexpr (mma_fits(T, 2, 1, 2)) return launch_t<T, 2, 2, 1>(a, maps, max_tiles, st, max_ctas);
    return KC_ERR_SHAPE;
  }
  if constexpr (mma_fits(T, 1, 2, 2))
    if (a.wide) return launch_t<T, 1, 1, 2>(a, maps, max_tiles, st, max_ctas);
  return launch_t<T, 1, 1, 1>(a, maps, max_tiles, st, max_ctas);
}

size_t mma_part_bytes() { return (size_t)num_sms() * 2 * MM * MN * sizeof(float); }  // MI * NT <= 2 per item
size_t mma_cnt_bytes() { return (size_t)num_sms() * sizeof(int); }

int launch_mma_grouped(const MmaArgs& a, const MmaMaps& maps, int max_tiles, cudaStream_t st, int max_ctas) {
  if (max_tiles <= 0) return KC_OK;
  if (!mma_supported(a.type, a.cols, a.n_mat)) return KC_ERR_SHAPE;
  if (a.type == T_Q4_K) return launch_type<T_Q4_K>(a, maps, max_tiles, st, max_ctas);
  if (a.type == T_Q6_K) return launch_type<T_Q6_K>(a, maps, max_tiles, st, max_ctas);
  return launch_type<T_Q8_0>(a, maps, max_tiles, st, max_ctas);
}

}  // namespace kc
