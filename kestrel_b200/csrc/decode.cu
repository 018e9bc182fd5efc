// Decode-sized grouped dequant-dot: the reference's Q8_K / Q8Row integer
// kernels (crates/kestrel-engine/src/avx2.rs:49-58, 351-419) bit for bit, for
// experts with 1..3 routed rows and dense products with n < 4.
//
// Memory-bound design:
//  * Work unit = one 32-row tile of one expert matrix, streamed through the
//    row's K segments. Units are dealt to the CTAs round-robin, so each CTA
//    gets a mix of experts with 1, 2 and 3 rows; a CTA takes its units DW at
//    a time (a "group"); the producer warp issues the group's stages
//    segment-major (segment 0 of every unit, then segment 1, ...), so all
//    units of a group advance together through a deep ring of stages.
//  * A stage is the 32 rows x `ks` superblocks of a segment -- one contiguous
//    range of the tiled device layout (common.cuh), one cp.async.bulk --
//    followed by the unit's activation records (int8 values, block sums,
//    scale) of those superblocks, one bulk copy per superblock. The ring
//    (~220 KB per SM) is tracked by mbarriers.
//  * Consumers: 2 * DW warps. In a full group every unit has two warps, each
//    holding 16 rows with two threads per row, four of the reference's eight
//    32-bit AVX2 lanes per thread. The last, partial group of a CTA spreads
//    its units over all warps (four or eight threads per row), so the tail
//    does not run on a few warps. Scales are decoded per row-superblock in
//    each thread; the per-lane float chains run in superblock order as in the
//    reference, and the row's first thread gathers the eight lanes (warp
//    shuffles) for the hsum. Integer sums are exact in any order.
#include <algorithm>

#include "common.cuh"
#include "decode.h"
#include "decode_dev.cuh"
#include "kernels.h"

namespace kc {

// ---------------------------------------------------------------------------
// Activation records (layout in decode.h).
// Q8KRow::quantize (qdot.rs:347-367); optional SwiGLU first. One warp per
// (slot, superblock): lane l owns elements 8l..8l+7.
template <bool SWIGLU>
__global__ void q8k_records_kernel(const float* __restrict__ x, const float* __restrict__ u,
                                   const int* __restrict__ slot_src, int64_t n_slots, const int* __restrict__ n_slots_dev, int64_t cols,
                                   uint8_t* __restrict__ rec, int64_t rec_slots, float* __restrict__ f32out,
                                   __half* __restrict__ f16out) {
  pdl_enter();
  const int64_t nb = cols / 256;
  const int64_t gw = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (gw >= n_slots * nb) return;
  if (n_slots_dev && gw / nb >= *n_slots_dev) return;
  const int64_t slot = gw / nb, b = gw % nb;
  const int64_t src = slot_src ? slot_src[slot] : slot;
  const float* xp = x + src * cols + b * 256 + lane * 8;
  float v[8];
  {
    float4 a0 = reinterpret_cast<const float4*>(xp)[0], a1 = reinterpret_cast<const float4*>(xp)[1];
    v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w; v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
  }
  if (SWIGLU) {
    const float* up = u + src * cols + b * 256 + lane * 8;
    float4 b0 = reinterpret_cast<const float4*>(up)[0], b1 = reinterpret_cast<const float4*>(up)[1];
    float w[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i)  // transformer.rs:558: g / (1 + exp(-g)) * u
      v[i] = __fmul_rn(__fdiv_rn(v[i], __fadd_rn(1.0f, exp_rn(-v[i]))), w[i]);
    if (f32out) {
      float4* o = reinterpret_cast<float4*>(f32out + slot * cols + b * 256 + lane * 8);
      o[0] = make_float4(v[0], v[1], v[2], v[3]);
      o[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
  }
  if (f16out) {
    __half2 h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(f16out + slot * cols + b * 256 + lane * 8) = *reinterpret_cast<uint4*>(h);
  }
  if (!rec) return;
  q8k_store_record(v, rec + rec_index(b, slot, rec_slots) * kRecK, lane);
}

// Q8Row::quantize (qdot.rs:29-49); optional SwiGLU first. One warp per
// (slot, 32-block).
template <bool SWIGLU>
__global__ void q8_records_kernel(const float* __restrict__ x, const float* __restrict__ u,
                                  const int* __restrict__ slot_src, int64_t n_slots, const int* __restrict__ n_slots_dev, int64_t cols,
                                  uint8_t* __restrict__ rec, int64_t rec_slots, float* __restrict__ f32out,
                                  __half* __restrict__ f16out) {
  pdl_enter();
  const int64_t nb = cols / 32;
  const int64_t gw = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (gw >= n_slots * nb) return;
  if (n_slots_dev && gw / nb >= *n_slots_dev) return;
  const int64_t slot = gw / nb, b = gw % nb;
  const int64_t src = slot_src ? slot_src[slot] : slot;
  float v = x[src * cols + b * 32 + lane];
  if (SWIGLU) {
    v = __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, exp_rn(-v))), u[src * cols + b * 32 + lane]);
    if (f32out) f32out[slot * cols + b * 32 + lane] = v;
  }
  if (f16out) f16out[slot * cols + b * 32 + lane] = __float2half_rn(v);
  if (!rec) return;
  float amax = fabsf(v);
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float scale = __fdiv_rn(amax, 127.0f);
  const float inv = scale > 0.f ? __fdiv_rn(1.0f, scale) : 0.f;
  const int qi = q8_round(__fmul_rn(v, inv));
  uint8_t* rb = rec + ((b / 8) * rec_slots + slot) * kRecQ8;
  rb[(b % 8) * 32 + lane] = (uint8_t)(int8_t)qi;
  if (lane == 0) reinterpret_cast<float*>(rb + 256)[b % 8] = scale;
}

void launch_act_records(bool kquant, const float* x, const float* u, const int* slot_src, int64_t n_slots,
                        int64_t cols, uint8_t* rec, int64_t rec_slots, float* f32out, __half* f16out,
                        cudaStream_t st, const int* n_slots_dev) {
  const int64_t warps = n_slots * (kquant ? cols / 256 : cols / 32);
  if (warps <= 0) return;
  const int grid = ceil_div(warps, 8);
  if (kquant) {
    if (u) launch_k(q8k_records_kernel<true>, grid, 256, 0, st, x, u, slot_src, n_slots, n_slots_dev, cols, rec, rec_slots, f32out, f16out);
    else launch_k(q8k_records_kernel<false>, grid, 256, 0, st, x, u, slot_src, n_slots, n_slots_dev, cols, rec, rec_slots, f32out, f16out);
  } else {
    if (u) launch_k(q8_records_kernel<true>, grid, 256, 0, st, x, u, slot_src, n_slots, n_slots_dev, cols, rec, rec_slots, f32out, f16out);
    else launch_k(q8_records_kernel<false>, grid, 256, 0, st, x, u, slot_src, n_slots, n_slots_dev, cols, rec, rec_slots, f32out, f16out);
  }
}

// ---------------------------------------------------------------------------
// Stage geometry: a stage is one 32-row tile x a segment of `ks` consecutive
// superblocks (Q8_0: chunks of 8 blocks), followed by the unit's activation
// records for those superblocks: kStageSB (4) K-quant superblocks -- or the
// whole row when it has fewer -- or one Q8_0 chunk of 8 blocks per stage. The
// bulk-copy engine's throughput grows with the size of its copies up to
// ~18 KB (a B200 streaming probe: ~4 TB/s with 9.2 KB copies, 6.3-7 TB/s from
// 18 KB), so a Q4_K stage of four superblocks (18.4 KB of weights) gives a
// 9-stage ring; rows whose 4-superblock stages would leave no more than DW
// stages (Q6_K at ff = 14336) take two per stage. (Measured on configs[1] at
// 16 tokens: four superblocks per stage 5% faster per layer call than two;
// one superblock per stage 13% slower than two.)
DecodeGeom decode_geom(int t, int64_t cols) {
  DecodeGeom g = decode_geom_ks(t, cols, t == T_Q8_0 ? 1 : kStageSB);
  // Stages of more than two superblocks only while the ring keeps more than
  // DW of them.
  if (g.ks > 2 && DSMEM / g.stage_bytes <= DW) g = decode_geom_ks(t, cols, 2);
  return g;
}

DecodeGeom decode_geom_ks(int t, int64_t cols, int ks) {
  DecodeGeom g{};
  g.type = t;
  g.nb32 = t == T_Q8_0 ? (int)(cols / 32) : 0;
  g.nsb = tiled_nsb(t, cols);
  g.ks = std::max(1, std::min(g.nsb, ks));
  g.nseg = (g.nsb + g.ks - 1) / g.ks;
  g.tile_bytes = tiled_tile_bytes(t, cols);
  int mx = 0;
  for (int sg = 0; sg < g.nseg; ++sg) {
    const int a = sg * g.ks, b = std::min(g.nsb, a + g.ks);
    const int64_t end = b == g.nsb ? g.tile_bytes : tiled_sb_offset(t, cols, b);
    mx = std::max(mx, (int)(end - tiled_sb_offset(t, cols, a)));
  }
  g.rec_off = ((mx + 127) / 128) * 128;
  // Records of a stage: K-quant, per superblock pair of the stage the pair
  // block of up to DMAXS slots (two records each, whether the pair holds one
  // superblock or two); Q8, ks chunks of DMAXS records.
  const int rb = rec_bytes_of(t != T_Q8_0);
  const int rec_region = t != T_Q8_0 ? ((g.ks + 1) / 2) * DMAXS * 2 * rb : g.ks * DMAXS * rb;
  g.stage_bytes = ((g.rec_off + rec_region + 127) / 128) * 128;
  return g;
}


// Producer warps: warp p issues the stages of units p * DUP .. p * DUP + DUP - 1
// of each group (one lane per unit). Spreading the group's units over several
// warps lets their copies issue in parallel instead of one lane after another.
constexpr int DPW = 4;
constexpr int DUP = DW / DPW;  // units (lanes) per producer warp
constexpr int DEC_THREADS = 32 * (DC + DPW);
static_assert(DW % DPW == 0, "producer layout");

// Producer-warp barrier (named barrier 1): the DPW warps move from segment to
// segment together.
__device__ __forceinline__ void producer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(DPW * 32) : "memory");
}

template <int T>
__global__ void __launch_bounds__(DEC_THREADS, 1) decode_kernel(DecodeArgs a, DecodeGeom g, int n_stages) {
  // With a.early the expert list and offsets were written before the
  // previous kernel ran (only the activation records come from it): the
  // producer reads them (L2) and starts the first lap's weight copies before
  // waiting for the previous kernel, whose tail then overlaps the weight
  // stream's ramp. Otherwise everything waits first.
  if (a.early) pdl_trigger();
  else pdl_enter();
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[DMAX_STAGES], empty[DMAX_STAGES];
  __shared__ int rel[DMAX_STAGES];  // release counts per slot (count_wait)
  __shared__ int list_s[DMAX_E], off_s[DMAX_E + 1];
  constexpr int R = TypeR<T>::R;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_list = min(__ldcg(a.n_list), DMAX_E);
  const int tiles = (int)(padded_rows(a.rows) / DR);
  const int per_expert = a.n_mat * tiles;
  const int total = n_list * per_expert;
  if (total == 0) return;
  for (int i = tid; i < n_list; i += blockDim.x) list_s[i] = __ldcg(a.list + i);
  for (int i = tid; i <= a.n_experts && i <= DMAX_E; i += blockDim.x) off_s[i] = __ldcg(a.offsets + i);
  if (tid == 0) {
    for (int s = 0; s < n_stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], DARR);
      rel[s] = 0;
    }
    fence_mbar_init();
  }
  __syncthreads();
  // Units are dealt to the CTAs round-robin (unit b, b + G, b + 2G, ...): a
  // CTA's groups then mix experts with 1, 2 and 3 rows, whose compute
  // differs, and every CTA gets the same mix on average.
  const int G = gridDim.x, b = blockIdx.x;
  const int n_units = b < total ? (total - b + G - 1) / G : 0;
  if (n_units <= 0) return;
  const int n_groups = (n_units + DW - 1) / DW;
  uint8_t* ring = smem;
  auto unit_at = [&](int i) { return unit_pos(b + i * G, tiles, a.n_mat, a.tile_major, n_list); };

  if (warp < DPW) {
    // Producers: group by group, segment-major, one stage per (segment, unit):
    // the segment's weight bytes of the unit's 32-row tile (one bulk copy),
    // then the unit's activation records of each superblock of the segment
    // (one bulk copy per superblock: ns records are contiguous). Lane l of
    // producer warp p issues unit w = p * DUP + l's stage of every segment.
    // All 32 lanes of the producer warps run the loops (the named barrier
    // counts whole warps); lanes >= DUP issue nothing.
    int last = -1;  // highest stage number this lane issued
    const uint64_t wpol = l2_evict_first();  // weights are read once
    const int w = warp * DUP + lane;
    const bool lane_on = lane < DUP;
    bool ok = true;
    // Unit meta and byte ranges of group gi for this lane.
    // K-quant records: one copy per stage, the pair block of the unit's slots
    // (ns * 2 records; a stage's superblocks are one aligned pair). Q8 records:
    // one copy per chunk (a stage is one chunk).
    constexpr bool KQ = T != T_Q8_0;
    auto unit_ptrs = [&](int gi, const uint8_t*& up, const uint8_t*& rp, int& rbytes) {
      const UnitPos p = unit_at(gi * DW + w);
      const UnitMeta um = meta_at(list_s, off_s, p.li);
      up = (p.m == 0 ? a.w[0] : a.w[1]) + (int64_t)expert_pos(a.slot, um.e - a.expert_base) * a.expert_stride +
           (int64_t)p.tile * g.tile_bytes;
      rp = a.rec + (int64_t)um.slot0 * (KQ ? 2 * R : R);
      rbytes = um.ns * (KQ ? 2 * R : R);
    };
    // Record bytes of a stage (K-quant: one pair block per superblock pair).
    auto stage_rec_bytes = [&](int sb0, int sb1, int rbytes) {
      return KQ ? (uint32_t)(((sb1 - sb0 + 1) / 2) * rbytes) : (uint32_t)((sb1 - sb0) * rbytes);
    };
    if (a.early) {
      // First lap (stages 0 .. n_stages-1, no slot to wait for): weights now,
      // the records after the wait below.
      for (int gi = 0; gi < n_groups; ++gi) {
        const int wg = min(DW, n_units - gi * DW);
        if (gi * g.nseg * DW >= n_stages) break;
        const bool active = lane_on && w < wg;
        const uint8_t *up = nullptr, *rp = nullptr;
        int rbytes = 0;
        if (active) unit_ptrs(gi, up, rp, rbytes);
        int64_t off0 = 0;
        for (int seg = 0; seg < g.nseg; ++seg) {
          const int sb0 = seg * g.ks, sb1 = min(g.nsb, sb0 + g.ks);
          const int64_t off1 = sb1 == g.nsb ? g.tile_bytes : tiled_sb_offset(g.type, a.cols, sb1);
          const int sid = gi * g.nseg * DW + seg * wg + w;
          if (active && sid < n_stages) {
            const uint32_t wbytes = (uint32_t)(off1 - off0);
            mbar_expect_tx(&full[sid], wbytes + stage_rec_bytes(sb0, sb1, rbytes));
            bulk_g2s_hint(ring + (int64_t)sid * g.stage_bytes, up + off0, wbytes, &full[sid], wpol);
          }
          off0 = off1;
        }
      }
      pdl_wait();
    }
    for (int gi = 0; gi < n_groups; ++gi) {
      const int wg = min(DW, n_units - gi * DW);
      const bool active = lane_on && w < wg;
      const uint8_t *up = nullptr, *rp = nullptr;
      int rbytes = 0;
      if (active) unit_ptrs(gi, up, rp, rbytes);
      int64_t off0 = 0;
      for (int seg = 0; seg < g.nseg; ++seg) {
        const int sb0 = seg * g.ks, sb1 = min(g.nsb, sb0 + g.ks);
        const int64_t off1 = sb1 == g.nsb ? g.tile_bytes : tiled_sb_offset(g.type, a.cols, sb1);
        if (active && ok) {
          const int sid = gi * g.nseg * DW + seg * wg + w;
          const int st = sid % n_stages;
          const uint32_t ph = (uint32_t)((sid / n_stages) & 1);
          const bool weights_sent = a.early && sid < n_stages;
          if (sid >= n_stages && !mbar_wait(&empty[st], ph ^ 1u, a.status, W_DEC_EMPTY)) {
            ok = false;
          } else {
            const uint32_t wbytes = (uint32_t)(off1 - off0);
            uint8_t* dst = ring + (int64_t)st * g.stage_bytes;
            if (!weights_sent) {
              mbar_expect_tx(&full[st], wbytes + stage_rec_bytes(sb0, sb1, rbytes));
              bulk_g2s_hint(dst, up + off0, wbytes, &full[st], wpol);
            }
            if (KQ) {
              // sb0 is even (a multiple of the even kStageSB, or 0 when one
              // stage holds the whole row), so the stage's superblocks are
              // whole pairs (the last one possibly half).
              for (int pr = 0; pr < (sb1 - sb0 + 1) / 2; ++pr)
                bulk_g2s(dst + g.rec_off + pr * (DMAXS * 2 * R),
                         rp + (int64_t)((sb0 >> 1) + pr) * a.rec_slots * (2 * R), (uint32_t)rbytes, &full[st]);
            } else {
              for (int sb = sb0; sb < sb1; ++sb)
                bulk_g2s(dst + g.rec_off + (sb - sb0) * (DMAXS * R), rp + (int64_t)sb * a.rec_slots * R,
                         (uint32_t)rbytes, &full[st]);
            }
            last = sid;
          }
        }
        off0 = off1;
        // All producer lanes stay within one segment of each other (a lane
        // waiting for a slot could otherwise be passed by the others), so a
        // slot's previous lap (n_stages > DW stages back) is always issued
        // before a lane waits for its release. Every producer thread runs
        // the same (gi, seg) iterations, so all reach this barrier alike.
        producer_sync();
      }
    }
    // Keep the CTA alive until every copy has landed (bounded): one thread
    // waits for the last lap, stages nseg * n_units - n_stages .. the last
    // (the stage count is fixed, so no later lap of those slots exists).
    // After a failed wait some stages were never issued; their drain waits
    // end at the bound.
    (void)last;
    if (warp == 0 && lane == 0) {
      const int total = g.nseg * n_units;
      bool live = true;
      for (int k = max(0, total - n_stages); k < total && live; ++k)
        live = mbar_wait(&full[k % n_stages], (uint32_t)((k / n_stages) & 1), a.status, W_DEC_DRAIN);
    }
    return;
  }

  // Consumers: in group gi (wg units), warp c serves unit c / TPR with
  // TPR = tpr_of(wg) threads per row; the TPR warps of a unit split its 32
  // rows, 32 / TPR each.
  const int c = warp - DPW;
  bool ok = true;
  for (int gi = 0; gi < n_groups; ++gi) {
    const int wg = min(DW, n_units - gi * DW);
    const int tpr = tpr_of(wg);
    const int u = c / tpr;
    if (u >= wg) continue;
    const UnitPos p = unit_at(gi * DW + u);
    const UnitMeta um = meta_at(list_s, off_s, p.li);
    const int row = (c % tpr) * (DR / tpr) + lane / tpr;
    const int r = p.tile * DR + row;
    const int r_out = r < a.rows ? r : -1;  // padding rows are computed, not stored
    float* out = (p.m == 0 ? a.out[0] : a.out[1]) + (int64_t)um.slot0 * a.out_stride;
    const int sid0 = gi * g.nseg * DW + u;
    // Stage records: K-quant [slot][superblock of the pair], Q8 [chunk][slot].
    constexpr int SR = T != T_Q8_0 ? 2 * R : R, SBS = T != T_Q8_0 ? R : DMAXS * R;
    if (tpr == 2)
      run_unit_ns<T, 2, SR, SBS>(um.ns, a, g, ring, full, empty, rel, n_stages, sid0, wg, lane, row, out, r_out, ok);
    else if (tpr == 4)
      run_unit_ns<T, 4, SR, SBS>(um.ns, a, g, ring, full, empty, rel, n_stages, sid0, wg, lane, row, out, r_out, ok);
    else
      run_unit_ns<T, 8, SR, SBS>(um.ns, a, g, ring, full, empty, rel, n_stages, sid0, wg, lane, row, out, r_out, ok);
  }
}

template <int T>
static int launch_decode_t(const DecodeArgs& a, const DecodeGeom& g, int max_units, cudaStream_t st, int max_ctas) {
  const int n_stages = std::min(DMAX_STAGES, DSMEM / g.stage_bytes);
  if (n_stages <= DW) return KC_ERR_SHAPE;
  const size_t smem = (size_t)n_stages * g.stage_bytes;
  static PerDeviceOnce attr;
  if (smem_attr_once(attr, decode_kernel<T>, DSMEM) != cudaSuccess) return KC_ERR_CUDA;
  const int cap = max_ctas > 0 ? std::min(max_ctas, num_sms()) : num_sms();
  const int grid = std::min(cap, std::max(1, max_units));
  launch_k(decode_kernel<T>, grid, DEC_THREADS, smem, st, a, g, n_stages);
  return KC_OK;
}

int launch_decode(const DecodeArgs& a, int max_units, cudaStream_t st, int max_ctas) {
  if (a.rec_slots <= 0 || a.n_experts < 1 || a.n_experts > DMAX_E) return KC_ERR_SHAPE;
  const DecodeGeom g = decode_geom(a.type, a.cols);
  switch (a.type) {
    case T_Q4_K: return launch_decode_t<T_Q4_K>(a, g, max_units, st, max_ctas);
    case T_Q6_K: return launch_decode_t<T_Q6_K>(a, g, max_units, st, max_ctas);
    case T_Q8_0: return launch_decode_t<T_Q8_0>(a, g, max_units, st, max_ctas);
    default: return KC_ERR_TYPE;
  }
}

}  // namespace kc
