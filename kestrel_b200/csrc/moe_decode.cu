// The routed-expert layer of a decode batch in one persistent launch: the
// arithmetic of router_logits_kernel, route_kernel, dispatch_kernel, the
// records kernels, decode_kernel (gate/up, then down) and combine_kernel,
// bit for bit, without the seven launch boundaries between them. One CTA per
// SM; every CTA holds the whole batch's routing in shared memory.
//
//  Phase 0 (all CTAs): router logits (CTA b computes experts b, b + G, ... for
//    every token, rows staged by bulk copies, the router rows issued before
//    the wait on the previous kernel) and the Q8_K / Q8 records of the input
//    rows (the other warps); zero the completion counters. Grid barrier.
//  Phase 1 (every CTA, redundantly): top-k of every token (route_row) and the
//    dispatch metadata (slots grouped by ascending expert, tokens ascending
//    within an expert; each token's selections ordered by expert id for the
//    combine), all in shared memory. CTA 0 publishes ids / weights.
//  Phase 2 (all CTAs): decode_kernel's producer / consumer ring over a unit
//    sequence that holds the gate/up units (expert, matrix, 32-row tile),
//    then the down units (expert, 32-row tile), dealt round-robin over the
//    CTAs. A warp that finishes rows adds them to the counter of its (expert,
//    256-row chunk); the warp completing a chunk writes the SwiGLU records of
//    the expert's slots for it and raises the chunk's ready flag. The producer
//    issues a down stage's weights at once and its records after the flags of
//    its chunks are up. Down rows count per 32-row output tile; the warp
//    completing a tile forms the combine of that tile for every token.
//
// All cross-CTA waits (grid barrier, ready flags) and mbarrier waits are
// bounded; a CTA only waits on work of CTAs that are resident (the grid is at
// most one CTA per SM at one CTA per SM occupancy, and phase-2 waits point at
// gate/up work, which never waits on anything).
#include <algorithm>

#include "common.cuh"
#include "decode_dev.cuh"
#include "kernels.h"
#include "moe_decode.h"
#include "route_dev.cuh"

namespace kc {

constexpr int MK_MAXT = 3;      // tokens: experts then get at most three rows (the int8 path)
constexpr int MK_MAXK = 16;
constexpr int MK_MAXA = MK_MAXT * MK_MAXK;
constexpr int MK_MAX_E = 512;
constexpr int MK_SMEM = 210 * 1024;
constexpr int MK_HDR = 32;      // sync words: [0] barrier count, [1] barrier generation
// Bytes one mbarrier phase waits for (expect_tx) in phase 0. Every other
// mbarrier in this library waits for at most ~37 KB per phase; a phase-0
// buffer of exactly 64 KB (4 rows of 16 KB at d = 4096) faulted the GPU, so
// phase 0 stays within 32 KB per buffer.
constexpr int MK_MAX_TX = 32 * 1024;

int moe_decode_sync_words(int E, int ff, int d) {
  const int nch = (ff + 255) / 256;
  return MK_HDR + 2 * E * nch + (int)(padded_rows(d) / DR);
}

struct MkParams {
  MoeDecodeArgs a;
  DecodeGeom gu, dn;  // stage_bytes of both = the ring's slot size
  int n_stages;
  int kc;             // phase-0 K chunk (floats)
};

// run_unit's view of the output.
struct UnitArgs {
  int* status;
  int64_t out_stride;
};

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(int* p, int v) {
  asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Orders this thread's earlier generic-proxy observations (a ready flag and
// the data it guards) before its later bulk copies, which read through the
// async proxy.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Bounded wait until *f != 0.
__device__ bool wait_flag(const int* f, int* status) {
  if (ld_acquire(f) != 0) return true;
  const uint64_t t0 = globaltimer();
  while (ld_acquire(f) == 0) {
    if (globaltimer() - t0 > kWaitLimitNs) {
      report(status, KC_ERR_TIMEOUT | (W_MK_FLAG << 8));
      return false;
    }
    __nanosleep(32);
  }
  return true;
}

// Grid-wide barrier: a count and a generation word. The last CTA to arrive
// resets the count and advances the generation; the others wait (bounded) for
// the generation read before they arrived to change.
__device__ bool grid_barrier(int* bar, int* status, int* ok_s) {
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    const int g0 = ld_acquire(bar + 1);
    __threadfence();
    const int old = atomicAdd(bar, 1);
    if (old == (int)gridDim.x - 1) {
      atomicExch(bar, 0);
      __threadfence();
      atomicAdd(bar + 1, 1);
    } else {
      const uint64_t t0 = globaltimer();
      while (ld_acquire(bar + 1) == g0) {
        if (globaltimer() - t0 > kWaitLimitNs) {
          report(status, KC_ERR_TIMEOUT | (W_MK_BARRIER << 8));
          ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
    __threadfence();
    *ok_s = ok;
  }
  __syncthreads();
  return *ok_s != 0;
}

// Q8Row::quantize of one 32-block held one value per lane (q8_records_kernel's
// arithmetic), into block bl of the Q8 record rb.
__device__ __forceinline__ void q8_store_block(float v, uint8_t* rb, int bl, int lane) {
  float amax = fabsf(v);
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float scale = __fdiv_rn(amax, 127.0f);
  const float inv = scale > 0.f ? __fdiv_rn(1.0f, scale) : 0.f;
  rb[bl * 32 + lane] = (uint8_t)(int8_t)q8_round(__fmul_rn(v, inv));
  if (lane == 0) reinterpret_cast<float*>(rb + 256)[bl] = scale;
}

// transformer.rs:558: g / (1 + exp(-g)) * u.
__device__ __forceinline__ float swiglu1(float g, float u) {
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, exp_rn(-g))), u);
}

template <int TG, int TD>
__global__ void __launch_bounds__(DTHREADS, 1) moe_decode_kernel(MkParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[DMAX_STAGES], empty[DMAX_STAGES], p0bar[2];
  __shared__ int list_s[MK_MAX_E], off_s[MK_MAX_E + 1];
  __shared__ int slot_tok_s[MK_MAXA], csl_s[MK_MAXA];
  __shared__ float cwt_s[MK_MAXA];
  __shared__ int nlist_s, ok_s;
  const MoeDecodeArgs& a = p.a;
  constexpr int RG = TypeR<TG>::R, RD = TypeR<TD>::R;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, b = blockIdx.x;
  const int n = a.n_tok, E = a.E, k = a.k, d = a.d, ff = a.ff, A = n * k;
  const DecodeGeom& gu = p.gu;
  const DecodeGeom& dn = p.dn;
  const int nch = dn.nsb;  // 256-element chunks of the down input
  int* cnt = a.sync + MK_HDR;
  int* flags = cnt + E * nch;
  int* tcnt = flags + E * nch;
  const int tg = (int)(padded_rows(ff) / DR), td = (int)(padded_rows(d) / DR);

  // ---- Phase 0: router logits, input records, counters --------------------
  const int kc = p.kc, kcp = kc + 8;  // padded shared rows: a warp's 4 token rows hit distinct banks
  const int nchunk = (d + kc - 1) / kc;
  const int my_e = b < E ? (E - b + G - 1) / G : 0;
  const int total_q = my_e * nchunk;
  float* pbuf = reinterpret_cast<float*>(smem);  // [2][1 + n][kcp]
  const int nlog = n * 8, lw = (nlog + 31) / 32;  // logit threads, and the warps holding them
  if (tid == 0) {
    mbar_init(&p0bar[0], 1);
    mbar_init(&p0bar[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto chunk_of = [&](int q, int& e, int& k0, int& kn) {
    e = b + (q / nchunk) * G;
    k0 = (q % nchunk) * kc;
    kn = min(kc, d - k0);
  };
  auto issue_router = [&](int q) {
    int e, k0, kn;
    chunk_of(q, e, k0, kn);
    float* buf = pbuf + (q & 1) * (1 + n) * kcp;
    mbar_expect_tx(&p0bar[q & 1], (uint32_t)kn * 4u * (uint32_t)(1 + n));
    bulk_g2s(buf, a.router + (int64_t)e * d + k0, (uint32_t)kn * 4u, &p0bar[q & 1]);
  };
  auto issue_rows = [&](int q) {
    int e, k0, kn;
    chunk_of(q, e, k0, kn);
    float* buf = pbuf + (q & 1) * (1 + n) * kcp;
    for (int s = 0; s < n; ++s)
      bulk_g2s(buf + (1 + s) * kcp, a.h + (int64_t)s * d + k0, (uint32_t)kn * 4u, &p0bar[q & 1]);
  };
  // The router is constant: its rows stream before the wait on the previous
  // kernel, which wrote h.
  if (tid == 0)
    for (int q = 0; q < min(2, total_q); ++q) issue_router(q);
  pdl_wait();
  pdl_trigger();
  if (tid == 0)
    for (int q = 0; q < min(2, total_q); ++q) issue_rows(q);
  {
    const int nz = 2 * E * nch + td;
    for (int i = b * blockDim.x + tid; i < nz; i += G * blockDim.x) cnt[i] = 0;
  }
  if (warp < lw) {
    // Logits of (expert e, token s) by the 8 threads s*8 .. s*8+7 (lane j):
    // router_logits_kernel's per-lane chains and folds.
    const int s = tid >> 3, j = tid & 7;
    const bool valid = tid < nlog;
    const bool gemm = n >= 4;
    float a0 = 0.f, a1 = 0.f;
    bool m1 = false, okw = true;
    for (int q = 0; q < total_q; ++q) {
      int e, k0, kn;
      chunk_of(q, e, k0, kn);
      if (q % nchunk == 0) {
        a0 = 0.f;
        a1 = 0.f;
        const int tile = e / 48, trows = min(48, E - tile * 48), rows3 = trows / 3 * 3;
        m1 = !((e - tile * 48) < rows3 && s < n / 4 * 4);
      }
      // After a timed-out wait the thread stays in the loop (the named barrier
      // below counts every logit thread) but waits and computes no more.
      if (okw && !mbar_wait(&p0bar[q & 1], (uint32_t)((q >> 1) & 1), a.status, W_MK_ROUTER)) okw = false;
      if (valid && okw) {
        const float* buf = pbuf + (q & 1) * (1 + n) * kcp;
        const float* wr = buf + j;
        const float* xr = buf + (1 + s) * kcp + j;
        int cc = 0;
        for (; cc + 64 <= kn; cc += 64) {
          float wv[8], xv[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            wv[u] = wr[cc + 8 * u];
            xv[u] = xr[cc + 8 * u];
          }
          if (gemm) {
#pragma unroll
            for (int u = 0; u < 8; ++u) rl_step<true>(wv[u], xv[u], u & 1, m1, a0, a1);
          } else {
#pragma unroll
            for (int u = 0; u < 8; ++u) rl_step<false>(wv[u], xv[u], u & 1, m1, a0, a1);
          }
        }
        for (; cc < kn; cc += 8) {
          if (gemm) rl_step<true>(wr[cc], xr[cc], (cc >> 3) & 1, m1, a0, a1);
          else rl_step<false>(wr[cc], xr[cc], (cc >> 3) & 1, m1, a0, a1);
        }
      }
      if (q % nchunk == nchunk - 1) {
        float v;
        if (!gemm) {
          float sum = -0.0f;
#pragma unroll
          for (int l = 0; l < 8; ++l) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, a0, l, 8));
          v = sum;
        } else {
          v = hsum8_group(m1 ? __fadd_rn(a0, a1) : a0);
        }
        if (valid && j == 0) a.logits[(int64_t)s * E + e] = v;
      }
      if (q + 2 < total_q) {
        // Every logit thread is done with buffer q & 1 before it is refilled.
        asm volatile("bar.sync 1, %0;" ::"r"(lw * 32) : "memory");
        if (tid == 0) {
          issue_router(q + 2);
          issue_rows(q + 2);
        }
      }
    }
  } else {
    // Activation records of the input rows, one warp per (token, chunk of 256).
    const int nrw = DC + 1 - lw;
    const int nrc = tiled_nsb(TG, d);
    for (int t = b * nrw + (warp - lw); t < n * nrc; t += G * nrw) {
      const int s = t / nrc, c = t - s * nrc;
      const float* xp = a.h + (int64_t)s * d + (int64_t)c * 256;
      uint8_t* rb = a.xrec + ((int64_t)c * n + s) * RG;
      if (TG != T_Q8_0) {
        const float4 x0 = reinterpret_cast<const float4*>(xp + lane * 8)[0];
        const float4 x1 = reinterpret_cast<const float4*>(xp + lane * 8)[1];
        const float v[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        q8k_store_record(v, rb, lane);
      } else {
        const int nblk = min(8, d / 32 - 8 * c);
        for (int bl = 0; bl < nblk; ++bl) q8_store_block(xp[bl * 32 + lane], rb, bl, lane);
      }
    }
  }
  if (!grid_barrier(a.sync, a.status, &ok_s)) return;

  // ---- Phase 1: top-k and dispatch, in every CTA ---------------------------
  {
    float* lg_s = reinterpret_cast<float*>(smem);          // [n][E] logits
    float* p_s = lg_s + n * E;                              // [n][E] probabilities
    float* selw_s = p_s + n * E;                            // [n][RT_MAXK]
    int* seli_s = reinterpret_cast<int*>(selw_s + n * RT_MAXK);
    int* ids_s = seli_s + n * RT_MAXK;                      // [A]
    float* w_s = reinterpret_cast<float*>(ids_s + A);       // [A]
    int* cnt_s = reinterpret_cast<int*>(w_s + A);           // [E]
    for (int i = tid; i < n * E; i += blockDim.x) lg_s[i] = __ldcg(a.logits + i);
    for (int i = tid; i < E; i += blockDim.x) cnt_s[i] = 0;
    __syncthreads();
    if (warp < n)
      route_row(lg_s + warp * E, E, k, a.norm_topk, a.weights_scale, p_s + warp * E, selw_s + warp * RT_MAXK,
                seli_s + warp * RT_MAXK, lane, ids_s + warp * k, w_s + warp * k);
    __syncthreads();
    for (int i = tid; i < A; i += blockDim.x) {
      const int e = ids_s[i];
      if (e >= 0 && e < E) atomicAdd(&cnt_s[e], 1);
    }
    __syncthreads();
    if (warp == 0) {
      // Slot offsets in expert order, and the list of experts with rows.
      int base = 0, lbase = 0;
      for (int e0 = 0; e0 < E; e0 += 32) {
        const int e = e0 + lane;
        const int c = e < E ? cnt_s[e] : 0, f = c > 0 ? 1 : 0;
        int ic = c, il = f;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int t1 = __shfl_up_sync(0xffffffffu, ic, o), t2 = __shfl_up_sync(0xffffffffu, il, o);
          if (lane >= o) {
            ic += t1;
            il += t2;
          }
        }
        if (e < E) {
          off_s[e] = base + ic - c;
          if (f) list_s[lbase + il - 1] = e;
        }
        base += __shfl_sync(0xffffffffu, ic, 31);
        lbase += __shfl_sync(0xffffffffu, il, 31);
      }
      if (lane == 0) {
        off_s[E] = base;
        nlist_s = lbase;
      }
    }
    __syncthreads();
    for (int i = tid; i < A; i += blockDim.x) {
      const int s = i / k, jj = i - s * k, e = ids_s[i];
      int slot = -1;
      if (e >= 0 && e < E) {
        int rank = 0;  // earlier tokens that chose e (tokens ascend within an expert)
        for (int i2 = 0; i2 < s * k; ++i2) rank += ids_s[i2] == e ? 1 : 0;
        slot = off_s[e] + rank;
        slot_tok_s[slot] = s;
      }
      int r = 0;  // position of the selection in the token's expert-id order
      for (int j2 = 0; j2 < k; ++j2) {
        const int e2 = ids_s[s * k + j2];
        r += (e2 < e || (e2 == e && j2 < jj)) ? 1 : 0;
      }
      csl_s[s * k + r] = slot;
      cwt_s[s * k + r] = w_s[i];
      if (b == 0) {
        a.ids[i] = e;
        a.w[i] = w_s[i];
      }
    }
    if (tid == 0) {
      for (int s = 0; s < p.n_stages; ++s) {
        mbar_init(&full[s], 1);
        mbar_init(&empty[s], DARR);
      }
      fence_mbar_init();
    }
    __syncthreads();
  }

  // ---- Phase 2: gate/up units, then down units ------------------------------
  const int n_list = nlist_s;
  const int U_gu = n_list * 2 * tg, U = U_gu + n_list * td;
  const int n_units = b < U ? (U - b + G - 1) / G : 0;
  const int n_gu = b < U_gu ? (U_gu - b + G - 1) / G : 0;
  const int n_dn = n_units - n_gu;
  const int n_stages = p.n_stages;
  const int base_dn = n_gu * gu.nseg;  // first stage of the down units
  uint8_t* ring = smem;
  auto gu_pos = [&](int i) { return unit_pos(b + i * G, tg, 2); };
  auto dn_pos = [&](int j) { return unit_pos(b + (n_gu + j) * G - U_gu, td, 1); };

  if (warp == 0) {
    int last = -1;  // highest stage number this lane issued in full
    if (lane < DW) {
      const int w = lane;
      bool ok = true;
      for (int gi = 0; gi * DW < n_gu; ++gi) {
        const int wg = min(DW, n_gu - gi * DW);
        const bool active = w < wg;
        UnitMeta um{};
        const uint8_t* up = nullptr;
        if (active) {
          const UnitPos ps = gu_pos(gi * DW + w);
          um = meta_at(list_s, off_s, ps.li);
          up = (ps.m == 0 ? a.gate : a.up) + (int64_t)um.e * a.mb_gate + (int64_t)ps.tile * gu.tile_bytes;
        }
        int64_t off0 = 0;
        for (int seg = 0; seg < gu.nseg; ++seg) {
          const int sb0 = seg * gu.ks, sb1 = min(gu.nsb, sb0 + gu.ks);
          const int64_t off1 = sb1 == gu.nsb ? gu.tile_bytes : tiled_sb_offset(TG, d, sb1);
          if (active && ok) {
            const int sid = gi * gu.nseg * DW + seg * wg + w;
            const int st = sid % n_stages;
            const uint32_t ph = (uint32_t)((sid / n_stages) & 1);
            if (sid >= n_stages && !mbar_wait(&empty[st], ph ^ 1u, a.status, W_DEC_EMPTY)) {
              ok = false;
            } else {
              const uint32_t wbytes = (uint32_t)(off1 - off0);
              uint8_t* dst = ring + (int64_t)st * gu.stage_bytes;
              mbar_expect_tx(&full[st], wbytes + (uint32_t)((sb1 - sb0) * um.ns * RG));
              bulk_g2s(dst, up + off0, wbytes, &full[st]);
              for (int sb = sb0; sb < sb1; ++sb)
                for (int s = 0; s < um.ns; ++s)
                  bulk_g2s(dst + gu.rec_off + (sb - sb0) * (DMAXS * RG) + s * RG,
                           a.xrec + ((int64_t)sb * n + slot_tok_s[um.slot0 + s]) * RG, (uint32_t)RG, &full[st]);
              last = sid;
            }
          }
          off0 = off1;
          __syncwarp((1u << DW) - 1u);
        }
      }
      for (int gj = 0; gj * DW < n_dn; ++gj) {
        const int wg = min(DW, n_dn - gj * DW);
        const bool active = w < wg;
        UnitMeta um{};
        int li = 0;
        const uint8_t* up = nullptr;
        if (active) {
          const UnitPos ps = dn_pos(gj * DW + w);
          li = ps.li;
          um = meta_at(list_s, off_s, ps.li);
          up = a.down + (int64_t)um.e * a.mb_down + (int64_t)ps.tile * dn.tile_bytes;
        }
        int64_t off0 = 0;
        for (int seg = 0; seg < dn.nseg; ++seg) {
          const int sb0 = seg * dn.ks, sb1 = min(dn.nsb, sb0 + dn.ks);
          const int64_t off1 = sb1 == dn.nsb ? dn.tile_bytes : tiled_sb_offset(TD, ff, sb1);
          if (active && ok) {
            const int sid = base_dn + gj * dn.nseg * DW + seg * wg + w;
            const int st = sid % n_stages;
            const uint32_t ph = (uint32_t)((sid / n_stages) & 1);
            if (sid >= n_stages && !mbar_wait(&empty[st], ph ^ 1u, a.status, W_DEC_EMPTY)) {
              ok = false;
            } else {
              const uint32_t wbytes = (uint32_t)(off1 - off0);
              uint8_t* dst = ring + (int64_t)st * dn.stage_bytes;
              mbar_expect_tx(&full[st], wbytes + (uint32_t)((sb1 - sb0) * um.ns * RD));
              bulk_g2s(dst, up + off0, wbytes, &full[st]);
              // The SwiGLU records of chunk c exist once its ready flag is up.
              for (int c = sb0; c < sb1 && ok; ++c) {
                if (!wait_flag(flags + li * nch + c, a.status)) {
                  ok = false;
                  break;
                }
                fence_proxy_async_global();
                bulk_g2s(dst + dn.rec_off + (c - sb0) * (DMAXS * RD), a.arec + ((int64_t)c * A + um.slot0) * RD,
                         (uint32_t)(um.ns * RD), &full[st]);
              }
              if (ok) last = sid;
            }
          }
          off0 = off1;
          __syncwarp((1u << DW) - 1u);
        }
      }
    }
    // Keep the CTA alive until every copy issued in full has landed (bounded).
#pragma unroll
    for (int o = 16; o; o >>= 1) last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
    if (lane == 0)
      for (int q = max(0, last + 1 - n_stages); q <= last; ++q)
        mbar_wait(&full[q % n_stages], (uint32_t)((q / n_stages) & 1), a.status, W_DEC_DRAIN);
    return;
  }

  // Consumers.
  const int c = warp - 1;
  bool ok = true;
  const UnitArgs ua_g{a.status, (int64_t)ff}, ua_d{a.status, (int64_t)d};
  for (int gi = 0; gi * DW < n_gu; ++gi) {
    const int wg = min(DW, n_gu - gi * DW);
    const int tpr = tpr_of(wg);
    const int ul = c / tpr;
    if (ul >= wg) continue;
    const UnitPos ps = gu_pos(gi * DW + ul);
    const UnitMeta um = meta_at(list_s, off_s, ps.li);
    const int row = (c % tpr) * (DR / tpr) + lane / tpr;
    const int r = ps.tile * DR + row;
    const int r_out = r < ff ? r : -1;
    float* out = (ps.m == 0 ? a.g : a.u) + (int64_t)um.slot0 * ff;
    const int sid0 = gi * gu.nseg * DW + ul;
    if (tpr == 2) run_unit_ns<TG, 2>(um.ns, ua_g, gu, ring, full, empty, n_stages, sid0, wg, lane, row, out, r_out, ok);
    else if (tpr == 4) run_unit_ns<TG, 4>(um.ns, ua_g, gu, ring, full, empty, n_stages, sid0, wg, lane, row, out, r_out, ok);
    else run_unit_ns<TG, 8>(um.ns, ua_g, gu, ring, full, empty, n_stages, sid0, wg, lane, row, out, r_out, ok);
    // Count this warp's rows towards the expert's 256-row chunk.
    const int ch = ps.tile >> 3;
    const int idx = ps.li * nch + ch;
    __threadfence();
    __syncwarp();
    int fin = 0;
    if (lane == 0) {
      const int add = DR / tpr, expect = 2 * DR * (min(tg, 8 * ch + 8) - 8 * ch);
      fin = atomicAdd(&cnt[idx], add) + add == expect ? 1 : 0;
    }
    if (__shfl_sync(0xffffffffu, fin, 0)) {
      // Last rows of the chunk: SwiGLU records of every slot of the expert.
      __threadfence();
      for (int s = um.slot0; s < off_s[um.e + 1]; ++s) {
        const float* gp = a.g + (int64_t)s * ff + (int64_t)ch * 256;
        const float* upp = a.u + (int64_t)s * ff + (int64_t)ch * 256;
        uint8_t* rb = a.arec + ((int64_t)ch * A + s) * RD;
        if (TD != T_Q8_0) {
          float v[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = swiglu1(__ldcg(gp + lane * 8 + i), __ldcg(upp + lane * 8 + i));
          q8k_store_record(v, rb, lane);
        } else {
          const int nblk = min(8, ff / 32 - 8 * ch);
          for (int bl = 0; bl < nblk; ++bl)
            q8_store_block(swiglu1(__ldcg(gp + bl * 32 + lane), __ldcg(upp + bl * 32 + lane)), rb, bl, lane);
        }
      }
      __threadfence();
      __syncwarp();
      if (lane == 0) st_release(flags + idx, 1);
    }
  }
  // A partial last gate/up group leaves some consumer warps idle; without a
  // wait they would start the down units up to two laps of the ring ahead of
  // the slots' releases, where an mbarrier's phase parity no longer tells the
  // laps apart. All consumer warps meet here first (named barrier 2), so every
  // gate/up stage is released before any down stage is waited on.
  if (n_gu % DW != 0 && n_dn > 0) asm volatile("bar.sync 2, %0;" ::"r"(DC * 32) : "memory");
  for (int gj = 0; gj * DW < n_dn; ++gj) {
    const int wg = min(DW, n_dn - gj * DW);
    const int tpr = tpr_of(wg);
    const int ul = c / tpr;
    if (ul >= wg) continue;
    const UnitPos ps = dn_pos(gj * DW + ul);
    const UnitMeta um = meta_at(list_s, off_s, ps.li);
    const int row = (c % tpr) * (DR / tpr) + lane / tpr;
    const int r = ps.tile * DR + row;
    const int r_out = r < d ? r : -1;
    float* out = a.y + (int64_t)um.slot0 * d;
    const int sid0 = base_dn + gj * dn.nseg * DW + ul;
    if (tpr == 2) run_unit_ns<TD, 2>(um.ns, ua_d, dn, ring, full, empty, n_stages, sid0, wg, lane, row, out, r_out, ok);
    else if (tpr == 4) run_unit_ns<TD, 4>(um.ns, ua_d, dn, ring, full, empty, n_stages, sid0, wg, lane, row, out, r_out, ok);
    else run_unit_ns<TD, 8>(um.ns, ua_d, dn, ring, full, empty, n_stages, sid0, wg, lane, row, out, r_out, ok);
    __threadfence();
    __syncwarp();
    int fin = 0;
    if (lane == 0) {
      const int add = DR / tpr;
      fin = atomicAdd(&tcnt[ps.tile], add) + add == n_list * DR ? 1 : 0;
    }
    if (__shfl_sync(0xffffffffu, fin, 0)) {
      // Last rows of the output tile: combine_kernel's sum for every token,
      // the token's selections in expert-id order, from +0.0.
      __threadfence();
      const int rr = ps.tile * DR + lane;
      if (rr < d)
        for (int s = 0; s < n; ++s) {
          float o = 0.f;
          for (int jj = 0; jj < k; ++jj) {
            const int slot = csl_s[s * k + jj];
            if (slot >= 0) o = __fadd_rn(o, __fmul_rn(cwt_s[s * k + jj], __ldcg(a.y + (int64_t)slot * d + rr)));
          }
          a.out[(int64_t)s * d + rr] = o;
        }
    }
  }
}

namespace {

size_t phase1_bytes(int n, int E, int k) {
  return (size_t)n * E * 8 + (size_t)n * RT_MAXK * 8 + (size_t)n * k * 8 + (size_t)E * 4;
}

bool pair_instantiated(int tg, int td) {
  return (tg == T_Q4_K && (td == T_Q6_K || td == T_Q4_K || td == T_Q8_0)) || (tg == T_Q6_K && td == T_Q6_K) ||
         (tg == T_Q8_0 && td == T_Q8_0);
}

}  // namespace

bool moe_decode_supported(int n_tok, int E, int k, int d, int ff, int t_gate, int t_up, int t_down) {
  if (n_tok < 1 || n_tok > MK_MAXT || E < 1 || E > MK_MAX_E || k < 1 || k > MK_MAXK || k > E) return false;
  if (t_gate != t_up || !pair_instantiated(t_gate, t_down)) return false;
  if (d % 256 != 0 || d <= 0 || ff <= 0) return false;
  if (t_down == T_Q8_0 ? ff % 32 != 0 : ff % 256 != 0) return false;
  const DecodeGeom gu = decode_geom(t_gate, d), dn = decode_geom(t_down, ff);
  const int slot = std::max(gu.stage_bytes, dn.stage_bytes);
  if (MK_SMEM / slot <= DW) return false;
  if (phase1_bytes(n_tok, E, k) > (size_t)MK_SMEM) return false;
  return true;
}

template <int TG, int TD>
static int launch_t(const MkParams& p, size_t smem, cudaStream_t st) {
  static int occ = -1;
  if (occ < 0) {
    cudaFuncSetAttribute(moe_decode_kernel<TG, TD>, cudaFuncAttributeMaxDynamicSharedMemorySize, MK_SMEM);
    int blocks = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, moe_decode_kernel<TG, TD>, DTHREADS, MK_SMEM) !=
        cudaSuccess)
      blocks = 0;
    occ = blocks;
  }
  // The grid barrier needs every CTA resident at once.
  if (occ < 1) return KC_ERR_SHAPE;
  launch_k(moe_decode_kernel<TG, TD>, num_sms(), DTHREADS, smem, st, p);
  return KC_OK;
}

int launch_moe_decode(const MoeDecodeArgs& a, cudaStream_t st) {
  if (!moe_decode_supported(a.n_tok, a.E, a.k, a.d, a.ff, a.t_gate, a.t_gate, a.t_down)) return KC_ERR_SHAPE;
  if (((uintptr_t)a.h & 15) != 0 || ((uintptr_t)a.router & 15) != 0) return KC_ERR_SHAPE;
  MkParams p{};
  p.a = a;
  p.gu = decode_geom(a.t_gate, a.d);
  p.dn = decode_geom(a.t_down, a.ff);
  const int slot = std::max(p.gu.stage_bytes, p.dn.stage_bytes);
  p.gu.stage_bytes = p.dn.stage_bytes = slot;
  p.n_stages = std::min(DMAX_STAGES, MK_SMEM / slot);
  // Phase-0 K chunk: double-buffered router row + n token rows (padded by 8
  // floats) within the ring's bytes, and at most MK_MAX_TX bytes per buffer
  // (one mbarrier phase); a multiple of 256 floats, at most d.
  const int n = a.n_tok;
  int kc = (int)((size_t)MK_SMEM / (2 * (size_t)(1 + n) * 4)) - 8;
  kc = std::min(kc, MK_MAX_TX / (4 * (1 + n)));
  kc = std::max(256, kc / 256 * 256);
  p.kc = std::min(kc, a.d);
  const size_t p0 = 2 * (size_t)(1 + n) * (p.kc + 8) * 4;
  if (p0 > (size_t)MK_SMEM) return KC_ERR_SHAPE;
  const size_t smem = std::max({(size_t)p.n_stages * slot, p0, phase1_bytes(n, a.E, a.k)});
  const int tg = a.t_gate, td = a.t_down;
  if (tg == T_Q4_K && td == T_Q6_K) return launch_t<T_Q4_K, T_Q6_K>(p, smem, st);
  if (tg == T_Q4_K && td == T_Q4_K) return launch_t<T_Q4_K, T_Q4_K>(p, smem, st);
  if (tg == T_Q4_K && td == T_Q8_0) return launch_t<T_Q4_K, T_Q8_0>(p, smem, st);
  if (tg == T_Q6_K && td == T_Q6_K) return launch_t<T_Q6_K, T_Q6_K>(p, smem, st);
  if (tg == T_Q8_0 && td == T_Q8_0) return launch_t<T_Q8_0, T_Q8_0>(p, smem, st);
  return KC_ERR_TYPE;
}

}  // namespace kc
