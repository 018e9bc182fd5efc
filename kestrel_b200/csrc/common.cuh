// Shared device helpers for the sm_100a MoE FFN kernels.
//
// The library is compiled with --fmad=false: nvcc may not contract a*b+c into
// an FMA anywhere, exactly like Rust, which only fuses where Kestrel's kernels
// call _mm256_fmadd_ps. Where the reference fuses, the kernels call
// __fmaf_rn explicitly.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>
#include <utility>

#include "../../include/kestrel_cuda.h"

namespace kc {

// ggml type ids with CUDA kernels (crates/kestrel-gguf/src/types.rs:48-86).
enum : int { T_F32 = 0, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14 };

// ----------------------------------------------------------------------------
// Device weight layouts. Quantized matrices are stored "tiled": rows are
// grouped in tiles of 32 (the row count is padded to a multiple of 32 with
// zero rows), and inside a tile the bytes are superblock-major. Within one
// superblock of a tile every field is stored as planes of 16-byte row chunks,
// [chunk][32 rows][16 B], so that
//  * the 32 rows x a run of superblocks a decode stage needs are one
//    contiguous range (one bulk copy of several KB), and
//  * a warp whose thread i reads row i's chunk c touches 512 contiguous
//    bytes of shared memory (no bank conflicts).
// Per superblock-tile (32 rows), offsets in bytes:
//   Q4_K  (4608 B): hdr[32][16 B] (d, dmin, 12 scale bytes) at 0
//                   | qs chunk c = 0..7 (qs bytes 16c..16c+15) at 512 + 512c
//   Q6_K  (6720 B): ql chunk c = 0..7 at 512c | qh chunk c = 0..3 at 4096 + 512c
//                   | sc[32][16 B] at 6144 | d[32][2 B] at 6656
//   Q8_0  chunk of nblk <= 8 blocks (1024*nblk + 512 B):
//                   qs chunk c = 0..2*nblk-1 (block c/2, bytes 16*(c%2)..) at 512c
//                   | d[32][8 x 2 B] at 1024*nblk
// The bytes are a permutation of GGUF's (plus zero padding); the arithmetic
// on them is unchanged. F32 matrices stay row-major (rows padded to 16 B).
constexpr int kTileRows = 32;
constexpr int kPlane = kTileRows * 16;  // one 16-byte chunk of every row of a tile

__host__ __device__ inline int64_t round16(int64_t v) { return (v + 15) & ~int64_t(15); }
// Position of a local expert's matrices in its stacked buffer: the expert
// itself (HBM-resident table) or the HBM slot a host-streamed expert was
// copied into for this call.
__device__ __forceinline__ int expert_pos(const int* slot, int local) { return slot ? __ldg(slot + local) : local; }

// Superblocks (Q8_0: chunks of 8 blocks) per row.
__host__ __device__ inline int tiled_nsb(int t, int64_t cols) {
  return t == T_Q8_0 ? (int)((cols / 32 + 7) / 8) : (int)(cols / 256);
}
// Bytes of superblock-tile `sb` (Q8_0: chunk sb) of one tile.
__host__ __device__ inline int tiled_sbt_bytes(int t, int64_t cols, int sb) {
  if (t == T_Q4_K) return 4608;
  if (t == T_Q6_K) return 6720;
  const int nb32 = (int)(cols / 32);
  const int nblk = nb32 - 8 * sb < 8 ? nb32 - 8 * sb : 8;
  return 1024 * nblk + 512;
}
// Byte offset of superblock-tile sb inside a tile.
__host__ __device__ inline int64_t tiled_sb_offset(int t, int64_t cols, int sb) {
  if (t == T_Q4_K) return 4608ll * sb;
  if (t == T_Q6_K) return 6720ll * sb;
  return 8704ll * sb;  // all chunks before the last are full
}
__host__ __device__ inline int64_t tiled_tile_bytes(int t, int64_t cols) {
  const int nsb = tiled_nsb(t, cols);
  return tiled_sb_offset(t, cols, nsb - 1) + tiled_sbt_bytes(t, cols, nsb - 1);
}
__host__ __device__ inline int64_t padded_rows(int64_t rows) { return (rows + kTileRows - 1) / kTileRows * kTileRows; }
// Bytes of a whole [rows, cols] matrix in the device layout.
__host__ __device__ inline int64_t dev_matrix_bytes(int t, int64_t rows, int64_t cols) {
  if (t == T_F32) return rows * round16(cols * 4);
  return padded_rows(rows) / kTileRows * tiled_tile_bytes(t, cols);
}
__host__ __device__ inline int64_t gguf_row_bytes(int t, int64_t cols) {
  switch (t) {
    case T_F32: return cols * 4;
    case T_Q8_0: return cols / 32 * 34;
    case T_Q4_K: return cols / 256 * 144;
    case T_Q6_K: return cols / 256 * 210;
    default: return -1;
  }
}
inline int block_elems(int t) {
  switch (t) {
    case T_F32: return 1;
    case T_Q8_0: return 32;
    case T_Q4_K: case T_Q6_K: return 256;
    default: return 0;
  }
}

// ----------------------------------------------------------------------------
__device__ __forceinline__ float h2f(uint32_t bits16) {
  return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xFFFF)));
}

// exp of a float evaluated in double and rounded once to float. Rust's
// f32::exp calls the C library's expf, which is correctly rounded except for
// rare arguments; this agrees with it on all but ~0.06% of arguments (there by
// one ulp), where CUDA's single-precision expf differs far more often.
__device__ __forceinline__ float exp_rn(float x) { return (float)exp((double)x); }

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Kernel-side error reporting: the first failure wins; the host reads the word
// in kc_sync and maps it to a kc_status.
__device__ __forceinline__ void report(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

// Limit for every spin-wait in this library: after it expires the waiting
// thread records KC_ERR_TIMEOUT and stops waiting. Generous against time
// slicing or preemption of the GPU; every wait still ends.
constexpr uint64_t kWaitLimitNs = 4000000000ull;  // 4 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// ---- mbarrier -------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Arrive `count` times at once.
__device__ __forceinline__ void mbar_arrive_cnt(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait on a phase parity. Returns false if the phase did not complete
// within kWaitLimitNs, and records KC_ERR_TIMEOUT with the wait's site tag in
// bits 8.. of the status word (kc_last_error names the site).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int site = 0) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kWaitLimitNs) {
      report(status, KC_ERR_TIMEOUT | (site << 8));
      return false;
    }
  }
  return true;
}
// Release counters of a stage ring (shared memory): each consumer warp adds
// its share of the DARR releases of a stage; lap L of a slot may be consumed
// once the slot's counter reaches L * DARR. A monotonic count cannot alias an
// older lap the way a phase parity can when consumers run at very different
// speeds (the previous lap of a slot may not even be issued yet when a fast
// consumer arrives: producer lanes issue a segment's stages independently).
__device__ __forceinline__ void count_add(int* c, int v) {
  asm volatile("red.shared.add.s32 [%0], %1;" ::"r"(smem_u32(c)), "r"(v) : "memory");
}
__device__ __forceinline__ int count_read(const int* c) {
  int v;
  asm volatile("ld.volatile.shared.s32 %0, [%1];" : "=r"(v) : "r"(smem_u32(c)) : "memory");
  return v;
}
// Bounded wait until *c >= target; records KC_ERR_TIMEOUT with the site tag
// and returns false after kWaitLimitNs.
__device__ __forceinline__ bool count_wait(const int* c, int target, int* status, int site) {
  if (count_read(c) >= target) return true;
  const uint64_t t0 = globaltimer();
  while (count_read(c) < target) {
    if (globaltimer() - t0 > kWaitLimitNs) {
      report(status, KC_ERR_TIMEOUT | (site << 8));
      return false;
    }
  }
  return true;
}

// Site tags of the bounded waits.
enum : int {
  W_DEC_EMPTY = 1, W_DEC_FULL = 2, W_DEC_DRAIN = 3, W_MMA_RAW_EMPTY = 4, W_MMA_OP_EMPTY_P = 5, W_MMA_DRAIN = 6,
  W_MMA_OP_FULL = 7, W_MMA_ACC_EMPTY = 8, W_MMA_RAW_FULL = 9, W_MMA_OP_EMPTY_D = 10, W_MMA_ACC_FULL = 11,
  W_ROUTER = 12, W_MMA_TC_DRAIN = 13, W_DEC_PREV = 14, W_EP_PEER = 15, W_EP_PATH = 16, W_MMA_BOUND = 17
};

// ---- bulk async copy (TMA, non-tensor): global -> shared ------------------
// Both addresses 16-byte aligned, size a multiple of 16 (checked by callers).
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// L2 eviction-priority policies (createpolicy) for the cache hints below:
// weights streamed once are read evict_first.
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// bulk_g2s with an L2 cache-policy hint.
__device__ __forceinline__ void bulk_g2s_hint(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
          "r"(smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// ---- Kestrel arithmetic helpers -------------------------------------------
// scale_min_k4 (crates/kestrel-engine/src/quant.rs:54-60) for all eight
// sub-blocks of a Q4_K superblock, from the 12 packed scale bytes held in
// three little-endian words.
__device__ __forceinline__ void q4k_scales(uint32_t w0, uint32_t w1, uint32_t w2, int sc[8], int mn[8]) {
  // bytes q[0..3] = w0, q[4..7] = w1, q[8..11] = w2
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t qj = (w0 >> (8 * j)) & 0xFF, qj4 = (w1 >> (8 * j)) & 0xFF, qj8 = (w2 >> (8 * j)) & 0xFF;
    sc[j] = qj & 63;
    mn[j] = qj4 & 63;
    sc[j + 4] = (qj8 & 0xF) | ((qj >> 6) << 4);
    mn[j + 4] = (qj8 >> 4) | ((qj4 >> 6) << 4);
  }
}

// hsum (avx2.rs:19-27) over the eight lanes held by eight consecutive threads
// (lane j = thread j of the group): ((v0+v4)+(v2+v6)) + ((v1+v5)+(v3+v7)).
// Valid in the group's first thread.
__device__ __forceinline__ float hsum8_group(float v) {
  v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 4, 8));
  v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 2, 8));
  v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 1, 8));
  return v;
}

// Rust `x.round() as i32` then `.clamp(-127, 127)`: round half away from
// zero, NaN -> 0, saturating.
__device__ __forceinline__ int q8_round(float v) {
  float r = roundf(v);
  if (r != r) return 0;
  r = fminf(fmaxf(r, -127.f), 127.f);
  return (int)r;
}

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// One Q8_K activation record (Q8KRow::quantize, qdot.rs:347-367) of the 256
// values a warp holds, 8 per lane (lane l: elements 8l .. 8l+7), stored at rb:
// q[256] int8 | bsums int16[16] at 256 | pair sums int16[8] at 288 | d f32 at
// 304 (then 12 zero bytes).
__device__ __forceinline__ void q8k_store_record(const float (&v)[8], uint8_t* rb, int lane) {
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
  const int s16 = s + __shfl_xor_sync(0xffffffffu, s, 1);     // bsums[lane / 2]
  const int s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 2);  // bsums pair lane / 4
  *reinterpret_cast<uint2*>(rb + lane * 8) = make_uint2(packed[0], packed[1]);
  if ((lane & 1) == 0) reinterpret_cast<int16_t*>(rb + 256)[lane / 2] = (int16_t)s16;
  if ((lane & 3) == 0) reinterpret_cast<int16_t*>(rb + 288)[lane / 4] = (int16_t)s32;
  if (lane == 0) reinterpret_cast<float*>(rb + 304)[0] = scale;
  if (lane >= 1 && lane < 4) reinterpret_cast<uint32_t*>(rb + 304)[lane] = 0u;
}

inline int ceil_div(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

// ---- programmatic dependent launch -----------------------------------------
// The layer's kernels are launched so that the next one may start (launch,
// prologue) while the previous one drains. Each of them calls pdl_wait()
// before its first access to global memory written by earlier work -- which
// returns once the previous kernel in the stream has completed and its
// writes are visible -- and then pdl_trigger() to let the next one launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_enter() {
  pdl_wait();
  pdl_trigger();
}
// KESTREL_PDL=0 launches them as ordinary stream-ordered kernels.
bool pdl_enabled();
// Every launch_k adds one (kc_kernel_launches reads it).
extern std::atomic<int64_t> g_kernel_launches;

// Kernel attributes such as cudaFuncAttributeMaxDynamicSharedMemorySize are
// per device: a process that drives several GPUs (one context each) must set
// them on every device it launches on. One PerDeviceOnce per call site runs
// its setter once per device, the first time a host thread launches there
// with that device current; concurrent first calls are serialised.
struct PerDeviceOnce {
  static constexpr int kMaxDev = 64;
  std::atomic<uint64_t> done{0};
  std::mutex mu;
  template <typename Fn>
  cudaError_t run(Fn&& setter) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDev) return cudaErrorInvalidDevice;
    const uint64_t bit = 1ull << dev;
    if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
    std::lock_guard<std::mutex> lock(mu);
    if (done.load(std::memory_order_relaxed) & bit) return cudaSuccess;
    e = setter();
    if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_release);
    return e;
  }
};
// Raises kernel's dynamic shared-memory limit to `bytes` on the current
// device, once per device (per call site through `once`).
template <typename... KArgs>
inline cudaError_t smem_attr_once(PerDeviceOnce& once, void (*kernel)(KArgs...), int bytes) {
  return once.run([&] { return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes); });
}
template <typename... KArgs, typename... Args>
inline void launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                     Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
}

}  // namespace kc
