// Activation quantization (Q8_K / Q8 rows), this library's weight quantizer,
// GGUF -> device-layout repacking, and the integer block-sum diagnostic.
#include "common.cuh"
#include "kernels.h"

namespace kc {

// ---------------------------------------------------------------------------
// Q8KRow::quantize (crates/kestrel-engine/src/qdot.rs:347-367), bit-exact:
// d = amax/127 (IEEE division), inv = 1/d (0 if d == 0), q = clamp(round(x*inv)).
// One warp per 256-block; lane l owns elements 8l..8l+7, so the pair of lanes
// (2m, 2m+1) owns the 16 values of bsums[m].
__global__ void q8k_quantize_kernel(const float* __restrict__ x, const int* __restrict__ row_map, int64_t n_rows,
                                    int64_t cols, int8_t* __restrict__ q, float* __restrict__ d,
                                    int32_t* __restrict__ bsums) {
  int64_t nb = cols / 256;
  int64_t gw = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  int lane = threadIdx.x & 31;
  if (gw >= n_rows * nb) return;
  int64_t r = gw / nb, b = gw % nb;
  int64_t src_row = row_map ? row_map[r] : r;
  if (src_row < 0) return;
  const float4* xp = reinterpret_cast<const float4*>(x + src_row * cols + b * 256 + lane * 8);
  float4 a0 = xp[0], a1 = xp[1];
  float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  float scale = __fdiv_rn(amax, 127.0f);
  float inv = scale > 0.f ? __fdiv_rn(1.0f, scale) : 0.f;
  int s = 0;
  uint32_t packed[2] = {0, 0};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int qi = q8_round(__fmul_rn(v[i], inv));
    s += qi;
    packed[i / 4] |= (uint32_t)(qi & 0xFF) << (8 * (i % 4));
  }
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  *reinterpret_cast<uint2*>(q + r * cols + b * 256 + lane * 8) = make_uint2(packed[0], packed[1]);
  if ((lane & 1) == 0) bsums[r * (cols / 16) + b * 16 + lane / 2] = s;
  if (lane == 0) d[r * nb + b] = scale;
}

// Q8Row::quantize (qdot.rs:29-49): blocks of 32, s16 = sums of each half.
// One warp handles one 32-block; lane = element.
__global__ void q8_quantize_kernel(const float* __restrict__ x, const int* __restrict__ row_map, int64_t n_rows,
                                   int64_t cols, int8_t* __restrict__ q, float* __restrict__ d,
                                   int32_t* __restrict__ s16) {
  int64_t nb = cols / 32;
  int64_t gw = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  int lane = threadIdx.x & 31;
  if (gw >= n_rows * nb) return;
  int64_t r = gw / nb, b = gw % nb;
  int64_t src_row = row_map ? row_map[r] : r;
  if (src_row < 0) return;
  float v = x[src_row * cols + b * 32 + lane];
  float amax = fabsf(v);
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  float scale = __fdiv_rn(amax, 127.0f);
  float inv = scale > 0.f ? __fdiv_rn(1.0f, scale) : 0.f;
  int qi = q8_round(__fmul_rn(v, inv));
  q[r * cols + b * 32 + lane] = (int8_t)qi;
  int s = qi;
#pragma unroll
  for (int o = 8; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) s16[r * (cols / 16) + 2 * b] = s;
  if (lane == 16) s16[r * (cols / 16) + 2 * b + 1] = s;
  if (lane == 0) d[r * nb + b] = scale;
}

void launch_q8k_quantize(const float* x, const int* row_map, int64_t n_rows, int64_t cols, int8_t* q, float* d,
                         int32_t* bsums, cudaStream_t st) {
  int64_t warps = n_rows * (cols / 256);
  if (warps <= 0) return;
  q8k_quantize_kernel<<<ceil_div(warps, 8), 256, 0, st>>>(x, row_map, n_rows, cols, q, d, bsums);
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
}

void launch_q8_quantize(const float* x, const int* row_map, int64_t n_rows, int64_t cols, int8_t* q, float* d,
                        int32_t* s16, cudaStream_t st) {
  int64_t warps = n_rows * (cols / 32);
  if (warps <= 0) return;
  q8_quantize_kernel<<<ceil_div(warps, 8), 256, 0, st>>>(x, row_map, n_rows, cols, q, d, s16);
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
}

// ---------------------------------------------------------------------------
// Weight quantizer: the rules of kestrel_b200/ggml.py, in the same float32
// operation order (IEEE mul/div/add, round-half-even, f16 round-to-nearest),
// so both produce identical bytes. One thread per block. Used to build the
// benchmark's weights on the GPU; not on the inference path.
__device__ __forceinline__ float f16r(float v) { return __half2float(__float2half_rn(v)); }
__device__ __forceinline__ uint16_t f16bits(float v) { return __half_as_ushort(__float2half_rn(v)); }
__device__ __forceinline__ float safe_div(float a, float b) { return b > 0.f ? __fdiv_rn(a, b) : 0.f; }
__device__ __forceinline__ float clampf(float v, float lo, float hi) { return fminf(fmaxf(v, lo), hi); }

__global__ void quantize_q4_k_kernel(const float* __restrict__ x, int64_t nblocks, uint8_t* __restrict__ out) {
  int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  const float* xb = x + b * 256;
  float scale[8], mins[8];
  float smax = 0.f, mmax = 0.f;
  for (int j = 0; j < 8; ++j) {
    float lo = xb[j * 32], hi = xb[j * 32];
    for (int l = 1; l < 32; ++l) {
      lo = fminf(lo, xb[j * 32 + l]);
      hi = fmaxf(hi, xb[j * 32 + l]);
    }
    lo = fminf(lo, 0.f);
    scale[j] = __fadd_rn(__fdiv_rn(__fsub_rn(hi, lo), 15.f), 0.f);  // +0.0 for constant blocks
    mins[j] = __fsub_rn(0.f, lo);  // +0.0 (not -0.0) for non-negative blocks
    smax = fmaxf(smax, scale[j]);
    mmax = fmaxf(mmax, mins[j]);
  }
  float d16 = f16r(__fdiv_rn(smax, 63.f)), dm16 = f16r(__fdiv_rn(mmax, 63.f));
  int sc[8], mm[8];
  for (int j = 0; j < 8; ++j) {
    sc[j] = (int)clampf(rintf(safe_div(scale[j], d16)), 0.f, 63.f);
    mm[j] = (int)clampf(rintf(safe_div(mins[j], dm16)), 0.f, 63.f);
  }
  // Assemble the 144-byte block as 36 words and store it as nine 16-byte
  // vectors (blocks are 16-byte aligned).
  uint32_t wv[36];
  wv[0] = (uint32_t)f16bits(d16) | ((uint32_t)f16bits(dm16) << 16);
  uint32_t sb[12];
  for (int j = 0; j < 4; ++j) {
    sb[j] = (uint32_t)(sc[j] | ((sc[j + 4] >> 4) << 6)) & 0xFF;
    sb[4 + j] = (uint32_t)(mm[j] | ((mm[j + 4] >> 4) << 6)) & 0xFF;
    sb[8 + j] = (uint32_t)((sc[j + 4] & 0xF) | ((mm[j + 4] & 0xF) << 4)) & 0xFF;
  }
  for (int w = 0; w < 3; ++w)
    wv[1 + w] = sb[4 * w] | (sb[4 * w + 1] << 8) | (sb[4 * w + 2] << 16) | (sb[4 * w + 3] << 24);
  for (int k = 0; k < 4; ++k) {
    float D0 = __fmul_rn(d16, (float)sc[2 * k]), M0 = __fmul_rn(dm16, (float)mm[2 * k]);
    float D1 = __fmul_rn(d16, (float)sc[2 * k + 1]), M1 = __fmul_rn(dm16, (float)mm[2 * k + 1]);
    for (int w = 0; w < 8; ++w) {
      uint32_t word = 0;
      for (int bb = 0; bb < 4; ++bb) {
        int l = 4 * w + bb;
        int q0 = (int)clampf(rintf(safe_div(__fadd_rn(xb[64 * k + l], M0), D0)), 0.f, 15.f);
        int q1 = (int)clampf(rintf(safe_div(__fadd_rn(xb[64 * k + 32 + l], M1), D1)), 0.f, 15.f);
        word |= (uint32_t)(q0 | (q1 << 4)) << (8 * bb);
      }
      wv[4 + 8 * k + w] = word;
    }
  }
  uint4* o4 = reinterpret_cast<uint4*>(out + b * 144);
  for (int i = 0; i < 9; ++i) o4[i] = make_uint4(wv[4 * i], wv[4 * i + 1], wv[4 * i + 2], wv[4 * i + 3]);
}

__global__ void quantize_q6_k_kernel(const float* __restrict__ x, int64_t nblocks, uint8_t* __restrict__ out) {
  int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  const float* xb = x + b * 256;
  float s[16], smax = 0.f;
  for (int j = 0; j < 16; ++j) {
    float a = 0.f;
    for (int l = 0; l < 16; ++l) a = fmaxf(a, fabsf(xb[16 * j + l]));
    s[j] = __fdiv_rn(a, 31.f);
    smax = fmaxf(smax, s[j]);
  }
  float d16 = f16r(__fdiv_rn(smax, 127.f));
  int sc[16];
  for (int j = 0; j < 16; ++j) sc[j] = (int)clampf(rintf(safe_div(s[j], d16)), -128.f, 127.f);
  uint8_t o[210];
  for (int i = 0; i < 192; ++i) o[i] = 0;
  for (int i = 0; i < 256; ++i) {
    int j = i / 16;
    float D = __fmul_rn(d16, (float)sc[j]);
    int q = (int)clampf(rintf(safe_div(xb[i], D)), -32.f, 31.f) + 32;
    int h = i / 128, r = (i % 128) / 32, l = i % 32;
    int qlidx = h * 64 + l + ((r & 1) ? 32 : 0);
    o[qlidx] |= (uint8_t)((q & 0xF) << ((r >> 1) * 4));
    o[128 + h * 32 + l] |= (uint8_t)((q >> 4) << (2 * r));
  }
  for (int j = 0; j < 16; ++j) o[192 + j] = (uint8_t)(int8_t)sc[j];
  uint16_t hd = f16bits(d16);
  o[208] = hd & 0xFF;
  o[209] = hd >> 8;
  uint16_t* o16 = reinterpret_cast<uint16_t*>(out + b * 210);
  for (int i = 0; i < 105; ++i) o16[i] = (uint16_t)(o[2 * i] | (o[2 * i + 1] << 8));
}

__global__ void quantize_q8_0_kernel(const float* __restrict__ x, int64_t nblocks, uint8_t* __restrict__ out) {
  int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  const float* xb = x + b * 32;
  float amax = 0.f;
  for (int l = 0; l < 32; ++l) amax = fmaxf(amax, fabsf(xb[l]));
  float d16 = f16r(__fdiv_rn(amax, 127.f));
  float inv = safe_div(1.f, d16);
  uint16_t* o16 = reinterpret_cast<uint16_t*>(out + b * 34);
  o16[0] = f16bits(d16);
  for (int l = 0; l < 32; l += 2) {
    uint32_t q0 = (uint8_t)(int8_t)(int)clampf(rintf(__fmul_rn(xb[l], inv)), -127.f, 127.f);
    uint32_t q1 = (uint8_t)(int8_t)(int)clampf(rintf(__fmul_rn(xb[l + 1], inv)), -127.f, 127.f);
    o16[1 + l / 2] = (uint16_t)(q0 | (q1 << 8));
  }
}

int launch_quantize(int t, const float* x, int64_t rows, int64_t cols, void* out, cudaStream_t st) {
  int64_t be = block_elems(t);
  if (be <= 1 || cols % be) return KC_ERR_SHAPE;
  int64_t nblocks = rows * cols / be;
  if (nblocks == 0) return KC_OK;
  int grid = ceil_div(nblocks, 128);
  uint8_t* o = static_cast<uint8_t*>(out);
  if (t == T_Q4_K) quantize_q4_k_kernel<<<grid, 128, 0, st>>>(x, nblocks, o);
  else if (t == T_Q6_K) quantize_q6_k_kernel<<<grid, 128, 0, st>>>(x, nblocks, o);
  else if (t == T_Q8_0) quantize_q8_0_kernel<<<grid, 128, 0, st>>>(x, nblocks, o);
  else return KC_ERR_TYPE;
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
  return KC_OK;
}

// ---------------------------------------------------------------------------
// GGUF rows -> tiled device layout (see common.cuh). `n_mats` stacked matrices
// of `rows` rows each; matrix m starts at m * dev_matrix_bytes in dst. One
// thread per (row, superblock); destination padding was zeroed by the caller.
__global__ void repack_tiled_kernel(int t, const uint8_t* __restrict__ src, int64_t n_mats, int64_t rows,
                                    int64_t cols, uint8_t* __restrict__ dst) {
  const int nsb = tiled_nsb(t, cols);
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_mats * rows * nsb) return;
  const int sb = (int)(i % nsb);
  const int64_t gr = i / nsb;  // global row over all matrices
  const int64_t m = gr / rows, r = gr % rows;
  const int64_t tile = r / kTileRows;
  const int rr = (int)(r % kTileRows);
  const uint8_t* srow = src + gr * gguf_row_bytes(t, cols);
  uint8_t* sbt = dst + m * dev_matrix_bytes(t, rows, cols) + tile * tiled_tile_bytes(t, cols) +
                 tiled_sb_offset(t, cols, sb);
  if (t == T_Q4_K) {
    const uint8_t* b = srow + 144 * sb;
    for (int x = 0; x < 16; ++x) sbt[16 * rr + x] = b[x];
    for (int c = 0; c < 8; ++c)
      for (int x = 0; x < 16; ++x) sbt[kPlane + kPlane * c + 16 * rr + x] = b[16 + 16 * c + x];
  } else if (t == T_Q6_K) {
    const uint8_t* b = srow + 210 * sb;
    for (int c = 0; c < 8; ++c)
      for (int x = 0; x < 16; ++x) sbt[kPlane * c + 16 * rr + x] = b[16 * c + x];
    for (int c = 0; c < 4; ++c)
      for (int x = 0; x < 16; ++x) sbt[8 * kPlane + kPlane * c + 16 * rr + x] = b[128 + 16 * c + x];
    for (int x = 0; x < 16; ++x) sbt[12 * kPlane + 16 * rr + x] = b[192 + x];
    sbt[13 * kPlane + 2 * rr] = b[208];
    sbt[13 * kPlane + 2 * rr + 1] = b[209];
  } else {
    const int nb32 = (int)(cols / 32);
    const int nblk = min(8, nb32 - 8 * sb);
    for (int bl = 0; bl < nblk; ++bl) {
      const uint8_t* b = srow + 34 * (8 * sb + bl);
      for (int x = 0; x < 32; ++x) sbt[kPlane * (2 * bl + (x >> 4)) + 16 * rr + (x & 15)] = b[2 + x];
      sbt[2 * kPlane * nblk + 16 * rr + 2 * bl] = b[0];
      sbt[2 * kPlane * nblk + 16 * rr + 2 * bl + 1] = b[1];
    }
  }
}

__global__ void repack_copy_rows_kernel(const uint8_t* __restrict__ src, int64_t rows, int64_t row_bytes,
                                        int64_t dst_stride, uint8_t* __restrict__ dst) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * dst_stride) return;
  int64_t r = i / dst_stride, c = i % dst_stride;
  dst[i] = c < row_bytes ? src[r * row_bytes + c] : 0;
}

// `src` holds n_mats stacked GGUF matrices [rows, cols]; dst receives them in
// the device layout (dst must hold n_mats * dev_matrix_bytes).
int launch_repack(int t, const void* src, int64_t n_mats, int64_t rows, int64_t cols, void* dst, cudaStream_t st) {
  const uint8_t* s = static_cast<const uint8_t*>(src);
  uint8_t* d = static_cast<uint8_t*>(dst);
  if (rows == 0 || n_mats == 0) return KC_OK;
  if (t == T_F32) {
    const int64_t rb = cols * 4, ds = round16(rb);
    repack_copy_rows_kernel<<<ceil_div(n_mats * rows * ds, 256), 256, 0, st>>>(s, n_mats * rows, rb, ds, d);
    g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
    return KC_OK;
  }
  if (t != T_Q4_K && t != T_Q6_K && t != T_Q8_0) return KC_ERR_TYPE;
  if (cudaMemsetAsync(d, 0, n_mats * dev_matrix_bytes(t, rows, cols), st) != cudaSuccess) return KC_ERR_CUDA;
  const int64_t n = n_mats * rows * tiled_nsb(t, cols);
  repack_tiled_kernel<<<ceil_div(n, 128), 128, 0, st>>>(t, s, n_mats, rows, cols, d);
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
  return KC_OK;
}

// ---------------------------------------------------------------------------
// Diagnostic: per-superblock integer sums (the eight AVX2 lanes of sumi plus
// the min/offset term) of GGUF K-quant rows against Q8_K activation rows.
// One thread per (act row, weight row, superblock); plain loops.
__global__ void block_sums_kernel(int t, const uint8_t* __restrict__ w, int64_t rows, int64_t cols,
                                  const int8_t* __restrict__ q, const int32_t* __restrict__ bsums, int n_act,
                                  int32_t* __restrict__ out) {
  int64_t nb = cols / 256;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)n_act * rows * nb) return;
  int64_t a = i / (rows * nb), r = (i / nb) % rows, b = i % nb;
  const int8_t* xq = q + a * cols + b * 256;
  const int32_t* bs = bsums + a * (cols / 16) + b * 16;
  int32_t* o = out + i * 9;
  if (t == T_Q4_K) {
    const uint8_t* blk = w + r * nb * 144 + b * 144;
    uint32_t w0 = blk[4] | blk[5] << 8 | blk[6] << 16 | (uint32_t)blk[7] << 24;
    uint32_t w1 = blk[8] | blk[9] << 8 | blk[10] << 16 | (uint32_t)blk[11] << 24;
    uint32_t w2 = blk[12] | blk[13] << 8 | blk[14] << 16 | (uint32_t)blk[15] << 24;
    int sc[8], mn[8];
    q4k_scales(w0, w1, w2, sc, mn);
    int mins = 0;
    for (int j = 0; j < 8; ++j) o[j] = 0;
    for (int k = 0; k < 4; ++k) {
      for (int j = 0; j < 8; ++j) {
        int plo = 0, phi = 0;
        for (int e = 4 * j; e < 4 * j + 4; ++e) {
          plo += (blk[16 + 32 * k + e] & 0xF) * xq[64 * k + e];
          phi += (blk[16 + 32 * k + e] >> 4) * xq[64 * k + 32 + e];
        }
        o[j] += sc[2 * k] * plo + sc[2 * k + 1] * phi;
      }
      mins += mn[2 * k] * (bs[4 * k] + bs[4 * k + 1]) + mn[2 * k + 1] * (bs[4 * k + 2] + bs[4 * k + 3]);
    }
    o[8] = mins;
  } else {
    const uint8_t* blk = w + r * nb * 210 + b * 210;
    int offs = 0;
    for (int j = 0; j < 8; ++j) o[j] = 0;
    for (int h = 0; h < 2; ++h) {
      const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192 + h * 8);
      for (int ri = 0; ri < 4; ++ri) {
        for (int j = 0; j < 8; ++j) {
          int p = 0;
          for (int e = 4 * j; e < 4 * j + 4; ++e) {
            int src = (ri & 1) ? blk[h * 64 + 32 + e] : blk[h * 64 + e];
            int nib = ri < 2 ? (src & 0xF) : (src >> 4);
            int v = nib | (((blk[128 + h * 32 + e] >> (2 * ri)) & 3) << 4);
            p += v * xq[h * 128 + ri * 32 + e];
          }
          o[j] += (j < 4 ? sc[2 * ri] : sc[2 * ri + 1]) * p;
        }
        int k16 = h * 8 + ri * 2;
        offs += sc[2 * ri] * bs[k16] + sc[2 * ri + 1] * bs[k16 + 1];
      }
    }
    o[8] = offs;
  }
}

void launch_block_sums(int t, const void* w, int64_t rows, int64_t cols, const int8_t* q, const int32_t* bsums,
                       int n_act, int32_t* out, cudaStream_t st) {
  int64_t n = (int64_t)n_act * rows * (cols / 256);
  if (n == 0) return;
  block_sums_kernel<<<ceil_div(n, 128), 128, 0, st>>>(t, static_cast<const uint8_t*>(w), rows, cols, q, bsums,
                                                      n_act, out);
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
}

}  // namespace kc
