// NCCL communicator set-up for expert parallelism.
#include <nccl.h>

#include <cstring>

#include "common.cuh"
#include "ep.h"

namespace kc {

int ep_unique_id(char out[128]) {
  if (!out) return KC_ERR_ARG;
  ncclUniqueId id;
  if (ncclGetUniqueId(&id) != ncclSuccess) return KC_ERR_NCCL;
  static_assert(sizeof(id.internal) == 128, "NCCL unique id size");
  std::memcpy(out, id.internal, 128);
  return KC_OK;
}

int ep_init(EpState& s, int rank, int world, const char uid[128]) {
  if (world < 1 || rank < 0 || rank >= world || !uid) {
    s.err = "bad rank/world/uid";
    return KC_ERR_ARG;
  }
  ep_free(s);
  if (world == 1) {
    s.world = 1;
    s.rank = 0;
    return KC_OK;
  }
  ncclUniqueId id;
  std::memcpy(id.internal, uid, 128);
  ncclComm_t comm;
  ncclResult_t r = ncclCommInitRank(&comm, world, id, rank);
  if (r != ncclSuccess) {
    s.err = std::string("ncclCommInitRank: ") + ncclGetErrorString(r);
    return KC_ERR_NCCL;
  }
  s.comm = comm;
  s.world = world;
  s.rank = rank;
  return KC_OK;
}

void ep_free(EpState& s) {
  if (s.comm) ncclCommDestroy(static_cast<ncclComm_t>(s.comm));
  s.comm = nullptr;
  s.world = 1;
  s.rank = 0;
}

const char* ep_last_error(const EpState& s) { return s.err.c_str(); }

}  // namespace kc

// ===========================================================================
// Exchange plans and packing kernels.
namespace kc {

constexpr int EP_THREADS = 1024;

// Exclusive block scan of N ints per thread (EP_THREADS threads). Returns the
// block totals in tot. `sh` holds 32 * N ints.
template <int N>
__device__ __forceinline__ void block_scan(const int (&v)[N], int (&ex)[N], int (&tot)[N], int* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int inc[N];
#pragma unroll
  for (int i = 0; i < N; ++i) inc[i] = v[i];
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
    for (int i = 0; i < N; ++i) {
      const int x = __shfl_up_sync(0xffffffffu, inc[i], o);
      if (lane >= o) inc[i] += x;
    }
  }
  if (lane == 31)
#pragma unroll
    for (int i = 0; i < N; ++i) sh[warp * N + i] = inc[i];
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int i = 0; i < N; ++i) {
      int u = sh[lane * N + i];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int x = __shfl_up_sync(0xffffffffu, u, o);
        if (lane >= o) u += x;
      }
      sh[lane * N + i] = u;  // inclusive over warps
    }
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < N; ++i) {
    ex[i] = (warp > 0 ? sh[(warp - 1) * N + i] : 0) + inc[i] - v[i];
    tot[i] = sh[31 * N + i];
  }
  __syncthreads();
}

__global__ void __launch_bounds__(EP_THREADS) ep_plan_kernel(const int* __restrict__ ids, int n_tok, int k, int G,
                                                              int epr, int T, int* __restrict__ send_tok,
                                                              int* __restrict__ ret_pos, int* __restrict__ xch_out) {
  pdl_enter();
  __shared__ int sh[32 * 2 * kEpMaxWorld];
  __shared__ int base_f[kEpMaxWorld], base_c[kEpMaxWorld], off_c[kEpMaxWorld];
  const int tid = threadIdx.x;
  if (tid < kEpMaxWorld) {
    base_f[tid] = 0;
    base_c[tid] = 0;
  }
  // Pass 1: rows sent to / result rows expected from every rank.
  int tf[kEpMaxWorld] = {}, tc[kEpMaxWorld] = {};
  for (int r0 = 0; r0 < n_tok; r0 += EP_THREADS) {
    const int s = r0 + tid;
    int v[2 * kEpMaxWorld] = {}, ex[2 * kEpMaxWorld], tot[2 * kEpMaxWorld];
    if (s < n_tok)
      for (int j = 0; j < k; ++j) {
        const int e = ids[(int64_t)s * k + j];
        const int r = e >= 0 ? e / epr : -1;
#pragma unroll
        for (int q = 0; q < kEpMaxWorld; ++q) v[kEpMaxWorld + q] += (r == q) ? 1 : 0;
      }
#pragma unroll
    for (int q = 0; q < kEpMaxWorld; ++q) v[q] = v[kEpMaxWorld + q] > 0 ? 1 : 0;
    block_scan<2 * kEpMaxWorld>(v, ex, tot, sh);
#pragma unroll
    for (int q = 0; q < kEpMaxWorld; ++q) {
      tf[q] += tot[q];
      tc[q] += tot[kEpMaxWorld + q];
    }
  }
  if (tid == 0) {
    int run = 0;
    for (int q = 0; q < G; ++q) {
      off_c[q] = run;
      run += tc[q];
      xch_out[2 * q] = tf[q];
      xch_out[2 * q + 1] = tc[q];
    }
  }
  __syncthreads();
  // Pass 2: positions.
  for (int r0 = 0; r0 < n_tok; r0 += EP_THREADS) {
    const int s = r0 + tid;
    int v[2 * kEpMaxWorld] = {}, ex[2 * kEpMaxWorld], tot[2 * kEpMaxWorld];
    if (s < n_tok)
      for (int j = 0; j < k; ++j) {
        const int e = ids[(int64_t)s * k + j];
        const int r = e >= 0 ? e / epr : -1;
#pragma unroll
        for (int q = 0; q < kEpMaxWorld; ++q) v[kEpMaxWorld + q] += (r == q) ? 1 : 0;
      }
#pragma unroll
    for (int q = 0; q < kEpMaxWorld; ++q) v[q] = v[kEpMaxWorld + q] > 0 ? 1 : 0;
    block_scan<2 * kEpMaxWorld>(v, ex, tot, sh);
    if (s < n_tok) {
#pragma unroll
      for (int q = 0; q < kEpMaxWorld; ++q)
        if (q < G && v[q]) send_tok[(int64_t)q * T + base_f[q] + ex[q]] = s;
      for (int j = 0; j < k; ++j) {
        const int e = ids[(int64_t)s * k + j];
        if (e < 0 || e / epr >= G) {
          ret_pos[(int64_t)s * k + j] = 0;
          continue;
        }
        const int r = e / epr;
        int rank = 0;
        for (int j2 = 0; j2 < k; ++j2) {
          const int e2 = ids[(int64_t)s * k + j2];
          rank += (e2 >= 0 && e2 / epr == r && e2 < e) ? 1 : 0;
        }
        int exc = 0;
#pragma unroll
        for (int q = 0; q < kEpMaxWorld; ++q)
          if (q == r) exc = base_c[q] + ex[kEpMaxWorld + q];
        ret_pos[(int64_t)s * k + j] = off_c[r] + exc + rank;
      }
    }
    __syncthreads();
    if (tid == 0)
#pragma unroll
      for (int q = 0; q < kEpMaxWorld; ++q) {
        base_f[q] += tot[q];
        base_c[q] += tot[kEpMaxWorld + q];
      }
    __syncthreads();
  }
}

void launch_ep_plan(const int* ids, int n_tok, int k, int world, int epr, int T, int* send_tok, int* ret_pos,
                    int* xch_out, cudaStream_t st) {
  launch_k(ep_plan_kernel, 1, EP_THREADS, 0, st, ids, n_tok, k, world, epr, T, send_tok, ret_pos, xch_out);
}

// One warp per (destination, row): rows r's section starts at the prefix of
// the rows sent to ranks before r.
__global__ void ep_pack_kernel(const float* __restrict__ h, const int* __restrict__ ids, const float* __restrict__ w,
                               const int* __restrict__ send_tok, const int* __restrict__ xch_out, int G, int T,
                               int k, int d, float* __restrict__ sendbuf, int32_t* __restrict__ sendmeta) {
  pdl_enter();
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  const int r = (int)(gw / T), i = (int)(gw % T);
  if (r >= G || i >= xch_out[2 * r]) return;
  int off = 0;
  for (int q = 0; q < r; ++q) off += xch_out[2 * q];
  const int s = send_tok[(int64_t)r * T + i];
  const int64_t row = off + i;
  const float4* src = reinterpret_cast<const float4*>(h + (int64_t)s * d);
  float4* dst = reinterpret_cast<float4*>(sendbuf + row * d);
  for (int c = lane; c < d / 4; c += 32) dst[c] = src[c];
  for (int c = lane; c < k; c += 32) {
    sendmeta[row * 2 * k + c] = ids[(int64_t)s * k + c];
    sendmeta[row * 2 * k + k + c] = __float_as_int(w[(int64_t)s * k + c]);
  }
}

void launch_ep_pack(const float* h, const int* ids, const float* w, const int* send_tok, const int* xch_out,
                    int world, int T, int k, int d, float* sendbuf, int32_t* sendmeta, cudaStream_t st) {
  const int64_t warps = (int64_t)world * T;
  if (warps <= 0) return;
  launch_k(ep_pack_kernel, ceil_div(warps * 32, 256), 256, 0, st, h, ids, w, send_tok, xch_out, world, T, k, d,
           sendbuf, sendmeta);
}

__global__ void ep_local_ids_kernel(const int32_t* __restrict__ meta, int n_recv, int k, int first, int n_local,
                                    int* __restrict__ ids_loc, float* __restrict__ w_loc) {
  pdl_enter();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)n_recv * k) return;
  const int64_t row = i / k, j = i % k;
  const int e = meta[row * 2 * k + j];
  ids_loc[i] = (e >= first && e < first + n_local) ? e - first : -1;
  w_loc[i] = __int_as_float(meta[row * 2 * k + k + j]);
}

void launch_ep_local_ids(const int32_t* recvmeta, int n_recv, int k, int first, int n_local, int* ids_loc,
                         float* w_loc, cudaStream_t st) {
  const int64_t n = (int64_t)n_recv * k;
  if (n <= 0) return;
  launch_k(ep_local_ids_kernel, ceil_div(n, 256), 256, 0, st, recvmeta, n_recv, k, first, n_local, ids_loc, w_loc);
}

__global__ void __launch_bounds__(EP_THREADS) ep_ret_plan_kernel(const int* __restrict__ ids_loc, int n_recv, int k,
                                                                  int* __restrict__ pos) {
  pdl_enter();
  __shared__ int sh[32];
  __shared__ int base;
  if (threadIdx.x == 0) base = 0;
  __syncthreads();
  for (int r0 = 0; r0 < n_recv; r0 += EP_THREADS) {
    const int i = r0 + threadIdx.x;
    int c[1] = {0}, ex[1], tot[1];
    if (i < n_recv)
      for (int j = 0; j < k; ++j) c[0] += ids_loc[(int64_t)i * k + j] >= 0 ? 1 : 0;
    block_scan<1>(c, ex, tot, sh);
    if (i < n_recv)
      for (int j = 0; j < k; ++j) {
        const int e = ids_loc[(int64_t)i * k + j];
        if (e < 0) {
          pos[(int64_t)i * k + j] = -1;
          continue;
        }
        int rank = 0;
        for (int j2 = 0; j2 < k; ++j2) {
          const int e2 = ids_loc[(int64_t)i * k + j2];
          rank += (e2 >= 0 && e2 < e) ? 1 : 0;
        }
        pos[(int64_t)i * k + j] = base + ex[0] + rank;
      }
    __syncthreads();
    if (threadIdx.x == 0) base += tot[0];
    __syncthreads();
  }
}

void launch_ep_ret_plan(const int* ids_loc, int n_recv, int k, int* ret_send_pos, cudaStream_t st) {
  if (n_recv <= 0) return;
  launch_k(ep_ret_plan_kernel, 1, EP_THREADS, 0, st, ids_loc, n_recv, k, ret_send_pos);
}

// One warp per (row, selection).
__global__ void ep_ret_pack_kernel(const float* __restrict__ y, const int* __restrict__ tok_slot,
                                   const int* __restrict__ pos, int n_recv, int k, int d, int cap,
                                   float* __restrict__ out) {
  pdl_enter();
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  if (gw >= (int64_t)n_recv * k) return;
  const int p = pos[gw];
  if (p < 0 || p >= cap) return;  // cap: rows the return buffer holds
  const float4* src = reinterpret_cast<const float4*>(y + (int64_t)tok_slot[gw] * d);
  float4* dst = reinterpret_cast<float4*>(out + (int64_t)p * d);
  for (int c = lane; c < d / 4; c += 32) dst[c] = src[c];
}

void launch_ep_ret_pack(const float* y, const int* tok_slot, const int* ret_send_pos, int n_recv, int k, int d,
                        int cap, float* retsend, cudaStream_t st) {
  const int64_t warps = (int64_t)n_recv * k;
  if (warps <= 0) return;
  launch_k(ep_ret_pack_kernel, ceil_div(warps * 32, 256), 256, 0, st, y, tok_slot, ret_send_pos, n_recv, k, d,
           cap, retsend);
}

// ---- NCCL steps ---------------------------------------------------------------
int ep_exchange_counts(EpState& s, const int* send_dev, int* recv_dev, cudaStream_t st) {
  ncclComm_t comm = static_cast<ncclComm_t>(s.comm);
  ncclResult_t r = ncclGroupStart();
  for (int q = 0; q < s.world && r == ncclSuccess; ++q) {
    if (q == s.rank) continue;
    r = ncclSend(send_dev + 2 * q, 2, ncclInt32, q, comm, st);
    if (r == ncclSuccess) r = ncclRecv(recv_dev + 2 * q, 2, ncclInt32, q, comm, st);
  }
  const ncclResult_t r2 = ncclGroupEnd();
  if (r != ncclSuccess || r2 != ncclSuccess) {
    s.err = std::string("count exchange: ") + ncclGetErrorString(r != ncclSuccess ? r : r2);
    return KC_ERR_NCCL;
  }
  if (cudaMemcpyAsync(recv_dev + 2 * s.rank, send_dev + 2 * s.rank, 2 * sizeof(int), cudaMemcpyDeviceToDevice,
                      st) != cudaSuccess) {
    s.err = "count exchange: self copy failed";
    return KC_ERR_CUDA;
  }
  return KC_OK;
}

int ep_alltoallv(EpState& s, const EpA2A* parts, int n_parts, cudaStream_t st) {
  ncclComm_t comm = static_cast<ncclComm_t>(s.comm);
  const int me = s.rank;
  for (int p = 0; p < n_parts; ++p)
    if (parts[p].send_bytes[me] != parts[p].recv_bytes[me]) {
      s.err = "all-to-all: own section sizes differ";
      return KC_ERR_STATE;
    }
  ncclResult_t r = ncclGroupStart();
  for (int p = 0; p < n_parts && r == ncclSuccess; ++p) {
    const EpA2A& a = parts[p];
    const char* sp = static_cast<const char*>(a.send);
    char* rp = static_cast<char*>(a.recv);
    for (int q = 0; q < s.world && r == ncclSuccess; ++q) {
      if (q == me) continue;
      if (a.send_bytes[q] > 0) r = ncclSend(sp + a.send_off[q], (size_t)a.send_bytes[q], ncclInt8, q, comm, st);
      if (r == ncclSuccess && a.recv_bytes[q] > 0)
        r = ncclRecv(rp + a.recv_off[q], (size_t)a.recv_bytes[q], ncclInt8, q, comm, st);
    }
  }
  const ncclResult_t r2 = ncclGroupEnd();
  if (r != ncclSuccess || r2 != ncclSuccess) {
    s.err = std::string("all-to-all: ") + ncclGetErrorString(r != ncclSuccess ? r : r2);
    return KC_ERR_NCCL;
  }
  for (int p = 0; p < n_parts; ++p) {
    const EpA2A& a = parts[p];
    if (a.send_bytes[me] > 0 &&
        cudaMemcpyAsync(static_cast<char*>(a.recv) + a.recv_off[me], static_cast<const char*>(a.send) + a.send_off[me],
                        (size_t)a.send_bytes[me], cudaMemcpyDeviceToDevice, st) != cudaSuccess) {
      s.err = "all-to-all: self copy failed";
      return KC_ERR_CUDA;
    }
  }
  return KC_OK;
}

}  // namespace kc
