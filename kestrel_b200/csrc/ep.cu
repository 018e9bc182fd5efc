// NCCL communicator set-up for expert parallelism.
#include <nccl.h>

#include <cstring>
#include <vector>

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
  ep_p2p_free(s);
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
                                                              int* __restrict__ ret_pos, int* __restrict__ xch_out,
                                                              int64_t ret_stride) {
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
        ret_pos[(int64_t)s * k + j] = (int)((ret_stride > 0 ? r * ret_stride : off_c[r]) + exc + rank);
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
                    int* xch_out, cudaStream_t st, int64_t ret_stride) {
  launch_k(ep_plan_kernel, 1, EP_THREADS, 0, st, ids, n_tok, k, world, epr, T, send_tok, ret_pos, xch_out,
           ret_stride);
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


// ===========================================================================
// Device-initiated exchange over NVLink peer memory (see ep.h).

static int64_t al256(int64_t v) { return (v + 255) & ~int64_t(255); }

void ep_p2p_free(EpState& s) {
  EpP2P& p = s.p2p;
  for (int r = 0; r < kEpMaxWorld; ++r)
    if (p.peer[r] && p.peer[r] != p.arena) cudaIpcCloseMemHandle(p.peer[r]);
  if (p.arena) cudaFree(p.arena);
  if (p.counter) cudaFree(p.counter);
  p = EpP2P{};
}

int ep_p2p_setup(EpState& s, int T, int d, int k, cudaStream_t st) {
  if (s.world < 2 || !s.comm) {
    s.err = "peer exchange needs an expert-parallel group";
    return KC_ERR_STATE;
  }
  if (T < 1 || d < 4 || d % 4 || k < 1 || k > 64) {
    s.err = "peer exchange: bad capacity";
    return KC_ERR_ARG;
  }
  ep_p2p_free(s);
  EpP2P& p = s.p2p;
  const int G = s.world;
  p.T = T;
  p.d = d;
  p.k = k;
  p.ret_cap = (int64_t)T * k;
  p.off_meta = al256((int64_t)G * T * d * 4);
  p.off_ret = p.off_meta + al256((int64_t)G * T * 2 * k * 4);
  p.off_lines = p.off_ret + al256((int64_t)G * p.ret_cap * d * 4);
  p.bytes = p.off_lines + al256((int64_t)G * 2 * 32 * 4);
  auto fail_cuda = [&](const char* what) {
    s.err = std::string("peer exchange: ") + what;
    ep_p2p_free(s);
    return KC_ERR_CUDA;
  };
  if (cudaMalloc(&p.arena, p.bytes) != cudaSuccess) return fail_cuda("arena allocation failed");
  if (cudaMemsetAsync(p.arena, 0, p.bytes, st) != cudaSuccess) return fail_cuda("arena clear failed");
  if (cudaMalloc(&p.counter, 2 * sizeof(int)) != cudaSuccess) return fail_cuda("counter allocation failed");
  if (cudaMemsetAsync(p.counter, 0, 2 * sizeof(int), st) != cudaSuccess) return fail_cuda("counter clear failed");
  cudaIpcMemHandle_t mine;
  if (cudaIpcGetMemHandle(&mine, p.arena) != cudaSuccess) return fail_cuda("cudaIpcGetMemHandle failed");
  // Share the handles (64 bytes each) with an NCCL all-gather.
  char* dbuf = nullptr;
  if (cudaMalloc(&dbuf, (size_t)(G + 1) * sizeof(mine)) != cudaSuccess) return fail_cuda("handle buffer");
  cudaMemcpyAsync(dbuf + G * sizeof(mine), &mine, sizeof(mine), cudaMemcpyHostToDevice, st);
  ncclResult_t r = ncclAllGather(dbuf + G * sizeof(mine), dbuf, sizeof(mine), ncclInt8,
                                 static_cast<ncclComm_t>(s.comm), st);
  std::vector<cudaIpcMemHandle_t> all(G);
  if (r == ncclSuccess)
    cudaMemcpyAsync(all.data(), dbuf, (size_t)G * sizeof(mine), cudaMemcpyDeviceToHost, st);
  const cudaError_t e = cudaStreamSynchronize(st);
  cudaFree(dbuf);
  if (r != ncclSuccess) {
    s.err = std::string("peer exchange: handle all-gather: ") + ncclGetErrorString(r);
    ep_p2p_free(s);
    return KC_ERR_NCCL;
  }
  if (e != cudaSuccess) return fail_cuda("handle exchange failed");
  for (int q = 0; q < G; ++q) {
    if (q == s.rank) {
      p.peer[q] = p.arena;
      continue;
    }
    void* ptr = nullptr;
    if (cudaIpcOpenMemHandle(&ptr, all[q], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
      return fail_cuda("cudaIpcOpenMemHandle failed (GPUs without peer access?)");
    p.peer[q] = static_cast<uint8_t*>(ptr);
  }
  p.seq = 0;
  p.ready = true;
  return KC_OK;
}

EpP2PArgs ep_p2p_args(const EpState& s, int* status) {
  EpP2PArgs a{};
  const EpP2P& p = s.p2p;
  for (int r = 0; r < kEpMaxWorld; ++r) a.peer[r] = p.peer[r];
  a.world = s.world;
  a.me = s.rank;
  a.T = p.T;
  a.d = p.d;
  a.k = p.k;
  a.ret_cap = p.ret_cap;
  a.off_meta = p.off_meta;
  a.off_ret = p.off_ret;
  a.off_lines = p.off_lines;
  a.seq = p.seq;
  a.counter = p.counter;
  a.status = status;
  a.path = kEpPathPeer;
  return a;
}

__device__ __forceinline__ uint32_t* ep_line(uint8_t* arena, int64_t off_lines, int src, int which) {
  return reinterpret_cast<uint32_t*>(arena + off_lines) + (src * 2 + which) * 32;
}

// The last CTA of a sending grid publishes (count, seq) on every rank's line.
// Every CTA fences its peer stores at system scope before counting itself.
__device__ __forceinline__ bool ep_last_cta(int* counter) {
  __shared__ int last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(counter, 1);
    last = prev == (int)(gridDim.x * gridDim.y) - 1;
    if (last) *counter = 0;  // ready for the next launch (nobody else touches it now)
  }
  __syncthreads();
  if (last) __threadfence_system();
  return last;
}

__device__ __forceinline__ void ep_publish(uint32_t* line, uint32_t count, uint32_t seq, uint32_t path = 0) {
  volatile uint32_t* v = line;
  v[1] = count;
  v[2] = path;
  __threadfence_system();
  v[0] = seq;
}

// One warp per (owner r, row i): rows of the home's tokens to r's arena at
// [me][i], then the last CTA publishes the counts.
__global__ void ep_p2p_send_kernel(const EpP2PArgs a, const float* __restrict__ h, const int* __restrict__ ids,
                                   const float* __restrict__ w, const int* __restrict__ send_tok,
                                   const int* __restrict__ xch_out, int T_home) {
  pdl_enter();
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  const int r = (int)(gw / T_home), i = (int)(gw % T_home);
  if (r < a.world && i < xch_out[2 * r]) {
    const int s = send_tok[(int64_t)r * T_home + i];
    uint8_t* base = a.peer[r];
    const int64_t row = (int64_t)a.me * a.T + i;
    const float4* src = reinterpret_cast<const float4*>(h + (int64_t)s * a.d);
    float4* dst = reinterpret_cast<float4*>(base) + row * (a.d / 4);
    for (int c = lane; c < a.d / 4; c += 32) dst[c] = src[c];
    int32_t* meta = reinterpret_cast<int32_t*>(base + a.off_meta) + row * 2 * a.k;
    for (int c = lane; c < a.k; c += 32) {
      meta[c] = ids[(int64_t)s * a.k + c];
      meta[a.k + c] = __float_as_int(w[(int64_t)s * a.k + c]);
    }
  }
  if (ep_last_cta(a.counter)) {
    for (int q = threadIdx.x; q < a.world; q += blockDim.x)
      ep_publish(ep_line(a.peer[q], a.off_lines, a.me, 0), (uint32_t)xch_out[2 * q], a.seq, (uint32_t)a.path);
  }
}

void launch_ep_p2p_send(const EpP2PArgs& a, const float* h, const int* ids, const float* w, const int* send_tok,
                        const int* xch_out, int T_home, cudaStream_t st) {
  const int64_t warps = (int64_t)a.world * T_home;
  launch_k(ep_p2p_send_kernel, ceil_div(std::max<int64_t>(warps, 1) * 32, 256), 256, 0, st, a, h, ids, w, send_tok,
           xch_out, T_home);
}

// One thread per source: bounded spin until its line carries this call's
// sequence number; on the rows line, then compare the source's path with
// this rank's.
__global__ void ep_p2p_wait_kernel(const EpP2PArgs a, int which) {
  pdl_enter();
  const int src = threadIdx.x;
  if (src >= a.world) return;
  // A call whose ranks already disagree on the path: nothing more will come.
  if (a.status && (*(volatile int*)a.status & 0xFF) == KC_ERR_STATE) return;
  volatile uint32_t* f = ep_line(a.peer[a.me], a.off_lines, src, which);
  if ((int)(*f - a.seq) < 0) {
    const uint64_t t0 = globaltimer();
    while ((int)(*f - a.seq) < 0) {
      if (globaltimer() - t0 > kWaitLimitNs) {
        report(a.status, KC_ERR_TIMEOUT | (W_EP_PEER << 8));
        break;
      }
    }
  }
  __threadfence_system();
  if (which == 0 && *f == a.seq && f[2] != (uint32_t)a.path) report(a.status, KC_ERR_STATE | (W_EP_PATH << 8));
}

__global__ void ep_p2p_announce_kernel(const EpP2PArgs a) {
  pdl_enter();
  for (int q = threadIdx.x; q < a.world; q += blockDim.x)
    ep_publish(ep_line(a.peer[q], a.off_lines, a.me, 0), 0u, a.seq, (uint32_t)a.path);
}

void launch_ep_p2p_announce(const EpP2PArgs& a, cudaStream_t st) {
  launch_k(ep_p2p_announce_kernel, 1, 32, 0, st, a);
}

void launch_ep_p2p_wait(const EpP2PArgs& a, int which, cudaStream_t st) {
  launch_k(ep_p2p_wait_kernel, 1, 32, 0, st, a, which);
}

__global__ void ep_p2p_local_ids_kernel(const EpP2PArgs a, int first, int n_local, int* __restrict__ ids_loc,
                                        float* __restrict__ w_loc) {
  pdl_enter();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)a.world * a.T * a.k) return;
  const int64_t row = i / a.k, j = i % a.k;
  const int src = (int)(row / a.T), r = (int)(row % a.T);
  const uint32_t cnt = ep_line(a.peer[a.me], a.off_lines, src, 0)[1];
  const int32_t* meta = reinterpret_cast<const int32_t*>(a.peer[a.me] + a.off_meta) + row * 2 * a.k;
  const bool valid = (uint32_t)r < cnt;
  const int e = valid ? meta[j] : -1;
  ids_loc[i] = (e >= first && e < first + n_local) ? e - first : -1;
  w_loc[i] = valid ? __int_as_float(meta[a.k + j]) : 0.f;
}

void launch_ep_p2p_local_ids(const EpP2PArgs& a, int first, int n_local, int* ids_loc, float* w_loc,
                             cudaStream_t st) {
  const int64_t n = (int64_t)a.world * a.T * a.k;
  launch_k(ep_p2p_local_ids_kernel, ceil_div(n, 256), 256, 0, st, a, first, n_local, ids_loc, w_loc);
}

__global__ void __launch_bounds__(EP_THREADS) ep_p2p_ret_plan_kernel(const int* __restrict__ ids_loc, int world,
                                                                      int T, int k, int* __restrict__ pos) {
  pdl_enter();
  __shared__ int sh[32];
  __shared__ int base, sec_base[kEpMaxWorld];
  if (threadIdx.x == 0) base = 0;
  __syncthreads();
  const int n = world * T;
  for (int r0 = 0; r0 < n; r0 += EP_THREADS) {
    const int q = r0 + threadIdx.x;
    int c[1] = {0}, ex[1], tot[1];
    if (q < n)
      for (int j = 0; j < k; ++j) c[0] += ids_loc[(int64_t)q * k + j] >= 0 ? 1 : 0;
    block_scan<1>(c, ex, tot, sh);
    if (q < n && q % T == 0) sec_base[q / T] = base + ex[0];
    __syncthreads();
    if (q < n)
      for (int j = 0; j < k; ++j) {
        const int e = ids_loc[(int64_t)q * k + j];
        if (e < 0) {
          pos[(int64_t)q * k + j] = -1;
          continue;
        }
        int rank = 0;
        for (int j2 = 0; j2 < k; ++j2) {
          const int e2 = ids_loc[(int64_t)q * k + j2];
          rank += (e2 >= 0 && e2 < e) ? 1 : 0;
        }
        pos[(int64_t)q * k + j] = base + ex[0] - sec_base[q / T] + rank;
      }
    __syncthreads();
    if (threadIdx.x == 0) base += tot[0];
    __syncthreads();
  }
}

void launch_ep_p2p_ret_plan(const int* ids_loc, int world, int T, int k, int* pos, cudaStream_t st) {
  launch_k(ep_p2p_ret_plan_kernel, 1, EP_THREADS, 0, st, ids_loc, world, T, k, pos);
}

// One warp per (row, selection): the result row to its source's arena at
// [me][pos]; then the last CTA publishes on every source's line [me][1].
__global__ void ep_p2p_ret_send_kernel(const EpP2PArgs a, const float* __restrict__ y,
                                       const int* __restrict__ tok_slot, const int* __restrict__ pos) {
  pdl_enter();
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  if (gw < (int64_t)a.world * a.T * a.k) {
    const int p = pos[gw];
    if (p >= 0 && p < a.ret_cap) {
      const int src = (int)(gw / a.k / a.T);
      const float4* s4 = reinterpret_cast<const float4*>(y + (int64_t)tok_slot[gw] * a.d);
      float4* d4 = reinterpret_cast<float4*>(a.peer[src] + a.off_ret) + ((int64_t)a.me * a.ret_cap + p) * (a.d / 4);
      for (int c = lane; c < a.d / 4; c += 32) d4[c] = s4[c];
    }
  }
  if (ep_last_cta(a.counter + 1)) {
    for (int q = threadIdx.x; q < a.world; q += blockDim.x)
      ep_publish(ep_line(a.peer[q], a.off_lines, a.me, 1), 0u, a.seq);
  }
}

void launch_ep_p2p_ret_send(const EpP2PArgs& a, const float* y, const int* tok_slot, const int* pos,
                            cudaStream_t st) {
  const int64_t warps = (int64_t)a.world * a.T * a.k;
  launch_k(ep_p2p_ret_send_kernel, ceil_div(warps * 32, 256), 256, 0, st, a, y, tok_slot, pos);
}

}  // namespace kc
