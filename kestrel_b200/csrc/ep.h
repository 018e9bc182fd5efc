// Expert parallelism (one process per GPU, NCCL over NVLink): group state, the
// exchange plans and the all-to-all steps of a layer (ep.cu).
//
// Experts of every layer are sharded in contiguous blocks: rank r owns global
// experts [r * epr, (r + 1) * epr), epr = E / world. Each rank routes its own
// tokens, sends every token once to each rank owning one of its experts, and
// gets back one result row per (token, selected expert), which it combines in
// ascending expert id exactly as on one GPU.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace kc {

constexpr int kEpMaxWorld = 8;

struct EpState {
  int world = 1;
  int rank = 0;
  void* comm = nullptr;  // ncclComm_t
  std::string err;
};

int ep_unique_id(char out[128]);
int ep_init(EpState& s, int rank, int world, const char uid[128]);
void ep_free(EpState& s);
const char* ep_last_error(const EpState& s);

// Home side, after routing: for each destination r, send_tok[r * T + i]
// (i < rows sent to r) lists the tokens sent to r in ascending order;
// xch_out[2r] = rows sent to r, xch_out[2r+1] = result rows expected back
// from r; ret_pos[s * k + j] = row of (token s, selection j) in the
// concatenated return buffer (sections in rank order, within a section tokens
// ascending, within a token its experts owned by r ascending).
void launch_ep_plan(const int* ids, int n_tok, int k, int world, int epr, int T, int* send_tok, int* ret_pos,
                    int* xch_out, cudaStream_t st);
// Pack the rows (and each row's k ids and weights as 2k 32-bit words) sent to
// every destination into contiguous sections in rank order.
void launch_ep_pack(const float* h, const int* ids, const float* w, const int* send_tok, const int* xch_out,
                    int world, int T, int k, int d, float* sendbuf, int32_t* sendmeta, cudaStream_t st);
// Owner side: ids of the received rows mapped to local experts (-1 where the
// expert belongs to another rank) and their weights.
void launch_ep_local_ids(const int32_t* recvmeta, int n_recv, int k, int first, int n_local, int* ids_loc,
                         float* w_loc, cudaStream_t st);
// Owner side: position of (received row i, selection j) in the return buffer
// (-1 for foreign experts): rows in received order, each row's local experts
// ascending -- the order every source computed in ret_pos.
void launch_ep_ret_plan(const int* ids_loc, int n_recv, int k, int* ret_send_pos, cudaStream_t st);
// Owner side: copy the result row of every local (row, selection) from y (by
// its slot) to its return position (positions >= cap, the rows retsend holds,
// are skipped).
void launch_ep_ret_pack(const float* y, const int* tok_slot, const int* ret_send_pos, int n_recv, int k, int d,
                        int cap, float* retsend, cudaStream_t st);

// Exchange two ints with every rank: recv[2r..2r+1] <- rank r's send[2*me..].
int ep_exchange_counts(EpState& s, const int* send_dev, int* recv_dev, cudaStream_t st);
// One buffer pair of an all-to-all: per-peer byte offsets and counts (host
// arrays of `world` entries).
struct EpA2A {
  const void* send;
  const int64_t* send_off;
  const int64_t* send_bytes;
  void* recv;
  const int64_t* recv_off;
  const int64_t* recv_bytes;
};
// All-to-all of n_parts buffer pairs in one NCCL group; the rank's own
// sections are copied on the device.
int ep_alltoallv(EpState& s, const EpA2A* parts, int n_parts, cudaStream_t st);

}  // namespace kc
