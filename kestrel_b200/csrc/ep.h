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

// Device-initiated exchange over NVLink peer memory. Every rank holds an
// arena (CUDA IPC, mapped by every peer) with fixed capacity: T tokens per
// source rank. Layout (byte offsets, the same on every rank):
//   rows [src][T][d] f32 | meta [src][T][2k] i32 (ids, weight bits)
//   | ret [owner][T * k][d] f32 | lines [src][2][32] u32 (flag, count, path)
// Senders store rows / results straight into the peer's arena, then publish
// (count, sequence number) on the line [sender][0 rows | 1 results]. The rows
// line also carries the exchange path the sender took in this call (peer
// memory or NCCL): every rank must take the same one, and a rank that sees
// another path reports KC_ERR_STATE instead of waiting for data that will
// not come.
struct EpP2P {
  bool ready = false;
  int T = 0, d = 0, k = 0;
  int64_t ret_cap = 0;  // result rows per owner section: T * k
  int64_t off_meta = 0, off_ret = 0, off_lines = 0, bytes = 0;
  uint8_t* arena = nullptr;
  uint8_t* peer[kEpMaxWorld] = {};  // every rank's arena, own included
  int* counter = nullptr;           // last-CTA counters of the two send kernels
  uint32_t seq = 0;                 // per-call sequence number, the same on every rank
};

struct EpState {
  int world = 1;
  int rank = 0;
  void* comm = nullptr;  // ncclComm_t
  std::string err;
  EpP2P p2p;
};

// Map the peer arenas for up to T tokens per rank of rows of d values with k
// selections (collective over the group; replaces an earlier mapping).
int ep_p2p_setup(EpState& s, int T, int d, int k, cudaStream_t st);
void ep_p2p_free(EpState& s);

struct EpP2PArgs {
  uint8_t* peer[kEpMaxWorld];
  int world, me, T, d, k;
  int64_t ret_cap, off_meta, off_ret, off_lines;
  uint32_t seq;
  int* counter;
  int* status;
  int path;  // this rank's exchange path in the call (kEpPathPeer / kEpPathNccl)
};
enum : int { kEpPathPeer = 1, kEpPathNccl = 2 };
EpP2PArgs ep_p2p_args(const EpState& s, int* status);
// Home: store the rows (and meta) for every owner into its arena at
// [me][i], then publish (count, seq) on each owner's line [me][0].
void launch_ep_p2p_send(const EpP2PArgs& a, const float* h, const int* ids, const float* w, const int* send_tok,
                        const int* xch_out, int T_home, cudaStream_t st);
// Wait (bounded) until every rank has published sequence a.seq on this rank's
// lines [src][which] (0: rows arrived, 1: results arrived). On the rows line
// it also checks that the source took this rank's path (a.path) and records
// KC_ERR_STATE if not; once the status holds KC_ERR_STATE the waits return at
// once, so a call whose ranks disagree ends quickly on every rank.
void launch_ep_p2p_wait(const EpP2PArgs& a, int which, cudaStream_t st);
// A rank that exchanges through NCCL while the peer arenas are mapped
// publishes (count 0, seq, path NCCL) on every rank's rows line, so that the
// ranks can compare paths before any NCCL call is made.
void launch_ep_p2p_announce(const EpP2PArgs& a, cudaStream_t st);
// Owner: local ids / weights of the arena's rows [src][T] (-1 beyond each
// source's count and for other owners' experts).
void launch_ep_p2p_local_ids(const EpP2PArgs& a, int first, int n_local, int* ids_loc, float* w_loc,
                             cudaStream_t st);
// Owner: position of (row, selection) in its source's result section: rows of
// a source in order, each row's local experts ascending (-1: not local).
void launch_ep_p2p_ret_plan(const int* ids_loc, int world, int T, int k, int* pos, cudaStream_t st);
// Owner: store every local (row, selection) result row into its source's
// arena at [me][pos], then publish seq on each source's line [me][1].
void launch_ep_p2p_ret_send(const EpP2PArgs& a, const float* y, const int* tok_slot, const int* pos,
                            cudaStream_t st);

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
// ret_stride > 0: owner r's section starts at r * ret_stride instead of the
// prefix of the sections before it (the fixed-capacity arena layout).
void launch_ep_plan(const int* ids, int n_tok, int k, int world, int epr, int T, int* send_tok, int* ret_pos,
                    int* xch_out, cudaStream_t st, int64_t ret_stride = 0);
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
