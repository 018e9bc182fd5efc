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
