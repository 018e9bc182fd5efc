// Expert-parallel group state (one process per GPU, NCCL over NVLink).
#pragma once

#include <string>

namespace kc {

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

}  // namespace kc
