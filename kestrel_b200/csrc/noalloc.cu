// kc_route_noalloc: expert routing (router logits -> softmax -> top-k ->
// renormalisation) that performs no device allocation of any kind.
//
// Some hosts cannot let a library call cudaMalloc: a Kestrel session whose
// memory ledger must account for every byte it places, a latency-critical
// decode thread that cannot afford the device-wide synchronisation that
// cudaMalloc/cudaFree may cause, or an embedding that hands out device memory
// only from its own pool. The regular entry points keep their scratch in a context workspace
// that grows with cudaMalloc; this one keeps its only scratch -- the
// [n_tok, n_expert] router logits -- in a fixed array compiled into the
// library. The array lives on every GPU that loads the library, for the life
// of the process.
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace kc {
void set_global_error(const char* msg);
}

namespace {

using namespace kc;

// Maximum n_tok * n_expert of one call: 65536 f32 logits (256 KB per GPU).
constexpr int64_t kRouteScratchFloats = 64 * 1024;
static __device__ __align__(256) float g_route_scratch[kRouteScratchFloats];
// Failure word of the call, cleared at its start (a 4-byte memset, no
// allocation). The logits kernel records a bounded wait that expired in it;
// the top-k kernel then writes every selection as id -1, weight 0, so such a
// call cannot pass for a good one.
static __device__ int g_route_status;

// Device address of g_route_scratch, resolved once per device. In host code
// the array's name is only a host-side handle; kernels must be given this
// address instead.
constexpr int kMaxDevices = 64;
float* g_scratch_addr[kMaxDevices] = {};
int* g_status_addr[kMaxDevices] = {};
std::mutex g_scratch_mu;

int scratch_for_current_device(float** out, int** status) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_global_error("kc_route_noalloc: no usable current CUDA device");
    return KC_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_route_scratch);
    if (e != cudaSuccess || !p) {
      set_global_error("kc_route_noalloc: cudaGetSymbolAddress of the routing scratch failed");
      return KC_ERR_CUDA;
    }
    void* q = nullptr;
    const cudaError_t e2 = cudaGetSymbolAddress(&q, g_route_status);
    if (e2 != cudaSuccess || !q) {
      set_global_error("kc_route_noalloc: cudaGetSymbolAddress of the status word failed");
      return KC_ERR_CUDA;
    }
    g_status_addr[dev] = static_cast<int*>(q);
    g_scratch_addr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_addr[dev];
  *status = g_status_addr[dev];
  return KC_OK;
}

}  // namespace

extern "C" KC_API int kc_route_noalloc(const float* router_w, int n_expert, int d, const float* h, int n_tok, int k,
                                       int norm_topk, float weights_scale, int32_t* topk_ids, float* topk_w,
                                       void* stream) {
  if (n_tok < 0 || n_expert <= 0 || d <= 0 || k < 1 || k > 64 || k > n_expert || n_expert > 1024) {
    set_global_error("kc_route_noalloc: bad arguments (need 1 <= k <= min(64, n_expert), n_expert <= 1024)");
    return KC_ERR_ARG;
  }
  if (n_tok == 0) return KC_OK;
  if (!router_w || !h || !topk_ids || !topk_w) {
    set_global_error("kc_route_noalloc: null buffer");
    return KC_ERR_ARG;
  }
  if ((int64_t)n_tok * n_expert > kRouteScratchFloats) {
    set_global_error("kc_route_noalloc: n_tok * n_expert exceeds the fixed scratch of 65536 logits");
    return KC_ERR_SHAPE;
  }
  float* logits = nullptr;
  int* status = nullptr;
  const int rc = scratch_for_current_device(&logits, &status);
  if (rc != KC_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Every logit the top-k stage reads is written first, so the logits need no
  // clearing between calls; the failure word does.
  cudaError_t e = cudaMemsetAsync(status, 0, sizeof(int), st);
  if (e != cudaSuccess) {
    set_global_error(cudaGetErrorString(e));
    return KC_ERR_CUDA;
  }
  launch_router_logits(router_w, d, n_expert, d, h, n_tok, logits, status, st);
  launch_route(logits, n_tok, n_expert, k, norm_topk, weights_scale, topk_ids, topk_w, st, status);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_global_error(cudaGetErrorString(e));
    return KC_ERR_CUDA;
  }
  return KC_OK;
}
