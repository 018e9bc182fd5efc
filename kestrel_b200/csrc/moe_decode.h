// The routed-expert layer of a decode batch in one persistent launch
// (moe_decode.cu): router logits, top-k, dispatch, gate/up, SwiGLU, down and
// the weighted combine, with the reference's arithmetic of the separate
// kernels (router.cu, decode.cu) bit for bit.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace kc {

struct MoeDecodeArgs {
  const float* router;  // [E, d] F32
  int E, k, d, ff;
  int norm_topk;
  float weights_scale;
  const uint8_t* gate;  // tiled expert tables (common.cuh), expert e at e * mb_gate / e * mb_down
  const uint8_t* up;
  const uint8_t* down;
  int64_t mb_gate, mb_down;
  int t_gate, t_down;
  const float* h;  // [n_tok, d] input rows
  int n_tok;
  float* out;      // [n_tok, d] the combine
  int* ids;        // [n_tok, k] top-k ids and weights (written by CTA 0)
  float* w;
  float* logits;   // workspace: [n_tok, E]
  uint8_t* xrec;   // [ceil(d / 256)][n_tok] activation records of the input rows
  float* g;        // [n_tok * k, ff] gate and up outputs per slot
  float* u;
  uint8_t* arec;   // [ceil(ff / 256)][n_tok * k] records of SwiGLU(g, u)
  float* y;        // [n_tok * k, d] down outputs per slot
  int* sync;       // moe_decode_sync_words(E, ff, d) ints, zero when first used
  int* status;
};

// Ints of the kernel's synchronisation area (grid barrier, completion counters
// and ready flags), to be zeroed once at allocation.
int moe_decode_sync_words(int E, int ff, int d);
// Shapes and types the fused kernel takes (one GPU, decode batches whose
// experts all get at most three rows: n_tok <= 3).
bool moe_decode_supported(int n_tok, int E, int k, int d, int ff, int t_gate, int t_up, int t_down);
int launch_moe_decode(const MoeDecodeArgs& a, cudaStream_t st);

}  // namespace kc
