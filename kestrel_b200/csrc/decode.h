// Decode-sized grouped dequant-dot (decode.cu) and its activation records.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace kc {

struct DecodeArgs {
  const uint8_t* w[2];     // matrices (gate, up) or (down / dense, unused)
  int n_mat;               // 1 or 2
  int64_t expert_stride;   // bytes between experts' matrices
  int expert_base;         // global id of the first expert held
  int rows, cols;          // one expert's matrix
  int type;                // KC_Q4_K / KC_Q6_K / KC_Q8_0
  const int* list;         // expert ids (1..3 rows each)
  const int* n_list;       // device scalar
  const int* offsets;      // [E+1] slot ranges
  const int* slot_src;     // activation record row of a slot (null: slot)
  const uint8_t* act;      // activation records
  int64_t act_stride;      // bytes per record row
  float* out[2];           // out[m][slot * out_stride + row]
  int64_t out_stride;
  int* status;
};

// Stage geometry of one weight type / row length (decode.cu).
struct DecodeGeom {
  int type;
  int nsb;       // superblocks per row (Q8_0: chunks of 8 blocks)
  int nb32;      // Q8_0 blocks per row
  int ks;        // superblocks per K segment
  int nseg;      // segments per row
  int64_t tile_bytes;  // bytes of one 16-row tile
  int stage_bytes;
};

DecodeGeom decode_geom(int t, int64_t cols);
int launch_decode(const DecodeArgs& a, int max_units, cudaStream_t st);

// Activation records (Q8_K for K-quant weights, Q8 per-32 for Q8_0): x rows
// [n_rows, cols] f32 -> records; with u != null the rows are first combined
// as SwiGLU g / (1 + exp(-g)) * u, and the combined rows are also written to
// f32out / f16out when those are non-null.
void launch_act_records(bool kquant, const float* x, const float* u, int64_t n_rows, int64_t cols, uint8_t* rec,
                        float* f32out, __half* f16out, cudaStream_t st);
inline int64_t act_rec_stride(bool kquant, int64_t cols) {
  return kquant ? cols / 256 * 336 : (cols / 32 + 7) / 8 * 288;
}

}  // namespace kc
