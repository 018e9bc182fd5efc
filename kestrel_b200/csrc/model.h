// Kernels of the dense decode path around the MoE layer (model.cu): the
// pieces of Transformer::forward_chunk (crates/kestrel-engine/src/
// transformer.rs:375-467) other than the quantized matvecs and the MoE FFN.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace kc {

// quant::get_row (quant.rs:342-345): x[s] = dequant_row(E row tok[s]) for a
// row-major GGUF tensor E (row_bytes per row). Ids >= n_vocab set the status
// word to KC_ERR_ARG and write zeros.
void launch_embed(const uint8_t* E, int t, int64_t row_bytes, const uint32_t* tok, int n, int d, int n_vocab,
                  float* x, int* status, cudaStream_t st);

// For each of `rows` rows of `dim` values: x += y (when y is non-null, x is
// updated in place), then out = rmsnorm(x, w) (transformer.rs:330-340).
void launch_add_rmsnorm(float* x, const float* y, const float* w, int rows, int dim, float eps, float* out,
                        cudaStream_t st);
// The general form: the addend is y or the MoE combine of the row's token
// (cy = the expert products per slot, with the dispatch's tok_slot and the
// routing ids / weights; row i is token tok0 + i), and the Q8_K records of
// out can be written for a following int8 product (rec: [dim / 256][rec_slots]
// records, row i in slot i).
struct NormArgs {
  float* x;
  const float* y;
  const float* cy;
  const int* tok_slot;
  const int* ids;
  const float* cw;
  int k, tok0;
  const float* w;
  int dim;
  float eps;
  float* out;
  uint8_t* rec;
  int64_t rec_slots;
};
void launch_add_rmsnorm(const NormArgs& a, int rows, cudaStream_t st);

// Per token s and head: the q / k / v rows of qkv [n, (nh + 2 nkv) * hd]
// get their bias (if any), q / k get rmsnorm over hd with qn / kn (if any)
// and RoPE at position pos0 + s from the (sin, cos) table [n_ctx][rd / 2];
// q goes to q_out [n, nh, hd], k and v to the f16 caches at row pos0 + s
// (transformer.rs:400-421).
struct QkPostArgs {
  const float* qkv;
  int n, nh, nkv, hd, rd, pos0;
  bool neox;
  float eps;
  const float *bq, *bk, *bv, *qn, *kn;
  const float2* rope;
  float* q_out;
  __half *kc, *vc;
  const int* pos_dev;  // non-null: the position of token 0 is *pos_dev (pos0 ignored)
  // Non-null: row s is its own sequence, at position row_pos[s], with its
  // caches at kc / vc + s * seq_stride (pos0 / pos_dev ignored).
  const int* row_pos;
  int64_t seq_stride;
};
void launch_qk_post(const QkPostArgs& a, cudaStream_t st);

// Causal GQA attention of n queries at positions pos0.. over the f16 caches
// (transformer.rs:594-631): out [n, nh * hd]. hd % 8 == 0 and at most
// attention_max_positions(hd) positions.
int attention_max_positions(int hd);
// pos_dev non-null: positions start at *pos_dev (at most max_pos of them).
// row_pos non-null: row s is its own sequence -- it attends to positions
// 0 .. row_pos[s] of the caches at kc / vc + s * seq_stride.
void launch_attention(const float* q, const __half* kc, const __half* vc, int n, int nh, int nkv, int hd, int pos0,
                      const int* pos_dev, int max_pos, float scale, float* out, cudaStream_t st,
                      const int* row_pos = nullptr, int64_t seq_stride = 0);

// Rows of independent sequences: hist[s * hist_stride + *step] = next[s] and
// ++pos[s] for s < n, then ++*step (one block).
void launch_advance_rows(const uint32_t* next, uint32_t* hist, int64_t hist_stride, int n, int* step, int* pos,
                         cudaStream_t st);

// hist[*step] = *next; ++*step; ++*pos (one thread).
void launch_advance(const uint32_t* next, uint32_t* hist, int* step, int* pos, cudaStream_t st);

// sampler::argmax (sampler.rs:104-112) of l [n]: the first maximum; for
// `rows` rows of l [rows][n], out[r] (one block per row).
void launch_argmax(const float* l, int n, uint32_t* out, cudaStream_t st, int rows = 1);

// Dense FFN activation in place: g = g / (1 + exp(-g)) * u (transformer.rs:449).
void launch_swiglu(float* g, const float* u, int64_t n, cudaStream_t st);

}  // namespace kc
