// Host-side launchers of the library's kernels (one definition per .cu file).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace kc {

// Slots per work tile of the tensor-core grouped products (the MMA's N).
constexpr int kMmaTileN = 256;

// Activation rows of a grouped product: slot i reads activation row
// slot_src[i] (or i when slot_src is null).
struct GroupedArgs {
  const uint8_t* w0;      // weights of the expert(s), device layout
  const uint8_t* w1;      // second matrix for the gate/up pair (or null)
  int64_t expert_stride;  // bytes between consecutive experts' matrices
  int expert_base;        // global id of the first expert held in w0 / w1
  const int* slot;        // host-streamed experts: slot of expert e (null: e - expert_base)
  int rows, cols;         // one expert's matrix (tiled device layout)
  int type;               // ggml type of w0 / w1
  const int* list;        // expert ids to process
  const int* n_list;      // device scalar: entries in list
  const int* offsets;     // [E+1]: slots of expert e are offsets[e] .. offsets[e+1]-1
  const int* slot_src;    // activation row of each slot (null: identity)
  const int8_t* aq;       // quantised activations [n_act][cols] (int8 path)
  const float* ad;        // their block scales
  const int32_t* asum;    // their per-16 sums
  const float* af;        // f32 activations [n_act][cols] (f32 path)
  float* out;             // out[slot * out_stride + row]
  float* out2;            // second matrix's output (pair products)
  int64_t out_stride;
  int* status;            // device status word (timeouts)
};

// quantize.cu
void launch_q8k_quantize(const float* x, const int* row_map, int64_t n_rows, int64_t cols, int8_t* q, float* d,
                         int32_t* bsums, cudaStream_t st);
void launch_q8_quantize(const float* x, const int* row_map, int64_t n_rows, int64_t cols, int8_t* q, float* d,
                        int32_t* s16, cudaStream_t st);
int launch_quantize(int t, const float* x, int64_t rows, int64_t cols, void* out, cudaStream_t st);
int launch_repack(int t, const void* src, int64_t n_mats, int64_t rows, int64_t cols, void* dst, cudaStream_t st);
void launch_block_sums(int t, const void* w, int64_t rows, int64_t cols, const int8_t* q, const int32_t* bsums,
                       int n_act, int32_t* out, cudaStream_t st);

// router.cu
// force_dot: always quant::dot's order (the reference's vector dots, e.g. the
// shared-expert gate), whatever n_tok.
void launch_router_logits(const float* w, int64_t row_stride_floats, int E, int d, const float* h, int n_tok,
                          float* logits, int* status, cudaStream_t st, bool force_dot = false);
// out[s, :] += g[s] * y[s, :] with g[s] = 1 / (1 + exp(-logit[s])) (logit
// null: g = 1): the shared expert's contribution (transformer.rs:577-585).
void launch_shared_add(const float* y, const float* logit, int n_tok, int d, float* out, cudaStream_t st);
// fail (optional): a status word written by earlier kernels of the call; when
// it is nonzero at the route kernel, every selection is written as id -1,
// weight 0.
void launch_route(const float* logits, int n_tok, int E, int k, int norm_topk, float weights_scale, int* ids,
                  float* w, cudaStream_t st, const int* fail = nullptr);
// Dispatch metadata of one routed batch (see router.cu).
struct DispatchOut {
  int* counts;     // [E]
  int* offsets;    // [E+1]
  int* slot_tok;   // [n_tok*k] token of each slot
  float* slot_w;   // [n_tok*k] routing weight of each slot
  int* tok_slot;   // [n_tok*k] slot of token s's j-th selection
  int* small_list; // experts with 1..3 rows (int8 path); value e | part << 16
                   // (rows 3 part .. of expert e; part 0 unless dispatched by rows)
  int* large_list; // experts with >= 4 rows (f32 path)
  int* n_lists;    // [2]: entries in small_list, large_list
  int* large_tt;   // [E+1]: prefix over large_list of ceil(rows / kMmaTileN) token tiles
};
// rows: each row computed as a batch of one would be -- every expert in the
// int8 list, in entries of at most three rows (value e | part << 16), none in
// the tcgen05 list.
int launch_dispatch(const int* ids, const float* w, int n_tok, int k, int E, const DispatchOut& o, cudaStream_t st,
                    bool rows = false);
// Small batches: route + dispatch in one launch (n_tok <= 32), and for decode
// batches (n_tok < 4, rec non-null) also the Q8_K records of each slot's
// input row (x [n_tok, d], records [d / 256][n_tok * k]).
bool route_dispatch_supported(int n_tok, int E, int k, int d, bool with_records);
void launch_route_dispatch(const float* logits, int n_tok, int E, int k, int norm_topk, float weights_scale, int* ids,
                           float* w, const DispatchOut& o, const float* x, int d, uint8_t* rec, cudaStream_t st,
                           bool rows = false);
// Metadata of a dense product: one group of n rows, slots = rows 0..n-1
// (rows: groups of at most three rows, all on the int8 path).
void launch_dense_meta(int n, const DispatchOut& o, cudaStream_t st, bool rows = false);
void launch_combine(const float* y, const int* tok_slot, const int* ids, const float* w, int n_tok, int k, int d,
                    float* out, cudaStream_t st);

// grouped.cu
int launch_grouped_f32(const GroupedArgs& a, bool pair, int max_experts, int max_rows_per_expert,
                       cudaStream_t st);

int num_sms();

}  // namespace kc
