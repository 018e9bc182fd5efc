// Decode-sized grouped dequant-dot (decode.cu) and its activation records.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace kc {

// Activation records, one per (superblock, slot).
//   Q8_K record (K-quant weights), 320 B: q[256] int8 | bsums int16[16] at 256
//     | pair sums int16[8] at 288 (bsums[2i] + bsums[2i+1]) | d f32 at 304
//   Q8 record (Q8_0 weights), per chunk of 8 blocks, 288 B: q[256] | d[8] f32
// Q8_K records are stored by superblock pairs: record (sb, slot) is number
// ((sb / 2) * rec_slots + slot) * 2 + sb % 2 (rec_index), so the records of an
// expert's consecutive slots for the two superblocks of a decode stage are one
// contiguous range. Q8 records are stored chunk-major: number
// chunk * rec_slots + slot.
constexpr int kRecK = 320;
constexpr int kRecQ8 = 288;
inline int rec_bytes_of(bool kquant) { return kquant ? kRecK : kRecQ8; }
__host__ __device__ __forceinline__ int64_t rec_index(int64_t sb, int64_t slot, int64_t rec_slots) {
  return ((sb >> 1) * rec_slots + slot) * 2 + (sb & 1);
}
// Records per slot of a row of `cols` values (Q8_K: superblocks rounded up to
// a pair).
inline int64_t rec_row_bytes(bool kquant, int64_t cols) {
  return kquant ? (cols / 256 + 1) / 2 * 2 * kRecK : (cols / 32 + 7) / 8 * kRecQ8;
}

struct DecodeArgs {
  const uint8_t* w[2];     // matrices (gate, up) or (down / dense, unused)
  int n_mat;               // 1 or 2
  int64_t expert_stride;   // bytes between experts' matrices
  int expert_base;         // global id of the first expert held
  // Host-streamed experts: expert e's matrices are at slot[e - expert_base]
  // * expert_stride (null: at e - expert_base).
  const int* slot;
  int rows, cols;          // one expert's matrix
  int type;                // KC_Q4_K / KC_Q6_K / KC_Q8_0
  const int* list;         // expert ids (1..3 rows each; e | part << 16, see meta_at)
  const int* n_list;       // device scalar
  const int* offsets;      // [n_experts + 1] slot ranges
  int n_experts;           // entries of offsets minus one (<= 1024)
  const uint8_t* rec;      // activation records (layout above)
  int64_t rec_slots;       // slots per superblock (pair) plane of rec
  float* out[2];           // out[m][slot * out_stride + row]
  int64_t out_stride;
  int* status;
  // The list, n_list and offsets were written before the previous kernel in
  // the stream (only rec comes from it): weights stream before the wait.
  bool early;
  // Units ordered tile by tile over the list entries (n_mat 1, all entries on
  // one matrix: expert_stride 0) rather than entry by entry.
  bool tile_major;
};

// Stage geometry of one weight type / row length (decode.cu).
struct DecodeGeom {
  int type;
  int nsb;       // superblocks per row (Q8_0: chunks of 8 blocks)
  int nb32;      // Q8_0 blocks per row
  int ks;        // superblocks per K segment (one pipeline stage)
  int nseg;      // segments per row
  int64_t tile_bytes;  // bytes of one 32-row tile
  int rec_off;         // weight bytes of the largest segment, rounded to 128:
                       // the stage's activation records start there
  int stage_bytes;     // rec_off + ks superblocks x 3 slots of records, rounded to 128
};

// K-quant superblocks per decode stage (even: a stage's records are whole
// superblock pairs): the weight bytes of one stage are 32 rows x kStageSB
// superblocks (fewer when the row has fewer), one bulk copy.
#ifndef KC_DECODE_STAGE_SB
#define KC_DECODE_STAGE_SB 4
#endif
constexpr int kStageSB = KC_DECODE_STAGE_SB;
static_assert(kStageSB >= 2 && kStageSB % 2 == 0, "stages hold whole superblock pairs");
DecodeGeom decode_geom(int t, int64_t cols);
// The geometry with ks superblocks per stage (1 for Q8_0; even or the whole
// row for K-quants).
DecodeGeom decode_geom_ks(int t, int64_t cols, int ks);
// max_units: an upper bound of the work units (expert x matrix x 32-row tile)
// used to size the grid; max_ctas (> 0) caps it below the SM count.
int launch_decode(const DecodeArgs& a, int max_units, cudaStream_t st, int max_ctas = 0);

// Activation records of `n_slots` rows: slot i reads row slot_src[i] of x (i
// when slot_src is null). With u != null the rows are first combined as
// SwiGLU g / (1 + exp(-g)) * u (x = g, both indexed by slot). Any of rec,
// f32out (SwiGLU only) and f16out may be null; f32out/f16out are written per
// slot ([n_slots, cols]).
// n_slots_dev (optional): device count of the valid slots; slots at or beyond
// it are skipped (their slot_src entries may be stale).
void launch_act_records(bool kquant, const float* x, const float* u, const int* slot_src, int64_t n_slots,
                        int64_t cols, uint8_t* rec, int64_t rec_slots, float* f32out, __half* f16out,
                        cudaStream_t st, const int* n_slots_dev = nullptr);

}  // namespace kc
