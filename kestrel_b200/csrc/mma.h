// tcgen05 grouped GEMM (mma.cu): experts with >= 4 rows and dense n >= 4.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace kc {

struct MmaArgs {
  const uint8_t* w[2];    // gate, up (n_mat = 2) or one matrix
  int n_mat;
  int64_t expert_stride;  // device bytes of one expert's matrix
  int expert_base;
  const int* slot;        // host-streamed experts: slot of expert e (null: e - expert_base)
  int rows, cols, type;
  const int* list;        // experts to process
  const int* n_list;      // device scalar
  const int* offsets;     // [E+1] slot ranges
  const int* tt_prefix;   // [n_list+1]: prefix of ceil(rows_e / kMmaTileN) token tiles
  float* out[2];          // out[m][slot * out_stride + row]
  int64_t out_stride;
  int* status;
  // Split-K workspace (null: no split): f32 partial tiles for up to gridDim
  // work items ([item][n_mat][128 x kMmaTileN]) and per-tile arrival counters
  // (zero before the first launch; each launch leaves them zero).
  float* part;
  int* tile_cnt;
  // Prefer items of one matrix x two 256-slot tiles (each weight block
  // dequantised once for up to 512 slots) over gate+up pairs x one tile: set
  // when experts are expected to hold more than 256 rows.
  int wide;
  // Most slots any tile of the launch holds (0: 256): sizes the activation
  // part of each operand stage, so that small tiles leave room for more
  // stages. A tile above it is reported as KC_ERR_SHAPE.
  int bn;
  // Every weight block is read by one work item only (no expert holds more
  // than one slot tile): the raw copies then carry an L2 evict_first hint.
  int read_once;
};
// Bytes of the split-K workspace a launch may use: partial tiles for one work
// item per SM, and one counter per SM.
size_t mma_part_bytes();
size_t mma_cnt_bytes();

// CUtensorMaps (128 bytes each) of an f16 row-major [rows, cols] activation
// matrix, 128B swizzle, boxes of 64 columns x 16, 32, 64, 128 and 256 rows: a
// work tile loads the smallest box that holds its slots.
constexpr int kMmaBoxes = 5;
struct MmaMaps {
  alignas(64) unsigned char m[kMmaBoxes][128];
};
int make_tmaps_f16(MmaMaps& maps, const void* ptr, int64_t rows, int64_t cols);
bool mma_supported(int t, int64_t cols, int n_mat);
// max_ctas > 0: at most that many CTAs (the kernel splits K over what it gets).
int launch_mma_grouped(const MmaArgs& a, const MmaMaps& maps, int max_tiles, cudaStream_t st, int max_ctas = 0);

}  // namespace kc
