// GGUF / KGUF model loading (loader.cu).
#pragma once

#include <stdint.h>

#include <string>

namespace kc {

// The context's upload entry points, called by gguf_load in file order.
struct LoadSink {
  void* ctx;
  int (*model_init)(void*, int, int, int, int, int, int, int, int, float, float, int);
  int (*model_tensor)(void*, int, int, int, const void*, int64_t, int64_t);
  int (*experts)(void*, int, int, int, int, int, const void*, int, const void*, int, const void*);
  int (*router)(void*, int, const float*, int, int, int, int, float);
  int (*shared)(void*, int, int, int, int, const void*, int, const void*, int, const void*, const float*);
  int64_t (*device_bytes_of)(int t, int64_t rows, int64_t cols);
};

// Parse `path` into a JSON description (no GPU).
int gguf_inspect(const char* path, std::string& json, std::string& err);
// Check that the model fits in free HBM, then declare and upload it.
int gguf_load(const char* path, int n_ctx, const LoadSink& sink, std::string& err, std::string& info);

}  // namespace kc
