// Decode attention over a progressive-quantised KV cache (decode.cu).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace spatten {

struct DecodeParams {
  int dtype;               // of v and out (kF16 / kBF16)
  int B, H, G, N, D;       // batch, query heads, KV heads, cache length, head dim
  int n_valid;             // keys 0 .. n_valid-1 of the cache hold data
  const int8_t* q8;        // [B, H, D]
  const float* q_scale;    // [B, H]
  const uint8_t* k_msb;    // [B, G, N, D/2]
  const uint8_t* k_lsb;    // [B, G, N, D/2]
  const float* k_scale;    // [B, G, N]
  const void* v;           // [B, G, N, D]
  float sm_scale;
  float* importance;       // [B, N]
  int top_k;
  const int64_t* kept;     // [B, top_k]
  void* out;               // [B, H, D]
};

struct DecodeWorkspace {
  float* scores;  // [B, H, N]
  float* part;    // [B, H, chunks, 2]
  float* st;      // [B, H, 2]
  float* ml;      // [B, H, splits, 2]
  float* o;       // [B, H, splits, D]
};

struct DecodeWorkspaceSizes {
  size_t scores, part, st, ml, o;
};

DecodeWorkspaceSizes decode_workspace_sizes(const DecodeParams& p);
cudaError_t launch_decode_importance(const DecodeParams& p, const DecodeWorkspace& w, cudaStream_t st);
cudaError_t launch_decode_attend(const DecodeParams& p, const DecodeWorkspace& w, cudaStream_t st);

}  // namespace spatten
