// Fused Q/K/V projection with head-indexed weight tiles and the quantisation
// epilogue (qkv_proj.cu).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace spatten {

struct ProjParams {
  int dtype;           // of x, w, bias and the fp outputs (kF16 / kBF16)
  int mode;            // 0: Q -> int8 + scale, K -> 4-bit planes + scale; 1: Q, K in dtype
  int B, S;            // tokens T = B * S (row t = b * S + s of x)
  int Kdim;            // input features
  int Hall, Dh, cur;   // heads of the weight, head dim, active heads
  const void* x;       // [T, Kdim], row stride x_st elements
  int64_t x_st;
  const void* w;       // [3 * Hall * Dh, Kdim] contiguous: Q rows, then K rows, then V rows
  const void* bias;    // [3 * Hall * Dh] or null
  const int64_t* heads;  // [cur] weight head of each active slot, null = slots 0 .. cur-1
  int8_t* q8;          // mode 0: [B, cur, S, Dh]
  float* q_scale;      //         [B, cur, S]
  uint8_t* k_msb;      //         [B, cur, S, Dh/2]
  uint8_t* k_lsb;      //         [B, cur, S, Dh/2]
  float* k_scale;      //         [B, cur, S]
  void* q;             // mode 1: [B, cur, S, Dh]
  void* k;             //         [B, cur, S, Dh]
  void* v;             // [B, cur, S, Dh]
};

cudaError_t launch_qkv_proj(const ProjParams& p, cudaStream_t st);
cudaError_t read_proj_device_error(unsigned int* code, bool reset);

}  // namespace spatten
