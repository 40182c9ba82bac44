// Fused Q/K/V projection with head-indexed weight tiles and the quantisation
// epilogue (qkv_proj.cu); the attention output projection of the kept tokens
// with its residual (out_proj.cu).
#pragma once
#include <cuda.h>
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

// 2-D TMA map over a row-major [rows, inner] matrix of 16-bit elements (row
// stride in bytes), box {64, box_rows}, 128-byte swizzle.
cudaError_t make_map_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, int inner, int rows,
                        int64_t row_bytes, int box_rows);

// out[b * L + j, :] = T(T(ctx[b * S + s] . W^T + bias) + res[b * S + s]),
// s = kept[b, j]: the K columns are the active heads' blocks of the context row
struct OutProjParams {
  int dtype;               // kF16 / kBF16 (ctx, w, bias, res, out)
  int B, S, L;             // input rows b * S + s; output rows b * L + j
  int N;                   // output features, multiple of 32
  int H, Dh, cur;          // heads of the context row, head dim (multiple of 64), active heads
  const int64_t* heads;    // [cur] active heads, null = 0 .. cur-1
  const int64_t* kept;     // [B, L] kept positions
  const void* ctx;         // [B * S, >= H * Dh], row stride ctx_st elements
  int64_t ctx_st;
  const void* w;           // [N, H * Dh] contiguous
  const void* bias;        // [N] or null
  const void* res;         // [B * S, >= N], row stride res_st elements
  int64_t res_st;
  void* out;               // [B * L, N] contiguous
};

cudaError_t launch_out_proj(const OutProjParams& p, cudaStream_t st);
cudaError_t read_out_proj_device_error(unsigned int* code, bool reset);

}  // namespace spatten
