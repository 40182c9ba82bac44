// Internal launcher declarations (host side) shared by the C-ABI layer.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace spatten {

// Device-side view of spatten_prog_attn_args plus the workspace layout.
struct AttnParams {
  int mode, dtype;
  int Z, H, Hkv, M, N, D;
  const void* q;
  int64_t q_sz, q_sh, q_sm;
  const float* q_scale;
  const void* k0;
  const void* k1;
  int64_t k_sz, k_sh, k_sn;
  const float* k_scale;
  const void* v;
  int64_t v_sz, v_sh, v_sn;
  void* out;
  int64_t o_sz, o_sh, o_sm;
  const int32_t* out_head_map;
  int out_head_slots;
  const float* bias;
  int64_t b_sz, b_sh, b_sm, b_sn;
  float sm_scale, refetch_thr, v_thr;
  int tile_m, tile_n;
  float tile_thr;
  int causal;
  int v_count;          // count V prune: zero the v_count smallest p of each row (0: off)
  const int32_t* key_limit;  // [Z, M]: row m sees keys n < key_limit[z*M+m] (null: causal / all)
  uint8_t* refetch_out;
  int32_t* score_out;   // [Z, H, ceil(M / score_rs), N]: rows m % score_rs == 0
  int score_rs;
  // workspace (per-CTA partial sums, reduced by importance_reduce)
  int mtiles;           // query tiles per (z, h)
  float* tok_partial;   // [Z, H, mtiles, N] or null
  float* head_partial;  // [Z, H, mtiles] or null
};

cudaError_t launch_quant(int dtype, bool planes, const void* x, int Z, int H, int M, int D,
                         int64_t sz, int64_t sh, int64_t sm, int8_t* q8, uint8_t* msb,
                         uint8_t* lsb, float* scale, cudaStream_t st, int n_sm);

// Largest count of the count V prune (smallest probabilities kept per thread).
constexpr int kMaxVPruneCount = 16;

// Rows of queries per CTA of the attention kernel (granularity of partials).
int attn_tile_rows(const AttnParams& p);
cudaError_t launch_prog_attn(const AttnParams& p, cudaStream_t st, int n_sm);
// tcgen05 kernel (QUANT, DENSE and COMPAT modes, fp16 / bf16)
int tc_tile_rows();
cudaError_t launch_prog_attn_tc(const AttnParams& p, cudaStream_t st);
// SIMT kernel for fp32 tensors (QUANT and DENSE modes, N <= f32_max_keys())
int f32_tile_rows();
int f32_max_keys();
cudaError_t launch_prog_attn_f32(const AttnParams& p, cudaStream_t st);
// device error word written by a kernel whose bounded wait ran out
cudaError_t read_device_error(unsigned int* code, bool reset);

// Record `msg` as the calling thread's spatten_last_error() and return `code`.
int set_last_error(int code, const char* msg);

cudaError_t launch_importance_reduce(const float* tok_partial, const float* head_partial, int Z,
                                     int H, int mtiles, int N, const float* tok_in,
                                     float* tok_out, float* head_out, cudaStream_t st);

cudaError_t launch_topk(const float* x, int rows, int n, int64_t row_stride, int k,
                        int64_t* out, cudaStream_t st);

cudaError_t launch_gather(const void* src, int64_t src_b, int64_t src_r, const int64_t* idx,
                          int64_t idx_b, int B, int K, int rows_per_idx, int64_t idx_scale,
                          int64_t row_bytes, void* dst, int64_t dst_b, int64_t dst_r,
                          cudaStream_t st, int n_sm, int64_t src_rows);

// Head importance scaling + top-k + next active heads (heads.cu); cur <= 1024.
cudaError_t launch_select_heads(const float* imp_in, float scale, const int64_t* heads, int cur, int keep,
                                float* imp_out, int64_t* next_heads, int32_t* next_heads32, cudaStream_t st);

// Residual add + LayerNorm over rows of n features (layernorm.cu).
bool add_layer_norm_supported(int n);
cudaError_t launch_add_layer_norm(const void* x, const void* res, const void* gamma, const void* beta,
                                  void* y, int64_t rows, int n, int64_t xs, int64_t rs, int64_t ys,
                                  int dtype, float eps, int n_sm, cudaStream_t st);

// Per-head RMSNorm + rotary embedding of Q and K, Q quantised (qk_prep.cu).
struct QkPrepParams {
  int dtype;                 // kF16 / kBF16: projections, weights, cos / sin, outputs
  int B, S, Hq, Hk, D;       // tokens t = b * S + s
  const void* q;             // [T, >= Hq * D] rows, row stride q_st elements
  int64_t q_st;
  const void* k;             // [T, >= Hk * D] rows, row stride k_st
  int64_t k_st;
  const void* q_w;           // [D] query norm weight
  const void* k_w;           // [D] key norm weight
  float eps;
  const void* cos;           // [B, S, D] element strides cs_sb, cs_ss (last dim contiguous)
  const void* sin;
  int64_t cs_sb, cs_ss;
  void* k_out;               // [T, Hk * D] rows, stride ko_st
  int64_t ko_st;
  void* q_out;               // [T, Hq * D] rows, stride qo_st, or null
  int64_t qo_st;
  int8_t* q8;                // [B, Hq, S, D] or null
  float* q_scale;            // [B, Hq, S]
};
cudaError_t launch_qk_prep(const QkPrepParams& p, cudaStream_t st);

}  // namespace spatten
