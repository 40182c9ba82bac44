/*
 * spatten_b200.h -- C ABI of the SpAtten sparse-attention hot path on B200
 * (sm_100a). Shared library: spatten_b200/lib/libspatten_b200.so
 *
 * Plain pointers, sizes and element strides only; every device pointer must
 * live on the current CUDA device, and `stream` is a cudaStream_t (NULL = the
 * legacy default stream). Calls are asynchronous on `stream` and allocate no
 * memory; where a kernel needs scratch, the caller passes a workspace whose
 * size the matching *_workspace_size() call returns.
 *
 * Every entry point returns SPATTEN_OK (0) or an error code; the message of
 * the last error on the calling thread is available from
 * spatten_last_error(). Invalid arguments are rejected before any launch.
 *
 * Reference interfaces replaced (paths within Merlin0224/SpAtten):
 *   spatten_quant_q_int8 / spatten_quant_k_planes
 *       the float K split `k_msb = key*0.8; k_lsb = key*0.2`
 *       (spatten_bert_ultimate.py:184-185), made integer.
 *   spatten_prog_attn
 *       triton_progressive_qk(q, k_msb, k_lsb, v, threshold, sm_scale)
 *       (spatten_bert_ultimate.py:103-122),
 *       spatten_progressive_attention(q, k_msb, k_lsb, v, threshold=0.1)
 *       (spatten_progressive_attention.py:82-102), and the attention core of
 *       SpattenBertSelfAttention.forward: QK^T, mask, softmax, V prune, P.V,
 *       head and token importance (spatten_bert.py:81-136).
 *   spatten_topk_indices
 *       torch.sort(torch.topk(x, k).indices) for the head and token cascade
 *       (spatten_bert.py:123-128, 143-148).
 *   spatten_gather_rows
 *       torch.gather of hidden states / cumulative scores on the token axis
 *       (module.py:53-54, 62-63) and torch.index_select of head rows of the
 *       Q/K/V weights (module.py:22-28).
 *   spatten_qkv_proj
 *       slice_linear_weights (module.py:12-34) + the Q/K/V projections of
 *       SpattenBertSelfAttention.forward (spatten_bert.py:72-78) + the K
 *       plane split (spatten_bert_ultimate.py:184-185), in one kernel.
 *   spatten_compact_out_proj
 *       the next layer's hidden-state gather (module.py:49-54) moved into the
 *       attention output projection + residual, so the FFN runs on the
 *       compacted sequence.
 *   spatten_add_layer_norm
 *       the residual add + LayerNorm of the HF BertLayer tail that the
 *       reference's encoder loop runs per layer (module.py:75).
 *   spatten_select_heads
 *       the head decision of the cascade: head importance, top-k and the
 *       next layer's active heads (spatten_bert.py:120-128, module.py:89).
 */
#ifndef SPATTEN_B200_H
#define SPATTEN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SPATTEN_OK 0
#define SPATTEN_ERR_INVALID 1     /* bad argument (shape, stride, pointer, dtype) */
#define SPATTEN_ERR_CUDA 2        /* a CUDA runtime call or launch failed */
#define SPATTEN_ERR_UNSUPPORTED 3 /* valid request outside what this library implements */

#define SPATTEN_DTYPE_F16 0
#define SPATTEN_DTYPE_BF16 1
#define SPATTEN_DTYPE_F32 2

#define SPATTEN_MODE_QUANT 0  /* int8 Q, 4-bit MSB/LSB K planes, row max-prob refetch */
#define SPATTEN_MODE_DENSE 1  /* float Q/K (progressive quantisation off) */
#define SPATTEN_MODE_COMPAT 2 /* float K planes with the reference's tile criterion (no mask) */

/* ABI version; bumped on any incompatible change of this header. */
int spatten_abi_version(void);
/* Message of the last failed call on this thread ("" if none). */
const char* spatten_last_error(void);
/* Device error word of the current device (synchronous; 0 = none). A kernel
 * whose bounded wait on a pipeline barrier runs out records a non-zero code
 * here and returns instead of hanging; `reset` clears the word. */
int spatten_device_error(unsigned int* code, int reset);

/*
 * Per-row symmetric int8 quantisation of Q.
 *   x      [Z, H, M, D] of `dtype`, element strides (sz, sh, sm), last dim contiguous
 *   q8     [Z, H, M, D] int8, contiguous
 *   scale  [Z, H, M] fp32, contiguous: scale = max|x| / 127, q8 = rint(x / scale)
 * D must be a multiple of 32 and at most 256.
 */
int spatten_quant_q_int8(const void* x, int dtype, int Z, int H, int M, int D, int64_t sz,
                         int64_t sh, int64_t sm, int8_t* q8, float* scale, void* stream);

/*
 * Per-row symmetric int8 quantisation of K, split into 4-bit planes.
 *   x      [Z, H, N, D] of `dtype`, element strides (sz, sh, sn)
 *   msb    [Z, H, N, D/2] uint8: k8 >> 4 (signed nibble), two per byte
 *   lsb    [Z, H, N, D/2] uint8: k8 & 15 (unsigned nibble), two per byte
 *   scale  [Z, H, N] fp32
 * Byte p of a packed row holds dim p (low nibble) and dim p + D/2 (high).
 */
int spatten_quant_k_planes(const void* x, int dtype, int Z, int H, int N, int D, int64_t sz,
                           int64_t sh, int64_t sn, uint8_t* msb, uint8_t* lsb, float* scale,
                           void* stream);

/* Arguments of spatten_prog_attn. Strides are in elements of the tensor's
 * own type (bytes for the packed planes); the last dimension is contiguous. */
typedef struct spatten_prog_attn_args {
  int mode;  /* SPATTEN_MODE_* */
  int dtype; /* element type of v and out (and of q / k for DENSE, COMPAT) */
  int Z, H, Hkv, M, N, D; /* batch, query heads, kv heads (H % Hkv == 0), queries, keys, head dim */

  const void* q; /* QUANT: int8 [Z,H,M,D]; else dtype */
  int64_t q_sz, q_sh, q_sm;
  const float* q_scale; /* QUANT: [Z,H,M] contiguous */

  const void* k0; /* QUANT: msb plane; DENSE: k; COMPAT: k_msb */
  const void* k1; /* QUANT: lsb plane; DENSE: unused; COMPAT: k_lsb */
  int64_t k_sz, k_sh, k_sn; /* shared by k0 and k1 */
  const float* k_scale;     /* QUANT: [Z,Hkv,N] contiguous */

  const void* v;
  int64_t v_sz, v_sh, v_sn;

  void* out; /* [Z, H, M, D] by strides; head h goes to slot out_head_map[h] if given */
  int64_t o_sz, o_sh, o_sm;
  const int32_t* out_head_map; /* optional device array [H] of slots in [0, out_head_slots) */
  int out_head_slots;          /* number of head slots of `out` (0 = H); a slot outside
                                  [0, out_head_slots) is not written */

  const float* bias; /* optional additive fp32 bias, element (z,h,m,n) at
                        z*b_sz + h*b_sh + m*b_sm + n*b_sn (0 strides broadcast) */
  int64_t b_sz, b_sh, b_sm, b_sn;

  float sm_scale;
  float refetch_thr; /* QUANT: refetch the LSB plane of a row when 1/l_msb < thr */
  float v_thr;       /* V prune: p < v_thr -> 0 (0 disables) */
  int tile_m, tile_n; /* COMPAT: criterion tile (32 or 64 each) */
  float tile_thr;     /* COMPAT: refetch a tile when max(q.k_msb*sm_scale) < tile_thr */
  int causal;         /* mask key n > m + (N - M) */

  float* tok_out;      /* optional [Z, N]: sum over heads and queries of pruned P */
  const float* tok_in; /* optional [Z, N]: added to tok_out (cumulative score) */
  float* head_out;     /* optional [H]: sum over (z, m, d) of |out| */
  uint8_t* refetch_out; /* optional QUANT [Z, H, M]: 1 where the row was refetched */
  int32_t* score_out;   /* optional QUANT [Z, H, M, N]: the exact integer score each row used,
                           q8.(16*msb) or, for a refetched row, q8.k8 (for verification) */
  int v_prune_count; /* count V prune (the reference's v_prune_num, spatten_bert.py:100-113):
                        in rows of more than v_prune_count keys, zero the v_prune_count
                        smallest probabilities (ties to the smaller key index), no
                        renormalisation; 0 disables, at most 16; QUANT and DENSE only.
                        Applies together with v_thr. (ABI version 2) */
  const int32_t* key_limit; /* optional [Z, M] int32, QUANT and DENSE: row m of batch z sees
                               keys n < key_limit[z*M + m] only (the causal mask of a
                               position-sorted subset of keys, e.g. a pruned KV cache);
                               replaces `causal` when set. (ABI version 3) */
  int score_row_stride; /* with score_out: write the scores of rows m % score_row_stride == 0
                           only, row m at row m / score_row_stride of a
                           [Z, H, ceil(M / score_row_stride), N] array (0 or 1: every row),
                           so a full-size launch can be verified from a sample of its rows
                           without a [Z, H, M, N] dump. (ABI version 4) */
} spatten_prog_attn_args;

/* Bytes of workspace spatten_prog_attn needs for these arguments (0 if no
 * importance output is requested). */
size_t spatten_prog_attn_workspace_size(const spatten_prog_attn_args* a);

/* Progressive sparse attention; see spatten_prog_attn_args. `workspace` must
 * hold spatten_prog_attn_workspace_size(a) bytes (256-byte aligned). */
int spatten_prog_attn(const spatten_prog_attn_args* a, void* workspace, size_t workspace_bytes,
                      void* stream);

/*
 * Allocation-free spatten_prog_attn, for callers that cannot call cudaMalloc:
 * hosts that fix their device-memory budget at start-up and forbid allocation
 * afterwards, and plugins limited to the memory their host hands them. No
 * counterpart in the reference, which has no C interface.
 *
 * The workspace comes from a fixed array of
 * spatten_prog_attn_noalloc_capacity() bytes (16 MiB) in device memory,
 * reserved on a GPU when the library's device code is loaded there (under
 * CUDA's lazy module loading: at the first use of one of its kernels, which
 * may be this call) and held until the process exits; a request needing more
 * (spatten_prog_attn_workspace_size) fails with SPATTEN_ERR_INVALID. Calls on
 * one device share the array: calls that may overlap on the GPU race, so
 * order them on one stream. Each call looks up the array's address on the
 * current device; the first call on a device may load the module there, so
 * make it before any stream capture.
 */
size_t spatten_prog_attn_noalloc_capacity(void);
int spatten_prog_attn_noalloc(const spatten_prog_attn_args* a, void* stream);

/*
 * Decode attention over a progressive-quantised KV cache with top-k token
 * selection: one new query per sequence, GQA (H query heads share G KV heads,
 * H / G in {1, 2, 4, 8}), D in {64, 128}. The cache is the prefill format: K
 * as packed 4-bit MSB / LSB planes [B, G, N, D/2] uint8 (byte p = dim p |
 * dim p+D/2 << 4) with a per-key fp32 scale [B, G, N], V [B, G, N, D]
 * fp16/bf16; keys 0 .. n_valid-1 hold data. Per step:
 *   spatten_decode_importance: MSB scores q8 . 16*msb of every valid key
 *     (only the MSB plane of the cache is read), softmax of every head over
 *     the keys, importance[b, n] = sum over the H heads of those
 *     probabilities (0 for n >= n_valid). With the KV heads split over ranks
 *     each rank sums its own heads; all-reduce before the top-k.
 *   spatten_topk_indices(importance, B, N, N, top_k, kept): the kept keys.
 *   spatten_decode_attend: exact int8 scores q8 . k8 over the kept keys
 *     (their LSB planes only), softmax, P.V -> out [B, H, D].
 * This is SpAtten's cascade token pruning applied to decoding: the token
 * importance of spatten_bert.py:136-150 over the cache, its top-k kept
 * (spatten_bert.py:143-148), and progressive quantisation's LSB fetched for
 * the kept keys only (spatten_bert_ultimate.py:58-74).
 */
typedef struct {
  int dtype;              /* SPATTEN_DTYPE_F16 or _BF16: v and out */
  int B, H, G, N, D;      /* batch, query heads, KV heads, cache length, head dim */
  int n_valid;            /* 1 <= n_valid <= N */
  const int8_t* q8;       /* [B, H, D] contiguous (spatten_quant_q_int8 of the query) */
  const float* q_scale;   /* [B, H] */
  const uint8_t* k_msb;   /* [B, G, N, D/2] contiguous */
  const uint8_t* k_lsb;   /* [B, G, N, D/2] contiguous (attend) */
  const float* k_scale;   /* [B, G, N] */
  const void* v;          /* [B, G, N, D] contiguous (attend) */
  float sm_scale;
  float* importance;      /* [B, N] fp32 out (importance) */
  int top_k;              /* kept keys per sequence (attend; sizes the workspace) */
  const int64_t* kept;    /* [B, top_k] key indices (attend; out-of-range entries are skipped) */
  void* out;              /* [B, H, D] out, dtype (attend) */
} spatten_decode_args;

/* Bytes of workspace both decode calls need (256-byte aligned). */
size_t spatten_decode_workspace_size(const spatten_decode_args* a);
int spatten_decode_importance(const spatten_decode_args* a, void* workspace, size_t workspace_bytes,
                              void* stream);
int spatten_decode_attend(const spatten_decode_args* a, void* workspace, size_t workspace_bytes,
                          void* stream);

/*
 * Fused Q/K/V projection of the active heads, with the quantisation the
 * attention kernel reads. Replaces, per layer of the cascade:
 *   slice_linear_weights (module.py:12-34): index_select of the active heads'
 *     rows of W_q, W_k, W_v and their biases -- no copy here: the weight
 *     tiles are loaded from the full weight at the active heads' rows;
 *   the projections q/k/v = F.linear(hidden, W_sliced, b_sliced)
 *     (spatten_bert.py:72-78);
 *   the K plane split (spatten_bert_ultimate.py:184-185), made integer, and
 *     the int8 query, as spatten_quant_q_int8 / spatten_quant_k_planes would
 *     compute them from the rounded projections.
 * x [B*S, Kdim] (row t = b*S + s, row stride x_row_stride elements); w
 * [3*Hall*Dh, Kdim] contiguous, the Q rows, then the K rows, then the V rows
 * (nn.Linear layout, the reference's query/key/value weights stacked); bias
 * [3*Hall*Dh] or NULL; heads [cur] int64 weight head of each active slot
 * (NULL: 0 .. cur-1). dtype f16 or bf16 for x, w, bias and the fp outputs.
 * Outputs are head-major, [B, cur, S, ...] contiguous:
 *   mode SPATTEN_PROJ_QUANT: q8 [.., Dh] int8 + q_scale [B, cur, S];
 *     k_msb, k_lsb [.., Dh/2] + k_scale [B, cur, S]; v [.., Dh];
 *   mode SPATTEN_PROJ_DENSE: q, k, v [.., Dh].
 * Dh in {64, 128}; Kdim a multiple of 8; x, w and every output 16-byte
 * aligned. The GEMM accumulates in fp32 on the tensor cores, adds the bias
 * and rounds to dtype before quantising (the values an unfused projection
 * stores; its accumulation order may differ in the last bit).
 */
#define SPATTEN_PROJ_QUANT 0
#define SPATTEN_PROJ_DENSE 1
typedef struct {
  int dtype;
  int mode;
  int B, S, Kdim;
  int Hall, Dh, cur;
  const void* x;
  int64_t x_row_stride;
  const void* w;
  const void* bias;
  const int64_t* heads;
  int8_t* q8;
  float* q_scale;
  uint8_t* k_msb;
  uint8_t* k_lsb;
  float* k_scale;
  void* q;
  void* k;
  void* v;
} spatten_qkv_proj_args;

int spatten_qkv_proj(const spatten_qkv_proj_args* a, void* stream);

/*
 * Per-head RMSNorm (QK-norm) + rotary position embedding of the query and key
 * projections, the query quantised to int8. No reference code (the reference
 * has no Qwen3 path): replaces, inside the Qwen3 drop-in, the HF modules'
 * q_norm / k_norm (Qwen3RMSNorm) and apply_rotary_pos_emb
 * (transformers/models/qwen3/modeling_qwen3.py) and the query's
 * spatten_quant_q_int8, with the HF arithmetic step for step: for each head
 * row x, y = T(x * rsqrtf(mean(x^2) + eps)), n = T(w * y),
 * out = T(T(n * cos) + T(rotate_half(n) * sin)) (T: rounding to dtype; the
 * sum of squares is taken in this kernel's own order), then Q's int8 rows
 * as spatten_quant_q_int8 computes them.
 * q [B*S, >= Hq*D], k [B*S, >= Hk*D] (row t = b*S + s, row strides in
 * elements); q_norm_w, k_norm_w [D]; cos, sin [B, S, D] (element strides
 * cs_b_stride, cs_s_stride). Outputs: k_out [B*S, Hk*D] rows (token-major,
 * like the HF key states); q_out (same layout, optional) and / or q8
 * [B, Hq, S, D] int8 + q_scale [B, Hq, S]. D in {64, 128}; dtype f16 / bf16;
 * pointers 16-byte aligned, strides multiples of 8 elements.
 */
typedef struct {
  int dtype;
  int B, S, Hq, Hk, D;
  const void* q;
  int64_t q_row_stride;
  const void* k;
  int64_t k_row_stride;
  const void* q_norm_w;
  const void* k_norm_w;
  float eps;
  const void* cos;
  const void* sin;
  int64_t cs_b_stride, cs_s_stride;
  void* k_out;
  int64_t k_out_row_stride;
  void* q_out;
  int64_t q_out_row_stride;
  int8_t* q8;
  float* q_scale;
} spatten_qk_norm_rope_args;

int spatten_qk_norm_rope(const spatten_qk_norm_rope_args* a, void* stream);

/*
 * Attention output projection + residual of the kept tokens only (the token
 * gather of the cascade folded into the GEMM's row loads). Replaces, for a
 * layer whose attention chose the tokens the next layer keeps, the gather of
 * the next layer's hidden states (module.py:49-54, torch.gather) moved ahead
 * of the first row-wise step after the attention, HF BertSelfOutput's
 * dense + residual add (transformers/models/bert/modeling_bert.py), so the
 * LayerNorm and the FFN that follow run on the compacted sequence:
 *   out[b*L + j, :] = T(T(ctx[b*S + s, :] . w^T + bias) + res[b*S + s, :]),
 *   s = kept[b, j]
 * (T: rounding to dtype). The dot product runs over the active heads'
 * column blocks of the context row only (heads[cur], null = 0 .. cur-1; the
 * other heads' blocks are zeros in the drop-in's context). ctx
 * [B*S, >= H*head_dim] and res [B*S, >= N] with row strides in elements; w
 * [N, H*head_dim] (nn.Linear layout) contiguous; bias [N] or null; kept
 * int64 [B, L] (positions outside [0, S) are clamped); out [B*L, N]
 * contiguous. dtype f16 / bf16; head_dim a multiple of 64; N a multiple of
 * 32; pointers 16-byte aligned; strides multiples of 8 elements.
 */
typedef struct {
  int dtype;
  int B, S, L, N;
  int H, head_dim, cur;
  const int64_t* heads;
  const int64_t* kept;
  const void* ctx;
  int64_t ctx_row_stride;
  const void* w;
  const void* bias;
  const void* res;
  int64_t res_row_stride;
  void* out;
} spatten_compact_out_proj_args;

int spatten_compact_out_proj(const spatten_compact_out_proj_args* a, void* stream);

/*
 * Top-k selection, indices returned in ascending order:
 *   out[r, :] = sort(topk(x[r, :n], k).indices), r < rows
 * Ties at the k-th value go to the smaller index. x fp32 with row stride
 * `x_row_stride` (elements); out int64 [rows, k] contiguous.
 */
int spatten_topk_indices(const float* x, int rows, int n, int64_t x_row_stride, int k,
                         int64_t* out, void* stream);

/*
 * Row gather (stream compaction):
 *   dst[b, i*rows_per_idx + j, :] = src[b, idx[b, i] * idx_scale + j, :]
 * for j < rows_per_idx, as raw bytes: row_bytes per row, strides in bytes
 * (batch, row). src holds src_rows rows per batch; a source row outside
 * [0, src_rows) zero-fills its destination row. idx int64 [B, K] with row
 * stride idx_b_stride (0 = one index list shared by all batches).
 */
int spatten_gather_rows(const void* src, int64_t src_b_stride, int64_t src_r_stride,
                        int64_t src_rows, const int64_t* idx, int64_t idx_b_stride, int B, int K,
                        int rows_per_idx,
                        int64_t idx_scale, int64_t row_bytes, void* dst, int64_t dst_b_stride,
                        int64_t dst_r_stride, void* stream);

/*
 * Residual add + LayerNorm over rows of n features (f16 / bf16):
 *   h = x + res (rounded to the element type; res may be NULL),
 *   y = (h - mean(h)) / sqrt(var(h) + eps) * gamma + beta
 * with the mean and the biased variance in fp32. Replaces, in the tail of
 * the HF BertLayer that the reference's encoder loop runs for every layer
 * (module.py:75), torch's add + layer_norm of BertOutput and the layer_norm
 * of BertSelfOutput (after spatten_compact_out_proj). Row strides in
 * elements; every row, gamma and beta start on a 16-byte boundary; n one of
 * 256, 512, 768, 1024, 1536, 2048 (SPATTEN_ERR_UNSUPPORTED otherwise).
 */
int spatten_add_layer_norm(const void* x, int64_t x_row_stride, const void* res, int64_t res_row_stride,
                           const void* gamma, const void* beta, void* y, int64_t y_row_stride,
                           int64_t rows, int n, int dtype, float eps, void* stream);

/*
 * Head decision of one cascade layer, one launch:
 *   importance_out[i] = importance[i] * scale            (i < cur; optional, may be `importance`)
 *   pos = ascending positions of the `keep` largest importance_out values
 *         (ties at the k-th value to the smaller position, as spatten_topk_indices)
 *   next_heads[j] = heads ? heads[pos[j]] : pos[j]       (int64 [keep])
 *   next_heads32[j] = the same as int32                  (optional)
 * Replaces `head_importance / count`, torch.topk + sort and the index of the
 * active head list (spatten_bert.py:120-128, module.py:89). 1 <= keep <= cur
 * <= 1024; all pointers on the device.
 */
int spatten_select_heads(const float* importance, float scale, const int64_t* heads, int cur, int keep,
                         float* importance_out, int64_t* next_heads, int32_t* next_heads32, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPATTEN_B200_H */
