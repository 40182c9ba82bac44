// extern "C" entry points of libspatten_b200.so (declared in include/spatten_b200.h).
//
// Every call validates its arguments on the host before any launch, records
// a message for spatten_last_error() and returns an error code; nothing here
// synchronises the stream or allocates device memory.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/spatten_b200.h"
#include "common.cuh"
#include "decode.h"
#include "kernels.h"
#include "proj.h"

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int ok() {
  g_err.clear();
  return SPATTEN_OK;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return fail(SPATTEN_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return ok();
}

int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

int esize(int dtype) { return dtype == SPATTEN_DTYPE_F32 ? 4 : 2; }

bool aligned(const void* p, int a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
bool smul(int64_t s, int64_t esz, int a) { return (s * esz) % a == 0; }

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

int check_quant_args(const void* x, int dtype, int Z, int H, int M, int D, int64_t s0,
                     int64_t s1, int64_t s2) {
  if (!x) return fail(SPATTEN_ERR_INVALID, "quant: null input");
  if (dtype < 0 || dtype > 2) return fail(SPATTEN_ERR_INVALID, "quant: bad dtype %d", dtype);
  if (Z < 0 || H < 0 || M < 0) return fail(SPATTEN_ERR_INVALID, "quant: negative shape");
  if (!(D == 32 || D == 64 || D == 128 || D == 256))
    return fail(SPATTEN_ERR_UNSUPPORTED, "quant: D=%d (need 32, 64, 128 or 256)", D);
  if (s0 < 0 || s1 < 0 || s2 < 0) return fail(SPATTEN_ERR_INVALID, "quant: negative stride");
  return SPATTEN_OK;
}

}  // namespace

int spatten::set_last_error(int code, const char* msg) {
  g_err = msg ? msg : "";
  return code;
}

extern "C" {

int spatten_abi_version(void) { return 4; }

const char* spatten_last_error(void) { return g_err.c_str(); }

int spatten_device_error(unsigned int* code, int reset) {
  if (!code) return fail(SPATTEN_ERR_INVALID, "device_error: null output");
  unsigned int proj = 0, out = 0;
  if (int e = cuda_status(spatten::read_device_error(code, reset != 0), "device_error read")) return e;
  if (int e = cuda_status(spatten::read_proj_device_error(&proj, reset != 0), "device_error read")) return e;
  if (int e = cuda_status(spatten::read_out_proj_device_error(&out, reset != 0), "device_error read")) return e;
  if (*code == 0) *code = proj;
  if (*code == 0) *code = out;
  return ok();
}

int spatten_quant_q_int8(const void* x, int dtype, int Z, int H, int M, int D, int64_t sz,
                         int64_t sh, int64_t sm, int8_t* q8, float* scale, void* stream) {
  if (int e = check_quant_args(x, dtype, Z, H, M, D, sz, sh, sm)) return e;
  if (!q8 || !scale) return fail(SPATTEN_ERR_INVALID, "quant_q_int8: null output");
  if ((int64_t)Z * H * M == 0) return ok();
  return cuda_status(spatten::launch_quant(dtype, false, x, Z, H, M, D, sz, sh, sm, q8, nullptr,
                                           nullptr, scale, (cudaStream_t)stream, sm_count()),
                     "quant_q_int8 launch");
}

int spatten_quant_k_planes(const void* x, int dtype, int Z, int H, int N, int D, int64_t sz,
                           int64_t sh, int64_t sn, uint8_t* msb, uint8_t* lsb, float* scale,
                           void* stream) {
  if (int e = check_quant_args(x, dtype, Z, H, N, D, sz, sh, sn)) return e;
  if (!msb || !lsb || !scale) return fail(SPATTEN_ERR_INVALID, "quant_k_planes: null output");
  if ((int64_t)Z * H * N == 0) return ok();
  return cuda_status(spatten::launch_quant(dtype, true, x, Z, H, N, D, sz, sh, sn, nullptr, msb,
                                           lsb, scale, (cudaStream_t)stream, sm_count()),
                     "quant_k_planes launch");
}

static int fill_params(const spatten_prog_attn_args* a, spatten::AttnParams& p) {
  if (!a) return fail(SPATTEN_ERR_INVALID, "prog_attn: null args");
  if (a->mode < 0 || a->mode > 2) return fail(SPATTEN_ERR_INVALID, "prog_attn: bad mode %d", a->mode);
  if (a->dtype < 0 || a->dtype > 2) return fail(SPATTEN_ERR_INVALID, "prog_attn: bad dtype %d", a->dtype);
  if (a->dtype == SPATTEN_DTYPE_F32 && a->mode == SPATTEN_MODE_COMPAT)
    return fail(SPATTEN_ERR_UNSUPPORTED, "prog_attn: COMPAT takes f16/bf16 planes");
  if (a->dtype == SPATTEN_DTYPE_F32 && a->N > spatten::f32_max_keys())
    return fail(SPATTEN_ERR_UNSUPPORTED, "prog_attn: fp32 supports N <= %d keys", spatten::f32_max_keys());
  if (a->Z < 1 || a->H < 1 || a->Hkv < 1 || a->M < 1 || a->N < 1)
    return fail(SPATTEN_ERR_INVALID, "prog_attn: empty shape Z=%d H=%d Hkv=%d M=%d N=%d", a->Z,
                a->H, a->Hkv, a->M, a->N);
  if (a->H % a->Hkv) return fail(SPATTEN_ERR_INVALID, "prog_attn: H %% Hkv != 0");
  if (a->H > 65535 || a->Z > 65535) return fail(SPATTEN_ERR_UNSUPPORTED, "prog_attn: Z or H > 65535");
  if (a->D != 64 && a->D != 128) return fail(SPATTEN_ERR_UNSUPPORTED, "prog_attn: D=%d (need 64 or 128)", a->D);
  if (!a->q || !a->k0 || !a->v || !a->out) return fail(SPATTEN_ERR_INVALID, "prog_attn: null q/k/v/out");
  const bool quant = a->mode == SPATTEN_MODE_QUANT;
  if (quant && (!a->q_scale || !a->k1 || !a->k_scale))
    return fail(SPATTEN_ERR_INVALID, "prog_attn: QUANT needs q_scale, lsb plane and k_scale");
  if (a->mode == SPATTEN_MODE_COMPAT && !a->k1) return fail(SPATTEN_ERR_INVALID, "prog_attn: COMPAT needs k_lsb");
  if (a->mode == SPATTEN_MODE_COMPAT &&
      !((a->tile_m == 32 || a->tile_m == 64) && (a->tile_n == 32 || a->tile_n == 64)))
    return fail(SPATTEN_ERR_UNSUPPORTED, "prog_attn: COMPAT tile %dx%d (need 32/64)", a->tile_m, a->tile_n);
  const int es = esize(a->dtype);
  const int qes = quant ? 1 : es;
  const int kes = quant ? 1 : es;
  // q: 4-byte fragment loads
  if (!aligned(a->q, 4) || !smul(a->q_sz, qes, 4) || !smul(a->q_sh, qes, 4) || !smul(a->q_sm, qes, 4))
    return fail(SPATTEN_ERR_INVALID, "prog_attn: q pointer/strides not 4-byte aligned");
  // k planes / k, v: 16-byte cp.async rows
  if (!aligned(a->k0, 16) || (a->k1 && !aligned(a->k1, 16)) || !smul(a->k_sz, kes, 16) ||
      !smul(a->k_sh, kes, 16) || !smul(a->k_sn, kes, 16))
    return fail(SPATTEN_ERR_INVALID, "prog_attn: k pointer/strides not 16-byte aligned");
  if (!aligned(a->v, 16) || !smul(a->v_sz, es, 16) || !smul(a->v_sh, es, 16) || !smul(a->v_sn, es, 16))
    return fail(SPATTEN_ERR_INVALID, "prog_attn: v pointer/strides not 16-byte aligned");
  if (!aligned(a->out, 4) || !smul(a->o_sz, es, 4) || !smul(a->o_sh, es, 4) || !smul(a->o_sm, es, 4))
    return fail(SPATTEN_ERR_INVALID, "prog_attn: out pointer/strides not 4-byte aligned");
  if (a->bias && !aligned(a->bias, 4)) return fail(SPATTEN_ERR_INVALID, "prog_attn: bias not aligned");
  if (a->q_scale && !aligned(a->q_scale, 4)) return fail(SPATTEN_ERR_INVALID, "prog_attn: q_scale not aligned");
  if (a->k_scale && !aligned(a->k_scale, 4)) return fail(SPATTEN_ERR_INVALID, "prog_attn: k_scale not aligned");
  if (a->q_sz < 0 || a->q_sh < 0 || a->q_sm < 0 || a->k_sz < 0 || a->k_sh < 0 || a->k_sn < 0 ||
      a->v_sz < 0 || a->v_sh < 0 || a->v_sn < 0 || a->o_sz < 0 || a->o_sh < 0 || a->o_sm < 0)
    return fail(SPATTEN_ERR_INVALID, "prog_attn: negative stride");
  if (a->tok_in && !a->tok_out) return fail(SPATTEN_ERR_INVALID, "prog_attn: tok_in without tok_out");
  if (a->v_prune_count < 0) return fail(SPATTEN_ERR_INVALID, "prog_attn: negative v_prune_count");
  if (a->v_prune_count > spatten::kMaxVPruneCount)
    return fail(SPATTEN_ERR_UNSUPPORTED, "prog_attn: v_prune_count %d > %d", a->v_prune_count,
                spatten::kMaxVPruneCount);
  if (a->v_prune_count > 0 && a->mode == SPATTEN_MODE_COMPAT)
    return fail(SPATTEN_ERR_UNSUPPORTED, "prog_attn: COMPAT has no count V prune");
  if ((a->key_limit || a->bias || a->causal) && a->mode == SPATTEN_MODE_COMPAT)
    return fail(SPATTEN_ERR_UNSUPPORTED, "prog_attn: COMPAT takes no mask (the reference op has none)");
  if (a->key_limit && !aligned(a->key_limit, 4)) return fail(SPATTEN_ERR_INVALID, "prog_attn: key_limit not aligned");
  if (a->score_row_stride < 0) return fail(SPATTEN_ERR_INVALID, "prog_attn: negative score_row_stride");
  p.mode = a->mode;
  p.dtype = a->dtype;
  p.Z = a->Z; p.H = a->H; p.Hkv = a->Hkv; p.M = a->M; p.N = a->N; p.D = a->D;
  p.q = a->q; p.q_sz = a->q_sz; p.q_sh = a->q_sh; p.q_sm = a->q_sm; p.q_scale = a->q_scale;
  p.k0 = a->k0; p.k1 = a->k1; p.k_sz = a->k_sz; p.k_sh = a->k_sh; p.k_sn = a->k_sn;
  p.k_scale = a->k_scale;
  p.v = a->v; p.v_sz = a->v_sz; p.v_sh = a->v_sh; p.v_sn = a->v_sn;
  p.out = a->out; p.o_sz = a->o_sz; p.o_sh = a->o_sh; p.o_sm = a->o_sm;
  p.out_head_map = a->out_head_map;
  p.out_head_slots = a->out_head_slots > 0 ? a->out_head_slots : a->H;
  p.bias = a->bias; p.b_sz = a->b_sz; p.b_sh = a->b_sh; p.b_sm = a->b_sm; p.b_sn = a->b_sn;
  p.sm_scale = a->sm_scale; p.refetch_thr = a->refetch_thr; p.v_thr = a->v_thr;
  p.tile_m = a->tile_m; p.tile_n = a->tile_n; p.tile_thr = a->tile_thr;
  p.causal = a->causal;
  // the reference prunes only rows longer than the count (spatten_bert.py:100)
  p.v_count = a->N > a->v_prune_count ? a->v_prune_count : 0;
  p.key_limit = a->key_limit;
  if (a->key_limit) p.causal = 0;
  p.refetch_out = quant ? a->refetch_out : nullptr;
  p.score_out = quant ? a->score_out : nullptr;
  p.score_rs = a->score_row_stride > 1 ? a->score_row_stride : 1;
  const int rows = spatten::attn_tile_rows(p);
  p.mtiles = (a->M + rows - 1) / rows;
  p.tok_partial = nullptr;
  p.head_partial = nullptr;
  return SPATTEN_OK;
}

static void workspace_layout(const spatten::AttnParams& p, bool tok, bool head, size_t& tok_bytes,
                             size_t& head_bytes) {
  tok_bytes = tok ? align256((size_t)p.Z * p.H * p.mtiles * p.N * sizeof(float)) : 0;
  head_bytes = head ? align256((size_t)p.Z * p.H * p.mtiles * sizeof(float)) : 0;
}

size_t spatten_prog_attn_workspace_size(const spatten_prog_attn_args* a) {
  spatten::AttnParams p;
  if (fill_params(a, p) != SPATTEN_OK) return 0;
  size_t tb, hb;
  workspace_layout(p, a->tok_out != nullptr, a->head_out != nullptr, tb, hb);
  return tb + hb;
}

int spatten_prog_attn(const spatten_prog_attn_args* a, void* workspace, size_t workspace_bytes,
                      void* stream) {
  spatten::AttnParams p;
  if (int e = fill_params(a, p)) return e;
  size_t tb, hb;
  workspace_layout(p, a->tok_out != nullptr, a->head_out != nullptr, tb, hb);
  if (tb + hb > 0) {
    if (!workspace || workspace_bytes < tb + hb)
      return fail(SPATTEN_ERR_INVALID, "prog_attn: workspace of %zu bytes needed, %zu given",
                  tb + hb, workspace_bytes);
    if (!aligned(workspace, 256)) return fail(SPATTEN_ERR_INVALID, "prog_attn: workspace not 256-byte aligned");
    uint8_t* w = static_cast<uint8_t*>(workspace);
    if (tb) p.tok_partial = reinterpret_cast<float*>(w);
    if (hb) p.head_partial = reinterpret_cast<float*>(w + tb);
  }
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = spatten::launch_prog_attn(p, st, sm_count());
  if (e != cudaSuccess) return cuda_status(e, "prog_attn launch");
  if (tb + hb > 0) {
    e = spatten::launch_importance_reduce(p.tok_partial, p.head_partial, p.Z, p.H, p.mtiles, p.N,
                                          a->tok_in, a->tok_out, a->head_out, st);
    if (e != cudaSuccess) return cuda_status(e, "importance reduce launch");
  }
  return ok();
}

int spatten_topk_indices(const float* x, int rows, int n, int64_t x_row_stride, int k,
                         int64_t* out, void* stream) {
  if (!x || !out) return fail(SPATTEN_ERR_INVALID, "topk: null pointer");
  if (rows < 0 || n < 1 || k < 1 || k > n)
    return fail(SPATTEN_ERR_INVALID, "topk: need rows >= 0, 1 <= k <= n (rows=%d n=%d k=%d)", rows, n, k);
  if (rows > 0 && x_row_stride < n) return fail(SPATTEN_ERR_INVALID, "topk: row stride < n");
  if (rows == 0) return ok();
  return cuda_status(spatten::launch_topk(x, rows, n, x_row_stride, k, out, (cudaStream_t)stream),
                     "topk launch");
}

int spatten_gather_rows(const void* src, int64_t src_b_stride, int64_t src_r_stride,
                        int64_t src_rows, const int64_t* idx, int64_t idx_b_stride, int B, int K,
                        int rows_per_idx, int64_t idx_scale, int64_t row_bytes, void* dst,
                        int64_t dst_b_stride, int64_t dst_r_stride, void* stream) {
  if (!src || !idx || !dst) return fail(SPATTEN_ERR_INVALID, "gather: null pointer");
  if (B < 0 || K < 0 || rows_per_idx < 1 || row_bytes < 1 || src_rows < 0)
    return fail(SPATTEN_ERR_INVALID, "gather: bad sizes");
  if (src_b_stride < 0 || src_r_stride < 0 || dst_b_stride < 0 || dst_r_stride < 0 || idx_b_stride < 0)
    return fail(SPATTEN_ERR_INVALID, "gather: negative stride");
  if ((int64_t)B * K == 0) return ok();
  return cuda_status(spatten::launch_gather(src, src_b_stride, src_r_stride, idx, idx_b_stride, B,
                                            K, rows_per_idx, idx_scale, row_bytes, dst,
                                            dst_b_stride, dst_r_stride, (cudaStream_t)stream,
                                            sm_count(), src_rows),
                     "gather launch");
}

int spatten_select_heads(const float* importance, float scale, const int64_t* heads, int cur, int keep,
                         float* importance_out, int64_t* next_heads, int32_t* next_heads32, void* stream) {
  if (!importance || !next_heads) return fail(SPATTEN_ERR_INVALID, "select_heads: null pointer");
  if (cur < 1 || cur > 1024) return fail(SPATTEN_ERR_UNSUPPORTED, "select_heads: cur=%d (need 1..1024)", cur);
  if (keep < 1 || keep > cur) return fail(SPATTEN_ERR_INVALID, "select_heads: keep=%d (need 1..%d)", keep, cur);
  if (!(scale == scale)) return fail(SPATTEN_ERR_INVALID, "select_heads: scale is NaN");
  return cuda_status(spatten::launch_select_heads(importance, scale, heads, cur, keep, importance_out, next_heads,
                                                  next_heads32, (cudaStream_t)stream),
                     "select_heads launch");
}

int spatten_add_layer_norm(const void* x, int64_t x_row_stride, const void* res, int64_t res_row_stride,
                           const void* gamma, const void* beta, void* y, int64_t y_row_stride,
                           int64_t rows, int n, int dtype, float eps, void* stream) {
  if (rows < 0 || n < 1) return fail(SPATTEN_ERR_INVALID, "add_layer_norm: bad sizes rows=%lld n=%d",
                                     (long long)rows, n);
  if (rows == 0) return ok();  // nothing to read or write (empty tensors may have null data)
  if (!x || !gamma || !beta || !y) return fail(SPATTEN_ERR_INVALID, "add_layer_norm: null pointer");
  if (dtype != SPATTEN_DTYPE_F16 && dtype != SPATTEN_DTYPE_BF16)
    return fail(SPATTEN_ERR_UNSUPPORTED, "add_layer_norm: dtype %d (need f16 or bf16)", dtype);
  if (!spatten::add_layer_norm_supported(n))
    return fail(SPATTEN_ERR_UNSUPPORTED, "add_layer_norm: n=%d (need 256, 512, 768, 1024, 1536 or 2048)", n);
  if (!(eps >= 0.f)) return fail(SPATTEN_ERR_INVALID, "add_layer_norm: eps must be >= 0");
  if (x_row_stride < n || y_row_stride < n || (res && res_row_stride < n))
    return fail(SPATTEN_ERR_INVALID, "add_layer_norm: row stride below n");
  // 16-byte rows: every row start (base + r * stride * 2 bytes) on a 16-byte boundary
  auto a16 = [](const void* p, int64_t s) {
    return (reinterpret_cast<uintptr_t>(p) % 16) == 0 && (s * 2) % 16 == 0;
  };
  if (!a16(x, x_row_stride) || !a16(y, y_row_stride) || (res && !a16(res, res_row_stride)) ||
      !a16(gamma, 0) || !a16(beta, 0))
    return fail(SPATTEN_ERR_INVALID, "add_layer_norm: rows, gamma and beta must start on 16-byte boundaries");
  return cuda_status(spatten::launch_add_layer_norm(x, res, gamma, beta, y, rows, n, x_row_stride,
                                                    res_row_stride, y_row_stride, dtype, eps, sm_count(),
                                                    (cudaStream_t)stream),
                     "add_layer_norm launch");
}

// mode 0: sizing (shape and input checks only), 1: importance, 2: attend
static int fill_decode(const spatten_decode_args* a, spatten::DecodeParams& p, int mode) {
  const bool attend = mode == 2;
  if (!a) return fail(SPATTEN_ERR_INVALID, "decode: null args");
  if (a->dtype != SPATTEN_DTYPE_F16 && a->dtype != SPATTEN_DTYPE_BF16)
    return fail(SPATTEN_ERR_UNSUPPORTED, "decode: dtype %d (need f16 or bf16)", a->dtype);
  if (a->B < 1 || a->H < 1 || a->G < 1 || a->N < 1)
    return fail(SPATTEN_ERR_INVALID, "decode: empty shape B=%d H=%d G=%d N=%d", a->B, a->H, a->G, a->N);
  if (a->H % a->G) return fail(SPATTEN_ERR_INVALID, "decode: H %% G != 0");
  const int r = a->H / a->G;
  if (r != 1 && r != 2 && r != 4 && r != 8)
    return fail(SPATTEN_ERR_UNSUPPORTED, "decode: %d query heads per KV head (need 1, 2, 4 or 8)", r);
  if (a->D != 64 && a->D != 128) return fail(SPATTEN_ERR_UNSUPPORTED, "decode: D=%d (need 64 or 128)", a->D);
  if (a->n_valid < 1 || a->n_valid > a->N)
    return fail(SPATTEN_ERR_INVALID, "decode: n_valid %d outside [1, N=%d]", a->n_valid, a->N);
  if (a->B > 65535 || a->G > 65535) return fail(SPATTEN_ERR_UNSUPPORTED, "decode: B or G > 65535");
  if (!a->q8 || !a->q_scale || !a->k_msb || !a->k_scale)
    return fail(SPATTEN_ERR_INVALID, "decode: null q8/q_scale/k_msb/k_scale");
  if (!aligned(a->q8, 16) || !aligned(a->k_msb, 16) || !aligned(a->q_scale, 4) || !aligned(a->k_scale, 4))
    return fail(SPATTEN_ERR_INVALID, "decode: q8/k_msb not 16-byte or scales not 4-byte aligned");
  if (attend) {
    if (!a->k_lsb || !a->v || !a->kept || !a->out)
      return fail(SPATTEN_ERR_INVALID, "decode attend: null k_lsb/v/kept/out");
    if (!aligned(a->k_lsb, 16) || !aligned(a->v, 16) || !aligned(a->out, 4) || !aligned(a->kept, 8))
      return fail(SPATTEN_ERR_INVALID, "decode attend: k_lsb/v not 16-byte, out/kept not aligned");
    if (a->top_k < 1) return fail(SPATTEN_ERR_INVALID, "decode attend: top_k %d < 1", a->top_k);
  } else if (mode == 1) {
    if (!a->importance) return fail(SPATTEN_ERR_INVALID, "decode importance: null importance");
    if (!aligned(a->importance, 4)) return fail(SPATTEN_ERR_INVALID, "decode importance: not aligned");
  }
  p.dtype = a->dtype;
  p.B = a->B; p.H = a->H; p.G = a->G; p.N = a->N; p.D = a->D; p.n_valid = a->n_valid;
  p.q8 = a->q8; p.q_scale = a->q_scale; p.k_msb = a->k_msb; p.k_lsb = a->k_lsb;
  p.k_scale = a->k_scale; p.v = a->v; p.sm_scale = a->sm_scale; p.importance = a->importance;
  p.top_k = attend ? a->top_k : 1; p.kept = a->kept; p.out = a->out;
  return SPATTEN_OK;
}

static void decode_layout(const spatten::DecodeParams& p, size_t (&off)[6]) {
  const spatten::DecodeWorkspaceSizes s = spatten::decode_workspace_sizes(p);
  off[0] = 0;
  off[1] = off[0] + align256(s.scores);
  off[2] = off[1] + align256(s.part);
  off[3] = off[2] + align256(s.st);
  off[4] = off[3] + align256(s.ml);
  off[5] = off[4] + align256(s.o);
}

size_t spatten_decode_workspace_size(const spatten_decode_args* a) {
  spatten::DecodeParams p;
  if (fill_decode(a, p, 0) != SPATTEN_OK) return 0;
  p.top_k = a->top_k > 0 ? a->top_k : 1;
  size_t off[6];
  decode_layout(p, off);
  return off[5];
}

static int decode_workspace(const spatten::DecodeParams& p, void* ws, size_t bytes,
                            spatten::DecodeWorkspace& w) {
  size_t off[6];
  decode_layout(p, off);
  if (!ws || bytes < off[5])
    return fail(SPATTEN_ERR_INVALID, "decode: workspace of %zu bytes needed, %zu given", off[5], bytes);
  if (!aligned(ws, 256)) return fail(SPATTEN_ERR_INVALID, "decode: workspace not 256-byte aligned");
  uint8_t* b = static_cast<uint8_t*>(ws);
  w.scores = reinterpret_cast<float*>(b + off[0]);
  w.part = reinterpret_cast<float*>(b + off[1]);
  w.st = reinterpret_cast<float*>(b + off[2]);
  w.ml = reinterpret_cast<float*>(b + off[3]);
  w.o = reinterpret_cast<float*>(b + off[4]);
  return SPATTEN_OK;
}

int spatten_decode_importance(const spatten_decode_args* a, void* workspace, size_t workspace_bytes,
                              void* stream) {
  spatten::DecodeParams p;
  if (int e = fill_decode(a, p, 1)) return e;
  p.top_k = a->top_k > 0 ? a->top_k : 1;
  spatten::DecodeWorkspace w;
  if (int e = decode_workspace(p, workspace, workspace_bytes, w)) return e;
  return cuda_status(spatten::launch_decode_importance(p, w, (cudaStream_t)stream), "decode importance launch");
}

int spatten_decode_attend(const spatten_decode_args* a, void* workspace, size_t workspace_bytes,
                          void* stream) {
  spatten::DecodeParams p;
  if (int e = fill_decode(a, p, 2)) return e;
  spatten::DecodeWorkspace w;
  if (int e = decode_workspace(p, workspace, workspace_bytes, w)) return e;
  return cuda_status(spatten::launch_decode_attend(p, w, (cudaStream_t)stream), "decode attend launch");
}

int spatten_qkv_proj(const spatten_qkv_proj_args* a, void* stream) {
  if (!a) return fail(SPATTEN_ERR_INVALID, "qkv_proj: null args");
  if (a->dtype != SPATTEN_DTYPE_F16 && a->dtype != SPATTEN_DTYPE_BF16)
    return fail(SPATTEN_ERR_UNSUPPORTED, "qkv_proj: dtype %d (need f16 or bf16)", a->dtype);
  if (a->mode != SPATTEN_PROJ_QUANT && a->mode != SPATTEN_PROJ_DENSE)
    return fail(SPATTEN_ERR_INVALID, "qkv_proj: mode %d", a->mode);
  if (a->B < 1 || a->S < 1 || a->Kdim < 1 || a->Hall < 1 || a->cur < 1 || a->cur > a->Hall)
    return fail(SPATTEN_ERR_INVALID, "qkv_proj: bad sizes B=%d S=%d Kdim=%d Hall=%d cur=%d", a->B, a->S,
                a->Kdim, a->Hall, a->cur);
  if (a->Dh != 64 && a->Dh != 128) return fail(SPATTEN_ERR_UNSUPPORTED, "qkv_proj: Dh=%d (need 64 or 128)", a->Dh);
  if ((int64_t)a->B * a->S > (int64_t)1 << 30 || (int64_t)3 * a->Hall * a->Dh > (int64_t)1 << 30)
    return fail(SPATTEN_ERR_UNSUPPORTED, "qkv_proj: too many rows");
  if (a->Kdim % 8) return fail(SPATTEN_ERR_UNSUPPORTED, "qkv_proj: Kdim %d not a multiple of 8", a->Kdim);
  if (a->x_row_stride < a->Kdim || a->x_row_stride % 8)
    return fail(SPATTEN_ERR_INVALID, "qkv_proj: x row stride %lld (need >= Kdim, multiple of 8)",
                (long long)a->x_row_stride);
  if (!a->x || !a->w || !a->v) return fail(SPATTEN_ERR_INVALID, "qkv_proj: null x/w/v");
  if (!aligned(a->x, 16) || !aligned(a->w, 16) || !aligned(a->v, 16) || (a->bias && !aligned(a->bias, 2)) ||
      (a->heads && !aligned(a->heads, 8)))
    return fail(SPATTEN_ERR_INVALID, "qkv_proj: x/w/v not 16-byte aligned or bias/heads misaligned");
  if (a->mode == SPATTEN_PROJ_QUANT) {
    if (!a->q8 || !a->q_scale || !a->k_msb || !a->k_lsb || !a->k_scale)
      return fail(SPATTEN_ERR_INVALID, "qkv_proj: null quantised output");
    if (!aligned(a->q8, 16) || !aligned(a->k_msb, 16) || !aligned(a->k_lsb, 16) || !aligned(a->q_scale, 4) ||
        !aligned(a->k_scale, 4))
      return fail(SPATTEN_ERR_INVALID, "qkv_proj: quantised outputs misaligned");
  } else {
    if (!a->q || !a->k) return fail(SPATTEN_ERR_INVALID, "qkv_proj: null q/k");
    if (!aligned(a->q, 16) || !aligned(a->k, 16)) return fail(SPATTEN_ERR_INVALID, "qkv_proj: q/k misaligned");
  }
  spatten::ProjParams p;
  p.dtype = a->dtype;
  p.mode = a->mode;
  p.B = a->B; p.S = a->S; p.Kdim = a->Kdim;
  p.Hall = a->Hall; p.Dh = a->Dh; p.cur = a->cur;
  p.x = a->x; p.x_st = a->x_row_stride; p.w = a->w; p.bias = a->bias; p.heads = a->heads;
  p.q8 = a->q8; p.q_scale = a->q_scale; p.k_msb = a->k_msb; p.k_lsb = a->k_lsb; p.k_scale = a->k_scale;
  p.q = a->q; p.k = a->k; p.v = a->v;
  return cuda_status(spatten::launch_qkv_proj(p, (cudaStream_t)stream), "qkv_proj launch");
}

int spatten_qk_norm_rope(const spatten_qk_norm_rope_args* a, void* stream) {
  if (!a) return fail(SPATTEN_ERR_INVALID, "qk_norm_rope: null args");
  if (a->dtype != SPATTEN_DTYPE_F16 && a->dtype != SPATTEN_DTYPE_BF16)
    return fail(SPATTEN_ERR_UNSUPPORTED, "qk_norm_rope: dtype %d (need f16 or bf16)", a->dtype);
  if (a->D != 64 && a->D != 128) return fail(SPATTEN_ERR_UNSUPPORTED, "qk_norm_rope: D=%d (need 64 or 128)", a->D);
  if (a->B < 1 || a->S < 1 || a->Hq < 1 || a->Hk < 1)
    return fail(SPATTEN_ERR_INVALID, "qk_norm_rope: empty shape B=%d S=%d Hq=%d Hk=%d", a->B, a->S, a->Hq, a->Hk);
  if ((int64_t)a->B * a->S > ((int64_t)1 << 31) - 1)
    return fail(SPATTEN_ERR_UNSUPPORTED, "qk_norm_rope: too many tokens");
  if (!a->q || !a->k || !a->q_norm_w || !a->k_norm_w || !a->cos || !a->sin || !a->k_out)
    return fail(SPATTEN_ERR_INVALID, "qk_norm_rope: null input or k_out");
  if (!a->q_out && !a->q8) return fail(SPATTEN_ERR_INVALID, "qk_norm_rope: neither q_out nor q8 given");
  if (a->q8 && !a->q_scale) return fail(SPATTEN_ERR_INVALID, "qk_norm_rope: q8 without q_scale");
  if (a->q_row_stride < (int64_t)a->Hq * a->D || a->k_row_stride < (int64_t)a->Hk * a->D ||
      a->k_out_row_stride < (int64_t)a->Hk * a->D || (a->q_out && a->q_out_row_stride < (int64_t)a->Hq * a->D))
    return fail(SPATTEN_ERR_INVALID, "qk_norm_rope: row stride shorter than the heads");
  if (a->cs_b_stride < 0 || a->cs_s_stride < a->D)
    return fail(SPATTEN_ERR_INVALID, "qk_norm_rope: bad cos/sin strides");
  const void* ptrs16[] = {a->q, a->k, a->q_norm_w, a->k_norm_w, a->cos, a->sin, a->k_out, a->q_out, a->q8};
  for (const void* ptr : ptrs16)
    if (ptr && !aligned(ptr, 16)) return fail(SPATTEN_ERR_INVALID, "qk_norm_rope: a pointer is not 16-byte aligned");
  const int64_t strides[] = {a->q_row_stride, a->k_row_stride, a->k_out_row_stride,
                             a->q_out ? a->q_out_row_stride : 0, a->cs_b_stride, a->cs_s_stride};
  for (int64_t s : strides)
    if (s % 8) return fail(SPATTEN_ERR_INVALID, "qk_norm_rope: strides must be multiples of 8 elements");
  if (a->q_scale && !aligned(a->q_scale, 4)) return fail(SPATTEN_ERR_INVALID, "qk_norm_rope: q_scale misaligned");
  spatten::QkPrepParams p;
  p.dtype = a->dtype;
  p.B = a->B; p.S = a->S; p.Hq = a->Hq; p.Hk = a->Hk; p.D = a->D;
  p.q = a->q; p.q_st = a->q_row_stride; p.k = a->k; p.k_st = a->k_row_stride;
  p.q_w = a->q_norm_w; p.k_w = a->k_norm_w; p.eps = a->eps;
  p.cos = a->cos; p.sin = a->sin; p.cs_sb = a->cs_b_stride; p.cs_ss = a->cs_s_stride;
  p.k_out = a->k_out; p.ko_st = a->k_out_row_stride;
  p.q_out = a->q_out; p.qo_st = a->q_out_row_stride;
  p.q8 = a->q8; p.q_scale = a->q_scale;
  return cuda_status(spatten::launch_qk_prep(p, (cudaStream_t)stream), "qk_norm_rope launch");
}

int spatten_compact_out_proj(const spatten_compact_out_proj_args* a, void* stream) {
  if (!a) return fail(SPATTEN_ERR_INVALID, "compact_out_proj: null args");
  if (a->dtype != SPATTEN_DTYPE_F16 && a->dtype != SPATTEN_DTYPE_BF16)
    return fail(SPATTEN_ERR_UNSUPPORTED, "compact_out_proj: dtype %d (need f16 or bf16)", a->dtype);
  if (a->B < 1 || a->S < 1 || a->L < 1 || a->N < 1 || a->H < 1 || a->cur < 1 || a->cur > a->H)
    return fail(SPATTEN_ERR_INVALID, "compact_out_proj: bad sizes B=%d S=%d L=%d N=%d H=%d cur=%d", a->B, a->S,
                a->L, a->N, a->H, a->cur);
  if (a->head_dim < 64 || a->head_dim % 64)
    return fail(SPATTEN_ERR_UNSUPPORTED, "compact_out_proj: head_dim %d (need a multiple of 64)", a->head_dim);
  if (a->N % 32) return fail(SPATTEN_ERR_UNSUPPORTED, "compact_out_proj: N %d not a multiple of 32", a->N);
  if ((int64_t)a->B * a->S > ((int64_t)1 << 31) - 1 || (int64_t)a->B * a->L > ((int64_t)1 << 31) - 1 ||
      (int64_t)a->H * a->head_dim > ((int64_t)1 << 30))
    return fail(SPATTEN_ERR_UNSUPPORTED, "compact_out_proj: too many rows or columns");
  if (!a->kept || !a->ctx || !a->w || !a->res || !a->out)
    return fail(SPATTEN_ERR_INVALID, "compact_out_proj: null kept/ctx/w/res/out");
  if (a->ctx_row_stride < (int64_t)a->H * a->head_dim || a->res_row_stride < a->N)
    return fail(SPATTEN_ERR_INVALID, "compact_out_proj: row stride shorter than the row");
  if (a->ctx_row_stride % 8 || a->res_row_stride % 8)
    return fail(SPATTEN_ERR_INVALID, "compact_out_proj: strides must be multiples of 8 elements");
  if (!aligned(a->ctx, 16) || !aligned(a->w, 16) || !aligned(a->res, 16) || !aligned(a->out, 16) ||
      (a->bias && !aligned(a->bias, 16)) || !aligned(a->kept, 8) || (a->heads && !aligned(a->heads, 8)))
    return fail(SPATTEN_ERR_INVALID, "compact_out_proj: a pointer is misaligned");
  spatten::OutProjParams p;
  p.dtype = a->dtype;
  p.B = a->B; p.S = a->S; p.L = a->L; p.N = a->N;
  p.H = a->H; p.Dh = a->head_dim; p.cur = a->cur;
  p.heads = a->heads; p.kept = a->kept;
  p.ctx = a->ctx; p.ctx_st = a->ctx_row_stride;
  p.w = a->w; p.bias = a->bias;
  p.res = a->res; p.res_st = a->res_row_stride;
  p.out = a->out;
  return cuda_status(spatten::launch_out_proj(p, (cudaStream_t)stream), "compact_out_proj launch");
}

}  // extern "C"
