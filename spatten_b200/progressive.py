"""Progressive-quantised sparse attention ops (host side of the C ABI).

Reference-compatible entry points, same names and argument meaning:

* ``triton_progressive_qk(q, k_msb, k_lsb, v, threshold, sm_scale)``
  (spatten_bert_ultimate.py:103-122): float K planes, and for every 32x32
  tile, if ``max(q.k_msb * sm_scale) < threshold`` the LSB plane is added.
* ``spatten_progressive_attention(q, k_msb, k_lsb, v, threshold=0.1)``
  (spatten_progressive_attention.py:82-102): the same rule on 64x64 tiles
  with ``sm_scale = 1/sqrt(D)``.

The integer op of the B200 build:

* ``progressive_attention(q, k, v, refetch_threshold=0.1, ...)`` quantises Q
  to int8 and K to 4-bit MSB/LSB planes, scores with exact int8 products,
  refetches the LSB plane only for rows whose maximum softmax probability
  falls below ``refetch_threshold``, prunes ``p < v_prune_threshold`` and can
  return the token / head importance the cascade needs.
* ``prog_attn(...)`` is the general form behind all of them (also used by the
  BERT drop-in with masks and head slots).

All tensors are CUDA tensors [Z, H, N, D] (last dim contiguous); every call
runs on the current torch stream and allocates its outputs with torch.
"""
import math
from typing import NamedTuple, Optional

import torch

from . import _native as N

_DT = {torch.float16: N.DTYPE_F16, torch.bfloat16: N.DTYPE_BF16, torch.float32: N.DTYPE_F32}
_F32_MIN = torch.finfo(torch.float32).min


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("spatten_b200 ops take CUDA tensors; there is no CPU path")


def _lastdim(t, name):
    if t.stride(-1) != 1:
        raise ValueError(f"{name}: last dimension must be contiguous")


def _as4d(x, name):
    if x.dim() == 3:
        x = x.unsqueeze(0)
    if x.dim() != 4:
        raise ValueError(f"{name}: expected [Z, H, N, D], got {tuple(x.shape)}")
    _lastdim(x, name)
    return x


def _ptr(t):
    return None if t is None else t.data_ptr()


class KPlanes(NamedTuple):
    """4-bit MSB/LSB planes of int8-quantised K (see quant_k_planes)."""
    msb: torch.Tensor    # uint8 [Z, H, N, D/2]
    lsb: torch.Tensor    # uint8 [Z, H, N, D/2]
    scale: torch.Tensor  # fp32 [Z, H, N]


class AttnResult(NamedTuple):
    out: torch.Tensor
    token_importance: Optional[torch.Tensor]  # [Z, N] sum over heads, queries of pruned P
    head_abs_sum: Optional[torch.Tensor]      # [H] sum over (z, m, d) of |out|
    refetch: Optional[torch.Tensor]           # [Z, H, M] bool, QUANT only
    scores: Optional[torch.Tensor] = None     # [Z, H, M / row stride, N] int32 scores used, QUANT only


def quant_q_int8(x):
    """Per-row symmetric int8: (q8 [Z,H,M,D] int8, scale [Z,H,M] fp32)."""
    _cuda(x)
    x4 = _as4d(x, "x")
    Z, H, M, D = x4.shape
    q8 = torch.empty((Z, H, M, D), dtype=torch.int8, device=x.device)
    sc = torch.empty((Z, H, M), dtype=torch.float32, device=x.device)
    N.check(N.lib.spatten_quant_q_int8(x4.data_ptr(), _DT[x.dtype], Z, H, M, D, x4.stride(0),
                                       x4.stride(1), x4.stride(2), q8.data_ptr(), sc.data_ptr(),
                                       _stream(x)))
    return q8, sc


def quant_k_planes(k):
    """Per-row symmetric int8 of K split into packed 4-bit planes (KPlanes)."""
    _cuda(k)
    k4 = _as4d(k, "k")
    Z, H, Nk, D = k4.shape
    msb = torch.empty((Z, H, Nk, D // 2), dtype=torch.uint8, device=k.device)
    lsb = torch.empty_like(msb)
    sc = torch.empty((Z, H, Nk), dtype=torch.float32, device=k.device)
    N.check(N.lib.spatten_quant_k_planes(k4.data_ptr(), _DT[k.dtype], Z, H, Nk, D, k4.stride(0),
                                         k4.stride(1), k4.stride(2), msb.data_ptr(),
                                         lsb.data_ptr(), sc.data_ptr(), _stream(k)))
    return KPlanes(msb, lsb, sc)


def _bias_view(bias, Z, H, M, Nk, device):
    if bias is None:
        return None
    if bias.dtype == torch.bool:
        bias = torch.zeros(bias.shape, dtype=torch.float32, device=device).masked_fill_(~bias, _F32_MIN)
    elif bias.dtype != torch.float32:
        bias = bias.float()
    while bias.dim() < 4:
        bias = bias.unsqueeze(0)
    return bias.expand(Z, H, M, Nk)


def prog_attn(q, k0, v, *, mode, k1=None, q_scale=None, k_scale=None, sm_scale=None,
              refetch_thr=0.1, v_thr=0.0, bias=None, causal=False, tile=(32, 32), tile_thr=0.0,
              tok_in=None, want_tok=False, want_head=False, want_refetch=False, want_scores=False,
              out=None, out_head_map=None, out_head_slots=0, v_prune_count=0, key_limit=None,
              score_row_stride=1):
    """General progressive attention (see spatten_prog_attn_args in
    include/spatten_b200.h). ``q`` int8 for QUANT; ``k0``/``k1`` are the
    MSB/LSB planes (QUANT), k (DENSE) or k_msb/k_lsb (COMPAT).
    ``v_prune_count`` (0..16) zeroes that many smallest probabilities of
    every row longer than it (the reference's count V prune). ``key_limit``
    [Z, M] int: row m of batch z sees keys n < key_limit[z, m] only (causal
    attention over a position-sorted subset of keys); replaces ``causal``.
    ``want_scores`` returns the integer scores of rows m % score_row_stride
    == 0 as [Z, H, ceil(M / score_row_stride), N] int32."""
    _cuda(q, k0, k1, v, q_scale, k_scale, bias, tok_in, out)
    q4, k04, v4 = _as4d(q, "q"), _as4d(k0, "k"), _as4d(v, "v")
    k14 = None if k1 is None else _as4d(k1, "k1")
    Z, H, M, D = q4.shape
    Hkv, Nk = v4.shape[1], v4.shape[2]
    if v.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise TypeError(f"v: dtype {v.dtype} (need float16, bfloat16 or float32)")
    if k14 is not None and k14.stride() != k04.stride():
        raise ValueError("k planes must share strides")
    if out is None:
        out4 = torch.empty((Z, H, M, D), dtype=v.dtype, device=v.device)
        out = out4
    else:
        out4 = _as4d(out, "out")
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    bv = _bias_view(bias, Z, H, M, Nk, v.device)
    a = N.ProgAttnArgs()
    a.mode, a.dtype = mode, _DT[v.dtype]
    a.Z, a.H, a.Hkv, a.M, a.N, a.D = Z, H, Hkv, M, Nk, D
    a.q = q4.data_ptr()
    a.q_sz, a.q_sh, a.q_sm = q4.stride()[:3]
    a.q_scale = _ptr(q_scale)
    a.k0, a.k1 = k04.data_ptr(), _ptr(k14)
    a.k_sz, a.k_sh, a.k_sn = k04.stride()[:3]
    a.k_scale = _ptr(k_scale)
    a.v = v4.data_ptr()
    a.v_sz, a.v_sh, a.v_sn = v4.stride()[:3]
    a.out = out4.data_ptr()
    a.o_sz, a.o_sh, a.o_sm = out4.stride()[:3]
    if out_head_map is not None:
        out_head_map = out_head_map.to(torch.int32)
    a.out_head_map = _ptr(out_head_map)
    a.out_head_slots = out_head_slots
    if bv is not None:
        a.bias = bv.data_ptr()
        a.b_sz, a.b_sh, a.b_sm, a.b_sn = bv.stride()
    a.sm_scale, a.refetch_thr, a.v_thr = float(sm_scale), float(refetch_thr), float(v_thr)
    a.tile_m, a.tile_n, a.tile_thr = int(tile[0]), int(tile[1]), float(tile_thr)
    a.causal = int(bool(causal))
    a.v_prune_count = int(v_prune_count)
    if key_limit is not None:
        _cuda(key_limit)
        if tuple(key_limit.shape) != (Z, M):
            raise ValueError(f"key_limit: shape {tuple(key_limit.shape)} (need {(Z, M)})")
        key_limit = key_limit.to(torch.int32).contiguous()
        a.key_limit = key_limit.data_ptr()
    tok = torch.empty((Z, Nk), dtype=torch.float32, device=v.device) if (want_tok or tok_in is not None) else None
    head = torch.empty((H,), dtype=torch.float32, device=v.device) if want_head else None
    ref = torch.empty((Z, H, M), dtype=torch.uint8, device=v.device) if want_refetch else None
    if tok_in is not None:
        tok_in = tok_in.float().contiguous()
    rs = max(1, int(score_row_stride))
    sco = torch.empty((Z, H, -(-M // rs), Nk), dtype=torch.int32, device=v.device) if want_scores else None
    a.score_row_stride = rs
    a.tok_out, a.tok_in, a.head_out, a.refetch_out = _ptr(tok), _ptr(tok_in), _ptr(head), _ptr(ref)
    a.score_out = _ptr(sco)
    ws_bytes = N.lib.spatten_prog_attn_workspace_size(a)
    ws = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device=v.device)
    N.check(N.lib.spatten_prog_attn(a, ws.data_ptr() if ws_bytes else None, ws_bytes, _stream(v)))
    # the kernel writes 0 / 1 bytes: a bool view, no conversion launch
    return AttnResult(out, tok, head, None if ref is None else ref.view(torch.bool), sco)


def _float_planes(*ts):
    """fp32 operands of the reference op are run in fp16 (the reference's
    Triton kernel contracts fp32 inputs in tf32 and rounds P and V to fp16)."""
    return [t.half() if t.dtype == torch.float32 else t for t in ts]


def triton_progressive_qk(q, k_msb, k_lsb, v, threshold, sm_scale):
    """Drop-in for spatten_bert_ultimate.triton_progressive_qk: float planes,
    32x32 tile criterion, output of q's dtype."""
    qq, km, kl, vv = _float_planes(q, k_msb, k_lsb, v)
    r = prog_attn(qq, km, vv, k1=kl, mode=N.MODE_COMPAT, sm_scale=sm_scale, tile=(32, 32),
                  tile_thr=threshold)
    return r.out.to(q.dtype)


def spatten_progressive_attention(q, k_msb, k_lsb, v, threshold=0.1):
    """Drop-in for spatten_progressive_attention.spatten_progressive_attention:
    64x64 tile criterion, sm_scale = 1/sqrt(D)."""
    qq, km, kl, vv = _float_planes(q, k_msb, k_lsb, v)
    r = prog_attn(qq, km, vv, k1=kl, mode=N.MODE_COMPAT, sm_scale=1.0 / math.sqrt(q.shape[-1]),
                  tile=(64, 64), tile_thr=threshold)
    return r.out.to(q.dtype)


def progressive_attention(q, k, v, refetch_threshold=0.1, v_prune_threshold=0.0, sm_scale=None,
                          attn_bias=None, causal=False, return_importance=False, k_planes=None,
                          v_prune_count=0):
    """Integer progressive attention on fp16/bf16 Q, K, V [Z, H, N, D].

    Returns ``out`` or, with ``return_importance``, an AttnResult with the
    token importance [Z, N], the per-head sum of |out| [H] and the refetch
    flags [Z, H, M]. ``k_planes`` (a KPlanes) skips the quantisation of K.
    ``v_prune_count`` applies the reference's count V prune as well."""
    q8, qs = quant_q_int8(q)
    kp = k_planes if k_planes is not None else quant_k_planes(k)
    r = prog_attn(q8, kp.msb, v, k1=kp.lsb, mode=N.MODE_QUANT, q_scale=qs, k_scale=kp.scale,
                  sm_scale=sm_scale, refetch_thr=refetch_threshold, v_thr=v_prune_threshold,
                  bias=attn_bias, causal=causal, want_tok=return_importance,
                  want_head=return_importance, want_refetch=return_importance,
                  v_prune_count=v_prune_count)
    return r if return_importance else r.out
