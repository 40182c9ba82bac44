"""Fused Q/K/V projection of the active heads (host side of spatten_qkv_proj).

One tensor-core kernel replaces, per layer of the cascade, the reference's
``slice_linear_weights`` (module.py:12-34: index_select of the active heads'
rows of W_q / W_k / W_v and their biases), the three projections of
``SpattenBertSelfAttention.forward`` (spatten_bert.py:72-78) and the
quantisation of Q and K that the progressive attention reads (the K plane
split of spatten_bert_ultimate.py:184-185, made integer). The weight is never
sliced: the kernel loads its tiles from the active heads' rows of the full
stacked weight.

``qkv_proj(x, w, bias, num_heads, head_dim, heads=None, quantize=True)``
    x     [B, S, Kdim] fp16 / bf16 (rows contiguous)
    w     [3 * num_heads * head_dim, Kdim]: the query, key and value weights
          stacked (nn.Linear layout)
    bias  [3 * num_heads * head_dim] or None
    heads int64 [cur] active heads (None: all)
returns ``QkvQuant(q8, q_scale, k_planes, v)`` (quantize=True: Q int8 +
scale, K as 4-bit MSB / LSB planes + scale) or ``QkvDense(q, k, v)``; every
output head-major [B, cur, S, ...], as the attention kernel reads them.
"""
from typing import NamedTuple

import torch

from . import _native as N
from .progressive import _DT, KPlanes, _stream


class QkvQuant(NamedTuple):
    q8: torch.Tensor       # int8 [B, cur, S, Dh]
    q_scale: torch.Tensor  # fp32 [B, cur, S]
    k_planes: KPlanes      # uint8 [B, cur, S, Dh/2] x 2, fp32 [B, cur, S]
    v: torch.Tensor        # [B, cur, S, Dh]


class QkvDense(NamedTuple):
    q: torch.Tensor  # [B, cur, S, Dh]
    k: torch.Tensor
    v: torch.Tensor


def qkv_proj(x, w, bias, num_heads, head_dim, heads=None, quantize=True):
    if not (x.is_cuda and w.is_cuda):
        raise ValueError("qkv_proj takes CUDA tensors; there is no CPU path")
    if x.dtype not in (torch.float16, torch.bfloat16) or w.dtype != x.dtype:
        raise ValueError("qkv_proj: x and w must both be fp16 or both bf16")
    if x.dim() != 3:
        raise ValueError(f"qkv_proj: x must be [B, S, Kdim], got {tuple(x.shape)}")
    B, S, Kdim = x.shape
    if x.stride(2) != 1 or x.stride(0) != S * x.stride(1):
        x = x.contiguous()
    w = w.contiguous()
    if tuple(w.shape) != (3 * num_heads * head_dim, Kdim):
        raise ValueError(f"qkv_proj: w must be [{3 * num_heads * head_dim}, {Kdim}], got {tuple(w.shape)}")
    if bias is not None:
        bias = bias.contiguous()
        if bias.dtype != x.dtype or bias.numel() != w.shape[0]:
            raise ValueError("qkv_proj: bias must match w's rows and x's dtype")
    if heads is not None:
        heads = heads.to(torch.int64).contiguous()
        cur = heads.numel()
    else:
        cur = num_heads
    dev, dt = x.device, x.dtype
    a = N.QkvProjArgs()
    a.dtype = _DT[dt]
    a.mode = N.PROJ_QUANT if quantize else N.PROJ_DENSE
    a.B, a.S, a.Kdim = B, S, Kdim
    a.Hall, a.Dh, a.cur = num_heads, head_dim, cur
    a.x, a.x_row_stride = x.data_ptr(), x.stride(1)
    a.w = w.data_ptr()
    a.bias = None if bias is None else bias.data_ptr()
    a.heads = None if heads is None else heads.data_ptr()
    v = torch.empty((B, cur, S, head_dim), dtype=dt, device=dev)
    a.v = v.data_ptr()
    if quantize:
        q8 = torch.empty((B, cur, S, head_dim), dtype=torch.int8, device=dev)
        qs = torch.empty((B, cur, S), dtype=torch.float32, device=dev)
        msb = torch.empty((B, cur, S, head_dim // 2), dtype=torch.uint8, device=dev)
        lsb = torch.empty_like(msb)
        ks = torch.empty((B, cur, S), dtype=torch.float32, device=dev)
        a.q8, a.q_scale, a.k_msb, a.k_lsb, a.k_scale = (t.data_ptr() for t in (q8, qs, msb, lsb, ks))
        N.check(N.lib.spatten_qkv_proj(a, _stream(x)))
        return QkvQuant(q8, qs, KPlanes(msb, lsb, ks), v)
    q = torch.empty_like(v)
    k = torch.empty_like(v)
    a.q, a.k = q.data_ptr(), k.data_ptr()
    N.check(N.lib.spatten_qkv_proj(a, _stream(x)))
    return QkvDense(q, k, v)


def compact_out_proj(ctx, res, kept, w, bias, num_heads, head_dim, heads=None):
    """Attention output projection + residual of the kept tokens only
    (host side of spatten_compact_out_proj): the gather of the next layer's
    hidden states (module.py:49-54) moved into the row loads of HF
    BertSelfOutput's dense layer, so what follows runs on the compacted rows.

        out[b, j] = T(T(ctx[b, s] @ w.T + bias) + res[b, s]),  s = kept[b, j]

    ctx  [B, S, num_heads * head_dim] (the attention context; only the
         ``heads`` column blocks are read, the others must be zero for the
         result to equal the dense layer's)
    res  [B, S, N] (the layer's input hidden states)
    kept int64 [B, L] positions; w [N, num_heads * head_dim]; bias [N] or None
    returns [B, L, N] in ctx's dtype."""
    if not (ctx.is_cuda and res.is_cuda and w.is_cuda and kept.is_cuda):
        raise ValueError("compact_out_proj takes CUDA tensors; there is no CPU path")
    if ctx.dtype not in (torch.float16, torch.bfloat16) or w.dtype != ctx.dtype or res.dtype != ctx.dtype:
        raise ValueError("compact_out_proj: ctx, res and w must share one dtype, fp16 or bf16")
    if ctx.dim() != 3 or res.dim() != 3 or kept.dim() != 2:
        raise ValueError("compact_out_proj: ctx, res must be [B, S, F], kept [B, L]")
    B, S, F = ctx.shape
    Nf = w.shape[0]
    if F != num_heads * head_dim or tuple(w.shape) != (Nf, F) or tuple(res.shape) != (B, S, Nf) \
            or kept.shape[0] != B:
        raise ValueError(f"compact_out_proj: shapes ctx {tuple(ctx.shape)}, res {tuple(res.shape)}, "
                         f"w {tuple(w.shape)}, kept {tuple(kept.shape)} do not match")
    if ctx.stride(2) != 1 or ctx.stride(0) != S * ctx.stride(1):
        ctx = ctx.contiguous()
    if res.stride(2) != 1 or res.stride(0) != S * res.stride(1):
        res = res.contiguous()
    w = w.contiguous()
    kept = kept.to(torch.int64).contiguous()
    if bias is not None:
        bias = bias.contiguous()
        if bias.dtype != ctx.dtype or bias.numel() != Nf:
            raise ValueError("compact_out_proj: bias must match w's rows and ctx's dtype")
    if heads is not None:
        heads = heads.to(torch.int64).contiguous()
        cur = heads.numel()
    else:
        cur = num_heads
    L = kept.shape[1]
    out = torch.empty(B, L, Nf, dtype=ctx.dtype, device=ctx.device)
    a = N.CompactOutProjArgs()
    a.dtype = _DT[ctx.dtype]
    a.B, a.S, a.L, a.N = B, S, L, Nf
    a.H, a.head_dim, a.cur = num_heads, head_dim, cur
    a.heads = heads.data_ptr() if heads is not None else None
    a.kept = kept.data_ptr()
    a.ctx, a.ctx_row_stride = ctx.data_ptr(), ctx.stride(1)
    a.w = w.data_ptr()
    a.bias = bias.data_ptr() if bias is not None else None
    a.res, a.res_row_stride = res.data_ptr(), res.stride(1)
    a.out = out.data_ptr()
    N.check(N.lib.spatten_compact_out_proj(a, _stream(ctx)))
    return out


LAYER_NORM_FEATURES = (256, 512, 768, 1024, 1536, 2048)


def add_layer_norm(x, weight, bias, eps, residual=None):
    """LayerNorm of ``x`` (+ ``residual``, the sum rounded to x's dtype as
    torch's add rounds it) over the last dimension, with affine ``weight`` /
    ``bias`` (host side of spatten_add_layer_norm): the residual add +
    LayerNorm of HF's BertOutput and the LayerNorm of BertSelfOutput in one
    launch. fp16 / bf16, last dimension in ``LAYER_NORM_FEATURES``; x,
    residual, weight and bias share one dtype. Returns a new tensor shaped
    like x."""
    if not (x.is_cuda and weight.is_cuda and bias.is_cuda):
        raise ValueError("add_layer_norm takes CUDA tensors; there is no CPU path")
    if x.dtype not in (torch.float16, torch.bfloat16) or weight.dtype != x.dtype or bias.dtype != x.dtype:
        raise ValueError("add_layer_norm: x, weight and bias must share one dtype, fp16 or bf16")
    n = x.shape[-1]
    if weight.numel() != n or bias.numel() != n:
        raise ValueError(f"add_layer_norm: weight / bias of {weight.numel()} / {bias.numel()} for {n} features")
    x2 = x.reshape(-1, n)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    r2 = None
    if residual is not None:
        if residual.shape != x.shape or residual.dtype != x.dtype:
            raise ValueError("add_layer_norm: residual must match x's shape and dtype")
        r2 = residual.reshape(-1, n)
        if r2.stride(-1) != 1:
            r2 = r2.contiguous()
    y = torch.empty(x2.shape, dtype=x.dtype, device=x.device)
    w, b = weight.contiguous(), bias.contiguous()
    N.check(N.lib.spatten_add_layer_norm(
        x2.data_ptr(), x2.stride(0), None if r2 is None else r2.data_ptr(), 0 if r2 is None else r2.stride(0),
        w.data_ptr(), b.data_ptr(), y.data_ptr(), y.stride(0), x2.shape[0], n, _DT[x.dtype], float(eps),
        _stream(x)))
    return y.view(x.shape)
