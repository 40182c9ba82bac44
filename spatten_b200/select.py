"""Cascade selection and compaction ops (host side of the C ABI).

* ``topk_indices(x, k)``  -- ``torch.sort(torch.topk(x, k).indices)`` per row
  (spatten_bert.py:123-128 for heads, :143-148 for tokens), radix select on
  the device; ties at the k-th value go to the smaller index.
* ``gather_rows(src, idx)`` -- ``torch.gather(src, 1, idx[..., None].expand)``
  for the kept tokens (module.py:53-54, 62-63).
* ``gather_head_rows(w, heads, head_dim)`` -- the head-row slicing of a
  Linear weight or bias (module.py:12-34, ``slice_linear_weights``).
"""
import torch

from . import _native as N


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


def topk_indices(x, k):
    """x [R, n] or [n] fp32 (CUDA) -> int64 [R, k] ascending top-k indices."""
    if not x.is_cuda:
        raise ValueError("topk_indices takes a CUDA tensor; there is no CPU path")
    squeeze = x.dim() == 1
    x2 = x.reshape(1, -1) if squeeze else x
    if x2.dtype != torch.float32:
        x2 = x2.float()
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    R, n = x2.shape
    out = torch.empty((R, k), dtype=torch.int64, device=x.device)
    N.check(N.lib.spatten_topk_indices(x2.data_ptr(), R, n, x2.stride(0), int(k), out.data_ptr(),
                                       _stream(x)))
    return out[0] if squeeze else out


def _gather(src3, idx2, rows_per_idx, idx_scale, shared_idx):
    """src3 [B, R, W] (row-contiguous), idx2 [B or 1, K] int64."""
    B, R, W = src3.shape
    K = idx2.shape[-1]
    esz = src3.element_size()
    out = torch.empty((B, K * rows_per_idx, W), dtype=src3.dtype, device=src3.device)
    idx2 = idx2.to(torch.int64).contiguous()
    N.check(N.lib.spatten_gather_rows(
        src3.data_ptr(), src3.stride(0) * esz, src3.stride(1) * esz, R,
        idx2.data_ptr(), 0 if shared_idx else idx2.stride(0), B, K, rows_per_idx, idx_scale,
        W * esz, out.data_ptr(), out.stride(0) * esz, out.stride(1) * esz, _stream(src3)))
    return out


def gather_rows(src, idx):
    """src [B, S, W...] or [B, S]; idx [B, K] -> src rows idx along dim 1."""
    if not (src.is_cuda and idx.is_cuda):
        raise ValueError("gather_rows takes CUDA tensors; there is no CPU path")
    B, S = src.shape[:2]
    tail = src.shape[2:]
    W = 1
    for d in tail:
        W *= d
    s3 = src.reshape(B, S, W)
    if s3.stride(-1) != 1:
        s3 = s3.contiguous()
    out = _gather(s3, idx, 1, 1, False)
    return out.reshape((B, idx.shape[1]) + tuple(tail))


def gather_head_rows(w, heads, head_dim):
    """Rows of the selected heads of a [H*head_dim, ...] weight or [H*head_dim]
    bias, in ``heads`` order -- a device-side ``slice_linear_weights``."""
    if not (w.is_cuda and heads.is_cuda):
        raise ValueError("gather_head_rows takes CUDA tensors; there is no CPU path")
    rows = w.shape[0]
    tail = w.shape[1:]
    W = 1
    for d in tail:
        W *= d
    s3 = w.reshape(1, rows, W)
    if s3.stride(-1) != 1:
        s3 = s3.contiguous()
    out = _gather(s3, heads.reshape(1, -1), head_dim, head_dim, True)
    return out.reshape((heads.numel() * head_dim,) + tuple(tail))


def select_heads(importance, scale, heads, keep):
    """Head decision of a cascade layer in one launch (spatten_select_heads):
    the importance scaled by ``scale`` (fp32 [cur]), the ``keep`` most
    important positions in ascending order (ties to the smaller position, as
    ``topk_indices``) and those positions mapped through ``heads`` (int64
    [cur] active heads, or None for 0..cur-1). Returns (scaled importance,
    next heads int64 [keep], next heads int32 [keep])."""
    if not importance.is_cuda:
        raise ValueError("select_heads takes CUDA tensors; there is no CPU path")
    imp = importance.reshape(-1)
    if imp.dtype != torch.float32 or not imp.is_contiguous():
        imp = imp.float().contiguous()
    cur = imp.numel()
    if heads is not None:
        heads = heads.to(torch.int64).contiguous()
        if heads.numel() != cur:
            raise ValueError(f"select_heads: {heads.numel()} heads for {cur} importance values")
    out = torch.empty(cur, dtype=torch.float32, device=imp.device)
    nxt = torch.empty(keep, dtype=torch.int64, device=imp.device)
    nxt32 = torch.empty(keep, dtype=torch.int32, device=imp.device)
    N.check(N.lib.spatten_select_heads(imp.data_ptr(), float(scale), None if heads is None else heads.data_ptr(),
                                       cur, int(keep), out.data_ptr(), nxt.data_ptr(), nxt32.data_ptr(),
                                       _stream(imp)))
    return out, nxt, nxt32
