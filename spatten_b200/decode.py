"""Decode attention over a progressive-quantised KV cache with top-k token
selection (SpAtten's cascade token pruning applied to decoding), on the
C-ABI kernels (``spatten_decode_*`` in include/spatten_b200.h).

A cache stores K as the prefill's packed 4-bit MSB / LSB planes with a per-key
scale (``quant_kv_cache``) and V as is. Per decode step and layer,
``decode_attention`` runs:

1. ``decode_importance``: MSB scores of every cached key for every query head
   (only the MSB plane is read), the softmax of each head over the keys and
   the token importance = the sum over the heads of those probabilities;
2. with the KV heads split over ranks (``process_group``), an all-reduce of
   the importance (each rank summed its own heads), so that every rank keeps
   the same keys;
3. the radix-select top-k of the importance (ties to the smaller index);
4. ``decode_attend``: exact int8 scores over the kept keys (their LSB planes
   only), softmax, P.V.

GQA: the H query heads share the G KV heads as in HF's ``repeat_kv``
(H / G in {1, 2, 4, 8}); D in {64, 128}; fp16 or bf16.
"""
import math
from collections import namedtuple

import torch

from . import _native as N
from .progressive import KPlanes, _stream, quant_k_planes, quant_q_int8
from .select import topk_indices

DecodeResult = namedtuple("DecodeResult", "out kept importance")
KVCache = namedtuple("KVCache", "planes v")  # planes: KPlanes [B, G, N, D/2] x2 + [B, G, N]; v [B, G, N, D]

_DT = {torch.float16: N.DTYPE_F16, torch.bfloat16: N.DTYPE_BF16}


def quant_kv_cache(k, v):
    """K [B, G, N, D] -> packed MSB / LSB planes + scales; V kept as is."""
    return KVCache(quant_k_planes(k), v)


def _args(q8, qs, cache, sm_scale, n_valid):
    planes, v = cache
    B, H, D = q8.shape
    G, Nk = planes.msb.shape[1], planes.msb.shape[2]
    for t, name in ((q8, "q8"), (planes.msb, "k_msb"), (planes.lsb, "k_lsb"), (planes.scale, "k_scale"),
                    (v, "v")):
        if not t.is_cuda:
            raise ValueError(f"{name}: CUDA tensor expected (no CPU path)")
        if not t.is_contiguous():
            raise ValueError(f"{name}: contiguous tensor expected")
    if v.dtype not in _DT:
        raise TypeError(f"v: dtype {v.dtype} (need float16 or bfloat16)")
    a = N.DecodeArgs()
    a.dtype = _DT[v.dtype]
    a.B, a.H, a.G, a.N, a.D = B, H, G, Nk, D
    a.n_valid = Nk if n_valid is None else int(n_valid)
    a.q8, a.q_scale = q8.data_ptr(), qs.data_ptr()
    a.k_msb, a.k_lsb, a.k_scale = planes.msb.data_ptr(), planes.lsb.data_ptr(), planes.scale.data_ptr()
    a.v = v.data_ptr()
    a.sm_scale = float(1.0 / math.sqrt(D) if sm_scale is None else sm_scale)
    return a


def _quant_query(q):
    """q [B, H, D] fp16/bf16 -> int8 [B, H, D] + scale [B, H]."""
    q8, qs = quant_q_int8(q.unsqueeze(2))
    return q8.view(q.shape), qs.view(q.shape[:2])


def _workspace(a, dev):
    n = N.lib.spatten_decode_workspace_size(a)
    return torch.empty((max(n, 1),), dtype=torch.uint8, device=dev), n


def decode_importance(q, cache, sm_scale=None, n_valid=None, q_quant=None):
    """Token importance [B, N] fp32 of the cache for queries q [B, H, D]."""
    q8, qs = q_quant if q_quant is not None else _quant_query(q)
    a = _args(q8, qs, cache, sm_scale, n_valid)
    imp = torch.empty((a.B, a.N), dtype=torch.float32, device=q8.device)
    a.importance = imp.data_ptr()
    a.top_k = 1
    ws, n = _workspace(a, q8.device)
    N.check(N.lib.spatten_decode_importance(a, ws.data_ptr(), n, _stream(q8)))
    return imp


def decode_attend(q, cache, kept, sm_scale=None, n_valid=None, q_quant=None):
    """Attention of q [B, H, D] over the kept keys [B, K] of the cache -> [B, H, D]."""
    q8, qs = q_quant if q_quant is not None else _quant_query(q)
    a = _args(q8, qs, cache, sm_scale, n_valid)
    kept = kept.to(torch.int64).contiguous()
    if tuple(kept.shape[:1]) != (a.B,) or kept.dim() != 2:
        raise ValueError(f"kept: shape {tuple(kept.shape)} (need [B, K])")
    out = torch.empty((a.B, a.H, a.D), dtype=cache.v.dtype, device=q8.device)
    a.top_k = kept.shape[1]
    a.kept, a.out = kept.data_ptr(), out.data_ptr()
    ws, n = _workspace(a, q8.device)
    N.check(N.lib.spatten_decode_attend(a, ws.data_ptr(), n, _stream(q8)))
    return out


def decode_attention(q, cache, top_k=2048, sm_scale=None, n_valid=None, process_group=None,
                     split_batch=False):
    """One decode step: importance, (all-reduce,) top-k, attention over the
    kept keys. ``q`` [B, H_local, D]; with ``process_group`` the cache holds
    this rank's KV heads and the importance is summed over all ranks' heads.
    With ``split_batch`` (and B a multiple of the group size) the sum and the
    selection are split over the batch instead (reduce-scatter, top-k of the
    rank's rows, all-gather of the kept indices: ``topk_by_batch_shard``);
    every rank still gets all B rows of kept keys, and ``importance`` of the
    result is then this rank's B / world summed rows."""
    qq = _quant_query(q)
    imp = decode_importance(q, cache, sm_scale, n_valid, q_quant=qq)
    nv = cache.planes.msb.shape[2] if n_valid is None else int(n_valid)
    k = min(int(top_k), nv)
    if process_group is not None and split_batch:
        from .distributed import topk_by_batch_shard
        kept, imp = topk_by_batch_shard(imp[:, :nv], k, process_group)
        out = decode_attend(q, cache, kept, sm_scale, n_valid, q_quant=qq)
        return DecodeResult(out, kept, imp)
    if process_group is not None:
        import torch.distributed as dist
        dist.all_reduce(imp, op=dist.ReduceOp.SUM, group=process_group)
    kept = topk_indices(imp[:, :nv], k)
    out = decode_attend(q, cache, kept, sm_scale, n_valid, q_quant=qq)
    return DecodeResult(out, kept, imp)


__all__ = ["DecodeResult", "KVCache", "KPlanes", "decode_attend", "decode_attention", "decode_importance",
           "quant_kv_cache"]
