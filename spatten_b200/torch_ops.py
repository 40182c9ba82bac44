"""The path's operators registered with the PyTorch dispatcher (``torch.ops.spatten``).

Thin ``torch.library`` custom ops over the same C-ABI calls as the Python API
(no second implementation): code that addresses ops by name -- graph
capture, ``torch.ops.spatten.<op>`` in TorchScript-free pipelines, operator
registries -- finds them under the ``spatten`` namespace:

* ``spatten::quant_q_int8(Tensor x) -> (Tensor q8, Tensor scale)``
* ``spatten::quant_k_planes(Tensor k) -> (Tensor msb, Tensor lsb, Tensor scale)``
* ``spatten::progressive_attention(Tensor q, Tensor k, Tensor v, float refetch_threshold,
  float v_prune_threshold, float sm_scale, bool causal)
  -> (Tensor out, Tensor token_importance, Tensor head_abs_sum, Tensor refetch)``
* ``spatten::topk_select(Tensor x, int k) -> Tensor`` (sorted indices of the k largest per row)
* ``spatten::gather_rows(Tensor src, Tensor idx) -> Tensor``

CUDA tensors only, like the rest of the package. Importing this module
registers the ops once.
"""
import torch

from . import progressive as _pg
from . import select as _sel


@torch.library.custom_op("spatten::quant_q_int8", mutates_args=())
def quant_q_int8(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    q8, s = _pg.quant_q_int8(x)
    return q8, s


@torch.library.custom_op("spatten::quant_k_planes", mutates_args=())
def quant_k_planes(k: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    kp = _pg.quant_k_planes(k)
    return kp.msb, kp.lsb, kp.scale


@torch.library.custom_op("spatten::progressive_attention", mutates_args=())
def progressive_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, refetch_threshold: float,
                          v_prune_threshold: float, sm_scale: float, causal: bool
                          ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    r = _pg.progressive_attention(q, k, v, refetch_threshold=refetch_threshold,
                                  v_prune_threshold=v_prune_threshold, sm_scale=sm_scale,
                                  causal=causal, return_importance=True)
    return r.out, r.token_importance, r.head_abs_sum, r.refetch


@torch.library.custom_op("spatten::topk_select", mutates_args=())
def topk_select(x: torch.Tensor, k: int) -> torch.Tensor:
    return _sel.topk_indices(x, k)


@torch.library.custom_op("spatten::gather_rows", mutates_args=())
def gather_rows(src: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    return _sel.gather_rows(src, idx)
