"""SpAtten sparse-attention hot path on B200 (sm_100a).

The compute path is the C-ABI library ``lib/libspatten_b200.so`` (hand-written
CUDA, see ``include/spatten_b200.h``); importing this package loads it and
raises if it is missing. The Python modules mirror the reference's
PyTorch-facing API:

* ``spatten_b200.progressive`` -- ``triton_progressive_qk``,
  ``spatten_progressive_attention`` and the integer ``progressive_attention``.
* ``spatten_b200.select``      -- cascade top-k and stream-compaction gathers.
* ``spatten_b200.bert``        -- ``SpattenBertSelfAttention``,
  ``spatten_encoder_forward``, ``slice_linear_weights``, ``patch_bert``.
* ``spatten_b200.qwen3``       -- ``SpattenQwen3Attention``, ``patch_qwen3``:
  Qwen3 prefill with cascade token pruning of the KV cache.
* ``spatten_b200.distributed`` -- batch / head sharding over ranks and the
  importance all-reduce.
* ``spatten_b200.torch_ops``   -- the same operators under ``torch.ops.spatten``.
"""
from ._native import LIB_PATH, SpattenError  # noqa: F401  (loads the library)
from .progressive import (  # noqa: F401
    AttnResult,
    KPlanes,
    prog_attn,
    progressive_attention,
    quant_k_planes,
    quant_q_int8,
    spatten_progressive_attention,
    triton_progressive_qk,
)
from .select import gather_head_rows, gather_rows, topk_indices  # noqa: F401

__all__ = [
    "AttnResult", "KPlanes", "LIB_PATH", "SpattenError", "gather_head_rows", "gather_rows",
    "prog_attn", "progressive_attention", "quant_k_planes", "quant_q_int8",
    "spatten_progressive_attention", "topk_indices", "triton_progressive_qk",
]
