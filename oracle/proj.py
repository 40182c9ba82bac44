"""Oracle: the active heads' Q/K/V projection followed by the quantisation
(numpy). Test infrastructure only (see ``oracle/__init__.py``).

Restates, for one layer of the cascade:

* ``slice_linear_weights`` (module.py:12-34): the rows of the active heads,
  ``W.view(H, Dh, Kdim)[heads]``, of each of W_q, W_k, W_v and of their
  biases;
* the projections ``F.linear(hidden, W_sliced, b_sliced)`` and
  ``transpose_for_scores`` (spatten_bert.py:39-45, 72-78): [B, cur, S, Dh];
* the activation's rounding to fp16 / bf16 (what the projection stores), then
  ``oracle.quant``'s int8 query and 4-bit K planes.

The products are summed in float64, so a GPU result that accumulates in fp32
in another order may round to the neighbouring fp16 / bf16 value now and
then; tests bound that, they do not expect bit equality of the projections.
"""
import numpy as np

from .quant import quant_k_planes, quant_rows_int8


def round_to(x, dtype):
    """float array -> the nearest fp16 / bf16 value (ties to even), as float32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        u = x.view(np.uint32).astype(np.uint64)
        r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16 << 16
        return (r & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
    raise ValueError(dtype)


def qkv_proj(x, w, bias, num_heads, head_dim, heads, dtype):
    """x [B, S, Kdim], w [3*H*Dh, Kdim], bias [3*H*Dh] or None (float arrays
    holding fp16 / bf16 values); heads: active head ids. Returns a dict with
    the rounded projections q, k, v [B, cur, S, Dh] (float32) and the
    quantised q8, q_scale, k_msb, k_lsb, k_scale."""
    x = np.asarray(x, dtype=np.float64)
    w = np.asarray(w, dtype=np.float64)
    B, S, K = x.shape
    H, D = num_heads, head_dim
    heads = np.asarray(heads, dtype=np.int64)
    out = {}
    for which, name in enumerate(("q", "k", "v")):
        rows = (which * H * D + heads[:, None] * D + np.arange(D)[None, :]).reshape(-1)
        y = x.reshape(B * S, K) @ w[rows].T
        if bias is not None:
            y = y + np.asarray(bias, dtype=np.float64)[rows]
        y = round_to(y, dtype).reshape(B, S, len(heads), D).transpose(0, 2, 1, 3)
        out[name] = np.ascontiguousarray(y)
    out["q8"], out["q_scale"] = quant_rows_int8(out["q"])
    out["k_msb"], out["k_lsb"], out["k_scale"] = quant_k_planes(out["k"])
    return out
