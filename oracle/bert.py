"""Oracle: the SpAtten cascade BERT encoder forward on the CPU (torch fp32).

Test infrastructure only (see ``oracle/__init__.py``).

Restates module.py:40-99 (``spatten_encoder_forward``) together with
spatten_bert.py:48-164 (``SpattenBertSelfAttention.forward``) as one function
over a Hugging Face ``BertModel``'s weights, with the same torch operations in
the same order so that, with the reference's own knobs, it reproduces the
reference bit for bit on the CPU (pinned by tests/test_oracle_golden.py
against vectors produced by the reference itself).

Knobs per layer (``LayerKnobs``) mirror the reference's module attributes
(spatten_bert.py:24-37, spatten_bert_ultimate.py:134-152) plus the ratio and
threshold knobs of the B200 build:

* ``head_keep_ratio`` / ``token_keep_ratio`` translate to the reference's
  counts with ``keep = max(1, ceil(ratio * current))`` evaluated exactly
  (``fractions.Fraction`` of the ratio's decimal repr).
* ``v_prune_threshold`` replaces the reference's per-row top count
  (spatten_bert.py:100-113) by ``p < thr -> 0`` (no renormalisation).
  Without it the count rule applies: with ``tie_rule="torch"`` exactly the
  reference's ``torch.topk``, with ``"smallest_index"`` (the device rule)
  the ``v_prune_num`` smallest by (score, key index); on the quantised core
  always the latter.
* ``enable_prog_quant`` routes the attention core through
  ``oracle.prog_attn.prog_attn_quant`` with ``quant_threshold`` as the row
  max-probability refetch threshold.
"""
import math
from dataclasses import dataclass
from fractions import Fraction

import numpy as np
import torch
import torch.nn.functional as F


def keep_count(ratio, current):
    """``max(1, ceil(ratio * current))`` evaluated exactly on the decimal ratio."""
    r = Fraction(repr(float(ratio)))
    return max(1, math.ceil(r * current))


@dataclass
class LayerKnobs:
    enable_head_prune: bool = False
    head_prune_num: int = 0
    head_keep_ratio: float = None
    enable_token_prune: bool = False
    token_prune_num: int = 0
    token_keep_ratio: float = None
    enable_v_prune: bool = False
    v_prune_num: int = 2
    v_prune_threshold: float = None
    enable_prog_quant: bool = False
    quant_threshold: float = 1.0


def eager_key_mask(attention_mask, dtype=torch.float32):
    """[B, S] 0/1 mask -> additive [B, 1, 1, S] (0 keep, finfo.min drop), the
    values HF's eager path adds per key."""
    if attention_mask is None:
        return None
    m = attention_mask.to(dtype)
    return ((1.0 - m) * torch.finfo(dtype).min)[:, None, None, :]


def _slice(linear, heads, n_heads, head_dim):
    # module.py:12-34
    w = linear.weight.view(n_heads, head_dim, -1)
    b = linear.bias.view(n_heads, head_dim)
    w = torch.index_select(w, 0, heads).reshape(-1, w.size(-1))
    b = torch.index_select(b, 0, heads).reshape(-1)
    return w, b


def _heads_view(x, n, d):
    bs, s, _ = x.shape
    return x.view(bs, s, n, d).permute(0, 2, 1, 3)


def _attention_core_quant(q, k, v, mask, sm_scale, refetch_thr, v_thr, v_count=0):
    from . import quant as oq
    from .prog_attn import prog_attn_quant
    qn = q.detach().numpy()
    kn = k.detach().numpy()
    q8, sq = oq.quant_rows_int8(qn)
    msb, lsb, sk = oq.quant_k_planes(kn)
    bias = None if mask is None else mask.detach().numpy().astype(np.float32)
    r = prog_attn_quant(q8, sq, msb, lsb, sk, v.detach().numpy(), sm_scale, refetch_thr,
                        v_thr or 0.0, bias=bias, v_count=v_count)
    ctx = torch.from_numpy(r["out"]).to(q.dtype)
    tok = torch.from_numpy(r["tok"]).to(q.dtype)
    return ctx, tok, r


def _topk_sorted(x, k, tie_rule):
    """sort(topk(x, k).indices) along the last axis. ``tie_rule="torch"`` is
    the reference's torch.topk (ties resolved by torch's CPU algorithm);
    ``"smallest_index"`` breaks ties at the k-th value towards smaller indices
    (the rule of the device top-k kernel)."""
    if tie_rule == "torch":
        return torch.sort(torch.topk(x, k=k, dim=-1).indices, dim=-1).values
    from .select import topk_sorted
    x2 = x.reshape(-1, x.shape[-1]).detach().numpy()
    return torch.from_numpy(topk_sorted(x2, k)).reshape(x.shape[:-1] + (k,))


def self_attention(attn, hidden, mask, active_heads, cumulative, kn: LayerKnobs, tie_rule="torch"):
    """One SpAtten self-attention (spatten_bert.py:48-164). Returns
    (full_context [B,S,H*D], next_heads, next_tokens, cumulative, info)."""
    n_heads = attn.num_attention_heads
    d = attn.attention_head_size
    bs, seq_len, _ = hidden.shape
    heads = active_heads if active_heads is not None else torch.arange(n_heads)
    cur = heads.size(0)
    wq, bq = _slice(attn.query, heads, n_heads, d)
    wk, bk = _slice(attn.key, heads, n_heads, d)
    wv, bv = _slice(attn.value, heads, n_heads, d)
    q = _heads_view(F.linear(hidden, wq, bq), cur, d)
    k = _heads_view(F.linear(hidden, wk, bk), cur, d)
    v = _heads_view(F.linear(hidden, wv, bv), cur, d)
    info = {}
    v_thr = kn.v_prune_threshold if kn.enable_v_prune else None
    v_count = kn.v_prune_num if (kn.enable_v_prune and v_thr is None and kn.v_prune_num > 0
                                 and seq_len > kn.v_prune_num) else 0
    if kn.enable_prog_quant:
        ctx, tok, r = _attention_core_quant(q, k, v, mask, 1.0 / math.sqrt(d),
                                            kn.quant_threshold, v_thr, v_count)
        info["refetch"] = r["refetch"]
    else:
        scores = torch.matmul(q, k.transpose(-1, -2))
        scores = scores / math.sqrt(d)
        if mask is not None:
            if mask.dim() > scores.dim():
                mask = mask.squeeze(1)
            scores = scores + mask
        probs = torch.softmax(scores, dim=-1)
        if kn.enable_v_prune:
            if v_thr is not None:
                probs = torch.where(probs < v_thr, torch.zeros_like(probs), probs)
            elif kn.v_prune_num > 0 and probs.size(-1) > kn.v_prune_num:
                if tie_rule == "torch":
                    keep_v = probs.size(-1) - kn.v_prune_num
                    _, idx = torch.topk(probs, k=keep_v, dim=-1)
                    m = torch.zeros_like(probs)
                    m.scatter_(-1, idx, 1)
                    probs = probs * m
                else:
                    # the device rule: drop the v_prune_num smallest by
                    # (score, key index)
                    from .prog_attn import _count_prune
                    sc = scores.detach().reshape(-1, scores.shape[-1]).numpy()
                    pr = probs.detach().reshape(-1, probs.shape[-1]).numpy().astype(np.float64)
                    pp, _ = _count_prune(pr, sc, kn.v_prune_num)
                    probs = torch.from_numpy(pp.astype(np.float32)).reshape(probs.shape)
        ctx = torch.matmul(probs, v)
        tok = probs.sum(dim=(1, 2))
    head_imp = ctx.abs().mean(dim=(0, 2, 3))
    info["head_importance"] = head_imp
    next_heads = heads
    if kn.enable_head_prune:
        prune = cur - keep_count(kn.head_keep_ratio, cur) if kn.head_keep_ratio is not None \
            else kn.head_prune_num
        if cur > prune:
            keep = max(1, cur - prune)
            if tie_rule == "torch":
                _, ti = torch.topk(head_imp, k=keep)
                next_heads = torch.sort(heads[ti]).values
            else:
                next_heads = heads[_topk_sorted(head_imp, keep, tie_rule)]
    if cumulative is None:
        cumulative = tok
    else:
        cumulative = cumulative + tok
    info["token_importance"] = cumulative.clone()
    next_tokens = None
    if kn.enable_token_prune:
        prune = seq_len - keep_count(kn.token_keep_ratio, seq_len) \
            if kn.token_keep_ratio is not None else kn.token_prune_num
        if seq_len > prune:
            keep = max(1, seq_len - prune)
            next_tokens = _topk_sorted(cumulative, keep, tie_rule)
    ctx = ctx.permute(0, 2, 1, 3).contiguous()
    full = torch.zeros(bs, seq_len, n_heads, d, dtype=hidden.dtype)
    full[:, :, heads, :] = ctx
    return full.view(bs, seq_len, -1), next_heads, next_tokens, cumulative, info


@torch.no_grad()
def spatten_bert_forward(model, input_ids, attention_mask=None, knobs=None, tie_rule="torch"):
    """Cascade forward (module.py:40-99). ``knobs``: list of LayerKnobs (one
    per layer) or a single LayerKnobs for all layers; ``tie_rule`` see
    ``_topk_sorted``. Returns a dict with the last hidden state and the
    per-layer pruning decisions."""
    layers = model.encoder.layer
    if knobs is None:
        knobs = LayerKnobs()
    if isinstance(knobs, LayerKnobs):
        knobs = [knobs] * len(layers)
    hidden = model.embeddings(input_ids=input_ids)
    mask = eager_key_mask(attention_mask, hidden.dtype)
    heads = tokens = cumulative = None
    rec = dict(heads=[], tokens=[], infos=[])
    for i, layer in enumerate(layers):
        if tokens is not None:
            idx = tokens.unsqueeze(-1).expand(-1, -1, hidden.size(-1))
            hidden = torch.gather(hidden, 1, idx)
            if mask is not None:
                mask = torch.gather(mask, 3, tokens.unsqueeze(1).unsqueeze(2))
            if cumulative is not None:
                cumulative = torch.gather(cumulative, 1, tokens)
        full, heads_n, tokens_n, cumulative, info = self_attention(
            layer.attention.self, hidden, mask, heads, cumulative, knobs[i], tie_rule)
        att_out = layer.attention.output(full, hidden)
        hidden = layer.output(layer.intermediate(att_out), att_out)
        heads, tokens = heads_n, tokens_n
        rec["heads"].append(heads.clone())
        rec["tokens"].append(None if tokens is None else tokens.clone())
        rec["infos"].append(info)
    rec["last_hidden_state"] = hidden
    return rec
