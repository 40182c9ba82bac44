"""Oracle: the SpAtten cascade Qwen3 prefill on the CPU.

Test infrastructure only (see ``oracle/__init__.py``).

The reference has no Qwen3 code, so parity for this path is unpinned by the
reference: this restatement defines the semantics of the B200 drop-in
(``spatten_b200.qwen3``) on top of the installed HF Qwen3 modules
(``transformers/models/qwen3/modeling_qwen3.py``: embeddings, RMSNorm,
QK-norm, RoPE ``apply_rotary_pos_emb``, MLP, GQA head sharing as in
``repeat_kv``), with the attention core of ``oracle.prog_attn`` (float64 on
fp32 scores). With pruning and quantisation off it reproduces HF's own eager
Qwen3 forward (pinned by tests/test_oracle_golden.py).

Per layer: attention of every query position over the keys kept so far (all
at layer 0), causal by position (query m sees kept keys at positions <= m);
token importance = sum over heads and queries of the pruned probabilities,
added to the kept keys' cumulative score; keep ``max(1, ceil(r * K))`` keys by
cumulative score (ties to the smaller position) for the next layer. Queries
are never pruned.
"""
import numpy as np
import torch
from transformers.models.qwen3.modeling_qwen3 import apply_rotary_pos_emb

from .bert import keep_count
from .prog_attn import prog_attn_dense, prog_attn_quant
from .quant import quant_k_planes, quant_rows_int8
from .select import topk_sorted


@torch.no_grad()
def spatten_qwen3_forward(model, input_ids, enable_token_prune=False, token_keep_ratio=None,
                          token_prune_num=0, enable_v_prune=False, v_prune_threshold=None,
                          v_prune_num=2, enable_prog_quant=False, quant_threshold=0.1):
    """Cascade prefill of a HF Qwen3Model / Qwen3ForCausalLM (fp32, CPU).
    Returns dict(last_hidden_state, positions=[per layer [B, K] attended],
    importance=[per layer [B, K] cumulative], refetch=[per layer], kth_gap
    (relative margin of the closest keep decision), refetch_gap)."""
    base = model.model if hasattr(model, "model") else model
    cfg = base.config
    B, S = input_ids.shape
    H, Hkv = cfg.num_attention_heads, cfg.num_key_value_heads
    d = getattr(cfg, "head_dim", cfg.hidden_size // H)
    x = base.embed_tokens(input_ids)
    position_ids = torch.arange(S)[None].expand(B, S)
    cos, sin = base.rotary_emb(x, position_ids)
    pos = np.tile(np.arange(S), (B, 1))
    cum = None
    rec = dict(positions=[], importance=[], refetch=[], kth_gap=np.inf, refetch_gap=np.inf)
    for layer in base.layers:
        a = layer.self_attn
        h = layer.input_layernorm(x)
        K = pos.shape[1]
        r, o = attention_layer(a, h, cos, sin, pos, enable_v_prune=enable_v_prune,
                               v_prune_threshold=v_prune_threshold, v_prune_num=v_prune_num,
                               enable_prog_quant=enable_prog_quant, quant_threshold=quant_threshold)
        if enable_prog_quant:
            rec["refetch"].append(r["refetch"])
            rec["refetch_gap"] = min(rec["refetch_gap"], r["refetch_gap"])
        x = x + a.o_proj(o)
        x = x + layer.mlp(layer.post_attention_layernorm(x))
        tok = r["tok"] if cum is None else r["tok"] + cum
        rec["positions"].append(pos.copy())
        rec["importance"].append(tok.copy())
        if enable_token_prune:
            keep = keep_count(token_keep_ratio, K) if token_keep_ratio is not None \
                else max(1, K - int(token_prune_num))
            if keep < K:
                srt = np.sort(tok, axis=1)
                # margin of the keep decision: the keep-th largest vs the next
                gap = np.min(np.abs(srt[:, K - keep] - srt[:, K - keep - 1]) /
                             np.maximum(np.abs(srt[:, K - keep]), 1e-30))
                rec["kth_gap"] = min(rec["kth_gap"], gap)
                idx = topk_sorted(tok, keep)
                pos = np.take_along_axis(pos, idx, axis=1)
                cum = np.take_along_axis(tok, idx, axis=1)
            else:
                cum = tok
        else:
            cum = tok
    rec["last_hidden_state"] = base.norm(x)
    return rec


@torch.no_grad()
def attention_layer(a, h, cos, sin, pos, enable_v_prune=False, v_prune_threshold=None,
                    v_prune_num=2, enable_prog_quant=False, quant_threshold=0.1):
    """The SpAtten attention of one Qwen3 layer (module ``a``) on its
    normalised input ``h`` [B, S, hidden] (fp32, CPU): Q/K/V projections,
    QK-norm, RoPE (cos / sin [B, S, D]), attention of every query position
    over the kept keys at positions ``pos`` [B, K] (ascending), causal by
    position. Returns (the core's dict -- see oracle.prog_attn --, the
    attention output [B, S, H * D] before ``o_proj``)."""
    B, S, _ = h.shape
    H, Hkv, d = a.config.num_attention_heads, a.config.num_key_value_heads, a.head_dim
    q = a.q_norm(a.q_proj(h).view(B, S, H, d))
    k = a.k_norm(a.k_proj(h).view(B, S, Hkv, d))
    v = a.v_proj(h).view(B, S, Hkv, d)
    q, k = apply_rotary_pos_emb(q, k, cos, sin, unsqueeze_dim=2)
    K = pos.shape[1]
    kk = np.stack([k[b].numpy()[pos[b]] for b in range(B)])  # [B, K, Hkv, d]
    vv = np.stack([v[b].numpy()[pos[b]] for b in range(B)])
    lim = np.stack([np.searchsorted(pos[b], np.arange(S), side="right") for b in range(B)])
    qh = q.permute(0, 2, 1, 3).numpy()
    kh = np.ascontiguousarray(kk.transpose(0, 2, 1, 3))
    vh = np.ascontiguousarray(vv.transpose(0, 2, 1, 3))
    v_thr, v_count = 0.0, 0
    if enable_v_prune:
        if v_prune_threshold is not None:
            v_thr = float(v_prune_threshold)
        elif v_prune_num > 0 and K > v_prune_num:
            v_count = int(v_prune_num)
    if enable_prog_quant:
        q8, sq = quant_rows_int8(qh)
        msb, lsb, sk = quant_k_planes(kh)
        r = prog_attn_quant(q8, sq, msb, lsb, sk, vh, a.scaling, quant_threshold, v_thr,
                            key_limit=lim, v_count=v_count)
    else:
        r = prog_attn_dense(qh, kh, vh, a.scaling, v_thr, key_limit=lim, v_count=v_count)
    o = torch.from_numpy(r["out"].astype(np.float32)).permute(0, 2, 1, 3).reshape(B, S, H * d)
    return r, o
