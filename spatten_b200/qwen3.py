"""Drop-in SpAtten cascade for Hugging Face Qwen3 prefill, on the C-ABI kernels.

``SpattenQwen3Attention(config, layer_idx)`` subclasses HF ``Qwen3Attention``
(installed ``transformers/models/qwen3/modeling_qwen3.py``: the projections
are the HF module's own; for fp16 / bf16 its per-head RMSNorm QK-norm and
RoPE run as one kernel, ``qk_norm_rope``, with the HF arithmetic and the
query's int8 quantisation; fp32 keeps the HF modules) and replaces its
attention core with the progressive sparse attention kernel:

* GQA: Q heads share KV heads as in HF's ``repeat_kv`` (head h reads KV head
  h // (H / Hkv)); the kernel indexes the shared KV head, nothing is repeated.
* Cascade token pruning applied to the KV cache: every layer attends over the
  keys kept so far (all keys at layer 0), adds its token importance -- the sum
  over heads and queries of the pruned probabilities, as in SpAtten's BERT
  cascade (spatten_bert.py:136-150) -- to the kept keys' cumulative score and
  keeps ``max(1, ceil(token_keep_ratio * K))`` of them (radix-select top-k,
  ties to the smaller position) for the next layer. Queries are never pruned:
  every position's hidden state goes through every layer.
* Causality over a pruned key set: the kept keys stay sorted by position, so
  query position m sees the prefix of keys whose position is <= m
  (``key_limit``); CTAs skip key tiles none of their rows sees.
* The KV cache (``past_key_values``, e.g. HF ``DynamicCache``) of layer i holds
  the keys and values layer i attended over, post-RoPE, in HF's
  [B, Hkv, K_i, D] layout; ``kept_positions`` gives their positions.
* Knobs: ``enable_token_prune`` with ``token_keep_ratio`` (or
  ``token_prune_num``), ``enable_v_prune`` with ``v_prune_threshold`` or the
  count ``v_prune_num`` (<= 16), ``enable_prog_quant`` with ``quant_threshold``
  (the row max-probability below which the LSB plane of K is refetched).

Prefill of unpadded batches only (the HF attention mask is not read: the
mask is the causal one). The cascade state is shared by all layers of a
model (``patch_qwen3``) and restarts at layer 0 of every forward.
"""
import math
from fractions import Fraction

import torch
from transformers.models.qwen3.modeling_qwen3 import Qwen3Attention, apply_rotary_pos_emb

from . import _native as N
from .progressive import prog_attn, quant_k_planes, quant_q_int8
from .select import gather_rows, topk_indices


def keep_count(ratio, current):
    """``max(1, ceil(ratio * current))``, exact on the ratio's decimal repr."""
    return max(1, math.ceil(Fraction(repr(float(ratio))) * current))


_DT = {torch.float16: N.DTYPE_F16, torch.bfloat16: N.DTYPE_BF16}


def qk_norm_rope(q, k, q_norm, k_norm, cos, sin, Hq, Hk, D, quantize_q):
    """QK-norm + RoPE of the projections in one kernel (spatten_qk_norm_rope):
    q [B, S, Hq*D], k [B, S, Hk*D] (fp16 / bf16, rows contiguous), the HF
    Qwen3RMSNorm modules ``q_norm`` / ``k_norm``, cos / sin [B, S, D].
    Returns (q [B, S, Hq, D] or None, q8 [B, Hq, S, D] or None, q_scale
    [B, Hq, S] or None, k [B, S, Hk, D]); q8 / q_scale when ``quantize_q``,
    q otherwise."""
    B, S, _ = q.shape
    if q.stride(2) != 1 or q.stride(0) != S * q.stride(1):
        q = q.contiguous()
    if k.stride(2) != 1 or k.stride(0) != S * k.stride(1):
        k = k.contiguous()
    if cos.stride(-1) != 1 or sin.stride() != cos.stride():
        cos, sin = cos.contiguous(), sin.contiguous()
    wq, wk = q_norm.weight.contiguous(), k_norm.weight.contiguous()
    dev, dt = q.device, q.dtype
    a = N.QkNormRopeArgs()
    a.dtype = _DT[dt]
    a.B, a.S, a.Hq, a.Hk, a.D = B, S, Hq, Hk, D
    a.q, a.q_row_stride = q.data_ptr(), q.stride(1)
    a.k, a.k_row_stride = k.data_ptr(), k.stride(1)
    a.q_norm_w, a.k_norm_w = wq.data_ptr(), wk.data_ptr()
    if float(k_norm.variance_epsilon) != float(q_norm.variance_epsilon):
        raise ValueError("qk_norm_rope: q_norm and k_norm must share their epsilon")
    a.eps = float(q_norm.variance_epsilon)
    a.cos, a.sin = cos.data_ptr(), sin.data_ptr()
    a.cs_b_stride = cos.stride(0) if cos.shape[0] == B else 0
    a.cs_s_stride = cos.stride(1)
    k_out = torch.empty((B, S, Hk, D), dtype=dt, device=dev)
    a.k_out, a.k_out_row_stride = k_out.data_ptr(), Hk * D
    q_out = q8 = qs = None
    if quantize_q:
        q8 = torch.empty((B, Hq, S, D), dtype=torch.int8, device=dev)
        qs = torch.empty((B, Hq, S), dtype=torch.float32, device=dev)
        a.q8, a.q_scale = q8.data_ptr(), qs.data_ptr()
    else:
        q_out = torch.empty((B, S, Hq, D), dtype=dt, device=dev)
        a.q_out, a.q_out_row_stride = q_out.data_ptr(), Hq * D
    N.check(N.lib.spatten_qk_norm_rope(a, torch.cuda.current_stream(dev).cuda_stream))
    return q_out, q8, qs, k_out


class CascadeState:
    """Kept key positions [B, K] (int64, ascending) and their cumulative
    token importance [B, K] (fp32), handed from layer to layer."""

    def __init__(self):
        self.positions = None
        self.cumulative = None
        self.kept_per_layer = []


class SpattenQwen3Attention(Qwen3Attention):
    """HF Qwen3Attention with the SpAtten cascade, on the B200 kernels."""

    def __init__(self, config, layer_idx):
        super().__init__(config, layer_idx)
        self.num_heads = config.num_attention_heads
        self.num_kv_heads = config.num_key_value_heads
        self.enable_token_prune = False
        self.token_keep_ratio = None
        self.token_prune_num = 0
        self.enable_v_prune = False
        self.v_prune_threshold = None
        self.v_prune_num = 2
        self.enable_prog_quant = False
        self.quant_threshold = 0.1
        self.cascade = CascadeState()
        # diagnostics of the last forward
        self.kept_positions = None      # [B, K] positions this layer attended over
        self.token_importance = None    # [B, K] cumulative importance after this layer
        self.last_refetch = None

    def _v_prune(self, K):
        v_thr, v_count = 0.0, 0
        if self.enable_v_prune:
            if self.v_prune_threshold is not None:
                v_thr = float(self.v_prune_threshold)
            elif self.v_prune_num > 0 and K > self.v_prune_num:
                v_count = int(self.v_prune_num)
                if v_count > N.MAX_V_PRUNE_COUNT:
                    raise NotImplementedError(
                        f"v_prune_num={v_count}: at most {N.MAX_V_PRUNE_COUNT} keys per row by count")
        return v_thr, v_count

    @torch.no_grad()
    def forward(self, hidden_states, position_embeddings, attention_mask=None, past_key_values=None,
                **kwargs):
        if not hidden_states.is_cuda:
            raise ValueError("SpattenQwen3Attention runs on the CUDA kernels only")
        B, S, _ = hidden_states.shape
        if past_key_values is not None and past_key_values.get_seq_length(self.layer_idx) > 0:
            raise NotImplementedError("SpattenQwen3Attention: prefill only (the cache already holds keys)")
        H, Hkv, d = self.num_heads, self.num_kv_heads, self.head_dim
        dev = hidden_states.device
        cos, sin = position_embeddings
        q8 = qs = None
        if hidden_states.dtype in _DT and d in (64, 128):
            # QK-norm + RoPE (+ the query's int8) in one kernel: the HF
            # arithmetic without its dozen elementwise launches
            q, q8, qs, k = qk_norm_rope(self.q_proj(hidden_states), self.k_proj(hidden_states), self.q_norm,
                                        self.k_norm, cos, sin, H, Hkv, d, self.enable_prog_quant)
        else:
            q = self.q_norm(self.q_proj(hidden_states).view(B, S, H, d))
            k = self.k_norm(self.k_proj(hidden_states).view(B, S, Hkv, d))
            q, k = apply_rotary_pos_emb(q, k, cos, sin, unsqueeze_dim=2)
        v = self.v_proj(hidden_states).view(B, S, Hkv, d)

        st = self.cascade
        if self.layer_idx == 0 or st.positions is None or st.positions.shape[0] != B:
            st.positions = torch.arange(S, device=dev).expand(B, S).contiguous()
            st.cumulative = None
            st.kept_per_layer = []
        pos = st.positions
        K = pos.shape[1]
        if K < S:  # the kept keys: a gather of rows [B, S, Hkv*d] -> [B, K, Hkv*d]
            k = gather_rows(k.reshape(B, S, Hkv * d), pos).view(B, K, Hkv, d)
            v = gather_rows(v.contiguous().view(B, S, Hkv * d), pos).view(B, K, Hkv, d)
        else:
            k = k.contiguous()
            v = v.contiguous()
        # query position m sees the kept keys at positions <= m
        qpos = torch.arange(S, device=dev).expand(B, S).contiguous()
        key_limit = torch.searchsorted(pos, qpos, right=True).to(torch.int32)

        out = torch.empty(B, S, H, d, dtype=hidden_states.dtype, device=dev)
        v_thr, v_count = self._v_prune(K)
        qh = q.permute(0, 2, 1, 3) if q is not None else None  # [B, H, S, d] views
        kh = k.permute(0, 2, 1, 3)   # [B, Hkv, K, d]
        vh = v.permute(0, 2, 1, 3)
        common = dict(sm_scale=self.scaling, v_thr=v_thr, v_prune_count=v_count, key_limit=key_limit,
                      tok_in=st.cumulative, want_tok=True, out=out.permute(0, 2, 1, 3))
        if self.enable_prog_quant:
            if q8 is None:
                q8, qs = quant_q_int8(qh)
            kp = quant_k_planes(kh)
            r = prog_attn(q8, kp.msb, vh, k1=kp.lsb, mode=N.MODE_QUANT, q_scale=qs, k_scale=kp.scale,
                          refetch_thr=float(self.quant_threshold), want_refetch=True, **common)
            self.last_refetch = r.refetch
        else:
            r = prog_attn(qh, kh, vh, mode=N.MODE_DENSE, **common)
        cum = r.token_importance
        self.kept_positions = pos
        self.token_importance = cum
        st.kept_per_layer.append(K)

        if past_key_values is not None:
            # the cache concatenates into a new contiguous [B, Hkv, K, d] tensor
            # itself: the head-major views go in as they are (one copy, not two)
            past_key_values.update(kh, vh, self.layer_idx)

        if self.enable_token_prune:
            keep = keep_count(self.token_keep_ratio, K) if self.token_keep_ratio is not None \
                else max(1, K - int(self.token_prune_num))
            if keep < K:
                idx = topk_indices(cum, keep)
                st.positions = pos.gather(1, idx)
                st.cumulative = cum.gather(1, idx)
            else:
                st.positions, st.cumulative = pos, cum
        else:
            st.positions, st.cumulative = pos, cum
        return self.o_proj(out.view(B, S, H * d)), None


def patch_qwen3(model, **knobs):
    """Swap every decoder layer's self-attention for SpattenQwen3Attention
    (weights carried over with load_state_dict), share one cascade state
    across the layers, and set ``knobs`` on every layer. ``model`` is a HF
    Qwen3Model or Qwen3ForCausalLM."""
    base = model.model if hasattr(model, "model") else model
    state = CascadeState()
    for i, layer in enumerate(base.layers):
        old = layer.self_attn
        new = SpattenQwen3Attention(base.config, old.layer_idx)
        new.load_state_dict(old.state_dict())
        new.to(device=old.q_proj.weight.device, dtype=old.q_proj.weight.dtype)
        new.cascade = state
        for k, v in knobs.items():
            setattr(new, k, v)
        layer.self_attn = new
    return model
