"""Drop-in SpAtten cascade for Hugging Face BERT, running on the C-ABI kernels.

Same API as the reference:

* ``SpattenBertSelfAttention(config)`` -- subclass of HF ``BertSelfAttention``
  with the reference's knobs and cascade attributes
  (spatten_bert.py:15-37, spatten_bert_ultimate.py:128-152), loadable with
  ``load_state_dict(orig.state_dict())``; ``forward(hidden, attention_mask)``
  returns ``(context [B, S, hidden], None)``.
* ``spatten_encoder_forward(self, hidden_states, attention_mask=None, **kw)``
  -- the cascade encoder loop (module.py:40-99), bound with
  ``encoder.forward = spatten_encoder_forward.__get__(encoder, BertEncoder)``.
* ``slice_linear_weights(linear, active_indices, num_heads, head_dim)``
  (module.py:12-34), on the device gather kernel.
* ``patch_bert(model)`` does the module swap and the binding in one call.

With the batch sharded over ranks (``process_group`` on every attention
module), the head importance is all-reduced before the head top-k, so all
ranks keep the same heads as a single process would on the whole batch.

Knobs (per attention module): ``enable_head_prune``/``head_prune_num``,
``enable_token_prune``/``token_prune_num``, ``enable_v_prune``/``v_prune_num``,
``enable_prog_quant``/``quant_threshold`` as in the reference, plus the ratio
and threshold knobs ``head_keep_ratio``, ``token_keep_ratio`` (keep
``max(1, ceil(ratio * current))``, overriding the count) and
``v_prune_threshold`` (zero ``p < thr``; used instead of the count when set;
without it ``v_prune_num`` <= 16 zeroes that many smallest probabilities of
every row, ties to the smaller key index).
``quant_threshold`` is the row max-probability below which a row's LSB plane
is refetched (the reference used it as a tile logit bound).

On CUDA every step runs through libspatten_b200: for fp16 / bf16 models one
tensor-core kernel projects the active heads' Q/K/V straight from the full
weight (no slicing copy) and quantises Q and K in its epilogue (fp32 models:
head-row weight gather, one library GEMM, the quantisation kernels); then the
fused attention (mask, softmax, V prune, P.V, importance, scatter into the
full-width context) and the radix-select top-k for heads and tokens. There is
no CPU path: a CPU module raises.
"""
import math
from fractions import Fraction

import torch
import torch.nn.functional as F
from transformers.modeling_outputs import BaseModelOutputWithPastAndCrossAttentions
from transformers.models.bert.modeling_bert import BertEncoder, BertSelfAttention
from transformers.pytorch_utils import apply_chunking_to_forward

from . import _native as N
from .progressive import prog_attn, quant_k_planes, quant_q_int8
from .proj import LAYER_NORM_FEATURES, add_layer_norm, compact_out_proj, qkv_proj
from .select import gather_head_rows, gather_rows, select_heads, topk_indices


def keep_count(ratio, current):
    """``max(1, ceil(ratio * current))``, exact on the ratio's decimal repr."""
    r = Fraction(repr(float(ratio)))
    return max(1, math.ceil(r * current))


def slice_linear_weights(linear_layer, active_indices, num_heads, head_dim):
    """Rows of the active heads of a Linear (module.py:12-34): (W [h*d, in], b [h*d])."""
    w = linear_layer.weight
    b = linear_layer.bias
    if not w.is_cuda:
        raise ValueError("slice_linear_weights: CUDA module expected (no CPU path)")
    return gather_head_rows(w, active_indices, head_dim), gather_head_rows(b, active_indices, head_dim)


def _mask_bias(attention_mask, B, S, per_key=True):
    """HF mask as passed to the attention module -> additive bias view, or None.
    Float masks are additive (eager); bool masks mark kept keys (sdpa). An
    encoder's mask is a key (padding) mask repeated over the query rows, so
    with ``per_key`` a [B, 1, Sq, Sk] mask is read from its first row: the
    kernel then stages it per key tile instead of loading a bias per score
    (HF materialises the full mask, e.g. while a CUDA graph is captured)."""
    if attention_mask is None:
        return None
    m = attention_mask
    if m.dim() == 2:            # [B, S] 0/1 padding mask
        m = m[:, None, None, :].to(torch.bool) if m.dtype != torch.bool else m[:, None, None, :]
    if m.dim() == 3:
        m = m[:, None]
    if per_key and m.dim() == 4 and m.shape[2] > 1:
        m = m[:, :, :1, :]
    if m.dtype == torch.bool:
        return torch.zeros(m.shape, dtype=torch.float32, device=m.device).masked_fill_(
            ~m, torch.finfo(torch.float32).min)
    return m.float()


class SpattenBertSelfAttention(BertSelfAttention):
    """HF BertSelfAttention with the SpAtten cascade, on the B200 kernels."""

    def __init__(self, config, *args, **kwargs):
        super().__init__(config, *args, **kwargs)
        self.layer_id = 0
        self.num_heads = config.num_attention_heads
        self.head_dim = int(config.hidden_size // config.num_attention_heads)
        # reference knobs
        self.head_prune_num = 0
        self.enable_head_prune = False
        self.next_active_head_indices = None
        self.next_active_head_indices32 = None  # int32 copy (the next layer's head-slot map)
        self.active_head_indices_for_this_layer = None
        self.enable_token_prune = False
        self.token_prune_num = 0
        self.cumulative_token_score = None
        self.next_active_token_indices = None
        self.enable_v_prune = False
        self.v_prune_num = 2
        self.enable_prog_quant = False
        self.quant_threshold = 1.0
        # ratio / threshold knobs
        self.head_keep_ratio = None
        self.token_keep_ratio = None
        self.v_prune_threshold = None
        # batch sharded over ranks: all-reduce head importance over this group
        # (the reference's head decision is batch-global)
        self.process_group = None
        # encoder loop: run this layer's output projection, LayerNorm and FFN
        # on the tokens the next layer keeps only (fp16 / bf16, eval mode)
        self.compact_ffn = True
        # diagnostics of the last forward
        self.last_refetch = None
        self.last_head_importance = None
        self._qkv_cache = None

    def _qkv_params(self):
        key = tuple((p.data_ptr(), p._version) for p in (
            self.query.weight, self.key.weight, self.value.weight,
            self.query.bias, self.key.bias, self.value.bias))
        if self._qkv_cache is None or self._qkv_cache[0] != key:
            w = torch.cat([self.query.weight, self.key.weight, self.value.weight], 0).detach()
            b = torch.cat([self.query.bias, self.key.bias, self.value.bias], 0).detach()
            self._qkv_cache = (key, w, b)
        return self._qkv_cache[1], self._qkv_cache[2]

    def _prune_counts(self, cur_heads, seq_len):
        hp = self.head_prune_num
        if self.head_keep_ratio is not None:
            hp = cur_heads - keep_count(self.head_keep_ratio, cur_heads)
        tp = self.token_prune_num
        if self.token_keep_ratio is not None:
            tp = seq_len - keep_count(self.token_keep_ratio, seq_len)
        return hp, tp

    @torch.no_grad()
    def forward(self, hidden_states, attention_mask=None, **kwargs):
        if not hidden_states.is_cuda:
            raise ValueError("SpattenBertSelfAttention runs on the CUDA kernels only")
        dev = hidden_states.device
        B, S, _ = hidden_states.shape
        H, d = self.num_heads, self.head_dim
        heads = self.active_head_indices_for_this_layer
        if heads is None:
            heads = torch.arange(H, device=dev)
        cur = heads.numel()
        # the int32 copy of `heads` that the encoder loop handed over with it
        # (the attention kernel's head-slot map); else prog_attn converts
        h32 = getattr(self, "_heads32", None)
        head_map = h32[1] if (h32 is not None and h32[0] is heads) else heads
        w, b = self._qkv_params()
        fused = hidden_states.dtype in (torch.float16, torch.bfloat16) and d in (64, 128)
        if fused:
            # one tensor-core kernel: the active heads' weight tiles read in
            # place (no slicing copy), Q / K quantised in its epilogue
            pr = qkv_proj(hidden_states, w, b, H, d, heads=heads, quantize=self.enable_prog_quant)
            v = pr.v                                       # [B, cur, S, d]
        else:
            # head-row gather of the concatenated Q/K/V weights, one GEMM
            rows = torch.cat([heads, heads + H, heads + 2 * H])
            wsel = gather_head_rows(w, rows, d)
            bsel = gather_head_rows(b, rows, d)
            qkv = F.linear(hidden_states, wsel, bsel)      # [B, S, 3*cur*d]
            qkv4 = qkv.view(B, S, 3, cur, d)
            q = qkv4[:, :, 0].permute(0, 2, 1, 3)          # [B, cur, S, d] strided views
            k = qkv4[:, :, 1].permute(0, 2, 1, 3)
            v = qkv4[:, :, 2].permute(0, 2, 1, 3)
        bias = _mask_bias(attention_mask, B, S, per_key=not getattr(self, "is_decoder", False))
        v_thr, v_count = 0.0, 0
        if self.enable_v_prune:
            if self.v_prune_threshold is not None:
                v_thr = float(self.v_prune_threshold)
            elif self.v_prune_num > 0 and S > self.v_prune_num:
                # the reference's rule (spatten_bert.py:100-113): zero the
                # v_prune_num smallest probabilities of every row
                v_count = int(self.v_prune_num)
                if v_count > N.MAX_V_PRUNE_COUNT:
                    raise NotImplementedError(
                        f"v_prune_num={v_count}: the B200 path prunes at most "
                        f"{N.MAX_V_PRUNE_COUNT} keys per row by count; use v_prune_threshold")
        # the context of the pruned heads reads as zeros (every head slot is
        # written when all heads are active)
        alloc = torch.empty if cur == H else torch.zeros
        full = alloc(B, S, H, d, dtype=hidden_states.dtype, device=dev)
        cum = self.cumulative_token_score
        common = dict(sm_scale=1.0 / math.sqrt(d), v_thr=v_thr, v_prune_count=v_count, bias=bias,
                      tok_in=cum,
                      want_tok=True, want_head=True, out=full.permute(0, 2, 1, 3),
                      out_head_map=head_map, out_head_slots=H)
        if self.enable_prog_quant:
            if fused:
                q8, qs, kp = pr.q8, pr.q_scale, pr.k_planes
            else:
                q8, qs = quant_q_int8(q)
                kp = quant_k_planes(k)
            r = prog_attn(q8, kp.msb, v, k1=kp.lsb, mode=N.MODE_QUANT, q_scale=qs,
                          k_scale=kp.scale, refetch_thr=float(self.quant_threshold),
                          want_refetch=True, **common)
            self.last_refetch = r.refetch
        else:
            if fused:
                q, k = pr.q, pr.k
            r = prog_attn(q, k, v, mode=N.MODE_DENSE, **common)
        if self.process_group is not None:
            from .distributed import allreduce_head_importance
            head_raw = allreduce_head_importance(r.head_abs_sum, B * S * d, self.process_group)
            scale = 1.0
        else:
            head_raw, scale = r.head_abs_sum, 1.0 / float(B * S * d)
        hp, tp = self._prune_counts(cur, S)
        next_heads, next32 = heads, head_map
        if self.enable_head_prune and cur > hp:
            keep = max(1, cur - hp)
            # importance, top-k and heads[pos] in one launch, with the int32
            # copy of the next heads that the next layer's head-slot map reads
            head_imp, next_heads, next32 = select_heads(head_raw, scale, heads, keep)
        else:
            head_imp = head_raw * scale if scale != 1.0 else head_raw
        self.last_head_importance = head_imp
        self.next_active_head_indices = next_heads
        self.next_active_head_indices32 = next32
        self.cumulative_token_score = r.token_importance
        next_tokens = None
        if self.enable_token_prune and S > tp:
            keep = max(1, S - tp)
            next_tokens = topk_indices(self.cumulative_token_score, keep)
        self.next_active_token_indices = next_tokens
        return (full.view(B, S, H * d), None)


def _compactable(layer, attn, hidden_states, last):
    """Whether the layer's tail (output projection, LayerNorm, FFN) can run on
    the kept tokens only: a row-wise tail in eval mode (no dropout), fp16 /
    bf16, head_dim a multiple of 64, hidden a multiple of 32, and a next layer
    to take the compacted rows."""
    if last or attn.training or not getattr(attn, "compact_ffn", False) or not attn.enable_token_prune:
        return False
    if getattr(layer, "is_decoder", False) or not hasattr(layer, "feed_forward_chunk"):
        return False
    so = getattr(layer.attention, "output", None)
    if so is None or not hasattr(so, "dense") or not hasattr(so, "LayerNorm"):
        return False
    return (hidden_states.is_cuda and hidden_states.dtype in (torch.float16, torch.bfloat16)
            and so.dense.weight.dtype == hidden_states.dtype and attn.head_dim % 64 == 0
            and hidden_states.shape[-1] % 32 == 0)


def _ln_fusable(ln, x):
    """Whether ``ln`` (an nn.LayerNorm over x's last dimension) can run as
    spatten_add_layer_norm."""
    return (isinstance(ln, torch.nn.LayerNorm) and ln.elementwise_affine and ln.weight is not None
            and ln.bias is not None and tuple(ln.normalized_shape) == (x.shape[-1],)
            and x.shape[-1] in LAYER_NORM_FEATURES and ln.weight.dtype == x.dtype
            and ln.bias.dtype == x.dtype)


def _layer_tail(layer, attn, ctx, hidden_states, kept):
    """HF BertLayer after its self-attention (BertSelfOutput, then the FFN
    chunk). With ``kept`` the next layer's token gather (module.py:49-54)
    runs first, folded into the output projection's row loads
    (``compact_out_proj``): every step of the tail is row-wise, so its rows
    for the kept tokens are the reference's rows, and the FFN skips the rows
    the next layer drops. The LayerNorms (and BertOutput's residual add) run
    as spatten_add_layer_norm; the FFN's dense layers and GELU stay HF's
    modules."""
    so = layer.attention.output
    if kept is None:
        a = so(ctx, hidden_states)
    else:
        y = compact_out_proj(ctx, hidden_states, kept, so.dense.weight, so.dense.bias,
                             attn.num_heads, attn.head_dim, heads=attn.active_head_indices_for_this_layer)
        ln = so.LayerNorm
        a = add_layer_norm(y, ln.weight, ln.bias, ln.eps) if _ln_fusable(ln, y) else ln(y)
    out = layer.output
    if (layer.chunk_size_feed_forward == 0 and hasattr(layer, "intermediate") and hasattr(out, "dense")
            and not out.training and _ln_fusable(getattr(out, "LayerNorm", None), a)):
        # BertOutput: LayerNorm(dense(intermediate) + a), dropout off in eval
        h = out.dense(layer.intermediate(a))
        return add_layer_norm(h, out.LayerNorm.weight, out.LayerNorm.bias, out.LayerNorm.eps, residual=a)
    return apply_chunking_to_forward(layer.feed_forward_chunk, layer.chunk_size_feed_forward,
                                     layer.seq_len_dim, a)


def spatten_encoder_forward(self, hidden_states, attention_mask=None, **kwargs):
    """Cascade encoder loop (module.py:40-99): per layer, compact the kept
    tokens' hidden states, key mask and cumulative score, hand the active
    heads and the score to the attention module, run the layer, and read its
    decisions back. In eval mode on fp16 / bf16 a layer whose attention chose
    the next layer's tokens runs its tail on those tokens only
    (``_layer_tail``), so the next layer's hidden states arrive compacted and
    are not gathered again (``compact_ffn = False`` on the attention module
    turns this off)."""
    active_heads = None
    active_heads32 = None
    active_tokens = None
    cumulative = None
    compacted = False
    n_layers = len(self.layer)
    if attention_mask is not None:
        # the key mask as an additive fp32 bias [B, 1, 1, S], converted once:
        # the layers gather its kept columns and read it as it is
        B0 = hidden_states.shape[0]
        attention_mask = _mask_bias(attention_mask, B0, hidden_states.shape[1]).expand(B0, -1, -1, -1)
        if attention_mask.shape[2] > 1:
            attention_mask = attention_mask[:, :, :1, :]
        attention_mask = attention_mask.contiguous()
    for i, layer in enumerate(self.layer):
        if active_tokens is not None:
            if not compacted:
                hidden_states = gather_rows(hidden_states, active_tokens)
            if attention_mask is not None:
                m = attention_mask
                if m.dim() == 4:      # [B, 1, Sq, Sk] -> key mask of query row 0, [B, 1, 1, K]
                    m = m[:, :, :1, :]
                attention_mask = gather_rows(m.reshape(m.shape[0], -1).unsqueeze(-1),
                                             active_tokens).reshape(m.shape[0], 1, 1, -1)
            if cumulative is not None:
                cumulative = gather_rows(cumulative, active_tokens)
        attn = layer.attention.self
        attn.active_head_indices_for_this_layer = active_heads
        attn._heads32 = (active_heads, active_heads32) if active_heads is not None else None
        attn.cumulative_token_score = cumulative
        if _compactable(layer, attn, hidden_states, last=(i == n_layers - 1)):
            ctx, _ = attn(hidden_states, attention_mask=attention_mask, **kwargs)
            kept = attn.next_active_token_indices
            hidden_states = _layer_tail(layer, attn, ctx, hidden_states, kept)
            compacted = kept is not None
        else:
            out = layer(hidden_states, attention_mask=attention_mask, **kwargs)
            hidden_states = out[0] if isinstance(out, (tuple, list)) else out
            compacted = False
        active_heads = attn.next_active_head_indices
        active_heads32 = getattr(attn, "next_active_head_indices32", None)
        active_tokens = attn.next_active_token_indices
        cumulative = attn.cumulative_token_score
    return BaseModelOutputWithPastAndCrossAttentions(
        last_hidden_state=hidden_states, past_key_values=None, hidden_states=None,
        attentions=None, cross_attentions=None)


def patch_bert(model, **knobs):
    """Swap every layer's self-attention for SpattenBertSelfAttention (weights
    carried over with load_state_dict, spatten_bert_ultimate.py:294-298),
    bind the cascade encoder loop (:300) and set ``knobs`` on every layer.
    ``process_group=`` makes the head decision global over a batch sharded
    across the group's ranks."""
    for i, layer in enumerate(model.encoder.layer):
        old = layer.attention.self
        new = SpattenBertSelfAttention(model.config)
        new.load_state_dict(old.state_dict())
        new.layer_id = i
        new.to(device=old.query.weight.device, dtype=old.query.weight.dtype)
        new.train(old.training)  # a fresh module is in training mode; keep the model's
        for k, v in knobs.items():
            setattr(new, k, v)
        layer.attention.self = new
    model.encoder.forward = spatten_encoder_forward.__get__(model.encoder, BertEncoder)
    return model
