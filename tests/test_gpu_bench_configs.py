"""GPU parity at the configurations bench.py measures.

Every number bench.py reports rests on these launches, so they are checked
at the benched shapes and precisions, against the oracle on the CPU:

* The op at the bench's own launch: batch 8 x 12 heads x S x 64, fp16 Q/K/V
  drawn N(0,1) from seed 1 (``bench.make_inputs``), refetch threshold 0.1, V
  prune 1e-3, token and head importance on, for S in {512, 2048, 4096, 8192}:
  the whole grid (two CTAs resident per SM, many waves). Checked: Q / K
  quantisation of every row bit-exact; refetch flag of every row; the exact
  integer score of a sample of rows of every (z, h) (a second launch writes
  rows m % 97 == 0 only, and must reproduce the first launch bit for bit);
  outputs of four (z, h) pairs in different CTAs and waves; token importance
  of one whole batch element (all 12 heads); the per-head |O| sums against
  the outputs the launch wrote.
* The BERT-base cascade in fp16 and bf16 on the path the bench times (fused
  QKV projection with Q / K quantised in its epilogue -> tcgen05 attention ->
  output projection on the compacted rows), batch 2 x 512, all knobs on,
  layer by layer. At each layer (i) the attention core against the oracle
  fed the layer's own int8 Q, K planes and V: refetch flags, token / head
  importance, context; (ii) the kept heads and tokens against the oracle's
  importance: identical wherever the decision is clear of the rounding band;
  (iii) the oracle's whole self-attention (fp32 projections) on the layer's
  input, upcast: the same decisions outside a wider band; (iv) the layer's
  tail (output projection, LayerNorm, FFN, the next layer's gather) against
  fp32 on the same context.
* The Qwen3 prefill in bf16 (Qwen3-0.6B attention geometry: hidden 1024, 16
  query / 8 KV heads, head_dim 128, QK-norm, RoPE theta 1e6), token keep 0.8,
  progressive quantisation 0.1, batch 2 x 2048, 4 layers: per layer the
  core with the layer's own operands (GQA, causal over the kept keys) and the
  kept key positions, then the oracle's whole attention from the upcast input.

A decision is "clear" when the oracle's value sits further than the band
from the k-th value (top-k) or the threshold (refetch): only there must the
kernel agree exactly, and the tests assert that such unclear decisions are
rare. Integer scores and quantised values have no band: they are exact.
"""
import copy
import math
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest
import torch

from oracle import prog_attn as opa
from oracle import quant as oq

pytestmark = pytest.mark.gpu

OUT_TOL = {torch.float16: 1e-2, torch.bfloat16: 2e-2}
TOK_RTOL = {torch.float16: 5e-4, torch.bfloat16: 4e-3}


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _pool_map(fn, items):
    with ThreadPoolExecutor(max_workers=max(1, min(len(items), os.cpu_count() or 1))) as ex:
        return list(ex.map(fn, items))


def _np(t):
    t = t.detach()
    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.float()  # numpy has no bf16
    return t.cpu().numpy()


def _chunk(n_keys):
    return max(128, (1 << 22) // max(1, n_keys))


def _decisions_match(gpu, ref_gap, what):
    """gpu == oracle everywhere except rows whose oracle value sits inside the
    band (``ref_gap`` = (oracle decision, ambiguous mask))."""
    ref, amb = ref_gap
    bad = (gpu != ref) & ~amb
    assert not bad.any(), f"{what}: {int(bad.sum())} clear decisions differ"
    assert amb.mean() < 1e-3, f"{what}: {amb.mean():.2e} of the decisions sit in the band"


def _topk_match(kept_idx, ref_vals, keep, band, what):
    """The kept set equals the oracle's top-``keep`` of ``ref_vals`` except for
    entries within ``band`` (relative) of the oracle's keep-th value."""
    kept_idx = np.asarray(kept_idx)
    ref_vals = np.asarray(ref_vals, np.float64)
    assert kept_idx.shape[-1] == keep, what
    for r in range(ref_vals.shape[0]):
        vals = ref_vals[r]
        kth = np.sort(vals)[::-1][keep - 1]
        tol = band * abs(kth) + 1e-12
        sel = np.zeros(vals.shape[0], bool)
        sel[kept_idx[r]] = True
        must_in = vals > kth + tol
        must_out = vals < kth - tol
        assert sel[must_in].all(), f"{what} row {r}: a clearly kept entry was dropped"
        assert not sel[must_out].any(), f"{what} row {r}: a clearly dropped entry was kept"


# --------------------------------------------------------------------- the op

OP_SEQS = [512, 2048, 4096, 8192]
SAMPLE_HEADS = [(0, 0), (2, 5), (5, 9), (7, 11)]  # (z, h): different CTAs and waves
TOK_BATCH = 3                                      # batch element checked over all heads
SCORE_ROW_STRIDE = 97                              # sampled rows: every query tile and lane quarter


@pytest.mark.parametrize("S", OP_SEQS)
def test_op_bench_launch_matches_oracle(S):
    import bench
    import spatten_b200 as sp
    from spatten_b200._native import MODE_QUANT
    q, k, v = bench.make_inputs(bench.SEED, S, torch)
    B, H, _, D = q.shape
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    q8, qs = sp.quant_q_int8(qd)
    kp = sp.quant_k_planes(kd)
    common = dict(mode=MODE_QUANT, q_scale=qs, k_scale=kp.scale, sm_scale=bench.SM_SCALE,
                  refetch_thr=bench.REFETCH_THR, v_thr=bench.V_THR, want_refetch=True)
    # the bench's launch (bench.py ours_arm: token and head importance on)
    r = sp.prog_attn(q8, kp.msb, vd, k1=kp.lsb, want_tok=True, want_head=True, **common)
    # the same grid again, writing the integer scores of rows m % 97 == 0
    rs = sp.prog_attn(q8, kp.msb, vd, k1=kp.lsb, want_scores=True, score_row_stride=SCORE_ROW_STRIDE,
                      **common)
    torch.cuda.synchronize()
    assert torch.equal(rs.out, r.out) and torch.equal(rs.refetch, r.refetch)

    # quantisation of every row
    q8n, sqn = oq.quant_rows_int8(q.float().numpy())
    assert np.array_equal(_np(q8), q8n) and np.array_equal(_np(qs), sqn)
    msb, lsb, skn = oq.quant_k_planes(k.float().numpy())
    assert np.array_equal(_np(kp.msb), msb) and np.array_equal(_np(kp.lsb), lsb)
    assert np.array_equal(_np(kp.scale), skn)

    vn = v.float().numpy()
    ch = _chunk(S)
    thr = bench.REFETCH_THR

    # refetch decision of every row of all B x H heads
    def decide(zh):
        z, h = zh
        return opa.quant_head(q8n[z, h], sqn[z, h], msb[z, h], lsb[z, h], skn[z, h], None,
                              bench.SM_SCALE, thr, decisions_only=True, chunk=ch)["maxprob"]
    mp = np.stack(_pool_map(decide, [(z, h) for z in range(B) for h in range(H)])).reshape(B, H, S)
    ref_flags = mp < thr
    _decisions_match(_np(r.refetch), (ref_flags, np.abs(mp - thr) <= 1e-4 * thr), "refetch")

    # sampled integer scores of every (z, h): the score the row used
    rows = np.arange(0, S, SCORE_ROW_STRIDE)
    sc = _np(rs.scores)
    flags = _np(r.refetch)
    k16 = (16 * oq.unpack_nibbles(msb, signed=True).astype(np.int16)).astype(np.int8)
    k8 = oq.k8_from_planes(msb, lsb)
    for z in range(B):
        for h in range(H):
            A = opa.int_scores(q8n[z, h, rows], k16[z, h])
            F = opa.int_scores(q8n[z, h, rows], k8[z, h])
            used = np.where(flags[z, h, rows][:, None], F, A)
            assert np.array_equal(sc[z, h], used), (z, h)

    # outputs of sampled heads and the token importance of one batch element
    heads = sorted(set(SAMPLE_HEADS) | {(TOK_BATCH, h) for h in range(H)})

    def full(zh):
        z, h = zh
        return zh, opa.quant_head(q8n[z, h], sqn[z, h], msb[z, h], lsb[z, h], skn[z, h], vn[z, h],
                                  bench.SM_SCALE, thr, bench.V_THR, chunk=ch)
    res = dict(_pool_map(full, heads))
    out = _np(r.out).astype(np.float32)
    for zh in SAMPLE_HEADS:
        o = res[zh]
        ok = ~(np.abs(o["maxprob"] - thr) <= 1e-4 * thr)  # rows whose decision is clear
        err = np.abs(out[zh][ok] - o["out"][ok]).max()
        assert err < OUT_TOL[torch.float16], (zh, err)
    tok = sum(res[(TOK_BATCH, h)]["tok"] for h in range(H))
    amb = sum(res[(TOK_BATCH, h)]["amb"] for h in range(H))
    got = _np(r.token_importance)[TOK_BATCH]
    allow = TOK_RTOL[torch.float16] * np.abs(tok) + 1e-6 + bench.V_THR * 1.001 * amb
    assert np.all(np.abs(got - tok) <= allow), np.max(np.abs(got - tok) - allow)
    # per-head |O| sums (the head importance) against the outputs written
    head_ref = r.out.float().abs().sum(dim=(0, 2, 3)).double().cpu().numpy()
    np.testing.assert_allclose(_np(r.head_abs_sum), head_ref, rtol=2e-3)


# ------------------------------------------------------------ BERT fp16 / bf16

BERT_TAIL_TOL = {torch.float16: 6e-2, torch.bfloat16: 4e-1}
BERT_UPCAST_BAND = {torch.float16: 2e-2, torch.bfloat16: 6e-2}


def _bert_models(dtype):
    import bench
    from transformers import BertConfig, BertModel
    from spatten_b200.bert import patch_bert
    torch.manual_seed(0)
    base = BertModel(BertConfig(attn_implementation="sdpa")).eval()
    gpu = patch_bert(copy.deepcopy(base).to("cuda", dtype).eval(), **bench.BERT_KNOBS)
    # the oracle runs on the device model's own (rounded) weights, in fp32
    ref = copy.deepcopy(base)
    ref.load_state_dict({k: v.float().cpu() for k, v in gpu.state_dict().items()})
    return gpu, ref.float().eval()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["fp16", "bf16"])
def test_bert_half_cascade_layerwise(dtype, monkeypatch):
    import bench
    import spatten_b200.bert as sb
    from oracle.bert import LayerKnobs, self_attention
    gpu, ref = _bert_models(dtype)
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(1000, 30522, (bench.BERT_B, bench.BERT_S), generator=g)[:2]

    cores, layers = [], []
    orig_pa, orig_fwd = sb.prog_attn, sb.SpattenBertSelfAttention.forward

    def pa(*a, **kw):
        r = orig_pa(*a, **kw)
        cores.append((a, kw, r))
        return r

    def fwd(self, hidden_states, attention_mask=None, **kw):
        heads = self.active_head_indices_for_this_layer
        cum = self.cumulative_token_score
        e = dict(hidden=hidden_states.clone(), heads=None if heads is None else heads.clone(),
                 cum=None if cum is None else cum.clone())
        out = orig_fwd(self, hidden_states, attention_mask, **kw)
        e.update(ctx=out[0].clone(), next_heads=self.next_active_head_indices.clone(),
                 next_tokens=self.next_active_token_indices.clone(),
                 cum_out=self.cumulative_token_score.clone(), refetch=self.last_refetch.clone(),
                 head_imp=self.last_head_importance.clone(), core=cores[-1])
        layers.append(e)
        return out

    monkeypatch.setattr(sb, "prog_attn", pa)
    monkeypatch.setattr(sb.SpattenBertSelfAttention, "forward", fwd)
    with torch.no_grad():
        final = gpu(input_ids=ids.cuda()).last_hidden_state
    assert len(layers) == 12
    kn = LayerKnobs(**bench.BERT_KNOBS)
    for i, e in enumerate(layers):
        a, kw, r = e["core"]
        q8, msb, v = _np(a[0]), _np(a[1]), _np(a[2]).astype(np.float32)
        lsb, qs, ks = _np(kw["k1"]), _np(kw["q_scale"]), _np(kw["k_scale"])
        tok_in = None if kw.get("tok_in") is None else _np(kw["tok_in"]).astype(np.float64)
        Bz, cur, S, _ = q8.shape
        heads = np.arange(12) if e["heads"] is None else _np(e["heads"])
        sm = kw["sm_scale"]
        ch = _chunk(S)

        # (i) the attention core on the layer's own operands
        def core(zh):
            z, h = zh
            return zh, opa.quant_head(q8[z, h], qs[z, h], msb[z, h], lsb[z, h], ks[z, h], v[z, h], sm,
                                      kn.quant_threshold, kn.v_prune_threshold, chunk=ch)
        res = dict(_pool_map(core, [(z, h) for z in range(Bz) for h in range(cur)]))
        mp = np.stack([[res[(z, h)]["maxprob"] for h in range(cur)] for z in range(Bz)])
        thr = kn.quant_threshold
        _decisions_match(_np(r.refetch), (mp < thr, np.abs(mp - thr) <= 1e-4 * thr), f"layer {i} refetch")
        ctx = _np(r.out).astype(np.float32)  # [B, 12 slots, S, d]
        for z in range(Bz):
            for h in range(cur):
                err = np.abs(ctx[z, heads[h]] - res[(z, h)]["out"]).max()
                assert err < OUT_TOL[dtype], (i, z, h, err)
        tok = np.stack([sum(res[(z, h)]["tok"] for h in range(cur)) for z in range(Bz)])
        amb = np.stack([sum(res[(z, h)]["amb"] for h in range(cur)) for z in range(Bz)])
        cum = tok + (tok_in if tok_in is not None else 0.0)
        allow = TOK_RTOL[dtype] * np.abs(cum) + 1e-6 + kn.v_prune_threshold * 1.001 * amb
        assert np.all(np.abs(_np(r.token_importance) - cum) <= allow), i
        head_abs = np.array([sum(res[(z, h)]["head_abs"] for z in range(Bz)) for h in range(cur)])
        np.testing.assert_allclose(_np(r.head_abs_sum), head_abs, rtol=5e-3)

        # (ii) decisions against the oracle's importance on the same operands
        keep_h = _np(e["next_heads"])
        pos_h = np.searchsorted(heads, keep_h)
        assert np.array_equal(heads[pos_h], keep_h)
        _topk_match(pos_h[None], (head_abs / (Bz * S * 64))[None], keep_h.size, 5e-3, f"layer {i} heads")
        _topk_match(_np(e["next_tokens"]), cum, e["next_tokens"].shape[1], 2 * TOK_RTOL[dtype] + 1e-3,
                    f"layer {i} tokens")

        # (iii) the oracle's whole self-attention on the layer's input, upcast
        hid = e["hidden"].float().cpu()
        cum_in = None if e["cum"] is None else e["cum"].float().cpu()
        heads_t = torch.from_numpy(heads).long()
        _, nh, nt, cum_o, info = self_attention(ref.encoder.layer[i].attention.self, hid, None, heads_t,
                                                cum_in, kn, tie_rule="smallest_index")
        agree = (info["refetch"] == _np(e["refetch"])).mean()
        assert agree > 0.99, (i, agree)
        band = BERT_UPCAST_BAND[dtype]
        _topk_match(_np(e["next_tokens"]), cum_o.numpy(), nt.shape[1], band, f"layer {i} tokens (upcast)")
        hi = info["head_importance"].numpy()
        _topk_match(pos_h[None], hi[None], keep_h.size, band, f"layer {i} heads (upcast)")

        # (iv) the layer's tail on the same context, in fp32, against the next input
        lay = ref.encoder.layer[i]
        with torch.no_grad():
            att = lay.attention.output(e["ctx"].float().cpu(), hid)
            h2 = lay.output(lay.intermediate(att), att)
        if i + 1 < len(layers):
            h2 = torch.gather(h2, 1, e["next_tokens"].cpu()[..., None].expand(-1, -1, h2.shape[-1]))
            nxt = layers[i + 1]["hidden"].float().cpu()
        else:
            nxt = final.float().cpu()
        err = (nxt - h2).abs().max().item()
        assert err < BERT_TAIL_TOL[dtype], (i, err)


# ----------------------------------------------------------------- Qwen3 bf16

def _qwen3_models():
    from transformers import Qwen3Config, Qwen3Model
    from spatten_b200.qwen3 import patch_qwen3
    cfg = Qwen3Config(vocab_size=4096, hidden_size=1024, intermediate_size=3072, num_hidden_layers=4,
                      num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                      max_position_embeddings=4096, rope_theta=1e6, tie_word_embeddings=True,
                      attn_implementation="sdpa")
    torch.manual_seed(0)
    base = Qwen3Model(cfg).eval()
    import bench
    gpu = patch_qwen3(copy.deepcopy(base).to("cuda", torch.bfloat16).eval(), **bench.QWEN3_KNOBS)
    ref = copy.deepcopy(base)
    ref.load_state_dict({k: v.float().cpu() for k, v in gpu.state_dict().items()})
    return gpu, ref.float().eval()


def test_qwen3_bf16_cascade_layerwise(monkeypatch):
    import bench
    import spatten_b200.qwen3 as sq
    from oracle.qwen3 import attention_layer
    gpu, ref = _qwen3_models()
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, 4096, (2, 2048), generator=g)
    cores, layers = [], []
    orig_pa, orig_fwd = sq.prog_attn, sq.SpattenQwen3Attention.forward

    def pa(*a, **kw):
        r = orig_pa(*a, **kw)
        cores.append((a, kw, r))
        return r

    def fwd(self, hidden_states, position_embeddings, *args, **kw):
        st = self.cascade
        pos = None if self.layer_idx == 0 else st.positions.clone()
        e = dict(hidden=hidden_states.clone(), cos=position_embeddings[0].clone(),
                 sin=position_embeddings[1].clone(), pos=pos)
        out = orig_fwd(self, hidden_states, position_embeddings, *args, **kw)
        e.update(core=cores[-1], positions=self.kept_positions.clone(), refetch=self.last_refetch.clone(),
                 next_pos=st.positions.clone(), cum=self.token_importance.clone())
        layers.append(e)
        return out

    monkeypatch.setattr(sq, "prog_attn", pa)
    monkeypatch.setattr(sq.SpattenQwen3Attention, "forward", fwd)
    with torch.no_grad():
        gpu(input_ids=ids.cuda())
    assert len(layers) == 4
    knobs = bench.QWEN3_KNOBS
    thr = knobs["quant_threshold"]
    for i, e in enumerate(layers):
        a, kw, r = e["core"]
        q8, msb, v = _np(a[0]), _np(a[1]), _np(a[2]).astype(np.float32)
        lsb, qs, ks = _np(kw["k1"]), _np(kw["q_scale"]), _np(kw["k_scale"])
        lim = _np(kw["key_limit"])
        tok_in = None if kw.get("tok_in") is None else _np(kw["tok_in"]).astype(np.float64)
        Bz, H, S, _ = q8.shape
        Hkv, K = msb.shape[1], msb.shape[2]
        sm = kw["sm_scale"]
        ch = _chunk(K)

        def core(zh):
            z, h = zh
            kh = h // (H // Hkv)
            return zh, opa.quant_head(q8[z, h], qs[z, h], msb[z, kh], lsb[z, kh], ks[z, kh], v[z, kh], sm,
                                      thr, kw["v_thr"], excl=opa._limit_mask(lim[z], K), chunk=ch)
        res = dict(_pool_map(core, [(z, h) for z in range(Bz) for h in range(H)]))
        mp = np.stack([[res[(z, h)]["maxprob"] for h in range(H)] for z in range(Bz)])
        _decisions_match(_np(r.refetch), (mp < thr, np.abs(mp - thr) <= 1e-4 * thr), f"layer {i} refetch")
        out = _np(r.out).astype(np.float32)
        for z in range(Bz):
            for h in range(H):
                err = np.abs(out[z, h] - res[(z, h)]["out"]).max()
                assert err < OUT_TOL[torch.bfloat16], (i, z, h, err)
        tok = np.stack([sum(res[(z, h)]["tok"] for h in range(H)) for z in range(Bz)])
        amb = np.stack([sum(res[(z, h)]["amb"] for h in range(H)) for z in range(Bz)])
        cum = tok + (tok_in if tok_in is not None else 0.0)
        allow = TOK_RTOL[torch.bfloat16] * np.abs(cum) + 1e-6 + kw["v_thr"] * 1.001 * amb
        assert np.all(np.abs(_np(r.token_importance) - cum) <= allow), i
        # kept key positions for the next layer: the top-k of the cumulative score
        pos = _np(e["positions"])
        keep = e["next_pos"].shape[1]
        nxt = _np(e["next_pos"])
        kept = np.stack([np.searchsorted(pos[z], nxt[z]) for z in range(Bz)])
        assert np.array_equal(np.take_along_axis(pos, kept, 1), nxt)
        _topk_match(kept, cum, keep, 2 * TOK_RTOL[torch.bfloat16] + 1e-3, f"layer {i} keys")
        # the oracle's whole attention (fp32 projections, QK-norm, RoPE) on the upcast input
        with torch.no_grad():
            ro, _ = attention_layer(ref.layers[i].self_attn, e["hidden"].float().cpu(),
                                    e["cos"].float().cpu(), e["sin"].float().cpu(), pos,
                                    enable_prog_quant=knobs["enable_prog_quant"], quant_threshold=thr)
        agree = (ro["refetch"] == _np(e["refetch"])).mean()
        assert agree > 0.98, (i, agree)
        cum_o = ro["tok"] + (tok_in if tok_in is not None else 0.0)
        _topk_match(kept, cum_o, keep, 8e-2, f"layer {i} keys (upcast)")
