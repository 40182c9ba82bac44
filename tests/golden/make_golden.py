"""Generate the golden fixtures in this folder by running the reference itself.

Run from the repository root, where the reference checkout is readable:

    python tests/golden/make_golden.py /root/reference

It imports the reference's own modules unchanged (``module.py``,
``spatten_bert.py``, ``spatten_bert_ultimate.py``,
``spatten_progressive_attention.py``) and runs them on the CPU; the Triton
kernels run under the Triton CPU interpreter (``TRITON_INTERPRET=1``). The
outputs are stored as small ``.npz`` files next to this script. The tests
read only those files; nothing at test time needs the reference.

Fixtures:

* ``bert_cascade.npz`` -- BERT-base (random init, seed 0, eager masks, fp32)
  through the reference's ``spatten_encoder_forward`` +
  ``spatten_bert.SpattenBertSelfAttention``: pruning off, the reference's
  count knobs (the 0.9 ratios translated per layer),
  the count V-prune at v_prune_num = 2 (the module's default) and 16 (the
  reference's benchmark setting, benchmark_seq_len.py), and a padded batch.
* ``prog_compat.npz`` -- ``triton_progressive_qk`` (tile 32x32) at thresholds
  +100 / -100 / a mid value, and ``spatten_progressive_attention`` (tile
  64x64) at N=64 where it is exact.
* ``prog_quant_extremes.npz`` -- int8 planes dequantised into float planes
  fed to ``triton_progressive_qk`` at +100 (always refetch) and -100 (never).
"""
import copy
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.bert import keep_count  # noqa: E402
from oracle import quant as oq  # noqa: E402


def build_bert(seed=0, n_layers=12, max_pos=512):
    from transformers import BertConfig, BertModel
    torch.manual_seed(seed)
    cfg = BertConfig(attn_implementation="eager", num_hidden_layers=n_layers,
                     max_position_embeddings=max_pos)
    return BertModel(cfg).eval()


def cascade_schedule(n_layers, seq, heads, tok_ratio, head_ratio):
    """Per-layer (token_prune_num, head_prune_num) equivalent to the ratios."""
    out = []
    s, h = seq, heads
    for _ in range(n_layers):
        tp = s - keep_count(tok_ratio, s)
        hp = h - keep_count(head_ratio, h)
        out.append((tp, hp))
        s, h = s - tp, h - hp
    return out


def ref_bert_run(ref_root, model, ids, mask, schedule, v_prune_num=None):
    sys.path.insert(0, ref_root)
    from module import spatten_encoder_forward
    from spatten_bert import SpattenBertSelfAttention
    from transformers.models.bert.modeling_bert import BertEncoder
    m = copy.deepcopy(model)
    for i, layer in enumerate(m.encoder.layer):
        sd = layer.attention.self.state_dict()
        a = SpattenBertSelfAttention(m.config)
        a.load_state_dict(sd)
        a.layer_id = i
        if schedule is not None:
            tp, hp = schedule[i]
            a.enable_head_prune = True
            a.head_prune_num = hp
            a.enable_token_prune = True
            a.token_prune_num = tp
        if v_prune_num is not None:
            a.enable_v_prune = True
            a.v_prune_num = v_prune_num
        layer.attention.self = a
    m.encoder.forward = spatten_encoder_forward.__get__(m.encoder, BertEncoder)
    m.eval()
    with torch.no_grad():
        out = m(input_ids=ids, attention_mask=mask).last_hidden_state
    heads, toks = [], []
    for layer in m.encoder.layer:
        a = layer.attention.self
        heads.append(a.next_active_head_indices.numpy().copy())
        t = a.next_active_token_indices
        toks.append(None if t is None else t.numpy().copy())
    return out.numpy(), heads, toks


def make_bert(ref_root):
    model = build_bert()
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(1000, 30522, (1, 128), generator=g)
    mask = torch.ones(1, 128, dtype=torch.long)
    sched = cascade_schedule(12, 128, 12, 0.9, 0.9)
    res = {"ids": ids.numpy(), "schedule": np.array(sched)}
    off, _, _ = ref_bert_run(ref_root, model, ids, mask, None)
    res["off_out"] = off
    for tag, vp in (("casc", None), ("cascv", 2), ("cascv16", 16)):
        out, heads, toks = ref_bert_run(ref_root, model, ids, mask, sched, vp)
        res[f"{tag}_out"] = out
        for i, (h, t) in enumerate(zip(heads, toks)):
            res[f"{tag}_heads_{i}"] = h
            res[f"{tag}_tokens_{i}"] = t
    # padded batch of two, seq 64, second row padded after 48 tokens
    g = torch.Generator().manual_seed(1)
    ids2 = torch.randint(1000, 30522, (2, 64), generator=g)
    mask2 = torch.ones(2, 64, dtype=torch.long)
    mask2[1, 48:] = 0
    sched2 = cascade_schedule(12, 64, 12, 0.9, 0.9)
    out, heads, toks = ref_bert_run(ref_root, model, ids2, mask2, sched2)
    res["pad_ids"] = ids2.numpy()
    res["pad_mask"] = mask2.numpy()
    res["pad_schedule"] = np.array(sched2)
    res["pad_out"] = out
    for i, (h, t) in enumerate(zip(heads, toks)):
        res[f"pad_heads_{i}"] = h
        res[f"pad_tokens_{i}"] = t
    np.savez_compressed(os.path.join(HERE, "bert_cascade.npz"), **res)
    print("bert_cascade.npz", {k: v.shape for k, v in res.items() if k.endswith("_out")})


def make_compat(ref_root):
    sys.path.insert(0, ref_root)
    from spatten_bert_ultimate import triton_progressive_qk
    from spatten_progressive_attention import spatten_progressive_attention
    res = {}
    g = torch.Generator().manual_seed(3)
    Z, H, M, N, D = 1, 2, 96, 128, 64
    q = torch.randn(Z, H, M, D, generator=g).half()
    km = (torch.randn(Z, H, N, D, generator=g) * 0.8).half()
    kl = (torch.randn(Z, H, N, D, generator=g) * 0.2).half()
    v = torch.randn(Z, H, N, D, generator=g).half()
    res.update(q=q.numpy(), k_msb=km.numpy(), k_lsb=kl.numpy(), v=v.numpy())
    # tile maxima of the scaled MSB score, to place a mid threshold between them
    s = (q.float() @ km.float().transpose(-1, -2)) * 0.125
    tmax = s.view(Z, H, M // 32, 32, N // 32, 32).amax(dim=(3, 5)).flatten().sort().values
    mid = float((tmax[tmax.numel() // 2 - 1] + tmax[tmax.numel() // 2]) / 2)
    for tag, thr in (("hi", 100.0), ("lo", -100.0), ("mid", mid)):
        res[f"out_{tag}"] = triton_progressive_qk(q, km, kl, v, thr, 0.125).float().numpy()
        res[f"thr_{tag}"] = np.float32(thr)
    # the standalone 64x64 kernel is exact only for N <= 64
    q6, k6m, k6l, v6 = (x[:, :, :64].contiguous() for x in (q, km, kl, v))
    s6 = (q6.float() @ k6m.float().transpose(-1, -2)) * 0.125
    mx = float(s6.amax(dim=(2, 3))[0, 0])
    for tag, thr in (("hi", 100.0), ("lo", -100.0), ("h0", mx + 0.01)):
        res[f"spa_out_{tag}"] = spatten_progressive_attention(q6, k6m, k6l, v6, threshold=thr).float().numpy()
        res[f"spa_thr_{tag}"] = np.float32(thr)
    np.savez_compressed(os.path.join(HERE, "prog_compat.npz"), **res)
    print("prog_compat.npz", sorted(res))


def make_quant_extremes(ref_root):
    sys.path.insert(0, ref_root)
    from spatten_bert_ultimate import triton_progressive_qk
    g = torch.Generator().manual_seed(4)
    Z, H, N, D = 1, 2, 128, 64
    q = torch.randn(Z, H, N, D, generator=g).half()
    k = torch.randn(Z, H, N, D, generator=g).half()
    v = torch.randn(Z, H, N, D, generator=g).half()
    q8, sq = oq.quant_rows_int8(q.float().numpy())
    msb_p, lsb_p, sk = oq.quant_k_planes(k.float().numpy())
    msb = oq.unpack_nibbles(msb_p, signed=True).astype(np.float32)
    lsb = oq.unpack_nibbles(lsb_p, signed=False).astype(np.float32)
    qd = torch.from_numpy(q8.astype(np.float32) * sq[..., None])
    kmd = torch.from_numpy(16.0 * msb * sk[..., None])
    kld = torch.from_numpy(lsb * sk[..., None])
    res = dict(q=q.numpy(), k=k.numpy(), v=v.numpy())
    res["out_always"] = triton_progressive_qk(qd, kmd, kld, v.float(), 100.0, 0.125).numpy()
    res["out_never"] = triton_progressive_qk(qd, kmd, kld, v.float(), -100.0, 0.125).numpy()
    np.savez_compressed(os.path.join(HERE, "prog_quant_extremes.npz"), **res)
    print("prog_quant_extremes.npz", sorted(res))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the reference checkout>")
    ref = sys.argv[1]
    make_compat(ref)
    make_quant_extremes(ref)
    make_bert(ref)
