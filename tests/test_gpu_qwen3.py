"""GPU parity of the Qwen3 prefill drop-in (spatten_b200.qwen3).

The reference has no Qwen3 code, so the bar is: with pruning off, HF's own
eager Qwen3 forward (1e-3 in fp32); with the cascade, the CPU oracle
(oracle/qwen3.py) -- the kept key positions identical at every layer, the
refetch flags identical, hidden states within 1e-3 (fp32); bf16 on the
tcgen05 kernel (head_dim 128, GQA, key_limit causality): the cascade's
structure and the KV cache contents.
"""
import copy

import numpy as np
import pytest
import torch

from oracle.qwen3 import spatten_qwen3_forward

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _ids(seed, B=2, S=300):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 1000, (B, S), generator=g)


def _patched(model, dtype=torch.float32, **knobs):
    from spatten_b200.qwen3 import patch_qwen3
    return patch_qwen3(copy.deepcopy(model).to(device="cuda", dtype=dtype).eval(), **knobs)


def _conditioned_ids(model, knobs, seeds=range(1, 40)):
    """Token ids whose keep decisions sit clear of ties (relative margin 1e-4
    between the last kept and the first dropped cumulative score) and whose
    refetch decisions are clear of the threshold."""
    for seed in seeds:
        ids = _ids(seed)
        rec = spatten_qwen3_forward(model, ids, **knobs)
        if rec["kth_gap"] > 1e-4 and rec["refetch_gap"] > 1e-4:
            return ids, rec
    pytest.fail("no well-conditioned input")


def test_qwen3_pruning_off_matches_hf(qwen3_model):
    ids = _ids(0)
    hf = copy.deepcopy(qwen3_model).cuda().eval()
    m = _patched(qwen3_model)
    with torch.no_grad():
        ref = hf(input_ids=ids.cuda()).last_hidden_state
        out = m(input_ids=ids.cuda()).last_hidden_state
    assert (out - ref).abs().max().item() < 1e-3


@pytest.mark.parametrize("v_thr", [None, 1e-3], ids=["no_vprune", "vprune"])
@pytest.mark.parametrize("quant", [False, True], ids=["dense", "prog_quant"])
def test_qwen3_cascade_matches_oracle(qwen3_model, quant, v_thr):
    """Kept positions and refetch flags exact; hidden states within 1e-3, or
    5e-3 with the V-prune threshold on: a probability within rounding of the
    threshold (the op-level tests allow 1e-4 relative) may be pruned by one
    implementation and kept by the other, moving an attention output by up to
    thr * |v|, which the later layers carry forward. With progressive
    quantisation 1e-2: the oracle computes Q and K on the CPU, the module on
    the GPU (RMSNorm, RoPE differ by an ulp), and an ulp on a value that sits
    on a rounding boundary of the int8 quantisation moves its code by one and
    a score by up to |q8| integer units (~0.6 % of a probability here); the
    op-level tests, which feed both sides the same int8 inputs, are exact."""
    knobs = dict(enable_token_prune=True, token_keep_ratio=0.8, enable_v_prune=v_thr is not None,
                 v_prune_threshold=v_thr, enable_prog_quant=quant, quant_threshold=0.1)
    ids, rec = _conditioned_ids(qwen3_model, knobs)
    m = _patched(qwen3_model, **knobs)
    with torch.no_grad():
        out = m(input_ids=ids.cuda()).last_hidden_state
    for i, layer in enumerate(m.layers):
        a = layer.self_attn
        assert np.array_equal(a.kept_positions.cpu().numpy(), rec["positions"][i]), i
        if quant:
            assert np.array_equal(a.last_refetch.cpu().numpy(), rec["refetch"][i]), i
    assert [layer.self_attn.kept_positions.shape[1] for layer in m.layers] == [300, 240, 192]
    tol = 1e-2 if quant else (1e-3 if v_thr is None else 5e-3)
    assert (out.cpu() - rec["last_hidden_state"]).abs().max().item() < tol


def test_qwen3_count_v_prune_matches_oracle(qwen3_model):
    knobs = dict(enable_token_prune=True, token_keep_ratio=0.8, enable_v_prune=True, v_prune_num=2)
    ids, rec = _conditioned_ids(qwen3_model, knobs)
    m = _patched(qwen3_model, **knobs)
    with torch.no_grad():
        out = m(input_ids=ids.cuda()).last_hidden_state
    for i, layer in enumerate(m.layers):
        assert np.array_equal(layer.self_attn.kept_positions.cpu().numpy(), rec["positions"][i]), i
    assert (out.cpu() - rec["last_hidden_state"]).abs().max().item() < 1e-3


def test_qwen3_bf16_cascade_and_kv_cache(qwen3_model):
    """bf16 on the tcgen05 kernel: the KV cache of layer i holds the keys and
    values layer i attended over (post-RoPE, HF layout), the kept counts follow
    the keep ratio and the kept positions stay sorted."""
    from transformers import DynamicCache
    knobs = dict(enable_token_prune=True, token_keep_ratio=0.8, enable_prog_quant=True,
                 quant_threshold=0.1)
    ids = _ids(3, B=2, S=520).cuda()
    m = _patched(qwen3_model, torch.bfloat16, **knobs)
    cache = DynamicCache(config=m.config)
    with torch.no_grad():
        out = m(input_ids=ids, past_key_values=cache, use_cache=True).last_hidden_state
    assert out.dtype == torch.bfloat16 and torch.isfinite(out.float()).all()
    K = 520
    for i, layer in enumerate(m.layers):
        a = layer.self_attn
        p = a.kept_positions
        assert p.shape == (2, K), i
        assert (p[:, 1:] > p[:, :-1]).all()
        kc, vc = cache.layers[i].keys, cache.layers[i].values
        assert tuple(kc.shape) == (2, 2, K, 128) and tuple(vc.shape) == (2, 2, K, 128)
        K = max(1, -(-4 * K // 5))
    # layer-0 keys in the cache = the HF module's RoPE'd, QK-normed keys (the
    # fused kernel sums the squares of a row in its own order: a value may sit
    # a rounding step away where the fp32 norm lands on a rounding boundary)
    from transformers.models.qwen3.modeling_qwen3 import apply_rotary_pos_emb
    a0 = m.layers[0].self_attn
    with torch.no_grad():
        h = m.layers[0].input_layernorm(m.embed_tokens(ids))
        q = a0.q_norm(a0.q_proj(h).view(2, 520, 4, 128))
        k = a0.k_norm(a0.k_proj(h).view(2, 520, 2, 128))
        pid = torch.arange(520, device="cuda")[None].expand(2, 520)
        cos, sin = m.rotary_emb(h, pid)
        _, k = apply_rotary_pos_emb(q, k, cos, sin, unsqueeze_dim=2)
    _assert_within_one_step(cache.layers[0].keys, k.permute(0, 2, 1, 3))


def _assert_within_one_step(got, ref, min_equal=0.999):
    """Equal but for a few elements a rounding step or two apart: a one-step
    difference of a normalised value (summation order of the squares) passes
    through RoPE's two rounded products and their rounded sum, so it is
    bounded by two steps at the scale of the row (its largest magnitude)."""
    g, r = got.float(), ref.float()
    bits = 7 if ref.dtype == torch.bfloat16 else 10
    tol = r.abs().amax(-1, keepdim=True) * 2.0 ** -bits * 2
    d = (g - r).abs()
    assert (d <= tol).all(), float((d / tol.clamp_min(1e-30)).max())
    assert (d == 0).float().mean().item() >= min_equal


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("quant", [True, False])
def test_qk_norm_rope_matches_hf_modules(qwen3_model, dt, quant):
    """The fused QK-norm + RoPE (+ query int8) kernel against the HF modules
    it replaces (Qwen3RMSNorm, apply_rotary_pos_emb) and spatten_quant_q_int8
    on the same projections: keys / queries equal but for rare differences of
    a rounding step or two at the row's scale, int8 queries within 1."""
    import spatten_b200 as sp
    from transformers.models.qwen3.modeling_qwen3 import apply_rotary_pos_emb
    from spatten_b200.qwen3 import qk_norm_rope
    m = copy.deepcopy(qwen3_model).to(device="cuda", dtype=dt).eval()
    a0 = m.layers[0].self_attn
    g = torch.Generator().manual_seed(11)
    with torch.no_grad():  # norm weights away from their all-ones init
        for w in (a0.q_norm.weight, a0.k_norm.weight):
            w.copy_((0.5 + torch.rand(w.shape, generator=g)).to(dt))
    ids = _ids(5, B=2, S=300).cuda()
    with torch.no_grad():
        h = m.layers[0].input_layernorm(m.embed_tokens(ids))
        pid = torch.arange(300, device="cuda")[None].expand(2, 300)
        cos, sin = m.rotary_emb(h, pid)
        qp, kp = a0.q_proj(h), a0.k_proj(h)
        H, Hk, D = a0.config.num_attention_heads, a0.config.num_key_value_heads, a0.head_dim
        q_ref = a0.q_norm(qp.view(2, 300, H, D))
        k_ref = a0.k_norm(kp.view(2, 300, Hk, D))
        q_ref, k_ref = apply_rotary_pos_emb(q_ref, k_ref, cos, sin, unsqueeze_dim=2)
        q, q8, qs, k = qk_norm_rope(qp, kp, a0.q_norm, a0.k_norm, cos, sin, H, Hk, D, quant)
    _assert_within_one_step(k, k_ref)
    if quant:
        rq8, rqs = sp.quant_q_int8(q_ref.permute(0, 2, 1, 3))
        dq = (q8.int() - rq8.int()).abs()
        assert dq.max().item() <= 1 and (dq == 0).float().mean().item() >= 0.999
        torch.testing.assert_close(qs, rqs, rtol=2.0 ** -7, atol=0)
    else:
        _assert_within_one_step(q, q_ref)
