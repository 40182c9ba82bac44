"""GPU parity of the fused Q/K/V projection (spatten_b200.proj.qkv_proj, the
C ABI's spatten_qkv_proj) against the oracle (oracle/proj.py: the reference's
head-row slicing + projections + the int8 / 4-bit-plane quantisation).

The kernel accumulates in fp32 on the tensor cores, the oracle in float64:
a projection may round to the neighbouring fp16 / bf16 value, which can move
a quantised value by one step. Bounds: projections within 1 ulp of the
activation type (rtol 2^-8 fp16, 2^-7 bf16 plus a small atol), quantised
values within 1 of the oracle's and equal for >= 99 % of them, scales within
one ulp of the max element (relative 2^-8)."""
import numpy as np
import pytest
import torch

from oracle.proj import qkv_proj as oracle_proj
from oracle.quant import k8_from_planes

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


RTOL = {torch.float16: 2.0 ** -8, torch.bfloat16: 2.0 ** -7}
DT = {torch.float16: "f16", torch.bfloat16: "bf16"}


def _inputs(B, S, K, H, D, dt, seed, bias=True):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, S, K, generator=g).to(dt)
    w = (torch.randn(3 * H * D, K, generator=g) / K ** 0.5).to(dt)
    b = (torch.randn(3 * H * D, generator=g) * 0.1).to(dt) if bias else None
    return x, w, b


def _close(got, ref, dt):
    got = got.float().cpu().numpy()
    np.testing.assert_allclose(got, ref, rtol=RTOL[dt], atol=1e-3)


CASES = [
    # B, S, K, H, D, heads (None = all), dtype, bias
    (2, 100, 768, 12, 64, [0, 2, 3, 5, 6, 7, 8, 9, 10, 11, 1], torch.float16, True),
    (1, 300, 768, 12, 64, None, torch.float16, True),
    (3, 77, 1024, 8, 128, None, torch.bfloat16, True),
    (2, 129, 1024, 8, 128, [7, 1, 4], torch.float16, False),
    (1, 64, 256, 4, 64, [3], torch.bfloat16, True),
]


@pytest.mark.parametrize("case", CASES)
def test_qkv_proj_quant_matches_oracle(case):
    from spatten_b200.proj import qkv_proj
    B, S, K, H, D, heads, dt, bias = case
    x, w, b = _inputs(B, S, K, H, D, dt, seed=S + K)
    hl = list(range(H)) if heads is None else heads
    ht = None if heads is None else torch.tensor(heads, device="cuda")
    r = qkv_proj(x.cuda(), w.cuda(), None if b is None else b.cuda(), H, D, heads=ht, quantize=True)
    torch.cuda.synchronize()
    o = oracle_proj(x.float().numpy(), w.float().numpy(), None if b is None else b.float().numpy(), H, D, hl,
                    DT[dt])
    _close(r.v, o["v"], dt)
    q8 = r.q8.cpu().numpy().astype(np.int16)
    dq = np.abs(q8 - o["q8"].astype(np.int16))
    assert dq.max() <= 1 and (dq == 0).mean() >= 0.99
    np.testing.assert_allclose(r.q_scale.cpu().numpy(), o["q_scale"], rtol=2.0 ** -8, atol=0)
    k8 = k8_from_planes(r.k_planes.msb.cpu().numpy(), r.k_planes.lsb.cpu().numpy()).astype(np.int16)
    rk8 = k8_from_planes(o["k_msb"], o["k_lsb"]).astype(np.int16)
    dk = np.abs(k8 - rk8)
    assert dk.max() <= 1 and (dk == 0).mean() >= 0.99
    np.testing.assert_allclose(r.k_planes.scale.cpu().numpy(), o["k_scale"], rtol=2.0 ** -8, atol=0)


def test_qkv_proj_quantises_its_own_projection_exactly():
    """The epilogue's quantisation is the quant kernels' arithmetic, bit for
    bit: quantising the dense mode's rounded Q and K with spatten_quant_*
    gives the quant mode's outputs exactly (same GEMM, same rounding)."""
    import spatten_b200 as sp
    from spatten_b200.proj import qkv_proj
    x, w, b = _inputs(2, 200, 768, 12, 64, torch.float16, seed=5)
    x, w, b = x.cuda(), w.cuda(), b.cuda()
    heads = torch.tensor([4, 0, 9, 2, 11], device="cuda")
    rq = qkv_proj(x, w, b, 12, 64, heads=heads, quantize=True)
    rd = qkv_proj(x, w, b, 12, 64, heads=heads, quantize=False)
    assert torch.equal(rq.v, rd.v)
    q8, qs = sp.quant_q_int8(rd.q)
    assert torch.equal(q8, rq.q8) and torch.equal(qs, rq.q_scale)
    kp = sp.quant_k_planes(rd.k)
    assert torch.equal(kp.msb, rq.k_planes.msb) and torch.equal(kp.lsb, rq.k_planes.lsb)
    assert torch.equal(kp.scale, rq.k_planes.scale)


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_qkv_proj_dense_matches_torch(dt):
    """Dense mode against torch's own F.linear of the sliced weights (the
    reference's path), within one ulp."""
    from spatten_b200.proj import qkv_proj
    B, S, K, H, D = 2, 150, 768, 12, 64
    x, w, b = _inputs(B, S, K, H, D, dt, seed=11)
    x, w, b = x.cuda(), w.cuda(), b.cuda()
    heads = torch.tensor([1, 3, 5, 7, 9, 11, 0], device="cuda")
    r = qkv_proj(x, w, b, H, D, heads=heads, quantize=False)
    for which, got in enumerate((r.q, r.k, r.v)):
        rows = (which * H * D + heads[:, None] * D + torch.arange(D, device="cuda")[None, :]).reshape(-1)
        ref = torch.nn.functional.linear(x, w[rows], b[rows])
        ref = ref.view(B, S, heads.numel(), D).permute(0, 2, 1, 3)
        torch.testing.assert_close(got.float(), ref.float(), rtol=RTOL[dt], atol=2e-3)


# --- attention output projection of the kept tokens (spatten_compact_out_proj) ----

OUT_CASES = [
    # B, S, L (kept), H, D, N (features), active heads (None = all), dtype, bias
    (2, 300, 270, 12, 64, 768, [0, 2, 3, 5, 6, 7, 8, 9, 10, 11, 1], torch.float16, True),
    (3, 77, 70, 8, 128, 1024, None, torch.bfloat16, True),
    (1, 200, 131, 4, 64, 96, [3, 1], torch.float16, False),  # partial row and feature tiles
    (2, 64, 1, 12, 64, 768, None, torch.bfloat16, True),     # one kept token per sequence
    (4, 512, 461, 12, 64, 768, [4, 0, 9, 2, 11, 7, 5, 1, 10, 3], torch.float16, True),
]
OUT_ATOL = {torch.float16: 4e-3, torch.bfloat16: 3e-2}


@pytest.mark.parametrize("case", OUT_CASES)
def test_compact_out_proj_matches_torch(case):
    """Against the unfused layer in torch fp32 (dense over the whole context
    row, rounded where the dense layer and the residual add round) followed
    by the gather of the kept rows: within one or two ulps, most elements
    identical."""
    from spatten_b200.proj import compact_out_proj
    B, S, L, H, D, Nf, heads, dt, bias = case
    g = torch.Generator().manual_seed(S + L + Nf)
    ctx = torch.randn(B, S, H, D, generator=g)
    if heads is not None:  # pruned heads' blocks are zeros in the drop-in's context
        off = torch.ones(H, dtype=torch.bool)
        off[heads] = False
        ctx[:, :, off] = 0
    ctx = ctx.reshape(B, S, H * D).to(dt)
    res = torch.randn(B, S, Nf, generator=g).to(dt)
    w = (torch.randn(Nf, H * D, generator=g) / (H * D) ** 0.5).to(dt)
    b = (torch.randn(Nf, generator=g) * 0.1).to(dt) if bias else None
    kept = torch.sort(torch.stack([torch.randperm(S, generator=g)[:L] for _ in range(B)]), dim=1).values
    out = compact_out_proj(ctx.cuda(), res.cuda(), kept.cuda(), w.cuda(), None if b is None else b.cuda(),
                           H, D, heads=None if heads is None else torch.tensor(heads).cuda())
    y = ctx.float() @ w.float().T
    if b is not None:
        y = y + b.float()
    y = (y.to(dt).float() + res.float()).to(dt)
    ref = torch.gather(y, 1, kept[:, :, None].expand(-1, -1, Nf))
    assert out.shape == (B, L, Nf) and out.dtype == dt
    got = out.cpu()
    torch.testing.assert_close(got.float(), ref.float(), rtol=2 * RTOL[dt], atol=OUT_ATOL[dt])
    assert (got == ref).float().mean().item() > 0.97


LN_CASES = [
    # rows, n, dtype, residual, eps
    (32 * 461, 768, torch.float16, True, 1e-12),
    (1000, 768, torch.float16, False, 1e-12),
    (77, 1024, torch.bfloat16, True, 1e-5),
    (9, 256, torch.bfloat16, False, 1e-6),
    (1, 2048, torch.float16, True, 1e-5),
    (0, 768, torch.float16, True, 1e-12),
]


@pytest.mark.parametrize("case", LN_CASES)
def test_add_layer_norm_matches_torch(case):
    """spatten_add_layer_norm against torch's add (rounded to the dtype) +
    F.layer_norm on the same GPU tensors: the statistics are summed in a
    different order (two passes in registers against Welford), so an output
    may differ by one ulp; > 98 % identical."""
    from spatten_b200.proj import add_layer_norm
    rows, n, dt, with_res, eps = case
    g = torch.Generator().manual_seed(rows + n)
    x = (torch.randn(rows, n, generator=g) * 3 + 0.5).to(dt).cuda()
    res = torch.randn(rows, n, generator=g).to(dt).cuda() if with_res else None
    w = (1 + 0.1 * torch.randn(n, generator=g)).to(dt).cuda()
    b = (0.1 * torch.randn(n, generator=g)).to(dt).cuda()
    got = add_layer_norm(x, w, b, eps, residual=res)
    h = x + res if with_res else x
    ref = torch.nn.functional.layer_norm(h, (n,), w, b, eps)
    assert got.shape == x.shape and got.dtype == dt
    if rows == 0:
        return
    torch.testing.assert_close(got.float(), ref.float(), rtol=RTOL[dt], atol=RTOL[dt])
    assert (got == ref).float().mean().item() > 0.98


def test_add_layer_norm_strided_rows():
    """Rows with a stride above n (a view of wider rows) are read in place."""
    from spatten_b200.proj import add_layer_norm
    g = torch.Generator().manual_seed(5)
    wide = torch.randn(64, 1024, generator=g).half().cuda()
    x = wide[:, :768]
    w = torch.ones(768, dtype=torch.float16, device="cuda")
    b = torch.zeros(768, dtype=torch.float16, device="cuda")
    got = add_layer_norm(x, w, b, 1e-12)
    ref = torch.nn.functional.layer_norm(x, (768,), w, b, 1e-12)
    torch.testing.assert_close(got.float(), ref.float(), rtol=RTOL[torch.float16], atol=RTOL[torch.float16])
