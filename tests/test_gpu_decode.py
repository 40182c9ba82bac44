"""GPU parity of the decode attention (spatten_b200.decode) against the
oracle (oracle/decode.py): importance within 1e-5 relative, kept key indices
identical (inputs whose keep decisions clear ties by 1e-4), outputs within
1e-2 (fp16) / 2e-2 (bf16)."""
import numpy as np
import pytest
import torch

from oracle.decode import decode_attention as oracle_decode

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 1e-2, torch.bfloat16: 2e-2}


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _case(B, H, G, N, D, dt, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, D, generator=g).to(dt).cuda()
    k = torch.randn(B, G, N, D, generator=g).to(dt).cuda()
    v = torch.randn(B, G, N, D, generator=g).to(dt).cuda()
    return q, k, v


@pytest.mark.parametrize("B,H,G,N,D,top_k,n_valid,dt", [
    (3, 8, 2, 3000, 128, 300, 2900, torch.float16),
    (2, 8, 1, 1500, 128, 257, None, torch.bfloat16),
    # one KV head and its 4 query heads: a Qwen3-8B layer split over 8 ranks
    (2, 4, 1, 4096, 128, 512, None, torch.bfloat16),
    (2, 4, 4, 700, 64, 100, 650, torch.float16),
    (1, 16, 2, 2048, 128, 2048, None, torch.bfloat16),
    (1, 32, 8, 16384, 128, 2048, 16000, torch.bfloat16),
])
def test_decode_matches_oracle(B, H, G, N, D, top_k, n_valid, dt):
    from spatten_b200.decode import _quant_query, decode_attention, quant_kv_cache
    for seed in range(0, 30, 3):
        q, k, v = _case(B, H, G, N, D, dt, seed)
        cache = quant_kv_cache(k, v)
        q8, qs = _quant_query(q)
        o = oracle_decode(q8.cpu().numpy(), qs.cpu().numpy(), cache.planes.msb.cpu().numpy(),
                          cache.planes.lsb.cpu().numpy(), cache.planes.scale.cpu().numpy(),
                          v.float().cpu().numpy(), D ** -0.5, top_k, n_valid)
        if o["kth_gap"] > 1e-4:
            break
    else:
        pytest.fail("no well-conditioned input")
    r = decode_attention(q, cache, top_k=top_k, n_valid=n_valid)
    nv = N if n_valid is None else n_valid
    imp = r.importance.cpu().numpy()
    assert np.all(imp[:, nv:] == 0)
    np.testing.assert_allclose(imp[:, :nv], o["importance"][:, :nv], rtol=1e-5, atol=1e-7)
    assert np.array_equal(r.kept.cpu().numpy(), o["kept"])
    assert np.abs(r.out.float().cpu().numpy() - o["out"]).max() < TOL[dt]


def test_decode_attend_skips_out_of_range_keys():
    """Kept indices outside [0, n_valid) contribute nothing (no fault)."""
    from spatten_b200.decode import decode_attend, quant_kv_cache
    q, k, v = _case(1, 4, 1, 600, 128, torch.float16, 1)
    cache = quant_kv_cache(k, v)
    kept = torch.tensor([[0, 5, 599, 700, -1]], device="cuda")
    ref = decode_attend(q, cache, kept[:, :3], n_valid=600)
    got = decode_attend(q, cache, kept, n_valid=600)
    assert torch.allclose(got.float(), ref.float(), atol=1e-3)
