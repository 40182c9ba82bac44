"""The allocation-free attention entry point, spatten_prog_attn_noalloc.

Callers that cannot allocate device memory after start-up (a host with a
fixed memory budget, a plugin limited to the buffers its host hands it) use
spatten_prog_attn_noalloc, which takes its workspace from a fixed 16 MiB
array inside the library instead of a caller-allocated buffer. These tests
call it through the C ABI twice in a row and compare each result with the
allocating entry point (spatten_prog_attn) on the same inputs, and check that
a request too large for the array is refused before anything runs.

This file is named to be collected last so that, if it fails, a run that
stops at the first failure (pytest -x) has already run every other test; no
test depends on the order. It passes alone in a fresh process (where its
first call is also the first use of the array on the device) and after every
other test (where the array holds an earlier call's partial sums, which the
second call of each test overwrites as well).
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _rnd(shape, seed, dtype=torch.float16):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(dtype).cuda()


def _args(N, q8, qs, kp, v, out, bias, tok_in, tok, head, ref):
    Z, H, M, D = q8.shape
    a = N.ProgAttnArgs()
    a.mode, a.dtype = N.MODE_QUANT, N.DTYPE_F16
    a.Z, a.H, a.Hkv, a.M, a.N, a.D = Z, H, v.shape[1], M, v.shape[2], D
    a.q, (a.q_sz, a.q_sh, a.q_sm) = q8.data_ptr(), q8.stride()[:3]
    a.q_scale = qs.data_ptr()
    a.k0, a.k1 = kp.msb.data_ptr(), kp.lsb.data_ptr()
    a.k_sz, a.k_sh, a.k_sn = kp.msb.stride()[:3]
    a.k_scale = kp.scale.data_ptr()
    a.v, (a.v_sz, a.v_sh, a.v_sn) = v.data_ptr(), v.stride()[:3]
    a.out, (a.o_sz, a.o_sh, a.o_sm) = out.data_ptr(), out.stride()[:3]
    if bias is not None:
        a.bias = bias.data_ptr()
        a.b_sz, a.b_sh, a.b_sm, a.b_sn = bias.stride()
    a.sm_scale, a.refetch_thr, a.v_thr = 0.125, 0.1, 1e-3
    a.tok_out = tok.data_ptr() if tok is not None else None
    a.tok_in = tok_in.data_ptr() if tok_in is not None else None
    a.head_out = head.data_ptr() if head is not None else None
    a.refetch_out = ref.data_ptr() if ref is not None else None
    return a


def test_noalloc_matches_allocating_entry_point_twice():
    import spatten_b200 as sp
    from spatten_b200 import _native as N
    Z, H, Hkv, M, Nk, D = 2, 4, 2, 300, 333, 64
    q, k, v = _rnd((Z, H, M, D), 1), _rnd((Z, Hkv, Nk, D), 2), _rnd((Z, Hkv, Nk, D), 3)
    keep = torch.ones(Z, Nk, dtype=torch.bool)
    keep[1, 300:] = False
    bias = torch.zeros(Z, Nk).masked_fill_(~keep, torch.finfo(torch.float32).min)
    bias = bias.cuda()[:, None, None, :].expand(Z, H, M, Nk)
    cum = torch.rand(Z, Nk, device="cuda")
    q8, qs = sp.quant_q_int8(q)
    kp = sp.quant_k_planes(k)
    # allocating entry point (workspace from torch)
    ref = sp.prog_attn(q8, kp.msb, v, k1=kp.lsb, mode=N.MODE_QUANT, q_scale=qs, k_scale=kp.scale,
                       sm_scale=0.125, refetch_thr=0.1, v_thr=1e-3, bias=bias, tok_in=cum,
                       want_tok=True, want_head=True, want_refetch=True)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream().cuda_stream
    assert N.lib.spatten_prog_attn_noalloc_capacity() == 16 << 20
    for _ in range(2):
        out = torch.full((Z, H, M, D), float("nan"), dtype=torch.float16, device="cuda")
        tok = torch.full((Z, Nk), float("nan"), device="cuda")
        head = torch.full((H,), float("nan"), device="cuda")
        refetch = torch.full((Z, H, M), 7, dtype=torch.uint8, device="cuda")
        a = _args(N, q8, qs, kp, v, out, bias, cum, tok, head, refetch)
        N.check(N.lib.spatten_prog_attn_noalloc(a, stream))
        torch.cuda.synchronize()
        assert (out.float() - ref.out.float()).abs().max().item() < 1e-2
        np.testing.assert_allclose(tok.cpu().numpy(), ref.token_importance.cpu().numpy(), rtol=1e-4)
        np.testing.assert_allclose(head.cpu().numpy(), ref.head_abs_sum.cpu().numpy(), rtol=5e-3)
        assert torch.equal(refetch.bool(), ref.refetch)


def test_noalloc_refuses_workspace_beyond_the_array():
    import spatten_b200 as sp
    from spatten_b200 import _native as N
    # token-importance partials of this shape need ~50 MB > 16 MiB
    Z, H, M, Nk, D = 8, 12, 4096, 4096, 64
    q8 = torch.zeros((Z, H, M, D), dtype=torch.int8, device="cuda")
    qs = torch.ones((Z, H, M), device="cuda")
    kp = sp.quant_k_planes(torch.zeros((Z, H, Nk, D), dtype=torch.float16, device="cuda"))
    v = torch.zeros((Z, H, Nk, D), dtype=torch.float16, device="cuda")
    out = torch.empty((Z, H, M, D), dtype=torch.float16, device="cuda")
    tok = torch.empty((Z, Nk), device="cuda")
    a = _args(N, q8, qs, kp, v, out, None, None, tok, None, None)
    need = N.lib.spatten_prog_attn_workspace_size(a)
    assert need > N.lib.spatten_prog_attn_noalloc_capacity()
    rc = N.lib.spatten_prog_attn_noalloc(a, torch.cuda.current_stream().cuda_stream)
    assert rc == N.ERR_INVALID
    assert b"exceeds" in N.lib.spatten_last_error()
