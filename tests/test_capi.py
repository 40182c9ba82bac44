"""The C-ABI library loads, exports every symbol include/*.h declares, and
rejects invalid arguments on the host (no GPU needed: nothing here launches)."""
import ctypes
import glob
import os
import re

import pytest

from tests.conftest import ROOT


def _declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(spatten_[a-z_0-9]+)\s*\(",
                             src, flags=re.M):
            names.add(m.group(1))
    return names


def test_header_declares_entry_points():
    names = _declared_symbols()
    for n in ("spatten_prog_attn", "spatten_quant_k_planes", "spatten_quant_q_int8",
              "spatten_topk_indices", "spatten_gather_rows", "spatten_last_error",
              "spatten_abi_version", "spatten_prog_attn_workspace_size"):
        assert n in names, n


def test_library_exports_every_declared_symbol():
    from spatten_b200 import _native as N
    lib = ctypes.CDLL(N.LIB_PATH)
    missing = [n for n in _declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing
    # the Python bindings cover the whole header
    assert _declared_symbols() <= set(N.SIGNATURES)


def test_abi_version():
    from spatten_b200 import _native as N
    assert N.lib.spatten_abi_version() == N.ABI_VERSION


def _args(lib_mod, **kw):
    N = lib_mod
    a = N.ProgAttnArgs()
    a.mode, a.dtype = N.MODE_QUANT, N.DTYPE_F16
    a.Z, a.H, a.Hkv, a.M, a.N, a.D = 2, 4, 4, 100, 257, 64
    a.q = a.k0 = a.k1 = a.v = a.out = 1 << 20
    a.q_scale = a.k_scale = 1 << 20
    a.q_sz, a.q_sh, a.q_sm = 4 * 100 * 64, 100 * 64, 64
    a.k_sz, a.k_sh, a.k_sn = 4 * 257 * 32, 257 * 32, 32
    a.v_sz, a.v_sh, a.v_sn = 4 * 257 * 64, 257 * 64, 64
    a.o_sz, a.o_sh, a.o_sm = 4 * 100 * 64, 100 * 64, 64
    a.sm_scale, a.refetch_thr = 0.125, 0.1
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def test_workspace_size_matches_partials():
    from spatten_b200 import _native as N
    a = _args(N)
    assert N.lib.spatten_prog_attn_workspace_size(a) == 0
    a.tok_out = 1 << 21
    a.head_out = 1 << 22
    ws = N.lib.spatten_prog_attn_workspace_size(a)
    mtiles = (100 + 127) // 128  # QUANT/DENSE: 128 query rows per CTA
    tok = 2 * 4 * mtiles * 257 * 4
    head = 2 * 4 * mtiles * 4
    r = lambda x: (x + 255) // 256 * 256  # noqa: E731
    assert ws == r(tok) + r(head)


@pytest.mark.parametrize("field,value,code", [
    ("mode", 7, 1), ("dtype", 9, 1), ("D", 96, 3), ("M", 0, 1), ("N", 0, 1),
    ("Hkv", 3, 1), ("q", 0, 1), ("k1", 0, 1), ("k0", (1 << 20) + 8, 1), ("v_sn", 65, 1),
    ("q_sm", -64, 1),
])
def test_prog_attn_rejects_bad_args(field, value, code):
    from spatten_b200 import _native as N
    a = _args(N, **{field: value})
    rc = N.lib.spatten_prog_attn(a, None, 0, None)
    assert rc == code
    assert N.lib.spatten_last_error().decode()


def test_prog_attn_requires_workspace():
    from spatten_b200 import _native as N
    a = _args(N, tok_out=1 << 21)
    assert N.lib.spatten_prog_attn(a, None, 0, None) == N.ERR_INVALID
    assert b"workspace" in N.lib.spatten_last_error()


@pytest.mark.parametrize("count,mode,code", [(-1, 0, "ERR_INVALID"), (17, 0, "ERR_UNSUPPORTED"),
                                             (17, 1, "ERR_UNSUPPORTED"), (2, 2, "ERR_UNSUPPORTED")])
def test_count_v_prune_limits(count, mode, code):
    """The count V prune takes 0..16 keys per row, QUANT and DENSE only."""
    from spatten_b200 import _native as N
    a = _args(N, v_prune_count=count, mode=mode, tile_m=32, tile_n=32)
    assert N.lib.spatten_prog_attn(a, ctypes.c_void_p(0x1000), 1 << 20, None) == getattr(N, code)


def test_fp32_limits():
    from spatten_b200 import _native as N
    a = _args(N, dtype=N.DTYPE_F32, mode=N.MODE_COMPAT, tile_m=32, tile_n=32)
    assert N.lib.spatten_prog_attn(a, None, 0, None) == N.ERR_UNSUPPORTED
    a = _args(N, dtype=N.DTYPE_F32, N=9000)
    assert N.lib.spatten_prog_attn(a, None, 0, None) == N.ERR_UNSUPPORTED


def test_compat_tile_validation():
    from spatten_b200 import _native as N
    a = _args(N, mode=N.MODE_COMPAT, tile_m=16, tile_n=32)
    a.k_sn = 64
    assert N.lib.spatten_prog_attn(a, None, 0, None) == N.ERR_UNSUPPORTED


def test_topk_gather_quant_reject_bad_args():
    from spatten_b200 import _native as N
    L = N.lib
    assert L.spatten_topk_indices(None, 1, 4, 4, 2, None, None) == N.ERR_INVALID
    assert L.spatten_topk_indices(1 << 20, 1, 4, 4, 5, 1 << 21, None) == N.ERR_INVALID
    assert L.spatten_topk_indices(1 << 20, 2, 4, 3, 2, 1 << 21, None) == N.ERR_INVALID
    assert L.spatten_gather_rows(None, 0, 0, 1, None, 0, 1, 1, 1, 1, 4, None, 0, 0, None) == N.ERR_INVALID
    assert L.spatten_gather_rows(1 << 20, 0, 4, 1, 1 << 21, 0, 1, 1, 0, 1, 4, 1 << 22, 0, 4, None) == N.ERR_INVALID
    assert L.spatten_quant_q_int8(1 << 20, 0, 1, 1, 1, 48, 0, 0, 48, 1 << 21, 1 << 22, None) == N.ERR_UNSUPPORTED
    assert L.spatten_quant_k_planes(None, 0, 1, 1, 1, 64, 0, 0, 64, 1, 1, 1, None) == N.ERR_INVALID
    # empty work is a no-op that succeeds without touching the device
    assert L.spatten_topk_indices(1 << 20, 0, 4, 4, 2, 1 << 21, None) == N.OK
    assert L.spatten_gather_rows(1 << 20, 0, 4, 1, 1 << 21, 0, 0, 1, 1, 1, 4, 1 << 22, 0, 4, None) == N.OK


def test_ops_refuse_cpu_tensors():
    import torch
    import spatten_b200 as sp
    x = torch.zeros(1, 1, 4, 64, dtype=torch.float16)
    with pytest.raises(ValueError, match="no CPU path"):
        sp.quant_q_int8(x)
    with pytest.raises(ValueError, match="no CPU path"):
        sp.topk_indices(torch.zeros(4), 2)


def test_torch_ops_registered():
    """The operators are reachable by name under torch.ops.spatten."""
    import torch
    import spatten_b200.torch_ops  # noqa: F401
    for name in ("quant_q_int8", "quant_k_planes", "progressive_attention", "topk_select",
                 "gather_rows"):
        assert hasattr(torch.ops.spatten, name), name


def test_decode_args_validation():
    """The decode entry points validate before any launch; the workspace size
    does not depend on which call follows."""
    import ctypes
    from spatten_b200 import _native as N
    a = N.DecodeArgs()
    a.dtype, a.B, a.H, a.G, a.N, a.D, a.n_valid = N.DTYPE_BF16, 2, 8, 2, 1000, 128, 900
    a.q8 = a.q_scale = a.k_msb = a.k_lsb = a.k_scale = a.v = 1 << 20
    a.sm_scale, a.top_k = 0.088, 100
    n = N.lib.spatten_decode_workspace_size(a)
    assert n > 0 and n % 256 == 0
    assert N.lib.spatten_decode_importance(a, ctypes.c_void_p(1 << 24), n, None) == N.ERR_INVALID  # no output
    a.H = 12  # 6 query heads per KV head
    assert N.lib.spatten_decode_workspace_size(a) == 0
    assert N.lib.spatten_decode_importance(a, None, 0, None) == N.ERR_UNSUPPORTED
    a.H, a.n_valid = 8, 1001
    assert N.lib.spatten_decode_attend(a, None, 0, None) == N.ERR_INVALID


def test_qkv_proj_args_validation():
    """The fused projection rejects bad arguments before any launch."""
    from spatten_b200 import _native as N
    assert N.lib.spatten_qkv_proj(None, None) == N.ERR_INVALID
    a = N.QkvProjArgs()
    a.dtype, a.mode, a.B, a.S, a.Kdim, a.Hall, a.Dh, a.cur = N.DTYPE_F16, N.PROJ_QUANT, 2, 100, 768, 12, 64, 11
    a.x = a.w = a.v = 1 << 20
    a.x_row_stride = 768
    assert N.lib.spatten_qkv_proj(a, None) == N.ERR_INVALID  # quantised outputs missing
    a.q8 = a.q_scale = a.k_msb = a.k_lsb = a.k_scale = 1 << 21
    a.dtype = N.DTYPE_F32
    assert N.lib.spatten_qkv_proj(a, None) == N.ERR_UNSUPPORTED
    a.dtype, a.Dh = N.DTYPE_BF16, 96
    assert N.lib.spatten_qkv_proj(a, None) == N.ERR_UNSUPPORTED
    a.Dh, a.cur = 64, 13  # more active heads than the weight has
    assert N.lib.spatten_qkv_proj(a, None) == N.ERR_INVALID
    a.cur, a.x_row_stride = 11, 700
    assert N.lib.spatten_qkv_proj(a, None) == N.ERR_INVALID
    a.x_row_stride, a.x = 768, (1 << 20) + 8  # x not 16-byte aligned
    assert N.lib.spatten_qkv_proj(a, None) == N.ERR_INVALID


def test_qk_norm_rope_args_validation():
    """The fused QK-norm + RoPE rejects bad arguments before any launch."""
    from spatten_b200 import _native as N
    assert N.lib.spatten_qk_norm_rope(None, None) == N.ERR_INVALID
    a = N.QkNormRopeArgs()
    a.dtype, a.B, a.S, a.Hq, a.Hk, a.D = N.DTYPE_BF16, 2, 100, 16, 8, 128
    a.q = a.k = a.q_norm_w = a.k_norm_w = a.cos = a.sin = a.k_out = 1 << 20
    a.q_row_stride, a.k_row_stride, a.k_out_row_stride = 2048, 1024, 1024
    a.cs_b_stride, a.cs_s_stride, a.eps = 100 * 128, 128, 1e-6
    assert N.lib.spatten_qk_norm_rope(a, None) == N.ERR_INVALID  # neither q_out nor q8
    a.q8, a.q_scale = 1 << 21, 1 << 22
    a.D = 96
    assert N.lib.spatten_qk_norm_rope(a, None) == N.ERR_UNSUPPORTED
    a.D, a.dtype = 128, N.DTYPE_F32
    assert N.lib.spatten_qk_norm_rope(a, None) == N.ERR_UNSUPPORTED
    a.dtype, a.q_row_stride = N.DTYPE_BF16, 1000  # shorter than Hq * D
    assert N.lib.spatten_qk_norm_rope(a, None) == N.ERR_INVALID
    a.q_row_stride, a.k = 2048, (1 << 20) + 4
    assert N.lib.spatten_qk_norm_rope(a, None) == N.ERR_INVALID


def test_compact_out_proj_args_validation():
    """The kept-token output projection rejects bad arguments before any
    launch."""
    from spatten_b200 import _native as N
    assert N.lib.spatten_compact_out_proj(None, None) == N.ERR_INVALID
    a = N.CompactOutProjArgs()
    a.dtype, a.B, a.S, a.L, a.N, a.H, a.head_dim, a.cur = N.DTYPE_F16, 4, 512, 461, 768, 12, 64, 10
    a.ctx = a.w = a.res = a.out = 1 << 20
    a.ctx_row_stride, a.res_row_stride = 768, 768
    assert N.lib.spatten_compact_out_proj(a, None) == N.ERR_INVALID  # kept missing
    a.kept = 1 << 21
    a.dtype = N.DTYPE_F32
    assert N.lib.spatten_compact_out_proj(a, None) == N.ERR_UNSUPPORTED
    a.dtype, a.head_dim = N.DTYPE_BF16, 96
    assert N.lib.spatten_compact_out_proj(a, None) == N.ERR_UNSUPPORTED
    a.head_dim, a.N = 64, 100  # features not a multiple of 32
    assert N.lib.spatten_compact_out_proj(a, None) == N.ERR_UNSUPPORTED
    a.N, a.cur = 768, 13  # more active heads than the context row has
    assert N.lib.spatten_compact_out_proj(a, None) == N.ERR_INVALID
    a.cur, a.ctx_row_stride = 10, 700
    assert N.lib.spatten_compact_out_proj(a, None) == N.ERR_INVALID
    a.ctx_row_stride, a.res = 768, (1 << 20) + 8  # residual not 16-byte aligned
    assert N.lib.spatten_compact_out_proj(a, None) == N.ERR_INVALID
    a.res, a.L = 1 << 20, 0
    assert N.lib.spatten_compact_out_proj(a, None) == N.ERR_INVALID


def test_compat_rejects_masks():
    """The reference op has no mask: COMPAT refuses a bias, causal or key limit."""
    from spatten_b200 import _native as N
    for field, val in (("bias", 0x1000), ("causal", 1), ("key_limit", 0x1000)):
        a = _args(N, mode=N.MODE_COMPAT, tile_m=32, tile_n=32)
        setattr(a, field, val)
        assert N.lib.spatten_prog_attn(a, None, 0, None) == N.ERR_UNSUPPORTED, field


def test_add_layer_norm_args_validation():
    """The residual add + LayerNorm rejects bad arguments before any launch;
    zero rows is a no-op (empty tensors may carry null pointers)."""
    from spatten_b200 import _native as N
    f = N.lib.spatten_add_layer_norm
    p = 1 << 20
    # x, x_stride, res, res_stride, gamma, beta, y, y_stride, rows, n, dtype, eps, stream
    assert f(None, 768, None, 0, p, p, p, 768, 10, 768, N.DTYPE_F16, 1e-12, None) == N.ERR_INVALID
    assert f(p, 768, None, 0, p, p, p, 768, 10, 768, N.DTYPE_F32, 1e-12, None) == N.ERR_UNSUPPORTED
    assert f(p, 768, None, 0, p, p, p, 768, 10, 700, N.DTYPE_F16, 1e-12, None) == N.ERR_UNSUPPORTED
    assert f(p, 700, None, 0, p, p, p, 768, 10, 768, N.DTYPE_F16, 1e-12, None) == N.ERR_INVALID  # stride < n
    assert f(p, 768, p, 100, p, p, p, 768, 10, 768, N.DTYPE_F16, 1e-12, None) == N.ERR_INVALID  # res stride
    assert f(p + 8, 768, None, 0, p, p, p, 768, 10, 768, N.DTYPE_BF16, 1e-12, None) == N.ERR_INVALID  # align
    assert f(p, 772, None, 0, p, p, p, 768, 10, 768, N.DTYPE_BF16, 1e-12, None) == N.ERR_INVALID  # row align
    assert f(p, 768, None, 0, p, p, p, 768, 10, 768, N.DTYPE_F16, -1.0, None) == N.ERR_INVALID  # eps
    assert f(p, 768, None, 0, p, p, p, 768, -1, 768, N.DTYPE_F16, 1e-12, None) == N.ERR_INVALID
    assert f(None, 0, None, 0, None, None, None, 0, 0, 768, N.DTYPE_F16, 1e-12, None) == N.OK


def test_select_heads_args_validation():
    """The head decision rejects bad sizes before any launch."""
    from spatten_b200 import _native as N
    f = N.lib.spatten_select_heads
    p = 1 << 20
    # importance, scale, heads, cur, keep, importance_out, next_heads, next_heads32, stream
    assert f(None, 1.0, None, 12, 10, None, p, None, None) == N.ERR_INVALID
    assert f(p, 1.0, None, 12, 10, None, None, None, None) == N.ERR_INVALID
    assert f(p, 1.0, None, 0, 1, None, p, None, None) == N.ERR_UNSUPPORTED
    assert f(p, 1.0, None, 1025, 1, None, p, None, None) == N.ERR_UNSUPPORTED
    assert f(p, 1.0, None, 12, 0, None, p, None, None) == N.ERR_INVALID
    assert f(p, 1.0, None, 12, 13, None, p, None, None) == N.ERR_INVALID
    assert f(p, float("nan"), None, 12, 10, None, p, None, None) == N.ERR_INVALID
