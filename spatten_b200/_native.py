"""ctypes bindings of libspatten_b200.so (the C ABI in include/spatten_b200.h).

The library is the only compute path: if it is missing or fails to load,
importing this module raises. There is no CPU fallback.
"""
import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "lib", "libspatten_b200.so")

OK = 0
ERR_INVALID = 1
ERR_CUDA = 2
ERR_UNSUPPORTED = 3

DTYPE_F16, DTYPE_BF16, DTYPE_F32 = 0, 1, 2
MODE_QUANT, MODE_DENSE, MODE_COMPAT = 0, 1, 2
PROJ_QUANT, PROJ_DENSE = 0, 1

ABI_VERSION = 4
MAX_V_PRUNE_COUNT = 16  # spatten_prog_attn_args.v_prune_count limit

c_i64 = ctypes.c_int64
c_vp = ctypes.c_void_p
c_int = ctypes.c_int
c_float = ctypes.c_float


class ProgAttnArgs(ctypes.Structure):
    """Mirror of ``spatten_prog_attn_args`` (field order and types match)."""
    _fields_ = [
        ("mode", c_int), ("dtype", c_int),
        ("Z", c_int), ("H", c_int), ("Hkv", c_int), ("M", c_int), ("N", c_int), ("D", c_int),
        ("q", c_vp), ("q_sz", c_i64), ("q_sh", c_i64), ("q_sm", c_i64),
        ("q_scale", c_vp),
        ("k0", c_vp), ("k1", c_vp), ("k_sz", c_i64), ("k_sh", c_i64), ("k_sn", c_i64),
        ("k_scale", c_vp),
        ("v", c_vp), ("v_sz", c_i64), ("v_sh", c_i64), ("v_sn", c_i64),
        ("out", c_vp), ("o_sz", c_i64), ("o_sh", c_i64), ("o_sm", c_i64),
        ("out_head_map", c_vp), ("out_head_slots", c_int),
        ("bias", c_vp), ("b_sz", c_i64), ("b_sh", c_i64), ("b_sm", c_i64), ("b_sn", c_i64),
        ("sm_scale", c_float), ("refetch_thr", c_float), ("v_thr", c_float),
        ("tile_m", c_int), ("tile_n", c_int), ("tile_thr", c_float), ("causal", c_int),
        ("tok_out", c_vp), ("tok_in", c_vp), ("head_out", c_vp), ("refetch_out", c_vp),
        ("score_out", c_vp), ("v_prune_count", c_int), ("key_limit", c_vp),
        ("score_row_stride", c_int),
    ]


class DecodeArgs(ctypes.Structure):
    """Mirror of spatten_decode_args (include/spatten_b200.h)."""
    _fields_ = [
        ("dtype", c_int), ("B", c_int), ("H", c_int), ("G", c_int), ("N", c_int), ("D", c_int),
        ("n_valid", c_int),
        ("q8", c_vp), ("q_scale", c_vp), ("k_msb", c_vp), ("k_lsb", c_vp), ("k_scale", c_vp),
        ("v", c_vp), ("sm_scale", c_float), ("importance", c_vp), ("top_k", c_int), ("kept", c_vp),
        ("out", c_vp),
    ]


class QkvProjArgs(ctypes.Structure):
    """Mirror of spatten_qkv_proj_args (include/spatten_b200.h)."""
    _fields_ = [
        ("dtype", c_int), ("mode", c_int), ("B", c_int), ("S", c_int), ("Kdim", c_int),
        ("Hall", c_int), ("Dh", c_int), ("cur", c_int),
        ("x", c_vp), ("x_row_stride", c_i64), ("w", c_vp), ("bias", c_vp), ("heads", c_vp),
        ("q8", c_vp), ("q_scale", c_vp), ("k_msb", c_vp), ("k_lsb", c_vp), ("k_scale", c_vp),
        ("q", c_vp), ("k", c_vp), ("v", c_vp),
    ]


class QkNormRopeArgs(ctypes.Structure):
    """Mirror of spatten_qk_norm_rope_args (include/spatten_b200.h)."""
    _fields_ = [
        ("dtype", c_int), ("B", c_int), ("S", c_int), ("Hq", c_int), ("Hk", c_int), ("D", c_int),
        ("q", c_vp), ("q_row_stride", c_i64), ("k", c_vp), ("k_row_stride", c_i64),
        ("q_norm_w", c_vp), ("k_norm_w", c_vp), ("eps", c_float), ("cos", c_vp), ("sin", c_vp),
        ("cs_b_stride", c_i64), ("cs_s_stride", c_i64), ("k_out", c_vp), ("k_out_row_stride", c_i64),
        ("q_out", c_vp), ("q_out_row_stride", c_i64), ("q8", c_vp), ("q_scale", c_vp),
    ]


class CompactOutProjArgs(ctypes.Structure):
    """Mirror of spatten_compact_out_proj_args (include/spatten_b200.h)."""
    _fields_ = [
        ("dtype", c_int), ("B", c_int), ("S", c_int), ("L", c_int), ("N", c_int),
        ("H", c_int), ("head_dim", c_int), ("cur", c_int), ("heads", c_vp), ("kept", c_vp),
        ("ctx", c_vp), ("ctx_row_stride", c_i64), ("w", c_vp), ("bias", c_vp),
        ("res", c_vp), ("res_row_stride", c_i64), ("out", c_vp),
    ]


# name -> (restype, argtypes); every entry point declared in include/spatten_b200.h
SIGNATURES = {
    "spatten_abi_version": (c_int, []),
    "spatten_last_error": (ctypes.c_char_p, []),
    "spatten_device_error": (c_int, [ctypes.POINTER(ctypes.c_uint), c_int]),
    "spatten_quant_q_int8": (c_int, [c_vp, c_int, c_int, c_int, c_int, c_int, c_i64, c_i64, c_i64,
                                     c_vp, c_vp, c_vp]),
    "spatten_quant_k_planes": (c_int, [c_vp, c_int, c_int, c_int, c_int, c_int, c_i64, c_i64,
                                       c_i64, c_vp, c_vp, c_vp, c_vp]),
    "spatten_prog_attn_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(ProgAttnArgs)]),
    "spatten_prog_attn": (c_int, [ctypes.POINTER(ProgAttnArgs), c_vp, ctypes.c_size_t, c_vp]),
    "spatten_prog_attn_noalloc_capacity": (ctypes.c_size_t, []),
    "spatten_prog_attn_noalloc": (c_int, [ctypes.POINTER(ProgAttnArgs), c_vp]),
    "spatten_topk_indices": (c_int, [c_vp, c_int, c_int, c_i64, c_int, c_vp, c_vp]),
    "spatten_decode_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(DecodeArgs)]),
    "spatten_decode_importance": (c_int, [ctypes.POINTER(DecodeArgs), c_vp, ctypes.c_size_t, c_vp]),
    "spatten_decode_attend": (c_int, [ctypes.POINTER(DecodeArgs), c_vp, ctypes.c_size_t, c_vp]),
    "spatten_qkv_proj": (c_int, [ctypes.POINTER(QkvProjArgs), c_vp]),
    "spatten_qk_norm_rope": (c_int, [ctypes.POINTER(QkNormRopeArgs), c_vp]),
    "spatten_compact_out_proj": (c_int, [ctypes.POINTER(CompactOutProjArgs), c_vp]),
    "spatten_gather_rows": (c_int, [c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_int, c_int, c_int,
                                    c_i64, c_i64, c_vp, c_i64, c_i64, c_vp]),
    "spatten_add_layer_norm": (c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp, c_i64, c_i64, c_int,
                                       c_int, ctypes.c_float, c_vp]),
    "spatten_select_heads": (c_int, [c_vp, ctypes.c_float, c_vp, c_int, c_int, c_vp, c_vp, c_vp, c_vp]),
}


class SpattenError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"[spatten error {code}] {msg}")
        self.code = code


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python spatten_b200/build.py` "
            "(the CUDA library is the only compute path)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    v = lib.spatten_abi_version()
    if v != ABI_VERSION:
        raise ImportError(f"libspatten_b200 ABI {v} != {ABI_VERSION}; rebuild the library")
    return lib


lib = _load()


def check(code):
    """Raise SpattenError for a non-zero status of a library call."""
    if code != OK:
        raise SpattenError(code, lib.spatten_last_error().decode(errors="replace"))
    return code
