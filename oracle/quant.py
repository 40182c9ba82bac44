"""Oracle: per-row symmetric int8 quantisation and 4-bit K planes (numpy).

Test infrastructure only (see ``oracle/__init__.py``).

The reference splits K into two *float* planes, ``k_msb = 0.8*K`` and
``k_lsb = 0.2*K`` (spatten_bert_ultimate.py:184-185). The progressive
quantisation of this library uses real integer planes instead:

* ``scale = max_d |x| / 127``  (fp32 division)
* ``x8 = clamp(rint(x / scale), -127, 127)``  (fp32 division, round half to
  even); a row whose max is 0 has scale 0 and x8 = 0.
* ``msb = x8 >> 4`` (arithmetic shift, -8..7), ``lsb = x8 & 15`` (0..15), so
  ``x8 == 16*msb + lsb``.
* Packing, two 4-bit values per byte, split at D/2: byte ``p`` of a row holds
  dim ``p`` in its low nibble and dim ``p + D/2`` in its high nibble. With
  this split a 4-byte word of the packed row expands to two 4-byte groups of
  consecutive dims with only shifts and masks.
"""
import numpy as np


def quant_rows_int8(x):
    """Quantise the last axis of ``x`` to int8 with a per-row fp32 scale."""
    xf = np.asarray(x, dtype=np.float32)
    amax = np.max(np.abs(xf), axis=-1)
    scale = (amax / np.float32(127.0)).astype(np.float32)
    safe = np.where(scale == 0, np.float32(1.0), scale).astype(np.float32)
    q = np.rint(xf / safe[..., None])
    q = np.clip(q, -127, 127)
    q = np.where(scale[..., None] == 0, 0, q).astype(np.int8)
    return q, scale


def split_planes(k8):
    """int8 K -> (msb int8 in [-8,7], lsb uint8 in [0,15]) with k8 == 16*msb+lsb."""
    k8 = np.asarray(k8, dtype=np.int8)
    msb = (k8.astype(np.int16) >> 4).astype(np.int8)
    lsb = (k8.astype(np.int16) & 15).astype(np.uint8)
    return msb, lsb


def pack_nibbles(v):
    """Pack 4-bit values (last axis D, even) into D/2 bytes, split at D/2."""
    v = np.asarray(v)
    d = v.shape[-1]
    assert d % 2 == 0
    lo = v[..., : d // 2].astype(np.int16) & 15
    hi = v[..., d // 2:].astype(np.int16) & 15
    return (lo | (hi << 4)).astype(np.uint8)


def unpack_nibbles(p, signed):
    """Inverse of :func:`pack_nibbles`; ``signed`` sign-extends each nibble."""
    p = np.asarray(p, dtype=np.uint8).astype(np.int16)
    lo = p & 15
    hi = (p >> 4) & 15
    v = np.concatenate([lo, hi], axis=-1)
    if signed:
        v = np.where(v >= 8, v - 16, v)
        return v.astype(np.int8)
    return v.astype(np.uint8)


def quant_k_planes(k):
    """K (..., D) -> (msb_packed (..., D/2) u8, lsb_packed (..., D/2) u8, scale (...) f32)."""
    k8, scale = quant_rows_int8(k)
    msb, lsb = split_planes(k8)
    return pack_nibbles(msb), pack_nibbles(lsb), scale


def k8_from_planes(msb_packed, lsb_packed):
    """Rebuild int8 K from the packed planes: 16*msb + lsb."""
    msb = unpack_nibbles(msb_packed, signed=True).astype(np.int16)
    lsb = unpack_nibbles(lsb_packed, signed=False).astype(np.int16)
    return (16 * msb + lsb).astype(np.int8)
