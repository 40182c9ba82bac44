"""Oracle: decode attention over a progressive-quantised KV cache with top-k
token selection (CPU, numpy).

Test infrastructure only (see ``oracle/__init__.py``).

The reference has no decode path, so parity for it is unpinned by the
reference; this restatement defines the semantics of ``spatten_decode_*``
from SpAtten's cascade rules: token importance = the sum over heads of the
softmax probabilities (spatten_bert.py:136-142), here of the MSB scores of
every cached key; keep the top-k by importance (spatten_bert.py:143-148,
ties to the smaller index); progressive quantisation's LSB read for the kept
keys only, whose exact int8 scores give the attention output.
"""
import numpy as np

from .prog_attn import int_scores
from .quant import unpack_nibbles
from .select import topk_sorted


def decode_attention(q8, sq, msb_p, lsb_p, sk, v, sm_scale, top_k, n_valid=None):
    """q8 [B, H, D] int8, sq [B, H]; planes [B, G, N, D/2] uint8; sk [B, G, N];
    v [B, G, N, D]. Returns dict(importance [B, N], kept [B, K], out [B, H, D],
    kth_gap: relative margin of the closest keep decision)."""
    q8 = np.asarray(q8, np.int8)
    B, H, D = q8.shape
    G, N = msb_p.shape[1], msb_p.shape[2]
    R = H // G
    nv = N if n_valid is None else int(n_valid)
    k = min(int(top_k), nv)
    imp = np.zeros((B, N))
    out = np.zeros((B, H, D))
    kept = np.zeros((B, k), np.int64)
    gap = np.inf
    for b in range(B):
        for g in range(G):
            msb = unpack_nibbles(msb_p[b, g, :nv], signed=True).astype(np.int16)
            c = (np.asarray(sq[b, g * R:(g + 1) * R], np.float32) * np.float32(sm_scale)).astype(np.float32)
            cs = (c[:, None] * np.asarray(sk[b, g, :nv], np.float32)[None, :]).astype(np.float32)
            A = int_scores(q8[b, g * R:(g + 1) * R], (16 * msb).astype(np.int8))
            s = (A.astype(np.float32) * cs).astype(np.float64)
            e = np.exp(s - s.max(axis=1, keepdims=True))
            imp[b, :nv] += (e / e.sum(axis=1, keepdims=True)).sum(axis=0)
        srt = np.sort(imp[b, :nv])
        if k < nv:
            gap = min(gap, abs(srt[nv - k] - srt[nv - k - 1]) / max(abs(srt[nv - k]), 1e-30))
        kept[b] = topk_sorted(imp[b:b + 1, :nv], k)[0]
        for g in range(G):
            kk = kept[b]
            msb = unpack_nibbles(msb_p[b, g, kk], signed=True).astype(np.int16)
            lsb = unpack_nibbles(lsb_p[b, g, kk], signed=False).astype(np.int16)
            F = int_scores(q8[b, g * R:(g + 1) * R], (16 * msb + lsb).astype(np.int8))
            c = (np.asarray(sq[b, g * R:(g + 1) * R], np.float32) * np.float32(sm_scale)).astype(np.float32)
            cs = (c[:, None] * np.asarray(sk[b, g, kk], np.float32)[None, :]).astype(np.float32)
            s = (F.astype(np.float32) * cs).astype(np.float64)
            e = np.exp(s - s.max(axis=1, keepdims=True))
            p = e / e.sum(axis=1, keepdims=True)
            out[b, g * R:(g + 1) * R] = p @ np.asarray(v[b, g, kk], np.float64)
    return dict(importance=imp, kept=kept, out=out, kth_gap=gap)
