"""Oracle: progressive-quantised sparse attention on the CPU (numpy).

Test infrastructure only (see ``oracle/__init__.py``).

Three modes, each a restatement for one (batch, head) at a time:

``prog_attn_quant``  -- integer MSB/LSB planes. This is the op asked for the
    B200 build; the reference has only the float split. Scores are exact
    integers: A = q8 . (16*msb) (the MSB-only score) and F = q8 . k8 (the full
    score), dequantised as ``s = fp32(A) * (fp32(sq*sm_scale) * sk) + bias``
    in fp32. Pass 1 takes the row statistics of the MSB score; a row is
    *refetched* (its LSB plane is read and the full score is used) when its
    maximum softmax probability ``1/l`` is below ``refetch_thr``.
    Softmax/pruning/importance then follow spatten_bert.py:
      softmax over keys                         spatten_bert.py:93
      local V prune (new rule: p < v_thr -> 0,  spatten_bert.py:100-113
        no renormalisation; and/or the reference's count rule: zero the
        v_count smallest p of each row, ties to the smaller key index)
      context = P' V                            spatten_bert.py:116
      head importance = sum |context|           spatten_bert.py:120-121
      token importance = sum_{h,q} P'           spatten_bert.py:136
``prog_attn_dense``  -- float Q/K scores (progressive quantisation off).
``prog_attn_compat`` -- the reference op's float planes and its *tile*
    criterion: for each BM x BN tile, if max(q.k_msb * sm_scale) < threshold
    then the tile's scores become q.k_msb*sm_scale + q.k_lsb*sm_scale
    (spatten_bert_ultimate.py:58-74, BM=BN=32 at :108;
    spatten_progressive_attention.py:38-60, BM=BN=64 at :85-86). Tiles only
    cover valid rows and keys (the reference pads tail keys with score 0 and
    tail rows with q=0, spatten_bert_ultimate.py:52,64; that padding is not
    reproduced).

Softmax, sums and P.V are evaluated in float64 on the fp32 scores, so the
oracle is independent of summation order. Integer scores are evaluated with
fp32 matmuls: every product of two int8 values and every partial sum over
D <= 128 terms is an integer below 2**24, hence exact in fp32.
"""
import numpy as np

FP32_MIN = np.float32(np.finfo(np.float32).min)


def _kv_head(h, n_heads, n_kv_heads):
    return h // (n_heads // n_kv_heads)


def _bias_for(bias, z, h, m, n):
    if bias is None:
        return None
    b = np.asarray(bias, dtype=np.float32)
    b = np.broadcast_to(b, b.shape[:-2] + (m, n)) if b.ndim >= 2 else b
    while b.ndim < 4:
        b = b[None]
    zi = z if b.shape[0] > 1 else 0
    hi = h if b.shape[1] > 1 else 0
    return np.broadcast_to(b[zi, hi], (m, n)).astype(np.float32)


def _causal_mask(m, n):
    i = np.arange(m)[:, None]
    j = np.arange(n)[None, :]
    return j > i + (n - m)


def _limit_mask(limit, n):
    """Excluded keys of rows that see keys n < limit[m] only."""
    return np.arange(n)[None, :] >= np.asarray(limit)[:, None]


def _softmax_rows(s, excluded=None):
    """float64 softmax over the last axis; ``excluded`` entries get p = 0."""
    s64 = s.astype(np.float64)
    if excluded is not None:
        s64 = np.where(excluded, -np.inf, s64)
    mx = np.max(s64, axis=-1, keepdims=True)
    none = ~np.isfinite(mx)  # a row that sees no key: p = 0, l = 0
    e = np.where(none, 0.0, np.exp(s64 - np.where(none, 0.0, mx)))
    l = np.sum(e, axis=-1, keepdims=True)
    p = np.where(l > 0, e / np.where(l > 0, l, 1.0), 0.0)
    return p, mx[..., 0], l[..., 0]


def int_scores(q8, k8):
    """Exact int32 q8 . k8^T (see module docstring for why fp32 is exact)."""
    r = np.asarray(q8, np.float32) @ np.asarray(k8, np.float32).T
    return r.astype(np.int64).astype(np.int32)


def _count_prune(p, s, v_count):
    """The reference's count rule (spatten_bert.py:100-113): in every row of
    more than ``v_count`` keys, zero the ``v_count`` smallest probabilities
    (no renormalisation). The order is that of the fp32 scores ``s`` (p is
    monotone in s within a row), ties to the smaller key index. Returns the
    pruned p and the smallest relative gap between the v_count-th and the
    next score over rows where both are finite and differ (how robust the
    choice is to the rounding of another implementation's scores)."""
    m, n = s.shape
    if v_count <= 0 or n <= v_count:
        return p, np.inf
    pp = p.copy()
    gap = np.inf
    keys = np.arange(n)
    for r in range(m):
        order = np.lexsort((keys, s[r].astype(np.float64)))
        pp[r, order[:v_count]] = 0.0
        a, b = float(s[r, order[v_count - 1]]), float(s[r, order[v_count]])
        if np.isfinite(a) and np.isfinite(b) and a != b:  # exact ties order by key anywhere
            gap = min(gap, abs(b - a) / max(abs(a), abs(b), 1e-30))
    return pp, gap


def _finish(p, vv, v_thr, s=None, v_count=0):
    pp = np.where(p < v_thr, 0.0, p) if v_thr > 0 else p
    cgap = np.inf
    if v_count > 0:
        pp, cgap = _count_prune(pp, s, v_count)
    out = pp @ vv.astype(np.float64)
    return pp, out, cgap


def quant_head(q8, sq, msb_p, lsb_p, sk, v, sm_scale, refetch_thr, v_thr=0.0, bias=None,
               excl=None, band=1e-4, v_count=0, return_scores=False, decisions_only=False,
               chunk=1024):
    """One (batch, head) of :func:`prog_attn_quant`, over the query rows in
    chunks of ``chunk`` (every step is row-wise except the column sums of the
    token importance, which add up over the chunks), so that full-size heads
    fit in memory and heads can run on several threads.

    q8 [M, D] int8, sq [M], msb_p / lsb_p [N, D/2] packed planes, sk [N],
    v [N, D] (unused with ``decisions_only``), bias [M, N] or None, excl
    [M, N] bool (keys a row does not see) or None. With ``decisions_only``
    only the refetch decisions and the MSB max-probabilities are computed
    (pass 1 of the op)."""
    from .quant import unpack_nibbles
    q8 = np.asarray(q8, np.int8)
    M = q8.shape[0]
    msb = unpack_nibbles(msb_p, signed=True).astype(np.int16)
    k16 = (16 * msb).astype(np.int8)
    k8 = None
    if not decisions_only:
        lsb = unpack_nibbles(lsb_p, signed=False).astype(np.int16)
        k8 = (16 * msb + lsb).astype(np.int8)
    N = k16.shape[0]
    skf = np.asarray(sk, np.float32)
    refetch = np.zeros(M, bool)
    maxprob = np.zeros(M)
    res = dict(refetch=refetch, maxprob=maxprob)
    if not decisions_only:
        out = np.zeros((M, q8.shape[1]))
        tok = np.zeros(N)
        amb = np.zeros(N)
        res.update(out=out, tok=tok, amb=amb, head_abs=0.0, pgap=np.inf, cgap=np.inf)
        if return_scores:
            res["A"] = np.zeros((M, N), np.int32)
            res["F"] = np.zeros((M, N), np.int32)
    for r0 in range(0, M, chunk):
        rows = slice(r0, min(M, r0 + chunk))
        ex = excl[rows] if excl is not None else None
        A = int_scores(q8[rows], k16)
        c = (np.asarray(sq[rows], np.float32) * np.float32(sm_scale)).astype(np.float32)
        cs = (c[:, None] * skf[None, :]).astype(np.float32)
        s_msb = (A.astype(np.float32) * cs).astype(np.float32)
        if bias is not None:
            s_msb = (s_msb + bias[rows]).astype(np.float32)
        _, _, l1 = _softmax_rows(s_msb, ex)
        with np.errstate(divide="ignore"):  # a row that sees no key: l = 0
            mp = 1.0 / l1
        rf = mp < refetch_thr
        refetch[rows] = rf
        maxprob[rows] = mp
        if decisions_only:
            continue
        F = int_scores(q8[rows], k8)
        s_full = (F.astype(np.float32) * cs).astype(np.float32)
        if bias is not None:
            s_full = (s_full + bias[rows]).astype(np.float32)
        s = np.where(rf[:, None], s_full, s_msb)
        p, _, _ = _softmax_rows(s, ex)
        if v_thr > 0:
            res["pgap"] = min(res["pgap"], np.min(np.abs(p - v_thr)) / v_thr)
            amb += (np.abs(p - v_thr) < band * v_thr).sum(axis=0)
        s_ord = np.where(ex, -np.inf, s) if ex is not None else s
        pp, o, g = _finish(p, np.asarray(v), v_thr, s_ord, v_count)
        res["cgap"] = min(res["cgap"], g)
        out[rows] = o
        tok += pp.sum(axis=0)
        res["head_abs"] += np.abs(o).sum()
        if return_scores:
            res["A"][rows] = A
            res["F"][rows] = F
    return res


def prog_attn_quant(q8, sq, msb_p, lsb_p, sk, v, sm_scale, refetch_thr, v_thr=0.0,
                    bias=None, causal=False, return_scores=False, band=1e-4, v_count=0,
                    key_limit=None):
    """Integer progressive attention. Shapes: q8 [Z,H,M,D] int8, sq [Z,H,M],
    msb_p/lsb_p [Z,Hkv,N,D/2] uint8 (packed, see oracle.quant), sk [Z,Hkv,N],
    v [Z,Hkv,N,D]. ``v_count`` > 0 applies the reference's count V prune (on
    top of ``v_thr``). ``key_limit`` [Z, M]: row m sees keys n < key_limit[z, m]
    (replaces ``causal``). Returns a dict of float64 outputs and diagnostics."""
    q8 = np.asarray(q8, np.int8)
    Z, H, M, D = q8.shape
    Hkv, N = msb_p.shape[1], msb_p.shape[2]
    out = np.zeros((Z, H, M, D))
    refetch = np.zeros((Z, H, M), bool)
    maxprob = np.zeros((Z, H, M))
    tok_h = np.zeros((Z, H, N))
    head_abs = np.zeros((Z, H))
    amb = np.zeros((Z, N))
    pgap = np.inf
    cgap = np.inf
    scores = {}
    excl0 = _causal_mask(M, N) if causal else None
    for z in range(Z):
        excl = _limit_mask(key_limit[z], N) if key_limit is not None else excl0
        for h in range(H):
            kh = _kv_head(h, H, Hkv)
            r = quant_head(q8[z, h], sq[z, h], msb_p[z, kh], lsb_p[z, kh], sk[z, kh], v[z, kh],
                           sm_scale, refetch_thr, v_thr, bias=_bias_for(bias, z, h, M, N),
                           excl=excl, band=band, v_count=v_count, return_scores=return_scores)
            pgap = min(pgap, r["pgap"])
            cgap = min(cgap, r["cgap"])
            amb[z] += r["amb"]
            out[z, h] = r["out"]
            refetch[z, h] = r["refetch"]
            maxprob[z, h] = r["maxprob"]
            tok_h[z, h] = r["tok"]
            head_abs[z, h] = r["head_abs"]
            if return_scores:
                scores[(z, h)] = (r["A"], r["F"])
    res = dict(out=out, refetch=refetch, maxprob_msb=maxprob, tok_per_head=tok_h,
               tok=tok_h.sum(axis=1), head_abs=head_abs, vprune_gap=pgap, vprune_amb=amb,
               vcount_gap=cgap, refetch_gap=np.min(np.abs(maxprob - refetch_thr)) / max(abs(refetch_thr), 1e-30))
    if return_scores:
        res["scores"] = scores
    return res


def prog_attn_dense(q, k, v, sm_scale, v_thr=0.0, bias=None, causal=False, band=1e-4, v_count=0,
                    key_limit=None):
    """Float attention with V pruning and importance (progressive quant off).
    Scores: fp32(q) . fp32(k) * sm_scale + bias, evaluated in float64 then
    rounded to fp32."""
    q = np.asarray(q, np.float32)
    Z, H, M, D = q.shape
    Hkv, N = k.shape[1], k.shape[2]
    out = np.zeros((Z, H, M, D))
    tok_h = np.zeros((Z, H, N))
    head_abs = np.zeros((Z, H))
    amb = np.zeros((Z, N))
    pgap = np.inf
    cgap = np.inf
    excl0 = _causal_mask(M, N) if causal else None
    for z in range(Z):
        excl = _limit_mask(key_limit[z], N) if key_limit is not None else excl0
        for h in range(H):
            kh = _kv_head(h, H, Hkv)
            s = (q[z, h].astype(np.float64) @ np.asarray(k[z, kh], np.float64).T).astype(np.float32)
            s = (s * np.float32(sm_scale)).astype(np.float32)
            bb = _bias_for(bias, z, h, M, N)
            if bb is not None:
                s = (s + bb).astype(np.float32)
            p, _, _ = _softmax_rows(s, excl)
            if v_thr > 0:
                pgap = min(pgap, np.min(np.abs(p - v_thr)) / v_thr)
                amb[z] += (np.abs(p - v_thr) < band * v_thr).sum(axis=0)
            s_ord = np.where(excl, -np.inf, s) if excl is not None else s
            pp, o, g = _finish(p, np.asarray(v[z, kh]), v_thr, s_ord, v_count)
            cgap = min(cgap, g)
            out[z, h] = o
            tok_h[z, h] = pp.sum(axis=0)
            head_abs[z, h] = np.abs(o).sum()
    return dict(out=out, tok_per_head=tok_h, tok=tok_h.sum(axis=1), head_abs=head_abs,
                vprune_gap=pgap, vprune_amb=amb, vcount_gap=cgap)


def prog_attn_compat(q, k_msb, k_lsb, v, threshold, sm_scale, bm=32, bn=32):
    """Reference float-plane op semantics (tile criterion). Returns dict with
    ``out`` [Z,H,M,D], ``tile_refetch`` [Z,H,ceil(M/bm),ceil(N/bn)] and the
    smallest relative distance of a tile max to the threshold."""
    q = np.asarray(q, np.float32)
    Z, H, M, D = q.shape
    N = k_msb.shape[2]
    out = np.zeros((Z, H, M, D))
    tm, tn = -(-M // bm), -(-N // bn)
    tiles = np.zeros((Z, H, tm, tn), bool)
    gap = np.inf
    for z in range(Z):
        for h in range(H):
            s1 = (q[z, h].astype(np.float64) @ np.asarray(k_msb[z, h], np.float64).T).astype(np.float32)
            s1 = (s1 * np.float32(sm_scale)).astype(np.float32)
            s2 = (q[z, h].astype(np.float64) @ np.asarray(k_lsb[z, h], np.float64).T).astype(np.float32)
            s2 = (s2 * np.float32(sm_scale)).astype(np.float32)
            s = s1.copy()
            for a in range(tm):
                for b in range(tn):
                    blk = s1[a * bm:(a + 1) * bm, b * bn:(b + 1) * bn]
                    mx = float(blk.max())
                    gap = min(gap, abs(mx - threshold))
                    if mx < threshold:
                        tiles[z, h, a, b] = True
                        s[a * bm:(a + 1) * bm, b * bn:(b + 1) * bn] = (
                            blk + s2[a * bm:(a + 1) * bm, b * bn:(b + 1) * bn]).astype(np.float32)
            p, _, _ = _softmax_rows(s)
            out[z, h] = p @ np.asarray(v[z, h], np.float64)
    return dict(out=out, tile_refetch=tiles, threshold_gap=gap)


def reduce_importance(tok_per_head, head_abs, cumulative=None):
    """Token importance [Z,N] = sum over heads (and queries, already summed);
    head importance [H] = mean |context| over (batch, query, dim) -- the
    reference's ``context_layer.abs().mean(dim=(0, 2, 3))``
    (spatten_bert.py:119-121). ``head_abs`` is the per-(z,h) sum of |o|."""
    tok = tok_per_head.sum(axis=1)
    if cumulative is not None:
        tok = tok + cumulative
    return tok, head_abs
