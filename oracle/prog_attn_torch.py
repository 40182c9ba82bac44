"""Timed CPU baseline of the integer progressive attention (torch fp32, all cores).

Test/bench infrastructure only (see ``oracle/__init__.py``): used by
``bench.py`` for its ``cpu_baseline`` figure and its ``--impl reference`` arm,
never by the product path.

The reference has no CPU implementation of the progressive op; its CPU path
for the attention core is spatten_bert.py:81-136, which materialises the
[heads, S, S] probabilities with torch fp32 ops. This module restates the
integer progressive op (same rules as ``oracle.prog_attn.prog_attn_quant``)
in that style: batched fp32 matmuls (exact on int8 operands, see
``oracle/prog_attn.py``), softmax, threshold V prune, P.V and the token
importance, over blocks of query rows to bound memory, using every thread
torch has.
"""
import torch


def unpack_planes(msb_p, lsb_p):
    """Packed uint8 planes [.., D/2] -> (16*msb, lsb) as fp32 [.., D]."""
    m = msb_p.to(torch.int16)
    l = lsb_p.to(torch.int16)
    mlo, mhi = m & 15, (m >> 4) & 15
    msb = torch.cat([mlo, mhi], dim=-1)
    msb = torch.where(msb >= 8, msb - 16, msb)
    lsb = torch.cat([l & 15, (l >> 4) & 15], dim=-1)
    return (16 * msb).float(), lsb.float()


def quant_rows(x):
    """torch restatement of oracle.quant.quant_rows_int8 (fp32 division, rint)."""
    xf = x.float()
    s = xf.abs().amax(dim=-1) / 127.0
    safe = torch.where(s == 0, torch.ones_like(s), s)
    q = torch.round(xf / safe[..., None]).clamp_(-127, 127)
    q = torch.where(s[..., None] == 0, torch.zeros_like(q), q)
    return q, s


def prog_attn_quant_torch(q8, sq, k16, klsb, sk, v, sm_scale, refetch_thr, v_thr, rows=512):
    """One batch element: q8 [H,M,D] fp32 (int values), sq [H,M], k16/klsb
    [H,N,D] fp32 (16*msb, lsb), sk [H,N], v [H,N,D] fp32. Returns
    (out [H,M,D], tok [N])."""
    H, M, D = q8.shape
    out = torch.empty((H, M, D), dtype=torch.float32)
    tok = torch.zeros((k16.shape[1],), dtype=torch.float32)
    kf = k16 + klsb
    for r0 in range(0, M, rows):
        r1 = min(M, r0 + rows)
        qb = q8[:, r0:r1]
        cs = (sq[:, r0:r1] * sm_scale)[:, :, None] * sk[:, None, :]
        s_msb = torch.matmul(qb, k16.transpose(1, 2)) * cs
        l1 = torch.exp(s_msb - s_msb.amax(-1, keepdim=True)).sum(-1)
        rf = (1.0 / l1) < refetch_thr
        if bool(rf.any()):
            s_full = torch.matmul(qb, kf.transpose(1, 2)) * cs
            s = torch.where(rf[..., None], s_full, s_msb)
        else:
            s = s_msb
        p = torch.softmax(s, dim=-1)
        if v_thr > 0:
            p = torch.where(p < v_thr, torch.zeros_like(p), p)
        out[:, r0:r1] = torch.matmul(p, v)
        tok += p.sum(dim=(0, 1))
    return out, tok


def run_sample(q, k, v, sm_scale, refetch_thr, v_thr):
    """Full CPU op (quantise + attend) for one batch element: q, k, v [H,S,D]."""
    q8, sq = quant_rows(q)
    k8, sk = quant_rows(k)
    msb = torch.div(k8, 16, rounding_mode="floor")
    k16, klsb = 16 * msb, k8 - 16 * msb
    return prog_attn_quant_torch(q8, sq, k16, klsb, sk, v.float(), sm_scale, refetch_thr, v_thr)
