"""Oracle: top-k index selection and row gathers (numpy).

Test infrastructure only (see ``oracle/__init__.py``).

``topk_sorted`` restates the reference's pruning decision
``sort(topk(x, k).indices)`` (spatten_bert.py:123-130 for heads,
spatten_bert.py:143-150 for tokens): the k largest entries of each row, their
indices returned in ascending order. Ties at the k-th value are broken towards
the smaller index (torch leaves the tie order unspecified; the selected *set*
is what the cascade consumes, so a fixed rule is pinned here).

``gather_rows`` restates the cascade's token compaction
(``torch.gather`` on dim 1, module.py:53-54 and :62-63) and
``gather_head_rows`` the head-row weight slicing
(``index_select`` on a [heads, head_dim, hidden] view, module.py:22-32).
"""
import numpy as np


def topk_sorted(x, k):
    """Rows of ``x`` [R, n] -> int64 [R, k] ascending indices of the top k."""
    x = np.asarray(x, dtype=np.float32)
    R, n = x.shape
    assert 0 < k <= n
    out = np.empty((R, k), np.int64)
    for r in range(R):
        # sort by (-value, index): the first k are the top k with ties to the
        # smaller index; np.lexsort sorts by the last key first.
        order = np.lexsort((np.arange(n), -x[r].astype(np.float64)))
        out[r] = np.sort(order[:k])
    return out


def kth_gap(x, k):
    """Smallest gap between the k-th and (k+1)-th largest value over rows
    (how well-conditioned a top-k decision is)."""
    x = np.sort(np.asarray(x, np.float64), axis=-1)[:, ::-1]
    if k >= x.shape[1]:
        return np.inf
    return float(np.min(x[:, k - 1] - x[:, k]))


def gather_rows(src, idx):
    """src [B, S, W], idx [B, K] -> [B, K, W]."""
    src = np.asarray(src)
    idx = np.asarray(idx)
    return np.take_along_axis(src, idx[:, :, None], axis=1)


def gather_head_rows(w, heads, head_dim):
    """w [H*head_dim, ...] -> rows of the selected heads, in ``heads`` order."""
    w = np.asarray(w)
    H = w.shape[0] // head_dim
    v = w.reshape((H, head_dim) + w.shape[1:])
    return v[np.asarray(heads)].reshape((-1,) + w.shape[1:])
