"""Embedding quality metrics used by the end-to-end parity bars (GPU, via torch).

knn_preservation and label_accuracy follow the definitions of the reference's
knn_structure_score_cpp (src/embedding_utils.cpp:1386-1520): the mean fraction
of each point's k high-dimensional neighbours found among its k nearest
neighbours in the layout, and the mean fraction of those layout neighbours that
share the point's label.  Evaluated over every point, in row blocks.
"""
import numpy as np


def layout_knn(y, k, block=4096, rows=None):
    """The k nearest layout neighbours (self excluded) of every point, or of
    the points `rows` (a fixed sample at large n), among all points."""
    import torch

    Y = torch.from_numpy(np.ascontiguousarray(y, np.float32)).cuda()
    rows = np.arange(Y.shape[0]) if rows is None else np.asarray(rows, np.int64)
    out = np.empty((rows.size, k), np.int64)
    for s in range(0, rows.size, block):
        e = min(rows.size, s + block)
        r = torch.from_numpy(rows[s:e]).cuda()
        d = torch.cdist(Y[r], Y)
        d[torch.arange(e - s, device=Y.device), r] = float("inf")
        out[s:e] = torch.topk(d, k, largest=False).indices.cpu().numpy()
    return out


def knn_preservation(y, idx, k=15, rows=None):
    nn = layout_knn(y, k, rows=rows)
    hi = np.asarray(idx)[:, :k] if rows is None else np.asarray(idx)[rows, :k]
    hits = (nn[:, :, None] == hi[:, None, :]).any(-1).sum(1)
    return float(hits.mean() / k)


def label_accuracy(y, labels, k=15, rows=None):
    nn = layout_knn(y, k, rows=rows)
    lab = np.asarray(labels)
    own = lab if rows is None else lab[rows]
    return float((lab[nn] == own[:, None]).mean())


def within_reference(ours, ref, rel=0.02, z=2.0):
    """Seed-averaged bar for Hogwild runs, whose quality moves from seed to seed
    by about as much as the bar itself: mean(ours) must reach (1 - rel) *
    mean(ref) minus z standard errors of the difference of the two means.
    Returns (passed, message)."""
    a, b = np.asarray(ours, np.float64), np.asarray(ref, np.float64)
    se = float(np.sqrt(a.var(ddof=1) / a.size + b.var(ddof=1) / b.size))
    floor = (1.0 - rel) * b.mean() - z * se
    msg = f"mean {a.mean():.5f} vs reference {b.mean():.5f} (se of difference {se:.5f}, floor {floor:.5f})"
    return bool(a.mean() >= floor), msg


def tsne_kl(row_ptr, col, val, y, block=4096):
    """Exact KL(P || Q) of a t-SNE layout, as evaluate_kl_f
    (src/tsne_neighbors.cpp:1247-1276): Z over all ordered pairs i != j in
    double, per-entry p log((p + 1e-9) / (q + 1e-9))."""
    import torch

    Y = torch.from_numpy(np.ascontiguousarray(y, np.float32)).cuda().double()
    n = Y.shape[0]
    z = 0.0
    for s in range(0, n, block):
        e = min(n, s + block)
        d2 = torch.cdist(Y[s:e], Y) ** 2
        q = 1.0 / (1.0 + d2)
        q[torch.arange(e - s, device=Y.device), torch.arange(s, e, device=Y.device)] = 0.0
        z += float(q.sum())
    rows = torch.repeat_interleave(torch.arange(n, device=Y.device),
                                   torch.from_numpy(np.diff(row_ptr)).cuda())
    cols = torch.from_numpy(np.asarray(col, np.int64)).cuda()
    p = torch.from_numpy(np.asarray(val, np.float64)).cuda()
    d2 = ((Y[rows] - Y[cols]) ** 2).sum(1)
    qn = (1.0 / (1.0 + d2)) / z
    return float((p * torch.log((p + 1e-9) / (qn + 1e-9))).sum())
