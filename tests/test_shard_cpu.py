"""The sharded t-SNE decomposition, checked on the CPU with gloo ranks.

A sharded session splits one iteration's gradient by points: each rank spreads
the charges of its own block of points, the charge grids are summed across
ranks, every rank convolves the summed grid, and each rank finishes the
gradient of its own points; the blocks are then gathered.  This file restates
that data flow in NumPy (float64 FFT convolution, charges in 64-bit fixed point
as on the device) and runs it as two gloo processes, checking that

  * the summed fixed-point charges, hence the gathered gradient, are
    bit-identical to the one-rank result (what makes a sharded device run
    independent of the number of GPUs);
  * Z taken from the grid identity (sum of charge * phi_q over the nodes, - n)
    needs no collective of its own and matches the oracle's Z;
  * the gathered gradient matches the oracle's FFT gradient
    (compute_gradient_fft_grid_f, src/tsne_neighbors.cpp:1076-1182).

The host-side pieces of the device path -- the row blocks of shard_rows and
the NCCL id exchange -- are checked here too.
"""
import os
import socket

import numpy as np
import pytest

import oracle as O
from fastembedr_b200 import api

WORLD = 2


def geometry(y, g):
    """Grid geometry of compute_gradient_fft_grid_f (:1090-1106), in float32."""
    y = y.astype(np.float32)
    mn, mx = y.min(0), y.max(0)
    c = np.float32(0.5) * (mn + mx)
    span = np.float32(max(mx[0] - mn[0], mx[1] - mn[1]))
    half = np.float32(0.55) * span + np.float32(1e-3)
    lower = c - half
    spacing = np.float32(2.0) * half / np.float32(g - 1)
    return lower, spacing


def cells(y, lower, spacing, g):
    t = (y.astype(np.float32) - lower) * (np.float32(1.0) / spacing)
    t = np.clip(t, 0.0, np.float32(g - 1))
    o = np.clip(np.floor(t).astype(np.int64), 0, g - 2)
    return o, (t - o).astype(np.float32)


def splat_fixed(y, rows, lower, spacing, g, scale):
    """Charges {1, x, y} of points `rows`, each contribution rounded to
    2**-log2(scale) units and summed as int64 (order-independent)."""
    o, t = cells(y[rows], lower, spacing, g)
    w = [(1 - t[:, 0]) * (1 - t[:, 1]), t[:, 0] * (1 - t[:, 1]), (1 - t[:, 0]) * t[:, 1], t[:, 0] * t[:, 1]]
    off = [(0, 0), (1, 0), (0, 1), (1, 1)]
    q = np.zeros((3, g, g), np.int64)
    p = y[rows].astype(np.float64)
    for wk, (dx, dy) in zip(w, off):
        wk = wk.astype(np.float64)
        for plane, v in enumerate((wk, wk * p[:, 0], wk * p[:, 1])):
            np.add.at(q[plane], (o[:, 1] + dy, o[:, 0] + dx), np.rint(v * scale).astype(np.int64))
    return q


def potentials(charges, spacing, g):
    """Linear convolution of the charges with q = 1/(1+d^2) and q^2 on the
    zero-padded 2g torus: planes phi_q2, phi_xq2, phi_yq2, phi_q."""
    m = 2 * g
    d = np.arange(m)
    d = np.where(d < g, d, d - m).astype(np.float64) * float(spacing)
    d2 = d[None, :] ** 2 + d[:, None] ** 2
    kq = 1.0 / (1.0 + d2)
    kq[g, :] = 0.0
    kq[:, g] = 0.0
    fq, fq2 = np.fft.rfft2(kq), np.fft.rfft2(kq * kq)
    out = []
    for plane, kern in ((0, fq2), (1, fq2), (2, fq2), (0, fq)):
        pad = np.zeros((m, m))
        pad[:g, :g] = charges[plane]
        out.append(np.fft.irfft2(np.fft.rfft2(pad) * kern, s=(m, m))[:g, :g])
    return out


def gather(pot, y, rows, lower, spacing, g):
    o, t = cells(y[rows], lower, spacing, g)
    tx, ty = t[:, 0].astype(np.float64), t[:, 1].astype(np.float64)
    i0, j0 = o[:, 1], o[:, 0]

    def at(p):
        return ((1 - tx) * (1 - ty) * p[i0, j0] + tx * (1 - ty) * p[i0, j0 + 1] +
                (1 - tx) * ty * p[i0 + 1, j0] + tx * ty * p[i0 + 1, j0 + 1])

    return [at(p) for p in pot]


def sharded_gradient(P, y, ex, g, world, rank, reduce_charges, gather_rows):
    """One gradient evaluation of a `world`-way sharded session, as rank `rank`."""
    n = y.shape[0]
    lower, spacing = geometry(y, g)
    begin, end = api.shard_rows(n, world, rank)
    scale = 2.0 ** 40
    local = splat_fixed(y, np.arange(begin, end), lower, spacing, g, scale)
    charges = reduce_charges(local).astype(np.float64) / scale
    pot = potentials(charges, spacing, g)
    z = float((charges[0] * pot[3]).sum()) - n
    rows = np.arange(begin, end)
    phi_q2, phi_xq2, phi_yq2, _ = gather(pot, y, rows, lower, spacing, g)
    yr = y[rows].astype(np.float64)
    grad = np.zeros((end - begin, 2))
    grad[:, 0] = -(yr[:, 0] * phi_q2 - phi_xq2) / z
    grad[:, 1] = -(yr[:, 1] * phi_q2 - phi_yq2) / z
    grad += O.tsne_attractive(P, y, ex)[begin:end]
    return gather_rows(grad, n), z


def _rank(rank, world, port, outdir):
    import torch
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    data = np.load(os.path.join(outdir, "problem.npz"))
    P = O.Csr(data["row_ptr"], data["col"], data["val"])

    def reduce_charges(local):
        t = torch.from_numpy(local)
        dist.all_reduce(t)
        return t.numpy()

    def gather_rows(block, n):
        per = api.shard_rows(n, world, 0)[1]
        buf = torch.zeros((per, 2), dtype=torch.float64)
        buf[:block.shape[0]] = torch.from_numpy(block)
        parts = [torch.zeros_like(buf) for _ in range(world)]
        dist.all_gather(parts, buf)
        return torch.cat(parts).numpy()[:n]

    grad, z = sharded_gradient(P, data["y"], float(data["ex"]), int(data["grid"]), world, rank,
                               reduce_charges, gather_rows)
    np.savez(os.path.join(outdir, f"rank{rank}.npz"), grad=grad, z=z)
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_match_one_rank_and_oracle(tsne_golden, tmp_path):
    import torch.multiprocessing as mp

    g = tsne_golden
    P = O.Csr(g["row_ptr"], g["col"], g["val"])
    y, ex, grid = g["states"][1], float(g["exaggeration"][1]), int(g["grid"])
    np.savez(tmp_path / "problem.npz", row_ptr=g["row_ptr"], col=g["col"], val=g["val"], y=y, ex=ex, grid=grid)
    mp.start_processes(_rank, args=(WORLD, _free_port(), str(tmp_path)), nprocs=WORLD, join=True,
                       start_method="spawn")
    one, z1 = sharded_gradient(P, y, ex, grid, 1, 0, lambda c: c, lambda b, n: b)
    for r in range(WORLD):
        got = np.load(tmp_path / f"rank{r}.npz")
        assert np.array_equal(got["grad"], one)
        assert float(got["z"]) == z1
    want, zref = O.tsne_gradient_fft(P, y, ex, grid, return_z=True)
    rel = np.linalg.norm(one - want) / np.linalg.norm(want)
    assert rel < 1e-4, rel
    assert abs(z1 - zref) / abs(zref) < 1e-5


@pytest.mark.parametrize("n,world", [(1, 1), (100, 8), (1000, 3), (6000, 2), (1_000_000, 8), (33, 2)])
def test_shard_rows_partition(n, world):
    blocks = [api.shard_rows(n, world, r) for r in range(world)]
    assert blocks[0][0] == 0 and blocks[-1][1] == n
    for (b0, e0), (b1, e1) in zip(blocks, blocks[1:]):
        assert e0 == b1
    per = blocks[0][1] - blocks[0][0] if world > 1 else None
    for b, e in blocks:
        assert (b % 32 == 0 or b == n) and 0 <= e - b  # empty trailing blocks start at n
        if per is not None:
            assert e - b <= per
    if per is not None:
        assert per % 32 == 0 or per == n
        # the in-place all-gather writes world * per rows: within the padding the session allocates
        assert world * per - n < 32 * 256


def test_nccl_unique_id_is_fresh():
    a, b = api.nccl_unique_id(), api.nccl_unique_id()
    assert len(a) == 128 and len(b) == 128 and a != b
