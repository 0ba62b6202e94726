"""The sharded UMAP epoch, checked on the CPU with gloo ranks.

A sharded UMAP session gives rank r a block of vertices and the edges that
touch it; each epoch the rank applies the moves of its own vertices against
the epoch-start layout and the blocks are then all-gathered.  In the Jacobi
mode every force is evaluated at the epoch-start positions, so this split is
exact: the oracle's Jacobi epoch (a restatement of embed_epoch_coo_delta_kernel
+ apply_delta_sanitize_layout_kernel, src/embedding_cuda_kernels.cpp:3136-3222)
run on a rank's edge subset gives, on that rank's vertices, the bits of the
unsharded epoch -- provided negatives are keyed on the tail vertex, as the
device-KNN path keys them, not on the edge's position in the list.
"""
import os
import socket

import numpy as np

import oracle as O
from fastembedr_b200 import api

WORLD = 2
EPOCHS = 4


def rank_edges(heads, tails, n, world, rank):
    b, e = api.umap_shard_vertices(n, world, rank)
    keep = ((heads >= b) & (heads < e)) | ((tails >= b) & (tails < e))
    return heads[keep], tails[keep], keep


def sharded_epochs(heads, tails, eps, y, n_epochs, world, rank, gather):
    n = y.shape[0]
    h, t, keep = rank_edges(heads, tails, n, world, rank)
    p = eps[keep]
    b, e = api.umap_shard_vertices(n, world, rank)
    for epoch in range(EPOCHS):
        full = O.umap_epoch_delta(h, t, p, y, epoch, n_epochs, hash_key_is_tail=True)
        y = gather(full[b:e], n)
    return y


def _rank(rank, world, port, outdir):
    import torch
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    d = np.load(os.path.join(outdir, "problem.npz"))

    def gather(block, n):
        per = api.umap_shard_vertices(n, world, 0)[1]
        buf = torch.zeros((per, 2), dtype=torch.float32)
        buf[:block.shape[0]] = torch.from_numpy(np.ascontiguousarray(block))
        parts = [torch.zeros_like(buf) for _ in range(world)]
        dist.all_gather(parts, buf)
        return torch.cat(parts).numpy()[:n].copy()

    y = sharded_epochs(d["heads"], d["tails"], d["eps"], d["init"], int(d["n_epochs"]), world, rank, gather)
    np.save(os.path.join(outdir, f"rank{rank}.npy"), y)
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_reproduce_the_unsharded_jacobi_epochs(umap_golden, tmp_path):
    import torch.multiprocessing as mp

    u = umap_golden
    heads = np.repeat(np.arange(u["offsets"].size - 1), np.diff(u["offsets"])).astype(np.int32)
    tails = np.asarray(u["neighbors"], np.int32)
    eps = np.asarray(u["epochs_per_sample"], np.float32)
    init = np.asarray(u["init"], np.float32)
    n_epochs = 50
    np.savez(tmp_path / "problem.npz", heads=heads, tails=tails, eps=eps, init=init, n_epochs=n_epochs)
    mp.start_processes(_rank, args=(WORLD, _free_port(), str(tmp_path)), nprocs=WORLD, join=True,
                       start_method="spawn")
    want = init.copy()
    for epoch in range(EPOCHS):
        want = O.umap_epoch_delta(heads, tails, eps, want, epoch, n_epochs, hash_key_is_tail=True)
    assert np.abs(want - init).max() > 0  # the epochs moved something
    for r in range(WORLD):
        got = np.load(tmp_path / f"rank{r}.npy")
        assert np.array_equal(got, want)


def test_shard_vertices_partition():
    for n, world in ((1, 1), (10, 3), (5000, 2), (2_000_000, 8), (7, 8)):
        blocks = [api.umap_shard_vertices(n, world, r) for r in range(world)]
        assert blocks[0][0] == 0 and blocks[-1][1] == n
        assert all(e0 == b1 for (_, e0), (b1, _) in zip(blocks, blocks[1:]))
        assert all(e - b <= -(-n // world) for b, e in blocks)
