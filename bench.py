"""Benchmark of the B200 embedding-optimizer backend.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload tsne_1m|tsne_70k|tsne_10k]

A *step* is one openTSNE optimizer iteration (gradient + update) over the whole
workload.  The default workload is configuration 3 of the benchmark set
(N = 1,000,000 points, 20-component anisotropic Gaussian mixture in 50-D with
Dirichlet weights, exact k = 90 KNN, perplexity 30, FFT grid repulsion) -- the
configuration the headline metric (t-SNE iterations/s at N = 1M) is quoted on.

Our arm (--impl ours) prints one JSON line with
  value      iterations/s with P, layout and optimizer state resident in HBM
  e2e        iterations/s of the full C-ABI call (fastembedr_cuda_opentsne_fft_from_knn_float)
             from pageable host KNN, as the reference's R wrapper passes it, to host layout:
             H2D, P build, 750 iterations, D2H (the same call from pinned buffers beside it)
  roofline   the fused gradient/update kernel: algorithmic bytes per launch over its
             CUDA-event duration, against MEASURED_PEAKS.json's HBM copy bandwidth
  cpu_baseline  the reference's own CPU loop (oracle/_ref) on the first iterations of the
             same workload (about 10 s of loop, --cpu-seconds), all host threads
The reference arm (--impl reference) times the reference's own CPU
implementation of the same loop (rank 0 only); with --reference-backend cuda it
times the reference's own CUDA backend through the e2e entry point instead.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    "tsne_1m": dict(spec="tsne_1m", k=90, perplexity=30.0),
    "tsne_70k": dict(spec="tsne_70k", k=90, perplexity=30.0),
    "tsne_10k": dict(spec="tsne_10k", k=90, perplexity=30.0),
    "tsne_200k": dict(spec="tsne_200k", k=90, perplexity=30.0),
    # N = 2M, generated like configuration 3: the size the scaling target names
    "tsne_2m": dict(spec="tsne_2m", k=90, perplexity=30.0),
    # UMAP configurations 1 and 4: k = 15 fuzzy graph, negative_sample_rate 5,
    # a/b for min_dist 0.1, learning rate 1, start U(-10, 10).
    "umap_70k": dict(spec="umap_70k", k=15, kind="umap", n_epochs=500),
    "umap_2m": dict(spec="umap_2m", k=15, kind="umap", n_epochs=200),
}
UMAP_NSR, UMAP_MIN_DIST, UMAP_LR = 5, 0.1, 1.0
EE_ITER, N_ITER, EE, EX, MOM = 250, 500, 12.0, 1.0, 0.8
MIN_GAIN, MAX_STEP = 0.01, 5.0
FALLBACK_HBM_GBS = 6650.0


L2_BYTES = 126 * 1024 * 1024  # B200


def l2_note(stream_bytes: int, what: str) -> str:
    """How the timed loop relates to L2: no flush is made between iterations,
    so only a streamed input larger than L2 makes the figure an HBM one."""
    if stream_bytes > L2_BYTES:
        return f"inputs larger than L2 ({what} is {stream_bytes / 1e9:.2f} GB), no flush"
    return f"inputs fit in L2 ({what} is {stream_bytes / 1e9:.3f} GB): an in-L2 figure, not an HBM one"


def median_call_seconds(call, reps: int = 3) -> float:
    """Median wall time of `reps` calls of a synchronous call, after one warm call."""
    call()
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        call()
        times.append(time.perf_counter() - t0)
    return float(np.median(times))


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def make_inputs(workload: str, device: str, producer: str = "b200"):
    """The workload's exact KNN and init.  The reference arm builds its inputs
    with torch's brute force (producer="torch"), so it runs no code of this
    library; both give the exact KNN."""
    from fastembedr_b200 import synthetic as S

    w = WORKLOADS[workload]
    spec = S.CONFIGS[w["spec"]]
    t0 = time.time()
    x, _ = S.gaussian_mixture(spec)
    idx, dist = S.exact_knn(x, w["k"], device=device, producer=producer)
    log(f"[bench] {workload}: n={spec.n} k={w['k']} inputs in {time.time() - t0:.1f}s")
    return idx, dist, S.tsne_init(spec.n, seed=0)


def phase_params(i: int, n: int):
    """Parameters of iteration i of the default schedule (250 early + 500 normal)."""
    if (i % (EE_ITER + N_ITER)) < EE_ITER:
        return EE, MOM, float(np.float32(n / EE))
    return EX, MOM, float(np.float32(n / EX))


def run_schedule(sess, start: int, count: int, n: int, init=None):
    """Iterations [start, start+count) of back-to-back standard runs: every
    750 iterations the session restarts from `init` with fresh optimizer state
    (a new run), so every timed iteration belongs to the standard schedule."""
    i = start
    while i < start + count:
        if init is not None and i > 0 and i % (EE_ITER + N_ITER) == 0:
            sess.set_layout(init, reset_state=True)
        ex, mom, lr = phase_params(i, n)
        cyc = i % (EE_ITER + N_ITER)
        left = (EE_ITER - cyc) if cyc < EE_ITER else (EE_ITER + N_ITER - cyc)
        step = min(left, start + count - i)
        sess.iterate(step, ex, mom, lr, MIN_GAIN, MAX_STEP)
        i += step


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def profile_traffic(kernel: str, workload: str):
    """DRAM bytes per launch from the committed ncu summary, if one exists."""
    path = os.path.join(ROOT, "profiles", f"{kernel}_{workload}.md")
    if not os.path.exists(path):
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", open(path).read())
    return float(m.group(1)) if m else None


def cpu_baseline_tsne(idx, dist, perplexity, init, chunk: int, seconds: float,
                      max_iters: int = EE_ITER + N_ITER):
    """The reference's own CPU loop on the first iterations of the standard
    schedule: chunks of at most `chunk` iterations (none crossing the phase
    boundary), continuing the optimizer state, until the loop has run
    `seconds` or `max_iters` iterations (at most one run); P build excluded."""
    import oracle as O

    threads = os.cpu_count() or 1
    n = idx.shape[0]
    max_iters = min(max_iters, EE_ITER + N_ITER)
    use_ref = O.ref_available()
    t0 = time.time()
    P = O.ref_tsne_build_p(idx, dist, perplexity, threads=threads) if use_ref else O.tsne_build_p(idx, dist, perplexity)
    setup = time.time() - t0

    def sample(variant, limit_s, limit_iters):
        upd = np.zeros_like(init)
        gains = np.ones_like(init)
        y = O.tsne_zero_mean(init)
        iters, secs = 0, 0.0
        while secs < limit_s and iters < limit_iters:
            ex, mom, lr = phase_params(iters, n)
            step = min(chunk, (EE_ITER if iters < EE_ITER else EE_ITER + N_ITER) - iters, limit_iters - iters)
            if use_ref:
                y, upd, gains, s = O.ref_tsne_iterate(P, y, upd, gains, step, ex, mom, lr, MIN_GAIN, MAX_STEP,
                                                      threads=threads, variant=variant)
            else:
                t1 = time.time()
                y, upd, gains = O.tsne_iterate(P, y, upd, gains, step, ex, mom, lr, MIN_GAIN, MAX_STEP)
                s = time.time() - t1
            iters, secs = iters + step, secs + s
        return iters, secs

    iters, secs = sample("O2", seconds, max_iters)
    kind, cores = ("reference", threads) if use_ref else ("port", 1)
    out = {"value": iters / secs, "unit": "iterations/s", "cores": cores, "kind": kind, "iterations": iters,
           "seconds": secs, "flags": "-O2 (R's default package build)" if use_ref else "-O2",
           "sample": f"the first {iters} optimizer iterations of the full n={n} workload, {secs:.1f}s of loop "
                     f"(P build {setup:.1f}s excluded), {cores} threads"}
    if use_ref and O.ref_available("O3"):
        it3, s3 = sample("O3", float("inf"), iters)  # the same iterations
        out["O3"] = {"value": it3 / s3, "seconds": s3, "flags": "-O3 -march=x86-64-v3"}
    return out


def bench_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    w = WORKLOADS[args.workload]
    device = "cuda" if _cuda_ok() else None
    idx, dist, init = make_inputs(args.workload, device, producer="torch")
    base = cpu_baseline_tsne(idx, dist, w["perplexity"], init, args.cpu_iters, args.cpu_seconds,
                             max_iters=max(args.cpu_iters, args.steps))
    iters = base["iterations"]
    line = {
        "impl": "reference", "metric": "tsne_iterations_per_second", "value": base["value"],
        "unit": "iterations/s", "n_gpus": 0, "steps": iters, "warmup": 0,
        "ms_per_step": 1000.0 / base["value"], "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "n": int(idx.shape[0]), "k": w["k"],
                   "perplexity": w["perplexity"], "grid": "reference CPU policy"},
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample", "flags", "O3")
                         if k in base},
        "e2e": {"value": base["value"], "unit": "iterations/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def bench_reference_umap(args):
    """The reference's CPU path end to end on the host: its own fuzzy graph
    (build_graph_csr_native_direct_values, src/fast_knn_umap.cpp:1553-1771) as
    COO, then its COO optimizer on the first epochs; only the optimizer is timed."""
    rank, _, _ = dist_env()
    if rank != 0:
        return 0
    import oracle as O

    idx, dist, init = umap_inputs(args.workload, "cuda" if _cuda_ok() else None, producer="torch")
    t0 = time.time()
    g = O.ref_umap_graph(idx, dist, threads=os.cpu_count() or 1) if O.ref_available() else O.umap_graph(idx, dist)
    graph = {"heads": g.heads(), "tails": g.neighbors, "epochs_per_sample": g.epochs_per_sample}
    log(f"[bench] reference CPU graph: {graph['heads'].size} edges in {time.time() - t0:.1f}s")
    base = cpu_baseline_umap(graph, init)
    line = {
        "impl": "reference", "metric": "umap_edge_updates_per_second", "value": base["value"],
        "unit": "edge_updates/s", "n_gpus": 0, "steps": 1, "warmup": 0,
        "ms_per_step": None, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "n": int(idx.shape[0]), "k": int(idx.shape[1]),
                   "n_edges": int(graph["heads"].size)},
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample", "flags", "O3")
                         if k in base},
        "e2e": {"value": base["value"], "unit": "edge_updates/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def reference_cuda_tsne(idx, dist, init, perplexity, reps: int = 1):
    """The reference's own CUDA backend (oracle/_ref/libferef_cuda.so, its
    src/embedding_cuda_kernels.cpp built for sm_100a) on the same host KNN,
    through the same entry point as our e2e leg: the GPU bar, reported beside
    the CPU baseline and never part of our timed region.  None when not built."""
    import oracle as O

    if not O.ref_cuda_available():
        return None
    n, k = idx.shape

    def call():
        O.ref_cuda_tsne(idx, dist, init, perplexity=perplexity, early_exaggeration_iter=EE_ITER, n_iter=N_ITER,
                        early_exaggeration=EE, exaggeration=EX, momentum=MOM, min_gain=MIN_GAIN,
                        max_step_norm=MAX_STEP)

    secs = median_call_seconds(call, reps)  # the warm call loads modules and makes cuFFT plans
    return {"value": (EE_ITER + N_ITER) / secs, "unit": "iterations/s", "seconds_per_call": secs,
            "timing": f"median of {reps} call(s) after a warm one",
            "grid": "reference CUDA policy (G = 1024 at n >= 100k)",
            "call": "fastembedr_cuda_opentsne_fft_from_knn_float of the reference (750 iterations, pageable host "
                    "KNN), src/embedding_cuda_kernels.cpp built for sm_100a"}


def reference_cuda_umap(idx, dist, n_epochs, graph_edges, units, reps: int = 3):
    """The reference's own CUDA fused UMAP path (graph, diffusion start,
    epochs) on the same host KNN; edge updates counted as this library's
    positive samples of a whole run (the same schedule).  None when not built."""
    import oracle as O
    from fastembedr_b200 import api

    if not O.ref_cuda_available():
        return None
    n, k = idx.shape
    a, b = api.find_ab_params(1.0, UMAP_MIN_DIST)
    sni = api.umap_config(n, k)["spectral_n_iter"]

    def call():
        O.ref_cuda_umap_fused(idx, dist, n_epochs, negative_sample_rate=UMAP_NSR, learning_rate=UMAP_LR,
                              a=a, b=b, spectral_n_iter=sni, seed=42)

    secs = median_call_seconds(call, reps)
    return {"value": units / secs, "unit": "edge_updates/s", "seconds_per_call": secs,
            "timing": f"median of {reps} calls after a warm one", "n_edges": int(graph_edges),
            "call": f"fastembedr_cuda_umap_from_knn_spectral_float of the reference ({n_epochs} epochs, host KNN: "
                    f"graph, diffusion start, epochs), src/embedding_cuda_kernels.cpp built for sm_100a"}


def bench_reference_cuda(args):
    """The reference's own CUDA backend (oracle/_ref/libferef_cuda.so, its
    src/embedding_cuda_kernels.cpp built for sm_100a), timed through the same
    entry point as our arm's e2e leg: host KNN in, host layout out, whole call.
    Opt-in (--reference-backend cuda): the GPU bar beside the CPU reference arm."""
    rank, _, local = dist_env()
    if rank != 0:
        return 0
    import torch

    import oracle as O

    if not O.ref_cuda_available():
        print(json.dumps({"impl": "reference", "backend": "cuda",
                          "unavailable": "oracle/_ref/libferef_cuda.so not built"}), flush=True)
        return 0
    torch.cuda.set_device(local)
    w = WORKLOADS[args.workload]
    umap = w.get("kind") == "umap"
    reps = 3
    if umap:
        from fastembedr_b200 import api

        idx, dist, _ = umap_inputs(args.workload, f"cuda:{local}", producer="torch")
        n, k = idx.shape
        a, b = api.find_ab_params(1.0, UMAP_MIN_DIST)
        sni = api.umap_config(n, k)["spectral_n_iter"]
        with api.UmapSession.from_knn(idx, dist) as s:
            units, _ = s.count_samples(0, w["n_epochs"], UMAP_NSR)
            n_edges = s.info()["n_edges"]

        def call():
            O.ref_cuda_umap_fused(idx, dist, w["n_epochs"], negative_sample_rate=UMAP_NSR, learning_rate=UMAP_LR,
                                  a=a, b=b, spectral_n_iter=sni, seed=42)

        metric, unit = "umap_edge_updates_per_second", "edge_updates/s"
        entry = (f"fastembedr_cuda_umap_from_knn_spectral_float ({w['n_epochs']} epochs, host KNN: graph, "
                 f"diffusion start, epochs)")
        cfg = {"workload": args.workload, "n": int(n), "k": int(k), "n_edges": int(n_edges),
               "units": "positive samples of this library's edge list for the schedule"}
    else:
        idx, dist, init = make_inputs(args.workload, f"cuda:{local}", producer="torch")
        n, k = idx.shape
        units = EE_ITER + N_ITER

        def call():
            O.ref_cuda_tsne(idx, dist, init, perplexity=w["perplexity"], early_exaggeration_iter=EE_ITER,
                            n_iter=N_ITER, early_exaggeration=EE, exaggeration=EX, momentum=MOM,
                            min_gain=MIN_GAIN, max_step_norm=MAX_STEP)

        metric, unit = "tsne_iterations_per_second", "iterations/s"
        entry = "fastembedr_cuda_opentsne_fft_from_knn_float (750 iterations, host KNN)"
        cfg = {"workload": args.workload, "n": int(n), "k": int(k), "perplexity": w["perplexity"],
               "grid": "reference CUDA policy"}
    secs = median_call_seconds(call, reps)  # the warm call loads modules and makes cuFFT plans
    value = units / secs
    line = {
        "impl": "reference", "backend": "cuda (the reference's src/embedding_cuda_kernels.cpp, sm_100a)",
        "metric": metric, "value": value, "unit": unit, "n_gpus": 1, "steps": reps, "warmup": 1,
        "timing": f"median of {reps} calls after a warm one",
        "ms_per_step": None, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic", "config": cfg, "seconds_per_call": secs, "call": entry,
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": int(idx.size * 8),
                "d2h_bytes_per_step": int(n * 8)},
    }
    print(json.dumps(line), flush=True)
    return 0


def _cuda_ok():
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def shared_inputs(args, rank: int, world: int, local: int):
    """The workload's KNN and init, made on rank 0 and broadcast, so that every
    rank of a sharded run holds identical inputs."""
    import torch
    import torch.distributed as tdist

    if world == 1:
        return make_inputs(args.workload, f"cuda:{local}")
    from fastembedr_b200 import synthetic as S

    w = WORKLOADS[args.workload]
    n, k = S.CONFIGS[w["spec"]].n, w["k"]
    if rank == 0:
        idx, dist, init = make_inputs(args.workload, f"cuda:{local}")
        t = [torch.from_numpy(idx).cuda(), torch.from_numpy(dist).cuda(), torch.from_numpy(init).cuda()]
    else:
        t = [torch.empty((n, k), dtype=torch.int32, device="cuda"),
             torch.empty((n, k), dtype=torch.float32, device="cuda"),
             torch.empty((n, 2), dtype=torch.float32, device="cuda")]
    for x in t:
        tdist.broadcast(x, 0)
    return tuple(x.cpu().numpy() for x in t)


def bench_ours(args):
    import torch
    import torch.distributed as tdist

    from fastembedr_b200 import _lib, api

    rank, world, local = dist_env()
    w = WORKLOADS[args.workload]
    idx, dist, init = shared_inputs(args, rank, world, local)
    n, k = idx.shape
    if not api.cuda_available():
        raise RuntimeError("libfastembedr_b200 reports no usable B200")

    # --- device-resident loop (value) ---
    d_idx = torch.from_numpy(idx).cuda()
    d_dist = torch.from_numpy(dist).cuda()
    t0 = time.time()
    sess = api.TsneSession.from_knn(d_idx, d_dist, perplexity=w["perplexity"], init=init)
    if world > 1:
        # One process per GPU: each rank owns 1/world of the points (rows of P),
        # the charge grid is all-reduced and the layout all-gathered per iteration.
        sess.shard_over()
    info = sess.info()
    log(f"[bench] rank {rank}: P nnz={info['nnz']} padded={info['nnz_padded']} G={info['grid']} "
        f"(setup {time.time() - t0:.2f}s)")
    del d_idx, d_dist
    stream = torch.cuda.ExternalStream(sess.stream)
    init_dev = torch.from_numpy(init).cuda()  # restarts inside the timed region copy D2D
    torch.cuda.synchronize()
    run_schedule(sess, 0, args.warmup, n)
    sess.set_layout(init_dev, reset_state=True)  # the timed region starts a fresh standard run
    for i in (0, EE_ITER):  # both phases' iteration graphs are captured before timing
        sess.prepare(*phase_params(i, n), MIN_GAIN, MAX_STEP)
    torch.cuda.synchronize()
    if world > 1:
        tdist.barrier()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        start.record(stream)
        run_schedule(sess, 0, args.steps, n, init_dev)
        stop.record(stream)
        torch.cuda.synchronize()
    elapsed_ms = start.elapsed_time(stop)
    if world > 1:
        t = torch.tensor([elapsed_ms], device="cuda")
        tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    ms_per_step = elapsed_ms / args.steps
    # The whole job advances one iteration per step on every rank together.
    value = args.steps / (elapsed_ms / 1000.0)

    # --- one complete standard run (250 + 500 iterations, spatial reorders
    # included) in a single CUDA-event interval, beside the K timed steps ---
    full_iters = EE_ITER + N_ITER
    sess.set_layout(init_dev, reset_state=True)
    torch.cuda.synchronize()
    if world > 1:
        tdist.barrier()
    start.record(stream)
    run_schedule(sess, 0, full_iters, n)
    stop.record(stream)
    torch.cuda.synchronize()
    full_ms = start.elapsed_time(stop)
    if world > 1:
        t = torch.tensor([full_ms], device="cuda")
        tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
        full_ms = float(t.item())
    full_run = {"iterations": full_iters, "ms": full_ms, "value": full_iters / (full_ms / 1000.0),
                "unit": "iterations/s", "timing": "one CUDA-event interval around a whole standard run from the "
                                                  "init (P and state resident)"}

    # --- per-kernel CUDA-event timing of one full standard run (roofline) ---
    sess.set_layout(init_dev, reset_state=True)
    sess.profile(True)
    prof_iters = EE_ITER + N_ITER
    run_schedule(sess, 0, prof_iters, n, init_dev)
    times = sess.kernel_times()
    sess.profile(False)
    grid = info["grid"]
    nnz = info["nnz"]
    # Algorithmic bytes of one grad_update launch: row_ptr, (col, val) per symmetric entry,
    # layout read, update/gains read+write, layout write, potentials (4 floats per node).
    # A shard streams its own rows: 1/world of the points and (rows are interleaved
    # in Morton order) about 1/world of P.
    rows = n / world
    alg_bytes = 4 * (rows + 1) + 8 * nnz / world + 8 * rows + 16 * rows + 24 * rows + 16 * grid * grid
    # The attraction + update of every row runs in staged_grad_kernel (row blocks
    # whose column union is staged in shared memory) or grad_update_kernel (the
    # rest); both launch once per iteration, so their sum is one "launch".
    gu_ms, gu_cnt = times["grad_update_kernel"]
    st_ms, _ = times.get("staged_grad_kernel", (0.0, 0))
    gu_avg_s = (gu_ms + st_ms) / max(gu_cnt, 1) / 1000.0
    per_rank_gu = [gu_avg_s * 1000.0]
    if world > 1:
        # every rank's attraction time: the slowest rank paces the collectives
        box = [None] * world
        tdist.all_gather_object(box, gu_avg_s * 1000.0)
        per_rank_gu = box
    hbm, peak_kind = peaks()
    achieved = alg_bytes / gu_avg_s / 1e9
    total_ms = sum(v[0] for v in times.values())
    kernel_share = {kname: round(v[0] / total_ms, 4) for kname, v in times.items()}

    # --- end to end through the public API from host buffers ---
    # The reference's R wrapper hands the library pageable std::vector copies
    # (src/embedding_cuda_impl.cpp:776-784, 817), so the headline e2e passes
    # plain (pageable) host arrays; the same call from pinned buffers is
    # reported beside it.
    e2e = None
    if not args.skip_e2e and world == 1:
        import ctypes

        L = _lib.load()
        idx_cm = np.ascontiguousarray(idx.T)
        dist_cm = np.ascontiguousarray(dist.T)
        init_h = np.ascontiguousarray(init, dtype=np.float32)
        out_h = np.empty((n, 2), np.float32)

        def e2e_call(i_ptr, d_ptr, init_ptr, out_ptr):
            def call():
                rc = L.fastembedr_cuda_opentsne_fft_from_knn_float(
                    ctypes.c_void_p(i_ptr), ctypes.c_void_p(d_ptr),
                    ctypes.cast(init_ptr, ctypes.POINTER(ctypes.c_float)), 1, n, k, 2,
                    w["perplexity"], EE_ITER, N_ITER, EE, EX, 0.0, 1, MOM, MOM, MIN_GAIN, MAX_STEP, 42, 0,
                    ctypes.cast(out_ptr, ctypes.POINTER(ctypes.c_float)))
                _lib.check(rc, "fastembedr_cuda_opentsne_fft_from_knn_float")
            return call

        e2e_s = median_call_seconds(e2e_call(idx_cm.ctypes.data, dist_cm.ctypes.data, init_h.ctypes.data,
                                             out_h.ctypes.data))  # the warm call loads the module
        p_idx = torch.from_numpy(idx_cm).pin_memory()
        p_dist = torch.from_numpy(dist_cm).pin_memory()
        p_init = torch.from_numpy(init_h).pin_memory()
        p_out = torch.empty((n, 2), dtype=torch.float32).pin_memory()
        pinned_s = median_call_seconds(e2e_call(p_idx.data_ptr(), p_dist.data_ptr(), p_init.data_ptr(),
                                                p_out.data_ptr()))
        del p_idx, p_dist, p_init, p_out
        e2e = {"value": (EE_ITER + N_ITER) / e2e_s, "unit": "iterations/s",
               "h2d_bytes_per_step": int(idx_cm.nbytes + dist_cm.nbytes + init_h.nbytes),
               "d2h_bytes_per_step": int(out_h.nbytes), "seconds_per_call": e2e_s,
               "host_buffers": "pageable (numpy), as the reference's R wrapper passes them",
               "timing": "median of 3 calls after a warm one",
               "call": "fastembedr_cuda_opentsne_fft_from_knn_float (750 iterations, host KNN)",
               "pinned": {"value": (EE_ITER + N_ITER) / pinned_s, "seconds_per_call": pinned_s}}
    elif not args.skip_e2e:
        # Every rank: pinned host KNN -> device, P build, shard, 750 iterations,
        # layout back to the host; max over ranks.  The NCCL communicator is made
        # once per process, like the process group, and lent to each run.
        idx_h = torch.from_numpy(idx).pin_memory()
        dist_h = torch.from_numpy(dist).pin_memory()
        out_h = torch.empty((n, 2), dtype=torch.float32).pin_memory()
        comm = api.NcclComm.over()

        def call():
            d_i = idx_h.cuda(non_blocking=True)
            d_d = dist_h.cuda(non_blocking=True)
            torch.cuda.synchronize()
            with api.TsneSession.from_knn(d_i, d_d, perplexity=w["perplexity"], init=init) as s2:
                s2.shard_comm(comm)
                s2.run(EE_ITER, N_ITER, EE, EX, "auto", MOM, MOM, MIN_GAIN, MAX_STEP)

        call()
        tdist.barrier()
        t0 = time.perf_counter()
        call()
        e2e_s = time.perf_counter() - t0
        t = torch.tensor([e2e_s], device="cuda")
        tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
        e2e_s = float(t.item())
        e2e = {"value": (EE_ITER + N_ITER) / e2e_s, "unit": "iterations/s",
               "h2d_bytes_per_step": int(idx_h.numel() * 4 + dist_h.numel() * 4 + init.size * 4),
               "d2h_bytes_per_step": int(out_h.numel() * 4), "seconds_per_call": e2e_s,
               "call": "TsneSession.from_knn + shard_comm + run (750 iterations, pinned host KNN), every rank; "
                       "communicator made once per process"}
        comm.close()

    sess.close()
    # Baselines, outside every timed region: the reference's own CPU loop
    # (cpu_baseline) and its own CUDA backend (reference_cuda, the GPU bar).
    cpu = ref_gpu = None
    if rank == 0 and world == 1 and not args.skip_cpu:
        cpu = cpu_baseline_tsne(idx, dist, w["perplexity"], init, args.cpu_iters, args.cpu_seconds)
        if not args.skip_reference_cuda:
            ref_gpu = reference_cuda_tsne(idx, dist, init, w["perplexity"])
    del idx, dist
    # UMAP edge updates/s, the metric's second half, on configuration 4
    # (N = 2M), in the same line.
    umap = None
    if args.workload == "tsne_1m" and not args.skip_umap:
        umap = umap_measure("umap_2m", WORKLOADS["umap_2m"]["n_epochs"], 3, args.skip_e2e, args.skip_cpu,
                            ref_cuda=not args.skip_reference_cuda)
    if rank == 0:
        per_iter = 7  # splat, 3 FFT passes, staged + gather gradient/update, statistics (NCCL not counted)
        line = {
            "metric": "tsne_iterations_per_second", "value": value, "unit": "iterations/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": args.workload, "n": int(n), "k": int(k), "perplexity": w["perplexity"],
                       "grid": grid, "nnz": int(nnz), "schedule": "250 early (ex 12) + 500 normal, lr n/ex",
                       "l2": l2_note(8 * info["nnz_padded"], "P"),
                       "parallelism": f"points sharded over {world} GPUs (NCCL all-reduce of the charge grid "
                                      f"+ all-gather of the layout per iteration)" if world > 1 else "single"},
            "roofline": {"kernel": "staged_grad_kernel + grad_update_kernel (attraction, gather, update)",
                         "bound": "hbm", "achieved": achieved,
                         "peak": hbm, "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / hbm,
                         "algorithmic_bytes_per_launch": alg_bytes,
                         "avg_launch_ms": gu_avg_s * 1000.0,
                         "traffic": profile_traffic("grad_update_kernel", args.workload) if world == 1 else None},
            "kernel_share": kernel_share,
            "kernel_ms": {kname: v[0] / max(v[1], 1) for kname, v in times.items()},
            "grad_update_ms_per_rank": per_rank_gu,
            # per iteration: splat, 3 FFT passes, the two gradient/update kernels,
            # statistics; 5 per spatial reorder (Morton keys, permutation, row fill,
            # staged-block build, group cost, every 50 iterations at n >= 4096; CUB
            # sort/scan kernels not counted); 3 per run restart (permute-in,
            # statistics, gains fill).
            "gpu_launches": per_iter * args.steps + (5 * (args.steps // 50) if n >= 4096 else 0)
                            + 3 * ((args.steps - 1) // (EE_ITER + N_ITER)),
            "clocks": clocks.summary(),
            "e2e": e2e,
            "full_run": full_run,
            "cpu_baseline": cpu,
        }
        if ref_gpu is not None:
            line["reference_cuda"] = ref_gpu
        if umap is not None:
            line["umap"] = umap
        print(json.dumps(line), flush=True)
    return 0


def umap_inputs(workload: str, device, producer: str = "b200"):
    from fastembedr_b200 import synthetic as S

    w = WORKLOADS[workload]
    spec = S.CONFIGS[w["spec"]]
    t0 = time.time()
    x, _ = S.gaussian_mixture(spec)
    idx, dist = S.exact_knn(x, w["k"], device=device, producer=producer)
    log(f"[bench] {workload}: n={spec.n} k={w['k']} inputs in {time.time() - t0:.1f}s")
    return idx, dist, S.umap_random_init(spec.n, seed=0)


CPU_UMAP_SAMPLES = 4e7  # positive samples in the CPU sample: ~10-15 s of the reference loop on 16 threads


def cpu_sample_epochs(p, budget: float = CPU_UMAP_SAMPLES, lo: int = 3, hi: int = 100) -> int:
    """The most epochs (lo..hi) whose positive samples, sum of floor((E-1)/p),
    stay within `budget`: a CPU sample of bounded length that still runs past
    the first epochs (an edge of period p first fires at epoch p)."""
    stride = max(1, p.size // 1_000_000)  # sizing only: an every-stride-th edge estimate
    sub = p[::stride]

    def pos(e):
        return int(np.floor(np.float32(e - 1) / sub).astype(np.int64).sum()) * stride

    if pos(lo) > budget:
        return lo
    while lo < hi:  # largest e with pos(e) <= budget
        mid = (lo + hi + 1) // 2
        if pos(mid) <= budget:
            lo = mid
        else:
            hi = mid - 1
    return lo


def cpu_baseline_umap(graph, init, epochs: int = 0):
    """The reference's own CPU COO optimizer (fast_knn_umap_coo_replay_cpp) on
    the same edge list, epochs 0 .. epochs-1 of a schedule, all host threads;
    by default as many epochs (3-100) as keep the sample near
    CPU_UMAP_SAMPLES positive samples."""
    import oracle as O

    threads = os.cpu_count() or 1
    h, t, p = graph["heads"], graph["tails"], graph["epochs_per_sample"].astype(np.float32)
    if epochs <= 0:
        epochs = cpu_sample_epochs(p)
    pos = int(np.floor(np.float32(epochs - 1) / p).astype(np.int64).sum())
    if O.ref_available():
        t0 = time.time()
        O.ref_umap_coo_replay(h, t, (1.0 / p).astype(np.float32), p, init, epochs, min_dist=UMAP_MIN_DIST,
                              negative_sample_rate=UMAP_NSR, learning_rate=UMAP_LR, threads=threads)
        secs, kind, cores = time.time() - t0, "reference", threads
    else:
        t0 = time.time()
        y = init.copy()
        for e in range(epochs):
            y = O.umap_epoch_delta(h, t, p, y, e, epochs)
        secs, kind, cores = time.time() - t0, "port", 1
    out = {"value": pos / secs, "unit": "edge_updates/s", "cores": cores, "kind": kind,
           "flags": "-O2 (R's default package build)" if kind == "reference" else "-O2",
           "sample": f"epochs 0-{epochs - 1} of the full edge list ({h.size} edges, {pos} positive samples), "
                     f"{cores} threads"}
    if kind == "reference" and O.ref_available("O3"):
        t0 = time.time()
        O.ref_umap_coo_replay(h, t, (1.0 / p).astype(np.float32), p, init, epochs, min_dist=UMAP_MIN_DIST,
                              negative_sample_rate=UMAP_NSR, learning_rate=UMAP_LR, threads=threads, variant="O3")
        s3 = time.time() - t0
        out["O3"] = {"value": pos / s3, "seconds": s3, "flags": "-O3 -march=x86-64-v3"}
    return out


def umap_measure(workload: str, steps: int, warmup: int, skip_e2e: bool, skip_cpu: bool, ref_cuda: bool):
    """A step is one UMAP epoch over the whole edge list; the metric counts
    positive edge samples applied per second (negative samples alongside).
    Returns the JSON line (rank 0; None on other ranks)."""
    import torch
    import torch.distributed as tdist

    from fastembedr_b200 import _lib, api

    rank, world, local = dist_env()
    w = WORKLOADS[workload]
    n_epochs = w["n_epochs"]
    if world == 1 or rank == 0:
        idx, dist, init = umap_inputs(workload, f"cuda:{local}")
    if world > 1:
        # Rank 0's inputs on every rank.
        from fastembedr_b200 import synthetic as S

        nn = S.CONFIGS[w["spec"]].n
        t = ([torch.from_numpy(idx).cuda(), torch.from_numpy(dist).cuda(), torch.from_numpy(init).cuda()]
             if rank == 0 else
             [torch.empty((nn, w["k"]), dtype=torch.int32, device="cuda"),
              torch.empty((nn, w["k"]), dtype=torch.float32, device="cuda"),
              torch.empty((nn, 2), dtype=torch.float32, device="cuda")])
        for x in t:
            tdist.broadcast(x, 0)
        idx, dist, init = (x.cpu().numpy() for x in t)
    n, k = idx.shape
    a, b = api.find_ab_params(1.0, UMAP_MIN_DIST)
    d_idx, d_dist = torch.from_numpy(idx).cuda(), torch.from_numpy(dist).cuda()
    t0 = time.time()
    sess = api.UmapSession.from_knn(d_idx, d_dist)
    if world > 1:
        # Rank r owns the r-th block of vertices; layout all-gathered per epoch.
        sess.shard_over()
    info = sess.info()
    log(f"[bench] umap: n={n} edges={info['n_edges']} (set-up {time.time() - t0:.2f}s)")
    del d_idx, d_dist
    init_dev = torch.from_numpy(init).cuda()
    stream = torch.cuda.ExternalStream(sess.stream)

    def spans(e0, count):
        """(cyc_begin, cyc_end) pieces of epochs e0 .. e0+count of back-to-back runs of the schedule."""
        e = e0
        while e < e0 + count:
            cyc = e % n_epochs
            step = min(n_epochs - cyc, e0 + count - e)
            yield cyc, cyc + step
            e += step

    def run(e0, count):
        for c0, c1 in spans(e0, count):
            if c0 == 0:
                sess.set_layout(init_dev)  # a new run of the schedule starts from the init
            sess.run(c0, c1, n_epochs, UMAP_NSR, UMAP_LR, UMAP_MIN_DIST, seed=42, optimizer_mode=0)

    run(0, warmup)
    torch.cuda.synchronize()
    if world > 1:
        tdist.barrier()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record(stream)
        run(0, steps)
        stop.record(stream)
        torch.cuda.synchronize()
    elapsed_ms = start.elapsed_time(stop)
    if world > 1:
        tt = torch.tensor([elapsed_ms], device="cuda")
        tdist.all_reduce(tt, op=tdist.ReduceOp.MAX)
        elapsed_ms = float(tt.item())
    pos = neg = 0
    for c0, c1 in spans(0, steps):
        p_, n_ = sess.count_samples(c0, c1, UMAP_NSR)
        pos, neg = pos + p_, neg + n_
    value = pos / (elapsed_ms / 1000.0)

    # Device time per epoch of single-epoch launches (epoch kernel + sanitize);
    # algorithmic bytes 12 E + 16 N (head, tail, period per edge; layout read + write).
    sess.set_layout(init_dev)
    probe = list(range(1, min(n_epochs, 41)))
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record(stream)
    for e in probe:
        sess.run(e, e + 1, n_epochs, UMAP_NSR, UMAP_LR, UMAP_MIN_DIST, seed=42, optimizer_mode=0)
    ev[1].record(stream)
    torch.cuda.synchronize()
    epoch_s = ev[0].elapsed_time(ev[1]) / 1000.0 / len(probe)
    alg_bytes = 12 * info["n_edges"] + 16 * n
    hbm, peak_kind = peaks()
    achieved = alg_bytes / epoch_s / 1e9

    graph = sess.graph()
    sess_total_pos, _ = sess.count_samples(0, n_epochs, UMAP_NSR)
    e2e = None
    if not skip_e2e and world == 1:
        # Pageable host arrays, as the reference's R wrapper passes them.
        idx_cm = np.ascontiguousarray(idx.T)
        dist_cm = np.ascontiguousarray(dist.T)
        out_h = np.empty((n, 2), np.float32)
        import ctypes

        L = _lib.load()
        sni = api.umap_config(n, k)["spectral_n_iter"]

        def call():
            rc = L.fastembedr_cuda_umap_from_knn_spectral_float(
                ctypes.c_void_p(idx_cm.ctypes.data), ctypes.c_void_p(dist_cm.ctypes.data), n, k, n_epochs,
                UMAP_NSR, UMAP_LR, a, b, 1.0, sni, 42, 0, 0,
                ctypes.cast(out_h.ctypes.data, ctypes.POINTER(ctypes.c_float)))
            _lib.check(rc, "fastembedr_cuda_umap_from_knn_spectral_float")

        e2e_s = median_call_seconds(call)
        total_pos, _ = sess.count_samples(0, n_epochs, UMAP_NSR)
        e2e = {"value": total_pos / e2e_s, "unit": "edge_updates/s",
               "h2d_bytes_per_step": int(idx_cm.nbytes + dist_cm.nbytes),
               "d2h_bytes_per_step": int(out_h.nbytes), "seconds_per_call": e2e_s,
               "host_buffers": "pageable (numpy), as the reference's R wrapper passes them",
               "timing": "median of 3 calls after a warm one",
               "call": f"fastembedr_cuda_umap_from_knn_spectral_float ({n_epochs} epochs, host KNN: graph, "
                       f"diffusion start, epochs)"}
    sess.close()
    cpu = ref_gpu = None
    if rank == 0 and world == 1 and not skip_cpu:
        cpu = cpu_baseline_umap(graph, init)
        if ref_cuda:
            ref_gpu = reference_cuda_umap(idx, dist, n_epochs, graph_edges=info["n_edges"],
                                          units=int(sess_total_pos))
    if world > 1:
        tdist.barrier()
        if rank != 0:
            return None
    line = {
        "metric": "umap_edge_updates_per_second", "value": value, "unit": "edge_updates/s",
        "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": elapsed_ms / steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": workload, "n": int(n), "k": int(k), "n_edges": int(info["n_edges"]),
                   "n_epochs": n_epochs, "negative_sample_rate": UMAP_NSR, "min_dist": UMAP_MIN_DIST,
                   "optimizer": "Hogwild per sample (device-KNN path)", "init": "U(-10, 10)",
                   "parallelism": (f"vertices sharded over {world} GPUs (per-epoch NCCL all-gather of the "
                                   f"layout)" if world > 1 else "single"),
                   "l2": l2_note(12 * info["n_edges"], "the edge list")},
        "negative_samples_per_second": neg / (elapsed_ms / 1000.0),
        "epochs_per_second": steps / (elapsed_ms / 1000.0),
        "edges_scanned_per_second": info["n_edges"] * steps / (elapsed_ms / 1000.0),
        "roofline": {"kernel": "umap_epoch_kernel over the epoch's firing edges (+ their CUB select and the "
                               "sanitize)", "bound": "hbm", "achieved": achieved,
                     "peak": hbm, "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / hbm,
                     "algorithmic_bytes_per_launch": alg_bytes, "avg_launch_ms": epoch_s * 1000.0,
                     "traffic": profile_traffic("umap_epoch_kernel", workload)},
        "gpu_launches": 2 * steps,  # epoch kernel + sanitize per epoch (the CUB select's kernels are CUB's)
        "clocks": clocks.summary(), "e2e": e2e, "cpu_baseline": cpu,
    }
    if ref_gpu is not None:
        line["reference_cuda"] = ref_gpu
    return line


def bench_umap(args):
    line = umap_measure(args.workload, args.steps, args.warmup, args.skip_e2e, args.skip_cpu,
                        ref_cuda=not args.skip_reference_cuda)
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1500)
    ap.add_argument("--warmup", type=int, default=30)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="tsne_1m")
    ap.add_argument("--cpu-iters", type=int, default=5, help="iterations per chunk of the CPU sample")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="loop time of the CPU sample")
    ap.add_argument("--skip-e2e", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-umap", action="store_true", help="leave the UMAP block out of the t-SNE line")
    ap.add_argument("--skip-reference-cuda", action="store_true",
                    help="leave out the reference CUDA backend's time (reference_cuda)")
    ap.add_argument("--reference-backend", choices=["cpu", "cuda"], default="cpu",
                    help="with --impl reference: the reference's CPU loop (default) or its own CUDA backend")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    umap = WORKLOADS[args.workload].get("kind") == "umap"
    if args.impl == "reference" and args.reference_backend == "cuda":
        return bench_reference_cuda(args)
    if args.impl == "reference":
        return bench_reference_umap(args) if umap else bench_reference(args)
    import torch
    import torch.distributed as tdist

    _, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        tdist.init_process_group("nccl", init_method="env://", timeout=datetime.timedelta(seconds=300),
                                 device_id=torch.device("cuda", local))
    try:
        rc = bench_umap(args) if umap else bench_ours(args)
    except BaseException:
        if world == 1:
            raise
        # A failure on one rank: report it now and leave without further
        # collectives (a barrier here would wait for ranks that are still in
        # the bench's own collectives); the others end at the process-group
        # timeout.
        import traceback

        traceback.print_exc()
        sys.stderr.flush()
        os._exit(1)
    if world > 1:
        tdist.barrier()
        tdist.destroy_process_group()
    return rc


if __name__ == "__main__":
    sys.exit(main())
