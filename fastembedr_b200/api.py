"""Host-side mirror of the reference interface for the optimizer path.

The reference reaches its CUDA optimizer from R: ``opentsne_knn(knn,
backend = "cuda")`` and ``umap_knn(knn, backend = "cuda")`` resolve their
parameters (R/tsne_affinity_dispatch.R, R/fast_knn_umap.R), then the C++
wrapper (src/embedding_cuda_impl.cpp) converts matrices and calls the C ABI.
R is not part of this build, so this module plays the wrapper's role for
Python callers and tests: the same parameter policies, the same C-ABI calls,
the same provenance strings, errors raised as exceptions.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass, field
from typing import Any, Dict, Optional, Tuple

import numpy as np

from . import _lib
from ._lib import CudaBackendError, check

# Provenance labels returned by the reference wrapper (src/embedding_cuda_impl.cpp:2194-2217),
# asserted by the reference tests (tests/testthat/test-tsne.R:243-244).
TSNE_OPTIMIZER_LABEL = "opentsne_fitsne_fft_grid_native_cuda"
TSNE_REPULSION_LABEL = "fft_grid_cuda_cufft"
UMAP_UPDATE_RULE_LABEL = "native_cuda_atomic_coo_umap_schedule"


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int32)


def _ptr(a: np.ndarray, ctype):
    return a.ctypes.data_as(ctypes.POINTER(ctype))


def cuda_available() -> bool:
    return bool(_lib.load().fastembedr_cuda_available())


def version() -> str:
    return _lib.load().fe_b200_version().decode()


def release_memory() -> None:
    """Returns the device memory the library keeps between calls (a pool per
    GPU, up to FASTEMBEDR_B200_RETAIN_MB) to the driver (fe_b200_release_memory)."""
    check(_lib.load().fe_b200_release_memory(), "fe_b200_release_memory")


# ------------------------------------------------------------------ parameter policy


def tsne_auto_parameters(n: int, k: int, perplexity: Optional[float] = None) -> Dict[str, Any]:
    """Restates tsne_auto_parameters_cpp (src/tsne_neighbors.cpp:1573-1618)."""
    if n < 2:
        raise ValueError("`n` must be at least 2.")
    if k < 1:
        raise ValueError("`k` must be positive.")
    missing = perplexity is None or not math.isfinite(perplexity) or perplexity <= 0.0
    max_n = max(1, (n - 1) // 3)
    max_k = max(1, k // 3)
    resolved = float(min(30, min(max_n, max_k))) if missing else float(perplexity)
    max_resolved = min(max_n, max_k) if missing else max_n
    resolved = max(1.0, min(resolved, float(max_resolved)))
    ee = 12.0
    return {
        "perplexity": resolved,
        "n_neighbors": max(1, min(n - 1, int(math.ceil(resolved)))),
        "early_exaggeration": ee,
        "exaggeration": 1.0,
        "learning_rate": float(n) / ee,
        "early_exaggeration_iter": 250,
        "n_iter": 500,
    }


def find_ab_params(spread: float = 1.0, min_dist: float = 0.1) -> Tuple[float, float]:
    """UMAP curve parameters a, b for (spread, min_dist).

    Restates find_ab_params (src/fast_knn_umap.cpp:428-488, used by the CUDA
    wrapper at src/embedding_cuda_impl.cpp:478-532): tabulated values for the
    common settings, otherwise a coarse grid search refined by 80 gradient steps.
    """
    table = {(1.0, 0.01): (1.895605865596314, 0.8006377738365004),
             (1.0, 0.1): (1.5769434601962196, 0.8950608781227859),
             (1.0, 0.5): (0.5830300199018228, 1.3341669931033755)}
    for (s, m), ab in table.items():
        if abs(spread - s) < 1e-12 and abs(min_dist - m) < 1e-12:
            return ab
    xs = (spread * 3.0) * np.arange(300, dtype=np.float64) / 299.0
    ys = np.where(xs < min_dist, 1.0, np.exp(-(xs - min_dist) / spread))
    best = (1.5769434601962196, 0.8950608781227859)
    best_loss = math.inf
    loga = -4.0
    while loga <= 4.0001:
        b = 0.25
        while b <= 2.0001:
            a = math.exp(loga)
            loss = 0.0
            for x, y in zip(xs, ys):
                e = 1.0 / (1.0 + a * math.pow(x, 2.0 * b)) - y
                loss += e * e
            if loss < best_loss:
                best_loss, best = loss, (a, b)
            b += 0.05
        loga += 0.2
    a, b = best
    for _ in range(80):
        ga = gb = 0.0
        for x0, y in zip(xs, ys):
            x = max(x0, 1e-6)
            x2b = math.pow(x, 2.0 * b)
            den = 1.0 + a * x2b
            e = 1.0 / den - y
            ga += e * (-x2b / (den * den))
            gb += e * (-(a * x2b * 2.0 * math.log(x)) / (den * den))
        a = max(1e-4, a - 0.01 * ga)
        b = max(0.1, b - 0.01 * gb)
    return a, b


def resolve_index_offset(indices: np.ndarray) -> int:
    """1 when every index lies in [1, n] (R's 1-based KNN), else 0
    (src/embedding_cuda_impl.cpp:886-895)."""
    n = indices.shape[0]
    return 1 if indices.size and indices.min() >= 1 and indices.max() <= n else 0


def column_major(a: np.ndarray, dtype) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=dtype).T)


# ------------------------------------------------------------------ openTSNE


@dataclass
class EmbeddingResult:
    Y: np.ndarray
    config: Dict[str, Any] = field(default_factory=dict)


def opentsne_knn(indices, distances, n_components: int = 2, perplexity: Optional[float] = 30.0,
                 early_exaggeration_iter: int = 250, n_iter: int = 500,
                 early_exaggeration: float = 12.0, exaggeration: float = 1.0,
                 learning_rate="auto", initial_momentum: float = 0.8, final_momentum: float = 0.8,
                 min_gain: float = 0.01, max_step_norm="auto", init: Optional[np.ndarray] = None,
                 seed: int = 42, index_offset: Optional[int] = None) -> EmbeddingResult:
    """openTSNE-style t-SNE from KNN on the B200 backend.

    ``indices``/``distances`` are (n, k) host arrays (0- or 1-based indices,
    self excluded) or CUDA tensors (then the device-KNN entry point is used and
    nothing is copied).  Defaults follow R/fast_knn_tsne.R:39-60 and
    R/tsne_affinity_dispatch.R (momentum 0.8/0.8, min_gain 0.01,
    max_step_norm "auto" = 5, learning_rate "auto" = n / exaggeration).
    """
    on_device = hasattr(indices, "is_cuda") and indices.is_cuda
    n, k = (int(indices.shape[0]), int(indices.shape[1]))
    if perplexity is None:
        perplexity = tsne_auto_parameters(n, k)["perplexity"]
    lr_auto = isinstance(learning_rate, str)
    lr = 0.0 if lr_auto else float(learning_rate)
    msn = 5.0 if isinstance(max_step_norm, str) else float(max_step_norm)
    out = np.zeros((n, 2), np.float32)
    init_arr = None if init is None else _f32(init)
    L = _lib.load()
    if on_device:
        import torch

        idx_cm = indices.to(torch.int32).t().contiguous()
        dist_cm = distances.to(torch.float32).t().contiguous()
        off = index_offset if index_offset is not None else int(
            bool((idx_cm.min() >= 1).item() and (idx_cm.max() <= n).item()))
        rc = L.fastembedr_cuda_opentsne_fft_from_device_knn_float(
            ctypes.c_void_p(idx_cm.data_ptr()), ctypes.c_void_p(dist_cm.data_ptr()),
            None if init_arr is None else _ptr(init_arr, ctypes.c_float), int(init_arr is not None),
            n, k, n_components, perplexity, early_exaggeration_iter, n_iter, early_exaggeration,
            exaggeration, lr, int(lr_auto), initial_momentum, final_momentum, min_gain, msn,
            seed & 0xFFFFFFFF, off, _ptr(out, ctypes.c_float))
        entry = "fastembedr_cuda_opentsne_fft_from_device_knn_float"
    else:
        idx = np.asarray(indices)
        off = index_offset if index_offset is not None else resolve_index_offset(idx)
        idx_cm = column_major(idx, np.int32)
        dist_cm = column_major(distances, np.float32)
        rc = L.fastembedr_cuda_opentsne_fft_from_knn_float(
            ctypes.c_void_p(idx_cm.ctypes.data), ctypes.c_void_p(dist_cm.ctypes.data),
            None if init_arr is None else _ptr(init_arr, ctypes.c_float), int(init_arr is not None),
            n, k, n_components, perplexity, early_exaggeration_iter, n_iter, early_exaggeration,
            exaggeration, lr, int(lr_auto), initial_momentum, final_momentum, min_gain, msn,
            seed & 0xFFFFFFFF, off, _ptr(out, ctypes.c_float))
        entry = "fastembedr_cuda_opentsne_fft_from_knn_float"
    if rc != 0:
        raise CudaBackendError("CUDA openTSNE FFT-grid failed: " + _lib.last_error())
    return EmbeddingResult(out, {
        "optimizer": TSNE_OPTIMIZER_LABEL, "repulsion": TSNE_REPULSION_LABEL, "entry_point": entry,
        "perplexity": perplexity, "learning_rate": "auto" if lr_auto else lr,
        "max_step_norm": msn, "backend": "cuda", "device": "B200 (sm_100a)",
    })


def knn_exact(data, k: int, exclude_self: bool = True, device_output: bool = False):
    """Exact Euclidean KNN on the device (fe_b200_knn_exact): the GPU-KNN
    producer.  `data` is (n, p), a numpy array or a CUDA tensor (float32 or
    float64).  Returns 0-based (n, k) int32 indices and float32 distances,
    ascending -- numpy arrays, or with device_output the column-major CUDA
    tensors (k, n) the device-KNN entry points take (1-based)."""
    import torch

    if isinstance(data, torch.Tensor) and data.is_cuda:
        dt = data.to(torch.float64 if data.dtype == torch.float64 else torch.float32)
        cm = dt.t().contiguous()
        n, p = data.shape
        ptr, on_dev, dbl = cm.data_ptr(), 1, int(dt.dtype == torch.float64)
        keep = cm
    else:
        arr = np.asarray(data)
        dbl = int(arr.dtype == np.float64)
        arr = arr.astype(np.float64 if dbl else np.float32, copy=False)
        keep = np.ascontiguousarray(arr.T)
        n, p = arr.shape
        ptr, on_dev = keep.ctypes.data, 0
    d_idx = torch.empty((k, n), dtype=torch.int32, device="cuda")
    d_dist = torch.empty((k, n), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    rc = _lib.load().fe_b200_knn_exact(ctypes.c_void_p(ptr), dbl, on_dev, n, p, k, int(exclude_self),
                                       ctypes.c_void_p(d_idx.data_ptr()), ctypes.c_void_p(d_dist.data_ptr()))
    del keep
    check(rc, "fe_b200_knn_exact")
    if device_output:
        return d_idx, d_dist
    # (n, k) row-major host arrays, like every other KNN in this package
    return (np.ascontiguousarray(d_idx.t().cpu().numpy() - 1, dtype=np.int32),
            np.ascontiguousarray(d_dist.t().cpu().numpy()))


def landmark_tsne_transform(indices, distances, reference_data, query_data, reference_layout,
                            perplexity: float = 30.0, n_iter: int = 250, early_exaggeration_iter: int = 50,
                            learning_rate: float = 0.1, early_exaggeration: float = 4.0,
                            exaggeration: float = 1.5, initial_momentum: float = 0.8,
                            final_momentum: float = 0.8, max_grad_norm: float = 0.25,
                            max_step_norm: float = float("inf"), n_negatives: Optional[int] = None,
                            exact_repulsion_threshold: int = 4096, seed: int = 1009, affine_neighbors: int = 12,
                            affine_ridge: float = 1e-3, max_extrapolation: float = 2.5,
                            index_offset: int = 0) -> np.ndarray:
    """Places query points in a fixed reference layout (the openTSNE transform
    behind landmark_tsne_transform_cuda_gpu_cpp, src/embedding_cuda_impl.cpp:2486-2580,
    and fastembedr_cuda_landmark_tsne_from_device_knn): `indices` / `distances`
    are the queries' KNN into the reference, (n_query, k), on the device (torch
    CUDA tensors) or on the host (copied to the device here); the data and the
    reference layout are (n, d) host arrays.  Defaults follow the R wrapper
    (R/landmark_model.R:442-477): n_negatives = n_reference up to the exact
    threshold, else min(256, n_reference)."""
    import torch

    n_ref, dim = np.asarray(reference_data).shape
    n_q, k = tuple(indices.shape)
    if n_negatives is None:
        n_negatives = n_ref if n_ref <= exact_repulsion_threshold else min(256, n_ref)
    # column-major (R) device KNN
    ti = torch.as_tensor(indices).to(device="cuda", dtype=torch.int32).t().contiguous()
    td = torch.as_tensor(distances).to(device="cuda", dtype=torch.float32).t().contiguous()
    rd = np.ascontiguousarray(np.asarray(reference_data, np.float32).T).reshape(-1)
    qd = np.ascontiguousarray(np.asarray(query_data, np.float32).T).reshape(-1)
    rl = np.ascontiguousarray(np.asarray(reference_layout, np.float32).T).reshape(-1)
    out = np.zeros((n_q, 2), np.float32)
    torch.cuda.synchronize()
    rc = _lib.load().fastembedr_cuda_landmark_tsne_from_device_knn(
        ctypes.c_void_p(ti.data_ptr()), ctypes.c_void_p(td.data_ptr()), index_offset, _ptr(rd, ctypes.c_float),
        _ptr(qd, ctypes.c_float), _ptr(rl, ctypes.c_float), n_ref, n_q, dim, k, perplexity, n_iter,
        early_exaggeration_iter, learning_rate, early_exaggeration, exaggeration, initial_momentum,
        final_momentum, max_grad_norm, max_step_norm, n_negatives, exact_repulsion_threshold,
        seed & 0xFFFFFFFF, affine_neighbors, affine_ridge, max_extrapolation, _ptr(out, ctypes.c_float))
    check(rc, "fastembedr_cuda_landmark_tsne_from_device_knn")
    return out


class TsneSession:
    """Device-resident t-SNE state (P, layout, gains, update) across calls."""

    def __init__(self, handle: int, n: int):
        self._h = ctypes.c_void_p(handle)
        self.n = n

    @classmethod
    def from_knn(cls, indices, distances, perplexity: float = 30.0, init=None, seed: int = 42,
                 grid_size: int = 0, index_offset: Optional[int] = None) -> "TsneSession":
        L = _lib.load()
        h = ctypes.c_void_p()
        on_device = hasattr(indices, "is_cuda") and indices.is_cuda
        n, k = int(indices.shape[0]), int(indices.shape[1])
        init_arr = None if init is None else _f32(init)
        keep = []
        if on_device:
            import torch

            idx_cm = indices.to(torch.int32).t().contiguous()
            dist_cm = distances.to(torch.float32).t().contiguous()
            keep = [idx_cm, dist_cm]
            off = 0 if index_offset is None else index_offset
            ip, dp = ctypes.c_void_p(idx_cm.data_ptr()), ctypes.c_void_p(dist_cm.data_ptr())
            init_dev = None
            if init_arr is not None:
                init_dev = torch.from_numpy(init_arr).cuda()
                keep.append(init_dev)
            init_p = None if init_dev is None else ctypes.cast(init_dev.data_ptr(), ctypes.POINTER(ctypes.c_float))
        else:
            idx = np.asarray(indices)
            off = index_offset if index_offset is not None else resolve_index_offset(idx)
            idx_cm = column_major(idx, np.int32)
            dist_cm = column_major(distances, np.float32)
            keep = [idx_cm, dist_cm]
            ip, dp = ctypes.c_void_p(idx_cm.ctypes.data), ctypes.c_void_p(dist_cm.ctypes.data)
            init_p = None if init_arr is None else _ptr(init_arr, ctypes.c_float)
        check(L.fe_b200_tsne_create(ip, dp, n, k, off, perplexity, init_p, seed & 0xFFFFFFFF,
                                    grid_size, int(on_device), ctypes.byref(h)), "fe_b200_tsne_create")
        del keep
        return cls(h.value, n)

    @classmethod
    def from_csr(cls, row_ptr, col, val, init, grid_size: int = 0) -> "TsneSession":
        L = _lib.load()
        rp, c, v, y = _i32(row_ptr), _i32(col), _f32(val), _f32(init)
        h = ctypes.c_void_p()
        check(L.fe_b200_tsne_create_csr(_ptr(rp, ctypes.c_int), _ptr(c, ctypes.c_int), _ptr(v, ctypes.c_float),
                                        y.shape[0], _ptr(y, ctypes.c_float), grid_size, ctypes.byref(h)),
              "fe_b200_tsne_create_csr")
        return cls(h.value, y.shape[0])

    def iterate(self, n_iter: int, exaggeration: float, momentum: float, learning_rate: float,
                min_gain: float = 0.01, max_step_norm: float = 5.0) -> None:
        check(_lib.load().fe_b200_tsne_iterate(self._h, n_iter, exaggeration, momentum, learning_rate,
                                               min_gain, max_step_norm), "fe_b200_tsne_iterate")

    def prepare(self, exaggeration: float, momentum: float, learning_rate: float, min_gain: float = 0.01,
                max_step_norm: float = 5.0) -> None:
        """Captures the iteration graphs for this parameter set ahead of iterate()."""
        check(_lib.load().fe_b200_tsne_prepare(self._h, exaggeration, momentum, learning_rate, min_gain,
                                               max_step_norm), "fe_b200_tsne_prepare")

    def run(self, early_exaggeration_iter=250, n_iter=500, early_exaggeration=12.0, exaggeration=1.0,
            learning_rate="auto", initial_momentum=0.8, final_momentum=0.8, min_gain=0.01,
            max_step_norm=5.0) -> np.ndarray:
        auto = isinstance(learning_rate, str)
        lr_e = float(np.float32(self.n / early_exaggeration)) if auto else learning_rate
        lr_n = float(np.float32(self.n / exaggeration)) if auto else learning_rate
        self.iterate(early_exaggeration_iter, early_exaggeration, initial_momentum, lr_e, min_gain, max_step_norm)
        self.iterate(n_iter, exaggeration, final_momentum, lr_n, min_gain, max_step_norm)
        return self.layout()

    def gradient(self, exaggeration: float) -> Tuple[np.ndarray, float]:
        g = np.zeros((self.n, 2), np.float32)
        z = ctypes.c_double(0.0)
        check(_lib.load().fe_b200_tsne_gradient(self._h, exaggeration, _ptr(g, ctypes.c_float),
                                                ctypes.byref(z)), "fe_b200_tsne_gradient")
        return g, z.value

    def layout(self) -> np.ndarray:
        y = np.zeros((self.n, 2), np.float32)
        check(_lib.load().fe_b200_tsne_get_layout(self._h, ctypes.c_void_p(y.ctypes.data), 0),
              "fe_b200_tsne_get_layout")
        return y

    def set_layout(self, y, reset_state: bool = True) -> None:
        """Sets the layout from a host array or a CUDA tensor of shape (n, 2)."""
        if hasattr(y, "is_cuda") and y.is_cuda:
            import torch

            y = y.to(torch.float32).contiguous()
            check(_lib.load().fe_b200_tsne_set_layout(self._h, ctypes.c_void_p(y.data_ptr()), 1,
                                                      int(reset_state)), "fe_b200_tsne_set_layout")
            return
        y = _f32(y)
        check(_lib.load().fe_b200_tsne_set_layout(self._h, ctypes.c_void_p(y.ctypes.data), 0,
                                                  int(reset_state)), "fe_b200_tsne_set_layout")

    def state(self) -> Tuple[np.ndarray, np.ndarray]:
        u = np.zeros((self.n, 2), np.float32)
        g = np.zeros((self.n, 2), np.float32)
        check(_lib.load().fe_b200_tsne_get_state(self._h, _ptr(u, ctypes.c_float), _ptr(g, ctypes.c_float)),
              "fe_b200_tsne_get_state")
        return u, g

    def set_state(self, update, gains) -> None:
        u, g = _f32(update), _f32(gains)
        check(_lib.load().fe_b200_tsne_set_state(self._h, _ptr(u, ctypes.c_float), _ptr(g, ctypes.c_float)),
              "fe_b200_tsne_set_state")

    def info(self) -> Dict[str, int]:
        n, g = ctypes.c_int(), ctypes.c_int()
        nnz, nnzp = ctypes.c_longlong(), ctypes.c_longlong()
        check(_lib.load().fe_b200_tsne_info(self._h, ctypes.byref(n), ctypes.byref(g), ctypes.byref(nnz),
                                            ctypes.byref(nnzp)), "fe_b200_tsne_info")
        return {"n": n.value, "grid": g.value, "nnz": nnz.value, "nnz_padded": nnzp.value}

    def set_interpolation(self, mode: str) -> None:
        """"bilinear" (the reference's grid, the default) or "lagrange"
        (FIt-SNE boxes with three Lagrange nodes per side)."""
        code = {"bilinear": 0, "lagrange": 1}[mode]
        check(_lib.load().fe_b200_tsne_set_interpolation(self._h, code), "fe_b200_tsne_set_interpolation")

    def staged_blocks(self) -> Tuple[int, int]:
        """(staged, total) 128-row blocks of this session's rows at the last
        spatial reorder; staged blocks gather y from shared memory."""
        st, tot = ctypes.c_int(), ctypes.c_int()
        check(_lib.load().fe_b200_tsne_staged_blocks(self._h, ctypes.byref(st), ctypes.byref(tot)),
              "fe_b200_tsne_staged_blocks")
        return st.value, tot.value

    def p(self):
        inf = self.info()
        rp = np.zeros(inf["n"] + 1, np.int32)
        c = np.zeros(inf["nnz"], np.int32)
        v = np.zeros(inf["nnz"], np.float32)
        check(_lib.load().fe_b200_tsne_get_p(self._h, _ptr(rp, ctypes.c_int), _ptr(c, ctypes.c_int),
                                             _ptr(v, ctypes.c_float)), "fe_b200_tsne_get_p")
        nnz = int(rp[-1])
        return rp, c[:nnz].copy(), v[:nnz].copy()

    @property
    def stream(self) -> int:
        return int(_lib.load().fe_b200_tsne_stream(self._h) or 0)

    def profile(self, enable: bool) -> None:
        check(_lib.load().fe_b200_tsne_profile(self._h, int(enable)), "fe_b200_tsne_profile")

    def kernel_times(self) -> Dict[str, Tuple[float, int]]:
        """Per-kind CUDA-event totals (ms, launches) since profiling was enabled;
        the collective kinds appear only for sharded sessions."""
        kinds = 9
        ms = np.zeros(kinds, np.float64)
        cnt = np.zeros(kinds, np.int64)
        L = _lib.load()
        check(L.fe_b200_tsne_kernel_times(self._h, _ptr(ms, ctypes.c_double), _ptr(cnt, ctypes.c_longlong),
                                          kinds), "fe_b200_tsne_kernel_times")
        return {L.fe_b200_tsne_kernel_name(i).decode(): (float(ms[i]), int(cnt[i]))
                for i in range(kinds) if i < 5 or cnt[i] > 0}

    def shard(self, unique_id: bytes, nranks: int, rank: int) -> None:
        """Makes this session rank `rank` of an nranks-way sharded run (one
        process per GPU).  Every rank must hold an identical session and make
        the same calls from then on; see fe_b200_tsne_shard."""
        uid = (ctypes.c_ubyte * len(unique_id)).from_buffer_copy(unique_id)
        check(_lib.load().fe_b200_tsne_shard(self._h, uid, len(unique_id), nranks, rank), "fe_b200_tsne_shard")

    def shard_comm(self, comm: "NcclComm") -> None:
        """Shards this session on a communicator lent by the caller (kept open)."""
        check(_lib.load().fe_b200_tsne_shard_comm(self._h, comm.handle), "fe_b200_tsne_shard_comm")

    def shard_over(self, group=None) -> None:
        """Shards over a torch.distributed process group (any backend): rank 0
        makes the communicator id and the group broadcasts it."""
        import torch.distributed as dist

        box = [nccl_unique_id() if dist.get_rank(group) == 0 else None]
        dist.broadcast_object_list(box, src=dist.get_global_rank(group, 0) if group is not None else 0,
                                   group=group)
        self.shard(box[0], dist.get_world_size(group), dist.get_rank(group))

    def close(self) -> None:
        if self._h is not None and self._h.value:
            _lib.load().fe_b200_tsne_destroy(self._h)
        self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def nccl_unique_id() -> bytes:
    """A new NCCL communicator id (128 bytes) for TsneSession.shard."""
    buf = (ctypes.c_ubyte * 128)()
    check(_lib.load().fe_b200_nccl_unique_id(buf, 128), "fe_b200_nccl_unique_id")
    return bytes(buf)


class NcclComm:
    """An NCCL communicator made once and lent to sessions in turn
    (fe_b200_comm_create): repeated sharded runs then skip NCCL's set-up.
    Sessions sharing it must not run concurrently and must close first."""

    def __init__(self, unique_id: bytes, nranks: int, rank: int):
        uid = (ctypes.c_ubyte * len(unique_id)).from_buffer_copy(unique_id)
        h = ctypes.c_void_p()
        check(_lib.load().fe_b200_comm_create(uid, len(unique_id), nranks, rank, ctypes.byref(h)),
              "fe_b200_comm_create")
        self._h = h
        self.nranks, self.rank = nranks, rank

    @classmethod
    def over(cls, group=None) -> "NcclComm":
        """Joins every rank of a torch.distributed group (any backend)."""
        import torch.distributed as dist

        box = [nccl_unique_id() if dist.get_rank(group) == 0 else None]
        dist.broadcast_object_list(box, src=dist.get_global_rank(group, 0) if group is not None else 0,
                                   group=group)
        return cls(box[0], dist.get_world_size(group), dist.get_rank(group))

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    def close(self) -> None:
        if self._h is not None and self._h.value:
            _lib.load().fe_b200_comm_destroy(self._h)
        self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def shard_rows(n: int, nranks: int, rank: int) -> Tuple[int, int]:
    """Internal rows [begin, end) that `rank` owns in an nranks-way sharded
    t-SNE session: blocks of ceil(n / nranks) rows rounded up to whole warps
    (32 rows), the last block short (mirrors session_shard)."""
    per = -(-n // nranks)
    per = (per + 31) & ~31
    begin = min(n, rank * per)
    return begin, min(n, begin + per)


def umap_shard_vertices(n: int, nranks: int, rank: int) -> Tuple[int, int]:
    """Vertices [begin, end) that `rank` owns in an nranks-way sharded UMAP
    session: blocks of ceil(n / nranks), the last one short (mirrors
    fe_b200_umap_shard)."""
    per = -(-n // nranks)
    begin = min(n, rank * per)
    return begin, min(n, begin + per)


# ------------------------------------------------------------------ UMAP


def umap_config(n: int, k: int) -> Dict[str, Any]:
    """Size rules of the reference's UMAP defaults (fast_knn_umap_config,
    R/fast_knn_umap.R:1191-1224)."""
    if n >= 10000:
        return {"n_epochs": 200, "min_dist": 0.01, "negative_sample_rate": 5,
                "spectral_n_iter": 30 if k <= 15 else 20, "learning_rate": 1.0, "repulsion_strength": 1.0}
    return {"n_epochs": 500, "min_dist": 0.01, "negative_sample_rate": 5,
            "spectral_n_iter": 60 if n >= 500 else 50, "learning_rate": 1.0, "repulsion_strength": 1.0}


def umap_knn(indices, distances, n_epochs: Optional[int] = None, negative_sample_rate: Optional[int] = None,
             learning_rate: Optional[float] = None, min_dist: Optional[float] = None,
             repulsion_strength: Optional[float] = None, spectral_n_iter: Optional[int] = None,
             seed: int = 42, optimizer_mode: int = 0, graph_mode: str = "fuzzy",
             index_offset: Optional[int] = None) -> EmbeddingResult:
    """UMAP from KNN on the B200 backend: device fuzzy graph, diffusion start and
    COO edge SGD in one call (the fused path of umap_knn(backend = "cuda"),
    src/embedding_cuda_impl.cpp:1566-1768).

    ``indices``/``distances`` are (n, k) host arrays (0- or 1-based, self
    excluded) or CUDA tensors (device-KNN entry point, nothing copied).
    ``graph_mode="binary"`` sets every graph weight to 1; the reference offers it
    on the device-KNN entry point only, so host inputs are moved to the device
    for it.  Unset parameters follow the reference's size rules (umap_config).
    """
    on_device = hasattr(indices, "is_cuda") and indices.is_cuda
    n, k = (int(indices.shape[0]), int(indices.shape[1]))
    cfg = umap_config(n, k)
    n_epochs = cfg["n_epochs"] if n_epochs is None else int(n_epochs)
    nsr = cfg["negative_sample_rate"] if negative_sample_rate is None else int(negative_sample_rate)
    lr = cfg["learning_rate"] if learning_rate is None else float(learning_rate)
    md = cfg["min_dist"] if min_dist is None else float(min_dist)
    rep = cfg["repulsion_strength"] if repulsion_strength is None else float(repulsion_strength)
    sni = cfg["spectral_n_iter"] if spectral_n_iter is None else int(spectral_n_iter)
    if graph_mode not in ("fuzzy", "binary"):
        raise ValueError("graph_mode must be 'fuzzy' or 'binary'")
    binary = graph_mode == "binary"
    a, b = find_ab_params(1.0, md)
    out = np.zeros((n, 2), np.float32)
    L = _lib.load()
    if binary and not on_device:
        import torch

        indices = torch.as_tensor(np.asarray(indices), dtype=torch.int32, device="cuda")
        distances = torch.as_tensor(np.asarray(distances), dtype=torch.float32, device="cuda")
        on_device = True
    if on_device:
        import torch

        idx_cm = indices.to(torch.int32).t().contiguous()
        dist_cm = distances.to(torch.float32).t().contiguous()
        off = index_offset if index_offset is not None else int(
            bool((idx_cm.min() >= 1).item() and (idx_cm.max() <= n).item()))
        rc = L.fastembedr_cuda_umap_from_device_knn_spectral_float(
            ctypes.c_void_p(idx_cm.data_ptr()), ctypes.c_void_p(dist_cm.data_ptr()), n, k, n_epochs, nsr, lr, a,
            b, rep, sni, seed & 0xFFFFFFFF, off, optimizer_mode, int(binary), _ptr(out, ctypes.c_float))
        entry = "fastembedr_cuda_umap_from_device_knn_spectral_float"
    else:
        idx = np.asarray(indices)
        off = index_offset if index_offset is not None else resolve_index_offset(idx)
        idx_cm = column_major(idx, np.int32)
        dist_cm = column_major(distances, np.float32)
        rc = L.fastembedr_cuda_umap_from_knn_spectral_float(
            ctypes.c_void_p(idx_cm.ctypes.data), ctypes.c_void_p(dist_cm.ctypes.data), n, k, n_epochs, nsr, lr,
            a, b, rep, sni, seed & 0xFFFFFFFF, off, optimizer_mode, _ptr(out, ctypes.c_float))
        entry = "fastembedr_cuda_umap_from_knn_spectral_float"
    if rc != 0:
        raise CudaBackendError("CUDA fused UMAP failed: " + _lib.last_error())
    return EmbeddingResult(out, {
        "entry_point": entry, "n_epochs": n_epochs, "negative_sample_rate": nsr, "learning_rate": lr,
        "min_dist": md, "a": a, "b": b, "spectral_n_iter": sni, "graph_mode": graph_mode,
        "optimizer_mode": optimizer_mode, "backend": "cuda", "device": "B200 (sm_100a)",
    })


class UmapSession:
    """The device-KNN UMAP path with its graph, edge list and layout resident
    on the device (fe_b200_umap_*): set-up once, then epoch ranges."""

    def __init__(self, handle: int, n: int):
        self._h = ctypes.c_void_p(handle)
        self.n = n

    @classmethod
    def from_knn(cls, indices, distances, index_offset: Optional[int] = None, graph_mode: str = "fuzzy",
                 spectral_n_iter: Optional[int] = None, seed: int = 42) -> "UmapSession":
        if graph_mode not in ("fuzzy", "binary"):
            raise ValueError("graph_mode must be 'fuzzy' or 'binary'")
        on_device = hasattr(indices, "is_cuda") and indices.is_cuda
        n, k = int(indices.shape[0]), int(indices.shape[1])
        sni = umap_config(n, k)["spectral_n_iter"] if spectral_n_iter is None else int(spectral_n_iter)
        h = ctypes.c_void_p()
        if on_device:
            import torch

            idx_cm = indices.to(torch.int32).t().contiguous()
            dist_cm = distances.to(torch.float32).t().contiguous()
            off = index_offset if index_offset is not None else int(
                bool((idx_cm.min() >= 1).item() and (idx_cm.max() <= n).item()))
            ip, dp = ctypes.c_void_p(idx_cm.data_ptr()), ctypes.c_void_p(dist_cm.data_ptr())
        else:
            idx = np.asarray(indices)
            off = index_offset if index_offset is not None else resolve_index_offset(idx)
            idx_cm = column_major(idx, np.int32)
            dist_cm = column_major(distances, np.float32)
            ip, dp = ctypes.c_void_p(idx_cm.ctypes.data), ctypes.c_void_p(dist_cm.ctypes.data)
        check(_lib.load().fe_b200_umap_create(ip, dp, n, k, off, int(on_device), int(graph_mode == "binary"), sni,
                                              seed & 0xFFFFFFFF, ctypes.byref(h)), "fe_b200_umap_create")
        return cls(h.value, n)

    def run(self, epoch_begin: int, epoch_end: int, n_epochs: int, negative_sample_rate: int = 5,
            learning_rate: float = 1.0, min_dist: float = 0.1, repulsion_strength: float = 1.0, seed: int = 42,
            optimizer_mode: int = 0) -> None:
        """Epochs [epoch_begin, epoch_end) of an n_epochs schedule (0: Hogwild per sample, 1: Jacobi)."""
        a, b = find_ab_params(1.0, min_dist)
        check(_lib.load().fe_b200_umap_run(self._h, epoch_begin, epoch_end, n_epochs, negative_sample_rate,
                                           learning_rate, a, b, repulsion_strength, seed & 0xFFFFFFFF,
                                           optimizer_mode), "fe_b200_umap_run")

    def count_samples(self, epoch_begin: int, epoch_end: int, negative_sample_rate: int = 5) -> Tuple[int, int]:
        """(positive, negative) edge samples that epochs [epoch_begin, epoch_end) apply."""
        pos, neg = ctypes.c_longlong(), ctypes.c_longlong()
        check(_lib.load().fe_b200_umap_count_samples(self._h, epoch_begin, epoch_end, negative_sample_rate,
                                                     ctypes.byref(pos), ctypes.byref(neg)),
              "fe_b200_umap_count_samples")
        return pos.value, neg.value

    def shard(self, unique_id: bytes, nranks: int, rank: int) -> None:
        """Makes this session rank `rank` of an nranks-way run (one process per
        GPU); see fe_b200_umap_shard."""
        uid = (ctypes.c_ubyte * len(unique_id)).from_buffer_copy(unique_id)
        check(_lib.load().fe_b200_umap_shard(self._h, uid, len(unique_id), nranks, rank), "fe_b200_umap_shard")

    def shard_comm(self, comm: "NcclComm") -> None:
        """Shards this session on a communicator lent by the caller (kept open)."""
        check(_lib.load().fe_b200_umap_shard_comm(self._h, comm.handle), "fe_b200_umap_shard_comm")

    def shard_over(self, group=None) -> None:
        """Shards over a torch.distributed process group (any backend)."""
        import torch.distributed as dist

        box = [nccl_unique_id() if dist.get_rank(group) == 0 else None]
        dist.broadcast_object_list(box, src=dist.get_global_rank(group, 0) if group is not None else 0,
                                   group=group)
        self.shard(box[0], dist.get_world_size(group), dist.get_rank(group))

    def layout(self) -> np.ndarray:
        y = np.zeros((self.n, 2), np.float32)
        check(_lib.load().fe_b200_umap_get_layout(self._h, ctypes.c_void_p(y.ctypes.data), 0),
              "fe_b200_umap_get_layout")
        return y

    def set_layout(self, y) -> None:
        if hasattr(y, "is_cuda") and y.is_cuda:
            import torch

            y = y.to(torch.float32).contiguous()
            check(_lib.load().fe_b200_umap_set_layout(self._h, ctypes.c_void_p(y.data_ptr()), 1),
                  "fe_b200_umap_set_layout")
            return
        y = _f32(y)
        check(_lib.load().fe_b200_umap_set_layout(self._h, ctypes.c_void_p(y.ctypes.data), 0),
              "fe_b200_umap_set_layout")

    def info(self) -> Dict[str, int]:
        n, e = ctypes.c_int(), ctypes.c_longlong()
        check(_lib.load().fe_b200_umap_info(self._h, ctypes.byref(n), ctypes.byref(e)), "fe_b200_umap_info")
        return {"n": n.value, "n_edges": e.value}

    def graph(self) -> Dict[str, np.ndarray]:
        e = self.info()["n_edges"]
        h, t, p = np.zeros(e, np.int32), np.zeros(e, np.int32), np.zeros(e, np.float32)
        check(_lib.load().fe_b200_umap_get_graph(self._h, ctypes.c_void_p(h.ctypes.data),
                                                 ctypes.c_void_p(t.ctypes.data), ctypes.c_void_p(p.ctypes.data)),
              "fe_b200_umap_get_graph")
        return {"heads": h, "tails": t, "epochs_per_sample": p}

    @property
    def stream(self) -> int:
        return int(_lib.load().fe_b200_umap_stream(self._h) or 0)

    def close(self) -> None:
        if self._h is not None and self._h.value:
            _lib.load().fe_b200_umap_destroy(self._h)
        self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def umap_graph_dump(indices, distances, index_offset: Optional[int] = None) -> Dict[str, Any]:
    """The device-KNN fuzzy graph as a rank-major COO list
    (fastembedr_cuda_umap_graph_dump_from_knn; umap_cuda_graph_dump_impl,
    src/embedding_cuda_impl.cpp:1838-1896)."""
    idx = np.asarray(indices)
    n, k = idx.shape
    off = index_offset if index_offset is not None else resolve_index_offset(idx)
    width = min(256, 2 * k)
    cap = n * width
    idx_cm = column_major(idx, np.int32)
    dist_cm = column_major(distances, np.float64)
    heads, tails = np.full(cap, -1, np.int32), np.full(cap, -1, np.int32)
    weights, eps = np.zeros(cap, np.float32), np.zeros(cap, np.float32)
    w_out, c_out = ctypes.c_int(0), ctypes.c_int(0)
    rc = _lib.load().fastembedr_cuda_umap_graph_dump_from_knn(
        ctypes.c_void_p(idx_cm.ctypes.data), ctypes.c_void_p(dist_cm.ctypes.data), n, k, off,
        _ptr(heads, ctypes.c_int), _ptr(tails, ctypes.c_int), _ptr(weights, ctypes.c_float),
        _ptr(eps, ctypes.c_float), ctypes.byref(w_out), ctypes.byref(c_out))
    if rc != 0:
        raise CudaBackendError("CUDA UMAP graph dump failed: " + _lib.last_error())
    m = c_out.value
    return {"heads": heads[:m].copy(), "tails": tails[:m].copy(), "weights": weights[:m].copy(),
            "epochs_per_sample": eps[:m].copy(), "width": w_out.value, "capacity": m}


def umap_optimize_coo(heads, tails, weights, epochs_per_sample, init, n_epochs: int = 500,
                      negative_sample_rate: int = 5, learning_rate: float = 1.0,
                      min_dist: float = 0.1, repulsion_strength: float = 1.0, seed: int = 42,
                      optimizer_mode: int = 0) -> np.ndarray:
    """The CUDA COO UMAP optimizer (umap_cuda_optimize_coo_impl,
    src/embedding_cuda_impl.cpp:1898-1957): a, b from min_dist, then the C ABI."""
    h, t, w, e, y = _i32(heads), _i32(tails), _f32(weights), _f32(epochs_per_sample), _f32(init)
    if not (h.size == t.size == w.size == e.size):
        raise ValueError("COO heads, tails, weights, and epochs_per_sample must have the same length")
    if y.ndim != 2 or y.shape[1] != 2:
        raise ValueError("CUDA COO UMAP optimizer requires a two-dimensional initialization")
    a, b = find_ab_params(1.0, min_dist)
    out = np.zeros_like(y)
    rc = _lib.load().fastembedr_cuda_umap_optimize_coo(
        _ptr(h, ctypes.c_int), _ptr(t, ctypes.c_int), _ptr(w, ctypes.c_float), _ptr(e, ctypes.c_float),
        _ptr(y, ctypes.c_float), y.shape[0], h.size, n_epochs, negative_sample_rate, learning_rate,
        a, b, repulsion_strength, seed & 0xFFFFFFFF, optimizer_mode, _ptr(out, ctypes.c_float))
    if rc != 0:
        raise CudaBackendError("CUDA COO UMAP optimizer failed: " + _lib.last_error())
    return out


def umap_epochs(heads, tails, epochs_per_sample, layout, epoch_begin: int, epoch_end: int,
                n_epochs: int, negative_sample_rate: int = 5, learning_rate: float = 1.0,
                a: float = 1.5769434601962196, b: float = 0.8950608781227859,
                repulsion_strength: float = 1.0, seed: int = 42, optimizer_mode: int = 1,
                hash_key_is_tail: bool = False) -> Tuple[np.ndarray, int]:
    """Runs epochs [epoch_begin, epoch_end) from ``layout``; returns (layout, positive samples)."""
    h, t, e = _i32(heads), _i32(tails), _f32(epochs_per_sample)
    y = _f32(layout).copy()
    cnt = ctypes.c_longlong(0)
    check(_lib.load().fe_b200_umap_epochs(
        _ptr(h, ctypes.c_int), _ptr(t, ctypes.c_int), _ptr(e, ctypes.c_float), h.size,
        _ptr(y, ctypes.c_float), y.shape[0], epoch_begin, epoch_end, n_epochs, negative_sample_rate,
        learning_rate, a, b, repulsion_strength, seed & 0xFFFFFFFF, optimizer_mode,
        int(hash_key_is_tail), ctypes.byref(cnt)), "fe_b200_umap_epochs")
    return y, int(cnt.value)
