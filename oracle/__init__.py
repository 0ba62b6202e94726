"""Parity checkers for the fastEmbedR optimizer hot path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke`` and the
CPU-baseline legs of ``bench.py`` may import this package; the product
(``fastembedr_b200``) never does.

Two checkers live here:

* ``liboracle.so`` -- a C restatement of the reference algorithms
  (``fe_oracle.c``; every function cites the reference routine it follows).
* ``_ref/libferef.so`` -- the reference's *own* CPU sources
  (``src/tsne_neighbors.cpp``, ``src/fast_knn_umap.cpp``) compiled unmodified
  through a small Rcpp stand-in (``rcpp_shim/Rcpp.h``).  It pins the
  restatement and is the CPU baseline.  It can only be rebuilt where the
  reference sources exist; elsewhere a prebuilt copy is used if present.

All embeddings are row-major ``float32[n, 2]``; KNN inputs are ``(n, k)``
arrays (converted to R's column-major layout here).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libferef.so")
# The same reference sources built at -O3 for x86-64-v3 hosts (a second CPU
# baseline beside R's default -O2; see Makefile).
REF_O3_SO = os.path.join(HERE, "_ref", "libferef_o3.so")
REF_VARIANTS = {"O2": REF_SO, "O3": REF_O3_SO}

_c_int_p = ctypes.POINTER(ctypes.c_int)
_c_float_p = ctypes.POINTER(ctypes.c_float)
_c_double_p = ctypes.POINTER(ctypes.c_double)

_lib = None
_ref = None
_ref_variants = {}


def build(ref_src: Optional[str] = None) -> None:
    """Compile the C restatement and, when the reference sources exist, ``_ref``."""
    cmd = ["make", "-s", "-C", HERE]
    if ref_src is not None:
        cmd.append(f"REF_SRC={ref_src}")
    subprocess.run(cmd, check=True)


def _ptr(a: np.ndarray, ctype):
    return a.ctypes.data_as(ctypes.POINTER(ctype))


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build()
        L = ctypes.CDLL(ORACLE_SO)
        L.or_tsne_grid_size.restype = ctypes.c_int
        L.or_tsne_build_p.restype = ctypes.c_longlong
        L.or_tsne_kl.restype = ctypes.c_double
        L.or_umap_powf.restype = ctypes.c_float
        L.or_umap_powf.argtypes = [ctypes.c_float, ctypes.c_float]
        L.or_umap_positive_samples.argtypes = [ctypes.c_float, ctypes.c_int]
        L.or_umap_negative_samples.argtypes = [ctypes.c_float, ctypes.c_int, ctypes.c_int]
        L.or_umap_negative_vertex.argtypes = [ctypes.c_int, ctypes.c_uint32, ctypes.c_int,
                                              ctypes.c_int, ctypes.c_uint32, ctypes.c_int]
        L.or_umap_graph.restype = ctypes.c_longlong
        L.or_umap_pack_coo.restype = ctypes.c_longlong
        _lib = L
    return _lib


def host_supports_x86_64_v3() -> bool:
    """Whether this host's CPU runs x86-64-v3 code (AVX2, BMI1/2, F16C, FMA,
    LZCNT, MOVBE), so that the -O3 build cannot stop on an illegal instruction."""
    try:
        with open("/proc/cpuinfo") as f:
            flags = next((line.split(":", 1)[1].split() for line in f if line.startswith("flags")), [])
    except OSError:
        return False
    return {"avx2", "bmi1", "bmi2", "f16c", "fma", "abm", "movbe"} <= set(flags)


def ref_available(variant: str = "O2") -> bool:
    if variant == "O3" and not host_supports_x86_64_v3():
        return False
    return os.path.exists(REF_VARIANTS[variant])


def ref(variant: str = "O2") -> ctypes.CDLL:
    """The reference's own CPU code (raises if it was never built); `variant`
    "O3" is the same code built at -O3 for x86-64-v3 hosts."""
    global _ref
    if variant != "O2":
        if variant not in _ref_variants:
            _ref_variants[variant] = _load_ref(REF_VARIANTS[variant])
        return _ref_variants[variant]
    if _ref is None:
        _ref = _load_ref(REF_SO)
    return _ref


def _load_ref(path: str) -> ctypes.CDLL:
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} missing: build it where the reference sources exist")
    R = ctypes.CDLL(path)
    R.feref_tsne_last_error.restype = ctypes.c_char_p
    R.feref_umap_last_error.restype = ctypes.c_char_p
    R.feref_tsne_p_build.restype = ctypes.c_void_p
    R.feref_tsne_p_build.argtypes = [_c_int_p, _c_float_p, ctypes.c_int, ctypes.c_int,
                                     ctypes.c_double, ctypes.c_int]
    R.feref_tsne_p_nnz.restype = ctypes.c_longlong
    R.feref_tsne_p_nnz.argtypes = [ctypes.c_void_p]
    R.feref_tsne_p_copy.argtypes = [ctypes.c_void_p, _c_int_p, _c_int_p, _c_float_p]
    R.feref_tsne_p_free.argtypes = [ctypes.c_void_p]
    R.feref_tsne_gradient_fft.argtypes = [_c_int_p, _c_int_p, _c_float_p, ctypes.c_int,
                                          _c_float_p, ctypes.c_float, ctypes.c_int,
                                          ctypes.c_int, _c_float_p]
    R.feref_tsne_gradient_exact.argtypes = [_c_int_p, _c_int_p, _c_float_p, ctypes.c_int,
                                            _c_float_p, ctypes.c_float, ctypes.c_int,
                                            _c_float_p]
    R.feref_tsne_attractive.argtypes = R.feref_tsne_gradient_exact.argtypes
    R.feref_tsne_update.argtypes = [_c_float_p, _c_float_p, _c_float_p, _c_float_p,
                                    ctypes.c_int, ctypes.c_float, ctypes.c_float,
                                    ctypes.c_float, ctypes.c_float, ctypes.c_int]
    R.feref_tsne_zero_mean.argtypes = [_c_float_p, ctypes.c_int]
    R.feref_tsne_iterate.argtypes = [_c_int_p, _c_int_p, _c_float_p, ctypes.c_int, _c_float_p,
                                     _c_float_p, _c_float_p, ctypes.c_int, ctypes.c_float,
                                     ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                     ctypes.c_float, ctypes.c_int, ctypes.c_int, _c_double_p]
    R.feref_tsne_kl.argtypes = [_c_int_p, _c_int_p, _c_float_p, ctypes.c_int, _c_float_p,
                                ctypes.c_int, _c_double_p]
    R.feref_tsne_run.argtypes = [_c_int_p, _c_float_p, ctypes.c_int, ctypes.c_int, _c_float_p,
                                 ctypes.c_double, ctypes.c_int, ctypes.c_int, ctypes.c_double,
                                 ctypes.c_double, ctypes.c_double, ctypes.c_int,
                                 ctypes.c_double, ctypes.c_double, ctypes.c_double,
                                 ctypes.c_double, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                 _c_float_p]
    R.feref_tsne_grid_size.argtypes = [ctypes.c_int, ctypes.c_int]
    R.feref_tsne_auto_parameters.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_double,
                                             ctypes.c_int, _c_double_p]
    R.feref_umap_graph.restype = ctypes.c_void_p
    R.feref_umap_graph.argtypes = [_c_int_p, _c_float_p, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_int]
    R.feref_umap_graph_nnz.restype = ctypes.c_longlong
    R.feref_umap_graph_nnz.argtypes = [ctypes.c_void_p]
    R.feref_umap_graph_copy.argtypes = [ctypes.c_void_p, _c_int_p, _c_int_p, _c_float_p,
                                        _c_float_p, _c_float_p]
    R.feref_umap_graph_free.argtypes = [ctypes.c_void_p]
    R.feref_umap_coo_replay.argtypes = [_c_int_p, _c_int_p, _c_float_p, _c_float_p,
                                        _c_float_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_double, ctypes.c_int, ctypes.c_double,
                                        ctypes.c_double, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_int, _c_float_p]
    R.feref_umap_csr_optimize.argtypes = [_c_int_p, _c_int_p, _c_float_p, _c_float_p,
                                          ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_double, ctypes.c_int, ctypes.c_double,
                                          ctypes.c_double, ctypes.c_int, ctypes.c_int,
                                          _c_float_p]
    R.feref_umap_powf.restype = ctypes.c_float
    R.feref_umap_powf.argtypes = [ctypes.c_float, ctypes.c_float]
    R.feref_umap_positive_samples.argtypes = [ctypes.c_float, ctypes.c_int]
    R.feref_umap_negative_samples.argtypes = [ctypes.c_float, ctypes.c_int, ctypes.c_int]
    R.feref_umap_negative_vertex.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_int, ctypes.c_longlong, ctypes.c_int]
    R.feref_find_ab.argtypes = [ctypes.c_double, ctypes.c_double, _c_double_p, _c_double_p]
    return R


def _cm(a: np.ndarray, dtype) -> np.ndarray:
    """(n, k) array -> R column-major buffer."""
    return np.ascontiguousarray(np.asarray(a, dtype=dtype).T)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int32)


class Csr:
    """Symmetric t-SNE P (or a UMAP graph) in CSR form."""

    def __init__(self, row_ptr, col, val):
        self.row_ptr = _i32(row_ptr)
        self.col = _i32(col)
        self.val = _f32(val)

    @property
    def n(self) -> int:
        return self.row_ptr.size - 1

    @property
    def nnz(self) -> int:
        return int(self.row_ptr[-1])


# ---------------------------------------------------------------- restatement


def tsne_grid_size(n: int, grid_override: int = 0) -> int:
    return lib().or_tsne_grid_size(n, grid_override)


def tsne_build_p(idx: np.ndarray, dist: np.ndarray, perplexity: float, index_offset: int = 0) -> Csr:
    n, k = idx.shape
    idx_cm, dist_cm = _cm(idx, np.int32), _cm(dist, np.float32)
    row_ptr = np.zeros(n + 1, np.int32)
    col = np.zeros(2 * n * k, np.int32)
    val = np.zeros(2 * n * k, np.float32)
    nnz = lib().or_tsne_build_p(_ptr(idx_cm, ctypes.c_int), _ptr(dist_cm, ctypes.c_float),
                                n, k, index_offset, ctypes.c_double(perplexity),
                                _ptr(row_ptr, ctypes.c_int), _ptr(col, ctypes.c_int),
                                _ptr(val, ctypes.c_float))
    if nnz < 0:
        raise ValueError("invalid KNN input for t-SNE affinities")
    return Csr(row_ptr, col[:nnz].copy(), val[:nnz].copy())


def tsne_gradient_fft(P: Csr, y: np.ndarray, exaggeration: float, grid_size: int,
                      return_z: bool = False):
    y = _f32(y)
    grad = np.zeros_like(y)
    z = ctypes.c_double(0.0)
    lib().or_tsne_gradient_fft(_ptr(P.row_ptr, ctypes.c_int), _ptr(P.col, ctypes.c_int),
                               _ptr(P.val, ctypes.c_float), P.n, _ptr(y, ctypes.c_float),
                               ctypes.c_float(exaggeration), grid_size,
                               _ptr(grad, ctypes.c_float), ctypes.byref(z))
    return (grad, z.value) if return_z else grad


def tsne_repulsive_fft(y: np.ndarray, grid_size: int):
    y = _f32(y)
    grad = np.zeros_like(y)
    z = ctypes.c_double(0.0)
    lib().or_tsne_repulsive_fft(_ptr(y, ctypes.c_float), y.shape[0], grid_size,
                                _ptr(grad, ctypes.c_float), ctypes.byref(z))
    return grad, z.value


def tsne_attractive(P: Csr, y: np.ndarray, exaggeration: float) -> np.ndarray:
    y = _f32(y)
    grad = np.zeros_like(y)
    lib().or_tsne_attractive(_ptr(P.row_ptr, ctypes.c_int), _ptr(P.col, ctypes.c_int),
                             _ptr(P.val, ctypes.c_float), P.n, _ptr(y, ctypes.c_float),
                             ctypes.c_float(exaggeration), _ptr(grad, ctypes.c_float))
    return grad


def tsne_gradient_exact(P: Csr, y: np.ndarray, exaggeration: float) -> np.ndarray:
    y = _f32(y)
    grad = np.zeros_like(y)
    lib().or_tsne_gradient_exact(_ptr(P.row_ptr, ctypes.c_int), _ptr(P.col, ctypes.c_int),
                                 _ptr(P.val, ctypes.c_float), P.n, _ptr(y, ctypes.c_float),
                                 ctypes.c_float(exaggeration), _ptr(grad, ctypes.c_float))
    return grad


def tsne_update(y, update, gains, grad, learning_rate, momentum, min_gain=0.01, max_step_norm=5.0):
    """One update + re-centering; returns new (y, update, gains)."""
    y, update, gains, grad = (_f32(a).copy() for a in (y, update, gains, grad))
    lib().or_tsne_update(_ptr(y, ctypes.c_float), _ptr(update, ctypes.c_float),
                         _ptr(gains, ctypes.c_float), _ptr(grad, ctypes.c_float), y.shape[0],
                         ctypes.c_float(learning_rate), ctypes.c_float(momentum),
                         ctypes.c_float(min_gain), ctypes.c_float(max_step_norm))
    return y, update, gains


def tsne_iterate(P: Csr, y, update, gains, iters, exaggeration, momentum, learning_rate,
                 min_gain=0.01, max_step_norm=5.0, grid_size=0):
    y, update, gains = (_f32(a).copy() for a in (y, update, gains))
    g = grid_size or tsne_grid_size(P.n)
    lib().or_tsne_iterate(_ptr(P.row_ptr, ctypes.c_int), _ptr(P.col, ctypes.c_int),
                          _ptr(P.val, ctypes.c_float), P.n, _ptr(y, ctypes.c_float),
                          _ptr(update, ctypes.c_float), _ptr(gains, ctypes.c_float), iters,
                          ctypes.c_float(exaggeration), ctypes.c_float(momentum),
                          ctypes.c_float(learning_rate), ctypes.c_float(min_gain),
                          ctypes.c_float(max_step_norm), g)
    return y, update, gains


def tsne_zero_mean(y):
    y = _f32(y).copy()
    lib().or_tsne_zero_mean(_ptr(y, ctypes.c_float), y.shape[0])
    return y


def tsne_kl(P: Csr, y: np.ndarray) -> float:
    y = _f32(y)
    return float(lib().or_tsne_kl(_ptr(P.row_ptr, ctypes.c_int), _ptr(P.col, ctypes.c_int),
                                  _ptr(P.val, ctypes.c_float), P.n, _ptr(y, ctypes.c_float)))


def tsne_run(P: Csr, init: np.ndarray, early_exaggeration_iter=250, n_iter=500,
             early_exaggeration=12.0, exaggeration=1.0, learning_rate=None,
             initial_momentum=0.8, final_momentum=0.8, min_gain=0.01, max_step_norm=5.0,
             grid_size: int = 0) -> np.ndarray:
    init = _f32(init)
    out = np.zeros_like(init)
    n = init.shape[0]
    g = grid_size or tsne_grid_size(n)
    lr_auto = learning_rate is None
    lib().or_tsne_run(_ptr(P.row_ptr, ctypes.c_int), _ptr(P.col, ctypes.c_int),
                      _ptr(P.val, ctypes.c_float), n, _ptr(init, ctypes.c_float),
                      early_exaggeration_iter, n_iter, ctypes.c_float(early_exaggeration),
                      ctypes.c_float(exaggeration), ctypes.c_float(learning_rate or 0.0),
                      int(lr_auto), ctypes.c_float(initial_momentum),
                      ctypes.c_float(final_momentum), ctypes.c_float(min_gain),
                      ctypes.c_float(max_step_norm), g, _ptr(out, ctypes.c_float))
    return out


def umap_powf(x: float, b: float) -> float:
    return lib().or_umap_powf(x, b)


def umap_positive_samples(period: float, epoch: int) -> int:
    return lib().or_umap_positive_samples(period, epoch)


def umap_negative_samples(period: float, nsr: int, epoch: int) -> int:
    return lib().or_umap_negative_samples(period, nsr, epoch)


def umap_negative_vertex(n, seed, epoch, head, key, sample) -> int:
    return lib().or_umap_negative_vertex(n, seed & 0xFFFFFFFF, epoch, head, key & 0xFFFFFFFF, sample)


def umap_find_ab(spread: float = 1.0, min_dist: float = 0.1):
    a, b = ctypes.c_double(), ctypes.c_double()
    lib().or_umap_find_ab(ctypes.c_double(spread), ctypes.c_double(min_dist),
                          ctypes.byref(a), ctypes.byref(b))
    return a.value, b.value


class UmapGraph:
    """Fuzzy-union CSR graph plus the COO view the CUDA optimizer consumes."""

    def __init__(self, offsets, neighbors, weights, epochs_per_sample, max_weight):
        self.offsets = _i32(offsets)
        self.neighbors = _i32(neighbors)
        self.weights = _f32(weights)
        self.epochs_per_sample = _f32(epochs_per_sample)
        self.max_weight = float(max_weight)

    @property
    def n(self) -> int:
        return self.offsets.size - 1

    def heads(self) -> np.ndarray:
        """CSR -> COO head expansion (as src/embedding_cuda_bridge.cpp:343-376 does)."""
        counts = np.diff(self.offsets)
        return np.repeat(np.arange(self.n, dtype=np.int32), counts)


def umap_graph(idx: np.ndarray, dist: np.ndarray, index_offset: int = 0) -> UmapGraph:
    n, k = idx.shape
    idx_cm, dist_cm = _cm(idx, np.int32), _cm(dist, np.float32)
    offsets = np.zeros(n + 1, np.int32)
    cap = 2 * n * k
    nb = np.zeros(cap, np.int32)
    w = np.zeros(cap, np.float32)
    eps = np.zeros(cap, np.float32)
    maxw = ctypes.c_float(0.0)
    nnz = lib().or_umap_graph(_ptr(idx_cm, ctypes.c_int), _ptr(dist_cm, ctypes.c_float), n, k,
                              index_offset, _ptr(offsets, ctypes.c_int), _ptr(nb, ctypes.c_int),
                              _ptr(w, ctypes.c_float), _ptr(eps, ctypes.c_float), ctypes.byref(maxw))
    if nnz < 0:
        raise ValueError("invalid KNN input for the UMAP graph")
    return UmapGraph(offsets, nb[:nnz].copy(), w[:nnz].copy(), eps[:nnz].copy(), maxw.value)


def umap_device_graph(idx: np.ndarray, dist: np.ndarray, index_offset: int = 0, binary: bool = False):
    """The device-KNN path's dense fuzzy graph: (nbr, w), each (n, width)."""
    n, k = idx.shape
    width = lib().or_umap_graph_width(k)
    idx_cm, dist_cm = _cm(idx, np.int32), _cm(dist, np.float32)
    nbr = np.zeros((n, width), np.int32)
    w = np.zeros((n, width), np.float32)
    rc = lib().or_umap_device_graph(_ptr(idx_cm, ctypes.c_int), _ptr(dist_cm, ctypes.c_float), n, k,
                                    index_offset, int(binary), _ptr(nbr, ctypes.c_int), _ptr(w, ctypes.c_float))
    if rc < 0:
        raise MemoryError("or_umap_device_graph")
    return nbr, w


def umap_pack_coo(nbr: np.ndarray, w: np.ndarray, rank_major: bool = True) -> dict:
    """Non-empty slots of a dense graph as COO arrays."""
    nbr, w = _i32(nbr), _f32(w)
    n, width = nbr.shape
    cap = n * width
    heads, tails = np.zeros(cap, np.int32), np.zeros(cap, np.int32)
    weights, eps = np.zeros(cap, np.float32), np.zeros(cap, np.float32)
    m = lib().or_umap_pack_coo(_ptr(nbr, ctypes.c_int), _ptr(w, ctypes.c_float), n, width, int(rank_major),
                               _ptr(heads, ctypes.c_int), _ptr(tails, ctypes.c_int),
                               _ptr(weights, ctypes.c_float), _ptr(eps, ctypes.c_float))
    return {"heads": heads[:m].copy(), "tails": tails[:m].copy(), "weights": weights[:m].copy(),
            "epochs_per_sample": eps[:m].copy()}


def umap_diffusion_init(nbr: np.ndarray, w: np.ndarray, seed: int, iters: int) -> np.ndarray:
    nbr, w = _i32(nbr), _f32(w)
    n, width = nbr.shape
    out = np.zeros((n, 2), np.float32)
    lib().or_umap_diffusion_init(_ptr(nbr, ctypes.c_int), _ptr(w, ctypes.c_float), n, width,
                                 ctypes.c_uint32(seed & 0xFFFFFFFF), iters, _ptr(out, ctypes.c_float))
    return out


def umap_epoch_delta(heads, tails, epochs_per_sample, layout, epoch, n_epochs,
                     negative_sample_rate=5, learning_rate=1.0, a=1.5769434601962196,
                     b=0.8950608781227859, repulsion_strength=1.0, seed=42,
                     hash_key_is_tail=False, max_abs_coord=16.0) -> np.ndarray:
    heads, tails, eps = _i32(heads), _i32(tails), _f32(epochs_per_sample)
    y = _f32(layout).copy()
    lib().or_umap_epoch_delta(_ptr(heads, ctypes.c_int), _ptr(tails, ctypes.c_int),
                              _ptr(eps, ctypes.c_float), heads.size, _ptr(y, ctypes.c_float),
                              y.shape[0], epoch, n_epochs, negative_sample_rate,
                              ctypes.c_float(learning_rate), ctypes.c_float(a), ctypes.c_float(b),
                              ctypes.c_float(repulsion_strength), ctypes.c_uint32(seed & 0xFFFFFFFF),
                              int(hash_key_is_tail), ctypes.c_float(max_abs_coord))
    return y


def umap_replay_serial(heads, tails, epochs_per_sample, layout, epoch_begin, epoch_end, n_epochs,
                       negative_sample_rate=5, learning_rate=1.0, a=1.5769434601962196,
                       b=0.8950608781227859, repulsion_strength=1.0, seed=42,
                       hash_key_is_tail=False, sanitize_each_epoch=True) -> np.ndarray:
    heads, tails, eps = _i32(heads), _i32(tails), _f32(epochs_per_sample)
    y = _f32(layout).copy()
    lib().or_umap_replay_serial(_ptr(heads, ctypes.c_int), _ptr(tails, ctypes.c_int),
                                _ptr(eps, ctypes.c_float), heads.size, _ptr(y, ctypes.c_float),
                                y.shape[0], epoch_begin, epoch_end, n_epochs, negative_sample_rate,
                                ctypes.c_float(learning_rate), ctypes.c_float(a),
                                ctypes.c_float(b), ctypes.c_float(repulsion_strength),
                                ctypes.c_uint32(seed & 0xFFFFFFFF), int(hash_key_is_tail),
                                int(sanitize_each_epoch))
    return y


# ------------------------------------------------------------ the reference


def _ref_check(rc: int, which: str = "tsne", variant: str = "O2") -> None:
    if rc != 0:
        R = ref(variant)
        msg = (R.feref_tsne_last_error() if which == "tsne" else R.feref_umap_last_error())
        raise RuntimeError(f"reference {which} call failed: {msg.decode()}")


def ref_tsne_grid_size(n: int, grid_override: int = 0) -> int:
    return ref().feref_tsne_grid_size(n, grid_override)


def ref_tsne_build_p(idx: np.ndarray, dist: np.ndarray, perplexity: float, threads: int = 1) -> Csr:
    n, k = idx.shape
    idx_cm, dist_cm = _cm(idx, np.int32), _cm(dist, np.float32)
    R = ref()
    h = R.feref_tsne_p_build(_ptr(idx_cm, ctypes.c_int), _ptr(dist_cm, ctypes.c_float), n, k,
                             perplexity, threads)
    if not h:
        raise RuntimeError("reference P build failed: " + R.feref_tsne_last_error().decode())
    nnz = R.feref_tsne_p_nnz(h)
    row_ptr = np.zeros(n + 1, np.int32)
    col = np.zeros(nnz, np.int32)
    val = np.zeros(nnz, np.float32)
    R.feref_tsne_p_copy(h, _ptr(row_ptr, ctypes.c_int), _ptr(col, ctypes.c_int), _ptr(val, ctypes.c_float))
    R.feref_tsne_p_free(h)
    return Csr(row_ptr, col, val)


def ref_tsne_gradient_fft(P: Csr, y, exaggeration, threads=1, grid_override=0) -> np.ndarray:
    y = _f32(y)
    grad = np.zeros_like(y)
    _ref_check(ref().feref_tsne_gradient_fft(
        _ptr(P.row_ptr, ctypes.c_int), _ptr(P.col, ctypes.c_int), _ptr(P.val, ctypes.c_float), P.n,
        _ptr(y, ctypes.c_float), exaggeration, threads, grid_override, _ptr(grad, ctypes.c_float)))
    return grad


def ref_tsne_gradient_exact(P: Csr, y, exaggeration, threads=1) -> np.ndarray:
    y = _f32(y)
    grad = np.zeros_like(y)
    _ref_check(ref().feref_tsne_gradient_exact(
        _ptr(P.row_ptr, ctypes.c_int), _ptr(P.col, ctypes.c_int), _ptr(P.val, ctypes.c_float), P.n,
        _ptr(y, ctypes.c_float), exaggeration, threads, _ptr(grad, ctypes.c_float)))
    return grad


def ref_tsne_update(y, update, gains, grad, learning_rate, momentum, min_gain=0.01,
                    max_step_norm=5.0, threads=1):
    y, update, gains, grad = (_f32(a).copy() for a in (y, update, gains, grad))
    _ref_check(ref().feref_tsne_update(
        _ptr(y, ctypes.c_float), _ptr(update, ctypes.c_float), _ptr(gains, ctypes.c_float),
        _ptr(grad, ctypes.c_float), y.shape[0], learning_rate, momentum, min_gain,
        max_step_norm, threads))
    return y, update, gains


def ref_tsne_iterate(P: Csr, y, update, gains, iters, exaggeration, momentum, learning_rate,
                     min_gain=0.01, max_step_norm=5.0, threads=1, grid_override=0, variant="O2"):
    """The reference's own iteration loop; returns (y, update, gains, loop_seconds)."""
    y, update, gains = (_f32(a).copy() for a in (y, update, gains))
    secs = ctypes.c_double(0.0)
    _ref_check(ref(variant).feref_tsne_iterate(
        _ptr(P.row_ptr, ctypes.c_int), _ptr(P.col, ctypes.c_int), _ptr(P.val, ctypes.c_float), P.n,
        _ptr(y, ctypes.c_float), _ptr(update, ctypes.c_float), _ptr(gains, ctypes.c_float), iters,
        exaggeration, momentum, learning_rate, min_gain, max_step_norm, threads, grid_override,
        ctypes.byref(secs)), "tsne", variant)
    return y, update, gains, secs.value


def ref_tsne_kl(P: Csr, y, threads=1) -> float:
    y = _f32(y)
    out = ctypes.c_double(0.0)
    _ref_check(ref().feref_tsne_kl(_ptr(P.row_ptr, ctypes.c_int), _ptr(P.col, ctypes.c_int),
                                   _ptr(P.val, ctypes.c_float), P.n, _ptr(y, ctypes.c_float),
                                   threads, ctypes.byref(out)))
    return out.value


def ref_tsne_run(idx, dist, init=None, perplexity=30.0, early_exaggeration_iter=250, n_iter=500,
                 early_exaggeration=12.0, exaggeration=1.0, learning_rate=None,
                 initial_momentum=0.8, final_momentum=0.8, min_gain=0.01, max_step_norm=5.0,
                 threads=1, seed=42, grid_override=0) -> np.ndarray:
    """knn_tsne_opentsne_float_cpp (the reference CPU backend of opentsne_knn)."""
    n, k = idx.shape
    idx_cm, dist_cm = _cm(idx, np.int32), _cm(dist, np.float32)
    out = np.zeros((n, 2), np.float32)
    init_p = None
    if init is not None:
        init = _f32(init)
        init_p = _ptr(init, ctypes.c_float)
    lr_auto = learning_rate is None
    _ref_check(ref().feref_tsne_run(
        _ptr(idx_cm, ctypes.c_int), _ptr(dist_cm, ctypes.c_float), n, k, init_p, perplexity,
        early_exaggeration_iter, n_iter, early_exaggeration, exaggeration,
        float(learning_rate or 0.0), int(lr_auto), initial_momentum, final_momentum, min_gain,
        max_step_norm, threads, seed, grid_override, _ptr(out, ctypes.c_float)))
    return out


def ref_tsne_auto_parameters(n: int, k: int, perplexity: float = 30.0, perplexity_missing=False):
    out = np.zeros(6, np.float64)
    _ref_check(ref().feref_tsne_auto_parameters(n, k, perplexity, int(perplexity_missing),
                                                _ptr(out, ctypes.c_double)))
    keys = ("perplexity", "n_neighbors", "early_exaggeration", "learning_rate",
            "early_exaggeration_iter", "n_iter")
    return dict(zip(keys, out.tolist()))


def ref_umap_graph(idx, dist, threads=1) -> UmapGraph:
    n, k = idx.shape
    idx_cm, dist_cm = _cm(idx, np.int32), _cm(dist, np.float32)
    R = ref()
    h = R.feref_umap_graph(_ptr(idx_cm, ctypes.c_int), _ptr(dist_cm, ctypes.c_float), n, k, threads)
    if not h:
        raise RuntimeError("reference UMAP graph failed: " + R.feref_umap_last_error().decode())
    nnz = R.feref_umap_graph_nnz(h)
    off = np.zeros(n + 1, np.int32)
    nb = np.zeros(nnz, np.int32)
    w = np.zeros(nnz, np.float32)
    eps = np.zeros(nnz, np.float32)
    maxw = ctypes.c_float(0.0)
    R.feref_umap_graph_copy(h, _ptr(off, ctypes.c_int), _ptr(nb, ctypes.c_int),
                            _ptr(w, ctypes.c_float), _ptr(eps, ctypes.c_float), ctypes.byref(maxw))
    R.feref_umap_graph_free(h)
    return UmapGraph(off, nb, w, eps, maxw.value)


def ref_umap_coo_replay(heads, tails, weights, epochs_per_sample, init, n_epochs, min_dist=0.1,
                        negative_sample_rate=5, learning_rate=1.0, repulsion_strength=1.0,
                        threads=1, seed=42, sanitize_each_epoch=True, variant="O2") -> np.ndarray:
    heads, tails, w, eps, init = _i32(heads), _i32(tails), _f32(weights), _f32(epochs_per_sample), _f32(init)
    out = np.zeros_like(init)
    _ref_check(ref(variant).feref_umap_coo_replay(
        _ptr(heads, ctypes.c_int), _ptr(tails, ctypes.c_int), _ptr(w, ctypes.c_float),
        _ptr(eps, ctypes.c_float), _ptr(init, ctypes.c_float), init.shape[0], heads.size,
        n_epochs, min_dist, negative_sample_rate, learning_rate, repulsion_strength, threads,
        seed, int(sanitize_each_epoch), _ptr(out, ctypes.c_float)), "umap", variant)
    return out


def ref_umap_csr_optimize(g: UmapGraph, init, n_epochs, min_dist=0.1, negative_sample_rate=5,
                          learning_rate=1.0, repulsion_strength=1.0, threads=1, seed=42):
    init = _f32(init)
    out = np.zeros_like(init)
    _ref_check(ref().feref_umap_csr_optimize(
        _ptr(g.offsets, ctypes.c_int), _ptr(g.neighbors, ctypes.c_int), _ptr(g.weights, ctypes.c_float),
        _ptr(init, ctypes.c_float), g.n, g.neighbors.size, n_epochs, min_dist,
        negative_sample_rate, learning_rate, repulsion_strength, threads, seed,
        _ptr(out, ctypes.c_float)), "umap")
    return out


def ref_umap_powf(x: float, b: float) -> float:
    return ref().feref_umap_powf(x, b)


def ref_umap_positive_samples(period, epoch) -> int:
    return ref().feref_umap_positive_samples(period, epoch)


def ref_umap_negative_samples(period, nsr, epoch) -> int:
    return ref().feref_umap_negative_samples(period, nsr, epoch)


def ref_umap_negative_vertex(n, seed, epoch, head, edge, sample) -> int:
    return ref().feref_umap_negative_vertex(n, seed, epoch, head, edge, sample)


def ref_find_ab(spread=1.0, min_dist=0.1):
    a, b = ctypes.c_double(), ctypes.c_double()
    ref().feref_find_ab(spread, min_dist, ctypes.byref(a), ctypes.byref(b))
    return a.value, b.value


# ------------------------------------------------- the reference's CUDA backend

REF_CUDA_SO = os.path.join(HERE, "_ref", "libferef_cuda.so")
_ref_cuda = None


def ref_cuda_available() -> bool:
    return os.path.exists(REF_CUDA_SO)


def ref_cuda() -> ctypes.CDLL:
    """The reference's own CUDA backend, src/embedding_cuda_kernels.cpp (needs a GPU to run)."""
    global _ref_cuda
    if _ref_cuda is None:
        if not os.path.exists(REF_CUDA_SO):
            raise FileNotFoundError(f"{REF_CUDA_SO} missing: build it where the reference sources exist")
        C = ctypes.CDLL(REF_CUDA_SO)
        I, F, U = ctypes.c_int, ctypes.c_float, ctypes.c_uint
        C.fastembedr_cuda_embedding_last_error.restype = ctypes.c_char_p
        C.fastembedr_cuda_available.restype = ctypes.c_bool
        C.fastembedr_cuda_umap_graph_dump_from_knn.argtypes = [
            _c_int_p, _c_double_p, I, I, I, _c_int_p, _c_int_p, _c_float_p, _c_float_p, _c_int_p, _c_int_p]
        C.fastembedr_cuda_umap_from_knn_spectral_float.argtypes = [
            _c_int_p, _c_float_p, I, I, I, I, F, F, F, F, I, U, I, I, _c_float_p]
        C.fastembedr_cuda_umap_optimize_coo.argtypes = [
            _c_int_p, _c_int_p, _c_float_p, _c_float_p, _c_float_p, I, I, I, I, F, F, F, F, U, I, _c_float_p]
        C.fastembedr_cuda_opentsne_fft_from_knn_float.argtypes = [
            _c_int_p, _c_float_p, _c_float_p, I, I, I, I, F, I, I, F, F, F, I, F, F, F, F, U, I, _c_float_p]
        C.fastembedr_cuda_landmark_tsne_from_device_knn.argtypes = [
            ctypes.c_void_p, ctypes.c_void_p, I, _c_float_p, _c_float_p, _c_float_p, I, I, I, I, F, I, I, F, F, F,
            F, F, F, F, I, I, U, I, F, F, _c_float_p]
        _ref_cuda = C
    return _ref_cuda


def _ref_cuda_check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"reference CUDA {what} failed: "
                           f"{ref_cuda().fastembedr_cuda_embedding_last_error().decode()}")


def ref_cuda_umap_graph_dump(idx: np.ndarray, dist: np.ndarray, index_offset: int = 0) -> dict:
    """fastembedr_cuda_umap_graph_dump_from_knn of the reference (rank-major COO)."""
    n, k = idx.shape
    width = min(256, 2 * k)
    cap = n * width
    idx_cm, dist_cm = _cm(idx, np.int32), _cm(dist, np.float64)
    heads, tails = np.full(cap, -1, np.int32), np.full(cap, -1, np.int32)
    weights, eps = np.zeros(cap, np.float32), np.zeros(cap, np.float32)
    w_out, c_out = ctypes.c_int(0), ctypes.c_int(0)
    rc = ref_cuda().fastembedr_cuda_umap_graph_dump_from_knn(
        _ptr(idx_cm, ctypes.c_int), _ptr(dist_cm, ctypes.c_double), n, k, index_offset,
        _ptr(heads, ctypes.c_int), _ptr(tails, ctypes.c_int), _ptr(weights, ctypes.c_float),
        _ptr(eps, ctypes.c_float), ctypes.byref(w_out), ctypes.byref(c_out))
    _ref_cuda_check(rc, "UMAP graph dump")
    m = c_out.value
    return {"heads": heads[:m].copy(), "tails": tails[:m].copy(), "weights": weights[:m].copy(),
            "epochs_per_sample": eps[:m].copy(), "width": w_out.value, "capacity": m}


def ref_cuda_umap_fused(idx: np.ndarray, dist: np.ndarray, n_epochs: int, negative_sample_rate: int = 5,
                        learning_rate: float = 1.0, a: float = 1.5769434601962196, b: float = 0.8950608781227859,
                        repulsion_strength: float = 1.0, spectral_n_iter: int = 30, seed: int = 42,
                        index_offset: int = 0, optimizer_mode: int = 0) -> np.ndarray:
    """fastembedr_cuda_umap_from_knn_spectral_float of the reference."""
    n, k = idx.shape
    idx_cm, dist_cm = _cm(idx, np.int32), _cm(dist, np.float32)
    out = np.zeros((n, 2), np.float32)
    rc = ref_cuda().fastembedr_cuda_umap_from_knn_spectral_float(
        _ptr(idx_cm, ctypes.c_int), _ptr(dist_cm, ctypes.c_float), n, k, n_epochs, negative_sample_rate,
        learning_rate, a, b, repulsion_strength, spectral_n_iter, seed & 0xFFFFFFFF, index_offset,
        optimizer_mode, _ptr(out, ctypes.c_float))
    _ref_cuda_check(rc, "fused UMAP")
    return out


def ref_cuda_tsne(idx: np.ndarray, dist: np.ndarray, init: np.ndarray, perplexity: float = 30.0,
                  early_exaggeration_iter: int = 250, n_iter: int = 500, early_exaggeration: float = 12.0,
                  exaggeration: float = 1.0, momentum: float = 0.8, min_gain: float = 0.01,
                  max_step_norm: float = 5.0, seed: int = 42, index_offset: int = 0) -> np.ndarray:
    """fastembedr_cuda_opentsne_fft_from_knn_float of the reference
    (src/embedding_cuda_kernels.cpp:5453-6008 behind the prototype at
    src/embedding_cuda_impl.cpp:100-120): host KNN to host layout, learning
    rate "auto", the grid from the reference's own CUDA policy."""
    n, k = idx.shape
    idx_cm, dist_cm = _cm(idx, np.int32), _cm(dist, np.float32)
    init = np.ascontiguousarray(init, np.float32)
    out = np.zeros((n, 2), np.float32)
    rc = ref_cuda().fastembedr_cuda_opentsne_fft_from_knn_float(
        _ptr(idx_cm, ctypes.c_int), _ptr(dist_cm, ctypes.c_float), _ptr(init, ctypes.c_float), 1, n, k, 2,
        perplexity, early_exaggeration_iter, n_iter, early_exaggeration, exaggeration, 0.0, 1, momentum,
        momentum, min_gain, max_step_norm, seed & 0xFFFFFFFF, index_offset, _ptr(out, ctypes.c_float))
    _ref_cuda_check(rc, "openTSNE FFT")
    return out


def ref_cuda_landmark_tsne(d_indices: int, d_distances: int, index_offset: int, reference_data: np.ndarray,
                           query_data: np.ndarray, reference_layout: np.ndarray, k: int, perplexity: float = 30.0,
                           n_iter: int = 250, early_exaggeration_iter: int = 50, learning_rate: float = 0.1,
                           early_exaggeration: float = 4.0, exaggeration: float = 1.5,
                           initial_momentum: float = 0.8, final_momentum: float = 0.8, max_grad_norm: float = 0.25,
                           max_step_norm: float = float("inf"), n_negatives: int = 256,
                           exact_repulsion_threshold: int = 4096, seed: int = 1009, affine_neighbors: int = 12,
                           affine_ridge: float = 1e-3, max_extrapolation: float = 2.5) -> np.ndarray:
    """fastembedr_cuda_landmark_tsne_from_device_knn of the reference
    (src/embedding_cuda_kernels.cpp:3496-3610): device KNN pointers of the
    queries into the reference (column-major n_query x k), host data and layout
    as (n, d) arrays (passed in R's column-major order), host layout out.
    Defaults are the R wrapper's (R/landmark_model.R:442-477)."""
    n_ref, dim = reference_data.shape
    n_q = query_data.shape[0]
    rd = np.ascontiguousarray(np.asarray(reference_data, np.float32).T).reshape(-1)
    qd = np.ascontiguousarray(np.asarray(query_data, np.float32).T).reshape(-1)
    rl = np.ascontiguousarray(np.asarray(reference_layout, np.float32).T).reshape(-1)
    out = np.zeros((n_q, 2), np.float32)
    rc = ref_cuda().fastembedr_cuda_landmark_tsne_from_device_knn(
        ctypes.c_void_p(d_indices), ctypes.c_void_p(d_distances), index_offset, _ptr(rd, ctypes.c_float),
        _ptr(qd, ctypes.c_float), _ptr(rl, ctypes.c_float), n_ref, n_q, dim, k, perplexity, n_iter,
        early_exaggeration_iter, learning_rate, early_exaggeration, exaggeration, initial_momentum, final_momentum,
        max_grad_norm, max_step_norm, n_negatives, exact_repulsion_threshold, seed & 0xFFFFFFFF, affine_neighbors,
        affine_ridge, max_extrapolation, _ptr(out, ctypes.c_float))
    _ref_cuda_check(rc, "landmark t-SNE")
    return out


def pca_start(x: np.ndarray) -> np.ndarray:
    """PCA start of the PCA-initialised openTSNE entry points, restated:
    column means in double, the data centred in float (as the reference's
    raft_tsvd_scores_to_device, src/embedding_cuda_kernels.cpp:3357-3390), the two
    leading eigenvectors of the covariance (RAFT TSVD's COV_EIG_DQ solver),
    scores signed so that each component's largest-magnitude score is positive
    (the TSVD sign flip), then centred and scaled so the larger standard
    deviation is 1e-4 (finalize_tsne_pca_init_stats_kernel /
    scale_tsne_pca_init_kernel, :1336-1404).  x: (n, p)."""
    x = np.asarray(x)
    mean = x.astype(np.float64).mean(0)
    xc = (x.astype(np.float32) - mean.astype(np.float32)).astype(np.float32)
    xd = xc.astype(np.float64)
    w, v = np.linalg.eigh(xd.T @ xd)
    v = v[:, np.argsort(-w, kind="stable")[:2]]
    s = xd @ v
    for c in range(2):
        if s[np.argmax(np.abs(s[:, c])), c] < 0:
            s[:, c] = -s[:, c]
    s = s.astype(np.float32).astype(np.float64)
    n = s.shape[0]
    mu = s.mean(0)
    ss = np.maximum((s * s).sum(0) - s.sum(0) ** 2 / n, 0.0)
    sd = np.sqrt(ss / max(n - 1, 1))
    scale = 1e-4 / sd.max() if np.isfinite(sd.max()) and sd.max() > 0 else 1.0
    return ((s - mu) * scale).astype(np.float32)


def _lagrange3(t):
    """Quadratic Lagrange basis at the nodes (j + 1/2) / 3, j = 0, 1, 2."""
    t0, t1, t2 = 1.0 / 6.0, 0.5, 5.0 / 6.0
    return np.stack([4.5 * (t - t1) * (t - t2), -9.0 * (t - t0) * (t - t2), 4.5 * (t - t0) * (t - t1)], -1)


def tsne_gradient_lagrange(P: Csr, y: np.ndarray, exaggeration: float, grid_size: int, return_z: bool = False):
    """The openTSNE gradient with FIt-SNE's box interpolation, restated in double
    (Linderman et al., "Fast interpolation-based t-SNE", Nature Methods 2019):
    square boxes of about one unit (intervals_per_integer = 1), at least 50 and at
    most grid_size // 3 per side, over the layout's bounding square from its lower
    corner; three nodes per box and side at (j + 1/2)/3 of the box, which form a
    uniform grid of spacing box / 3; charges {1, y_x, y_y} spread with quadratic
    Lagrange weights; linear convolution (zero-padded FFT) with 1/(1+d^2) and
    its square; the potentials gathered with the same weights;
    Z = sum_i phi_q(y_i) - n.  The attraction is the reference's
    (add_sparse_attractive_gradient_f, src/tsne_neighbors.cpp:985-1012)."""
    y = np.asarray(y, np.float32)
    yd = y.astype(np.float64)
    n = y.shape[0]
    g = grid_size
    lo = y.min(0).astype(np.float64)
    ext = float((y.max(0) - y.min(0)).max())
    if not np.isfinite(ext) or ext <= 0:
        ext = 1.0
    boxes = max(1, min(g // 3, max(50, int(np.ceil(np.float32(ext))))))
    box = ext / boxes
    h = box / 3.0
    u = (yd - lo) / box
    b = np.clip(np.floor(u), 0, boxes - 1).astype(np.int64)
    t = np.clip(u - b, 0.0, 1.0)
    wx, wy = _lagrange3(t[:, 0]), _lagrange3(t[:, 1])
    charges = np.zeros((3, g, g))
    nodes = []
    for k in range(3):
        for j in range(3):
            w = wx[:, j] * wy[:, k]
            ix, iy = 3 * b[:, 0] + j, 3 * b[:, 1] + k
            nodes.append((w, iy, ix))
            np.add.at(charges[0], (iy, ix), w)
            np.add.at(charges[1], (iy, ix), w * yd[:, 0])
            np.add.at(charges[2], (iy, ix), w * yd[:, 1])
    m = 2 * g
    off = np.arange(m)
    off = np.where(off < g, off, off - m).astype(np.float64) * h
    d2 = off[:, None] ** 2 + off[None, :] ** 2
    kq = 1.0 / (1.0 + d2)
    kq[g, :] = 0.0
    kq[:, g] = 0.0
    fq, fq2 = np.fft.rfft2(kq), np.fft.rfft2(kq * kq)

    def conv(c, kf):
        pad = np.zeros((m, m))
        pad[:g, :g] = c
        return np.fft.irfft2(np.fft.rfft2(pad) * kf, s=(m, m))[:g, :g]

    phi_q, phi_q2 = conv(charges[0], fq), conv(charges[0], fq2)
    phi_x, phi_y = conv(charges[1], fq2), conv(charges[2], fq2)
    gq = np.zeros(n)
    gq2 = np.zeros(n)
    gx = np.zeros(n)
    gy = np.zeros(n)
    for w, iy, ix in nodes:
        gq += w * phi_q[iy, ix]
        gq2 += w * phi_q2[iy, ix]
        gx += w * phi_x[iy, ix]
        gy += w * phi_y[iy, ix]
    z = float(gq.sum() - n)
    rep = -np.stack([yd[:, 0] * gq2 - gx, yd[:, 1] * gq2 - gy], 1) / z
    rows = np.repeat(np.arange(n), np.diff(P.row_ptr))
    dd = yd[rows] - yd[P.col]
    q = 1.0 / (1.0 + (dd * dd).sum(1))
    att = np.zeros((n, 2))
    np.add.at(att, rows, (exaggeration * P.val.astype(np.float64) * q)[:, None] * dd)
    grad = (rep + att).astype(np.float32)
    return (grad, z) if return_z else grad
