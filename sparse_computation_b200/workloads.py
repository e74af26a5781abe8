"""Seeded synthetic inputs with the shapes, sparsities and value laws of the
five benchmark configurations (the reference publishes no dataset; its one
shipped matrix is a 512x512 transformer weight with all values 1).

Every matrix is returned as CSR arrays (indptr int32, indices int32 ascending
per row, data float64 holding float32-exact values, so the float32 that the
kernels and the CPU reference see is the same number).

  config1()          512x512, Bernoulli keep 0.10, N(0, 0.05^2); B 512x32
  config2(s, ...)    512x512 magnitude-pruned N(0, 0.05^2) to sparsity s
  config3(shape)     2048x512 / 512x2048, 90% sparse, per-row keep ~ Beta(2,18)
  config4()          96-matrix transformer-base stack, 80% magnitude-pruned
  config5()          16384x16384, 95%: half the nonzeros in aligned 4x1
                     vertical runs, half unstructured, N(0, 0.02^2)
"""
from __future__ import annotations

from typing import List, Tuple

import numpy as np

CSRArrays = Tuple[int, int, np.ndarray, np.ndarray, np.ndarray]  # m, n, indptr, indices, data


def csr_from_coords(m: int, n: int, rows: np.ndarray, cols: np.ndarray, vals: np.ndarray) -> CSRArrays:
    """Sorted, duplicate-free CSR from coordinates (first value of a duplicate wins)."""
    lin = rows.astype(np.int64) * n + cols.astype(np.int64)
    lin, first = np.unique(lin, return_index=True)
    vals = np.asarray(vals)[first]
    r = (lin // n).astype(np.int64)
    c = (lin % n).astype(np.int32)
    indptr = np.zeros(m + 1, np.int64)
    np.add.at(indptr, r + 1, 1)
    indptr = np.cumsum(indptr).astype(np.int32)
    return m, n, indptr, c, vals.astype(np.float32).astype(np.float64)


def csr_from_dense(A: np.ndarray) -> CSRArrays:
    r, c = np.nonzero(A)
    return csr_from_coords(A.shape[0], A.shape[1], r, c, A[r, c])


def dense_b(k: int, n: int, seed: int) -> np.ndarray:
    """B (k x n) float32 U(-1, 1), row-major."""
    return np.random.default_rng(seed).uniform(-1.0, 1.0, size=(k, n)).astype(np.float32)


def magnitude_pruned(m: int, n: int, sparsity: float, sigma: float, seed: int) -> CSRArrays:
    """Draws N(0, sigma^2) weights and zeroes the smallest |w| until `sparsity`."""
    rng = np.random.default_rng(seed)
    W = rng.normal(0.0, sigma, size=(m, n)).astype(np.float32)
    keep = int(round((1.0 - sparsity) * m * n))
    flat = np.abs(W).ravel()
    if keep <= 0:
        W[:] = 0
    elif keep < flat.size:
        thr_idx = np.argpartition(flat, flat.size - keep)[: flat.size - keep]
        W.ravel()[thr_idx] = 0
    return csr_from_dense(W)


def config1() -> Tuple[CSRArrays, np.ndarray]:
    m = n = 512
    mask = np.random.default_rng(1).random((m, n)) < 0.10
    vals = np.random.default_rng(2).normal(0.0, 0.05, size=(m, n)).astype(np.float32)
    A = np.where(mask, vals, 0).astype(np.float32)
    return csr_from_dense(A), dense_b(n, 32, 3)


CONFIG2_SPARSITIES = (0.50, 0.70, 0.80, 0.90, 0.95, 0.98)


def config2(sparsity: float, n_cols_b: int) -> Tuple[CSRArrays, np.ndarray]:
    s_idx = CONFIG2_SPARSITIES.index(sparsity) if sparsity in CONFIG2_SPARSITIES else int(sparsity * 100)
    a = magnitude_pruned(512, 512, sparsity, 0.05, 10 + s_idx)
    return a, dense_b(512, n_cols_b, 1000 + s_idx)


def row_skewed(m: int, n: int, seed: int, sigma: float = 0.05) -> CSRArrays:
    """Per-row keep probability ~ Beta(2, 18) (mean 0.10), N(0, sigma^2) values."""
    rng = np.random.default_rng(seed)
    p = rng.beta(2.0, 18.0, size=m)
    mask = rng.random((m, n)) < p[:, None]
    vals = rng.normal(0.0, sigma, size=(m, n)).astype(np.float32)
    return csr_from_dense(np.where(mask, vals, 0).astype(np.float32))


def config3(shape: Tuple[int, int], n_cols_b: int) -> Tuple[CSRArrays, np.ndarray]:
    seed = 20 if shape == (2048, 512) else 21
    a = row_skewed(shape[0], shape[1], seed)
    return a, dense_b(shape[1], n_cols_b, 2000 + seed)


def config4_shapes() -> List[Tuple[str, int, int]]:
    """(name, rows, cols) of the 96 weights of a 6+6-layer transformer-base."""
    out = []
    for layer in range(6):
        for w in ("q", "k", "v", "o"):
            out.append((f"enc{layer}.self_attn.{w}", 512, 512))
        out.append((f"enc{layer}.ffn1", 2048, 512))
        out.append((f"enc{layer}.ffn2", 512, 2048))
    for layer in range(6):
        for w in ("q", "k", "v", "o"):
            out.append((f"dec{layer}.self_attn.{w}", 512, 512))
        for w in ("q", "k", "v", "o"):
            out.append((f"dec{layer}.encdec_attn.{w}", 512, 512))
        out.append((f"dec{layer}.ffn1", 2048, 512))
        out.append((f"dec{layer}.ffn2", 512, 2048))
    return out


def config4(n_cols_b: int = 128):
    """[(name, csr, B)] for the 96 matrices, 80% magnitude-pruned, seed 100 + index."""
    out = []
    for i, (name, m, n) in enumerate(config4_shapes()):
        a = magnitude_pruned(m, n, 0.80, 0.05, 100 + i)
        out.append((name, a, dense_b(n, n_cols_b, 5000 + i)))
    return out


def config5(n: int = 16384, density: float = 0.05, n_cols_b: int = 128, seed: int = 500):
    """Scale-out matrix: half the nonzeros in 4x1 vertical runs starting on
    rows that are multiples of 4, half unstructured; N(0, 0.02^2) values."""
    rng = np.random.default_rng(seed)
    target = int(density * n * n)
    n_runs = target // 8
    run_r = rng.integers(0, n // 4, size=n_runs, dtype=np.int64) * 4
    run_c = rng.integers(0, n, size=n_runs, dtype=np.int64)
    rr = (run_r[:, None] + np.arange(4)[None, :]).ravel()
    rc = np.repeat(run_c, 4)
    n_un = target - 4 * n_runs
    ur = rng.integers(0, n, size=n_un, dtype=np.int64)
    uc = rng.integers(0, n, size=n_un, dtype=np.int64)
    rows = np.concatenate([rr, ur])
    cols = np.concatenate([rc, uc])
    vals = rng.normal(0.0, 0.02, size=rows.size).astype(np.float32)
    vals[vals == 0] = np.float32(1e-8)
    a = csr_from_coords(n, n, rows, cols, vals)
    return a, dense_b(n, n_cols_b, seed + 1)


def write_mtx(path: str, a: CSRArrays) -> None:
    """Writes CSR arrays as a 'coordinate real general' Matrix-Market file
    (1-based, values with %.9g, which round-trips float32)."""
    m, n, indptr, indices, data = a
    rows = np.repeat(np.arange(m), np.diff(indptr))
    with open(path, "w") as f:
        f.write("%%MatrixMarket matrix coordinate real general\n")
        f.write(f"{m} {n} {len(indices)}\n")
        for r, c, v in zip(rows, indices, data):
            f.write(f"{r + 1} {c + 1} {float(v):.9g}\n")
