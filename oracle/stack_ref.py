"""CPU restatement of one decode/verify step of the 27B-shaped stack.

TEST INFRASTRUCTURE ONLY (checker for codpiece_b200.stack and the timed CPU
reference arm of bench.py). Every projection is the oracle's restated
ggml-cpu mul_mat; the elementwise ops follow ggml-cpu's definitions:
rms_norm sums x*x in double (ggml_float), mean and scale in fp32; silu(x) =
x / (1 + exp(-x)); the residual adds are fp32 (codpiece-model/src/qwen35.rs:
2534-2537, 2777-2783). Tensor parallelism is emulated by summing per-rank
partials in rank order, which is what an allreduce computes.
"""
from __future__ import annotations

import numpy as np

from . import cpq_oracle as O


def rms_norm(x: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    x = np.asarray(x, np.float32)
    sq = (x * x).astype(np.float64).sum(axis=1)
    mean = (sq / x.shape[1]).astype(np.float32)
    scale = (np.float32(1.0) / np.sqrt(mean + np.float32(eps))).astype(np.float32)
    return (x * scale[:, None]).astype(np.float32)


def silu_mul(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = g.astype(np.float32)
    with np.errstate(over="ignore"):  # exp(-g) = inf for g << 0 gives silu = 0, as in float arithmetic
        return ((g / (np.float32(1.0) + np.exp(-g))) * u).astype(np.float32)


def layer_step(h: np.ndarray, lw: dict, k: int, nthreads: int = 0) -> np.ndarray:
    """One layer on the full (unsharded) weights. lw maps kind -> (uint8 rows, n_rows, k_elems)."""
    Q4 = O.Q4_K
    xn = rms_norm(h)
    wq, nq, _ = lw["q"]
    q = O.mul_mat(Q4, wq, k, nq, xn, nthreads)
    for kind in ("k", "v"):
        w, n, _ = lw[kind]
        O.mul_mat(Q4, w, k, n, xn, nthreads)
    wo, no, ko = lw["o"]
    h = (h + O.mul_mat(Q4, wo, ko, no, q, nthreads)).astype(np.float32)
    xn = rms_norm(h)
    wg, nf, _ = lw["gate"]
    wu, _, _ = lw["up"]
    g = O.mul_mat(Q4, wg, k, nf, xn, nthreads)
    u = O.mul_mat(Q4, wu, k, nf, xn, nthreads)
    a = silu_mul(g, u)
    wd, nd, kd = lw["down"]
    return (h + O.mul_mat(Q4, wd, kd, nd, a, nthreads)).astype(np.float32)


def head_step(h: np.ndarray, head: np.ndarray, k: int, n_vocab: int, nthreads: int = 0):
    logits = O.mul_mat(O.Q6_K, head, k, n_vocab, rms_norm(h), nthreads)
    return logits, logits.argmax(axis=1).astype(np.int32)
