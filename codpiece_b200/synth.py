"""Seeded synthetic inputs for the benchmark configs (numpy, host side).

No dataset or checkpoint is involved: the configs fix shapes and value
distributions, and every value comes from ``numpy.random.default_rng(seed)``
(seed 0 unless stated), drawn in the order the functions below document.

* Q8_0 weight: d = fp16(|N(0, 0.02)| / 127) per 32-block, quants uniform in
  [-127, 127].
* Q4_K weight: d, dmin = fp16(|N(0, 0.01)|); eight six-bit scales and eight
  six-bit mins uniform in 0..63; 4-bit quants uniform in 0..15.
* Q6_K weight: ql and qh uniform bytes, int8 scales uniform, d = fp16(|N(0, 0.01)|).
* Activations: fp32 N(0, 1).

Blocks are packed in ggml's byte layout (the same layout libcpq reads).
"""
from __future__ import annotations

import numpy as np

Q8_0, Q4_K, Q6_K = 8, 12, 14


def pack_q4_K_scales(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """Pack [..., 8] six-bit scales and mins into ggml's 12-byte Q4_K field.

    Bytes 0-3: scale j (low 6 bits) with the top 2 bits of scale j+4;
    bytes 4-7: min j with the top 2 bits of min j+4; bytes 8-11: low nibble of
    scale j+4 and (high nibble) low nibble of min j+4.
    """
    sc = sc.astype(np.uint8)
    mn = mn.astype(np.uint8)
    out = np.empty(sc.shape[:-1] + (12,), np.uint8)
    out[..., 0:4] = sc[..., 0:4] | ((sc[..., 4:8] >> 4) << 6)
    out[..., 4:8] = mn[..., 0:4] | ((mn[..., 4:8] >> 4) << 6)
    out[..., 8:12] = (sc[..., 4:8] & 15) | ((mn[..., 4:8] & 15) << 4)
    return out


def pack_q4_K_quants(q: np.ndarray) -> np.ndarray:
    """[..., 256] values 0..15 -> [..., 128] bytes: qs[32j+l] = q[64j+l] | q[64j+32+l] << 4."""
    q = q.astype(np.uint8).reshape(q.shape[:-1] + (4, 2, 32))
    return (q[..., 0, :] | (q[..., 1, :] << 4)).reshape(q.shape[:-3] + (128,))


def q4_K_weights(rng: np.random.Generator, n: int, k: int) -> np.ndarray:
    nb = k // 256
    d = np.abs(rng.normal(0.0, 0.01, size=(n, nb))).astype(np.float16)
    dmin = np.abs(rng.normal(0.0, 0.01, size=(n, nb))).astype(np.float16)
    sc = rng.integers(0, 64, size=(n, nb, 8), dtype=np.uint8)
    mn = rng.integers(0, 64, size=(n, nb, 8), dtype=np.uint8)
    q = rng.integers(0, 16, size=(n, nb, 256), dtype=np.uint8)
    out = np.empty((n, nb, 144), np.uint8)
    out[..., 0:2] = d.view(np.uint8).reshape(n, nb, 2)
    out[..., 2:4] = dmin.view(np.uint8).reshape(n, nb, 2)
    out[..., 4:16] = pack_q4_K_scales(sc, mn)
    out[..., 16:144] = pack_q4_K_quants(q)
    return out.reshape(n, nb * 144)


def q6_K_weights(rng: np.random.Generator, n: int, k: int) -> np.ndarray:
    nb = k // 256
    out = np.empty((n, nb, 210), np.uint8)
    out[..., 0:208] = rng.integers(0, 256, size=(n, nb, 208), dtype=np.uint8)  # ql, qh, int8 scales
    d = np.abs(rng.normal(0.0, 0.01, size=(n, nb))).astype(np.float16)
    out[..., 208:210] = d.view(np.uint8).reshape(n, nb, 2)
    return out.reshape(n, nb * 210)


def q8_0_weights(rng: np.random.Generator, n: int, k: int) -> np.ndarray:
    nb = k // 32
    d = (np.abs(rng.normal(0.0, 0.02, size=(n, nb))) / 127.0).astype(np.float16)
    q = rng.integers(-127, 128, size=(n, nb, 32), dtype=np.int8)
    out = np.empty((n, nb, 34), np.uint8)
    out[..., 0:2] = d.view(np.uint8).reshape(n, nb, 2)
    out[..., 2:34] = q.view(np.uint8)
    return out.reshape(n, nb * 34)


WEIGHTS = {Q8_0: q8_0_weights, Q4_K: q4_K_weights, Q6_K: q6_K_weights}


def weights(qtype: int, n: int, k: int, seed: int = 0) -> np.ndarray:
    return WEIGHTS[qtype](np.random.default_rng(seed), n, k)


def activations(m: int, k: int, seed: int = 0) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal((m, k), dtype=np.float32)


def config_inputs(qtype: int, n: int, k: int, m: int, seed: int = 0):
    """Weight then activation from one generator (the order the configs are drawn in)."""
    rng = np.random.default_rng(seed)
    w = WEIGHTS[qtype](rng, n, k)
    x = rng.standard_normal((m, k), dtype=np.float32)
    return w, x
