"""ctypes wrapper of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Restated ggml-cpu semantics for quantized mul_mat (see cpq_oracle.h). Used by
tests/ as the parity checker and by bench.py as the timed CPU baseline.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libcpq_oracle.so"

F32, F16, Q8_0, Q4_K, Q6_K, Q8_K = 0, 1, 8, 12, 14, 15
BLOCK = {Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210), Q8_K: (256, 292)}
VEC_DOT = {Q4_K: Q8_K, Q6_K: Q8_K, Q8_0: Q8_0}
Q8_0_X86_AVX2, Q8_0_PORTABLE = 0, 1

_lib = None


def build(force: bool = False) -> Path:
    srcs = [HERE / n for n in ("cpq_oracle.c", "cpq_oracle_avx2.c", "cpq_oracle_gdn.c", "cpq_oracle.h", "Makefile")]
    if force or not LIB_PATH.exists() or any(s.stat().st_mtime > LIB_PATH.stat().st_mtime for s in srcs):
        env = dict(os.environ)
        env.pop("CC", None)
        subprocess.run(["make", "-s", "-B" if force else "-s", "-C", str(HERE)], check=True, env=env)
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        vp, i64, sz = C.c_void_p, C.c_int64, C.c_size_t
        L.oq_quantize_act.argtypes = [C.c_int, vp, i64, i64, vp, C.c_int]
        L.oq_mul_mat.argtypes = [C.c_int, vp, i64, i64, sz, vp, i64, vp, C.c_int, C.c_int, C.c_int]
        L.oq_mul_mat_q.argtypes = [C.c_int, vp, i64, i64, sz, vp, i64, vp, C.c_int, C.c_int]
        L.oq_mul_mat_f32.argtypes = [vp, i64, i64, vp, i64, vp]
        L.oq_mul_mat_f32.restype = None
        for f in ("oq_dequantize_row_q8_0", "oq_dequantize_row_q4_K", "oq_dequantize_row_q6_K"):
            getattr(L, f).argtypes = [vp, vp, i64]
            getattr(L, f).restype = None
        L.oq_fp32_to_fp16.argtypes = [C.c_float]
        L.oq_fp32_to_fp16.restype = C.c_uint16
        L.oq_fp16_to_fp32.argtypes = [C.c_uint16]
        L.oq_fp16_to_fp32.restype = C.c_float
        L.oq_quantize_row_q8_0.argtypes = [vp, vp, i64, C.c_int]
        L.oq_quantize_row_q8_0.restype = None
        L.oq_quantize_row_q8_K.argtypes = [vp, vp, i64]
        L.oq_quantize_row_q8_K.restype = None
        L.oq_gated_delta_net.argtypes = [vp] * 8 + [i64] * 6 + [C.c_int, C.c_int, i64]
        _lib = L
    return _lib


def _p(a: np.ndarray) -> C.c_void_p:
    return C.c_void_p(a.ctypes.data)


def row_bytes(qtype: int, k: int) -> int:
    blk, size = BLOCK[qtype]
    assert k % blk == 0
    return k // blk * size


def quantize_act(wtype: int, x: np.ndarray, variant: int = Q8_0_X86_AVX2) -> np.ndarray:
    """[M, K] fp32 -> [M, row_bytes(vec_dot_type)] uint8 ggml blocks."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.ndim == 1:
        x = x[None]
    m, k = x.shape
    out = np.zeros((m, row_bytes(VEC_DOT[wtype], k)), np.uint8)
    assert lib().oq_quantize_act(wtype, _p(x), k, m, _p(out), variant) == 0
    return out


def mul_mat(wtype: int, w: np.ndarray, k: int, n: int, x: np.ndarray, nthreads: int = 0, simd: int = 1,
            variant: int = Q8_0_X86_AVX2) -> np.ndarray:
    """Y [M, N] = ggml-cpu mul_mat(W [N rows], X [M, K])."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.ndim == 1:
        x = x[None]
    m = x.shape[0]
    y = np.empty((m, n), np.float32)
    rb = row_bytes(wtype, k)
    assert w.size >= n * rb
    assert lib().oq_mul_mat(wtype, _p(w), k, n, rb, _p(x), m, _p(y), nthreads, simd, variant) == 0
    return y


def mul_mat_q(wtype: int, w: np.ndarray, k: int, n: int, xq: np.ndarray, m: int, nthreads: int = 0,
              simd: int = 1) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8)
    xq = np.ascontiguousarray(xq, dtype=np.uint8)
    y = np.empty((m, n), np.float32)
    assert lib().oq_mul_mat_q(wtype, _p(w), k, n, row_bytes(wtype, k), _p(xq), m, _p(y), nthreads, simd) == 0
    return y


def dequantize(wtype: int, w: np.ndarray, k: int, n: int) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8).reshape(n, row_bytes(wtype, k))
    out = np.empty((n, k), np.float32)
    f = {Q8_0: "oq_dequantize_row_q8_0", Q4_K: "oq_dequantize_row_q4_K", Q6_K: "oq_dequantize_row_q6_K"}[wtype]
    fn = getattr(lib(), f)
    for r in range(n):
        fn(C.c_void_p(w[r].ctypes.data), C.c_void_p(out[r].ctypes.data), k)
    return out


def mul_mat_f32(w: np.ndarray, x: np.ndarray) -> np.ndarray:
    """F32 ggml mul_mat: w [N, K], x [M, K] -> [M, N]."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, k = w.shape
    m = x.shape[0]
    y = np.empty((m, n), np.float32)
    lib().oq_mul_mat_f32(_p(w), k, n, _p(x), m, _p(y))
    return y


def fp32_to_fp16_bits(f: float) -> int:
    return int(lib().oq_fp32_to_fp16(f))


def max_threads() -> int:
    return int(lib().oq_max_threads())


def gated_delta_net(q: np.ndarray, k: np.ndarray, v: np.ndarray, g: np.ndarray, beta: np.ndarray,
                    state: np.ndarray, n_snap: int = 1):
    """ggml_gated_delta_net on contiguous arrays (numpy order = ggml ne reversed):
    q, k [n_seqs_qk, T, H_qk, S_v]; v [n_seqs, T, H, S_v]; g [n_seqs, T, H] or
    [n_seqs, T, H, S_v] (per-row decay); beta [n_seqs, T, H]; state
    [n_seqs, H, S_v (col), S_v (i)]. Returns (attn [n_seqs, T, H, S_v],
    states [slots, n_seqs, H, S_v, S_v]) with slots = min(n_snap, T) (1 if
    n_snap <= 1)."""
    q, k, v, g, beta, state = (np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v, g, beta, state))
    n_seqs, t, h, sv = v.shape
    n_seqs_qk, _, h_qk, _ = q.shape
    kda = int(g.ndim == 4)
    slots = min(n_snap, t) if n_snap > 1 else 1
    attn = np.empty_like(v)
    states = np.zeros((slots, n_seqs, h, sv, sv), np.float32)
    d = n_seqs * h * sv * sv
    assert lib().oq_gated_delta_net(_p(q), _p(k), _p(v), _p(g), _p(beta), _p(state), _p(attn), _p(states), sv, h,
                                    h_qk, t, n_seqs, n_seqs_qk, kda, n_snap, d) == 0
    return attn, states
