"""The CPU oracle, pinned before it is trusted.

Pins: gguf-py (llama.cpp's own Python implementation of the block formats)
for dequantization and the portable Q8_0 quantizer, via committed fixtures
(tests/golden/make_golden.py); the F32 mul_mat layout of
crates/codpiece-ggml-sys/tests/smoke.rs:18-60; hand-derived known answers for
the Q8_K quantizer (ggml quantize_row_q8_K_ref semantics).
"""
import struct
from pathlib import Path

import numpy as np
import pytest

from codpiece_b200 import synth

GOLDEN = Path(__file__).resolve().parent / "golden" / "gguf_py_fixtures.npz"


def q8k_fields(blob: np.ndarray):
    """Split one 292-byte block_q8_K into (d, qs, bsums)."""
    b = bytes(blob)
    d = struct.unpack("<f", b[:4])[0]
    qs = np.frombuffer(b[4:260], np.int8)
    bs = np.frombuffer(b[260:292], np.int16)
    return d, qs, bs


def test_fp16_conversion_matches_ieee(oracle):
    rng = np.random.default_rng(1)
    vals = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * np.float32(10.0) ** rng.integers(-9, 5, 20000),
        np.array([0.0, -0.0, 65504.0, 65519.0, 65520.0, 1e9, 6.0e-8, 3.0e-8, 2.9e-8, 6.1e-5, 2.0 ** -24,
                  1.0 + 2.0 ** -11, 1.0 + 3 * 2.0 ** -11], np.float32),
    ]).astype(np.float32)
    mine = np.array([oracle.fp32_to_fp16_bits(float(v)) for v in vals], np.uint16)
    with np.errstate(over="ignore"):
        ref = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(mine, ref)


def test_dequantize_matches_gguf_py_fixtures(oracle):
    g = np.load(GOLDEN)
    for name, qt in (("q8_0", oracle.Q8_0), ("q4_K", oracle.Q4_K), ("q6_K", oracle.Q6_K)):
        blocks, deq = g[f"{name}_blocks"], g[f"{name}_deq"]
        blk = oracle.BLOCK[qt][0]
        mine = oracle.dequantize(qt, blocks.reshape(-1), blk * blocks.shape[0], 1).reshape(deq.shape)
        assert np.array_equal(mine.view(np.uint32), deq.view(np.uint32)), name


def test_portable_q8_0_quantizer_matches_gguf_py(oracle):
    g = np.load(GOLDEN)
    x = g["q8_0_quant_x"]
    mine = oracle.quantize_act(oracle.Q8_0, x, variant=oracle.Q8_0_PORTABLE)
    assert np.array_equal(mine, g["q8_0_quant_portable"])


def test_gguf_py_live_cross_check(oracle):
    gg = pytest.importorskip("gguf")
    from gguf import GGMLQuantizationType as T

    for qt, gt in ((oracle.Q8_0, T.Q8_0), (oracle.Q4_K, T.Q4_K), (oracle.Q6_K, T.Q6_K)):
        w = synth.weights(qt, 5, 1024, seed=11)
        ref = gg.quants.dequantize(w, gt).reshape(5, 1024)
        assert np.array_equal(oracle.dequantize(qt, w, 1024, 5).view(np.uint32), ref.astype(np.float32).view(np.uint32))


def test_q8_K_known_answers(oracle):
    x = np.zeros((4, 256), np.float32)
    # block 0: all zero -> d = 0, quants 0, bsums 0
    # block 1: single element 2.0 -> max = 2, iscale = -63.5, q = -127, d = 1/-63.5
    x[1, 5] = 2.0
    # block 2: -127 first, +127 later (same magnitude, the first wins): max = -127,
    #          iscale = -127/max = 1, d = 1; ties at .5 round to even:
    #          2.5 -> 2, 3.5 -> 4, -2.5 -> -2
    x[2, 0] = -127.0
    x[2, 4] = 127.0
    x[2, 17] = 2.5
    x[2, 18] = 3.5
    x[2, 19] = -2.5
    # block 3: max = -4 -> iscale = 31.75, q = -127 at the max, rne(31.75) = 32
    x[3, 100] = -4.0
    x[3, 101] = 1.0
    q = oracle.quantize_act(oracle.Q4_K, x.reshape(1, -1))[0].reshape(4, 292)

    d, qs, bs = q8k_fields(q[0])
    assert d == 0.0 and not qs.any() and not bs.any()

    d, qs, bs = q8k_fields(q[1])
    assert d == np.float32(1.0) / np.float32(-63.5)
    assert qs[5] == -127 and np.count_nonzero(qs) == 1 and bs[0] == -127 and np.count_nonzero(bs) == 1

    d, qs, bs = q8k_fields(q[2])
    assert d == 1.0
    assert qs[0] == -127 and qs[4] == 127
    assert list(qs[17:20]) == [2, 4, -2]
    assert bs[0] == 0 and bs[1] == 4

    d, qs, bs = q8k_fields(q[3])
    assert d == np.float32(1.0) / np.float32(31.75)
    assert qs[100] == -127 and qs[101] == 32 and bs[6] == -95


def test_q8_K_structure_on_baseline_activations(oracle):
    x = synth.activations(16, 5120, seed=3)
    q = oracle.quantize_act(oracle.Q4_K, x).reshape(-1, 292)
    for blob, xb in zip(q[:200], x.reshape(-1, 256)[:200]):
        d, qs, bs = q8k_fields(blob)
        assert np.array_equal(bs, qs.reshape(16, 16).sum(1))
        assert np.abs(qs).max() == 127
        # d * q reconstructs x to half a step
        assert np.abs(d * qs.astype(np.float32) - xb).max() <= abs(d) * 0.5 * (1 + 1e-5)


def test_q8_0_x86_rounds_half_to_even_portable_away(oracle):
    x = np.zeros((1, 32), np.float32)
    x[0, 0] = 127.0  # amax 127: d = 1 and 127/amax = 1 exactly, so x*id = x
    x[0, 1] = 2.5
    x[0, 2] = -3.5
    x[0, 3] = 0.5
    avx2 = oracle.quantize_act(oracle.Q8_0, x, variant=oracle.Q8_0_X86_AVX2)[0]
    port = oracle.quantize_act(oracle.Q8_0, x, variant=oracle.Q8_0_PORTABLE)[0]
    assert list(avx2[2:6].view(np.int8)) == [127, 2, -4, 0]
    assert list(port[2:6].view(np.int8)) == [127, 3, -4, 1]
    assert avx2[:2].view(np.float16)[0] == 1.0


def test_f32_mul_mat_layout_matches_smoke_rs(oracle):
    # smoke.rs:29-54: A ne=[2,3] = [[1,2],[3,4],[5,6]], B ne=[2,2] = [[1,1],[2,2]]
    a = np.array([[1, 2], [3, 4], [5, 6]], np.float32)
    b = np.array([[1, 1], [2, 2]], np.float32)
    out = oracle.mul_mat_f32(a, b)
    assert out.reshape(-1).tolist() == [3.0, 7.0, 11.0, 6.0, 14.0, 22.0]


@pytest.mark.parametrize("qt", [synth.Q4_K, synth.Q6_K, synth.Q8_0])
def test_simd_integer_totals_equal_scalar(oracle, qt):
    w, x = synth.config_inputs(qt, 48, 2048, 5, seed=9)
    y1 = oracle.mul_mat(qt, w, 2048, 48, x, simd=1)
    y0 = oracle.mul_mat(qt, w, 2048, 48, x, simd=0)
    assert np.array_equal(y1.view(np.uint32), y0.view(np.uint32))


@pytest.mark.parametrize("qt", [synth.Q4_K, synth.Q6_K, synth.Q8_0])
def test_quantized_product_tracks_float_product(oracle, qt):
    # the only difference to a float matmul on dequantized weights is the int8
    # activation re-quantization (~0.5-1% of max|y| at these distributions)
    w, x = synth.config_inputs(qt, 32, 5120, 3, seed=4)
    y = oracle.mul_mat(qt, w, 5120, 32, x)
    yf = x @ oracle.dequantize(qt, w, 5120, 32).T
    err = np.abs(y - yf).max() / np.abs(yf).max()
    assert 1e-4 < err < 3e-2


def test_empty_and_minimal_shapes(oracle):
    w = synth.weights(synth.Q4_K, 3, 256, seed=2)
    y = oracle.mul_mat(synth.Q4_K, w, 256, 3, np.zeros((0, 256), np.float32))
    assert y.shape == (0, 3)
    x = synth.activations(1, 256, seed=2)
    y = oracle.mul_mat(synth.Q4_K, w, 256, 3, x)
    assert y.shape == (1, 3) and np.isfinite(y).all()


@pytest.mark.parametrize("qt", [synth.Q4_K, synth.Q6_K, synth.Q8_0])
def test_block_dots_match_gguf_py_dequantization(oracle, qt):
    """The integer block dots (scales, mins, the Q6_K -32 offset, bsums) against the
    definition they implement: gguf-py's dequantized weights (llama.cpp's own Python
    decoding of the formats) times the dequantized activation blocks d * q, summed in
    float64. Only fp32 rounding separates the two."""
    gg = pytest.importorskip("gguf")
    from gguf import GGMLQuantizationType as T

    gt = {synth.Q4_K: T.Q4_K, synth.Q6_K: T.Q6_K, synth.Q8_0: T.Q8_0}[qt]
    n, k, m = 16, 2048, 3
    w, x = synth.config_inputs(qt, n, k, m, seed=21)
    wd = gg.quants.dequantize(w, gt).reshape(n, k).astype(np.float64)
    xq = oracle.quantize_act(qt, x)                          # [m, row bytes] of Q8_K / Q8_0 blocks
    if qt == synth.Q8_0:
        blk = xq.reshape(m, k // 32, 34)
        d = blk[:, :, :2].copy().view(np.float16).astype(np.float64)[..., 0]
        q = blk[:, :, 2:].view(np.int8).astype(np.float64)
        xd = (q * d[..., None]).reshape(m, k)
    else:
        blk = xq.reshape(m, k // 256, 292)
        d = blk[:, :, :4].copy().view(np.float32).astype(np.float64)[..., 0]
        q = blk[:, :, 4:260].view(np.int8).astype(np.float64)
        xd = (q * d[..., None]).reshape(m, k)
    ref = xd @ wd.T
    y = oracle.mul_mat(qt, w, k, n, x).astype(np.float64)
    assert np.abs(y - ref).max() <= 1e-5 * np.abs(ref).max()
