"""Chunked-prefill parity (M > 16 tokens): the tcgen05 GEMM (Q4_K, Q8_0, Q6_K) against the CPU oracle.

The oracle is ggml-cpu's integer-exact Q4_K x Q8_K dot (ggml_vec_dot_q4_K_q8_K);
the tensor-core path multiplies fp16 images of both operands in fp32, so
the bar is the path's stated tolerance, max relative error 1e-3. At the
benchmark's full prefill shapes (M = 512 and 2048 tokens) the oracle checks
row slices at the start, middle (ragged offsets) and end of W, and every
output row is cross-checked for the first and last 16 tokens against the
M <= 16 integer path (itself pinned to the oracle).
"""
import numpy as np
import pytest

from codpiece_b200 import synth
from tests.conftest import TOL, rel_err
from tests.test_gpu_parity import edge_activations

pytestmark = pytest.mark.gpu


def _mm():
    from codpiece_b200 import mul_mat as mm
    return mm


@pytest.mark.parametrize("n,k,m", [
    (128, 256, 17),      # smallest tensor-core case: one tile, one superblock
    (7, 256, 33),        # fewer rows than one 128-row tile
    (129, 512, 256),     # one row past a tile, a full 256-token tile
    (1000, 1280, 257),   # two balanced token tiles of 144
    (384, 2048, 100),
    (256, 5120, 512),    # config-3 K, two token tiles
])
def test_prefill_matches_oracle(cuda, oracle, n, k, m):
    mm = _mm()
    w_np, x_np = synth.config_inputs(synth.Q4_K, n, k, m, seed=n + 7 * k + m)
    w = mm.QTensor.from_numpy(synth.Q4_K, k, n, w_np)
    y = mm.mul_mat(w, cuda.from_numpy(x_np).cuda()).cpu().numpy()
    ref = oracle.mul_mat(oracle.Q4_K, w_np, k, n, x_np)
    assert y.shape == ref.shape
    assert rel_err(y, ref) <= TOL
    assert mm.device_status(0) == 0


def test_prefill_edge_activations(cuda, oracle):
    """All-zero, tiny, tied and exact-127 Q8_K blocks in a 40-token batch."""
    mm = _mm()
    n, k, m = 640, 5120, 40
    w_np = synth.weights(synth.Q4_K, n, k, seed=41)
    x_np = edge_activations(m, k, seed=42)
    x_np[5] = 0.0                                     # a whole zero token
    w = mm.QTensor.from_numpy(synth.Q4_K, k, n, w_np)
    y = mm.mul_mat(w, cuda.from_numpy(x_np).cuda()).cpu().numpy()
    ref = oracle.mul_mat(oracle.Q4_K, w_np, k, n, x_np)
    assert np.all(y[5] == 0.0)
    assert rel_err(y, ref) <= TOL


@pytest.mark.parametrize("n,k,m", [(17408, 5120, 512), (5120, 17408, 512), (17408, 5120, 2048), (5120, 17408, 2048)])
def test_prefill_config3_shapes(cuda, oracle, n, k, m):
    """ffn_up/gate (17408 x 5120) and ffn_down (5120 x 17408) at M = 512 and 2048."""
    mm = _mm()
    w = mm.synth_weights(mm.TYPE_Q4_K, k, n, seed=n ^ k ^ m)
    x_np = synth.activations(m, k, seed=m + 3)
    x = cuda.from_numpy(x_np).cuda()
    y = mm.mul_mat(w, x)
    assert mm.device_status(0) == 0
    y_np = y.cpu().numpy()
    assert np.isfinite(y_np).all()
    w_np = w.data.cpu().numpy().reshape(n, -1)
    rows = np.r_[0:128, n // 2 - 37:n // 2 + 91, n - 128:n]
    ref = oracle.mul_mat(oracle.Q4_K, np.ascontiguousarray(w_np[rows]).reshape(-1), k, len(rows), x_np)
    assert rel_err(y_np[:, rows], ref) <= TOL
    # every row, first and last 16 tokens, against the integer M <= 16 path
    for sl in (slice(0, 16), slice(m - 16, m)):
        y16 = mm.mul_mat(w, x[sl].contiguous()).cpu().numpy()
        assert rel_err(y_np[sl], y16) <= TOL


def test_prefill_deterministic_and_strided_output(cuda):
    mm = _mm()
    n, k, m = 1000, 5120, 300
    w = mm.synth_weights(mm.TYPE_Q4_K, k, n, seed=9)
    x = cuda.randn(m, k, device="cuda")
    a = mm.mul_mat(w, x)
    b = mm.mul_mat(w, x)
    assert cuda.equal(a, b)
    big = cuda.full((m, n + 24), 7.0, device="cuda")
    (c,) = mm.mul_mat_fused([w], x, outs=[big[:, 8:8 + n]])
    assert cuda.equal(c, a)
    assert bool((big[:, :8] == 7.0).all()) and bool((big[:, 8 + n:] == 7.0).all())


def test_prefill_multi_equals_separate_calls(cuda):
    """q/k/v sharing one input: one fp16 activation image, one launch per weight, same bits."""
    mm = _mm()
    ws = [mm.synth_weights(mm.TYPE_Q4_K, 5120, n, seed=s) for s, n in ((1, 6144), (2, 1024), (3, 1024))]
    x = cuda.randn(96, 5120, device="cuda")
    for w, y in zip(ws, mm.mul_mat_multi(ws, x)):
        assert cuda.equal(y, mm.mul_mat(w, x))


# ---- Q8_0 and Q6_K weights on the same tensor-core GEMM (M > 16) ----------------------------
# Q8_0 activations are Q8_0-quantized (d = fp16(amax / 127)) before the fp16 image; Q6_K ones Q8_K.
# Q6_K rows reach shared memory through a tensor map whose rows are groups of L weight rows
# (L * row bytes a multiple of 16: L = 8 for one superblock per row, 4 for two, 2 for 20);
# N not a multiple of L (the (7, 256) and (130, 512) cases) runs on the integer GEMV instead,
# in passes of 16 tokens.

@pytest.mark.parametrize("qt,n,k,m", [
    (synth.Q8_0, 128, 256, 17),
    (synth.Q8_0, 7, 256, 33),
    (synth.Q8_0, 129, 512, 256),
    (synth.Q8_0, 1000, 1280, 257),
    (synth.Q8_0, 5120, 5120, 64),     # configs[0]'s matrix in a prefill chunk
    (synth.Q6_K, 128, 256, 17),
    (synth.Q6_K, 8, 256, 33),
    (synth.Q6_K, 7, 256, 33),
    (synth.Q6_K, 136, 512, 256),
    (synth.Q6_K, 130, 512, 40),
    (synth.Q6_K, 1000, 1280, 257),
    (synth.Q6_K, 640, 5120, 100),
])
def test_prefill_q8_0_q6_k_match_oracle(cuda, oracle, qt, n, k, m):
    mm = _mm()
    w_np, x_np = synth.config_inputs(qt, n, k, m, seed=n + 5 * k + m)
    w = mm.QTensor.from_numpy(qt, k, n, w_np)
    y = mm.mul_mat(w, cuda.from_numpy(x_np).cuda()).cpu().numpy()
    ref = oracle.mul_mat(qt, w_np, k, n, x_np)
    assert y.shape == ref.shape
    assert rel_err(y, ref) <= TOL
    assert mm.device_status(0) == 0


@pytest.mark.parametrize("qt", [synth.Q8_0, synth.Q6_K])
def test_prefill_q8_0_q6_k_edge_activations(cuda, oracle, qt):
    mm = _mm()
    n, k, m = 384, 5120, 40
    w_np = synth.weights(qt, n, k, seed=43)
    x_np = edge_activations(m, k, seed=44)
    x_np[3] = 0.0
    w = mm.QTensor.from_numpy(qt, k, n, w_np)
    y = mm.mul_mat(w, cuda.from_numpy(x_np).cuda()).cpu().numpy()
    assert np.all(y[3] == 0.0)
    assert rel_err(y, oracle.mul_mat(qt, w_np, k, n, x_np)) <= TOL


@pytest.mark.parametrize("qt,n,k,m", [(synth.Q8_0, 5120, 5120, 512), (synth.Q8_0, 17408, 5120, 512),
                                      (synth.Q6_K, 151936, 5120, 512), (synth.Q6_K, 5120, 17408, 300),
                                      # 64-token chunks: K split into ranges whose partials are added in order
                                      (synth.Q4_K, 5120, 17408, 64), (synth.Q8_0, 5120, 17408, 64),
                                      (synth.Q6_K, 5120, 5120, 64)])
def test_prefill_q8_0_q6_k_full_shapes(cuda, oracle, qt, n, k, m):
    """The Q8_0 trunk shapes and the Q6_K head at a 512-token chunk, and K-split 64-token chunks: oracle on row slices,
    every row for the first and last 16 tokens against the M <= 16 integer path."""
    mm = _mm()
    w = mm.synth_weights(qt, k, n, seed=n ^ k ^ m ^ qt)
    x_np = synth.activations(m, k, seed=m + 11)
    x = cuda.from_numpy(x_np).cuda()
    y = mm.mul_mat(w, x)
    assert mm.device_status(0) == 0
    y_np = y.cpu().numpy()
    assert np.isfinite(y_np).all()
    w_np = w.data.cpu().numpy().reshape(n, -1)
    rows = np.r_[0:128, n // 2 - 37:n // 2 + 91, n - 128:n]
    ref = oracle.mul_mat(qt, np.ascontiguousarray(w_np[rows]).reshape(-1), k, len(rows), x_np)
    assert rel_err(y_np[:, rows], ref) <= TOL
    for sl in (slice(0, 16), slice(m - 16, m)):
        y16 = mm.mul_mat(w, x[sl].contiguous()).cpu().numpy()
        assert rel_err(y_np[sl], y16) <= TOL
    del y, y_np


def test_prefill_q8_0_multi_equals_separate_calls(cuda):
    mm = _mm()
    ws = [mm.synth_weights(mm.TYPE_Q8_0, 5120, n, seed=s) for s, n in ((4, 6144), (5, 1024), (6, 1024))]
    x = cuda.randn(96, 5120, device="cuda")
    for w, y in zip(ws, mm.mul_mat_multi(ws, x)):
        assert cuda.equal(y, mm.mul_mat(w, x))
