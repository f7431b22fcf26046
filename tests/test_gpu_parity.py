"""GPU parity: libcpq through its C ABI against the CPU oracle.

Bar: activation re-quantization byte-identical to the oracle (Q8_K and the
x86 AVX2 Q8_0 semantics); fp32 outputs within max relative error 1e-3
(tests.conftest.TOL), at the benchmark configs' shapes and distributions
plus ragged and minimal edge cases.
"""
import ctypes as C

import numpy as np
import pytest

from codpiece_b200 import synth
from tests.conftest import TOL, rel_err

pytestmark = pytest.mark.gpu


def _mm():
    from codpiece_b200 import mul_mat as mm
    return mm


def edge_activations(m, k, seed):
    x = synth.activations(m, k, seed=seed)
    x[0, :256] = 0.0                                  # all-zero Q8_K block
    x[0, 256:512] = 0.0
    x[0, 300] = -2.0                                  # single element, negative max
    x[0, 512:768] = np.linspace(-127, 127, 256)       # exact -127/127 ends
    x[0, 768] = 127.0                                 # amax 127 -> ties at .5 exact
    x[0, 769:800] = np.arange(31) + 0.5 - 15
    if m > 1:
        x[1, 1024:1280] = 1e-30                       # tiny but non-zero
        x[1, 1280:1536] = -5.0                        # ties on magnitude: first wins
    return x.astype(np.float32)


@pytest.mark.parametrize("qt,m,k", [(synth.Q4_K, 16, 17408), (synth.Q6_K, 3, 5120), (synth.Q8_0, 5, 5120),
                                    (synth.Q8_0, 2, 17408)])
def test_activation_quantization_is_bit_exact(cuda, oracle, qt, m, k):
    mm = _mm()
    x = edge_activations(m, k, seed=5)
    got = mm.quantize_act(qt, cuda.from_numpy(x).cuda()).cpu().numpy()
    ref = oracle.quantize_act(qt, x)
    assert got.shape == ref.shape
    assert np.array_equal(got, ref), f"{int((got != ref).sum())} bytes differ"


CASES = [
    # (type, N, K, M) -- config 1, 2, 3 shapes and ragged/minimal ones
    (synth.Q8_0, 5120, 5120, 1),
    (synth.Q8_0, 5120, 5120, 4),
    (synth.Q4_K, 17408, 5120, 1),
    (synth.Q4_K, 5120, 17408, 1),
    (synth.Q4_K, 6144, 5120, 2),
    (synth.Q4_K, 1024, 5120, 4),
    (synth.Q4_K, 5120, 6144, 8),
    (synth.Q4_K, 6144, 5120, 16),
    (synth.Q4_K, 17408, 5120, 3),
    (synth.Q4_K, 7, 256, 1),
    (synth.Q4_K, 33, 1280, 5),
    (synth.Q6_K, 4099, 5120, 1),
    (synth.Q6_K, 4099, 5120, 8),
    (synth.Q6_K, 5, 768, 2),
    (synth.Q6_K, 1, 256, 1),
    # even N, K % 1024 == 0: the row-pair kernel (gemv_q6k.cuh), every token-count instance
    (synth.Q6_K, 4098, 5120, 1),
    (synth.Q6_K, 4098, 5120, 8),
    (synth.Q6_K, 6, 1024, 3),
    (synth.Q6_K, 2048, 2048, 5),
    (synth.Q6_K, 302, 3072, 2),
    (synth.Q6_K, 1000, 5120, 12),
    (synth.Q6_K, 300, 1536, 1),  # K % 1024 != 0: the generic kernel
    (synth.Q6_K, 4096, 5120, 16),  # int8 MMA tiles of 8 rows, tokens gid and gid + 8
    (synth.Q6_K, 4096, 5120, 9),
    (synth.Q6_K, 4104, 7680, 8),   # K at the MMA kernel's limit (30 superblocks)
    (synth.Q6_K, 64, 256, 2),      # one superblock: a single warp of the CTA has work
    (synth.Q6_K, 2048, 5120, 33),  # three weight passes of up to 16 tokens
    (synth.Q8_0, 9, 96, 7),
    (synth.Q8_0, 1001, 2080, 1),
    # even N, K % 256 == 0: the Q8_0 row-pair kernel (gemv_q6k.cuh); config 1's shape first
    (synth.Q8_0, 5120, 5120, 1),
    (synth.Q8_0, 1002, 2048, 3),
    (synth.Q8_0, 64, 256, 8),
    (synth.Q8_0, 1000, 5120, 12),
    # narrower rings when 8 warps x 2 stages do not fit: 6 x 2 (K = 6144 at M = 4 and 8, K = 8192
    # at M = 2) and 4 x 2 (K = 10240, the token quantized in-kernel)
    (synth.Q8_0, 6144, 6144, 4),
    (synth.Q8_0, 2000, 6144, 8),
    (synth.Q8_0, 1002, 8192, 2),
    (synth.Q8_0, 500, 10240, 1),
    (synth.Q4_K, 300, 2048, 40),
]


@pytest.mark.parametrize("qt,n,k,m", CASES)
def test_mul_mat_matches_oracle(cuda, oracle, qt, n, k, m):
    mm = _mm()
    w_np, x_np = synth.config_inputs(qt, n, k, m, seed=n + k + m)
    w = mm.QTensor.from_numpy(qt, k, n, w_np)
    y = mm.mul_mat(w, cuda.from_numpy(x_np).cuda()).cpu().numpy()
    ref = oracle.mul_mat(qt, w_np, k, n, x_np)
    assert y.shape == ref.shape
    assert rel_err(y, ref) <= TOL
    assert mm.device_status(0) == 0


def test_q6_K_head_full_size(cuda, oracle):
    """Config 3's Q6_K head [151936 x 5120] at M = 1, 4 and 16, weights made on the device."""
    mm = _mm()
    n, k = 151936, 5120
    w = mm.synth_weights(mm.TYPE_Q6_K, k, n, seed=77)
    w_np = w.data.cpu().numpy()
    x_np = synth.activations(16, k, seed=78)
    x = cuda.from_numpy(x_np).cuda()
    for m in (1, 4, 16):
        y = mm.mul_mat(w, x[:m]).cpu().numpy()
        assert rel_err(y, oracle.mul_mat(oracle.Q6_K, w_np, k, n, x_np[:m])) <= TOL


def test_multi_equals_separate_calls(cuda):
    mm = _mm()
    ws = [mm.synth_weights(mm.TYPE_Q4_K, 5120, n, seed=s) for s, n in ((1, 6144), (2, 1024), (3, 1024))]
    x = cuda.randn(4, 5120, device="cuda")
    multi = mm.mul_mat_multi(ws, x)
    for w, y in zip(ws, multi):
        # one launch over all three changes the stream-K split, hence the fp32 sum order
        assert rel_err(y.cpu().numpy(), mm.mul_mat(w, x).cpu().numpy()) <= 1e-6


def test_synth_shards_equal_slices_of_the_whole(cuda):
    mm = _mm()
    full = mm.synth_weights(mm.TYPE_Q4_K, 2048, 64, seed=5)
    rows = mm.synth_weights(mm.TYPE_Q4_K, 2048, 16, seed=5, row0=24)
    cols = mm.synth_weights(mm.TYPE_Q4_K, 768, 64, seed=5, blk0=3)
    f = full.data.view(64, -1)
    assert cuda.equal(rows.data.view(16, -1), f[24:40])
    assert cuda.equal(cols.data.view(64, -1), f[:, 3 * 144:6 * 144])
    q6 = mm.synth_weights(mm.TYPE_Q6_K, 512, 3, seed=6).data.cpu().numpy().reshape(3, 2, 210)
    d = q6[..., 208:210].copy().view(np.float16).astype(np.float32)
    assert np.isfinite(d).all() and (d >= 0).all() and d.max() < 0.1


def test_unsupported_and_invalid_are_reported_not_fatal(cuda):
    from codpiece_b200 import _lib
    mm = _mm()
    L = _lib.lib()
    w = mm.synth_weights(mm.TYPE_Q4_K, 512, 8, seed=1)
    x = cuda.randn(2, 512, device="cuda")
    y = cuda.empty(2, 8, device="cuda")
    wd, xd, yd = w.desc(), mm.f32_desc(x), mm.f32_desc(y)
    st = C.c_void_p(0)
    bad = w.desc()
    bad.type = 1  # F16 weight: not on this path
    assert L.cpq_mul_mat(C.byref(bad), C.byref(xd), C.byref(yd), st) == 2
    bad = w.desc()
    bad.ne[2] = 2  # 3-D
    assert L.cpq_mul_mat(C.byref(bad), C.byref(xd), C.byref(yd), st) == 2
    bad = w.desc()
    bad.ne[0] = 500  # not a block multiple
    assert L.cpq_mul_mat(C.byref(bad), C.byref(xd), C.byref(yd), st) == 1
    x2 = cuda.randn(2, 256, device="cuda")
    assert L.cpq_mul_mat(C.byref(wd), C.byref(mm.f32_desc(x2)), C.byref(yd), st) == 1  # K mismatch
    bad = w.desc()
    bad.data = w.data.data_ptr() + 8  # misaligned
    assert L.cpq_mul_mat(C.byref(bad), C.byref(xd), C.byref(yd), st) == 2
    assert L.cpq_mul_mat_ws(C.byref(wd), C.byref(xd), C.byref(yd), None, 0, st) == 3
    assert b"workspace" in L.cpq_last_error() or b"cpq_init" in L.cpq_last_error()
    # the RMS prologue's residual output may not overwrite its input
    xa = cuda.randn(8, 512, device="cuda")
    with pytest.raises(_lib.CpqError, match="alias"):
        mm.mul_mat_fused([w], xa, mode=mm.PRO_RMS, h_out=xa)
    # and a valid call still works afterwards
    assert L.cpq_mul_mat(C.byref(wd), C.byref(xd), C.byref(yd), C.c_void_p(cuda.cuda.current_stream().cuda_stream)) == 0
    cuda.cuda.synchronize()
    assert mm.device_status(0) == 0


def test_empty_batch_is_a_no_op(cuda):
    mm = _mm()
    w = mm.synth_weights(mm.TYPE_Q4_K, 512, 8, seed=1)
    y = mm.mul_mat(w, cuda.empty(0, 512, device="cuda"))
    assert y.shape == (0, 8)


def test_results_are_deterministic(cuda):
    mm = _mm()
    w = mm.synth_weights(mm.TYPE_Q4_K, 5120, 17408, seed=3)
    x = cuda.randn(3, 5120, device="cuda")
    a = mm.mul_mat(w, x)
    b = mm.mul_mat(w, x)
    assert cuda.equal(a, b)


def test_elementwise_ops_match_reference(cuda):
    from oracle import stack_ref
    mm = _mm()
    x_np = synth.activations(3, 5120, seed=12) * 7
    x = cuda.from_numpy(x_np).cuda()
    assert rel_err(mm.rms_norm(x).cpu().numpy(), stack_ref.rms_norm(x_np)) <= 1e-6
    g_np, u_np = synth.activations(2, 4096, seed=13) * 4, synth.activations(2, 4096, seed=14)
    got = mm.swiglu(cuda.from_numpy(g_np).cuda(), cuda.from_numpy(u_np).cuda()).cpu().numpy()
    assert rel_err(got, stack_ref.silu_mul(g_np, u_np)) <= 1e-6
    t = cuda.from_numpy(np.array([[1, 5, 5, 2], [7, 0, 7, 7]], np.float32)).cuda()
    assert mm.argmax(t).cpu().tolist() == [1, 0]


@pytest.mark.parametrize("m", [1, 3, 8, 13, 16, 64])
def test_fused_prologues_match_oracle(cuda, oracle, m):
    """cpq_mul_mat_fused: rms_norm(x + r) * g and silu(x) * r before quantization."""
    from oracle import stack_ref
    mm = _mm()
    k, n = 5120, 1024
    w_np = synth.weights(synth.Q4_K, n, k, seed=31)
    w = mm.QTensor.from_numpy(synth.Q4_K, k, n, w_np)
    x_np = synth.activations(m, k, seed=32) * 3
    r_np = synth.activations(m, k, seed=33)
    g_np = (1.0 + 0.1 * synth.activations(1, k, seed=34)[0]).astype(np.float32)
    x, r, g = (cuda.from_numpy(a).cuda() for a in (x_np, r_np, g_np))
    h_out = cuda.empty_like(x)
    (y,) = mm.mul_mat_fused([w], x, mode=mm.PRO_RMS, r=r, g=g, h_out=h_out)
    h_ref = (x_np + r_np).astype(np.float32)
    assert np.array_equal(h_out.cpu().numpy(), h_ref)
    xn = (stack_ref.rms_norm(h_ref) * g_np).astype(np.float32)
    assert rel_err(y.cpu().numpy(), oracle.mul_mat(oracle.Q4_K, w_np, k, n, xn)) <= TOL
    # SwiGLU before ffn_down (K = 17408)
    kd = 17408
    wd_np = synth.weights(synth.Q4_K, 512, kd, seed=35)
    wd = mm.QTensor.from_numpy(synth.Q4_K, kd, 512, wd_np)
    gt_np, up_np = synth.activations(m, kd, seed=36) * 2, synth.activations(m, kd, seed=37)
    (yd,) = mm.mul_mat_fused([wd], cuda.from_numpy(gt_np).cuda(), mode=mm.PRO_SWIGLU, r=cuda.from_numpy(up_np).cuda())
    act = stack_ref.silu_mul(gt_np, up_np)
    assert rel_err(yd.cpu().numpy(), oracle.mul_mat(oracle.Q4_K, wd_np, kd, 512, act)) <= TOL
