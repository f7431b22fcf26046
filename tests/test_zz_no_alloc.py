"""cpq_mul_mat_noalloc: the entry point for callers that cannot allocate.

Callers that run the product inside a host engine that owns all device
memory, or on a thread that must not take cudaMalloc's implicit device
synchronization, call cpq_mul_mat_noalloc: the same
Q4_K decode product as cpq_mul_mat, with its scratch in a static device array
every GPU using the library holds until exit, instead of a workspace. These checks call
it through the C ABI, twice in a row (the array keeps the previous call's
contents), and compare each result with cpq_mul_mat's within the parity
tolerance; sizes beyond the array's limits must be refused without a launch.

The file is named to be collected last, so a failure here cannot hide the
other tests; it also passes on its own in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

from tests.conftest import TOL, rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,k,m", [(17408, 5120, 1), (5120, 17408, 1), (17408, 5120, 2), (1031, 2048, 3)])
def test_noalloc_matches_cpq_mul_mat_on_two_calls_in_a_row(cuda, n, k, m):
    from codpiece_b200 import _lib
    from codpiece_b200 import mul_mat as mm

    torch = cuda
    L = _lib.lib()
    w = mm.synth_weights(mm.TYPE_Q4_K, k, n, seed=n + k)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):
        x = torch.randn(m, k, device="cuda", generator=torch.Generator(device="cuda").manual_seed(call))
        ref = mm.mul_mat(w, x).cpu().numpy()  # the existing entry point (library workspace)
        y = torch.full((m, n), float("nan"), device="cuda")
        rc = L.cpq_mul_mat_noalloc(C.byref(w.desc()), C.byref(mm.f32_desc(x)), C.byref(mm.f32_desc(y)), stream)
        assert rc == 0, L.cpq_last_error()
        torch.cuda.synchronize()
        got = y.cpu().numpy()
        assert np.isfinite(got).all()
        assert rel_err(got, ref) <= TOL
    assert mm.device_status(0) == 0


def test_noalloc_refuses_sizes_beyond_its_scratch(cuda):
    from codpiece_b200 import _lib
    from codpiece_b200 import mul_mat as mm

    torch = cuda
    L = _lib.lib()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    w = mm.synth_weights(mm.TYPE_Q4_K, 512, 64, seed=1)
    x = torch.randn(4, 512, device="cuda")  # M = 4 > 3
    y = torch.empty(4, 64, device="cuda")
    assert L.cpq_mul_mat_noalloc(C.byref(w.desc()), C.byref(mm.f32_desc(x)), C.byref(mm.f32_desc(y)), stream) == 2
    assert b"static scratch limit" in L.cpq_last_error()
    wq6 = mm.synth_weights(mm.TYPE_Q6_K, 512, 64, seed=2)
    x1 = torch.randn(1, 512, device="cuda")
    y1 = torch.empty(1, 64, device="cuda")
    assert L.cpq_mul_mat_noalloc(C.byref(wq6.desc()), C.byref(mm.f32_desc(x1)), C.byref(mm.f32_desc(y1)), stream) == 2
