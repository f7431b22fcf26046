"""GPU: a bounded device-side wait that nothing satisfies gives up with an
error status instead of hanging, and the context stays usable.

The wait limit is shortened to 5 ms (cpq_set_wait_limit_ns). A one-rank
all-reduce channel is asked for the sum of an all-reduce that no rank ever
produced (cpq_tp_ar_add): its words never carry the expected sequence
number, so the consumer's waits run out. The device error word then reports
kDevErrWaitTimeout through cpq_device_status (CPQ_ERR_DEVICE), clearing it
resets the scratch, and a valid product afterwards matches the oracle. No
fault, trap or endless loop is involved: the kernel gives up by itself.
"""
import ctypes as C

import pytest

from tests.conftest import TOL, rel_err

pytestmark = pytest.mark.gpu


def test_a_wait_nothing_satisfies_gives_up_with_an_error_status(cuda, oracle):
    from codpiece_b200 import _lib, synth
    from codpiece_b200 import mul_mat as mm

    torch = cuda
    L = _lib.lib()
    assert mm.device_status(0) == 0
    ch = mm.ArChannel(1, 0, 5120, 0)
    ch.connect([ch.ipc_handle])
    x = torch.randn(1, 5120, device="cuda")
    out = torch.empty_like(x)
    _lib.check(L.cpq_set_wait_limit_ns(0, 5_000_000), "cpq_set_wait_limit_ns")
    try:
        ch.add(x, out)                     # the sum of an all-reduce nobody produced
        torch.cuda.synchronize()           # returns: the waits gave up after 5 ms
        word = C.c_uint32(0)
        rc = L.cpq_device_status(0, C.byref(word), 1)
        assert rc == 7, L.cpq_last_error()  # CPQ_ERR_DEVICE
        assert word.value & 1               # kDevErrWaitTimeout
    finally:
        _lib.check(L.cpq_set_wait_limit_ns(0, 2_000_000_000), "cpq_set_wait_limit_ns")
        ch.close()
    assert mm.device_status(0) == 0        # cleared
    w_np, x_np = synth.config_inputs(synth.Q4_K, 512, 5120, 2, seed=5)
    w = mm.QTensor.from_numpy(mm.TYPE_Q4_K, 5120, 512, w_np)
    y = mm.mul_mat(w, torch.from_numpy(x_np).cuda()).cpu().numpy()
    assert rel_err(y, oracle.mul_mat(oracle.Q4_K, w_np, 5120, 512, x_np)) <= TOL
    assert mm.device_status(0) == 0
