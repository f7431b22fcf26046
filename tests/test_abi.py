"""The C-ABI library loads and exports every entry point include/cpq.h declares.

CPU only: no compute call is made; host-side validation paths that return
before touching a device are exercised.
"""
import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "cpq.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(cpq_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def L():
    from codpiece_b200 import _lib, build
    build.build()
    return _lib.lib()


def test_header_declares_the_boundary():
    names = declared_functions()
    for must in ("cpq_mul_mat", "cpq_quantize_act", "cpq_tp_allreduce_f32", "cpq_tp_split_state", "cpq_last_error",
                 "cpq_init"):
        assert must in names


def test_every_declared_symbol_is_exported(L):
    from codpiece_b200 import _lib
    lib_path = _lib.LIB_PATH
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib_path)], capture_output=True, text=True, check=True)
    exported = set(re.findall(r"\b(cpq_[a-z0-9_]+)\b", out.stdout))
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, missing
    assert sorted(_lib.EXPORTED) == declared_functions()
    for n in declared_functions():
        assert hasattr(L, n)


def test_library_is_sm100a_only_and_links_no_nccl(L):
    from codpiece_b200 import _lib
    out = subprocess.run(["readelf", "-d", str(_lib.LIB_PATH)], capture_output=True, text=True, check=True).stdout
    assert "libnccl" not in out  # NCCL is dlopen'ed on first use
    assert "libtorch" not in out
    src = (ROOT / "codpiece_b200" / "build.py").read_text()
    assert "arch=compute_100a,code=sm_100a" in src


def test_version_and_status_strings(L):
    assert L.cpq_abi_version() == 1
    assert L.cpq_status_string(0) == b"success"
    assert L.cpq_status_string(2) == b"unsupported"


def test_validation_rejects_before_any_device_work(L):
    from codpiece_b200._lib import CpqTensor
    w = CpqTensor()
    w.type = 12
    w.ne[:] = [5120, 4, 1, 1]
    w.nb[:] = [144, 2880, 2880 * 4, 2880 * 4]
    w.data = 0x1000
    x = CpqTensor()
    x.type = 0
    x.ne[:] = [5120, 1, 1, 1]
    x.nb[:] = [4, 20480, 20480, 20480]
    x.data = 0x2000
    y = CpqTensor()
    y.type = 0
    y.ne[:] = [4, 1, 1, 1]
    y.nb[:] = [4, 16, 16, 16]
    y.data = 0x3000
    ws = C.c_void_p(0)
    bad = CpqTensor.from_buffer_copy(w)
    bad.type = 30  # BF16
    assert L.cpq_mul_mat_ws(C.byref(bad), C.byref(x), C.byref(y), ws, 0, None) == 2
    assert b"BF16" in L.cpq_last_error() or b"unknown" in L.cpq_last_error() or b"not Q4_K" in L.cpq_last_error()
    bad = CpqTensor.from_buffer_copy(w)
    bad.ne[3] = 2
    assert L.cpq_mul_mat_ws(C.byref(bad), C.byref(x), C.byref(y), ws, 0, None) == 2
    bady = CpqTensor.from_buffer_copy(y)
    bady.ne[0] = 5
    assert L.cpq_mul_mat_ws(C.byref(w), C.byref(x), C.byref(bady), ws, 0, None) == 1
    # a valid request without workspace reports it instead of launching
    assert L.cpq_mul_mat_ws(C.byref(w), C.byref(x), C.byref(y), ws, 0, None) == 3
    # empty batch: success, nothing launched
    x0 = CpqTensor.from_buffer_copy(x)
    x0.ne[1] = 0
    y0 = CpqTensor.from_buffer_copy(y)
    y0.ne[1] = 0
    assert L.cpq_mul_mat_ws(C.byref(w), C.byref(x0), C.byref(y0), ws, 0, None) == 0
    assert L.cpq_mul_mat_workspace_size(C.byref(w), C.byref(x)) >= 5120 + 20 * 4 + 320 * 2


def test_quantize_act_rejects_bad_shapes(L):
    assert L.cpq_quantize_act(12, None, None, 100, 1, None) == 1   # K not a multiple of 256
    assert L.cpq_quantize_act(30, None, None, 256, 1, None) == 2   # BF16 has no vec_dot_type here
    assert L.cpq_quantize_act(12, None, None, 256, 0, None) == 0   # empty


def test_plan_and_channel_arguments_are_validated_on_the_host(L):
    """cpq_decode_plan_create / cpq_tp_ar_create / cpq_tp_ar_add reject bad arguments before any device call."""
    from codpiece_b200 import _lib
    plan = C.c_void_p()
    assert L.cpq_decode_plan_create(None, 1, 0, C.byref(plan)) == 1          # no phases
    assert L.cpq_decode_plan_create((_lib.CpqDecodePhase * 1)(), 0, 0, C.byref(plan)) == 1
    assert L.cpq_decode_plan_create((_lib.CpqDecodePhase * 1)(), 1, 0, None) == 1
    ph = (_lib.CpqDecodePhase * 1)()
    ph[0].mode, ph[0].n_w = 7, 1                                                # bad prologue mode
    assert L.cpq_decode_plan_create(ph, 1, 0, C.byref(plan)) == 1
    ph[0].mode, ph[0].n_w = 0, 4                                                # too many weights
    assert L.cpq_decode_plan_create(ph, 1, 0, C.byref(plan)) == 1
    assert b"n_w" in L.cpq_last_error()
    L.cpq_decode_plan_destroy(None)                                             # NULL is ignored
    ar = C.c_void_p()
    h = C.create_string_buffer(64)
    assert L.cpq_tp_ar_create(0, 9, 0, 5120, C.byref(ar), h) == 1              # world > 8
    assert L.cpq_tp_ar_create(0, 2, 2, 5120, C.byref(ar), h) == 1              # rank out of range
    assert L.cpq_tp_ar_create(0, 2, 0, 0, C.byref(ar), h) == 1                 # n_max
    assert L.cpq_tp_ar_create(0, 2, 0, 5120, None, h) == 1
    assert L.cpq_tp_ar_connect(None, h) == 1
    assert L.cpq_tp_ar_add(None, None, None, 8, 1, None) == 1
    L.cpq_tp_ar_destroy(None)


def test_trunk_arguments_are_validated_on_the_host(L):
    """cpq_trunk_create rejects bad arguments before any device call."""
    from codpiece_b200 import _lib
    t = C.c_void_p()
    layers = (_lib.CpqTrunkLayer * 1)()
    assert L.cpq_trunk_create(None, 1, 5120, 1e-6, None, 0, C.byref(t)) == 1     # no layers
    assert L.cpq_trunk_create(layers, 0, 5120, 1e-6, None, 0, C.byref(t)) == 1
    assert L.cpq_trunk_create(layers, 1, 5120, 1e-6, None, 0, None) == 1
    assert L.cpq_trunk_create(layers, 1, 5000, 1e-6, None, 0, C.byref(t)) == 2   # n_embd not a multiple of 256
    assert L.cpq_trunk_create(layers, 1, 256 * 25, 1e-6, None, 0, C.byref(t)) == 2  # above the RMS image limit
    q = _lib.CpqTensor()
    q.type = 12
    q.ne[:] = [5120, 256, 1, 1]
    q.nb[:] = [144, 2880, 2880 * 256, 2880 * 256]
    q.data = 0x1000
    layers[0].q = C.pointer(q)                                                   # q without o
    assert L.cpq_trunk_create(layers, 1, 5120, 1e-6, None, 0, C.byref(t)) == 1
    assert b"q and o" in L.cpq_last_error()
    layers[0].q = None                                                           # no attention on one rank
    assert L.cpq_trunk_create(layers, 1, 5120, 1e-6, None, 0, C.byref(t)) == 1
    assert not t.value
    L.cpq_trunk_destroy(None)                                                    # NULL is ignored
    assert L.cpq_trunk_run(None, None, None, None) == 1


def test_wait_limit_is_validated_on_the_host(L):
    assert L.cpq_set_wait_limit_ns(-1, 1_000_000) == 1
    assert L.cpq_set_wait_limit_ns(0, 10) == 1                 # below 1 us
    assert L.cpq_set_wait_limit_ns(0, 61_000_000_000) == 1     # above 60 s
    assert b"wait limit" in L.cpq_last_error()
