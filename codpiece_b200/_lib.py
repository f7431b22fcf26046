"""ctypes binding of libcpq.so (the C ABI declared in include/cpq.h).

The product path has no fallback: if libcpq.so is missing or fails to load,
every operator raises. Nothing here imports or calls the CPU oracle.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libcpq.so"

TYPE_F32, TYPE_F16, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_K = 0, 1, 8, 12, 14, 15

STATUS = {
    0: "CPQ_SUCCESS",
    1: "CPQ_ERR_INVALID_ARG",
    2: "CPQ_ERR_UNSUPPORTED",
    3: "CPQ_ERR_NOT_INITIALIZED",
    4: "CPQ_ERR_WORKSPACE",
    5: "CPQ_ERR_CUDA",
    6: "CPQ_ERR_NCCL",
    7: "CPQ_ERR_DEVICE",
}

# Every symbol include/cpq.h declares (checked by tests/test_abi.py).
EXPORTED = [
    "cpq_init", "cpq_release", "cpq_mul_mat_workspace_size", "cpq_mul_mat", "cpq_mul_mat_ws",
    "cpq_mul_mat_multi", "cpq_mul_mat_fused", "cpq_mul_mat_noalloc", "cpq_quantize_act", "cpq_rms_norm",
    "cpq_swiglu", "cpq_add_inplace", "cpq_argmax", "cpq_gated_delta_net",
    "cpq_decode_plan_create", "cpq_decode_plan_run", "cpq_decode_plan_destroy",
    "cpq_trunk_create", "cpq_trunk_run", "cpq_trunk_phases", "cpq_trunk_destroy",
    "cpq_gguf_open", "cpq_gguf_close", "cpq_gguf_n_tensors", "cpq_gguf_find_tensor", "cpq_gguf_tensor_at",
    "cpq_gguf_get_u64", "cpq_gguf_get_str", "cpq_gguf_shard_shape", "cpq_gguf_read_shard", "cpq_gguf_load_shard",
    "cpq_tp_split_state", "cpq_tp_unique_id", "cpq_tp_comm_init", "cpq_tp_allreduce_f32", "cpq_tp_comm_check",
    "cpq_tp_comm_destroy", "cpq_tp_ar_create", "cpq_tp_ar_connect", "cpq_tp_ar_destroy", "cpq_tp_ar_add", "cpq_tp_ar_zero", "cpq_tp_ar_argmax", "cpq_mul_mat_fused_ar",
    "cpq_synth_weights", "cpq_device_status", "cpq_set_wait_limit_ns", "cpq_last_error", "cpq_status_string",
    "cpq_abi_version",
]


class CpqTensor(C.Structure):
    _fields_ = [("type", C.c_int32), ("ne", C.c_int64 * 4), ("nb", C.c_size_t * 4), ("data", C.c_void_p)]


class CpqHparams(C.Structure):
    _fields_ = [(n, C.c_int64) for n in (
        "n_layer", "n_embd", "n_head", "n_head_kv", "head_k", "head_v", "n_ff",
        "n_k_heads", "n_v_heads", "d_state", "d_inner", "full_attn_interval", "n_vocab")] + [
        ("q_has_gate", C.c_int32), ("split_output", C.c_int32)]


class CpqSplitState(C.Structure):
    _fields_ = [("axis", C.c_int32), ("n_segments", C.c_uint32), ("ne", C.c_int64 * 256), ("nr", C.c_uint32 * 16)]


class CpqPrologue(C.Structure):
    _fields_ = [("mode", C.c_int32), ("r", C.c_void_p), ("g", C.c_void_p), ("h_out", C.c_void_p), ("eps", C.c_float)]


class CpqDecodePhase(C.Structure):
    _fields_ = [("mode", C.c_int32), ("n_w", C.c_int32), ("x", C.c_void_p), ("r", C.c_void_p), ("g", C.c_void_p),
                ("h_out", C.c_void_p), ("eps", C.c_float), ("w", C.POINTER(CpqTensor) * 3), ("y", C.c_void_p * 3)]


class CpqTrunkLayer(C.Structure):
    _fields_ = [(n, C.POINTER(CpqTensor)) for n in ("q", "k", "v", "o", "gate", "up", "down")] + [
        ("attn_norm", C.c_void_p), ("ffn_norm", C.c_void_p), ("o_ranks", C.c_uint32)]


class CpqGgufTensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("type", C.c_int32), ("n_dims", C.c_int32), ("ne", C.c_int64 * 4),
                ("offset", C.c_uint64), ("bytes", C.c_uint64)]


PRO_NONE, PRO_RMS, PRO_SWIGLU = 0, 1, 2


class CpqError(RuntimeError):
    def __init__(self, status: int, where: str, msg: str):
        super().__init__(f"{where}: {STATUS.get(status, status)}: {msg}")
        self.status = status


_lib = None


def lib() -> C.CDLL:
    """Load libcpq.so once (raises if it is absent: there is no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is missing: run codpiece_b200.build.build() (nvcc, sm_100a)")
    L = C.CDLL(str(LIB_PATH))
    vp, i32, i64, sz, st = C.c_void_p, C.c_int32, C.c_int64, C.c_size_t, C.c_int
    P = C.POINTER
    sig = {
        "cpq_init": (st, [C.c_int, sz]),
        "cpq_release": (st, [C.c_int]),
        "cpq_mul_mat_workspace_size": (sz, [P(CpqTensor), P(CpqTensor)]),
        "cpq_mul_mat": (st, [P(CpqTensor), P(CpqTensor), P(CpqTensor), vp]),
        "cpq_mul_mat_ws": (st, [P(CpqTensor), P(CpqTensor), P(CpqTensor), vp, sz, vp]),
        "cpq_mul_mat_multi": (st, [P(P(CpqTensor)), P(P(CpqTensor)), C.c_int, P(CpqTensor), vp]),
        "cpq_mul_mat_fused": (st, [P(P(CpqTensor)), P(P(CpqTensor)), C.c_int, P(CpqTensor), P(CpqPrologue), vp]),
        "cpq_mul_mat_noalloc": (st, [P(CpqTensor), P(CpqTensor), P(CpqTensor), vp]),
        "cpq_quantize_act": (st, [i32, vp, vp, i64, i64, vp]),
        "cpq_rms_norm": (st, [vp, vp, vp, i64, i64, C.c_float, vp]),
        "cpq_swiglu": (st, [vp, vp, vp, i64, vp]),
        "cpq_add_inplace": (st, [vp, vp, i64, vp]),
        "cpq_argmax": (st, [vp, i64, i64, vp, vp]),
        "cpq_gated_delta_net": (st, [P(CpqTensor)] * 7 + [C.c_int32, vp, i64, vp]),
        "cpq_decode_plan_create": (st, [P(CpqDecodePhase), C.c_int, C.c_int, P(vp)]),
        "cpq_decode_plan_run": (st, [vp, vp]),
        "cpq_decode_plan_destroy": (None, [vp]),
        "cpq_trunk_create": (st, [P(CpqTrunkLayer), C.c_int, i64, C.c_float, vp, C.c_int, P(vp)]),
        "cpq_trunk_run": (st, [vp, vp, vp, vp]),
        "cpq_trunk_phases": (C.c_int, [vp]),
        "cpq_trunk_destroy": (None, [vp]),
        "cpq_gguf_open": (st, [C.c_char_p, P(vp)]),
        "cpq_gguf_close": (None, [vp]),
        "cpq_gguf_n_tensors": (i64, [vp]),
        "cpq_gguf_find_tensor": (i64, [vp, C.c_char_p]),
        "cpq_gguf_tensor_at": (st, [vp, i64, P(CpqGgufTensor)]),
        "cpq_gguf_get_u64": (st, [vp, C.c_char_p, P(C.c_uint64)]),
        "cpq_gguf_get_str": (st, [vp, C.c_char_p, P(C.c_char_p)]),
        "cpq_gguf_shard_shape": (st, [vp, i64, P(CpqSplitState), C.c_int, C.c_int, P(i64), P(i64), P(sz)]),
        "cpq_gguf_read_shard": (st, [vp, i64, P(CpqSplitState), C.c_int, C.c_int, vp, sz]),
        "cpq_gguf_load_shard": (st, [vp, i64, P(CpqSplitState), C.c_int, C.c_int, vp, sz]),
        "cpq_tp_split_state": (CpqSplitState, [C.c_char_p, P(CpqHparams), i64, i64, C.c_int]),
        "cpq_tp_unique_id": (st, [vp]),
        "cpq_tp_comm_init": (st, [P(vp), C.c_int, C.c_int, vp, C.c_int, C.c_int]),
        "cpq_tp_allreduce_f32": (st, [vp, vp, sz, vp]),
        "cpq_tp_comm_check": (st, [vp]),
        "cpq_tp_comm_destroy": (st, [vp, C.c_int]),
        "cpq_tp_ar_create": (st, [C.c_int, C.c_int, C.c_int, i64, P(vp), vp]),
        "cpq_tp_ar_connect": (st, [vp, vp]),
        "cpq_tp_ar_destroy": (None, [vp]),
        "cpq_tp_ar_add": (st, [vp, vp, vp, i64, i64, vp]),
        "cpq_tp_ar_zero": (st, [vp, i64, i64, vp]),
        "cpq_tp_ar_argmax": (st, [vp, vp, i64, i64, i64, i64, vp, vp]),
        "cpq_mul_mat_fused_ar": (st, [P(P(CpqTensor)), P(P(CpqTensor)), C.c_int, P(CpqTensor), P(CpqPrologue), vp, vp,
                                      vp]),
        "cpq_synth_weights": (st, [i32, vp, i64, i64, sz, C.c_uint64, i64, i64, vp]),
        "cpq_device_status": (st, [C.c_int, P(C.c_uint32), C.c_int]),
        "cpq_set_wait_limit_ns": (st, [C.c_int, C.c_uint64]),
        "cpq_last_error": (C.c_char_p, []),
        "cpq_status_string": (C.c_char_p, [C.c_int]),
        "cpq_abi_version": (C.c_int, []),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def check(status: int, where: str) -> None:
    if status != 0:
        raise CpqError(status, where, lib().cpq_last_error().decode(errors="replace"))
