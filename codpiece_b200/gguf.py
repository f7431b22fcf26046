"""GGUF files through libcpq (include/cpq.h cpq_gguf_*): the tensor directory,
metadata, and tensor-parallel shards placed on the device.

Mirrors codpiece's loading path: crates/codpiece-gguf/src/lib.rs:346-460
(GgufFile::open: header, KVs, directory, validity checks) and
crates/codpiece-model/src/lib.rs:128-311 (Weights::load: each tensor read
once and written to its device, sliced per device by the split rules of
split.rs under tensor parallelism). A shard is what cpq_tp_split_state gives
one device: whole rows for Axis1 (q/k/v/gate/up), K ranges of whole quant
blocks for Axis0 (attn_output/ffn_down), the whole tensor when mirrored.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import tp
from ._lib import CpqGgufTensor, CpqSplitState, check, lib

# ggml type id -> (elements per block, bytes per block) for the types on this path
BLOCKS = {0: (1, 4), 1: (1, 2), 8: (32, 34), 12: (256, 144), 14: (256, 210), 15: (256, 292)}


@dataclass
class TensorInfo:
    name: str
    type: int
    ne: tuple
    offset: int
    bytes: int


def _c_split(st: tp.SplitState | None, n_devices: int) -> CpqSplitState | None:
    if st is None:
        return None
    c = CpqSplitState()
    c.axis = st.axis
    c.n_segments = st.n_segments
    for i, v in enumerate(st.ne[:256]):
        c.ne[i] = v
    for i, v in enumerate(st.nr[:16]):
        c.nr[i] = v
    return c


class GgufFile:
    """An open GGUF file (header and directory read; tensor data read on demand)."""

    def __init__(self, path: str):
        self.handle = C.c_void_p()
        check(lib().cpq_gguf_open(str(path).encode(), C.byref(self.handle)), "cpq_gguf_open")
        self.tensors: list[TensorInfo] = []
        for i in range(lib().cpq_gguf_n_tensors(self.handle)):
            t = CpqGgufTensor()
            check(lib().cpq_gguf_tensor_at(self.handle, i, C.byref(t)), "cpq_gguf_tensor_at")
            self.tensors.append(TensorInfo(t.name.decode(), int(t.type), tuple(int(v) for v in t.ne[:max(t.n_dims, 1)]),
                                           int(t.offset), int(t.bytes)))
        self._index = {t.name: i for i, t in enumerate(self.tensors)}

    def index(self, name: str) -> int:
        if name not in self._index:
            raise KeyError(f"tensor {name} is not in the file")
        return self._index[name]

    def u64(self, key: str) -> int:
        v = C.c_uint64()
        check(lib().cpq_gguf_get_u64(self.handle, key.encode(), C.byref(v)), "cpq_gguf_get_u64")
        return int(v.value)

    def str(self, key: str) -> str:
        v = C.c_char_p()
        check(lib().cpq_gguf_get_str(self.handle, key.encode(), C.byref(v)), "cpq_gguf_get_str")
        return v.value.decode()

    def split_for(self, name: str, hp: tp.Hparams, n_devices: int) -> tp.SplitState | None:
        """The split state of a tensor by its name (split.rs rules); None on one device."""
        if n_devices <= 1:
            return None
        t = self.tensors[self.index(name)]
        blck = BLOCKS.get(t.type, (1, 1))[0]
        st = tp.split_state(name, hp, t.ne[0], blck, n_devices)
        if st.axis == tp.AXIS_1:
            st = tp.split_state(name, hp, t.ne[1] if len(t.ne) > 1 else 1, blck, n_devices)
        return st

    def shard_shape(self, name: str, split: tp.SplitState | None = None, n_devices: int = 1, device_index: int = 0):
        ne0, ne1, nbytes = C.c_int64(), C.c_int64(), C.c_size_t()
        cs = _c_split(split, n_devices)
        check(lib().cpq_gguf_shard_shape(self.handle, self.index(name), C.byref(cs) if cs else None, n_devices,
                                         device_index, C.byref(ne0), C.byref(ne1), C.byref(nbytes)),
              "cpq_gguf_shard_shape")
        return int(ne0.value), int(ne1.value), int(nbytes.value)

    def read_shard(self, name: str, split: tp.SplitState | None = None, n_devices: int = 1,
                   device_index: int = 0) -> np.ndarray:
        """Device device_index's shard as host bytes (uint8, dense rows)."""
        _, _, nbytes = self.shard_shape(name, split, n_devices, device_index)
        out = np.empty(nbytes, dtype=np.uint8)
        cs = _c_split(split, n_devices)
        check(lib().cpq_gguf_read_shard(self.handle, self.index(name), C.byref(cs) if cs else None, n_devices,
                                        device_index, out.ctypes.data_as(C.c_void_p), nbytes), "cpq_gguf_read_shard")
        return out

    def load_qtensor(self, name: str, split: tp.SplitState | None = None, n_devices: int = 1, device_index: int = 0,
                     device=None):
        """Device device_index's shard of a quantized weight, placed on `device`, as a mul_mat QTensor."""
        import torch

        from . import mul_mat as mm
        t = self.tensors[self.index(name)]
        ne0, ne1, nbytes = self.shard_shape(name, split, n_devices, device_index)
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        data = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        cs = _c_split(split, n_devices)
        with torch.cuda.device(dev):
            check(lib().cpq_gguf_load_shard(self.handle, self.index(name), C.byref(cs) if cs else None, n_devices,
                                            device_index, C.c_void_p(data.data_ptr()), nbytes), "cpq_gguf_load_shard")
        return mm.QTensor(t.type, ne0, ne1, data)

    def close(self) -> None:
        if self.handle:
            lib().cpq_gguf_close(self.handle)
            self.handle = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
