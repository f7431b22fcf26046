"""Host-side mirror of ggml's mul_mat operator surface over libcpq.

ggml's contract (crates/codpiece-ggml-sys/tests/smoke.rs:29-54): W has
ne = [K, N], X has ne = [K, M] (F32), and mul_mat(W, X) has ne = [N, M] with
Y[m, n] = dot(W row n, X row m). In torch terms X is a [M, K] float32 tensor
and Y a [M, N] float32 tensor; W is a :class:`QTensor` holding ggml's packed
row bytes on the device.

Every call goes through the C ABI of libcpq.so (include/cpq.h). There is no
CPU or PyTorch fallback: a missing library or an unsupported shape raises.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import PRO_NONE, PRO_RMS, PRO_SWIGLU, CpqPrologue, CpqTensor, CpqTrunkLayer, check, lib

TYPE_F32, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_K = (
    _lib.TYPE_F32, _lib.TYPE_Q8_0, _lib.TYPE_Q4_K, _lib.TYPE_Q6_K, _lib.TYPE_Q8_K)

# (elements per block, bytes per block): crates/codpiece-gguf/src/lib.rs:179-186
BLOCK = {TYPE_Q8_0: (32, 34), TYPE_Q4_K: (256, 144), TYPE_Q6_K: (256, 210), TYPE_Q8_K: (256, 292)}
TYPE_NAMES = {TYPE_Q8_0: "Q8_0", TYPE_Q4_K: "Q4_K", TYPE_Q6_K: "Q6_K", TYPE_Q8_K: "Q8_K", TYPE_F32: "F32"}
VEC_DOT_TYPE = {TYPE_Q4_K: TYPE_Q8_K, TYPE_Q6_K: TYPE_Q8_K, TYPE_Q8_0: TYPE_Q8_0}

DEFAULT_WORKSPACE = 64 << 20


def row_bytes(qtype: int, k: int) -> int:
    blk, size = BLOCK[qtype]
    if k % blk:
        raise ValueError(f"K={k} is not a multiple of the {TYPE_NAMES[qtype]} block ({blk})")
    return k // blk * size


@dataclass
class QTensor:
    """A quantized weight in ggml layout on a CUDA device.

    ``data`` is a uint8 CUDA tensor of N rows x row_stride bytes; ``k``/``n``
    are ggml's ne[0]/ne[1].
    """

    qtype: int
    k: int
    n: int
    data: torch.Tensor
    row_stride: int = 0

    def __post_init__(self):
        if self.row_stride == 0:
            self.row_stride = row_bytes(self.qtype, self.k)
        if self.data.dtype != torch.uint8 or not self.data.is_cuda:
            raise TypeError("QTensor.data must be a uint8 CUDA tensor")
        if self.data.numel() < self.n * self.row_stride:
            raise ValueError("QTensor.data is smaller than n * row_stride")

    @classmethod
    def from_numpy(cls, qtype: int, k: int, n: int, blocks: np.ndarray, device="cuda") -> "QTensor":
        """Upload packed ggml rows (uint8 [n, row_bytes]) to the device."""
        rb = row_bytes(qtype, k)
        arr = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(n, rb)
        return cls(qtype, k, n, torch.from_numpy(arr).to(device).reshape(-1), rb)

    @classmethod
    def empty(cls, qtype: int, k: int, n: int, device="cuda") -> "QTensor":
        rb = row_bytes(qtype, k)
        return cls(qtype, k, n, torch.empty(n * rb, dtype=torch.uint8, device=device), rb)

    @property
    def nbytes(self) -> int:
        return self.n * row_bytes(self.qtype, self.k)

    def desc(self) -> CpqTensor:
        d = CpqTensor()
        d.type = self.qtype
        d.ne[:] = [self.k, self.n, 1, 1]
        bs = BLOCK[self.qtype][1]
        d.nb[:] = [bs, self.row_stride, self.row_stride * self.n, self.row_stride * self.n]
        d.data = self.data.data_ptr()
        return d


def f32_desc(t: torch.Tensor) -> CpqTensor:
    """ggml descriptor of a [M, K] float32 tensor (ne = [K, M])."""
    if t.dtype != torch.float32 or t.dim() != 2 or t.stride(1) != 1:
        raise TypeError("expected a 2-D float32 tensor with contiguous rows")
    d = CpqTensor()
    d.type = TYPE_F32
    m, k = t.shape
    d.ne[:] = [k, m, 1, 1]
    d.nb[:] = [4, t.stride(0) * 4, t.stride(0) * 4 * m, t.stride(0) * 4 * m]
    d.data = t.data_ptr()
    return d


def _stream(stream) -> C.c_void_p:
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


_ws_bytes: dict[int, int] = {}


def init(device: int | None = None, workspace_bytes: int = DEFAULT_WORKSPACE) -> None:
    """Allocate (or grow) libcpq's per-device workspace. Call before graph capture."""
    dev = torch.cuda.current_device() if device is None else int(device)
    if _ws_bytes.get(dev, 0) >= workspace_bytes:
        return
    check(lib().cpq_init(dev, workspace_bytes), "cpq_init")
    _ws_bytes[dev] = workspace_bytes


def _ensure_workspace(w: QTensor, x: torch.Tensor) -> None:
    dev = x.device.index if x.device.index is not None else torch.cuda.current_device()
    need = lib().cpq_mul_mat_workspace_size(C.byref(w.desc()), C.byref(f32_desc(x)))
    if _ws_bytes.get(dev, 0) < need:
        init(dev, max(need, DEFAULT_WORKSPACE))


def mul_mat(w: QTensor, x: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """ggml_mul_mat(W, X) executed on the GPU: returns Y [M, N] float32."""
    if x.dim() == 1:
        x = x.unsqueeze(0)
    if out is None:
        out = torch.empty(x.shape[0], w.n, dtype=torch.float32, device=x.device)
    _ensure_workspace(w, x)
    wd, xd, yd = w.desc(), f32_desc(x), f32_desc(out)
    check(lib().cpq_mul_mat(C.byref(wd), C.byref(xd), C.byref(yd), _stream(stream)), "cpq_mul_mat")
    return out


def mul_mat_multi(ws: list[QTensor], x: torch.Tensor, outs: list[torch.Tensor] | None = None,
                  stream=None) -> list[torch.Tensor]:
    """Several weights sharing one input (q/k/v, gate/up): one quantization, one launch."""
    if x.dim() == 1:
        x = x.unsqueeze(0)
    if outs is None:
        outs = [torch.empty(x.shape[0], w.n, dtype=torch.float32, device=x.device) for w in ws]
    _ensure_workspace(ws[0], x)
    wds = [w.desc() for w in ws]
    yds = [f32_desc(o) for o in outs]
    xd = f32_desc(x)
    n = len(ws)
    warr = (C.POINTER(CpqTensor) * n)(*[C.pointer(d) for d in wds])
    yarr = (C.POINTER(CpqTensor) * n)(*[C.pointer(d) for d in yds])
    check(lib().cpq_mul_mat_multi(warr, yarr, n, C.byref(xd), _stream(stream)), "cpq_mul_mat_multi")
    return outs


def _ptr(t):
    return None if t is None else t.data_ptr()


def mul_mat_fused(ws: list[QTensor], x: torch.Tensor, outs: list[torch.Tensor] | None = None, *, mode: int = PRO_NONE,
                  r: torch.Tensor | None = None, g: torch.Tensor | None = None, h_out: torch.Tensor | None = None,
                  eps: float = 1e-6, stream=None, r_ar: "ArChannel | None" = None,
                  y_ar: "ArChannel | None" = None) -> list[torch.Tensor]:
    """Y_i = W_i x quantize(f(X)) with f the fused prologue (include/cpq.h cpq_prologue):
    PRO_RMS: rms_norm(X + r) * g (X + r stored to h_out when given); PRO_SWIGLU: silu(X) * r.

    With a fused-allreduce channel (cpq_mul_mat_fused_ar): y_ar all-reduces
    Y_0 through the channel instead of storing it; r_ar makes the RMS
    residual r the sum over ranks of the channel's last all-reduced value."""
    if x.dim() == 1:
        x = x.unsqueeze(0)
    if outs is None:
        outs = [torch.empty(x.shape[0], w.n, dtype=torch.float32, device=x.device) for w in ws]
    _ensure_workspace(ws[0], x)
    wds = [w.desc() for w in ws]
    yds = [f32_desc(o) for o in outs]
    xd = f32_desc(x)
    n = len(ws)
    warr = (C.POINTER(CpqTensor) * n)(*[C.pointer(d) for d in wds])
    yarr = (C.POINTER(CpqTensor) * n)(*[C.pointer(d) for d in yds])
    pro = CpqPrologue(mode, _ptr(r), _ptr(g), _ptr(h_out), eps)
    if r_ar is None and y_ar is None:
        check(lib().cpq_mul_mat_fused(warr, yarr, n, C.byref(xd), C.byref(pro), _stream(stream)), "cpq_mul_mat_fused")
    else:
        check(lib().cpq_mul_mat_fused_ar(warr, yarr, n, C.byref(xd), C.byref(pro),
                                         r_ar.handle if r_ar is not None else None,
                                         y_ar.handle if y_ar is not None else None, _stream(stream)),
              "cpq_mul_mat_fused_ar")
    return outs


def quantize_act(wtype: int, x: torch.Tensor, stream=None) -> torch.Tensor:
    """ggml-cpu's re-quantization of X rows to W's vec_dot_type, as raw ggml block bytes."""
    if x.dim() == 1:
        x = x.unsqueeze(0)
    x = x.contiguous()
    m, k = x.shape
    vt = VEC_DOT_TYPE[wtype]
    out = torch.empty(m * row_bytes(vt, k), dtype=torch.uint8, device=x.device)
    check(lib().cpq_quantize_act(wtype, C.c_void_p(x.data_ptr()), C.c_void_p(out.data_ptr()), k, m, _stream(stream)),
          "cpq_quantize_act")
    return out.view(m, -1)


def rms_norm(x: torch.Tensor, g: torch.Tensor | None = None, eps: float = 1e-6, out=None, stream=None):
    m, k = x.shape
    out = torch.empty_like(x) if out is None else out
    check(lib().cpq_rms_norm(C.c_void_p(x.data_ptr()), C.c_void_p(g.data_ptr() if g is not None else 0),
                             C.c_void_p(out.data_ptr()), k, m, eps, _stream(stream)), "cpq_rms_norm")
    return out


def swiglu(gate: torch.Tensor, up: torch.Tensor, out=None, stream=None):
    out = torch.empty_like(gate) if out is None else out
    check(lib().cpq_swiglu(C.c_void_p(gate.data_ptr()), C.c_void_p(up.data_ptr()), C.c_void_p(out.data_ptr()),
                           gate.numel(), _stream(stream)), "cpq_swiglu")
    return out


def add_(y: torch.Tensor, x: torch.Tensor, stream=None):
    check(lib().cpq_add_inplace(C.c_void_p(y.data_ptr()), C.c_void_p(x.data_ptr()), y.numel(), _stream(stream)),
          "cpq_add_inplace")
    return y


def argmax(x: torch.Tensor, out=None, stream=None) -> torch.Tensor:
    m, n = x.shape
    out = torch.empty(m, dtype=torch.int32, device=x.device) if out is None else out
    check(lib().cpq_argmax(C.c_void_p(x.data_ptr()), n, m, C.c_void_p(out.data_ptr()), _stream(stream)), "cpq_argmax")
    return out


def synth_weights(qtype: int, k: int, n: int, seed: int, row0: int = 0, blk0: int = 0, k_blocks: int | None = None,
                  device="cuda", stream=None) -> QTensor:
    """Seeded synthetic weight rows [row0, row0+n) x blocks [blk0, blk0+k_blocks) generated on the device."""
    blk, _ = BLOCK[qtype]
    nblk = k // blk if k_blocks is None else k_blocks
    w = QTensor.empty(qtype, nblk * blk, n, device=device)
    check(lib().cpq_synth_weights(qtype, C.c_void_p(w.data.data_ptr()), n, nblk, w.row_stride, seed, row0, blk0,
                                  _stream(stream)), "cpq_synth_weights")
    return w


def device_status(device: int = 0, clear: bool = True) -> int:
    word = C.c_uint32(0)
    rc = lib().cpq_device_status(device, C.byref(word), 1 if clear else 0)
    if rc not in (0, 7):
        check(rc, "cpq_device_status")
    return word.value


@dataclass
class DecodePhase:
    """One phase of a decode plan (include/cpq.h cpq_decode_phase): up to three
    Q4_K weights applied to one input vector through a fused prologue."""

    weights: list
    outs: list
    x: torch.Tensor
    mode: int = PRO_NONE
    r: torch.Tensor | None = None
    g: torch.Tensor | None = None
    h_out: torch.Tensor | None = None
    eps: float = 1e-6


class DecodePlan:
    """A chain of decode phases run as one persistent kernel (cpq_decode_plan_*).

    The plan bakes in the device pointers of the weights and buffers: keep
    them alive (this object holds references) and reuse the same buffers
    every step. run() is capturable in a CUDA graph."""

    def __init__(self, phases: list[DecodePhase], device: int | None = None):
        dev = torch.cuda.current_device() if device is None else device
        self._keep = phases
        self._descs = []
        arr = (_lib.CpqDecodePhase * len(phases))()
        for i, ph in enumerate(phases):
            if not 1 <= len(ph.weights) <= 3 or len(ph.outs) != len(ph.weights):
                raise ValueError("a decode phase has 1..3 weights and one output per weight")
            c = arr[i]
            c.mode, c.n_w = ph.mode, len(ph.weights)
            c.x, c.r, c.g, c.h_out, c.eps = _ptr(ph.x), _ptr(ph.r), _ptr(ph.g), _ptr(ph.h_out), ph.eps
            for j, (w, y) in enumerate(zip(ph.weights, ph.outs)):
                if y.numel() < w.n or not y.is_contiguous():
                    raise ValueError("decode phase output must be a contiguous vector of N floats")
                d = w.desc()
                self._descs.append(d)
                c.w[j] = C.pointer(d)
                c.y[j] = y.data_ptr()
        self._arr = arr
        self.handle = C.c_void_p()
        check(lib().cpq_decode_plan_create(arr, len(phases), dev, C.byref(self.handle)), "cpq_decode_plan_create")
        self.n_phases = len(phases)

    def run(self, stream=None) -> None:
        check(lib().cpq_decode_plan_run(self.handle, _stream(stream)), "cpq_decode_plan_run")

    def close(self) -> None:
        if self.handle:
            lib().cpq_decode_plan_destroy(self.handle)
            self.handle = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass


@dataclass
class TrunkLayer:
    """One layer of a decode trunk (include/cpq.h cpq_trunk_layer): this rank's
    Q4_K shards; q and o are None on a rank without attention rows in the
    layer (tensor parallel), o_ranks the bit mask of ranks that hold them
    (0 = all)."""

    q: QTensor | None
    k: QTensor | None
    v: QTensor | None
    o: QTensor | None
    gate: QTensor
    up: QTensor
    down: QTensor
    attn_norm: torch.Tensor | None = None
    ffn_norm: torch.Tensor | None = None
    o_ranks: int = 0


class Trunk:
    """A rank's whole decode trunk as one persistent kernel (cpq_trunk_*).

    run(h_in, h_out) is one decode step (M = 1): h_out receives the residual
    stream after the last layer. Pointers are baked in at creation: keep the
    weights alive (this object holds references). Capturable in a CUDA graph."""

    def __init__(self, layers: list[TrunkLayer], n_embd: int, eps: float = 1e-6, ar: "ArChannel | None" = None,
                 device: int | None = None):
        dev = torch.cuda.current_device() if device is None else device
        self._keep = layers
        self._descs = []
        arr = (CpqTrunkLayer * len(layers))()
        for i, L in enumerate(layers):
            c = arr[i]
            for name in ("q", "k", "v", "o", "gate", "up", "down"):
                w = getattr(L, name)
                if w is not None:
                    d = w.desc()
                    self._descs.append(d)
                    setattr(c, name, C.pointer(d))
            c.attn_norm = _ptr(L.attn_norm)
            c.ffn_norm = _ptr(L.ffn_norm)
            c.o_ranks = int(L.o_ranks)
        self._arr = arr
        self.ar = ar
        self.handle = C.c_void_p()
        check(lib().cpq_trunk_create(arr, len(layers), int(n_embd), float(eps), ar.handle if ar is not None else None,
                                     dev, C.byref(self.handle)), "cpq_trunk_create")
        self.n_phases = int(lib().cpq_trunk_phases(self.handle))

    def run(self, h_in: torch.Tensor, h_out: torch.Tensor, stream=None) -> torch.Tensor:
        check(lib().cpq_trunk_run(self.handle, C.c_void_p(h_in.data_ptr()), C.c_void_p(h_out.data_ptr()),
                                  _stream(stream)), "cpq_trunk_run")
        return h_out

    def close(self) -> None:
        if self.handle:
            lib().cpq_trunk_destroy(self.handle)
            self.handle = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass


class ArChannel:
    """A fused-allreduce channel over NVLink peer memory (include/cpq.h cpq_tp_ar_*).

    Create one per rank, exchange the 64-byte IPC handles (``handle``) in rank
    order (e.g. torch.distributed.all_gather_object), then connect()."""

    def __init__(self, world: int, rank: int, n_max: int, device: int | None = None):
        dev = torch.cuda.current_device() if device is None else device
        self.handle = C.c_void_p()
        buf = C.create_string_buffer(64)
        check(lib().cpq_tp_ar_create(dev, world, rank, n_max, C.byref(self.handle), buf), "cpq_tp_ar_create")
        self.ipc_handle = buf.raw
        self.world, self.rank = world, rank

    def connect(self, handles: list[bytes]) -> None:
        if len(handles) != self.world or any(len(h) != 64 for h in handles):
            raise ValueError("one 64-byte handle per rank expected")
        blob = C.create_string_buffer(b"".join(handles), 64 * self.world)
        check(lib().cpq_tp_ar_connect(self.handle, blob), "cpq_tp_ar_connect")

    def add(self, x: torch.Tensor, out: torch.Tensor, stream=None) -> torch.Tensor:
        """out = x + the sum over ranks of the last value all-reduced through the channel."""
        m, k = x.shape
        check(lib().cpq_tp_ar_add(self.handle, C.c_void_p(x.data_ptr()), C.c_void_p(out.data_ptr()), k, m,
                                  _stream(stream)), "cpq_tp_ar_add")
        return out

    def zero(self, n: int, m: int, stream=None) -> None:
        """Contribute zeros (m tokens x n) to the next all-reduce (a rank without rows of it)."""
        check(lib().cpq_tp_ar_zero(self.handle, n, m, _stream(stream)), "cpq_tp_ar_zero")

    def argmax(self, logits: torch.Tensor, row0: int, out: torch.Tensor, stream=None) -> torch.Tensor:
        """Greedy tokens when the vocabulary is split across ranks: logits [m, n] are this rank's
        rows row0 .. row0 + n - 1; out[m] (int32) = the global argmax (lowest index on ties)."""
        m, n = logits.shape
        check(lib().cpq_tp_ar_argmax(self.handle, C.c_void_p(logits.data_ptr()), n, m, logits.stride(0), int(row0),
                                     C.c_void_p(out.data_ptr()), _stream(stream)), "cpq_tp_ar_argmax")
        return out

    def close(self) -> None:
        if self.handle:
            lib().cpq_tp_ar_destroy(self.handle)
            self.handle = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass
