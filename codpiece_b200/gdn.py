"""Host-side mirror of ggml_gated_delta_net over libcpq (include/cpq.h
cpq_gated_delta_net).

The op of codpiece's GDN layers (crates/codpiece-model/src/qwen35.rs:2719:
``ggml_gated_delta_net(ctx, q, k, v, g, beta, state, k_snap)``). Tensors are
torch CUDA float32 in ggml's order reversed: q, k [n_seqs_qk, T, H_qk, S_v]
(rows contiguous; any other strides, e.g. views into the conv output as
qwen35.rs:2689-2706 makes them), v [n_seqs, T, H, S_v], g [n_seqs, T, H] or
[n_seqs, T, H, S_v], beta [n_seqs, T, H], state [n_seqs, H, S_v, S_v]
(column-major per head: state[s, h, col, i] = S[i][col]). There is no CPU
fallback.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._lib import CpqTensor, check, lib


def desc(t: torch.Tensor) -> CpqTensor:
    """ggml descriptor of a float32 CUDA tensor of up to 4 dimensions (ne = shape reversed)."""
    if t.dtype != torch.float32 or not t.is_cuda or t.dim() > 4:
        raise TypeError("expected a float32 CUDA tensor of at most 4 dimensions")
    shape = list(t.shape)[::-1] + [1] * (4 - t.dim())
    strides = [s * 4 for s in list(t.stride())[::-1]] + [0] * (4 - t.dim())
    for d in range(t.dim(), 4):
        strides[d] = strides[d - 1] * shape[d - 1] if d else 4
    d = CpqTensor()
    d.type = _lib.TYPE_F32
    d.ne[:] = shape
    d.nb[:] = strides
    d.data = t.data_ptr()
    return d


def state_slots(n_snap: int, t: int) -> int:
    return min(n_snap, t) if n_snap > 1 else 1


def gated_delta_net(q, k, v, g, beta, state, n_snap: int = 1, cache: torch.Tensor | None = None,
                    cache_slot_stride: int = 0, out: torch.Tensor | None = None, stream=None):
    """Returns (attn [n_seqs, T, H, S_v], states [slots, n_seqs, H, S_v, S_v]); the
    states are views of ``cache`` when one is given, else of the op's dst."""
    n_seqs, t, h, sv = v.shape
    if g.dim() == 3:  # [n_seqs, T, H] is ggml's [1, H, T, n_seqs]
        g = g.unsqueeze(-1)
    if beta.dim() == 3:
        beta = beta.unsqueeze(-1)
    n_attn = n_seqs * t * h * sv
    d_set = n_seqs * h * sv * sv
    slots = state_slots(n_snap, t)
    if out is None:
        out = torch.empty(n_attn + (0 if cache is not None else slots * d_set), dtype=torch.float32, device=v.device)
    s = stream if stream is not None else torch.cuda.current_stream()
    cache_ptr = C.c_void_p(cache.data_ptr()) if cache is not None else None
    check(lib().cpq_gated_delta_net(C.byref(desc(q)), C.byref(desc(k)), C.byref(desc(v)), C.byref(desc(g)),
                                    C.byref(desc(beta)), C.byref(desc(state)), C.byref(desc(out)), int(n_snap),
                                    cache_ptr, int(cache_slot_stride), C.c_void_p(s.cuda_stream)),
          "cpq_gated_delta_net")
    attn = out[:n_attn].view(n_seqs, t, h, sv)
    if cache is not None:
        stride = cache_slot_stride if slots > 1 else d_set
        states = torch.as_strided(cache, (slots, n_seqs, h, sv, sv), (stride, h * sv * sv, sv * sv, sv, 1))
    else:
        states = out[n_attn:n_attn + slots * d_set].view(slots, n_seqs, h, sv, sv)
    return attn, states
