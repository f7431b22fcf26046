"""Tensor-parallel partitioning (host side) over libcpq's split rules.

``split_state`` calls ``cpq_tp_split_state`` (include/cpq.h), the C++
restatement of crates/codpiece-model/src/split.rs. The helpers here turn a
split state into per-device index ranges and slice ggml-layout weights:

* Axis1 (column-parallel: q/k/v, gate/up) splits ne[1] = output rows, so a
  device owns whole rows of W.
* Axis0 (row-parallel: attn_output, ffn_down) splits ne[0] = K, so a device
  owns a range of quant blocks in every row; its partial products are summed
  by an allreduce. Granularity is always a multiple of the block size, so a
  block is never cut (split.rs:227-230).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

from ._lib import CpqHparams, lib

AXIS_0, AXIS_1, AXIS_2, MIRRORED, PARTIAL = 0, 1, 2, 3, 4


@dataclass(frozen=True)
class Hparams:
    """Model hyper-parameters the split rules read (qwen35.rs:45-148)."""

    n_layer: int
    n_embd: int
    n_head: int
    n_head_kv: int
    head_k: int
    head_v: int
    n_ff: int
    n_k_heads: int
    n_v_heads: int
    d_state: int
    d_inner: int
    full_attn_interval: int
    n_vocab: int
    q_has_gate: bool = True
    split_output: bool = False

    def c(self) -> CpqHparams:
        h = CpqHparams()
        for f in ("n_layer", "n_embd", "n_head", "n_head_kv", "head_k", "head_v", "n_ff", "n_k_heads",
                  "n_v_heads", "d_state", "d_inner", "full_attn_interval", "n_vocab"):
            setattr(h, f, int(getattr(self, f)))
        h.q_has_gate = 1 if self.q_has_gate else 0
        h.split_output = 1 if self.split_output else 0
        return h


# The production 27B hyper-parameters (split.rs:340-362).
HP_QWEN35_27B = Hparams(n_layer=64, n_embd=5120, n_head=24, n_head_kv=4, head_k=256, head_v=256, n_ff=17408,
                        n_k_heads=16, n_v_heads=48, d_state=128, d_inner=6144, full_attn_interval=4,
                        n_vocab=248320, q_has_gate=True)

# The benchmark's synthetic 27B-shaped stack: 64 attention-style layers (no
# recurrent layers, so every layer counts toward the same rotation), a plain q
# of 24 heads x 256 (no interleaved gate), vocab 151936.
HP_BENCH_27B = Hparams(n_layer=64, n_embd=5120, n_head=24, n_head_kv=4, head_k=256, head_v=256, n_ff=17408,
                       n_k_heads=16, n_v_heads=48, d_state=128, d_inner=6144, full_attn_interval=1,
                       n_vocab=151936, q_has_gate=False)


@dataclass
class SplitState:
    axis: int
    n_segments: int
    ne: list[int]   # ne[segment * n_devices + device]
    nr: list[int]

    def extents(self, n_devices: int, segment: int = 0) -> list[int]:
        return self.ne[segment * n_devices:(segment + 1) * n_devices]

    def ranges(self, n_devices: int) -> list[tuple[int, int]]:
        """[start, end) per device along the split axis (single-segment splits)."""
        if self.axis not in (AXIS_0, AXIS_1, AXIS_2):
            raise ValueError("mirrored tensors have no per-device range")
        if self.n_segments != 1:
            raise ValueError("multi-segment split: use extents() per segment")
        out, lo = [], 0
        for e in self.extents(n_devices):
            out.append((lo, lo + e))
            lo += e
        return out


def split_state(name: str, hp: Hparams, extent: int, blck: int, n_devices: int) -> SplitState:
    st = lib().cpq_tp_split_state(name.encode(), C.byref(hp.c()), int(extent), int(blck), int(n_devices))
    n = st.n_segments
    return SplitState(int(st.axis), int(n), [int(v) for v in st.ne[:max(n, 1) * n_devices]],
                      [int(v) for v in st.nr[:max(n, 1)]])


def layer_names(il: int) -> dict[str, str]:
    p = f"blk.{il}."
    return {k: p + v for k, v in (("q", "attn_q.weight"), ("k", "attn_k.weight"), ("v", "attn_v.weight"),
                                  ("o", "attn_output.weight"), ("gate", "ffn_gate.weight"),
                                  ("up", "ffn_up.weight"), ("down", "ffn_down.weight"))}


@dataclass
class LayerShards:
    """Per-device ranges of one layer: rows for column-parallel weights, K
    element ranges for row-parallel ones."""

    q: list[tuple[int, int]]
    k: list[tuple[int, int]]
    v: list[tuple[int, int]]
    o: list[tuple[int, int]]
    gate: list[tuple[int, int]]
    up: list[tuple[int, int]]
    down: list[tuple[int, int]]


def layer_shards(hp: Hparams, il: int, n_devices: int, blck: int = 256) -> LayerShards:
    names = layer_names(il)
    q_rows = hp.n_head * hp.head_k * (2 if hp.q_has_gate else 1)
    kv_rows = hp.n_head_kv * hp.head_k
    o_k = hp.n_head * hp.head_v
    r = {}
    for key, extent in (("q", q_rows), ("k", kv_rows), ("v", kv_rows), ("o", o_k), ("gate", hp.n_ff),
                        ("up", hp.n_ff), ("down", hp.n_ff)):
        st = split_state(names[key], hp, extent, blck, n_devices)
        r[key] = st.ranges(n_devices) if n_devices > 1 else [(0, extent)]
    sh = LayerShards(**r)
    if n_devices > 1:
        # the row-parallel K slices must line up with the column-parallel outputs that feed them
        assert sh.gate == sh.up == sh.down, "gate/up/down split mismatch"
        assert sh.q == sh.o, "q/attn_output split mismatch"
    return sh
