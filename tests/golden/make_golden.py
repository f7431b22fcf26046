"""Generate the golden fixtures under tests/golden/ from gguf-py.

gguf-py (the ``gguf`` package, 0.19.0 in this image) is llama.cpp's own Python
implementation of the GGUF block formats. It is the only executable piece of
the reference's lineage available here (ggml itself is not vendored), so it
pins two things the oracle restates:

* dequantization of Q8_0, Q4_K and Q6_K blocks (gguf/quants.py
  ``dequantize_blocks``), and
* the portable Q8_0 quantizer (gguf/quants.py ``Q8_0.quantize_blocks``, which
  states it is bit-exact with ggml's ``quantize_row_q8_0_ref``).

Run from the repository root:  python tests/golden/make_golden.py
The fixtures are small (.npz) and committed; tests read them on any machine.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from codpiece_b200 import synth  # noqa: E402

OUT = Path(__file__).resolve().parent


def random_blocks(rng, qtype: int, nblocks: int) -> np.ndarray:
    """Uniform random block bytes with finite fp16 scales (every quant/scale bit pattern)."""
    size = {synth.Q8_0: 34, synth.Q4_K: 144, synth.Q6_K: 210}[qtype]
    b = rng.integers(0, 256, size=(nblocks, size), dtype=np.uint8)
    d_off = {synth.Q8_0: [0], synth.Q4_K: [0, 2], synth.Q6_K: [208]}[qtype]
    for off in d_off:
        d = (rng.standard_normal(nblocks) * 0.01).astype(np.float16)
        b[:, off:off + 2] = d.view(np.uint8).reshape(nblocks, 2)
    return b


def main() -> None:
    from gguf import GGMLQuantizationType as T
    from gguf import quants

    rng = np.random.default_rng(20261201)
    arrays = {}
    for name, qt, gt, k in (("q8_0", synth.Q8_0, T.Q8_0, 512), ("q4_K", synth.Q4_K, T.Q4_K, 512),
                            ("q6_K", synth.Q6_K, T.Q6_K, 512)):
        n = 6
        w = synth.weights(qt, n, k, seed=7)                       # BASELINE-distributed rows
        bsize = {synth.Q8_0: 34, synth.Q4_K: 144, synth.Q6_K: 210}[qt]
        r = random_blocks(rng, qt, 64)                             # arbitrary bit patterns
        blocks = np.concatenate([w.reshape(-1, bsize), r], axis=0)
        deq = quants.dequantize(blocks, gt).astype(np.float32)
        arrays[f"{name}_blocks"] = blocks
        arrays[f"{name}_deq"] = deq.reshape(blocks.shape[0], -1)

    # portable Q8_0 quantizer: normal data plus edge blocks (zeros, ties at .5, a
    # single non-zero element, negative-max blocks, subnormal-range scales)
    x = rng.standard_normal((8, 256)).astype(np.float32)
    edge = np.zeros((4, 256), np.float32)
    edge[1, :32] = np.arange(32, dtype=np.float32) - 15.5            # halves against amax 15.5
    edge[2, 40] = -3.0
    edge[2, 64:96] = np.linspace(-127, 127, 32, dtype=np.float32)
    edge[3, 96:128] = np.float32(1e-6) * (np.arange(32, dtype=np.float32) - 16)
    edge[3, 128:160] = 2.5
    edge[3, 160] = 127.0                                             # amax 127: d = 1, ties 2.5 exact
    xq = np.concatenate([x, edge], axis=0)
    arrays["q8_0_quant_x"] = xq
    arrays["q8_0_quant_portable"] = quants.quantize(xq, T.Q8_0).reshape(xq.shape[0], -1)

    np.savez_compressed(OUT / "gguf_py_fixtures.npz", **arrays)
    print("wrote", OUT / "gguf_py_fixtures.npz", {k: v.shape for k, v in arrays.items()})


if __name__ == "__main__":
    main()
