"""GGUF reader and shard extraction (cpq_gguf_*), on the host.

Follows the reference reader's own tests (crates/codpiece-gguf/src/lib.rs:
462-560: a minimal file parses, a bad magic is refused, Q8_0 / Q6_K sizing)
and its validity checks (offsets aligned, in order, inside the data section),
plus the tensor-parallel shards the loader cuts by the split rules: Axis1
shards are whole rows, Axis0 shards K ranges of whole blocks, and both
recombine to the tensor.
"""
import numpy as np
import pytest

from tests.helpers import gguf_writer as gw

Q8_0, Q4_K, Q6_K, F32 = 8, 12, 14, 0
SIZES = {Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210), F32: (1, 4)}


def _hp():
    from codpiece_b200 import tp
    return tp.Hparams(n_layer=1, n_embd=512, n_head=2, n_head_kv=1, head_k=128, head_v=128, n_ff=1024, n_k_heads=2,
                      n_v_heads=2, d_state=16, d_inner=256, full_attn_interval=1, n_vocab=64, q_has_gate=False)


def _tensor(rng, name, ty, ne0, ne1):
    blk, bb = SIZES[ty]
    return (name, ty, (ne0, ne1), rng.integers(0, 256, size=ne0 // blk * bb * ne1, dtype=np.uint8).tobytes())


def _file(tmp_path, version=3, **kw):
    rng = np.random.default_rng(0)
    tensors = [_tensor(rng, "blk.0.attn_q.weight", Q8_0, 512, 256), _tensor(rng, "blk.0.ffn_gate.weight", Q4_K, 512, 1024),
               _tensor(rng, "blk.0.ffn_down.weight", Q4_K, 1024, 512), _tensor(rng, "output.weight", Q6_K, 512, 64),
               _tensor(rng, "output_norm.weight", F32, 512, 1)]
    kvs = [("general.architecture", gw.STRING, "qwen35"), ("qwen35.block_count", gw.U32, 1),
           ("general.alignment", gw.U32, 32), ("qwen35.rope.freq_base", gw.F32, 1e6),
           ("tokenizer.ggml.tokens", gw.ARRAY, (gw.STRING, ["<a>", "b", "cc"])),
           ("tokenizer.ggml.scores", gw.ARRAY, (gw.F32, [0.0, 1.0, 2.0]))]
    path = tmp_path / "m.gguf"
    gw.write_gguf(path, kvs, tensors, version=version, **kw)
    return path, tensors


@pytest.mark.parametrize("version", [1, 2, 3])
def test_directory_and_metadata(tmp_path, version):
    from codpiece_b200 import gguf
    path, tensors = _file(tmp_path, version=version)
    with gguf.GgufFile(path) as g:
        assert [t.name for t in g.tensors] == [t[0] for t in tensors]
        for info, (name, ty, ne, data) in zip(g.tensors, tensors):
            assert info.type == ty and info.ne == ne and info.bytes == len(data) and info.offset % 32 == 0
        assert g.str("general.architecture") == "qwen35"
        assert g.u64("qwen35.block_count") == 1
        raw = path.read_bytes()
        t = g.tensors[g.index("output.weight")]
        assert raw[t.offset:t.offset + t.bytes] == tensors[3][3]
        with pytest.raises(Exception):
            g.u64("qwen35.rope.freq_base")  # a float, not an integer
        with pytest.raises(KeyError):
            g.index("nope")


def test_reference_sizing():
    # crates/codpiece-gguf/src/lib.rs:546-550: Q8_0 is 34 B per 32, Q6_K 420 B per 512
    assert SIZES[Q8_0] == (32, 34) and 512 // SIZES[Q6_K][0] * SIZES[Q6_K][1] == 420


@pytest.mark.parametrize("bad", ["magic", "version", "past_end", "overlap", "misaligned", "truncated"])
def test_malformed_files_are_refused(tmp_path, bad):
    from codpiece_b200 import gguf
    from codpiece_b200._lib import CpqError
    rng = np.random.default_rng(1)
    ts = [_tensor(rng, "a", Q8_0, 64, 4), _tensor(rng, "b", Q8_0, 64, 4)]  # 272 B each
    path = tmp_path / "bad.gguf"
    if bad == "magic":
        path.write_bytes(b"NOPE0000")
    elif bad == "version":
        data = bytearray(gw.gguf_bytes([], ts))
        data[4:8] = (4).to_bytes(4, "little")
        path.write_bytes(bytes(data))
    elif bad == "past_end":
        gw.write_gguf(path, [], ts, offsets=[0, 4096])
        path.write_bytes(path.read_bytes()[:-(4096 - 288)])  # the second tensor runs past the file
    elif bad == "overlap":
        gw.write_gguf(path, [], ts, offsets=[0, 256])
    elif bad == "misaligned":
        gw.write_gguf(path, [], ts, offsets=[0, 304])
    else:
        path.write_bytes(gw.gguf_bytes([("k", gw.STRING, "x" * 100)], ts)[:40])
    with pytest.raises(CpqError):
        gguf.GgufFile(path)


def test_tensor_parallel_shards_recombine(tmp_path):
    """TP2 shards by the split rules: ffn_gate by rows (Axis1), ffn_down by K
    (Axis0, whole Q4_K blocks), the head mirrored; each recombines to the tensor."""
    from codpiece_b200 import gguf, tp
    path, tensors = _file(tmp_path)
    whole = {t[0]: np.frombuffer(t[3], dtype=np.uint8) for t in tensors}
    hp = _hp()
    with gguf.GgufFile(path) as g:
        for name in ("blk.0.ffn_gate.weight", "blk.0.ffn_down.weight", "output.weight"):
            st = g.split_for(name, hp, 2)
            shards = [g.read_shard(name, st, 2, d) for d in range(2)]
            info = g.tensors[g.index(name)]
            blk, bb = SIZES[info.type]
            row = info.ne[0] // blk * bb
            if st.axis == tp.AXIS_1:
                assert np.array_equal(np.concatenate(shards), whole[name])
                assert all(s.size % row == 0 and s.size for s in shards)
            elif st.axis == tp.AXIS_0:
                rows = info.ne[1]
                parts = [s.reshape(rows, -1) for s in shards]
                assert np.array_equal(np.concatenate(parts, axis=1), whole[name].reshape(rows, row))
                assert all(p.shape[1] % bb == 0 for p in parts)
            else:
                assert all(np.array_equal(s, whole[name]) for s in shards)
        assert g.split_for("blk.0.ffn_gate.weight", hp, 2).axis == tp.AXIS_1
        assert g.split_for("blk.0.ffn_down.weight", hp, 2).axis == tp.AXIS_0
        assert np.array_equal(g.read_shard("blk.0.attn_q.weight"), whole["blk.0.attn_q.weight"])
