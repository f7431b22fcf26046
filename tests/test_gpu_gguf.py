"""GGUF -> device: tensors loaded from a synthetic GGUF file, whole (TP1) and
as TP2 shards cut by the split rules, multiply like the oracle on the same bytes.

Axis1 shards (ffn_gate, attn_q) give the rows of the whole product; Axis0
shards (ffn_down) give partial sums over their K range that add up to it; the
mirrored head (output.weight) is the whole tensor on each device.
"""
import numpy as np
import pytest

from codpiece_b200 import synth
from tests.conftest import TOL, rel_err
from tests.helpers import gguf_writer as gw

pytestmark = pytest.mark.gpu

N_EMBD, N_FF, N_VOCAB = 2048, 4096, 1000


def _hp():
    from codpiece_b200 import tp
    return tp.Hparams(n_layer=1, n_embd=N_EMBD, n_head=16, n_head_kv=2, head_k=128, head_v=128, n_ff=N_FF,
                      n_k_heads=16, n_v_heads=16, d_state=128, d_inner=2048, full_attn_interval=1, n_vocab=N_VOCAB,
                      q_has_gate=False)


TENSORS = [("blk.0.attn_q.weight", synth.Q8_0, N_EMBD, N_EMBD), ("blk.0.ffn_gate.weight", synth.Q4_K, N_EMBD, N_FF),
           ("blk.0.ffn_down.weight", synth.Q4_K, N_FF, N_EMBD), ("output.weight", synth.Q6_K, N_EMBD, N_VOCAB)]


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    ts = [(name, qt, (k, n), synth.weights(qt, n, k, seed=i + 1).tobytes()) for i, (name, qt, k, n) in enumerate(TENSORS)]
    path = tmp_path_factory.mktemp("gguf") / "synthetic.gguf"
    gw.write_gguf(path, [("general.architecture", gw.STRING, "qwen35"), ("general.alignment", gw.U32, 64)], ts,
                  alignment=64)
    return path, {name: np.frombuffer(data, dtype=np.uint8) for name, _, _, data in ts}


@pytest.mark.parametrize("m", [1, 8])
def test_gguf_tp1_and_tp2_shards_match_oracle(cuda, oracle, model, m):
    from codpiece_b200 import gguf, tp
    from codpiece_b200 import mul_mat as mm
    path, whole = model
    hp = _hp()
    with gguf.GgufFile(path) as g:
        for name, qt, k, n in TENSORS:
            x_np = synth.activations(m, k, seed=k + n + m)
            ref = oracle.mul_mat(qt, whole[name], k, n, x_np)
            w1 = g.load_qtensor(name)
            assert (w1.qtype, w1.k, w1.n) == (qt, k, n)
            assert np.array_equal(w1.data.cpu().numpy(), whole[name])
            y1 = mm.mul_mat(w1, cuda.from_numpy(x_np).cuda()).cpu().numpy()
            assert rel_err(y1, ref) <= TOL, name

            st = g.split_for(name, hp, 2)
            shards = [g.load_qtensor(name, st, 2, d) for d in range(2)]
            if st.axis == tp.AXIS_1:
                r0 = 0
                for s in shards:
                    assert s.k == k
                    y = mm.mul_mat(s, cuda.from_numpy(x_np).cuda()).cpu().numpy()
                    assert rel_err(y, ref[:, r0:r0 + s.n]) <= TOL, name
                    r0 += s.n
                assert r0 == n
            elif st.axis == tp.AXIS_0:
                k0, total = 0, np.zeros_like(ref)
                for s in shards:
                    assert s.n == n
                    xs = np.ascontiguousarray(x_np[:, k0:k0 + s.k])
                    y = mm.mul_mat(s, cuda.from_numpy(xs).cuda()).cpu().numpy()
                    assert rel_err(y, oracle.mul_mat(qt, s.data.cpu().numpy(), s.k, n, xs)) <= TOL, name
                    total += y
                    k0 += s.k
                assert k0 == k
                # the K ranges hold whole Q8_K / Q8_0 blocks: only the fp32 summation order differs
                assert rel_err(total, ref) <= TOL, name
            else:
                for s in shards:
                    assert (s.k, s.n) == (k, n)
                    assert np.array_equal(s.data.cpu().numpy(), whole[name])
    assert mm.device_status(0) == 0
