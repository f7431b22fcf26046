"""GPU: the persistent decode trunk (cpq_trunk_*) against the CPU restatement
and against the per-call stack.

Full-width layers of the 27B-shaped stack. At a reduced depth the trunk's
residual stream and the head on top of it are checked against the oracle;
at full depth (64 layers) the trunk is checked against the per-call path
(itself checked against the oracle layer by layer), a size-independent
property. Repeated runs (each run advances the trunk's epochs and must
reproduce the first run bit for bit) and a CUDA-graph replay are checked too.
"""
import numpy as np
import pytest

from tests.conftest import TOL, rel_err

pytestmark = pytest.mark.gpu


def _full_layer_weights(stack, il):
    lw = stack.layers[il]
    return {kind: (getattr(lw, kind).data.cpu().numpy(), getattr(lw, kind).n, getattr(lw, kind).k)
            for kind in ("q", "k", "v", "o", "gate", "up", "down")}


def _per_call(stack):
    """One step of the same stack through the per-call path (cpq_mul_mat_fused chain)."""
    trunk, stack.trunk = stack.trunk, None
    try:
        stack.step_body()
    finally:
        stack.trunk = trunk
    return stack.h_final.clone(), stack.logits.clone(), stack.tok.clone()


def test_trunk_matches_cpu_restatement(cuda, oracle):
    from codpiece_b200 import mul_mat as mm
    from codpiece_b200 import stack as st
    from codpiece_b200 import tp
    from oracle import stack_ref

    torch = cuda
    s = st.Stack(tp.HP_BENCH_27B, n_layer=2, m=1, seed=3, use_trunk=True)
    assert s.trunk.n_phases == 8
    h0 = torch.randn(1, 5120, generator=torch.Generator().manual_seed(7)).cuda()
    s.h.copy_(h0)
    s.step_body()
    torch.cuda.synchronize()
    assert mm.device_status(0) == 0
    h = h0.cpu().numpy()
    for il in range(2):
        h = stack_ref.layer_step(h, _full_layer_weights(s, il), 5120)
    logits, tok = stack_ref.head_step(h, s.head.data.cpu().numpy(), 5120, tp.HP_BENCH_27B.n_vocab)
    assert rel_err(s.h_final.cpu().numpy(), h) <= TOL
    assert rel_err(s.logits.cpu().numpy(), logits) <= TOL
    t = int(s.tok.cpu()[0])
    assert t == tok[0] or abs(logits[0, t] - logits[0, tok[0]]) <= TOL * np.abs(logits[0]).max()
    s.release()


@pytest.mark.parametrize("layers", [5, 64])
def test_trunk_matches_per_call_stack(cuda, layers):
    """Same weights, same input: the trunk and the per-call chain agree within the
    parity bound at full depth (gate/up run as 16-row pairs in the trunk, so
    their sums are added in another order)."""
    from codpiece_b200 import mul_mat as mm
    from codpiece_b200 import stack as st
    from codpiece_b200 import tp

    torch = cuda
    s = st.Stack(tp.HP_BENCH_27B, n_layer=layers, m=1, seed=9, use_trunk=True)
    h0 = torch.randn(1, 5120, generator=torch.Generator().manual_seed(2)).cuda()
    s.h.copy_(h0)
    h_ref, logits_ref, tok_ref = _per_call(s)
    s.h.copy_(h0)
    s.step_body()
    torch.cuda.synchronize()
    assert mm.device_status(0) == 0
    assert rel_err(s.h_final.cpu().numpy(), h_ref.cpu().numpy()) <= TOL
    assert rel_err(s.logits.cpu().numpy(), logits_ref.cpu().numpy()) <= TOL
    lr = logits_ref.cpu().numpy()[0]
    t, tr = int(s.tok.cpu()[0]), int(tok_ref.cpu()[0])
    assert t == tr or abs(lr[t] - lr[tr]) <= TOL * np.abs(lr).max()
    s.release()


def test_trunk_repeats_and_graph_replay(cuda):
    """Every run reproduces the first bit for bit (epochs advance between runs),
    also from a captured CUDA graph, and the device error word stays clear."""
    from codpiece_b200 import mul_mat as mm
    from codpiece_b200 import stack as st
    from codpiece_b200 import tp

    torch = cuda
    s = st.Stack(tp.HP_BENCH_27B, n_layer=3, m=1, seed=4, use_trunk=True)
    h0 = torch.randn(1, 5120, device="cuda")
    outs = []
    for _ in range(3):
        s.h.copy_(h0)
        s.step_body()
        torch.cuda.synchronize()
        outs.append((s.h_final.clone(), s.logits.clone(), s.tok.clone()))
    for o in outs[1:]:
        assert all(torch.equal(a, b) for a, b in zip(outs[0], o))
    s.h.copy_(h0)
    s.capture()
    for _ in range(2):
        s.h.copy_(h0)
        s.replay()
        torch.cuda.synchronize()
        assert torch.equal(s.h_final, outs[0][0]) and torch.equal(s.logits, outs[0][1])
    assert mm.device_status(0) == 0
    s.release()
