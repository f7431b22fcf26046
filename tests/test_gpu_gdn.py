"""GPU parity of cpq_gated_delta_net against the CPU oracle (oracle/cpq_oracle_gdn.c).

Cases follow the GDN layers of the 27B trunk (S_v 128, 48 v heads over 16
q/k heads, q/k/v as views into the conv output, qwen35.rs:2689-2719): decode
(T = 1), speculative verify with rollback snapshots (T = 8, K = 8), a
prefill chunk longer than the kernel's token staging (T = 37), batched
sequences, the per-row decay form, the small head sizes, the cache output
and an in-place state update. Bar: max |gpu - oracle| / max |oracle| <= 1e-3
(tests.conftest.TOL) for the attention rows and every state slot.
"""
import numpy as np
import pytest

from tests.conftest import TOL, rel_err

pytestmark = pytest.mark.gpu


def _inputs(rng, n_seqs, t, h, h_qk, sv, kda, n_seqs_qk=None):
    n_seqs_qk = n_seqs_qk or n_seqs
    q = rng.standard_normal((n_seqs_qk, t, h_qk, sv)).astype(np.float32)
    k = rng.standard_normal((n_seqs_qk, t, h_qk, sv)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((n_seqs, t, h, sv)).astype(np.float32)
    g = -rng.uniform(0.01, 2.0, size=(n_seqs, t, h, sv) if kda else (n_seqs, t, h)).astype(np.float32)
    beta = rng.uniform(0.0, 1.0, size=(n_seqs, t, h)).astype(np.float32)
    state = (0.1 * rng.standard_normal((n_seqs, h, sv, sv))).astype(np.float32)
    return q, k, v, g, beta, state


def _check(torch, got, ref):
    attn, states = got
    ref_attn, ref_states = ref
    assert tuple(attn.shape) == ref_attn.shape and tuple(states.shape) == ref_states.shape
    assert rel_err(attn.cpu().numpy(), ref_attn) <= TOL
    for j in range(ref_states.shape[0]):
        assert rel_err(states[j].cpu().numpy(), ref_states[j]) <= TOL, f"slot {j}"


@pytest.mark.parametrize("t,n_snap", [(1, 1), (8, 8), (8, 3), (37, 4), (2, 1)])
def test_trunk_gdn_layer_from_conv_views(cuda, oracle, t, n_snap):
    """q, k, v as strided views into one [T, conv_dim] conv output, as the GDN layer makes them."""
    from codpiece_b200 import gdn
    torch = cuda
    sv, h, h_qk = 128, 48, 16
    key_dim = sv * h_qk
    rng = np.random.default_rng(t * 10 + n_snap)
    q, k, v, g, beta, state = _inputs(rng, 1, t, h, h_qk, sv, False)
    conv = np.concatenate([q.reshape(t, key_dim), k.reshape(t, key_dim), v.reshape(t, h * sv)], axis=1)
    conv_d = torch.from_numpy(conv).cuda()
    qd = conv_d[:, :key_dim].unflatten(-1, (h_qk, sv)).unsqueeze(0)
    kd = conv_d[:, key_dim:2 * key_dim].unflatten(-1, (h_qk, sv)).unsqueeze(0)
    vd = conv_d[:, 2 * key_dim:].unflatten(-1, (h, sv)).unsqueeze(0)
    assert t == 1 or not qd.is_contiguous()
    args = [torch.from_numpy(a).cuda() for a in (g, beta, state)]
    got = gdn.gated_delta_net(qd, kd, vd, *args, n_snap=n_snap)
    _check(torch, got, oracle.gated_delta_net(q, k, v, g, beta, state, n_snap=n_snap))
    assert torch.equal(args[2].cpu(), torch.from_numpy(state)), "the input state is not modified"


@pytest.mark.parametrize("sv,h,h_qk,n_seqs,n_seqs_qk,t,kda,n_snap", [
    (64, 6, 2, 1, 1, 3, True, 1),     # per-row decay
    (128, 4, 4, 2, 2, 5, True, 5),
    (32, 5, 1, 3, 1, 2, False, 1),    # sequences share q/k
    (16, 3, 3, 2, 1, 17, False, 2),   # 16-wide heads, two staging chunks
    (128, 48, 16, 4, 4, 1, False, 1),  # batched decode of 4 sequences
])
def test_gdn_shapes_match_oracle(cuda, oracle, sv, h, h_qk, n_seqs, n_seqs_qk, t, kda, n_snap):
    from codpiece_b200 import gdn
    rng = np.random.default_rng(sv + h + t + n_seqs)
    ins = _inputs(rng, n_seqs, t, h, h_qk, sv, kda, n_seqs_qk)
    got = gdn.gated_delta_net(*(cuda.from_numpy(a).cuda() for a in ins), n_snap=n_snap)
    _check(cuda, got, oracle.gated_delta_net(*ins, n_snap=n_snap))


def test_gdn_cache_output_and_in_place_state(cuda, oracle):
    """The _fused_cache form: states into a caller's slots (stride wider than one set);
    with K = 1 the cache may be the input state itself (updated in place)."""
    from codpiece_b200 import gdn
    torch = cuda
    sv, h, t = 128, 8, 6
    rng = np.random.default_rng(11)
    ins = _inputs(rng, 1, t, h, 2, sv, False)
    ref = oracle.gated_delta_net(*ins, n_snap=4)
    d_set = h * sv * sv
    cache = torch.full((4 * d_set + 4 * 1024,), float("nan"), device="cuda")
    dev = [torch.from_numpy(a).cuda() for a in ins]
    got = gdn.gated_delta_net(*dev, n_snap=4, cache=cache, cache_slot_stride=d_set + 1024)
    _check(torch, got, ref)
    assert torch.isnan(cache[d_set:d_set + 1024]).all(), "the gap between slots is untouched"

    ref1 = oracle.gated_delta_net(*ins, n_snap=1)
    st = dev[5]
    got1 = gdn.gated_delta_net(*dev[:5], st, n_snap=1, cache=st)
    _check(torch, got1, ref1)
    assert rel_err(st.view(1, h, sv, sv).cpu().numpy(), ref1[1][0]) <= TOL


def test_gdn_decode_is_launched_on_the_given_stream(cuda, oracle):
    """Captured in a CUDA graph and replayed: the state advances one token per replay."""
    from codpiece_b200 import gdn
    torch = cuda
    sv, h, h_qk = 128, 48, 16
    rng = np.random.default_rng(5)
    q, k, v, g, beta, state = _inputs(rng, 1, 1, h, h_qk, sv, False)
    dev = [torch.from_numpy(a).cuda() for a in (q, k, v, g, beta, state)]
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        gdn.gated_delta_net(*dev[:5], dev[5], cache=dev[5])  # warm-up (one token)
    s.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        gdn.gated_delta_net(*dev[:5], dev[5], cache=dev[5])
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    ref_state = state
    for _ in range(3):
        _, sts = oracle.gated_delta_net(q, k, v, g, beta, ref_state)
        ref_state = sts[0]
    assert rel_err(dev[5].cpu().numpy(), ref_state) <= TOL
    del graph
