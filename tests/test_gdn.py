"""Gated delta-net on the host: the oracle pinned against a second formulation
of the reference, and the C ABI's argument checks (no GPU needed).

The oracle (oracle/cpq_oracle_gdn.c) restates the fused CUDA kernel
(gated_delta_net.cu:4-167). Here it is checked against a float64 numpy
restatement of the same recurrence as ggml builds it from plain ops,
llm_build_delta_net_base::build_delta_net_autoregressive
(notes/reference/delta-net-base.cpp:289-372: q scaled by 1/sqrt(S_k), state
decayed by exp(g), sk = sum_rows(S * k), d = (v - sk) * beta, S += k (x) d,
o = sum_rows(S * q), k repeated over the v heads), one token at a time.
For a per-row decay (KDA, g [S_v, H, T, n_seqs]) the fused kernel decays the
key dimension i, the one contracted with k and q (gated_delta_net.cu:113-134),
while the graph builder's broadcast of g would decay the other one; codpiece's
layers use the per-head decay (GDA), where both agree. The restatement below
follows the fused kernel for KDA.
"""
import ctypes as C

import numpy as np
import pytest


def _inputs(rng, n_seqs, t, h, h_qk, sv, kda, n_seqs_qk=None):
    n_seqs_qk = n_seqs_qk or n_seqs
    q = rng.standard_normal((n_seqs_qk, t, h_qk, sv)).astype(np.float32)
    k = rng.standard_normal((n_seqs_qk, t, h_qk, sv)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)  # qwen35.rs:2708-2709 l2-normalises q and k
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((n_seqs, t, h, sv)).astype(np.float32)
    g = -rng.uniform(0.01, 2.0, size=(n_seqs, t, h, sv) if kda else (n_seqs, t, h)).astype(np.float32)
    beta = rng.uniform(0.0, 1.0, size=(n_seqs, t, h)).astype(np.float32)
    state = (0.1 * rng.standard_normal((n_seqs, h, sv, sv))).astype(np.float32)
    return q, k, v, g, beta, state


def graph_autoregressive(q, k, v, g, beta, state):
    """delta-net-base.cpp:289-372 in float64, applied token by token; returns
    (attn [n_seqs, T, H, S_v], per-token states [T, n_seqs, H, col, i])."""
    n_seqs, t, h, sv = v.shape
    h_qk = q.shape[2]
    rq3 = n_seqs // q.shape[0]
    s = state.astype(np.float64).transpose(0, 1, 3, 2).copy()  # [seq, h, i, col] = S[i][col]
    attn = np.zeros((n_seqs, t, h, sv))
    states = np.zeros((t, n_seqs, h, sv, sv))
    scale = 1.0 / np.sqrt(np.float32(sv))
    for tt in range(t):
        for sq in range(n_seqs):
            for hh in range(h):
                kk = k[sq // rq3, tt, hh % h_qk].astype(np.float64)  # ggml_repeat: head hh reads hh % H_k
                qq = q[sq // rq3, tt, hh % h_qk].astype(np.float64) * scale
                ge = np.exp(g[sq, tt, hh].astype(np.float64))
                m = s[sq, hh] * (ge[:, None] if g.ndim == 4 else ge)
                sk = m.T @ kk
                d = (v[sq, tt, hh] - sk) * beta[sq, tt, hh]
                m = m + np.outer(kk, d)
                attn[sq, tt, hh] = m.T @ qq
                s[sq, hh] = m
        states[tt] = s.transpose(0, 1, 3, 2)
    return attn, states


@pytest.mark.parametrize("kda", [False, True])
@pytest.mark.parametrize("sv,h,h_qk,n_seqs,t", [(128, 3, 1, 1, 1), (32, 6, 2, 2, 1), (16, 4, 4, 1, 5)])
def test_oracle_matches_graph_formulation(oracle, kda, sv, h, h_qk, n_seqs, t):
    rng = np.random.default_rng(sv + h + t)
    q, k, v, g, beta, state = _inputs(rng, n_seqs, t, h, h_qk, sv, kda)
    attn, states = oracle.gated_delta_net(q, k, v, g, beta, state, n_snap=1)
    ref_attn, ref_states = graph_autoregressive(q, k, v, g, beta, state)
    assert np.abs(attn - ref_attn).max() <= 1e-5 * max(1.0, np.abs(ref_attn).max())
    assert np.abs(states[0] - ref_states[-1]).max() <= 1e-5 * max(1.0, np.abs(ref_states).max())


def test_oracle_snapshot_slots(oracle):
    """K > 1: slot j holds the state j tokens before the last (gated_delta_net.cu:145-157);
    slots at or beyond T are not written."""
    rng = np.random.default_rng(7)
    q, k, v, g, beta, state = _inputs(rng, 1, 5, 2, 1, 16, False)
    _, ref_states = graph_autoregressive(q, k, v, g, beta, state)
    for n_snap in (3, 5, 8):
        _, states = oracle.gated_delta_net(q, k, v, g, beta, state, n_snap=n_snap)
        assert states.shape[0] == min(n_snap, 5)
        for j in range(states.shape[0]):
            assert np.abs(states[j] - ref_states[4 - j]).max() <= 1e-5


def test_oracle_gqa_sequence_sharing(oracle):
    """v heads read q/k head h % H_qk and sequences share q/k rows in groups of n_seqs / n_seqs_qk."""
    rng = np.random.default_rng(3)
    q, k, v, g, beta, state = _inputs(rng, 4, 2, 6, 3, 32, False, n_seqs_qk=2)
    attn, states = oracle.gated_delta_net(q, k, v, g, beta, state)
    ref_attn, ref_states = graph_autoregressive(q, k, v, g, beta, state)
    assert np.abs(attn - ref_attn).max() <= 1e-5
    assert np.abs(states[0] - ref_states[-1]).max() <= 1e-5


def _t(ne, data=0x10000):
    from codpiece_b200._lib import CpqTensor
    d = CpqTensor()
    d.type = 0
    d.ne[:] = list(ne) + [1] * (4 - len(ne))
    nb = [4]
    for e in d.ne[:3]:
        nb.append(nb[-1] * e)
    d.nb[:] = nb
    d.data = data
    return d


@pytest.mark.parametrize("bad", ["sv", "g", "beta", "state", "dst", "k_snap", "qk", "type", "cache"])
def test_abi_rejects_bad_shapes_without_a_launch(bad):
    """Argument checks run before anything touches a device, so they are exercised here on the host."""
    from codpiece_b200._lib import lib
    sv, h, t, n = 128, 4, 2, 1
    q, k, v = _t([sv, 2, t, n]), _t([sv, 2, t, n]), _t([sv, h, t, n])
    g, beta, state = _t([1, h, t, n]), _t([1, h, t, n]), _t([sv, sv, h, n])
    dst = _t([sv * h * t * n + sv * sv * h * n])
    k_snap, cache, stride = 1, None, 0
    if bad == "sv":
        v = _t([48, h, t, n])
    elif bad == "g":
        g = _t([3, h, t, n])
    elif bad == "beta":
        beta = _t([1, h, t + 1, n])
    elif bad == "state":
        state = _t([sv, sv, h - 1, n])
    elif bad == "dst":
        dst = _t([sv * h * t * n])
    elif bad == "k_snap":
        k_snap = -1
    elif bad == "qk":
        k = _t([sv, 3, t, n])
    elif bad == "type":
        v.type = 1
    else:
        k_snap, cache, stride = 2, C.c_void_p(0x20000), 16
    rc = lib().cpq_gated_delta_net(*(C.byref(x) for x in (q, k, v, g, beta, state, dst)), k_snap, cache, stride, None)
    assert rc in (1, 2), rc  # CPQ_ERR_INVALID_ARG, CPQ_ERR_UNSUPPORTED
