"""GPU: decode plans (cpq_decode_plan_*), the persistent decode kernel.

A plan runs the same arithmetic as the separate act_prep + row-GEMV
launches, but splits the work differently (a stream-K share per warp across
the whole grid, where the per-call GEMV gives each CTA a range): the
superblock dot products are the same and only the order in which they are
summed differs. So a plan's outputs are compared with those launches to
within fp32 summation-order error for the first phase (identical inputs) and
to the parity tolerance down the chain (a last-bit difference can move one
Q8_K rounding), plan against plan bit for bit, and the stack built on a plan
against the CPU restatement like the per-call stack.
"""
import ctypes as C

import numpy as np
import pytest

from tests.conftest import TOL, rel_err

pytestmark = pytest.mark.gpu


def _mm():
    from codpiece_b200 import mul_mat as mm
    return mm


def test_plan_phases_match_separate_calls(cuda):
    """RMS with residual and h_out, a plain phase, a SwiGLU phase; three weights in one phase."""
    torch = cuda
    mm = _mm()
    e, q, f = 5120, 6144, 17408
    wq = mm.synth_weights(mm.TYPE_Q4_K, e, q, seed=1)
    wk = mm.synth_weights(mm.TYPE_Q4_K, e, 1024, seed=2)
    wv = mm.synth_weights(mm.TYPE_Q4_K, e, 1000, seed=3)      # ragged: 1000 rows
    wo = mm.synth_weights(mm.TYPE_Q4_K, q, e, seed=4)
    wg = mm.synth_weights(mm.TYPE_Q4_K, e, f, seed=5)
    wu = mm.synth_weights(mm.TYPE_Q4_K, e, f, seed=6)
    wd = mm.synth_weights(mm.TYPE_Q4_K, f, e, seed=7)
    gen = torch.Generator(device="cpu").manual_seed(11)
    h = torch.randn(e, generator=gen).cuda()
    r = torch.randn(e, generator=gen).cuda()
    nw = (1.0 + 0.1 * torch.randn(e, generator=gen)).cuda()
    z = lambda n: torch.zeros(n, device="cuda")  # noqa: E731
    yq, yk, yv, yo, yg, yu, yd, hh = z(q), z(1024), z(1000), z(e), z(f), z(f), z(e), z(e)
    plan = mm.DecodePlan([
        mm.DecodePhase([wq, wk, wv], [yq, yk, yv], h, mm.PRO_RMS, r=r, g=nw, h_out=hh, eps=1e-6),
        mm.DecodePhase([wo], [yo], yq),
        mm.DecodePhase([wg, wu], [yg, yu], hh, mm.PRO_RMS, r=yo, eps=1e-6),
        mm.DecodePhase([wd], [yd], yg, mm.PRO_SWIGLU, r=yu),
    ])
    plan.run()
    torch.cuda.synchronize()
    assert mm.device_status(0) == 0
    # the same chain as separate fused calls
    v = lambda t: t.view(1, -1)  # noqa: E731
    hh2 = torch.empty_like(hh)
    q2, k2, v2 = mm.mul_mat_fused([wq, wk, wv], v(h), mode=mm.PRO_RMS, r=v(r), g=nw, h_out=v(hh2), eps=1e-6)
    (o2,) = mm.mul_mat_fused([wo], q2)
    hh3 = torch.empty_like(hh)
    g2, u2 = mm.mul_mat_fused([wg, wu], v(hh2), mode=mm.PRO_RMS, r=o2, h_out=v(hh3), eps=1e-6)
    (d2,) = mm.mul_mat_fused([wd], g2, mode=mm.PRO_SWIGLU, r=u2)
    torch.cuda.synchronize()
    assert torch.equal(hh, hh2.view(-1))
    for a, b in ((yq, q2), (yk, k2), (yv, v2)):  # same image: summation order only
        assert rel_err(a.cpu().numpy(), b.view(-1).cpu().numpy()) <= 1e-5
    for a, b in ((yo, o2), (yg, g2), (yu, u2), (yd, d2)):
        assert rel_err(a.cpu().numpy(), b.view(-1).cpu().numpy()) <= TOL
    # and again (counters and the grid barrier are reset by every run): bit for bit
    yd_first = yd.clone()
    yd.zero_()
    plan.run()
    torch.cuda.synchronize()
    assert torch.equal(yd, yd_first)
    plan.close()


def test_plan_stack_matches_per_call_stack(cuda):
    from codpiece_b200 import stack as st
    from codpiece_b200 import tp

    torch = cuda
    h0 = torch.randn(1, 5120, generator=torch.Generator().manual_seed(5)).cuda()
    outs = []
    for use_plan in (False, True):
        s = st.Stack(tp.HP_BENCH_27B, n_layer=4, m=1, seed=8, use_plan=use_plan)
        s.h.copy_(h0)
        s.step_body()
        torch.cuda.synchronize()
        outs.append((s.h_final.clone(), s.logits.clone(), s.tok.clone()))
        s.release()
    assert rel_err(outs[0][0].cpu().numpy(), outs[1][0].cpu().numpy()) <= TOL
    assert rel_err(outs[0][1].cpu().numpy(), outs[1][1].cpu().numpy()) <= TOL
    # the same token, unless the two top logits are within the tolerance of each other
    t0, t1 = int(outs[0][2].view(-1)[0]), int(outs[1][2].view(-1)[0])
    lg = outs[0][1].view(-1)
    assert t0 == t1 or abs(float(lg[t0] - lg[t1])) <= TOL * float(lg.abs().max())


def test_plan_stack_matches_cpu_restatement_and_replays(cuda, oracle):
    from codpiece_b200 import stack as st
    from codpiece_b200 import tp
    from oracle import stack_ref
    from tests.test_gpu_stack import _full_layer_weights

    torch = cuda
    s = st.Stack(tp.HP_BENCH_27B, n_layer=2, m=1, seed=3, use_plan=True)
    h0 = torch.randn(1, 5120, generator=torch.Generator().manual_seed(7)).cuda()
    s.h.copy_(h0)
    s.step_body()
    torch.cuda.synchronize()
    eager = (s.h_final.clone(), s.logits.clone(), s.tok.clone())
    h = h0.cpu().numpy()
    for il in range(2):
        h = stack_ref.layer_step(h, _full_layer_weights(s, il), 5120)
    logits, tok = stack_ref.head_step(h, s.head.data.cpu().numpy(), 5120, tp.HP_BENCH_27B.n_vocab)
    assert rel_err(eager[0].cpu().numpy(), h) <= TOL
    assert rel_err(eager[1].cpu().numpy(), logits) <= TOL
    # captured in a CUDA graph, replayed
    s.h.copy_(h0)
    s.capture()
    s.h.copy_(h0)
    s.replay()
    torch.cuda.synchronize()
    assert torch.equal(s.h_final, eager[0]) and torch.equal(s.logits, eager[1]) and torch.equal(s.tok, eager[2])
    s.release()
    assert _mm().device_status(0) == 0


def test_plan_rejects_bad_phases(cuda):
    torch = cuda
    mm = _mm()
    from codpiece_b200._lib import CpqError
    w = mm.synth_weights(mm.TYPE_Q4_K, 512, 64, seed=1)
    w6 = mm.synth_weights(mm.TYPE_Q6_K, 512, 64, seed=1)
    x, y = torch.zeros(512, device="cuda"), torch.zeros(64, device="cuda")
    with pytest.raises(CpqError, match="UNSUPPORTED"):
        mm.DecodePlan([mm.DecodePhase([w6], [y], x)])
    with pytest.raises(CpqError, match="UNSUPPORTED"):
        mm.DecodePlan([mm.DecodePhase([w], [y], x.view(-1)[1:])])  # misaligned input
    with pytest.raises(CpqError, match="INVALID_ARG"):
        mm.DecodePlan([mm.DecodePhase([w], [y], x, mm.PRO_RMS, r=x, h_out=x)])  # h_out aliases x
    with pytest.raises(ValueError):
        mm.DecodePlan([mm.DecodePhase([w, w, w, w], [y, y, y, y], x)])
    assert mm.device_status(0) == 0
