"""Tensor-parallel host logic on CPU: two gloo ranks, oracle arithmetic.

Each rank slices the full ggml-layout weights by the reference's split rules
(column-parallel gate/up rows, row-parallel ffn_down K blocks), computes its
partial with the CPU oracle and allreduces it with gloo; the result must equal
the unsharded product to fp32 rounding. A second test makes one rank fail
before the collective and checks that the survivor gets an error within the
process-group timeout instead of hanging.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _ffn_rank(rank, world, port, q):
    import torch
    import torch.distributed as dist

    from codpiece_b200 import synth, tp
    from oracle import cpq_oracle as O
    from oracle import stack_ref

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        e, ff = 5120, 17408
        hp = tp.HP_BENCH_27B
        rng = np.random.default_rng(0)
        wg = synth.q4_K_weights(rng, ff, e)
        wu = synth.q4_K_weights(rng, ff, e)
        wd = synth.q4_K_weights(rng, e, ff)
        x = rng.standard_normal((2, e), dtype=np.float32)
        sh = tp.layer_shards(hp, 5, world)
        f0, f1 = sh.gate[rank]
        d0, d1 = sh.down[rank]
        assert (f0, f1) == (d0, d1)
        xn = stack_ref.rms_norm(x)
        g = O.mul_mat(O.Q4_K, wg[f0:f1], e, f1 - f0, xn)          # column-parallel: whole rows
        u = O.mul_mat(O.Q4_K, wu[f0:f1], e, f1 - f0, xn)
        a = stack_ref.silu_mul(g, u)
        rb = 144
        wd_k = np.ascontiguousarray(wd[:, d0 // 256 * rb:d1 // 256 * rb])  # row-parallel: K blocks of every row
        part = O.mul_mat(O.Q4_K, wd_k, d1 - d0, e, a)
        t = torch.from_numpy(part.copy())
        dist.all_reduce(t)
        if rank == 0:
            gf = O.mul_mat(O.Q4_K, wg, e, ff, xn)
            uf = O.mul_mat(O.Q4_K, wu, e, ff, xn)
            full = O.mul_mat(O.Q4_K, wd, ff, e, stack_ref.silu_mul(gf, uf))
            err = float(np.abs(t.numpy() - full).max() / np.abs(full).max())
            q.put(("ok", err, [b - a for a, b in sh.gate]))
    except Exception as ex:  # noqa: BLE001
        q.put(("error", repr(ex), None))
        raise
    finally:
        dist.destroy_process_group()


def test_two_rank_ffn_equals_unsharded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ffn_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    status, err, shares = q.get(timeout=5)
    assert status == "ok", err
    assert shares == [8704, 8704]
    assert err <= 1e-5  # same integer block dots, only the fp32 sum order differs
    assert all(p.exitcode == 0 for p in procs)


def _dying_rank(rank, world, port, q):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # leaves between steps, before its collective
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        q.put("no-error")
    except Exception as ex:  # noqa: BLE001
        q.put("error:" + type(ex).__name__)


def test_peer_failure_surfaces_as_error_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert procs[1].exitcode == 3
    msg = q.get(timeout=5)
    assert msg.startswith("error:"), msg


def test_comm_init_without_a_gpu_reports_an_error():
    import ctypes as C

    import torch

    if torch.cuda.is_available():
        pytest.skip("CPU-only check")
    from codpiece_b200 import _lib
    L = _lib.lib()
    h = C.c_void_p()
    rc = L.cpq_tp_comm_init(C.byref(h), 2, 0, C.create_string_buffer(128), 0, 2000)
    assert rc in (5, 6)  # CUDA or NCCL error, returned rather than aborting
    assert L.cpq_tp_comm_init(C.byref(h), 2, 5, C.create_string_buffer(128), 0, 2000) == 1
