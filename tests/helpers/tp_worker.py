"""One rank of the tensor-parallel stack check (launched by tests/test_gpu_tp.py
through torch.distributed.run, one process per GPU). Modes: "nccl" (per-call
projections, NCCL all-reduce), "ar" (per-call, fused NVLink all-reduce),
"trunk" (the persistent trunk kernel, all-reduce inside it), "split" (as
"ar", with the LM head's vocabulary split over the ranks and the greedy
token found across them, cpq_tp_ar_argmax).

Every rank builds its shard of a few-layer 27B-shaped stack (split.rs rules,
NCCL allreduce through libcpq), runs one decode/verify step, and rank 0 also
runs the same stack unsharded (TP1) on its own GPU; the results must agree
within the parity tolerance and the greedy tokens must match. Rank 0 writes a
JSON verdict to argv[1].
"""
import datetime
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))


def main() -> int:
    import numpy as np
    import torch
    import torch.distributed as dist

    out_path = sys.argv[1]
    layers = int(sys.argv[2]) if len(sys.argv) > 2 else 2
    m = int(sys.argv[3]) if len(sys.argv) > 3 else 1
    mode = sys.argv[4] if len(sys.argv) > 4 else "nccl"
    fused_ar = mode in ("ar", "trunk", "split")
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    from codpiece_b200 import stack as st
    from codpiece_b200 import tp

    obj = [st.Comm.unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    comm = st.Comm(world, rank, obj[0], local, timeout_ms=60000)
    h0 = torch.randn(m, 5120, generator=torch.Generator().manual_seed(11)) * 2
    def exchange(handle: bytes) -> list:
        got = [None] * world
        dist.all_gather_object(got, handle)
        return got

    import dataclasses
    hp = dataclasses.replace(tp.HP_BENCH_27B, split_output=True) if mode == "split" else tp.HP_BENCH_27B
    s = st.Stack(hp, layers, rank, world, comm, m=m, seed=5, ar_exchange=exchange if fused_ar else None,
                 use_trunk=mode == "trunk")
    assert s.split_head == (mode == "split")
    assert (s.trunk is not None) == (mode == "trunk")
    assert (s.ar is not None) == fused_ar
    s.h.copy_(h0)
    s.step_body()
    torch.cuda.synchronize()
    if fused_ar:  # a second step and a captured replay must agree with the first
        first = (s.h_final.clone(), s.logits.clone())
        s.h.copy_(h0)
        s.step_body()
        s.h.copy_(h0)
        s.capture()
        s.h.copy_(h0)
        s.replay()
        torch.cuda.synchronize()
        assert torch.equal(first[0], s.h_final) and torch.equal(first[1], s.logits)
        from codpiece_b200 import mul_mat as mm
        assert mm.device_status(local) == 0
    logits_tp = s.logits.cpu().numpy()
    h_tp = s.h_final.cpu().numpy()
    tok_tp = s.tok.cpu().numpy()
    # every rank ends with the same greedy tokens
    gathered = [None] * world
    dist.all_gather_object(gathered, tok_tp.tolist())
    verdict = {}
    if rank == 0:
        ref = st.Stack(tp.HP_BENCH_27B, layers, 0, 1, None, m=m, seed=5)
        ref.h.copy_(h0)
        ref.step_body()
        torch.cuda.synchronize()
        hr = ref.h_final.cpu().numpy()
        lr = ref.logits.cpu().numpy()[:, :logits_tp.shape[1]]  # rank 0's rows of a split head
        verdict = {
            "world": world, "layers": layers, "m": m, "fused_ar": fused_ar, "mode": mode,
            "logits_rel": float(np.abs(logits_tp - lr).max() / np.abs(lr).max()),
            "h_rel": float(np.abs(h_tp - hr).max() / np.abs(hr).max()),
            "tok_tp": tok_tp.tolist(), "tok_ref": ref.tok.cpu().numpy().tolist(),
            "ranks_agree": all(g == gathered[0] for g in gathered),
        }
        comm.check()
    dist.barrier(device_ids=[local])
    s.release()
    dist.barrier(device_ids=[local])
    comm.destroy()
    dist.destroy_process_group()
    if rank == 0:
        Path(out_path).write_text(json.dumps(verdict))
    return 0


if __name__ == "__main__":
    sys.exit(main())
