#!/usr/bin/env python3
"""Benchmark: quantized mul_mat weight GB/s and 27B-stack decode ms/token.

Workload (every N): the 27B-shaped stack of BASELINE config 5 --
64 layers of Q4_K q/k/v/o/gate/up/down (hidden 5120, q 6144, kv 1024,
FFN 17408) plus a Q6_K head over vocab 151936 -- decoding M = 1
token per step, tensor-parallel over N GPUs (one process per GPU). Each
projection is one fused call (activation image + decode GEMV) and the
row-parallel partial sums cross NVLink inside the GEMV (--nccl: through NCCL);
From 4 ranks on (or with --trunk) each rank's 64 layers run as one
persistent kernel instead (cpq_trunk_run, the all-reduce inside it);
--per-call keeps one call per projection at every N. The head is a fused Q6_K mul_mat
plus argmax; at N > 1 its rows (the vocabulary) are split over the ranks
(split.rs's optional N split) and the greedy token is found across them
through the NVLink channel (--mirrored-head: the whole head on every rank,
split.rs's default).
Its FFN projections are exactly BASELINE config 2's Q4_K mat-vec shapes,
64 times over.

  value      model GB/s = the unsharded model's weight bytes (12.906 GB, the
             head counted once) / max-over-ranks ms per token (CUDA events,
             inputs resident in HBM); bytes each rank streams are
             config.weight_bytes_per_rank
  tp_parity  N > 1: a 2-layer stack decoded (M = 1, trunk) and verified
             (M = 8, per-call MMA GEMVs), both through the fused NVLink
             all-reduce, on all ranks against the same stack on one GPU
             before timing; the run fails if either differs by more than 1e-3
  e2e        the same through the public API with host buffers: hidden state
             uploaded from pinned memory and the greedy token read back
             every step
  roofline   the dominant kernel, the Q4_K mul_mat on config 2's shapes,
             timed live over back-to-back launches on rotating weights
             (larger than L2), against MEASURED_PEAKS.json hbm_gbs
  cpu_baseline  the CPU oracle (restated ggml-cpu semantics, AVX2 + OpenMP)
             on config 2's three matrices at M = 1, rank 0 at N = 1

  prefill    BASELINE config 4: the Q4_K prefill GEMM on tcgen05
             at M = 512 and 2048 for both FFN shapes, TFLOP/s through
             mul_mat (activation pre-pass included) against
             MEASURED_PEAKS.json bf16_tflops
  verify     the same 64-layer stack stepping M = 8 tokens (the speculative
             verify batch of configs[4]) on all N GPUs (fused NVLink all-reduce;
             --nccl: NCCL)
  small_configs  configs[0] (Q8_0 [5120 x 5120] mat-vec, M = 1) and configs[2]
             (one layer's q/k/v/o and the Q6_K head at M = 2, 4, 8, 16):
             weight GB/s of each mul_mat on rotating weights larger than L2

--impl reference times the reference's CPU path for this operator (the
oracle restatement: ggml itself is not available) on a bounded sample of the
same stack (a few layers per step) and prints the same metric.

--profile CASE runs one small fixed case for ncu, its measured launches
inside an NVTX range named "step" (ncu --nvtx --nvtx-include step/):
  decode_ffn   Q4_K mul_mat M=1 on config 2's gate and down shapes, 2 calls each
  prefill_512  Q4_K mul_mat M=512 on [17408 x 5120], 1 call
  prefill_q8_0_512 / prefill_q6k_512  the same for Q8_0 / Q6_K weights
  verify_ffn   Q4_K mul_mat M=8 on config 2's gate and down shapes, 1 call each
  stack        --steps replays of the captured stack decode step (--trunk: the trunk kernel)
  head         Q6_K mul_mat on the head [151936 x 5120] at M = 1 and M = 8, 1 call each
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Q4_K mat-vec weight GB/s vs HBM peak; 27B-stack decode ms/tok at 1-8 GPUs"
FALLBACK_HBM_GBS = 6650.0
Q4K_FFN = ((17408, 5120), (17408, 5120), (5120, 17408))  # gate, up, down: (N, K)


def log(*a):
    print(*a, file=sys.stderr, flush=True)


FALLBACK_BF16_TFLOPS = 1590.0


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def tensor_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        if "bf16_tflops" in d:
            return float(d["bf16_tflops"]), "measured (burst)"
    return FALLBACK_BF16_TFLOPS, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.rows, self.proc = gpu, [], None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception as e:  # noqa: BLE001
            log("clock sampler unavailable:", e)
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:  # noqa: BLE001
                self.proc.kill()
            self.t.join(timeout=2)
        sm = [float(r[1]) for r in self.rows if len(r) > 2 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) > 2 and r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in self.rows:
            for i, n in enumerate(names):
                if len(r) > 5 + i and r[5 + i].lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.rows)}


# the sources the decode GEMV (act_prep_kernel + gemv_q4k_row_kernel) is compiled from
ROW_GEMV_SOURCES = ("common.cuh", "q8k_block.cuh", "act_prep.cuh", "gemv_row.cuh")


def source_hash(files=ROW_GEMV_SOURCES) -> str:
    import hashlib
    h = hashlib.sha256()
    for f in files:
        h.update((ROOT / "codpiece_b200" / "csrc" / f).read_bytes())
    return h.hexdigest()[:16]


def traffic_from_profiles():
    """Per-launch DRAM bytes of the Q4_K GEMV from the committed ncu summary, used only when the
    summary was captured from the kernel sources in this tree (its source_sha256 line matches).
    Returns (bytes or None, note)."""
    p = ROOT / "profiles" / "gemv_q4k_row_ffn.md"
    if not p.exists():
        return None, "no ncu summary"
    traffic, src = None, None
    for line in p.read_text().splitlines():
        t = line.strip()
        if t.startswith("traffic_bytes_per_launch:"):
            try:
                traffic = int(t.split(":", 1)[1].strip().split()[0])
            except ValueError:
                traffic = None
        elif t.startswith("source_sha256:"):
            src = t.split(":", 1)[1].strip().split()[0]
    if src != source_hash():
        return None, "ncu summary was captured from other kernel sources"
    return traffic, f"ncu capture of these sources (source_sha256 {src})"


def cpu_baseline(seconds: float = 10.0):
    """Oracle on config 2's three Q4_K matrices at M = 1, all host threads."""
    from codpiece_b200 import synth
    from oracle import cpq_oracle as O

    O.build()
    nthreads = os.cpu_count() or 1
    mats = [(synth.weights(synth.Q4_K, n, k, seed=i), n, k) for i, (n, k) in enumerate(Q4K_FFN)]
    xs = {k: synth.activations(1, k, seed=10 + k) for _, k in Q4K_FFN}
    total_b, t0, reps = 0, time.perf_counter(), 0
    while True:
        for w, n, k in mats:
            O.mul_mat(O.Q4_K, w, k, n, xs[k], nthreads=nthreads)
            total_b += w.nbytes
        reps += 1
        dt = time.perf_counter() - t0
        if dt >= seconds:
            break
    return {"value": round(total_b / dt / 1e9, 3), "unit": "GB/s", "cores": nthreads, "kind": "port",
            "sample": f"config 2 Q4_K gate/up/down [17408x5120, 17408x5120, 5120x17408] at M=1, {reps} passes "
                      f"({dt:.1f} s) on {nthreads} threads; restated ggml-cpu semantics (AVX2 integer dots, "
                      f"OpenMP over rows)"}


def kernel_roofline(torch, mm, stream, sets: int = 4, reps: int = 20):
    """Average duration of one config-2 Q4_K mul_mat (M=1) over rotating weights (> L2)."""
    hbm, kind = peaks()
    ws = []
    for s in range(sets):
        for i, (n, k) in enumerate(Q4K_FFN):
            ws.append(mm.synth_weights(mm.TYPE_Q4_K, k, n, seed=9000 + 3 * s + i))
    xs = {k: torch.randn(1, k, device="cuda") for _, k in Q4K_FFN}
    ys = [torch.empty(1, w.n, device="cuda") for w in ws]
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for w, y in zip(ws, ys):
            mm.mul_mat(w, xs[w.k], out=y)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    with torch.cuda.graph(g):
        for w, y in zip(ws, ys):
            mm.mul_mat(w, xs[w.k], out=y)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cur = torch.cuda.current_stream()
    e0.record(cur)
    for _ in range(reps):
        g.replay()
    e1.record(cur)
    torch.cuda.synchronize()
    per_op_s = e0.elapsed_time(e1) / 1e3 / (reps * len(ws))
    algo = sum(w.nbytes + 4 * w.k + 4 * w.n for w in ws) / len(ws)
    ach = algo / per_op_s / 1e9
    traffic, traffic_note = traffic_from_profiles()
    del g
    return {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s", "frac": round(ach / hbm, 4),
            "traffic": traffic, "traffic_source": traffic_note, "peak_kind": kind,
            "kernel": "Q4_K mul_mat M=1 (act_prep_kernel + gemv_q4k_row_kernel<1>), config 2 shapes",
            "algorithmic_bytes_per_launch": int(algo), "avg_launch_us": round(per_op_s * 1e6, 3),
            "launches_timed": reps * len(ws)}


def prefill_roofline(torch, mm, reps: int = 10):
    """Q4_K prefill mul_mat TFLOP/s (tcgen05 GEMM + its activation pre-pass)."""
    peak, kind = tensor_peak()
    cases = []
    cur = torch.cuda.current_stream()
    for m in (512, 2048):
        for n, k in ((17408, 5120), (5120, 17408)):
            ws = [mm.synth_weights(mm.TYPE_Q4_K, k, n, seed=7000 + i) for i in range(2)]
            x = torch.randn(m, k, device="cuda")
            y = torch.empty(m, n, device="cuda")
            for _ in range(3):
                for w in ws:
                    mm.mul_mat(w, x, out=y)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(cur)
            for _ in range(reps):
                for w in ws:
                    mm.mul_mat(w, x, out=y)
            e1.record(cur)
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (reps * len(ws))
            tf = 2.0 * m * n * k / us / 1e6
            cases.append({"m": m, "n": n, "k": k, "us": round(us, 2), "tflops": round(tf, 1)})
            del ws, x, y
    best = max(cases, key=lambda c: c["tflops"])
    tot_flop = sum(2.0 * c["m"] * c["n"] * c["k"] for c in cases)
    tot_us = sum(c["us"] for c in cases)
    ach = tot_flop / tot_us / 1e6
    # the same GEMM for the production trunk's Q8_0 and the Q6_K head / fallback at a 512-token chunk
    others = []
    for qt, n, k in ((mm.TYPE_Q8_0, 17408, 5120), (mm.TYPE_Q8_0, 5120, 17408), (mm.TYPE_Q6_K, 17408, 5120),
                     (mm.TYPE_Q6_K, 151936, 5120)):
        m = 512
        nw = 1 if n * k > 200_000_000 else 2
        ws = [mm.synth_weights(qt, k, n, seed=7100 + i) for i in range(nw)]
        x = torch.randn(m, k, device="cuda")
        y = torch.empty(m, n, device="cuda")
        for _ in range(2):
            for w in ws:
                mm.mul_mat(w, x, out=y)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(cur)
        for _ in range(reps):
            for w in ws:
                mm.mul_mat(w, x, out=y)
        e1.record(cur)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (reps * nw)
        tf = 2.0 * m * n * k / us / 1e6
        others.append({"type": mm.TYPE_NAMES[qt], "m": m, "n": n, "k": k, "us": round(us, 2), "tflops": round(tf, 1),
                       "frac": round(tf / peak, 4)})
        del ws, x, y
    return {"bound": "tensor", "achieved": round(ach, 1), "peak": peak, "unit": "TFLOP/s",
            "frac": round(ach / peak, 4), "peak_kind": kind,
            "kernel": "Q4_K mul_mat M>16: act_f16_kernel + gemm_q4k_tc_kernel (2-SM tcgen05, fp16 operands, "
                      "fp32 TMEM accumulators)",
            "achieved_is": "FLOP-weighted over the four configs[3] cases", "best": best, "cases": cases,
            "q8_0_q6_k_m512": others}


def _time_graph(torch, calls, reps: int = 10):
    """Average duration of one of `calls` (closures that enqueue one mul_mat), replayed in a CUDA graph."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for c in calls:
            c()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for c in calls:
            c()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    cur = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    for _ in range(reps):
        g.replay()
    e1.record(cur)
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) * 1e3 / (reps * len(calls))


def small_configs(torch, mm):
    """configs[0] (Q8_0 [5120x5120] mat-vec, M = 1) and configs[2] (one layer's Q4_K q/k/v/o and the Q6_K
    head [151936x5120] at M = 2, 4, 8, 16): weight GB/s of each mul_mat, rotating weights larger than L2."""
    hbm, kind = peaks()
    out = {"peak_gbs": hbm, "peak_kind": kind}
    q8 = [mm.synth_weights(mm.TYPE_Q8_0, 5120, 5120, seed=8000 + i) for i in range(24)]  # 668 MB
    x1 = torch.randn(1, 5120, device="cuda")
    y1 = torch.empty(1, 5120, device="cuda")
    us = _time_graph(torch, [lambda w=w: mm.mul_mat(w, x1, out=y1) for w in q8])
    out["config1_q8_0_m1"] = {"us": round(us, 2), "GBs": round(q8[0].nbytes / us / 1e3, 1),
                              "frac": round(q8[0].nbytes / us / 1e3 / hbm, 4)}
    del q8
    sets = []
    for sidx in range(6):  # 6 x 41 MB > L2
        sd = 8100 + 10 * sidx
        sets.append((mm.synth_weights(mm.TYPE_Q4_K, 5120, 6144, seed=sd),
                     mm.synth_weights(mm.TYPE_Q4_K, 5120, 1024, seed=sd + 1),
                     mm.synth_weights(mm.TYPE_Q4_K, 5120, 1024, seed=sd + 2),
                     mm.synth_weights(mm.TYPE_Q4_K, 6144, 5120, seed=sd + 3)))
    head = mm.synth_weights(mm.TYPE_Q6_K, 5120, 151936, seed=8200)
    attn_bytes = sum(w.nbytes for w in sets[0])
    per_m = []
    for m in (2, 4, 8, 16):
        x = torch.randn(m, 5120, device="cuda")
        xo = torch.randn(m, 6144, device="cuda")
        outs = [torch.empty(m, n, device="cuda") for n in (6144, 1024, 1024)]
        yo = torch.empty(m, 5120, device="cuda")
        calls = []
        for q, k, v, o in sets:
            calls.append(lambda q=q, k=k, v=v: mm.mul_mat_multi([q, k, v], x, outs))
            calls.append(lambda o=o: mm.mul_mat(o, xo, out=yo))
        us_pair = _time_graph(torch, calls) * 2  # one q/k/v call + one o call
        yh = torch.empty(m, 151936, device="cuda")
        us_head = _time_graph(torch, [lambda: mm.mul_mat(head, x, out=yh)], reps=5)
        per_m.append({"m": m, "attn_set_us": round(us_pair, 2), "attn_GBs": round(attn_bytes / us_pair / 1e3, 1),
                      "head_us": round(us_head, 1), "head_GBs": round(head.nbytes / us_head / 1e3, 1),
                      "head_frac": round(head.nbytes / us_head / 1e3 / hbm, 4)})
        del x, xo, outs, yo, yh
    out["config3_verify_small_m"] = per_m
    del sets, head
    out["gdn"] = gdn_recurrence(torch)
    return out


def gdn_recurrence(torch):
    """The GDN recurrence of one 27B GDN layer (48 v heads x 128, 16 q/k heads): T = 1 decode and
    T = 8 verify with 8 rollback snapshots; state bytes read + written per launch / duration,
    24 layers' states rotated (> L2)."""
    from codpiece_b200 import gdn
    hbm, _ = peaks()
    res = []
    for t, n_snap in ((1, 1), (8, 8)):
        g = torch.Generator(device="cpu").manual_seed(t)
        q = torch.nn.functional.normalize(torch.randn(1, t, 16, 128, generator=g), dim=-1).cuda()
        k = torch.nn.functional.normalize(torch.randn(1, t, 16, 128, generator=g), dim=-1).cuda()
        v = torch.randn(1, t, 48, 128, generator=g).cuda()
        gg = -torch.rand(1, t, 48, generator=g).cuda()
        b = torch.rand(1, t, 48, generator=g).cuda()
        states = [0.1 * torch.randn(1, 48, 128, 128, device="cuda") for _ in range(24)]
        slots = gdn.state_slots(n_snap, t)
        outs = [torch.empty(t * 48 * 128 + slots * 48 * 128 * 128, device="cuda") for _ in range(24)]
        us = _time_graph(torch, [lambda s=s_, o=o_: gdn.gated_delta_net(q, k, v, gg, b, s, n_snap=n_snap, out=o)
                                 for s_, o_ in zip(states, outs)])
        byts = 4 * 48 * 128 * 128 * (1 + slots)
        res.append({"t": t, "k_snap": n_snap, "us": round(us, 2), "state_GBs": round(byts / us / 1e3, 1),
                    "frac": round(byts / us / 1e3 / hbm, 4)})
        del states, outs
    return res


def model_bytes(tp, layers: int, head: bool = True) -> int:
    """Weight bytes of the unsharded stack: Q4_K 144 B per 256 weights, the Q6_K head 210 B per 256."""
    hp = tp.HP_BENCH_27B
    e, q, kv, ff = hp.n_embd, hp.n_head * hp.head_k, hp.n_head_kv * hp.head_k, hp.n_ff
    per_layer = sum(n * k // 256 * 144 for n, k in ((q, e), (kv, e), (kv, e), (e, q), (ff, e), (ff, e), (e, ff)))
    return layers * per_layer + (hp.n_vocab * e // 256 * 210 if head else 0)


def verify_step(torch, st, tp, layers: int, rank: int, world: int, comm, barrier, m: int = 8, steps: int = 10,
                exchange=None, hp=None):
    """configs[4]'s verify step: the same stack at M = 8 tokens on all ranks (MMA GEMVs; at N > 1 the
    row-parallel partial sums go through the fused NVLink all-reduce when exchange is given, else NCCL).
    Max over ranks of the device time."""
    stack = st.Stack(hp or tp.HP_BENCH_27B, layers, rank, world, comm, m=m, seed=0, ar_exchange=exchange)
    stack.h.copy_(torch.randn(m, 5120, generator=torch.Generator().manual_seed(5)).cuda())
    stack.capture()
    for _ in range(3):
        stack.replay()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        stack.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    stack.release()
    return ms


def tp_parity(torch, st, tp, comm, exchange, rank: int, world: int, layers: int = 2, hp=None):
    """N > 1: a few full-width layers decoded through the trunk (M = 1) and verified (M = 8, per-call MMA
    GEMVs), both with the fused NVLink all-reduce, on all ranks, against the same stack on rank 0's GPU
    alone (the per-call path, itself checked against the CPU oracle by the tests). Returns rank 0's verdict."""
    import torch.distributed as dist
    out = {}
    for m, trunk in ((1, True), (8, False)):
        h0 = torch.randn(m, 5120, generator=torch.Generator().manual_seed(11 + m)) * 2
        s = st.Stack(hp or tp.HP_BENCH_27B, layers, rank, world, comm, m=m, seed=5, ar_exchange=exchange,
                     use_trunk=trunk)
        s.h.copy_(h0)
        s.step_body()
        torch.cuda.synchronize()
        h_tp, logits_tp, tok_tp = s.h_final.cpu(), s.logits.cpu(), s.tok.cpu()
        toks = [None] * world
        dist.all_gather_object(toks, tok_tp.tolist())
        s.release()
        del s
        if rank == 0:
            ref = st.Stack(tp.HP_BENCH_27B, layers, 0, 1, None, m=m, seed=5)
            ref.h.copy_(h0)
            ref.step_body()
            torch.cuda.synchronize()
            hr = ref.h_final.cpu()
            lr = ref.logits.cpu()[:, :logits_tp.shape[1]]  # rank 0's rows of a split head (all when mirrored)
            key = "decode_m1_trunk" if trunk else "verify_m8_fused_ar"
            out[key] = {"h_rel": float((h_tp - hr).abs().max() / hr.abs().max()),
                        "logits_rel": float((logits_tp - lr).abs().max() / lr.abs().max()),
                        "tok_match": tok_tp.tolist() == ref.tok.cpu().tolist(),
                        "ranks_agree": all(t == toks[0] for t in toks)}
            ref.release()
            del ref
        dist.barrier()
    if rank == 0:
        out["layers"] = layers
        out["ok"] = all(v["h_rel"] <= 1e-3 and v["logits_rel"] <= 1e-3 and v["ranks_agree"]
                        for k, v in out.items() if isinstance(v, dict))
    return out


def profile_case(args) -> int:
    """One small fixed case for ncu (see the module docstring)."""
    import torch

    torch.cuda.set_device(0)
    from codpiece_b200 import build as cbuild
    if not cbuild.LIB.exists():
        cbuild.build()
    from codpiece_b200 import mul_mat as mm
    mm.init(0, 1 << 30)
    nvtx = torch.cuda.nvtx
    if args.profile == "decode_ffn":
        calls = [(mm.synth_weights(mm.TYPE_Q4_K, k, n, seed=11 + i), torch.randn(1, k, device="cuda"))
                 for i, (n, k) in enumerate(((17408, 5120), (5120, 17408)))]
        for w, x in calls:
            mm.mul_mat(w, x)
        torch.cuda.synchronize()
        nvtx.range_push("step")
        for _ in range(2):
            for w, x in calls:
                mm.mul_mat(w, x)
        torch.cuda.synchronize()
        nvtx.range_pop()
    elif args.profile == "prefill_512":
        w = mm.synth_weights(mm.TYPE_Q4_K, 5120, 17408, seed=21)
        x = torch.randn(512, 5120, device="cuda")
        mm.mul_mat(w, x)
        torch.cuda.synchronize()
        nvtx.range_push("step")
        mm.mul_mat(w, x)
        torch.cuda.synchronize()
        nvtx.range_pop()
    elif args.profile in ("prefill_q8_0_512", "prefill_q6k_512"):
        qt = mm.TYPE_Q8_0 if args.profile == "prefill_q8_0_512" else mm.TYPE_Q6_K
        w = mm.synth_weights(qt, 5120, 17408, seed=22)
        x = torch.randn(512, 5120, device="cuda")
        mm.mul_mat(w, x)
        torch.cuda.synchronize()
        nvtx.range_push("step")
        mm.mul_mat(w, x)
        torch.cuda.synchronize()
        nvtx.range_pop()
    elif args.profile == "verify_ffn":
        calls = [(mm.synth_weights(mm.TYPE_Q4_K, k, n, seed=41 + i), torch.randn(8, k, device="cuda"))
                 for i, (n, k) in enumerate(((17408, 5120), (5120, 17408)))]
        for w, x in calls:
            mm.mul_mat(w, x)
        torch.cuda.synchronize()
        nvtx.range_push("step")
        for w, x in calls:
            mm.mul_mat(w, x)
        torch.cuda.synchronize()
        nvtx.range_pop()
    elif args.profile == "head":
        w = mm.synth_weights(mm.TYPE_Q6_K, 5120, 151936, seed=31)
        xs = [torch.randn(m, 5120, device="cuda") for m in (1, 8)]
        for x in xs:
            mm.mul_mat(w, x)
        torch.cuda.synchronize()
        nvtx.range_push("step")
        for x in xs:
            mm.mul_mat(w, x)
        torch.cuda.synchronize()
        nvtx.range_pop()
    elif args.profile == "stack":
        from codpiece_b200 import stack as st
        from codpiece_b200 import tp
        stack = st.Stack(tp.HP_BENCH_27B, args.layers, 0, 1, None, m=args.m, seed=0,
                         use_trunk=args.m == 1 and args.trunk)
        stack.h.copy_(torch.randn(args.m, 5120, device="cuda"))
        stack.capture()
        for _ in range(args.warmup):
            stack.replay()
        torch.cuda.synchronize()
        nvtx.range_push("step")
        for _ in range(args.steps):
            stack.replay()
        torch.cuda.synchronize()
        nvtx.range_pop()
        stack.release()
    else:
        log(f"unknown --profile case {args.profile}")
        return 2
    assert mm.device_status(0) == 0
    log(f"profile case {args.profile}: ok")
    return 0


def reference_arm(args, rank):
    """CPU reference (restated ggml-cpu mul_mat) on a bounded sample of the stack."""
    if rank != 0:
        return 0
    import numpy as np

    from codpiece_b200 import synth
    from oracle import cpq_oracle as O
    from oracle import stack_ref

    O.build()
    nthreads = os.cpu_count() or 1
    e, q, kv, ff = 5120, 6144, 1024, 17408
    layers = []
    for il in range(args.ref_layers):
        rng = np.random.default_rng(100 + il)
        lw = {}
        for kind, n, k in (("q", q, e), ("k", kv, e), ("v", kv, e), ("o", e, q), ("gate", ff, e), ("up", ff, e),
                           ("down", e, ff)):
            lw[kind] = (synth.q4_K_weights(rng, n, k), n, k)
        layers.append(lw)
    wbytes = sum(w.nbytes for lw in layers for (w, _, _) in lw.values())
    h0 = synth.activations(args.m, e, seed=1)
    times = []
    for it in range(args.warmup + args.steps):
        h = h0.copy()
        t0 = time.perf_counter()
        for lw in layers:
            h = stack_ref.layer_step(h, lw, e, nthreads)
        dt = time.perf_counter() - t0
        if it >= args.warmup:
            times.append(dt)
    t = sum(times) / len(times)
    val = wbytes / t / 1e9
    line = {"metric": METRIC, "value": round(val, 3), "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t * 1e3, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8 dots, fp32 accumulate", "data": "synthetic",
            "config": {"workload": f"27B-shaped Q4_K stack decode, sample of {args.ref_layers} layers per step "
                                   f"(no head), M={args.m}", "layers_per_step": args.ref_layers, "m": args.m,
                       "same_config": False,
                       "comparability": "weight GB/s of the same per-layer arithmetic (RMS norms, Q8_K re-quantization, "
                                        "q/k/v/o/gate/up/down Q4_K dots, SwiGLU, residual adds) on a bounded sample "
                                        "of the stack; the GPU arm's value is the whole 64-layer stack plus the Q6_K "
                                        "head per token, in the same unit"},
            "cpu_baseline": {"value": round(val, 3), "unit": "GB/s", "cores": nthreads, "kind": "port",
                             "sample": f"{args.ref_layers} stack layers ({wbytes / 1e9:.2f} GB of Q4_K weights) per "
                                       f"step, restated ggml-cpu semantics, {nthreads} threads"},
            "e2e": {"value": round(val, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=64)
    ap.add_argument("--m", type=int, default=1)
    ap.add_argument("--ref-layers", type=int, default=2)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-verify", action="store_true")
    ap.add_argument("--no-small", action="store_true", help="skip the configs[0] / configs[2] lines")
    ap.add_argument("--nccl", action="store_true", help="TP partial sums through NCCL (not with --trunk)")
    ap.add_argument("--trunk", action="store_true", help="the persistent trunk kernel at every N")
    ap.add_argument("--per-call", action="store_true", help="one call per projection at every N")
    ap.add_argument("--mirrored-head", action="store_true", help="the LM head on every rank (no vocabulary split)")
    ap.add_argument("--no-parity", action="store_true", help="skip the N > 1 parity check")
    ap.add_argument("--profile", default=None,
                    choices=["decode_ffn", "verify_ffn", "prefill_512", "prefill_q8_0_512", "prefill_q6k_512", "stack",
                             "head"])
    ap.add_argument("--source-hash", action="store_true",
                    help="print the hash of the decode GEMV's sources (the source_sha256 of its ncu summary)")
    args = ap.parse_args()
    if args.source_hash:
        print(source_hash())
        return 0
    if args.profile:
        return profile_case(args)
    if args.warmup < 3:
        log("warmup raised to 3 (timing rule)")
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus != world:
        log(f"--gpus {args.gpus} but WORLD_SIZE={world}: using WORLD_SIZE")
        args.gpus = world

    if args.impl == "reference":
        return reference_arm(args, rank)

    import datetime

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))

    from codpiece_b200 import build as cbuild
    if not cbuild.LIB.exists():
        cbuild.build()
    from codpiece_b200 import mul_mat as mm
    from codpiece_b200 import stack as st
    from codpiece_b200 import tp

    comm = None
    if world > 1:
        obj = [st.Comm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        comm = st.Comm(world, rank, obj[0], local, timeout_ms=120000)

    def exchange(handle: bytes) -> list:
        got = [None] * world
        dist.all_gather_object(got, handle)
        return got

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    # the LM head: split over the ranks by vocabulary rows (split.rs's optional N split, greedy token
    # through cpq_tp_ar_argmax) when the fused all-reduce runs, else mirrored (split.rs's default)
    import dataclasses
    split_head = world > 1 and not args.nccl and not args.mirrored_head
    hp = dataclasses.replace(tp.HP_BENCH_27B, split_output=True) if split_head else tp.HP_BENCH_27B
    parity = None
    if world > 1 and not args.no_parity:
        parity = tp_parity(torch, st, tp, comm, exchange, rank, world, hp=hp)
        ok = [parity.get("ok", True) if rank == 0 else True]
        dist.broadcast_object_list(ok, src=0)
        if not ok[0]:
            if rank == 0:
                log(f"TP parity check failed: {parity}")
            comm.destroy()
            dist.destroy_process_group()
            return 3
        torch.cuda.empty_cache()

    # default: the trunk kernel from 4 ranks on (there the per-projection launch chain and the
    # all-reduce waits dominate); one call per projection below, where it is the faster path
    use_trunk = args.m == 1 and not args.nccl and (args.trunk or (world >= 4 and not args.per_call))
    t_build = time.perf_counter()
    stack = st.Stack(hp, args.layers, rank, world, comm, m=args.m, seed=0,
                     ar_exchange=exchange if (world > 1 and not args.nccl) else None, use_trunk=use_trunk)
    g = torch.Generator(device="cpu").manual_seed(1234)
    h0 = torch.randn(args.m, 5120, generator=g).cuda()
    stack.h.copy_(h0)
    stack.capture()
    torch.cuda.synchronize()
    log(f"[rank {rank}] stack built + captured in {time.perf_counter() - t_build:.1f} s, "
        f"{stack.weight_bytes() / 1e9:.3f} GB of weights on this rank")

    cur = torch.cuda.current_stream()
    for _ in range(args.warmup):
        stack.h.copy_(h0)
        stack.replay()
    torch.cuda.synchronize()

    # ---- timed region: device-resident inputs ----
    # The sampler starts first so that its process start-up skew between ranks
    # lands before the barrier, not inside the max-over-ranks window.
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    for _ in range(args.steps):
        stack.replay()
    e1.record(cur)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps

    # ---- e2e: host buffers through the public API ----
    h_host = h0.cpu().pin_memory()
    tok_host = torch.empty(args.m, dtype=torch.int32).pin_memory()
    for _ in range(2):
        stack.h.copy_(h_host, non_blocking=True)
        stack.replay()
        tok_host.copy_(stack.tok, non_blocking=True)
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(cur)
    for _ in range(args.steps):
        stack.h.copy_(h_host, non_blocking=True)
        stack.replay()
        tok_host.copy_(stack.tok, non_blocking=True)
        cur.synchronize()  # the caller needs the token before the next step
    f1.record(cur)
    torch.cuda.synchronize()
    barrier()
    ms_e2e = f0.elapsed_time(f1) / args.steps

    t = torch.tensor([ms, ms_e2e], dtype=torch.float64, device="cuda")
    b = torch.tensor([float(stack.weight_bytes())], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(b, op=dist.ReduceOp.MAX)
    ms, ms_e2e = float(t[0]), float(t[1])
    rank_bytes = float(b[0])
    total_bytes = float(model_bytes(tp, args.layers))
    launches = stack.launches_per_step() * args.steps

    roof = prefill = verify = None
    small = None
    if rank == 0:
        roof = kernel_roofline(torch, mm, cur)
        if not args.no_prefill:
            prefill = prefill_roofline(torch, mm)
        if world == 1 and not args.no_small:
            small = small_configs(torch, mm)
    barrier()
    ar_mode = ("none" if world == 1 else "nccl" if stack.ar is None else
               "inside the trunk kernel over NVLink peer memory (cpq_trunk_run)" if stack.trunk is not None else
               "fused into the GEMV over NVLink peer memory (cpq_mul_mat_fused_ar)")
    path = "trunk" if stack.trunk is not None else "per-call"
    stack.release()
    del stack
    torch.cuda.empty_cache()
    if not args.no_verify:
        vms = verify_step(torch, st, tp, args.layers, rank, world, comm, barrier,
                          exchange=exchange if (world > 1 and not args.nccl) else None, hp=hp)
        tv = torch.tensor([vms], dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(tv, op=dist.ReduceOp.MAX)
        vms = float(tv[0])
        verify = {"m": 8, "ms_per_step": round(vms, 4), "tok_per_s": round(8e3 / vms, 1),
                  "model_GBs": round(total_bytes / vms / 1e6, 1), "layers": args.layers,
                  "tp_allreduce": "none" if world == 1 else "nccl" if args.nccl else
                  "fused into the MMA GEMV over NVLink peer memory"}
    barrier()
    if comm is not None:
        comm.destroy()
    if world > 1:
        dist.destroy_process_group()

    if rank != 0:
        return 0
    cpu = None
    if world == 1 and not args.no_cpu:
        cpu = cpu_baseline(args.cpu_seconds)
    hbm, _ = peaks()
    value = total_bytes / (ms / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8 dots (Q4_K/Q6_K x Q8_K), fp32 accumulate", "data": "synthetic",
        "config": {"workload": "27B-shaped stack decode (BASELINE config 5): 64 x Q4_K q/k/v/o/gate/up/down + "
                               "Q6_K head [151936x5120], M=1, TP=N",
                   "head": ("split over the ranks by vocabulary rows, greedy token through cpq_tp_ar_argmax"
                            if split_head else "mirrored" if world > 1 else "whole"),
                   "path": path,
                   "tp_allreduce": ar_mode,
                   "layers": args.layers, "m": args.m, "tp": world, "hidden": 5120, "ffn": 17408,
                   "vocab": 151936, "parallelism": f"tp{world}",
                   "model_bytes": int(total_bytes),
                   "weight_bytes_per_rank": int(rank_bytes),
                   "ms_per_token": round(ms, 4), "tok_per_s": round(1e3 / ms * args.m, 2),
                   "l2": "weights per rank exceed L2 (126 MB) every step; no flush needed",
                   "frac_of_hbm_per_rank": round(rank_bytes / (ms / 1e3) / 1e9 / hbm, 4)},
        "e2e": {"value": round(total_bytes / (ms_e2e / 1e3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(ms_e2e, 4), "h2d_bytes_per_step": 4 * 5120 * args.m,
                "d2h_bytes_per_step": 4 * args.m},
        "gpu_launches": launches,
        "clocks": clk,
        "roofline": roof,
        "cpu_baseline": cpu,
        "prefill": prefill,
        "verify": verify,
        "tp_parity": parity,
        "parity": {"activation_blocks": "byte-identical to the CPU oracle (tests/)",
                   "outputs": "max |y - y_oracle| / max |y_oracle| <= 1e-3 (tests/)",
                   "oracle_pinning": "partial: dequantization and the portable Q8_0 quantizer pinned to gguf-py "
                                     "fixtures, the block dots pinned to gguf-py's dequantization; the Q8_K and "
                                     "AVX2 Q8_0 quantizers' rounding rules are restatements (ggml is not available)"},
        "small_configs": small,
    }
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
