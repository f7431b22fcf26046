"""The 27B-shaped quantized decoder stack, tensor-parallel over N GPUs.

This is the benchmark's multi-GPU workload: n_layer layers of random-init
Q4_K projections (hidden 5120, q 6144, k/v 1024, FFN 17408) and a Q6_K LM
head over vocab 151936, run as decode (M = 1) or verify (M = 2..16) steps.
Each layer follows codpiece's qwen35 trunk (crates/codpiece-model/src/
qwen35.rs:2554-2786) with the attention core left out:

    xn = rms_norm(h)                             (2534-2537)
    q, k, v = W_q xn, W_k xn, W_v xn             (3029, 3047, 3051)
    h = h + allreduce(W_o q)                     (3197; q stands in for the attention output)
    xn = rms_norm(h)
    g, u = W_gate xn, W_up xn                    (2779-2780)
    h = h + allreduce(W_down (silu(g) * u))      (2781-2783)
    token = argmax(W_head rms_norm(h))           (2797-2818)

Tensor parallelism follows the reference's split rules (cpq_tp_split_state):
q/k/v/gate/up column-parallel (each rank owns output rows), attn_output and
ffn_down row-parallel (each rank owns a K range of quant blocks; its fp32
partials are summed by an NCCL allreduce), the LM head mirrored. One process
per GPU; every op is a libcpq call, and a whole step is captured in one CUDA
graph per rank.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import mul_mat as mm
from . import tp
from ._lib import check, lib

KIND_IDS = {"q": 0, "k": 1, "v": 2, "o": 3, "gate": 4, "up": 5, "down": 6, "head": 7}


def tensor_seed(seed: int, layer: int, kind: str) -> int:
    return (seed * 1_000_003 + layer * 16 + KIND_IDS[kind]) & 0xFFFFFFFFFFFFFFFF


@dataclass
class LayerWeights:
    q: mm.QTensor | None
    k: mm.QTensor | None
    v: mm.QTensor | None
    o: mm.QTensor | None
    gate: mm.QTensor | None
    up: mm.QTensor | None
    down: mm.QTensor | None


class Comm:
    """NCCL communicator of one rank (cpq_tp_comm_* in include/cpq.h)."""

    def __init__(self, nranks: int, rank: int, uid: bytes, device: int, timeout_ms: int = 60000):
        self.handle = C.c_void_p()
        buf = C.create_string_buffer(uid, 128)
        check(lib().cpq_tp_comm_init(C.byref(self.handle), nranks, rank, buf, device, timeout_ms), "cpq_tp_comm_init")
        self.nranks = nranks

    @staticmethod
    def unique_id() -> bytes:
        buf = C.create_string_buffer(128)
        check(lib().cpq_tp_unique_id(buf), "cpq_tp_unique_id")
        return buf.raw

    def allreduce_(self, t: torch.Tensor, stream=None) -> None:
        s = (stream or torch.cuda.current_stream()).cuda_stream
        check(lib().cpq_tp_allreduce_f32(self.handle, C.c_void_p(t.data_ptr()), t.numel(), C.c_void_p(s)),
              "cpq_tp_allreduce_f32")

    def check(self) -> None:
        check(lib().cpq_tp_comm_check(self.handle), "cpq_tp_comm_check")

    def destroy(self, abort: bool = False) -> None:
        if self.handle:
            lib().cpq_tp_comm_destroy(self.handle, 1 if abort else 0)
            self.handle = C.c_void_p()


class Stack:
    """This rank's shard of the stack plus its activation buffers."""

    def __init__(self, hp: tp.Hparams, n_layer: int, rank: int = 0, world: int = 1, comm: Comm | None = None,
                 m: int = 1, seed: int = 0, head: bool = True, device: int | None = None, eps: float = 1e-6,
                 use_plan: bool = False, ar_exchange=None, use_trunk: bool = False):
        self.hp, self.n_layer, self.rank, self.world, self.comm, self.m = hp, n_layer, rank, world, comm, m
        self.eps = eps
        self.dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        e = hp.n_embd
        nb_e = e // 256
        self.layers: list[LayerWeights] = []
        self.shards: list[tp.LayerShards] = []
        for il in range(n_layer):
            sh = tp.layer_shards(hp, il, world)
            self.shards.append(sh)
            (q0, q1), (k0, k1), (v0, v1) = sh.q[rank], sh.k[rank], sh.v[rank]
            (o0, o1), (f0, f1), (d0, d1) = sh.o[rank], sh.gate[rank], sh.down[rank]

            def rows(kind, r0, r1, k_elems=e):
                if r1 <= r0:
                    return None
                return mm.synth_weights(mm.TYPE_Q4_K, k_elems, r1 - r0, tensor_seed(seed, il, kind), row0=r0,
                                        device=self.dev)

            def kslice(kind, n_rows, c0, c1):
                if c1 <= c0:
                    return None
                return mm.synth_weights(mm.TYPE_Q4_K, c1 - c0, n_rows, tensor_seed(seed, il, kind), row0=0,
                                        blk0=c0 // 256, device=self.dev)

            self.layers.append(LayerWeights(
                q=rows("q", q0, q1), k=rows("k", k0, k1), v=rows("v", v0, v1), o=kslice("o", e, o0, o1),
                gate=rows("gate", f0, f1), up=rows("up", f0, f1), down=kslice("down", e, d0, d1)))
        # the head: mirrored (split.rs's default) or, with hp.split_output, this rank's rows of the
        # vocabulary (split.rs's N split), the greedy token then found across ranks (cpq_tp_ar_argmax)
        self.head_row0, n_head = 0, hp.n_vocab
        if head and hp.split_output and world > 1:
            ext = tp.split_state("output.weight", hp, hp.n_vocab, 256, world).ne[:world]
            self.head_row0, n_head = int(sum(ext[:rank])), int(ext[rank])
        self.head = (mm.synth_weights(mm.TYPE_Q6_K, e, n_head, tensor_seed(seed, 0, "head"), row0=self.head_row0,
                                      device=self.dev) if head else None)
        self.split_head = head and n_head != hp.n_vocab
        del nb_e
        f = lambda n: torch.zeros(m, n, dtype=torch.float32, device=self.dev)  # noqa: E731
        qmax = max((s.q[rank][1] - s.q[rank][0]) for s in self.shards) or 1
        kmax = max((s.k[rank][1] - s.k[rank][0]) for s in self.shards) or 1
        fmax = max((s.gate[rank][1] - s.gate[rank][0]) for s in self.shards) or 1
        self.h, self.h_alt, self.xn = f(e), f(e), f(e)
        self.h_final = self.h
        self.qb, self.kb, self.vb = f(qmax), f(kmax), f(kmax)
        self.part = f(e)
        self.gb, self.ub, self.act = f(fmax), f(fmax), f(fmax)
        self.logits = f(n_head) if head else None
        self.tok = torch.zeros(m, dtype=torch.int32, device=self.dev)
        mm.init(self.dev.index, 64 << 20)
        self.graph: torch.cuda.CUDAGraph | None = None
        self.plan: mm.DecodePlan | None = None
        self.trunk: mm.Trunk | None = None
        # Row-parallel partial sums: through the fused NVLink allreduce when the
        # caller supplies a handle exchange (decode M <= 3 with the head), else NCCL.
        self.ar: mm.ArChannel | None = None
        if ar_exchange is not None and world > 1 and m <= 16 and head:
            self.ar = mm.ArChannel(world, rank, m * e, self.dev.index)
            self.ar.connect(list(ar_exchange(self.ar.ipc_handle)))
        if self.split_head and self.ar is None:
            raise ValueError("a split LM head needs the fused all-reduce channel (ar_exchange) for its argmax")
        if use_plan:
            if world != 1 or m != 1:
                raise ValueError("decode plans run the single-GPU M = 1 step")
            self._build_plan()
        if use_trunk:
            if m != 1:
                raise ValueError("the decode trunk runs M = 1 steps")
            if world > 1 and self.ar is None:
                raise ValueError("a tensor-parallel trunk needs the fused all-reduce channel (ar_exchange)")
            self._build_trunk()

    # -- bytes -------------------------------------------------------------
    def weight_bytes(self) -> int:
        n = 0
        for lw in self.layers:
            for w in (lw.q, lw.k, lw.v, lw.o, lw.gate, lw.up, lw.down):
                n += w.nbytes if w is not None else 0
        return n + (self.head.nbytes if self.head is not None else 0)

    def launches_per_step(self) -> int:
        """libcpq kernels one step launches (NCCL's and torch's own kernels not counted)."""
        m = self.m

        def fused(qtype: int, prologue: bool) -> int:
            if qtype == mm.TYPE_Q4_K and m <= 3:
                return 2  # activation image (with the prologue) + row GEMV
            groups = (m + 15) // 16 if qtype == mm.TYPE_Q4_K else (m + 7) // 8
            return (1 if prologue else 0) + 2 * groups

        n = 0
        if self.trunk is not None:
            return 1 + (fused(mm.TYPE_Q6_K, True) + 1 if self.head is not None else 0)
        if self.plan is not None:
            return 1 + fused(mm.TYPE_Q6_K, True) + 1 if self.head is not None else 1
        for il, lw in enumerate(self.layers):
            if lw.q is not None or lw.k is not None or lw.v is not None:
                n += fused(mm.TYPE_Q4_K, True)
            elif il > 0:
                n += 1  # residual add
            n += fused(mm.TYPE_Q4_K, False) if lw.o is not None else 0
            n += fused(mm.TYPE_Q4_K, True) * 2  # gate/up, down
        if self.head is not None:
            n += fused(mm.TYPE_Q6_K, True) + 1
        else:
            n += 1
        return n

    def _build_trunk(self) -> None:
        """The whole trunk of step_body() as one persistent kernel (cpq_trunk_*);
        the head stays a fused call + argmax. o_ranks: the ranks with attention
        rows in each layer (at TP8 the split rules give them to half of the ranks)."""
        layers = []
        for sh, lw in zip(self.shards, self.layers):
            o_ranks = 0
            for r, (q0, q1) in enumerate(sh.q):
                if q1 > q0:
                    o_ranks |= 1 << r
            layers.append(mm.TrunkLayer(q=lw.q, k=lw.k, v=lw.v, o=lw.o, gate=lw.gate, up=lw.up, down=lw.down,
                                        o_ranks=o_ranks if self.world > 1 else 0))
        self.trunk = mm.Trunk(layers, self.hp.n_embd, eps=self.eps, ar=self.ar, device=self.dev.index)

    def _build_plan(self) -> None:
        """The 64-layer trunk of step_body() as one decode plan (4 phases per
        layer); the head stays a separate fused call + argmax."""
        phases = []
        h, h_alt = self.h, self.h_alt
        part_live = False
        for lw in self.layers:
            ws = [w for w in (lw.q, lw.k, lw.v) if w is not None]
            outs = [self._sl(b, w.n).view(-1) for w, b in ((lw.q, self.qb), (lw.k, self.kb), (lw.v, self.vb))
                    if w is not None]
            if part_live:
                phases.append(mm.DecodePhase(ws, outs, h.view(-1), mm.PRO_RMS, r=self.part.view(-1),
                                             h_out=h_alt.view(-1), eps=self.eps))
                h, h_alt = h_alt, h
            else:
                phases.append(mm.DecodePhase(ws, outs, h.view(-1), mm.PRO_RMS, eps=self.eps))
            phases.append(mm.DecodePhase([lw.o], [self.part.view(-1)], self._sl(self.qb, lw.o.k).view(-1)))
            nf = lw.gate.n
            g, u = self._sl(self.gb, nf).view(-1), self._sl(self.ub, nf).view(-1)
            phases.append(mm.DecodePhase([lw.gate, lw.up], [g, u], h.view(-1), mm.PRO_RMS, r=self.part.view(-1),
                                         h_out=h_alt.view(-1), eps=self.eps))
            h, h_alt = h_alt, h
            phases.append(mm.DecodePhase([lw.down], [self.part.view(-1)], g, mm.PRO_SWIGLU, r=u))
            part_live = True
        self.plan = mm.DecodePlan(phases, self.dev.index)
        self._plan_h = (h, h_alt)

    # -- one step ----------------------------------------------------------
    def _sl(self, buf: torch.Tensor, n: int) -> torch.Tensor:
        # a contiguous [m, n] view at the front of a flat buffer
        return buf.view(-1)[: self.m * n].view(self.m, n)

    def step_body(self) -> None:
        """Enqueue one decode/verify step on the current stream.

        Four fused calls per layer: the residual add of the previous projection
        and the RMS norm run in the quantizer of the next one (h ping-pongs
        between two buffers), SwiGLU runs in the quantizer of ffn_down.
        On return self.h holds the final residual stream."""
        h, h_alt = self.h, self.h_alt
        part_live = False  # self.part holds a projection output still to be added to h
        if self.trunk is not None:
            self.trunk.run(h, h_alt)
            if self.head is not None:
                mm.mul_mat_fused([self.head], h_alt, [self.logits], mode=mm.PRO_RMS, eps=self.eps)
                self._argmax()
            self.h_final = h_alt
            return
        if self.plan is not None:
            self.plan.run()
            h, h_alt = self._plan_h
            part_live = len(self.layers) > 0
        ch = self.ar
        for lw in ([] if self.plan is not None else self.layers):
            # attention block: xn = rms(h [+ part]) -> q, k, v
            ws, outs = [], []
            for w, b in ((lw.q, self.qb), (lw.k, self.kb), (lw.v, self.vb)):
                if w is not None:
                    ws.append(w)
                    outs.append(self._sl(b, w.n))
            if part_live:
                if ws and ch is not None:
                    mm.mul_mat_fused(ws, h, outs, mode=mm.PRO_RMS, h_out=h_alt, eps=self.eps, r_ar=ch)
                    h, h_alt = h_alt, h
                elif ws:
                    mm.mul_mat_fused(ws, h, outs, mode=mm.PRO_RMS, r=self.part, h_out=h_alt, eps=self.eps)
                    h, h_alt = h_alt, h
                elif ch is not None:
                    ch.add(h, h)  # no attention rows on this rank: fold the all-reduced residual in place
                else:
                    mm.add_(h, self.part)  # no attention rows on this rank: fold the residual in place
            elif ws:
                mm.mul_mat_fused(ws, h, outs, mode=mm.PRO_RMS, eps=self.eps)
            # o projection (row-parallel)
            if ch is not None and lw.o is not None:
                mm.mul_mat_fused([lw.o], self._sl(self.qb, lw.o.k), [self.part], y_ar=ch)
            elif ch is not None:
                ch.zero(self.hp.n_embd, self.m)  # no attention rows: a zero share of the all-reduce
            elif lw.o is not None:
                mm.mul_mat(lw.o, self._sl(self.qb, lw.o.k), out=self.part)
            else:
                self.part.zero_()
            if self.world > 1 and ch is None:
                self.comm.allreduce_(self.part)
            # ffn: xn = rms(h + part) -> gate, up ; h_alt = h + part
            nf = lw.gate.n
            g, u = self._sl(self.gb, nf), self._sl(self.ub, nf)
            if ch is not None:
                mm.mul_mat_fused([lw.gate, lw.up], h, [g, u], mode=mm.PRO_RMS, h_out=h_alt, eps=self.eps, r_ar=ch)
            else:
                mm.mul_mat_fused([lw.gate, lw.up], h, [g, u], mode=mm.PRO_RMS, r=self.part, h_out=h_alt,
                                 eps=self.eps)
            h, h_alt = h_alt, h
            # down (row-parallel) with silu(gate) * up fused into its quantizer
            if lw.down is not None:
                mm.mul_mat_fused([lw.down], g, [self.part], mode=mm.PRO_SWIGLU, r=u, y_ar=ch)
            elif ch is not None:
                ch.zero(self.hp.n_embd, self.m)
            else:
                self.part.zero_()
            if self.world > 1 and ch is None:
                self.comm.allreduce_(self.part)
            part_live = True
        if self.head is not None:
            if ch is not None and part_live:
                # the head is Q6_K: materialize h + allreduce(part) through a Q4_K-free path
                self._head_prologue_ar(h, h_alt)
                mm.mul_mat_fused([self.head], h_alt, [self.logits], mode=mm.PRO_RMS, eps=self.eps)
            else:
                mm.mul_mat_fused([self.head], h, [self.logits], mode=mm.PRO_RMS, r=self.part, h_out=h_alt,
                                 eps=self.eps)
            h, h_alt = h_alt, h
            self._argmax()
        elif part_live:
            mm.add_(h, self.part)
        self.h_final = h

    def capture(self) -> None:
        """Capture step_body() into a CUDA graph (run one eager step first to warm up)."""
        s = torch.cuda.Stream(device=self.dev)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self.step_body()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize(self.dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.step_body()
        self.graph = g

    def replay(self) -> None:
        self.graph.replay()

    def _argmax(self) -> None:
        """The greedy token: over this rank's logits, or across ranks when the head is split."""
        if self.split_head:
            self.ar.argmax(self.logits, self.head_row0, self.tok)
        else:
            mm.argmax(self.logits, out=self.tok)

    def _head_prologue_ar(self, h, h_out) -> None:
        """h_out = h + allreduce(part) for the Q6_K head (outside the Q4_K decode GEMV)."""
        self.ar.add(h, h_out)

    def release(self) -> None:
        self.graph = None
        if self.trunk is not None:
            self.trunk.close()
            self.trunk = None
        if self.ar is not None:
            self.ar.close()
            self.ar = None
        if self.plan is not None:
            self.plan.close()
            self.plan = None
