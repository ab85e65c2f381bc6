"""Expert-parallel protocol (momij_b200/ep.py) with world_size 2 over gloo on
CPU: the per-rank kernels are the oracle, so this checks the dispatch slots,
the empty-row convention, the exchanges and the combine order -- each rank's
result must equal, bit for bit, the single-process oracle on all tokens with
all experts.  The GPU kernels of the same protocol are covered by
tests/test_gpu_ep.py."""
from __future__ import annotations

import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from momij_b200 import synth as S
from momij_b200.ep import ExpertParallelMoE, shard_experts
from oracle import oracle as O

M_LOCAL, E, K, H, I, GS = 3, 8, 2, 256, 256, 64


class OracleOps:
    """Per-rank kernels of the protocol restated with the oracle (host)."""

    def __init__(self, wts_local):
        self.w = wts_local

    def route(self, logits, K, inds, scores):
        i, s = O.route(logits.numpy(), K)
        inds.copy_(torch.from_numpy(i))
        scores.copy_(torch.from_numpy(s))

    def dispatch(self, inds, x, send_x, send_meta, slot_map, status, *, E, world, capacity):
        ind = inds.numpy().reshape(-1)
        eloc = E // world
        send_meta.fill_(-1)
        status.zero_()
        seen = [0] * world
        for p, e in enumerate(ind):
            d = int(e) // eloc
            slot = d * capacity + seen[d]
            seen[d] += 1
            slot_map[p] = slot
            send_meta[slot] = int(e) - d * eloc
            send_x[slot] = x[p // inds.shape[1]]

    def experts(self, recv_x, recv_meta, act, down):
        meta = recv_meta.numpy()
        rows = np.nonzero(meta >= 0)[0]
        if len(rows) == 0:
            return
        xs = recv_x.numpy().view(np.uint16)[rows]
        ind = meta[rows].astype(np.int32)
        w = self.w
        ug = O.gqmm2(xs, w["w_ug"], w["s_ug"], w["b_ug"], ind, len(rows), 1, H, 2 * I, GS)
        a = O.clamped_swiglu(ug, I)
        d = O.gqmm2(a, w["w_dn"], w["s_dn"], w["b_dn"], ind, len(rows), 1, I, H, GS)
        down.numpy().view(np.uint16)[rows] = d

    def combine(self, back, scores, slot_map, status, h):
        b = back.numpy().view(np.uint16)[slot_map.numpy()]
        out = O.score_resid(b, scores.numpy(), h.numpy().view(np.uint16), h.shape[0], scores.shape[1], H)
        h.copy_(torch.from_numpy(out.view(np.int16)))


def _inputs():
    M = 2 * M_LOCAL
    w = S.expert_weights(E, H, I, GS)
    x = S.activations(M, H)
    lg = S.logits_normal(M, E)
    return w, x, lg


def _rank(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w, x, lg = _inputs()
        mine = slice(rank * M_LOCAL, (rank + 1) * M_LOCAL)
        layer = ExpertParallelMoE(OracleOps(shard_experts(w, rank, world)), E=E, H=H, I=I, K=K,
                                  M=M_LOCAL, dtype=torch.int16)
        h = torch.from_numpy(x[mine].copy().view(np.int16))
        layer.forward(torch.from_numpy(lg[mine].copy()), h)
        q.put((rank, h.numpy().view(np.uint16).copy(), layer.slot_map.numpy().copy()))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_protocol_matches_single_process_oracle():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        while len(got) < world:
            r, h, sm = q.get(timeout=180)  # spawned ranks import torch first
            got[r] = (h, sm)
    except Exception:
        pass
    for p in procs:
        p.join(timeout=60)
        if p.exitcode is None:
            p.kill()
        assert p.exitcode == 0, "a rank failed"
    assert len(got) == world
    w, x, lg = _inputs()
    M = 2 * M_LOCAL
    inds, scores = O.route(lg, K)
    ref, _ = O.expert_ffn(x, w, inds, scores, M, H, I, K, GS, resid_h=x)
    for r in range(world):
        h, sm = got[r]
        np.testing.assert_array_equal(h, ref[r * M_LOCAL:(r + 1) * M_LOCAL])
        assert len(set(sm.tolist())) == M_LOCAL * K  # every pair its own slot


def test_single_rank_protocol_without_a_process_group():
    w, x, lg = _inputs()
    M = 2 * M_LOCAL
    layer = ExpertParallelMoE(OracleOps(w), E=E, H=H, I=I, K=K, M=M, dtype=torch.int16)
    h = torch.from_numpy(x.copy().view(np.int16))
    layer.forward(torch.from_numpy(lg.copy()), h)
    inds, scores = O.route(lg, K)
    ref, _ = O.expert_ffn(x, w, inds, scores, M, H, I, K, GS, resid_h=x)
    np.testing.assert_array_equal(h.numpy().view(np.uint16), ref)
