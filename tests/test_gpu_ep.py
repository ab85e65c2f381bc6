"""Expert-parallel decode on the GPU (momij_b200/ep.py with the C-ABI kernels):
one rank must give the same bits as the single-GPU layer (moe.forward into the
residual stream); with two GPUs, two NCCL ranks must give the same bits as
one rank on all tokens."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

from momij_b200 import synth as S
from oracle import oracle as O
from parity_util import assert_ffn_parity

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from momij_b200 import moe
    from momij_b200.ep import ExpertParallelMoE, GpuOps

M, E, K, H, I, GS = 16, 16, 4, 1024, 512, 64


def _run_ep(wts, lg, x, M_, world=1, group=None, device="cuda"):
    layer = ExpertParallelMoE(GpuOps(wts, H=H, I=I, gs=GS), E=E, H=H, I=I, K=K, M=M_, group=group,
                              device=torch.device(device))
    h = torch.from_numpy(x.copy().view(np.int16)).to(device).view(torch.bfloat16)
    layer.forward(torch.from_numpy(lg.copy()).to(device), h)
    torch.cuda.synchronize()
    assert int(layer.status.item()) == 0
    return h.view(torch.int16).cpu().numpy().view(np.uint16)


def test_one_rank_equals_the_single_gpu_layer():
    wd = moe.device_expert_weights(E, H, I, GS)
    lg, x = S.logits_normal(M, E), S.activations(M, H)
    h_ep = _run_ep(wd, lg, x, M)
    h = torch.from_numpy(x.copy().view(np.int16)).cuda().view(torch.bfloat16)
    ws = moe.new_workspace(M, K, H, I)
    moe.forward(torch.from_numpy(lg).cuda(), h, wd, None, H=H, I=I, Ktop=K, gs=GS, M=M, resid_h=h,
                workspace=ws)
    moe.synchronize(workspace=ws)
    np.testing.assert_array_equal(h_ep, h.view(torch.int16).cpu().numpy().view(np.uint16))
    # and the oracle (host weights of the same generator)
    w = S.expert_weights(E, H, I, GS)
    inds, scores = O.route(lg, K)
    ref, st = O.expert_ffn(x, w, inds, scores, M, H, I, K, GS, resid_h=x)
    assert_ffn_parity(h_ep, ref, st["down"], scores, 0, "expert-parallel world=1")


def _rank(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from momij_b200 import moe as m
        ml = M // world
        wd = m.device_expert_weights(E, H, I, GS, experts=(rank * E // world, (rank + 1) * E // world),
                                     device=f"cuda:{rank}")
        lg, x = S.logits_normal(M, E), S.activations(M, H)
        mine = slice(rank * ml, (rank + 1) * ml)
        h = _run_ep(wd, lg[mine], x[mine], ml, world, None, f"cuda:{rank}")
        q.put((rank, h))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_two_ranks_equal_one_rank():
    import torch.multiprocessing as mp
    world = 2
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        while len(got) < world:
            r, h = q.get(timeout=120)
            got[r] = h
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.exitcode is None:
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    wd = moe.device_expert_weights(E, H, I, GS)
    lg, x = S.logits_normal(M, E), S.activations(M, H)
    h1 = _run_ep(wd, lg, x, M)
    np.testing.assert_array_equal(np.concatenate([got[0], got[1]]), h1)


# ---- the same layer through the C-ABI object (momij_moe_ep_init/forward) -------

def _run_c_ep(wts, lg, x, M_, rank=0, world=1, uid=None, device="cuda"):
    ep = moe.EpLayer(rank=rank, world=world, E=E, H=H, I=I, K=K, max_tokens=M_, gs=GS, unique_id=uid)
    h = torch.from_numpy(x.copy().view(np.int16)).to(device).view(torch.bfloat16)
    ep.forward(h, wts, logits=torch.from_numpy(lg.copy()).to(device), resid_h=h)
    ep.status()
    out = h.view(torch.int16).cpu().numpy().view(np.uint16)
    ep.close()
    return out


def test_c_abi_one_rank_equals_the_single_gpu_layer():
    wd = moe.device_expert_weights(E, H, I, GS)
    lg, x = S.logits_normal(M, E), S.activations(M, H)
    h_c = _run_c_ep(wd, lg, x, M)
    h = torch.from_numpy(x.copy().view(np.int16)).cuda().view(torch.bfloat16)
    ws = moe.new_workspace(M, K, H, I)
    moe.forward(torch.from_numpy(lg).cuda(), h, wd, None, H=H, I=I, Ktop=K, gs=GS, M=M, resid_h=h, workspace=ws)
    moe.synchronize(workspace=ws)
    np.testing.assert_array_equal(h_c, h.view(torch.int16).cpu().numpy().view(np.uint16))


def _c_rank(rank, world, uid, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    from momij_b200 import moe as m
    ml = M // world
    wd = m.device_expert_weights(E, H, I, GS, experts=(rank * E // world, (rank + 1) * E // world),
                                 device=f"cuda:{rank}")
    lg, x = S.logits_normal(M, E), S.activations(M, H)
    mine = slice(rank * ml, (rank + 1) * ml)
    q.put((rank, _run_c_ep(wd, lg[mine], x[mine], ml, rank, world, uid, f"cuda:{rank}")))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_c_abi_two_ranks_equal_one_rank():
    import torch.multiprocessing as mp
    world = 2
    uid = moe.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_c_rank, args=(r, world, uid, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        while len(got) < world:
            r, h = q.get(timeout=120)
            got[r] = h
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.exitcode is None:
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    wd = moe.device_expert_weights(E, H, I, GS)
    lg, x = S.logits_normal(M, E), S.activations(M, H)
    np.testing.assert_array_equal(np.concatenate([got[0], got[1]]), _run_c_ep(wd, lg, x, M))
