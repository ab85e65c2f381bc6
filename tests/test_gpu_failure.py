"""Failure detection without a GPU fault: every device-side wait of the
fused decode layer is bounded, and the two ways a call can end early -- a
wait that gives up (MOMIJ_ERR_TIMEOUT) and the stop flag (MOMIJ_ERR_STOPPED,
the reference's stopFlag: SeedlessMetal.swift:2185, 2730) -- are reported
through momij_moe_synchronize and leave the workspace usable: the next call
on the same workspace gives the oracle's result.

The timeout is produced on the host side by setting the wait bound to zero
polls (momij_set_spin_limit(-1)): every mbarrier and grid-barrier wait then
gives up at once, no wait is left spinning and no memory is touched out of
bounds.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from momij_b200 import synth as S
from oracle import oracle as O

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from momij_b200 import moe


def _layer(M=2, H=1024, I=512, E=16, K=4, gs=64, seed=5):
    w = S.expert_weights(E, H, I, gs, seed=seed)
    x = S.activations(M, H, seed=seed)
    lg = S.logits_normal(M, E, 0, seed)
    dw = {k: torch.from_numpy(v.view(np.int32) if k.startswith("w_") else v.view(np.int16)).cuda()
          for k, v in w.items()}
    for k in ("s_ug", "b_ug", "s_dn", "b_dn"):
        dw[k] = dw[k].view(torch.bfloat16)
    xd = torch.from_numpy(x.view(np.int16)).cuda().view(torch.bfloat16)
    i_ref, s_ref = O.route(lg, K)
    y_ref, _ = O.expert_ffn(x, w, i_ref, s_ref, M, H, I, K, gs)
    return dict(w=w, dw=dw, x=x, xd=xd, lg=torch.from_numpy(lg).cuda(), y_ref=y_ref, M=M, H=H, I=I, K=K,
                gs=gs)


def _run(L, ws):
    y = torch.empty(L["M"], L["H"], dtype=torch.bfloat16, device="cuda")
    moe.forward(L["lg"], L["xd"], L["dw"], y, H=L["H"], I=L["I"], Ktop=L["K"], gs=L["gs"], M=L["M"],
                workspace=ws)
    return y


def _rel(y, ref):
    g = O.np_half_to_f64(y.view(torch.int16).cpu().numpy().view(np.uint16))
    r = O.np_half_to_f64(ref)
    return float((np.sqrt(((g - r) ** 2).sum(axis=1)) / np.sqrt((r ** 2).sum(axis=1))).max())


@pytest.mark.parametrize("M,engine", [(1, None), (2, None), (2, "tc")])
def test_wait_timeout_is_reported_and_the_workspace_stays_usable(M, engine, monkeypatch):
    """The streaming kernel (one token, and two tokens in one launch) and
    the batched tcgen05 kernel."""
    if engine:
        monkeypatch.setenv("MOMIJ_DECODE_MROW", engine)
    L = _layer(M=M)
    ws = moe.new_workspace(L["M"], L["K"], L["H"], L["I"])
    try:
        moe.set_spin_limit(-1)
        _run(L, ws)
        with pytest.raises(moe.SeedlessError) as ei:
            moe.synchronize(workspace=ws)
        assert ei.value.status == moe.TIMEOUT
    finally:
        moe.set_spin_limit(0)
    for _ in range(2):  # the same workspace, twice: barrier and completion counters are back at zero
        y = _run(L, ws)
        moe.synchronize(workspace=ws)
        assert _rel(y, L["y_ref"]) <= 2e-3


def test_stop_flag_skips_the_call_and_clears():
    L = _layer(M=1, seed=6)
    ws = moe.new_workspace(L["M"], L["K"], L["H"], L["I"])
    flag = torch.ones(1, dtype=torch.int32, device="cuda")
    try:
        moe.set_stop_flag(flag)
        _run(L, ws)
        with pytest.raises(moe.SeedlessError) as ei:
            moe.synchronize(workspace=ws)
        assert ei.value.status == moe.STOPPED
        flag.zero_()
        y = _run(L, ws)
        moe.synchronize(workspace=ws)
        assert _rel(y, L["y_ref"]) <= 2e-3
    finally:
        moe.set_stop_flag(None)
