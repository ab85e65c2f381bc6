"""GPU parity of the dense pieces around the expert path -- the router gate
GEMV, the fused decode router, RMSNorm -- and of the whole MoE block
(rmsnorm -> gate -> route -> experts with the fused residual), against the
oracle restatements (oracle/oracle.py: gate_logits, fused_router, rms_norm,
route, expert_ffn).
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

TD = {0: torch.bfloat16, 1: torch.float16}


def half_bits(a32: np.ndarray, dt: int) -> np.ndarray:
    return S.f32_to_half_bits(np.ascontiguousarray(a32, np.float32), dt)


def dev(bits: np.ndarray, dt: int) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).cuda().view(TD[dt])


def gate_weights(E, H, dt, seed=3, scale=None):
    scale = 1.0 / np.sqrt(H) if scale is None else scale
    return half_bits(S.normal_f32(E * H, seed, 901).reshape(E, H) * np.float32(scale), dt)


@pytest.mark.parametrize("M,H,E,xdt,wdt", [(1, 4096, 128, 0, 0), (8, 2048, 256, 0, 1), (37, 4096, 64, 1, 1)])
def test_router_logits_match_float64(M, H, E, xdt, wdt):
    x = S.activations(M, H, dtype=xdt)
    w = gate_weights(E, H, wdt)
    lg = moe.router_logits(dev(x, xdt), dev(w, wdt)).cpu().numpy().astype(np.float64)
    ref = O.gate_logits(x, w, xdt, wdt)
    mag = np.abs(O.np_half_to_f64(x, xdt)) @ np.abs(O.np_half_to_f64(w, wdt)).T
    err = np.abs(lg - ref) / mag
    assert err.max() <= 2e-6, err.max()


@pytest.mark.parametrize("M,H,E,K", [(1, 4096, 128, 8), (4, 4096, 128, 8), (2, 2048, 256, 4), (1, 1024, 512, 8)])
def test_fused_router_matches_reference_semantics(M, H, E, K):
    x = S.activations(M, H, seed=7)
    w = gate_weights(E, H, 0, seed=11)
    ctr = torch.zeros(1, dtype=torch.int32, device="cuda")
    logits = torch.empty(M, E, dtype=torch.float32, device="cuda")
    for _ in range(2):  # the counter is back at zero after every call
        inds, scores = moe.fused_router(dev(x, 0), dev(w, 0), K, ctr, logits=logits)
        torch.cuda.synchronize()
        assert int(ctr.item()) == 0
        lg = logits.cpu().numpy()
        i_ref, s_ref = O.fused_router(lg, K)
        assert (inds.cpu().numpy() == i_ref).all()
        np.testing.assert_allclose(scores.cpu().numpy(), s_ref, rtol=2e-6, atol=1e-9)
        # the selection on exact logits agrees too (no near-ties here)
        i_exact, _ = O.fused_router(O.gate_logits(x, w).astype(np.float32), K)
        assert (inds.cpu().numpy() == i_exact).all()


def test_fused_router_tie_order_follows_the_scan():
    """Equal logits: copies of one gate row at experts 1, 16, 33 and 64 (and
    zero rows, whose probabilities tie too)."""
    M, H, E, K = 1, 1024, 128, 8
    x = S.activations(M, H, seed=2)
    w = gate_weights(E, H, 0, seed=4).copy()
    for e in (16, 33, 64):
        w[e] = w[1]
    w[90:100] = 0
    ctr = torch.zeros(1, dtype=torch.int32, device="cuda")
    logits = torch.empty(M, E, dtype=torch.float32, device="cuda")
    inds, scores = moe.fused_router(dev(x, 0), dev(w, 0), K, ctr, logits=logits)
    lg = logits.cpu().numpy()
    assert lg[0, 1] == lg[0, 16] == lg[0, 33] == lg[0, 64]
    i_ref, s_ref = O.fused_router(lg, K)
    assert (inds.cpu().numpy() == i_ref).all()
    # force the copies into the top-8: make their logit the largest
    w2 = w.copy()
    l_all = O.gate_logits(x, w)[0]
    l1 = l_all[1]
    # a power-of-two factor (exact in bf16) that lifts the copies above every other logit
    f = np.sign(l1) * 2.0 ** np.ceil(np.log2(np.abs(l_all).max() / abs(l1)) + 1)
    for e in (1, 16, 33, 64):
        w2[e] = half_bits(O.np_half_to_f64(w[1], 0).astype(np.float32) * np.float32(f), 0)
    inds, scores = moe.fused_router(dev(x, 0), dev(w2, 0), K, ctr, logits=logits)
    lg = logits.cpu().numpy()
    i_ref, _ = O.fused_router(lg, K)
    got = inds.cpu().numpy()
    assert (got == i_ref).all()
    assert lg[0, 1] == lg[0].max()
    # lower simdgroup first (1 and 16 in simdgroup 0, then 33, then 64); within
    # simdgroup 0 the smaller bit-reversed lane: 16 (10000 -> 00001) before 1
    assert list(got[0, :4]) == [16, 1, 33, 64]


@pytest.mark.parametrize("M,H,dt", [(1, 4096, 0), (5, 2048, 1), (3, 1024, 0)])
def test_rms_norm_matches_oracle(M, H, dt):
    x = S.activations(M, H, seed=9, dtype=dt)
    w = half_bits(1.0 + 0.1 * S.normal_f32(H, 5, 902), dt)
    out = moe.rms_norm(dev(x, dt), dev(w, dt), 1e-6).view(torch.int16).cpu().numpy().view(np.uint16)
    ref = O.rms_norm(x, w, 1e-6, dt)
    diff = np.abs(out.astype(np.int32) - ref.astype(np.int32))
    assert diff.max() <= 1 and (diff == 0).mean() >= 0.99, (diff.max(), (diff == 0).mean())


@pytest.mark.parametrize("M", [1, 4])
def test_moe_block_matches_oracle(M):
    H, I, E, K, gs = 1024, 512, 16, 4, 64
    w = S.expert_weights(E, H, I, gs, seed=13)
    dw = {k: torch.from_numpy(v.view(np.int32) if k.startswith("w_") else v.view(np.int16)).cuda()
          for k, v in w.items()}
    for k in ("s_ug", "b_ug", "s_dn", "b_dn"):
        dw[k] = dw[k].view(torch.bfloat16)
    h0 = S.activations(M, H, seed=14)
    nw = half_bits(1.0 + 0.1 * S.normal_f32(H, 6, 903), 0)
    wg = gate_weights(E, H, 0, seed=15, scale=4.0 / np.sqrt(H))
    h = dev(h0, 0).clone()
    inds = torch.empty(M, K, dtype=torch.int32, device="cuda")
    scores = torch.empty(M, K, dtype=torch.float32, device="cuda")
    moe.moe_block(h, dev(nw, 0), 1e-6, dev(wg, 0), dw, I=I, Ktop=K, gs=gs, inds=inds, scores=scores)
    torch.cuda.synchronize()
    # oracle: the same stages
    xn = O.rms_norm(h0, nw, 1e-6, 0)
    lg = O.gate_logits(xn, wg).astype(np.float32)
    i_ref, s_ref = O.route(lg, K)
    h_ref, _ = O.expert_ffn(xn, w, i_ref, s_ref, M, H, I, K, gs, resid_h=h0.copy())
    assert (inds.cpu().numpy() == i_ref).all()
    got = h.view(torch.int16).cpu().numpy().view(np.uint16)
    assert not (got == h0).all()  # h was updated
    # the staged roundings agree: a rare 1-ulp difference where the GPU's
    # fp32 RMS sum rounds the other way
    diff = np.abs(got.astype(np.int32) - h_ref.astype(np.int32))
    assert diff.max() <= 1 and (diff == 0).mean() >= 0.99, (diff.max(), (diff == 0).mean())
