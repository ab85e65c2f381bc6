"""GPU parity tests: libmomij_moe.so (through its C ABI) against the CPU oracle.

Test names follow the reference's SeedlessMetalTests (momij
MomijCoreTests.swift:204-1347) where a counterpart exists; the checks there
are kernel-vs-kernel, here every kernel is also checked against the oracle.
Tolerance: see tests/parity_util.py (max per-vector rel-L2 <= 2e-3 and every
element within 2 ulps of the 16-bit format).
"""
from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

from momij_b200 import synth as S
from oracle import oracle as O
from parity_util import assert_ffn_parity, assert_parity

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from momij_b200 import moe
DEV = "cuda"
TD = {0: torch.bfloat16, 1: torch.float16}


def dev16(a: np.ndarray, dt: int) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(DEV).view(TD[dt])


def host16(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def dev_weights(w: dict, dt: int) -> dict:
    out = {}
    for k, v in w.items():
        if k.startswith("w_"):
            out[k] = torch.from_numpy(v.view(np.int32)).to(DEV)
        else:
            out[k] = dev16(v, dt)
    return out


def run_ffn(x, w, inds, scores, M, H, I, K, gs, dt, resid=None):
    dw = dev_weights(w, dt)
    y = torch.empty(M, H, dtype=TD[dt], device=DEV)
    h = dev16(resid, dt) if resid is not None else None
    ws = moe.new_workspace(M, K, H, I)
    moe.expert_ffn(dev16(x, dt), dw, torch.from_numpy(inds).to(DEV),
                   torch.from_numpy(scores).to(DEV), None if h is not None else y, H=H, I=I,
                   Ktop=K, gs=gs, M=M, resid_h=h, workspace=ws)
    moe.synchronize(workspace=ws)
    return host16(h if h is not None else y), ws


# ---- synthetic generator on the device == numpy generator ------------------

def test_device_synth_matches_numpy_generator():
    wd = moe.device_expert_weights(4, 512, 256, 64, layer=3, seed=11)
    wh = S.expert_weights(4, 512, 256, 64, layer=3, seed=11)
    for k in wh:
        got = wd[k].view(torch.int32 if k.startswith("w_") else torch.int16).cpu().numpy()
        got = got.view(np.uint32 if k.startswith("w_") else np.uint16)
        assert (got == wh[k]).all(), k
    t = torch.empty(1000, dtype=torch.bfloat16, device=DEV)
    moe.synth_fill(t, 2, seed=5, stream_id=S.stream_id(2, S.KIND_X))
    assert (host16(t) == S.normal_half(1000, 5, S.stream_id(2, S.KIND_X))).all()


# ---- router ------------------------------------------------------------------

@pytest.mark.parametrize("M,E,K", [(1, 128, 8), (8, 128, 8), (64, 256, 8), (3, 64, 4), (5, 1000, 32)])
def test_route_indices_bit_exact(M, E, K):
    lg = S.logits_normal(M, E, seed=M + E)
    inds, scores = moe.route(torch.from_numpy(lg).to(DEV), K)
    torch.cuda.synchronize()
    i_ref, s_ref = O.route(lg, K)
    assert (inds.cpu().numpy() == i_ref).all()
    np.testing.assert_allclose(scores.cpu().numpy(), s_ref, rtol=2e-6, atol=1e-7)


def tie_heavy_logits(M: int, E: int, seed: int, levels: int = 3) -> np.ndarray:
    rng = np.random.default_rng(seed)
    vals = np.array([-0.0, 0.0] + [float(v) for v in np.linspace(-1.0, 1.0, levels)], np.float32)
    return vals[rng.integers(0, len(vals), size=(M, E))].astype(np.float32)


def test_route_ties_follow_the_reference_tree():
    lg = np.zeros((3, 64), np.float32)
    lg[0, [7, 3, 40, 41]] = 2.0
    lg[1, 3], lg[1, 5] = -0.0, 0.0
    lg[1, [0, 1, 2, 4]] = -1.0
    lg[1, 6:] = -1.0
    lg[2, :] = -1.0
    inds, scores = moe.route(torch.from_numpy(lg).to(DEV), 6)
    i_ref, s_ref = O.route(lg, 6)
    got = inds.cpu().numpy()
    assert (got == i_ref).all()
    for m in range(3):
        assert got[m].tolist() == O.tree_route_indices(lg[m], 6)
    assert got[0, :4].tolist() == [40, 41, 3, 7]  # bit-reversed order of the tied experts
    assert got[1, :2].tolist() == [5, 3]          # -0.0 and +0.0 tie
    np.testing.assert_allclose(scores.cpu().numpy(), s_ref, rtol=2e-6)


@pytest.mark.parametrize("M,E,K", [(4, 16, 8), (8, 128, 8), (3, 256, 16), (2, 300, 8)])
def test_route_tie_heavy_logits_bit_exact(M, E, K):
    lg = tie_heavy_logits(M, E, seed=7 * E + K)
    inds, _ = moe.route(torch.from_numpy(lg).to(DEV), K)
    i_ref, _ = O.route(lg, K)
    assert (inds.cpu().numpy() == i_ref).all()


def test_route_nan_logits_follow_the_tree():
    lg = S.logits_normal(3, 128, seed=11)
    lg[0, 0] = np.nan   # position 0 keeps a NaN: selected first
    lg[1, 5] = np.nan   # a NaN at position 5 is dropped by the stage s = 4
    lg[2, [7, 70]] = np.nan
    inds, _ = moe.route(torch.from_numpy(lg).to(DEV), 8)
    got = inds.cpu().numpy()
    for m in range(3):
        assert got[m].tolist() == O.tree_route_indices(lg[m], 8)


def test_permute_matches_oracle():
    lg = S.logits_zipf(300, 128, seed=2)
    i_ref, s_ref = O.route(lg, 8)
    off, pair, wt = moe.permute(torch.from_numpy(i_ref).to(DEV), torch.from_numpy(s_ref).to(DEV), 128)
    o2, p2, w2 = O.permute(i_ref, s_ref, 128)
    assert (off.cpu().numpy() == o2).all()
    assert (pair.cpu().numpy() == p2).all()
    assert (wt.cpu().numpy() == w2).all()


# ---- gather-GEMV ---------------------------------------------------------------

@pytest.mark.parametrize("M,Ktop,K,N,E,gs,dt,lhs", [
    (1, 8, 512, 64, 16, 64, 0, False),
    (1, 4, 2048, 96, 8, 128, 0, False),
    (2, 4, 256, 80, 8, 64, 0, True),      # ragged N (not a multiple of 16)
    (4, 2, 1024, 33, 6, 64, 1, False),    # fp16, odd N
    (8, 8, 768, 128, 32, 128, 0, True),
    (3, 3, 4096, 40, 5, 64, 0, False),
])
def test_gqmm2_matches_oracle(M, Ktop, K, N, E, gs, dt, lhs):
    w = S.codes(E * N * K // 16, 1, 100).reshape(E, N, K // 16)
    s = S.affine_uniform(E * N * K // gs, S.SCALE_A, S.SCALE_C, 1, 101, dt).reshape(E, N, K // gs)
    b = S.affine_uniform(E * N * K // gs, S.BIAS_A, S.BIAS_C, 1, 102, dt).reshape(E, N, K // gs)
    rows = M * Ktop if lhs else M
    x = S.normal_half(rows * K, 1, 103, dt).reshape(rows, K)
    inds = np.argsort(S.logits_normal(M, E, seed=M + 17), axis=1)[:, :Ktop].astype(np.int32)
    ref = O.gqmm2(x, w, s, b, inds, M, Ktop, K, N, gs, lhs, dt)
    out = torch.empty(M * Ktop, N, dtype=TD[dt], device=DEV)
    ws = moe.new_workspace(M, Ktop, 0, 0)
    moe.gqmm2(dev16(x, dt), torch.from_numpy(w.view(np.int32)).to(DEV), dev16(s, dt), dev16(b, dt),
              torch.from_numpy(inds).to(DEV), out, Ktop=Ktop, K=K, N=N, gs=gs, lhs_per_expert=lhs,
              M=M, workspace=ws)
    moe.synchronize(workspace=ws)
    assert_parity(host16(out), ref, dt, "gqmm2")


@pytest.mark.parametrize("M,K,N", [
    (1, 2048, 3072),   # QKV of a 2048-wide model (q 2048, k and v 512 each)
    (8, 2048, 2048),   # O projection, verify batch
    (1, 4096, 6144),   # QKV at hidden 4096
    (4, 4096, 4096),   # O at hidden 4096
])
def test_dense_projection_ktop1(M, K, N):
    """The dense 2-bit projections of attention reuse gqmm2 with one "expert"
    and Ktop = 1 (SeedlessMetal.swift:951-952, 1001-1002: inds all zero,
    lhsPerExpert false)."""
    gs, dt = 64, 0
    w = S.codes(N * K // 16, 2, 110).reshape(1, N, K // 16)
    s = S.affine_uniform(N * K // gs, S.SCALE_A, S.SCALE_C, 2, 111, dt).reshape(1, N, K // gs)
    b = S.affine_uniform(N * K // gs, S.BIAS_A, S.BIAS_C, 2, 112, dt).reshape(1, N, K // gs)
    x = S.normal_half(M * K, 2, 113, dt).reshape(M, K)
    inds = np.zeros((M, 1), np.int32)
    ref = O.gqmm2(x, w, s, b, inds, M, 1, K, N, gs, False, dt)
    out = torch.empty(M, N, dtype=TD[dt], device=DEV)
    ws = moe.new_workspace(M, 1, 0, 0)
    moe.gqmm2(dev16(x, dt), torch.from_numpy(w.view(np.int32)).to(DEV), dev16(s, dt), dev16(b, dt),
              torch.from_numpy(inds).to(DEV), out, Ktop=1, K=K, N=N, gs=gs, M=M, workspace=ws)
    moe.synchronize(workspace=ws)
    assert_parity(host16(out), ref, dt, "dense gqmm2")


def test_gqmm2_repeated_expert_in_token():
    """gqmm2 callers may repeat an expert inside a token (the reference test
    uses arbitrary inds); the plan splits such runs into more units."""
    M, Ktop, K, N, E, gs = 1, 8, 512, 48, 4, 64
    w = S.codes(E * N * K // 16, 2, 0).reshape(E, N, K // 16)
    s = S.affine_uniform(E * N * K // gs, S.SCALE_A, S.SCALE_C, 2, 1).reshape(E, N, K // gs)
    b = S.affine_uniform(E * N * K // gs, S.BIAS_A, S.BIAS_C, 2, 2).reshape(E, N, K // gs)
    x = S.normal_half(M * Ktop * K, 2, 3).reshape(M * Ktop, K)
    inds = np.array([[1, 1, 1, 3, 0, 1, 3, 3]], np.int32)
    ref = O.gqmm2(x, w, s, b, inds, M, Ktop, K, N, gs, True)
    out = torch.empty(M * Ktop, N, dtype=torch.bfloat16, device=DEV)
    ws = moe.new_workspace(M, Ktop, 0, 0)
    moe.gqmm2(dev16(x, 0), torch.from_numpy(w.view(np.int32)).to(DEV), dev16(s, 0), dev16(b, 0),
              torch.from_numpy(inds).to(DEV), out, Ktop=Ktop, K=K, N=N, gs=gs, lhs_per_expert=True,
              M=M, workspace=ws)
    moe.synchronize(workspace=ws)
    assert_parity(host16(out), ref, 0, "repeated experts")


def test_gqmm2_mrow_matches_sequential():
    """M=2 batched == two M=1 calls, bit for bit (MomijCoreTests.swift:251-314,
    same fixture: bytes (i*17+3)&0xff, x=(i%17-8)*0.01, s=0.02, b=-0.02)."""
    H, N, E, Ktop, M, gs = 512, 128, 8, 2, 2, 128
    nbytes = E * N * (H // 16) * 4
    w = np.array([(i * 17 + 3) & 0xFF for i in range(nbytes)], np.uint8).view(np.uint32)
    w = w.reshape(E, N, H // 16)
    x = S.f32_to_half_bits(np.array([(i % 17 - 8) * 0.01 for i in range(M * H)], np.float32))
    x = x.reshape(M, H)
    s = np.full((E, N, H // gs), S.f32_to_half_bits(np.array([0.02], np.float32))[0], np.uint16)
    b = np.full((E, N, H // gs), S.f32_to_half_bits(np.array([-0.02], np.float32))[0], np.uint16)
    inds = np.array([[1, 3], [2, 5]], np.int32)
    wd = torch.from_numpy(w.view(np.int32)).to(DEV)
    sd, bd = dev16(s, 0), dev16(b, 0)
    yM = torch.empty(M * Ktop, N, dtype=torch.bfloat16, device=DEV)
    ws = moe.new_workspace(M, Ktop, 0, 0)
    moe.gqmm2(dev16(x, 0), wd, sd, bd, torch.from_numpy(inds).to(DEV), yM, Ktop=Ktop, K=H, N=N,
              gs=gs, M=M, workspace=ws)
    seq = []
    for m in range(M):
        y1 = torch.empty(Ktop, N, dtype=torch.bfloat16, device=DEV)
        moe.gqmm2(dev16(x[m:m + 1], 0), wd, sd, bd, torch.from_numpy(inds[m:m + 1]).to(DEV), y1,
                  Ktop=Ktop, K=H, N=N, gs=gs, M=1, workspace=moe.new_workspace(1, Ktop, 0, 0))
        seq.append(host16(y1))
    torch.cuda.synchronize()
    assert (host16(yM) == np.concatenate(seq)).all()
    ref = O.gqmm2(x, w, s, b, inds, M, Ktop, H, N, gs)
    assert_parity(host16(yM), ref, 0, "mrow fixture")


@pytest.mark.parametrize("M,H,I,E,K,gs,dt", [
    (1, 512, 256, 8, 4, 64, 0),
    (8, 1024, 512, 32, 8, 64, 0),
    (2, 768, 1280, 16, 4, 128, 1),
])
def test_up_swiglu_matches_oracle(M, H, I, E, K, gs, dt):
    w = S.expert_weights(E, H, I, gs, seed=4, dtype=dt)
    x = S.activations(M, H, seed=4, dtype=dt)
    inds, scores = O.route(S.logits_ar1(M, E, seed=4), K)
    ug = O.gqmm2(x, w["w_ug"], w["s_ug"], w["b_ug"], inds, M, K, H, 2 * I, gs, False, dt)
    act_ref = O.clamped_swiglu(ug, I, 7.0, dt)
    dw = dev_weights(w, dt)
    act = torch.empty(M * K, I, dtype=TD[dt], device=DEV)
    ws = moe.new_workspace(M, K, 0, 0)
    moe.gqmm2_up_swiglu(dev16(x, dt), dw["w_ug"], dw["s_ug"], dw["b_ug"],
                        torch.from_numpy(inds).to(DEV), act, Ktop=K, K=H, I=I, gs=gs, M=M,
                        workspace=ws)
    moe.synchronize(workspace=ws)
    assert_parity(host16(act), act_ref, dt, "up_swiglu", atol_frac=1e-4)
    # the unfused path (gqmm2 N=2I + elementwise SwiGLU) agrees too
    ugd = torch.empty(M * K, 2 * I, dtype=TD[dt], device=DEV)
    moe.gqmm2(dev16(x, dt), dw["w_ug"], dw["s_ug"], dw["b_ug"], torch.from_numpy(inds).to(DEV), ugd,
              Ktop=K, K=H, N=2 * I, gs=gs, M=M, workspace=ws)
    act2 = torch.empty_like(act)
    moe.clamped_swiglu(ugd, act2, I=I, rows=M * K)
    torch.cuda.synchronize()
    assert_parity(host16(ugd), ug, dt, "gqmm2 up||gate")
    assert (host16(act2) == host16(act)).all()


@pytest.mark.parametrize("M,H,I,E,K,gs,dt", [
    (1, 2048, 1024, 64, 4, 64, 0),   # BASELINE config 0 shapes
    (4, 1024, 512, 16, 4, 64, 0),
    (2, 512, 768, 12, 3, 128, 1),
    (1, 1024, 512, 16, 4, 64, 1),    # fp16 on the streaming kernel
    (3, 2048, 1024, 32, 8, 64, 1),   # fp16, three tokens in one streaming launch, K = 8
])
def test_fused_expert_matches_oracle(M, H, I, E, K, gs, dt):
    w = S.expert_weights(E, H, I, gs, seed=9, dtype=dt)
    x = S.activations(M, H, seed=9, dtype=dt)
    inds, scores = O.route(S.logits_normal(M, E, seed=9), K)
    y_ref, st = O.expert_ffn(x, w, inds, scores, M, H, I, K, gs, 7.0, dt)
    y, _ = run_ffn(x, w, inds, scores, M, H, I, K, gs, dt)
    assert_ffn_parity(y, y_ref, st["down"], scores, dt, "fused expert")
    # score_resid variant: h += y with the two-kernel rounding
    h0 = S.normal_half(M * H, 9, 77, dt).reshape(M, H)
    h_ref, _ = O.expert_ffn(x, w, inds, scores, M, H, I, K, gs, 7.0, dt, resid_h=h0)
    h, _ = run_ffn(x, w, inds, scores, M, H, I, K, gs, dt, resid=h0)
    assert_ffn_parity(h, h_ref, st["down"], scores, dt, "fused expert resid")


@pytest.mark.parametrize("M,H,I,E,K,gs,dt,rho", [
    (1, 1024, 512, 16, 4, 64, 0, None),
    (8, 2048, 1024, 64, 8, 64, 0, 0.7),
    (3, 768, 1536, 24, 6, 128, 1, 0.7),
    (5, 4096, 256, 32, 8, 64, 0, None),
])
def test_fused_layer_and_multikernel_path_match_oracle(M, H, I, E, K, gs, dt, rho, monkeypatch):
    """The one-kernel decode layers (the streaming kernel, one launch for a
    batch of up to 8 tokens, and the batched tcgen05 kernel) and the
    multi-kernel path (route/plan, up, down, combine kernels on the GEMV
    engine) all match the oracle, call after call on one workspace (the
    grid-barrier and completion counters return to zero); repeated calls of
    the fused layer give the same bits."""
    w = S.expert_weights(E, H, I, gs, seed=13, dtype=dt)
    dw = dev_weights(w, dt)
    ws = moe.new_workspace(M, K, H, I)
    outs = {}
    for path in ("1", "tc", "0"):  # fused (streaming kernel), batched tcgen05, multi-kernel
        monkeypatch.setenv("MOMIJ_FUSED", "0" if path == "0" else "1")
        monkeypatch.setenv("MOMIJ_DECODE_MROW", "tc" if path == "tc" else "auto")
        for call in range(4):
            lay = call % 2  # calls 2 and 3 repeat the inputs of calls 0 and 1
            x = S.activations(M, H, layer=lay, seed=13, dtype=dt)
            lg = (S.logits_ar1(M, E, rho, lay, 13) if rho else S.logits_normal(M, E, lay, 13))
            y = torch.empty(M, H, dtype=TD[dt], device=DEV)
            h0 = S.normal_half(M * H, 13, 99, dt).reshape(M, H)
            h = dev16(h0, dt)
            inds = torch.empty(M, K, dtype=torch.int32, device=DEV)
            scores = torch.empty(M, K, dtype=torch.float32, device=DEV)
            moe.forward(torch.from_numpy(lg).to(DEV), dev16(x, dt), dw, y, H=H, I=I, Ktop=K, gs=gs,
                        M=M, inds=inds, scores=scores, workspace=ws)
            moe.forward(torch.from_numpy(lg).to(DEV), dev16(x, dt), dw, None, H=H, I=I, Ktop=K,
                        gs=gs, M=M, resid_h=h, workspace=ws)
            moe.synchronize(workspace=ws)
            outs[(path, call)] = (host16(y), host16(h), inds.cpu().numpy(), scores.cpu().numpy())
            i_ref, s_ref = O.route(lg, K)
            y_ref, st = O.expert_ffn(x, w, i_ref, s_ref, M, H, I, K, gs, 7.0, dt)
            h_ref, _ = O.expert_ffn(x, w, i_ref, s_ref, M, H, I, K, gs, 7.0, dt, resid_h=h0)
            assert (outs[(path, call)][2] == i_ref).all()
            assert_ffn_parity(outs[(path, call)][0], y_ref, st["down"], s_ref, dt, f"path {path} call {call}")
            assert_ffn_parity(outs[(path, call)][1], h_ref, st["down"], s_ref, dt, f"path {path} call {call} resid")
    for path in ("1", "tc"):
        for call in (2, 3):
            for a, b in zip(outs[(path, call)], outs[(path, call - 2)]):
                assert (a == b).all(), (path, call)


def test_fused_expert_mrow_matches_sequential():
    """Batched M=4 equals four M=1 steps exactly (MomijCoreTests.swift:317-405)."""
    M, H, I, E, K, gs = 4, 1024, 512, 16, 4, 64
    w = S.expert_weights(E, H, I, gs, seed=21)
    x = S.activations(M, H, seed=21)
    inds, scores = O.route(S.logits_ar1(M, E, seed=21), K)
    yM, _ = run_ffn(x, w, inds, scores, M, H, I, K, gs, 0)
    for m in range(M):
        y1, _ = run_ffn(x[m:m + 1], w, inds[m:m + 1], scores[m:m + 1], 1, H, I, K, gs, 0)
        assert (y1 == yM[m:m + 1]).all(), m


def test_golden_vectors_on_gpu():
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_moe.npz"))
    meta = json.loads(bytes(z["meta"]).decode())
    for c in meta:
        M, H, I, E, K, gs, dt = (c[k] for k in ("M", "H", "I", "E", "Ktop", "gs", "dtype"))
        w = S.expert_weights(E, H, I, gs, layer=0, seed=c["seed"], dtype=dt)
        x = S.activations(M, H, layer=0, seed=c["seed"], dtype=dt)
        lg = (S.logits_ar1(M, E, 0.7, 0, c["seed"]) if c["logits"] == "ar1"
              else S.logits_normal(M, E, 0, c["seed"]))
        dw = dev_weights(w, dt)
        y = torch.empty(M, H, dtype=TD[dt], device=DEV)
        inds = torch.empty(M, K, dtype=torch.int32, device=DEV)
        scores = torch.empty(M, K, dtype=torch.float32, device=DEV)
        ws = moe.new_workspace(M, K, H, I)
        moe.forward(torch.from_numpy(lg).to(DEV), dev16(x, dt), dw, y, H=H, I=I, Ktop=K, gs=gs, M=M,
                    inds=inds, scores=scores, workspace=ws)
        moe.synchronize(workspace=ws)
        assert (inds.cpu().numpy() == z[c["name"] + "/inds"]).all(), c["name"]
        np.testing.assert_allclose(scores.cpu().numpy(), z[c["name"] + "/scores"], rtol=2e-6)
        assert_ffn_parity(host16(y), z[c["name"] + "/y"], z[c["name"] + "/down"],
                          z[c["name"] + "/scores"], dt, c["name"])


# ---- BASELINE shapes (one layer at full size) ------------------------------

def _gather_host_weights(wd: dict, experts: np.ndarray) -> dict:
    idx = torch.from_numpy(experts.astype(np.int64)).to(DEV)
    out = {}
    for k, v in wd.items():
        a = v.index_select(0, idx).contiguous()
        a = a.view(torch.int32 if k.startswith("w_") else torch.int16).cpu().numpy()
        out[k] = a.view(np.uint32 if k.startswith("w_") else np.uint16)
    return out


@pytest.mark.parametrize("M,rho", [(1, None), (8, 0.7)])
def test_config1_config2_layer_matches_oracle(M, rho):
    """BASELINE configs 1 (M=1) and 2 (M=8, rho=0.7): H=4096, E=128, top-8,
    I=1536, gs64.  The oracle runs on the selected experts only."""
    H, I, E, K, gs = 4096, 1536, 128, 8, 64
    wd = moe.device_expert_weights(E, H, I, gs, layer=0, seed=0)
    x = S.activations(M, H, layer=0, seed=0)
    lg = S.logits_ar1(M, E, rho, 0, 0) if rho else S.logits_normal(M, E, 0, 0)
    y = torch.empty(M, H, dtype=torch.bfloat16, device=DEV)
    inds = torch.empty(M, K, dtype=torch.int32, device=DEV)
    scores = torch.empty(M, K, dtype=torch.float32, device=DEV)
    ws = moe.new_workspace(M, K, H, I)
    moe.forward(torch.from_numpy(lg).to(DEV), dev16(x, 0), wd, y, H=H, I=I, Ktop=K, gs=gs, M=M,
                inds=inds, scores=scores, workspace=ws)
    moe.synchronize(workspace=ws)
    i_ref, s_ref = O.route(lg, K)
    assert (inds.cpu().numpy() == i_ref).all()
    uniq, remap = np.unique(i_ref, return_inverse=True)
    wh = _gather_host_weights(wd, uniq)
    y_ref, st = O.expert_ffn(x, wh, remap.reshape(M, K).astype(np.int32), s_ref, M, H, I, K, gs)
    assert_ffn_parity(host16(y), y_ref, st["down"], s_ref, 0, f"config M={M}")


# ---- error behaviour ---------------------------------------------------------

def test_expert_index_out_of_range_is_reported():
    M, H, I, E, K = 1, 256, 256, 4, 2
    w = dev_weights(S.expert_weights(E, H, I, 64), 0)
    x = dev16(S.activations(M, H), 0)
    y = torch.zeros(M, H, dtype=torch.bfloat16, device=DEV)
    ws = moe.new_workspace(M, K, H, I)
    bad = torch.tensor([[1, 4]], dtype=torch.int32, device=DEV)
    sc = torch.tensor([[0.5, 0.5]], dtype=torch.float32, device=DEV)
    moe.expert_ffn(x, w, bad, sc, y, H=H, I=I, Ktop=K, M=M, workspace=ws)
    with pytest.raises(moe.SeedlessError) as ei:
        moe.synchronize(workspace=ws)
    assert ei.value.status == moe.EXPERT_INDEX
    assert (y.cpu() == 0).all()  # nothing written
    # the workspace stays usable for a valid call afterwards
    good = torch.tensor([[1, 3]], dtype=torch.int32, device=DEV)
    moe.expert_ffn(x, w, good, sc, y, H=H, I=I, Ktop=K, M=M, workspace=ws)
    moe.synchronize(workspace=ws)


def test_unsupported_shapes_are_refused_on_the_host():
    x = torch.zeros(1, 100, dtype=torch.bfloat16, device=DEV)
    w = torch.zeros(2, 8, 7, dtype=torch.int32, device=DEV)
    s = torch.zeros(2, 8, 2, dtype=torch.bfloat16, device=DEV)
    out = torch.zeros(1, 8, dtype=torch.bfloat16, device=DEV)
    inds = torch.zeros(1, 1, dtype=torch.int32, device=DEV)
    for K, gs in ((100, 64), (512, 32), (8192, 64)):
        with pytest.raises(moe.SeedlessError) as ei:
            moe.gqmm2(x, w, s, s, inds, out, Ktop=1, K=K, N=8, gs=gs, M=1)
        assert ei.value.status == moe.UNSUPPORTED_SHAPE


def test_empty_batch_is_a_no_op():
    w = dev_weights(S.expert_weights(4, 256, 256, 64), 0)
    x = torch.zeros(0, 256, dtype=torch.bfloat16, device=DEV)
    y = torch.zeros(0, 256, dtype=torch.bfloat16, device=DEV)
    inds = torch.zeros(0, 2, dtype=torch.int32, device=DEV)
    sc = torch.zeros(0, 2, dtype=torch.float32, device=DEV)
    moe.expert_ffn(x, w, inds, sc, y, H=256, I=256, Ktop=2, M=0,
                   workspace=moe.new_workspace(1, 2, 256, 256))
    torch.cuda.synchronize()


# ---- large batches with few tokens per expert (expert-parallel sizes) ---------

@pytest.mark.parametrize("M,H,I,E,K", [
    (64, 4096, 512, 64, 8),   # slices shrink to fit the token digits: CTAs loop over slices
    (24, 1024, 512, 256, 8),
])
def test_large_batch_gemv_path_matches_oracle(M, H, I, E, K):
    """M > 8 with fewer than 32 pairs per expert stays on the GEMV path
    (units of <= 4 pairs, per-vector digits)."""
    gs = 64
    w = S.expert_weights(E, H, I, gs, seed=21)
    x = S.activations(M, H, seed=21)
    inds, scores = O.route(S.logits_normal(M, E, seed=21), K)
    y_ref, st = O.expert_ffn(x, w, inds, scores, M, H, I, K, gs)
    y, _ = run_ffn(x, w, inds, scores, M, H, I, K, gs, 0)
    assert_ffn_parity(y, y_ref, st["down"], scores, 0, f"large batch M={M}")
    # and through moe.forward (router on the GPU)
    dw = dev_weights(w, 0)
    xd = dev16(x, 0)
    yd = torch.empty(M, H, dtype=torch.bfloat16, device=DEV)
    ws = moe.new_workspace(M, K, H, I)
    moe.forward(torch.from_numpy(S.logits_normal(M, E, seed=21)).to(DEV), xd, dw, yd, H=H, I=I, Ktop=K,
                M=M, workspace=ws)
    moe.synchronize(workspace=ws)
    # the GPU router's scores may differ from the oracle's in the last bit
    # (fp32 softmax), so this leg is held to the oracle tolerance
    assert_ffn_parity(host16(yd), y_ref, st["down"], scores, 0, f"large batch forward M={M}")


def test_workspace_reuse_across_batch_sizes():
    """One workspace for calls of different batch sizes (it is carved per
    call, so a large call's buffers overlap a small call's counters): the
    fused kernels clear their completion counters themselves."""
    H, I, E, K, gs = 1024, 512, 32, 4, 64
    wd = moe.device_expert_weights(E, H, I, gs, seed=3)
    w = S.expert_weights(E, H, I, gs, seed=3)
    ws = moe.new_workspace(64, K, H, I)
    for M in (64, 8, 1, 64, 1):
        x = S.activations(M, H, seed=M)
        lg = S.logits_normal(M, E, 0, M)
        y = torch.zeros(M, H, dtype=torch.bfloat16, device=DEV)
        moe.forward(torch.from_numpy(lg).to(DEV), dev16(x, 0), wd, y, H=H, I=I, Ktop=K, gs=gs, M=M, workspace=ws)
        moe.synchronize(workspace=ws)
        i_ref, s_ref = O.route(lg, K)
        ref, _ = O.expert_ffn(x, w, i_ref, s_ref, M, H, I, K, gs)
        g, r = O.np_half_to_f64(host16(y)), O.np_half_to_f64(ref)
        rel = np.sqrt(((g - r) ** 2).sum(1)) / np.sqrt((r ** 2).sum(1))
        assert rel.max() <= 2e-3, (M, rel.max())
