"""CPU tests of the oracle (the parity checker), pinned three ways:

* against the independent float64 numpy restatement (dense dequantised W);
* against exact rational arithmetic on the reference's own kernel-test
  fixture (momij MomijCoreTests.swift:264-274: weight bytes (i*17+3)&0xff,
  x = (i%17-8)*0.01, scales 0.02, biases -0.02);
* against the committed golden vectors (tests/golden/golden_moe.npz).
"""
from __future__ import annotations

import json
import os
from fractions import Fraction

import numpy as np
import pytest

from momij_b200 import synth as S
from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden_moe.npz")


@pytest.mark.parametrize("M,H,I,E,K,gs,dt", [
    (1, 256, 256, 4, 2, 64, 0),
    (3, 512, 256, 8, 3, 128, 0),
    (2, 256, 512, 6, 4, 64, 1),
    (1, 2048, 1024, 64, 4, 64, 0),  # BASELINE config 0 shapes
])
def test_c_oracle_matches_numpy_restatement(M, H, I, E, K, gs, dt):
    w = S.expert_weights(E, H, I, gs, dtype=dt, seed=7)
    x = S.activations(M, H, dtype=dt, seed=7)
    lg = S.logits_normal(M, E, seed=7)
    inds, scores = O.route(lg, K)
    y, st = O.expert_ffn(x, w, inds, scores, M, H, I, K, gs, 7.0, dt)
    y2, st2 = O.np_expert_ffn(x, w, inds, scores, M, H, I, K, gs, 7.0, dt)
    for k in ("ug", "act", "down"):
        assert (st[k] == st2[k]).all(), k
    assert (y == y2).all()


def tie_heavy_logits(M: int, E: int, seed: int, levels: int = 3) -> np.ndarray:
    """Logits drawn from a few values (with signed zeros) so that most
    selections are decided by the router's tie rule."""
    rng = np.random.default_rng(seed)
    vals = np.array([-0.0, 0.0] + [float(v) for v in np.linspace(-1.0, 1.0, levels)], np.float32)
    return vals[rng.integers(0, len(vals), size=(M, E))].astype(np.float32)


def test_route_matches_numpy_and_the_reference_tree():
    lg = S.logits_normal(16, 128, seed=3)
    i1, s1 = O.route(lg, 8)
    i2, s2 = O.np_route(lg, 8)
    assert (i1 == i2).all()
    np.testing.assert_allclose(s1, s2, rtol=1e-6, atol=0)
    np.testing.assert_allclose(s1.sum(axis=1), 1.0, rtol=1e-6)
    # descending logit order
    sel = np.take_along_axis(lg, i1, axis=1)
    assert (np.diff(sel, axis=1) <= 0).all()
    # exact ties go where maple_route_top8's strict-'>' tree puts them: the
    # smallest bit-reversed index, not the lowest index
    t = np.zeros((3, 16), np.float32)
    t[0, [3, 5, 9]] = 1.0
    t[1, :] = -2.0
    t[2, :] = -1.0
    t[2, 3], t[2, 5] = -0.0, 0.0  # signed zeros tie
    it, st = O.route(t, 4)
    assert it[0].tolist() == [9, 5, 3, 0]
    assert it[1].tolist() == [0, 8, 4, 12]
    assert it[2].tolist() == [5, 3, 0, 8]
    np.testing.assert_allclose(st[1], 0.25, rtol=1e-7)
    for m in range(3):
        assert it[m].tolist() == O.tree_route_indices(t[m], 4)


@pytest.mark.parametrize("E,K", [(16, 8), (64, 8), (128, 8), (256, 16), (300, 8)])
def test_route_follows_the_literal_tree_on_ties(E, K):
    lg = tie_heavy_logits(6, E, seed=E + K)
    i1, _ = O.route(lg, K)
    i2, _ = O.np_route(lg, K)
    assert (i1 == i2).all()
    for m in range(lg.shape[0]):
        assert i1[m].tolist() == O.tree_route_indices(lg[m], K)


def test_permute_is_a_stable_counting_sort():
    lg = S.logits_normal(9, 32, seed=5)
    inds, scores = O.route(lg, 4)
    off, pair, wt = O.permute(inds, scores, 32)
    flat = inds.reshape(-1)
    order = np.argsort(flat, kind="stable")
    assert (pair == order).all()
    assert (off == np.concatenate([[0], np.cumsum(np.bincount(flat, minlength=32))])).all()
    assert (wt == scores.reshape(-1)[order]).all()


def _exact_bf16(fr: Fraction) -> int:
    """Round an exact rational to bf16 bits, ties to even."""
    if fr == 0:
        return 0
    sign = 0x8000 if fr < 0 else 0
    a = abs(fr)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    if Fraction(2) ** e > a:
        e -= 1
    q = Fraction(2) ** (e - 7)
    r = a / q
    n = r.numerator // r.denominator
    rem = r - n
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and n % 2 == 1):
        n += 1
    v = n * q
    return sign | int(O.np_f64_to_half(np.array([float(v)]), 0)[0])


def test_reference_fixture_exact_rationals():
    """gqmm2 on the reference test fixture vs exact rational arithmetic."""
    H, N, E, Ktop, M, gs = 512, 16, 8, 2, 2, 64
    nbytes = E * N * (H // 16) * 4
    w = np.array([(i * 17 + 3) & 0xFF for i in range(nbytes)], np.uint8).view(np.uint32)
    w = w.reshape(E, N, H // 16)
    xv = np.array([(i % 17 - 8) * 0.01 for i in range(M * H)], np.float32)
    x = S.f32_to_half_bits(xv, 0).reshape(M, H)
    s = np.full((E, N, H // gs), S.f32_to_half_bits(np.array([0.02], np.float32))[0], np.uint16)
    b = np.full((E, N, H // gs), S.f32_to_half_bits(np.array([-0.02], np.float32))[0], np.uint16)
    inds = np.array([1, 3, 2, 5], np.int32)  # the reference test's indices
    out = O.gqmm2(x, w, s, b, inds, M, Ktop, H, N, gs)
    sv = Fraction(float(O.np_half_to_f64(s[0, 0, :1])[0]))
    bv = Fraction(float(O.np_half_to_f64(b[0, 0, :1])[0]))
    xf = [Fraction(float(v)) for v in O.np_half_to_f64(x.reshape(-1))]
    for mk in range(M * Ktop):
        e, m = int(inds[mk]), mk // Ktop
        for n in range(N):
            acc = Fraction(0)
            for k in range(H):
                q = (int(w[e, n, k // 16]) >> (2 * (k % 16))) & 3
                acc += (sv * q + bv) * xf[m * H + k]
            assert int(out[mk, n]) == _exact_bf16(acc), (mk, n)


def test_golden_vectors():
    z = np.load(GOLDEN)
    meta = json.loads(bytes(z["meta"]).decode())
    assert len(meta) >= 4
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "make_golden", os.path.join(os.path.dirname(GOLDEN), "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    case_inputs, sha = mg.case_inputs, mg.sha
    for c in meta:
        w, x, lg = case_inputs(c["M"], c["H"], c["I"], c["E"], c["Ktop"], c["gs"], c["dtype"],
                               c["logits"], c["seed"])
        got = {k: sha(v) for k, v in w.items()}
        got.update(x=sha(x), logits=sha(lg))
        assert got == c["input_sha256"], c["name"]
        inds, scores = O.route(lg, c["Ktop"])
        assert (inds == z[c["name"] + "/inds"]).all()
        np.testing.assert_array_equal(scores, z[c["name"] + "/scores"])
        y, st = O.expert_ffn(x, w, inds, scores, c["M"], c["H"], c["I"], c["Ktop"], c["gs"], 7.0,
                             c["dtype"])
        for k in ("ug", "act", "down"):
            assert (st[k] == z[c["name"] + "/" + k]).all(), (c["name"], k)
        assert (y == z[c["name"] + "/y"]).all(), c["name"]


def test_score_resid_two_kernel_rounding():
    rng = np.random.default_rng(0)
    M, K, H = 2, 3, 64
    down = S.f32_to_half_bits(rng.standard_normal((M * K, H)).astype(np.float32))
    sc = rng.random((M, K)).astype(np.float32)
    h0 = S.f32_to_half_bits(rng.standard_normal((M, H)).astype(np.float32))
    y = O.score_reduce(down, sc, M, K, H)
    h = h0.copy()
    O.lib().oracle_score_resid(down.ctypes.data_as(O._u16p), sc.ctypes.data_as(O._f32p),
                               h.ctypes.data_as(O._u16p), M, K, H, 0)
    expect = O.np_f64_to_half(O.np_half_to_f64(h0) + O.np_half_to_f64(y))
    assert (h == expect).all()


def test_bad_expert_index_is_rejected():
    w = S.expert_weights(4, 256, 256, 64)
    x = S.activations(1, 256)
    with pytest.raises(O.OracleError):
        O.gqmm2(x, w["w_ug"], w["s_ug"], w["b_ug"], np.array([0, 4], np.int32), 1, 2, 256, 512, 64)
