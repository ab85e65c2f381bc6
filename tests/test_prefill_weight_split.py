"""Why the prefill grouped GEMM multiplies hi + lo bf16 weight tiles
(`momij_b200/csrc/prefill.cu`): a CPU model at config-3 shapes (H = 4096,
I = 1536, E = 128, top-8, Zipf(1.1) routing) of the expert FFN with the
dequantised weight w = s*q + b entered three ways, every GEMV accumulated in
float64 and every staged rounding of the reference path kept:

* exact w (the oracle's arithmetic);
* hi + lo, hi = bf16(w), lo = bf16(w - hi) -- the kernel's split (two
  kind::f16 MMAs with the same bf16 activation tile);
* one fp16 rounding of w (activations converted to fp16, exact for them),
  the cheaper single-MMA alternative.

Over the 10 sampled tokens the split gives the exact weights' outputs bit
for bit, while the single fp16 rounding already misses the 2e-3 per-row bar
before any fp32 accumulation error (median row 2.1e-3, worst 2.7e-3):
the path's staged bf16 roundings turn its small weight errors into one-ulp
flips of about a quarter of the outputs.
"""
from __future__ import annotations

import numpy as np

from momij_b200 import synth as S
from oracle import oracle as O

H, I, E, K, GS = 4096, 1536, 128, 8, 64


def _bf16(v32: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 (ties to even), returned as float32."""
    u = v32.astype(np.float32).view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return r.view(np.float32)


def _dequant32(w, s, b):
    """Dense float32 s*q + b (exact in float32 for bf16 scales and biases)."""
    N, words = w.shape
    shifts = (2 * np.arange(16, dtype=np.uint32))[None, None, :]
    q = ((w[:, :, None] >> shifts) & np.uint32(3)).reshape(N, words * 16).astype(np.float32)
    sf = np.repeat(S.half_bits_to_f32(s).reshape(N, -1), GS, axis=1)
    bf = np.repeat(S.half_bits_to_f32(b).reshape(N, -1), GS, axis=1)
    return sf * q + bf


def _variants(W32):
    """The three weight matrices, each exact in float32."""
    hi = _bf16(W32)
    return {"exact": W32, "hilo": hi + _bf16(W32 - hi), "f16": W32.astype(np.float16).astype(np.float32)}


def _r16(v, dtype=0):
    return O.np_half_to_f64(O.np_f64_to_half(v, dtype), dtype)


def test_hi_lo_split_meets_the_bar_and_one_fp16_rounding_does_not_leave_room():
    T = 10
    lg = S.logits_zipf(2048, E, 1.1)
    rows = np.linspace(0, 2047, T).astype(int)
    inds, scores = O.route(lg[rows], K)
    x = O.np_half_to_f64(S.activations(2048, H)[rows], 0)
    out = {m: np.zeros((T, H)) for m in ("exact", "hilo", "f16")}
    for e in np.unique(inds):  # one expert at a time, all of its tokens together
        t, k = np.nonzero(inds == e)
        w = S.expert_weights_one(int(e), H, I, GS)
        ug_w = _variants(_dequant32(w["w_ug"], w["s_ug"], w["b_ug"]))
        dn_w = _variants(_dequant32(w["w_dn"], w["s_dn"], w["b_dn"]))
        for mode in out:
            xv = _r16(x[t], 1) if mode == "f16" else x[t]
            ug = _r16(xv @ ug_w[mode].T.astype(np.float64))
            u = np.clip(ug[:, :I], -7.0, 7.0)
            g = np.minimum(ug[:, I:], 7.0)
            act = _r16(g / (1.0 + np.exp(-g)) * u)
            av = _r16(act, 1) if mode == "f16" else act
            dn = _r16(av @ dn_w[mode].T.astype(np.float64))
            # the combine in float64 (the same order for every variant)
            np.add.at(out[mode], t, dn * scores[t, k][:, None])
    ref = _r16(out["exact"])
    rel = {}
    for mode in ("hilo", "f16"):
        got = _r16(out[mode])
        rel[mode] = np.sqrt(((got - ref) ** 2).sum(axis=1)) / np.sqrt((ref ** 2).sum(axis=1))
    assert rel["hilo"].max() <= 1e-3, rel["hilo"].max()
    assert np.median(rel["f16"]) >= 1e-3, np.median(rel["f16"])
