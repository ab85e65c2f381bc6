"""Generates tests/golden/golden_moe.npz: golden vectors for the MoE path.

Each case's inputs come from the seeded generator in momij_b200/synth.py
(recorded by parameters and a SHA-256 of every input array, so the test can
prove it rebuilt the same inputs) and its outputs from the C oracle
(oracle/moe_oracle.c), cross-checked here against the independent float64
numpy restatement (oracle/oracle.py np_*) before anything is written.

Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from momij_b200 import synth as S  # noqa: E402
from oracle import oracle as O  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden_moe.npz")

# name, M, H, I, E, Ktop, gs, dtype, logits kind, seed
CASES = [
    ("bf16_gs64_m1", 1, 512, 256, 8, 4, 64, S.DT_BF16, "normal", 0),
    ("bf16_gs64_m4_ar1", 4, 256, 512, 16, 4, 64, S.DT_BF16, "ar1", 1),
    ("f16_gs128_m2", 2, 512, 256, 8, 2, 128, S.DT_F16, "normal", 2),
    ("bf16_gs128_m8_ar1", 8, 256, 256, 32, 8, 128, S.DT_BF16, "ar1", 3),
]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def case_inputs(M, H, I, E, Ktop, gs, dtype, lk, seed):
    w = S.expert_weights(E, H, I, gs, layer=0, seed=seed, dtype=dtype)
    x = S.activations(M, H, layer=0, seed=seed, dtype=dtype)
    lg = S.logits_ar1(M, E, 0.7, 0, seed) if lk == "ar1" else S.logits_normal(M, E, 0, seed)
    return w, x, lg


def main() -> None:
    arrays, meta = {}, []
    for name, M, H, I, E, Ktop, gs, dtype, lk, seed in CASES:
        w, x, lg = case_inputs(M, H, I, E, Ktop, gs, dtype, lk, seed)
        inds, scores = O.route(lg, Ktop)
        i2, s2 = O.np_route(lg, Ktop)
        assert (inds == i2).all() and np.allclose(scores, s2, rtol=1e-6, atol=0)
        y, st = O.expert_ffn(x, w, inds, scores, M, H, I, Ktop, gs, 7.0, dtype)
        y2, st2 = O.np_expert_ffn(x, w, inds, scores, M, H, I, Ktop, gs, 7.0, dtype)
        assert (y == y2).all() and all((st[k] == st2[k]).all() for k in st)
        hashes = {k: sha(v) for k, v in w.items()}
        hashes.update(x=sha(x), logits=sha(lg))
        meta.append(dict(name=name, M=M, H=H, I=I, E=E, Ktop=Ktop, gs=gs, dtype=dtype, logits=lk,
                         seed=seed, input_sha256=hashes))
        arrays[f"{name}/inds"] = inds
        arrays[f"{name}/scores"] = scores
        arrays[f"{name}/ug"] = st["ug"]
        arrays[f"{name}/act"] = st["act"]
        arrays[f"{name}/down"] = st["down"]
        arrays[f"{name}/y"] = y
    arrays["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes, {len(CASES)} cases)")


if __name__ == "__main__":
    main()
