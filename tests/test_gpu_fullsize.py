"""Full-size parity of the BASELINE configurations that batch many tokens, on
one GPU, against the float64 oracle (per-row relative
L2 of y = MoE(x) <= 2e-3, router indices bit-exact):

  * config 3 -- prefill of 2048 tokens, hidden 4096, 128 experts, top-8,
    intermediate 1536, Zipf(1.1) routing (16 to ~900 tokens per expert), on
    the grouped tcgen05 path; 48 sampled rows, among them rows routed to the
    most and to the least loaded expert;
  * config 4 -- 64 tokens, hidden 4096, 256 experts, top-8, intermediate
    1024 (the expert-parallel configuration's batch, here on one GPU); every
    row.

The weights are generated on the GPU by the seeded generator (the same
stream the host generator produces); the oracle reads the selected experts
back to the host.
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

TOL = 2e-3


def _host_experts(W, experts):
    out = {}
    for k, t in W.items():
        sel = t[torch.as_tensor(experts, device=t.device, dtype=torch.long)]
        if k.startswith("w_"):
            out[k] = np.ascontiguousarray(sel.view(torch.int32).cpu().numpy().view(np.uint32))
        else:
            out[k] = np.ascontiguousarray(sel.view(torch.int16).cpu().numpy().view(np.uint16))
    return out


def _check_rows(W, x, lg, y, inds, rows, H, I, K, gs):
    """Rows `rows` of y and inds against the oracle (routing from the logits)."""
    i_ref, s_ref = O.route(np.ascontiguousarray(lg[rows]), K)
    assert (inds[rows] == i_ref).all(), "router indices differ from the reference's"
    uniq, remap = np.unique(i_ref, return_inverse=True)
    wh = _host_experts(W, uniq)
    n = len(rows)
    y_ref, _ = O.expert_ffn(np.ascontiguousarray(x[rows]), wh, remap.reshape(n, K).astype(np.int32), s_ref,
                            n, H, I, K, gs)
    g = O.np_half_to_f64(y[rows])
    r = O.np_half_to_f64(y_ref)
    rel = np.sqrt(((g - r) ** 2).sum(axis=1)) / np.maximum(np.sqrt((r ** 2).sum(axis=1)), 1e-30)
    return rel


def _forward(W, x, lg, M, H, I, K, gs):
    xd = torch.from_numpy(x.view(np.int16)).cuda().view(torch.bfloat16)
    y = torch.empty(M, H, dtype=torch.bfloat16, device="cuda")
    inds = torch.empty(M, K, dtype=torch.int32, device="cuda")
    scores = torch.empty(M, K, dtype=torch.float32, device="cuda")
    ws = moe.new_workspace(M, K, H, I)
    moe.forward(torch.from_numpy(lg).cuda(), xd, W, y, H=H, I=I, Ktop=K, gs=gs, M=M, inds=inds, scores=scores,
                workspace=ws)
    moe.synchronize(workspace=ws)
    return y.view(torch.int16).cpu().numpy().view(np.uint16), inds.cpu().numpy()


def test_config3_prefill_full_size():
    M, H, I, E, K, gs = 2048, 4096, 1536, 128, 8, 64
    W = moe.device_expert_weights(E, H, I, gs, layer=0, seed=0)
    x = S.activations(M, H, 0, 0)
    lg = S.logits_zipf(M, E, 1.1, 0, 0)
    y, inds = _forward(W, x, lg, M, H, I, K, gs)
    counts = np.bincount(inds.ravel(), minlength=E)
    busiest = int(counts.argmax())
    idlest = int(np.flatnonzero(counts)[counts[np.flatnonzero(counts)].argmin()])
    assert counts[busiest] >= 128, "Zipf(1.1) should put several row blocks on the busiest expert"
    rng = np.random.default_rng(0)
    rows = set(rng.choice(M, 16, replace=False).tolist())
    rows |= set(np.flatnonzero((inds == busiest).any(axis=1))[:16].tolist())
    rows |= set(np.flatnonzero((inds == idlest).any(axis=1))[:16].tolist())
    rows = np.array(sorted(rows))
    rel = _check_rows(W, x, lg, y, inds, rows, H, I, K, gs)
    print(f"config 3: {len(rows)} rows, busiest expert {busiest} ({counts[busiest]} tokens), "
          f"idlest {idlest} ({counts[idlest]}); worst row rel-L2 {rel.max():.3e}")
    assert rel.max() <= TOL, rel.max()


def test_config4_full_size_one_gpu():
    M, H, I, E, K, gs = 64, 4096, 1024, 256, 8, 64
    W = moe.device_expert_weights(E, H, I, gs, layer=0, seed=0)
    x = S.activations(M, H, 0, 0)
    lg = S.logits_normal(M, E, 0, 0)
    y, inds = _forward(W, x, lg, M, H, I, K, gs)
    rel = _check_rows(W, x, lg, y, inds, np.arange(M), H, I, K, gs)
    print(f"config 4 (one GPU): {M} rows, worst row rel-L2 {rel.max():.3e}")
    assert rel.max() <= TOL, rel.max()
