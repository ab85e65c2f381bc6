"""GPU test of momij_moe_gqmm2_noalloc, the gather-GEMV entry point for
callers that cannot allocate device memory (for example a binding that owns
only its inputs and outputs, or an engine that forbids cudaMalloc inside its
token loop).  It keeps its work plan in a fixed array inside the library
instead of a caller workspace.

The test calls it through the C ABI twice in a row, with different inputs,
and checks each output against momij_moe_gqmm2 (the workspace entry point)
on the same inputs: bit-identical, and within the parity tolerance used by
the other GPU tests.  The file is named to be collected last.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from momij_b200 import synth as S
from parity_util import assert_parity

pytestmark = pytest.mark.gpu


def _bind():
    from momij_b200 import moe
    fn = moe.lib.momij_moe_gqmm2_noalloc
    vp, i = ctypes.c_void_p, ctypes.c_int
    fn.argtypes = [vp] * 6 + [i] * 8 + [vp]
    fn.restype = i
    return moe, fn


def _case(M, Ktop, K, N, E, gs, lhs, seed):
    w = S.codes(E * N * K // 16, seed, 1).reshape(E, N, K // 16)
    s = S.affine_uniform(E * N * K // gs, S.SCALE_A, S.SCALE_C, seed, 2).reshape(E, N, K // gs)
    b = S.affine_uniform(E * N * K // gs, S.BIAS_A, S.BIAS_C, seed, 3).reshape(E, N, K // gs)
    rows = M * Ktop if lhs else M
    x = S.normal_half(rows * K, seed, 4).reshape(rows, K)
    inds = np.argsort(S.logits_normal(M, E, seed=seed), axis=1)[:, :Ktop].astype(np.int32)
    dev = "cuda"
    return dict(
        x=torch.from_numpy(x.view(np.int16)).to(dev).view(torch.bfloat16),
        w=torch.from_numpy(w.view(np.int32)).to(dev),
        s=torch.from_numpy(s.view(np.int16)).to(dev).view(torch.bfloat16),
        b=torch.from_numpy(b.view(np.int16)).to(dev).view(torch.bfloat16),
        inds=torch.from_numpy(inds).to(dev), M=M, Ktop=Ktop, K=K, N=N, E=E, gs=gs, lhs=lhs)


def test_noalloc_gqmm2_matches_workspace_entry_point_twice():
    moe, noalloc = _bind()
    stream = torch.cuda.current_stream().cuda_stream
    cases = [_case(1, 8, 2048, 96, 16, 64, False, 31), _case(2, 4, 1024, 80, 12, 128, True, 32)]
    for c in cases:
        P, N = c["M"] * c["Ktop"], c["N"]
        got = torch.full((P, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        rc = noalloc(c["x"].data_ptr(), c["w"].data_ptr(), c["s"].data_ptr(), c["b"].data_ptr(),
                     c["inds"].data_ptr(), got.data_ptr(), c["M"], c["Ktop"], c["K"], N, c["E"],
                     c["gs"], int(c["lhs"]), moe.DTYPE_BF16, stream)
        assert rc == moe.OK, moe.status_string(rc)
        ref = torch.empty_like(got)
        moe.gqmm2(c["x"], c["w"], c["s"], c["b"], c["inds"], ref, Ktop=c["Ktop"], K=c["K"], N=N,
                  gs=c["gs"], lhs_per_expert=c["lhs"], M=c["M"])
        torch.cuda.synchronize()
        g = got.view(torch.int16).cpu().numpy().view(np.uint16)
        r = ref.view(torch.int16).cpu().numpy().view(np.uint16)
        assert_parity(g, r, 0, "noalloc vs workspace gqmm2")
        assert (g == r).all()


def test_noalloc_rejects_sizes_beyond_its_array():
    moe, noalloc = _bind()
    z = torch.zeros(16, dtype=torch.int32, device="cuda")
    p = z.data_ptr()
    rc = noalloc(p, p, p, p, p, p, 129, 8, 256, 8, 4, 64, 0, moe.DTYPE_BF16, None)
    assert rc == moe.WORKSPACE


def test_noalloc_at_its_full_size_matches_the_oracle():
    """M*Ktop exactly MOMIJ_NOALLOC_MAX_PAIRS (the array's sizing) against the
    CPU oracle."""
    from oracle import oracle as O
    moe, noalloc = _bind()
    M, Ktop, K, N, E, gs = 128, 8, 512, 48, 16, 64
    assert M * Ktop == 1024
    w = S.codes(E * N * K // 16, 41, 1).reshape(E, N, K // 16)
    s = S.affine_uniform(E * N * K // gs, S.SCALE_A, S.SCALE_C, 41, 2).reshape(E, N, K // gs)
    b = S.affine_uniform(E * N * K // gs, S.BIAS_A, S.BIAS_C, 41, 3).reshape(E, N, K // gs)
    x = S.normal_half(M * K, 41, 4).reshape(M, K)
    inds = np.argsort(S.logits_normal(M, E, seed=41), axis=1)[:, :Ktop].astype(np.int32)
    ref = O.gqmm2(x, w, s, b, inds, M, Ktop, K, N, gs, False, 0)
    got = torch.full((M * Ktop, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda()
    xd, wd, sd, bd = d(x), torch.from_numpy(w.view(np.int32)).cuda(), d(s), d(b)  # alive across the call
    idd = torch.from_numpy(inds).cuda()
    rc = noalloc(xd.data_ptr(), wd.data_ptr(), sd.data_ptr(), bd.data_ptr(), idd.data_ptr(), got.data_ptr(), M,
                 Ktop, K, N, E, gs, 0, moe.DTYPE_BF16, torch.cuda.current_stream().cuda_stream)
    assert rc == moe.OK
    torch.cuda.synchronize()
    assert_parity(got.view(torch.int16).cpu().numpy().view(np.uint16), ref, 0, "noalloc at 1024 pairs")


def test_noalloc_bad_index_leaves_out_untouched_then_recovers():
    """An expert index out of range: the call writes nothing to `out` (it
    stays NaN); the next valid call rewrites the stale plan and is correct."""
    moe, noalloc = _bind()
    stream = torch.cuda.current_stream().cuda_stream
    c = _case(2, 4, 1024, 64, 8, 64, False, 33)
    P, N = c["M"] * c["Ktop"], c["N"]
    bad = c["inds"].clone()
    bad[1, 2] = c["E"]  # out of range
    got = torch.full((P, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    rc = noalloc(c["x"].data_ptr(), c["w"].data_ptr(), c["s"].data_ptr(), c["b"].data_ptr(), bad.data_ptr(),
                 got.data_ptr(), c["M"], c["Ktop"], c["K"], N, c["E"], c["gs"], 0, moe.DTYPE_BF16, stream)
    assert rc == moe.OK  # enqueued; the index error has no channel here
    torch.cuda.synchronize()
    assert torch.isnan(got.float()).all()
    rc = noalloc(c["x"].data_ptr(), c["w"].data_ptr(), c["s"].data_ptr(), c["b"].data_ptr(),
                 c["inds"].data_ptr(), got.data_ptr(), c["M"], c["Ktop"], c["K"], N, c["E"], c["gs"], 0,
                 moe.DTYPE_BF16, stream)
    assert rc == moe.OK
    ref = torch.empty_like(got)
    moe.gqmm2(c["x"], c["w"], c["s"], c["b"], c["inds"], ref, Ktop=c["Ktop"], K=c["K"], N=N, gs=c["gs"], M=c["M"])
    torch.cuda.synchronize()
    assert (got.view(torch.int16).cpu() == ref.view(torch.int16).cpu()).all()
