"""CPU tests of the C ABI: the library loads, exports every declared symbol,
and its host-side logic (status strings, sizes, refusals) works without a GPU.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from momij_b200 import moe, synth as S


def test_library_exports_every_header_symbol():
    syms = moe.header_symbols()
    assert len(syms) >= 14
    lib = ctypes.CDLL(moe.LIB_PATH)
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing


def test_status_strings_and_version():
    assert moe.status_string(moe.OK) == "ok"
    assert moe.status_string(moe.UNSUPPORTED_SHAPE) == "unsupported shape"
    assert moe.status_string(moe.EXPERT_INDEX) == "expert index out of range"
    assert moe.status_string(12345) == "unknown status"
    assert moe.lib.momij_version() >= 100


def test_workspace_size_grows_with_pairs():
    a = moe.workspace_size(1, 8, 4096, 1536)
    b = moe.workspace_size(8, 8, 4096, 1536)
    assert 0 < a < b
    # plan (8-int header + 5 ints per pair) + act + down + inds + scores + one
    # completion counter per 64 output rows + the grouped path's tables
    # (offsets for up to 1024 experts, pair ids, weights, status words, block
    # list of up to P/128 + 1025 blocks) + its exact-recomputation list (a
    # 16-B count, 16-B entries for one in 8 up||gate outputs), 256-B aligned
    P, I = 8, 1536
    up = lambda n: -(-n // 256) * 256
    grp = 4 * (1025 + 2 * P + 4 + 4 + 4 * (P // 128 + 1024 + 1))
    fix = 16 + 16 * -(-P * I // 8)
    expect = (up(4 * (8 + 5 * P)) + P * I * 2 + P * 4096 * 2 + 256 + 256 + 256 + up(grp) + up(fix))
    assert a == expect
    assert moe.workspace_size(-1, 8, 16, 16) == 0


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device refusal")
def test_entry_points_refuse_without_device():
    lib = moe.lib
    rc = lib.momij_moe_route(None, 1, 8, 2, None, None, None)
    assert rc == moe.NO_DEVICE
    rc = lib.momij_moe_gqmm2(None, None, None, None, None, None, 1, 1, 256, 8, 4, 64, 0, 0,
                             None, 0, None)
    assert rc == moe.NO_DEVICE


def test_synth_generator_moments_and_ranges():
    x = S.normal_f32(200_000, 0, 8)
    assert abs(float(x.mean())) < 0.01 and abs(float(x.std()) - 1.0) < 0.01
    assert np.abs(x).max() <= 6.0
    s = S.half_bits_to_f32(S.affine_uniform(100_000, S.SCALE_A, S.SCALE_C, 0, 1))
    assert s.min() >= 0.00499 and s.max() <= 0.02002
    b = S.half_bits_to_f32(S.affine_uniform(100_000, S.BIAS_A, S.BIAS_C, 0, 2))
    assert b.min() >= -0.0301 and b.max() <= 0.0
    c = S.codes(50_000, 0, 0)
    q = (c[:, None] >> (2 * np.arange(16, dtype=np.uint32))[None, :]) & 3
    counts = np.bincount(q.ravel().astype(np.int64), minlength=4) / q.size
    assert np.allclose(counts, 0.25, atol=0.005)


def test_ar1_logits_share_experts():
    lg = S.logits_ar1(8, 128, 0.7)
    top = np.argsort(-lg, axis=1)[:, :8]
    overlap = [len(set(top[t]) & set(top[t - 1])) / 8 for t in range(1, 8)]
    assert 0.2 < float(np.mean(overlap)) < 0.9


def test_zipf_logits_are_skewed():
    lg = S.logits_zipf(2048, 128, 1.1)
    top = np.argsort(-lg, axis=1)[:, :8]
    cnt = np.bincount(top.ravel(), minlength=128)
    assert cnt.max() > 10 * cnt.min() and cnt.min() >= 1
