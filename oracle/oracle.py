"""Python access to the CPU oracle (TEST INFRASTRUCTURE ONLY).

Two independent restatements of the reference's MoE expert semantics live
here, so that each can check the other:

* ``C`` -- ctypes bindings to ``lib/libmomij_oracle.so`` (moe_oracle.c), the
  oracle the GPU parity tests and the CPU baseline use.
* ``np_*`` -- a float64 numpy restatement written from the dense dequantised
  weight matrix ``W = s*q + b`` (MLX affine, MapleMoE.swift:65-75 via
  SeedlessMetal.swift:2145-2221), a different formulation from the C code's
  per-group ``s*sum(q*x) + b*sum(x)`` factorisation.

Parity against MLX gather_qmm itself is unpinned: MLX (mlx-swift 0.31.6) is
not vendored and cannot run here.  Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg may use this module.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libmomij_oracle.so")

_u16p = ctypes.POINTER(ctypes.c_uint16)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_i32p = ctypes.POINTER(ctypes.c_int32)
_f32p = ctypes.POINTER(ctypes.c_float)


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        c_int, c_float = ctypes.c_int, ctypes.c_float
        L.oracle_route.argtypes = [_f32p, c_int, c_int, c_int, _i32p, _f32p]
        L.oracle_permute.argtypes = [_i32p, _f32p, c_int, c_int, c_int, _i32p, _i32p, _f32p]
        L.oracle_gqmm2.argtypes = [_u16p, _u32p, _u16p, _u16p, _i32p, _u16p] + [c_int] * 8
        L.oracle_clamped_swiglu.argtypes = [_u16p, _u16p, c_int, c_int, c_float, c_int]
        L.oracle_score_reduce.argtypes = [_u16p, _f32p, _u16p, c_int, c_int, c_int, c_int]
        L.oracle_score_resid.argtypes = [_u16p, _f32p, _u16p, c_int, c_int, c_int, c_int]
        L.oracle_expert_ffn.argtypes = ([_u16p, _u32p, _u16p, _u16p, _u32p, _u16p, _u16p, _i32p,
                                         _f32p, _u16p, _u16p] + [c_int] * 6 + [c_float, c_int]
                                        + [_u16p] * 3)
        L.oracle_half_to_double.argtypes = [ctypes.c_uint16, c_int]
        L.oracle_half_to_double.restype = ctypes.c_double
        L.oracle_double_to_half.argtypes = [ctypes.c_double, c_int]
        L.oracle_double_to_half.restype = ctypes.c_uint16
        L.oracle_num_threads.restype = c_int
        L.oracle_set_num_threads.argtypes = [c_int]
        _lib = L
    return _lib


def _p(a: np.ndarray, t):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(t)


class OracleError(RuntimeError):
    pass


def route(logits: np.ndarray, K: int):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    M, E = logits.shape
    inds = np.zeros((M, K), np.int32)
    scores = np.zeros((M, K), np.float32)
    rc = lib().oracle_route(_p(logits, _f32p), M, E, K, _p(inds, _i32p), _p(scores, _f32p))
    if rc:
        raise OracleError(f"oracle_route rc={rc}")
    return inds, scores


def permute(inds: np.ndarray, scores: np.ndarray, E: int):
    inds = np.ascontiguousarray(inds, np.int32)
    scores = np.ascontiguousarray(scores, np.float32)
    M, K = inds.shape
    off = np.zeros(E + 1, np.int32)
    pair = np.zeros(M * K, np.int32)
    wt = np.zeros(M * K, np.float32)
    rc = lib().oracle_permute(_p(inds, _i32p), _p(scores, _f32p), M, K, E, _p(off, _i32p),
                              _p(pair, _i32p), _p(wt, _f32p))
    if rc:
        raise OracleError(f"oracle_permute rc={rc}")
    return off, pair, wt


def gqmm2(x, w, s, b, inds, M, Ktop, Kdim, N, gs, lhs_per_expert=False, dtype=0):
    E = w.shape[0]
    out = np.zeros((M * Ktop, N), np.uint16)
    rc = lib().oracle_gqmm2(_p(x, _u16p), _p(w, _u32p), _p(s, _u16p), _p(b, _u16p),
                            _p(np.ascontiguousarray(inds, np.int32), _i32p), _p(out, _u16p),
                            M, Ktop, Kdim, N, E, gs, int(lhs_per_expert), dtype)
    if rc:
        raise OracleError(f"oracle_gqmm2 rc={rc}")
    return out


def clamped_swiglu(ug: np.ndarray, I: int, clamp: float = 7.0, dtype: int = 0):
    rows = ug.shape[0]
    act = np.zeros((rows, I), np.uint16)
    lib().oracle_clamped_swiglu(_p(ug, _u16p), _p(act, _u16p), rows, I, clamp, dtype)
    return act


def score_reduce(down, scores, M, Ktop, H, dtype=0):
    y = np.zeros((M, H), np.uint16)
    lib().oracle_score_reduce(_p(down, _u16p), _p(np.ascontiguousarray(scores, np.float32), _f32p),
                              _p(y, _u16p), M, Ktop, H, dtype)
    return y


def score_resid(down, scores, h, M, Ktop, H, dtype=0):
    """h = cast(h + cast(sum_k score * down)) in k order (maple_score_resid); returns a copy."""
    h = np.ascontiguousarray(h.copy())
    lib().oracle_score_resid(_p(np.ascontiguousarray(down), _u16p),
                             _p(np.ascontiguousarray(scores, np.float32), _f32p), _p(h, _u16p), M, Ktop,
                             H, dtype)
    return h


def expert_ffn(x, wts: dict, inds, scores, M, H, I, Ktop, gs, clamp=7.0, dtype=0,
               resid_h: np.ndarray | None = None):
    """Returns (y, staged) where staged holds the rounded intermediates."""
    E = wts["w_ug"].shape[0]
    y = np.zeros((M, H), np.uint16)
    ug = np.zeros((M * Ktop, 2 * I), np.uint16)
    act = np.zeros((M * Ktop, I), np.uint16)
    down = np.zeros((M * Ktop, H), np.uint16)
    h = None if resid_h is None else np.ascontiguousarray(resid_h.copy())
    rc = lib().oracle_expert_ffn(
        _p(x, _u16p), _p(wts["w_ug"], _u32p), _p(wts["s_ug"], _u16p), _p(wts["b_ug"], _u16p),
        _p(wts["w_dn"], _u32p), _p(wts["s_dn"], _u16p), _p(wts["b_dn"], _u16p),
        _p(np.ascontiguousarray(inds, np.int32), _i32p),
        _p(np.ascontiguousarray(scores, np.float32), _f32p), _p(y, _u16p),
        None if h is None else _p(h, _u16p), M, H, I, E, Ktop, gs, clamp, dtype,
        _p(ug, _u16p), _p(act, _u16p), _p(down, _u16p))
    if rc:
        raise OracleError(f"oracle_expert_ffn rc={rc}")
    return (h if h is not None else y), {"ug": ug, "act": act, "down": down}


def num_threads() -> int:
    return int(lib().oracle_num_threads())


def set_num_threads(n: int) -> None:
    lib().oracle_set_num_threads(int(n))


# ---- independent float64 numpy restatement --------------------------------

def np_half_to_f64(h: np.ndarray, dtype: int = 0) -> np.ndarray:
    h = np.asarray(h, np.uint16)
    if dtype == 1:
        return h.view(np.float16).astype(np.float64)
    return (h.astype(np.uint32) << np.uint32(16)).view(np.float32).astype(np.float64)


def np_f64_to_half(v: np.ndarray, dtype: int = 0) -> np.ndarray:
    """Round float64 straight to bf16/fp16 (ties to even) via frexp/rint."""
    v = np.asarray(v, np.float64)
    mant = 10 if dtype == 1 else 7
    expb = 5 if dtype == 1 else 8
    bias = (1 << (expb - 1)) - 1
    emin = 1 - bias
    a = np.abs(v)
    _, e = np.frexp(a)
    e = np.maximum(e - 1, emin)
    q = np.ldexp(1.0, e - mant)
    r = np.rint(a / q) * q
    with np.errstate(over="ignore"):
        if dtype == 1:
            out = r.astype(np.float16).view(np.uint16)
        else:
            out = (r.astype(np.float32).view(np.uint32) >> np.uint32(16)).astype(np.uint16)
    out = np.where(np.signbit(v), out | np.uint16(0x8000), out).astype(np.uint16)
    return out


def np_dequant(w: np.ndarray, s: np.ndarray, b: np.ndarray, gs: int, dtype: int = 0) -> np.ndarray:
    """[N, K/16] u32 + [N, K/gs] scales/biases -> dense float64 [N, K]."""
    N, words = w.shape
    shifts = (2 * np.arange(16, dtype=np.uint32))[None, None, :]
    q = ((w[:, :, None] >> shifts) & np.uint32(3)).reshape(N, words * 16).astype(np.float64)
    sf = np.repeat(np_half_to_f64(s, dtype), gs, axis=1)
    bf = np.repeat(np_half_to_f64(b, dtype), gs, axis=1)
    return sf * q + bf


def np_route(logits: np.ndarray, K: int):
    """Independent restatement of the router: the selection order of
    maple_route_top8's strict-'>' reduction tree (SeedlessMetal.swift:
    2764-2775) is, among equal values, the smallest bit-reversed index over the
    tree's width (256, or the next power of two above E); without NaN logits
    this is a sort by (value descending, bit-reversed index ascending)."""
    lg32 = np.asarray(logits, np.float32)
    lg = lg32.astype(np.float64)
    M, E = lg.shape
    W = 256
    while W < E:
        W *= 2
    bits = W.bit_length() - 1
    e = np.arange(E)
    rev = np.zeros(E, np.int64)
    for i in range(bits):
        rev |= ((e >> i) & 1) << (bits - 1 - i)
    val = np.where(lg == 0.0, 0.0, lg)  # -0 == +0
    order = np.lexsort((np.broadcast_to(rev, lg.shape), -val), axis=1)[:, :K]
    p = np.exp(lg - lg.max(axis=1, keepdims=True))
    p /= p.sum(axis=1, keepdims=True)
    sel = np.take_along_axis(p, order, axis=1)
    return order.astype(np.int32), (sel / sel.sum(axis=1, keepdims=True)).astype(np.float32)


def tree_route_indices(logits_row: np.ndarray, K: int) -> list[int]:
    """Literal step-by-step replay of maple_route_top8's selection loop
    (SeedlessMetal.swift:2764-2781) for one token: K rounds of a 256-wide (or
    wider, for E > 256) reduction in which position t < s takes t + s only if
    strictly greater; selected experts and positions >= E drop out.  Pure
    Python: small cases only."""
    lg = [float(v) for v in np.asarray(logits_row, np.float32)]
    E = len(lg)
    W = 256
    while W < E:
        W *= 2
    used = set()
    out = []
    for _ in range(K):
        red = [lg[t] if t < E else float("-inf") for t in range(W)]
        ri = list(range(W))
        live = [t < E and t not in used for t in range(W)]
        s = W // 2
        while s > 0:
            for t in range(s):
                if live[t + s] and (not live[t] or red[t + s] > red[t]):
                    red[t], ri[t], live[t] = red[t + s], ri[t + s], True
            s //= 2
        out.append(ri[0])
        used.add(ri[0])
    return out


def np_gqmm2(x, w, s, b, inds, M, Ktop, gs, lhs_per_expert=False, dtype=0):
    inds = np.asarray(inds).reshape(-1)
    xf = np_half_to_f64(x, dtype)
    outs = []
    for mk in range(M * Ktop):
        e = int(inds[mk])
        W = np_dequant(w[e], s[e], b[e], gs, dtype)
        xr = xf[mk if lhs_per_expert else mk // Ktop]
        outs.append(W @ xr)
    return np_f64_to_half(np.stack(outs), dtype)


def np_expert_ffn(x, wts, inds, scores, M, H, I, Ktop, gs, clamp=7.0, dtype=0):
    ug = np_gqmm2(x, wts["w_ug"], wts["s_ug"], wts["b_ug"], inds, M, Ktop, gs, False, dtype)
    u = np.clip(np_half_to_f64(ug[:, :I], dtype), -clamp, clamp)
    g = np.minimum(np_half_to_f64(ug[:, I:], dtype), clamp)
    act = np_f64_to_half(g / (1.0 + np.exp(-g)) * u, dtype)
    dn = np_gqmm2(act, wts["w_dn"], wts["s_dn"], wts["b_dn"], inds, M, Ktop, gs, True, dtype)
    d = np_half_to_f64(dn, dtype).reshape(M, Ktop, H)
    y = (d * np.asarray(scores, np.float64).reshape(M, Ktop, 1)).sum(axis=1)
    return np_f64_to_half(y, dtype), {"ug": ug, "act": act, "down": dn}


# ---- router GEMV, fused router, RMSNorm (numpy restatements) --------------

def gate_logits(x, w_gate, x_dtype: int = 0, w_dtype: int = 0) -> np.ndarray:
    """Router logits [M, E] = x [M, H] W_gate [E, H]^T from the 16-bit bit
    patterns, in float64 (every product exact, the sum to ~2^-50):
    maple_batched_gemv / maple_gate_gemv (SeedlessMetal.swift:2542-2595)
    without their fp32 rounding."""
    return np_half_to_f64(x, x_dtype) @ np_half_to_f64(w_gate, w_dtype).T


def _f32(v):
    return np.float32(v)


def fused_router(logits_f32: np.ndarray, K: int):
    """MapleFused.fusedRouter's selection and scores (MapleFused.swift:
    139-240) on given fp32 logits, with its fp32 staging and summation order:
    max; e_j = exp(l_j - max); the sum per thread t over j = t, t+256, ...,
    then a 32-lane shuffle-down tree, then the eight simdgroups in order;
    p_j = e_j * (1 / (sum + 1e-20)); top-K over p with the scan's tie order
    (lower simdgroup, then smaller bit-reversed lane, then lower j within a
    thread); scores p_k / (sum_k p_k + 1e-20), the sum in selection order.
    Pure Python loops over E: small cases only."""
    lg = np.asarray(logits_f32, np.float32)
    M, E = lg.shape
    inds = np.zeros((M, K), np.int32)
    scores = np.zeros((M, K), np.float32)

    def rev5(v):
        return int(f"{v:05b}"[::-1], 2)

    for m in range(M):
        row = lg[m]
        mx = _f32(row.max())
        ev = np.exp((row - mx).astype(np.float64)).astype(np.float32)
        part = [np.float32(0)] * 256
        for t in range(256):
            acc = np.float32(0)
            for j in range(t, E, 256):
                acc = _f32(acc + ev[j])
            part[t] = acc
        sg_sums = []
        for sg in range(8):
            lane = [part[sg * 32 + l] for l in range(32)]
            off = 16
            while off >= 1:
                for l in range(32 - off):
                    lane[l] = _f32(lane[l] + lane[l + off])
                off //= 2
            sg_sums.append(lane[0])
        tot = sg_sums[0]
        for v in sg_sums[1:]:
            tot = _f32(tot + v)
        inv = _f32(np.float32(1.0) / _f32(tot + np.float32(1e-20)))
        p = (ev * inv).astype(np.float32)
        key = [(-float(p[j]), ((j & 255) >> 5), rev5(j & 31), j) for j in range(E)]
        order = sorted(range(E), key=lambda j: key[j])[:K]
        sel = [p[j] for j in order]
        ssum = np.float32(0)
        for v in sel:
            ssum = _f32(ssum + v)
        inds[m] = order
        scores[m] = [_f32(v / _f32(ssum + np.float32(1e-20))) for v in sel]
    return inds, scores


def rms_norm(x, w, eps: float, dtype: int = 0) -> np.ndarray:
    """maple_rms_norm (SeedlessMetal.swift:2496-2527): inv = 1/sqrt(sum x^2 / H
    + eps) (here from a float64 sum, rounded to fp32), out = round((x * inv)
    * w) with both products rounded to fp32, then to the 16-bit dtype."""
    xf = np_half_to_f64(x, dtype)
    wf = np_half_to_f64(w, dtype)
    H = xf.shape[1]
    ss = (xf * xf).sum(axis=1)
    inv = (1.0 / np.sqrt((ss / H).astype(np.float32).astype(np.float64) + np.float32(eps))).astype(np.float32)
    t = (xf.astype(np.float32) * inv[:, None]).astype(np.float32)
    o = (t * wf.astype(np.float32)).astype(np.float32)
    return np_f64_to_half(o.astype(np.float64), dtype)
