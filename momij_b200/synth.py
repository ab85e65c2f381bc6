"""Seeded synthetic inputs for the 2-bit MoE path (one documented generator).

Every value is a pure function of ``(seed, stream, index)`` built from
integer hashing, so the numpy version here and the CUDA fill kernel in
``libmomij_moe.so`` (``momij_synth_fill``) produce bit-identical tensors:

* ``hash(seed, stream, i) = splitmix64(seed*C1 + stream*C2 + i)`` (64-bit
  wrap-around arithmetic).
* packed codes: the upper 32 bits of the hash, i.e. 16 codes uniform in
  {0..3} per uint32 (MLX affine 2-bit layout, code j at bits [2j, 2j+1]).
* uniform ``u = (hash >> 40) * 2**-24`` (exact in float32), mapped as
  ``a*u + c`` in float32 (two separately rounded operations), then rounded to
  bf16/fp16 with ties to even.  Scales use ``a=0.015, c=0.005``
  (~U(0.005, 0.02)), biases ``a=0.03, c=-0.03`` (~U(-0.03, 0)).
* normal: Irwin-Hall sum of twelve 16-bit uniforms taken from three hashes,
  ``(S - 393210) / 65536``; mean 0, variance 1, |x| <= 6, exact in float32.

The configurations in BASELINE.json ask for "N(0,1)" activations and logits;
the Irwin-Hall variate stands in for that (same first two moments), chosen
because it needs no transcendental function and is therefore reproducible
bit for bit on the host and on the GPU.

Streams: ``stream_id(layer, kind)`` with the kinds below.
"""
from __future__ import annotations

import numpy as np

M64 = np.uint64(0xFFFFFFFFFFFFFFFF)
C1 = np.uint64(0xD1B54A32D192ED03)
C2 = np.uint64(0x8CB92BA72F3D8DD7)

KIND_W_UG, KIND_S_UG, KIND_B_UG, KIND_W_DN, KIND_S_DN, KIND_B_DN = range(6)
KIND_X, KIND_LOGITS, KIND_RESID = 8, 9, 10

SCALE_A, SCALE_C = 0.015, 0.005
BIAS_A, BIAS_C = 0.03, -0.03

DT_BF16, DT_F16 = 0, 1


def stream_id(layer: int, kind: int) -> int:
    return layer * 16 + kind


def splitmix64(z: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = z + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def hash64(seed: int, stream: int, idx: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        base = np.uint64(seed) * C1 + np.uint64(stream) * C2
        return splitmix64(base + idx.astype(np.uint64))


def f32_to_half_bits(f: np.ndarray, dtype: int = DT_BF16) -> np.ndarray:
    """float32 -> bf16/fp16 bit patterns, round to nearest even."""
    f = np.asarray(f, dtype=np.float32)
    if dtype == DT_F16:
        return f.astype(np.float16).view(np.uint16)
    u = f.view(np.uint32).astype(np.uint64)
    r = (u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)
    nan = np.isnan(f)
    out = r.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def half_bits_to_f32(h: np.ndarray, dtype: int = DT_BF16) -> np.ndarray:
    h = np.asarray(h, dtype=np.uint16)
    if dtype == DT_F16:
        return h.view(np.float16).astype(np.float32)
    return (h.astype(np.uint32) << np.uint32(16)).view(np.float32)


def codes(n_words: int, seed: int, stream: int, start: int = 0) -> np.ndarray:
    idx = np.arange(start, start + n_words, dtype=np.uint64)
    return (hash64(seed, stream, idx) >> np.uint64(32)).astype(np.uint32)


def uniform01(n: int, seed: int, stream: int, start: int = 0) -> np.ndarray:
    idx = np.arange(start, start + n, dtype=np.uint64)
    h = hash64(seed, stream, idx) >> np.uint64(40)
    return h.astype(np.float32) * np.float32(2.0 ** -24)


def affine_uniform(n: int, a: float, c: float, seed: int, stream: int, dtype: int = DT_BF16,
                   start: int = 0) -> np.ndarray:
    u = uniform01(n, seed, stream, start)
    v = (np.float32(a) * u).astype(np.float32) + np.float32(c)
    return f32_to_half_bits(v.astype(np.float32), dtype)


def normal_f32(n: int, seed: int, stream: int, start: int = 0) -> np.ndarray:
    idx = np.arange(3 * start, 3 * (start + n), dtype=np.uint64)
    h = hash64(seed, stream, idx).reshape(n, 3)
    s = np.zeros(n, dtype=np.int64)
    for j in range(3):
        for t in range(4):
            s += ((h[:, j] >> np.uint64(16 * t)) & np.uint64(0xFFFF)).astype(np.int64)
    return ((s - 393210).astype(np.float64) / 65536.0).astype(np.float32)


def normal_half(n: int, seed: int, stream: int, dtype: int = DT_BF16, start: int = 0) -> np.ndarray:
    return f32_to_half_bits(normal_f32(n, seed, stream, start), dtype)


# ---- expert weights (MLX affine 2-bit, transpose=true layout) -------------

def expert_weights(E: int, H: int, I: int, gs: int = 64, layer: int = 0, seed: int = 0,
                   dtype: int = DT_BF16) -> dict:
    """w_ug [E,2I,H/16] u32 (rows < I are up, rows >= I gate), s_ug/b_ug
    [E,2I,H/gs]; w_dn [E,H,I/16], s_dn/b_dn [E,H,I/gs] (16-bit bit patterns)."""
    nug, ndn = E * 2 * I, E * H
    return {
        "w_ug": codes(nug * H // 16, seed, stream_id(layer, KIND_W_UG)).reshape(E, 2 * I, H // 16),
        "s_ug": affine_uniform(nug * H // gs, SCALE_A, SCALE_C, seed, stream_id(layer, KIND_S_UG),
                               dtype).reshape(E, 2 * I, H // gs),
        "b_ug": affine_uniform(nug * H // gs, BIAS_A, BIAS_C, seed, stream_id(layer, KIND_B_UG),
                               dtype).reshape(E, 2 * I, H // gs),
        "w_dn": codes(ndn * I // 16, seed, stream_id(layer, KIND_W_DN)).reshape(E, H, I // 16),
        "s_dn": affine_uniform(ndn * I // gs, SCALE_A, SCALE_C, seed, stream_id(layer, KIND_S_DN),
                               dtype).reshape(E, H, I // gs),
        "b_dn": affine_uniform(ndn * I // gs, BIAS_A, BIAS_C, seed, stream_id(layer, KIND_B_DN),
                               dtype).reshape(E, H, I // gs),
    }


def expert_weights_one(e: int, H: int, I: int, gs: int = 64, layer: int = 0, seed: int = 0,
                       dtype: int = DT_BF16) -> dict:
    """Expert e's slice of expert_weights(E, ...) for any E > e (the same
    elements of the same streams), without generating the other experts."""
    out = {}
    for k, kind, shape in (("w_ug", KIND_W_UG, (2 * I, H // 16)), ("w_dn", KIND_W_DN, (H, I // 16))):
        n = shape[0] * shape[1]
        out[k] = codes(n, seed, stream_id(layer, kind), e * n).reshape(shape)
    for k, kind, shape, a, c in (("s_ug", KIND_S_UG, (2 * I, H // gs), SCALE_A, SCALE_C),
                                 ("b_ug", KIND_B_UG, (2 * I, H // gs), BIAS_A, BIAS_C),
                                 ("s_dn", KIND_S_DN, (H, I // gs), SCALE_A, SCALE_C),
                                 ("b_dn", KIND_B_DN, (H, I // gs), BIAS_A, BIAS_C)):
        n = shape[0] * shape[1]
        out[k] = affine_uniform(n, a, c, seed, stream_id(layer, kind), dtype, e * n).reshape(shape)
    return out


def activations(M: int, H: int, layer: int = 0, seed: int = 0, dtype: int = DT_BF16) -> np.ndarray:
    return normal_half(M * H, seed, stream_id(layer, KIND_X), dtype).reshape(M, H)


def logits_normal(M: int, E: int, layer: int = 0, seed: int = 0) -> np.ndarray:
    return normal_f32(M * E, seed, stream_id(layer, KIND_LOGITS)).reshape(M, E)


def logits_ar1(M: int, E: int, rho: float = 0.7, layer: int = 0, seed: int = 0) -> np.ndarray:
    """Correlated router logits across consecutive tokens:
    z_t = rho*z_{t-1} + sqrt(1-rho^2)*eps_t (float32, eps Irwin-Hall normal)."""
    eps = normal_f32(M * E, seed, stream_id(layer, KIND_LOGITS)).reshape(M, E)
    z = np.empty_like(eps)
    z[0] = eps[0]
    a, c = np.float32(rho), np.float32(np.sqrt(1.0 - rho * rho))
    for t in range(1, M):
        z[t] = (a * z[t - 1]).astype(np.float32) + (c * eps[t]).astype(np.float32)
    return z


def logits_zipf(M: int, E: int, s: float = 1.1, layer: int = 0, seed: int = 0) -> np.ndarray:
    """Zipf(s)-skewed routing: log p_e + Gumbel noise, so that the top-K of a
    token's logits is a draw of K experts without replacement with
    probability proportional to p_e = (e+1)^-s / sum."""
    ranks = np.arange(1, E + 1, dtype=np.float64)
    logp = -s * np.log(ranks)
    logp -= np.log(np.exp(logp).sum())
    u = uniform01(M * E, seed, stream_id(layer, KIND_LOGITS)).astype(np.float64)
    u = np.clip(u, 2.0 ** -25, 1.0 - 2.0 ** -25)
    g = -np.log(-np.log(u))
    return (logp[None, :] + g.reshape(M, E)).astype(np.float32)


def unique_experts_per_layer(inds: np.ndarray) -> int:
    return int(np.unique(inds).size)


def expert_bytes(H: int, I: int, gs: int) -> int:
    """Algorithmic bytes of one expert: 3*H*I codes at 2 bits plus one 16-bit
    scale and bias per gs columns of each of the three projections."""
    codes_ug = (2 * I) * (H // 16) * 4
    sb_ug = (2 * I) * (H // gs) * 2 * 2
    codes_dn = H * (I // 16) * 4
    sb_dn = H * (I // gs) * 2 * 2
    return codes_ug + sb_ug + codes_dn + sb_dn
