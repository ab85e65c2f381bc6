"""Python host interface over libmomij_moe.so (the C ABI in include/momij_moe.h).

Names and argument meanings mirror the reference's operator surface
(momij swift/Sources/MomijCore/SeedlessMetal.swift: ``gqmm2`` :312-438,
``gqmm2UpSwiglu`` :441-484, ``encodeClampedSwiglu`` :486-498,
``encodeFusedExpert``/``fusedExpertStep`` :503-572, ``encodeRoute``
:1266-1281; MapleSeedlessMoE.swift ``SeedlessMoELayer.run`` :61-77), and
errors surface as :class:`SeedlessError` carrying the C status code, as the
reference throws ``SeedlessError.unsupportedShape`` / ``.notReady``.

Tensors are torch tensors used only as device memory: weights are uint32
(packed codes) and int16/uint16-sized 16-bit buffers (bf16 or fp16, passed
as ``torch.bfloat16``/``torch.float16``), indices int32, logits/scores fp32.
There is no CPU fallback: if the CUDA library is missing this module raises
at import time.
"""
from __future__ import annotations

import ctypes
import os
import re

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("MOMIJ_LIB_PATH") or os.path.join(HERE, "lib", "libmomij_moe.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "momij_moe.h")

OK, UNSUPPORTED_SHAPE, NOT_READY, NO_DEVICE, INVALID_ARGUMENT = 0, 1, 2, 3, 4
EXPERT_INDEX, WORKSPACE, CUDA, NCCL, TIMEOUT, STOPPED = 5, 6, 7, 8, 9, 10
DTYPE_BF16, DTYPE_F16 = 0, 1
MAX_PAIRS = 1024          # gqmm2 surfaces (MOMIJ_MAX_PAIRS)
MAX_GROUPED_PAIRS = 65536  # expert_ffn / forward through the grouped path


class SeedlessError(RuntimeError):
    """Raised for a non-zero status from the C ABI (mirrors SeedlessError)."""

    def __init__(self, status: int, where: str = ""):
        self.status = int(status)
        super().__init__(f"{where}: {status_string(status)} (status {status})")


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m momij_b200.build` "
            "(the MoE path has no CPU fallback)")
    L = ctypes.CDLL(LIB_PATH)
    vp, i, f, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
    L.momij_status_string.argtypes = [i]
    L.momij_status_string.restype = ctypes.c_char_p
    L.momij_version.restype = i
    L.momij_device_sm_count.restype = i
    L.momij_moe_synchronize.argtypes = [vp, vp]
    L.momij_moe_route.argtypes = [vp, i, i, i, vp, vp, vp]
    L.momij_moe_permute.argtypes = [vp, vp, i, i, i, vp, vp, vp, vp]
    L.momij_moe_workspace_size.argtypes = [i, i, i, i]
    L.momij_moe_workspace_size.restype = sz
    L.momij_moe_gqmm2.argtypes = [vp] * 6 + [i] * 8 + [vp, sz, vp]
    L.momij_moe_gqmm2_up_swiglu.argtypes = [vp] * 6 + [i] * 6 + [f, i, vp, sz, vp]
    L.momij_moe_clamped_swiglu.argtypes = [vp, vp, i, i, f, i, vp]
    L.momij_moe_score_reduce.argtypes = [vp, vp, vp, i, i, i, i, vp]
    L.momij_moe_score_resid.argtypes = [vp, vp, vp, i, i, i, i, vp]
    L.momij_moe_expert_ffn.argtypes = [vp] * 11 + [i] * 6 + [f, i, vp, sz, vp]
    L.momij_moe_forward.argtypes = [vp] * 12 + [i] * 6 + [f, i, vp, sz, vp]
    L.momij_moe_ep_dispatch.argtypes = [vp, vp] + [i] * 6 + [vp, vp, vp, vp, vp]
    L.momij_moe_ep_combine.argtypes = [vp, vp, vp, vp, vp, i, i, i, i, vp, vp]
    L.momij_synth_fill.argtypes = [vp, ctypes.c_int64, i, f, f, ctypes.c_uint64,
                                   ctypes.c_uint64, ctypes.c_int64, i, vp]
    L.momij_moe_router_logits.argtypes = [vp, vp, vp, i, i, i, i, i, vp]
    L.momij_moe_fused_router.argtypes = [vp] * 6 + [i] * 6 + [vp]
    L.momij_rms_norm.argtypes = [vp, vp, vp, i, i, f, i, vp]
    L.momij_moe_block_workspace_size.argtypes = [i, i, i, i, i]
    L.momij_moe_block_workspace_size.restype = sz
    L.momij_moe_block.argtypes = [vp, vp, f, vp, i] + [vp] * 8 + [i] * 6 + [f, i, vp, sz, vp]
    L.momij_nccl_unique_id.argtypes = [vp]
    L.momij_moe_ep_init.argtypes = [vp, vp] + [i] * 8 + [f, i, ctypes.POINTER(vp)]
    L.momij_moe_ep_forward.argtypes = [vp] * 13 + [i, vp]
    L.momij_moe_ep_status.argtypes = [vp, vp]
    L.momij_moe_ep_destroy.argtypes = [vp]
    L.momij_set_stop_flag.argtypes = [vp]
    L.momij_set_spin_limit.argtypes = [i]
    L.momij_profile_enable.argtypes = [i]
    L.momij_layer_trace.argtypes = [vp, sz]
    L.momij_profile_read.argtypes = [i, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(i)]
    return L


lib = _load()


def status_string(status: int) -> str:
    return lib.momij_status_string(int(status)).decode()


def header_symbols() -> list[str]:
    """Function names declared in include/momij_moe.h."""
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(momij_[a-z_0-9]+)\s*\(",
                                 src, re.M)))


def _check(rc: int, where: str) -> None:
    if rc != OK:
        raise SeedlessError(rc, where)


def _ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_contiguous():
        raise ValueError("tensors must be contiguous")
    return t.data_ptr()


def _stream(stream) -> int | None:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    return int(stream)


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return DTYPE_BF16
    if t.dtype == torch.float16:
        return DTYPE_F16
    raise TypeError(f"activations must be bf16 or fp16, got {t.dtype}")


def workspace_size(M: int, Ktop: int, H: int, I: int) -> int:
    return int(lib.momij_moe_workspace_size(M, Ktop, H, I))


def new_workspace(M: int, Ktop: int, H: int, I: int, device=None) -> torch.Tensor:
    """Zero-filled workspace (the kernels keep it reusable across calls)."""
    n = max(workspace_size(M, Ktop, H, I), 256)
    return torch.zeros(n, dtype=torch.uint8, device=device or "cuda")


def synchronize(stream=None, workspace: torch.Tensor | None = None) -> None:
    _check(lib.momij_moe_synchronize(_stream(stream), _ptr(workspace)), "synchronize")


def set_stop_flag(flag: torch.Tensor | None) -> None:
    """Process-wide stop flag (a device int32 tensor, or None): non-zero makes
    every later call skip its work and report STOPPED (the reference's
    stopFlag buffer)."""
    if flag is not None and (flag.dtype != torch.int32 or not flag.is_cuda):
        raise TypeError("the stop flag is a CUDA int32 tensor")
    _check(lib.momij_set_stop_flag(_ptr(flag)), "set_stop_flag")


def set_spin_limit(polls: int) -> None:
    """Bound of the device-side waits (0: default, -1: give up at once)."""
    _check(lib.momij_set_spin_limit(int(polls)), "set_spin_limit")


# ---- router -----------------------------------------------------------------

def route(logits: torch.Tensor, K: int, inds: torch.Tensor | None = None,
          scores: torch.Tensor | None = None, stream=None):
    """encodeRoute: logits [M,E] fp32 -> (inds [M,K] int32, scores [M,K] fp32)."""
    M, E = logits.shape
    inds = inds if inds is not None else torch.empty(M, K, dtype=torch.int32, device=logits.device)
    scores = scores if scores is not None else torch.empty(M, K, dtype=torch.float32,
                                                           device=logits.device)
    _check(lib.momij_moe_route(_ptr(logits), M, E, K, _ptr(inds), _ptr(scores), _stream(stream)),
           "route")
    return inds, scores


def permute(inds: torch.Tensor, scores: torch.Tensor, E: int, stream=None):
    M, K = inds.shape
    dev = inds.device
    off = torch.empty(E + 1, dtype=torch.int32, device=dev)
    pair = torch.empty(M * K, dtype=torch.int32, device=dev)
    wt = torch.empty(M * K, dtype=torch.float32, device=dev)
    _check(lib.momij_moe_permute(_ptr(inds), _ptr(scores), M, K, E, _ptr(off), _ptr(pair),
                                 _ptr(wt), _stream(stream)), "permute")
    return off, pair, wt


# ---- gather-GEMV operators (SeedlessMetal surface) ---------------------------

def gqmm2(x, w, scales, biases, inds, out, *, Ktop: int, K: int, N: int, gs: int = 64,
          lhs_per_expert: bool = False, M: int = 1, workspace=None, stream=None):
    """out[M*Ktop, N] = gather-qmv of x[M or M*Ktop, K] with experts inds[M*Ktop]."""
    E = w.shape[0]
    ws = workspace if workspace is not None else new_workspace(M, Ktop, 0, 0, x.device)
    _check(lib.momij_moe_gqmm2(_ptr(x), _ptr(w), _ptr(scales), _ptr(biases), _ptr(inds),
                               _ptr(out), M, Ktop, K, N, E, gs, int(lhs_per_expert),
                               _dtype_code(x), _ptr(ws), ws.numel(), _stream(stream)), "gqmm2")
    return out


def gqmm2_up_swiglu(x, w, scales, biases, inds, out, *, Ktop: int, K: int, I: int, gs: int = 64,
                    M: int = 1, clamp: float = 7.0, workspace=None, stream=None):
    E = w.shape[0]
    ws = workspace if workspace is not None else new_workspace(M, Ktop, 0, 0, x.device)
    _check(lib.momij_moe_gqmm2_up_swiglu(_ptr(x), _ptr(w), _ptr(scales), _ptr(biases), _ptr(inds),
                                         _ptr(out), M, Ktop, K, I, E, gs, clamp, _dtype_code(x),
                                         _ptr(ws), ws.numel(), _stream(stream)), "gqmm2UpSwiglu")
    return out


def ep_dispatch(inds, x, send_x, send_meta, slot_map, status, *, E: int, world: int,
                capacity: int, stream=None) -> None:
    """Expert-parallel dispatch (momij_moe_ep_dispatch): packs this rank's
    (token, slot) pairs into per-destination rows of send_x / send_meta."""
    M, K = inds.shape
    H = x.shape[1]
    _check(lib.momij_moe_ep_dispatch(_ptr(inds), _ptr(x), M, K, E, world, capacity, H, _ptr(send_x),
                                     _ptr(send_meta), _ptr(slot_map), _ptr(status), _stream(stream)),
           "epDispatch")


def ep_combine(back, scores, slot_map, status, y=None, *, resid_h=None, stream=None) -> None:
    """Expert-parallel combine (momij_moe_ep_combine) in k order."""
    M, K = scores.shape
    H = back.shape[1]
    out = resid_h if resid_h is not None else y
    _check(lib.momij_moe_ep_combine(_ptr(back), _ptr(scores), _ptr(slot_map),
                                    None if resid_h is not None else _ptr(y),
                                    _ptr(resid_h) if resid_h is not None else None, M, K, H,
                                    _dtype_code(out), _ptr(status), _stream(stream)), "epCombine")


def clamped_swiglu(ug, act, *, I: int, rows: int, clamp: float = 7.0, stream=None):
    _check(lib.momij_moe_clamped_swiglu(_ptr(ug), _ptr(act), rows, I, clamp, _dtype_code(ug),
                                        _stream(stream)), "clampedSwiglu")
    return act


def score_reduce(down, scores, y, *, H: int, Ktop: int, M: int = 1, stream=None):
    _check(lib.momij_moe_score_reduce(_ptr(down), _ptr(scores), _ptr(y), M, Ktop, H,
                                      _dtype_code(down), _stream(stream)), "scoreReduce")
    return y


def score_resid(down, scores, h, *, H: int, Ktop: int, M: int = 1, stream=None):
    _check(lib.momij_moe_score_resid(_ptr(down), _ptr(scores), _ptr(h), M, Ktop, H,
                                     _dtype_code(down), _stream(stream)), "scoreResid")
    return h


def expert_ffn(x, wts: dict, inds, scores, y=None, *, H: int, I: int, Ktop: int, gs: int = 64,
               M: int = 1, clamp: float = 7.0, resid_h=None, workspace=None, stream=None):
    """encodeFusedExpert: up||gate + SwiGLU, down, score-weighted combine."""
    E = wts["w_ug"].shape[0]
    ws = workspace if workspace is not None else new_workspace(M, Ktop, H, I, x.device)
    _check(lib.momij_moe_expert_ffn(
        _ptr(x), _ptr(wts["w_ug"]), _ptr(wts["s_ug"]), _ptr(wts["b_ug"]), _ptr(wts["w_dn"]),
        _ptr(wts["s_dn"]), _ptr(wts["b_dn"]), _ptr(inds), _ptr(scores), _ptr(y), _ptr(resid_h),
        M, H, I, E, Ktop, gs, clamp, _dtype_code(x), _ptr(ws), ws.numel(), _stream(stream)),
        "fusedExpert")
    return resid_h if resid_h is not None else y


def forward(logits, x, wts: dict, y=None, *, H: int, I: int, Ktop: int, gs: int = 64, M: int = 1,
            clamp: float = 7.0, inds=None, scores=None, resid_h=None, workspace=None,
            stream=None):
    """MapleMoE.callAsFunction: route from logits, then the expert FFN."""
    E = wts["w_ug"].shape[0]
    ws = workspace if workspace is not None else new_workspace(M, Ktop, H, I, x.device)
    _check(lib.momij_moe_forward(
        _ptr(logits), _ptr(x), _ptr(wts["w_ug"]), _ptr(wts["s_ug"]), _ptr(wts["b_ug"]),
        _ptr(wts["w_dn"]), _ptr(wts["s_dn"]), _ptr(wts["b_dn"]), _ptr(inds), _ptr(scores),
        _ptr(y), _ptr(resid_h), M, H, I, E, Ktop, gs, clamp, _dtype_code(x), _ptr(ws), ws.numel(),
        _stream(stream)), "moeForward")
    return resid_h if resid_h is not None else y


# ---- per-kernel timing ----------------------------------------------------------

KERNEL_PLAN, KERNEL_UP, KERNEL_ROWS, KERNEL_COMBINE, KERNEL_LAYER = 0, 1, 2, 3, 4


def profile_enable(on: bool = True) -> None:
    _check(lib.momij_profile_enable(int(on)), "profile_enable")


def profile_read(kernel_id: int) -> tuple[float, int]:
    """(total milliseconds, launches) recorded for one kernel id."""
    ms, n = ctypes.c_double(0.0), ctypes.c_int(0)
    _check(lib.momij_profile_read(kernel_id, ctypes.byref(ms), ctypes.byref(n)), "profile_read")
    return ms.value, n.value


def profile_reset() -> None:
    _check(lib.momij_profile_reset(), "profile_reset")


# ---- synthetic inputs on the device ------------------------------------------

def synth_fill(dst: torch.Tensor, kind: int, *, a: float = 0.0, c: float = 0.0, seed: int = 0,
               stream_id: int = 0, start: int = 0, stream=None) -> torch.Tensor:
    dtype = DTYPE_F16 if dst.dtype == torch.float16 else DTYPE_BF16
    _check(lib.momij_synth_fill(_ptr(dst), dst.numel(), kind, a, c, seed, stream_id, start, dtype,
                                _stream(stream)), "synth_fill")
    return dst


def device_expert_weights(E: int, H: int, I: int, gs: int = 64, layer: int = 0, seed: int = 0,
                          dtype=torch.bfloat16, device="cuda", experts: tuple | None = None) -> dict:
    """The tensors of momij_b200.synth.expert_weights, generated on the GPU;
    experts=(lo, hi) generates only that slice (an expert-parallel shard)."""
    from . import synth as S
    dt = dtype
    lo, hi = experts if experts is not None else (0, E)

    def codes(shape, kind):
        per = shape[1] * shape[2]
        t = torch.empty((hi - lo,) + shape[1:], dtype=torch.int32, device=device)
        return synth_fill(t, 0, seed=seed, stream_id=S.stream_id(layer, kind), start=lo * per)

    def half(shape, kind, a, c):
        per = shape[1] * shape[2]
        t = torch.empty((hi - lo,) + shape[1:], dtype=dt, device=device)
        return synth_fill(t, 1, a=a, c=c, seed=seed, stream_id=S.stream_id(layer, kind), start=lo * per)

    return {
        "w_ug": codes((E, 2 * I, H // 16), S.KIND_W_UG),
        "s_ug": half((E, 2 * I, H // gs), S.KIND_S_UG, S.SCALE_A, S.SCALE_C),
        "b_ug": half((E, 2 * I, H // gs), S.KIND_B_UG, S.BIAS_A, S.BIAS_C),
        "w_dn": codes((E, H, I // 16), S.KIND_W_DN),
        "s_dn": half((E, H, I // gs), S.KIND_S_DN, S.SCALE_A, S.SCALE_C),
        "b_dn": half((E, H, I // gs), S.KIND_B_DN, S.BIAS_A, S.BIAS_C),
    }


class MoELayer:
    """Per-layer weights + reusable workspace (SeedlessMoELayer analogue,
    MapleSeedlessMoE.swift:7-78): ``run(x, inds, scores) -> y``."""

    def __init__(self, wts: dict, *, H: int, I: int, Ktop: int, gs: int = 64, max_M: int = 8,
                 clamp: float = 7.0):
        self.wts, self.H, self.I, self.Ktop, self.gs, self.clamp = wts, H, I, Ktop, gs, clamp
        self.max_M = max_M
        self.workspace = new_workspace(max_M, Ktop, H, I, wts["w_ug"].device)

    def run(self, x, inds, scores, y=None, stream=None):
        M = x.shape[0]
        if M > self.max_M:
            raise SeedlessError(UNSUPPORTED_SHAPE, "MoELayer.run")
        y = y if y is not None else torch.empty(M, self.H, dtype=x.dtype, device=x.device)
        return expert_ffn(x, self.wts, inds, scores, y, H=self.H, I=self.I, Ktop=self.Ktop,
                          gs=self.gs, M=M, clamp=self.clamp, workspace=self.workspace,
                          stream=stream)


# ---- router GEMV, fused router, RMSNorm, MoE block ---------------------------

def router_logits(x: torch.Tensor, w_gate: torch.Tensor, logits: torch.Tensor | None = None, *,
                  stream=None) -> torch.Tensor:
    """logits [M, E] (fp32) = x [M, H] @ w_gate [E, H]^T (maple_batched_gemv)."""
    M, H = x.shape
    E = w_gate.shape[0]
    if logits is None:
        logits = torch.empty(M, E, dtype=torch.float32, device=x.device)
    _check(lib.momij_moe_router_logits(_ptr(x), _ptr(w_gate), _ptr(logits), M, H, E, _dtype_code(x),
                                       _dtype_code(w_gate), _stream(stream)), "router_logits")
    return logits


def fused_router(x: torch.Tensor, w_gate: torch.Tensor, K: int, counter: torch.Tensor, *, logits=None,
                 inds=None, scores=None, stream=None):
    """MapleFused.fusedRouter: gate GEMV + softmax + top-K + renormalisation in
    one launch; ``counter`` is a persistent zeroed int32/uint32 device word."""
    M, H = x.shape
    E = w_gate.shape[0]
    dev = x.device
    logits = torch.empty(M, E, dtype=torch.float32, device=dev) if logits is None else logits
    inds = torch.empty(M, K, dtype=torch.int32, device=dev) if inds is None else inds
    scores = torch.empty(M, K, dtype=torch.float32, device=dev) if scores is None else scores
    _check(lib.momij_moe_fused_router(_ptr(x), _ptr(w_gate), _ptr(counter), _ptr(logits), _ptr(inds),
                                      _ptr(scores), M, H, E, K, _dtype_code(x), _dtype_code(w_gate),
                                      _stream(stream)), "fused_router")
    return inds, scores


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor | None = None, *,
             stream=None) -> torch.Tensor:
    """maple_rms_norm: out = round((x * rsqrt(mean(x^2) + eps)) * w)."""
    M, H = x.shape
    out = torch.empty_like(x) if out is None else out
    _check(lib.momij_rms_norm(_ptr(x), _ptr(w), _ptr(out), M, H, float(eps), _dtype_code(x), _stream(stream)),
           "rms_norm")
    return out


def block_workspace_size(M: int, Ktop: int, H: int, I: int, E: int) -> int:
    return int(lib.momij_moe_block_workspace_size(M, Ktop, H, I, E))


def moe_block(h: torch.Tensor, norm_w: torch.Tensor, eps: float, w_gate: torch.Tensor, wts: dict, *,
              I: int, Ktop: int, gs: int = 64, clamp: float = 7.0, inds=None, scores=None, workspace=None,
              stream=None) -> torch.Tensor:
    """SeedlessMetal.encodeMoEBlock: h += MoE(rmsnorm(h)) in place (gate GEMV,
    top-K routing, experts with the fused score-residual rounding)."""
    M, H = h.shape
    E = w_gate.shape[0]
    need = block_workspace_size(M, Ktop, H, I, E)
    if workspace is None:  # zeroed: completion counters and barrier words start at zero
        workspace = torch.zeros(need, dtype=torch.uint8, device=h.device)
    _check(lib.momij_moe_block(_ptr(h), _ptr(norm_w), float(eps), _ptr(w_gate), _dtype_code(w_gate),
                               _ptr(wts["w_ug"]), _ptr(wts["s_ug"]), _ptr(wts["b_ug"]), _ptr(wts["w_dn"]),
                               _ptr(wts["s_dn"]), _ptr(wts["b_dn"]), _ptr(inds), _ptr(scores), M, H, I, E,
                               Ktop, gs, float(clamp), _dtype_code(h), _ptr(workspace), workspace.numel(),
                               _stream(stream)), "moe_block")
    return h


# ---- expert-parallel layer object (momij_moe_ep_*) ------------------------------

def nccl_unique_id() -> bytes:
    """128 bytes of a fresh ncclUniqueId (rank 0 makes it; every rank passes it
    to EpLayer)."""
    buf = ctypes.create_string_buffer(128)
    _check(lib.momij_nccl_unique_id(buf), "ncclUniqueId")
    return buf.raw


class EpLayer:
    """One rank of an expert-parallel MoE layer behind the C ABI: the
    communicator (made from ``unique_id`` for world > 1) and the exchange
    buffers for up to ``max_tokens`` tokens per call."""

    def __init__(self, *, rank: int, world: int, E: int, H: int, I: int, K: int, max_tokens: int,
                 gs: int = 64, clamp: float = 7.0, dtype=torch.bfloat16, unique_id: bytes | None = None):
        self.E, self.H, self.I, self.K, self.world = E, H, I, K, world
        code = DTYPE_BF16 if dtype == torch.bfloat16 else DTYPE_F16
        uid = ctypes.create_string_buffer(unique_id, 128) if unique_id is not None else None
        h = ctypes.c_void_p()
        _check(lib.momij_moe_ep_init(None, uid, rank, world, E, H, I, K, max_tokens, gs, float(clamp), code,
                                     ctypes.byref(h)), "epInit")
        self._h = h

    def forward(self, x: torch.Tensor, wts: dict, *, logits=None, inds=None, scores=None, y=None,
                resid_h=None, stream=None):
        """One layer for this rank's tokens x [M, H] with its local experts
        ``wts``; y (or resid_h, updated in place) receives the result.  Call
        ``status()`` before trusting the output."""
        M = x.shape[0]
        _check(lib.momij_moe_ep_forward(self._h, _ptr(logits), _ptr(inds), _ptr(scores), _ptr(x),
                                        _ptr(wts["w_ug"]), _ptr(wts["s_ug"]), _ptr(wts["b_ug"]),
                                        _ptr(wts["w_dn"]), _ptr(wts["s_dn"]), _ptr(wts["b_dn"]), _ptr(y),
                                        _ptr(resid_h), M, _stream(stream)), "epForward")
        return y if y is not None else resid_h

    def status(self, stream=None) -> None:
        """Synchronises the stream; raises SeedlessError on a failed layer."""
        _check(lib.momij_moe_ep_status(self._h, _stream(stream)), "epStatus")

    def close(self) -> None:
        if self._h:
            lib.momij_moe_ep_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
