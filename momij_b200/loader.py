"""Maple checkpoint loading: sharded safetensors + ``sanitize`` into the tensors
the MoE kernels take.

Follows momij's WeightStore (swift/Sources/MomijCore/WeightStore.swift) and
MapleConfig (MapleConfig.swift):

* ``config.json`` -> :class:`MapleConfig` (the fields and defaults of
  MapleConfig.swift:5-48; ``expert_group_size`` = quantization.group_size,
  default 128, :140);
* ``model.safetensors.index.json`` -> ``weight_map``; every shard named there
  is read, in sorted order (WeightStore.swift:9-24);
* optionally bf16 -> fp16 (``WeightStore.metalF16``, :27-29; the reference
  converts for its Metal kernels, the CUDA kernels take either, so the
  default keeps the stored dtype);
* ``sanitize`` (:46-91): every ``<p>.row_alpha`` becomes ``<p>.scales`` =
  alpha repeated over the row's groups and ``<p>.biases`` = -scales (a 2-bit
  row with one alpha per row); per layer, q/k/v_proj {weight, scales,
  biases} are concatenated along rows into ``qkv_proj``, and the
  switch_mlp's up_proj and gate_proj along their output rows (axis 1) into
  ``up_gate_proj`` -- up rows first, the layout of the kernels' w_ug.

The safetensors container is read with numpy memory maps (the format: a
little-endian u64 header length, a JSON header of name -> dtype, shape,
data_offsets, then the data).  16-bit floats stay bit patterns (uint16).
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass, field

import numpy as np

_DT = {"BF16": np.uint16, "F16": np.uint16, "U32": np.uint32, "I32": np.int32, "F32": np.float32,
       "U8": np.uint8, "I64": np.int64, "U16": np.uint16, "I16": np.int16}


@dataclass
class MapleConfig:
    model_type: str = "maple"
    hidden_size: int = 2048
    intermediate_size: int = 5120
    moe_intermediate_size: int = 512
    num_hidden_layers: int = 24
    num_attention_heads: int = 16
    num_key_value_heads: int = 4
    head_dim: int = 128
    vocab_size: int = 151_936
    num_experts: int = 256
    num_experts_per_tok: int = 8
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10_000.0
    sliding_window: int = 512
    partial_rotary_factor: float = 0.5
    tie_word_embeddings: bool = False
    layer_types: list = field(default_factory=list)
    quantization: dict | None = None

    @property
    def expert_bits(self) -> int:
        return int((self.quantization or {}).get("bits", 2))

    @property
    def expert_group_size(self) -> int:
        return int((self.quantization or {}).get("group_size", 128))

    @classmethod
    def load(cls, model_dir: str) -> "MapleConfig":
        raw = json.load(open(os.path.join(model_dir, "config.json")))
        known = {k: v for k, v in raw.items() if k in cls.__dataclass_fields__}
        return cls(**known)


class SafetensorsTensor:
    """A tensor of a safetensors file: dtype name, shape and a numpy view."""

    def __init__(self, dtype: str, shape: list, data: np.ndarray):
        self.dtype = dtype
        self.shape = tuple(shape)
        self.data = data

    def __repr__(self):
        return f"SafetensorsTensor({self.dtype}, {self.shape})"


def read_safetensors(path: str) -> dict[str, SafetensorsTensor]:
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(n))
    base = 8 + n
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        dt = meta["dtype"]
        if dt not in _DT:
            raise ValueError(f"{path}: tensor {name} has unsupported dtype {dt}")
        s, e = meta["data_offsets"]
        arr = mm[base + s:base + e].view(_DT[dt]).reshape(meta["shape"])
        out[name] = SafetensorsTensor(dt, meta["shape"], arr)
    return out


def write_safetensors(path: str, tensors: dict[str, tuple[str, np.ndarray]], metadata: dict | None = None) -> None:
    """Writes {name: (dtype name, array)} (16-bit floats as uint16 bit patterns)."""
    header, off, blobs = {}, 0, []
    for name in sorted(tensors):
        dt, arr = tensors[name]
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if metadata:
        header["__metadata__"] = metadata
    hb = json.dumps(header).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for b in blobs:
            f.write(b)


def _bf16_to_f16_bits(bits: np.ndarray) -> np.ndarray:
    f32 = (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)
    return f32.astype(np.float16).view(np.uint16)


def _half_to_f32(bits: np.ndarray, dt: str) -> np.ndarray:
    if dt == "F16":
        return bits.view(np.float16).astype(np.float32)
    return (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)


def _f32_to_half(v: np.ndarray, dt: str) -> np.ndarray:
    if dt == "F16":
        return v.astype(np.float16).view(np.uint16)
    u = v.astype(np.float32).view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)
    return r.astype(np.uint16)


class WeightStore:
    """All tensors of a Maple checkpoint directory after ``sanitize``:
    ``arrays[name] = SafetensorsTensor``."""

    def __init__(self, model_dir: str, config: MapleConfig | None = None, to_f16: bool = False):
        self.config = config or MapleConfig.load(model_dir)
        idx = json.load(open(os.path.join(model_dir, "model.safetensors.index.json")))
        wm = idx.get("weight_map", {})
        self.arrays: dict[str, SafetensorsTensor] = {}
        for shard in sorted(set(wm.values())):
            for k, t in read_safetensors(os.path.join(model_dir, shard)).items():
                if to_f16 and t.dtype == "BF16":
                    t = SafetensorsTensor("F16", t.shape, _bf16_to_f16_bits(np.asarray(t.data)))
                self.arrays[k] = t
        self.sanitize()

    def get(self, name: str):
        return self.arrays.get(name)

    def req(self, name: str) -> SafetensorsTensor:
        if name not in self.arrays:
            raise KeyError(f"missing weight: {name}")
        return self.arrays[name]

    def sanitize(self) -> None:
        gs = self.config.expert_group_size
        for key in [k for k in self.arrays if k.endswith(".row_alpha")]:
            alpha = self.arrays.pop(key)
            prefix = key[: -len(".row_alpha")]
            packed = self.arrays.get(prefix + ".weight")
            if packed is None:
                continue
            n_groups = packed.shape[-1] * 16 // gs
            a = np.asarray(alpha.data)
            scales = np.ascontiguousarray(np.broadcast_to(a[..., None], a.shape + (n_groups,)))
            neg = _f32_to_half(-_half_to_f32(scales, alpha.dtype), alpha.dtype)  # exact: sign flip
            self.arrays[prefix + ".scales"] = SafetensorsTensor(alpha.dtype, scales.shape, scales)
            self.arrays[prefix + ".biases"] = SafetensorsTensor(alpha.dtype, neg.shape, neg)
        for l in range(self.config.num_hidden_layers):
            attn = f"model.layers.{l}.self_attn"
            for suffix in ("weight", "scales", "biases"):
                names = [f"{attn}.{p}_proj.{suffix}" for p in ("q", "k", "v")]
                if all(n in self.arrays for n in names):
                    parts = [self.arrays.pop(n) for n in names]
                    cat = np.concatenate([np.asarray(p.data) for p in parts], axis=0)
                    self.arrays[f"{attn}.qkv_proj.{suffix}"] = SafetensorsTensor(parts[0].dtype, cat.shape, cat)
            mlp = f"model.layers.{l}.mlp.switch_mlp"
            for suffix in ("weight", "scales", "biases"):
                up, gate = f"{mlp}.up_proj.{suffix}", f"{mlp}.gate_proj.{suffix}"
                if up in self.arrays and gate in self.arrays:
                    u, g = self.arrays.pop(up), self.arrays.pop(gate)
                    cat = np.concatenate([np.asarray(u.data), np.asarray(g.data)], axis=1)
                    self.arrays[f"{mlp}.up_gate_proj.{suffix}"] = SafetensorsTensor(u.dtype, cat.shape, cat)

    # ---- the MoE layer's tensors in the kernels' layout ------------------------
    def moe_layer(self, layer: int) -> dict:
        """{w_ug, s_ug, b_ug, w_dn, s_dn, b_dn, gate, norm} numpy arrays of
        one layer (codes uint32, 16-bit values as uint16 bit patterns) and the
        dtype name of the 16-bit tensors."""
        p = f"model.layers.{layer}"
        sw = f"{p}.mlp.switch_mlp"
        t = {
            "w_ug": self.req(f"{sw}.up_gate_proj.weight"), "s_ug": self.req(f"{sw}.up_gate_proj.scales"),
            "b_ug": self.req(f"{sw}.up_gate_proj.biases"), "w_dn": self.req(f"{sw}.down_proj.weight"),
            "s_dn": self.req(f"{sw}.down_proj.scales"), "b_dn": self.req(f"{sw}.down_proj.biases"),
            "gate": self.req(f"{p}.mlp.gate.weight"), "norm": self.req(f"{p}.post_attention_layernorm.weight"),
        }
        out = {k: np.ascontiguousarray(v.data) for k, v in t.items()}
        out["dtype"] = t["s_ug"].dtype
        out["gate_dtype"] = t["gate"].dtype
        return out


def to_device(layer: dict, device="cuda") -> dict:
    """The arrays of WeightStore.moe_layer as torch tensors (codes int32,
    16-bit tensors as torch.bfloat16 / torch.float16 by their dtype name)."""
    import torch
    td = {"BF16": torch.bfloat16, "F16": torch.float16}
    out = {}
    for k, v in layer.items():
        if k in ("dtype", "gate_dtype"):
            continue
        v = np.array(v)  # a writable copy (the store's arrays may be read-only maps)
        if k.startswith("w_"):
            out[k] = torch.from_numpy(v.view(np.int32)).to(device)
        else:
            dt = layer["gate_dtype"] if k == "gate" else layer["dtype"]
            out[k] = torch.from_numpy(v.view(np.int16)).to(device).view(td[dt])
    return out
