"""Maple checkpoint loading (momij_b200/loader.py, after WeightStore.swift):
a synthetic two-shard checkpoint is written with the safetensors writer,
loaded, and its sanitized tensors checked against the reference's rules
(row_alpha -> scales / biases = -scales, q/k/v -> qkv_proj along rows,
up/gate -> up_gate_proj along the expert rows); a GPU test runs the loaded
layer through the MoE path against the oracle.
"""
from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

from momij_b200 import loader as LD
from momij_b200 import synth as S
from oracle import oracle as O

H, I, E, K, GS, L = 512, 256, 8, 2, 64, 2


def _bf16(a):
    return S.f32_to_half_bits(np.ascontiguousarray(a, np.float32), 0)


def _make_checkpoint(path):
    rng = np.random.default_rng(0)
    cfg = {"hidden_size": H, "moe_intermediate_size": I, "num_hidden_layers": L, "num_experts": E,
           "num_experts_per_tok": K, "rms_norm_eps": 1e-6, "num_attention_heads": 4, "num_key_value_heads": 2,
           "head_dim": 64, "quantization": {"bits": 2, "group_size": GS}}
    json.dump(cfg, open(os.path.join(path, "config.json"), "w"))
    shards = [{}, {}]
    raw = {}
    for l in range(L):
        t = shards[l]
        p = f"model.layers.{l}"
        for proj, n in (("q", 256), ("k", 128), ("v", 128), ("o", H)):
            k_in = H if proj != "o" else 256
            t[f"{p}.self_attn.{proj}_proj.weight"] = ("U32", rng.integers(0, 2**32, (n, k_in // 16), dtype=np.uint32))
            t[f"{p}.self_attn.{proj}_proj.row_alpha"] = ("BF16", _bf16(rng.uniform(0.005, 0.02, n)))
        for proj in ("up", "gate"):
            t[f"{p}.mlp.switch_mlp.{proj}_proj.weight"] = ("U32", rng.integers(0, 2**32, (E, I, H // 16), dtype=np.uint32))
            t[f"{p}.mlp.switch_mlp.{proj}_proj.row_alpha"] = ("BF16", _bf16(rng.uniform(0.005, 0.02, (E, I))))
        t[f"{p}.mlp.switch_mlp.down_proj.weight"] = ("U32", rng.integers(0, 2**32, (E, H, I // 16), dtype=np.uint32))
        t[f"{p}.mlp.switch_mlp.down_proj.scales"] = ("BF16", _bf16(rng.uniform(0.005, 0.02, (E, H, I // GS))))
        t[f"{p}.mlp.switch_mlp.down_proj.biases"] = ("BF16", _bf16(rng.uniform(-0.03, 0.0, (E, H, I // GS))))
        t[f"{p}.mlp.gate.weight"] = ("BF16", _bf16(rng.standard_normal((E, H)) / np.sqrt(H)))
        t[f"{p}.post_attention_layernorm.weight"] = ("BF16", _bf16(1.0 + 0.1 * rng.standard_normal(H)))
        raw.update({k: v[1] for k, v in t.items()})
    wm = {}
    for i, t in enumerate(shards):
        name = f"model-{i + 1:05d}-of-00002.safetensors"
        LD.write_safetensors(os.path.join(path, name), t, {"format": "mlx"})
        wm.update({k: name for k in t})
    json.dump({"metadata": {}, "weight_map": wm}, open(os.path.join(path, "model.safetensors.index.json"), "w"))
    return raw


def test_sanitize_follows_the_reference(tmp_path):
    raw = _make_checkpoint(str(tmp_path))
    st = LD.WeightStore(str(tmp_path))
    assert st.config.expert_group_size == GS and st.config.num_experts == E
    assert not any(k.endswith(".row_alpha") for k in st.arrays)
    for l in range(L):
        a = f"model.layers.{l}.self_attn"
        for proj in ("q", "k", "v"):
            assert f"{a}.{proj}_proj.weight" not in st.arrays
        qkv = st.req(f"{a}.qkv_proj.weight").data
        assert np.array_equal(qkv, np.concatenate([raw[f"{a}.{p}_proj.weight"] for p in "qkv"], axis=0))
        alphas = np.concatenate([raw[f"{a}.{p}_proj.row_alpha"] for p in "qkv"])
        sc = st.req(f"{a}.qkv_proj.scales").data
        assert sc.shape == (512, H // GS) and (sc == alphas[:, None]).all()
        bi = st.req(f"{a}.qkv_proj.biases").data
        assert (bi == (alphas ^ np.uint16(0x8000))[:, None]).all()  # -alpha: the sign bit
        # o_proj keeps its name; its row_alpha became scales/biases too
        assert st.req(f"{a}.o_proj.scales").data.shape == (H, 256 // GS)
        m = f"model.layers.{l}.mlp.switch_mlp"
        ug = st.req(f"{m}.up_gate_proj.weight").data
        assert ug.shape == (E, 2 * I, H // 16)
        assert np.array_equal(ug[:, :I], raw[f"{m}.up_proj.weight"]) and np.array_equal(ug[:, I:], raw[f"{m}.gate_proj.weight"])
        s_ug = st.req(f"{m}.up_gate_proj.scales").data
        assert s_ug.shape == (E, 2 * I, H // GS)
        assert (s_ug[:, I:] == raw[f"{m}.gate_proj.row_alpha"][..., None]).all()
        lay = st.moe_layer(l)
        assert lay["w_dn"].shape == (E, H, I // 16) and lay["gate"].shape == (E, H) and lay["dtype"] == "BF16"


def test_f16_conversion(tmp_path):
    raw = _make_checkpoint(str(tmp_path))
    st = LD.WeightStore(str(tmp_path), to_f16=True)
    g = st.req("model.layers.0.mlp.gate.weight")
    assert g.dtype == "F16"
    want = ((raw["model.layers.0.mlp.gate.weight"].astype(np.uint32) << 16).view(np.float32)).astype(np.float16)
    assert np.array_equal(g.data.view(np.float16), want)


def test_safetensors_round_trip(tmp_path):
    p = str(tmp_path / "x.safetensors")
    t = {"a": ("F32", np.arange(12, dtype=np.float32).reshape(3, 4)), "b": ("U32", np.arange(5, dtype=np.uint32))}
    LD.write_safetensors(p, t)
    r = LD.read_safetensors(p)
    assert set(r) == {"a", "b"} and r["a"].shape == (3, 4)
    assert np.array_equal(r["a"].data, t["a"][1]) and np.array_equal(r["b"].data, t["b"][1])


@pytest.mark.gpu
def test_loaded_layer_runs_through_the_moe_path(tmp_path):
    from momij_b200 import moe
    _make_checkpoint(str(tmp_path))
    st = LD.WeightStore(str(tmp_path))
    lay = st.moe_layer(1)
    dw = LD.to_device(lay)
    M = 3
    x = S.activations(M, H, seed=21)
    lg = S.logits_normal(M, E, 0, 22)
    y = torch.empty(M, H, dtype=torch.bfloat16, device="cuda")
    ws = moe.new_workspace(M, K, H, I)
    moe.forward(torch.from_numpy(lg).cuda(), torch.from_numpy(x.view(np.int16)).cuda().view(torch.bfloat16),
                dw, y, H=H, I=I, Ktop=K, gs=GS, M=M, workspace=ws)
    moe.synchronize(workspace=ws)
    i_ref, s_ref = O.route(lg, K)
    y_ref, _ = O.expert_ffn(x, {k: lay[k] for k in ("w_ug", "s_ug", "b_ug", "w_dn", "s_dn", "b_dn")}, i_ref, s_ref,
                            M, H, I, K, GS)
    g = O.np_half_to_f64(y.view(torch.int16).cpu().numpy().view(np.uint16))
    r = O.np_half_to_f64(y_ref)
    rel = np.sqrt(((g - r) ** 2).sum(1)) / np.sqrt((r ** 2).sum(1))
    assert rel.max() <= 2e-3, rel.max()
