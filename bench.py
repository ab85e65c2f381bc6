#!/usr/bin/env python
"""Benchmark of the 2-bit MoE gather-GEMV path (BASELINE.json metric).

One *step* is one token (M=1, config 1) or one verify batch (M=8, config 2)
through 48 MoE layers with distinct weights: per layer the router top-k,
up||gate gather-GEMV + SwiGLU, down gather-GEMV, score-weighted combine into
the residual stream (h += MoE(h)).  Weights are generated on the GPU from the
seeded generator (36 GB for config 1), so every step streams ~2.3 GB of
distinct expert weights: inputs larger than L2, no flush needed.

Timing: W untimed steps, then K steps replayed from one CUDA graph, bracketed
by a barrier + synchronize, CUDA events on the launching stream, max over
ranks.  `e2e` repeats the K steps through the public API with the step's
inputs copied from pinned host memory and the output read back inside the
timed region.  The decode roofline is taken from the timed graph itself (one
kernel per layer: the layer time is ms_per_step / layers).

Launched with more than one rank (torchrun, WORLD_SIZE > 1) the default
config is config 4 (expert parallelism over NCCL, strong scaling); a single
process runs config 1.  After the timed region every config checks layer 0's
output for a few tokens against the CPU oracle and reports it as `parity`.

`--impl reference` times the CPU restatement of the reference's path
(oracle/, OpenMP over all host cores) on rank 0: the reference itself is
Swift + Metal + MLX and cannot run on this box.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    "decode": dict(desc="BASELINE config 1: decode M=1, H=4096, E=128, top-8, I=1536, gs64, "
                        "48 layers with distinct weights", H=4096, I=1536, E=128, K=8, gs=64, M=1,
                   L=48, rho=None),
    "verify": dict(desc="BASELINE config 2: verify batch M=8 (rho=0.7 correlated logits), "
                        "config-1 shapes, 48 layers", H=4096, I=1536, E=128, K=8, gs=64, M=8,
                   L=48, rho=0.7),
    "prefill": dict(desc="BASELINE config 3: prefill of 2048 tokens through one MoE layer, "
                         "Zipf(1.1) routing, grouped tcgen05 GEMM path", H=4096, I=1536, E=128,
                    K=8, gs=64, M=2048, L=1, rho=None, zipf=1.1),
    "ep": dict(desc="BASELINE config 4: expert-parallel decode, 64 concurrent sequences (M=64 per "
                    "step), H=4096, E=256, top-8, I=1024, gs64, 48 layers, N(0,1) router logits "
                    "(uniform expert choice); experts sharded evenly over the GPUs, all-to-all "
                    "dispatch/combine over NCCL", H=4096, I=1024, E=256, K=8, gs=64, M=64, L=48,
               rho=None, ep=True),
}
METRIC = "2-bit MoE gather-GEMV tokens/s"


def load_peaks(key: str = "hbm_gbs") -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)[key]), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}.get(key, 0.0), "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        try:
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        except Exception:
            pass
        finally:
            try:
                os.unlink(self.path)
            except Exception:
                pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if "Active" in r[5 + i]
                          and "Not" not in r[5 + i]})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


def dist_setup():
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ---------------------------------------------------------------------------
# CPU leg: the oracle (CPU restatement of the reference path), all host cores
# ---------------------------------------------------------------------------

def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_layer_sample(cfg: dict, wh: dict, x: np.ndarray, inds: np.ndarray, scores: np.ndarray,
                     budget_s: float) -> dict:
    """Times oracle.expert_ffn on one layer's selected experts for ~budget_s."""
    from oracle import oracle as O
    O.set_num_threads(host_cores())
    M, H, I, K, gs = cfg["M"], cfg["H"], cfg["I"], cfg["K"], cfg["gs"]
    if M > 64:  # large batches: a bounded sample of the tokens, scaled per token
        M, x, inds, scores = 64, x[:64], inds[:64], scores[:64]
    O.expert_ffn(x, wh, inds, scores, M, H, I, K, gs)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        O.expert_ffn(x, wh, inds, scores, M, H, I, K, gs)
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = (time.perf_counter() - t0) / n
    tok_s = M / (dt * cfg["L"])
    return {"value": tok_s, "unit": "tokens/s", "cores": O.num_threads(), "kind": "port",
            "sample": f"{n} evaluations of one layer's expert FFN ({M} token(s), "
                      f"{len(np.unique(inds))} experts, {dt * 1e3:.1f} ms each); tokens/s scaled to "
                      f"{cfg['L']} layers",
            "layer_ms": dt * 1e3}


def cfg_logits(S, cfg: dict, layer: int) -> np.ndarray:
    M, E = cfg["M"], cfg["E"]
    if cfg.get("zipf"):
        return S.logits_zipf(M, E, cfg["zipf"], layer, 0)
    if cfg["rho"]:
        return S.logits_ar1(M, E, cfg["rho"], layer, 0)
    return S.logits_normal(M, E, layer, 0)


def host_layer_inputs(cfg: dict, layer: int = 0):
    """Host copies of one layer's inputs for the CPU leg (selected experts only)."""
    import torch
    from momij_b200 import moe, synth as S
    H, I, E, K, gs, M = (cfg[k] for k in ("H", "I", "E", "K", "gs", "M"))
    lg = cfg_logits(S, cfg, layer)
    from oracle import oracle as O
    inds, scores = O.route(lg, K)
    uniq, remap = np.unique(inds, return_inverse=True)
    wd = moe.device_expert_weights(E, H, I, gs, layer=layer, seed=0)
    idx = torch.from_numpy(uniq.astype(np.int64)).cuda()
    wh = {k: v.index_select(0, idx).view(torch.int32 if k.startswith("w_") else torch.int16)
          .cpu().numpy().view(np.uint32 if k.startswith("w_") else np.uint16) for k, v in wd.items()}
    del wd
    x = S.activations(M, H, layer, 0)
    return wh, x, remap.reshape(M, K).astype(np.int32), scores


def oracle_check(cfg: dict, W0: dict, lg0: np.ndarray, x_rows: np.ndarray, y_rows: np.ndarray,
                 inds_rows: np.ndarray, expert_lo: int = 0) -> dict:
    """Layer-0 outputs of a few tokens against the CPU oracle: per-row
    rel-L2 of y = MoE(x) (no residual) and whether the router indices are
    bit-exact.  W0 holds experts [expert_lo, expert_lo + E_local) on the GPU;
    experts outside it (other ranks' shards) are regenerated on the host from
    the seeded generator."""
    import torch
    from momij_b200 import synth as S
    from oracle import oracle as O
    H, I, K, gs, E = cfg["H"], cfg["I"], cfg["K"], cfg["gs"], cfg["E"]
    i_ref, s_ref = O.route(np.ascontiguousarray(lg0, np.float32), K)
    idx_exact = bool((np.asarray(inds_rows) == i_ref).all())
    uniq, remap = np.unique(i_ref, return_inverse=True)
    e_loc = W0["w_ug"].shape[0]
    wh = {k: [] for k in ("w_ug", "s_ug", "b_ug", "w_dn", "s_dn", "b_dn")}
    for e in uniq:
        e = int(e)
        if expert_lo <= e < expert_lo + e_loc:
            for k in wh:
                t = W0[k][e - expert_lo]
                wh[k].append(t.view(torch.int32 if k.startswith("w_") else torch.int16).cpu().numpy()
                             .view(np.uint32 if k.startswith("w_") else np.uint16))
        else:
            one = S.expert_weights_one(e, H, I, gs, layer=0, seed=0)
            for k in wh:
                wh[k].append(one[k])
    wh = {k: np.ascontiguousarray(np.stack(v)) for k, v in wh.items()}
    n = x_rows.shape[0]
    y_ref, _ = O.expert_ffn(np.ascontiguousarray(x_rows), wh, remap.reshape(n, K).astype(np.int32), s_ref,
                            n, H, I, K, gs)
    g = O.np_half_to_f64(np.asarray(y_rows))
    r = O.np_half_to_f64(y_ref)
    rel = np.sqrt(((g - r) ** 2).sum(axis=1)) / np.maximum(np.sqrt((r ** 2).sum(axis=1)), 1e-30)
    return {"tokens": int(n), "max_rel_l2": float(rel.max()), "idx_exact": idx_exact,
            "bit_identical_frac": float((np.asarray(y_rows) == y_ref).mean()), "tol": 2e-3}


def run_reference(args, cfg) -> None:
    world, rank, _ = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0
    if rank != 0:
        return
    from momij_b200 import synth as S
    from oracle import oracle as O
    # every host core this process may use (torchrun sets OMP_NUM_THREADS=1)
    O.set_num_threads(host_cores())
    H, I, E, K, gs, M = (cfg[k] for k in ("H", "I", "E", "K", "gs", "M"))
    # The CPU leg needs no GPU: generate the selected experts' weights on the host.
    lg = cfg_logits(S, cfg, 0)
    inds, scores = O.route(lg, K)
    uniq, remap = np.unique(inds, return_inverse=True)
    full = {}
    for k, kind, shape in (("w_ug", S.KIND_W_UG, (2 * I, H // 16)), ("w_dn", S.KIND_W_DN, (H, I // 16))):
        n = shape[0] * shape[1]
        full[k] = np.stack([S.codes(n, 0, S.stream_id(0, kind), int(e) * n).reshape(shape) for e in uniq])
    for k, kind, shape, a, c in (("s_ug", S.KIND_S_UG, (2 * I, H // gs), S.SCALE_A, S.SCALE_C),
                                 ("b_ug", S.KIND_B_UG, (2 * I, H // gs), S.BIAS_A, S.BIAS_C),
                                 ("s_dn", S.KIND_S_DN, (H, I // gs), S.SCALE_A, S.SCALE_C),
                                 ("b_dn", S.KIND_B_DN, (H, I // gs), S.BIAS_A, S.BIAS_C)):
        n = shape[0] * shape[1]
        full[k] = np.stack([S.affine_uniform(n, a, c, 0, S.stream_id(0, kind), 0, int(e) * n)
                            .reshape(shape) for e in uniq])
    x = S.activations(M, H, 0, 0)
    rinds = remap.reshape(M, K).astype(np.int32)
    if M > 64:  # large batches: each step is a bounded sample of 64 tokens, scaled per token
        M, x, rinds, scores = 64, x[:64], rinds[:64], scores[:64]
    for _ in range(args.warmup):
        O.expert_ffn(x, full, rinds, scores, M, H, I, K, gs)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.expert_ffn(x, full, rinds, scores, M, H, I, K, gs)
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    tok_s = M / (dt * cfg["L"])
    line = {
        "impl": "reference", "metric": METRIC, "value": tok_s, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "strong" if cfg.get("ep") else "weak",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": cfg["desc"], "H": H, "E": E, "top_k": K, "I": I, "gs": gs, "M": M,
                   "layers": cfg["L"], "parallelism": "cpu"},
        "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": O.num_threads(),
                         "kind": "port",
                         "sample": f"each step = one layer's expert FFN ({M} token(s), {len(uniq)} "
                                   f"experts) on the host; tokens/s scaled to {cfg['L']} layers. "
                                   "The reference (Swift/Metal/MLX) cannot run here; this is the "
                                   "oracle's CPU restatement of its path."},
        "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU leg
# ---------------------------------------------------------------------------

def run_gpu(args, cfg) -> None:
    import torch
    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    from momij_b200 import moe, synth as S

    H, I, E, K, gs, M, L = (cfg[k] for k in ("H", "I", "E", "K", "gs", "M", "L"))
    P = M * K
    dev = torch.device("cuda", local)
    W = [moe.device_expert_weights(E, H, I, gs, layer=l, seed=0, device=dev) for l in range(L)]
    lg_host = np.stack([cfg_logits(S, cfg, l) for l in range(L)])
    x_host = S.activations(M, H, 0, 0)
    logits = torch.from_numpy(lg_host).to(dev)
    h0 = torch.from_numpy(x_host.view(np.int16)).to(dev).view(torch.bfloat16)
    h = h0.clone()
    ws = moe.new_workspace(M, K, H, I, dev)
    inds_all = torch.empty(L, M, K, dtype=torch.int32, device=dev)
    scores_all = torch.empty(L, M, K, dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)

    # algorithmic bytes: the distinct experts each layer streams
    eb = S.expert_bytes(H, I, gs)
    up_bytes = (2 * I) * (H // 16) * 4 + (2 * I) * (H // gs) * 4
    dn_bytes = eb - up_bytes

    def step():
        for l in range(L):
            moe.forward(logits[l], h, W[l], None, H=H, I=I, Ktop=K, gs=gs, M=M, inds=inds_all[l],
                        scores=scores_all[l], resid_h=h, workspace=ws, stream=stream)

    # eager warm-up (also validates the status once)
    with torch.cuda.stream(stream):
        step()
    moe.synchronize(stream, ws)
    # algorithmic bytes: the distinct experts each layer streams (from the
    # router outputs the GPU itself produced)
    ih = inds_all.cpu().numpy()
    uniq = [len(np.unique(ih[l])) for l in range(L)]
    bytes_per_step = sum(uniq) * eb

    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    torch.cuda.synchronize()

    # CUDAGraph.replay() launches on the *current* stream: keep it `stream`,
    # the stream the timing events are recorded on.
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph.replay()
    torch.cuda.synchronize()
    barrier(world)

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        barrier(world)
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            ev1.record(stream)
        torch.cuda.synchronize()
    dev_ms = ev0.elapsed_time(ev1)
    barrier(world)
    dev_ms = max_over_ranks(dev_ms, world)
    clocks = clk.summary()
    moe.synchronize(stream, ws)

    ms_per_step = dev_ms / args.steps
    tok_s = world * M * args.steps / (dev_ms / 1e3)

    # --- e2e: host inputs -> public API -> host output, copies in the timed region
    x_pin = torch.from_numpy(x_host.view(np.int16)).view(torch.bfloat16).pin_memory()
    lg_pin = torch.from_numpy(lg_host).pin_memory()
    y_pin = torch.empty(M, H, dtype=torch.bfloat16).pin_memory()
    for _ in range(2):
        with torch.cuda.stream(stream):
            h.copy_(x_pin, non_blocking=True)
            logits.copy_(lg_pin, non_blocking=True)
            graph.replay()
            y_pin.copy_(h, non_blocking=True)
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(args.steps):
            h.copy_(x_pin, non_blocking=True)
            logits.copy_(lg_pin, non_blocking=True)
            graph.replay()
            y_pin.copy_(h, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world)
    e2e_tok_s = world * M * args.steps / (e2e_ms / 1e3)
    h2d = x_pin.numel() * 2 + lg_pin.numel() * 4
    d2h = y_pin.numel() * 2

    # --- live per-kernel durations (instrumented graph: one event pair per launch)
    moe.profile_reset()
    moe.profile_enable(True)
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2, stream=stream):
        step()
    moe.profile_enable(False)
    reps = max(3, min(args.steps, 10))
    kids = (moe.KERNEL_PLAN, moe.KERNEL_UP, moe.KERNEL_ROWS, moe.KERNEL_COMBINE, moe.KERNEL_LAYER)
    kt = {kid: [0.0, 0] for kid in kids}
    try:
        for _ in range(reps):
            with torch.cuda.stream(stream):
                g2.replay()
            torch.cuda.synchronize()
            for kid in kids:
                ms, n = moe.profile_read(kid)
                kt[kid][0] += ms
                kt[kid][1] += n
    except moe.SeedlessError as e:
        print(f"warning: per-kernel timing unavailable: {e}", file=sys.stderr)
    moe.profile_reset()
    del g2
    avg = {kid: (kt[kid][0] / kt[kid][1] if kt[kid][1] else None) for kid in kt}
    launches_per_layer = sum(1 for kid in kids if kt[kid][1]) or 1
    peak, peak_kind = load_peaks()
    tensor_roof = None
    if cfg.get("zipf"):
        # grouped tcgen05 path: tensor-bound; the up||gate GEMM dominates
        tpeak, tpeak_kind = load_peaks("bf16_tflops")
        flops = 2.0 * P * (2 * I) * H  # algorithmic (the hi/lo split issues twice this)
        t_ms = avg[moe.KERNEL_UP]
        ach = flops / (t_ms * 1e-3) / 1e12 if t_ms else None
        tensor_roof = {"bound": "tensor", "kernel": "grouped_gemm_kernel<up||gate+SwiGLU> (tcgen05)",
                       "achieved": ach, "peak": tpeak, "unit": "TFLOP/s",
                       "frac": (ach / tpeak) if ach else None, "traffic": None,
                       "peak_source": tpeak_kind, "flops_per_launch": flops,
                       "avg_launch_us": {"permute+blocks": _us(avg[moe.KERNEL_PLAN]),
                                         "up": _us(avg[moe.KERNEL_UP]), "down": _us(avg[moe.KERNEL_ROWS]),
                                         "combine": _us(avg[moe.KERNEL_COMBINE])}}
    timed_layer_ms = ms_per_step / L
    if avg[moe.KERNEL_LAYER]:
        # the whole layer is one kernel, the only launch of the layer in the
        # timed graph: its duration there is ms_per_step / L
        m1 = os.environ.get("MOMIJ_DECODE_M1", "")
        mrow = os.environ.get("MOMIJ_DECODE_MROW", "")
        streaming = m1 == "" and (M == 1 or mrow != "tc")
        dom_kernel = ("moe_token_kernel (route + up||gate/SwiGLU + down + combine; TMA-fed stages, "
                      "u8xs8 mma.sync" + ("; the batch's tokens one after another)" if M > 1 else ")")
                      if streaming else
                      "moe_layer_kernel (route + up||gate/SwiGLU + down + combine, warp-level u8xs8 mma)"
                      if M == 1 and m1 == "warp" else
                      "moe_decode_kernel (route + up||gate/SwiGLU + down + combine, tcgen05)")
        dom_bytes = (sum(uniq) / L) * eb
        dom_ms = timed_layer_ms
        dom_source = "timed graph: ms_per_step / layers (one launch per layer)"
    else:
        dom_kernel = "gemv_kernel<up||gate+SwiGLU>"
        dom_bytes = (sum(uniq) / L) * up_bytes
        dom_ms = avg[moe.KERNEL_UP]
        dom_source = "CUDA-event pair around each launch in an instrumented replay"
    achieved = dom_bytes / (dom_ms * 1e-3) / 1e9 if dom_ms else None
    traffic = None
    tf = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tf):
        try:
            traffic = json.load(open(tf)).get(args.config, {}).get("traffic_bytes_per_launch")
        except Exception:
            traffic = None
    if tensor_roof is not None:
        tensor_roof["traffic"] = traffic

    # --- parity: layer 0 on the initial activations, y = MoE(x), against the oracle
    parity = None
    if rank == 0:
        nchk = min(M, 4)
        y_chk = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
        i_chk = torch.empty(M, K, dtype=torch.int32, device=dev)
        s_chk = torch.empty(M, K, dtype=torch.float32, device=dev)
        with torch.cuda.stream(stream):
            moe.forward(logits[0], h0, W[0], y_chk, H=H, I=I, Ktop=K, gs=gs, M=M, inds=i_chk,
                        scores=s_chk, workspace=ws, stream=stream)
        moe.synchronize(stream, ws)
        parity = oracle_check(cfg, W[0], lg_host[0][:nchk], x_host[:nchk],
                              y_chk[:nchk].view(torch.int16).cpu().numpy().view(np.uint16),
                              i_chk[:nchk].cpu().numpy())

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        wh, xh, ih, sh = host_layer_inputs(cfg, 0)
        cpu = cpu_layer_sample(cfg, wh, xh, ih, sh, args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": ("bf16 tcgen05 GEMM (weights as hi+lo bf16), f32 accumulate, bf16 I/O"
                      if cfg.get("zipf") else
                      "u8 code classes x s8 activation digits -> s32 (mma.sync m16n8k32), f32 scale/bias "
                      "epilogue, bf16 I/O" if (os.environ.get("MOMIJ_DECODE_M1", "") in ("", "warp") and
                                                (M == 1 or os.environ.get("MOMIJ_DECODE_MROW", "") != "tc")) else
                      "tcgen05.mma kind::i8 (u8 code classes x s8 activation digits -> s32 in TMEM), f32 "
                      "scale/bias epilogue, bf16 I/O"),
            "data": "synthetic (seeded generator, momij_b200/synth.py)",
            "config": {"workload": cfg["desc"], "H": H, "E": E, "top_k": K, "I": I, "gs": gs,
                       "M": M, "layers": L, "global_batch": M * world,
                       "parallelism": "replicas" if world > 1 else "single",
                       "l2": f"inputs larger than L2: {bytes_per_step / 1e9:.2f} GB of distinct "
                             "expert weights streamed per step"},
            "hbm_tbs": bytes_per_step / (ms_per_step * 1e-3) / 1e12,
            "hbm_frac_of_peak": bytes_per_step / (ms_per_step * 1e-3) / 1e9 / peak,
            "roofline": tensor_roof if tensor_roof else {"bound": "hbm", "kernel": dom_kernel,
                         "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": (achieved / peak) if achieved else None, "traffic": traffic,
                         "peak_source": peak_kind,
                         "bytes_per_launch": dom_bytes,
                         "launch_us": _us(dom_ms), "launch_us_source": dom_source,
                         "diag_event_pair_us": {"plan": _us(avg[moe.KERNEL_PLAN]),
                                                "up": _us(avg[moe.KERNEL_UP]),
                                                "down": _us(avg[moe.KERNEL_ROWS]),
                                                "combine": _us(avg[moe.KERNEL_COMBINE]),
                                                "layer": _us(avg[moe.KERNEL_LAYER])}},
            "parity": parity,
            "clocks": clocks,
            "e2e": {"value": e2e_tok_s, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms / args.steps},
            "gpu_launches": launches_per_layer * L * args.steps,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    del graph
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_ep(args, cfg) -> None:
    """Config 4: M tokens per step split evenly over the ranks (each rank owns
    M/N sequences and E/N experts); per layer route -> momij_moe_ep_forward
    (the C-ABI expert-parallel layer: dispatch -> NCCL send/recv of the
    destination segments -> local experts -> send/recv back -> combine).
    Strong scaling: the total work per step is fixed as N grows.  On one GPU
    the step is the plain single-GPU layer (moe.forward), the best one-GPU
    path."""
    import torch
    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    from momij_b200 import moe, synth as S

    H, I, E, K, gs, M, L = (cfg[k] for k in ("H", "I", "E", "K", "gs", "M", "L"))
    if M % world or E % world:
        raise SystemExit(f"ep config needs N dividing M={M} and E={E}")
    Ml, El = M // world, E // world
    lo = rank * El
    dev = torch.device("cuda", local)
    W = [moe.device_expert_weights(E, H, I, gs, layer=l, seed=0, device=dev, experts=(lo, lo + El))
         for l in range(L)]
    mine = slice(rank * Ml, (rank + 1) * Ml)
    lg_host = np.ascontiguousarray(np.stack([cfg_logits(S, cfg, l)[mine] for l in range(L)]))
    x_host = np.ascontiguousarray(S.activations(M, H, 0, 0)[mine])
    logits = torch.from_numpy(lg_host).to(dev)
    h = torch.from_numpy(x_host.view(np.int16)).to(dev).view(torch.bfloat16)
    stream = torch.cuda.Stream(device=dev)
    eplayer = None
    if world > 1:  # one NCCL communicator for the layer object, from rank 0's unique id
        import torch.distributed as dist
        uid = [moe.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        eplayer = moe.EpLayer(rank=rank, world=world, E=E, H=H, I=I, K=K, max_tokens=Ml, gs=gs, unique_id=uid[0])
    ws = moe.new_workspace(Ml, K, H, I, dev)
    inds_all = torch.empty(L, Ml, K, dtype=torch.int32, device=dev)
    scores_all = torch.empty(L, Ml, K, dtype=torch.float32, device=dev)

    def step():
        for l in range(L):
            if world == 1:
                moe.forward(logits[l], h, W[l], None, H=H, I=I, Ktop=K, gs=gs, M=Ml, inds=inds_all[l],
                            scores=scores_all[l], resid_h=h, workspace=ws, stream=stream)
            else:
                moe.route(logits[l], K, inds_all[l], scores_all[l], stream=stream)
                eplayer.forward(h, W[l], inds=inds_all[l], scores=scores_all[l], resid_h=h, stream=stream)

    with torch.cuda.stream(stream):
        step()
    torch.cuda.synchronize()
    if eplayer is not None:
        eplayer.status(stream)
    else:
        moe.synchronize(stream, ws)
    # algorithmic bytes of this rank: its experts that the step's tokens select
    ih = inds_all.cpu().numpy()
    if world > 1:  # every rank's routing, to count the local experts used
        import torch.distributed as dist
        g = [torch.empty_like(inds_all) for _ in range(world)]
        dist.all_gather(g, inds_all)
        ih = np.concatenate([t.cpu().numpy() for t in g], axis=1)
    eb = S.expert_bytes(H, I, gs)
    used = [int(((np.unique(ih[l]) >= lo) & (np.unique(ih[l]) < lo + El)).sum()) for l in range(L)]
    bytes_per_step = sum(used) * eb

    graph = None
    if os.environ.get("MOMIJ_EP_GRAPH", "1") != "0":
        try:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                step()
            torch.cuda.synchronize()
        except Exception as e:  # eager fallback keeps the same collectives on every rank
            print(f"warning: graph capture failed ({e}); timing eager launches", file=sys.stderr)
            graph = None
            torch.cuda.synchronize()
    ok = torch.tensor([1 if graph is not None else 0], device=dev)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if not int(ok.item()):
        graph = None

    def run():
        with torch.cuda.stream(stream):
            if graph is not None:
                graph.replay()
            else:
                step()

    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    barrier(world)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        barrier(world)
        ev0.record(stream)
        for _ in range(args.steps):
            run()
        ev1.record(stream)
        torch.cuda.synchronize()
    dev_ms = max_over_ranks(ev0.elapsed_time(ev1), world)
    clocks = clk.summary()
    ms_per_step = dev_ms / args.steps
    tok_s = M * args.steps / (dev_ms / 1e3)

    x_pin = torch.from_numpy(x_host.view(np.int16)).view(torch.bfloat16).pin_memory()
    lg_pin = torch.from_numpy(lg_host).pin_memory()
    y_pin = torch.empty(Ml, H, dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        with torch.cuda.stream(stream):
            h.copy_(x_pin, non_blocking=True)
            logits.copy_(lg_pin, non_blocking=True)
        run()
        with torch.cuda.stream(stream):
            y_pin.copy_(h, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world)
    e2e_tok_s = M * args.steps / (e2e_ms / 1e3)

    # per-kernel durations from one instrumented eager step
    moe.profile_reset()
    moe.profile_enable(True)
    with torch.cuda.stream(stream):
        step()
    torch.cuda.synchronize()
    moe.profile_enable(False)
    kids = (moe.KERNEL_PLAN, moe.KERNEL_UP, moe.KERNEL_ROWS, moe.KERNEL_COMBINE, moe.KERNEL_LAYER)
    kt = {kid: moe.profile_read(kid) for kid in kids}
    moe.profile_reset()
    launches = sum(n for _, n in kt.values())
    up_ms = kt[moe.KERNEL_UP][0] / max(kt[moe.KERNEL_UP][1], 1)
    dn_ms = kt[moe.KERNEL_ROWS][0] / max(kt[moe.KERNEL_ROWS][1], 1)
    up_b = (2 * I) * (H // 16) * 4 + (2 * I) * (H // gs) * 4
    up_bytes = sum(used) / L * up_b
    achieved = up_bytes / (up_ms * 1e-3) / 1e9 if kt[moe.KERNEL_UP][1] else None
    peak, peak_kind = load_peaks()
    if world > 1:  # dispatch + combine gathers/kernels beside the instrumented ones
        launches += 3 * L

    # --- parity (after the timed region): layer 0 of this rank's first tokens
    # from the initial activations, y = MoE(x), against the oracle; the worst
    # row and whether every rank's router indices match, over all ranks
    nchk = min(Ml, 8)
    x0 = torch.from_numpy(np.ascontiguousarray(x_host[:nchk]).view(np.int16)).to(dev).view(torch.bfloat16)
    y0 = torch.empty(nchk, H, dtype=torch.bfloat16, device=dev)
    i0 = torch.empty(Ml, K, dtype=torch.int32, device=dev)
    s0 = torch.empty(Ml, K, dtype=torch.float32, device=dev)
    with torch.cuda.stream(stream):
        moe.route(logits[0][:nchk].contiguous(), K, i0[:nchk], s0[:nchk], stream=stream)
        if world == 1:
            moe.forward(logits[0][:nchk].contiguous(), x0, W[0], y0, H=H, I=I, Ktop=K, gs=gs, M=nchk,
                        workspace=ws, stream=stream)
        else:
            eplayer.forward(x0, W[0], inds=i0[:nchk], scores=s0[:nchk], y=y0, stream=stream)
    if eplayer is not None:
        eplayer.status(stream)
    else:
        moe.synchronize(stream, ws)
    pr = oracle_check(cfg, W[0], lg_host[0][:nchk], x_host[:nchk],
                      y0.view(torch.int16).cpu().numpy().view(np.uint16), i0[:nchk].cpu().numpy(), expert_lo=lo)
    pv = torch.tensor([pr["max_rel_l2"], 1.0 if pr["idx_exact"] else 0.0], dtype=torch.float64, device=dev)
    if world > 1:
        import torch.distributed as dist
        mx = pv[:1].clone()
        mn = pv[1:].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(mn, op=dist.ReduceOp.MIN)
        pv = torch.cat([mx, mn])
    parity = {"tokens": nchk * world, "ranks": world, "max_rel_l2": float(pv[0].item()),
              "idx_exact": bool(pv[1].item() == 1.0), "tol": 2e-3}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        wh, xh, ihh, sh = host_layer_inputs(cfg, 0)
        cpu = cpu_layer_sample(cfg, wh, xh, ihh, sh, args.cpu_seconds)
    if rank == 0:
        line = {
            "metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "u8xs8->s32 tensor-core dot, f32 epilogue, bf16 I/O",
            "data": "synthetic (seeded generator, momij_b200/synth.py)",
            "config": {"workload": cfg["desc"], "H": H, "E": E, "top_k": K, "I": I, "gs": gs,
                       "M": M, "layers": L, "global_batch": M, "tokens_per_rank": Ml,
                       "experts_per_rank": El,
                       "parallelism": f"ep{world}" if world > 1 else "single",
                       "graph": graph is not None,
                       "l2": f"inputs larger than L2: {bytes_per_step / 1e9:.2f} GB of distinct "
                             "expert weights streamed per step on rank 0"},
            "hbm_tbs_rank0": bytes_per_step / (ms_per_step * 1e-3) / 1e12,
            "roofline": {"bound": "hbm", "kernel": "gemv_kernel<up||gate+SwiGLU>",
                         "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": (achieved / peak) if achieved else None, "traffic": None,
                         "peak_source": peak_kind, "bytes_per_launch": up_bytes,
                         "avg_launch_us": {"up": _us(up_ms), "down": _us(dn_ms),
                                           "plan": _us(kt[moe.KERNEL_PLAN][0] / max(kt[moe.KERNEL_PLAN][1], 1)),
                                           "combine": _us(kt[moe.KERNEL_COMBINE][0]
                                                          / max(kt[moe.KERNEL_COMBINE][1], 1)),
                                           "layer": _us(kt[moe.KERNEL_LAYER][0] / max(kt[moe.KERNEL_LAYER][1], 1))}},
            "launches_per_layer": {str(k): v[1] / L for k, v in kt.items()},
            "parity": parity,
            "clocks": clocks,
            "e2e": {"value": e2e_tok_s, "unit": "tokens/s", "h2d_bytes_per_step": x_pin.numel() * 2
                    + lg_pin.numel() * 4, "d2h_bytes_per_step": y_pin.numel() * 2,
                    "ms_per_step": e2e_ms / args.steps},
            "gpu_launches": launches * args.steps,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    del graph
    if eplayer is not None:
        torch.cuda.synchronize()
        eplayer.close()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def _us(ms):
    return None if ms is None else ms * 1e3


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="momij", choices=["momij", "reference"])
    ap.add_argument("--config", default=None, choices=sorted(CONFIGS),
                    help="default: decode (config 1) on one process; ep (config 4) under "
                         "torchrun with more than one rank")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--layers", type=int, default=None,
                    help="override the 48 layers (profiling captures of a small case only; "
                         "the reported metric is defined on 48 layers)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "momij" else args.warmup
    if args.config is None:
        args.config = "ep" if int(os.environ.get("WORLD_SIZE", "1")) > 1 else "decode"
    cfg = dict(CONFIGS[args.config])
    if args.layers:
        cfg["L"] = args.layers
        cfg["desc"] += f" [profiling case: {args.layers} layers]"
    if args.impl == "reference":
        run_reference(args, cfg)
    elif cfg.get("ep"):
        run_ep(args, cfg)
    else:
        run_gpu(args, cfg)


if __name__ == "__main__":
    main()
