"""Expert-parallel MoE layer (north-star config 4): experts sharded evenly and
contiguously over the ranks of a torch.distributed group, one all-to-all to
dispatch the (token, slot) pairs to the ranks owning their experts and one to
return the expert outputs, then the score-weighted combine in k order.

Per layer, on every rank (M tokens of its own, K slots each):
  route -> dispatch (momij_moe_ep_dispatch: fixed-capacity rows per
  destination, deterministic slots; the destination's expert indices ride in
  one extra row of its segment) -> all_to_all(rows) -> local experts
  (momij_moe_gqmm2_up_swiglu + momij_moe_gqmm2 over the received rows; empty
  rows carry expert -1 and are skipped) -> all_to_all(outputs) -> combine
  (momij_moe_ep_combine into the residual stream).

The buffers hold `capacity = M*K` pair rows (+ the index row) per
destination, so no rank ever needs the counts on the host (no device-to-host synchronisation per layer);
the exchanges are all_to_all_single with equal splits over NCCL (NVLink).
The result has the same bits as the single-GPU path on the same tokens: each
pair's expert output is computed with the same kernel and the combine sums in
the same order.

`ops` supplies the per-rank kernels (GpuOps: the C ABI); the collectives come
from torch.distributed, so the same protocol runs on CPU tensors over gloo.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import moe


class GpuOps:
    """Per-rank kernels through libmomij_moe.so."""

    def __init__(self, wts_local: dict, *, H: int, I: int, gs: int = 64, clamp: float = 7.0,
                 stream=None):
        self.w, self.H, self.I, self.gs, self.clamp, self.stream = wts_local, H, I, gs, clamp, stream
        self.ws = None

    def route(self, logits, K, inds, scores):
        moe.route(logits, K, inds, scores, stream=self.stream)

    def dispatch(self, inds, x, send_x, send_meta, slot_map, status, *, E, world, capacity):
        moe.ep_dispatch(inds, x, send_x, send_meta, slot_map, status, E=E, world=world,
                        capacity=capacity, stream=self.stream)

    def experts(self, recv_x, recv_meta, act, down):
        rows = recv_x.shape[0]
        if self.ws is None:
            self.ws = moe.new_workspace(rows, 1, 0, 0, recv_x.device)
        w = self.w
        moe.gqmm2_up_swiglu(recv_x, w["w_ug"], w["s_ug"], w["b_ug"], recv_meta, act, Ktop=1, K=self.H,
                            I=self.I, gs=self.gs, M=rows, clamp=self.clamp, workspace=self.ws,
                            stream=self.stream)
        moe.gqmm2(act, w["w_dn"], w["s_dn"], w["b_dn"], recv_meta, down, Ktop=1, K=self.I, N=self.H,
                  gs=self.gs, M=rows, workspace=self.ws, stream=self.stream)

    def combine(self, back, scores, slot_map, status, h):
        moe.ep_combine(back, scores, slot_map, status, resid_h=h, stream=self.stream)


class ExpertParallelMoE:
    """One MoE FFN layer sharded by expert over `group` (rank r owns experts
    [r*E/world, (r+1)*E/world)); forward() updates the rank's residual stream
    h [M, H] in place from its router logits [M, E]."""

    def __init__(self, ops, *, E: int, H: int, I: int, K: int, M: int, group=None,
                 device=None, dtype=torch.bfloat16):
        self.ops, self.E, self.H, self.I, self.K, self.M = ops, E, H, I, K, M
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        if E % self.world:
            raise ValueError("experts must split evenly over the ranks")
        # per destination: M*K pair rows (a rank's pairs may all go to one
        # owner) + one row whose first words carry the rows' local expert
        # indices, so one all-to-all moves rows and indices together
        self.capacity = M * K
        self.seg = self.capacity + 1
        if self.seg > H // 2:
            raise ValueError("the index row needs M*K + 1 <= H / 2")
        if self.world * self.seg > moe.MAX_PAIRS:
            # the experts step runs gqmm2 with one slot per received row
            raise ValueError(f"world * (M*K + 1) = {self.world * self.seg} received rows exceeds "
                             f"{moe.MAX_PAIRS} (MOMIJ_MAX_PAIRS): use fewer tokens per rank")
        rows = self.world * self.seg
        dev = device if device is not None else torch.device("cpu")
        self.inds = torch.empty(M, K, dtype=torch.int32, device=dev)
        self.scores = torch.empty(M, K, dtype=torch.float32, device=dev)
        self.send_x = torch.zeros(rows, H, dtype=dtype, device=dev)
        self.send_meta = torch.full((rows,), -1, dtype=torch.int32, device=dev)
        self.act = torch.zeros(rows, I, dtype=dtype, device=dev)
        self.down = torch.zeros(rows, H, dtype=dtype, device=dev)
        if self.world == 1:  # nothing to exchange: the receive side aliases the send side
            self.recv_x, self.recv_meta, self.back = self.send_x, self.send_meta, self.down
        else:
            self.recv_x = torch.zeros(rows, H, dtype=dtype, device=dev)
            self.recv_meta = torch.full((rows,), -1, dtype=torch.int32, device=dev)
            self.back = torch.zeros(rows, H, dtype=dtype, device=dev)
        self.slot_map = torch.empty(M * K, dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)

    def _exchange(self, out, inp):
        if out is inp:
            return
        if self.world == 1:
            out.copy_(inp)
        else:  # the exchange only moves bytes: 16-bit rows travel as int32 pairs
            if inp.element_size() == 2:
                out, inp = out.view(torch.int32), inp.view(torch.int32)
            dist.all_to_all_single(out, inp, group=self.group)

    def check(self) -> None:
        """Waits for the layer and raises SeedlessError if it failed: a bad
        expert index or capacity overflow (the status word; the combine then
        leaves h untouched) or an error of the experts' kernels."""
        if self.status.is_cuda:
            torch.cuda.current_stream(self.status.device).synchronize()
        s = int(self.status.item())
        if s != moe.OK:
            raise moe.SeedlessError(s, "expertParallel")
        if getattr(self.ops, "ws", None) is not None:
            moe.synchronize(getattr(self.ops, "stream", None), self.ops.ws)

    def forward(self, logits, h):
        """Enqueues one layer (no host synchronisation).  h is updated only
        when the layer succeeds: call check() (or read `status`) before
        trusting it."""
        o = self.ops
        o.route(logits, self.K, self.inds, self.scores)
        o.dispatch(self.inds, h, self.send_x, self.send_meta, self.slot_map, self.status, E=self.E,
                   world=self.world, capacity=self.seg)
        if self.world > 1:
            w, c = self.world, self.capacity
            sx = self.send_x.view(torch.int32).view(w, self.seg, -1)
            sx[:, c, :self.seg].copy_(self.send_meta.view(w, self.seg))  # slot c itself is empty (-1)
            self._exchange(self.recv_x, self.send_x)
            rx = self.recv_x.view(torch.int32).view(w, self.seg, -1)
            self.recv_meta.view(w, self.seg).copy_(rx[:, c, :self.seg])
        o.experts(self.recv_x, self.recv_meta, self.act, self.down)
        self._exchange(self.back, self.down)
        o.combine(self.back, self.scores, self.slot_map, self.status, h)
        return h


def shard_experts(wts: dict, rank: int, world: int) -> dict:
    """The expert slice [rank*E/world, (rank+1)*E/world) of a weight dict."""
    E = wts["w_ug"].shape[0]
    lo, hi = rank * E // world, (rank + 1) * E // world
    return {k: (v[lo:hi].contiguous() if isinstance(v, torch.Tensor) else v[lo:hi].copy())
            for k, v in wts.items()}
