"""The training step: render TRAIN -> fused L1+SSIM -> render backward -> (all-reduce) -> Adam.

Mirrors one iteration of GSX's session loop (gsx-runtime.c:1413-1536, without density control)
on the B200 path.  Parameters and gradients each live in ONE flat fp32 allocation with the GS
field order of gsx-core.h:287-302 (mean3d, logscale, rotation, opacity, sh0..sh3), every field
16-byte aligned, so the data-parallel gradient exchange is a single NCCL all-reduce over one
contiguous span (no per-field launches, no packing copies).
"""
from __future__ import annotations

import numpy as np
import torch

from . import FORWARD_TRAIN, Adam, Camera, ParamGroup, RenderContext, Renderer, l1_ssim

FIELD_ORDER = ("mean3d", "logscale", "rotation", "opacity", "sh0", "sh1", "sh2", "sh3")
FIELD_COLS = {"mean3d": (3,), "logscale": (3,), "rotation": (4,), "opacity": (), "sh0": (3,), "sh1": (3, 3),
              "sh2": (5, 3), "sh3": (7, 3)}
DEFAULT_LR = {"mean3d": 1e-3, "logscale": 1e-2, "rotation": 1e-2, "opacity": 1e-2, "sh0": 1e-2, "sh1": 1e-2,
              "sh2": 1e-2, "sh3": 1e-2}


class GaussianModel:
    """Gaussian parameters and gradients as views into two flat, 16-byte-aligned allocations."""

    def __init__(self, arrays: dict, device="cuda:0", sh_degree: int = 0):
        self.n = int(arrays["mean3d"].shape[0])
        self.sh_degree = sh_degree
        self.fields = [f for f in FIELD_ORDER if f in ("mean3d", "logscale", "rotation", "opacity", "sh0")
                       or int(f[2]) <= sh_degree]
        offs, o = {}, 0
        for f in self.fields:
            cnt = self.n * int(np.prod(FIELD_COLS[f], dtype=np.int64))
            offs[f] = (o, cnt)
            o += (cnt + 3) // 4 * 4
        self.numel = o
        self.offsets = offs
        # each field's padded [begin, end) in the flat buffers (16-byte aligned on both ends)
        self.field_ranges = {f: (a, a + (c + 3) // 4 * 4) for f, (a, c) in offs.items()}
        self._bind(torch.zeros(o, dtype=torch.float32, device=device), torch.zeros(o, dtype=torch.float32, device=device))
        for f in self.fields:
            src = np.ascontiguousarray(arrays[f], dtype=np.float32).reshape(self.params[f].shape)
            self.params[f].copy_(torch.from_numpy(src))

    def _bind(self, flat_param, flat_grad):
        self.flat_param, self.flat_grad = flat_param, flat_grad
        self.params, self.grads = {}, {}
        for f in self.fields:
            a, c = self.offsets[f]
            shape = (self.n,) + FIELD_COLS[f]
            self.params[f] = self.flat_param[a:a + c].view(shape)
            self.grads[f] = self.flat_grad[a:a + c].view(shape)

    def rebind(self, flat_param, flat_grad):
        """Move the parameters into other flat buffers (e.g. ones mapped into the peer ranks)."""
        flat_param.copy_(self.flat_param)
        flat_grad.zero_()
        self._bind(flat_param, flat_grad)


class Trainer:
    """One view per call of step(); `group` is a torch.distributed process group (None = 1 GPU)."""

    def __init__(self, model: GaussianModel, width: int, height: int, lr: dict | None = None, l1_weight=0.8,
                 ssim_weight=0.2, background=(0.0, 0.0, 0.0), group=None, device="cuda:0", exchange="fused"):
        """exchange (with a group): "fused" = gsx_b200.dp.ShardedAdam (gradient average + sharded Adam +
        parameter all-gather in one NVLink kernel per rank), through the NVSwitch (multimem reduce-load and
        multicast store) from 4 ranks up where every GPU supports it, else over peer loads and stores;
        "nvls" / "peer" force one form; "nccl" = all-reduce AVG then Adam everywhere."""
        self.model = model
        self.renderer = Renderer(width, height)
        self.ctx = RenderContext(torch.device(device).index or 0)
        self.out = torch.empty((3, height, width), dtype=torch.float32, device=device)
        self.loss_map = torch.empty_like(self.out)
        self.grad_rgb = torch.empty_like(self.out)
        self.loss_sum = torch.zeros(1, dtype=torch.float32, device=device)
        self.l1_weight, self.ssim_weight = l1_weight, ssim_weight
        self.background = background
        self.group = group
        lr = dict(DEFAULT_LR, **(lr or {}))
        self.sharded = None
        self.exchange = "nccl" if group is not None else None
        if group is not None and exchange in ("fused", "nvls", "peer"):
            self._setup_fused(model, group, device, lr, exchange)
        if self.sharded is None:
            self.optim = Adam([ParamGroup(f, model.params[f], model.grads[f], lr[f]) for f in model.fields])

    def _setup_fused(self, model, group, device, lr, exchange):
        """Map the flat buffers into every rank (NVSwitch multicast or CUDA IPC) and build the sharded
        optimizer.  The opening functions agree on the outcome across ranks (every rank runs the same
        collectives even when one fails locally), so all ranks fall back together: multicast -> peer
        mappings -> NCCL."""
        import warnings

        import torch.distributed as dist
        from .dp import ShardedAdam, open_multicast_buffers, open_peer_buffers
        bufs, err, form = None, None, None
        if exchange == "nvls" or (exchange == "fused" and dist.get_world_size(group) >= 4):
            bufs, err = open_multicast_buffers(model.numel, group, device, count=2)
            form = "nvls"
            if bufs is None:
                warnings.warn(f"NVSwitch multicast exchange unavailable ({err}); trying peer mappings")
        if bufs is None:
            bufs, err = open_peer_buffers(model.numel, group, device, count=2)
            form = "peer"
        if bufs is None:
            warnings.warn(f"fused NVLink exchange unavailable ({err}); using NCCL")
            return
        self._peer = bufs
        model.rebind(bufs[0].local, bufs[1].local)
        self.sharded = ShardedAdam(bufs[0], bufs[1], model.field_ranges, lr, group, device)
        self.optim = None
        self.exchange = "fused-" + form

    def step(self, camera: Camera, target, events=None):
        """One training iteration on `camera` against `target` ([3,H,W] on the device).
        Returns the device scalar holding the summed loss map of this view.  `events`, if given, is
        ((loss_start, loss_end), (adam_start, adam_end)) CUDA events recorded around those launches."""
        self.gradients(camera, target, events)
        return self.update(events)

    def gradients(self, camera: Camera, target, events=None):
        """Render TRAIN, fused L1+SSIM, render backward: this rank's gradients in model.flat_grad."""
        m = self.model
        self.renderer.render(self.ctx, m.params, camera, self.out, background=self.background,
                             sh_degree=m.sh_degree, forward_type=FORWARD_TRAIN)
        self.loss_sum.zero_()
        if events:
            events[0][0].record()
        l1_ssim(self.out, target, self.loss_map, self.grad_rgb, self.l1_weight, self.ssim_weight,
                loss_sum=self.loss_sum, overwrite=True)
        if events:
            events[0][1].record()
        self.renderer.backward(self.ctx, self.grad_rgb, m.grads)

    def update(self, events=None):
        """The gradient exchange (with a group) and Adam; returns the loss-sum device scalar."""
        m = self.model
        if self.sharded is not None:
            if events:
                events[1][0].record()
            self.sharded.step()
            if events:
                events[1][1].record()
            return self.loss_sum
        if self.group is not None:
            allreduce_mean(m.flat_grad, self.group)
        if events:
            events[1][0].record()
        self.optim.step(force_all=True)
        if events:
            events[1][1].record()
        return self.loss_sum

    def check_exchange(self, camera: Camera, target) -> dict:
        """Validate the sharded exchange on the hardware: from the current state, one step through the
        fused exchange, and the same step through the reference exchange (NCCL all-reduce AVG of the
        gradients, then the single-GPU Adam kernel over every parameter with the full moments gathered
        from the shards).  Returns the largest absolute and relative difference of the updated parameters
        (fused vs reference, max over ranks) and whether every rank holds bit-identical parameters.
        Leaves the model in the fused step's state."""
        import torch
        import torch.distributed as dist

        from . import Adam, ParamGroup
        from .dp import ALIGN, shard_bounds
        if self.sharded is None or self.group is None:
            raise RuntimeError("check_exchange needs the fused exchange on a process group")
        m, sh, grp = self.model, self.sharded, self.group
        world = dist.get_world_size(grp)
        self.gradients(camera, target)
        p0, g0 = m.flat_param.clone(), m.flat_grad.clone()
        # full moments from the shards (padded to the largest shard for one all-gather each)
        width = max(e - b for b, e in (shard_bounds(m.numel, world, r) for r in range(world)))
        width = max(width, ALIGN)
        full = []
        for mom in (sh.m1, sh.m2):
            pad = torch.zeros(width, dtype=torch.float32, device=mom.device)
            pad[: sh.end - sh.begin].copy_(mom[: sh.end - sh.begin])
            every = torch.empty(world * width, dtype=torch.float32, device=mom.device)
            dist.all_gather_into_tensor(every, pad, group=grp)
            f = torch.zeros(m.numel, dtype=torch.float32, device=mom.device)
            for r in range(world):
                b, e = shard_bounds(m.numel, world, r)
                f[b:e].copy_(every[r * width: r * width + (e - b)])
            full.append(f)
        steps = sh.steps
        self.update()  # the fused exchange
        torch.cuda.synchronize()
        p_fused = m.flat_param.clone()
        # the reference exchange from the same state
        g_avg = g0.clone()
        allreduce_mean(g_avg, grp)
        p_ref = p0.clone()
        groups = [ParamGroup(f, p_ref[a:b], g_avg[a:b], sh.lr[f]) for f, (a, b) in m.field_ranges.items()]
        opt = Adam(groups)
        for i, (f, (a, b)) in enumerate(m.field_ranges.items()):
            opt.m1[i].copy_(full[0][a:b])
            opt.m2[i].copy_(full[1][a:b])
            opt.steps[i] = steps
        opt.step(force_all=True)
        torch.cuda.synchronize()
        diff = (p_fused - p_ref).abs()
        moved = (p_ref - p0).abs()
        # one unit in the last place of each reference parameter: the two exchanges sum the gradients in
        # different orders, so a parameter may round one ulp apart; the relative check of the update only
        # covers updates resolved to at least 2^12 ulps, where that rounding is below 2.5e-4
        ulp = (torch.nextafter(p_ref, torch.full_like(p_ref, float("inf"))) - p_ref).abs()
        resolved = moved >= ulp * 4096
        rel = float((diff / moved.clamp_min(1e-30))[resolved].max()) if bool(resolved.any()) else 0.0
        stats = torch.tensor([float(diff.max()), rel],
                             dtype=torch.float64, device=p0.device)
        dist.all_reduce(stats, op=dist.ReduceOp.MAX, group=grp)
        # bit-identical replicas: a position-weighted hash of the parameter bits, compared over ranks
        bits = p_fused.view(torch.int32).to(torch.int64)
        h = int((bits * (torch.arange(bits.numel(), device=bits.device, dtype=torch.int64) % 1021 + 1)).sum())
        hashes = [None] * world
        dist.all_gather_object(hashes, h, group=grp)
        return {"reference": "NCCL all-reduce AVG + single-GPU Adam over every parameter (moments gathered)",
                "max_abs_diff": float(stats[0]), "max_rel_diff_of_update": float(stats[1]),
                "replicas_identical": all(x == hashes[0] for x in hashes)}

    def close(self):
        """Release the peer mappings: every rank unmaps, a barrier, then every rank frees its own."""
        if self.sharded is not None:
            import torch
            import torch.distributed as dist
            torch.cuda.synchronize()
            for b in self._peer:
                b.close_peers()
            dist.barrier(group=self.group)
            for b in self._peer:
                b.free()
            self.sharded = None


def allreduce_mean(flat, group):
    """In-place mean of `flat` over the ranks of `group`: one collective over the whole span.
    NCCL averages in the collective (ReduceOp.AVG); other backends (gloo, used by the CPU tests)
    sum and scale."""
    import torch.distributed as dist
    if dist.get_backend(group) == "nccl":
        dist.all_reduce(flat, op=dist.ReduceOp.AVG, group=group)
    else:
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
        flat.div_(dist.get_world_size(group))


class HostFeed:
    """Per-step host I/O of a training loop: each step's target image goes from pinned host memory to
    the device on a copy stream, double-buffered, so the upload of step s+1 overlaps step s; each
    step's loss comes back into pinned host memory and is read one step later (no per-step stall of
    the compute stream).  Every step still moves its full target in and its loss out."""

    def __init__(self, shape, device):
        import torch
        self.device = torch.device(device)
        self.copy_stream = torch.cuda.Stream(self.device)
        self.buf = [torch.empty(shape, dtype=torch.float32, device=self.device) for _ in range(2)]
        self.ready = [torch.cuda.Event() for _ in range(2)]
        self.free = [None, None]
        self.loss_host = torch.zeros(2, dtype=torch.float32).pin_memory()
        self.loss_ev = [torch.cuda.Event() for _ in range(2)]
        self.pending = [False, False]

    def upload(self, host_tensor, slot: int):
        """Queue the copy of `host_tensor` (pinned) into buffer `slot` once its previous user is done."""
        import torch
        with torch.cuda.stream(self.copy_stream):
            if self.free[slot] is not None:
                self.copy_stream.wait_event(self.free[slot])
            self.buf[slot].copy_(host_tensor, non_blocking=True)
            self.ready[slot].record(self.copy_stream)

    def target(self, slot: int):
        """Buffer `slot` for the compute stream (ordered after its upload)."""
        import torch
        torch.cuda.current_stream(self.device).wait_event(self.ready[slot])
        return self.buf[slot]

    def finish(self, slot: int, loss):
        """The step that used buffer `slot` is queued: release the buffer and queue its loss read."""
        import torch
        ev = torch.cuda.Event()
        ev.record()
        self.free[slot] = ev
        self.loss_host[slot:slot + 1].copy_(loss, non_blocking=True)
        self.loss_ev[slot].record()
        self.pending[slot] = True

    def read_loss(self, slot: int) -> float:
        """The loss of the step that used buffer `slot` (waits only for that step)."""
        if not self.pending[slot]:
            return float("nan")
        self.loss_ev[slot].synchronize()
        self.pending[slot] = False
        return float(self.loss_host[slot])
