"""Data-parallel training over NVLink with the fused gradient exchange + sharded Adam.

Two forms of the exchange kernel: peer loads and stores over CUDA IPC mappings (below), and NVLink
SHARP through the NVSwitch (MulticastBuffers: the switch sums the gradients and replicates the updated
parameters; fewer bytes per rank from 4 ranks up).

One process per GPU.  The flat parameter and gradient buffers of every rank are mapped into every
other rank's process (CUDA IPC over the NVSwitch fabric); each rank owns one contiguous shard of the
flat parameter space and runs gsx_b200_dp_reduce_adam_gather on it: peer loads of the shard's
gradients from all ranks, the average, Adam with shard-local moments, peer stores of the updated
shard into all ranks' parameters.  Two collectives order it on the stream: one before (every rank's
backward has finished writing its gradients) and one after (every rank's shard has landed in every
parameter buffer before anyone renders again).

The same arithmetic as an average all-reduce (sum in rank order, times 1/world) followed by Adam on
every rank, so the replicas stay identical; the moments are sharded (1/world of them per rank).
"""
from __future__ import annotations

import ctypes
import math

from ._capi import GsxError, INVALID_ARGUMENT, check, lib

ALIGN = 4  # elements: shard and segment bounds stay 16-byte aligned


class _CudaArray:
    """A raw device pointer presented to torch through __cuda_array_interface__."""

    def __init__(self, ptr: int, numel: int):
        self.__cuda_array_interface__ = {"shape": (numel,), "typestr": "<f4", "data": (ptr, False), "version": 3}


def shard_bounds(numel: int, world: int, rank: int):
    """[begin, end) of rank's shard of `numel` flat elements: contiguous, multiples of 4 elements,
    sizes as even as the alignment allows (earlier ranks take the remainder)."""
    if world < 1 or not 0 <= rank < world or numel % ALIGN:
        raise GsxError(INVALID_ARGUMENT, "shard_bounds: numel a multiple of 4, 0 <= rank < world")
    units = numel // ALIGN
    base, extra = divmod(units, world)
    b = rank * base + min(rank, extra)
    e = b + base + (1 if rank < extra else 0)
    return b * ALIGN, e * ALIGN


def shard_segments(field_ranges: dict, begin: int, end: int):
    """The runs of one field inside [begin, end): [(field, run_begin, run_end)] in flat order."""
    out = []
    for f, (a, b) in field_ranges.items():
        lo, hi = max(a, begin), min(b, end)
        if lo < hi:
            out.append((f, lo, hi))
    return sorted(out, key=lambda s: s[1])


class DeviceIpc:
    """The device-memory and CUDA IPC calls the peer mapping needs (the C ABI).  A stand-in with the
    same methods lets the host-side protocol run on CPU ranks (tests)."""

    def alloc(self, nbytes: int) -> int:
        raw = ctypes.c_void_p()
        check(lib().gsx_b200_device_alloc(nbytes, ctypes.byref(raw)))
        return raw.value

    def handle(self, ptr: int) -> bytes:
        h = (ctypes.c_ubyte * 64)()
        check(lib().gsx_b200_ipc_handle(ctypes.c_void_p(ptr), h))
        return bytes(h)

    def open(self, handle: bytes) -> int:
        p = ctypes.c_void_p()
        check(lib().gsx_b200_ipc_open((ctypes.c_ubyte * 64).from_buffer_copy(handle), ctypes.byref(p)))
        return p.value

    def close(self, ptr: int) -> None:
        lib().gsx_b200_ipc_close(ctypes.c_void_p(ptr))

    def free(self, ptr: int) -> None:
        lib().gsx_b200_device_free(ctypes.c_void_p(ptr))

    def tensor(self, ptr: int, numel: int, device):
        import torch
        return torch.as_tensor(_CudaArray(ptr, numel), device=device)


class PeerBuffers:
    """One flat f32 device buffer of `numel` elements per rank, every rank's buffer mapped into this
    process.  `local` is this rank's buffer as a torch tensor; `ptrs[r]` is rank r's buffer here.
    Built by open_peer_buffers, which keeps every rank in step when a rank fails."""

    def __init__(self, api, world: int, rank: int, own: int, local):
        self.api, self.world, self.rank = api, world, rank
        self._own, self.local = own, local
        self.ptrs = [own if r == rank else None for r in range(world)]
        self._opened = []

    def close_peers(self):
        """Unmap the other ranks' buffers (call on every rank before any rank frees its own)."""
        for p in self._opened:
            self.api.close(p)
        self._opened = []

    def free(self):
        if self._own:
            self.local = None
            self.api.free(self._own)
            self._own = None


def _agree(ok: bool, group) -> bool:
    """Every rank learns whether all ranks succeeded (one object all-gather; works on NCCL and gloo)."""
    import torch.distributed as dist
    flags = [None] * dist.get_world_size(group)
    dist.all_gather_object(flags, bool(ok), group=group)
    return all(flags)


def open_peer_buffers(numel: int, group, device, count: int = 2, api=None):
    """`count` PeerBuffers of `numel` f32 each, or (None, reason) on EVERY rank if any rank failed.

    Every rank runs the same collectives in the same order whatever happens locally: stage 1 allocates
    and exports IPC handles (a failed rank contributes None to the handle all-gather), stage 2 maps the
    peers and agrees on the result.  On failure every rank unmaps what it opened, meets a barrier (so no
    buffer is freed while a peer still maps it) and frees what it allocated."""
    import torch.distributed as dist
    api = api or DeviceIpc()
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    bufs, err = [], None
    handles_mine = None
    try:
        for _ in range(count):
            own = api.alloc(numel * 4)
            bufs.append(PeerBuffers(api, world, rank, own, None))
            bufs[-1].local = api.tensor(own, numel, device)
            bufs[-1].local.zero_()
        handles_mine = [api.handle(b._own) for b in bufs]
    except Exception as e:  # noqa: BLE001 - reported through the all-gather below
        err, handles_mine = e, None
    every = [None] * world
    dist.all_gather_object(every, handles_mine, group=group)
    ok = all(h is not None for h in every)
    if ok:
        try:
            for k, b in enumerate(bufs):
                for r in range(world):
                    if r != rank:
                        p = api.open(every[r][k])
                        b.ptrs[r] = p
                        b._opened.append(p)
        except Exception as e:  # noqa: BLE001 - agreed on below
            err = e
    ok = _agree(ok and err is None, group)
    if ok:
        return tuple(bufs), None
    for b in bufs:
        b.close_peers()
    dist.barrier(group=group)
    for b in bufs:
        b.free()
    return None, (str(err) if err is not None else "failed on another rank")


class MulticastBuffers:
    """One flat f32 buffer of `numel` elements per rank in symmetric memory, with an NVSwitch multicast
    address bound to all ranks' buffers (`mc_ptr`): a multimem store there writes every rank's copy, a
    multimem reduce-load returns the sum over the ranks.  Built by open_multicast_buffers."""

    def __init__(self, world: int, rank: int, local, handle):
        self.world, self.rank = world, rank
        self.local, self.handle = local, handle
        self.mc_ptr = int(handle.multicast_ptr)

    def close_peers(self):
        pass

    def free(self):
        self.local, self.handle = None, None


def multicast_supported(device) -> bool:
    """This process's GPU can bind memory to NVSwitch multicast objects."""
    import torch
    try:
        from torch.distributed._symmetric_memory import DeviceType
        return bool(torch._C._distributed_c10d._SymmetricMemory.has_multicast_support(
            DeviceType.CUDA, torch.device(device).index or 0))
    except Exception:  # noqa: BLE001 - no symmetric memory in this build: not supported
        return False


def open_multicast_buffers(numel: int, group, device, count: int = 2):
    """`count` MulticastBuffers of `numel` f32 each, or (None, reason) on EVERY rank when any rank
    cannot: multicast support, the allocations and the multicast addresses are agreed on collectively,
    so all ranks take the same exchange."""
    import torch
    import torch.distributed as dist
    import torch.distributed._symmetric_memory as symm_mem
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    if not _agree(multicast_supported(device), group):
        return None, "NVSwitch multicast is not supported on every rank"
    tensors, err = [], None
    try:
        for _ in range(count):
            tensors.append(symm_mem.empty(numel, dtype=torch.float32, device=device))
    except Exception as e:  # noqa: BLE001 - agreed on below
        err = e
    if not _agree(err is None, group):
        return None, str(err) if err is not None else "symmetric allocation failed on another rank"
    bufs = []
    for t in tensors:
        h = symm_mem.rendezvous(t, group)
        t.zero_()
        bufs.append(MulticastBuffers(world, rank, t, h))
    if not _agree(all(b.mc_ptr != 0 for b in bufs), group):
        for b in bufs:
            b.free()
        return None, "no multicast address on every rank"
    torch.cuda.synchronize(device)
    dist.barrier(group=group)
    return tuple(bufs), None


class Segment(ctypes.Structure):
    _fields_ = [("begin", ctypes.c_uint64), ("end", ctypes.c_uint64), ("learning_rate", ctypes.c_float),
                ("beta1", ctypes.c_float), ("beta2", ctypes.c_float), ("epsilon", ctypes.c_float),
                ("weight_decay", ctypes.c_float), ("max_grad", ctypes.c_float),
                ("inv_bias_correction1", ctypes.c_double), ("inv_bias_correction2", ctypes.c_double)]


class ShardedAdam:
    """Adam over this rank's shard, fused with the gradient average and the parameter all-gather.
    `field_ranges` maps each role to its [begin, end) in the flat buffers; `lr` maps role -> rate."""

    def __init__(self, params, grads, field_ranges: dict, lr: dict, group, device, beta1=0.9, beta2=0.999,
                 epsilon=1e-8):
        """params / grads: PeerBuffers (peer loads and stores, gsx_b200_dp_reduce_adam_gather) or
        MulticastBuffers (NVSwitch reduce-load and multicast store, gsx_b200_dp_nvls_reduce_adam_broadcast)."""
        import torch
        self.params, self.grads, self.group = params, grads, group
        self.nvls = isinstance(params, MulticastBuffers)
        self.world, self.rank = params.world, params.rank
        numel = params.local.numel()
        self.begin, self.end = shard_bounds(numel, self.world, self.rank)
        self.runs = shard_segments(field_ranges, self.begin, self.end)
        n = self.end - self.begin
        self.m1 = torch.zeros(max(n, ALIGN), dtype=torch.float32, device=device)
        self.m2 = torch.zeros(max(n, ALIGN), dtype=torch.float32, device=device)
        self.lr = dict(lr)
        self.beta1, self.beta2, self.epsilon = beta1, beta2, epsilon
        self.steps = 0
        self.token = torch.zeros(1, dtype=torch.float32, device=device)
        self.kernel_events = None  # optional list receiving (start, end) CUDA events around each launch
        if not self.nvls:
            P = ctypes.c_void_p * self.world
            self._params = P(*self.params.ptrs)
            self._grads = P(*self.grads.ptrs)

    def _barrier(self):
        import torch.distributed as dist
        dist.all_reduce(self.token, group=self.group)

    def step(self, stream=None):
        from . import _stream_handle
        self.steps += 1
        b1 = float(ctypes.c_float(self.beta1).value)
        b2 = float(ctypes.c_float(self.beta2).value)
        segs = (Segment * max(len(self.runs), 1))()
        for k, (f, a, b) in enumerate(self.runs):
            s = segs[k]
            s.begin, s.end = a, b
            s.learning_rate, s.beta1, s.beta2, s.epsilon = self.lr[f], self.beta1, self.beta2, self.epsilon
            s.weight_decay, s.max_grad = 0.0, 0.0
            s.inv_bias_correction1 = 1.0 / (1.0 - math.pow(b1, self.steps))
            s.inv_bias_correction2 = 1.0 / (1.0 - math.pow(b2, self.steps))
        self._barrier()
        ev = None
        if self.kernel_events is not None:
            import torch
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        if self.nvls:
            check(lib().gsx_b200_dp_nvls_reduce_adam_broadcast(
                self.world, ctypes.c_void_p(self.params.mc_ptr), ctypes.c_void_p(self.grads.mc_ptr),
                ctypes.c_void_p(self.params.local.data_ptr()), ctypes.c_void_p(self.m1.data_ptr()),
                ctypes.c_void_p(self.m2.data_ptr()), self.begin, self.end, segs, len(self.runs), _stream_handle(stream)))
        else:
            check(lib().gsx_b200_dp_reduce_adam_gather(self.world, self.rank, self._params, self._grads,
                                                       ctypes.c_void_p(self.m1.data_ptr()),
                                                       ctypes.c_void_p(self.m2.data_ptr()), self.begin, self.end, segs,
                                                       len(self.runs), _stream_handle(stream)))
        if ev is not None:
            ev[1].record()
            self.kernel_events.append(ev)
        self._barrier()

    def nvlink_bytes(self) -> int:
        """Bytes this rank moves over NVLink per step and direction.  Peer form: its shard's gradients read
        from the other ranks and its updated shard written to them, 2 (world - 1) shards.  Multicast form:
        out, all its gradients to the switch plus its updated shard; in, the reduced shard plus every
        rank's updated shard: 1 + 1/world of the flat buffer."""
        shard = (self.end - self.begin) * 4
        if self.nvls:
            return shard * self.world + shard
        return 2 * (self.world - 1) * shard
