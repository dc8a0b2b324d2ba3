"""Host-side data-parallel logic on CPU (gloo, world size 2): no GPU needed.

Covers what the multi-GPU training step does besides the kernels: the flat gradient layout (one
collective per step), the averaging all-reduce (NCCL AVG on the GPU, SUM + scale on gloo), replicas
staying identical after an update, and a rank that dies before the collective being detected by the
survivor as an error instead of a hang.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gsx_b200.train import FIELD_ORDER, GaussianModel, allreduce_mean


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _scene(n, seed):
    rng = np.random.default_rng(seed)
    return dict(mean3d=rng.normal(size=(n, 3)).astype(np.float32), rotation=rng.normal(size=(n, 4)).astype(np.float32),
                logscale=rng.normal(size=(n, 3)).astype(np.float32), opacity=rng.normal(size=n).astype(np.float32),
                sh0=rng.normal(size=(n, 3)).astype(np.float32), sh1=rng.normal(size=(n, 3, 3)).astype(np.float32))


def _worker(rank, world, port, mode, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        model = GaussianModel(_scene(101, 0), device="cpu", sh_degree=1)
        if mode == "dead_peer":
            if rank == 1:
                os._exit(0)  # leaves between steps, before the collective
            try:
                allreduce_mean(model.flat_grad, dist.group.WORLD)
                out.put((rank, "no error"))
            except Exception as e:  # noqa: BLE001 - any backend error is the detection we want
                out.put((rank, "detected: " + type(e).__name__))
            return
        # rank-specific gradients, then one averaging collective over the whole flat span
        for i, f in enumerate(model.fields):
            model.grads[f].fill_(float(rank + 1) * (i + 1))
        allreduce_mean(model.flat_grad, dist.group.WORLD)
        lr = 0.1
        model.flat_param.sub_(lr * model.flat_grad)  # stand-in update: identical on every rank
        out.put((rank, model.flat_grad.numpy().copy(), model.flat_param.numpy().copy(),
                 {f: (model.params[f].data_ptr() - model.flat_param.data_ptr()) for f in model.fields}))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:  # noqa: BLE001
                pass


def _run(mode, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    for _ in range(world if mode != "dead_peer" else 1):
        results.append(q.get(timeout=60))
    for p in procs:
        p.join(timeout=60)
    return results


def test_flat_layout_is_aligned_and_in_gsx_field_order():
    m = GaussianModel(_scene(37, 1), device="cpu", sh_degree=1)
    assert m.fields == [f for f in FIELD_ORDER if f in m.fields]
    prev = -1
    for f in m.fields:
        off = m.params[f].data_ptr() - m.flat_param.data_ptr()
        assert off % 16 == 0 and off > prev
        prev = off
        assert m.grads[f].data_ptr() - m.flat_grad.data_ptr() == off
    np.testing.assert_array_equal(m.params["sh1"].numpy(), _scene(37, 1)["sh1"])


def test_gradient_average_and_replicas_stay_identical():
    res = sorted(_run("ok"), key=lambda r: r[0])
    (_, g0, p0, off0), (_, g1, p1, off1) = res
    np.testing.assert_array_equal(g0, g1)
    np.testing.assert_array_equal(p0, p1)
    assert off0 == off1
    # mean of (1 * k) and (2 * k) for field k
    m = GaussianModel(_scene(101, 0), device="cpu", sh_degree=1)
    for i, f in enumerate(m.fields):
        a = off0[f] // 4
        assert g0[a] == pytest.approx(1.5 * (i + 1))


def test_dead_peer_is_detected_not_hung():
    res = _run("dead_peer")
    assert res[0][0] == 0
    assert res[0][1].startswith("detected"), res


def _band_worker(rank, world, port, height, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        from gsx_b200 import band_rows
        mine = torch.tensor(band_rows(height, rank, world), dtype=torch.int64)
        every = [torch.zeros(2, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(every, mine)
        if rank == 0:
            out.put([tuple(int(x) for x in t) for t in every])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("height,world", [(2160, 2), (2160, 8), (101, 3), (20, 4)])
def test_band_rows_partition_the_frame(height, world):
    """Each rank's band starts on a tile row; the bands, gathered over gloo, tile [0, height) in rank order."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_band_worker, args=(r, world, port, height, q)) for r in range(world)]
    for p in procs:
        p.start()
    bands = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    pos = 0
    for b0, b1 in bands:
        assert b0 == pos and b1 >= b0 and (b0 % 16 == 0 or b1 == b0)
        pos = b1
    assert pos == height
    tiles = [(b1 - b0 + 15) // 16 for b0, b1 in bands if b1 > b0]
    assert max(tiles) - min(tiles) <= 1


@pytest.mark.parametrize("numel,world", [(4, 1), (400, 3), (12348, 8), (16, 8), (1_000_000, 4)])
def test_shards_cover_the_flat_space(numel, world):
    from gsx_b200.dp import shard_bounds, shard_segments
    bounds = [shard_bounds(numel, world, r) for r in range(world)]
    pos = 0
    for b, e in bounds:
        assert b == pos and e >= b and b % 4 == 0 and e % 4 == 0
        pos = e
    assert pos == numel
    ranges = {"a": (0, numel // 2 // 4 * 4), "b": (numel // 2 // 4 * 4, numel)}
    covered = 0
    for b, e in bounds:
        runs = shard_segments(ranges, b, e)
        for f, lo, hi in runs:
            assert ranges[f][0] <= lo < hi <= ranges[f][1] and b <= lo and hi <= e
            covered += hi - lo
    assert covered == numel


class _FakeIpc:
    """Host stand-in for the device/IPC calls of gsx_b200.dp.open_peer_buffers: CPU tensors as
    'device buffers', integer ids as pointers and handles.  `fail` = (stage, rank) makes that call
    raise on that rank only."""

    def __init__(self, rank, fail):
        self.rank, self.fail = rank, fail
        self.live, self.opened, self.next = {}, set(), 1000 * (rank + 1)

    def _maybe_fail(self, stage):
        if self.fail == (stage, self.rank):
            raise RuntimeError(f"injected {stage} failure on rank {self.rank}")

    def alloc(self, nbytes):
        self._maybe_fail("alloc")
        self.next += 1
        self.live[self.next] = torch.zeros(nbytes // 4)
        return self.next

    def handle(self, ptr):
        return int(ptr).to_bytes(8, "little")

    def open(self, handle):
        self._maybe_fail("open")
        p = int.from_bytes(handle, "little") + 10**6
        self.opened.add(p)
        return p

    def close(self, ptr):
        self.opened.remove(ptr)

    def free(self, ptr):
        del self.live[ptr]

    def tensor(self, ptr, numel, device):
        return self.live[ptr][:numel]


def _peer_worker(rank, world, port, fail, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        from gsx_b200.dp import open_peer_buffers
        api = _FakeIpc(rank, fail)
        bufs, err = open_peer_buffers(64, dist.group.WORLD, "cpu", count=2, api=api)
        # a collective after the setup: every rank must still be in step
        t = torch.ones(1)
        dist.all_reduce(t)
        ptrs = [list(b.ptrs) for b in bufs] if bufs else None
        out.put((rank, bufs is not None, err, len(api.live), len(api.opened), float(t.item()), ptrs))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fail", [None, ("alloc", 1), ("open", 1), ("open", 0)])
def test_peer_mapping_failure_on_one_rank_falls_back_on_every_rank(fail):
    """A failure of the allocation or of a peer mapping on ONE rank: every rank still runs the same
    collectives, every rank returns no buffers (NCCL fallback), releases what it mapped and allocated,
    and the next collective completes (no mismatched collectives, no hang)."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, world, port, fail, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=120) for _ in range(world)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok, err, live, opened, total, ptrs in res:
        assert total == world
        if fail is None:
            assert ok and err is None and live == 2 and opened == 2 * (world - 1)
            assert all(None not in p for p in ptrs)
        else:
            assert not ok and err and live == 0 and opened == 0, (rank, err, live, opened)


def test_balanced_bands_cover_the_frame_and_even_out_work():
    """The equal-work cut of large-frame inference: whole tile rows, in order, covering [0, height),
    the same on every rank, and no band above the ideal share by more than one tile row's cost."""
    from gsx_b200 import balanced_band_rows
    rng = np.random.default_rng(3)
    height = 2160
    tiles = (height + 15) // 16
    costs = (rng.gamma(0.5, 1000.0, tiles) * (np.arange(tiles) > 40)).astype(np.uint32)  # empty sky, dense ground
    for world in (1, 2, 3, 4, 8):
        bands = [balanced_band_rows(costs, height, r, world) for r in range(world)]
        pos = 0
        for b0, b1 in bands:
            assert b0 == pos and b1 >= b0 and b0 % 16 == 0
            pos = b1
        assert pos == height
        share = [int(costs[b0 // 16:(b1 + 15) // 16].sum()) for b0, b1 in bands]
        assert max(share) <= costs.sum() / world + costs.max()
    # no work anywhere: the even split
    from gsx_b200 import band_rows
    assert balanced_band_rows(np.zeros(tiles, np.uint32), height, 2, 8) == band_rows(height, 2, 8)
