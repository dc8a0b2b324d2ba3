"""The fused data-parallel exchange on real GPUs (one process per GPU, NCCL for the two ordering
collectives), in both forms: CUDA IPC peer mappings, and NVSwitch multicast (multimem reduce-load and
multicast store).  After a few training steps the replicas are bit-identical and agree with the NCCL
all-reduce + Adam path to float rounding; Trainer.check_exchange compares one step of each form with
the NCCL reference from the same state.  Skipped on a box with fewer than two GPUs (the single-GPU
emulation in test_gpu_dp.py covers the peer form's arithmetic)."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, exchange, q):
    import torch.distributed as dist

    from gsx_b200 import scenes
    from gsx_b200.train import GaussianModel, Trainer
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device(f"cuda:{rank}"))
    try:
        dev = f"cuda:{rank}"
        g, cam = scenes.small_scene(0, 20000, 160, 120, 0, scale_mu=-2.5)
        t = scenes.small_scene(1, 20000, 160, 120, 0, scale_mu=-2.5)[0]
        model = GaussianModel(g, dev)
        teacher = GaussianModel(t, dev)
        import gsx_b200 as gb
        target = torch.empty((3, 120, 160), device=dev)
        ctx = gb.RenderContext(rank)
        gb.Renderer(160, 120).render(ctx, teacher.params, cam, target, forward_type=gb.FORWARD_INFERENCE)
        ctx.close()
        # each rank trains on its own camera (shifted view)
        cam = gb.Camera(cam.width, cam.height, cam.fx, cam.fy, cam.cx + 3.0 * rank, cam.cy, cam.rot_xyzw, cam.transl,
                        cam.near_plane, cam.far_plane)
        tr = Trainer(model, 160, 120, group=dist.group.WORLD, device=dev, exchange=exchange)
        for _ in range(4):
            tr.step(cam, target)
        torch.cuda.synchronize()
        out = model.flat_param.cpu().numpy().copy()
        chk = tr.check_exchange(cam, target) if tr.sharded is not None else None
        form = tr.exchange
        tr.close()
        q.put((rank, (out, chk, form)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _run(exchange, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, exchange, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return [res[r] for r in range(world)]


@pytest.mark.parametrize("exchange", ["peer", "nvls"])
def test_fused_exchange_two_gpus(exchange):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    res = _run(exchange)
    (p0, chk0, form), (p1, chk1, _) = res
    if exchange == "nvls" and form != "fused-nvls":
        pytest.skip(f"NVSwitch multicast not available here (exchange fell back to {form})")
    assert form == "fused-" + exchange
    np.testing.assert_array_equal(p0, p1)
    # the same step through the NCCL reference: replicas identical, updates equal to rounding
    for chk in (chk0, chk1):
        assert chk["replicas_identical"]
        assert chk["max_rel_diff_of_update"] <= 1e-3, chk
    nccl = _run("nccl")
    np.testing.assert_array_equal(nccl[0][0], nccl[1][0])
    # separate runs: the backward's atomic order differs, Adam amplifies it (two NCCL runs differ as much)
    np.testing.assert_allclose(p0, nccl[0][0], rtol=2e-3, atol=1e-4)
    assert np.abs(p0).sum() > 0
