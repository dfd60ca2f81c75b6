"""The sharded step on several GPUs: each rank steps what the plan gives it
(whole Muon matrices by LPT, one range of the AdamW arena), the arenas are
all-gathered over NCCL, and every parameter must equal the single-GPU step
bit for bit. Needs two or more GPUs; skipped otherwise."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _model():
    import bench

    # a 4-layer slice of the 1.2B shapes keeps the test small
    m = bench.hybrid_model(2048, 4, 8192, 4096)
    return [(k, s, r) for k, (_, s, r) in enumerate(m)]


def _fill(step, model, seed):
    import torch

    gen = torch.Generator(device="cuda").manual_seed(seed)
    for k, (_, s, _) in enumerate(model):
        step.param(k).normal_(0, 0.02, generator=gen)
        step.grad(k).normal_(0, 1e-3, generator=gen)


def _host_grads(model, it):
    rng = np.random.default_rng(100 + it)
    return [rng.standard_normal(s, dtype=np.float32) * np.float32(1e-3) for _, s, _ in model]


def _host_worker(rank, world, step, model, mmn, q):
    """Each rank steps its shard from host grads and writes back only what it
    stepped; the single-GPU step from the same host grads (run here, on this
    rank's GPU) must agree on every element written, and the device arenas,
    completed by the exchange, must agree everywhere."""
    import torch

    single = mmn.OptimizerStep(model, mmn.StepConfig(use_graph=False), device=rank,
                               stream=torch.cuda.current_stream(rank).cuda_stream)
    _fill(single, model, 0)
    step.connect_peers()
    written = 0
    for it in range(2):
        grads = _host_grads(model, it)
        outs = [np.full(s, np.nan, np.float32) for _, s, _ in model]
        step.step_host(grads, outs)
        step.exchange_fence()
        want = [np.empty(s, np.float32) for _, s, _ in model]
        single.step_host(grads, want)
        for k in range(len(model)):
            hit = ~np.isnan(outs[k])
            np.testing.assert_array_equal(outs[k][hit].view(np.uint32), want[k][hit].view(np.uint32),
                                          err_msg=f"rank {rank} step {it} slot {k}")
            if it == 1:
                written += int(hit.sum())
    step.sync()
    torch.cuda.synchronize()
    for k in range(len(model)):
        np.testing.assert_array_equal(step.param(k).cpu().numpy().view(np.uint32),
                                      want[k].view(np.uint32), err_msg=f"rank {rank} arena slot {k}")
    single.close()
    q.put((rank, written))


def _worker(rank, world, port, q, exchange):
    import sys

    sys.path.insert(0, ROOT)
    import datetime

    import torch
    import torch.distributed as dist

    import magicmindnet_b200 as mmn
    from magicmindnet_b200.step import _view

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device(f"cuda:{rank}"))
    try:
        model = _model()
        cfg = mmn.StepConfig(rank=rank, world_size=world, use_graph=False)
        step = mmn.OptimizerStep(model, cfg, device=rank,
                                 stream=torch.cuda.current_stream(rank).cuda_stream)
        _fill(step, model, 0)
        if exchange == "host":
            try:
                _host_worker(rank, world, step, model, mmn, q)
            except Exception as e:  # reported to the parent, which fails at once
                q.put((rank, f"{type(e).__name__}: {e}"))
                raise
            step.close()
            return
        if exchange == "fused":
            step.connect_peers()
        for _ in range(2):
            step.step()
            if exchange == "fused":
                step.exchange_fence()
                continue
            gl = step.gather_layout()
            for key, reg in (("adamw_param", "adamw_region"), ("muon_param", "muon_region")):
                full = _view(gl[key], (gl[reg] * world,), "f32", rank)
                dist.all_gather_into_tensor(full, full[rank * gl[reg]:(rank + 1) * gl[reg]].clone())
        step.sync()
        torch.cuda.synchronize()
        out = [step.param(k).cpu().numpy().copy() for k in range(len(model))]
        if rank == 0:
            q.put(out)
        step.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["nccl", "fused", "host"])
def test_sharded_step_equals_single_gpu(mmn, exchange):
    import torch
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs two or more GPUs")
    model = _model()
    if exchange == "host":
        _run_host(model, world)
        return
    single = mmn.OptimizerStep(model, mmn.StepConfig(use_graph=False), device=0)
    _fill(single, model, 0)
    single.step()
    single.step()
    single.sync()
    want = [single.param(k).cpu().numpy().copy() for k in range(len(model))]
    single.close()

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, exchange)) for r in range(world)]
    for p in procs:
        p.start()
    got = q.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for k, (a, b) in enumerate(zip(got, want)):
        np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32), err_msg=str(k))


def _spawn(world, exchange):
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, exchange)) for r in range(world)]
    for p in procs:
        p.start()
    return procs, q


def _run_host(model, world):
    procs, q = _spawn(world, "host")
    got = dict(q.get(timeout=900) for _ in range(world))
    bad = {r: v for r, v in got.items() if not isinstance(v, int)}
    assert not bad, bad
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    # every element was written back by exactly one rank (outputs are NaN-filled)
    assert sum(got.values()) == sum(int(np.prod(s)) for _, s, _ in model)
