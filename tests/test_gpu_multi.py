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
        # "<exchange>-<ns mode>" runs the sharded step in that Newton-Schulz mode
        exchange, _, mode = exchange.partition("-")
        cfg = mmn.StepConfig(rank=rank, world_size=world, use_graph=False,
                             ns_mode=mode or "reference")
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


@pytest.mark.parametrize("exchange", ["nccl", "fused", "host", "fused-tf32", "fused-fp32"])
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
    mode = exchange.partition("-")[2] or "reference"
    single = mmn.OptimizerStep(model, mmn.StepConfig(use_graph=False, ns_mode=mode), device=0)
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


# ------------------------------------------------------------------ grad reduction
def _local_grads(model, world, bf16):
    """Every rank's local grads (rank r from seed 500 + r), generated alike on
    every process, and their rank-ordered fp32 sum (rounded to bf16 once)."""
    import torch

    per_rank = []
    for r in range(world):
        gen = torch.Generator(device="cuda").manual_seed(500 + r)
        gs = []
        for _, s, _ in model:
            g = torch.empty(s, device="cuda").normal_(0, 1e-3, generator=gen)
            gs.append((g * 1024.0).bfloat16() if bf16 else g)
        per_rank.append(gs)
    sums = []
    for k in range(len(model)):
        acc = per_rank[0][k].float()
        for r in range(1, world):
            acc = acc + per_rank[r][k].float()
        sums.append(acc.bfloat16() if bf16 else acc)
    return per_rank, sums


def _host_values(t):
    """float32 host values of a device grad (bf16 widened exactly)."""
    import torch

    if t.dtype == torch.bfloat16:
        from oracle import reference_optim as R

        return R.bf16_from_bits(t.view(torch.int16).cpu().numpy())
    return t.cpu().numpy()


def _check_reduced_against_oracle(step, model, world, rank, per_rank, bf16):
    """The parts this rank steps (its Muon matrices, its range of the AdamW
    arena) must hold the oracle's rank-ordered sum of every rank's local grads,
    bit for bit. Returns the number of elements compared."""
    import torch

    import magicmindnet_b200 as mmn
    from oracle import reference_optim as R

    plan = mmn.shard_plan(model, world)
    lo, hi = rank * plan["adamw_region"], (rank + 1) * plan["adamw_region"]
    torch.cuda.synchronize()
    checked = 0
    for k, (_, s, _) in enumerate(model):
        n = int(np.prod(s))
        if plan["owner"][k] == rank:
            a, b = 0, n
        elif plan["owner"][k] == -1:
            a = min(max(lo - plan["offset"][k], 0), n)
            b = min(max(hi - plan["offset"][k], 0), n)
        else:
            continue
        if a == b:
            continue
        got = _host_values(step.grad(k).reshape(-1)[a:b])
        want = R.grad_allreduce([_host_values(g.reshape(-1)[a:b]) for g in
                                 (per_rank[r][k] for r in range(world))], bf16)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32),
                                      err_msg=f"rank {rank} slot {k} [{a}:{b}]")
        checked += b - a
    return checked


def _reduce_cfg(mmn, bf16, **kw):
    if bf16:
        return mmn.StepConfig(grad_dtype="bf16", loss_scaling=True, loss_scale_init=1024.0,
                              use_graph=False, **kw)
    return mmn.StepConfig(use_graph=False, **kw)


def _reduce_worker(rank, world, port, q, bf16):
    import sys

    sys.path.insert(0, ROOT)
    import datetime

    import torch
    import torch.distributed as dist

    import magicmindnet_b200 as mmn

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device(f"cuda:{rank}"))
    try:
        model = _model()
        step = mmn.OptimizerStep(model, _reduce_cfg(mmn, bf16, rank=rank, world_size=world,
                                                    reduce_grads=True),
                                 device=rank, stream=torch.cuda.current_stream(rank).cuda_stream)
        _fill(step, model, 0)
        per_rank, _ = _local_grads(model, world, bf16)
        for k in range(len(model)):
            step.grad(k).copy_(per_rank[rank][k])
        step.connect_peers()
        step.reduce_grads()
        checked = _check_reduced_against_oracle(step, model, world, rank, per_rank, bf16)
        step.step()
        step.exchange_fence()
        out = [step.param(k).cpu().numpy().copy() for k in range(len(model))]
        skipped = None
        if bf16:
            # a +inf in the last rank's local grad of a matrix rank 0 owns: the
            # sum there is +inf, so every rank skips the next step
            plan = mmn.shard_plan(model, world)
            k0 = next(k for k, o in enumerate(plan["owner"]) if o == 0)
            for k in range(len(model)):
                step.grad(k).copy_(per_rank[rank][k])
            if rank == world - 1:
                step.grad(k0).view(-1)[7] = float("inf")
            before = [step.param(k).clone() for k in range(len(model))]
            step.reduce_grads()
            step.step()
            step.exchange_fence()
            torch.cuda.synchronize()
            same = all(torch.equal(step.param(k), before[k]) for k in range(len(model)))
            skipped = (same, step.loss_scale())
        step.sync()
        q.put((rank, out, (skipped, checked)))
        step.close()
    except Exception as e:  # reported to the parent, which fails at once
        q.put((rank, f"{type(e).__name__}: {e}", None))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("bf16", [False, True])
def test_reduced_grads_step_equals_single_gpu_on_summed_grads(mmn, bf16):
    """Data parallelism end to end: each rank holds its own local grads, the
    fused reduction sums them over NVLink in rank order, each rank steps its
    shard and pushes it to the peers. Every rank's parameters must equal, bit
    for bit, one GPU stepping the rank-ordered sum of the grads. With bf16 grads
    and loss scaling, a +inf in one rank's local grads skips the step on every
    rank and halves every rank's scale. Before the step, each rank's reduced
    parts are compared with the oracle's rank-ordered sum (grad_allreduce) bit
    for bit."""
    import torch
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs two or more GPUs")
    model = _model()
    single = mmn.OptimizerStep(model, _reduce_cfg(mmn, bf16), device=0)
    _fill(single, model, 0)
    _, sums = _local_grads(model, world, bf16)
    for k in range(len(model)):
        single.grad(k).copy_(sums[k])
    single.step()
    single.sync()
    want = [single.param(k).cpu().numpy().copy() for k in range(len(model))]
    scale0 = single.loss_scale()[0]
    single.close()
    del sums

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_reduce_worker, args=(r, world, port, q, bf16))
             for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        r, out, skipped = q.get(timeout=900)
        got[r] = (out, skipped)
    for p in procs:
        p.join(timeout=120)
    checked = 0
    for r, (out, extra) in got.items():
        assert not isinstance(out, str), (r, out)
        skipped, n = extra
        checked += n
        for k, (a, b) in enumerate(zip(out, want)):
            np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32),
                                          err_msg=f"rank {r} slot {k}")
        if bf16:
            same, (scale, nskip) = skipped
            assert same, r
            assert (scale, nskip) == (scale0 / 2, 1), r
    # the ranks' reduced parts, each equal to the oracle's sum, cover every grad
    assert checked == sum(int(np.prod(s)) for _, s, _ in model)
    for p in procs:
        assert p.exitcode == 0


# ------------------------------------------------------------------ checkpoints
def _ckpt_worker(rank, world, port, q, path):
    import sys

    sys.path.insert(0, ROOT)
    import datetime

    import torch
    import torch.distributed as dist

    import magicmindnet_b200 as mmn

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device(f"cuda:{rank}"))
    try:
        model = _model()
        names = [f"t{k}" for k in range(len(model))]
        stream = torch.cuda.current_stream(rank).cuda_stream

        def make():
            s = mmn.OptimizerStep(model, mmn.StepConfig(rank=rank, world_size=world,
                                                        use_graph=False),
                                  device=rank, stream=stream)
            s.connect_peers()
            return s

        def grads(step, seed):
            gen = torch.Generator(device="cuda").manual_seed(seed)
            for k, (_, s, _) in enumerate(model):
                step.grad(k).normal_(0, 1e-3, generator=gen)

        a = make()
        _fill(a, model, 0)
        for it in range(2):
            grads(a, 10 + it)
            a.step()
            a.exchange_fence()
        a.sync()
        mmn.save_state(a, f"{path}.{rank}", names)
        b = make()
        for k in range(len(model)):
            b.param(k).copy_(a.param(k))
        mmn.load_state(b, f"{path}.{rank}", names)
        for it in range(2):
            for s in (a, b):
                grads(s, 20 + it)
                s.step()
                s.exchange_fence()
        a.sync()
        b.sync()
        torch.cuda.synchronize()
        bad = [k for k in range(len(model)) if not torch.equal(a.param(k), b.param(k))]
        for k in range(len(model)):
            lo, hi = a.stepped_range(k)
            if hi <= lo:
                continue
            which = ("m", "v") if a.routes[k] == "adamw" else ("velocity",)
            for w in which:
                sa = a.get_state(k, w).reshape(-1)[lo:hi]
                sb = b.get_state(k, w).reshape(-1)[lo:hi]
                if not np.array_equal(sa.view(np.uint32), sb.view(np.uint32)):
                    bad.append((k, w))
        q.put((rank, bad))
        a.close()
        b.close()
    except Exception as e:  # reported to the parent, which fails at once
        q.put((rank, f"{type(e).__name__}: {e}"))
        raise
    finally:
        dist.destroy_process_group()


def test_sharded_checkpoint_resume_is_bit_exact(tmp_path):
    """Each rank saves what it steps (its Muon matrices, its AdamW slices) and a
    fresh sharded handle resumes from it: the next steps match bit for bit."""
    import torch
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs two or more GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    path = str(tmp_path / "optim.safetensors")
    procs = [ctx.Process(target=_ckpt_worker, args=(r, world, port, q, path))
             for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=900) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
    for r, bad in got.items():
        assert bad == [], (r, bad)
    for p in procs:
        assert p.exitcode == 0


# ------------------------------------------------------------------ sharded scan
def _scan_grads_for(model, it, bad_slot=None):
    """Replicated bf16 grads of step `it` (seed 700 + it), with a +inf in
    bad_slot when given."""
    import torch

    gen = torch.Generator(device="cuda").manual_seed(700 + it)
    gs = [(torch.empty(s, device="cuda").normal_(0, 1e-3, generator=gen) * 1024.0).bfloat16()
          for _, s, _ in model]
    if bad_slot is not None:
        gs[bad_slot].view(-1)[3] = float("inf")
    return gs


def _scan_worker(rank, world, port, q, bad_slot):
    import sys

    sys.path.insert(0, ROOT)
    import datetime

    import torch
    import torch.distributed as dist

    import magicmindnet_b200 as mmn

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device(f"cuda:{rank}"))
    try:
        model = _model()
        step = mmn.OptimizerStep(model, _reduce_cfg(mmn, True, rank=rank, world_size=world,
                                                    scan_shard=True),
                                 device=rank, stream=torch.cuda.current_stream(rank).cuda_stream)
        _fill(step, model, 0)
        step.connect_peers()
        for it in range(3):  # step 1 has a +inf in a slot another rank steps
            gs = _scan_grads_for(model, it, bad_slot if it == 1 else None)
            if it < 2:
                for k in range(len(model)):
                    step.grad(k).copy_(gs[k])
                step.scan_grads()
                step.step()
            else:  # from host memory: this rank's grads in through scan_grads
                host = [g.cpu() for g in gs]
                outs = [np.empty(s, np.float32) for _, s, _ in model]
                step.scan_grads(host)
                step.step_host([None] * len(model), outs)
            step.exchange_fence()
        step.sync()
        torch.cuda.synchronize()
        out = [step.param(k).cpu().numpy().copy() for k in range(len(model))]
        q.put((rank, out, step.loss_scale()))
        step.close()
    except Exception as e:  # reported to the parent, which fails at once
        q.put((rank, f"{type(e).__name__}: {e}", None))
        raise
    finally:
        dist.destroy_process_group()


def test_sharded_nonfinite_scan_equals_single_gpu(mmn):
    """Loss-scaled sharded step with the sharded scan (scan_shard): each rank
    scans only what it steps and sets every rank's flag. A +inf in a slot the
    last rank steps skips step 1 on every rank and halves every scale; the
    three steps (the last from host memory) equal one GPU bit for bit."""
    import torch
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs two or more GPUs")
    model = _model()
    plan = mmn.shard_plan(model, world)
    bad_slot = next(k for k, o in enumerate(plan["owner"]) if o == world - 1)
    single = mmn.OptimizerStep(model, _reduce_cfg(mmn, True), device=0)
    _fill(single, model, 0)
    for it in range(3):
        gs = _scan_grads_for(model, it, bad_slot if it == 1 else None)
        for k in range(len(model)):
            single.grad(k).copy_(gs[k])
        single.step()
    single.sync()
    want = [single.param(k).cpu().numpy().copy() for k in range(len(model))]
    scale = single.loss_scale()
    single.close()
    assert scale[1] == 1  # the single-GPU run skipped step 1 too

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_scan_worker, args=(r, world, port, q, bad_slot))
             for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        r, out, sc = q.get(timeout=900)
        got[r] = (out, sc)
    for p in procs:
        p.join(timeout=120)
    for r, (out, sc) in got.items():
        assert not isinstance(out, str), (r, out)
        assert sc == scale, (r, sc, scale)
        for k, (a, b) in enumerate(zip(out, want)):
            np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32),
                                          err_msg=f"rank {r} slot {k}")
    for p in procs:
        assert p.exitcode == 0


@pytest.mark.gpu
@pytest.mark.parametrize("handoff", ["reduce_grads", "scan_shard"])
def test_step_needs_the_grad_handoff_first(mmn, handoff):
    """A reduce_grads (scan_shard) handle refuses a step whose grads did not
    go through reduce_grads (scan_grads) since the last step, before anything
    is enqueued: otherwise it would step this rank's unreduced grads, or
    without any rank's non-finite verdict. One GPU: a rank of two whose peers
    are never connected, so the hand-off itself is refused too."""
    model = [(0, (64, 64), "muon"), (1, (64,), "adamw")]
    cfg = _reduce_cfg(mmn, True, rank=0, world_size=2, **{handoff: True})
    step = mmn.OptimizerStep(model, cfg, device=0)
    try:
        calls = [lambda: step.step()]
        if handoff == "scan_shard":  # (a reduce_grads handle takes no host-memory step)
            calls.append(lambda: step.step_host([None, None], [None, None]))
        for call in calls:
            with pytest.raises(mmn.MmnError) as e:
                call()
            assert e.value.code == -5  # MMN_E_STATE
            assert ("reduce_grads" if handoff == "reduce_grads" else "scan_grads") in str(e.value)
        from magicmindnet_b200 import _native as N

        with pytest.raises(mmn.MmnError, match="connect the peers first"):
            if handoff == "reduce_grads":
                N.check(N.lib().mmn_optim_reduce_grads(step._h))
            else:
                N.check(N.lib().mmn_optim_scan_grads(step._h, None))
        step.sync()
    finally:
        step.close()
