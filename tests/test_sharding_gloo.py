"""The sharded step's host logic on CPU, with gloo ranks (no GPU).

Every rank computes the plan through the C ABI (mmn_optim_plan), steps only
what the plan gives it (Muon matrices it owns, its range of the flat AdamW
arena) with the oracle's arithmetic, and the arenas are then all-gathered.
The gathered result must be bitwise identical to one unsharded step: the plan
covers every element exactly once and the arithmetic does not depend on the
partition. The GPU path uses the same plan and kernels whose results do not
depend on which rank runs them."""
import os
import socket

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

ADAMW = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)


def model_params(n_layer=4, d=64, vocab=256):
    """Chatbot-shaped tensors in call order with the tagged routing (block
    matrices to Muon, embed / lm_head / LayerNorm to AdamW)."""
    from magicmindnet_b200.step import chatbot_param_order

    out = []
    for name, shape in chatbot_param_order(vocab, n_layer, d):
        route = "adamw" if (name in ("embed", "lm_head") or len(shape) == 1) else "muon"
        out.append((name, shape, route))
    return out


def make_values(seed, model):
    rng = np.random.default_rng(seed)
    p = [rng.normal(0, 0.02, s).astype(np.float32) for _, s, _ in model]
    g = [rng.normal(0, 1e-3, s).astype(np.float32) for _, s, _ in model]
    return p, g


def step_shard(oracle, model, plan, rank, world, p, g, t_base):
    """One step of this rank's share, on flat arenas laid out by the plan."""
    areg, mreg = plan["adamw_region"], plan["muon_region"]
    a_arena = np.zeros(areg * world, np.float32)
    m_arena = np.zeros(mreg * world, np.float32)
    for k, (_, s, route) in enumerate(model):
        arena = a_arena if route == "adamw" else m_arena
        off = plan["offset"][k]
        arena[off:off + p[k].size] = p[k].reshape(-1)
    lo, hi = rank * areg, (rank + 1) * areg
    t = t_base
    for k, (_, s, route) in enumerate(model):
        if route == "adamw":
            t += 1  # the per-call counter, in call order (lib.rs:41-43)
            off, n = plan["offset"][k], p[k].size
            a, b = max(off, lo), min(off + n, hi)
            if a < b:
                seg = a_arena[a:b].copy()
                m = np.zeros(b - a, np.float32)
                v = np.zeros(b - a, np.float32)
                oracle.adamw_update(seg, m, v, g[k].reshape(-1)[a - off:b - off].copy(), t=t, **ADAMW)
                a_arena[a:b] = seg
        elif plan["owner"][k] == rank:
            mu = oracle.Muon(oracle.MuonConfig(), order=oracle.GEMM_F64)
            w = p[k].copy()
            mu.step_matrix(0, w, g[k])
            off = plan["offset"][k]
            m_arena[off:off + w.size] = w.reshape(-1)
    return a_arena, m_arena


def _worker(rank, world, port, q):
    import sys

    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist

    from oracle import reference_optim as oracle
    from magicmindnet_b200.step import shard_plan

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        model = model_params()
        plan = shard_plan([(k, s, r) for k, (_, s, r) in enumerate(model)], world)
        plans = [None] * world
        dist.all_gather_object(plans, plan)
        assert all(pl == plan for pl in plans), "ranks disagree on the plan"
        p, g = make_values(0, model)
        a_arena, m_arena = step_shard(oracle, model, plan, rank, world, p, g, t_base=0)
        areg, mreg = plan["adamw_region"], plan["muon_region"]
        outs = []
        for arena, reg in ((a_arena, areg), (m_arena, mreg)):
            mine = torch.from_numpy(arena[rank * reg:(rank + 1) * reg].copy())
            parts = [torch.empty(reg, dtype=torch.float32) for _ in range(world)]
            dist.all_gather(parts, mine)
            outs.append(torch.cat(parts).numpy())
        if rank == 0:
            q.put((plan, outs[0], outs[1]))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_sharded_step_equals_unsharded(oracle):
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    plan, a_gathered, m_gathered = q.get(timeout=300)
    for pr in procs:
        pr.join(timeout=120)
        assert pr.exitcode == 0

    # both ranks own some Muon matrices, and every matrix has one owner
    model = model_params()
    owners = [plan["owner"][k] for k, (_, _, r) in enumerate(model) if r == "muon"]
    assert set(owners) == {0, 1}

    # the same step unsharded (world 1) gives the same bits
    from magicmindnet_b200.step import shard_plan

    plan1 = shard_plan([(k, s, r) for k, (_, s, r) in enumerate(model)], 1)
    p, g = make_values(0, model)
    a1, m1 = step_shard(oracle, model, plan1, 0, 1, p, g, t_base=0)
    for k, (_, s, route) in enumerate(model):
        n = int(np.prod(s))
        if route == "adamw":
            got = a_gathered[plan["offset"][k]:plan["offset"][k] + n]
            want = a1[plan1["offset"][k]:plan1["offset"][k] + n]
        else:
            got = m_gathered[plan["offset"][k]:plan["offset"][k] + n]
            want = m1[plan1["offset"][k]:plan1["offset"][k] + n]
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


def test_plan_balances_the_8b_shapes_over_8_ranks():
    """The 5.36e9-parameter GQA shapes (d_model 4096, 32 layers, k/v 1024, FFN
    14336): each of 8 ranks gets the same Newton-Schulz work."""
    import bench
    from magicmindnet_b200.step import shard_plan

    model = bench.WORKLOADS["hybrid_8b"]["model"]()
    plan = shard_plan([(k, s, r) for k, (_, s, r) in enumerate(model)], 8)
    load = [0.0] * 8
    for k, (_, s, r) in enumerate(model):
        if r == "muon":
            n, m = min(s), max(s)
            load[plan["owner"][k]] += 5 * (4.0 * n * n * m + 2.0 * n ** 3)
    assert max(load) / min(load) < 1.01
    assert plan["adamw_region"] * 8 >= sum(int(np.prod(s)) for _, s, r in model if r == "adamw")


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_plan_covers_every_element_once(world):
    from magicmindnet_b200.step import shard_plan

    model = model_params(n_layer=3, d=96, vocab=200)
    plan = shard_plan([(k, s, r) for k, (_, s, r) in enumerate(model)], world)
    a_used = np.zeros(plan["adamw_region"] * world, np.int32)
    m_used = np.zeros(plan["muon_region"] * world, np.int32)
    for k, (_, s, r) in enumerate(model):
        n = int(np.prod(s))
        off = plan["offset"][k]
        if r == "adamw":
            assert plan["owner"][k] == -1
            a_used[off:off + n] += 1
        else:
            o = plan["owner"][k]
            assert 0 <= o < world
            assert o * plan["muon_region"] <= off and off + n <= (o + 1) * plan["muon_region"]
            m_used[off:off + n] += 1
    assert a_used.max() == 1 and m_used.max() == 1
    assert plan["adamw_region"] % 64 == 0
