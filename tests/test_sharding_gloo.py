"""The N > 1 host path on CPU: two gloo ranks shard one decode batch with
b200attn.sharding.plan_shards, compute their shards (here with the oracle: no GPU on the
CPU suite), reassemble with gather_shards and time with max_over_ranks; the result must
equal the single-process computation of the whole batch."""
import os
import socket

import numpy as np
import pytest

import oracle


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem():
    B, Hq, Hkv, D, max_seq = 8, 4, 2, 32, 96
    lens = oracle.splitmix_uniform_int(71, B, 1, max_seq - 1)
    q = oracle.splitmix_normal(72, B * Hq * D).reshape(B, Hq, D)
    kc = oracle.splitmix_normal(73, B * Hkv * max_seq * D).reshape(B, Hkv, max_seq, D)
    vc = oracle.splitmix_normal(74, B * Hkv * max_seq * D).reshape(B, Hkv, max_seq, D)
    return dict(B=B, Hq=Hq, Hkv=Hkv, D=D, max_seq=max_seq, lens=lens, q=q, kc=kc, vc=vc)


def _attend(p, idx):
    return oracle.attend_cache(p["q"][idx], p["kc"][idx], p["vc"][idx], p["lens"][idx], B=len(idx), Hq=p["Hq"],
                               Hkv=p["Hkv"], D=p["D"], max_seq=p["max_seq"], scale=float(1 / np.sqrt(p["D"])),
                               n_threads=1)


def _rank_main(rank, world, port, result_q):
    import torch
    import torch.distributed as dist
    from b200attn import sharding
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        p = _problem()
        plan = sharding.plan_shards(p["lens"].astype(np.int64) + 1, world)
        local = torch.from_numpy(_attend(p, plan[rank]))
        full = sharding.gather_shards(local, plan)
        slowest = sharding.max_over_ranks([1.0 + rank, 10.0 - rank])
        result_q.put((rank, [x.tolist() for x in plan], full.numpy(), slowest))
    finally:
        dist.destroy_process_group()


def test_plan_shards_is_balanced_and_covers_every_unit():
    from b200attn import sharding
    cost = np.array([9, 1, 8, 2, 7, 3, 6, 4], np.int64)
    plan = sharding.plan_shards(cost, 2)
    assert sorted(np.concatenate(plan).tolist()) == list(range(8))
    assert [len(p) for p in plan] == [4, 4]
    loads = [int(cost[p].sum()) for p in plan]
    assert max(loads) - min(loads) <= 2  # LPT on 9..1: 20 / 20
    with pytest.raises(ValueError):
        sharding.plan_shards(np.ones(7, np.int64), 2)


def test_max_over_ranks_without_a_process_group_is_the_identity():
    from b200attn import sharding
    assert sharding.max_over_ranks([3.5, 1.25]) == [3.5, 1.25]


def test_two_gloo_ranks_reassemble_the_single_process_result():
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    p = _problem()
    want = _attend(p, np.arange(p["B"]))
    plans = {r: plan for r, plan, _, _ in results}
    assert plans[0] == plans[1]  # both ranks derive the same plan from the same costs
    for rank, _, full, slowest in results:
        np.testing.assert_array_equal(full, want)  # per-sequence work is independent: bit-exact
        assert slowest == [2.0, 10.0]


def _bad_count_rank(rank, claimed_world, port, result_q):
    """A rank that joins a group whose declared size is larger than the ranks that exist."""
    from datetime import timedelta
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=claimed_world, timeout=timedelta(seconds=4))
        result_q.put((rank, "joined"))
        dist.destroy_process_group()
    except Exception as e:  # the rendezvous gives up: the failure surfaces on the host as an exception
        result_q.put((rank, type(e).__name__))


def test_group_init_with_a_bad_rank_count_fails_on_the_host_within_its_timeout():
    """Failure detection on the host: two processes start a group that declares three ranks.  The
    rendezvous never completes, and each rank gets an exception within the group's timeout instead of
    hanging (the same holds for NCCL, whose init goes through the same rendezvous)."""
    import time
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_bad_count_rank, args=(r, 3, port, q)) for r in range(2)]
    t0 = time.time()
    for pr in procs:
        pr.start()
    results = dict(q.get(timeout=120) for _ in range(2))
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    assert set(results) == {0, 1}
    assert all(v != "joined" for v in results.values()), results
    assert time.time() - t0 < 110
