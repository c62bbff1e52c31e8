"""Several GPUs from one process: b2a_group (one context per device + an NCCL clique)
and the sharded entry points, which compute equal shards on their own devices and
reassemble them with one grouped ncclAllGather.

* One rank (every GPU box): the sharded decode and encoder calls equal the oracle.
* Two ranks (boxes with two GPUs visible): a decode batch is partitioned by
  (sequence, kv head) with b2a_partition_units, each unit passed as a sequence with
  one kv head; the gathered output, permuted back, equals the whole batch's oracle
  result on both devices.
* Bad device lists are NCCL failures (B2A_ENCCL), found by NCCL's argument checks.
"""
import math

import numpy as np
import pytest

import oracle
from helpers import assert_close, normal, to_dev, to_np

pytestmark = pytest.mark.gpu


def _n_gpus():
    import torch
    return torch.cuda.device_count()


def _units_problem(seed):
    """A Qwen-shaped decode batch (14/2 heads, D=64, head-major fp16 cache)."""
    B, Hq, Hkv, D, S = 6, 14, 2, 64, 1500
    lens = np.array([1499, 3, 700, 64, 1024, 17], np.int32)
    q = normal(seed, (B, Hq, D), oracle.F16)
    kn, vn = normal(seed + 1, (B, Hkv, D), oracle.F16), normal(seed + 2, (B, Hkv, D), oracle.F16)
    kc, vc = normal(seed + 3, (B, Hkv, S, D), oracle.F16), normal(seed + 4, (B, Hkv, S, D), oracle.F16)
    scale = float(np.float32(1 / math.sqrt(D)))
    want, kc_w, vc_w = oracle.decode(q, kn, vn, kc, vc, lens, B=B, Hq=Hq, Hkv=Hkv, D=D, max_seq=S, scale=scale,
                                     rope_theta=1e6, rope_mode=oracle.ROPE_DECODERONLY,
                                     cache_layout=oracle.KV_HEAD_MAJOR, cache_dtype=oracle.F16)
    return dict(B=B, Hq=Hq, Hkv=Hkv, D=D, S=S, lens=lens, q=q, kn=kn, vn=vn, kc=kc, vc=vc, scale=scale, want=want)


def _unit_tensors(p, units, device):
    """The units (sequence, kv head) as sequences of one kv head and G q heads on `device`."""
    import torch
    G = p["Hq"] // p["Hkv"]
    b = np.array([u // p["Hkv"] for u in units])
    h = np.array([u % p["Hkv"] for u in units])
    dev = lambda a: to_dev(np.ascontiguousarray(a), oracle.F16).to(device)
    q = dev(np.stack([p["q"][bi, hi * G:(hi + 1) * G] for bi, hi in zip(b, h)]))
    kn = dev(np.stack([p["kn"][bi, hi:hi + 1] for bi, hi in zip(b, h)]))
    vn = dev(np.stack([p["vn"][bi, hi:hi + 1] for bi, hi in zip(b, h)]))
    kc = dev(np.stack([p["kc"][bi, hi:hi + 1] for bi, hi in zip(b, h)]))
    vc = dev(np.stack([p["vc"][bi, hi:hi + 1] for bi, hi in zip(b, h)]))
    lens = torch.from_numpy(p["lens"][b].astype(np.int32)).to(device)
    return q, kn, vn, kc, vc, lens


def _run_sharded_decode(p, devices):
    import torch
    import b200attn
    n = len(devices)
    G, D = p["Hq"] // p["Hkv"], p["D"]
    units = p["B"] * p["Hkv"]
    pad = (-units) % n  # equal shards: pad with copies of unit 0 (their outputs are dropped)
    cost = np.concatenate([(p["lens"].repeat(p["Hkv"]) + 1).astype(np.int64), np.zeros(pad, np.int64)])
    plan = [np.flatnonzero(b200attn.partition_units(cost, n) == r) for r in range(n)]
    per = len(plan[0])
    args = [[] for _ in range(6)]
    o_shard, o_all = [], []
    for r, d in enumerate(devices):
        for i, t in enumerate(_unit_tensors(p, [u if u < units else 0 for u in plan[r]], f"cuda:{d}")):
            args[i].append(t)
        o_shard.append(torch.empty(per, G, D, device=f"cuda:{d}"))
        o_all.append(torch.full((n * per, G, D), float("nan"), device=f"cuda:{d}"))
    with b200attn.Group(devices) as grp:
        assert grp.size() == n
        grp.decode(*args, o_shard, o_all, p["scale"], kv_layout=b200attn.KV_HEAD_MAJOR, rope_mode=b200attn.ROPE_NEOX,
                   rope_theta=1e6)
        grp.check_device_status()
        for d in devices:
            torch.cuda.synchronize(d)
        order = np.concatenate(plan)  # gathered row i holds unit order[i]
        for r, d in enumerate(devices):
            got = to_np(o_all[r])
            full = np.empty((units, G, D), np.float32)
            for i, u in enumerate(order):
                if u < units:
                    full[u] = got[i]
            want = p["want"].reshape(p["B"], p["Hkv"], G, D).reshape(units, G, D)
            assert_close(full, want, what=f"sharded decode gathered on device {d}")


def test_group_one_rank_sharded_decode_and_encoder(ctx):
    import torch
    import b200attn
    _run_sharded_decode(_units_problem(1200), [0])
    # encoder: MiniLM-shaped shard through the sharded mha, one rank
    B, H, S, D = 4, 3, 96, 32
    lens = np.array([96, 5, 40, 0], np.int32)
    q, k, v = (normal(1300 + i, (B, S, H, D), oracle.F16) for i in range(3))
    want = oracle.encoder_minilm(q, k, v, lens, B=B, H=H, S=S, D=D, layout=1)
    y = torch.empty((B, S, H, D), device="cuda")
    yall = torch.full((B, S, H, D), float("nan"), device="cuda")
    with b200attn.Group([0]) as grp:
        grp.mha([to_dev(q, oracle.F16)], [to_dev(k, oracle.F16)], [to_dev(v, oracle.F16)], [y], [yall],
                1 / math.sqrt(D), key_lengths=[torch.from_numpy(lens).cuda()], layout=b200attn.SEQ_MAJOR)
        grp.check_device_status()
    torch.cuda.synchronize()
    assert_close(to_np(yall), want, what="sharded encoder, one rank")


@pytest.mark.skipif("_n_gpus() < 2")
def test_group_two_ranks_partition_by_sequence_and_kv_head(ctx):
    _run_sharded_decode(_units_problem(1400), [0, 1])


def test_group_with_a_device_nccl_rejects_is_b2a_enccl(ctx):
    import b200attn
    with pytest.raises(b200attn.B200RuntimeException) as ei:
        b200attn.Group([0, 4096])
    assert ei.value.status == b200attn.B2A_ENCCL
