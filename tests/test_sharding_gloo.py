"""Layer-sharded host logic on CPU ranks over gloo (the N>1 path without a GPU).

Each rank scores its block of layer 0's heads with the oracle's column sums, the
per-head scores are all-gathered through ``sharding.gather_head_scores``, and
every rank must end with the single-process per-head scores bit for bit and the
same keep set; the per-layer size all-gather must give every rank the same
global layer table.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from nexusquant_b200 import sharding as S  # noqa: E402

B, H, T, D, L, PB, SW, RATE = 1, 5, 300, 64, 7, 1, 16, 0.6


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _keys():
    rng = np.random.default_rng(11)
    return rng.standard_normal((B, H, T, D)).astype(np.float32)


def _per_head(K, h0, h1):
    from oracle import oracle as orc
    obs = min(32, T)
    scale = float(np.float32(D ** -0.5))
    out = np.zeros((B, h1 - h0, T), np.float32)
    for bi in range(B):
        for hi in range(h0, h1):
            out[bi, hi - h0] = orc.attn_colsum(K[bi, hi, T - obs:], K[bi, hi], scale).astype(np.float32)
    return out


def _worker(rank, world, port, q, mode="layers"):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from oracle import oracle as orc
        plan = S.make_plan(L, H, PB, rank, world, mode=mode)
        K = _keys()
        ph = torch.from_numpy(_per_head(K, plan.head_begin, plan.head_end))
        allh = S.gather_head_scores(ph, plan)
        full = _per_head(K, 0, H)
        assert allh.shape == (B, H, T)
        assert np.array_equal(allh.numpy(), full), "gathered per-head scores differ from single-process"
        imp = allh.double().sum(1).numpy() / H
        mask = orc.keep_mask(imp, T, SW, RATE)
        masks = [torch.zeros(B * T, dtype=torch.uint8) for _ in range(world)]
        dist.all_gather(masks, torch.from_numpy(mask.astype(np.uint8).reshape(-1)))
        for m in masks:
            assert torch.equal(m, masks[0]), "keep sets differ across ranks"
        # per-layer size table
        comp = [1000 + 7 * l for l in plan.quantized]
        prot = [50000 + l for l in plan.protected]
        sizes = S.local_layer_sizes(plan, comp, prot)
        sizes_all = S.gather_layer_index(sizes, plan)
        table_async, work = S.gather_layer_index(sizes, plan, async_op=True)
        if work is not None:
            work.wait()
        assert torch.equal(table_async, sizes_all)
        prot_set = S.protected_layers(L, PB)
        if mode == "layers":
            owners = S.layer_owners(S.assign_layers(L, prot_set, world), L)
            table = S.layer_table(sizes_all, owners)
            off = 0
            for l, (r, o, n) in enumerate(table):
                assert o == off and n == (50000 + l if l in prot_set else 1000 + 7 * l)
                assert l in S.make_plan(L, H, PB, r, world).layers
                off += n
        else:
            # every rank holds its head slice of every layer: world blocks per layer
            assert plan.layers == tuple(range(L)) and plan.layer_heads == (plan.head_begin, plan.head_end)
            units = S.unit_table(sizes_all)
            assert [(l, r) for l, r, _, _ in units] == [(l, r) for l in range(L) for r in range(world)]
            off = 0
            for l, r, o, n in units:
                assert o == off and n == (50000 + l if l in prot_set else 1000 + 7 * l)
                off += n
        q.put((rank, "ok", mask.sum()))
        dist.destroy_process_group()
    except Exception as e:  # report to the parent, which fails the test
        q.put((rank, f"{type(e).__name__}: {e}", None))
        raise


@pytest.mark.parametrize("world,mode", [(2, "layers"), (3, "layers"), (5, "heads")])
def test_sharded_keep_set_and_index_gloo(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    assert all(st == "ok" for _, st, _ in res), res
    assert len({int(n) for _, _, n in res}) == 1


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_assign_layers_config4(world):
    prot = S.protected_layers(80, 2)
    assert prot == {0, 1, 78, 79}
    asg = S.assign_layers(80, prot, world)
    owners = S.layer_owners(asg, 80)  # every layer exactly once
    assert len(owners) == 80
    nq = [sum(1 for l in a if l not in prot) for a in asg]
    assert max(nq) == -(-76 // world)  # compressed layers as even as possible
    assert sum(len(a) for a in asg) == 80
    assert asg == S.assign_layers(80, prot, world)  # deterministic


@pytest.mark.parametrize("heads,world", [(8, 1), (8, 2), (8, 3), (8, 8), (5, 2), (2, 4)])
def test_head_blocks_cover_heads(heads, world):
    seen = []
    for r in range(world):
        h0, h1, per = S.head_block(heads, r, world)
        assert 0 <= h0 <= h1 <= heads and h1 - h0 <= per
        seen += list(range(h0, h1))
    assert seen == list(range(heads))


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_head_plan_config4_is_even(world):
    """Config 4 (80 layers, 8 KV heads) under mode="heads": every rank compresses 8/world heads
    of all 76 quantized layers and gathers the same slice of the 4 protected ones."""
    plans = [S.make_plan(80, 8, 2, r, world, mode="heads") for r in range(world)]
    assert all(p.mode == "heads" for p in plans)
    assert [p.layer_heads for p in plans] == [(r * 8 // world, (r + 1) * 8 // world) for r in range(world)]
    assert all(len(p.quantized) == 76 and len(p.protected) == 4 for p in plans)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_auto_plan_config4_keeps_whole_layers(world):
    """mode="auto" on config 4: 8 KV heads split over 2-8 ranks would leave fewer than
    MIN_HEADS_PER_RANK per rank, so ranks own whole layers; the scored head blocks still
    cover every head once and the quantized layers are as even as whole layers allow."""
    plans = [S.make_plan(80, 8, 2, r, world) for r in range(world)]
    assert all(p.mode == "layers" and p.layer_heads == (0, 8) for p in plans)
    assert sorted(l for p in plans for l in p.layers) == list(range(80))
    assert max(len(p.quantized) for p in plans) == -(-76 // world)
    assert [h for p in plans for h in range(p.head_begin, p.head_end)] == list(range(8))


def test_auto_plan_heads_when_every_rank_keeps_enough():
    assert S.make_plan(32, 32, 2, 0, 4).mode == "heads"   # 8 heads per rank
    assert S.make_plan(32, 32, 2, 0, 8).mode == "layers"  # 4 heads per rank
    assert S.make_plan(80, 8, 2, 0, 1).mode == "heads"    # one rank: the whole cache


def test_plan_modes():
    assert S.make_plan(80, 8, 2, 0, 3).mode == "layers"  # 3 does not divide 8
    with pytest.raises(ValueError):
        S.make_plan(80, 8, 2, 0, 3, mode="heads")


def test_plan_rejects_bad_rank():
    with pytest.raises(ValueError):
        S.make_plan(4, 8, 0, 2, 2)
    with pytest.raises(ValueError):
        S.layer_owners([[0, 1], [1]], 3)
