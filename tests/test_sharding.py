"""Multi-rank logic on CPU (gloo, world size 2): value-head sharding.

The path shards by value head with no collective in the data path
(gdn_recoverssm_b200.sharding).  These tests check that the head split
partitions key and value heads consistently with the GQA mapping, that a
sharded verify + commit (each rank its heads of one common problem, run with
the CPU executors) reassembles to the unsharded result, and that the
benchmark's only collective -- the MAX of per-rank timings -- behaves.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gdn_recoverssm_b200 import synthetic
from gdn_recoverssm_b200.sharding import head_shard, max_over_ranks
from oracle import cpu_executors as X


@pytest.mark.parametrize("cfg", sorted(synthetic.CONFIGS))
@pytest.mark.parametrize("world", [1, 2, 4])
def test_head_shard_partitions_heads_and_keeps_gqa_pairs(cfg, world):
    s = synthetic.CONFIGS[cfg]
    H, HV = s["H"], s["HV"]
    if H % world:
        with pytest.raises(ValueError):
            head_shard(H, HV, world, 0)
        return
    shards = [head_shard(H, HV, world, r) for r in range(world)]
    assert all(x.value_heads == HV // world and x.key_heads == H // world for x in shards)
    assert shards[0].key_begin == 0 and shards[-1].key_end == H
    assert shards[0].value_begin == 0 and shards[-1].value_end == HV
    for a, b in zip(shards, shards[1:]):
        assert a.key_end == b.key_begin and a.value_end == b.value_begin
    ratio = HV // H
    for x in shards:
        for hv in range(x.value_begin, x.value_end):
            assert x.key_begin <= hv // ratio < x.key_end


def test_head_shard_rejects_bad_splits():
    with pytest.raises(ValueError):
        head_shard(16, 32, 3, 0)
    with pytest.raises(ValueError):
        head_shard(16, 24, 1, 0)
    with pytest.raises(ValueError):
        head_shard(16, 32, 2, 2)


def _problem(seed=0, B=6, H=2, HV=4, D=16, Q=3):
    gen = torch.Generator().manual_seed(seed)
    T = B * Q
    unit = lambda x: x / x.norm(dim=-1, keepdim=True)  # noqa: E731
    q = unit(torch.randn(T, H, D, generator=gen))
    k = unit(torch.randn(T, H, D, generator=gen))
    v = torch.randn(T, HV, D, generator=gen)
    g = -torch.nn.functional.softplus(torch.randn(T, HV, generator=gen))
    beta = torch.sigmoid(torch.randn(T, HV, generator=gen))
    state = torch.randn(2 * B + 1, HV, D, D, generator=gen) * 0.1
    src = torch.arange(1, B + 1, dtype=torch.int32)
    fin = torch.arange(B + 1, 2 * B + 1, dtype=torch.int32)
    qsl = torch.arange(B + 1, dtype=torch.int32) * Q
    acc = torch.randint(1, Q + 1, (B,), generator=gen, dtype=torch.int32)
    return dict(q=q, k=k, v=v, g=g, beta=beta, state=state, src=src, fin=fin, qsl=qsl, acc=acc, Q=Q, D=D)


def _run(p, k0, k1, v0, v1):
    """Verify + fold of heads [v0, v1) (keys [k0, k1)) with the CPU executors."""
    B, Q, D = p["src"].shape[0], p["Q"], p["D"]
    q, k = p["q"][:, k0:k1].contiguous(), p["k"][:, k0:k1].contiguous()
    v, g, beta = (p[n][:, v0:v1].contiguous() for n in ("v", "g", "beta"))
    state = p["state"][:, v0:v1].clone()
    HV = v1 - v0
    records = torch.zeros(B, HV, Q, 2 * D + 1)
    out = torch.zeros(q.shape[0], HV, D)
    zeros = torch.zeros(B, dtype=torch.int32)
    X.verify_packed(q, k, v, g, beta, state, p["qsl"], p["src"], records, out, spec_query_len=Q, scale=D**-0.5)
    X.fold_packed(state, records, p["src"], p["acc"], p["fin"], zeros, zeros, rows=B)
    return out, records, state


def _rank_main(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.set_num_threads(1)
        p = _problem()
        H, HV = p["q"].shape[1], p["v"].shape[1]
        sh = head_shard(H, HV, world, rank)
        out, records, state = _run(p, sh.key_begin, sh.key_end, sh.value_begin, sh.value_end)
        # reassemble on every rank (test only: the path itself never communicates)
        outs = [torch.empty_like(out) for _ in range(world)]
        recs = [torch.empty_like(records) for _ in range(world)]
        states = [torch.empty_like(state) for _ in range(world)]
        dist.all_gather(outs, out)
        dist.all_gather(recs, records)
        dist.all_gather(states, state)
        times = max_over_ranks([float(rank + 1), 10.0 - rank])
        if rank == 0:
            result_q.put((torch.cat(outs, 1), torch.cat(recs, 1), torch.cat(states, 1), times))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_gloo_world2_sharded_path_reassembles_to_unsharded():
    world = 2
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, result_q)) for r in range(world)]
    for pr in procs:
        pr.start()
    try:
        got = result_q.get(timeout=120)
    finally:
        for pr in procs:
            pr.join(timeout=120)
            if pr.is_alive():
                pr.kill()
    for pr in procs:
        assert pr.exitcode == 0
    out, records, state, times = got
    p = _problem()
    ref_out, ref_rec, ref_state = _run(p, 0, p["q"].shape[1], 0, p["v"].shape[1])
    torch.testing.assert_close(out, ref_out, rtol=1e-6, atol=1e-7)
    torch.testing.assert_close(records, ref_rec, rtol=1e-6, atol=1e-7)
    torch.testing.assert_close(state, ref_state, rtol=1e-6, atol=1e-7)
    assert times == [2.0, 10.0]  # MAX over ranks of (rank + 1, 10 - rank)


def _failing_rank_main(rank, world, port, result_q):
    """Rank 1 fails between steps (an exception before the timing reduction);
    rank 0 must learn of it on the host -- an error from its next collective
    within the short process-group timeout -- instead of waiting forever."""
    import datetime

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    torch.set_num_threads(1)
    p = _problem()
    sh = head_shard(p["q"].shape[1], p["v"].shape[1], world, rank)
    _run(p, sh.key_begin, sh.key_end, sh.value_begin, sh.value_end)
    if rank == 1:
        raise RuntimeError("injected failure on rank 1")
    try:
        max_over_ranks([1.0])
        result_q.put("no error")
    except Exception as exc:  # noqa: BLE001 -- any collective error is the expected outcome
        result_q.put(f"error: {type(exc).__name__}")


def test_gloo_failed_rank_surfaces_as_an_error_on_the_others():
    world = 2
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_rank_main, args=(r, world, port, result_q)) for r in range(world)]
    for pr in procs:
        pr.start()
    try:
        got = result_q.get(timeout=120)
    finally:
        for pr in procs:
            pr.join(timeout=60)
            if pr.is_alive():
                pr.kill()
    assert got.startswith("error"), got
    assert procs[1].exitcode != 0


def test_max_over_ranks_without_process_group_is_identity():
    assert max_over_ranks([1.5, 2.5]) == [1.5, 2.5]
