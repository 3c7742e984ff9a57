"""GPU parity of the grouped commit through GroupedCommitCoordinator across
several buckets (grouped_commit.py:896-1016): four align-mode GDN groups with
homogeneous layouts become a bucket of three and a bucket of one, each
launching its grouped plan, conv compaction and fold, followed by the
cross-bucket AND-valid publication of the shared block column.  Every plan
array, every state and conv page and the published column / acceptance arrays
are compared with the oracle (grouped_plan, fold, compact_conv,
publish_grouped_align): integers bit-exact, states within 1e-5.
"""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import gdn_oracle as O
from tests.test_gpu_parity import assert_fp32_close

pytestmark = pytest.mark.gpu

GROUPS, ROWS, REQS, H, HV, D, Q, BLOCKS, BLOCK, CONV = 4, 6, 8, 2, 4, 32, 4, 64, 8, 16


@pytest.fixture(scope="module")
def g():
    import gdn_recoverssm_b200 as pkg
    from gdn_recoverssm_b200 import _native

    _native.ops()
    return pkg


def test_coordinator_two_buckets_and_publication(g):
    rng = np.random.default_rng(99)
    dev = "cuda"
    req = rng.permutation(REQS)[:ROWS].astype(np.int64)            # native row -> request
    qlen = np.full(ROWS, Q)
    qlen[4] = 2
    qsl = np.concatenate([[0], np.cumsum(qlen)]).astype(np.int32)
    C = rng.integers(0, 40, REQS).astype(np.int32)
    C[req[:3]] = BLOCK - 2                                         # rows that cross a block
    sampled = rng.integers(0, Q + 1, REQS).astype(np.int32)
    sampled[req[:3]] = Q
    mapping = rng.permutation(REQS).astype(np.int32)
    mapping[req[5]] = -1                                           # a request with no persistent slot
    W = -(-(48 + Q) // BLOCK)

    contexts, payloads, pools, convs, groups_np = [], [], [], [], []
    for grp in range(GROUPS):
        pages = rng.permutation(np.arange(1, BLOCKS))[: 3 * ROWS].reshape(ROWS, 3)
        src = pages[:, 0].astype(np.int32)
        bt = np.zeros((REQS, W), dtype=np.int32)
        for r in range(ROWS):
            col = C[req[r]] // BLOCK
            bt[req[r], col] = pages[r, 1]
            bt[req[r], min(col + 1, W - 1)] = pages[r, 2]
        state = torch.randn(BLOCKS, HV, D, D, device=dev) * 0.1
        conv = torch.randn(BLOCKS, CONV, 3 + Q - 1, device=dev).to(torch.bfloat16)
        rec = torch.randn(ROWS, HV, Q, 2 * D + 1, device=dev) * 0.1
        rec[..., 2 * D] = torch.rand(ROWS, HV, Q, device=dev) * 0.5 + 0.5   # decays in (0.5, 1)
        pools.append((state, state.clone()))
        convs.append((conv, conv.clone()))
        ctx = g.GDNRecoverSSMCommitContext.from_tensors([conv], [state], [rec], spec_query_len=Q, max_num_reqs=ROWS)
        contexts.append((ctx, rec))
        payloads.append(SimpleNamespace(
            state_indices=torch.tensor(src, device=dev), query_start_loc=torch.tensor(qsl, device=dev),
            request_indices=torch.tensor(req, device=dev), block_table=torch.tensor(bt, device=dev),
            num_computed_tokens=torch.tensor(C, device=dev), block_size=BLOCK,
            request_rows=tuple(int(x) for x in req), query_lens=tuple(int(x) for x in qlen)))
        groups_np.append(dict(state_indices=src, query_start_loc=qsl, request_indices=req, num_blocks=BLOCKS,
                              block_table=bt, num_computed=C, block_size=BLOCK))
    metadata = [SimpleNamespace(recoverssm_commit=p, recoverssm_builder=SimpleNamespace(), recoverssm_context=c)
                for p, (c, _) in zip(payloads, contexts)]
    cols = torch.full((REQS,), -9, dtype=torch.int32, device=dev)
    acc = torch.full((REQS,), 7, dtype=torch.int32, device=dev)
    coord = g.GroupedCommitCoordinator()
    coord.commit(metadata, torch.tensor(sampled, device=dev), torch.tensor(mapping, device=dev), cols, acc)
    torch.cuda.synchronize()
    assert int(torch.ops.gdn_recoverssm_ac.device_status()) == 0
    buckets = list(coord._buckets.values())
    assert [len(b.contexts) for b in buckets] == [3, 1] and coord.last_launch_count == 3 + 3 + 1

    o_cols = np.full(REQS, -9)
    o_acc = np.full(REQS, 7)
    pub = []
    for b, members in zip(buckets, ([0, 1, 2], [3])):
        plan = O.grouped_plan(sampled, [groups_np[m] for m in members], rows=ROWS, plan_capacity=b.capacity,
                              spec_query_len=Q, align=True, publish=False)
        for key, t in (("source", b.source), ("length", b.length), ("final", b.final), ("boundary", b.boundary),
                       ("boundary_len", b.boundary_len), ("valid", b.valid), ("col", b.col)):
            assert t.cpu().numpy().astype(np.int64).tolist() == plan[key].astype(np.int64).tolist(), key
        pub.append((plan["valid"], plan["col"], b.capacity, len(members)))
        common = dict(layer_groups=list(range(len(members))), plan_capacity=b.capacity, rows=ROWS,
                      source=plan["source"], lengths=plan["length"], finals=plan["final"],
                      boundaries=plan["boundary"], boundary_lens=plan["boundary_len"], num_blocks=BLOCKS)
        want_states = [pools[m][1].cpu().numpy() for m in members]
        O.fold(want_states, [contexts[m][1].cpu().numpy() for m in members], None, None, record_rows=ROWS,
               layout="packed", query_len=Q, **common)
        want_convs = [convs[m][1].float().cpu().numpy() for m in members]
        O.compact_conv(want_convs, history=contexts[0][0].conv_history_len, align=True, **common)
        for i, m in enumerate(members):
            assert_fp32_close(pools[m][0].cpu().numpy(), want_states[i], what=f"group {m} states")
            assert np.array_equal(convs[m][0].float().cpu().numpy(), want_convs[i]), f"group {m} conv"
    assert (plan["length"] > 0).any()
    O.publish_grouped_align(pub, req, mapping, o_cols, o_acc, ROWS)
    assert cols.cpu().numpy().tolist() == o_cols.tolist()
    assert acc.cpu().numpy().tolist() == o_acc.tolist()
    assert (o_acc == 1).any(), "the case publishes at least one row"
