"""Randomised per-context commit plans on the GPU against the NumPy oracle,
bit-exact.

The plan is integer work, so every output array (commit length, final page,
boundary page and length, validity, block column) must equal the oracle's
restatement of the reference plan (kernels.py:936-1072) on every row.  Each
case draws the metadata the reference tests and the kernel's bounds checks
care about: accepted counts below zero and past the window, empty, ragged,
reversed and over-long query windows, null / negative / out-of-pool slots,
request mappings that point past the accepted and computed arrays or the
block table, negative computed counts and counts near 2^31 (the int32 wrap of
the reference's align arithmetic), block-table entries outside the pool, and
block sizes from one window to 2^30.  Only the plan launch runs (no fold).
The grouped plan over one to three groups, and its align publication into
the persistent column / acceptance arrays, is fuzzed the same way.
"""

import numpy as np
import pytest
import torch

from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu

KEYS = ("commit_lens", "final", "boundary", "boundary_lens", "valid", "col")


@pytest.fixture(scope="module")
def g():
    import gdn_recoverssm_b200 as pkg
    from gdn_recoverssm_b200 import _native

    _native.ops()
    return pkg


def _case(rng, Q, B, blocks):
    qlen = rng.integers(0, Q + 1, B)
    qsl = np.concatenate([[0], np.cumsum(qlen)]).astype(np.int64)
    k = rng.integers(0, B + 1)
    if B > 2:
        qsl[k] = qsl[k] + rng.integers(-3, 4)  # reversed / over-long windows around row k
    slots = rng.integers(1, blocks, B)
    slots[rng.random(B) < 0.1] = 0
    slots[rng.random(B) < 0.05] = -int(rng.integers(1, 5))
    slots[rng.random(B) < 0.05] = blocks + int(rng.integers(0, 5))
    n_acc = B + int(rng.integers(0, 4))
    accepted = rng.integers(-2, Q + 3, n_acc)
    return qsl, slots, accepted


@pytest.mark.parametrize("seed", range(64))
def test_context_plan_matches_oracle(g, seed):
    rng = np.random.default_rng(1000 + seed)
    dev = "cuda"
    Q = int(rng.integers(1, 9))
    B = int(rng.integers(1, 300))
    blocks = int(rng.integers(8, 400))
    HV, D = 2, 32
    qsl, slots, accepted = _case(rng, Q, B, blocks)
    align = seed % 4 != 3
    idx_dtype = torch.int64 if seed % 3 == 0 else torch.int32
    state = torch.zeros(blocks, HV, D, D, device=dev)
    rec = torch.zeros(B, HV, Q, 2 * D + 1, device=dev)
    conv = torch.zeros(blocks, 8, 2 + Q, dtype=torch.bfloat16, device=dev)
    ctx = g.GDNRecoverSSMCommitContext.from_tensors([conv], [state], [rec], spec_query_len=Q, max_num_reqs=B)
    req = None
    if seed % 2 == 1:  # a request mapping, some entries past the accepted / computed arrays and the table
        req = rng.permutation(B + 4)[:B].astype(np.int64)
        req[rng.random(B) < 0.05] = -1
    kw, okw = {}, {}
    if align:
        bs = int(rng.choice([Q, 16, 64, 1000, 1 << 30]))
        bs = max(bs, Q)
        W = int(rng.integers(1, 10))
        rows_t = B + int(rng.integers(0, 3))
        table = rng.integers(-2, blocks + 3, (rows_t, W))
        computed = rng.integers(0, W * min(bs, 1 << 20), B + int(rng.integers(0, 3)))
        computed[rng.random(computed.shape[0]) < 0.05] = -int(rng.integers(1, 100))
        computed[rng.random(computed.shape[0]) < 0.05] = (1 << 31) - int(rng.integers(1, 9))  # int32 wrap
        kw = dict(block_table=torch.tensor(table, dtype=idx_dtype, device=dev),
                  num_computed_tokens=torch.tensor(computed, dtype=idx_dtype, device=dev), mamba_block_size=bs)
        okw = dict(block_table=table, num_computed=computed, block_size=bs)
    specs = ctx.make_commit_specs(
        torch.tensor(accepted, dtype=idx_dtype, device=dev), torch.tensor(slots, dtype=idx_dtype, device=dev),
        torch.tensor(qsl, dtype=idx_dtype, device=dev),
        request_indices=None if req is None else torch.tensor(req, dtype=idx_dtype, device=dev),
        commit_conv=False, **kw)
    assert specs[0].name == "commit_plan"
    ctx.plan.fill_(-77)
    specs[0].launch()
    torch.cuda.synchronize()
    want = O.prepare_commit_plan(accepted, slots, qsl, spec_query_len=Q, num_blocks=blocks, request_indices=req, **okw)
    got = {"commit_lens": ctx.commit_lens, "final": ctx.final_state_indices, "boundary": ctx.boundary_state_indices,
           "boundary_lens": ctx.boundary_recovery_lens, "valid": ctx.align_valid, "col": ctx.align_col}
    for key in KEYS:
        g_ = got[key][:B].cpu().numpy().astype(np.int64)
        bad = np.nonzero(g_ != want[key])[0]
        assert bad.size == 0, f"{key}: rows {bad[:8].tolist()} got {g_[bad[:8]].tolist()} want {want[key][bad[:8]].tolist()}"
    # the cases exercise both outcomes
    if B > 20:
        assert 0 < int(want["valid"].sum()) < B or not align


@pytest.mark.parametrize("seed", range(32))
def test_grouped_plan_matches_oracle(g, seed):
    """The grouped plan (grouped_commit.py:31-222) over one to three groups
    with independent pages, tables and block sizes, and its align
    publication into the persistent column / acceptance arrays."""
    rng = np.random.default_rng(5000 + seed)
    dev = "cuda"
    G = int(rng.integers(1, 4))
    Q = int(rng.integers(1, 9))
    rows = int(rng.integers(1, 200))
    cap = rows + int(rng.integers(0, 5))
    reqs = rows + int(rng.integers(0, 6))
    align = seed % 4 != 3
    publish = align and seed % 2 == 0
    idx_dtype = torch.int64 if seed % 3 == 0 else torch.int32
    sampled = rng.integers(-2, Q + 3, max(1, reqs + int(rng.integers(-2, 3))))
    base_req = rng.permutation(reqs + 3)[:rows].astype(np.int64)
    groups_np, groups_t = [], []
    for gi in range(G):
        blocks = int(rng.integers(8, 300))
        qsl, slots, _ = _case(rng, Q, rows, blocks)
        req = base_req.copy()
        if rng.random() < 0.5:  # a group whose mapping differs on some rows
            flip = rng.random(rows) < 0.05
            req[flip] = rng.integers(-1, reqs + 3, int(flip.sum()))
        grp = dict(state_indices=slots, query_start_loc=qsl, request_indices=req, num_blocks=blocks)
        t = dict(state=torch.tensor(slots, dtype=idx_dtype, device=dev), qsl=torch.tensor(qsl, dtype=idx_dtype, device=dev),
                 req=torch.tensor(req, dtype=idx_dtype, device=dev), table=None, computed=None, bs=1)
        if align:
            bs = max(int(rng.choice([Q, 16, 64, 1000])), Q)
            W = int(rng.integers(1, 10))
            table = rng.integers(-2, blocks + 3, (max(1, reqs + int(rng.integers(-2, 3))), W))
            computed = rng.integers(0, W * bs, max(1, reqs + int(rng.integers(-2, 3))))
            computed[rng.random(computed.shape[0]) < 0.05] = -int(rng.integers(1, 100))
            grp.update(block_table=table, num_computed=computed, block_size=bs)
            t.update(table=torch.tensor(table, dtype=idx_dtype, device=dev),
                     computed=torch.tensor(computed, dtype=idx_dtype, device=dev), bs=bs)
        groups_np.append(grp)
        groups_t.append(t)
    n_slots = reqs + 2
    # an injective request -> slot map inside the persistent arrays (two rows
    # publishing into one slot would race in the reference too), some unmapped
    mapping = rng.permutation(n_slots + 3)[: reqs + int(rng.integers(0, 3))].astype(np.int64)
    mapping[(mapping >= n_slots) | (rng.random(mapping.shape[0]) < 0.1)] = -1
    cols0 = rng.integers(-5, 5, n_slots)
    acc0 = rng.integers(-5, 5, n_slots)
    cols_np, acc_np = cols0.copy(), acc0.copy()
    want = O.grouped_plan(sampled, groups_np, rows=rows, plan_capacity=cap, spec_query_len=Q, align=align,
                          publish=publish, idx_mapping=mapping, persistent_cols=cols_np, persistent_accepted=acc_np)
    out = torch.zeros(7, G * cap, dtype=torch.int32, device=dev)
    cols = torch.tensor(cols0, dtype=torch.int32, device=dev)
    acc = torch.tensor(acc0, dtype=torch.int32, device=dev)
    torch.ops.gdn_recoverssm_ac.grouped_plan(
        torch.tensor(sampled, dtype=idx_dtype, device=dev), [t["state"] for t in groups_t], [t["qsl"] for t in groups_t],
        [t["req"] for t in groups_t], [t["table"] for t in groups_t], [t["computed"] for t in groups_t],
        [grp["num_blocks"] for grp in groups_np], [t["bs"] for t in groups_t], *out.unbind(0),
        torch.tensor(mapping, dtype=idx_dtype, device=dev), cols, acc, rows, cap, Q, align, publish)
    torch.cuda.synchronize()
    for i, key in enumerate(("source", "length", "final", "boundary", "boundary_len", "valid", "col")):
        got = out[i].cpu().numpy().astype(np.int64)
        bad = np.nonzero(got != want[key])[0]
        assert bad.size == 0, f"{key}: offsets {bad[:8].tolist()} got {got[bad[:8]].tolist()} want {want[key][bad[:8]].tolist()}"
    assert np.array_equal(cols.cpu().numpy().astype(np.int64), cols_np), "published columns"
    assert np.array_equal(acc.cpu().numpy().astype(np.int64), acc_np), "published acceptance"
