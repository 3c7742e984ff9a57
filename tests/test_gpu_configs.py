"""GPU parity at the benchmark configurations (1-4), EVERY unit.

For each configuration at full size the CUDA verify + commit runs once and is
checked against a float64 torch restatement of the same semantics
(tests/torch_reference.py, pinned on CPU to the NumPy oracle) evaluated on the
GPU for every (row, value head) unit:

* every output token: bf16 within one ulp of the float64 value (or 1e-5 of
  the token's largest output magnitude, for near-zero results of a
  cancelling sum);
* every record of every unit: max-relative and l2-relative error <= 1e-5;
* every plan row bit-exact against the NumPy oracle's plan;
* every final page and every boundary snapshot: the float64 state after the
  row's accepted prefix (after its boundary length), per unit <= 1e-5 --
  against plain sequential decode of the same tokens, so for config 3
  (Q = 1) this is "one verify + commit equals one recurrent decode step";
* the fold alone: every final page against a float64 re-fold of the kernel's
  own records from the checkpoint, per unit <= 1e-5;
* the checkpoint pool bit-identical after verify, and every page that no plan
  row names bit-identical after the commit.
"""

import numpy as np
import pytest
import torch

from oracle import gdn_oracle as O
from tests.torch_reference import rel_errors_per_unit, rounded_ok, verify_rows

pytestmark = pytest.mark.gpu
TOL = 1e-5


@pytest.fixture(scope="module")
def g():
    import gdn_recoverssm_b200 as pkg
    from gdn_recoverssm_b200 import _native

    _native.ops()
    return pkg


def _oracle_plan(wl):
    meta = wl.extra["meta"]
    align = wl.block_table is not None
    return O.prepare_commit_plan(
        meta["accepted"].numpy(), meta["state_indices"].numpy(), meta["qsl"].numpy(), spec_query_len=wl.Q,
        num_blocks=wl.state.shape[0], block_table=meta["block_table"].numpy() if align else None,
        num_computed=meta["num_computed"].numpy() if align else None, block_size=wl.block_size,
    )


@pytest.mark.parametrize("cfg", [1, 2, 3, 4])
def test_config_every_unit(g, cfg):
    from gdn_recoverssm_b200 import synthetic

    wl = synthetic.make(cfg, "cuda", seed=3, conv_dim=16)
    B, HV, D, Q = wl.B, wl.HV, wl.D, wl.Q
    pool0 = wl.state.clone()
    wl.records.fill_(-17.0)
    wl.out.fill_(-23.0)
    g.gdn_recoverssm_verify(wl.g, wl.beta, wl.q, wl.k, wl.v, checkpoint_state=wl.state, replay_cache=wl.records,
                            query_start_loc=wl.qsl, state_indices=wl.state_indices, spec_query_len=Q, out=wl.out)
    torch.cuda.synchronize()
    assert torch.equal(wl.state, pool0), "verify wrote the checkpoint pool"
    assert int(torch.ops.gdn_recoverssm_ac.device_status()) == 0
    records = wl.records.clone()

    ctx = g.GDNRecoverSSMCommitContext.from_tensors([wl.conv], [wl.state], [wl.records], spec_query_len=Q,
                                                    max_num_reqs=B)
    kw = {}
    if wl.block_table is not None:
        kw = dict(block_table=wl.block_table, num_computed_tokens=wl.num_computed, mamba_block_size=wl.block_size)
    ctx.commit(wl.accepted, wl.state_indices, wl.qsl, **kw)
    torch.cuda.synchronize()
    assert int(torch.ops.gdn_recoverssm_ac.device_status()) == 0

    plan = _oracle_plan(wl)
    got = {"commit_lens": ctx.commit_lens, "final": ctx.final_state_indices, "boundary": ctx.boundary_state_indices,
           "boundary_lens": ctx.boundary_recovery_lens, "valid": ctx.align_valid, "col": ctx.align_col}
    for key, t in got.items():
        assert np.array_equal(t[:B].cpu().numpy().astype(np.int64), plan[key]), f"plan {key}"
    assert plan["valid"].all(), "synthetic rows must all be valid"
    n = torch.tensor(plan["commit_lens"], device="cuda")
    fin = torch.tensor(plan["final"], device="cuda")
    bnd = torch.tensor(plan["boundary"], device="cuda")
    blen = torch.tensor(plan["boundary_lens"], device="cuda")
    snap = (bnd > 0) & (bnd < wl.state.shape[0]) & (bnd != fin) & (blen > 0)
    if cfg in (2, 4):
        assert bool(snap.any()), "align configs must exercise boundary snapshots"

    # pages no plan row names: bit-identical
    named = torch.zeros(wl.state.shape[0], dtype=torch.bool, device="cuda")
    named[fin] = True
    named[bnd[snap]] = True
    assert torch.equal(wl.state[~named], pool0[~named]), "the commit wrote a page no plan row names"

    q, k, v = wl.q[0], wl.k[0], wl.v[0]
    chunk = max(1, int(1.5e9 // (HV * D * D * 8 * 8)))
    worst = {"records": [0.0, 0.0], "final": [0.0, 0.0], "boundary": [0.0, 0.0], "fold": [0.0, 0.0]}
    bad_out = 0
    for r0 in range(0, B, chunk):
        r1 = min(B, r0 + chunk)
        res = verify_rows(q, k, v, wl.g, wl.beta, pool0, wl.qsl, wl.state_indices, Q=Q,
                          rows=(r0, r1), capture={"final": n, "boundary": blen})
        assert bool(res["valid"].all() & res["live"].all())
        # outputs of every token (bf16)
        got_out = wl.out[0][res["token"]]  # [R, Q, HV, V]
        bad_out += int((~rounded_ok(got_out.float(), res["out"], 7, -126)).sum())
        # records of every unit
        e = rel_errors_per_unit(records[r0:r1], res["records"], 2)
        worst["records"] = [max(worst["records"][i], float(e[i].max())) for i in range(2)]
        # final pages against float64 sequential decode of the accepted prefix
        e = rel_errors_per_unit(wl.state[fin[r0:r1]], res["final"], 2)
        worst["final"] = [max(worst["final"][i], float(e[i].max())) for i in range(2)]
        # boundary snapshots against the state after the boundary length
        rows = snap[r0:r1].nonzero().flatten()
        if rows.numel():
            e = rel_errors_per_unit(wl.state[bnd[r0:r1][rows]], res["boundary"][rows], 2)
            worst["boundary"] = [max(worst["boundary"][i], float(e[i].max())) for i in range(2)]
        # the fold alone: float64 re-fold of the kernel's own records
        h = pool0[wl.state_indices[r0:r1].long()].double()
        rec = records[r0:r1].double()  # [R, HV, Q, V + K + 1]
        for t in range(Q):
            step = (t < n[r0:r1])[:, None, None, None]
            c, kk, d = rec[:, :, t, :D], rec[:, :, t, D : 2 * D], rec[:, :, t, 2 * D]
            h = torch.where(step, h * d[..., None, None] + c[..., :, None] * kk[..., None, :], h)
        e = rel_errors_per_unit(wl.state[fin[r0:r1]], h, 2)
        worst["fold"] = [max(worst["fold"][i], float(e[i].max())) for i in range(2)]
        del res, h, rec
    print(f"config {cfg}: worst per-unit (max-rel, l2-rel) {worst}; bf16 outputs off by > 1 ulp: {bad_out}")
    assert bad_out == 0, f"{bad_out} output elements beyond one bf16 ulp"
    for key, e in worst.items():
        assert max(e) <= TOL, f"{key} rel error {e}"
