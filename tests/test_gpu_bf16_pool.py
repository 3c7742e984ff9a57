"""GPU parity with a bf16 state pool (the reference accepts fp32 or bf16
states, csrc/ops.cpp:100-106): verify reads the bf16 checkpoint (CUDA-core
kernel), the commit folds into bf16 pages.  Records and outputs are compared
with the float64 oracle run on the same bf16 state values; folded pages are
the oracle's float64 fold of the kernel's own records, within one bf16 ulp
(the kernel folds in fp32 and rounds once at the store) or, for near-zero
results of a cancelling fold, 1e-5 of the tile row's largest magnitude.
"""

import numpy as np
import pytest
import torch

from oracle import gdn_oracle as O
from tests.test_gpu_parity import assert_fp32_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def g():
    import gdn_recoverssm_b200 as pkg
    from gdn_recoverssm_b200 import _native

    _native.ops()
    return pkg


def _unit(x):
    return x / np.linalg.norm(x, axis=-1, keepdims=True)


@pytest.mark.parametrize("D,Q,align", [(128, 4, True), (64, 3, False)], ids=["K128-align", "K64-none"])
def test_bf16_pool_verify_and_commit(g, D, Q, align):
    rng = np.random.default_rng(D + Q)
    ROWS, H, HV, BLOCKS, BLOCK = 16, 2, 4, 64, 16
    dev = "cuda"
    qsl = (np.arange(ROWS + 1) * Q).astype(np.int32)
    T = int(qsl[-1])
    ids = rng.permutation(np.arange(1, BLOCKS))[: 3 * ROWS].reshape(ROWS, 3)
    src = ids[:, 0].astype(np.int32)
    acc = rng.integers(1, Q + 1, ROWS).astype(np.int32)
    q = torch.tensor(_unit(rng.standard_normal((T, H, D))), dtype=torch.bfloat16, device=dev)
    k = torch.tensor(_unit(rng.standard_normal((T, H, D))), dtype=torch.bfloat16, device=dev)
    v = torch.tensor(rng.standard_normal((T, HV, D)), dtype=torch.bfloat16, device=dev)
    gg = torch.tensor(-np.log1p(np.exp(rng.standard_normal((T, HV)))), dtype=torch.float32, device=dev)
    beta = torch.tensor(1 / (1 + np.exp(-rng.standard_normal((T, HV)))), dtype=torch.float32, device=dev)
    state = (torch.randn(BLOCKS, HV, D, D, device=dev) * 0.1).to(torch.bfloat16)
    state0 = state.float().cpu().numpy().astype(np.float64)
    rec = torch.zeros(ROWS, HV, Q, 2 * D + 1, device=dev)
    out = torch.zeros(1, T, HV, D, dtype=torch.bfloat16, device=dev)
    src_d, qsl_d = torch.tensor(src, device=dev), torch.tensor(qsl, device=dev)
    g.gdn_recoverssm_verify(gg, beta, q[None], k[None], v[None], checkpoint_state=state, replay_cache=rec,
                            query_start_loc=qsl_d, state_indices=src_d, spec_query_len=Q, out=out)
    conv = torch.zeros(BLOCKS, 8, 3 + Q - 1, dtype=torch.bfloat16, device=dev)
    ctx = g.GDNRecoverSSMCommitContext.from_tensors([conv], [state], [rec], spec_query_len=Q, max_num_reqs=ROWS)
    kw = {}
    if align:
        C = rng.integers(0, 200, ROWS)
        C[:4] = BLOCK - 2
        W = -(-(200 + Q) // BLOCK)
        bt = np.zeros((ROWS, W), dtype=np.int32)
        bt[np.arange(ROWS), C // BLOCK] = ids[:, 1]
        bt[np.arange(ROWS), np.minimum(C // BLOCK + 1, W - 1)] = ids[:, 2]
        kw = dict(block_table=torch.tensor(bt, device=dev), num_computed_tokens=torch.tensor(C.astype(np.int32),
                  device=dev), mamba_block_size=BLOCK)
    ctx.commit(torch.tensor(acc, device=dev), src_d, qsl_d, commit_conv=False, **kw)
    torch.cuda.synchronize()
    assert int(torch.ops.gdn_recoverssm_ac.device_status()) == 0

    o_out, o_rec = O.verify_batch(q.double().cpu().numpy(), k.double().cpu().numpy(), v.double().cpu().numpy(),
                                  gg.double().cpu().numpy(), beta.double().cpu().numpy(), state0, qsl, src,
                                  spec_query_len=Q, records=np.zeros(tuple(rec.shape)))
    assert_fp32_close(rec.double().cpu().numpy(), o_rec, what="records")
    got_out = out[0].double().cpu().numpy()
    assert np.max(np.abs(got_out - o_out)) <= 2 ** -7 * np.abs(o_out).max()

    lens = ctx.commit_lens[:ROWS].cpu().numpy()
    fin = ctx.final_state_indices[:ROWS].cpu().numpy()
    bnd = ctx.boundary_state_indices[:ROWS].cpu().numpy()
    blen = ctx.boundary_recovery_lens[:ROWS].cpu().numpy()
    want = [state0.copy()]
    O.fold(want, [rec.cpu().numpy()], None, None, layer_groups=[0], plan_capacity=ctx.commit_lens.shape[0], rows=ROWS,
           source=src, lengths=lens, finals=fin, boundaries=bnd, boundary_lens=blen, num_blocks=BLOCKS,
           record_rows=ROWS, layout="packed", query_len=Q)
    got = state.float().cpu().numpy().astype(np.float64)
    pages = np.unique(np.concatenate([fin[lens > 0], bnd[(lens > 0) & (blen > 0) & (bnd > 0)]]))
    assert len(pages) > 0
    w = want[0][pages]
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(w), 1e-30))) - 7)
    # one bf16 ulp, or 1e-5 of the tile row's largest magnitude: the floor for
    # near-zero results of a cancelling h * d + c * k, which no fp32 fold pins
    # to the ulp of the result
    floor = 1e-5 * np.abs(w).max(axis=-1, keepdims=True)
    ratio = np.abs(got[pages] - w) / np.maximum(ulp, floor)
    bad = ratio > 1.01
    if bad.any():
        pi = np.unique(np.nonzero(bad)[0])
        info = [(int(pages[i]), int(bad[i].sum()), float(ratio[i].max())) for i in pi[:8]]
        role = {int(x): "fin" for x in fin[lens > 0]}
        role.update({int(x): "bnd" for x in bnd[(lens > 0) & (blen > 0) & (bnd > 0)]})
        raise AssertionError(f"folded bf16 pages beyond one ulp: {len(pi)} pages, (page, count, max ulps): {info}, "
                             f"roles {[role.get(p_, '?') for p_, _, _ in info]}, max {ratio.max():.2f}")
    others = np.setdiff1d(np.arange(BLOCKS), np.concatenate([pages, src]))
    assert np.array_equal(got[others], state0[others])
