"""GPU parity at the reference's deployed TP4 geometry (the shape its index-range
simulation and record-byte tests use: 1418 checkpoint pages, 128 rows, 12
value heads over 4 key heads, Q = 4, K = V = 128), three layers in one commit
context, align mode with block tables, typed records with bf16 keys.

One verify per layer, then one grouped commit (plan -> conv compaction ->
fold over all three layers), every result against the float64 oracle:
outputs and records of every unit, the plan bit-exact, every page the plan
names (fold of the kernel's own records, boundary snapshots) and the conv
windows bit-exact; a sample of pages no plan row names is checked untouched.
The oracle runs on the used pages only (remapped to a compact pool).
"""

import numpy as np
import pytest
import torch

from oracle import gdn_oracle as O
from tests.test_gpu_k128 import _assert_rounded_close
from tests.test_gpu_parity import assert_fp32_close

pytestmark = pytest.mark.gpu

BLOCKS, ROWS, H, HV, D, Q, LAYERS = 1418, 128, 4, 12, 128, 4, 3
BLOCK, MAX_POS, CONV_DIM = 64, 4096, 64


@pytest.fixture(scope="module")
def g():
    import gdn_recoverssm_b200 as pkg
    from gdn_recoverssm_b200 import _native

    _native.ops()
    return pkg


def _unit(x):
    return x / np.linalg.norm(x, axis=-1, keepdims=True)


def test_deployed_geometry_three_layers(g):
    rng = np.random.default_rng(2024)
    qlen = np.full(ROWS, Q)
    qlen[rng.choice(ROWS, 16, replace=False)] = rng.integers(1, Q, 16)  # ragged windows
    qsl = np.concatenate([[0], np.cumsum(qlen)]).astype(np.int32)
    T = int(qsl[-1])
    W = -(-(MAX_POS + Q) // BLOCK)
    ids = rng.permutation(np.arange(1, BLOCKS))[: 3 * ROWS].reshape(ROWS, 3)
    src = ids[:, 0].astype(np.int32)
    src[[5, 77]] = 0  # null rows
    C = rng.integers(0, MAX_POS, ROWS)
    C[:8] = BLOCK - 2  # rows that cross a block boundary when they accept >= 2 tokens
    bt = np.zeros((ROWS, W), dtype=np.int32)
    bt[np.arange(ROWS), C // BLOCK] = ids[:, 1]
    bt[np.arange(ROWS), np.minimum(C // BLOCK + 1, W - 1)] = ids[:, 2]
    acc = rng.integers(0, Q + 1, ROWS).astype(np.int32)
    acc[:8] = Q

    dev = "cuda"
    act = torch.bfloat16
    layers = []
    for _ in range(LAYERS):
        state = torch.randn(BLOCKS, HV, D, D, device=dev) * 0.1
        layers.append(dict(
            q=torch.tensor(_unit(rng.standard_normal((T, H, D))), dtype=act, device=dev),
            k=torch.tensor(_unit(rng.standard_normal((T, H, D))), dtype=act, device=dev),
            v=torch.tensor(rng.standard_normal((T, HV, D)), dtype=act, device=dev),
            g=torch.tensor(-np.log1p(np.exp(rng.standard_normal((T, HV)))), dtype=torch.float32, device=dev),
            beta=torch.tensor(1 / (1 + np.exp(-rng.standard_normal((T, HV)))), dtype=torch.float32, device=dev),
            state=state, state0=state.clone(),
            conv=torch.randn(BLOCKS, CONV_DIM, 3 + Q - 1, device=dev).to(act),
            rec=g.ReplayRecordBuffers.allocate(ROWS, HV, H, Q, D, D, device=dev, key_dtype=act),
            out=torch.zeros(1, T, HV, D, dtype=act, device=dev),
        ))
    for L in layers:
        L["conv0"] = L["conv"].clone()
    qsl_d, src_d = torch.tensor(qsl, device=dev), torch.tensor(src, device=dev)

    for L in layers:
        g.gdn_recoverssm_verify(L["g"], L["beta"], L["q"][None], L["k"][None], L["v"][None],
                                checkpoint_state=L["state"], replay_cache=L["rec"], query_start_loc=qsl_d,
                                state_indices=src_d, spec_query_len=Q, out=L["out"])
    ctx = g.GDNRecoverSSMCommitContext.from_tensors([L["conv"] for L in layers], [L["state"] for L in layers],
                                                    [L["rec"] for L in layers], spec_query_len=Q, max_num_reqs=ROWS)
    ctx.commit(torch.tensor(acc, device=dev), src_d, qsl_d, block_table=torch.tensor(bt, device=dev),
               num_computed_tokens=torch.tensor(C.astype(np.int32), device=dev), mamba_block_size=BLOCK)
    torch.cuda.synchronize()
    assert int(torch.ops.gdn_recoverssm_ac.device_status()) == 0

    # ---- plan: bit-exact ---------------------------------------------------- #
    plan = O.prepare_commit_plan(acc, src, qsl, spec_query_len=Q, num_blocks=BLOCKS, block_table=bt,
                                 num_computed=C, block_size=BLOCK)
    lens = ctx.commit_lens[:ROWS].cpu().numpy()
    fin = ctx.final_state_indices[:ROWS].cpu().numpy()
    bnd = ctx.boundary_state_indices[:ROWS].cpu().numpy()
    blen = ctx.boundary_recovery_lens[:ROWS].cpu().numpy()
    assert np.array_equal(lens, plan["commit_lens"])
    assert np.array_equal(fin, plan["final"])
    assert np.array_equal(blen, plan["boundary_lens"])
    valid = plan["valid"].astype(bool)
    assert np.array_equal(bnd[valid], plan["boundary"][valid])
    assert (lens > 0).sum() > ROWS // 2 and ((blen > 0) & (bnd > 0)).any(), "the case exercises folds and snapshots"

    # ---- the used pages, remapped to a compact pool (index 0 = null) -------- #
    used = np.unique(np.concatenate([src, bt[bt > 0]]))
    used = used[used > 0]
    remap = np.zeros(BLOCKS, dtype=np.int64)
    remap[used] = np.arange(1, len(used) + 1)
    gather = torch.tensor(used, device=dev, dtype=torch.long)
    untouched = np.setdiff1d(np.arange(1, BLOCKS), used)
    sample = torch.tensor(rng.choice(untouched, 64, replace=False), device=dev, dtype=torch.long)

    f64 = lambda t: t.double().cpu().numpy()  # noqa: E731
    for li, L in enumerate(layers):
        # verify: every unit's outputs and typed records
        state0 = np.zeros((len(used) + 1, HV, D, D), dtype=np.float32)
        state0[1:] = L["state0"][gather].cpu().numpy()
        o_out = np.full((T, HV, D), -23.0)
        o_rec = (np.full((ROWS, HV, Q, D), -17.0), np.full((ROWS, H, Q, D), -16.0), np.full((ROWS, HV, Q), -19.0))
        g_out = L["out"][0].double().cpu().numpy()
        O.verify_batch(f64(L["q"]), f64(L["k"]), f64(L["v"]), f64(L["g"]), f64(L["beta"]), state0.astype(np.float64),
                       qsl, remap[src], spec_query_len=Q, record_rows=ROWS, layout="soa", out=o_out, records=o_rec)
        live = o_out != -23.0
        _assert_rounded_close(np.where(live, g_out, -23.0), o_out, 7, -126, f"layer {li} bf16 output")
        rec = L["rec"]
        for got_t, want, sentinel, name in zip((rec.correction, rec.key, rec.decay), o_rec, (-17.0, -16.0, -19.0),
                                              ("correction", "key", "decay")):
            got = f64(got_t)
            m = want != sentinel
            if name == "key":
                assert np.array_equal(got[m], want[m]), f"layer {li}: bf16 key records keep the input bits"
            else:
                assert_fp32_close(got[m], want[m], what=f"layer {li} {name}")
        # fold of the kernel's own records over the used pages
        pool = [state0.copy()]
        O.fold(pool, [rec.correction.cpu().numpy()], [rec.key.float().cpu().numpy()], [rec.decay.cpu().numpy()],
               layer_groups=[0], plan_capacity=ROWS, rows=ROWS, source=remap[src], lengths=lens, finals=remap[fin],
               boundaries=remap[bnd], boundary_lens=blen, num_blocks=len(used) + 1, record_rows=ROWS, layout="soa",
               query_len=Q)
        got_pages = L["state"][gather].cpu().numpy()
        for p in range(len(used)):
            assert_fp32_close(got_pages[p], pool[0][p + 1], what=f"layer {li} page {used[p]}")
        assert torch.equal(L["state"][sample], L["state0"][sample]), f"layer {li}: untouched pages changed"
        # conv windows, bit-exact
        conv0 = np.zeros((len(used) + 1, CONV_DIM, 3 + Q - 1), dtype=np.float32)
        conv0[1:] = L["conv0"][gather].float().cpu().numpy()
        O.compact_conv([conv0], layer_groups=[0], plan_capacity=ROWS, rows=ROWS, source=remap[src], lengths=lens,
                       finals=remap[fin], boundaries=remap[bnd], boundary_lens=blen, num_blocks=len(used) + 1,
                       history=ctx.conv_history_len, align=True)
        assert np.array_equal(L["conv"][gather].float().cpu().numpy(), conv0[1:]), f"layer {li}: conv windows"
        assert torch.equal(L["conv"][sample], L["conv0"][sample])
