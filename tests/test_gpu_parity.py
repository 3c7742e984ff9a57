"""GPU parity: the CUDA path (through torch.ops.gdn_recoverssm_ac -> C ABI)
against the reference-Triton fixtures and the float64 oracle.

Tolerances (north star): plan / slot / accepted-prefix / boundary indexing and
conv-window copies bit-exact; fp32 states, records and outputs within 1e-5
relative (``max|d| / max|ref|`` and ``||d|| / ||ref||``); bf16 outputs within
one bf16 ulp of the oracle value rounded once (the kernel computes in fp32 and
rounds once, like the reference).
"""

import numpy as np
import pytest
import torch

from oracle import gdn_oracle as O
from tests import golden_io
from tests.test_oracle_pins import CONTEXT_CASES, VERIFY_CASES, oracle_verify_from_fixture

pytestmark = pytest.mark.gpu
TOL = 1e-5


@pytest.fixture(scope="module")
def pkg():
    import gdn_recoverssm_b200 as g
    from gdn_recoverssm_b200 import _native

    _native.ops()  # fail loudly if the sm_100a build is missing
    return g


def _dev(t):
    return t.cuda() if isinstance(t, torch.Tensor) else torch.as_tensor(t).cuda()


def _np(t):
    return t.detach().double().cpu().numpy() if isinstance(t, torch.Tensor) else np.asarray(t)


def assert_fp32_close(got, want, tol=TOL, what=""):
    inf_rel, l2_rel = O.rel_errors(_np(got), _np(want))
    assert inf_rel <= tol and l2_rel <= tol, f"{what}: max-rel {inf_rel:.3g}, l2-rel {l2_rel:.3g} > {tol}"


def assert_bf16_within_ulp(got, want_f64, what=""):
    """Each bf16 output is the fp64 oracle value rounded to bf16, or its
    neighbour when the fp32 computation lands across a rounding boundary."""
    got = _np(got)
    want = _np(want_f64)
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(want), 1e-30))) - 7)
    assert np.all(np.abs(got - want) <= ulp * 1.01 + 1e-30), what
    rounded = torch.from_numpy(want).float().bfloat16().double().numpy()
    assert np.mean(got == rounded) > 0.97, what


def _verify_cuda(g, c):
    """Run the package verify on a fixture's inputs with sentinel outputs."""
    T, HV, V = c["v"].shape
    H, K = c["q"].shape[1], c["q"].shape[2]
    Q, R = c["spec_query_len"], c["record_rows"]
    act = c["q"].dtype
    out = torch.full((1, T, HV, V), -23.0, dtype=act, device="cuda")
    if c["layout"] == "packed":
        cache = torch.full((R, HV, Q, V + K + 1), -17.0, device="cuda")
    else:
        kd = act if c["normalized"] else torch.float32
        cache = g.ReplayRecordBuffers(
            torch.full((R, HV, Q, V), -17.0, device="cuda"),
            torch.full((R, H, Q, K), -16.0, dtype=kd, device="cuda"),
            torch.full((R, HV, Q), -19.0, device="cuda"),
        )
    state = _dev(c["state"])
    before = state.clone()
    g.gdn_recoverssm_verify(
        _dev(c["g"])[None], _dev(c["beta"])[None], _dev(c["q"])[None], _dev(c["k"])[None], _dev(c["v"])[None],
        checkpoint_state=state, replay_cache=cache, query_start_loc=_dev(c["qsl"]),
        state_indices=_dev(c["state_indices"]), spec_query_len=Q, qk_already_normalized=bool(c["normalized"]),
        out=out,
    )
    torch.cuda.synchronize()
    assert torch.equal(state, before), "verify modified the read-only checkpoint"
    return out[0].cpu(), cache


@pytest.mark.parametrize("name", VERIFY_CASES)
def test_verify_matches_oracle_and_reference_fixture(pkg, name):
    c = golden_io.load(name)
    out, cache = _verify_cuda(pkg, c)
    o_out, o_recs = oracle_verify_from_fixture(c)
    sentinel_out = _np(c["out"]) == -23.0
    assert np.array_equal(_np(out) == -23.0, sentinel_out), "output store mask differs from the reference"
    live = ~sentinel_out
    if out.dtype == torch.bfloat16:
        assert_bf16_within_ulp(_np(out)[live], o_out[live], "verify output")
    else:
        assert_fp32_close(_np(out)[live], o_out[live], what="verify output")
    if c["layout"] == "packed":
        rec = _np(cache.cpu())
        ref = _np(c["records"])
        assert np.array_equal(rec == -17.0, ref == -17.0), "record store mask differs from the reference"
        m = rec != -17.0
        assert_fp32_close(rec[m], o_recs[m], what="packed records")
    else:
        for got, ref_key, mine, sentinel in zip(
            (cache.correction, cache.key, cache.decay), ("corr", "key", "decay"), o_recs, (-17.0, -16.0, -19.0)
        ):
            got = _np(got.cpu())
            ref = _np(c[ref_key])
            assert np.array_equal(got == sentinel, ref == sentinel), f"{ref_key} store mask differs"
            m = got != sentinel
            if ref_key == "key" and c["normalized"]:
                assert np.array_equal(got[m], ref[m]), "pre-normalised keys must keep their input bits"
            else:
                assert_fp32_close(got[m], mine[m], what=ref_key)


def _context_cuda(g, c):
    layers = int(c["layers"])
    Q = c["spec_query_len"]
    states = [_dev(c[f"state_before{i}"]) for i in range(layers)]
    convs = [_dev(c[f"conv_before{i}"]) for i in range(layers)]
    if c["layout"] == "packed":
        records = [_dev(c[f"records{i}"]) for i in range(layers)]
    else:
        records = [g.ReplayRecordBuffers(_dev(c[f"corr{i}"]), _dev(c[f"key{i}"]), _dev(c[f"decay{i}"]))
                   for i in range(layers)]
    rows = len(c["src"])
    ctx = g.GDNRecoverSSMCommitContext.from_tensors(convs, states, records, spec_query_len=Q, max_num_reqs=rows)
    kw = dict(request_indices=_dev(c["request_indices"]))
    if c["align"]:
        kw.update(block_table=_dev(c["block_table"]), num_computed_tokens=_dev(c["num_computed"]),
                  mamba_block_size=int(c["block_size"]))
    ctx.commit(_dev(c["accepted"]), _dev(c["src"]), _dev(c["qsl"]), **kw)
    torch.cuda.synchronize()
    return ctx, states, convs


@pytest.mark.parametrize("name", CONTEXT_CASES)
def test_context_commit_matches_reference_fixture(pkg, name):
    c = golden_io.load(name)
    ctx, states, convs = _context_cuda(pkg, c)
    rows = len(c["src"])
    plan = {
        "commit_lens": ctx.commit_lens, "final": ctx.final_state_indices, "boundary": ctx.boundary_state_indices,
        "boundary_lens": ctx.boundary_recovery_lens, "valid": ctx.align_valid, "col": ctx.align_col,
    }
    for key, t in plan.items():
        assert t[:rows].cpu().tolist() == _np(c[key]).astype(np.int64).tolist(), key
    for i in range(int(c["layers"])):
        assert_fp32_close(states[i].cpu(), golden_io.full_after(c, "state", i), what=f"state layer {i}")
        assert torch.equal(convs[i].cpu(), golden_io.full_after(c, "conv", i)), f"conv layer {i}"


def test_grouped_commit_matches_reference_fixture(pkg):
    from types import SimpleNamespace

    g = pkg
    c = golden_io.load("grouped_align_soa")
    Q = c["spec_query_len"]
    rows = len(c["request_indices"])
    entries, states, convs = [], [], []
    for grp in range(2):
        st = [_dev(c[f"state_before{grp * 2 + l}"]) for l in range(2)]
        cv = [_dev(c[f"conv_before{grp * 2 + l}"]) for l in range(2)]
        recs = [g.ReplayRecordBuffers(_dev(c[f"corr{grp * 2 + l}"]), _dev(c[f"key{grp * 2 + l}"]),
                                      _dev(c[f"decay{grp * 2 + l}"])) for l in range(2)]
        states += st
        convs += cv
        ctx = g.GDNRecoverSSMCommitContext.from_tensors(cv, st, recs, spec_query_len=Q, max_num_reqs=rows)
        payload = SimpleNamespace(
            state_indices=_dev(c[f"state_indices{grp}"]), query_start_loc=_dev(c["qsl"]),
            request_indices=_dev(c["request_indices"]), block_table=_dev(c[f"block_table{grp}"]),
            num_computed_tokens=_dev(c["computed"]), block_size=int(c["block_size"]),
            request_rows=tuple(int(x) for x in c["request_indices"]), query_lens=tuple(
                int(c["qsl"][r + 1] - c["qsl"][r]) for r in range(rows)),
        )
        entries.append(g.CommitEntry(None, payload, ctx))
    bucket = g.GroupedCommitBucket(tuple(e.context for e in entries))
    cols = torch.full((6,), -9, dtype=torch.int32, device="cuda")
    acc = torch.full((6,), 7, dtype=torch.int32, device="cuda")
    for spec in bucket.make_specs(entries, _dev(c["sampled"]), _dev(c["mapping"]), cols, acc):
        spec.launch()
    torch.cuda.synchronize()
    for key, t in (("source", bucket.source), ("length", bucket.length), ("final", bucket.final),
                   ("boundary", bucket.boundary), ("boundary_len", bucket.boundary_len), ("valid", bucket.valid),
                   ("col", bucket.col)):
        assert t.cpu().tolist() == _np(c["plan_" + key]).astype(np.int64).tolist(), key
    assert cols.cpu().tolist() == _np(c["cols"]).astype(np.int64).tolist()
    assert acc.cpu().tolist() == _np(c["accepted"]).astype(np.int64).tolist()
    for i in range(4):
        assert_fp32_close(states[i].cpu(), golden_io.full_after(c, "state", i), what=f"state {i}")
        assert torch.equal(convs[i].cpu(), golden_io.full_after(c, "conv", i)), f"conv {i}"


def test_config0_verify_then_commit_equals_sequential_decode(pkg):
    """BASELINE config 0 end to end: verify + per-context commit == the
    reference (fixture) and == plain sequential decode of the accepted prefix."""
    g = pkg
    c = golden_io.load("config0")
    Q = c["spec_query_len"]
    state = _dev(c["state_before"])
    rec = torch.zeros(_np(c["records"]).shape, device="cuda")
    out = torch.zeros((1,) + tuple(c["v"].shape), device="cuda")
    g.gdn_recoverssm_verify(_dev(c["g"])[None], _dev(c["beta"])[None], _dev(c["q"])[None], _dev(c["k"])[None],
                            _dev(c["v"])[None], checkpoint_state=state, replay_cache=rec,
                            query_start_loc=_dev(c["qsl"]), state_indices=_dev(c["state_indices"]),
                            spec_query_len=Q, out=out)
    conv = torch.zeros(8, 16, 3 + Q - 1, device="cuda")
    ctx = g.GDNRecoverSSMCommitContext.from_tensors([conv], [state], [rec], spec_query_len=Q, max_num_reqs=4)
    ctx.commit(_dev(c["accepted"]), _dev(c["state_indices"]), _dev(c["qsl"]))
    torch.cuda.synchronize()
    assert_fp32_close(out[0].cpu(), c["out"], what="config0 output vs reference")
    assert_fp32_close(rec.cpu(), c["records"], what="config0 records vs reference")
    assert_fp32_close(state.cpu(), golden_io.full_after(c, "state"), what="config0 state vs reference")
    for b in range(4):
        sl = slice(b * Q, (b + 1) * Q)
        for hv in range(4):
            s0 = _np(c["state_before"])[int(c["state_indices"][b]), hv]
            o, _, mids = O.sequential_reference(s0, _np(c["q"])[sl, hv], _np(c["k"])[sl, hv], _np(c["v"])[sl, hv],
                                                _np(c["g"])[sl, hv], _np(c["beta"])[sl, hv], 64**-0.5)
            assert_fp32_close(out[0, sl, hv].cpu(), o, what="output vs sequential")
            a = int(c["accepted"][b])
            assert_fp32_close(state[int(c["state_indices"][b]), hv].cpu(), mids[a - 1], what="state vs sequential")


def test_capi_direct_call_matches_torch_op(pkg):
    """The C ABI called with raw device pointers (ctypes, no torch op) gives
    bit-identical results to the torch-op path."""
    from gdn_recoverssm_b200 import capi

    g = pkg
    c = golden_io.load("verify_packed_bf16_q4")
    out_a, rec_a = _verify_cuda(g, c)
    T, HV, V = c["v"].shape
    H, K = c["q"].shape[1], c["q"].shape[2]
    Q, R = c["spec_query_len"], c["record_rows"]
    q, k, v = _dev(c["q"])[None], _dev(c["k"])[None], _dev(c["v"])[None]
    gg, beta, state = _dev(c["g"]), _dev(c["beta"]), _dev(c["state"])
    qsl, idx = _dev(c["qsl"]), _dev(c["state_indices"])
    out = torch.full((1, T, HV, V), -23.0, dtype=q.dtype, device="cuda")
    rec = torch.full((R, HV, Q, V + K + 1), -17.0, device="cuda")
    B = idx.shape[0]
    config = [B, T, H, HV, Q, state.shape[0], R, 0, q.stride(1), k.stride(1), v.stride(1), gg.stride(0),
              beta.stride(0), *state.stride()[:3], *rec.stride()[:3], *rec.stride()[:3], *rec.stride()[:3],
              out.stride(1), qsl.stride(0), idx.stride(0)]
    capi.verify(q, k, v, gg, beta, state, rec, rec, rec, out, qsl, idx, config, K**-0.5, flags=capi.RECORD_PACKED)
    torch.cuda.synchronize()
    assert torch.equal(out[0].cpu(), out_a)
    assert torch.equal(rec.cpu(), rec_a.cpu())
    status = torch.ops.gdn_recoverssm_ac.device_status()
    assert status == 0


def test_op_rejects_bad_arguments_before_launch(pkg):
    g = pkg
    c = golden_io.load("verify_packed_bf16_q4")
    T, HV, V = c["v"].shape
    bad = torch.zeros(1, T, HV, V, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="spec_query_len"):
        g.gdn_recoverssm_verify(_dev(c["g"]), _dev(c["beta"]), _dev(c["q"])[None], _dev(c["k"])[None],
                                _dev(c["v"])[None], checkpoint_state=_dev(c["state"]),
                                replay_cache=torch.zeros(4, HV, 9, 2 * V + 1, device="cuda"),
                                query_start_loc=_dev(c["qsl"]), state_indices=_dev(c["state_indices"]),
                                spec_query_len=9, out=bad)
    # the torch op itself refuses a config that does not match the tensors
    ops = torch.ops.gdn_recoverssm_ac
    with pytest.raises(RuntimeError, match="GDN RecoverSSM"):
        ops.verify_ext(_dev(c["q"])[None], _dev(c["k"])[None], _dev(c["v"])[None], _dev(c["g"]), _dev(c["beta"]),
                       _dev(c["state"]), bad, bad, bad, bad, _dev(c["qsl"]), _dev(c["state_indices"]),
                       [0] * 28, 1.0, 1)


def test_fold_op_rejects_page_and_record_bounds_past_its_tensors(pkg):
    """The fold bounds pages by config[5] and record rows by config[6]; the
    op refuses values beyond the state pool / records it was given (and rows
    beyond the plan capacity) before any launch."""
    from gdn_recoverssm_b200 import synthetic

    g = pkg
    ops = torch.ops.gdn_recoverssm_ac
    wl = synthetic.make(1, "cuda", seed=4, rows=8, pool=32, conv_dim=8)
    ctx = g.GDNRecoverSSMCommitContext.from_tensors([wl.conv], [wl.state], [wl.records], spec_query_len=wl.Q,
                                                    max_num_reqs=wl.B)
    plan, fold = ctx.make_commit_specs(wl.accepted, wl.state_indices, wl.qsl, commit_conv=False)
    plan.launch()
    before = wl.state.clone()
    for field, value, what in ((5, wl.state.shape[0] + 1, "page bound"), (6, wl.B + 1, "record rows"),
                               (0, wl.B + 1, "plan capacity")):
        cfg = list(fold.args[-2])
        cfg[field] = value
        with pytest.raises(RuntimeError, match="GDN RecoverSSM"):
            ops.fold_ext(*fold.args[:-2], cfg, fold.args[-1])
    torch.cuda.synchronize()
    assert torch.equal(wl.state, before), "a refused fold launched"
    fold.launch()
    torch.cuda.synchronize()
    assert not torch.equal(wl.state, before)


@pytest.mark.parametrize("act", [torch.bfloat16, torch.float16])
def test_reference_schema_ops_match_the_extended_ops(pkg, act):
    """The drop-ins for the reference's native ops -- gdn_recoverssm_ac::verify
    and ::fold with their exact schemas (typed records, no flags; what the
    reference's AscendC backend calls) -- give bit-identical results to the
    extended ops the Python layer launches; the fold of typed records with
    bf16 / fp16 key planes matches the float64 oracle."""
    from gdn_recoverssm_b200 import synthetic

    g = pkg
    ops = torch.ops.gdn_recoverssm_ac
    wl = synthetic.make(1, "cuda", seed=21, rows=8, pool=32, conv_dim=8)
    q, k, v = wl.q.to(act), wl.k.to(act), wl.v.to(act)
    H, HV, D, Q, B = wl.H, wl.HV, wl.D, wl.Q, wl.B
    results = []
    for reference_schema in (False, True):
        state = wl.state.clone()
        rec = g.ReplayRecordBuffers.allocate(B, HV, H, Q, D, D, device="cuda", key_dtype=act)
        out = torch.zeros(wl.out.shape, dtype=act, device="cuda")
        specs = []
        g.gdn_recoverssm_verify(wl.g, wl.beta, q, k, v, checkpoint_state=state, replay_cache=rec,
                                query_start_loc=wl.qsl, state_indices=wl.state_indices, spec_query_len=Q, out=out,
                                _collect=specs)
        (spec,) = specs
        assert spec.args[-1] == 0  # typed records, pre-normalised q/k: the reference's own op applies
        if reference_schema:
            ops.verify(*spec.args[:-1])
        else:
            spec.launch()
        conv = torch.zeros(wl.state.shape[0], 8, 3 + Q - 1, dtype=act, device="cuda")
        ctx = g.GDNRecoverSSMCommitContext.from_tensors([conv], [state], [rec], spec_query_len=Q, max_num_reqs=B)
        cspecs = ctx.make_commit_specs(wl.accepted, wl.state_indices, wl.qsl, commit_conv=False)
        plan, fold = cspecs[0], cspecs[-1]
        plan.launch()
        assert fold.args[-1] == 0
        if reference_schema:
            ops.fold(*fold.args[:-1])
        else:
            fold.launch()
        torch.cuda.synchronize()
        results.append((out.cpu(), rec.correction.cpu(), rec.key.cpu(), rec.decay.cpu(), state.cpu()))
    for a, b in zip(*results):
        assert torch.equal(a, b)
    assert int(ops.device_status()) == 0
    # the fold of the typed records (key planes in the activation dtype) against the oracle
    _, corr, key, decay, got = results[1]
    want = [wl.state.double().cpu().numpy()]
    O.fold(want, [corr.numpy()], [key.float().numpy()], [decay.numpy()], layer_groups=[0],
           plan_capacity=ctx.commit_lens.shape[0], rows=B, source=wl.state_indices.cpu().numpy(),
           lengths=ctx.commit_lens.cpu().numpy(), finals=ctx.final_state_indices.cpu().numpy(),
           boundaries=ctx.boundary_state_indices.cpu().numpy(), boundary_lens=ctx.boundary_recovery_lens.cpu().numpy(),
           num_blocks=wl.state.shape[0], record_rows=B, layout="soa", query_len=Q)
    assert_fp32_close(got.double().numpy(), want[0], what="typed-record fold")
