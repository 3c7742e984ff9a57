"""Pin the CPU oracle before trusting it (CPU only).

Two kinds of evidence:

* the reference test-suite's known answers, restated here as values
  (plugin/tests/test_math_oracle.py, test_ascendc_selftest_oracle.py,
  test_grouped_commit.py);
* fixtures produced by running the reference's own Triton kernels
  (``tests/golden/make_golden.py``): verify outputs/records, per-context and
  grouped plans (bit-exact), folded states and compacted conv windows.
"""

import numpy as np
import pytest
import torch

from oracle import gdn_oracle as O
from tests import golden_io

RTOL = 1e-9


def _case(seed=0, T=4, V=8, K=8):
    rng = np.random.default_rng(seed)
    s0 = rng.standard_normal((V, K)) * 0.5
    q = rng.standard_normal((T, K))
    k = rng.standard_normal((T, K))
    v = rng.standard_normal((T, V))
    a = rng.standard_normal(T) * 0.5
    beta = 1.0 / (1.0 + np.exp(-rng.standard_normal(T)))
    return s0, q, k, v, O.gdn_gate(0.3, -0.1, a), beta


# ---- test_math_oracle.py known answers ------------------------------------ #
def test_verify_matches_sequential_and_checkpoint_is_read_only():
    s0, q, k, v, g, beta = _case(T=5)
    scale = k.shape[-1] ** -0.5
    ref_out, _, _ = O.sequential_reference(s0, q, k, v, g, beta, scale)
    keep = s0.copy()
    out, _ = O.verify_records(s0, q, k, v, g, beta, scale)
    np.testing.assert_allclose(out, ref_out, rtol=RTOL, atol=RTOL)
    np.testing.assert_array_equal(s0, keep)


def test_commit_every_accept_length_and_zero_is_identity():
    s0, q, k, v, g, beta = _case(T=5)
    scale = k.shape[-1] ** -0.5
    _, _, mids = O.sequential_reference(s0, q, k, v, g, beta, scale)
    _, recs = O.verify_records(s0, q, k, v, g, beta, scale)
    np.testing.assert_array_equal(O.commit(s0, recs, 0), s0)
    for a in range(1, 6):
        np.testing.assert_allclose(O.commit(s0, recs, a), mids[a - 1], rtol=RTOL, atol=RTOL)


def test_record_layout_is_corr_key_decay():
    s0, q, k, v, g, beta = _case(T=3, V=5, K=7)
    _, recs = O.verify_records(s0, q, k, v, g, beta, 7**-0.5)
    assert recs.shape == (3, 5 + 7 + 1)
    np.testing.assert_allclose(recs[:, 12], np.exp(g), rtol=RTOL)
    np.testing.assert_allclose(recs[:, 5:12], O.l2_unit(k), rtol=RTOL)


def test_commit_plan_known_answers():
    # test_math_oracle.py:238-250
    assert O.commit_plan(128, 128, 3, 8) == (1, None, 0)
    assert O.commit_plan(127, 128, 1, 8) == (0, 0, 1)
    assert O.commit_plan(127, 128, 0, 8) == (0, None, 0)
    assert O.commit_plan(126, 128, 4, 8) == (1, 0, 2)
    assert O.commit_plan(128 * 8, 128, 4, 8) == (7, None, 0)


@pytest.mark.parametrize("computed,accepted", [(124, 4), (125, 3), (126, 2), (127, 1), (128, 1), (255, 1)])
def test_commit_destination_is_allocated(computed, accepted):
    # test_math_oracle.py:180-203
    col, _, _ = O.commit_plan(computed, 128, accepted, 8)
    assert col <= max(-(-(computed + accepted) // 128) - 1, 0)


def test_single_pass_boundary_known_answer():
    # test_math_oracle.py:206-235: h <- 0.5 h + 1 from 10: 6, 4, 3; the wrong
    # two-pass shape gives 2.25.
    recs = np.array([[1.0, 1.0, 0.5]] * 3)
    s0 = np.array([[10.0]])
    assert O.commit(s0, recs, 3)[0, 0] == pytest.approx(3.0, abs=1e-12)
    assert O.commit(s0, recs, 2)[0, 0] == pytest.approx(4.0, abs=1e-12)
    assert O.commit(np.array([[3.0]]), recs, 2)[0, 0] == pytest.approx(2.25, abs=1e-12)
    # the same through the launch-level fold: final page 1, boundary page 2
    recs_p = np.array([[[[1.0, 1.0, 0.5]] * 3]])  # [R=1, HV=1, Q=3, 3]
    pool = np.zeros((4, 1, 1, 1))
    pool[1] = 10.0
    O.fold([pool], [recs_p], None, None, layer_groups=[0], plan_capacity=1, rows=1,
           source=[1], lengths=[3], finals=[1], boundaries=[2], boundary_lens=[2],
           num_blocks=4, record_rows=1)
    assert pool[1, 0, 0, 0] == pytest.approx(3.0) and pool[2, 0, 0, 0] == pytest.approx(4.0)


def test_non_square_commit():
    rng = np.random.default_rng(7)
    V, K = 5, 7
    h0 = rng.standard_normal((V, K))
    recs = rng.standard_normal((4, V + K + 1))
    recs[:, V + K] = rng.random(4) * 0.5
    ref = h0.copy()
    for t in range(3):
        ref = ref * recs[t, V + K] + np.outer(recs[t, :V], recs[t, V : V + K])
    np.testing.assert_allclose(O.commit(h0, recs, 3), ref, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("C,A,expected", [(126, 1, 0), (127, 1, 0), (128, 1, 1), (124, 4, 0), (255, 1, 1)])
def test_running_column_follows_commit_target(C, A, expected):
    # test_math_oracle.py:310-330
    assert O.commit_plan(C, 128, A, 64)[0] == expected


# ---- test_ascendc_selftest_oracle.py hand-computed answers ---------------- #
def test_hand_computed_prefixes():
    # three value heads sharing one key head, 2x2 states, zero checkpoint
    q = np.array([[1.0, 0.0], [0.0, 1.0]])
    v = np.array([[1.0, 2.0], [3.0, 4.0]])
    outs = []
    for hv in range(3):
        o, _, mids = O.sequential_reference(np.zeros((2, 2)), q, q, v, np.zeros(2), np.full(2, 0.5), 1.0)
        outs.append(o)
        np.testing.assert_array_equal(mids[0][:, 0], [0.5, 1.0])
        np.testing.assert_array_equal(mids[0][:, 1], [0.0, 0.0])
        np.testing.assert_array_equal(mids[1][:, 1], [1.5, 2.0])
    np.testing.assert_array_equal(outs[0], [[0.5, 1.0], [1.5, 2.0]])


def test_hand_computed_fold():
    # fold_reference: ones checkpoint, keys e0/e1, corr [[2,4],[6,8]], decay 0.5
    recs = np.array([[2.0, 4.0, 1.0, 0.0, 0.5], [6.0, 8.0, 0.0, 1.0, 0.5]])
    got = O.commit(np.ones((2, 2)), recs, 2)
    np.testing.assert_array_equal(got, [[1.25, 6.25], [2.25, 8.25]])


# ---- test_grouped_commit.py plan goldens ---------------------------------- #
def _grouped_groups(n, sources_per_group=None, blocks=64):
    groups = []
    for g in range(n):
        src = (8, 4) if sources_per_group is None else sources_per_group[g]
        bt = np.array([[2, 3, 4, 5], [6, 7, 8, 9], [10, 11, 12, 13]]) + g * 20
        groups.append(dict(
            state_indices=np.array(src), query_start_loc=np.array([0, 4, 8]),
            request_indices=np.array([2, 0]), block_table=bt,
            num_computed=np.array([3, 0, 7]), block_size=4,
            num_blocks=blocks if np.isscalar(blocks) else blocks[g],
        ))
    return groups


def _run_grouped(groups, align=True, sampled=(1, 0, 3), mapping=(5, -1, 1)):
    cols = np.full(6, -9)
    acc = np.full(6, 7)
    plan = O.grouped_plan(np.array(sampled), groups, rows=2, plan_capacity=8, spec_query_len=4,
                          align=align, publish=True, idx_mapping=np.array(mapping),
                          persistent_cols=cols, persistent_accepted=acc)
    return plan, cols, acc


def test_grouped_plan_goldens():
    plan, cols, acc = _run_grouped(_grouped_groups(3))
    for g in range(3):
        s = g * 8
        assert plan["final"][s : s + 2].tolist() == [12 + 20 * g, 2 + 20 * g]
        assert plan["boundary"][s] == 11 + 20 * g
        assert plan["boundary_len"][s] == 1
        assert plan["length"][s : s + 2].tolist() == [3, 1]
    assert cols.tolist() == [-9, 2, -9, -9, -9, 0]
    assert acc.tolist() == [7, 1, 7, 7, 7, 1]


def test_invalid_group_cannot_publish():
    plan, cols, acc = _run_grouped(_grouped_groups(2, [(8, 4), (0, 9)]))
    assert plan["length"][8] == 0
    assert cols[1] == -9 and acc[1] == 7
    assert cols[5] == 0 and acc[5] == 1


def test_none_plan_never_publishes():
    plan, cols, acc = _run_grouped(_grouped_groups(1), align=False)
    assert plan["final"][:2].tolist() == [8, 4]
    assert plan["length"][:2].tolist() == [3, 1]
    assert acc.tolist() == [7] * 6


def test_zero_acceptance_and_finished_slots():
    plan, cols, acc = _run_grouped(_grouped_groups(1), sampled=(0, 0, 0), mapping=(-1, -1, -1))
    assert plan["length"][:2].tolist() == [0, 0]
    assert cols.tolist() == [-9] * 6 and acc.tolist() == [7] * 6


def test_group_local_invalid_boundary_is_canonicalised():
    groups = _grouped_groups(2, blocks=[16, 64])
    groups[0]["block_table"][2, 1] = 32  # invalid only in the small pool
    plan, _, _ = _run_grouped(groups)
    assert plan["final"][0] == 12
    assert plan["boundary"][0] == 0 and plan["boundary_len"][0] == 0
    assert plan["boundary"][8] == 31


# ---- reference-Triton fixtures -------------------------------------------- #
VERIFY_CASES = [
    "verify_packed_bf16_q4",
    "verify_soa_bf16_q4",
    "verify_packed_fp32_l2_q3",
    "verify_soa_fp32_l2_q8",
    "verify_packed_bf16_q1",
]


def _np(t):
    return t.double().numpy() if isinstance(t, torch.Tensor) else np.asarray(t)


def oracle_verify_from_fixture(c):
    """Run the oracle on a verify fixture's inputs with sentinel-filled outputs."""
    T, HV, V = c["v"].shape
    H, K = c["q"].shape[1], c["q"].shape[2]
    Q, R = c["spec_query_len"], c["record_rows"]
    out = np.full((T, HV, V), -23.0)
    if c["layout"] == "packed":
        recs = np.full((R, HV, Q, V + K + 1), -17.0)
    else:
        recs = (np.full((R, HV, Q, V), -17.0), np.full((R, H, Q, K), -16.0), np.full((R, HV, Q), -19.0))
    O.verify_batch(_np(c["q"]), _np(c["k"]), _np(c["v"]), _np(c["g"]), _np(c["beta"]), _np(c["state"]),
                   c["qsl"], c["state_indices"], spec_query_len=Q, normalize_qk=not c["normalized"],
                   record_rows=R, layout=c["layout"], out=out, records=recs)
    return out, recs


@pytest.mark.parametrize("name", VERIFY_CASES)
def test_oracle_matches_reference_triton_verify(name):
    c = golden_io.load(name)
    out, recs = oracle_verify_from_fixture(c)
    ref_out = _np(c["out"])
    if c["out"].dtype == torch.bfloat16:
        # Triton's CPU interpreter truncates fp32 -> bf16 where the device rounds
        # to nearest, so the fixture is only pinned to one bf16 ulp here.
        ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(ref_out), 1e-30))) - 7)
        assert np.all(np.abs(out - ref_out) <= ulp * 1.01)
    else:
        assert max(O.rel_errors(out, ref_out)) < 1e-5
    # sentinels must match exactly (null rows, padding, rows past record_rows)
    if c["layout"] == "packed":
        ref_r = _np(c["records"])
        assert np.array_equal(ref_r == -17.0, recs == -17.0)
        assert max(O.rel_errors(recs, ref_r)) < 1e-5
    else:
        for mine, key, sentinel in zip(recs, ("corr", "key", "decay"), (-17.0, -16.0, -19.0)):
            ref_r = _np(c[key])
            assert np.array_equal(ref_r == sentinel, mine == sentinel), key
            assert max(O.rel_errors(mine, ref_r)) < 1e-5, key
        if c["normalized"]:
            # pre-normalised low-precision keys keep their exact input bits
            assert np.array_equal(recs[1][recs[1] != -16.0], _np(c["key"])[recs[1] != -16.0])


CONTEXT_CASES = [
    "context_commit_none_packed", "context_commit_align_packed", "context_commit_align_soa", "context_plan_int32",
]


def oracle_context_commit(c):
    """Oracle run of plan -> conv -> fold for a per-context commit fixture."""
    align = bool(c["align"])
    rows = len(c["src"])
    nb = c["state_before0"].shape[0]
    plan = O.prepare_commit_plan(
        c["accepted"], c["src"], c["qsl"], spec_query_len=c["spec_query_len"], num_blocks=nb,
        request_indices=c["request_indices"],
        block_table=c.get("block_table") if align else None,
        num_computed=c.get("num_computed") if align else None,
        block_size=c.get("block_size") if align else None,
    )
    layers = int(c["layers"])
    states = [_np(c[f"state_before{i}"]).astype(np.float32) for i in range(layers)]
    convs = [_np(c[f"conv_before{i}"]).astype(np.float32) for i in range(layers)]
    if c["layout"] == "packed":
        recs = ([_np(c[f"records{i}"]) for i in range(layers)], None, None)
    else:
        recs = tuple([_np(c[f"{n}{i}"]) for i in range(layers)] for n in ("corr", "key", "decay"))
    common = dict(layer_groups=[0] * layers, plan_capacity=rows, rows=rows, source=np.asarray(c["src"]),
                  lengths=plan["commit_lens"], finals=plan["final"], boundaries=plan["boundary"],
                  boundary_lens=plan["boundary_lens"], num_blocks=nb)
    O.compact_conv(convs, history=c["history"], align=align, **common)
    O.fold(states, *recs, record_rows=rows, layout=c["layout"], query_len=c["spec_query_len"], **common)
    return plan, states, convs


@pytest.mark.parametrize("name", CONTEXT_CASES)
def test_oracle_matches_reference_triton_context_commit(name):
    c = golden_io.load(name)
    plan, states, convs = oracle_context_commit(c)
    for key in ("commit_lens", "final", "boundary", "boundary_lens", "valid", "col"):
        assert plan[key].tolist() == _np(c[key]).astype(np.int64).tolist(), key
    for i in range(int(c["layers"])):
        want = golden_io.full_after(c, "state", i).double().numpy()
        assert max(O.rel_errors(states[i], want)) < 1e-6
        assert np.array_equal(convs[i], golden_io.full_after(c, "conv", i).numpy())


def oracle_grouped(c):
    groups = []
    for g in range(2):
        groups.append(dict(
            state_indices=_np(c[f"state_indices{g}"]).astype(np.int64), query_start_loc=_np(c["qsl"]).astype(np.int64),
            request_indices=_np(c["request_indices"]).astype(np.int64), block_table=_np(c[f"block_table{g}"]).astype(np.int64),
            num_computed=_np(c["computed"]).astype(np.int64), block_size=c["block_size"], num_blocks=c["num_blocks"],
        ))
    cols = np.full(6, -9)
    acc = np.full(6, 7)
    rows = len(c["request_indices"])
    plan = O.grouped_plan(_np(c["sampled"]), groups, rows=rows, plan_capacity=c["capacity"],
                          spec_query_len=c["spec_query_len"], align=True, publish=True,
                          idx_mapping=_np(c["mapping"]), persistent_cols=cols, persistent_accepted=acc)
    states = [_np(c[f"state_before{i}"]).astype(np.float32) for i in range(4)]
    convs = [_np(c[f"conv_before{i}"]).astype(np.float32) for i in range(4)]
    recs = tuple([_np(c[f"{n}{i}"]) for i in range(4)] for n in ("corr", "key", "decay"))
    common = dict(layer_groups=_np(c["layer_groups"]), plan_capacity=c["capacity"], rows=rows,
                  source=plan["source"], lengths=plan["length"], finals=plan["final"],
                  boundaries=plan["boundary"], boundary_lens=plan["boundary_len"], num_blocks=c["num_blocks"])
    O.compact_conv(convs, history=c["history"], align=True, **common)
    O.fold(states, *recs, record_rows=c["capacity"], layout="soa", query_len=c["spec_query_len"], **common)
    return plan, cols, acc, states, convs


def test_oracle_matches_reference_triton_grouped_commit():
    c = golden_io.load("grouped_align_soa")
    plan, cols, acc, states, convs = oracle_grouped(c)
    for key in ("source", "length", "final", "boundary", "boundary_len", "valid", "col"):
        assert plan[key].tolist() == _np(c["plan_" + key]).astype(np.int64).tolist(), key
    assert cols.tolist() == _np(c["cols"]).astype(np.int64).tolist()
    assert acc.tolist() == _np(c["accepted"]).astype(np.int64).tolist()
    for i in range(4):
        assert max(O.rel_errors(states[i], golden_io.full_after(c, "state", i).double().numpy())) < 1e-6
        assert np.array_equal(convs[i], golden_io.full_after(c, "conv", i).numpy())


def test_config0_verify_and_commit_match_reference():
    c = golden_io.load("config0")
    Q = c["spec_query_len"]
    out, recs = O.verify_batch(_np(c["q"]), _np(c["k"]), _np(c["v"]), _np(c["g"]), _np(c["beta"]),
                               _np(c["state_before"]), c["qsl"], c["state_indices"], spec_query_len=Q,
                               records=np.zeros(_np(c["records"]).shape))
    assert max(O.rel_errors(out, _np(c["out"]))) < 1e-5
    assert max(O.rel_errors(recs, _np(c["records"]))) < 1e-5
    # and each unit equals the test_math_oracle semantics (sequential decode)
    for b in range(4):
        for hv in range(4):
            sl = slice(b * Q, (b + 1) * Q)
            s0 = _np(c["state_before"])[int(c["state_indices"][b]), hv]
            o, _, mids = O.sequential_reference(s0, _np(c["q"])[sl, hv], _np(c["k"])[sl, hv], _np(c["v"])[sl, hv],
                                                _np(c["g"])[sl, hv], _np(c["beta"])[sl, hv], 64**-0.5)
            assert max(O.rel_errors(out[sl, hv], o)) < 1e-6
            a = int(c["accepted"][b])
            want = golden_io.full_after(c, "state")[int(c["state_indices"][b]), hv].double().numpy()
            assert max(O.rel_errors(mids[a - 1], want)) < 1e-5
