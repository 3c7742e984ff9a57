"""CPU pins of the float64 torch restatement (tests/torch_reference.py) that the
full-size GPU parity tests use as their checker: on small cases with every
masking rule (ragged and empty windows, a window running past the last
token, null / negative / out-of-pool slots, GQA, in-kernel normalisation) it
must equal the NumPy oracle (oracle.gdn_oracle.verify_batch / commit), which is
itself pinned to the reference's known answers and Triton fixtures."""

import numpy as np
import pytest
import torch

from oracle import gdn_oracle as O
from tests import golden_io
from tests.torch_reference import rel_errors_per_unit, rounded_ok, verify_rows


def _case(seed, Q, H, HV, D=16, rows=10, blocks=14, normalize=False):
    rng = np.random.default_rng(seed)
    qlen = rng.integers(0, Q + 1, rows)
    qlen[0], qlen[1] = Q, 0
    qsl = np.concatenate([[0], np.cumsum(qlen)]).astype(np.int32)
    T = max(int(qsl[-1]) - 1, 1)  # the last row's final token lies past T
    slots = rng.permutation(np.arange(1, blocks))[:rows].astype(np.int32)
    slots[2], slots[3], slots[4] = 0, blocks, -1
    q = rng.standard_normal((T, H, D))
    k = rng.standard_normal((T, H, D))
    if not normalize:
        q /= np.linalg.norm(q, axis=-1, keepdims=True)
        k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((T, HV, D))
    g = -np.log1p(np.exp(rng.standard_normal((T, HV))))
    beta = 1.0 / (1.0 + np.exp(-rng.standard_normal((T, HV))))
    state = rng.standard_normal((blocks, HV, D, D)) * 0.1
    return q, k, v, g, beta, state, qsl, slots


@pytest.mark.parametrize("Q,H,HV,normalize", [(1, 2, 4, False), (3, 1, 3, True), (4, 2, 4, False), (8, 2, 2, True)])
def test_torch_reference_equals_numpy_oracle(Q, H, HV, normalize):
    q, k, v, g, beta, state, qsl, slots = _case(7 + Q, Q, H, HV, normalize=normalize)
    T, _, D = q.shape
    rows = len(slots)
    o_out = np.full((T, HV, D), np.nan)
    o_rec = np.full((rows, HV, Q, 2 * D + 1), np.nan)
    O.verify_batch(q, k, v, g, beta, state, qsl, slots, spec_query_len=Q, normalize_qk=normalize, out=o_out,
                   records=o_rec, record_rows=rows)
    lens = torch.tensor(np.minimum(np.maximum(np.diff(qsl), 0), Q) // 2, dtype=torch.int64)
    t = lambda x: torch.tensor(x)  # noqa: E731
    res = verify_rows(t(q), t(k), t(v), t(g), t(beta), t(state), t(qsl), t(slots), Q=Q, normalize=normalize,
                      capture={"half": lens})
    # outputs: scatter the window positions back to tokens
    got_out = np.full((T, HV, D), np.nan)
    tok, valid = res["token"].numpy(), res["valid"].numpy()
    for r in range(rows):
        for s in range(Q):
            if valid[r, s]:
                got_out[tok[r, s]] = res["out"][r, s].numpy()
    assert np.array_equal(np.isnan(got_out), np.isnan(o_out))
    m = ~np.isnan(o_out)
    assert np.allclose(got_out[m], o_out[m], rtol=1e-12, atol=1e-12)
    rec = res["records"].numpy()
    assert np.array_equal(np.isnan(rec), np.isnan(o_rec))
    m = ~np.isnan(o_rec)
    assert np.allclose(rec[m], o_rec[m], rtol=1e-12, atol=1e-12)
    # captured prefix states equal the oracle's fold of its own records
    for r in range(rows):
        if not res["live"][r]:
            continue
        for hv in range(HV):
            want = O.commit(state[slots[r], hv], o_rec[r, hv], int(lens[r]))
            assert np.allclose(res["half"][r, hv].numpy(), want, rtol=1e-12, atol=1e-12)


def test_torch_reference_row_ranges_agree_with_the_whole_batch():
    q, k, v, g, beta, state, qsl, slots = _case(3, 4, 2, 4)
    t = lambda x: torch.tensor(x)  # noqa: E731
    whole = verify_rows(t(q), t(k), t(v), t(g), t(beta), t(state), t(qsl), t(slots), Q=4)
    a = verify_rows(t(q), t(k), t(v), t(g), t(beta), t(state), t(qsl), t(slots), Q=4, rows=(0, 4))
    b = verify_rows(t(q), t(k), t(v), t(g), t(beta), t(state), t(qsl), t(slots), Q=4, rows=(4, len(slots)))
    for key in ("out", "records"):
        assert torch.equal(torch.cat([a[key], b[key]]).nan_to_num(7.0), whole[key].nan_to_num(7.0))


def test_torch_reference_matches_reference_triton_fixture():
    """The packed fp32 in-kernel-L2 verify fixture produced by the reference's
    own Triton kernels."""
    c = golden_io.load("verify_packed_fp32_l2_q3")
    Q = int(c["spec_query_len"])
    res = verify_rows(c["q"].double(), c["k"].double(), c["v"].double(), c["g"], c["beta"], c["state"], c["qsl"],
                      c["state_indices"], Q=Q, normalize=not bool(c["normalized"]))
    out = c["out"].double()
    tok, valid = res["token"], res["valid"]
    R = c["records"].shape[0]
    for r in range(len(c["state_indices"])):
        for s in range(Q):
            if valid[r, s]:
                want = res["out"][r, s]
                assert float(rel_errors_per_unit(out[tok[r, s]], want, 2)[0]) < 2e-6
    rec = res["records"][:R]
    stored = ~torch.isnan(rec)
    emax, _ = rel_errors_per_unit(c["records"].double(), rec, 2)
    assert stored.any() and float(emax.max()) < 2e-6


def test_rounded_ok_accepts_one_ulp_and_rejects_two():
    want = torch.tensor([[1.0, 3.0, -0.5, float("nan")]], dtype=torch.float64)
    one = want.clone()
    one[0, 1] = 3.0 + 2.0 ** -6  # one bf16 ulp at 3.0 (exponent 1, 7 mantissa bits)
    assert bool(rounded_ok(one.nan_to_num(0.0), want, 7, -126).all())
    two = want.clone()
    two[0, 1] = 3.0 + 2.0 ** -5
    assert not bool(rounded_ok(two.nan_to_num(0.0), want, 7, -126).all())
