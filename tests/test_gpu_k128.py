"""GPU parity of verify at the production head size K = V = 128.

With an fp32 state pool this shape runs the tensor-core kernel (tcgen05 MMAs
on a three-product tf32 split of S and X); with a bf16 pool the CUDA-core
kernel.  Every case is checked element by element against the float64 oracle
(oracle.gdn_oracle.verify_batch), with the edge cases the reference kernel
masks: ragged windows (qlen 0 .. Q), a window running past the last token,
null / negative / out-of-pool slots, rows past ``record_rows``, GQA, packed and
typed records, in-kernel q/k normalisation, every window template (Q = 1, 2,
3..4, 5..8) and every activation dtype.  State values carry all 23 mantissa
bits and span four decades, so a tf32 product that lost its low part would
miss the 1e-5 bound by two orders of magnitude.
"""

import numpy as np
import pytest
import torch

from oracle import gdn_oracle as O
from tests.test_gpu_parity import assert_fp32_close

pytestmark = pytest.mark.gpu
D = 128

CASES = [
    # Q, activation, record layout, normalise in kernel, H, HV, state dtype
    (1, torch.bfloat16, "packed", False, 2, 4, torch.float32),
    (2, torch.bfloat16, "soa", True, 2, 4, torch.float32),
    (3, torch.float32, "packed", True, 2, 4, torch.float32),
    (4, torch.bfloat16, "packed", False, 2, 4, torch.float32),
    (4, torch.float16, "soa", False, 1, 4, torch.float32),
    (5, torch.bfloat16, "packed", True, 2, 4, torch.float32),
    (8, torch.bfloat16, "soa", False, 2, 4, torch.float32),
    (8, torch.float32, "packed", False, 4, 4, torch.float32),
    (7, torch.float16, "packed", True, 2, 4, torch.float32),
    (6, torch.bfloat16, "soa", True, 1, 4, torch.float32),
    (4, torch.bfloat16, "packed", False, 2, 4, torch.bfloat16),
    # exact operands with a window shorter than the instantiation's (Q = 3 on
    # the 4-token kernel, Q = 6 on the 8-token one): the tokens past Q are
    # masked through the mask-free correction chain
    (3, torch.bfloat16, "packed", False, 2, 4, torch.float32),
    (6, torch.bfloat16, "packed", False, 1, 4, torch.float32),
    # fp16 exact operands at Q = 8: activations staged in shared memory
    (8, torch.float16, "packed", False, 2, 4, torch.float32),
]


@pytest.fixture(scope="module")
def pkg():
    import gdn_recoverssm_b200 as g
    from gdn_recoverssm_b200 import _native

    _native.ops()
    return g


def _case(seed, Q, act, H, HV, state_dtype, normalize, rows=12, blocks=16):
    rng = np.random.default_rng(seed)
    qlen = rng.integers(0, Q + 1, rows)
    qlen[0], qlen[1] = Q, 0
    qsl = np.concatenate([[0], np.cumsum(qlen)]).astype(np.int32)
    T = max(int(qsl[-1]) - 1, 1)  # the last row's final token lies past T: masked
    slots = rng.permutation(np.arange(1, blocks))[:rows].astype(np.int32)
    slots[2], slots[3], slots[4] = 0, blocks, -1  # null, out of pool, negative
    q = rng.standard_normal((T, H, D))
    k = rng.standard_normal((T, H, D))
    if not normalize:
        q /= np.linalg.norm(q, axis=-1, keepdims=True)
        k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((T, HV, D))
    g = -np.log1p(np.exp(rng.standard_normal((T, HV))))
    beta = 1.0 / (1.0 + np.exp(-rng.standard_normal((T, HV))))
    scale_rows = 10.0 ** rng.uniform(-2, 2, (blocks, HV, D, 1))
    state = rng.standard_normal((blocks, HV, D, D)) * 0.1 * scale_rows
    t = dict(
        q=torch.tensor(q, dtype=act), k=torch.tensor(k, dtype=act), v=torch.tensor(v, dtype=act),
        g=torch.tensor(g, dtype=torch.float32), beta=torch.tensor(beta, dtype=torch.float32),
        state=torch.tensor(state, dtype=torch.float32).to(state_dtype),
        qsl=torch.tensor(qsl), slots=torch.tensor(slots),
    )
    return t


def _assert_rounded_close(got, want, mantissa_bits, min_normal_exp, what):
    """[T, HV, V] low-precision outputs: each element within one ulp of the
    float64 oracle value (subnormal ulp below the normal range), or within
    the fp32 tolerance (1e-5) of its (token, head) output vector's largest
    magnitude -- the floor for near-zero outputs of a cancelling 128-term sum,
    which no fp32 computation pins to the ulp of the result."""
    live = want != -23.0
    expo = np.maximum(np.floor(np.log2(np.maximum(np.abs(want), 1e-300))), min_normal_exp)
    ulp = np.exp2(expo - mantissa_bits)
    vmax = np.abs(np.where(live, want, 0.0)).max(axis=-1, keepdims=True)
    ok = (np.abs(got - want) <= ulp * 1.01) | (np.abs(got - want) <= 1e-5 * vmax)
    assert np.all(ok | ~live), f"{what}: {int((~ok & live).sum())} elements off"


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"Q{c[0]}-{str(c[1])[6:]}-{c[2]}-n{int(c[3])}-H{c[4]}-{str(c[6])[6:]}")
def test_verify_k128_matches_oracle(pkg, case):
    Q, act, layout, normalize, H, HV, state_dtype = case
    c = _case(1234 + Q, Q, act, H, HV, state_dtype, normalize)
    T = c["q"].shape[0]
    rows = c["slots"].shape[0]
    R = rows - 2  # the last two rows have no record row
    dev = {n: x.cuda() for n, x in c.items()}
    out = torch.full((1, T, HV, D), -23.0, dtype=act, device="cuda")
    if layout == "packed":
        cache = torch.full((R, HV, Q, 2 * D + 1), -17.0, device="cuda")
    else:
        kd = torch.float32 if normalize else act
        cache = pkg.ReplayRecordBuffers(
            torch.full((R, HV, Q, D), -17.0, device="cuda"),
            torch.full((R, H, Q, D), -16.0, dtype=kd, device="cuda"),
            torch.full((R, HV, Q), -19.0, device="cuda"),
        )
    before = dev["state"].clone()
    pkg.gdn_recoverssm_verify(
        dev["g"][None], dev["beta"][None], dev["q"][None], dev["k"][None], dev["v"][None],
        checkpoint_state=dev["state"], replay_cache=cache, query_start_loc=dev["qsl"], state_indices=dev["slots"],
        spec_query_len=Q, qk_already_normalized=not normalize, out=out,
    )
    torch.cuda.synchronize()
    assert torch.equal(dev["state"], before), "verify modified the read-only checkpoint"
    assert int(torch.ops.gdn_recoverssm_ac.device_status()) == 0

    f64 = lambda x: x.double().numpy()
    o_out = np.full((T, HV, D), -23.0)
    if layout == "packed":
        o_rec = np.full((R, HV, Q, 2 * D + 1), -17.0)
    else:
        o_rec = (np.full((R, HV, Q, D), -17.0), np.full((R, H, Q, D), -16.0), np.full((R, HV, Q), -19.0))
    O.verify_batch(f64(c["q"]), f64(c["k"]), f64(c["v"]), f64(c["g"]), f64(c["beta"]), f64(c["state"]),
                   c["qsl"].numpy(), c["slots"].numpy(), spec_query_len=Q, normalize_qk=normalize, record_rows=R,
                   layout=layout, out=o_out, records=o_rec)

    got = out[0].double().cpu().numpy()
    assert np.array_equal(got == -23.0, o_out == -23.0), "output store mask"
    live = o_out != -23.0
    if act == torch.float32:
        assert_fp32_close(got[live], o_out[live], what="output")
    elif act == torch.bfloat16:
        _assert_rounded_close(got, o_out, 7, -126, "bf16 output")
    else:
        _assert_rounded_close(got, o_out, 10, -14, "f16 output")
    if layout == "packed":
        rec = cache.double().cpu().numpy()
        assert np.array_equal(rec == -17.0, o_rec == -17.0), "record store mask"
        m = o_rec != -17.0
        assert_fp32_close(rec[m], o_rec[m], what="packed records")
    else:
        for got_t, want, sentinel, name in zip((cache.correction, cache.key, cache.decay), o_rec, (-17.0, -16.0, -19.0),
                                              ("correction", "key", "decay")):
            g_np = got_t.double().cpu().numpy()
            assert np.array_equal(g_np == sentinel, want == sentinel), f"{name} store mask"
            m = want != sentinel
            if name == "key" and not normalize:
                assert np.array_equal(g_np[m], want[m]), "pre-normalised keys keep their input bits"
            else:
                assert_fp32_close(g_np[m], want[m], what=name)


@pytest.mark.parametrize("Q", [4, 8])
def test_verify_k128_long_walks_alternating_live_and_null_rows(pkg, Q):
    """Many units per CTA (2048 rows x 8 value heads over the persistent
    grid, ~37 units per CTA at Q = 4, ~55 at Q = 8) with live, null, negative
    and out-of-pool slots and empty windows interleaved at random, so that
    every CTA's walk switches between its live and null paths many times (at
    Q = 8 the next unit's rows are staged in shared memory, refilled across
    those switches): every unit's outputs and records against the float64
    restatement, null rows' outputs zero and their records untouched."""
    from tests.torch_reference import rel_errors_per_unit, rounded_ok, verify_rows

    B, H, HV, blocks = 2048, 2, 8, 64
    gen = torch.Generator().manual_seed(77)
    kind = torch.randint(0, 10, (B,), generator=gen)
    slots = 1 + torch.randint(0, blocks - 1, (B,), generator=gen)
    slots = torch.where(kind < 3, torch.zeros_like(slots), slots)  # null
    slots = torch.where(kind == 3, torch.full_like(slots, blocks), slots)  # out of pool
    slots = torch.where(kind == 4, torch.full_like(slots, -2), slots)  # negative
    qlen = torch.randint(0, Q + 1, (B,), generator=gen)
    qlen = torch.where(kind == 5, torch.zeros_like(qlen), qlen)  # live slot, empty window
    qsl = torch.cat([torch.zeros(1, dtype=torch.int64), torch.cumsum(qlen, 0)]).to(torch.int32)
    T = int(qsl[-1])
    unit = lambda x: x / x.norm(dim=-1, keepdim=True)  # noqa: E731
    q = unit(torch.randn(1, T, H, D, generator=gen)).to(torch.bfloat16).cuda()
    k = unit(torch.randn(1, T, H, D, generator=gen)).to(torch.bfloat16).cuda()
    v = torch.randn(1, T, HV, D, generator=gen).to(torch.bfloat16).cuda()
    g = (-torch.nn.functional.softplus(torch.randn(T, HV, generator=gen))).cuda()
    beta = torch.sigmoid(torch.randn(T, HV, generator=gen)).cuda()
    state = (torch.randn(blocks, HV, D, D, generator=gen) * 0.1).cuda()
    records = torch.full((B, HV, Q, 2 * D + 1), -17.0, device="cuda")
    out = torch.full((1, T, HV, D), -23.0, dtype=torch.bfloat16, device="cuda")
    slots_d, qsl_d = slots.to(torch.int32).cuda(), qsl.cuda()
    pkg.gdn_recoverssm_verify(g, beta, q, k, v, checkpoint_state=state, replay_cache=records, query_start_loc=qsl_d,
                              state_indices=slots_d, spec_query_len=Q, out=out)
    torch.cuda.synchronize()
    assert int(torch.ops.gdn_recoverssm_ac.device_status()) == 0
    res = verify_rows(q[0], k[0], v[0], g, beta, state, qsl_d, slots_d, Q=Q)
    got_out = out[0][res["token"].clamp(0, T - 1)].float()  # [B, Q, HV, V]
    want_out = torch.where(res["valid"][:, :, None, None], res["out"], torch.full_like(res["out"], float("nan")))
    assert bool(rounded_ok(got_out, want_out, 7, -126).all()), "outputs"
    null_rows = ~res["live"]
    assert bool((got_out[null_rows][res["valid"][null_rows]] == 0).all()), "null rows must output zeros"
    stored = ~torch.isnan(res["records"])
    assert torch.equal(records != -17.0, stored), "record store mask"
    emax, el2 = rel_errors_per_unit(records, res["records"], 2)
    assert float(emax.max()) <= 1e-5 and float(el2.max()) <= 1e-5, (float(emax.max()), float(el2.max()))
    assert int(null_rows.sum()) > 500 and int(res["live"].sum()) > 500
