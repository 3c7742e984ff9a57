"""GPU parity of the fused-gating verify (``gdn_recoverssm_verify_gated``).

The kernel prologue turns the raw model inputs into the per-token gates,
``g = -exp(A_log[h]) * softplus(a + dt_bias[h])`` with the upstream
``softplus_beta`` / ``softplus_threshold`` form and ``beta = sigmoid(b)``
(docs/reference/recoverssm_gdn_upstream.py:111-151), then runs the same verify
as ``gdn_recoverssm_verify``.  Each case is checked against the float64 oracle
fed with ``oracle.gdn_oracle.gdn_gate`` / ``sigmoid`` of the same rounded
inputs, on both verify kernels (tensor-core K = V = 128 with an fp32 pool,
CUDA-core K = V in {32, 64} and the bf16 pool), with raw ``a`` / ``b`` in fp32
and in the activation dtype, both softplus branches (a low threshold puts
part of the tokens on the linear branch), ragged windows, null / out-of-pool
slots and rows past ``record_rows``.
"""

import numpy as np
import pytest
import torch

from oracle import gdn_oracle as O
from tests.test_gpu_k128 import _assert_rounded_close
from tests.test_gpu_parity import assert_fp32_close

pytestmark = pytest.mark.gpu

CASES = [
    # D, Q, activation, a/b dtype, records, normalise in kernel, H, HV, softplus beta, threshold, state dtype
    (128, 4, torch.bfloat16, torch.bfloat16, "packed", True, 2, 4, 1.0, 20.0, torch.float32),
    (128, 8, torch.bfloat16, torch.float32, "soa", False, 2, 4, 1.0, 1.5, torch.float32),
    (128, 1, torch.float32, torch.float32, "packed", True, 4, 4, 2.0, 20.0, torch.float32),
    (128, 4, torch.bfloat16, torch.bfloat16, "packed", False, 2, 4, 1.0, 20.0, torch.bfloat16),
    (64, 4, torch.float32, torch.float32, "packed", False, 2, 4, 1.0, 20.0, torch.float32),
    (64, 3, torch.bfloat16, torch.bfloat16, "soa", True, 1, 4, 0.5, 1.0, torch.float32),
    (32, 2, torch.float16, torch.float16, "packed", True, 2, 2, 1.0, 20.0, torch.float32),
]


@pytest.fixture(scope="module")
def pkg():
    import gdn_recoverssm_b200 as g
    from gdn_recoverssm_b200 import _native

    _native.ops()
    return g


def _inputs(seed, D, Q, act, ab_dtype, H, HV, normalize, rows=12, blocks=16, a_shift=0.0):
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
    dt = np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), HV))
    return dict(
        q=torch.tensor(q, dtype=act), k=torch.tensor(k, dtype=act),
        v=torch.tensor(rng.standard_normal((T, HV, D)), dtype=act),
        a=torch.tensor(a_shift + 2.0 * rng.standard_normal((T, HV)), dtype=ab_dtype),
        b=torch.tensor(2.0 * rng.standard_normal((T, HV)), dtype=ab_dtype),
        A_log=torch.tensor(np.log(rng.uniform(1.0, 16.0, HV)), dtype=torch.float32),
        dt_bias=torch.tensor(dt + np.log(-np.expm1(-dt)), dtype=torch.float32),  # softplus(dt_bias) = dt
        state=torch.tensor(rng.standard_normal((blocks, HV, D, D)) * 0.1, dtype=torch.float32),
        qsl=torch.tensor(qsl), slots=torch.tensor(slots),
    )


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"D{c[0]}-Q{c[1]}-{str(c[2])[6:]}-ab{str(c[3])[6:]}-{c[4]}"
                                                      f"-n{int(c[5])}-sb{c[8]}-thr{c[9]}-{str(c[10])[6:]}")
def test_verify_gated_matches_oracle(pkg, case):
    D, Q, act, ab_dtype, layout, normalize, H, HV, sb, thr, state_dtype = case
    # a low threshold comes with larger a, so that part of the tokens take the linear branch
    c = _inputs(4321 + D + Q, D, Q, act, ab_dtype, H, HV, normalize, a_shift=0.0 if thr >= 20.0 else 5.0)
    c["state"] = c["state"].to(state_dtype)
    T, rows = c["q"].shape[0], c["slots"].shape[0]
    R = rows - 2  # the last two rows have no record row
    dev = {n: x.cuda() for n, x in c.items()}
    out = torch.full((1, T, HV, D), -23.0, dtype=act, device="cuda")
    if layout == "packed":
        cache = torch.full((R, HV, Q, 2 * D + 1), -17.0, device="cuda")
    else:
        cache = pkg.ReplayRecordBuffers(
            torch.full((R, HV, Q, D), -17.0, device="cuda"),
            torch.full((R, H, Q, D), -16.0, dtype=torch.float32 if normalize else act, device="cuda"),
            torch.full((R, HV, Q), -19.0, device="cuda"),
        )
    before = dev["state"].clone()
    pkg.gdn_recoverssm_verify_gated(
        dev["A_log"], dev["a"], dev["b"][None], dev["dt_bias"], dev["q"][None], dev["k"][None], dev["v"][None],
        checkpoint_state=dev["state"], replay_cache=cache, query_start_loc=dev["qsl"], state_indices=dev["slots"],
        spec_query_len=Q, softplus_beta=sb, softplus_threshold=thr, use_qk_l2norm_in_kernel=normalize, out=out,
    )
    torch.cuda.synchronize()
    assert torch.equal(dev["state"], before), "verify modified the read-only checkpoint"
    assert int(torch.ops.gdn_recoverssm_ac.device_status()) == 0

    f64 = lambda x: x.double().numpy()
    a64, b64 = f64(c["a"]), f64(c["b"])
    g = O.gdn_gate(f64(c["A_log"]), f64(c["dt_bias"]), a64, sb, thr)
    if thr < 20.0:  # the case exercises both softplus branches
        x = sb * (a64 + f64(c["dt_bias"]))
        assert (x > thr).any() and (x <= thr).any()
    o_out = np.full((T, HV, D), -23.0)
    if layout == "packed":
        o_rec = np.full((R, HV, Q, 2 * D + 1), -17.0)
    else:
        o_rec = (np.full((R, HV, Q, D), -17.0), np.full((R, H, Q, D), -16.0), np.full((R, HV, Q), -19.0))
    O.verify_batch(f64(c["q"]), f64(c["k"]), f64(c["v"]), g, O.sigmoid(b64), f64(c["state"]), c["qsl"].numpy(),
                   c["slots"].numpy(), spec_query_len=Q, normalize_qk=normalize, record_rows=R, layout=layout,
                   out=o_out, records=o_rec)

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
        checks = [(cache, o_rec, -17.0, "packed records")]
    else:
        checks = zip((cache.correction, cache.key, cache.decay), o_rec, (-17.0, -16.0, -19.0),
                     ("correction", "key", "decay"))
    for got_t, want, sentinel, name in checks:
        g_np = got_t.double().cpu().numpy()
        assert np.array_equal(g_np == sentinel, want == sentinel), f"{name} store mask"
        m = want != sentinel
        assert_fp32_close(g_np[m], want[m], what=name)


def test_gated_equals_ungated_with_host_gates(pkg):
    """The fused prologue and the plain entry point fed with the same gates
    (computed on the host in float64 and rounded to fp32) agree to the fp32
    tolerance on outputs and records: one verify, two ways of getting g."""
    D, Q, HV, H = 128, 4, 4, 2
    c = _inputs(77, D, Q, torch.bfloat16, torch.float32, H, HV, True)
    dev = {n: x.cuda() for n, x in c.items()}
    T, rows = c["q"].shape[0], c["slots"].shape[0]
    g = O.gdn_gate(c["A_log"].double().numpy(), c["dt_bias"].double().numpy(), c["a"].double().numpy())
    beta = O.sigmoid(c["b"].double().numpy())
    res = []
    for gated in (True, False):
        out = torch.zeros(1, T, HV, D, dtype=torch.bfloat16, device="cuda")
        cache = torch.zeros(rows, HV, Q, 2 * D + 1, device="cuda")
        kw = dict(checkpoint_state=dev["state"], replay_cache=cache, query_start_loc=dev["qsl"],
                  state_indices=dev["slots"], spec_query_len=Q, out=out)
        if gated:
            pkg.gdn_recoverssm_verify_gated(dev["A_log"], dev["a"], dev["b"], dev["dt_bias"], dev["q"][None],
                                            dev["k"][None], dev["v"][None], **kw)
        else:
            pkg.gdn_recoverssm_verify(torch.tensor(g, dtype=torch.float32, device="cuda"),
                                      torch.tensor(beta, dtype=torch.float32, device="cuda"), dev["q"][None],
                                      dev["k"][None], dev["v"][None], qk_already_normalized=False, **kw)
        torch.cuda.synchronize()
        res.append((out.double().cpu().numpy(), cache.double().cpu().numpy()))
    assert_fp32_close(res[0][1], res[1][1], what="records")
    o0, o1 = res[0][0], res[1][0]
    vmax = np.abs(o1).max(axis=-1, keepdims=True)
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(o1), 1e-30))) - 7)
    assert np.all((np.abs(o0 - o1) <= ulp * 1.01) | (np.abs(o0 - o1) <= 1e-5 * vmax)), "outputs"
    assert int(torch.ops.gdn_recoverssm_ac.device_status()) == 0


def test_capi_gated_direct_call_matches_torch_op(pkg):
    """gdn_rssm_verify_gated called through ctypes with raw device pointers
    (the binding a non-torch host would use) gives bit-identical results to
    the torch op."""
    from gdn_recoverssm_b200 import capi

    D, Q, HV, H = 128, 4, 4, 2
    c = _inputs(91, D, Q, torch.bfloat16, torch.bfloat16, H, HV, True)
    dev = {n: x.cuda() for n, x in c.items()}
    T, rows = c["q"].shape[0], c["slots"].shape[0]
    res = []
    for direct in (False, True):
        out = torch.zeros(1, T, HV, D, dtype=torch.bfloat16, device="cuda")
        cache = torch.zeros(rows, HV, Q, 2 * D + 1, device="cuda")
        specs = []
        pkg.gdn_recoverssm_verify_gated(dev["A_log"], dev["a"], dev["b"], dev["dt_bias"], dev["q"][None],
                                        dev["k"][None], dev["v"][None], checkpoint_state=dev["state"],
                                        replay_cache=cache, query_start_loc=dev["qsl"], state_indices=dev["slots"],
                                        spec_query_len=Q, out=out, _collect=specs)
        (q, k, v, a, b, A_log, dt_bias, state, corr, key, decay, o, qsl, idx, config, scale, sb, thr,
         flags) = specs[0].args
        if direct:
            capi.verify_gated(q, k, v, a, b, A_log, dt_bias, state, corr, key, decay, o, qsl, idx, config, scale, sb,
                              thr, flags=flags)
        else:
            specs[0].launch()
        torch.cuda.synchronize()
        res.append((out.cpu(), cache.cpu()))
    assert torch.equal(res[0][0], res[1][0]) and torch.equal(res[0][1], res[1][1])
    assert int(torch.ops.gdn_recoverssm_ac.device_status()) == 0
