"""State drift over many speculative steps (K = V = 128, fp32 state pool).

64 consecutive verify -> commit steps, each step's folded state feeding the
next: the tensor-core verify (split tf32 / bf16 products) writes the records
the fold consumes, so any bias of the split would accumulate here.  After every
step the pool pages are compared with float64 sequential decode of exactly the
accepted tokens (tests/torch_reference.py, the state carried in float64 from
the same start): per (row, value head) max-relative and l2-relative error
<= 1e-5 at every step.  The same 64 steps also run through the CUDA-core
verify kernel (fp32 FMAs, flag GDN_RSSM_VERIFY_CUDA_CORES) on its own pool, and
both worst errors are reported side by side (reference behaviour:
plugin/tests/test_math_oracle.py:34-92, selftest.py:61-89).
"""

import pytest
import torch

from tests.torch_reference import rel_errors_per_unit, verify_rows

pytestmark = pytest.mark.gpu
TOL = 1e-5
CUDA_CORES = 0x20000  # GDN_RSSM_VERIFY_CUDA_CORES


@pytest.fixture(scope="module")
def g():
    import gdn_recoverssm_b200 as pkg
    from gdn_recoverssm_b200 import _native

    _native.ops()
    return pkg


def _step_inputs(gen, T, H, HV, D, act):
    unit = lambda x: x / x.norm(dim=-1, keepdim=True)  # noqa: E731
    q = unit(torch.randn(1, T, H, D, generator=gen, device="cuda")).to(act)
    k = unit(torch.randn(1, T, H, D, generator=gen, device="cuda")).to(act)
    v = torch.randn(1, T, HV, D, generator=gen, device="cuda").to(act)
    gg = -torch.nn.functional.softplus(torch.randn(T, HV, generator=gen, device="cuda"))
    beta = torch.sigmoid(torch.randn(T, HV, generator=gen, device="cuda"))
    return q, k, v, gg, beta


@pytest.mark.parametrize("align", [False, True], ids=["in_place", "align"])
def test_state_drift_over_64_steps(g, align):
    """``in_place``: none mode, every row commits into its own page.
    ``align``: block size 4, 2 tokens computed: a row with n <= 2 accepted
    tokens commits in place; with n >= 3 its window crosses the block
    boundary, the snapshot after 2 tokens overwrites the source page (the
    boundary page aliases the source) and the final state moves to the row's
    other page, which is the next step's source."""
    B, H, HV, D, Q, steps = 64, 4, 8, 128, 4, 64
    T = B * Q
    act = torch.bfloat16
    gen = torch.Generator(device="cuda").manual_seed(2024 + int(align))
    cpu = torch.Generator().manual_seed(99)
    blocks = 2 * B + 1
    pool0 = torch.randn(blocks, HV, D, D, generator=gen, device="cuda") * 0.1
    pools = {"tensor_cores": pool0.clone(), "cuda_cores": pool0.clone()}
    ref = pool0.double()
    cur = torch.arange(1, B + 1, dtype=torch.int32, device="cuda")  # row r owns pages 1 + r and 1 + B + r
    qsl = torch.arange(B + 1, dtype=torch.int32, device="cuda") * Q
    records = {name: torch.zeros(B, HV, Q, 2 * D + 1, device="cuda") for name in pools}
    conv = torch.zeros(blocks, 8, 3 + Q - 1, dtype=act, device="cuda")
    ctxs = {name: g.GDNRecoverSSMCommitContext.from_tensors([conv], [pools[name]], [records[name]],
                                                            spec_query_len=Q, max_num_reqs=B) for name in pools}
    worst = {name: [0.0, 0.0] for name in pools}
    crossed = 0
    for step in range(steps):
        q, k, v, gg, beta = _step_inputs(gen, T, H, HV, D, act)
        acc = torch.randint(1, Q + 1, (B,), generator=cpu, dtype=torch.int32).cuda()
        src = cur.clone()
        kw = {}
        if align:
            other = torch.where(src <= B, src + B, src - B).to(torch.int32)
            kw = dict(block_table=torch.stack([src, other], dim=1), mamba_block_size=4,
                      num_computed_tokens=torch.full((B,), 2, dtype=torch.int32, device="cuda"))
            cross = acc >= 3
            fin = torch.where(cross, other, src)
        else:
            cross = torch.zeros(B, dtype=torch.bool, device="cuda")
            fin = src
        for name, pool in pools.items():
            specs = []
            g.gdn_recoverssm_verify(gg, beta, q, k, v, checkpoint_state=pool, replay_cache=records[name],
                                    query_start_loc=qsl, state_indices=src, spec_query_len=Q, _collect=specs)
            spec = specs[0]
            if name == "cuda_cores":
                spec.args = spec.args[:-1] + (spec.args[-1] | CUDA_CORES,)
            spec.launch()
            ctxs[name].commit(acc, src, qsl, **kw)
        two = torch.full((B,), 2, dtype=torch.int64, device="cuda")
        res = verify_rows(q[0], k[0], v[0], gg, beta, ref, qsl, src, Q=Q, capture={"final": acc, "boundary": two})
        ref[src[cross].long()] = res["boundary"][cross]
        ref[fin.long()] = res["final"]
        torch.cuda.synchronize()
        crossed += int(cross.sum())
        for name, pool in pools.items():
            checked = torch.cat([fin, src[cross]]).long()
            e = rel_errors_per_unit(pool[checked], ref[checked], 2)
            worst[name] = [max(worst[name][i], float(e[i].max())) for i in range(2)]
            assert max(float(e[0].max()), float(e[1].max())) <= TOL, f"{name} step {step}: {e}"
        cur = fin.to(torch.int32)
    assert int(torch.ops.gdn_recoverssm_ac.device_status()) == 0
    if align:
        assert crossed > 0
    print(f"drift over {steps} steps ({'align' if align else 'in place'}), worst per-unit (max-rel, l2-rel): "
          f"tensor cores {worst['tensor_cores']}, CUDA cores {worst['cuda_cores']}")
