"""Generate golden fixtures by running the REFERENCE's own Triton kernels.

Run in the build container only (it needs the read-only reference checkout):

    python tests/golden/make_golden.py /path/to/reference

It loads ``plugin/gdn_recoverssm_ascend/kernels.py`` and ``grouped_commit.py``
with ``TRITON_INTERPRET=1`` (Triton's CPU interpreter) and five stub modules
standing in for vLLM / vllm-ascend, calls the reference's public entry points
(``gdn_recoverssm_verify``, ``GDNRecoverSSMCommitContext.commit``,
``GroupedCommitBucket.make_specs``) on small seeded inputs, and writes every
input and output array to ``tests/golden/*.npz``.  The committed fixtures are
what the tests read; the reference is never read at test time.

bf16 tensors are stored as float32 arrays (exact) next to a ``<name>__dtype``
entry.
"""

from __future__ import annotations

import importlib.util
import logging
import os
import sys
import types
from pathlib import Path
from types import SimpleNamespace

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent


def _load_reference(root: Path):
    import triton
    import triton.language as tl

    def stub(name, **attrs):
        m = types.ModuleType(name)
        m.__dict__.update(attrs)
        m.__path__ = []
        sys.modules[name] = m

    for n in (
        "vllm",
        "vllm.v1",
        "vllm.v1.attention",
        "vllm.v1.attention.backends",
        "vllm_ascend",
        "vllm_ascend.ops",
        "vllm_ascend.ops.triton",
    ):
        stub(n)
    stub("vllm.logger", init_logger=logging.getLogger)
    stub("vllm.triton_utils", tl=tl, triton=triton)
    stub("vllm.v1.attention.backends.utils", NULL_BLOCK_ID=0)
    stub(
        "vllm_ascend.ops.triton.triton_utils",
        get_ub_size_bytes=lambda: 196608,
        get_vectorcore_num=lambda: 8,
    )
    pkg_dir = root / "plugin" / "gdn_recoverssm_ascend"
    pkg = types.ModuleType("gdn_recoverssm_ascend")
    pkg.__path__ = [str(pkg_dir)]
    sys.modules["gdn_recoverssm_ascend"] = pkg
    mods = {}
    for name in ("kernels", "grouped_commit"):
        spec = importlib.util.spec_from_file_location(
            f"gdn_recoverssm_ascend.{name}", pkg_dir / f"{name}.py"
        )
        m = importlib.util.module_from_spec(spec)
        sys.modules[spec.name] = m
        spec.loader.exec_module(m)
        mods[name] = m
    return mods["kernels"], mods["grouped_commit"]


def _np(t: torch.Tensor):
    t = t.detach().cpu()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.float().numpy(), str(t.dtype).split(".")[-1]
    return t.numpy().copy(), str(t.dtype).split(".")[-1]


def _changed(before, after):
    """Pages of ``after`` that differ from ``before``: ``(page ids, values)``."""
    diff = (before != after).reshape(before.shape[0], -1).any(dim=1)
    ids = diff.nonzero().flatten()
    return ids.to(torch.int32), after[ids].clone()


def _save(name, **tensors):
    arrays = {}
    for key in [k for k in tensors if "_after" in k]:
        before = tensors[key.replace("_after", "_before")]
        ids, vals = _changed(before, tensors.pop(key))
        tensors[key + "_pages"] = ids
        tensors[key] = vals
    for key, value in tensors.items():
        if isinstance(value, torch.Tensor):
            arr, dt = _np(value)
            arrays[key] = arr
            arrays[key + "__dtype"] = np.array(dt)
        else:
            arrays[key] = np.asarray(value)
    np.savez_compressed(HERE / f"{name}.npz", **arrays)
    print("wrote", name, sum(a.nbytes for a in arrays.values()), "bytes raw")


def _unit(x):
    return x / x.float().norm(dim=-1, keepdim=True).clamp_min(1e-6).to(x.dtype)


def _verify_inputs(gen, *, T, H, HV, D, act, beta_dtype, normalized):
    q = torch.randn(T, H, D, generator=gen)
    k = torch.randn(T, H, D, generator=gen)
    if normalized:
        q, k = _unit(q), _unit(k)
    q, k = q.to(act), k.to(act)
    v = torch.randn(T, HV, D, generator=gen).to(act)
    g = -torch.nn.functional.softplus(torch.randn(T, HV, generator=gen))
    beta = torch.sigmoid(torch.randn(T, HV, generator=gen)).to(beta_dtype)
    return q, k, v, g.float(), beta


def verify_case(K, name, *, layout, act, beta_dtype, normalized, Q, D=32, H=2, HV=4, seed=0):
    """Rows: full window, short window, null slot, out-of-pool slot, full window
    past ``record_rows``, zero-length padding."""
    gen = torch.Generator().manual_seed(seed)
    qlens = [Q, max(Q - 1, 1), Q, Q, Q, 0]
    B = len(qlens)
    qsl = torch.tensor([0] + list(np.cumsum(qlens)), dtype=torch.int32)
    T = int(qsl[-1])
    blocks = 9
    slots = torch.tensor([3, 7, 0, blocks + 2, 5, 0], dtype=torch.int32)
    record_rows = 4
    q, k, v, g, beta = _verify_inputs(
        gen, T=T, H=H, HV=HV, D=D, act=act, beta_dtype=beta_dtype, normalized=normalized
    )
    state = (torch.randn(blocks, HV, D, D, generator=gen) * 0.1).float()
    state_before = state.clone()
    out = torch.full((1, T, HV, D), -23.0, dtype=act)
    if layout == "packed":
        rec = torch.full((record_rows, HV, Q, 2 * D + 1), -17.0)
        cache = rec
    else:
        corr = torch.full((record_rows, HV, Q, D), -17.0)
        key = torch.full((record_rows, H, Q, D), -16.0, dtype=act if normalized else torch.float32)
        decay = torch.full((record_rows, HV, Q), -19.0)
        cache = K.ReplayRecordBuffers(corr, key, decay)
    K.gdn_recoverssm_verify(
        g[None],
        beta[None],
        q[None],
        k[None],
        v[None],
        checkpoint_state=state,
        replay_cache=cache,
        query_start_loc=qsl,
        state_indices=slots,
        spec_query_len=Q,
        qk_already_normalized=normalized,
        out=out,
    )
    assert torch.equal(state, state_before)
    extra = (
        dict(records=rec)
        if layout == "packed"
        else dict(corr=cache.correction, key=cache.key, decay=cache.decay)
    )
    _save(
        name,
        q=q,
        k=k,
        v=v,
        g=g,
        beta=beta,
        state=state,
        qsl=qsl,
        state_indices=slots,
        out=out[0],
        spec_query_len=Q,
        normalized=int(normalized),
        layout=layout,
        record_rows=record_rows,
        **extra,
    )


def config0_case(K, seed=0):
    """B=4, H=HV=4, K=V=64, Q=4, fp32 everywhere, pool of 8
    slots with distinct random ids, accepted ~ U{1..4}; verify then the
    per-context commit in none mode."""
    gen = torch.Generator().manual_seed(seed)
    B, H, HV, D, Q = 4, 4, 4, 64, 4
    T = B * Q
    q = _unit(torch.randn(T, H, D, generator=gen))
    k = _unit(torch.randn(T, H, D, generator=gen))
    v = torch.randn(T, HV, D, generator=gen)
    g = -torch.nn.functional.softplus(torch.randn(T, HV, generator=gen))
    beta = torch.sigmoid(torch.randn(T, HV, generator=gen))
    state = torch.randn(8, HV, D, D, generator=gen) * 0.1
    state0 = state.clone()
    slots = (torch.randperm(7, generator=gen)[:B] + 1).to(torch.int32)
    accepted = torch.randint(1, Q + 1, (B,), generator=gen, dtype=torch.int32)
    qsl = torch.arange(B + 1, dtype=torch.int32) * Q
    rec = torch.zeros(B, HV, Q, 2 * D + 1)
    out = torch.zeros(1, T, HV, D)
    K.gdn_recoverssm_verify(
        g[None], beta[None], q[None], k[None], v[None],
        checkpoint_state=state, replay_cache=rec, query_start_loc=qsl,
        state_indices=slots, spec_query_len=Q, out=out,
    )
    conv = torch.zeros(8, 16, 3 + Q - 1)
    ctx = K.GDNRecoverSSMCommitContext.from_tensors(
        [conv], [state], [rec], spec_query_len=Q, max_num_reqs=B
    )
    ctx.commit(accepted, slots, qsl)
    _save(
        "config0",
        q=q, k=k, v=v, g=g, beta=beta, state_before=state0, state_after=state,
        qsl=qsl, state_indices=slots, accepted=accepted, out=out[0], records=rec,
        commit_lens=ctx.commit_lens[:B], final=ctx.final_state_indices[:B],
        spec_query_len=Q,
    )


def context_commit_case(K, name, *, align, soa, layers=1, seed=1, D=32, H=2, HV=4, Q=4):
    """Per-context plan -> conv -> fold through ``GDNRecoverSSMCommitContext``.

    Rows: full accept, zero accept, null source, reordered request, short
    window, accepted above qlen.  Every request owns distinct pages so that no
    row reads a page another row writes (launch order would then matter).  In
    align mode the source is the request's running column page, so a crossed
    boundary aliases the source page (the serving pattern).
    """
    gen = torch.Generator().manual_seed(seed)
    blocks, rows, hist, cdim = 20, 6, 3, 16
    states = [torch.randn(blocks, HV, D, D, generator=gen) * 0.1 for _ in range(layers)]
    convs = [torch.randn(blocks, cdim, hist + Q - 1, generator=gen) for _ in range(layers)]
    if soa:
        records = [
            K.ReplayRecordBuffers(
                torch.randn(rows, HV, Q, D, generator=gen) * 0.1,
                _unit(torch.randn(rows, H, Q, D, generator=gen)).to(torch.bfloat16),
                torch.rand(rows, HV, Q, generator=gen) * 0.5 + 0.45,
            )
            for _ in range(layers)
        ]
    else:
        records = []
        for _ in range(layers):
            r = torch.randn(rows, HV, Q, 2 * D + 1, generator=gen) * 0.1
            r[..., D : 2 * D] = _unit(torch.randn(rows, HV, Q, D, generator=gen))
            r[..., 2 * D] = torch.rand(rows, HV, Q, generator=gen) * 0.5 + 0.45
            records.append(r)
    states0 = [s.clone() for s in states]
    convs0 = [c.clone() for c in convs]
    ctx = K.GDNRecoverSSMCommitContext.from_tensors(
        convs, states, records, spec_query_len=Q, max_num_reqs=rows
    )
    qlens = [Q, Q, Q, Q, 2, 3]
    qsl = torch.tensor([0] + list(np.cumsum(qlens)), dtype=torch.int32)
    req = torch.tensor([0, 1, 2, 4, 3, 5], dtype=torch.int64)
    acc = torch.tensor([4, 0, 3, 2, 1, 4], dtype=torch.int32)
    kw = dict(request_indices=req)
    extra = {}
    if align:
        bs, W = 4, 3
        # request r owns pages 1 + 3r .. 3 + 3r
        bt = (torch.arange(rows * W, dtype=torch.int32) + 1).reshape(rows, W)
        computed = torch.tensor([2, 5, 0, 7, 3, 1], dtype=torch.int32)
        bt[5, 1] = blocks + 5  # request 5's next page is outside the pool
        src = torch.tensor(
            [int(bt[int(r), int(computed[int(r)]) // bs]) for r in req], dtype=torch.int32
        )
        src[2] = 0  # null source row
        kw.update(block_table=bt, num_computed_tokens=computed, mamba_block_size=bs)
        extra = dict(block_table=bt, num_computed=computed, block_size=bs)
    else:
        src = torch.tensor([3, 4, 0, 6, 8, 9], dtype=torch.int32)
    ctx.commit(acc, src, qsl, **kw)
    arrays = dict(
        src=src, qsl=qsl, request_indices=req, accepted=acc, spec_query_len=Q,
        commit_lens=ctx.commit_lens[:rows], final=ctx.final_state_indices[:rows],
        boundary=ctx.boundary_state_indices[:rows], boundary_lens=ctx.boundary_recovery_lens[:rows],
        valid=ctx.align_valid[:rows], col=ctx.align_col[:rows], history=hist,
        align=int(align), layout="soa" if soa else "packed", layers=layers, **extra,
    )
    for i in range(layers):
        arrays[f"state_before{i}"] = states0[i]
        arrays[f"state_after{i}"] = states[i]
        arrays[f"conv_before{i}"] = convs0[i]
        arrays[f"conv_after{i}"] = convs[i]
        if soa:
            arrays[f"corr{i}"] = records[i].correction
            arrays[f"key{i}"] = records[i].key
            arrays[f"decay{i}"] = records[i].decay
        else:
            arrays[f"records{i}"] = records[i]
    _save(name, **arrays)


def plan_int32_case(K, name, *, seed=9, D=32, H=2, HV=4, Q=4):
    """Per-context align commit whose counts exercise the plan's int32
    arithmetic: int64 accepted counts past 2^31 (truncated on load), a
    computed count near 2^31 whose end position and next boundary wrap, an
    int64 computed count that truncates to a small one, and negative counts."""
    gen = torch.Generator().manual_seed(seed)
    blocks, rows, hist, cdim, bs, W = 24, 7, 3, 16, 64, 3
    states = [torch.randn(blocks, HV, D, D, generator=gen) * 0.1]
    convs = [torch.randn(blocks, cdim, hist + Q - 1, generator=gen)]
    r = torch.randn(rows, HV, Q, 2 * D + 1, generator=gen) * 0.1
    r[..., D : 2 * D] = _unit(torch.randn(rows, HV, Q, D, generator=gen))
    r[..., 2 * D] = torch.rand(rows, HV, Q, generator=gen) * 0.5 + 0.45
    records = [r]
    states0 = [s.clone() for s in states]
    convs0 = [c.clone() for c in convs]
    ctx = K.GDNRecoverSSMCommitContext.from_tensors(convs, states, records, spec_query_len=Q, max_num_reqs=rows)
    big = 1 << 31
    acc = torch.tensor([big + 3, (1 << 32) + 2, 3, 4, 2, -1, 4], dtype=torch.int64)
    computed = torch.tensor([5, 5, big - 2, (1 << 32) + 62, big + 1, 7, big - 3], dtype=torch.int64)
    qsl = torch.arange(rows + 1, dtype=torch.int32) * Q
    req = torch.arange(rows, dtype=torch.int64)
    bt = (torch.arange(rows * W, dtype=torch.int32) + 1).reshape(rows, W)
    src = bt[:, 0].clone()
    ctx.commit(acc, src, qsl, request_indices=req, block_table=bt, num_computed_tokens=computed,
               mamba_block_size=bs)
    arrays = dict(
        src=src, qsl=qsl, request_indices=req, accepted=acc, spec_query_len=Q, block_table=bt,
        num_computed=computed, block_size=bs, num_blocks=blocks,
        commit_lens=ctx.commit_lens[:rows], final=ctx.final_state_indices[:rows],
        boundary=ctx.boundary_state_indices[:rows], boundary_lens=ctx.boundary_recovery_lens[:rows],
        valid=ctx.align_valid[:rows], col=ctx.align_col[:rows], history=hist, records0=records[0],
        align=1, layout="packed", layers=1,
        state_before0=states0[0], state_after0=states[0], conv_before0=convs0[0], conv_after0=convs[0],
    )
    _save(name, **arrays)


def grouped_case(K, Gm, name, *, seed=2, D=32, H=2, HV=4, Q=4):
    """Two KV groups x two layers through ``GroupedCommitBucket.make_specs``:
    reordered requests, a null row, boundary crossings, an invalid group row,
    zero acceptance, publication into persistent columns."""
    gen = torch.Generator().manual_seed(seed)
    blocks, rows, hist, cdim, bs = 16, 4, 3, 16, 4
    tables = (
        torch.tensor([[1, 2, 7, 0], [4, 5, 6, 0], [0, 0, 0, 0], [9, 10, 11, 12], [13, 14, 15, 3]], dtype=torch.int32),
        torch.tensor([[3, 4, 7, 0], [1, 2, 6, 0], [0, 0, 0, 0], [8, 9, 10, 11], [12, 14, 15, 0]], dtype=torch.int32),
    )
    computed = torch.tensor([bs - 1, 1, 0, 2, 6], dtype=torch.int32)
    host_rows = (1, 0, 2, 4)
    qlens = (Q, Q, 0, Q)
    qsl = torch.tensor([0] + list(np.cumsum(qlens)), dtype=torch.int32)
    sampled = torch.tensor([Q, Q - 1, 0, 2, 3], dtype=torch.int32)
    mapping = torch.tensor([2, 0, -1, 5, 4], dtype=torch.int32)
    cols = torch.full((6,), -9, dtype=torch.int32)
    accepted = torch.full((6,), 7, dtype=torch.int32)
    entries, arrays = [], {}
    for grp in range(2):
        states, convs, records = [], [], []
        for layer in range(2):
            states.append(torch.randn(blocks, HV, D, D, generator=gen) * 0.1)
            convs.append(torch.randn(blocks, cdim, hist + Q - 1, generator=gen))
            records.append(
                K.ReplayRecordBuffers(
                    torch.randn(rows, HV, Q, D, generator=gen) * 0.1,
                    _unit(torch.randn(rows, H, Q, D, generator=gen)).to(torch.bfloat16),
                    torch.rand(rows, HV, Q, generator=gen) * 0.5 + 0.45,
                )
            )
            i = grp * 2 + layer
            arrays[f"state_before{i}"] = states[-1].clone()
            arrays[f"conv_before{i}"] = convs[-1].clone()
            arrays[f"corr{i}"] = records[-1].correction
            arrays[f"key{i}"] = records[-1].key
            arrays[f"decay{i}"] = records[-1].decay
        ctx = K.GDNRecoverSSMCommitContext.from_tensors(
            convs, states, records, spec_query_len=Q, max_num_reqs=rows
        )
        table = torch.zeros(rows, Q, dtype=torch.int32)
        table[:, 0] = torch.tensor([int(tables[grp][r, 0]) for r in host_rows], dtype=torch.int32)
        payload = SimpleNamespace(
            state_indices=table[:, 0],
            query_start_loc=qsl,
            request_indices=torch.tensor(host_rows, dtype=torch.int64),
            block_table=tables[grp],
            num_computed_tokens=computed,
            block_size=bs,
            request_rows=host_rows,
            query_lens=qlens,
        )
        arrays[f"state_indices{grp}"] = table[:, 0].clone()
        arrays[f"block_table{grp}"] = tables[grp]
        entries.append(Gm.CommitEntry(None, payload, ctx))
    bucket = Gm.GroupedCommitBucket(tuple(e.context for e in entries))
    for spec in bucket.make_specs(entries, sampled, mapping, cols, accepted):
        spec.launch()
    for i, (st, cv) in enumerate(zip(bucket.checkpoints, bucket.conv_states)):
        arrays[f"state_after{i}"] = st
        arrays[f"conv_after{i}"] = cv
    _save(
        name,
        qsl=qsl, request_indices=torch.tensor(host_rows, dtype=torch.int64),
        computed=computed, sampled=sampled, mapping=mapping,
        cols=cols, accepted=accepted, block_size=bs, spec_query_len=Q, history=hist,
        capacity=bucket.capacity, layer_groups=bucket.layer_groups,
        plan_source=bucket.source, plan_length=bucket.length, plan_final=bucket.final,
        plan_boundary=bucket.boundary, plan_boundary_len=bucket.boundary_len,
        plan_valid=bucket.valid, plan_col=bucket.col, num_blocks=blocks,
        **arrays,
    )


def main(root):
    K, Gm = _load_reference(Path(root))
    torch.manual_seed(0)
    verify_case(K, "verify_packed_bf16_q4", layout="packed", act=torch.bfloat16,
                beta_dtype=torch.float32, normalized=True, Q=4)
    verify_case(K, "verify_soa_bf16_q4", layout="soa", act=torch.bfloat16,
                beta_dtype=torch.bfloat16, normalized=True, Q=4, seed=3)
    verify_case(K, "verify_packed_fp32_l2_q3", layout="packed", act=torch.float32,
                beta_dtype=torch.float32, normalized=False, Q=3, seed=4)
    verify_case(K, "verify_soa_fp32_l2_q8", layout="soa", act=torch.float32,
                beta_dtype=torch.float32, normalized=False, Q=8, seed=5)
    verify_case(K, "verify_packed_bf16_q1", layout="packed", act=torch.bfloat16,
                beta_dtype=torch.float32, normalized=True, Q=1, seed=6)
    config0_case(K)
    context_commit_case(K, "context_commit_none_packed", align=False, soa=False)
    context_commit_case(K, "context_commit_align_packed", align=True, soa=False, seed=7)
    context_commit_case(K, "context_commit_align_soa", align=True, soa=True, layers=2, seed=8)
    grouped_case(K, Gm, "grouped_align_soa")
    plan_int32_case(K, "context_plan_int32")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <reference checkout>")
    main(sys.argv[1])
