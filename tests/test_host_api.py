"""Host-side contract tests (CPU only): the C ABI library loads and exports
every entry point the header declares, rejects bad arguments before any launch
(no GPU needed), and the Python entry points keep the reference's
signatures, ValueError checks and byte accounting."""

import re
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "gdn_recoverssm_b200.h"


def _declared():
    text = HEADER.read_text()
    return re.findall(r"GDN_RSSM_API\s+[\w\s\*]+?\b(gdn_rssm_\w+)\s*\(", text)


def test_library_exports_every_declared_symbol():
    from gdn_recoverssm_b200 import capi

    names = _declared()
    assert len(names) == 10, names
    lib = capi.lib()
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(capi.PROTOTYPES)
    assert lib.gdn_rssm_abi_version() == 1


def test_libraries_link_the_shared_cpp_runtime():
    """Neither built library carries a private static C++ runtime: the torch
    ops throw c10::Error through torch's own libstdc++, and a private copy's
    iostreams crash while formatting a check's message."""
    import shutil
    import subprocess

    from gdn_recoverssm_b200 import build

    nm = shutil.which("nm")
    if nm is None:
        pytest.skip("nm not available")
    for lib in (build.CAPI_LIB, build.TORCH_LIB):
        out = subprocess.run([nm, "-D", "--defined-only", str(lib)], capture_output=True, text=True).stdout
        assert "__cxa_throw" not in out and "_ZNSt8ios_base4InitC" not in out, lib.name


def test_torch_ops_register_reference_schemas():
    from gdn_recoverssm_b200 import _native

    ops = _native.ops()
    assert ops.abi_version() == 1
    verify = str(ops.verify.default._schema)
    fold = str(ops.fold.default._schema)
    # the reference's native schemas (csrc/ops.cpp:243-251), argument for argument
    assert verify == (
        "gdn_recoverssm_ac::verify(Tensor q, Tensor k, Tensor v, Tensor g, Tensor beta, Tensor state, "
        "Tensor(a!) correction, Tensor(b!) key, Tensor(c!) decay, Tensor(d!) out, Tensor qsl, Tensor indices, "
        "int[] config, float scale) -> ()"
    )
    assert fold.startswith("gdn_recoverssm_ac::fold(Tensor(a!) state, Tensor correction, Tensor key, Tensor decay,")
    assert fold.endswith("Tensor boundary_lengths, int[] config) -> ()")
    # the fused-gating form: upstream argument order for the gate inputs
    gated = str(ops.verify_gated_ext.default._schema)
    assert gated.startswith("gdn_recoverssm_ac::verify_gated_ext(Tensor q, Tensor k, Tensor v, Tensor a, Tensor b, "
                            "Tensor A_log, Tensor dt_bias, Tensor state, Tensor(a!) correction,")
    assert gated.endswith("float scale, float softplus_beta, float softplus_threshold, int flags) -> ()")


def _verify_call(lib, capi, config, **over):
    args = dict(act=capi.BF16, state=capi.F32, beta=capi.F32, key=capi.F32, qsl=capi.I32, idx=capi.I32, K=128, V=128,
                flags=capi.RECORD_PACKED)
    args.update(over)
    cfg = capi.int64_array(config)
    return lib.gdn_rssm_verify(*([None] * 12), cfg, len(config), 1.0, args["act"], args["state"], args["beta"],
                               args["key"], args["qsl"], args["idx"], args["K"], args["V"], args["flags"], None)


def capi_flags_unknown():
    return 1 << 20  # not a verify flag (GDN_RSSM_VERIFY_TEST_NO_TILE is 1 << 16)


def _good_config():
    # rows, tokens, H, HV, Q, blocks, record_rows, null, ... strides
    return [4, 16, 2, 4, 4, 8, 4, 0] + [1] * 20


@pytest.mark.parametrize(
    "mutate,over,match",
    [
        (lambda c: c[:27], {}, "28 fields"),
        (lambda c: c[:7] + [1] + c[8:], {}, "null block"),
        (lambda c: c, {"K": 64}, "K and V must be equal"),
        (lambda c: c, {"K": 96, "V": 96}, "K and V must be equal"),
        (lambda c: c[:4] + [9] + c[5:], {}, "spec_query_len"),
        (lambda c: c[:2] + [3] + c[3:], {}, "multiple"),
        (lambda c: c, {"beta": 2}, "beta"),
        (lambda c: c, {"flags": 0, "key": 1, "act": 0}, "low-precision key"),
        (lambda c: c, {"state": 2}, "state must be"),
        (lambda c: c[:1] + [100] + c[2:], {}, "activation capacity"),
        (lambda c: [2**31, 2**31] + c[2:], {}, "below 2^31"),
        (lambda c: c[:5] + [2**31] + c[6:], {}, "below 2^31"),
        (lambda c: c, {"flags": capi_flags_unknown()}, "unknown verify flags"),
    ],
)
def test_capi_verify_rejects_before_launch(mutate, over, match):
    from gdn_recoverssm_b200 import capi

    lib = capi.lib()
    rc = _verify_call(lib, capi, mutate(_good_config()), **over)
    assert rc == capi.EINVAL
    assert match in capi.last_error()


@pytest.mark.parametrize(
    "over,match",
    [
        (dict(A_log=None), "needs A_log"),
        (dict(dt_bias=None), "gating needs A_log, dt_bias"),
        (dict(sb=0.0), "softplus_beta > 0"),
        (dict(sb=float("nan")), "softplus_beta > 0"),
        (dict(gate=2), "the gate must be FP32"),  # fp16 raw a with bf16 activations
        (dict(b=2), "beta must be FP32 or the activation dtype"),
    ],
)
def test_capi_verify_gated_rejects_before_launch(over, match):
    import ctypes

    from gdn_recoverssm_b200 import capi

    lib = capi.lib()
    dummy = ctypes.c_void_p(256)  # never dereferenced: validation fails first
    args = dict(A_log=dummy, dt_bias=dummy, sb=1.0, gate=capi.BF16, b=capi.F32)
    args.update(over)
    cfg = capi.int64_array(_good_config())
    rc = lib.gdn_rssm_verify_gated(*([None] * 5), args["A_log"], args["dt_bias"], *([None] * 7), cfg, 28, 1.0,
                                   args["sb"], 20.0, capi.BF16, capi.F32, args["gate"], args["b"], capi.F32, capi.I32,
                                   capi.I32, 128, 128, capi.RECORD_PACKED, None)
    assert rc == capi.EINVAL
    assert match in capi.last_error()


def test_capi_fold_and_plans_reject_before_launch():
    from gdn_recoverssm_b200 import capi

    lib = capi.lib()
    cfg = capi.int64_array([4] * 16)
    rc = lib.gdn_rssm_fold(*([None] * 9), capi.index_view(None), *([None] * 4), 0, cfg, 16, capi.F32, capi.F32, 128,
                           128, 0, None)
    assert rc == capi.EINVAL and "17 fields" in capi.last_error()
    group = capi.PlanGroup()
    rc = lib.gdn_rssm_grouped_plan(capi.index_view(None), group, 4, *([None] * 7), capi.index_view(None),
                                   capi.out_view(None), capi.out_view(None), 2, 8, 4, 0, 1, 1, None)
    assert rc == capi.EINVAL and "one to three groups" in capi.last_error()
    rc = lib.gdn_rssm_commit_plan(*([capi.index_view(None)] * 4), capi.table_view(None), capi.index_view(None),
                                  *([None] * 6), 2, 9, 16, 4, 0, None)
    assert rc == capi.EINVAL and "plan geometry" in capi.last_error()
    rc = lib.gdn_rssm_compact_conv(*([None] * 5), capi.index_view(None), *([None] * 4), 1, 2, 1, 4, 16, 3, 2, 8, 0,
                                   capi.F32, 0, None)
    assert rc == capi.EINVAL and "window" in capi.last_error()


@pytest.mark.parametrize(
    "conv_dim,history,window,match",
    [
        (16, 9, 12, "conv history longer than 8 tokens"),
        (16, 3, 65, "window longer than 64"),
        (65535 * 64 + 1, 3, 6, "too many channels"),
        (16, 0, 6, "shorter than its window"),
    ],
)
def test_capi_compact_conv_rejects_geometry(conv_dim, history, window, match):
    from gdn_recoverssm_b200 import capi

    lib = capi.lib()
    # plan_len, rows, layers, capacity, conv_dim, history, window, num_blocks, null, dtype, align
    rc = lib.gdn_rssm_compact_conv(*([None] * 5), capi.index_view(None), *([None] * 4), 8, 2, 1, 4, conv_dim,
                                   history, window, 8, 0, capi.BF16, 1, None)
    assert rc == capi.EINVAL and match in capi.last_error()


# ---- Python entry points -------------------------------------------------- #
def test_record_geometry_bytes_matches_reference_deployment():
    from gdn_recoverssm_b200 import kernels

    kw = dict(rows=128, num_layers=48, num_value_heads=12, num_key_heads=4, window=4, key_dim=128, value_dim=128)
    # reference test_record_buffers.py:112-137: deployed TP4 geometry
    assert kernels.record_geometry_bytes(**kw, key_dtype=torch.float32) == 193.125 * 1024**2
    assert kernels.record_geometry_bytes(**kw, key_dtype=torch.bfloat16) == 169.125 * 1024**2
    rec = kernels.ReplayRecordBuffers.allocate(3, 6, 2, 4, 8, 8, device="cpu", key_dtype=torch.bfloat16)
    assert rec.shape == (3, 6, 4, 17)
    assert kernels.record_nbytes(rec) == kernels.record_geometry_bytes(3, 1, 6, 2, 4, 8, 8, torch.bfloat16)
    with pytest.raises(ValueError, match="GDN RecoverSSM: record head/row geometry is invalid"):
        kernels.ReplayRecordBuffers.allocate(3, 6, 4, 4, 8, 8, device="cpu")


def _verify_inputs(T=8, H=2, HV=4, D=32, Q=4):
    return dict(
        g=torch.zeros(1, T, HV), beta=torch.ones(1, T, HV), q=torch.zeros(1, T, H, D, dtype=torch.bfloat16),
        k=torch.zeros(1, T, H, D, dtype=torch.bfloat16), v=torch.zeros(1, T, HV, D, dtype=torch.bfloat16),
        checkpoint_state=torch.zeros(5, HV, D, D), replay_cache=torch.zeros(2, HV, Q, 2 * D + 1),
        query_start_loc=torch.tensor([0, 4, 8], dtype=torch.int32),
        state_indices=torch.tensor([1, 2], dtype=torch.int32), spec_query_len=Q,
    )


@pytest.mark.parametrize(
    "change,match",
    [
        (dict(q=torch.zeros(8, 2, 32)), "q must have shape"),
        (dict(spec_query_len=9), r"spec_query_len must be in \[1, 8\]"),
        (dict(replay_cache=torch.zeros(2, 4, 4, 64)), "packed replay record shape"),
        (dict(checkpoint_state=torch.zeros(5, 4, 32, 16)), "checkpoint shape is incompatible"),
        (dict(query_start_loc=torch.tensor([0, 4], dtype=torch.int32)), "query metadata is incompatible"),
        (dict(g=torch.zeros(1, 7, 4)), "gate or beta shape"),
        (dict(replay_cache=torch.zeros(2, 4, 4, 65, dtype=torch.float16)), "packed records must remain FP32"),
    ],
)
def test_verify_argument_errors_raise_before_launch(change, match):
    from gdn_recoverssm_b200 import gdn_recoverssm_verify

    kw = _verify_inputs()
    kw.update(change)
    g, beta, q, k, v = (kw.pop(n) for n in ("g", "beta", "q", "k", "v"))
    with pytest.raises(ValueError, match="GDN RecoverSSM: " + match):
        gdn_recoverssm_verify(g, beta, q, k, v, **kw)


def _gated_inputs(**over):
    kw = _verify_inputs()
    g, beta = kw.pop("g"), kw.pop("beta")
    kw.update(a=g, b=beta, A_log=torch.zeros(4), dt_bias=torch.zeros(4))
    kw.update(over)
    return kw


@pytest.mark.parametrize(
    "change,match",
    [
        (dict(A_log=torch.zeros(3)), "A_log or dt_bias shape is incompatible"),
        (dict(dt_bias=torch.zeros(1, 4)), "A_log or dt_bias shape is incompatible"),
        (dict(A_log=torch.zeros(4, dtype=torch.float64)), "A_log and dt_bias must be FP32"),
        (dict(a=torch.zeros(1, 8, 4, dtype=torch.float16)), "a must be FP32 or the activation dtype"),
        (dict(b=torch.zeros(1, 8, 3)), "gate or beta shape"),
        (dict(softplus_beta=0.0), "softplus_beta must be positive"),
        (dict(spec_query_len=0), r"spec_query_len must be in \[1, 8\]"),
    ],
)
def test_verify_gated_argument_errors_raise_before_launch(change, match):
    from gdn_recoverssm_b200 import gdn_recoverssm_verify_gated

    kw = _gated_inputs(**change)
    A_log, a, b, dt_bias, q, k, v = (kw.pop(n) for n in ("A_log", "a", "b", "dt_bias", "q", "k", "v"))
    with pytest.raises(ValueError, match="GDN RecoverSSM: " + match):
        gdn_recoverssm_verify_gated(A_log, a, b, dt_bias, q, k, v, **kw)


def test_verify_gated_collects_one_native_launch():
    from gdn_recoverssm_b200 import gdn_recoverssm_verify_gated

    kw = _gated_inputs()
    A_log, a, b, dt_bias, q, k, v = (kw.pop(n) for n in ("A_log", "a", "b", "dt_bias", "q", "k", "v"))
    specs = []
    gdn_recoverssm_verify_gated(A_log, a, b, dt_bias, q, k, v, softplus_beta=2.0, softplus_threshold=15.0,
                                use_qk_l2norm_in_kernel=False, _collect=specs, **kw)
    assert len(specs) == 1 and specs[0].name == "verify_gated"
    args = specs[0].args
    assert args[5] is not None and tuple(args[5].shape) == (4,)
    assert args[14][:8] == [2, 8, 2, 4, 4, 5, 2, 0]
    assert args[16:] == (2.0, 15.0, 1)  # softplus_beta, threshold, flags = packed records, no in-kernel norm


def test_verify_collects_one_native_launch_without_running_it():
    from gdn_recoverssm_b200 import gdn_recoverssm_verify

    kw = _verify_inputs()
    g, beta, q, k, v = (kw.pop(n) for n in ("g", "beta", "q", "k", "v"))
    specs = []
    out = gdn_recoverssm_verify(g, beta, q, k, v, _collect=specs, **kw)
    assert out.shape == (1, 8, 4, 32) and len(specs) == 1 and specs[0].name == "verify"
    config = specs[0].args[12]
    assert len(config) == 28 and config[:8] == [2, 8, 2, 4, 4, 5, 2, 0]


def test_empty_batches_return_without_a_launch():
    """No tokens (or no rows): the output comes back untouched and nothing is
    launched -- the reference returns early the same way (kernels.py:854-856);
    CPU tensors prove that no native op ran."""
    from gdn_recoverssm_b200 import gdn_recoverssm_verify

    kw = _verify_inputs(T=0)
    kw["query_start_loc"] = torch.zeros(3, dtype=torch.int32)
    g, beta, q, k, v = (kw.pop(n) for n in ("g", "beta", "q", "k", "v"))
    out = gdn_recoverssm_verify(g, beta, q, k, v, **kw)
    assert out.shape == (1, 0, 4, 32)
    kw = _verify_inputs(T=0)
    kw.update(query_start_loc=torch.zeros(1, dtype=torch.int32), state_indices=torch.zeros(0, dtype=torch.int32))
    g, beta, q, k, v = (kw.pop(n) for n in ("g", "beta", "q", "k", "v"))
    assert gdn_recoverssm_verify(g, beta, q, k, v, **kw).shape == (1, 0, 4, 32)


def test_cpu_tensors_fail_loudly_in_the_native_op():
    """No CPU fallback: the op refuses non-CUDA tensors."""
    from gdn_recoverssm_b200 import gdn_recoverssm_verify

    kw = _verify_inputs()
    g, beta, q, k, v = (kw.pop(n) for n in ("g", "beta", "q", "k", "v"))
    with pytest.raises(RuntimeError, match="CUDA"):
        gdn_recoverssm_verify(g, beta, q, k, v, **kw)


def _context(g, *, soa=True, dtype=torch.bfloat16, blocks=64, layers=2):
    states = [torch.zeros(blocks, 6, 32, 32) for _ in range(layers)]
    convs = [torch.zeros(blocks, 32, 6, dtype=dtype) for _ in range(layers)]
    if soa:
        recs = [g.ReplayRecordBuffers.allocate(8, 6, 2, 4, 32, 32, device="cpu", key_dtype=dtype) for _ in range(layers)]
    else:
        recs = [torch.zeros(8, 6, 4, 65) for _ in range(layers)]
    return g.GDNRecoverSSMCommitContext.from_tensors(convs, states, recs, spec_query_len=4, max_num_reqs=8)


def test_context_tables_and_validation():
    import gdn_recoverssm_b200 as g

    ctx = _context(g)
    assert ctx.conv_history_len == 3 and ctx.num_blocks == 64 and ctx.record_layout == "soa"
    assert ctx.state_base_addrs.tolist() == [s.data_ptr() for s in ctx.checkpoints]
    assert ctx.key_block_strides.tolist() == [2 * 4 * 32] * 2
    assert ctx.num_key_heads == 2 and ctx.record_rows == 8
    with pytest.raises(ValueError, match="packed and typed records cannot share"):
        g.GDNRecoverSSMCommitContext.from_tensors(
            [torch.zeros(8, 32, 6)] * 2, [torch.zeros(8, 6, 32, 32)] * 2,
            [torch.zeros(8, 6, 4, 65), g.ReplayRecordBuffers.allocate(8, 6, 2, 4, 32, 32, device="cpu")],
            spec_query_len=4, max_num_reqs=8)
    with pytest.raises(ValueError, match="conv state is shorter than its window"):
        g.GDNRecoverSSMCommitContext.from_tensors(
            [torch.zeros(8, 32, 3)], [torch.zeros(8, 6, 32, 32)], [torch.zeros(8, 6, 4, 65)], spec_query_len=4,
            max_num_reqs=8)
    specs = ctx.make_commit_specs(torch.ones(2, dtype=torch.int32), torch.tensor([1, 2], dtype=torch.int32),
                                  torch.tensor([0, 4, 8], dtype=torch.int32))
    assert [s.name for s in specs] == ["commit_plan", "compact_conv", "fold"]
    with pytest.raises(ValueError, match="align metadata is incomplete"):
        ctx.commit(torch.ones(2, dtype=torch.int32), torch.tensor([1, 2], dtype=torch.int32),
                   torch.tensor([0, 4, 8], dtype=torch.int32), block_table=torch.zeros(2, 4, dtype=torch.int32))


def test_context_views_are_made_once_and_share_storage():
    """The plan and table row views a commit passes every step are made once
    at construction: the same tensor objects on every access and every step's
    specs, views of the one plan / table tensor (so a launch's writes show in
    them)."""
    import gdn_recoverssm_b200 as g

    ctx = _context(g)
    rows = (ctx.commit_lens, ctx.final_state_indices, ctx.boundary_state_indices, ctx.boundary_recovery_lens,
            ctx.align_valid, ctx.align_col)
    assert all(a is b for a, b in zip(rows, (ctx.commit_lens, ctx.final_state_indices, ctx.boundary_state_indices,
                                             ctx.boundary_recovery_lens, ctx.align_valid, ctx.align_col)))
    for i, r in enumerate(rows):
        assert r.data_ptr() == ctx.plan[i].data_ptr() and r.shape == ctx.plan[i].shape
    ctx.plan[1].fill_(5)
    assert int(ctx.final_state_indices.sum()) == 5 * ctx.plan.shape[1]
    assert ctx.state_base_addrs is ctx.state_base_addrs and ctx.key_block_strides is ctx.key_block_strides
    assert ctx.state_base_addrs.data_ptr() == ctx.tables.table[0].data_ptr()
    args = (torch.ones(2, dtype=torch.int32), torch.tensor([1, 2], dtype=torch.int32),
            torch.tensor([0, 4, 8], dtype=torch.int32))
    a, b = ctx.make_commit_specs(*args), ctx.make_commit_specs(*args)
    assert all(x is y for x, y in zip(a[-1].args, b[-1].args) if isinstance(x, torch.Tensor) and x.dim() == 1
               and x.dtype == torch.int64), "the fold's table views are the same objects every step"


def _entry(g, context, group=0, align=True):
    from types import SimpleNamespace

    p = SimpleNamespace(
        state_indices=torch.tensor([8, 4], dtype=torch.int32), query_start_loc=torch.tensor([0, 4, 8], dtype=torch.int32),
        request_indices=torch.tensor([2, 0], dtype=torch.int64),
        block_table=(torch.arange(12, dtype=torch.int32).reshape(3, 4) + 2 + 20 * group) if align else None,
        num_computed_tokens=torch.tensor([3, 0, 7], dtype=torch.int32) if align else None, block_size=4 if align else None,
        request_rows=(2, 0), query_lens=(4, 4),
    )
    meta = SimpleNamespace(recoverssm_commit=p, recoverssm_builder=SimpleNamespace(), recoverssm_context=context)
    return g.CommitEntry(meta, p, context)


def _inputs():
    return (torch.tensor([1, 0, 3], dtype=torch.int32), torch.tensor([5, -1, 1], dtype=torch.int32),
            torch.full((6,), -9, dtype=torch.int32), torch.full((6,), 7, dtype=torch.int32))


def test_bucket_builds_three_specs_and_rejects_bad_steps():
    import gdn_recoverssm_b200 as g

    ctxs = [_context(g) for _ in range(3)]
    entries = [_entry(g, c, i) for i, c in enumerate(ctxs)]
    bucket = g.GroupedCommitBucket(ctxs)
    assert bucket.layer_groups.tolist() == [0, 0, 1, 1, 2, 2] and bucket.capacity == 8
    specs = bucket.make_specs(entries, *_inputs())
    assert [s.name for s in specs] == ["grouped_plan", "compact_conv", "fold"]
    sampled, mapping, cols, acc = _inputs()
    with pytest.raises(ValueError, match="must not alias"):
        bucket.make_specs(entries, sampled, mapping, cols, sampled)
    with pytest.raises(ValueError, match="different KV epoch"):
        bucket.make_specs([_entry(g, _context(g))] * 3, *_inputs())
    with pytest.raises(ValueError, match="homogeneous layer layouts"):
        g.GroupedCommitBucket([_context(g), _context(g, dtype=torch.float32)])
    with pytest.raises(ValueError, match="one to three contexts"):
        g.GroupedCommitBucket([_context(g) for _ in range(4)])


def test_coordinator_buckets_and_publication_counts(monkeypatch):
    import gdn_recoverssm_b200 as g
    from gdn_recoverssm_b200 import kernels

    launched = []
    monkeypatch.setattr(kernels._LaunchSpec, "launch", lambda self: launched.append(self.name))
    coord = g.GroupedCommitCoordinator()
    ctxs = [_context(g) for _ in range(3)]
    entries = [_entry(g, c, i) for i, c in enumerate(ctxs)]
    coord.commit([e.metadata for e in entries], *_inputs())
    assert coord.last_group_count == 3 and coord.last_launch_count == 3
    first = next(iter(coord._buckets.values()))
    coord.commit([e.metadata for e in entries], *_inputs())
    assert next(iter(coord._buckets.values())) is first
    # seven homogeneous groups: buckets of 3 + 3 + 1 plus one AND-valid publication
    seven = [_entry(g, _context(g), i % 2) for i in range(7)]
    launched.clear()
    coord.commit([e.metadata for e in seven], *_inputs())
    assert coord.last_launch_count == 10 and launched[-1] == "publish_align"
    assert [len(b.contexts) for b in coord._buckets.values()] == [3, 3, 1]
    # heterogeneous layouts: separate buckets
    mixed = [_entry(g, _context(g)), _entry(g, _context(g, dtype=torch.float32), 1)]
    coord.commit([e.metadata for e in mixed], *_inputs())
    assert coord.last_launch_count == 7 and len(coord._buckets) == 2
    bad = [_entry(g, _context(g)), _entry(g, _context(g), 1)]
    bad[1].payload.block_size = 8
    with pytest.raises(ValueError, match="must agree"):
        coord.commit([e.metadata for e in bad], *_inputs())


def test_algorithmic_byte_model_matches_the_survey_formula():
    """The roofline's byte counts (synthetic.verify_bytes / commit_bytes /
    conv_bytes) at config 2: U*V*K*4 + T*H*K*2*2 + T*HV*V*2 + T*HV*(4+4) +
    T*HV*V*2 + T*HV*(V+K+1)*4 + 8*B for verify; the fold's read + write of
    every working unit, boundary snapshots and accepted records."""
    from types import SimpleNamespace

    from gdn_recoverssm_b200 import synthetic

    B, H, HV, D, Q = 512, 16, 32, 128, 4
    T = B * Q
    act = torch.empty(0, dtype=torch.bfloat16)
    wl = SimpleNamespace(B=B, H=H, HV=HV, D=D, Q=Q, tokens=T, units=B * HV, q=act, a=None,
                         beta=torch.empty(0, dtype=torch.float32),
                         conv=torch.empty(1, 8192, 6, dtype=torch.bfloat16))
    want = (B * HV * D * D * 4 + T * H * D * 2 * 2 + T * HV * D * 2 + T * HV * 8 + T * HV * D * 2
            + T * HV * (2 * D + 1) * 4 + 8 * B)
    assert synthetic.verify_bytes(wl) == want == 1191972864
    lens = torch.tensor([4, 0, 2, 1] * (B // 4))
    working = int((lens > 0).sum())
    fold = working * HV * D * D * 4 * 2 + 3 * HV * D * D * 4 + int(lens.sum()) * HV * (2 * D + 1) * 4 + 24 * B
    assert synthetic.commit_bytes(wl, lens, 3) == fold
    assert synthetic.conv_bytes(wl, lens, 3, 3) == (working + 3) * 8192 * 3 * 2 * 2
    # the dim-first conv pool's sector floor: whole channel blocks of the
    # source (read), the final page (read + write, or write when in place) and
    # each boundary snapshot (read + write, or write when it is the source)
    page = 8192 * 6 * 2
    src = torch.arange(1, B + 1)
    fin = torch.where(torch.arange(B) % 2 == 0, src, src + 1000)  # every other row in place
    bnd = torch.zeros(B, dtype=torch.long)
    written = torch.zeros(B, dtype=torch.bool)
    bnd[2], written[2] = 2000, True     # a distinct boundary page (row 2 works, in place)
    bnd[3], written[3] = src[3], True   # a boundary that is the source (row 3 works)
    n_inplace = int(((lens > 0) & (fin == src)).sum())
    n_moved = working - n_inplace
    want_floor = (working + 2 * n_moved + n_inplace + 2 + 1) * page
    assert synthetic.conv_floor_bytes(wl, lens, src, fin, bnd, written) == want_floor
    wl.a = act  # fused gating: raw a, b in the activation dtype instead of g, beta
    wl.b = act
    assert synthetic.verify_bytes(wl) == want - T * HV * 4
