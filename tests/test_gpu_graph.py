"""CUDA-graph capture of the path (the reference's plugin runs verify inside
vLLM's captured decode graphs): verify + commit captured once and replayed
give bit-identical outputs, records and states to eager launches on the same
inputs, for the tensor-core (K = V = 128) and the CUDA-core (K = V = 64)
verify kernels.  And the benchmark's form -- whole steps (verify + every
commit launch) captured several to a graph and the graph replayed -- equals
the same number of eager steps after every replay, in place (config 1: the
state carries from step to step) and through block tables (config 2)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def g():
    import gdn_recoverssm_b200 as pkg
    from gdn_recoverssm_b200 import _native

    _native.ops()
    return pkg


def _step(g, wl, ctx, align_kw, conv):
    g.gdn_recoverssm_verify(wl.g, wl.beta, wl.q, wl.k, wl.v, checkpoint_state=wl.state, replay_cache=wl.records,
                            query_start_loc=wl.qsl, state_indices=wl.state_indices, spec_query_len=wl.Q, out=wl.out)
    ctx.commit(wl.accepted, wl.state_indices, wl.qsl, commit_conv=conv, **align_kw)


@pytest.mark.parametrize("cfg,rows,pool,conv", [(2, 16, 64, False), (2, 16, 64, True), (0, None, None, False)])
def test_captured_step_replays_bit_exactly(g, cfg, rows, pool, conv):
    """The plan, conv compaction and fold are programmatic dependents of the
    kernel before each; captured, they keep those dependencies as graph edges."""
    from gdn_recoverssm_b200 import synthetic

    wl = synthetic.make(cfg, "cuda", seed=5, rows=rows, pool=pool, conv_dim=16)
    align_kw = {}
    if wl.block_table is not None:
        align_kw = dict(block_table=wl.block_table, num_computed_tokens=wl.num_computed,
                        mamba_block_size=wl.block_size)
    ctx = g.GDNRecoverSSMCommitContext.from_tensors([wl.conv], [wl.state], [wl.records], spec_query_len=wl.Q,
                                                    max_num_reqs=wl.B)
    state0, conv0 = wl.state.clone(), wl.conv.clone()

    # eager
    _step(g, wl, ctx, align_kw, conv)
    torch.cuda.synchronize()
    eager = (wl.out.clone(), wl.records.clone(), wl.state.clone(), wl.conv.clone())

    # captured: restore the inputs, capture once, replay
    wl.state.copy_(state0)
    wl.conv.copy_(conv0)
    wl.out.zero_()
    wl.records.zero_()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            _step(g, wl, ctx, align_kw, conv)
    torch.cuda.current_stream().wait_stream(stream)
    wl.state.copy_(state0)  # capture does not run the kernels, but start from the same pool
    wl.conv.copy_(conv0)
    wl.out.zero_()
    wl.records.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(wl.out, eager[0])
    assert torch.equal(wl.records, eager[1])
    assert torch.equal(wl.state, eager[2])
    assert torch.equal(wl.conv, eager[3])
    if conv:
        assert not torch.equal(wl.conv, conv0), "the conv windows were compacted"
    assert int(torch.ops.gdn_recoverssm_ac.device_status()) == 0
    del graph


def _stepper(g, wl):
    ctx = g.GDNRecoverSSMCommitContext.from_tensors([wl.conv], [wl.state], [wl.records], spec_query_len=wl.Q,
                                                    max_num_reqs=wl.B)
    kw = {}
    if wl.block_table is not None:
        kw = dict(block_table=wl.block_table, num_computed_tokens=wl.num_computed, mamba_block_size=wl.block_size)
    specs = ctx.make_commit_specs(wl.accepted, wl.state_indices, wl.qsl, commit_conv=True, **kw)

    def step():
        g.gdn_recoverssm_verify(wl.g, wl.beta, wl.q, wl.k, wl.v, checkpoint_state=wl.state,
                                replay_cache=wl.records, query_start_loc=wl.qsl, state_indices=wl.state_indices,
                                spec_query_len=wl.Q, out=wl.out)
        for sp in specs:
            sp.launch()

    return ctx, step


def _snapshot(wl, ctx):
    return [wl.out.clone(), wl.records.clone(), wl.state.clone(), wl.conv.clone(), ctx.commit_lens.clone(),
            ctx.final_state_indices.clone(), ctx.boundary_state_indices.clone()]


@pytest.mark.parametrize("cfg,rows,pool", [(1, None, None), (2, 64, 320)])
def test_graph_replay_equals_eager_steps(g, cfg, rows, pool):
    from gdn_recoverssm_b200 import synthetic

    eager = synthetic.make(cfg, "cuda", seed=11, conv_dim=24, rows=rows, pool=pool)
    replay = synthetic.make(cfg, "cuda", seed=11, conv_dim=24, rows=rows, pool=pool)
    assert torch.equal(eager.state, replay.state)
    ctx_e, step_e = _stepper(g, eager)
    ctx_r, step_r = _stepper(g, replay)
    step_e()  # one eager step each: lazy set-up outside the capture
    step_r()
    torch.cuda.synchronize()
    per_graph = 2
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(per_graph):
            step_r()
    state_before = replay.state.clone()
    for _ in range(3):
        graph.replay()
        for _ in range(per_graph):
            step_e()
        torch.cuda.synchronize()
        for a, b in zip(_snapshot(eager, ctx_e), _snapshot(replay, ctx_r)):
            assert torch.equal(a, b)
    assert int(torch.ops.gdn_recoverssm_ac.device_status()) == 0
    if cfg == 1:  # in place: the replays carried the state forward
        assert not torch.equal(replay.state, state_before)
    del graph
