"""CUDA-graph capture of the path (the reference's plugin runs verify inside
vLLM's captured decode graphs): verify + commit captured once and replayed
give bit-identical outputs, records and states to eager launches on the same
inputs, for the tensor-core (K = V = 128) and the CUDA-core (K = V = 64)
verify kernels."""

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
