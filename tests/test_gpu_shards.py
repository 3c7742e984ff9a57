"""Value-head sharding on one GPU: each rank's CUDA launches equal the slice of
the unsharded run.

For world sizes 2, 4 and 8 and every rank, the rank's workload
(``synthetic.make(..., world=, rank=)``: its value heads, the key heads they
read and a state pool of its heads only, the values being exactly those heads'
values of the unsharded workload) goes through the same verify + commit as a
serving rank launches, and its outputs, records and whole state pool must be
bit-identical to the corresponding head slice of the unsharded run.  This is
the reference's tensor-parallel head split (builder.py:205-208,
startup_patch.py:165-192: ``heads // tp`` per rank) with no collective: no
unit's arithmetic depends on which rank, CTA or wave runs it.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def g():
    import gdn_recoverssm_b200 as pkg
    from gdn_recoverssm_b200 import _native

    _native.ops()
    return pkg


def _run(g, wl):
    g.gdn_recoverssm_verify(wl.g, wl.beta, wl.q, wl.k, wl.v, checkpoint_state=wl.state, replay_cache=wl.records,
                            query_start_loc=wl.qsl, state_indices=wl.state_indices, spec_query_len=wl.Q, out=wl.out)
    ctx = g.GDNRecoverSSMCommitContext.from_tensors([wl.conv], [wl.state], [wl.records], spec_query_len=wl.Q,
                                                    max_num_reqs=wl.B)
    kw = {}
    if wl.block_table is not None:
        kw = dict(block_table=wl.block_table, num_computed_tokens=wl.num_computed, mamba_block_size=wl.block_size)
    ctx.commit(wl.accepted, wl.state_indices, wl.qsl, commit_conv=False, **kw)
    torch.cuda.synchronize()


@pytest.mark.parametrize("cfg", [2, 4])
def test_every_rank_equals_its_slice_of_the_unsharded_run(g, cfg):
    from gdn_recoverssm_b200 import synthetic

    full = synthetic.make(cfg, "cuda", seed=5, conv_dim=8)
    state0 = full.state.clone()
    _run(g, full)
    assert not torch.equal(full.state, state0), "the unsharded commit changed nothing"
    checked = 0
    for world in (2, 4, 8):
        for rank in range(world):
            wl = synthetic.make(cfg, "cuda", seed=5, world=world, rank=rank, conv_dim=8)
            sh = wl.extra["shard"]
            vs, ks = slice(sh.value_begin, sh.value_end), slice(sh.key_begin, sh.key_end)
            assert wl.HV == full.HV // world and wl.H == full.H // world
            # the rank's inputs are its heads' values of the unsharded workload
            assert torch.equal(wl.q, full.q[:, :, ks]) and torch.equal(wl.k, full.k[:, :, ks])
            assert torch.equal(wl.v, full.v[:, :, vs]) and torch.equal(wl.g, full.g[:, vs])
            assert torch.equal(wl.beta, full.beta[:, vs]) and torch.equal(wl.state, state0[:, vs])
            _run(g, wl)
            assert torch.equal(wl.out, full.out[:, :, vs]), f"outputs world {world} rank {rank}"
            assert torch.equal(wl.records, full.records[:, vs]), f"records world {world} rank {rank}"
            assert torch.equal(wl.state, full.state[:, vs]), f"state pool world {world} rank {rank}"
            checked += 1
            del wl
    assert checked == 14
    assert int(torch.ops.gdn_recoverssm_ac.device_status()) == 0
