"""GPU parity of the conv-history compaction in the commit, on both of its
paths: the contiguous dim-first pool staged through shared memory in chunks
(odd channel counts and windows so that the 16-byte copies leave a tail,
several chunks, bf16 and fp32) and the general-stride path (a token-first
pool passed with ``conv_dim_first=False``).  Align mode with block tables, so
boundary snapshots occur -- among them a boundary page that aliases the
source, one that is the final page, and a final page that is the source --
and the in-place mode without block tables; every page the plan names is
compared bit-exactly with the oracle's compaction, and untouched pages must
stay unchanged.
"""

import numpy as np
import pytest
import torch

from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu

ROWS, H, HV, D, Q, BLOCKS, BLOCK = 24, 2, 4, 32, 4, 96, 16

CASES = [
    # conv channels, window (history = window - Q + 1), dtype, dim-first pool, align mode
    (100, 5, torch.bfloat16, True, True),     # contiguous: tail of the 16-byte copies
    (1500, 6, torch.float32, True, True),     # contiguous: several chunks
    (300, 6, torch.bfloat16, False, True),    # token-first pool: general-stride path
    (1500, 6, torch.bfloat16, True, False),   # contiguous, in place (final page = source)
    (300, 5, torch.float32, False, False),    # general strides, in place
]


@pytest.fixture(scope="module")
def g():
    import gdn_recoverssm_b200 as pkg
    from gdn_recoverssm_b200 import _native

    _native.ops()
    return pkg


def _case_id(c):
    return f"dim{c[0]}-w{c[1]}-{str(c[2])[6:]}-{'dimfirst' if c[3] else 'tokfirst'}-{'align' if c[4] else 'inplace'}"


@pytest.mark.parametrize("case", CASES, ids=_case_id)
def test_conv_compaction_matches_oracle(g, case):
    dim, window, dtype, dim_first, align = case
    rng = np.random.default_rng(dim + window)
    dev = "cuda"
    ids = rng.permutation(np.arange(1, BLOCKS))[: 3 * ROWS].reshape(ROWS, 3)
    src = ids[:, 0].astype(np.int32)
    C = rng.integers(0, 256, ROWS)
    C[:6] = BLOCK - 2
    W = -(-(256 + Q) // BLOCK)
    bt = np.zeros((ROWS, W), dtype=np.int32)
    bt[np.arange(ROWS), C // BLOCK] = ids[:, 1]
    bt[np.arange(ROWS), np.minimum(C // BLOCK + 1, W - 1)] = ids[:, 2]
    # rows 3-5 cross a block (C = BLOCK - 2, Q accepted): boundary column
    # C // BLOCK, final column C // BLOCK + 1
    bt[3, C[3] // BLOCK] = src[3]  # the boundary page is the source
    bt[4, C[4] // BLOCK] = bt[4, C[4] // BLOCK + 1]  # the boundary page is the final page
    bt[5, C[5] // BLOCK + 1] = src[5]  # the final page is the source
    acc = rng.integers(1, Q + 1, ROWS).astype(np.int32)
    acc[:6] = Q
    qsl = (np.arange(ROWS + 1) * Q).astype(np.int32)

    if dim_first:
        conv = torch.randn(BLOCKS, dim, window, device=dev).to(dtype)
        conv_view = conv
    else:  # token-first storage, passed transposed
        conv = torch.randn(BLOCKS, window, dim, device=dev).to(dtype)
        conv_view = conv.transpose(1, 2)
    conv0 = conv_view.float().cpu().numpy().copy()
    state = torch.randn(BLOCKS, HV, D, D, device=dev) * 0.1
    rec = torch.zeros(ROWS, HV, Q, 2 * D + 1, device=dev)
    ctx = g.GDNRecoverSSMCommitContext.from_tensors([conv], [state], [rec], spec_query_len=Q, max_num_reqs=ROWS,
                                                    conv_dim_first=dim_first)
    kw = {}
    if align:
        kw = dict(block_table=torch.tensor(bt, device=dev), num_computed_tokens=torch.tensor(C.astype(np.int32), device=dev),
                  mamba_block_size=BLOCK)
    ctx.commit(torch.tensor(acc, device=dev), torch.tensor(src, device=dev), torch.tensor(qsl, device=dev), **kw)
    torch.cuda.synchronize()
    assert int(torch.ops.gdn_recoverssm_ac.device_status()) == 0

    lens = ctx.commit_lens[:ROWS].cpu().numpy()
    fin = ctx.final_state_indices[:ROWS].cpu().numpy()
    bnd = ctx.boundary_state_indices[:ROWS].cpu().numpy()
    blen = ctx.boundary_recovery_lens[:ROWS].cpu().numpy()
    if align:
        assert ((bnd > 0) & (blen > 0)).any(), "the case takes boundary snapshots"
        assert bnd[3] == src[3] and bnd[4] == fin[4] and fin[5] == src[5], "the aliasing rows"
    else:
        assert np.array_equal(fin, src), "in place without block tables"
    want = [conv0.copy()]
    O.compact_conv(want, layer_groups=[0], plan_capacity=ctx.commit_lens.shape[0], rows=ROWS, source=src,
                   lengths=lens, finals=fin, boundaries=bnd, boundary_lens=blen, num_blocks=BLOCKS,
                   history=ctx.conv_history_len, align=align)
    got = conv_view.float().cpu().numpy()
    assert np.array_equal(got, want[0])
    touched = np.unique(np.concatenate([src, fin, bnd]))
    untouched = np.setdiff1d(np.arange(BLOCKS), touched)
    assert np.array_equal(got[untouched], conv0[untouched])
