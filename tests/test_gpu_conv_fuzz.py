"""Randomised conv-history compactions on the GPU against the oracle,
bit-exact.

Each case draws a conv pool geometry (channel counts that do and do not fill
whole 1024-channel chunks and 16-byte copies, windows from Q to Q + 7, bf16,
fp16 and fp32, dim-first and token-first storage), a batch with ragged
windows and accepted counts, and -- in align mode -- block tables whose
boundary and final pages alias the source page or each other on some rows.
The commit runs as a serving step does (plan, conv compaction, fold); every
conv page is then compared with the oracle's compaction driven by the GPU's
own plan arrays (the plan itself is checked separately, bit-exact), and pages
no row names must be unchanged.
"""

import numpy as np
import pytest
import torch

from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu

DTYPES = (torch.bfloat16, torch.float16, torch.float32)


@pytest.fixture(scope="module")
def g():
    import gdn_recoverssm_b200 as pkg
    from gdn_recoverssm_b200 import _native

    _native.ops()
    return pkg


@pytest.mark.parametrize("seed", range(20))
def test_conv_compaction_fuzz(g, seed):
    rng = np.random.default_rng(7000 + seed)
    dev = "cuda"
    Q = int(rng.integers(1, 9))
    hist = int(rng.integers(1, 9))
    window = hist + Q - 1
    dim = int(rng.choice([1, 7, 64, 100, 513, 1024, 1500, 2048, 3001]))
    dtype = DTYPES[seed % 3]
    dim_first = seed % 4 != 1
    align = seed % 5 != 4
    B = int(rng.integers(1, 40))
    blocks = 4 * B + 8
    HV, D = 2, 32
    pages = rng.permutation(np.arange(1, blocks))[: 3 * B].reshape(B, 3)
    src = pages[:, 0].astype(np.int32)
    qlen = rng.integers(0, Q + 1, B)
    qsl = np.concatenate([[0], np.cumsum(qlen)]).astype(np.int32)
    acc = rng.integers(0, Q + 2, B).astype(np.int32)
    kw = {}
    if align:
        bs = max(int(rng.choice([Q, 8, 16, 64])), Q)
        C = rng.integers(0, 4 * bs, B).astype(np.int32)
        W = int(4 * bs // bs + 2)
        bt = np.zeros((B, W), dtype=np.int32)
        col = C // bs
        bt[np.arange(B), col] = pages[:, 1]
        bt[np.arange(B), np.minimum(col + 1, W - 1)] = pages[:, 2]
        for r in range(B):  # aliasing on some rows
            u = rng.random()
            if u < 0.15:
                bt[r, col[r]] = src[r]                   # boundary (or final) page = source
            elif u < 0.3:
                bt[r, min(col[r] + 1, W - 1)] = src[r]   # final page = source
            elif u < 0.4:
                bt[r, col[r]] = bt[r, min(col[r] + 1, W - 1)]  # boundary page = final page
        kw = dict(block_table=torch.tensor(bt, device=dev), num_computed_tokens=torch.tensor(C, device=dev),
                  mamba_block_size=bs)
    if dim_first:
        conv = (torch.randn(blocks, dim, window, device=dev) * 4).to(dtype)
        view = conv
    else:
        conv = (torch.randn(blocks, window, dim, device=dev) * 4).to(dtype)
        view = conv.transpose(1, 2)
    conv0 = view.float().cpu().numpy().copy()
    state = torch.randn(blocks, HV, D, D, device=dev) * 0.1
    rec = torch.zeros(B, HV, Q, 2 * D + 1, device=dev)
    ctx = g.GDNRecoverSSMCommitContext.from_tensors([conv], [state], [rec], spec_query_len=Q, max_num_reqs=B,
                                                    conv_dim_first=dim_first)
    assert ctx.conv_history_len == hist
    ctx.commit(torch.tensor(acc, device=dev), torch.tensor(src, device=dev), torch.tensor(qsl, device=dev), **kw)
    torch.cuda.synchronize()
    assert int(torch.ops.gdn_recoverssm_ac.device_status()) == 0
    lens = ctx.commit_lens[:B].cpu().numpy()
    fin = ctx.final_state_indices[:B].cpu().numpy()
    bnd = ctx.boundary_state_indices[:B].cpu().numpy()
    blen = ctx.boundary_recovery_lens[:B].cpu().numpy()
    want = [conv0.copy()]
    O.compact_conv(want, layer_groups=[0], plan_capacity=ctx.commit_lens.shape[0], rows=B, source=src, lengths=lens,
                   finals=fin, boundaries=bnd, boundary_lens=blen, num_blocks=blocks, history=hist, align=align)
    got = view.float().cpu().numpy()
    bad = np.argwhere(got != want[0])
    assert bad.shape[0] == 0, f"{bad.shape[0]} elements differ, first {bad[:4].tolist()}"
    touched = np.unique(np.concatenate([src, fin, bnd]))
    untouched = np.setdiff1d(np.arange(blocks), touched)
    assert np.array_equal(got[untouched], conv0[untouched])
    assert int((lens > 0).sum()) > 0 or B < 4
