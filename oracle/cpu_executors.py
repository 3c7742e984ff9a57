"""Torch CPU executors for verify + commit: the timed CPU baseline.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  These restate the
reference's own CPU executors ``_cpu_verify`` / ``_cpu_commit``
(plugin/tests/test_record_buffers.py:264-352: float32 torch, vectorised over
value heads) and additionally vectorise over a chunk of sequence rows so that
one call uses every host thread torch is given.  Semantics follow
``gdn_oracle.verify_batch`` / ``gdn_oracle.fold`` for the benchmark workloads
(packed fp32 records, pre-normalised q/k); they are not used as a parity
reference.
"""

from __future__ import annotations

import torch


def verify_packed(q, k, v, g, beta, state, qsl, state_indices, records, out, *, spec_query_len, scale, row_chunk=32):
    """Batched CPU verify.  q, k ``[T, H, K]``; v, out ``[T, HV, V]``;
    g, beta ``[T, HV]``; state ``[blocks, HV, V, K]`` fp32; records
    ``[R, HV, Q, V+K+1]`` fp32.  Rows with a null slot get zero output."""
    T, H, K = q.shape
    HV, V = v.shape[1], v.shape[2]
    ratio = HV // H
    Q = spec_query_len
    B = state_indices.shape[0]
    nb = state.shape[0]
    for r0 in range(0, B, row_chunk):
        r1 = min(B, r0 + row_chunk)
        rows = torch.arange(r0, r1)
        slots = state_indices[r0:r1].long()
        ok = (slots > 0) & (slots < nb)
        bos = qsl[r0:r1].long()
        qlen = qsl[r0 + 1 : r1 + 1].long() - bos
        s = state[slots.clamp(0, nb - 1)].float().clone()  # [n, HV, V, K]
        for t in range(Q):
            tok = bos + t
            valid = (t < qlen) & (tok >= 0) & (tok < T)
            live = valid & ok
            tk = tok.clamp(0, T - 1)
            kk = k[tk].float().repeat_interleave(ratio, 1)  # [n, HV, K]
            qq = q[tk].float().repeat_interleave(ratio, 1) * scale
            vv = v[tk].float()
            d = torch.exp(g[tk].float())  # [n, HV]
            bb = beta[tk].float()
            s_dec = s * d[:, :, None, None]
            corr = (vv - torch.einsum("nhvk,nhk->nhv", s_dec, kk)) * bb[:, :, None]
            s_new = s_dec + corr[:, :, :, None] * kk[:, :, None, :]
            m = live[:, None, None, None]
            s = torch.where(m, s_new, s)
            o = torch.einsum("nhvk,nhk->nhv", s, qq)
            idx = tok[valid]
            out[idx] = torch.where(live[valid, None, None], o[valid], torch.zeros_like(o[valid])).to(out.dtype)
            lr = rows[live]
            if lr.numel():
                rec = records[lr, :, t]
                rec[:, :, :V] = corr[live]
                rec[:, :, V : V + K] = kk[live]
                rec[:, :, V + K] = d[live]
                records[lr, :, t] = rec
    return out


def fold_packed(state, records, source, lengths, finals, boundaries, boundary_lens, *, rows, row_chunk=32):
    """Batched CPU fold of one layer (per-context plan arrays ``[B]``).  State
    ``[blocks, HV, V, K]`` fp32 updated in place; records packed fp32."""
    nb = state.shape[0]
    V = state.shape[2]
    K = state.shape[3]
    for r0 in range(0, rows, row_chunk):
        r1 = min(rows, r0 + row_chunk)
        src = source[r0:r1].long()
        n = lengths[r0:r1].long()
        fin = finals[r0:r1].long()
        ok = (src > 0) & (src < nb) & (fin > 0) & (fin < nb) & (n > 0)
        if not bool(ok.any()):
            continue
        rows_ok = torch.arange(r0, r1)[ok]
        src, n, fin = src[ok], n[ok], fin[ok]
        bidx = boundaries[r0:r1].long()[ok]
        blen = boundary_lens[r0:r1].long()[ok]
        store_b = (bidx > 0) & (bidx < nb) & (bidx != fin) & (blen > 0)
        h = state[src].float().clone()
        snap = h.clone()
        for t in range(int(n.max())):
            rec = records[rows_ok, :, t]  # [m, HV, V+K+1]
            c, kk, d = rec[:, :, :V], rec[:, :, V : V + K], rec[:, :, V + K]
            h_new = torch.addcmul(h * d[:, :, None, None], c[:, :, :, None], kk[:, :, None, :])
            active = (t < n)[:, None, None, None]
            h = torch.where(active, h_new, h)
            take = (store_b & (blen == t + 1))[:, None, None, None]
            snap = torch.where(take, h, snap)
        sb = store_b.nonzero().flatten()
        if sb.numel():
            state[bidx[sb]] = snap[sb].to(state.dtype)
        state[fin] = h.to(state.dtype)
    return state
