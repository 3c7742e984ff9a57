"""Float64 torch restatement of verify and of the accepted-prefix state, batched
over units so that it checks EVERY unit of the full-size configurations on
the GPU.

TEST INFRASTRUCTURE ONLY: the checker of the CUDA path, never shipped.  It
restates the same launch-level semantics as ``oracle.gdn_oracle.verify_batch``
(reference kernels.py:491-697: null / out-of-pool slots, padding tokens,
record rows, GQA key head ``hv // (HV // H)``) in float64 torch, vectorised over
a range of sequence rows and all value heads, on whatever device its inputs
live.  ``tests/test_torch_reference.py`` pins it to the NumPy oracle on CPU.
"""

from __future__ import annotations

import torch


def _l2_rsqrt(x):
    """``x * rsqrt(sum(x^2) + 1e-6)``: the in-kernel normalisation (kernels.py:644-647)."""
    return x / torch.sqrt((x * x).sum(-1, keepdim=True) + 1e-6)


def verify_rows(q, k, v, g, beta, state, qsl, slots, *, Q, scale=None, normalize=False, rows=None, capture=None):
    """Float64 verify of sequence rows ``rows = (r0, r1)``.

    Inputs as the verify op takes them: q, k ``[T, H, K]``; v ``[T, HV, V]``;
    g, beta ``[T, HV]``; ``state`` the checkpoint pool ``[blocks, HV, V, K]``;
    qsl ``[B + 1]``; slots ``[B]``.  Returns a dict:

    * ``out`` ``[R, Q, HV, V]``: the output of window token ``t`` of each row
      (token ``bos + t``); 0 for a valid token of a null / out-of-pool row; NaN
      where the kernel stores nothing (``t >= qlen`` or the token is outside
      ``[0, T)``);
    * ``records`` ``[R, HV, Q, V + K + 1]``: ``[corr, k_hat, decay]`` of every
      token the kernel records (live slot, valid token), NaN elsewhere --
      whether the row is below ``record_rows`` is the caller's test;
    * ``token`` ``[R, Q]`` (int64): the token index of each window position,
      and ``valid`` ``[R, Q]`` / ``live`` ``[R]`` (bool) the masks above;
    * for each ``name -> counts`` of ``capture`` (``counts`` an int tensor
      ``[B]``): ``name`` ``[R, HV, V, K]``, the state after the row's first
      ``counts[r]`` valid tokens (the checkpoint itself for 0).
    """
    T, H, K = q.shape
    HV, V = v.shape[1], v.shape[2]
    nb = state.shape[0]
    r0, r1 = rows if rows is not None else (0, slots.shape[0])
    R = r1 - r0
    dev = q.device
    if scale is None:
        scale = K**-0.5
    ratio = HV // H
    qsl64 = qsl.to(device=dev, dtype=torch.int64)
    bos = qsl64[r0:r1]
    qlen = qsl64[r0 + 1 : r1 + 1] - bos
    t_idx = torch.arange(Q, device=dev)
    tok = bos[:, None] + t_idx[None, :]
    valid = (t_idx[None, :] < qlen[:, None]) & (tok >= 0) & (tok < T)
    slot = slots[r0:r1].to(device=dev, dtype=torch.int64)
    live = (slot > 0) & (slot < nb)
    tokc = tok.clamp(0, max(T - 1, 0))
    kh = torch.arange(HV, device=dev) // ratio
    qq = q[tokc].double()[:, :, kh]  # [R, Q, HV, K]
    kk = k[tokc].double()[:, :, kh]
    if normalize:
        qq, kk = _l2_rsqrt(qq), _l2_rsqrt(kk)
    vv = v[tokc].double()  # [R, Q, HV, V]
    gg = g[tokc].double()  # [R, Q, HV]
    bb = beta[tokc].double()
    S = state[slot.clamp(0, nb - 1)].double()  # [R, HV, V, K]
    nan = torch.tensor(float("nan"), dtype=torch.float64, device=dev)
    out = torch.full((R, Q, HV, V), float("nan"), dtype=torch.float64, device=dev)
    records = torch.full((R, HV, Q, V + K + 1), float("nan"), dtype=torch.float64, device=dev)
    caps = {}
    counts = {}
    for name, c in (capture or {}).items():
        counts[name] = c.to(device=dev, dtype=torch.int64)[r0:r1]
        caps[name] = torch.where((counts[name] == 0)[:, None, None, None], S, nan)
    for t in range(Q):
        m = valid[:, t] & live  # [R]
        d = torch.exp(gg[:, t])  # [R, HV]
        Sd = S * d[..., None, None]
        kt = kk[:, t]
        corr = (vv[:, t] - torch.einsum("rhvk,rhk->rhv", Sd, kt)) * bb[:, t][..., None]
        Sn = Sd + corr[..., :, None] * kt[..., None, :]
        o = torch.einsum("rhvk,rhk->rhv", Sn, qq[:, t] * scale)
        S = torch.where(m[:, None, None, None], Sn, S)
        zero = valid[:, t] & ~live
        out[:, t] = torch.where(m[:, None, None], o, torch.where(zero[:, None, None], torch.zeros_like(o), nan))
        rec = torch.cat([corr, kt, d[..., None]], dim=-1)
        records[:, :, t] = torch.where(m[:, None, None], rec, nan)
        for name in caps:
            hit = (counts[name] == t + 1)[:, None, None, None]
            caps[name] = torch.where(hit, S, caps[name])
    res = {"out": out, "records": records, "token": tok, "valid": valid, "live": live}
    res.update(caps)
    return res


def rel_errors_per_unit(got, want, dims):
    """Per-unit ``(max|d| / max|want|, ||d|| / ||want||)`` over the trailing
    ``dims`` dimensions (NaN entries of ``want`` ignored); returns the two
    error tensors over the leading dimensions."""
    m = ~torch.isnan(want)
    w = torch.where(m, want, torch.zeros_like(want))
    dlt = torch.where(m, got.double() - w, torch.zeros_like(w))
    red = tuple(range(-dims, 0))
    wmax = w.abs().amax(dim=red)
    wl2 = torch.sqrt((w * w).sum(dim=red))
    emax = dlt.abs().amax(dim=red) / torch.where(wmax > 0, wmax, torch.ones_like(wmax))
    el2 = torch.sqrt((dlt * dlt).sum(dim=red)) / torch.where(wl2 > 0, wl2, torch.ones_like(wl2))
    return emax, el2


def rounded_ok(got, want, mantissa_bits, min_normal_exp):
    """Low-precision outputs ``[..., V]``: each element within one ulp of the
    float64 value (subnormal ulp below the normal range), or within 1e-5 of
    its output vector's largest magnitude -- the floor for near-zero results
    of a cancelling 128-term sum, which no fp32 computation pins to the ulp of
    the result.  NaN entries of ``want`` are not checked."""
    m = ~torch.isnan(want)
    w = torch.where(m, want, torch.zeros_like(want))
    expo = torch.floor(torch.log2(w.abs().clamp_min(1e-300))).clamp_min(min_normal_exp)
    ulp = torch.exp2(expo - mantissa_bits)
    vmax = w.abs().amax(dim=-1, keepdim=True)
    err = (got.double() - w).abs()
    ok = (err <= ulp * 1.01) | (err <= 1e-5 * vmax)
    return ok | ~m
