"""Float64 NumPy oracle for the GDN RecoverSSM verify + commit path.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): the checker for the CUDA
path, never imported by the shipped package.

Reference citations are ``path:line`` inside the reference project
(``plugin/gdn_recoverssm_ascend/...``, ``plugin/tests/...``).

Every per-unit function works on one (sequence row, value head) "unit": the
state tile is ``S[V, K]`` (value rows, key columns), records are
``[corr(V), k_hat(K), decay(1)]``.  The batch functions restate the launch-level
semantics of each reference kernel, including its masking of null rows,
padding tokens and invalid plan rows, so that the CUDA kernels can be compared
element for element (integer outputs bit-exact, float outputs within 1e-5).
"""

from __future__ import annotations

import numpy as np

NULL_BLOCK_ID = 0  # vllm.v1.attention.backends.utils.NULL_BLOCK_ID (kernels.py:57)
MAX_SPEC_QUERY_LEN = 8  # kernels.py:101


# --------------------------------------------------------------------------- #
# per-unit math (plugin/tests/test_math_oracle.py)
# --------------------------------------------------------------------------- #
def softplus(x, beta=1.0, threshold=20.0):
    """Overflow-safe softplus (test_math_oracle.py:25-26); ``beta`` and
    ``threshold`` as in docs/reference/recoverssm_gdn_upstream.py:141-145
    (``log(1 + exp(beta*x)) / beta`` while ``beta*x <= threshold``, else x)."""
    x = np.asarray(x, dtype=np.float64)
    bx = beta * x
    return np.where(bx > threshold, x, np.log1p(np.exp(np.minimum(bx, threshold))) / beta)


def gdn_gate(a_log, dt_bias, a, beta=1.0, threshold=20.0):
    """Log-space decay ``g = -exp(A_log) * softplus(a + dt_bias)`` (test_math_oracle.py:29-31;
    upstream verify prologue docs/reference/recoverssm_gdn_upstream.py:111-146)."""
    return -np.exp(a_log) * softplus(np.asarray(a, np.float64) + dt_bias, beta, threshold)


def sigmoid(b):
    """``beta = sigmoid(b)`` of the upstream prologue (recoverssm_gdn_upstream.py:147-151)."""
    return 1.0 / (1.0 + np.exp(-np.asarray(b, np.float64)))


def l2_unit(x):
    """``x / max(||x||, 1e-6)`` per last axis -- the NumPy oracle's normalisation
    (test_math_oracle.py:41-42)."""
    x = np.asarray(x, dtype=np.float64)
    return x / np.maximum(np.linalg.norm(x, axis=-1, keepdims=True), 1e-6)


def l2_rsqrt(x):
    """``x * rsqrt(sum(x^2) + 1e-6)`` -- the kernel's in-kernel L2 form, same
    epsilon as FLA ``l2norm_fwd`` (kernels.py:644-647)."""
    x = np.asarray(x, dtype=np.float64)
    return x / np.sqrt(np.sum(x * x, axis=-1, keepdims=True) + 1e-6)


def sequential_reference(state0, q, k, v, g, beta, scale):
    """Plain recurrent GDN decode, one token at a time (test_math_oracle.py:34-53).

    Returns ``(outputs[T, V], final_state[V, K], mids)`` where ``mids[t]`` is the
    state after token ``t``.  q/k are L2-normalised inside (``l2_unit``).
    """
    k_hat, q_hat = l2_unit(k), l2_unit(q)
    s = np.array(state0, dtype=np.float64, copy=True)
    v = np.asarray(v, np.float64)
    outs = np.empty((len(k_hat), v.shape[-1]))
    mids = []
    for t in range(len(k_hat)):
        s = np.exp(g[t]) * s
        corr = beta[t] * (v[t] - s @ k_hat[t])
        s = s + np.outer(corr, k_hat[t])
        mids.append(s.copy())
        outs[t] = (s @ q_hat[t]) * scale
    return outs, s, mids


def verify_records(state0, q, k, v, g, beta, scale):
    """Verify of one unit from a read-only checkpoint: ``(outputs, records)``
    with records ``[corr(V), k_hat(K), decay]`` (test_math_oracle.py:56-75)."""
    k_hat, q_hat = l2_unit(k), l2_unit(q)
    s = np.array(state0, dtype=np.float64, copy=True)
    v = np.asarray(v, np.float64)
    n_v, n_k = v.shape[-1], k_hat.shape[-1]
    outs = np.empty((len(k_hat), n_v))
    recs = np.empty((len(k_hat), n_v + n_k + 1))
    for t in range(len(k_hat)):
        d = np.exp(g[t])
        s = d * s
        corr = beta[t] * (v[t] - s @ k_hat[t])
        s = s + np.outer(corr, k_hat[t])
        outs[t] = (s @ q_hat[t]) * scale
        recs[t, :n_v] = corr
        recs[t, n_v : n_v + n_k] = k_hat[t]
        recs[t, n_v + n_k] = d
    return outs, recs


def commit(state0, records, accepted):
    """Fold the accepted prefix ``h <- h*decay + corr (x) k_hat``
    (test_math_oracle.py:78-92).  ``accepted == 0`` returns the state unchanged."""
    h = np.array(state0, dtype=np.float64, copy=True)
    n_v, n_k = h.shape
    if records.shape[1] != n_v + n_k + 1:
        raise ValueError("record width must be V + K + 1")
    for t in range(int(accepted)):
        r = np.asarray(records[t], np.float64)
        h = h * r[n_v + n_k] + np.outer(r[:n_v], r[n_v : n_v + n_k])
    return h


def commit_plan(num_computed, block_size, accepted, table_width):
    """Align-mode destination arithmetic of one row: ``(final_col,
    boundary_col or None, boundary_len)`` (test_math_oracle.py:156-177;
    kernels.py:999-1035)."""
    end = num_computed + accepted
    final_col = min(max(end - 1, 0) // block_size, table_width - 1)
    next_boundary = (num_computed // block_size + 1) * block_size
    if end >= next_boundary:
        return final_col, next_boundary // block_size - 1, next_boundary - num_computed
    return final_col, None, 0


# --------------------------------------------------------------------------- #
# launch-level semantics
# --------------------------------------------------------------------------- #
def _f64(x):
    return np.asarray(x, dtype=np.float64)


def verify_batch(
    q,
    k,
    v,
    g,
    beta,
    state,
    query_start_loc,
    state_indices,
    *,
    spec_query_len,
    scale=None,
    normalize_qk=False,
    record_rows=None,
    layout="packed",
    out=None,
    records=None,
):
    """Launch-level verify (kernels.py:491-697, host wrapper :700-928).

    Shapes: q, k ``[T, H, K]``; v ``[T, HV, V]``; g, beta ``[T, HV]``; state
    ``[blocks, HV, V, K]``; qsl ``[B + 1]``; state_indices ``[B]``.

    ``out`` (``[T, HV, V]``) and ``records`` (packed ``[R, HV, Q, V+K+1]`` or a
    ``(corr[R,HV,Q,V], key[R,H,Q,K], decay[R,HV,Q])`` tuple) are updated in
    place from their initial contents, so entries the kernel must not touch keep
    their sentinel values.  Semantics:

    * null / out-of-pool slot (``<= 0`` or ``>= blocks``): zero output for
      ``t < min(Q, qlen)`` and in-range tokens, no records (:569-583);
    * token ``t`` is valid iff ``t < qlen`` and ``0 <= bos + t < T`` (:609);
      invalid tokens leave the state unchanged and store nothing (:653-665);
    * records only when ``row < record_rows`` (:604);
    * GQA: key head ``= hv // (HV // H)`` (:559);
    * packed key record = the (optionally normalised) fp32 key; typed (SoA)
      key record is written once per key head by ``hv % ratio == 0`` with the
      raw input key (or the normalised one when normalising in-kernel)
      (:666-697).
    """
    q, k, v, g, beta = map(_f64, (q, k, v, g, beta))
    state = _f64(state)
    T, H, K = q.shape
    HV, V = v.shape[1], v.shape[2]
    Q = int(spec_query_len)
    ratio = HV // H
    if scale is None:
        scale = K**-0.5
    nb = state.shape[0]
    qsl = np.asarray(query_start_loc, dtype=np.int64)
    idx = np.asarray(state_indices, dtype=np.int64)
    B = idx.shape[0]
    if out is None:
        out = np.zeros((T, HV, V))
    if record_rows is None:
        record_rows = (records.shape[0] if layout == "packed" else records[0].shape[0]) if records is not None else B
    for b in range(B):
        bos, eos = int(qsl[b]), int(qsl[b + 1])
        qlen = eos - bos
        slot = int(idx[b])
        for hv in range(HV):
            h = hv // ratio
            if slot <= NULL_BLOCK_ID or slot >= nb:
                for t in range(Q):
                    tok = bos + t
                    if t < qlen and 0 <= tok < T:
                        out[tok, hv] = 0.0
                continue
            s = state[slot, hv].copy()
            rec_ok = b < record_rows
            for t in range(Q):
                tok = bos + t
                if not (t < qlen and 0 <= tok < T):
                    continue  # masked token: no state change, no stores
                qq, kk = q[tok, h].copy(), k[tok, h].copy()
                if normalize_qk:
                    qq, kk = l2_rsqrt(qq), l2_rsqrt(kk)
                d = np.exp(g[tok, hv])
                s = s * d
                corr = (v[tok, hv] - s @ kk) * beta[tok, hv]
                s = s + np.outer(corr, kk)
                out[tok, hv] = s @ (qq * scale)
                if not rec_ok or records is None:
                    continue
                if layout == "packed":
                    records[b, hv, t, :V] = corr
                    records[b, hv, t, V : V + K] = kk
                    records[b, hv, t, V + K] = d
                else:
                    c_rec, k_rec, d_rec = records
                    c_rec[b, hv, t] = corr
                    d_rec[b, hv, t] = d
                    if hv % ratio == 0:
                        k_rec[b, h, t] = kk if normalize_qk else k[tok, h]
    return out, records


def _i32(x):
    """Two's-complement int32 value of an integer (the wrap of the reference
    kernels' ``.to(tl.int32)`` loads and int32 sums)."""
    return (int(x) + (1 << 31)) % (1 << 32) - (1 << 31)


def _load(arr, i, default=None):
    """Bounded table read; the CUDA kernels treat an out-of-range index as an
    invalid row (the reference would read out of bounds)."""
    if 0 <= i < len(arr):
        return int(arr[i])
    return default


def prepare_commit_plan(
    num_accepted,
    state_indices,
    query_start_loc,
    *,
    spec_query_len,
    num_blocks,
    request_indices=None,
    block_table=None,
    num_computed=None,
    block_size=None,
):
    """Per-context commit plan (kernels.py:936-1072).

    Returns dict of int arrays ``[B]``: ``commit_lens, final, boundary,
    boundary_lens, valid, col``.  Differences from the grouped plan that this
    restatement keeps: an invalid boundary page of a VALID row is stored as is
    (only its length is zeroed, :1059-1066), and ``col`` is stored unmasked.
    The accepted and computed counts are loaded as int32 and the align
    arithmetic runs in int32 (:978-1035), so values past 2^31 wrap; the
    divisions only matter on rows with ``computed >= 0`` (the others are
    invalid), where floor and truncating division agree.
    """
    Q = int(spec_query_len)
    src = np.asarray(state_indices, dtype=np.int64)
    qsl = np.asarray(query_start_loc, dtype=np.int64)
    acc = np.asarray(num_accepted, dtype=np.int64)
    B = src.shape[0]
    align = block_table is not None
    res = {n: np.zeros(B, dtype=np.int64) for n in ("commit_lens", "final", "boundary", "boundary_lens", "valid", "col")}
    for r in range(B):
        req = r if request_indices is None else int(request_indices[r])
        a = _load(acc, req)
        a = None if a is None else _i32(a)
        bos, eos = int(qsl[r]), int(qsl[r + 1])
        qlen = _i32(eos - bos)
        source = int(src[r])
        n = min(max(a if a is not None else 0, 0), qlen, Q)
        final, boundary, blen, col = source, NULL_BLOCK_ID, 0, 0
        row_ok = a is not None
        if align:
            c = _load(num_computed, req)
            if c is None or not (0 <= req < block_table.shape[0]):
                row_ok, c = False, 0
            c = _i32(c)
            W = block_table.shape[1]
            end = _i32(c + n)
            col = min(max(_i32(end - 1), 0) // block_size, W - 1)
            final = int(block_table[req, col]) if row_ok else NULL_BLOCK_ID
            nxt = _i32((c // block_size + 1) * block_size)
            crosses = end >= nxt
            blen = _i32(nxt - c)
            bcol = nxt // block_size - 1
            boundary = int(block_table[req, bcol]) if (row_ok and crosses and 0 <= bcol < W) else NULL_BLOCK_ID
        geometry = bos >= 0 and bos <= eos and qlen <= Q
        valid = (
            row_ok
            and NULL_BLOCK_ID < source < num_blocks
            and NULL_BLOCK_ID < final < num_blocks
            and geometry
            and 0 < n <= qlen
        )
        if align:
            valid = valid and c >= 0
            if not (NULL_BLOCK_ID < boundary < num_blocks):
                blen = 0
        res["commit_lens"][r] = n if valid else 0
        res["final"][r] = final if valid else NULL_BLOCK_ID
        res["boundary"][r] = boundary if valid else NULL_BLOCK_ID
        res["boundary_lens"][r] = blen if valid else 0
        res["valid"][r] = int(valid)
        res["col"][r] = col
    return res


def grouped_plan(
    sampled,
    groups,
    *,
    rows,
    plan_capacity,
    spec_query_len,
    align,
    publish=False,
    idx_mapping=None,
    persistent_cols=None,
    persistent_accepted=None,
):
    """Grouped plan over 1-3 KV-cache groups (grouped_commit.py:31-222).

    ``groups`` is a list of dicts with ``state_indices, query_start_loc,
    request_indices, num_blocks`` and, in align mode, ``block_table,
    num_computed, block_size``.  Returns dict of int arrays
    ``[groups * capacity]`` (``source, length, final, boundary, boundary_len,
    valid, col``; entries past ``rows`` of each group are left 0) and applies the
    publication to ``persistent_cols`` / ``persistent_accepted`` in place:
    when every group's row is valid, all share the same column and request, and
    ``slot = idx_mapping[request] >= 0``, write ``cols[slot] = col`` and
    ``accepted[slot] = 1`` (:214-222).  A group-local invalid boundary is
    canonicalised to null before the bucket-wide pool bound could legalise it
    (:192-199).
    """
    Q = int(spec_query_len)
    G = len(groups)
    size = G * plan_capacity
    out = {n: np.zeros(size, dtype=np.int64) for n in ("source", "length", "final", "boundary", "boundary_len", "valid", "col")}
    samp = np.asarray(sampled, dtype=np.int64)
    for row in range(rows):
        all_valid = True
        shared_col = shared_req = None
        for gi, grp in enumerate(groups):
            req = int(grp["request_indices"][row])
            source = int(grp["state_indices"][row])
            qsl = grp["query_start_loc"]
            bos, eos = int(qsl[row]), int(qsl[row + 1])
            qlen = eos - bos
            a = _load(samp, req)
            a = None if a is None else _i32(a)  # loaded .to(tl.int32) (:152)
            row_ok = a is not None
            n = min(max(a if a is not None else 0, 0), qlen, Q)
            final, boundary, blen, col = source, NULL_BLOCK_ID, 0, 0
            computed_ok = True
            nb_g = int(grp["num_blocks"])
            if align:
                c = _load(grp["num_computed"], req)
                bt = grp["block_table"]
                if c is None or not (0 <= req < bt.shape[0]):
                    row_ok, c = False, 0
                bs, W = int(grp["block_size"]), bt.shape[1]
                computed_ok = c >= 0
                pos = c + n
                col = min(max(pos - 1, 0) // bs, W - 1)
                final = int(bt[req, col]) if row_ok else NULL_BLOCK_ID
                nxt = (c // bs + 1) * bs
                crossed = pos >= nxt
                blen = nxt - c
                bcol = nxt // bs - 1
                boundary = int(bt[req, bcol]) if (row_ok and crossed and computed_ok and 0 <= bcol < W) else NULL_BLOCK_ID
            geometry = bos >= 0 and bos <= eos and qlen <= Q
            valid = (
                row_ok
                and geometry
                and NULL_BLOCK_ID < source < nb_g
                and NULL_BLOCK_ID < final < nb_g
                and 0 < n <= qlen
                and computed_ok
            )
            if not (NULL_BLOCK_ID < boundary < nb_g):
                blen, boundary = 0, NULL_BLOCK_ID
            off = gi * plan_capacity + row
            out["source"][off] = source if valid else NULL_BLOCK_ID
            out["length"][off] = n if valid else 0
            out["final"][off] = final if valid else NULL_BLOCK_ID
            out["boundary"][off] = boundary if valid else NULL_BLOCK_ID
            out["boundary_len"][off] = blen if valid else 0
            out["valid"][off] = int(valid)
            out["col"][off] = col
            if gi == 0:
                shared_col, shared_req = col, req
            else:
                all_valid = all_valid and col == shared_col and req == shared_req
            all_valid = all_valid and valid
        if publish and align:
            slot = _load(idx_mapping, shared_req, -1)
            if all_valid and slot >= 0:
                persistent_cols[slot] = shared_col
                persistent_accepted[slot] = 1
    return out


def publish_grouped_align(buckets, request_indices, idx_mapping, persistent_cols, persistent_accepted, rows):
    """Cross-bucket AND-valid publication (grouped_commit.py:531-560).

    ``buckets`` is a list of ``(valid[], col[], capacity, group_count)``.  The
    shared column is bucket 0 / group 0's column of the row.
    """
    for row in range(rows):
        v0, c0 = buckets[0][0], buckets[0][1]
        shared = int(c0[row])
        ok = True
        for valid, col, cap, groups in buckets:
            for gi in range(groups):
                off = gi * cap + row
                ok = ok and int(valid[off]) != 0 and int(col[off]) == shared
        req = int(request_indices[row])
        slot = _load(idx_mapping, req, -1)
        if ok and slot >= 0:
            persistent_cols[slot] = shared
            persistent_accepted[slot] = 1
    del v0


def fold(
    states,
    corrections,
    keys,
    decays,
    *,
    layer_groups,
    plan_capacity,
    rows,
    source,
    lengths,
    finals,
    boundaries,
    boundary_lens,
    num_blocks,
    record_rows,
    layout="packed",
    source_stride=1,
    query_len=MAX_SPEC_QUERY_LEN,
):
    """Multi-layer accepted-prefix fold (grouped_commit.py:325-480; per-context
    variant kernels.py:1172-1324; AscendC fold.h:192-237).

    ``states`` is a list of per-layer pools ``[blocks, HV, V, K]`` (updated in
    place, float64 math, result cast back to the pool dtype).  Records: packed
    list of ``[R, HV, Q, V+K+1]`` (``keys``/``decays`` ignored) or typed lists
    ``corr[R,HV,Q,V]``, ``key[R,H,Q,K]``, ``decay[R,HV,Q]``.

    Per (layer, row, head): plan row ``p = layer_groups[layer] * capacity +
    row``; work only if ``0 < src < blocks``, ``0 < final < blocks``,
    ``0 < n <= query_len`` and ``row < record_rows``.  One fold from the
    ORIGINAL source state; the boundary snapshot is stored mid-fold when
    ``t + 1 == boundary_len`` and the boundary page is valid and differs from
    the final page; the final state is stored last.
    """
    for layer, pool in enumerate(states):
        grp = int(layer_groups[layer])
        HV, V, K = pool.shape[1:]
        for row in range(rows):
            p = grp * plan_capacity + row
            src = int(source[p * source_stride]) if source_stride else int(source[p])
            n = int(lengths[p])
            fin = int(finals[p])
            if not (
                NULL_BLOCK_ID < src < num_blocks
                and NULL_BLOCK_ID < fin < num_blocks
                and 0 < n <= query_len
                and row < record_rows
            ):
                continue
            b_idx, b_len = int(boundaries[p]), int(boundary_lens[p])
            store_b = NULL_BLOCK_ID < b_idx < num_blocks and b_idx != fin and b_len > 0
            h = pool[src].astype(np.float64)  # [HV, V, K], read before any store
            snapshot = None
            for t in range(n):
                if layout == "packed":
                    rec = _f64(corrections[layer][row, :, t])  # [HV, V+K+1]
                    c, kk, d = rec[:, :V], rec[:, V : V + K], rec[:, V + K]
                else:
                    c = _f64(corrections[layer][row, :, t])
                    kh = _f64(keys[layer][row, :, t])
                    kk = np.repeat(kh, HV // kh.shape[0], axis=0)
                    d = _f64(decays[layer][row, :, t])
                h = h * d[:, None, None] + c[:, :, None] * kk[:, None, :]
                if store_b and t + 1 == b_len:
                    snapshot = h.copy()
            if snapshot is not None:
                pool[b_idx] = snapshot.astype(pool.dtype)
            pool[fin] = h.astype(pool.dtype)
    return states


def compact_conv(
    convs,
    *,
    layer_groups,
    plan_capacity,
    rows,
    source,
    lengths,
    finals,
    boundaries,
    boundary_lens,
    num_blocks,
    history,
    align,
    source_stride=1,
    check_boundary_differs=False,
):
    """Conv-window compaction (grouped_commit.py:225-322; per-context
    kernels.py:1075-1169).  ``convs`` are per-layer ``[blocks, dim, len]`` views
    (dim-first).  For a working row: ``final[:, h] = src[:, n - 1 + h]`` and, in
    align mode with a valid boundary page, ``boundary[:, h] = src[:, blen - 1 +
    h]`` for ``h < history``; both windows are read before either store, the
    boundary is stored first.  A row works iff ``src > 0``, ``n != 0`` and
    ``0 < final < blocks``.
    """
    for layer, conv in enumerate(convs):
        grp = int(layer_groups[layer])
        for row in range(rows):
            p = grp * plan_capacity + row
            src = int(source[p * source_stride])
            n = int(lengths[p])
            fin = int(finals[p])
            if not (src > NULL_BLOCK_ID and n != 0 and NULL_BLOCK_ID < fin < num_blocks):
                continue
            fin_vals = conv[src][:, n - 1 : n - 1 + history].copy()
            b_idx, b_len = int(boundaries[p]), int(boundary_lens[p])
            b_vals = None
            if align and NULL_BLOCK_ID < b_idx < num_blocks:
                b_vals = conv[src][:, b_len - 1 : b_len - 1 + history].copy()
            if b_vals is not None:
                conv[b_idx][:, :history] = b_vals
            conv[fin][:, :history] = fin_vals
    return convs


# --------------------------------------------------------------------------- #
# error measures used by the parity tests
# --------------------------------------------------------------------------- #
def rel_errors(got, want):
    """``(max|d| / max|want|, ||d|| / ||want||)`` -- element-wise relative error
    is meaningless on near-zero state entries (selftest.py:97-117), so parity is
    stated against the tensor's scale."""
    got, want = _f64(got), _f64(want)
    d = np.abs(got - want)
    scale_inf = max(float(np.abs(want).max()) if want.size else 0.0, 1e-30)
    scale_2 = max(float(np.linalg.norm(want)), 1e-30)
    return float(d.max() if d.size else 0.0) / scale_inf, float(np.linalg.norm(d)) / scale_2
