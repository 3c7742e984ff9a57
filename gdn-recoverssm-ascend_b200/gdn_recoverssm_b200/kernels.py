"""RecoverSSM verify + per-context commit for Gated DeltaNet on B200 (sm_100a).

Drop-in host layer for the reference module
``plugin/gdn_recoverssm_ascend/kernels.py``: the same public names, call
signatures, argument checks (``ValueError("GDN RecoverSSM: ...")`` raised
before any launch) and buffer contracts, with every launch going to the
hand-written CUDA kernels through ``torch.ops.gdn_recoverssm_ac`` (the C ABI
in ``include/gdn_recoverssm_b200.h``).  There is no Triton, no dispatch
between backends and no CPU fallback: CPU tensors are rejected by the ops.

Public entry points (reference line numbers):
  * ``gdn_recoverssm_verify``                 kernels.py:700-928
  * ``gdn_recoverssm_verify_gated``           gates fused into the prologue,
    argument names of docs/reference/recoverssm_gdn_upstream.py:175-330
  * ``ReplayRecordBuffers``                   kernels.py:166-247
  * ``record_nbytes`` / ``record_geometry_bytes`` kernels.py:250-294
  * ``GDNRecoverSSMCommitContext.from_tensors`` kernels.py:1421-1565
  * ``GDNRecoverSSMCommitContext.commit`` / ``make_commit_specs``
                                              kernels.py:1648-1676,1823-2052
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass, field
from typing import Any, Callable

import torch

from . import _native
from .tables import LayerTables

NULL_BLOCK_ID = 0  # page 0 is the null page
MAX_SPEC_QUERY_LEN = 8  # window bound of every kernel (kernels.py:101)
SUPPORTED_HEAD_DIMS = (32, 64, 128)

# flags of the extended native ops (include/gdn_recoverssm_b200.h)
_RECORD_PACKED = 1
_NORMALIZE_QK = 2
_ACT_DTYPES = (torch.float32, torch.bfloat16, torch.float16)
_INDEX_DTYPES = (torch.int32, torch.int64)
_FOLD_PACKED = 1


def _require(cond: bool, msg: str) -> None:
    """Argument validation raising ``ValueError`` before any launch, with the
    reference's message format (kernels.py:143-151)."""
    if not cond:
        raise ValueError(f"GDN RecoverSSM: {msg}")


@dataclass
class _LaunchSpec:
    """One native launch: the op and its exact arguments.

    ``make_commit_specs`` / ``GroupedCommitBucket.make_specs`` return these
    without launching, mirroring the reference's spec objects
    (kernels.py:1327-1348); ``launch()`` runs the op on the current stream.
    """

    name: str
    op: Callable
    args: tuple
    kwargs: dict = field(default_factory=dict)

    def launch(self) -> None:
        self.op(*self.args, **self.kwargs)

    def compile_only(self) -> None:
        """Kernels are compiled ahead of time (sm_100a); only resolve the op."""
        _native.ops()


@dataclass(frozen=True)
class ReplayRecordBuffers:
    """Typed (SoA) per-step records: ``correction [rows, HV, Q, V]`` fp32,
    ``key [rows, H, Q, K]`` (one key per GQA key head; pre-normalised
    low-precision keys keep their exact input bits) and ``decay [rows, HV, Q]``
    fp32 (kernels.py:166-247)."""

    correction: torch.Tensor
    key: torch.Tensor
    decay: torch.Tensor

    @property
    def shape(self) -> tuple[int, int, int, int]:
        rows, heads, window, value_dim = self.correction.shape
        return (rows, heads, window, value_dim + self.key.shape[-1] + 1)

    @property
    def dtype(self):
        return torch.float32

    @property
    def device(self):
        return self.correction.device

    @property
    def num_key_heads(self) -> int:
        return int(self.key.shape[1])

    @property
    def key_dtype(self):
        return self.key.dtype

    @property
    def record_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.correction, self.key, self.decay))

    @classmethod
    def allocate(cls, rows, num_value_heads, num_key_heads, window, value_dim, key_dim, *, device,
                 key_dtype=torch.float32):
        _require(
            rows > 0
            and num_key_heads > 0
            and 0 < window <= MAX_SPEC_QUERY_LEN
            and value_dim > 0
            and key_dim > 0
            and num_value_heads > 0
            and num_value_heads % num_key_heads == 0,
            "record head/row geometry is invalid",
        )
        _require(key_dtype in (torch.float16, torch.bfloat16, torch.float32), "record keys require FP16, BF16 or FP32")
        return cls(
            torch.zeros((rows, num_value_heads, window, value_dim), dtype=torch.float32, device=device),
            torch.zeros((rows, num_key_heads, window, key_dim), dtype=key_dtype, device=device),
            torch.zeros((rows, num_value_heads, window), dtype=torch.float32, device=device),
        )


def record_nbytes(record) -> int:
    """Bytes held by one layer's records (packed tensor or typed buffers)."""
    if isinstance(record, ReplayRecordBuffers):
        return record.record_bytes
    return record.numel() * record.element_size()


def record_geometry_bytes(rows, num_layers, num_value_heads, num_key_heads, window, key_dim, value_dim,
                          key_dtype=torch.float32) -> int:
    """Physical bytes of typed records for a model geometry, keys deduplicated
    per key head and stored in ``key_dtype`` (kernels.py:258-294)."""
    _require(min(rows, num_layers, num_value_heads, num_key_heads, window, key_dim, value_dim) > 0,
             "record geometry must be positive")
    _require(num_value_heads % num_key_heads == 0, "value heads must be a multiple of key heads")
    _require(key_dtype in (torch.float16, torch.bfloat16, torch.float32), "record keys require FP16, BF16 or FP32")
    key_bytes = 4 if key_dtype == torch.float32 else 2
    per_token = num_value_heads * value_dim * 4 + num_key_heads * key_dim * key_bytes + num_value_heads * 4
    return rows * num_layers * window * per_token


# --------------------------------------------------------------------------- #
# verify
# --------------------------------------------------------------------------- #
def gdn_recoverssm_verify(
    g: torch.Tensor,
    beta: torch.Tensor,
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    checkpoint_state: torch.Tensor,
    replay_cache,
    query_start_loc: torch.Tensor,
    state_indices: torch.Tensor,
    spec_query_len: int,
    scale: float | None = None,
    qk_already_normalized: bool = True,
    out: torch.Tensor | None = None,
    _collect: list | None = None,
) -> torch.Tensor:
    """Verify a speculative window against its checkpoint without modifying the
    checkpoint (reference kernels.py:700-928).

    ``g`` (log-space decay) and ``beta`` (already sigmoid) are ``[1, T, HV]``
    or ``[T, HV]``; q, k ``[1, T, H, K]``; v ``[1, T, HV, V]``;
    ``checkpoint_state`` ``[blocks, HV, V, K]`` (read-only); ``replay_cache``
    is either a packed fp32 ``[rows, HV, Q, V + K + 1]`` tensor or a
    ``ReplayRecordBuffers``.  ``qk_already_normalized=False`` L2-normalises
    q/k inside the kernel (``x * rsqrt(sum(x^2) + 1e-6)``).  Returns ``out``
    ``[1, T, HV, V]``.  Launches on the current CUDA stream.
    """
    return _verify(g, beta, q, k, v, checkpoint_state, replay_cache, query_start_loc, state_indices, spec_query_len,
                   scale, qk_already_normalized, out, _collect, None)


def gdn_recoverssm_verify_gated(
    A_log: torch.Tensor,
    a: torch.Tensor,
    b: torch.Tensor,
    dt_bias: torch.Tensor,
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    checkpoint_state: torch.Tensor,
    replay_cache,
    query_start_loc: torch.Tensor,
    state_indices: torch.Tensor,
    spec_query_len: int,
    scale: float | None = None,
    softplus_beta: float = 1.0,
    softplus_threshold: float = 20.0,
    use_qk_l2norm_in_kernel: bool = True,
    out: torch.Tensor | None = None,
    _collect: list | None = None,
) -> torch.Tensor:
    """Verify with the gates computed in the kernel prologue from the raw
    model inputs (the fused-gating form of
    ``docs/reference/recoverssm_gdn_upstream.py:175-330``, kernel math :111-150):
    per token and value head ``g = -exp(A_log[h]) * softplus(a + dt_bias[h])``
    with ``softplus(x) = log(1 + exp(sb*x)) / sb`` while ``sb*x <= threshold``
    (``x`` above it), ``decay = exp(g)`` and ``beta = sigmoid(b)``.

    ``a``, ``b`` are ``[T, HV]`` or ``[1, T, HV]`` in FP32 or the activation
    dtype; ``A_log`` and ``dt_bias`` are FP32 ``[HV]``.  Everything else (and
    the records, indexed by request row as in ``gdn_recoverssm_verify``) is
    exactly ``gdn_recoverssm_verify``; ``use_qk_l2norm_in_kernel=True``
    normalises q/k in the kernel.
    """
    HV = v.shape[-2] if v.ndim == 4 else -1
    _require(tuple(A_log.shape) == (HV,) and tuple(dt_bias.shape) == (HV,), "A_log or dt_bias shape is incompatible")
    _require(A_log.dtype == torch.float32 and dt_bias.dtype == torch.float32, "A_log and dt_bias must be FP32")
    _require(A_log.device == q.device and dt_bias.device == q.device, "inputs must be on the same device")
    _require(softplus_beta > 0, "softplus_beta must be positive")
    gate = (A_log.contiguous(), dt_bias.contiguous(), float(softplus_beta), float(softplus_threshold))
    return _verify(a, b, q, k, v, checkpoint_state, replay_cache, query_start_loc, state_indices, spec_query_len,
                   scale, not use_qk_l2norm_in_kernel, out, _collect, gate)


def _verify(g, beta, q, k, v, checkpoint_state, replay_cache, query_start_loc, state_indices, spec_query_len, scale,
            qk_already_normalized, out, _collect, gate):
    """Shared validation and launch of both verify forms; ``gate`` is
    ``(A_log, dt_bias, softplus_beta, softplus_threshold)`` for the fused
    gating form (``g`` / ``beta`` then carry the raw ``a`` / ``b``).

    Every shape and stride tuple is read once: the checks run on every decode
    step, so their host cost is per-step latency."""
    qshape = q.shape
    _require(len(qshape) == 4 and qshape[0] == 1, "q must have shape [1, tokens, heads, dim]")
    _, total, H, K = qshape
    _require(k.shape == qshape, "q and k shapes differ")
    vshape = v.shape
    _require(len(vshape) == 4 and vshape[0] == 1 and vshape[1] == total,
             "v must have shape [1, tokens, value heads, dim]")
    HV, V = vshape[2], vshape[3]
    _require(H > 0 and HV >= H and HV % H == 0, "value heads must be a positive multiple of the q/k heads")
    _require(g.numel() == total * HV and beta.numel() == total * HV, "gate or beta shape is incompatible")
    # [T, HV] as given, else a view (a reshape per call costs host time per step)
    g2 = g if g.shape == (total, HV) else g.reshape(total, HV)
    beta2 = beta if beta.shape == (total, HV) else beta.reshape(total, HV)
    gs, bs = g2.stride(), beta2.stride()
    _require(gs[1] == 1 and bs[1] == 1, "gate and beta heads must be contiguous")
    _require(0 < spec_query_len <= MAX_SPEC_QUERY_LEN, f"spec_query_len must be in [1, {MAX_SPEC_QUERY_LEN}]")
    qs, ks, vs = q.stride(), k.stride(), v.stride()
    _require(qs[3] == 1 and qs[2] == K and ks[3] == 1 and ks[2] == K, "q and k heads must be contiguous")
    _require(vs[3] == 1 and vs[2] == V, "v heads must be contiguous")
    cshape = checkpoint_state.shape
    _require(len(cshape) == 4, "checkpoint must be four-dimensional")
    nb = cshape[0]
    _require(cshape[1] == HV and cshape[2] == V and cshape[3] == K, "checkpoint shape is incompatible")
    _require(K == V and K in SUPPORTED_HEAD_DIMS, f"K and V must be equal and one of {SUPPORTED_HEAD_DIMS}")
    qdt = q.dtype
    if gate is None:
        _require(g2.dtype == torch.float32, "gate must be FP32 log-space decay")
    else:
        _require(g2.dtype in (torch.float32, qdt), "a must be FP32 or the activation dtype")
    _require(beta2.dtype in (torch.float32, qdt), "beta must be FP32 or the activation dtype")
    _require(qdt in _ACT_DTYPES and k.dtype == qdt and v.dtype == qdt, "q/k/v must share one FP32/BF16/FP16 dtype")
    cdt = checkpoint_state.dtype
    _require(cdt == torch.float32 or (cdt == torch.bfloat16 and K >= 64),
             "checkpoint must be FP32 (or BF16 with K >= 64)")
    soa = isinstance(replay_cache, ReplayRecordBuffers)
    if soa:
        corr, key_record, decay_record = replay_cache.correction, replay_cache.key, replay_cache.decay
        rshape = corr.shape
        _require(
            len(rshape) == 4
            and tuple(rshape[1:]) == (HV, spec_query_len, V)
            and tuple(key_record.shape) == (rshape[0], H, spec_query_len, K)
            and tuple(decay_record.shape) == (rshape[0], HV, spec_query_len),
            "typed record geometry is incompatible",
        )
        _require(corr.dtype == decay_record.dtype == torch.float32, "correction and decay records must remain FP32")
        _require(
            key_record.dtype in (torch.float16, torch.bfloat16, torch.float32)
            and (key_record.dtype == torch.float32 or (qk_already_normalized and key_record.dtype == k.dtype)),
            "low-precision key records require already-normalized input dtype",
        )
        rs, key_strides, decay_strides = corr.stride(), key_record.stride(), decay_record.stride()
        _require(rs[-1] == 1 and key_strides[-1] == 1 and decay_strides[-1] == 1,
                 "typed record innermost dimensions must be contiguous")
        key_strides = key_strides[:3]
    else:
        corr = key_record = decay_record = replay_cache
        rshape = corr.shape
        _require(len(rshape) == 4 and rshape[1] == HV and rshape[2] == spec_query_len and rshape[3] == V + K + 1,
                 "packed replay record shape is incompatible")
        _require(corr.dtype == torch.float32, "packed records must remain FP32")
        rs = corr.stride()
        _require(rs[3] == 1, "packed record innermost dimension must be contiguous")
        key_strides = decay_strides = rs[:3]
    _require(rshape[0] >= 1, "replay buffer has no rows")
    sshape, lshape = state_indices.shape, query_start_loc.shape
    _require(len(sshape) == 1, "state indices must be one-dimensional")
    _require(len(lshape) == 1 and lshape[0] == sshape[0] + 1, "query metadata is incompatible")
    batch = sshape[0]
    _require(total <= batch * spec_query_len, "speculative decode input exceeds its activation capacity")
    _require(query_start_loc.dtype in _INDEX_DTYPES and state_indices.dtype in _INDEX_DTYPES,
             "query metadata must be int32 or int64")
    dev = q.device
    _require(
        k.device == dev and v.device == dev and g.device == dev and beta.device == dev
        and checkpoint_state.device == dev and corr.device == dev and key_record.device == dev
        and decay_record.device == dev and query_start_loc.device == dev and state_indices.device == dev
        and (out is None or out.device == dev),
        "inputs must be on the same device",
    )
    if scale is None:
        scale = K**-0.5
    if out is None:
        out = torch.empty(1, total, HV, V, dtype=v.dtype, device=dev)
    os_ = out.stride()
    _require(tuple(out.shape) == (1, total, HV, V) and os_[2] == V and os_[3] == 1 and out.dtype == v.dtype,
             "output shape or layout is incompatible")
    if total == 0 or batch == 0:
        return out
    cs = checkpoint_state.stride()
    config = [
        batch, total, H, HV, spec_query_len, nb, rshape[0], NULL_BLOCK_ID,
        qs[1], ks[1], vs[1], gs[0], bs[0],
        cs[0], cs[1], cs[2],
        rs[0], rs[1], rs[2],
        *key_strides, *decay_strides,
        os_[1], query_start_loc.stride(0), state_indices.stride(0),
    ]
    flags = (0 if soa else _RECORD_PACKED) | (0 if qk_already_normalized else _NORMALIZE_QK)
    if gate is None:
        spec = _LaunchSpec(
            "verify",
            _native.ops().verify_ext,
            (q, k, v, g2, beta2, checkpoint_state, corr, key_record, decay_record, out, query_start_loc,
             state_indices, config, float(scale), flags),
        )
    else:
        A_log, dt_bias, sb, thr = gate
        spec = _LaunchSpec(
            "verify_gated",
            _native.ops().verify_gated_ext,
            (q, k, v, g2, beta2, A_log, dt_bias, checkpoint_state, corr, key_record, decay_record, out,
             query_start_loc, state_indices, config, float(scale), sb, thr, flags),
        )
    if _collect is None:
        spec.launch()
    else:
        _collect.append(spec)
    return out


# --------------------------------------------------------------------------- #
# per-context commit
# --------------------------------------------------------------------------- #
_PLAN_ROWS = ("commit_lens", "final_state_indices", "boundary_state_indices", "boundary_recovery_lens",
              "align_valid", "align_col")


def _same_layout(tensors, signature) -> bool:
    """Every tensor has the first one's ``signature``."""
    first = signature(tensors[0])
    return all(signature(t) == first for t in tensors[1:])


def _record_planes(replays, num_value_heads, value_dim, key_dim, window, device):
    """The correction / key / decay plane of every layer's records and the key
    head count, after checking that all layers share one record geometry
    (packed fp32 ``[R, HV, Q, V + K + 1]`` or typed SoA buffers)."""
    typed = [isinstance(r, ReplayRecordBuffers) for r in replays]
    _require(all(typed) or not any(typed), "packed and typed records cannot share a commit context")
    if not typed[0]:
        ok = all(r.ndim == 4 for r in replays) and _same_layout(
            replays, lambda r: (tuple(r.shape), r.dtype, r.stride()[1:], r.device))
        r0 = replays[0]
        ok = ok and tuple(r0.shape[1:]) == (num_value_heads, window, value_dim + key_dim + 1)
        ok = ok and r0.dtype == torch.float32 and r0.device == device
        _require(ok, "layers need matching packed FP32 replay buffers")
        planes = tuple(replays)
        return planes, planes, planes, num_value_heads
    corrs = tuple(r.correction for r in replays)
    keys = tuple(r.key for r in replays)
    decays = tuple(r.decay for r in replays)
    heads = int(keys[0].shape[1])
    _require(heads > 0 and num_value_heads % heads == 0, "record key heads are incompatible")
    rows = int(corrs[0].shape[0])
    expected = ((rows, num_value_heads, window, value_dim), (rows, heads, window, key_dim),
                (rows, num_value_heads, window))
    ok = all(
        (tuple(c.shape), tuple(k.shape), tuple(d.shape)) == expected and all(t.device == device for t in (c, k, d))
        for c, k, d in zip(corrs, keys, decays)
    )
    ok = ok and all(c.dtype == torch.float32 and d.dtype == torch.float32 for c, d in zip(corrs, decays))
    ok = ok and keys[0].dtype in (torch.float16, torch.bfloat16, torch.float32)
    ok = ok and all(_same_layout(p, lambda t: (t.dtype, t.stride()[1:])) for p in (corrs, keys, decays))
    _require(ok, "layers need matching typed replay geometry/dtypes/strides")
    return corrs, keys, decays, heads


class GDNRecoverSSMCommitContext:
    """Commit state of one set of GDN layers (kernels.py:1399-2052): the
    layers' checkpoint pools, conv pools and records, their per-layer address
    and stride tables (one device tensor, ``tables.LayerTables``) and the
    reusable plan buffers (one int32 tensor, a row per plan array).  Build it
    with ``from_tensors``; the attribute names are the reference's, since the
    serving code and the grouped commit read them."""

    def __init__(self, *, conv_states, checkpoints, replays, planes, num_key_heads, spec_query_len, conv_history_len,
                 max_num_reqs):
        device = checkpoints[0].device
        corrs, keys, decays = planes
        self.checkpoints = tuple(checkpoints)
        self.conv_states = tuple(conv_states)
        self.replays = tuple(replays)
        self.records = list(replays)
        self.spec_query_len = int(spec_query_len)
        self.conv_history_len = int(conv_history_len)
        self.num_blocks = int(checkpoints[0].shape[0])
        self.num_key_heads = int(num_key_heads)
        self.record_layout = "soa" if isinstance(replays[0], ReplayRecordBuffers) else "packed"
        self.record_rows = int(corrs[0].shape[0])
        self.key_dtype = keys[0].dtype
        self.record_bytes = sum(record_nbytes(r) for r in replays)
        self.tables = LayerTables(device, (self.checkpoints, self.conv_states, corrs, keys, decays))
        self.plan = torch.zeros(len(_PLAN_ROWS), max_num_reqs, dtype=torch.int32, device=device)
        self._plan_rows = tuple(self.plan.unbind(0))  # row views made once (per-step host time)
        self.layer_groups = torch.zeros(len(self.checkpoints), dtype=torch.int32, device=device)

    # per-layer tables (row views of self.tables)
    state_base_addrs = property(lambda self: self.tables["state_addr"])
    state_block_strides = property(lambda self: self.tables["state_block"])
    conv_state_base_addrs = property(lambda self: self.tables["conv_addr"])
    conv_state_block_strides = property(lambda self: self.tables["conv_block"])
    conv_state_dim_strides = property(lambda self: self.tables["conv_dim"])
    conv_state_token_strides = property(lambda self: self.tables["conv_token"])
    correction_base_addrs = replay_base_addrs = property(lambda self: self.tables["corr_addr"])
    correction_block_strides = replay_block_strides = property(lambda self: self.tables["corr_block"])
    key_base_addrs = property(lambda self: self.tables["key_addr"])
    key_block_strides = property(lambda self: self.tables["key_block"])
    decay_base_addrs = property(lambda self: self.tables["decay_addr"])
    decay_block_strides = property(lambda self: self.tables["decay_block"])
    # plan buffers (row views of self.plan)
    commit_lens = property(lambda self: self._plan_rows[0])
    final_state_indices = property(lambda self: self._plan_rows[1])
    boundary_state_indices = property(lambda self: self._plan_rows[2])
    boundary_recovery_lens = property(lambda self: self._plan_rows[3])
    align_valid = property(lambda self: self._plan_rows[4])
    align_col = property(lambda self: self._plan_rows[5])

    @classmethod
    def from_tensors(cls, conv_states, checkpoints, replays, *, spec_query_len: int, max_num_reqs: int,
                     conv_dim_first: bool = True) -> "GDNRecoverSSMCommitContext":
        """Check that every layer shares one page layout and bind the layers
        (kernels.py:1421-1565): checkpoints ``[blocks, HV, V, K]``, conv pools
        ``[blocks, dim, window]`` (or ``[blocks, window, dim]`` with
        ``conv_dim_first=False``) with window = history + Q - 1, and packed or
        typed records.  The kernels take raw pointers, so nothing here is
        trusted later."""
        layers = len(checkpoints)
        _require(layers > 0, "commit requires at least one layer")
        _require(len(conv_states) == layers == len(replays), "conv, state and replay lists differ")
        _require(0 < spec_query_len <= MAX_SPEC_QUERY_LEN, f"spec_query_len must be in [1, {MAX_SPEC_QUERY_LEN}]")
        convs = [c if conv_dim_first else c.transpose(-1, -2) for c in conv_states]
        _require(checkpoints[0].ndim == 4, "checkpoint must be four-dimensional")
        blocks, value_heads, value_dim, key_dim = checkpoints[0].shape
        device = checkpoints[0].device
        _require(_same_layout(checkpoints, lambda s: (tuple(s.shape), s.dtype, s.stride()[1:], s.device)),
                 "layers need matching checkpoints")
        corrs, keys, decays, heads = _record_planes(replays, value_heads, value_dim, key_dim, spec_query_len, device)
        _require(convs[0].ndim == 3 and convs[0].shape[0] == blocks,
                 "conv state must be [blocks, dim, window] with the checkpoint's block count")
        _require(_same_layout(convs, lambda c: (tuple(c.shape), c.dtype, c.stride()[1:])) and all(
            c.device == device for c in convs), "layers need matching conv states")
        history = int(convs[0].shape[2]) - spec_query_len + 1
        _require(history > 0, "conv state is shorter than its window")
        return cls(conv_states=convs, checkpoints=checkpoints, replays=replays, planes=(corrs, keys, decays),
                   num_key_heads=heads, spec_query_len=spec_query_len, conv_history_len=history,
                   max_num_reqs=max_num_reqs)

    def _fold_config(self, batch):
        """The fold's 17 configuration fields for ``batch`` rows."""
        ref, soa = self.checkpoints[0], self.record_layout == "soa"
        record = self.replays[0]
        rr = record.correction if soa else record
        typed = (record.key.stride(1), record.key.stride(2), record.decay.stride(1), record.decay.stride(2)) \
            if soa else (0, 0, 0, 0)
        return [batch, len(self.checkpoints), ref.shape[1], self.num_key_heads, self.spec_query_len, self.num_blocks,
                rr.shape[0], self.plan.shape[1], NULL_BLOCK_ID, ref.stride(1), ref.stride(2), rr.stride(1),
                rr.stride(2), *typed]

    def _record_args(self):
        ref, soa = self.checkpoints[0], self.record_layout == "soa"
        record = self.replays[0]
        planes = (record.correction, record.key, record.decay) if soa else (record, record, record)
        t = self.tables
        return (ref, *planes, t["state_addr"], t["state_block"], t["corr_addr"], t["corr_block"], t["key_addr"],
                t["key_block"], t["decay_addr"], t["decay_block"], self.layer_groups)

    def _specs(self, accepted, request_indices, state_indices, qsl, block_table, computed, block_size,
                     commit_conv):
        """The step's launches: plan, conv compaction, fold; the conv compaction
        and the fold are programmatic dependents of the launch before each."""
        ops = _native.ops()
        batch = state_indices.shape[0]
        plan_rows = self._plan_rows[:4]
        specs = [_LaunchSpec("commit_plan", ops.commit_plan, (
            accepted, request_indices, state_indices, qsl, block_table, computed, *self._plan_rows,
            self.spec_query_len, self.num_blocks, block_size))]
        if commit_conv:
            conv, t = self.conv_states[0], self.tables
            specs.append(_LaunchSpec("compact_conv", ops.compact_conv, (
                conv, t["conv_addr"], t["conv_block"], t["conv_dim"], t["conv_token"], self.layer_groups,
                state_indices, *plan_rows, batch, self.plan.shape[1], int(conv.shape[1]), self.conv_history_len,
                int(conv.shape[2]), self.num_blocks, block_table is not None)))
        flags = 0 if self.record_layout == "soa" else _FOLD_PACKED
        specs.append(_LaunchSpec("fold", ops.fold_ext, (
            *self._record_args(), state_indices, *plan_rows, self._fold_config(batch), flags)))
        return specs

    def make_commit_specs(self, num_accepted_tokens, state_indices, query_start_loc, request_indices=None,
                          block_table=None, num_computed_tokens=None, mamba_block_size=None,
                          commit_conv=True) -> tuple:
        """The launch specs of one step, without launching them (kernels.py:1648-1676)."""
        specs: list[_LaunchSpec] = []
        self.commit(num_accepted_tokens, state_indices, query_start_loc, request_indices=request_indices,
                    block_table=block_table, num_computed_tokens=num_computed_tokens,
                    mamba_block_size=mamba_block_size, commit_conv=commit_conv, _collect=specs)
        return tuple(specs)

    def commit(self, num_accepted_tokens, state_indices, query_start_loc, request_indices=None, block_table=None,
               num_computed_tokens=None, mamba_block_size=None, commit_conv=True, _collect=None) -> None:
        """Fold each row's accepted prefix into every layer's checkpoint and
        compact the conv history: plan -> conv -> fold on the current stream
        (kernels.py:1823-2052).  In align mode (block table, computed counts
        and block size given) the state lands in the block holding the last
        committed token and a crossed block boundary is snapshotted mid-fold."""
        batch = state_indices.shape[0]
        if batch == 0:
            return
        _require(state_indices.ndim == 1, "state indices must be one-dimensional")
        _require(batch <= self.commit_lens.shape[0], "commit batch exceeds its plan capacity")
        _require(query_start_loc.ndim == 1 and query_start_loc.shape[0] == batch + 1, "commit metadata is incompatible")
        _require(request_indices is None or request_indices.shape[0] >= batch, "request mapping is too short")
        _require(num_accepted_tokens.ndim == 1 and (request_indices is not None or num_accepted_tokens.shape[0] >= batch),
                 "accepted-token counts are too short")
        align_args = (block_table, num_computed_tokens, mamba_block_size)
        _require(all(x is None for x in align_args) or all(x is not None for x in align_args),
                 "align metadata is incomplete")
        _require(mamba_block_size is None or mamba_block_size >= self.spec_query_len,
                 "align block size must cover one speculative window")
        _require(block_table is None or (block_table.ndim == 2 and block_table.shape[1] > 0),
                 "block table must be two-dimensional with a positive width")
        dev = self.checkpoints[0].device
        _require(
            all(t_ is None or t_.device == dev for t_ in (num_accepted_tokens, state_indices, query_start_loc,
                                                         request_indices, block_table, num_computed_tokens)),
            "commit inputs must be on the same device",
        )
        plan_in = (num_accepted_tokens, request_indices, state_indices, query_start_loc, block_table,
                   num_computed_tokens, int(mamba_block_size or 1))
        specs = self._specs(*plan_in, commit_conv)
        if _collect is not None:
            _collect.extend(specs)
            return
        for spec in specs:
            spec.launch()
        self._last_specs = tuple(specs)


__all__ = [
    "GDNRecoverSSMCommitContext",
    "ReplayRecordBuffers",
    "gdn_recoverssm_verify",
    "record_geometry_bytes",
    "record_nbytes",
    "MAX_SPEC_QUERY_LEN",
    "NULL_BLOCK_ID",
]
