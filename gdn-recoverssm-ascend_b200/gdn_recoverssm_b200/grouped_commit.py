"""Step-owned grouped recovery: one plan, one conv pass, one fold per bucket.

Drop-in host layer for the reference module
``plugin/gdn_recoverssm_ascend/grouped_commit.py``: ``CommitEntry``,
``GroupedCommitBucket`` (``__init__`` / ``make_specs``) and
``GroupedCommitCoordinator.commit`` keep the reference's signatures, bucketing
rules and ``ValueError`` messages; the three launches per bucket (plan, conv
compaction, fold) and the cross-bucket publication go to the CUDA kernels via
``torch.ops.gdn_recoverssm_ac``.

A bucket holds one to three KV-cache groups (commit contexts) that share one
layer layout and one set of logical rows; plan row of (layer, row) is
``layer_groups[layer] * capacity + row``.  All per-layer tables of a bucket
live in one device tensor (``tables.LayerTables``) and all seven plan arrays
in one int32 tensor, a row each.
"""

from __future__ import annotations

import logging
from dataclasses import dataclass
from typing import Any, NamedTuple

import torch

from . import _native
from .kernels import _FOLD_PACKED, NULL_BLOCK_ID, _LaunchSpec
from .tables import LayerTables, as_int64_bits

logger = logging.getLogger("gdn_recoverssm_b200.grouped_commit")

MAX_GROUPS_PER_BUCKET = 3  # the flat three-group launch of the reference plan kernel (grouped_commit.py:31-222)


@dataclass(frozen=True)
class CommitEntry:
    """One GDN group's part of a step: its attention metadata, the commit
    payload the metadata builder attached, and the commit context it binds."""

    metadata: Any
    payload: Any
    context: Any


class _Plane(NamedTuple):
    """What two layers' tensors of one kind must share to be addressed by the
    same launch: dtype and the per-page (or per-row) strides, plus the page
    shape where the kernels read it from the reference tensor."""

    dtype: Any
    shape: tuple | None
    strides: tuple


def _plane(t, with_shape=True) -> _Plane:
    return _Plane(t.dtype, tuple(t.shape[1:]) if with_shape else None, tuple(t.stride()[1:]))


class _Layout(NamedTuple):
    """Layout signature of a commit context (grouped_commit.py:490-517): two
    contexts share a bucket only when every field agrees."""

    device: Any
    state: _Plane
    conv: _Plane
    conv_history: int
    window: int
    record_layout: str
    key_heads: int
    correction: _Plane
    key: _Plane
    decay: _Plane


def _record_planes(rec, layout):
    """(correction, key, decay) planes of one layer's records (the packed
    tensor three times over)."""
    if layout == "soa":
        return rec.correction, rec.key, rec.decay
    return rec, rec, rec


def _planes_of(context):
    return _record_planes(context.records[0], context.record_layout)


def _layout_of(context) -> _Layout:
    corr, key, decay = _planes_of(context)
    state = context.checkpoints[0]
    return _Layout(
        device=state.device, state=_plane(state), conv=_plane(context.conv_states[0]),
        conv_history=context.conv_history_len, window=context.spec_query_len, record_layout=context.record_layout,
        key_heads=context.num_key_heads, correction=_plane(corr, False), key=_plane(key, False),
        decay=_plane(decay, False),
    )


def _row_evidence(entry):
    """The step's logical rows as the host knows them (grouped_commit.py:520-528):
    ``("rows", request rows, query lengths, block size, align)`` when the
    payload carries per-row host evidence for every row, else an identity
    that matches no other entry -- without that evidence a group cannot share
    a launch with another group."""
    payload = entry.payload
    rows = int(payload.state_indices.shape[0])
    request_rows = tuple(getattr(payload, "request_rows", ()))
    query_lens = tuple(getattr(payload, "query_lens", ()))
    if len(request_rows) == rows == len(query_lens):
        return ("rows", request_rows, query_lens, payload.block_size, payload.block_table is not None)
    return ("opaque", id(entry.metadata))


def _publisher_descriptors(buckets):
    """Device table of (valid ptr, col ptr, capacity, groups) per bucket for
    the cross-bucket publication, cached on the first bucket while the same
    plan buffers are in use; it keeps those buffers referenced."""
    owner = buckets[0]
    key = tuple((id(b.plan), b.capacity, len(b.contexts)) for b in buckets)
    if getattr(owner, "_publisher_key", None) != key:
        rows = [(as_int64_bits(b.valid.data_ptr()), as_int64_bits(b.col.data_ptr()), b.capacity, len(b.contexts))
                for b in buckets]
        owner._publisher_descriptors = torch.tensor([v for r in rows for v in r], dtype=torch.int64,
                                                    device=owner.device)
        owner._publisher_plan_owners = tuple(b.plan for b in buckets)
        owner._publisher_key = key
    return owner._publisher_descriptors


def _publish_spec(buckets, request_indices, idx_mapping, persistent_cols, persistent_accepted, rows):
    """AND-valid publication after every bucket committed (grouped_commit.py:531-610)."""
    return _LaunchSpec(
        "publish_align",
        _native.ops().publish_align,
        (_publisher_descriptors(buckets), request_indices, idx_mapping, persistent_cols, persistent_accepted, rows),
    )


_PLAN_ROWS = ("source", "length", "final", "boundary", "boundary_len", "valid", "col")


class GroupedCommitBucket:
    """Per-layer tables and per-group plan storage of one KV epoch: the
    contexts of one to three GDN groups (grouped_commit.py:613-893)."""

    def __init__(self, contexts):
        contexts = tuple(contexts)
        if not 0 < len(contexts) <= MAX_GROUPS_PER_BUCKET:
            raise ValueError("one recovery bucket requires one to three contexts")
        layout = _layout_of(contexts[0])
        if any(_layout_of(c) != layout for c in contexts[1:]):
            raise ValueError("grouped recovery requires homogeneous layer layouts")
        capacity = min(int(c.record_rows) for c in contexts)
        if capacity <= 0:
            raise ValueError("grouped recovery has no record rows")
        self.contexts = contexts
        self.capacity = capacity
        self.device = layout.device
        self.spec_query_len = layout.window
        self.record_layout = layout.record_layout
        self.num_key_heads = layout.key_heads
        self.conv_history_len = layout.conv_history
        # layers in group order; layer_groups maps each to its group's plan rows
        members = [(g, i) for g, c in enumerate(contexts) for i in range(len(c.checkpoints))]
        self.checkpoints = tuple(contexts[g].checkpoints[i] for g, i in members)
        self.conv_states = tuple(contexts[g].conv_states[i] for g, i in members)
        self.records = tuple(contexts[g].records[i] for g, i in members)
        self.layer_groups = torch.tensor([g for g, _ in members], dtype=torch.int32, device=self.device)
        planes = [_record_planes(r, self.record_layout) for r in self.records]
        self.corrections, self.keys, self.decays = (tuple(p[j] for p in planes) for j in range(3))
        self.tables = LayerTables(self.device, (self.checkpoints, self.conv_states, self.corrections, self.keys,
                                                self.decays))
        # the fold bounds pages by the largest pool; the grouped plan bounds
        # every group's pages by its own pool, and the op checks the bound
        # against the tensor it is given: the largest pool
        self.max_blocks = max(int(c.num_blocks) for c in contexts)
        self._largest_pool = max(self.checkpoints, key=lambda t: t.shape[0])
        self.plan = torch.zeros(len(_PLAN_ROWS), capacity * len(contexts), dtype=torch.int32, device=self.device)
        self._plan_rows = tuple(self.plan.unbind(0))  # row views made once (per-step host time)

    source = property(lambda self: self._plan_rows[0])
    length = property(lambda self: self._plan_rows[1])
    final = property(lambda self: self._plan_rows[2])
    boundary = property(lambda self: self._plan_rows[3])
    boundary_len = property(lambda self: self._plan_rows[4])
    valid = property(lambda self: self._plan_rows[5])
    col = property(lambda self: self._plan_rows[6])
    state_addrs = property(lambda self: self.tables["state_addr"])
    state_block_strides = property(lambda self: self.tables["state_block"])
    conv_addrs = property(lambda self: self.tables["conv_addr"])
    conv_block_strides = property(lambda self: self.tables["conv_block"])
    conv_dim_strides = property(lambda self: self.tables["conv_dim"])
    conv_token_strides = property(lambda self: self.tables["conv_token"])
    correction_addrs = property(lambda self: self.tables["corr_addr"])
    correction_block_strides = property(lambda self: self.tables["corr_block"])
    key_addrs = property(lambda self: self.tables["key_addr"])
    key_block_strides = property(lambda self: self.tables["key_block"])
    decay_addrs = property(lambda self: self.tables["decay_addr"])
    decay_block_strides = property(lambda self: self.tables["decay_block"])

    def _step_payloads(self, entries, sampled, idx_mapping, persistent_cols, persistent_accepted):
        """Validate one step's entries against this bucket (grouped_commit.py:670-726)
        and return ``(payloads, rows, align)``."""
        if len(entries) != len(self.contexts) or any(e.context is not c for e, c in zip(entries, self.contexts)):
            raise ValueError("grouped recovery bucket belongs to a different KV epoch")
        payloads = tuple(e.payload for e in entries)
        row_counts = [int(p.state_indices.shape[0]) for p in payloads]
        rows = row_counts[0]
        if not 0 < rows <= self.capacity:
            raise ValueError(
                f"grouped recovery rows out of range: rows={rows}, record capacity={self.capacity}, "
                f"groups={len(payloads)}, state_indices shapes={[tuple(p.state_indices.shape) for p in payloads]}"
            )
        if len(set(row_counts)) != 1:
            raise ValueError("grouped recovery row counts differ")
        modes = {p.block_table is not None for p in payloads}
        if len(modes) != 1:
            raise ValueError("grouped recovery cannot mix align and none plans")
        align = modes.pop()
        if any(p.request_indices is None for p in payloads):
            raise ValueError("grouped recovery requires an explicit native row mapping")
        per_group = ("state_indices", "query_start_loc", "request_indices") + (
            ("block_table", "num_computed_tokens") if align else ())
        inputs = [sampled, idx_mapping, persistent_accepted] + [getattr(p, n) for p in payloads for n in per_group]
        if align:
            inputs.append(persistent_cols)
        if any(t is None or t.device != self.device for t in inputs):
            raise ValueError("grouped recovery inputs must share the checkpoint device")
        if sampled.data_ptr() == persistent_accepted.data_ptr():
            raise ValueError("sampled counts must not alias persistent acceptance output")
        for p in payloads:
            self._check_group(p, rows, align, sampled, idx_mapping)
        return payloads, rows, align

    def _check_group(self, payload, rows, align, sampled, idx_mapping):
        if payload.query_start_loc.numel() < rows + 1:
            raise ValueError("grouped recovery offsets are shorter than their rows")
        if align:
            if payload.block_size is None or payload.block_size < self.spec_query_len:
                raise ValueError("align blocks must cover the speculative window")
            if payload.block_table.shape[1] <= 0:
                raise ValueError("align block table has no columns")
        host_rows = tuple(getattr(payload, "request_rows", ()))
        limit = min(sampled.numel(), idx_mapping.numel())
        if len(host_rows) == rows and not all(0 <= r < limit for r in host_rows):
            raise ValueError("native request mapping exceeds the sampled batch")

    @staticmethod
    def _group_lists(payloads, contexts, align):
        """The grouped plan's per-group inputs, list by list."""
        groups = list(zip(payloads, contexts))
        return (
            [p.state_indices for p, _ in groups],
            [p.query_start_loc for p, _ in groups],
            [p.request_indices for p, _ in groups],
            [p.block_table if align else None for p, _ in groups],
            [p.num_computed_tokens if align else None for p, _ in groups],
            [int(c.num_blocks) for _, c in groups],
            [int(p.block_size) if align else 1 for p, _ in groups],
        )

    def make_specs(self, entries, sampled, idx_mapping, persistent_cols, persistent_accepted, *, publish_align=True):
        """Validate one step's entries and return the (plan, conv, fold)
        launch specs without launching them (grouped_commit.py:670-893)."""
        payloads, rows, align = self._step_payloads(entries, sampled, idx_mapping, persistent_cols,
                                                    persistent_accepted)
        ops = _native.ops()
        plan = _LaunchSpec("grouped_plan", ops.grouped_plan, (
            sampled, *self._group_lists(payloads, self.contexts, align), *self._plan_rows,
            idx_mapping, persistent_cols if align else None, persistent_accepted if align else None,
            rows, self.capacity, self.spec_query_len, align, bool(align and publish_align),
        ))
        plan_views = (self.source, self.length, self.final, self.boundary, self.boundary_len)
        conv = self.conv_states[0]
        compact = _LaunchSpec("compact_conv", ops.compact_conv, (
            conv, self.conv_addrs, self.conv_block_strides, self.conv_dim_strides, self.conv_token_strides,
            self.layer_groups, *plan_views, rows, self.capacity, int(conv.shape[1]), self.conv_history_len,
            int(conv.shape[2]), self.max_blocks, align,
        ))
        fold = _LaunchSpec("fold", ops.fold_ext, self._fold_args(rows, plan_views))
        return plan, compact, fold

    def _fold_args(self, rows, plan_views):
        soa = self.record_layout == "soa"
        state, corr, key, decay = self._largest_pool, self.corrections[0], self.keys[0], self.decays[0]
        typed = (key.stride(1), key.stride(2), decay.stride(1), decay.stride(2)) if soa else (0, 0, 0, 0)
        config = [rows, len(self.checkpoints), state.shape[1], self.num_key_heads, self.spec_query_len,
                  self.max_blocks, self.capacity, self.capacity, NULL_BLOCK_ID, state.stride(1), state.stride(2),
                  corr.stride(1), corr.stride(2), *typed]
        t = self.tables
        return (state, corr, key, decay, t["state_addr"], t["state_block"], t["corr_addr"], t["corr_block"],
                t["key_addr"], t["key_block"], t["decay_addr"], t["decay_block"], self.layer_groups, *plan_views,
                config, 0 if soa else _FOLD_PACKED)


class GroupedCommitCoordinator:
    """One coordinator per recurrent-state owner (grouped_commit.py:896-1016):
    buckets the step's GDN groups by layout and logical rows, at most three
    per bucket, launches each bucket and, with several align buckets, one
    AND-valid publication after all of them.  Buckets are cached per epoch
    (the identity of their contexts) and only the current step's are kept."""

    def __init__(self):
        self._buckets = {}
        self._seen = set()
        self.steps = 0
        self.last_launch_count = 0
        self.last_group_count = 0
        self.last_rows = 0

    @staticmethod
    def _entries(metadata):
        for m in metadata:
            payload = getattr(m, "recoverssm_commit", None)
            if payload is None or getattr(m, "recoverssm_builder", None) is None:
                continue
            context = getattr(m, "recoverssm_context", None)
            if context is None:
                raise RuntimeError("a serving RecoverSSM commit has no producer binding epoch")
            yield CommitEntry(m, payload, context)

    @staticmethod
    def _step_is_align(entries) -> bool:
        """One step is all align or all none; align groups must share their
        logical rows and window (they publish one column per request)."""
        align = [e.payload.block_table is not None for e in entries]
        if not any(align):
            return False
        if not all(align):
            raise ValueError("one recovery step cannot mix align and none ownership")
        evidence = {_row_evidence(e) for e in entries}
        if len(evidence) != 1 or next(iter(evidence))[0] != "rows":
            raise ValueError("GDN groups must agree on logical rows, query lengths and align block size")
        if len({e.context.spec_query_len for e in entries}) != 1:
            raise ValueError("GDN groups must agree on the speculative window")
        return True

    @staticmethod
    def _partition(entries):
        """Entries grouped by (layout, logical rows) in first-seen order, each
        group cut into buckets of at most three."""
        by_key = {}
        for e in entries:
            by_key.setdefault((_layout_of(e.context), _row_evidence(e)), []).append(e)
        return [members[i : i + MAX_GROUPS_PER_BUCKET] for members in by_key.values()
                for i in range(0, len(members), MAX_GROUPS_PER_BUCKET)]

    def _bucket_for(self, subset):
        contexts = tuple(e.context for e in subset)
        epoch = tuple(map(id, contexts))
        bucket = self._buckets.get(epoch)
        if bucket is None:
            # a bucket the metadata builder prepared at start-up for exactly these contexts
            prepared = getattr(subset[0].metadata.recoverssm_builder, "_prepared_group_bucket", None)
            same = prepared is not None and len(prepared.contexts) == len(contexts) and all(
                a is b for a, b in zip(prepared.contexts, contexts))
            bucket = prepared if same else GroupedCommitBucket(contexts)
        return epoch, bucket

    def commit(self, metadata, sampled, idx_mapping, persistent_cols, persistent_accepted):
        entries = list(self._entries(metadata))
        if not entries:
            self.last_launch_count = self.last_group_count = self.last_rows = 0
            return
        align = self._step_is_align(entries)
        subsets = self._partition(entries)
        current, launches = {}, 0
        for subset in subsets:
            epoch, bucket = self._bucket_for(subset)
            current[epoch] = bucket
            specs = bucket.make_specs(subset, sampled, idx_mapping, persistent_cols, persistent_accepted,
                                      publish_align=len(subsets) == 1)
            for spec in specs:
                spec.launch()
            launches += len(specs)
        rows = int(entries[0].payload.state_indices.shape[0])
        if align and len(subsets) > 1:
            _publish_spec(tuple(current.values()), entries[0].payload.request_indices, idx_mapping, persistent_cols,
                          persistent_accepted, rows).launch()
            launches += 1
        self._buckets = current  # old epochs are dropped: no KV or record tensor outlives its epoch here
        self.steps += 1
        self.last_launch_count, self.last_group_count, self.last_rows = launches, len(entries), rows
        shape = (len(entries), len(subsets))
        if shape not in self._seen:
            self._seen.add(shape)
            logger.info("GDN recovery coordinator: groups=%d buckets=%d launches=%d", *shape, launches)


__all__ = ["CommitEntry", "GroupedCommitBucket", "GroupedCommitCoordinator"]
