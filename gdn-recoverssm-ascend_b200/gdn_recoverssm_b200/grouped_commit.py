"""Step-owned grouped recovery: one plan, one conv pass, one fold per bucket.

Drop-in host layer for the reference module
``plugin/gdn_recoverssm_ascend/grouped_commit.py``: ``CommitEntry``,
``GroupedCommitBucket`` (``__init__`` / ``make_specs``) and
``GroupedCommitCoordinator.commit`` keep the reference's signatures, bucketing
rules and ``ValueError`` checks; the three launches per bucket (plan, conv
compaction, fold) and the cross-bucket publication go to the CUDA kernels via
``torch.ops.gdn_recoverssm_ac``.

A bucket holds one to three layout-homogeneous KV-cache groups; plan row of
(layer, row) is ``layer_groups[layer] * capacity + row``.
"""

from __future__ import annotations

import logging
from dataclasses import dataclass
from typing import Any

import torch

from . import _native
from .kernels import _FOLD_PACKED, NULL_BLOCK_ID, _LaunchSpec, _ptr_table, _require

logger = logging.getLogger("gdn_recoverssm_b200.grouped_commit")


@dataclass(frozen=True)
class CommitEntry:
    metadata: Any
    payload: Any
    context: Any


def _layout_key(context):
    """Everything that must agree for two contexts to share one launch."""
    state = context.checkpoints[0]
    conv = context.conv_states[0]
    record = context.records[0]
    soa = context.record_layout == "soa"
    rr = record.correction if soa else record
    kr = record.key if soa else record
    dr = record.decay if soa else record
    return (
        state.device, state.dtype, tuple(state.shape[1:]), tuple(state.stride()[1:]),
        conv.dtype, tuple(conv.shape[1:]), tuple(conv.stride()[1:]),
        context.conv_history_len, context.spec_query_len, context.record_layout, context.num_key_heads,
        rr.dtype, tuple(rr.stride()[1:]), kr.dtype, tuple(kr.stride()[1:]), dr.dtype, tuple(dr.stride()[1:]),
    )


def _logical_key(entry):
    """Host evidence of the logical rows; without it a group cannot share a
    launch with another group."""
    p = entry.payload
    rows = int(p.state_indices.shape[0])
    host_rows = tuple(getattr(p, "request_rows", ()))
    host_lens = tuple(getattr(p, "query_lens", ()))
    if len(host_rows) != rows or len(host_lens) != rows:
        return (id(entry.metadata),)
    return (host_rows, host_lens, p.block_size, p.block_table is not None)


def _publisher_descriptors(buckets):
    """Persistent device table (valid ptr, col ptr, capacity, groups) per bucket."""
    owner = buckets[0]
    key = tuple((id(b.valid), id(b.col), b.capacity, len(b.contexts)) for b in buckets)
    if getattr(owner, "_publisher_key", None) != key:
        values = []
        for b in buckets:
            for value in (b.valid.data_ptr(), b.col.data_ptr(), b.capacity, len(b.contexts)):
                values.append(value if value < (1 << 63) else value - (1 << 64))
        owner._publisher_descriptors = torch.tensor(values, dtype=torch.int64, device=owner.device)
        owner._publisher_plan_owners = tuple((b.valid, b.col) for b in buckets)
        owner._publisher_key = key
    return owner._publisher_descriptors


def _publish_spec(buckets, request_indices, idx_mapping, persistent_cols, persistent_accepted, rows):
    """AND-valid publication after all buckets committed (grouped_commit.py:531-610)."""
    return _LaunchSpec(
        "publish_align",
        _native.ops().publish_align,
        (_publisher_descriptors(buckets), request_indices, idx_mapping, persistent_cols, persistent_accepted, rows),
    )


class GroupedCommitBucket:
    """Stable per-layer address tables and per-group plan storage for one
    KV epoch (grouped_commit.py:613-893)."""

    def __init__(self, contexts):
        self.contexts = tuple(contexts)
        if not 0 < len(contexts) <= 3:
            raise ValueError("one recovery bucket requires one to three contexts")
        key = _layout_key(contexts[0])
        if any(_layout_key(c) != key for c in contexts[1:]):
            raise ValueError("grouped recovery requires homogeneous layer layouts")
        self.capacity = min(int(c.record_rows) for c in contexts)
        if self.capacity <= 0:
            raise ValueError("grouped recovery has no record rows")
        self.device = contexts[0].checkpoints[0].device
        self.checkpoints = tuple(t for c in contexts for t in c.checkpoints)
        self.conv_states = tuple(t for c in contexts for t in c.conv_states)
        self.records = tuple(t for c in contexts for t in c.records)
        self.layer_groups = torch.tensor(
            [g for g, c in enumerate(contexts) for _ in c.checkpoints], dtype=torch.int32, device=self.device
        )
        self.max_blocks = max(int(c.num_blocks) for c in contexts)
        self.spec_query_len = int(contexts[0].spec_query_len)
        self.record_layout = contexts[0].record_layout
        self.num_key_heads = int(contexts[0].num_key_heads)
        self.conv_history_len = int(contexts[0].conv_history_len)
        self.state_addrs = _ptr_table(self.checkpoints, self.device)
        self.conv_addrs = _ptr_table(self.conv_states, self.device)
        self.state_block_strides = self._strides(self.checkpoints, 0)
        self.conv_block_strides = self._strides(self.conv_states, 0)
        self.conv_dim_strides = self._strides(self.conv_states, 1)
        self.conv_token_strides = self._strides(self.conv_states, 2)
        soa = self.record_layout == "soa"
        self.corrections = tuple(r.correction if soa else r for r in self.records)
        self.keys = tuple(r.key if soa else r for r in self.records)
        self.decays = tuple(r.decay if soa else r for r in self.records)
        self.correction_addrs = _ptr_table(self.corrections, self.device)
        self.key_addrs = _ptr_table(self.keys, self.device)
        self.decay_addrs = _ptr_table(self.decays, self.device)
        self.correction_block_strides = self._strides(self.corrections, 0)
        self.key_block_strides = self._strides(self.keys, 0)
        self.decay_block_strides = self._strides(self.decays, 0)
        size = self.capacity * len(contexts)
        self.source = torch.zeros(size, dtype=torch.int32, device=self.device)
        self.length = torch.zeros_like(self.source)
        self.final = torch.zeros_like(self.source)
        self.boundary = torch.zeros_like(self.source)
        self.boundary_len = torch.zeros_like(self.source)
        self.valid = torch.zeros_like(self.source)
        self.col = torch.zeros_like(self.source)

    def _strides(self, tensors, dim):
        return torch.tensor([t.stride(dim) for t in tensors], dtype=torch.int64, device=self.device)

    def make_specs(self, entries, sampled, idx_mapping, persistent_cols, persistent_accepted, *, publish_align=True):
        """Validate one step's entries and return the (plan, conv, fold)
        launch specs without launching them (grouped_commit.py:670-893)."""
        contexts = tuple(e.context for e in entries)
        if len(contexts) != len(self.contexts) or any(a is not b for a, b in zip(contexts, self.contexts)):
            raise ValueError("grouped recovery bucket belongs to a different KV epoch")
        p = tuple(e.payload for e in entries)
        rows = int(p[0].state_indices.shape[0])
        if not 0 < rows <= self.capacity:
            raise ValueError(
                f"grouped recovery rows out of range: rows={rows}, record capacity={self.capacity}, "
                f"groups={len(p)}, state_indices shapes={[tuple(x.state_indices.shape) for x in p]}"
            )
        if any(int(x.state_indices.shape[0]) != rows for x in p):
            raise ValueError("grouped recovery row counts differ")
        align = p[0].block_table is not None
        if any((x.block_table is not None) != align for x in p):
            raise ValueError("grouped recovery cannot mix align and none plans")
        if any(x.request_indices is None for x in p):
            raise ValueError("grouped recovery requires an explicit native row mapping")
        required = [sampled, idx_mapping, persistent_accepted]
        for x in p:
            required.extend((x.state_indices, x.query_start_loc, x.request_indices))
            if align:
                required.extend((x.block_table, x.num_computed_tokens))
        if align:
            required.append(persistent_cols)
        if any(t is None or t.device != self.device for t in required):
            raise ValueError("grouped recovery inputs must share the checkpoint device")
        if sampled.data_ptr() == persistent_accepted.data_ptr():
            raise ValueError("sampled counts must not alias persistent acceptance output")
        for x in p:
            if x.query_start_loc.numel() < rows + 1:
                raise ValueError("grouped recovery offsets are shorter than their rows")
            if align and (x.block_size is None or x.block_size < self.spec_query_len):
                raise ValueError("align blocks must cover the speculative window")
            if align and x.block_table.shape[1] <= 0:
                raise ValueError("align block table has no columns")
            host_rows = tuple(getattr(x, "request_rows", ()))
            if len(host_rows) == rows and any(
                r < 0 or r >= sampled.numel() or r >= idx_mapping.numel() for r in host_rows
            ):
                raise ValueError("native request mapping exceeds the sampled batch")
        ops = _native.ops()
        plan = _LaunchSpec(
            "grouped_plan",
            ops.grouped_plan,
            (
                sampled,
                [x.state_indices for x in p],
                [x.query_start_loc for x in p],
                [x.request_indices for x in p],
                [x.block_table if align else None for x in p],
                [x.num_computed_tokens if align else None for x in p],
                [int(c.num_blocks) for c in contexts],
                [int(x.block_size) if align else 1 for x in p],
                self.source, self.length, self.final, self.boundary, self.boundary_len, self.valid, self.col,
                idx_mapping, persistent_cols if align else None, persistent_accepted if align else None,
                rows, self.capacity, self.spec_query_len, align, bool(align and publish_align),
            ),
        )
        conv = self.conv_states[0]
        compact = _LaunchSpec(
            "compact_conv",
            ops.compact_conv,
            (conv, self.conv_addrs, self.conv_block_strides, self.conv_dim_strides, self.conv_token_strides,
             self.layer_groups, self.source, self.length, self.final, self.boundary, self.boundary_len, rows,
             self.capacity, int(conv.shape[1]), self.conv_history_len, int(conv.shape[2]), self.max_blocks, align),
        )
        state = self.checkpoints[0]
        _, hv, _, _ = state.shape
        soa = self.record_layout == "soa"
        rr, kr, dr = self.corrections[0], self.keys[0], self.decays[0]
        config = [
            rows, len(self.checkpoints), hv, self.num_key_heads, self.spec_query_len, self.max_blocks,
            self.capacity, self.capacity, NULL_BLOCK_ID, state.stride(1), state.stride(2), rr.stride(1),
            rr.stride(2), kr.stride(1) if soa else 0, kr.stride(2) if soa else 0, dr.stride(1) if soa else 0,
            dr.stride(2) if soa else 0,
        ]
        fold = _LaunchSpec(
            "fold",
            ops.fold_ext,
            (state, rr, kr, dr, self.state_addrs, self.state_block_strides, self.correction_addrs,
             self.correction_block_strides, self.key_addrs, self.key_block_strides, self.decay_addrs,
             self.decay_block_strides, self.layer_groups, self.source, self.length, self.final, self.boundary,
             self.boundary_len, config, 0 if soa else _FOLD_PACKED),
        )
        return plan, compact, fold


class GroupedCommitCoordinator:
    """One coordinator per recurrent-state owner: buckets the step's GDN groups
    by layout and logical rows (at most three per bucket), launches each
    bucket and, with several align buckets, one AND-valid publication
    (grouped_commit.py:896-1016)."""

    def __init__(self):
        self._buckets = {}
        self._seen = set()
        self.steps = 0
        self.last_launch_count = 0
        self.last_group_count = 0
        self.last_rows = 0

    def commit(self, metadata, sampled, idx_mapping, persistent_cols, persistent_accepted):
        entries = []
        for m in metadata:
            p = getattr(m, "recoverssm_commit", None)
            builder = getattr(m, "recoverssm_builder", None)
            if p is None or builder is None:
                continue
            context = getattr(m, "recoverssm_context", None)
            if context is None:
                raise RuntimeError("a serving RecoverSSM commit has no producer binding epoch")
            entries.append(CommitEntry(m, p, context))
        if not entries:
            self.last_launch_count = self.last_group_count = self.last_rows = 0
            return
        aligned = [e for e in entries if e.payload.block_table is not None]
        if aligned:
            if len(aligned) != len(entries):
                raise ValueError("one recovery step cannot mix align and none ownership")
            logical = _logical_key(aligned[0])
            if len(logical) == 1 or any(_logical_key(e) != logical for e in aligned[1:]):
                raise ValueError("GDN groups must agree on logical rows, query lengths and align block size")
            if any(e.context.spec_query_len != entries[0].context.spec_query_len for e in entries):
                raise ValueError("GDN groups must agree on the speculative window")
        logical_groups = {}
        for entry in entries:
            logical_groups.setdefault((_layout_key(entry.context), _logical_key(entry)), []).append(entry)
        grouped = [items[s : s + 3] for items in logical_groups.values() for s in range(0, len(items), 3)]
        live = {}
        launches = 0
        for subset in grouped:
            contexts = tuple(e.context for e in subset)
            epoch = tuple(id(c) for c in contexts)
            bucket = self._buckets.get(epoch)
            if bucket is None:
                prepared = getattr(subset[0].metadata.recoverssm_builder, "_prepared_group_bucket", None)
                if (
                    prepared is not None
                    and len(prepared.contexts) == len(contexts)
                    and all(a is b for a, b in zip(prepared.contexts, contexts))
                ):
                    bucket = prepared
                else:
                    bucket = GroupedCommitBucket(contexts)
            live[epoch] = bucket
            specs = bucket.make_specs(subset, sampled, idx_mapping, persistent_cols, persistent_accepted,
                                      publish_align=len(grouped) == 1)
            for spec in specs:
                spec.launch()
            launches += len(specs)
        if aligned and len(grouped) > 1:
            buckets = tuple(live.values())
            _publish_spec(buckets, entries[0].payload.request_indices, idx_mapping, persistent_cols,
                          persistent_accepted, int(entries[0].payload.state_indices.shape[0])).launch()
            launches += 1
        self._buckets = live
        self.steps += 1
        self.last_launch_count = launches
        self.last_group_count = len(entries)
        self.last_rows = int(entries[0].payload.state_indices.shape[0])
        reason = (len(entries), len(grouped))
        if reason not in self._seen:
            self._seen.add(reason)
            logger.info("GDN recovery coordinator: groups=%d buckets=%d launches=%d", len(entries), len(grouped),
                        launches)


__all__ = ["CommitEntry", "GroupedCommitBucket", "GroupedCommitCoordinator"]
