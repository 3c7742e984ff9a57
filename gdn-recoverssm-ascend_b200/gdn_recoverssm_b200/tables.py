"""Per-layer address and stride tables of a set of GDN layers.

The fold and conv-compaction kernels address every layer of a commit through
int64 tables: the base address of each layer's state pool, conv pool and
record planes, and their page / row strides (the reference passes one device
tensor per table, kernels.py:1525-1565, grouped_commit.py:641-657).  Here all
of a layer set's tables live in ONE int64 device tensor ``[rows, layers]``
filled by a single host-to-device copy; each named table is a contiguous row
view of it, which is what the native ops take.  The tensors whose addresses
the table holds are kept referenced by the object, so the raw pointers stay
valid as long as it lives.
"""

from __future__ import annotations

import torch

# row name -> (plane, what): plane indexes the tensors given to LayerTables,
# what is "addr" (data pointer) or a stride dimension
_ROWS = (
    ("state_addr", 0, "addr"),
    ("state_block", 0, 0),
    ("conv_addr", 1, "addr"),
    ("conv_block", 1, 0),
    ("conv_dim", 1, 1),
    ("conv_token", 1, 2),
    ("corr_addr", 2, "addr"),
    ("corr_block", 2, 0),
    ("key_addr", 3, "addr"),
    ("key_block", 3, 0),
    ("decay_addr", 4, "addr"),
    ("decay_block", 4, 0),
)
_INDEX = {name: i for i, (name, _, _) in enumerate(_ROWS)}


def as_int64_bits(addr: int) -> int:
    """A data pointer as the int64 holding the same 64 bits (addresses with the
    top bit set would overflow a plain conversion)."""
    return addr - (1 << 64) if addr >= (1 << 63) else addr


class LayerTables:
    """All per-layer tables of one layer set (``layers`` entries each):
    state / conv / correction / key / decay base addresses, the page (row)
    stride of each, and the conv pool's channel and token strides.

    ``planes`` = (checkpoints, conv_states, corrections, keys, decays), one
    tensor per layer in each; with packed records the three record planes are
    the same tensors."""

    def __init__(self, device, planes):
        planes = tuple(tuple(p) for p in planes)
        layers = len(planes[0])
        if any(len(p) != layers for p in planes):
            raise ValueError("GDN RecoverSSM: layer tables need one tensor per layer in every plane")
        values = []
        for _, plane, what in _ROWS:
            ts = planes[plane]
            values.append([as_int64_bits(t.data_ptr()) if what == "addr" else int(t.stride(what)) for t in ts])
        self.table = torch.tensor(values, dtype=torch.int64, device=device)
        self.owners = planes  # the addresses in the table stay valid while this object lives
        self.layers = layers
        # the row views, made once: a commit passes several per step, and a
        # view made per access costs host time on every step
        self._rows = {name: self.table[i] for name, i in _INDEX.items()}

    def __getitem__(self, name: str) -> torch.Tensor:
        return self._rows[name]
