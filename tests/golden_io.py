"""Load the committed golden fixtures (``tests/golden/*.npz``).

Fixtures were produced by ``tests/golden/make_golden.py`` from the reference's
own Triton kernels; bf16/fp16 tensors are stored as exact float32 values with a
``<name>__dtype`` companion entry.  ``<x>_after`` arrays hold only the changed
pages, listed in ``<x>_after_pages``.
"""

from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
_DT = {
    "float32": torch.float32,
    "bfloat16": torch.bfloat16,
    "float16": torch.float16,
    "int32": torch.int32,
    "int64": torch.int64,
}


def load(name):
    """Return ``dict``: tensors restored to their recorded dtype, scalars as
    Python values."""
    raw = np.load(GOLDEN / f"{name}.npz")
    out = {}
    for key in raw.files:
        if key.endswith("__dtype"):
            continue
        arr = raw[key]
        dt = raw.get(key + "__dtype") if key + "__dtype" in raw.files else None
        if dt is not None:
            out[key] = torch.from_numpy(arr.copy()).to(_DT[str(dt)])
        elif arr.ndim == 0:
            out[key] = arr.item()
        else:
            out[key] = arr
    return out


def full_after(case, prefix, i=""):
    """Rebuild the complete ``<prefix>_after<i>`` tensor from the stored pages."""
    before = case[f"{prefix}_before{i}"].clone()
    pages = case[f"{prefix}_after{i}_pages"].long()
    before[pages] = case[f"{prefix}_after{i}"]
    return before
