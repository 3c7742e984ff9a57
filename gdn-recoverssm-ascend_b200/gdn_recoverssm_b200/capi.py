"""ctypes binding of the C ABI (``include/gdn_recoverssm_b200.h``).

This is the boundary a non-torch host binds (cgo / JNI / N-API stubs would
mirror these prototypes).  The helpers at the bottom pass torch tensors'
device pointers straight through, with no torch op in between; the tests use
them to check the C ABI itself against the torch-op path.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, Structure, c_char_p, c_float, c_int32, c_int64, c_uint32, c_void_p

import torch

from . import _native

F32, BF16, F16, I32, I64 = 0, 1, 2, 3, 4
OK, EINVAL, ECUDA, EUNSUPPORTED = 0, 1, 2, 3
RECORD_PACKED, NORMALIZE_QK = 1, 2
FOLD_PACKED = 1
VERIFY_FIELDS, FOLD_FIELDS = 28, 17

_DTYPE = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16, torch.int32: I32, torch.int64: I64}


class IndexView(Structure):
    _fields_ = [("data", c_void_p), ("stride", c_int64), ("length", c_int64), ("dtype", c_int32)]


class OutView(Structure):
    _fields_ = [("data", c_void_p), ("stride", c_int64), ("length", c_int64), ("dtype", c_int32)]


class TableView(Structure):
    _fields_ = [
        ("data", c_void_p),
        ("rows", c_int64),
        ("cols", c_int64),
        ("row_stride", c_int64),
        ("col_stride", c_int64),
        ("dtype", c_int32),
    ]


class PlanGroup(Structure):
    _fields_ = [
        ("state_indices", IndexView),
        ("query_start_loc", IndexView),
        ("request_indices", IndexView),
        ("num_computed", IndexView),
        ("block_table", TableView),
        ("num_blocks", c_int64),
        ("block_size", c_int64),
    ]


# name -> (restype, argtypes): every entry point the header declares.
PROTOTYPES = {
    "gdn_rssm_abi_version": (c_int64, []),
    "gdn_rssm_last_error": (c_char_p, []),
    "gdn_rssm_device_status": (c_int32, [POINTER(c_int32), c_void_p]),
    "gdn_rssm_verify": (
        c_int32,
        [c_void_p] * 12 + [POINTER(c_int64), c_int64, c_float] + [c_int32] * 8 + [c_uint32, c_void_p],
    ),
    "gdn_rssm_verify_gated": (
        c_int32,
        [c_void_p] * 14 + [POINTER(c_int64), c_int64] + [c_float] * 3 + [c_int32] * 9 + [c_uint32, c_void_p],
    ),
    "gdn_rssm_fold": (
        c_int32,
        [c_void_p] * 9 + [IndexView] + [c_void_p] * 4 + [c_int64, POINTER(c_int64), c_int64] + [c_int32] * 4
        + [c_uint32, c_void_p],
    ),
    "gdn_rssm_commit_plan": (
        c_int32,
        [IndexView] * 4 + [TableView, IndexView] + [c_void_p] * 6 + [c_int64] * 5 + [c_void_p],
    ),
    "gdn_rssm_grouped_plan": (
        c_int32,
        [IndexView, POINTER(PlanGroup), c_int32] + [c_void_p] * 7 + [IndexView, OutView, OutView] + [c_int64] * 4
        + [c_int32, c_int32, c_void_p],
    ),
    "gdn_rssm_publish_align": (
        c_int32,
        [c_void_p, c_int32, IndexView, IndexView, OutView, OutView, c_int64, c_void_p],
    ),
    "gdn_rssm_compact_conv": (
        c_int32,
        [c_void_p] * 5 + [IndexView] + [c_void_p] * 4 + [c_int64] * 9 + [c_int32, c_int32, c_void_p],
    ),
}


def lib():
    """The loaded C ABI library with prototypes attached."""
    handle = _native.capi()
    if not getattr(handle, "_gdn_prototyped", False):
        for name, (restype, argtypes) in PROTOTYPES.items():
            fn = getattr(handle, name)
            fn.restype = restype
            fn.argtypes = argtypes
        handle._gdn_prototyped = True
    return handle


def last_error() -> str:
    msg = lib().gdn_rssm_last_error()
    return msg.decode() if msg else ""


def check(rc: int) -> None:
    if rc != OK:
        raise RuntimeError(f"C ABI call failed (code {rc}): {last_error()}")


def dtype_code(dtype) -> int:
    return _DTYPE[dtype]


def ptr(t):
    return None if t is None else t.data_ptr()


def index_view(t) -> IndexView:
    if t is None:
        return IndexView(None, 0, 0, I32)
    return IndexView(t.data_ptr(), t.stride(0), t.shape[0], _DTYPE[t.dtype])


def out_view(t) -> OutView:
    if t is None:
        return OutView(None, 0, 0, I32)
    return OutView(t.data_ptr(), t.stride(0), t.shape[0], _DTYPE[t.dtype])


def table_view(t) -> TableView:
    if t is None:
        return TableView(None, 0, 0, 0, 0, I32)
    return TableView(t.data_ptr(), t.shape[0], t.shape[1], t.stride(0), t.stride(1), _DTYPE[t.dtype])


def int64_array(values):
    arr = (c_int64 * len(values))(*[int(v) for v in values])
    return arr


def current_stream_handle(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def verify(q, k, v, g, beta, state, correction, key, decay, out, qsl, indices, config, scale, *, flags, stream=None):
    """Call ``gdn_rssm_verify`` with torch tensors' raw device pointers."""
    K, V = q.shape[-1], v.shape[-1]
    packed = bool(flags & RECORD_PACKED)
    cfg = int64_array(config)
    corr_ptr = correction.data_ptr()
    key_ptr = corr_ptr + 4 * V if packed else key.data_ptr()
    decay_ptr = corr_ptr + 4 * (V + K) if packed else decay.data_ptr()
    rc = lib().gdn_rssm_verify(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr(), state.data_ptr(), corr_ptr,
        key_ptr, decay_ptr, out.data_ptr(), qsl.data_ptr(), indices.data_ptr(), cfg, len(config), float(scale),
        _DTYPE[q.dtype], _DTYPE[state.dtype], _DTYPE[beta.dtype], F32 if packed else _DTYPE[key.dtype],
        _DTYPE[qsl.dtype], _DTYPE[indices.dtype], K, V, flags,
        current_stream_handle() if stream is None else stream,
    )
    check(rc)


def verify_gated(q, k, v, a, b, A_log, dt_bias, state, correction, key, decay, out, qsl, indices, config, scale,
                 softplus_beta, softplus_threshold, *, flags, stream=None):
    """Call ``gdn_rssm_verify_gated`` with torch tensors' raw device pointers."""
    K, V = q.shape[-1], v.shape[-1]
    packed = bool(flags & RECORD_PACKED)
    cfg = int64_array(config)
    corr_ptr = correction.data_ptr()
    key_ptr = corr_ptr + 4 * V if packed else key.data_ptr()
    decay_ptr = corr_ptr + 4 * (V + K) if packed else decay.data_ptr()
    rc = lib().gdn_rssm_verify_gated(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), a.data_ptr(), b.data_ptr(), A_log.data_ptr(), dt_bias.data_ptr(),
        state.data_ptr(), corr_ptr, key_ptr, decay_ptr, out.data_ptr(), qsl.data_ptr(), indices.data_ptr(), cfg,
        len(config), float(scale), float(softplus_beta), float(softplus_threshold), _DTYPE[q.dtype],
        _DTYPE[state.dtype], _DTYPE[a.dtype], _DTYPE[b.dtype], F32 if packed else _DTYPE[key.dtype],
        _DTYPE[qsl.dtype], _DTYPE[indices.dtype], K, V, flags,
        current_stream_handle() if stream is None else stream,
    )
    check(rc)
