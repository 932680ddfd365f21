"""Host-side plumbing shared by the ops: dtype tags, streams, the status word.

Every op enqueues on torch's current CUDA stream of the tensors' device.  Index
errors found on the device (bad token id, block, slot) are ORed into a per-
device int32 status word owned here; :func:`check_errors` reads and clears it.
With ``TINYSERVER_B200_CHECK=1`` in the environment every op checks it right
away (one stream sync per op: for tests and debugging, not for serving).
"""

from __future__ import annotations

import contextlib
import ctypes
import os

import torch

from . import _capi

_DTYPE_TAG = {torch.float32: _capi.QF_F32, torch.float16: _capi.QF_F16,
              torch.bfloat16: _capi.QF_BF16}
_INDEX_TAG = {torch.int32: _capi.QF_I32, torch.int64: _capi.QF_I64}

_status_words: dict[int, torch.Tensor] = {}
_work_counters: dict[tuple[int, int], torch.Tensor] = {}
SYNC_CHECK = os.environ.get("TINYSERVER_B200_CHECK", "0") not in ("", "0")


def dtype_tag(t: torch.Tensor, what: str) -> int:
    try:
        return _DTYPE_TAG[t.dtype]
    except KeyError:
        raise ValueError(f"{what}: dtype {t.dtype} not supported (float32/float16/bfloat16)")


def index_tag(t: torch.Tensor, what: str) -> int:
    try:
        return _INDEX_TAG[t.dtype]
    except KeyError:
        raise ValueError(f"{what}: index dtype {t.dtype} not supported (int32/int64)")


def require_cuda(what: str, *tensors: torch.Tensor | None) -> torch.device:
    """All tensors on one CUDA device; the library has no CPU path."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise ValueError(f"{what}: tinyserver_b200 ops take CUDA tensors only "
                             f"(got a tensor on {t.device}); there is no CPU path")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"{what}: tensors on different devices ({dev} and {t.device})")
    if dev is None:
        raise ValueError(f"{what}: no tensor arguments")
    return dev


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_SAME_DEVICE = contextlib.nullcontext()


def on_device(device: torch.device):
    """Make ``device`` the current CUDA device around a launch.  The library
    launches on the current device, and a stream handle of 0 (torch's default
    stream) means the current device's default stream, so tensors on cuda:1
    while cuda:0 is current need the switch.  No switch when it is current."""
    idx = device.index
    if idx is None or idx == torch.cuda.current_device():
        return _SAME_DEVICE
    return torch.cuda.device(idx)


def status_word(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    w = _status_words.get(idx)
    if w is None:
        if torch.cuda.is_current_stream_capturing():
            # made here, the word would be zeroed only by a node of this graph
            # and would live in the graph's private memory pool
            raise RuntimeError("tinyserver_b200: call any op on this device once outside "
                               "CUDA graph capture before capturing (it makes the device's "
                               "status word)")
        w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status_words[idx] = w
    return w


def work_counter(device: torch.device) -> torch.Tensor:
    """Two int32 words for the persistent prefill attention kernel, one pair
    per (device, current stream).  Zero when made; each call claims its work
    items from it and leaves it at zero when it completes, so calls queued in
    order on one stream share a pair, and calls on other streams, which may
    overlap on the GPU, get pairs of their own."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, stream_ptr(torch.device("cuda", idx)))
    w = _work_counters.get(key)
    if w is not None:
        return w
    w = torch.zeros(2, dtype=torch.int32, device=torch.device("cuda", idx))
    if torch.cuda.is_current_stream_capturing():
        # Made during a CUDA graph capture, this pair's zero fill exists only as
        # a node of that graph, so it is not kept for later calls: this call
        # gets a pair of its own that the graph zeroes on every replay.
        return w
    _work_counters[key] = w
    return w


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def read_flags(device: torch.device, clear: bool = True) -> int:
    """Synchronise the current stream and return (and clear) the status word."""
    w = status_word(device)
    out = ctypes.c_int32(0)
    with on_device(device):
        rc = _capi.lib().qf_read_status(w.data_ptr(), ctypes.byref(out), int(clear),
                                        stream_ptr(device))
    if rc not in (_capi.QF_OK, _capi.QF_ERR_DEVICE):
        _capi.check(rc, "qf_read_status")
    return out.value


def check_errors(device: torch.device | int | None = None) -> None:
    """Raise IndexError if any op on ``device`` flagged an out-of-range index
    since the last check (the reference raises IndexError for a bad token id)."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    elif isinstance(device, int):
        device = torch.device("cuda", device)
    flags = read_flags(device)
    if flags:
        names = [n for bit, n in _capi.FLAG_NAMES.items() if flags & bit]
        if flags & _capi.QF_FLAG_TIMEOUT:
            raise RuntimeError("tinyserver_b200: " + "; ".join(names))
        raise IndexError("tinyserver_b200: " + "; ".join(names))


def after_op(device: torch.device) -> None:
    if SYNC_CHECK:
        check_errors(device)
