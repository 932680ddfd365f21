"""Batched token sampling on B200 (CUDA only, no fallback).

:func:`sample_tokens` has the signature, argument meaning and errors of the
reference's ``sample_tokens`` (server/model/sampling.py:118-194): per-row
temperature (<= 0 is greedy), top-k (0 or >= vocab disables), top-p (1.0
disables) and one uniform in [0, 1) per row, applied as top-k, then top-p
over the survivors, then an inverse-CDF pick.  It is a pure function of its
arguments and a row's token does not depend on the other rows.  One kernel
launch; no sort, no host synchronisation.

:func:`uniforms_from_seeds` is the reference's counter-based noise
(server/model/determinism.py:54-73) computed on the GPU, and
:func:`sample_tokens_seeded` fuses it into the sampling launch.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch

from .. import _capi
from .._runtime import on_device, require_cuda, stream_ptr

__all__ = ["LOWEST_TEMPERATURE", "sample_tokens", "sample_tokens_seeded", "uniforms_from_seeds"]

LOWEST_TEMPERATURE = 1e-5  # sampling.py:5; the kernel clamps in float32 as torch does

_LOGIT_TAG = {torch.float32: _capi.QF_F32, torch.float16: _capi.QF_F16,
              torch.bfloat16: _capi.QF_BF16}


def _check_param(name: str, tensor: torch.Tensor, batch_size: int) -> None:
    if tensor.shape != (batch_size,):
        raise ValueError(f"Expected {name} shape [{batch_size}], got {tuple(tensor.shape)}")


def _as_u64_bits(values: Sequence[int] | torch.Tensor, device: torch.device) -> torch.Tensor:
    """int64 tensor holding each value's low 64 bits (the hash masks its
    inputs to 64 bits, determinism.py:37)."""
    if isinstance(values, torch.Tensor):
        return values.to(device=device, dtype=torch.int64)
    wrapped = [((int(v) + (1 << 63)) % (1 << 64)) - (1 << 63) for v in values]
    return torch.tensor(wrapped, dtype=torch.int64, device=device)


# Which kernels sample a batch: "cluster" runs each row on a cluster of CTAs
# (one row's ~10 steps back to back, ~37 rows in flight on a B200); "wide"
# runs every step as one launch over all rows, with a workspace of
# qf_sample_workspace_bytes(batch), and hands the rows it cannot finish to the
# cluster kernel; "auto" takes "wide" from WIDE_MIN_ROWS rows on.  Every path
# gives the same tokens.
_PATHS = {"auto": 0, "cluster": 1, "wide": 2}
WIDE_MIN_ROWS, WIDE_MAX_ROWS = 128, 65535


def _launch(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor,
            top_p: torch.Tensor, uniforms: torch.Tensor | None, seeds: torch.Tensor | None,
            steps: torch.Tensor | None, what: str, path: str = "auto") -> torch.Tensor:
    if logits.ndim != 2:
        raise ValueError(f"Expected logits shape [B, vocab_size], got {logits.ndim}D")
    batch_size, vocab_size = logits.shape
    _check_param("temperature", temperature, batch_size)
    _check_param("top_k", top_k, batch_size)
    _check_param("top_p", top_p, batch_size)
    if uniforms is not None:
        _check_param("uniforms", uniforms, batch_size)
    else:
        _check_param("seeds", seeds, batch_size)
        _check_param("steps", steps, batch_size)
    if vocab_size == 0:
        raise ValueError("Expected a non-empty vocabulary")
    if path not in _PATHS:
        raise ValueError(f"{what}: path must be one of {sorted(_PATHS)}, got {path!r}")
    dev = require_cuda(what, logits, temperature, top_k, top_p, uniforms, seeds, steps)
    out = torch.empty(batch_size, dtype=torch.int64, device=dev)
    if batch_size == 0:
        return out
    x = logits if logits.dtype in _LOGIT_TAG else logits.float()
    if x.stride(1) != 1:
        x = x.contiguous()
    temp = temperature.float().contiguous()
    tk = top_k if top_k.dtype in (torch.int32, torch.int64) else top_k.long()
    tk = tk.contiguous()
    tp = top_p.float().contiguous()
    a = _capi.SampleArgs()
    a.logits, a.logits_row_stride = x.data_ptr(), x.stride(0)
    a.batch, a.vocab = batch_size, vocab_size
    a.dtype = _LOGIT_TAG[x.dtype]
    a.temperature = temp.data_ptr()
    a.top_k = tk.data_ptr()
    a.top_k_type = _capi.QF_I64 if tk.dtype == torch.int64 else _capi.QF_I32
    a.top_p = tp.data_ptr()
    if uniforms is not None:
        u = uniforms.float().contiguous()
        a.uniforms = u.data_ptr()
    else:
        sd, st = seeds.to(torch.int64).contiguous(), steps.to(torch.int64).contiguous()
        a.seeds, a.steps = sd.data_ptr(), st.data_ptr()
    a.out = out.data_ptr()
    a.path = _PATHS[path]
    ws = None
    if path == "wide" or (path == "auto" and WIDE_MIN_ROWS <= batch_size <= WIDE_MAX_ROWS):
        nbytes = _capi.lib().qf_sample_workspace_bytes(batch_size)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        a.workspace, a.workspace_bytes = ws.data_ptr(), nbytes
    with on_device(dev):
        _capi.check(_capi.lib().qf_sample_tokens(a, stream_ptr(dev)), what)
    return out


@torch.inference_mode()
def sample_tokens(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor,
                  top_p: torch.Tensor, uniforms: torch.Tensor, *,
                  path: str = "auto") -> torch.Tensor:
    """Sample one token per row of ``logits`` [B, vocab].

    temperature [B]: rows <= 0 are greedy (argmax, lowest index among equal
    maxima); top_k [B]: 0 (or >= vocab) disables; top_p [B]: 1.0 disables;
    uniforms [B] in [0, 1).  Returns [B] int64 token ids on the logits'
    device.  Same ValueErrors as the reference for a wrong rank or shape.
    ``path`` picks the kernels ("auto", "cluster", "wide"; see _PATHS); the
    tokens do not depend on it."""
    return _launch(logits, temperature, top_k, top_p, uniforms, None, None, "sample_tokens",
                   path)


@torch.inference_mode()
def sample_tokens_seeded(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor,
                         top_p: torch.Tensor, seeds: torch.Tensor | Sequence[int],
                         steps: torch.Tensor | Sequence[int], *,
                         path: str = "auto") -> torch.Tensor:
    """``sample_tokens(logits, ..., uniforms_from_seeds(seeds, steps))`` with
    the uniforms computed inside the sampling kernel (no separate launch, no
    host-to-device copy of the noise)."""
    if logits.ndim != 2:
        raise ValueError(f"Expected logits shape [B, vocab_size], got {logits.ndim}D")
    if len(seeds) != len(steps):
        raise ValueError(
            f"seeds and steps must be the same length, got {len(seeds)} and {len(steps)}")
    dev = logits.device
    return _launch(logits, temperature, top_k, top_p, None, _as_u64_bits(seeds, dev),
                   _as_u64_bits(steps, dev), "sample_tokens_seeded", path)


def uniforms_from_seeds(seeds: Sequence[int] | torch.Tensor, steps: Sequence[int] | torch.Tensor,
                        device: str | torch.device = "cuda") -> torch.Tensor:
    """Per-row uniform noise [B] (float32, on a CUDA device): row i depends
    only on (seeds[i], steps[i]), as in the reference
    (determinism.py:54-73); computed by a kernel."""
    if len(seeds) != len(steps):
        raise ValueError(
            f"seeds and steps must be the same length, got {len(seeds)} and {len(steps)}")
    dev = torch.device(device)
    if dev.type == "cuda" and dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    sd, st = _as_u64_bits(seeds, dev), _as_u64_bits(steps, dev)
    require_cuda("uniforms_from_seeds", sd, st)
    out = torch.empty(sd.numel(), dtype=torch.float32, device=dev)
    with on_device(dev):
        rc = _capi.lib().qf_uniforms_from_seeds(sd.contiguous().data_ptr(),
                                                st.contiguous().data_ptr(), sd.numel(),
                                                out.data_ptr(), stream_ptr(dev))
    _capi.check(rc, "uniforms_from_seeds")
    return out
