"""Grow-only device scratch buffers for the drop-in entry points (the reference's
launchers are destination-passing for outputs; temporaries such as the permuted rows
of a gathered GEMM operand are owned here)."""

from __future__ import annotations

import torch

_bufs: dict[tuple, torch.Tensor] = {}


def scratch(name: str, numel: int, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    key = (name, dtype, device)
    t = _bufs.get(key)
    if t is None or t.numel() < numel:
        t = torch.empty(max(numel, 1), dtype=dtype, device=device)
        _bufs[key] = t
    return t[:numel]


_converted: dict[tuple, torch.Tensor] = {}


def converted(key_t: torch.Tensor, tag: str, make) -> torch.Tensor:
    """Cache a weight-layout conversion (made once per weight version, like the
    reference's load-time `wgt_from_gate`)."""
    key = (tag, key_t.data_ptr(), key_t._version, tuple(key_t.shape), key_t.dtype)
    t = _converted.get(key)
    if t is None:
        if len(_converted) > 16:
            _converted.clear()
        t = make()
        _converted[key] = t
    return t
