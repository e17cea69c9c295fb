"""Module-tree cloning for the decoder-rewrite helpers (fp16 / INT8 FFN swaps, norm-quant blocks,
INT8 QKV and attention-out projections): every container in the tree is a new object with its
own parameter, buffer and child tables, while the tensors themselves are shared, so a rewritten
decoder can be offloaded or reloaded without touching the caller's module.  A module reachable
under two names stays one object in the clone."""
from __future__ import annotations

import copy

from torch import nn


def clone_containers(module: nn.Module, memo: dict | None = None) -> nn.Module:
    """ref: opt/int8_attention_out.py:13-26 (clone_containers)."""
    memo = {} if memo is None else memo
    if id(module) in memo:
        return memo[id(module)]
    twin = copy.copy(module)
    memo[id(module)] = twin
    twin._parameters = dict(module._parameters)
    twin._buffers = dict(module._buffers)
    twin._modules = {name: None if child is None else clone_containers(child, memo)
                     for name, child in module._modules.items()}
    return twin


def selected_indices(count: int, indices=None) -> tuple[int, ...]:
    """Block indices to rewrite (all when None): nonempty, unique, in range, plain ints.
    ref: opt/int8_qkv.py:24-30."""
    chosen = tuple(range(count)) if indices is None else tuple(indices)
    if not chosen or len(set(chosen)) != len(chosen):
        raise ValueError("nonempty unique block indices required")
    if any(type(i) is not int or not 0 <= i < count for i in chosen):
        raise ValueError("block index out of range or not an integer")
    return chosen


def require_backend() -> None:
    """The rewritten modules run on this package's native library; fail before any rewrite when it
    cannot be loaded (the reference checks its comfy-kitchen build the same way,
    opt/int8_swiglu_fused.py:69-75)."""
    from .. import _lib
    try:
        _lib.load()
    except Exception as exc:  # noqa: BLE001 - re-raised with the contract's error type
        raise RuntimeError(f"h3vae_b200 native library unavailable: {exc}") from None
