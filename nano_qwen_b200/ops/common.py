"""Small helpers shared by the op wrappers."""

from __future__ import annotations

import torch


def grad_buffer(p: torch.Tensor) -> torch.Tensor:
    """fp32 gradient buffer of a parameter, created (zeroed) on first use.

    Parameters placed in a ``FlatParamStore`` already carry a view into the
    store's flat gradient buffer; kernels accumulate into it in place.  A
    fully sharded store hands out the view of its gathered gradient buffer
    (its parameters may be bf16 while their gradients are fp32).
    """
    store = getattr(p, "_nq_store", None)
    if store is not None and hasattr(store, "grad_of"):
        return store.grad_of(p)
    if p.grad is None:
        p.grad = torch.zeros(p.shape, dtype=torch.float32, device=p.device)
    return p.grad


def rows(x: torch.Tensor) -> torch.Tensor:
    """Collapse leading dims: [..., H] -> [T, H] (contiguous)."""
    x2 = x.reshape(-1, x.shape[-1])
    return x2 if x2.is_contiguous() else x2.contiguous()


def wants_grad(*tensors) -> bool:
    return torch.is_grad_enabled() and any(
        t is not None and isinstance(t, torch.Tensor) and t.requires_grad for t in tensors)
