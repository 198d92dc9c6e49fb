"""Drop-in replacement for the reference's ``gsp.runtime`` module
(gsp/runtime.py of StealthEyeLLC/grammar-sparse-projection).

constrained_projection keeps the reference's signature, ProjectionResult, mode
strings ("dense-unconstrained", "dense-selected", "sparse-gather") and
ValueError messages. The work runs on the device through libgsp_b200.so:

  1. gsp_ids_to_bitmask turns the id list into a bitmask; setting bits both
     deduplicates and sorts the ids (gsp/runtime.py:43) and counts the ids out
     of range, which the host reads back once to raise the reference's errors;
  2. gsp_row_sparse_compact projects only those rows and writes the logits in
     ascending token order, i.e. exactly ProjectionResult.logits.

The mode string reports the reference's density rule (gsp/runtime.py:44-48);
both modes produce identical values here, because the row-sparse kernel reads
no more of W than a dense projection would.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from . import _native


@dataclass(frozen=True)
class ProjectionResult:
    token_ids: torch.Tensor
    logits: torch.Tensor
    mode: str


def _check_operands(hidden: torch.Tensor, weight: torch.Tensor) -> None:
    if weight.device.type != "cuda" or hidden.device.type != "cuda":
        raise ValueError("hidden and weight must be CUDA tensors")
    if weight.ndim != 2:
        raise ValueError("weight must have shape [V, D]")
    if hidden.ndim not in (1, 2) or hidden.shape[-1] != weight.shape[1]:
        raise ValueError("hidden must have shape [D] or [B, D] matching weight")
    if hidden.dtype != weight.dtype:
        raise ValueError("hidden and weight dtypes must match")
    _native.dtype_code(weight.dtype)


def constrained_projection(
    hidden: torch.Tensor,
    weight: torch.Tensor,
    allowed_ids: Optional[torch.Tensor],
    *,
    dense_threshold: float = 0.30,
) -> ProjectionResult:
    """Project only legal vocabulary rows.

    Returns logits paired with the token ids they belong to, ids ascending and
    unique; the distribution equals dense projection followed by masking every
    token outside allowed_ids (gsp/runtime.py:16-51).
    """
    _check_operands(hidden, weight)
    vocab = weight.shape[0]
    hidden_2d = hidden.reshape(1, -1) if hidden.ndim == 1 else hidden
    if not hidden_2d.is_contiguous():
        hidden_2d = hidden_2d.contiguous()
    weight_c = weight if weight.is_contiguous() else weight.contiguous()
    batch = hidden_2d.shape[0]
    dev = weight.device

    if allowed_ids is None:
        ids = torch.arange(vocab, device=dev, dtype=torch.long)
        logits = torch.empty((batch, vocab), device=dev, dtype=weight.dtype)
        if batch == 1:
            _native.row_sparse(hidden_2d, weight_c, None, logits=logits)
        else:
            _native.dense_masked(hidden_2d, weight_c, None, logits=logits)
        return ProjectionResult(ids, logits[0] if hidden.ndim == 1 else logits, "dense-unconstrained")

    ids_in = allowed_ids.to(device=dev, dtype=torch.long)
    if ids_in.ndim != 1:
        raise ValueError("allowed_ids must be one-dimensional")
    if ids_in.numel() == 0:
        raise ValueError("grammar produced an empty legal-token set")
    ids_in = ids_in.contiguous()
    words = (vocab + 31) // 32
    mask = torch.empty((1, words), device=dev, dtype=torch.int32)
    stats = torch.empty(2, device=dev, dtype=torch.int64)
    _native.ids_to_bitmask(ids_in, vocab, mask, stats)
    unique, out_of_range = stats.tolist()
    if out_of_range:
        raise ValueError("allowed_ids contains an out-of-range token ID")

    density = unique / vocab
    mode = "dense-selected" if density >= dense_threshold else "sparse-gather"
    # One shared mask row for every request (row stride 0).
    mask_b = mask.expand(batch, words)
    compact = torch.empty(batch * unique, device=dev, dtype=weight.dtype)
    compact_ids = torch.empty(batch * unique, device=dev, dtype=torch.long)
    offsets = torch.empty(batch + 1, device=dev, dtype=torch.long)
    _native.row_sparse_compact(hidden_2d, weight_c, mask_b, compact, compact_ids, offsets)
    logits = compact.view(batch, unique)
    token_ids = compact_ids[:unique]
    return ProjectionResult(token_ids, logits[0] if hidden.ndim == 1 else logits, mode)
