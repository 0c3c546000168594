"""Total cost of an assignment (reference sources/torchmatch/assignment/_cost.py:8-61)."""

from __future__ import annotations

import torch


def assignment_cost(cost: torch.Tensor, matches: torch.Tensor, *, reduction: str = "sum"):
    """Gather ``cost`` at a row->col mapping (``-1`` rows contribute 0).

    ``reduction``: ``"sum"`` (default), ``"mean"`` over matched rows, or
    ``"none"`` for the per-row costs.  (N, M)/(N,) gives a scalar,
    (B, N, M)/(B, N) gives (B,).
    """
    squeeze = cost.ndim == 2
    if squeeze:
        cost, matches = cost.unsqueeze(0), matches.unsqueeze(0)
    hit = matches >= 0
    per_row = torch.gather(cost, 2, matches.clamp(min=0).unsqueeze(-1)).squeeze(-1)
    per_row = torch.where(hit, per_row, per_row.new_zeros(()))
    if reduction == "none":
        out = per_row
    elif reduction == "mean":
        out = per_row.sum(dim=-1) / hit.sum(dim=-1).clamp(min=1).to(per_row.dtype)
    else:
        out = per_row.sum(dim=-1)
    return out[0] if squeeze else out
