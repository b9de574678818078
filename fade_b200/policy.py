"""Tier selection for one layer: ``_assign_one_layer`` (fade/policy.py:232-274).

The reference's policies (H2O, learned, position) end in this helper: sinks
and the recent window stay FP16, the middle tokens are ranked by their
accumulated attention score and the top ``int4_budget`` go to INT4, the next
``int2_budget`` to INT2, the rest are evicted.  It runs on the scores' device
(a CUDA tensor keeps the selection on the GPU: one sort, no host sync), and
its output feeds ``TieredKVCache.apply_tier_assignment``.
"""

from __future__ import annotations

import torch
from torch import Tensor

from fade_b200.cache import TIER_EVICT, TIER_FP16, TIER_INT2, TIER_INT4


def _assign_one_layer(S: int, scores: Tensor, n_sink: int, recent_window: int, int4_budget: int | None,
                      int2_budget: int) -> Tensor:
    """[S] int64 tiers in ascending position order.

    ``int4_budget=None`` (or a budget covering the whole middle) keeps every
    middle token in INT4 and evicts nothing.  Ranking is by descending score;
    the reference takes the same single descending sort, so equal scores are
    the only source of a possible difference (torch's sort order among ties).
    The middle is the contiguous range [n_sink, S - recent_window) and the
    tiers are set with slices and index_fill_, so on a CUDA tensor the
    selection makes no host synchronisation.
    """
    dev = scores.device
    head = min(n_sink, S)
    tail = max(head, S - recent_window)
    tiers = torch.full((S,), TIER_FP16, dtype=torch.long, device=dev)
    n_mid = tail - head
    if n_mid == 0:
        return tiers
    if int4_budget is None or int4_budget >= n_mid:
        tiers[head:tail] = TIER_INT4
        return tiers
    tiers[head:tail] = TIER_EVICT
    order = scores[head:tail].argsort(descending=True) + head
    tiers.index_fill_(0, order[:int4_budget], TIER_INT4)
    n2 = min(max(int2_budget, 0), n_mid - int4_budget)
    if n2 > 0:
        tiers.index_fill_(0, order[int4_budget:int4_budget + n2], TIER_INT2)
    return tiers


def assign_counts(S: int, n_sink: int, recent_window: int, int4_budget: int | None,
                  int2_budget: int) -> tuple[int, int, int]:
    """(FP16, INT4, INT2) entries of ``_assign_one_layer``'s result with the
    same arguments, from the budgets alone (for
    ``TieredKVCache.apply_tier_assignment(..., counts=...)``)."""
    head = min(n_sink, S)
    tail = max(head, S - recent_window)
    n_mid = tail - head
    if int4_budget is None or int4_budget >= n_mid:
        return S - n_mid, n_mid, 0
    b4 = max(int4_budget, 0)
    return S - n_mid, b4, min(max(int2_budget, 0), n_mid - b4)


__all__ = ["_assign_one_layer", "assign_counts"]
