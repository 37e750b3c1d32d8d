"""The reference's strict-path clock sweep as torch CPU ops -- TEST
INFRASTRUCTURE ONLY (the timed CPU baseline of a per-call pop).

``KVCacheAdapter._pop_reusable_slots`` (adapter.py:472-525) runs on CPU
tensors as a handful of torch ops per call: an availability mask with the
blocked slots cleared (``index_fill_``), the scan order from ``search_start``,
the mask and usage gathered in scan order (``index_select``), then one
boolean selection per usage class until ``count`` slots are found, an aging
pass over every slot when the last class is above 0, and the new scan start.
This module runs the same op sequence on the packed ``slot_meta`` words
(4-bit pin | 4-bit usage << 4, adapter.py:17-36) so that its time is the time
the reference's CPU path takes for one pop.  It is checked against the pops
recorded from the reference and against the C restatement by the CPU tests.
"""
from __future__ import annotations

import torch

PIN_BITS = 4
FIELD_MASK = 15


def pop_reusable_slots(slot_meta: torch.Tensor, search_start: torch.Tensor, blocked: torch.Tensor,
                       count: int) -> torch.Tensor:
    """Grouped-order pop on CPU uint8 ``slot_meta`` / int64 ``search_start``,
    both changed in place.  Raises RuntimeError when too few slots are free."""
    n = slot_meta.numel()
    if count == 0:
        return torch.empty(0, dtype=torch.int64)
    pins = torch.bitwise_and(slot_meta, FIELD_MASK)
    usage = torch.bitwise_right_shift(slot_meta, PIN_BITS)
    free = pins.eq(0)
    if blocked.numel():
        free.index_fill_(0, blocked, False)
    order = torch.remainder(torch.arange(n, dtype=torch.int64) + search_start[0], n)
    free_in_order = free.index_select(0, order)
    usage_in_order = usage.index_select(0, order)
    picked: list[torch.Tensor] = []
    have = 0
    for cls in range(FIELD_MASK + 1):
        members = order[free_in_order & usage_in_order.eq(cls)]
        take = members[: count - have]
        if take.numel() == 0:
            continue
        picked.append(take)
        have += take.numel()
        if have == count:
            if cls > 0:
                aged = torch.clamp(usage.to(torch.int32) - cls, min=0).to(torch.uint8)
                slot_meta.copy_(torch.bitwise_or(pins, torch.bitwise_left_shift(aged, PIN_BITS)))
            victims = torch.cat(picked)
            search_start[0] = (victims[-1] + 1) % n
            return victims
    raise RuntimeError("insufficient capacity")
