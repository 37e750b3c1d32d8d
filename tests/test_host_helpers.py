"""CPU: host-side helpers of the adapter that need no device."""
from __future__ import annotations

import torch

from kv_cache_adapter_b200 import adapter as adapter_mod


def test_last_occurrences_keeps_the_last_of_each_id():
    ids = torch.tensor([3, 1, 3, 0, 1, 3])
    got = adapter_mod._last_occurrences(ids, 5)
    assert got.tolist() == [-1, -1, -1, 0, 1, 3]
    # an index_copy_ applied in order leaves what the filtered scatter leaves
    rows = torch.arange(6, dtype=torch.float32).view(6, 1)
    want = torch.zeros(5, 1).index_copy_(0, ids, rows)
    keep = got >= 0
    assert torch.equal(torch.zeros(5, 1).index_copy_(0, got[keep], rows[keep]), want)


def test_last_occurrences_marks_out_of_range_ids():
    got = adapter_mod._last_occurrences(torch.tensor([2, -4, 9, 2]), 5)
    assert got.tolist() == [-1, 5, 5, 2]  # bad ids become `size`, which a mover rejects


def test_take_handles_uint16_words():
    words = torch.tensor([1, 2, 65535, 7], dtype=torch.uint16)
    got = adapter_mod._take(words, torch.tensor([2, 0, 2]))
    assert got.dtype == torch.uint16 and got.to(torch.int32).tolist() == [65535, 1, 65535]
    assert adapter_mod._take(torch.tensor([5, 6]), torch.tensor([1])).tolist() == [6]
