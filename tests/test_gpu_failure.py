"""GPU failure detection without a fault: a bounded device-side wait that
runs out (a flag that nothing sets) reports KVCA_ERR_DEVICE_TIMEOUT through
the status word, and the context stays usable."""
from __future__ import annotations

import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _selftest(ext, flag: torch.Tensor, from_value: int) -> int:
    return ext._lib_handle.kvca_wait_selftest(ctypes.c_void_p(flag.data_ptr()), from_value,
                                              ctypes.c_void_p(ext.status_word(DEV).data_ptr()),
                                              ext._stream(DEV))


def test_bounded_wait_runs_out_and_reports():
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as ext

    ext.check_status(DEV)
    flag = torch.zeros(1, dtype=torch.int32, device=DEV)  # nothing sets it
    t0 = time.perf_counter()
    assert _selftest(ext, flag, 0) == 0
    with pytest.raises(RuntimeError, match="bounded device-side wait"):
        ext.check_status(DEV)
    assert time.perf_counter() - t0 < 30.0
    # the context is still usable
    actual = torch.arange(32, dtype=torch.float32, device=DEV).view(4, 8)
    assert torch.equal(ext.gather_blocks(actual, torch.tensor([2, 0], device=DEV)), actual[[2, 0]])
    ext.check_status(DEV)


def test_bounded_wait_ends_when_the_word_differs():
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as ext

    flag = torch.ones(1, dtype=torch.int32, device=DEV)
    assert _selftest(ext, flag, 0) == 0
    ext.check_status(DEV)
