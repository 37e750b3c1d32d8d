"""KVCacheAdapter with 16-bit slot metadata (KVCA_SLOT_META_BITS=16), run in a
child process because the width is fixed when the adapter module loads."""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

from conftest import REPO


def _run(mode: str) -> None:
    env = dict(os.environ, KVCA_SLOT_META_BITS="16")
    proc = subprocess.run([sys.executable, str(REPO / "tests" / "meta16_program.py"), mode], env=env,
                          capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stdout[-2000:] + proc.stderr[-4000:]


def test_meta16_pins_and_usage_on_cpu():
    _run("cpu")


@pytest.mark.gpu
def test_meta16_adapter_paths_match_oracle():
    _run("gpu")


def test_meta16_reference_scenarios_on_cpu():
    """Scenarios recorded from the reference's own 16-bit mode."""
    _run("golden")


@pytest.mark.gpu
def test_meta16_reference_scenarios_on_gpu():
    _run("golden-gpu")
