"""Seeded input generators shared by the fixture script, the tests and bench.py.

Everything here is deterministic from its seed (Python ``random.Random`` and
numpy ``default_rng``, whose streams are stable across versions), so the
fixture generator, the CPU oracle and the GPU runs consume identical inputs.
"""
from __future__ import annotations

import hashlib
import random

import numpy as np
import torch

# ---------------------------------------------------------------------------
# Clock-sweep cases
# ---------------------------------------------------------------------------


def pop_case_params(count: int, seed: int, *, usage_max: int, pin_max: int):
    """Random single-pop cases over small tables, covering: T = 0 and T > 0,
    empty classes, pinned and blocked slots (duplicates included), every
    search start, and requests larger than the available set."""
    rng = random.Random(seed)
    for case in range(count):
        kind = case % 6
        n = rng.choice([1, 2, 3, 5, 8, 16, 17, 31, 33, 64, 100, 127, 128, 129, 255, 300])
        if kind == 0:  # uniform usage
            usage = [rng.randint(0, usage_max) for _ in range(n)]
        elif kind == 1:  # no zero usage: forces aging
            usage = [rng.randint(1, usage_max) for _ in range(n)]
        elif kind == 2:  # low usage, like a warm cache
            usage = [rng.randint(0, 3) for _ in range(n)]
        elif kind == 3:  # saturated
            usage = [rng.choice([usage_max, usage_max - 1, 1]) for _ in range(n)]
        elif kind == 4:  # sparse zeros
            usage = [0 if rng.random() < 0.05 else rng.randint(1, 6) for _ in range(n)]
        else:
            usage = [rng.randint(2, 5) for _ in range(n)]
        pin_p = rng.choice([0.0, 0.1, 0.3, 0.7])
        pins = [0 if rng.random() >= pin_p else rng.choice([1, 2, pin_max]) for _ in range(n)]
        nb = rng.choice([0, 0, 1, 2, max(1, n // 4), max(1, n // 2)])
        blocked = [rng.randrange(n) for _ in range(nb)]
        search_start = rng.randrange(n)
        available = sum(1 for i in range(n) if pins[i] == 0 and i not in set(blocked))
        if rng.random() < 0.12:
            want = available + rng.randint(1, 3)  # too many: insufficient capacity
        else:
            want = rng.randint(1, max(1, available)) if available else 1
        yield {
            "usage": usage,
            "pins": pins,
            "blocked": blocked,
            "search_start": search_start,
            "count": want,
        }


# ---------------------------------------------------------------------------
# Adapter scenarios (load / save / release sequences)
# ---------------------------------------------------------------------------


def scenario_specs(count: int, seed: int):
    rng = random.Random(seed)
    shapes = [[2], [3], [2, 4], [4], [2, 2, 2, 2]]
    for case in range(count):
        num_actual = rng.randint(1, 6)
        num_logical = rng.randint(num_actual, 12)
        block_shape = rng.choice(shapes)
        numel = int(np.prod(block_shape))
        present = [i for i in range(num_logical) if rng.random() < 0.7]
        initial = {
            str(i): [float(round(rng.uniform(-100, 100), 2)) for _ in range(numel)] for i in present
        }
        yield {
            "case": case,
            "seed": seed * 1000 + case,
            "num_actual": num_actual,
            "num_logical": num_logical,
            "block_shape": block_shape,
            "initial": initial,
            "num_ops": rng.randint(6, 18),
        }


def scenario_ops(spec: dict):
    """Deterministic op list for a scenario (independent of the adapter state)."""
    rng = random.Random(spec["seed"])
    numel = int(np.prod(spec["block_shape"]))
    loaded: list[int] = []
    ops = []
    for _ in range(spec["num_ops"]):
        r = rng.random()
        if r < 0.4:
            k = rng.randint(1, min(spec["num_actual"] + 1, spec["num_logical"]))
            ids = rng.sample(range(spec["num_logical"]), k)
            ops.append({"op": "load", "ids": ids})
            loaded.extend(ids)
        elif r < 0.7:
            k = rng.randint(1, min(spec["num_actual"] + 1, spec["num_logical"]))
            ids = rng.sample(range(spec["num_logical"]), k)
            data = [float(round(rng.uniform(-100, 100), 2)) for _ in range(k * numel)]
            ops.append({"op": "save", "ids": ids, "data": data})
        else:
            pool = sorted(set(loaded))
            if not pool:
                continue
            k = rng.randint(1, len(pool))
            ids = rng.sample(pool, k)
            for i in ids:
                loaded.remove(i)
            ops.append({"op": "release", "ids": ids})
    return ops


# ---------------------------------------------------------------------------
# Clock stress (pop + refill + Zipf re-access)
# ---------------------------------------------------------------------------


def clock_params(num_slots: int, num_steps: int, alloc_per_step: int, reaccess_per_step: int,
                 *, seed: int = 1234, zipf_s: float = 1.1, pinned_frac: float = 0.05,
                 usage_hi: int = 3) -> dict:
    return {
        "num_slots": int(num_slots),
        "num_steps": int(num_steps),
        "alloc_per_step": int(alloc_per_step),
        "reaccess_per_step": int(reaccess_per_step),
        "seed": int(seed),
        "zipf_s": float(zipf_s),
        "pinned_frac": float(pinned_frac),
        "usage_hi": int(usage_hi),
    }


def clock_stream_params_small() -> list[dict]:
    return [
        clock_params(2048, 400, 1, 1, seed=1234),
        clock_params(2048, 120, 16, 16, seed=1235),
        clock_params(1000, 200, 7, 9, seed=1236),
        clock_params(4096, 60, 256, 256, seed=1237),
        clock_params(300, 150, 3, 40, seed=1238, usage_hi=15, pinned_frac=0.2),
    ]


def clock_initial_meta(params: dict, pack) -> torch.Tensor:
    """usage ~ U{0..usage_hi}, pin = 1 with probability pinned_frac (else 0)."""
    rng = np.random.default_rng(params["seed"])
    n = params["num_slots"]
    usage = rng.integers(0, params["usage_hi"] + 1, size=n, dtype=np.int64)
    pins = (rng.random(n) < params["pinned_frac"]).astype(np.int64)
    return pack(torch.from_numpy(pins), torch.from_numpy(usage))


def zipf_reaccess(params: dict) -> torch.Tensor:
    """Truncated Zipf(s) over ranks 1..N by inverse CDF in float64, mapped to
    slot ids through a seeded permutation: num_steps * reaccess_per_step ids."""
    n = params["num_slots"]
    total = params["num_steps"] * params["reaccess_per_step"]
    rng = np.random.default_rng(params["seed"] + 7919)
    weights = np.arange(1, n + 1, dtype=np.float64) ** (-params["zipf_s"])
    cdf = np.cumsum(weights)
    cdf /= cdf[-1]
    u = rng.random(total)
    ranks = np.minimum(np.searchsorted(cdf, u, side="right"), n - 1)
    perm = rng.permutation(n)
    return torch.from_numpy(perm[ranks].astype(np.int64))


def sha256_of(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().cpu().contiguous().numpy().tobytes()).hexdigest()
