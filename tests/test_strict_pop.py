"""CPU: the torch restatement of the reference's strict-path pop (the timed CPU
baseline of the per-call pop) against the pop cases recorded from the
reference itself and against the C restatement on the clock-stress table;
and the oracle's per-step threshold trace of a clock stream."""
from __future__ import annotations

import json

import numpy as np
import torch

import oracle
from oracle import strict_pop


def test_strict_pop_matches_recorded_reference_pops(golden_dir):
    cases = json.loads((golden_dir / "pop_u8.json").read_text())
    for i, c in enumerate(cases):
        meta = torch.tensor(c["slot_meta"], dtype=torch.uint8)
        ss = torch.tensor([c["search_start"]], dtype=torch.int64)
        blocked = torch.tensor(c["blocked"], dtype=torch.int64)
        if c["error"] is not None:
            try:
                strict_pop.pop_reusable_slots(meta, ss, blocked, c["count"])
            except RuntimeError:
                continue
            raise AssertionError(f"case {i}: no error")
        got = strict_pop.pop_reusable_slots(meta, ss, blocked, c["count"])
        assert got.tolist() == c["selected"], i
        assert meta.tolist() == c["after_slot_meta"], i
        assert int(ss[0]) == c["after_search_start"], i


def test_strict_pop_matches_c_restatement_on_the_stress_table():
    rng = np.random.default_rng(3)
    n = 1 << 16
    usage = rng.integers(0, 4, n)
    pins = (rng.random(n) < 0.05).astype(np.int64)
    meta = torch.from_numpy((pins | (usage << 4)).astype(np.uint8))
    meta_c = meta.clone()
    ss, ss_c = torch.zeros(1, dtype=torch.int64), torch.zeros(1, dtype=torch.int64)
    for call in range(30):
        blocked = torch.from_numpy(rng.integers(0, n, call % 5 * 7).astype(np.int64))
        count = int(rng.integers(1, 20_000))
        got = strict_pop.pop_reusable_slots(meta, ss, blocked, count)
        want = oracle.pop_reusable_slots(meta_c, ss_c, blocked, count)
        assert torch.equal(got, want) and torch.equal(meta, meta_c) and torch.equal(ss, ss_c), call


def test_clock_stream_trace_marks_the_aging_steps():
    """Each traced step's threshold equals the one a single pop on the same
    state finds (0: took usage-0 slots only; T > 0: aged every slot by T)."""
    rng = np.random.default_rng(11)
    n, steps, k = 512, 300, 5
    usage = rng.integers(1, 4, n)  # no zeros: the first pop ages
    pins = (rng.random(n) < 0.1).astype(np.int64)
    meta0 = torch.from_numpy((pins | (usage << 4)).astype(np.uint8))
    reacc = torch.from_numpy(rng.integers(0, n, steps * k).astype(np.int64))
    meta, ss = meta0.clone(), torch.zeros(1, dtype=torch.int64)
    victims, done, rc, th = oracle.clock_stream(meta, ss, steps, k, reacc, k, trace=True)
    assert rc == 0 and done == steps and int(th[0]) >= 1 and int((th > 0).sum()) >= 2
    m, s = meta0.clone(), torch.zeros(1, dtype=torch.int64)
    for step in range(steps):
        before = (m >> 4).clone()
        v = oracle.pop_reusable_slots(m, s, torch.empty(0, dtype=torch.int64), k)
        t = int(th[step])
        assert torch.equal(v, victims[step * k:(step + 1) * k])
        assert torch.equal(m >> 4, torch.clamp(before.to(torch.int64) - t, min=0).to(torch.uint8)), step
        m[v] = (m[v] & 15) | (1 << 4)
        ids = reacc[step * k:(step + 1) * k]
        w = m[ids]
        m[ids] = (w & 15) | (torch.clamp((w >> 4).to(torch.int64) + 1, max=15).to(torch.uint8) << 4)
    assert torch.equal(m, meta)
