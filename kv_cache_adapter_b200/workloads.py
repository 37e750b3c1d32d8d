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


# ---------------------------------------------------------------------------
# Decode append + gather mix (reshape-and-cache with clock eviction)
# ---------------------------------------------------------------------------


class DecodeMix:
    """A paged KV pool serving `seqs` decoding sequences, one token each per step.

    The pool (``num_blocks`` blocks of ``block_size`` tokens, every block of
    every plane = layer x K/V) starts full: every block holds a resident
    logical block, unpinned, usage uniform in 0..3.  Each sequence owns one
    pinned block it is filling (seeded random fill positions, so sequences
    fill up on different steps).  One step:

      1. every sequence whose block is full gets a new one: the clock sweep
         pops that many victims (the pool is full, so each one evicts its
         logical block), the victims' bytes of every plane are gathered into
         a spill chunk (the copy an LMCache-style store would take), the new
         blocks are committed as freshly saved and pinned (pin 1, usage 1)
         and the full blocks are released (pin 1 -> 0);
      2. one token per sequence is scattered into every plane through the
         per-token slot_mapping = block * block_size + position.

    ``ops`` supplies pop_reusable_slots, gather_layers, commit_save_metadata,
    release_metadata and scatter_tokens (the CUDA module, or a CPU stand-in in
    the tests); when it also has ``append_step`` the bookkeeping of step 1
    and the slot_mapping of step 2 run as that one launch.  All per-step state lives on the device; the host only keeps
    the fill positions, which decide which sequences need a block, so steps
    issue no host<->device traffic and a whole cycle of ``block_size`` steps
    can be captured in a CUDA graph (``capture_cycle``).

    ``pipelined`` (CUDA op set with ``append_step``): the bookkeeping runs on
    a stream of its own, one step ahead of the moves.  Step i + 1's
    bookkeeping reads and writes only metadata (slot_meta, l2p / p2l,
    search_start, the sequences' blocks and positions) and its own half of
    double-buffered victim and slot_mapping arrays, so it overlaps step i's
    gather and scatter, which touch only cache bytes; step i + 1's moves
    still wait for its bookkeeping.  Step i's bookkeeping waits for the
    moves of step i - 2, the last readers of the buffer half it rewrites.
    The moves stay in order on the caller's stream (a block released at step
    i and popped at step i + 1 is spilled after step i's scatter wrote its
    last token).  Results are the same bytes as unpipelined.  (Running the
    spill gathers on a third stream, so that step i + 1's gather overlaps
    step i's scatter, is safe, as the pop of a step precedes that step's
    release, but was slower on B200: 36.9 against 29.3 us per step with 8
    KV heads.)
    """

    CYCLE_BUFFERS = 3  # cycles of victims / slot mappings in flight; also the cycles per capture_cycles replay

    def __init__(self, ops, device, *, layers: int = 32, heads: int = 1, head_dim: int = 128,
                 block_size: int = 16, num_blocks: int = 65536, seqs: int = 256,
                 dtype=torch.float16, seed: int = 1234, max_steps: int = 1000):
        self.ops = ops
        self.device = device
        self.layers, self.block_size, self.seqs = layers, block_size, seqs
        self.num_blocks = num_blocks
        gen_dev = torch.Generator(device=device).manual_seed(seed) if device.type == "cuda" else \
            torch.Generator().manual_seed(seed)
        self.kv = torch.empty((layers, 2, num_blocks, block_size, heads, head_dim), dtype=dtype, device=device)
        self.kv.normal_(generator=gen_dev)
        self.block_planes = [self.kv[l, 0] for l in range(layers)] + [self.kv[l, 1] for l in range(layers)]
        self.token_planes = [p.reshape(num_blocks, block_size, heads * head_dim) for p in self.block_planes]
        table = getattr(ops, "PlaneTable", None)
        self.block_table = table(self.block_planes, 1) if table else self.block_planes
        self.token_table = table(self.token_planes, 2) if table else self.token_planes
        self.num_planes = len(self.block_planes)
        self.row_shape = (heads * head_dim,)
        rng = np.random.default_rng(seed)
        # logical ids: the resident ones, then fresh ids for new blocks
        self.num_logical = num_blocks + seqs * (max_steps // block_size + 2)
        resident = rng.permutation(num_blocks).astype(np.int64)  # logical id of each slot
        l2p = np.full(self.num_logical, -1, np.int64)
        l2p[resident] = np.arange(num_blocks)
        usage = rng.integers(0, 4, num_blocks)
        pins = np.zeros(num_blocks, np.int64)
        cur_block = rng.choice(num_blocks, seqs, replace=False).astype(np.int64)
        pins[cur_block] = 1
        self.pos = rng.integers(0, block_size, seqs).astype(np.int64)
        meta = (pins & 15) | ((usage & 15) << 4)
        self.slot_meta = torch.tensor(meta.astype(np.uint8), device=device)
        self.l2p = torch.tensor(l2p, device=device)
        self.p2l = torch.tensor(resident, device=device)
        self.search_start = torch.zeros(1, dtype=torch.int64, device=device)
        # device copies (never aliases of the host arrays, also on the CPU)
        self.cur_block_dev = torch.tensor(cur_block, device=device)
        self.cur_logical_dev = torch.tensor(resident[cur_block], device=device)
        self.pos_dev = torch.tensor(self.pos, device=device)
        self.next_logical_dev = torch.tensor([num_blocks], dtype=torch.int64, device=device)
        self.spill = torch.empty((seqs, self.num_planes, 1, block_size, heads, head_dim), dtype=dtype,
                                 device=device)
        self.empty_ids = torch.empty(0, dtype=torch.int64, device=device)
        # one-launch bookkeeping when the op set has it (the CUDA module)
        self._append = getattr(ops, "append_step", None)
        # whole-cycle booking (append_steps): a cycle = block_size steps, after
        # which the fill positions repeat, so every sequence gets exactly one
        # new block per cycle
        self._append_many = getattr(ops, "append_steps", None)
        # victims and slot mappings of CYCLE_BUFFERS cycles: the booking of
        # cycle k rewrites the buffer that the moves of cycle k - 3 read, so
        # the booking stream may run up to two cycles ahead of the moves
        # (with two buffers each booking waited for the previous cycle's
        # moves, and the current cycle's last step waited for that booking:
        # B200, 1 KV head, 5.3 against 4.6 us per decode step)
        self.cycle_victims = [torch.empty(seqs, dtype=torch.int64, device=device)
                              for _ in range(self.CYCLE_BUFFERS)]
        self.cycle_slot_mapping = [torch.empty((block_size, seqs), dtype=torch.int64, device=device)
                                   for _ in range(self.CYCLE_BUFFERS)]
        self._cycles_on = False
        self._cycle_queue = []  # (buffer, need offsets) of the cycles booked and not yet moved
        self._cycle_half = 0  # the buffer of the next cycle to book
        self._cycle_booked = self._cycle_moved = None
        self._pair = getattr(ops, "scatter_tokens_gather_layers", None)
        self._head_gathered = False  # the first gather of the next cycle to move went with the previous one
        # a whole cycle's moves in one launch (move_cycle) when the op set has it
        self._cycle_op = getattr(ops, "move_cycle", None)
        self._one_launch = False
        self._schedules = {}  # fill positions (bytes) -> (need, offsets on the device, offsets on the host)
        self.victims_bufs = [torch.empty(seqs, dtype=torch.int64, device=device) for _ in range(2)]
        self.slot_mapping_bufs = [torch.empty(seqs, dtype=torch.int64, device=device) for _ in range(2)]
        self._half = 0  # the buffer half of the next step
        self._pipelined = False
        self._book_stream = None
        self._booked = self._moved = None
        self._need = {}  # need set (bytes) -> (index tensor, ones, arange) on the device
        self.evictions = 0
        self.tokens = 0
        self.gathered_blocks = 0

    @property
    def slot_mapping_buf(self) -> torch.Tensor:
        """The slot_mapping of the last step."""
        return self.slot_mapping_bufs[self._half ^ 1]

    @property
    def pipelined(self) -> bool:
        return self._pipelined

    @pipelined.setter
    def pipelined(self, on: bool) -> None:
        on = bool(on) and self.device.type == "cuda" and self._append is not None
        if on and self._book_stream is None:
            self._book_stream = torch.cuda.Stream(self.device)
            self._booked = [torch.cuda.Event() for _ in range(2)]
            self._moved = [torch.cuda.Event() for _ in range(2)]
        if on != self._pipelined:  # switch between steps with nothing in flight on the side stream
            torch.cuda.current_stream(self.device).wait_stream(self._book_stream)
            self._book_stream.wait_stream(torch.cuda.current_stream(self.device))
        self._pipelined = on

    def need_new_blocks(self) -> np.ndarray:
        return np.nonzero(self.pos == self.block_size)[0]

    def _need_tensors(self, need: np.ndarray):
        key = need.tobytes()
        got = self._need.get(key)
        if got is None:
            c = int(need.size)
            got = (torch.tensor(need, device=self.device), torch.ones(c, dtype=torch.uint8, device=self.device),
                   torch.arange(c, dtype=torch.int64, device=self.device))
            self._need[key] = got
            if self._pipelined:  # made on the caller's stream, read on the bookkeeping stream
                self._book_stream.wait_stream(torch.cuda.current_stream(self.device))
        return got

    def step(self, token_rows: torch.Tensor, *, check: bool = False):
        """token_rows: (1, num_planes, seqs, *row) chunk of this step's tokens.
        Returns the spill chunk of the blocks evicted this step (a view)."""
        need = self.need_new_blocks()
        c = int(need.size)
        spill = self.spill[:c]
        if self._append is not None:
            need_dev = self._need_tensors(need)[0] if c else self.empty_ids
            h = self._half
            self._half ^= 1
            victims = self.victims_bufs[h][:c]
            slot_mapping = self.slot_mapping_bufs[h]

            def book():
                self._append(self.slot_meta, self.search_start, self.l2p, self.p2l, need_dev, self.cur_block_dev,
                             self.cur_logical_dev, self.pos_dev, self.block_size, self.next_logical_dev, victims,
                             slot_mapping, check=check)

            if self._pipelined:
                moves = torch.cuda.current_stream(self.device)
                self._book_stream.wait_event(self._moved[h])  # step i - 2's moves: the last readers of half h
                with torch.cuda.stream(self._book_stream):
                    book()
                    self._booked[h].record(self._book_stream)
                moves.wait_event(self._booked[h])
            else:
                book()
            if c:
                self.ops.gather_layers(self.block_table, victims, spill, blocks_per_chunk=1, check=check)
                self.pos[need] = 0
                self.evictions += c
                self.gathered_blocks += c
            self.ops.scatter_tokens(self.token_table, slot_mapping, token_rows, tokens_per_chunk=self.seqs,
                                    check=check)
            if self._pipelined:
                self._moved[h].record(torch.cuda.current_stream(self.device))
            self.pos += 1
            self.tokens += self.seqs
            return spill
        if c:
            ops = self.ops
            need_dev, ones, offsets = self._need_tensors(need)
            victims = ops.pop_reusable_slots(self.slot_meta, self.search_start, self.empty_ids, c, check=check)
            evicted = self.p2l.index_select(0, victims)
            ops.gather_layers(self.block_table, victims, spill, blocks_per_chunk=1, check=check)
            new_ids = self.next_logical_dev + offsets
            self.next_logical_dev += c
            ops.commit_save_metadata(self.l2p, self.p2l, self.slot_meta, evicted, new_ids, victims, ones, ones,
                                     check=check)
            ops.release_metadata(self.l2p, self.slot_meta, self.cur_logical_dev.index_select(0, need_dev),
                                 check=check)
            self.cur_block_dev.index_copy_(0, need_dev, victims)
            self.cur_logical_dev.index_copy_(0, need_dev, new_ids)
            self.pos[need] = 0
            self.pos_dev.index_fill_(0, need_dev, 0)
            self.evictions += c
            self.gathered_blocks += c
        slot_mapping = self.cur_block_dev * self.block_size + self.pos_dev
        self.ops.scatter_tokens(self.token_table, slot_mapping, token_rows, tokens_per_chunk=self.seqs,
                                check=check)
        self.pos += 1
        self.pos_dev += 1
        self.tokens += self.seqs
        return spill

    def capture_cycle(self, token_rows: torch.Tensor):
        """Capture the next ``block_size`` steps (one full cycle of the fill
        positions, after which the schedule repeats) into a CUDA graph and
        return (graph, evictions per replay).  Every need set of the cycle
        must have been seen in eager steps before (their index tensors are
        made outside the capture), so run at least one cycle eagerly first;
        replaying the graph then advances the device state by one cycle."""
        counters = (self.evictions, self.tokens, self.gathered_blocks)
        pos = self.pos.copy()
        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        graph = torch.cuda.CUDAGraph()
        if self._pipelined:
            stream.wait_stream(self._book_stream)
        with torch.cuda.stream(stream):
            with torch.cuda.graph(graph, stream=stream):
                if self._pipelined:  # fork the bookkeeping stream from the capture; no outside events
                    for ev in self._moved:
                        ev.record(stream)
                    self._book_stream.wait_stream(stream)
                for _ in range(self.block_size):
                    self.step(token_rows, check=False)
        torch.cuda.current_stream(self.device).wait_stream(stream)
        if self._pipelined:  # later eager steps wait on real records, not on captured ones
            cur = torch.cuda.current_stream(self.device)
            self._book_stream.wait_stream(cur)
            for ev in self._moved + self._booked:
                ev.record(cur)
        per_replay = self.evictions - counters[0]
        self.evictions, self.tokens, self.gathered_blocks = counters
        assert np.array_equal(self.pos, pos)  # a full cycle: the schedule repeats
        return graph, per_replay

    # ---- whole-cycle booking --------------------------------------------
    #
    # The bookkeeping of a step reads and writes only metadata, and which
    # sequences need a block in the next block_size steps follows from the
    # fill positions.  So one append_steps launch books a whole cycle (pop,
    # commit, release and slot_mapping of each of its steps, in order), on
    # the bookkeeping stream, ahead of the token moves: while the moves of
    # cycle c run, cycle c + 1 is booked.  Victims and slot_mapping rotate
    # through CYCLE_BUFFERS buffers by cycle; cycle c + 1's booking waits
    # for the moves of cycle c + 1 - CYCLE_BUFFERS, the last readers of its
    # buffer, so the booking stream may run ahead.  The moves of each step
    # (the spill gather of its victims, then its token scatter) stay in step
    # order on the caller's stream, so every byte moved equals step-by-step.

    def _cycle_schedule(self, pos: np.ndarray):
        """Need lists of the block_size steps from fill positions `pos`, as
        device tensors (need ids, CSR offsets) and the offsets on the host
        (cached: the schedule repeats every cycle)."""
        key = pos.tobytes()
        got = self._schedules.get(key)
        if got is None:
            pos = pos.copy()
            ids, offs = [], [0]
            for _ in range(self.block_size):
                need = np.nonzero(pos == self.block_size)[0]
                ids.append(need)
                offs.append(offs[-1] + int(need.size))
                pos[need] = 0
                pos += 1
            need_all = np.concatenate(ids).astype(np.int64)
            got = (torch.tensor(need_all, device=self.device),
                   torch.tensor(np.array(offs, np.int64), device=self.device), offs)
            self._schedules[key] = got
            # made on the caller's stream, read on the bookkeeping stream
            self._book_stream.wait_stream(torch.cuda.current_stream(self.device))
        return got

    def start_cycles(self, one_launch: bool = False) -> None:
        """Switch to whole-cycle booking and book the next cycle.  Call at a
        step count that is a multiple of block_size, with the per-step
        pipeline off.  Each step's scatter is paired with the next step's
        gather in one launch, and the spill holds the last step's victims;
        ``one_launch`` (op sets with move_cycle): each cycle's moves are one
        move_cycle launch instead, whose spill holds the whole cycle's
        victims (row offsets[q] + i: victim i of step q)."""
        assert self._append_many is not None and self.device.type == "cuda" and not self._cycles_on
        assert not self._pipelined
        self._one_launch = bool(one_launch)
        assert not self._one_launch or self._cycle_op is not None
        assert (self.pos >= 1).all()  # past the first step: the fill positions repeat every cycle
        if self._book_stream is None:
            self._book_stream = torch.cuda.Stream(self.device)
            self._booked = [torch.cuda.Event() for _ in range(2)]
            self._moved = [torch.cuda.Event() for _ in range(2)]
        if self._cycle_booked is None:
            self._cycle_booked = [torch.cuda.Event() for _ in range(self.CYCLE_BUFFERS)]
            self._cycle_moved = [torch.cuda.Event() for _ in range(self.CYCLE_BUFFERS)]
        self._book_stream.wait_stream(torch.cuda.current_stream(self.device))
        self._cycles_on = True
        self._head_gathered = False
        self._book_cycle()

    def _book_cycle(self) -> None:
        need, offsets, offs = self._cycle_schedule(self.pos)
        h = self._cycle_half
        self._cycle_half = (h + 1) % self.CYCLE_BUFFERS
        bs = self._book_stream
        bs.wait_event(self._cycle_moved[h])  # the moves of the cycle CYCLE_BUFFERS back read buffer h
        with torch.cuda.stream(bs):
            self._append_many(self.slot_meta, self.search_start, self.l2p, self.p2l, need, offsets,
                              self.cur_block_dev, self.cur_logical_dev, self.pos_dev, self.block_size,
                              self.next_logical_dev, self.cycle_victims[h][: offs[-1]],
                              self.cycle_slot_mapping[h], check=False)
            self._cycle_booked[h].record(bs)
        self._cycle_queue.append((h, offs, offsets))

    def _move_cycle(self, token_rows: torch.Tensor) -> None:
        """The moves of the oldest booked cycle.  ``token_rows``: one step's
        rows ``(1, P, seqs, *row)`` for every step, or ``(block_size, P, seqs,
        *row)`` with step i's rows at index i.  In one-launch mode the
        cycle's gathers and scatters are one move_cycle launch.  Otherwise,
        with the pair op, step i's token scatter and step i + 1's spill
        gather go in one launch: the pop of step i + 1 precedes its release,
        so its victims were unpinned while step i wrote, and step i writes
        only its sequences' current, pinned blocks.  The last scatter of the
        cycle takes the first gather of the next cycle when that one is
        booked already."""
        h, offs, offsets = self._cycle_queue.pop(0)
        cur = torch.cuda.current_stream(self.device)
        cur.wait_event(self._cycle_booked[h])
        victims, slot_mapping = self.cycle_victims[h], self.cycle_slot_mapping[h]
        per_step = token_rows.shape[0] > 1
        assert token_rows.shape[0] in (1, self.block_size)
        if self._one_launch:
            self._cycle_op(self.token_table, slot_mapping, token_rows, self.block_table, victims[: offs[-1]],
                           offsets, self.spill[: offs[-1]], check=False)
            self._cycle_moved[h].record(cur)
            self.evictions += offs[-1]
            self.gathered_blocks += offs[-1]
            self.tokens += self.block_size * self.seqs
            return
        pair = self._pair
        if pair is None or not self._head_gathered:
            a, b = offs[0], offs[1]
            if b > a:
                self.ops.gather_layers(self.block_table, victims[a:b], self.spill[: b - a], blocks_per_chunk=1,
                                       check=False)
        self._head_gathered = False
        for step in range(self.block_size):
            if pair is None:
                if step > 0 and offs[step + 1] > offs[step]:
                    a, b = offs[step], offs[step + 1]
                    self.ops.gather_layers(self.block_table, victims[a:b], self.spill[: b - a],
                                           blocks_per_chunk=1, check=False)
                self.ops.scatter_tokens(self.token_table, slot_mapping[step],
                                        token_rows[step:step + 1] if per_step else token_rows,
                                        tokens_per_chunk=self.seqs, check=False)
                continue
            if step + 1 < self.block_size:  # with the next step's gather
                nv = victims[offs[step + 1]:offs[step + 2]]
            elif self._cycle_queue:  # with the next cycle's first gather
                nh, noffs, _ = self._cycle_queue[0]
                cur.wait_event(self._cycle_booked[nh])
                nv = self.cycle_victims[nh][noffs[0]:noffs[1]]
                self._head_gathered = True
            else:
                nv = self.empty_ids
            # the indices come from the booking (another stream, waited for) and
            # the token rows from before the cycle, and after the first pair of
            # the cycle the kernels before a pair are pairs, which write none of
            # them; the first one waits for whatever the caller ran before
            pair(self.token_table, slot_mapping[step], token_rows[step:step + 1] if per_step else token_rows,
                 self.block_table, nv,
                 self.spill[: nv.numel()], tokens_per_chunk=self.seqs, blocks_per_chunk=1,
                 inputs_ready=step > 0, check=False)
        self._cycle_moved[h].record(cur)
        self.evictions += offs[-1]
        self.gathered_blocks += offs[-1]
        self.tokens += self.block_size * self.seqs

    def run_cycle(self, token_rows: torch.Tensor) -> None:
        """Book the cycle after the next one's moves, then enqueue the next
        cycle's moves (block_size steps, each with the same token rows)."""
        assert self._cycles_on
        self._book_cycle()
        self._move_cycle(token_rows)

    def stop_cycles(self, token_rows: torch.Tensor) -> None:
        """Move the cycle booked ahead and leave whole-cycle booking: the
        state then equals that of the same number of single steps."""
        assert self._cycles_on
        self._move_cycle(token_rows)
        assert not self._cycle_queue
        torch.cuda.current_stream(self.device).wait_stream(self._book_stream)
        self._cycles_on = False

    def capture_cycles(self, token_rows: torch.Tensor):
        """Capture CYCLE_BUFFERS cycles of ``run_cycle`` (the buffers rotate by
        cycle, so a replay ends on the buffer it started from) into a CUDA
        graph: within a replay the bookings of the next cycles overlap the
        moves of the current one.  The schedule's tensors must exist (run a
        cycle eagerly first).  Replays must be issued on the caller's stream
        after anything else on the bookkeeping stream; returns (graph,
        evictions per replay)."""
        assert self._cycles_on
        counters = (self.evictions, self.tokens, self.gathered_blocks)
        queue, half, head = list(self._cycle_queue), self._cycle_half, self._head_gathered
        cur = torch.cuda.current_stream(self.device)
        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(cur)
        stream.wait_stream(self._book_stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(graph, stream=stream):
                # fork the bookkeeping stream; the booked cycle and the moved
                # ones before the replay are done when it starts
                for ev in self._cycle_booked + self._cycle_moved:
                    ev.record(stream)
                self._book_stream.wait_stream(stream)
                for _ in range(self.CYCLE_BUFFERS):
                    self.run_cycle(token_rows)
                stream.wait_stream(self._book_stream)
        cur.wait_stream(stream)
        self._book_stream.wait_stream(cur)
        for ev in self._cycle_booked + self._cycle_moved:  # later eager cycles wait on real records
            ev.record(cur)
        per_replay = self.evictions - counters[0]
        self.evictions, self.tokens, self.gathered_blocks = counters
        assert self._cycle_half == half and [q[0] for q in self._cycle_queue] == [q[0] for q in queue]
        assert self._head_gathered == head
        return graph, per_replay
