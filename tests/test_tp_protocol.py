"""Model check of the 2-rank peer reduction's slot / epoch protocol (redline_tiny_b200/tp.py, csrc/rl_tp.cu) on the
CPU: each rank is its stream's program order - per reduction e (slot e & 1): the projection GEMM writes the rank's
partial into slot s here and in the other rank's buffer, the signal stores e into the other rank's pad, the LayerNorm
waits until its own pad holds e for the other rank and then reads both partials of slot s. Random interleavings of the
two programs must never let a write of a slot overlap a read of it (the write comes only after every rank finished
the read of the previous epoch in that slot), and every read must see both partials of its own epoch.

The same check for the W-rank reduce-scatter form (tp.PeerRS: receive slots, the gathered A operand, two signals and
two waits per reduction) at 2, 3 and 4 ranks, and that dropping its all-gather wait breaks it."""

import random


def _run(seed, reductions=12, split_steps=True):
    rng = random.Random(seed)
    W = 2
    # mem[rank][slot][writer] = epoch of the partial stored there; pad[rank][slot][writer] = last signalled epoch
    mem = [[[0] * W for _ in range(2)] for _ in range(W)]
    pad = [[[0] * W for _ in range(2)] for _ in range(W)]
    reading = [[None] * W for _ in range(W)]   # reading[rank][writer] = (slot, epoch) while a read is in progress

    def program(r):
        for e in range(1, reductions + 1):
            s = e & 1
            for dst in range(W):               # mirror epilogue: the partial lands here and in the peer's buffer
                for w in range(W):
                    if reading[dst][w] is not None and reading[dst][w][0] == s:
                        raise AssertionError(f"rank {r} writes slot {s} (epoch {e}) while rank {dst} reads it")
                mem[dst][s][r] = e
                if split_steps:
                    yield
            for dst in range(W):               # signal: pad_dst[s][r] = e after the partial
                pad[dst][s][r] = e
            yield
            while any(pad[r][s][w] < e for w in range(W) if w != r):   # bounded wait in the kernel; here a yield
                yield
            for w in range(W):                 # the LayerNorm reads both partials of slot s
                reading[r][w] = (s, e)
                if mem[r][s][w] != e:
                    raise AssertionError(f"rank {r} reads epoch {mem[r][s][w]} of rank {w} in slot {s}, wants {e}")
                if split_steps:
                    yield
            for w in range(W):
                reading[r][w] = None
            yield

    progs = [program(r) for r in range(W)]
    live = list(range(W))
    steps = 0
    while live:
        r = rng.choice(live)
        try:
            next(progs[r])
        except StopIteration:
            live.remove(r)
        steps += 1
        assert steps < 100000, "no progress"


def test_slot_protocol_random_interleavings():
    for seed in range(3000):
        _run(seed)


def test_single_slot_would_race():
    """The check has teeth: with one slot for every reduction a write can overlap the other rank's read."""
    import pytest

    def one_slot(seed):
        rng = random.Random(seed)
        W = 2
        mem = [[0] * W for _ in range(W)]
        pad = [[0] * W for _ in range(W)]
        reading = [None] * W

        def program(r):
            for e in range(1, 9):
                for dst in range(W):
                    if reading[dst] is not None:
                        raise AssertionError("overlap")
                    mem[dst][r] = e
                    yield
                for dst in range(W):
                    pad[dst][r] = e
                yield
                while pad[r][1 - r] < e:
                    yield
                reading[r] = e
                yield
                reading[r] = None
                yield
        progs = [program(r) for r in range(W)]
        live = list(range(W))
        while live:
            r = rng.choice(live)
            try:
                next(progs[r])
            except StopIteration:
                live.remove(r)

    with pytest.raises(AssertionError):
        for seed in range(3000):
            one_slot(seed)


def _run_rs(seed, W, reductions=8, ag_wait=True):
    """The W-rank peer reduce-scatter (tp.PeerRS): per reduction e (slot s = e & 1) each rank's stream runs
    (a) the GEMM that reads its whole A operand `a` (the previous reduction's LayerNorm rows from every rank),
    (b) the projection GEMM storing its partial rows for owner o into o's receive slot [s][r], for every o,
    (c) the signal pad_rs[o][s][r] = e, (d) the bounded wait for pad_rs[r][s][w] >= e, (e) the LayerNorm reading its
    W received partials of slot s and storing its rows of y into every rank's `a`, (f) the signal pad_ag[o][r] = e,
    (g) the wait for pad_ag[r][w] >= e. No write may overlap a read of the same buffer, and every read must see the
    epoch it is meant to."""
    rng = random.Random(seed)
    recv = [[[0] * W for _ in range(2)] for _ in range(W)]       # recv[rank][slot][src] = epoch stored
    arows = [[0] * W for _ in range(W)]                            # arows[rank][owner] = epoch of those rows
    pad_rs = [[[0] * W for _ in range(2)] for _ in range(W)]
    pad_ag = [[0] * W for _ in range(W)]
    reading_recv = [None] * W                                      # (slot) while rank's LayerNorm reads recv
    reading_a = [False] * W                                        # while rank's GEMM reads its a

    def program(r):
        for e in range(1, reductions + 1):
            s = e & 1
            reading_a[r] = True                                    # (a)
            for o in range(W):
                if arows[r][o] != e - 1:
                    raise AssertionError(f"rank {r} reads rows of {o} at epoch {arows[r][o]}, wants {e - 1}")
                yield
            reading_a[r] = False
            for o in range(W):                                     # (b)
                if reading_recv[o] == s:
                    raise AssertionError(f"rank {r} writes slot {s} of rank {o} (epoch {e}) while {o} reads it")
                recv[o][s][r] = e
                yield
            for o in range(W):                                     # (c)
                pad_rs[o][s][r] = e
            yield
            while any(pad_rs[r][s][w] < e for w in range(W) if w != r):   # (d)
                yield
            reading_recv[r] = s                                    # (e)
            for w in range(W):
                if recv[r][s][w] != e:
                    raise AssertionError(f"rank {r} reads epoch {recv[r][s][w]} of rank {w} in slot {s}, wants {e}")
                yield
            for o in range(W):
                if reading_a[o]:
                    raise AssertionError(f"rank {r} writes its rows into rank {o}'s a while {o} reads it")
                arows[o][r] = e
                yield
            reading_recv[r] = None
            for o in range(W):                                     # (f)
                pad_ag[o][r] = e
            yield
            while ag_wait and any(pad_ag[r][w] < e for w in range(W) if w != r):   # (g)
                yield

    progs = [program(r) for r in range(W)]
    live = list(range(W))
    steps = 0
    while live:
        r = rng.choice(live)
        try:
            next(progs[r])
        except StopIteration:
            live.remove(r)
        steps += 1
        assert steps < 200000, "no progress"


def test_reduce_scatter_protocol_random_interleavings():
    for W in (2, 3, 4):
        for seed in range(600):
            _run_rs(seed, W)


def test_reduce_scatter_protocol_needs_the_all_gather_wait():
    """The check has teeth: without the wait after the all-gather signal a rank's GEMM can read rows that another
    rank has not stored yet, or that rank can store rows while it reads them."""
    import pytest
    with pytest.raises(AssertionError):
        for seed in range(600):
            _run_rs(seed, 3, ag_wait=False)
