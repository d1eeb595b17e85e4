"""A model of the low-latency all-reduce protocol (``csrc/kernels/allreduce_ll.cu``) checked
under random schedules, for groups of 2, 4 and 8 ranks (the GPU tests reach 2 and 4).

Every rank's buffer holds 8-byte words {payload, epoch} in slots [epoch parity][source rank]
[position]; a call at epoch e uses parity e & 1.  Each (rank, position) is a thread of the
rank's kernel; a rank starts its next call only when all its threads finished the current
one (consecutive launches on one stream).  Stores to a peer become visible after a random
delay and in any order; a word is written as a unit.  A read waits until its word carries the
call's epoch.  Calls mix the one-shot exchange (push the partial to every peer, sum every
rank's word in rank order) and the two-shot exchange (push to the slice owner; the owner
sums, adds the residual and pushes the result to every peer), as the set-up timing does.

Checked: no schedule deadlocks (a slot overwritten by epoch e + 2 before its epoch-e reader
read it would leave that reader waiting forever), and after every call all ranks hold the
exact rank-ordered sums.
"""
import random

import pytest


def _run(world: int, modes: list[str], seed: int, max_delay: int = 6, npos_per_rank: int = 2):
    rnd = random.Random(seed)
    H = world * npos_per_rank
    words: dict = {}                      # (buffer rank, parity, src, pos) -> (value, epoch)
    pending: list = []                    # (visible_at, key, word)
    h = [[0] * H for _ in range(world)]   # residual stream, identical on every rank
    expect = [0] * H
    step = 0

    def partial(r, c, p):
        return (r + 1) * 1000 + c * 10 + p

    def write(dst, par, src, pos, word):
        pending.append((step + rnd.randint(0, max_delay), (dst, par, src, pos), word))

    def thread(r, c, pos, mode):
        """One kernel thread: yields ('wait', key, epoch) and receives the payload."""
        e = c + 1
        par = e & 1
        mine = partial(r, c, pos)
        if mode == "oneshot":
            for p in range(world):
                if p != r:
                    write(p, par, r, pos, (mine, e))
            s = 0
            for p in range(world):  # rank order
                s += mine if p == r else (yield ("wait", (r, par, p, pos), e))
            h[r][pos] += s
            return
        owner = pos // (H // world)
        if owner != r:
            write(owner, par, r, pos, (mine, e))
            h[r][pos] = yield ("wait", (r, par, owner, pos), e)
            return
        s = 0
        for p in range(world):
            s += mine if p == r else (yield ("wait", (r, par, p, pos), e))
        h[r][pos] += s
        for p in range(world):
            if p != r:
                write(p, par, r, pos, (h[r][pos], e))

    # per rank: the current call index and its live threads [(gen, waiting-on or None)]
    call = [0] * world
    live: list[list] = [[] for _ in range(world)]

    def start_call(r):
        c = call[r]
        live[r] = []
        for pos in range(H):
            g = thread(r, c, pos, modes[c])
            try:
                live[r].append([g, g.send(None)])
            except StopIteration:
                pass

    for r in range(world):
        start_call(r)
    while True:
        step += 1
        # deliver stores whose time has come (any order among them)
        rnd.shuffle(pending)
        keep = []
        for t, k, w in pending:
            if t <= step:
                words[k] = w
            else:
                keep.append((t, k, w))
        pending = keep
        runnable = []
        for r in range(world):
            if call[r] >= len(modes):
                continue
            for i, (g, want) in enumerate(live[r]):
                _, key, e = want
                word = words.get(key)
                if word is not None and word[1] == e:
                    runnable.append((r, i, word[0]))
        if not runnable:
            if all(call[r] >= len(modes) for r in range(world)):
                break
            if not pending:
                raise AssertionError(f"deadlock at step {step}: calls {call}")
            continue
        r, i, val = rnd.choice(runnable)
        g = live[r][i][0]
        try:
            live[r][i][1] = g.send(val)
        except StopIteration:
            live[r].pop(i)
        if not live[r] and call[r] < len(modes):
            call[r] += 1          # the rank's kernel for this call finished
            if call[r] < len(modes):
                start_call(r)
    for c in range(len(modes)):
        for pos in range(H):
            expect[pos] += sum(partial(r, c, pos) for r in range(world))
    for r in range(world):
        assert h[r] == expect, (r, h[r], expect)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ll_protocol_random_schedules(world):
    rnd = random.Random(world)
    for seed in range(40):
        n = rnd.randint(3, 9)
        modes = [rnd.choice(["oneshot", "twoshot"]) for _ in range(n)]
        _run(world, modes, seed=seed * 101 + world)


def test_model_detects_a_broken_protocol():
    """Sanity check of the model: with a single slot parity (every call writing where the
    previous call's readers may still read), some schedule must fail."""
    failures = 0
    for seed in range(60):
        try:
            _run_single_parity(4, ["oneshot"] * 6, seed)
        except AssertionError:
            failures += 1
    assert failures > 0


def _run_single_parity(world, modes, seed):
    """The same protocol with the parity forced to 0 (one slot set for all epochs)."""
    rnd = random.Random(seed)
    H = world * 2
    words, pending = {}, []
    h = [[0] * H for _ in range(world)]
    step = 0

    def write(dst, src, pos, word):
        pending.append((step + rnd.randint(0, 6), (dst, src, pos), word))

    def thread(r, c, pos):
        e = c + 1
        mine = (r + 1) * 1000 + c * 10 + pos
        for p in range(world):
            if p != r:
                write(p, r, pos, (mine, e))
        s = 0
        for p in range(world):
            s += mine if p == r else (yield ("wait", (r, p, pos), e))
        h[r][pos] += s

    call = [0] * world
    live = [[] for _ in range(world)]

    def start(r):
        live[r] = []
        for pos in range(H):
            g = thread(r, call[r], pos)
            try:
                live[r].append([g, g.send(None)])
            except StopIteration:
                pass

    for r in range(world):
        start(r)
    while True:
        step += 1
        rnd.shuffle(pending)
        keep = []
        for t, k, w in pending:
            if t <= step:
                # a newer epoch's word replaces an older one (no parity separation)
                words[k] = w
            else:
                keep.append((t, k, w))
        pending = keep
        runnable = []
        for r in range(world):
            if call[r] >= len(modes):
                continue
            for i, (g, want) in enumerate(live[r]):
                _, key, e = want
                w = words.get(key)
                if w is not None and w[1] == e:
                    runnable.append((r, i, w[0]))
        if not runnable:
            if all(call[r] >= len(modes) for r in range(world)):
                break
            if not pending:
                raise AssertionError("deadlock")
            continue
        # favour the fastest rank so that it runs ahead of slow readers
        r, i, val = min(runnable, key=lambda x: (call[x[0]] * -1, rnd.random()))
        g = live[r][i][0]
        try:
            live[r][i][1] = g.send(val)
        except StopIteration:
            live[r].pop(i)
        if not live[r] and call[r] < len(modes):
            call[r] += 1
            if call[r] < len(modes):
                start(r)
