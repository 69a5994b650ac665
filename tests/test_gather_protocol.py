"""A model check of the multi-GPU gather's epoch protocol (CPU only).

nvb_paged_decode_gather(_capturable) (csrc/gather.cu): at step n every rank
stores its heads of the result into output set n & 1 of every rank (peer
stores over NVLink), then releases epoch n into each peer's flag slot and
waits until every peer's epoch n has arrived in its own slots. Release and
acquire at system scope mean a peer that sees epoch n from rank p also sees
all of p's step-n stores. Work on a rank's stream runs in order.

The model runs N ranks under a random scheduler: each peer store lands at
any time before the storing rank's release, and ranks run independently
except through the flags. A consumer of step n reads the rank's set n & 1
and must see every rank's step-n contribution, and none of a later step's.
The documented contract holds: enqueue the readers of step n before the
rank's next call. The model also shows what goes wrong with the readers
enqueued after the next call: a peer one step ahead overwrites the set.
"""
import random

import pytest


def run(seed, world, steps, readers_after_next_call=False):
    rng = random.Random(seed)
    # buf[q][s][p]: the step whose rank-p contribution sits in rank q's output set s
    buf = [[[0] * world for _ in range(2)] for _ in range(world)]
    flag = [[0] * world for _ in range(world)]  # flag[q][p]: last epoch rank p released into rank q's slots
    pending = []  # stores issued but not landed: (p, q, s, n)
    violations = []

    def stream(r):
        """Rank r's stream: the ops its host enqueued, in order."""
        ops = []
        for n in range(1, steps + 1):
            ops.append(("step", n))
            if not readers_after_next_call:
                ops.append(("read", n))
            elif n >= 2:
                ops.append(("read", n - 1))
        if readers_after_next_call:
            ops.append(("read", steps))
        for op, n in ops:
            if op == "read":
                s = n & 1
                yield "run"
                seen = list(buf[r][s])
                if seen != [n] * world:
                    violations.append((r, n, seen))
                continue
            s = n & 1
            for q in range(world):  # the combine's stores into every rank's set n & 1
                pending.append((r, q, s, n))
            # release: visible only after this rank's step-n stores landed
            while any(p == r and m == n for p, _, _, m in pending):
                yield "blocked"
            for q in range(world):
                flag[q][r] = n
            # acquire: wait for every peer's epoch n
            while any(flag[r][p] < n for p in range(world)):
                yield "blocked"

    gens = {r: stream(r) for r in range(world)}
    state = {r: "run" for r in range(world)}
    done = set()
    for _ in range(100000):
        live = [r for r in gens if r not in done]
        if not live and not pending:
            return violations
        choices = [("rank", r) for r in live] + [("land", i) for i in range(len(pending))]
        kind, x = rng.choice(choices)
        if kind == "land":
            p, q, s, n = pending.pop(x)
            buf[q][s][p] = n
            continue
        try:
            state[x] = next(gens[x])
        except StopIteration:
            done.add(x)
    raise AssertionError("the exchange did not finish (deadlock)")


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_readers_before_next_call_see_every_step_complete(world):
    for seed in range(80):
        assert run(seed, world, steps=7) == [], seed


def test_readers_after_next_call_can_be_overwritten():
    """The placement the contract rules out does race: some schedule lets a
    peer one step ahead store step n + 2 into the set before it is read."""
    found = [v for seed in range(200) for v in run(seed, 2, steps=6, readers_after_next_call=True)]
    assert found, "expected a schedule where a later step overwrites an unread set"
    assert any(seen[p] > n for _, n, seen in found for p in range(2))
