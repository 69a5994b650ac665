"""A model check of the tensor-core kernels' mbarrier protocols (CPU only):
the two decode kernels, the one-tile prefill kernel (csrc/prefill_tile.cu)
and the pair prefill kernel (csrc/prefill.cu), the last two modelled further
down.

csrc/decode_mma.cu and csrc/decode_persistent.cu stream K and V tiles
through one ring of kStages shared-memory slots (load n: K of tile n / 2
when n is even, its V when odd, in slot n % kStages), and coordinate a TMA
producer, an MMA-issuing thread, the tensor pipe and the softmax warps with
mbarriers waited on by phase parity. This test restates each role's loop as
a Python generator, with every wait's parity computed by the same formula as
the CUDA source, and runs them under a random scheduler with TMA loads that
land in any order and tensor-core operations that complete in issue order.

It checks, over random tile counts, masked tiles, item streams and ring
depths:
  * no deadlock;
  * every parity formula names the phase the waiter means (parity ==
    intended phase & 1), and no barrier ever runs two phases ahead of a
    waiter that has not yet passed its wait (a parity wait would alias);
  * no slot is reloaded before the MMA that reads it has run, every MMA
    reads the load it expects after it landed, the softmax zeroes V rows only
    of the tile's own landed V, P and S buffers are rewritten only after
    their readers, O is rescaled only between two tiles' PVs, and an item's
    first PV (which restarts O) runs only after the previous item's epilogue
    read O.

The four softmax warps act in lockstep on every barrier they share, so they
are one actor here (arrival counts 4 -> 1, the item ring's 5 -> 2).
"""
import random

import pytest


class Bar:
    def __init__(self, name, count):
        self.name, self.count, self.pending, self.done = name, count, count, 0

    def __repr__(self):
        return f"{self.name}(done={self.done}, pending={self.pending}/{self.count})"


class Sim:
    def __init__(self, seed, stages):
        self.rng = random.Random(seed)
        self.S = stages
        self.bars = {}
        self.waiting = {}  # actor -> (bar, k)
        self.loads = []  # in-flight TMA loads: (callback)
        self.tqs = {"mma": []}  # tensor-core operations per issuing thread, in issue order
        # data state
        self.slot_load = [None] * stages
        self.slot_ready = [False] * stages
        self.consumed = set()
        self.s_buf = [None, None]
        self.s_read = set()
        self.p_buf = None
        self.pv_done = -1
        self.q_item = None
        self.q_ready = False
        self.tile_item = {}
        self.first_tile = {}  # item -> first global tile
        self.last_tile = {}
        self.epilogue_done = set()
        self.s_done_tiles = set()

    def bar(self, name, count=1):
        if name not in self.bars:
            self.bars[name] = Bar(name, count)
        return self.bars[name]

    def arrive(self, name):
        b = self.bars[name]
        b.pending -= 1
        assert b.pending >= 0, b
        if b.pending == 0:
            b.done += 1
            b.pending = b.count
            for actor, (wb, k) in self.waiting.items():
                assert not (wb is b and b.done > k + 1), f"{b} ran two phases past a waiter of phase {k} ({actor})"

    # a wait instruction yielded by an actor
    @staticmethod
    def wait(name, parity, k):
        assert parity == (k & 1), f"parity formula {parity} names another phase than {k} on {name}"
        return ("wait", name, k)

    def run(self, actors):
        live = {a: g for a, g in actors.items()}
        instr = {}
        for a, g in live.items():
            instr[a] = next(g, None)

        def ready(a):
            i = instr[a]
            if i is None:
                return False
            if i[0] == "wait":
                b = self.bars[i[1]]
                return b.done >= i[2] + 1
            if i[0] == "tensor":
                return bool(self.tqs[i[1]])
            return True

        steps = 0
        while True:
            steps += 1
            assert steps < 200000, "simulation did not finish"
            for a, i in instr.items():
                if i is not None and i[0] == "wait":
                    b = self.bars[i[1]]
                    assert b.done <= i[2] + 1, f"{a} waits for phase {i[2]} of {b}: parity would alias"
                    self.waiting[a] = (b, i[2])
                else:
                    self.waiting.pop(a, None)
            choices = [("actor", a) for a in instr if ready(a)] + [("load", j) for j in range(len(self.loads))]
            if not choices:
                unfinished = [a for a, i in instr.items() if i is not None and not a.startswith("tensor")]
                if not unfinished and not any(self.tqs.values()):
                    return
                raise AssertionError(f"deadlock: {[(a, instr[a]) for a in unfinished]} bars={list(self.bars.values())}")
            kind, x = self.rng.choice(choices)
            if kind == "load":
                cb = self.loads.pop(x)
                cb()
                continue
            self.waiting.pop(x, None)  # it has passed its wait before it runs on
            try:
                instr[x] = next(live[x])
            except StopIteration:
                instr[x] = None

    # ---------------------------------------------------------------- events
    def issue_load(self, n, ok):
        s = n % self.S
        prev = self.slot_load[s]
        assert prev is None or (prev == n - self.S and prev in self.consumed), \
            f"load {n} overwrites slot {s} holding load {prev} before its MMA ran"
        self.slot_load[s], self.slot_ready[s] = n, False

        def land():
            assert self.slot_load[s] == n
            self.slot_ready[s] = True
            self.arrive(f"Full{s}")

        if ok:
            self.loads.append(land)
        else:  # invalid page: the producer arrives without a copy (stale slot, masked)
            land()

    def read_slot(self, n):
        s = n % self.S
        assert self.slot_load[s] == n and self.slot_ready[s], f"MMA reads load {n}, slot {s} holds {self.slot_load[s]}"
        self.consumed.add(n)

    def tensor(self, q="mma"):
        """One issuing thread's tcgen05 operations: they complete in issue
        order, and a commit arrives once everything before it completed."""
        while True:
            yield ("tensor", q)
            op = self.tqs[q].pop(0)
            if callable(op):
                op()
            elif op[0] == "S":
                _, g, item = op
                assert self.q_item == item and self.q_ready, f"S of tile {g} (item {item}) without its Q"
                self.read_slot(2 * g)
                sb = g & 1
                assert g < 2 or (g - 2) in self.s_read, f"S of tile {g} overwrites S of tile {g - 2} before it was read"
                self.s_buf[sb] = g
                self.s_done_tiles.add(g)
            elif op[0] == "PV":
                _, g = op
                self.read_slot(2 * g + 1)
                assert self.p_buf == g, f"PV of tile {g} reads P of tile {self.p_buf}"
                assert self.pv_done == g - 1, f"PV of tile {g} after PV of tile {self.pv_done}"
                item = self.tile_item[g]
                if self.first_tile[item] == g:  # restarts O: the previous item's epilogue must have read it
                    prev = [i for i in self.last_tile if self.last_tile[i] < g]
                    if prev:
                        assert max(prev, key=lambda i: self.last_tile[i]) in self.epilogue_done, \
                            f"item {item}'s first PV overwrites O before the previous epilogue read it"
                self.pv_done = g
            elif op[0] == "commit":
                self.arrive(op[1])
            elif op[0] == "qfree":
                self.arrive(op[1])

    def softmax_tile(self, g, j, masked, rescale):
        """Body of one softmax tile after SFull: returns the waits and checks as a generator."""
        sb = g & 1
        assert self.s_buf[sb] == g, f"softmax reads S of tile {g}, buffer holds {self.s_buf[sb]}"
        self.s_read.add(g)
        self.arrive(f"SFree{sb}")
        if j >= 1:
            yield self.wait("ODone", (g - 1) & 1, g - 1)
        if masked:
            n = 2 * g + 1
            s = n % self.S
            yield self.wait(f"Full{s}", (n // self.S) & 1, n // self.S)
            assert self.slot_load[s] == n and self.slot_ready[s] and n not in self.consumed, \
                f"softmax zeroes V rows of tile {g} in slot {s} holding load {self.slot_load[s]}"
        assert self.pv_done == g - 1, f"P of tile {g} written while PV of tile {self.pv_done + 1} may read P"
        self.p_buf = g
        if j >= 1 and rescale:
            assert self.pv_done == g - 1, "O rescaled while a PV is in flight"
        self.arrive("PFull")


# -------------------------------------------------- decode_mma_kernel (one item per CTA)
def run_decode_mma(seed, stages, ntiles, masked, page_ok):
    sim = Sim(seed, stages)
    S = stages
    for s in range(S):
        sim.bar(f"Full{s}"), sim.bar(f"Empty{s}")
    for s in range(2):
        sim.bar(f"SFull{s}"), sim.bar(f"SFree{s}")
    sim.bar("PFull"), sim.bar("ODone")
    for g in range(ntiles):
        sim.tile_item[g] = 0
    sim.first_tile[0], sim.last_tile[0] = 0, ntiles - 1
    sim.q_item, sim.q_ready = 0, True  # Q^T is written by the softmax warps before the roles start
    rng = random.Random(seed + 1)
    rescale = [rng.random() < 0.3 for _ in range(ntiles)]

    def producer():  # decode_mma.cu, warp 0
        for n in range(2 * ntiles):
            slot = n % S
            if n >= S:
                yield Sim.wait(f"Empty{slot}", ((n // S) + 1) & 1, n // S - 1)
            sim.issue_load(n, page_ok[n >> 1])
            yield ("step",)

    def mma():  # decode_mma.cu, warp 1
        def issue_pv(t):
            n, slot = 2 * t + 1, (2 * t + 1) % S
            yield Sim.wait("PFull", t & 1, t)
            yield Sim.wait(f"Full{slot}", (n // S) & 1, n // S)
            sim.tqs["mma"] += [("PV", t), ("commit", f"Empty{slot}"), ("commit", "ODone")]

        for j in range(ntiles):
            n, slot, sb = 2 * j, (2 * j) % S, j & 1
            yield Sim.wait(f"Full{slot}", (n // S) & 1, n // S)
            if j >= 2:
                yield Sim.wait(f"SFree{sb}", ((j >> 1) + 1) & 1, (j >> 1) - 1)
            sim.tqs["mma"] += [("S", j, 0), ("commit", f"Empty{slot}"), ("commit", f"SFull{sb}")]
            if j >= 1:
                yield from issue_pv(j - 1)
        yield from issue_pv(ntiles - 1)

    def softmax():  # decode_mma.cu, warps 2..5
        for j in range(ntiles):
            yield Sim.wait(f"SFull{j & 1}", (j >> 1) & 1, j >> 1)
            yield from sim.softmax_tile(j, j, masked[j], rescale[j])
        yield Sim.wait("ODone", (ntiles - 1) & 1, ntiles - 1)
        assert sim.pv_done == ntiles - 1
        sim.epilogue_done.add(0)

    sim.run({"producer": producer(), "mma": mma(), "softmax": softmax(), "tensor": sim.tensor("mma")})
    assert sim.pv_done == ntiles - 1 and 0 in sim.epilogue_done


# ------------------------------------------- decode_persistent_kernel (a stream of items)
def run_persistent(seed, stages, item_tiles, masked_p):
    sim = Sim(seed, stages)
    S = stages
    for s in range(S):
        sim.bar(f"Full{s}"), sim.bar(f"Empty{s}")
    for s in range(2):
        sim.bar(f"SFull{s}"), sim.bar(f"SFree{s}")
        sim.bar(f"ItemFull{s}"), sim.bar(f"ItemEmpty{s}", 2)  # MMA thread + softmax (4 warps -> 1 actor)
        sim.bar(f"QFull{s}")
    sim.bar("QEmpty"), sim.bar("PFull"), sim.bar("ODone")
    rng = random.Random(seed + 1)
    g = 0
    for i, nt in enumerate(item_tiles):
        if nt:
            sim.first_tile[i], sim.last_tile[i] = g, g + nt - 1
            for _ in range(nt):
                sim.tile_item[g] = i
                g += 1
    total = g
    masked = [rng.random() < masked_p for _ in range(total)]
    page_ok = [rng.random() < 0.9 for _ in range(total)]
    rescale = [rng.random() < 0.3 for _ in range(total)]
    END = -1
    items = list(item_tiles) + [END]
    ring = [None, None]

    def producer():  # decode_persistent.cu, warp 0
        g = ni = 0
        for i, nt in enumerate(items):
            if i >= 2:
                yield Sim.wait(f"ItemEmpty{i & 1}", ((i >> 1) + 1) & 1, (i >> 1) - 1)
            ring[i & 1] = (i, nt)
            sim.arrive(f"ItemFull{i & 1}")
            if nt == END:
                break
            if nt == 0:
                continue
            qb = ni & 1
            if ni >= 1:
                yield Sim.wait("QEmpty", (ni - 1) & 1, ni - 1)
            prev = [k for k in sim.last_tile if k < i]
            if prev:
                assert sim.last_tile[max(prev)] in sim.s_done_tiles, f"Q of item {i} overwrites Q still read by S"
            sim.q_item, sim.q_ready = i, False

            def q_land(i=i, qb=qb):
                assert sim.q_item == i
                sim.q_ready = True
                sim.arrive(f"QFull{qb}")

            sim.loads.append(q_land)
            ni += 1
            for _j in range(nt):
                for n in (2 * g, 2 * g + 1):
                    slot = n % S
                    if n >= S:
                        yield Sim.wait(f"Empty{slot}", ((n // S) + 1) & 1, n // S - 1)
                    sim.issue_load(n, page_ok[g])
                    yield ("step",)
                g += 1

    def mma():  # decode_persistent.cu, warp 1
        g = ni = 0

        def issue_pv(gt):
            n, slot = 2 * gt + 1, (2 * gt + 1) % S
            yield Sim.wait("PFull", gt & 1, gt)
            yield Sim.wait(f"Full{slot}", (n // S) & 1, n // S)
            sim.tqs["mma"] += [("PV", gt), ("commit", f"Empty{slot}"), ("commit", "ODone")]

        for i in range(len(items)):
            yield Sim.wait(f"ItemFull{i & 1}", (i >> 1) & 1, i >> 1)
            idx, nt = ring[i & 1]
            assert idx == i
            sim.arrive(f"ItemEmpty{i & 1}")
            if nt == END:
                break
            if nt == 0:
                continue
            qb = ni & 1
            yield Sim.wait(f"QFull{qb}", (ni >> 1) & 1, ni >> 1)
            ni += 1
            for j in range(nt):
                n, slot, sb = 2 * g, (2 * g) % S, g & 1
                yield Sim.wait(f"Full{slot}", (n // S) & 1, n // S)
                if g >= 2:
                    yield Sim.wait(f"SFree{sb}", ((g >> 1) + 1) & 1, (g >> 1) - 1)
                sim.tqs["mma"] += [("S", g, i), ("commit", f"Empty{slot}"), ("commit", f"SFull{sb}")]
                if j == nt - 1:
                    sim.tqs["mma"].append(("qfree", "QEmpty"))
                if j >= 1:
                    yield from issue_pv(g - 1)
                g += 1
            yield from issue_pv(g - 1)

    def softmax():  # decode_persistent.cu, warps 2..5
        g = 0
        for i in range(len(items)):
            yield Sim.wait(f"ItemFull{i & 1}", (i >> 1) & 1, i >> 1)
            idx, nt = ring[i & 1]
            assert idx == i
            sim.arrive(f"ItemEmpty{i & 1}")
            if nt == END:
                break
            if nt == 0:
                continue
            for j in range(nt):
                yield Sim.wait(f"SFull{g & 1}", (g >> 1) & 1, g >> 1)
                yield from sim.softmax_tile(g, j, masked[g], rescale[g])
                g += 1
            yield Sim.wait("ODone", (g - 1) & 1, g - 1)
            assert sim.pv_done == g - 1
            sim.epilogue_done.add(i)

    sim.run({"producer": producer(), "mma": mma(), "softmax": softmax(), "tensor": sim.tensor("mma")})
    assert sim.pv_done == total - 1
    assert sim.epilogue_done == {i for i, nt in enumerate(item_tiles) if nt}


# The kernels use 3 slots; 2 and 4 (the old split rings' K/V alternation
# patterns) and 5 check that the formulas do not depend on the depth.
@pytest.mark.parametrize("stages", [2, 3, 4, 5])
def test_decode_mma_ring_protocol(stages):
    for seed in range(60):
        rng = random.Random(1000 * stages + seed)
        ntiles = rng.choice([1, 2, 3, 4, 5, 7, 12])
        masked = [rng.random() < 0.4 for _ in range(ntiles)]
        page_ok = [rng.random() < 0.9 for _ in range(ntiles)]
        run_decode_mma(seed, stages, ntiles, masked, page_ok)


@pytest.mark.parametrize("stages", [2, 3, 4, 5])
def test_persistent_ring_protocol(stages):
    for seed in range(40):
        rng = random.Random(2000 * stages + seed)
        item_tiles = [rng.choice([0, 1, 1, 2, 3, 5]) for _ in range(rng.randint(1, 7))]
        run_persistent(seed, stages, item_tiles, masked_p=0.4)


def test_model_catches_a_wrong_parity():
    """The model is not vacuous: a producer that waits for the previous
    load's release instead of the slot's (parity off by one) is caught."""

    def bad(seed):
        sim = Sim(seed, 3)
        S = 3
        for s in range(S):
            sim.bar(f"Full{s}"), sim.bar(f"Empty{s}")

        def producer():
            for n in range(8):
                slot = n % S
                if n >= S:
                    yield Sim.wait(f"Empty{slot}", (n // S) & 1, n // S - 1)  # wrong parity
                sim.issue_load(n, True)

        sim.run({"producer": producer(), "tensor": sim.tensor("mma")})

    with pytest.raises(AssertionError, match="parity formula"):
        bad(0)


def test_model_catches_an_early_reload():
    """A producer that skips the wait for a slot's release reloads it before
    the MMA read it, and the model reports the overwrite."""
    sim = Sim(0, 3)
    for s in range(3):
        sim.bar(f"Full{s}"), sim.bar(f"Empty{s}")

    def producer():
        for n in range(6):
            sim.issue_load(n, True)
            yield ("step",)

    with pytest.raises(AssertionError, match="overwrites slot"):
        sim.run({"producer": producer(), "tensor": sim.tensor("mma")})


# ------------------------------------------------ prefill_tile_kernel (csrc/prefill_tile.cu)
# Roles: warp 0 publishes items and loads Q (2 stages) and K (2 stages); warp
# 3 loads V (2 stages); warp 1 issues S = Q K^T into three TMEM S/P buffers;
# warp 2 fixes V rows past the keys and issues O += P V (a second issuing
# thread, so S and PV are two independent in-order streams); two softmax
# warpgroups each take 64 keys of every row and meet at a max exchange per
# tile (and once more for the row sums); the epilogue warpgroup reads the
# softmax's row statistics and O. Arrival counts in the model: PFull 8 -> 2
# (one per half), the exchange 64 -> 2, the item ring's 15 readers -> 6,
# StatsFull / StatsFree 128 -> 1, OFree 4 -> 1.
def run_prefill_tile(seed, item_tiles, rescale_p=0.3, page_p=0.9):
    sim = Sim(seed, 2)
    sim.tqs = {"s": [], "pv": []}
    B = sim.bar
    for s in range(2):
        for n in ("QFull", "QFree", "KFull", "KEmpty", "VFull", "VEmpty", "ItemFull"):
            B(f"{n}{s}")
        B(f"ItemEmpty{s}", 6)
    for b in range(3):
        B(f"SFull{b}"), B(f"PVDone{b}"), B(f"PFull{b}", 2)
    for n in ("ODone", "OFree", "StatsFull", "StatsFree", "Drain", "PVDrain"):
        B(n)
    B("Xchg", 2)
    rng = random.Random(seed + 7)
    first, g = {}, 0
    for i, n in enumerate(item_tiles):
        first[i] = g
        g += n
    total = g
    keyed = [i for i, n in enumerate(item_tiles) if n > 0]
    item_of = {}
    for i in keyed:
        for t in range(first[i], first[i] + item_tiles[i]):
            item_of[t] = i
    ok = [rng.random() < page_p for _ in range(total)]
    rescale = [rng.random() < rescale_p for _ in range(total)]
    END = -1
    items = list(item_tiles) + [END]
    ring = [None, None]
    st = {
        "q": [None, None], "q_landed": [False, False], "k": [None, None], "k_landed": [False, False],
        "v": [None, None], "v_landed": [False, False], "s_done": set(), "pv_done": -1,
        "buf": [None, None, None], "s_read": {}, "p_written": {}, "o_item": None, "o_read": set(),
        "stats": None, "stats_read": set(),
    }

    def load(kind, stage, what, barname, real=True):
        st[kind][stage], st[kind + "_landed"][stage] = what, False

        def land():
            assert st[kind][stage] == what
            st[kind + "_landed"][stage] = True
            sim.arrive(barname)

        if real:
            sim.loads.append(land)
        else:
            land()

    def take(i):
        yield Sim.wait(f"ItemFull{i & 1}", (i >> 1) & 1, i >> 1)
        idx, n = ring[i & 1]
        assert idx == i
        sim.arrive(f"ItemEmpty{i & 1}")
        return n

    def producer():  # warp 0: items, Q and K
        gt = ix = k_issued = 0
        for i, n in enumerate(items):
            if i >= 2:
                yield Sim.wait(f"ItemEmpty{i & 1}", ((i >> 1) + 1) & 1, (i >> 1) - 1)
            ring[i & 1] = (i, n)
            sim.arrive(f"ItemFull{i & 1}")
            if n == END:
                break
            if n == 0:
                continue
            qs = ix & 1
            if ix >= 2:
                yield Sim.wait(f"QFree{qs}", ((ix >> 1) + 1) & 1, (ix >> 1) - 1)
                prev = keyed[ix - 2]
                assert first[prev] + item_tiles[prev] - 1 in st["s_done"], "Q reloaded before its last S"
            load("q", qs, i, f"QFull{qs}")
            ix += 1
            for j in range(n):
                g, s = gt + j, (gt + j) & 1
                if g >= 2:
                    yield Sim.wait(f"KEmpty{s}", ((g >> 1) + 1) & 1, (g >> 1) - 1)
                    assert g - 2 in st["s_done"], f"K of tile {g} overwrites K of tile {g - 2} before its S"
                load("k", s, g, f"KFull{s}", ok[g])
                k_issued = g + 1
                yield ("step",)
            gt += n
        for s in range(2):  # drain
            if k_issued > s:
                last = k_issued - 1 - ((k_issued - 1 - s) & 1)
                yield Sim.wait(f"KFull{s}", ((k_issued - 1 - s) >> 1) & 1, last >> 1)
            if ix > s:
                last = ix - 1 - ((ix - 1 - s) & 1)
                yield Sim.wait(f"QFull{s}", ((ix - 1 - s) >> 1) & 1, last >> 1)

    def v_producer():  # warp 3
        gt = v_issued = 0
        for i in range(len(items)):
            n = yield from take(i)
            if n == END:
                break
            for j in range(n):
                g, s = gt + j, (gt + j) & 1
                if g >= 2:
                    yield Sim.wait(f"VEmpty{s}", ((g >> 1) + 1) & 1, (g >> 1) - 1)
                    assert st["pv_done"] >= g - 2, f"V of tile {g} overwrites V of tile {g - 2} before its PV"
                load("v", s, g, f"VFull{s}", ok[g])
                v_issued = g + 1
                yield ("step",)
            gt += n
        for s in range(2):
            if v_issued > s:
                last = v_issued - 1 - ((v_issued - 1 - s) & 1)
                yield Sim.wait(f"VFull{s}", ((v_issued - 1 - s) >> 1) & 1, last >> 1)

    def s_issuer():  # warp 1
        gt = ix = 0
        for i in range(len(items)):
            n = yield from take(i)
            if n == END:
                break
            if n == 0:
                continue
            qs = ix & 1
            for j in range(n):
                t, ks, buf = gt + j, (gt + j) & 1, (gt + j) % 3
                yield Sim.wait(f"KFull{ks}", (t >> 1) & 1, t >> 1)
                if j == 0:
                    yield Sim.wait(f"QFull{qs}", (ix >> 1) & 1, ix >> 1)
                if t >= 3:
                    yield Sim.wait(f"PVDone{buf}", ((t - 3) // 3) & 1, (t - 3) // 3)

                def exec_s(t=t, ks=ks, buf=buf, qs=qs, i=i):
                    assert st["q"][qs] == i and st["q_landed"][qs], f"S of tile {t} without item {i}'s Q"
                    assert st["k"][ks] == t and st["k_landed"][ks], f"S of tile {t} reads K of tile {st['k'][ks]}"
                    assert t < 3 or st["pv_done"] >= t - 3, f"S of tile {t} overwrites P of tile {t - 3} before its PV"
                    st["s_done"].add(t)
                    st["buf"][buf] = t
                    st["s_read"][t], st["p_written"][t] = set(), set()

                sim.tqs["s"] += [exec_s, lambda b=buf: sim.arrive(f"SFull{b}"), lambda k=ks: sim.arrive(f"KEmpty{k}")]
                if j == n - 1:
                    sim.tqs["s"].append(lambda q=qs: sim.arrive(f"QFree{q}"))
            ix += 1
            gt += n
        sim.tqs["s"].append(lambda: sim.arrive("Drain"))
        yield Sim.wait("Drain", 0, 0)

    def pv_issuer():  # warp 2: V fixer + PV
        gt = ix = 0
        for i in range(len(items)):
            n = yield from take(i)
            if n == END:
                break
            if n == 0:
                continue
            for j in range(n):
                g, s, buf = gt + j, (gt + j) & 1, (gt + j) % 3
                yield Sim.wait(f"VFull{s}", (g >> 1) & 1, g >> 1)
                assert st["v"][s] == g and st["v_landed"][s] and st["pv_done"] < g, f"V fixer on tile {g}"
                if j == 0 and ix > 0:
                    yield Sim.wait("OFree", (ix - 1) & 1, ix - 1)
                yield Sim.wait(f"PFull{buf}", (g // 3) & 1, g // 3)

                def exec_pv(g=g, s=s, buf=buf, j=j, i=i):
                    assert st["v"][s] == g and st["v_landed"][s], f"PV of tile {g} reads V of tile {st['v'][s]}"
                    assert st["buf"][buf] == g and st["p_written"][g] == {0, 1}, f"PV of tile {g} without its P"
                    assert st["pv_done"] == g - 1
                    if j == 0:
                        prev = [k for k in keyed if k < i]
                        assert not prev or prev[-1] in st["o_read"], f"item {i}'s first PV before O of {prev[-1]} was read"
                        st["o_item"] = i
                    st["pv_done"] = g

                sim.tqs["pv"] += [exec_pv, lambda b=buf: sim.arrive(f"PVDone{b}"), lambda s=s: sim.arrive(f"VEmpty{s}")]
                if j == n - 1:
                    sim.tqs["pv"].append(lambda: sim.arrive("ODone"))
            ix += 1
            gt += n
        sim.tqs["pv"].append(lambda: sim.arrive("PVDrain"))
        yield Sim.wait("PVDrain", 0, 0)

    def softmax(h):  # warps 4..11, half h of every row's keys
        t = ix = xc = 0

        def exchange():
            nonlocal xc
            sim.arrive("Xchg")
            yield Sim.wait("Xchg", xc & 1, xc)
            xc += 1

        for i in range(len(items)):
            n = yield from take(i)
            if n == END:
                break
            if n == 0:
                continue
            for j in range(n):
                buf = t % 3
                yield Sim.wait(f"SFull{buf}", (t // 3) & 1, t // 3)
                assert st["buf"][buf] == t and not st["p_written"][t], f"softmax reads S of tile {t}"
                st["s_read"][t].add(h)
                yield from exchange()
                assert st["s_read"][t] == {0, 1}, "P stored over S columns the other half has not read"
                st["p_written"][t].add(h)
                if j >= 1 and rescale[t]:
                    pb = (t - 1) % 3
                    yield Sim.wait(f"PVDone{pb}", ((t - 1) // 3) & 1, (t - 1) // 3)
                    assert st["pv_done"] == t - 1, f"O rescaled at tile {t} with PV {st['pv_done']} done"
                sim.arrive(f"PFull{buf}")
                t += 1
            yield from exchange()
            if h == 0:
                if ix > 0:
                    yield Sim.wait("StatsFree", (ix - 1) & 1, ix - 1)
                    assert keyed[ix - 1] in st["stats_read"], "row statistics overwritten before the epilogue read them"
                st["stats"] = i
                sim.arrive("StatsFull")
            ix += 1

    def epilogue():  # warps 12..15
        ix = 0
        for i in range(len(items)):
            n = yield from take(i)
            if n == END:
                break
            if n == 0:
                continue
            yield Sim.wait("StatsFull", ix & 1, ix)
            assert st["stats"] == i, f"epilogue of item {i} reads statistics of item {st['stats']}"
            st["stats_read"].add(i)
            sim.arrive("StatsFree")
            yield Sim.wait("ODone", ix & 1, ix)
            assert st["o_item"] == i and st["pv_done"] == first[i] + item_tiles[i] - 1, f"epilogue of item {i}"
            st["o_read"].add(i)
            sim.arrive("OFree")
            ix += 1

    sim.run({"producer": producer(), "v_producer": v_producer(), "s_issuer": s_issuer(), "pv_issuer": pv_issuer(),
             "softmax0": softmax(0), "softmax1": softmax(1), "epilogue": epilogue(),
             "tensor_s": sim.tensor("s"), "tensor_pv": sim.tensor("pv")})
    assert st["pv_done"] == total - 1 and st["o_read"] == set(keyed)


def test_prefill_tile_protocol():
    for seed in range(150):
        rng = random.Random(3000 + seed)
        item_tiles = [rng.choice([0, 1, 1, 2, 3, 4, 6]) for _ in range(rng.randint(1, 8))]
        run_prefill_tile(seed, item_tiles)


# ----------------------------------------------------- prefill_kernel (csrc/prefill.cu)
# Pairs of query tiles A and B (chains x = 0, 1) share every K/V tile of an
# item. Warp 0 publishes items and loads K (2 stages; an item's first K tile
# before its Q tiles) and each chain's Q buffer; warp 3 loads V (2 stages)
# and hands each stage's real-key count to the fixer in shared memory; warp 1
# issues S_A and S_B per K tile (each S_x single-buffered, so S_x of a tile
# waits for PV_x of its previous tile); warp 2 zeroes V rows past the keys
# and issues PV_A and PV_B; one softmax warpgroup per chain; the epilogue
# reads each chain's statistics and O. Counts in the model: PFull and OFree
# 4 -> 1, StatsFull / StatsFree 128 -> 1, the item ring's 15 readers -> 6.
def run_prefill_pair(seed, pairs, rescale_p=0.3, page_p=0.9):
    sim = Sim(seed, 2)
    sim.tqs = {"s": [], "pv": []}
    B = sim.bar
    for s in range(2):
        for n in ("QFull", "QFree", "KFull", "KEmpty", "VFull", "VEmpty", "SFull", "PFull", "PVDone", "ODone",
                  "OFree", "StatsFull", "StatsFree", "ItemFull"):
            B(f"{n}{s}")
        B(f"ItemEmpty{s}", 6)
    B("Drain"), B("PVDrain")
    rng = random.Random(seed + 11)
    END = None
    items = list(pairs) + [END]
    ring = [None, None]
    nt_of = [max(a, b) for a, b in pairs]
    total = sum(nt_of)
    ok = [rng.random() < page_p for _ in range(total)]
    # chain tile numbering: (item, j, x) -> t in chain x's order
    tnum, last_t, first_t, cnt = {}, {}, {}, [0, 0]
    for i, (na, nb) in enumerate(pairs):
        for x, n in ((0, na), (1, nb)):
            for j in range(n):
                tnum[(i, j, x)] = cnt[x]
                cnt[x] += 1
            if n:
                first_t[(i, x)], last_t[(i, x)] = tnum[(i, 0, x)], tnum[(i, n - 1, x)]
    rescale = [[rng.random() < rescale_p for _ in range(cnt[x])] for x in range(2)]
    st = {
        "q": [None, None], "q_landed": [False, False], "k": [None, None], "k_landed": [False, False],
        "v": [None, None], "v_landed": [False, False], "v_real": [None, None], "v_real_read": set(),
        "s_exec": set(), "pv_exec": set(), "sbuf": [None, None], "pv_done": [-1, -1], "o_item": [None, None],
        "o_read": [set(), set()], "stats": [None, None], "stats_read": [set(), set()],
    }
    g_first = []
    g = 0
    for i in range(len(pairs)):
        g_first.append(g)
        g += nt_of[i]

    def needs(i, j):  # chains that read KV tile j of item i
        return [x for x in range(2) if j < pairs[i][x]]

    def load(kind, stage, what, barname, real=True):
        st[kind][stage], st[kind + "_landed"][stage] = what, False

        def land():
            assert st[kind][stage] == what
            st[kind + "_landed"][stage] = True
            sim.arrive(barname)

        if real:
            sim.loads.append(land)
        else:
            land()

    def take(i):
        yield Sim.wait(f"ItemFull{i & 1}", (i >> 1) & 1, i >> 1)
        idx, it = ring[i & 1]
        assert idx == i
        sim.arrive(f"ItemEmpty{i & 1}")
        return it

    def producer():  # warp 0
        gt = k_issued = 0
        ixq = [0, 0]
        lastq = [None, None]
        for i, it in enumerate(items):
            if i >= 2:
                yield Sim.wait(f"ItemEmpty{i & 1}", ((i >> 1) + 1) & 1, (i >> 1) - 1)
            ring[i & 1] = (i, it)
            sim.arrive(f"ItemFull{i & 1}")
            if it is END:
                break
            nt = nt_of[i]
            if nt == 0:
                continue

            def load_k(j, i=i, gt=gt):
                nonlocal k_issued
                g, s = gt + j, (gt + j) & 1
                if g >= 2:
                    yield Sim.wait(f"KEmpty{s}", ((g >> 1) + 1) & 1, (g >> 1) - 1)
                    pi, pj = st["k"][s]
                    assert all((pi, pj, x) in st["s_exec"] for x in needs(pi, pj)), f"K of tile {g} over an unread K"
                load("k", s, (i, j), f"KFull{s}", ok[g])
                k_issued = g + 1

            yield from load_k(0)
            for x in range(2):
                if pairs[i][x] == 0:
                    continue
                if ixq[x] >= 1:
                    yield Sim.wait(f"QFree{x}", (ixq[x] - 1) & 1, ixq[x] - 1)
                    pi = lastq[x]
                    assert (pi, pairs[pi][x] - 1, x) in st["s_exec"], f"Q_{x} reloaded before its last S"
                load("q", x, i, f"QFull{x}")
                lastq[x] = i
                ixq[x] += 1
            for j in range(1, nt):
                yield from load_k(j)
                yield ("step",)
            gt += nt
        for s in range(2):
            if k_issued > s:
                last = k_issued - 1 - ((k_issued - 1 - s) & 1)
                yield Sim.wait(f"KFull{s}", ((k_issued - 1 - s) >> 1) & 1, last >> 1)
            if ixq[s] > 0:
                yield Sim.wait(f"QFull{s}", (ixq[s] - 1) & 1, ixq[s] - 1)

    def v_producer():  # warp 3
        gt = v_issued = 0
        for i in range(len(items)):
            it = yield from take(i)
            if it is END:
                break
            for j in range(nt_of[i]):
                g, s = gt + j, (gt + j) & 1
                if g >= 2:
                    yield Sim.wait(f"VEmpty{s}", ((g >> 1) + 1) & 1, (g >> 1) - 1)
                    pi, pj = st["v"][s]
                    assert all((pi, pj, x) in st["pv_exec"] for x in needs(pi, pj)), f"V of tile {g} over an unread V"
                    assert (pi, pj) in st["v_real_read"], "real-key count overwritten before the fixer read it"
                st["v_real"][s] = (i, j)
                load("v", s, (i, j), f"VFull{s}", ok[g])
                v_issued = g + 1
                yield ("step",)
            gt += nt_of[i]
        for s in range(2):
            if v_issued > s:
                last = v_issued - 1 - ((v_issued - 1 - s) & 1)
                yield Sim.wait(f"VFull{s}", ((v_issued - 1 - s) >> 1) & 1, last >> 1)

    def s_issuer():  # warp 1
        gt = 0
        tx, ixq = [0, 0], [0, 0]
        for i in range(len(items)):
            it = yield from take(i)
            if it is END:
                break
            for j in range(nt_of[i]):
                g, ks = gt + j, (gt + j) & 1
                yield Sim.wait(f"KFull{ks}", (g >> 1) & 1, g >> 1)
                for x in range(2):
                    if j >= pairs[i][x]:
                        continue
                    if j == 0:
                        yield Sim.wait(f"QFull{x}", ixq[x] & 1, ixq[x])
                    if tx[x] >= 1:
                        yield Sim.wait(f"PVDone{x}", (tx[x] - 1) & 1, tx[x] - 1)

                    def exec_s(i=i, j=j, x=x, ks=ks, t=tx[x]):
                        assert st["q"][x] == i and st["q_landed"][x], f"S_{x} of item {i} without its Q"
                        assert st["k"][ks] == (i, j) and st["k_landed"][ks], f"S_{x} reads K {st['k'][ks]}"
                        assert st["pv_done"][x] == t - 1, f"S_{x} of tile {t} overwrites P_{x} before its PV"
                        st["s_exec"].add((i, j, x))
                        st["sbuf"][x] = ("S", t)

                    sim.tqs["s"] += [exec_s, lambda x=x: sim.arrive(f"SFull{x}")]
                    if j == pairs[i][x] - 1:
                        sim.tqs["s"].append(lambda x=x: sim.arrive(f"QFree{x}"))
                        ixq[x] += 1
                    tx[x] += 1
                sim.tqs["s"].append(lambda ks=ks: sim.arrive(f"KEmpty{ks}"))
            gt += nt_of[i]
        sim.tqs["s"].append(lambda: sim.arrive("Drain"))
        yield Sim.wait("Drain", 0, 0)

    def pv_issuer():  # warp 2: V fixer + PV
        gt = 0
        tx, ixo = [0, 0], [0, 0]
        prev_item = [None, None]
        for i in range(len(items)):
            it = yield from take(i)
            if it is END:
                break
            for j in range(nt_of[i]):
                g, s = gt + j, (gt + j) & 1
                yield Sim.wait(f"VFull{s}", (g >> 1) & 1, g >> 1)
                assert st["v_real"][s] == (i, j), "fixer reads another tile's real-key count"
                st["v_real_read"].add((i, j))
                assert st["v"][s] == (i, j) and st["v_landed"][s], f"fixer zeroes V {st['v'][s]}"
                assert not any((i, j, x) in st["pv_exec"] for x in range(2)), "V rows zeroed after a PV read them"
                for x in range(2):
                    if j >= pairs[i][x]:
                        continue
                    if j == 0 and ixo[x] > 0:
                        yield Sim.wait(f"OFree{x}", (ixo[x] - 1) & 1, ixo[x] - 1)
                    yield Sim.wait(f"PFull{x}", tx[x] & 1, tx[x])

                    def exec_pv(i=i, j=j, x=x, s=s, t=tx[x], prev=prev_item[x]):
                        assert st["sbuf"][x] == ("P", t), f"PV_{x} of tile {t} reads {st['sbuf'][x]}"
                        assert st["v"][s] == (i, j) and st["v_landed"][s], f"PV_{x} reads V {st['v'][s]}"
                        assert st["pv_done"][x] == t - 1
                        if j == 0:
                            assert prev is None or prev in st["o_read"][x], f"O_{x} restarted before item {prev} was read"
                            st["o_item"][x] = i
                        st["pv_exec"].add((i, j, x))
                        st["pv_done"][x] = t

                    sim.tqs["pv"] += [exec_pv, lambda x=x: sim.arrive(f"PVDone{x}")]
                    if j == pairs[i][x] - 1:
                        sim.tqs["pv"].append(lambda x=x: sim.arrive(f"ODone{x}"))
                        ixo[x] += 1
                        prev_item[x] = i
                    tx[x] += 1
                sim.tqs["pv"].append(lambda s=s: sim.arrive(f"VEmpty{s}"))
            gt += nt_of[i]
        sim.tqs["pv"].append(lambda: sim.arrive("PVDrain"))
        yield Sim.wait("PVDrain", 0, 0)

    def softmax(x):  # warps 4..7 (A) or 8..11 (B)
        t = ix = 0
        for i in range(len(items)):
            it = yield from take(i)
            if it is END:
                break
            n = pairs[i][x]
            if n == 0:
                continue
            for j in range(n):
                yield Sim.wait(f"SFull{x}", t & 1, t)
                assert st["sbuf"][x] == ("S", t), f"softmax {x} reads {st['sbuf'][x]} for tile {t}"
                if j >= 1 and rescale[x][t]:
                    yield Sim.wait(f"PVDone{x}", (t - 1) & 1, t - 1)
                    assert st["pv_done"][x] == t - 1, f"O_{x} rescaled at tile {t} with PV {st['pv_done'][x]}"
                st["sbuf"][x] = ("P", t)
                sim.arrive(f"PFull{x}")
                t += 1
            if ix > 0:
                yield Sim.wait(f"StatsFree{x}", (ix - 1) & 1, ix - 1)
                assert st["stats"][x] in st["stats_read"][x], f"statistics {x} overwritten before they were read"
            st["stats"][x] = i
            sim.arrive(f"StatsFull{x}")
            ix += 1

    def epilogue():  # warps 12..15
        ixo = [0, 0]
        for i in range(len(items)):
            it = yield from take(i)
            if it is END:
                break
            for x in range(2):
                if pairs[i][x] == 0:
                    continue
                yield Sim.wait(f"StatsFull{x}", ixo[x] & 1, ixo[x])
                assert st["stats"][x] == i
                st["stats_read"][x].add(i)
                sim.arrive(f"StatsFree{x}")
                yield Sim.wait(f"ODone{x}", ixo[x] & 1, ixo[x])
                assert st["o_item"][x] == i and st["pv_done"][x] == last_t[(i, x)], f"epilogue {x} of item {i}"
                st["o_read"][x].add(i)
                sim.arrive(f"OFree{x}")
                ixo[x] += 1

    sim.run({"producer": producer(), "v_producer": v_producer(), "s_issuer": s_issuer(), "pv_issuer": pv_issuer(),
             "softmax0": softmax(0), "softmax1": softmax(1), "epilogue": epilogue(),
             "tensor_s": sim.tensor("s"), "tensor_pv": sim.tensor("pv")})
    for x in range(2):
        assert st["pv_done"][x] == cnt[x] - 1
        assert st["o_read"][x] == {i for i, p in enumerate(pairs) if p[x]}


def test_prefill_pair_protocol():
    for seed in range(150):
        rng = random.Random(4000 + seed)
        pairs = []
        for _ in range(rng.randint(1, 7)):
            a = rng.choice([0, 1, 2, 3, 5])
            b = rng.choice([0, a, a, a + 1, max(0, a - 1)])
            pairs.append((a, b))
        run_prefill_pair(seed, pairs)
