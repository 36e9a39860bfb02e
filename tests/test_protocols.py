"""CPU models of the synchronisation inside the attention kernels, run under
many random schedules: the prefill kernel's split instance
(lean-infer_b200/csrc/la_prefill.cu, prefill_kernel<true>: items of one query
tile, both softmax warpgroups on the tile's two key halves, S double buffered
in TMEM) and pair instance (prefill_kernel<false>: items of two query tiles
sharing the K/V tiles), the decode kernel's stage ring and sub-chunk merge
(la_decode.cu), and the KV-head-sharded decode's all-gather over peer memory
(la_p2p.cu).

Every actor follows the kernel's order of waits, arrivals and commits: the TMA
producer, the MMA issuer, softmax warpgroups 0 and 1, the epilogue, plus the
TMA engine (copies land in any order) and the tensor core (MMAs execute and
commits arrive in issue order). Barriers behave as mbarriers do: a parity wait
passes while the number of completed phases has the other parity, so a barrier
two phases ahead of its waiter passes the wait as well. Shared memory, the K/V
ring and TMEM carry version tags, and every read checks that it sees the
version the kernel means, so a wait that passes on the wrong phase, or a write
that lands before the last read of what it overwrites, fails the run; so does a
deadlock. Planted mistakes must be caught: for the split instance the three
bugs met while building it (the row-max exchange on one barrier and one slot
per half, one P-ready barrier counting both halves, the epilogue waiting on
the PV barrier's parity); for the pair instance the orderings it relies on
(S_i(j+1) behind PV_i(j), the O-empty wait before an item's first PV, Q
released after an item's last S); for decode, a merge slot rewritten before
it was read, in both directions.

The row-max decision to rescale O is data dependent in the kernel; the model
draws it at random per warpgroup and step, which covers every case."""
import random

import pytest


class Bar:
    def __init__(self, name, count):
        self.name, self.count = name, count
        self.pending, self.tx, self.phases = count, 0, 0

    def _check(self):
        if self.pending == 0 and self.tx == 0:
            self.phases += 1
            self.pending = self.count

    def arrive(self, expect_tx=0):
        assert self.pending > 0, f"{self.name}: arrival beyond the expected count"
        self.tx += expect_tx
        self.pending -= 1
        self._check()

    def complete_tx(self, n):
        self.tx -= n
        self._check()

    def ready(self, parity):
        return (self.phases & 1) != parity


class Hazard(AssertionError):
    pass


def run_schedule(m, actors, max_ticks=200000):
    """Run the actors, the TMA engine and the tensor core of model m under a
    random schedule drawn from m.rng; raise Hazard on a bad read, a deadlock
    or a schedule that does not end."""
    blocked = [None] * len(actors)  # (bar, parity) an actor waits on
    done = [False] * len(actors)

    def advance(i):
        try:
            cmd = next(actors[i])
        except StopIteration:
            done[i] = True
            return
        blocked[i] = (cmd[1], cmd[2]) if cmd[0] == "wait" else None

    for i in range(len(actors)):
        advance(i)
    # Each run gives every actor and engine its own speed, from 1/64 to 64,
    # so that some schedules let one side run far ahead of another.
    speed = {key: 2.0 ** m.rng.uniform(-6, 6) for key in [("actor", i) for i in range(len(actors))] +
             [("tma", None), ("tc", None)]}
    for _ in range(max_ticks):
        choices = [("actor", i) for i in range(len(actors))
                   if not done[i] and (blocked[i] is None or blocked[i][0].ready(blocked[i][1]))]
        if m.tma:
            choices.append(("tma", None))
        if m.tc:
            choices.append(("tc", None))
        if not choices:
            if all(done):
                return
            waits = [f"{blocked[i][0].name}/{blocked[i][1]}" for i in range(len(actors)) if not done[i]]
            raise Hazard(f"deadlock: waiting on {waits}")
        kind, i = m.rng.choices(choices, weights=[speed[c] for c in choices])[0]
        if kind == "actor":
            blocked[i] = None
            advance(i)
        elif kind == "tma":
            region, tag, bar, nbytes = m.tma.pop(m.rng.randrange(len(m.tma)))
            m.write(region, tag)
            bar.complete_tx(nbytes)
        else:
            op, arg = m.tc.pop(0)
            if op == "mma":
                arg()
            else:
                arg.arrive()
    raise Hazard("schedule did not finish")


class Model:
    STAGES = 4

    def __init__(self, items, rng, plant=None):
        self.items, self.rng, self.plant = items, rng, plant
        B = Bar
        self.q_full, self.q_empty = B("q_full", 1), B("q_empty", 1)
        self.kv_full = [B(f"kv_full{i}", 1) for i in range(self.STAGES)]
        self.kv_empty = [B(f"kv_empty{i}", 1) for i in range(self.STAGES)]
        self.s_full = [B(f"s_full{i}", 1) for i in range(2)]
        self.s_free = B("s_free", 1)
        self.o_empty, self.o_full = B("o_empty", 1), B("o_full", 1)
        self.st_full, self.st_empty = B("st_full", 2), B("st_empty", 1)
        self.x_full = [B(f"x_full{i}", 1) for i in range(4)]
        self.ph_full = [B(f"ph_full{i}", 1) for i in range(4)]
        self.p_full = B("p_full", 2)  # planted: one P-ready barrier for both halves
        self.mem = {}          # region -> version tag
        self.tma = []          # copies in flight: (region, tag, bar, bytes)
        self.tc = []           # tensor-core queue: ("mma", fn) | ("commit", bar)
        self.starts = []       # global S / PV index of each item's first tile
        t = 0
        for n in items:
            self.starts.append(t)
            t += n

    # -- helpers
    def read(self, region, want):
        got = self.mem.get(region)
        if got != want:
            raise Hazard(f"read {region}: found {got}, expected {want}")

    def write(self, region, tag):
        self.mem[region] = tag

    # -- actors (generators yielding ("wait", bar, parity) or ("step",))
    def producer(self):
        nld = kq = 0
        for k, n in enumerate(self.items):
            yield ("wait", self.q_empty, (kq & 1) ^ 1)
            self.q_full.arrive(expect_tx=1)
            self.tma.append(("Q", ("Q", k), self.q_full, 1))
            kq += 1
            yield ("step",)
            for j in range(n):
                for kind in ("K", "V"):
                    st = nld % self.STAGES
                    yield ("wait", self.kv_empty[st], ((nld // self.STAGES) & 1) ^ 1)
                    self.kv_full[st].arrive(expect_tx=1)
                    self.tma.append((f"R{st}", (kind, k, j), self.kv_full[st], 1))
                    nld += 1
                    yield ("step",)

    def mma(self):
        nld = kq = sc = cp = items_done = 0
        for k, n in enumerate(self.items):
            yield ("wait", self.q_full, kq & 1)
            kq += 1
            base = nld
            nld += 2 * n
            b0 = sc & 1

            def issue_s(kpos, j, last):
                nonlocal sc
                b, t = sc & 1, sc

                def run(b=b, t=t, kpos=kpos, j=j, k=k):
                    self.read("Q", ("Q", k))
                    self.read(f"R{kpos % self.STAGES}", ("K", k, j))
                    for r in range(4):
                        self.write(f"S{b}.{r}", ("S", t))
                self.tc.append(("mma", run))
                self.tc.append(("commit", self.s_full[b]))
                self.tc.append(("commit", self.kv_empty[kpos % self.STAGES]))
                if last:
                    self.tc.append(("commit", self.q_empty))
                sc += 1

            for jj in range(min(n, 2)):
                kpos = base + 2 * jj
                yield ("wait", self.kv_full[kpos % self.STAGES], (kpos // self.STAGES) & 1)
                issue_s(kpos, jj, jj == n - 1)
                yield ("step",)
            for j in range(n):
                vi = base + 2 * j + 1
                yield ("wait", self.kv_full[vi % self.STAGES], (vi // self.STAGES) & 1)
                if self.plant == "one_p_barrier":
                    yield ("wait", self.p_full, cp & 1)
                else:
                    yield ("wait", self.ph_full[cp & 1], (cp >> 1) & 1)
                    yield ("wait", self.ph_full[2 + (cp & 1)], (cp >> 1) & 1)
                if j == 0:
                    if items_done > 0:
                        yield ("wait", self.o_empty, (items_done - 1) & 1)
                    items_done += 1
                t, buf = cp, (b0 + j) & 1

                def pv(t=t, buf=buf, vi=vi, j=j, k=k):
                    self.read(f"S{buf}.0", ("P", t, 0))
                    self.read(f"S{buf}.1", ("P", t, 1))
                    self.read(f"R{vi % self.STAGES}", ("V", k, j))
                    for h in range(2):
                        if j > 0:
                            self.read(f"O{h}", ("O", k, j))
                        self.write(f"O{h}", ("O", k, j + 1))
                self.tc.append(("mma", pv))
                self.tc.append(("commit", self.s_free))
                self.tc.append(("commit", self.kv_empty[vi % self.STAGES]))
                if j == n - 1:
                    self.tc.append(("commit", self.o_full))
                cp += 1
                yield ("step",)
                if j + 2 < n:
                    kpos = base + 2 * (j + 2)
                    yield ("wait", self.kv_full[kpos % self.STAGES], (kpos // self.STAGES) & 1)
                    issue_s(kpos, j + 2, j + 3 == n)
                    yield ("step",)

    def softmax(self, h):
        t = nst = 0
        for k, n in enumerate(self.items):
            for j in range(n):
                buf = t & 1
                yield ("wait", self.s_full[buf], (t >> 1) & 1)
                self.read(f"S{buf}.{2 * h}", ("S", t))       # this half's 64 columns
                self.read(f"S{buf}.{2 * h + 1}", ("S", t))
                yield ("step",)
                sb = t & 1
                if self.plant == "one_exchange_barrier":  # one slot and one barrier per half
                    xw, xr, xbar, xpar = f"xmax.{h}", f"xmax.{h ^ 1}", self.x_full[h ^ 1], t & 1
                    mine = self.x_full[h]
                else:
                    xw, xr, xbar, xpar = f"xmax{sb}.{h}", f"xmax{sb}.{h ^ 1}", self.x_full[sb * 2 + (h ^ 1)], (t >> 1) & 1
                    mine = self.x_full[sb * 2 + h]
                self.write(xw, t)
                mine.arrive()
                yield ("step",)
                yield ("wait", xbar, xpar)
                self.read(xr, t)
                yield ("step",)
                self.write(f"S{buf}.{h}", ("P", t, h))       # P of keys 64h..64h+63: columns 32h..32h+31
                yield ("step",)
                if j >= 1 and self.rng.random() < 0.5:      # this half of O is rescaled
                    yield ("wait", self.s_free, (t - 1) & 1)
                    self.read(f"O{h}", ("O", k, j))
                    yield ("step",)
                (self.p_full if self.plant == "one_p_barrier" else self.ph_full[h * 2 + sb]).arrive()
                t += 1
                yield ("step",)
            yield ("wait", self.st_empty, (nst & 1) ^ 1)
            self.write(f"stats{h}", k)
            self.st_full.arrive()
            nst += 1
            yield ("step",)

    def epilogue(self):
        cp = 0
        for k, n in enumerate(self.items):
            cp += n
            yield ("wait", self.st_full, k & 1)
            self.read("stats0", k)
            self.read("stats1", k)
            self.st_empty.arrive()
            yield ("step",)
            if self.plant == "epilogue_on_pv_parity":
                yield ("wait", self.s_free, (cp - 1) & 1)
            else:
                yield ("wait", self.o_full, k & 1)
            self.read("O0", ("O", k, n))
            self.read("O1", ("O", k, n))
            self.o_empty.arrive()
            yield ("step",)

    def run(self):
        run_schedule(self, [self.producer(), self.mma(), self.softmax(0), self.softmax(1), self.epilogue()])


class PairModel(Model):
    """The pair instance (prefill_kernel<false>): items of two query tiles that
    share every K/V tile; S_i in its own TMEM columns with P_i written over
    them; the MMA issuer interleaves PV_0(j), S_0(j+1), PV_1(j), S_1(j+1), so
    S_i(j+1) overwrites P_i(j) only because it is issued behind PV_i(j); the
    epilogue names an item's last PV_i by the PV barrier's parity. Items are
    (n0, n1): K/V tiles of tile 0 and of tile 1 (0: no second tile; tile 1,
    the later queries, may need one tile more)."""

    def __init__(self, items, rng, plant=None):
        super().__init__([max(a, b) for a, b in items], rng, plant)
        self.pairs = items
        B = Bar
        self.s_full = [B(f"s_full{i}", 1) for i in range(2)]
        self.s_free = [B(f"s_free{i}", 1) for i in range(2)]
        self.p_full = [B(f"p_full{i}", 1) for i in range(2)]
        self.o_empty = [B(f"o_empty{i}", 1) for i in range(2)]
        self.st_full = [B(f"st_full{i}", 1) for i in range(2)]
        self.st_empty = [B(f"st_empty{i}", 1) for i in range(2)]

    def producer(self):
        nld = kq = 0
        for k, (n0, n1) in enumerate(self.pairs):
            yield ("wait", self.q_empty, (kq & 1) ^ 1)
            tiles = 2 if n1 else 1
            self.q_full.arrive(expect_tx=tiles)
            for i in range(tiles):
                self.tma.append((f"Q{i}", ("Q", k, i), self.q_full, 1))
            kq += 1
            yield ("step",)
            for j in range(max(n0, n1)):
                for kind in ("K", "V"):
                    st = nld % self.STAGES
                    yield ("wait", self.kv_empty[st], ((nld // self.STAGES) & 1) ^ 1)
                    self.kv_full[st].arrive(expect_tx=1)
                    self.tma.append((f"R{st}", (kind, k, j), self.kv_full[st], 1))
                    nld += 1
                    yield ("step",)

    def mma(self):
        nld = kq = 0
        sc, cp, items_i = [0, 0], [0, 0], [0, 0]
        for k, (n0, n1) in enumerate(self.pairs):
            n = max(n0, n1)
            yield ("wait", self.q_full, kq & 1)
            base = nld
            nld += 2 * n

            def issue_s(i, kpos, j):
                t = sc[i]

                def run(i=i, t=t, kpos=kpos, j=j, k=k):
                    self.read(f"Q{i}", ("Q", k, i))
                    self.read(f"R{kpos % self.STAGES}", ("K", k, j))
                    self.write(f"S{i}", ("S", i, t))
                self.tc.append(("mma", run))
                self.tc.append(("commit", self.s_full[i]))
                sc[i] += 1

            def issue_pv(i, j, vi):
                yield ("wait", self.p_full[i], cp[i] & 1)
                if j == 0:
                    if items_i[i] > 0 and self.plant != "no_o_empty_wait":
                        yield ("wait", self.o_empty[i], (items_i[i] - 1) & 1)
                    items_i[i] += 1
                t = cp[i]

                def pv(i=i, t=t, vi=vi, j=j, k=k):
                    self.read(f"S{i}", ("P", i, t))
                    self.read(f"R{vi % self.STAGES}", ("V", k, j))
                    if j > 0:
                        self.read(f"O{i}", ("O", k, j))
                    self.write(f"O{i}", ("O", k, j + 1))
                self.tc.append(("mma", pv))
                self.tc.append(("commit", self.s_free[i]))
                cp[i] += 1

            yield ("wait", self.kv_full[base % self.STAGES], (base // self.STAGES) & 1)
            issue_s(0, base, 0)
            if n1 > 0:
                issue_s(1, base, 0)
            self.tc.append(("commit", self.kv_empty[base % self.STAGES]))
            if n == 1 or self.plant == "q_empty_early":
                self.tc.append(("commit", self.q_empty))
            yield ("step",)
            for j in range(n):
                vi, ki = base + 2 * j + 1, base + 2 * j + 2
                a0, a1, nx0, nx1 = j < n0, j < n1, j + 1 < n0, j + 1 < n1
                yield ("wait", self.kv_full[vi % self.STAGES], (vi // self.STAGES) & 1)
                if nx0 or nx1:
                    yield ("wait", self.kv_full[ki % self.STAGES], (ki // self.STAGES) & 1)
                if self.plant == "s_before_pv":  # S_0(j+1) ahead of PV_0(j): P_0(j) overwritten
                    if nx0:
                        issue_s(0, ki, j + 1)
                    if a0:
                        yield from issue_pv(0, j, vi)
                else:
                    if a0:
                        yield from issue_pv(0, j, vi)
                    if nx0:
                        issue_s(0, ki, j + 1)
                yield ("step",)
                if a1:
                    yield from issue_pv(1, j, vi)
                self.tc.append(("commit", self.kv_empty[vi % self.STAGES]))
                if nx1:
                    issue_s(1, ki, j + 1)
                if j + 1 < n:
                    self.tc.append(("commit", self.kv_empty[ki % self.STAGES]))
                    if j + 2 == n and self.plant != "q_empty_early":
                        self.tc.append(("commit", self.q_empty))
                yield ("step",)
            kq += 1

    def softmax(self, i):
        t = nst = 0
        for k, (n0, n1) in enumerate(self.pairs):
            ni = n1 if i else n0
            for j in range(ni):
                yield ("wait", self.s_full[i], t & 1)
                self.read(f"S{i}", ("S", i, t))
                yield ("step",)
                self.write(f"S{i}", ("P", i, t))
                yield ("step",)
                if j >= 1 and self.rng.random() < 0.5:  # O_i rescaled in place: PV_i(j-1) is in
                    self.read(f"O{i}", ("O", k, j))
                    yield ("step",)
                self.p_full[i].arrive()
                t += 1
                yield ("step",)
            if ni:
                yield ("wait", self.st_empty[i], (nst & 1) ^ 1)
                self.write(f"stats{i}", k)
                self.st_full[i].arrive()
                nst += 1
                yield ("step",)

    def epilogue(self):
        cp, items_i = [0, 0], [0, 0]
        for k, (n0, n1) in enumerate(self.pairs):
            for i, ni in enumerate((n0, n1)):
                if ni == 0:
                    continue
                cp[i] += ni
                yield ("wait", self.st_full[i], items_i[i] & 1)
                self.read(f"stats{i}", k)
                self.st_empty[i].arrive()
                yield ("step",)
                yield ("wait", self.s_free[i], (cp[i] - 1) & 1)
                self.read(f"O{i}", ("O", k, ni))
                self.o_empty[i].arrive()
                items_i[i] += 1
                yield ("step",)


PAIR_SETS = [[(1, 1)], [(3, 3)], [(2, 0)], [(1, 2), (3, 4)], [(4, 4), (1, 0), (2, 3), (1, 1)],
             [(5, 5), (2, 2), (1, 2), (3, 0), (2, 2)]]


@pytest.mark.parametrize("items", PAIR_SETS)
def test_pair_instance_protocol(items):
    for seed in range(150):
        PairModel(items, random.Random(seed * 104729 + len(items))).run()


@pytest.mark.parametrize("plant", ["s_before_pv", "no_o_empty_wait", "q_empty_early"])
def test_pair_planted_mistakes_are_caught(plant):
    caught = 0
    for seed in range(300):
        try:
            PairModel([(4, 4), (1, 2), (3, 3), (2, 0)], random.Random(seed), plant=plant).run()
        except Hazard:
            caught += 1
    assert caught > 0, f"the planted mistake {plant} went unnoticed in 300 schedules"


class DecodeModel:
    """The decode kernel's stage ring and sub-chunk merge
    (lean-infer_b200/csrc/la_decode.cu, paged_decode_kernel): two producer
    warps take the even and the odd units; for each of its units a producer
    waits the stage's empty barrier (one arrival per consumer warp), writes
    the stage descriptor into shared memory and starts its copies; consumer
    warps wait the full barrier, read descriptor and tiles, release the stage;
    at each segment end every sub-chunk warp leaves its softmax state in a
    merge slot (after the previous merge was read: mg_empty, one arrival per
    kv head) and the merging warp of each kv head, j = (segment end) % nsub,
    reads the slots in sub-chunk order once all warps have written (mg_full,
    one arrival per warp)."""

    STAGES = 3
    PRODUCERS = 2

    def __init__(self, units, seg_ends, hkv, warps, rng, plant=None):
        self.units, self.ends, self.hkv, self.warps = units, seg_ends, hkv, warps
        self.rng, self.plant = rng, plant
        self.full = [Bar(f"full{i}", 1) for i in range(self.STAGES)]
        self.empty = [Bar(f"empty{i}", warps) for i in range(self.STAGES)]
        self.mg_full, self.mg_empty = Bar("mg_full", warps), Bar("mg_empty", hkv)
        self.mem, self.tma, self.tc = {}, [], []

    read = Model.read
    write = Model.write

    def producer(self, pid=0, nprod=1):
        for k in range(pid, self.units, nprod):
            s = k % self.STAGES
            yield ("wait", self.empty[s], ((k // self.STAGES) & 1) ^ 1)
            self.write(f"D{s}", k)
            self.full[s].arrive(expect_tx=1)
            self.tma.append((f"R{s}", k, self.full[s], 1))
            yield ("step",)

    def consumer(self, w):
        j, h = w // self.hkv, w % self.hkv
        nsub = self.warps // self.hkv
        seg = 0
        for k in range(self.units):
            s = k % self.STAGES
            yield ("wait", self.full[s], (k // self.STAGES) & 1)
            self.read(f"D{s}", k)
            self.read(f"R{s}", k)
            yield ("step",)
            self.empty[s].arrive()
            yield ("step",)
            if k in self.ends and nsub > 1:
                jm = seg % nsub
                if not (self.plant == "no_mg_empty_wait" and j != jm):
                    yield ("wait", self.mg_empty, (seg & 1) ^ 1)
                self.write(f"M{w}", seg)
                self.mg_full.arrive()
                yield ("step",)
                if j == jm:
                    yield ("wait", self.mg_full, seg & 1)
                    if self.plant == "release_before_read":
                        self.mg_empty.arrive()
                        yield ("step",)
                    for jj in range(0 if jm else 1, nsub):
                        self.read(f"M{jj * self.hkv + h}", seg)
                        yield ("step",)
                    if self.plant != "release_before_read":
                        self.mg_empty.arrive()
                    yield ("step",)
                seg += 1

    def run(self):
        # two producer warps issue the even and the odd units
        run_schedule(self, [self.producer(pid, self.PRODUCERS) for pid in range(self.PRODUCERS)] +
                     [self.consumer(w) for w in range(self.warps)])


@pytest.mark.parametrize("hkv,warps", [(8, 8), (4, 8), (2, 8), (1, 8)])
def test_decode_ring_and_merge_protocol(hkv, warps):
    for seed in range(100):
        rng = random.Random(seed * 31 + hkv)
        units = rng.randrange(1, 12)
        ends = {k for k in range(units) if rng.random() < 0.4} | {units - 1}
        DecodeModel(units, ends, hkv, warps, rng).run()


@pytest.mark.parametrize("plant", ["no_mg_empty_wait", "release_before_read"])
def test_decode_planted_mistakes_are_caught(plant):
    caught = 0
    for seed in range(300):
        try:
            DecodeModel(10, {1, 2, 4, 5, 7, 9}, 2, 8, random.Random(seed), plant=plant).run()
        except Hazard:
            caught += 1
    assert caught > 0, f"the planted mistake {plant} went unnoticed in 300 schedules"


class GatherModel:
    """The KV-head-sharded decode's fused all-gather
    (lean-infer_b200/csrc/la_p2p.cu, sharding.NVLinkAllGatherDecode): in call
    n every rank stores its heads' outputs into slot n % slots of every rank's
    gather buffer (the decode kernels, finished and fenced before the barrier
    kernel starts on the same stream), then publishes epoch n + 1 into every
    rank's signal words and waits until each peer's epoch in its own words
    has reached n + 1; the o_proj that follows reads its own slot, and only
    after it does the rank's stream reach the next call's kernels."""

    def __init__(self, world, calls, slots, rng):
        self.world, self.calls, self.slots, self.rng = world, calls, slots, rng
        self.sig = [[0] * world for _ in range(world)]  # sig[q][r]: last epoch rank r published to rank q
        self.mem, self.tma, self.tc = {}, [], []

    read = Model.read
    write = Model.write

    def rank(self, r):
        for n in range(self.calls):
            slot = n % self.slots
            for q in range(self.world):  # this rank's heads into every rank's slot
                self.write(f"G{q}.{slot}.{r}", n)
                yield ("step",)
            for q in range(self.world):  # publish epoch n + 1
                self.sig[q][r] = n + 1
                yield ("step",)
            for q in range(self.world):  # wait for every peer's epoch
                yield ("until", lambda q=q, n=n: self.sig[r][q] >= n + 1)
            for q in range(self.world):  # o_proj reads the gathered heads
                self.read(f"G{r}.{slot}.{q}", n)
                yield ("step",)

    def run(self, max_ticks=200000):
        actors = [self.rank(r) for r in range(self.world)]
        done = [False] * self.world
        until = [None] * self.world  # condition a rank spins on
        speed = [2.0 ** self.rng.uniform(-6, 6) for _ in range(self.world)]
        for _ in range(max_ticks):
            live = [r for r in range(self.world) if not done[r] and (until[r] is None or until[r]())]
            if not live:
                if all(done):
                    return
                raise Hazard("deadlock: every unfinished rank waits for an epoch")
            r = self.rng.choices(live, weights=[speed[i] for i in live])[0]
            try:
                cmd = next(actors[r])
                until[r] = cmd[1] if cmd[0] == "until" else None
            except StopIteration:
                done[r] = True
        raise Hazard("schedule did not finish")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_gather_slots_protocol(world):
    for seed in range(100):
        GatherModel(world, 6, 2, random.Random(seed * 13 + world)).run()


def test_gather_single_slot_is_caught():
    caught = 0
    for seed in range(300):
        try:
            GatherModel(4, 6, 1, random.Random(seed)).run()
        except Hazard:
            caught += 1
    assert caught > 0, "one gather slot for consecutive calls went unnoticed in 300 schedules"


ITEM_SETS = [[1], [2], [3], [4, 1], [1, 3, 2], [5, 1, 1, 4], [2, 2, 2, 2, 2]]


@pytest.mark.parametrize("items", ITEM_SETS)
def test_split_instance_protocol(items):
    for seed in range(150):
        Model(items, random.Random(seed * 7919 + len(items))).run()


@pytest.mark.parametrize("plant", ["one_exchange_barrier", "one_p_barrier", "epilogue_on_pv_parity"])
def test_planted_mistakes_are_caught(plant):
    caught = 0
    for seed in range(300):
        try:
            Model([5, 1, 4, 3], random.Random(seed), plant=plant).run()
        except Hazard:
            caught += 1
    assert caught > 0, f"the planted mistake {plant} went unnoticed in 300 schedules"
