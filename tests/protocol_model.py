"""Explicit-state model of the mbarrier protocols of the tcgen05 kernels on the QLoRA step's path
(csrc/tc_gemm.cuh, csrc/tc_gemm_pair.cuh, csrc/lora_xa.cu, csrc/lora_dx.cu), for the CPU tests.

It checks the hand-offs between a kernel's roles, not the kernels' arithmetic: each role (TMA
producer, MMA issuer, masking / epilogue threads, store thread) is written out as the sequence of
waits, arrivals, copies and MMAs the kernel's loops perform, with the same stage / phase / buffer
bookkeeping, and every interleaving of the roles and of the asynchronous agents is explored. A
deadlock here is a wait that could never complete (a bounded wait that gives up on the GPU); a
hazard is a shared-memory stage or TMEM buffer reused or read out of order.

Each role is an unrolled list of ops; the checker explores every interleaving of role steps and
asynchronous agents (TMA load completions in any order, tcgen05 MMA/commit FIFO per issuing
thread, TMA-store source reads in order). mbarrier semantics follow PTX: phase counter, pending
arrivals, tx count; a phase completes when pending == 0 and tx == 0; try_wait.parity(p) succeeds
iff (phase & 1) != p. Hazards: smem stage generations (TMA overwrite before every reader of the
previous generation is done; read before landed / before masked), TMEM buffers (MMA into a
buffer whose tile i-2 is still being drained; epilogue read before the tile's MMAs are done).
"""
import sys


class Hazard(Exception):
    pass


class Bar:
    __slots__ = ("count", "phase", "pending", "tx")

    def __init__(self, count):
        self.count, self.phase, self.pending, self.tx = count, 0, count, 0

    def key(self):
        return (self.phase, self.pending, self.tx)

    def clone(self):
        b = Bar.__new__(Bar)
        b.count, b.phase, b.pending, b.tx = self.count, self.phase, self.pending, self.tx
        return b

    def _maybe(self):
        if self.pending == 0 and self.tx == 0:
            self.phase += 1
            self.pending = self.count

    def arrive(self, who):
        if self.pending <= 0:
            raise Hazard(f"arrival beyond count by {who}")
        self.pending -= 1
        self._maybe()

    def expect_arrive(self, nbytes, who):
        self.tx += nbytes
        self.arrive(who)

    def complete_tx(self, nbytes):
        self.tx -= nbytes
        self._maybe()

    def done(self, parity):
        return (self.phase & 1) != parity


class World:
    def __init__(self, roles, bars, params):
        self.roles = roles
        self.pc = {r: 0 for r in roles}
        self.bars = bars
        self.p = params
        self.tma = ()
        self.mmaq = {}
        self.stq = {}
        self.ev = {}

    def clone(self):
        w = self.__class__.__new__(self.__class__)
        w.roles, w.p = self.roles, self.p
        w.pc = dict(self.pc)
        w.bars = {k: b.clone() for k, b in self.bars.items()}
        w.tma = self.tma
        w.mmaq = dict(self.mmaq)
        w.stq = dict(self.stq)
        w.ev = dict(self.ev)
        return w

    def key(self):
        return (tuple(sorted(self.pc.items())),
                tuple((k, b.key()) for k, b in sorted(self.bars.items())),
                tuple(sorted(self.tma, key=repr)), tuple(sorted(self.mmaq.items())),
                tuple(sorted(self.stq.items())), tuple(sorted(self.ev.items(), key=repr)))

    def get(self, *k):
        return self.ev.get(k, 0)

    def inc(self, *k):
        self.ev[k] = self.ev.get(k, 0) + 1

    def enabled(self):
        moves = []
        for r, ops in self.roles.items():
            i = self.pc[r]
            if i >= len(ops):
                continue
            op = ops[i]
            if op[0] == "wait":
                if self.bars[op[1]].done(op[2]):
                    moves.append(("role", r))
            elif op[0] == "store_wait_read":
                if not self.stq.get(r):
                    moves.append(("role", r))
            else:
                moves.append(("role", r))
        for j in range(len(self.tma)):
            moves.append(("tma", j))
        for q, fifo in self.mmaq.items():
            if fifo:
                moves.append(("mma", q))
        for q, fifo in self.stq.items():
            if fifo:
                moves.append(("st", q))
        return moves

    def finished(self):
        return all(self.pc[r] >= len(ops) for r, ops in self.roles.items()) and not self.tma \
            and not any(self.mmaq.values()) and not any(self.stq.values())

    def describe(self):
        out = []
        for r, ops in self.roles.items():
            i = self.pc[r]
            out.append(f"{r}@{i}:{ops[i] if i < len(ops) else 'end'}")
        out.append("bars " + ", ".join(f"{k}={b.key()}" for k, b in sorted(self.bars.items())))
        out.append(f"tma {self.tma} mmaq {self.mmaq} stq {self.stq}")
        return "\n  ".join(out)

    def apply(self, m):
        kind, x = m
        if kind == "tma":
            bar, nbytes, s, g = self.tma[x]
            self.tma = self.tma[:x] + self.tma[x + 1:]
            self.inc("landed", s, g)
            self.bars[bar].complete_tx(nbytes)
            return
        if kind == "mma":
            head, rest = self.mmaq[x][0], self.mmaq[x][1:]
            self.mmaq[x] = rest
            if head[0] == "mma":
                _, s, g, tile = head
                self.inc("mma_done", s, g)
                self.inc("tile_mma_done", tile)
            else:
                for b in head[1]:
                    self.bars[b].arrive(f"commit by {x}")
            return
        if kind == "st":
            (s, g), rest = self.stq[x][0], self.stq[x][1:]
            self.stq[x] = rest
            self.inc("store_read", s, g)
            return
        r = x
        op = self.roles[r][self.pc[r]]
        self.pc[r] += 1
        P = self.p
        t = op[0]
        if t in ("wait", "store_wait_read"):
            return
        if t == "arrive":
            for b in op[1]:
                self.bars[b].arrive(r)
        elif t == "expect":
            self.bars[op[1]].expect_arrive(op[2], r)
        elif t == "tma_load":
            _, bar, nbytes, s, g = op
            if g > 0:
                pg = g - 1
                if P["masked"] and self.get("masks", s, pg) != P["maskers"]:
                    raise Hazard(f"{r}: TMA into stage {s} gen {g} before masking of gen {pg}")
                if self.get("mma_done", s, pg) != P["mma_per_stage"]:
                    raise Hazard(f"{r}: TMA into stage {s} gen {g} before MMAs of gen {pg} done")
                if P["store"] and self.get("store_read", s, pg) != 1:
                    raise Hazard(f"{r}: TMA into stage {s} gen {g} before the xd store read {pg}")
            self.tma = self.tma + ((bar, nbytes, s, g),)
        elif t == "mask":
            _, s, g = op
            if self.get("landed", s, g) != P["loads_per_stage"]:
                raise Hazard(f"{r}: masks stage {s} gen {g} before it landed")
            self.inc("masks", s, g)
        elif t == "mma":
            _, s, g, tile, first = op
            if self.get("landed", s, g) != P["loads_per_stage"]:
                raise Hazard(f"{r}: MMA reads stage {s} gen {g} before it landed")
            if P["masked"] and self.get("masks", s, g) != P["maskers"]:
                raise Hazard(f"{r}: MMA reads stage {s} gen {g} before it is masked")
            if first and tile >= 2 and self.get("epi_done", tile - 2) != P["epilogue"]:
                raise Hazard(f"{r}: MMA of tile {tile} into a buffer tile {tile - 2} still drains")
            self.mmaq[r] = self.mmaq.get(r, ()) + (("mma", s, g, tile),)
        elif t == "commit":
            self.mmaq[r] = self.mmaq.get(r, ()) + (("commit", op[1]),)
        elif t == "store":
            _, s, g = op
            if P["masked"] and self.get("masks", s, g) != P["maskers"]:
                raise Hazard(f"{r}: stores stage {s} gen {g} before it is masked")
            self.stq[r] = self.stq.get(r, ()) + ((s, g),)
        elif t == "epi_read":
            _, tile = op
            if self.get("tile_mma_done", tile) != P["mma_per_tile"]:
                raise Hazard(f"{r}: reads tile {tile} before its MMAs are done")
        elif t == "epi_done":
            self.inc("epi_done", op[1])
        elif t == "c_load":          # dx tile cb, generation g, into the C ring by TMA
            _, bar, nbytes, cb, g = op
            if g > 0 and self.get("store_read", ("c", cb), g - 1) != 1:
                raise Hazard(f"{r}: dx tile {cb} gen {g} loaded before gen {g - 1} was stored")
            self.tma = self.tma + ((bar, nbytes, ("c", cb), g),)
        elif t == "c_rewrite":
            _, cb, g = op
            if self.get("landed", ("c", cb), g) != 1:
                raise Hazard(f"{r}: rewrites dx tile {cb} gen {g} before it landed")
            self.inc("c_rw", cb, g)
        elif t == "c_store":
            _, cb, g = op
            if self.get("c_rw", cb, g) != P["epilogue"]:
                raise Hazard(f"{r}: stores dx tile {cb} gen {g} before every row is rewritten")
            self.stq[r] = self.stq.get(r, ()) + ((("c", cb), g),)
        else:
            raise ValueError(op)


def explore(world, limit=30_000_000):
    seen = set()
    stack = [world]
    n = 0
    while stack:
        w = stack.pop()
        k = w.key()
        if k in seen:
            continue
        seen.add(k)
        n += 1
        if n > limit:
            return n, "limit"
        moves = w.enabled()
        if not moves:
            if not w.finished():
                raise Hazard("DEADLOCK:\n  " + w.describe())
            continue
        for m in moves:
            w2 = w.clone()
            w2.apply(m)
            stack.append(w2)
    return n, "complete"


def _adv(s, ph, S):
    return (0, ph ^ 1) if s + 1 == S else (s + 1, ph)


# ---------------------------------------------------------------------- lora_xa (csrc/lora_xa.cu)
def lora_xa(S, nk, mbs, maskers, store, masked=True, empty_count=None):
    prod, mma, st = [], [], []
    mk = [[] for _ in range(maskers)]
    s, ph, it = 0, 0, 0
    for i in range(mbs):
        for kb in range(nk):
            g = it // S
            prod += [("wait", f"empty{s}", ph ^ 1), ("expect", f"full{s}", 2),
                     ("tma_load", f"full{s}", 1, s, g), ("tma_load", f"full{s}", 1, s, g)]
            s, ph = _adv(s, ph, S)
            it += 1
    s, ph, it = 0, 0, 0
    ready = "masked" if masked else "full"
    for i in range(mbs):
        buf = i & 1
        mma.append(("wait", f"tempty{buf}", ((i >> 1) & 1) ^ 1))
        for kb in range(nk):
            g = it // S
            mma += [("wait", f"{ready}{s}", ph), ("mma", s, g, i, kb == 0),
                    ("commit", (f"empty{s}",))]
            s, ph = _adv(s, ph, S)
            it += 1
        mma.append(("commit", (f"tfull{buf}",)))
    mma += [("commit", ("drain",)), ("wait", "drain", 0)]
    for t in range(maskers):
        s, ph, it = 0, 0, 0
        for i in range(mbs):
            if masked:
                for kb in range(nk):
                    g = it // S
                    mk[t] += [("wait", f"full{s}", ph), ("mask", s, g),
                              ("arrive", (f"masked{s}",))]
                    s, ph = _adv(s, ph, S)
                    it += 1
            buf = i & 1
            mk[t] += [("wait", f"tfull{buf}", (i >> 1) & 1), ("epi_read", i), ("epi_done", i),
                      ("arrive", (f"tempty{buf}",))]
    if store:
        s, ph, it = 0, 0, 0
        for i in range(mbs):
            for kb in range(nk):
                g = it // S
                st += [("wait", f"masked{s}", ph), ("store", s, g), ("store_wait_read",),
                       ("arrive", (f"empty{s}",))]
                s, ph = _adv(s, ph, S)
                it += 1
    bars = {}
    for k in range(S):
        bars[f"full{k}"] = Bar(1)
        bars[f"masked{k}"] = Bar(maskers)
        bars[f"empty{k}"] = Bar(empty_count or (2 if store else 1))
    for b in range(2):
        bars[f"tfull{b}"] = Bar(1)
        bars[f"tempty{b}"] = Bar(maskers)
    bars["drain"] = Bar(1)
    roles = {"prod": prod, "mma": mma}
    for t in range(maskers):
        roles[f"mask{t}"] = mk[t]
    if store:
        roles["store"] = st
    params = {"masked": masked, "maskers": maskers, "mma_per_stage": 1, "store": store,
              "loads_per_stage": 2, "epilogue": maskers, "mma_per_tile": nk}
    return World(roles, bars, params)


# ------------------------------------------------------------ one-CTA GEMM (csrc/tc_gemm.cuh)
def gemm1(S, nk, tiles, epi, epi_parity_flip=0):
    prod, mma = [], []
    ep = [[] for _ in range(epi)]
    s, ph, it = 0, 0, 0
    for t in range(tiles):
        for kb in range(nk):
            g = it // S
            prod += [("wait", f"empty{s}", ph ^ 1), ("expect", f"full{s}", 2),
                     ("tma_load", f"full{s}", 1, s, g), ("tma_load", f"full{s}", 1, s, g)]
            s, ph = _adv(s, ph, S)
            it += 1
    s, ph, it = 0, 0, 0
    for t in range(tiles):
        buf = t & 1
        mma.append(("wait", f"tempty{buf}", ((t >> 1) & 1) ^ 1))
        for kb in range(nk):
            g = it // S
            mma += [("wait", f"full{s}", ph), ("mma", s, g, t, kb == 0), ("commit", (f"empty{s}",))]
            s, ph = _adv(s, ph, S)
            it += 1
        mma.append(("commit", (f"tfull{buf}",)))
    mma += [("commit", ("drain",)), ("wait", "drain", 0)]
    for e in range(epi):
        for t in range(tiles):
            buf = t & 1
            ep[e] += [("wait", f"tfull{buf}", ((t >> 1) & 1) ^ epi_parity_flip), ("epi_read", t),
                      ("epi_done", t), ("arrive", (f"tempty{buf}",))]
    bars = {}
    for k in range(S):
        bars[f"full{k}"] = Bar(1)
        bars[f"empty{k}"] = Bar(1)
    for b in range(2):
        bars[f"tfull{b}"] = Bar(1)
        bars[f"tempty{b}"] = Bar(epi)
    bars["drain"] = Bar(1)
    roles = {"prod": prod, "mma": mma}
    for e in range(epi):
        roles[f"epi{e}"] = ep[e]
    params = {"masked": False, "maskers": 0, "mma_per_stage": 1, "store": False,
              "loads_per_stage": 2, "epilogue": epi, "mma_per_tile": nk}
    return World(roles, bars, params)


# ------------------------------------------------------ 2-SM GEMM (csrc/tc_gemm_pair.cuh)
def gemm_pair(S, nk, tiles, epi, leader_bytes=4):
    """Leader L and follower F. Both CTAs' loads (A + B half each) complete on the leader's
    full[s], whose bytes (both CTAs') only the leader arms; the leader's commits arrive on the
    same barrier in both CTAs (empty, tfull); every epilogue warp of both CTAs arrives on the
    leader's tempty."""
    roles = {}
    for c in "LF":
        prod = []
        s, ph, it = 0, 0, 0
        for t in range(tiles):
            for kb in range(nk):
                g = it // S
                prod.append(("wait", f"empty{c}{s}", ph ^ 1))
                if c == "L":
                    prod.append(("expect", f"fullL{s}", leader_bytes))
                prod += [("tma_load", f"fullL{s}", 1, s, g), ("tma_load", f"fullL{s}", 1, s, g)]
                s, ph = _adv(s, ph, S)
                it += 1
        roles[f"prod{c}"] = prod
    mma = []
    s, ph, it = 0, 0, 0
    for t in range(tiles):
        buf = t & 1
        mma.append(("wait", f"temptyL{buf}", ((t >> 1) & 1) ^ 1))
        for kb in range(nk):
            g = it // S
            mma += [("wait", f"fullL{s}", ph), ("mma", s, g, t, kb == 0),
                    ("commit", (f"emptyL{s}", f"emptyF{s}"))]
            s, ph = _adv(s, ph, S)
            it += 1
        mma.append(("commit", (f"tfullL{buf}", f"tfullF{buf}")))
    mma += [("commit", ("drainL",)), ("wait", "drainL", 0)]
    roles["mmaL"] = mma
    for c in "LF":
        for e in range(epi):
            ops = []
            for t in range(tiles):
                buf = t & 1
                ops += [("wait", f"tfull{c}{buf}", (t >> 1) & 1), ("epi_read", t), ("epi_done", t),
                        ("arrive", (f"temptyL{buf}",))]
            roles[f"epi{c}{e}"] = ops
    bars = {}
    for k in range(S):
        bars[f"fullL{k}"] = Bar(1)
        bars[f"emptyL{k}"] = Bar(1)
        bars[f"emptyF{k}"] = Bar(1)
    for b in range(2):
        bars[f"tfullL{b}"] = Bar(1)
        bars[f"tfullF{b}"] = Bar(1)
        bars[f"temptyL{b}"] = Bar(2 * epi)
    bars["drainL"] = Bar(1)
    params = {"masked": False, "maskers": 0, "mma_per_stage": 1, "store": False,
              "loads_per_stage": 4, "epilogue": 2 * epi, "mma_per_tile": nk}
    return World(roles, bars, params)


# ----------------------------------------------- masked input gradient (csrc/lora_dx.cu)
def lora_dx(S, nk, tiles, epi):
    """Producer: per tile, wait cempty[cb], load the dx tile (cfull), then the operand ring.
    MMA as in the GEMM. Epilogue threads: wait tfull and cfull, rewrite their rows, arrive tempty
    and cdone; thread 0 of them (the storer) then waits cdone, TMA-stores the tile, waits for the
    store's read and arrives cempty."""
    prod, mma = [], []
    ep = [[] for _ in range(epi)]
    s, ph, it = 0, 0, 0
    for i in range(tiles):
        cb = i & 1
        prod += [("wait", f"cempty{cb}", ((i >> 1) & 1) ^ 1), ("expect", f"cfull{cb}", 1),
                 ("c_load", f"cfull{cb}", 1, cb, i >> 1)]
        for kb in range(nk):
            g = it // S
            prod += [("wait", f"empty{s}", ph ^ 1), ("expect", f"full{s}", 2),
                     ("tma_load", f"full{s}", 1, s, g), ("tma_load", f"full{s}", 1, s, g)]
            s, ph = _adv(s, ph, S)
            it += 1
    s, ph, it = 0, 0, 0
    for i in range(tiles):
        buf = i & 1
        mma.append(("wait", f"tempty{buf}", ((i >> 1) & 1) ^ 1))
        for kb in range(nk):
            g = it // S
            mma += [("wait", f"full{s}", ph), ("mma", s, g, i, kb == 0), ("commit", (f"empty{s}",))]
            s, ph = _adv(s, ph, S)
            it += 1
        mma.append(("commit", (f"tfull{buf}",)))
    mma += [("commit", ("drain",)), ("wait", "drain", 0)]
    for e in range(epi):
        for i in range(tiles):
            buf = cb = i & 1
            par = (i >> 1) & 1
            ep[e] += [("wait", f"tfull{buf}", par), ("wait", f"cfull{cb}", par), ("epi_read", i),
                      ("c_rewrite", cb, i >> 1), ("epi_done", i), ("arrive", (f"tempty{buf}",)),
                      ("arrive", (f"cdone{cb}",))]
            if e == 0:
                ep[e] += [("wait", f"cdone{cb}", par), ("c_store", cb, i >> 1),
                          ("store_wait_read",), ("arrive", (f"cempty{cb}",))]
    bars = {}
    for k in range(S):
        bars[f"full{k}"] = Bar(1)
        bars[f"empty{k}"] = Bar(1)
    for b in range(2):
        bars[f"cfull{b}"] = Bar(1)
        bars[f"cdone{b}"] = Bar(epi)
        bars[f"cempty{b}"] = Bar(1)
        bars[f"tfull{b}"] = Bar(1)
        bars[f"tempty{b}"] = Bar(epi)
    bars["drain"] = Bar(1)
    roles = {"prod": prod, "mma": mma}
    for e in range(epi):
        roles[f"epi{e}"] = ep[e]
    params = {"masked": False, "maskers": 0, "mma_per_stage": 1, "store": False,
              "loads_per_stage": 2, "epilogue": epi, "mma_per_tile": nk}
    return World(roles, bars, params)


# ------------------------------------------------------------- generic ring model (NF4 kernel)
class RingWorld(World):
    """The vocabulary for kernels with several rings and thread-written operands:
        ("load", bar, nbytes, ring, s, g)  TMA into ring stage s, generation g
        ("write", ring, s, g)              one thread's part of a thread-written stage
        ("read", ring, s, g)               a thread reads a stage (must be complete)
        ("use", ring, s, g)                a thread is done with a stage
        ("mma2", ((ring, s, g), ...), tile, first)   MMA reading those stages
    A stage may be refilled once all its consumers of the previous generation are done
    (need_use[ring]); it is complete once need_ready[ring] loads / writes landed."""

    def apply(self, m):
        kind, x = m
        P = self.p
        if kind == "tma":
            bar, nbytes, ring, s, g = self.tma[x]
            self.tma = self.tma[:x] + self.tma[x + 1:]
            self.inc("ready", ring, s, g)
            self.bars[bar].complete_tx(nbytes)
            return
        if kind == "mma":
            head, rest = self.mmaq[x][0], self.mmaq[x][1:]
            self.mmaq[x] = rest
            if head[0] == "mma2":
                for ring, s, g in head[1]:
                    self.inc("used", ring, s, g)
                self.inc("tile_mma_done", head[2])
            else:
                for b in head[1]:
                    self.bars[b].arrive(f"commit by {x}")
            return
        r = x
        op = self.roles[r][self.pc[r]]
        t = op[0]
        if t not in ("load", "write", "read", "use", "mma2"):
            return World.apply(self, m)
        self.pc[r] += 1

        def refill_ok(ring, s, g):
            if g > 0 and self.get("used", ring, s, g - 1) != P["need_use"][ring]:
                raise Hazard(f"{r}: refills {ring} stage {s} gen {g} before gen {g - 1} is used")

        def complete(ring, s, g, who):
            if self.get("ready", ring, s, g) != P["need_ready"][ring]:
                raise Hazard(f"{who}: reads {ring} stage {s} gen {g} before it is complete")

        if t == "load":
            _, bar, nbytes, ring, s, g = op
            refill_ok(ring, s, g)
            self.tma = self.tma + ((bar, nbytes, ring, s, g),)
        elif t == "write":
            _, ring, s, g = op
            refill_ok(ring, s, g)
            self.inc("ready", ring, s, g)
        elif t == "read":
            _, ring, s, g = op
            complete(ring, s, g, r)
        elif t == "use":
            _, ring, s, g = op
            self.inc("used", ring, s, g)
        elif t == "mma2":
            _, stages, tile, first = op
            for ring, s, g in stages:
                complete(ring, s, g, r)
            if first and tile >= P["acc_sets"] and \
                    self.get("epi_done", tile - P["acc_sets"]) != P["epilogue"]:
                raise Hazard(f"{r}: MMA of tile {tile} into accumulators still being drained")
            self.mmaq[r] = self.mmaq.get(r, ()) + (("mma2", stages, tile),)


def nf4_gemm(SB, SA, SC, nk0, nk1, tiles, warps_per_group=2, epi=1, groups=2):
    """csrc/tc_nf4_gemm.cuh: B ring by TMA (warp 0), codes ring by TMA (warp 6, segment-0
    k-blocks only), A ring written by `groups` dequant groups taking alternate k-blocks (item it
    goes to group it % groups; every group steps through every stage index), one accumulator set
    (tfull[0] / tempty[0], parity t & 1). Each group is modelled as `warps_per_group` threads:
    fullA counts the group's threads, emptyC one arrival per warp.

    A group waits for an item's codes only after that item's A slot is free, and its own previous
    item (two items back) read the codes stage before that, so no codes stage is waited on two
    generations ahead of its fills while the codes ring has at least as many stages as there are
    groups (the kernel: 8 stages, 2 groups). With a one-stage ring the checker finds the parity
    aliasing: a group would take an unfilled stage for a filled one."""
    nk = nk0 + nk1
    W = warps_per_group
    roles = {}
    ops, st, ph, it = [], 0, 0, 0
    for t in range(tiles):
        for kb in range(nk):
            ops += [("wait", f"emptyB{st}", ph ^ 1), ("expect", f"fullB{st}", 1),
                    ("load", f"fullB{st}", 1, "B", st, it // SB)]
            st, ph = _adv(st, ph, SB)
            it += 1
    roles["prodB"] = ops
    ops, st, ph, it = [], 0, 0, 0
    for t in range(tiles):
        for kb in range(nk0):
            ops += [("wait", f"emptyC{st}", ph ^ 1), ("expect", f"fullC{st}", 1),
                    ("load", f"fullC{st}", 1, "C", st, it // SC)]
            st, ph = _adv(st, ph, SC)
            it += 1
    roles["prodC"] = ops
    ops = []
    sb = sa = 0
    pbh = pah = 0
    it = 0
    for t in range(tiles):
        ops.append(("wait", "tempty0", (t & 1) ^ 1))
        for kb in range(nk):
            ops += [("wait", f"fullB{sb}", pbh), ("wait", f"fullA{sa}", pah),
                    ("mma2", (("B", sb, it // SB), ("A", sa, it // SA)), t, kb == 0),
                    ("commit", (f"emptyB{sb}",)), ("commit", (f"emptyA{sa}",))]
            sb, pbh = _adv(sb, pbh, SB)
            sa, pah = _adv(sa, pah, SA)
            it += 1
        ops.append(("commit", ("tfull0",)))
    ops += [("commit", ("drain",)), ("wait", "drain", 0)]
    roles["mma"] = ops
    for e in range(epi):
        roles[f"epi{e}"] = sum(([("wait", "tfull0", t & 1), ("epi_read", t), ("epi_done", t),
                                 ("arrive", ("tempty0",))] for t in range(tiles)), [])
    for grp in range(groups):
        for w in range(W):
            ops = []
            sa = sc = 0
            pah = pch = 0
            it = itc = 0
            for t in range(tiles):
                for kb in range(nk):
                    seg0 = kb < nk0
                    if it % groups == grp:
                        ops.append(("wait", f"emptyA{sa}", pah ^ 1))
                        if seg0:
                            ops += [("wait", f"fullC{sc}", pch), ("read", "C", sc, itc // SC),
                                    ("write", "A", sa, it // SA), ("use", "C", sc, itc // SC),
                                    ("arrive", (f"emptyC{sc}",))]
                        else:
                            ops.append(("write", "A", sa, it // SA))
                        ops.append(("arrive", (f"fullA{sa}",)))
                    sa, pah = _adv(sa, pah, SA)
                    if seg0:
                        sc, pch = _adv(sc, pch, SC)
                        itc += 1
                    it += 1
            roles[f"deq{grp}.{w}"] = ops
    bars = {}
    for k in range(SB):
        bars[f"fullB{k}"], bars[f"emptyB{k}"] = Bar(1), Bar(1)
    for k in range(SA):
        bars[f"fullA{k}"], bars[f"emptyA{k}"] = Bar(W), Bar(1)
    for k in range(SC):
        bars[f"fullC{k}"], bars[f"emptyC{k}"] = Bar(1), Bar(W)
    bars["tfull0"], bars["tempty0"], bars["drain"] = Bar(1), Bar(epi), Bar(1)
    params = {"need_use": {"B": 1, "A": 1, "C": W}, "need_ready": {"B": 1, "A": W, "C": 1},
              "acc_sets": 1, "epilogue": epi, "mma_per_tile": nk}
    w = RingWorld.__new__(RingWorld)
    World.__init__(w, roles, bars, params)
    return w
