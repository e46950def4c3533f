"""Randomised models of the mbarrier protocols of the tcgen05 attention kernels
(onionop.jl_b200/csrc/fa_fwd_sm100.cu, fa_bwd_sm100.cu), for tests on the CPU.

Each kernel role (TMA producer, MMA issuer, softmax / elementwise warpgroups,
tile provider, dQ warps) is a generator that yields the waits and arrivals the
kernel code performs, in the kernel's order.  The tensor pipe is an in-order
queue (tcgen05 operations of one thread run in issue order; a commit arrives
once everything issued before it is done), TMA loads and stores complete at
random times, and a random scheduler interleaves everything.  Shared-memory
buffers and TMEM column ranges carry tags of the data they hold: every read
checks the tag it expects, every overwrite checks that the old data has been
consumed.  A wait for phase k models the hardware's parity test: it passes
once k+1 phases completed and is a hang if k+2 have (the parity repeats).

The models restate the kernels' protocols by hand; a change to a kernel's
barriers should be mirrored here.  `plant` removes one wait (a planted mistake,
on the CPU) so the tests can check that the model notices.
"""
from __future__ import annotations

import random


class ProtocolBug(Exception):
    pass


class _Bar:
    def __init__(self, name, count):
        self.name, self.count, self.pending, self.done = name, count, 0, 0

    def arrive(self):
        self.pending += 1
        if self.pending == self.count:
            self.pending, self.done = 0, self.done + 1


class _Sim:
    def __init__(self, seed, slow_tma: bool = False, slow_roles=()):
        # slow_tma: a copy in flight lands only rarely while anything else can
        # run (long TMA latencies), which exposes waits on copies that the
        # uniform schedule would nearly always find already landed; roles in
        # slow_roles likewise run only rarely while anything else can.
        self.slow_tma = slow_tma
        self.slow_roles = set(slow_roles)
        self.rng = random.Random(seed)
        self.bars, self.mem, self.pipe, self.asyncs = {}, {}, [], []
        self.executed = set()

    def bar(self, name, count=1):
        self.bars[name] = _Bar(name, count)

    def expect(self, key, tag):
        if self.mem.get(key) != tag:
            raise ProtocolBug(f"{key}: expected {tag}, holds {self.mem.get(key)}")

    def mma(self, op_id, fn):
        self.pipe.append(("mma", op_id, fn))

    def commit(self, bar):
        self.pipe.append(("commit", bar))

    def run(self, roles, max_steps=400000):
        blocked = {n: None for n in roles}
        finished = set()

        def runnable(n):
            w = blocked[n]
            if w is None:
                return True
            if w[0] == "until":
                return w[1]()
            b, k = self.bars[w[0]], w[1]
            if b.done >= k + 2:
                raise ProtocolBug(f"{n}: phase overrun on {b.name} (waits phase {k}, {b.done} done)")
            return b.done >= k + 1

        for _ in range(max_steps):
            c = [("role", n) for n in roles if n not in finished and runnable(n)]
            if self.pipe:
                c.append(("pipe", None))
            if self.asyncs:
                c.append(("async", None))
            if not c:
                if len(finished) == len(roles):
                    return
                raise ProtocolBug(f"deadlock: {[(n, blocked[n]) for n in roles if n not in finished]}")
            if self.slow_tma and len(c) > 1 and c[-1][0] == "async" and self.rng.random() < 0.97:
                c.pop()
            if self.slow_roles and self.rng.random() < 0.97:
                fast = [x for x in c if not (x[0] == "role" and x[1] in self.slow_roles)]
                if fast:
                    c = fast
            kind, n = self.rng.choice(c)
            if kind == "pipe":
                op = self.pipe.pop(0)
                if op[0] == "mma":
                    op[2]()
                    self.executed.add(op[1])
                else:
                    self.bars[op[1]].arrive()
            elif kind == "async":
                fn, b = self.asyncs.pop(self.rng.randrange(len(self.asyncs)))
                fn()
                if b is not None:
                    self.bars[b].arrive()
            else:
                blocked[n] = None
                try:
                    a = next(roles[n])
                except StopIteration:
                    finished.add(n)
                    continue
                if a[0] == "wait":
                    blocked[n] = (a[1], a[2])
                elif a[0] == "until":
                    blocked[n] = ("until", a[1])
                elif a[0] == "arrive":
                    self.bars[a[1]].arrive()
                else:
                    a[1]()
        raise ProtocolBug("no progress")


def _wait(plant, name, phase):
    """A wait, unless it is the planted mistake."""
    return ("do", lambda: None) if plant == name else ("wait", name, phase)


# ------------------------------------------------------------------ forward
def forward(n_kt: int, pair: bool, seed: int, rescale_p: float = 0.5, plant: str | None = None):
    """fa_fwd_sm100_kernel: Q once; K/V 2-stage ring; pair tiles in a 3-slot ring
    loaded two key tiles ahead; S in two TMEM buffers (P aliases its tile's S);
    one softmax warpgroup; PV(j) after PFull(j); S(j+1) issued before waiting
    PFull(j)."""
    sim = _Sim(seed)
    sim.bar("QFull")
    for s in range(2):
        for n in ("KFull", "VFull", "KVEmpty", "SFull", "PFull"):
            sim.bar(f"{n}{s}")
    for s in range(3):
        sim.bar(f"PairFull{s}")
        sim.bar(f"PairEmpty{s}")
    for n in ("OStep", "OFinal", "MmaDone"):
        sim.bar(n)
    o = {"n": 0}

    def producer():
        yield ("do", lambda: None)
        if n_kt == 0:
            return
        sim.asyncs.append((lambda: sim.mem.__setitem__("Q", "q"), "QFull"))

        def load_pair(j):
            slot = j % 3
            if j >= 3:
                yield _wait(plant, f"PairEmpty{slot}", j // 3 - 1)

            def land(j=j, slot=slot):
                if j >= 3 and ("S", j - 3) not in sim.executed:
                    raise ProtocolBug(f"pair slot {slot} reloaded before S({j - 3}) read it")
                sim.mem[f"pair{slot}"] = j
            sim.asyncs.append((land, f"PairFull{slot}"))
        if pair:
            yield from load_pair(0)
            if n_kt >= 2:
                yield from load_pair(1)
        for j in range(n_kt):
            s = j % 2
            if j >= 2:
                yield _wait(plant, f"KVEmpty{s}", j // 2 - 1)

            def land_kv(j=j, s=s):
                if j >= 2 and ("PV", j - 2) not in sim.executed:
                    raise ProtocolBug(f"K/V stage {s} reloaded before PV({j - 2}) read it")
                sim.mem[f"K{s}"] = sim.mem[f"V{s}"] = j
            sim.asyncs.append((land_kv, f"KFull{s}"))
            sim.asyncs.append((lambda: None, f"VFull{s}"))
            if pair and j + 2 < n_kt:
                yield from load_pair(j + 2)

    def mma():
        if n_kt == 0:
            yield ("do", lambda: None)
            return
        yield ("wait", "QFull", 0)

        def issue_s(j):
            s = j % 2
            yield _wait(plant, f"KFull{s}", j // 2)
            if pair:
                yield _wait(plant, f"PairFull{j % 3}", j // 3)

            def run(j=j, s=s):
                sim.expect("Q", "q")
                sim.expect(f"K{s}", j)
                if pair:
                    sim.expect(f"pair{j % 3}", j)
                if j >= 2 and ("PV", j - 2) not in sim.executed:
                    raise ProtocolBug(f"S({j}) overwrites P({j - 2}) before PV read it")
                sim.mem[f"S{j & 1}"] = ("S", j)
            sim.mma(("S", j), run)
            if pair:
                sim.commit(f"PairEmpty{j % 3}")
            sim.commit(f"SFull{j & 1}")

        yield from issue_s(0)
        for j in range(n_kt):
            if j + 1 < n_kt:
                yield from issue_s(j + 1)
            s = j % 2
            yield _wait(plant, f"PFull{j & 1}", j >> 1)
            yield ("wait", f"VFull{s}", j // 2)

            def pv(j=j, s=s):
                sim.expect(f"S{j & 1}", ("P", j))
                sim.expect(f"V{s}", j)
                if o["n"] != j:
                    raise ProtocolBug(f"O holds {o['n']} products at PV({j})")
                o["n"] += 1
            sim.mma(("PV", j), pv)
            sim.commit(f"KVEmpty{s}")
            sim.commit("OStep")
            if j == n_kt - 1:
                sim.commit("OFinal")
        sim.commit("MmaDone")
        yield ("wait", "MmaDone", 0)

    def softmax():
        yield ("do", lambda: None)
        for j in range(n_kt):
            yield _wait(plant, f"SFull{j & 1}", j >> 1)

            def sm(j=j):
                sim.expect(f"S{j & 1}", ("S", j))
                sim.mem[f"S{j & 1}"] = ("P", j)
            yield ("do", sm)
            if j > 0 and sim.rng.random() < rescale_p:
                yield _wait(plant, "OStep", j - 1)

                def resc(j=j):
                    if o["n"] != j:
                        raise ProtocolBug(f"O rescaled with {o['n']} products at key tile {j}")
                yield ("do", resc)
            yield ("arrive", f"PFull{j & 1}")
        if n_kt:
            yield _wait(plant, "OFinal", 0)

            def fin():
                if o["n"] != n_kt:
                    raise ProtocolBug(f"O read with {o['n']} of {n_kt} products")
            yield ("do", fin)

    sim.run({"producer": producer(), "mma": mma(), "softmax": softmax()})


# ------------------------------------------------------------------ backward (E = 64)
def backward(T: int, pair: bool, seed: int, plant: str | None = None, slow_roles=(), slow_tma: bool = False):
    """fa_bwd_sm100_kernel (E = 64): Q/dO 2-stage ring per 128-query tile; two
    64-query halves with their own TMEM Sᵀ/dPᵀ and elementwise warpgroups;
    products (dV, dK) per half, S(t+1, half) right behind them; per tile dQ
    from the tile's dS buffer (2 buffers), drained by 4 dQ warps that then
    stage fp32 rows in that buffer; with a pair bias the MMA warp TMA-stores
    each dS half (bulk_wait_read<2> per half, <0> before the dQ commit) and the
    pair arrives in a 4-slot ring of half tiles, loaded by the Q/dO producer
    after each tile's Q/dO; slot 3 is the V tile's shared memory, free once V
    is in TMEM.  K and V go
    from their TMA
    tile into TMEM (the score MMAs' A operand) by the elementwise threads once
    KVFull completes; the MMA warp waits KVTmem before its first score."""
    sim = _Sim(seed, slow_tma, slow_roles)
    for n, c in (("KVFull", 1), ("KVTmem", 2), ("DQFull", 1), ("DQEmpty", 4), ("Final", 1)):
        sim.bar(n, c)
    for i in range(2):
        for n, c in (("QFull", 1), ("QEmpty", 1), ("SFull", 1), ("PFull", 1), ("DSEmpty", 4), ("TileFull", 1),
                     ("TileEmpty", 2)):
            sim.bar(f"{n}{i}", c)
    for i in range(4):
        sim.bar(f"PairFull{i}")
        sim.bar(f"PairEmpty{i}")
    stored, drained, lse_reads, pair_reads, staged = set(), {}, {}, set(), set()

    def producer():
        yield ("do", lambda: None)
        sim.asyncs.append((lambda: sim.mem.__setitem__("KV", "kv"), "KVFull"))
        for t in range(T):
            s = t & 1
            if t >= 2:
                yield _wait(plant, f"QEmpty{s}", (t >> 1) - 1)

            def landq(t=t, s=s):
                if t >= 2 and not {("P", t - 2, 0), ("P", t - 2, 1)} <= sim.executed:
                    raise ProtocolBug(f"Q/dO stage {s} reloaded before the products of tile {t - 2}")
                sim.mem[f"Q{s}"] = t
            sim.asyncs.append((landq, f"QFull{s}"))
            if pair:
                for h in range(2):
                    yield from load_pair(2 * t + h)

    def load_pair(n):
        slot = n % 4
        if n >= 4:
            yield _wait(plant, f"PairEmpty{slot}", n // 4 - 1)
        if n == 3:   # slot 3 is V's shared tile: free once V is in TMEM
            yield _wait(plant, "KVTmem", 0)

        def landp(n=n, slot=slot):
            if n >= 4 and (n - 4) not in pair_reads:
                raise ProtocolBug(f"pair slot {slot} reloaded before half {n - 4} read it")
            if slot == 3 and sim.mem.get("KVT1") != "kv":
                raise ProtocolBug("pair slot 3 overwrites V before it was copied into TMEM")
            sim.mem[f"pair{slot}"] = n
        sim.asyncs.append((landp, f"PairFull{slot}"))

    def mma():
        yield ("wait", "KVFull", 0)
        yield _wait(plant, "KVTmem", 0)
        issued = []

        def issue_s(t, h):
            if h == 0:
                yield _wait(plant, f"QFull{t & 1}", t >> 1)

            def run(t=t, h=h):
                sim.expect("KVT0", "kv")
                sim.expect("KVT1", "kv")
                sim.expect(f"Q{t & 1}", t)
                if t > 0 and ("P", t - 1, h) not in sim.executed:
                    raise ProtocolBug(f"S({t},{h}) overwrites P/dS before products({t - 1},{h})")
                sim.mem[f"S{h}"] = ("S", t)
            sim.mma(("S", t, h), run)
            sim.commit(f"SFull{h}")

        yield from issue_s(0, 0)
        yield from issue_s(0, 1)
        for t in range(T):
            for h in range(2):
                yield _wait(plant, f"PFull{h}", t)
                if pair:
                    def store(t=t, h=h):
                        sim.expect(f"ds{t & 1}{h}", ("dS", t))
                        issued.append((t, h))

                        def done(k=(t, h)):
                            sim.expect(f"ds{k[0] & 1}{k[1]}", ("dS", k[0]))
                            stored.add(k)
                        sim.asyncs.append((done, None))
                    yield ("do", store)
                    if plant != "bulk_wait_read2":
                        yield ("until", lambda n=len(issued): all(k in stored for k in issued[:n - 2]))

                def prod(t=t, h=h):
                    sim.expect(f"S{h}", ("P", t))
                    sim.expect(f"Q{t & 1}", t)
                sim.mma(("P", t, h), prod)
                if h == 1:
                    sim.commit(f"QEmpty{t & 1}")
                if t + 1 < T:
                    yield from issue_s(t + 1, h)
            if t > 0:
                yield _wait(plant, "DQEmpty", t - 1)
            if pair and plant != "bulk_wait_read0":
                yield ("until", lambda n=len(issued): all(k in stored for k in issued[:n]))

            def dq(t=t):
                for h in range(2):
                    sim.expect(f"ds{t & 1}{h}", ("dS", t))
                if t > 0 and len(drained.get(t - 1, ())) < 4:
                    raise ProtocolBug(f"dQ({t}) overwrites dQ({t - 1}) before it was drained")
                sim.mem["DQ"] = t
            sim.mma(("DQ", t), dq)
            sim.commit("DQFull")
        sim.commit("Final")
        yield ("wait", "Final", 0)

    def provider():
        yield ("do", lambda: None)
        for t in range(T):
            if t >= 2:
                yield _wait(plant, f"TileEmpty{t & 1}", (t >> 1) - 1)

            def wr(t=t):
                old = sim.mem.get(f"lse{t & 1}")
                if old is not None and len(lse_reads.get(old, ())) < 2:
                    raise ProtocolBug(f"lse/delta of tile {old} overwritten before both halves read them")
                sim.mem[f"lse{t & 1}"] = t
            yield ("do", wr)
            yield ("arrive", f"TileFull{t & 1}")

    def elementwise(h):
        yield _wait(plant, "KVFull", 0)

        def to_tmem(h=h):
            sim.expect("KV", "kv")
            sim.mem[f"KVT{h}"] = "kv"
        yield ("do", to_tmem)
        yield ("arrive", "KVTmem")
        for t in range(T):
            yield _wait(plant, f"TileFull{t & 1}", t >> 1)
            yield _wait(plant, f"SFull{h}", t)
            if t >= 2:
                yield _wait(plant, f"DSEmpty{t & 1}", (t >> 1) - 1)
            n = 2 * t + h
            if pair:
                yield _wait(plant, f"PairFull{n % 4}", n // 4)

            def ew(t=t, h=h, n=n):
                sim.expect(f"lse{t & 1}", t)
                lse_reads.setdefault(t, set()).add(h)
                sim.expect(f"S{h}", ("S", t))
                if pair:
                    sim.expect(f"pair{n % 4}", n)
                    pair_reads.add(n)
                old = sim.mem.get(f"ds{t & 1}{h}")
                if old is not None and (old != ("stg", t - 2) or (t - 2) not in staged):
                    raise ProtocolBug(f"dS buffer {t & 1} half {h} rewritten while it holds {old}")
                sim.mem[f"S{h}"] = ("P", t)
                sim.mem[f"ds{t & 1}{h}"] = ("dS", t)
            yield ("do", ew)
            yield ("arrive", f"TileEmpty{t & 1}")
            if pair:
                yield ("arrive", f"PairEmpty{n % 4}")
            yield ("arrive", f"PFull{h}")

    def dq_warp(w):
        for t in range(T):
            yield _wait(plant, "DQFull", t)

            def rd(t=t, w=w):
                sim.expect("DQ", t)
                drained.setdefault(t, set()).add(w)
            yield ("do", rd)
            yield ("arrive", "DQEmpty")

            def stage(t=t):
                if ("DQ", t) not in sim.executed:
                    raise ProtocolBug(f"staging into the dS buffer before dQ({t}) read it")
                if pair and not {(t, 0), (t, 1)} <= stored:
                    raise ProtocolBug(f"staging of tile {t} before its dS stores read the buffer")
                for h in range(2):
                    if sim.mem.get(f"ds{t & 1}{h}") not in (("dS", t), ("stg", t)):
                        raise ProtocolBug(f"staging into dS buffer {t & 1} holding {sim.mem.get(f'ds{t & 1}{h}')}")
                    sim.mem[f"ds{t & 1}{h}"] = ("stg", t)
            yield ("do", stage)
            if w == 3:
                yield ("do", lambda t=t: staged.add(t))
            yield ("arrive", f"DSEmpty{t & 1}")

    roles = {"producer": producer(), "mma": mma(), "provider": provider(), "ew0": elementwise(0),
             "ew1": elementwise(1)}
    for w in range(4):
        roles[f"dq{w}"] = dq_warp(w)
    sim.run(roles)


# ------------------------------------------------------------------ backward (E = 128)
def backward128(T: int, seed: int, plant: str | None = None, slow_tma: bool = False):
    """fa_bwd128_sm100_kernel (E = 128, no pair): Q/dO 3-stage ring per 64-query
    step; steps alternate between two elementwise warpgroups, each with its own
    TMEM Sᵀ and dPᵀ buffers; the packed Pᵀ/dSᵀ overwrite the step's Sᵀ columns,
    dQᵀ is written into the warpgroup's dPᵀ columns once the elementwise step is
    done with them, and read out by 4 dQ warps that then stage fp32 boxes in the
    warpgroup's dS buffer.  Per step: products (dV, dK) and dQᵀ behind PFull;
    Sᵀ(t+2) right behind them; dPᵀ(t+2) after DQEmpty (dQᵀ(t) read)."""
    sim = _Sim(seed, slow_tma)
    sim.bar("KVFull")
    sim.bar("Final")
    for s in range(3):
        sim.bar(f"QFull{s}")
        sim.bar(f"QEmpty{s}")
    for w in range(2):
        for n, c in (("SFull", 1), ("PFull", 1), ("DQFull", 1), ("DQEmpty", 4), ("DSEmpty", 4), ("TileFull", 1),
                     ("TileEmpty", 1)):
            sim.bar(f"{n}{w}", c)
    drained, lse_reads, ew_done = {}, set(), set()

    def producer():
        yield ("do", lambda: None)
        if T == 0:
            return
        sim.asyncs.append((lambda: sim.mem.__setitem__("KV", "kv"), "KVFull"))
        for t in range(T):
            s = t % 3
            if t >= 3:
                yield _wait(plant, f"QEmpty{s}", t // 3 - 1)

            def landq(t=t, s=s):
                if t >= 3 and ("P", t - 3) not in sim.executed:
                    raise ProtocolBug(f"Q/dO stage {s} reloaded before the products of step {t - 3}")
                sim.mem[f"Q{s}"] = t
            sim.asyncs.append((landq, f"QFull{s}"))

    def mma():
        if T == 0:
            yield ("do", lambda: None)
        else:
            yield ("wait", "KVFull", 0)

        def score(t, dp):
            w = t & 1

            def run(t=t, w=w, dp=dp):
                sim.expect("KV", "kv")
                sim.expect(f"Q{t % 3}", t)
                if dp:
                    if t >= 2 and len(drained.get(t - 2, ())) < 4:
                        raise ProtocolBug(f"dP({t}) overwrites dQ({t - 2}) before it was drained")
                    sim.mem[f"DP{w}"] = ("dP", t)
                else:
                    if t >= 2 and ("P", t - 2) not in sim.executed:
                        raise ProtocolBug(f"S({t}) overwrites P/dS({t - 2}) before the products read them")
                    sim.mem[f"S{w}"] = ("S", t)
            sim.mma(("dP" if dp else "S", t), run)

        for t in range(min(T, 2)):
            yield _wait(plant, f"QFull{t % 3}", t // 3)
            score(t, False)
            score(t, True)
            sim.commit(f"SFull{t & 1}")
        for t in range(T):
            w = t & 1
            yield _wait(plant, f"PFull{w}", t >> 1)

            def prod(t=t, w=w):
                sim.expect(f"S{w}", ("P", t))
                sim.expect(f"Q{t % 3}", t)
            sim.mma(("P", t), prod)
            sim.commit(f"QEmpty{t % 3}")

            def dq(t=t, w=w):
                sim.expect(f"ds{w}", ("dS", t))
                if t not in ew_done:
                    raise ProtocolBug(f"dQ({t}) overwrites dP({t}) before the elementwise step read it")
                sim.mem[f"DP{w}"] = ("dQ", t)
            sim.mma(("DQ", t), dq)
            sim.commit(f"DQFull{w}")
            if t + 2 < T:
                yield _wait(plant, f"QFull{(t + 2) % 3}", (t + 2) // 3)
                score(t + 2, False)
                yield _wait(plant, f"DQEmpty{w}", t >> 1)
                score(t + 2, True)
                sim.commit(f"SFull{w}")
        sim.commit("Final")
        yield ("wait", "Final", 0)

    def provider():
        yield ("do", lambda: None)
        for t in range(T):
            w = t & 1
            if t >= 2:
                yield _wait(plant, f"TileEmpty{w}", (t >> 1) - 1)

            def wr(t=t, w=w):
                old = sim.mem.get(f"lse{w}")
                if old is not None and old not in lse_reads:
                    raise ProtocolBug(f"lse/delta of step {old} overwritten before its warpgroup read them")
                sim.mem[f"lse{w}"] = t
            for _ in range(sim.rng.randrange(0, 40) if slow_tma else 0):   # global lse/delta loads in flight
                yield ("do", lambda: None)
            yield ("do", wr)
            yield ("arrive", f"TileFull{w}")

    def elementwise(w):
        yield ("do", lambda: None)
        for t in range(w, T, 2):
            n = t >> 1
            yield _wait(plant, f"TileFull{w}", n)
            yield _wait(plant, f"SFull{w}", n)
            if n >= 1:
                yield _wait(plant, f"DSEmpty{w}", n - 1)

            def ew(t=t, w=w):
                sim.expect(f"lse{w}", t)
                lse_reads.add(t)
                sim.expect(f"S{w}", ("S", t))
                sim.expect(f"DP{w}", ("dP", t))
                old = sim.mem.get(f"ds{w}")
                if old is not None and old != ("stg", t - 2, 4):
                    raise ProtocolBug(f"dS buffer {w} rewritten while it holds {old}")
                sim.mem[f"S{w}"] = ("P", t)
                sim.mem[f"ds{w}"] = ("dS", t)
                ew_done.add(t)
            yield ("do", ew)
            yield ("arrive", f"TileEmpty{w}")
            yield ("arrive", f"PFull{w}")

    def dq_warp(wi):
        for t in range(T):
            w = t & 1
            yield _wait(plant, f"DQFull{w}", t >> 1)

            def rd(t=t, w=w, wi=wi):
                sim.expect(f"DP{w}", ("dQ", t))
                drained.setdefault(t, set()).add(wi)
            yield ("do", rd)
            yield ("arrive", f"DQEmpty{w}")

            def stage(t=t, w=w):
                if ("DQ", t) not in sim.executed:
                    raise ProtocolBug(f"staging into dS buffer {w} before dQ({t}) read it")
                cur = sim.mem.get(f"ds{w}")
                if cur == ("dS", t):
                    sim.mem[f"ds{w}"] = ("stg", t, 1)
                elif isinstance(cur, tuple) and cur[:2] == ("stg", t):
                    sim.mem[f"ds{w}"] = ("stg", t, cur[2] + 1)
                else:
                    raise ProtocolBug(f"staging of step {t} into dS buffer {w} holding {cur}")
            yield ("do", stage)
            yield ("arrive", f"DSEmpty{w}")

    roles = {"producer": producer(), "mma": mma(), "provider": provider(), "ew0": elementwise(0),
             "ew1": elementwise(1)}
    for wi in range(4):
        roles[f"dq{wi}"] = dq_warp(wi)
    sim.run(roles)


# ------------------------------------------------------------------ forward, two tiles
def forward2(nkt0: int, nkt1: int, seed: int, stages: int = 2, rescale_p: float = 0.5,
             plant: str | None = None, slow_tma: bool = False, pair: bool = False):
    """fa_fwd2_sm100_kernel: two query tiles per CTA, one S buffer and one O
    accumulator per tile, one K/V ring both tiles read.  Per key tile j the MMA
    warp waits V_j (and K_{j+1}), then per tile t: PFull_t(j) -> PV_t(j),
    OStep_t, and S_t(j+1) behind it (same TMEM columns as P_t(j)) or OFinal_t;
    KVEmpty_j once both tiles' MMAs of step j are issued.  With a causal mask
    the second tile has one key tile more (nkt1 = nkt0 + 1).  With a pair bias
    the pair tiles of (tile t, key tile j) go through one 3-slot ring in score
    order (j major, t minor): the producer loads those of key tile j + 1 after
    K/V_j, the u-th into slot u % 3 once PairEmpty says the score MMA of tile
    u - 3 retired; the MMA warp waits PairFull before each score."""
    sim = _Sim(seed, slow_tma)
    S = stages
    nkt = [nkt0, nkt1]
    n_kt = max(nkt)
    order = [(t, j) for j in range(n_kt) for t in range(2) if j < nkt[t]]   # pair tile u
    sim.bar("QFull")
    sim.bar("MmaDone")
    for slot in range(3):
        sim.bar(f"PairFull{slot}")
        sim.bar(f"PairEmpty{slot}")
    for s in range(S):
        for n in ("KFull", "VFull", "KVEmpty"):
            sim.bar(f"{n}{s}")
    for t in range(2):
        for n in ("SFull", "PFull", "OStep", "OFinal"):
            sim.bar(f"{n}{t}")
    o = {0: 0, 1: 0}

    def producer():
        yield ("do", lambda: None)
        if n_kt == 0:
            return
        sim.asyncs.append((lambda: sim.mem.__setitem__("Q", "q"), "QFull"))
        issued = {"u": 0}

        def load_pairs(j):
            for t in range(2):
                if j >= nkt[t]:
                    continue
                u = issued["u"]
                slot = u % 3
                if u >= 3:
                    yield _wait(plant, f"PairEmpty{slot}", u // 3 - 1)

                def land(u=u, slot=slot):
                    if u >= 3 and ("S",) + order[u - 3] not in sim.executed:
                        raise ProtocolBug(f"pair slot {slot} reloaded before S{order[u - 3]} read it")
                    sim.mem[f"pair{slot}"] = order[u]
                sim.asyncs.append((land, f"PairFull{slot}"))
                issued["u"] = u + 1
        if pair:
            yield from load_pairs(0)
        for j in range(n_kt):
            s = j % S
            if j >= S:
                yield _wait(plant, f"KVEmpty{s}", j // S - 1)

            def land_k(j=j, s=s):
                if j >= S and any(("S", t, j - S + 1) not in sim.executed for t in range(2) if j - S + 1 < nkt[t]):
                    raise ProtocolBug(f"K stage {s} reloaded before S(j={j - S + 1}) read it")
                sim.mem[f"K{s}"] = j

            def land_v(j=j, s=s):
                if j >= S and any(("PV", t, j - S) not in sim.executed for t in range(2) if j - S < nkt[t]):
                    raise ProtocolBug(f"V stage {s} reloaded before PV({j - S}) read it")
                sim.mem[f"V{s}"] = j
            sim.asyncs.append((land_k, f"KFull{s}"))
            sim.asyncs.append((land_v, f"VFull{s}"))
            if pair and j + 1 < n_kt:
                yield from load_pairs(j + 1)

    def mma():
        if n_kt == 0:
            yield ("do", lambda: None)
            return
        yield ("wait", "QFull", 0)
        used = {"u": 0}

        def pair_ready():
            if pair:
                u = used["u"]
                yield _wait(plant, f"PairFull{u % 3}", u // 3)

        def issue_s(t, j):
            u = used["u"]

            def run(t=t, j=j, u=u):
                sim.expect("Q", "q")
                sim.expect(f"K{j % S}", j)
                if pair:
                    sim.expect(f"pair{u % 3}", (t, j))
                if j > 0 and ("PV", t, j - 1) not in sim.executed:
                    raise ProtocolBug(f"S_{t}({j}) overwrites P_{t}({j - 1}) before PV read it")
                sim.mem[f"S{t}"] = ("S", j)
            sim.mma(("S", t, j), run)
            if pair:
                sim.commit(f"PairEmpty{u % 3}")
                used["u"] = u + 1
            sim.commit(f"SFull{t}")

        yield _wait(plant, "KFull0", 0)
        for t in range(2):
            if nkt[t] > 0:
                yield from pair_ready()
                issue_s(t, 0)
        for j in range(n_kt):
            s = j % S
            yield _wait(plant, f"VFull{s}", j // S)
            if j + 1 < n_kt:
                yield _wait(plant, f"KFull{(j + 1) % S}", (j + 1) // S)
            for t in range(2):
                if j >= nkt[t]:
                    continue
                yield _wait(plant, f"PFull{t}", j)
                if j + 1 < nkt[t]:
                    yield from pair_ready()

                def pv(t=t, j=j, s=s):
                    sim.expect(f"S{t}", ("P", j))
                    sim.expect(f"V{s}", j)
                    if o[t] != j:
                        raise ProtocolBug(f"O_{t} holds {o[t]} products at PV({j})")
                    o[t] += 1
                sim.mma(("PV", t, j), pv)
                sim.commit(f"OStep{t}")
                if j == nkt[t] - 1:
                    sim.commit(f"OFinal{t}")
                else:
                    issue_s(t, j + 1)
            sim.commit(f"KVEmpty{s}")
        sim.commit("MmaDone")
        yield ("wait", "MmaDone", 0)

    def softmax(t):
        yield ("do", lambda: None)
        for j in range(nkt[t]):
            yield _wait(plant, f"SFull{t}", j)

            def sm(t=t, j=j):
                sim.expect(f"S{t}", ("S", j))
                sim.mem[f"S{t}"] = ("P", j)
            yield ("do", sm)
            if j > 0 and sim.rng.random() < rescale_p:
                yield _wait(plant, f"OStep{t}", j - 1)

                def resc(t=t, j=j):
                    if o[t] != j:
                        raise ProtocolBug(f"O_{t} rescaled with {o[t]} products at key tile {j}")
                yield ("do", resc)
            yield ("arrive", f"PFull{t}")
        if nkt[t]:
            yield _wait(plant, f"OFinal{t}", 0)

            def fin(t=t):
                if o[t] != nkt[t]:
                    raise ProtocolBug(f"O_{t} read with {o[t]} of {nkt[t]} products")
            yield ("do", fin)

    sim.run({"producer": producer(), "mma": mma(), "sm0": softmax(0), "sm1": softmax(1)})
