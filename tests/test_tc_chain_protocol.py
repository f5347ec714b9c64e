"""CPU model of the mbarrier protocol of the tcgen05 chain kernel
(fastaf_kernel_b200/csrc/gdn_prefill_tc.cu), run under random schedules.

The kernel hands every chunk between six roles -- the MMA-issuing thread, the copy
thread, four prep warps, eight state warps and four output-store warps -- through
mbarriers only (no block-wide barrier in the chunk loop).  The model runs each warp as a coroutine that follows the
kernel's waits, reads, writes and arrives in the kernel's order; MMA batches and
copies are asynchronous events.  The tensor pipe is in order (tcgen05.mma and
tcgen05.commit issued by one thread complete in issue order, a commit arriving once
every earlier MMA is done); copies land in any order and complete their barrier's
transaction count.

Each schedule checks:
  * no deadlock: every role finishes and every asynchronous operation completes;
  * every parity wait on the k-th completion of a barrier is evaluated while the
    barrier has completed k or k + 1 phases (k - 1 would pass early on the previous
    phase of the same parity; k + 2 would have lapped it);
  * every read sees the chunk and stage of the data it expects (buffers carry tags);
  * no warp writes a buffer, and no copy is issued into one, while an asynchronous
    operation that reads or writes it is in flight; no MMA batch is issued on an
    operand whose copy is still in flight.
Buffers: shared-memory stages (K, Q, V, P, gates) x 2, the T' and T'' tiles, -W hi/lo
and (Gamma Q)^T (per TMEM lane quadrant of the warp that writes them); TMEM S (per
state half and quadrant), the [128, 256) hi/lo/delta region in 16-column blocks,
W^T, [U | X] and O^T (per quadrant); the output staging tile (per column block, written
by the prep warp of that TMEM lane quadrant and read by every store warp).

The kernel's barrier counts are read from the source and compared with the model's.
Planted protocol mistakes (a missing condition or wait) must be caught.

The give-up path is modelled too: with `timeouts` on, any wait whose barrier is not
complete may run out (the role raises the shared abort flag and stops), and once the
flag is up every wait that is not yet satisfied returns false.  The issuing thread
then waits for the last commit of every batch kind it issued and the copy thread for
every copy it issued; the schedule must end with every role finished and no MMA or
copy still in flight (the CTA frees TMEM and exits after the last role).
"""
import os
import random
import re

import pytest

KERNEL = os.path.join(os.path.dirname(__file__), "..", "fastaf_kernel_b200", "csrc", "gdn_prefill_tc.cu")


class ProtocolError(AssertionError):
    pass


class Bar:
    """mbarrier: `count` arrivals plus a transaction byte count per phase."""

    def __init__(self, name, count):
        self.name, self.count = name, count
        self.pending, self.tx, self.done = count, 0, 0

    def _complete(self):
        if self.pending == 0 and self.tx == 0:
            self.done += 1
            self.pending = self.count

    def arrive(self, tx=0):
        self.tx += tx
        self.pending -= 1
        self._complete()

    def complete_tx(self, n):
        self.tx -= n
        self._complete()

    def test(self, k, where):
        """Hardware parity test for the k-th completion (0-based), with the invariant."""
        p = self.done
        if p < k or p > k + 1:
            raise ProtocolError(f"{where}: wait for completion {k} of {self.name} evaluated after {p}")
        return (p & 1) != (k & 1)


class Sim:
    def __init__(self, nch, plant=None):
        self.nch, self.plant = nch, plant
        self.abort = False
        self.tags = {}
        self.copy_w = {}      # part -> in-flight copies writing it
        self.mma_r = {}       # part -> in-flight MMA batches reading it
        self.mma_w = {}       # part -> in-flight MMA batches writing it
        self.pipe = []        # in-order tensor pipe: ("mma", reads, writes) / ("commit", bar)
        self.copies = []      # in-flight copies: (part, tag, bar)
        counts = dict(tma0=1, tma1=1, wdone=1, udone=1, d=1, s=1, qs=4, w=4, ss=8, ds=8, tw=1, tu=1,
                      free0=1, free1=1, oread=4, ofull=4, ofree=4)
        self.counts = counts
        self.b = {k: Bar(k, v) for k, v in counts.items()}

    # ---------------------------------------------------------------- data
    @staticmethod
    def _inc(d, p):
        d[p] = d.get(p, 0) + 1

    @staticmethod
    def _dec(d, p):
        d[p] -= 1

    def read(self, part, tag, who):
        if self.copy_w.get(part) or self.mma_w.get(part):
            raise ProtocolError(f"{who} reads {part} while an async write of it is in flight")
        if self.tags.get(part) != tag:
            raise ProtocolError(f"{who} reads {part}: holds {self.tags.get(part)}, expected {tag}")

    def write(self, part, tag, who):
        if self.copy_w.get(part) or self.mma_w.get(part) or self.mma_r.get(part):
            raise ProtocolError(f"{who} writes {part} while an async access of it is in flight")
        self.tags[part] = tag

    def mma(self, reads, writes, who):
        """reads: {part: tag}; writes: {part: (expected previous tag or None, new tag)}."""
        for p in list(reads) + list(writes):
            if self.copy_w.get(p):
                raise ProtocolError(f"{who} issued while the copy of {p} is in flight")
        for p in reads:
            self._inc(self.mma_r, p)
        for p in writes:
            self._inc(self.mma_w, p)
        self.pipe.append(("mma", reads, writes, who))

    def commit(self, bar):
        self.pipe.append(("commit", self.b[bar]))

    def copy(self, parts, tag, bar, who):
        b = self.b[bar]
        b.arrive(tx=len(parts))
        for p in parts:
            if self.copy_w.get(p) or self.mma_r.get(p) or self.mma_w.get(p):
                raise ProtocolError(f"{who}: copy into {p} while an async access of it is in flight")
            self._inc(self.copy_w, p)
            self.copies.append((p, tag, b))

    def retire_pipe(self):
        e = self.pipe.pop(0)
        if e[0] == "commit":
            e[1].arrive()
            return
        _, reads, writes, who = e
        for p, t in reads.items():
            if self.tags.get(p) != t:
                raise ProtocolError(f"{who} executes on {p} = {self.tags.get(p)}, expected {t}")
        for p, (prev, t) in writes.items():
            if prev is not None and self.tags.get(p) != prev:
                raise ProtocolError(f"{who} accumulates into {p} = {self.tags.get(p)}, expected {prev}")
        for p in reads:
            self._dec(self.mma_r, p)
        for p, (_, t) in writes.items():
            self._dec(self.mma_w, p)
            self.tags[p] = t

    def retire_copy(self, i):
        p, tag, b = self.copies.pop(i)
        self._dec(self.copy_w, p)
        self.tags[p] = tag
        b.complete_tx(1)


Q4 = range(4)


def _stage(st):
    return [(x, st) for x in ("K", "Q", "V", "P", "G")]


def _r(blocks, tag):
    return {("R", bl, q): tag for bl in blocks for q in Q4}


# ------------------------------------------------------------------ MMA batches
def mma6w(sim, c):   # W^T = K^T T''^T
    st = c & 1
    sim.mma({("K", st): c, ("T2",): c}, {("W", q): (None, c) for q in Q4}, f"W^T({c})")
    sim.commit("wdone")


def mma6u(sim, c):   # [U | X] = V^T [T'_hi | T'_lo]^T
    st = c & 1
    sim.mma({("V", st): c, ("T1",): c}, {("UX", q): (None, ("u", c)) for q in Q4}, f"U({c})")
    sim.commit("udone")


def _delta_b_operands(c):
    return {**{("WH", q): c for q in Q4}, **{("WL", q): c for q in Q4}, **{("QS", q): c for q in Q4}}


def mma8(sim, c):    # [U | X | O] += S_hi [-W_hi | -W_lo | Gamma Q]^T; U += S_lo (-W_hi)^T
    reads = {**_r(range(8), ("Ssplit", c)), **_delta_b_operands(c)}
    writes = {**{("UX", q): (("u", c), ("delta", c)) for q in Q4},
              **{("O", q): (("zero", c), ("qs", c)) for q in Q4}}
    sim.mma(reads, writes, f"delta({c})")
    sim.commit("d")


def mma10(sim, c):   # S += delta'^T K, O^T += delta^T P^T
    st = c & 1
    reads = {**_r(range(6), ("dsplit", c)), ("K", st): c, ("P", st): c}
    writes = {**{("S", hs, q): (("Sdec", c), ("S", c + 1)) for hs in (0, 1) for q in Q4},
              **{("O", q): (("qs", c), ("out", c)) for q in Q4}}
    sim.mma(reads, writes, f"S update({c})")
    sim.commit("s")
    sim.commit(f"free{st}")


# ------------------------------------------------------------------ roles
# A role yields ("wait", bar, k) for a bounded, abort-aware wait (it receives True, or
# False once it gave up or saw the abort flag), ("drain", bar, k) for a wait on its own
# asynchronous work (always satisfied in the end), ("wait_forever", bar, k) for a planted
# wait without the abort check, "spin" for a probe round of the issuing thread, or None to
# let others run.
def issuer(sim):
    b, nch, plant = sim.b, sim.nch, sim.plant
    n6w = n6u = n8 = n10 = 0
    while n10 < nch:
        progress = False
        if n10 < n8 and b["ds"].test(n10, "issue S update"):
            mma10(sim, n10)
            n10 += 1
            progress = True
        if (n8 < n6u and b["ss"].test(n8, "issue delta") and b["w"].test(n8, "issue delta")
              and b["qs"].test(n8, "issue delta")
              and (n8 == 0 or plant == "no_oread" or b["oread"].test(n8 - 1, "issue delta"))):
            mma8(sim, n8)
            n8 += 1
            progress = True
        if (n6w < nch and (n6w <= n8 or plant == "w_early") and b["tw"].test(n6w, "issue W")
                and b[f"tma{n6w & 1}"].test(n6w >> 1, "issue W")):
            mma6w(sim, n6w)
            n6w += 1
            progress = True
        if n6u < n6w and (n6u <= n10 or plant == "u_early") and b["tu"].test(n6u, "issue U"):
            mma6u(sim, n6u)
            n6u += 1
            progress = True
        sim.progress = progress
        if not progress and sim.abort:
            break                                   # (the idle bookkeeping sees the flag)
        if not progress and sim.timeouts and sim.rng.random() < 0.01:
            sim.abort = True                        # the idle timer ran out
            break
        yield "spin"
    for bar, n in (("wdone", n6w), ("udone", n6u), ("d", n8), ("s", n10)):
        if n:
            yield ("drain", bar, n - 1)
    for c in range(max(0, n10 - 2), n10):
        yield ("drain", f"free{c & 1}", c >> 1)


def copier(sim):
    issued = n_tw = n_tu = 0
    failed = False
    for c in range(sim.nch):
        st = c & 1
        if c >= 1 and not (yield ("wait", "wdone", c - 1)):
            failed = True
            break
        sim.copy([("T2",)], c, "tw", f"copy T''({c})")
        n_tw += 1
        if c >= 2 and sim.plant != "no_free_wait" and not (yield ("wait", f"free{st}", (c - 2) >> 1)):
            failed = True
            break
        sim.copy(_stage(st), c, f"tma{st}", f"copy stage({c})")
        issued += 1
        if c >= 1 and not (yield ("wait", "udone", c - 1)):
            failed = True
            break
        sim.copy([("T1",)], c, "tu", f"copy T'({c})")
        n_tu += 1
        yield None
    if sim.plant == "copy_drain_on_own_failure_only" and not failed:
        return
    for cc in range(max(0, issued - 2), issued):
        yield ("drain", f"tma{cc & 1}", cc >> 1)
    if n_tw:
        yield ("drain", "tw", n_tw - 1)
    if n_tu:
        yield ("drain", "tu", n_tu - 1)


def prep(sim, q):
    who = f"prep{q}"
    out_bar = "s"

    def write_out(c):
        sim.read(("O", q), ("out", c), who)
        yield None
        sim.write(("O", q), ("zero", c + 1), who)
        sim.b["oread"].arrive()
        if c > 0 and sim.plant != "no_ofree_wait" and not (yield ("wait", "ofree", c - 1)):
            return False
        yield None                                  # bf16 rows into the staging tile
        sim.write(("STG", q), ("out", c), who)
        yield None
        sim.b["ofull"].arrive()
        return True

    for c in range(sim.nch):
        st = c & 1
        if not (yield ("wait", f"tma{st}", c >> 1)):
            break
        if c > 0 and not (yield ("wait", "d", c - 1)):
            break
        sim.read(("G", st), c, who)
        sim.read(("Q", st), c, who)
        yield None
        sim.write(("QS", q), c, who)
        if c == 0:
            sim.write(("O", q), ("zero", 0), who)
        yield None
        sim.b["qs"].arrive()
        if not (yield ("wait", "wdone", c)):
            break
        sim.read(("W", q), c, who)
        yield None
        sim.write(("WH", q), c, who)
        sim.write(("WL", q), c, who)
        yield None
        sim.b["w"].arrive()
        if c > 0:
            if not (yield ("wait", out_bar, c - 1)):
                break
            if not (yield from write_out(c - 1)):
                break
    if not sim.abort and sim.nch and (yield ("wait", out_bar, sim.nch - 1)):
        yield from write_out(sim.nch - 1)


def store(sim, sw):
    who = f"store{sw}"
    handoff = "wait_forever" if sim.plant == "unbounded_handoff" else "wait"
    for c in range(sim.nch):
        yield None                                  # gate rows of chunk c into registers
        if not (yield (handoff, "ofull", c)):
            break
        for q in Q4:                                # the loop over the chunk's rows reads the
            sim.read(("STG", q), ("out", c), who)   # tile from its first step to its last
        yield None                                  # (gated) rows to global
        yield None
        for q in Q4:
            sim.read(("STG", q), ("out", c), who)
        sim.b["ofree"].arrive()


def state(sim, hs, q):
    who = f"state{hs}.{q}"
    split_blocks = (2 * hs, 2 * hs + 1, 4 + 2 * hs, 5 + 2 * hs)
    delta_blocks = (hs, 2 + hs, 4 + hs)
    s_bar, ss_bar = "s", "ss"
    sim.write(("S", hs, q), ("S", 0), who)
    yield None
    ok = True
    for c in range(sim.nch):
        st = c & 1
        if c > 0 and not (ok := (yield ("wait", s_bar, c - 1))):
            break
        if not (ok := (yield ("wait", f"tma{st}", c >> 1))):
            break
        sim.read(("G", st), c, who)
        sim.read(("S", hs, q), ("S", c), who)
        yield None
        for bl in split_blocks:
            sim.write(("R", bl, q), ("Ssplit", c), who)
        sim.write(("S", hs, q), ("Sdec", c), who)
        yield None
        sim.b[ss_bar].arrive()
        if not (ok := (yield ("wait", "d", c))):
            break
        sim.read(("UX", q), ("delta", c), who)
        sim.read(("G", st), c, who)
        yield None
        for bl in delta_blocks:
            sim.write(("R", bl, q), ("dsplit", c), who)
        yield None
        sim.b["ds"].arrive()
    if ok and sim.nch and (yield ("wait", "s", sim.nch - 1)):
        sim.read(("S", hs, q), ("S", sim.nch), who)


def run(nch, seed, plant=None, max_steps=400000, timeouts=False):
    sim = Sim(nch, plant)
    rng = random.Random(seed)
    sim.rng, sim.timeouts = rng, timeouts
    roles = {"issuer": issuer(sim), "copier": copier(sim)}
    roles.update({f"prep{q}": prep(sim, q) for q in Q4})
    roles.update({f"state{hs}.{q}": state(sim, hs, q) for hs in (0, 1) for q in Q4})
    roles.update({f"store{sw}": store(sim, sw) for sw in Q4})
    waiting = {}    # role -> (kind, bar, k)
    done = set()

    def step(name, value=None):
        try:
            r = roles[name].send(value)
        except StopIteration:
            done.add(name)
            return
        if isinstance(r, tuple):
            waiting[name] = r

    for name in roles:      # start every coroutine (up to its first yield)
        step(name)
    for _ in range(max_steps):
        live = [n for n in roles if n not in done]
        if not live:
            if sim.pipe or sim.copies:
                raise ProtocolError(f"CTA exits with {len(sim.pipe)} MMA entries and {len(sim.copies)} "
                                    "copies in flight")
            return sim
        ready = []
        for n in live:
            if n == "issuer" and n not in waiting:
                continue
            if n in waiting:
                kind, bar, k = waiting[n]
                if sim.b[bar].test(k, n):
                    ready.append(("role", n, True))
                elif kind == "wait" and (sim.abort or (timeouts and rng.random() < 0.002)):
                    ready.append(("role", n, False))
                continue
            ready.append(("role", n, None))
        if sim.pipe:
            ready.append(("pipe", None, None))
        ready += [("copy", i, None) for i in range(len(sim.copies))]
        spinning = "issuer" in live and "issuer" not in waiting
        if not ready and not spinning:
            raise ProtocolError(f"deadlock: waiting {waiting}")
        if spinning and (not ready or rng.random() < 0.3):
            step("issuer")
            if (not ready and not sim.progress and "issuer" not in done and "issuer" not in waiting
                    and not sim.timeouts):
                raise ProtocolError(f"deadlock (issuer idle): waiting {waiting}")
            continue
        kind, x, val = ready[rng.randrange(len(ready))]
        if kind == "pipe":
            sim.retire_pipe()
        elif kind == "copy":
            sim.retire_copy(x)
        else:
            if val is False and not sim.abort:
                sim.abort = True        # this wait ran out: raise the flag
            waiting.pop(x, None)
            step(x, val)
    raise ProtocolError("schedule did not finish")


CHUNKS = [1, 2, 3, 4, 5, 8, 17]


@pytest.mark.parametrize("nch", CHUNKS)
def test_protocol_random_schedules(nch):
    for seed in range(60):
        sim = run(nch, 1000 * nch + seed)
        for hs in (0, 1):
            for q in Q4:
                assert sim.tags[("S", hs, q)] == ("S", nch)


@pytest.mark.parametrize("plant", ["w_early", "u_early", "no_free_wait", "no_oread", "no_ofree_wait"])
def test_planted_protocol_mistakes_are_caught(plant):
    with pytest.raises(ProtocolError):
        for seed in range(200):
            run(5, seed, plant)


@pytest.mark.parametrize("nch", [1, 2, 3, 5, 9])
def test_give_up_path_terminates_with_nothing_in_flight(nch):
    """Random waits run out: every role still finishes, nothing deadlocks, and no MMA
    or copy is in flight when the CTA exits; some schedules give up early, some late."""
    aborted = 0
    for seed in range(150):
        sim = run(nch, 7000 * nch + seed, timeouts=True)
        aborted += sim.abort
    assert aborted > 30


@pytest.mark.parametrize("plant,nch,seeds", [("unbounded_handoff", 4, 400),
                                              ("copy_drain_on_own_failure_only", 1, 2000)])
def test_planted_give_up_mistakes_are_caught(plant, nch, seeds):
    """A staging hand-off that cannot give up (a wait without the abort check) deadlocks
    once a prep warp stopped; a copy thread that drains only after its own wait failed
    leaves copies in flight when another role gave up."""
    with pytest.raises(ProtocolError):
        for seed in range(seeds):
            run(nch, 31000 + seed, plant, timeouts=True)


def test_barrier_counts_match_the_kernel():
    """The kernel's mbar_init counts equal the model's."""
    src = open(KERNEL).read()
    consts = {k: int(v) for k, v in re.findall(r"constexpr int (k\w+) = (\d+);", src)}
    inits = {name[2:]: int(n) if n.isdigit() else consts[n]
             for name, n in re.findall(r"mbar_init\((b_\w+), (\w+)\)", src)}
    assert inits == Sim(1).counts
