"""CPU: randomised models of the tensor-core kernels' mbarrier protocols —
fa_fwd_tc_kernel (llm-runner_b200/csrc/fa_tc.cuh), the two wide-head kernels
(fa_wide.cuh, checked against these models before their first GPU run), the
QKV projection's CTA-pair GEMM (qkv_proj.cuh) and the exact fp32 kernel on
the tensor cores (exact_tc.cuh, checked before its first GPU run).

Each model runs the kernel's roles as coroutines under a random scheduler
with random stalls: the TMA producer(s), the MMA-issuing warp, the softmax
warps, an in-order MMA pipe (MMAs and tcgen05.commit arrivals in issue
order) and a TMA engine that completes loads in any order. It checks that
every mbarrier wait observes the phase it means (a parity wait is only
unambiguous while the barrier is at most one phase ahead of it), that
nothing deadlocks, and the data hazards the barriers exist for: a ring slot
reloaded before its MMAs ran, Q replaced before the unit's last S MMA, S
overwriting an unread S or an unconsumed P, P read before it was written, O
rescaled while a P.V MMA may still write it, O overwritten before the
epilogue read it. The models follow the kernels' schedules as written; a
change to a kernel's barrier protocol must be made here too.
"""
import random

import pytest


class Bar:
    """An mbarrier with `count` arrivals per phase; c = phases completed."""

    def __init__(self, name, count):
        self.name, self.count, self.pending, self.c = name, count, 0, 0

    def arrive(self):
        self.pending += 1
        assert self.pending <= self.count, self.name
        if self.pending == self.count:
            self.pending = 0
            self.c += 1


class Fail(Exception):
    pass


def wait(bar, intended):
    """Generator: waits until phase `intended` of bar has completed, checking
    that the parity test is unambiguous at every poll."""
    parity = intended & 1
    while True:
        if not (bar.c == intended or bar.c == intended + 1):
            raise Fail(f"aliasing on {bar.name}: count {bar.c}, intended {intended}")
        if (bar.c & 1) != parity:
            return
        yield False


class TxBar:
    """An mbarrier with a transaction count: a phase completes when its
    arrivals are in and the bytes armed with them have landed; bytes that
    belong to a later phase are an error."""

    def __init__(self, name, count):
        self.name, self.count, self.pending, self.c, self.tx = name, count, 0, 0, 0

    def _check(self):
        if self.pending == self.count and self.tx == 0:
            self.pending = 0
            self.c += 1

    def arrive(self, expect=0):
        self.pending += 1
        self.tx += expect
        if self.pending > self.count:
            raise Fail(f"{self.name}: too many arrivals")
        self._check()

    def complete_tx(self, n, phase):
        if phase != self.c:
            raise Fail(f"{self.name}: bytes of phase {phase} land in phase {self.c}")
        self.tx -= n
        self._check()


def run_single(seed, QCH, VCH, NST, nblk, units, p_rescale, per_buffer_p=True,
               pv_wait_every_block=True):
    """fa_wide_tc_kernel: QCH K chunks and VCH V chunks per key block through an
    NST-slot ring; per_buffer_p / pv_wait_every_block are the kernel's choices
    (False plants the protocol bug each one prevents)."""
    rng = random.Random(seed)
    bars = {}

    def B(name, count=1):
        if name not in bars:
            bars[name] = Bar(name, count)
        return bars[name]

    q_full, q_empty = B("q_full"), B("q_empty")
    kv_full = [B(f"kv_full{i}") for i in range(NST)]
    kv_empty = [B(f"kv_empty{i}") for i in range(NST)]
    s_full = [B(f"s_full{b}") for b in range(2)]
    p_half = [B(f"p_half{i}", 4) for i in range(4)]
    pv_done, o_full, o_empty = B("pv_done"), B("o_full"), B("o_empty", 4)

    # state
    slot_tag = [None] * NST
    slot_consumed = [True] * NST
    q_tag = None
    s_exec = {}            # (unit) -> number of S chunk MMAs executed
    tma_q = []             # outstanding loads: (kind, tag, slot, bar)
    q_pending = {}         # Q loads outstanding per unit
    mma_q = []             # issued MMA-pipe ops in order
    # TMEM per warp: S buffer content tag, P halves written, O state
    sbuf = [[None, None] for _ in range(4)]      # ('S', jj, chunks) / ('P', jj, halves)
    o_state = {"last_pv": None, "epi_read": set(), "unit": None}
    pv_exec = set()         # (jj, half, c) executed
    done_flags = {}

    jb_of_unit = [u * nblk for u in range(units)]

    # -------------------------------------------------------------- producer
    def producer():
        nonlocal q_tag
        pos = 0
        for k in range(units):
            if k > 0:
                yield from wait(q_empty, k - 1)
            q_pending[k] = QCH
            for c in range(QCH):
                tma_q.append(("Q", (k, c), None, q_full))
            yield True
            for i in range(nblk + 1):
                seq = []
                if i < nblk:
                    seq += [("K", (k, i, c)) for c in range(QCH)]
                if i >= 1:
                    seq += [("V", (k, i - 1, c)) for c in range(VCH)]
                for kind, tag in seq:
                    slot, rnd = pos % NST, pos // NST
                    if rnd > 0:
                        yield from wait(kv_empty[slot], rnd - 1)
                    tma_q.append((kind, tag, slot, kv_full[slot]))
                    pos += 1
                    yield True
        done_flags["producer"] = True

    # ----------------------------------------------------------- MMA warp
    def mma_warp():
        pos = 0
        jb = 0

        def issue_s(k, jj, j):
            nonlocal pos
            for c in range(QCH):
                slot = pos % NST
                yield from wait(kv_full[slot], pos // NST)
                mma_q.append(("S", (k, jj, j, c, slot)))
                mma_q.append(("commit", kv_empty[slot]))
                pos += 1
                yield True
            mma_q.append(("commit", s_full[jj & 1]))

        def issue_pv(k, jj, j):
            nonlocal pos
            base = pos
            for c in range(VCH):
                u = base + c
                yield from wait(kv_full[u % NST], u // NST)
            for half in range(2):
                if per_buffer_p:
                    yield from wait(p_half[2 * (jj & 1) + half], jj >> 1)
                else:
                    yield from wait(p_half[half], jj)
                for c in range(VCH):
                    mma_q.append(("PV", (k, jj, j, half, c, (base + c) % NST)))
                yield True
            for c in range(VCH):
                mma_q.append(("commit", kv_empty[(base + c) % NST]))
            pos += VCH

        for k in range(units):
            yield from wait(q_full, k)
            yield from issue_s(k, jb, 0)
            if nblk > 1:
                yield from issue_s(k, jb + 1, 1)
            if nblk <= 2:
                mma_q.append(("commit", q_empty))
            for j in range(nblk):
                jj = jb + j
                if j == 0 and k > 0:
                    yield from wait(o_empty, k - 1)
                yield from issue_pv(k, jj, j)
                mma_q.append(("commit", pv_done))
                if j + 2 < nblk:
                    yield from issue_s(k, jj + 2, j + 2)
                    if j + 3 == nblk:
                        mma_q.append(("commit", q_empty))
            mma_q.append(("commit", o_full))
            jb += nblk
        done_flags["mma"] = True

    # ------------------------------------------------------------- softmax
    def softmax(w):
        jb = 0
        for k in range(units):
            for j in range(nblk):
                jj = jb + j
                yield from wait(s_full[jj & 1], jj >> 1)
                tag = sbuf[w][jj & 1]
                if tag != ("S", jj, QCH):
                    raise Fail(f"warp {w} reads S buffer {jj & 1} = {tag}, want S_{jj}")
                yield True
                need = j == 0 or rng.random() < p_rescale
                if jj > 0 and pv_wait_every_block:
                    yield from wait(pv_done, jj - 1)
                if need and j > 0 and not pv_wait_every_block:
                    yield from wait(pv_done, jj - 1)
                if need and j > 0:
                    # O must be quiescent and hold PV up to block jj-1
                    if o_state["last_pv"] != (jj - 1, 1, VCH - 1):
                        raise Fail(f"rescale at {jj}: O last written by {o_state['last_pv']}")
                    yield True
                # P halves
                for half in range(2):
                    st = sbuf[w][jj & 1]
                    sbuf[w][jj & 1] = ("P", jj, half + 1)
                    (p_half[2 * (jj & 1) + half] if per_buffer_p else p_half[half]).arrive()
                    yield True
            jb += nblk
            yield from wait(o_full, k)
            last = jb - 1
            if o_state["last_pv"] != (last, 1, VCH - 1):
                raise Fail(f"epilogue of unit {k}: O last written by {o_state['last_pv']}")
            yield True
            o_state["epi_read"].add((k, w))
            o_empty.arrive()
            yield True
        done_flags[f"softmax{w}"] = True

    # ---------------------------------------------------------- MMA pipe
    def mma_pipe_step():
        nonlocal q_tag
        if not mma_q:
            return False
        op, a = mma_q.pop(0)
        if op == "commit":
            a.arrive()
            return True
        if op == "S":
            k, jj, j, c, slot = a
            if q_tag != k:
                raise Fail(f"S_{jj} reads Q of unit {q_tag}, want {k}")
            if slot_tag[slot] != ("K", (k, j, c)):
                raise Fail(f"S_{jj} chunk {c} reads slot {slot} = {slot_tag[slot]}")
            for w in range(4):
                cur = sbuf[w][jj & 1]
                if c == 0:
                    # overwriting: previous content must be P_{jj-2} consumed
                    if cur is not None and cur[0] == "P":
                        pj = cur[1]
                        if not all((pj, h, cc) in pv_exec for h in range(2) for cc in range(VCH)):
                            raise Fail(f"S_{jj} overwrites P_{pj} before PV_{pj}")
                    if cur is not None and cur[0] == "S":
                        raise Fail(f"S_{jj} overwrites unread S_{cur[1]}")
                    sbuf[w][jj & 1] = ("S", jj, 1)
                else:
                    assert cur == ("S", jj, c), cur
                    sbuf[w][jj & 1] = ("S", jj, c + 1)
            slot_consumed[slot] = True
            s_exec[k] = s_exec.get(k, 0) + 1
            return True
        if op == "PV":
            k, jj, j, half, c, slot = a
            for w in range(4):
                cur = sbuf[w][jj & 1]
                if not (cur is not None and cur[0] == "P" and cur[1] == jj and cur[2] >= half + 1):
                    raise Fail(f"PV_{jj} half {half} reads {cur} (warp {w})")
            if slot_tag[slot] != ("V", (k, j, c)):
                raise Fail(f"PV_{jj} reads slot {slot} = {slot_tag[slot]}")
            if j == 0 and half == 0:
                if k > 0 and not all((k - 1, w) in o_state["epi_read"] for w in range(4)):
                    raise Fail(f"unit {k} PV_0 overwrites O before the epilogue read it")
            o_state["last_pv"] = (jj, half, c)
            pv_exec.add((jj, half, c))
            if half == 1:
                slot_consumed[slot] = True
            return True
        raise AssertionError(op)

    # ---------------------------------------------------------- TMA engine
    def tma_step():
        nonlocal q_tag
        if not tma_q:
            return False
        i = rng.randrange(len(tma_q))
        kind, tag, slot, bar = tma_q.pop(i)
        if kind == "Q":
            k, c = tag
            if k > 0 and s_exec.get(k - 1, 0) != nblk * QCH:
                raise Fail(f"Q of unit {k} lands before unit {k-1}'s S MMAs ran")
            q_pending[k] -= 1
            if q_pending[k] == 0:
                q_tag = k
                bar.arrive()
            return True
        if not slot_consumed[slot]:
            raise Fail(f"load {tag} overwrites slot {slot} ({slot_tag[slot]}) before use")
        slot_tag[slot] = (kind, tag)
        slot_consumed[slot] = False
        bar.arrive()
        return True

    actors = {"producer": producer(), "mma": mma_warp()}
    for w in range(4):
        actors[f"softmax{w}"] = softmax(w)
    live = dict(actors)
    sleep = {}
    idle = 0
    steps = 0
    while True:
        steps += 1
        if steps > 5_000_000:
            raise Fail("too many steps")
        if not live and not mma_q and not tma_q:
            return steps
        names = list(live.keys()) + ["pipe", "tma"]
        ch = rng.choice(names)
        if sleep.get(ch, 0) > steps:
            continue
        if rng.random() < 0.01:
            # a long stall of this actor (other warps' issue, memory latency)
            sleep[ch] = steps + rng.randint(1, 400)
            continue
        if ch == "pipe":
            progressed = mma_pipe_step()
        elif ch == "tma":
            progressed = tma_step()
        else:
            try:
                progressed = bool(next(live[ch]))
            except StopIteration:
                del live[ch]
                progressed = True
        idle = 0 if progressed else idle + 1
        if idle > 20000:
            raise Fail(f"deadlock; live={list(live)} mma_q={mma_q[:3]} tma_q={tma_q[:3]}")



def run_pair(seed, QCH, NSTK, NSTV, nblk, units, p_rescale, odd_waits_its_slots=True):
    """fa_wide_pair_kernel: both CTAs' producers (their bytes complete on the
    even CTA's barriers), the even CTA's MMA warp, 8 softmax warps.
    odd_waits_its_slots=False plants a bug (the odd CTA reloads a K slot
    without waiting for its release)."""
    rng = random.Random(seed)
    # barriers per CTA (index 0 = even); tx barriers only used at rank 0
    def mk(name, count=1):
        return [TxBar(f"{name}@{r}", count) for r in range(2)]
    q_full, q_empty = mk("q_full"), mk("q_empty")
    k_full = [mk(f"k_full{i}") for i in range(NSTK)]
    k_empty = [mk(f"k_empty{i}") for i in range(NSTK)]
    v_full = [mk(f"v_full{i}") for i in range(NSTV)]
    v_empty = [mk(f"v_empty{i}") for i in range(NSTV)]
    s_full = [mk(f"s_full{b}") for b in range(2)]
    p_half = [mk(f"p_half{i}", 8) for i in range(4)]
    pv_done, o_full, o_empty = mk("pv_done"), mk("o_full"), mk("o_empty", 8)

    kslot = [[None] * NSTK for _ in range(2)]
    kused = [[True] * NSTK for _ in range(2)]
    vslot = [[None] * NSTV for _ in range(2)]
    vused = [[True] * NSTV for _ in range(2)]
    qtag = [None, None]
    s_exec = {}
    tma_q = []
    mma_q = []
    sbuf = [[[None, None] for _ in range(4)] for _ in range(2)]
    o_last = {"pv": None}
    epi = set()
    pv_exec = set()

    def producer(r):
        kpos = vpos = 0
        for k in range(units):
            if k > 0:
                yield from wait(q_empty[r], k - 1)
            if r == 0:
                q_full[0].arrive(expect=2)
            tma_q.append(("Q", r, (k,), None, q_full[0], q_full[0].c))
            yield True
            for i in range(nblk + 1):
                if i < nblk:
                    for c in range(QCH):
                        slot, rnd = kpos % NSTK, kpos // NSTK
                        if rnd > 0 and (r == 0 or odd_waits_its_slots):
                            yield from wait(k_empty[slot][r], rnd - 1)
                        bar = k_full[slot][0]
                        if r == 0:
                            bar.arrive(expect=2)
                        tma_q.append(("K", r, (k, i, c), slot, bar, rnd))
                        kpos += 1
                        yield True
                if i >= 1:
                    slot, rnd = vpos % NSTV, vpos // NSTV
                    if rnd > 0:
                        yield from wait(v_empty[slot][r], rnd - 1)
                    bar = v_full[slot][0]
                    if r == 0:
                        bar.arrive(expect=2)
                    tma_q.append(("V", r, (k, i - 1), slot, bar, rnd))
                    vpos += 1
                    yield True

    def mma_warp():
        kpos = vpos = 0
        jb = 0

        def both(name_bars):
            mma_q.append(("commit", name_bars[0]))
            mma_q.append(("commit", name_bars[1]))

        def issue_s(k, jj, j):
            nonlocal kpos
            for c in range(QCH):
                slot = kpos % NSTK
                yield from wait(k_full[slot][0], kpos // NSTK)
                mma_q.append(("S", (k, jj, j, c, slot)))
                both(k_empty[slot])
                kpos += 1
                yield True
            both(s_full[jj & 1])

        def issue_pv(k, jj, j):
            nonlocal vpos
            slot = vpos % NSTV
            yield from wait(v_full[slot][0], vpos // NSTV)
            for half in range(2):
                yield from wait(p_half[2 * (jj & 1) + half][0], jj >> 1)
                mma_q.append(("PV", (k, jj, j, half, slot)))
                yield True
            both(v_empty[slot])
            vpos += 1

        for k in range(units):
            yield from wait(q_full[0], k)
            yield from issue_s(k, jb, 0)
            if nblk > 1:
                yield from issue_s(k, jb + 1, 1)
            if nblk <= 2:
                both(q_empty)
            for j in range(nblk):
                jj = jb + j
                if j == 0 and k > 0:
                    yield from wait(o_empty[0], k - 1)
                yield from issue_pv(k, jj, j)
                both(pv_done)
                if j + 2 < nblk:
                    yield from issue_s(k, jj + 2, j + 2)
                    if j + 3 == nblk:
                        both(q_empty)
            both(o_full)
            jb += nblk

    def softmax(r, w):
        jb = 0
        for k in range(units):
            for j in range(nblk):
                jj = jb + j
                yield from wait(s_full[jj & 1][r], jj >> 1)
                if sbuf[r][w][jj & 1] != ("S", jj, QCH):
                    raise Fail(f"cta {r} warp {w} reads {sbuf[r][w][jj & 1]} want S_{jj}")
                yield True
                need = j == 0 or rng.random() < p_rescale
                if jj > 0:
                    yield from wait(pv_done[r], jj - 1)
                if need and j > 0:
                    if o_last["pv"] != (jj - 1, 1):
                        raise Fail(f"rescale at {jj}: O last written by {o_last['pv']}")
                    yield True
                for half in range(2):
                    sbuf[r][w][jj & 1] = ("P", jj, half + 1)
                    p_half[2 * (jj & 1) + half][0].arrive()
                    yield True
            jb += nblk
            yield from wait(o_full[r], k)
            if o_last["pv"] != (jb - 1, 1):
                raise Fail(f"epilogue unit {k}: O last written by {o_last['pv']}")
            yield True
            epi.add((k, r, w))
            o_empty[0].arrive()
            yield True

    def pipe_step():
        if not mma_q:
            return False
        op, a = mma_q.pop(0)
        if op == "commit":
            a.arrive()
            return True
        if op == "S":
            k, jj, j, c, slot = a
            for r in range(2):
                if qtag[r] != k:
                    raise Fail(f"S_{jj} reads Q{r} of unit {qtag[r]}")
                if kslot[r][slot] != (k, j, c):
                    raise Fail(f"S_{jj} chunk {c} reads K slot {slot}@{r} = {kslot[r][slot]}")
                kused[r][slot] = True
                for w in range(4):
                    cur = sbuf[r][w][jj & 1]
                    if c == 0:
                        if cur is not None and cur[0] == "P" and not (
                                (cur[1], 0) in pv_exec and (cur[1], 1) in pv_exec):
                            raise Fail(f"S_{jj} overwrites P_{cur[1]} before its PV")
                        if cur is not None and cur[0] == "S":
                            raise Fail(f"S_{jj} overwrites unread S_{cur[1]}")
                        sbuf[r][w][jj & 1] = ("S", jj, 1)
                    else:
                        assert cur == ("S", jj, c), cur
                        sbuf[r][w][jj & 1] = ("S", jj, c + 1)
            s_exec[k] = s_exec.get(k, 0) + 1
            return True
        if op == "PV":
            k, jj, j, half, slot = a
            for r in range(2):
                for w in range(4):
                    cur = sbuf[r][w][jj & 1]
                    if not (cur and cur[0] == "P" and cur[1] == jj and cur[2] >= half + 1):
                        raise Fail(f"PV_{jj} half {half} reads {cur} (cta {r} warp {w})")
                if vslot[r][slot] != (k, j):
                    raise Fail(f"PV_{jj} reads V slot {slot}@{r} = {vslot[r][slot]}")
                if half == 1:
                    vused[r][slot] = True
            if j == 0 and half == 0 and k > 0:
                if not all((k - 1, r, w) in epi for r in range(2) for w in range(4)):
                    raise Fail(f"unit {k} PV_0 overwrites O before the epilogue read it")
            o_last["pv"] = (jj, half)
            pv_exec.add((jj, half))
            return True
        raise AssertionError(op)

    def tma_step():
        if not tma_q:
            return False
        i = rng.randrange(len(tma_q))
        kind, r, tag, slot, bar, phase = tma_q.pop(i)
        if kind == "Q":
            (k,) = tag
            if k > 0 and s_exec.get(k - 1, 0) != nblk * QCH:
                raise Fail(f"Q{r} of unit {k} lands before unit {k-1}'s S MMAs ran")
            qtag[r] = k
            bar.complete_tx(1, k)
            return True
        if kind == "K":
            if not kused[r][slot]:
                raise Fail(f"K load {tag}@{r} overwrites slot {slot} before use")
            kslot[r][slot] = tag
            kused[r][slot] = False
        else:
            if not vused[r][slot]:
                raise Fail(f"V load {tag}@{r} overwrites slot {slot} before use")
            vslot[r][slot] = tag
            vused[r][slot] = False
        bar.complete_tx(1, phase)
        return True

    live = {"prod0": producer(0), "prod1": producer(1), "mma": mma_warp()}
    for r in range(2):
        for w in range(4):
            live[f"sm{r}{w}"] = softmax(r, w)
    sleep = {}
    idle = 0
    steps = 0
    while True:
        steps += 1
        if steps > 5_000_000:
            raise Fail("too many steps")
        if not live and not mma_q and not tma_q:
            return steps
        names = list(live.keys()) + ["pipe", "tma"]
        ch = rng.choice(names)
        if sleep.get(ch, 0) > steps:
            continue
        if rng.random() < 0.01:
            sleep[ch] = steps + rng.randint(1, 400)
            continue
        if ch == "pipe":
            progressed = pipe_step()
        elif ch == "tma":
            progressed = tma_step()
        else:
            try:
                progressed = bool(next(live[ch]))
            except StopIteration:
                del live[ch]
                progressed = True
        idle = 0 if progressed else idle + 1
        if idle > 20000:
            raise Fail(f"deadlock; live={list(live)} mma_q={mma_q[:3]} tma_q={tma_q[:3]}")




def run_fa128(seed, NST, nblk, units, p_rescale, pv_first=True):
    """fa_fwd_tc_kernel (fa_tc.cuh): two query tiles per unit, one S buffer
    per tile, K_j / V_j through an NST-slot ring, MMA order S0(0), S1(0),
    then per block PV0(j) (two halves), S0(j+1), PV1(j), S1(j+1). The
    softmax rescales O without waiting for P.V: S_t(j) is issued after
    PV_t(j-1), so seeing S_t(j) complete implies PV_t(j-1) has.
    pv_first=False plants a bug: tile 0's next S issued before its P.V."""
    rng = random.Random(seed)
    q_full, q_empty = Bar("q_full", 1), Bar("q_empty", 1)
    kv_full = [Bar(f"kv_full{i}", 1) for i in range(NST)]
    kv_empty = [Bar(f"kv_empty{i}", 1) for i in range(NST)]
    s_full = [Bar(f"s_full{t}", 1) for t in range(2)]
    p_half = [Bar(f"p_half{i}", 4) for i in range(4)]
    o_full = [Bar(f"o_full{t}", 1) for t in range(2)]
    o_empty = [Bar(f"o_empty{t}", 4) for t in range(2)]
    slot_tag, slot_uses = [None] * NST, [0] * NST
    q_tag, s_done = [None], {}
    tma_q, mma_q = [], []
    sbuf = [[None] * 4 for _ in range(2)]        # per tile, per warp: ("S"|"P", jj, halves)
    o_last = [None, None]                          # (jj, half) of the last PV per tile
    epi = set()

    def producer():
        u = 0
        for k in range(units):
            if k > 0:
                yield from wait(q_empty, k - 1)
            tma_q.append(("Q", k, None, q_full))
            yield True
            for j in range(nblk):
                for kind in ("K", "V"):
                    slot, rnd = u % NST, u // NST
                    if rnd > 0:
                        yield from wait(kv_empty[slot], rnd - 1)
                    tma_q.append((kind, (k, j), slot, kv_full[slot]))
                    u += 1
                    yield True

    def mma():
        jb = 0
        for k in range(units):
            ub = 2 * jb
            yield from wait(q_full, k)
            yield from wait(kv_full[ub % NST], ub // NST)
            for t in range(2):
                mma_q.append(("S", (t, jb, ub % NST, k, 0)))
                mma_q.append(("commit", s_full[t]))
            mma_q.append(("commit", kv_empty[ub % NST]))
            if nblk == 1:
                mma_q.append(("commit", q_empty))
            yield True
            for j in range(nblk):
                jj = jb + j
                uV, uK = 2 * jj + 1, 2 * jj + 2
                more = j + 1 < nblk
                yield from wait(kv_full[uV % NST], uV // NST)
                for t in range(2):
                    if j == 0 and k > 0:
                        yield from wait(o_empty[t], k - 1)
                    early = t == 0 and more and not pv_first
                    if early:
                        yield from wait(kv_full[uK % NST], uK // NST)
                        mma_q.append(("S", (0, jj + 1, uK % NST, k, j + 1)))
                        mma_q.append(("commit", s_full[0]))
                    for half in range(2):
                        yield from wait(p_half[2 * t + half], jj)
                        mma_q.append(("PV", (t, jj, half, uV % NST, k, j)))
                    if t == 0:
                        if more and not early:
                            yield from wait(kv_full[uK % NST], uK // NST)
                            mma_q.append(("S", (0, jj + 1, uK % NST, k, j + 1)))
                            mma_q.append(("commit", s_full[0]))
                        elif not more:
                            mma_q.append(("commit", o_full[0]))
                    else:
                        mma_q.append(("commit", kv_empty[uV % NST]))
                        if more:
                            mma_q.append(("S", (1, jj + 1, uK % NST, k, j + 1)))
                            mma_q.append(("commit", s_full[1]))
                            mma_q.append(("commit", kv_empty[uK % NST]))
                            if j + 2 == nblk:
                                mma_q.append(("commit", q_empty))
                        else:
                            mma_q.append(("commit", o_full[1]))
                    yield True
            jb += nblk

    def softmax(t, w):
        jb = 0
        for k in range(units):
            for j in range(nblk):
                jj = jb + j
                yield from wait(s_full[t], jj)
                if sbuf[t][w] != ("S", jj, 0):
                    raise Fail(f"tile {t} warp {w} reads {sbuf[t][w]}, want S_{jj}")
                yield True
                if j > 0 and (j == 0 or rng.random() < p_rescale):
                    if o_last[t] != (jj - 1, 1):
                        raise Fail(f"rescale tile {t} at {jj}: O last written by {o_last[t]}")
                for half in range(2):
                    sbuf[t][w] = ("P", jj, half + 1)
                    p_half[2 * t + half].arrive()
                    yield True
            jb += nblk
            yield from wait(o_full[t], k)
            if o_last[t] != (jb - 1, 1):
                raise Fail(f"epilogue tile {t} unit {k}: O last written by {o_last[t]}")
            yield True
            epi.add((k, t, w))
            o_empty[t].arrive()
            yield True

    def pipe_step():
        if not mma_q:
            return False
        op, a = mma_q.pop(0)
        if op == "commit":
            a.arrive()
            return True
        if op == "S":
            t, jj, slot, k, j = a
            if q_tag[0] != k or slot_tag[slot] != ("K", (k, j)):
                raise Fail(f"S_{t}({jj}) reads Q {q_tag[0]} / slot {slot_tag[slot]}")
            slot_uses[slot] -= 1
            for w in range(4):
                cur = sbuf[t][w]
                if cur is not None and (cur[0] == "S" or o_last[t] != (cur[1], 1)):
                    raise Fail(f"S_{t}({jj}) overwrites {cur} before it was consumed")
                sbuf[t][w] = ("S", jj, 0)
            s_done[k] = s_done.get(k, 0) + 1
            return True
        t, jj, half, slot, k, j = a
        for w in range(4):
            cur = sbuf[t][w]
            if not (cur and cur[0] == "P" and cur[1] == jj and cur[2] >= half + 1):
                raise Fail(f"PV_{t}({jj}) half {half} reads {cur}")
        if slot_tag[slot] != ("V", (k, j)):
            raise Fail(f"PV_{t}({jj}) reads slot {slot_tag[slot]}")
        if half == 1:
            slot_uses[slot] -= 1
        if j == 0 and half == 0 and k > 0 and not all((k - 1, t, w) in epi for w in range(4)):
            raise Fail(f"unit {k} PV_{t} overwrites O before the epilogue read it")
        o_last[t] = (jj, half)
        return True

    def tma_step():
        if not tma_q:
            return False
        kind, tag, slot, bar = tma_q.pop(rng.randrange(len(tma_q)))
        if kind == "Q":
            if tag > 0 and s_done.get(tag - 1, 0) != 2 * nblk:
                raise Fail(f"Q of unit {tag} lands before unit {tag - 1}'s S MMAs ran")
            q_tag[0] = tag
        else:
            if slot_uses[slot] != 0:
                raise Fail(f"{kind}{tag} overwrites slot {slot} ({slot_tag[slot]}) in use")
            slot_tag[slot], slot_uses[slot] = (kind, tag), 2
        bar.arrive()
        return True

    live = {"prod": producer(), "mma": mma()}
    for t in range(2):
        for w in range(4):
            live[f"sm{t}{w}"] = softmax(t, w)
    _schedule(rng, live, pipe_step, tma_step, mma_q, tma_q)


def run_qkv_pair(seed, NST, k_blocks, tiles, p_stall=0.0, wait_acc_empty=True):
    """qkv_proj_pair_kernel (qkv_proj.cuh): per tile, k_blocks stages through
    an NST-slot ring (each CTA loads its half; both CTAs' bytes complete on
    the even CTA's full[st], which the even CTA arms); the even CTA's MMA
    warp accumulates a tile into TMEM buffer local % 2 and commits empty[st]
    and acc_full[buf] to both CTAs; 4 epilogue warps per CTA read their rows
    and arrive on the even CTA's acc_empty[buf] (8 arrivals).
    wait_acc_empty=False plants a bug: a tile accumulates into a TMEM buffer
    the epilogues may still be reading."""
    rng = random.Random(seed)
    full = [TxBar(f"full{i}", 1) for i in range(NST)]
    empty = [[Bar(f"empty{i}@{r}", 1) for r in range(2)] for i in range(NST)]
    acc_full = [[Bar(f"acc_full{b}@{r}", 1) for r in range(2)] for b in range(2)]
    acc_empty = [Bar(f"acc_empty{b}", 8) for b in range(2)]
    stage = [[None] * NST for _ in range(2)]       # (tile, kb) held per CTA and slot
    used = [[True] * NST for _ in range(2)]
    acc = [None, None]                              # (tile, k blocks accumulated)
    read = set()
    tma_q, mma_q = [], []

    def producer(r):
        it = 0
        for t in range(tiles):
            for kb in range(k_blocks):
                st, rnd = it % NST, it // NST
                if rnd > 0:
                    yield from wait(empty[st][r], rnd - 1)
                if r == 0:
                    full[st].arrive(expect=2)
                tma_q.append((r, st, (t, kb), rnd))
                it += 1
                yield True

    def mma():
        it = 0
        for local in range(tiles):
            buf = local & 1
            if local >= 2 and wait_acc_empty:
                yield from wait(acc_empty[buf], (local >> 1) - 1)
            for kb in range(k_blocks):
                st = it % NST
                yield from wait(full[st], it // NST)
                mma_q.append(("MMA", (local, kb, st, buf)))
                mma_q.append(("commit", empty[st][0]))
                mma_q.append(("commit", empty[st][1]))
                it += 1
                yield True
            mma_q.append(("commit", acc_full[buf][0]))
            mma_q.append(("commit", acc_full[buf][1]))

    def epilogue(r, w):
        for local in range(tiles):
            buf = local & 1
            yield from wait(acc_full[buf][r], local >> 1)
            if acc[buf] != (local, k_blocks):
                raise Fail(f"epilogue of tile {local} reads {acc[buf]}")
            if rng.random() < p_stall:
                yield False
            read.add((local, r, w))
            acc_empty[buf].arrive()
            yield True

    def pipe_step():
        if not mma_q:
            return False
        op, a = mma_q.pop(0)
        if op == "commit":
            a.arrive()
            return True
        local, kb, st, buf = a
        for r in range(2):
            if stage[r][st] != (local, kb):
                raise Fail(f"MMA of tile {local} k {kb} reads stage {stage[r][st]} on CTA {r}")
            used[r][st] = True
        if kb == 0:
            if local >= 2 and not all((local - 2, r, w) in read
                                      for r in range(2) for w in range(4)):
                raise Fail(f"tile {local} overwrites accumulator {buf} before it was read")
            acc[buf] = (local, 1)
        else:
            if acc[buf] != (local, kb):
                raise Fail(f"accumulator {buf} holds {acc[buf]} at tile {local} k {kb}")
            acc[buf] = (local, kb + 1)
        return True

    def tma_step():
        if not tma_q:
            return False
        r, st, tag, rnd = tma_q.pop(rng.randrange(len(tma_q)))
        if not used[r][st]:
            raise Fail(f"CTA {r} reloads stage {st} with {tag} before its MMA ran")
        stage[r][st], used[r][st] = tag, False
        full[st].complete_tx(1, rnd)
        return True

    live = {"prod0": producer(0), "prod1": producer(1), "mma": mma()}
    for r in range(2):
        for w in range(4):
            live[f"epi{r}{w}"] = epilogue(r, w)
    _schedule(rng, live, pipe_step, tma_step, mma_q, tma_q)


def run_exact_tc(seed, nblk, p_rescale, wait_pv=True):
    """attn_exact_tc_kernel (exact_tc.cuh): one query tile; per block j the
    slots 0-3 hold K, r(K), V, r(V) of block j; S_j lands in TMEM buffer j&1
    (MMA order S_0, then per block S_{j+1}, PV_j); the softmax reads S_j, waits
    for PV_{j-1}, may rescale O, then writes g(P_j) over S_j and r(P_j) into
    the one r(P) buffer. wait_pv=False plants a bug: r(P_j)
    written (and O rescaled) without waiting for PV_{j-1}."""
    rng = random.Random(seed)
    q_full = Bar("q_full", 1)
    kv_full = [Bar(f"kv_full{i}", 1) for i in range(4)]
    kv_empty = [Bar(f"kv_empty{i}", 1) for i in range(4)]
    s_full = [Bar(f"s_full{b}", 1) for b in range(2)]
    p_full, pv_done = Bar("p_full", 4), Bar("pv_done", 1)
    slot_tag, slot_busy = [None] * 4, [False] * 4
    q_in = [False]
    sbuf = [[None] * 4 for _ in range(2)]  # per buffer, per warp: ("S"|"P", j)
    pl = [None] * 4                        # r(P) buffer, per warp: j
    o_last = [None]                        # last PV applied to O
    tma_q, mma_q = [], []

    def producer():
        tma_q.append(("Q", 0, None, q_full))
        yield True
        for j in range(nblk):
            for s_ in range(4):
                if j > 0:
                    yield from wait(kv_empty[s_], j - 1)
                tma_q.append(("KV", j, s_, kv_full[s_]))
                yield True

    def mma():
        yield from wait(q_full, 0)
        yield from wait(kv_full[0], 0)
        yield from wait(kv_full[1], 0)
        mma_q.extend([("S", 0), ("commit", s_full[0]), ("commit", kv_empty[0]),
                      ("commit", kv_empty[1])])
        yield True
        for j in range(nblk):
            if j + 1 < nblk:
                yield from wait(kv_full[0], j + 1)
                yield from wait(kv_full[1], j + 1)
                mma_q.extend([("S", j + 1), ("commit", s_full[(j + 1) & 1]),
                              ("commit", kv_empty[0]), ("commit", kv_empty[1])])
                yield True
            yield from wait(p_full, j)
            yield from wait(kv_full[2], j)
            yield from wait(kv_full[3], j)
            mma_q.extend([("PV", j), ("commit", pv_done), ("commit", kv_empty[2]),
                          ("commit", kv_empty[3])])
            yield True

    def softmax(w):
        for j in range(nblk):
            b = j & 1
            yield from wait(s_full[b], j >> 1)
            if sbuf[b][w] != ("S", j):
                raise Fail(f"warp {w} reads {sbuf[b][w]}, want S_{j}")
            yield True
            if j > 0 and wait_pv:
                yield from wait(pv_done, j - 1)
            sbuf[b][w] = ("P", j)
            yield True
            if j > 0 and rng.random() < p_rescale and o_last[0] != j - 1:
                raise Fail(f"O rescaled at {j} while PV_{j - 1} may still write it")
            if j > 0 and o_last[0] != j - 1:
                raise Fail(f"r(P_{j}) written while PV_{j - 1} may still read r(P)")
            pl[w] = j
            yield True
            p_full.arrive()
            yield True
        yield from wait(pv_done, nblk - 1)
        if o_last[0] != nblk - 1:
            raise Fail(f"epilogue reads O after PV_{o_last[0]}")

    def pipe_step():
        if not mma_q:
            return False
        op, a = mma_q.pop(0)
        if op == "commit":
            a.arrive()
            return True
        j = a
        if op == "S":
            if not q_in[0] or slot_tag[0] != j or slot_tag[1] != j:
                raise Fail(f"S_{j} reads Q {q_in[0]} / K slots {slot_tag[:2]}")
            slot_busy[0] = slot_busy[1] = False
            b = j & 1
            for w in range(4):
                cur = sbuf[b][w]
                if cur is not None and (cur[0] == "S" or o_last[0] is None or o_last[0] < cur[1]):
                    raise Fail(f"S_{j} overwrites {cur} before it was consumed")
                sbuf[b][w] = ("S", j)
            return True
        b = j & 1
        for w in range(4):
            if sbuf[b][w] != ("P", j) or pl[w] != j:
                raise Fail(f"PV_{j} reads P {sbuf[b][w]} / r(P) {pl[w]}")
        if slot_tag[2] != j or slot_tag[3] != j:
            raise Fail(f"PV_{j} reads V slots {slot_tag[2:]}")
        slot_busy[2] = slot_busy[3] = False
        o_last[0] = j
        return True

    def tma_step():
        if not tma_q:
            return False
        kind, j, s_, bar = tma_q.pop(rng.randrange(len(tma_q)))
        if kind == "Q":
            q_in[0] = True
        else:
            if slot_busy[s_]:
                raise Fail(f"block {j} overwrites slot {s_} (block {slot_tag[s_]}) in use")
            slot_tag[s_], slot_busy[s_] = j, True
        bar.arrive()
        return True

    live = {"prod": producer(), "mma": mma()}
    for w in range(4):
        live[f"sm{w}"] = softmax(w)
    _schedule(rng, live, pipe_step, tma_step, mma_q, tma_q)


def _schedule(rng, live, pipe_step, tma_step, mma_q, tma_q):
    """Runs the roles under a random scheduler with random stalls until all
    are done; raises Fail on a deadlock."""
    sleep, idle, steps = {}, 0, 0
    while live or mma_q or tma_q:
        steps += 1
        if steps > 5_000_000:
            raise Fail("too many steps")
        ch = rng.choice(list(live) + ["pipe", "tma"])
        if sleep.get(ch, 0) > steps:
            continue
        if rng.random() < 0.01:
            sleep[ch] = steps + rng.randint(1, 400)
            continue
        if ch == "pipe":
            progressed = pipe_step()
        elif ch == "tma":
            progressed = tma_step()
        else:
            try:
                progressed = bool(next(live[ch]))
            except StopIteration:
                del live[ch]
                progressed = True
        idle = 0 if progressed else idle + 1
        if idle > 20000:
            raise Fail(f"deadlock; live={list(live)} mma_q={mma_q[:3]} tma_q={tma_q[:3]}")


def _configs_single():
    for seed in range(6):
        for qch, vch, nst in ((8, 4, 6), (6, 3, 8)):
            for nblk in (1, 2, 3, 5):
                for units in (1, 3):
                    yield seed * 100 + nblk * 10 + units, qch, vch, nst, nblk, units, \
                        (0.0, 0.3, 1.0)[seed % 3]


def _configs_pair():
    for seed in range(6):
        for qch, nstk, nstv in ((8, 8, 1), (6, 8, 2)):
            for nblk in (1, 2, 3, 5):
                for units in (1, 3):
                    yield seed * 100 + nblk * 10 + units, qch, nstk, nstv, nblk, units, \
                        (0.0, 0.3, 1.0)[seed % 3]


def test_fa128_protocol():
    for seed in range(6):
        for nst in (4, 8):
            for nblk in (1, 2, 3, 5):
                for units in (1, 3):
                    run_fa128(seed * 100 + nblk * 10 + units, nst, nblk, units,
                              (0.0, 0.3, 1.0)[seed % 3])


def test_qkv_pair_protocol():
    for seed in range(8):
        for nst in (4, 6):
            for k_blocks in (1, 3, 7):
                for tiles in (1, 3, 5):
                    run_qkv_pair(seed * 100 + k_blocks * 10 + tiles, nst, k_blocks, tiles,
                                 (0.0, 0.5)[seed % 2])


def test_model_finds_accumulator_overwrite():
    with pytest.raises(Fail, match="overwrites accumulator"):
        for seed in range(20):
            run_qkv_pair(seed, 4, 3, 5, 0.5, wait_acc_empty=False)


def test_model_finds_p_overwrite():
    with pytest.raises(Fail):
        for seed in range(6):
            run_fa128(seed, 4, 3, 2, 0.3, pv_first=False)


def test_single_cta_protocol():
    for cfg in _configs_single():
        run_single(*cfg)


def test_pair_protocol():
    for cfg in _configs_pair():
        run_pair(*cfg)


def test_model_finds_phase_aliasing():
    """One P barrier per key half instead of per S buffer, with PV's
    completion observed only when rescaling: the softmax can then complete
    a P phase twice before the MMA warp looks (it runs a block ahead)."""
    with pytest.raises(Fail, match="aliasing"):
        for cfg in _configs_single():
            run_single(*cfg, per_buffer_p=False, pv_wait_every_block=False)


def test_model_finds_ring_overrun():
    with pytest.raises(Fail):
        for cfg in _configs_pair():
            run_pair(*cfg, odd_waits_its_slots=False)


def test_exact_tc_protocol():
    for seed in range(10):
        for nblk in (1, 2, 3, 4, 7):
            run_exact_tc(seed * 100 + nblk, nblk, (0.0, 0.5, 1.0)[seed % 3])


def test_model_finds_r_of_p_overwrite():
    with pytest.raises(Fail):
        for seed in range(40):
            run_exact_tc(seed, 5, 0.0, wait_pv=False)
