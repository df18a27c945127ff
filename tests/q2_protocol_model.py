"""Executable model of the synchronisation protocol of the two-query-tile prefill kernel
(csrc/prefill_q2.cu): the TMA producers, the MMA issuer and the two softmax warpgroups run as
coroutines against mbarriers with the hardware's phase semantics, tcgen05 operations execute in
issue order with random delays, and every shared buffer (Q tiles, K/V stages, S/P and O in TMEM)
carries a tag of what it holds.  Random interleavings of random work lists check:

* no deadlock: some role or pending completion can always make progress;
* no aliased wait: while a role waits for phase k of a barrier, the barrier never completes
  phase k + 1 (a parity wait would then test the wrong phase);
* every read sees the data it expects (the right item and tile), every write lands on a buffer
  no pending operation still needs, and V rows past the item's keys are zeroed before any PV
  reads the last tile.
"""
from __future__ import annotations

import random
from collections import deque

KBN = 128
K_STAGES = 2
V_STAGES = 2


class Bug(Exception):
    pass


class Barrier:
    def __init__(self, name, count):
        self.name, self.count = name, count
        self.pending = 0
        self.completed = 0          # completed phases
        self.waiting = {}           # role -> phase index it waits for

    def arrive(self):
        self.pending += 1
        if self.pending == self.count:
            self.pending = 0
            self.completed += 1
            for role, k in self.waiting.items():
                if self.completed > k + 1:
                    raise Bug(f"{self.name}: {role} waits for phase {k}, barrier completed "
                              f"{self.completed} phases (aliased parity wait)")

    def passes(self, k):
        # try_wait.parity(k & 1) on the hardware: true iff the current phase's parity differs
        if self.completed > k + 1:
            raise Bug(f"{self.name}: wait for phase {k} after {self.completed} completions")
        return self.completed == k + 1


class Sim:
    def __init__(self, items, tq, rng, mutation=None):
        self.mutation = mutation   # a deliberate protocol mistake, to check the model sees it
        self.rng = rng
        self.items = items
        self.tq = tq
        b = lambda name, count=1: Barrier(name, count)
        self.q_full, self.q_empty = b("QFull"), b("QEmpty")
        self.k_full = [b(f"KFull{i}") for i in range(K_STAGES)]
        self.k_empty = [b(f"KEmpty{i}") for i in range(K_STAGES)]
        self.v_full = [b(f"VFull{i}") for i in range(V_STAGES)]
        self.v_empty = [b(f"VEmpty{i}") for i in range(V_STAGES)]
        self.s_full = [b("SFull0"), b("SFull1")]
        self.p_full = [b("PFull0", 4), b("PFull1", 4)]
        self.pv_done = [b("PvDone0"), b("PvDone1")]
        self.o_empty = [b("OEmpty0", 4), b("OEmpty1", 4)]
        self.begin = [b("Begin0"), b("Begin1")]
        self.final = b("Final")
        # buffer tags
        self.q_tag = None
        self.k_tag = [None] * K_STAGES
        self.v_tag = [None] * V_STAGES
        self.v_zeroed = [False] * V_STAGES
        self.s_tag = [None, None]      # S/P buffer of warpgroup w: ("S"|"P", item, tile)
        self.o_tag = [None, None]      # ("O", item, tile of the last PV)
        self.tc_queue = deque()        # issued tcgen05 ops, executed in order
        self.async_events = []         # TMA completions: (callable)
        self.done_roles = set()

    # ---- tcgen05 ops ---------------------------------------------------------------------------
    def mma_s(self, w, stage, item, tile):
        self.tc_queue.append(("S", w, stage, item, tile))

    def mma_pv(self, w, stage, item, tile, acc, needs_zero_last):
        self.tc_queue.append(("PV", w, stage, item, tile, acc, needs_zero_last))

    def commit(self, bar):
        self.tc_queue.append(("C", bar))

    def exec_tc(self):
        op = self.tc_queue.popleft()
        if op[0] == "S":
            _, w, stage, item, tile = op
            if self.q_tag != item:
                raise Bug(f"S{w}({item},{tile}) reads Q of {self.q_tag}")
            if self.k_tag[stage] != (item, tile):
                raise Bug(f"S{w}({item},{tile}) reads K stage {stage} holding {self.k_tag[stage]}")
            self.s_tag[w] = ("S", item, tile)
        elif op[0] == "PV":
            _, w, stage, item, tile, acc, last_zero = op
            if self.s_tag[w] != ("P", item, tile):
                raise Bug(f"PV{w}({item},{tile}) reads {self.s_tag[w]}")
            if self.v_tag[stage] != (item, tile):
                raise Bug(f"PV{w}({item},{tile}) reads V stage {stage} holding {self.v_tag[stage]}")
            if last_zero and not self.v_zeroed[stage]:
                raise Bug(f"PV{w}({item},{tile}) reads the last V tile before it was zeroed")
            if acc and self.o_tag[w] != ("O", item, tile - 1):
                raise Bug(f"PV{w}({item},{tile}) accumulates onto {self.o_tag[w]}")
            self.o_tag[w] = ("O", item, tile)
        else:
            op[1].arrive()

    def tc_reads_stage(self, kind, stage):
        for op in self.tc_queue:
            if kind == "K" and op[0] == "S" and op[2] == stage:
                return True
            if kind == "V" and op[0] == "PV" and op[2] == stage:
                return True
            if kind == "Q" and op[0] == "S":
                return True
        return False

    # ---- waits ---------------------------------------------------------------------------------
    def wait(self, role, bar, k):
        bar.waiting[role] = k
        while not bar.passes(k):
            yield "blocked"
        del bar.waiting[role]

    # ---- roles ---------------------------------------------------------------------------------
    def producer(self, is_k):
        role = "K" if is_k else "V"
        nst = K_STAGES if is_k else V_STAGES
        full = self.k_full if is_k else self.v_full
        empty = self.k_empty if is_k else self.v_empty
        kv_it = 0
        for n, it in enumerate(self.items):
            if is_k:
                yield from self.wait(role, self.q_empty, n - 1)
                if self.tc_reads_stage("Q", 0):
                    raise Bug("Q reloaded while an S still reads it")

                def land_q(n=n):
                    self.q_tag = n
                    self.q_full.arrive()
                self.async_events.append(land_q)
            for j in range(it["n_kv_all"]):
                st = kv_it % nst
                if self.mutation != "no_empty_wait":
                    yield from self.wait(role, empty[st], kv_it // nst - 1)
                if self.tc_reads_stage("K" if is_k else "V", st):
                    raise Bug(f"{role} stage {st} refilled while an MMA still reads it")

                def land(st=st, tag=(n, j)):
                    if is_k:
                        self.k_tag[st] = tag
                    else:
                        self.v_tag[st] = tag
                        self.v_zeroed[st] = False
                    full[st].arrive()
                self.async_events.append(land)
                kv_it += 1
                yield
        self.done_roles.add(role)

    def mma(self):
        role = "MMA"
        n_items, kv_it = 0, 0
        c = [0, 0]
        for n, it in enumerate(self.items):
            n_kv = it["n_kv_all"]
            nk = it["n_kv"]
            # warpgroup 0 zeroes the V tail when it attends the item's last KV tile
            zw = 0 if nk[0] == n_kv else 1
            needs_zero = it["kv_end_all"] < n_kv * KBN
            yield from self.wait(role, self.q_full, n)
            yield from self.wait(role, self.k_full[kv_it % K_STAGES], kv_it // K_STAGES)
            for w in (0, 1):
                if nk[w] == 0:
                    continue
                self.mma_s(w, kv_it % K_STAGES, n, 0)
                self.commit(self.s_full[w])
            self.commit(self.k_empty[kv_it % K_STAGES])
            if n_kv == 1:
                self.commit(self.q_empty)
            for w in (0, 1):
                yield from self.wait(role, self.o_empty[w],
                                     n if self.mutation == "wrong_o_phase" else n - 1)
                # only a warpgroup without rows in the item waits for Begin
                if nk[w] == 0:
                    self.begin[w].arrive()
            for j in range(n_kv):
                f = kv_it + j
                zero_here = needs_zero and j == n_kv - 1
                yield from self.wait(role, self.v_full[f % V_STAGES], f // V_STAGES)
                # (implied by the PFull waits below when warpgroup 0 zeroes; kept as in the kernel)
                if zero_here:
                    yield from self.wait(role, self.p_full[zw], c[zw] + j)
                for w in (0, 1):
                    if j >= nk[w]:
                        continue
                    yield from self.wait(role, self.p_full[w], c[w] + j)
                    if self.mutation == "s_before_pv" and j + 1 < nk[w]:
                        yield from self.wait(role, self.k_full[(f + 1) % K_STAGES],
                                             (f + 1) // K_STAGES)
                        self.mma_s(w, (f + 1) % K_STAGES, n, j + 1)
                    self.mma_pv(w, f % V_STAGES, n, j, j > 0, zero_here)
                    self.commit(self.pv_done[w])
                    if j + 1 < nk[w]:
                        first = (w == 0) or (j + 1 >= nk[0])
                        last = (w == 1) or (j + 1 >= nk[1])
                        if self.mutation == "release_k_early":
                            last = first
                        if first:
                            yield from self.wait(role, self.k_full[(f + 1) % K_STAGES],
                                                 (f + 1) // K_STAGES)
                        self.mma_s(w, (f + 1) % K_STAGES, n, j + 1)
                        self.commit(self.s_full[w])
                        if last:
                            self.commit(self.k_empty[(f + 1) % K_STAGES])
                            if j + 1 == n_kv - 1:
                                self.commit(self.q_empty)
                self.commit(self.v_empty[f % V_STAGES])
            kv_it += n_kv
            c[0] += nk[0]
            c[1] += nk[1]
            n_items += 1
            yield
        self.commit(self.final)
        yield from self.wait(role, self.final, 0)
        self.done_roles.add(role)

    def softmax_warp(self, w, quarter):
        role = f"SM{w}.{quarter}"
        c, kv_it, idle = 0, 0, 0
        for n, it in enumerate(self.items):
            n_kv = it["n_kv"][w]
            zw = 0 if it["n_kv"][0] == it["n_kv_all"] else 1
            if self.mutation == "wrong_zeroer":
                # the warpgroup with the latest rows zeroes, while the MMA warp assumes the rule
                zw = 1 if it["n_kv"][1] > 0 else 0
            zeroer = w == zw and it["kv_end_all"] < it["n_kv_all"] * KBN
            # a warpgroup with rows is gated by its first SFull wait; one without waits for Begin
            if n_kv == 0 and self.mutation != "no_begin":
                yield from self.wait(role, self.begin[w], idle)
            if n_kv == 0:
                idle += 1
            for j in range(n_kv):
                yield from self.wait(role, self.s_full[w], c + j)
                if self.s_tag[w] not in (("S", n, j), ("P", n, j)):
                    raise Bug(f"{role} reads S of {self.s_tag[w]}, expects ({n},{j})")
                if j >= 1 and self.o_tag[w] != ("O", n, j - 1):
                    raise Bug(f"{role} rescales O holding {self.o_tag[w]}, expects ({n},{j-1})")
                yield
                # P written over the S columns (all four warps write their rows)
                if self.s_tag[w] not in (("S", n, j), ("P", n, j)):
                    raise Bug(f"{role}: S/P overwritten during the softmax of ({n},{j})")
                self.s_tag[w] = ("P", n, j)
                if zeroer and j == it["n_kv_all"] - 1:
                    fv = kv_it + j
                    yield from self.wait(role, self.v_full[fv % V_STAGES], fv // V_STAGES)
                    if self.v_tag[fv % V_STAGES] != (n, j):
                        raise Bug(f"{role} zeroes V stage holding {self.v_tag[fv % V_STAGES]}")
                    self.v_zero_count[fv % V_STAGES] += 1
                    if self.v_zero_count[fv % V_STAGES] == 4:
                        self.v_zeroed[fv % V_STAGES] = True
                        self.v_zero_count[fv % V_STAGES] = 0
                self.p_full[w].arrive()
            if n_kv > 0:
                yield from self.wait(role, self.pv_done[w],
                                     c + n_kv - (2 if self.mutation == "early_epilogue" else 1))
                if self.o_tag[w] != ("O", n, n_kv - 1):
                    raise Bug(f"{role} epilogue reads O holding {self.o_tag[w]}")
            yield
            self.o_empty[w].arrive()
            c += n_kv
            kv_it += it["n_kv_all"]
        self.done_roles.add(role)

    def run(self):
        self.v_zero_count = [0] * V_STAGES
        roles = [self.producer(True), self.producer(False), self.mma()]
        roles += [self.softmax_warp(w, q) for w in (0, 1) for q in range(4)]
        live = list(roles)
        spins = 0   # consecutive role steps that only re-tested a wait
        while live or self.tc_queue or self.async_events:
            choices = []
            if live:
                choices.append("role")
            if self.tc_queue:
                choices.append("tc")
            if self.async_events:
                choices.append("tma")
            kind = self.rng.choice(choices)
            if kind == "tc":
                self.exec_tc()
                spins = 0
            elif kind == "tma":
                ev = self.async_events.pop(self.rng.randrange(len(self.async_events)))
                ev()
                spins = 0
            else:
                r = self.rng.choice(live)
                try:
                    spins = spins + 1 if next(r) == "blocked" else 0
                except StopIteration:
                    live.remove(r)
                    spins = 0
            if spins > 200 * max(1, len(live)) and not self.tc_queue and not self.async_events:
                waits = sorted(f"{b.name}:{k}" for b in self._all_bars()
                               for k in b.waiting.values())
                raise Bug("deadlock, waiting on " + ", ".join(waits))

    def _all_bars(self):
        out = [self.q_full, self.q_empty, self.final]
        for group in (self.k_full, self.k_empty, self.v_full, self.v_empty, self.s_full,
                      self.p_full, self.pv_done, self.o_empty, self.begin):
            out += group
        return out


def make_items(rng, tq, n_items):
    """Random work items in the kernel's decomposition: pairs of query tiles of tq tokens of a
    sequence with a cached prefix; the last pair of a sequence may hold one tile."""
    items = []
    while len(items) < n_items:
        count = rng.randint(1, 5 * tq)
        prior = rng.choice([0, rng.randint(0, 3 * KBN)])
        ctx = prior + count
        for p in range((count + 2 * tq - 1) // (2 * tq)):
            t_begin = p * 2 * tq
            pos0 = ctx - count + t_begin
            n_q = [max(0, min(tq, count - t_begin - t * tq)) for t in (0, 1)]
            kv_end = [pos0 + t * tq + n_q[t] for t in (0, 1)]
            n_kv = [(kv_end[t] + KBN - 1) // KBN if n_q[t] > 0 else 0 for t in (0, 1)]
            items.append({"n_kv": n_kv, "n_kv_all": max(n_kv),
                          "kv_end_all": kv_end[1] if n_q[1] > 0 else kv_end[0]})
    return items[:n_items]


def check(trials=300, seed=0, mutation=None):
    """Runs random trials; returns the first Bug message (None if every trial passed)."""
    rng = random.Random(seed)
    for trial in range(trials):
        tq = rng.choice([8, 16, 32, 64, 128])
        items = make_items(rng, tq, rng.randint(1, 12))
        try:
            Sim(items, tq, random.Random(rng.random()), mutation).run()
        except Bug as e:
            return f"trial {trial}: {e}"
    return None


MUTATIONS = ("wrong_zeroer", "release_k_early", "wrong_o_phase", "no_begin", "s_before_pv",
             "no_empty_wait", "early_epilogue")
