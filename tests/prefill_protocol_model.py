"""Executable model of the synchronisation protocol of the tensor-core prefill kernel
(csrc/prefill.cu, prefill_tc_kernel), for checking it without a GPU.

The roles of one CTA -- the K and V TMA producers, the MMA issuer and the eight softmax warps of
the two warpgroups -- run as coroutines against mbarriers with the hardware's phase semantics;
tcgen05 operations execute in issue order after random delays, TMA fills land in random order,
and every shared buffer (Q, the K and V stages, the S/P buffers and O accumulators in TMEM, the
(max, sum) exchange) carries a tag of what it holds.  Random work lists under random
interleavings check that there is no deadlock, that no parity wait can see a later phase than the
one it means (a barrier never completes phase k + 1 while someone waits for phase k), and that
every read sees the item and tile it expects.  The sequences of waits, arrivals and commits follow
the kernel's code path by path; a change to the kernel's protocol belongs here too.
"""
from __future__ import annotations

import random
from collections import deque

KBN = 128
K_STAGES = 3
V_STAGES = 2
SOFTMAX_WARPS = 8


class Bug(Exception):
    pass


class Barrier:
    def __init__(self, name, count):
        self.name, self.count = name, count
        self.pending = 0
        self.completed = 0
        self.waiting = {}

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
        if self.completed > k + 1:
            raise Bug(f"{self.name}: wait for phase {k} after {self.completed} completions")
        return self.completed == k + 1


class Sim:
    def __init__(self, items, rng, mutation=None):
        self.items, self.rng, self.mutation = items, rng, mutation
        b = Barrier
        self.q_full, self.q_empty = b("QFull", 1), b("QEmpty", 1)
        self.k_full = [b(f"KFull{i}", 1) for i in range(K_STAGES)]
        self.k_empty = [b(f"KEmpty{i}", 1) for i in range(K_STAGES)]
        self.v_full = [b(f"VFull{i}", 1) for i in range(V_STAGES)]
        self.v_empty = [b(f"VEmpty{i}", 1) for i in range(V_STAGES)]
        self.s_full = [b("SFull0", 1), b("SFull1", 1)]
        self.p_full = [b("PFull0", 4), b("PFull1", 4)]
        self.pv_done = [b("PvDone0", 1), b("PvDone1", 1)]
        self.o_empty = b("OEmpty", SOFTMAX_WARPS)
        self.xchg = b("Xchg", SOFTMAX_WARPS)
        self.final = b("Final", 1)
        self.q_tag = None
        self.k_tag = [None] * K_STAGES
        self.v_tag = [None] * V_STAGES
        self.v_zeroed = [False] * V_STAGES
        self.v_zero_count = [0] * V_STAGES
        self.s_tag = [None, None]        # ("S"|"P", item, tile)
        self.o_tag = [None, None]        # ("O", item, tile of the last PV into it)
        self.xch = [dict(), dict()]      # exchange buffer by item parity: warpgroup -> item
        self.tc_queue = deque()
        self.async_events = []

    # ---- tcgen05 --------------------------------------------------------------------------------
    def exec_tc(self):
        op = self.tc_queue.popleft()
        if op[0] == "S":
            _, w, stage, item, tile = op
            if self.q_tag != item:
                raise Bug(f"S({item},{tile}) reads Q of {self.q_tag}")
            if self.k_tag[stage] != (item, tile):
                raise Bug(f"S({item},{tile}) reads K stage {stage} holding {self.k_tag[stage]}")
            self.s_tag[w] = ("S", item, tile)
        elif op[0] == "PV":
            _, w, stage, item, tile, acc, zero_needed = op
            if self.s_tag[w] != ("P", item, tile):
                raise Bug(f"PV({item},{tile}) reads {self.s_tag[w]}")
            if self.v_tag[stage] != (item, tile):
                raise Bug(f"PV({item},{tile}) reads V stage {stage} holding {self.v_tag[stage]}")
            if zero_needed and not self.v_zeroed[stage]:
                raise Bug(f"PV({item},{tile}) reads the last V tile before it was zeroed")
            if acc and self.o_tag[w] != ("O", item, tile - 2):
                raise Bug(f"PV({item},{tile}) accumulates onto {self.o_tag[w]}")
            self.o_tag[w] = ("O", item, tile)
        else:
            op[1].arrive()

    def pending_reads(self, kind, stage=None):
        for op in self.tc_queue:
            if kind == "K" and op[0] == "S" and op[2] == stage:
                return True
            if kind == "V" and op[0] == "PV" and op[2] == stage:
                return True
            if kind == "Q" and op[0] == "S":
                return True
        return False

    def wait(self, role, bar, k):
        bar.waiting[role] = k
        while not bar.passes(k):
            yield "blocked"
        del bar.waiting[role]

    # ---- roles (prefill.cu, in order) -------------------------------------------------------------
    def producer(self, is_k):
        role = "K" if is_k else "V"
        nst = K_STAGES if is_k else V_STAGES
        full = self.k_full if is_k else self.v_full
        empty = self.k_empty if is_k else self.v_empty
        kv_it = 0
        for n, it in enumerate(self.items):
            if is_k:
                yield from self.wait(role, self.q_empty, n - 1)
                if self.pending_reads("Q"):
                    raise Bug("Q reloaded while an S still reads it")

                def land_q(n=n):
                    self.q_tag = n
                    self.q_full.arrive()
                self.async_events.append(land_q)
            for j in range(it["n_kv"]):
                st = kv_it % nst
                yield from self.wait(role, empty[st], kv_it // nst - 1)
                if self.pending_reads(role, st):
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

    def mma(self):
        role = "MMA"
        kv_it = s_it = 0
        for n, it in enumerate(self.items):
            n_kv = it["n_kv"]
            needs_zero = it["kv_end"] < n_kv * KBN
            yield from self.wait(role, self.q_full, n)

            def issue_s_tile(g, f, tile):
                wg = g & 1
                yield from self.wait(role, self.k_full[f % K_STAGES], f // K_STAGES)
                self.tc_queue.append(("S", wg, f % K_STAGES, n, tile))
                self.tc_queue.append(("C", self.s_full[wg]))
                self.tc_queue.append(("C", self.k_empty[f % K_STAGES]))

            for j in range(min(2, n_kv)):
                yield from issue_s_tile(s_it + j, kv_it + j, j)
            if n_kv <= 2:
                self.tc_queue.append(("C", self.q_empty))
            phase = n if self.mutation == "wrong_o_phase" else n - 1
            yield from self.wait(role, self.o_empty, phase)
            for j in range(n_kv):
                g, f = s_it + j, kv_it + j
                wg = g & 1
                yield from self.wait(role, self.p_full[wg], g >> 1)
                yield from self.wait(role, self.v_full[f % V_STAGES], f // V_STAGES)
                early_s = self.mutation == "s_before_pv" and j + 2 < n_kv
                if early_s:
                    yield from issue_s_tile(g + 2, f + 2, j + 2)
                self.tc_queue.append(("PV", wg, f % V_STAGES, n, j, j >= 2,
                                      needs_zero and j == n_kv - 1))
                self.tc_queue.append(("C", self.pv_done[wg]))
                self.tc_queue.append(("C", self.v_empty[f % V_STAGES]))
                if j + 2 < n_kv:
                    if not early_s:
                        yield from issue_s_tile(g + 2, f + 2, j + 2)
                    if j + 2 == n_kv - 1:
                        self.tc_queue.append(("C", self.q_empty))
            kv_it += n_kv
            s_it += n_kv
            yield
        self.tc_queue.append(("C", self.final))
        yield from self.wait(role, self.final, 0)

    def softmax_warp(self, w, quarter):
        role = f"SM{w}.{quarter}"
        s_it = kv_it = 0
        for n, it in enumerate(self.items):
            n_kv = it["n_kv"]
            needs_zero = it["kv_end"] < n_kv * KBN
            j0 = (s_it ^ w) & 1
            j = j0
            while j < n_kv:
                gt = s_it + j
                yield from self.wait(role, self.s_full[w], gt >> 1)
                if self.s_tag[w] not in (("S", n, j), ("P", n, j)):
                    raise Bug(f"{role} reads S holding {self.s_tag[w]}, expects ({n},{j})")
                if j >= 2 and self.o_tag[w] != ("O", n, j - 2):
                    raise Bug(f"{role} rescales O holding {self.o_tag[w]}, expects ({n},{j-2})")
                yield
                if self.s_tag[w] not in (("S", n, j), ("P", n, j)):
                    raise Bug(f"{role}: S/P overwritten during the softmax of ({n},{j})")
                self.s_tag[w] = ("P", n, j)
                if j == n_kv - 1 and needs_zero:
                    fv = kv_it + j
                    yield from self.wait(role, self.v_full[fv % V_STAGES], fv // V_STAGES)
                    if self.v_tag[fv % V_STAGES] != (n, j):
                        raise Bug(f"{role} zeroes V stage holding {self.v_tag[fv % V_STAGES]}")
                    self.v_zero_count[fv % V_STAGES] += 1
                    if self.v_zero_count[fv % V_STAGES] == 4:
                        self.v_zeroed[fv % V_STAGES] = True
                        self.v_zero_count[fv % V_STAGES] = 0
                self.p_full[w].arrive()
                j += 2
            # epilogue: last PV of this warpgroup, (m, l) exchange, merge of both accumulators
            if j0 < n_kv and self.mutation != "no_pvdone_wait":
                gl = s_it + (j - 2)
                yield from self.wait(role, self.pv_done[w], gl >> 1)
            self.xch[n & 1][(w, quarter)] = n
            self.xchg.arrive()
            if self.mutation != "no_xchg_wait":
                yield from self.wait(role, self.xchg, n)
            other = [v for (ww, q), v in self.xch[n & 1].items() if ww != w and q == quarter]
            if other != [n]:
                raise Bug(f"{role} reads the exchange holding {other}, expects item {n}")
            for ww in (0, 1):
                jw0 = (s_it ^ ww) & 1
                if jw0 < n_kv:
                    last = jw0 + ((n_kv - 1 - jw0) // 2) * 2
                    if self.o_tag[ww] != ("O", n, last):
                        raise Bug(f"{role} merges O{ww} holding {self.o_tag[ww]}, expects "
                                  f"({n},{last})")
            yield
            self.o_empty.arrive()
            s_it += n_kv
            kv_it += n_kv

    def run(self):
        live = [self.producer(True), self.producer(False), self.mma()]
        live += [self.softmax_warp(w, q) for w in (0, 1) for q in range(4)]
        spins = 0
        while live or self.tc_queue or self.async_events:
            choices = (["role"] if live else []) + (["tc"] if self.tc_queue else []) + \
                      (["tma"] if self.async_events else [])
            kind = self.rng.choice(choices)
            if kind == "tc":
                self.exec_tc()
                spins = 0
            elif kind == "tma":
                self.async_events.pop(self.rng.randrange(len(self.async_events)))()
                spins = 0
            else:
                r = self.rng.choice(live)
                try:
                    spins = spins + 1 if next(r) == "blocked" else 0
                except StopIteration:
                    live.remove(r)
                    spins = 0
            if spins > 200 * max(1, len(live)) and not self.tc_queue and not self.async_events:
                raise Bug("deadlock")


def make_items(rng, tq, n_items):
    """Random work items as the plan makes them: tiles of tq query tokens of sequences with a
    cached prefix, each attending up to its last token."""
    items = []
    while len(items) < n_items:
        count = rng.randint(1, 4 * tq)
        prior = rng.choice([0, rng.randint(0, 3 * KBN)])
        for k in range((count + tq - 1) // tq):
            n_q = min(tq, count - k * tq)
            kv_end = prior + k * tq + n_q
            items.append({"n_kv": (kv_end + KBN - 1) // KBN, "kv_end": kv_end})
    return items[:n_items]


MUTATIONS = ("wrong_o_phase", "s_before_pv", "no_pvdone_wait", "no_xchg_wait")


def check(trials=300, seed=0, mutation=None):
    """Random trials; returns the first Bug message, or None when every trial passed."""
    rng = random.Random(seed)
    for trial in range(trials):
        tq = rng.choice([8, 16, 32, 64, 128])
        items = make_items(rng, tq, rng.randint(1, 12))
        try:
            Sim(items, random.Random(rng.random()), mutation).run()
        except Bug as e:
            return f"trial {trial}: {e}"
    return None
