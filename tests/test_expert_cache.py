"""The host-streamed experts' cache policy (kestrel_b200/csrc/expert_cache.h),
on the CPU: a small C++ driver (tests/expert_cache_driver.cpp) runs the
header's class on scripted calls, and the results are checked
* against hand-worked cases of ExpertStore's rules
  (crates/kestrel-memory/src/expert.rs): LRU order, the LFRU score
  `(heat << 8) | (255 - age)` and its admission margin `hs > cs + cs/4 +
  (4 << 8)` (expert.rs:305-331), scratch loads for experts the cache does not
  admit, prefetch used / wasted / late counts (expert.rs:358-521), decay
  (expert.rs:545-551);
* against RefCache below, a separate Python restatement of the same rules,
  on seeded random traces of demand calls, prefetches, landed copies and
  decays over several layers and both policies."""
import os
import random
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def driver(tmp_path_factory):
    cxx = shutil.which("g++")
    if not cxx:
        pytest.skip("g++ not found")
    exe = str(tmp_path_factory.mktemp("xc") / "expert_cache_driver")
    subprocess.run([cxx, "-std=c++17", "-O1", "-Wall", "-Werror", "-I", os.path.join(ROOT, "kestrel_b200", "csrc"),
                    os.path.join(ROOT, "tests", "expert_cache_driver.cpp"), "-o", exe], check=True)
    return exe


def run(exe, script):
    out = subprocess.run([exe], input="\n".join(script) + "\n", capture_output=True, text=True, check=True)
    return out.stdout.splitlines()


def demand(layer, experts):
    return f"demand {layer} {len(experts)} " + " ".join(map(str, experts))


def prefetch(layer, experts):
    return f"prefetch {layer} {len(experts)} " + " ".join(map(str, experts))


STATS = ["requests", "hits", "late", "misses", "scratch_loads", "prefetch_issued", "prefetch_used",
         "prefetch_wasted", "evictions", "forced", "cached", "spec_pauses"]


def stats(line):
    assert line.startswith("T ")
    return dict(zip(STATS, map(int, line.split()[1:])))


def test_lru_evicts_least_recent(driver):
    out = run(driver, ["config 2 0 1", demand(0, [1]), demand(0, [2]), demand(0, [1]), demand(0, [3]),
                       "slot 0 1", "slot 0 2", "slot 0 3", "stats"])
    assert out[0] == "D 0 | 1:0 |"
    assert out[1] == "D 1 | 2:1 |"
    assert out[2] == "D 0 | |"           # hit
    assert out[3] == "D 1 | 3:1 |"       # 2 was used before 1: evicted
    assert out[4:7] == ["S 0", "S -1", "S 1"]
    s = stats(out[7])
    assert (s["requests"], s["hits"], s["misses"], s["evictions"]) == (4, 1, 3, 1)


def test_call_experts_are_not_victims(driver):
    """A call needing more experts than the cache holds evicts none of its
    own: capacity 2 + scratch 1 serve 3 experts at once."""
    out = run(driver, ["config 2 1 1", demand(0, [4, 5]), demand(0, [1, 4, 5]), "stats"])
    assert out[0] == "D 0 1 | 4:0 5:1 |"
    # 4 and 5 are hits; 1 cannot displace either of them: a scratch load.
    assert out[1] == "D 2 0 1 | 1:2 |"
    s = stats(out[2])
    assert (s["hits"], s["misses"], s["scratch_loads"], s["evictions"]) == (2, 3, 1, 0)


def test_too_many_experts_fail(driver):
    """A call whose experts do not fit at once fails, and the experts it had
    admitted are not left behind as resident (nothing was copied)."""
    out = run(driver, ["config 2 1 0", demand(0, [1, 2, 3, 4]), "slot 0 1", "slot 0 2", "stats",
                       demand(0, [1, 2]), "stats"])
    assert out[0] == "D fail"
    assert out[1:3] == ["S -1", "S -1"]
    assert stats(out[3])["cached"] == 0
    assert out[4] == "D 0 1 | 1:0 2:1 |"


def test_lfru_admission_margin(driver):
    """LFRU: a cold expert does not displace a hot one until its score beats
    the victim's by a quarter plus 4 << 8 (expert.rs:321-331); meanwhile it is
    served from a scratch slot."""
    script = ["config 1 1 0"] + [demand(0, [1])] * 5 + [demand(0, [2])] + ["heat 0 1", "heat 0 2", "slot 0 2",
                                                                          "stats"]
    out = run(driver, script)
    assert out[5] == "D 1 | 2:1 |"   # scratch slot 1, expert 1 stays
    assert out[6] == "H 5 5" and out[7] == "H 1 6" and out[8] == "S -1"
    s = stats(out[9])
    assert (s["scratch_loads"], s["evictions"], s["misses"]) == (1, 0, 2)
    # Expert 1: heat 5, last use at clock 5. Each call of expert 2 alone
    # raises its heat by one and ages expert 1 by one. At the get of the
    # 11th such call, score(2) = (11 << 8) | 255 = 3071 against
    # score(1) = (5 << 8) | (255 - 11) = 1524, whose margin is
    # 1524 + 381 + 1024 = 2929: admitted, 1 evicted. At the 10th,
    # (10 << 8) | 255 = 2815 does not beat 1525 + 381 + 1024 = 2930.
    script = ["config 1 1 0"] + [demand(0, [1])] * 5 + [demand(0, [2])] * 12 + ["slot 0 1", "slot 0 2", "stats"]
    out = run(driver, script)
    calls = out[5:17]
    assert calls[:10] == ["D 1 | 2:1 |"] * 10
    assert calls[10] == "D 0 | 2:0 |" and calls[11] == "D 0 | |"
    assert out[17:19] == ["S -1", "S 0"]
    s = stats(out[19])
    assert (s["scratch_loads"], s["evictions"], s["hits"]) == (10, 1, 4 + 1)


def test_prefetch_used_wasted_late(driver):
    out = run(driver, ["config 3 0 1", prefetch(0, [1, 2]),
                       demand(0, [1]),            # 1: still landing -> late, wait on its slot
                       "done 0", "done 1",
                       demand(0, [2]),            # 2: landed -> hit, prefetch used
                       prefetch(0, [3]),          # free slot 2
                       prefetch(0, [4]),          # cache full; LRU victim must not be 2 (latest call) -> 1
                       "stats", "slot 0 1", "slot 0 4"])
    assert out[0] == "P 1:0 2:1"
    assert out[1] == "D 0 | | 0"
    assert out[2] == "D 1 | |"
    assert out[3] == "P 3:2"
    # 3's copy has not landed (pending) so it is no victim; 2 is the latest
    # call's; 1 goes.
    assert out[4] == "P 4:0"
    s = stats(out[5])
    assert (s["prefetch_issued"], s["prefetch_used"], s["late"], s["hits"], s["prefetch_wasted"]) == (4, 2, 1, 1, 0)
    assert out[6:8] == ["S -1", "S 0"]
    # 3 evicted without use: a wasted prefetch.
    out = run(driver, ["config 1 0 1", prefetch(0, [3]), "done 0", demand(1, [7]), "stats"])
    assert out[1] == "D 0 | 7:0 |"
    assert stats(out[2])["prefetch_wasted"] == 1


def test_speculative_pool(driver):
    """LFRU with a full cache: a cold prediction is not admitted, so it goes
    to a speculative slot (after the scratch slots); the call that routes to
    it is served from there (prefetch used); a full pool replaces its oldest
    landed guess (prefetch wasted)."""
    hot = ["config 2 1 0 2"] + [demand(0, [1, 2])] * 6
    out = run(driver, hot + [prefetch(0, [5]), "done 3", demand(0, [1, 2, 5]), "stats"])
    assert out[6] == "P 5:3"
    assert out[7] == "D 0 1 3 | |"
    s = stats(out[8])
    assert (s["prefetch_issued"], s["prefetch_used"], s["hits"], s["misses"]) == (1, 1, 10 + 3, 2)
    # two guesses fill the pool; a third replaces the oldest landed one
    out = run(driver, hot + [prefetch(0, [5, 6]), "done 3", prefetch(0, [7]), "stats"])
    assert out[6] == "P 5:3 6:4"
    assert out[7] == "P 7:3"
    assert stats(out[8])["prefetch_wasted"] == 1


def test_speculative_pool_pauses_when_unused(driver):
    """After 128 speculative loads of which fewer than half were used, the
    pool pauses for the next 4096 non-admissible predictions
    (expert.rs:470-487)."""
    script = ["config 1 0 0 1"] + [demand(0, [0])] * 4
    for i in range(129):
        script += [prefetch(0, [1 + i % 50]), "done 1"]
    script += ["stats"]
    out = run(driver, script)
    s = stats(out[-1])
    assert s["spec_pauses"] == 1 and s["prefetch_issued"] == 128 and s["prefetch_wasted"] == 127


def test_decay_halves_heat(driver):
    out = run(driver, ["config 4 0 0"] + [demand(0, [1])] * 5 + [demand(0, [2])] + ["decay", "heat 0 1",
                                                                                   "heat 0 2", "decay", "heat 0 2"])
    assert out[-3].split()[1] == "2" and out[-2].split()[1] == "0" and out[-1].split()[1] == "0"


class RefCache:
    """ExpertStore's rules (expert.rs:305-551) as the GPU serves them: a
    call's experts are resident together and never evict one another;
    non-admitted experts take scratch slots, then forced LRU admissions;
    predictions are loaded only when admitted."""

    def __init__(self, capacity, scratch, lru, spec=0):
        self.cap, self.scr, self.lru, self.nspec = capacity, scratch, lru, spec
        self.spec = []                     # [(key, slot)], oldest first
        self.sslot = [dict(held=False, pending=False, call=0) for _ in range(spec)]
        self.window = [0, 0]               # speculative loads issued, used
        self.paused = 0
        self.slots = [None] * capacity   # slot -> dict(key, prefetched, pending, call)
        self.where = {}
        self.heat, self.last = {}, {}
        self.clock = self.call = 0
        self.need = None
        self.st = dict.fromkeys(STATS, 0)

    def score(self, k):
        last = self.last.get(k, 0)
        if self.lru:
            return last
        age = self.clock - last
        return (self.heat.get(k, 0) << 8) | (0 if age >= 255 else 255 - age)

    def touch(self, k):
        self.clock += 1
        self.heat[k] = self.heat.get(k, 0) + 1
        self.last[k] = self.clock

    def victim(self, k, pf, force):
        cands = [s for s, sl in enumerate(self.slots)
                 if sl is not None and not sl["pending"] and
                 (sl["call"] != self.call if pf else sl["key"] not in self.need)]
        if not cands:
            return None
        best = min(cands, key=lambda s: (self.score(self.slots[s]["key"]), s))
        cs = self.score(self.slots[best]["key"])
        if force or self.lru:
            return best
        return best if self.score(k) > cs + (cs >> 2) + (4 << 8) else None

    def admit(self, k, pf, force=False):
        if None in self.slots:
            s = self.slots.index(None)
        else:
            s = self.victim(k, pf, force)
            if s is None:
                return None
            old = self.slots[s]
            del self.where[old["key"]]
            self.st["evictions"] += 1
            self.st["prefetch_wasted"] += old["prefetched"]
        self.slots[s] = dict(key=k, prefetched=pf, pending=False, call=0)
        self.where[k] = s
        return s

    def demand(self, layer, experts):
        self.call += 1
        self.need = {(layer, e) for e in experts}
        loads, waits, demanded = [], [], set()
        for e in experts:
            k = (layer, e)
            if k in self.where:
                continue
            s = self.admit(k, False)
            if s is not None:
                self.st["misses"] += 1
                demanded.add(e)
                loads.append((e, s))
        ready = [e for e in experts if (layer, e) in self.where and e not in demanded and
                 not self.slots[self.where[(layer, e)]]["pending"]]
        order = ready + [e for e in experts if e not in ready]
        slot = {}
        nxt = self.cap
        for e in order:
            k = (layer, e)
            self.st["requests"] += 1
            self.touch(k)
            if k in self.where:
                sl = self.slots[self.where[k]]
                if sl["prefetched"]:
                    sl["prefetched"] = False
                    self.st["prefetch_used"] += 1
                if e in demanded:
                    pass
                elif not sl["pending"]:
                    self.st["hits"] += 1
                else:
                    self.st["late"] += 1
                    waits.append(self.where[k])
                sl["call"] = self.call
                slot[e] = self.where[k]
                continue
            j = next((j for j, (kk, _) in enumerate(self.spec) if kk == k), None)
            if j is not None:
                s = self.spec[j][1]
                self.spec[j] = self.spec[-1]
                self.spec.pop()
                self.window[1] += 1
                self.st["prefetch_used"] += 1
                ss = self.sslot[s - self.cap - self.scr]
                ss["held"] = False
                ss["call"] = self.call
                if ss["pending"]:
                    self.st["late"] += 1
                    waits.append(s)
                else:
                    self.st["hits"] += 1
                slot[e] = s
                continue
            self.st["misses"] += 1
            s = self.admit(k, False)
            if s is None:
                if nxt < self.cap + self.scr:
                    self.st["scratch_loads"] += 1
                    slot[e] = nxt
                    loads.append((e, nxt))
                    nxt += 1
                    continue
                s = self.admit(k, False, force=True)
                if s is None:
                    for e2, s2 in loads:  # admitted but never copied: dropped
                        if s2 < self.cap:
                            del self.where[self.slots[s2]["key"]]
                            self.slots[s2] = None
                    self.need = None
                    return "D fail"
                self.st["forced"] += 1
            self.slots[s]["call"] = self.call
            slot[e] = s
            loads.append((e, s))
        for e in experts:
            if slot[e] < self.cap:
                self.slots[slot[e]]["call"] = self.call
        self.need = None
        return ("D " + " ".join(str(slot[e]) for e in experts) + " |" +
                "".join(f" {e}:{s}" for e, s in loads) + " |" + "".join(f" {s}" for s in waits))

    def prefetch(self, layer, experts):
        self.need = set()
        loads = []
        for e in experts:
            k = (layer, e)
            if k in self.where:
                continue
            s = self.admit(k, True)
            if s is not None:
                self.st["prefetch_issued"] += 1
                self.slots[s]["pending"] = True
                loads.append((e, s))
                continue
            if self.paused:
                self.paused -= 1
                if self.paused == 0:
                    self.window = [0, 0]
                continue
            if self.nspec == 0 or any(kk == k for kk, _ in self.spec):
                continue
            if self.window[0] >= 128:
                acc = self.window[1] / self.window[0]
                self.window = [0, 0]
                if acc < 0.5:
                    self.st["spec_pauses"] += 1
                    self.paused = 4096
                    continue
            slot = None
            if len(self.spec) < self.nspec:
                slot = next((self.cap + self.scr + j for j, ss in enumerate(self.sslot)
                             if not ss["held"] and ss["call"] != self.call), None)
            else:
                j = next((j for j, (_, s2) in enumerate(self.spec)
                          if not self.sslot[s2 - self.cap - self.scr]["pending"]), None)
                if j is not None:
                    self.st["prefetch_wasted"] += 1
                    slot = self.spec.pop(j)[1]
            if slot is None:
                continue
            ss = self.sslot[slot - self.cap - self.scr]
            ss["held"] = ss["pending"] = True
            self.spec.append((k, slot))
            self.window[0] += 1
            self.st["prefetch_issued"] += 1
            loads.append((e, slot))
        self.need = None
        return "P" + "".join(f" {e}:{s}" for e, s in loads)

    def done(self, s):
        if 0 <= s < self.cap and self.slots[s] is not None:
            self.slots[s]["pending"] = False
        if 0 <= s - self.cap - self.scr < self.nspec:
            self.sslot[s - self.cap - self.scr]["pending"] = False

    def decay(self):
        self.heat = {k: h >> 1 for k, h in self.heat.items() if h >> 1}

    def stats(self):
        st = dict(self.st, cached=sum(sl is not None for sl in self.slots))
        return "T " + " ".join(str(st[k]) for k in STATS)


@pytest.mark.parametrize("lru", [0, 1])
@pytest.mark.parametrize("seed", range(6))
def test_random_traces_match_restatement(driver, lru, seed):
    rnd = random.Random(seed * 2 + lru)
    cap, scr, spec = rnd.randint(2, 10), rnd.randint(0, 4), rnd.randint(0, 3)
    n_exp, layers = rnd.choice([6, 12, 24]), rnd.randint(1, 3)
    ref = RefCache(cap, scr, lru, spec)
    script, want = [f"config {cap} {scr} {lru} {spec}"], []
    for _ in range(300):
        r = rnd.random()
        layer = rnd.randrange(layers)
        if r < 0.55:
            # skewed popularity so that both hits and evictions occur
            m = rnd.randint(1, min(n_exp, cap + scr + 1))
            experts = sorted(set(min(n_exp - 1, int(rnd.paretovariate(1.2)) - 1 + rnd.randrange(3))
                                 for _ in range(m)))
            script.append(demand(layer, experts))
            want.append(ref.demand(layer, experts))
        elif r < 0.75:
            experts = sorted(rnd.sample(range(n_exp), rnd.randint(1, 4)))
            script.append(prefetch(layer, experts))
            want.append(ref.prefetch(layer, experts))
        elif r < 0.93:
            s = rnd.randrange(cap + scr + spec)
            script.append(f"done {s}")
            ref.done(s)
        else:
            script.append("decay")
            ref.decay()
        if rnd.random() < 0.1:
            script.append("stats")
            want.append(ref.stats())
    script.append("stats")
    want.append(ref.stats())
    got = run(driver, script)
    assert len(got) == len(want)
    for i, (g, w) in enumerate(zip(got, want)):
        assert g == w, (i, g, w)
