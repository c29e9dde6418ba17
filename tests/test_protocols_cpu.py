"""The mbarrier hand-off protocols of two warp-specialised kernels, modelled
on the CPU and run under random interleavings (no GPU).

Each model follows its kernel step for step: waits on a barrier phase (the
parity of item j's use of a buffer is (j / buffers) & 1), arrivals, the
tensor core or copy engine completing asynchronously.  Every run must
finish (no deadlock), no wait may target a phase more than one behind the
barrier (parities would alias), and every buffer is read only after it was
written for that item and rewritten only after its readers are done.

  prefill_tc_pipe.cu  softmax warps / converter warps (K and V operands of a
                      tile in two steps) / an MMA-issuing lane taking whichever
                      of S(j), PV(j) is ready / a copy warp; PV(j) is
                      its P-hi products then its P-lo products, with a commit
                      between them; MMAs complete in issue order.
  engine_kernels.cu   gemv_q8_stream_kernel: dot warps / copy producer /
                      chain warp over (row block, chunk) items.
  gemm_q8_tc.cu       gemm_q8_tc_kernel: TMA producer (two groups per stage) /
                      MMA issuer (one TMEM buffer per group) / epilogue warps.
"""
import random

import pytest


class Bar:
    def __init__(self, count):
        self.count, self.pending, self.done = count, count, 0

    def arrive(self):
        self.pending -= 1
        if self.pending == 0:
            self.done += 1
            self.pending = self.count

    def ready(self, use):
        """Has the phase of this barrier's use number `use` completed?"""
        assert self.done <= use + 1, ("parity would alias", self.done, use)
        return self.done >= use + 1


def run_prefill(n_kt, seed, rescale_prob, n_conv=8):
    """prefill_tc_pipe_kernel.  Converter warps turn staged tile j into K and
    V operand tiles of buffer j%2 in two steps: K once S(j-2) has read K of
    that buffer (s_full), V once PV(j-2) has read V (op_empty); k_full and
    v_full tell the issuer.  S(j) needs K(j) and the S columns of its TMEM
    buffer (where P(j-2) hi lives) freed by PV(j-2)'s P-hi products (ph_free);
    PV(j) needs P(j) and V(j).  P(j) lo goes into columns PV(j-2)'s P-lo
    products read, which in-order completion has finished before S(j)."""
    R = random.Random(seed)
    B = {}
    for b in (0, 1):
        for k, c in (("stf", 1), ("ste", n_conv), ("kf", n_conv), ("vf", n_conv), ("ope", 1),
                     ("sf", 1), ("pf", 4), ("phf", 1)):
            B[(k, b)] = Bar(c)
    st = {"stage": {}, "opK": {}, "opV": {}, "S": {}, "P": {}, "Plo": {}, "O": 0,
          "sdone": set(), "phdone": set(), "pvdone": set()}
    mma, cps = [], []
    sm = [{"j": 0, "ph": 0} for _ in range(4)]
    cv = [{"j": 0, "ph": 0} for _ in range(n_conv)]
    iss = {"ns": 0, "np": 0, "staged": 0}
    for j in range(min(2, n_kt)):
        cps.append(j)
        iss["staged"] += 1
    for _ in range(300000):
        acts = []
        for w, s in enumerate(sm):
            j = s["j"]
            if j >= n_kt:
                if s["ph"] == 0 and B[("ope", (n_kt - 1) & 1)].ready((n_kt - 1) >> 1):
                    acts.append(("smfin", w))
                continue
            b = j & 1
            if s["ph"] == 0 and B[("sf", b)].ready(j >> 1):
                acts.append(("smS", w, False))
            elif s["ph"] == 1:
                resc = j > 0 and R.random() < rescale_prob
                if not resc or B[("ope", b ^ 1)].ready((j - 1) >> 1):
                    acts.append(("smP", w, resc))
        for w, s in enumerate(cv):
            j = s["j"]
            if j >= n_kt:
                continue
            if s["ph"] == 0 and B[("stf", j & 1)].ready(j >> 1) and \
                    (j < 2 or B[("sf", j & 1)].ready((j - 2) >> 1)):
                acts.append(("cvK", w))
            elif s["ph"] == 1 and (j < 2 or B[("ope", j & 1)].ready((j - 2) >> 1)):
                acts.append(("cvV", w))
        ns, np_, sg = iss["ns"], iss["np"], iss["staged"]
        if ns < n_kt and ns <= np_ + 1 and B[("kf", ns & 1)].ready(ns >> 1) and \
                (ns < 2 or B[("phf", ns & 1)].ready((ns - 2) >> 1)):
            acts.append(("S",))
        if np_ < ns and B[("pf", np_ & 1)].ready(np_ >> 1) and B[("vf", np_ & 1)].ready(np_ >> 1):
            acts.append(("PV",))
        if sg < n_kt and B[("ste", sg & 1)].ready((sg - 2) >> 1):
            acts.append(("stage",))
        if mma:
            acts.append(("mma",))
        acts += [("cp",)] * len(cps)
        if not acts:
            finished = np_ >= n_kt and all(s["ph"] == 2 for s in sm) and not mma and not cps
            return "ok" if finished else "deadlock"
        a = R.choice(acts)
        if a[0] == "smS":
            w = a[1]
            j = sm[w]["j"]
            assert st["S"].get((j & 1, w)) == ("S", j)
            sm[w]["ph"] = 1
        elif a[0] == "smP":
            w, j = a[1], sm[a[1]]["j"]
            if a[2]:
                assert st["O"] == j  # O holds PV(0..j-1) when it is rescaled
            assert j < 2 or (j - 2) in st["pvdone"]  # PV(j-2) has read P lo
            st["P"][(j & 1, w)] = j
            st["S"][(j & 1, w)] = ("P", j)
            st["Plo"][(j & 1, w)] = j
            B[("pf", j & 1)].arrive()
            sm[w]["j"] += 1
            sm[w]["ph"] = 0
        elif a[0] == "smfin":
            assert st["O"] == n_kt
            sm[a[1]]["ph"] = 2
        elif a[0] == "cvK":
            w, j = a[1], cv[a[1]]["j"]
            assert st["stage"].get(j & 1) == j
            assert j < 2 or (j - 2) in st["sdone"]  # S(j-2) has read this K buffer
            st["opK"][(j & 1, w)] = j
            B[("kf", j & 1)].arrive()
            cv[w]["ph"] = 1
        elif a[0] == "cvV":
            w, j = a[1], cv[a[1]]["j"]
            assert st["stage"].get(j & 1) == j
            assert j < 2 or (j - 2) in st["pvdone"]  # PV(j-2) has read this V buffer
            st["opV"][(j & 1, w)] = j
            B[("ste", j & 1)].arrive()
            B[("vf", j & 1)].arrive()
            cv[w]["j"] += 1
            cv[w]["ph"] = 0
        elif a[0] == "S":
            j = iss["ns"]
            assert all(st["opK"].get((j & 1, w)) == j for w in range(n_conv))
            assert all(st["P"].get((j & 1, w)) in (None, j - 2) for w in range(4))
            # S(j) writes the S columns: the products that read P(j-2) hi there
            # must have completed, not merely be queued ahead of it
            assert ("PVh", j - 2) not in mma
            mma.append(("S", j))
            iss["ns"] += 1
        elif a[0] == "PV":
            j = iss["np"]
            assert all(st["P"].get((j & 1, w)) == j for w in range(4))
            assert all(st["opV"].get((j & 1, w)) == j for w in range(n_conv))
            mma.append(("PVh", j))
            mma.append(("PVl", j))
            iss["np"] += 1
        elif a[0] == "stage":
            cps.append(iss["staged"])
            iss["staged"] += 1
        elif a[0] == "mma":  # the tensor core completes in issue order
            kind, j = mma.pop(0)
            if kind == "S":
                # its operands were not rewritten while it was in flight
                assert all(st["opK"].get((j & 1, w)) == j for w in range(n_conv))
                assert j < 2 or (j - 2) in st["phdone"]  # P(j-2) hi was read
                for w in range(4):
                    st["S"][(j & 1, w)] = ("S", j)
                st["sdone"].add(j)
                B[("sf", j & 1)].arrive()
            elif kind == "PVh":  # Phi Vhi + Phi Vlo, then the ph_free commit
                assert all(st["opV"].get((j & 1, w)) == j for w in range(n_conv))
                assert all(st["S"].get((j & 1, w)) == ("P", j) for w in range(4))
                st["phdone"].add(j)
                B[("phf", j & 1)].arrive()
            else:  # Plo Vhi, then the op_empty commit
                assert all(st["opV"].get((j & 1, w)) == j for w in range(n_conv))
                assert all(st["Plo"].get((j & 1, w)) == j for w in range(4))
                assert st["O"] == j
                st["O"] = j + 1
                st["pvdone"].add(j)
                B[("ope", j & 1)].arrive()
        else:  # a copy lands (copies complete in any order)
            j = cps.pop(R.randrange(len(cps)))
            st["stage"][j & 1] = j
            B[("stf", j & 1)].arrive()
    return "livelock"


def run_gemv(items, seed, n_stages=3, n_dot=8):
    R = random.Random(seed)
    full = [Bar(1) for _ in range(n_stages)]
    empty = [Bar(n_dot) for _ in range(n_stages)]
    ready = [Bar(n_dot), Bar(n_dot)]
    done = [Bar(1), Bar(1)]
    stage, tab = {}, {}
    dots = [0] * n_dot
    chain = 0
    issued = min(n_stages, items)
    cps = list(range(issued))
    for _ in range(200000):
        acts = []
        for w in range(n_dot):
            it = dots[w]
            if it < items and full[it % n_stages].ready(it // n_stages) and \
                    (it < 2 or done[it & 1].ready((it - 2) >> 1)):
                acts.append(("dot", w))
        if issued < items and empty[issued % n_stages].ready((issued - n_stages) // n_stages):
            acts.append(("issue",))
        if chain < items and ready[chain & 1].ready(chain >> 1):
            acts.append(("chain",))
        acts += [("cp",)] * len(cps)
        if not acts:
            return "ok" if chain == items and all(d == items for d in dots) else "deadlock"
        a = R.choice(acts)
        if a[0] == "dot":
            w, it = a[1], dots[a[1]]
            assert stage.get(it % n_stages) == it  # the stage holds this item
            assert tab.get((it & 1, w)) in (None, it - 2)  # the chain consumed the last use
            tab[(it & 1, w)] = it
            empty[it % n_stages].arrive()
            ready[it & 1].arrive()
            dots[w] += 1
        elif a[0] == "issue":
            assert all(d > issued - n_stages for d in dots)  # nobody still reads the stage
            cps.append(issued)
            issued += 1
        elif a[0] == "chain":
            assert all(tab.get((chain & 1, w)) == chain for w in range(n_dot))
            done[chain & 1].arrive()
            chain += 1
        else:
            it = cps.pop(R.randrange(len(cps)))
            stage[it % n_stages] = it
            full[it % n_stages].arrive()
    return "livelock"


def run_gemm_tc(ng, seed, n_stages=4, n_buf=4, n_epi=8):
    """gemm_q8_tc_kernel.  The producer loads K slice c (groups 2c, 2c+1)
    into stage c % S once the MMAs of slice c - S have completed (empty);
    the issuer, for group g, waits for its slice (full, at even g) and for
    the epilogue to have read buffer g % NB's previous group (dempty), then
    issues two products into that buffer and commits dfull, and commits
    empty after a slice's last group; the epilogue warps read each group's
    buffer in order and release it."""
    R = random.Random(seed)
    nch = (ng + 1) // 2
    B = {}
    for s_ in range(n_stages):
        B[("full", s_)] = Bar(1)
        B[("empty", s_)] = Bar(1)
    for b in range(n_buf):
        B[("dfull", b)] = Bar(1)
        B[("dempty", b)] = Bar(n_epi)
    stage, tmem = {}, {}
    mma, cps = [], []
    prod = {"c": 0}
    iss = {"g": 0}
    epi = [0] * n_epi
    for _ in range(200000):
        acts = []
        c = prod["c"]
        if c < nch and (c < n_stages or B[("empty", c % n_stages)].ready(c // n_stages - 1)):
            acts.append(("copy",))
        g = iss["g"]
        if g < ng:
            cc, b = g >> 1, g % n_buf
            ok = (g & 1) or B[("full", cc % n_stages)].ready(cc // n_stages)
            if ok and (g < n_buf or B[("dempty", b)].ready(g // n_buf - 1)):
                acts.append(("mma",))
        for w in range(n_epi):
            ge = epi[w]
            if ge < ng and B[("dfull", ge % n_buf)].ready(ge // n_buf):
                acts.append(("epi", w))
        if mma:
            acts.append(("done",))
        acts += [("land",)] * len(cps)
        if not acts:
            ok = iss["g"] >= ng and all(e >= ng for e in epi) and not mma and not cps
            return "ok" if ok else "deadlock"
        a = R.choice(acts)
        if a[0] == "copy":
            c = prod["c"]
            # the slice this copy overwrites has no product in flight
            assert all(k != ("slice", c - n_stages) for k in mma)
            cps.append(c)
            prod["c"] += 1
        elif a[0] == "land":
            c = cps.pop(R.randrange(len(cps)))
            stage[c % n_stages] = c
            B[("full", c % n_stages)].arrive()
        elif a[0] == "mma":
            g = iss["g"]
            cc, b = g >> 1, g % n_buf
            assert stage.get(cc % n_stages) == cc  # its slice has landed
            mma.append(("group", g))
            if (g & 1) or g == ng - 1:
                mma.append(("slice", cc))
            iss["g"] += 1
        elif a[0] == "done":  # products complete in issue order
            kind, v = mma.pop(0)
            if kind == "group":
                b = v % n_buf
                # the buffer's previous group was read by every epilogue warp
                assert all(e >= v - n_buf + 1 for e in epi)
                assert stage.get((v >> 1) % n_stages) == v >> 1
                tmem[b] = v
                B[("dfull", b)].arrive()
            else:
                B[("empty", v % n_stages)].arrive()
        else:
            w = a[1]
            ge = epi[w]
            assert tmem.get(ge % n_buf) == ge
            epi[w] += 1
            B[("dempty", ge % n_buf)].arrive()
    return "livelock"


@pytest.mark.parametrize("ng", [1, 2, 3, 4, 5, 8, 9, 17])
def test_gemm_tc_protocol(ng):
    for seed in range(200):
        assert run_gemm_tc(ng, seed) == "ok", (ng, seed)


@pytest.mark.parametrize("n_kt", [1, 2, 3, 4, 7, 10])
def test_prefill_pipeline_protocol(n_kt):
    for seed in range(150):
        for rp in (0.0, 0.5, 1.0):
            assert run_prefill(n_kt, seed, rp) == "ok", (n_kt, seed, rp)


@pytest.mark.parametrize("items", [1, 2, 3, 4, 5, 9, 16])
def test_gemv_stream_protocol(items):
    for seed in range(300):
        assert run_gemv(items, seed) == "ok", (items, seed)
