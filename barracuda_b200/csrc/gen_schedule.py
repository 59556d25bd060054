"""Generates bc_schedule.hpp: the pass schedules of the register/shared-memory
/cluster NTT kernels, and checks them.

A transform of N = 2^L points runs as a few *passes*.  A pass owns a group
of position bits [lo, hi]: every thread holds E = 2^loge coefficients in
registers whose positions differ in those bits (plus `extra` bits below lo
when the group is narrower than loge), and runs the hi-lo+1 butterfly
stages of that group in registers.  Between passes the coefficients go
through shared memory; with a thread-block cluster of C = 2^logc CTAs, the
polynomial is spread over the CTAs' shared memories and one exchange (the
phase change) goes through distributed shared memory.

Per phase the CTA of cluster rank r owns the positions whose `rank` bits
spell r.  Within a phase, every other position bit has a *local* bit index
(a per-phase permutation chosen here), and the coefficient of position p
lives in shared-memory word swz(local(p)) with
swz(x) = x + (x >> 5) + (x >> 10) + (x >> 15) (one pad word per 32, 1024,
32768).  Local bit i moves the word by 2^(i mod 5) banks, so a warp access
is free of bank conflicts when its lanes vary bits whose local indices have
distinct residues mod 5 (a small search picks the local orders); lanes of
a pass are listed in residue order.  The guarantee is for 32-bit words: the
64-bit-word path (moduli >= 2^31) may see 2-way conflicts.  swz is additive
over disjoint bit sets, so every access is a per-thread base plus a
compile-time offset.

Lanes and warps: when pass B follows pass A in the same phase, the first
puts the register bits that B adds in its lanes and the second puts the
register bits that A drops in its lanes (both plus common bits x, when fewer
than five bits change); both keep the same warp bits, so the data they
exchange never leaves a warp and the pass boundary needs only __syncwarp().
Passes that cannot be paired that way exchange through the whole CTA
(__syncthreads()).

Global memory is read and written by separate cooperative stages (16-byte
accesses of coefficient pairs in natural order), whose shared-memory
accesses are constrained the same way.  Gentleman-Sande transforms run the
passes in reverse order.

    python barracuda_b200/csrc/gen_schedule.py   # rewrites bc_schedule.hpp
"""
from __future__ import annotations

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "bc_schedule.hpp")

# (L, variant): (loge, logc, passes [(hi, lo, extras)], rank bits phase 0, rank bits phase 1, split)
# Variants: 4 = 16 coefficients per thread (512-thread CTAs of 2^13 words);
# 5 = 32 per thread (CTAs of up to 2^14 words); 6 = 32 per thread in
# 256-thread CTAs of 2^13 words (more, smaller CTAs per SM); 7 = 32 per
# thread in 128-thread CTAs of 2^12 words.  Clusters of 16 CTAs (L=17 V6,
# L=16 V7) are a non-portable size that B200 allows.
# `split` = number of passes in phase 0 (the remaining passes are phase 1).
CONFIGS = {
    (10, 5): (5, 0, [(9, 5, []), (4, 0, [])], [], [], 2),
    (11, 5): (5, 0, [(10, 10, [0, 1, 2, 3]), (9, 5, []), (4, 0, [])], [], [], 3),
    (12, 5): (5, 0, [(11, 10, [0, 1, 2]), (9, 5, []), (4, 0, [])], [], [], 3),
    (13, 5): (5, 0, [(12, 10, [0, 1]), (9, 5, []), (4, 0, [])], [], [], 3),
    (14, 5): (5, 0, [(13, 10, [0]), (9, 5, []), (4, 0, [])], [], [], 3),
    (15, 5): (5, 1, [(14, 10, []), (9, 5, []), (4, 0, [])], [9], [10], 1),
    (16, 5): (5, 2, [(15, 13, [0, 1]), (12, 8, []), (7, 5, [0, 1]), (4, 0, [])], [6, 7], [8, 9], 2),
    (17, 5): (5, 3, [(16, 13, [0]), (12, 8, []), (7, 5, [0, 1]), (4, 0, [])], [5, 6, 7], [8, 9, 10], 2),
    (14, 6): (5, 1, [(13, 10, [0]), (9, 5, []), (4, 0, [])], [9], [10], 1),
    (15, 6): (5, 2, [(14, 10, []), (9, 5, []), (4, 0, [])], [8, 9], [10, 11], 1),
    (16, 6): (5, 3, [(15, 13, [0, 1]), (12, 8, []), (7, 5, [0, 1]), (4, 0, [])], [5, 6, 7], [8, 9, 10], 2),
    (17, 6): (5, 4, [(16, 13, [0]), (12, 8, []), (7, 5, [0, 1]), (4, 0, [])], [4, 5, 6, 7], [8, 9, 10, 11], 2),
    (16, 7): (5, 4, [(15, 13, [0, 1]), (12, 8, []), (7, 5, [0, 1]), (4, 0, [])], [4, 5, 6, 7], [8, 9, 10, 11], 2),
    (10, 4): (4, 0, [(9, 8, [0, 1]), (7, 4, []), (3, 0, [])], [], [], 3),
    (11, 4): (4, 0, [(10, 8, [0]), (7, 4, []), (3, 0, [])], [], [], 3),
    (12, 4): (4, 0, [(11, 8, []), (7, 4, []), (3, 0, [])], [], [], 3),
    (13, 4): (4, 0, [(12, 12, [0, 1, 2]), (11, 8, []), (7, 4, []), (3, 0, [])], [], [], 4),
    (14, 4): (4, 1, [(13, 12, [0, 1]), (11, 8, []), (7, 4, []), (3, 0, [])], [6], [8], 2),
    (15, 4): (4, 2, [(14, 12, [0]), (11, 8, []), (7, 4, []), (3, 0, [])], [5, 6], [8, 9], 2),
    (16, 4): (4, 3, [(15, 12, []), (11, 8, []), (7, 4, []), (3, 0, [])], [5, 6, 7], [8, 9, 10], 2),
    (17, 4): (4, 4, [(16, 16, [0, 1, 2]), (15, 12, []), (11, 8, []), (7, 4, []), (3, 0, [])],
              [4, 5, 6, 7], [8, 9, 10, 11], 3),
}


class Pass:
    def __init__(self, hi, lo, extras):
        self.hi, self.lo, self.extras = hi, lo, list(extras)
        self.bits = list(range(lo, hi + 1))
        self.reg = self.bits + self.extras  # m bit j <-> position bit reg[j]
        self.lanes = []
        self.warps = []
        self.rank = []
        self.phase = 0
        self.sync_after = "block"  # exchange to the next pass (CT order): warp/block/cluster


def swz(x):
    """Padded shared-memory word of local index x."""
    return x + (x >> 5) + (x >> 10) + (x >> 15)


def free_bits(L, rank):
    return [b for b in range(L) if b not in rank]


# ----------------------------------------------------------------- lanes

def lane_options(L, loge, logc, passes, rank0, rank1, split, pair=True):
    """Per pass: its phase, rank bits, sync kind, and the candidate lane sets
    (paired passes share the extra bit x)."""
    import itertools
    n = len(passes)
    phase = [0 if i < split else 1 for i in range(n)]
    ranks = [rank0 if phase[i] == 0 else rank1 for i in range(n)]
    thread_bits = []
    for i, p in enumerate(passes):
        tb = [b for b in range(L) if b not in p.reg and b not in ranks[i]]
        assert len(tb) == L - logc - loge
        thread_bits.append(tb)
        p.rank = ranks[i]
        p.phase = phase[i]
        p.sync_after = "block"
        if logc and i == split - 1:
            p.sync_after = "cluster"
    # pair passes (i, i+1) of the same phase: the register bits that pass
    # i+1 adds (new_b) are lanes of pass i, the ones it drops (new_a) are
    # lanes of pass i+1, both keep the same warp bits and share the other
    # lanes xs -- then the data they exchange never leaves a warp.
    units = []  # (pass indices, list of candidate lane tuples per index)
    i = 0
    while i < n:
        if pair and i + 1 < n:
            a, b = passes[i], passes[i + 1]
            new_b = [x for x in b.reg if x not in a.reg]
            new_a = [x for x in a.reg if x not in b.reg]
            if (phase[i] == phase[i + 1] and len(new_b) == len(new_a) <= 5
                    and all(x in thread_bits[i] for x in new_b)):
                common = sorted(x for x in thread_bits[i] if x in thread_bits[i + 1])
                k = 5 - len(new_b)
                if len(common) >= k:
                    cands = [(tuple(new_b) + xs, tuple(new_a) + xs) for xs in itertools.combinations(common, k)]
                    units.append(((i, i + 1), cands))
                    a.sync_after = "warp"
                    i += 2
                    continue
        cands = [(c,) for c in itertools.combinations(sorted(thread_bits[i]), 5)]
        units.append(((i,), cands))
        i += 1
    # The passes on either side of the phase change store into the other
    # phase's layout (CT: pass split-1 into phase 1, GS: pass split into
    # phase 0), so their lanes must be local bits there too.
    if logc:
        avoid = {split - 1: set(rank1), split: set(rank0)}
        units = [(idx, [c for c in cands
                        if all(not (set(ln) & avoid.get(j, set())) for j, ln in zip(idx, c))])
                 for idx, cands in units]
    return units, thread_bits


# ------------------------------------------------------- local bit orders

def access_sets(L, logc, passes, split):
    """(phase, lane bits, fixed, remote) of every shared-memory access
    pattern; `fixed` accesses keep their lane order (the cooperative
    stages), the lane order of passes is free; `remote` marks the stores
    of the phase change into another CTA's shared memory."""
    sets = []
    for i, p in enumerate(passes):
        sets.append((p.phase, p, False, False))
        if logc and p.sync_after == "cluster":
            sets.append((1 - p.phase, p, False, True))  # CT: remote write into the next phase
        if logc and i == split:
            sets.append((0, p, False, True))  # GS: pass `split` writes into phase 0
    sets.append((passes[0].phase, coop_lanes(L, passes[0].rank, True), True, False))
    sets.append((passes[-1].phase, coop_lanes(L, passes[-1].rank, False), True, False))
    return sets


def solve_orders(L, rank0, rank1, sets, passes):
    """Per phase, give the non-rank bits local indices (residues mod 5) so
    that every access varies 5 bits of distinct residues; then list the
    lanes of every pass in residue order.

    Within a residue class the slot is free (only residues decide banks).
    The lanes of the remote store into a phase take the lowest slot of
    their classes, i.e. local indices 0..4: a warp's distributed-shared-
    memory store then covers 32 consecutive words (4-5 sectors) instead of
    up to 32 scattered sectors."""
    out = {}
    for ph, rank in ((0, rank0), (1, rank1)):
        bits = free_bits(L, rank)
        nloc = len(bits)
        cap = [len([i for i in range(nloc) if i % 5 == r]) for r in range(5)]
        groups, pinned, first = [], {}, []
        for s_ph, acc, fixed, remote in sets:
            if s_ph != ph:
                continue
            lanes = acc if fixed else acc.lanes
            for b in lanes:
                assert b not in rank, ("lane on a rank bit", L, ph)
            groups.append(list(lanes))
            if remote:
                first += [b for b in lanes if b not in first]
        involved = sorted({b for g in groups for b in g}, key=lambda b: -sum(b in g for g in groups))
        res = dict(pinned)
        used = [0] * 5
        for b, r in res.items():
            used[r] += 1

        def ok(b, r):
            if used[r] >= cap[r]:
                return False
            for g in groups:
                if b in g and any(res.get(x) == r for x in g if x != b):
                    return False
            return True

        def bt(k):
            if k == len(involved):
                return True
            b = involved[k]
            if b in res:
                return bt(k + 1)
            for r in range(5):
                if ok(b, r):
                    res[b] = r
                    used[r] += 1
                    if bt(k + 1):
                        return True
                    used[r] -= 1
                    del res[b]
            return False

        if not bt(0):
            return None
        slots = {r: [i for i in range(nloc) if i % 5 == r] for r in range(5)}
        order = {}
        for b in first + sorted(b for b in res if b not in first):
            order[b] = slots[res[b]].pop(0)
        rest = sorted(i for r in range(5) for i in slots[r])
        for b in bits:
            if b not in order:
                order[b] = rest.pop(0)
        assert sorted(order.values()) == list(range(nloc))
        out[ph] = order
    # lane order of each pass: residue j on lane j in its own phase
    for p in passes:
        o = out[p.phase]
        p.lanes = sorted(p.lanes, key=lambda b: o[b] % 5)
    return out


def coop_lanes(L, rank, nat):
    """Lane bits (as position bits) of the cooperative global stages: thread
    tid moves natural-order elements 2*tid (+ j*2T), i.e. its lanes vary
    element-index bits 1..5."""
    mirrored = [L - 1 - b for b in rank]
    free_nat = [b for b in range(L) if b not in (rank if nat else mirrored)]
    lane_nat = free_nat[1:6]
    return lane_nat if nat else [L - 1 - b for b in lane_nat]


def build(L, variant):
    loge, logc, passes_spec, rank0, rank1, split = CONFIGS[(L, variant)]
    logt = L - logc - loge
    assert logt >= 5, (L, loge, logc)
    passes = [Pass(*p) for p in passes_spec]
    assert len(rank0) == logc and len(rank1) == logc
    seen = []
    for p in passes:
        assert p.hi >= p.lo and p.hi - p.lo + 1 + len(p.extras) == loge, (L, p.hi, p.lo)
        seen += list(range(p.hi, p.lo - 1, -1))
        for x in p.extras:
            assert x < p.lo, "extra register bits must lie below the pass"
    assert seen == list(range(L - 1, -1, -1)), seen
    import itertools
    orders = None
    for pair in (True, False):  # warp-local exchanges where a layout allows them
        units, thread_bits = lane_options(L, loge, logc, passes, rank0, rank1, split, pair)
        for tries, choice in enumerate(itertools.product(*[c for _, c in units])):
            for (idx, _), lanes in zip(units, choice):
                for i, ln in zip(idx, lanes):
                    passes[i].lanes = list(ln)
                    passes[i].warps = [x for x in sorted(thread_bits[i]) if x not in ln]
            orders = solve_orders(L, rank0, rank1, access_sets(L, logc, passes, split), passes)
            if orders is not None or tries > 20000:
                break
        if orders is not None:
            break
    assert orders is not None, ("no bank-conflict-free schedule", L, loge, logc)
    s = dict(L=L, variant=variant, loge=loge, logc=logc, logt=logt, passes=passes, split=split,
             rank0=rank0, rank1=rank1, orders=orders)
    check(s)
    return s


# ----------------------------------------------------------------- checks

def local_index(p, order):
    return sum(((p >> b) & 1) << k for b, k in order.items())


def positions(ps, rank_val, t, m):
    p = 0
    for j, b in enumerate(ps.reg):
        p |= ((m >> j) & 1) << b
    for j, b in enumerate(ps.lanes):
        p |= ((t >> j) & 1) << b
    for j, b in enumerate(ps.warps):
        p |= ((t >> (5 + j)) & 1) << b
    for j, b in enumerate(ps.rank):
        p |= ((rank_val >> j) & 1) << b
    return p


def conflict_free(addrs):
    """32 word addresses of one warp access hit 32 distinct banks (32-bit
    words).  64-bit words (the q >= 2^31 path) may see 2-way conflicts."""
    return len({a & 31 for a in addrs}) == 32


def check(s):
    """Bijectivity, warp-locality of paired exchanges, conflict-free shared
    memory for every access, and coverage of the cooperative stages."""
    L, loge, logc, passes, split = s["L"], s["loge"], s["logc"], s["passes"], s["split"]
    E, C, T = 1 << loge, 1 << logc, 1 << s["logt"]
    orders = s["orders"]
    for i, ps in enumerate(passes):
        covered = set()
        for r in range(C):
            for t in range(T):
                for m in range(E):
                    covered.add(positions(ps, r, t, m))
        assert len(covered) == 1 << L, ("not a bijection", L, i)
        layouts = [(orders[ps.phase], False)]
        if logc and ps.sync_after == "cluster":
            layouts.append((orders[1 - ps.phase], True))
        if logc and i == split:
            layouts.append((orders[0], True))
        for order, remote in layouts:
            for w in range(min(T // 32, 4)):
                for m in range(E):
                    addrs = [swz(local_index(positions(ps, 0, w * 32 + l, m), order)) for l in range(32)]
                    assert conflict_free(addrs), ("bank conflict", L, loge, i)
                    if remote:  # 32 consecutive 4-byte words: at most 5 32-byte sectors
                        assert len({a >> 3 for a in addrs}) <= 5, ("scattered remote store", L, loge, i)
        if ps.sync_after == "warp":
            nxt = passes[i + 1]
            for r in range(C):
                for w in range(T // 32):
                    wrote = {positions(ps, r, w * 32 + l, m) for l in range(32) for m in range(E)}
                    read = {positions(nxt, r, w * 32 + l, m) for l in range(32) for m in range(E)}
                    assert wrote == read, ("exchange leaves the warp", L, loge, i)
    check_coop(s)


def check_coop(s):
    L, loge, logc, passes = s["L"], s["loge"], s["logc"], s["passes"]
    C, T = 1 << logc, 1 << s["logt"]
    local = 1 << (L - logc)
    for ps, nat in ((passes[0], True), (passes[-1], False)):
        rank = ps.rank
        order = s["orders"][ps.phase]
        mirrored = [L - 1 - b for b in rank]
        free_nat = [b for b in range(L) if b not in (rank if nat else mirrored)]
        for r in range(C):
            seen = set()
            for j in range(local // (2 * T)):
                for w in range(T // 32):
                    addrs = [[], []]
                    for lane in range(32):
                        i = 2 * (w * 32 + lane) + 2 * j * T
                        for e in range(2):
                            k = sum((((i + e) >> n) & 1) << b for n, b in enumerate(free_nat))
                            rb = rank if nat else mirrored
                            k |= sum(((r >> n) & 1) << b for n, b in enumerate(rb))
                            p = k if nat else int(format(k, f"0{L}b")[::-1], 2)
                            seen.add(p)
                            addrs[e].append(swz(local_index(p, order)))
                    assert all(conflict_free(a) for a in addrs), ("coop bank conflict", L, loge, nat)
            owned = {p for p in range(1 << L)
                     if all(((p >> b) & 1) == ((r >> n) & 1) for n, b in enumerate(rank))}
            assert seen == owned, ("coop coverage", L, loge, nat)


# ------------------------------------------------------------------- emit

def emit(scheds):
    out = ["// Generated by gen_schedule.py -- pass schedules of the fast NTT kernels.",
           "// Do not edit by hand: change CONFIGS in gen_schedule.py and rerun it.",
           "#pragma once", "", "namespace bc {", "namespace fast {", "",
           "enum SyncKind { kSyncWarp = 0, kSyncBlock = 1, kSyncCluster = 2 };", "",
           "struct PassDesc {",
           "    int hi, lo;       // processed position bits (inclusive)",
           "    int nreg;         // register bits: hi-lo+1 processed, then extras",
           "    int reg[5];       // register index bit j <-> position bit reg[j]",
           "    int lane[5];      // lane bit j <-> position bit lane[j]",
           "    int nwarp;",
           "    int warp[10];     // warp index bit j <-> position bit warp[j]",
           "    int phase;        // 0 or 1 (which rank bits the CTA owns)",
           "    int sync_after;   // exchange with the next pass in CT order (SyncKind)",
           "};", "",
           "struct BitTable {",
           "    int b[18];",
           "};", "",
           "template <int L, int V> struct Sched;", ""]
    sync = {"warp": 0, "block": 1, "cluster": 2}
    for s in scheds:
        L, loge, logc = s["L"], s["loge"], s["logc"]
        ps = s["passes"]

        def arr(v, n):
            v = list(v) + [0] * (n - len(v))
            return "{" + ", ".join(str(x) for x in v) + "}"

        def order_table(ph):
            o = s["orders"][ph]
            return arr([o.get(b, -1) for b in range(L)], 18)
        out.append(f"template <> struct Sched<{L}, {s['variant']}> {{")
        out.append(f"    static constexpr int kLogE = {loge}, kLogC = {logc}, kLogT = {s['logt']}, kPasses = {len(ps)}, "
                   f"kSplit = {s['split']};")
        out.append(f"    __host__ __device__ static constexpr int rank0(int j) {{ return BitTable{{{arr(s['rank0'], 18)}}}.b[j]; }}")
        out.append(f"    __host__ __device__ static constexpr int rank1(int j) {{ return BitTable{{{arr(s['rank1'], 18)}}}.b[j]; }}")
        out.append("    // local bit index of position bit b in phase 0 / 1 (-1: a rank bit)")
        out.append(f"    __host__ __device__ static constexpr int local0(int b) {{ return BitTable{{{order_table(0)}}}.b[b]; }}")
        out.append(f"    __host__ __device__ static constexpr int local1(int b) {{ return BitTable{{{order_table(1)}}}.b[b]; }}")
        out.append("    __host__ __device__ static constexpr PassDesc pass(int i) {")
        for i, p in enumerate(ps):
            out.append(f"        if (i == {i}) return PassDesc{{{p.hi}, {p.lo}, {len(p.reg)}, {arr(p.reg, 5)}, "
                       f"{arr(p.lanes, 5)}, {len(p.warps)}, {arr(p.warps, 10)}, {p.phase}, {sync[p.sync_after]}}};")
        out.append("        return PassDesc{};")
        out.append("    }")
        out.append("};")
        out.append("")
    out.append("// hi bit of the pass that processes position bit b in schedule (L, V)")
    out.append("__host__ __device__ constexpr int sched_pass_hi(int L, int V, int b) {")
    for s in scheds:
        conds = " : ".join(f"b >= {p.lo} ? {p.hi}" for p in s["passes"])
        out.append(f"    if (L == {s['L']} && V == {s['variant']}) return {conds} : -1;")
    out.append("    return -1;")
    out.append("}")
    out.append("")
    out.append("// log2 of the cluster size of schedule (L, V); -1 if there is none")
    out.append("__host__ __device__ constexpr int sched_logc(int L, int V) {")
    for s in scheds:
        out.append(f"    if (L == {s['L']} && V == {s['variant']}) return {s['logc']};")
    out.append("    return -1;")
    out.append("}")
    out.append("")
    out += ["}  // namespace fast", "}  // namespace bc", ""]
    return "\n".join(out)


def all_schedules():
    return [build(*k) for k in sorted(CONFIGS)]


def main():
    scheds = all_schedules()
    for s in scheds:
        kinds = [p.sync_after for p in s["passes"][:-1]]
        print(f"L={s['L']:2d} V={s['variant']} E={1 << s['loge']:2d} C={1 << s['logc']} T={1 << s['logt']}: "
              f"exchanges {kinds}")
    with open(OUT, "w") as f:
        f.write(emit(scheds))
    print("wrote", OUT)


if __name__ == "__main__":
    sys.exit(main())
