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
spell r.  Its shared-memory word of position p is swz(local(p)): local()
drops the rank bits, swz(x) = x + (x >> 5) + (x >> 10) + (x >> 15) pads the
array.  Local bit i then moves the bank by 2^(i mod 5), so a warp access is
free of bank conflicts whenever its 32 lanes vary 5 position bits whose local
indices are distinct modulo 5; the lane bits of every pass are chosen (and
checked) that way.  swz is additive over disjoint bits, so every access is a
per-thread base plus a compile-time offset.

Lane bits of the first Cooley-Tukey pass are the lowest thread bits
(coalesced loads of natural-order input); lane bits of the last pass are the
highest thread bits, highest first, so that consecutive lanes store
consecutive natural indices bitrev(p).  Gentleman-Sande transforms run the
same passes in reverse order.

    python barracuda_b200/csrc/gen_schedule.py   # rewrites bc_schedule.hpp
"""
from __future__ import annotations

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "bc_schedule.hpp")

# (L, loge, logc): (passes [(hi, lo, extras)], rank bits phase 0, rank bits phase 1, split)
# `split` = number of passes in phase 0 (the remaining passes are phase 1).
CONFIGS = {
    # 32-bit words, 32 coefficients per thread
    (10, 5, 0): ([(9, 5, []), (4, 0, [])], [], [], 2),
    (11, 5, 0): ([(10, 10, [0, 1, 2, 3]), (9, 5, []), (4, 0, [])], [], [], 3),
    (12, 5, 0): ([(11, 10, [0, 1, 2]), (9, 5, []), (4, 0, [])], [], [], 3),
    (13, 5, 0): ([(12, 10, [0, 1]), (9, 5, []), (4, 0, [])], [], [], 3),
    (14, 5, 0): ([(13, 10, [0]), (9, 5, []), (4, 0, [])], [], [], 3),
    (15, 5, 1): ([(14, 10, []), (9, 5, []), (4, 0, [])], [9], [10], 1),
    (16, 5, 2): ([(15, 13, [0, 1]), (12, 8, []), (7, 5, [0, 1]), (4, 0, [])], [6, 7], [8, 9], 2),
    (17, 5, 3): ([(16, 13, [0]), (12, 8, []), (7, 5, [0, 1]), (4, 0, [])], [5, 6, 7], [8, 9, 10], 2),
    # 64-bit words, 16 coefficients per thread
    (10, 4, 0): ([(9, 8, [0, 1]), (7, 4, []), (3, 0, [])], [], [], 3),
    (11, 4, 0): ([(10, 8, [0]), (7, 4, []), (3, 0, [])], [], [], 3),
    (12, 4, 0): ([(11, 8, []), (7, 4, []), (3, 0, [])], [], [], 3),
    (13, 4, 0): ([(12, 12, [0, 1, 2]), (11, 8, []), (7, 4, []), (3, 0, [])], [], [], 4),
    (14, 4, 1): ([(13, 12, [0, 1]), (11, 8, []), (7, 4, []), (3, 0, [])], [6], [8], 2),
    (15, 4, 2): ([(14, 12, [0]), (11, 8, []), (7, 4, []), (3, 0, [])], [5, 6], [8, 9], 2),
    (16, 4, 3): ([(15, 12, []), (11, 8, []), (7, 4, []), (3, 0, [])], [5, 6, 7], [8, 9, 10], 2),
}


class Pass:
    def __init__(self, hi, lo, extras):
        self.hi, self.lo, self.extras = hi, lo, list(extras)
        self.reg = list(range(lo, hi + 1)) + self.extras  # m bit j <-> position bit reg[j]
        self.lanes = []
        self.warps = []


def local_map(L, rank):
    """position bit -> local index bit (rank bits removed)."""
    m, k = {}, 0
    for b in range(L):
        if b in rank:
            continue
        m[b] = k
        k += 1
    return m


def choose_lanes(cands, lmaps, avoid_first=None):
    """5 candidate bits whose local positions are distinct mod 5 in every
    given layout (greedy from the front of `cands`)."""
    import itertools
    for combo in itertools.combinations(cands, 5):
        ok = True
        for lm in lmaps:
            if len({lm[b] % 5 for b in combo}) != 5:
                ok = False
                break
        if ok:
            return list(combo)
    return None


def build(L, loge, logc):
    passes_spec, rank0, rank1, split = CONFIGS[(L, loge, logc)]
    E = 1 << loge
    local_bits = L - logc
    logt = local_bits - loge
    assert logt >= 5, (L, loge, logc)
    passes = [Pass(*p) for p in passes_spec]
    assert len(rank0) == logc and len(rank1) == logc
    # every bit processed exactly once, high to low
    seen = []
    for p in passes:
        assert p.hi >= p.lo and p.hi - p.lo + 1 + len(p.extras) == loge, (L, p.hi, p.lo)
        seen += list(range(p.hi, p.lo - 1, -1))
        for x in p.extras:
            assert x < p.lo, "extra register bits must lie below the pass"
    assert seen == list(range(L - 1, -1, -1)), seen
    n = len(passes)
    for i, p in enumerate(passes):
        rank = rank0 if i < split else rank1
        for b in rank:
            assert b not in p.reg, (L, i, b)
        thread_bits = [b for b in range(L) if b not in p.reg and b not in rank]
        assert len(thread_bits) == logt
        lm_here = local_map(L, rank)
        layouts = [lm_here]
        if logc and i == split - 1:
            layouts.append(local_map(L, rank1))  # remote write lands in phase-1 layout
        if i == 0:
            lanes = sorted(thread_bits)[:5]
        elif i == n - 1:
            lanes = sorted(thread_bits, reverse=True)[:5]
        else:
            lanes = choose_lanes(sorted(thread_bits), layouts)
        assert lanes is not None, (L, i)
        p.lanes = lanes
        p.warps = [b for b in sorted(thread_bits) if b not in lanes]
        p.rank = rank
    check(L, loge, logc, passes, split)
    check_coop(L, loge, logc, passes, split)
    return dict(L=L, loge=loge, logc=logc, logt=logt, passes=passes, split=split,
                rank0=rank0, rank1=rank1)


def swz(x):
    """Padded shared-memory word of local index x: one pad word per 32, per
    1024 and per 32768 words.  Additive over disjoint bit sets, so a word of
    (thread bits | register bits) is thread base + a compile-time offset."""
    return x + (x >> 5) + (x >> 10) + (x >> 15)


def compress(p, lm):
    return sum(((p >> b) & 1) << k for b, k in lm.items())


def positions(L, ps, rank_val, t, m):
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


def check(L, loge, logc, passes, split):
    """Bijectivity, in-CTA ownership and conflict-free shared-memory access."""
    E, C, T = 1 << loge, 1 << logc, 1 << (L - logc - loge)
    for i, ps in enumerate(passes):
        covered = set()
        for r in range(C):
            for t in range(T):
                for m in range(E):
                    covered.add(positions(L, ps, r, t, m))
        assert len(covered) == 1 << L, ("not a bijection", L, i)
        rank = ps.rank
        layouts = [local_map(L, rank)]
        if logc and i == split - 1:
            layouts.append(local_map(L, passes[split].rank))
        for lm in layouts:
            for w in range(min(T // 32, 4)):
                for m in range(E):
                    banks = {swz(compress(positions(L, ps, 0, w * 32 + l, m), lm)) & 31 for l in range(32)}
                    assert len(banks) == 32, ("bank conflict", L, loge, i)


def check_coop(L, loge, logc, passes, split):
    """The cooperative HBM <-> shared-memory stages: thread tid, iteration j
    moves natural indices k, k+1 (k = natural(2*tid + 2*j*T)).  Check that
    every owned coefficient is moved once and that the two 32-bit shared
    accesses of a warp hit 32 distinct banks."""
    C, T = 1 << logc, 1 << (L - logc - loge)
    local = 1 << (L - logc)
    for phase_pass, nat in ((passes[0], True), (passes[-1], False),
                            (passes[-1], True), (passes[0], False)):
        rank = phase_pass.rank
        lm = local_map(L, rank)
        mirrored = [L - 1 - b for b in rank]
        free_nat = [b for b in range(L) if b not in (rank if nat else mirrored)]
        for r in range(C):
            seen = set()
            for j in range(local // (2 * T)):
                for w in range(T // 32):
                    banks = [set(), set()]
                    for lane in range(32):
                        i = 2 * (w * 32 + lane) + 2 * j * T
                        for e in range(2):
                            k = sum(((i + e) >> n & 1) << b for n, b in enumerate(free_nat))
                            rb = rank if nat else mirrored
                            k |= sum(((r >> n) & 1) << b for n, b in enumerate(rb))
                            p = k if nat else int(format(k, f"0{L}b")[::-1], 2)
                            seen.add(p)
                            banks[e].add(swz(compress(p, lm)) & 31)
                    assert all(len(bk) == 32 for bk in banks), ("coop bank conflict", L, loge, nat)
            owned = {p for p in range(1 << L)
                     if all(((p >> b) & 1) == ((r >> n) & 1) for n, b in enumerate(rank))}
            assert seen == owned, ("coop coverage", L, loge, nat)


def emit(scheds):
    out = ["// Generated by gen_schedule.py -- pass schedules of the fast NTT kernels.",
           "// Do not edit by hand: change CONFIGS in gen_schedule.py and rerun it.",
           "#pragma once", "", "namespace bc {", "namespace fast {", "",
           "struct PassDesc {",
           "    int hi, lo;       // processed position bits (inclusive)",
           "    int nreg;         // register bits: hi-lo+1 processed, then extras",
           "    int reg[5];       // register index bit j <-> position bit reg[j]",
           "    int lane[5];      // lane bit j <-> position bit lane[j]",
           "    int nwarp;",
           "    int warp[10];     // warp index bit j <-> position bit warp[j]",
           "    int phase;        // 0 or 1 (which rank bits the CTA owns)",
           "};", "",
           "struct RankBits {",
           "    int b[3];",
           "};", "",
           "template <int L, int LOGE> struct Sched;", ""]
    for s in scheds:
        L, loge, logc = s["L"], s["loge"], s["logc"]
        ps = s["passes"]

        def arr(v, n):
            v = list(v) + [0] * (n - len(v))
            return "{" + ", ".join(str(x) for x in v) + "}"
        out.append(f"template <> struct Sched<{L}, {loge}> {{")
        out.append(f"    static constexpr int kLogC = {logc}, kLogT = {s['logt']}, kPasses = {len(ps)}, "
                   f"kSplit = {s['split']};")
        out.append(f"    __host__ __device__ static constexpr int rank0(int j) {{ return RankBits{arr(s['rank0'], 3)}.b[j]; }}")
        out.append(f"    __host__ __device__ static constexpr int rank1(int j) {{ return RankBits{arr(s['rank1'], 3)}.b[j]; }}")
        out.append("    __host__ __device__ static constexpr PassDesc pass(int i) {")
        for i, p in enumerate(ps):
            ph = 0 if i < s["split"] else 1
            out.append(f"        if (i == {i}) return PassDesc{{{p.hi}, {p.lo}, {len(p.reg)}, {arr(p.reg, 5)}, "
                       f"{arr(p.lanes, 5)}, {len(p.warps)}, {arr(p.warps, 10)}, {ph}}};")
        out.append("        return PassDesc{};")
        out.append("    }")
        out.append("};")
        out.append("")
    out += ["}  // namespace fast", "}  // namespace bc", ""]
    return "\n".join(out)


def all_schedules():
    return [build(*k) for k in sorted(CONFIGS)]


def main():
    text = emit(all_schedules())
    with open(OUT, "w") as f:
        f.write(text)
    print("wrote", OUT)


if __name__ == "__main__":
    sys.exit(main())
