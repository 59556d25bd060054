"""GPU checks of the persistent, prefetching forms of the transform kernels,
which are selectable but not the default: BARRACUDA_NTT_PERSISTENT=1 stages
the next polynomial with per-thread cp.async copies, =2 with one bulk copy
(TMA) per polynomial completed through an mbarrier (one-CTA schedules,
N <= 2^13; cp.async above).  The variable is read once per process, so each
mode runs in a child process.  Batches hold more polynomials than the grid
has resident CTAs, so every CTA runs several iterations and prefetches."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import sys
import numpy as np
sys.path.insert(0, {root!r})
import barracuda_b200 as bc
from oracle import oracle as O

dev = bc.Device(0)
for logn, bits, limbs, batch in ((10, 31, 2, 700), (12, 31, 3, 300), (13, 31, 2, 400), (13, 30, 2, 400),
                                 (12, 60, 2, 400), (14, 31, 2, 40), (16, 31, 2, 8)):
    n = 1 << logn
    qs = bc.ntt_primes(bits, n, limbs)
    psis = [bc.negacyclic_root(q, n) for q in qs]
    for mode in (bc.NEGACYCLIC, bc.CYCLIC):
        roots = psis if mode == bc.NEGACYCLIC else [p * p % q for p, q in zip(psis, qs)]
        plan = bc.NttPlan(dev, n, qs, roots, mode=mode)
        total = limbs * batch * n
        src, dst, back = (bc.FheTensor(dev, 2 * total) for _ in range(3))
        plan.fill_uniform(src, batch, seed=logn * 7 + bits)
        plan.forward(src, dst, batch)
        plan.inverse(dst, back, batch)
        dev.synchronize()
        x, X = src.to_u64(), dst.to_u64()
        assert (back.to_u64() == x).all(), ("round trip", logn, bits, mode)
        for l, p in ((0, 0), (limbs - 1, batch - 1), (limbs - 1, batch // 2)):
            off = (l * batch + p) * n
            xs = x[off:off + n]
            if mode == bc.NEGACYCLIC:
                want = O.exact_negacyclic_ntt(xs, n, qs[l], roots[l])
            else:
                want = O.exact_ntt(xs, n, qs[l], roots[l])
            assert (X[off:off + n] == want).all(), ("forward", logn, bits, mode, l, p)
        for t in (src, dst, back):
            t.free()
        plan.close()
dev.close()
print("persistent ok")
"""


@pytest.mark.parametrize("mode", ["1", "2"])
def test_persistent_prefetch_matches_oracle(mode):
    env = dict(os.environ, BARRACUDA_NTT_PERSISTENT=mode)
    r = subprocess.run([sys.executable, "-c", CHILD.format(root=ROOT)], env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0 and "persistent ok" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]
