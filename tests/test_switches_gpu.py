"""GPU checks of the tuning switches (environment variables read once per
process): each setting runs in a child process and must give the oracle's
results.  The defaults are covered by every other GPU test; these are the
non-default cluster scheduling policies, the selectable schedule variants of
the N = 2^10..2^17 transforms (with the fused polynomial product on each)
and the automorphism kernels above the shared-memory size."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import sys
sys.path.insert(0, {root!r})
import barracuda_b200 as bc
from oracle import oracle as O

dev = bc.Device(0)
for logn, limbs, batch in {cases!r}:
    n = 1 << logn
    qs = bc.ntt_primes(31, n, limbs)
    psis = [bc.negacyclic_root(q, n) for q in qs]
    plan = bc.NttPlan(dev, n, qs, psis, mode=bc.NEGACYCLIC)
    total = limbs * batch * n
    src, dst, back, rot, other, prod = (bc.FheTensor(dev, 2 * total) for _ in range(6))
    plan.fill_uniform(src, batch, seed=logn + 11)
    plan.fill_uniform(other, batch, seed=logn + 12)
    plan.forward(src, dst, batch)
    plan.inverse(dst, back, batch)
    plan.automorphism(src, rot, batch, 5 ** 3 % (2 * n))
    plan.polymul(src, other, prod, batch)
    dev.synchronize()
    x, X, R, Y, P = src.to_u64(), dst.to_u64(), rot.to_u64(), other.to_u64(), prod.to_u64()
    assert (back.to_u64() == x).all(), ("round trip", logn)
    for l in range(limbs):
        off = (l * batch + batch - 1) * n
        xs, ys = x[off:off + n], Y[off:off + n]
        assert (X[off:off + n] == O.exact_negacyclic_ntt(xs, n, qs[l], psis[l])).all(), ("forward", logn, l)
        assert (R[off:off + n] == O.automorphism(xs, n, 5 ** 3 % (2 * n), qs[l])).all(), ("automorphism", logn, l)
        want = O.batch_polymul("ref_negacyclic", xs, ys, n, [qs[l]], [psis[l]])
        assert (P[off:off + n] == want).all(), ("polymul", logn, l)
    for t in (src, dst, back, rot, other, prod):
        t.free()
    plan.close()
dev.close()
print("switches ok")
"""

SETTINGS = [
    ({"BARRACUDA_CLUSTER_POLICY": "0"}, [(14, 2, 8), (16, 2, 4), (17, 1, 2)]),
    ({"BARRACUDA_CLUSTER_POLICY": "1"}, [(15, 2, 4), (16, 2, 4)]),
    ({"BARRACUDA_NTT_VARIANT": "4"}, [(12, 2, 8), (16, 2, 4)]),
    ({"BARRACUDA_NTT_VARIANT": "5"}, [(14, 2, 8), (16, 2, 4)]),
    ({"BARRACUDA_NTT_VARIANT_FWD": "7", "BARRACUDA_NTT_VARIANT_INV": "6"}, [(16, 2, 4)]),
    ({"BARRACUDA_AUTOMORPH_KERNEL": "cluster"}, [(15, 2, 4), (16, 1, 4)]),
    ({"BARRACUDA_AUTOMORPH_KERNEL": "scatter"}, [(14, 2, 4), (16, 1, 4)]),
]


@pytest.mark.parametrize("env,cases", SETTINGS, ids=[",".join(f"{k}={v}" for k, v in e.items()) for e, _ in SETTINGS])
def test_switch_matches_oracle(env, cases):
    child_env = dict(os.environ, **env)
    r = subprocess.run([sys.executable, "-c", CHILD.format(root=ROOT, cases=cases)], env=child_env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "switches ok" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]
