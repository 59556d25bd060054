"""GPU check of bc_polymul_static_scratch, the polynomial product that keeps
its temporary in the library's static device buffer instead of allocating:
through the C ABI, two calls in a row must give exactly what bc_polymul gives
on the same inputs.  Named to be collected last, so that it also runs after
every other GPU test has used the device."""
import ctypes

import pytest

import barracuda_b200 as bc
from barracuda_b200 import _native as N

pytestmark = pytest.mark.gpu
MAX_COEFFS = 1 << 21  # BC_POLYMUL_STATIC_MAX_COEFFS


def _plan(device, n, limbs, bits, mode):
    qs = bc.ntt_primes(bits, n, limbs)
    roots = [bc.negacyclic_root(q, n) for q in qs]
    if mode == bc.CYCLIC:
        roots = [r * r % q for r, q in zip(roots, qs)]
    return bc.NttPlan(device, n, qs, roots, mode=mode)


def _buf(device, count):
    return bc.FheTensor(device, 2 * count)


@pytest.mark.parametrize("logn,limbs,batch,bits,mode", [
    (15, 2, 8, 31, bc.NEGACYCLIC),   # fused cluster kernels, no scratch
    (15, 2, 4, 31, bc.CYCLIC),       # unfused path in the static buffer
    (14, 2, 4, 60, bc.NEGACYCLIC),   # 64-bit words, fused cluster kernels
    (17, 1, 2, 31, bc.NEGACYCLIC),
    (17, 1, 2, 60, bc.NEGACYCLIC),   # multi-pass global path in the static buffer
    (12, 2, 2, 31, bc.NEGACYCLIC),   # fused size: no scratch at all
    (14, 2, 4, 60, bc.CYCLIC),       # unfused path, 64-bit words
])
def test_static_scratch_polymul_matches_polymul(device, logn, limbs, batch, bits, mode):
    n = 1 << logn
    plan = _plan(device, n, limbs, bits, mode)
    total = limbs * batch * n
    assert total <= MAX_COEFFS
    a, b = _buf(device, total), _buf(device, total)
    want, got = _buf(device, total), _buf(device, total)
    lib = N.lib()
    for call, seed in enumerate((11, 29)):  # two calls in a row, fresh inputs each
        plan.fill_uniform(a, batch, seed=seed)
        plan.fill_uniform(b, batch, seed=seed + 1)
        N.check(lib.bc_polymul(plan.handle, a.ptr, b.ptr, want.ptr, batch, None, None))
        N.check(lib.bc_polymul_static_scratch(plan.handle, a.ptr, b.ptr, got.ptr, batch, None, None))
        device.synchronize()
        assert (got.to_u64() == want.to_u64()).all(), (call, logn, bits, mode)
    plan.close()


def test_static_scratch_polymul_rejects_oversize_and_strided(device):
    # cyclic above the fused size: the case where bc_polymul would allocate
    n, limbs = 1 << 15, 4
    batch = MAX_COEFFS // (limbs * n) + 1
    plan = _plan(device, n, limbs, 31, bc.CYCLIC)
    total = limbs * batch * n
    a, b, c = _buf(device, total), _buf(device, total), _buf(device, total)
    lib = N.lib()
    st = lib.bc_polymul_static_scratch(plan.handle, a.ptr, b.ptr, c.ptr, batch, None, None)
    assert st == 2 and "static scratch limit" in N.last_error()
    lay = N.bc_layout(limb_stride=n, poly_stride=limbs * n)
    st = lib.bc_polymul_static_scratch(plan.handle, a.ptr, b.ptr, c.ptr, 2, ctypes.byref(lay), None)
    assert st == 6 and "default layout" in N.last_error()
    plan.close()
