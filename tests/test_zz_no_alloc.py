"""GPU check of bc_polymul_static_scratch, the polynomial product for callers
that cannot allocate device memory during a call (device memory reserved up
front by another allocator, or a fixed device-memory budget while serving): it
keeps its temporary in the library's static device buffer instead of the
context's memory pool.  Through the C ABI, two calls in a row must give
exactly what bc_polymul gives on the same inputs, and a sampled limb-
polynomial must equal the oracle's product.  Named to be collected last, so
that it also runs after every other GPU test has used the device."""
import ctypes

import numpy as np
import pytest

import barracuda_b200 as bc
from barracuda_b200 import _native as N
from oracle import oracle as O

pytestmark = pytest.mark.gpu
MAX_COEFFS = 1 << 21  # BC_POLYMUL_STATIC_MAX_COEFFS


def _plan(device, n, limbs, bits, mode, root_power=1):
    """Negacyclic plans take psi; cyclic plans psi^2 (a primitive N-th root),
    or psi^(2 * root_power) to make the root non-primitive."""
    qs = bc.ntt_primes(bits, n, limbs)
    roots = [bc.negacyclic_root(q, n) for q in qs]
    if mode == bc.CYCLIC:
        roots = [pow(r, 2 * root_power, q) for r, q in zip(roots, qs)]
    return bc.NttPlan(device, n, qs, roots, mode=mode), qs, roots


def _buf(device, count, offset_words=0):
    """A device buffer of `count` u64 words, its pointer moved `offset_words`
    words into the allocation (8 bytes breaks the 16-byte alignment the
    fused kernels need)."""
    t = bc.FheTensor(device, 2 * (count + offset_words))
    return t, t.ptr + 8 * offset_words


def _read(device, ptr, count):
    out = np.empty(count, np.uint64)
    N.check(N.lib().bc_buf_d2h(device.handle, out.ctypes.data, ptr, out.nbytes))
    return out


def _oracle_product(a, b, n, q, r, mode, bits):
    if mode == bc.NEGACYCLIC:
        kind = "ref_negacyclic" if bits == 31 else "exact_negacyclic"
    else:
        kind = "ref_cyclic" if bits == 31 else "exact_cyclic"
    return O.batch_polymul(kind, a, b, n, [q], [r])


# (logn, limbs, batch, bits, mode, root_power, C offset in words)
CASES = [
    (15, 2, 8, 31, bc.NEGACYCLIC, 1, 0),  # fused cluster kernels: bc_polymul itself, no scratch
    (15, 2, 4, 31, bc.CYCLIC, 1, 0),      # primitive cyclic root: fused cluster kernels as well
    (15, 2, 4, 31, bc.CYCLIC, 2, 0),      # non-primitive root: reference chain in the static buffer
    (14, 2, 4, 60, bc.CYCLIC, 2, 0),      # the same, 64-bit words
    (12, 2, 2, 31, bc.NEGACYCLIC, 1, 0),  # fused size: no scratch at all
    (18, 1, 4, 31, bc.NEGACYCLIC, 1, 0),  # above the cluster kernels: multi-pass global path
    (18, 1, 2, 60, bc.CYCLIC, 1, 0),      # the same, cyclic, 64-bit words
    (16, 1, 4, 31, bc.NEGACYCLIC, 1, 1),  # C unaligned: transforms into C take the global path
]


@pytest.mark.parametrize("logn,limbs,batch,bits,mode,root_power,c_off", CASES)
def test_static_scratch_polymul_matches_polymul(device, logn, limbs, batch, bits, mode, root_power, c_off):
    n = 1 << logn
    plan, qs, roots = _plan(device, n, limbs, bits, mode, root_power)
    total = limbs * batch * n
    assert total <= MAX_COEFFS
    (ta, a), (tb, b) = _buf(device, total), _buf(device, total)
    (tw, want), (tg, got) = _buf(device, total, c_off), _buf(device, total, c_off)
    lib = N.lib()
    for call, seed in enumerate((11, 29)):  # two calls in a row, fresh inputs each
        plan.fill_uniform(a, batch, seed=seed)
        plan.fill_uniform(b, batch, seed=seed + 1)
        N.check(lib.bc_polymul(plan.handle, a, b, want, batch, None, None))
        N.check(lib.bc_polymul_static_scratch(plan.handle, a, b, got, batch, None, None))
        device.synchronize()
        G = _read(device, got, total)
        assert (G == _read(device, want, total)).all(), (call, logn, bits, mode)
    # one limb-polynomial against the oracle, independently of bc_polymul
    l = limbs - 1
    off = (l * batch + batch - 1) * n
    A, B = _read(device, a + 8 * off, n), _read(device, b + 8 * off, n)
    assert (G[off:off + n] == _oracle_product(A, B, n, qs[l], roots[l], mode, bits)).all()
    plan.close()


@pytest.mark.parametrize("logn,mode,root_power", [(15, bc.CYCLIC, 2), (18, bc.NEGACYCLIC, 1)])
def test_static_scratch_polymul_aliasing(device, logn, mode, root_power):
    """C may alias A, B or both, in the static buffer's chain too."""
    n, limbs, batch = 1 << logn, 1, 2
    plan, qs, roots = _plan(device, n, limbs, 31, mode, root_power)
    total = limbs * batch * n
    (ta, a), (tb, b), (tc, c), (tr, ref), (ts, sq) = (_buf(device, total) for _ in range(5))
    plan.fill_uniform(a, batch, seed=3)
    plan.fill_uniform(b, batch, seed=4)
    lib = N.lib()
    N.check(lib.bc_polymul(plan.handle, a, b, ref, batch, None, None))
    N.check(lib.bc_polymul(plan.handle, a, a, sq, batch, None, None))
    device.synchronize()
    A, B = _read(device, a, total), _read(device, b, total)
    want, want_sq = _read(device, ref, total), _read(device, sq, total)

    def put(ptr, x):
        N.check(lib.bc_buf_h2d(device.handle, ptr, x.ctypes.data, x.nbytes))

    put(c, A)
    N.check(lib.bc_polymul_static_scratch(plan.handle, c, b, c, batch, None, None))  # C aliases A
    device.synchronize()
    assert (_read(device, c, total) == want).all()
    put(c, B)
    N.check(lib.bc_polymul_static_scratch(plan.handle, a, c, c, batch, None, None))  # C aliases B
    device.synchronize()
    assert (_read(device, c, total) == want).all()
    put(c, A)
    N.check(lib.bc_polymul_static_scratch(plan.handle, c, c, c, batch, None, None))  # A == B == C
    device.synchronize()
    got_sq = _read(device, c, total)
    assert (got_sq == want_sq).all()
    off = (batch - 1) * n
    mode_kind = "ref_cyclic" if mode == bc.CYCLIC else "ref_negacyclic"
    assert (got_sq[off:off + n] == O.batch_polymul(mode_kind, A[off:off + n], A[off:off + n], n,
                                                   [qs[0]], [roots[0]])).all()
    plan.close()


def test_static_scratch_polymul_rejects_oversize_and_strided(device):
    # above the cluster kernels, where bc_polymul would take a pool temporary
    n, limbs = 1 << 18, 4
    batch = MAX_COEFFS // (limbs * n) + 1
    plan, _, _ = _plan(device, n, limbs, 31, bc.NEGACYCLIC)
    total = limbs * batch * n
    (ta, a), (tb, b), (tc, c) = (_buf(device, total) for _ in range(3))
    lib = N.lib()
    st = lib.bc_polymul_static_scratch(plan.handle, a, b, c, batch, None, None)
    assert st == 2 and "static scratch limit" in N.last_error()
    lay = N.bc_layout(limb_stride=n, poly_stride=limbs * n)
    st = lib.bc_polymul_static_scratch(plan.handle, a, b, c, 2, ctypes.byref(lay), None)
    assert st == 6 and "default layout" in N.last_error()
    plan.close()
