"""GPU parity of the rotation, modulus-switch and key-switch ops (FheRotate,
FheModulusSwitch, FheKeySwitch) and of their batched forms (bc_automorphism,
bc_modulus_switch, bc_decompose) against the CPU oracle, through the C ABI.

Bar: bit-exact.  Rotation and key switch reproduce the reference's shaders
for any input; modulus switching is the exact rounding (the reference's
shader agrees wherever its 64-bit product does not wrap, which the oracle
tests pin)."""
import os
import subprocess
import sys

import numpy as np
import pytest

import barracuda_b200 as bc
from barracuda_b200 import _native as N
from oracle import oracle as O
from tests.helpers import random_poly

pytestmark = pytest.mark.gpu
OL = O.lib()


def upload(dev, arr):
    return bc.FheTensor.from_u32(np.ascontiguousarray(np.asarray(arr, np.uint64)).view(np.uint32), dev)


def rotate(dev, x, n, r, q):
    return bc.FheRotate.new(upload(dev, x), n, r, q).execute().to_u64()


def _plan(device, n, limbs, bits):
    qs = bc.ntt_primes(bits, n, limbs)
    return bc.NttPlan(device, n, qs, [bc.negacyclic_root(q, n) for q in qs], mode=bc.NEGACYCLIC), qs


def test_golden_cases_on_gpu(device, kats):
    seen = set()
    for c in kats["cases"]:
        k, name = c["kind"], c["name"]
        if k == "rotate":
            x = c["input"]
            for r in c["rotations"]:
                x = rotate(device, x, c["degree"], r, c["modulus"])
            assert [int(v) for v in x] == c["expect"], name
        elif k == "modulus_switch":
            t = upload(device, c["input"])
            out = bc.FheModulusSwitch.new(t, c["degree"], c["modulus_old"], c["modulus_new"]).execute()
            assert [int(v) for v in out.to_u64()] == c["exact"], name
        elif k == "key_switch":
            t = upload(device, c["input"])
            out = bc.FheKeySwitch.new(t, c["degree"], c["modulus"], c["decomp_base"],
                                      c["decomp_levels"]).execute()
            assert [int(v) for v in out.to_u64()] == c["expect"], name
        else:
            continue
        seen.add(k)
    assert seen == {"rotate", "modulus_switch", "key_switch"}


@pytest.mark.parametrize("logn", [2, 3, 8, 12, 13, 14, 16, 17])
def test_fhe_rotate_matches_reference(device, logn):
    """Every rotation class (negative, zero, extremes) on reduced inputs plus
    words above q and zeros (the shader's negation wraps / keeps 0)."""
    n = 1 << logn
    q = O.ntt_prime(30, n, 0) if logn > 2 else 257
    rng = np.random.default_rng(logn)
    x = random_poly(rng, n, q)
    x[rng.integers(0, n, max(1, n // 16))] = 0
    x[rng.integers(0, n, max(1, n // 16))] = rng.integers(q, 2**64 - 1, max(1, n // 16), dtype=np.uint64)
    for r in sorted({-n // 2, -(n // 4) - 1, -1, 0, 1, 5 % (n // 2 + 1), n // 2}):
        assert (rotate(device, x, n, r, q) == O.ref_rotate(x, n, r, q)).all(), r


@pytest.mark.parametrize("logn,limbs,batch,bits", [(4, 2, 3, 31), (10, 3, 4, 31), (12, 2, 5, 60),
                                                   (13, 2, 3, 31), (14, 2, 3, 60), (15, 1, 2, 31),
                                                   (16, 2, 2, 31), (17, 1, 2, 60)])
def test_plan_automorphism_matches_oracle(device, logn, limbs, batch, bits):
    n = 1 << logn
    plan, qs = _plan(device, n, limbs, bits)
    total = limbs * batch * n
    src, dst = bc.FheTensor(device, 2 * total), bc.FheTensor(device, 2 * total)
    plan.fill_uniform(src, batch, seed=logn)
    x = src.to_u64()
    for g in (1, 3, 5 ** 3 % (2 * n) | 1, 2 * n - 1, 2 * (n // 2) + 1 - 2):
        g = g % (2 * n) | 1
        plan.automorphism(src, dst, batch, g)
        device.synchronize()
        y = dst.to_u64()
        for l in range(limbs):
            for p in {0, batch - 1}:
                off = (l * batch + p) * n
                assert (y[off:off + n] == O.automorphism(x[off:off + n], n, g, qs[l])).all(), (g, l, p)
    plan.close()


def test_plan_automorphism_strided_layout(device):
    """[poly][limb][N] layout (ciphertext-major) and both kernel paths."""
    for logn in (12, 15):
        n, limbs, batch = 1 << logn, 3, 4
        plan, qs = _plan(device, n, limbs, 31)
        lay = bc.Layout(limb_stride=n, poly_stride=limbs * n)
        total = limbs * batch * n
        src, dst = bc.FheTensor(device, 2 * total), bc.FheTensor(device, 2 * total)
        plan.fill_uniform(src, batch, seed=3, layout=lay)
        g = 2 * 77 + 1
        plan.automorphism(src, dst, batch, g, layout=lay)
        device.synchronize()
        x, y = src.to_u64(), dst.to_u64()
        for p in range(batch):
            for l in range(limbs):
                o = (p * limbs + l) * n
                assert (y[o:o + n] == O.automorphism(x[o:o + n], n, g, qs[l])).all(), (logn, p, l)
        plan.close()


@pytest.mark.parametrize("logn", [12, 16])
def test_automorphism_is_a_ring_homomorphism_at_full_size(device, logn):
    """sigma(a * b) == sigma(a) * sigma(b) under the negacyclic product, and
    sigma_g then sigma_(g^-1) is the identity: size-independent properties at
    N = 2^16 with 2 limbs x 8 polynomials."""
    n, limbs, batch = 1 << logn, 2, 8
    plan, qs = _plan(device, n, limbs, 31)
    total = limbs * batch * n
    a, b, ab, t1, t2, t3 = (bc.FheTensor(device, 2 * total) for _ in range(6))
    plan.fill_uniform(a, batch, seed=11)
    plan.fill_uniform(b, batch, seed=12)
    g = 2 * 1234 % (2 * n) + 1
    plan.polymul(a, b, ab, batch)
    plan.automorphism(ab, t1, batch, g)          # sigma(a b)
    plan.automorphism(a, t2, batch, g)
    plan.automorphism(b, t3, batch, g)
    plan.polymul(t2, t3, ab, batch)              # sigma(a) sigma(b)
    device.synchronize()
    assert (t1.to_u64() == ab.to_u64()).all()
    ginv = pow(g, -1, 2 * n)
    plan.automorphism(t2, t1, batch, ginv)
    device.synchronize()
    assert (t1.to_u64() == a.to_u64()).all()
    plan.close()


@pytest.mark.parametrize("kernel", ["gather", "scatter", "cluster", "direct"])
def test_automorphism_kernel_variants(kernel):
    """Each automorphism kernel (the defaults pick one per N) passes the
    batched parity tests, run in a child process with the override set."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, BARRACUDA_AUTOMORPH_KERNEL=kernel)
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider",
                        os.path.join(root, "tests", "test_rns_gpu.py"), "-k", "plan_automorphism"],
                       env=env, cwd=root, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]


MODSWITCH_PAIRS = [(257, 17), (12289, 6145), (2**31 - 1, 2**30 + 3), (1 << 40, 3), (2**61 - 1, 2**60 + 33),
                   (1152921504606584833, 288230376151711777), (2**64 - 59, 2**63 + 29), (2**64 - 59, 1),
                   (2**64 - 1, 2**64 - 2), (1, 0), (7, 0), (2**63, 2**62)]


@pytest.mark.parametrize("q_old,q_new", MODSWITCH_PAIRS)
def test_modulus_switch_exact(device, q_old, q_new):
    """FheModulusSwitch on reduced, arbitrary and near-2^64 words: the exact
    rounding; where the shader's product does not wrap, also the shader's
    value."""
    n = 4096
    rng = np.random.default_rng(q_old % 99991 + q_new % 7)
    x = np.concatenate([rng.integers(0, min(q_old, 2**64 - 1), n // 2, dtype=np.uint64),
                        rng.integers(0, 2**64 - 1, n // 4, dtype=np.uint64, endpoint=True),
                        np.uint64(2**64 - 1) - rng.integers(0, 100, n // 4, dtype=np.uint64)])
    if q_old > 2:  # exact halves: c q_new = (k + 1/2) q_old where such c exist
        x[:4] = [0, 1, q_old - 1, q_old // 2]
    got = bc.FheModulusSwitch.new(upload(device, x), n, q_old, q_new).execute().to_u64()
    assert (got == O.exact_modulus_switch(x, q_old, q_new)).all()
    ref = O.ref_modulus_switch(x, q_old, q_new)
    small = np.array([int(c) * q_new < 2**64 for c in x]) & (q_old <= 2**63)
    assert (got[small] == ref[small]).all()


def test_modulus_switch_batched_in_place_and_large(device):
    count = (1 << 22) + 7
    rng = np.random.default_rng(4)
    x = rng.integers(0, 2**64 - 1, count, dtype=np.uint64, endpoint=True)
    t = upload(device, x)
    q_old, q_new = (1 << 62) - 57, (1 << 50) - 27
    bc.modulus_switch(device, t, t, count, q_old, q_new)
    device.synchronize()
    want = O.exact_modulus_switch(x, q_old, q_new)
    assert (t.to_u64() == want).all()
    with pytest.raises(bc.BarracudaError):
        bc.modulus_switch(device, t, t, count, 17, 17)


@pytest.mark.parametrize("base,levels", [(2, 32), (16, 16), (1 << 16, 4), (1 << 24, 3), (12289, 5), (3, 32)])
def test_decompose_matches_oracle(device, base, levels):
    count = 3000
    rng = np.random.default_rng(base + levels)
    x = rng.integers(0, 2**64 - 1, count, dtype=np.uint64, endpoint=True)
    src, dst = upload(device, x), bc.FheTensor(device, 2 * count * levels)
    bc.decompose(device, src, dst, count, base, levels)
    device.synchronize()
    assert (dst.to_u64().reshape(levels, count) == O.decompose(x, base, levels)).all()


def test_key_switch_is_a_copy_and_rejects(device):
    n = 1 << 12
    x = np.random.default_rng(0).integers(0, 2**64 - 1, n, dtype=np.uint64, endpoint=True)
    out = bc.FheKeySwitch.new(upload(device, x), n, 12289, 1 << 16, 3).execute().to_u64()
    assert (out == O.ref_key_switch(x, 1 << 16, 3)).all() and (out == x).all()
    with pytest.raises(bc.BarracudaError):
        bc.FheKeySwitch.new(upload(device, x), n, 12289, 1, 3)


def test_rns_ops_reject_bad_arguments(device):
    n = 1 << 10
    plan, _ = _plan(device, n, 1, 31)
    a, b = bc.FheTensor(device, 2 * n), bc.FheTensor(device, 2 * n * 4)
    for g in (0, 2, 2 * n, 2 * n + 1):
        with pytest.raises(bc.BarracudaError):
            plan.automorphism(a, b, 1, g)
    with pytest.raises(bc.BarracudaError):
        plan.automorphism(a, a, 1, 3)             # must not be in place
    with pytest.raises(bc.BarracudaError):
        bc.decompose(device, a, a, n, 16, 4)      # overlapping
    with pytest.raises(bc.BarracudaError):
        bc.decompose(device, a, b, n, 1, 4)
    with pytest.raises(bc.BarracudaError):
        bc.decompose(device, a, b, n, 16, 33)
    lib = N.lib()
    assert lib.bc_fhe_rotate(device.handle, a.ptr, 2 * n, n, 1, 17, a.ptr) == N.BC_ERR_INVALID_INPUT
    plan.close()
