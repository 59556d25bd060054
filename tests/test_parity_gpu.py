"""GPU parity of the CUDA path against the CPU oracle and the reference's
known answers.  Everything runs through the C ABI (libbarracuda_fhe.so).

Bar: bit-exact.  For moduli below 2^31 the target is the reference's own
algorithm (oracle/ref_wgsl.c); for wider moduli, where the reference
truncates its products, the target is exact u128 arithmetic."""
import ctypes

import numpy as np
import pytest

import barracuda_b200 as bc
from barracuda_b200 import _native as N
from oracle import oracle as O
from tests.helpers import find_root_of_unity, modinv, random_poly, resolve_root

pytestmark = pytest.mark.gpu
OL = O.lib()


def upload(dev, arr):
    return bc.FheTensor.from_u32(np.ascontiguousarray(np.asarray(arr, np.uint64)).view(np.uint32), dev)


def ntt(dev, x, n, q, r):
    return np.array(bc.FheNtt.new(upload(dev, x), n, q, r).execute().to_u64())


def intt(dev, x, n, q, r):
    return np.array(bc.FheIntt.new(upload(dev, x), n, q, r).execute().to_u64())


def coeff_op(dev, op, a, b, n, q):
    cls = {"add": bc.FhePolyAdd, "sub": bc.FhePolySub, "mul": bc.FhePolyMul}[op]
    return np.array(cls.new(upload(dev, a), upload(dev, b), n, q).execute().to_u64())


# ------------------------------------------------------------ reference ops

def test_golden_cases_on_gpu(device, kats):
    rng = np.random.default_rng(17)
    for c in kats["cases"]:
        k, name = c["kind"], c["name"]
        if k == "ntt":
            assert list(ntt(device, c["input"], c["degree"], c["modulus"], c["root"])) == c["expect"], name
        elif k == "roundtrip":
            n, q = c["degree"], c["modulus"]
            r = resolve_root(c["root"], n, q)
            back = intt(device, ntt(device, c["input"], n, q, r), n, q, bc.compute_inverse_root(n, q, r))
            assert [int(v) for v in back] == [v % q for v in c["input"]], name
        elif k == "linearity":
            n, q = c["degree"], c["modulus"]
            r = resolve_root(c["root"], n, q)
            a, b = np.array(c["a"], np.uint64), np.array(c["b"], np.uint64)
            lhs = ntt(device, coeff_op(device, "add", a, b, n, q), n, q, r)
            rhs = coeff_op(device, "add", ntt(device, a, n, q, r), ntt(device, b, n, q, r), n, q)
            assert (lhs == rhs).all()
        elif k in ("poly_add", "poly_sub", "poly_mul"):
            got = coeff_op(device, k[5:], c["a"], c["b"], c["degree"], c["modulus"])
            assert list(got) == c["expect"], name
        elif k == "poly_add_assoc":
            n, q = c["degree"], c["modulus"]
            a, b, cc = c["a"], c["b"], c["c"]
            lhs = coeff_op(device, "add", coeff_op(device, "add", a, b, n, q), cc, n, q)
            assert (lhs == coeff_op(device, "add", a, coeff_op(device, "add", b, cc, n, q), n, q)).all()
        elif k == "ntt_zero":
            n, q = c["degree"], c["modulus"]
            assert (ntt(device, c["input"], n, q, resolve_root(c["root"], n, q)) == 0).all()
        elif k == "ntt_range":
            n, q = c["degree"], c["modulus"]
            r = resolve_root(c["root"], n, q)
            got = ntt(device, c["input"], n, q, r)
            assert (got < q).all() and (got == O.ref_ntt(c["input"], n, q, r)).all()
        elif k == "pointwise":
            n, q = c["degree"], c["modulus"]
            out = bc.FhePointwiseMul.new(upload(device, c["a"]), upload(device, c["b"]), n, q).execute()
            assert [int(v) for v in out.to_u64()] == c["expect"]
        elif k in ("pointwise_identity", "pointwise_zero"):
            n, q = c["degree"], c["modulus"]
            r = resolve_root(c["root"], n, q)
            x = random_poly(rng, n, q)
            other = np.zeros(n, np.uint64)
            if k == "pointwise_identity":
                other[0] = 1
            X = bc.FheNtt.new(upload(device, x), n, q, r).execute()
            Y = bc.FheNtt.new(upload(device, other), n, q, r).execute()
            got = bc.FhePointwiseMul.new(X, Y, n, q).execute().to_u64()
            want = O.ref_ntt(x, n, q, r) if k == "pointwise_identity" else np.zeros(n, np.uint64)
            assert (got == want).all(), name
        elif k.startswith("fast_mul"):
            n, q = c["degree"], c["modulus"]
            r = resolve_root(c["root"], n, q)
            a, b, cc = (random_poly(rng, n, q) for _ in range(3))

            def fm(x, y):
                return bc.FheFastPolyMul.new(upload(device, x), upload(device, y), n, q, r).execute().to_u64()
            if k == "fast_mul_naive":
                assert (fm(a, b) == O.cyclic_convolution(a, b, n, q)).all()
            elif k == "fast_mul_commutative":
                assert (fm(a, b) == fm(b, a)).all()
            else:
                lhs = fm(a, (b + cc) % np.uint64(q))
                assert (lhs == (fm(a, b) + fm(a, cc)) % np.uint64(q)).all()


@pytest.mark.parametrize("logn", list(range(1, 15)))
def test_fhe_ntt_intt_match_reference_restatement(device, logn):
    n = 1 << logn
    rng = np.random.default_rng(logn)
    for bits in (14, 30, 31):
        q = O.ntt_prime(bits, n, 1)
        if q == 0:
            continue
        psi = O.psi(q, n)
        w = OL.orc_mulmod(psi, psi, q)
        x = random_poly(rng, n, q)
        got = ntt(device, x, n, q, w)
        assert (got == O.ref_ntt(x, n, q, w)).all(), (n, q)
        winv = bc.compute_inverse_root(n, q, w)
        assert (intt(device, got, n, q, winv) == x).all()
        assert (intt(device, x, n, q, winv) == O.ref_intt(x, n, q, winv)).all()


def test_structure_faithful_for_invalid_roots(device):
    """Roots that are not primitive N-th roots (the canary's omega = 11 for
    N = 8, arbitrary values) still reproduce the reference's DIT output."""
    rng = np.random.default_rng(5)
    for n, q, w in [(8, 12289, 11), (64, 12289, 3), (1024, 12289, 7), (4096, 2147352577, 12345),
                    (16, 257, 256), (4, 17, 0), (16, 97, 1)]:
        x = random_poly(rng, n, q)
        assert (ntt(device, x, n, q, w) == O.ref_ntt(x, n, q, w)).all(), (n, q, w)
        assert (intt(device, x, n, q, w) == O.ref_intt(x, n, q, w)).all(), (n, q, w)


def test_inputs_below_2_32_match_reference_after_reduction(device):
    rng = np.random.default_rng(9)
    for n in (4, 256, 4096):
        q = O.ntt_prime(31, n, 0)
        w = OL.orc_mulmod(O.psi(q, n), O.psi(q, n), q)
        x = rng.integers(0, 2**32, n, dtype=np.uint64)
        assert (ntt(device, x, n, q, w) == O.ref_ntt(x, n, q, w) % np.uint64(q)).all()


def test_wide_input_reports_invalid_input_and_device_survives(device):
    n, q = 16, 12289
    w = find_root_of_unity(n, q)
    x = np.ones(n, np.uint64)
    x[3] = 1 << 40
    with pytest.raises(bc.BarracudaError) as e:
        ntt(device, x, n, q, w)
    assert e.value.kind == "InvalidInput"
    # the context is still usable afterwards (fhe_fault_tests.rs:95-128)
    y = random_poly(np.random.default_rng(0), n, q)
    assert (ntt(device, y, n, q, w) == O.ref_ntt(y, n, q, w)).all()


def test_intt_edge_cases(device):
    # degree 1 (allowed by FheIntt::new), non-congruent and even moduli
    for n, q, r in [(1, 17, 1), (1, 2**31 - 1, 5), (8, 100, 3), (16, 19, 2), (4, 2, 1), (8, 1, 0)]:
        x = np.arange(n, dtype=np.uint64) % np.uint64(q)
        assert (intt(device, x, n, q, r) == O.ref_intt(x, n, q, r) % np.uint64(q)).all(), (n, q)


def test_modulus_one(device):
    # q = 1 passes FheNtt's congruence check; every residue is 0
    for n in (2, 16):
        assert (ntt(device, np.zeros(n, np.uint64), n, 1, 0) == 0).all()


def test_pointwise_matches_reference(device):
    rng = np.random.default_rng(2)
    for n, q in [(4, 12289), (1024, 2147352577), (65536, 998244353), (8, 3)]:
        a = rng.integers(0, 2**32, n, dtype=np.uint64)
        b = rng.integers(0, 2**32, n, dtype=np.uint64)
        got = bc.FhePointwiseMul.new(upload(device, a), upload(device, b), n, q).execute().to_u64()
        assert (got == O.ref_pointwise(a, b, n, q)).all(), (n, q)
    # modulus 0: the reference keeps the low 32 bits of each product
    a = rng.integers(0, 2**32, 16, dtype=np.uint64)
    b = rng.integers(0, 2**32, 16, dtype=np.uint64)
    got = bc.FhePointwiseMul.new(upload(device, a), upload(device, b), 16, 0).execute().to_u64()
    assert (got == O.ref_pointwise(a, b, 16, 0)).all()


@pytest.mark.parametrize("logn", [2, 5, 10, 12, 14, 15, 16])
def test_fast_poly_mul_matches_reference_chain(device, logn):
    n = 1 << logn
    rng = np.random.default_rng(logn + 50)
    q = O.ntt_prime(31, n, 0)
    w = OL.orc_mulmod(O.psi(q, n), O.psi(q, n), q)
    a, b = random_poly(rng, n, q), random_poly(rng, n, q)
    got = bc.FheFastPolyMul.new(upload(device, a), upload(device, b), n, q, w).execute().to_u64()
    assert (got == O.ref_fast_poly_mul(a, b, n, q, w)).all()
    if n <= 1024:
        assert (got == O.cyclic_convolution(a, b, n, q)).all()


def test_wide_moduli_are_exact(device):
    """Moduli in [2^31, 2^62): exact residues (the reference diverges here)."""
    rng = np.random.default_rng(8)
    for bits in (32, 45, 60, 62):
        for n in (4, 64, 4096):
            q = O.ntt_prime(bits, n, 0)
            w = OL.orc_mulmod(O.psi(q, n), O.psi(q, n), q)
            x = random_poly(rng, n, q)
            got = ntt(device, x, n, q, w)
            assert (got == O.exact_ntt(x, n, q, w)).all(), (bits, n)
            assert (intt(device, got, n, q, bc.compute_inverse_root(n, q, w)) == x).all()


# ------------------------------------------------------------ batched plans

def _plan(device, n, limbs, bits, mode):
    qs = bc.ntt_primes(bits, n, limbs)
    roots = [bc.negacyclic_root(q, n) for q in qs]
    if mode == bc.CYCLIC:
        roots = [r * r % q for r, q in zip(roots, qs)]
    return bc.NttPlan(device, n, qs, roots, mode=mode), qs, roots


def _alloc(device, count):
    return bc.FheTensor(device, 2 * count)


@pytest.mark.parametrize("logn,limbs,batch", [(12, 1, 1), (12, 3, 5), (14, 4, 3), (15, 2, 2),
                                              (16, 2, 2), (17, 1, 2), (10, 8, 9), (3, 2, 7)])
@pytest.mark.parametrize("bits", [31, 60])
def test_plan_negacyclic_matches_oracle(device, logn, limbs, batch, bits):
    n = 1 << logn
    plan, qs, psis = _plan(device, n, limbs, bits, bc.NEGACYCLIC)
    total = limbs * batch * n
    src, dst, back = _alloc(device, total), _alloc(device, total), _alloc(device, total)
    plan.fill_uniform(src, batch, seed=1234)
    plan.forward(src, dst, batch)
    plan.inverse(dst, back, batch)
    device.synchronize()
    x, X, xb = src.to_u64(), dst.to_u64(), back.to_u64()
    assert (xb == x).all()
    for l in range(limbs):
        q = qs[l]
        assert (x[l * batch * n:(l + 1) * batch * n] < q).all()
        # seeded generator parity with the oracle
        cnt = min(64, batch * n)
        assert (x[l * batch * n: l * batch * n + cnt] == O.seeded_fill(cnt, 1234, l * batch * n, q)).all()
        for p in {0, batch - 1}:
            off = (l * batch + p) * n
            want = (O.ref_negacyclic_ntt(x[off:off + n], n, q, psis[l]) if bits == 31
                    else O.exact_negacyclic_ntt(x[off:off + n], n, q, psis[l]))
            assert (X[off:off + n] == want).all(), (l, p)


@pytest.mark.parametrize("logn,limbs,batch", [(12, 2, 3), (14, 2, 2), (16, 1, 2)])
def test_plan_cyclic_matches_reference(device, logn, limbs, batch):
    n = 1 << logn
    plan, qs, ws = _plan(device, n, limbs, 31, bc.CYCLIC)
    total = limbs * batch * n
    src, dst, back = _alloc(device, total), _alloc(device, total), _alloc(device, total)
    plan.fill_uniform(src, batch, seed=99)
    plan.forward(src, dst, batch)
    plan.inverse(dst, back, batch)
    device.synchronize()
    x, X = src.to_u64(), dst.to_u64()
    assert (back.to_u64() == x).all()
    for l in range(limbs):
        off = l * batch * n
        assert (X[off:off + n] == O.ref_ntt(x[off:off + n], n, qs[l], ws[l])).all()


def test_plan_strided_ciphertext_layout_and_in_place(device):
    """[ct][2][limb][N] layout (config 3 shape, reduced) and in-place use."""
    n, limbs, cts = 1 << 12, 3, 4
    plan, qs, psis = _plan(device, n, limbs, 31, bc.NEGACYCLIC)
    lay = bc.Layout(limb_stride=n, poly_stride=limbs * n)
    total = cts * 2 * limbs * n
    buf = _alloc(device, total)
    plan.fill_uniform(buf, 2 * cts, seed=7, layout=lay)
    x = buf.to_u64().copy()
    plan.forward(buf, buf, 2 * cts, layout=lay)
    device.synchronize()
    X = buf.to_u64()
    for p in (0, 5):
        for l in range(limbs):
            off = p * limbs * n + l * n
            assert (X[off:off + n] == O.ref_negacyclic_ntt(x[off:off + n], n, qs[l], psis[l])).all()
    plan.inverse(buf, buf, 2 * cts, layout=lay)
    device.synchronize()
    assert (buf.to_u64() == x).all()


@pytest.mark.parametrize("logn,bits", [(10, 31), (12, 31), (14, 31), (15, 60), (16, 31), (17, 31), (16, 60)])
def test_forward_mul_and_inverse_mul_match_chains(device, logn, bits):
    """C = NTT(A) * B^ and C = INTT(A^ * B^) in one launch equal the
    transform-then-pointwise chains; aliasing C with either input."""
    n, limbs, batch = 1 << logn, 2, 3
    plan, qs, _ = _plan(device, n, limbs, bits, bc.NEGACYCLIC)
    total = limbs * batch * n
    a, b, bh, t, c = (_alloc(device, total) for _ in range(5))
    plan.fill_uniform(a, batch, seed=3)
    plan.fill_uniform(b, batch, seed=4)
    plan.forward(b, bh, batch)                  # B^ = NTT(B)
    plan.forward(a, t, batch)
    plan.pointwise_mul(t, bh, t, batch)         # chain: NTT(A) * B^
    plan.forward_mul(a, bh, c, batch)
    device.synchronize()
    want_f = t.to_u64().copy()
    assert (c.to_u64() == want_f).all()
    plan.pointwise_mul(bh, bh, t, batch)        # chain: INTT(B^ * B^)
    plan.inverse(t, t, batch)
    plan.inverse_mul(bh, bh, c, batch)
    device.synchronize()
    want_i = t.to_u64().copy()
    assert (c.to_u64() == want_i).all()
    # in place: C = A, then C = B^
    x = _alloc(device, total)
    plan.fill_uniform(x, batch, seed=3)
    plan.forward_mul(x, bh, x, batch)
    device.synchronize()
    assert (x.to_u64() == want_f).all()
    y = _alloc(device, total)
    plan.forward(b, y, batch)
    plan.forward_mul(a, y, y, batch)
    device.synchronize()
    assert (y.to_u64() == want_f).all()
    plan.forward(b, y, batch)
    plan.inverse_mul(y, y, y, batch)
    device.synchronize()
    assert (y.to_u64() == want_i).all()
    plan.close()


def test_forward_mul_inverse_mul_compose_to_polymul(device):
    """INTT(NTT(A) * NTT(B)) through the fused forward equals bc_polymul and
    the oracle's negacyclic convolution."""
    n, limbs, batch = 1 << 10, 2, 2
    plan, qs, _ = _plan(device, n, limbs, 31, bc.NEGACYCLIC)
    total = limbs * batch * n
    a, b, bh, c, want = (_alloc(device, total) for _ in range(5))
    plan.fill_uniform(a, batch, seed=8)
    plan.fill_uniform(b, batch, seed=9)
    plan.forward(b, bh, batch)
    plan.forward_mul(a, bh, c, batch)
    plan.inverse(c, c, batch)
    plan.polymul(a, b, want, batch)
    device.synchronize()
    C, W, A, B = c.to_u64(), want.to_u64(), a.to_u64(), b.to_u64()
    assert (C == W).all()
    assert (C[:n] == O.negacyclic_convolution(A[:n], B[:n], n, qs[0])).all()
    plan.close()


def test_forward_mul_fallbacks_and_wide_words(device):
    """B^ words in [q, 2^32) are reduced first; odd strides and cyclic plans
    take the two-launch path with the same result."""
    n, limbs, batch = 1 << 12, 2, 2
    plan, qs, _ = _plan(device, n, limbs, 31, bc.NEGACYCLIC)
    rng = np.random.default_rng(5)
    total = limbs * batch * n
    A = rng.integers(0, qs[-1], total, dtype=np.uint64)
    Bh = rng.integers(0, 2**32, total, dtype=np.uint64)   # not reduced
    a, bh, c = upload(device, A), upload(device, Bh), _alloc(device, total)
    plan.forward_mul(a, bh, c, batch)
    X = _alloc(device, total)
    plan.forward(a, X, batch)
    device.synchronize()
    Xh, C = X.to_u64(), c.to_u64()
    for l in range(limbs):
        for p in range(batch):
            o = (l * batch + p) * n
            assert (C[o:o + n] == O.exact_poly_mul(Xh[o:o + n], Bh[o:o + n], qs[l])).all(), (l, p)
    # odd poly stride: [limb][poly] with a one-word gap, not 16-byte aligned
    lay = bc.Layout(limb_stride=batch * (n + 1), poly_stride=n + 1)
    big = limbs * batch * (n + 1)
    a2, b2, c2, t2 = (_alloc(device, big) for _ in range(4))
    plan.fill_uniform(a2, batch, seed=1, layout=lay)
    plan.fill_uniform(b2, batch, seed=2, layout=lay)
    plan.forward_mul(a2, b2, c2, batch, layout=lay)
    plan.forward(a2, t2, batch, layout=lay)
    plan.pointwise_mul(t2, b2, t2, batch, layout=lay)
    device.synchronize()
    C2, T2 = c2.to_u64(), t2.to_u64()
    for l in range(limbs):
        for p in range(batch):
            o = l * batch * (n + 1) + p * (n + 1)
            assert (C2[o:o + n] == T2[o:o + n]).all(), (l, p)
    plan.close()
    cplan, _, _ = _plan(device, n, limbs, 31, bc.CYCLIC)
    a3, b3, c3, t3 = (_alloc(device, total) for _ in range(4))
    cplan.fill_uniform(a3, batch, seed=1)
    cplan.fill_uniform(b3, batch, seed=2)
    cplan.inverse_mul(a3, b3, c3, batch)
    cplan.pointwise_mul(a3, b3, t3, batch)
    cplan.inverse(t3, t3, batch)
    device.synchronize()
    assert (c3.to_u64() == t3.to_u64()).all()
    cplan.close()


@pytest.mark.parametrize("logn", [12, 13, 14, 15, 16, 17])
@pytest.mark.parametrize("bits", [31, 60])
def test_forward_and_inverse_add_sub_match_the_reference_chain(device, logn, bits):
    """C = NTT(A) +- B^ and C = INTT(A^ +- B^) in one launch (FhePolyAdd /
    FhePolySub fused into the transform) equal the reference chain value by
    value on one polynomial of every limb: the oracle's transform (the
    reference's algorithm for q < 2^31, exact u128 math above) followed by
    the reference's coefficient op."""
    n, limbs, batch = 1 << logn, 2, 2
    plan, qs, psis = _plan(device, n, limbs, bits, bc.NEGACYCLIC)
    total = limbs * batch * n
    a, b, bh, c = (_alloc(device, total) for _ in range(4))
    plan.fill_uniform(a, batch, seed=13)
    plan.fill_uniform(b, batch, seed=14)
    plan.forward(b, bh, batch)  # B^ = NTT(B), canonical
    device.synchronize()
    A, Bh = a.to_u64(), bh.to_u64()
    offs = [(l * batch + 1) * n for l in range(limbs)]
    Asel = np.concatenate([A[o:o + n] for o in offs])
    Bsel = np.concatenate([Bh[o:o + n] for o in offs])
    fwd, inv = (("negacyclic_ntt", "negacyclic_intt") if bits == 31
                else ("exact_negacyclic_ntt", "exact_negacyclic_intt"))
    NA = O.batch_transform(fwd, Asel, n, qs, psis)
    for name, fwd_op, inv_op, coeff in (("add", plan.forward_add, plan.inverse_add, O.ref_poly_add),
                                        ("sub", plan.forward_sub, plan.inverse_sub, O.ref_poly_sub)):
        fwd_op(a, bh, c, batch)
        device.synchronize()
        C = c.to_u64()
        for l, o in enumerate(offs):
            sl = slice(l * n, (l + 1) * n)
            assert (C[o:o + n] == coeff(NA[sl], Bsel[sl], qs[l])).all(), ("forward", name, l)
        inv_op(bh, bh if name == "add" else a, c, batch)
        device.synchronize()
        C = c.to_u64()
        other = Bsel if name == "add" else Asel
        pre = np.concatenate([coeff(Bsel[l * n:(l + 1) * n], other[l * n:(l + 1) * n] % np.uint64(qs[l]), qs[l])
                              for l in range(limbs)])
        want = O.batch_transform(inv, pre, n, qs, psis)
        for l, o in enumerate(offs):
            assert (C[o:o + n] == want[l * n:(l + 1) * n]).all(), ("inverse", name, l)
    plan.close()


def test_add_sub_fused_aliasing_fallbacks_and_wide_words(device):
    """C may alias A or B^; cyclic plans and odd strides take the two-launch
    path with the same result; B^ words in [q, 2^32) are reduced first; a word
    >= 2^32 on a plan whose moduli are below 2^31 is reported."""
    n, limbs, batch = 1 << 14, 2, 2
    plan, qs, _ = _plan(device, n, limbs, 31, bc.NEGACYCLIC)
    total = limbs * batch * n
    rng = np.random.default_rng(21)
    A = rng.integers(0, qs[-1], total, dtype=np.uint64)
    Bh = rng.integers(0, 2**32, total, dtype=np.uint64)  # not reduced
    a, bh, c, x = upload(device, A), upload(device, Bh), _alloc(device, total), _alloc(device, total)
    plan.forward(a, x, batch)
    plan.forward_sub(a, bh, c, batch)
    device.synchronize()
    X, C = x.to_u64(), c.to_u64()
    for l in range(limbs):
        sl = slice(l * batch * n, (l + 1) * batch * n)
        q = np.uint64(qs[l])
        want = (X[sl] + q - Bh[sl] % q) % q
        assert (C[sl] == want).all(), l
    # aliasing: C = A, then C = B^
    y = upload(device, A)
    plan.forward_add(y, bh, y, batch)
    plan.forward_add(a, bh, c, batch)
    device.synchronize()
    assert (y.to_u64() == c.to_u64()).all()
    z = upload(device, Bh)
    plan.inverse_sub(a, z, z, batch)
    plan.inverse_sub(a, bh, c, batch)
    device.synchronize()
    assert (z.to_u64() == c.to_u64()).all()
    # cyclic plan: two launches, same result as the device chain
    cplan, cqs, _ = _plan(device, n, limbs, 31, bc.CYCLIC)
    cplan.forward(a, x, batch)
    cplan.forward_add(a, bh, c, batch)
    device.synchronize()
    X, C = x.to_u64(), c.to_u64()
    for l in range(limbs):
        sl = slice(l * batch * n, (l + 1) * batch * n)
        q = np.uint64(cqs[l])
        assert (C[sl] == (X[sl] + Bh[sl] % q) % q).all(), l
    # odd strides on the negacyclic plan: the two-launch path
    lay = bc.Layout(limb_stride=batch * (n + 1), poly_stride=n + 1)
    big = limbs * batch * (n + 1)
    a2, b2, c2, t2 = (_alloc(device, big) for _ in range(4))
    plan.fill_uniform(a2, batch, seed=1, layout=lay)
    plan.fill_uniform(b2, batch, seed=2, layout=lay)
    plan.inverse_add(a2, b2, c2, batch, layout=lay)
    plan.poly_add(a2, b2, t2, batch, layout=lay)
    plan.inverse(t2, t2, batch, layout=lay)
    device.synchronize()
    C2, T2 = c2.to_u64(), t2.to_u64()
    for l in range(limbs):
        for p in range(batch):
            o = l * batch * (n + 1) + p * (n + 1)
            assert (C2[o:o + n] == T2[o:o + n]).all(), (l, p)
    # a word >= 2^32 in B^ is reported, on both paths
    bad = Bh.copy()
    bad[7] = 2**40
    wb = upload(device, bad)
    with pytest.raises(bc.BarracudaError):
        plan.forward_add(a, wb, c, batch)
        device.synchronize()
    with pytest.raises(bc.BarracudaError):
        cplan.inverse_sub(a, wb, c, batch)
        device.synchronize()
    cplan.close()
    plan.close()


@pytest.mark.parametrize("logn", [10, 12, 14])
def test_polymul_shared_memory_path_for_odd_strides(device, logn):
    """Layouts the cluster kernels cannot take (odd strides) route negacyclic
    products to the single-CTA shared-memory kernel: same result as the
    schoolbook negacyclic convolution."""
    n, limbs, batch = 1 << logn, 2, 2
    plan, qs, _ = _plan(device, n, limbs, 31, bc.NEGACYCLIC)
    lay = bc.Layout(limb_stride=batch * (n + 1), poly_stride=n + 1)
    big = limbs * batch * (n + 1)
    a, b, c = (_alloc(device, big) for _ in range(3))
    plan.fill_uniform(a, batch, seed=21, layout=lay)
    plan.fill_uniform(b, batch, seed=22, layout=lay)
    plan.polymul(a, b, c, batch, layout=lay)
    device.synchronize()
    A, B, C = a.to_u64(), b.to_u64(), c.to_u64()
    for l, p in ((0, 0), (1, 1)):
        o = l * batch * (n + 1) + p * (n + 1)
        assert (C[o:o + n] == O.negacyclic_convolution(A[o:o + n], B[o:o + n], n, qs[l])).all(), (l, p)
    plan.close()


def _exact_negacyclic(x, n, q, psi):
    """Exact O(N log N) negacyclic forward transform of one polynomial (oracle)."""
    _, out = O.baseline_run("exact_negacyclic_ntt", x, n, [q], [psi], 1)
    return out


# N = 2^18 .. 2^24 run on the two-pass (2^18, 32-bit words) and three-pass
# kernels; 30-bit primes take the [0, 4q) word flavour, 31-bit [0, 2q), 60-bit
# the 64-bit words.
MULTIPASS_CASES = [(18, 31), (18, 30), (18, 60), (19, 31), (19, 60), (20, 31), (20, 30), (21, 60),
                   (22, 31), (23, 60), (24, 31), (24, 60)]


def _exact_cyclic_inverse(y, n, q, w):
    """N^-1 * NTT_{w^-1}(y), exact (oracle)."""
    t = O.exact_ntt(y, n, q, pow(w, -1, q))
    return O.exact_poly_mul(t, np.full(n, pow(n, -1, q), dtype=np.uint64), q)


@pytest.mark.parametrize("logn,bits", MULTIPASS_CASES)
@pytest.mark.parametrize("mode", [bc.NEGACYCLIC, bc.CYCLIC])
def test_plan_multipass_matches_oracle(device, logn, bits, mode):
    """N above the cluster kernels: exact forward and inverse values on the
    first and the last limb-polynomial of the batch, and the round trip of
    every one."""
    n, limbs, batch = 1 << logn, 2, 2
    plan, qs, roots = _plan(device, n, limbs, bits, mode)
    assert plan.info["kernel_kind"] == 2
    total = limbs * batch * n
    src, dst, back, inv = (_alloc(device, total) for _ in range(4))
    plan.fill_uniform(src, batch, seed=logn + bits)
    plan.forward(src, dst, batch)
    plan.inverse(dst, back, batch)
    plan.inverse(src, inv, batch)
    device.synchronize()
    x, X, Y = src.to_u64(), dst.to_u64(), inv.to_u64()
    assert (back.to_u64() == x).all()
    # the oracle takes ~8 s per transform at 2^24: one polynomial from 2^22 up
    for l, p in ((0, 0), (1, batch - 1)) if logn < 22 else ((1, batch - 1),):
        off = (l * batch + p) * n
        xs, q, r = x[off:off + n], qs[l], roots[l]
        if mode == bc.NEGACYCLIC:
            want_f = O.exact_negacyclic_ntt(xs, n, q, r)
            want_i = O.exact_negacyclic_intt(xs, n, q, r)
        else:
            want_f = O.exact_ntt(xs, n, q, r)
            want_i = _exact_cyclic_inverse(xs, n, q, r)
        assert (X[off:off + n] == want_f).all(), ("forward", l, p)
        assert (Y[off:off + n] == want_i).all(), ("inverse", l, p)
    plan.close()


@pytest.mark.parametrize("logn,limbs,batch", [(18, 3, 3), (19, 1, 5)])
def test_plan_multipass_reference_stage_structure(device, logn, limbs, batch):
    """Cyclic plans whose root is not a primitive N-th root (psi^4, a
    primitive N/2-th root): the outputs then depend on the reference's exact
    stage structure, which the multi-pass kernels follow through the plan's
    tables.  Forward and inverse against the restatement of the reference's
    shaders (exact below 2^31), on every limb, with odd limb and batch counts."""
    n = 1 << logn
    qs = bc.ntt_primes(31, n, limbs)
    roots = [pow(bc.negacyclic_root(q, n), 4, q) for q in qs]
    plan = bc.NttPlan(device, n, qs, roots, mode=bc.CYCLIC)
    assert plan.info["kernel_kind"] == 2
    total = limbs * batch * n
    src, dst, inv = (_alloc(device, total) for _ in range(3))
    plan.fill_uniform(src, batch, seed=logn * 3 + limbs)
    plan.forward(src, dst, batch)
    plan.inverse(src, inv, batch)
    device.synchronize()
    x, X, Y = src.to_u64(), dst.to_u64(), inv.to_u64()
    for l in range(limbs):
        off = (l * batch + (l % batch)) * n
        xs, q, w = x[off:off + n], qs[l], roots[l]
        assert (X[off:off + n] == O.ref_ntt(xs, n, q, w)).all(), ("forward", l)
        assert (Y[off:off + n] == O.ref_intt(xs, n, q, modinv(w, q))).all(), ("inverse", l)
    plan.close()


@pytest.mark.parametrize("logn,bits", [(18, 31), (20, 60), (21, 31)])
def test_plan_multipass_layouts(device, logn, bits):
    """The multi-pass kernels take any layout: padded strides, limbs not
    adjacent, unaligned pointers and in-place calls give the compact
    layout's results."""
    n, limbs, batch = 1 << logn, 2, 2
    plan, qs, psis = _plan(device, n, limbs, bits, bc.NEGACYCLIC)
    total = limbs * batch * n
    src, want = _alloc(device, total), _alloc(device, total)
    plan.fill_uniform(src, batch, seed=7)
    plan.forward(src, want, batch)
    device.synchronize()
    x, W = src.to_u64(), want.to_u64()
    pad, gap = 3, 5  # words after each polynomial, words between limbs
    lay = bc.Layout(limb_stride=batch * (n + pad) + gap, poly_stride=n + pad)
    words = limbs * lay.limb_stride + 1
    big_in, big_out = _alloc(device, words), _alloc(device, words)
    host = np.zeros(words, dtype=np.uint64)
    for l in range(limbs):
        for p in range(batch):
            o = 1 + l * lay.limb_stride + p * lay.poly_stride  # one word in: 8-byte aligned only
            host[o:o + n] = x[(l * batch + p) * n:(l * batch + p + 1) * n]
    N.check(N.lib().bc_buf_h2d(device.handle, big_in.ptr, host.ctypes.data, host.nbytes))
    base_in, base_out = big_in.ptr + 8, big_out.ptr + 8
    plan.forward(base_in, base_out, batch, layout=lay)
    plan.forward(base_in, base_in, batch, layout=lay)  # in place
    device.synchronize()
    out, inplace = big_out.to_u64(), big_in.to_u64()
    for l in range(limbs):
        for p in range(batch):
            o = 1 + l * lay.limb_stride + p * lay.poly_stride
            ref = W[(l * batch + p) * n:(l * batch + p + 1) * n]
            assert (out[o:o + n] == ref).all(), (l, p)
            assert (inplace[o:o + n] == ref).all(), (l, p)
    plan.close()


def test_reference_ops_from_threads_evict_cached_plans(device):
    """bc_fhe_ntt from four threads over 48 (N, q) pairs, more than the
    context's 32 cached plans: plans evicted while another thread runs on
    them stay alive until that call ends, and every result is exact."""
    import threading
    params = [(1 << (6 + i % 4), O.ntt_prime(30, 1 << (6 + i % 4), i)) for i in range(48)]
    errors = []

    def worker(tid):
        rng = np.random.default_rng(tid)
        try:
            for k in range(3 * len(params)):
                n, q = params[(k * 7 + tid * 13) % len(params)]
                w = pow(O.psi(q, n), 2, q)
                x = random_poly(rng, n, q)
                got = ntt(device, x, n, q, w)
                if not (got == O.ref_ntt(x, n, q, w)).all():
                    errors.append((tid, n, q))
        except Exception as e:  # pragma: no cover - reported below
            errors.append((tid, repr(e)))

    threads = [threading.Thread(target=worker, args=(t,)) for t in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=300)
    assert not errors, errors[:5]


def test_plan_shared_by_two_streams_multipass(device):
    """One plan, two streams, different batch sizes in flight at once on the
    multi-pass path: each call has its own temporary, so both results equal
    the single-stream ones."""
    import torch
    n, limbs = 1 << 18, 1
    plan, qs, psis = _plan(device, n, limbs, 31, bc.NEGACYCLIC)
    bufs = {}
    for batch in (2, 6):
        src, dst = _alloc(device, batch * n), _alloc(device, batch * n)
        plan.fill_uniform(src, batch, seed=batch)
        plan.forward(src, dst, batch)
        device.synchronize()
        bufs[batch] = (src, dst, dst.to_u64().copy())
    streams = {2: torch.cuda.Stream(), 6: torch.cuda.Stream()}
    for _ in range(3):
        for batch, (src, dst, _) in bufs.items():
            plan.forward(src, dst, batch, stream=streams[batch].cuda_stream)
    torch.cuda.synchronize()
    for batch, (_, dst, want) in bufs.items():
        assert (dst.to_u64() == want).all(), batch
    plan.close()


@pytest.mark.parametrize("logn,bits", [(12, 31), (14, 31), (15, 31), (16, 31), (17, 31), (13, 30), (16, 30),
                                       (13, 60), (15, 60)])
@pytest.mark.parametrize("mode", [bc.NEGACYCLIC, bc.CYCLIC])
def test_plan_polymul_matches_chain(device, logn, bits, mode):
    n, limbs, batch = 1 << logn, 2, 2
    plan, qs, roots = _plan(device, n, limbs, bits, mode)
    total = limbs * batch * n
    a, b, c = _alloc(device, total), _alloc(device, total), _alloc(device, total)
    plan.fill_uniform(a, batch, seed=1)
    plan.fill_uniform(b, batch, seed=2)
    plan.polymul(a, b, c, batch)
    device.synchronize()
    A, B, C = a.to_u64(), b.to_u64(), c.to_u64()
    for l in range(limbs):
        off = (l * batch + 1) * n
        q, r = qs[l], roots[l]
        if mode == bc.NEGACYCLIC:
            if bits <= 31:
                want = O.ref_negacyclic_intt(O.ref_pointwise(O.ref_negacyclic_ntt(A[off:off + n], n, q, r),
                                                             O.ref_negacyclic_ntt(B[off:off + n], n, q, r), n, q),
                                             n, q, r)
            else:
                Xa = O.exact_negacyclic_ntt(A[off:off + n], n, q, r)
                Xb = O.exact_negacyclic_ntt(B[off:off + n], n, q, r)
                want = O.exact_negacyclic_intt(np.array([OL.orc_mulmod(int(u), int(v), q)
                                                         for u, v in zip(Xa, Xb)], np.uint64), n, q, r)
        else:
            if bits <= 31:
                want = O.ref_fast_poly_mul(A[off:off + n], B[off:off + n], n, q, r)
            else:
                w = r
                Xa, Xb = O.exact_ntt(A[off:off + n], n, q, w), O.exact_ntt(B[off:off + n], n, q, w)
                prod = np.array([OL.orc_mulmod(int(u), int(v), q) for u, v in zip(Xa, Xb)], np.uint64)
                winv = modinv(w, q)
                ninv = modinv(n, q)
                want = np.array([OL.orc_mulmod(int(v), ninv, q) for v in O.exact_ntt(prod, n, q, winv)], np.uint64)
        assert (C[off:off + n] == want).all(), (l, mode, bits)


def test_plan_pointwise(device):
    n, limbs, batch = 1 << 12, 2, 3
    plan, qs, _ = _plan(device, n, limbs, 31, bc.NEGACYCLIC)
    total = limbs * batch * n
    a, b, c = _alloc(device, total), _alloc(device, total), _alloc(device, total)
    plan.fill_uniform(a, batch, seed=3)
    plan.fill_uniform(b, batch, seed=4)
    plan.pointwise_mul(a, b, c, batch)
    device.synchronize()
    A, B, C = a.to_u64(), b.to_u64(), c.to_u64()
    for l in range(limbs):
        sl = slice(l * batch * n, (l + 1) * batch * n)
        assert (C[sl] == O.ref_pointwise(A[sl], B[sl], batch * n, qs[l])).all()


@pytest.mark.parametrize("logn", [15, 18])
def test_cyclic_polymul_non_primitive_root_takes_the_reference_chain(device, logn):
    """A cyclic root that is not a primitive N-th root (here an N/2-th root)
    keeps the reference's stage structure: bc_polymul takes the unfused chain
    through a pool temporary and equals FheFastPolyMul's output bit for bit.
    N = 2^18 is above the cluster kernels, where every cyclic product takes
    that chain."""
    n, limbs, batch = 1 << logn, 2, 2
    qs = bc.ntt_primes(31, n, limbs)
    psis = [bc.negacyclic_root(q, n) for q in qs]
    roots = [pow(p, 4, q) for p, q in zip(psis, qs)] if logn == 15 else [p * p % q for p, q in zip(psis, qs)]
    plan = bc.NttPlan(device, n, qs, roots, mode=bc.CYCLIC)
    total = limbs * batch * n
    a, b, c = _alloc(device, total), _alloc(device, total), _alloc(device, total)
    plan.fill_uniform(a, batch, seed=5)
    plan.fill_uniform(b, batch, seed=6)
    for _ in range(2):  # the pool temporary is reused by the second call
        plan.polymul(a, b, c, batch)
    device.synchronize()
    A, B, C = a.to_u64(), b.to_u64(), c.to_u64()
    for l in range(limbs):
        off = (l * batch + 1) * n
        want = O.ref_fast_poly_mul(A[off:off + n], B[off:off + n], n, qs[l], roots[l])
        assert (C[off:off + n] == want).all(), (logn, l)
    plan.close()


@pytest.mark.parametrize("mode", [bc.NEGACYCLIC, bc.CYCLIC])
@pytest.mark.parametrize("bits", [31, 60])
def test_polymul_aliasing(device, bits, mode):
    """C may alias A, B or both (squaring in place); results as with separate buffers."""
    n, limbs, batch = 1 << 15, 2, 2
    plan, qs, roots = _plan(device, n, limbs, bits, mode)
    total = limbs * batch * n
    a, b, c, ref, sq = (_alloc(device, total) for _ in range(5))
    plan.fill_uniform(a, batch, seed=3)
    plan.fill_uniform(b, batch, seed=4)
    plan.polymul(a, b, ref, batch)
    plan.polymul(a, a, sq, batch)
    device.synchronize()
    A, B, want, want_sq = a.to_u64(), b.to_u64(), ref.to_u64(), sq.to_u64()

    def put(t, x):
        N.check(N.lib().bc_buf_h2d(device.handle, t.ptr, x.ctypes.data, x.nbytes))

    put(c, A)
    plan.polymul(c, b, c, batch)          # C aliases A
    device.synchronize()
    assert (c.to_u64() == want).all()
    put(c, B)
    plan.polymul(a, c, c, batch)          # C aliases B
    device.synchronize()
    assert (c.to_u64() == want).all()
    put(c, A)
    plan.polymul(c, c, c, batch)          # A == B == C
    device.synchronize()
    assert (c.to_u64() == want_sq).all()


def test_digest_is_order_sensitive(device):
    n = 4096
    a = np.arange(n, dtype=np.uint64)
    t = upload(device, a)
    out = _alloc(device, 1)
    bc.digest(device, t, n, out)
    device.synchronize()
    d1 = int(out.to_u64()[0])
    t2 = upload(device, a[::-1].copy())
    bc.digest(device, t2, n, out)
    device.synchronize()
    assert d1 != int(out.to_u64()[0])


def test_digest_matches_oracle_and_adds_over_shards(device):
    rng = np.random.default_rng(5)
    x = rng.integers(0, 2**63, 10000, dtype=np.uint64)
    t = upload(device, x)
    out = _alloc(device, 1)
    got = []
    for first, lo, hi in ((0, 0, 10000), (0, 0, 3000), (3000, 3000, 10000)):
        sub = upload(device, x[lo:hi])
        bc.digest(device, sub, hi - lo, out, first_index=first)
        device.synchronize()
        got.append(int(out.to_u64()[0]))
        assert got[-1] == O.digest(x[lo:hi], first)
    assert got[0] == (got[1] + got[2]) % 2**64


# ------------------------------------------------------- coefficient-wise ops

COEFF_MODULI = [1, 97, 100, 12289, 2147352577, 4294967291, 1152921504606584833,
                (1 << 63) + 29, (1 << 64) - 59]


def _coeff_inputs(rng, n, q):
    """Reduced values, arbitrary u64 words, and values next to 2^64 (wrap-around)."""
    top = np.uint64(2**64 - 1)
    parts = [rng.integers(0, q, n // 2, dtype=np.uint64, endpoint=False) if q > 1 else np.zeros(n // 2, np.uint64),
             rng.integers(0, 2**64 - 1, n // 4, dtype=np.uint64, endpoint=True),
             top - rng.integers(0, 1000, n - n // 2 - n // 4, dtype=np.uint64)]
    x = np.concatenate(parts)
    rng.shuffle(x)
    return x


@pytest.mark.parametrize("q", COEFF_MODULI)
def test_coeff_ops_match_reference_and_exact(device, q):
    """FhePolyAdd / FhePolySub: bit-exact with the reference's shaders for any
    u64 inputs; FhePolyMul: the exact residue (a * b) mod q.  Degree 1000
    (the ops take any degree)."""
    n = 1000
    rng = np.random.default_rng(q % 1000003)
    a, b = _coeff_inputs(rng, n, q), _coeff_inputs(rng, n, q)
    assert (coeff_op(device, "add", a, b, n, q) == O.ref_poly_add(a, b, q)).all()
    assert (coeff_op(device, "sub", a, b, n, q) == O.ref_poly_sub(a, b, q)).all()
    assert (coeff_op(device, "mul", a, b, n, q) == O.exact_poly_mul(a, b, q)).all()


@pytest.mark.parametrize("bits", [31, 60])
def test_plan_coeff_ops(device, bits):
    """Batched bc_poly_add / _sub / _mul over limbs x polynomials, strided layout."""
    n, limbs, batch = 1 << 12, 3, 5
    plan, qs, _ = _plan(device, n, limbs, bits, bc.NEGACYCLIC)
    lay = bc.Layout(limb_stride=n, poly_stride=limbs * n)  # [poly][limb][N]
    total = limbs * batch * n
    rng = np.random.default_rng(bits)
    A = rng.integers(0, 2**64 - 1, total, dtype=np.uint64, endpoint=True)
    B = rng.integers(0, 2**64 - 1, total, dtype=np.uint64, endpoint=True)
    A[: total // 2] %= np.uint64(qs[0])
    a, b, c = upload(device, A), upload(device, B), _alloc(device, total)
    for op, ref in (("add", O.ref_poly_add), ("sub", O.ref_poly_sub), ("mul", O.exact_poly_mul)):
        getattr(plan, f"poly_{op}")(a, b, c, batch, layout=lay)
        device.synchronize()
        C = c.to_u64()
        for p in range(batch):
            for l in range(limbs):
                o = (p * limbs + l) * n
                assert (C[o:o + n] == ref(A[o:o + n], B[o:o + n], qs[l])).all(), (op, p, l)
    plan.close()


# ------------------------------------------------------------- IPC methods

def test_ipc_fhe_methods_on_gpu(device):
    """fhe.ntt / fhe.intt / fhe.pointwise_mul over the NDJSON transport, against
    the reference's known vector and the oracle."""
    from barracuda_b200 import ipc
    srv = ipc.FheIpc(device).serve_tcp("127.0.0.1", 0)
    try:
        r = ipc.call(srv.server_address, {"jsonrpc": "2.0", "method": "barracuda.fhe.ntt", "id": 1,
                                          "params": {"modulus": 17, "degree": 4, "root_of_unity": 4,
                                                     "coefficients": [1, 2, 3, 4]}})
        assert r == {"jsonrpc": "2.0", "id": 1, "result": {"degree": 4, "modulus": 17, "result": [10, 7, 15, 6],
                                                            "status": "completed"}}
        r = ipc.call(srv.server_address, {"jsonrpc": "2.0", "method": "fhe.intt", "id": 2,
                                          "params": {"modulus": 17, "degree": 4, "inv_root_of_unity": 13,
                                                     "coefficients": [10, 7, 15, 6]}})
        assert r["result"]["result"] == [1, 2, 3, 4]
        n, q = 64, 12289
        rng = np.random.default_rng(5)
        a, b = random_poly(rng, n, q), random_poly(rng, n, q)
        r = ipc.call(srv.server_address, {"jsonrpc": "2.0", "method": "fhe.pointwise_mul", "id": 3,
                                          "params": {"modulus": q, "degree": n, "a": [int(v) for v in a],
                                                     "b": [int(v) for v in b]}})
        assert r["result"]["result"] == [int(v) for v in O.ref_pointwise(a, b, n, q)]
        r = ipc.call(srv.server_address, {"jsonrpc": "2.0", "method": "fhe.ntt", "id": 4,
                                          "params": {"modulus": 19, "degree": 8, "root_of_unity": 2,
                                                     "coefficients": list(range(8))}})
        assert r["error"] == {"code": ipc.INTERNAL_ERROR, "message":
                              "NTT setup failed: Device error: Modulus 19 must satisfy q ≡ 1 (mod 2N) where N=8"}
    finally:
        srv.shutdown()
        srv.server_close()
