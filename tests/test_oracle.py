"""Pins the CPU oracle (oracle/, a C restatement of the reference WGSL path)
against the reference's own known answers and against exact arithmetic."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import compute_primitive_root, find_root_of_unity, modinv, random_poly, resolve_root

L = O.lib()


def test_golden_cases(kats):
    rng = np.random.default_rng(7)
    for c in kats["cases"]:
        k = c["kind"]
        if k == "twiddles":
            assert list(O.ref_twiddles(c["degree"], c["modulus"], c["root"])) == c["expect"], c["name"]
        elif k == "modinv":
            assert L.orc_ref_modinv(c["a"], c["m"]) == c["expect"], c["name"]
        elif k == "inverse_root":
            assert L.orc_ref_compute_inverse_root(c["degree"], c["modulus"], c["root"]) == c["expect"]
        elif k == "ntt":
            assert list(O.ref_ntt(c["input"], c["degree"], c["modulus"], c["root"])) == c["expect"]
        elif k == "roundtrip":
            n, q = c["degree"], c["modulus"]
            r = resolve_root(c["root"], n, q)
            back = O.ref_intt(O.ref_ntt(c["input"], n, q, r), n, q, modinv(r, q))
            assert [int(v) % q for v in back] == [v % q for v in c["input"]], c["name"]
        elif k == "linearity":
            n, q = c["degree"], c["modulus"]
            r = resolve_root(c["root"], n, q)
            a, b = np.array(c["a"], np.uint64), np.array(c["b"], np.uint64)
            # NTT(FhePolyAdd(a, b)) == FhePolyAdd(NTT(a), NTT(b))
            lhs = O.ref_ntt(O.ref_poly_add(a, b, q), n, q, r)
            rhs = O.ref_poly_add(O.ref_ntt(a, n, q, r), O.ref_ntt(b, n, q, r), q)
            assert (lhs == rhs).all()
        elif k == "ntt_zero":
            n, q = c["degree"], c["modulus"]
            assert (O.ref_ntt(c["input"], n, q, resolve_root(c["root"], n, q)) == 0).all()
        elif k == "ntt_range":
            n, q = c["degree"], c["modulus"]
            assert (O.ref_ntt(c["input"], n, q, resolve_root(c["root"], n, q)) < q).all()
        elif k == "pointwise":
            assert list(O.ref_pointwise(c["a"], c["b"], c["degree"], c["modulus"])) == c["expect"]
        elif k == "pointwise_identity":
            n, q = c["degree"], c["modulus"]
            r = resolve_root(c["root"], n, q)
            x = random_poly(rng, n, q)
            one = np.zeros(n, np.uint64)
            one[0] = 1
            got = O.ref_pointwise(O.ref_ntt(x, n, q, r), O.ref_ntt(one, n, q, r), n, q)
            assert (got == O.ref_ntt(x, n, q, r)).all()
        elif k == "pointwise_zero":
            n, q = c["degree"], c["modulus"]
            r = resolve_root(c["root"], n, q)
            x = random_poly(rng, n, q)
            got = O.ref_pointwise(O.ref_ntt(x, n, q, r), O.ref_ntt(np.zeros(n, np.uint64), n, q, r), n, q)
            assert (got == 0).all()
        elif k == "fast_mul_naive":
            n, q = c["degree"], c["modulus"]
            r = resolve_root(c["root"], n, q)
            a, b = random_poly(rng, n, q), random_poly(rng, n, q)
            assert (O.ref_fast_poly_mul(a, b, n, q, r) == O.cyclic_convolution(a, b, n, q)).all()
        elif k == "fast_mul_commutative":
            n, q = c["degree"], c["modulus"]
            r = resolve_root(c["root"], n, q)
            a, b = random_poly(rng, n, q), random_poly(rng, n, q)
            assert (O.ref_fast_poly_mul(a, b, n, q, r) == O.ref_fast_poly_mul(b, a, n, q, r)).all()
        elif k == "fast_mul_distributive":
            n, q = c["degree"], c["modulus"]
            r = resolve_root(c["root"], n, q)
            a, b, cc = (random_poly(rng, n, q) for _ in range(3))
            lhs = O.ref_fast_poly_mul(a, (b + cc) % np.uint64(q), n, q, r)
            rhs = (O.ref_fast_poly_mul(a, b, n, q, r) + O.ref_fast_poly_mul(a, cc, n, q, r)) % np.uint64(q)
            assert (lhs == rhs).all()
        elif k in ("poly_add", "poly_sub", "poly_mul"):
            f = {"poly_add": O.ref_poly_add, "poly_sub": O.ref_poly_sub, "poly_mul": O.ref_poly_mul}[k]
            assert list(f(c["a"], c["b"], c["modulus"])) == c["expect"], c["name"]
            if k == "poly_mul":
                assert list(O.exact_poly_mul(c["a"], c["b"], c["modulus"])) == c["expect"], c["name"]
        elif k == "poly_add_assoc":
            q = c["modulus"]
            a, b, cc = c["a"], c["b"], c["c"]
            lhs = O.ref_poly_add(O.ref_poly_add(a, b, q), cc, q)
            assert (lhs == O.ref_poly_add(a, O.ref_poly_add(b, cc, q), q)).all()
        elif k == "rotate":
            n, q, x = c["degree"], c["modulus"], c["input"]
            for r in c["rotations"]:
                x = O.ref_rotate(x, n, r, q)
            assert [int(v) for v in x] == c["expect"], c["name"]
            for r in c.get("same_as_rotations", []):
                assert (O.ref_rotate(c["input"], n, r, q) == x).all(), c["name"]
        elif k == "modulus_switch":
            x, qo, qn = c["input"], c["modulus_old"], c["modulus_new"]
            assert [int(v) for v in O.ref_modulus_switch(x, qo, qn)] == c["expect"], c["name"]
            assert [int(v) for v in O.exact_modulus_switch(x, qo, qn)] == c["exact"], c["name"]
        elif k == "key_switch":
            got = O.ref_key_switch(c["input"], c["decomp_base"], c["decomp_levels"])
            assert [int(v) for v in got] == c["expect"], c["name"]
        else:
            raise AssertionError(f"unknown kind {k}")


def test_known_roots_and_ntt_params(kats):
    for d, m, r in kats["known_roots"]["values"]:
        assert pow(r, d, m) == 1 and pow(r, d // 2, m) != 1
        assert find_root_of_unity(d, m) == r
    for m, d in kats["ntt_params"]["values"]:
        r = compute_primitive_root(d, m)
        assert pow(r, d, m) == 1 and pow(r, d // 2, m) != 1, (m, d, r)


def test_wgsl_helpers_are_exact_products():
    rng = np.random.default_rng(1)
    for _ in range(2000):
        a, b = (int(x) for x in rng.integers(0, 2**64, 2, dtype=np.uint64))
        assert L.orc_wgsl_u64_mul(a, b) == (a * b) % 2**64
        a32, b32 = a & 0xFFFFFFFF, b & 0xFFFFFFFF
        assert L.orc_wgsl_mul32_wide(a32, b32) == a32 * b32


@pytest.mark.parametrize("n", [2, 4, 8, 64, 256])
def test_reference_restatement_exact_below_2_31(n):
    """For q < 2^31 the reference chain is exact: restatement == u128 math."""
    rng = np.random.default_rng(n)
    for bits in (14, 20, 30, 31):
        q = O.ntt_prime(bits, n, 0)
        psi = O.psi(q, n)
        w = L.orc_mulmod(psi, psi, q)
        x = random_poly(rng, n, q)
        assert (O.ref_ntt(x, n, q, w) == O.exact_ntt(x, n, q, w)).all()
        assert (O.ref_ntt(x, n, q, w) == O.exact_dft(x, n, q, w)).all()
        assert (O.ref_negacyclic_ntt(x, n, q, psi) == O.exact_negacyclic_ntt(x, n, q, psi)).all()
        X = O.exact_negacyclic_ntt(x, n, q, psi)
        assert (O.ref_negacyclic_intt(X, n, q, psi) == x).all()
        assert (O.exact_negacyclic_intt(X, n, q, psi) == x).all()


def test_reference_diverges_at_or_above_2_31():
    """Pins (documents) the reference's truncated arithmetic for wide moduli:
    fhe_ntt.wgsl:45-110 keeps only the low 64 product bits and its bit-serial
    reduction overflows once q >= 2^31.  The CUDA path computes exact residues
    there instead, so parity with the reference is claimed only below 2^31."""
    n = 64
    rng = np.random.default_rng(3)
    for bits in (32, 60):
        q = O.ntt_prime(bits, n, 0)
        psi = O.psi(q, n)
        w = L.orc_mulmod(psi, psi, q)
        x = random_poly(rng, n, q)
        ref = O.ref_ntt(x, n, q, w)
        assert not (ref % np.uint64(q) == O.exact_ntt(x, n, q, w)).all()


def test_reference_domain_extends_to_u32_inputs():
    """For q < 2^31 and inputs below 2^32 (not necessarily < q) the reference
    output, canonically reduced, is the exact transform of x mod q."""
    rng = np.random.default_rng(11)
    for n in (4, 16, 128):
        q = O.ntt_prime(31, n, 0)
        w = L.orc_mulmod(O.psi(q, n), O.psi(q, n), q)
        x = rng.integers(0, 2**32, n, dtype=np.uint64)
        ref = O.ref_ntt(x, n, q, w) % np.uint64(q)
        assert (ref == O.exact_ntt(x % np.uint64(q), n, q, w)).all()
        inv = O.ref_intt(x, n, q, modinv(w, q)) % np.uint64(q)
        back = O.exact_ntt(x % np.uint64(q), n, q, modinv(w, q))
        ninv = modinv(n, q)
        assert (inv == np.array([L.orc_mulmod(int(v), ninv, q) for v in back], np.uint64)).all()


@pytest.mark.parametrize("n", [4, 8, 32, 256])
def test_negacyclic_chain_is_negacyclic_convolution(n):
    rng = np.random.default_rng(n + 100)
    q = O.ntt_prime(31, n, 2)
    psi = O.psi(q, n)
    a, b = random_poly(rng, n, q), random_poly(rng, n, q)
    A, B = O.ref_negacyclic_ntt(a, n, q, psi), O.ref_negacyclic_ntt(b, n, q, psi)
    C = O.ref_pointwise(A, B, n, q)
    assert (O.ref_negacyclic_intt(C, n, q, psi) == O.negacyclic_convolution(a, b, n, q)).all()


def test_invalid_root_canary_is_structure_dependent():
    """validate_gpu.rs:277 passes omega = 11 for N = 8, q = 12289, but
    11^8 != 1 mod 12289: the forward output is not a DFT, so only the
    reference's DIT network reproduces it (the round trip still holds)."""
    n, q, w = 8, 12289, 11
    assert pow(w, n, q) != 1
    x = np.arange(1, 9, dtype=np.uint64)
    assert not (O.ref_ntt(x, n, q, w) == O.exact_dft(x, n, q, w)).all()
    assert (O.ref_intt(O.ref_ntt(x, n, q, w), n, q, modinv(w, q)) == x).all()


def test_prime_families_match_plan():
    # largest primes q = 1 mod 2N below 2^31 (reference-exact family) and 2^60 (60-bit family)
    assert O.ntt_prime(31, 1 << 12, 0) == 2147377153
    assert O.ntt_prime(31, 1 << 14, 0) == 2147352577
    assert O.ntt_prime(31, 1 << 16, 0) == 2147352577
    assert O.ntt_prime(31, 1 << 17, 0) == 2146959361
    assert O.ntt_prime(60, 1 << 12, 0) == 1152921504606830593
    assert O.ntt_prime(60, 1 << 14, 0) == 1152921504606748673
    assert O.ntt_prime(60, 1 << 16, 0) == 1152921504606584833
    for n in (1 << 12, 1 << 16, 1 << 17):
        for i in range(3):
            q = O.ntt_prime(31, n, i)
            assert L.orc_is_prime(q) and (q - 1) % (2 * n) == 0 and q < 2**31
            psi = O.psi(q, n)
            assert L.orc_powmod(psi, n, q) == q - 1


def test_seeded_generator_uniform_range():
    q = O.ntt_prime(31, 4096, 0)
    v = O.seeded_fill(1 << 16, 0, 0, q)
    assert (v < q).all()
    assert abs(float(v.mean()) / q - 0.5) < 0.01
    assert O.seeded_fill(8, 5, 100, q).tolist() == [L.orc_seeded_value(5, 100 + i, q) for i in range(8)]


def test_poly_ops_restatement_vs_exact():
    """FhePolyAdd/Sub match (a +- b) mod q for reduced inputs; FhePolyMul's
    shader matches the exact product only while a * b < 1001 q and its 32x32
    partial products do not overflow, which the reference's own tests stay
    within.  The CUDA path computes the exact residue everywhere."""
    rng = np.random.default_rng(3)
    for q in (97, 100, 12289, 2147352577, 1152921504606584833):
        a = rng.integers(0, q, 2000, dtype=np.uint64)
        b = rng.integers(0, q, 2000, dtype=np.uint64)
        add = np.array([(int(x) + int(y)) % q for x, y in zip(a, b)], np.uint64)
        sub = np.array([(int(x) - int(y)) % q for x, y in zip(a, b)], np.uint64)
        assert (O.ref_poly_add(a, b, q) == add).all()
        assert (O.ref_poly_sub(a, b, q) == sub).all()
        exact = np.array([int(x) * int(y) % q for x, y in zip(a, b)], np.uint64)
        assert (O.exact_poly_mul(a, b, q) == exact).all()
        small = rng.integers(0, 31, 2000, dtype=np.uint64) % np.uint64(q)  # a * b < 1001 q
        assert (O.ref_poly_mul(small, small, q) == O.exact_poly_mul(small, small, q)).all()
    # divergence pinned: operands near a 31-bit modulus leave the shader's range
    q = 2147352577
    a = np.array([q - 1, q - 2, 123456789], np.uint64)
    assert (O.ref_poly_mul(a, a, q) != O.exact_poly_mul(a, a, q)).all()


def _py_automorphism(x, n, g, q):
    out = [0] * n
    for i, v in enumerate(int(t) for t in x):
        p = i * g % (2 * n)
        out[p % n] = ((q - v) % 2**64 if v else 0) if p >= n else v
    return out


@pytest.mark.parametrize("n", [4, 8, 64, 1024])
def test_rotate_oracle_is_the_ring_automorphism(n):
    """FheRotate's map is X -> X^g on Z_q[X]/(X^N + 1): it agrees with a
    Python restatement, composes by multiplying galois elements mod 2N, and
    is a ring homomorphism of the negacyclic product (inputs below q)."""
    rng = np.random.default_rng(n)
    q = O.ntt_prime(30, n, 0)
    a, b = random_poly(rng, n, q), random_poly(rng, n, q)
    for r in sorted({-n // 2, -1, 0, 1, 3 % (n // 2 + 1), n // 2}):
        g = L.orc_ref_rotate_galois(n, r)
        ra = O.ref_rotate(a, n, r, q)
        assert [int(v) for v in ra] == _py_automorphism(a, n, g, q)
        assert (ra == O.automorphism(a, n, g, q)).all()
        prod = O.negacyclic_convolution(a, b, n, q)
        assert (O.ref_rotate(prod, n, r, q) ==
                O.negacyclic_convolution(ra, O.ref_rotate(b, n, r, q), n, q)).all()
        for g2 in (3, 2 * n - 1):
            both = O.automorphism(ra, n, g2, q)
            assert (both == O.automorphism(a, n, g * g2 % (2 * n), q)).all()
    assert (O.ref_rotate(a, n, 0, q) == a).all()


def test_modulus_switch_restatement_vs_exact():
    """The shader's wrapping u64 product equals the exact rounding wherever
    c * q_new < 2^64 (and q_old <= 2^63); the exact map agrees with Python
    integers everywhere."""
    rng = np.random.default_rng(5)
    for _ in range(3000):
        qo = int(rng.integers(2, 2**int(rng.integers(2, 65)), dtype=np.uint64, endpoint=False)) | 1
        qn = int(rng.integers(0, qo, dtype=np.uint64))
        c = int(rng.integers(0, 2**64, dtype=np.uint64))
        want = ((2 * c * qn + qo) // (2 * qo)) % qn if qn else 0
        assert L.orc_exact_modulus_switch1(c, qo, qn) == want, (c, qo, qn)
        if c * qn < 2**64 and qo <= 2**63:
            assert L.orc_ref_modulus_switch1(c, qo, qn) == want, (c, qo, qn)
    assert L.orc_ref_modulus_switch1(5, 1, 0) == 0 and L.orc_exact_modulus_switch1(5, 1, 0) == 0


def test_decompose_oracle_digits():
    rng = np.random.default_rng(3)
    x = rng.integers(0, 2**64, 257, dtype=np.uint64)
    for base, levels in ((2, 64 // 2), (16, 16), (1 << 16, 4), (1 << 24, 3), (12289, 5), (3, 32)):
        levels = min(levels, 32)
        d = O.decompose(x, base, levels)
        for i in (0, 1, 100, 256):
            v = int(x[i])
            for l in range(levels):
                assert int(d[l, i]) == (v // base**l) % base
    # FheKeySwitch's net effect is a copy of its input
    assert (O.ref_key_switch(x, 1 << 16, 3) == x).all()
