"""Shared helpers for the tests: the reference's own test utilities restated
(tests/fhe/helpers.rs) and seeded input generation."""
import numpy as np

from oracle import oracle

KNOWN_ROOTS = [(4, 17, 4), (4, 97, 22), (4, 257, 241), (4, 12289, 1479), (8, 97, 64), (16, 97, 8)]


def compute_primitive_root(degree, modulus):
    return int(oracle.lib().orc_ref_compute_primitive_root(degree, modulus))


def find_root_of_unity(degree, modulus):
    """tests/fhe/helpers.rs:53-100 find_root_of_unity."""
    for d, m, r in KNOWN_ROOTS:
        if d == degree and m == modulus:
            return r
    if (modulus - 1) % (2 * degree) == 0:
        root = compute_primitive_root(degree, modulus)
        if pow(root, degree, modulus) == 1 and root != 1:
            return root
    for cand in range(2, min(modulus, 100)):
        if pow(cand, degree, modulus) == 1 and all(pow(cand, k, modulus) != 1 for k in range(1, degree)):
            return cand
    return None


def resolve_root(spec, degree, modulus):
    if isinstance(spec, int):
        return spec
    if spec == "compute_primitive_root":
        return compute_primitive_root(degree, modulus)
    return find_root_of_unity(degree, modulus)


def random_poly(rng, degree, modulus):
    return (rng.integers(0, 2**63, size=degree, dtype=np.uint64) % np.uint64(modulus)).astype(np.uint64)


def modinv(a, m):
    return int(oracle.lib().orc_ref_modinv(a, m))
