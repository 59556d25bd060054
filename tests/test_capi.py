"""CPU tests of the C ABI library: it loads, exports every declared symbol, and
its host-side logic (validation text, roots, primes, tables, shard split)
matches the reference and the oracle.  No kernel is launched here."""
import ctypes
import os
import re

import numpy as np
import pytest

import barracuda_b200 as bc
from barracuda_b200 import _native as N
from oracle import oracle as O
from tests.helpers import compute_primitive_root

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "barracuda_fhe.h")


def declared_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(bc_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = N.lib()
    syms = declared_symbols()
    assert len(syms) >= 39
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing
    # and the Python binding declares a signature for each of them
    assert sorted(N.SIGNATURES) == syms


def test_abi_version():
    assert N.lib().bc_abi_version() == 1


def _check_msg(fn, *args):
    st = fn(*args)
    return st, (N.last_error() if st else "")


def test_fhe_ntt_validation_messages():
    L = N.lib()
    assert _check_msg(L.bc_fhe_ntt_check, 6, 4, 17, 4) == (
        N.BC_ERR_DEVICE, "Input length 6 doesn't match expected 8 (degree 4 * 2)")
    assert _check_msg(L.bc_fhe_ntt_check, 6, 3, 17, 4) == (
        N.BC_ERR_DEVICE, "Degree 3 must be a power of 2 ≥ 2 for NTT")
    assert _check_msg(L.bc_fhe_ntt_check, 2, 1, 17, 4) == (
        N.BC_ERR_DEVICE, "Degree 1 must be a power of 2 ≥ 2 for NTT")
    assert _check_msg(L.bc_fhe_ntt_check, 8, 4, 0, 4) == (N.BC_ERR_DEVICE, "Modulus must be non-zero")
    assert _check_msg(L.bc_fhe_ntt_check, 16, 8, 19, 2) == (
        N.BC_ERR_DEVICE, "Modulus 19 must satisfy q ≡ 1 (mod 2N) where N=8")
    assert L.bc_fhe_ntt_check(8, 4, 17, 4) == 0
    # q = 1 passes the reference's congruence check ((1 - 1) % 2N == 0)
    assert L.bc_fhe_ntt_check(8, 4, 1, 0) == 0


@pytest.mark.parametrize("op", ["add", "sub", "mul"])
def test_fhe_poly_coeff_validation_messages(op):
    """FhePolyAdd/Sub/Mul::new (ops/fhe_poly_{add,sub,mul}.rs): lengths, then modulus."""
    L = N.lib()
    f = getattr(L, f"bc_fhe_poly_{op}_check")
    assert _check_msg(f, 14, 16, 8, 97) == (
        N.BC_ERR_DEVICE, "poly_a length 14 doesn't match expected 16 (degree 8 * 2)")
    assert _check_msg(f, 16, 10, 8, 97) == (
        N.BC_ERR_DEVICE, "poly_b length 10 doesn't match expected 16 (degree 8 * 2)")
    assert _check_msg(f, 16, 16, 8, 0) == (N.BC_ERR_DEVICE, "Modulus must be non-zero")
    assert f(16, 16, 8, 97) == 0
    assert f(6, 6, 3, 100) == 0  # no power-of-two or prime requirement
    assert f(0, 0, 0, 5) == 0


def test_fhe_intt_validation_messages():
    L = N.lib()
    assert _check_msg(L.bc_fhe_intt_check, 6, 4, 17, 13) == (
        N.BC_ERR_DEVICE, "Input length 6 doesn't match expected 8 (degree 4 * 2)")
    assert _check_msg(L.bc_fhe_intt_check, 6, 3, 17, 13) == (
        N.BC_ERR_DEVICE, "Degree 3 must be a power of 2 for INTT")
    assert _check_msg(L.bc_fhe_intt_check, 0, 0, 17, 13) == (
        N.BC_ERR_DEVICE, "Degree 0 must be a power of 2 for INTT")
    assert _check_msg(L.bc_fhe_intt_check, 8, 4, 0, 13) == (N.BC_ERR_DEVICE, "Modulus must be non-zero")
    assert L.bc_fhe_intt_check(2, 1, 17, 1) == 0          # degree 1 is accepted
    assert L.bc_fhe_intt_check(16, 8, 19, 2) == 0         # no congruence check


def test_pair_validation_messages():
    L = N.lib()
    for fn, extra in ((L.bc_fhe_pointwise_mul_check, ()), (L.bc_fhe_fast_poly_mul_check, (4,))):
        assert _check_msg(fn, 12, 12, 6, 17, *extra) == (N.BC_ERR_DEVICE, "Degree must be power of 2, got 6")
        assert _check_msg(fn, 4, 4, 2, 17, *extra) == (
            N.BC_ERR_DEVICE, "Degree must be in range [4, 65_536], got 2")
        assert _check_msg(fn, 2**18, 2**18, 2**17, 17, *extra) == (
            N.BC_ERR_DEVICE, "Degree must be in range [4, 65_536], got 131072")
        assert _check_msg(fn, 6, 8, 4, 17, *extra) == (
            N.BC_ERR_DEVICE, "Input A has wrong length: expected 8, got 6")
        assert _check_msg(fn, 8, 10, 4, 17, *extra) == (
            N.BC_ERR_DEVICE, "Input B has wrong length: expected 8, got 10")
        assert fn(8, 8, 4, 17, *extra) == 0


def test_rejection_fixtures(kats):
    """Every constructor rejection the reference's fault tests assert."""
    L = N.lib()
    for op, ln, d, q, root, expect_err in kats["rejections"]["values"]:
        r = compute_primitive_root(d, q) if root == "compute_primitive_root" else root
        st = L.bc_fhe_ntt_check(ln, d, q, r)
        assert (st != 0) == expect_err, (op, ln, d, q)


def test_rotate_switch_validation_messages():
    """FheRotate / FheModulusSwitch / FheKeySwitch ::new: degree, the op's own
    parameter, then the input length; all InvalidInput."""
    L, E = N.lib(), N.BC_ERR_INVALID_INPUT
    for d in (0, 2, 3, 6):
        msg = f"Degree must be power of 2 >= 4, got {d}"
        assert _check_msg(L.bc_fhe_rotate_check, 8, d, 1, 17) == (E, msg)
        assert _check_msg(L.bc_fhe_modulus_switch_check, 8, d, 17, 5) == (E, msg)
        assert _check_msg(L.bc_fhe_key_switch_check, 8, d, 17, 16, 3) == (E, msg)
    assert _check_msg(L.bc_fhe_rotate_check, 8, 4, 3, 17) == (
        E, "Rotation 3 out of range [-2, 2] for degree 4")
    assert _check_msg(L.bc_fhe_rotate_check, 16, 8, -5, 17) == (
        E, "Rotation -5 out of range [-4, 4] for degree 8")
    assert _check_msg(L.bc_fhe_rotate_check, 8, 4, -2**31, 17)[0] == E
    assert _check_msg(L.bc_fhe_rotate_check, 6, 4, 1, 17) == (
        E, "Input must have 8 elements (degree=4, u64 emulated), got 6")
    assert _check_msg(L.bc_fhe_modulus_switch_check, 8, 4, 12289, 12289) == (
        E, "New modulus (12289) must be < old modulus (12289)")
    assert _check_msg(L.bc_fhe_modulus_switch_check, 10, 4, 12289, 6145) == (
        E, "Input must have 8 elements (degree=4, u64 emulated), got 10")
    assert _check_msg(L.bc_fhe_key_switch_check, 8, 4, 17, 1, 3) == (
        E, "Decomposition base must be in [2, 2^24], got 1")
    assert _check_msg(L.bc_fhe_key_switch_check, 8, 4, 17, (1 << 24) + 1, 3) == (
        E, "Decomposition base must be in [2, 2^24], got 16777217")
    assert _check_msg(L.bc_fhe_key_switch_check, 8, 4, 17, 16, 33) == (
        E, "Decomposition levels must be in [1, 32], got 33")
    assert _check_msg(L.bc_fhe_key_switch_check, 4, 4, 17, 16, 3) == (
        E, "Input must have 8 elements (degree=4, u64 emulated), got 4")
    assert L.bc_fhe_rotate_check(8, 4, -2, 17) == 0
    assert L.bc_fhe_modulus_switch_check(8, 4, 1, 0) == 0   # q_new = 0 < q_old = 1 passes
    assert L.bc_fhe_key_switch_check(8, 4, 0, 1 << 24, 32) == 0


def test_op_rejection_fixtures(kats):
    """Every constructor rejection the ops' own unit tests assert."""
    L = N.lib()
    fns = {"rotate": L.bc_fhe_rotate_check, "modulus_switch": L.bc_fhe_modulus_switch_check,
           "key_switch": L.bc_fhe_key_switch_check}
    for op, args, expect_err in kats["op_rejections"]["values"]:
        assert (fns[op](*args) != 0) == expect_err, (op, args)


def test_rotation_galois_matches_oracle():
    L = N.lib()
    for d in (4, 8, 1024, 1 << 16):
        for r in sorted({-d // 2, -3 % (d // 2 + 1), -1, 0, 1, 2, d // 2}):
            assert L.bc_rotation_galois(d, r) == O.lib().orc_ref_rotate_galois(d, r)
        assert L.bc_rotation_galois(d, d // 2 + 1) == 0


class _Shape:
    """Stands in for a device tensor: only len() is consulted by new()."""

    def __init__(self, n):
        self.n = n
        self.device = None

    def len(self):
        return self.n


def test_python_mirror_raises_like_rust():
    with pytest.raises(bc.BarracudaError) as e:
        bc.FheNtt.new(_Shape(8), 4, 0, 4)
    assert str(e.value) == "Device error: Modulus must be non-zero"
    assert e.value.kind == "Device"
    with pytest.raises(bc.BarracudaError):
        bc.FheIntt.new(_Shape(6), 3, 17, 13)
    with pytest.raises(bc.BarracudaError):
        bc.FhePointwiseMul.new(_Shape(8), _Shape(8), 2, 17)
    with pytest.raises(bc.BarracudaError):
        bc.FheFastPolyMul.new(_Shape(8), _Shape(6), 4, 17, 4)
    with pytest.raises(bc.BarracudaError) as e:
        bc.FheRotate.new(_Shape(8), 4, 3, 12289)
    assert e.value.kind == "InvalidInput"
    assert str(e.value) == "Invalid input: Rotation 3 out of range [-2, 2] for degree 4"
    with pytest.raises(bc.BarracudaError):
        bc.FheModulusSwitch.new(_Shape(8), 4, 12289, 12289)
    with pytest.raises(bc.BarracudaError):
        bc.FheKeySwitch.new(_Shape(8), 4, 12289, 1 << 16, 0)


def test_roots_match_reference_restatement():
    L = O.lib()
    rng = np.random.default_rng(5)
    cases = [(4, 17), (8, 97), (8, 257), (16, 257), (8, 12289), (16, 12289), (32, 998244353),
             (4, 1), (0, 17), (4, 19), (1024, 12289), (4096, 2**31 - 1)]
    cases += [(int(1 << rng.integers(1, 12)), int(rng.integers(2, 2**40))) for _ in range(200)]
    for d, q in cases:
        assert bc.compute_primitive_root(d, q) == L.orc_ref_compute_primitive_root(d, q), (d, q)
    for a, m in [(3, 7), (4, 17), (0, 5), (6, 9), (5, 0), (1, 1), (2**61 - 1, 2**62 - 57)]:
        assert bc.compute_inverse_root(8, m, a) == L.orc_ref_compute_inverse_root(8, m, a)


def test_primes_and_negacyclic_roots():
    L = O.lib()
    for bits in (20, 31, 60):
        for logn in (4, 12, 16, 17):
            n = 1 << logn
            for i in range(3):
                q = bc.ntt_prime(bits, n, i)
                assert q == O.ntt_prime(bits, n, i)
                if q == 0:  # fewer than i+1 such primes below 2^bits
                    assert bc.negacyclic_root(q, n) == 0
                    continue
                assert bc.negacyclic_root(q, n) == O.psi(q, n)
                assert L.orc_powmod(bc.negacyclic_root(q, n), n, q) == q - 1


def test_partition_balanced_and_covering():
    for units in (0, 1, 7, 128, 1000, 12288):
        for shards in (1, 2, 3, 4, 8):
            pieces = [bc.partition(units, shards, s) for s in range(shards)]
            assert sum(c for _, c in pieces) == units
            assert max(c for _, c in pieces) - min(c for _, c in pieces) <= 1
            pos = 0
            for b, c in pieces:
                assert b == pos
                pos += c
    with pytest.raises(bc.BarracudaError):
        bc.partition(8, 2, 2)


def _twiddle(n, q, root, inv_root, mode, table, k):
    w, wq = ctypes.c_uint64(), ctypes.c_uint64()
    N.check(N.lib().bc_debug_twiddle(n, q, root, inv_root, mode, table, k, ctypes.byref(w),
                                     ctypes.byref(wq)))
    return w.value, wq.value


def _brev(x, bits):
    return int(format(x, f"0{bits}b")[::-1], 2) if bits else 0


@pytest.mark.parametrize("n", [2, 4, 16, 256])
def test_twiddle_tables_follow_definitions(n):
    """Entry m + i of the Cooley-Tukey table (m = 2^s butterfly groups):
    cyclic  w = omega^(bitrev_s(i) * N / 2m)   (the reference DIT twiddle
            omega^(l * N / 2^(s+1)) with l = bitrev_s(i), fhe_ntt.wgsl:238-241)
    negacyclic w = psi^(bitrev_logN(m + i)); inverse tables carry N^-1 in
    their last stage.  Shoup companions are floor(w * 2^W / q)."""
    L = n.bit_length() - 1
    for bits, W in ((31, 32), (60, 64)):
        q = O.ntt_prime(bits, n, 0)
        psi = O.psi(q, n)
        omega = psi * psi % q
        oinv = pow(omega, q - 2, q)
        ninv = pow(n, q - 2, q)
        for k in range(1, n):
            s = k.bit_length() - 1
            m, i = 1 << s, k - (1 << s)
            want = pow(omega, _brev(i, s) * n // (2 * m), q)
            assert _twiddle(n, q, omega, oinv, 0, 0, k) == (want, (want << W) // q)
            want_inv = pow(oinv, _brev(i, s) * n // (2 * m), q)
            if m == n // 2:
                want_inv = want_inv * ninv % q
            assert _twiddle(n, q, omega, oinv, 0, 1, k)[0] == want_inv
            want_neg = pow(psi, _brev(k, L), q)
            assert _twiddle(n, q, psi, 0, 1, 0, k)[0] == want_neg
            want_neg_inv = pow(psi, (q - 1 - _brev(k, L)) % (q - 1), q)
            if k == 1:
                want_neg_inv = want_neg_inv * ninv % q
            assert _twiddle(n, q, psi, 0, 1, 1, k)[0] == want_neg_inv


def test_plan_rejects_bad_parameters_without_gpu():
    w, wq = ctypes.c_uint64(), ctypes.c_uint64()
    L = N.lib()
    st = L.bc_debug_twiddle(16, 97, 8, 0, 1, 0, 1, ctypes.byref(w), ctypes.byref(wq))
    assert st == N.BC_ERR_INVALID_INPUT      # 8 is an N-th root, not a 2N-th root
    assert "primitive 2N-th root" in N.last_error()
    st = L.bc_debug_twiddle(16, 2**62 + 33, 3, 0, 0, 0, 1, ctypes.byref(w), ctypes.byref(wq))
    assert st == N.BC_ERR_UNSUPPORTED
    st = L.bc_debug_twiddle(12, 97, 3, 0, 0, 0, 1, ctypes.byref(w), ctypes.byref(wq))
    assert st == N.BC_ERR_INVALID_INPUT


def test_no_gpu_reports_device_not_available():
    """Without a GPU the context call fails with a status, never a crash."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    st = N.lib().bc_ctx_create(0, ctypes.byref(h))
    assert st in (N.BC_ERR_DEVICE_NOT_AVAILABLE, N.BC_ERR_GPU)
    assert N.last_error()
