"""ctypes wrapper of liboracle.so -- the CPU restatement of barraCuda's FHE NTT path.

TEST INFRASTRUCTURE ONLY.  Imported by tests/, by __graft_entry__.smoke() and by
bench.py's cpu_baseline / ``--impl reference`` legs, always as the checker or
the timed CPU baseline.  The product package (barracuda_b200) never imports it.

Function names mirror the reference: ``ref_ntt`` is FheNtt::execute
(crates/barracuda/src/ops/fhe_ntt/compute.rs:29-143), ``ref_intt`` is
FheIntt::execute (fhe_intt/compute.rs:27-168), ``ref_pointwise`` is
FhePointwiseMul::execute (fhe_pointwise_mul.rs:119-155), ``ref_fast_poly_mul`` is
FheFastPolyMul::execute (fhe_fast_poly_mul.rs:122-154).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "liboracle.so")
_lib = None

_u64p = ctypes.POINTER(ctypes.c_uint64)


def build() -> str:
    """Compile liboracle.so with the Makefile beside this file."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def _stale() -> bool:
    if not os.path.exists(_SO):
        return True
    t = os.path.getmtime(_SO)
    srcs = [os.path.join(_HERE, f) for f in ("ref_wgsl.c", "ref_poly.c", "ref_rns.c", "exact.c", "baseline.c", "oracle.h")]
    return any(os.path.exists(f) and os.path.getmtime(f) > t for f in srcs)


def lib():
    global _lib
    if _lib is None:
        if _stale():
            build()
        L = ctypes.CDLL(_SO)
        u32, u64, i32 = ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int
        sig = {
            "orc_wgsl_u64_mul": (u64, [u64, u64]),
            "orc_wgsl_u64_mod_simple": (u64, [u64, u64]),
            "orc_wgsl_mul32_wide": (u64, [u32, u32]),
            "orc_wgsl_pointwise_mod_mul": (u64, [u64, u64, u64, u64]),
            "orc_ref_twiddles": (None, [u32, u64, u64, _u64p]),
            "orc_ref_mod_pow": (u64, [u64, u64, u64]),
            "orc_ref_compute_primitive_root": (u64, [u32, u64]),
            "orc_ref_modinv": (u64, [u64, u64]),
            "orc_ref_compute_inverse_root": (u64, [u32, u64, u64]),
            "orc_ref_fastmul_modinv": (u64, [u64, u64]),
            "orc_ref_ntt": (None, [_u64p, _u64p, u32, u64, u64]),
            "orc_ref_intt": (None, [_u64p, _u64p, u32, u64, u64]),
            "orc_ref_pointwise": (None, [_u64p, _u64p, _u64p, u32, u64]),
            "orc_ref_fast_poly_mul": (None, [_u64p, _u64p, _u64p, u32, u64, u64]),
            "orc_ref_negacyclic_ntt": (None, [_u64p, _u64p, u32, u64, u64]),
            "orc_ref_negacyclic_intt": (None, [_u64p, _u64p, u32, u64, u64]),
            "orc_mulmod": (u64, [u64, u64, u64]),
            "orc_powmod": (u64, [u64, u64, u64]),
            "orc_is_prime": (i32, [u64]),
            "orc_ntt_prime": (u64, [u32, u32, u32]),
            "orc_smallest_generator": (u64, [u64]),
            "orc_psi": (u64, [u64, u32]),
            "orc_exact_dft": (None, [_u64p, _u64p, u32, u64, u64]),
            "orc_exact_ntt": (None, [_u64p, _u64p, u32, u64, u64]),
            "orc_exact_negacyclic_ntt": (None, [_u64p, _u64p, u32, u64, u64]),
            "orc_exact_negacyclic_intt": (None, [_u64p, _u64p, u32, u64, u64]),
            "orc_cyclic_convolution": (None, [_u64p, _u64p, _u64p, u32, u64]),
            "orc_negacyclic_convolution": (None, [_u64p, _u64p, _u64p, u32, u64]),
            "orc_seeded_value": (u64, [u64, u64, u64]),
            "orc_seeded_fill": (None, [_u64p, ctypes.c_size_t, u64, u64, u64]),
            "orc_digest": (u64, [_u64p, ctypes.c_size_t, u64]),
            "orc_ref_poly_add1": (u64, [u64, u64, u64]),
            "orc_ref_poly_sub1": (u64, [u64, u64, u64]),
            "orc_ref_poly_mul1": (u64, [u64, u64, u64]),
            "orc_ref_poly_add": (None, [_u64p, _u64p, _u64p, u32, u64]),
            "orc_ref_poly_sub": (None, [_u64p, _u64p, _u64p, u32, u64]),
            "orc_ref_poly_mul": (None, [_u64p, _u64p, _u64p, u32, u64]),
            "orc_exact_poly_mul": (None, [_u64p, _u64p, _u64p, u32, u64]),
            "orc_ref_rotate_galois": (u32, [u32, ctypes.c_int32]),
            "orc_ref_rotate": (None, [_u64p, _u64p, u32, ctypes.c_int32, u64]),
            "orc_automorphism": (None, [_u64p, _u64p, u32, u32, u64]),
            "orc_ref_modulus_switch1": (u64, [u64, u64, u64]),
            "orc_exact_modulus_switch1": (u64, [u64, u64, u64]),
            "orc_ref_modulus_switch": (None, [_u64p, _u64p, u32, u64, u64]),
            "orc_exact_modulus_switch": (None, [_u64p, _u64p, ctypes.c_size_t, u64, u64]),
            "orc_ref_key_switch": (None, [_u64p, _u64p, u32, u32, u32]),
            "orc_decompose": (None, [_u64p, _u64p, ctypes.c_size_t, u32, u32]),
            "orc_baseline_run": (ctypes.c_double,
                                 [i32, _u64p, _u64p, u32, u32, _u64p, _u64p, u32, i32]),
            "orc_batch_polymul": (ctypes.c_double,
                                  [i32, _u64p, _u64p, _u64p, u32, u32, _u64p, _u64p, u32, i32]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def _arr(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.uint64))


def _p(a: np.ndarray):
    return a.ctypes.data_as(_u64p)


def _unary(fname, x, n, q, r):
    x = _arr(x)
    assert x.size == n
    out = np.zeros(n, dtype=np.uint64)
    getattr(lib(), fname)(_p(x), _p(out), n, q, r)
    return out


def ref_ntt(x, degree, modulus, root):
    return _unary("orc_ref_ntt", x, degree, modulus, root)


def ref_intt(x, degree, modulus, inv_root):
    return _unary("orc_ref_intt", x, degree, modulus, inv_root)


def ref_negacyclic_ntt(x, degree, modulus, psi):
    return _unary("orc_ref_negacyclic_ntt", x, degree, modulus, psi)


def ref_negacyclic_intt(x, degree, modulus, psi):
    return _unary("orc_ref_negacyclic_intt", x, degree, modulus, psi)


def exact_dft(x, n, q, w):
    return _unary("orc_exact_dft", x, n, q, w)


def exact_ntt(x, n, q, w):
    return _unary("orc_exact_ntt", x, n, q, w)


def exact_negacyclic_ntt(x, n, q, psi):
    return _unary("orc_exact_negacyclic_ntt", x, n, q, psi)


def exact_negacyclic_intt(x, n, q, psi):
    return _unary("orc_exact_negacyclic_intt", x, n, q, psi)


def ref_pointwise(a, b, degree, modulus):
    a, b = _arr(a), _arr(b)
    out = np.zeros(degree, dtype=np.uint64)
    lib().orc_ref_pointwise(_p(a), _p(b), _p(out), degree, modulus)
    return out


def ref_fast_poly_mul(a, b, degree, modulus, root):
    a, b = _arr(a), _arr(b)
    out = np.zeros(degree, dtype=np.uint64)
    lib().orc_ref_fast_poly_mul(_p(a), _p(b), _p(out), degree, modulus, root)
    return out


def cyclic_convolution(a, b, n, q):
    a, b = _arr(a), _arr(b)
    out = np.zeros(n, dtype=np.uint64)
    lib().orc_cyclic_convolution(_p(a), _p(b), _p(out), n, q)
    return out


def negacyclic_convolution(a, b, n, q):
    a, b = _arr(a), _arr(b)
    out = np.zeros(n, dtype=np.uint64)
    lib().orc_negacyclic_convolution(_p(a), _p(b), _p(out), n, q)
    return out


def ref_twiddles(degree, modulus, root):
    out = np.zeros(degree, dtype=np.uint64)
    lib().orc_ref_twiddles(degree, modulus, root, _p(out))
    return out


def seeded_fill(count, seed, g0, q):
    out = np.zeros(count, dtype=np.uint64)
    lib().orc_seeded_fill(_p(out), count, seed, g0, q)
    return out


def _binary(fname, a, b, q):
    a, b = _arr(a), _arr(b)
    assert a.size == b.size
    out = np.zeros(a.size, dtype=np.uint64)
    getattr(lib(), fname)(_p(a), _p(b), _p(out), a.size, q)
    return out


def ref_poly_add(a, b, q):
    """FhePolyAdd::execute (ops/fhe_poly_add.rs:128-175, fhe_poly_add.wgsl)."""
    return _binary("orc_ref_poly_add", a, b, q)


def ref_poly_sub(a, b, q):
    """FhePolySub::execute (ops/fhe_poly_sub.rs, fhe_poly_sub.wgsl)."""
    return _binary("orc_ref_poly_sub", a, b, q)


def ref_poly_mul(a, b, q):
    """FhePolyMul::execute (ops/fhe_poly_mul.rs:82-133, fhe_poly_mul.wgsl)."""
    return _binary("orc_ref_poly_mul", a, b, q)


def exact_poly_mul(a, b, q):
    return _binary("orc_exact_poly_mul", a, b, q)


def ref_rotate(x, degree, rotation, modulus):
    """FheRotate::execute (ops/fhe_rotate.rs:140-183, fhe_rotate.wgsl)."""
    x = _arr(x)
    out = np.zeros(degree, dtype=np.uint64)
    lib().orc_ref_rotate(_p(x), _p(out), degree, rotation, modulus)
    return out


def automorphism(x, degree, galois, modulus):
    x = _arr(x)
    out = np.zeros(degree, dtype=np.uint64)
    lib().orc_automorphism(_p(x), _p(out), degree, galois, modulus)
    return out


def ref_modulus_switch(x, q_old, q_new):
    """FheModulusSwitch::execute (ops/fhe_modulus_switch.rs:124-166, .wgsl)."""
    x = _arr(x)
    out = np.zeros(x.size, dtype=np.uint64)
    lib().orc_ref_modulus_switch(_p(x), _p(out), x.size, q_old, q_new)
    return out


def exact_modulus_switch(x, q_old, q_new):
    x = _arr(x)
    out = np.zeros(x.size, dtype=np.uint64)
    lib().orc_exact_modulus_switch(_p(x), _p(out), x.size, q_old, q_new)
    return out


def ref_key_switch(x, decomp_base, decomp_levels):
    """FheKeySwitch::execute (ops/fhe_key_switch.rs:162-222, .wgsl)."""
    x = _arr(x)
    out = np.zeros(x.size, dtype=np.uint64)
    lib().orc_ref_key_switch(_p(x), _p(out), x.size, decomp_base, decomp_levels)
    return out


def decompose(x, base, levels):
    """Every base-B digit of every coefficient, digit-major (levels, len(x))."""
    x = _arr(x)
    out = np.zeros(x.size * levels, dtype=np.uint64)
    lib().orc_decompose(_p(x), _p(out), x.size, base, levels)
    return out.reshape(levels, x.size)


def digest(x, first_index=0):
    x = _arr(x)
    return int(lib().orc_digest(_p(x), x.size, first_index))


def ntt_prime(bits, degree, index):
    return int(lib().orc_ntt_prime(bits, degree, index))


def psi(q, degree):
    return int(lib().orc_psi(q, degree))


def __getattr__(name):
    # plain scalar entry points: oracle.orc_powmod(...) etc.
    if name.startswith("orc_"):
        return getattr(lib(), name)
    raise AttributeError(name)


BASELINE_KIND = {"ntt": 0, "intt": 1, "negacyclic_ntt": 2, "negacyclic_intt": 3,
                 "exact_negacyclic_ntt": 4, "exact_negacyclic_intt": 5}
POLYMUL_KIND = {"ref_cyclic": 0, "ref_negacyclic": 1, "exact_negacyclic": 2, "exact_cyclic": 3}


def baseline_run(kind, x, degree, moduli, roots, threads):
    """Time the reference restatement on len(x)/degree polynomials; returns (seconds, out)."""
    x = _arr(x)
    count = x.size // degree
    out = np.zeros_like(x)
    m, r = _arr(moduli), _arr(roots)
    secs = lib().orc_baseline_run(BASELINE_KIND[kind], _p(x), _p(out), degree, count,
                                  _p(m), _p(r), m.size, threads)
    return secs, out


def _threads(threads):
    return threads if threads else (os.cpu_count() or 1)


def batch_transform(kind, x, degree, moduli, roots, threads=None):
    """`kind` (a BASELINE_KIND name) of each limb-polynomial of x (back to back);
    polynomial p uses moduli[p] and roots[p].  Multi-threaded."""
    return baseline_run(kind, x, degree, moduli, roots, _threads(threads))[1]


def batch_polymul(kind, a, b, degree, moduli, roots, threads=None):
    """Products of the limb-polynomial pairs of a and b (back to back); pair p
    uses moduli[p] and roots[p]; `kind` is a POLYMUL_KIND name.  Multi-threaded."""
    a, b = _arr(a), _arr(b)
    c = np.zeros_like(a)
    m, r = _arr(moduli), _arr(roots)
    lib().orc_batch_polymul(POLYMUL_KIND[kind], _p(a), _p(b), _p(c), degree, a.size // degree,
                            _p(m), _p(r), m.size, _threads(threads))
    return c
