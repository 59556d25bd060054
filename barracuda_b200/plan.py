"""Batched NTT plans over RNS limbs (the new batched path behind the C ABI).

A plan covers ``n_limbs`` moduli of one degree N.  Buffers are device pointers
(ints) or CUDA tensors whose ``data_ptr()`` holds u64 coefficients (torch
``int64`` or ``uint64`` storage); element (limb l, polynomial p, coefficient j)
is at ``l * limb_stride + p * poly_stride + j``.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

from . import _native as N
from ._native import check, lib
from .ops import Device

CYCLIC = N.BC_NTT_CYCLIC
NEGACYCLIC = N.BC_NTT_NEGACYCLIC


def _ptr(x) -> int:
    if x is None:
        return 0
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return int(x.data_ptr())
    if hasattr(x, "ptr"):
        return int(x.ptr)
    raise TypeError(f"cannot take a device pointer of {type(x)!r}")


def _u64_array(vals) -> ctypes.Array:
    arr = (ctypes.c_uint64 * len(vals))()
    for i, v in enumerate(vals):
        arr[i] = int(v)
    return arr


def ntt_prime(bits: int, degree: int, index: int = 0) -> int:
    """index-th largest prime q < 2^bits with q == 1 (mod 2N)."""
    return int(lib().bc_ntt_prime(bits, degree, index))


def ntt_primes(bits: int, degree: int, count: int) -> list:
    return [ntt_prime(bits, degree, i) for i in range(count)]


def negacyclic_root(modulus: int, degree: int) -> int:
    """psi = g^((q-1)/2N) with g the smallest generator of Z_q^*."""
    return int(lib().bc_negacyclic_root(modulus, degree))


def partition(units: int, shards: int, shard: int):
    """Balanced contiguous split: (begin, count) of shard `shard`."""
    b, c = ctypes.c_uint64(), ctypes.c_uint64()
    check(lib().bc_partition(units, shards, shard, ctypes.byref(b), ctypes.byref(c)))
    return int(b.value), int(c.value)


@dataclass
class Layout:
    limb_stride: int
    poly_stride: int

    def c(self) -> N.bc_layout:
        return N.bc_layout(self.limb_stride, self.poly_stride)


class NttPlan:
    """Twiddle tables and kernel choice for n_limbs moduli of degree N on one device."""

    def __init__(self, device: Device, degree: int, moduli: Sequence[int], roots: Sequence[int],
                 mode: int = NEGACYCLIC, inv_roots: Optional[Sequence[int]] = None):
        self.device = device
        self.degree = int(degree)
        self.moduli = [int(q) for q in moduli]
        self.n_limbs = len(self.moduli)
        h = ctypes.c_void_p()
        inv = _u64_array(inv_roots) if inv_roots is not None else None
        check(lib().bc_plan_create(device.handle, self.degree, self.n_limbs,
                                   _u64_array(self.moduli), _u64_array(roots), inv, mode,
                                   ctypes.byref(h)))
        self.handle = h
        self.mode = mode
        info = N.bc_plan_info()
        check(lib().bc_plan_info_get(h, ctypes.byref(info)))
        self.info = {f: getattr(info, f) for f, _ in N.bc_plan_info._fields_}

    def _layout(self, layout: Optional[Layout]):
        return ctypes.byref(layout.c()) if layout is not None else None

    def forward(self, src, dst, batch: int, layout: Optional[Layout] = None, stream: int = 0):
        check(lib().bc_ntt_forward(self.handle, _ptr(src), _ptr(dst), batch, self._layout(layout),
                                   stream or None))

    def inverse(self, src, dst, batch: int, layout: Optional[Layout] = None, stream: int = 0):
        check(lib().bc_ntt_inverse(self.handle, _ptr(src), _ptr(dst), batch, self._layout(layout),
                                   stream or None))

    def pointwise_mul(self, a, b, c, batch: int, layout: Optional[Layout] = None, stream: int = 0):
        check(lib().bc_pointwise_mul(self.handle, _ptr(a), _ptr(b), _ptr(c), batch,
                                     self._layout(layout), stream or None))

    def forward_mul(self, a, b_hat, c, batch: int, layout: Optional[Layout] = None, stream: int = 0):
        """C = NTT(A) * B^ (one fused launch on negacyclic plans)."""
        check(lib().bc_ntt_forward_mul(self.handle, _ptr(a), _ptr(b_hat), _ptr(c), batch,
                                       self._layout(layout), stream or None))

    def inverse_mul(self, a_hat, b_hat, c, batch: int, layout: Optional[Layout] = None, stream: int = 0):
        """C = INTT(A^ * B^) (one fused launch on negacyclic plans)."""
        check(lib().bc_ntt_inverse_mul(self.handle, _ptr(a_hat), _ptr(b_hat), _ptr(c), batch,
                                       self._layout(layout), stream or None))

    def forward_add(self, a, b_hat, c, batch: int, layout: Optional[Layout] = None, stream: int = 0):
        """C = NTT(A) + B^ mod q (one fused launch on negacyclic plans)."""
        check(lib().bc_ntt_forward_add(self.handle, _ptr(a), _ptr(b_hat), _ptr(c), batch,
                                       self._layout(layout), stream or None))

    def forward_sub(self, a, b_hat, c, batch: int, layout: Optional[Layout] = None, stream: int = 0):
        """C = NTT(A) - B^ mod q (one fused launch on negacyclic plans)."""
        check(lib().bc_ntt_forward_sub(self.handle, _ptr(a), _ptr(b_hat), _ptr(c), batch,
                                       self._layout(layout), stream or None))

    def inverse_add(self, a_hat, b_hat, c, batch: int, layout: Optional[Layout] = None, stream: int = 0):
        """C = INTT(A^ + B^ mod q) (one fused launch on negacyclic plans)."""
        check(lib().bc_ntt_inverse_add(self.handle, _ptr(a_hat), _ptr(b_hat), _ptr(c), batch,
                                       self._layout(layout), stream or None))

    def inverse_sub(self, a_hat, b_hat, c, batch: int, layout: Optional[Layout] = None, stream: int = 0):
        """C = INTT(A^ - B^ mod q) (one fused launch on negacyclic plans)."""
        check(lib().bc_ntt_inverse_sub(self.handle, _ptr(a_hat), _ptr(b_hat), _ptr(c), batch,
                                       self._layout(layout), stream or None))

    def poly_add(self, a, b, c, batch: int, layout: Optional[Layout] = None, stream: int = 0):
        check(lib().bc_poly_add(self.handle, _ptr(a), _ptr(b), _ptr(c), batch, self._layout(layout),
                                stream or None))

    def poly_sub(self, a, b, c, batch: int, layout: Optional[Layout] = None, stream: int = 0):
        check(lib().bc_poly_sub(self.handle, _ptr(a), _ptr(b), _ptr(c), batch, self._layout(layout),
                                stream or None))

    def poly_mul(self, a, b, c, batch: int, layout: Optional[Layout] = None, stream: int = 0):
        check(lib().bc_poly_mul(self.handle, _ptr(a), _ptr(b), _ptr(c), batch, self._layout(layout),
                                stream or None))

    def polymul(self, a, b, c, batch: int, layout: Optional[Layout] = None, stream: int = 0):
        check(lib().bc_polymul(self.handle, _ptr(a), _ptr(b), _ptr(c), batch, self._layout(layout),
                               stream or None))

    def automorphism(self, src, dst, batch: int, galois: int, layout: Optional[Layout] = None,
                     stream: int = 0):
        """X -> X^galois on every polynomial (galois odd, < 2N); src and dst must not overlap."""
        check(lib().bc_automorphism(self.handle, _ptr(src), _ptr(dst), batch, self._layout(layout),
                                    galois, stream or None))

    def fill_uniform(self, dst, batch: int, seed: int, first_poly: int = 0,
                     total_polys: Optional[int] = None, layout: Optional[Layout] = None,
                     stream: int = 0):
        total = batch if total_polys is None else total_polys
        check(lib().bc_fill_uniform(self.handle, _ptr(dst), batch, self._layout(layout), seed,
                                    first_poly, total, stream or None))

    def close(self):
        if self.handle:
            lib().bc_plan_destroy(self.handle)
            self.handle = None

    def __del__(self):  # pragma: no cover
        try:
            if self.device.handle:
                self.close()
        except Exception:
            pass


def modulus_switch(device: Device, src, dst, count: int, modulus_old: int, modulus_new: int,
                   stream: int = 0):
    """round(c * new / old) mod new over count words (in place allowed)."""
    check(lib().bc_modulus_switch(device.handle, _ptr(src), _ptr(dst), count, modulus_old,
                                  modulus_new, stream or None))


def decompose(device: Device, src, dst, count: int, base: int, levels: int, stream: int = 0):
    """dst[l * count + i] = digit l (base `base`) of src[i], l < levels."""
    check(lib().bc_decompose(device.handle, _ptr(src), _ptr(dst), count, base, levels,
                             stream or None))


def calibrate_butterflies(device: Device, word_bits: int = 32) -> float:
    """Register-only modular butterflies per second on this GPU (roofline's integer term)."""
    out = ctypes.c_double()
    check(lib().bc_calibrate_butterflies(device.handle, word_bits, ctypes.byref(out)))
    return out.value


def digest(device: Device, buf, count: int, out, stream: int = 0, first_index: int = 0):
    check(lib().bc_digest(device.handle, _ptr(buf), count, first_index, _ptr(out), stream or None))
