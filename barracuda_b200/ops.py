"""Python mirror of barraCuda's FHE op API (crates/barracuda/src/ops/fhe_*.rs).

Same names, constructor arguments, validation (order and message text) and
execute semantics as the Rust ops; everything runs through the C ABI of
libbarracuda_fhe.so, so these classes are what a parity test written like the
reference's own tests calls::

    dev = Device(0)
    t = create_fhe_poly_tensor([1, 2, 3, 4], dev)
    out = FheNtt.new(t, 4, 17, 4).execute()      # tests/fhe/ntt.rs style
    assert read_poly_from_tensor(out) == [10, 7, 15, 6]

``FheNtt.new`` raises BarracudaError exactly where ``FheNtt::new`` returns Err.
"""
from __future__ import annotations

import ctypes
import math
from typing import Iterable, Sequence

import numpy as np

from . import _native as N
from ._native import BarracudaError, check, lib

__all__ = [
    "BarracudaError", "Device", "FheTensor", "create_fhe_poly_tensor", "read_poly_from_tensor",
    "compute_primitive_root", "compute_inverse_root", "FheNtt", "FheIntt", "FhePointwiseMul",
    "FheFastPolyMul", "FheRotate", "FheModulusSwitch", "FheKeySwitch", "rotation_galois",
]


class Device:
    """One GPU (the role WgpuDevice plays for this path): a bc_ctx and its stream."""

    def __init__(self, ordinal: int = 0):
        h = ctypes.c_void_p()
        check(lib().bc_ctx_create(ordinal, ctypes.byref(h)))
        self.handle = h
        self.ordinal = ordinal

    def stream(self) -> int:
        s = ctypes.c_void_p()
        check(lib().bc_ctx_stream(self.handle, ctypes.byref(s)))
        return s.value or 0

    def synchronize(self) -> None:
        check(lib().bc_ctx_sync(self.handle))

    def close(self) -> None:
        if self.handle:
            lib().bc_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass


class FheTensor:
    """Device buffer of u32 words: ``len()`` counts u32 words like Tensor::len()."""

    def __init__(self, device: Device, n_u32: int):
        self.device = device
        self._len = int(n_u32)
        p = ctypes.c_void_p()
        check(lib().bc_buf_alloc(device.handle, max(8, (self._len + 1) // 2 * 8), ctypes.byref(p)))
        self.ptr = p.value

    def len(self) -> int:
        return self._len

    def __len__(self) -> int:
        return self._len

    @classmethod
    def from_u32(cls, words: np.ndarray, device: Device) -> "FheTensor":
        words = np.ascontiguousarray(np.asarray(words, dtype=np.uint32))
        t = cls(device, words.size)
        if words.size:
            check(lib().bc_buf_h2d(device.handle, t.ptr, words.ctypes.data, words.nbytes))
        return t

    def to_vec_u32(self) -> np.ndarray:
        out = np.zeros(self._len, dtype=np.uint32)
        if self._len:
            check(lib().bc_buf_d2h(self.device.handle, out.ctypes.data, self.ptr, out.nbytes))
        return out

    def to_u64(self) -> np.ndarray:
        return self.to_vec_u32().view(np.uint64) if self._len % 2 == 0 else \
            np.frombuffer(np.append(self.to_vec_u32(), np.uint32(0)).tobytes(), dtype=np.uint64)

    def free(self) -> None:
        if self.ptr:
            lib().bc_buf_free(self.device.handle, self.ptr)
            self.ptr = None

    def __del__(self):  # pragma: no cover
        try:
            if self.device.handle:
                self.free()
        except Exception:
            pass


def create_fhe_poly_tensor(poly: Iterable[int], device: Device) -> FheTensor:
    """ops/fhe_poly_add.rs:185: u64 coefficients -> [lo32, hi32] u32 words."""
    arr = np.ascontiguousarray(np.asarray(list(poly) if not isinstance(poly, np.ndarray) else poly,
                                          dtype=np.uint64))
    return FheTensor.from_u32(arr.view(np.uint32), device)


def read_poly_from_tensor(t: FheTensor) -> list:
    """tests/fhe/helpers.rs:110-127: u32 pairs -> u64 coefficients."""
    return [int(v) for v in t.to_u64()]


def compute_primitive_root(degree: int, modulus: int) -> int:
    """ops/fhe_ntt/mod.rs:210-242."""
    return int(lib().bc_compute_primitive_root(degree, modulus))


def compute_inverse_root(degree: int, modulus: int, root: int) -> int:
    """ops/fhe_intt/mod.rs:202-204."""
    return int(lib().bc_compute_inverse_root(degree, modulus, root))


class FheNtt:
    """ops/fhe_ntt/mod.rs:71-171; execute() is compute.rs:29-143 (consumes the op)."""

    def __init__(self, input: FheTensor, degree: int, modulus: int, root_of_unity: int):
        check(lib().bc_fhe_ntt_check(input.len(), degree, modulus, root_of_unity))
        self.input, self.degree, self.modulus, self.root_of_unity = input, degree, modulus, root_of_unity

    @classmethod
    def new(cls, input, degree, modulus, root_of_unity) -> "FheNtt":
        return cls(input, degree, modulus, root_of_unity)

    def execute(self) -> FheTensor:
        out = FheTensor(self.input.device, 2 * self.degree)
        check(lib().bc_fhe_ntt(self.input.device.handle, self.input.ptr, self.input.len(),
                               self.degree, self.modulus, self.root_of_unity, out.ptr))
        return out


class FheIntt:
    """ops/fhe_intt/mod.rs:58-160; execute() is compute.rs:27-168."""

    def __init__(self, input: FheTensor, degree: int, modulus: int, inv_root_of_unity: int):
        check(lib().bc_fhe_intt_check(input.len(), degree, modulus, inv_root_of_unity))
        self.input, self.degree, self.modulus = input, degree, modulus
        self.inv_root_of_unity = inv_root_of_unity

    @classmethod
    def new(cls, input, degree, modulus, inv_root_of_unity) -> "FheIntt":
        return cls(input, degree, modulus, inv_root_of_unity)

    def execute(self) -> FheTensor:
        out = FheTensor(self.input.device, 2 * self.degree)
        check(lib().bc_fhe_intt(self.input.device.handle, self.input.ptr, self.input.len(),
                                self.degree, self.modulus, self.inv_root_of_unity, out.ptr))
        return out


class FhePointwiseMul:
    """ops/fhe_pointwise_mul.rs:34-156."""

    def __init__(self, input_a: FheTensor, input_b: FheTensor, degree: int, modulus: int):
        check(lib().bc_fhe_pointwise_mul_check(input_a.len(), input_b.len(), degree, modulus))
        if input_a.device is not input_b.device:
            raise BarracudaError(N.BC_ERR_DEVICE, "input_a and input_b must be on the same device")
        self.input_a, self.input_b, self.degree, self.modulus = input_a, input_b, degree, modulus

    @classmethod
    def new(cls, input_a, input_b, degree, modulus) -> "FhePointwiseMul":
        return cls(input_a, input_b, degree, modulus)

    def execute(self) -> FheTensor:
        out = FheTensor(self.input_a.device, 2 * self.degree)
        check(lib().bc_fhe_pointwise_mul(self.input_a.device.handle, self.input_a.ptr,
                                         self.input_a.len(), self.input_b.ptr, self.input_b.len(),
                                         self.degree, self.modulus, out.ptr))
        return out


class _FheCoeffOp:
    """Coefficient-wise op of the reference's FHE API; subclasses name the C entry point."""
    _name = ""

    def __init__(self, poly_a: FheTensor, poly_b: FheTensor, degree: int, modulus: int):
        L = lib()
        # same order as the Rust constructors: lengths, same device, modulus
        st = getattr(L, f"bc_fhe_poly_{self._name}_check")(poly_a.len(), poly_b.len(), degree, 1)
        check(st)
        if poly_a.device is not poly_b.device:
            raise BarracudaError(N.BC_ERR_DEVICE, "poly_a and poly_b must be on the same device")
        check(getattr(L, f"bc_fhe_poly_{self._name}_check")(poly_a.len(), poly_b.len(), degree, modulus))
        self.poly_a, self.poly_b, self.degree, self.modulus = poly_a, poly_b, degree, modulus

    @classmethod
    def new(cls, poly_a, poly_b, degree, modulus):
        return cls(poly_a, poly_b, degree, modulus)

    def execute(self) -> FheTensor:
        out = FheTensor(self.poly_a.device, 2 * self.degree)
        check(getattr(lib(), f"bc_fhe_poly_{self._name}")(
            self.poly_a.device.handle, self.poly_a.ptr, self.poly_a.len(), self.poly_b.ptr,
            self.poly_b.len(), self.degree, self.modulus, out.ptr))
        return out


class FhePolyAdd(_FheCoeffOp):
    """ops/fhe_poly_add.rs:47-175: (a + b) mod q per coefficient."""
    _name = "add"


class FhePolySub(_FheCoeffOp):
    """ops/fhe_poly_sub.rs: (a - b) mod q per coefficient."""
    _name = "sub"


class FhePolyMul(_FheCoeffOp):
    """ops/fhe_poly_mul.rs:34-133: (a * b) mod q per coefficient, exact."""
    _name = "mul"


class FheRotate:
    """ops/fhe_rotate.rs:64-183: Galois automorphism X -> X^(2r+1) (negative r
    counts from degree); coefficients that wrap past X^N are negated as
    modulus - c (0 stays 0)."""

    def __init__(self, input: FheTensor, degree: int, rotation: int, modulus: int):
        if not -2**31 <= rotation < 2**31:
            raise OverflowError(f"rotation {rotation} does not fit an i32")
        check(lib().bc_fhe_rotate_check(input.len(), degree, rotation, modulus))
        self.input, self.degree, self.rotation, self.modulus = input, degree, rotation, modulus

    @classmethod
    def new(cls, input, degree, rotation, modulus) -> "FheRotate":
        return cls(input, degree, rotation, modulus)

    def execute(self) -> FheTensor:
        out = FheTensor(self.input.device, 2 * self.degree)
        check(lib().bc_fhe_rotate(self.input.device.handle, self.input.ptr, self.input.len(),
                                  self.degree, self.rotation, self.modulus, out.ptr))
        return out


def rotation_galois(degree: int, rotation: int) -> int:
    """Galois element 2r + 1 that FheRotate applies (0 when out of range)."""
    return int(lib().bc_rotation_galois(degree, rotation))


class FheModulusSwitch:
    """ops/fhe_modulus_switch.rs:60-167: round(c * new / old) mod new, with the
    product kept exact (the reference's shader wraps it at 2^64)."""

    def __init__(self, input: FheTensor, degree: int, modulus_old: int, modulus_new: int):
        check(lib().bc_fhe_modulus_switch_check(input.len(), degree, modulus_old, modulus_new))
        self.input, self.degree = input, degree
        self.modulus_old, self.modulus_new = modulus_old, modulus_new

    @classmethod
    def new(cls, input, degree, modulus_old, modulus_new) -> "FheModulusSwitch":
        return cls(input, degree, modulus_old, modulus_new)

    def execute(self) -> FheTensor:
        out = FheTensor(self.input.device, 2 * self.degree)
        check(lib().bc_fhe_modulus_switch(self.input.device.handle, self.input.ptr, self.input.len(),
                                          self.degree, self.modulus_old, self.modulus_new, out.ptr))
        return out


class FheKeySwitch:
    """ops/fhe_key_switch.rs:70-223: validates the decomposition parameters;
    execute() returns a copy of the input, as the reference's two passes do
    (the second stores the input over the first's digits)."""

    def __init__(self, input: FheTensor, degree: int, modulus: int, decomp_base: int,
                 decomp_levels: int):
        check(lib().bc_fhe_key_switch_check(input.len(), degree, modulus, decomp_base, decomp_levels))
        self.input, self.degree, self.modulus = input, degree, modulus
        self.decomp_base, self.decomp_levels = decomp_base, decomp_levels

    @classmethod
    def new(cls, input, degree, modulus, decomp_base, decomp_levels) -> "FheKeySwitch":
        return cls(input, degree, modulus, decomp_base, decomp_levels)

    def execute(self) -> FheTensor:
        out = FheTensor(self.input.device, 2 * self.degree)
        check(lib().bc_fhe_key_switch(self.input.device.handle, self.input.ptr, self.input.len(),
                                      self.degree, self.modulus, self.decomp_base,
                                      self.decomp_levels, out.ptr))
        return out


class FheFastPolyMul:
    """ops/fhe_fast_poly_mul.rs:39-171; execute() runs one fused kernel."""

    def __init__(self, input_a: FheTensor, input_b: FheTensor, degree: int, modulus: int,
                 root_of_unity: int):
        check(lib().bc_fhe_fast_poly_mul_check(input_a.len(), input_b.len(), degree, modulus,
                                               root_of_unity))
        self.input_a, self.input_b, self.degree = input_a, input_b, degree
        self.modulus, self.root_of_unity = modulus, root_of_unity

    @classmethod
    def new(cls, input_a, input_b, degree, modulus, root_of_unity) -> "FheFastPolyMul":
        return cls(input_a, input_b, degree, modulus, root_of_unity)

    def execute(self) -> FheTensor:
        out = FheTensor(self.input_a.device, 2 * self.degree)
        check(lib().bc_fhe_fast_poly_mul(self.input_a.device.handle, self.input_a.ptr,
                                         self.input_a.len(), self.input_b.ptr, self.input_b.len(),
                                         self.degree, self.modulus, self.root_of_unity, out.ptr))
        return out

    def expected_speedup(self) -> float:
        """fhe_fast_poly_mul.rs:160-170."""
        n = float(self.degree)
        return n / math.log2(n) * 0.164
