"""barracuda_b200 -- B200-native (sm_100a) FHE NTT path of ecoPrimals/barraCuda.

The product is libbarracuda_fhe.so (C ABI: include/barracuda_fhe.h).  This
package builds it in-tree (``barracuda_b200.build``), binds it with ctypes
(``_native``) and mirrors the reference op API (``ops``) and the batched plan
API (``plan``) on top of it, and splits a job over GPUs (``shard``).  There is
no CPU fallback: without the library every call raises.
"""
from ._native import BarracudaError, NativeLibraryMissing, LIB_PATH  # noqa: F401
from .ops import (  # noqa: F401
    Device, FheTensor, create_fhe_poly_tensor, read_poly_from_tensor, compute_primitive_root,
    compute_inverse_root, FheNtt, FheIntt, FhePointwiseMul, FheFastPolyMul, FhePolyAdd, FhePolySub,
    FhePolyMul, FheRotate, FheModulusSwitch, FheKeySwitch, rotation_galois,
)
from .plan import (  # noqa: F401
    NttPlan, Layout, CYCLIC, NEGACYCLIC, ntt_prime, ntt_primes, negacyclic_root, partition, digest,
    modulus_switch, decompose, calibrate_butterflies,
)
from .shard import Shard, ShardGroup, ShardFailure, job_digest  # noqa: F401
