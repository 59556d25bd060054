"""Writes tests/golden/reference_kats.json: the known-answer tests and fixed
vectors that ecoPrimals/barraCuda's own tests hold for the FHE NTT path.

The reference is Rust + WGSL and cannot be built or run in this environment,
so its vectors are transcribed here from the test sources (cited per case,
paths inside the reference repository).  Where the reference states an
expected output, it is recorded under "expect"; where it only asserts a
property (round trip, linearity, range), the case records the inputs and the
property name, and the tests check the property.

    python tests/golden/make_golden.py   # rewrites reference_kats.json
"""
import json
import os

HERE = os.path.dirname(os.path.abspath(__file__))

CASES = [
    {"name": "twiddles_4_17_4", "kind": "twiddles", "degree": 4, "modulus": 17, "root": 4,
     "expect": [1, 4, 16, 13],
     "source": "crates/barracuda/src/ops/fhe_ntt/tests.rs:7-17"},
    {"name": "modinv_3_7", "kind": "modinv", "a": 3, "m": 7, "expect": 5,
     "source": "crates/barracuda/src/ops/fhe_intt/tests.rs:7-9"},
    {"name": "modinv_4_17", "kind": "modinv", "a": 4, "m": 17, "expect": 13,
     "source": "crates/barracuda/src/ops/fhe_intt/tests.rs:11-12"},
    {"name": "inverse_root_4_17_4", "kind": "inverse_root", "degree": 4, "modulus": 17, "root": 4,
     "expect": 13, "source": "crates/barracuda/src/ops/fhe_intt/tests.rs:15-19"},
    {"name": "ntt_1234_q17", "kind": "ntt", "degree": 4, "modulus": 17, "root": 4,
     "input": [1, 2, 3, 4], "expect": [10, 7, 15, 6],
     "source": "crates/barracuda/examples/fhe_ntt_validation.rs:84-120 (printed expected value)"},
    {"name": "roundtrip_canary_4_17_4", "kind": "roundtrip", "degree": 4, "modulus": 17, "root": 4,
     "input": [1, 2, 3, 4], "source": "crates/barracuda/src/bin/validate_gpu.rs:55,276"},
    {"name": "roundtrip_canary_8_12289_11", "kind": "roundtrip", "degree": 8, "modulus": 12289,
     "root": 11, "input": [1, 2, 3, 4, 5, 6, 7, 8],
     "source": "crates/barracuda/src/bin/validate_gpu.rs:55,277 (11 is not a primitive 8th root)"},
    {"name": "roundtrip_prop_4_17", "kind": "roundtrip", "degree": 4, "modulus": 17,
     "root": "compute_primitive_root", "input": [1, 2, 3, 4],
     "source": "crates/barracuda/tests/property/fhe_properties.rs:79-105"},
    {"name": "roundtrip_prop_8_257", "kind": "roundtrip", "degree": 8, "modulus": 257,
     "root": "compute_primitive_root", "input": [(i * 7) % 257 for i in range(1, 9)],
     "source": "crates/barracuda/tests/property/fhe_properties.rs:109-138"},
    {"name": "intt_of_ntt_ones_4_17", "kind": "roundtrip", "degree": 4, "modulus": 17,
     "root": "known_root", "input": [1, 1, 1, 1],
     "source": "crates/barracuda/tests/fhe/intt.rs:49-85"},
    {"name": "linearity_8_257", "kind": "linearity", "degree": 8, "modulus": 257,
     "root": "compute_primitive_root", "a": [i * 5 for i in range(8)], "b": [i * 3 for i in range(8)],
     "source": "crates/barracuda/tests/property/fhe_properties.rs:440-488"},
    {"name": "ntt_zero_16_12289", "kind": "ntt_zero", "degree": 16, "modulus": 12289,
     "root": "find_root_of_unity", "input": [0] * 16,
     "source": "crates/barracuda/tests/fhe/ntt.rs:152-179"},
    {"name": "ntt_max_coeff_8_12289", "kind": "ntt_range", "degree": 8, "modulus": 12289,
     "root": "find_root_of_unity", "input": [12288] * 8,
     "source": "crates/barracuda/tests/fhe/ntt.rs:181-208"},
    {"name": "ntt_known_vector_range_4_17_4", "kind": "ntt_range", "degree": 4, "modulus": 17,
     "root": 4, "input": [1, 2, 3, 4], "source": "crates/barracuda/tests/fhe/ntt.rs:11-40"},
    {"name": "pointwise_12289", "kind": "pointwise", "degree": 4, "modulus": 12289,
     "a": [100, 200, 300, 400], "b": [5, 10, 15, 20], "expect": [500, 2000, 4500, 8000],
     "source": "crates/barracuda/src/bin/validate_gpu.rs:94-130"},
    {"name": "pointwise_identity_4_12289", "kind": "pointwise_identity", "degree": 4,
     "modulus": 12289, "root": "find_root_of_unity",
     "source": "crates/barracuda/tests/fhe/pointwise.rs:49-100"},
    {"name": "pointwise_zero_16_97", "kind": "pointwise_zero", "degree": 16, "modulus": 97,
     "root": "find_root_of_unity", "source": "crates/barracuda/tests/fhe/pointwise.rs:102-140"},
    {"name": "fast_mul_vs_naive_4_12289", "kind": "fast_mul_naive", "degree": 4, "modulus": 12289,
     "root": "find_root_of_unity", "source": "crates/barracuda/tests/fhe/fast_poly_mul.rs:10-73"},
    {"name": "fast_mul_commutative_32_12289", "kind": "fast_mul_commutative", "degree": 32,
     "modulus": 12289, "root": "find_root_of_unity",
     "source": "crates/barracuda/tests/fhe/fast_poly_mul.rs:75-110"},
    {"name": "fast_mul_distributive_4_12289", "kind": "fast_mul_distributive", "degree": 4,
     "modulus": 12289, "root": "find_root_of_unity",
     "source": "crates/barracuda/tests/fhe/fast_poly_mul.rs:112-170"},
    {"name": "poly_add_8_97", "kind": "poly_add", "degree": 8, "modulus": 97,
     "a": [1, 2, 3, 4, 5, 6, 7, 8], "b": [10, 20, 30, 40, 50, 60, 70, 80],
     "expect": [11, 22, 33, 44, 55, 66, 77, 88],
     "source": "crates/barracuda/src/ops/fhe_poly_add.rs:203-251"},
    {"name": "poly_add_reduce_4_100", "kind": "poly_add", "degree": 4, "modulus": 100,
     "a": [50, 60, 70, 80], "b": [60, 50, 40, 30], "expect": [10, 10, 10, 10],
     "source": "crates/barracuda/src/ops/fhe_poly_add.rs:254-302"},
    {"name": "poly_sub_8_97", "kind": "poly_sub", "degree": 8, "modulus": 97,
     "a": [50, 60, 70, 80, 90, 85, 75, 65], "b": [10, 20, 30, 40, 50, 60, 70, 80],
     "expect": [40, 40, 40, 40, 40, 25, 5, 82],
     "source": "crates/barracuda/src/ops/fhe_poly_sub.rs:171-217"},
    {"name": "poly_mul_8_97", "kind": "poly_mul", "degree": 8, "modulus": 97,
     "a": [2, 3, 4, 5, 6, 7, 8, 9], "b": [5, 4, 3, 2, 10, 10, 10, 10],
     "expect": [10, 12, 12, 10, 60, 70, 80, 90],
     "source": "crates/barracuda/src/ops/fhe_poly_mul.rs:160-205"},
    {"name": "poly_add_prop_4_257", "kind": "poly_add", "degree": 4, "modulus": 257,
     "a": [10, 20, 30, 40], "b": [5, 15, 25, 35], "expect": [15, 35, 55, 75],
     "source": "crates/barracuda/tests/property/fhe_properties.rs:266-291 (expected from the test's mod_add)"},
    {"name": "poly_sub_prop_4_257", "kind": "poly_sub", "degree": 4, "modulus": 257,
     "a": [40, 30, 20, 10], "b": [5, 15, 25, 35], "expect": [35, 15, 252, 232],
     "source": "crates/barracuda/tests/property/fhe_properties.rs:293-318 (expected from the test's mod_sub)"},
    {"name": "poly_add_assoc_4_257", "kind": "poly_add_assoc", "degree": 4, "modulus": 257,
     "a": [10, 20, 30, 40], "b": [5, 15, 25, 35], "c": [3, 7, 11, 13],
     "source": "crates/barracuda/tests/property/fhe_properties.rs:320-365"},
]

# tests/fhe/helpers.rs:21-28 -- (degree, modulus, root), all primitive roots
KNOWN_ROOTS = [[4, 17, 4], [4, 97, 22], [4, 257, 241], [4, 12289, 1479], [8, 97, 64], [16, 97, 8]]

# tests/property/fhe_proptest.rs:156-164 -- (modulus, degree) with valid
# compute_primitive_root results
NTT_PARAMS = [[17, 4], [97, 8], [257, 8], [257, 16], [12289, 8], [12289, 16], [998244353, 32]]

# Constructor rejections, tests/fhe_fault_tests.rs and tests/fhe/error_handling.rs:
# [op, input_len_u32, degree, modulus, root, expect_error]
REJECTIONS = (
    [["ntt", 2 * max(d, 1), d, 257, 3, True] for d in [0, 3, 5, 6, 7, 9, 10, 15, 17, 100]]
    + [["ntt", 2 * n, 8, 257, "compute_primitive_root", True] for n in [0, 1, 4, 7, 9, 16]]
    + [["ntt", 8, 4, 0, 4, True], ["ntt", 16, 8, 19, 2, True]]
    + [["ntt", 2 * d, d, 12289, 11, True] for d in [3, 5, 6, 7, 9, 10, 15]]
    + [["ntt", 0, 0, 12289, 11, True]]
    + [["ntt", 8, 4, 17, "compute_primitive_root", False],
       ["ntt", 16, 8, 257, "compute_primitive_root", False]]
)
REJECTIONS_SOURCE = ("crates/barracuda/tests/fhe_fault_tests.rs:17-148; "
                     "crates/barracuda/tests/fhe/error_handling.rs:7-55")


def main():
    doc = {
        "about": "Known answers and fixed vectors transcribed from ecoPrimals/barraCuda tests "
                 "(see make_golden.py).",
        "cases": CASES,
        "known_roots": {"values": KNOWN_ROOTS, "source": "crates/barracuda/tests/fhe/helpers.rs:21-28"},
        "ntt_params": {"values": NTT_PARAMS,
                       "source": "crates/barracuda/tests/property/fhe_proptest.rs:156-199"},
        "rejections": {"values": REJECTIONS, "source": REJECTIONS_SOURCE},
    }
    with open(os.path.join(HERE, "reference_kats.json"), "w") as f:
        json.dump(doc, f, indent=1)
        f.write("\n")


if __name__ == "__main__":
    main()
