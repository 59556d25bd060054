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


# ---- FheRotate, FheModulusSwitch, FheKeySwitch ----
# The reference's tests for these ops (tests/property/fhe_properties.rs:
# 141-260, 368-433) assert properties that contradict the ops' own shaders,
# and return early without an FHE device, so they have never checked the
# shaders.  Each case below keeps the test's inputs; "expect" is derived here
# from the shader's formula in plain Python (not from the C oracle), and
# "test_asserts" records what the Rust test claims and why it cannot hold.


def _rotate_shader(x, degree, rotation, modulus):
    """fhe_rotate.rs:150-155 + fhe_rotate.wgsl:98-128."""
    r = degree + rotation if rotation < 0 else rotation
    g = (2 * r + 1) % 2**32
    out = [None] * degree
    for i, v in enumerate(x):
        p = ((i * g) % 2**32) % (2 * degree)
        if p >= degree:
            out[p - degree] = 0 if v == 0 else (modulus - v) % 2**64
        else:
            out[p] = v
    return out


def _modswitch_shader(x, q_old, q_new):
    """fhe_modulus_switch.wgsl:103-131 (u64 product and doubling wrap)."""
    out = []
    for c in x:
        scaled = (c * q_new) % 2**64
        quo, rem = scaled // q_old, scaled % q_old
        if (rem * 2) % 2**64 >= q_old:
            quo += 1
        out.append(quo % q_new if q_new else 0)
    return out


def _modswitch_exact(x, q_old, q_new):
    """round(c * q_new / q_old) mod q_new, ties up, in Python integers."""
    return [((c * q_new + (q_old - 1) // 2 + (1 if q_old % 2 == 0 else 0)) // q_old) % q_new
            if q_new else 0 for c in x]


ROT_IN = list(range(8))
ROT_IN10 = [i * 10 for i in range(8)]
CASES += [
    {"name": "rotate_compose_8_257", "kind": "rotate", "degree": 8, "modulus": 257,
     "rotations": [2, 3], "input": ROT_IN,
     "expect": _rotate_shader(_rotate_shader(ROT_IN, 8, 2, 257), 8, 3, 257),
     "same_as_rotations": [1],
     "test_asserts": "rotate(2) then rotate(3) == rotate(5); rotate(5) is rejected for degree 8 "
                     "(|5| > 4), and X^5 then X^7 is X^35 = X^3 mod X^16 - 1, i.e. rotate(1)",
     "source": "crates/barracuda/tests/property/fhe_properties.rs:195-232"},
    {"name": "rotate_inverse_8_257", "kind": "rotate", "degree": 8, "modulus": 257,
     "rotations": [3, -3], "input": ROT_IN10,
     "expect": _rotate_shader(_rotate_shader(ROT_IN10, 8, 3, 257), 8, -3, 257),
     "test_asserts": "rotate(3) then rotate(-3) == identity; the galois elements are 7 and "
                     "2 * (8 - 3) + 1 = 11, and 7 * 11 = 77 = 13 mod 16, not 1",
     "source": "crates/barracuda/tests/property/fhe_properties.rs:234-260"},
    {"name": "rotate_wrap_negate_8_257", "kind": "rotate", "degree": 8, "modulus": 257,
     "rotations": [1], "input": [0, 1, 2, 300, 4, 0, 6, 7],
     "expect": _rotate_shader([0, 1, 2, 300, 4, 0, 6, 7], 8, 1, 257),
     "source": "crates/barracuda/src/ops/fhe_rotate.wgsl:52-63 (a negated 0 stays 0; "
               "300 > q negates to 257 - 300 mod 2^64)"},
    {"name": "modulus_switch_4_257_17", "kind": "modulus_switch", "degree": 4,
     "modulus_old": 257, "modulus_new": 17, "input": [10, 20, 30, 40],
     "expect": _modswitch_shader([10, 20, 30, 40], 257, 17),
     "exact": _modswitch_exact([10, 20, 30, 40], 257, 17),
     "test_asserts": "output == input % 17 = [10, 3, 13, 6]; the op scales by 17/257 first",
     "source": "crates/barracuda/tests/property/fhe_properties.rs:144-166"},
    {"name": "modulus_switch_doc_60_58", "kind": "modulus_switch", "degree": 4,
     "modulus_old": 1152921504606584833, "modulus_new": 288230376151711777,
     "input": [0, 1, 2, 63],
     "expect": _modswitch_shader([0, 1, 2, 63], 1152921504606584833, 288230376151711777),
     "exact": _modswitch_exact([0, 1, 2, 63], 1152921504606584833, 288230376151711777),
     "source": "crates/barracuda/src/ops/fhe_modulus_switch.rs:42-50 (doc example moduli; "
               "inputs with c * q_new < 2^64, where the shader's u64 product is exact)"},
    {"name": "modulus_switch_doc_wrap_60_58", "kind": "modulus_switch", "degree": 4,
     "modulus_old": 1152921504606584833, "modulus_new": 288230376151711777,
     "input": [64, 1000, 1152921504606584832, 576460752303292416],
     "expect": _modswitch_shader([64, 1000, 1152921504606584832, 576460752303292416],
                                 1152921504606584833, 288230376151711777),
     "exact": _modswitch_exact([64, 1000, 1152921504606584832, 576460752303292416],
                               1152921504606584833, 288230376151711777),
     "source": "crates/barracuda/src/ops/fhe_modulus_switch.rs:42-50 (doc example moduli; "
               "c * q_new >= 2^64: the shader's product wraps, the exact result differs)"},
    {"name": "key_switch_4_257", "kind": "key_switch", "degree": 4, "modulus": 257,
     "decomp_base": 2, "decomp_levels": 4, "input": [100, 150, 200, 250],
     "expect": [100, 150, 200, 250],
     "test_asserts": "len(output) == degree * levels = 16; the output buffer is the input's size "
                     "(fhe_key_switch.rs:167-172), and its values are the input "
                     "(accumulate_switched copies binding 0)",
     "source": "crates/barracuda/tests/property/fhe_properties.rs:371-402"},
    {"name": "key_switch_det_4_257", "kind": "key_switch", "degree": 4, "modulus": 257,
     "decomp_base": 2, "decomp_levels": 4, "input": [50, 100, 150, 200],
     "expect": [50, 100, 150, 200],
     "source": "crates/barracuda/tests/property/fhe_properties.rs:405-433"},
]

# Constructor rejections in the ops' own unit tests: [op, args, expect_error]
# with args (input_len_u32, degree, ...) in the constructor's order.
OP_REJECTIONS = [
    ["rotate", [8, 3, 1, 12289], True],
    ["rotate", [8, 4, 3, 12289], True],
    ["rotate", [8, 4, -3, 12289], True],
    ["rotate", [8, 4, 2, 12289], False],
    ["rotate", [8, 4, -2, 12289], False],
    ["modulus_switch", [8, 3, 12289, 6145], True],
    ["modulus_switch", [8, 4, 12289, 12289], True],
    ["modulus_switch", [8, 4, 12289, 6145], False],
    ["key_switch", [8, 3, 12289, 1 << 16, 3], True],
    ["key_switch", [8, 4, 12289, 1, 3], True],
    ["key_switch", [8, 4, 12289, 1 << 16, 0], True],
    ["key_switch", [8, 4, 12289, 1 << 16, 3], False],
]
OP_REJECTIONS_SOURCE = ("crates/barracuda/src/ops/fhe_rotate.rs:189-205; "
                        "fhe_modulus_switch.rs:177-199; fhe_key_switch.rs:234-250")

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
        "op_rejections": {"values": OP_REJECTIONS, "source": OP_REJECTIONS_SOURCE},
    }
    with open(os.path.join(HERE, "reference_kats.json"), "w") as f:
        json.dump(doc, f, indent=1)
        f.write("\n")


if __name__ == "__main__":
    main()
