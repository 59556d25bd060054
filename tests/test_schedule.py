"""CPU checks of the fast kernels' index machinery (barracuda_b200/csrc/
gen_schedule.py): every pass maps (CTA rank, thread, register) bijectively
onto positions, every shared-memory access of a warp hits 32 distinct banks,
the cooperative HBM stages move every owned coefficient exactly once, and the
committed bc_schedule.hpp is what the generator produces."""
import importlib.util
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GEN = os.path.join(ROOT, "barracuda_b200", "csrc", "gen_schedule.py")


def _gen():
    spec = importlib.util.spec_from_file_location("gen_schedule", GEN)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_schedules_check_and_header_is_current():
    g = _gen()
    scheds = g.all_schedules()  # runs check() and check_coop() on every config
    assert {(s["L"], s["loge"]) for s in scheds} >= {(L, 5) for L in range(10, 18)}
    with open(g.OUT) as f:
        assert f.read() == g.emit(scheds), "bc_schedule.hpp is stale: rerun gen_schedule.py"


def test_padded_layout_is_additive_and_bank_spreading():
    g = _gen()
    for a in range(0, 1 << 14, 37):
        for b in (1 << 5, 3 << 10, 1 << 13, 0b10101):
            if a & b == 0:
                assert g.swz(a | b) == g.swz(a) + g.swz(b)
    # lane bits with distinct residues mod 5 spread a warp over 32 banks
    bits = [0, 6, 12, 3, 9]  # residues 0, 1, 2, 3, 4
    banks = {g.swz(sum(((l >> j) & 1) << b for j, b in enumerate(bits))) & 31 for l in range(32)}
    assert len(banks) == 32
