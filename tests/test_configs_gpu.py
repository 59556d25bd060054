"""Parity of the CUDA path on the five benchmark configurations at their full
sizes, through the C ABI.

At full size every limb-polynomial is checked through size-independent
properties: the round trip is the identity (digests of the whole batch), and
for products NTT(c) = NTT(a) * NTT(b).  A few sampled limb-polynomials per
config are checked value by value against the oracle: the reference's own
algorithm (oracle/ref_wgsl.c) for moduli below 2^31, exact u128 arithmetic for
the 60-bit family, where the reference truncates its products.  Inputs are
the seeded uniform values of bc_fill_uniform, regenerated on the host by the
oracle for the samples.  Bar: bit-exact."""
import numpy as np
import pytest
import torch

import barracuda_b200 as bc
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _roots(qs, n, mode):
    psis = [bc.negacyclic_root(q, n) for q in qs]
    return psis if mode == bc.NEGACYCLIC else [p * p % q for p, q in zip(psis, qs)]


def _host(t, lo, n):
    return t[lo:lo + n].cpu().numpy().view(np.uint64).copy()


def _forward_oracle(x, n, q, r, bits, mode):
    if mode == bc.NEGACYCLIC:
        return O.ref_negacyclic_ntt(x, n, q, r) if bits == 31 else O.exact_negacyclic_ntt(x, n, q, r)
    return O.ref_ntt(x, n, q, r) if bits == 31 else O.exact_ntt(x, n, q, r)


def _digest(dev, t, count, stream):
    out = torch.zeros(1, dtype=torch.int64, device="cuda")
    bc.digest(dev, t, count, out, stream=stream)
    torch.cuda.synchronize()
    return int(out.item()) & (2**64 - 1)


@pytest.fixture(scope="module")
def stream():
    """An explicit stream (handle 0 would mean the context stream to the C ABI)."""
    torch.cuda.set_device(0)
    prev = torch.cuda.current_stream()
    s = torch.cuda.Stream()
    torch.cuda.set_stream(s)
    yield s
    torch.cuda.synchronize()
    torch.cuda.set_stream(prev)


def _batch_case(device, stream, n, limbs, batch, bits, lay_kind, samples, seed=0):
    """Fills, forwards, samples, inverses; returns nothing, asserts parity."""
    sh = stream.cuda_stream
    qs = bc.ntt_primes(bits, n, limbs)
    psis = _roots(qs, n, bc.NEGACYCLIC)
    plan = bc.NttPlan(device, n, qs, psis, mode=bc.NEGACYCLIC)
    if lay_kind == "limb_major":
        lay = bc.Layout(limb_stride=batch * n, poly_stride=n)
        off = lambda l, p: (l * batch + p) * n  # noqa: E731
    else:  # [ct][2][limb][N]: poly index = 2 * ct + j
        lay = bc.Layout(limb_stride=n, poly_stride=limbs * n)
        off = lambda l, p: (p * limbs + l) * n  # noqa: E731
    words = limbs * batch * n
    x = torch.empty(words, dtype=torch.int64, device="cuda")
    y = torch.empty_like(x)
    plan.fill_uniform(x, batch, seed=seed, layout=lay, stream=sh)
    d_in = _digest(device, x, words, sh)
    plan.forward(x, y, batch, layout=lay, stream=sh)
    torch.cuda.synchronize()
    rng = np.random.default_rng(n + limbs + bits)
    for _ in range(samples):
        l, p = int(rng.integers(limbs)), int(rng.integers(batch))
        xin = _host(x, off(l, p), n)
        # the device generator is the oracle's counter-based generator
        g0 = (l * batch + p) * n
        assert (xin == O.seeded_fill(n, seed, g0, qs[l])).all(), (n, l, p)
        want = _forward_oracle(xin, n, qs[l], psis[l], bits, bc.NEGACYCLIC)
        assert (_host(y, off(l, p), n) == want).all(), (n, bits, l, p)
    plan.inverse(y, y, batch, layout=lay, stream=sh)  # in place
    assert _digest(device, y, words, sh) == d_in, "round trip is not the identity"
    device.synchronize()
    plan.close()
    del x, y


@pytest.mark.parametrize("bits", [31, 60])
def test_config0_single_roundtrip_n4096(device, stream, bits):
    """Config 0: N=4096, one limb, batch 1; forward bit-exact, round trip identity,
    and the reference op API (twist + FheNtt with omega = psi^2) agrees for q < 2^31."""
    n = 4096
    q = bc.ntt_prime(bits, n, 0)
    psi = bc.negacyclic_root(q, n)
    x = O.seeded_fill(n, 0, 0, q)
    plan = bc.NttPlan(device, n, [q], [psi], mode=bc.NEGACYCLIC)
    t = torch.from_numpy(x.view(np.int64).copy()).cuda()
    y = torch.empty_like(t)
    sh = stream.cuda_stream
    plan.forward(t, y, 1, stream=sh)
    torch.cuda.synchronize()
    X = y.cpu().numpy().view(np.uint64)
    assert (X == _forward_oracle(x, n, q, psi, bits, bc.NEGACYCLIC)).all()
    if bits == 31:
        tw = np.array([pow(psi, j, q) for j in range(n)], np.uint64)
        twisted = O.ref_pointwise(x, tw, n, q)
        via_ops = np.array(bc.FheNtt.new(bc.FheTensor.from_u32(twisted.view(np.uint32), device), n, q,
                                         psi * psi % q).execute().to_u64())
        assert (via_ops == X).all()
    plan.inverse(y, y, 1, stream=sh)
    torch.cuda.synchronize()
    assert (y.cpu().numpy().view(np.uint64) == x).all()
    plan.close()


@pytest.mark.parametrize("bits", [60, 31])
def test_config1_batched_forward_n2_14(device, stream, bits):
    """Config 1: N=2^14, 16 limbs x 64 polynomials, limb-major contiguous."""
    _batch_case(device, stream, 1 << 14, 16, 64, bits, "limb_major", samples=4)


@pytest.mark.parametrize("bits", [31, 60])
def test_config3_ciphertext_batch_n2_16(device, stream, bits):
    """Config 3: N=2^16, 48 limbs, 128 ciphertexts x 2 polynomials, [ct][2][limb][N]."""
    _batch_case(device, stream, 1 << 16, 48, 256, bits, "ct_major", samples=3)


@pytest.mark.parametrize("logn", [12, 13, 14, 15, 16, 17])
@pytest.mark.parametrize("bits", [60, 31])
def test_config4_size_sweep(device, stream, logn, bits):
    """Config 4: N in 2^12..2^17, 8 to 64 limbs, batch sized to about 2 GB (u64)."""
    n = 1 << logn
    limbs = 64 if logn <= 13 else (16 if logn <= 15 else 8)
    batch = max(1, (2 << 30) // (8 * n * limbs))
    _batch_case(device, stream, n, limbs, batch, bits, "limb_major", samples=1)


@pytest.mark.parametrize("mode", [bc.NEGACYCLIC, bc.CYCLIC])
@pytest.mark.parametrize("bits", [60, 31])
def test_config2_polymul_n2_15(device, stream, mode, bits):
    """Config 2: NTT(a), NTT(b), pointwise, INTT at N=2^15, 32 limbs x 32 pairs.
    Full batch: NTT(c) = NTT(a) * NTT(b) on samples, exact; for q < 2^31 the
    sampled products also equal the reference's own NTT -> pointwise -> INTT chain."""
    n, limbs, batch = 1 << 15, 32, 32
    sh = stream.cuda_stream
    qs = bc.ntt_primes(bits, n, limbs)
    roots = _roots(qs, n, mode)
    plan = bc.NttPlan(device, n, qs, roots, mode=mode)
    words = limbs * batch * n
    a = torch.empty(words, dtype=torch.int64, device="cuda")
    b, c = torch.empty_like(a), torch.empty_like(a)
    plan.fill_uniform(a, batch, seed=1, stream=sh)
    plan.fill_uniform(b, batch, seed=2, stream=sh)
    plan.polymul(a, b, c, batch, stream=sh)
    torch.cuda.synchronize()
    rng = np.random.default_rng(bits + mode)
    for _ in range(2):
        l, p = int(rng.integers(limbs)), int(rng.integers(batch))
        o = (l * batch + p) * n
        A, B, C = _host(a, o, n), _host(b, o, n), _host(c, o, n)
        q, r = qs[l], roots[l]
        fwd = (lambda v: O.exact_negacyclic_ntt(v, n, q, r)) if mode == bc.NEGACYCLIC else \
            (lambda v: O.exact_ntt(v, n, q, r))
        FA, FB, FC = fwd(A), fwd(B), fwd(C)
        prod = np.array([O.lib().orc_mulmod(int(u), int(v), q) for u, v in zip(FA, FB)], np.uint64)
        assert (FC == prod).all(), (bits, mode, l, p)
        if bits == 31:
            if mode == bc.CYCLIC:
                want = O.ref_fast_poly_mul(A, B, n, q, r)
            else:
                want = O.ref_negacyclic_intt(O.ref_pointwise(O.ref_negacyclic_ntt(A, n, q, r),
                                                             O.ref_negacyclic_ntt(B, n, q, r), n, q), n, q, r)
            assert (C == want).all(), (mode, l, p)
    plan.close()
