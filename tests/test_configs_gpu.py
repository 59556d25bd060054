"""Parity of the CUDA path on the five benchmark configurations at their full
sizes, through the C ABI.

At full size every limb-polynomial is checked through a size-independent
property: the round trip is the identity (digests of the whole batch).  Every
limb is also checked value by value against the oracle, on the first and the
last polynomial of the batch and on one in between: the forward transform of
the seeded input, and the inverse transform applied to a fresh input (not only
through the round trip, which could hide an error the inverse undoes).  The
oracle is the reference's own algorithm (oracle/ref_wgsl.c) for moduli below
2^31 and exact u128 arithmetic for the 60-bit family, where the reference
truncates its products; it runs on all host threads.  Inputs are the seeded
uniform values of bc_fill_uniform, regenerated on the host by the oracle.
Bar: bit-exact."""
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


def _gather(t, offs, n):
    """The limb-polynomials at word offsets `offs` of device tensor t, back to back (host)."""
    return np.concatenate([_host(t, o, n) for o in offs])


def _limb_samples(limbs, batch, rng, every_poly_ends=True):
    """(limb, poly) pairs: every limb on the first and last polynomial and on
    one polynomial in between (every limb once when every_poly_ends is False)."""
    pairs = []
    for l in range(limbs):
        mid = int(rng.integers(batch))
        pairs.append((l, mid))
        if every_poly_ends:
            pairs.extend([(l, 0), (l, batch - 1)])
    return sorted(set(pairs))


def _batch_case(device, stream, n, limbs, batch, bits, lay_kind, every_poly_ends=True, seed=0):
    """Fills, forwards and inverses a full batch; asserts every sampled limb-
    polynomial against the oracle (forward of the input, inverse of a fresh
    input) and the whole-batch round trip by digest."""
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
    y, z = torch.empty_like(x), torch.empty_like(x)
    plan.fill_uniform(x, batch, seed=seed, layout=lay, stream=sh)
    d_in = _digest(device, x, words, sh)
    plan.forward(x, y, batch, layout=lay, stream=sh)
    plan.inverse(x, z, batch, layout=lay, stream=sh)  # a fresh input for the inverse
    torch.cuda.synchronize()
    rng = np.random.default_rng(n + limbs + bits)
    pairs = _limb_samples(limbs, batch, rng, every_poly_ends)
    assert {l for l, _ in pairs} == set(range(limbs))
    offs = [off(l, p) for l, p in pairs]
    xin = _gather(x, offs, n)
    # the device generator is the oracle's counter-based generator
    for k, (l, p) in enumerate(pairs[:4] + pairs[-4:]):
        kk = pairs.index((l, p))
        assert (xin[kk * n:(kk + 1) * n] == O.seeded_fill(n, seed, (l * batch + p) * n, qs[l])).all(), (n, l, p)
    mods = [qs[l] for l, _ in pairs]
    roots = [psis[l] for l, _ in pairs]
    fwd_kind, inv_kind = (("negacyclic_ntt", "negacyclic_intt") if bits == 31
                          else ("exact_negacyclic_ntt", "exact_negacyclic_intt"))
    want_f = O.batch_transform(fwd_kind, xin, n, mods, roots)
    want_i = O.batch_transform(inv_kind, xin, n, mods, roots)
    got_f, got_i = _gather(y, offs, n), _gather(z, offs, n)
    for k, (l, p) in enumerate(pairs):
        sl = slice(k * n, (k + 1) * n)
        assert (got_f[sl] == want_f[sl]).all(), ("forward", n, bits, l, p)
        assert (got_i[sl] == want_i[sl]).all(), ("inverse", n, bits, l, p)
    del z
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
    _batch_case(device, stream, 1 << 14, 16, 64, bits, "limb_major")


@pytest.mark.parametrize("bits", [31, 60])
def test_config3_ciphertext_batch_n2_16(device, stream, bits):
    """Config 3: N=2^16, 48 limbs, 128 ciphertexts x 2 polynomials, [ct][2][limb][N].
    Every limb of the first and the last ciphertext, and of one in between."""
    _batch_case(device, stream, 1 << 16, 48, 256, bits, "ct_major")


@pytest.mark.parametrize("logn", [12, 13, 14, 15, 16, 17])
@pytest.mark.parametrize("bits", [60, 31])
def test_config4_size_sweep(device, stream, logn, bits):
    """Config 4: N in 2^12..2^17, 8 to 64 limbs, batch sized to about 2 GB (u64);
    every limb checked once per N."""
    n = 1 << logn
    limbs = 64 if logn <= 13 else (16 if logn <= 15 else 8)
    batch = max(1, (2 << 30) // (8 * n * limbs))
    _batch_case(device, stream, n, limbs, batch, bits, "limb_major", every_poly_ends=False)


@pytest.mark.parametrize("mode", [bc.NEGACYCLIC, bc.CYCLIC])
@pytest.mark.parametrize("bits", [60, 31])
def test_config2_polymul_n2_15(device, stream, mode, bits):
    """Config 2: NTT(a), NTT(b), pointwise, INTT at N=2^15, 32 limbs x 32 pairs.
    One pair of every limb is checked value by value: for q < 2^31 against the
    reference's own chain (FheFastPolyMul for the cyclic mode, the ops chained
    with a psi twist for the negacyclic one), for the 60-bit family against the
    exact product."""
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
    pairs = [(l, int(rng.integers(batch))) for l in range(limbs)]
    offs = [(l * batch + p) * n for l, p in pairs]
    A, B, C = _gather(a, offs, n), _gather(b, offs, n), _gather(c, offs, n)
    if bits == 31:
        kind = "ref_cyclic" if mode == bc.CYCLIC else "ref_negacyclic"
    else:
        kind = "exact_cyclic" if mode == bc.CYCLIC else "exact_negacyclic"
    want = O.batch_polymul(kind, A, B, n, [qs[l] for l, _ in pairs], [roots[l] for l, _ in pairs])
    for k, (l, p) in enumerate(pairs):
        sl = slice(k * n, (k + 1) * n)
        assert (C[sl] == want[sl]).all(), (bits, mode, l, p)
    plan.close()
