"""Temperature / top-p sampling (hetero/backends.py:106-120).

The oracle (oracle/sample.py) draws with the uniform variate taken outside,
which is how the device sampler (hq4_sample) receives it; here it is pinned
against the reference's own NumpyBackend.sample on identically seeded
generators (when the reference tree is mounted), and against numpy's
Generator.choice on the oracle's own probabilities everywhere."""
import numpy as np
import pytest

from oracle import refmodel
from oracle import sample as osm


def _cases(n_trials=300, seed=0):
    rng = np.random.default_rng(seed)
    for t in range(n_trials):
        n = int(rng.integers(2, 3000))
        z = (rng.standard_normal(n) * rng.uniform(0.1, 8.0)).astype(np.float32)
        temp = float(rng.choice([0.0, 0.3, 0.7, 1.0, 1.7]))
        top_p = float(rng.choice([1.0, 0.9, 0.5, 0.95, 0.2]))
        yield t, z, temp, top_p


def test_oracle_draw_is_generator_choice():
    for t, z, temp, top_p in _cases():
        if temp <= 0:
            continue
        p = osm.probabilities(z, temp, top_p)
        a = np.random.default_rng(1000 + t)
        b = np.random.default_rng(1000 + t)
        assert int(a.choice(len(p), p=p)) == osm.draw(p, b.random()), t
        assert a.random() == b.random()  # one variate consumed on both sides


@pytest.mark.skipif(not refmodel.available(), reason="reference tree not mounted")
def test_oracle_matches_reference_sample():
    import sys
    if refmodel.REF_ROOT not in sys.path:
        sys.path.insert(0, refmodel.REF_ROOT)
    from hetero.backends import NumpyBackend
    sample = NumpyBackend.sample  # a plain function of its arguments (backends.py:106-120)
    for t, z, temp, top_p in _cases():
        a = np.random.default_rng(2000 + t)
        b = np.random.default_rng(2000 + t)
        ref = sample(None, z, temp, top_p, a)
        u = b.random() if temp > 0 else 0.0
        assert ref == osm.sample_with_u(z, temp, top_p, u), t


def _draw_ok(p, u, got, ref, tol=5e-5):
    """got is the reference draw, or u lies within tol of the edge of got's
    interval in the reference's cumulative distribution (fp32 cumulative sums
    over 152064 entries carry ~1e-5 of rounding, differently ordered on the
    device, so a variate that close to an edge may land on either side)."""
    if got == ref:
        return True
    cdf = p.astype(np.float64).cumsum()
    cdf /= cdf[-1]
    lo = cdf[got - 1] if got > 0 else 0.0
    hi = cdf[got]
    return p[got] > 0 and (abs(u - lo) <= tol or abs(u - hi) <= tol or lo - tol <= u <= hi + tol)


@pytest.mark.gpu
@pytest.mark.parametrize("n", [152064, 1000, 7])
def test_device_sampler_matches_oracle(cuda, n):
    """hq4_sample against the oracle with the same uniform variate: the same
    token, or (rarely, for the full vocabulary) a neighbour of it when u lies
    within rounding of their shared cumulative edge; never a token outside
    the nucleus."""
    import torch
    from hetero_infer_b200 import _lib
    lib = _lib.load()
    rng = np.random.default_rng(n)
    out = torch.empty(1, dtype=torch.int32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    lib.hq4_device_status(1)
    same = 0
    trials = 60
    for t in range(trials):
        z = (rng.standard_normal(n) * rng.uniform(0.5, 12.0)).astype(np.float32)
        temp = float(rng.choice([0.3, 0.7, 1.0, 1.7]))
        top_p = float(rng.choice([1.0, 0.9, 0.5, 0.95, 0.1]))
        u = float(rng.random())
        zd = torch.from_numpy(z).cuda()
        assert lib.hq4_sample(zd.data_ptr(), n, temp, top_p, u, out.data_ptr(), st) == 0
        got = int(out.item())
        p = osm.probabilities(z, temp, top_p)
        ref = osm.draw(p, u)
        assert _draw_ok(p, u, got, ref), f"trial {t}: {got} vs {ref} (u={u})"
        same += got == ref
    assert lib.hq4_device_status(0) == 0
    assert same >= trials - 4, f"only {same} of {trials} draws equal"


@pytest.mark.gpu
def test_backend_sample_advances_the_generator_like_the_reference(cuda):
    """CudaBackend.sample draws on the device with one rng.random() per call,
    so a seeded stream of calls gives the reference procedure's tokens."""
    import torch
    from hetero_infer_b200.cuda_model import CudaBackend
    be = CudaBackend()
    rng_a, rng_b = np.random.default_rng(9), np.random.default_rng(9)
    zrng = np.random.default_rng(3)
    for _ in range(20):
        z = (zrng.standard_normal(5000) * 4).astype(np.float32)
        got = be.sample(torch.from_numpy(z).cuda(), 0.8, 0.9, rng_a)
        u = rng_b.random()
        p = osm.probabilities(z, 0.8, 0.9)
        assert _draw_ok(p, u, got, osm.draw(p, u))
    assert rng_a.random() == rng_b.random()
    assert be.sample(torch.from_numpy(z).cuda(), 0.0, 1.0, rng_a) == int(z.argmax())
