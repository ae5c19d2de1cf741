"""Edge cases of the stage kernels through the C ABI.

argmax follows numpy's z.argmax() (hetero/backends.py:106-109): the first NaN
wins, else the largest value with the lowest index among equals, and -inf
rows give index 0 -- the result is always a valid index.  The embedding
gather reads nothing for an id outside the table: the row is zeros and the
device status word gets bit 1."""
import numpy as np
import pytest


@pytest.fixture(scope="module")
def lib(cuda):
    from hetero_infer_b200 import _lib
    return _lib.load()


def _argmax(lib, x):
    import torch
    d = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    idx = torch.full((1,), -7, dtype=torch.int32, device="cuda")
    val = torch.empty(1, dtype=torch.float32, device="cuda")
    rc = lib.hq4_argmax(d.data_ptr(), d.numel(), idx.data_ptr(), None, 0, None, val.data_ptr(),
                        torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    return int(idx.item()), float(val.item())


def _cases():
    rng = np.random.default_rng(3)
    out = []
    for n in (1, 31, 1024, 1025, 76032, 152064):
        out.append(rng.standard_normal(n).astype(np.float32))
    z = np.full(5000, np.nan, np.float32)
    out.append(z)                                        # all NaN -> 0
    z = rng.standard_normal(5000).astype(np.float32)
    z[[777, 3001]] = np.nan
    out.append(z)                                        # first NaN
    z = rng.standard_normal(5000).astype(np.float32)
    z[4999] = np.nan
    z[10] = np.inf
    out.append(z)                                        # NaN beats +inf
    out.append(np.full(3000, -np.inf, np.float32))       # all -inf -> 0
    z = np.full(3000, -np.inf, np.float32)
    z[2500] = -1e30
    out.append(z)
    z = np.zeros(70000, np.float32)
    z[[69999, 40000, 1500]] = 2.0
    out.append(z)                                        # ties -> lowest
    out.append(np.round(rng.standard_normal(152064) * 2).astype(np.float32))  # many ties
    z = np.full(2048, -np.finfo(np.float32).max, np.float32)
    out.append(z)
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("ci", range(len(_cases())))
def test_argmax_is_numpy_argmax(lib, ci):
    z = _cases()[ci]
    i, v = _argmax(lib, z)
    assert i == int(z.argmax())
    assert 0 <= i < z.size
    if np.isnan(z[i]):
        assert np.isnan(v)
    else:
        assert v == z[i]


@pytest.mark.gpu
def test_embed_rejects_out_of_range_ids(lib):
    import torch
    vocab, hidden = 1000, 256
    rng = np.random.default_rng(0)
    table = torch.from_numpy((rng.standard_normal((vocab, hidden)) * 0.02).astype(np.float16)).cuda()
    st = torch.cuda.current_stream().cuda_stream
    lib.hq4_device_status(1)
    ids = torch.tensor([5, 999, 0], dtype=torch.int32, device="cuda")
    out = torch.empty((3, hidden), dtype=torch.float32, device="cuda")
    assert lib.hq4_embed_f16(table.data_ptr(), ids.data_ptr(), 3, hidden, vocab, out.data_ptr(), st) == 0
    torch.cuda.synchronize()
    assert torch.equal(out, table[ids.long()].float())
    assert lib.hq4_device_status(0) == 0
    ids = torch.tensor([7, vocab, -1, 2 ** 31 - 1, 3], dtype=torch.int32, device="cuda")
    out = torch.full((5, hidden), 9.0, dtype=torch.float32, device="cuda")
    assert lib.hq4_embed_f16(table.data_ptr(), ids.data_ptr(), 5, hidden, vocab, out.data_ptr(), st) == 0
    torch.cuda.synchronize()
    assert torch.equal(out[0], table[7].float()) and torch.equal(out[4], table[3].float())
    assert float(out[1:4].abs().sum()) == 0.0
    assert lib.hq4_device_status(1) & 2
    assert lib.hq4_device_status(0) == 0
    assert lib.hq4_embed_f16(table.data_ptr(), ids.data_ptr(), 5, hidden, 0, out.data_ptr(), st) == -1


@pytest.mark.gpu
def test_argmax_pair_and_pick_token_match_numpy_over_shards(lib):
    """Row-sharded greedy pick: per-shard pairs (value bits, global index) and
    the pick over them equal np.argmax over the whole vector, NaN included."""
    import torch
    rng = np.random.default_rng(5)
    st = torch.cuda.current_stream().cuda_stream
    for trial in range(40):
        n = int(rng.integers(8, 5000))
        z = np.round(rng.standard_normal(n) * 3).astype(np.float32)
        if trial % 4 == 1:
            z[rng.integers(0, n, size=2)] = np.nan
        elif trial % 4 == 2:
            z[:] = -np.inf
        world = int(rng.integers(1, 9))
        pairs = torch.empty((world, 2), dtype=torch.int32, device="cuda")
        d = torch.from_numpy(z).cuda()
        for r in range(world):
            lo, hi = n * r // world, n * (r + 1) // world
            if hi == lo:
                pairs[r, 0] = torch.tensor([np.float32(-np.inf)]).view(torch.int32)[0]
                pairs[r, 1] = 2 ** 31 - 1
                continue
            assert lib.hq4_argmax_pair(d[lo:].data_ptr(), hi - lo, lo, pairs[r].data_ptr(), st) == 0
        tok = torch.empty(1, dtype=torch.int32, device="cuda")
        hist = torch.zeros(4, dtype=torch.int32, device="cuda")
        assert lib.hq4_pick_token(pairs.data_ptr(), world, tok.data_ptr(), hist.data_ptr(), 2, st) == 0
        torch.cuda.synchronize()
        assert int(tok.item()) == int(z.argmax()) == int(hist[2].item()), (trial, world)


def _attention_ref(q, kc, vc, p0, n_heads, n_kv, scale):
    """float64 restatement of the reference's sdpa (hetero/cpu_model.py:233-252)
    for the decode layout: query token i sits at position p0 + i and attends
    to cache rows [0, p0 + i]."""
    L, H, D = q.shape
    G = n_heads // n_kv
    out = np.zeros((L, H, D))
    for i in range(L):
        n = p0 + i + 1
        for h in range(H):
            k = kc[h // G, :n].astype(np.float64)
            v = vc[h // G, :n].astype(np.float64)
            s = k @ q[i, h].astype(np.float64) * scale
            e = np.exp(s - s.max())
            out[i, h] = (e / e.sum()) @ v
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("n_heads,n_kv,head_dim,p0,n_tokens", [
    (28, 4, 128, 0, 1),       # first token: one key
    (28, 4, 128, 37, 1),
    (28, 4, 128, 480, 1),     # long context: two key rounds per thread
    (28, 4, 128, 10, 5),      # prefill rows, causal
    (8, 8, 64, 100, 3),       # no grouping, head_dim 64
    (4, 1, 256, 300, 2),      # head_dim 256: two value-pass column rounds
])
def test_attention_matches_float64_sdpa(lib, n_heads, n_kv, head_dim, p0, n_tokens):
    import torch
    max_ctx = 512
    rng = np.random.default_rng(p0 + head_dim)
    q = rng.standard_normal((n_tokens, n_heads, head_dim)).astype(np.float32)
    kc = rng.standard_normal((n_kv, max_ctx, head_dim)).astype(np.float32)
    vc = rng.standard_normal((n_kv, max_ctx, head_dim)).astype(np.float32)
    scale = float(1.0 / np.sqrt(head_dim))
    dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, kc, vc))
    out = torch.full((n_tokens, n_heads, head_dim), float("nan"), device="cuda")
    pos = torch.tensor([p0], dtype=torch.int32, device="cuda")
    rc = lib.hq4_attention(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), out.data_ptr(), n_heads, n_kv, head_dim,
                           max_ctx, pos.data_ptr(), n_tokens, scale, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    ref = _attention_ref(q, kc, vc, p0, n_heads, n_kv, scale)
    got = out.cpu().numpy().astype(np.float64)
    err = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert err < 2e-6, err
