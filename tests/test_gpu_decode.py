"""Decode kernels on the GPU (bb_decode, bb_decode_route) against the oracle's restatements of
kernels/bigger_bird_decode.py and kernels/bigger_bird_route.py."""
import numpy as np
import pytest
import torch

from oracle import bigbird_oracle as orc

pytestmark = pytest.mark.gpu
DEV = "cuda"
ATOL_MAX, ATOL_MEAN = 2e-2, 2e-3


def close(got, want, what):
    err = np.abs(got.float().cpu().numpy() - want)
    assert err.max() <= ATOL_MAX and err.mean() <= ATOL_MEAN, f"{what}: max {err.max():.4g} mean {err.mean():.4g}"


def make(H=32, hk=8, cap=32768, d=128, dtype=torch.bfloat16, seed=3):
    g = torch.Generator(device=DEV).manual_seed(seed)
    q = (torch.randn(H, d, device=DEV, generator=g) * 0.5).to(dtype)
    k = (torch.randn(hk, cap, d, device=DEV, generator=g) * 0.5).to(dtype)
    v = torch.randn(hk, cap, d, device=DEV, generator=g).to(dtype)
    return q, k, v


def routes(rows, R, lo, hi, seed=5):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return torch.stack([torch.randperm(hi - lo, device=DEV, generator=g)[:R] + lo for _ in range(rows)]).sort(-1).values


def np32(t):
    return t.float().cpu().numpy()


@pytest.mark.parametrize("mode", ["pooled", "per_head"])
@pytest.mark.parametrize("d", [128, 64, 96, 32])
def test_decode_matches_oracle(mode, d):
    from utmist_bigger_bird_b200 import bigger_bird_decode
    H, hk, cap, front, window, R = 32, 8, 32768, 64, 4096, 512
    q, k, v = make(H, hk, cap, d)
    idx = routes(hk if mode == "pooled" else H, R, front, cap - window)
    out = bigger_bird_decode(q, k, v, idx, front=front, window=window, scale=d ** -0.5)
    want = orc.decode(np32(q), np32(k), np32(v), idx.cpu().numpy(), front=front, window=window, scale=d ** -0.5)
    assert out.shape == (H, d) and out.dtype == q.dtype
    close(out, want, f"decode {mode} d={d}")


def test_dense_decode_and_device_length():
    """front=0, window=capacity, no routes: dense flash-decoding over the first n keys, with n given
    as a host int and as a 1-element GPU tensor (keys at >= n ignored)."""
    from utmist_bigger_bird_b200 import bigger_bird_decode
    H, hk, cap, d = 32, 8, 16384, 128
    q, k, v = make(H, hk, cap, d)
    none = torch.empty(hk, 0, dtype=torch.int64, device=DEV)
    for n in (cap, 9000, 130):
        want = orc.decode(np32(q), np32(k), np32(v), np.zeros((hk, 0), np.int64), front=0, window=cap,
                          scale=d ** -0.5, n=n)
        # window = cap with n < cap: positions n - cap + j < 0 are skipped, i.e. the first n keys.
        got = bigger_bird_decode(q, k, v, none, front=0, window=cap, scale=d ** -0.5,
                                 n=torch.tensor([n], device=DEV))
        close(got, want, f"dense n={n} (device length)")
    got = bigger_bird_decode(q, k, v, none, front=0, window=cap, scale=d ** -0.5)
    close(got, orc.decode(np32(q), np32(k), np32(v), np.zeros((hk, 0), np.int64), front=0, window=cap,
                          scale=d ** -0.5), "dense full cache")


def test_decode_cuda_graph_follows_device_length():
    """A CUDA graph captured once reads the cache length from the GPU on every replay."""
    from utmist_bigger_bird_b200 import bigger_bird_decode
    H, hk, cap, d, front, window, R = 32, 8, 16384, 128, 64, 1024, 256
    q, k, v = make(H, hk, cap, d)
    idx = routes(hk, R, front, 8000 - window)
    n_t = torch.tensor([12000], device=DEV)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            bigger_bird_decode(q, k, v, idx, front=front, window=window, scale=d ** -0.5, n=n_t)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = bigger_bird_decode(q, k, v, idx, front=front, window=window, scale=d ** -0.5, n=n_t)
    for n in (8000, 12000, 16384):
        n_t.fill_(n)
        graph.replay()
        torch.cuda.synchronize()
        eager = bigger_bird_decode(q, k, v, idx, front=front, window=window, scale=d ** -0.5, n=n)
        assert torch.equal(out, eager), n
        close(out, orc.decode(np32(q), np32(k), np32(v), idx.cpu().numpy(), front=front, window=window,
                              scale=d ** -0.5, n=n), f"graph n={n}")


def test_pooled_probs_and_route_match_oracle():
    from utmist_bigger_bird_b200 import bigger_bird_route, pooled_probs
    H, hk, cap, d, front, window, kr = 32, 8, 32768, 128, 64, 4096, 512
    q, k, _ = make(H, hk, cap, d)
    for n in (None, 20000):
        p = pooled_probs(q, k, front=front, window=window, scale=d ** -0.5, n=n)
        want = orc.pooled_probs(np32(q), np32(k), front=front, window=window, scale=d ** -0.5, n=n)
        got = p.cpu().numpy()
        assert ((got == -1) == (want == -1)).all(), "same masked positions"
        live = want != -1
        np.testing.assert_allclose(got[live], want[live], rtol=2e-2, atol=2e-9)
        idx = bigger_bird_route(q, k, kr, front=front, window=window, scale=d ** -0.5, n=n)
        assert idx.dtype == torch.int64 and idx.shape == (hk, kr)
        nn = cap if n is None else n
        assert ((idx >= front) & (idx < nn - window)).all()
        for h in range(hk):
            chosen = got[h, idx[h].cpu().numpy()]
            rest = np.delete(got[h], idx[h].cpu().numpy())
            assert chosen.min() >= rest.max(), "top-k of the kernel's own probabilities"


def test_decode_errors():
    from utmist_bigger_bird_b200 import bigger_bird_decode, pooled_probs
    q, k, v = make(32, 8, 1024, 128)
    idx = routes(8, 16, 64, 512)
    with pytest.raises(ValueError):
        bigger_bird_decode(q.cpu(), k, v, idx)
    with pytest.raises(ValueError):
        bigger_bird_decode(q, k, v[:, :512], idx)
    with pytest.raises(ValueError):
        bigger_bird_decode(q, k, v, idx[:3])
    with pytest.raises(ValueError):
        bigger_bird_decode(q, k, v, idx, front=64, window=4096)       # cache shorter than front + window
    with pytest.raises(ValueError):
        pooled_probs(q.float(), k)


@pytest.mark.parametrize("splits", [1, 7, 5000])
def test_decode_explicit_splits(splits):
    """Caller-chosen split counts (one split, an odd count, more than the cap of 4096) give the
    same output as the oracle."""
    from utmist_bigger_bird_b200 import bigger_bird_decode
    H, hk, cap, d, front, window, R = 32, 8, 16384, 128, 64, 4096, 256
    q, k, v = make(H, hk, cap, d)
    idx = routes(hk, R, front, cap - window)
    out = bigger_bird_decode(q, k, v, idx, front=front, window=window, scale=d ** -0.5, splits=splits)
    want = orc.decode(np32(q), np32(k), np32(v), idx.cpu().numpy(), front=front, window=window, scale=d ** -0.5)
    close(out, want, f"splits={splits}")


@pytest.mark.parametrize("d", [128, 64])
def test_decode_route_index_dtypes(d):
    """Routes as int64 (the dtype bigger_bird_route returns) and as int32 are read as given (no
    conversion pass): the outputs are bit-identical."""
    from utmist_bigger_bird_b200 import bigger_bird_decode
    H, hk, cap, front, window, R = 32, 8, 16384, 64, 4096, 300
    q, k, v = make(H, hk, cap, d)
    idx = routes(hk, R, front, cap - window)
    assert idx.dtype == torch.int64
    kw = dict(front=front, window=window, scale=d ** -0.5)
    o64 = bigger_bird_decode(q, k, v, idx, **kw)
    o32 = bigger_bird_decode(q, k, v, idx.to(torch.int32), **kw)
    assert torch.equal(o64, o32)
    # a strided int64 view (every other column of a wider tensor) is made contiguous first
    wide = torch.stack([idx, idx], -1).reshape(hk, 2 * R)[:, ::2]
    assert torch.equal(bigger_bird_decode(q, k, v, wide, **kw), o64)
    want = orc.decode(np32(q), np32(k), np32(v), idx.cpu().numpy(), **kw)
    close(o64, want, f"int64 routes d={d}")


def test_decode_route_output_widths():
    """bigger_bird_route's int64 routes (written as int64 by the top-k) equal the int32 output of
    the same call, and both are the reference's dtype-independent position sets."""
    from utmist_bigger_bird_b200 import _ops, bigger_bird_route
    H, hk, cap, d, front, window, R = 32, 8, 16384, 128, 64, 4096, 300
    q, k, _ = make(H, hk, cap, d)
    i64 = bigger_bird_route(q, k, R, front=front, window=window, scale=d ** -0.5)
    assert i64.dtype == torch.int64 and i64.shape == (hk, R)
    i32 = torch.empty(hk, R, dtype=torch.int32, device=DEV)
    _ops.decode_route_(q, k, front=front, window=window, scale=d ** -0.5, k_route=R, idx_out=i32)
    assert torch.equal(i64, i32.long())
    assert bool((i64[:, 1:] > i64[:, :-1]).all())
