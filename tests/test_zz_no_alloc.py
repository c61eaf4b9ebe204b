"""bb_routes_noalloc: routing for callers that cannot allocate device memory.

Some hosts reserve the whole GPU for their own memory pool, or reach this library through an
FFI without any device allocator, so they cannot pass a fresh workspace to bb_routes. The
no-allocation entry point keeps its scratch in a fixed array inside the library. This test calls
it through the C ABI twice in a row and checks both results against bb_routes (same kernels, so
the routes and column scores must be identical), and checks that an oversized request is
rejected before anything runs. The file name makes pytest collect it last.
"""
import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu


def _args(q, k, qpos, out_idx, out_col, budget):
    from utmist_bigger_bird_b200 import _lib
    H, n, d = q.shape
    return _lib.RoutesArgs(q=q.data_ptr(), sq_h=q.stride(0), sq_t=q.stride(1),
                           k=k.data_ptr(), sk_h=k.stride(0), sk_t=k.stride(1), qpos=qpos.data_ptr(),
                           heads=H, kv_heads=k.shape[0], n=n, d=d, r=qpos.numel(), sink=64, window=2048,
                           budget=budget, scaling=d ** -0.5, pool=_lib.BB_POOL_MEAN, dtype=_lib.BB_BF16,
                           out_idx=out_idx.data_ptr(), so_h=budget,
                           out_col=None if out_col is None else out_col.data_ptr())


def test_routes_noalloc_matches_workspace_entry_point():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from utmist_bigger_bird_b200 import _lib
    L = _lib.lib()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    H, hk, n, d, budget = 32, 8, 16384, 128, 256
    qpos = torch.arange(n - 64, n, device=dev)
    results = []
    for seed in (0, 1):                      # two calls in a row, different inputs
        # call 0 keeps the column scores in the scratch array too; call 1 also returns them
        keep_col = seed == 1
        g = torch.Generator(device=dev).manual_seed(seed)
        q = torch.randn(H, n, d, device=dev, generator=g).to(torch.bfloat16)
        k = torch.randn(hk, n, d, device=dev, generator=g).to(torch.bfloat16)
        want_idx = torch.empty(H, budget, dtype=torch.int32, device=dev)
        want_col = torch.empty(H, n, dtype=torch.float32, device=dev) if keep_col else None
        a = _args(q, k, qpos, want_idx, want_col, budget)
        nbytes = C.c_size_t(0)
        _lib.check(L.bb_routes_workspace_size(C.byref(a), C.byref(nbytes)), "routes")
        ws = torch.empty(nbytes.value, dtype=torch.uint8, device=dev)
        _lib.check(L.bb_routes(C.byref(a), C.c_void_p(ws.data_ptr()), nbytes.value, stream), "routes")
        got_idx = torch.full((H, budget), -7, dtype=torch.int32, device=dev)
        got_col = torch.full((H, n), float("nan"), dtype=torch.float32, device=dev) if keep_col else None
        b = _args(q, k, qpos, got_idx, got_col, budget)
        _lib.check(L.bb_routes_noalloc(C.byref(b), stream), "routes_noalloc")
        torch.cuda.synchronize(dev)
        assert torch.equal(got_idx, want_idx), f"call {seed}: routes differ"
        if keep_col:
            assert torch.equal(got_col, want_col), f"call {seed}: column scores differ"
        assert (got_idx[:, 1:] > got_idx[:, :-1]).all()
        results.append(got_idx.clone())
    assert not torch.equal(results[0], results[1])   # the second call did not reuse stale output

    # A request larger than the fixed scratch is refused with a clear error, before any launch.
    big = _lib.RoutesArgs(heads=32, kv_heads=8, n=1 << 20, d=128, r=64, sink=64, window=2048, budget=256,
                          scaling=0.088, dtype=_lib.BB_BF16)
    status = L.bb_routes_noalloc(C.byref(big), stream)
    assert status == _lib.BB_ERR_WORKSPACE
    msg = L.bb_last_error().decode()
    assert "scratch" in msg and str(24 << 20) in msg
