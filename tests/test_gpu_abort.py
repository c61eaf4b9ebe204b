"""The abort path of the attention kernels' bounded waits, on the GPU, without a GPU fault.

Every wait of a tcgen05 attention CTA on another warp's progress is bounded. The test hook
``bb_debug_stall_attention`` makes the MMA warp of every CTA wait for a barrier that nothing
completes, and ``bb_set_wait_limit_ns`` shortens the limit: the wait runs out, the CTA records a
fault code, its other warps leave their loops, in-flight copies are drained and tensor memory is
freed; the other CTAs of the launch see the launch's abort serial and leave at once. The host then
reads the fault code, and the next normal launch on the same context must be correct (it would
stall in ``tcgen05.alloc`` if an aborted CTA had kept its tensor memory).
"""
import ctypes as C
import time

import numpy as np
import pytest
import torch

from oracle import bigbird_oracle as orc

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _fault(L):
    code = C.c_int(-1)
    from utmist_bigger_bird_b200 import _lib
    _lib.check(L.bb_device_fault(C.byref(code)), "device_fault")
    return code.value


def _inputs(h, gq, n, seed):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(h, n, 128, generator=g) * 0.3).to(torch.bfloat16)
    k = torch.randn(h // gq, n, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(h // gq, n, 128, generator=g).to(torch.bfloat16)
    idx = torch.stack([torch.randperm(n - 400, generator=g)[:96] + 64 for _ in range(h)]).sort(-1).values.int()
    return q, k, v, idx[:, None]


@pytest.mark.parametrize("h,gq,n", [(32, 4, 8192), (4, 1, 2048)], ids=["pair_7_waves", "single_head"])
def test_stalled_wait_aborts_and_next_launch_is_correct(h, gq, n):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from utmist_bigger_bird_b200 import _lib, bigger_bird_flash
    L = _lib.lib()
    q, k, v, idx = (t.to(DEV) for t in _inputs(h, gq, n, seed=h + n))
    kw = dict(front=64, window=256, num_heads=h, kv_groups=gq, scale=128 ** -0.5)
    bigger_bird_flash(q, k, v, idx, **kw)          # warm-up: library loaded, maps encoded
    torch.cuda.synchronize()
    assert _fault(L) == 0
    limit_ns = 50_000_000
    _lib.check(L.bb_set_wait_limit_ns(limit_ns), "set_wait_limit_ns")
    _lib.check(L.bb_debug_stall_attention(1), "debug_stall_attention")
    try:
        t0 = time.perf_counter()
        aborted = bigger_bird_flash(q, k, v, idx, **kw)
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
    finally:
        _lib.check(L.bb_debug_stall_attention(0), "debug_stall_attention")
        _lib.check(L.bb_set_wait_limit_ns(2_000_000_000), "set_wait_limit_ns")
    code = _fault(L)
    assert code != 0, "the stalled wait did not record a fault code"
    # Every CTA left through its abort path: no P.V was issued, so every output row is zero.
    assert torch.count_nonzero(aborted) == 0
    # With 128 query rows and 2 heads per CTA the grid has (n / 128) * (h / 2) CTAs (7 waves of
    # 148 for the pair case); without the launch-wide abort each wave would wait out the limit.
    assert elapsed < 0.5, f"abort took {elapsed:.3f} s"
    # The context is usable and the kernels are correct again.
    out = bigger_bird_flash(q, k, v, idx, **kw)
    torch.cuda.synchronize()
    assert _fault(L) == 0
    rows = np.unique(np.concatenate([np.arange(0, n, 97), np.arange(n - 3, n)]))
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    want = orc.flash(f(q), f(k), f(v), idx.cpu().numpy(), rows=rows, **kw)
    err = np.abs(f(out)[:, rows] - want)
    assert err.max() <= 2e-2 and err.mean() <= 2e-3, (err.max(), err.mean())

