"""C-ABI checks that need no GPU: the library loads, exports every entry point declared in
include/bb_b200.h, its struct layouts match the ctypes mirrors (checked against the header
compiled with gcc), and host-side validation reports the reference's errors."""
import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest
import torch

from utmist_bigger_bird_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "bb_b200.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"BB_API\s+(?:const\s+)?\w+\*?\s+\*?(bb_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    names = declared_functions()
    assert len(names) >= 9, names
    for name in names:
        assert hasattr(L, name), name
        assert name in _lib.EXPORTS, f"{name} has no ctypes prototype"
    assert L.bb_abi_version() == _lib.ABI_VERSION


def test_struct_layouts_match_header(tmp_path):
    structs = {"bb_routes_args": _lib.RoutesArgs, "bb_flash_args": _lib.FlashArgs,
               "bb_prefill_args": _lib.PrefillArgs, "bb_evict_args": _lib.EvictArgs,
               "bb_decode_args": _lib.DecodeArgs}
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", "-o", str(exe), str(src)], check=True)
    got = {}
    for line in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines():
        s, f, v = line.split()
        got[(s, f)] = int(v)
    for cname, py in structs.items():
        assert got[(cname, "size")] == C.sizeof(py), cname
        for fname, _ in py._fields_:
            assert got[(cname, fname)] == getattr(py, fname).offset, (cname, fname)


def _flash_args(**kw):
    base = dict(bh=32, t=100, n=200, d=128, num_heads=32, kv_groups=4, front=64, window=256,
                route_k=8, route_groups=1, route_chunk=256, row_begin=0, row_end=100, scale=0.1, dtype=1)
    base.update(kw)
    return _lib.FlashArgs(**base)


@pytest.mark.parametrize("kw,status,msg", [
    (dict(n=50), 2, "at least as long"),
    (dict(window=0), 1, "window >= 1"),
    (dict(front=-1), 1, "front >= 0"),
    (dict(dtype=2), 3, "f16 or bf16"),
    (dict(d=136), 7, "head_dim"),
    (dict(num_heads=32, kv_groups=5), 2, "multiples"),
    (dict(row_end=101), 1, "row range"),
])
def test_flash_host_validation(kw, status, msg):
    L = _lib.lib()
    nbytes = C.c_size_t(0)
    a = _flash_args(**kw)
    assert L.bb_flash_workspace_size(C.byref(a), C.byref(nbytes)) == status
    assert msg in L.bb_last_error().decode()


def test_flash_workspace_sizes():
    L = _lib.lib()
    nbytes = C.c_size_t(0)
    # main pass of the 128K layer: plenty of CTAs, no key split; the workspace holds only the routed
    # K and V rows gathered once per call ([bh, groups, route_k rounded up to 128, d] bf16 each) and
    # each 128-slot routed tile's smallest position (int32, the area rounded up to 256 bytes)
    a = _flash_args(t=131072, n=131072, window=16384, route_k=512, route_chunk=131072, row_end=131072 - 256)
    want = 2 * a.bh * a.route_groups * 512 * 128 * 2 + -(-a.bh * a.route_groups * 4 * 4 // 256) * 256
    assert L.bb_flash_workspace_size(C.byref(a), C.byref(nbytes)) == 0
    assert nbytes.value == want
    a.route_k = 500  # padded to whole 128-slot tiles
    assert L.bb_flash_workspace_size(C.byref(a), C.byref(nbytes)) == 0
    assert nbytes.value == want
    a.d, a.route_k = 64, 512  # head_dim 64 runs on the mma.sync kernel, which gathers in-kernel
    assert L.bb_flash_workspace_size(C.byref(a), C.byref(nbytes)) == 0 and nbytes.value == 0
    # exact tail: 256 rows over n keys split across the machine -> partials workspace of
    # [splits, bh, t, 128] fp32 plus [splits, bh, t] (max, sum) pairs. The split count minimises whole
    # waves of CTAs (148 SMs without a GPU) times each CTA's key tiles plus ~10 tiles of fixed cost:
    # 9 at 128K (288 CTAs, 2 waves of 114 + 10), 4 at 32K (128 CTAs, 1 wave of 64 + 10).
    for n, splits in ((131072, 9), (32768, 4)):
        a = _flash_args(t=256, n=n, front=0, window=n, route_k=0, route_chunk=n, row_end=256)
        want = splits * a.bh * 256 * 128 * 4 + splits * a.bh * 256 * 8
        assert L.bb_flash_workspace_size(C.byref(a), C.byref(nbytes)) == 0
        assert nbytes.value == want, (n, nbytes.value, want)


def test_routes_host_validation():
    L = _lib.lib()
    nbytes = C.c_size_t(0)
    a = _lib.RoutesArgs(heads=32, kv_heads=8, n=1000, d=128, r=64, sink=64, window=256, budget=128,
                        scaling=0.088, dtype=1)
    assert L.bb_routes_workspace_size(C.byref(a), C.byref(nbytes)) == 0 and nbytes.value > 0
    a.r = 300
    assert L.bb_routes_workspace_size(C.byref(a), C.byref(nbytes)) == 7
    a.r, a.heads = 64, 30
    assert L.bb_routes_workspace_size(C.byref(a), C.byref(nbytes)) == 2
    a.heads, a.budget = 32, 2000
    assert L.bb_routes_workspace_size(C.byref(a), C.byref(nbytes)) == 1
    # a missing workspace is reported, not dereferenced
    a.budget = 16
    assert L.bb_routes(C.byref(a), None, 0, None) == 5
    assert "workspace" in L.bb_last_error().decode()


def test_prefill_workspace_covers_parts():
    L = _lib.lib()
    a = _lib.PrefillArgs(heads=32, kv_heads=8, n=131072, d=128, r=64, sink=64, window=16384, budget=512,
                         exact_tail=256, scope_chunk=4096, scaling=0.088, dtype=1)
    nbytes = C.c_size_t(0)
    assert L.bb_sparse_prefill_workspace_size(C.byref(a), C.byref(nbytes)) == 0
    assert nbytes.value >= 32 * 131072 * 4        # the [H, n] fp32 column scores


def test_python_surface_rejects_cpu_tensors():
    from utmist_bigger_bird_b200 import RDAttention, bigger_bird_flash, rope_inplace
    q = torch.randn(4, 16, 32, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        bigger_bird_flash(q, q[:2], q[:2], torch.full((4, 1, 1), -1, dtype=torch.int32), num_heads=4, kv_groups=2)
    with pytest.raises(ValueError):
        rope_inplace(q[None], torch.ones(1, 16, 32, dtype=torch.bfloat16), torch.ones(1, 16, 32, dtype=torch.bfloat16))
    from types import SimpleNamespace
    base = SimpleNamespace(config=SimpleNamespace(num_attention_heads=4, num_key_value_heads=2), layer_idx=0,
                           head_dim=32, scaling=32 ** -0.5, q_proj=None, k_proj=None, v_proj=None, o_proj=None)
    with pytest.raises(ValueError, match="route_pool"):
        RDAttention(base, route_pool="sum")
    with pytest.raises(ValueError, match="route_queries"):
        RDAttention(base, route_queries="first")
    with pytest.raises(ValueError, match="scope_chunk"):
        RDAttention(base, scope_chunk=100)
    attn = RDAttention(base)
    with pytest.raises(ValueError, match="CUDA"):
        attn.routes(q[None], q[None, :2])


@pytest.mark.parametrize("kw,msg", [
    (dict(sink=60, window=50), "sink + window <= n"),
    (dict(keep=90), "keep must lie"),
    (dict(heads=7), "multiple of kv_heads"),
    (dict(dtype=9), "dtype"),
    (dict(pool=-1), "pool"),
])
def test_kv_evict_host_validation(kw, msg):
    """bb_kv_evict's argument checks run on the host (no device needed)."""
    L = _lib.lib()
    args = dict(heads=8, kv_heads=2, n=100, d=32, sink=8, window=16, keep=20, budget=4, dtype=_lib.BB_BF16)
    args.update(kw)
    a = _lib.EvictArgs(**args)
    nbytes = C.c_size_t(0)
    st = L.bb_kv_evict_workspace_size(C.byref(a), C.byref(nbytes))
    assert st != 0 and msg in L.bb_last_error().decode()


def test_kv_evict_workspace_size():
    L = _lib.lib()
    a = _lib.EvictArgs(heads=32, kv_heads=8, n=131072, d=128, sink=64, window=16384, keep=2048, budget=512,
                       dtype=_lib.BB_BF16)
    nbytes = C.c_size_t(0)
    assert L.bb_kv_evict_workspace_size(C.byref(a), C.byref(nbytes)) == 0
    cells = 8 * 131072
    assert nbytes.value >= cells * (1 + 4 + 4) + 8 * 2048 * 4


@pytest.mark.parametrize("kw,fn,msg", [
    (dict(dtype=_lib.BB_F32), "bb_decode_workspace_size", "fp16 or bf16"),
    (dict(heads=7), "bb_decode_workspace_size", "multiple of kv_heads"),
    (dict(d=136), "bb_decode_workspace_size", "head_dim"),
    (dict(n=5000), "bb_decode_workspace_size", "n must lie"),
    (dict(route_rows=3, route_k=8), "bb_decode_workspace_size", "pooled"),
    (dict(heads=64, kv_heads=2), "bb_decode_workspace_size", "query heads per KV head"),
    (dict(route_k=5000), "bb_decode_route_workspace_size", "k_route"),
])
def test_decode_host_validation(kw, fn, msg):
    """bb_decode / bb_decode_route argument checks run on the host (no device needed)."""
    L = _lib.lib()
    args = dict(heads=32, kv_heads=8, d=128, cap=4096, n=4096, front=64, window=512, route_rows=8, route_k=0,
                scale=0.088, dtype=_lib.BB_BF16)
    args.update(kw)
    a = _lib.DecodeArgs(**args)
    nbytes = C.c_size_t(0)
    assert getattr(L, fn)(C.byref(a), C.byref(nbytes)) != 0
    assert msg in L.bb_last_error().decode()


def test_wait_limit_must_be_positive():
    """bb_set_wait_limit_ns refuses 0 on the host, before touching a device."""
    L = _lib.lib()
    assert L.bb_set_wait_limit_ns(0) == _lib.BB_ERR_ARG
    assert "positive" in L.bb_last_error().decode()


def test_routes_workspace_holds_long_row_topk_scratch():
    """Rows longer than one cluster's shared memory (1M keys) select in two levels: the routing
    workspace grows by the candidate buffers (32 segments x budget positions and values per row,
    plus the second level's picks); at 128K there is no such scratch."""
    L = _lib.lib()

    def ws(n):
        a = _lib.RoutesArgs(heads=32, kv_heads=8, n=n, d=128, r=64, sink=64, window=16384, budget=512,
                            scaling=0.088, dtype=_lib.BB_BF16)
        nbytes = C.c_size_t(0)
        assert L.bb_routes_workspace_size(C.byref(a), C.byref(nbytes)) == 0
        return nbytes.value

    def al(x):
        return (x + 255) // 256 * 256

    n = 1 << 20
    col = al(32 * n * 4)
    cand = al(32 * (n // 32768) * 512 * 4)
    assert ws(n) - ws(n // 2 + 1) > col // 2            # the column scores grow with n
    a = _lib.RoutesArgs(heads=32, kv_heads=8, n=n, d=128, r=64, sink=64, window=16384, budget=0,
                        scaling=0.088, dtype=_lib.BB_BF16)
    no_topk = C.c_size_t(0)
    assert L.bb_routes_workspace_size(C.byref(a), C.byref(no_topk)) == 0
    assert ws(n) - no_topk.value == 2 * cand + al(32 * 512 * 4)
    a.n = 131072
    small = C.c_size_t(0)
    assert L.bb_routes_workspace_size(C.byref(a), C.byref(small)) == 0
    assert ws(131072) == small.value
