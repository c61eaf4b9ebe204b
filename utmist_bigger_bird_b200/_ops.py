"""torch-tensor wrappers over the C ABI (device pointers, element strides, current stream).

Every function launches on ``torch.cuda.current_stream()`` and returns without synchronising.
Scratch memory comes from torch's caching allocator and is passed to the library explicitly.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib

_DT = {torch.float16: _lib.BB_F16, torch.bfloat16: _lib.BB_BF16, torch.float32: _lib.BB_F32}


def _stream(t: torch.Tensor):
    return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _rows_ok(t: torch.Tensor) -> bool:
    """Innermost stride 1 and every row on a 16-byte boundary (the kernels' load granularity)."""
    es = t.element_size()
    return (t.stride(-1) == 1 or t.shape[-1] == 1) and t.data_ptr() % 16 == 0 and all(
        (s * es) % 16 == 0 for s in t.stride()[:-1])


def rows_view(t: torch.Tensor) -> torch.Tensor:
    """``t`` itself when the kernels can read it in place, else a contiguous copy."""
    return t if _rows_ok(t) else t.contiguous()


def _workspace(nbytes: int, device) -> torch.Tensor | None:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device) if nbytes else None


def rope_inplace_(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [B, H, T, D] (any strides with innermost 1), cos/sin [B or 1, T, D] -> x rotated in place."""
    if not x.is_cuda:
        raise ValueError("rope_inplace requires CUDA tensors")
    if x.dtype not in _DT or cos.dtype != x.dtype or sin.dtype != x.dtype:
        raise ValueError("rope_inplace: x, cos and sin must share one of f16/bf16/f32")
    if x.ndim != 4 or cos.ndim != 3 or cos.shape != sin.shape or cos.stride() != sin.stride():
        raise ValueError("rope_inplace: x [B,H,T,D] and cos/sin [B,T,D] expected")
    B, H, T, D = x.shape
    if cos.shape[-2:] != (T, D) or cos.shape[0] not in (1, B):
        raise ValueError("rope_inplace: cos/sin do not match x")
    if x.stride(-1) != 1 or cos.stride(-1) != 1:
        raise ValueError("rope_inplace: innermost stride must be 1")
    scb = 0 if cos.shape[0] == 1 else cos.stride(0)
    _lib.check(_lib.lib().bb_rope_inplace(_ptr(x), _DT[x.dtype], B, H, T, D, x.stride(0), x.stride(1),
                                          x.stride(2), _ptr(cos), _ptr(sin), scb, cos.stride(1),
                                          _stream(x)), "rope_inplace")
    return x


def routes_(q: torch.Tensor, k: torch.Tensor, qpos: torch.Tensor, *, sink: int, window: int,
            budget: int, scaling: float, pool: str = "mean", out_col: torch.Tensor | None = None):
    """q [H, n, d], k [Hk, n, d] (post-RoPE), qpos [r] int64 -> int32 [H, budget] sorted."""
    if q.dtype not in (torch.float16, torch.bfloat16) or k.dtype != q.dtype:
        raise ValueError("routes requires CUDA FP16/BF16 q and k")
    q, k = rows_view(q), rows_view(k)
    qpos = qpos.to(device=q.device, dtype=torch.int64).contiguous()
    H, n, d = q.shape
    out = torch.empty((H, budget), dtype=torch.int32, device=q.device)
    a = _lib.RoutesArgs(q=q.data_ptr(), sq_h=q.stride(0), sq_t=q.stride(1),
                        k=k.data_ptr(), sk_h=k.stride(0), sk_t=k.stride(1), qpos=qpos.data_ptr(),
                        heads=H, kv_heads=k.shape[0], n=n, d=d, r=qpos.numel(), sink=sink,
                        window=window, budget=budget, scaling=scaling,
                        pool=_lib.BB_POOL_MAX if pool == "max" else _lib.BB_POOL_MEAN,
                        dtype=_DT[q.dtype], out_idx=out.data_ptr(), so_h=max(budget, 1),
                        out_col=out_col.data_ptr() if out_col is not None else None)
    L = _lib.lib()
    nbytes = C.c_size_t(0)
    _lib.check(L.bb_routes_workspace_size(C.byref(a), C.byref(nbytes)), "routes")
    ws = _workspace(nbytes.value, q.device)
    _lib.check(L.bb_routes(C.byref(a), _ptr(ws), nbytes.value, _stream(q)), "routes")
    return out


def flash_(q, k, v, idx, out, *, front, window, num_heads, kv_groups, route_chunk, scale,
           token_mask=None, row_begin=0, row_end=None):
    """Launch the sparse flash kernel. q [BH,T,D], k/v [BH/g,N,D], idx [BH,G,K] int32,
    out [BH,T,D] (written on rows [row_begin, row_end))."""
    bh, t, d = q.shape
    row_end = t if row_end is None else row_end
    q, k, v = rows_view(q), rows_view(k), rows_view(v)
    if out.stride(-1) != 1:
        raise ValueError("out must have innermost stride 1")
    G, K = idx.shape[1], idx.shape[2]
    a = _lib.FlashArgs(q=q.data_ptr(), sq_h=q.stride(0), sq_t=q.stride(1),
                       k=k.data_ptr(), sk_h=k.stride(0), sk_t=k.stride(1),
                       v=v.data_ptr(), sv_h=v.stride(0), sv_t=v.stride(1),
                       idx=idx.data_ptr() if idx.numel() else None,
                       si_h=idx.stride(0), si_g=idx.stride(1), si_k=idx.stride(2),
                       token_mask=token_mask.data_ptr() if token_mask is not None else None,
                       sm_b=token_mask.stride(0) if token_mask is not None else 0,
                       sm_t=token_mask.stride(1) if token_mask is not None else 0,
                       out=out.data_ptr(), so_h=out.stride(0), so_t=out.stride(1),
                       bh=bh, t=t, n=k.shape[1], d=d, num_heads=num_heads, kv_groups=kv_groups,
                       front=front, window=window, route_k=K, route_groups=G, route_chunk=route_chunk,
                       row_begin=row_begin, row_end=row_end, scale=scale, dtype=_DT[q.dtype])
    L = _lib.lib()
    nbytes = C.c_size_t(0)
    _lib.check(L.bb_flash_workspace_size(C.byref(a), C.byref(nbytes)), "bigger_bird_flash")
    ws = _workspace(nbytes.value, q.device)
    _lib.check(L.bb_flash(C.byref(a), _ptr(ws), nbytes.value, _stream(q)), "bigger_bird_flash")
    return out


def sparse_prefill_(q, k, v, qpos, out, out_idx, *, sink, window, budget, exact_tail, scaling,
                    pool="mean", vertical_scope=0, scope_chunk=4096, cos=None, sin=None):
    """One C call for the whole layer: [RoPE] + routes + main pass + exact tail.
    q [H,n,d], k/v [Hk,n,d], out [H,n,d], out_idx [H,budget] int32, cos/sin [n,d] or None."""
    H, n, d = q.shape
    if cos is not None and (cos.stride(-1) != 1 or sin.stride() != cos.stride()):
        raise ValueError("cos/sin must share strides with innermost stride 1")
    qpos = qpos.to(device=q.device, dtype=torch.int64).contiguous()
    a = _lib.PrefillArgs(q=q.data_ptr(), sq_h=q.stride(0), sq_t=q.stride(1),
                         k=k.data_ptr(), sk_h=k.stride(0), sk_t=k.stride(1),
                         v=v.data_ptr(), sv_h=v.stride(0), sv_t=v.stride(1),
                         cos=cos.data_ptr() if cos is not None else None,
                         sin=sin.data_ptr() if sin is not None else None,
                         sc_t=cos.stride(0) if cos is not None else 0,
                         qpos=qpos.data_ptr(), out=out.data_ptr(), so_h=out.stride(0), so_t=out.stride(1),
                         out_idx=out_idx.data_ptr(), si_h=max(budget, 1),
                         heads=H, kv_heads=k.shape[0], n=n, d=d, r=qpos.numel(), sink=sink,
                         window=window, budget=budget, exact_tail=exact_tail,
                         vertical_scope=vertical_scope, scope_chunk=scope_chunk, scaling=scaling,
                         pool=_lib.BB_POOL_MAX if pool == "max" else _lib.BB_POOL_MEAN, dtype=_DT[q.dtype])
    L = _lib.lib()
    nbytes = C.c_size_t(0)
    _lib.check(L.bb_sparse_prefill_workspace_size(C.byref(a), C.byref(nbytes)), "sparse_prefill")
    ws = _workspace(nbytes.value, q.device)
    _lib.check(L.bb_sparse_prefill(C.byref(a), _ptr(ws), nbytes.value, _stream(q)), "sparse_prefill")
    return out


def kv_evict_(idx: torch.Tensor | None, col: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
              sink: int, window: int, keep: int, pool: int = 0, pool_back: int = 0):
    """KV eviction (RDAttention.evict, reference modal_rd/attention.py:226-259) in one C call.

    idx [H, budget] int32 routes (or None), col [H, n] fp32 column scores, k/v [Hk, n, d] ->
    (k_kept [Hk, L, d], v_kept [Hk, L, d], pos [Hk, L] int64) with L = sink + keep + window."""
    if not (k.is_cuda and v.is_cuda and col.is_cuda):
        raise ValueError("kv_evict requires CUDA tensors")
    if k.dtype not in _DT or v.dtype != k.dtype or col.dtype != torch.float32:
        raise ValueError("kv_evict: k and v must share one of f16/bf16/f32; col must be float32")
    k, v = rows_view(k), rows_view(v)
    col = col if col.stride(-1) == 1 else col.contiguous()
    Hk, n, d = k.shape
    H = col.shape[0]
    L = sink + keep + window
    out_k = torch.empty((Hk, L, d), dtype=k.dtype, device=k.device)
    out_v = torch.empty((Hk, L, d), dtype=v.dtype, device=v.device)
    pos = torch.empty((Hk, L), dtype=torch.int64, device=k.device)
    if idx is not None:
        idx = idx.to(dtype=torch.int32)
        idx = idx if idx.stride(-1) == 1 else idx.contiguous()
    a = _lib.EvictArgs(col=col.data_ptr(), sc_h=col.stride(0),
                       idx=idx.data_ptr() if idx is not None and idx.numel() else None,
                       si_h=idx.stride(0) if idx is not None else 0,
                       budget=idx.shape[-1] if idx is not None else 0,
                       k=k.data_ptr(), sk_h=k.stride(0), sk_t=k.stride(1),
                       v=v.data_ptr(), sv_h=v.stride(0), sv_t=v.stride(1),
                       out_k=out_k.data_ptr(), sok_h=out_k.stride(0), sok_t=out_k.stride(1),
                       out_v=out_v.data_ptr(), sov_h=out_v.stride(0), sov_t=out_v.stride(1),
                       out_pos=pos.data_ptr(), heads=H, kv_heads=Hk, n=n, d=d, sink=sink,
                       window=window, keep=keep, pool=pool, pool_back=pool_back, dtype=_DT[k.dtype])
    L_ = _lib.lib()
    nbytes = C.c_size_t(0)
    _lib.check(L_.bb_kv_evict_workspace_size(C.byref(a), C.byref(nbytes)), "kv_evict")
    ws = _workspace(nbytes.value, k.device)
    _lib.check(L_.bb_kv_evict(C.byref(a), _ptr(ws), nbytes.value, _stream(k)), "kv_evict")
    return out_k, out_v, pos


def _n_arg(n, cap, device):
    """(host n, device pointer or None, keep-alive tensor) for a cache length given as None, an int
    or a 1-element GPU integer tensor (read by the kernels at run time)."""
    if n is None:
        return cap, None, None
    if isinstance(n, torch.Tensor):
        t = n.reshape(-1)[:1]
        if t.dtype != torch.int64 or not t.is_contiguous() or t.device != device:
            t = t.to(device=device, dtype=torch.int64).contiguous()
        return cap, t.data_ptr(), t
    return int(n), None, None


def decode_(q, k, v, idx, out, *, front, window, scale, n=None, splits=0):
    """One-token sparse decode: q [H, d], k/v [Hkv, cap, d] (cache views), idx [Hkv or H, R] int32
    or int64 (or None), out [H, d]. ``n``: cache length (None = cap, int, or 1-element GPU tensor)."""
    H, d = q.shape
    hk, cap, _ = k.shape
    if k.stride(-1) != 1 or v.stride(-1) != 1 or q.stride(-1) != 1 or out.stride(-1) != 1:
        raise ValueError("decode: innermost strides must be 1")
    n_host, n_ptr, keep = _n_arg(n, cap, q.device)
    R = idx.shape[1] if idx is not None else 0
    a = _lib.DecodeArgs(q=q.data_ptr(), sq_h=q.stride(0), k=k.data_ptr(), sk_h=k.stride(0), sk_t=k.stride(1),
                        v=v.data_ptr(), sv_h=v.stride(0), sv_t=v.stride(1),
                        idx=idx.data_ptr() if R else None, si_r=idx.stride(0) if R else 0,
                        route_rows=idx.shape[0] if idx is not None else hk, route_k=R,
                        n=n_host, n_dev=n_ptr, cap=cap, heads=H, kv_heads=hk, d=d, front=front, window=window,
                        scale=scale, splits=splits or 0, out=out.data_ptr(), so_h=out.stride(0),
                        dtype=_DT[q.dtype], idx_i64=int(R > 0 and idx.dtype == torch.int64))
    L = _lib.lib()
    nbytes = C.c_size_t(0)
    _lib.check(L.bb_decode_workspace_size(C.byref(a), C.byref(nbytes)), "bigger_bird_decode")
    ws = _workspace(nbytes.value, q.device)
    _lib.check(L.bb_decode(C.byref(a), _ptr(ws), nbytes.value, _stream(q)), "bigger_bird_decode")
    del keep
    return out


def decode_route_(q, k, *, front, window, scale, n=None, k_route=0, probs=None, idx_out=None, splits=0):
    """Decode routing: pooled probabilities [Hkv, cap] fp32 into ``probs`` (optional) and the
    ``k_route`` most probable keys per KV head into ``idx_out`` [Hkv, k_route] int32 or int64 (optional)."""
    H, d = q.shape
    hk, cap, _ = k.shape
    if k.stride(-1) != 1 or q.stride(-1) != 1:
        raise ValueError("decode_route: innermost strides must be 1")
    n_host, n_ptr, keep = _n_arg(n, cap, q.device)
    a = _lib.DecodeArgs(q=q.data_ptr(), sq_h=q.stride(0), k=k.data_ptr(), sk_h=k.stride(0), sk_t=k.stride(1),
                        route_rows=hk, route_k=k_route, n=n_host, n_dev=n_ptr, cap=cap, heads=H, kv_heads=hk,
                        d=d, front=front, window=window, scale=scale, splits=splits or 0,
                        out_probs=probs.data_ptr() if probs is not None else None,
                        out_idx=idx_out.data_ptr() if idx_out is not None else None,
                        so_i=idx_out.stride(0) if idx_out is not None else 0, dtype=_DT[q.dtype],
                        out_idx_i64=int(idx_out is not None and idx_out.dtype == torch.int64))
    L = _lib.lib()
    nbytes = C.c_size_t(0)
    _lib.check(L.bb_decode_route_workspace_size(C.byref(a), C.byref(nbytes)), "bigger_bird_route")
    ws = _workspace(nbytes.value, q.device)
    _lib.check(L.bb_decode_route(C.byref(a), _ptr(ws), nbytes.value, _stream(q)), "bigger_bird_route")
    del keep


def silu_mul_(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """gate <- act(gate) * up in place (SwiGLU of a Llama MLP chunk; bit-identical to HF's
    ``act_fn(gate) * up``). gate/up: [..., I] CUDA tensors of one dtype, rows of stride >= I."""
    if not gate.is_cuda or gate.dtype not in _DT or up.dtype != gate.dtype or up.device != gate.device:
        raise ValueError("silu_mul_ requires CUDA gate/up of one dtype among fp16, bf16, fp32")
    if gate.shape != up.shape:
        raise ValueError(f"silu_mul_: shapes {tuple(gate.shape)} and {tuple(up.shape)} differ")
    cols = gate.shape[-1]
    g2, u2 = gate.reshape(-1, cols), up.reshape(-1, cols)
    if g2.data_ptr() != gate.data_ptr() or g2.stride(-1) != 1 or u2.stride(-1) != 1:
        raise ValueError("silu_mul_: gate must be viewable as rows with unit inner stride (in place)")
    if g2.shape[0] > 1 and (g2.stride(0) < cols or u2.stride(0) < cols):
        raise ValueError("silu_mul_: overlapping rows")
    _lib.check(_lib.lib().bb_silu_mul(_ptr(g2), max(g2.stride(0), cols), _ptr(u2), max(u2.stride(0), cols),
                                      g2.shape[0], cols, _DT[gate.dtype], _stream(gate)), "silu_mul")
    return gate


def embed_gather(table: torch.Tensor, ids: torch.Tensor, *, out: torch.Tensor | None = None) -> torch.Tensor:
    """Rows ``table[ids]`` gathered by a kernel on ``ids.device``; ``table`` may stay in page-locked
    host memory (read over the host link) or be on that device. Raises IndexError for ids out of
    range, like ``F.embedding``."""
    if not ids.is_cuda or ids.dtype != torch.int64:
        raise ValueError("embed_gather: ids must be a CUDA int64 tensor")
    if table.dim() != 2 or not table.is_contiguous():
        raise ValueError("embed_gather: table must be a contiguous [vocab, hidden] tensor")
    if not table.is_cuda and not table.is_pinned():
        raise ValueError("embed_gather: a host table must be pinned (page-locked)")
    vocab, hidden = table.shape
    ids_c = ids.contiguous()
    if out is None:
        out = torch.empty((*ids.shape, hidden), dtype=table.dtype, device=ids.device)
    elif out.shape != (*ids.shape, hidden) or out.dtype != table.dtype or not out.is_contiguous():
        raise ValueError("embed_gather: out must be a contiguous [*ids.shape, hidden] tensor of the table dtype")
    bad = torch.zeros(1, dtype=torch.int32, device=ids.device)
    _lib.check(_lib.lib().bb_embed_gather(_ptr(table), vocab, hidden * table.element_size(), _ptr(ids_c),
                                          ids_c.numel(), _ptr(out), _ptr(bad), _stream(ids)), "embed_gather")
    if int(bad.item()):
        raise IndexError("index out of range in self")
    return out



def rmsnorm_(x: torch.Tensor, weight: torch.Tensor, eps: float, *, residual: torch.Tensor | None = None,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """``weight * round(x * rsqrt(mean(x^2) + eps))`` over the last dim (LlamaRMSNorm's arithmetic,
    fp32 sum in a different order). With ``residual``, ``x += residual`` in place first (the
    decoder layer's residual add, fused)."""
    if not x.is_cuda or x.dtype not in _DT or weight.dtype != x.dtype or weight.device != x.device:
        raise ValueError("rmsnorm_ requires CUDA x and weight of one dtype among fp16, bf16, fp32")
    cols = x.shape[-1]
    if weight.shape != (cols,) or not weight.is_contiguous():
        raise ValueError("rmsnorm_: weight must be a contiguous [hidden] vector")
    x2 = x.reshape(-1, cols)
    if x2.data_ptr() != x.data_ptr() or x2.stride(-1) != 1:
        raise ValueError("rmsnorm_: x must be viewable as rows with unit inner stride")
    r2 = None
    if residual is not None:
        if residual.shape != x.shape or residual.dtype != x.dtype:
            raise ValueError("rmsnorm_: residual must match x")
        r2 = residual.reshape(-1, cols)
    if out is None:
        out = torch.empty_like(x, memory_format=torch.contiguous_format)
    y2 = out.reshape(-1, cols)
    rows = x2.shape[0]
    _lib.check(_lib.lib().bb_rmsnorm(_ptr(x2), x2.stride(0) if rows > 1 else cols, _ptr(r2),
                                     (r2.stride(0) if rows > 1 else cols) if r2 is not None else 0,
                                     _ptr(weight), _ptr(y2), y2.stride(0) if rows > 1 else cols, rows, cols,
                                     float(eps), _DT[x.dtype], _stream(x)), "rmsnorm")
    return out
