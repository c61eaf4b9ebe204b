"""Sequence-chunked MLP and RMSNorm for long-context prefill (drop-in for
``modal_rd/mlp_chunk.py``).

A Llama MLP at ~128K tokens materialises gate / up / activation tensors of [n, intermediate]
(~3.7 GB each in bf16 for Llama-3-8B), and an RMSNorm upcasts its whole input to fp32 with two
[n, hidden] fp32 temporaries. All of them are position-wise, so running them over slices of
``chunk`` tokens is exact and bounds those transients.

On CUDA, a SwiGLU MLP (``gate_proj`` / ``up_proj`` / ``down_proj`` without bias, SiLU activation)
runs its chunks as: the gate and up projections into two [chunk, intermediate] buffers shared by
every chunk of the call (cuBLAS GEMMs), the activation and product fused in place into the gate
buffer by ``bb_silu_mul`` (one pass instead of two, one [chunk, I] transient fewer), and the down
projection written straight into the output slice (no per-chunk result tensor and copy). Every op
has the shapes and roundings of HF's, so the result is bit-identical to the HF forward on the same
chunks. Other MLPs (biases, other activations, CPU tensors) and the norms run their own forward on
each chunk, as ``modal_rd/mlp_chunk.py:19-26`` does.
"""
from __future__ import annotations

import torch

from . import _ops

__all__ = ["install_chunked_mlp"]


def _is_swiglu(mlp) -> bool:
    # gate/up/down with a `weight` and no bias (nn.Linear, or the tensor-parallel blocks of
    # sharding.shard_llama, whose down projection sums over the ranks in `all_reduce_`).
    projs = [getattr(mlp, n, None) for n in ("gate_proj", "up_proj", "down_proj")]
    if any(p is None or getattr(p, "bias", None) is not None or not hasattr(p, "weight") for p in projs):
        return False
    return type(getattr(mlp, "act_fn", None)).__name__ in ("SiLU", "SiLUActivation")


def _swiglu_chunked(mlp, chunk: int, base):
    def forward(x):
        if not x.is_cuda:
            return _generic(base, chunk)(x)
        wg, wu, wd = mlp.gate_proj.weight, mlp.up_proj.weight, mlp.down_proj.weight
        n = x.shape[-2]
        step = chunk if 0 < chunk < n else n
        lead = x.shape[:-2]
        inter = wg.shape[0]
        out = torch.empty((*lead, n, wd.shape[0]), dtype=x.dtype, device=x.device)
        per_row = inter
        for b in lead:
            per_row *= b
        gbuf = torch.empty(per_row * step, dtype=x.dtype, device=x.device)
        ubuf = torch.empty_like(gbuf)
        for s in range(0, n, step):
            e = min(n, s + step)
            xs = x[..., s:e, :]
            g = gbuf[: per_row * (e - s)].view(*lead, e - s, inter)
            u = ubuf[: per_row * (e - s)].view(*lead, e - s, inter)
            torch.matmul(xs, wg.t(), out=g)
            torch.matmul(xs, wu.t(), out=u)
            _ops.silu_mul_(g, u)
            dst = out[..., s:e, :]
            if dst.is_contiguous():  # batch 1: straight into the output rows
                torch.matmul(g, wd.t(), out=dst)
            else:
                dst.copy_(torch.matmul(g, wd.t()))
        reduce = getattr(mlp.down_proj, "all_reduce_", None)  # tensor-parallel down projection
        return reduce(out) if reduce is not None else out

    return forward


def _generic(base, chunk: int):
    """``base`` over consecutive token slices of at most ``chunk`` rows, written into one output
    buffer whose trailing size comes from the first slice's result."""
    def forward(x):
        n = x.shape[-2]
        if n <= chunk:
            return base(x)
        pieces = x.split(chunk, dim=-2)
        head = base(pieces[0])
        out = head.new_empty((*head.shape[:-2], n, head.shape[-1]))
        out.narrow(-2, 0, head.shape[-2]).copy_(head)
        done = head.shape[-2]
        del head
        for piece in pieces[1:]:
            out.narrow(-2, done, piece.shape[-2]).copy_(base(piece))
            done += piece.shape[-2]
        return out

    return forward


def _chunk(module, chunk: int, native: bool = False):
    base = getattr(module, "_unchunked_forward", module.forward)
    module._unchunked_forward = base
    if chunk <= 0:
        module.forward = base
        return
    module.forward = _swiglu_chunked(module, chunk, base) if native and _is_swiglu(module) else _generic(base, chunk)


def install_chunked_mlp(model, chunk: int = 8192, norms: bool = True):
    """Wrap every decoder layer's MLP (and, with ``norms``, its RMSNorms and the final norm);
    idempotent. ``chunk <= 0`` restores the original forwards (modal_rd/mlp_chunk.py:31-41)."""
    for layer in model.model.layers:
        _chunk(layer.mlp, chunk, native=True)
        if norms:
            _chunk(layer.input_layernorm, chunk)
            _chunk(layer.post_attention_layernorm, chunk)
    if norms:
        _chunk(model.model.norm, chunk)
    return model
