"""Fused RMSNorm for the B200 whole-model path (opt-in; not a reference module).

HF's LlamaRMSNorm upcasts its input to fp32 and runs five elementwise/reduction kernels over
[n, hidden] (two fp32 temporaries; the reference bounds them by running the norm in chunks,
``modal_rd/mlp_chunk.py:36-40``). ``bb_rmsnorm`` reads each row once and writes it once, with
the same arithmetic (fp32 mean of squares, fp32 scale, rounded to the dtype, times the weight);
only the order of the fp32 sum differs, so the normalised value is within one ulp of HF's before
the weight multiply (two after it at most; over 99 % of outputs are bit-identical in the tests),
not bit-identical, which is why this is separate from ``install_chunked_mlp``. With ``install_inplace_residual``
the post-attention norm also absorbs the residual add before it (``x += attn_out`` rounded as
torch's ``add_``, then the norm, in one pass).
"""
from __future__ import annotations

import types

from . import _ops

__all__ = ["install_fused_rmsnorm"]


def _forward(self, hidden_states):
    x = hidden_states
    if x.is_cuda and x.dtype == self.weight.dtype and x.stride(-1) == 1 and (x.shape[-1] * x.element_size()) % 16 == 0:
        return _ops.rmsnorm_(x, self.weight, self.variance_epsilon)
    return self._unfused_forward(x)


def _fused_add(self, hidden_states, residual):
    """hidden_states += residual (in place), then the norm of the sum."""
    x = hidden_states
    if x.is_cuda and x.dtype == self.weight.dtype and x.is_contiguous() and residual.is_contiguous():
        return _ops.rmsnorm_(x, self.weight, self.variance_epsilon, residual=residual)
    x.add_(residual)
    return self(x)


def _patch(norm):
    if not hasattr(norm, "_unfused_forward"):
        norm._unfused_forward = norm.forward
    norm.forward = types.MethodType(_forward, norm)
    norm.fused_add = types.MethodType(_fused_add, norm)


def install_fused_rmsnorm(model):
    """Every decoder layer's two RMSNorms and the final norm run as one fused kernel on CUDA
    (other inputs use the module's own forward); idempotent."""
    for layer in model.model.layers:
        _patch(layer.input_layernorm)
        _patch(layer.post_attention_layernorm)
    _patch(model.model.norm)
    return model
