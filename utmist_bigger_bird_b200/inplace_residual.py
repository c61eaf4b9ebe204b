"""In-place residual adds in the Llama decoder layers (drop-in for
``modal_rd/inplace_residual.py``; an exact memory saver for long prefill).

HF's decoder layer computes ``residual + attn_out`` and ``residual + mlp_out`` into new [n, hidden]
tensors while its input is still referenced (and the model keeps ``inputs_embeds`` alive for the
whole layer loop). Adding in place into the layer's input makes the embedding output the one
residual-stream buffer of every layer: two [n, hidden] tensors fewer at the prefill peak
(~1 GB each at 128K tokens of a 4096-wide model). The adds are the same ops, so results are
bit-identical. The layer's input tensor is modified: do not pass ``inputs_embeds`` that are still
needed, or ask for ``output_hidden_states`` (they would alias). Inference only.
"""
from __future__ import annotations

import types

__all__ = ["install_inplace_residual"]


def _forward(self, hidden_states, attention_mask=None, position_ids=None, past_key_values=None, use_cache=False,
             position_embeddings=None, **kwargs):
    """LlamaDecoderLayer.forward with the two residual adds in place (inplace_residual.py:17-26)."""
    h = self.input_layernorm(hidden_states)
    h, _ = self.self_attn(hidden_states=h, attention_mask=attention_mask, position_ids=position_ids,
                          past_key_values=past_key_values, use_cache=use_cache,
                          position_embeddings=position_embeddings, **kwargs)
    fused = getattr(self.post_attention_layernorm, "fused_add", None)  # install_fused_rmsnorm
    if fused is not None:
        normed = fused(hidden_states, h)
    else:
        hidden_states.add_(h)
        normed = self.post_attention_layernorm(hidden_states)
    del h
    hidden_states.add_(self.mlp(normed))
    return hidden_states


def install_inplace_residual(model):
    """Patch every decoder layer's forward; idempotent (inplace_residual.py:29-33)."""
    for layer in model.model.layers:
        layer.forward = types.MethodType(_forward, layer)
    return model
