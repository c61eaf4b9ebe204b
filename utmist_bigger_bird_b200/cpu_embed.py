"""Keep the input embedding table in host memory (drop-in for ``modal_rd/cpu_embed.py``).

The Llama-3 table is [128256, 4096] bf16 = 1.05 GB of HBM, but a forward pass reads one row per
token. The table moves to page-locked host memory and the lookup for CUDA ids is one kernel
(``bb_embed_gather``) that reads the n rows straight over the host link into device memory: no
device-to-host copy of the ids, no CPU gather, no staging copy (the reference gathers with
``F.embedding`` on the CPU, pins the rows, then copies them). The rows are bit-identical. The table
is a plain attribute, not a Parameter, so ``model.parameters()`` and ``model.device`` still report
the GPU and HF ``generate`` is unaffected. Ids on the CPU are looked up on the CPU.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _ops

__all__ = ["CPUEmbedding", "install_cpu_embedding"]


class CPUEmbedding(nn.Module):
    """modal_rd/cpu_embed.py:13-25."""

    def __init__(self, embedding):
        super().__init__()
        self.weight_cpu = embedding.weight.detach().to("cpu").contiguous()
        if torch.cuda.is_available():
            self.weight_cpu = self.weight_cpu.pin_memory()
        self.padding_idx = embedding.padding_idx

    def forward(self, input_ids):
        if input_ids.is_cuda:
            return _ops.embed_gather(self.weight_cpu, input_ids.long())
        return F.embedding(input_ids, self.weight_cpu)


def install_cpu_embedding(model):
    """Move ``model.model.embed_tokens`` to page-locked host memory and free its GPU copy;
    idempotent (modal_rd/cpu_embed.py:28-35)."""
    emb = model.model.embed_tokens
    if not isinstance(emb, CPUEmbedding):
        model.model.embed_tokens = CPUEmbedding(emb)
        del emb
        if torch.cuda.is_available():
            torch.cuda.empty_cache()
    return model
