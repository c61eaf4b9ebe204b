"""Whole-model memory savers on the CPU: the host logic of install_chunked_mlp /
install_cpu_embedding / install_inplace_residual (tests/test_mlp_chunk.py,
tests/test_exact_memory_savers.py, tests/test_inplace_residual.py of the reference, on a CPU
model: chunks run the modules' own forwards there) and the C entry points' argument checks."""
import ctypes as C

import pytest
import torch
from transformers import LlamaConfig, LlamaForCausalLM

from utmist_bigger_bird_b200 import (CPUEmbedding, _lib, install_chunked_mlp, install_cpu_embedding,
                                     install_inplace_residual)


def tiny(n_layers=2, dtype=torch.float32):
    cfg = LlamaConfig(vocab_size=512, hidden_size=256, intermediate_size=1024, num_hidden_layers=n_layers,
                      num_attention_heads=8, num_key_value_heads=2, max_position_embeddings=8192)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).to(dtype).eval()


@pytest.mark.parametrize("n,chunk", [(300, 64), (300, 300), (257, 128)])
def test_chunked_mlp_and_norms_cpu(n, chunk):
    model = tiny()
    ids = torch.randint(0, 512, (1, n))
    with torch.inference_mode():
        want = model(ids).logits
        install_chunked_mlp(model, chunk)
        install_chunked_mlp(model, chunk)  # idempotent: wraps the original forward, not the wrapper
        got = model(ids).logits
        install_chunked_mlp(model, 0)
        restored = model(ids).logits
    torch.testing.assert_close(got, want, atol=1e-5, rtol=1e-5)
    assert torch.equal(restored, want)
    layer = model.model.layers[0]
    assert layer.mlp.forward == layer.mlp._unchunked_forward


def test_norms_flag_off_leaves_norms_alone():
    model = tiny(1)
    install_chunked_mlp(model, 64, norms=False)
    assert not hasattr(model.model.norm, "_unchunked_forward")
    assert hasattr(model.model.layers[0].mlp, "_unchunked_forward")


def test_inplace_residual_bit_identical_cpu():
    model = tiny()
    ids = torch.randint(0, 512, (1, 200))
    with torch.inference_mode():
        want = model(ids).logits
        install_inplace_residual(model)
        install_inplace_residual(model)
        got = model(ids).logits
    assert torch.equal(got, want)


def test_cpu_embedding_cpu_ids():
    model = tiny()
    ids = torch.randint(0, 512, (1, 100))
    with torch.inference_mode():
        want = model(ids).logits
        install_cpu_embedding(model)
        install_cpu_embedding(model)
        assert isinstance(model.model.embed_tokens, CPUEmbedding)
        got = model(ids).logits
    assert torch.equal(got, want)
    assert sum(p.numel() for p in model.parameters()) == sum(
        p.numel() for n, p in tiny().named_parameters() if "embed_tokens" not in n)


def test_memory_entry_points_check_arguments():
    L = _lib.lib()
    assert L.bb_silu_mul(None, 0, None, 0, 0, 8, _lib.BB_BF16, None) == 0            # empty: nothing to do
    assert L.bb_silu_mul(None, 8, None, 8, 4, 8, _lib.BB_BF16, None) != 0            # null pointers
    buf = (C.c_uint8 * 256)()
    p = C.cast(buf, C.c_void_p)
    assert L.bb_silu_mul(p, 8, p, 8, 2, 8, 7, None) != 0                             # bad dtype
    assert b"dtype" in L.bb_last_error()
    assert L.bb_silu_mul(p, 4, p, 8, 2, 8, _lib.BB_BF16, None) != 0                  # stride below row length
    assert L.bb_embed_gather(p, 10, 24, p, 1, p, p, None) != 0                         # row not 16-byte multiple
    assert L.bb_embed_gather(p, 0, 16, p, 1, p, p, None) != 0                          # empty vocab
    assert L.bb_embed_gather(p, 10, 16, p, 0, p, p, None) == 0                         # no ids
    assert L.bb_rmsnorm(p, 8, None, 0, p, p, 8, 0, 8, 1e-5, _lib.BB_BF16, None) == 0   # no rows
    assert L.bb_rmsnorm(None, 8, None, 0, p, p, 8, 2, 8, 1e-5, _lib.BB_BF16, None) != 0  # null x
    assert L.bb_rmsnorm(p, 12, None, 0, p, p, 12, 2, 12, 1e-5, _lib.BB_BF16, None) != 0  # rows not 16-byte multiples
    assert L.bb_rmsnorm(p, 8, None, 0, p, p, 8, 2, 8, 1e-5, 9, None) != 0              # bad dtype


def test_python_memory_ops_reject_cpu_tensors():
    from utmist_bigger_bird_b200 import _ops
    g = torch.zeros(4, 8, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        _ops.silu_mul_(g, g.clone())
    with pytest.raises(ValueError):
        _ops.embed_gather(torch.zeros(10, 8), torch.zeros(3, dtype=torch.int64))
