"""Whole-model memory savers on the GPU: the fused SwiGLU (bb_silu_mul) and the host-table gather
(bb_embed_gather) against the torch ops they replace, and the reference's own tests of the memory
savers (tests/test_mlp_chunk.py, tests/test_exact_memory_savers.py, tests/test_inplace_residual.py)
on the B200 path: bit-identical results, bounded transients, a lower prefill peak."""
import pytest
import torch
import torch.nn.functional as F
from transformers import DynamicCache, LlamaConfig, LlamaForCausalLM

from utmist_bigger_bird_b200 import (CPUEmbedding, _ops, install, install_chunked_mlp, install_cpu_embedding,
                                     install_inplace_residual)

pytestmark = pytest.mark.gpu
DEV = "cuda"


def tiny(n_layers=2, dtype=torch.bfloat16, hidden=256, inter=1024, heads=8):
    cfg = LlamaConfig(vocab_size=512, hidden_size=hidden, intermediate_size=inter, num_hidden_layers=n_layers,
                      num_attention_heads=heads, num_key_value_heads=2, max_position_embeddings=32768)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).to(DEV, dtype).eval()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("shape", [(300, 1024), (7, 14336), (33, 100)])
def test_silu_mul_bit_identical(dtype, shape):
    g = torch.Generator(device=DEV).manual_seed(1)
    gate = (torch.randn(*shape, device=DEV, generator=g) * 4).to(dtype)
    up = torch.randn(*shape, device=DEV, generator=g).to(dtype)
    want = F.silu(gate) * up
    got = _ops.silu_mul_(gate.clone(), up)
    assert torch.equal(got, want)


def test_silu_mul_strided_rows():
    base = torch.randn(64, 2 * 512, device=DEV).to(torch.bfloat16)
    gate, up = base[:, :512], base[:, 512:]  # rows of stride 1024
    want = F.silu(gate) * up
    _ops.silu_mul_(gate, up)
    assert torch.equal(gate, want)


@pytest.mark.parametrize("n,chunk", [(300, 64), (257, 128), (100, 1000)])
def test_chunked_norms_are_bit_identical(n, chunk):
    model = tiny(1)
    x = torch.randn(1, n, 256, device=DEV, dtype=torch.bfloat16)
    norms = [model.model.layers[0].input_layernorm, model.model.layers[0].post_attention_layernorm, model.model.norm]
    with torch.inference_mode():
        want = [m(x) for m in norms]
        install_chunked_mlp(model, chunk)
        got = [m(x) for m in norms]
        install_chunked_mlp(model, 0)
        restored = [m(x) for m in norms]
    assert all(torch.equal(g, w) for g, w in zip(got, want))
    assert all(torch.equal(r, w) for r, w in zip(restored, want))


@pytest.mark.parametrize("n,chunk", [(300, 64), (300, 300), (300, 1000), (257, 128)])
def test_chunked_mlp_matches_unchunked(n, chunk):
    """tests/test_mlp_chunk.py:16-27 (fp32 model): chunked == unchunked to 1e-5, restore exact."""
    model = tiny(dtype=torch.float32)
    ids = torch.randint(0, 512, (1, n), device=DEV)
    with torch.inference_mode():
        want = model(ids).logits
        install_chunked_mlp(model, chunk)
        got = model(ids).logits
        install_chunked_mlp(model, 0)
        restored = model(ids).logits
    torch.testing.assert_close(got, want, atol=1e-5, rtol=1e-5)
    assert torch.equal(restored, want)


@pytest.mark.parametrize("n,chunk", [(300, 64), (257, 128), (200, 512)])
def test_native_chunked_mlp_equals_hf_per_chunk(n, chunk):
    """bf16: the B200 chunk loop (GEMMs into shared buffers, fused SwiGLU, down projection into the
    output slice) is bit-identical to HF's MLP forward run on the same chunks."""
    model = tiny(1)
    mlp = model.model.layers[0].mlp
    x = torch.randn(1, n, 256, device=DEV, dtype=torch.bfloat16)
    with torch.inference_mode():
        want = torch.cat([mlp(x[:, s:s + chunk]) for s in range(0, n, chunk)], dim=1)
        install_chunked_mlp(model, chunk)
        got = mlp(x)
    assert torch.equal(got, want)


def test_chunking_bounds_mlp_transients():
    """tests/test_mlp_chunk.py:30-47: the [n, intermediate] transients are gone when chunked."""
    n, chunk = 4096, 512
    model = tiny(1, dtype=torch.float32)
    x = torch.randn(1, n, 256, device=DEV)
    mlp = model.model.layers[0].mlp

    def peak():
        torch.cuda.synchronize()
        torch.cuda.reset_peak_memory_stats()
        base = torch.cuda.memory_allocated()
        with torch.inference_mode():
            mlp(x)
        torch.cuda.synchronize()
        return torch.cuda.max_memory_allocated() - base

    full = peak()
    install_chunked_mlp(model, chunk)
    chunked = peak()
    assert full >= 2 * n * 1024 * 4
    assert chunked <= n * 256 * 4 + 2 * chunk * 1024 * 4 + (1 << 20)  # output + two chunk buffers
    assert chunked < full / 4


def test_cpu_embedding_is_bit_identical_and_frees_gpu():
    """tests/test_exact_memory_savers.py:69-82, with the lookup done by the host-table gather."""
    model = tiny()
    ids = torch.randint(0, 512, (1, 300), device=DEV)
    with torch.inference_mode():
        want = model(ids).logits
        gen_want = model.generate(ids[:, :50], max_new_tokens=5, do_sample=False)
    n_gpu = sum(p.numel() for p in model.parameters())
    install_cpu_embedding(model)
    install_cpu_embedding(model)
    emb = model.model.embed_tokens
    assert isinstance(emb, CPUEmbedding) and emb.weight_cpu.device.type == "cpu" and emb.weight_cpu.is_pinned()
    assert sum(p.numel() for p in model.parameters()) == n_gpu - 512 * 256
    assert model.device.type == "cuda"
    with torch.inference_mode():
        got = model(ids).logits
        gen_got = model.generate(ids[:, :50], max_new_tokens=5, do_sample=False)
    assert torch.equal(got, want) and torch.equal(gen_got, gen_want)


def test_embed_gather_rows_and_errors():
    table = torch.randn(1000, 64).to(torch.bfloat16).pin_memory()
    ids = torch.randint(0, 1000, (3, 77), device=DEV)
    got = _ops.embed_gather(table, ids)
    assert torch.equal(got.cpu(), table[ids.cpu()])
    dev_table = table.to(DEV)
    assert torch.equal(_ops.embed_gather(dev_table, ids), dev_table[ids])
    with pytest.raises(IndexError):
        _ops.embed_gather(table, torch.tensor([0, 1000], device=DEV))
    with pytest.raises(IndexError):
        _ops.embed_gather(table, torch.tensor([-1], device=DEV))
    with pytest.raises(ValueError):
        _ops.embed_gather(torch.randn(10, 64), ids)  # pageable host table


@torch.inference_mode()
def _run(model, ids, steps=6):
    cache = DynamicCache(config=model.config)
    out = model(input_ids=ids, past_key_values=cache, use_cache=True)
    logits, nxt, toks = [out.logits.float()], out.logits[0, -1].argmax().view(1, 1), []
    for _ in range(steps):
        o = model(input_ids=nxt, past_key_values=cache, use_cache=True)
        logits.append(o.logits.float())
        nxt = o.logits[0, -1].argmax().view(1, 1)
        toks.append(int(nxt))
    return logits, toks


@pytest.mark.parametrize("arm", [None, "dense_rd", "vs"])
@pytest.mark.parametrize("cpu_embed", [False, True])
def test_inplace_residual_bit_identical(arm, cpu_embed):
    """tests/test_inplace_residual.py:33-47: prefill + 6 decode steps, identical logits and tokens."""
    model = tiny(hidden=256, inter=512, heads=4)
    install_chunked_mlp(model, 64)
    if arm:
        install(model, arm, sink=4, window=64, vertical=16, exact_tail=8, block_m=16, block_n=16)
    if cpu_embed:
        install_cpu_embedding(model)
    ids = torch.randint(0, 512, (1, 300), device=DEV)
    want = _run(model, ids)
    install_inplace_residual(model)
    got = _run(model, ids)
    assert got[1] == want[1]
    assert all(torch.equal(a, b) for a, b in zip(got[0], want[0]))


@torch.inference_mode()
def test_lower_prefill_peak():
    """tests/test_inplace_residual.py:50-63: about one [n, hidden] bf16 tensor less at the peak."""
    model = tiny(4, hidden=1024, inter=2048, heads=16)
    ids = torch.randint(0, 512, (1, 16384), device=DEV)
    peaks = []
    for patch in (False, True):
        if patch:
            install_inplace_residual(model)
        torch.cuda.empty_cache()
        torch.cuda.reset_peak_memory_stats()
        base = torch.cuda.memory_allocated()
        model(input_ids=ids, logits_to_keep=1)
        peaks.append(torch.cuda.max_memory_allocated() - base)
    saved = (peaks[0] - peaks[1]) / (16384 * 1024 * 2)
    assert saved >= 0.9, (peaks, saved)


def test_shard_llama_single_rank_matches_install():
    """shard_llama with one rank (q/k/v rows of all heads, o_proj through GatheredOProj) gives the
    logits of the plain sparse install."""
    from utmist_bigger_bird_b200.sharding import shard_llama
    kw = dict(sink=4, window=64, vertical=16, exact_tail=8, block_m=16, block_n=16)
    model = tiny(hidden=256, inter=512, heads=4)
    ids = torch.randint(0, 512, (1, 300), device=DEV)
    install(model, "vs", **kw)
    with torch.inference_mode():
        want = model(ids).logits
    shard_llama(model, 0, 1, **kw)
    with torch.inference_mode():
        got = model(ids).logits
    torch.testing.assert_close(got, want, atol=2e-2, rtol=2e-2)
    assert (got.argmax(-1) == want.argmax(-1)).float().mean() > 0.99


def _ulps(a, b):
    """Distance in units of the last place between two bf16 tensors of the same sign pattern."""
    ia = a.contiguous().view(torch.int16).to(torch.int32)
    ib = b.contiguous().view(torch.int16).to(torch.int32)
    return (ia - ib).abs()


@pytest.mark.parametrize("n,hidden", [(300, 256), (4096, 4096), (17, 1024)])
def test_fused_rmsnorm_within_one_ulp_of_hf(n, hidden):
    """bb_rmsnorm against LlamaRMSNorm (bf16): the fp32 sum of squares runs in another order, so
    the normalised value may move by one ulp before the weight multiply (at most two after it, for
    weights above 1); almost all outputs are bit-identical."""
    from transformers.models.llama.modeling_llama import LlamaRMSNorm
    norm = LlamaRMSNorm(hidden, eps=1e-5).to(DEV, torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_(torch.randn(hidden, device=DEV) * 0.5 + 1)
    x = torch.randn(1, n, hidden, device=DEV).to(torch.bfloat16)
    want = norm(x)
    got = _ops.rmsnorm_(x, norm.weight, norm.variance_epsilon)
    u = _ulps(got, want)
    assert int(u.max()) <= 2
    assert (u == 0).float().mean() > 0.99
    r = torch.randn_like(x)
    x2 = x.clone()
    want_x = x + r
    want_y = norm(want_x)
    got_y = _ops.rmsnorm_(x2, norm.weight, norm.variance_epsilon, residual=r)
    assert torch.equal(x2, want_x), "residual add in place, rounded like torch"
    assert int(_ulps(got_y, want_y).max()) <= 2


def test_fused_rmsnorm_model_close_to_hf():
    """install_fused_rmsnorm + install_inplace_residual (fused residual add) on a tiny Llama: the
    prefill and decode logits stay within bf16 noise of the unfused model and pick the same tokens
    almost everywhere."""
    from utmist_bigger_bird_b200 import install_fused_rmsnorm
    model = tiny(hidden=256, inter=512, heads=4)
    ids = torch.randint(0, 512, (1, 300), device=DEV)
    want = _run(model, ids)
    install_inplace_residual(model)
    install_fused_rmsnorm(model)
    install_fused_rmsnorm(model)
    got = _run(model, ids)
    a, b = got[0][0], want[0][0]
    assert (a - b).abs().max() < 0.1
    assert (a.argmax(-1) == b.argmax(-1)).float().mean() > 0.97


def test_native_chunked_mlp_batch_two():
    """Leading batch dim: chunks are strided slices of the input and of the output (37 tokens, not
    a multiple of the chunk), still equal to HF's MLP on the same chunks."""
    model = tiny(1)
    mlp = model.model.layers[0].mlp
    x = torch.randn(2, 37, 256, device=DEV, dtype=torch.bfloat16)
    with torch.inference_mode():
        want = torch.cat([mlp(x[:, s:s + 8]) for s in range(0, 37, 8)], dim=1)
        install_chunked_mlp(model, 8)
        got = mlp(x)
    assert torch.equal(got, want)
