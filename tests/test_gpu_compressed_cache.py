"""Compressed key storage in an HF model: a tiny random Llama decodes with ``SunShapeCompressedCache``
(uint8 codeword indices in the cache, attention through the fused decode kernel) and with the
reference-style ``SunShapeCache`` (keys quantized then stored dequantized, native SDPA -- the
behaviour of the reference's cache.py:32-46, checked against the reference in test_gpu_boundary).
Logits of the prefill and of eight greedy decode steps must agree within the bf16 tolerance, per row."""
import numpy as np
import pytest
import torch

from tests.helpers import TOL_BF16, assert_close_rowwise, make_codec

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _tiny_llama():
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=8, num_key_value_heads=2, head_dim=64, max_position_embeddings=256,
                      attn_implementation="sdpa")
    return LlamaForCausalLM(cfg).to(DEV, torch.bfloat16).eval()


def _codecs(n_layers, head_dim=64, block_dim=8, mixed=False):
    g = torch.Generator().manual_seed(3)
    nb = head_dim // block_dim
    out = {}
    for layer in range(n_layers):
        heavy = torch.zeros(nb, dtype=torch.bool)
        if mixed:
            heavy[:2] = True
        out[layer] = make_codec(torch.randperm(head_dim, generator=g), torch.randn(nb, 256, block_dim, generator=g),
                                heavy, head_dim, block_dim, 256, DEV)
    return out


@pytest.mark.parametrize("mixed", [False, True])
def test_compressed_cache_decodes_like_fake_quant_cache(mixed):
    from sunshape_b200.cache import SunShapeCache
    from sunshape_b200.compressed_cache import SunShapeCompressedCache, SunShapeCompressedLayer

    model = _tiny_llama()
    codecs = _codecs(2, mixed=mixed)
    prompt = torch.randint(0, 512, (2, 12), generator=torch.Generator().manual_seed(1)).to(DEV)

    def run(cache, impl, feed=None):
        # greedy decode; the second run is fed the first run's tokens so both see the same history
        model.config._attn_implementation = impl
        logits, toks = [], []
        with torch.no_grad():
            out = model(input_ids=prompt, past_key_values=cache, use_cache=True)
            for i in range(8):
                logits.append(out.logits[:, -1].float())
                nxt = out.logits[:, -1].argmax(-1, keepdim=True) if feed is None else feed[i]
                toks.append(nxt)
                out = model(input_ids=nxt, past_key_values=cache, use_cache=True)
            logits.append(out.logits[:, -1].float())
        return torch.stack(logits, 1), toks

    ref, toks = run(SunShapeCache.from_codecs(codecs, config=model.config), "sdpa")
    cache = SunShapeCompressedCache.from_codecs(codecs, config=model.config)
    ours, _ = run(cache, "sunshape", feed=toks)
    model.config._attn_implementation = "sdpa"
    assert_close_rowwise(ours.cpu().numpy(), ref.cpu().numpy(), TOL_BF16, "logits")
    layer = cache.layers[0]
    assert isinstance(layer, SunShapeCompressedLayer) and layer.indices.dtype == torch.uint8
    assert cache.get_seq_length(0) == 12 + 8
    sb = layer.storage_bytes()
    assert sb["key_bytes_per_token_head"] < 64 * 2        # far below the dense bf16 key row
