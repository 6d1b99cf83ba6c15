"""Incremental decoding with a KV cache against the reference's way of producing next-token logits
(generate_torch.py:278-285: the whole context through the model, logits[0, -1]), computed by the oracle
under the fp16 recipe."""
import numpy as np
import pytest
import torch

from conftest import rel_err
from oracle import jishui_ref as oracle
from test_model_gpu import SMALL, _pair

pytestmark = pytest.mark.gpu


def _ref_logits(ref, ctx):
    t = torch.tensor([ctx], dtype=torch.long, device="cuda")
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.float16):
        return ref(t)[0, -1].float()


@pytest.mark.parametrize("kw", [SMALL, dict(SMALL, norm_type="layernorm", norm_bias=True, hidden_size=192,
                                             num_attention_heads=3, num_key_value_heads=3, intermediate_size=320)])
def test_kv_cache_decoding_matches_full_context(kw):
    from midstream_llm_b200.config import ModelConfig
    from midstream_llm_b200.decode import next_token_logits
    cfg = ModelConfig(**kw)
    ref, mine = _pair(cfg)
    rng = np.random.default_rng(0)
    ctx = rng.integers(3, cfg.vocab_size, size=300).tolist()  # not a multiple of the 256-token tile
    for step in range(6):
        got = torch.from_numpy(next_token_logits(mine, ctx, "cuda")).cuda()
        assert got.shape == (cfg.vocab_size,)
        e = rel_err(got, _ref_logits(ref, ctx))
        assert e < 5e-3, (step, e)
        ctx = ctx + [int(got.argmax())]
    dec = mine._kv_decoder
    assert dec.context == ctx[:-1]  # the cache covers the last context
    # A different prompt is prefilled from scratch.
    other = rng.integers(3, cfg.vocab_size, size=40).tolist()
    assert rel_err(torch.from_numpy(next_token_logits(mine, other)).cuda(), _ref_logits(ref, other)) < 5e-3
    # Changed weights invalidate the cache even when the context extends the previous one.
    with torch.no_grad():
        mine.layers[0].mlp.down_proj.weight.mul_(1.5)
        ref.layers[0].mlp.down_proj.weight.mul_(1.5)
    longer = other + [5]
    assert rel_err(torch.from_numpy(next_token_logits(mine, longer)).cuda(), _ref_logits(ref, longer)) < 5e-3
