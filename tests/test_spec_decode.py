"""MTP speculative decoding over static caches emits exactly the greedy continuation of
the main model (verification is greedy), for plain, windowed and YOCO models."""

import pytest
import torch

from tests.conftest import tiny_model_config


@pytest.mark.parametrize("ov", [{"mtp.depth": 2}, {"mtp.depth": 1, "layer_pattern": "GL"},
                                {"mtp.depth": 2, "layer_pattern": "GLXX"}, {"mtp.depth": 0}])
def test_spec_decode_equals_greedy(ov):
    from myk_llm_b200.infer import StaticDecoder
    from myk_llm_b200.models import MykLLM, generate

    torch.manual_seed(0)
    m = MykLLM(tiny_model_config(**ov)).eval()
    prompts = torch.randint(0, 512, (3, 12))
    ref = generate(m, prompts, 20, temperature=0.0)
    dec = StaticDecoder(m, batch_size=3, max_len=64)
    out, st = dec.generate(prompts, 20, check_every=2)
    assert torch.equal(out, ref), (out, ref)
    assert st.emitted >= 3 * 20
    if ov.get("mtp.depth", 0):
        assert 0.0 <= st.acceptance <= 1.0
