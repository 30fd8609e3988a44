"""On the GPU, with the sm_100a kernels: MTP speculative decoding over static caches, replayed
as a CUDA graph, emits exactly the greedy continuation that the eager ``generate()`` loop
produces (plain, windowed and YOCO models).  The output head is scaled up so that argmax
margins are far above bf16 rounding: the two paths run different kernels (static-cache
decode attention and skinny GEMMs against the growing-cache path), and a near-tie could
otherwise flip a token without either path being wrong."""

import pytest
import torch

from tests.conftest import tiny_model_config

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("ov", [{"mtp.depth": 2}, {"mtp.depth": 1, "layer_pattern": "GL"},
                                {"mtp.depth": 2, "layer_pattern": "GLXX"}])
def test_cuda_graph_spec_decode_equals_greedy(ov):
    from myk_llm_b200.infer import StaticDecoder
    from myk_llm_b200.models import MykLLM, generate

    torch.manual_seed(0)
    model = MykLLM(tiny_model_config(**ov)).cuda().eval()
    with torch.no_grad():
        model.lm_head.weight.mul_(40.0)
    prompts = torch.randint(0, 512, (3, 12), device="cuda")
    want = generate(model, prompts, 24, temperature=0.0)
    dec = StaticDecoder(model, batch_size=3, max_len=64, use_cuda_graph=True)
    got, stats = dec.generate(prompts, 24, check_every=2)
    assert torch.equal(got, want), (got, want)
    assert stats.emitted >= 3 * 24 and stats.rounds > 0
    from myk_llm_b200.ops import ext

    assert ext().take_status() == 0
