"""On the GPU, with the sm_100a kernels: MTP speculative decoding over static caches, replayed
as a CUDA graph, emits exactly the greedy continuation that the eager ``generate()`` loop
produces (plain, windowed, YOCO, DeltaNet / KDA, looped and n-gram models).  The output head is scaled up so that argmax
margins are far above bf16 rounding: the two paths run different kernels (static-cache
decode attention and skinny GEMMs against the growing-cache path), and a near-tie could
otherwise flip a token without either path being wrong."""

import pytest
import torch

from tests.conftest import tiny_model_config

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("ov", [{"mtp.depth": 2}, {"mtp.depth": 1, "layer_pattern": "GL"},
                                {"mtp.depth": 2, "layer_pattern": "GLXX"}, {"mtp.depth": 2, "layer_pattern": "GD"},
                                {"mtp.depth": 2, "layer_pattern": "DG", "deltanet.kind": "kda", "mtp.layer": "D"},
                                {"mtp.depth": 1, "layer_pattern": "GD", "loop.prelude": 1, "loop.core": 2,
                                 "loop.iterations": 2},
                                {"mtp.depth": 2, "ngram.orders": [2, 3], "ngram.num_buckets": 97, "ngram.dim": 32}])
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


@pytest.mark.parametrize("per_channel", [False, True])
def test_delta_spec_window_matches_recurrence(per_channel):
    """The speculative-window kernel (commit the pending prefix, run the window) against
    the fp32 token-by-token recurrence."""
    from myk_llm_b200 import ops
    from myk_llm_b200.ops import reference as ref

    torch.manual_seed(0)
    B, W, H, dk, dv = 5, 3, 4, 128, 128
    dev = "cuda"

    def inputs():
        q = torch.randn(B, W, H, dk, device=dev).bfloat16()
        k = torch.randn(B, W, H, dk, device=dev).bfloat16()
        v = torch.randn(B, W, H, dv, device=dev).bfloat16()
        g = -torch.rand(B, W, H, *((dk,) if per_channel else ()), device=dev) * 0.5
        beta = torch.rand(B, W, H, device=dev)
        return q, k, v, g, beta

    state0 = torch.randn(B, H, dk, dv, device=dev) * 0.1
    first, second = inputs(), inputs()
    pend = tuple(torch.zeros_like(t) for t in first)
    pending = torch.zeros(B, dtype=torch.int32, device=dev)
    state = state0.clone()
    o1 = ops.delta_spec_window(*first, state, pend, pending, per_channel_decay=per_channel)
    want1, _ = ref.delta_rule_ref(*first, initial_state=state0, per_channel_decay=per_channel)
    torch.testing.assert_close(o1.float(), want1.float(), atol=3e-2, rtol=3e-2)
    accepted = torch.tensor([0, 1, 2, 3, 2], dtype=torch.int32, device=dev)
    pending.copy_(accepted)
    o2 = ops.delta_spec_window(*second, state, pend, pending, per_channel_decay=per_channel)
    for b in range(B):
        n = int(accepted[b])
        sl = slice(b, b + 1)
        s = state0[sl]
        if n:
            _, s = ref.delta_rule_ref(*(t[sl, :n] for t in first), initial_state=s, per_channel_decay=per_channel)
        torch.testing.assert_close(state[sl], s, atol=1e-3, rtol=1e-3)
        want2, _ = ref.delta_rule_ref(*(t[sl] for t in second), initial_state=s, per_channel_decay=per_channel)
        torch.testing.assert_close(o2[sl].float(), want2.float(), atol=3e-2, rtol=3e-2)
    for p, t in zip(pend, second):
        assert torch.equal(p, t.to(p.dtype))
    from myk_llm_b200.ops import ext

    assert ext().take_status() == 0
