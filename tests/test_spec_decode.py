"""MTP speculative decoding over static caches emits exactly the greedy continuation of
the main model (verification is greedy), for plain, windowed, YOCO, DeltaNet / KDA,
looped and n-gram models; with oracle drafts (so rows accept 0..K tokens per round) the
DeltaNet states commit exactly the accepted prefix."""

import pytest
import torch

from tests.conftest import tiny_model_config


CASES = [{"mtp.depth": 2}, {"mtp.depth": 1, "layer_pattern": "GL"}, {"mtp.depth": 2, "layer_pattern": "GLXX"},
         {"mtp.depth": 0}, {"mtp.depth": 2, "layer_pattern": "GD"},
         {"mtp.depth": 1, "layer_pattern": "DG", "deltanet.kind": "kda"},
         {"mtp.depth": 2, "layer_pattern": "GD", "mtp.layer": "D"},
         {"mtp.depth": 1, "layer_pattern": "GD", "loop.prelude": 1, "loop.core": 2, "loop.iterations": 2},
         {"mtp.depth": 2, "ngram.orders": [2, 3], "ngram.num_buckets": 97, "ngram.dim": 32}]


@pytest.mark.parametrize("ov", CASES)
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


class _OracleDrafts:
    """Replace each round's MTP drafts with the true greedy continuation, corrupting some
    of them so that rows accept different numbers of drafts per round."""

    def __init__(self, dec, reference: torch.Tensor, vocab: int):
        self.dec, self.ref, self.vocab, self.round = dec, reference, vocab, 0
        self.inner = dec._round
        dec._round = self

    def __call__(self):
        self.inner()
        dec, K = self.dec, self.dec.K
        j = torch.arange(K)
        cols = (dec.seqlens.long()[:, None] + 1 + j[None]).clamp(max=self.ref.size(1) - 1)
        true = self.ref.gather(1, cols)
        rows = torch.arange(dec.B)[:, None]
        bad = (rows + j[None] + self.round) % 3 == 0
        dec.drafts.copy_(torch.where(bad, (true + 1) % self.vocab, true))
        self.round += 1


@pytest.mark.parametrize("ov", [{"mtp.depth": 2, "layer_pattern": "GD"}, {"mtp.depth": 3, "layer_pattern": "DD"},
                                {"mtp.depth": 2, "layer_pattern": "DG", "deltanet.kind": "kda", "mtp.layer": "D"},
                                {"mtp.depth": 2, "ngram.orders": [2, 3], "ngram.num_buckets": 97, "ngram.dim": 32}])
def test_spec_decode_commits_accepted_prefix(ov):
    from myk_llm_b200.infer import StaticDecoder
    from myk_llm_b200.models import MykLLM, generate

    torch.manual_seed(1)
    m = MykLLM(tiny_model_config(**ov)).eval()
    prompts = torch.randint(0, 512, (4, 10))
    new = 24
    ref = generate(m, prompts, new + 8, temperature=0.0)
    dec = StaticDecoder(m, batch_size=4, max_len=64, use_cuda_graph=False)
    _OracleDrafts(dec, ref, 512)
    out, st = dec.generate(prompts, new, check_every=1)
    assert torch.equal(out, ref[:, :10 + new]), (out, ref)
    assert 0.3 < st.acceptance < 1.0  # mixed acceptance: the commit saw every prefix length
