"""Static-cache decoding with multi-token-prediction (MTP) speculative decoding.

The reference only benchmarks the iteration time of an MTP verify + draft step for an
assumed acceptance rate (``scripts/benchmark_decode.py``); it has no decoding loop that
accepts or rejects drafts.  This module is that loop:

1. **Prefill** the prompts through the main model into preallocated per-layer caches
   (``StaticKV``: (batch, capacity, kv_heads, head_dim) plus one shared per-row
   ``seqlens``), then through every MTP module so their own attention caches cover the
   prompt.  The main model's greedy next token is the first "bonus" token.
2. **Round**: the window ``[bonus, d_1 .. d_K]`` (K = number of MTP depths) runs through
   the main model in one pass at positions ``seqlens + [0..K]``; ``y = argmax`` per
   position.  Row b accepts the longest prefix of drafts with ``d_i == y_{i-1}``
   (``a_b`` tokens) and emits ``d_1..d_a, y_a``; ``y_a`` becomes the next bonus.
3. MTP depth k then runs over the same window (its next-token inputs are the accepted
   tokens, the bonus and the earlier depths' fresh drafts), and position ``a_b`` of depth k
   gives draft ``d_k`` of the next round.  Finally ``seqlens += a + 1``.  Keys/values written
   for rejected positions lie beyond ``seqlens`` and are overwritten later.

DeltaNet layers keep a ``SpecDeltaState``: the committed conv/recurrent state plus the last
window's inputs, of which the first ``a_b + 1`` are folded in at the start of the next
window (one state read and one write per layer and round).  Looped models get one cache
entry per core iteration; n-gram models carry the last ``context`` committed tokens per row
as the embedding's left context.

Verification is greedy, so the emitted sequence equals plain greedy decoding of the main
model.  A round has static shapes and no host synchronisation, so on CUDA it is captured
once in a CUDA graph and replayed; the host looks at the output only every few rounds.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field

import torch

from ..models.mixers import DeltaNet, SpecDeltaState, StaticKV
from ..models.transformer import MykLLM


@dataclass
class DecodeStats:
    rounds: int = 0
    emitted: int = 0  # tokens emitted over all rows (excluding the prompt)
    accepted_drafts: int = 0
    drafted: int = 0
    prefill_s: float = 0.0
    decode_s: float = 0.0
    per_depth_accept: list[float] = field(default_factory=list)

    @property
    def acceptance(self) -> float:
        return self.accepted_drafts / max(1, self.drafted)

    @property
    def tokens_per_round(self) -> float:
        return self.emitted / max(1, self.rounds)


class StaticDecoder:
    """Greedy decoding over static caches, speculative with the model's MTP heads when
    ``draft_depth > 0`` (default: all of them)."""

    def __init__(self, model: MykLLM, batch_size: int, max_len: int, draft_depth: int | None = None,
                 use_cuda_graph: bool = True) -> None:
        cfg = model.config
        self.model = model.eval()
        self.cfg = cfg
        self.B, self.cap = batch_size, max_len
        self.K = len(model.mtp) if draft_depth is None else min(draft_depth, len(model.mtp))
        dev = model.device
        self.device = dev
        dt = torch.bfloat16 if dev.type == "cuda" else next(model.parameters()).dtype
        a = cfg.attention
        self.seqlens = torch.zeros(batch_size, dtype=torch.int32, device=dev)
        self.pending = torch.zeros(batch_size, dtype=torch.int32, device=dev)  # tokens the last round accepted
        cap = max_len + self.K + 2

        def kv():
            return StaticKV(torch.zeros(batch_size, cap, a.num_kv_heads, a.head_dim, dtype=dt, device=dev),
                            torch.zeros(batch_size, cap, a.num_kv_heads, a.head_dim, dtype=dt, device=dev),
                            self.seqlens)

        def state_for(block):
            if isinstance(block.mixer, DeltaNet):
                return SpecDeltaState(block.mixer.inner, batch_size, self.K + 1, self.pending, dt, dev)
            return kv()

        self.cache: list = [None if e is None else kv() if e == "shared_kv" else state_for(e)
                            for e in model.cache_blocks()]
        self.mtp_cache = [state_for(m.block) for m in list(model.mtp)[:self.K]]
        self.delta_states = [c for c in self.cache + self.mtp_cache if isinstance(c, SpecDeltaState)]
        ngram = model.embed.ngram
        self.context = ngram.context if ngram is not None else 0
        self.history = torch.zeros(batch_size, self.context, dtype=torch.long, device=dev)  # n-gram left context
        self._ctx_ar = torch.arange(self.context, device=dev)
        self.use_graph = use_cuda_graph and dev.type == "cuda"
        self.graph = None
        self.out_tokens = None

    # ---------------------------------------------------------------------------------
    def _main(self, ids, pos, prefix=None):
        return self.model(ids, position_ids=pos, cache=self.cache, use_cache=True, prefix_ids=prefix)

    def _head_argmax(self, h):
        return self.model.logits(h).float().argmax(-1)

    def _mtp(self, k, hidden, next_ids, pos):
        m = self.model.mtp[k]
        emb = self.model.embed.token(next_ids) if not hidden.is_cuda else \
            __import__("myk_llm_b200").ops.embedding(next_ids, self.model.embed.token.weight)
        x, _ = m(hidden, emb, pos, None, state=self.mtp_cache[k], use_cache=True)
        return x, m.final_norm(x, out_dtype=x.dtype if not x.is_cuda else torch.bfloat16)

    @torch.no_grad()
    def prefill(self, prompts: torch.Tensor) -> None:
        """prompts (batch, P) of equal length."""
        B, P = prompts.shape
        assert B == self.B
        self.seqlens.zero_()
        self.pending.zero_()
        for st in self.delta_states:
            st.reset()
            st.prefill = True
        pos = torch.arange(P, device=self.device).expand(B, -1)
        out = self._main(prompts, pos)
        y_last = self._head_argmax(out.hidden[:, -1:])[:, 0]
        # MTP modules over the prompt: depth k at position i sees token i+k (known inside
        # the prompt, else the greedy token / the previous depth's draft)
        hidden = out.residual
        ext = [prompts, y_last[:, None]]
        drafts = []
        for k in range(self.K):
            seq = torch.cat(ext + [d[:, None] for d in drafts], 1)
            nxt = seq[:, k + 1:k + 1 + P]
            hidden, hn = self._mtp(k, hidden, nxt, pos)
            drafts.append(self._head_argmax(hn[:, -1:])[:, 0])
        for st in self.delta_states:
            st.prefill = False
        if self.context:
            self.history.copy_(self.model.embed.ngram.padded_tokens(prompts, None)[:, -self.context:])
        self.seqlens += P
        self.bonus = y_last.clone()
        self.drafts = torch.stack(drafts, 1) if drafts else torch.zeros(B, 0, dtype=torch.long, device=self.device)

    def _round(self) -> None:
        """One verify + draft round on static buffers (graph-capturable)."""
        K, B = self.K, self.B
        w = torch.cat([self.bonus[:, None], self.drafts], 1)  # (B, K+1)
        pos = self.seqlens.long()[:, None] + self._ar[None, :K + 1]
        out = self._main(w, pos, self.history if self.context else None)
        y = self._head_argmax(out.hidden)  # (B, K+1)
        if K:
            match = (w[:, 1:] == y[:, :-1]).int()
            a = match.cumprod(1).sum(1)  # accepted drafts per row
        else:
            a = torch.zeros(B, dtype=torch.long, device=self.device)
        a = a.long()
        bonus = y.gather(1, a[:, None])[:, 0]
        # emitted tokens this round: w[1..a] and the bonus, written at out_len onward
        emit = torch.cat([w[:, 1:], torch.zeros_like(w[:, :1])], 1)
        emit.scatter_(1, a[:, None], bonus[:, None])
        cols = self.out_len[:, None] + self._ar[None, :K + 1]
        valid = self._ar[None, :K + 1] <= a[:, None]
        cols = torch.where(valid, cols, torch.full_like(cols, self.out_tokens.size(1) - 1))
        self.out_tokens.scatter_(1, cols.clamp(max=self.out_tokens.size(1) - 1), torch.where(valid, emit, self._pad))
        self.out_len += a + 1
        self.acc_sum += a
        if K:
            self.acc_depth += (self._ar[None, :K] < a[:, None]).long().sum(0)
        # drafts for the next round
        hidden = out.residual
        known = torch.cat([w, bonus[:, None]], 1)  # tokens at window positions 0..K+1 (valid up to a+1)
        fresh = []
        for k in range(K):
            # next-token input of depth k at window position i is the token at i+k+1
            idx = self._ar[None, :K + 1] + k + 1  # (1, K+1)
            take_known = idx <= a[:, None] + 1
            src = known.gather(1, idx.clamp(max=K + 1).expand(B, -1))
            # positions beyond a+1 come from this round's fresh drafts (a+2 -> fresh[0], ...)
            if fresh:
                fr = torch.stack(fresh, 1)  # (B, k)
                j = (idx - a[:, None] - 2).clamp(min=0, max=len(fresh) - 1)
                src = torch.where(take_known, src, fr.gather(1, j))
            else:
                src = torch.where(take_known, src, bonus[:, None].expand(-1, K + 1))
            hidden, hn = self._mtp(k, hidden, src, pos)
            hk = hn.gather(1, a[:, None, None].expand(-1, 1, hn.size(-1)))
            fresh.append(self._head_argmax(hk)[:, 0])
        self.bonus.copy_(bonus)
        if K:
            self.drafts.copy_(torch.stack(fresh, 1))
        if self.context:  # the accepted window tokens w[0..a] extend the n-gram context
            span = torch.cat([self.history, w], 1)
            idx = (a + 1)[:, None] + self._ctx_ar[None]
            self.history.copy_(span.gather(1, idx))
        self.pending.copy_((a + 1).int())
        self.seqlens += (a + 1).int()

    @torch.no_grad()
    def generate(self, prompts: torch.Tensor, max_new_tokens: int, check_every: int = 8) -> tuple[torch.Tensor, DecodeStats]:
        """Greedy continuation of ``prompts`` (batch, P): returns (tokens (batch, P + n),
        stats).  Every row gets at least ``max_new_tokens`` new tokens (trimmed to exactly
        that many)."""
        B, P = prompts.shape
        if P + max_new_tokens + self.K + 1 > self.cap + self.K + 2:
            raise ValueError("prompt + max_new_tokens exceeds the decoder capacity")
        st = DecodeStats()
        sync = torch.cuda.synchronize if self.device.type == "cuda" else (lambda: None)
        sync()
        t0 = time.perf_counter()
        self.prefill(prompts)
        sync()
        st.prefill_s = time.perf_counter() - t0
        self._ar = torch.arange(self.K + 2, device=self.device)
        self._pad = torch.zeros((), dtype=torch.long, device=self.device)
        self.out_tokens = torch.zeros(B, max_new_tokens + self.K + 2, dtype=torch.long, device=self.device)
        self.out_tokens[:, 0] = self.bonus
        self.out_len = torch.ones(B, dtype=torch.long, device=self.device)
        self.acc_sum = torch.zeros(B, dtype=torch.long, device=self.device)
        self.acc_depth = torch.zeros(max(1, self.K), dtype=torch.long, device=self.device)
        step = self._round
        if self.use_graph:
            step = self._graph_step()
        t1 = time.perf_counter()
        rounds = 0
        while True:
            for _ in range(check_every):
                step()
                rounds += 1
            if int(self.out_len.min()) >= max_new_tokens:
                break
        sync()
        st.decode_s = time.perf_counter() - t1
        st.rounds = rounds
        st.emitted = int(self.out_len.sum()) - B
        st.accepted_drafts = int(self.acc_sum.sum())
        st.drafted = rounds * B * self.K
        st.per_depth_accept = (self.acc_depth.float() / max(1, rounds * B)).tolist() if self.K else []
        toks = torch.cat([prompts, self.out_tokens[:, :max_new_tokens]], 1)
        return toks, st

    def _live_tensors(self) -> list[torch.Tensor]:
        """Decoder state a round mutates besides the attention caches (whose writes land
        beyond ``seqlens`` and are harmless to repeat)."""
        out = [self.seqlens, self.pending, self.history, self.bonus, self.drafts, self.out_tokens, self.out_len,
               self.acc_sum, self.acc_depth]
        for st in self.delta_states:
            out += [st.recurrent, *st.inputs] + ([st.conv, st.window_x] if st.conv is not None else [])
        return out

    def _graph_step(self):
        # warm up on a side stream, then capture one round
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        live = self._live_tensors()
        snap = [t.clone() for t in live]
        with torch.cuda.stream(s):
            self._round()
        torch.cuda.current_stream().wait_stream(s)
        for t, v in zip(live, snap):
            t.copy_(v)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._round()
        self.graph = g
        return g.replay
