"""Training entry point (pretraining and SFT share the loop).

    python -m myk_llm_b200.train configs/pretrain/200m.yaml [key.path=value ...]
    torchrun --nproc_per_node 8 -m myk_llm_b200.train configs/...yaml

A run lives in ``<output_dir>/<run_name>/`` (config.yaml, metrics.jsonl, tb/,
checkpoints/); re-running the same command resumes from the newest complete
checkpoint.  The loop follows the reference trainer (``src/myk_llm/train/trainer.py``):
gradient accumulation derived from the global batch, a loss normalised by the global
number of supervised tokens, gradient clipping, Muon + AdamW, periodic validation in
bits per byte, greedy samples and DCP checkpoints.

``Trainer`` is the programmatic API: ``Trainer(config).train_step(micro_batches)`` runs one
optimizer step from host batches (pinned host -> device copies included) and returns the
loss as a device tensor; ``fit()`` is the whole run.

Gradients of every 2-D weight live in one flat fp32 buffer per rank (``main_grad``
views): the GEMM epilogues and the embedding / loss kernels accumulate into it directly,
gradient accumulation needs no extra pass, and the sharded runtime reduce-scatters it.
"""

from __future__ import annotations

import argparse
import math
import os
import time
from dataclasses import replace
from pathlib import Path
from typing import Any

import torch

from .. import ops
from ..configuration import dump_yaml, load_config
from ..data import build_fixed_batches, build_loader
from ..data.config import Batch
from ..models import MykLLM, generate, load_model
from ..models.transformer import nvtx_range, set_nvtx
from ..ops.loss import check_unscaled_main_grad
from ..parallel.distributed import DistInfo, all_reduce_sum, init_distributed, parallelize, shutdown
from .checkpoint import latest_checkpoint, load_checkpoint, prune_checkpoints, save_checkpoint, step_dir
from .config import InitConfig, TrainConfig
from .objectives import Objective
from .optim import build_optimizers, lr_multiplier, set_lr


def log0(info: DistInfo, *args: Any) -> None:
    if info.is_main:
        print(*args, flush=True)


# -- initialisation ----------------------------------------------------------------------
def load_pretrained_embedding(source: str, row_map_path: str) -> torch.Tensor:
    """Token embedding of a HuggingFace safetensors checkpoint, optionally gathered down to
    a pruned vocabulary (row_map[new_id] = old_id)."""
    import json

    import numpy as np
    from safetensors import safe_open

    keys = ("model.language_model.embed_tokens.weight", "model.embed_tokens.weight")
    root = Path(source)
    files = sorted(root.glob("*.safetensors")) if root.is_dir() else [root]
    index = root / "model.safetensors.index.json"
    if index.exists():
        wm = json.loads(index.read_text())["weight_map"]
        files = [root / wm[k] for k in keys if k in wm][:1]
    for f in files:
        with safe_open(str(f), framework="pt", device="cpu") as h:
            for k in keys:
                if k in h.keys():
                    w = h.get_tensor(k)
                    if row_map_path:
                        w = w.index_select(0, torch.from_numpy(np.load(row_map_path).astype(np.int64)))
                    return w
    raise KeyError(f"no embedding tensor ({keys}) found under {source}")


def initialize_weights(model: MykLLM, config: InitConfig) -> None:
    if config.weights_from:
        src = load_model(config.weights_from, device="cpu")
        missing, unexpected = model.load_state_dict(src.state_dict(), strict=False)
        if unexpected:
            raise KeyError(f"unexpected weights in {config.weights_from}: {unexpected}")
        if missing:
            print(f"warm start: {len(missing)} tensors keep their fresh init: {missing[:8]}...")
    if config.embedding_from:
        w = load_pretrained_embedding(config.embedding_from, config.embedding_row_map)
        if w.shape != model.embed.token.weight.shape:
            raise ValueError(f"pretrained embedding {tuple(w.shape)} != model {tuple(model.embed.token.weight.shape)}")
        with torch.no_grad():
            model.embed.token.weight.copy_(w)
    if config.freeze_embedding:
        model.embed.token.weight.requires_grad_(False)


def token_byte_lengths(tokenizer) -> torch.Tensor:
    special = set(tokenizer.added_tokens_decoder)
    toks = tokenizer.convert_ids_to_tokens(list(range(len(tokenizer))))
    return torch.tensor([0 if i in special else len(t) for i, t in enumerate(toks)], dtype=torch.float64)


# -- gradient buffer ---------------------------------------------------------------------
class GradBuffer:
    """One flat fp32 gradient buffer for every trainable parameter (``main_grad`` views,
    also exposed as ``.grad``; autograd accumulates into an existing ``.grad`` in place).
    Zeroed with one memset per step; the clipping norm is one reduction over it."""

    def __init__(self, params: list[torch.nn.Parameter], device: torch.device) -> None:
        seen: set[int] = set()
        self.params = []
        for p in params:
            if p.requires_grad and p.is_cuda and id(p) not in seen:
                seen.add(id(p))
                self.params.append(p)
        total = sum((p.numel() + 15) // 16 * 16 for p in self.params)
        self.flat = torch.zeros(total, dtype=torch.float32, device=device)
        off = 0
        for p in self.params:
            n = p.numel()
            p.main_grad = self.flat[off:off + n].view(p.shape)
            p.grad = p.main_grad
            off += (n + 15) // 16 * 16
        self.ids = {id(p) for p in self.params}

    def zero_(self) -> None:
        self.flat.zero_()
        for p in self.params:
            if p.grad is None or p.grad.data_ptr() != p.main_grad.data_ptr():
                p.grad = p.main_grad


# -- the trainer -------------------------------------------------------------------------
class Trainer:
    def __init__(self, config: TrainConfig, info: DistInfo | None = None, build_data: bool = True,
                 tokenizer: Any = None) -> None:
        self.config = config
        self.info = info = info or init_distributed()
        set_nvtx(config.logging.nvtx)
        torch.manual_seed(config.seed)
        per_step = config.data.micro_batch_size * info.world_size
        if config.global_batch_size % per_step:
            raise ValueError(f"global_batch_size {config.global_batch_size} is not a multiple of micro_batch_size x "
                             f"ranks = {per_step}")
        self.grad_accum = config.global_batch_size // per_step
        self.tokens_per_step = config.global_batch_size * config.data.seq_len
        model = MykLLM(config.model)
        initialize_weights(model, config.init)
        self.tables = self._build_tables(model)
        model = model.to(info.device)
        self.raw_model = model
        self.model = parallelize(model, config.parallel, info)
        self.optimizers = build_optimizers(getattr(self.model, "optim_module", lambda: self.model)(), config.optimizer)
        self.base_lrs = [[g["lr"] for g in o.param_groups] for o in self.optimizers]
        attach = getattr(self.model, "attach_optimizers", None)
        if attach is not None:
            attach(self.optimizers)
        self.objective = Objective(config.objective, info.device)
        self.params = [p for p in self.model.parameters() if p.requires_grad]
        self.grads = None
        if info.device.type == "cuda" and not getattr(self.model, "owns_gradients", False) \
                and config.parallel.strategy != "fsdp":
            self.grads = GradBuffer(self.params, info.device)
        self.tokenizer = tokenizer
        self.loader = build_loader(config.data, info.rank, info.world_size) if build_data else None
        self.step = 0
        self.tokens_seen = 0

    def _build_tables(self, model: MykLLM):
        ng = self.config.optimizer.ngram
        if ng.update != "lazy" or model.embed.ngram is None:
            return None
        if self.info.enabled:
            raise NotImplementedError("optimizer.ngram.update=lazy is single-GPU only")
        from .ngram_tables import SparseNgramTables

        mod = model.embed.ngram
        c = self.config.optimizer
        return SparseNgramTables(mod, ng, c.lr, tuple(c.betas), c.eps, self.info.device,
                                 max_rows_per_step=self.tokens_per_step * len(mod.orders))

    # ---------------------------------------------------------------------------------
    def zero_grad(self) -> None:
        if getattr(self.model, "owns_gradients", False):
            self.model.zero_grad()
            return
        if self.grads is not None:
            self.grads.zero_()
        for p in self.params:
            if self.grads is None or id(p) not in self.grads.ids:
                p.grad = None

    def forward_backward(self, batch: Batch, normalizer: float) -> dict[str, torch.Tensor]:
        batch = batch.to(self.info.device)
        with nvtx_range("forward"):
            out = self.model(batch.input_ids, seqlens=batch.seqlens, head=self.objective.head(batch, normalizer))
        with nvtx_range("backward"):
            out.loss.backward()
        return out.sums

    def clip_and_step(self) -> torch.Tensor:
        grad_clip = self.config.optimizer.grad_clip
        fused = getattr(self.model, "optimizer_step", None)
        if fused is not None:
            norm = fused(grad_clip)
            ops.invalidate_weight_cache()
            return norm
        norm = self.grad_norm()
        coef = None
        if grad_clip and grad_clip > 0:
            # the clipping coefficient stays on the device and the optimizer kernels apply it
            # as they read each gradient: no extra pass over the gradients, no host sync
            coef = torch.clamp(grad_clip / (norm + 1e-6), max=1.0)
        for opt in self.optimizers:
            if coef is not None and hasattr(opt, "grad_scale"):
                opt.grad_scale = coef
            elif coef is not None:  # an optimizer without the hook: scale its gradients here
                gs = [p.grad for g in opt.param_groups for p in g["params"] if p.grad is not None]
                if gs:
                    torch._foreach_mul_(gs, coef)
            opt.step()
            if hasattr(opt, "grad_scale"):
                opt.grad_scale = None
        ops.invalidate_weight_cache()
        if self.tables is not None:
            self.tables.step()
        return norm

    def _grad_owners(self):
        owners = getattr(self.model, "grad_owners", None)
        return owners() if owners is not None else self.params

    def grad_norm(self) -> torch.Tensor:
        custom = getattr(self.model, "grad_norm", None)
        if custom is not None:
            return custom()
        parts = []
        others = []
        for p in self._grad_owners():
            if p.grad is None:
                continue
            if self.grads is not None and id(p) in self.grads.ids:
                continue
            g = p.grad
            others.append(g.to_local() if hasattr(g, "to_local") else g)
        if self.grads is not None:
            parts.append(torch.linalg.vector_norm(self.grads.flat).square())
        if others:
            parts.extend(n.float().square() for n in torch._foreach_norm(others))
        if not parts:
            return torch.zeros((), device=self.info.device)
        total = torch.stack([p.to(self.info.device) for p in parts]).sum()
        if self.config.parallel.strategy == "fsdp" and self.info.enabled:
            torch.distributed.all_reduce(total)
        return total.sqrt()

    def train_step(self, micro_batches: list[Batch], step: int | None = None) -> dict[str, torch.Tensor]:
        """One optimizer step over this rank's micro-batches.  Returns device tensors:
        ``loss`` (mean CE over the global batch), ``grad_norm`` and the loss sums."""
        self.step = self.step + 1 if step is None else step
        mult = lr_multiplier(self.step, self.config.steps, self.config.schedule)
        set_lr(self.optimizers, self.base_lrs, mult)
        if self.tables is not None:
            self.tables.set_lr_multiplier(mult)
            self.tables.begin_step([b.input_ids for b in micro_batches], None)
        normalizer = all_reduce_sum(sum(b.num_targets for b in micro_batches), self.info.device)
        self.zero_grad()
        sums: dict[str, torch.Tensor] = {}
        for b in micro_batches:
            s = self.forward_backward(b, normalizer)
            for k, v in s.items():
                sums[k] = sums[k] + v if k in sums else v.clone()
        with nvtx_range("optimizer"):
            norm = self.clip_and_step()
        self.tokens_seen += self.tokens_per_step
        out = {f"sum/{k}": v for k, v in sums.items()}
        out["loss"] = sums.get("ce", torch.zeros(())) / max(1.0, normalizer)
        out["grad_norm"] = norm
        out["normalizer"] = torch.tensor(normalizer)
        return out

    def check_health(self, loss: float, grad_norm: float, step: int) -> None:
        """Called at a point where the host has already synchronised with the device (the
        logging sync of ``fit``): raises if a bounded device wait gave up since the last
        check (a peer that never arrived, a stalled pipeline: the kernels wound down and
        left results incomplete) or if the loss or the gradient norm is not finite."""
        if self.info.device.type == "cuda":
            code = int(ops.ext().take_status())
            if code != 0:
                raise RuntimeError(f"step {step}: a device wait gave up (status {code}: the source line of the wait "
                                   "in csrc/); the step's results are incomplete")
        if not math.isfinite(loss):
            raise FloatingPointError(f"step {step}: non-finite training loss {loss}")
        if not math.isfinite(grad_norm):
            raise FloatingPointError(f"step {step}: non-finite gradient norm {grad_norm}")

    # ---------------------------------------------------------------------------------
    @torch.no_grad()
    def validate(self, val_sets: dict[str, list[Batch]], token_bytes: torch.Tensor | None) -> dict[str, float]:
        info = self.info
        self.model.eval()
        res = {}
        for name, batches in val_sets.items():
            loss_sum = count = nbytes = 0.0
            per = math.ceil(len(batches) / info.world_size)
            for i in range(per):
                idx = info.rank + i * info.world_size
                b = batches[idx % len(batches)].to(info.device)
                w = 1.0 if idx < len(batches) else 0.0
                out = self.model(b.input_ids, seqlens=b.seqlens, head=self.objective.head(b, 1.0))
                loss_sum += w * float(out.sums["ce"])
                count += w * b.num_targets
                if token_bytes is not None:
                    tg = b.targets[b.targets >= 0].cpu()
                    nbytes += w * float(token_bytes[tg].sum())
            loss_sum = all_reduce_sum(loss_sum, info.device)
            res[f"val/{name}/loss"] = loss_sum / max(1.0, all_reduce_sum(count, info.device))
            if token_bytes is not None:
                res[f"val/{name}/bpb"] = loss_sum / math.log(2) / max(1.0, all_reduce_sum(nbytes, info.device))
        self.model.train()
        return res

    def sample_text(self) -> list[str]:
        if self.tokenizer is None:
            return []
        self.model.eval()
        texts = []
        for prompt in self.config.eval.sample_prompts:
            if self.config.eval.sample_chat:
                ids = self.tokenizer.apply_chat_template([{"role": "user", "content": prompt}],
                                                         add_generation_prompt=True, return_tensors="pt",
                                                         return_dict=True)["input_ids"]
            else:
                ids = self.tokenizer(prompt, add_special_tokens=False, return_tensors="pt")["input_ids"]
            out = generate(self.raw_model, ids.to(self.info.device), self.config.eval.sample_tokens, temperature=0.0,
                           eos_token_id=self.tokenizer.eos_token_id)
            texts.append(self.tokenizer.decode(out[0].tolist()))
        self.model.train()
        return texts

    # ---------------------------------------------------------------------------------
    def fit(self, resume: str = "auto") -> None:
        config, info = self.config, self.info
        run_dir = Path(config.output_dir) / config.run_name
        loader = self.loader
        start = 1
        ck = latest_checkpoint(run_dir) if resume == "auto" else (Path(resume) if resume != "none" else None)
        if ck is not None:
            ts, ds = load_checkpoint(ck, self.model, self.optimizers, info)
            if self.tables is not None:
                self.tables.load(ck)
            start, self.tokens_seen = ts["step"] + 1, ts["tokens"]
            if ds is not None:
                loader.load_state_dict(ds)
            log0(info, f"resumed from {ck} at step {start}")
        elif config.init.checkpoint_from:
            load_checkpoint(Path(config.init.checkpoint_from), self.model,
                            self.optimizers if config.init.load_optimizer else None, info)
        val_sets = {
            vs.name: build_fixed_batches(replace(config.data, kind=vs.kind or config.data.kind, sources=vs.sources),
                                         config.eval.batches, config.eval.seed)
            for vs in config.eval.val_sets
        } if config.eval.interval > 0 else {}
        token_bytes = token_byte_lengths(self.tokenizer) if self.tokenizer is not None else None
        metrics = None
        if info.is_main:
            run_dir.mkdir(parents=True, exist_ok=True)
            name = "config.yaml" if ck is None else f"config.resume-{start:07d}.yaml"
            (run_dir / name).write_text(dump_yaml(config), encoding="utf-8")
            from .metrics import MetricsLogger

            metrics = MetricsLogger(run_dir / "metrics.jsonl", run_dir / "tb" if config.logging.tensorboard else None)
            if ck is None:
                metrics.log(0, {"params/total": self.raw_model.num_parameters(),
                                "params/non_embedding": self.raw_model.num_parameters(exclude_embeddings=True)})
        log0(info, f"run {run_dir}: {info.world_size} rank(s), micro batch {config.data.micro_batch_size} x accum "
                   f"{self.grad_accum} = {config.global_batch_size} seqs = {self.tokens_per_step:,} tokens/step")
        it = iter(loader)
        self.model.train()
        t0, win_tokens = time.perf_counter(), 0
        acc: dict[str, torch.Tensor] = {}
        norm_total = 0.0

        def is_ckpt(step: int) -> bool:
            if step == config.steps:
                return config.checkpoint.final
            return bool(config.checkpoint.interval and step % config.checkpoint.interval == 0)

        for step in range(start, config.steps + 1):
            batches = [next(it) for _ in range(self.grad_accum)]
            data_state = loader.state_dict() if is_ckpt(step) else None
            out = self.train_step(batches, step)
            for k, v in out.items():
                if k.startswith("sum/"):
                    acc[k] = acc[k] + v if k in acc else v
            norm_total += float(out["normalizer"])
            win_tokens += self.tokens_per_step
            if step % config.logging.interval == 0 or step == config.steps:
                if info.device.type == "cuda":
                    torch.cuda.synchronize()
                    check_unscaled_main_grad()
                dt = time.perf_counter() - t0
                rec = {f"train/{k[4:]}": all_reduce_sum(float(v), info.device) / max(1.0, norm_total)
                       for k, v in acc.items()}
                rec["train/loss"] = rec.get("train/ce", float("nan"))
                rec.update({"train/grad_norm": float(out["grad_norm"]),
                            "train/lr": self.optimizers[-1].param_groups[0]["lr"],
                            "perf/tokens_per_s": win_tokens / dt,
                            "perf/tokens_per_s_per_gpu": win_tokens / dt / info.world_size,
                            "perf/peak_mem_gb": (torch.cuda.max_memory_allocated() / 2 ** 30
                                                 if info.device.type == "cuda" else 0.0),
                            "tokens": self.tokens_seen})
                if self.tables is not None:
                    rec.update(self.tables.pop_stats())
                self.check_health(rec["train/loss"], rec["train/grad_norm"], step)
                if metrics is not None:
                    metrics.log(step, rec)
                log0(info, f"step {step:6d} loss {rec['train/loss']:.4f} lr {rec['train/lr']:.2e} "
                           f"gnorm {rec['train/grad_norm']:.2f} {rec['perf/tokens_per_s']:,.0f} tok/s "
                           f"mem {rec['perf/peak_mem_gb']:.1f}GB")
                t0, win_tokens, acc, norm_total = time.perf_counter(), 0, {}, 0.0
            if val_sets and (step % config.eval.interval == 0 or step == config.steps):
                r = self.validate(val_sets, token_bytes)
                if metrics is not None:
                    metrics.log(step, r)
                log0(info, f"step {step:6d} [val] " + " ".join(f"{k}={v:.4f}" for k, v in r.items()))
            if config.eval.sample_interval and step % config.eval.sample_interval == 0:
                for text in self.sample_text():
                    log0(info, f"--- sample ---\n{text}")
            if is_ckpt(step):
                target = step_dir(run_dir, step)
                extra = None
                if self.tables is not None:
                    target.mkdir(parents=True, exist_ok=True)
                    self.tables.save(target)
                    extra = self.tables.export_weights() if config.checkpoint.export_weights else None
                save_checkpoint(target, self.model, self.optimizers,
                                {"step": step, "tokens": self.tokens_seen, "world_size": info.world_size},
                                data_state, info, config.checkpoint.export_weights,
                                config.data.tokenizer if self.tokenizer is not None else None, extra)
                if info.is_main:
                    prune_checkpoints(run_dir, config.checkpoint.keep_last, config.checkpoint.keep_every)
                log0(info, f"saved {target}")
        if val_sets and start > config.steps:
            r = self.validate(val_sets, token_bytes)
            if metrics is not None:
                metrics.log(config.steps, r)
        if metrics is not None:
            metrics.close()
        if self.tables is not None:
            self.tables.close()
        loader.close()


def _load_tokenizer(path: str):
    if not path or not Path(path).exists():
        return None
    from transformers import AutoTokenizer

    return AutoTokenizer.from_pretrained(path)


def train(config: TrainConfig, resume: str = "auto") -> None:
    info = init_distributed()
    tok = _load_tokenizer(config.data.tokenizer)
    if tok is not None and len(tok) > config.model.vocab_size:
        raise ValueError(f"tokenizer has {len(tok)} tokens > model.vocab_size {config.model.vocab_size}")
    Trainer(config, info, tokenizer=tok).fit(resume)
    shutdown()


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("config", help="YAML run config")
    ap.add_argument("overrides", nargs="*", help="key.path=value overrides")
    ap.add_argument("--resume", default="auto", help="'auto', 'none', or a checkpoint dir")
    a = ap.parse_args(argv)
    os.environ.setdefault("HF_HOME", str(Path.cwd() / ".cache" / "hf"))
    train(load_config(TrainConfig, a.config, a.overrides), resume=a.resume)
