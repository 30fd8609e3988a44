"""Training checkpoints on torch.distributed.checkpoint (DCP).

The directory layout is an interface shared with the reference
(``src/myk_llm/train/checkpoint.py:1-110``), so checkpoints move between the frameworks:

    <run>/checkpoints/step_0000500/
        .metadata, __*_*.distcp   model + optimizer state as {"model", "optim"} of
                                  ``get_state_dict`` (reshardable to any GPU count)
        trainer.json              {"step", "tokens", "world_size"}; written last, so its
                                  presence means the checkpoint is complete
        data_rank{r}.pt           each rank's data-loader state
        model.safetensors, model.yaml (+ tokenizer)   optional portable export

Here the model and the optimizers are handed to DCP as ``Stateful`` entries
(``TrainState``), so DCP calls back for their state.  Around that, the data-parallel
runtime's hooks run (``sync_params_for_checkpoint`` / ``after_checkpoint_save`` /
``before_checkpoint_load`` / ``after_checkpoint_load``): the parameter-sharded runtime
materialises full tensors for a save and scatters loaded tensors into its shards.  ``trainer.json`` is written to a temporary name and
renamed, so a crash can never leave a half-written completion marker.
"""

from __future__ import annotations

import json
import os
import re
import shutil
from pathlib import Path
from typing import Any

import torch
import torch.distributed.checkpoint as dcp
from torch.distributed.checkpoint.state_dict import (StateDictOptions, get_model_state_dict,
                                                     get_optimizer_state_dict, set_model_state_dict,
                                                     set_optimizer_state_dict)
from torch.distributed.checkpoint.stateful import Stateful

from ..models import save_model
from ..parallel.distributed import DistInfo, barrier

STEP_PREFIX = "step_"
DONE_MARKER = "trainer.json"
_STEP_DIR = re.compile(rf"^{STEP_PREFIX}(\d+)$")


def step_dir(run_dir: Path, step: int) -> Path:
    return Path(run_dir) / "checkpoints" / f"{STEP_PREFIX}{step:07d}"


def _completed(run_dir: Path) -> list[tuple[int, Path]]:
    """(step, path) of every complete checkpoint, oldest first."""
    root = Path(run_dir) / "checkpoints"
    if not root.is_dir():
        return []
    found = []
    for child in root.iterdir():
        m = _STEP_DIR.match(child.name)
        if m and (child / DONE_MARKER).is_file():
            found.append((int(m.group(1)), child))
    return sorted(found)


def latest_checkpoint(run_dir: Path) -> Path | None:
    """Newest complete checkpoint (directories without ``trainer.json`` are a crash
    during a save and are ignored)."""
    done = _completed(run_dir)
    return done[-1][1] if done else None


def _base(model) -> torch.nn.Module:
    unwrap = getattr(model, "module_for_checkpoint", None)
    return unwrap() if unwrap is not None else model


def _hook(model, name: str) -> None:
    fn = getattr(model, name, None)
    if fn is not None:
        fn()


class TrainState:
    """Model and optimizers as the two top-level DCP entries ``"model"`` and ``"optim"``
    (the ``get_state_dict`` layout), each a ``Stateful`` that DCP calls back."""

    def __init__(self, model, optimizers) -> None:
        self.model, self.optimizers = model, list(optimizers or [])

    def entries(self) -> dict[str, Stateful]:
        out: dict[str, Stateful] = {"model": _ModelEntry(self)}
        if self.optimizers:
            out["optim"] = _OptimEntry(self)
        return out


class _ModelEntry(Stateful):
    def __init__(self, ts: TrainState) -> None:
        self.ts = ts

    def state_dict(self) -> dict[str, Any]:
        return get_model_state_dict(_base(self.ts.model))

    def load_state_dict(self, state: dict[str, Any]) -> None:
        set_model_state_dict(_base(self.ts.model), state)


class _OptimEntry(Stateful):
    def __init__(self, ts: TrainState) -> None:
        self.ts = ts

    def state_dict(self) -> dict[str, Any]:
        return get_optimizer_state_dict(_base(self.ts.model), self.ts.optimizers)

    def load_state_dict(self, state: dict[str, Any]) -> None:
        set_optimizer_state_dict(_base(self.ts.model), self.ts.optimizers, state)


def _write_marker(directory: Path, payload: dict) -> None:
    tmp = directory / f".{DONE_MARKER}.tmp"
    tmp.write_text(json.dumps(payload, indent=2), encoding="utf-8")
    os.replace(tmp, directory / DONE_MARKER)


def save_checkpoint(directory: Path, model, optimizers, trainer_state: dict, data_state: dict | None, info: DistInfo,
                    export_weights: bool, tokenizer: str | None = None,
                    extra_weights: dict[str, torch.Tensor] | None = None) -> None:
    """Every rank calls this.  Order: DCP shards, per-rank loader state, optional export,
    barrier, completion marker (rank 0), barrier."""
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    _hook(model, "sync_params_for_checkpoint")
    try:
        dcp.save(TrainState(model, optimizers).entries(), checkpoint_id=str(directory))
        torch.save(data_state, directory / f"data_rank{info.rank}.pt")
        if export_weights:
            export_model(directory, model, info, tokenizer, extra_weights)
    finally:
        _hook(model, "after_checkpoint_save")
    barrier()
    if info.is_main:
        _write_marker(directory, trainer_state)
    barrier()


def export_model(directory: Path, model, info: DistInfo, tokenizer: str | None = None,
                 extra_weights: dict[str, torch.Tensor] | None = None) -> None:
    """Portable ``model.safetensors`` + ``model.yaml`` (full tensors, written by rank 0)."""
    base = _base(model)
    full = get_model_state_dict(base, options=StateDictOptions(full_state_dict=True, cpu_offload=True))
    full.update(extra_weights or {})
    if info.is_main:
        save_model(directory, base.config, full, tokenizer)


def load_checkpoint(directory: Path, model, optimizers, info: DistInfo):
    """Load model (+ optimizer) state in place; returns (trainer state, this rank's loader
    state or None)."""
    directory = Path(directory)
    _hook(model, "before_checkpoint_load")
    dcp.load(TrainState(model, optimizers).entries(), checkpoint_id=str(directory))
    _hook(model, "after_checkpoint_load")
    marker = directory / DONE_MARKER
    trainer_state = json.loads(marker.read_text(encoding="utf-8")) if marker.exists() else {}
    loader_file = directory / f"data_rank{info.rank}.pt"
    data_state = torch.load(loader_file, weights_only=False) if loader_file.exists() else None
    return trainer_state, data_state


def prune_checkpoints(run_dir: Path, keep_last: int, keep_every: int) -> None:
    """Delete complete checkpoints beyond the newest ``keep_last``, except steps that are
    multiples of ``keep_every`` (``keep_last <= 0`` keeps everything)."""
    if keep_last <= 0:
        return
    done = _completed(run_dir)
    for step, path in done[:max(0, len(done) - keep_last)]:
        if keep_every and step % keep_every == 0:
            continue
        shutil.rmtree(path)
