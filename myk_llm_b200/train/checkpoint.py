"""Training checkpoints with torch.distributed.checkpoint (DCP).

The layout is the reference's (``src/myk_llm/train/checkpoint.py:1-110``) so checkpoints
interchange:

    <run>/checkpoints/step_0000500/
        .metadata, __*_*.distcp   sharded model + optimizer state ({"model", "optim"} from
                                  get_state_dict; any GPU count can load it)
        trainer.json              {"step", "tokens", "world_size"}, written LAST: its
                                  presence marks the checkpoint complete
        data_rank{r}.pt           each rank's data-loader state
        model.safetensors, model.yaml (+ tokenizer)   portable export (optional)

``latest_checkpoint`` ignores directories without ``trainer.json`` (a crash mid-save).
"""

from __future__ import annotations

import json
import shutil
from pathlib import Path
from typing import Any

import torch
import torch.distributed.checkpoint as dcp
from torch.distributed.checkpoint.state_dict import (StateDictOptions, get_model_state_dict, get_state_dict,
                                                     set_model_state_dict, set_state_dict)

from ..models import MykLLM, save_model
from ..parallel.distributed import DistInfo, barrier

STEP_PREFIX = "step_"


def step_dir(run_dir: Path, step: int) -> Path:
    return Path(run_dir) / "checkpoints" / f"{STEP_PREFIX}{step:07d}"


def latest_checkpoint(run_dir: Path) -> Path | None:
    cands = sorted((Path(run_dir) / "checkpoints").glob(f"{STEP_PREFIX}*"))
    done = [c for c in cands if (c / "trainer.json").exists()]
    return done[-1] if done else None


def _unwrap(model):
    return getattr(model, "module_for_checkpoint", lambda: model)()


def _app_state(model, optimizers) -> dict[str, Any]:
    m, o = get_state_dict(_unwrap(model), optimizers)
    return {"model": m, "optim": o}


def save_checkpoint(directory: Path, model, optimizers, trainer_state: dict, data_state: dict | None, info: DistInfo,
                    export_weights: bool, tokenizer: str | None = None,
                    extra_weights: dict[str, torch.Tensor] | None = None) -> None:
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    sync = getattr(model, "sync_params_for_checkpoint", None)
    if sync is not None:
        sync()
    dcp.save(_app_state(model, optimizers), checkpoint_id=str(directory))
    torch.save(data_state, directory / f"data_rank{info.rank}.pt")
    if export_weights:
        export_model(directory, model, info, tokenizer, extra_weights)
    done = getattr(model, "after_checkpoint_save", None)
    if done is not None:
        done()
    barrier()
    if info.is_main:
        (directory / "trainer.json").write_text(json.dumps(trainer_state, indent=2), encoding="utf-8")
    barrier()


def export_model(directory: Path, model, info: DistInfo, tokenizer: str | None = None,
                 extra_weights: dict[str, torch.Tensor] | None = None) -> None:
    base = _unwrap(model)
    state = get_model_state_dict(base, options=StateDictOptions(full_state_dict=True, cpu_offload=True))
    state.update(extra_weights or {})
    if info.is_main:
        save_model(directory, base.config, state, tokenizer)


def load_checkpoint(directory: Path, model, optimizers, info: DistInfo):
    """Load model (+ optimizer) state in place; returns (trainer_state, this rank's data state)."""
    directory = Path(directory)
    base = _unwrap(model)
    prepare = getattr(model, "before_checkpoint_load", None)
    if prepare is not None:
        prepare()
    if optimizers:
        state = _app_state(model, optimizers)
        dcp.load(state, checkpoint_id=str(directory))
        set_state_dict(base, optimizers, model_state_dict=state["model"], optim_state_dict=state["optim"])
    else:
        ms = get_model_state_dict(base)
        dcp.load({"model": ms}, checkpoint_id=str(directory))
        set_model_state_dict(base, ms)
    after = getattr(model, "after_checkpoint_load", None)
    if after is not None:
        after()
    ts_path = directory / "trainer.json"
    trainer_state = json.loads(ts_path.read_text(encoding="utf-8")) if ts_path.exists() else {}
    dp = directory / f"data_rank{info.rank}.pt"
    data_state = torch.load(dp, weights_only=False) if dp.exists() else None
    return trainer_state, data_state


def prune_checkpoints(run_dir: Path, keep_last: int, keep_every: int) -> None:
    if keep_last <= 0:
        return
    cks = sorted((Path(run_dir) / "checkpoints").glob(f"{STEP_PREFIX}*"))
    for path in cks[:-keep_last]:
        step = int(path.name.removeprefix(STEP_PREFIX))
        if keep_every and step % keep_every == 0:
            continue
        shutil.rmtree(path)
