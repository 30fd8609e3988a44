"""Training metrics: an append-only JSONL file that is flushed record by record (it
survives a crash up to the last logged step), plus TensorBoard scalars when the
``tensorboard`` package is importable.  Record layout (``{"step", "time", <name>: value}``)
and file names are the reference's (``src/myk_llm/train/metrics.py:15-38``), so the sweep
reports read either framework's runs.
"""

from __future__ import annotations

import json
import math
import time
from pathlib import Path
from typing import Any


def _scalars(metrics: dict[str, Any]):
    """(name, float) pairs of the finite-or-not numeric entries (bools excluded)."""
    for name, value in metrics.items():
        if isinstance(value, bool) or not isinstance(value, (int, float)):
            continue
        yield name, float(value)


class MetricsLogger:
    """``log(step, {...})`` appends one JSON line; usable as a context manager."""

    def __init__(self, jsonl_path, tensorboard_dir=None) -> None:
        self.jsonl_path = Path(jsonl_path)
        self.jsonl_path.parent.mkdir(parents=True, exist_ok=True)
        self._out = open(self.jsonl_path, "a", encoding="utf-8", buffering=1)  # line-buffered
        self._board = self._open_board(tensorboard_dir)

    @staticmethod
    def _open_board(directory):
        if directory is None:
            return None
        try:
            from torch.utils.tensorboard import SummaryWriter
        except Exception:  # noqa: BLE001  (tensorboard missing: JSONL only)
            return None
        return SummaryWriter(log_dir=str(directory))

    def log(self, step: int, metrics: dict[str, Any], wall_time: float | None = None) -> None:
        record = {"step": int(step), "time": time.time() if wall_time is None else wall_time}
        record.update(metrics)
        self._out.write(json.dumps(record, default=float) + "\n")
        if self._board is not None:
            for name, value in _scalars(metrics):
                if math.isfinite(value):
                    self._board.add_scalar(name, value, step)

    def close(self) -> None:
        if not self._out.closed:
            self._out.close()
        if self._board is not None:
            self._board.close()
            self._board = None

    def __enter__(self) -> "MetricsLogger":
        return self

    def __exit__(self, *exc) -> None:
        self.close()
