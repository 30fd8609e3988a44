"""Training metrics: durable append-only JSONL (flushed per record) plus optional
TensorBoard scalars (reference: ``src/myk_llm/train/metrics.py:15-38``)."""

from __future__ import annotations

import json
import time
from pathlib import Path
from typing import Any


class MetricsLogger:
    def __init__(self, jsonl_path, tensorboard_dir=None) -> None:
        self.jsonl_path = Path(jsonl_path)
        self.jsonl_path.parent.mkdir(parents=True, exist_ok=True)
        self._fh = self.jsonl_path.open("a", encoding="utf-8")
        self._tb: Any = None
        if tensorboard_dir is not None:
            try:
                from torch.utils.tensorboard import SummaryWriter

                self._tb = SummaryWriter(log_dir=str(tensorboard_dir))
            except Exception:  # tensorboard not installed: JSONL only
                self._tb = None

    def log(self, step: int, metrics: dict[str, Any], wall_time: float | None = None) -> None:
        rec = {"step": step, "time": wall_time if wall_time is not None else time.time(), **metrics}
        self._fh.write(json.dumps(rec) + "\n")
        self._fh.flush()
        if self._tb is not None:
            for k, v in metrics.items():
                if isinstance(v, (int, float)):
                    self._tb.add_scalar(k, v, step)

    def close(self) -> None:
        self._fh.close()
        if self._tb is not None:
            self._tb.close()
