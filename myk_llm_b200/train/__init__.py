"""Training runtime: trainer loop, optimizers, objectives, checkpoints, metrics."""

from .config import TrainConfig
from .trainer import Trainer, main, train

__all__ = ["TrainConfig", "Trainer", "main", "train"]
