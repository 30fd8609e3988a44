"""Training run configuration (one YAML file per run).

The schema is the reference's (``src/myk_llm/train/config.py:12-175``) so run configs
move between the two frameworks.  Extensions (all defaulted, so reference YAMLs load
unchanged): ``parallel.strategy`` also accepts ``sharded`` (this framework's own
sharded data parallel with peer-memory collectives) and ``fsdp`` keeps meaning torch
FSDP2 over NCCL (the baseline); ``parallel.mxfp8_grad_dtype`` chooses E4M3 (reference
behaviour) or E5M2 gradients for MXFP8.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Literal

from ..data.config import DataConfig, SourceConfig
from ..models.config import ModelConfig


@dataclass
class NgramOptimConfig:
    """dense: tables are plain AdamW parameters.  lazy: only the rows a step touches are
    gathered, updated (Adam) and written back; rows live on the GPU or in host memory,
    optionally prefetched; ``catch_up`` replays skipped steps in closed form."""

    update: Literal["dense", "lazy"] = "dense"
    placement: Literal["gpu", "host"] = "gpu"
    prefetch: bool = True
    lr_scale: float = 1.0
    weight_decay: float = 0.0
    second_moment: Literal["elementwise", "rowwise"] = "elementwise"
    catch_up: bool = False


@dataclass
class OptimizerConfig:
    name: Literal["muon", "adamw"] = "muon"
    lr: float = 3e-4
    betas: list[float] = field(default_factory=lambda: [0.9, 0.95])
    eps: float = 1e-8
    weight_decay: float = 0.1
    muon_lr: float | None = None
    muon_weight_decay: float | None = None
    muon_momentum: float = 0.95
    muon_nesterov: bool = True
    muon_ns_steps: int = 5
    muon_adjust_lr: Literal["original", "match_rms_adamw", "none"] = "match_rms_adamw"
    grad_clip: float = 1.0
    ngram: NgramOptimConfig = field(default_factory=NgramOptimConfig)


@dataclass
class ScheduleConfig:
    kind: Literal["cosine", "wsd", "constant"] = "cosine"
    warmup_ratio: float = 0.01
    min_lr_ratio: float = 0.1
    decay_ratio: float = 0.2


@dataclass
class DistillConfig:
    teacher: str = ""
    row_map: str = ""
    weight: float = 0.5
    temperature: float = 1.0
    chunk_size: int = 1024


@dataclass
class ObjectiveConfig:
    z_loss: float = 0.0
    mtp_weight: float = 0.3
    loss_chunk_size: int = 2048
    distill: DistillConfig = field(default_factory=DistillConfig)


@dataclass
class InitConfig:
    embedding_from: str = ""
    embedding_row_map: str = ""
    freeze_embedding: bool = False
    weights_from: str = ""
    checkpoint_from: str = ""
    load_optimizer: bool = False


@dataclass
class ParallelConfig:
    # auto: this framework's parameter-sharded data parallel when world_size > 1; sharded:
    # always that runtime; replicated: the same runtime with every parameter replicated
    # (only optimizer state and work sharded); fsdp: torch FSDP2 (NCCL baseline); none:
    # no data-parallel wrapper.
    strategy: Literal["auto", "fsdp", "sharded", "replicated", "none"] = "auto"
    param_dtype: Literal["fp32", "bf16"] = "fp32"
    reshard_after_forward: bool = True
    compile: bool = True
    activation_checkpointing: bool | int = False
    float8: Literal["none", "tensorwise", "rowwise", "rowwise_with_gw_hp", "mxfp8"] = "none"
    float8_skip_down_proj: bool = False
    mxfp8_grad_dtype: Literal["e4m3", "e5m2"] = "e4m3"


@dataclass
class CheckpointConfig:
    interval: int = 500
    final: bool = True
    keep_last: int = 3
    keep_every: int = 0
    export_weights: bool = True


@dataclass
class ValSetConfig:
    name: str
    sources: list[SourceConfig]
    kind: Literal["shards", "stream", "sft", "synthetic"] | None = None


@dataclass
class EvalConfig:
    interval: int = 0
    batches: int = 8
    seed: int = 999_983
    val_sets: list[ValSetConfig] = field(default_factory=list)
    sample_interval: int = 0
    sample_prompts: list[str] = field(default_factory=lambda: ["The meaning of life is"])
    sample_chat: bool = False
    sample_tokens: int = 64


@dataclass
class LoggingConfig:
    interval: int = 10
    tensorboard: bool = True
    nvtx: bool = False  # NVTX ranges per layer and per training phase (for timeline profilers)


@dataclass
class TrainConfig:
    run_name: str = "debug"
    output_dir: str = "runs"
    steps: int = 1000
    global_batch_size: int = 32
    seed: int = 0
    model: ModelConfig = field(default_factory=ModelConfig)
    data: DataConfig = field(default_factory=DataConfig)
    optimizer: OptimizerConfig = field(default_factory=OptimizerConfig)
    schedule: ScheduleConfig = field(default_factory=ScheduleConfig)
    objective: ObjectiveConfig = field(default_factory=ObjectiveConfig)
    init: InitConfig = field(default_factory=InitConfig)
    parallel: ParallelConfig = field(default_factory=ParallelConfig)
    checkpoint: CheckpointConfig = field(default_factory=CheckpointConfig)
    eval: EvalConfig = field(default_factory=EvalConfig)
    logging: LoggingConfig = field(default_factory=LoggingConfig)
