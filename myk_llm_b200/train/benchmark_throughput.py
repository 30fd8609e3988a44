"""Training throughput and peak memory of any run config on random packed tokens (one GPU),
through the real trainer step (model, objective, optimizers), so architecture variants
can be compared before a full run::

    python -m myk_llm_b200.train.benchmark_throughput configs/pretrain/200m.yaml
    python -m myk_llm_b200.train.benchmark_throughput configs/model/200m-dddg.yaml data.micro_batch_size=8
"""

from __future__ import annotations

import argparse
import json

import torch


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("config")
    ap.add_argument("overrides", nargs="*")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--steps", type=int, default=10)
    args = ap.parse_args(argv)
    from ..configuration import load_config
    from ..data.synthetic import SyntheticLoader
    from ..parallel.distributed import init_distributed
    from .config import TrainConfig
    from .trainer import Trainer

    cfg = load_config(TrainConfig, args.config, args.overrides + ["data.kind=synthetic", "logging.tensorboard=false"])
    cfg.data.synthetic.vocab_size = cfg.model.vocab_size
    cfg.global_batch_size = cfg.data.micro_batch_size
    info = init_distributed()
    tr = Trainer(cfg, info, build_data=False)
    ld = SyntheticLoader(cfg.data, 0, 1)
    batches = [ld.batch_at(i) for i in range(args.warmup + args.steps)]
    for i, b in enumerate(batches[:args.warmup]):
        tr.train_step([b.pin_memory()], i + 1)
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i, b in enumerate(batches[args.warmup:]):
        tr.train_step([b.pin_memory()], args.warmup + i + 1)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    tokens = cfg.data.micro_batch_size * cfg.data.seq_len
    print(json.dumps({"config": args.config, "overrides": args.overrides, "ms_per_step": ms,
                      "tokens_per_s": tokens / ms * 1e3, "peak_mem_gb": torch.cuda.max_memory_allocated() / 2**30,
                      "params_m": tr.raw_model.num_parameters() / 1e6}))


if __name__ == "__main__":
    main()
