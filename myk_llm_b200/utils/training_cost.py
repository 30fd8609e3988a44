"""Wall-clock hours of a run of ``total_tokens`` billion tokens at a measured throughput
of ``k_tokens_per_s`` thousand tokens per second (the reference's
``scripts/compute_total_training_cost.py``); with ``--gpus`` and ``--usd-per-gpu-hour``
also GPU-hours and cost::

    python -m myk_llm_b200.utils.training_cost 100 182 --gpus 1 --usd-per-gpu-hour 3.5
"""

from __future__ import annotations

import argparse


def training_hours(total_tokens_b: float, k_tokens_per_s: float) -> float:
    return total_tokens_b * 1e9 / (k_tokens_per_s * 1e3) / 3600


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("total_tokens_b", type=float, help="billions of tokens")
    ap.add_argument("k_tokens_per_s", type=float, help="whole-job throughput, thousands of tokens/s")
    ap.add_argument("--gpus", type=int, default=None)
    ap.add_argument("--usd-per-gpu-hour", type=float, default=None)
    args = ap.parse_args(argv)
    hours = training_hours(args.total_tokens_b, args.k_tokens_per_s)
    print(f"Total training time: {hours:.2f} hours")
    if args.gpus:
        print(f"GPU-hours: {hours * args.gpus:.1f}")
        if args.usd_per_gpu_hour:
            print(f"Cost: ${hours * args.gpus * args.usd_per_gpu_hour:,.0f}")


if __name__ == "__main__":
    main()
