"""myk_llm_b200: a B200-native (sm_100a) small-LLM research framework.

Public API mirrors the upstream ``myk_llm`` package: ``models`` (MykLLM, configs,
generate, save/load), ``train`` (trainer, optimizers, objectives, checkpoints), ``data``,
``infer`` (static-cache CUDA-graph decoding with MTP speculation), ``eval``, ``ops``
(hand-written sm_100a kernels) and ``parallel`` (process groups, sharded data parallel,
peer-memory collectives).
"""

__version__ = "0.1.0"
