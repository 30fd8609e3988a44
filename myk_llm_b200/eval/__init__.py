"""Evaluation: zero-shot log-likelihood benchmarks (:mod:`.bench`) and the chat
generation sanity check (:mod:`.chat_eval`)."""
