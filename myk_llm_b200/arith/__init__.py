"""Arithmetic length-generalisation testbed: character-level addition / multiplication
with direct, reversed or chain-of-thought answers (reference: ``src/myk_llm/arith``)."""
