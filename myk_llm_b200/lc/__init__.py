"""Synthetic long-context retrieval testbed: key -> value records and multi-hop chains
hidden in noise, exact-match accuracy over context length x needle depth x hop count
(reference: ``src/myk_llm/lc``)."""
