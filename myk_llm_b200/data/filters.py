"""Cheap document-quality heuristics used by streaming and pre-tokenisation.

Thresholds and checks are those of the reference (``src/myk_llm/data/filters.py:9-90``):
a hard cap on document length (truncation), minimum length, dominant-token fraction,
distinct-token ratio and duplicate-bigram fraction on long documents, and an expected
writing-system fraction (CJK vs Latin) on the raw text.
"""

from __future__ import annotations

from collections import Counter
from dataclasses import dataclass


@dataclass
class DocFilter:
    enabled: bool = True
    max_doc_tokens: int = 8192
    min_doc_tokens: int = 8
    max_top_token_frac: float = 0.5
    long_doc_tokens: int = 100
    min_distinct_ratio: float = 0.1
    max_dup_bigram_frac: float = 0.5
    min_script_frac: float = 0.3
    script_scan_chars: int = 20000

    def reject(self, ids: list[int]) -> bool:
        if not self.enabled:
            return False
        n = len(ids)
        if n < self.min_doc_tokens:
            return True
        counts = Counter(ids)
        if counts.most_common(1)[0][1] / n > self.max_top_token_frac:
            return True
        if n >= self.long_doc_tokens:
            if len(counts) / n < self.min_distinct_ratio:
                return True
            bigrams = len(set(zip(ids, ids[1:])))
            if 1.0 - bigrams / (n - 1) > self.max_dup_bigram_frac:
                return True
        return False

    def reject_text(self, text: str, script: str | None) -> bool:
        if not self.enabled or not script:
            return False
        cjk = latin = 0
        for ch in text[: self.script_scan_chars]:
            o = ord(ch)
            if 0x4E00 <= o <= 0x9FFF:
                cjk += 1
            elif o < 0x80 and ch.isalpha():
                latin += 1
        total = cjk + latin
        if total == 0:
            return True
        return (cjk if script == "cjk" else latin) / total < self.min_script_frac
