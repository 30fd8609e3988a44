"""Document-quality screening for streaming and pre-tokenisation.

The decisions (and the YAML field names and defaults that tune them) match the
reference's ``DocFilter`` (``src/myk_llm/data/filters.py:9-90``) so that the same corpus
passes the same documents in both frameworks: a length cap applied by truncation, a
minimum length, a dominant-token fraction, and on long documents a distinct-token ratio
and a repeated-bigram fraction; on the raw text, the share of the expected writing system
among CJK ideographs and ASCII letters.

The statistics are computed with numpy on whole arrays (token ids as one ``int64``
vector; bigrams packed into one 64-bit key each; the text's code points as one
``uint32`` vector), which keeps the filter cheap on the long documents it exists for.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

_CJK_LO, _CJK_HI = 0x4E00, 0x9FFF


def token_stats(ids) -> tuple[int, int, int, int]:
    """(length, count of the most frequent id, distinct ids, distinct adjacent pairs)."""
    a = np.asarray(ids, dtype=np.int64)
    n = int(a.size)
    if n == 0:
        return 0, 0, 0, 0
    _, counts = np.unique(a, return_counts=True)
    pairs = 0
    if n > 1:
        keys = (a[:-1] << np.int64(32)) ^ (a[1:] & np.int64(0xFFFFFFFF))
        pairs = int(np.unique(keys).size)
    return n, int(counts.max()), int(counts.size), pairs


def script_counts(text: str, limit: int) -> tuple[int, int]:
    """(CJK unified ideographs, ASCII letters) among the first ``limit`` characters."""
    head = text[:limit]
    if not head:
        return 0, 0
    cp = np.frombuffer(head.encode("utf-32-le"), dtype=np.uint32)
    cjk = int(np.count_nonzero((cp >= _CJK_LO) & (cp <= _CJK_HI)))
    lower = cp | np.uint32(0x20)  # ASCII letters fold onto a..z
    latin = int(np.count_nonzero((cp < 0x80) & (lower >= ord("a")) & (lower <= ord("z"))))
    return cjk, latin


@dataclass
class DocFilter:
    """Screening thresholds; ``reject`` looks at token ids, ``reject_text`` at raw text.
    Sources marked ``curated`` skip both (only ``max_doc_tokens`` truncation applies)."""

    enabled: bool = True
    max_doc_tokens: int = 8192       # truncation cap per document (0 = none)
    min_doc_tokens: int = 8
    max_top_token_frac: float = 0.5
    long_doc_tokens: int = 100       # the two ratio checks below apply from this length
    min_distinct_ratio: float = 0.1
    max_dup_bigram_frac: float = 0.5
    min_script_frac: float = 0.3
    script_scan_chars: int = 20000

    def reject(self, ids) -> bool:
        """True for degenerate token sequences (too short, one token dominating, too few
        distinct tokens, or looping phrases)."""
        if not self.enabled:
            return False
        n, top, distinct, pairs = token_stats(ids)
        if n < self.min_doc_tokens:
            return True
        if top > self.max_top_token_frac * n:
            return True
        if n < self.long_doc_tokens:
            return False
        return distinct < self.min_distinct_ratio * n or (n - 1 - pairs) > self.max_dup_bigram_frac * (n - 1)

    def reject_text(self, text: str, script: str | None) -> bool:
        """True when the expected script (``"cjk"`` or Latin otherwise) is under
        ``min_script_frac`` of the CJK + ASCII-letter characters, or there are none."""
        if not self.enabled or not script:
            return False
        cjk, latin = script_counts(text, self.script_scan_chars)
        if cjk + latin == 0:
            return True
        wanted = cjk if script == "cjk" else latin
        return wanted < self.min_script_frac * (cjk + latin)
