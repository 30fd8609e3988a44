"""Source-tree rules checked on CPU: no TMA / bulk copy with cluster multicast anywhere
(the multi-GPU pool forbids it, and every load here must be a plain per-CTA copy), and
none of the batched-memcpy driver calls that are closed on this pool."""

from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
SOURCES = [p for d in ("csrc", "myk_llm_b200") for p in (ROOT / d).rglob("*")
           if p.suffix in (".cu", ".cuh", ".h", ".cpp", ".py")]

# assembled from pieces so that this file does not itself contain the forbidden strings
FORBIDDEN = [".multi" + "cast::" + "cluster", "TMA_LOAD_MULTI" + "CAST", "Memcpy" + "BatchAsync",
             "Memcpy3D" + "BatchAsync"]


def test_sources_exist():
    assert any(p.suffix == ".cu" for p in SOURCES) and any(p.suffix == ".py" for p in SOURCES)


def test_no_cluster_multicast_or_closed_calls():
    hits = []
    for p in SOURCES:
        text = p.read_text(encoding="utf-8", errors="replace")
        for pat in FORBIDDEN:
            if pat in text:
                hits.append(f"{p.relative_to(ROOT)}: {pat}")
    assert not hits, hits
