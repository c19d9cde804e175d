"""Device-memory analysis: peak usage and the largest live allocations.

The reference finds its largest buffers by scanning the compiled program (the HLO big-buffer scan of
megagpt-speedrun/_diag_ragged.py:148-256 and grug-moe-pp/benchmark.py:270-295, which located a
278 GiB transient) and reads the compiler's memory analysis. With eager PyTorch the same questions
are answered from the CUDA caching allocator: ``peak_gb`` (high-water mark of allocated bytes since
the last reset), and ``largest_blocks`` / ``memory_report`` over ``torch.cuda.memory_snapshot()``
(every segment the allocator holds and its blocks, allocated or free), which show the biggest live
tensors and how much reserved memory sits in free blocks.
"""

from __future__ import annotations

import torch


def peak_gb(device=None) -> float:
    return torch.cuda.max_memory_allocated(device) / 1e9


def largest_blocks(snapshot: list[dict], n: int = 10) -> list[dict]:
    """The ``n`` largest allocated blocks: ``{"bytes", "address", "segment_bytes", "stream"}``."""
    blocks = []
    for seg in snapshot:
        for b in seg.get("blocks", []):
            if b.get("state") == "active_allocated":
                blocks.append({"bytes": int(b.get("size", 0)), "address": int(b.get("address", 0)),
                               "segment_bytes": int(seg.get("total_size", 0)), "stream": seg.get("stream", 0)})
    blocks.sort(key=lambda b: -b["bytes"])
    return blocks[:n]


def summarize(snapshot: list[dict]) -> dict:
    """Reserved, allocated and free-in-reserved bytes over all segments, and the segment count."""
    reserved = allocated = free = 0
    for seg in snapshot:
        reserved += int(seg.get("total_size", 0))
        for b in seg.get("blocks", []):
            if b.get("state") == "active_allocated":
                allocated += int(b.get("size", 0))
            elif b.get("state") == "inactive":
                free += int(b.get("size", 0))
    return {"reserved_bytes": reserved, "allocated_bytes": allocated, "free_in_reserved_bytes": free,
            "segments": len(snapshot)}


def memory_report(snapshot: list[dict] | None = None, n: int = 10) -> str:
    """Markdown summary of a snapshot (the current device's when ``snapshot`` is None)."""
    if snapshot is None:
        snapshot = torch.cuda.memory_snapshot()
    s = summarize(snapshot)
    lines = [f"reserved {s['reserved_bytes'] / 1e9:.2f} GB in {s['segments']} segments, allocated "
             f"{s['allocated_bytes'] / 1e9:.2f} GB, free inside reserved {s['free_in_reserved_bytes'] / 1e9:.2f} GB",
             "", "| rank | block MB | segment MB | stream |", "|---|---|---|---|"]
    for i, b in enumerate(largest_blocks(snapshot, n)):
        lines.append(f"| {i + 1} | {b['bytes'] / 2**20:.1f} | {b['segment_bytes'] / 2**20:.1f} | {b['stream']} |")
    return "\n".join(lines)
