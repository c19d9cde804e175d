"""Device-memory analysis over an allocator snapshot (synthetic: the snapshot format of
torch.cuda.memory_snapshot)."""

from marin_experiments_b200.utils import memory

SNAP = [
    {"total_size": 4 << 30, "stream": 0, "blocks": [
        {"size": 3 << 30, "state": "active_allocated", "address": 0x1000},
        {"size": 1 << 30, "state": "inactive", "address": 0x2000}]},
    {"total_size": 2 << 20, "stream": 7, "blocks": [
        {"size": 1 << 20, "state": "active_allocated", "address": 0x3000},
        {"size": 1 << 20, "state": "active_allocated", "address": 0x4000}]},
]


def test_summary_and_largest_blocks():
    s = memory.summarize(SNAP)
    assert s["reserved_bytes"] == (4 << 30) + (2 << 20) and s["segments"] == 2
    assert s["allocated_bytes"] == (3 << 30) + (2 << 20) and s["free_in_reserved_bytes"] == 1 << 30
    top = memory.largest_blocks(SNAP, 2)
    assert [b["bytes"] for b in top] == [3 << 30, 1 << 20] and top[0]["segment_bytes"] == 4 << 30
    text = memory.memory_report(SNAP, 3)
    assert "reserved 4.30 GB in 2 segments" in text and text.count("\n") == 6 and "| 1 | 3072.0 |" in text
