"""Receive-buffer layout of the reduce-to-owner transport (host-side arithmetic, CPU)."""
from rational_optimizer_b200.optim.tiller import layer_owner
import pytest

from rational_optimizer_b200.parallel.owner_reduce import counter_index, receive_layout, slot_bytes


def test_slot_sizes_per_transport():
    assert slot_bytes(1024, "f32") == 4096 and slot_bytes(1024, "bf16") == 2048
    # int8: values padded to 16 bytes, then one fp32 scale per 256 elements padded to 16 bytes
    assert slot_bytes(1024, "int8") == 1024 + 16
    assert slot_bytes(264, "int8") == 272 + 16  # 2 blocks -> 8 bytes of scales -> 16
    assert slot_bytes(4096 * 1024, "int8") == 4096 * 1024 + 4 * 16384
    assert all(slot_bytes(n, t) % 16 == 0 for n in (8, 264, 1000, 4104) for t in ("f32", "bf16", "int8"))


@pytest.mark.parametrize("transport", ["f32", "bf16", "int8"])
def test_layout_places_every_sender_slot_disjointly(transport):
    L, world = 18, 8
    sizes = [1024 * (13 + (l % 3)) + 8 * (l % 5) for l in range(L)]
    owners = [layer_owner(l, L, world) for l in range(L)]
    offsets, totals = receive_layout(sizes, owners, world, transport)
    assert sorted(offsets) == sorted(set(owners))
    for owner, table in offsets.items():
        spans = []
        for layer, base in table.items():
            assert owners[layer] == owner and base % 16 == 0
            sb = slot_bytes(sizes[layer], transport)
            spans += [(base + r * sb, base + (r + 1) * sb) for r in range(world)]
        spans.sort()
        assert spans[0][0] == 0 and spans[-1][1] == totals[owner]
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))  # back to back, no overlap
    # counters: one per owned layer, numbered in layer order
    for owner in set(owners):
        mine = [l for l in range(L) if owners[l] == owner]
        assert [counter_index(l, owners) for l in mine] == list(range(len(mine)))


def test_owner_map_matches_tiller_shards():
    from rational_optimizer_b200.optim.tiller import shard_bounds
    for L, world in ((18, 8), (18, 4), (4, 2), (3, 4)):
        for layer in range(L):
            r = layer_owner(layer, L, world)
            lo, hi = shard_bounds(L, r, world)
            assert lo <= layer < hi


def test_python_slot_sizes_match_the_kernels():
    from rational_optimizer_b200 import _ext
    if not _ext.available():
        pytest.skip("extension not built")
    C = _ext.ext()
    for t, mode in (("f32", 0), ("bf16", 1), ("int8", 2)):
        for n in (8, 256, 264, 1000, 4104, 4096 * 1024):
            assert C.owner_slot_bytes(n, mode) == slot_bytes(n, t), (t, n)
