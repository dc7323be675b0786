"""Receive-buffer layout of the reduce-to-owner transport (host-side arithmetic, CPU)."""
from rational_optimizer_b200.optim.tiller import layer_owner
from rational_optimizer_b200.parallel.owner_reduce import counter_index, receive_layout


def test_layout_places_every_sender_slot_disjointly():
    L, world = 18, 8
    sizes = [1024 * (13 + (l % 3)) for l in range(L)]
    owners = [layer_owner(l, L, world) for l in range(L)]
    offsets, totals = receive_layout(sizes, owners, world)
    assert sorted(offsets) == sorted(set(owners))
    for owner, table in offsets.items():
        spans = []
        for layer, base in table.items():
            assert owners[layer] == owner
            spans += [(base + r * sizes[layer], base + (r + 1) * sizes[layer]) for r in range(world)]
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
