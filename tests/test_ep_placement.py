"""Expert placement for expert parallelism (host logic, CPU)."""
import random

from mlxr_moe.ep import balanced_placement, placement_table, strided_placement


def test_strided_placement():
    assert strided_placement(8, 4) == [0, 1, 2, 3, 0, 1, 2, 3]
    assert placement_table(strided_placement(8, 4)) == [(r << 16) | (e // 4) for e, r in enumerate([0, 1, 2, 3] * 2)]


def test_balanced_placement_zipf_like():
    rnd = random.Random(0)
    E, world = 128, 8
    ranks = list(range(1, E + 1))
    rnd.shuffle(ranks)
    loads = [1000.0 / r ** 1.1 for r in ranks]  # Zipf(1.1) over a random expert ranking
    place = balanced_placement(loads, world)
    per = [sum(l for l, p in zip(loads, place) if p == r) for r in range(world)]
    assert sorted(set(place)) == list(range(world))
    # LPT guarantee: max <= mean + max single load
    assert max(per) <= sum(loads) / world + max(loads) + 1e-9
    strided = strided_placement(E, world)
    per_s = [sum(l for l, p in zip(loads, strided) if p == r) for r in range(world)]
    assert max(per) <= max(per_s)


def test_placement_table_local_indices():
    place = [2, 0, 2, 1, 0, 2]
    t = placement_table(place)
    assert [v >> 16 for v in t] == place
    assert [v & 0xFFFF for v in t] == [0, 0, 1, 0, 1, 2]
