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


def test_local_switch_slices_packed_and_split_layers():
    """Each rank keeps its experts of the switch layer, in placement order:
    the Gemma 4 packed gate_up_proj [E, 2I, .] and down_proj, or the split
    gate/up/down projections, sliced along the expert axis."""
    import torch

    from mlxr_moe.ep import local_switch
    from mlxr_moe.moe import PackedSwitchFfn, QuantizedSwitchLinear, SplitSwitchFfn

    E, I, D = 6, 4, 16

    def q(rows, kin, tag):
        w = torch.arange(E * rows * kin // 8, dtype=torch.int32).reshape(E, rows, kin // 8) + tag
        s = torch.full((E, rows, kin // 64 or 1), float(tag)).to(torch.bfloat16)
        return QuantizedSwitchLinear(w, s, s.clone(), 64, 4)

    mine = [4, 1]
    packed = local_switch(PackedSwitchFfn(q(2 * I, D, 100), q(D, I * 8, 200)), mine)
    assert isinstance(packed, PackedSwitchFfn)
    full = q(2 * I, D, 100)
    assert torch.equal(packed.gate_up_proj.weight, full.weight[mine])
    assert packed.gate_up_proj.weight.shape == (2, 2 * I, D // 8) and packed.gate_up_proj.weight.is_contiguous()
    assert packed.down_proj.weight.shape[0] == 2
    split = local_switch(SplitSwitchFfn(q(I, D, 1), q(I, D, 2), q(D, I * 8, 3)), mine)
    assert isinstance(split, SplitSwitchFfn)
    assert torch.equal(split.up_proj.weight, q(I, D, 2).weight[mine])
