"""Host-side planning of the residency tiers (no GPU): which layers stay in HBM
under a byte budget and which stream from pinned host memory.  The rule
follows the reference's partial residency (rwkv_ssd/runtime/residency.py:98-118):
the embedding and head first, then the outermost layers (0, L-1, 1, L-2, ...)
while they fit beside the device slots the streamed layers rotate through."""

from __future__ import annotations

import pytest

from rwkv_b200.residency import hot_layer_order, layer_of, plan_residency


def test_hot_layer_order_is_outermost_first():
    assert hot_layer_order(0) == []
    assert hot_layer_order(1) == [0]
    assert hot_layer_order(4) == [0, 3, 1, 2]
    assert hot_layer_order(5) == [0, 4, 1, 3, 2]
    for n in range(1, 40):
        order = hot_layer_order(n)
        assert sorted(order) == list(range(n))


def test_layer_of_names():
    assert layer_of("blocks.0.att.receptance.weight") == 0
    assert layer_of("blocks.31.ffn.value.weight") == 31
    assert layer_of("emb.weight") == -1
    assert layer_of("head.weight") == -1
    assert layer_of("ln_out.weight") == -1
    assert layer_of("xblocks.3.att") == -1


def test_plan_without_budget_or_when_everything_fits():
    sizes = {i: 100 for i in range(4)}
    assert plan_residency(sizes, 50, 4, hbm_budget=None) == []
    assert plan_residency(sizes, 50, 4, hbm_budget=450) == []  # exactly the model
    assert plan_residency(sizes, 50, 4, hbm_budget=10 ** 12) == []


def test_plan_keeps_the_outermost_layers_that_fit():
    sizes = {i: 100 for i in range(4)}
    # globals 50 + two slots of 100 + one layer
    assert plan_residency(sizes, 50, 4, hbm_budget=350) == [1, 2, 3]
    # 6 layers, room for two beside the slots: the first and the last stay
    six = {i: 100 for i in range(6)}
    assert plan_residency(six, 50, 6, hbm_budget=450) == [1, 2, 3, 4]
    assert plan_residency(six, 50, 6, hbm_budget=550) == [2, 3, 4]  # 0, 5, then 1
    # room for the globals and the slots only: every layer streams
    assert plan_residency(sizes, 50, 4, hbm_budget=250) == [0, 1, 2, 3]


def test_plan_skips_a_layer_that_does_not_fit_and_goes_on():
    sizes = {0: 100, 1: 10, 2: 10, 3: 300}
    # one slot of 300 B; room 119: layer 0 (100) fits, 3 (300) does not,
    # 1 (10) fits, 2 (10) no longer does
    assert plan_residency(sizes, 0, 4, hbm_budget=419, n_slots=1) == [2, 3]


def test_plan_reserves_one_device_slot_per_ring_slot():
    sizes = {i: 100 for i in range(4)}
    # budget 349: one slot leaves room for layer 0, two slots for none
    assert plan_residency(sizes, 50, 4, hbm_budget=349, n_slots=1) == [1, 2, 3]
    assert plan_residency(sizes, 50, 4, hbm_budget=349, n_slots=2) == [0, 1, 2, 3]


def test_plan_rejects_a_budget_below_the_globals_and_slots():
    sizes = {i: 100 for i in range(4)}
    with pytest.raises(ValueError):
        plan_residency(sizes, 50, 4, hbm_budget=249)


def test_explicit_resident_layers_win_over_the_budget():
    sizes = {i: 100 for i in range(4)}
    assert plan_residency(sizes, 50, 4, hbm_budget=None, resident_layers=[1, 2]) == [0, 3]
    assert plan_residency(sizes, 50, 4, hbm_budget=1, resident_layers=[0, 1, 2, 3]) == []


def test_blob_placement_keeps_code_payloads_16_byte_aligned():
    """Blobs packed back to back into one device image: each starts on a
    256-byte boundary plus the padding that puts its code payload (after the
    header and group records) on the 16-byte boundary the bulk copies need;
    no two blobs overlap."""
    from rwkv_b200 import synth
    from rwkv_b200.residency import _meta_bytes, _place

    shape = synth.PRESETS["tiny"]
    sd = synth.generate_state_dict(shape, 4, "cpu")
    for policy in ("sg8", "lut2"):
        pack = synth.make_pack(sd, policy=policy)
        items = [(n, e.payload, tuple(e.shape), e.codec) for n, e in pack.items() if e.codec != "none"]
        assert {c for *_, c in items} >= ({"sg8"} if policy == "sg8" else {"sg8", "lut2"})
        offs, heads, total = _place(items)
        end = 0
        for (name, payload, shp, _codec), off, head in zip(items, offs, heads):
            meta = _meta_bytes(head, shp[0], shp[1])
            assert (off + meta) % 16 == 0, name
            assert off % 8 == 0 and off >= end, name
            assert off - end < 256 + 16, name  # no more padding than the two alignments
            end = off + len(payload)
        assert total == end
