"""Host logic of the V4 expert tier (flyai_b200/v4_tier.py): token grouping and
the least-recently-used slot assignment."""
import numpy as np
import pytest

from flyai_b200.v4_tier import SlotCache, token_groups


def test_token_groups_fit_the_slots_and_cover_every_token():
    rng = np.random.default_rng(0)
    ids = np.stack([rng.choice(32, 6, replace=False) for _ in range(20)])
    for slots in (6, 8, 13, 32):
        groups = token_groups(ids, slots)
        assert groups[0][0] == 0 and groups[-1][1] == 20
        assert all(a < b for a, b in groups)
        assert all(groups[i][1] == groups[i + 1][0] for i in range(len(groups) - 1))
        for a, b in groups:
            assert len(set(ids[a:b].ravel())) <= slots
    assert token_groups(ids, 32) == [(0, 20)]
    assert token_groups(ids[:0], 8) == []
    with pytest.raises(ValueError):
        token_groups(ids, 5)


def test_slot_cache_reuses_and_evicts_least_recent_not_in_use():
    c = SlotCache(4)
    slot, loads = c.assign([3, 7])
    assert sorted(loads) == sorted((e, slot[e]) for e in (3, 7)) and c.loads == 2
    slot2, loads = c.assign([7, 9, 11])
    assert slot2[7] == slot[7] and [e for e, _ in loads] == [9, 11] and c.hits == 1
    # 3 is now the least recent and not wanted: it makes room for 12
    slot3, loads = c.assign([12, 9])
    assert loads == [(12, slot[3])]
    assert len(set(slot3.values())) == 2
    t = c.table(16)
    assert t[3] == -1 and t[12] == slot[3] and set(t[t >= 0]) <= set(range(4))
    with pytest.raises(ValueError):
        c.assign([0, 1, 2, 4, 5])


def test_slot_cache_never_evicts_an_expert_of_the_same_call():
    c = SlotCache(3)
    c.assign([0, 1, 2])
    slot, loads = c.assign([2, 5, 0])          # 1 is the only one free to go
    assert [e for e, _ in loads] == [5] and set(slot.values()) == {0, 1, 2}
