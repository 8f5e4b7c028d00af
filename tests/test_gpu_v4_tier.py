"""The V4 expert tier on the B200: routed experts in pinned host memory, a few
device slots (flyai_moe_experts_slots), against the same layer on the full bank
(W4A8MoE), bit for bit, score- and hash-routed, through loads, hits, evictions and
batches that run in token groups."""
import pytest
import torch

from flyai_b200 import synth
from flyai_b200.v4 import W4A8MoE
from flyai_b200.v4_tier import TieredW4A8MoE

pytestmark = pytest.mark.gpu

SMALL = dict(num_experts=32, top_k=6, hidden=256, inter=256)


@pytest.mark.parametrize("hash_vocab", [0, 8])
def test_tier_matches_full_bank(hash_vocab):
    layer = synth.make_v4_layer(**SMALL, seed=4, hash_vocab=hash_vocab, device="cuda")
    full = W4A8MoE.from_layer(layer, max_tokens=16)
    tier = TieredW4A8MoE.from_layer(layer, slots=10, max_tokens=16)
    for step, M in enumerate((1, 1, 2, 5, 16, 1, 3)):
        x = synth.make_tokens(M, SMALL["hidden"], seed=100 + step, device="cuda")
        ids = (torch.arange(M, device="cuda") * 3 + step) % 8 if hash_vocab else None
        want = full.forward(x, ids)
        got = tier.forward(x, ids)
        assert torch.equal(got, want), (step, M)
    st = tier.stats()
    assert st["loads"] > 10 and st["hits"] > 0 and st["resident"] == 10   # evictions happened
    assert tier.read_error()[0] == 0 and full.read_error()[0] == 0


def test_one_slot_per_expert_of_a_token():
    """slots == top_k: every token is its own group."""
    layer = synth.make_v4_layer(**SMALL, seed=9, device="cuda")
    full = W4A8MoE.from_layer(layer, max_tokens=8)
    tier = TieredW4A8MoE.from_layer(layer, slots=6, max_tokens=8)
    x = synth.make_tokens(8, SMALL["hidden"], seed=9, device="cuda")
    assert torch.equal(tier.forward(x), full.forward(x))
    with pytest.raises(ValueError):
        TieredW4A8MoE.from_layer(layer, slots=5, max_tokens=8).forward(x)
