"""Failure detection of the expert-parallel exchange on one GPU, without a fault.

Two mailboxes in one process stand for two ranks.  ``combine_ep`` waits, bounded
(~2 s), until every rank raised its flag in this rank's mailbox to the call's
epoch.  When the other rank never signals (a flag nothing sets) the wait runs out:
the kernel returns, the workspace error word carries the timeout bit, the output is
zero and the context stays usable.  When a second shard object plays the other
rank on the same stream (its rows and flag land before the combine runs, so no
kernel waits on another), the exchange reproduces the single-GPU layer bit for bit.
"""
import ctypes

import pytest
import torch

from flyai_b200 import _lib, synth
from flyai_b200.moe import Mxfp4MoE

pytestmark = pytest.mark.gpu
K_ERR_WAIT_TIMEOUT = 1


def _mailboxes(shard, n):
    nbytes = ctypes.c_size_t()
    _lib.call("flyai_moe_ep_mailbox_bytes", ctypes.byref(shard.desc), ctypes.byref(nbytes))
    boxes = []
    for _ in range(n):
        ptr = ctypes.c_void_p()
        _lib.call("flyai_moe_ep_alloc", nbytes, ctypes.byref(ptr))
        boxes.append(ptr)
    return boxes


class _RawInt32:
    """A device buffer the library allocated, seen by torch without a copy."""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = dict(shape=(n,), typestr="<i4", data=(ptr, False),
                                             version=3)


def _flag_words(box, n=64):
    """The first n int32 words of a mailbox (flags, then failure words) as a tensor."""
    return torch.as_tensor(_RawInt32(box.value, n), device="cuda")


def _peers(boxes, rank, epoch):
    p = _lib.EpPeers()
    p.world, p.rank, p.epoch, p.reserved = len(boxes), rank, epoch, 0
    for r, b in enumerate(boxes):
        p.mailbox[r] = b.value
    return p


@pytest.fixture(scope="module")
def layer():
    return synth.make_gpt_oss_layer(**synth.GPT_OSS_20B, seed=7)


def test_combine_wait_expires_when_a_rank_never_signals(layer):
    E = layer.router_w.shape[0]
    x = synth.make_tokens(5, layer.router_w.shape[1], seed=8).cuda()
    rank0 = Mxfp4MoE.from_layer(layer, expert_range=(0, E // 2), max_tokens=8, device="cuda")
    boxes = _mailboxes(rank0, 2)
    try:
        peers = _peers(boxes, 0, 1)
        rank0.route(x, logits=False)
        assert rank0.experts_ep(x, peers) == _lib.OK
        y = rank0.combine_ep(5, peers)          # rank 1's flag stays 0: the wait runs out
        torch.cuda.synchronize()
        bits, _ = rank0.read_error()
        assert bits & K_ERR_WAIT_TIMEOUT
        assert torch.count_nonzero(y) == 0
        # the context is still usable: a plain single-GPU call after the timeout is clean
        full = Mxfp4MoE.from_layer(layer, max_tokens=8, device="cuda")
        y_full, _, _ = full.forward(x)
        torch.cuda.synchronize()
        assert torch.isfinite(y_full.float()).all()
        assert full.read_error()[0] == 0
    finally:
        torch.cuda.synchronize()
        for b in boxes:
            _lib.call("flyai_moe_ep_free", b)


def test_two_shards_in_one_process_reproduce_the_layer(layer):
    E = layer.router_w.shape[0]
    x = synth.make_tokens(5, layer.router_w.shape[1], seed=9).cuda()
    shards = [Mxfp4MoE.from_layer(layer, expert_range=(r * E // 2, (r + 1) * E // 2), max_tokens=8,
                                  device="cuda") for r in range(2)]
    full = Mxfp4MoE.from_layer(layer, max_tokens=8, device="cuda")
    y_full, _, _ = full.forward(x)
    boxes = _mailboxes(shards[0], 2)
    try:
        for epoch in (1, 2):                  # both mailbox halves (epoch parity)
            for r in (1, 0):                  # rank 1's rows and flag land first
                shards[r].route(x, logits=False)
                assert shards[r].experts_ep(x, _peers(boxes, r, epoch)) == _lib.OK
            y = shards[0].combine_ep(5, _peers(boxes, 0, epoch))
            torch.cuda.synchronize()
            assert shards[0].read_error()[0] == 0
            assert torch.equal(y, y_full), epoch
    finally:
        torch.cuda.synchronize()
        for b in boxes:
            _lib.call("flyai_moe_ep_free", b)


@pytest.mark.parametrize("M", [1, 5, 16])
def test_one_launch_shards_reproduce_the_layer(layer, M):
    """flyai_moe_forward_ep: each shard's single launch routes every token, runs its
    own experts and stores their pair rows into both mailboxes; the combine then
    equals the single-GPU layer bit for bit, and the routing outputs equal it too.
    Both shards run in one process on one stream (rows and flags land before the
    combine, so nothing waits on another launch)."""
    E, H = layer.router_w.shape
    x = synth.make_tokens(M, H, seed=11 + M).cuda()
    shards = [Mxfp4MoE.from_layer(layer, expert_range=(r * E // 2, (r + 1) * E // 2), max_tokens=16,
                                  device="cuda") for r in range(2)]
    full = Mxfp4MoE.from_layer(layer, max_tokens=16, device="cuda")
    y_full, ids_full, wts_full = full.forward(x)
    boxes = _mailboxes(shards[0], 2)
    try:
        for epoch in (1, 2):                  # both mailbox halves (epoch parity)
            ids = torch.empty_like(ids_full)
            wts = torch.empty_like(wts_full)
            for r in (1, 0):
                assert shards[r].forward_ep(x, _peers(boxes, r, epoch), ids, wts) == _lib.OK
            y = shards[0].combine_ep(M, _peers(boxes, 0, epoch))
            torch.cuda.synchronize()
            assert shards[0].read_error()[0] == 0 and shards[1].read_error()[0] == 0
            assert torch.equal(y, y_full), epoch
            assert torch.equal(ids, ids_full) and torch.equal(wts, wts_full)
    finally:
        torch.cuda.synchronize()
        for b in boxes:
            _lib.call("flyai_moe_ep_free", b)


def test_combine_reports_a_rank_whose_expert_kernel_gave_up(layer):
    """A rank whose expert kernel gave up on a bounded wait raises its failure word
    to the epoch before its flag.  Here rank 1's flag and failure word are written
    from the host (the expert kernel's path to them needs a wait that runs out);
    rank 0's combine then folds nothing, reports the timeout bit and returns zeros
    instead of a layer missing rank 1's rows."""
    E = layer.router_w.shape[0]
    x = synth.make_tokens(5, layer.router_w.shape[1], seed=10).cuda()
    rank0 = Mxfp4MoE.from_layer(layer, expert_range=(0, E // 2), max_tokens=8, device="cuda")
    boxes = _mailboxes(rank0, 2)
    try:
        epoch = 1
        peers = _peers(boxes, 0, epoch)
        words = _flag_words(boxes[0])
        words[1] = epoch           # rank 1's flag in rank 0's mailbox
        words[16 + 1] = epoch      # and its failure word (kEpFailWord + rank)
        rank0.route(x, logits=False)
        assert rank0.experts_ep(x, peers) == _lib.OK
        y = rank0.combine_ep(5, peers)
        torch.cuda.synchronize()
        bits, _ = rank0.read_error()
        assert bits & K_ERR_WAIT_TIMEOUT
        assert torch.count_nonzero(y) == 0
        # a later epoch without a failure word folds normally again
        shard1 = Mxfp4MoE.from_layer(layer, expert_range=(E // 2, E), max_tokens=8, device="cuda")
        full = Mxfp4MoE.from_layer(layer, max_tokens=8, device="cuda")
        y_full, _, _ = full.forward(x)
        for r, sh in ((1, shard1), (0, rank0)):
            sh.route(x, logits=False)
            assert sh.experts_ep(x, _peers(boxes, r, 2)) == _lib.OK
        y2 = rank0.combine_ep(5, _peers(boxes, 0, 2))
        torch.cuda.synchronize()
        assert rank0.read_error()[0] == 0
        assert torch.equal(y2, y_full)
    finally:
        torch.cuda.synchronize()
        for b in boxes:
            _lib.call("flyai_moe_ep_free", b)
