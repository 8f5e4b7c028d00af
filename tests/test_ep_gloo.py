"""Expert-parallel host logic (flyai_b200/ep.py) on two CPU ranks over gloo.

Each rank drives ExpertParallelMoE with a shard whose route / experts_pairs /
combine are the CPU oracle restricted to the rank's expert range, so the test
checks the parts ep.py owns -- broadcast of x from the source rank, the
all-reduce of the weighted pair rows, the combine in ascending expert id --
against the single-process full layer, bit for bit, on every rank.  The GPU
kernels behind the same surface are covered by tests/test_gpu_moe.py
(expert-sharded sums equal the full layer)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flyai_b200 import synth
from flyai_b200.ep import ExpertParallelMoE, TokenShardedMoE, expert_range
from oracle import gpt_oss as og
from oracle.fp import round_bf16
from tests.golden_util import oracle_weights


class OracleShard:
    """The Mxfp4MoE shard surface, computed by the numpy oracle on the CPU."""

    def __init__(self, layer, lo, hi):
        self.w = oracle_weights(layer)
        self.lo, self.hi = lo, hi
        self.top_k = layer.top_k
        self.hidden = layer.hidden
        self.num_experts = layer.num_experts

    def route(self, x, logits=True):
        _, self.ids, self.wts = og.router(x.float().numpy(), self.w.router_w, self.w.router_b,
                                          self.top_k)
        return None, self.ids, self.wts

    def experts_pairs(self, x, out):
        xf = x.float().numpy()
        rows = np.zeros((xf.shape[0] * self.top_k, self.hidden), dtype=np.float32)
        for e in range(self.lo, self.hi):
            tok, slot = np.nonzero(self.ids == e)
            if tok.size == 0:
                continue
            y, _ = og.expert_forward(xf[tok], self.w, e)
            rows[tok * self.top_k + slot] = round_bf16(y * self.wts[tok, slot][:, None])
        out.copy_(torch.from_numpy(rows).bfloat16())
        return out

    def combine(self, rows, M):
        r = rows.float().numpy().reshape(M, self.top_k, self.hidden)
        y = np.zeros((M, self.hidden), dtype=np.float32)
        for t in range(M):
            for s in np.argsort(self.ids[t], kind="stable"):   # ascending expert id
                y[t] = round_bf16(y[t] + r[t, s])
        return torch.from_numpy(y).bfloat16()


class OraclePairs:
    """PairExperts' surface: a shard's experts on (row, expert, weight) triples."""

    def __init__(self, shard):
        self.shard = shard

    def run(self, rows, ids, wts):
        xf, ids, wts = rows.float().numpy(), ids.numpy(), wts.numpy()
        out = np.zeros_like(xf)
        for e in np.unique(ids):
            assert self.shard.lo <= e < self.shard.hi   # only this rank's experts arrive
            r = np.nonzero(ids == e)[0]
            y, _ = og.expert_forward(xf[r], self.shard.w, int(e))
            out[r] = round_bf16(y * wts[r][:, None])
        return torch.from_numpy(out).bfloat16()


def _sharded_main(rank, world, port, cuts, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    y = None
    try:
        layer = synth.make_gpt_oss_layer(num_experts=8, top_k=2, hidden=64, inter=64, seed=5)
        lo, hi = expert_range(8, world, rank)
        shard = OracleShard(layer, lo, hi)
        moe = TokenShardedMoE(shard, OraclePairs(shard))
        x = synth.make_tokens(7, 64, seed=11)
        y = moe.forward(x[cuts[rank]:cuts[rank + 1]]).float().numpy()   # uneven, possibly empty
    finally:
        q.put((rank, y))          # also after a failure, so the parent never waits forever
        dist.destroy_process_group()


@pytest.mark.parametrize("cuts", [(0, 3, 7), (0, 0, 7), (0, 7, 7, 7, 7)])
def test_token_sharded_ranks_match_full_layer(cuts):
    """Each rank routes its own tokens (none on some ranks); rows go to the expert
    owner and back; the ranks' outputs stacked are the full layer's."""
    world = len(cuts) - 1
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sharded_main, args=(r, world, port, cuts, q), daemon=True)
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        got = dict(q.get(timeout=120) for _ in range(world))   # small payloads, read first
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(got[r] is not None for r in range(world)), "a rank failed"
    layer = synth.make_gpt_oss_layer(num_experts=8, top_k=2, hidden=64, inter=64, seed=5)
    x = synth.make_tokens(7, 64, seed=11)
    ref = og.moe_forward(x.float().numpy(), oracle_weights(layer), 2)["y"]
    np.testing.assert_array_equal(np.concatenate([got[r] for r in range(world)]), ref)


def _rank_main(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        layer = synth.make_gpt_oss_layer(num_experts=8, top_k=2, hidden=64, inter=64, seed=4)
        lo, hi = expert_range(8, world, rank)
        moe = ExpertParallelMoE(OracleShard(layer, lo, hi), src=0)
        x = synth.make_tokens(5, 64, seed=9) if rank == 0 else torch.zeros(5, 64,
                                                                           dtype=torch.bfloat16)
        y = moe.forward(x)
        q.put((rank, y.float().numpy(), x.float().numpy()))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_expert_parallel_two_ranks_matches_full_layer():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    got = dict((r, (y, x)) for r, y, x in (q.get() for _ in range(world)))
    layer = synth.make_gpt_oss_layer(num_experts=8, top_k=2, hidden=64, inter=64, seed=4)
    x = synth.make_tokens(5, 64, seed=9)
    ref = og.moe_forward(x.float().numpy(), oracle_weights(layer), 2)["y"]
    for r in range(world):
        y, xr = got[r]
        np.testing.assert_array_equal(xr, x.float().numpy())   # broadcast reached every rank
        np.testing.assert_array_equal(y, ref)


def test_expert_range_partitions():
    assert [expert_range(128, 4, r) for r in range(4)] == [(0, 32), (32, 64), (64, 96), (96, 128)]
    try:
        expert_range(10, 4, 0)
    except ValueError:
        pass
    else:
        raise AssertionError("uneven split accepted")


class Dsv3OracleShard:
    """The Fp8MoE shard surface computed by the numpy oracle: this rank's routed
    experts' rows by flat pair index, then the shared expert's rows (rank holding
    expert 0 only); the combine is MoE.forward's fp32 fold."""

    def __init__(self, layer, lo, hi):
        from oracle import dsv3 as od
        self.od, self.layer, self.lo, self.hi = od, layer, lo, hi
        self.top_k, self.hidden = layer.top_k, layer.hidden
        self.cache = {}

    def expert(self, e):
        if e not in self.cache:
            w13, s13, w2, s2 = self.layer.expert(e)
            self.cache[e] = (w13.view(torch.uint8).numpy(), s13.numpy(), w2.view(torch.uint8).numpy(),
                             s2.numpy())
        return self.cache[e]

    def pair_rows(self, M):
        return M * (self.top_k + 1)

    def route(self, x, logits=True):
        L = self.layer
        self.ids, self.wts, _ = self.od.gate(x.float().numpy(), L.router_w.float().numpy(),
                                             L.bias.numpy(), L.top_k, L.n_group, L.topk_group,
                                             L.route_scale)
        return None, self.ids, self.wts

    def experts_pairs(self, x, out):
        xf = x.float().numpy()
        M, k, E = xf.shape[0], self.top_k, self.layer.num_experts
        rows = np.zeros((M * (k + 1), self.hidden), dtype=np.float32)
        for e in range(self.lo, self.hi):
            tok, slot = np.nonzero(self.ids == e)
            if tok.size:
                rows[tok * k + slot] = self.od.expert_forward(xf[tok], *self.expert(e),
                                                              weights=self.wts[tok, slot])
        if self.lo == 0:
            rows[M * k:] = self.od.expert_forward(xf, *self.expert(E))
        out.copy_(torch.from_numpy(rows).bfloat16())
        return out

    def combine(self, rows, M):
        r = rows.float().numpy()
        k = self.top_k
        y = np.zeros((M, self.hidden), dtype=np.float32)
        for t in range(M):
            for s in np.argsort(self.ids[t], kind="stable"):
                y[t] = (y[t] + r[t * k + s]).astype(np.float32)
            y[t] = (y[t] + r[M * k + t]).astype(np.float32)
        return torch.from_numpy(round_bf16(y)).bfloat16()


def _dsv3_rank_main(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        layer = synth.make_dsv3_layer(num_experts=32, top_k=4, hidden=256, inter=128, n_group=4,
                                      topk_group=2, seed=6)
        lo, hi = expert_range(32, world, rank)
        moe = ExpertParallelMoE(Dsv3OracleShard(layer, lo, hi), src=0)
        x = synth.make_tokens(6, 256, seed=3) if rank == 0 else torch.zeros(6, 256, dtype=torch.bfloat16)
        q.put((rank, moe.forward(x).float().numpy()))
    finally:
        dist.destroy_process_group()


def test_dsv3_expert_parallel_two_ranks_matches_full_layer():
    """The FP8 layer's pair rows carry the shared expert after the M*k pairs; the
    all-reduce and fold in ep.py must give the oracle's whole layer on every rank."""
    from oracle import dsv3 as od
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_dsv3_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    got = dict(q.get() for _ in range(world))
    layer = synth.make_dsv3_layer(num_experts=32, top_k=4, hidden=256, inter=128, n_group=4,
                                  topk_group=2, seed=6)
    sh = Dsv3OracleShard(layer, 0, 32)
    x = synth.make_tokens(6, 256, seed=3).float().numpy()
    ids, wts, _ = od.gate(x, layer.router_w.float().numpy(), layer.bias.numpy(), 4, 4, 2, 2.5)
    ref = od.moe_forward(x, ids, wts, sh.expert, 32)
    for r in range(world):
        np.testing.assert_array_equal(got[r], ref)
