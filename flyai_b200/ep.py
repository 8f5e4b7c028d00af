"""Expert parallelism for one MoE layer across the GPUs of a box.

The reference's only expert-parallel pattern (vendor/deepseek_v4_ref/inference/
model.py:620-647): rank r owns experts [r*E/W, (r+1)*E/W), every rank routes
the same tokens, computes its own experts, and an all-reduce of the partial
outputs gives every rank the layer output.  Here the exchanged tensor is the
[M*k, H] matrix of weighted per-(token, slot) expert rows rather than a partial
sum: each row is produced by exactly one rank and the others contribute zeros,
so the all-reduce rebuilds every row bit-exactly whatever order NCCL adds in,
and each rank then folds a token's k rows in ascending expert id with bf16
rounding after every add -- the reference's own accumulation order
(transformers/models/gpt_oss/modeling_gpt_oss.py:96-112).  The result is
identical on every rank and identical to the single-GPU layer.

Per step: route (replicated, identical ids) -> local experts -> exchange of the
pair rows -> combine.  With ``broadcast`` (the default) x is meaningful on
``src`` only -- the stage that owns the tokens -- and is broadcast first; with
``broadcast=False`` every rank already holds the same x, as in the reference's
pattern, and the step starts at the route.  With ``p2p`` (the default on GPUs) a verify-size call is
one launch per rank (flyai_moe_forward_ep: the routing in the expert kernel's
prologue, each pair row stored straight into every rank's mailbox over NVLink
through CUDA IPC mappings made once at set-up, a per-rank flag raised at the
end) and the combine waits for all flags.  The fallback, and the path of shapes
the peer-memory kernel does not take, is an NCCL all-reduce of the rows.
Collectives run on torch.distributed (NCCL on GPUs, gloo in the CPU tests).
"""
import ctypes

import torch

from . import _lib


def expert_range(num_experts, world, rank):
    """Contiguous expert shard of ``rank`` (model.py:620-626 partitioning)."""
    if num_experts % world:
        raise ValueError(f"{num_experts} experts do not divide over {world} ranks")
    per = num_experts // world
    return rank * per, (rank + 1) * per


class PeerMailboxes:
    """This rank's pair-row mailbox (flyai_moe_ep_alloc) and every other rank's,
    opened through CUDA IPC on this rank's device; ``peers`` is the
    flyai_moe_ep_peers block handed to the kernels, ``next_epoch`` numbers calls."""

    def __init__(self, shard, group=None):
        import torch.distributed as dist
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        if world > _lib.EP_MAX_RANKS:
            raise ValueError(f"peer-memory expert parallel takes at most {_lib.EP_MAX_RANKS} ranks")
        nbytes = ctypes.c_size_t()
        _lib.call("flyai_moe_ep_mailbox_bytes", ctypes.byref(shard.desc), ctypes.byref(nbytes))
        self.device = shard.device
        self._opened = []
        mine = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.call("flyai_moe_ep_alloc", nbytes, ctypes.byref(mine))
        self._mine = mine
        handle = (ctypes.c_uint8 * 64)()
        _lib.call("flyai_moe_ipc_get_handle", mine, handle)
        t = torch.tensor(list(handle), dtype=torch.uint8, device=self.device)
        gathered = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(gathered, t, group=group)
        self.peers = _lib.EpPeers(world=world, rank=rank, epoch=0, reserved=0)
        for r, g in enumerate(gathered):
            if r == rank:
                self.peers.mailbox[r] = mine.value
                continue
            h = (ctypes.c_uint8 * 64)(*g.cpu().tolist())
            ptr = ctypes.c_void_p()
            with torch.cuda.device(self.device):
                _lib.call("flyai_moe_ipc_open", h, ctypes.byref(ptr))
            self._opened.append(ptr)
            self.peers.mailbox[r] = ptr.value
        dist.barrier(group=group)   # every rank mapped every mailbox before the first call

    def next_epoch(self):
        self.peers.epoch += 1
        return self.peers

    def close(self):
        with torch.cuda.device(self.device):
            torch.cuda.synchronize()
            for ptr in self._opened:
                _lib.call("flyai_moe_ipc_close", ptr)
            self._opened = []
            if self._mine:
                _lib.call("flyai_moe_ep_free", self._mine)
                self._mine = None


class ExpertParallelMoE:
    """Drives a shard object with the ``route / experts_pairs / combine`` surface
    of ``flyai_b200.moe.Mxfp4MoE`` over a process group; with ``p2p`` (and a
    shard that has ``experts_ep``) the pair-row exchange goes through peer
    memory, see the module docstring."""

    def __init__(self, shard, group=None, src=0, p2p=True, broadcast=True):
        import torch.distributed as dist
        self.dist = dist
        self.shard = shard
        self.group = group
        self.src = src
        self.broadcast = broadcast
        self._pairs = None
        self.mail = None
        if p2p and hasattr(shard, "experts_ep") and dist.get_world_size(group) > 1:
            self.mail = PeerMailboxes(shard, group)

    def forward(self, x, out=None, ids=None, wts=None):
        """x: [M, H] bf16, the same on every rank (with ``broadcast``: meaningful on
        ``src``, overwritten elsewhere) -> y on every rank.  ids / wts: optional
        routing outputs of the one-launch path."""
        d = self.dist
        if self.broadcast:
            d.broadcast(x, src=self.src, group=self.group)
        M = x.shape[0]
        if self.mail is not None and hasattr(self.shard, "forward_ep"):
            peers = self.mail.next_epoch()
            if self.shard.forward_ep(x, peers, ids, wts) == _lib.OK:
                return self.shard.combine_ep(M, peers, out)
            self.mail.peers.epoch -= 1   # shape without the one-launch path: same on every rank
        self.shard.route(x, logits=False)
        if self.mail is not None:
            peers = self.mail.next_epoch()
            if self.shard.experts_ep(x, peers) == _lib.OK:
                return self.shard.combine_ep(M, peers, out)
            self.mail.peers.epoch -= 1   # shape without a peer-memory path: same on every rank
        rows = self.shard.experts_pairs(x, self._pair_buffer(M, x))
        d.all_reduce(rows, group=self.group)
        if out is not None:
            return self.shard.combine(rows, M, out)
        return self.shard.combine(rows, M)

    def close(self):
        if self.mail is not None:
            self.mail.close()
            self.mail = None

    def _pair_buffer(self, M, x):
        need = self.shard.pair_rows(M) if hasattr(self.shard, "pair_rows") else M * self.shard.top_k
        if self._pairs is None or self._pairs.shape[0] < need or self._pairs.device != x.device:
            self._pairs = torch.empty(max(need, 1), self.shard.hidden, dtype=torch.bfloat16,
                                      device=x.device)
        return self._pairs[:need]


class PairExperts:
    """A shard's experts applied to (token row, expert, routing weight) triples
    that other ranks sent: the shard's banks under an MXFP4 descriptor with caller
    routing (FLYAI_GATE_EXTERNAL) and one slot per row.  ``run`` returns the
    weighted bf16 rows, computed as the shard's own pair rows are."""

    def __init__(self, shard, max_rows=4096):
        self.shard = shard
        self.max_rows = max_rows
        self.desc = _lib.Desc.from_buffer_copy(shard.desc)
        self.desc.gating = _lib.GATE_EXTERNAL
        self.desc.top_k = 1
        self.desc.max_tokens = max_rows
        _lib.call("flyai_moe_check_desc", ctypes.byref(self.desc))
        nbytes = ctypes.c_size_t()
        _lib.call("flyai_moe_workspace_bytes", ctypes.byref(self.desc), ctypes.byref(nbytes))
        self.workspace = torch.zeros(nbytes.value, dtype=torch.uint8, device=shard.device)

    def run(self, rows, ids, wts, out=None):
        """rows bf16 [R, H]; ids int32 [R] (experts of this shard); wts fp32 [R]."""
        from .moe import _ptr, _stream
        R = rows.shape[0]
        out = out if out is not None else torch.empty_like(rows)
        ws = self.workspace
        with torch.cuda.device(self.shard.device):
            for r0 in range(0, R, self.max_rows):
                m = min(self.max_rows, R - r0)
                _lib.call("flyai_moe_route_ids", ctypes.byref(self.desc), m, _ptr(ids[r0:r0 + m]),
                          _ptr(wts[r0:r0 + m]), _ptr(ws), ws.numel(), _stream())
                _lib.call("flyai_moe_experts_pairs", ctypes.byref(self.desc), m, _ptr(rows[r0:r0 + m]),
                          ctypes.byref(self.shard.weights), _ptr(out[r0:r0 + m]), _ptr(ws), ws.numel(),
                          _stream())
        return out


class TokenShardedMoE:
    """Expert parallel with the tokens sharded by rank (prefill): each rank routes
    its own tokens over all experts, sends each (token, slot) pair's token row to
    the rank owning the expert (NCCL all-to-all, counts first), the owners compute
    the weighted rows (``pairs.run``) and send them back, and each rank folds its
    tokens' k rows with the layer's own combine -- every row crosses the links
    once each way, where the replicated path all-reduces the whole [M*k, H] pair
    matrix (the expert sharding of vendor/deepseek_v4_ref/inference/model.py:620-647,
    with each row moved once to its expert's owner instead of an all-reduce).
    ``shard``: this rank's layer shard (route, combine); ``pairs``: its
    ``PairExperts``.  Output for a rank's tokens equals the single-GPU layer's."""

    def __init__(self, shard, pairs, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.shard, self.pairs, self.group = shard, pairs, group
        self.world = dist.get_world_size(group)

    def forward(self, x, out=None):
        """x: this rank's tokens, bf16 [M_r, H] -> y for them."""
        d, g, W = self.dist, self.group, self.world
        sh = self.shard
        M, H, k = x.shape[0], sh.hidden, sh.top_k
        per = sh.num_experts // W
        if M > 0:
            _, ids, wts = sh.route(x, logits=False)
            ids = torch.as_tensor(ids).to(x.device).reshape(-1).to(torch.int32)
            wts = torch.as_tensor(wts).to(x.device).reshape(-1).float()
        else:
            ids = torch.empty(0, dtype=torch.int32, device=x.device)
            wts = torch.empty(0, dtype=torch.float32, device=x.device)
        dest = ids.long() // per
        order = torch.sort(dest, stable=True).indices          # pairs grouped by owner rank
        send = torch.bincount(dest, minlength=W).to(torch.int64)
        recv = torch.empty_like(send)
        d.all_to_all_single(recv, send, group=g)
        sc, rc = send.tolist(), recv.tolist()                    # split sizes (host)
        R = sum(rc)
        rows_recv = x.new_empty(R, H)
        d.all_to_all_single(rows_recv, x[order // k].contiguous(), rc, sc, group=g)
        ids_recv = torch.empty(R, dtype=torch.int32, device=x.device)
        d.all_to_all_single(ids_recv, ids[order].contiguous(), rc, sc, group=g)
        wts_recv = torch.empty(R, dtype=torch.float32, device=x.device)
        d.all_to_all_single(wts_recv, wts[order].contiguous(), rc, sc, group=g)
        done = self.pairs.run(rows_recv, ids_recv, wts_recv) if R else rows_recv
        back = x.new_empty(M * k, H)
        d.all_to_all_single(back, done.contiguous(), sc, rc, group=g)
        pair_out = x.new_empty(M * k, H)
        pair_out[order] = back
        if M == 0:
            return out if out is not None else x.new_empty(0, H)
        if out is not None:
            return sh.combine(pair_out, M, out)
        return sh.combine(pair_out, M)
