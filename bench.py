"""Benchmark: GPT-OSS-120B-shaped MXFP4 MoE layer on B200 (one JSON line on rank 0).

Headline (N=1): one verify-step MoE layer call at M=5 tokens (config 1: E=128,
top-4, H=I=2880), microseconds per layer, inputs resident in HBM, L2 flushed
(256 MiB write) before every timed step.  Also reported: the same call end to
end through the public API with host buffers (H2D x, D2H y + router scores),
the prefill chunk (config 2: M=2048, Zipf(1.1)-skewed router) in tokens/s, the
roofline of the expert-streaming kernels, and the reference CPU path timed on
this host.  At N=1 the line also carries "families": the DeepSeek-V3 FP8 layer
(config 3), the MiniMax-M2.5 NVFP4 layer (config 4, with its M=4096 prefill) and
the DeepSeek-V4-Flash W4A8 layer, each with its verify-size sweep, expert-kernel
roofline, end-to-end time and CPU oracle timing, and "linear": the seven dense
FP8 GEMMs of a DeepSeek-V4-Flash decode layer (flyai_fp8_linear), and "k3": the
Kimi-K3 routed experts behind moe_infer (caller-routed MXFP4 with situ).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

N>1 (torchrun, one rank per GPU): expert parallel -- rank r holds experts
[r*E/N, (r+1)*E/N); every rank holds the step's tokens, routes them, computes
its experts' weighted rows in one launch and publishes them to its peers over
NVLink peer memory; each rank folds all shards' rows in ascending expert id.
Total work is fixed, so scaling is strong; time is the max over ranks.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from flyai_b200 import synth  # noqa: E402

METRIC = "MoE layer us at M=5 verify (GPT-OSS-120B MXFP4, E=128 top-4, H=I=2880)"
H = I = 2880
E, K_TOP = 128, 4


class L2Flush:
    """Evicts the L2 (126 MB) before every timed step.  "write" (default): a
    256 MiB write; "writeread": that write, then a 256 MiB read, so the write's
    dirty lines are written back to HBM before the step instead of during it (on
    the GPT-OSS verify layer the two measure the same, within 0.5 %)."""

    def __init__(self, dev, mode="write"):
        self.mode = mode
        self.w = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        self.r = torch.ones(32 << 20, dtype=torch.int64, device=dev) if mode == "writeread" else None
        self.sink = torch.empty((), dtype=torch.int64, device=dev)
        self.note = ("flushed before every timed step: 256 MiB written, then 256 MiB read "
                     "(the written lines' write-backs finish before the step)" if mode == "writeread"
                     else "flushed (256 MiB write) before every timed step")

    def __call__(self):
        self.w.zero_()
        if self.r is not None:
            torch.sum(self.r, dim=0, out=self.sink)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="flyai", choices=["flyai", "reference"])
    p.add_argument("--workload", default="gptoss", choices=["gptoss", "dsv3", "m25", "v4"],
                   help="gptoss: the headline (configs 1-2; at N=1 the line also carries the "
                        "dsv3 / m25 / v4 layers as sub-objects); dsv3: the DeepSeek-V3 FP8 layer "
                        "(config 3); m25: the MiniMax-M2.5 NVFP4 layer (config 4); v4: the "
                        "DeepSeek-V4-Flash W4A8 layer")
    p.add_argument("--tokens", type=int, default=None,
                   help="verify-step tokens (default: 5; 1 for dsv3 and v4)")
    p.add_argument("--no-families", action="store_true",
                   help="default run: leave out the dsv3 / m25 / v4 sub-objects")
    p.add_argument("--prefill-tokens", type=int, default=None,
                   help="prefill chunk size (default: 2048 for gptoss, config 2; 4096 for m25, config 4)")
    p.add_argument("--no-prefill", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--ep-nccl", action="store_true",
                   help="expert parallel exchange by NCCL all-reduce instead of peer memory")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--sustain", type=int, default=2000,
                   help="untimed steps run under the clock sampler before timing")
    p.add_argument("--l2", default="write", choices=["write", "writeread"],
                   help="L2 flush before each timed step: a 256 MiB write (default), or the "
                        "write then a 256 MiB read (its write-backs finish before the step)")
    p.add_argument("--no-linear", action="store_true",
                   help="default run: leave out the dense FP8 linear sub-object")
    p.add_argument("--ep-prefill", default="replicated", choices=["replicated", "tokens"],
                   help="N>1 prefill leg: every rank routes all tokens and the pair rows are "
                        "all-reduced (default), or tokens sharded by rank with rows sent to "
                        "their expert's owner by NCCL all-to-all")
    p.add_argument("--no-k3", action="store_true",
                   help="default run: leave out the Kimi-K3 moe_infer sub-object")
    return p.parse_args()


# ---------------------------------------------------------------------------
class ClockSampler:
    """Samples SM clock and clock-event (throttle) reasons through NVML in a
    background thread while the timed work runs (read-only queries)."""

    def __init__(self, torch_index, period_s=0.002):
        self.torch_index = torch_index
        self.period = period_s
        self.samples = []
        self.max_mhz = None
        self._stop = None

    def __enter__(self):
        import threading
        try:
            import pynvml
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(self.torch_index).uuid)
            h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        except Exception:
            return self
        self._stop = threading.Event()

        def loop():
            while not self._stop.is_set():
                try:
                    self.samples.append((pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
                                         pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)))
                except Exception:
                    pass
                self._stop.wait(self.period)
        self._thread = threading.Thread(target=loop, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._stop is not None:
            self._stop.set()
            self._thread.join(timeout=2)
        return False

    def summary(self):
        try:
            import pynvml
            bits = {"hw_slowdown": pynvml.nvmlClocksEventReasonHwSlowdown,
                    "hw_thermal_slowdown": pynvml.nvmlClocksEventReasonHwThermalSlowdown,
                    "sw_thermal_slowdown": pynvml.nvmlClocksEventReasonSwThermalSlowdown,
                    "sw_power_cap": pynvml.nvmlClocksEventReasonSwPowerCap}
        except Exception:
            bits = {}
        reasons = sorted({n for _, r in self.samples for n, b in bits.items() if r & b})
        sm = [c for c, _ in self.samples]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(sm)}


# ---------------------------------------------------------------------------
def reference_layer_cpu(layer_cpu, x_cpu):
    """The reference's CPU path for the layer: transformers' GptOssTopKRouter and
    eager GptOssExperts (transformers/models/gpt_oss/modeling_gpt_oss.py:69-131)
    on bf16 weights dequantised by _convert_moe_packed_tensors (dequant done
    once, outside the timed call).  Falls back to the numpy oracle port when
    transformers is unavailable.  Returns (callable, kind)."""
    from types import SimpleNamespace
    try:
        from transformers.integrations.mxfp4 import _convert_moe_packed_tensors
        from transformers.models.gpt_oss.modeling_gpt_oss import GptOssExperts, GptOssTopKRouter
    except Exception:  # pragma: no cover - image always has transformers
        return oracle_layer_cpu(layer_cpu, x_cpu), "port"
    Ecount = layer_cpu.router_w.shape[0]
    cfg = SimpleNamespace(num_experts_per_tok=layer_cpu.top_k, num_local_experts=Ecount,
                          hidden_size=H, intermediate_size=I, _experts_implementation="eager")
    router = GptOssTopKRouter(cfg)
    router.weight.data = layer_cpu.router_w
    router.bias.data = layer_cpu.router_b
    with torch.no_grad():
        _, _, idx = router(x_cpu)
    hit = sorted(set(idx.flatten().tolist()))
    experts = GptOssExperts.__new__(GptOssExperts)
    torch.nn.Module.__init__(experts)
    experts.config, experts.has_gate, experts.has_bias, experts.is_transposed = cfg, True, True, True
    experts.intermediate_size, experts.num_experts, experts.hidden_size = I, Ecount, H
    experts.alpha, experts.limit = layer_cpu.alpha, layer_cpu.limit
    # only the experts this batch touches are materialised; the others are never read
    gate_up = {e: _convert_moe_packed_tensors(layer_cpu.w13_blocks[e:e + 1], layer_cpu.w13_scales[e:e + 1])[0]
               for e in hit}
    down = {e: _convert_moe_packed_tensors(layer_cpu.w2_blocks[e:e + 1], layer_cpu.w2_scales[e:e + 1])[0]
            for e in hit}

    class _Bank:
        def __init__(self, d):
            self.d = d

        def __getitem__(self, e):
            return self.d[int(e)]

    experts.gate_up_proj = _Bank(gate_up)
    experts.down_proj = _Bank(down)
    experts.gate_up_proj_bias = layer_cpu.w13_bias
    experts.down_proj_bias = layer_cpu.w2_bias

    def run():
        with torch.no_grad():
            _, scores, ids = router(x_cpu)
            return experts(x_cpu, ids, scores)
    return run, "reference"


def oracle_layer_cpu(layer_cpu, x_cpu):
    from oracle import gpt_oss as og
    f = lambda t: t.float().numpy()
    w = og.GptOssWeights(f(layer_cpu.router_w), f(layer_cpu.router_b), layer_cpu.w13_blocks.numpy(),
                         layer_cpu.w13_scales.numpy(), f(layer_cpu.w13_bias), layer_cpu.w2_blocks.numpy(),
                         layer_cpu.w2_scales.numpy(), f(layer_cpu.w2_bias), layer_cpu.limit)
    xn = x_cpu.float().numpy()
    return lambda: og.moe_forward(xn, w, layer_cpu.top_k)


def cpu_layer_on_host(layer_dev, x_dev):
    """Copy the batch's touched experts to host memory and return the timed CPU callable."""
    layer_cpu = synth.GptOssLayer(
        layer_dev.router_w.cpu(), layer_dev.router_b.cpu(), layer_dev.w13_blocks.cpu(),
        layer_dev.w13_scales.cpu(), layer_dev.w13_bias.cpu(), layer_dev.w2_blocks.cpu(),
        layer_dev.w2_scales.cpu(), layer_dev.w2_bias.cpu(), layer_dev.top_k)
    return reference_layer_cpu(layer_cpu, x_dev.cpu())


def time_cpu(fn, budget_s=20.0, max_calls=20, warm=1):
    """Median seconds per call (and the min / max around it) over up to max_calls
    calls within about budget_s -- the one statistic both CPU timings report."""
    for _ in range(warm):
        fn()
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < max_calls and (not times or time.perf_counter() < t_end):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    return statistics.median(times), len(times), (min(times), max(times))


def cpu_spread_us(spread):
    return {"min_us": round(spread[0] * 1e6, 1), "max_us": round(spread[1] * 1e6, 1)}


# ---------------------------------------------------------------------------
def touched_bytes(ids):
    distinct = int(torch.unique(ids.flatten()).numel())
    per_expert = (2 * I * H // 2 + 2 * I * H // 32 + 2 * I * 4) + (H * I // 2 + H * I // 32 + H * 4)
    return distinct * per_expert, distinct, per_expert


def profiled_traffic(world, M, seed):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary
    (captured on exactly this workload: 1 GPU, M=5, seed 0), else None."""
    if world != 1 or M != 5 or seed != 0:
        return None
    try:
        with open(os.path.join(ROOT, "profiles", "tc_moe_kernel_gptoss120b_verify_M5.md")) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    return int(line.split(":")[1])
    except OSError:
        pass
    return None


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference_arm(args, world, rank)
    if args.workload in ("dsv3", "m25", "v4"):
        return main_dsv3(args, world, rank, local)
    if args.tokens is None:
        args.tokens = 5
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    from flyai_b200.moe import Mxfp4MoE, launch_count, set_profile_events

    M, MP = args.tokens, args.prefill_tokens or 2048
    layer = synth.make_gpt_oss_layer(**synth.GPT_OSS_120B, seed=args.seed, device=dev)
    lo, hi = rank * E // world, (rank + 1) * E // world
    max_tok = max(M, 0 if args.no_prefill else MP)
    moe = Mxfp4MoE.from_layer(layer, expert_range=(lo, hi), max_tokens=max_tok, device=dev)
    x = synth.make_tokens(M, H, seed=args.seed, device=dev)
    y = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
    flush = L2Flush(dev, args.l2)


    ep = None
    if world > 1:
        from flyai_b200.ep import ExpertParallelMoE
        # tokens replicated on every rank (the reference's expert-parallel pattern)
        ep = ExpertParallelMoE(moe, p2p=not args.ep_nccl, broadcast=False)

    def layer_step(xin, yout):
        if world == 1:
            moe.forward(xin, out=yout)
            return
        ep.forward(xin, out=yout)

    def timed(step, steps, warmup, sampler=None, sustain_iters=0):
        ctx = sampler if sampler is not None else _Null()
        ctx.__enter__()
        for _ in range(warmup):
            flush()
            step()
        for _ in range(sustain_iters):          # clocks settle under load (same count on every rank)
            flush()
            step()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        n0 = launch_count()
        for i in range(steps):
            flush()
            starts[i].record()
            step()
            ends[i].record()
        torch.cuda.synchronize()
        ctx.__exit__(None, None, None)
        launches = launch_count() - n0
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / steps
        if dist:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms, launches

    # ---- headline: device-resident verify step ----
    sampler = ClockSampler(local)
    ms, launches = timed(lambda: layer_step(x, y), args.steps, args.warmup, sampler, sustain_iters=args.sustain)
    clocks = sampler.summary()

    # ---- end to end through the public API with host buffers ----
    x_h = x.cpu().pin_memory()
    y_h = torch.empty(M, H, dtype=torch.bfloat16).pin_memory()
    w_h = torch.empty(M, K_TOP, dtype=torch.bfloat16).pin_memory()
    x_in = torch.empty_like(x)

    ids_d = torch.empty(M, K_TOP, dtype=torch.int32, device=dev)
    wts_d = torch.empty(M, K_TOP, dtype=torch.bfloat16, device=dev)

    def e2e_step():
        x_in.copy_(x_h, non_blocking=True)
        if world == 1:
            _, _, wts = moe.forward(x_in, out=y)
        else:
            ep.forward(x_in, out=y, ids=ids_d, wts=wts_d)
            wts = wts_d
        y_h.copy_(y, non_blocking=True)
        w_h.copy_(wts, non_blocking=True)
    e2e_ms, _ = timed(e2e_step, args.steps, args.warmup)
    h2d = x.numel() * 2
    d2h = y.numel() * 2 + M * K_TOP * 2

    # ---- roofline of the dominant kernel ----
    _, ids, _ = moe.route(x, logits=False)
    torch.cuda.synchronize()
    bytes_all, distinct, per_expert = touched_bytes(ids)
    local_ids = ids[(ids >= lo) & (ids < hi)]
    bytes_local = int(torch.unique(local_ids).numel()) * per_expert
    # the fused expert kernel alone: the library records these events right
    # before and after its launch, inside the same layer calls
    k0 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    k1 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for _ in range(args.warmup):
        flush()
        layer_step(x, y)
    torch.cuda.synchronize()
    for i in range(args.steps):
        flush()
        set_profile_events(k0[i], k1[i])
        layer_step(x, y)
    set_profile_events(None, None)
    torch.cuda.synchronize()
    exp_ms = sum(a.elapsed_time(b) for a, b in zip(k0, k1)) / args.steps
    if dist:
        t = torch.tensor([exp_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        exp_ms = float(t.item())
    hbm_peak, peak_kind = peaks()
    achieved_gbs = bytes_local / (exp_ms * 1e-3) / 1e9
    layer_alg_bytes = bytes_all + E * H * 2 + 2 * M * H * 2
    layer_gbs = layer_alg_bytes / (ms * 1e-3) / 1e9 / world

    result = {
        "metric": METRIC, "value": round(ms * 1e3, 2), "unit": "us", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
        "dtype": "mxfp4(e2m1+e8m0) weights x bf16 activations, fp32 accumulate",
        "data": "synthetic (seeded; BASELINE config 1 distributions)",
        "config": {"workload": "gpt-oss-120b MoE layer verify M=5 (config 1)", "experts": E,
                   "top_k": K_TOP, "hidden": H, "inter": I, "tokens": M,
                   "parallelism": f"ep{world}", "l2": flush.note,
                   **({"ep_tokens": "replicated on every rank"} if world > 1 else {})},
        "e2e": {"value": round(e2e_ms * 1e3, 2), "unit": "us", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "clocks": clocks,
        "roofline": {"bound": "hbm", "achieved": round(achieved_gbs, 1), "peak": hbm_peak,
                     "unit": "GB/s", "frac": round(achieved_gbs / hbm_peak, 4),
                     "traffic": profiled_traffic(world, M, args.seed),
                     "kernel": "tc_moe_kernel<true> (route + gate/up + down + fold: the whole layer call, one launch)" if world == 1 else "tc_moe_kernel (gate/up + down of this rank's experts)",
                     "kernel_us": round(exp_ms * 1e3, 2),
                     "bytes_per_launch": bytes_local, "distinct_experts": distinct,
                     "peak_source": peak_kind,
                     "layer_hbm_frac": round(layer_gbs / hbm_peak, 4)},
    }

    # ---- prefill chunk (config 2): Zipf-skewed router, M=2048 ----
    if not args.no_prefill:
        zl = synth.make_gpt_oss_layer(**synth.GPT_OSS_120B, seed=args.seed, device=dev, zipf_s=1.1)
        moe.router_b.copy_(zl.router_b)
        del zl
        xp = synth.make_tokens(MP, H, seed=args.seed + 1, device=dev)
        yp = torch.empty(MP, H, dtype=torch.bfloat16, device=dev)
        psteps = max(3, min(args.steps, 10))
        pmode = "single GPU"
        if world > 1 and args.ep_prefill == "replicated":
            pms, _ = timed(lambda: layer_step(xp, yp), psteps, max(3, min(args.warmup, 3)))
            pmode = f"tokens replicated on {world} ranks, pair rows all-reduced"
        elif world > 1:
            # tokens sharded by rank: each routes its MP/N tokens, rows travel to their
            # expert's owner and back over NCCL all-to-all (flyai_b200.ep.TokenShardedMoE)
            from flyai_b200.ep import PairExperts, TokenShardedMoE
            tsm = TokenShardedMoE(moe, PairExperts(moe, max_rows=4096))
            a, b = rank * MP // world, (rank + 1) * MP // world
            xl, yl = xp[a:b].contiguous(), yp[a:b]
            pms, _ = timed(lambda: tsm.forward(xl, yl), psteps, max(3, min(args.warmup, 3)))
            pmode = f"tokens sharded over {world} ranks, rows to their expert's owner by NCCL all-to-all"
        else:
            pms, _ = timed(lambda: layer_step(xp, yp), psteps, max(3, min(args.warmup, 3)))
        _, pids, _ = moe.route(xp, logits=False)
        torch.cuda.synchronize()
        pb, pdist, _ = touched_bytes(pids)
        flops = 2.0 * MP * K_TOP * (2 * I * H + H * I)
        load = torch.bincount(pids.flatten(), minlength=E)
        result["prefill"] = {"tokens": MP, "us": round(pms * 1e3, 1),
                             "tok_per_s": round(MP / (pms * 1e-3), 1),
                             "hbm_frac": round(pb / (pms * 1e-3) / 1e9 / world / hbm_peak, 4),
                             "tflops": round(flops / (pms * 1e-3) / 1e12, 2),
                             "distinct_experts": pdist,
                             "max_expert_load": int(load.max()), "steps": psteps,
                             "parallelism": pmode}
        moe.router_b.copy_(layer.router_b)

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        fn, kind = cpu_layer_on_host(layer, x)
        t, n, spread = time_cpu(fn)
        result["cpu_baseline"] = {"value": round(t * 1e6, 1), "unit": "us", "cores": torch.get_num_threads(),
                                  "kind": kind, "statistic": "median", **cpu_spread_us(spread),
                                  "sample": f"{n} full layer calls at M={M} "
                                  "(router + touched experts; dequant to bf16 done once, untimed)"}
    if world == 1 and not args.no_families:
        # the other layer families of the path, each on its own (banks freed in between)
        del moe
        torch.cuda.empty_cache()
        fam = {}
        for wl in ("dsv3", "m25", "v4"):
            fam[wl] = family_result(args, wl, 1, 0, dev, None, steps=20, warmup=3, sustain=0,
                                    tokens=FAMILY_TOKENS[wl], compact=True)
            torch.cuda.empty_cache()
        result["families"] = fam
    if world == 1 and not args.no_linear:
        result["linear"] = linear_result(args, dev, flush)
    if world == 1 and not args.no_k3:
        result["k3"] = k3_result(args, dev, flush)
    if rank == 0:
        print(json.dumps(result), flush=True)
    if ep is not None:
        ep.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


FAMILY_TOKENS = {"dsv3": 1, "m25": 5, "v4": 1}


def main_dsv3(args, world, rank, local):
    """--workload dsv3 | m25 | v4 on its own: one JSON line for that layer family
    (expert parallel under torchrun: rank r holds experts [rE/N, (r+1)E/N))."""
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    tokens = args.tokens if args.tokens is not None else FAMILY_TOKENS[args.workload]
    result = family_result(args, args.workload, world, rank, dev, dist, steps=args.steps,
                           warmup=args.warmup, sustain=min(args.sustain, 500), tokens=tokens)
    if rank == 0:
        print(json.dumps(result), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def family_result(args, workload, world, rank, dev, dist, steps, warmup, sustain, tokens, compact=False):
    """Config 3 (dsv3): DeepSeek-V3-shaped FP8 layer (E=256 + 1 shared, top-8 of 4/8
    groups, H=7168, I=2048; 11.3 GB of banks).  Config 4 (m25): MiniMax-M2.5-shaped
    NVFP4 layer (E=256, top-8 sigmoid with a skewed correction bias, H=3072,
    I=1536; 2.1 GB) with its M=4096 prefill batch.  v4: DeepSeek-V4-Flash W4A8 layer
    (E=256 fp4 + 1 fp8 shared, top-6 sqrtsoftplus, H=4096, I=2048; 3.3 GB).  One GPU
    holds every expert at N=1; microseconds per layer call at M=tokens plus a sweep
    of verify sizes, the expert kernel alone, rooflines, and the CPU oracle port."""
    from flyai_b200.moe import launch_count, set_profile_events
    erange = (rank * 256 // world, (rank + 1) * 256 // world) if world > 1 else None
    if workload == "dsv3":
        from flyai_b200.dsv3 import Fp8MoE
        from oracle import dsv3 as od
        layer = synth.make_dsv3_layer(**synth.DSV3, seed=args.seed, device=dev)
        moe = Fp8MoE.from_layer(layer, max_tokens=64, device=dev, expert_range=erange)
        sweep_ms = (1, 8, 32)
        metric = (f"MoE layer us at M={tokens} (DeepSeek-V3 FP8, E=256+1 shared, top-8 of 4/8 "
                  "groups, H=7168, I=2048)")
        dtype = "e4m3 weights (fp32 128x128 scales) x e4m3 activations (fp32 1x128 scales), fp32 accumulate"
        cfg_extra = {"shared_experts": 1, "n_group": layer.n_group, "topk_group": layer.topk_group}
        kernel = "f8_moe_kernel (gate/up + down of one layer call, one launch)"
        wl_name = f"deepseek-v3 fp8 MoE layer M={tokens} (config 3)"
        data_cfg = "BASELINE config 3 distributions"

        def kernel_bytes_of(distinct):
            return (distinct + 1) * od.expert_bytes(Hd, Id)
    elif workload == "m25":
        from flyai_b200.m25 import Nvfp4MoE
        from oracle import m25 as od
        layer = synth.make_m25_layer(**synth.M25, seed=args.seed, device=dev)
        moe = Nvfp4MoE.from_layer(layer, max_tokens=64, device=dev, expert_range=erange)
        sweep_ms = (1, 5, 16, 64)
        metric = (f"MoE layer us at M={tokens} (MiniMax-M2.5 NVFP4, E=256 top-8 sigmoid, "
                  "skewed, H=3072, I=1536)")
        dtype = ("nvfp4 weights (e2m1 + e4m3/16 + fp32 global) x bf16 activations as 6 e2m1 terms "
                 "(ue4m3/16), fp32 accumulate")
        cfg_extra = {"skew": "20% of experts take ~60% of picks (correction bias +0.14)"}
        kernel = "nv4_moe_kernel (gate/up + down of one layer call, one launch)"
        wl_name = f"minimax-m2.5 nvfp4 MoE layer M={tokens} (config 4, verify size)"
        data_cfg = "BASELINE config 4 distributions"

        def kernel_bytes_of(distinct):
            return distinct * od.expert_bytes(Hd, Id)
    else:
        from flyai_b200.v4 import W4A8MoE
        from oracle import v4 as od
        layer = synth.make_v4_layer(**synth.V4, seed=args.seed, device=dev)
        moe = W4A8MoE.from_layer(layer, max_tokens=64, device=dev, expert_range=erange)
        sweep_ms = (1, 6, 32, 64)
        metric = (f"MoE layer us at M={tokens} (DeepSeek-V4-Flash W4A8, E=256 fp4 + 1 fp8 shared, "
                  "top-6 sqrtsoftplus, H=4096, I=2048)")
        dtype = ("e2m1 weights (e8m0/32) x e4m3 activations (ue8m0 1x128), shared expert e4m3 "
                 "(e8m0 128x128), fp32 accumulate")
        cfg_extra = {"shared_experts": 1, "swiglu_limit": layer.swiglu_limit,
                     "route_scale": layer.route_scale}
        kernel = "v4_moe_kernel (gate/up + down of routed and shared experts, one launch)"
        wl_name = f"deepseek-v4-flash w4a8 MoE layer M={tokens} (decode)"
        data_cfg = "V4-Flash config.json shapes, config 0 value distributions"

        def kernel_bytes_of(distinct):
            return distinct * od.expert_bytes(Hd, Id) + od.shared_bytes(Hd, Id)
    flush = L2Flush(dev, args.l2)
    Hd, Id, Ed, Kd = layer.hidden, layer.inter, layer.num_experts, layer.top_k
    hbm_peak, peak_kind = peaks()
    ep = None
    if world > 1:
        from flyai_b200.ep import ExpertParallelMoE
        ep = ExpertParallelMoE(moe, p2p=False)   # NCCL all-reduce of the pair rows

    def layer_step(xin, yout):
        if ep is None:
            moe.forward(xin, out=yout)
        else:
            ep.forward(xin, out=yout)

    def max_over_ranks(v):
        if dist is None:
            return v
        t = torch.tensor([v], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def touched(ids_np):   # the layer's algorithmic bytes: experts, router, x and y
        return od.touched_bytes(ids_np, ids_np.shape[0], Hd, Id, Ed)

    def measure(M, steps, warmup, sampler=None, sustain=0):
        x = synth.make_tokens(M, Hd, seed=args.seed + M, device=dev)
        y = torch.empty_like(x)
        for _ in range(warmup + sustain):
            flush()
            layer_step(x, y)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        ctx = sampler if sampler is not None else _Null()
        ctx.__enter__()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        kv = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        n0 = launch_count()
        for i in range(steps):
            flush()
            ev[i][0].record()
            layer_step(x, y)
            ev[i][1].record()
        torch.cuda.synchronize()
        ctx.__exit__(None, None, None)
        launches = launch_count() - n0
        for i in range(steps):          # the expert kernel alone, same calls
            flush()
            set_profile_events(*kv[i])
            layer_step(x, y)
        set_profile_events(None, None)
        torch.cuda.synchronize()
        ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in ev) / steps)
        kms = max_over_ranks(sum(a.elapsed_time(b) for a, b in kv) / steps)
        _, ids, _ = moe.route(x)
        torch.cuda.synchronize()
        ids_np = ids.cpu().numpy()
        distinct = len(set(ids_np.ravel().tolist()))
        lo, hi = erange if erange is not None else (0, Ed)
        local = len(set(v for v in ids_np.ravel().tolist() if lo <= v < hi))
        # bytes the busiest rank's expert kernel streams (the kernel time is the max over ranks)
        kbytes = kernel_bytes_of(distinct)
        if dist is not None:
            mine = kernel_bytes_of(local) if lo == 0 else kernel_bytes_of(local) - kernel_bytes_of(0)
            t = torch.tensor([mine], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            kbytes = int(t.item())
        lbytes = touched(ids_np)
        return dict(x=x, y=y, ms=ms, kms=kms, launches=launches, distinct=distinct,
                    kernel_bytes=kbytes, layer_bytes=lbytes, ids=ids_np)

    M = tokens
    sampler = ClockSampler(dev.index)
    head = measure(M, steps, warmup, sampler, sustain=sustain)
    clocks = sampler.summary()
    assert moe.read_error()[0] == 0
    sweep = {}
    for m in sweep_ms:
        r = head if m == M else measure(m, max(10, steps // 2), warmup)
        sweep[str(m)] = {"us": round(r["ms"] * 1e3, 2), "kernel_us": round(r["kms"] * 1e3, 2),
                         "distinct_experts": r["distinct"],
                         "layer_hbm_frac": round(r["layer_bytes"] / (r["ms"] * 1e-3) / 1e9 / world / hbm_peak, 4),
                         "kernel_hbm_frac": round(r["kernel_bytes"] / (r["kms"] * 1e-3) / 1e9 / hbm_peak, 4)}
    # end to end with host buffers: H2D x, D2H y
    x_h = head["x"].cpu().pin_memory()
    y_h = torch.empty_like(x_h).pin_memory()
    x_in = torch.empty_like(head["x"])
    y = head["y"]
    for _ in range(warmup):
        x_in.copy_(x_h, non_blocking=True)
        layer_step(x_in, y)
        y_h.copy_(y, non_blocking=True)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i in range(steps):
        flush()
        ev[i][0].record()
        x_in.copy_(x_h, non_blocking=True)
        layer_step(x_in, y)
        y_h.copy_(y, non_blocking=True)
        ev[i][1].record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in ev) / steps)
    achieved = head["kernel_bytes"] / (head["kms"] * 1e-3) / 1e9
    result = {
        "metric": metric,
        "value": round(head["ms"] * 1e3, 2), "unit": "us", "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": round(head["ms"], 5), "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": dtype,
        "data": f"synthetic (seeded; {data_cfg})",
        "config": {"workload": wl_name, "experts": Ed, "top_k": Kd, "hidden": Hd, "inter": Id,
                   "tokens": M, "parallelism": f"ep{world}",
                   "l2": flush.note, **cfg_extra},
        "e2e": {"value": round(e2e_ms * 1e3, 2), "unit": "us", "h2d_bytes_per_step": M * Hd * 2,
                "d2h_bytes_per_step": M * Hd * 2},
        "gpu_launches": head["launches"],
        "clocks": clocks,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4), "traffic": None,
                     "kernel": kernel,
                     "kernel_us": round(head["kms"] * 1e3, 2), "bytes_per_launch": head["kernel_bytes"],
                     "distinct_experts": head["distinct"], "peak_source": peak_kind,
                     "layer_hbm_frac": round(head["layer_bytes"] / (head["ms"] * 1e-3) / 1e9 / world / hbm_peak, 4)},
        "sweep": sweep,
    }
    if workload == "m25" and not args.no_prefill:
        result["prefill"] = m25_prefill(args, layer, erange, world, dev, flush, max_over_ranks, hbm_peak)
    if not args.no_cpu_baseline and rank == 0 and world == 1:
        xc = head["x"].float().cpu().numpy()
        rw, rb = layer.router_w.float().cpu().numpy(), layer.bias.cpu().numpy()
        if workload == "dsv3":
            cache = {}

            def get(e):
                if e not in cache:
                    w13, s13, w2, s2 = layer.expert(e)
                    cache[e] = (w13.view(torch.uint8).cpu().numpy(), s13.cpu().numpy(),
                                w2.view(torch.uint8).cpu().numpy(), s2.cpu().numpy())
                return cache[e]

            def fn():
                ids, wts, _ = od.gate(xc, rw, rb, Kd, layer.n_group, layer.topk_group, layer.route_scale)
                return od.moe_forward(xc, ids, wts, get, Ed)
            note = "gate + touched experts + shared, fp8 dequant inside the timed call"
        elif workload == "m25":
            cache = {}

            def get(e):
                if e not in cache:
                    w13, s13, g13, w2, s2, g2 = layer.expert(e)
                    s13b, s2b = s13.view(torch.uint8).cpu().numpy(), s2.view(torch.uint8).cpu().numpy()
                    w13n, w2n = w13.cpu().numpy(), w2.cpu().numpy()
                    top = od.dequant_nvfp4(w13n[:Id], s13b[:Id], float(g13[0]))
                    bot = od.dequant_nvfp4(w13n[Id:], s13b[Id:], float(g13[1]))
                    cache[e] = (np.concatenate([top, bot]), od.dequant_nvfp4(w2n, s2b, float(g2[0])))
                return cache[e]

            def fn():
                ids, wts, _ = od.router(xc, rw, rb, Kd, layer.route_scale)
                return od.moe_forward(xc, ids, wts, get)
            fn()   # dequantise the touched experts once, outside the timing
            note = "router + touched experts, NVFP4 dequant to bf16 done once, untimed"
        else:
            cache = {}

            def get(e):
                if e not in cache:
                    cache[e] = tuple(t.cpu().numpy() for t in layer.expert(e))
                return cache[e]
            sw = layer.shared()
            shared_np = (sw[0].view(torch.uint8).cpu().numpy(), sw[1].cpu().numpy(),
                         sw[2].view(torch.uint8).cpu().numpy(), sw[3].cpu().numpy())

            def fn():
                ids, wts, _ = od.gate(xc, rw, rb, Kd, layer.route_scale)
                return od.moe_forward(xc, ids, wts, get, lambda: shared_np, layer.swiglu_limit)
            note = "gate + touched fp4 experts + fp8 shared expert, dequant inside the timed call"
        t, n, spread = time_cpu(fn, budget_s=20.0, max_calls=5)
        result["cpu_baseline"] = {"value": round(t * 1e6, 1), "unit": "us", "cores": torch.get_num_threads(),
                                  "kind": "port", "statistic": "median", **cpu_spread_us(spread),
                                  "sample": f"{n} full layer calls at M={M} (numpy oracle: {note})"}
    if ep is not None:
        del ep
    del moe
    if compact:
        keep = ("metric", "value", "unit", "dtype", "config", "e2e", "gpu_launches", "roofline",
                "sweep", "prefill", "cpu_baseline")
        result = {k: v for k, v in result.items() if k in keep}
    return result


def linear_result(args, dev, flush):
    """The seven dense FP8 GEMMs of a DeepSeek-V4-Flash decode layer
    (engines/deepseek_v4/v4_fp8_gemv.py:6-14): attention wq_a, wkv, wq_b, wo_b, the
    indexer's wq_b, the shared expert's w1 and w3 as one stacked bank, and its w2;
    e4m3 weights with e8m0 128x128 block scales, ue8m0 activation scales.  Per token
    count: microseconds for the seven in sequence (L2 flushed before each layer),
    each GEMM alone, and the weight stream's roofline (weight bytes / time)."""
    from flyai_b200.linear import Fp8Linear
    from flyai_b200.moe import launch_count
    from oracle.fp8_linear import weight_bytes
    L = synth.V4_LINEARS
    specs = [("wq_a", ["wq_a"]), ("wkv", ["wkv"]), ("wq_b", ["wq_b"]), ("wo_b", ["wo_b"]),
             ("idx_wq_b", ["idx_wq_b"]), ("shared_w13", ["shared_w1", "shared_w3"]),
             ("shared_w2", ["shared_w2"])]
    lins = []
    for i, (name, parts) in enumerate(specs):
        made = [synth.make_fp8_linear(*L[pn], seed=args.seed + 7 * i + j, device=dev)
                for j, pn in enumerate(parts)]
        lin = Fp8Linear([w for w, _ in made], [s for _, s in made], scale_fmt="ue8m0", max_tokens=8,
                        device=dev)
        lins.append((name, lin, sum(weight_bytes(*L[pn], e8m0=True) for pn in parts)))
        del made
    total_bytes = sum(b for _, _, b in lins)
    hbm_peak, peak_kind = peaks()

    def graphed(fn):
        """fn captured in a CUDA graph (a decode step replays its layers that way),
        so the timed region holds no host launch gaps."""
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            fn()
        torch.cuda.current_stream().wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        return g

    def time_steps(g, steps, warmup):
        for _ in range(warmup):
            flush()
            g.replay()
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(steps)]
        for a, b in ev:
            flush()
            a.record()
            g.replay()
            b.record()
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in ev) / steps

    out = {}
    for M in (1, 4):
        xs = [synth.make_tokens(M, lin.K, seed=args.seed + 100 + i, device=dev)
              for i, (_, lin, _) in enumerate(lins)]
        ys = [torch.empty(M, lin.N, dtype=torch.bfloat16, device=dev) for _, lin, _ in lins]

        def layer():
            for (_, lin, _), x, y in zip(lins, xs, ys):
                lin(x, out=y)
        n0 = launch_count()
        layer()
        launches = launch_count() - n0
        ms = time_steps(graphed(layer), args.steps, args.warmup)
        each = {}
        for (name, lin, nbytes), x, y in zip(lins, xs, ys):
            ems = time_steps(graphed(lambda: lin(x, out=y)), args.steps, args.warmup)
            each[name] = {"us": round(ems * 1e3, 2), "gbs": round(nbytes / (ems * 1e-3) / 1e9, 1)}
        for _, lin, _ in lins:
            assert lin.read_error() == 0
        gbs = total_bytes / (ms * 1e-3) / 1e9
        out[f"M{M}"] = {"us_per_layer": round(ms * 1e3, 2), "gpu_launches_per_layer": launches,
                        "timing": "CUDA graph of the seven calls, replayed; CUDA events",
                        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm_peak,
                                     "unit": "GB/s", "frac": round(gbs / hbm_peak, 4),
                                     "peak_source": peak_kind,
                                     "kernel": "ln_gemm_kernel (+ ln_quant_kernel, ln_reduce_kernel)"},
                        "each": each}
    return {"workload": "DeepSeek-V4-Flash decode layer: 7 dense FP8 GEMMs (fp8 e4m3 + e8m0 128x128)",
            "weight_bytes_per_layer": total_bytes, "l2": flush.note,
            "data": "synthetic (seeded N(0,1) e4m3 weights, e8m0 scales 2^-10..2^-7, bf16 N(0,1) x)",
            **out}


def k3_result(args, dev, flush):
    """Kimi-K3 routed experts behind moe_infer (synth.K3: 896 MXFP4 experts, top-16,
    latent 2048, intermediate 1024, situ beta 4 / linear_beta 25), routing given by
    the caller: microseconds per moe_infer call at M = 1, 8, 64 (L2 flushed before
    each), the expert kernel alone, its HBM roofline on the distinct experts'
    MXFP4 bytes, and the CPU oracle on the host at M=1 (weights dequantised once,
    untimed)."""
    from flyai_b200.k3 import K3MoE
    from flyai_b200.moe import launch_count, set_profile_events
    from oracle import k3 as ok3
    from oracle.v4 import dequant_fp4
    layer = synth.make_k3_layer(**synth.K3, seed=args.seed, device=dev)
    moe = K3MoE.from_layer(layer, max_tokens=64, device=dev)
    hbm_peak, peak_kind = peaks()
    per_expert = ok3.expert_bytes(layer.hidden, layer.inter)
    out = {"workload": "Kimi-K3 routed experts (moe_infer): E=896 MXFP4, top-16, H=2048 (latent), "
                       "I=1024, situ", "l2": flush.note,
           "data": "synthetic (seeded e2m1 nibbles, e8m0 2^-9..2^-3, bf16 N(0,1) x, random top-16 "
                   "routing with positive weights)"}
    for M in (1, 8, 64):
        x = synth.make_tokens(M, layer.hidden, seed=args.seed, device=dev)
        ids, wts = layer.routing(M, seed=M, device=dev)
        y = torch.empty(M, layer.hidden, dtype=torch.bfloat16, device=dev)
        for _ in range(args.warmup):
            flush()
            moe.moe_infer(x, ids, wts, out=y)
        torch.cuda.synchronize()
        steps = args.steps
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(steps)]
        kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(steps)]
        n0 = launch_count()
        for (a, b), (ka, kb) in zip(ev, kev):
            flush()
            set_profile_events(ka, kb)
            a.record()
            moe.moe_infer(x, ids, wts, out=y)
            b.record()
        set_profile_events(None, None)
        torch.cuda.synchronize()
        launches = (launch_count() - n0) // steps
        ms = sum(a.elapsed_time(b) for a, b in ev) / steps
        kms = sum(a.elapsed_time(b) for a, b in kev) / steps
        distinct = int(torch.unique(ids).numel())
        nbytes = distinct * per_expert
        gbs = nbytes / (kms * 1e-3) / 1e9
        out[f"M{M}"] = {"us": round(ms * 1e3, 2), "kernel_us": round(kms * 1e3, 2),
                        "gpu_launches": launches, "distinct_experts": distinct,
                        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm_peak,
                                     "unit": "GB/s", "frac": round(gbs / hbm_peak, 4),
                                     "peak_source": peak_kind, "bytes_per_launch": nbytes,
                                     "kernel": "tc_moe_kernel<false> (situ gate/up + down)"}}
        assert moe.read_error()[0] == 0
    # CPU oracle at M=1 on the host cores (the touched experts dequantised untimed)
    x = synth.make_tokens(1, layer.hidden, seed=args.seed)
    ids, wts = layer.routing(1, seed=1, device="cpu")
    deq = {}
    for e in sorted(set(int(v) for v in ids.ravel())):
        w1, s1, w3, s3, w2, s2 = (t.cpu().numpy() for t in layer.expert(e))
        deq[e] = (dequant_fp4(w1, s1), dequant_fp4(w3, s3), dequant_fp4(w2, s2))
    xn, idn, wn = x.float().numpy(), ids.numpy(), wts.numpy()

    def cpu_call():
        rows = np.zeros((1, layer.top_k, layer.hidden), np.float32)
        for s_, e in enumerate(idn[0]):
            W1, W3, W2 = deq[int(e)]
            g = ok3.round_bf16((xn @ W1.T).astype(np.float32))
            u = ok3.round_bf16((xn @ W3.T).astype(np.float32))
            h = ok3.situ(g, u, layer.beta, layer.linear_beta)
            rows[:, s_] = ok3.round_bf16((h @ W2.T).astype(np.float32))
        acc = rows[:, 0] * wn[:, 0:1]
        for s_ in range(1, layer.top_k):
            acc = (acc + rows[:, s_] * wn[:, s_:s_ + 1]).astype(np.float32)
        return ok3.round_bf16(acc)
    t, n, spread = time_cpu(cpu_call, budget_s=10.0)
    out["cpu_baseline"] = {"value": round(t * 1e6, 1), "unit": "us", "cores": torch.get_num_threads(),
                           "kind": "port", "statistic": "median", **cpu_spread_us(spread),
                           "sample": f"{n} moe_infer calls at M=1 (16 experts; dequantised once, untimed)"}
    del moe
    torch.cuda.empty_cache()
    return out


def m25_prefill(args, layer, erange, world, dev, flush, max_over_ranks, hbm_peak):
    """Config 4's prefill batch (M=4096 by default) through the same layer: the
    NVFP4 prefill path (weights expanded to bf16 in shared memory, tcgen05
    kind::f16).  Microseconds per layer call, the expert kernel alone, and both
    rooflines: HBM (distinct experts' NVFP4 bytes + router + x/y) and bf16 tensor
    (2 * M * k * 3 * H * I flops against the measured cuBLAS bf16 figure)."""
    from flyai_b200.m25 import Nvfp4MoE
    from flyai_b200.moe import set_profile_events
    from oracle import m25 as od
    MP = args.prefill_tokens or 4096
    pmoe = Nvfp4MoE.from_layer(layer, max_tokens=MP, device=dev, expert_range=erange)
    pep = None
    if world > 1:
        from flyai_b200.ep import ExpertParallelMoE
        pep = ExpertParallelMoE(pmoe, p2p=False)
    xp = synth.make_tokens(MP, layer.hidden, seed=args.seed + 1, device=dev)
    yp = torch.empty_like(xp)

    def step():
        if pep is None:
            pmoe.forward(xp, out=yp)
        else:
            pep.forward(xp, out=yp)

    steps = max(3, min(args.steps, 10))
    for _ in range(3):
        flush()
        step()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    kv = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i in range(steps):
        flush()
        ev[i][0].record()
        step()
        ev[i][1].record()
    torch.cuda.synchronize()
    for i in range(steps):
        flush()
        set_profile_events(*kv[i])
        step()
    set_profile_events(None, None)
    torch.cuda.synchronize()
    assert pmoe.read_error()[0] == 0
    ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in ev) / steps)
    kms = max_over_ranks(sum(a.elapsed_time(b) for a, b in kv) / steps)
    _, ids, _ = pmoe.route(xp, logits=False)
    torch.cuda.synchronize()
    ids_np = ids.cpu().numpy()
    H, I, E, K = layer.hidden, layer.inter, layer.num_experts, layer.top_k
    lbytes = od.touched_bytes(ids_np, MP, H, I, E)
    flops = 2.0 * MP * K * 3 * H * I
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            tpeak, tkind = float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        tpeak, tkind = 1590.0, "fallback"
    load = np.bincount(ids_np.ravel(), minlength=E)
    del pep, pmoe
    torch.cuda.empty_cache()
    return {"tokens": MP, "us": round(ms * 1e3, 1), "kernel_us": round(kms * 1e3, 1),
            "tok_per_s": round(MP / (ms * 1e-3), 1),
            "hbm_frac": round(lbytes / (ms * 1e-3) / 1e9 / world / hbm_peak, 4),
            "tflops": round(flops / (ms * 1e-3) / 1e12, 2),
            "kernel_tflops": round(flops / (kms * 1e-3) / 1e12, 2),
            "tensor_frac": round(flops / (kms * 1e-3) / 1e12 / world / tpeak, 4),
            "tensor_peak_tflops": tpeak, "tensor_peak_source": tkind,
            "kernel": "nvp_moe_kernel (NVFP4 expanded to bf16 in shared memory, tcgen05 kind::f16)",
            "distinct_experts": int((load > 0).sum()), "max_expert_pairs": int(load.max())}


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def run_reference_arm(args, world, rank):
    """The reference's own CPU implementation, timed on this host's cores."""
    if rank != 0:
        return
    if args.tokens is None:
        args.tokens = 5
    layer = synth.make_gpt_oss_layer(**synth.GPT_OSS_120B, seed=args.seed)
    x = synth.make_tokens(args.tokens, H, seed=args.seed)
    fn, kind = reference_layer_cpu(layer, x)
    per_step = []
    for _ in range(args.warmup):
        fn()
    for _ in range(args.steps):
        t0 = time.perf_counter()
        fn()
        per_step.append(time.perf_counter() - t0)
        if sum(per_step) > 120:
            break
    # the median (with its spread), the statistic the GPU arm's cpu_baseline reports
    us = statistics.median(per_step) * 1e6
    spread = (min(per_step), max(per_step))
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(us, 1), "unit": "us",
        "n_gpus": world, "steps": len(per_step), "warmup": args.warmup,
        "ms_per_step": round(us / 1e3, 3), "higher_is_better": False, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16 (dequantised MXFP4 weights)",
        "data": "synthetic (seeded; BASELINE config 1 distributions)",
        "config": {"workload": "gpt-oss-120b MoE layer verify M=5 (config 1)", "experts": E,
                   "top_k": K_TOP, "hidden": H, "inter": I, "tokens": args.tokens,
                   "parallelism": "cpu"},
        "cpu_baseline": {"value": round(us, 1), "unit": "us", "cores": torch.get_num_threads(),
                         "kind": kind, "statistic": "median", **cpu_spread_us(spread),
                         "sample": f"{len(per_step)} layer calls at M={args.tokens}, "
                         "transformers eager router+experts on CPU, dequant untimed"},
        "e2e": {"value": round(us, 1), "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


if __name__ == "__main__":
    main()
