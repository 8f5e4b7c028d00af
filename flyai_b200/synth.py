"""Seeded synthetic MoE layers with the shapes and value distributions of the
benchmark configurations (no checkpoints are available offline).

GPT-OSS family (MXFP4, configs 0-2): packed e2m1 nibbles uniform over all 16
codes, e8m0 exponents uniform in [118, 124], biases bf16 N(0, 0.02), router
bf16 N(0, 0.02) with bf16 N(0, 0.02) bias, activations bf16 N(0, 1).  Config 2
shifts the router bias by a Zipf(s) expert-popularity profile (log of a Zipf
pmf over a seeded random ranking of the experts) to reproduce prefill load
imbalance.

DeepSeek-V3 family (FP8, config 3): router bf16 N(0, 0.02) [E, H], correction
bias fp32 N(0, 0.05); expert weights e4m3 from N(0, 1) with one fp32 scale per
128x128 block drawn lognormal(-6, 0.5).  Each expert (the shared one is index
E) has its own generator seed, so any subset of experts can be regenerated
alone -- the CPU oracle of a full-size layer only needs the touched ones.

MiniMax-M2.5 family (NVFP4, config 4): router bf16 N(0, 0.02), correction bias
N(0, 0.05) plus 0.14 on a seeded 20% of the experts (which then take ~60% of the
token picks), rounded to bf16 values; expert weights e2m1 nibbles uniform over all 16 codes, one
e4m3 scale per 16 elements uniform in [0.25, 4], fp32 global scale 1e-2 per
tensor; per-expert seeds as for DeepSeek-V3.

Tensors are drawn with ``torch.Generator`` in a fixed order, so the same seed
gives the same layer on any machine running this image (CPU generator) or on
any B200 (CUDA generator); the two generators give different layers.
"""
from dataclasses import dataclass

import torch

GPT_OSS_20B = dict(num_experts=32, top_k=4, hidden=2880, inter=2880)
GPT_OSS_120B = dict(num_experts=128, top_k=4, hidden=2880, inter=2880)
DSV3 = dict(num_experts=256, top_k=8, hidden=7168, inter=2048, n_group=8, topk_group=4,
            route_scale=2.5, n_shared=1)
M25 = dict(num_experts=256, top_k=8, hidden=3072, inter=1536)
# DeepSeek-V4-Flash MoE layer (vendor/deepseek_v4_ref/inference/config.json):
# dim 4096, moe_inter_dim 2048, 256 routed experts (fp4), 6 active, 1 shared
# expert (fp8), sqrtsoftplus scores, route_scale 1.5, swiglu_limit 10.
V4 = dict(num_experts=256, top_k=6, hidden=4096, inter=2048, route_scale=1.5, swiglu_limit=10.0)
# Kimi-K3 routed experts behind moe_infer: 896 MXFP4 experts per layer
# (engines/kimi_k3/k3_moe_mxfp4.py:260), top-16 (the probe router of its
# docstring), situ beta 4 / linear_beta 25 (the configuration
# engines/kimi_k3/k3_pipe.py:747 builds).  The latent expert width and the expert
# intermediate size are not in the reference tree: 2048 and 1024 stand in.
K3 = dict(num_experts=896, top_k=16, hidden=2048, inter=1024, beta=4.0, linear_beta=25.0)
# The fp8 weights [N, K] a DeepSeek-V4-Flash decode layer multiplies one token
# row by (engines/deepseek_v4/v4_fp8_gemv.py:10-14): attention, the ratio-4
# layers' indexer wq_b, and the shared expert (w1 and w3 read the same x).
V4_LINEARS = dict(wq_a=(1024, 4096), wkv=(512, 4096), wo_b=(4096, 8192), wq_b=(32768, 1024),
                  idx_wq_b=(8192, 1024), shared_w1=(2048, 4096), shared_w3=(2048, 4096),
                  shared_w2=(4096, 2048))


@dataclass
class GptOssLayer:
    router_w: torch.Tensor    # bf16 [E, H]
    router_b: torch.Tensor    # bf16 [E]
    w13_blocks: torch.Tensor  # uint8 [E, 2I, H/32, 16]
    w13_scales: torch.Tensor  # uint8 [E, 2I, H/32]
    w13_bias: torch.Tensor    # bf16 [E, 2I]
    w2_blocks: torch.Tensor   # uint8 [E, H, I/32, 16]
    w2_scales: torch.Tensor   # uint8 [E, H, I/32]
    w2_bias: torch.Tensor     # bf16 [E, H]
    top_k: int
    limit: float = 7.0
    alpha: float = 1.702

    @property
    def num_experts(self):
        return self.router_w.shape[0]

    @property
    def hidden(self):
        return self.router_w.shape[1]

    @property
    def inter(self):
        return self.w2_blocks.shape[2] * 32

    def to(self, device):
        kw = {f: getattr(self, f).to(device) for f in
              ("router_w", "router_b", "w13_blocks", "w13_scales", "w13_bias",
               "w2_blocks", "w2_scales", "w2_bias")}
        return GptOssLayer(top_k=self.top_k, limit=self.limit, alpha=self.alpha, **kw)


def make_gpt_oss_layer(num_experts, top_k, hidden, inter, seed=0, device="cpu",
                       zipf_s=None, scale_lo=118, scale_hi=124):
    g = torch.Generator(device=device).manual_seed(seed)
    E, H, I = num_experts, hidden, inter
    rnd = dict(generator=g, device=device)
    router_w = (torch.randn(E, H, **rnd) * 0.02).bfloat16()
    router_b = (torch.randn(E, **rnd) * 0.02).bfloat16()
    w13_blocks = torch.randint(0, 256, (E, 2 * I, H // 32, 16), dtype=torch.uint8, **rnd)
    w13_scales = torch.randint(scale_lo, scale_hi + 1, (E, 2 * I, H // 32), dtype=torch.uint8, **rnd)
    w13_bias = (torch.randn(E, 2 * I, **rnd) * 0.02).bfloat16()
    w2_blocks = torch.randint(0, 256, (E, H, I // 32, 16), dtype=torch.uint8, **rnd)
    w2_scales = torch.randint(scale_lo, scale_hi + 1, (E, H, I // 32), dtype=torch.uint8, **rnd)
    w2_bias = (torch.randn(E, H, **rnd) * 0.02).bfloat16()
    if zipf_s is not None:
        rank = torch.randperm(E, **rnd).float() + 1.0
        pmf = rank.pow(-zipf_s)
        pmf = pmf / pmf.sum()
        shift = pmf.log() - pmf.log().mean()
        router_b = (router_b.float() + shift).bfloat16()
    return GptOssLayer(router_w, router_b, w13_blocks, w13_scales, w13_bias,
                       w2_blocks, w2_scales, w2_bias, top_k)


def make_tokens(num_tokens, hidden, seed=0, device="cpu"):
    g = torch.Generator(device=device).manual_seed(seed + 1_000_003)
    return torch.randn(num_tokens, hidden, generator=g, device=device).bfloat16()


@dataclass
class Dsv3Layer:
    """Router of a DeepSeek-V3-style FP8 MoE layer plus a seeded expert factory.

    ``expert(e)`` -> (w13 e4m3 [2I, H] = [w1; w3], s13 fp32 [2I/128, H/128],
    w2 e4m3 [H, I], s2 fp32 [H/128, I/128]); e = num_experts is the shared expert."""
    router_w: torch.Tensor    # bf16 [E, H]
    bias: torch.Tensor        # fp32 [E] e_score_correction_bias
    inter: int
    top_k: int
    n_group: int
    topk_group: int
    route_scale: float
    n_shared: int
    seed: int
    device: str = "cpu"

    @property
    def num_experts(self):
        return self.router_w.shape[0]

    @property
    def hidden(self):
        return self.router_w.shape[1]

    def expert(self, e, device=None):
        device = device or self.device
        g = torch.Generator(device=device).manual_seed(self.seed * 1_000_003 + 7919 * (e + 1))
        rnd = dict(generator=g, device=device)
        H, I, B = self.hidden, self.inter, 128
        w13 = torch.randn(2 * I, H, **rnd).to(torch.float8_e4m3fn)
        s13 = (torch.randn(2 * I // B, H // B, **rnd) * 0.5 - 6.0).exp()
        w2 = torch.randn(H, I, **rnd).to(torch.float8_e4m3fn)
        s2 = (torch.randn(H // B, I // B, **rnd) * 0.5 - 6.0).exp()
        return w13, s13, w2, s2


def make_dsv3_layer(num_experts, top_k, hidden, inter, n_group, topk_group, route_scale=2.5,
                    n_shared=1, seed=0, device="cpu"):
    g = torch.Generator(device=device).manual_seed(seed)
    rnd = dict(generator=g, device=device)
    router_w = (torch.randn(num_experts, hidden, **rnd) * 0.02).bfloat16()
    bias = torch.randn(num_experts, **rnd) * 0.05
    return Dsv3Layer(router_w, bias, inter, top_k, n_group, topk_group, route_scale, n_shared,
                     seed, str(device))


@dataclass
class M25Layer:
    """Router of a MiniMax-M2.5-style NVFP4 MoE layer plus a seeded expert factory.

    ``expert(e)`` -> (w13 uint8 [2I, H/2] packed e2m1 of [w1; w3], s13 e4m3 [2I, H/16],
    g13 fp32 [2] (w1, w3 global scales), w2 uint8 [H, I/2], s2 e4m3 [H, I/16], g2 fp32 [1])."""
    router_w: torch.Tensor    # bf16 [E, H]
    bias: torch.Tensor        # fp32 [E] e_score_correction_bias
    inter: int
    top_k: int
    seed: int
    route_scale: float = 1.0
    global_scale: float = 1e-2
    device: str = "cpu"

    @property
    def num_experts(self):
        return self.router_w.shape[0]

    @property
    def hidden(self):
        return self.router_w.shape[1]

    def expert(self, e, device=None):
        device = device or self.device
        g = torch.Generator(device=device).manual_seed(self.seed * 1_000_003 + 104729 * (e + 1))
        rnd = dict(generator=g, device=device)
        H, I = self.hidden, self.inter
        w13 = torch.randint(0, 256, (2 * I, H // 2), dtype=torch.uint8, **rnd)
        s13 = (torch.rand(2 * I, H // 16, **rnd) * 3.75 + 0.25).to(torch.float8_e4m3fn)
        w2 = torch.randint(0, 256, (H, I // 2), dtype=torch.uint8, **rnd)
        s2 = (torch.rand(H, I // 16, **rnd) * 3.75 + 0.25).to(torch.float8_e4m3fn)
        g13 = torch.full((2,), self.global_scale, dtype=torch.float32, device=device)
        g2 = torch.full((1,), self.global_scale, dtype=torch.float32, device=device)
        return w13, s13, g13, w2, s2, g2


def make_m25_layer(num_experts, top_k, hidden, inter, seed=0, device="cpu", skew=0.14,
                   hot_frac=0.2, route_scale=1.0, global_scale=1e-2):
    g = torch.Generator(device=device).manual_seed(seed)
    rnd = dict(generator=g, device=device)
    router_w = (torch.randn(num_experts, hidden, **rnd) * 0.02).bfloat16()
    bias = torch.randn(num_experts, **rnd) * 0.05
    hot = torch.randperm(num_experts, **rnd)[: int(num_experts * hot_frac)]
    bias[hot] += skew
    bias = bias.bfloat16().float()   # a bf16 checkpoint buffer: same values in fp32 and bf16
    return M25Layer(router_w, bias, inter, top_k, seed, route_scale=route_scale,
                    global_scale=global_scale, device=str(device))


@dataclass
class V4Layer:
    """Router of a DeepSeek-V4-style W4A8 MoE layer plus seeded expert factories.

    ``expert(e)`` -> (w13 uint8 [2I, H/2] packed e2m1 of [w1; w3] (low nibble =
    even K), s13 uint8 [2I, H/32] e8m0, w2 uint8 [H, I/2], s2 uint8 [H, I/32]);
    ``shared()`` -> (w13 e4m3 [2I, H], s13 uint8 [2I/128, H/128] e8m0, w2 e4m3
    [H, I], s2 uint8 [H/128, I/128] e8m0) -- the shared expert of a "dtype fp8,
    scale_dtype fp8" checkpoint (power-of-two 128x128 block scales).  ``tid2eid``
    (int32 [vocab, k], repeats allowed) is set for a hash-routed layer."""
    router_w: torch.Tensor    # bf16 [E, H]
    bias: torch.Tensor        # fp32 [E] (score-routed layers)
    inter: int
    top_k: int
    route_scale: float
    swiglu_limit: float
    seed: int
    tid2eid: torch.Tensor = None
    device: str = "cpu"

    @property
    def num_experts(self):
        return self.router_w.shape[0]

    @property
    def hidden(self):
        return self.router_w.shape[1]

    def expert(self, e, device=None):
        device = device or self.device
        g = torch.Generator(device=device).manual_seed(self.seed * 1_000_003 + 15485863 * (e + 1))
        rnd = dict(generator=g, device=device)
        H, I = self.hidden, self.inter
        w13 = torch.randint(0, 256, (2 * I, H // 2), dtype=torch.uint8, **rnd)
        s13 = torch.randint(118, 125, (2 * I, H // 32), dtype=torch.uint8, **rnd)
        w2 = torch.randint(0, 256, (H, I // 2), dtype=torch.uint8, **rnd)
        s2 = torch.randint(118, 125, (H, I // 32), dtype=torch.uint8, **rnd)
        return w13, s13, w2, s2

    def shared(self, device=None):
        device = device or self.device
        g = torch.Generator(device=device).manual_seed(self.seed * 1_000_003 + 982451653)
        rnd = dict(generator=g, device=device)
        H, I, B = self.hidden, self.inter, 128
        w13 = torch.randn(2 * I, H, **rnd).to(torch.float8_e4m3fn)
        s13 = torch.randint(117, 121, (2 * I // B, H // B), dtype=torch.uint8, **rnd)
        w2 = torch.randn(H, I, **rnd).to(torch.float8_e4m3fn)
        s2 = torch.randint(117, 121, (H // B, I // B), dtype=torch.uint8, **rnd)
        return w13, s13, w2, s2


def make_v4_layer(num_experts, top_k, hidden, inter, route_scale=1.5, swiglu_limit=10.0, seed=0,
                  device="cpu", hash_vocab=0):
    """A V4 MoE layer; hash_vocab > 0 makes it hash-routed (the first n_hash_layers
    of the model) with a random tid2eid table of that many token ids."""
    g = torch.Generator(device=device).manual_seed(seed)
    rnd = dict(generator=g, device=device)
    router_w = (torch.randn(num_experts, hidden, **rnd) * 0.02).bfloat16()
    bias = torch.randn(num_experts, **rnd) * 0.05
    tid2eid = None
    if hash_vocab:
        tid2eid = torch.randint(0, num_experts, (hash_vocab, top_k), dtype=torch.int32, **rnd)
    return V4Layer(router_w, bias, inter, top_k, route_scale, swiglu_limit, seed, tid2eid,
                   str(device))


def make_fp8_linear(N, K, seed=0, e8m0=True, device="cpu"):
    """An fp8 Linear's (weight e4m3 [N, K] from N(0, 1), scale [N/128, K/128]):
    e8m0 bytes uniform in [117, 120] (a "scale_dtype fp8" checkpoint, as the V4
    shared expert), else fp32 lognormal(-6, 0.5) as the DeepSeek-V3 experts."""
    g = torch.Generator(device=device).manual_seed(seed * 1_000_003 + 7919 * N + K)
    rnd = dict(generator=g, device=device)
    w = torch.randn(N, K, **rnd).to(torch.float8_e4m3fn)
    if e8m0:
        s = torch.randint(117, 121, (N // 128, K // 128), dtype=torch.uint8, **rnd)
    else:
        s = torch.exp(torch.randn(N // 128, K // 128, **rnd) * 0.5 - 6.0)
    return w, s


@dataclass
class K3Layer:
    """Seeded Kimi-K3 MXFP4 experts (the checkpoint's ``mxfp4-pack-quantized``
    tensors, engines/kimi_k3/k3_moe_mxfp4.py:326-340): ``expert(e)`` -> (w1 uint8
    [I, H/2], s1 uint8 [I, H/32], w3, s3 alike, w2 uint8 [H, I/2], s2 uint8
    [H, I/32]): e2m1 nibbles uniform over all 16 codes (low nibble = even K), e8m0
    exponents uniform in [118, 124]; each expert has its own generator seed.
    ``routing(M)`` -> (topk_ids int64 [M, k], k distinct experts per token;
    topk_weight fp32 [M, k], positive, summing to 1 per token) standing in for
    KimiMoEGate's output."""
    num_experts: int
    top_k: int
    hidden: int
    inter: int
    beta: float
    linear_beta: float
    seed: int
    device: str = "cpu"

    def expert(self, e, device=None):
        device = device or self.device
        g = torch.Generator(device=device).manual_seed(self.seed * 1_000_003 + 7_368_787 * (e + 1))
        rnd = dict(generator=g, device=device)
        H, I = self.hidden, self.inter
        w1 = torch.randint(0, 256, (I, H // 2), dtype=torch.uint8, **rnd)
        s1 = torch.randint(118, 125, (I, H // 32), dtype=torch.uint8, **rnd)
        w3 = torch.randint(0, 256, (I, H // 2), dtype=torch.uint8, **rnd)
        s3 = torch.randint(118, 125, (I, H // 32), dtype=torch.uint8, **rnd)
        w2 = torch.randint(0, 256, (H, I // 2), dtype=torch.uint8, **rnd)
        s2 = torch.randint(118, 125, (H, I // 32), dtype=torch.uint8, **rnd)
        return w1, s1, w3, s3, w2, s2

    def routing(self, num_tokens, seed=0, device=None):
        device = device or self.device
        g = torch.Generator(device="cpu").manual_seed(self.seed * 7919 + seed + 17)
        ids = torch.stack([torch.randperm(self.num_experts, generator=g)[:self.top_k]
                           for _ in range(num_tokens)]) if num_tokens else \
            torch.zeros(0, self.top_k, dtype=torch.long)
        w = torch.rand(num_tokens, self.top_k, generator=g) + 0.05
        w = w / w.sum(-1, keepdim=True)
        return ids.to(device), w.float().to(device)


def make_k3_layer(num_experts, top_k, hidden, inter, beta=4.0, linear_beta=25.0, seed=0, device="cpu"):
    return K3Layer(num_experts, top_k, hidden, inter, beta, linear_beta, seed, str(device))
