"""GPT-2-small transformer block with swappable attention: the C5 workload (tokens/s through
the op inside a real block).

Reference counterpart: bench/gpt_block.py (the nanoGPT block LN -> causal self-attention ->
residual -> LN -> MLP -> residual at n_embd 768, 12 heads, T 1024, fp16; one CUDA-event pair
around the attention window inside each forward; warm, no L2 flush).  Differences, all stated
with the result: batch 16 and a token + position embedding in front of the block (the
configuration this build benchmarks), weights drawn N(0, 0.02) from a seeded generator, and two
ways of calling our op:

* ``fused_strided``    -- ``forward_strided`` on the [B, H, T, D] views of the projection output
                          (``view`` + ``permute``, no copy), output already in [B, T, H, D]
                          order, so the head merge is a view as well;
* ``fused_contiguous`` -- ``torch.ops.fused_attn.forward`` on ``.contiguous()`` copies, the
                          reference's binding path (gpt_block.py:132-135), copies inside the
                          timed attention window as there;

plus PyTorch SDPA with a pinned backend (flash / efficient / cuDNN; math as the plain reference,
which also runs on the CPU).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

VOCAB = 50257

FUSED_IMPLS = ("fused_strided", "fused_contiguous")
SDPA_IMPLS = ("sdpa_flash", "sdpa_efficient", "sdpa_cudnn", "sdpa_math")
IMPLS = FUSED_IMPLS + SDPA_IMPLS


@dataclass(frozen=True)
class GPTConfig:
    n_embd: int = 768
    n_head: int = 12
    seq: int = 1024
    batch: int = 16
    mlp_ratio: int = 4
    dtype: torch.dtype = torch.float16
    seed: int = 4

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_head

    def attention_flops(self) -> float:
        """Causal attention FLOPs of one forward (4*B*H*T^2*D, halved for the causal mask)."""
        return 2.0 * self.batch * self.n_head * self.seq * self.seq * self.head_dim

    def gemm_flops(self) -> float:
        """The block's four projections: qkv, out, MLP up and down (2 FLOPs per MAC)."""
        c, tok = self.n_embd, self.batch * self.seq
        return 2.0 * tok * c * (3 * c + c + 2 * self.mlp_ratio * c)


def _sdpa_backend(impl: str):
    from torch.nn.attention import SDPBackend

    return {"sdpa_flash": SDPBackend.FLASH_ATTENTION,
            "sdpa_efficient": SDPBackend.EFFICIENT_ATTENTION,
            "sdpa_cudnn": SDPBackend.CUDNN_ATTENTION,
            "sdpa_math": SDPBackend.MATH}[impl]


class CausalSelfAttention(nn.Module):
    """Fused qkv projection, causal attention through ``impl``, output projection.  With
    ``record=True`` each forward records one CUDA-event pair around the attention window (from
    the head split to the merged [B, T, C] tensor) into ``windows``."""

    def __init__(self, cfg: GPTConfig, impl: str):
        super().__init__()
        if impl not in IMPLS:
            raise ValueError(f"unknown attention impl {impl!r}; one of {IMPLS}")
        self.c_attn = nn.Linear(cfg.n_embd, 3 * cfg.n_embd)
        self.c_proj = nn.Linear(cfg.n_embd, cfg.n_embd)
        self.n_head = cfg.n_head
        self.impl = impl
        self.scale = 1.0 / math.sqrt(cfg.head_dim)
        self.record = False
        self.windows: list = []

    def attend(self, q, k, v):
        """[B, H, T, D] views -> [B, H, T, D] output (any strides)."""
        if self.impl == "fused_strided":
            import fused_attn

            return fused_attn.forward_strided(q, k, v, is_causal=True, scale=self.scale)
        if self.impl == "fused_contiguous":
            return torch.ops.fused_attn.forward(q.contiguous(), k.contiguous(), v.contiguous(),
                                                True, self.scale)[0]
        from torch.nn.attention import sdpa_kernel

        with sdpa_kernel([_sdpa_backend(self.impl)]):
            return F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=self.scale)

    def forward(self, x):
        b, t, c = x.shape
        qkv = self.c_attn(x)
        ev = None
        if self.record:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        q, k, v = qkv.view(b, t, 3, self.n_head, c // self.n_head).permute(2, 0, 3, 1, 4)
        y = self.attend(q, k, v).transpose(1, 2).reshape(b, t, c)
        if ev is not None:
            ev[1].record()
            self.windows.append(ev)
        return self.c_proj(y)


class Block(nn.Module):
    """Pre-LN transformer block: x + attn(ln_1(x)), then + mlp(ln_2(x)) with tanh-GELU."""

    def __init__(self, cfg: GPTConfig, impl: str):
        super().__init__()
        self.ln_1 = nn.LayerNorm(cfg.n_embd)
        self.attn = CausalSelfAttention(cfg, impl)
        self.ln_2 = nn.LayerNorm(cfg.n_embd)
        self.mlp = nn.Sequential(nn.Linear(cfg.n_embd, cfg.mlp_ratio * cfg.n_embd),
                                 nn.GELU(approximate="tanh"),
                                 nn.Linear(cfg.mlp_ratio * cfg.n_embd, cfg.n_embd))

    def forward(self, x):
        x = x + self.attn(self.ln_1(x))
        return x + self.mlp(self.ln_2(x))


class GPT2BlockModel(nn.Module):
    """Token + position embedding followed by one block: token ids [B, T] -> hidden [B, T, C]."""

    def __init__(self, cfg: GPTConfig, impl: str):
        super().__init__()
        self.cfg = cfg
        self.wte = nn.Embedding(VOCAB, cfg.n_embd)
        self.wpe = nn.Embedding(cfg.seq, cfg.n_embd)
        self.block = Block(cfg, impl)

    def forward(self, idx):
        pos = torch.arange(idx.shape[1], device=idx.device)
        return self.block(self.wte(idx) + self.wpe(pos))


def build_model(cfg: GPTConfig, impl: str, device) -> GPT2BlockModel:
    """The model with GPT-2's initialisation from ``cfg.seed``: every weight matrix and
    embedding N(0, 0.02), biases 0, LayerNorm weight 1 and bias 0 -- identical across impls."""
    model = GPT2BlockModel(cfg, impl)
    g = torch.Generator(device="cpu").manual_seed(cfg.seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("bias"):
                p.zero_()
            elif ".ln_" in name:
                p.fill_(1.0)
            else:
                p.copy_(torch.randn(p.shape, generator=g) * 0.02)
    return model.to(device=device, dtype=cfg.dtype).eval()


def token_ids(cfg: GPTConfig, device, seed: int | None = None) -> torch.Tensor:
    """[batch, seq] token ids uniform in [0, VOCAB), from a seeded CPU generator."""
    g = torch.Generator(device="cpu").manual_seed(cfg.seed if seed is None else seed)
    return torch.randint(0, VOCAB, (cfg.batch, cfg.seq), generator=g).to(device)


def measure(model: GPT2BlockModel, idx: torch.Tensor, warmup: int, iters: int) -> dict:
    """Warm timing as the reference's harness: ``warmup`` untimed forwards, then ``iters``
    forwards each between one CUDA-event pair, the attention window timed inside each, one
    synchronize at the end.  Returns median / p10 / p90 block ms, median attention ms and
    tokens/s."""
    attn = model.block.attn
    with torch.no_grad():
        for _ in range(warmup):
            model(idx)
        torch.cuda.synchronize()
        attn.windows.clear()
        attn.record = True
        pairs = []
        for _ in range(iters):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            model(idx)
            e1.record()
            pairs.append((e0, e1))
        torch.cuda.synchronize()
        attn.record = False
    blk = sorted(a.elapsed_time(b) for a, b in pairs)
    att = sorted(a.elapsed_time(b) for a, b in attn.windows[-iters:])

    def pct(xs, p):
        return xs[min(len(xs) - 1, max(0, int(round(p / 100 * (len(xs) - 1)))))]

    cfg = model.cfg
    ms = pct(blk, 50)
    return {"block_ms": ms, "block_ms_p10": pct(blk, 10), "block_ms_p90": pct(blk, 90),
            "attn_ms": pct(att, 50), "attn_pct": 100.0 * pct(att, 50) / ms,
            "tokens_per_s": cfg.batch * cfg.seq / (ms * 1e-3)}
