"""Calibration forward: the model pass that feeds the modifiers' activation hooks.

The reference's modifiers never run a model themselves: GPTQModifier.OnBatchCore relies on
the caller driving ``module.call()`` so that the hooks ActivationHookManager attached fire
(src/LLMCompressorSharp.Core/Algorithms/Gptq/GPTQModifier.cs:98-104; the tests drive a
Linear by hand, tests/LLMCompressorSharp.Tests/Algorithms/Gptq/GPTQEndToEndTests.cs:160-173).
This module supplies that caller:

- ``LlamaShape`` presets for the model shapes the job is quoted on;
- ``LlamaForCalibration``, a random-initialised LLaMA decoder with the usual module names
  (``model.layers.{i}.self_attn.q_proj`` ...), weights ~N(0, 0.02) from a seed, whose
  forward is ordinary torch (cuBLAS GEMMs and SDPA): it only produces the activations that
  reach the hooked Linear layers;
- ``drive(model, batches)``, which runs the forward on each calibration batch and then hands
  the batch to ``CompressionSession.run``, so every modifier's OnBatch sees hooks that have
  already fired for that batch.

The whole calibration set goes through the unquantised model once and every Hessian is
accumulated in that pass, as the reference does (GPTQModifier.cs:119-136 solves the layers
afterwards from those Hessians).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F


@dataclass(frozen=True)
class LlamaShape:
    hidden: int
    intermediate: int
    heads: int
    kv_heads: int
    layers: int
    vocab: int
    rope_theta: float = 10000.0
    rms_eps: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads


SHAPES = {
    "smollm2-135m": LlamaShape(576, 1536, 9, 3, 30, 49152, rope_theta=100000.0),
    "llama-2-7b": LlamaShape(4096, 11008, 32, 32, 32, 32000),
    "llama-3-8b": LlamaShape(4096, 14336, 32, 8, 32, 128256, rope_theta=500000.0),
    "llama-3-70b": LlamaShape(8192, 28672, 64, 8, 80, 128256, rope_theta=500000.0),
}


class RMSNorm(torch.nn.Module):
    def __init__(self, d: int, eps: float, dtype, device):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.ones(d, dtype=dtype, device=device), requires_grad=False)
        self.eps = eps

    def forward(self, x):
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return (y * self.weight.float()).to(x.dtype)


def _linear(n_in: int, n_out: int, dtype, device, g: torch.Generator) -> torch.nn.Linear:
    lin = torch.nn.Linear(n_in, n_out, bias=False, dtype=dtype, device=device)
    w = torch.randn(n_out, n_in, generator=g, dtype=torch.float32) * 0.02
    with torch.no_grad():
        lin.weight.copy_(w.to(dtype))
    lin.weight.requires_grad_(False)
    return lin


class Attention(torch.nn.Module):
    def __init__(self, s: LlamaShape, dtype, device, g):
        super().__init__()
        hd = s.head_dim
        self.s = s
        self.q_proj = _linear(s.hidden, s.heads * hd, dtype, device, g)
        self.k_proj = _linear(s.hidden, s.kv_heads * hd, dtype, device, g)
        self.v_proj = _linear(s.hidden, s.kv_heads * hd, dtype, device, g)
        self.o_proj = _linear(s.heads * hd, s.hidden, dtype, device, g)

    def forward(self, x, cos, sin):
        b, t, _ = x.shape
        s = self.s
        hd = s.head_dim
        q = self.q_proj(x).view(b, t, s.heads, hd).transpose(1, 2)
        k = self.k_proj(x).view(b, t, s.kv_heads, hd).transpose(1, 2)
        v = self.v_proj(x).view(b, t, s.kv_heads, hd).transpose(1, 2)
        q, k = _rope(q, cos, sin), _rope(k, cos, sin)
        rep = s.heads // s.kv_heads
        if rep > 1:
            k = k.repeat_interleave(rep, dim=1)
            v = v.repeat_interleave(rep, dim=1)
        o = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        return self.o_proj(o.transpose(1, 2).reshape(b, t, s.heads * hd))


class MLP(torch.nn.Module):
    def __init__(self, s: LlamaShape, dtype, device, g):
        super().__init__()
        self.gate_proj = _linear(s.hidden, s.intermediate, dtype, device, g)
        self.up_proj = _linear(s.hidden, s.intermediate, dtype, device, g)
        self.down_proj = _linear(s.intermediate, s.hidden, dtype, device, g)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class DecoderLayer(torch.nn.Module):
    def __init__(self, s: LlamaShape, dtype, device, g):
        super().__init__()
        self.input_layernorm = RMSNorm(s.hidden, s.rms_eps, dtype, device)
        self.self_attn = Attention(s, dtype, device, g)
        self.post_attention_layernorm = RMSNorm(s.hidden, s.rms_eps, dtype, device)
        self.mlp = MLP(s, dtype, device, g)

    def forward(self, x, cos, sin):
        x = x + self.self_attn(self.input_layernorm(x), cos, sin)
        return x + self.mlp(self.post_attention_layernorm(x))


def _rope(x, cos, sin):
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    return (x * cos + torch.cat((-x2, x1), dim=-1) * sin).to(x.dtype)


class _Body(torch.nn.Module):
    def __init__(self, s: LlamaShape, dtype, device, g):
        super().__init__()
        self.embed_tokens = torch.nn.Embedding(s.vocab, s.hidden, dtype=dtype, device=device)
        with torch.no_grad():
            self.embed_tokens.weight.copy_((torch.randn(s.vocab, s.hidden, generator=g) * 0.02).to(dtype))
        self.embed_tokens.weight.requires_grad_(False)
        self.layers = torch.nn.ModuleList(DecoderLayer(s, dtype, device, g) for _ in range(s.layers))
        self.norm = RMSNorm(s.hidden, s.rms_eps, dtype, device)


class LlamaForCalibration(torch.nn.Module):
    """Random-initialised LLaMA decoder (no LM head: calibration only needs the activations
    that reach the decoder's Linear layers).  Weights are drawn on the CPU from one seeded
    generator in a fixed order, so a shape and a seed give the same model on every device."""

    def __init__(self, shape: LlamaShape, dtype=torch.bfloat16, device="cpu", seed: int = 0):
        super().__init__()
        self.shape = shape
        g = torch.Generator().manual_seed(seed)
        self.model = _Body(shape, dtype, device, g)
        hd = shape.head_dim
        inv = 1.0 / (shape.rope_theta ** (torch.arange(0, hd, 2, dtype=torch.float32) / hd))
        self.register_buffer("inv_freq", inv.to(device), persistent=False)

    def rope_tables(self, t: int, dtype):
        pos = torch.arange(t, device=self.inv_freq.device, dtype=torch.float32)
        f = torch.outer(pos, self.inv_freq)
        emb = torch.cat((f, f), dim=-1)
        return emb.cos().to(dtype), emb.sin().to(dtype)

    @torch.no_grad()
    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        x = self.model.embed_tokens(ids)
        cos, sin = self.rope_tables(ids.shape[1], torch.float32)
        for layer in self.model.layers:
            x = layer(x, cos, sin)
        return self.model.norm(x)

    def linear_modules(self) -> dict:
        """HF-style names -> Linear modules (``state.named_modules``)."""
        return {n: m for n, m in self.named_modules() if isinstance(m, torch.nn.Linear)}

    def linear_weights(self) -> dict:
        """``<module>.weight`` -> weight tensor (``state.named_weights``)."""
        return {f"{n}.weight": m.weight for n, m in self.linear_modules().items()}


def calibration_batches(vocab: int, sequences: int, seq_len: int, batch: int, seed: int = 1, device="cpu"):
    """Uniform-random token ids [batch, seq_len], ``sequences`` in all (the last batch may be
    smaller), from one seeded CPU generator."""
    g = torch.Generator().manual_seed(seed)
    done = 0
    while done < sequences:
        b = min(batch, sequences - done)
        yield torch.randint(0, vocab, (b, seq_len), generator=g).to(device)
        done += b


def drive(model: torch.nn.Module, batches):
    """Run the calibration forward on each batch (firing every hook the modifiers attached),
    then yield the batch to the session."""
    for b in batches:
        model(b)
        yield b
