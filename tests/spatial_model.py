"""A small price-model-style network whose attention is written as the
eager RBF chain, for the compiled-model check (benchmark config 5).

Each block is pre-norm: RBF attention of every token (the target and its
comparables) over all tokens, with a per-head width sigma_h (coefficient
1 / (2 sigma_h^2)) and an additive key-padding bias, then a GELU MLP. The
attention is spelled the way a model author writes it eagerly,

    d2 = (q.unsqueeze(-2) - k.unsqueeze(-3)).pow(2).sum(-1)
    w = softmax(-d2 / (2 exp(log_sigma)^2) + bias)
    out = w @ v

which is the chain the reference's compile pass recognises and replaces
with torch.ops.vectra.rbf_attention (compiler/vectra_compiler/pattern.py:
90-112 lists the recognised spellings). `formulation` selects among them:
divisor or multiplier coefficient, softmax or exp / sum normalisation.
"""

import torch
from torch import nn


class SpatialBlock(nn.Module):

    def __init__(self, d_model, heads, ffn, coefficient='divisor',
                 normalization='softmax'):
        super().__init__()
        self.heads, self.dh = heads, d_model // heads
        self.coefficient, self.normalization = coefficient, normalization
        self.norm1 = nn.LayerNorm(d_model)
        self.qkv = nn.Linear(d_model, 3 * d_model)
        self.out = nn.Linear(d_model, d_model)
        self.log_sigma = nn.Parameter(0.3 * torch.randn(1, heads, 1, 1) + 0.7)
        self.norm2 = nn.LayerNorm(d_model)
        self.ff = nn.Sequential(nn.Linear(d_model, ffn), nn.GELU(),
                                nn.Linear(ffn, d_model))

    def attend(self, q, k, v, bias):
        d2 = (q.unsqueeze(-2) - k.unsqueeze(-3)).pow(2).sum(-1)
        if self.coefficient == 'divisor':
            logits = -d2 / (2 * torch.exp(self.log_sigma) ** 2)
        else:
            logits = -d2 * (0.5 * torch.exp(-2 * self.log_sigma))
        logits = logits + bias
        if self.normalization == 'softmax':
            w = torch.softmax(logits, dim=-1)
        else:
            e = torch.exp(logits)
            w = e / e.sum(-1, keepdim=True)
        return w @ v

    def forward(self, x, bias):
        b, n, _ = x.shape
        qkv = self.qkv(self.norm1(x)).view(b, n, 3, self.heads, self.dh)
        q, k, v = qkv.permute(2, 0, 3, 1, 4)
        a = self.attend(q, k, v, bias).transpose(1, 2).reshape(b, n, -1)
        x = x + self.out(a)
        return x + self.ff(self.norm2(x))


class SpatialNet(nn.Module):
    """Features of a target and its comparables [B, N, F] plus a key-padding
    bias [B, 1, 1, N] (0 valid, -inf padded) -> one prediction per target
    (read from token 0)."""

    def __init__(self, features=48, d_model=256, heads=8, layers=3,
                 ffn=1024, formulations=None):
        super().__init__()
        formulations = formulations or [('divisor', 'softmax')] * layers
        self.embed = nn.Linear(features, d_model)
        self.blocks = nn.ModuleList(
            SpatialBlock(d_model, heads, ffn, c, s) for c, s in formulations)
        self.norm = nn.LayerNorm(d_model)
        self.head = nn.Linear(d_model, 1)

    def forward(self, x, bias):
        h = self.embed(x)
        for block in self.blocks:
            h = block(h, bias)
        return self.head(self.norm(h[:, 0])).squeeze(-1)


def inputs(batch, comparables=64, features=48, seed=0, device='cpu',
           dtype=torch.float32):
    """Seeded features and a padding bias: target + `comparables` tokens,
    with a per-row count of valid comparables in [8, comparables]."""
    gen = torch.Generator().manual_seed(seed)
    n = comparables + 1
    x = torch.randn(batch, n, features, generator=gen)
    valid = torch.randint(8, comparables + 1, (batch,), generator=gen) + 1
    keep = torch.arange(n)[None, :] < valid[:, None]
    bias = torch.zeros(batch, n).masked_fill(~keep, float('-inf'))
    return (x.to(device=device, dtype=dtype),
            bias[:, None, None, :].to(device=device, dtype=dtype))
