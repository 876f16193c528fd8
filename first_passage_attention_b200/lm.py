"""Language-model training step built on the FirstPassageAttention layer (the reference's README describes this
model; the reference repository ships only the layer, kernel.py:512-530).

The model is a GPT-2-small-shaped decoder: token embedding (no positional embedding: FPA's field carries order),
`n_layers` pre-LayerNorm blocks of FirstPassageAttention and a 4x GELU MLP, a final LayerNorm and an output layer
tied to the embedding. Each block's field is the layer's own: per head delta, g, h are linear maps of x,
W = cumsum(delta), phi = W + g, psi = W + h, beta = softplus(beta_raw).

`LMTrainer.step` runs one optimisation step: fp16 autocast forward, cross-entropy of the next token, loss scaling
(torch.amp.GradScaler), backward, AdamW. Under torch.distributed the model is wrapped in DistributedDataParallel,
whose gradient all-reduce runs over NCCL.
"""
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from .ops import FirstPassageAttention


@dataclass
class LMConfig:
    vocab: int = 50304
    d_model: int = 768
    n_heads: int = 12
    n_layers: int = 12
    tau: float = 1.0
    beta_init: float = 1.0


class MLP(nn.Module):
    def __init__(self, d_model):
        super().__init__()
        self.fc = nn.Linear(d_model, 4 * d_model)
        self.proj = nn.Linear(4 * d_model, d_model)

    def forward(self, x):
        return self.proj(F.gelu(self.fc(x), approximate="tanh"))


class Block(nn.Module):
    def __init__(self, cfg, impl):
        super().__init__()
        self.ln1 = nn.LayerNorm(cfg.d_model)
        self.attn = FirstPassageAttention(cfg.d_model, cfg.n_heads, tau=cfg.tau, beta_init=cfg.beta_init, impl=impl)
        self.ln2 = nn.LayerNorm(cfg.d_model)
        self.mlp = MLP(cfg.d_model)

    def forward(self, x):
        x = x + self.attn(self.ln1(x))
        return x + self.mlp(self.ln2(x))


class FPALanguageModel(nn.Module):
    def __init__(self, cfg=LMConfig(), impl=None):
        super().__init__()
        self.cfg = cfg
        self.wte = nn.Embedding(cfg.vocab, cfg.d_model)
        self.blocks = nn.ModuleList(Block(cfg, impl) for _ in range(cfg.n_layers))
        self.ln_f = nn.LayerNorm(cfg.d_model)
        self.apply(self._init)

    @staticmethod
    def _init(m):
        if isinstance(m, nn.Linear):
            nn.init.normal_(m.weight, std=0.02)
            if m.bias is not None:
                nn.init.zeros_(m.bias)
        elif isinstance(m, nn.Embedding):
            nn.init.normal_(m.weight, std=0.02)

    def forward(self, idx):
        x = self.wte(idx)
        for blk in self.blocks:
            x = blk(x)
        return F.linear(self.ln_f(x), self.wte.weight)  # output layer tied to the embedding

    def n_params(self):
        return sum(p.numel() for p in self.parameters())


def make_tokens(batch, T, vocab, seed, device):
    """Token ids uniform over the vocabulary, [batch, T + 1] (inputs and next-token targets)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randint(0, vocab, (batch, T + 1), generator=g).to(device)


class LMTrainer:
    """One training step per call: fp16 autocast, next-token cross-entropy, GradScaler, AdamW; DDP when the
    default process group is initialised with more than one rank."""

    def __init__(self, model, lr=3e-4, weight_decay=0.1, ddp=None):
        self.model = model
        if ddp is None:
            ddp = torch.distributed.is_available() and torch.distributed.is_initialized() and \
                torch.distributed.get_world_size() > 1
        if ddp:
            dev = next(model.parameters()).device
            self.net = nn.parallel.DistributedDataParallel(model, device_ids=[dev.index] if dev.type == "cuda" else None)
        else:
            self.net = model
        dev_type = next(model.parameters()).device.type
        self.opt = torch.optim.AdamW(model.parameters(), lr=lr, weight_decay=weight_decay, betas=(0.9, 0.95),
                                     fused=dev_type == "cuda")
        self.amp = dev_type == "cuda"
        self.scaler = torch.amp.GradScaler("cuda", enabled=self.amp)

    def loss(self, tokens):
        inp, tgt = tokens[:, :-1], tokens[:, 1:]
        with torch.autocast(device_type="cuda", dtype=torch.float16, enabled=self.amp):
            logits = self.net(inp)
        return F.cross_entropy(logits.float().reshape(-1, logits.shape[-1]), tgt.reshape(-1))

    def step(self, tokens):
        """One optimisation step; returns the loss (a 0-d tensor on the model's device, not synchronised)."""
        loss = self.loss(tokens)
        self.scaler.scale(loss).backward()
        self.scaler.step(self.opt)
        self.scaler.update()
        self.opt.zero_grad(set_to_none=True)
        return loss.detach()
