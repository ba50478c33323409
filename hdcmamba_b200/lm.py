"""Language-model wrapper and the benchmark configurations.

The reference keeps its LM wrappers outside the package (train.py:116-151,
train_fineweb.py:23-94): token embedding -> HdcMamba backbone -> LayerNorm ->
lm_head tied to the embedding.  ``HdcMambaLM`` is that wrapper; the head is
``F.linear(h, embedding.weight)`` so that no extra Linear is constructed (an
extra module would consume RNG and change seeded weights).

``build_lm(cfg)`` creates the seeded synthetic-weight models of the benchmark
configurations: seed 0, every Linear/Conv1d/Embedding weight re-drawn
N(0, 0.02) in ``named_parameters`` order, norms at gamma=1 / beta=0, biases,
A_log, decay_log and gamma_buf at the reference's own init.
"""
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from .model import HdcMamba9v3Block, HdcMamba9v3Model, final_layer_norm


class HdcMambaLM(nn.Module):
    """Embedding -> blocks (or HdcMamba9v3Model) -> LayerNorm -> tied head."""

    def __init__(self, vocab_size, d_model, n_layers, d_state, num_heads, chunk_size=256, use_model=True,
                 semantics="fixed"):
        super().__init__()
        self.use_model = use_model
        self.embedding = nn.Embedding(vocab_size, d_model)
        if use_model:
            self.backbone = HdcMamba9v3Model(d_model, n_layers, d_state, num_slots=32, num_heads=num_heads,
                                             semantics=semantics)
        else:
            self.layers = nn.ModuleList([HdcMamba9v3Block(d_model=d_model, d_state=d_state, num_heads=num_heads,
                                                          chunk_size=chunk_size, semantics=semantics)
                                         for _ in range(n_layers)])
        self.norm = nn.LayerNorm(d_model)

    def hidden(self, ids):
        h = self.embedding(ids)  # a fresh activation: the layers update it in place
        if self.use_model:
            return self.backbone._forward(h, owns_input=True)
        for layer in self.layers:
            h = layer._forward_inplace(h)
        return h

    def forward(self, ids):
        return F.linear(final_layer_norm(self.norm, self.hidden(ids)), self.embedding.weight)


@dataclass(frozen=True)
class LMConfig:
    name: str
    vocab: int
    d_model: int
    n_layers: int
    d_state: int
    num_heads: int
    chunk_size: int
    use_model: bool
    batch: int
    seq_len: int


CONFIGS = {
    # the reference's CPU-runnable plumbing case (fp32)
    "c1": LMConfig("c1", 4096, 256, 2, 64, 8, 64, False, 1, 512),
    # 24 x d1024, H16, ds128 (train_fineweb.py:38), chunk 256 (model.py:399)
    "c4": LMConfig("c4", 50304, 1024, 24, 128, 16, 256, True, 8, 4096),
    # 12 x d768, H12, ds64 (train_fineweb.py:33), chunk 256, B1 x L32768
    "c5": LMConfig("c5", 50304, 768, 12, 64, 12, 256, True, 1, 32768),
}


def reinit_(module, std=0.02):
    """Re-draw every Linear / Conv1d / Embedding weight N(0, std) in named_parameters order."""
    mods = dict(module.named_modules())
    with torch.no_grad():
        for name, p in module.named_parameters():
            owner = mods[name.rsplit(".", 1)[0]] if "." in name else module
            if name.endswith("weight") and isinstance(owner, (nn.Linear, nn.Conv1d, nn.Embedding)):
                p.normal_(0.0, std)
    return module


def build_lm(cfg, seed=0, semantics="fixed"):
    """Seeded synthetic-weight LM for a config (constructed on CPU, fp32)."""
    if isinstance(cfg, str):
        cfg = CONFIGS[cfg]
    torch.manual_seed(seed)
    lm = HdcMambaLM(cfg.vocab, cfg.d_model, cfg.n_layers, cfg.d_state, cfg.num_heads, cfg.chunk_size,
                    cfg.use_model, semantics=semantics)
    return reinit_(lm).eval()


def synthetic_ids(cfg, seed=0, batch=None, seq_len=None):
    """Uniform token ids [B, L] from a dedicated generator."""
    if isinstance(cfg, str):
        cfg = CONFIGS[cfg]
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, cfg.vocab, (batch or cfg.batch, seq_len or cfg.seq_len), generator=g)
