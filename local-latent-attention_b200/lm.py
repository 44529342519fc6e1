"""Decoder-only language model around the drop-in attention block, the
data-parallel training harness of this package (and its generation loop).

What is kept from the reference, because checkpoints and configs must move
between the two (each an interface, not an implementation):
  * the ModelConfig fields (models.py:21-37);
  * the parameter names: embedding, position, blocks.{i}.norm1 / attn /
    norm2 / ff.w1 / ff.w2, norm, and lm_head tied to the embedding
    (models.py:505-518);
  * the pre-norm residual layer x + attn(norm1(x)), then x + ff(norm2(x)),
    with RMSNorm eps 1e-6 and an exact-GELU MLP (models.py:40-58, 491-502);
  * the GPT-2 style initial values (models.py:520-546): N(0, 0.02) for every
    linear weight and embedding, zero biases, the weights of the residual
    output projections (out, r_out, w2) scaled by 1/sqrt(2 n_layers), drawn
    in module order so that a seeded model equals the reference's.

Where the reference tree is importable, ``use_in_reference(models)`` points
its own attention switch (models.py:465-488) at this package instead, so the
reference's LocalLatentLM runs the B200 block in every layer.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint

from .module import LocalLatentAttentionB200


@dataclass
class ModelConfig:
    """The reference's ModelConfig fields (models.py:21-37)."""

    vocab_size: int = 128
    max_seq_len: int = 1024
    d_model: int = 128
    n_heads: int = 4
    n_layers: int = 4
    d_ff: int = 256
    dropout: float = 0.0
    local_window: int = 64
    local_block_size: int = 256
    latent_tokens: int = 16
    latent_d_model: int = 64
    latent_heads: int = 2
    latent_query_block_size: int = 0
    checkpoint_blocks: bool = False
    use_triton_kernel: bool = True


RESIDUAL_OUTPUTS = ("out", "r_out", "w2")  # linear layers whose output is added to the residual stream


class DecoderLayer(nn.Module):
    """norm1 -> LocalLatentAttentionB200 -> residual add, norm2 -> MLP ->
    residual add. The MLP is an nn.ModuleDict {w1, w2} so its parameters
    keep the reference's ff.w1 / ff.w2 names."""

    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        d = config.d_model
        self.norm1 = nn.RMSNorm(d, eps=1e-6)
        self.attn = LocalLatentAttentionB200(config)
        self.norm2 = nn.RMSNorm(d, eps=1e-6)
        self.ff = nn.ModuleDict({"w1": nn.Linear(d, config.d_ff), "w2": nn.Linear(config.d_ff, d)})
        self.p_drop = config.dropout

    def mlp(self, h: torch.Tensor) -> torch.Tensor:
        h = self.ff["w2"](F.gelu(self.ff["w1"](h)))
        return F.dropout(h, self.p_drop, self.training) if self.p_drop else h

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = x + self.attn(self.norm1(x))
        return x + self.mlp(self.norm2(x))


def gpt2_init_(model: nn.Module, n_layers: int, skip: nn.Module | None = None) -> None:
    """GPT-2 style initial values in module order (see the module docstring);
    `skip` (the tied output head) keeps the embedding's values."""
    residual_scale = (2.0 * n_layers) ** -0.5
    with torch.no_grad():
        for name, mod in model.named_modules():
            if mod is skip:
                continue
            if isinstance(mod, nn.Embedding):
                mod.weight.normal_(0.0, 0.02)
            elif isinstance(mod, nn.Linear):
                mod.weight.normal_(0.0, 0.02)
                if mod.bias is not None:
                    mod.bias.zero_()
                if name.split(".")[-1] in RESIDUAL_OUTPUTS:
                    mod.weight.mul_(residual_scale)


class LocalLatentLM(nn.Module):
    """Token + learned position embeddings, n_layers DecoderLayers, a final
    RMSNorm and the tied output head -> logits [B, T, vocab]."""

    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        self.config = config
        self.checkpoint_blocks = config.checkpoint_blocks
        self.embedding = nn.Embedding(config.vocab_size, config.d_model)
        self.position = nn.Embedding(config.max_seq_len, config.d_model)
        self.blocks = nn.ModuleList(DecoderLayer(config) for _ in range(config.n_layers))
        self.norm = nn.RMSNorm(config.d_model, eps=1e-6)
        self.lm_head = nn.Linear(config.d_model, config.vocab_size, bias=False)
        self.lm_head.weight = self.embedding.weight
        gpt2_init_(self, config.n_layers, skip=self.lm_head)

    def set_profile(self, enabled: bool) -> None:
        for layer in self.blocks:
            layer.attn.set_profile(enabled)

    def get_profile_stats(self) -> dict[str, float]:
        """Per-phase attention times averaged over the layers that recorded any."""
        per_layer = [s for s in (layer.attn.get_profile_stats() for layer in self.blocks) if s]
        keys = {k for s in per_layer for k in s}
        return {k: sum(s.get(k, 0.0) for s in per_layer) / len(per_layer) for k in keys} if per_layer else {}

    def forward(self, input_ids: torch.Tensor, targets: torch.Tensor | None = None) -> torch.Tensor:
        """Logits [B, T, vocab]; with `targets` [B, T], the mean next-token
        cross-entropy instead (computed in fp32 by `self.loss_head`, which a
        caller may replace by a compiled version of itself)."""
        T = input_ids.shape[1]
        x = self.embedding(input_ids) + self.position.weight[:T].unsqueeze(0)
        remat = self.checkpoint_blocks and self.training
        for layer in self.blocks:
            x = checkpoint(layer, x, use_reentrant=False) if remat else layer(x)
        if targets is not None:
            return self.loss_head(x, targets)
        return self.lm_head(self.norm(x))

    def loss_head(self, x: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        logits = self.lm_head(self.norm(x))
        return F.cross_entropy(logits.float().reshape(-1, logits.shape[-1]), targets.reshape(-1))


    # --- generation ---------------------------------------------------------

    @torch.no_grad()
    def generate(self, input_ids: torch.Tensor, max_new_tokens: int, temperature: float = 0.0,
                 top_k: int = 0, generator: torch.Generator | None = None,
                 incremental: bool = True) -> torch.Tensor:
        """Append max_new_tokens sampled tokens to input_ids [B, P] -> [B, P + n].

        The loop of the reference's generate.py:188-202 (context = the last
        max_seq_len tokens, next token from the last position's logits;
        temperature <= 0 is greedy, top_k > 0 keeps the k largest logits).
        With ``incremental`` each step runs only the new token through the
        layers, the attention layers from their decode caches; once the
        sequence outgrows max_seq_len (the context then slides and positions
        are re-based) it falls back to the full forward, as the reference."""
        ids = input_ids
        caches = None
        for _ in range(max_new_tokens):
            T = ids.shape[1]
            if incremental and T <= self.config.max_seq_len:
                if caches is None:
                    cap = min(self.config.max_seq_len, T + max_new_tokens)
                    caches = [blk.attn.new_decode_cache(cap) for blk in self.blocks]
                    logits = self._prefill(ids, caches)
                else:
                    logits = self._decode_one(ids[:, -1:], T - 1, caches)
            else:
                logits = self(ids[:, -self.config.max_seq_len:])[:, -1]
            ids = torch.cat([ids, _sample(logits.float(), temperature, top_k, generator)], dim=1)
        return ids

    def _prefill(self, ids: torch.Tensor, caches) -> torch.Tensor:
        T = ids.shape[1]
        x = self.embedding(ids) + self.position(torch.arange(T, device=ids.device)).unsqueeze(0)
        for blk, cache in zip(self.blocks, caches):
            x = x + blk.attn.prefill(blk.norm1(x), cache)
            x = x + blk.mlp(blk.norm2(x))
        return self.lm_head(self.norm(x[:, -1]))

    def _decode_one(self, tok: torch.Tensor, pos: int, caches) -> torch.Tensor:
        x = self.embedding(tok) + self.position.weight[pos].view(1, 1, -1)
        for blk, cache in zip(self.blocks, caches):
            x = x + blk.attn.decode(blk.norm1(x), cache)
            x = x + blk.mlp(blk.norm2(x))
        return self.lm_head(self.norm(x[:, -1]))


def use_in_reference(models_module) -> None:
    """Make the reference's models module build this package's block: after
    the call, its _build_attention (models.py:465-488) returns
    LocalLatentAttentionB200 for a config with use_triton_kernel set, so the
    reference's own TransformerBlock / LocalLatentLM run the B200 kernels
    (the same switch train.py's --use-triton-kernel sets)."""
    fallback = models_module._build_attention

    def build(config):
        if getattr(config, "use_triton_kernel", False):
            return LocalLatentAttentionB200(config)
        return fallback(config)

    models_module._build_attention = build


def _sample(logits: torch.Tensor, temperature: float, top_k: int, generator) -> torch.Tensor:
    """Next token [B, 1] from last-position logits [B, V] (generate.py:42-110
    without its repetition penalty and n-gram ban, which filter logits on the host)."""
    if temperature <= 0.0:
        return logits.argmax(dim=-1, keepdim=True)
    logits = logits / temperature
    if 0 < top_k < logits.shape[-1]:
        kth = torch.topk(logits, top_k, dim=-1).values[:, -1:]
        logits = logits.masked_fill(logits < kth, float("-inf"))
    return torch.multinomial(torch.softmax(logits, dim=-1), 1, generator=generator)


def build_optimizer(model: nn.Module, lr: float = 3e-4, weight_decay: float = 0.1):
    """AdamW(beta 0.9/0.95), decay on >= 2-D params only (train.py:851-859)."""
    decay, no_decay = [], []
    for p in model.parameters():
        if p.requires_grad:
            (decay if p.dim() >= 2 else no_decay).append(p)
    groups = [{"params": decay, "weight_decay": weight_decay}, {"params": no_decay, "weight_decay": 0.0}]
    return torch.optim.AdamW(groups, lr=lr, betas=(0.9, 0.95), fused=torch.cuda.is_available())


def train_step(model: nn.Module, optimizer, ids: torch.Tensor, targets: torch.Tensor, grad_clip: float = 1.0,
               autocast_dtype=torch.bfloat16) -> torch.Tensor:
    """One optimiser step: bf16 autocast forward, cross-entropy, backward
    (DDP all-reduces the grads), clip, AdamW. Returns the loss (on device)."""
    with torch.autocast(device_type=ids.device.type, dtype=autocast_dtype):
        loss = model(ids, targets)
    loss.backward()
    torch.nn.utils.clip_grad_norm_(model.parameters(), grad_clip)
    optimizer.step()
    optimizer.zero_grad(set_to_none=True)
    return loss.detach()
