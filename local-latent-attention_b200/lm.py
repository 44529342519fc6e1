"""Decoder LM around the drop-in attention block: the reference's
LocalLatentLM (models.py:505-576) with LocalLatentAttentionB200 in every
layer. Used as the multi-GPU data-parallel training harness.

Same module tree and state_dict names as the reference (embedding,
position, blocks.{i}.norm1/attn/norm2/ff.w1/ff.w2, norm, tied lm_head), the
same pre-norm residual block (models.py:491-502) and GPT-2 style init
(models.py:520-546).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint

from .module import LocalLatentAttentionB200


@dataclass
class ModelConfig:
    """Field-for-field the reference's ModelConfig (models.py:21-37)."""

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


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x):
        return F.rms_norm(x, (self.weight.shape[0],), self.weight, self.eps)


class FeedForward(nn.Module):
    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        self.w1 = nn.Linear(config.d_model, config.d_ff)
        self.w2 = nn.Linear(config.d_ff, config.d_model)
        self.dropout = nn.Dropout(config.dropout)

    def forward(self, x):
        return self.dropout(self.w2(F.gelu(self.w1(x))))


class TransformerBlock(nn.Module):
    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        self.norm1 = RMSNorm(config.d_model)
        self.norm2 = RMSNorm(config.d_model)
        self.attn = LocalLatentAttentionB200(config)
        self.ff = FeedForward(config)

    def forward(self, x):
        x = x + self.attn(self.norm1(x))
        return x + self.ff(self.norm2(x))


class LocalLatentLM(nn.Module):
    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        self.config = config
        self.checkpoint_blocks = config.checkpoint_blocks
        self.embedding = nn.Embedding(config.vocab_size, config.d_model)
        self.position = nn.Embedding(config.max_seq_len, config.d_model)
        self.blocks = nn.ModuleList([TransformerBlock(config) for _ in range(config.n_layers)])
        self.norm = RMSNorm(config.d_model)
        self.lm_head = nn.Linear(config.d_model, config.vocab_size, bias=False)
        self.lm_head.weight = self.embedding.weight
        self._init_weights(config.n_layers)

    def _init_weights(self, n_layers: int) -> None:
        output_projs = {"out", "r_out", "w2"}
        for name, module in self.named_modules():
            if module is self.lm_head:
                continue
            if isinstance(module, nn.Linear):
                nn.init.normal_(module.weight, mean=0.0, std=0.02)
                if module.bias is not None:
                    nn.init.zeros_(module.bias)
                if name.rsplit(".", 1)[-1] in output_projs:
                    module.weight.data.mul_(1.0 / math.sqrt(2 * n_layers))
            elif isinstance(module, nn.Embedding):
                nn.init.normal_(module.weight, mean=0.0, std=0.02)

    def set_profile(self, enabled: bool) -> None:
        for block in self.blocks:
            block.attn.set_profile(enabled)

    def get_profile_stats(self) -> dict[str, float]:
        totals: dict[str, float] = {}
        count = 0
        for block in self.blocks:
            stats = block.attn.get_profile_stats()
            if not stats:
                continue
            count += 1
            for k, v in stats.items():
                totals[k] = totals.get(k, 0.0) + v
        return {k: v / count for k, v in totals.items()} if count else {}

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        T = input_ids.shape[1]
        pos = torch.arange(T, device=input_ids.device)
        x = self.embedding(input_ids) + self.position(pos).unsqueeze(0)
        for block in self.blocks:
            if self.checkpoint_blocks and self.training:
                x = checkpoint(block, x, use_reentrant=False)
            else:
                x = block(x)
        return self.lm_head(self.norm(x))


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
            x = x + blk.ff(blk.norm2(x))
        return self.lm_head(self.norm(x[:, -1]))

    def _decode_one(self, tok: torch.Tensor, pos: int, caches) -> torch.Tensor:
        x = self.embedding(tok) + self.position.weight[pos].view(1, 1, -1)
        for blk, cache in zip(self.blocks, caches):
            x = x + blk.attn.decode(blk.norm1(x), cache)
            x = x + blk.ff(blk.norm2(x))
        return self.lm_head(self.norm(x[:, -1]))


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
        logits = model(ids)
        loss = F.cross_entropy(logits.float().reshape(-1, logits.shape[-1]), targets.reshape(-1))
    loss.backward()
    torch.nn.utils.clip_grad_norm_(model.parameters(), grad_clip)
    optimizer.step()
    optimizer.zero_grad(set_to_none=True)
    return loss.detach()
