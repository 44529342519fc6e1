"""Drop-in attention module backed by libllattn's sm_100a kernels.

``LocalLatentAttentionB200(config)`` has exactly the parameters, state_dict
keys and shapes of the reference's PyTorch ``LocalLatentAttention``
(models.py:61-96) — fused ``qkv_proj``, ``rq_proj``, ``rkv_proj``, ``r_out``,
``out`` (all with bias) and the shared ``gate_local``/``gate_remote``
``Linear(head_dim, 1, bias=False)`` — so checkpoints interchange, and the
same forward math (models.py:307-462). The projections stay cuBLAS GEMMs;
pooling and everything between the projections run in the custom ops of
``ops.py``. On CUDA the block runs as one autograd node
(``ops.BlockFunction``) whose backward fuses the gradient accumulation and
bias reductions around those GEMMs (under autocast, on the input and
weights cast to the autocast dtype); with profiling on, or parameters of
another dtype than the input outside autocast, it runs layer by layer under
autograd.

``build_attention(config)`` is the module switch of models.py:465-488: with
``config.use_triton_kernel`` set it returns this module.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch import Tensor

from . import ops


@dataclass
class DecodeCache:
    """Generation state of one LocalLatentAttentionB200 layer: the qkv_proj
    rows [B, capacity, 3d] and the attention inputs [B, capacity, d] of every
    token so far. The inputs are kept (not only a key/value window) because
    the latent chunking depends on the whole prefix length
    (models.py:175-183): chunk means are re-pooled from them each step."""

    capacity: int
    qkv: Tensor | None = None
    x: Tensor | None = None
    length: int = 0


class LocalLatentAttentionB200(nn.Module):
    def __init__(self, config) -> None:
        super().__init__()
        assert config.d_model % config.n_heads == 0
        assert config.latent_d_model % config.latent_heads == 0
        self.d_model = config.d_model
        self.n_heads = config.n_heads
        self.head_dim = config.d_model // config.n_heads
        self.window = config.local_window
        self.local_block_size = config.local_block_size
        self.latent_tokens = config.latent_tokens
        self.latent_heads = config.latent_heads
        self.latent_d_model = config.latent_d_model
        self.latent_head_dim = config.latent_d_model // config.latent_heads
        self.latent_query_block_size = max(0, config.latent_query_block_size)
        self.qkv_proj = nn.Linear(config.d_model, 3 * config.d_model)
        self.rq_proj = nn.Linear(config.d_model, config.latent_d_model)
        self.rkv_proj = nn.Linear(config.d_model, 2 * config.latent_d_model)
        self.r_out = nn.Linear(config.latent_d_model, config.d_model)
        self.out = nn.Linear(config.d_model, config.d_model)
        self.gate_local = nn.Linear(self.head_dim, 1, bias=False)
        self.gate_remote = nn.Linear(self.head_dim, 1, bias=False)
        self.dropout = nn.Dropout(config.dropout)
        self._n_layers = getattr(config, "n_layers", 1)
        # Added to the local gate logit; 0 reproduces the reference. Not a
        # parameter and not saved, so state_dicts stay interchangeable.
        self.gate_bias = 0.0
        self.profile_enabled = False
        self.profile_totals: dict[str, float] = {}
        self.profile_steps = 0
        self._profile_events: list = []

    # models.py:98-129: checkpoints with split q/k/v or rk/rv projections load
    # into the fused layout.
    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys,
                              unexpected_keys, error_msgs) -> None:
        def fuse(new: str, olds: tuple[str, ...]) -> None:
            for kind in ("weight", "bias"):
                key = f"{prefix}{new}.{kind}"
                old_keys = [f"{prefix}{o}.{kind}" for o in olds]
                if key not in state_dict and all(k in state_dict for k in old_keys):
                    state_dict[key] = torch.cat([state_dict.pop(k) for k in old_keys], dim=0)

        fuse("qkv_proj", ("q_proj", "k_proj", "v_proj"))
        fuse("rkv_proj", ("rk_proj", "rv_proj"))
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys,
                                      unexpected_keys, error_msgs)

    # --- profiling API of models.py:131-157 --------------------------------
    def set_profile(self, enabled: bool) -> None:
        self.profile_enabled = enabled
        self.profile_totals = {}
        self.profile_steps = 0
        self._profile_events = []

    def _drain_profile(self) -> None:
        for ev, geo in self._profile_events:
            ev[-1].synchronize()
            qkv = ev[0].elapsed_time(ev[1])
            pool = ev[1].elapsed_time(ev[2])
            core = ev[2].elapsed_time(ev[3])
            total = ev[0].elapsed_time(ev[4])
            for k, v in (("total_ms", total), ("qkv_ms", qkv), ("pool_ms", pool),
                         ("local_attention_ms", core), ("latent_attention_ms", 0.0),
                         ("gate_mix_ms", 0.0)):
                self.profile_totals[k] = self.profile_totals.get(k, 0.0) + v
            for k, v in geo.items():
                self.profile_totals[k] = self.profile_totals.get(k, 0.0) + float(v)
            self.profile_steps += 1
        self._profile_events = []

    def get_profile_stats(self) -> dict[str, float]:
        """Same keys as the reference (models.py:136-157). The fused op runs
        local + latent + gate as one library call: its time is reported as
        local_attention_ms and the latent / gate entries are 0 (per-kernel
        times come from the library's event profiler, llattn_profile_*).
        gate_mean is the mean local gate weight w_l over tokens and heads,
        recomputed in profile mode from the op's saved tensors (the fused
        kernels never materialise the weights)."""
        if not self.profile_enabled:
            return {}
        self._drain_profile()
        if self.profile_steps == 0:
            return {}
        n = self.profile_steps
        t = self.profile_totals
        return {
            "profile_local_latent_total_ms": t["total_ms"] / n,
            "profile_qkv_ms": t["qkv_ms"] / n,
            "profile_pool_ms": t["pool_ms"] / n,
            "profile_local_attention_ms": t["local_attention_ms"] / n,
            "profile_latent_attention_ms": t["latent_attention_ms"] / n,
            "profile_gate_mix_ms": t["gate_mix_ms"] / n,
            "profile_gate_mean": t["gate_mean"] / n,
            "profile_seq_len": t["seq_len"] / n,
            "profile_local_block_size": t["local_block_size"] / n,
            "profile_latent_count": t["latent_count"] / n,
            "profile_latent_chunk_size": t["chunk_size"] / n,
            "profile_latent_query_block_size": t["latent_query_block_size"] / n,
        }

    def forward(self, x: Tensor) -> Tensor:
        if self.training and self.dropout.p > 0:
            raise NotImplementedError("LocalLatentAttentionB200 does not implement attention dropout")
        B, T, d = x.shape
        prof = self.profile_enabled and x.is_cuda
        if x.is_cuda and not prof:
            params = (self.qkv_proj.weight, self.qkv_proj.bias, self.rq_proj.weight, self.rq_proj.bias,
                      self.rkv_proj.weight, self.rkv_proj.bias, self.r_out.weight, self.r_out.bias,
                      self.gate_local.weight, self.gate_remote.weight, self.out.weight, self.out.bias)
            cfg = (self.n_heads, self.latent_heads, self.window, self.local_block_size, self.latent_tokens,
                   self.latent_query_block_size, self.gate_bias)
            if torch.is_autocast_enabled("cuda"):
                # what autocast does to each linear layer, once for the block:
                # input and weights cast to the autocast dtype (autograd casts
                # the gradients back), the block itself run without autocast
                dt = torch.get_autocast_dtype("cuda")
                if dt in (torch.bfloat16, torch.float32):
                    with torch.autocast("cuda", enabled=False):
                        return ops.BlockFunction.apply(x.to(dt), *(p.to(dt) for p in params), cfg)
            elif all(p.dtype == x.dtype for p in params):
                return ops.BlockFunction.apply(x, *params, cfg)
        # per-layer path: profiling (events between the stages), mixed dtypes
        if prof:
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
            ev[0].record()
        qkv = self.qkv_proj(x)
        if prof:
            ev[1].record()
        pooled = ops.pool_chunks(x, self.latent_tokens)
        gkv = self.rkv_proj(pooled)
        if self.latent_query_block_size > 1:
            qsrc = ops.pool_query_blocks(x, self.latent_tokens, self.latent_query_block_size)
        else:
            qsrc = x
        rq = self.rq_proj(qsrc)
        if prof:
            ev[2].record()
        mixed = ops.llattn_attention(
            qkv, rq, gkv, self.r_out.weight, self.r_out.bias, self.gate_local.weight,
            self.gate_remote.weight, n_heads=self.n_heads, latent_heads=self.latent_heads,
            window=self.window, local_block_size=self.local_block_size,
            latent_tokens=self.latent_tokens, latent_query_block_size=self.latent_query_block_size,
            gate_bias=self.gate_bias)
        if prof:
            ev[3].record()
        y = self.out(mixed)
        if prof:
            ev[4].record()
            gate_mean = self._gate_mean(qkv, rq, gkv)  # after the timed phases
            geo = ops.geometry(T, self.latent_tokens, self.latent_query_block_size, self.window,
                               self.local_block_size)
            self._profile_events.append((ev, {
                "gate_mean": gate_mean, "seq_len": T, "local_block_size": geo["local_span"],
                "latent_count": geo["n_chunks"], "chunk_size": geo["chunk"],
                "latent_query_block_size": geo["qblock"]}))
        return y

    @torch.no_grad()
    def _gate_mean(self, qkv: Tensor, rq: Tensor, gkv: Tensor) -> Tensor:
        """Mean of w_l = sigmoid(local.g_l + gate_bias - remote.g_r) (the
        weight of models.py:424-437), from the core op's saved local output
        and latent rows: profile mode only. Returned as a device scalar."""
        dt = qkv.dtype
        outs = ops.attn_fwd(qkv.contiguous(), rq.to(dt).contiguous(), gkv.to(dt).contiguous(),
                            self.r_out.weight.to(dt).contiguous(), self.r_out.bias.float().contiguous(),
                            self.gate_local.weight.float().reshape(-1).contiguous(),
                            self.gate_remote.weight.float().reshape(-1).contiguous(), self.n_heads,
                            self.latent_heads, self.window, self.local_block_size, self.latent_tokens,
                            self.latent_query_block_size, float(self.gate_bias))
        local_out, lat = outs[1], outs[3]
        B, T, d = local_out.shape
        remote = F.linear(lat.float(), self.r_out.weight.float(), self.r_out.bias.float())
        qbs = ops.geometry(T, self.latent_tokens, self.latent_query_block_size)["qblock"]
        if qbs > 1:
            remote = remote.repeat_interleave(qbs, dim=1)[:, :T]
        hd = d // self.n_heads
        sl = local_out.float().view(B, T, self.n_heads, hd) @ self.gate_local.weight.float().reshape(-1)
        sr = remote.view(B, T, self.n_heads, hd) @ self.gate_remote.weight.float().reshape(-1)
        return torch.sigmoid(sl + self.gate_bias - sr).mean()

    # --- incremental generation ------------------------------------------

    def new_decode_cache(self, capacity: int) -> DecodeCache:
        return DecodeCache(capacity=int(capacity))

    def _store(self, cache: DecodeCache, x: Tensor, qkv: Tensor) -> None:
        B, n, d = x.shape
        if cache.qkv is None:
            cache.qkv = torch.empty(B, cache.capacity, qkv.shape[-1], dtype=qkv.dtype, device=x.device)
            cache.x = torch.empty(B, cache.capacity, d, dtype=x.dtype, device=x.device)
        if cache.length + n > cache.capacity:
            raise RuntimeError(f"llattn: decode cache full ({cache.length} + {n} > {cache.capacity} tokens)")
        cache.qkv[:, cache.length:cache.length + n] = qkv
        cache.x[:, cache.length:cache.length + n] = x
        cache.length += n

    def prefill(self, x: Tensor, cache: DecodeCache) -> Tensor:
        """Full forward of the first tokens [B, n, d] that also fills the cache."""
        if cache.length != 0:
            raise RuntimeError("llattn: prefill needs an empty decode cache")
        with torch.no_grad():
            y = self(x)
            self._store(cache, x, self.qkv_proj(x))
        return y

    def decode(self, x: Tensor, cache: DecodeCache) -> Tensor:
        """Outputs [B, n, d] of n new tokens [B, n, d] appended after the
        cached prefix, one token at a time. Row i equals the last row of
        this module's forward over the prefix extended by tokens 0..i (the
        computation the reference's generation loop repeats per token,
        generate.py:188-202), from the cache: qkv of one row, chunk means
        re-pooled over the prefix (the latent geometry follows its length),
        one ``llattn_decode`` launch."""
        ys = []
        with torch.no_grad():
            for i in range(x.shape[1]):
                xt = x[:, i:i + 1]
                self._store(cache, xt, self.qkv_proj(xt))
                T = cache.length
                xs = cache.x[:, :T].contiguous()
                gkv = self.rkv_proj(ops.pool_chunks(xs, self.latent_tokens))
                if self.latent_query_block_size > 1:
                    qrows = ops.pool_query_blocks(xs, self.latent_tokens, self.latent_query_block_size)
                    qb = ops.geometry(T, self.latent_tokens, self.latent_query_block_size)["qblock"]
                    src = qrows[:, (T - 1) // qb]
                else:
                    src = xt[:, 0]
                rq_row = self.rq_proj(src)
                mixed = ops.decode_core(
                    cache.qkv, T, rq_row, gkv, self.r_out.weight, self.r_out.bias, self.gate_local.weight,
                    self.gate_remote.weight, n_heads=self.n_heads, latent_heads=self.latent_heads,
                    window=self.window, local_block_size=self.local_block_size,
                    latent_tokens=self.latent_tokens, latent_query_block_size=self.latent_query_block_size,
                    gate_bias=self.gate_bias)
                ys.append(self.out(mixed))
        return torch.stack(ys, dim=1)


def build_attention(config) -> nn.Module:
    """The module switch of models.py:465-488: ``use_triton_kernel`` selects
    the B200 kernels, otherwise the caller's own PyTorch module is expected,
    so this always returns the B200 module (the reference constructor takes
    the same ModelConfig)."""
    return LocalLatentAttentionB200(config)
