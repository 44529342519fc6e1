"""Shared helpers of the parity tests: seeded inputs, the oracle run (CPU) and
the B200 run of the same block, and the error metric.

Error metrics, per tensor, both held to the same tolerance: max|a - b| /
max|b| (relative to the reference's largest magnitude) and the
Frobenius-relative ||a - b||_F / ||b||_F. Tolerances (from the parity
target): 1e-4 for float32 activations, 2e-2 for bfloat16.
"""

from __future__ import annotations

import torch

import llattn_oracle as O

TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.detach().double().cpu()
    b = b.detach().double().cpu()
    denom = b.abs().max().item()
    return (a - b).abs().max().item() / max(denom, 1e-30)


def frob_err(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.detach().double().cpu()
    b = b.detach().double().cpu()
    return (a - b).norm().item() / max(b.norm().item(), 1e-30)


def make_cfg(dims: dict) -> tuple[int, int, O.BlockCfg]:
    d = dict(dims)
    B, T = d.pop("B"), d.pop("T")
    return B, T, O.BlockCfg(**d)


def model_config(cfg: O.BlockCfg):
    """A ModelConfig-like object for the module constructor."""
    from types import SimpleNamespace

    return SimpleNamespace(d_model=cfg.d_model, n_heads=cfg.n_heads, local_window=cfg.local_window,
                           local_block_size=cfg.local_block_size, latent_tokens=cfg.latent_tokens,
                           latent_d_model=cfg.latent_d_model, latent_heads=cfg.latent_heads,
                           latent_query_block_size=cfg.latent_query_block_size, dropout=0.0,
                           n_layers=1, use_triton_kernel=True)


def oracle_block(params: dict, x: torch.Tensor, g: torch.Tensor, cfg, gate_bias=0.0,
                 dtype=torch.float64):
    """Reference forward + backward on the CPU in `dtype`."""
    p = {k: v.detach().to(dtype).clone().requires_grad_(True) for k, v in params.items()}
    xx = x.detach().to(dtype).clone().requires_grad_(True)
    y = O.block_forward(p, xx, cfg, gate_bias)
    y.backward(g.to(dtype))
    return y.detach(), xx.grad, {k: v.grad for k, v in p.items()}


def b200_block(params: dict, x: torch.Tensor, g: torch.Tensor, cfg, gate_bias=0.0,
               dtype=torch.float32, device="cuda"):
    """The same block through LocalLatentAttentionB200 on the GPU."""
    import llattn_b200

    m = llattn_b200.LocalLatentAttentionB200(model_config(cfg))
    m.load_state_dict({k: v.detach().clone() for k, v in params.items()})
    m = m.to(device=device, dtype=dtype)
    m.gate_bias = gate_bias
    xx = x.detach().to(device=device, dtype=dtype).requires_grad_(True)
    y = m(xx)
    y.backward(g.to(device=device, dtype=dtype))
    grads = {k: p.grad for k, p in m.named_parameters()}
    return y.detach(), xx.grad, grads


def compare(got, ref, tol: float, label: str = "") -> dict:
    y, dx, grads = got
    ry, rdx, rgrads = ref
    errs = {"y": rel_err(y, ry), "dx": rel_err(dx, rdx),
            "y/frob": frob_err(y, ry), "dx/frob": frob_err(dx, rdx)}
    for k in rgrads:
        errs[k] = rel_err(grads[k], rgrads[k])
        errs[k + "/frob"] = frob_err(grads[k], rgrads[k])
    bad = {k: v for k, v in errs.items() if not (v <= tol)}
    assert not bad, f"{label}: relative errors above {tol}: {bad}"
    return errs


def bf16_round_params(params: dict) -> dict:
    return {k: v.to(torch.bfloat16).to(torch.float32) for k, v in params.items()}
