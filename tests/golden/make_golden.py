"""Generate the golden vectors that pin the CPU oracle to the reference.

Runs the reference's own PyTorch ``LocalLatentAttention`` (models.py:61-462,
imported read-only from $LLATTN_REF_PATH, default the reference checkout) on
seeded inputs and stores inputs, weights, the output, dx and every parameter
gradient. The gate-bias cases add the bias with a forward hook on
``gate_local`` — the reference code itself is not modified.

Usage:  python tests/golden/make_golden.py   (needs the reference tree; the
committed .pt files are what the tests read, so the GPU box never needs it).
"""

import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("LLATTN_REF_PATH", "/root/reference")

# name: (dims, gate_bias, dtype)
SMALL = {
    "blocks_quirk": (dict(B=2, T=64, d_model=32, n_heads=2, local_window=8, local_block_size=16,
                          latent_tokens=8, latent_d_model=8, latent_heads=2), 0.0),
    "ragged_chunks": (dict(B=2, T=37, d_model=24, n_heads=3, local_window=6, local_block_size=10,
                           latent_tokens=5, latent_d_model=8, latent_heads=2), 0.0),
    "query_blocks": (dict(B=2, T=50, d_model=32, n_heads=4, local_window=7, local_block_size=12,
                          latent_tokens=7, latent_d_model=12, latent_heads=3,
                          latent_query_block_size=8), 0.0),
    "gate_plus8": (dict(B=2, T=64, d_model=32, n_heads=2, local_window=8, local_block_size=16,
                        latent_tokens=8, latent_d_model=8, latent_heads=2), 8.0),
    "gate_minus8": (dict(B=2, T=37, d_model=24, n_heads=3, local_window=6, local_block_size=10,
                         latent_tokens=5, latent_d_model=8, latent_heads=2), -8.0),
    "single_token": (dict(B=1, T=1, d_model=16, n_heads=2, local_window=4, local_block_size=256,
                          latent_tokens=4, latent_d_model=4, latent_heads=2), 0.0),
    "window_exceeds_T": (dict(B=1, T=20, d_model=16, n_heads=2, local_window=64,
                              local_block_size=256, latent_tokens=4, latent_d_model=8,
                              latent_heads=2), 0.0),
    "qblock_exceeds_T": (dict(B=2, T=5, d_model=16, n_heads=2, local_window=3, local_block_size=4,
                              latent_tokens=3, latent_d_model=8, latent_heads=2,
                              latent_query_block_size=8), 0.0),
    "more_latents_than_T": (dict(B=1, T=20, d_model=16, n_heads=2, local_window=5,
                                 local_block_size=8, latent_tokens=64, latent_d_model=8,
                                 latent_heads=2), 0.0),
}

CFG1 = dict(B=2, T=512, d_model=256, n_heads=4, local_window=128, local_block_size=256,
            latent_tokens=16, latent_d_model=32, latent_heads=2)


def run_reference(dims: dict, gate_bias: float, dtype: torch.dtype, seed: int = 0):
    sys.path.insert(0, REF)
    from models import LocalLatentAttention, ModelConfig  # noqa: E402

    dims = dict(dims)
    B, T = dims.pop("B"), dims.pop("T")
    torch.manual_seed(seed)
    m = LocalLatentAttention(ModelConfig(**dims)).to(dtype)
    if gate_bias:
        m.gate_local.register_forward_hook(lambda mod, inp, out: out + gate_bias)
    x = torch.randn(B, T, dims["d_model"], dtype=dtype, requires_grad=True)
    g = torch.randn(B, T, dims["d_model"], dtype=dtype)
    y = m(x)
    y.backward(g)
    return {
        "dims": dict(dims, B=B, T=T),
        "gate_bias": gate_bias,
        "x": x.detach(),
        "g": g,
        "params": {k: v.detach().clone() for k, v in m.state_dict().items()},
        "y": y.detach(),
        "dx": x.grad.detach(),
        "grads": {k: p.grad.detach().clone() for k, p in m.named_parameters()},
    }


def main() -> None:
    small = {name: run_reference(dims, bias, torch.float64) for name, (dims, bias) in SMALL.items()}
    torch.save(small, os.path.join(HERE, "small_f64.pt"))
    cfg1 = run_reference(CFG1, 0.0, torch.float32)
    # inputs and weights are regenerated from seed 0 by the tests; only their
    # checksums are kept, next to the reference outputs
    for key in ("x", "g"):
        t = cfg1.pop(key)
        cfg1[key + "_checksum"] = (t.double().sum().item(), t.double().abs().sum().item())
    params = cfg1.pop("params")
    cfg1["params_checksum"] = {k: (v.double().sum().item(), v.double().abs().sum().item())
                               for k, v in params.items()}
    torch.save(cfg1, os.path.join(HERE, "cfg1_f32.pt"))
    print("wrote", sorted(small), "and cfg1")


if __name__ == "__main__":
    main()
