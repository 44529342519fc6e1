"""Generate the golden vectors that pin the CPU oracle to the reference.

Runs the reference's own PyTorch ``LocalLatentAttention`` (models.py:61-462,
imported read-only from $LLATTN_REF_PATH, default a `reference` checkout
beside this repository) on seeded inputs and stores inputs, weights, the
output, dx and every parameter gradient; and the reference's own
``LocalLatentLM`` (models.py:505-576) at the 0.55b preset's attention
ratios (train.py:71-80: head_dim 88, latent_d_model 512 over 8 heads),
shrunk to 2 layers, storing its logits, loss and every gradient. The gate-bias cases add the bias with a forward hook on
``gate_local`` — the reference code itself is not modified.

Usage:  python tests/golden/make_golden.py   (needs the reference tree; the
committed .pt files are what the tests read, so the GPU box never needs it).
"""

import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("LLATTN_REF_PATH", os.path.join(ROOT, os.pardir, "reference"))

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
    # more than one 64-chunk key tile (100 chunks of 3 tokens; 150 chunks of 2
    # with query blocks of 8 and a 48-wide latent head)
    "many_chunks": (dict(B=1, T=300, d_model=32, n_heads=2, local_window=16, local_block_size=32,
                         latent_tokens=100, latent_d_model=64, latent_heads=2), 0.0),
    "many_chunks_qblocks": (dict(B=2, T=300, d_model=32, n_heads=2, local_window=16, local_block_size=32,
                                 latent_tokens=150, latent_d_model=48, latent_heads=1,
                                 latent_query_block_size=8), 0.0),
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


# LM golden: the 0.55b preset's block ratios (d_model 1408 / 16 heads = 88
# per head; latent 512 = 8 x 64) at d_model 176 with 2 heads, 2 layers
LM = dict(vocab_size=128, max_seq_len=128, d_model=176, n_heads=2, n_layers=2, d_ff=128, local_window=32,
          local_block_size=64, latent_tokens=16, latent_d_model=512, latent_heads=8)
LM_B = 2


def run_reference_lm():
    """Reference LocalLatentLM in float64 on weights rounded to bf16 values
    (the test builds the same weights from the seed with the package's own
    LocalLatentLM, whose seeded init equals the reference's, and rounds them
    the same way), tokens from seed 1, next-token cross-entropy. Gradients
    are stored in bf16 to keep the fixture small (2^-9 relative)."""
    sys.path.insert(0, REF)
    import torch.nn.functional as F
    from models import LocalLatentLM, ModelConfig  # noqa: E402

    torch.manual_seed(0)
    m = LocalLatentLM(ModelConfig(**LM))
    with torch.no_grad():
        for p in m.parameters():
            p.copy_(p.to(torch.bfloat16).float())
    m = m.double()
    gen = torch.Generator().manual_seed(1)
    ids = torch.randint(0, LM["vocab_size"], (LM_B, LM["max_seq_len"] + 1), generator=gen)
    logits = m(ids[:, :-1])
    loss = F.cross_entropy(logits.reshape(-1, LM["vocab_size"]), ids[:, 1:].reshape(-1))
    loss.backward()
    return {
        "cfg": dict(LM), "B": LM_B, "ids": ids,
        "params_checksum": {k: (v.double().sum().item(), v.double().abs().sum().item())
                            for k, v in m.state_dict().items()},
        "logits": logits.detach().float(), "loss": loss.item(),
        "grads": {k: p.grad.detach().to(torch.bfloat16) for k, p in m.named_parameters()},
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
    torch.save(run_reference_lm(), os.path.join(HERE, "lm_055b_small.pt"))
    print("wrote", sorted(small), "cfg1 and the LM golden")


if __name__ == "__main__":
    main()
