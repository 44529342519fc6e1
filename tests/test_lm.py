"""The LM harness (LocalLatentLM with the drop-in block): module tree and
state_dict names of the reference (models.py:505-576) on the CPU, and a few
training steps on the GPU."""

import pytest
import torch

from llattn_b200.lm import LocalLatentLM, ModelConfig, build_optimizer, train_step


def small_cfg(**kw):
    base = dict(vocab_size=512, max_seq_len=256, d_model=256, n_heads=2, n_layers=2, d_ff=512, local_window=64,
                latent_tokens=16, latent_d_model=64, latent_heads=2)
    base.update(kw)
    return ModelConfig(**base)


def test_state_dict_names_match_reference_layout():
    m = LocalLatentLM(small_cfg())
    keys = set(m.state_dict())
    expect = {"embedding.weight", "position.weight", "norm.weight", "lm_head.weight"}
    for i in range(2):
        p = f"blocks.{i}."
        expect |= {p + "norm1.weight", p + "norm2.weight", p + "ff.w1.weight", p + "ff.w1.bias", p + "ff.w2.weight",
                   p + "ff.w2.bias", p + "attn.gate_local.weight", p + "attn.gate_remote.weight"}
        for lin in ("qkv_proj", "rq_proj", "rkv_proj", "r_out", "out"):
            expect |= {p + f"attn.{lin}.weight", p + f"attn.{lin}.bias"}
    assert keys == expect
    assert m.lm_head.weight is m.embedding.weight  # tied (models.py:517)


def test_init_scales_output_projections():
    m = LocalLatentLM(small_cfg(n_layers=4))
    std_out = m.blocks[0].attn.out.weight.std().item()
    std_qkv = m.blocks[0].attn.qkv_proj.weight.std().item()
    assert abs(std_qkv - 0.02) < 0.003
    assert abs(std_out - 0.02 / (8 ** 0.5)) < 0.002
    assert m.blocks[0].attn.qkv_proj.bias.abs().max().item() == 0.0


def test_optimizer_groups():
    m = LocalLatentLM(small_cfg())
    opt = build_optimizer(m)
    decay, no_decay = opt.param_groups
    assert decay["weight_decay"] == 0.1 and no_decay["weight_decay"] == 0.0
    assert all(p.dim() >= 2 for p in decay["params"]) and all(p.dim() < 2 for p in no_decay["params"])


@pytest.mark.gpu
def test_lm_trains_on_gpu():
    torch.manual_seed(0)
    cfg = small_cfg()
    m = LocalLatentLM(cfg).cuda()
    opt = build_optimizer(m, lr=1e-3)
    gen = torch.Generator().manual_seed(0)
    # a learnable sequence: token t+1 = (token t + 1) mod V
    start = torch.randint(0, cfg.vocab_size, (4, 1), generator=gen)
    seq = (start + torch.arange(129)) % cfg.vocab_size
    ids, tgt = seq[:, :-1].cuda(), seq[:, 1:].cuda()
    losses = [train_step(m, opt, ids, tgt).item() for _ in range(30)]
    assert all(torch.isfinite(torch.tensor(losses)))
    assert losses[-1] < 0.5 * losses[0], losses
