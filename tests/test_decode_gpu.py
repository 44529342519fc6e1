"""Incremental decode (``llattn_decode``) against the full forward.

Row t of a decode run must equal the last row of the module's forward over
the (t+1)-token prefix: the computation the reference's generation loop
(generate.py:188-202) repeats per token, with every size (latent chunking,
local block span) derived from the prefix length. Also checked against the
CPU oracle on the same prefix, and greedy generation with the caches must
pick the tokens the full-recompute loop picks.
"""

from __future__ import annotations

import pytest
import torch

import llattn_oracle as O
from parity import TOL, make_cfg, model_config, rel_err

pytestmark = pytest.mark.gpu

CASES = {
    # token-wise latent queries; T crosses several chunk sizes (cs = ceil(T/8))
    "tokenwise_hd64": dict(B=2, T=40, d_model=256, n_heads=4, local_window=16, local_block_size=32,
                           latent_tokens=8, latent_d_model=32, latent_heads=2, latent_query_block_size=0),
    # block-pooled latent queries (the block of t is partial while it fills)
    "qblocks_hd64": dict(B=1, T=37, d_model=256, n_heads=4, local_window=12, local_block_size=16,
                         latent_tokens=6, latent_d_model=32, latent_heads=2, latent_query_block_size=8),
    # hd 128, window larger than the block span
    "tokenwise_hd128": dict(B=1, T=33, d_model=256, n_heads=2, local_window=20, local_block_size=8,
                            latent_tokens=5, latent_d_model=64, latent_heads=2, latent_query_block_size=0),
}


def _module(cfg, dtype):
    import llattn_b200

    m = llattn_b200.LocalLatentAttentionB200(model_config(cfg))
    m.load_state_dict(O.init_params(cfg, 0))
    return m.to(device="cuda", dtype=dtype).eval()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("case", sorted(CASES))
def test_decode_rows_match_prefix_forward(case, dtype):
    B, T, cfg = make_cfg(CASES[case])
    m = _module(cfg, dtype)
    gen = torch.Generator().manual_seed(1)
    x = torch.randn(B, T, cfg.d_model, generator=gen).to(device="cuda", dtype=dtype)
    prompt = 3
    cache = m.new_decode_cache(T)
    y0 = m.prefill(x[:, :prompt], cache)
    with torch.no_grad():
        assert rel_err(y0, m(x[:, :prompt])) == 0.0
        ys = m.decode(x[:, prompt:], cache)
        assert cache.length == T
        for t in range(prompt, T):
            full = m(x[:, :t + 1])[:, -1]
            err = rel_err(ys[:, t - prompt], full)
            assert err < TOL[dtype], f"{case} {dtype} row {t}: {err:.3e}"
            if dtype == torch.float32 and t % 7 == 0:  # and the oracle on the same prefix
                p = {k: v.detach().double().cpu() for k, v in m.state_dict().items()}
                ref = O.block_forward(p, x[:, :t + 1].double().cpu(), cfg)[:, -1]
                err = rel_err(ys[:, t - prompt], ref)
                assert err < TOL[dtype], f"{case} oracle row {t}: {err:.3e}"


def test_decode_cache_overflow_raises():
    B, T, cfg = make_cfg(CASES["tokenwise_hd64"])
    m = _module(cfg, torch.float32)
    cache = m.new_decode_cache(4)
    x = torch.randn(1, 5, cfg.d_model, device="cuda")
    m.prefill(x[:, :3], cache)
    m.decode(x[:, 3:4], cache)
    with pytest.raises(RuntimeError, match="cache full"):
        m.decode(x[:, 4:5], cache)


def test_lm_greedy_generation_matches_full_recompute():
    from llattn_b200.lm import LocalLatentLM, ModelConfig

    torch.manual_seed(0)
    cfg = ModelConfig(vocab_size=97, max_seq_len=48, d_model=128, n_heads=2, n_layers=2, d_ff=256,
                      local_window=8, local_block_size=16, latent_tokens=6, latent_d_model=32, latent_heads=2)
    model = LocalLatentLM(cfg).cuda().eval()
    prompt = torch.randint(0, cfg.vocab_size, (2, 5), device="cuda")
    fast = model.generate(prompt, 30, incremental=True)
    slow = model.generate(prompt, 30, incremental=False)
    assert torch.equal(fast, slow)
    # past max_seq_len the context slides and both paths recompute
    longer = model.generate(prompt, 50, incremental=True)
    assert torch.equal(longer[:, :35], fast)
