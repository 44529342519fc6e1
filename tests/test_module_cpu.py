"""Host-side checks of the drop-in module and ops (CPU only)."""

from types import SimpleNamespace

import pytest
import torch

import llattn_b200
import llattn_oracle as O
from parity import model_config


def cfg():
    return O.BlockCfg(d_model=32, n_heads=2, local_window=8, local_block_size=16,
                      latent_tokens=8, latent_d_model=8, latent_heads=2)


def test_state_dict_matches_reference_names_and_shapes():
    m = llattn_b200.LocalLatentAttentionB200(model_config(cfg()))
    ref = O.init_params(cfg())
    sd = m.state_dict()
    assert sorted(sd) == sorted(ref)
    for k in ref:
        assert sd[k].shape == ref[k].shape, k


def test_loads_reference_state_dict_and_legacy_split_keys():
    c = cfg()
    m = llattn_b200.LocalLatentAttentionB200(model_config(c))
    ref = O.init_params(c, seed=3)
    m.load_state_dict(ref)
    assert torch.equal(m.qkv_proj.weight, ref["qkv_proj.weight"])
    legacy = dict(ref)
    d = c.d_model
    w, b = legacy.pop("qkv_proj.weight"), legacy.pop("qkv_proj.bias")
    for i, n in enumerate(("q_proj", "k_proj", "v_proj")):
        legacy[n + ".weight"] = w[i * d:(i + 1) * d]
        legacy[n + ".bias"] = b[i * d:(i + 1) * d]
    w, b = legacy.pop("rkv_proj.weight"), legacy.pop("rkv_proj.bias")
    L = c.latent_d_model
    legacy["rk_proj.weight"], legacy["rv_proj.weight"] = w[:L], w[L:]
    legacy["rk_proj.bias"], legacy["rv_proj.bias"] = b[:L], b[L:]
    m2 = llattn_b200.LocalLatentAttentionB200(model_config(c))
    m2.load_state_dict(legacy)
    for k, v in ref.items():
        assert torch.equal(m2.state_dict()[k], v), k


def test_ops_have_no_cpu_path():
    x = torch.randn(2, 16, 8)
    with pytest.raises(Exception):
        llattn_b200.ops.pool_chunks(x, 4)


def test_profile_api_present():
    m = llattn_b200.LocalLatentAttentionB200(model_config(cfg()))
    m.set_profile(True)
    assert m.get_profile_stats() == {}
    m.set_profile(False)
    assert m.get_profile_stats() == {}


def test_dropout_in_training_is_rejected():
    c = model_config(cfg())
    c.dropout = 0.1
    m = llattn_b200.LocalLatentAttentionB200(c).train()
    with pytest.raises(NotImplementedError):
        m(torch.randn(1, 4, 32))


def test_decode_cache_bookkeeping_and_cpu_refusal():
    """The decode path keeps its cache on the host side consistent and, like
    every op, refuses CPU tensors instead of falling back."""
    import llattn_b200
    from llattn_b200 import ops

    cache = llattn_b200.DecodeCache(capacity=8)
    assert cache.length == 0 and cache.qkv is None
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.decode_core(torch.zeros(1, 8, 3 * 64), 1, torch.zeros(1, 32), torch.zeros(1, 1, 64),
                        torch.zeros(64, 32), torch.zeros(64), torch.zeros(16), torch.zeros(16), n_heads=4,
                        latent_heads=2, window=4, local_block_size=8, latent_tokens=4)


def test_seeded_construction_equals_reference_default_init():
    """bench.py builds its block under torch.manual_seed(0); the module's
    layers are created in the reference constructor's order, so the weights
    are the reference module's default init (the oracle's init_params)."""
    cfg = O.BlockCfg(d_model=128, n_heads=4, local_window=16, latent_tokens=8, latent_d_model=32)
    torch.manual_seed(0)
    m = llattn_b200.LocalLatentAttentionB200(model_config(cfg))
    ref = O.init_params(cfg, 0)
    sd = m.state_dict()
    assert set(sd) == set(ref)
    for k, v in ref.items():
        assert torch.equal(sd[k], v), k


def test_visible_pairs_matches_oracle_count():
    from llattn_b200.ops import visible_pairs

    for T, W, lbs in [(2048, 256, 256), (512, 128, 256), (16384, 512, 256), (37, 12, 16), (1, 4, 4), (300, 64, 32)]:
        assert visible_pairs(T, W, lbs) == O.local_pairs(T, W, lbs)


def test_fake_tensor_trace_of_the_block():
    """The custom ops' fake implementations (register_fake) let the whole
    block trace without a GPU: forward and backward of the drop-in module on
    FakeTensor CUDA inputs give the real op's shapes and dtypes. This is what
    torch.compile relies on (the reference's Triton path forbids compile,
    train.py:694-695)."""
    from torch._subclasses.fake_tensor import FakeTensorMode

    import llattn_b200

    cfg = SimpleNamespace(d_model=176, n_heads=2, local_window=32, local_block_size=64, latent_tokens=16,
                          latent_d_model=512, latent_heads=8, latent_query_block_size=0, dropout=0.0, n_layers=1,
                          use_triton_kernel=True)
    m = llattn_b200.LocalLatentAttentionB200(cfg)
    with FakeTensorMode() as fm:
        params = {k: fm.from_tensor(v).to(device="cuda", dtype=torch.bfloat16).requires_grad_(True)
                  for k, v in m.named_parameters()}
        x = torch.empty(2, 300, 176, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        y = torch.func.functional_call(m, params, (x,))
        assert y.shape == x.shape and y.dtype == torch.bfloat16 and y.device.type == "cuda"
        # the backward op's fake (autograd's engine itself needs a device to run)
        B, T, d, Ld, hd = 2, 300, 176, 512, 88
        bf = dict(device="cuda", dtype=torch.bfloat16)
        f32 = dict(device="cuda", dtype=torch.float32)
        qkv = torch.empty(B, T, 3 * d, **bf)
        outs = torch.ops.llattn_b200.attn_fwd(qkv, torch.empty(B, T, Ld, **bf), torch.empty(B, 16, 2 * Ld, **bf),
                                              torch.empty(d, Ld, **bf), torch.empty(d, **f32),
                                              torch.empty(hd, **f32), torch.empty(hd, **f32), 2, 8, 32, 64, 16, 0, 0.0)
        grads = torch.ops.llattn_b200.attn_bwd(outs[0], qkv, torch.empty(B, T, Ld, **bf),
                                               torch.empty(B, 16, 2 * Ld, **bf), torch.empty(d, Ld, **bf),
                                               torch.empty(d, **f32), torch.empty(hd, **f32), torch.empty(hd, **f32),
                                               *outs[1:], 2, 8, 32, 64, 16, 0, 0.0)
        want = [(B, T, 3 * d), (B, T, Ld), (B, 16, 2 * Ld), (d, Ld), (d,), (hd,), (hd,), (3 * d,)]
        assert [tuple(g.shape) for g in grads] == want
