"""The CPU oracle against golden vectors produced by the reference module
(tests/golden/make_golden.py). No GPU needed."""

import os

import pytest
import torch

import llattn_oracle as O
from parity import make_cfg, oracle_block, rel_err

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
SMALL = torch.load(os.path.join(GOLDEN, "small_f64.pt"))


@pytest.mark.parametrize("name", sorted(SMALL))
def test_oracle_matches_reference_small(name):
    case = SMALL[name]
    B, T, cfg = make_cfg(case["dims"])
    y, dx, grads = oracle_block(case["params"], case["x"], case["g"], cfg, case["gate_bias"])
    assert rel_err(y, case["y"]) < 1e-12
    assert rel_err(dx, case["dx"]) < 1e-12
    for k, ref in case["grads"].items():
        assert rel_err(grads[k], ref) < 1e-11, k


@pytest.mark.parametrize("name", sorted(SMALL))
def test_init_params_reproduce_reference_weights(name):
    case = SMALL[name]
    _, _, cfg = make_cfg(case["dims"])
    p = O.init_params(cfg, 0, torch.float64)
    for k, v in case["params"].items():
        assert torch.equal(p[k], v), k


def cfg1_inputs():
    case = torch.load(os.path.join(GOLDEN, "cfg1_f32.pt"))
    B, T, cfg = make_cfg(case["dims"])
    params = O.init_params(cfg, 0, torch.float32)
    x = torch.randn(B, T, cfg.d_model)
    g = torch.randn(B, T, cfg.d_model)
    return case, cfg, params, x, g


def test_cfg1_inputs_regenerate():
    case, cfg, params, x, g = cfg1_inputs()
    for key, t in (("x", x), ("g", g)):
        s, a = case[key + "_checksum"]
        assert abs(t.double().sum().item() - s) < 1e-6 * max(1.0, abs(a))
        assert abs(t.double().abs().sum().item() - a) < 1e-6 * a
    for k, (s, a) in case["params_checksum"].items():
        assert abs(params[k].double().sum().item() - s) <= 1e-9 * max(1.0, a), k


def test_oracle_matches_reference_cfg1_fp32():
    case, cfg, params, x, g = cfg1_inputs()
    y, dx, grads = oracle_block(params, x, g, cfg, 0.0, torch.float32)
    assert rel_err(y, case["y"]) < 1e-5
    assert rel_err(dx, case["dx"]) < 1e-5
    for k, ref in case["grads"].items():
        assert rel_err(grads[k], ref) < 1e-5, k


def test_local_pairs_count():
    # cfg1 and cfg2 pair counts of the local mask, per (batch, head)
    assert O.local_pairs(512, 128, 256) * 2 * 4 == 458232
    assert O.local_pairs(2048, 256, 256) * 16 * 12 == 94345920


def test_mask_matches_blockwise_definition():
    T, W, LBS = 50, 7, 12
    m = O.local_allowed(T, W, LBS)
    assert m.sum().item() == O.local_pairs(T, W, LBS)
    # first row of each later block sees one key fewer (block-boundary quirk)
    assert m[12].sum().item() == W - 1 and m[13].sum().item() == W
