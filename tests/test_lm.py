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


def _reference_models():
    """The reference's models module, imported read-only from
    $LLATTN_REF_PATH (default: a `reference` checkout beside this repository);
    the tests that need it skip where it is absent (e.g. the GPU box)."""
    import importlib
    import os
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    path = os.environ.get("LLATTN_REF_PATH", os.path.join(root, os.pardir, "reference"))
    if not os.path.exists(os.path.join(path, "models.py")):
        pytest.skip("reference tree not present")
    if path not in sys.path:
        sys.path.insert(0, path)
    return importlib.import_module("models")


SMALL_LM = dict(vocab_size=300, max_seq_len=128, d_model=176, n_heads=2, n_layers=2, d_ff=256, local_window=32,
                latent_tokens=8, latent_d_model=512, latent_heads=8)


def test_seeded_init_equals_reference_lm():
    """Same seed, same weights: the module tree is created and initialised in
    the reference LocalLatentLM's order (models.py:505-546)."""
    models = _reference_models()
    torch.manual_seed(0)
    ref = models.LocalLatentLM(models.ModelConfig(**SMALL_LM))
    torch.manual_seed(0)
    ours = LocalLatentLM(ModelConfig(**SMALL_LM))
    a, b = ref.state_dict(), ours.state_dict()
    assert set(a) == set(b)
    for k in a:
        assert torch.equal(a[k], b[k]), k


def test_reference_lm_builds_the_b200_block():
    """use_in_reference points the reference's own _build_attention at the
    B200 block: its LocalLatentLM then has the same parameters as ours."""
    import llattn_b200
    from llattn_b200.lm import use_in_reference

    models = _reference_models()
    saved = models._build_attention
    try:
        use_in_reference(models)
        cfg = models.ModelConfig(**SMALL_LM, use_triton_kernel=True)
        ref = models.LocalLatentLM(cfg)
        assert all(isinstance(blk.attn, llattn_b200.LocalLatentAttentionB200) for blk in ref.blocks)
        ours = LocalLatentLM(ModelConfig(**SMALL_LM))
        ours.load_state_dict(ref.state_dict(), strict=True)
        cfg_plain = models.ModelConfig(**SMALL_LM, use_triton_kernel=False)
        assert not isinstance(models.LocalLatentLM(cfg_plain).blocks[0].attn, llattn_b200.LocalLatentAttentionB200)
    finally:
        models._build_attention = saved


@pytest.mark.gpu
def test_lm_matches_reference_golden_bf16():
    """The package's LocalLatentLM on the GPU (bf16 autocast, the B200 block
    in both layers, on its tensor-core paths: head_dim 88 and latent width
    512) against the reference LocalLatentLM's float64 logits, loss and
    every gradient (tests/golden/lm_055b_small.pt, weights rebuilt from the
    same seed). Tolerance 2e-2 on max|a-b|/max|b| and the Frobenius ratio."""
    import os

    import torch.nn.functional as F
    from parity import TOL, frob_err, rel_err

    gold = torch.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "lm_055b_small.pt"))
    cfg = ModelConfig(**gold["cfg"])
    torch.manual_seed(0)
    m = LocalLatentLM(cfg)
    with torch.no_grad():
        for p in m.parameters():
            p.copy_(p.to(torch.bfloat16).float())
    for k, v in m.state_dict().items():  # same weights as the reference run
        s, a = gold["params_checksum"][k]
        assert abs(v.double().sum().item() - s) <= 1e-6 * max(1.0, a), k
    m = m.cuda()
    ids = gold["ids"].cuda()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        logits = m(ids[:, :-1])
        loss = F.cross_entropy(logits.float().reshape(-1, cfg.vocab_size), ids[:, 1:].reshape(-1))
    loss.backward()
    tol = TOL[torch.bfloat16]
    errs = {"logits": rel_err(logits.float(), gold["logits"]), "logits/frob": frob_err(logits.float(), gold["logits"]),
            "loss": abs(loss.item() - gold["loss"]) / abs(gold["loss"])}
    grads = dict(m.named_parameters())
    for k, g in gold["grads"].items():
        errs[k] = rel_err(grads[k].grad, g.float())
        errs[k + "/frob"] = frob_err(grads[k].grad, g.float())
    bad = {k: v for k, v in errs.items() if not v <= tol}
    print({k: round(v, 5) for k, v in errs.items()})
    assert not bad, bad


def _installed_reference_models():
    """The reference's models.py as installed in baseline/_ref (placed there by
    __graft_entry__.build(), travels with the working tree); skip where absent."""
    import importlib.util
    import os

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    path = os.path.join(root, "baseline", "_ref", "models.py")
    if not os.path.exists(path):
        pytest.skip("reference not installed in baseline/_ref")
    spec = importlib.util.spec_from_file_location("llattn_installed_reference_models", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.gpu
def test_reference_lm_runs_the_b200_block_at_cfg4_width():
    """The reference's own LocalLatentLM (models.py:505-576), built through its
    own _build_attention switched to the B200 block (use_in_reference), at the
    cfg4 width (d1536 H12 W256 Nl64 Ld64, d_ff 4096, vocab 32000; 2 layers,
    B2 x T512), trains on the GPU under bf16 autocast and matches the same
    model with the reference's PyTorch attention in fp32: logits, loss and
    every gradient within 2e-2 (max-norm and Frobenius)."""
    import torch.nn.functional as F
    from parity import TOL, frob_err, rel_err

    from llattn_b200.lm import use_in_reference

    models = _installed_reference_models()
    shape = dict(vocab_size=32000, max_seq_len=512, d_model=1536, n_heads=12, n_layers=2, d_ff=4096,
                 local_window=256, latent_tokens=64, latent_d_model=64, latent_heads=2)
    torch.manual_seed(0)
    ref = models.LocalLatentLM(models.ModelConfig(**shape, use_triton_kernel=False))
    with torch.no_grad():
        for p in ref.parameters():
            p.copy_(p.to(torch.bfloat16).float())
    saved = models._build_attention
    try:
        use_in_reference(models)
        ours = models.LocalLatentLM(models.ModelConfig(**shape, use_triton_kernel=True))
    finally:
        models._build_attention = saved
    ours.load_state_dict(ref.state_dict())
    gen = torch.Generator().manual_seed(3)
    ids = torch.randint(0, shape["vocab_size"], (2, 513), generator=gen).cuda()
    V = shape["vocab_size"]

    ref = ref.cuda()
    logits_r = ref(ids[:, :-1])
    loss_r = F.cross_entropy(logits_r.reshape(-1, V), ids[:, 1:].reshape(-1))
    loss_r.backward()
    ours = ours.cuda()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        logits = ours(ids[:, :-1])
        loss = F.cross_entropy(logits.float().reshape(-1, V), ids[:, 1:].reshape(-1))
    loss.backward()
    tol = TOL[torch.bfloat16]
    errs = {"logits": rel_err(logits.float(), logits_r), "logits/frob": frob_err(logits.float(), logits_r),
            "loss": abs(loss.item() - loss_r.item()) / abs(loss_r.item())}
    gr = dict(ref.named_parameters())
    for k, p in ours.named_parameters():
        errs[k] = rel_err(p.grad, gr[k].grad)
        errs[k + "/frob"] = frob_err(p.grad, gr[k].grad)
    bad = {k: v for k, v in errs.items() if not v <= tol}
    print(max(errs.values()))
    assert not bad, bad


@pytest.mark.gpu
def test_compiled_layers_match_eager_training_step():
    """Each decoder layer under torch.compile (the bench's LM setting: the
    B200 attention as opaque custom ops inside inductor's graph) gives the
    eager layer's loss and gradients within 2e-2."""
    import copy

    from parity import TOL, rel_err

    torch.manual_seed(0)
    eager = LocalLatentLM(small_cfg()).cuda()
    comp = copy.deepcopy(eager)
    for i, layer in enumerate(comp.blocks):
        comp.blocks[i] = torch.compile(layer, fullgraph=True)
    gen = torch.Generator().manual_seed(0)
    seq = torch.randint(0, 512, (2, 129), generator=gen).cuda()
    ids, tgt = seq[:, :-1], seq[:, 1:]
    losses, grads = [], []
    for m in (eager, comp):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits = m(ids)
            loss = torch.nn.functional.cross_entropy(logits.float().reshape(-1, 512), tgt.reshape(-1))
        loss.backward()
        losses.append(loss.item())
        grads.append({k.replace("._orig_mod", ""): p.grad for k, p in m.named_parameters()})
    assert abs(losses[0] - losses[1]) <= 1e-2 * abs(losses[0])
    for k, g in grads[0].items():
        assert rel_err(grads[1][k], g) <= TOL[torch.bfloat16], k
