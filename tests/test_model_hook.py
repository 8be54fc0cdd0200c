"""The DFlash drafter and its compute_loss(loss_fn=...) hook
(reference: models/dflash/tests/test_model.py). CPU checks run everywhere;
the fused-loss hook checks need the GPU."""
import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from models.dflash import DFlashSpeculator

B, S_CTX, D_TARGET, D_MODEL, V, BLOCK, LAYERS = 2, 16, 64, 32, 256, 4, 2


def _model(seed=42):
    torch.manual_seed(seed)
    head = nn.Linear(D_TARGET, V, bias=False)
    for p in head.parameters():
        p.requires_grad = False
    return DFlashSpeculator(d_target=D_TARGET, d_model=D_MODEL, target_vocab_size=V,
                            block_size=BLOCK, num_layers=LAYERS, target_lm_head=head), head


def test_shape_grads_and_frozen_head():
    model, head = _model()
    feats = torch.randn(B, S_CTX, D_TARGET)
    logits = model(feats)
    assert logits.shape == (B, BLOCK, V) and bool(torch.isfinite(logits).all())
    gt = torch.randint(0, V, (B, BLOCK))
    loss = model.compute_loss(feats, gt)
    assert loss.dim() == 0
    loss.backward()
    assert model.proj_in.weight.grad is not None
    assert model.slot_queries.grad is not None
    assert model.proj_out.weight.grad is not None
    assert head.weight.grad is None


def test_draft_is_argmax():
    model, _ = _model()
    model.eval()
    feats = torch.randn(B, S_CTX, D_TARGET)
    tok, lg = model.draft(feats)
    assert tok.shape == (B, BLOCK) and tok.dtype == torch.int64 and lg.shape == (B, BLOCK, V)
    assert bool((tok == model(feats).argmax(-1)).all())


def test_mask_rules():
    model, _ = _model()
    m = model._build_dflash_mask(S_ctx=4, S_block=2, device=torch.device("cpu"))
    assert bool((m[0, 0, :4, 4:] == float("-inf")).all())   # context cannot see block
    assert bool((m[0, 0, 4:, :4] == 0.0).all())             # block sees context
    assert bool((m[0, 0, 4:, 4:] == 0.0).all())             # block is bidirectional
    iu = torch.triu_indices(4, 4, offset=1)
    assert bool((m[0, 0, :4, :4][iu[0], iu[1]] == float("-inf")).all())  # causal context
    il = torch.tril_indices(4, 4)
    assert bool((m[0, 0, :4, :4][il[0], il[1]] == 0.0).all())


def test_structured_mask_equals_explicit_mask():
    """forward() applies the _build_dflash_mask rule by structure (a causal
    attention over the context, an unmasked one for the block queries); the
    result and every parameter gradient equal the explicit-mask form."""
    model, _ = _model(7)
    feats = torch.randn(B, S_CTX, D_TARGET)

    def explicit(m, x):
        b, s_ctx, _ = x.shape
        h = torch.cat([m.proj_in(x), m.slot_queries.expand(b, -1, -1)], dim=1)
        mask = m._build_dflash_mask(s_ctx, m.block_size, x.device)
        for layer in m.layers:
            h = layer(h, attn_mask=mask)
        return m.lm_head(m.final_norm(m.proj_out(m.norm_out(h)[:, s_ctx:, :])))

    a = model(feats)
    b = explicit(model, feats)
    assert (a - b).abs().max().item() < 1e-5
    ga = torch.autograd.grad(a.square().sum(), [p for p in model.parameters() if p.requires_grad])
    gb = torch.autograd.grad(b.square().sum(), [p for p in model.parameters() if p.requires_grad])
    for x, y in zip(ga, gb):
        assert (x - y).abs().max().item() <= 1e-5 * (1 + y.abs().max().item())


def test_batch_invariance():
    model, _ = _model()
    feats = torch.randn(B, S_CTX, D_TARGET)
    with torch.no_grad():
        single = model(feats[0:1])
        batched = model(feats)
    assert (single[0] - batched[0]).abs().max().item() < 1e-4


def test_state_dict_names():
    model, _ = _model()
    names = set(model.state_dict())
    for n in ("proj_in.weight", "slot_queries", "layers.0.norm1.weight", "layers.0.attn.q_proj.weight",
              "layers.0.attn.out_proj.weight", "layers.0.mlp.0.weight", "layers.0.mlp.2.weight",
              "norm_out.weight", "proj_out.weight", "final_norm.weight", "lm_head.weight"):
        assert n in names, n


@pytest.mark.gpu
def test_hook_swaps_objectives(cuda):
    from losses.dpace import dpace_loss
    from models.dflash import dflash_loss, dflash_objective

    model, _ = _model()
    gpu = model.cuda()
    gf = torch.randn(B, S_CTX, D_TARGET, device="cuda")
    gt = torch.randint(0, V, (B, BLOCK), device="cuda")
    target_logits = torch.randn(B, BLOCK, V, device="cuda")
    with torch.no_grad():
        ce_ref = F.cross_entropy(gpu(gf).reshape(-1, V), gt.reshape(-1))
        fused = dflash_loss(gpu(gf), target_logits, None, 4.0, False, "kl")
    assert bool(torch.isfinite(fused)) and abs(float(fused) - float(ce_ref)) > 1e-6

    out = gpu.compute_loss(gf, gt, loss_fn=dflash_objective(target_logits))
    out.backward()
    assert gpu.proj_in.weight.grad is not None and bool(torch.isfinite(gpu.proj_in.weight.grad).all())
    gpu.zero_grad(set_to_none=True)

    dp = gpu.compute_loss(gf, gt, loss_fn=lambda lg, tg: dpace_loss(lg, tg, 0.5))
    assert bool(torch.isfinite(dp))
    dp.backward()
    assert gpu.slot_queries.grad is not None and bool(torch.isfinite(gpu.slot_queries.grad).all())
    gpu.zero_grad(set_to_none=True)

    with torch.no_grad():
        l_ce = gpu.compute_loss(gf, gt)
        l_dp = gpu.compute_loss(gf, gt, loss_fn=lambda lg, tg: dpace_loss(lg, tg, 0.5))
    assert abs(float(l_ce) - float(l_dp)) > 1e-6


@pytest.mark.gpu
def test_hook_gradients_match_oracle(cuda):
    """Parameter gradients through the drafter with the fused D-PACE loss equal
    those with the CPU-oracle loss evaluated on the GPU logits."""
    from losses.dpace import dpace_loss
    from oracle.dpace import dpace_loss_torch

    model, _ = _model()
    gpu = model.cuda()
    gf = torch.randn(B, S_CTX, D_TARGET, device="cuda")
    gt = torch.randint(0, V, (B, BLOCK), device="cuda")
    gpu.compute_loss(gf, gt, loss_fn=lambda lg, tg: dpace_loss(lg, tg, 0.5)).backward()
    g1 = gpu.proj_in.weight.grad.clone()
    gpu.zero_grad(set_to_none=True)
    gpu.compute_loss(gf, gt, loss_fn=lambda lg, tg: dpace_loss_torch(lg, tg, 0.5)).backward()
    g2 = gpu.proj_in.weight.grad.clone()
    assert (g1 - g2).abs().max().item() <= 1e-6 + 1e-4 * g2.abs().max().item()
