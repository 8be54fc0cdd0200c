"""specdec.graphs.GraphedStep: the drafter's whole training step (forward,
D-PACE loss, backward, clip, AdamW) captured as one CUDA graph gives the same
losses and parameters as the same step run eagerly, on new inputs copied into
the graph's static buffers; a target id out of range surfaces at check()."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _model(seed):
    from models.dflash.model import DFlashSpeculator

    torch.manual_seed(seed)
    return DFlashSpeculator(d_target=512, d_model=256, target_vocab_size=1000, block_size=16, num_layers=2,
                            num_heads=4).cuda()


def _step_fn(model, opt, params):
    from losses import dpace_loss

    mask = torch.ones(4, 16, device="cuda")
    mask[:, 0] = 0.0

    def fn(feats, tokens):
        opt.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16, cache_enabled=False):
            loss = model.compute_loss(feats, tokens, loss_fn=lambda lg, tk: dpace_loss(lg, tk, 0.5, position_mask=mask))
        loss.backward()
        torch.nn.utils.clip_grad_norm_(params, 1.0)
        opt.step()
        return loss

    return fn


def _batches(n):
    g = torch.Generator(device="cuda").manual_seed(11)
    return [(torch.randn(4, 112, 512, device="cuda", generator=g),
             torch.randint(0, 1000, (4, 16), device="cuda", generator=g)) for _ in range(n)]


def test_graphed_step_matches_eager(cuda):
    from specdec.graphs import GraphedStep

    ma, mb = _model(0), _model(0)
    mb.load_state_dict(ma.state_dict())
    pa = [p for p in ma.parameters() if p.requires_grad]
    pb = [p for p in mb.parameters() if p.requires_grad]
    oa = torch.optim.AdamW(pa, lr=1e-3, capturable=True)
    ob = torch.optim.AdamW(pb, lr=1e-3, capturable=True)
    fa, fb = _step_fn(ma, oa, pa), _step_fn(mb, ob, pb)
    batches = _batches(5)
    # GraphedStep warms up with three steps on its example inputs: the eager model takes the same three
    for _ in range(3):
        fa(*batches[0])
    step = GraphedStep(fb, *batches[0], optimizers=(ob,))
    for f, t in batches[1:]:
        la = float(fa(f, t))
        lb = float(step(f, t))
        assert abs(la - lb) <= 1e-5 * abs(la), (la, lb)
    step.check()
    for (n, a), b in zip(ma.named_parameters(), mb.parameters()):
        assert torch.allclose(a, b, rtol=1e-4, atol=1e-6), n


def test_graphed_step_reports_target_range(cuda):
    from specdec.graphs import GraphedStep

    m = _model(1)
    params = [p for p in m.parameters() if p.requires_grad]
    opt = torch.optim.AdamW(params, lr=1e-3, capturable=True)
    f, t = _batches(1)[0]
    step = GraphedStep(_step_fn(m, opt, params), f, t, optimizers=(opt,))
    step(f, t)
    step.check()
    bad = t.clone()
    bad[1, 3] = 1000  # == V
    step(f, bad)
    with pytest.raises(ValueError):
        step.check()
    step(f, t)
    step.check()  # the next good replay clears the forward's status word
