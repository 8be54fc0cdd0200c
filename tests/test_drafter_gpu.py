"""The drafter's own layers on the library's kernels (specdec.drafter): RMSNorm
forward/backward and the DFlash-mask attention on the tensor cores, each
against a plain PyTorch reference of the same op (float64 for the norm,
float32 for the attention on the same bf16 inputs).

Tolerances:
- RMSNorm, fp32 activations: y, dx 1e-5 relative to the row's scale, dw
  1e-4 relative (a sum over all rows); bf16 activations: the output and dx
  within half a bf16 ulp (2^-8 relative) of the reference plus 1e-6.
- Attention (bf16 q/k/v): o within 1e-2 absolute + 1e-2 relative of the
  fp32 reference -- p is rounded to bf16 before the second product and o is
  stored in bf16, each a 2^-9 relative rounding -- and the log-sum-exp
  within 1e-3; gradients within 2e-2 absolute + 2e-2 relative.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref_rms(x, w, eps):
    x64, w64 = x.double(), w.double()
    return x64 * torch.rsqrt(x64.pow(2).mean(-1, keepdim=True) + eps) * w64


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("rows,D", [(1, 256), (100, 256), (16896, 256), (512, 4096), (37, 1000), (5, 257),
                                    (64, 2048), (8, 8192), (3, 8200), (300, 64)])
def test_rmsnorm_forward_backward(cuda, dtype, rows, D):
    from specdec import drafter

    g = torch.Generator(device="cuda").manual_seed(rows * 7 + D)
    x = (torch.randn(rows, D, device="cuda", generator=g) * 1.5).to(dtype).requires_grad_(True)
    w = (1.0 + 0.1 * torch.randn(D, device="cuda", generator=g)).requires_grad_(True)
    dy = torch.randn(rows, D, device="cuda", generator=g).to(dtype)
    eps = torch.finfo(dtype).eps
    y = drafter.rms_norm(x, w)
    y.backward(dy)
    xr = x.detach().double().requires_grad_(True)
    wr = w.detach().double().requires_grad_(True)
    yr = _ref_rms(xr, wr, eps)
    yr.backward(dy.double())
    assert y.dtype == dtype and x.grad.dtype == dtype and w.grad.dtype == torch.float32
    if dtype == torch.float32:
        scale = yr.detach().abs().amax(-1, keepdim=True) + 1e-12
        assert float(((y.double() - yr) / scale).abs().max()) <= 1e-5
        gs = xr.grad.abs().amax(-1, keepdim=True) + 1e-12
        assert float(((x.grad.double() - xr.grad) / gs).abs().max()) <= 1e-5
    else:
        assert bool(((y.double() - yr).abs() <= 2.0 ** -8 * yr.abs() + 1e-6).all())
        assert bool(((x.grad.double() - xr.grad).abs() <= 2.0 ** -8 * xr.grad.abs() + 1e-6 +
                     1e-5 * xr.grad.abs().amax(-1, keepdim=True)).all())
    assert float(((w.grad.double() - wr.grad).abs() / (wr.grad.abs().max() + 1e-12)).max()) <= 1e-4
    # bitwise repeatable (fixed-order weight-gradient reduction)
    w.grad = None
    drafter.rms_norm(x, w).backward(dy)
    g1 = w.grad.clone()
    w.grad = None
    drafter.rms_norm(x, w).backward(dy)
    assert torch.equal(g1, w.grad)


def _ref_attention(q, k, v, n_ctx, scale):
    """fp32 reference with the explicit DFlash mask; q/k/v [B, T, H, D]."""
    qh, kh, vh = (t.permute(0, 2, 1, 3).float() for t in (q, k, v))
    T = q.shape[1]
    i = torch.arange(T, device=q.device).view(T, 1)
    j = torch.arange(T, device=q.device).view(1, T)
    vis = (i >= n_ctx) | (j <= i)
    s = torch.matmul(qh, kh.transpose(-1, -2)) * scale
    s = s.masked_fill(~vis, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    o = torch.matmul(torch.softmax(s, dim=-1), vh)
    return o.permute(0, 2, 1, 3), lse


SHAPES = [(2, 528, 4, 512), (3, 100, 2, 90), (2, 300, 4, 200), (1, 257, 1, 0), (1, 200, 2, 200),
          (4, 129, 3, 1), (1, 640, 2, 500)]


def _qkv(B, T, H, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(B, T, H, 64, device="cuda", generator=g).to(torch.bfloat16) for _ in range(3)]


@pytest.mark.parametrize("B,T,H,n_ctx", SHAPES)
def test_attention_forward_matches_reference(cuda, B, T, H, n_ctx):
    from specdec import _lib

    q, k, v = _qkv(B, T, H, B * 1000 + T)
    lib = _lib.load()
    o = torch.empty_like(q)
    lse = torch.empty(B, H, T, device="cuda")
    status = torch.zeros((1,), dtype=torch.int32, device="cuda")  # sticky: set only on an expired wait
    rc = lib.specdec_dflash_attention_forward(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                              lse.data_ptr(), B, T, H, 64, n_ctx, 0.125, status.data_ptr(),
                                              torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.OK, _lib.last_error()
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    o_ref, lse_ref = _ref_attention(q, k, v, n_ctx, 0.125)
    err = (o.float() - o_ref).abs()
    assert bool((err <= 1e-2 + 1e-2 * o_ref.abs()).all()), float(err.max())
    assert float((lse - lse_ref).abs().max()) <= 1e-3
    # deterministic: the same bits twice
    o2 = torch.empty_like(q)
    lib.specdec_dflash_attention_forward(q.data_ptr(), k.data_ptr(), v.data_ptr(), o2.data_ptr(),
                                         lse.data_ptr(), B, T, H, 64, n_ctx, 0.125, None,
                                         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert torch.equal(o, o2)


@pytest.mark.parametrize("B,T,H,n_ctx", SHAPES)
def test_attention_backward_matches_reference(cuda, B, T, H, n_ctx):
    from specdec import drafter

    q, k, v = _qkv(B, T, H, 7 + T)
    do = torch.randn(B, T, H, 64, device="cuda").to(torch.bfloat16)
    qs, ks, vs = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = drafter.dflash_attention(qs, ks, vs, n_ctx)
    o.backward(do)
    qr, kr, vr = (t.float().clone().requires_grad_(True) for t in (q, k, v))
    o_ref, _ = _ref_attention(qr, kr, vr, n_ctx, 0.125)
    o_ref.backward(do.float())
    for got, want in ((qs.grad, qr.grad), (ks.grad, kr.grad), (vs.grad, vr.grad)):
        err = (got.float() - want).abs()
        assert bool((err <= 2e-2 + 2e-2 * want.abs()).all()), float(err.max())
    # bitwise repeatable (no atomics)
    g1 = [t.grad.clone() for t in (qs, ks, vs)]
    for t in (qs, ks, vs):
        t.grad = None
    drafter.dflash_attention(qs, ks, vs, n_ctx).backward(do)
    for a, t in zip(g1, (qs, ks, vs)):
        assert torch.equal(a, t.grad)


def test_attention_rejects_bad_arguments(cuda):
    from specdec import _lib

    lib = _lib.load()
    q, k, v = _qkv(1, 16, 1, 3)
    o = torch.empty_like(q)
    lse = torch.empty(1, 1, 16, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert lib.specdec_dflash_attention_forward(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                                lse.data_ptr(), 1, 16, 1, 32, 0, 0.125, None, s) == _lib.ERR_ARGUMENT
    assert lib.specdec_dflash_attention_forward(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                                lse.data_ptr(), 1, 16, 1, 64, 17, 0.125, None, s) == _lib.ERR_ARGUMENT
    assert lib.specdec_dflash_attention_forward(q.data_ptr() + 2, k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                                lse.data_ptr(), 1, 16, 1, 64, 0, 0.125, None, s) == _lib.ERR_ARGUMENT


def test_drafter_with_kernels_matches_plain_torch(cuda):
    """A small DFlashSpeculator under bf16 autocast: the library's norm and
    attention kernels against torch's own modules (nn.RMSNorm math, SDPA):
    logits and parameter gradients agree to bf16 accuracy."""
    from models.dflash.model import DFlashSpeculator
    from specdec import drafter

    torch.manual_seed(0)
    m = DFlashSpeculator(d_target=512, d_model=256, target_vocab_size=1000, block_size=16, num_layers=2,
                         num_heads=4).cuda()
    feats = torch.randn(2, 112, 512, device="cuda")
    tokens = torch.randint(0, 1000, (2, 16), device="cuda")

    def run(enabled):
        drafter.set_enabled(enabled)
        m.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits = m(feats)
            loss = torch.nn.functional.cross_entropy(logits.float().reshape(-1, 1000), tokens.reshape(-1))
        loss.backward()
        return logits.float().detach(), float(loss), {n: p.grad.clone() for n, p in m.named_parameters()
                                                      if p.grad is not None}

    try:
        lk, lossk, gk = run(True)
        lt, losst, gt = run(False)
    finally:
        drafter.set_enabled(True)
    assert abs(lossk - losst) <= 2e-2 * abs(losst)
    assert float((lk - lt).abs().max()) <= 5e-2 * float(lt.abs().max()) + 5e-2
    for n, g in gt.items():
        rel = float((gk[n].float() - g.float()).norm() / (g.float().norm() + 1e-12))
        assert rel <= 5e-2, (n, rel)


@pytest.mark.parametrize("n_ctx", [0, 384])
def test_attention_forward_rescale_path(cuda, n_ctx):
    """Scores that grow tile by tile (key j scaled by 1 + j / 16): a row's
    reference maximum is raised several times and O is rescaled in tensor
    memory each time; output, lse and the backward still match the fp32
    reference."""
    from specdec import _lib, drafter

    B, T, H = 2, 528, 2
    g = torch.Generator(device="cuda").manual_seed(123)
    q = torch.randn(B, T, H, 64, device="cuda", generator=g)
    k = torch.randn(B, T, H, 64, device="cuda", generator=g)
    k = k * (1.0 + torch.arange(T, device="cuda", dtype=torch.float32) / 16.0).view(1, T, 1, 1)
    v = torch.randn(B, T, H, 64, device="cuda", generator=g)
    q, k, v = (t.to(torch.bfloat16) for t in (q, k, v))
    lib = _lib.load()
    o = torch.empty_like(q)
    lse = torch.empty(B, H, T, device="cuda")
    status = torch.zeros((1,), dtype=torch.int32, device="cuda")  # sticky: set only on an expired wait
    rc = lib.specdec_dflash_attention_forward(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                              lse.data_ptr(), B, T, H, 64, n_ctx, 0.125, status.data_ptr(),
                                              torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.OK, _lib.last_error()
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    o_ref, lse_ref = _ref_attention(q, k, v, n_ctx, 0.125)
    assert float((lse_ref.amax() - lse_ref.amin())) > 20.0  # the scores do span several 2^8 steps
    err = (o.float() - o_ref).abs()
    assert bool((err <= 1e-2 + 1e-2 * o_ref.abs()).all()), float(err.max())
    assert float(((lse - lse_ref).abs() / lse_ref.abs().clamp_min(1.0)).max()) <= 1e-3
    do = torch.randn(B, T, H, 64, device="cuda", generator=g).to(torch.bfloat16)
    qs, ks, vs = (t.clone().requires_grad_(True) for t in (q, k, v))
    drafter.dflash_attention(qs, ks, vs, n_ctx).backward(do)
    qr, kr, vr = (t.float().clone().requires_grad_(True) for t in (q, k, v))
    _ref_attention(qr, kr, vr, n_ctx, 0.125)[0].backward(do.float())
    # keys up to 34x larger make dQ = dS K sum ~500 products of that size with dS rounded to
    # bf16 (2^-9): the bound is relative to each gradient's own scale
    for got, want in ((qs.grad, qr.grad), (ks.grad, kr.grad), (vs.grad, vr.grad)):
        err = (got.float() - want).abs()
        scale = float(want.abs().max())
        assert float(err.max()) <= 2e-2 * scale, (float(err.max()), scale)
        assert float(err.norm() / want.norm()) <= 1e-2
