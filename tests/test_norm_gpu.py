"""The decoder block's fused elementwise launches against the unfused PyTorch
expressions they replace: rms_norm (the reference's model.py:34-38) with the
residual add before it, and the silu(gate) * up of swiglu_mlp (model.py:70-74).

The residual sum must be bit-identical (both round the fp32 sum once); the norm
may differ from the unfused form only by the order of its fp32 mean (one unit
in the last place of the output dtype at most); silu_mul by the exp used."""

import pytest
import torch

import pallas_flash as pf

pytestmark = pytest.mark.gpu

ULP = {torch.float32: 2e-6, torch.bfloat16: 2 ** -7, torch.float16: 2 ** -10}


def unfused_norm(x, w, eps):
    xf = x.to(torch.float32)
    var = xf.square().mean(dim=-1, keepdim=True)
    return (xf * torch.rsqrt(var + eps) * w).to(x.dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(16, 1, 512), (2, 128, 512), (3, 5, 64), (1, 1, 1000), (4, 7, 4096)])
def test_add_rms_norm_matches_unfused(dtype, shape):
    g = torch.Generator(device="cuda").manual_seed(shape[-1] + shape[1])
    x = torch.randn(shape, device="cuda", generator=g).to(dtype)
    r = torch.randn(shape, device="cuda", generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(shape[-1], device="cuda", generator=g)).to(dtype)
    xs, h = pf.add_rms_norm(x, r, w, 1e-5)
    torch.testing.assert_close(xs, x + r, rtol=0, atol=0)
    want = unfused_norm(x + r, w, 1e-5)
    tol = ULP[dtype] * float(want.abs().max()) * 1.01
    assert float((h.float() - want.float()).abs().max()) <= tol
    # no residual: x passes through, h is rms_norm(x)
    x2, h2 = pf.add_rms_norm(x, None, w, 1e-5)
    assert x2.data_ptr() == x.data_ptr()
    assert float((h2.float() - unfused_norm(x, w, 1e-5).float()).abs().max()) <= tol
    assert float((pf.rms_norm(x, w, 1e-5).float() - h2.float()).abs().max()) == 0.0


def test_add_rms_norm_zero_row_and_bad_shapes():
    x = torch.zeros((2, 64), device="cuda", dtype=torch.bfloat16)
    w = torch.ones(64, device="cuda", dtype=torch.bfloat16)
    _, h = pf.add_rms_norm(x, None, w, 1e-5)
    assert torch.count_nonzero(h) == 0
    with pytest.raises(ValueError):
        pf.add_rms_norm(x, None, torch.ones(63, device="cuda", dtype=torch.bfloat16), 1e-5)
    with pytest.raises(ValueError):
        pf.add_rms_norm(x, torch.zeros((1, 64), device="cuda", dtype=torch.bfloat16), w, 1e-5)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n", [(16, 1, 1408), (3, 77), (1,), (2, 128, 1408)])
def test_silu_mul_matches_unfused(dtype, n):
    g = torch.Generator(device="cuda").manual_seed(sum(n))
    a = (3 * torch.randn(n, device="cuda", generator=g)).to(dtype)
    b = torch.randn(n, device="cuda", generator=g).to(dtype)
    got = pf.silu_mul(a, b)
    want = torch.nn.functional.silu(a) * b
    tol = 2 * ULP[dtype] * float(want.abs().max()) + 1e-6
    assert float((got.float() - want.float()).abs().max()) <= tol


def test_silu_mul_on_a_fused_projection_equals_separate_halves():
    g = torch.Generator(device="cuda").manual_seed(3)
    gu = torch.randn((16, 1, 2 * 1408), device="cuda", generator=g).to(torch.bfloat16)
    fused = pf.silu_mul(gu)
    split = pf.silu_mul(gu[..., :1408].contiguous(), gu[..., 1408:].contiguous())
    assert fused.shape == (16, 1, 1408)
    torch.testing.assert_close(fused, split, rtol=0, atol=0)


def test_swiglu_mlp_with_fused_projection_tracks_weight_updates():
    from pallas_flash import model
    g = torch.Generator(device="cuda").manual_seed(4)
    x = torch.randn((16, 1, 512), device="cuda", generator=g).to(torch.bfloat16)
    wg, wu = (0.05 * torch.randn((512, 1408), device="cuda", generator=g)).to(torch.bfloat16), \
             (0.05 * torch.randn((512, 1408), device="cuda", generator=g)).to(torch.bfloat16)
    wd = (0.05 * torch.randn((1408, 512), device="cuda", generator=g)).to(torch.bfloat16)
    want = (torch.nn.functional.silu(x @ wg) * (x @ wu)) @ wd
    got = model.swiglu_mlp(x, wg, wu, wd)
    assert float((got.float() - want.float()).abs().max()) <= 0.02 * float(want.abs().max())
    wu.mul_(2.0)  # in-place update: the cached concatenation must not be reused
    want2 = (torch.nn.functional.silu(x @ wg) * (x @ wu)) @ wd
    got2 = model.swiglu_mlp(x, wg, wu, wd)
    assert float((got2.float() - want2.float()).abs().max()) <= 0.02 * float(want2.abs().max())


@pytest.mark.parametrize("pos,C", [(0, 512), (511, 512), (512, 512), (4222, 512), (7, 1)])
def test_decode_positions(pos, C):
    from pallas_flash import _lib
    B = 16
    p = torch.tensor([pos], dtype=torch.long, device="cuda")
    slots, lens, rows = (torch.full((B,), -1, dtype=torch.int32, device="cuda") for _ in range(3))
    _lib.check(_lib.lib().pf_decode_positions(p.data_ptr(), C, slots.data_ptr(), lens.data_ptr(),
                                              rows.data_ptr(), B, _lib.stream_of(p)))
    torch.cuda.synchronize()
    assert int(p.item()) == pos + 1
    assert slots.tolist() == [pos % C] * B
    assert lens.tolist() == [min(pos + 1, C)] * B
    assert rows.tolist() == [pos] * B


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_argmax_embed_matches_torch_argmax_and_lookup(dtype):
    from pallas_flash import _lib
    rows, vocab, dim = 6, 32000, 512
    g = torch.Generator(device="cuda").manual_seed(5)
    logits = torch.randn((rows, vocab), device="cuda", generator=g).to(dtype)
    logits[1, 100] = logits[1, 31000] = 1e4         # tie: the first index wins
    logits[2] = float("-inf")                        # all -inf: index 0
    logits[3, 7] = float("nan")                      # NaN ranks above every number
    logits[3, 9] = 1e4
    logits[4, 5] = logits[4, 6] = float("nan")       # first NaN
    logits[5, vocab - 1] = 1e4                       # the last column
    embed = torch.randn((vocab, dim), device="cuda", generator=g).to(dtype)
    token = torch.full((rows, 1), -1, dtype=torch.long, device="cuda")
    x = torch.zeros((rows, 1, dim), dtype=dtype, device="cuda")
    _lib.check(_lib.lib().pf_argmax_embed(logits.data_ptr(), vocab, vocab, rows, token.data_ptr(), embed.data_ptr(),
                                          x.data_ptr(), dim, _lib.dtype_code(dtype), _lib.stream_of(logits)))
    want = torch.argmax(logits, dim=-1, keepdim=True)
    assert token.tolist() == want.tolist()
    assert [t[0] for t in token.tolist()][1:] == [100, 0, 7, 5, vocab - 1]
    assert torch.equal(x, embed[token])
    # row stride larger than the vocabulary (a view of a wider buffer), no embedding
    wide = torch.randn((rows, vocab + 64), device="cuda", generator=g).to(dtype)
    tok2 = torch.full((rows,), -1, dtype=torch.long, device="cuda")
    _lib.check(_lib.lib().pf_argmax_embed(wide.data_ptr(), vocab + 64, vocab, rows, tok2.data_ptr(), None, None,
                                          0, _lib.dtype_code(dtype), _lib.stream_of(wide)))
    assert tok2.tolist() == torch.argmax(wide[:, :vocab], dim=-1).tolist()


def test_norm_and_swiglu_are_differentiable_like_the_unfused_expressions():
    """Gradients through add_rms_norm / rms_norm / swiglu_mlp (kernel forward, closed-form
    backward) match torch autograd of the unfused expressions (fp32, relative 1e-4)."""
    from pallas_flash import model
    g = torch.Generator(device="cuda").manual_seed(6)

    def leaf(*shape, scale=1.0):
        return (scale * torch.randn(shape, device="cuda", generator=g)).requires_grad_(True)

    x, r, w = leaf(3, 5, 64), leaf(3, 5, 64), leaf(64)
    wg, wu, wd = leaf(64, 96, scale=0.1), leaf(64, 96, scale=0.1), leaf(96, 64, scale=0.1)
    cot_x, cot_h = torch.randn((3, 5, 64), device="cuda", generator=g), torch.randn((3, 5, 64), device="cuda",
                                                                                  generator=g)

    def run(fused):
        for t in (x, r, w, wg, wu, wd):
            t.grad = None
        if fused:
            xs, h = model.add_rms_norm(x, r, w, 1e-5)
            out = model.swiglu_mlp(h, wg, wu, wd) + model.rms_norm(xs, w, 1e-5)
        else:
            xs = x + r
            h = unfused_norm(xs, w, 1e-5)
            out = (torch.nn.functional.silu(h @ wg) * (h @ wu)) @ wd + unfused_norm(xs, w, 1e-5)
        ((xs * cot_x).sum() + (out * cot_h).sum()).backward()
        return [t.grad.clone() for t in (x, r, w, wg, wu, wd)]

    got, want = run(True), run(False)
    for name, a, b in zip(("x", "residual", "weight", "w_gate", "w_up", "w_down"), got, want):
        rel = float((a - b).abs().max() / b.abs().max())
        assert rel < 1e-4, (name, rel)
