"""zl_linear_swiglu (the MLP gate/up projection with silu(gate) * up fused into
its epilogue) through the C ABI against a plain PyTorch fp32 reference of the
same op: silu(x W_gate^T) * (x W_up^T) from the bf16 inputs upcast to fp32.
The kernel accumulates in fp32 and rounds the product to bf16 once, so the
tolerance is the bf16 rounding of the output plus accumulation-order noise:
2e-2 absolute + 2e-2 relative."""
import pytest

pytestmark = pytest.mark.gpu


def _run(ctx, M, K, I, seed, w_std=0.02):
    import torch
    from zealot_b200 import lib
    from zealot_b200.context import ptr
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn((2 * I, K), generator=g, device="cuda") * w_std).to(torch.bfloat16)
    out = torch.full((M, I), float("nan"), dtype=torch.bfloat16, device="cuda")
    rc = lib.zl_linear_swiglu(ctx.handle, ptr(x), ptr(w), ptr(out), M, K, I, ctx.stream())
    assert rc == 0, lib.zl_last_error()
    ctx.check_status()
    xf, wf = x.float(), w.float()
    gate, up = xf @ wf[:I].T, xf @ wf[I:].T
    ref = torch.nn.functional.silu(gate) * up
    return out.float(), ref


@pytest.mark.parametrize("M,K,I", [(1, 64, 128), (7, 128, 256), (130, 256, 384), (300, 4096, 1024),
                                   (513, 1024, 2048)])
def test_linear_swiglu_matches_fp32_reference(ctx, M, K, I):
    """Ragged row counts (partial 128-row tiles, rows past M never written), one
    and many k-blocks, several output strips."""
    import torch
    got, ref = _run(ctx, M, K, I, seed=M + K + I, w_std=1.0 / K ** 0.5)
    torch.testing.assert_close(got, ref, atol=2e-2, rtol=2e-2)


def test_linear_swiglu_c4_shape(ctx):
    """The C4 layer shape: 4,344 rows (8 x 512 prefill + 248 decode), hidden 4096,
    intermediate 14336, weights N(0, 0.02) as the engine-step bench draws them."""
    import torch
    got, ref = _run(ctx, 4344, 4096, 14336, seed=4)
    torch.testing.assert_close(got, ref, atol=2e-2, rtol=2e-2)


def test_linear_swiglu_rejects_unsupported_shapes(ctx):
    import torch
    from zealot_b200 import lib
    from zealot_b200.context import ptr
    x = torch.zeros((4, 128), dtype=torch.bfloat16, device="cuda")
    w = torch.zeros((2 * 128, 128), dtype=torch.bfloat16, device="cuda")
    out = torch.zeros((4, 128), dtype=torch.bfloat16, device="cuda")
    assert lib.zl_linear_swiglu(ctx.handle, ptr(x), ptr(w), ptr(out), 4, 100, 128, ctx.stream()) == 6
    assert lib.zl_linear_swiglu(ctx.handle, ptr(x), ptr(w), ptr(out), 4, 128, 96, ctx.stream()) == 6
    assert lib.zl_linear_swiglu(ctx.handle, ptr(x), ptr(w), ptr(out), 0, 128, 128, ctx.stream()) == 0
    assert lib.zl_linear_swiglu(ctx.handle, ptr(x), 0, ptr(out), 4, 128, 128, ctx.stream()) == 1
    ctx.check_status()
