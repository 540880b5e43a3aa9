"""GPU: the row-copy kernel (esa_copy_rows) that moves the sequence split's
K / V rows and partial dK / dV between [B, S, H, D] tensors and
per-head-group [rows, B, heads, D] buffers, against torch's copy of the same
views: bit-identical (a 16-bit copy moves bits; fp32 -> bf16 / fp16 rounds
to nearest even, as torch's cast does)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.mark.parametrize("src_dt,dst_dt", [
    (torch.bfloat16, torch.bfloat16), (torch.float16, torch.float16),
    (torch.float32, torch.bfloat16), (torch.float32, torch.float16)])
@pytest.mark.parametrize("B,S,ng,hg,D", [(1, 4099, 4, 4, 128), (2, 517, 2, 3, 64),
                                          (3, 33, 1, 1, 8)])
def test_copy_rows_matches_torch(esa, src_dt, dst_dt, B, S, ng, hg, D):
    g = torch.Generator().manual_seed(B * 1000 + S + D)
    # to the buffer: [B, S, H, D] -> [ng, rows, B, hg * D] rows at an offset
    k = (torch.randn(B, S, ng * hg, D, generator=g) * 3).to(DEV, src_dt)
    if src_dt == torch.float32:   # values near bf16 / fp16 rounding midpoints and overflow
        k[0, 0, 0, :4] = torch.tensor([1.00390625, 1.01171875, 70000.0, -3e-8])
    off, rows = 5, S + 7
    buf = torch.full((ng, rows, B, hg, D), 7.0, device=DEV, dtype=dst_dt)
    want = buf.clone()
    src = k.unflatten(2, (ng, hg)).flatten(3, 4).permute(2, 1, 0, 3)
    want[:, off:off + S].flatten(3, 4).copy_(src)
    esa.ops.copy_rows(buf[:, off:off + S].flatten(3, 4), src)
    assert torch.equal(buf.view(torch.int16), want.view(torch.int16))
    # back: [ng, S, B, hg * D] -> [B, S, H, D]
    part = (torch.randn(ng, S, B, hg, D, generator=g)).to(DEV, src_dt)
    out = torch.empty((B, S, ng, hg, D), device=DEV, dtype=dst_dt)
    ref = torch.empty_like(out)
    ref.flatten(3, 4).permute(2, 1, 0, 3).copy_(part.flatten(3, 4))
    esa.ops.copy_rows(out.flatten(3, 4).permute(2, 1, 0, 3), part.flatten(3, 4))
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


def test_copy_rows_large_grid(esa):
    """More rows than the grid's warps (each warp strides over rows), C5's
    row length (4 heads x 128)."""
    g = torch.Generator(device=DEV).manual_seed(3)
    src = torch.randn(4, 65536, 1, 512, device=DEV, generator=g)
    dst = torch.empty(1, 65536, 4, 512, device=DEV, dtype=torch.bfloat16).permute(2, 1, 0, 3)
    esa.ops.copy_rows(dst, src)
    assert torch.equal(dst, src.to(torch.bfloat16))


def test_copy_rows_rejects_unaligned_views(esa):
    x = torch.zeros(2, 3, 4, 16, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(esa._lib.EsaError, match="esa_copy_rows"):
        esa.ops.copy_rows(x[..., 4:12], x[..., :8].clone())
    with pytest.raises(ValueError):
        esa.ops.copy_rows(x, x[..., :8])
