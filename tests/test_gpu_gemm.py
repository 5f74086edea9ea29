"""The tcgen05 bf16 GEMM and the Muon preconditioner kernels against torch and the reference's recipe (GPU)."""
import numpy as np
import pytest
import torch

from conftest import load_golden
from opus_b200 import ops
from oracle import reference_torch as rt

pytestmark = pytest.mark.gpu
DEV = "cuda"


def bf16_ulps(got: torch.Tensor, want: torch.Tensor) -> torch.Tensor:
    """Distance in bf16 units in the last place between two bf16 tensors (sign-magnitude order)."""
    def key(x):
        i = x.contiguous().view(torch.int16).to(torch.int32)
        return torch.where(i < 0, -(i & 0x7FFF), i)
    return (key(got) - key(want)).abs()


def assert_bf16_close(got, want, max_ulps=1, max_frac=0.02, acc=1e-5, what=""):
    """Equal up to the last-place rounding of f32 sums taken in another order.

    bf16 x bf16 products are exact in f32, so the only difference from torch is
    the order of the f32 additions; after rounding to bf16 an element differs
    only when its f32 sum lies next to a rounding boundary: few elements
    differ, by max_ulps of their value, or -- where the sum cancels to a value
    far below the largest entry, whose ulp is tiny -- by the f32 accumulation
    error, acc times the largest entry.
    """
    d = bf16_ulps(got, want)
    frac = float((d > 0).float().mean())
    g, w = got.double(), want.double()
    ulp = torch.ldexp(torch.ones_like(w), torch.frexp(w.abs().clamp_min(1e-30))[1] - 8)
    bad = (g - w).abs() > max_ulps * ulp + acc * w.abs().max()
    assert frac <= max_frac and not bool(bad.any()), \
        f"{what}: {frac:.4f} differ, {int(bad.sum())} beyond {max_ulps} ulps + {acc} of the largest entry"


@pytest.mark.parametrize("M,N,K", [(300, 264, 200), (1024, 768, 768), (5, 8, 8), (256, 512, 4096), (513, 1032, 72)])
def test_gemm_bf16_matches_torch(M, N, K):
    torch.manual_seed(M + N + K)
    a = torch.randn(M, K, device=DEV).bfloat16()
    b = torch.randn(N, K, device=DEV).bfloat16()
    ref = a.double() @ b.double().T
    got32 = ops.gemm_bf16(a, b, out_dtype=torch.float32, alpha=0.5)
    ops.check_device_error("gemm_bf16")
    err = (got32.double() - 0.5 * ref).abs().max() / (0.5 * ref).abs().max()
    assert float(err) < 1e-5
    got16 = ops.gemm_bf16(a, b, out_dtype=torch.bfloat16)
    assert_bf16_close(got16, (a.float() @ b.float().T).bfloat16(), what="bf16 output")


def test_gemm_bf16_split_operand_and_accumulate():
    torch.manual_seed(1)
    x = torch.randn(777, 520, device=DEV)
    b = torch.randn(136, 520, device=DEV).bfloat16()
    hi, lo = ops.split_bf16(x)
    ref = x.double() @ b.double().T
    out = torch.full((777, 136), 3.0, device=DEV)
    ops.gemm_bf16(hi, b, out_dtype=torch.float32, a_lo=lo, out=out, accumulate=True)
    ops.check_device_error("gemm_bf16 split")
    err = (out.double() - 3.0 - ref).abs().max() / ref.abs().max()
    assert float(err) < 2 ** -15


def test_gemm_bf16_rejects_bad_shapes():
    a = torch.zeros(4, 12, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="multiples of 8"):
        ops.gemm_bf16(a, torch.zeros(8, 12, device=DEV, dtype=torch.bfloat16))
    empty = ops.gemm_bf16(torch.zeros(0, 16, device=DEV, dtype=torch.bfloat16),
                          torch.zeros(8, 16, device=DEV, dtype=torch.bfloat16))
    assert empty.shape == (0, 8)


@pytest.mark.parametrize("d_out,d_in,dtype", [(256, 128, torch.bfloat16), (768, 3072, torch.float32),
                                              (1024, 1024, torch.bfloat16), (72, 44, torch.float32),
                                              (2048, 512, torch.bfloat16)])
def test_muon_S_matches_reference_recipe(d_out, d_in, dtype):
    """S from the kernels == the reference's bf16 torch recipe on the same GPU, up to last-place rounding."""
    torch.manual_seed(d_out)
    m = (torch.randn(d_out, d_in, device=DEV) * 1e-3).to(dtype)
    got = ops.muon_S(m)
    ops.check_device_error("muon_S")
    want = rt.muon_S(m)
    assert got.dtype == torch.bfloat16 and got.shape == (d_out, d_out)
    assert torch.equal(got, got.T), "S must be exactly symmetric"
    assert_bf16_close(got, want, max_ulps=2, max_frac=0.05, what="S")
    rel = (got.float() - want.float()).abs().max() / want.float().abs().max()
    assert float(rel) < 1e-2


def test_muon_S_identity_below_the_norm_threshold():
    for scale in (0.0, 1e-12):
        m = torch.full((64, 32), scale, device=DEV)
        got = ops.muon_S(m)
        assert torch.equal(got, torch.eye(64, device=DEV, dtype=torch.bfloat16))


def test_muon_S_golden():
    """The fixtures recorded from the reference (CPU bf16 arithmetic), within last-place rounding."""
    g = load_golden("muon")
    for i in range(int(g["n"])):
        m = torch.from_numpy(g[f"m{i}"]).to(DEV)
        got = ops.muon_S(m).float().cpu()
        want = torch.from_numpy(g[f"S{i}"])
        assert_bf16_close(got.bfloat16(), want.bfloat16(), max_ulps=2, max_frac=0.05, what=f"S{i}")
    zero = ops.muon_S(torch.zeros(8, 8, device=DEV)).float().cpu().numpy()
    np.testing.assert_array_equal(zero, g["S_zero"])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("d_out", [768, 200])
def test_muon_transform_matches_einsum(dtype, d_out):
    torch.manual_seed(d_out)
    g = (torch.randn(3, 257, d_out, device=DEV) * 1e-3).to(dtype)
    S = ops.muon_S(torch.randn(d_out, 96, device=DEV))
    got = ops.muon_transform(g, S, symmetric=True)
    ops.check_device_error("muon_transform")
    want = rt.muon_transform(g, S)
    assert got.dtype == dtype and got.shape == g.shape
    if dtype == torch.bfloat16:
        assert_bf16_close(got, want, what="transform")
    else:
        err = (got.double() - want.double()).abs().max() / want.double().abs().max()
        assert float(err) < 1e-5
    # an S that is not symmetric: the einsum's transpose is honoured
    R = torch.randn(d_out, d_out, device=DEV).bfloat16()
    got_r = ops.muon_transform(g.float(), R)
    want_r = rt.muon_transform(g.float(), R)
    err = (got_r.double() - want_r.double()).abs().max() / want_r.double().abs().max()
    assert float(err) < 1e-4
