"""The full single-layer operator (256 x 1024 tokens, 768 -> 3072, k = 16384) through
size-independent properties, where the float64 oracle would take minutes (GPU).

- CountSketch is linear in dL/dZ: the sketch of 2 * dLdZ (exact in bf16) is twice the sketch.
- Summing candidates into one row (rows_div) equals the column sum of their rows.
- The ghost contraction against the de-sketched target equals phi . tau of the sketches.
- The fixed-point shared sketch equals the f32 global-atomic path.

And sampled rows of full-size launches against the float64 oracle: rows are
independent, so a few rows check the full launch's job dealing and
per-candidate scales at a fraction of the oracle's cost.
"""
import numpy as np
import pytest
import torch

from opus_b200 import ops
from opus_b200.train.random_projection import GradientProjector

pytestmark = pytest.mark.gpu
DEV = "cuda"
B, T, D_IN, D_OUT, K = 256, 1024, 768, 3072, 16384


@pytest.fixture(scope="module")
def operator():
    g = torch.Generator(device=DEV).manual_seed(1234)
    a = torch.randn(B, T, D_IN, generator=g, device=DEV).to(torch.bfloat16)
    dz = (torch.randn(B, T, D_OUT, generator=g, device=DEV) * 1e-3).to(torch.bfloat16)
    diag = torch.rand(D_OUT, D_IN, generator=g, device=DEV) * (1e-3 - 1e-6) + 1e-6
    proj = GradientProjector(sketch_dim=K, seed=42, device="cuda")
    packed = proj.packed_table(D_OUT * D_IN, 0, torch.device(DEV))
    load = proj.max_bucket_load(D_OUT * D_IN, 0, torch.device(DEV))
    table = ops.build_sketch_table(packed, D_OUT, D_IN, diag=diag)
    phi = ops.sketch_gemm(dz, a, table, K, max_bucket_load=load)
    ops.check_device_error("full-size sketch")
    return dict(a=a, dz=dz, diag=diag, packed=packed, load=load, table=table, phi=phi)


def rel(x, y):
    x, y = x.double(), y.double()
    return float((x - y).abs().max() / y.abs().max().clamp_min(1e-30))


def test_linearity_in_dldz(operator):
    o = operator
    phi2 = ops.sketch_gemm(o["dz"] * 2, o["a"], o["table"], K, max_bucket_load=o["load"])
    assert rel(phi2, 2 * o["phi"]) < 1e-5


def test_rows_div_sums_candidates(operator):
    o = operator
    summed = ops.sketch_gemm(o["dz"], o["a"], o["table"], K, rows_div=B, max_bucket_load=o["load"])
    assert summed.shape == (1, K)
    assert rel(summed[0], o["phi"].double().sum(0)) < 1e-4


def test_fixed_point_equals_global_atomics(operator):
    o = operator
    plain = ops.sketch_gemm(o["dz"], o["a"], o["table"], K, max_bucket_load=0)
    assert rel(o["phi"], plain) < 1e-5


def test_ghost_identity_at_full_size(operator):
    o = operator
    V = torch.randn(D_IN, D_OUT, device=DEV) / D_IN ** 0.5
    tau = ops.sketch_dense(V, o["packed"], D_OUT, D_IN, K, transposed=True)
    via_sketch = ops.sketch_dot(o["phi"], tau)
    v = ops.desketch(tau, o["packed"], D_OUT, D_IN, diag=o["diag"])
    via_ghost = ops.ghost_score(o["a"], o["dz"], v)
    assert rel(via_ghost, via_sketch) < 1e-3
    sim = ops.sketch_gram(o["phi"])
    assert rel(sim, (o["phi"].double() @ o["phi"].double().T)) < 2e-5
    assert torch.allclose(sim, sim.T, rtol=1e-5, atol=1e-5 * float(sim.abs().max()))


def _oracle_rows(dz, a, h, s, k, diag, rows):
    """float64 oracle sketches of the given candidates (the reference's project_full_gradient)."""
    from oracle import opus_oracle as orc

    d = None if diag is None else diag.cpu().numpy()
    return np.stack([orc.project_full_gradient(dz[b:b + 1].float().cpu().numpy(), a[b:b + 1].float().cpu().numpy(),
                                               h, s, k, diag=d)[0] for b in rows])


def _check_rows(got, want, what):
    """Each sampled row within 1e-4 of its largest bucket; the rows' Gram (a similarity block) within 1e-3."""
    for i in range(want.shape[0]):
        err = np.abs(got[i] - want[i]).max() / np.abs(want[i]).max()
        assert err < 1e-4, f"{what} row {i}: {err:.3e}"
    gram_got, gram_want = got @ got.T, want @ want.T
    diag_err = np.abs(np.diag(gram_got) - np.diag(gram_want)) / np.diag(gram_want)
    assert diag_err.max() < 1e-3, f"{what} squared norms: {diag_err.max():.3e}"


def test_sampled_rows_of_the_full_launch_match_the_oracle(operator):
    """8 rows of the full 256-candidate launch (jobs dealt over every SM, per-candidate fixed-point scales)."""
    from oracle import opus_oracle as orc

    o = operator
    rows = [0, 1, 37, 100, 128, 129, 200, 255]
    h, s = orc.hash_sign_tables(D_OUT * D_IN, 0, K, seed=42, device="cuda")
    want = _oracle_rows(o["dz"], o["a"], h, s, K, o["diag"], rows)
    _check_rows(o["phi"][rows].double().cpu().numpy(), want, "k=16384")


def test_sampled_rows_at_the_gpt2_xl_mlp_shape():
    """k = 65536 at 1600 -> 6400 with 128 candidates (the shared-memory prefix plus L2 atomics above it)."""
    from oracle import opus_oracle as orc

    d_in, d_out, k, nb = 1600, 6400, 65536, 128
    g = torch.Generator(device=DEV).manual_seed(77)
    a = torch.randn(nb, T, d_in, generator=g, device=DEV).to(torch.bfloat16)
    dz = (torch.randn(nb, T, d_out, generator=g, device=DEV) * 1e-3).to(torch.bfloat16)
    diag = torch.rand(d_out, d_in, generator=g, device=DEV) * (1e-3 - 1e-6) + 1e-6
    proj = GradientProjector(sketch_dim=k, seed=42, device="cuda")
    packed = proj.packed_table(d_out * d_in, 3, torch.device(DEV))
    load = proj.max_bucket_load(d_out * d_in, 3, torch.device(DEV))
    table = ops.build_sketch_table(packed, d_out, d_in, diag=diag)
    phi = ops.sketch_gemm(dz, a, table, k, max_bucket_load=load)
    ops.check_device_error("k=65536 sketch")
    rows = [0, 63, 64, 127]
    h, s = orc.hash_sign_tables(d_out * d_in, 3, k, seed=42, device="cuda")
    want = _oracle_rows(dz, a, h, s, k, diag, rows)
    _check_rows(phi[rows].double().cpu().numpy(), want, "k=65536")
