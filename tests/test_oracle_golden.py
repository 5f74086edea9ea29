"""Pin the NumPy oracle against golden vectors recorded from the reference (CPU only)."""
import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import opus_oracle as orc


def test_hash_sign_tables_bit_exact():
    g = load_golden("tables")
    for i in range(int(g["n"])):
        numel, pid, k, seed = (int(x) for x in g[f"case{i}"])
        h, s = orc.hash_sign_tables(numel, pid, k, seed=seed, device="cpu")
        np.testing.assert_array_equal(h, g[f"h{i}"].astype(np.int64))
        np.testing.assert_array_equal(s, g[f"s{i}"].astype(np.float32))
        assert h.min() >= 0 and h.max() < k


def test_pack_tables_roundtrip():
    h, s = orc.hash_sign_tables(5000, 2, 777, seed=1)
    packed = orc.pack_tables(h, s)
    np.testing.assert_array_equal(packed & 0x7FFFFFFF, h)
    np.testing.assert_array_equal(np.where(packed >> 31, -1.0, 1.0).astype(np.float32), s)


def test_project_full_gradient_matches_reference():
    g = load_golden("project")
    for i in range(int(g["n"])):
        k, pid, two_d = (int(x) for x in g[f"meta{i}"])
        dLdZ, a = g[f"g{i}"], g[f"a{i}"]
        d_out, d_in = dLdZ.shape[-1], a.shape[-1]
        h, s = orc.hash_sign_tables(d_out * d_in, pid, k, seed=42)
        phi = orc.project_full_gradient(dLdZ, a, h, s, k, diag=g.get(f"diag{i}"), S=g.get(f"S{i}"))
        ref = g[f"phi{i}"]
        scale = np.abs(ref).max()
        np.testing.assert_allclose(phi, ref, rtol=1e-4, atol=1e-5 * scale)


def test_layer_bf16_scores_match_reference():
    g = load_golden("layer_bf16")
    B, k, pid = int(g["B"]), int(g["k"]), int(g["pid"])
    dLdZ, a = g["g"], g["a"]
    h, s = orc.hash_sign_tables(dLdZ.shape[-1] * a.shape[-1], pid, k, seed=42)
    pt = orc.project_full_gradient(dLdZ[:B], a[:B], h, s, k, diag=g["diag"])
    pv = orc.project_full_gradient(dLdZ[B:], a[B:], h, s, k)
    np.testing.assert_allclose(pt, g["phi_t"], rtol=1e-4, atol=1e-6 * np.abs(g["phi_t"]).max())
    np.testing.assert_allclose((pt @ pv.T).mean(1), g["score"], rtol=1e-4, atol=1e-6 * np.abs(g["score"]).max())
    np.testing.assert_allclose(pt @ pt.T, g["sim"], rtol=1e-4, atol=1e-6 * np.abs(g["sim"]).max())


def test_stochastic_selection_matches_reference():
    g = load_golden("select")
    for i in range(int(g["n"])):
        sel = orc.stochastic_greedy_selection(g[f"scores{i}"], g[f"sim{i}"], int(g[f"K{i}"]),
                                              temperature=float(g[f"temp{i}"]), uniforms=g[f"uni{i}"])
        assert sel == list(g[f"sel{i}"]), str(g[f"name{i}"])


def test_stochastic_selection_global_rng_stream():
    g = load_golden("select")
    np.random.seed(1000)
    sel = orc.stochastic_greedy_selection(g["scores0"], g["sim0"], int(g["K0"]), temperature=float(g["temp0"]))
    assert sel == list(g["sel0"])


def test_greedy_selection_matches_reference():
    g = load_golden("select")
    for i in range(int(g["n"])):
        assert orc.greedy_selection(g[f"scores{i}"], g[f"sim{i}"], int(g[f"K{i}"])) == list(g[f"greedy{i}"])
    assert orc.greedy_selection(g["nan_scores"], g["nan_sim"], 5) == list(g["nan_greedy"])


@pytest.mark.parametrize("n", [1, 5, 7, 8, 9, 127, 128, 129, 255, 256, 300, 1000, 4097, 8192])
def test_pairwise_sum_is_numpy_order(n):
    rng = np.random.default_rng(n)
    x = (rng.random(n) * 10.0 ** rng.integers(-6, 6, n)).astype(np.float32)
    assert orc.pairwise_sum_f32(x) == x.sum()


def test_choice_from_uniform_is_numpy_choice():
    rng = np.random.default_rng(3)
    for trial in range(50):
        n = int(rng.integers(2, 300))
        p = rng.random(n).astype(np.float32) ** 3
        p /= p.sum()
        np.random.seed(trial)
        want = np.random.choice(n, p=p)
        np.random.seed(trial)
        u = np.random.random_sample()
        assert orc.choice_from_uniform(p, u) == want


def test_muon_S_matches_reference():
    g = load_golden("muon")
    for i in range(int(g["n"])):
        S = orc.muon_S(g[f"m{i}"])
        ref = g[f"S{i}"]
        # bf16 results: allow one bf16 ulp where float32 GEMM accumulation orders differ
        np.testing.assert_allclose(S, ref, rtol=2 ** -7, atol=2 ** -7 * np.abs(ref).max())
        d_out, d_in = g[f"m{i}"].shape
        assert orc.muon_scale(0.02, d_out, d_in, 0.95) == pytest.approx(float(g[f"C{i}"]), rel=1e-6)
    np.testing.assert_array_equal(orc.muon_S(np.zeros((8, 8), np.float32)), g["S_zero"])


def test_inv_rms_is_ieee_float32():
    """1/(sqrt(v)+eps) with each float32 step correctly rounded (what torch computes on CUDA).

    Each step is evaluated in float64 and rounded once to float32, which is
    correctly rounded for sqrt, add and divide of float32 operands.
    """
    v = np.random.default_rng(0).uniform(1e-9, 1e-2, 10000).astype(np.float32)
    s = np.sqrt(v.astype(np.float64)).astype(np.float32)
    x = (s.astype(np.float64) + np.float64(np.float32(1e-8))).astype(np.float32)
    ref = (1.0 / x.astype(np.float64)).astype(np.float32)
    np.testing.assert_array_equal(orc.inv_rms(v, 1e-8), ref)


def test_ghost_identity_equals_sketch_dot():
    """<G_b, D o s o tau[h]> == CS(D o G_b) . tau: the identity the ghost kernel relies on."""
    rng = np.random.default_rng(4)
    B, T, d_out, d_in, k = 3, 20, 16, 24, 64
    g = rng.standard_normal((B, T, d_out))
    a = rng.standard_normal((B, T, d_in))
    h, s = orc.hash_sign_tables(d_out * d_in, 0, k)
    D = rng.uniform(0.1, 1.0, (d_out, d_in))
    tau = rng.standard_normal(k)
    phi = orc.project_full_gradient(g, a, h, s, k, diag=D)
    V = D * s.reshape(d_out, d_in) * tau[h].reshape(d_out, d_in)
    np.testing.assert_allclose(orc.ghost_score(a, g, V), phi @ tau, rtol=1e-10)
