"""Device Boltzmann / greedy selection against the reference's selections (GPU)."""
import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import opus_oracle as orc
from opus_b200 import ops
from opus_b200.train import data_selection as ds

pytestmark = pytest.mark.gpu
DEV = "cuda"


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(DEV)


def test_boltzmann_matches_reference_golden():
    g = load_golden("select")
    for i in range(int(g["n"])):
        K = int(g[f"K{i}"])
        idx = ops.boltzmann_select(dev(g[f"scores{i}"]), dev(g[f"sim{i}"]), K, float(g[f"temp{i}"]),
                                   dev(g[f"uni{i}"]))
        ops.check_device_error("boltzmann")
        assert idx.cpu().tolist() == list(g[f"sel{i}"]), str(g[f"name{i}"])


def test_greedy_matches_reference_golden():
    g = load_golden("select")
    for i in range(int(g["n"])):
        idx = ops.greedy_select(dev(g[f"scores{i}"]), dev(g[f"sim{i}"]), int(g[f"K{i}"]))
        assert idx.cpu().tolist() == list(g[f"greedy{i}"])
    idx = ops.greedy_select(dev(g["nan_scores"]), dev(g["nan_sim"]), 5)
    assert idx.cpu().tolist() == list(g["nan_greedy"])


def test_greedy_more_picks_than_candidates():
    sc = np.array([3.0, 1.0, 2.0], np.float32)
    sim = np.zeros((3, 3), np.float32)
    got = ops.greedy_select(dev(sc), dev(sim), 5).cpu().tolist()
    assert got == orc.greedy_selection(sc, sim, 5)


@pytest.mark.parametrize("n,K,temp,spread", [(1024, 256, 1.0, 1.0), (4096, 64, 0.7, 3.0), (8192, 32, 1.5, 1.0),
                                             (257, 100, 0.5, 30.0), (129, 129, 1.0, 1.0)])
def test_boltzmann_matches_oracle_random(n, K, temp, spread):
    rng = np.random.default_rng(n + K)
    sc = (rng.standard_normal(n) * spread).astype(np.float32)
    m = rng.standard_normal((n, n)).astype(np.float32) * np.float32(0.01)
    sim = ((m + m.T) / 2).astype(np.float32)
    uni = rng.random(K)
    want = orc.stochastic_greedy_selection(sc, sim, K, temperature=temp, uniforms=uni)
    got = ops.boltzmann_select(dev(sc), dev(sim), K, temp, dev(uni)).cpu().tolist()
    ops.check_device_error("boltzmann")
    assert got == want


def test_public_stochastic_selection_uses_numpy_stream():
    g = load_golden("select")
    np.random.seed(1000)
    sel = ds.stochastic_greedy_selection(g["scores0"], g["sim0"], int(g["K0"]), temperature=float(g["temp0"]))
    assert [int(x) for x in sel] == list(g["sel0"])
    assert ds.greedy_selection(g["scores1"], g["sim1"], int(g["K1"])) == list(g["greedy1"])


def test_stochastic_selection_too_many_picks():
    with pytest.raises(ValueError):
        ds.stochastic_greedy_selection(np.zeros(3, np.float32), np.zeros((3, 3), np.float32), 4)
