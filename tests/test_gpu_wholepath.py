"""The drop-in API on the GPU reproduces the reference's scores, similarity and picks."""
import numpy as np
import pytest
import torch

from conftest import load_golden
from opus_b200.train import data_selection as ds
from test_host_logic import LORA_SCENARIOS, SCENARIOS, assert_close_scores, rebuild, rebuild_lora

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("name", SCENARIOS)
def test_compute_scores_match_reference(name):
    g = load_golden(f"wholepath_{name}")
    proj_on, per_val = (bool(x) for x in g["cfg"])
    model, opt, loader, batch = rebuild(g, device=DEV)
    if proj_on:
        # tables from the CPU generator, as in the recorded reference run
        ds.initialize_projector(sketch_dim=1024, seed=42, device="cpu", enabled=True)
    else:
        ds.initialize_projector(enabled=False)
    scores, sim = ds.compute_GradProd_GC_per_iter(model, torch.device(DEV), batch, loader, opt,
                                                  ds.find_GClayers(model), preconditioner=str(g["precond"]),
                                                  score_len=128, per_val=per_val)
    assert isinstance(scores, np.ndarray) and scores.dtype == np.float32
    assert_close_scores(scores, g["scores"])
    assert_close_scores(sim, g["sim"])


@pytest.mark.parametrize("name", LORA_SCENARIOS)
def test_lora_scores_match_reference(name):
    """GCLoRALinear layers through the device path: rank-4 factors padded to the kernels' widths."""
    g = load_golden(f"wholepath_{name}")
    model, opt, loader, batch = rebuild_lora(g, device=DEV)
    if bool(g["cfg"][0]):
        ds.initialize_projector(sketch_dim=1024, seed=42, device="cpu", enabled=True)
    else:
        ds.initialize_projector(enabled=False)
    scores, sim = ds.compute_GradProd_GC_per_iter(model, torch.device(DEV), batch, loader, opt,
                                                  ds.find_GClayers(model), preconditioner="adamw", score_len=128)
    assert_close_scores(scores, g["scores"])
    assert_close_scores(sim, g["sim"])


@pytest.mark.parametrize("method", ["stochastic", "greedy"])
def test_get_batch_opus_matches_reference(method):
    g = load_golden(f"getbatch_{method}")
    model, opt, loader, _ = rebuild(g, device=DEV)
    ds.initialize_projector(sketch_dim=1024, seed=42, device="cpu", enabled=True)
    cand = torch.from_numpy(g["cand"]).to(DEV)
    layers = ds.find_GClayers(model)
    ds._GBG_CALL_ID = 0
    sc, sm = ds.get_batch_opus(model, cand, cand.clone(), None, None, opt, layers, loader, 0.5, 128,
                               selection_method=method, temperature=1.0, score_len=128, preconditioner="adamw",
                               return_scores_only=True, n_windows=2)
    assert sc.device.type == "cuda"
    assert_close_scores(sc.cpu().numpy(), g["scores"])
    assert_close_scores(sm.cpu().numpy(), g["sim"])
    np.random.seed(int(g["np_seed"]))
    ds._GBG_CALL_ID = 0
    idx = ds.get_batch_opus(model, cand, cand.clone(), None, None, opt, layers, loader, 0.5, 128,
                            selection_method=method, temperature=1.0, score_len=128, preconditioner="adamw",
                            n_windows=2)
    assert idx.dtype == torch.int64 and idx.device.type == "cuda"
    assert idx.cpu().tolist() == list(g["idx"])
