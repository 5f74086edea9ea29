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


def _scores_both_modes(model, opt, loader, batch, layers, precond="adamw"):
    out = {}
    for mode in ("batch", "stream"):
        ds.CAPTURE_MODE = mode
        try:
            out[mode] = ds.compute_GradProd_GC_per_iter(model, torch.device(DEV), dict(batch), loader, opt, layers,
                                                        preconditioner=precond, score_len=128)
        finally:
            ds.CAPTURE_MODE = "stream"
    return out


@pytest.mark.parametrize("name", ["adamw_proj", "muon_proj", "auto_mixed", "adamw_noproj"])
def test_streaming_capture_equals_batch_capture(name):
    """Scoring from backward hooks (each dL/dZ used as it appears) == one autograd call for every layer."""
    g = load_golden(f"wholepath_{name}")
    model, opt, loader, batch = rebuild(g, device=DEV)
    if bool(g["cfg"][0]):
        ds.initialize_projector(sketch_dim=1024, seed=42, device="cpu", enabled=True)
    else:
        ds.initialize_projector(enabled=False)
    out = _scores_both_modes(model, opt, loader, batch, ds.find_GClayers(model), str(g["precond"]))
    assert_close_scores(out["stream"][0], out["batch"][0], rtol=1e-5)
    assert_close_scores(out["stream"][1], out["batch"][1], rtol=1e-5)
    assert_close_scores(out["stream"][0], g["scores"])


def test_streaming_capture_falls_back_without_a_root():
    """A frozen embedding leaves the first layer's input without grad: the batch capture takes over."""
    g = load_golden("wholepath_adamw_proj")
    model, opt, loader, batch = rebuild(g, device=DEV)
    model.embed.weight.requires_grad_(False)
    ds.initialize_projector(sketch_dim=1024, seed=42, device="cpu", enabled=True)
    out = _scores_both_modes(model, opt, loader, batch, ds.find_GClayers(model))
    np.testing.assert_array_equal(out["stream"][0], out["batch"][0])


def test_streaming_capture_lowers_peak_memory():
    """No layer's dL/dZ outlives its hook: the capture's peak device memory drops."""
    from opus_b200.layers import GCLinear
    from tiny_model import ProxyLoader, TinyLM

    torch.manual_seed(0)
    model = TinyLM(GCLinear, vocab=512, d=256, hidden=2048, n_layers=6).to(DEV)
    layers = ds.find_GClayers(model)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3, betas=(0.9, 0.95))
    cand = torch.randint(0, 512, (24, 256), device=DEV)
    prox = torch.randint(0, 512, (4, 256), device=DEV)
    loader = ProxyLoader({"input_ids": prox, "attention_mask": torch.ones_like(prox), "labels": prox.clone()})
    batch = {"input_ids": cand, "attention_mask": torch.ones_like(cand), "labels": cand.clone()}
    ds.initialize_projector(sketch_dim=4096, seed=42, device="cuda", enabled=True)
    peaks = {}
    for mode in ("batch", "stream", "batch", "stream"):
        ds.CAPTURE_MODE = mode
        try:
            torch.cuda.synchronize()
            torch.cuda.reset_peak_memory_stats()
            base = torch.cuda.memory_allocated()
            ds.compute_GradProd_GC_per_iter(model, torch.device(DEV), dict(batch), loader, opt, layers,
                                            preconditioner="adamw", score_len=256)
            torch.cuda.synchronize()
            peaks[mode] = torch.cuda.max_memory_allocated() - base
        finally:
            ds.CAPTURE_MODE = "stream"
    assert peaks["stream"] < peaks["batch"], peaks


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("V", [50257, 50304])
def test_chunked_token_loss_bit_identical_on_gpu(dtype, V, monkeypatch):
    """GPT-2 vocabularies (odd and 16-byte-aligned rows): values equal the reference's on CUDA too."""
    from test_host_logic import token_loss_pair
    torch.manual_seed(0)
    N, T = 6, 257
    logits = (torch.randn(N, T, V, device=DEV) * 4).to(dtype)
    labels = torch.randint(0, V, (N, T), device=DEV)
    labels[2, 100:140] = -100
    chunk = 2 * T * V * logits.element_size()  # three chunks of two samples
    ref_l, ref_g, l, g = token_loss_pair(logits, labels, chunk, monkeypatch)
    assert torch.equal(ref_l, l) and torch.equal(ref_g, g)


def test_chunked_token_loss_lowers_peak_memory(monkeypatch):
    """Forward + backward peak above the logits: about one gradient-sized buffer instead of several."""
    torch.manual_seed(0)
    N, T, V = 8, 512, 50304
    logits = torch.randn(N, T, V, device=DEV)
    labels = torch.randint(0, V, (N, T), device=DEV)
    size = logits.numel() * logits.element_size()
    monkeypatch.setattr(ds, "TOKEN_LOSS_CHUNK_BYTES", size // 8)
    peaks = []
    for f in (__import__("test_host_logic")._reference_token_loss, ds.per_sample_token_loss):
        x = logits.clone().requires_grad_()
        torch.cuda.synchronize()
        torch.cuda.reset_peak_memory_stats()
        base = torch.cuda.memory_allocated()
        f(x, labels).mean().backward()
        torch.cuda.synchronize()
        peaks.append((torch.cuda.max_memory_allocated() - base) / size)
        del x
    assert peaks[1] < 1.6 and peaks[0] > peaks[1] + 1.0, peaks


def test_gpt2_width_scores_match_reference():
    """Two GPT-2-small-wide blocks at T = 1024, vocab 50257, k = 8192, AdamW (v = 1e-4): the
    configuration's layer shapes, scores and similarity against the reference's."""
    from opus_b200.layers import GCLinear
    from tiny_model import ProxyLoader, SmallGPT2

    g = load_golden("wholepath_gpt2width")
    torch.manual_seed(int(g["seed"]))
    model = SmallGPT2(GCLinear)
    # the reference run's weights (float64 sums: the order follows the host CPU's vector width)
    assert abs(model.weight_checksum() - float(g["checksum"])) <= 1e-12 * abs(float(g["checksum"]))
    model.to(DEV)
    adam = torch.optim.AdamW(model.parameters(), lr=6e-4, betas=(0.9, 0.95), eps=1e-8)
    for p in model.parameters():
        adam.state[p] = {"step": torch.tensor(1.0), "exp_avg": torch.zeros_like(p),
                         "exp_avg_sq": torch.full_like(p, 1e-4)}
    ds.initialize_projector(sketch_dim=8192, seed=42, device="cpu", enabled=True)
    cand, prox = torch.from_numpy(g["cand"]).to(DEV), torch.from_numpy(g["prox"]).to(DEV)
    batch = {"input_ids": cand, "attention_mask": torch.ones_like(cand), "labels": cand.clone()}
    loader = ProxyLoader({"input_ids": prox, "attention_mask": torch.ones_like(prox), "labels": prox.clone()})
    scores, sim = ds.compute_GradProd_GC_per_iter(model, torch.device(DEV), batch, loader, adam,
                                                  ds.find_GClayers(model), preconditioner="adamw", score_len=1024)
    assert_close_scores(scores, g["scores"])
    assert_close_scores(sim, g["sim"])


def test_gpt2m_muon_scores_match_reference():
    """One GPT-2-medium-wide block (d 1024, MLP 4096) at T = 1024, k = 32768, Muon momentum
    buffers from a seed: the Muon configuration's layer shapes against the reference."""
    from opus_b200.layers import GCLinear
    from tiny_model import MuonLike, ProxyLoader, SmallGPT2

    g = load_golden("wholepath_gpt2m_muon")
    torch.manual_seed(int(g["seed"]))
    model = SmallGPT2(GCLinear, n_layer=1, d=1024, n_head=16, mlp=4096)
    assert abs(model.weight_checksum() - float(g["checksum"])) <= 1e-12 * abs(float(g["checksum"]))
    gc = [m for m in model.modules() if isinstance(m, GCLinear)]
    muon = MuonLike([m.weight for m in gc], lr=0.02, momentum=0.95)
    gen = torch.Generator().manual_seed(int(g["momentum_seed"]))
    buffers = [torch.randn(m.weight.shape, generator=gen) * 1e-3 for m in gc]
    model.to(DEV)
    for m, buf in zip(gc, buffers):
        muon.state[m.weight] = {"momentum_buffer": buf.to(DEV)}
    ds.initialize_projector(sketch_dim=32768, seed=42, device="cpu", enabled=True)
    cand, prox = torch.from_numpy(g["cand"]).to(DEV), torch.from_numpy(g["prox"]).to(DEV)
    batch = {"input_ids": cand, "attention_mask": torch.ones_like(cand), "labels": cand.clone()}
    loader = ProxyLoader({"input_ids": prox, "attention_mask": torch.ones_like(prox), "labels": prox.clone()})
    scores, sim = ds.compute_GradProd_GC_per_iter(model, torch.device(DEV), batch, loader, muon,
                                                  ds.find_GClayers(model), preconditioner="muon", score_len=1024)
    assert_close_scores(scores, g["scores"])
    assert_close_scores(sim, g["sim"])


def _muon_for(model, seed):
    from opus_b200.layers import GCLinear
    from tiny_model import MuonLike

    gc = [m for m in model.modules() if isinstance(m, GCLinear)]
    muon = MuonLike([m.weight for m in gc], lr=0.02, momentum=0.95)
    gen = torch.Generator().manual_seed(seed)
    buffers = [torch.randn(m.weight.shape, generator=gen) * 1e-3 for m in gc]
    return muon, list(zip(gc, buffers))


def _scores_on_gpu(model, g, opt, precond, k, score_len):
    from tiny_model import ProxyLoader

    ds.initialize_projector(sketch_dim=k, seed=42, device="cpu", enabled=True)
    cand, prox = torch.from_numpy(g["cand"]).to(DEV), torch.from_numpy(g["prox"]).to(DEV)
    batch = {"input_ids": cand, "attention_mask": torch.ones_like(cand), "labels": cand.clone()}
    loader = ProxyLoader({"input_ids": prox, "attention_mask": torch.ones_like(prox), "labels": prox.clone()})
    return ds.compute_GradProd_GC_per_iter(model, torch.device(DEV), batch, loader, opt, ds.find_GClayers(model),
                                           preconditioner=precond, score_len=score_len)


def test_gpt2xl_adamw_scores_match_reference():
    """One GPT-2-XL-wide block (d 1600, MLP 6400), T = 1024, k = 65536 (a shared-memory sketch of
    the first 32768 buckets, L2 atomics above), AdamW: against the reference."""
    from opus_b200.layers import GCLinear
    from tiny_model import SmallGPT2

    g = load_golden("wholepath_gpt2xl_adamw")
    torch.manual_seed(int(g["seed"]))
    model = SmallGPT2(GCLinear, n_layer=1, d=1600, n_head=25, mlp=6400)
    assert abs(model.weight_checksum() - float(g["checksum"])) <= 1e-12 * abs(float(g["checksum"]))
    model.to(DEV)
    adam = torch.optim.AdamW(model.parameters(), lr=6e-4, betas=(0.9, 0.95), eps=1e-8)
    for p in model.parameters():
        adam.state[p] = {"step": torch.tensor(1.0), "exp_avg": torch.zeros_like(p),
                         "exp_avg_sq": torch.full_like(p, 1e-4)}
    scores, sim = _scores_on_gpu(model, g, adam, "adamw", 65536, 1024)
    assert_close_scores(scores, g["scores"])
    assert_close_scores(sim, g["sim"])


def test_qwen3_muon_scores_match_reference():
    """One Qwen3-style block (d 2048, GQA 16/8 x 128, SwiGLU 6144, 7 capture layers), T = 4096,
    vocab 151936, k = 131072, Muon: the Qwen3 configuration's shapes against the reference."""
    from opus_b200.layers import GCLinear
    from tiny_model import SmallQwen3

    g = load_golden("wholepath_qwen3_muon")
    torch.manual_seed(int(g["seed"]))
    model = SmallQwen3(GCLinear)
    assert abs(model.weight_checksum() - float(g["checksum"])) <= 1e-12 * abs(float(g["checksum"]))
    muon, buffers = _muon_for(model, int(g["momentum_seed"]))
    model.to(DEV)
    for m, buf in buffers:
        muon.state[m.weight] = {"momentum_buffer": buf.to(DEV)}
    scores, sim = _scores_on_gpu(model, g, muon, "muon", 131072, 4096)
    assert_close_scores(scores, g["scores"])
    assert_close_scores(sim, g["sim"])


@pytest.mark.parametrize("name", ["adamw_proj", "muon_proj", "lora_proj"])
@pytest.mark.parametrize("exact", [False, True])
def test_score_shard_streams_like_batch_capture(name, exact, monkeypatch):
    """The sharded scorer at world size 1: streaming hooks == one autograd call == the reference."""
    from opus_b200.train import distributed as sd

    g = load_golden(f"wholepath_{name}")
    model, opt, loader, batch = (rebuild_lora if name.startswith("lora") else rebuild)(g, device=DEV)
    ds.initialize_projector(sketch_dim=1024, seed=42, device="cpu", enabled=True)
    proxy = loader._fixed_batch
    n = proxy["input_ids"].shape[0]
    out = {}
    for mode in ("stream", "batch"):
        monkeypatch.setattr(ds, "CAPTURE_MODE", mode)
        out[mode] = sd.score_shard(model, torch.device(DEV), dict(batch), dict(proxy), n, opt,
                                   ds.find_GClayers(model), preconditioner=str(g["precond"]), score_len=128,
                                   exact_similarity=exact)
    for mode in ("stream", "batch"):
        assert_close_scores(out[mode][0].cpu().numpy(), g["scores"])
        assert_close_scores(out[mode][1].cpu().numpy(), g["sim"])


@pytest.mark.parametrize("name,rows", [("adamw_proj", 2), ("adamw_proj_perval", 3), ("muon_proj", 4),
                                       ("auto_mixed", 1), ("sgd_proj", 5)])
def test_capture_in_passes_matches_reference(name, rows, monkeypatch):
    """Candidates and proxies captured a few rows per forward/backward give the reference's whole-batch values."""
    g = load_golden(f"wholepath_{name}")
    per_val = bool(g["cfg"][1])
    model, opt, loader, batch = rebuild(g, device=DEV)
    ds.initialize_projector(sketch_dim=1024, seed=42, device="cpu", enabled=True)
    monkeypatch.setattr(ds, "CAPTURE_ROWS", rows)
    assert ds._use_passes(batch["input_ids"].shape[0] + 2, ds.find_GClayers(model), 128, torch.device(DEV))
    scores, sim = ds.compute_GradProd_GC_per_iter(model, torch.device(DEV), batch, loader, opt,
                                                  ds.find_GClayers(model), preconditioner=str(g["precond"]),
                                                  score_len=128, per_val=per_val)
    assert_close_scores(scores, g["scores"])
    assert_close_scores(sim, g["sim"])


def test_get_batch_opus_in_passes_matches_reference(monkeypatch):
    """The public call with the capture split into passes: the reference's scores and picks."""
    g = load_golden("getbatch_stochastic")
    model, opt, loader, _ = rebuild(g, device=DEV)
    ds.initialize_projector(sketch_dim=1024, seed=42, device="cpu", enabled=True)
    monkeypatch.setattr(ds, "CAPTURE_ROWS", 3)
    cand = torch.from_numpy(g["cand"]).to(DEV)
    layers = ds.find_GClayers(model)
    ds._GBG_CALL_ID = 0
    sc, sm = ds.get_batch_opus(model, cand, cand.clone(), None, None, opt, layers, loader, 0.5, 128,
                               selection_method="stochastic", temperature=1.0, score_len=128,
                               preconditioner="adamw", return_scores_only=True, n_windows=2)
    assert_close_scores(sc.cpu().numpy(), g["scores"])
    assert_close_scores(sm.cpu().numpy(), g["sim"])
    np.random.seed(int(g["np_seed"]))
    ds._GBG_CALL_ID = 0
    idx = ds.get_batch_opus(model, cand, cand.clone(), None, None, opt, layers, loader, 0.5, 128,
                            selection_method="stochastic", temperature=1.0, score_len=128, preconditioner="adamw",
                            n_windows=2)
    assert idx.cpu().tolist() == list(g["idx"])


def test_score_shard_in_passes_matches_single_pass(monkeypatch):
    """World size 1: the sharded scorer with its capture split into passes equals the single-pass scorer."""
    from opus_b200.train import distributed as sd

    g = load_golden("wholepath_muon_proj")
    model, opt, loader, batch = rebuild(g, device=DEV)
    ds.initialize_projector(sketch_dim=1024, seed=42, device="cpu", enabled=True)
    proxy = loader._fixed_batch
    layers = ds.find_GClayers(model)
    n = proxy["input_ids"].shape[0]
    one = sd.score_shard(model, torch.device(DEV), dict(batch), proxy, n, opt, layers, preconditioner="muon",
                         score_len=128)
    monkeypatch.setattr(ds, "CAPTURE_ROWS", 2)
    split = sd.score_shard(model, torch.device(DEV), dict(batch), proxy, n, opt, layers, preconditioner="muon",
                           score_len=128)
    assert_close_scores(split[0].cpu().numpy(), one[0].cpu().numpy(), rtol=1e-4)
    assert_close_scores(split[1].cpu().numpy(), one[1].cpu().numpy(), rtol=1e-4)
    assert_close_scores(split[0].cpu().numpy(), g["scores"])


@pytest.mark.parametrize("name", ["adamw_proj", "muon_proj"])
def test_folded_row_scale_equals_scaled_dldz(name, monkeypatch):
    """A round in passes with dL/dZ's per-sample factor applied by the sketch kernel (the default)
    gives the values of the same round with the layer's own dL/dZ * N tensors."""
    g = load_golden(f"wholepath_{name}")
    model, opt, loader, batch = rebuild(g, device=DEV)
    ds.initialize_projector(sketch_dim=1024, seed=42, device="cpu", enabled=True)
    monkeypatch.setattr(ds, "CAPTURE_ROWS", 2)
    layers = ds.find_GClayers(model)
    args = (model, torch.device(DEV), batch, loader, opt, layers)
    kw = dict(preconditioner=str(g["precond"]), score_len=128)
    calls = []
    real = ds._layer_pairs

    def spy(layer, zg, train_bs, fold_scale=False):
        out = real(layer, zg, train_bs, fold_scale)
        calls.append(out[0].scale)
        return out

    monkeypatch.setattr(ds, "_layer_pairs", spy)
    folded = ds.compute_GradProd_GC_per_iter(*args, **kw)
    assert calls and all(s == 2.0 for s in calls)  # every GCLinear pair left its factor to the kernel
    monkeypatch.setattr(ds, "_layer_pairs", lambda layer, zg, train_bs, fold_scale=False: real(layer, zg, train_bs))
    scaled = ds.compute_GradProd_GC_per_iter(*args, **kw)
    assert_close_scores(folded[0], scaled[0])
    assert_close_scores(folded[1], scaled[1])
