"""Record golden vectors by running the reference OPUS implementation.

Run in a container that has the reference checkout (read-only is fine):

    python tests/golden/make_golden.py --reference <path of the reference checkout>

It imports the reference's OPUS package, runs its own functions on seeded
synthetic inputs on the CPU and writes the inputs and outputs next to this
script as .npz files.  The fixtures pin the NumPy oracle (oracle/) and the
CUDA path; nothing at test time needs the reference.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))  # tests/ for tiny_model

from tiny_model import (MuonLike, ProxyLoader, SmallGPT2, SmallQwen3, TinyLM, lora_factory,  # noqa: E402
                        state_to_numpy, zipf_tokens)


def save(name: str, **arrays) -> None:
    path = HERE / f"{name}.npz"
    np.savez_compressed(path, **{k: np.asarray(v) for k, v in arrays.items()})
    print(f"wrote {path.name} ({path.stat().st_size // 1024} KB)")


def gen_tables(rp):
    cases = [(6144, 0, 512, 42), (6144, 3, 1000, 7), (24576, 5, 16384, 42), (4608, 11, 8192, 123)]
    out = {}
    for i, (numel, pid, k, seed) in enumerate(cases):
        proj = rp.GradientProjector(sketch_dim=k, seed=seed, device="cpu", enabled=True)
        h, s = proj._get_hash_and_sign(numel, pid)
        out[f"case{i}"] = np.array([numel, pid, k, seed], dtype=np.int64)
        out[f"h{i}"] = h.numpy().astype(np.int32)
        out[f"s{i}"] = s.numpy().astype(np.int8)
    save("tables", n=np.array(len(cases)), **out)


def gen_project(rp):
    rng = np.random.default_rng(1)
    cases = [
        dict(B=3, T=40, d_out=72, d_in=48, k=512, diag=True, S=False, two_d=False, pid=1),
        dict(B=2, T=16, d_out=24, d_in=40, k=256, diag=False, S=False, two_d=False, pid=0),
        dict(B=4, T=1, d_out=40, d_in=16, k=128, diag=True, S=False, two_d=True, pid=2),
        dict(B=2, T=8, d_out=16, d_in=8, k=64, diag=False, S=True, two_d=False, pid=3),
    ]
    out = {}
    for i, c in enumerate(cases):
        shp_g = (c["B"], c["d_out"]) if c["two_d"] else (c["B"], c["T"], c["d_out"])
        shp_a = (c["B"], c["d_in"]) if c["two_d"] else (c["B"], c["T"], c["d_in"])
        g = rng.standard_normal(shp_g).astype(np.float32)
        a = rng.standard_normal(shp_a).astype(np.float32)
        diag = rng.uniform(1e-6, 1e-3, (c["d_out"], c["d_in"])).astype(np.float32) if c["diag"] else None
        S = (np.eye(c["d_out"]) + 0.1 * rng.standard_normal((c["d_out"], c["d_out"]))).astype(np.float32) \
            if c["S"] else None
        proj = rp.GradientProjector(sketch_dim=c["k"], seed=42, device="cpu", enabled=True)
        phi = proj.project_full_gradient(torch.from_numpy(g), torch.from_numpy(a), param_id=c["pid"],
                                         preconditioner_S=None if S is None else torch.from_numpy(S),
                                         diagonal_preconditioner=None if diag is None else torch.from_numpy(diag))
        out[f"meta{i}"] = np.array([c["k"], c["pid"], int(c["two_d"])], dtype=np.int64)
        out[f"g{i}"], out[f"a{i}"], out[f"phi{i}"] = g, a, phi.numpy()
        if diag is not None:
            out[f"diag{i}"] = diag
        if S is not None:
            out[f"S{i}"] = S
    save("project", n=np.array(len(cases)), **out)


def gen_select(ds):
    rng = np.random.default_rng(2)
    cases = []

    def sym(n, scale):
        m = rng.standard_normal((n, n)).astype(np.float32) * np.float32(scale)
        return ((m + m.T) / 2).astype(np.float32)

    cases.append(("random", rng.standard_normal(64).astype(np.float32), sym(64, 0.1), 16, 1.0))
    cases.append(("shift700", (800 + 5 * rng.standard_normal(48)).astype(np.float32), sym(48, 1.0), 12, 1.0))
    cases.append(("overflow_uniform", (100 + rng.standard_normal(40)).astype(np.float32), sym(40, 0.01), 8, 1.0))
    cases.append(("ties", np.ones(32, dtype=np.float32), np.zeros((32, 32), np.float32), 8, 1.0))
    cases.append(("big_pairwise", rng.standard_normal(300).astype(np.float32) * 3, sym(300, 0.05), 50, 0.5))
    cases.append(("tiny_probs", (rng.standard_normal(200) * 40).astype(np.float32), sym(200, 0.5), 30, 0.7))
    cases.append(("n512", rng.standard_normal(512).astype(np.float32), sym(512, 0.02), 64, 1.5))
    out = {}
    for i, (name, sc, sim, K, temp) in enumerate(cases):
        np.random.seed(1000 + i)
        sel = ds.stochastic_greedy_selection(sc, sim, K, temperature=temp)
        np.random.seed(1000 + i)
        uni = np.random.random_sample(K)
        gsel = ds.greedy_selection(sc, sim, K)
        out[f"name{i}"] = np.array(name)
        out[f"scores{i}"], out[f"sim{i}"] = sc, sim
        out[f"K{i}"], out[f"temp{i}"] = np.array(K), np.array(temp)
        out[f"sel{i}"] = np.array(sel, dtype=np.int64)
        out[f"uni{i}"] = uni
        out[f"greedy{i}"] = np.array(gsel, dtype=np.int64)
    # greedy with a NaN entry (np.argmax returns the first NaN)
    sc = rng.standard_normal(20).astype(np.float32)
    sc[7] = np.nan
    out["nan_scores"] = sc
    out["nan_sim"] = sym(20, 0.1)
    out["nan_greedy"] = np.array(ds.greedy_selection(sc, out["nan_sim"], 5), dtype=np.int64)
    save("select", n=np.array(len(cases)), **out)


SCENARIOS = {
    # name: (precond, projection, per_val, optimizer kind, dtype)
    "adamw_proj": ("adamw", True, False, "adamw", "f32"),
    "adamw_proj_perval": ("adamw", True, True, "adamw", "f32"),
    "adamw_noproj": ("adamw", False, False, "adamw", "f32"),
    "sgd_proj": ("sgd", True, False, "adamw", "f32"),
    "sgd_noproj": ("sgd", False, False, "adamw", "f32"),
    "muon_proj": ("muon", True, False, "muon", "f32"),
    "auto_mixed": ("auto", True, False, "mixed", "f32"),
}


# projection off with one score column per proxy, and Muon without projection (the ghost Gram
# of the factors, after the candidate dL/dZ's Muon transform); own seeds, so the fixtures above
# are unchanged when these are generated
EXTRA_SCENARIOS = {
    "adamw_noproj_perval": ("adamw", False, True, "adamw", "f32"),
    "muon_noproj": ("muon", False, False, "muon", "f32"),
}


def build_workload(rng, ref_linear, opt_kind, B=6, n=2, T=128, vocab=256):
    torch.manual_seed(0)
    model = TinyLM(ref_linear, vocab=vocab)
    cand = zipf_tokens(rng, B, T, vocab)
    prox = zipf_tokens(rng, n, T, vocab)
    gc = [m for m in model.modules() if isinstance(m, ref_linear)]
    opt_arrays = {}
    opts = []
    adam_params = [m.weight for m in gc] if opt_kind == "adamw" else [m.weight for i, m in enumerate(gc) if i % 2 == 0]
    muon_params = [m.weight for m in gc] if opt_kind == "muon" else [m.weight for i, m in enumerate(gc) if i % 2 == 1]
    if opt_kind in ("adamw", "mixed"):
        adam = torch.optim.AdamW(adam_params, lr=6e-4, betas=(0.9, 0.95), eps=1e-8)
        for j, p in enumerate(adam_params):
            v = rng.uniform(1e-6, 1e-3, tuple(p.shape)).astype(np.float32)
            adam.state[p] = {"step": torch.tensor(3.0), "exp_avg": torch.zeros_like(p),
                             "exp_avg_sq": torch.from_numpy(v)}
            opt_arrays[f"adam_v{j}"] = v
        opts.append(adam)
    if opt_kind in ("muon", "mixed"):
        muon = MuonLike(muon_params, lr=0.02, momentum=0.95)
        for j, p in enumerate(muon_params):
            m = (rng.standard_normal(tuple(p.shape)) * 1e-3).astype(np.float32)
            muon.state[p] = {"momentum_buffer": torch.from_numpy(m)}
            opt_arrays[f"muon_m{j}"] = m
        opts.append(muon)
    return model, cand, prox, opts, opt_arrays


def gen_wholepath(ds, ref_linear, scenarios=None, seed0=100):
    for si, (name, (precond, proj_on, per_val, opt_kind, _dt)) in enumerate((scenarios or SCENARIOS).items()):
        rng = np.random.default_rng(seed0 + si)
        model, cand, prox, opts, opt_arrays = build_workload(rng, ref_linear, opt_kind)
        weights = state_to_numpy(model)
        if proj_on:
            ds.initialize_projector(sketch_dim=1024, seed=42, device="cpu", enabled=True)
        else:
            ds.initialize_projector(enabled=False)
        ct, pt = torch.from_numpy(cand), torch.from_numpy(prox)
        batch_train = {"input_ids": ct, "attention_mask": torch.ones_like(ct), "labels": ct.clone()}
        loader = ProxyLoader({"input_ids": pt, "attention_mask": torch.ones_like(pt), "labels": pt.clone()})
        layers = ds.find_GClayers(model)
        scores, sim = ds.compute_GradProd_GC_per_iter(model, torch.device("cpu"), batch_train, loader,
                                                      opts if len(opts) > 1 else opts[0], layers,
                                                      preconditioner=precond, score_len=128, per_val=per_val,
                                                      return_tracin_and_similarity=True)
        save(f"wholepath_{name}", cand=cand, prox=prox, scores=scores, sim=sim,
             cfg=np.array([int(proj_on), int(per_val)]), precond=np.array(precond), opt_kind=np.array(opt_kind),
             **{f"w/{k}": v for k, v in weights.items()}, **opt_arrays)
    if scenarios is not None:
        return

    # get_batch_opus end to end: stochastic and greedy selection
    for method in ("stochastic", "greedy"):
        rng = np.random.default_rng(7)
        model, cand, prox, opts, opt_arrays = build_workload(rng, ref_linear, "adamw", B=8)
        weights = state_to_numpy(model)
        ds.initialize_projector(sketch_dim=1024, seed=42, device="cpu", enabled=True)
        ds._GBG_CALL_ID = 0
        ct, pt = torch.from_numpy(cand), torch.from_numpy(prox)
        loader = ProxyLoader({"input_ids": pt, "attention_mask": torch.ones_like(pt), "labels": pt.clone()})
        layers = ds.find_GClayers(model)
        sc, sm = ds.get_batch_opus(model, ct, ct.clone(), None, None, opts[0], layers, loader, 0.5, 128,
                                   selection_method=method, temperature=1.0, score_len=128,
                                   preconditioner="adamw", return_scores_only=True, n_windows=2)
        np.random.seed(77)
        ds._GBG_CALL_ID = 0
        idx = ds.get_batch_opus(model, ct, ct.clone(), None, None, opts[0], layers, loader, 0.5, 128,
                                selection_method=method, temperature=1.0, score_len=128, preconditioner="adamw",
                                n_windows=2)
        save(f"getbatch_{method}", cand=cand, prox=prox, scores=sc.numpy(), sim=sm.numpy(), idx=idx.numpy(),
             np_seed=np.array(77), **{f"w/{k}": v for k, v in weights.items()}, **opt_arrays)


def gen_ppl(ds, ref_linear):
    """get_batch_opus with selection_strategy="ppl": per-sequence model loss ranked high / low / mid."""
    rng = np.random.default_rng(21)
    torch.manual_seed(3)
    model = TinyLM(ref_linear, vocab=256)
    cand = zipf_tokens(rng, 10, 128, 256)
    ct = torch.from_numpy(cand)
    out = {}
    for mode in ("high", "low", "mid"):
        for ratio in (0.3, 0.9):  # mid: enough candidates near the median, and the fill path
            idx = ds.get_batch_opus(model, ct, ct.clone(), None, None, None, [], None, ratio, 128,
                                    selection_strategy="ppl", selection_method=mode, score_len=128)
            out[f"{mode}_{ratio}"] = idx.numpy()
    save("ppl", cand=cand, **out, **{f"w/{k}": v for k, v in state_to_numpy(model).items()})


def gen_gpt2_width(ds, ref_linear):
    """compute_GradProd_GC_per_iter on two GPT-2-small-wide blocks at T = 1024, k = 8192, AdamW with
    second moments 1e-4 (the GPT-2-small configuration's layer shapes; weights from the seed)."""
    rng = np.random.default_rng(31)
    torch.manual_seed(5)
    model = SmallGPT2(ref_linear)
    cand = zipf_tokens(rng, 4, 1024, 50257)
    prox = zipf_tokens(rng, 2, 1024, 50257)
    adam = torch.optim.AdamW(model.parameters(), lr=6e-4, betas=(0.9, 0.95), eps=1e-8)
    for p in model.parameters():
        adam.state[p] = {"step": torch.tensor(1.0), "exp_avg": torch.zeros_like(p),
                         "exp_avg_sq": torch.full_like(p, 1e-4)}
    ds.initialize_projector(sketch_dim=8192, seed=42, device="cpu", enabled=True)
    ct, pt = torch.from_numpy(cand), torch.from_numpy(prox)
    batch_train = {"input_ids": ct, "attention_mask": torch.ones_like(ct), "labels": ct.clone()}
    loader = ProxyLoader({"input_ids": pt, "attention_mask": torch.ones_like(pt), "labels": pt.clone()})
    scores, sim = ds.compute_GradProd_GC_per_iter(model, torch.device("cpu"), batch_train, loader, adam,
                                                  ds.find_GClayers(model), preconditioner="adamw", score_len=1024,
                                                  per_val=False, return_tracin_and_similarity=True)
    save("wholepath_gpt2width", cand=cand, prox=prox, scores=scores, sim=sim, seed=np.array(5),
         checksum=np.array(model.weight_checksum()))


def muon_state(model, ref_linear, seed: int):
    """MuonLike optimizer over the capture layers' weights, momentum buffers N(0, 1e-3) from the seed."""
    gc = [m for m in model.modules() if isinstance(m, ref_linear)]
    muon = MuonLike([m.weight for m in gc], lr=0.02, momentum=0.95)
    gen = torch.Generator().manual_seed(seed)
    for m in gc:
        muon.state[m.weight] = {"momentum_buffer": torch.randn(m.weight.shape, generator=gen) * 1e-3}
    return muon


def gen_gpt2m_muon(ds, ref_linear):
    """compute_GradProd_GC_per_iter with Muon on one GPT-2-medium-wide block (d 1024, MLP 4096),
    T = 1024, k = 32768 (the GPT-2-medium configuration's layer shapes and sketch size)."""
    rng = np.random.default_rng(41)
    torch.manual_seed(7)
    model = SmallGPT2(ref_linear, n_layer=1, d=1024, n_head=16, mlp=4096)
    cand = zipf_tokens(rng, 4, 1024, 50257)
    prox = zipf_tokens(rng, 2, 1024, 50257)
    muon = muon_state(model, ref_linear, 8)
    ds.initialize_projector(sketch_dim=32768, seed=42, device="cpu", enabled=True)
    ct, pt = torch.from_numpy(cand), torch.from_numpy(prox)
    batch_train = {"input_ids": ct, "attention_mask": torch.ones_like(ct), "labels": ct.clone()}
    loader = ProxyLoader({"input_ids": pt, "attention_mask": torch.ones_like(pt), "labels": pt.clone()})
    scores, sim = ds.compute_GradProd_GC_per_iter(model, torch.device("cpu"), batch_train, loader, muon,
                                                  ds.find_GClayers(model), preconditioner="muon", score_len=1024,
                                                  per_val=False, return_tracin_and_similarity=True)
    save("wholepath_gpt2m_muon", cand=cand, prox=prox, scores=scores, sim=sim, seed=np.array(7),
         momentum_seed=np.array(8), checksum=np.array(model.weight_checksum()))


def gen_gpt2xl_adamw(ds, ref_linear):
    """One GPT-2-XL-wide block (d 1600, MLP 6400), T = 1024, k = 65536, AdamW (v = 1e-4): the
    GPT-2-XL configuration's layer shapes and sketch size."""
    rng = np.random.default_rng(51)
    torch.manual_seed(9)
    model = SmallGPT2(ref_linear, n_layer=1, d=1600, n_head=25, mlp=6400)
    cand = zipf_tokens(rng, 4, 1024, 50257)
    prox = zipf_tokens(rng, 2, 1024, 50257)
    adam = torch.optim.AdamW(model.parameters(), lr=6e-4, betas=(0.9, 0.95), eps=1e-8)
    for p in model.parameters():
        adam.state[p] = {"step": torch.tensor(1.0), "exp_avg": torch.zeros_like(p),
                         "exp_avg_sq": torch.full_like(p, 1e-4)}
    ds.initialize_projector(sketch_dim=65536, seed=42, device="cpu", enabled=True)
    ct, pt = torch.from_numpy(cand), torch.from_numpy(prox)
    batch_train = {"input_ids": ct, "attention_mask": torch.ones_like(ct), "labels": ct.clone()}
    loader = ProxyLoader({"input_ids": pt, "attention_mask": torch.ones_like(pt), "labels": pt.clone()})
    scores, sim = ds.compute_GradProd_GC_per_iter(model, torch.device("cpu"), batch_train, loader, adam,
                                                  ds.find_GClayers(model), preconditioner="adamw", score_len=1024,
                                                  per_val=False, return_tracin_and_similarity=True)
    save("wholepath_gpt2xl_adamw", cand=cand, prox=prox, scores=scores, sim=sim, seed=np.array(9),
         checksum=np.array(model.weight_checksum()))


def gen_qwen3_muon(ds, ref_linear):
    """One Qwen3-style block (d 2048, GQA 16/8 heads of 128, SwiGLU 6144), T = 4096, vocab 151936,
    k = 131072, Muon momentum buffers from a seed: the Qwen3 configuration's shapes."""
    rng = np.random.default_rng(61)
    torch.manual_seed(11)
    model = SmallQwen3(ref_linear)
    cand = zipf_tokens(rng, 2, 4096, 151936)
    prox = zipf_tokens(rng, 1, 4096, 151936)
    muon = muon_state(model, ref_linear, 12)
    ds.initialize_projector(sketch_dim=131072, seed=42, device="cpu", enabled=True)
    ct, pt = torch.from_numpy(cand), torch.from_numpy(prox)
    batch_train = {"input_ids": ct, "attention_mask": torch.ones_like(ct), "labels": ct.clone()}
    loader = ProxyLoader({"input_ids": pt, "attention_mask": torch.ones_like(pt), "labels": pt.clone()})
    scores, sim = ds.compute_GradProd_GC_per_iter(model, torch.device("cpu"), batch_train, loader, muon,
                                                  ds.find_GClayers(model), preconditioner="muon", score_len=4096,
                                                  per_val=False, return_tracin_and_similarity=True)
    save("wholepath_qwen3_muon", cand=cand, prox=prox, scores=scores, sim=sim, seed=np.array(11),
         momentum_seed=np.array(12), checksum=np.array(model.weight_checksum()))


LORA_SCENARIOS = {"lora_proj": True, "lora_noproj": False}


def build_lora_workload(rng, ref_lora, B=6, n=2, T=128, vocab=256):
    """TinyLM whose capture layers are rank-4 LoRA linears, with nonzero B so both factors carry gradient."""
    torch.manual_seed(0)
    model = TinyLM(lora_factory(ref_lora), vocab=vocab)
    gc = [m for m in model.modules() if isinstance(m, ref_lora)]
    with torch.no_grad():
        for m in gc:
            m.lora_B.copy_(torch.from_numpy((rng.standard_normal(tuple(m.lora_B.shape)) * 0.1).astype(np.float32)))
    params = [p for m in gc for p in (m.lora_A, m.lora_B)]
    adam = torch.optim.AdamW(params, lr=6e-4, betas=(0.9, 0.95), eps=1e-8)
    opt_arrays = {}
    for j, p in enumerate(params):
        v = rng.uniform(1e-6, 1e-3, tuple(p.shape)).astype(np.float32)
        adam.state[p] = {"step": torch.tensor(3.0), "exp_avg": torch.zeros_like(p), "exp_avg_sq": torch.from_numpy(v)}
        opt_arrays[f"adam_v{j}"] = v
    cand = zipf_tokens(rng, B, T, vocab)
    prox = zipf_tokens(rng, n, T, vocab)
    return model, cand, prox, adam, opt_arrays


def gen_wholepath_lora(ds, ref_lora):
    for si, (name, proj_on) in enumerate(LORA_SCENARIOS.items()):
        rng = np.random.default_rng(300 + si)
        model, cand, prox, adam, opt_arrays = build_lora_workload(rng, ref_lora)
        weights = state_to_numpy(model)
        if proj_on:
            ds.initialize_projector(sketch_dim=1024, seed=42, device="cpu", enabled=True)
        else:
            ds.initialize_projector(enabled=False)
        ct, pt = torch.from_numpy(cand), torch.from_numpy(prox)
        batch_train = {"input_ids": ct, "attention_mask": torch.ones_like(ct), "labels": ct.clone()}
        loader = ProxyLoader({"input_ids": pt, "attention_mask": torch.ones_like(pt), "labels": pt.clone()})
        layers = ds.find_GClayers(model)
        scores, sim = ds.compute_GradProd_GC_per_iter(model, torch.device("cpu"), batch_train, loader, adam, layers,
                                                      preconditioner="adamw", score_len=128, per_val=False,
                                                      return_tracin_and_similarity=True)
        save(f"wholepath_{name}", cand=cand, prox=prox, scores=scores, sim=sim,
             cfg=np.array([int(proj_on), 0]), precond=np.array("adamw"), opt_kind=np.array("lora_adamw"),
             **{f"w/{k}": v for k, v in weights.items()}, **opt_arrays)


def gen_windows(ds):
    out = {}
    x = torch.arange(6 * 512, dtype=torch.int64).view(6, 512)
    for step in range(3):
        g = ds.make_window_generator(step=step, rank=1, device="cpu")
        w, idx = ds._random_windows(x, 128, align_to=128, g=g)
        out[f"idx{step}"] = idx.numpy()
    save("windows", **out)


def gen_layer_bf16(rp):
    """One bf16 layer scored the reference way (project_full_gradient + mean dot + Gram)."""
    rng = np.random.default_rng(5)
    B, n, T, d_out, d_in, k = 6, 3, 64, 96, 64, 2048
    g = torch.from_numpy(rng.standard_normal((B + n, T, d_out)).astype(np.float32) * 1e-3).bfloat16()
    a = torch.from_numpy(rng.standard_normal((B + n, T, d_in)).astype(np.float32)).bfloat16()
    diag = torch.from_numpy(rng.uniform(1e-6, 1e-3, (d_out, d_in)).astype(np.float32))
    proj = rp.GradientProjector(sketch_dim=k, seed=42, device="cpu", enabled=True)
    pt = proj.project_full_gradient(g[:B], a[:B], param_id=4, diagonal_preconditioner=diag)
    pv = proj.project_full_gradient(g[B:], a[B:], param_id=4)
    score = (pt @ pv.T).mean(dim=1)
    sim = pt @ pt.T
    save("layer_bf16", g=g.float().numpy(), a=a.float().numpy(), diag=diag.numpy(), B=np.array(B), k=np.array(k),
         pid=np.array(4), phi_t=pt.numpy(), score=score.numpy(), sim=sim.numpy())


def gen_muon(ds):
    """The reference's Muon S matrices for a few momentum buffers (and the identity cases)."""
    rng = np.random.default_rng(9)
    out = {}
    shapes = [(16, 24), (32, 16), (48, 48)]
    for i, shp in enumerate(shapes):
        p = torch.nn.Parameter(torch.zeros(shp))
        opt = MuonLike([p])
        m = (rng.standard_normal(shp) * 1e-3).astype(np.float32)
        opt.state[p] = {"momentum_buffer": torch.from_numpy(m)}
        S = ds._get_muon_S_matrix(p, opt)
        out[f"m{i}"], out[f"S{i}"] = m, S.float().numpy()
        out[f"C{i}"] = ds.global_C_t_muon(opt, p).numpy()
    p = torch.nn.Parameter(torch.zeros(8, 8))
    opt = MuonLike([p])
    opt.state[p] = {"momentum_buffer": torch.zeros(8, 8)}
    out["S_zero"] = ds._get_muon_S_matrix(p, opt).float().numpy()
    save("muon", n=np.array(len(shapes)), **out)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout (gszfwsb/OPUS)")
    ap.add_argument("--only", default=None, help="regenerate one fixture family (e.g. lora)")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import OPUS.train.data_selection as ds  # reference package
    import OPUS.train.random_projection as rp
    from OPUS.layers.linear import GCLinear
    from OPUS.layers.lora_layers import GCLoRALinear

    torch.set_num_threads(8)
    if args.only == "lora":
        gen_wholepath_lora(ds, GCLoRALinear)
        return 0
    if args.only == "ppl":
        gen_ppl(ds, GCLinear)
        return 0
    if args.only == "noproj_extra":
        gen_wholepath(ds, GCLinear, EXTRA_SCENARIOS, 200)
        return 0
    if args.only == "gpt2width":
        gen_gpt2_width(ds, GCLinear)
        gen_gpt2m_muon(ds, GCLinear)
        return 0
    if args.only == "gpt2xl":
        gen_gpt2xl_adamw(ds, GCLinear)
        return 0
    if args.only == "qwen3":
        gen_qwen3_muon(ds, GCLinear)
        return 0
    gen_tables(rp)
    gen_project(rp)
    gen_select(ds)
    gen_windows(ds)
    gen_layer_bf16(rp)
    gen_muon(ds)
    gen_wholepath(ds, GCLinear)
    gen_wholepath(ds, GCLinear, EXTRA_SCENARIOS, 200)
    gen_wholepath_lora(ds, GCLoRALinear)
    gen_ppl(ds, GCLinear)
    gen_gpt2_width(ds, GCLinear)
    gen_gpt2m_muon(ds, GCLinear)
    gen_gpt2xl_adamw(ds, GCLinear)
    gen_qwen3_muon(ds, GCLinear)
    return 0


if __name__ == "__main__":
    sys.exit(main())
