"""Host-side logic of the drop-in package on CPU: capture, preconditioner plans,
proxy plumbing, windows and argument checks; whole-path scores via the oracle."""
import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import opus_oracle as orc
from opus_b200.layers import GCLinear, GCLoRALinear, LoRALinear
from opus_b200.train import data_selection as ds
from tiny_model import MuonLike, ProxyLoader, TinyLM, load_numpy_state, lora_factory

SCENARIOS = ["adamw_proj", "adamw_proj_perval", "adamw_noproj", "adamw_noproj_perval", "sgd_proj", "sgd_noproj",
             "muon_proj", "muon_noproj", "auto_mixed"]


def rebuild(g, device="cpu"):
    """TinyLM with this package's GCLinear, weights and optimizer state from a fixture."""
    model = TinyLM(GCLinear)
    load_numpy_state(model, g)
    model.to(device)
    gc = [m for m in model.modules() if isinstance(m, GCLinear)]
    kind = str(g.get("opt_kind", np.array("adamw")))
    opts = []
    adam_params = [m.weight for m in gc] if kind == "adamw" else [m.weight for i, m in enumerate(gc) if i % 2 == 0]
    muon_params = [m.weight for m in gc] if kind == "muon" else [m.weight for i, m in enumerate(gc) if i % 2 == 1]
    if kind in ("adamw", "mixed"):
        adam = torch.optim.AdamW(adam_params, lr=6e-4, betas=(0.9, 0.95), eps=1e-8)
        for j, p in enumerate(adam_params):
            adam.state[p] = {"step": torch.tensor(3.0), "exp_avg": torch.zeros_like(p),
                             "exp_avg_sq": torch.from_numpy(g[f"adam_v{j}"]).to(device)}
        opts.append(adam)
    if kind in ("muon", "mixed"):
        muon = MuonLike(muon_params, lr=0.02, momentum=0.95)
        for j, p in enumerate(muon_params):
            muon.state[p] = {"momentum_buffer": torch.from_numpy(g[f"muon_m{j}"]).to(device)}
        opts.append(muon)
    cand = torch.from_numpy(g["cand"]).to(device)
    prox = torch.from_numpy(g["prox"]).to(device)
    loader = ProxyLoader({"input_ids": prox, "attention_mask": torch.ones_like(prox), "labels": prox.clone()})
    batch = {"input_ids": cand, "attention_mask": torch.ones_like(cand), "labels": cand.clone()}
    return model, (opts if len(opts) > 1 else opts[0]), loader, batch


LORA_SCENARIOS = ["lora_proj", "lora_noproj"]


def rebuild_lora(g, device="cpu"):
    """TinyLM with this package's rank-4 GCLoRALinear layers, weights and AdamW state from a fixture."""
    model = TinyLM(lora_factory(GCLoRALinear))
    load_numpy_state(model, g)
    model.to(device)
    gc = [m for m in model.modules() if isinstance(m, GCLoRALinear)]
    params = [p for m in gc for p in (m.lora_A, m.lora_B)]
    adam = torch.optim.AdamW(params, lr=6e-4, betas=(0.9, 0.95), eps=1e-8)
    for j, p in enumerate(params):
        adam.state[p] = {"step": torch.tensor(3.0), "exp_avg": torch.zeros_like(p),
                         "exp_avg_sq": torch.from_numpy(g[f"adam_v{j}"]).to(device)}
    cand = torch.from_numpy(g["cand"]).to(device)
    prox = torch.from_numpy(g["prox"]).to(device)
    loader = ProxyLoader({"input_ids": prox, "attention_mask": torch.ones_like(prox), "labels": prox.clone()})
    batch = {"input_ids": cand, "attention_mask": torch.ones_like(cand), "labels": cand.clone()}
    return model, adam, loader, batch


def assert_close_scores(got, want, rtol=1e-3):
    """Every score / similarity element within rtol of its own reference value.

    The north star's 1e-3 relative error holds per element.  Only an element
    whose reference value is exactly zero (relative error undefined) gets an
    absolute bound instead: rtol * 1e-6 of the largest reference value.
    """
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    assert got.shape == want.shape, (got.shape, want.shape)
    err = np.abs(got - want)
    zero = want == 0
    bound = np.where(zero, rtol * 1e-6 * np.abs(want).max(), rtol * np.abs(want))
    bad = ~(err <= bound)
    if bad.any():
        i = np.unravel_index(int(np.argmax(np.where(bad, err / np.maximum(bound, 1e-300), 0))), want.shape)
        raise AssertionError(f"{int(bad.sum())} of {want.size} elements outside rtol={rtol}; worst at {i}: "
                             f"got {got[i]!r}, want {want[i]!r} (relative {err[i] / max(abs(want[i]), 1e-300):.3e})")


@pytest.fixture(autouse=True)
def _reference_muon_on_cpu(monkeypatch):
    """plan_layers runs on the CPU here: the Muon S and transform come from the reference's own torch recipe
    (oracle/reference_torch.py); the tcgen05 kernels that replace them need a GPU and have GPU tests."""
    from opus_b200 import ops
    from oracle import reference_torch as rt

    monkeypatch.setattr(ops, "muon_S", rt.muon_S)
    monkeypatch.setattr(ops, "muon_transform", rt.muon_transform)


@pytest.mark.parametrize("name", SCENARIOS)
def test_wholepath_oracle_matches_reference(name):
    g = load_golden(f"wholepath_{name}")
    proj_on, per_val = (bool(x) for x in g["cfg"])
    model, opt, loader, batch = rebuild(g)
    layers = ds.find_GClayers(model)
    pairs, B, n = ds.capture_pairs(model, batch, loader, layers, score_len=128)
    plans = ds.plan_layers(pairs, opt, str(g["precond"]), "cpu")
    score = np.zeros((B, n) if per_val else B)
    sim = np.zeros((B, B))
    for pl in plans:
        d_out, d_in = pl.g_t.shape[-1], pl.a_t.shape[-1]
        h, s = orc.hash_sign_tables(d_out * d_in, pl.pid, 1024, seed=42)
        diag = None if pl.exp_avg_sq is None else orc.inv_rms(pl.exp_avg_sq.numpy(), pl.eps)
        sc, sm = orc.layer_scores(pl.g_t.float().numpy(), pl.a_t.numpy(), pl.g_v.numpy(), pl.a_v.numpy(), h, s,
                                  1024, C=pl.c, diag=diag, per_val=per_val, projection=proj_on)
        score += sc
        sim += sm
    assert_close_scores(score, g["scores"])
    assert_close_scores(sim, g["sim"])


@pytest.mark.parametrize("name", LORA_SCENARIOS)
def test_wholepath_lora_oracle_matches_reference(name):
    """LoRA layers: two (dL/dZ, A) pairs per layer, AdamW state on lora_A and lora_B."""
    g = load_golden(f"wholepath_{name}")
    proj_on = bool(g["cfg"][0])
    model, opt, loader, batch = rebuild_lora(g)
    layers = ds.find_GClayers(model)
    pairs, B, n = ds.capture_pairs(model, batch, loader, layers, score_len=128)
    assert len(pairs) == 2 * len(layers)
    plans = ds.plan_layers(pairs, opt, "adamw", "cpu")
    score, sim = np.zeros(B), np.zeros((B, B))
    for pl in plans:
        d_out, d_in = pl.g_t.shape[-1], pl.a_t.shape[-1]
        h, s = orc.hash_sign_tables(d_out * d_in, pl.pid, 1024, seed=42)
        diag = None if pl.exp_avg_sq is None else orc.inv_rms(pl.exp_avg_sq.numpy(), pl.eps)
        sc, sm = orc.layer_scores(pl.g_t.float().numpy(), pl.a_t.numpy(), pl.g_v.numpy(), pl.a_v.numpy(), h, s,
                                  1024, C=pl.c, diag=diag, projection=proj_on)
        score += sc
        sim += sm
    assert_close_scores(score, g["scores"])
    assert_close_scores(sim, g["sim"])


@pytest.mark.parametrize("method", ["stochastic", "greedy"])
def test_get_batch_selection_oracle(method):
    g = load_golden(f"getbatch_{method}")
    np.random.seed(int(g["np_seed"]))
    if method == "stochastic":
        idx = orc.stochastic_greedy_selection(g["scores"], g["sim"], 4, temperature=1.0)
    else:
        idx = orc.greedy_selection(g["scores"], g["sim"], 4)
    assert idx == list(g["idx"])


def test_random_windows_match_reference():
    g = load_golden("windows")
    x = torch.arange(6 * 512, dtype=torch.int64).view(6, 512)
    for step in range(3):
        gen = ds.make_window_generator(step=step, rank=1, device="cpu")
        _, idx = ds._random_windows(x, 128, align_to=128, g=gen)
        np.testing.assert_array_equal(idx.numpy(), g[f"idx{step}"])


def test_windows_identity_when_short():
    x = torch.arange(2 * 128).view(2, 128)
    w, idx = ds._random_windows(x, 256)
    assert torch.equal(w, x) and idx.shape == (2, 128)


def test_group_kind_and_scalars():
    assert ds._group_kind({"betas": (0.9, 0.95)}) == "adamw"
    assert ds._group_kind({"momentum": 0.95}) == "muon"
    assert ds._group_kind({"lr": 1.0}) == "unknown"
    p = torch.nn.Parameter(torch.zeros(64, 32))
    adam = torch.optim.AdamW([p], lr=3e-4, betas=(0.8, 0.95))
    adam.state[p] = {"step": torch.tensor(7.0)}
    assert float(ds.global_C_t(adam, p)) == float(orc.adamw_scale(3e-4, 0.8, 0.95, 7))
    muon = MuonLike([p], lr=0.05, momentum=0.9)
    assert float(ds.global_C_t_muon(muon, p)) == float(orc.muon_scale(0.05, 64, 32, 0.9))
    assert ds._get_step_from_optimizer(torch.optim.AdamW([torch.nn.Parameter(torch.zeros(2))])) == 1


def test_find_group_falls_back_to_first():
    p, q = torch.nn.Parameter(torch.zeros(2)), torch.nn.Parameter(torch.zeros(2))
    opt = torch.optim.SGD([{"params": [p], "lr": 1.0}, {"params": [q], "lr": 2.0}])
    assert ds._find_group_for_param(opt, q)["lr"] == 2.0
    assert ds._find_group_for_param(opt, torch.nn.Parameter(torch.zeros(2)))["lr"] == 1.0


class _Loader:
    def __init__(self, n):
        self.n = n

    def __iter__(self):
        return iter([{"input_ids": torch.full((1, 4), i)} for i in range(self.n)])


def test_proxy_batch_modes():
    ld = _Loader(3)
    firsts = [int(ds._sample_proxy_batch_for_step(ld)["input_ids"][0, 0]) for _ in range(4)]
    assert firsts == [0, 1, 2, 0]  # refresh every call, wraps around
    ld = _Loader(3)
    ld._proxy_refresh_interval = 2
    firsts = [int(ds._sample_proxy_batch_for_step(ld)["input_ids"][0, 0]) for _ in range(4)]
    assert firsts == [0, 0, 1, 1]
    ld = _Loader(3)
    ld._proxy_mode = "fixed"
    assert [int(ds._sample_proxy_batch_for_step(ld)["input_ids"][0, 0]) for _ in range(3)] == [0, 0, 0]
    ld._fixed_batch = {"input_ids": torch.full((1, 4), 9)}
    b = ds._sample_proxy_batch_for_step(ld)
    assert int(b["input_ids"][0, 0]) == 9
    b["input_ids"] = None  # a copy: the pinned batch is untouched
    assert ld._fixed_batch["input_ids"] is not None


def test_get_batch_opus_argument_checks():
    model = TinyLM(GCLinear)
    seq = torch.zeros(4, 128, dtype=torch.long)
    with pytest.raises(AssertionError):
        ds.get_batch_opus(model, seq, seq, None, None, None, [], None, 0.5, 128, score_len=100)
    with pytest.raises(ValueError):
        ds.get_batch_opus(model, torch.zeros(3, 100, dtype=torch.long), seq, None, None, None, [], None, 0.5, 128,
                          score_len=128)
    with pytest.raises(ValueError):
        ds.get_batch_opus(model, torch.zeros(10, dtype=torch.long), seq, None, None, None, [], None, 0.5, 128,
                          score_len=128)
    with pytest.raises(ValueError):
        ds.get_batch_opus(model, seq, seq, None, None, None, [], None, 0.5, 128, score_len=128,
                          selection_strategy="bogus")
    idx = ds.get_batch_opus(model, seq.view(-1), seq.view(-1), None, None, None, [], None, 0.5, 128,
                            score_len=128, selection_strategy="random")
    assert idx.shape == (2,) and len(set(idx.tolist())) == 2


def test_capture_requires_gc_layers():
    model = TinyLM(GCLinear)
    seq = torch.zeros(2, 128, dtype=torch.long)
    loader = ProxyLoader({"input_ids": seq, "attention_mask": torch.ones_like(seq), "labels": seq})
    batch = {"input_ids": seq, "attention_mask": torch.ones_like(seq), "labels": seq}
    with pytest.raises(RuntimeError):
        ds.capture_pairs(model, batch, loader, [GCLinear(2, 2)], score_len=128)  # never called: no Z


def test_gclinear_capture_and_decomposition():
    lin = GCLinear(6, 4, bias=True)
    x = torch.randn(3, 5, 6)
    z = lin(x)
    assert lin.layer_input is x and lin.pre_activation is z
    dz = torch.randn(3, 5, 4)
    g, a = lin.pe_grad_gradcomp(dz)
    assert torch.equal(g, dz * 3) and a is x  # 3-D inputs: no ones column
    x2 = torch.randn(3, 6)
    lin(x2)
    g2, a2 = lin.pe_grad_gradcomp(torch.randn(3, 4))
    assert a2.shape == (3, 7) and torch.all(a2[:, -1] == 1)
    w, b = lin.per_example_gradient(torch.randn(3, 4))
    assert w.shape == (3, 4, 6) and b.shape == (3, 4)
    # per-sample squared norms: |g a^T|^2 + |g|^2
    dz2 = torch.randn(3, 4)
    gz = (dz2 * 3).pow(2).sum(1)
    torch.testing.assert_close(lin.pe_grad_sqnorm(dz2), gz * x2.pow(2).sum(1) + gz)


def test_lora_layers():
    torch.manual_seed(0)
    lin = LoRALinear(8, 6, r=2, lora_alpha=4)
    torch.nn.init.normal_(lin.lora_B)
    x = torch.randn(5, 8)
    y_train = lin(x)
    lin.eval()
    assert lin.merged
    torch.testing.assert_close(lin(x), y_train)
    lin.train()
    assert not lin.merged
    torch.testing.assert_close(lin(x), y_train)
    gl = GCLoRALinear(8, 6, r=2)
    out = gl(torch.randn(2, 3, 8))
    assert gl.pre_activation is out
    pairs = gl.pe_grad_gradcomp(torch.randn(2, 3, 6))
    (g_a, a_a), (g_b, a_b) = pairs
    assert g_a.shape == (2, 3, 2) and a_a.shape == (2, 3, 8)
    assert g_b.shape == (2, 3, 6) and a_b.shape == (2, 3, 2)


def test_find_gc_layers():
    model = TinyLM(GCLinear)
    assert len(ds.find_GClayers(model)) == 4


def _reference_token_loss(logits, labels):
    """data_selection.py:380-389 verbatim in behaviour: shifted copy, cross entropy over every row."""
    shift_logits = logits[..., :-1, :].contiguous()
    shift_labels = labels[..., 1:].contiguous()
    tok = torch.nn.functional.cross_entropy(shift_logits.view(-1, shift_logits.size(-1)), shift_labels.view(-1),
                                            reduction="none", ignore_index=-100).view(shift_labels.size())
    mask = (shift_labels != -100).float()
    return (tok * mask).sum(dim=-1) / mask.sum(dim=-1)


def token_loss_pair(logits, labels, chunk_bytes, monkeypatch):
    """(reference loss, reference grad, chunked loss, chunked grad) for the same logits."""
    monkeypatch.setattr(ds, "TOKEN_LOSS_CHUNK_BYTES", chunk_bytes)
    out = []
    for f in (_reference_token_loss, ds.per_sample_token_loss):
        x = logits.clone().requires_grad_()
        loss = f(x, labels)
        loss.mean().backward()
        out += [loss.detach(), x.grad]
    return out


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("V", [97, 128])
@pytest.mark.parametrize("chunk_bytes", [1, 20000, 1 << 30])
def test_chunked_token_loss_bit_identical(dtype, V, chunk_bytes, monkeypatch):
    """Chunked per-sample loss == the reference's loss and dL/dlogits, bit for bit, ignored labels included."""
    torch.manual_seed(V)
    logits = (torch.randn(7, 34, V) * 3).to(dtype)  # 33 shifted rows: odd chunk alignment
    labels = torch.randint(0, V, (7, 34))
    labels[1, 5:9] = -100
    labels[3, :] = -100
    labels[3, 4] = 2
    ref_l, ref_g, l, g = token_loss_pair(logits, labels, chunk_bytes, monkeypatch)
    assert torch.equal(ref_l, l) and torch.equal(ref_g, g)


@pytest.mark.parametrize("mode", ["high", "low", "mid"])
@pytest.mark.parametrize("ratio", [0.3, 0.9])
def test_ppl_strategy_matches_reference(mode, ratio):
    """selection_strategy="ppl": the reference's loss ranking, mid quantile band and fill path included."""
    g = load_golden("ppl")
    torch.manual_seed(3)
    model = TinyLM(GCLinear, vocab=256)
    load_numpy_state(model, g)
    ct = torch.from_numpy(g["cand"])
    idx = ds.get_batch_opus(model, ct, ct.clone(), None, None, None, [], None, ratio, 128,
                            selection_strategy="ppl", selection_method=mode, score_len=128)
    assert idx.tolist() == g[f"{mode}_{ratio}"].tolist()


@pytest.mark.parametrize("B,T,d_in,d_out,ghost", [
    (64, 64, 768, 3072, True), (64, 128, 768, 3072, True), (64, 256, 768, 3072, False),
    (64, 1024, 768, 3072, False), (16, 128, 768, 768, True), (8, 512, 768, 768, True),
    (6, 128, 64, 128, True),  # the whole-path fixtures' tiny layers
])
def test_ghost_gram_cost_model(B, T, d_in, d_out, ghost):
    """The projection-off similarity picks the path that measured faster on a B200."""
    assert ds.ghost_gram_cheaper(B, T, d_in, d_out) is ghost


def test_capture_pass_planning(monkeypatch):
    """rows_per_pass: a forced count wins, a CPU device never splits; Muon detection by group or name."""
    model = TinyLM(GCLinear)
    layers = ds.find_GClayers(model)
    assert ds.rows_per_pass(layers, 128, "cpu") >= 1 << 20
    monkeypatch.setattr(ds, "CAPTURE_ROWS", 3)
    assert ds.rows_per_pass(layers, 128, "cuda") == 3
    assert ds._pairs(layers) == len(layers)
    adam = torch.optim.AdamW(model.parameters())
    muon = MuonLike(list(model.parameters())[:1])
    assert not ds._has_muon(adam, "adamw") and ds._has_muon(adam, "muon")
    assert ds._has_muon([adam, muon], "auto") and not ds._has_muon(adam, "auto")
    assert not ds._has_muon([adam, muon], "sgd")


def test_adamw_table_reserve_counts_adamw_pairs_only():
    """The bytes a round in passes keeps for AdamW epilogue tables: 8 per element of every 128 x 256 tile."""
    model = TinyLM(GCLinear)
    layers = ds.find_GClayers(model)
    params = [layer.weight for layer in layers]
    want = sum(-(-p.shape[0] // 128) * -(-p.shape[1] // 256) * 128 * 256 * 8 for p in params)
    adam = torch.optim.AdamW(model.parameters())
    assert ds._adamw_table_bytes(layers, adam, "adamw") == want
    assert ds._adamw_table_bytes(layers, adam, "auto") == want
    assert ds._adamw_table_bytes(layers, adam, "sgd") == 0 and ds._adamw_table_bytes(layers, adam, "muon") == 0
    muon = MuonLike(params[:1])
    rest = torch.optim.AdamW([p for p in model.parameters() if p is not params[0]])
    first = -(-params[0].shape[0] // 128) * -(-params[0].shape[1] // 256) * 128 * 256 * 8
    assert ds._adamw_table_bytes(layers, [rest, muon], "auto") == want - first


@pytest.mark.parametrize("rows,step", [(128, 29), (16, 29), (0, 8), (7, 1), (144, 24), (5, 100)])
def test_pass_ranges_cover_rows_in_balanced_passes(rows, step):
    """As few passes as the step allows, contiguous, covering every row once, sizes within one."""
    ranges = ds.pass_ranges(rows, step)
    assert len(ranges) == -(-rows // step)
    assert [lo for lo, _ in ranges[1:]] == [hi for _, hi in ranges[:-1]]
    assert (ranges[0][0] if ranges else 0) == 0 and (ranges[-1][1] if ranges else 0) == rows
    sizes = [hi - lo for lo, hi in ranges]
    assert all(0 < n <= step for n in sizes) and (not sizes or max(sizes) - min(sizes) <= 1)


def test_capture_in_passes_needs_the_projector():
    ds.initialize_projector(enabled=False)
    with pytest.raises(ValueError, match="projector"):
        ds.capture_in_passes(None, "cpu", {"input_ids": torch.zeros(1, 4)}, None, None, [], "adamw", 4)
