"""OPUS scoring and selection (drop-in for OPUS/train/data_selection.py).

Same public functions, arguments, return types and exceptions as the
reference module; the numeric work runs in the sm_100a kernels of
libopus_b200.so:

  stage 1  capture        GCLinear stashes (A, Z); autograd gives G = dL/dZ
  stage 2  ghost scores   ops.ghost_score         (projection off)
  stage 3  CountSketch    ops.sketch_gemm         (fused per-sample GEMM + scatter)
  stage 4  precondition   folded into the sketch table (AdamW diagonal) or
                          applied to G (Muon S) / to the dense target
  stage 5  selection      ops.boltzmann_select / ops.greedy_select

Scores use one sketch pass per layer for the candidates: the reference
sketches the candidates twice (once for the scores, data_selection.py:509,
once for the similarity, :572) with identical inputs, and averages the
proxy-side dot products, which equals one dot with the summed proxy sketch
(CountSketch is linear), so the proxy batch is reduced to one sketch row.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from .. import ops
from .random_projection import GradientProjector

_RANDOM_PROJECTION_AVAILABLE = True

# Global projector instance (data_selection.py:27-28)
_GLOBAL_PROJECTOR: GradientProjector | None = None


def initialize_projector(sketch_dim: int = 16384, seed: int = 42, device: str = "cuda", enabled: bool = True):
    """Create (or disable) the global CountSketch projector (data_selection.py:31-68)."""
    global _GLOBAL_PROJECTOR
    if enabled and sketch_dim > 0:
        _GLOBAL_PROJECTOR = GradientProjector(sketch_dim=sketch_dim, seed=seed, device=device, enabled=True)
        max_grad_dim = 10_240_000  # largest GPT-2 XL layer (MLP), as the reference reports
        print(f"[Random Projection] Initialized: dim={sketch_dim}, compression≈{max_grad_dim / sketch_dim:.0f}x, "
              f"seed={seed}")
    else:
        _GLOBAL_PROJECTOR = None
        print("[Random Projection] Disabled (using full-dimensional gradients)")


def get_projector():
    """The global projector, or None when projection is disabled (data_selection.py:71-73)."""
    return _GLOBAL_PROJECTOR


_GBG_CALL_ID = 0


def make_window_generator(step: int, rank: int, base_seed: int = 12345, device: str = "cuda"):
    """Deterministic generator for window starts (data_selection.py:79-83)."""
    g = torch.Generator(device=device)
    g.manual_seed(base_seed + step * 100003 + rank * 1009)
    return g


def _as_opt_list(optimizer_or_list):
    return list(optimizer_or_list) if isinstance(optimizer_or_list, (list, tuple)) else [optimizer_or_list]


def _build_param2opt_map(optimizers):
    """param -> owning optimizer (data_selection.py:93-100); later optimizers win."""
    return {p: opt for opt in optimizers for g in opt.param_groups for p in g["params"]}


def _group_kind(group):
    """adamw if the group has betas, muon if it has momentum (data_selection.py:103-109)."""
    if "betas" in group:
        return "adamw"
    if "momentum" in group:
        return "muon"
    return "unknown"


def _get_rank_safe():
    if torch.distributed.is_available() and torch.distributed.is_initialized():
        return torch.distributed.get_rank()
    return 0


def _copy_batch_dict(batch):
    return dict(batch.items())


def _next_batch(loader):
    try:
        return next(loader._it)
    except StopIteration:
        loader._it = iter(loader)
        return next(loader._it)


def _sample_proxy_batch_for_step(validation_loader):
    """One proxy batch per selection round (data_selection.py:124-157).

    A batch pinned in ``_fixed_batch`` wins; otherwise ``_proxy_mode`` "fixed"
    reuses the first batch drawn and "refresh" draws a new one every
    ``_proxy_refresh_interval`` calls.
    """
    fixed = getattr(validation_loader, "_fixed_batch", None)
    if fixed is not None:
        return _copy_batch_dict(fixed)
    if not hasattr(validation_loader, "_it"):
        validation_loader._it = iter(validation_loader)
    mode = getattr(validation_loader, "_proxy_mode", "refresh")
    interval = max(1, int(getattr(validation_loader, "_proxy_refresh_interval", 1)))
    cached = getattr(validation_loader, "_cached_proxy_batch", None)
    calls = int(getattr(validation_loader, "_proxy_call_count", 0))
    if mode == "fixed":
        if cached is None:
            cached = _next_batch(validation_loader)
            validation_loader._cached_proxy_batch = cached
        return _copy_batch_dict(cached)
    if cached is None or calls % interval == 0:
        cached = _next_batch(validation_loader)
        validation_loader._cached_proxy_batch = cached
    validation_loader._proxy_call_count = calls + 1
    return _copy_batch_dict(cached)


def _get_step_from_optimizer(optimizer):
    """Largest state['step'] over the optimizer's params, at least 1 (data_selection.py:160-168)."""
    t = 1
    for g in optimizer.param_groups:
        for p in g["params"]:
            st = optimizer.state.get(p, None)
            if st is not None and "step" in st:
                t = max(t, int(st["step"]))
    return t


def _find_group_for_param(optimizer, p):
    """Param group holding p by identity, else the first group (data_selection.py:171-179)."""
    for g in optimizer.param_groups:
        if any(gp is p for gp in g.get("params", ())):
            return g
    return optimizer.param_groups[0]


def _C_t_value(optimizer, p, t=None) -> float:
    g = _find_group_for_param(optimizer, p)
    beta1, beta2 = g["betas"]
    if t is None:
        t = _get_step_from_optimizer(optimizer)
    num = max(1e-16, 1.0 - beta2 ** t) ** 0.5
    den = max(1e-16, 1.0 - beta1 ** t)
    return g["lr"] * (1.0 - beta1) * num / den


def global_C_t(optimizer, p):
    """AdamW scalar lr*(1-b1)*sqrt(1-b2^t)/(1-b1^t) as a float32 tensor (data_selection.py:182-195)."""
    return torch.tensor(_C_t_value(optimizer, p), dtype=torch.float32, device=p.device)


def _inv_rms_scalar_for_param(p, group, state):
    """Mean of the AdamW diagonal (data_selection.py:198-205)."""
    v = state.get("exp_avg_sq", None)
    if v is None:
        return torch.tensor(1.0, dtype=torch.float32, device=p.device)
    return (v.sqrt() + group.get("eps", 1e-8)).reciprocal().to(dtype=torch.float32).mean()


def _inv_rms_tensor_for_param(group, state):
    """AdamW diagonal 1/(sqrt(v)+eps) in float32, or None (data_selection.py:208-214)."""
    v = state.get("exp_avg_sq", None)
    if v is None:
        return None
    return (v.sqrt() + group.get("eps", 1e-8)).reciprocal().to(dtype=torch.float32)


def _C_t_muon_value(optimizer, p) -> float:
    g = _find_group_for_param(optimizer, p)
    lr = g["lr"] * max(1, p.size(-2) / p.size(-1)) ** 0.5 * getattr(p, "lr_mul", 1.0)
    mu = g.get("momentum", 0.0)
    return lr * (1.0 - mu ** 2)


def global_C_t_muon(optimizer, p):
    """Muon scalar eff_lr * (1 - momentum^2) (data_selection.py:217-225)."""
    return torch.tensor(_C_t_muon_value(optimizer, p), dtype=torch.float32, device=p.device)


def _get_muon_S_matrix(p, optimizer):
    """S = a I + b A + c A^2 with A = m~ m~^T, m~ = m/||m|| in bf16 (data_selection.py:228-252).

    Identity when the parameter has no momentum buffer or ||m|| < 1e-7.  The
    norm, the normalisation, both GEMMs and the combination run in
    ops.muon_S (tcgen05 GEMMs rounding to bf16 where the reference's bf16
    torch ops round); the norm test happens on the device, so no host sync.
    """
    state = optimizer.state.get(p, None)
    if state is None or "momentum_buffer" not in state:
        return torch.eye(p.shape[0], dtype=torch.bfloat16, device=p.device)
    return ops.muon_S(state["momentum_buffer"].to(device=p.device))


def weighted_grad_dotprod(A1, B1, A2, B2, diagonal_weight: torch.Tensor, weight_rhs: bool = False,
                          chunk_rows: int = 32) -> torch.Tensor:
    """<D o G1_i, G2_j> (or <D o G1_i, D o G2_j>) for all pairs (data_selection.py:255-292).

    A* are dL/dZ factors [B, D_out] / [B, T, D_out], B* activations.  The
    per-sample gradients are formed once per side by the tensor-core GEMM with
    a dense epilogue (ops.per_sample_grad), then contracted with one Gram pass.
    """
    if diagonal_weight.ndim != 2:
        raise ValueError(f"Expected diagonal_weight with shape [D_out, D_in], got {tuple(diagonal_weight.shape)}")
    if A1.dim() != B1.dim() or A1.dim() not in (2, 3):
        raise ValueError(f"Unexpected input shape: {A1.size()}, grad_output shape: {B1.size()}")
    D = diagonal_weight.to(device=A1.device, dtype=torch.float32)
    lhs = _materialize(A1, B1, D)
    rhs = _materialize(A2, B2, D if weight_rhs else None)
    return ops.sketch_gram(lhs, rhs)


def _materialize(dLdZ, a, diag=None):
    """Per-sample gradients D o (dLdZ_b^T a_b) flattened to [B, D_out*D_in] in f32."""
    if dLdZ.dim() == 2:
        dLdZ, a = dLdZ.unsqueeze(1), a.unsqueeze(1)
    return ops.per_sample_grad(dLdZ, a, diag=diag)


def find_GClayers(model):
    """All GCLinear / GCLoRALinear modules of the model (data_selection.py:295-299)."""
    from ..layers.linear import GCLinear
    from ..layers.lora_layers import GCLoRALinear
    return [m for m in model.modules() if isinstance(m, (GCLinear, GCLoRALinear))]


def _random_windows(x, win_len, align_to=128, g=None):
    """Random aligned windows of length win_len (data_selection.py:302-315)."""
    N, T = x.size()
    if T <= win_len:
        idx = torch.arange(min(T, win_len), device=x.device).expand(N, -1)
        return x[:, :win_len], idx
    max_start = T - win_len
    starts = torch.randint(0, max_start + 1, (N,), device=x.device, generator=g)
    if align_to is not None and align_to > 1:
        starts = torch.clamp((starts // align_to) * align_to, 0, max_start)
    idx = starts[:, None] + torch.arange(win_len, device=x.device)[None, :]
    return x.gather(1, idx), idx


# ----------------------------------------------------------------- scoring core
class _Pair:
    """One (dL/dZ, A) factor pair split into candidate and proxy rows; `scale` multiplies dL/dZ
    (1 when the layer already applied its per-sample scaling)."""
    __slots__ = ("p", "g_t", "a_t", "g_v", "a_v", "scale")

    def __init__(self, p, g_t, a_t, g_v, a_v, scale=1.0):
        self.p, self.g_t, self.a_t, self.g_v, self.a_v, self.scale = p, g_t, a_t, g_v, a_v, scale


def capture_pairs(model, batch_train, validation_loader, trainable_layers, score_len=512, batch_val=None):
    """Stage 1: (dL/dZ, A) of every captured layer for candidates and proxies.

    One forward over the candidates and the round's proxy batch with dropout
    off, per-sample mean next-token cross-entropy (labels -100 ignored),
    dL/dZ by autograd to each layer's stored pre-activation, then each
    layer's factorisation split into candidate / proxy halves
    (data_selection.py:345-445).  Returns (pairs, n_candidates, n_proxies).
    batch_val, when given, replaces the loader's proxy batch (a rank's share
    of it in sharded selection).
    """
    loss, layers_kept, z_list, train_bs, val_bs = _capture_forward(model, batch_train, validation_loader,
                                                                   trainable_layers, score_len, batch_val)
    z_grads = torch.autograd.grad(loss.mean(), z_list, retain_graph=False, allow_unused=True)
    del loss

    pairs: list[_Pair] = []
    for layer, zg in zip(layers_kept, z_grads):
        if zg is None:
            continue
        pairs.extend(_layer_pairs(layer, zg, train_bs))
    return pairs, train_bs, val_bs


# bytes of logits one chunk of the per-position loss covers
TOKEN_LOSS_CHUNK_BYTES = 1 << 30


class _ShiftedTokenLoss(torch.autograd.Function):
    """Per-position next-token cross entropy [N, T-1] from logits [N, T, V], by chunks of samples.

    The reference (data_selection.py:381-387) copies logits[:, :-1] into a
    contiguous tensor and runs cross_entropy over all of it.  That keeps the
    copy and the whole log-softmax alive for the backward, whose dense
    [N*(T-1), V] temporaries and zero-filled [N, T, V] slice gradient come on
    top.  Here each chunk of samples runs the same torch cross_entropy and
    nothing is kept but the logits; the backward recomputes each chunk and
    writes its gradient into one [N, T, V] tensor.

    Rows are independent in log_softmax / nll_loss, but inside a row torch's
    CUDA kernels pick their reduction order from the row's 16-byte alignment.
    So when a row (V elements) is a multiple of 16 bytes -- GPT-2's padded
    50304-entry vocabulary, Llama's, Qwen's -- a chunk runs on all T
    positions of the logits in place, the last one taking label -100 so that
    position t meets label t+1.  Otherwise a chunk copies its shifted rows,
    as the reference does, and chunks start at sample multiples that give
    every row the alignment it has in the reference's copy.  Either way every
    loss and gradient value equals the reference's.
    """

    @staticmethod
    def forward(ctx, logits, labels):
        N, T, _ = logits.shape
        out = torch.zeros(N, T - 1, dtype=logits.dtype, device=logits.device)
        for s, e, rows, lab in _token_loss_chunks(logits, labels):
            loss = torch.nn.functional.cross_entropy(rows, lab, reduction="none", ignore_index=-100)
            out[s:e] = loss.view(e - s, -1)[:, :T - 1]
        ctx.save_for_backward(logits, labels)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        logits, labels = ctx.saved_tensors
        N, T, V = logits.shape
        grad = torch.empty_like(logits)
        for s, e, rows, lab in _token_loss_chunks(logits, labels):
            in_place = rows.shape[0] == (e - s) * T
            g = grad_out[s:e]
            if in_place:  # the last position carries label -100 and gradient 0
                g = torch.cat([g, g.new_zeros(e - s, 1)], dim=1)
            with torch.enable_grad():
                rows = rows.detach().requires_grad_()
                loss = torch.nn.functional.cross_entropy(rows, lab, reduction="none", ignore_index=-100)
                (part,) = torch.autograd.grad(loss, rows, g.reshape(-1))
            if in_place:
                grad[s:e] = part.view(e - s, T, V)
            else:
                grad[s:e, :-1] = part.view(e - s, T - 1, V)
                grad[s:e, -1] = 0
        return grad, None


def _token_loss_chunks(logits, labels):
    """(first sample, end sample, rows [R, V], their labels [R]) of each chunk of the shifted loss."""
    N, T, V = logits.shape
    esz = logits.element_size()
    step = max(1, TOKEN_LOSS_CHUNK_BYTES // max(1, T * V * esz))
    in_place = (V * esz) % 16 == 0
    if not in_place:  # chunk starts s with s * (T-1) * V * esz a multiple of 16 bytes
        m = 16 // math.gcd(16, (T - 1) * V * esz)
        step = max(m, step - step % m)
    for s in range(0, N, step):
        e = min(N, s + step)
        if in_place:
            lab = torch.full((e - s, T), -100, dtype=labels.dtype, device=labels.device)
            lab[:, :-1] = labels[s:e, 1:]
            yield s, e, logits[s:e].view(-1, V), lab.view(-1)
        else:
            yield s, e, logits[s:e, :-1].contiguous().view(-1, V), labels[s:e, 1:].reshape(-1)


def per_sample_token_loss(logits, labels):
    """Mean next-token cross entropy of each sample over its non-ignored positions (data_selection.py:380-389)."""
    if logits.dim() != 3 or logits.shape[1] < 2:
        shift_logits = logits[..., :-1, :].contiguous()
        shift_labels = labels[..., 1:].contiguous()
        tok_loss = torch.nn.functional.cross_entropy(shift_logits.view(-1, shift_logits.size(-1)),
                                                     shift_labels.view(-1), reduction="none",
                                                     ignore_index=-100).view(shift_labels.size())
    else:
        shift_labels = labels[..., 1:]
        tok_loss = _ShiftedTokenLoss.apply(logits.contiguous(), labels)
    mask = (shift_labels != -100).float()
    return (tok_loss * mask).sum(dim=-1) / mask.sum(dim=-1)


def _capture_forward(model, batch_train, validation_loader, trainable_layers, score_len, batch_val):
    """The capture forward: per-sample mean token loss over candidates + proxies, and the kept layers.

    Returns (loss [N], kept layers, their pre-activations Z, n_candidates, n_proxies).
    """
    if batch_val is None:
        batch_val = _sample_proxy_batch_for_step(validation_loader)
    else:
        batch_val = _copy_batch_dict(batch_val)
    val_bs = batch_val["input_ids"].shape[0]
    train_bs = batch_train["input_ids"].shape[0]

    L = min(batch_train["input_ids"].shape[1], batch_val["input_ids"].shape[1])
    if score_len is not None:
        L = min(L, score_len)
    for bd in (batch_train, batch_val):
        for key in ("input_ids", "attention_mask", "labels"):
            bd[key] = bd[key][:, :L]

    labels = torch.cat([batch_train["labels"], batch_val["labels"]], dim=0)
    inputs = {k: torch.cat([batch_train[k], batch_val[k]], dim=0) for k in batch_train.keys() if k != "labels"}
    del batch_train, batch_val
    was_training = model.training
    model.eval()
    logits = model(input_seq=inputs["input_ids"], target_seq=None, sliding_window_num_blocks=None)
    if was_training:
        model.train()

    loss = per_sample_token_loss(logits, labels)
    del logits

    raw = [layer.pre_activation for layer in trainable_layers]
    keep = [i for i, z in enumerate(raw) if isinstance(z, torch.Tensor) and z.requires_grad and z.grad_fn is not None]
    if not keep:
        raise RuntimeError("No usable pre_activations captured. Check GC hooks / forward path.")
    return loss, [trainable_layers[i] for i in keep], [raw[i] for i in keep], train_bs, val_bs


def _plain_gclinear(layer) -> bool:
    """A capture layer whose factors are this package's GCLinear ones: (dL/dZ * N, A)."""
    from ..layers.linear import GCLinear
    return isinstance(layer, GCLinear) and type(layer).pe_grad_gradcomp is GCLinear.pe_grad_gradcomp


def _layer_pairs(layer, zg, train_bs, fold_scale=False):
    """(dL/dZ, A) factor pairs of one layer split into candidate / proxy halves (data_selection.py:413-445).

    fold_scale: for this package's GCLinear on 3-D inputs, hand over dL/dZ as
    autograd gives it and the per-sample factor N (linear.py:118-119) as the
    pair's scale, which the sketch kernel applies in f32, instead of a pass
    over dL/dZ that writes dL/dZ * N.
    """
    if fold_scale and zg.dim() == 3 and _plain_gclinear(layer) and layer.layer_input is not None \
            and layer.layer_input.dim() == 3:
        g, a = zg.detach(), layer.layer_input.detach()
        return [_Pair(getattr(layer, "weight", None), g[:train_bs], a[:train_bs], g[train_bs:], a[train_bs:],
                      float(zg.shape[0]))]
    parts = layer.pe_grad_gradcomp(zg, per_sample=True)
    if isinstance(parts, tuple) and len(parts) == 2 and all(isinstance(x, torch.Tensor) for x in parts):
        parts = [parts]
    else:
        parts = list(parts)
    lparams = [getattr(layer, n) for n in ("lora_A", "lora_B") if hasattr(layer, n)]
    out = []
    for i, (g, a) in enumerate(parts):
        p = lparams[i] if i < len(lparams) else getattr(layer, "weight", None)
        g, a = g.detach(), a.detach()
        out.append(_Pair(p, g[:train_bs], a[:train_bs], g[train_bs:], a[train_bs:]))
    return out


class LayerPlan:
    """Stage-4 inputs of one (dL/dZ, A) pair: what the kernels apply.

    g_t is the candidate dL/dZ after the Muon transform (if any); c is the
    float32 product C_t * layer_scale; exp_avg_sq / eps give the AdamW
    diagonal folded into the candidate sketch table; gscale is the factor
    still owed to dL/dZ (its per-sample scaling, when the capture left it to
    the sketch kernel), 1 otherwise.
    """
    __slots__ = ("pid", "kind", "g_t", "a_t", "g_v", "a_v", "c", "exp_avg_sq", "eps", "gscale")

    def __init__(self, pid, kind, g_t, a_t, g_v, a_v, c, exp_avg_sq, eps, gscale=1.0):
        self.pid, self.kind, self.g_t, self.a_t, self.g_v, self.a_v = pid, kind, g_t, a_t, g_v, a_v
        self.c, self.exp_avg_sq, self.eps, self.gscale = c, exp_avg_sq, eps, gscale


class _PrecondTables:
    """Per-parameter preconditioner state (data_selection.py:447-506, :545-569)."""

    def __init__(self, params, optimizer, preconditioner):
        self.param2opt = _build_param2opt_map(_as_opt_list(optimizer))
        self.auto_mode = preconditioner == "auto"
        self.preconditioner = preconditioner
        self.S_map, self.muon_scale, self.adamw = {}, {}, {}
        steps = {}  # the optimizer-wide step, once per optimizer rather than once per parameter
        for p in {q for q in params if q is not None}:
            opt_p = self.param2opt.get(p, None)
            if opt_p is None:
                continue
            group = _find_group_for_param(opt_p, p)
            kind = _group_kind(group) if self.auto_mode else preconditioner
            if kind == "muon":
                if p in opt_p.state:
                    self.S_map[p] = _get_muon_S_matrix(p, opt_p)
                # the float32 scalars stay on the host: no device round trip per layer
                self.muon_scale[p] = np.float32(_C_t_muon_value(opt_p, p))
            elif kind == "adamw":
                if id(opt_p) not in steps:
                    steps[id(opt_p)] = _get_step_from_optimizer(opt_p)
                self.adamw[p] = (np.float32(_C_t_value(opt_p, p, steps[id(opt_p)])), group, opt_p.state.get(p, {}))

    def plan(self, pid, pr, device):
        p, g_t = pr.p, pr.g_t
        scale = np.float32(1.0)
        layer_scale = 1.0
        v_sq, eps = None, 1e-8
        eff = "sgd"
        if p is not None:
            opt_p = self.param2opt.get(p, None)
            if opt_p is not None:
                eff = _group_kind(_find_group_for_param(opt_p, p)) if self.auto_mode else self.preconditioner
                if eff == "muon" and p in self.S_map:
                    # dLdZ_t <- einsum('...o,po->...p', dLdZ_t, S^T) (data_selection.py:495-500)
                    g_t = ops.muon_transform(g_t, self.S_map[p].to(g_t.device), symmetric=True)
                    scale = self.muon_scale[p]
                elif eff == "adamw" and p in self.adamw:
                    scale, group_p, state_p = self.adamw[p]
                    if state_p.get("exp_avg_sq", None) is not None:
                        v_sq, eps = state_p["exp_avg_sq"], group_p.get("eps", 1e-8)
                if eff != "sgd" and p.ndim >= 2:
                    layer_scale = 1.0 / float((p.shape[-1] * p.shape[-2]) ** 0.5)
        c = float(np.float32(scale * np.float32(layer_scale)))  # float32 C * ls, as the tensor product
        if v_sq is not None:
            v_sq = v_sq.detach().to(device=device, dtype=torch.float32)
        return LayerPlan(pid, eff, g_t, pr.a_t, pr.g_v, pr.a_v, c, v_sq, eps, pr.scale)


def plan_layers(pairs, optimizer, preconditioner, device):
    """Preconditioner per pair, as data_selection.py:447-506 and :545-569 resolve it.

    'auto' picks per param group (betas -> adamw, momentum -> muon); Muon's S
    transforms the candidate dL/dZ (the proxy side stays untransformed);
    AdamW contributes C_t and its diagonal 1/(sqrt(v)+eps); a preconditioned
    matrix parameter also gets layer_scale = 1/sqrt(d_out d_in).
    """
    tables = _PrecondTables([pr.p for pr in pairs], optimizer, preconditioner)
    return [tables.plan(pid, pr, device) for pid, pr in enumerate(pairs)]


# Capture mode of _score_and_similarity: "stream" scores each layer from a
# backward hook as soon as its dL/dZ exists (no layer's gradient outlives its
# use); "batch" takes every layer's dL/dZ from one autograd call first.
CAPTURE_MODE = "stream"


def _score_plan(pl, projector, score, sim, val_bs, per_val):
    """One (dL/dZ, A) pair's contribution to score and sim (data_selection.py:469-591)."""
    if pl.g_t.dim() == 2:
        g_t, a_t, g_v, a_v = pl.g_t.unsqueeze(1), pl.a_t.unsqueeze(1), pl.g_v.unsqueeze(1), pl.a_v.unsqueeze(1)
    else:
        g_t, a_t, g_v, a_v = pl.g_t, pl.a_t, pl.g_v, pl.a_v
    c = pl.c
    if projector is not None and projector.enabled:
        # stage 3 + 4: one fused sketch pass for the candidates (AdamW
        # diagonal in the table), one for the proxy batch summed to a row
        phi_t = projector.sketch(g_t, a_t, pl.pid, exp_avg_sq=pl.exp_avg_sq, eps=pl.eps)
        if per_val:
            phi_v = projector.sketch(g_v, a_v, pl.pid)
            ops.sketch_gram(phi_t, phi_v, alpha=c, out=score, accumulate=True)
        elif val_bs > 0:
            tau = projector.sketch(g_v, a_v, pl.pid, rows_div=val_bs)
            ops.sketch_dot(phi_t, tau[0], alpha=c / val_bs, out=score, accumulate=True)
        if sim is not None:
            ops.sketch_gram(phi_t, alpha=c * c, out=sim, accumulate=True)
    else:
        _score_dense(g_t, a_t, g_v, a_v, pl.exp_avg_sq, pl.eps, c, per_val, score)
        if sim is not None:
            d_out, d_in = g_t.shape[2], a_t.shape[2]
            if pl.exp_avg_sq is None and ghost_gram_cheaper(g_t.shape[0], g_t.shape[1], d_in, d_out):
                # <G_i, G_j> straight from the factors (grad_dotprod's value, data_selection.py:597-619)
                ops.ghost_gram(a_t, g_t, alpha=c * c, out=sim, accumulate=True)
            else:
                diag = None if pl.exp_avg_sq is None else ops_inv_rms(pl.exp_avg_sq, pl.eps).reshape(d_out, d_in)
                ops.sketch_gram(_materialize(g_t, a_t, diag), alpha=c * c, out=sim, accumulate=True)


# Rates and fixed costs the cost model below uses, fitted to both paths measured on a B200
# (bf16 operands; 64 candidates x 64-1024 tokens at 768x3072, 8-16 at 768x768, 128 at 1600x6400).
_GHOST_GRAM_FLOPS = 0.8e15        # ghost Gram at full 128-token blocks (shorter windows fill less)
_GHOST_GRAM_FIXED_S = 2e-5
_MATERIALISE_FLOPS = 0.8e15       # per-sample gradient GEMM (dense epilogue)
_MATERIALISE_BYTES = 3.0e12       # writing the gradients and reading them back for the Gram
_GRAM_FLOPS = 0.35e15             # 3xTF32 Gram of the gradients (three products)
_MATERIALISE_FIXED_S = 1.5e-4


def ghost_gram_cheaper(B: int, T: int, d_in: int, d_out: int) -> bool:
    """Whether the ghost Gram beats materialising per-sample gradients for one layer's similarity.

    Ghost: B(B+1)/2 pairs x 2 T^2 (d_in + d_out) flop, at a rate that falls with
    windows shorter than its 128-token blocks.  Materialise: B x 2 T d_in d_out
    flop, B d_in d_out f32 written and read, and the Gram's B(B+1)/2 x 2 d_in d_out
    x 3.  Measured: ghost 0.33 against 0.51 ms at 64 x 128 tokens, 768x3072;
    0.09 against 0.22 ms at 8 x 512, 768x768; 1.36 against 0.53 ms at 64 x 256,
    768x3072; 6.1 against 0.95 ms at 64 x 512.
    """
    pairs = B * (B + 1) / 2
    fill = min(1.0, T / 128.0)
    ghost = _GHOST_GRAM_FIXED_S + pairs * 2.0 * T * T * (d_in + d_out) / (_GHOST_GRAM_FLOPS * fill)
    numel = float(d_in) * d_out
    mat = (_MATERIALISE_FIXED_S + B * 2.0 * T * numel / _MATERIALISE_FLOPS + B * numel * 8.0 / _MATERIALISE_BYTES
           + pairs * 2.0 * numel * 3.0 / _GRAM_FLOPS)
    return ghost < mat


def _pairs_per_layer(layer) -> int:
    """Factor pairs pe_grad_gradcomp returns: two for LoRA layers (A and B), one otherwise."""
    return 2 if (hasattr(layer, "lora_A") and hasattr(layer, "lora_B")) else 1


def _score_and_similarity(model, device, batch_train, validation_loader, optimizer, trainable_layers,
                          preconditioner="adamw", score_len=512, per_val=False, with_similarity=True):
    """Device tensors (score [B] or [B, n], sim [B, B] or None) for one window."""
    batch_val = _sample_proxy_batch_for_step(validation_loader)  # one proxy batch per round, whichever mode
    if CAPTURE_MODE == "stream":
        rows = batch_train["input_ids"].shape[0] + batch_val["input_ids"].shape[0]
        seq = min(batch_train["input_ids"].shape[1], batch_val["input_ids"].shape[1], score_len or 1 << 30)
        if _use_passes(rows, trainable_layers, seq, device, model, _has_muon(optimizer, preconditioner)):
            score, phis, cs, _ = capture_in_passes(model, device, batch_train, batch_val, optimizer,
                                                   trainable_layers, preconditioner, score_len, per_val=per_val,
                                                   keep_sketches=with_similarity)
            sim = None
            if with_similarity:
                sim = torch.zeros(phis.shape[1], phis.shape[1], device=device, dtype=torch.float32)
                for pid in range(phis.shape[0]):
                    ops.sketch_gram(phis[pid], alpha=cs[pid] * cs[pid], out=sim, accumulate=True)
            return score, sim
        out = _score_and_similarity_stream(model, device, batch_train, batch_val, optimizer, trainable_layers,
                                           preconditioner, score_len, per_val, with_similarity)
        if out is not None:
            return out
    pairs, train_bs, val_bs = capture_pairs(model, batch_train, validation_loader, trainable_layers, score_len,
                                            batch_val=batch_val)
    plans = plan_layers(pairs, optimizer, preconditioner, device)
    del pairs
    projector = get_projector()
    score = torch.zeros((train_bs, val_bs) if per_val else (train_bs,), device=device, dtype=torch.float32)
    sim = torch.zeros((train_bs, train_bs), device=device, dtype=torch.float32) if with_similarity else None
    for pl in plans:
        _score_plan(pl, projector, score, sim, val_bs, per_val)
    return score, sim


def stream_capture(model, device, batch_train, batch_val, optimizer, trainable_layers, preconditioner, score_len,
                   make_handler, precond: dict | None = None, fold_scale: bool = False):
    """Capture forward, then one backward whose per-layer hooks hand each (dL/dZ, A) pair to a handler.

    The backward pass is asked only for the gradient of the first kept
    layer's input, which every captured Z feeds, so autograd frees each dL/dZ
    once its hook has used it and no layer's gradient outlives its hook.
    make_handler(train_bs, val_bs, n_plans) is called once after the forward
    and returns on_plan(LayerPlan); plans arrive in backward order and carry
    their pair id, which follows the forward order as in the batch capture.
    Returns False when a layer's hook did not fire (a captured output the
    loss does not reach, or no usable root): the caller then falls back to the
    batch capture.  precond: a dict that keeps the preconditioner state
    (Muon S matrices, AdamW scalars) across the passes of one round; it is
    filled by the first pass that gets it.  fold_scale: plans of this
    package's GCLinear layers carry dL/dZ unscaled and its per-sample factor
    as gscale (the handler must apply it).
    """
    loss, layers_kept, z_list, train_bs, val_bs = _capture_forward(
        model, dict(batch_train), None, trainable_layers, score_len, batch_val)
    root = getattr(layers_kept[0], "layer_input", None)
    if not (isinstance(root, torch.Tensor) and root.requires_grad):
        return False
    params = []
    pid_base = []
    for layer in layers_kept:
        pid_base.append(len(params))
        names = ("lora_A", "lora_B") if _pairs_per_layer(layer) == 2 else ()
        params.extend([getattr(layer, n) for n in names] or [getattr(layer, "weight", None)])
    tables = None if precond is None else precond.get("tables")
    if tables is None:
        tables = _PrecondTables(params, optimizer, preconditioner)
        if precond is not None:
            precond["tables"] = tables
    on_plan = make_handler(train_bs, val_bs, len(params))
    fired = [False] * len(layers_kept)
    bad = []

    def make_hook(li):
        def hook(grad):
            try:
                pairs = _layer_pairs(layers_kept[li], grad, train_bs, fold_scale)
                if len(pairs) != _pairs_per_layer(layers_kept[li]):
                    bad.append(li)
                    return None
                for i, pr in enumerate(pairs):
                    on_plan(tables.plan(pid_base[li] + i, pr, device))
                fired[li] = True
            except Exception as exc:  # surfaced after backward: an exception inside autograd loses context
                bad.append(exc)
            return None
        return hook

    handles = [z.register_hook(make_hook(li)) for li, z in enumerate(z_list)]
    try:
        torch.autograd.grad(loss.mean(), [root], retain_graph=False, allow_unused=True)
    finally:
        for h in handles:
            h.remove()
    for b in bad:
        if isinstance(b, Exception):
            raise b
    return not bad and all(fired)


def _score_and_similarity_stream(model, device, batch_train, batch_val, optimizer, trainable_layers,
                                 preconditioner, score_len, per_val, with_similarity):
    """Streaming capture: each layer is scored from a backward hook on its Z (stream_capture).

    Returns None when a hook did not fire; the caller then falls back to the
    batch capture with fresh sums.
    """
    projector = get_projector()
    out = {}

    def make_handler(train_bs, val_bs, n_plans):
        score = torch.zeros((train_bs, val_bs) if per_val else (train_bs,), device=device, dtype=torch.float32)
        sim = torch.zeros((train_bs, train_bs), device=device, dtype=torch.float32) if with_similarity else None
        out["score"], out["sim"] = score, sim
        return lambda pl: _score_plan(pl, projector, score, sim, val_bs, per_val)

    if not stream_capture(model, device, batch_train, batch_val, optimizer, trainable_layers, preconditioner,
                          score_len, make_handler):
        return None
    return out["score"], out["sim"]


# Sequences per capture pass.  None: as many as the device's free memory
# holds (rows_per_pass); an int forces that many (tests use it to run the
# pass-splitting path at small sizes).
CAPTURE_ROWS: int | None = None
# Share of the free device memory a capture pass may fill with activations.
CAPTURE_MEMORY_FRACTION = 0.8
# Activation bytes per token of a capture pass, in units of one (d_in + d_out)
# row per capture layer in the model dtype (measured peaks: about 1.0 for
# GPT-2 small in f32 and bf16, 0.8 for GPT-2 XL in bf16, about 1.3 for a
# Qwen3-style block with its SwiGLU MLP and q/k norms); the logits and their
# gradient are counted apart, from the model's embedding width.
CAPTURE_BYTES_PER_ROW = 1.5


def rows_per_pass(trainable_layers, seq_len: int, device, reserve_bytes: int = 0, model=None,
                  muon: bool = True) -> int:
    """Sequences one capture forward + backward can hold on the device.

    A pass keeps every layer's activations alive until its backward hook has
    run; measured on GPT-2-shaped models the peak is about one
    (d_in + d_out) row per token per capture layer, in the model dtype, plus
    the logits.  The estimate takes CAPTURE_BYTES_PER_ROW times that per token,
    plus the logits and their gradient (the model's largest embedding width),
    against CAPTURE_MEMORY_FRACTION of the free memory, after reserve_bytes
    for what the round keeps (its candidate sketches) and, when muon, room for
    one d_out x d_out bf16 matrix per layer (the Muon S the first pass builds).
    """
    if CAPTURE_ROWS is not None:
        return max(1, int(CAPTURE_ROWS))
    device = torch.device(device)
    if device.type != "cuda":
        return 1 << 30
    per_tok, elt = 0, 2
    for layer in trainable_layers:
        w = getattr(layer, "weight", None)
        if isinstance(w, torch.Tensor) and w.dim() == 2:
            per_tok += (w.shape[0] + w.shape[1]) * w.element_size()
            reserve_bytes += 2 * w.shape[0] * w.shape[0] if muon else 0
            elt = w.element_size()
    per_tok = int(CAPTURE_BYTES_PER_ROW * per_tok)
    if model is not None:
        vocab = max((m.num_embeddings for m in model.modules() if isinstance(m, torch.nn.Embedding)), default=0)
        per_tok += 2 * vocab * elt
    per_tok = max(1, per_tok)
    free, _ = torch.cuda.mem_get_info(device)
    free += torch.cuda.memory_reserved(device) - torch.cuda.memory_allocated(device)
    budget = CAPTURE_MEMORY_FRACTION * free - reserve_bytes
    return max(1, int(budget // (per_tok * max(1, seq_len))))


def pass_ranges(rows: int, step: int) -> list[tuple[int, int]]:
    """Row ranges [lo, hi) of a capture in passes of at most `step` rows: as few passes as
    that allows, of balanced sizes (no short last pass)."""
    n_pass = -(-rows // max(1, step))
    return [(rows * i // n_pass, rows * (i + 1) // n_pass) for i in range(n_pass)]


def _pairs(trainable_layers) -> int:
    return sum(_pairs_per_layer(layer) for layer in trainable_layers)


def _has_muon(optimizer, preconditioner) -> bool:
    """Whether any capture layer may take the Muon preconditioner (and so an S matrix)."""
    if preconditioner == "muon":
        return True
    if preconditioner != "auto":
        return False
    return any(_group_kind(g) == "muon" for opt in _as_opt_list(optimizer) for g in opt.param_groups)


def _adamw_table_bytes(trainable_layers, optimizer, preconditioner) -> int:
    """Device bytes of the AdamW epilogue tables a round in passes keeps (one per AdamW pair).

    The table holds 16 bytes per element pair of every 128 x 256 tile of the
    layer (ops.sketch_table_entries); the other preconditioners use the
    projector's cached sign tables.
    """
    if preconditioner not in ("adamw", "auto"):
        return 0
    p2o = _build_param2opt_map(_as_opt_list(optimizer))
    total = 0
    for layer in trainable_layers:
        names = ("lora_A", "lora_B") if _pairs_per_layer(layer) == 2 else ("weight",)
        for name in names:
            p = getattr(layer, name, None)
            if not isinstance(p, torch.Tensor) or p.dim() != 2:
                continue
            opt = p2o.get(p)
            if opt is None or (preconditioner == "auto" and _group_kind(_find_group_for_param(opt, p)) != "adamw"):
                continue
            tiles = -(-p.shape[0] // 128) * -(-p.shape[1] // 256)
            total += tiles * 128 * 256 * 8
    return total


def _use_passes(rows: int, trainable_layers, seq_len: int, device, model=None, muon: bool = True) -> bool:
    projector = get_projector()
    if projector is None or not projector.enabled:
        return False  # the projection-off similarity needs every candidate's factors at once
    reserve = 4 * projector.sketch_dim * rows * _pairs(trainable_layers)
    return rows > rows_per_pass(trainable_layers, seq_len, device, reserve, model, muon)


def capture_in_passes(model, device, batch_train, batch_val, optimizer, trainable_layers, preconditioner, score_len,
                      per_val=False, keep_sketches=True, reduce_targets=None, n_proxy_total=None):
    """Scores of a round whose candidates and proxies are captured in several forward/backward passes.

    The reference runs one forward and one backward over candidates and
    proxies together (data_selection.py:355-406); at GPT-2-XL widths that
    holds hundreds of GB of activations.  Per-sample gradients do not depend
    on which other samples share the batch (the batch-mean gradient is scaled
    back by the batch size, linear.py:118-119), so the rows are split:

    1. proxy passes: each layer's proxy sketches summed into one target row
       per layer, taus [L, k] (per_val: the proxy sketches [L, n, k]);
       reduce_targets(taus), when given, sums the ranks' partial targets;
    2. candidate passes: each layer's candidate sketches (AdamW diagonal in
       the table, Muon transform applied) scored against the layer's target,
       score += c_l / n * phi_l . tau_l, and kept in phis [L, B, k] when
       keep_sketches, for the similarity sum_l c_l^2 phi_l phi_l^T.

    Rows per pass come from rows_per_pass.  The preconditioner state (Muon S)
    is built once per round.  Returns (score [B] or [B, n], phis or None,
    per-layer scales c_l, taus).  Needs the CountSketch projector.
    """
    projector = get_projector()
    if projector is None or not projector.enabled:
        raise ValueError("capture in passes needs the CountSketch projector (initialize_projector(enabled=True))")
    k = projector.sketch_dim
    B = batch_train["input_ids"].shape[0]
    n = batch_val["input_ids"].shape[0] if batch_val is not None else 0
    n_total = n if n_proxy_total is None else int(n_proxy_total)
    seq = min(batch_train["input_ids"].shape[1], score_len or 1 << 30)
    # kept across the passes: the candidate sketches, and each AdamW layer's epilogue table
    # (the optimizer state does not move within a round, so one build serves every pass)
    reserve = 4 * k * (B + n) * _pairs(trainable_layers) + _adamw_table_bytes(trainable_layers, optimizer,
                                                                            preconditioner)
    step = rows_per_pass(trainable_layers, seq, device, reserve, model, _has_muon(optimizer, preconditioner))
    precond: dict = {}
    st: dict = {"tables": {}}

    def rows_of(batch, lo, hi):
        return {key: v[lo:hi] for key, v in batch.items()}

    empty_train = rows_of(batch_train, 0, 0)
    empty_val = rows_of(batch_train, 0, 0) if batch_val is None else rows_of(batch_val, 0, 0)

    def ensure(n_plans):
        if "taus" not in st:
            st["taus"] = (torch.zeros(n_plans, n, k, device=device, dtype=torch.float32) if per_val else
                          torch.zeros(n_plans, k, device=device, dtype=torch.float32))
            st["cs"] = [0.0] * n_plans

    # 1. proxy passes
    for lo, hi in pass_ranges(n, step):

        def proxy_handler(train_bs, val_bs, n_plans, lo=lo, hi=hi):
            ensure(n_plans)

            def on_plan(pl):
                g_v, a_v = (pl.g_v.unsqueeze(1), pl.a_v.unsqueeze(1)) if pl.g_v.dim() == 2 else (pl.g_v, pl.a_v)
                if per_val:
                    projector.sketch(g_v, a_v, pl.pid, out=st["taus"][pl.pid, lo:hi], alpha=pl.gscale)
                else:
                    projector.sketch(g_v, a_v, pl.pid, rows_div=g_v.shape[0], out=st["taus"][pl.pid:pl.pid + 1],
                                     accumulate=True, alpha=pl.gscale)
            return on_plan

        if not stream_capture(model, device, empty_train, rows_of(batch_val, lo, hi), optimizer, trainable_layers,
                              preconditioner, score_len, proxy_handler, precond, fold_scale=True):
            raise RuntimeError("capture in passes: a capture layer's backward hook did not fire")
    if reduce_targets is not None:
        if "taus" not in st:  # this rank holds no proxy rows: learn the layer count from the first candidate pass
            st["defer_reduce"] = True
        else:
            reduce_targets(st["taus"])

    # 2. candidate passes
    score = torch.zeros((B, n) if per_val else (B,), device=device, dtype=torch.float32)
    for lo, hi in pass_ranges(B, step):

        def cand_handler(train_bs, val_bs, n_plans, lo=lo, hi=hi):
            ensure(n_plans)
            if st.pop("defer_reduce", False):
                reduce_targets(st["taus"])
            if keep_sketches and "phis" not in st:
                st["phis"] = torch.zeros(n_plans, B, k, device=device, dtype=torch.float32)

            def on_plan(pl):
                g_t, a_t = (pl.g_t.unsqueeze(1), pl.a_t.unsqueeze(1)) if pl.g_t.dim() == 2 else (pl.g_t, pl.a_t)
                st["cs"][pl.pid] = pl.c
                out = st["phis"][pl.pid, lo:hi] if keep_sketches else None
                phi = projector.sketch(g_t, a_t, pl.pid, exp_avg_sq=pl.exp_avg_sq, eps=pl.eps, out=out,
                                       table_cache=st["tables"], alpha=pl.gscale)
                if per_val:
                    ops.sketch_gram(phi, st["taus"][pl.pid], alpha=pl.c, out=score[lo:hi], accumulate=True)
                elif n_total > 0 and not keep_sketches:
                    ops.sketch_dot(phi, st["taus"][pl.pid], alpha=pl.c / n_total, out=score[lo:hi],
                                   accumulate=True)
            return on_plan

        if not stream_capture(model, device, rows_of(batch_train, lo, hi), empty_val, optimizer, trainable_layers,
                              preconditioner, score_len, cand_handler, precond, fold_scale=True):
            raise RuntimeError("capture in passes: a capture layer's backward hook did not fire")
    if keep_sketches and not per_val and n_total > 0 and "phis" in st:
        # the kept sketches give every layer's score term in one launch (not one per layer and pass)
        alphas = torch.tensor([c / n_total for c in st["cs"]], dtype=torch.float32, device=device)
        ops.sketch_dot_layers(st["phis"], st["taus"], alphas, out=score, accumulate=True)
    return score, st.get("phis"), st.get("cs", []), st.get("taus")


def ops_inv_rms(v: torch.Tensor, eps: float) -> torch.Tensor:
    """1/(sqrt(v)+eps) in float32 (the AdamW diagonal, data_selection.py:208-214), on the device."""
    return ops.adam_diag(v, eps)


def _score_dense(g_t, a_t, g_v, a_v, v_sq, eps, c, per_val, score):
    """Projection-off scores via the ghost kernel against the dense proxy target.

    score_b += c * <D o G_b, mean_j G_vj> = c / n * <G_b, D o sum_j G_vj>
    (weighted_grad_dotprod / grad_dotprod, data_selection.py:255-292,
    597-619; per_val: one column per proxy j).  The target D o sum_j G_vj is
    the per-sample-gradient kernel run over all proxy tokens as one sample
    (its dense epilogue applies D); D comes from ops.adam_diag.
    """
    d_out, d_in = g_t.shape[2], a_t.shape[2]
    n = g_v.shape[0]
    if n == 0:
        return
    diag = None if v_sq is None else ops_inv_rms(v_sq, eps).reshape(d_out, d_in)
    gt_p, at_p = _pad8(g_t), _pad8(a_t)
    do_p, di_p = gt_p.shape[2], at_p.shape[2]

    def pair(w):  # f32 target [d_out * d_in] -> bf16 (hi, lo) pair at the kernel's widths
        w = w.view(d_out, d_in)
        if (do_p, di_p) != (d_out, d_in):
            w = torch.nn.functional.pad(w, (0, di_p - d_in, 0, do_p - d_out))
        return ops.dense_target_pair(w)

    if per_val:
        targets = ops.per_sample_grad(g_v, a_v, diag=diag)
        for j in range(n):
            score[:, j] += ops.ghost_score(at_p, gt_p, pair(targets[j]), alpha=c)
    else:
        T = g_v.shape[1]
        w = ops.per_sample_grad(g_v.reshape(1, n * T, d_out), a_v.reshape(1, n * T, d_in), diag=diag)
        ops.ghost_score(at_p, gt_p, pair(w[0]), alpha=c / n, out=score, accumulate=True)


def _pad8(x):
    d = x.shape[-1]
    p = (d + 7) // 8 * 8
    return x if p == d else torch.nn.functional.pad(x, (0, p - d))


def compute_GradProd_GC_per_iter(model, device, batch_train, validation_loader, optimizer, trainable_layers,
                                 preconditioner="adamw", score_len=512, per_val=False,
                                 return_tracin_and_similarity=True):
    """OPUS step-wise scores and candidate similarity (data_selection.py:318-594).

    Returns NumPy float32 (scores [B] or [B, n], similarity [B, B] or None),
    as the reference does.
    """
    score, sim = _score_and_similarity(model, device, batch_train, validation_loader, optimizer, trainable_layers,
                                       preconditioner=preconditioner, score_len=score_len, per_val=per_val,
                                       with_similarity=return_tracin_and_similarity)
    score_np = score.detach().cpu().numpy()
    if return_tracin_and_similarity:
        return score_np, sim.detach().cpu().numpy()
    return score_np, None


def grad_dotprod(A1, B1, A2, B2) -> torch.Tensor:
    """<G1_i, G2_j> for all pairs (data_selection.py:597-604)."""
    if A1.dim() == 2 and B1.dim() == 2:
        return grad_dotprod_non_sequential(A1, B1, A2, B2)
    if A1.dim() == 3 and B1.dim() == 3:
        return grad_dotprod_sequential(A1, B1, A2, B2)
    raise ValueError(f"Unexpected input shape: {A1.size()}, grad_output shape: {B1.size()}")


def grad_dotprod_non_sequential(A1, B1, A2, B2):
    """(A1 A2^T) * (B1 B2^T) for single-token samples (data_selection.py:607-611)."""
    return torch.matmul(A1, A2.T) * torch.matmul(B1, B2.T)


def grad_dotprod_sequential(A1, B1, A2, B2, chunk_size=1024):
    """Flattened per-sample gradient Gram (data_selection.py:614-619), argument order as the reference."""
    lhs = _materialize(A1, B1)
    rhs = _materialize(A2, B2)
    return ops.sketch_gram(lhs, rhs)


# ----------------------------------------------------------------- selection
def _to_device_pair(scores, interaction_matrix):
    dev = torch.device("cuda", torch.cuda.current_device())
    s = torch.as_tensor(np.asarray(scores, dtype=np.float32) if not torch.is_tensor(scores) else scores)
    m = torch.as_tensor(np.asarray(interaction_matrix, dtype=np.float32)
                        if not torch.is_tensor(interaction_matrix) else interaction_matrix)
    return s.to(dev, torch.float32), m.to(dev, torch.float32)


def greedy_selection(scores, interaction_matrix, K):
    """Greedy pick with interaction penalty (data_selection.py:622-638), on the device.

    Returns a list of K np.int64 indices like the reference.
    """
    s, m = _to_device_pair(scores, interaction_matrix)
    idx = ops.greedy_select(s, m, int(K))
    return [np.int64(i) for i in idx.cpu().numpy()]


def stochastic_greedy_selection(scores, interaction_matrix, K, temperature=1.0):
    """Boltzmann sampling of K with interaction penalty (data_selection.py:641-675), on the device.

    Draws one double per pick from NumPy's global RNG, the stream
    np.random.choice consumes in the reference, so a seeded NumPy state gives
    the reference's indices.
    """
    s, m = _to_device_pair(scores, interaction_matrix)
    K = int(K)
    if K > s.numel():
        raise ValueError("zero-size array to reduction operation maximum which has no identity")
    u = torch.from_numpy(np.random.random_sample(K).astype(np.float64))
    idx = ops.boltzmann_select(s, m, K, float(temperature), u)
    ops.check_device_error("stochastic_greedy_selection")
    return [np.int64(i) for i in idx.cpu().numpy()]


def _select_on_device(scores, sim, K, method, temperature):
    if method == "greedy":
        return ops.greedy_select(scores, sim, K)
    if method == "stochastic":
        if K > scores.numel():
            raise ValueError("zero-size array to reduction operation maximum which has no identity")
        u = torch.from_numpy(np.random.random_sample(K).astype(np.float64))
        idx = ops.boltzmann_select(scores, sim, K, float(temperature), u)
        ops.check_device_error("stochastic_greedy_selection")
        return idx
    raise ValueError(f"Unknown selection method: {method}")


def get_batch_opus(model, buffer_seq, buffer_labels, proxy_seq, proxy_labels, optimizer, trainable_layers,
                   validation_loader, selection_ratio, seq_len, selection_strategy="opus", selection_method="greedy",
                   temperature=1.5, score_len=512, preconditioner="adamw", return_scores_only: bool = False,
                   n_windows: int = 1):
    """OPUS batch selection (data_selection.py:678-836).

    Returns the selected indices (LongTensor on buffer_seq.device), or
    (scores [N], interaction [N, N]) float32 tensors if return_scores_only.
    """
    device = buffer_seq.device
    score_len = min(score_len, seq_len)
    assert score_len % 128 == 0, "score_len must be multiple of 128 (FlexAttention BLOCK_SIZE)"

    def to_batches(x, L):
        if x.dim() == 1:
            n = x.size(0) // L
            if n == 0:
                raise ValueError(f"Length insufficient: {x.size(0)} < {L}")
            return x[: n * L].view(n, L)
        if x.dim() == 2 and x.size(1) == L:
            return x
        raise ValueError(f"Expected [N,{L}] or [T], got {tuple(x.shape)}")

    buffer_seq = to_batches(buffer_seq, seq_len)
    buffer_labels = to_batches(buffer_labels, seq_len)
    if proxy_seq is not None:
        proxy_seq = to_batches(proxy_seq, seq_len)
        proxy_labels = to_batches(proxy_labels, seq_len)
    num_buf = buffer_seq.size(0)
    num_to_select = max(1, int(num_buf * selection_ratio))

    def model_loss_one(seq_1d, lab_1d, use_score_len=False):
        L = score_len if use_score_len else seq_len
        win_blocks = torch.tensor(L // 128, dtype=torch.int32, device=seq_1d.device)
        return model(seq_1d[:L], lab_1d[:L], win_blocks)

    if selection_strategy == "random":
        return torch.randperm(num_buf, device=device)[:num_to_select]

    if selection_strategy == "ppl":
        mode = (selection_method or "high").lower()
        with torch.no_grad():
            losses = torch.stack([model_loss_one(buffer_seq[i], buffer_labels[i], use_score_len=True).detach()
                                  for i in range(num_buf)])
        if mode == "low":
            return torch.topk(-losses, k=num_to_select, largest=True)[1]
        if mode == "mid":
            ql = torch.quantile(losses, torch.tensor(0.2, device=losses.device))
            qh = torch.quantile(losses, torch.tensor(0.8, device=losses.device))
            mask = (losses >= ql) & (losses <= qh)
            mid_idx = torch.nonzero(mask, as_tuple=False).squeeze(-1)
            if mid_idx.numel() >= num_to_select:
                median = torch.quantile(losses, torch.tensor(0.5, device=losses.device))
                order = torch.topk(-torch.abs(losses[mid_idx] - median), k=num_to_select, largest=True)[1]
                return mid_idx[order]
            remaining = num_to_select - mid_idx.numel()
            fill_mask = ~mask
            dist_all = torch.full_like(losses, float("inf"))
            below, above = losses < ql, losses > qh
            dist_all[below] = ql - losses[below]
            dist_all[above] = losses[above] - qh
            dist_all[~fill_mask] = float("inf")
            fill_k = min(remaining, int(fill_mask.sum().item()))
            fill_order = torch.topk(-dist_all, k=fill_k, largest=True)[1]
            return torch.cat([mid_idx, fill_order.to(mid_idx.device)], dim=0)
        return torch.topk(losses, k=num_to_select, largest=True)[1]

    if selection_strategy == "opus":
        global _GBG_CALL_ID
        n_windows = max(1, int(n_windows))
        scores = sim = None
        pinned_here = False
        if getattr(validation_loader, "_fixed_batch", None) is None:
            validation_loader._fixed_batch = _sample_proxy_batch_for_step(validation_loader)
            pinned_here = True
        try:
            for _ in range(n_windows):
                gen = make_window_generator(step=_GBG_CALL_ID, rank=_get_rank_safe(), device=buffer_seq.device.type)
                _GBG_CALL_ID += 1
                win_inputs, idx = _random_windows(buffer_seq, score_len, align_to=128, g=gen)
                batch_train = {"input_ids": win_inputs, "attention_mask": torch.ones_like(win_inputs),
                               "labels": buffer_labels.gather(1, idx)}
                w_scores, w_sim = _score_and_similarity(model, buffer_seq.device, batch_train, validation_loader,
                                                        optimizer, trainable_layers, preconditioner=preconditioner,
                                                        score_len=score_len, per_val=False, with_similarity=True)
                if scores is None:
                    scores, sim = w_scores, w_sim
                else:
                    scores += w_scores
                    sim += w_sim
        finally:
            if pinned_here:
                validation_loader._fixed_batch = None
        scores /= n_windows
        sim /= n_windows
        if return_scores_only:
            return scores.to(torch.float32), sim.to(torch.float32)
        return _select_on_device(scores, sim, num_to_select, selection_method, temperature).to(buffer_seq.device)

    raise ValueError(f"Unknown selection strategy: {selection_strategy}")
