"""The reference's CPU selection path restated op for op in torch — test and baseline infrastructure only.

bench.py's CPU legs (the cpu_baseline field and --impl reference) time
these functions on the host cores: they follow the operation sequence of
gszfwsb/OPUS's own torch code for one selection round, which cannot be run
on a machine where the reference checkout is absent.  tests/ check them
against the fixtures recorded from the reference (tests/golden/).  Nothing in
opus_b200/ imports this file.

  capture_pairs            OPUS/train/data_selection.py:355-445
  project_full_gradient    OPUS/train/random_projection.py:134-193
  round_scores             OPUS/train/data_selection.py:469-591 (AdamW)
  muon_S, muon_transform   OPUS/train/data_selection.py:228-252, :495-500

The CPU host-logic tests also use muon_S and muon_transform in place of the
library's tcgen05 versions, which need a GPU.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def project_full_gradient(dLdZ, a, h, s, k, diag=None, S=None):
    """CountSketch of every sample's preconditioned gradient, [B, k] float32.

    random_projection.py:155-193: the optional dense S transform as an
    einsum, then row chunks of 32 (all rows when d_out <= 32): the chunk's
    per-sample gradients by bmm in float32, times the diagonal's rows, times
    the signs, scatter_add_ into the sketch.
    """
    if S is not None:
        dLdZ = torch.einsum("...o,po->...p", dLdZ.float(), S.float().T).to(dLdZ.dtype)
    if dLdZ.dim() == 2:
        B, d_out = dLdZ.shape
        d_in = a.shape[1]
    else:
        B, _, d_out = dLdZ.shape
        d_in = a.shape[2]
    h = torch.as_tensor(h).view(d_out, d_in)
    s = torch.as_tensor(s).view(d_out, d_in)
    sketches = torch.zeros(B, k, dtype=torch.float32)
    chunk = 32 if d_out > 32 else d_out
    a_f, g_f = a.float(), dLdZ.float()
    diag = None if diag is None else torch.as_tensor(diag).float()
    for o0 in range(0, d_out, chunk):
        o1 = min(o0 + chunk, d_out)
        if dLdZ.dim() == 3:
            gc = torch.bmm(g_f[:, :, o0:o1].transpose(1, 2), a_f)
        else:
            gc = torch.einsum("bo,bi->boi", g_f[:, o0:o1], a_f)
        if diag is not None:
            gc = gc * diag[o0:o1].unsqueeze(0)
        idx = h[o0:o1].reshape(1, -1).expand(B, -1)
        sketches.scatter_add_(1, idx, gc.reshape(B, -1) * s[o0:o1].reshape(1, -1))
    return sketches


def capture_pairs(model, layers, tokens, labels, n_candidates):
    """(dL/dZ * N, A) of every capture layer, split candidates / proxies (data_selection.py:355-445).

    One eval-mode forward over all rows, per-sample mean next-token cross
    entropy (labels -100 ignored), autograd to every layer's stored
    pre-activation, and the per-sample scaling by the batch size.
    """
    was = model.training
    model.eval()
    logits = model(input_seq=tokens, target_seq=None, sliding_window_num_blocks=None)
    if was:
        model.train()
    shift_logits = logits[..., :-1, :].contiguous()
    shift_labels = labels[..., 1:].contiguous()
    tok = F.cross_entropy(shift_logits.view(-1, shift_logits.size(-1)), shift_labels.view(-1), reduction="none",
                          ignore_index=-100).view(shift_labels.size())
    mask = (shift_labels != -100).float()
    loss = (tok * mask).sum(dim=-1) / mask.sum(dim=-1)
    zs = [layer.pre_activation for layer in layers]
    grads = torch.autograd.grad(loss.mean(), zs, allow_unused=True)
    N = tokens.shape[0]
    out = []
    for layer, g in zip(layers, grads):
        a = layer.layer_input.detach()
        g = g.detach() * N
        out.append(((g[:n_candidates], a[:n_candidates]), (g[n_candidates:], a[n_candidates:])))
    return out


def round_scores(pairs, tables, k, diags, scales):
    """Scores and similarity of one AdamW round as the reference forms them (data_selection.py:469-591).

    The candidates are sketched twice (once for the scores with the
    diagonal, once more for the similarity), the proxies once without it;
    score += C*ls * mean_j(phi_t . phi_v_j), sim += (C*ls)^2 phi phi^T.
    tables[i] = (h, s) of pair i, diags[i] its AdamW diagonal, scales[i] = C*ls.
    """
    score = sim = None
    for i, ((g_t, a_t), (g_v, a_v)) in enumerate(pairs):
        h, s = tables[i]
        phi_t = project_full_gradient(g_t, a_t, h, s, k, diag=diags[i])
        phi_v = project_full_gradient(g_v, a_v, h, s, k)
        part = scales[i] * (phi_t @ phi_v.T).mean(dim=1)
        score = part if score is None else score + part
        phi_s = project_full_gradient(g_t, a_t, h, s, k, diag=diags[i])
        gram = scales[i] ** 2 * (phi_s @ phi_s.T)
        sim = gram if sim is None else sim + gram
    return score, sim


def muon_S(m):
    """S = a I + b A + c A^2, A = m~ m~^T, m~ = m / ||m|| in bf16 torch ops (data_selection.py:238-252).

    The identity when ||m|| < 1e-7.  Runs on m's device.
    """
    m = m.to(dtype=torch.bfloat16)
    eye = torch.eye(m.shape[0], dtype=torch.bfloat16, device=m.device)
    norm = torch.norm(m)
    if norm < 1e-7:
        return eye
    mt = m / norm
    A = mt @ mt.T
    return 3.4445 * eye + -4.7750 * A + 2.0315 * (A @ A)


def muon_transform(dLdZ, S, symmetric=False):
    """dLdZ <- einsum('...o,po->...p', dLdZ.float(), S.float().T).to(dLdZ.dtype) (data_selection.py:497-498)."""
    return torch.einsum("...o,po->...p", dLdZ.float(), S.float().T).to(dLdZ.dtype)
