"""CPU oracle of the OPUS selection path — test infrastructure only.

A NumPy restatement of the reference algorithm (gszfwsb/OPUS,
OPUS/train/data_selection.py and OPUS/train/random_projection.py), used as
the checker for the CUDA path by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py.  Nothing in opus_b200/ imports it.

Parity pinning: tests/golden/ holds fixtures produced by running the
reference itself (tests/golden/make_golden.py imports the reference package
and records its inputs and outputs); tests/test_oracle_golden.py checks every
function here against them (hash/sign tables and selections bit-exactly,
floating-point outputs to 1e-5 relative).

Third-party arithmetic the reference delegates: torch.Generator/torch.randint
(bucket/sign tables; reproduced by calling torch with the reference's seeding
recipe), torch bmm/scatter_add_ (restated in float64 below) and NumPy
float32 exp / pairwise sum / RandomState.choice (restated with the same
NumPy operations and an explicit uniform per draw).
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


# ----------------------------------------------------------------- H1 tables
def hash_sign_tables(numel: int, param_id: int, k: int, seed: int = 42, device: str = "cpu"):
    """Bucket (int64) and sign (float32 +-1) tables of one parameter.

    random_projection.py:51-70: Generator(device).manual_seed(seed + param_id *
    1000003 + numel); buckets = randint(0, k); then, from the same generator,
    signs = randint(0, 2) * 2 - 1.  The draws are torch's, so torch is called.
    """
    import torch

    gen = torch.Generator(device=device)
    gen.manual_seed(seed + param_id * 1000003 + numel)
    h = torch.randint(0, k, (numel,), generator=gen, device=device, dtype=torch.long)
    s = torch.randint(0, 2, (numel,), generator=gen, device=device, dtype=torch.float32) * 2 - 1
    return h.cpu().numpy(), s.cpu().numpy()


def pack_tables(h: np.ndarray, s: np.ndarray) -> np.ndarray:
    """uint32 bucket | (sign < 0) << 31 — the packed layout the kernels read."""
    return (h.astype(np.uint32) | ((s < 0).astype(np.uint32) << np.uint32(31))).astype(np.uint32)


# ----------------------------------------------------------------- stage 3
def per_sample_grads(dLdZ: np.ndarray, a: np.ndarray, dtype=np.float64) -> np.ndarray:
    """G_b = dLdZ_b^T a_b, [B, d_out, d_in] (random_projection.py:181-184)."""
    g = np.asarray(dLdZ, dtype=dtype)
    x = np.asarray(a, dtype=dtype)
    if g.ndim == 2:
        return g[:, :, None] * x[:, None, :]
    return np.matmul(g.transpose(0, 2, 1), x)


def project_full_gradient(dLdZ, a, h, s, k, diag=None, S=None, precision="f64") -> np.ndarray:
    """phi_b = CountSketch(diag o (dLdZ_b S)^T a_b), [B, k].

    random_projection.py:134-193: optional dense left preconditioner S
    (dLdZ <- dLdZ @ S), per-sample gradient, times diag, times sign,
    scatter-added into bucket h.  precision "f64" (the checker) forms the
    gradients in float64; "f32" forms them in float32 as the reference does
    (the timed CPU baseline).  The reference's 32-row chunking does not
    change the result.
    """
    dt = np.float32 if precision == "f32" else np.float64
    g = np.asarray(dLdZ, dtype=dt)
    if S is not None:
        g = g @ np.asarray(S, dtype=dt)
    G = per_sample_grads(g, a, dtype=dt)
    B = G.shape[0]
    w = np.asarray(s, dtype=dt).reshape(G.shape[1:])
    if diag is not None:
        w = w * np.asarray(diag, dtype=dt).reshape(G.shape[1:])
    hh = np.asarray(h, dtype=np.int64).reshape(-1)
    out = np.zeros((B, k), dtype=np.float64)
    for b in range(B):
        out[b] = np.bincount(hh, weights=(G[b] * w).reshape(-1), minlength=k)
    return out


def dense_sketch(W, h, s, k, diag=None) -> np.ndarray:
    """CountSketch of one dense matrix (random_projection.py:72-99), float64 [k]."""
    x = np.asarray(W, dtype=np.float64).reshape(-1) * np.asarray(s, dtype=np.float64).reshape(-1)
    if diag is not None:
        x = x * np.asarray(diag, dtype=np.float64).reshape(-1)
    return np.bincount(np.asarray(h, dtype=np.int64).reshape(-1), weights=x, minlength=k)


# ----------------------------------------------------------------- stage 4
def inv_rms(v, eps=1e-8) -> np.ndarray:
    """AdamW diagonal 1/(sqrt(v) + eps) in float32 (data_selection.py:208-214)."""
    v = np.asarray(v, dtype=F32)
    return (F32(1.0) / (np.sqrt(v) + F32(eps))).astype(F32)


def adamw_scale(lr, beta1, beta2, t) -> np.float32:
    """C_t = lr (1-b1) sqrt(1-b2^t) / (1-b1^t) (data_selection.py:182-195)."""
    num = max(1e-16, 1.0 - beta2 ** t) ** 0.5
    den = max(1e-16, 1.0 - beta1 ** t)
    return F32(lr * (1.0 - beta1) * num / den)


def muon_scale(lr, d_out, d_in, momentum, lr_mul=1.0) -> np.float32:
    """C_t = lr sqrt(max(1, d_out/d_in)) lr_mul (1 - mu^2) (data_selection.py:217-225)."""
    return F32(lr * max(1, d_out / d_in) ** 0.5 * lr_mul * (1.0 - momentum ** 2))


def bf16_round(x) -> np.ndarray:
    """Round float32 values to bfloat16 (nearest-even), returned as float32."""
    u = np.asarray(x, dtype=F32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16 << 16
    out = (rounded & 0xFFFFFFFF).astype(np.uint32).view(F32)
    nan = np.isnan(np.asarray(x, dtype=F32))
    return np.where(nan, F32(np.nan), out).astype(F32)


def muon_S(m) -> np.ndarray:
    """S = a I + b A + c A^2, A = m~ m~^T, m~ = m / ||m||, bf16 steps (data_selection.py:228-252).

    Each bf16 tensor op of the reference is a float64 evaluation rounded to
    bf16; float32-accumulated GEMMs may differ in the last bf16 bit.
    """
    mb = bf16_round(m).astype(np.float64)
    n = mb.shape[0]
    norm = bf16_round(np.float32(np.sqrt((mb * mb).sum()))).astype(np.float64)
    if norm < 1e-7:
        return np.eye(n, dtype=F32)
    mt = bf16_round((mb / norm).astype(F32)).astype(np.float64)
    A = bf16_round((mt @ mt.T).astype(F32)).astype(np.float64)
    A2 = bf16_round((A @ A).astype(F32)).astype(np.float64)
    a, b, c = 3.4445, -4.7750, 2.0315
    t1 = bf16_round((a * np.eye(n)).astype(F32)).astype(np.float64)
    t2 = bf16_round((b * A).astype(F32)).astype(np.float64)
    t3 = bf16_round((c * A2).astype(F32)).astype(np.float64)
    return bf16_round(bf16_round((t1 + t2).astype(F32)).astype(np.float64) + t3).astype(F32)


# ----------------------------------------------------------------- stage 2
def ghost_score(a, dLdZ, V) -> np.ndarray:
    """score_b = sum_t dLdZ[b,t] . (V a[b,t]) = <G_b, V>, float64 (V is [d_out, d_in])."""
    A = np.asarray(a, dtype=np.float64)
    G = np.asarray(dLdZ, dtype=np.float64)
    U = np.einsum("bti,oi->bto", A, np.asarray(V, dtype=np.float64), optimize=True)
    return np.einsum("bto,bto->b", U, G, optimize=True)


def layer_scores(dLdZ_t, a_t, dLdZ_v, a_v, h, s, k, C=1.0, layer_scale=1.0, diag=None, S=None,
                 per_val=False, projection=True):
    """One layer's score and similarity contributions (data_selection.py:478-588).

    projection=True: phi_t = CS(D o G_t) (candidates with the AdamW diagonal,
    Muon S applied to dLdZ_t), phi_v = CS(G_v) (proxies: no preconditioner);
    score += C ls mean_j phi_t . phi_vj; sim += (C ls)^2 phi_t phi_t^T.
    projection=False: the same inner products on dense per-sample gradients.
    """
    g_t = np.asarray(dLdZ_t, dtype=np.float64)
    if S is not None:
        g_t = g_t @ np.asarray(S, dtype=np.float64)
    c = float(F32(F32(C) * F32(layer_scale)))
    if projection:
        pt = project_full_gradient(g_t, a_t, h, s, k, diag=diag)
        pv = project_full_gradient(dLdZ_v, a_v, h, s, k)
    else:
        Gt = per_sample_grads(g_t, a_t).reshape(g_t.shape[0], -1)
        Gv = per_sample_grads(dLdZ_v, a_v).reshape(np.shape(dLdZ_v)[0], -1)
        pt = Gt * (1.0 if diag is None else np.asarray(diag, dtype=np.float64).reshape(1, -1))
        pv = Gv
    dots = pt @ pv.T
    score = c * dots if per_val else c * dots.mean(axis=1)
    if not projection and diag is not None:
        sim = c * c * (pt @ pt.T)
    else:
        sim = c * c * (pt @ pt.T)
    return score, sim


# ----------------------------------------------------------------- stage 5
def pairwise_sum_f32(a: np.ndarray) -> np.float32:
    """NumPy's float32 reduction order: 0 + pairwise(a), 8-accumulator blocks of <=128."""

    def leaf(x):
        n = len(x)
        if n < 8:
            r = F32(0.0)
            for v in x:
                r = F32(r + v)
            return r
        acc = [F32(x[j]) for j in range(8)]
        i = 8
        while i < n - (n % 8):
            for j in range(8):
                acc[j] = F32(acc[j] + x[i + j])
            i += 8
        r = F32(F32(F32(acc[0] + acc[1]) + F32(acc[2] + acc[3])) + F32(F32(acc[4] + acc[5]) + F32(acc[6] + acc[7])))
        while i < n:
            r = F32(r + x[i])
            i += 1
        return r

    def rec(x):
        n = len(x)
        if n <= 128:
            return leaf(x)
        n2 = n // 2
        n2 -= n2 % 8
        return F32(rec(x[:n2]) + rec(x[n2:]))

    return F32(F32(0.0) + rec(np.asarray(a, dtype=F32)))


def choice_from_uniform(p: np.ndarray, u: float) -> int:
    """np.random.choice(len(p), p=p) given its uniform draw u.

    RandomState.choice: p as float64, cdf = cumsum(p), cdf /= cdf[-1],
    index = searchsorted(cdf, u, side='right').  Raises ValueError as choice
    does when p does not sum to 1 within sqrt(eps) of its dtype.
    """
    p64 = np.asarray(p, dtype=np.float64)
    atol = max(np.sqrt(np.finfo(np.float64).eps), np.sqrt(np.finfo(np.asarray(p).dtype).eps))
    if np.isnan(p64).any():
        raise ValueError("probabilities contain NaN")
    if abs(p64.sum() - 1.0) > atol:
        raise ValueError("probabilities do not sum to 1")
    cdf = p64.cumsum()
    cdf /= cdf[-1]
    return int(cdf.searchsorted(u, side="right"))


def stochastic_greedy_selection(scores, interaction_matrix, K, temperature=1.0, uniforms=None):
    """Boltzmann sampling with interaction penalty (data_selection.py:641-675).

    Same float32 NumPy arithmetic as the reference; draw i uses uniforms[i]
    (the double np.random.choice would draw) or, if None, the global NumPy RNG.
    """
    scores = np.array(scores, dtype=F32, copy=True)
    sim = np.asarray(interaction_matrix, dtype=F32)
    n = len(scores)
    avail = np.ones(n, dtype=bool)
    picked = []
    for i in range(K):
        cur = scores[avail]
        x = cur / temperature
        if np.max(x) > 700:
            x = x - np.max(x)
        p = np.exp(x)
        tot = p.sum()
        if tot == 0 or not np.isfinite(tot):
            p = np.ones_like(p) / len(p)
        else:
            p /= tot
        idx_avail = np.where(avail)[0]
        u = np.random.random_sample() if uniforms is None else float(uniforms[i])
        sel = int(idx_avail[choice_from_uniform(p, u)])
        picked.append(sel)
        scores -= sim[sel, :]
        avail[sel] = False
    return picked


def greedy_selection(scores, interaction_matrix, K):
    """Argmax pick with interaction penalty (data_selection.py:622-638)."""
    scores = np.array(scores, dtype=F32, copy=True)
    sim = np.asarray(interaction_matrix, dtype=F32)
    picked = []
    for _ in range(K):
        i = int(np.argmax(scores))
        picked.append(i)
        scores -= sim[i, :]
        scores[i] = -np.inf
    return picked


# ------------------------------------------------------- candidate buffer stream
def candidate_buffers(file_tokens, buffer_size: int, world: int, n_buffers: int):
    """The reference's rank-0 buffer fill (train.py:1038-1079), then each rank's slice (:1081-1084).

    file_tokens: the payload of each training file in cycle order.  Rank 0
    keeps a current file and position, copies buffer_size * world + 1 tokens
    per buffer, moving to the next file (cyclically) whenever the current one
    cannot supply the rest.  Returns, per buffer, the list of every rank's
    [rank*B, rank*B + B + 1) slice as int32.
    """
    files = [np.asarray(t) for t in file_tokens]
    fi = 0
    tokens, pos = files[0], 0
    out = []
    for _ in range(n_buffers):
        needed = buffer_size * world + 1
        cand = np.empty(needed, dtype=np.int32)
        filled = 0
        while filled < needed:
            remaining = needed - filled
            if pos + remaining >= len(tokens):
                available = len(tokens) - pos
                if available > 0:
                    cand[filled:filled + available] = tokens[pos:].astype(np.int32)
                    filled += available
                fi = (fi + 1) % len(files)
                tokens, pos = files[fi], 0
            else:
                cand[filled:filled + remaining] = tokens[pos:pos + remaining].astype(np.int32)
                pos += remaining
                filled += remaining
        out.append([cand[r * buffer_size:r * buffer_size + buffer_size + 1] for r in range(world)])
    return out


# ------------------------------------------- redistribution of the selection
def redistribute_selected(global_idx, inputs_per_rank, targets_per_rank):
    """The reference's steps 5a-5e after a global selection (train.py:1181-1249).

    global_idx: the picks over the concatenated candidates of all ranks, the
    same on every rank.  inputs_per_rank / targets_per_rank: each rank's
    candidate rows [b, seq_len].  Each rank masks the picks that fall in its
    range (pick order kept), all ranks all-gather their selected rows padded
    to the largest count, concatenate the real rows in rank order and take an
    even share, the first (total % world) ranks one row more; a rank whose
    share is empty takes row 0 of the concatenation.  Returns each rank's
    (inputs, targets).
    """
    world = len(inputs_per_rank)
    b = inputs_per_rank[0].shape[0]
    g = np.asarray(global_idx, dtype=np.int64)
    sel_in, sel_tg = [], []
    for r in range(world):
        mask = (g >= r * b) & (g < r * b + b)
        local = g[mask] - r * b
        sel_in.append(inputs_per_rank[r][local])
        sel_tg.append(targets_per_rank[r][local])
    counts = [len(x) for x in sel_in]
    if sum(counts) > 0:
        all_in = np.concatenate([x for x, c in zip(sel_in, counts) if c > 0])
        all_tg = np.concatenate([x for x, c in zip(sel_tg, counts) if c > 0])
    out = []
    for r in range(world):
        if sum(counts) == 0:  # no picks at all: every rank keeps its own first row
            out.append((inputs_per_rank[r][:1], targets_per_rank[r][:1]))
            continue
        total = all_in.shape[0]
        per, rem = divmod(total, world)
        start = r * per + min(r, rem)
        cnt = per + (1 if r < rem else 0)
        end = start + cnt
        if cnt == 0:
            start, end = 0, 1
        out.append((all_in[start:end], all_tg[start:end]))
    return out
