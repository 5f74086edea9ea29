"""One global OPUS selection over a candidate batch sharded across ranks.

One process per GPU (torchrun), NCCL between them.  The reference's global
mode (train.py:1100-1178) all-gathers every rank's candidate token ids to
rank 0, which scores and selects the whole batch alone and broadcasts the
picks.  Here each rank scores the candidates it already holds:

1. rank 0's proxy batch is broadcast (as the reference does) and every rank
   takes a contiguous share of it; each rank sketches its share of the proxy
   gradient sum for every layer, and one all-reduce(sum) of the stacked
   [L, k] target sketches gives every rank the full target;
2. each rank computes its candidates' scores and their local similarity
   block (the Gram of its own sketches);
3. one all-gather of the scores [B_loc] and one of the local blocks
   [B_loc, B_loc];
4. every rank runs the same global draw -- the same uniforms, drawn from
   NumPy's global stream on rank 0 and broadcast -- over the gathered scores
   with the block-diagonal interaction matrix, so the picks agree without a
   broadcast; each rank keeps the picks that fall in its shard.

By default the similarity between candidates on different ranks is zero
(only scores and the local blocks cross GPUs), so the picks equal a
single-process selection over the concatenated scores with the
block-diagonal matrix.  With exact_similarity=True every rank also
all-gathers each layer's candidate sketches and forms its full row block of
the similarity, the row blocks are all-gathered, and the draw uses the dense
matrix: the picks are then those of the reference's global mode, which
scores every candidate on rank 0.  Every rank must hold the same number of
candidates.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from .. import ops
from . import data_selection as ds


def rank_and_world(group=None) -> tuple[int, int]:
    if not (dist.is_available() and dist.is_initialized()):
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous share [lo, hi) of n items for a rank; the first n % world ranks get one more."""
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def allreduce_target_sketches(taus: torch.Tensor, group=None) -> torch.Tensor:
    """Sum the ranks' partial proxy sketches [L, k] in place (NCCL all-reduce)."""
    if rank_and_world(group)[1] > 1:
        dist.all_reduce(taus, op=dist.ReduceOp.SUM, group=group)
    return taus


def gather_scores_and_blocks(score: torch.Tensor, sim: torch.Tensor, group=None):
    """All-gather scores [B_loc] -> [W*B_loc] and similarity blocks [B_loc, B_loc] -> [W, B_loc, B_loc]."""
    rank, world = rank_and_world(group)
    b = score.numel()
    if sim.shape != (b, b):
        raise ValueError(f"local similarity must be [{b}, {b}], got {tuple(sim.shape)}")
    score = score.reshape(-1).contiguous()
    sim = sim.contiguous()
    if world == 1:
        return score, sim.unsqueeze(0)
    scores = [torch.empty_like(score) for _ in range(world)]
    blocks = [torch.empty_like(sim) for _ in range(world)]
    dist.all_gather(scores, score, group=group)
    dist.all_gather(blocks, sim, group=group)
    return torch.cat(scores), torch.stack(blocks)


def gather_scores(score: torch.Tensor, group=None) -> torch.Tensor:
    _, world = rank_and_world(group)
    score = score.reshape(-1).contiguous()
    if world == 1:
        return score
    parts = [torch.empty_like(score) for _ in range(world)]
    dist.all_gather(parts, score, group=group)
    return torch.cat(parts)


def shared_uniforms(n_select: int, device, group=None, src: int = 0) -> torch.Tensor:
    """n_select doubles from rank src's NumPy global stream (np.random.choice's draws), on every rank."""
    rank, world = rank_and_world(group)
    u = torch.empty(n_select, dtype=torch.float64)
    if rank == src:
        u = torch.from_numpy(np.random.random_sample(n_select).astype(np.float64))
    u = u.to(device)
    if world > 1:
        dist.broadcast(u, src=dist.get_global_rank(group, src) if group is not None else src, group=group)
    return u


def local_picks(global_idx: torch.Tensor, rank: int, b_local: int) -> torch.Tensor:
    """The picks that fall in this rank's shard, as local indices (pick order kept)."""
    lo = rank * b_local
    mask = (global_idx >= lo) & (global_idx < lo + b_local)
    return global_idx[mask] - lo


def redistribution_plan(global_idx, b_local: int, world: int) -> list[list[tuple[int, int]]]:
    """Every rank's share of the selected rows as (source rank, local row), in receive order.

    The reference's global mode (train.py:1184-1247) orders the selected rows
    by source rank, pick order inside a rank, and gives rank d the rows
    [d*per + min(d, rem), that + per + (d < rem)) of that order, with
    per, rem = divmod(total, world); a rank whose share is empty takes the
    first row of the order.  With no picks at all every rank keeps its own
    row 0.
    """
    idx = [int(g) for g in global_idx]
    if any(g < 0 or g >= b_local * world for g in idx):
        raise ValueError(f"global indices must lie in [0, {b_local * world})")
    by_source: list[list[int]] = [[] for _ in range(world)]
    for g in idx:
        by_source[g // b_local].append(g % b_local)
    order = [(q, i) for q in range(world) for i in by_source[q]]
    if not order:
        return [[(d, 0)] for d in range(world)]
    per, rem = divmod(len(order), world)
    shares = []
    for d in range(world):
        start, cnt = d * per + min(d, rem), per + (1 if d < rem else 0)
        shares.append(order[start:start + cnt] if cnt else order[:1])
    return shares


def redistribute_selected(global_idx, inputs: torch.Tensor, targets: torch.Tensor, group=None):
    """This rank's share of the globally selected sequences (train.py:1181-1249).

    inputs / targets: this rank's candidate rows [b, seq_len] (every rank the
    same b); global_idx: the picks over all ranks' candidates, the same on
    every rank.  The reference all-gathers every rank's selected rows padded
    to the largest count and keeps a slice; here every rank derives the whole
    plan from the picks it already has, and one all_to_all of the packed
    rows (inputs and targets side by side as bytes) moves each row that
    changes rank exactly once, with no padding.  Returns (inputs, targets) of
    this rank's share, on the inputs' device, equal to the reference's.
    """
    rank, world = rank_and_world(group)
    if inputs.shape[0] != targets.shape[0]:
        raise ValueError("inputs and targets must hold the same number of rows")
    b = inputs.shape[0]
    picks = global_idx.tolist() if torch.is_tensor(global_idx) else list(global_idx)
    shares = redistribution_plan(picks, b, world)
    device = inputs.device
    if world == 1:
        rows = torch.tensor([i for _, i in shares[0]], dtype=torch.long, device=device)
        return inputs.index_select(0, rows), targets.index_select(0, rows)
    send = [[i for q, i in shares[d] if q == rank] for d in range(world)]
    rows = torch.tensor([i for part in send for i in part], dtype=torch.long, device=device)
    recv = [sum(1 for q, _ in shares[rank] if q == src) for src in range(world)]
    x = inputs.index_select(0, rows).contiguous().view(torch.uint8)
    y = targets.index_select(0, rows).contiguous().view(torch.uint8)
    nx = x.shape[1]
    packed = torch.cat([x, y], dim=1)
    out = torch.empty(sum(recv), packed.shape[1], dtype=torch.uint8, device=device)
    dist.all_to_all_single(out, packed, recv, [len(part) for part in send], group=group)
    # fresh row-major storage: a one-row slice keeps its offset and row stride into out
    got_x = torch.empty(out.shape[0], nx, dtype=torch.uint8, device=device).copy_(out[:, :nx])
    got_y = torch.empty(out.shape[0], out.shape[1] - nx, dtype=torch.uint8, device=device).copy_(out[:, nx:])
    return got_x.view(inputs.dtype), got_y.view(targets.dtype)


def gather_sketches(phi: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather one layer's candidate sketches [B_loc, k] -> [W*B_loc, k] in rank order."""
    _, world = rank_and_world(group)
    phi = phi.contiguous()
    if world == 1:
        return phi
    parts = [torch.empty_like(phi) for _ in range(world)]
    dist.all_gather(parts, phi, group=group)
    return torch.cat(parts)


def gather_similarity_rows(sim_rows: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather row blocks [B_loc, W*B_loc] of the dense similarity -> [W*B_loc, W*B_loc]."""
    _, world = rank_and_world(group)
    sim_rows = sim_rows.contiguous()
    if world == 1:
        return sim_rows
    parts = [torch.empty_like(sim_rows) for _ in range(world)]
    dist.all_gather(parts, sim_rows, group=group)
    return torch.cat(parts)


def select_global(score: torch.Tensor, sim: torch.Tensor, n_select: int, method: str = "stochastic",
                  temperature: float = 1.0, uniforms: torch.Tensor | None = None, group=None):
    """Steps 3-4: gather, then the identical global draw on every rank.

    score [B_loc] is this rank's; sim is its local block [B_loc, B_loc], or
    its row block [B_loc, W*B_loc] of the dense similarity (exact global
    similarity).  Returns (global indices [n_select] int64, this rank's picks
    as local indices).
    """
    rank, world = rank_and_world(group)
    b = score.numel()
    if sim.dim() == 2 and sim.shape == (b, b * world) and world > 1:
        scores = gather_scores(score, group)
        blocks = gather_similarity_rows(sim, group)
    else:
        scores, blocks = gather_scores_and_blocks(score, sim, group)
    n = scores.numel()
    if method == "greedy":
        idx = ops.greedy_select(scores, blocks, int(n_select))
    elif method == "stochastic":
        if n_select > n:
            raise ValueError("zero-size array to reduction operation maximum which has no identity")
        if uniforms is None:
            uniforms = shared_uniforms(int(n_select), scores.device, group)
        idx = ops.boltzmann_select(scores, blocks, int(n_select), float(temperature), uniforms)
        ops.check_device_error("global stochastic_greedy_selection")
    else:
        raise ValueError(f"Unknown selection method: {method}")
    return idx, local_picks(idx, rank, score.numel())


def broadcast_batch(batch: dict | None, device, group=None, src: int = 0) -> dict:
    """Rank src's proxy batch dict (input_ids int32/int64, labels int64, [n, T]) on every rank."""
    rank, world = rank_and_world(group)
    if world == 1:
        return batch
    keys = ("input_ids", "labels")
    meta = torch.zeros(4, dtype=torch.int64, device=device)
    if rank == src:
        ids = batch["input_ids"]
        meta[0], meta[1] = ids.shape[0], ids.shape[1]
        meta[2] = 1 if ids.dtype == torch.int64 else 0
    dist.broadcast(meta, src=src, group=group)
    n, t, ids64 = int(meta[0]), int(meta[1]), int(meta[2])
    if rank == src:
        out = {key: batch[key].to(device).contiguous() for key in keys}
    else:
        out = {"input_ids": torch.empty(n, t, dtype=torch.int64 if ids64 else torch.int32, device=device),
               "labels": torch.empty(n, t, dtype=torch.int64, device=device)}
    for key in keys:
        dist.broadcast(out[key], src=src, group=group)
    out["attention_mask"] = torch.ones_like(out["input_ids"])
    return out


def score_shard(model, device, batch_train, proxy_share, n_proxy_total, optimizer, trainable_layers,
                preconditioner="adamw", score_len=512, group=None, exact_similarity=False):
    """Steps 1-2 on one rank: scores [B_loc] and similarity.

    proxy_share is this rank's rows of the round's proxy batch (possibly
    none); the per-layer proxy sketch sums are all-reduced so every rank
    scores against the mean over all n_proxy_total proxies.  The similarity
    is the local block [B_loc, B_loc], or with exact_similarity the row block
    [B_loc, W*B_loc] against every rank's candidates (one all-gather of the
    sketches per layer).  Needs the CountSketch projector
    (initialize_projector(enabled=True)).

    With the streaming capture (the default) each layer is sketched from a
    backward hook, as in the single-process path, so no layer's dL/dZ
    outlives its hook; only the candidate sketches [B_loc, k] of every layer
    are kept until the one all-reduce of the target sketches after the
    backward.  The batch capture (one autograd call over every layer) is the
    fallback when a hook cannot fire.
    """
    projector = ds.get_projector()
    if projector is None or not projector.enabled:
        raise ValueError("sharded selection needs the CountSketch projector (initialize_projector(enabled=True))")
    _, world = rank_and_world(group)

    def shaped(pl):
        if pl.g_t.dim() == 2:
            return pl.g_t.unsqueeze(1), pl.a_t.unsqueeze(1), pl.g_v.unsqueeze(1), pl.a_v.unsqueeze(1)
        return pl.g_t, pl.a_t, pl.g_v, pl.a_v

    rows = batch_train["input_ids"].shape[0] + (proxy_share["input_ids"].shape[0] if proxy_share else 0)
    seq = min(batch_train["input_ids"].shape[1], score_len or 1 << 30)
    if ds.CAPTURE_MODE == "stream" and ds._use_passes(rows, trainable_layers, seq, device, model,
                                                      ds._has_muon(optimizer, preconditioner)):
        # the rank's rows do not fit one capture: proxy passes, one all-reduce, candidate passes
        score, phis, cs, _ = ds.capture_in_passes(
            model, device, batch_train, proxy_share, optimizer, trainable_layers, preconditioner, score_len,
            reduce_targets=lambda t: allreduce_target_sketches(t, group), n_proxy_total=n_proxy_total)
        b = phis.shape[1]
        sim = torch.zeros(b, b * world if exact_similarity else b, device=device, dtype=torch.float32)
        for pid in range(phis.shape[0]):
            other = gather_sketches(phis[pid], group) if exact_similarity else phis[pid]
            ops.sketch_gram(phis[pid], other, alpha=cs[pid] * cs[pid], out=sim, accumulate=True)
        return score, sim

    state = {}

    def make_handler(train_bs, val_bs, n_plans):
        taus = torch.zeros(n_plans, projector.sketch_dim, device=device, dtype=torch.float32)
        sim = torch.zeros(train_bs, train_bs * world if exact_similarity else train_bs, device=device,
                          dtype=torch.float32)
        state.update(train_bs=train_bs, taus=taus, sim=sim, phis=[None] * n_plans, cs=[0.0] * n_plans)

        def on_plan(pl):
            g_t, a_t, g_v, a_v = shaped(pl)
            if g_v.shape[0] > 0:
                projector.sketch(g_v, a_v, pl.pid, rows_div=g_v.shape[0], out=taus[pl.pid:pl.pid + 1],
                                 accumulate=True)
            phi_t = projector.sketch(g_t, a_t, pl.pid, exp_avg_sq=pl.exp_avg_sq, eps=pl.eps)
            state["phis"][pl.pid], state["cs"][pl.pid] = phi_t, pl.c
            if not exact_similarity:
                ops.sketch_gram(phi_t, alpha=pl.c * pl.c, out=sim, accumulate=True)
        return on_plan

    streamed = ds.CAPTURE_MODE == "stream" and ds.stream_capture(
        model, device, batch_train, proxy_share, optimizer, trainable_layers, preconditioner, score_len,
        make_handler)
    if not streamed:
        state.clear()
        pairs, train_bs, _ = ds.capture_pairs(model, batch_train, None, trainable_layers, score_len,
                                              batch_val=proxy_share)
        plans = ds.plan_layers(pairs, optimizer, preconditioner, device)
        del pairs
        on_plan = make_handler(train_bs, None, len(plans))
        for pl in plans:
            on_plan(pl)
        del plans
    taus, sim, phis, cs, train_bs = state["taus"], state["sim"], state["phis"], state["cs"], state["train_bs"]
    allreduce_target_sketches(taus, group)
    score = torch.zeros(train_bs, device=device, dtype=torch.float32)
    for pid, phi_t in enumerate(phis):  # the pair ids' forward order, on every rank
        if n_proxy_total > 0:
            ops.sketch_dot(phi_t, taus[pid], alpha=cs[pid] / n_proxy_total, out=score, accumulate=True)
        if exact_similarity:
            ops.sketch_gram(phi_t, gather_sketches(phi_t, group), alpha=cs[pid] * cs[pid], out=sim, accumulate=True)
        phis[pid] = None
    return score, sim


def get_batch_opus_global(model, buffer_seq, buffer_labels, optimizer, trainable_layers, validation_loader,
                          selection_ratio, seq_len, selection_method="greedy", temperature=1.5, score_len=512,
                          preconditioner="adamw", group=None, exact_similarity=False):
    """One global OPUS selection over the candidates of all ranks (the global mode of train.py:1100-1178).

    Every rank passes its own candidate shard (the same number of sequences
    on every rank).  Returns (global indices [K] on every rank, this rank's
    picks as indices into its buffer), K = max(1, int(N_global * ratio)).
    exact_similarity: the dense cross-rank similarity (the reference's global
    mode) instead of the block-diagonal one.
    """
    rank, world = rank_and_world(group)
    device = buffer_seq.device
    score_len = min(score_len, seq_len)
    if buffer_seq.dim() == 1:
        n = buffer_seq.numel() // seq_len
        buffer_seq = buffer_seq[: n * seq_len].view(n, seq_len)
        buffer_labels = buffer_labels[: n * seq_len].view(n, seq_len)
    b_local = buffer_seq.shape[0]
    proxy = ds._sample_proxy_batch_for_step(validation_loader) if rank == 0 else None
    proxy = broadcast_batch(proxy, device, group)
    n_proxy = proxy["input_ids"].shape[0]
    lo, hi = shard_range(n_proxy, rank, world)
    share = {key: v[lo:hi] for key, v in proxy.items()}
    # the score windows of get_batch_opus (identity when score_len == seq_len)
    gen = ds.make_window_generator(step=ds._GBG_CALL_ID, rank=rank, device=device.type)
    ds._GBG_CALL_ID += 1
    win_inputs, idx = ds._random_windows(buffer_seq, score_len, align_to=128, g=gen)
    batch_train = {"input_ids": win_inputs, "attention_mask": torch.ones_like(win_inputs),
                   "labels": buffer_labels.gather(1, idx)}
    score, sim = score_shard(model, device, batch_train, share, n_proxy, optimizer, trainable_layers,
                             preconditioner=preconditioner, score_len=score_len, group=group,
                             exact_similarity=exact_similarity)
    n_select = max(1, int(b_local * world * selection_ratio))
    return select_global(score, sim, n_select, method=selection_method, temperature=temperature, group=group)
