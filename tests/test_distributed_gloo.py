"""Sharded global selection over gloo ranks on the CPU (no GPU).

Each rank captures its own candidates and its share of the proxy batch, the
per-layer proxy sketches are all-reduced, scores and local similarity blocks
are all-gathered and every rank draws the same picks.  The sketch arithmetic
here is the oracle's (the device kernels are covered by the GPU tests); what
is under test is the choreography: sharded capture, the collectives, the
shared uniforms and the local/global index mapping.  The gathered scores must
equal the reference's single-process scores of the whole batch.
"""
import os
import queue
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import load_golden
from oracle import opus_oracle as orc
from opus_b200.train import data_selection as ds
from opus_b200.train import distributed as sd
from test_host_logic import assert_close_scores, rebuild

K_SKETCH = 1024
N_PICK = 3
NP_SEED = 11


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def block_diag(blocks: np.ndarray) -> np.ndarray:
    q, b, _ = blocks.shape
    out = np.zeros((q * b, q * b), blocks.dtype)
    for r in range(q):
        out[r * b:(r + 1) * b, r * b:(r + 1) * b] = blocks[r]
    return out


def _rank_worker(rank, world, port, scenario, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(1)
    from opus_b200 import ops
    from oracle import reference_torch as rt

    # CPU ranks: the Muon S and transform from the reference's torch recipe (the kernels need a GPU)
    ops.muon_S, ops.muon_transform = rt.muon_S, rt.muon_transform
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        g = load_golden(f"wholepath_{scenario}")
        model, opt, loader, batch = rebuild(g)
        layers = ds.find_GClayers(model)
        b = batch["input_ids"].shape[0] // world
        mine = {key: v[rank * b:(rank + 1) * b] for key, v in batch.items()}
        proxy = sd.broadcast_batch(loader._fixed_batch if rank == 0 else None, torch.device("cpu"))
        n = proxy["input_ids"].shape[0]
        lo, hi = sd.shard_range(n, rank, world)
        share = {key: v[lo:hi] for key, v in proxy.items()}
        pairs, bt, nv = ds.capture_pairs(model, mine, None, layers, score_len=128, batch_val=share)
        assert (bt, nv) == (b, hi - lo)
        plans = ds.plan_layers(pairs, opt, str(g["precond"]), "cpu")
        taus = torch.zeros(len(plans), K_SKETCH, dtype=torch.float64)
        phis = []
        for li, pl in enumerate(plans):
            d_out, d_in = pl.g_t.shape[-1], pl.a_t.shape[-1]
            h, s = orc.hash_sign_tables(d_out * d_in, pl.pid, K_SKETCH, seed=42)
            diag = None if pl.exp_avg_sq is None else orc.inv_rms(pl.exp_avg_sq.numpy(), pl.eps)
            phis.append(orc.project_full_gradient(pl.g_t.float().numpy(), pl.a_t.numpy(), h, s, K_SKETCH, diag=diag))
            if nv:
                pv = orc.project_full_gradient(pl.g_v.numpy(), pl.a_v.numpy(), h, s, K_SKETCH)
                taus[li] = torch.from_numpy(pv.sum(axis=0))
        sd.allreduce_target_sketches(taus)
        score = np.zeros(b)
        sim = np.zeros((b, b))
        rows = np.zeros((b, b * world))  # exact global similarity: this rank's row block
        for li, pl in enumerate(plans):
            c = float(np.float32(pl.c))
            score += c / n * (phis[li] @ taus[li].numpy())
            sim += c * c * (phis[li] @ phis[li].T)
            every = sd.gather_sketches(torch.from_numpy(phis[li])).numpy()
            rows += c * c * (phis[li] @ every.T)
        scores, blocks = sd.gather_scores_and_blocks(torch.from_numpy(score), torch.from_numpy(sim))
        dense = sd.gather_similarity_rows(torch.from_numpy(rows)).numpy()
        np.random.seed(NP_SEED)  # only rank 0's stream is drawn from
        u = sd.shared_uniforms(N_PICK, torch.device("cpu"))
        picks = orc.stochastic_greedy_selection(scores.numpy().astype(np.float32),
                                                block_diag(blocks.numpy()).astype(np.float32), N_PICK,
                                                temperature=1.0, uniforms=u.numpy())
        local = sd.local_picks(torch.tensor(picks, dtype=torch.int64), rank, b).tolist()
        exact_picks = orc.stochastic_greedy_selection(scores.numpy().astype(np.float32), dense.astype(np.float32),
                                                      N_PICK, temperature=1.0, uniforms=u.numpy())
        out_q.put((rank, scores.numpy(), blocks.numpy(), u.numpy(), picks, local, dense, exact_picks))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(180)
@pytest.mark.parametrize("scenario,world", [("adamw_proj", 2), ("muon_proj", 3), ("sgd_proj", 2)])
def test_sharded_selection_choreography(scenario, world):
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_worker, args=(r, world, port, scenario, out_q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, *rest = out_q.get(timeout=150)
            results[rank] = rest
    except queue.Empty:
        pytest.fail("a rank did not report")
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    g = load_golden(f"wholepath_{scenario}")
    B = g["cand"].shape[0]
    b = B // world
    want_u = np.random.RandomState(NP_SEED).random_sample(N_PICK)
    picks0 = results[0][3]
    mapped = []
    for r in range(world):
        scores, blocks, u, picks, local, dense, exact_picks = results[r]
        assert_close_scores(dense, g["sim"])  # exact global similarity == the reference's whole-batch matrix
        assert exact_picks == results[0][6]
        assert_close_scores(scores, g["scores"])  # sharded scores == the reference's whole-batch scores
        for q in range(world):
            assert_close_scores(blocks[q], g["sim"][q * b:(q + 1) * b, q * b:(q + 1) * b])
        np.testing.assert_array_equal(u, want_u)
        assert picks == picks0
        mapped += [r * b + i for i in local]
    assert sorted(mapped) == sorted(picks0)


def test_shard_range_covers_every_item_once():
    for n in range(0, 23):
        for world in range(1, 6):
            parts = [sd.shard_range(n, r, world) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(parts[r][1] == parts[r + 1][0] for r in range(world - 1))
            sizes = [hi - lo for lo, hi in parts]
            assert max(sizes) - min(sizes) <= 1


def test_local_picks_keep_order():
    idx = torch.tensor([7, 2, 5, 3, 6], dtype=torch.int64)
    assert sd.local_picks(idx, 0, 4).tolist() == [2, 3]
    assert sd.local_picks(idx, 1, 4).tolist() == [3, 1, 2]


def test_single_process_gather_is_identity():
    s = torch.arange(4, dtype=torch.float32)
    m = torch.eye(4)
    scores, blocks = sd.gather_scores_and_blocks(s, m)
    assert torch.equal(scores, s) and blocks.shape == (1, 4, 4)
    with pytest.raises(ValueError):
        sd.gather_scores_and_blocks(s, torch.eye(3))


def _redistribution_case(world, b, T, picks, seed):
    rng = np.random.default_rng(seed)
    inputs = [rng.integers(0, 50257, (b, T)).astype(np.int32) for _ in range(world)]
    targets = [rng.integers(-100, 50257, (b, T)).astype(np.int64) for _ in range(world)]
    return inputs, targets, orc.redistribute_selected(picks, inputs, targets)


REDISTRIBUTION_CASES = [
    (2, 6, 5, [7, 1, 3, 11, 0, 8]),      # mixed sources, pick order kept inside a source
    (3, 4, 3, [9]),                       # one pick: ranks 1 and 2 take row 0 of the order
    (3, 4, 3, [5, 6, 4, 7]),              # every pick on rank 1
    (4, 8, 2, list(range(31, -1, -2))),   # total % world == 0
    (4, 3, 4, [2, 11, 5, 6, 0]),          # remainder 1
]


@pytest.mark.parametrize("world,b,T,picks", REDISTRIBUTION_CASES)
def test_redistribution_plan_matches_reference(world, b, T, picks):
    inputs, targets, want = _redistribution_case(world, b, T, picks, seed=world * 100 + b)
    shares = sd.redistribution_plan(picks, b, world)
    for d in range(world):
        got_in = np.stack([inputs[q][i] for q, i in shares[d]])
        got_tg = np.stack([targets[q][i] for q, i in shares[d]])
        np.testing.assert_array_equal(got_in, want[d][0])
        np.testing.assert_array_equal(got_tg, want[d][1])
    with pytest.raises(ValueError):
        sd.redistribution_plan([b * world], b, world)


def _redistribute_worker(rank, world, port, b, T, picks, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        inputs, targets, _ = _redistribution_case(world, b, T, picks, seed=world * 100 + b)
        x, y = sd.redistribute_selected(torch.tensor(picks), torch.from_numpy(inputs[rank]),
                                        torch.from_numpy(targets[rank]))
        out_q.put((rank, x.numpy(), y.numpy(), str(x.dtype), str(y.dtype)))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(180)
@pytest.mark.parametrize("world,b,T,picks", REDISTRIBUTION_CASES[:3])
def test_redistribute_selected_over_gloo(world, b, T, picks):
    """One all_to_all of the packed rows gives every rank the reference's share."""
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_redistribute_worker, args=(r, world, port, b, T, picks, out_q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, *rest = out_q.get(timeout=150)
            results[rank] = rest
    except queue.Empty:
        pytest.fail("a rank did not report")
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    _, _, want = _redistribution_case(world, b, T, picks, seed=world * 100 + b)
    for r in range(world):
        x, y, dx, dy = results[r]
        assert (dx, dy) == ("torch.int32", "torch.int64")
        np.testing.assert_array_equal(x, want[r][0])
        np.testing.assert_array_equal(y, want[r][1])


def test_redistribute_selected_single_process():
    inputs, targets, want = _redistribution_case(1, 5, 3, [4, 0, 2], seed=1)
    x, y = sd.redistribute_selected(torch.tensor([4, 0, 2]), torch.from_numpy(inputs[0]),
                                    torch.from_numpy(targets[0]))
    np.testing.assert_array_equal(x.numpy(), want[0][0])
    np.testing.assert_array_equal(y.numpy(), want[0][1])
