"""Sharded global selection on two or more GPUs over NCCL (skipped with fewer GPUs).

Each rank scores its candidate shard with the device kernels, the proxy
sketches are all-reduced and the scores and local similarity blocks are
all-gathered; the gathered scores must match the reference's single-process
scores, and every rank must draw the same picks as the oracle on the gathered
block-diagonal data; the selected rows then reach the ranks the reference's
redistribution gives them.
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

pytestmark = pytest.mark.gpu
N_PICK = 3
NP_SEED = 11


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, scenario, out_q, capture_rows=None):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    ds.CAPTURE_ROWS = capture_rows  # a small count splits each rank's capture into passes
    try:
        g = load_golden(f"wholepath_{scenario}")
        model, opt, loader, batch = rebuild(g, device=dev)
        ds.initialize_projector(sketch_dim=1024, seed=42, device="cpu", enabled=True)
        layers = ds.find_GClayers(model)
        b = batch["input_ids"].shape[0] // world
        mine = {key: v[rank * b:(rank + 1) * b] for key, v in batch.items()}
        proxy = sd.broadcast_batch(loader._fixed_batch if rank == 0 else None, dev)
        n = proxy["input_ids"].shape[0]
        lo, hi = sd.shard_range(n, rank, world)
        share = {key: v[lo:hi] for key, v in proxy.items()}
        score, sim = sd.score_shard(model, dev, mine, share, n, opt, layers, preconditioner=str(g["precond"]),
                                    score_len=128)
        scores, blocks = sd.gather_scores_and_blocks(score, sim)
        np.random.seed(NP_SEED)
        gidx, lidx = sd.select_global(score, sim, N_PICK, method="stochastic", temperature=1.0)
        ggreedy, _ = sd.select_global(score, sim, N_PICK, method="greedy")
        # exact global similarity: row blocks against every rank's sketches
        score_x, rows = sd.score_shard(model, dev, mine, share, n, opt, layers, preconditioner=str(g["precond"]),
                                       score_len=128, exact_similarity=True)
        dense = sd.gather_similarity_rows(rows)
        np.random.seed(NP_SEED)
        gexact, _ = sd.select_global(score_x, rows, N_PICK, method="stochastic", temperature=1.0)
        # the whole public call: same picks on every rank
        np.random.seed(NP_SEED)
        cand = batch["input_ids"][rank * b:(rank + 1) * b]
        full_idx, _ = sd.get_batch_opus_global(model, cand, cand.clone(), opt, layers, loader, 0.5, 128,
                                               selection_method="stochastic", temperature=1.0, score_len=128,
                                               preconditioner=str(g["precond"]))
        # the selected rows moved to their ranks (one all_to_all over NCCL)
        rx, ry = sd.redistribute_selected(full_idx, cand.to(torch.int32), cand.to(torch.int64) + 1)
        torch.cuda.synchronize()
        out_q.put((rank, scores.cpu().numpy(), blocks.cpu().numpy(), gidx.cpu().tolist(), lidx.cpu().tolist(),
                   ggreedy.cpu().tolist(), full_idx.cpu().tolist(), dense.cpu().numpy(), gexact.cpu().tolist(),
                   cand.cpu().numpy(), rx.cpu().numpy(), ry.cpu().numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("scenario,capture_rows", [("adamw_proj", None), ("muon_proj", None), ("muon_proj", 1)])
def test_sharded_selection_on_gpus(scenario, capture_rows):
    world = min(torch.cuda.device_count(), 3)
    if world < 2:
        pytest.skip("needs two or more GPUs")
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, scenario, out_q, capture_rows))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, *rest = out_q.get(timeout=240)
            results[rank] = rest
    except queue.Empty:
        pytest.fail("a rank did not report")
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    g = load_golden(f"wholepath_{scenario}")
    b = g["cand"].shape[0] // world
    scores, blocks = results[0][0], results[0][1]
    assert_close_scores(scores, g["scores"])
    for q in range(world):
        assert_close_scores(blocks[q], g["sim"][q * b:(q + 1) * b, q * b:(q + 1) * b])
    dense = np.zeros((world * b, world * b), np.float32)
    for q in range(world):
        dense[q * b:(q + 1) * b, q * b:(q + 1) * b] = blocks[q]
    uni = np.random.RandomState(NP_SEED).random_sample(N_PICK)
    want = orc.stochastic_greedy_selection(scores.astype(np.float32), dense, N_PICK, temperature=1.0, uniforms=uni)
    want_greedy = orc.greedy_selection(scores.astype(np.float32), dense, N_PICK)
    want_exact = orc.stochastic_greedy_selection(scores.astype(np.float32), g["sim"].astype(np.float32), N_PICK,
                                                 temperature=1.0, uniforms=uni)
    cands = [results[r][8].astype(np.int32) for r in range(world)]
    moved = orc.redistribute_selected(results[0][5], cands, [c.astype(np.int64) + 1 for c in cands])
    mapped = []
    for r in range(world):
        _, _, gidx, lidx, ggreedy, full_idx, dense_r, gexact, _, rx, ry = results[r]
        np.testing.assert_array_equal(rx, moved[r][0])
        np.testing.assert_array_equal(ry, moved[r][1])
        assert_close_scores(dense_r, g["sim"])  # the reference's whole-batch similarity
        assert gexact == want_exact
        assert gidx == want and ggreedy == want_greedy
        assert full_idx == results[0][5]
        mapped += [r * b + i for i in lidx]
    assert sorted(mapped) == sorted(want)
