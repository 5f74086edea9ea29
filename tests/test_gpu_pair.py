"""The CTA-pair sketch GEMM (OPUS_SKETCH_PAIR=1: tcgen05.mma.cta_group::2 over 256 x 256 tiles)
against the oracle and the one-CTA kernel (GPU).

Shapes cover an odd o-block count (the pair's second o-block lies past d_out), a
sketch larger than shared memory (L2 updates above the on-chip prefix), both tile
walks, summed rows (rows_div) and the f32 split path.
"""
import numpy as np
import pytest
import torch

from oracle import opus_oracle as orc
from opus_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def tables(numel, pid, k):
    h, s = orc.hash_sign_tables(numel, pid, k, seed=42, device=DEV)
    packed = ops.pack_hash_sign(torch.from_numpy(h).to(DEV), torch.from_numpy(s).to(DEV), k)
    return h, s, packed


def rel_err(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-30))


PAIR_SHAPES = [
    # B, T, d_out, d_in, k
    (2, 64, 256, 256, 4096),       # one o-block pair, one column block
    (3, 100, 384, 512, 8192),      # three o-blocks: the second pair has no second o-block
    (2, 130, 520, 264, 1000),      # ragged rows and columns, odd k
    (4, 64, 256, 1024, 65536),     # sketch larger than shared memory
    (2, 70, 640, 384, 131072),     # five o-blocks, k = 131072
    (5, 33, 1024, 256, 16384),     # many rows, short sequences
    (3, 1, 256, 512, 32768),       # one token per row: a single, mostly zero-filled k-block
    (2, 65, 384, 256, 65536),      # one token past a 64-token stage
]


@pytest.mark.parametrize("stage_tokens", ["64", "32"])
@pytest.mark.parametrize("B,T,d_out,d_in,k", PAIR_SHAPES)
def test_pair_sketch_matches_oracle(B, T, d_out, d_in, k, stage_tokens, monkeypatch):
    monkeypatch.setenv("OPUS_SKETCH_PAIR", "1")
    monkeypatch.setenv("OPUS_SKETCH_PAIR_STAGE_TOKENS", stage_tokens)
    torch.manual_seed(B * 7 + d_out)
    g = (torch.randn(B, T, d_out, device=DEV) * 1e-3).bfloat16()
    a = torch.randn(B, T, d_in, device=DEV).bfloat16()
    h, s, packed = tables(d_out * d_in, 2, k)
    diag = torch.rand(d_out, d_in, device=DEV) * 1e-3 + 1e-6
    table = ops.build_sketch_table(packed, d_out, d_in, diag=diag)
    load = ops.bucket_max_load(packed, k)
    phi = ops.sketch_gemm(g, a, table, k, max_bucket_load=load)
    ops.check_device_error("pair sketch_gemm")
    want = orc.project_full_gradient(g.float().cpu().numpy(), a.float().cpu().numpy(), h, s, k,
                                     diag=diag.cpu().numpy())
    assert rel_err(phi.cpu().numpy(), want) <= 1e-4
    # the global-atomic path (no fixed point) through the pair as well
    plain = ops.sketch_gemm(g, a, table, k, max_bucket_load=0)
    ops.check_device_error("pair sketch_gemm, f32 atomics")
    assert rel_err(plain.cpu().numpy(), want) <= 1e-4


@pytest.mark.parametrize("order", ["ob", "cb"])
def test_pair_walks_and_rows_div_match_one_cta(order, monkeypatch):
    """Both walks, summed rows and accumulation: the pair equals the one-CTA kernel."""
    B, T, d_out, d_in, k = 6, 96, 768, 1280, 65536
    torch.manual_seed(5)
    g = (torch.randn(B, T, d_out, device=DEV) * 1e-3).bfloat16()
    a = torch.randn(B, T, d_in, device=DEV).bfloat16()
    _, _, packed = tables(d_out * d_in, 6, k)
    table = ops.build_sketch_table(packed, d_out, d_in, exp_avg_sq=torch.full((d_out, d_in), 1e-4, device=DEV))
    load = ops.bucket_max_load(packed, k)
    one = ops.sketch_gemm(g, a, table, k, max_bucket_load=load)
    one_div = ops.sketch_gemm(g, a, table, k, rows_div=3, max_bucket_load=load)
    monkeypatch.setenv("OPUS_SKETCH_PAIR", "1")
    monkeypatch.setenv("OPUS_SKETCH_ORDER", order)
    two = ops.sketch_gemm(g, a, table, k, max_bucket_load=load)
    two_div = ops.sketch_gemm(g, a, table, k, rows_div=3, max_bucket_load=load)
    ops.sketch_gemm(g, a, table, k, out=two, accumulate=True, max_bucket_load=load)
    ops.check_device_error("pair sketch_gemm walks")
    assert rel_err(two_div.cpu().numpy(), one_div.cpu().numpy()) <= 1e-5
    assert rel_err(two.cpu().numpy(), 2 * one.cpu().numpy()) <= 1e-5


def test_pair_f32_split_inputs(monkeypatch):
    monkeypatch.setenv("OPUS_SKETCH_PAIR", "1")
    B, T, d_out, d_in, k = 3, 50, 384, 264, 2048
    torch.manual_seed(9)
    g = torch.randn(B, T, d_out, device=DEV) * 1e-2
    a = torch.randn(B, T, d_in, device=DEV)
    h, s, packed = tables(d_out * d_in, 1, k)
    table = ops.build_sketch_table(packed, d_out, d_in)
    phi = ops.sketch_gemm(g, a, table, k, max_bucket_load=ops.bucket_max_load(packed, k))
    ops.check_device_error("pair sketch_gemm, f32 split")
    want = orc.project_full_gradient(g.cpu().numpy(), a.cpu().numpy(), h, s, k)
    assert rel_err(phi.cpu().numpy(), want) <= 1e-4
