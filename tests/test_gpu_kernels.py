"""Parity of the sm_100a kernels with the oracle (GPU)."""
import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import opus_oracle as orc
from opus_b200 import ops
from opus_b200.train.random_projection import GradientProjector

pytestmark = pytest.mark.gpu
DEV = "cuda"


def cuda_tables(numel, pid, k, seed=42):
    """The reference's table recipe on the CUDA generator, plus the packed table."""
    h, s = orc.hash_sign_tables(numel, pid, k, seed=seed, device=DEV)
    packed = ops.pack_hash_sign(torch.from_numpy(h).to(DEV), torch.from_numpy(s).to(DEV), k)
    return h, s, packed


def rel_close(got, want, rtol, what=""):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    scale = max(np.abs(want).max(), 1e-30)
    err = np.abs(got - want).max() / scale
    assert err <= rtol, f"{what}: max |err| / max |ref| = {err:.3e} > {rtol}"


def test_pack_bit_exact():
    h, s, packed = cuda_tables(100_003, 7, 16384)
    np.testing.assert_array_equal(packed.cpu().numpy().view(np.uint32), orc.pack_tables(h, s))


def test_pack_rejects_out_of_range_bucket():
    h = torch.tensor([0, 5, 16], dtype=torch.int64, device=DEV)
    s = torch.tensor([1.0, -1.0, 1.0], device=DEV)
    with pytest.raises(RuntimeError, match="0x201"):
        ops.pack_hash_sign(h, s, 16)
    # the device error word was cleared: a valid call succeeds afterwards
    ops.pack_hash_sign(h, s, 17)


def decode_table(table, d_out, d_in):
    """Host decode of the tiled epilogue table back to [d_out, d_in] buckets and weights."""
    n_ob, n_cb = -(-d_out // 128), -(-d_in // 256)
    t = table.cpu().numpy().view(np.uint32).reshape(n_ob, n_cb, 8, 16, 128, 4)
    bucket = np.zeros((n_ob * 128, n_cb * 256), np.uint32)
    weight = np.zeros((n_ob * 128, n_cb * 256), np.float32)
    for ob in range(n_ob):
        for cb in range(n_cb):
            blk = t[ob, cb]  # [j, p, r, 4]
            for e in range(2):
                cols = (np.arange(8)[:, None] * 32 + np.arange(16)[None, :] * 2 + e)  # [j, p]
                b = blk[..., e].transpose(2, 0, 1)  # [r, j, p]
                w = blk[..., 2 + e].transpose(2, 0, 1).view(np.float32)
                bucket[ob * 128:(ob + 1) * 128, cb * 256 + cols] = b
                weight[ob * 128:(ob + 1) * 128, cb * 256 + cols] = w
    return bucket, weight


@pytest.mark.parametrize("numel,k,offset", [(3072 * 768, 16384, 0), (1_000_003, 65536, 1), (37, 8, 3),
                                            (100_000, 32768, 2), (5, 131072, 0)])
def test_bucket_counts_match_bincount(numel, k, offset):
    """Shared-memory (k <= 32768) and global-atomic histograms, misaligned starts."""
    rng = np.random.default_rng(numel)
    buckets = rng.integers(0, k, numel + offset).astype(np.uint32)
    signs = rng.integers(0, 2, numel + offset).astype(np.uint32) << np.uint32(31)
    packed = torch.from_numpy((buckets | signs).view(np.int32)).to(DEV)[offset:]
    counts, mx = ops.bucket_counts(packed, k)
    ops.check_device_error("bucket_counts")
    want = np.bincount(buckets[offset:].astype(np.int64), minlength=k)
    np.testing.assert_array_equal(counts.cpu().numpy(), want)
    assert int(mx.item()) == int(want.max())


def test_bucket_counts_empty_and_bad_bucket():
    counts, mx = ops.bucket_counts(torch.empty(0, dtype=torch.int32, device=DEV), 16)
    assert int(mx.item()) == 0 and int(counts.sum().item()) == 0
    bad = torch.tensor([1, 2, 40, 3], dtype=torch.int32, device=DEV)
    counts, _ = ops.bucket_counts(bad, 16)
    with pytest.raises(RuntimeError, match="0x201"):
        ops.check_device_error("bucket_counts")
    assert counts.cpu().tolist()[:4] == [0, 1, 1, 1]


def test_bucket_max_load_of_reference_tables():
    h, s, packed = cuda_tables(3072 * 768, 0, 16384)
    assert ops.bucket_max_load(packed, 16384) == int(np.bincount(h, minlength=16384).max())


@pytest.mark.parametrize("d_out,d_in", [(128, 256), (72, 48), (200, 520)])
def test_table_layout_and_adam_diag(d_out, d_in):
    k = 4096
    h, s, packed = cuda_tables(d_out * d_in, 1, k)
    v = np.random.default_rng(0).uniform(1e-9, 1e-3, (d_out, d_in)).astype(np.float32)
    table = ops.build_sketch_table(packed, d_out, d_in, exp_avg_sq=torch.from_numpy(v).to(DEV), eps=1e-8)
    bucket, weight = decode_table(table, d_out, d_in)
    np.testing.assert_array_equal(bucket[:d_out, :d_in], h.reshape(d_out, d_in))
    want = s.reshape(d_out, d_in) * orc.inv_rms(v, 1e-8)
    np.testing.assert_array_equal(weight[:d_out, :d_in], want)  # bit-exact AdamW diagonal
    assert not weight[d_out:, :].any() and not weight[:, d_in:].any()
    diag = torch.rand(d_out, d_in, device=DEV)
    _, weight2 = decode_table(ops.build_sketch_table(packed, d_out, d_in, diag=diag), d_out, d_in)
    np.testing.assert_array_equal(weight2[:d_out, :d_in], s.reshape(d_out, d_in) * diag.cpu().numpy())


SKETCH_SHAPES = [
    # B, T, d_out, d_in, k
    (1, 64, 128, 256, 512),
    (2, 100, 72, 48, 512),
    (3, 1, 8, 8, 64),
    (2, 130, 200, 264, 1000),
    (4, 64, 384, 768, 16384),
    (2, 70, 128, 256, 32768),
    (2, 64, 136, 264, 65536),     # shared-memory sketch of the first 32768 buckets, L2 atomics above
    (3, 40, 136, 264, 40001),     # odd k: rows of phi start off 16-byte boundaries
    (2, 64, 128, 512, 131072),
    (5, 33, 136, 520, 8192),
    (3, 200, 272, 520, 50000),    # 32-token stages: 45056 buckets in shared memory, the rest in L2
]


@pytest.mark.parametrize("fixed_point", [True, False])
@pytest.mark.parametrize("B,T,d_out,d_in,k", SKETCH_SHAPES)
def test_sketch_gemm_matches_oracle(B, T, d_out, d_in, k, fixed_point):
    torch.manual_seed(B * 1000 + T)
    g = (torch.randn(B, T, d_out, device=DEV) * 1e-3).bfloat16()
    a = torch.randn(B, T, d_in, device=DEV).bfloat16()
    h, s, packed = cuda_tables(d_out * d_in, 3, k)
    diag = torch.rand(d_out, d_in, device=DEV) * 1e-3 + 1e-6
    table = ops.build_sketch_table(packed, d_out, d_in, diag=diag)
    load = ops.bucket_max_load(packed, k) if fixed_point else 0
    assert load == int(np.bincount(h, minlength=k).max()) or not fixed_point
    phi = ops.sketch_gemm(g, a, table, k, max_bucket_load=load)
    ops.check_device_error("sketch_gemm")
    want = orc.project_full_gradient(g.float().cpu().numpy(), a.float().cpu().numpy(), h, s, k,
                                     diag=diag.cpu().numpy())
    rel_close(phi.cpu().numpy(), want, 1e-4, "phi")


@pytest.mark.parametrize("B,T,d_out,d_in,k", [sh for sh in SKETCH_SHAPES if sh[4] > 32768 and sh[2] > 128])
def test_sketch_gemm_one_cta_large_sketch_matches_oracle(B, T, d_out, d_in, k, monkeypatch):
    """The one-CTA kernel at the sketch sizes where CTA pairs are the default."""
    monkeypatch.setenv("OPUS_SKETCH_PAIR", "0")
    torch.manual_seed(B * 1000 + T)
    g = (torch.randn(B, T, d_out, device=DEV) * 1e-3).bfloat16()
    a = torch.randn(B, T, d_in, device=DEV).bfloat16()
    h, s, packed = cuda_tables(d_out * d_in, 3, k)
    table = ops.build_sketch_table(packed, d_out, d_in)
    phi = ops.sketch_gemm(g, a, table, k, max_bucket_load=ops.bucket_max_load(packed, k))
    ops.check_device_error("sketch_gemm one CTA")
    want = orc.project_full_gradient(g.float().cpu().numpy(), a.float().cpu().numpy(), h, s, k)
    rel_close(phi.cpu().numpy(), want, 1e-4, "phi, one CTA")


def test_sketch_gemm_outliers_and_nonfinite():
    """Updates far above the first tile's scale, and NaN, take the exact f32 path.

    300 work units over at most 148 CTAs: each CTA sees two or more
    consecutive tiles of a candidate, and every odd o-block of candidate 0 is
    1e6 times larger than the even ones, so a CTA that scaled on an even tile
    meets outliers on the next one.
    """
    B, T, d_out, d_in, k = 4, 64, 9600, 256, 4096
    g = (torch.randn(B, T, d_out, device=DEV) * 1e-3)
    g[0].view(T, 75, 128)[:, 1::2, :] *= 1e6
    g[1, 5, 200] = float("nan")   # candidate 1: NaN reaches a set of buckets
    g = g.bfloat16()
    a = torch.randn(B, T, d_in, device=DEV).bfloat16()
    h, s, packed = cuda_tables(d_out * d_in, 4, k)
    table = ops.build_sketch_table(packed, d_out, d_in)
    phi = ops.sketch_gemm(g, a, table, k, max_bucket_load=ops.bucket_max_load(packed, k)).cpu().numpy()
    want = orc.project_full_gradient(g.float().cpu().numpy(), a.float().cpu().numpy(), h, s, k)
    rel_close(phi[0], want[0], 1e-4, "outlier candidate")
    np.testing.assert_array_equal(np.isnan(phi[1]), np.isnan(want[1]))
    assert np.isnan(phi[1]).any()


def test_sketch_gemm_rows_div_and_accumulate():
    B, T, d_out, d_in, k = 6, 48, 64, 128, 2048
    g = torch.randn(B, T, d_out, device=DEV).bfloat16()
    a = torch.randn(B, T, d_in, device=DEV).bfloat16()
    h, s, packed = cuda_tables(d_out * d_in, 0, k)
    table = ops.build_sketch_table(packed, d_out, d_in)
    load = ops.bucket_max_load(packed, k)
    per = orc.project_full_gradient(g.float().cpu().numpy(), a.float().cpu().numpy(), h, s, k)
    grouped = ops.sketch_gemm(g, a, table, k, rows_div=4, max_bucket_load=load)  # rows {0..3}, {4, 5}
    rel_close(grouped.cpu().numpy(), np.stack([per[:4].sum(0), per[4:].sum(0)]), 1e-4, "rows_div")
    out = ops.sketch_gemm(g, a, table, k, max_bucket_load=load)
    ops.sketch_gemm(g, a, table, k, out=out, accumulate=True, max_bucket_load=load)
    rel_close(out.cpu().numpy(), 2 * per, 1e-4, "accumulate")


@pytest.mark.parametrize("B,T,d_out,d_in,k", [(8, 96, 384, 1024, 65536), (5, 64, 256, 512, 4096)])
def test_sketch_gemm_merged_rows_match_sum_of_samples(B, T, d_out, d_in, k):
    """rows_div = B: the whole batch becomes one row of B*T tokens whose tiles are dealt over the SMs."""
    torch.manual_seed(B * k)
    g = (torch.randn(B, T, d_out, device=DEV) * 1e-2).bfloat16()
    a = torch.randn(B, T, d_in, device=DEV).bfloat16()
    h, s, packed = cuda_tables(d_out * d_in, 3, k)
    table = ops.build_sketch_table(packed, d_out, d_in)
    load = ops.bucket_max_load(packed, k)
    per = orc.project_full_gradient(g.float().cpu().numpy(), a.float().cpu().numpy(), h, s, k)
    got = ops.sketch_gemm(g, a, table, k, rows_div=B, max_bucket_load=load)
    ops.check_device_error("sketch_gemm merged rows")
    assert got.shape == (1, k)
    rel_close(got.cpu().numpy(), per.sum(0, keepdims=True), 1e-4, "merged rows")


def test_sketch_gemm_f32_inputs_split():
    B, T, d_out, d_in, k = 3, 50, 96, 64, 1024
    g = torch.randn(B, T, d_out, device=DEV)
    a = torch.randn(B, T, d_in, device=DEV)
    h, s, packed = cuda_tables(d_out * d_in, 2, k)
    phi = ops.sketch_gemm(g, a, ops.build_sketch_table(packed, d_out, d_in), k,
                          max_bucket_load=ops.bucket_max_load(packed, k))
    want = orc.project_full_gradient(g.cpu().numpy(), a.cpu().numpy(), h, s, k)
    rel_close(phi.cpu().numpy(), want, 2e-5, "f32 split")


def test_project_full_gradient_golden():
    gd = load_golden("project")
    for i in range(int(gd["n"])):
        k, pid, _two_d = (int(x) for x in gd[f"meta{i}"])
        proj = GradientProjector(sketch_dim=k, seed=42, device="cpu")
        S = gd.get(f"S{i}")
        diag = gd.get(f"diag{i}")
        phi = proj.project_full_gradient(torch.from_numpy(gd[f"g{i}"]).to(DEV), torch.from_numpy(gd[f"a{i}"]).to(DEV),
                                         param_id=pid, preconditioner_S=None if S is None else torch.from_numpy(S).to(DEV),
                                         diagonal_preconditioner=None if diag is None else torch.from_numpy(diag).to(DEV))
        rel_close(phi.cpu().numpy(), gd[f"phi{i}"], 1e-4, f"golden project case {i}")


@pytest.mark.parametrize("transposed", [False, True])
@pytest.mark.parametrize("d_out,d_in,k", [(64, 96, 256), (3072, 768, 16384), (200, 300, 1001), (512, 1024, 40000),
                                         (100, 36, 100000)])
def test_sketch_dense(transposed, d_out, d_in, k):
    """Shared-memory sketch per CTA (k up to ~55000; odd k flushes scalar), L2 atomics above."""
    h, s, packed = cuda_tables(d_out * d_in, 5, k)
    W = torch.randn(d_out, d_in, device=DEV)
    diag = torch.rand(d_out, d_in, device=DEV)
    src = W.T.contiguous() if transposed else W
    load = ops.bucket_max_load(packed, k)
    out = ops.sketch_dense(src, packed, d_out, d_in, k, transposed=transposed, diag=diag, max_bucket_load=load)
    want = orc.dense_sketch(W.cpu().numpy(), h, s, k, diag=diag.cpu().numpy())
    rel_close(out.cpu().numpy(), want, 1e-5, "dense sketch")
    # without the load bound the share's element count bounds the fixed point: rounding about 100 times
    # coarser (at most count / 2^31 of the share's largest value per element), still far inside 1e-3
    coarse = ops.sketch_dense(src, packed, d_out, d_in, k, transposed=transposed, diag=diag)
    rel_close(coarse.cpu().numpy(), want, 3e-4, "dense sketch, count bound")


@pytest.mark.parametrize("transposed", [False, True])
def test_sketch_dense_row_shards_sum_to_whole(transposed):
    """Ranks sketch their rows of the target; the partial sketches add up to the whole one."""
    d_out, d_in, k = 3072, 768, 16384
    h, s, packed = cuda_tables(d_out * d_in, 6, k)
    W = torch.randn(d_out, d_in, device=DEV)
    src = W.T.contiguous() if transposed else W
    whole = orc.dense_sketch(W.cpu().numpy(), h, s, k)
    load = ops.bucket_max_load(packed, k)
    for world in (3, 8):
        acc = torch.zeros(k, device=DEV)
        for r in range(world):
            lo, hi = r * d_out // world, (r + 1) * d_out // world
            ops.sketch_dense(src, packed, d_out, d_in, k, transposed=transposed, out=acc, accumulate=True,
                             rows=(lo, hi), max_bucket_load=load)
        rel_close(acc.cpu().numpy(), whole, 1e-5, f"row shards x{world}")
    empty = ops.sketch_dense(src, packed, d_out, d_in, k, transposed=transposed, rows=(5, 5))
    assert not empty.any()
    with pytest.raises(ValueError):
        ops.sketch_dense(src, packed, d_out, d_in, k, rows=(10, d_out + 1))


def test_sketch_dot_and_gram():
    rng = np.random.default_rng(1)
    A = rng.standard_normal((70, 3000)).astype(np.float32)
    Bm = rng.standard_normal((9, 3000)).astype(np.float32)
    tau = rng.standard_normal(3000).astype(np.float32)
    tA, tB, tt = (torch.from_numpy(x).to(DEV) for x in (A, Bm, tau))
    rel_close(ops.sketch_dot(tA, tt, alpha=0.5).cpu().numpy(), 0.5 * A.astype(np.float64) @ tau, 1e-5, "dot")
    rel_close(ops.sketch_gram(tA, alpha=2.0).cpu().numpy(), 2.0 * A.astype(np.float64) @ A.T, 1e-5, "gram")
    out = ops.sketch_gram(tA, tB)
    ops.sketch_gram(tA, tB, out=out, accumulate=True)
    rel_close(out.cpu().numpy(), 2.0 * A.astype(np.float64) @ Bm.T, 1e-5, "gram ab")


@pytest.mark.parametrize("ra,rb,k", [(256, 256, 16384), (300, 130, 4100), (17, 260, 64), (5, 3, 3001), (128, 128, 32768)])
def test_sketch_gram_tensor_core_and_simt(ra, rb, k):
    """3xTF32 tcgen05 path (k % 4 == 0) and the SIMT path (k % 4 != 0) against float64."""
    rng = np.random.default_rng(ra * 7 + rb + k)
    A = (rng.standard_normal((ra, k)) * rng.uniform(0.1, 10.0, (ra, 1))).astype(np.float32)
    Bm = rng.standard_normal((rb, k)).astype(np.float32)
    tA, tB = torch.from_numpy(A).to(DEV), torch.from_numpy(Bm).to(DEV)
    got = ops.sketch_gram(tA, tB, alpha=0.25).cpu().numpy()
    rel_close(got, 0.25 * A.astype(np.float64) @ Bm.T.astype(np.float64), 2e-5, f"gram {ra}x{rb}x{k}")
    ops.check_device_error("sketch_gram")


@pytest.mark.parametrize("ra,k", [(256, 65536), (300, 65540), (129, 70000), (1000, 8192)])
def test_sketch_gram_self_upper_tiles(ra, k):
    """phi phi^T computes the tiles on and above the diagonal (one operand load on the diagonal)
    and mirrors the others; partial last tiles and accumulation included.  The diagonal is a
    sum of squares, on which the tensor cores' f32 accumulation errs one way (about 6e-7 per
    32-wide k-block, at most 64 k-blocks per CTA), hence 1e-4 rather than 2e-5."""
    rng = np.random.default_rng(ra + k)
    A = (rng.standard_normal((ra, k)) * rng.uniform(0.1, 10.0, (ra, 1))).astype(np.float32)
    tA = torch.from_numpy(A).to(DEV)
    want = A.astype(np.float64) @ A.T.astype(np.float64)
    got = ops.sketch_gram(tA, alpha=0.5)
    ops.check_device_error("self gram")
    rel_close(got.cpu().numpy(), 0.5 * want, 1e-4, f"self gram {ra}x{k}")
    ops.sketch_gram(tA, out=got, alpha=0.5, accumulate=True)
    rel_close(got.cpu().numpy(), want, 1e-4, f"self gram accumulate {ra}x{k}")
    # a distinct buffer with the same values takes the general path and agrees
    rel_close(ops.sketch_gram(tA, tA.clone()).cpu().numpy(), want, 1e-4, "general path")


def test_sketch_gram_nonfinite():
    """Entries are non-finite exactly where the f32 product is (an inf may come out as NaN:
    the split's hi * lo term is inf * 0 when the other operand is exactly a tf32)."""
    A = torch.randn(8, 256, device=DEV)
    A[2, 7] = float("inf")
    A[5, 9] = float("nan")
    got = ops.sketch_gram(A).cpu().numpy()
    want = A.cpu().double().numpy() @ A.cpu().double().numpy().T
    np.testing.assert_array_equal(np.isfinite(got), np.isfinite(want))
    fin = np.isfinite(want)
    rel_close(got[fin], want[fin], 2e-5, "finite entries")


def test_split_bf16():
    x = torch.randn(10001, device=DEV) * 100
    hi, lo = ops.split_bf16(x)
    assert torch.equal(hi, x.bfloat16())
    err = (hi.float() + lo.float() - x).abs() / x.abs()
    assert float(err.max()) < 2 ** -15


@pytest.mark.parametrize("B,T,d_in,d_out", [(2, 128, 64, 256), (3, 100, 48, 72), (2, 300, 264, 520),
                                            (4, 256, 768, 3072)])
def test_ghost_score_matches_oracle(B, T, d_in, d_out):
    torch.manual_seed(T)
    a = torch.randn(B, T, d_in, device=DEV).bfloat16()
    g = (torch.randn(B, T, d_out, device=DEV) * 1e-3).bfloat16()
    V = torch.randn(d_out, d_in, device=DEV) / d_in ** 0.5
    got = ops.ghost_score(a, g, ops.dense_target_pair(V), alpha=1.5)
    ops.check_device_error("ghost_score")
    want = 1.5 * orc.ghost_score(a.float().cpu().numpy(), g.float().cpu().numpy(), V.cpu().numpy())
    rel_close(got.cpu().numpy(), want, 1e-4, "ghost")


@pytest.mark.parametrize("d_out,d_in,precond", [(384, 256, "diag"), (384, 256, "adam"), (64, 96, "none"),
                                                 (7, 9, "adam"), (3, 5, "diag")])
def test_desketch_bit_exact(d_out, d_in, precond):
    """v = scale * D * s * tau[h] as bf16 hi and lo = bf16(v - hi); 4-wide and scalar paths."""
    k = 1000
    h, s, packed = cuda_tables(d_out * d_in, 2, k)
    rng = np.random.default_rng(d_out * d_in)
    tau = rng.standard_normal(k).astype(np.float32)
    w = rng.uniform(1e-9, 1e-3, (d_out, d_in)).astype(np.float32)
    kw = {"diag": dict(diag=torch.from_numpy(w).to(DEV)), "adam": dict(exp_avg_sq=torch.from_numpy(w).to(DEV)),
          "none": {}}[precond]
    got = ops.desketch(torch.from_numpy(tau).to(DEV), packed, d_out, d_in, scale=0.75, eps=1e-8, **kw)
    d = {"diag": w, "adam": orc.inv_rms(w, 1e-8), "none": np.ones_like(w)}[precond].reshape(-1)
    x = (np.float32(0.75) * d) * tau[h]
    x = np.where(s < 0, -x, x).astype(np.float32)
    hi = orc.bf16_round(x)
    lo = orc.bf16_round((x - hi).astype(np.float32))
    g = got.float().cpu().numpy().reshape(2, -1)
    np.testing.assert_array_equal(g[0], hi)
    np.testing.assert_array_equal(g[1], lo)


def test_ghost_equals_sketch_dot_through_desketch():
    """<G_b, D s tau[h]> by the ghost kernel == CS(D o G_b) . tau by the sketch kernels."""
    B, T, d_out, d_in, k = 4, 256, 384, 256, 4096
    a = torch.randn(B, T, d_in, device=DEV).bfloat16()
    g = (torch.randn(B, T, d_out, device=DEV) * 1e-2).bfloat16()
    h, s, packed = cuda_tables(d_out * d_in, 9, k)
    v = torch.rand(d_out, d_in, device=DEV) * 1e-3
    tau = torch.randn(k, device=DEV)
    phi = ops.sketch_gemm(g, a, ops.build_sketch_table(packed, d_out, d_in, exp_avg_sq=v), k,
                          max_bucket_load=ops.bucket_max_load(packed, k))
    via_sketch = ops.sketch_dot(phi, tau, alpha=0.25)
    vt = ops.desketch(tau, packed, d_out, d_in, scale=0.25, exp_avg_sq=v)
    via_ghost = ops.ghost_score(a, g, vt)
    rel_close(via_ghost.cpu().numpy(), via_sketch.cpu().numpy(), 1e-4, "ghost vs sketch")


def test_empty_inputs():
    """Zero candidates, zero tokens or zero picks: every entry point returns without a launch error."""
    k = 512
    h, s, packed = cuda_tables(64 * 64, 0, k)
    table = ops.build_sketch_table(packed, 64, 64)
    phi = ops.sketch_gemm(torch.empty(0, 16, 64, device=DEV, dtype=torch.bfloat16),
                          torch.empty(0, 16, 64, device=DEV, dtype=torch.bfloat16), table, k)
    assert phi.shape == (0, k)
    phi0 = ops.sketch_gemm(torch.empty(3, 0, 64, device=DEV, dtype=torch.bfloat16),
                           torch.empty(3, 0, 64, device=DEV, dtype=torch.bfloat16), table, k)
    assert phi0.shape == (3, k) and not phi0.any()
    assert ops.sketch_dot(torch.empty(0, k, device=DEV), torch.zeros(k, device=DEV)).numel() == 0
    assert ops.sketch_gram(torch.empty(0, k, device=DEV)).numel() == 0
    sc = torch.randn(5, device=DEV)
    sim = torch.zeros(5, 5, device=DEV)
    assert ops.boltzmann_select(sc, sim, 0, 1.0, torch.empty(0, dtype=torch.float64)).numel() == 0
    assert ops.greedy_select(sc, sim, 0).numel() == 0
    ops.check_device_error("empty inputs")


@pytest.mark.parametrize("B,T,d_out,d_in,dtype,with_diag", [
    (3, 64, 128, 256, torch.bfloat16, True),
    (2, 100, 72, 48, torch.bfloat16, False),      # partial tiles in both dimensions
    (2, 70, 136, 264, torch.bfloat16, True),
    (3, 33, 20, 30, torch.float32, True),         # widths padded to 8, f32 split into bf16 hi/lo
    (4, 1, 384, 768, torch.bfloat16, True),
])
def test_per_sample_grad_matches_oracle(B, T, d_out, d_in, dtype, with_diag):
    """Dense epilogue of the tensor-core GEMM: exact per-sample gradients, times the diagonal."""
    torch.manual_seed(B + T + d_out)
    g = (torch.randn(B, T, d_out, device=DEV) * 1e-3).to(dtype)
    a = torch.randn(B, T, d_in, device=DEV).to(dtype)
    diag = torch.rand(d_out, d_in, device=DEV) * 1e-3 + 1e-6 if with_diag else None
    got = ops.per_sample_grad(g, a, diag=diag)
    ops.check_device_error("per_sample_grad")
    gd, ad = g.double().cpu().numpy(), a.double().cpu().numpy()
    want = np.einsum("bto,btc->boc", gd, ad)
    if with_diag:
        want = want * diag.double().cpu().numpy()
    rel_close(got.cpu().numpy(), want.reshape(B, -1), 1e-4 if dtype == torch.float32 else 1e-5, "per_sample_grad")
    # accumulate adds onto what is there
    acc = got.clone()
    ops.per_sample_grad(g, a, diag=diag, out=acc, accumulate=True)
    rel_close(acc.cpu().numpy(), 2 * want.reshape(B, -1), 1e-4 if dtype == torch.float32 else 1e-5, "accumulate")


def test_per_sample_grad_empty_and_tokenless():
    g = torch.zeros(0, 8, 16, device=DEV, dtype=torch.bfloat16)
    a = torch.zeros(0, 8, 24, device=DEV, dtype=torch.bfloat16)
    assert ops.per_sample_grad(g, a).shape == (0, 16 * 24)
    g = torch.zeros(2, 0, 16, device=DEV, dtype=torch.bfloat16)
    a = torch.zeros(2, 0, 24, device=DEV, dtype=torch.bfloat16)
    out = torch.full((2, 16 * 24), 5.0, device=DEV)
    assert not ops.per_sample_grad(g, a, out=out).any()  # no tokens: zero gradients


def test_bounded_wait_reports_and_the_context_survives():
    """A wait that nothing releases ends after its limit with an error code; later kernels still run."""
    import ctypes
    import time

    from opus_b200 import _lib

    assert _lib.device_error() == 0  # nothing pending from earlier tests
    t0 = time.monotonic()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert _lib.load().opus_selftest_stalled_wait(stream) == _lib.OPUS_OK
    assert _lib.device_error() == 0x106  # synchronises: the kernel has returned on its own
    assert 0.9 < time.monotonic() - t0 < 60
    assert _lib.device_error() == 0  # reading clears the word
    h, s, packed = cuda_tables(4096, 1, 256)  # the context is still usable
    assert torch.equal(packed.cpu() & 0x7FFFFFFF, torch.from_numpy(h.astype(np.int32)))
    ops.check_device_error("after the stalled wait")


@pytest.mark.parametrize("B,T,d_in,d_out,dtype", [
    (5, 200, 72, 136, torch.bfloat16),     # two token blocks (one partial), partial feature blocks
    (3, 64, 256, 128, torch.float32),      # f32: bf16 hi/lo, three products per GEMM
    (1, 130, 20, 30, torch.float32),       # widths padded to 8
    (7, 128, 768, 3072, torch.bfloat16),   # GPT-2-small MLP widths
])
def test_ghost_gram_matches_materialised_gram(B, T, d_in, d_out, dtype):
    """sum over token pairs of (a_i a_j^T) o (g_i g_j^T) == <G_i, G_j> of the per-sample gradients."""
    torch.manual_seed(B * 100 + T)
    a = torch.randn(B, T, d_in, device=DEV).to(dtype)
    g = (torch.randn(B, T, d_out, device=DEV) * 1e-2).to(dtype)
    got = ops.ghost_gram(a, g, alpha=0.5)
    ops.check_device_error("ghost_gram")
    G = np.einsum("bto,btc->boc", g.double().cpu().numpy(), a.double().cpu().numpy()).reshape(B, -1)
    want = 0.5 * G @ G.T
    rel_close(got.cpu().numpy(), want, 1e-4 if dtype == torch.float32 else 2e-5, "ghost gram")
    ops.ghost_gram(a, g, alpha=0.5, out=got, accumulate=True)
    rel_close(got.cpu().numpy(), 2 * want, 1e-4 if dtype == torch.float32 else 2e-5, "ghost gram accumulate")


def test_ghost_gram_empty():
    a = torch.zeros(3, 0, 16, device=DEV, dtype=torch.bfloat16)
    g = torch.zeros(3, 0, 24, device=DEV, dtype=torch.bfloat16)
    out = torch.full((3, 3), 7.0, device=DEV)
    assert not ops.ghost_gram(a, g, out=out).any()
    assert ops.ghost_gram(a[:0], g[:0]).shape == (0, 0)


@pytest.mark.parametrize("n", [1, 7, 4096, 1000003])
def test_adam_diag_bit_exact(n):
    """1 / (sqrt(v) + eps) equals torch's CUDA result bit for bit (data_selection.py:208-214)."""
    torch.manual_seed(n)
    v = torch.rand(n, device=DEV) * 1e-3
    v[: min(n, 3)] = 0.0
    got = ops.adam_diag(v, 1e-8)
    assert torch.equal(got, (v.sqrt() + 1e-8).reciprocal())
    odd = v[1:]  # a 4-byte-offset view takes the scalar path
    assert torch.equal(ops.adam_diag(odd, 1e-6), (odd.sqrt() + 1e-6).reciprocal())


@pytest.mark.parametrize("n,d,k", [(5, 3000, 1024), (17, 4099, 4096), (1, 2_359_296, 16384)])
def test_sketch_dense_rows_match_oracle(n, d, k):
    """project_batch: every row of a [n, d] batch in one launch (odd d takes the scalar path)."""
    h, s, packed = cuda_tables(d, 2, k)
    X = torch.randn(n, d, device=DEV)
    proj = GradientProjector(sketch_dim=k, seed=42, device="cuda")
    got = proj.project_batch(X, 2)
    ops.check_device_error("sketch_dense_rows")
    assert got.shape == (n, k)
    for i in range(n):
        rel_close(got[i].cpu().numpy(), orc.dense_sketch(X[i].cpu().numpy()[None], h, s, k), 1e-5, f"row {i}")
    one = proj.project_vector(X[0], 2)
    rel_close(one.cpu().numpy(), got[0].cpu().numpy(), 1e-5, "project_vector == row 0")


@pytest.mark.parametrize("stage_tokens", ["64", "32"])
def test_sketch_gemm_stage_depths_match_oracle(stage_tokens, monkeypatch):
    """A large sketch on the one-CTA kernel with either pipeline depth forced: 32768 or 45056
    buckets in shared memory (CTA pairs, the default at this size, are off)."""
    monkeypatch.setenv("OPUS_SKETCH_PAIR", "0")
    monkeypatch.setenv("OPUS_SKETCH_STAGE_TOKENS", stage_tokens)
    B, T, d_out, d_in, k = 3, 150, 256, 768, 65536
    torch.manual_seed(11)
    g = (torch.randn(B, T, d_out, device=DEV) * 1e-3).bfloat16()
    a = torch.randn(B, T, d_in, device=DEV).bfloat16()
    h, s, packed = cuda_tables(d_out * d_in, 4, k)
    table = ops.build_sketch_table(packed, d_out, d_in)
    phi = ops.sketch_gemm(g, a, table, k, max_bucket_load=ops.bucket_max_load(packed, k))
    ops.check_device_error("sketch_gemm stage depth")
    want = orc.project_full_gradient(g.float().cpu().numpy(), a.float().cpu().numpy(), h, s, k)
    rel_close(phi.cpu().numpy(), want, 1e-4, f"phi, {stage_tokens}-token stages")


@pytest.mark.parametrize("order,jobs", [("ob", "tiles"), ("cb", "tiles"), ("ob", "lines"), ("cb", "lines")])
@pytest.mark.parametrize("d_out,d_in", [(384, 768), (768, 256)])
def test_sketch_gemm_tile_walks_match_oracle(order, jobs, d_out, d_in, monkeypatch):
    """Either tile walk and either job cut (OPUS_SKETCH_ORDER / OPUS_SKETCH_JOBS forced), with and
    without the diagonal: the same sketches, the per-sample gradients too."""
    monkeypatch.setenv("OPUS_SKETCH_ORDER", order)
    monkeypatch.setenv("OPUS_SKETCH_JOBS", jobs)
    B, T, k = 5, 70, 8192
    torch.manual_seed(d_out + d_in)
    g = (torch.randn(B, T, d_out, device=DEV) * 1e-3).bfloat16()
    a = torch.randn(B, T, d_in, device=DEV).bfloat16()
    diag = torch.rand(d_out, d_in, device=DEV) + 0.5
    h, s, packed = cuda_tables(d_out * d_in, 5, k)
    table = ops.build_sketch_table(packed, d_out, d_in, diag=diag)
    phi = ops.sketch_gemm(g, a, table, k, max_bucket_load=ops.bucket_max_load(packed, k))
    dense = ops.per_sample_grad(g, a, diag=diag)
    ops.check_device_error(f"sketch_gemm walk {order}/{jobs}")
    gn, an = g.float().cpu().numpy(), a.float().cpu().numpy()
    want = orc.project_full_gradient(gn, an, h, s, k, diag=diag.cpu().numpy())
    rel_close(phi.cpu().numpy(), want, 1e-4, f"phi, walk {order}/{jobs}")
    want_dense = orc.per_sample_grads(gn, an) * diag.cpu().numpy()[None]
    rel_close(dense.cpu().numpy().reshape(want_dense.shape), want_dense, 1e-5, f"dense, walk {order}/{jobs}")


@pytest.mark.parametrize("pair", ["0", "1"])
@pytest.mark.parametrize("k", [8192, 65536])
def test_sketch_gemm_alpha_scales_every_update(pair, k, monkeypatch):
    """alpha (the per-sample factor of dL/dZ) multiplies the sketch, to the fixed-point quantum (the scale of
    each job's shared sketch follows the scaled values, so its grid moves with alpha) and the rounding of the
    f32 sums (the L2 reductions and the per-job flushes add in no fixed order)."""
    monkeypatch.setenv("OPUS_SKETCH_PAIR", pair)
    B, T, d_out, d_in = 4, 80, 384, 512
    torch.manual_seed(k)
    g = (torch.randn(B, T, d_out, device=DEV) * 1e-3).bfloat16()
    a = torch.randn(B, T, d_in, device=DEV).bfloat16()
    h, s, packed = cuda_tables(d_out * d_in, 8, k)
    table = ops.build_sketch_table(packed, d_out, d_in, exp_avg_sq=torch.full((d_out, d_in), 1e-4, device=DEV))
    load = ops.bucket_max_load(packed, k)
    one = ops.sketch_gemm(g, a, table, k, max_bucket_load=load)
    four = ops.sketch_gemm(g, a, table, k, max_bucket_load=load, alpha=4.0)
    tw = ops.sketch_gemm(g, a, table, k, max_bucket_load=load, alpha=24.0)
    ops.check_device_error("sketch_gemm alpha")
    rel_close(four.cpu().numpy(), 4 * one.cpu().numpy(), 1e-5, "alpha 4")
    rel_close(tw.cpu().numpy(), 24 * one.cpu().numpy(), 1e-5, "alpha 24")


@pytest.mark.parametrize("epi", ["8", "12", "16"])
@pytest.mark.parametrize("pair", ["0", "1"])
@pytest.mark.parametrize("B,T,d_out,d_in,k", [(3, 100, 384, 512, 8192), (2, 130, 520, 264, 1000),
                                              (4, 64, 256, 1024, 65536), (2, 70, 640, 384, 131072)])
def test_sketch_gemm_epilogue_widths_match_oracle(B, T, d_out, d_in, k, pair, epi, monkeypatch):
    """The scatter with 8, 12 or 16 epilogue warps (32-, 16- or 8-column chunks dealt round-robin),
    one CTA and pairs."""
    monkeypatch.setenv("OPUS_SKETCH_EPI_WARPS", epi)
    monkeypatch.setenv("OPUS_SKETCH_PAIR", pair)
    torch.manual_seed(B * 31 + d_out)
    g = (torch.randn(B, T, d_out, device=DEV) * 1e-3).bfloat16()
    a = torch.randn(B, T, d_in, device=DEV).bfloat16()
    h, s, packed = cuda_tables(d_out * d_in, 9, k)
    diag = torch.rand(d_out, d_in, device=DEV) * 1e-3 + 1e-6
    table = ops.build_sketch_table(packed, d_out, d_in, diag=diag)
    phi = ops.sketch_gemm(g, a, table, k, max_bucket_load=ops.bucket_max_load(packed, k))
    ops.check_device_error(f"sketch_gemm, {epi} epilogue warps")
    want = orc.project_full_gradient(g.float().cpu().numpy(), a.float().cpu().numpy(), h, s, k,
                                     diag=diag.cpu().numpy())
    rel_close(phi.cpu().numpy(), want, 1e-4, f"phi, {epi} epilogue warps")


@pytest.mark.parametrize("epi", ["8", "12", "16"])
@pytest.mark.parametrize("pair", ["0", "1"])
@pytest.mark.parametrize("d_out,d_in", [(296, 520), (224, 504), (1600, 1600), (136, 264)])
def test_sketch_gemm_padded_edges_match_oracle(d_out, d_in, pair, epi, monkeypatch):
    """Edges of the padded tiles the scatter skips: a last o-block whose second TMEM lane quarter
    holds 8 real rows (296 = 2*128 + 40) or whose last quarter holds none (224 = 128 + 96), and
    a last column block with 8 real columns (520, 264) or 248 (504)."""
    monkeypatch.setenv("OPUS_SKETCH_EPI_WARPS", epi)
    monkeypatch.setenv("OPUS_SKETCH_PAIR", pair)
    B, T, k = 2, 70, 65536
    torch.manual_seed(d_out * 3 + d_in)
    g = (torch.randn(B, T, d_out, device=DEV) * 1e-3).bfloat16()
    a = torch.randn(B, T, d_in, device=DEV).bfloat16()
    h, s, packed = cuda_tables(d_out * d_in, 11, k)
    diag = torch.rand(d_out, d_in, device=DEV) * 1e-3 + 1e-6
    table = ops.build_sketch_table(packed, d_out, d_in, diag=diag)
    phi = ops.sketch_gemm(g, a, table, k, max_bucket_load=ops.bucket_max_load(packed, k))
    ops.check_device_error(f"sketch_gemm padded edges, {epi} epilogue warps")
    want = orc.project_full_gradient(g.float().cpu().numpy(), a.float().cpu().numpy(), h, s, k,
                                     diag=diag.cpu().numpy())
    rel_close(phi.cpu().numpy(), want, 1e-4, f"phi, padded edges, {epi} epilogue warps")


@pytest.mark.parametrize("L,B,k,rows", [(5, 7, 65536, (2, 9)), (3, 4, 1000, (0, 4)), (1, 1, 8192, (0, 1))])
def test_sketch_dot_layers_matches_per_layer_dots(L, B, k, rows):
    """Every layer's score term in one launch == per-layer sketch_dot == float64, on a row slice of a
    longer buffer (the layer stride is the whole buffer's rows)."""
    torch.manual_seed(L * B + k)
    lo, hi = rows
    full = torch.randn(L, hi + 3, k, device=DEV)
    phis = full[:, lo:hi]
    taus = torch.randn(L, k, device=DEV)
    alphas = torch.rand(L, device=DEV) + 0.5
    got = ops.sketch_dot_layers(phis, taus, alphas)
    ops.check_device_error("sketch_dot_layers")
    per = torch.zeros(hi - lo, device=DEV)
    for l in range(L):
        ops.sketch_dot(phis[l].contiguous(), taus[l], alpha=float(alphas[l]), out=per, accumulate=True)
    want = (phis.double() * taus.double()[:, None, :]).sum(-1).mul(alphas.double()[:, None]).sum(0)
    rel_close(got.cpu().numpy(), want.cpu().numpy(), 1e-5, "sketch_dot_layers")
    rel_close(per.cpu().numpy(), want.cpu().numpy(), 1e-5, "per-layer sketch_dot")
    acc = ops.sketch_dot_layers(phis, taus, alphas, out=got.clone(), accumulate=True)
    rel_close(acc.cpu().numpy(), 2 * want.cpu().numpy(), 1e-5, "accumulate")
