"""Torch-tensor front end of the C ABI (include/opus_b200.h).

Every function here takes CUDA tensors, launches on the current CUDA stream of
the tensors' device and returns CUDA tensors.  There is no CPU path: a CPU
tensor or a missing libopus_b200.so raises.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

_ERR_BAD_PROBS = 0x301


def _stream(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _cuda(t: torch.Tensor, name: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the OPUS B200 path runs on the GPU only)")
    return t


def _contig(t: torch.Tensor) -> torch.Tensor:
    return t if t.is_contiguous() else t.contiguous()


def check_device_error(what: str = "opus kernel") -> None:
    """Synchronise and raise if a kernel recorded a device-side error."""
    code = _lib.device_error()
    if code == _ERR_BAD_PROBS:
        raise ValueError(f"{what}: probabilities do not sum to 1")
    if code:
        raise RuntimeError(f"{what}: device error 0x{code:x}")


# --------------------------------------------------------------------- tables
def pack_hash_sign(hash_: torch.Tensor, sign: torch.Tensor, k: int, validate: bool = True) -> torch.Tensor:
    """int64 buckets + float32 +-1 signs -> uint32 (stored as int32) packed table."""
    _cuda(hash_, "hash")
    _cuda(sign, "sign")
    if hash_.dtype != torch.int64 or sign.dtype != torch.float32:
        raise ValueError("hash must be int64 and sign float32")
    if hash_.numel() != sign.numel():
        raise ValueError("hash and sign must have the same number of elements")
    h, s = _contig(hash_.reshape(-1)), _contig(sign.reshape(-1))
    out = torch.empty(h.numel(), dtype=torch.int32, device=h.device)
    _lib.check(_lib.load().opus_pack_hash_sign(_ptr(h), _ptr(s), h.numel(), int(k), _ptr(out), _stream(h)),
               "opus_pack_hash_sign")
    if validate:
        check_device_error("opus_pack_hash_sign (bucket outside [0,k) or sign not +-1)")
    return out


def bucket_counts(packed: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-bucket element counts [k] int32 and their max [1] int64, on the device."""
    _cuda(packed, "packed")
    packed = _contig(packed.reshape(-1))
    if packed.dtype not in (torch.int32, torch.uint32):
        raise ValueError("packed table must be 32-bit")
    counts = torch.empty(int(k), dtype=torch.int32, device=packed.device)
    out = torch.empty(1, dtype=torch.int64, device=packed.device)
    _lib.check(_lib.load().opus_bucket_max_load(_ptr(packed), packed.numel(), int(k), _ptr(counts), counts.numel(),
                                               _ptr(out), _stream(packed)), "opus_bucket_max_load")
    return counts, out


def bucket_max_load(packed: torch.Tensor, k: int) -> int:
    """Largest number of elements sharing one bucket (bounds the fixed-point sketch)."""
    return int(bucket_counts(packed, k)[1].item())


def sketch_table_entries(d_out: int, d_in: int) -> int:
    return int(_lib.load().opus_sketch_table_entries(int(d_out), int(d_in)))


def build_sketch_table(packed: torch.Tensor, d_out: int, d_in: int, diag: torch.Tensor | None = None,
                       exp_avg_sq: torch.Tensor | None = None, eps: float = 1e-8,
                       out: torch.Tensor | None = None) -> torch.Tensor:
    """Tiled (bucket, sign*D) epilogue table for sketch_gemm; 16 bytes per entry."""
    _cuda(packed, "packed")
    n = sketch_table_entries(d_out, d_in)
    if packed.numel() != d_out * d_in:
        raise ValueError(f"packed table has {packed.numel()} elements, layer has {d_out * d_in}")
    for name, t in (("diag", diag), ("exp_avg_sq", exp_avg_sq)):
        if t is not None:
            _cuda(t, name)
            if t.numel() != d_out * d_in:
                raise ValueError(f"{name} has {t.numel()} elements, layer has {d_out * d_in}")
    diag = None if diag is None else _contig(diag.to(torch.float32))
    exp_avg_sq = None if exp_avg_sq is None else _contig(exp_avg_sq.to(torch.float32))
    if out is None or out.numel() * out.element_size() < n * 16:
        out = torch.empty(n * 4, dtype=torch.int32, device=packed.device)
    _lib.check(_lib.load().opus_build_sketch_table(_ptr(packed), _ptr(diag), _ptr(exp_avg_sq), float(eps), int(d_out),
                                                  int(d_in), _ptr(out), n, _stream(packed)),
               "opus_build_sketch_table")
    return out


def adam_diag(exp_avg_sq: torch.Tensor, eps: float = 1e-8) -> torch.Tensor:
    """The AdamW diagonal 1 / (sqrt(v) + eps) in f32, elementwise, same shape as v."""
    _cuda(exp_avg_sq, "exp_avg_sq")
    v = _contig(exp_avg_sq.to(torch.float32))
    out = torch.empty_like(v)
    _lib.check(_lib.load().opus_adam_diag(_ptr(v), float(eps), v.numel(), _ptr(out), _stream(v)), "opus_adam_diag")
    return out


# --------------------------------------------------------------------- stage 3
def split_bf16(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    _cuda(x, "x")
    x = _contig(x.to(torch.float32))
    hi = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    lo = torch.empty_like(hi)
    _lib.check(_lib.load().opus_split_bf16(_ptr(x), x.numel(), _ptr(hi), _ptr(lo), _stream(x)), "opus_split_bf16")
    return hi, lo


def _as3d(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dim() == 2:
        return t.unsqueeze(0)
    if t.dim() != 3:
        raise ValueError(f"Unexpected {name} shape: {tuple(t.shape)}")
    return t


# Longest row (in tokens) that sketch_gemm forms by merging samples that share an output row.
MERGE_TOKENS = 16384


def sketch_gemm(dLdZ: torch.Tensor, a: torch.Tensor, table: torch.Tensor, k: int, rows_div: int = 1,
                out: torch.Tensor | None = None, accumulate: bool = False,
                max_bucket_load: int = 0, alpha: float = 1.0) -> torch.Tensor:
    """phi[b // rows_div] (+)= alpha * CountSketch(w o (dLdZ_b^T a_b)) for every candidate b.

    dLdZ [B, T, d_out] and a [B, T, d_in] in bf16 (tensor cores directly) or
    f32 (split into bf16 hi/lo; hi*hi + hi*lo + lo*hi accumulated).
    max_bucket_load (see bucket_max_load) enables the fixed-point
    shared-memory sketch; 0 adds every update with f32 global atomics.
    alpha multiplies every update in f32 (the per-sample scaling of dL/dZ).
    """
    _cuda(dLdZ, "dLdZ")
    _cuda(a, "a")
    if dLdZ.dim() != 3 or a.dim() != 3 or dLdZ.shape[:2] != a.shape[:2]:
        raise ValueError(f"Unexpected dLdZ/a shapes: {tuple(dLdZ.shape)}, {tuple(a.shape)}")
    B, T, d_out = dLdZ.shape
    d_in = a.shape[2]
    rows = 0 if B == 0 else (B + rows_div - 1) // rows_div
    # The sketch is linear, and the G of a row of r*T tokens is the sum of its
    # r rows' G: samples that share an output row are merged into one long row
    # (a view), which scatters into the sketch once instead of r times.  The
    # merged row is kept to MERGE_TOKENS tokens: its G is one f32 accumulation
    # over all of them, whose rounding error grows with the length.
    g = math.gcd(rows_div, B)
    r = max([d for d in range(1, g + 1) if g % d == 0 and d * T <= MERGE_TOKENS] or [1])
    if r > 1:
        dLdZ = _contig(dLdZ).view(B // r, r * T, d_out)
        a = _contig(a).view(B // r, r * T, d_in)
        B, T, rows_div = B // r, r * T, rows_div // r
    if out is None:
        out = torch.empty(rows, k, dtype=torch.float32, device=dLdZ.device)
        accumulate = False
    if out.dtype != torch.float32 or not out.is_contiguous() or out.numel() < rows * k:
        raise ValueError("out must be a contiguous float32 tensor of at least [rows, k]")
    n_entries = table.numel() * table.element_size() // 16
    lib = _lib.load()

    def launch(g: torch.Tensor, x: torch.Tensor, acc: bool) -> None:
        _lib.check(lib.opus_sketch_gemm(_ptr(g), _ptr(x), _lib.DTYPE_BF16, B, T, d_out, d_in, _ptr(table), n_entries,
                                        int(k), int(max_bucket_load), int(rows_div), _ptr(out), int(acc),
                                        float(alpha), _stream(g)),
                   "opus_sketch_gemm")

    if dLdZ.dtype == torch.bfloat16 and a.dtype == torch.bfloat16:
        launch(_contig(dLdZ), _contig(a), accumulate)
    else:
        g_hi, g_lo = split_bf16(dLdZ)
        a_hi, a_lo = split_bf16(a)
        launch(g_hi, a_hi, accumulate)
        launch(g_hi, a_lo, True)
        launch(g_lo, a_hi, True)
    return out


def ghost_gram(a: torch.Tensor, dLdZ: torch.Tensor, alpha: float = 1.0, out: torch.Tensor | None = None,
               accumulate: bool = False) -> torch.Tensor:
    """S[i, j] (+)= alpha * <G_i, G_j>, G_b = dLdZ_b^T a_b, for every candidate pair, without forming any G_b.

    a [B, T, d_in], dLdZ [B, T, d_out] in bf16 (tensor cores directly) or f32
    (split into bf16 hi/lo; hi*hi + hi*lo + lo*hi per product).  Widths that
    are not multiples of 8 are zero-padded (zero features add nothing).
    """
    _cuda(a, "a")
    _cuda(dLdZ, "dLdZ")
    if dLdZ.dim() != 3 or a.dim() != 3 or dLdZ.shape[:2] != a.shape[:2]:
        raise ValueError(f"Unexpected dLdZ/a shapes: {tuple(dLdZ.shape)}, {tuple(a.shape)}")
    B, T, d_out = dLdZ.shape
    d_in = a.shape[2]
    if out is None:
        out = torch.empty(B, B, dtype=torch.float32, device=a.device)
        accumulate = False
    if out.dtype != torch.float32 or not out.is_contiguous() or out.numel() < B * B:
        raise ValueError("out must be a contiguous float32 tensor of at least [B, B]")
    a, dLdZ = _pad8(a), _pad8(dLdZ)
    lib = _lib.load()
    if a.dtype == torch.bfloat16 and dLdZ.dtype == torch.bfloat16:
        parts = (_contig(a), None, _contig(dLdZ), None)
    else:
        a_hi, a_lo = split_bf16(a)
        g_hi, g_lo = split_bf16(dLdZ)
        parts = (a_hi, a_lo, g_hi, g_lo)
    _lib.check(lib.opus_ghost_gram(_ptr(parts[0]), _ptr(parts[1]), _ptr(parts[2]), _ptr(parts[3]), _lib.DTYPE_BF16,
                                   B, T, a.shape[2], dLdZ.shape[2], float(alpha), _ptr(out), int(accumulate),
                                   _stream(a)), "opus_ghost_gram")
    return out


def _pad8(x: torch.Tensor) -> torch.Tensor:
    d = x.shape[-1]
    p = (d + 7) // 8 * 8
    return x if p == d else torch.nn.functional.pad(x, (0, p - d))


def per_sample_grad(dLdZ: torch.Tensor, a: torch.Tensor, diag: torch.Tensor | None = None,
                    out: torch.Tensor | None = None, accumulate: bool = False) -> torch.Tensor:
    """out[b] (+)= (diag o dLdZ_b^T a_b) flattened: exact per-sample gradients [B, d_out*d_in] in f32.

    dLdZ [B, T, d_out] and a [B, T, d_in] in bf16 (tensor cores directly) or
    f32 (split into bf16 hi/lo; hi*hi + hi*lo + lo*hi accumulated).  Widths
    that are not multiples of 8 are zero-padded for the kernel and the result
    is cut back to [B, d_out*d_in].
    """
    _cuda(dLdZ, "dLdZ")
    _cuda(a, "a")
    if dLdZ.dim() != 3 or a.dim() != 3 or dLdZ.shape[:2] != a.shape[:2]:
        raise ValueError(f"Unexpected dLdZ/a shapes: {tuple(dLdZ.shape)}, {tuple(a.shape)}")
    B, T, d_out = dLdZ.shape
    d_in = a.shape[2]
    if diag is not None:
        if tuple(diag.shape) != (d_out, d_in):
            raise ValueError(f"diag must be [{d_out}, {d_in}], got {tuple(diag.shape)}")
        diag = _contig(_cuda(diag, "diag").to(torch.float32))
    if out is None:
        out = torch.empty(B, d_out * d_in, dtype=torch.float32, device=dLdZ.device)
        accumulate = False
    if out.dtype != torch.float32 or not out.is_contiguous() or out.numel() < B * d_out * d_in:
        raise ValueError("out must be a contiguous float32 tensor of at least [B, d_out * d_in]")
    do_p, di_p = (d_out + 7) // 8 * 8, (d_in + 7) // 8 * 8
    padded = (do_p, di_p) != (d_out, d_in)
    if padded:
        dLdZ = torch.nn.functional.pad(dLdZ, (0, do_p - d_out))
        a = torch.nn.functional.pad(a, (0, di_p - d_in))
        if diag is not None:
            diag = torch.nn.functional.pad(diag, (0, di_p - d_in, 0, do_p - d_out))
        target = torch.empty(B, do_p * di_p, dtype=torch.float32, device=dLdZ.device)
    else:
        target = out
    lib = _lib.load()

    def launch(g: torch.Tensor, x: torch.Tensor, acc: bool) -> None:
        _lib.check(lib.opus_per_sample_grad(_ptr(g), _ptr(x), _lib.DTYPE_BF16, B, T, do_p, di_p, _ptr(diag),
                                            _ptr(target), int(acc), _stream(g)), "opus_per_sample_grad")

    first_acc = accumulate and not padded
    if dLdZ.dtype == torch.bfloat16 and a.dtype == torch.bfloat16:
        launch(_contig(dLdZ), _contig(a), first_acc)
    else:
        g_hi, g_lo = split_bf16(dLdZ)
        a_hi, a_lo = split_bf16(a)
        launch(g_hi, a_hi, first_acc)
        launch(g_hi, a_lo, True)
        launch(g_lo, a_hi, True)
    if padded:
        view = target.view(B, do_p, di_p)[:, :d_out, :d_in].reshape(B, d_out * d_in)
        dst = out.view(-1)[:B * d_out * d_in].view(B, d_out * d_in)
        if accumulate:
            dst += view
        else:
            dst.copy_(view)
    return out


def sketch_dense(w: torch.Tensor, packed: torch.Tensor, d_out: int, d_in: int, k: int, transposed: bool = False,
                 diag: torch.Tensor | None = None, out: torch.Tensor | None = None,
                 accumulate: bool = False, rows: tuple[int, int] | None = None,
                 max_bucket_load: int = 0) -> torch.Tensor:
    """sketch[h] += s * diag * W for a dense [d_out, d_in] (or [d_in, d_out] if transposed) matrix.

    rows=(lo, hi) adds only the rows lo <= o < hi of the [d_out, d_in] layout.
    max_bucket_load (bucket_max_load of the table) tightens the fixed-point
    scale of the shared-memory sketch; 0 falls back to the element count.
    """
    _cuda(w, "w")
    _cuda(packed, "packed")
    if w.numel() != d_out * d_in:
        raise ValueError(f"w has {w.numel()} elements, expected {d_out * d_in}")
    w = _contig(w.to(torch.float32))
    diag = None if diag is None else _contig(diag.to(torch.float32))
    lo, hi = (0, d_out) if rows is None else (int(rows[0]), int(rows[1]))
    if out is None:
        out = torch.empty(k, dtype=torch.float32, device=w.device)
        accumulate = False
    _lib.check(_lib.load().opus_sketch_dense(_ptr(w), int(bool(transposed)), _ptr(packed), _ptr(diag), int(d_out),
                                            int(d_in), lo, hi, int(k), int(max_bucket_load), _ptr(out),
                                            int(accumulate), _stream(w)), "opus_sketch_dense")
    return out


def sketch_dense_rows(w: torch.Tensor, packed: torch.Tensor, k: int, out: torch.Tensor | None = None,
                      accumulate: bool = False, max_bucket_load: int = 0) -> torch.Tensor:
    """CountSketch of every row of a [n, numel] matrix with one table of numel elements, [n, k] f32."""
    _cuda(w, "w")
    _cuda(packed, "packed")
    if w.dim() != 2 or w.shape[1] != packed.numel():
        raise ValueError(f"w must be [n, {packed.numel()}], got {tuple(w.shape)}")
    w = _contig(w.to(torch.float32))
    n = w.shape[0]
    if out is None:
        out = torch.empty(n, k, dtype=torch.float32, device=w.device)
        accumulate = False
    if out.dtype != torch.float32 or not out.is_contiguous() or out.numel() < n * k:
        raise ValueError("out must be a contiguous float32 tensor of at least [n, k]")
    _lib.check(_lib.load().opus_sketch_dense_rows(_ptr(w), n, w.shape[1], _ptr(_contig(packed)), int(k),
                                                 int(max_bucket_load), _ptr(out), int(accumulate), _stream(w)),
               "opus_sketch_dense_rows")
    return out


# --------------------------------------------------------------------- stage 2
def desketch(tau: torch.Tensor, packed: torch.Tensor, d_out: int, d_in: int, scale: float = 1.0,
             diag: torch.Tensor | None = None, exp_avg_sq: torch.Tensor | None = None,
             eps: float = 1e-8) -> torch.Tensor:
    """Dense target v = scale * D * s * tau[h] as a bf16 (hi, lo) pair [2, d_out, d_in]."""
    _cuda(tau, "tau")
    tau = _contig(tau.to(torch.float32))
    diag = None if diag is None else _contig(diag.to(torch.float32))
    exp_avg_sq = None if exp_avg_sq is None else _contig(exp_avg_sq.to(torch.float32))
    out = torch.empty(2, d_out, d_in, dtype=torch.bfloat16, device=tau.device)
    _lib.check(_lib.load().opus_desketch(_ptr(tau), _ptr(packed), _ptr(diag), _ptr(exp_avg_sq), float(eps), int(d_out),
                                        int(d_in), tau.numel(), float(scale), _ptr(out), _stream(tau)),
               "opus_desketch")
    return out


def dense_target_pair(v: torch.Tensor) -> torch.Tensor:
    """f32 [d_out, d_in] target -> bf16 (hi, lo) pair [2, d_out, d_in] for ghost_score."""
    hi, lo = split_bf16(v)
    return torch.stack([hi, lo])


def ghost_score(a: torch.Tensor, dLdZ: torch.Tensor, v_pair: torch.Tensor, alpha: float = 1.0,
                out: torch.Tensor | None = None, accumulate: bool = False) -> torch.Tensor:
    """score[b] (+)= alpha * <dLdZ_b^T a_b, v> without forming per-sample gradients."""
    _cuda(a, "a")
    _cuda(dLdZ, "dLdZ")
    if a.dim() != 3 or dLdZ.dim() != 3 or a.shape[:2] != dLdZ.shape[:2]:
        raise ValueError(f"Unexpected a/dLdZ shapes: {tuple(a.shape)}, {tuple(dLdZ.shape)}")
    B, T, d_in = a.shape
    d_out = dLdZ.shape[2]
    if v_pair.shape != (2, d_out, d_in) or v_pair.dtype != torch.bfloat16:
        raise ValueError(f"v_pair must be bf16 [2, {d_out}, {d_in}], got {v_pair.dtype} {tuple(v_pair.shape)}")
    if out is None:
        out = torch.empty(B, dtype=torch.float32, device=a.device)
        accumulate = False
    lib = _lib.load()
    v_pair = _contig(v_pair)

    def launch(x: torch.Tensor, g: torch.Tensor, acc: bool) -> None:
        _lib.check(lib.opus_ghost_score(_ptr(x), _ptr(g), _lib.DTYPE_BF16, B, T, d_in, d_out, _ptr(v_pair),
                                        float(alpha), _ptr(out), int(acc), _stream(x)), "opus_ghost_score")

    if a.dtype == torch.bfloat16 and dLdZ.dtype == torch.bfloat16:
        launch(_contig(a), _contig(dLdZ), accumulate)
    else:
        a_hi, a_lo = split_bf16(a)
        g_hi, g_lo = split_bf16(dLdZ)
        launch(a_hi, g_hi, accumulate)
        launch(a_lo, g_hi, True)
        launch(a_hi, g_lo, True)
    return out


# --------------------------------------------------------------------- dots
def sketch_dot(phi: torch.Tensor, tau: torch.Tensor, alpha: float = 1.0, out: torch.Tensor | None = None,
               accumulate: bool = False) -> torch.Tensor:
    _cuda(phi, "phi")
    phi, tau = _contig(phi), _contig(tau)
    B, k = phi.shape
    if tau.numel() != k:
        raise ValueError("tau length must equal the sketch dimension")
    if out is None:
        out = torch.empty(B, dtype=torch.float32, device=phi.device)
        accumulate = False
    _lib.check(_lib.load().opus_sketch_dot(_ptr(phi), _ptr(tau), B, k, float(alpha), _ptr(out), int(accumulate),
                                          _stream(phi)), "opus_sketch_dot")
    return out


def sketch_dot_layers(phis: torch.Tensor, taus: torch.Tensor, alphas: torch.Tensor,
                      out: torch.Tensor | None = None, accumulate: bool = False) -> torch.Tensor:
    """out[b] (+)= sum_l alphas[l] * phis[l, b] . taus[l], every layer in one launch.

    phis [L, B, k] (each layer's [B, k] block contiguous; the layer stride may be
    larger, as for rows [lo, hi) of a longer buffer), taus [L, k], alphas [L] f32.
    """
    _cuda(phis, "phis")
    if phis.dim() != 3 or phis.stride(2) != 1 or phis.stride(1) != phis.shape[2]:
        raise ValueError("phis must be [L, B, k] with contiguous [B, k] blocks")
    L, B, k = phis.shape
    taus = _contig(taus.to(torch.float32))
    alphas = _contig(alphas.to(device=phis.device, dtype=torch.float32))
    if taus.shape != (L, k) or alphas.numel() != L:
        raise ValueError(f"taus must be [{L}, {k}] and alphas [{L}]")
    if out is None:
        out = torch.empty(B, dtype=torch.float32, device=phis.device)
        accumulate = False
    _lib.check(_lib.load().opus_sketch_dot_layers(_ptr(phis), int(phis.stride(0)), _ptr(taus), _ptr(alphas), L, B,
                                                 k, _ptr(out), int(accumulate), _stream(phis)),
               "opus_sketch_dot_layers")
    return out


def sketch_gram(phi_a: torch.Tensor, phi_b: torch.Tensor | None = None, alpha: float = 1.0,
                out: torch.Tensor | None = None, accumulate: bool = False) -> torch.Tensor:
    _cuda(phi_a, "phi_a")
    phi_a = _contig(phi_a)
    phi_b = phi_a if phi_b is None else _contig(phi_b)
    ra, k = phi_a.shape
    rb = phi_b.shape[0]
    if phi_b.shape[1] != k:
        raise ValueError("sketch dimensions differ")
    if out is None:
        out = torch.empty(ra, rb, dtype=torch.float32, device=phi_a.device)
        accumulate = False
    _lib.check(_lib.load().opus_sketch_gram(_ptr(phi_a), ra, _ptr(phi_b), rb, k, float(alpha), _ptr(out),
                                           int(accumulate), _stream(phi_a)), "opus_sketch_gram")
    return out


# --------------------------------------------------------------------- stage 4 (Muon)
def gemm_bf16(a: torch.Tensor, b: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16, alpha: float = 1.0,
              a_lo: torch.Tensor | None = None, out: torch.Tensor | None = None,
              accumulate: bool = False) -> torch.Tensor:
    """C = alpha * (a (+ a_lo)) @ b^T on the tensor cores: a [M, K], b [N, K] bf16, f32 accumulation.

    out_dtype bfloat16 rounds every f32 sum once (torch's .to(bfloat16));
    float32 keeps it (accumulate adds into out).  K and N multiples of 8.
    """
    _cuda(a, "a")
    _cuda(b, "b")
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[1]:
        raise ValueError(f"gemm_bf16: a [M, K] and b [N, K] expected, got {tuple(a.shape)}, {tuple(b.shape)}")
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16 or (a_lo is not None and a_lo.dtype != torch.bfloat16):
        raise ValueError("gemm_bf16: operands must be bf16")
    if a_lo is not None and a_lo.shape != a.shape:
        raise ValueError("gemm_bf16: a_lo must have a's shape")
    if out_dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("gemm_bf16: out_dtype must be bfloat16 or float32")
    M, K = a.shape
    N = b.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=out_dtype, device=a.device)
        accumulate = False
    if out.dtype != out_dtype or not out.is_contiguous() or out.numel() < M * N:
        raise ValueError(f"out must be a contiguous {out_dtype} tensor of at least [M, N]")
    if M == 0:
        return out
    dt = _lib.DTYPE_BF16 if out_dtype == torch.bfloat16 else _lib.DTYPE_F32
    a, b = _contig(a), _contig(b)
    a_lo = None if a_lo is None else _contig(a_lo)
    _lib.check(_lib.load().opus_gemm_bf16(_ptr(a), _ptr(a_lo), _ptr(b), M, N, K, float(alpha), _ptr(out), dt,
                                         int(accumulate), _stream(a)), "opus_gemm_bf16")
    return out


def muon_S(m: torch.Tensor) -> torch.Tensor:
    """Muon preconditioner S = a I + b A + c A^2, A = m~ m~^T, m~ = m / ||m||, as bf16 [d_out, d_out].

    m: the momentum buffer [d_out, d_in] (f32 or bf16; other dtypes are cast
    to bf16 first, as the reference does).  Every step rounds to bf16 where
    the reference's bf16 torch arithmetic does; the identity when
    ||m|| < 1e-7.  Widths that are not multiples of 8 are zero-padded (zero
    rows and columns change neither the norm nor the valid block of S).
    """
    _cuda(m, "m")
    if m.dim() != 2:
        raise ValueError(f"muon_S: momentum buffer must be 2-D, got {tuple(m.shape)}")
    if m.dtype not in (torch.float32, torch.bfloat16):
        m = m.to(torch.bfloat16)
    d_out, d_in = m.shape
    do_p, di_p = (d_out + 7) // 8 * 8, (d_in + 7) // 8 * 8
    if (do_p, di_p) != (d_out, d_in):
        m = torch.nn.functional.pad(m, (0, di_p - d_in, 0, do_p - d_out))
    m = _contig(m)
    lib = _lib.load()
    ws_bytes = int(lib.opus_muon_S_workspace_bytes(do_p, di_p))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=m.device)
    S = torch.empty(do_p, do_p, dtype=torch.bfloat16, device=m.device)
    dt = _lib.DTYPE_F32 if m.dtype == torch.float32 else _lib.DTYPE_BF16
    _lib.check(lib.opus_muon_S(_ptr(m), dt, do_p, di_p, _ptr(ws), ws_bytes, _ptr(S), _stream(m)), "opus_muon_S")
    return S if do_p == d_out else S[:d_out, :d_out].contiguous()


def muon_transform(dLdZ: torch.Tensor, S: torch.Tensor, symmetric: bool = False) -> torch.Tensor:
    """einsum('...o,po->...p', dLdZ.float(), S.float().T).to(dLdZ.dtype) on the tensor cores.

    The Muon candidate transform (data_selection.py:495-500): out[..., p] =
    sum_o dLdZ[..., o] S[o, p].  bf16 dLdZ with a bf16 S is one GEMM with a
    bf16 output; f32 dLdZ is split into bf16 hi/lo (two products, f32
    output); an f32 S that bf16 does not hold exactly is split as well.
    symmetric=True skips the transpose of S (the S of muon_S is symmetric).
    """
    _cuda(dLdZ, "dLdZ")
    _cuda(S, "S")
    d_out = dLdZ.shape[-1]
    if S.shape != (d_out, d_out):
        raise ValueError(f"S must be [{d_out}, {d_out}], got {tuple(S.shape)}")
    lead = dLdZ.shape[:-1]
    g = dLdZ.reshape(-1, d_out)
    Bm = S if symmetric else S.t()
    p = (d_out + 7) // 8 * 8
    if p != d_out:
        g = torch.nn.functional.pad(g, (0, p - d_out))
        Bm = torch.nn.functional.pad(Bm, (0, p - d_out, 0, p - d_out))
    Bm = _contig(Bm)
    if Bm.dtype == torch.bfloat16:
        b_hi, b_lo = Bm, None
    else:
        b_hi, b_lo = split_bf16(Bm)
        if not bool(torch.any(b_lo != 0)):
            b_lo = None
    if g.dtype == torch.bfloat16 and b_lo is None:
        out = gemm_bf16(g, b_hi, out_dtype=torch.bfloat16)
    else:
        if g.dtype == torch.bfloat16:
            g_hi, g_lo = _contig(g), None
        else:
            g_hi, g_lo = split_bf16(g)
        out = gemm_bf16(g_hi, b_hi, out_dtype=torch.float32, a_lo=g_lo)
        if b_lo is not None:
            gemm_bf16(g_hi, b_lo, out_dtype=torch.float32, out=out, accumulate=True)
        out = out.to(dLdZ.dtype)
    if p != d_out:
        out = out[:, :d_out]
    return out.reshape(*lead, d_out)


def kernel_launches() -> int:
    """Kernels the library has launched in this process so far."""
    return int(_lib.load().opus_kernel_launches())


# --------------------------------------------------------------------- stage 5
def _sim_operand(sim: torch.Tensor, n: int) -> tuple[torch.Tensor, int]:
    """Dense [n, n] interaction matrix (block 0) or block-diagonal blocks [q, b, b] (block b, q*b == n)."""
    sim = _contig(sim.to(torch.float32))
    if sim.dim() == 3:
        q, b, b2 = sim.shape
        if b != b2 or q * b != n:
            raise ValueError(f"interaction blocks must be [q, b, b] with q*b == {n}, got {tuple(sim.shape)}")
        return sim, b
    if sim.shape != (n, n):
        raise ValueError(f"interaction matrix must be [{n}, {n}]")
    return sim, 0


def boltzmann_select(scores: torch.Tensor, sim: torch.Tensor, n_select: int, temperature: float,
                     uniforms: torch.Tensor) -> torch.Tensor:
    """Stochastic greedy selection on the device; uniforms: float64 [n_select] (one per draw).

    sim is the dense [n, n] interaction matrix, or [q, b, b] blocks of a
    block-diagonal one (candidates sharded over q ranks of b each).
    """
    _cuda(scores, "scores")
    scores = _contig(scores.to(torch.float32).reshape(-1))
    n = scores.numel()
    sim, block = _sim_operand(sim, n)
    if n_select > n:
        raise ValueError(f"cannot select {n_select} of {n} candidates")
    uniforms = _contig(uniforms.to(device=scores.device, dtype=torch.float64).reshape(-1))
    if uniforms.numel() < n_select:
        raise ValueError("need one uniform per draw")
    out = torch.empty(n_select, dtype=torch.int64, device=scores.device)
    lib = _lib.load()
    if block:
        rc = lib.opus_boltzmann_select_blocks(_ptr(scores), _ptr(sim), n, block, int(n_select), float(temperature),
                                              _ptr(uniforms), _ptr(out), _stream(scores))
    else:
        rc = lib.opus_boltzmann_select(_ptr(scores), _ptr(sim), n, int(n_select), float(temperature),
                                       _ptr(uniforms), _ptr(out), _stream(scores))
    _lib.check(rc, "opus_boltzmann_select")
    return out


def greedy_select(scores: torch.Tensor, sim: torch.Tensor, n_select: int) -> torch.Tensor:
    """Greedy selection on the device; sim dense [n, n] or block-diagonal blocks [q, b, b]."""
    _cuda(scores, "scores")
    scores = _contig(scores.to(torch.float32).reshape(-1))
    n = scores.numel()
    sim, block = _sim_operand(sim, n)
    out = torch.empty(n_select, dtype=torch.int64, device=scores.device)
    lib = _lib.load()
    if block:
        rc = lib.opus_greedy_select_blocks(_ptr(scores), _ptr(sim), n, block, int(n_select), _ptr(out),
                                           _stream(scores))
    else:
        rc = lib.opus_greedy_select(_ptr(scores), _ptr(sim), n, int(n_select), _ptr(out), _stream(scores))
    _lib.check(rc, "opus_greedy_select")
    return out


