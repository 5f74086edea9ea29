"""CountSketch projector (drop-in for OPUS/train/random_projection.py:21-198).

A weight element p of a layer is hashed to bucket h(p) in [0, k) with sign
s(p) in {-1, +1}; the sketch of a vector u is phi[j] = sum_{h(p)=j} s(p) u[p].
The tables come from the reference's own generator recipe
(random_projection.py:51-70): a torch.Generator on the projector's device
seeded with seed + param_id * 1000003 + numel, drawing the buckets with
torch.randint(0, k) and then, from the same generator, the signs with
torch.randint(0, 2) * 2 - 1.  They are generated once, packed on the compute
device into 4 bytes per element (bucket | sign bit) and kept; all projection
work runs in the sm_100a kernels of libopus_b200.so.
"""
from __future__ import annotations

import torch

from .. import ops


def _round8(n: int) -> int:
    return (n + 7) // 8 * 8


class GradientProjector:
    """CountSketch projector with the reference's constructor and methods."""

    def __init__(self, sketch_dim: int = 16384, seed: int = 42, device: str = "cuda", enabled: bool = True):
        self.sketch_dim = sketch_dim
        self.seed = seed
        self.device = device
        self.enabled = enabled
        # Reference-visible tables, filled only by explicit _get_hash_and_sign calls.
        self.hash_functions: dict = {}
        self.sign_functions: dict = {}
        # (numel, param_id, compute device) -> packed uint32 table (int32 storage)
        self._packed: dict = {}
        # (numel, param_id) -> largest bucket load (bounds the fixed-point sketch)
        self._max_load: dict = {}
        # (numel, param_id, d_out, d_in, compute device) -> sign-only epilogue table
        self._sign_tables: dict = {}

    # ------------------------------------------------------------ tables
    def _generate(self, param_numel: int, param_id: int) -> tuple[torch.Tensor, torch.Tensor]:
        gen = torch.Generator(device=self.device)
        gen.manual_seed(self.seed + param_id * 1000003 + param_numel)
        h = torch.randint(0, self.sketch_dim, (param_numel,), generator=gen, device=self.device, dtype=torch.long)
        s = torch.randint(0, 2, (param_numel,), generator=gen, device=self.device, dtype=torch.float32) * 2 - 1
        return h, s

    def _get_hash_and_sign(self, param_numel: int, param_id: int):
        """The reference's (bucket int64, sign float32) tables, cached per (numel, param_id)."""
        key = (param_numel, param_id)
        if key not in self.hash_functions:
            self.hash_functions[key], self.sign_functions[key] = self._generate(param_numel, param_id)
        return self.hash_functions[key], self.sign_functions[key]

    def packed_table(self, param_numel: int, param_id: int, device) -> torch.Tensor:
        """Packed uint32 (bucket | sign<<31) table on `device`, generated once."""
        device = torch.device(device)
        key = (param_numel, param_id, device)
        t = self._packed.get(key)
        if t is None:
            cached = (param_numel, param_id) in self.hash_functions
            h, s = self._get_hash_and_sign(param_numel, param_id) if cached else self._generate(param_numel, param_id)
            t = ops.pack_hash_sign(h.to(device), s.to(device), self.sketch_dim)
            self._packed[key] = t
            if (param_numel, param_id) not in self._max_load:
                self._max_load[(param_numel, param_id)] = ops.bucket_max_load(t, self.sketch_dim)
        return t

    def max_bucket_load(self, param_numel: int, param_id: int, device) -> int:
        """Largest number of a parameter's elements hashed to one bucket."""
        self.packed_table(param_numel, param_id, device)
        return self._max_load[(param_numel, param_id)]

    def layer_table(self, d_out: int, d_in: int, param_id: int, device, diag: torch.Tensor | None = None,
                    exp_avg_sq: torch.Tensor | None = None, eps: float = 1e-8) -> tuple[torch.Tensor, int, int]:
        """Epilogue table of a [d_out, d_in] layer for ops.sketch_gemm, padded to multiples of 8.

        Returns (table, d_out_padded, d_in_padded).  Padded elements carry
        bucket 0 and weight 0.  Without a preconditioner the table is cached.
        """
        device = torch.device(device)
        numel = d_out * d_in
        do_p, di_p = _round8(d_out), _round8(d_in)
        key = (numel, param_id, d_out, d_in, device)
        if diag is None and exp_avg_sq is None and key in self._sign_tables:
            return self._sign_tables[key], do_p, di_p
        packed = self.packed_table(numel, param_id, device)
        if (do_p, di_p) != (d_out, d_in):
            pad = torch.zeros(do_p, di_p, dtype=packed.dtype, device=device)
            pad[:d_out, :d_in] = packed.view(d_out, d_in)
            packed = pad

            def padded(x):
                if x is None:
                    return None
                y = torch.zeros(do_p, di_p, dtype=torch.float32, device=device)
                y[:d_out, :d_in] = x.reshape(d_out, d_in)
                return y

            diag, exp_avg_sq = padded(diag), padded(exp_avg_sq)
        table = ops.build_sketch_table(packed, do_p, di_p, diag=diag, exp_avg_sq=exp_avg_sq, eps=eps)
        if diag is None and exp_avg_sq is None:
            self._sign_tables[key] = table
        return table, do_p, di_p

    # ------------------------------------------------------------ projections
    def project_vector(self, vector: torch.Tensor, param_id: int) -> torch.Tensor:
        """CountSketch of one vector (random_projection.py:72-99)."""
        if not self.enabled:
            return vector
        flat = vector.flatten()
        numel = flat.numel()
        packed = self.packed_table(numel, param_id, flat.device)
        return ops.sketch_dense(flat, packed, 1, numel, self.sketch_dim,
                                max_bucket_load=self.max_bucket_load(numel, param_id, flat.device))

    def project_batch(self, vectors: torch.Tensor, param_id: int) -> torch.Tensor:
        """CountSketch of each row of a [B, d] batch (random_projection.py:101-132)."""
        if not self.enabled:
            return vectors
        B, d = vectors.shape
        packed = self.packed_table(d, param_id, vectors.device)
        return ops.sketch_dense_rows(vectors, packed, self.sketch_dim,  # every row in one launch
                                     max_bucket_load=self.max_bucket_load(d, param_id, vectors.device))

    def project_full_gradient(self, dLdZ: torch.Tensor, a: torch.Tensor, param_id: int,
                              preconditioner_S: torch.Tensor | None = None,
                              diagonal_preconditioner: torch.Tensor | None = None) -> torch.Tensor:
        """phi_b = CountSketch(D o (S-transformed dLdZ_b)^T a_b) for every sample b.

        Same contract as random_projection.py:134-193: dLdZ [B, D_out] or
        [B, T, D_out], a [B, D_in] or [B, T, D_in], optional dense left
        preconditioner S [D_out, D_out] and AdamW diagonal D [D_out, D_in];
        returns float32 [B, sketch_dim].  One fused kernel pass per layer
        replaces the reference's 32-row chunk loop.
        """
        if not self.enabled:
            raise ValueError("Projector is disabled but project_full_gradient was called")
        if preconditioner_S is not None:  # random_projection.py:155-158, on the tensor cores
            dLdZ = ops.muon_transform(dLdZ, preconditioner_S.to(dLdZ.device))
        if dLdZ.dim() == 2:
            dLdZ, a = dLdZ.unsqueeze(1), a.unsqueeze(1)
        elif dLdZ.dim() != 3:
            raise ValueError(f"Unexpected dLdZ shape: {dLdZ.shape}")
        return self.sketch(dLdZ, a, param_id, diag=diagonal_preconditioner)

    def sketch(self, dLdZ: torch.Tensor, a: torch.Tensor, param_id: int, diag: torch.Tensor | None = None,
               exp_avg_sq: torch.Tensor | None = None, eps: float = 1e-8, rows_div: int = 1,
               out: torch.Tensor | None = None, accumulate: bool = False,
               table_cache: dict | None = None, alpha: float = 1.0) -> torch.Tensor:
        """Per-sample sketches of [B, T, *] factors (rows_div > 1 sums groups of samples).

        table_cache: a dict that keeps the preconditioned tables of this call's
        parameter for later calls with the same diagonal (the passes of one
        round); the caller owns it and drops it when the optimizer state moves.
        alpha: f32 factor on the sketch (dL/dZ's per-sample scaling).
        """
        B, T, d_out = dLdZ.shape
        d_in = a.shape[2]
        if diag is not None:
            diag = diag.to(device=dLdZ.device, dtype=torch.float32)
        cached = None if table_cache is None else table_cache.get(param_id)
        if cached is not None:
            table, do_p, di_p = cached
        else:
            table, do_p, di_p = self.layer_table(d_out, d_in, param_id, dLdZ.device, diag=diag,
                                                 exp_avg_sq=exp_avg_sq, eps=eps)
            if table_cache is not None and (diag is not None or exp_avg_sq is not None):
                table_cache[param_id] = (table, do_p, di_p)
        if do_p != d_out:
            dLdZ = torch.nn.functional.pad(dLdZ, (0, do_p - d_out))
        if di_p != d_in:
            a = torch.nn.functional.pad(a, (0, di_p - d_in))
        # padded elements (bucket 0, weight 0) add exact zeros: they do not count toward the load
        load = self.max_bucket_load(d_out * d_in, param_id, dLdZ.device)
        return ops.sketch_gemm(dLdZ, a, table, self.sketch_dim, rows_div=rows_div, out=out, accumulate=accumulate,
                               max_bucket_load=load, alpha=alpha)

    def clear_cache(self):
        """Drop every cached table (random_projection.py:195-198)."""
        self.hash_functions.clear()
        self.sign_functions.clear()
        self._packed.clear()
        self._sign_tables.clear()
        self._max_load.clear()
