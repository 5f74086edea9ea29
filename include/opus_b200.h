/*
 * opus_b200.h — C ABI of libopus_b200.so, the B200 (sm_100a) kernels behind
 * the OPUS per-iteration data-selection path.
 *
 * Conventions
 *   - Every entry point returns int: 0 (OPUS_OK) on success, otherwise an
 *     OPUS_ERR_* code; opus_last_error() returns the message of the last
 *     failure on the calling thread.  No C++ exception crosses this boundary.
 *   - All array arguments are device pointers owned by the caller (unless
 *     stated otherwise); nothing is retained after the call returns.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Calls are
 *     asynchronous with respect to the host; results are valid after the
 *     stream is synchronised.
 *   - Device-side failures (a bounded wait that expired) are recorded in a
 *     per-device error word; opus_device_error() synchronises the device and
 *     returns and clears it.
 *   - Matrices are row-major.  A layer weight is [d_out, d_in]; its per-sample
 *     gradient is G_b = sum_t dLdZ[b,t,:]^T a[b,t,:], flattened row-major,
 *     which is the element order of the CountSketch tables.
 *
 * Reference interfaces (gszfwsb/OPUS) each entry point replaces are cited as
 * path:line.
 */
#ifndef OPUS_B200_H_
#define OPUS_B200_H_

#include <stdint.h>

#if defined(__GNUC__)
#define OPUS_API __attribute__((visibility("default")))
#else
#define OPUS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define OPUS_ABI_VERSION 3

#define OPUS_OK 0
#define OPUS_ERR_INVALID 1     /* bad argument (maps to ValueError) */
#define OPUS_ERR_CUDA 2        /* CUDA runtime/driver failure (RuntimeError) */
#define OPUS_ERR_UNSUPPORTED 3 /* shape/dtype outside what the kernels handle */
#define OPUS_ERR_DEVICE 4      /* device-side error word was set */

#define OPUS_DTYPE_BF16 0
#define OPUS_DTYPE_F32 1

/* Library version (OPUS_ABI_VERSION). */
OPUS_API int opus_abi_version(void);

/* Message of the last failing call on this thread ("" if none). */
OPUS_API const char* opus_last_error(void);

/* Synchronise the current device, store its device error word in *code
 * (0 = none) and clear it.  Returns OPUS_ERR_DEVICE when *code != 0. */
OPUS_API int opus_device_error(int* code);

/*
 * Self-test of the bounded waits (no reference counterpart).  Every pipelined
 * kernel waits on mbarriers with a wall-clock limit (1 s) and, when a wait
 * runs out, records a code in the device error word, sets its CTA's abort
 * flag and returns instead of hanging.  This launches one thread that waits
 * on an mbarrier nothing arrives on: after the limit it records 0x106, which
 * opus_device_error then reports, and the context stays usable.
 */
OPUS_API int opus_selftest_stalled_wait(void* stream);

/*
 * H1 — pack the reference's CountSketch tables.
 * Replaces the tensors built by GradientProjector._get_hash_and_sign
 * (OPUS/train/random_projection.py:51-70): hash int64 in [0,k) and sign
 * float32 in {-1,+1}, one per weight element.  Output: one uint32 per element,
 * bucket in bits [0,31), bit 31 set when the sign is -1 (4 B/elem instead of
 * 12).  Fails with OPUS_ERR_INVALID if a bucket is outside [0,k) or a sign is
 * not +-1 (checked on the device; reported through opus_device_error).
 */
OPUS_API int opus_pack_hash_sign(const int64_t* hash, const float* sign, int64_t numel, int64_t k,
                        uint32_t* packed, void* stream);

/*
 * H1 — per-bucket element counts of a packed table and their maximum.
 * opus_sketch_gemm sizes its int32 fixed-point shared-memory sketch by the
 * largest bucket load.  The reference has no such step: its scatter_add_
 * (OPUS/train/random_projection.py:317) accumulates in f32 and needs no bound.
 *   counts: caller-owned scratch of counts_len >= k int32, zeroed here and
 *           left holding the histogram; out_max: one int64 on the device.
 * A bucket outside [0,k) is skipped and reported through opus_device_error.
 */
OPUS_API int opus_bucket_max_load(const uint32_t* packed, int64_t numel, int64_t k, int* counts,
                                  int64_t counts_len, int64_t* out_max, void* stream);

/*
 * The same maximum as opus_bucket_max_load, computed without allocating any
 * device memory: no reference counterpart (the reference has no bucket-load
 * step at all).  Some hosts cannot hand the library a k-entry workspace: a
 * process that reserves its device memory up front and treats any later
 * allocation as a failure, or an out-of-memory path that needs the bound
 * while the allocator has nothing left to give.  This entry point counts in a
 * static device array of the library instead.
 *   - k <= 262144 (1 MB of counts); larger k is rejected with OPUS_ERR_INVALID.
 *   - The first call on each device looks up the array's address
 *     (cudaGetSymbolAddress) with that device current; make that first call
 *     before any stream capture.  The address is kept per device and per
 *     context: after cudaDeviceReset the next call looks it up again.
 *   - Every call zeroes the array on its stream before counting.  Calls that
 *     overlap on one device share the array and race: serialise them.
 *   - *out_max (one int64 on the device) is -1 when a bucket lies outside
 *     [0,k); the library's device error word is not touched.
 */
OPUS_API int opus_bucket_max_load_noalloc(const uint32_t* packed, int64_t numel, int64_t k, int64_t* out_max,
                                          void* stream);

/* P3 — the AdamW diagonal D = 1 / (sqrt(v) + eps) of n second moments, f32,
 * with torch's correctly rounded sqrt, add and reciprocal
 * (_inv_rms_tensor_for_param, OPUS/train/data_selection.py:208-214). */
OPUS_API int opus_adam_diag(const float* exp_avg_sq, float eps, int64_t n, float* out, void* stream);

/* Number of 16-byte entries of the tiled epilogue table for a [d_out,d_in] layer. */
OPUS_API int64_t opus_sketch_table_entries(int d_out, int d_in);

/*
 * P3 + H1 — per-layer epilogue table for opus_sketch_gemm: for every weight
 * element (o,c) the bucket h(o,c) and the weight s(o,c)*D(o,c), where D is
 *   - diag[o,c]                          if diag != NULL,
 *   - 1/(sqrt(exp_avg_sq[o,c]) + eps)    if exp_avg_sq != NULL (AdamW),
 *   - 1                                  otherwise (SGD / Muon / proxy side).
 * Replaces _inv_rms_tensor_for_param (OPUS/train/data_selection.py:208-214)
 * and the per-chunk `grad_chunk * diag` / `* s` products of
 * project_full_gradient (OPUS/train/random_projection.py:186-190).
 */
OPUS_API int opus_build_sketch_table(const uint32_t* packed, const float* diag, const float* exp_avg_sq,
                            float eps, int d_out, int d_in, void* table, int64_t table_entries,
                            void* stream);

/*
 * S-proj (stage 3) — per-sample CountSketch of preconditioned per-sample
 * gradients, fused: a tcgen05 GEMM forms each 128x256 tile of
 * G_b = dLdZ_b^T a_b in TMEM and its epilogue scatters w(o,c)*G_b[o,c] into
 * the sketch row of candidate b; G_b never reaches HBM.
 *   dLdZ: [n_rows, seq_len, d_out], a: [n_rows, seq_len, d_in], contiguous;
 *         dtype must be OPUS_DTYPE_BF16 (f32 operands: split each with
 *         opus_split_bf16 and accumulate hi*hi + hi*lo + lo*hi, CountSketch
 *         being linear).  d_out and d_in must be multiples of 8.
 *   phi:  [ceil(n_rows/rows_div), k] f32; row b/rows_div receives candidate b
 *         (rows_div = n_rows sums the proxy batch into one row).
 *   max_bucket_load: the largest number of weight elements sharing one bucket
 *         (max of the bucket histogram).  It bounds the CTA's 32-bit
 *         fixed-point shared-memory sketch so no bucket can overflow; <= 0
 *         sends every update to f32 global atomics instead (exact, slower).
 *   accumulate = 0 zeroes phi first.
 *   alpha: f32 factor on every update (1 for the reference's values).  The
 *         capture's per-sample scaling of dL/dZ by the batch size
 *         (OPUS/layers/linear.py:118-119) can ride here instead of a pass
 *         over dL/dZ.
 * Accuracy: each update is rounded to a power-of-two quantum of at most
 * 2^-(log2(2^31/max_bucket_load) - 3) times the largest |w G| of a sample
 * of the job's first tile in the CTA, itself at most the tile's largest
 * (~1e-6 relative for GPT-2 layers); larger, NaN or Inf updates are added
 * exactly in f32.
 * Replaces GradientProjector.project_full_gradient
 * (OPUS/train/random_projection.py:134-193) on 3-D inputs.
 */
OPUS_API int opus_sketch_gemm(const void* dLdZ, const void* a, int dtype, int n_rows, int seq_len, int d_out,
                     int d_in, const void* table, int64_t table_entries, int64_t k, int max_bucket_load,
                     int rows_div, float* phi, int accumulate, float alpha, void* stream);

/*
 * G-ghost (projection off) — exact per-sample gradients for the similarity.
 * Replaces the per-sample gradient materialisation of weighted_grad_dotprod
 * (OPUS/train/data_selection.py:255-292, 32-row chunks of the per-example
 * gradient of OPUS/layers/linear.py:41-68, times the diagonal) and of
 * grad_dotprod (OPUS/train/data_selection.py:597-619).
 *   out[b, o*d_in + c] (+)= diag[o, c] * sum_t dLdZ[b, t, o] * a[b, t, c]
 * dLdZ [n_rows, seq_len, d_out] and a [n_rows, seq_len, d_in] bf16 (dtype
 * OPUS_DTYPE_BF16), d_out and d_in multiples of 8; diag [d_out, d_in] f32 or
 * NULL (no weighting); out [n_rows, d_out*d_in] f32, written in full unless
 * accumulate.  The tcgen05 GEMM of opus_sketch_gemm with a dense epilogue:
 * each element has one writer, so no scatter and no atomics (vector
 * reductions when accumulating).
 */
/*
 * G-ghost Gram (projection off, SGD / Muon) — the candidate similarity
 * without per-sample gradients: S[i, j] (+)= alpha * <G_i, G_j> for every
 * pair, G_b = dLdZ_b^T a_b, as sum over token pairs of
 * (a_i a_j^T) o (dLdZ_i dLdZ_j^T): two tcgen05 GEMMs per 128 x 128 token block
 * with a fused row-dot epilogue.  Equals the Gram of the per-sample gradients
 * of grad_dotprod (OPUS/train/data_selection.py:597-619); cheaper than
 * materialising them when 2 T^2 (d_in + d_out) (B + 1) / 2 < 2 T d_in d_out
 * + B d_in d_out per candidate, i.e. for short windows.  a [n_rows, seq_len,
 * d_in], dLdZ [n_rows, seq_len, d_out] bf16 (a_lo / dLdZ_lo: the lo halves of
 * f32 operands split with opus_split_bf16, or both NULL); d_in, d_out
 * multiples of 8; S [n_rows, n_rows] f32, zeroed first unless accumulate.
 */
OPUS_API int opus_ghost_gram(const void* a, const void* a_lo, const void* dLdZ, const void* dLdZ_lo, int dtype,
                    int n_rows, int seq_len, int d_in, int d_out, float alpha, float* S, int accumulate,
                    void* stream);

OPUS_API int opus_per_sample_grad(const void* dLdZ, const void* a, int dtype, int n_rows, int seq_len, int d_out,
                         int d_in, const float* diag, float* out, int accumulate, void* stream);

/*
 * K1 — dense CountSketch of one [d_out,d_in] f32 matrix (the proxy target
 * direction): sketch[h(o,c)] += s(o,c) * diag(o,c) * w(o,c), with w read as
 * w[o*d_in+c] (transposed = 0) or w[c*d_out+o] (transposed = 1); diag may be
 * NULL.  Only rows row_begin <= o < row_end are added (0, d_out for the whole
 * matrix): ranks that share the target each sketch their rows and sum the
 * partial sketches.  max_bucket_load: the table's largest bucket load
 * (opus_bucket_max_load), or 0 when unknown; it bounds the int32 fixed-point
 * shared-memory sketch, and the element count bounds it otherwise, at about
 * 100 times coarser rounding (still below 1e-4 of the largest bucket).
 * Replaces GradientProjector.project_vector
 * (OPUS/train/random_projection.py:72-99).
 */
OPUS_API int opus_sketch_dense(const float* w, int transposed, const uint32_t* packed, const float* diag,
                               int d_out, int d_in, int row_begin, int row_end, int64_t k, int max_bucket_load,
                               float* sketch, int accumulate, void* stream);

/*
 * K1 batched — the CountSketch of each of n_vec vectors of numel f32 values
 * (w[v * numel + i], table element i), into sketches[v * k + h]; one launch
 * for GradientProjector.project_batch (OPUS/train/random_projection.py:
 * 101-132), which sketches a [B, d] batch row by row.  n_vec <= 65535.
 */
OPUS_API int opus_sketch_dense_rows(const float* w, int n_vec, int64_t numel, const uint32_t* packed, int64_t k,
                                    int max_bucket_load, float* sketches, int accumulate, void* stream);

/*
 * K2 — de-sketched target for the ghost contraction:
 * v[o,c] = scale * D(o,c) * s(o,c) * tau[h(o,c)] written as a bf16 pair
 * v_bf16 = [2, d_out, d_in] (hi = bf16(v), lo = bf16(v - hi)), D as in
 * opus_build_sketch_table.  With it, <D o G_b, s . tau[h]> over the
 * sketch equals the dense inner product <G_b, v> (CountSketch is linear), the
 * identity behind data_selection.py:509-523.
 */
OPUS_API int opus_desketch(const float* tau, const uint32_t* packed, const float* diag, const float* exp_avg_sq,
                  float eps, int d_out, int d_in, int64_t k, float scale, void* v_bf16, void* stream);

/*
 * K3 (stage 2) — ghost per-sample inner products against a dense target:
 * score[b] (+)= alpha * sum_t dLdZ[b,t,:] . (v a[b,t,:]), i.e. <G_b, v>,
 * without forming G_b.  tcgen05 GEMM U = a v^T per 128-token x 256-output
 * tile with a fused row-dot epilogue against the dLdZ tile; U never reaches
 * HBM.  a, dLdZ: bf16 [n_rows, seq_len, d_in|d_out]; v_bf16: the bf16 pair
 * [2, d_out, d_in] (hi, lo) of the f32 target, both multiplied (two MMAs per
 * K step) so the target keeps ~16 mantissa bits.  accumulate = 0 zeroes
 * score[0:n_rows] first.
 * Replaces the score side of weighted_grad_dotprod / grad_dotprod
 * (OPUS/train/data_selection.py:255-292, 597-619) with the target averaged
 * over the proxy batch.
 */
OPUS_API int opus_ghost_score(const void* a, const void* dLdZ, int dtype, int n_rows, int seq_len, int d_in,
                     int d_out, const void* v_bf16, float alpha, float* score, int accumulate,
                     void* stream);

/* score[b] (+)= alpha * phi[b,:] . tau[:]  (data_selection.py:523, 531-536). */
OPUS_API int opus_sketch_dot(const float* phi, const float* tau, int n_rows, int64_t k, float alpha, float* score,
                    int accumulate, void* stream);

/*
 * The same summed over layers in one launch:
 *   score[b] (+)= sum_l alphas[l] * phi[l][b,:] . tau[l][:]
 * phi[l] is the [n_rows, k] f32 block at phi + l * layer_stride (floats),
 * tau[l] the k floats at tau + l * k, alphas [n_layers] f32 on the device.
 * The scores of a round whose per-layer candidate sketches are kept for the
 * similarity: the per-layer score terms of compute_GradProd_GC_per_iter
 * (OPUS/train/data_selection.py:509-536), summed over its layer loop.
 */
OPUS_API int opus_sketch_dot_layers(const float* phi, int64_t layer_stride, const float* tau, const float* alphas,
                           int n_layers, int n_rows, int64_t k, float* score, int accumulate, void* stream);

/* out[i,j] (+)= alpha * phi_a[i,:] . phi_b[j,:]; out is [rows_a, rows_b]
 * (data_selection.py:523 per_val, 579 + 587-588 similarity). */
OPUS_API int opus_sketch_gram(const float* phi_a, int rows_a, const float* phi_b, int rows_b, int64_t k, float alpha,
                     float* out, int accumulate, void* stream);

/*
 * S1 (stage 5) — Boltzmann sampling of n_select of n candidates with the
 * interaction penalty, on one CTA.  uniforms[i] is the double the reference's
 * i-th np.random.choice call draws (np.random.random_sample()).  Same float32
 * arithmetic as stochastic_greedy_selection (data_selection.py:641-675):
 * scaled = score/T, max-shift only above 700, float32 exp, numpy pairwise
 * float32 sum, uniform fallback for a zero/non-finite sum, float64 cumsum and
 * searchsorted(side='right').  n <= 8192; n_select <= n.  out_idx: int64.
 */
OPUS_API int opus_boltzmann_select(const float* scores, const float* sim, int n, int n_select, double temperature,
                          const double* uniforms, int64_t* out_idx, void* stream);

/* S2 — greedy_selection (data_selection.py:622-638): argmax (first max; NaN
 * wins as in np.argmax), scores -= sim[idx], scores[idx] = -inf. */
OPUS_API int opus_greedy_select(const float* scores, const float* sim, int n, int n_select, int64_t* out_idx,
                       void* stream);

/*
 * Global selection over candidates sharded across ranks (the choreography of
 * the reference's global mode, train.py:1100-1178, with the candidates scored
 * where they live): the same samplers with a block-diagonal interaction
 * matrix, sim_blocks [n/block, block, block] holding each rank's local
 * similarity; entries outside the blocks are zero, so a pick penalises only
 * its own block (x - 0 == x exactly).  Results equal opus_boltzmann_select /
 * opus_greedy_select on the dense block-diagonal matrix.  block must divide n.
 */
OPUS_API int opus_boltzmann_select_blocks(const float* scores, const float* sim_blocks, int n, int block,
                                          int n_select, double temperature, const double* uniforms,
                                          int64_t* out_idx, void* stream);
OPUS_API int opus_greedy_select_blocks(const float* scores, const float* sim_blocks, int n, int block, int n_select,
                                       int64_t* out_idx, void* stream);

/* f32 -> bf16 pair: hi = bf16_rn(x), lo = bf16_rn(x - hi), n elements.
 * Used to feed f32 activations/gradients to the bf16 tensor-core kernels. */
OPUS_API int opus_split_bf16(const float* x, int64_t n, void* hi, void* lo, void* stream);

/*
 * K2 Muon — dense bf16 GEMM on tcgen05: C[m,n] (+)= alpha * sum_k
 * (A[m,k] + A_lo[m,k]) * B[n,k], A [M, K] and B [N, K] bf16 row-major (K
 * contiguous), A_lo the lo half of an f32 A split with opus_split_bf16 or
 * NULL.  c_dtype OPUS_DTYPE_BF16 rounds each f32 sum to bf16 (torch's
 * .to(bfloat16)); OPUS_DTYPE_F32 writes f32 (accumulate adds into C).
 * K and N multiples of 8; pointers 16-byte aligned.  With B = S^T this is the
 * candidate transform einsum('...o,po->...p', dLdZ.float(), S.float().T)
 * (OPUS/train/data_selection.py:495-500, :559-563;
 * OPUS/train/random_projection.py:158).
 */
OPUS_API int opus_gemm_bf16(const void* a, const void* a_lo, const void* b, int M, int N, int K, float alpha,
                            void* c, int c_dtype, int accumulate, void* stream);

/*
 * K2 Muon — the preconditioner S = a I + b A + c A^2 with A = m~ m~^T,
 * m~ = m / ||m||_F, a, b, c = 3.4445, -4.7750, 2.0315, for one momentum
 * buffer m [d_out, d_in] (f32 or bf16; f32 is rounded to bf16 first), written
 * as bf16 [d_out, d_out].  Every step rounds to bf16 where torch's bf16
 * arithmetic does; the identity when ||m|| < 1e-7.  workspace: device memory
 * of opus_muon_S_workspace_bytes(d_out, d_in) bytes, 256-byte aligned.
 * d_out, d_in multiples of 8.  Replaces _get_muon_S_matrix
 * (OPUS/train/data_selection.py:228-252).
 */
OPUS_API int64_t opus_muon_S_workspace_bytes(int d_out, int d_in);
OPUS_API int opus_muon_S(const void* m, int m_dtype, int d_out, int d_in, void* workspace, int64_t workspace_bytes,
                         void* S, void* stream);

/* Number of kernels this library has launched in the process so far (all
 * devices).  Instrumentation with no counterpart in the reference: the
 * difference over a region counts the library's launches in it. */
OPUS_API int64_t opus_kernel_launches(void);

#ifdef __cplusplus
}
#endif

#endif /* OPUS_B200_H_ */
