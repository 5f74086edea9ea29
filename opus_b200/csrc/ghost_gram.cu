// Ghost Gram of per-sample gradients (projection off), sm_100a.
//
// S[i, j] += alpha * <G_i, G_j> for every candidate pair, G_b = dLdZ_b^T a_b,
// evaluated as sum_{t,s} (a_i a_j^T)[t,s] * (g_i g_j^T)[t,s] without forming
// any G_b.  A unit is a pair i <= j, a 128-token block t of candidate i and
// a 128-token block s of candidate j.  Two tcgen05 GEMMs, both operands
// K-major with 128-byte swizzle, accumulate in TMEM:
//   P = a_i[t] a_j[s]^T  (K = d_in),   Q = g_i[t] g_j[s]^T  (K = d_out);
// the epilogue reads P and Q row by row (row = token of block t), forms the
// row dot products, reduces them over the block and adds the result into
// S[i, j] and S[j, i].  P and Q never leave the SM.
//
// bf16 operands go to the tensor cores as they are; f32 operands arrive as
// bf16 (hi, lo) pairs and each product is hi*hi + hi*lo + lo*hi.
//
// Warp roles as in the other tcgen05 kernels: warp 0 TMA, warp 1 TMEM and
// UMMA issue, warps 2..5 epilogue.  Each unit takes 256 TMEM columns (P and
// Q), and two units' accumulators alternate, so the epilogue of one unit
// overlaps the MMAs of the next.  Units are numbered pair-major and split into
// contiguous ranges per CTA.  Token rows past seq_len and features past
// d_in / d_out come from the tensor maps' zero fill and add nothing.
#include "opus_common.cuh"

namespace opus {
namespace {

constexpr int kGgThreads = 192;
constexpr int kGgEpi = 128;
constexpr int kGgM = 128;                          // tokens per block (UMMA M and N)
constexpr int kGgBK = 64;                          // features per stage (one 128-B swizzle row)
constexpr int kGgKSteps = kGgBK / 16;
constexpr int kGgTile = kGgM * kGgBK * 2;          // 16 KB: 128 tokens x 64 features, bf16
constexpr uint32_t kGgSBO = 1024;                  // 8 rows x 128 B
constexpr uint32_t kGgIdesc = make_idesc(1, 0, 0, kGgM, kGgM);
constexpr int kGgCols = 2 * kGgM;                  // P and Q of one unit

// Unit u -> (i, j, t-block, s-block): pairs i <= j row by row, then t, then s.
__device__ __forceinline__ void gg_unit(int64_t u, int n_tb, int n_rows, int& i, int& j, int& tb, int& sb) {
  const int64_t per_pair = (int64_t)n_tb * n_tb;
  int64_t p = u / per_pair;
  const int64_t r = u % per_pair;
  tb = static_cast<int>(r / n_tb);
  sb = static_cast<int>(r % n_tb);
  i = 0;
  while (p >= n_rows - i) {
    p -= n_rows - i;
    ++i;
  }
  j = i + static_cast<int>(p);
}

// The unit after (i, j, t-block, s-block) in the same order.
__device__ __forceinline__ void gg_next(int n_tb, int n_rows, int& i, int& j, int& tb, int& sb) {
  if (++sb < n_tb) return;
  sb = 0;
  if (++tb < n_tb) return;
  tb = 0;
  if (++j < n_rows) return;
  ++i;
  j = i;
}

__global__ void __launch_bounds__(kGgThreads, 1)
    ghost_gram_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_al,
                      const __grid_constant__ CUtensorMap tm_g, const __grid_constant__ CUtensorMap tm_gl,
                      int split, int n_rows, int n_tb, int n_kb_a, int n_kb_g, int stages, int64_t units,
                      float alpha, float* __restrict__ S, int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  const int tiles = split ? 4 : 2;  // per stage: row hi, column hi (+ row lo, column lo)
  const size_t stage_bytes = (size_t)tiles * kGgTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)stages * stage_bytes);
  uint64_t* full = bars;
  uint64_t* empty = full + stages;
  uint64_t* tfull = empty + stages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t u_begin = units * blockIdx.x / gridDim.x;
  const int64_t u_end = units * (blockIdx.x + 1) / gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kGgEpi);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_a);
    prefetch_tmap(&tm_g);
    if (split) {
      prefetch_tmap(&tm_al);
      prefetch_tmap(&tm_gl);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * kGgCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      int i, j, tb, sb;
      gg_unit(u_begin, n_tb, n_rows, i, j, tb, sb);
      for (int64_t u = u_begin; u < u_end && ok; ++u, gg_next(n_tb, n_rows, i, j, tb, sb)) {
        for (int kb = 0; kb < n_kb_a + n_kb_g; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, err, kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          const bool on_a = kb < n_kb_a;
          const CUtensorMap* hi = on_a ? &tm_a : &tm_g;
          const CUtensorMap* lo = on_a ? &tm_al : &tm_gl;
          const int k0 = (on_a ? kb : kb - n_kb_a) * kGgBK;
          uint8_t* st = smem + (size_t)s * stage_bytes;
          mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(stage_bytes));
          tma_load_3d(st, hi, &full[s], k0, tb * kGgM, i);
          tma_load_3d(st + kGgTile, hi, &full[s], k0, sb * kGgM, j);
          if (split) {
            tma_load_3d(st + 2 * kGgTile, lo, &full[s], k0, tb * kGgM, i);
            tma_load_3d(st + 3 * kGgTile, lo, &full[s], k0, sb * kGgM, j);
          }
          if (++s == stages) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t aph = 0;
      bool ok = true;
      for (int64_t u = u_begin; u < u_end && ok; ++u) {
        if (!mbar_wait(&tempty[acc], aph ^ 1, abort_flag, err, kDevTimeoutMma)) break;
        tc_fence_after();
        for (int kb = 0; kb < n_kb_a + n_kb_g; ++kb) {
          if (!mbar_wait(&full[s], ph, abort_flag, err, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const bool on_a = kb < n_kb_a;
          const int kq = on_a ? kb : kb - n_kb_a;  // the k-block within P or Q
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kGgCols + (on_a ? 0 : kGgM));
          const uint32_t sr = smem_u32(smem + (size_t)s * stage_bytes);
          const uint32_t sc = sr + kGgTile, srl = sr + 2 * kGgTile, scl = sr + 3 * kGgTile;
#pragma unroll
          for (int kk = 0; kk < kGgKSteps; ++kk) {
            const uint64_t dr = make_sdesc_sw128(sr + kk * 32, 16, kGgSBO);
            const uint64_t dc = make_sdesc_sw128(sc + kk * 32, 16, kGgSBO);
            umma_bf16(d_tmem, dr, dc, kGgIdesc, (kq | kk) != 0 ? 1u : 0u);
            if (split) {
              const uint64_t drl = make_sdesc_sw128(srl + kk * 32, 16, kGgSBO);
              const uint64_t dcl = make_sdesc_sw128(scl + kk * 32, 16, kGgSBO);
              umma_bf16(d_tmem, dr, dcl, kGgIdesc, 1u);
              umma_bf16(d_tmem, drl, dc, kGgIdesc, 1u);
            }
          }
          umma_commit(&empty[s]);
          if (++s == stages) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          aph ^= 1;
        }
      }
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, err, kDevTimeoutDrain);
    }
  } else {
    // ---------------------------------------------------------- epilogue
    // thread = row (token of block t); P and Q of the unit side by side in TMEM
    const int q = warp & 3;
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
    int acc = 0;
    uint32_t aph = 0;
    int i, j, tb, sb;
    gg_unit(u_begin, n_tb, n_rows, i, j, tb, sb);
    for (int64_t u = u_begin; u < u_end; ++u, gg_next(n_tb, n_rows, i, j, tb, sb)) {
      if (!mbar_wait(&tfull[acc], aph, abort_flag, err, kDevTimeoutEpilogue)) break;
      tc_fence_after();
      float dot = 0.0f;
#pragma unroll 1
      for (int c = 0; c < kGgM / 32; ++c) {
        uint32_t p[32], qv[32];
        tmem_ld32(tmem_base + lane_addr + static_cast<uint32_t>(acc * kGgCols + c * 32), p);
        tmem_ld32(tmem_base + lane_addr + static_cast<uint32_t>(acc * kGgCols + kGgM + c * 32), qv);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) dot = fmaf(__uint_as_float(p[e]), __uint_as_float(qv[e]), dot);
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        aph ^= 1;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
      if (lane == 0) {
        atomicAdd(S + (int64_t)i * n_rows + j, alpha * dot);
        if (i != j) atomicAdd(S + (int64_t)j * n_rows + i, alpha * dot);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, 2 * kGgCols);
}

// [n_rows, seq_len, width] bf16 as a 3-D map with 64-feature x 128-token boxes.
int gg_map(CUtensorMap* map, const void* x, int n_rows, int seq_len, int width) {
  const uint64_t dims[3] = {(uint64_t)width, (uint64_t)seq_len, (uint64_t)n_rows};
  const uint64_t strides[2] = {(uint64_t)width * 2, (uint64_t)seq_len * width * 2};
  const uint32_t box[3] = {kGgBK, kGgM, 1};
  return encode_tmap(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, x, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace
}  // namespace opus

using namespace opus;

extern "C" int opus_ghost_gram(const void* a, const void* a_lo, const void* dLdZ, const void* dLdZ_lo, int dtype,
                               int n_rows, int seq_len, int d_in, int d_out, float alpha, float* S, int accumulate,
                               void* stream) {
  if (dtype != OPUS_DTYPE_BF16)
    return set_error(OPUS_ERR_UNSUPPORTED,
                     "ghost_gram: operands must be bf16 (split f32 operands into bf16 hi/lo with opus_split_bf16)");
  if (n_rows < 0 || seq_len < 0 || d_in <= 0 || d_out <= 0)
    return set_error(OPUS_ERR_INVALID, "ghost_gram: bad sizes");
  if (d_in % 8 != 0 || d_out % 8 != 0)
    return set_error(OPUS_ERR_UNSUPPORTED, "ghost_gram: d_in and d_out must be multiples of 8 (got %d, %d)", d_in,
                     d_out);
  if ((a_lo == nullptr) != (dLdZ_lo == nullptr))
    return set_error(OPUS_ERR_INVALID, "ghost_gram: give both lo halves or neither");
  if (n_rows == 0) return OPUS_OK;
  if (!S || (seq_len > 0 && (!a || !dLdZ))) return set_error(OPUS_ERR_INVALID, "ghost_gram: NULL pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (!accumulate) OPUS_CUDA_TRY(cudaMemsetAsync(S, 0, (size_t)n_rows * n_rows * sizeof(float), st));
  if (seq_len == 0) return OPUS_OK;
  const int split = a_lo != nullptr ? 1 : 0;
  CUtensorMap tm_a, tm_al, tm_g, tm_gl;
  if (int rc = gg_map(&tm_a, a, n_rows, seq_len, d_in)) return rc;
  if (int rc = gg_map(&tm_g, dLdZ, n_rows, seq_len, d_out)) return rc;
  if (split) {
    if (int rc = gg_map(&tm_al, a_lo, n_rows, seq_len, d_in)) return rc;
    if (int rc = gg_map(&tm_gl, dLdZ_lo, n_rows, seq_len, d_out)) return rc;
  } else {
    tm_al = tm_a;
    tm_gl = tm_g;
  }
  const size_t stage_bytes = (size_t)(split ? 4 : 2) * kGgTile;
  const size_t fixed = 1024 + 8 * (2 * 8 + 5) + 32;
  int stages = 0;
  for (int s = 6; s >= 2; --s)
    if (fixed + (size_t)s * stage_bytes <= (size_t)max_smem_optin()) {
      stages = s;
      break;
    }
  if (stages == 0) return set_error(OPUS_ERR_UNSUPPORTED, "ghost_gram: shared memory too small");
  const size_t smem = fixed + (size_t)stages * stage_bytes;
  OPUS_CUDA_TRY(cudaFuncSetAttribute(ghost_gram_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int n_tb = (seq_len + kGgM - 1) / kGgM;
  const int64_t pairs = (int64_t)n_rows * (n_rows + 1) / 2;
  const int64_t units = pairs * n_tb * n_tb;
  const int n_kb_a = (d_in + kGgBK - 1) / kGgBK, n_kb_g = (d_out + kGgBK - 1) / kGgBK;
  const int64_t grid = units < sm_count() ? units : sm_count();
  ghost_gram_kernel<<<(int)grid, kGgThreads, smem, st>>>(tm_a, tm_al, tm_g, tm_gl, split, n_rows, n_tb, n_kb_a,
                                                          n_kb_g, stages, units, alpha, S, device_error_word());
  ::opus::note_launch();
  OPUS_CUDA_TRY(cudaGetLastError());
  return OPUS_OK;
}
