// Sketch Gram blocks: out[i,j] (+)= alpha * phi_a[i,:] . phi_b[j,:], f32.
//
// Tensor-core path (gram_tc_kernel): 128x128 output tiles, the k range split
// across CTAs (f32 vector reductions combine the splits).  TMA brings f32
// tiles of both operands (128 rows x 32 k, 128-byte swizzle); four converter
// warps split every element in shared memory into hi = x with its low 13
// mantissa bits cleared (exactly a tf32) and lo = x - hi (exact in f32), and
// three kind::tf32 MMAs (hi.hi + hi.lo + lo.hi) accumulate in TMEM: the
// product error is that of lo.lo and of lo's tf32 rounding, about 2^-21 of
// |phi_a| |phi_b|.  The same warps then add the tile into out.  A non-finite
// element keeps lo = 0, so an entry is non-finite exactly where the f32
// product is, though an inf can come out as NaN (hi * lo = inf * 0 when the
// other operand is exactly a tf32).
//
// SIMT path (gram_kernel), for rows whose byte stride is not a multiple of
// 16 (k % 4 != 0) or unaligned operands: 64x64 tiles, 4x4 per thread.
#include "opus_common.cuh"

namespace opus {
namespace {

constexpr int kGT = 64;   // output tile
constexpr int kGK = 32;   // k chunk
constexpr int kGThreads = 256;

__global__ void __launch_bounds__(kGThreads) gram_kernel(const float* __restrict__ A, int ra,
                                                         const float* __restrict__ B, int rb, int64_t k,
                                                         int64_t k_per_split, float alpha, float* __restrict__ out,
                                                         int accumulate, int atomic_out) {
  __shared__ float As[kGK][kGT + 4];
  __shared__ float Bs[kGK][kGT + 4];
  const int i0 = blockIdx.y * kGT, j0 = blockIdx.x * kGT;
  const int64_t kb = blockIdx.z * k_per_split;
  const int64_t ke = min(k, kb + k_per_split);
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4] = {};
  for (int64_t kc = kb; kc < ke; kc += kGK) {
    // load 64 rows x 32 k of each operand, stored k-major in shared memory
    for (int e = threadIdx.x; e < kGT * kGK; e += kGThreads) {
      const int row = e / kGK, kk = e % kGK;
      const int64_t kidx = kc + kk;
      const int ia = i0 + row, jb = j0 + row;
      As[kk][row] = (ia < ra && kidx < ke) ? A[(int64_t)ia * k + kidx] : 0.0f;
      Bs[kk][row] = (jb < rb && kidx < ke) ? B[(int64_t)jb * k + kidx] : 0.0f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < kGK; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w};
      const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) acc[x][y] = fmaf(av[x], bv[y], acc[x][y]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int x = 0; x < 4; ++x) {
    const int i = i0 + ty * 4 + x;
    if (i >= ra) continue;
#pragma unroll
    for (int y = 0; y < 4; ++y) {
      const int j = j0 + tx * 4 + y;
      if (j >= rb) continue;
      float* o = out + (int64_t)i * rb + j;
      const float v = alpha * acc[x][y];
      if (atomic_out) atomicAdd(o, v);
      else *o = accumulate ? *o + v : v;
    }
  }
}


// ---- tensor-core path
constexpr int kTcThreads = 192;  // warp 0 TMA, warp 1 TMEM + MMA, warps 2..5 convert + epilogue
constexpr int kTcConv = 128;
constexpr int kTcM = 128;
constexpr int kTcN = 128;
constexpr int kTcBK = 32;                         // f32 k per stage: one 128-byte swizzle row
constexpr int kTcTile = kTcM * kTcBK * 4;         // 16 KB
constexpr int kTcStage = 4 * kTcTile;             // a, b (f32 -> hi in place), a_lo, b_lo
constexpr int kTcStages = 3;
constexpr uint32_t kTcSBO = 1024;
constexpr uint32_t kTcIdesc = make_idesc(2, 0, 0, kTcM, kTcN);
constexpr size_t kTcSmem = 1024 + (size_t)kTcStages * kTcStage + 256;

__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
  if (isfinite(x)) {
    hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
    lo = x - hi;
  } else {
    hi = x;
    lo = 0.0f;
  }
}

constexpr int64_t kTcMaxKbPerSplit = 64;  // 2048 of k per CTA: accumulation bias below ~4e-5

__global__ void __launch_bounds__(kTcThreads, 1)
    gram_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b, int ra, int rb,
                   int tiles_j, int n_tiles, int kb_per_split, int n_kb, float alpha, float* __restrict__ out,
                   int vec_out, int sym, int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)kTcStages * kTcStage);
  uint64_t* full = bars;
  uint64_t* conv = full + kTcStages;
  uint64_t* empty = conv + kTcStages;
  uint64_t* tfull = empty + kTcStages;
  uint64_t* drain = tfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x % n_tiles, split = blockIdx.x / n_tiles;
  int ti, tj;
  if (sym) {  // upper-triangle tiles ti <= tj of the tiles_j x tiles_j grid, row by row
    int t = tile;
    ti = 0;
    while (t >= tiles_j - ti) {
      t -= tiles_j - ti;
      ++ti;
    }
    tj = ti + t;
  } else {
    ti = tile / tiles_j;
    tj = tile % tiles_j;
  }
  // a diagonal tile of a self-Gram multiplies a block by itself: one operand load and split
  const bool self_tile = sym && ti == tj;
  const int kb0 = split * kb_per_split;
  const int kb1 = min(n_kb, kb0 + kb_per_split);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], kTcConv);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_a);
    prefetch_tmap(&tm_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTcN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, err, kDevTimeoutProducer)) break;
        uint8_t* st = smem + (size_t)s * kTcStage;
        mbar_arrive_expect_tx(&full[s], self_tile ? kTcTile : 2 * kTcTile);
        tma_load_2d(st, &tm_a, &full[s], kb * kTcBK, ti * kTcM);
        if (!self_tile) tma_load_2d(st + kTcTile, &tm_b, &full[s], kb * kTcBK, tj * kTcN);
        if (++s == kTcStages) {
          s = 0;
          ph ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&conv[s], ph, abort_flag, err, kDevTimeoutMma)) break;
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + (size_t)s * kTcStage);
        const uint32_t sal = sa + 2 * kTcTile;
        const uint32_t sb = self_tile ? sa : sa + kTcTile, sbl = self_tile ? sal : sa + 3 * kTcTile;
#pragma unroll
        for (int kk = 0; kk < kTcBK / 8; ++kk) {
          const uint64_t dah = make_sdesc_sw128(sa + kk * 32, 16, kTcSBO);
          const uint64_t dbh = make_sdesc_sw128(sb + kk * 32, 16, kTcSBO);
          const uint64_t dal = make_sdesc_sw128(sal + kk * 32, 16, kTcSBO);
          const uint64_t dbl = make_sdesc_sw128(sbl + kk * 32, 16, kTcSBO);
          umma_tf32(tmem_base, dah, dbh, kTcIdesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          umma_tf32(tmem_base, dah, dbl, kTcIdesc, 1u);
          umma_tf32(tmem_base, dal, dbh, kTcIdesc, 1u);
        }
        umma_commit(&empty[s]);
        if (++s == kTcStages) {
          s = 0;
          ph ^= 1;
        }
      }
      umma_commit(tfull);
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, err, kDevTimeoutDrain);
    }
  } else {
    // converters: each of the 128 threads splits 32 float4 of a stage (a and b)
    const int ct = threadIdx.x - 64;
    int s = 0;
    uint32_t ph = 0;
    bool ok = true;
    for (int kb = kb0; kb < kb1; ++kb) {
      if (!mbar_wait(&full[s], ph, abort_flag, err, kDevTimeoutEpilogue)) {
        ok = false;
        break;
      }
      float4* src = reinterpret_cast<float4*>(smem + (size_t)s * kTcStage);
      float4* dst = reinterpret_cast<float4*>(smem + (size_t)s * kTcStage + 2 * kTcTile);
#pragma unroll 4
      for (int e = ct; e < (self_tile ? kTcTile : 2 * kTcTile) / 16; e += kTcConv) {
        const float4 x = src[e];
        float4 h, l;
        split_tf32(x.x, h.x, l.x);
        split_tf32(x.y, h.y, l.y);
        split_tf32(x.z, h.z, l.z);
        split_tf32(x.w, h.w, l.w);
        src[e] = h;
        dst[e] = l;
      }
      fence_proxy_async_smem();
      mbar_arrive(&conv[s]);
      if (++s == kTcStages) {
        s = 0;
        ph ^= 1;
      }
    }
    // epilogue: TMEM lane quarter (warp & 3) holds rows 32q .. 32q+31
    if (ok && kb1 > kb0 && mbar_wait(tfull, 0, abort_flag, err, kDevTimeoutEpilogue)) {
      tc_fence_after();
      const int q = warp & 3;
      const int i = ti * kTcM + q * 32 + lane;
      const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
#pragma unroll 1
      for (int c = 0; c < kTcN / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem_base + lane_addr + static_cast<uint32_t>(c * 32), v);
        tmem_ld_wait();
        if (i >= ra) continue;
        const int j0 = tj * kTcN + c * 32;
        float* o = out + (int64_t)i * rb + j0;
        if (vec_out && j0 + 32 <= rb) {
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            red_add_v4(o + e, alpha * __uint_as_float(v[e]), alpha * __uint_as_float(v[e + 1]),
                       alpha * __uint_as_float(v[e + 2]), alpha * __uint_as_float(v[e + 3]));
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (j0 + e < rb) atomicAdd(o + e, alpha * __uint_as_float(v[e]));
        }
        if (sym && ti < tj) {
          // the mirrored block: element (i, j) also goes to (j, i); lane i writes column i, so
          // each warp reduction covers 32 consecutive floats of row j
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (j0 + e < rb) atomicAdd(out + (int64_t)(j0 + e) * rb + i, alpha * __uint_as_float(v[e]));
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTcN);
}

int launch_gram_tc(const float* phi_a, int rows_a, const float* phi_b, int rows_b, int64_t k, float alpha, float* out,
                   cudaStream_t st) {
  // phi_a phi_a^T with a long k: only the tiles on and above the diagonal are computed (the
  // operand loads they save outweigh the mirrored block's reductions from k = 65536 up)
  const int sym = (phi_a == phi_b && rows_a == rows_b && k >= 65536) ? 1 : 0;
  CUtensorMap tm_a, tm_b;
  {
    const uint64_t dims[2] = {(uint64_t)k, (uint64_t)rows_a};
    const uint64_t strides[1] = {(uint64_t)k * 4};
    const uint32_t box[2] = {kTcBK, kTcM};
    int rc = encode_tmap(&tm_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, phi_a, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {(uint64_t)k, (uint64_t)rows_b};
    const uint64_t strides[1] = {(uint64_t)k * 4};
    const uint32_t box[2] = {kTcBK, kTcN};
    int rc = encode_tmap(&tm_b, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, phi_b, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  if ((size_t)max_smem_optin() < kTcSmem) return set_error(OPUS_ERR_UNSUPPORTED, "sketch_gram: shared memory too small");
  OPUS_CUDA_TRY(cudaFuncSetAttribute(gram_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem));
  const int tiles_i = (rows_a + kTcM - 1) / kTcM, tiles_j = (rows_b + kTcN - 1) / kTcN;
  const int64_t n_tiles64 = sym ? (int64_t)tiles_i * (tiles_i + 1) / 2 : (int64_t)tiles_i * tiles_j;
  if (n_tiles64 > 0x7fffffff) return set_error(OPUS_ERR_UNSUPPORTED, "sketch_gram: too many tiles");
  const int n_tiles = static_cast<int>(n_tiles64);
  const int n_kb = static_cast<int>((k + kTcBK - 1) / kTcBK);
  // About one CTA per SM, at least 4 k-blocks (128 k) per CTA, and at most kTcMaxKbPerSplit
  // k-blocks: the tensor cores' f32 accumulation errs by about 6e-7 of the running sum per
  // 32-wide k-block, one way, so an all-positive sum (a self-similarity) accumulated over n
  // k-blocks in TMEM is off by about 6e-7 n; the splits are added with rounded f32 atomics.
  int64_t splits = (sm_count() + n_tiles - 1) / n_tiles;
  if (splits > (n_kb + 3) / 4) splits = (n_kb + 3) / 4;
  const int64_t min_splits = (n_kb + kTcMaxKbPerSplit - 1) / kTcMaxKbPerSplit;
  if (splits < min_splits) splits = min_splits;
  if (splits < 1) splits = 1;
  const int kb_per_split = static_cast<int>((n_kb + splits - 1) / splits);
  splits = (n_kb + kb_per_split - 1) / kb_per_split;
  const int64_t grid = splits * n_tiles;
  if (grid > 0x7fffffff) return set_error(OPUS_ERR_UNSUPPORTED, "sketch_gram: grid too large");
  const int vec_out = (rows_b % 4 == 0) && ((reinterpret_cast<uintptr_t>(out) & 15) == 0);
  gram_tc_kernel<<<(int)grid, kTcThreads, kTcSmem, st>>>(tm_a, tm_b, rows_a, rows_b, tiles_j, n_tiles, kb_per_split,
                                                        n_kb, alpha, out, vec_out, sym, device_error_word());
  ::opus::note_launch();
  OPUS_CUDA_TRY(cudaGetLastError());
  return OPUS_OK;
}

}  // namespace
}  // namespace opus

using namespace opus;

extern "C" int opus_sketch_gram(const float* phi_a, int rows_a, const float* phi_b, int rows_b, int64_t k, float alpha,
                                float* out, int accumulate, void* stream) {
  if (rows_a < 0 || rows_b < 0 || k <= 0) return set_error(OPUS_ERR_INVALID, "sketch_gram: bad sizes");
  if (rows_a == 0 || rows_b == 0) return OPUS_OK;
  if (!phi_a || !phi_b || !out) return set_error(OPUS_ERR_INVALID, "sketch_gram: NULL pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool tc_ok = (k % 4 == 0) && ((reinterpret_cast<uintptr_t>(phi_a) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(phi_b) & 15) == 0);
  if (tc_ok) {
    if (!accumulate) OPUS_CUDA_TRY(cudaMemsetAsync(out, 0, (size_t)rows_a * rows_b * sizeof(float), st));
    return launch_gram_tc(phi_a, rows_a, phi_b, rows_b, k, alpha, out, st);
  }
  const int ti = (rows_a + kGT - 1) / kGT, tj = (rows_b + kGT - 1) / kGT;
  const int64_t tiles = (int64_t)ti * tj;
  int64_t splits = (2 * (int64_t)sm_count() + tiles - 1) / tiles;
  const int64_t max_splits = (k + 255) / 256;
  if (splits > max_splits) splits = max_splits;
  if (splits > 65535) splits = 65535;
  if (splits < 1) splits = 1;
  int64_t kps = (k + splits - 1) / splits;
  kps = (kps + kGK - 1) / kGK * kGK;
  splits = (k + kps - 1) / kps;
  const int atomic_out = splits > 1 ? 1 : 0;
  if (atomic_out && !accumulate) OPUS_CUDA_TRY(cudaMemsetAsync(out, 0, (size_t)rows_a * rows_b * sizeof(float), st));
  dim3 grid(tj, ti, (unsigned)splits);
  gram_kernel<<<grid, kGThreads, 0, st>>>(phi_a, rows_a, phi_b, rows_b, k, kps, alpha, out, accumulate, atomic_out);
  ::opus::note_launch();
  OPUS_CUDA_TRY(cudaGetLastError());
  return OPUS_OK;
}
