// Ghost per-sample inner products against a dense target (stage 2), sm_100a.
//
// score[b] += alpha * sum_t dLdZ[b,t,:] . (v a[b,t,:]) = alpha * <G_b, v>,
// evaluated without forming G_b: a tcgen05 GEMM U = a v^T over a 128-token x
// 256-output tile (K = d_in, both operands K-major, 128-byte swizzle), with
// v supplied as a bf16 pair (hi, lo) so that hi + lo carries ~16 mantissa
// bits; the two MMAs per K step accumulate into the same TMEM accumulator.
// The epilogue reads U from TMEM, multiplies it by the matching dLdZ tile
// (TMA-staged in shared memory), reduces over the 256 outputs per token and
// over the tokens of a candidate, and adds the result into score[b].  U never
// reaches HBM.
//
// Warp roles as in the sketch GEMM: warp 0 TMA, warp 1 TMEM + UMMA issue,
// warps 2..5 epilogue; two 256-column accumulators double-buffer the
// epilogue against the next tile's MMAs.  Units (token block, output block)
// are numbered token-block-major and split into contiguous ranges per CTA.
#include "opus_common.cuh"

namespace opus {
namespace {

constexpr int kThreads = 192;
constexpr int kEpi = 128;
constexpr int kTM = 128;              // tokens per tile (UMMA M)
constexpr int kTN = 256;              // outputs per tile (UMMA N)
constexpr int kBK = 64;               // d_in per stage (one 128-B swizzle row)
constexpr int kKSteps = kBK / 16;
constexpr int kATile = kTM * kBK * 2;            // 16 KB
constexpr int kVTile = kTN * kBK * 2;            // 32 KB (hi or lo)
constexpr int kStage = kATile + 2 * kVTile;      // 80 KB
constexpr int kStages = 2;
constexpr int kGBox = kTM * 64 * 2;              // 16 KB: 128 tokens x 64 outputs
constexpr int kGTile = 4 * kGBox;                // 64 KB
constexpr uint32_t kSBO = 1024;                  // 8 rows x 128 B
constexpr uint32_t kIdesc = make_idesc(1, 0, 0, kTM, kTN);
constexpr size_t kSmemBytes = 1024 + (size_t)kStages * kStage + kGTile + 256;

__global__ void __launch_bounds__(kThreads, 1)
    ghost_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_v,
                 const __grid_constant__ CUtensorMap tm_g, int64_t n_tok, int seq_len, int d_in, int n_nb,
                 float alpha, float* __restrict__ score, int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* stage_mem = smem;
  uint8_t* g_tile = smem + (size_t)kStages * kStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(g_tile + kGTile);
  uint64_t* full = bars;
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* gfull = tempty + 2;
  uint64_t* gempty = gfull + 1;
  uint64_t* drain = gempty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n_mb = (n_tok + kTM - 1) / kTM;
  const int64_t units = n_mb * n_nb;
  const int64_t u_begin = units * blockIdx.x / gridDim.x;
  const int64_t u_end = units * (blockIdx.x + 1) / gridDim.x;
  const int n_kb = (d_in + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kEpi);
    }
    mbar_init(gfull, 1);
    mbar_init(gempty, kEpi);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_a);
    prefetch_tmap(&tm_v);
    prefetch_tmap(&tm_g);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * kTN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0, gph = 0;
      bool ok = true;
      for (int64_t u = u_begin; u < u_end && ok; ++u) {
        const int mb = static_cast<int>(u / n_nb), nb = static_cast<int>(u % n_nb);
        for (int kb = 0; kb < n_kb; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, err, kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], kStage);
          uint8_t* sa = stage_mem + (size_t)s * kStage;
          tma_load_2d(sa, &tm_a, &full[s], kb * kBK, mb * kTM);
          tma_load_3d(sa + kATile, &tm_v, &full[s], kb * kBK, nb * kTN, 0);
          tma_load_3d(sa + kATile + kVTile, &tm_v, &full[s], kb * kBK, nb * kTN, 1);
          if (++s == kStages) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        // dLdZ tile of this unit, once the previous unit's epilogue released it
        if (!mbar_wait(gempty, gph ^ 1, abort_flag, err, kDevTimeoutProducer)) break;
        mbar_arrive_expect_tx(gfull, kGTile);
        for (int i = 0; i < 4; ++i) tma_load_2d(g_tile + i * kGBox, &tm_g, gfull, nb * kTN + i * 64, mb * kTM);
        gph ^= 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t aph = 0;
      bool ok = true;
      for (int64_t u = u_begin; u < u_end && ok; ++u) {
        if (!mbar_wait(&tempty[acc], aph ^ 1, abort_flag, err, kDevTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kTN);
        for (int kb = 0; kb < n_kb; ++kb) {
          if (!mbar_wait(&full[s], ph, abort_flag, err, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(stage_mem + (size_t)s * kStage);
          const uint32_t shi = sa + kATile, slo = shi + kVTile;
#pragma unroll
          for (int kk = 0; kk < kKSteps; ++kk) {
            const uint64_t da = make_sdesc_sw128(sa + kk * 32, 16, kSBO);
            const uint64_t dh = make_sdesc_sw128(shi + kk * 32, 16, kSBO);
            const uint64_t dl = make_sdesc_sw128(slo + kk * 32, 16, kSBO);
            umma_bf16(d_tmem, da, dh, kIdesc, (kb | kk) != 0 ? 1u : 0u);
            umma_bf16(d_tmem, da, dl, kIdesc, 1u);
          }
          umma_commit(&empty[s]);
          if (++s == kStages) {
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
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
    int acc = 0;
    uint32_t aph = 0, gph = 0;
    for (int64_t u = u_begin; u < u_end; ++u) {
      const int64_t mb = u / n_nb;
      if (!mbar_wait(&tfull[acc], aph, abort_flag, err, kDevTimeoutEpilogue)) break;
      if (!mbar_wait(gfull, gph, abort_flag, err, kDevTimeoutEpilogue)) break;
      tc_fence_after();
      float dot = 0.0f;
      const uint8_t* grow = g_tile + r * 128;
#pragma unroll 1
      for (int j = 0; j < kTN / 32; ++j) {
        uint32_t v[32];
        tmem_ld32(tmem_base + lane_addr + static_cast<uint32_t>(acc * kTN + j * 32), v);
        tmem_ld_wait();
        const uint8_t* box = grow + (j >> 1) * kGBox;
        const int h = j & 1;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const int chunk = (4 * h + cc) ^ (r & 7);
          const uint4 gq = *reinterpret_cast<const uint4*>(box + chunk * 16);
          const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gq);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 gf = __bfloat1622float2(g2[e]);
            dot = fmaf(__uint_as_float(v[cc * 8 + 2 * e]), gf.x, dot);
            dot = fmaf(__uint_as_float(v[cc * 8 + 2 * e + 1]), gf.y, dot);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      mbar_arrive(gempty);
      if (++acc == 2) {
        acc = 0;
        aph ^= 1;
      }
      gph ^= 1;
      const int64_t tok = mb * kTM + r;
      const int64_t b = tok < n_tok ? tok / seq_len : -1;
      const int64_t b0 = __shfl_sync(0xffffffffu, b, 0);
      const bool uniform = __all_sync(0xffffffffu, b == b0);
      if (uniform) {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
        if (lane == 0 && b0 >= 0) atomicAdd(score + b0, alpha * dot);
      } else if (b >= 0) {
        atomicAdd(score + b, alpha * dot);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, 2 * kTN);
}

}  // namespace
}  // namespace opus

using namespace opus;

extern "C" int opus_ghost_score(const void* a, const void* dLdZ, int dtype, int n_rows, int seq_len, int d_in,
                                int d_out, const void* v_bf16, float alpha, float* score, int accumulate,
                                void* stream) {
  if (dtype != OPUS_DTYPE_BF16)
    return set_error(OPUS_ERR_UNSUPPORTED,
                     "ghost_score: operands must be bf16 (split f32 operands into bf16 hi/lo with opus_split_bf16)");
  if (n_rows < 0 || seq_len < 0 || d_in <= 0 || d_out <= 0)
    return set_error(OPUS_ERR_INVALID, "ghost_score: bad sizes");
  if (!score || !v_bf16 || (n_rows > 0 && seq_len > 0 && (!a || !dLdZ)))
    return set_error(OPUS_ERR_INVALID, "ghost_score: NULL pointer");
  if (d_in % 8 != 0 || d_out % 8 != 0)
    return set_error(OPUS_ERR_UNSUPPORTED, "ghost_score: d_in and d_out must be multiples of 8 (got %d, %d)", d_in,
                     d_out);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (!accumulate && n_rows > 0) OPUS_CUDA_TRY(cudaMemsetAsync(score, 0, (size_t)n_rows * sizeof(float), st));
  if (n_rows == 0 || seq_len == 0) return OPUS_OK;
  const int64_t n_tok = (int64_t)n_rows * seq_len;
  CUtensorMap tm_a, tm_v, tm_g;
  {
    const uint64_t dims[2] = {(uint64_t)d_in, (uint64_t)n_tok};
    const uint64_t strides[1] = {(uint64_t)d_in * 2};
    const uint32_t box[2] = {kBK, kTM};
    int rc = encode_tmap(&tm_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[3] = {(uint64_t)d_in, (uint64_t)d_out, 2};
    const uint64_t strides[2] = {(uint64_t)d_in * 2, (uint64_t)d_in * d_out * 2};
    const uint32_t box[3] = {kBK, kTN, 1};
    int rc = encode_tmap(&tm_v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, v_bf16, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {(uint64_t)d_out, (uint64_t)n_tok};
    const uint64_t strides[1] = {(uint64_t)d_out * 2};
    const uint32_t box[2] = {64, kTM};
    int rc = encode_tmap(&tm_g, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dLdZ, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  if ((size_t)max_smem_optin() < kSmemBytes) return set_error(OPUS_ERR_UNSUPPORTED, "ghost_score: shared memory too small");
  OPUS_CUDA_TRY(cudaFuncSetAttribute(ghost_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
  const int n_nb = (d_out + kTN - 1) / kTN;
  const int64_t units = ((n_tok + kTM - 1) / kTM) * n_nb;
  const int grid = static_cast<int>(units < sm_count() ? units : sm_count());
  ghost_kernel<<<grid, kThreads, kSmemBytes, st>>>(tm_a, tm_v, tm_g, n_tok, seq_len, d_in, n_nb, alpha, score,
                                                  device_error_word());
  ::opus::note_launch();
  OPUS_CUDA_TRY(cudaGetLastError());
  return OPUS_OK;
}
