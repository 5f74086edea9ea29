// Dense bf16 GEMMs of the Muon preconditioner (stage 4), sm_100a.
//
//   C[m, n] = epilogue( sum_k (A[m,k] (+ A_lo[m,k])) * B[n,k] )
//
// A [M, K] and B [N, K] are bf16 and K-major (row-major with K contiguous);
// A_lo is the optional lo half of an f32 A split with opus_split_bf16.  The
// three uses on the selection path (OPUS/train/data_selection.py:228-252,
// :495-500, :559-563; OPUS/train/random_projection.py:158):
//
//   A = m~ m~^T                       bf16 output (torch's bf16 matmul rounding)
//   S = a I + b A + c (A A^T)         the same GEMM with an elementwise epilogue
//                                     that rounds to bf16 where torch does
//   dLdZ <- dLdZ S^T                  the candidate transform: bf16 output for
//                                     bf16 dLdZ, f32 for a split f32 dLdZ
//
// bf16 x bf16 products are exact in the f32 accumulator, so each output
// differs from torch's (f32 or cuBLAS bf16) GEMM only by the order of the f32
// additions before the final rounding.
//
// Tiles: a CTA computes 256 rows x 256 columns as two tcgen05 M=128 halves
// that share every B stage, so one 64-deep K stage moves 64 KB (A 2 x 16 KB,
// B 32 KB; with A_lo 96 KB) for 2*256*256*64 flop.  The two 256-column f32
// accumulators fill the 512 TMEM columns.  Tiles are dealt round-robin in
// row-block-major order, so the CTAs working at one time share their A rows
// and sweep B through L2.
//
// Warp roles (320 threads, one CTA per SM): warp 0 TMA producer; warp 1 TMEM
// allocation and single-thread MMA issue; warps 2..9 epilogue, two warps per
// TMEM lane quarter (one per M half).  Every mbarrier wait is bounded.
#include "opus_common.cuh"

namespace opus {
namespace {

constexpr int kGmThreads = 320;
constexpr int kGmEpiThreads = 256;
constexpr int kHalfM = 128;                       // UMMA M
constexpr int kGmTileM = 2 * kHalfM;              // rows per CTA tile
constexpr int kGmTileN = 256;                     // UMMA N
constexpr int kGmBK = 64;                         // K per stage: one 128-byte swizzle row of bf16
constexpr int kGmKSteps = kGmBK / 16;
constexpr int kAHalfBytes = kHalfM * kGmBK * 2;   // 16 KB
constexpr int kBTileBytes = kGmTileN * kGmBK * 2; // 32 KB
constexpr int kRingBytes = 192 * 1024;
constexpr int kMaxStages = 4;
constexpr uint32_t kGmSBO = 1024;                 // 8 rows x 128 B
constexpr uint32_t kGmIdesc = make_idesc(/*bf16*/ 1, /*A K-major*/ 0, /*B K-major*/ 0, kHalfM, kGmTileN);

enum : int { kEpiF32 = 0, kEpiBF16 = 1, kEpiMuonS = 2 };

struct GemmParams {
  int M, N, K;
  int n_nb;           // column tiles
  int stages, stage_bytes, split, epi, accumulate;
  int64_t units;      // row tiles x column tiles
  float alpha;
  void* out;          // [M, N] row-major, f32 or bf16
  const __nv_bfloat16* aux;  // Muon S: the A matrix [M, N]
  const float* norm;         // Muon S: ||m|| as rounded to bf16
  float ca, cb, cc, norm_min;
};

__device__ __forceinline__ float bf_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// One element of S = a*I + b*A + c*(A@A) with torch's bf16 rounding points:
// each product and sum is computed in f32 and rounded to bf16, A@A is the
// bf16-rounded GEMM output.
__device__ __forceinline__ float muon_s_elem(const GemmParams& p, float acc, float a_in, bool diag) {
  const float a2 = bf_round(acc);
  const float t1 = diag ? bf_round(p.ca) : 0.0f;
  const float t2 = bf_round(__fmul_rn(p.cb, a_in));
  const float s12 = bf_round(__fadd_rn(t1, t2));
  const float t3 = bf_round(__fmul_rn(p.cc, a2));
  return __fadd_rn(s12, t3);  // rounded to bf16 by the caller's pack
}

__global__ void __launch_bounds__(kGmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_alo,
                const __grid_constant__ CUtensorMap tm_b, const GemmParams p, int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)p.stages * p.stage_bytes);
  uint64_t* empty = full + kMaxStages;
  uint64_t* tfull = empty + kMaxStages;
  uint64_t* tempty = tfull + 1;
  uint64_t* drain = tempty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_kb = (p.K + kGmBK - 1) / kGmBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, kGmEpiThreads);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_a);
    if (p.split) prefetch_tmap(&tm_alo);
    prefetch_tmap(&tm_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * kGmTileN);
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
      bool ok = true;
      for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
        const int mb = static_cast<int>(u / p.n_nb), nb = static_cast<int>(u % p.n_nb);
        for (int kb = 0; kb < n_kb; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, err, kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], p.stage_bytes);
          uint8_t* st = ring + (size_t)s * p.stage_bytes;
          tma_load_2d(st, &tm_a, &full[s], kb * kGmBK, mb * kGmTileM);
          tma_load_2d(st + kAHalfBytes, &tm_a, &full[s], kb * kGmBK, mb * kGmTileM + kHalfM);
          uint8_t* sb = st + 2 * kAHalfBytes;
          if (p.split) {
            tma_load_2d(sb, &tm_alo, &full[s], kb * kGmBK, mb * kGmTileM);
            tma_load_2d(sb + kAHalfBytes, &tm_alo, &full[s], kb * kGmBK, mb * kGmTileM + kHalfM);
            sb += 2 * kAHalfBytes;
          }
          tma_load_2d(sb, &tm_b, &full[s], kb * kGmBK, nb * kGmTileN);
          if (++s == p.stages) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0, aph = 0;
      bool ok = true;
      const uint32_t d0 = tmem_base, d1 = tmem_base + kGmTileN;
      for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
        if (!mbar_wait(tempty, aph ^ 1, abort_flag, err, kDevTimeoutMma)) break;
        tc_fence_after();
        for (int kb = 0; kb < n_kb; ++kb) {
          if (!mbar_wait(&full[s], ph, abort_flag, err, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(ring + (size_t)s * p.stage_bytes);
          const uint32_t sb = sa + (p.split ? 4 : 2) * kAHalfBytes;
#pragma unroll
          for (int kk = 0; kk < kGmKSteps; ++kk) {
            const uint64_t db = make_sdesc_sw128(sb + kk * 32, 16, kGmSBO);
            const uint32_t acc = (kb | kk) != 0 ? 1u : 0u;
            umma_bf16(d0, make_sdesc_sw128(sa + kk * 32, 16, kGmSBO), db, kGmIdesc, acc);
            umma_bf16(d1, make_sdesc_sw128(sa + kAHalfBytes + kk * 32, 16, kGmSBO), db, kGmIdesc, acc);
            if (p.split) {
              umma_bf16(d0, make_sdesc_sw128(sa + 2 * kAHalfBytes + kk * 32, 16, kGmSBO), db, kGmIdesc, 1u);
              umma_bf16(d1, make_sdesc_sw128(sa + 3 * kAHalfBytes + kk * 32, 16, kGmSBO), db, kGmIdesc, 1u);
            }
          }
          umma_commit(&empty[s]);
          if (++s == p.stages) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(tfull);
        aph ^= 1;
      }
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, err, kDevTimeoutDrain);
    }
  } else {
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = half * kHalfM + q * 32 + lane;  // row inside the tile
    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(half * kGmTileN);
    const bool identity = p.epi == kEpiMuonS && *p.norm < p.norm_min;
    uint32_t aph = 0;
    for (int64_t u = blockIdx.x; u < p.units; u += gridDim.x) {
      const int mb = static_cast<int>(u / p.n_nb), nb = static_cast<int>(u % p.n_nb);
      if (!mbar_wait(tfull, aph, abort_flag, err, kDevTimeoutEpilogue)) break;
      tc_fence_after();
      const int64_t m = (int64_t)mb * kGmTileM + r;
      const bool row_ok = m < p.M;
#pragma unroll 1
      for (int j = 0; j < kGmTileN / 32; ++j) {
        uint32_t v[32];
        tmem_ld32(taddr + static_cast<uint32_t>(j * 32), v);
        tmem_ld_wait();
        const int n0 = nb * kGmTileN + j * 32;
        if (!row_ok || n0 >= p.N) continue;
        const int cols = p.N - n0 < 32 ? p.N - n0 : 32;  // a multiple of 8
        if (p.epi == kEpiF32) {
          float* o = static_cast<float*>(p.out) + m * p.N + n0;
#pragma unroll
          for (int c = 0; c < 32; c += 4) {
            if (c < cols) {
              float4 x = make_float4(p.alpha * __uint_as_float(v[c]), p.alpha * __uint_as_float(v[c + 1]),
                                     p.alpha * __uint_as_float(v[c + 2]), p.alpha * __uint_as_float(v[c + 3]));
              if (p.accumulate) {
                const float4 y = *reinterpret_cast<const float4*>(o + c);
                x.x += y.x;
                x.y += y.y;
                x.z += y.z;
                x.w += y.w;
              }
              *reinterpret_cast<float4*>(o + c) = x;
            }
          }
        } else {
          __nv_bfloat16* o = static_cast<__nv_bfloat16*>(p.out) + m * p.N + n0;
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            if (c < cols) {
              uint4 pk;
              uint32_t* w = reinterpret_cast<uint32_t*>(&pk);
              if (p.epi == kEpiBF16) {
#pragma unroll
                for (int e = 0; e < 4; ++e)
                  w[e] = pack_bf2(p.alpha * __uint_as_float(v[c + 2 * e]), p.alpha * __uint_as_float(v[c + 2 * e + 1]));
              } else {
                const uint4 ain = *reinterpret_cast<const uint4*>(p.aux + m * p.N + n0 + c);
                const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&ain);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const int64_t col = n0 + c + 2 * e;
                  const float2 af = __bfloat1622float2(a2[e]);
                  float s0, s1;
                  if (identity) {
                    s0 = col == m ? 1.0f : 0.0f;
                    s1 = col + 1 == m ? 1.0f : 0.0f;
                  } else {
                    s0 = muon_s_elem(p, __uint_as_float(v[c + 2 * e]), af.x, col == m);
                    s1 = muon_s_elem(p, __uint_as_float(v[c + 2 * e + 1]), af.y, col + 1 == m);
                  }
                  w[e] = pack_bf2(s0, s1);
                }
              }
              *reinterpret_cast<uint4*>(o + c) = pk;
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(tempty);
      aph ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, 2 * kGmTileN);
}

// ---------------------------------------------------------------- ||m|| and m / ||m||
constexpr int kNormThreads = 256;
constexpr int kNormMaxBlocks = 512;

__device__ __forceinline__ float load_as_bf16(const void* m, int m_f32, int64_t i) {
  return m_f32 ? bf_round(static_cast<const float*>(m)[i]) : __bfloat162float(static_cast<const __nv_bfloat16*>(m)[i]);
}

// partial[block] = sum of squares (in double) of this block's share of bf16(m).
__global__ void __launch_bounds__(kNormThreads) sumsq_kernel(const void* m, int m_f32, int64_t n, double* partial) {
  __shared__ double red[kNormThreads / 32];
  double s = 0.0;
  for (int64_t i = (int64_t)blockIdx.x * kNormThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kNormThreads) {
    const double x = load_as_bf16(m, m_f32, i);
    s = fma(x, x, s);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < kNormThreads / 32; ++w) t += red[w];
    partial[blockIdx.x] = t;
  }
}

// norm = bf16(sqrt(sum)), as torch.norm returns for a bf16 tensor, and
// mt = bf16(m / norm) with the division in f32 (torch's bf16 division).
// Every block adds the partial sums in the same order, so all see one norm.
__global__ void __launch_bounds__(kNormThreads)
    normalize_kernel(const void* m, int m_f32, int64_t n, const double* partial, int n_parts, float* norm_out,
                     __nv_bfloat16* mt) {
  __shared__ float s_norm;
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int i = 0; i < n_parts; ++i) t += partial[i];
    s_norm = bf_round(static_cast<float>(sqrt(t)));
    if (blockIdx.x == 0) *norm_out = s_norm;
  }
  __syncthreads();
  const float nrm = s_norm;
  for (int64_t i = (int64_t)blockIdx.x * kNormThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kNormThreads)
    mt[i] = __float2bfloat16_rn(__fdiv_rn(load_as_bf16(m, m_f32, i), nrm));
}

int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }

int launch_gemm(const void* a, const void* a_lo, const void* b, int M, int N, int K, GemmParams p,
                cudaStream_t st) {
  if (M < 0 || N <= 0 || K <= 0) return set_error(OPUS_ERR_INVALID, "gemm_bf16: bad sizes M=%d N=%d K=%d", M, N, K);
  if (K % 8 != 0 || N % 8 != 0)
    return set_error(OPUS_ERR_UNSUPPORTED, "gemm_bf16: K and N must be multiples of 8 (got K=%d, N=%d)", K, N);
  if (M == 0) return OPUS_OK;
  CUtensorMap tm_a, tm_alo, tm_b;
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)K * 2};
    const uint32_t box[2] = {kGmBK, kHalfM};
    int rc = encode_tmap(&tm_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    tm_alo = tm_a;
    if (a_lo != nullptr) {
      rc = encode_tmap(&tm_alo, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a_lo, dims, strides, box,
                       CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc) return rc;
    }
  }
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)N};
    const uint64_t strides[1] = {(uint64_t)K * 2};
    const uint32_t box[2] = {kGmBK, kGmTileN};
    int rc = encode_tmap(&tm_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  p.M = M;
  p.N = N;
  p.K = K;
  p.split = a_lo != nullptr;
  p.stage_bytes = (p.split ? 4 : 2) * kAHalfBytes + kBTileBytes;
  p.stages = kRingBytes / p.stage_bytes;
  if (p.stages > kMaxStages) p.stages = kMaxStages;
  p.n_nb = (N + kGmTileN - 1) / kGmTileN;
  p.units = (int64_t)((M + kGmTileM - 1) / kGmTileM) * p.n_nb;
  const size_t smem = 1024 + (size_t)p.stages * p.stage_bytes + 256;
  if ((size_t)max_smem_optin() < smem) return set_error(OPUS_ERR_UNSUPPORTED, "gemm_bf16: shared memory too small");
  OPUS_CUDA_TRY(cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int grid = static_cast<int>(p.units < sm_count() ? p.units : sm_count());
  gemm_kernel<<<grid, kGmThreads, smem, st>>>(tm_a, tm_alo, tm_b, p, device_error_word());
  note_launch();
  OPUS_CUDA_TRY(cudaGetLastError());
  return OPUS_OK;
}

GemmParams base_params() {
  GemmParams p{};
  p.alpha = 1.0f;
  return p;
}

}  // namespace
}  // namespace opus

using namespace opus;

extern "C" int opus_gemm_bf16(const void* a, const void* a_lo, const void* b, int M, int N, int K, float alpha,
                              void* c, int c_dtype, int accumulate, void* stream) {
  if (M == 0) return OPUS_OK;
  if (!c || !a || !b) return set_error(OPUS_ERR_INVALID, "gemm_bf16: NULL pointer");
  if (c_dtype != OPUS_DTYPE_F32 && c_dtype != OPUS_DTYPE_BF16)
    return set_error(OPUS_ERR_INVALID, "gemm_bf16: c_dtype must be OPUS_DTYPE_F32 or OPUS_DTYPE_BF16");
  if (accumulate && c_dtype != OPUS_DTYPE_F32)
    return set_error(OPUS_ERR_UNSUPPORTED, "gemm_bf16: accumulate needs an f32 output");
  if ((reinterpret_cast<uintptr_t>(c) & 15) != 0) return set_error(OPUS_ERR_INVALID, "gemm_bf16: C not 16-byte aligned");
  GemmParams p = base_params();
  p.alpha = alpha;
  p.epi = c_dtype == OPUS_DTYPE_F32 ? kEpiF32 : kEpiBF16;
  p.accumulate = accumulate ? 1 : 0;
  p.out = c;
  return launch_gemm(a, a_lo, b, M, N, K, p, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int64_t opus_muon_S_workspace_bytes(int d_out, int d_in) {
  if (d_out <= 0 || d_in <= 0) return 0;
  return 256 + (int64_t)kNormMaxBlocks * 8 + align256((int64_t)d_out * d_in * 2) +
         align256((int64_t)d_out * d_out * 2);
}

extern "C" int opus_muon_S(const void* m, int m_dtype, int d_out, int d_in, void* workspace,
                           int64_t workspace_bytes, void* S, void* stream) {
  if (d_out <= 0 || d_in <= 0) return set_error(OPUS_ERR_INVALID, "muon_S: bad sizes d_out=%d d_in=%d", d_out, d_in);
  if (!m || !workspace || !S) return set_error(OPUS_ERR_INVALID, "muon_S: NULL pointer");
  if (m_dtype != OPUS_DTYPE_F32 && m_dtype != OPUS_DTYPE_BF16)
    return set_error(OPUS_ERR_INVALID, "muon_S: m_dtype must be OPUS_DTYPE_F32 or OPUS_DTYPE_BF16");
  if (d_out % 8 != 0 || d_in % 8 != 0)
    return set_error(OPUS_ERR_UNSUPPORTED, "muon_S: d_out and d_in must be multiples of 8 (got %d, %d)", d_out, d_in);
  if (workspace_bytes < opus_muon_S_workspace_bytes(d_out, d_in))
    return set_error(OPUS_ERR_INVALID, "muon_S: workspace of %lld bytes, need %lld", (long long)workspace_bytes,
                     (long long)opus_muon_S_workspace_bytes(d_out, d_in));
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return set_error(OPUS_ERR_INVALID, "muon_S: workspace must be 256-byte aligned");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* norm = reinterpret_cast<float*>(ws);
  double* partial = reinterpret_cast<double*>(ws + 256);
  __nv_bfloat16* mt = reinterpret_cast<__nv_bfloat16*>(ws + 256 + (int64_t)kNormMaxBlocks * 8);
  __nv_bfloat16* amat = reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<uint8_t*>(mt) +
                                                         align256((int64_t)d_out * d_in * 2));
  const int64_t n = (int64_t)d_out * d_in;
  const int m_f32 = m_dtype == OPUS_DTYPE_F32;
  int64_t want = (n + kNormThreads * 8 - 1) / (kNormThreads * 8);
  const int parts = static_cast<int>(want < 1 ? 1 : (want > kNormMaxBlocks ? kNormMaxBlocks : want));
  sumsq_kernel<<<parts, kNormThreads, 0, st>>>(m, m_f32, n, partial);
  note_launch();
  OPUS_CUDA_TRY(cudaGetLastError());
  int64_t blocks = (n + kNormThreads * 4 - 1) / (kNormThreads * 4);
  if (blocks > 4 * sm_count()) blocks = 4 * sm_count();
  normalize_kernel<<<(int)blocks, kNormThreads, 0, st>>>(m, m_f32, n, partial, parts, norm, mt);
  note_launch();
  OPUS_CUDA_TRY(cudaGetLastError());
  // A = m~ m~^T, rounded to bf16 as torch's bf16 matmul output
  GemmParams pa = base_params();
  pa.epi = kEpiBF16;
  pa.out = amat;
  int rc = launch_gemm(mt, nullptr, mt, d_out, d_out, d_in, pa, st);
  if (rc) return rc;
  // S = a I + b A + c (A A^T); the identity when ||m|| < 1e-7
  GemmParams ps = base_params();
  ps.epi = kEpiMuonS;
  ps.out = S;
  ps.aux = amat;
  ps.norm = norm;
  // the Python floats of the reference, converted to f32 as torch converts a scalar operand
  ps.ca = static_cast<float>(3.4445);
  ps.cb = static_cast<float>(-4.7750);
  ps.cc = static_cast<float>(2.0315);
  ps.norm_min = 1e-7f;
  return launch_gemm(amat, nullptr, amat, d_out, d_out, d_out, ps, st);
}
