// Memory-bound kernels of the selection path:
//   opus_sketch_dense  K1: CountSketch of one dense matrix (proxy target)
//   opus_sketch_dot    score[b] (+)= alpha * phi[b] . tau
//   opus_split_bf16    f32 -> bf16 hi + bf16 lo (x ~= hi + lo to 2^-16)
#include "opus_common.cuh"

namespace opus {
namespace {

constexpr int kDenseThreads = 256;
constexpr int kDenseTile = 32;  // 32 x 32 (o, c) tiles

// Grid-stride over 32x32 tiles of rows [row_begin, row_end) of the
// [d_out, d_in] grid (a rank's share of the target in sharded selection).  The weight tile is
// read in its stored orientation (coalesced either way) and staged through
// shared memory; the packed table is read row-major; every element is added
// to its bucket with an f32 reduction in L2 (shared-memory float atomics are
// compare-and-swap loops, and one matrix gives each bucket only ~numel/k
// updates).
__global__ void __launch_bounds__(kDenseThreads) dense_sketch_kernel(const float* __restrict__ w, int transposed,
                                                                     const uint32_t* __restrict__ packed,
                                                                     const float* __restrict__ diag, int d_out,
                                                                     int d_in, int row_begin, int row_end, int64_t k,
                                                                     float* __restrict__ out) {
  __shared__ float tile_w[kDenseTile][kDenseTile + 1];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  const int rows = row_end - row_begin;
  const int n_to = (rows + kDenseTile - 1) / kDenseTile, n_tc = (d_in + kDenseTile - 1) / kDenseTile;
  const int64_t n_tiles = (int64_t)n_to * n_tc;
  for (int64_t t = blockIdx.x; t < n_tiles; t += gridDim.x) {
    const int o0 = row_begin + static_cast<int>(t / n_tc) * kDenseTile, c0 = static_cast<int>(t % n_tc) * kDenseTile;
    if (transposed) {
      for (int rr = ty; rr < kDenseTile; rr += 8) {
        const int c = c0 + rr, o = o0 + tx;
        tile_w[tx][rr] = (o < row_end && c < d_in) ? w[(int64_t)c * d_out + o] : 0.0f;
      }
      __syncthreads();
    }
    for (int rr = ty; rr < kDenseTile; rr += 8) {
      const int o = o0 + rr, c = c0 + tx;
      if (o < row_end && c < d_in) {
        const int64_t idx = (int64_t)o * d_in + c;
        const uint32_t hv = packed[idx];
        float x = transposed ? tile_w[rr][tx] : w[idx];
        if (diag != nullptr) x = x * diag[idx];
        if (hv & 0x80000000u) x = -x;
        const uint32_t bucket = hv & 0x7FFFFFFFu;
        if (bucket < static_cast<uint64_t>(k)) atomicAdd(out + bucket, x);
      }
    }
    if (transposed) __syncthreads();
  }
}

// The same CountSketch with a CTA-private f32 sketch in shared memory: each
// CTA adds its share of the elements into its own copy of the k buckets
// (shared-memory atomics), then adds that copy to the output once, with
// 16-byte vector reductions over consecutive buckets.  Random 4-byte L2
// atomics, one per element, run at about 0.64 per clock per SM; the flush is
// k sequential floats per CTA.  1024 threads: thread (ty, tx) takes element
// (o0 + ty, c0 + tx) of each 32 x 32 tile, eight tiles at a time so that
// eight independent loads of each input are in flight per thread.
constexpr int kDenseSmemThreads = 1024;

constexpr int kDenseGroup = 8;  // tiles whose loads a thread has in flight together

__global__ void __launch_bounds__(kDenseSmemThreads) dense_sketch_smem_kernel(
    const float* __restrict__ w, int transposed, const uint32_t* __restrict__ packed, const float* __restrict__ diag,
    int d_out, int d_in, int row_begin, int row_end, int k, float* __restrict__ out) {
  __shared__ float tile_w[kDenseGroup][kDenseTile][kDenseTile + 1];
  extern __shared__ __align__(16) float sk[];  // k buckets
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 32
  for (int i = threadIdx.x; i < k; i += kDenseSmemThreads) sk[i] = 0.0f;
  __syncthreads();
  const int rows = row_end - row_begin;
  const int n_to = (rows + kDenseTile - 1) / kDenseTile, n_tc = (d_in + kDenseTile - 1) / kDenseTile;
  const int64_t n_tiles = (int64_t)n_to * n_tc;
  for (int64_t t0 = (int64_t)blockIdx.x * kDenseGroup; t0 < n_tiles; t0 += (int64_t)gridDim.x * kDenseGroup) {
    if (transposed) {
#pragma unroll
      for (int g = 0; g < kDenseGroup; ++g) {
        const int64_t t = t0 + g;
        const int o0 = row_begin + static_cast<int>(t / n_tc) * kDenseTile;
        const int c0 = static_cast<int>(t % n_tc) * kDenseTile;
        const int c = c0 + ty, o = o0 + tx;
        tile_w[g][tx][ty] = (t < n_tiles && o < row_end && c < d_in) ? w[(int64_t)c * d_out + o] : 0.0f;
      }
      __syncthreads();
    }
    float x[kDenseGroup], dg[kDenseGroup];
    uint32_t hv[kDenseGroup];
    bool in[kDenseGroup];
#pragma unroll
    for (int g = 0; g < kDenseGroup; ++g) {
      const int64_t t = t0 + g;
      const int o = row_begin + static_cast<int>(t / n_tc) * kDenseTile + ty;
      const int c = static_cast<int>(t % n_tc) * kDenseTile + tx;
      in[g] = t < n_tiles && o < row_end && c < d_in;
      const int64_t idx = (int64_t)o * d_in + c;
      hv[g] = in[g] ? packed[idx] : 0u;
      x[g] = transposed ? tile_w[g][ty][tx] : (in[g] ? w[idx] : 0.0f);
      dg[g] = (in[g] && diag != nullptr) ? diag[idx] : 1.0f;
    }
#pragma unroll
    for (int g = 0; g < kDenseGroup; ++g) {
      if (!in[g]) continue;
      float v = x[g];
      if (diag != nullptr) v = v * dg[g];
      if (hv[g] & 0x80000000u) v = -v;
      const uint32_t bucket = hv[g] & 0x7FFFFFFFu;
      if (bucket < static_cast<uint32_t>(k)) atomicAdd(sk + bucket, v);
    }
    if (transposed) __syncthreads();
  }
  __syncthreads();
  if ((k & 3) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0) {
    const float4* s4 = reinterpret_cast<const float4*>(sk);
    for (int i = threadIdx.x; i < k / 4; i += kDenseSmemThreads) {
      const float4 v = s4[i];
      if (v.x != 0.0f || v.y != 0.0f || v.z != 0.0f || v.w != 0.0f) red_add_v4(out + 4 * i, v.x, v.y, v.z, v.w);
    }
  } else {
    for (int i = threadIdx.x; i < k; i += kDenseSmemThreads)
      if (sk[i] != 0.0f) atomicAdd(out + i, sk[i]);
  }
}

// One CTA per (row, 4096-element chunk): 128-bit loads, warp shuffle + shared
// reduction, one f32 atomic per CTA (1024 CTAs for 256 rows of 16384).
constexpr int kDotChunk = 4096;

__global__ void __launch_bounds__(256) sketch_dot_kernel(const float* __restrict__ phi, const float* __restrict__ tau,
                                                         int64_t k, int n_chunks, float alpha,
                                                         float* __restrict__ score) {
  const int64_t row = blockIdx.x / n_chunks;
  const int64_t c0 = (int64_t)(blockIdx.x % n_chunks) * kDotChunk;
  const int64_t c1 = min(k, c0 + kDotChunk);
  const float* p = phi + row * k;
  float acc = 0.0f;
  if ((k & 3) == 0) {
    const float4* p4 = reinterpret_cast<const float4*>(p);
    const float4* t4 = reinterpret_cast<const float4*>(tau);
#pragma unroll 4
    for (int64_t i = c0 / 4 + threadIdx.x; i < c1 / 4; i += 256) {
      const float4 a = __ldcs(p4 + i), b = __ldg(t4 + i);
      acc = fmaf(a.x, b.x, acc);
      acc = fmaf(a.y, b.y, acc);
      acc = fmaf(a.z, b.z, acc);
      acc = fmaf(a.w, b.w, acc);
    }
  } else {
    for (int64_t i = c0 + threadIdx.x; i < c1; i += 256) acc = fmaf(p[i], tau[i], acc);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  __shared__ float part[8];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int i = 0; i < 8; ++i) t += part[i];
    atomicAdd(score + row, alpha * t);
  }
}

__global__ void split_bf16_kernel(const float* __restrict__ x, int64_t n, __nv_bfloat16* __restrict__ hi,
                                  __nv_bfloat16* __restrict__ lo) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    hi[i] = h;
    lo[i] = __float2bfloat16_rn(v - __bfloat162float(h));
  }
}

}  // namespace
}  // namespace opus

using namespace opus;

extern "C" {

int opus_sketch_dense(const float* w, int transposed, const uint32_t* packed, const float* diag, int d_out, int d_in,
                      int row_begin, int row_end, int64_t k, float* sketch, int accumulate, void* stream) {
  if (d_out <= 0 || d_in <= 0 || k <= 0 || k > 0x7FFFFFFF) return set_error(OPUS_ERR_INVALID, "sketch_dense: bad sizes");
  if (row_begin < 0 || row_end > d_out || row_begin > row_end)
    return set_error(OPUS_ERR_INVALID, "sketch_dense: rows [%d, %d) outside [0, %d)", row_begin, row_end, d_out);
  if (!w || !packed || !sketch) return set_error(OPUS_ERR_INVALID, "sketch_dense: NULL pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (!accumulate) OPUS_CUDA_TRY(cudaMemsetAsync(sketch, 0, (size_t)k * sizeof(float), st));
  if (row_end == row_begin) return OPUS_OK;
  const int64_t n_tiles =
      (int64_t)((row_end - row_begin + kDenseTile - 1) / kDenseTile) * ((d_in + kDenseTile - 1) / kDenseTile);
  const size_t smem = (size_t)k * sizeof(float);
  const int64_t numel = (int64_t)(row_end - row_begin) * d_in;
  if (smem + sizeof(float) * kDenseGroup * kDenseTile * (kDenseTile + 1) + 1024 <= (size_t)max_smem_optin()) {
    // one CTA per SM at most, and at least ~k elements per CTA so the flushes (k floats each) stay
    // below the element updates
    const int64_t n_groups = (n_tiles + kDenseGroup - 1) / kDenseGroup;
    int64_t grid = numel / k;
    if (grid > sm_count()) grid = sm_count();
    if (grid > n_groups) grid = n_groups;
    if (grid < 1) grid = 1;
    OPUS_CUDA_TRY(cudaFuncSetAttribute(dense_sketch_smem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem)));
    dense_sketch_smem_kernel<<<(int)grid, kDenseSmemThreads, smem, st>>>(w, transposed, packed, diag, d_out, d_in,
                                                                        row_begin, row_end, static_cast<int>(k),
                                                                        sketch);
    ::opus::note_launch();
  } else {
    int64_t grid = (int64_t)sm_count() * 8;
    if (grid > n_tiles) grid = n_tiles;
    dense_sketch_kernel<<<(int)grid, kDenseThreads, 0, st>>>(w, transposed, packed, diag, d_out, d_in, row_begin,
                                                             row_end, k, sketch);
    ::opus::note_launch();
  }
  OPUS_CUDA_TRY(cudaGetLastError());
  return OPUS_OK;
}

int opus_sketch_dot(const float* phi, const float* tau, int n_rows, int64_t k, float alpha, float* score,
                    int accumulate, void* stream) {
  if (n_rows < 0 || k <= 0) return set_error(OPUS_ERR_INVALID, "sketch_dot: bad sizes");
  if (n_rows == 0) return OPUS_OK;
  if (!phi || !tau || !score) return set_error(OPUS_ERR_INVALID, "sketch_dot: NULL pointer");
  if (((reinterpret_cast<uintptr_t>(phi) | reinterpret_cast<uintptr_t>(tau)) & 15) != 0 && (k & 3) == 0)
    return set_error(OPUS_ERR_INVALID, "sketch_dot: phi and tau must be 16-byte aligned");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (!accumulate) OPUS_CUDA_TRY(cudaMemsetAsync(score, 0, (size_t)n_rows * sizeof(float), st));
  const int64_t n_chunks = (k + kDotChunk - 1) / kDotChunk;
  const int64_t grid = (int64_t)n_rows * n_chunks;
  if (grid > 0x7fffffff) return set_error(OPUS_ERR_UNSUPPORTED, "sketch_dot: too many rows");
  sketch_dot_kernel<<<(int)grid, 256, 0, st>>>(phi, tau, k, (int)n_chunks, alpha, score);
  ::opus::note_launch();
  OPUS_CUDA_TRY(cudaGetLastError());
  return OPUS_OK;
}

int opus_split_bf16(const float* x, int64_t n, void* hi, void* lo, void* stream) {
  if (n < 0) return set_error(OPUS_ERR_INVALID, "split_bf16: bad size");
  if (n == 0) return OPUS_OK;
  if (!x || !hi || !lo) return set_error(OPUS_ERR_INVALID, "split_bf16: NULL pointer");
  int64_t grid = (n + 255) / 256;
  if (grid > (int64_t)sm_count() * 16) grid = (int64_t)sm_count() * 16;
  split_bf16_kernel<<<(int)grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      x, n, reinterpret_cast<__nv_bfloat16*>(hi), reinterpret_cast<__nv_bfloat16*>(lo));
  ::opus::note_launch();
  OPUS_CUDA_TRY(cudaGetLastError());
  return OPUS_OK;
}

}  // extern "C"
