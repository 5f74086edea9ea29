// Sketch Gram blocks: out[i,j] (+)= alpha * phi_a[i,:] . phi_b[j,:] in f32.
// 64x64 output tile per CTA, 4x4 per thread, K staged through shared memory
// in chunks of 32; the k range is split across CTAs (f32 atomics combine the
// splits) so that small candidate counts still fill the GPU.
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

}  // namespace
}  // namespace opus

using namespace opus;

extern "C" int opus_sketch_gram(const float* phi_a, int rows_a, const float* phi_b, int rows_b, int64_t k, float alpha,
                                float* out, int accumulate, void* stream) {
  if (rows_a < 0 || rows_b < 0 || k <= 0) return set_error(OPUS_ERR_INVALID, "sketch_gram: bad sizes");
  if (rows_a == 0 || rows_b == 0) return OPUS_OK;
  if (!phi_a || !phi_b || !out) return set_error(OPUS_ERR_INVALID, "sketch_gram: NULL pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
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
  OPUS_CUDA_TRY(cudaGetLastError());
  return OPUS_OK;
}
