// CountSketch tables and preconditioner folding (memory-bound, one pass each).
//
//   opus_pack_hash_sign     int64 bucket + f32 sign  ->  uint32 (bucket | neg<<31)
//   opus_build_sketch_table packed + AdamW diag      ->  tiled epilogue table
//   opus_desketch           tau + packed + diag      ->  dense bf16 hi/lo target
//   opus_bucket_max_load    packed                   ->  per-bucket counts, their max
//   opus_bucket_max_load_noalloc                     ->  the max, counting in static device memory
#include <mutex>

#include "opus_common.cuh"
#include "sketch_layout.cuh"

namespace opus {
namespace {

__global__ void pack_kernel(const int64_t* __restrict__ hash, const float* __restrict__ sign, int64_t numel,
                            int64_t k, uint32_t* __restrict__ out, int* err) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < numel; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t h = hash[i];
    const float s = sign[i];
    uint32_t v = 0;
    if (h < 0 || h >= k || !(s == 1.0f || s == -1.0f)) {
      record_device_error(err, kDevBadBucket);
    } else {
      v = static_cast<uint32_t>(h) | (s < 0.0f ? 0x80000000u : 0u);
    }
    out[i] = v;
  }
}

// AdamW diagonal exactly as torch evaluates (v.sqrt() + eps).reciprocal() in
// f32: correctly rounded sqrt, f32 add, correctly rounded reciprocal.
__device__ __forceinline__ float adam_diag(float v, float eps) {
  return __frcp_rn(__fadd_rn(__fsqrt_rn(v), eps));
}

__device__ __forceinline__ float element_weight(const float* diag, const float* v, float eps, int64_t idx) {
  if (diag != nullptr) return diag[idx];
  if (v != nullptr) return adam_diag(v[idx], eps);
  return 1.0f;
}

// One CTA per (tile, 32-column chunk): stage 128 rows x 32 columns of the
// packed table and weights in shared memory with coalesced row reads, then
// write them in the epilogue's lane-fastest order with coalesced 16-B stores.
__global__ void __launch_bounds__(256) build_table_kernel(const uint32_t* __restrict__ packed,
                                                          const float* __restrict__ diag,
                                                          const float* __restrict__ v, float eps, int d_out,
                                                          int d_in, int n_cb, uint4* __restrict__ table) {
  __shared__ uint32_t sh[kTileM][kChunkCols + 1];
  __shared__ float sw[kTileM][kChunkCols + 1];
  const int tile = blockIdx.x / kChunksPerTile;
  const int j = blockIdx.x % kChunksPerTile;
  const int ob = tile / n_cb, cb = tile % n_cb;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = cb * kTileN + j * kChunkCols + lane;
  // 16 rows per warp, all loads issued before any use
  uint32_t hv[kTileM / 8];
  float src[kTileM / 8];
#pragma unroll
  for (int i = 0; i < kTileM / 8; ++i) {
    const int o = ob * kTileM + warp + 8 * i;
    const bool in = o < d_out && c < d_in;
    const int64_t idx = (int64_t)o * d_in + c;
    hv[i] = in ? packed[idx] : 0u;
    src[i] = in ? (diag != nullptr ? diag[idx] : (v != nullptr ? v[idx] : 1.0f)) : 0.0f;
  }
#pragma unroll
  for (int i = 0; i < kTileM / 8; ++i) {
    const int r = warp + 8 * i;
    const float d = (diag == nullptr && v != nullptr) ? adam_diag(src[i], eps) : src[i];
    const float wv = (hv[i] & 0x80000000u) ? -d : d;
    sh[r][lane] = hv[i] & 0x7FFFFFFFu;
    sw[r][lane] = (ob * kTileM + r < d_out && c < d_in) ? wv : 0.0f;
  }
  __syncthreads();
  uint4* out = table + ((int64_t)tile * kChunksPerTile + j) * (kPairsPerChunk * kTileM);
  for (int e = threadIdx.x; e < kPairsPerChunk * kTileM; e += 256) {
    const int p = e / kTileM, r = e % kTileM;
    uint4 q;
    q.x = sh[r][2 * p];
    q.y = sh[r][2 * p + 1];
    q.z = __float_as_uint(sw[r][2 * p]);
    q.w = __float_as_uint(sw[r][2 * p + 1]);
    out[e] = q;
  }
}

// Four elements per thread: 16-byte loads of the packed table and the
// diagonal, tau gathered through the read-only cache (k floats, L1-resident
// for the usual sketch sizes), 8-byte stores of four bf16 hi and four lo.
__device__ __forceinline__ void desketch_one(float t, uint32_t hv, float d, float scale, __nv_bfloat16& h,
                                             __nv_bfloat16& l) {
  float x = __fmul_rn(__fmul_rn(scale, d), t);
  if (hv & 0x80000000u) x = -x;
  h = __float2bfloat16_rn(x);
  l = __float2bfloat16_rn(x - __bfloat162float(h));
}

__global__ void desketch_kernel(const float* __restrict__ tau, const uint32_t* __restrict__ packed,
                                const float* __restrict__ diag, const float* __restrict__ v, float eps,
                                int64_t numel, float scale, __nv_bfloat16* __restrict__ hi,
                                __nv_bfloat16* __restrict__ lo, int vec) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t start = 0;
  if (vec) {
    const int64_t n4 = numel / 4;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
      const uint4 hv = __ldcs(reinterpret_cast<const uint4*>(packed) + i);
      float4 d = make_float4(1.0f, 1.0f, 1.0f, 1.0f);
      if (diag != nullptr) {
        d = __ldcs(reinterpret_cast<const float4*>(diag) + i);
      } else if (v != nullptr) {
        const float4 q = __ldcs(reinterpret_cast<const float4*>(v) + i);
        d = make_float4(adam_diag(q.x, eps), adam_diag(q.y, eps), adam_diag(q.z, eps), adam_diag(q.w, eps));
      }
      __align__(8) __nv_bfloat16 h[4], l[4];
      desketch_one(__ldg(tau + (hv.x & 0x7FFFFFFFu)), hv.x, d.x, scale, h[0], l[0]);
      desketch_one(__ldg(tau + (hv.y & 0x7FFFFFFFu)), hv.y, d.y, scale, h[1], l[1]);
      desketch_one(__ldg(tau + (hv.z & 0x7FFFFFFFu)), hv.z, d.z, scale, h[2], l[2]);
      desketch_one(__ldg(tau + (hv.w & 0x7FFFFFFFu)), hv.w, d.w, scale, h[3], l[3]);
      __stcs(reinterpret_cast<uint2*>(hi) + i, *reinterpret_cast<const uint2*>(h));
      __stcs(reinterpret_cast<uint2*>(lo) + i, *reinterpret_cast<const uint2*>(l));
    }
    start = n4 * 4;
  }
  for (int64_t i = start + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < numel; i += stride) {
    const uint32_t hv = packed[i];
    desketch_one(tau[hv & 0x7FFFFFFFu], hv, element_weight(diag, v, eps, i), scale, hi[i], lo[i]);
  }
}

// D = 1 / (sqrt(v) + eps) elementwise: 16-byte loads and stores when aligned,
// four loads in flight per thread.
constexpr int kDiagUnroll = 4;

__global__ void adam_diag_kernel(const float* __restrict__ v, float eps, int64_t n, float* __restrict__ out,
                                 int vec) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t start = 0;
  if (vec) {
    const int64_t n4 = n / 4;
    const float4* v4 = reinterpret_cast<const float4*>(v);
    float4* o4 = reinterpret_cast<float4*>(out);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride * kDiagUnroll) {
      float4 q[kDiagUnroll];
#pragma unroll
      for (int u = 0; u < kDiagUnroll; ++u) {
        const int64_t iu = i + u * stride;
        q[u] = iu < n4 ? __ldcs(v4 + iu) : make_float4(1.f, 1.f, 1.f, 1.f);
      }
#pragma unroll
      for (int u = 0; u < kDiagUnroll; ++u) {
        const int64_t iu = i + u * stride;
        if (iu < n4)
          __stcs(o4 + iu, make_float4(adam_diag(q[u].x, eps), adam_diag(q[u].y, eps), adam_diag(q[u].z, eps),
                                      adam_diag(q[u].w, eps)));
      }
    }
    start = n4 * 4;
  }
  for (int64_t i = start + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = adam_diag(v[i], eps);
}

int grid_for(int64_t n, int threads) {
  int64_t g = (n + threads - 1) / threads;
  const int64_t cap = (int64_t)sm_count() * 16;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return static_cast<int>(g);
}

// Per-bucket element counts of a packed table.  Up to kHistSmemBuckets
// buckets each CTA counts into shared memory (native int32 shared atomics) and
// adds its nonzero bins to the global counts once; larger sketches count
// straight into the global array (L2 atomics).  An entry whose bucket is not
// below k is skipped and recorded as kDevBadBucket.
constexpr int kHistThreads = 512;
constexpr int kHistSmemBuckets = 32768;  // 128 KB of shared counts

template <bool kShared>
__global__ void __launch_bounds__(kHistThreads) bucket_hist_kernel(const uint32_t* __restrict__ packed, int64_t numel,
                                                                  uint32_t k, int* __restrict__ counts, int* err) {
  extern __shared__ int sh_counts[];
  if (kShared) {
    for (uint32_t i = threadIdx.x; i < k; i += blockDim.x) sh_counts[i] = 0;
    __syncthreads();
  }
  int* dst = kShared ? sh_counts : counts;
  bool bad = false;
  auto count = [&](uint32_t v) {
    const uint32_t b = v & 0x7FFFFFFFu;
    if (b < k) atomicAdd(dst + b, 1); else bad = true;
  };
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  // 16-byte loads over the aligned body, scalar loads over the rest
  const int64_t mis = static_cast<int64_t>(reinterpret_cast<uintptr_t>(packed) & 15);
  int64_t head = mis == 0 ? 0 : (16 - mis) / 4;
  if (head > numel) head = numel;
  const int64_t n4 = (numel - head) / 4;
  const uint4* p4 = reinterpret_cast<const uint4*>(packed + head);
  for (int64_t i = tid; i < n4; i += stride) {
    const uint4 v = __ldg(p4 + i);
    count(v.x);
    count(v.y);
    count(v.z);
    count(v.w);
  }
  for (int64_t i = tid; i < head; i += stride) count(packed[i]);
  for (int64_t i = head + n4 * 4 + tid; i < numel; i += stride) count(packed[i]);
  if (bad) record_device_error(err, kDevBadBucket);
  if (kShared) {
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < k; i += blockDim.x) {
      const int c = sh_counts[i];
      if (c) atomicAdd(counts + i, c);
    }
  }
}

// One CTA: max over the k counts.
__global__ void __launch_bounds__(1024) bucket_max_kernel(const int* __restrict__ counts, int64_t k,
                                                          int64_t* __restrict__ out) {
  int mx = 0;
  for (int64_t i = threadIdx.x; i < k; i += 1024) mx = max(mx, counts[i]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  __shared__ int part[32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    mx = part[threadIdx.x];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (threadIdx.x == 0) *out = mx;
  }
}

// Counts (zeroed here) then their max; counts holds the histogram afterwards.
int launch_bucket_max_load(const uint32_t* packed, int64_t numel, int64_t k, int* counts, int64_t* out_max,
                           cudaStream_t st) {
  OPUS_CUDA_TRY(cudaMemsetAsync(counts, 0, (size_t)k * sizeof(int), st));
  if (numel > 0) {
    int* err = device_error_word();
    if (k <= kHistSmemBuckets) {
      // enough CTAs to stream the table, few enough that the k-bin flushes stay
      // well below the element count
      int64_t grid = numel / (8 * k);
      grid = grid < 1 ? 1 : (grid > sm_count() ? sm_count() : grid);
      const size_t smem = (size_t)k * sizeof(int);
      OPUS_CUDA_TRY(cudaFuncSetAttribute(bucket_hist_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem));
      bucket_hist_kernel<true><<<(int)grid, kHistThreads, smem, st>>>(packed, numel, (uint32_t)k, counts, err);
      ::opus::note_launch();
    } else {
      bucket_hist_kernel<false><<<grid_for(numel / 4 + 1, kHistThreads), kHistThreads, 0, st>>>(
          packed, numel, (uint32_t)k, counts, err);
      ::opus::note_launch();
    }
    OPUS_CUDA_TRY(cudaGetLastError());
  }
  bucket_max_kernel<<<1, 1024, 0, st>>>(counts, k, out_max);
  ::opus::note_launch();
  OPUS_CUDA_TRY(cudaGetLastError());
  return OPUS_OK;
}

// ---- the max bucket load without any allocation
// Counting needs k int32 of scratch.  This variant keeps it in a static
// device array of the module (one copy per device, reserved when the module
// loads) instead of a caller's buffer: slot 0 is the bad-bucket flag and the
// counts start 64 ints (256 B) in.  Both are zeroed on the stream by every
// call; calls that overlap on one device share the array and race.
constexpr int64_t kNoAllocMaxBuckets = 262144;  // 1 MB of counts
constexpr int kNoAllocCountsOffset = 64;
constexpr int kNoAllocMaxDevices = 64;

std::mutex g_noalloc_mu;
int* g_noalloc_ptr[kNoAllocMaxDevices] = {nullptr};
// the context each cached address belongs to: after cudaDeviceReset the
// module is loaded again into a new context and the address is looked up anew
CUcontext g_noalloc_ctx[kNoAllocMaxDevices] = {nullptr};

}  // namespace

static __device__ __align__(256) int g_noalloc_scratch[kNoAllocCountsOffset + kNoAllocMaxBuckets];

namespace {

// Device address of the static scratch for the current device, looked up by
// the first call on that device (in its current context) and cached.
int noalloc_scratch(int** out) {
  int dev = 0;
  OPUS_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return set_error(OPUS_ERR_UNSUPPORTED, "bucket_max_load_noalloc: device %d beyond %d", dev, kNoAllocMaxDevices);
  CUcontext ctx = nullptr;
  int rc = current_context(&ctx);
  if (rc != OPUS_OK) return rc;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr || ctx == nullptr || g_noalloc_ctx[dev] != ctx) {
    void* p = nullptr;
    OPUS_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));  // makes the primary context current if none was
    rc = current_context(&ctx);
    if (rc != OPUS_OK) return rc;
    g_noalloc_ptr[dev] = static_cast<int*>(p);
    g_noalloc_ctx[dev] = ctx;
  }
  *out = g_noalloc_ptr[dev];
  return OPUS_OK;
}

// One CTA: max over the k counts, or -1 when the flag records a bucket >= k.
__global__ void __launch_bounds__(1024) bucket_max_flagged_kernel(const int* __restrict__ counts, int64_t k,
                                                                  const int* __restrict__ bad,
                                                                  int64_t* __restrict__ out) {
  int mx = 0;
  for (int64_t i = threadIdx.x; i < k; i += 1024) mx = max(mx, counts[i]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  __shared__ int part[32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    mx = part[threadIdx.x];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (threadIdx.x == 0) *out = *bad ? -1 : mx;
  }
}

int launch_bucket_max_load_noalloc(const uint32_t* packed, int64_t numel, int64_t k, int64_t* out_max,
                                   cudaStream_t st) {
  int* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != OPUS_OK) return rc;
  int* bad = scratch;
  int* counts = scratch + kNoAllocCountsOffset;
  OPUS_CUDA_TRY(cudaMemsetAsync(scratch, 0, (size_t)(kNoAllocCountsOffset + k) * sizeof(int), st));
  if (numel > 0) {
    if (k <= kHistSmemBuckets) {
      int64_t grid = numel / (8 * k);
      grid = grid < 1 ? 1 : (grid > sm_count() ? sm_count() : grid);
      const size_t smem = (size_t)k * sizeof(int);
      OPUS_CUDA_TRY(cudaFuncSetAttribute(bucket_hist_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem));
      bucket_hist_kernel<true><<<(int)grid, kHistThreads, smem, st>>>(packed, numel, (uint32_t)k, counts, bad);
      ::opus::note_launch();
    } else {
      bucket_hist_kernel<false><<<grid_for(numel / 4 + 1, kHistThreads), kHistThreads, 0, st>>>(
          packed, numel, (uint32_t)k, counts, bad);
      ::opus::note_launch();
    }
    OPUS_CUDA_TRY(cudaGetLastError());
  }
  bucket_max_flagged_kernel<<<1, 1024, 0, st>>>(counts, k, bad, out_max);
  ::opus::note_launch();
  OPUS_CUDA_TRY(cudaGetLastError());
  return OPUS_OK;
}

}  // namespace
}  // namespace opus

using namespace opus;

extern "C" {

int opus_pack_hash_sign(const int64_t* hash, const float* sign, int64_t numel, int64_t k, uint32_t* packed,
                        void* stream) {
  if (numel < 0 || k <= 0 || k > 0x7FFFFFFF) return set_error(OPUS_ERR_INVALID, "pack: bad numel/k");
  if (numel == 0) return OPUS_OK;
  if (!hash || !sign || !packed) return set_error(OPUS_ERR_INVALID, "pack: NULL pointer");
  int* err = device_error_word();
  pack_kernel<<<grid_for(numel, 256), 256, 0, (cudaStream_t)stream>>>(hash, sign, numel, k, packed, err);
  ::opus::note_launch();
  OPUS_CUDA_TRY(cudaGetLastError());
  return OPUS_OK;
}

int64_t opus_sketch_table_entries(int d_out, int d_in) {
  if (d_out <= 0 || d_in <= 0) return 0;
  return table_entries(d_out, d_in);
}

int opus_build_sketch_table(const uint32_t* packed, const float* diag, const float* exp_avg_sq, float eps,
                            int d_out, int d_in, void* table, int64_t table_entries_given, void* stream) {
  if (d_out <= 0 || d_in <= 0) return set_error(OPUS_ERR_INVALID, "table: bad shape %d x %d", d_out, d_in);
  if (!packed || !table) return set_error(OPUS_ERR_INVALID, "table: NULL pointer");
  if (table_entries_given < table_entries(d_out, d_in))
    return set_error(OPUS_ERR_INVALID, "table: buffer holds %lld entries, need %lld",
                     (long long)table_entries_given, (long long)table_entries(d_out, d_in));
  if ((reinterpret_cast<uintptr_t>(table) & 15) != 0) return set_error(OPUS_ERR_INVALID, "table: not 16-B aligned");
  const int n_ob = ceil_div(d_out, kTileM), n_cb = ceil_div(d_in, kTileN);
  const int blocks = n_ob * n_cb * kChunksPerTile;
  build_table_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(packed, diag, exp_avg_sq, eps, d_out, d_in, n_cb,
                                                              reinterpret_cast<uint4*>(table));
  ::opus::note_launch();
  OPUS_CUDA_TRY(cudaGetLastError());
  return OPUS_OK;
}

int opus_desketch(const float* tau, const uint32_t* packed, const float* diag, const float* exp_avg_sq, float eps,
                  int d_out, int d_in, int64_t k, float scale, void* v_bf16, void* stream) {
  if (d_out <= 0 || d_in <= 0 || k <= 0) return set_error(OPUS_ERR_INVALID, "desketch: bad shape");
  if (!tau || !packed || !v_bf16) return set_error(OPUS_ERR_INVALID, "desketch: NULL pointer");
  const int64_t numel = (int64_t)d_out * d_in;
  __nv_bfloat16* hi = reinterpret_cast<__nv_bfloat16*>(v_bf16);
  __nv_bfloat16* lo = hi + numel;
  const uintptr_t al = reinterpret_cast<uintptr_t>(packed) | reinterpret_cast<uintptr_t>(diag) |
                       reinterpret_cast<uintptr_t>(exp_avg_sq);
  const int vec = (al & 15) == 0 && (reinterpret_cast<uintptr_t>(hi) & 7) == 0 && (reinterpret_cast<uintptr_t>(lo) & 7) == 0;
  desketch_kernel<<<grid_for(vec ? numel / 4 + 1 : numel, 256), 256, 0, (cudaStream_t)stream>>>(
      tau, packed, diag, exp_avg_sq, eps, numel, scale, hi, lo, vec);
  ::opus::note_launch();
  OPUS_CUDA_TRY(cudaGetLastError());
  return OPUS_OK;
}

int opus_adam_diag(const float* exp_avg_sq, float eps, int64_t n, float* out, void* stream) {
  if (n < 0) return set_error(OPUS_ERR_INVALID, "adam_diag: negative size");
  if (n == 0) return OPUS_OK;
  if (!exp_avg_sq || !out) return set_error(OPUS_ERR_INVALID, "adam_diag: NULL pointer");
  const int vec = ((reinterpret_cast<uintptr_t>(exp_avg_sq) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
  const int64_t per_thread = vec ? 4 * kDiagUnroll : 1;
  adam_diag_kernel<<<grid_for(n / per_thread + 1, 256), 256, 0, (cudaStream_t)stream>>>(exp_avg_sq, eps, n, out,
                                                                                         vec);
  ::opus::note_launch();
  OPUS_CUDA_TRY(cudaGetLastError());
  return OPUS_OK;
}

int opus_bucket_max_load(const uint32_t* packed, int64_t numel, int64_t k, int* counts, int64_t counts_len,
                         int64_t* out_max, void* stream) {
  if (numel < 0 || k <= 0 || k > 0x7FFFFFFF) return set_error(OPUS_ERR_INVALID, "bucket_max_load: bad numel/k");
  if (counts_len < k)
    return set_error(OPUS_ERR_INVALID, "bucket_max_load: counts holds %lld entries, need %lld", (long long)counts_len,
                     (long long)k);
  if ((numel > 0 && !packed) || !counts || !out_max) return set_error(OPUS_ERR_INVALID, "bucket_max_load: NULL pointer");
  return launch_bucket_max_load(packed, numel, k, counts, out_max, (cudaStream_t)stream);
}

int opus_bucket_max_load_noalloc(const uint32_t* packed, int64_t numel, int64_t k, int64_t* out_max, void* stream) {
  if (numel < 0 || k <= 0) return set_error(OPUS_ERR_INVALID, "bucket_max_load_noalloc: bad numel/k");
  if (k > kNoAllocMaxBuckets)
    return set_error(OPUS_ERR_INVALID, "bucket_max_load_noalloc: k=%lld exceeds the static scratch of %lld buckets",
                     (long long)k, (long long)kNoAllocMaxBuckets);
  if ((numel > 0 && !packed) || !out_max) return set_error(OPUS_ERR_INVALID, "bucket_max_load_noalloc: NULL pointer");
  return launch_bucket_max_load_noalloc(packed, numel, k, out_max, (cudaStream_t)stream);
}

}  // extern "C"
