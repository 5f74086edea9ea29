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

// The same CountSketch with a CTA-private int32 sketch in shared memory.
// Float atomics on shared memory are compare-and-swap loops on this GPU
// (about 0.76 updates per clock per SM), integer adds are native (5-7), so
// each CTA makes two passes over its contiguous share of the elements:
//   1. the largest finite |w * diag| of the share (M);
//   2. every element times S = 2^e, rounded to int32 and added into bucket
//      h of the shared sketch, where M * S <= cap = 2^30 / L, L the largest
//      number of the share's elements one bucket can receive: the table's
//      largest bucket load when the caller gives it, else the share's element
//      count.  With the rounding (at most 1/2 per element) no bucket can
//      overflow whatever the data.  Buckets at or
//      above k_sm (sketches larger than shared memory) and non-finite values
//      go to the output with f32 global atomics.
// The second pass re-reads the share, which the first pass has just brought
// into L2.  The sketch is converted back (q / S) and added to the output once,
// with 16-byte vector reductions.  Rounding error per element is at most
// M * L / 2^31: about 1e-7 of the share's largest value with the table's
// bucket load (about 2e-5 with the element count of a GPT-2-XL MLP matrix's
// share).  A CTA handles one vector (blockIdx.y) of a batch.
//
// Flat layout (w[o * d_in + c], the packed table's order): a unit is 4
// consecutive elements read as float4 / uint4.  Transposed layout
// (w[c * d_out + o]): a unit is a 32 x 32 tile staged through shared memory;
// pass 1 then bounds |w * diag| by max|w| * max|diag| of the tiles.
constexpr int kDenseSmemThreads = 1024;
constexpr int kDenseUnroll = 2;

__device__ __forceinline__ float finite_abs(float x) {
  const float a = fabsf(x);
  return a <= 3.0e38f ? a : 0.0f;
}

__device__ __forceinline__ float block_max(float m, float* red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = red[threadIdx.x];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (threadIdx.x == 0) red[0] = m;
  }
  __syncthreads();
  m = red[0];
  __syncthreads();
  return m;
}

// S = 2^e with M * S <= cap, or 0 when the share holds no nonzero finite value.
__device__ __forceinline__ float fixed_scale(float M, int64_t count) {
  if (!(M > 0.0f) || count <= 0) return 0.0f;
  const double cap = 1073741824.0 / static_cast<double>(count);
  int e;
  frexp(cap / static_cast<double>(M), &e);  // cap / M in [2^(e-1), 2^e)
  return ldexpf(1.0f, max(-126, min(126, e - 1)));
}

__device__ __forceinline__ void add_fixed(int* sk, float* out, uint32_t hv, float x, float S, int k, int k_sm) {
  if (hv & 0x80000000u) x = -x;
  const uint32_t bucket = hv & 0x7FFFFFFFu;
  if (bucket >= static_cast<uint32_t>(k) || x == 0.0f) return;
  if (bucket < static_cast<uint32_t>(k_sm) && fabsf(x) <= 3.0e38f && S > 0.0f)
    atomicAdd(sk + bucket, __float2int_rn(x * S));
  else
    atomicAdd(out + bucket, x);
}

__device__ void flush_fixed(int* sk, float* out, int k_sm, float S) {
  __syncthreads();
  if (S > 0.0f) {
    const float inv = 1.0f / S;  // S is a power of two: exact
    if ((k_sm & 3) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0) {
      const int4* s4 = reinterpret_cast<const int4*>(sk);
      for (int i = threadIdx.x; i < k_sm / 4; i += kDenseSmemThreads) {
        const int4 q = s4[i];
        if (q.x | q.y | q.z | q.w)
          red_add_v4(out + 4 * i, (float)q.x * inv, (float)q.y * inv, (float)q.z * inv, (float)q.w * inv);
      }
    } else {
      for (int i = threadIdx.x; i < k_sm; i += kDenseSmemThreads)
        if (sk[i] != 0) atomicAdd(out + i, (float)sk[i] * inv);
    }
  }
}

__global__ void __launch_bounds__(kDenseSmemThreads) dense_sketch_flat_kernel(
    const float* __restrict__ w, const uint32_t* __restrict__ packed, const float* __restrict__ diag, int64_t e_begin,
    int64_t e_end, int k, int k_sm, int max_load, float* __restrict__ out, int64_t w_stride, int64_t out_stride,
    int vec) {
  extern __shared__ __align__(16) int sk[];
  __shared__ float red[32];
  w += (int64_t)blockIdx.y * w_stride;
  out += (int64_t)blockIdx.y * out_stride;
  for (int i = threadIdx.x; i < k_sm; i += kDenseSmemThreads) sk[i] = 0;
  // this CTA's elements: [a, b) of [e_begin, e_end), multiples of 4 when vectorised
  const int64_t n = e_end - e_begin;
  const int64_t units = vec ? n / 4 : n;
  const int64_t u0 = units * blockIdx.x / gridDim.x, u1 = units * (blockIdx.x + 1) / gridDim.x;
  const bool last = blockIdx.x == gridDim.x - 1;
  const int64_t tail0 = e_begin + (vec ? units * 4 : n);  // scalar tail [tail0, e_end), last CTA only
  const int64_t count = (u1 - u0) * (vec ? 4 : 1) + (last ? e_end - tail0 : 0);
  // pass 1: the share's largest finite |w * diag|
  float m = 0.0f;
  if (vec) {
    const float4* w4 = reinterpret_cast<const float4*>(w + e_begin);
    const float4* d4 = diag != nullptr ? reinterpret_cast<const float4*>(diag + e_begin) : nullptr;
    for (int64_t u = u0 + threadIdx.x; u < u1; u += kDenseSmemThreads * kDenseUnroll) {
      float4 x[kDenseUnroll], d[kDenseUnroll];
#pragma unroll
      for (int j = 0; j < kDenseUnroll; ++j) {
        const int64_t uj = u + (int64_t)j * kDenseSmemThreads;
        x[j] = uj < u1 ? __ldg(w4 + uj) : make_float4(0.f, 0.f, 0.f, 0.f);
        d[j] = (diag != nullptr && uj < u1) ? __ldg(d4 + uj) : make_float4(1.f, 1.f, 1.f, 1.f);
      }
#pragma unroll
      for (int j = 0; j < kDenseUnroll; ++j)
        m = fmaxf(m, fmaxf(fmaxf(finite_abs(x[j].x * d[j].x), finite_abs(x[j].y * d[j].y)),
                           fmaxf(finite_abs(x[j].z * d[j].z), finite_abs(x[j].w * d[j].w))));
    }
  } else {
    for (int64_t u = u0 + threadIdx.x; u < u1; u += kDenseSmemThreads)
      m = fmaxf(m, finite_abs(w[e_begin + u] * (diag != nullptr ? diag[e_begin + u] : 1.0f)));
  }
  if (last)
    for (int64_t i = tail0 + threadIdx.x; i < e_end; i += kDenseSmemThreads)
      m = fmaxf(m, finite_abs(w[i] * (diag != nullptr ? diag[i] : 1.0f)));
  const int64_t load = max_load > 0 && max_load < count ? max_load : count;
  const float S = fixed_scale(block_max(m, red), load);  // its barriers also order the sketch zeroing
  // pass 2: the scatter
  if (vec) {
    const float4* w4 = reinterpret_cast<const float4*>(w + e_begin);
    const float4* d4 = diag != nullptr ? reinterpret_cast<const float4*>(diag + e_begin) : nullptr;
    const uint4* h4 = reinterpret_cast<const uint4*>(packed + e_begin);
    for (int64_t u = u0 + threadIdx.x; u < u1; u += kDenseSmemThreads * kDenseUnroll) {
      float4 x[kDenseUnroll], d[kDenseUnroll];
      uint4 h[kDenseUnroll];
#pragma unroll
      for (int j = 0; j < kDenseUnroll; ++j) {
        const int64_t uj = u + (int64_t)j * kDenseSmemThreads;
        const bool in = uj < u1;
        x[j] = in ? __ldg(w4 + uj) : make_float4(0.f, 0.f, 0.f, 0.f);
        h[j] = in ? __ldcs(h4 + uj) : make_uint4(0u, 0u, 0u, 0u);
        d[j] = (diag != nullptr && in) ? __ldg(d4 + uj) : make_float4(1.f, 1.f, 1.f, 1.f);
      }
#pragma unroll
      for (int j = 0; j < kDenseUnroll; ++j) {
        add_fixed(sk, out, h[j].x, x[j].x * d[j].x, S, k, k_sm);
        add_fixed(sk, out, h[j].y, x[j].y * d[j].y, S, k, k_sm);
        add_fixed(sk, out, h[j].z, x[j].z * d[j].z, S, k, k_sm);
        add_fixed(sk, out, h[j].w, x[j].w * d[j].w, S, k, k_sm);
      }
    }
  } else {
    for (int64_t u = u0 + threadIdx.x; u < u1; u += kDenseSmemThreads) {
      const int64_t i = e_begin + u;
      add_fixed(sk, out, packed[i], w[i] * (diag != nullptr ? diag[i] : 1.0f), S, k, k_sm);
    }
  }
  if (last)
    for (int64_t i = tail0 + threadIdx.x; i < e_end; i += kDenseSmemThreads)
      add_fixed(sk, out, packed[i], w[i] * (diag != nullptr ? diag[i] : 1.0f), S, k, k_sm);
  flush_fixed(sk, out, k_sm, S);
}

// Transposed layout: 32 x 32 tiles of rows [row_begin, row_end), staged
// through shared memory so both the weight (stored [d_in, d_out]) and the
// table (stored [d_out, d_in]) are read coalesced.  Thread (ty, tx) takes
// element (o0 + ty, c0 + tx) of each tile of its group of kDenseGroup.
constexpr int kDenseGroup = 8;

__global__ void __launch_bounds__(kDenseSmemThreads) dense_sketch_tiles_kernel(
    const float* __restrict__ w, const uint32_t* __restrict__ packed, const float* __restrict__ diag, int d_out,
    int d_in, int row_begin, int row_end, int k, int k_sm, int max_load, float* __restrict__ out) {
  __shared__ float tile_w[kDenseGroup][kDenseTile][kDenseTile + 1];
  __shared__ float red[32];
  extern __shared__ __align__(16) int sk[];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 32
  for (int i = threadIdx.x; i < k_sm; i += kDenseSmemThreads) sk[i] = 0;
  const int rows = row_end - row_begin;
  const int n_to = (rows + kDenseTile - 1) / kDenseTile, n_tc = (d_in + kDenseTile - 1) / kDenseTile;
  const int64_t n_tiles = (int64_t)n_to * n_tc;
  const int64_t t_begin = n_tiles * blockIdx.x / gridDim.x, t_end = n_tiles * (blockIdx.x + 1) / gridDim.x;
  // pass 1: max |w| and max |diag| over the CTA's tiles bound every |w * diag|
  float mw = 0.0f, md = diag != nullptr ? 0.0f : 1.0f;
  int64_t count = 0;
  for (int64_t t = t_begin; t < t_end; ++t) {
    const int o0 = row_begin + static_cast<int>(t / n_tc) * kDenseTile, c0 = static_cast<int>(t % n_tc) * kDenseTile;
    const int c = c0 + ty, o = o0 + tx;  // w read along o (its contiguous axis)
    if (o < row_end && c < d_in) mw = fmaxf(mw, finite_abs(__ldg(w + (int64_t)c * d_out + o)));
    const int oo = o0 + ty, cc = c0 + tx;  // diag read along c
    if (diag != nullptr && oo < row_end && cc < d_in) md = fmaxf(md, finite_abs(__ldg(diag + (int64_t)oo * d_in + cc)));
    count += (int64_t)(min(kDenseTile, row_end - o0)) * min(kDenseTile, d_in - c0);
  }
  mw = block_max(mw, red);
  md = block_max(md, red);
  const float S = fixed_scale(mw * md, max_load > 0 && max_load < count ? max_load : count);
  // pass 2: groups of kDenseGroup tiles, each thread with a load of every input in flight per tile
  for (int64_t t0 = t_begin; t0 < t_end; t0 += kDenseGroup) {
#pragma unroll
    for (int g = 0; g < kDenseGroup; ++g) {
      const int64_t t = t0 + g;
      const int o0 = row_begin + static_cast<int>(t / n_tc) * kDenseTile;
      const int c0 = static_cast<int>(t % n_tc) * kDenseTile;
      const int c = c0 + ty, o = o0 + tx;
      tile_w[g][tx][ty] = (t < t_end && o < row_end && c < d_in) ? __ldg(w + (int64_t)c * d_out + o) : 0.0f;
    }
    __syncthreads();
    float x[kDenseGroup], dg[kDenseGroup];
    uint32_t hv[kDenseGroup];
    bool in[kDenseGroup];
#pragma unroll
    for (int g = 0; g < kDenseGroup; ++g) {
      const int64_t t = t0 + g;
      const int o = row_begin + static_cast<int>(t / n_tc) * kDenseTile + ty;
      const int c = static_cast<int>(t % n_tc) * kDenseTile + tx;
      in[g] = t < t_end && o < row_end && c < d_in;
      const int64_t idx = (int64_t)o * d_in + c;
      hv[g] = in[g] ? __ldcs(packed + idx) : 0u;
      x[g] = tile_w[g][ty][tx];
      dg[g] = (in[g] && diag != nullptr) ? __ldg(diag + idx) : 1.0f;
    }
#pragma unroll
    for (int g = 0; g < kDenseGroup; ++g)
      if (in[g]) add_fixed(sk, out, hv[g], x[g] * dg[g], S, k, k_sm);
    __syncthreads();
  }
  flush_fixed(sk, out, k_sm, S);
}

// One CTA per (row, 8192-element chunk): each of the 256 threads issues its
// eight 16-byte loads of phi (streaming, not kept in L1) and of tau (kept:
// every row reads it again) before any arithmetic, warp shuffle + shared
// reduction, one f32 atomic per CTA (2 CTAs per row at k = 16384, 8 at 65536).
// A persistent grid that prefetches the next chunk measured slower: its
// doubled registers leave one CTA per SM.
constexpr int kDotChunk = 8192;
constexpr int kDotThreads = 256;
constexpr int kDotVec = kDotChunk / 4 / kDotThreads;  // 8 float4 per thread

// Several layers in one launch: CTA (layer, row, chunk) reads phi from layer l's
// block (phi + l * layer_stride) and tau[l], and adds alphas[l] (a device array,
// or `alpha` when null) times its partial dot to score[row].
__global__ void __launch_bounds__(kDotThreads) sketch_dot_kernel(const float* __restrict__ phi,
                                                                 const float* __restrict__ tau_all, int64_t k,
                                                                 int n_chunks, float alpha, float* __restrict__ score,
                                                                 int n_rows, int64_t layer_stride,
                                                                 const float* __restrict__ alphas) {
  const int64_t per_layer = (int64_t)n_rows * n_chunks;
  const int64_t layer = blockIdx.x / per_layer;
  const int64_t in_layer = blockIdx.x % per_layer;
  const int64_t row = in_layer / n_chunks;
  const int64_t c0 = (int64_t)(in_layer % n_chunks) * kDotChunk;
  const int64_t c1 = min(k, c0 + kDotChunk);
  const float* p = phi + layer * layer_stride + row * k;
  const float* tau = tau_all + layer * k;
  if (alphas != nullptr) alpha = alphas[layer];
  float acc = 0.0f;
  if ((k & 3) == 0) {
    const float4* p4 = reinterpret_cast<const float4*>(p);
    const float4* t4 = reinterpret_cast<const float4*>(tau);
    float4 a[kDotVec], b[kDotVec];
#pragma unroll
    for (int j = 0; j < kDotVec; ++j) {
      const int64_t i = c0 / 4 + threadIdx.x + (int64_t)j * kDotThreads;
      const bool in = i < c1 / 4;
      a[j] = in ? __ldcs(p4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      b[j] = in ? __ldg(t4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int j = 0; j < kDotVec; ++j) {
      acc = fmaf(a[j].x, b[j].x, acc);
      acc = fmaf(a[j].y, b[j].y, acc);
      acc = fmaf(a[j].z, b[j].z, acc);
      acc = fmaf(a[j].w, b[j].w, acc);
    }
  } else {
    for (int64_t i = c0 + threadIdx.x; i < c1; i += kDotThreads) acc = fmaf(p[i], tau[i], acc);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  __shared__ float part[kDotThreads / 32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int i = 0; i < kDotThreads / 32; ++i) t += part[i];
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

int launch_dense(const float* w, int transposed, const uint32_t* packed, const float* diag, int d_out, int d_in,
                 int row_begin, int row_end, int64_t k, int max_load, float* sketch, int n_vec, int64_t w_stride,
                 int64_t out_stride, cudaStream_t st) {
  const int64_t numel = (int64_t)(row_end - row_begin) * d_in;
  if (numel == 0 || n_vec == 0) return OPUS_OK;
  // shared-memory sketch: all k buckets when they fit, else the largest prefix (a multiple of 1024)
  const size_t staging = transposed ? sizeof(float) * kDenseGroup * kDenseTile * (kDenseTile + 1) : 0;
  const size_t fixed = staging + 32 * sizeof(float) + 1024;
  const size_t limit = static_cast<size_t>(max_smem_optin());
  int64_t k_sm = k;
  if (fixed + (size_t)k * 4 > limit) k_sm = static_cast<int64_t>((limit - fixed) / 4) & ~int64_t(1023);
  const size_t smem = (size_t)k_sm * 4;
  // one CTA per SM (1024 threads of about 50 registers fill the register file), and at least ~k elements per
  // CTA, so the flushes (k_sm floats each) stay below the element updates
  int64_t grid = numel / (k > 4096 ? k : 4096);
  if (grid > (int64_t)sm_count()) grid = sm_count();
  if (grid < 1) grid = 1;
  if (transposed) {
    OPUS_CUDA_TRY(cudaFuncSetAttribute(dense_sketch_tiles_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem)));
    const int64_t n_tiles =
        (int64_t)((row_end - row_begin + kDenseTile - 1) / kDenseTile) * ((d_in + kDenseTile - 1) / kDenseTile);
    if (grid > n_tiles) grid = n_tiles;
    dense_sketch_tiles_kernel<<<(int)grid, kDenseSmemThreads, smem, st>>>(w, packed, diag, d_out, d_in, row_begin,
                                                                         row_end, static_cast<int>(k),
                                                                         static_cast<int>(k_sm), max_load, sketch);
    ::opus::note_launch();
  } else {
    const int64_t e0 = (int64_t)row_begin * d_in, e1 = (int64_t)row_end * d_in;
    const uintptr_t al = reinterpret_cast<uintptr_t>(w + e0) | reinterpret_cast<uintptr_t>(packed + e0) |
                         (diag ? reinterpret_cast<uintptr_t>(diag + e0) : 0) | (uintptr_t)(w_stride * 4);
    const int vec = (al & 15) == 0;
    OPUS_CUDA_TRY(cudaFuncSetAttribute(dense_sketch_flat_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem)));
    const dim3 g((unsigned)grid, (unsigned)n_vec);
    dense_sketch_flat_kernel<<<g, kDenseSmemThreads, smem, st>>>(w, packed, diag, e0, e1, static_cast<int>(k),
                                                                 static_cast<int>(k_sm), max_load, sketch,
                                                                 w_stride, out_stride, vec);
    ::opus::note_launch();
  }
  OPUS_CUDA_TRY(cudaGetLastError());
  return OPUS_OK;
}

}  // namespace
}  // namespace opus

using namespace opus;

extern "C" {

int opus_sketch_dense(const float* w, int transposed, const uint32_t* packed, const float* diag, int d_out, int d_in,
                      int row_begin, int row_end, int64_t k, int max_bucket_load, float* sketch, int accumulate,
                      void* stream) {
  if (d_out <= 0 || d_in <= 0 || k <= 0 || k > 0x7FFFFFFF) return set_error(OPUS_ERR_INVALID, "sketch_dense: bad sizes");
  if (row_begin < 0 || row_end > d_out || row_begin > row_end)
    return set_error(OPUS_ERR_INVALID, "sketch_dense: rows [%d, %d) outside [0, %d)", row_begin, row_end, d_out);
  if (!w || !packed || !sketch) return set_error(OPUS_ERR_INVALID, "sketch_dense: NULL pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (!accumulate) OPUS_CUDA_TRY(cudaMemsetAsync(sketch, 0, (size_t)k * sizeof(float), st));
  return launch_dense(w, transposed, packed, diag, d_out, d_in, row_begin, row_end, k, max_bucket_load, sketch, 1, 0,
                      0, st);
}

int opus_sketch_dense_rows(const float* w, int n_vec, int64_t numel, const uint32_t* packed, int64_t k,
                           int max_bucket_load, float* sketches, int accumulate, void* stream) {
  if (n_vec < 0 || numel <= 0 || numel > 0x7FFFFFFF || k <= 0 || k > 0x7FFFFFFF || n_vec > 65535)
    return set_error(OPUS_ERR_INVALID, "sketch_dense_rows: bad sizes (n_vec=%d numel=%lld k=%lld)", n_vec,
                     (long long)numel, (long long)k);
  if (n_vec == 0) return OPUS_OK;
  if (!w || !packed || !sketches) return set_error(OPUS_ERR_INVALID, "sketch_dense_rows: NULL pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (!accumulate) OPUS_CUDA_TRY(cudaMemsetAsync(sketches, 0, (size_t)n_vec * k * sizeof(float), st));
  return launch_dense(w, 0, packed, nullptr, 1, static_cast<int>(numel), 0, 1, k, max_bucket_load, sketches, n_vec,
                      numel, k, st);
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
  sketch_dot_kernel<<<(int)grid, kDotThreads, 0, st>>>(phi, tau, k, (int)n_chunks, alpha, score, n_rows, 0,
                                                         nullptr);
  ::opus::note_launch();
  OPUS_CUDA_TRY(cudaGetLastError());
  return OPUS_OK;
}

int opus_sketch_dot_layers(const float* phi, int64_t layer_stride, const float* tau, const float* alphas,
                           int n_layers, int n_rows, int64_t k, float* score, int accumulate, void* stream) {
  if (n_rows < 0 || n_layers < 0 || k <= 0 || layer_stride < (int64_t)n_rows * k)
    return set_error(OPUS_ERR_INVALID, "sketch_dot_layers: bad sizes");
  if (n_rows == 0) return OPUS_OK;
  if (!score || (n_layers > 0 && (!phi || !tau || !alphas)))
    return set_error(OPUS_ERR_INVALID, "sketch_dot_layers: NULL pointer");
  if ((k & 3) == 0 && (((reinterpret_cast<uintptr_t>(phi) | reinterpret_cast<uintptr_t>(tau)) & 15) != 0 ||
                       (layer_stride & 3) != 0))
    return set_error(OPUS_ERR_INVALID, "sketch_dot_layers: phi, tau and the layer stride must be 16-byte aligned");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (!accumulate) OPUS_CUDA_TRY(cudaMemsetAsync(score, 0, (size_t)n_rows * sizeof(float), st));
  if (n_layers == 0) return OPUS_OK;
  const int64_t n_chunks = (k + kDotChunk - 1) / kDotChunk;
  const int64_t grid = (int64_t)n_layers * n_rows * n_chunks;
  if (grid > 0x7fffffff) return set_error(OPUS_ERR_UNSUPPORTED, "sketch_dot_layers: too many rows");
  sketch_dot_kernel<<<(int)grid, kDotThreads, 0, st>>>(phi, tau, k, (int)n_chunks, 1.0f, score, n_rows,
                                                         layer_stride, alphas);
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
