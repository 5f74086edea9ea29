// Stage 5: Boltzmann (softmax-temperature) and greedy selection with the
// interaction penalty, each on one 1024-thread CTA with the scores held in
// shared memory.  The float32 / float64 operation order follows numpy so the
// same uniforms give the same indices as the host implementation:
//   - scaled = score / T in float32, shifted by its max only if max > 700;
//   - p = exp(scaled) rounded to float32 (computed in double);
//   - sum = numpy's pairwise float32 sum (0 + blocks of <=128 with 8
//     accumulators, halves rounded down to a multiple of 8);
//   - p /= sum in float32, or 1/m when the sum is 0 or not finite;
//   - cdf = float64 running sum, cdf /= cdf[-1], idx = #{cdf <= u}.
// The float64 running sum is evaluated exactly with an int64 scan whenever
// every p is a multiple of 2^-52 (then no partial sum rounds); otherwise one
// thread runs the sequential float64 recurrence.
#include "opus_common.cuh"

namespace opus {
namespace {

constexpr int kSelThreads = 1024;
constexpr int kSelMax = 8192;
constexpr int kPwBlock = 128;
constexpr int kMaxLeaves = 256;

struct SelShared {
  double cdf[kSelMax];
  float scores[kSelMax];
  float pc[kSelMax];
  int pidx[kSelMax];
  unsigned char avail[kSelMax];
  int leaf_start[kMaxLeaves];
  int leaf_len[kMaxLeaves];
  float leaf_sum[kMaxLeaves];
  long long scan_ll[kSelThreads / 32];
  double red_d[kSelThreads / 32];
  int red_i[kSelThreads / 32];
  float red_f[kSelThreads / 32];
  int n_leaves;
  int m;
  float smax;
  int any_nan;
  float total;
  int not_exact;
  double cdf_total;
  int pick;
};

// ---- numpy pairwise float32 sum
__device__ float pw_leaf(const float* a, int n) {
  if (n < 8) {
    float res = 0.0f;
    for (int i = 0; i < n; ++i) res = __fadd_rn(res, a[i]);
    return res;
  }
  float r[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) r[j] = a[j];
  int i = 8;
  for (; i < n - (n % 8); i += 8) {
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = __fadd_rn(r[j], a[i + j]);
  }
  float res = __fadd_rn(__fadd_rn(__fadd_rn(r[0], r[1]), __fadd_rn(r[2], r[3])),
                        __fadd_rn(__fadd_rn(r[4], r[5]), __fadd_rn(r[6], r[7])));
  for (; i < n; ++i) res = __fadd_rn(res, a[i]);
  return res;
}

__device__ void pw_enumerate(int a, int n, SelShared& s) {
  if (n <= kPwBlock) {
    s.leaf_start[s.n_leaves] = a;
    s.leaf_len[s.n_leaves] = n;
    s.n_leaves++;
    return;
  }
  int n2 = n / 2;
  n2 -= n2 % 8;
  pw_enumerate(a, n2, s);
  pw_enumerate(a + n2, n - n2, s);
}

__device__ float pw_combine(int n, const SelShared& s, int& leaf) {
  if (n <= kPwBlock) return s.leaf_sum[leaf++];
  int n2 = n / 2;
  n2 -= n2 % 8;
  const float l = pw_combine(n2, s, leaf);
  const float r = pw_combine(n - n2, s, leaf);
  return __fadd_rn(l, r);
}

// ---- block helpers (1024 threads = 32 warps)
__device__ long long block_excl_scan_ll(long long v, SelShared& s, long long* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  long long x = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const long long y = __shfl_up_sync(0xffffffffu, x, off);
    if (lane >= off) x += y;
  }
  if (lane == 31) s.scan_ll[warp] = x;
  __syncthreads();
  if (warp == 0) {
    long long w = s.scan_ll[lane];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, w, off);
      if (lane >= off) w += y;
    }
    s.scan_ll[lane] = w;  // inclusive per-warp totals
  }
  __syncthreads();
  const long long before = (warp > 0 ? s.scan_ll[warp - 1] : 0) + (x - v);
  if (total) *total = s.scan_ll[31];
  __syncthreads();
  return before;
}

__device__ int block_sum_i(int v, SelShared& s) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  if (lane == 0) s.red_i[warp] = v;
  __syncthreads();
  int t = 0;
  for (int i = 0; i < 32; ++i) t += s.red_i[i];
  __syncthreads();
  return t;
}

__device__ double block_sum_d(double v, SelShared& s) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  if (lane == 0) s.red_d[warp] = v;
  __syncthreads();
  double t = 0.0;
  for (int i = 0; i < 32; ++i) t += s.red_d[i];
  __syncthreads();
  return t;
}

__global__ void __launch_bounds__(kSelThreads, 1)
    boltzmann_kernel(const float* __restrict__ scores_in, const float* __restrict__ sim, int n, int n_select,
                     float temp, const double* __restrict__ uniforms, int64_t* __restrict__ out_idx, int* err) {
  extern __shared__ __align__(16) uint8_t sel_smem[];
  SelShared& s = *reinterpret_cast<SelShared*>(sel_smem);
  const int tid = threadIdx.x;
  for (int i = tid; i < n; i += kSelThreads) {
    s.scores[i] = scores_in[i];
    s.avail[i] = 1;
  }
  __syncthreads();
  const int per = (n + kSelThreads - 1) / kSelThreads;
  const int lo = min(n, tid * per), hi = min(n, lo + per);

  for (int r = 0; r < n_select; ++r) {
    // (1) compact available scores, scaled by 1/T in float32
    int cnt = 0;
    for (int i = lo; i < hi; ++i) cnt += s.avail[i];
    long long m_ll = 0;
    int pos = static_cast<int>(block_excl_scan_ll(cnt, s, &m_ll));
    const int m = static_cast<int>(m_ll);
    for (int i = lo; i < hi; ++i) {
      if (s.avail[i]) {
        s.pc[pos] = __fdiv_rn(s.scores[i], temp);
        s.pidx[pos] = i;
        ++pos;
      }
    }
    __syncthreads();
    // (2) max over scaled values (NaN anywhere -> np.max is NaN -> no shift)
    float lmax = -INFINITY;
    int lnan = 0;
    for (int i = tid; i < m; i += kSelThreads) {
      const float x = s.pc[i];
      if (isnan(x)) lnan = 1; else lmax = fmaxf(lmax, x);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, off));
      lnan |= __shfl_xor_sync(0xffffffffu, lnan, off);
    }
    if ((tid & 31) == 0) {
      s.red_f[tid >> 5] = lmax;
      s.red_i[tid >> 5] = lnan;
    }
    __syncthreads();
    if (tid == 0) {
      float mx = -INFINITY;
      int nn = 0;
      for (int i = 0; i < 32; ++i) {
        mx = fmaxf(mx, s.red_f[i]);
        nn |= s.red_i[i];
      }
      s.smax = mx;
      s.any_nan = nn;
      s.n_leaves = 0;
      pw_enumerate(0, m, s);
    }
    __syncthreads();
    const bool shift = !s.any_nan && s.smax > 700.0f;
    const float smax = s.smax;
    // (3) p = exp(scaled) in float32
    for (int i = tid; i < m; i += kSelThreads) {
      float x = s.pc[i];
      if (shift) x = __fsub_rn(x, smax);
      s.pc[i] = static_cast<float>(exp(static_cast<double>(x)));
    }
    __syncthreads();
    // (4) numpy pairwise sum: leaves in parallel, tree combine on one thread
    if (tid < s.n_leaves) s.leaf_sum[tid] = pw_leaf(s.pc + s.leaf_start[tid], s.leaf_len[tid]);
    __syncthreads();
    if (tid == 0) {
      int leaf = 0;
      s.total = __fadd_rn(0.0f, pw_combine(m, s, leaf));
    }
    __syncthreads();
    const float total = s.total;
    const bool uniform = (total == 0.0f) || !isfinite(total);
    const float inv_m = __fdiv_rn(1.0f, static_cast<float>(m));
    // (5) normalise (contiguous ownership of compacted positions from here on)
    const int pm = (m + kSelThreads - 1) / kSelThreads;
    const int plo = min(m, tid * pm), phi_ = min(m, plo + pm);
    int not_exact = 0;
    long long fixed_sum = 0;
    double dsum = 0.0;
    for (int i = plo; i < phi_; ++i) {
      const float p = uniform ? inv_m : __fdiv_rn(s.pc[i], total);
      s.pc[i] = p;
      const double x = static_cast<double>(p) * 0x1p52;
      if (x != trunc(x)) not_exact = 1;
      fixed_sum += static_cast<long long>(x);
      dsum += static_cast<double>(p);
    }
    not_exact = block_sum_i(not_exact, s);
    const double psum = block_sum_d(dsum, s);
    // np.random.choice rejects p whose sum is off by more than sqrt(eps_f32).
    if (tid == 0 && fabs(psum - 1.0) > 3.4526698300124393e-04) record_device_error(err, 0x301);
    const double u = uniforms[r];
    int below = 0;
    if (!not_exact) {
      long long tot = 0;
      long long run = block_excl_scan_ll(fixed_sum, s, &tot);
      const double cdf_last = static_cast<double>(tot) * 0x1p-52;
      for (int i = plo; i < phi_; ++i) {
        run += static_cast<long long>(static_cast<double>(s.pc[i]) * 0x1p52);
        const double c = __ddiv_rn(static_cast<double>(run) * 0x1p-52, cdf_last);
        below += (c <= u) ? 1 : 0;
      }
    } else {
      if (tid == 0) {
        double acc = 0.0;
        for (int i = 0; i < m; ++i) {
          acc = __dadd_rn(acc, static_cast<double>(s.pc[i]));
          s.cdf[i] = acc;
        }
        s.cdf_total = acc;
      }
      __syncthreads();
      const double cdf_last = s.cdf_total;
      for (int i = plo; i < phi_; ++i) below += (__ddiv_rn(s.cdf[i], cdf_last) <= u) ? 1 : 0;
    }
    const int idx = block_sum_i(below, s);
    const int sel = s.pidx[idx < m ? idx : m - 1];
    if (tid == 0) out_idx[r] = sel;
    // (6) interaction penalty on every score (float32), retire the pick
    const float* row = sim + (int64_t)sel * n;
    for (int i = tid; i < n; i += kSelThreads) s.scores[i] = __fsub_rn(s.scores[i], row[i]);
    __syncthreads();
    if (tid == 0) s.avail[sel] = 0;
    __syncthreads();
  }
}

// np.argmax order: the first NaN if any, else the first maximum.
struct ArgMax {
  float v;
  int i;
};
__device__ __forceinline__ ArgMax better(ArgMax a, ArgMax b) {
  const bool an = isnan(a.v), bn = isnan(b.v);
  if (an || bn) {
    if (an && bn) return a.i < b.i ? a : b;
    return an ? a : b;
  }
  if (a.v > b.v) return a;
  if (b.v > a.v) return b;
  return a.i < b.i ? a : b;
}

__global__ void __launch_bounds__(kSelThreads, 1)
    greedy_kernel(const float* __restrict__ scores_in, const float* __restrict__ sim, int n, int n_select,
                  int64_t* __restrict__ out_idx) {
  extern __shared__ __align__(16) uint8_t sel_smem[];
  float* scores = reinterpret_cast<float*>(sel_smem);
  __shared__ float rv[32];
  __shared__ int ri[32];
  __shared__ int pick;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < n; i += kSelThreads) scores[i] = scores_in[i];
  __syncthreads();
  const int per = (n + kSelThreads - 1) / kSelThreads;
  const int lo = min(n, tid * per), hi = min(n, lo + per);
  for (int r = 0; r < n_select; ++r) {
    ArgMax best{-INFINITY, 0x7fffffff};
    for (int i = lo; i < hi; ++i) best = better(best, ArgMax{scores[i], i});
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      ArgMax o;
      o.v = __shfl_xor_sync(0xffffffffu, best.v, off);
      o.i = __shfl_xor_sync(0xffffffffu, best.i, off);
      best = better(best, o);
    }
    if (lane == 0) {
      rv[warp] = best.v;
      ri[warp] = best.i;
    }
    __syncthreads();
    if (tid == 0) {
      ArgMax b{rv[0], ri[0]};
      for (int w = 1; w < 32; ++w) b = better(b, ArgMax{rv[w], ri[w]});
      // all entries -inf: np.argmax returns 0
      pick = (b.i == 0x7fffffff) ? 0 : b.i;
      out_idx[r] = pick;
    }
    __syncthreads();
    const int sel = pick;
    const float* row = sim + (int64_t)sel * n;
    for (int i = tid; i < n; i += kSelThreads) scores[i] = __fsub_rn(scores[i], row[i]);
    __syncthreads();
    if (tid == 0) scores[sel] = -INFINITY;
    __syncthreads();
  }
}

}  // namespace
}  // namespace opus

using namespace opus;

extern "C" {

int opus_boltzmann_select(const float* scores, const float* sim, int n, int n_select, double temperature,
                          const double* uniforms, int64_t* out_idx, void* stream) {
  if (n <= 0 || n > kSelMax) return set_error(OPUS_ERR_UNSUPPORTED, "boltzmann: n=%d outside [1, %d]", n, kSelMax);
  if (n_select < 0 || n_select > n)
    return set_error(OPUS_ERR_INVALID, "boltzmann: cannot select %d of %d candidates", n_select, n);
  if (n_select == 0) return OPUS_OK;
  if (!scores || !sim || !uniforms || !out_idx) return set_error(OPUS_ERR_INVALID, "boltzmann: NULL pointer");
  const size_t smem = sizeof(SelShared);
  OPUS_CUDA_TRY(cudaFuncSetAttribute(boltzmann_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  boltzmann_kernel<<<1, kSelThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
      scores, sim, n, n_select, static_cast<float>(temperature), uniforms, out_idx, device_error_word());
  OPUS_CUDA_TRY(cudaGetLastError());
  return OPUS_OK;
}

int opus_greedy_select(const float* scores, const float* sim, int n, int n_select, int64_t* out_idx, void* stream) {
  if (n <= 0 || n > 4 * kSelMax) return set_error(OPUS_ERR_UNSUPPORTED, "greedy: n=%d outside [1, %d]", n, 4 * kSelMax);
  if (n_select < 0) return set_error(OPUS_ERR_INVALID, "greedy: negative n_select");
  if (n_select == 0) return OPUS_OK;
  if (!scores || !sim || !out_idx) return set_error(OPUS_ERR_INVALID, "greedy: NULL pointer");
  const size_t smem = (size_t)n * sizeof(float);
  if (smem > 48 * 1024)
    OPUS_CUDA_TRY(cudaFuncSetAttribute(greedy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  greedy_kernel<<<1, kSelThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(scores, sim, n, n_select, out_idx);
  OPUS_CUDA_TRY(cudaGetLastError());
  return OPUS_OK;
}

}  // extern "C"
