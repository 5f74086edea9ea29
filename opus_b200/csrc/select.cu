// Stage 5: Boltzmann (softmax-temperature) and greedy selection with the
// interaction penalty on one CTA with the scores held in shared memory (one
// warp for up to 4096 candidates, 1024 threads above).  The float32 / float64 operation order follows numpy so the
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
  long long scan_ll[32];
  double red_d[32];
  int red_i[32];
  float red_f[32];
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

// ---- block helpers (NT threads = NT/32 warps, NT a power of two in [64, 1024])
template <int NT>
__device__ long long block_excl_scan_ll(long long v, SelShared& s, long long* total) {
  constexpr int W = NT / 32;
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
    long long w = lane < W ? s.scan_ll[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, w, off);
      if (lane >= off) w += y;
    }
    if (lane < W) s.scan_ll[lane] = w;  // inclusive per-warp totals
  }
  __syncthreads();
  const long long before = (warp > 0 ? s.scan_ll[warp - 1] : 0) + (x - v);
  if (total) *total = s.scan_ll[W - 1];
  __syncthreads();
  return before;
}

// Sum of an int and a double over the block in one barrier pair.
template <int NT>
__device__ void block_sum_id(int& vi, double& vd, SelShared& s) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    vi += __shfl_xor_sync(0xffffffffu, vi, off);
    vd += __shfl_xor_sync(0xffffffffu, vd, off);
  }
  if (lane == 0) {
    s.red_i[warp] = vi;
    s.red_d[warp] = vd;
  }
  __syncthreads();
  int ti = 0;
  double td = 0.0;
  for (int i = 0; i < NT / 32; ++i) {
    ti += s.red_i[i];
    td += s.red_d[i];
  }
  __syncthreads();
  vi = ti;
  vd = td;
}

template <int NT>
__global__ void __launch_bounds__(NT, 1)
    boltzmann_kernel(const float* __restrict__ scores_in, const float* __restrict__ sim, int n, int n_select,
                     float temp, const double* __restrict__ uniforms, int64_t* __restrict__ out_idx, int* err) {
  constexpr int kSelThreads = NT;
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
    const double u = uniforms[r];
    // (1) compact available scores scaled by 1/T (float32) and take their exp
    //     (no shift: the max only matters above 700, handled below)
    int cnt = 0;
    for (int i = lo; i < hi; ++i) cnt += s.avail[i];
    long long m_ll = 0;
    const int base = static_cast<int>(block_excl_scan_ll<NT>(cnt, s, &m_ll));
    const int m = static_cast<int>(m_ll);
    float lmax = -INFINITY;
    int lnan = 0;
    {
      int pos = base;
      for (int i = lo; i < hi; ++i) {
        if (s.avail[i]) {
          const float x = __fdiv_rn(s.scores[i], temp);
          s.cdf[pos] = x;   // scaled score, kept for the rare shifted recomputation
          s.pc[pos] = static_cast<float>(exp(static_cast<double>(x)));
          s.pidx[pos] = i;
          ++pos;
          if (isnan(x)) lnan = 1; else lmax = fmaxf(lmax, x);
        }
      }
    }
    // (2) max over scaled values (NaN anywhere -> np.max is NaN -> no shift)
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
      for (int i = 0; i < NT / 32; ++i) {
        mx = fmaxf(mx, s.red_f[i]);
        nn |= s.red_i[i];
      }
      s.smax = mx;
      s.any_nan = nn;
      s.n_leaves = 0;
      pw_enumerate(0, m, s);
    }
    __syncthreads();
    if (!s.any_nan && s.smax > 700.0f) {
      // (3') x - max in float32 before the exp, as the reference does above 700
      const float smax = s.smax;
      for (int i = base; i < base + cnt; ++i)
        s.pc[i] = static_cast<float>(exp(static_cast<double>(__fsub_rn(static_cast<float>(s.cdf[i]), smax))));
      __syncthreads();
    }
    // (4) numpy pairwise sum: leaves of <= 128 with 8 lanes each (lane j holds
    //     accumulator r[j]; ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)), then the tail;
    //     shorter leaves are a plain running sum), tree combine on one thread
    const int n_leaves = s.n_leaves;
    for (int l0 = 0; l0 < n_leaves; l0 += NT / 8) {
      const int leaf = l0 + (tid >> 3), j = tid & 7;
      const bool active = leaf < n_leaves;
      const int a0 = active ? s.leaf_start[leaf] : 0;
      const int ln = active ? s.leaf_len[leaf] : 0;
      const int full = ln >= 8 ? ln - (ln % 8) : 0;
      float acc = 0.0f;
      if (full >= 8) {
        acc = s.pc[a0 + j];
        for (int i = 8; i < full; i += 8) acc = __fadd_rn(acc, s.pc[a0 + i + j]);
      }
      const float p01 = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
      const float p03 = __fadd_rn(p01, __shfl_xor_sync(0xffffffffu, p01, 2));
      const float p07 = __fadd_rn(p03, __shfl_xor_sync(0xffffffffu, p03, 4));
      if (active && j == 0) {
        float res = full >= 8 ? p07 : 0.0f;
        for (int i = full; i < ln; ++i) res = __fadd_rn(res, s.pc[a0 + i]);
        s.leaf_sum[leaf] = res;
      }
    }
    __syncthreads();
    if (tid == 0) {
      int leaf = 0;
      s.total = __fadd_rn(0.0f, pw_combine(m, s, leaf));
    }
    __syncthreads();
    const float total = s.total;
    const bool uniform = (total == 0.0f) || !isfinite(total);
    const float inv_m = __fdiv_rn(1.0f, static_cast<float>(m));
    // (5) normalise (each thread its own compacted range [base, base + cnt))
    const int plo = base, phi_ = base + cnt;
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
    block_sum_id<NT>(not_exact, dsum, s);
    const double psum = dsum;
    // np.random.choice rejects p whose sum is off by more than sqrt(eps_f32).
    if (tid == 0 && fabs(psum - 1.0) > 3.4526698300124393e-04) record_device_error(err, 0x301);
    int below = 0;
    if (!not_exact) {
      long long tot = 0;
      long long run = block_excl_scan_ll<NT>(fixed_sum, s, &tot);
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
    double unused = 0.0;
    block_sum_id<NT>(below, unused, s);
    const int idx = below;
    const int sel = s.pidx[idx < m ? idx : m - 1];
    if (tid == 0) out_idx[r] = sel;
    // (6) interaction penalty on every score (float32), retire the pick
    const float* row = sim + (int64_t)sel * n;
    for (int i = tid; i < n; i += kSelThreads) s.scores[i] = __fsub_rn(s.scores[i], row[i]);
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
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const float tf = static_cast<float>(temperature);
  int* err = device_error_word();
  // one candidate per thread up to 1024 candidates, then 1024 threads
#define OPUS_LAUNCH_BOLTZMANN(NT)                                                                              \
  OPUS_CUDA_TRY(cudaFuncSetAttribute(boltzmann_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
  boltzmann_kernel<NT><<<1, NT, smem, st>>>(scores, sim, n, n_select, tf, uniforms, out_idx, err)
  if (n <= 128) {
    OPUS_LAUNCH_BOLTZMANN(128);
  } else if (n <= 256) {
    OPUS_LAUNCH_BOLTZMANN(256);
  } else if (n <= 512) {
    OPUS_LAUNCH_BOLTZMANN(512);
  } else {
    OPUS_LAUNCH_BOLTZMANN(1024);
  }
#undef OPUS_LAUNCH_BOLTZMANN
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
