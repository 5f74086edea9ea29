// Stage 5: Boltzmann (softmax-temperature) and greedy selection with the
// interaction penalty on one CTA with the scores held in shared memory (128
// to 1024 threads, chosen by the candidate count).  The float32 / float64
// operation order follows numpy so the same uniforms give the same indices as
// the host implementation:
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

// Thread t owns the contiguous original indices [t*per, (t+1)*per), so the
// compacted (available-only) order is thread order and then index order
// inside a thread.  Each owned element keeps its compacted position, which
// only moves down by one when an earlier element is picked.
template <int NT>
__global__ void __launch_bounds__(NT, 1)
    boltzmann_kernel(const float* __restrict__ scores_in, const float* __restrict__ sim, int n, int n_select,
                     float temp, const double* __restrict__ uniforms, int64_t* __restrict__ out_idx, int* err) {
  constexpr int W = NT / 32;
  extern __shared__ __align__(16) uint8_t sel_smem[];
  SelShared& s = *reinterpret_cast<SelShared*>(sel_smem);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (n + NT - 1) / NT;
  const int lo = min(n, tid * per), hi = min(n, lo + per);
  for (int i = tid; i < n; i += NT) {
    s.scores[i] = scores_in[i];
    s.avail[i] = 1;
    s.pidx[i] = i;         // compacted position -> original index (rewritten as picks retire)
  }
  __syncthreads();
  int m = n;               // available candidates

  for (int r = 0; r < n_select; ++r) {
    const double u = uniforms[r];
    // (1) scaled scores of this thread's available elements, their max and
    //     count; the exp lands at the compacted positions after barrier 2
    int cnt = 0;
    for (int i = lo; i < hi; ++i) cnt += s.avail[i];
    float lmax = -INFINITY;
    int lnan = 0;
    for (int i = lo; i < hi; ++i) {
      if (!s.avail[i]) continue;
      const float x = __fdiv_rn(s.scores[i], temp);
      s.cdf[i] = x;  // exp is taken after the max is known (shift above 700)
      if (isnan(x)) lnan = 1; else lmax = fmaxf(lmax, x);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, off));
      lnan |= __shfl_xor_sync(0xffffffffu, lnan, off);
    }
    // compacted base of this thread = exclusive prefix of the per-thread counts
    int wx = cnt;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, wx, off);
      if (lane >= off) wx += y;
    }
    if (lane == 31) s.red_i[warp] = wx;
    if (lane == 0) {
      s.red_f[warp] = lmax;
      s.scan_ll[warp] = lnan;
    }
    __syncthreads();                                                   // barrier 1
    int base = wx - cnt;
    for (int w = 0; w < warp; ++w) base += s.red_i[w];
    if (tid == 0) {
      float mx = -INFINITY;
      int nn = 0;
      for (int w = 0; w < W; ++w) {
        mx = fmaxf(mx, s.red_f[w]);
        nn |= static_cast<int>(s.scan_ll[w]);
      }
      s.smax = mx;
      s.any_nan = nn;
      s.n_leaves = 0;
      pw_enumerate(0, m, s);
    }
    __syncthreads();                                                   // barrier 2
    const bool do_shift = !s.any_nan && s.smax > 700.0f;
    const float smax = s.smax;
    {
      int pos = base;
      for (int i = lo; i < hi; ++i) {
        if (!s.avail[i]) continue;
        float x = static_cast<float>(s.cdf[i]);
        if (do_shift) x = __fsub_rn(x, smax);
        s.pc[pos] = static_cast<float>(exp(static_cast<double>(x)));
        s.pidx[pos] = i;
        ++pos;
      }
    }
    __syncthreads();                                                   // barrier 3
    // (2) numpy pairwise sum: leaves of <= 128, 8 lanes each (lane j holds
    //     accumulator r[j]; ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)), then the
    //     tail; shorter leaves are a running sum), tree combine on thread 0
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
    __syncthreads();                                                   // barrier 4
    if (tid == 0) {
      int leaf = 0;
      s.total = __fadd_rn(0.0f, n_leaves == 1 ? s.leaf_sum[0] : pw_combine(m, s, leaf));
      s.pick = 0;
    }
    __syncthreads();                                                   // barrier 5
    const float total = s.total;
    const bool uniform = (total == 0.0f) || !isfinite(total);
    const float inv_m = __fdiv_rn(1.0f, static_cast<float>(m));
    // (3) normalise this thread's compacted range [base, base + cnt); exact
    //     int64 running sum when every p is a multiple of 2^-52
    int not_exact = 0;
    long long fsum = 0;
    double dsum = 0.0;
    for (int i = base; i < base + cnt; ++i) {
      const float p = uniform ? inv_m : __fdiv_rn(s.pc[i], total);
      s.pc[i] = p;
      const double x = static_cast<double>(p) * 0x1p52;
      if (x != trunc(x)) not_exact = 1;
      fsum += static_cast<long long>(x);
      dsum += static_cast<double>(p);
    }
    long long fx = fsum;
    double dx = dsum;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, fx, off);
      if (lane >= off) fx += y;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      dx += __shfl_xor_sync(0xffffffffu, dx, off);
      not_exact |= __shfl_xor_sync(0xffffffffu, not_exact, off);
    }
    if (lane == 31) s.scan_ll[warp] = fx;
    if (lane == 0) {
      s.red_d[warp] = dx;
      s.red_i[warp] = not_exact;
    }
    __syncthreads();                                                   // barrier 6
    long long fbase = fx - fsum;
    long long ftot = 0;
    double psum = 0.0;
    int ne = 0;
    for (int w = 0; w < W; ++w) {
      if (w < warp) fbase += s.scan_ll[w];
      ftot += s.scan_ll[w];
      psum += s.red_d[w];
      ne |= s.red_i[w];
    }
    // np.random.choice rejects p whose sum is off by more than sqrt(eps_f32).
    if (tid == 0 && fabs(psum - 1.0) > 3.4526698300124393e-04) record_device_error(err, 0x301);
    int below = 0;
    if (!ne) {
      const double cdf_last = static_cast<double>(ftot) * 0x1p-52;
      long long run = fbase;
      for (int i = base; i < base + cnt; ++i) {
        run += static_cast<long long>(static_cast<double>(s.pc[i]) * 0x1p52);
        below += (__ddiv_rn(static_cast<double>(run) * 0x1p-52, cdf_last) <= u) ? 1 : 0;
      }
    } else {
      if (tid == 0) {
        double acc = 0.0;
        for (int i = 0; i < m; ++i) {
          acc = __dadd_rn(acc, static_cast<double>(s.pc[i]));
          s.cdf[i] = acc;   // scaled scores are no longer needed in this draw
        }
        s.cdf_total = acc;
      }
      __syncthreads();
      const double cdf_last = s.cdf_total;
      for (int i = base; i < base + cnt; ++i) below += (__ddiv_rn(s.cdf[i], cdf_last) <= u) ? 1 : 0;
    }
    // (4) searchsorted(side='right') = number of cdf entries <= u
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) below += __shfl_xor_sync(0xffffffffu, below, off);
    if (lane == 0 && below) atomicAdd(&s.pick, below);
    __syncthreads();                                                   // barrier 7
    const int idx = min(s.pick, m - 1);
    const int sel = s.pidx[idx];
    if (tid == 0) out_idx[r] = sel;
    // (5) interaction penalty on every score (float32), retire the pick
    const float* row = sim + (int64_t)sel * n;
    for (int i = tid; i < n; i += NT) s.scores[i] = __fsub_rn(s.scores[i], row[i]);
    if (tid == 0) s.avail[sel] = 0;
    --m;
    __syncthreads();                                                   // barrier 8
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
