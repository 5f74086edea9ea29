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
// every p is a multiple of 2^-52 (then no partial sum rounds), and the
// division by cdf[-1] with the comparison against u becomes one integer
// threshold per draw; otherwise one thread runs the sequential float64
// recurrence and every element is divided.
#include "opus_common.cuh"

namespace opus {
namespace {

constexpr int kSelThreads = 1024;
constexpr int kSelMax = 8192;
constexpr int kPwBlock = 128;
// numpy splits a length-m sum at m/2 rounded down to a multiple of 8 until a
// piece is <= 128 long; for m <= 8192 the pieces at depth 7 are <= 79 long,
// so the split tree has at most 8 levels of at most 128 nodes.
constexpr int kLevels = 8;
constexpr int kLevelSlots = 128;

struct SelShared {
  double cdf[kSelMax];
  float scores[kSelMax];
  float pc[kSelMax];
  int pidx[kSelMax];
  unsigned char avail[kSelMax];
  int lvl_start[kLevels][kLevelSlots];
  int lvl_len[kLevels][kLevelSlots];   // 0 = no node in this slot
  float lvl_sum[kLevels][kLevelSlots];
  int leaf_slot[kLevels * kLevelSlots];  // (level << 7) | slot of every leaf
  int n_leaves;
  int tree_depth;
  long long scan_ll[32];
  double red_d[32];
  int red_i[32];
  int red_ne[32];
  int red_cnt[32];
  float red_f[32];
  int red_nan[32];
  float total;
  double cdf_total;
};

// ---- numpy pairwise float32 sum, as a split tree built level by level
// One warp: the node in slot j of level d has children in slots 2j, 2j+1 of
// level d+1 (left piece first, as numpy adds left + right).
__device__ void pw_tree_build(int m, SelShared& s, int lane) {
  if (lane == 0) {
    s.lvl_start[0][0] = 0;
    s.lvl_len[0][0] = m;
  }
  int nl = 0, depth = kLevels - 1;
  for (int d = 0; d < kLevels; ++d) {
    __syncwarp();
    const int width = 1 << d;
    bool more = false;
    for (int j0 = 0; j0 < width; j0 += 32) {
      const int j = j0 + lane;
      const int len = j < width ? s.lvl_len[d][j] : 0;
      const bool leaf = len > 0 && len <= kPwBlock;
      if (d + 1 < kLevels && j < width) {
        const int start = s.lvl_start[d][j];
        int n2 = 0;
        if (len > kPwBlock) {
          n2 = len / 2;
          n2 -= n2 % 8;
        }
        s.lvl_start[d + 1][2 * j] = start;
        s.lvl_len[d + 1][2 * j] = n2;
        s.lvl_start[d + 1][2 * j + 1] = start + n2;
        s.lvl_len[d + 1][2 * j + 1] = len > kPwBlock ? len - n2 : 0;
      }
      const unsigned bal = __ballot_sync(0xffffffffu, leaf);
      if (leaf) s.leaf_slot[nl + __popc(bal & ((1u << lane) - 1u))] = (d << 7) | j;
      nl += __popc(bal);
      more |= __any_sync(0xffffffffu, len > kPwBlock);
    }
    if (!more) {
      depth = d;  // deepest level holding a node
      break;
    }
  }
  if (lane == 0) {
    s.n_leaves = nl;
    s.tree_depth = depth;
  }
}

// One warp, after every leaf sum is in lvl_sum: internal nodes bottom-up.
__device__ float pw_tree_sum(SelShared& s, int lane) {
  for (int d = s.tree_depth - 1; d >= 0; --d) {
    __syncwarp();
    const int width = 1 << d;
    for (int j = lane; j < width; j += 32)
      if (s.lvl_len[d][j] > kPwBlock) s.lvl_sum[d][j] = __fadd_rn(s.lvl_sum[d + 1][2 * j], s.lvl_sum[d + 1][2 * j + 1]);
  }
  __syncwarp();
  return s.lvl_sum[0][0];
}

__device__ __forceinline__ unsigned long long shr128(unsigned long long h, unsigned long long l, int k) {
  if (k >= 128) return 0ull;
  if (k >= 64) return h >> (k - 64);
  if (k == 0) return l;
  return (l >> k) | (h << (64 - k));
}

// For integers 0 <= X < 2^53 and 0 < L < 2^54: the largest X with
// RN(X / L) <= u in float64 (-1 if none).  RN(q) <= u holds exactly when q is
// below the midpoint (2U+1) * 2^(e-1) between u = U * 2^e and its successor,
// or equal to it with U even (ties to even); with R = (2U+1) * L that is
// X * 2^(1-e) < R (or == R), evaluated in 128-bit integers.
__device__ long long cdf_threshold(double u, long long L) {
  if (isnan(u) || u < 0.0) return -1;
  if (u >= 1.0) return 0x7fffffffffffffffll;
  if (u == 0.0) return 0;
  const unsigned long long bits = static_cast<unsigned long long>(__double_as_longlong(u));
  const int ex = static_cast<int>((bits >> 52) & 0x7ff);
  if (ex == 0) return 0;  // subnormal u: X / L >= 2^-54 for every X >= 1
  const unsigned long long U = (bits & 0xFFFFFFFFFFFFFull) | (1ull << 52);
  const int sh = 1076 - ex;
  const unsigned long long a = 2 * U + 1;
  const unsigned long long lo = a * static_cast<unsigned long long>(L);
  const unsigned long long hi = __umul64hi(a, static_cast<unsigned long long>(L));
  unsigned long long t = shr128(hi - (lo == 0 ? 1ull : 0ull), lo - 1ull, sh);
  if ((U & 1ull) == 0 && sh < 128) {
    const bool tie = sh >= 64 ? (lo == 0 && (hi & ((1ull << (sh - 64)) - 1ull)) == 0)
                              : (lo & ((1ull << sh) - 1ull)) == 0;
    if (tie) t = shr128(hi, lo, sh);
  }
  return static_cast<long long>(t);
}

// Thread t owns the contiguous original indices [t*per, (t+1)*per): their
// scores, availability and interaction penalties, so no barrier separates one
// draw from the next.  The compacted (available-only) order is thread order,
// then index order inside a thread.
template <int NT>
__global__ void __launch_bounds__(NT, 1)
    boltzmann_kernel(const float* __restrict__ scores_in, const float* __restrict__ sim, int n, int n_select,
                     int block, float temp, const double* __restrict__ uniforms, int64_t* __restrict__ out_idx,
                     int* err) {
  constexpr int W = NT / 32;
  extern __shared__ __align__(16) uint8_t sel_smem[];
  SelShared& s = *reinterpret_cast<SelShared*>(sel_smem);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (n + NT - 1) / NT;
  const int lo = min(n, tid * per), hi = min(n, lo + per);
  for (int i = lo; i < hi; ++i) {
    s.scores[i] = scores_in[i];
    s.avail[i] = 1;
  }

  for (int r = 0; r < n_select; ++r) {
    const int m = n - r;  // available candidates
    const double u = uniforms[r];
    // (1) scaled scores of the owned available elements, their max and count;
    //     warp 0 also lays out the pairwise-sum tree for m elements
    int cnt = 0;
    float lmax = -INFINITY;
    int lnan = 0;
    for (int i = lo; i < hi; ++i) {
      if (!s.avail[i]) continue;
      ++cnt;
      const float x = __fdiv_rn(s.scores[i], temp);
      s.cdf[i] = x;
      if (isnan(x)) lnan = 1; else lmax = fmaxf(lmax, x);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, off));
      lnan |= __shfl_xor_sync(0xffffffffu, lnan, off);
    }
    int wx = cnt;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, wx, off);
      if (lane >= off) wx += y;
    }
    if (lane == 31) s.red_i[warp] = wx;
    if (lane == 0) {
      s.red_f[warp] = lmax;
      s.red_nan[warp] = lnan;
    }
    if (warp == 0) pw_tree_build(m, s, lane);
    __syncthreads();                                                   // barrier 1
    // (2) every warp combines the per-warp partials itself: compacted base,
    //     max, NaN flag; then exp at the compacted positions (shifted by the
    //     max only above 700, as the reference does)
    int base;
    float smax;
    bool any_nan;
    {
      const int ci = lane < W ? s.red_i[lane] : 0;
      int incl = ci;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += y;
      }
      base = __shfl_sync(0xffffffffu, incl - ci, warp) + (wx - cnt);
      float mx = lane < W ? s.red_f[lane] : -INFINITY;
      int nn = lane < W ? s.red_nan[lane] : 0;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        nn |= __shfl_xor_sync(0xffffffffu, nn, off);
      }
      smax = mx;
      any_nan = nn != 0;
    }
    const bool do_shift = !any_nan && smax > 700.0f;
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
    __syncthreads();                                                   // barrier 2
    // (3) leaf sums, 8 lanes per leaf: lane j holds numpy's accumulator r[j],
    //     combined as ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)), then the tail;
    //     leaves shorter than 8 are a running sum from 0
    const int n_leaves = s.n_leaves;
    for (int l0 = 0; l0 < n_leaves; l0 += NT / 8) {
      const int leaf = l0 + (tid >> 3), j = tid & 7;
      const bool active = leaf < n_leaves;
      const int slot = active ? s.leaf_slot[leaf] : 0;
      const int d = slot >> 7, sj = slot & (kLevelSlots - 1);
      const int a0 = active ? s.lvl_start[d][sj] : 0;
      const int ln = active ? s.lvl_len[d][sj] : 0;
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
        s.lvl_sum[d][sj] = res;
      }
    }
    __syncthreads();                                                   // barrier 3
    if (warp == 0) {
      const float root = pw_tree_sum(s, lane);
      if (lane == 0) s.total = __fadd_rn(0.0f, root);
    }
    __syncthreads();                                                   // barrier 4
    const float total = s.total;
    const bool uniform = (total == 0.0f) || !isfinite(total);
    const float inv_m = __fdiv_rn(1.0f, static_cast<float>(m));
    // (4) normalise the owned compacted range [base, base + cnt); p * 2^52
    //     is an integer for every p >= 2^-29, and then the float64 running
    //     sum is exact and equals an int64 scan
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
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, fx, off);
      if (lane >= off) fx += y;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      dsum += __shfl_xor_sync(0xffffffffu, dsum, off);
      not_exact |= __shfl_xor_sync(0xffffffffu, not_exact, off);
    }
    if (lane == 31) s.scan_ll[warp] = fx;
    if (lane == 0) {
      s.red_d[warp] = dsum;
      s.red_ne[warp] = not_exact;
    }
    __syncthreads();                                                   // barrier 5
    long long fbase, ftot;
    bool exact;
    {
      const long long wt = lane < W ? s.scan_ll[lane] : 0;
      long long incl = wt;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const long long y = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += y;
      }
      fbase = __shfl_sync(0xffffffffu, incl - wt, warp) + (fx - fsum);
      ftot = __shfl_sync(0xffffffffu, incl, 31);
      double pd = lane < W ? s.red_d[lane] : 0.0;
      int ne = lane < W ? s.red_ne[lane] : 0;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        pd += __shfl_xor_sync(0xffffffffu, pd, off);
        ne |= __shfl_xor_sync(0xffffffffu, ne, off);
      }
      exact = ne == 0;
      // np.random.choice rejects p whose sum is off by more than sqrt(eps_f32).
      if (tid == 0 && fabs(pd - 1.0) > 3.4526698300124393e-04) record_device_error(err, 0x301);
    }
    // (5) searchsorted(cdf / cdf[-1], u, 'right') = #{cdf entries <= u}
    int below = 0;
    if (exact) {
      const long long thr = cdf_threshold(u, ftot);
      long long run = fbase;
      for (int i = base; i < base + cnt; ++i) {
        run += static_cast<long long>(static_cast<double>(s.pc[i]) * 0x1p52);
        below += run <= thr ? 1 : 0;
      }
    } else {
      if (tid == 0) {
        double acc = 0.0;
        for (int i = 0; i < m; ++i) {
          acc = __dadd_rn(acc, static_cast<double>(s.pc[i]));
          s.cdf[i] = acc;  // the scaled scores of this draw are consumed
        }
        s.cdf_total = acc;
      }
      __syncthreads();
      const double cdf_last = s.cdf_total;
      for (int i = base; i < base + cnt; ++i) below += (__ddiv_rn(s.cdf[i], cdf_last) <= u) ? 1 : 0;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) below += __shfl_xor_sync(0xffffffffu, below, off);
    if (lane == 0) s.red_cnt[warp] = below;
    __syncthreads();                                                   // barrier 6
    int pick = lane < W ? s.red_cnt[lane] : 0;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) pick += __shfl_xor_sync(0xffffffffu, pick, off);
    const int sel = s.pidx[min(pick, m - 1)];
    if (tid == 0) out_idx[r] = sel;
    // (6) interaction penalty on every owned score (float32); the owner of
    //     the pick retires it.  Block-diagonal sim: [n/block, block, block],
    //     and only the pick's own block has nonzero entries (x - 0 == x).
    const float* row = sim + (int64_t)sel * n;
    int plo = lo, phi = hi;
    if (block > 0) {
      const int q0 = sel - sel % block;
      row = sim + (int64_t)sel * block - q0;
      plo = max(lo, q0);
      phi = min(hi, q0 + block);
    }
    for (int i = plo; i < phi; ++i) s.scores[i] = __fsub_rn(s.scores[i], row[i]);
    if (sel >= lo && sel < hi) s.avail[sel] = 0;
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
    greedy_kernel(const float* __restrict__ scores_in, const float* __restrict__ sim, int n, int block, int n_select,
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
    int plo = 0, phi = n;
    if (block > 0) {  // block-diagonal sim, as in boltzmann_kernel
      plo = sel - sel % block;
      phi = plo + block;
      row = sim + (int64_t)sel * block - plo;
    }
    for (int i = plo + tid; i < phi; i += kSelThreads) scores[i] = __fsub_rn(scores[i], row[i]);
    __syncthreads();
    if (tid == 0) scores[sel] = -INFINITY;
    __syncthreads();
  }
}

}  // namespace
}  // namespace opus

using namespace opus;

extern "C" {

}  // extern "C"

namespace {

int launch_boltzmann(const float* scores, const float* sim, int n, int block, int n_select, double temperature,
                     const double* uniforms, int64_t* out_idx, void* stream) {
  if (n <= 0 || n > kSelMax) return set_error(OPUS_ERR_UNSUPPORTED, "boltzmann: n=%d outside [1, %d]", n, kSelMax);
  if (n_select < 0 || n_select > n)
    return set_error(OPUS_ERR_INVALID, "boltzmann: cannot select %d of %d candidates", n_select, n);
  if (block < 0 || (block > 0 && n % block != 0))
    return set_error(OPUS_ERR_INVALID, "boltzmann: block %d does not divide n=%d", block, n);
  if (n_select == 0) return OPUS_OK;
  if (!scores || !sim || !uniforms || !out_idx) return set_error(OPUS_ERR_INVALID, "boltzmann: NULL pointer");
  const size_t smem = sizeof(SelShared);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const float tf = static_cast<float>(temperature);
  int* err = device_error_word();
  // one candidate per thread up to 1024 candidates, then 1024 threads
#define OPUS_LAUNCH_BOLTZMANN(NT)                                                                              \
  OPUS_CUDA_TRY(cudaFuncSetAttribute(boltzmann_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
  boltzmann_kernel<NT><<<1, NT, smem, st>>>(scores, sim, n, n_select, block, tf, uniforms, out_idx, err)
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

int launch_greedy(const float* scores, const float* sim, int n, int block, int n_select, int64_t* out_idx,
                  void* stream) {
  if (n <= 0 || n > 4 * kSelMax) return set_error(OPUS_ERR_UNSUPPORTED, "greedy: n=%d outside [1, %d]", n, 4 * kSelMax);
  if (n_select < 0) return set_error(OPUS_ERR_INVALID, "greedy: negative n_select");
  if (block < 0 || (block > 0 && n % block != 0))
    return set_error(OPUS_ERR_INVALID, "greedy: block %d does not divide n=%d", block, n);
  if (n_select == 0) return OPUS_OK;
  if (!scores || !sim || !out_idx) return set_error(OPUS_ERR_INVALID, "greedy: NULL pointer");
  const size_t smem = (size_t)n * sizeof(float);
  if (smem > 48 * 1024)
    OPUS_CUDA_TRY(cudaFuncSetAttribute(greedy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  greedy_kernel<<<1, kSelThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(scores, sim, n, block, n_select,
                                                                                   out_idx);
  OPUS_CUDA_TRY(cudaGetLastError());
  return OPUS_OK;
}

}  // namespace

extern "C" {

int opus_boltzmann_select(const float* scores, const float* sim, int n, int n_select, double temperature,
                          const double* uniforms, int64_t* out_idx, void* stream) {
  return launch_boltzmann(scores, sim, n, 0, n_select, temperature, uniforms, out_idx, stream);
}

int opus_boltzmann_select_blocks(const float* scores, const float* sim_blocks, int n, int block, int n_select,
                                 double temperature, const double* uniforms, int64_t* out_idx, void* stream) {
  if (block <= 0) return set_error(OPUS_ERR_INVALID, "boltzmann: block must be positive");
  return launch_boltzmann(scores, sim_blocks, n, block, n_select, temperature, uniforms, out_idx, stream);
}

int opus_greedy_select(const float* scores, const float* sim, int n, int n_select, int64_t* out_idx, void* stream) {
  return launch_greedy(scores, sim, n, 0, n_select, out_idx, stream);
}

int opus_greedy_select_blocks(const float* scores, const float* sim_blocks, int n, int block, int n_select,
                              int64_t* out_idx, void* stream) {
  if (block <= 0) return set_error(OPUS_ERR_INVALID, "greedy: block must be positive");
  return launch_greedy(scores, sim_blocks, n, block, n_select, out_idx, stream);
}

}  // extern "C"
