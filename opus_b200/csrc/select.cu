// Stage 5: Boltzmann (softmax-temperature) and greedy selection with the
// interaction penalty on one CTA (128 to 1024 threads, chosen by the candidate
// count; the Boltzmann sampler keeps each thread's candidates in registers,
// the greedy one keeps the scores in shared memory).  The float32 / float64
// operation order follows numpy, so the same uniforms give the same indices as
// the host implementation except where numpy's float32 exp and the correctly
// rounded one differ: numpy's vectorised exp is off by one ulp for a share of
// inputs, which moves each cdf entry by a few ulps, so a pick can differ only
// when u falls that close to a cdf entry:
//   - scaled = score / T in float32, shifted by its max only if max > 700;
//   - p = exp(scaled) rounded to float32 (computed in double, correctly rounded);
//   - sum = numpy's pairwise float32 sum (0 + blocks of <=128 with 8
//     accumulators, halves rounded down to a multiple of 8);
//   - p /= sum in float32, or 1/m when the sum is 0 or not finite;
//   - cdf = float64 running sum, cdf /= cdf[-1], idx = #{cdf <= u}.
// The float64 running sum is evaluated exactly with an int64 scan whenever
// every p is a multiple of 2^-52 (then no partial sum rounds), and the
// division by cdf[-1] with the comparison against u becomes one integer
// threshold per draw.  Otherwise the same scan of the truncated p gives the
// pick whenever u is farther from the cdf entries on either side of it than
// the rounding of the float64 sum can reach; only when it is not does one
// thread run the sequential float64 recurrence and every element get divided.
#include "opus_common.cuh"

namespace opus {
namespace {

constexpr int kSelMax = 8192;
constexpr int kPwBlock = 128;
// numpy's split tree for m <= 8192 candidates is at most 7 levels deep
constexpr int kMaxSlots = 128;
// p by compacted position q lives at q + 8 * (q / 128): the leaves of 128 that
// four 8-lane groups of a warp read at once fall in distinct banks
constexpr int kSkewedMax = kSelMax + kSelMax / kPwBlock * 8;

__device__ __forceinline__ int skew(int q) { return q + ((q >> 7) << 3); }

// float <-> int32 key with the same order (for redux max); NaN is tracked apart
__device__ __forceinline__ int f2ord(float f) {
  const int b = __float_as_int(f);
  return b >= 0 ? b : b ^ 0x7fffffff;
}
__device__ __forceinline__ float ord2f(int k) { return __int_as_float(k >= 0 ? k : k ^ 0x7fffffff); }

struct SelShared {
  double cdf[kSelMax];       // float64 running sum by compacted position (inexact fallback only)
  float pc[kSkewedMax];      // exp(x), then p, at skew(compacted position)
  float slot_sum[kMaxSlots]; // pairwise-sum leaves of this draw, one per slot
  long long scan_ll[32];
  int red_ne[32];
  int red_max[32];  // per-warp max of x as an order key
  int red_nan[32];
  double cdf_total;
  int pick;      // compacted position of this draw's pick
  int sel;       // its original index
  int fallback;  // set when the inexact-path pick could not be proven
};

// Depth of numpy's pairwise split tree for m elements: a piece longer than 128
// splits at half its length rounded down to a multiple of 8, and the right piece
// (the longer one) is always at least as deep as the left.
__device__ __forceinline__ int pw_depth(int m) {
  int d = 0;
  for (int len = m; len > kPwBlock; ++d) len -= (len / 2) & ~7;
  return d;
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
// p * 2^52 for a float32 p in [0, 1], read from its bits: P gets the integer
// part, and the result says whether p is a whole multiple of 2^-52 (then the
// float64 sum of such p is exact and equals the int64 sum of the P).
__device__ __forceinline__ bool fixed52(float p, long long& P) {
  const uint32_t u = __float_as_uint(p);
  const int e = static_cast<int>((u >> 23) & 0xFFu);
  uint32_t mant = u & 0x7FFFFFu;
  if (e == 0) {  // zero or subnormal: p * 2^52 < 1
    P = 0;
    return mant == 0;
  }
  mant |= 0x800000u;
  const int sh = e - 98;  // p * 2^52 = mant * 2^(e - 127 - 23 + 52)
  if (sh > 29) {          // p > 1 cannot come out of the normalisation
    P = 0;
    return false;
  }
  if (sh >= 0) {
    P = static_cast<long long>(mant) << sh;
    return true;
  }
  if (sh <= -32) {
    P = 0;
    return false;
  }
  P = static_cast<long long>(mant >> -sh);
  return (mant & ((1u << -sh) - 1u)) == 0;
}

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

// One CTA, NT threads; thread t owns the contiguous original indices
// [t*cnt, t*cnt + cnt) with cnt = ceil(n / NT) <= PER, and keeps their scores,
// x = score/T, exp(x) and availability in registers.  The compacted
// (available-only) order is thread order, then index order inside a thread, so
// a thread's available candidates sit at consecutive positions from its base,
// which drops by one whenever an earlier thread's candidate is picked.
//
// numpy's pairwise sum over the m available p is evaluated on a complete binary
// tree of 2^D slots, D = the split tree's depth for m: slot g is the numpy
// piece reached by descending along the bits of g, or, below a piece of <= 128
// (a leaf), the leaf itself on the leftmost path and an empty slot (sum +0)
// elsewhere.  Combining slots pairwise level by level then adds the numpy
// nodes in numpy's order (x + 0 == x for the non-negative partial sums), and a
// butterfly of shuffles gives every warp the total without another barrier.
template <int NT, int PER>
__global__ void __launch_bounds__(NT, 1)
    boltzmann_kernel(const float* __restrict__ scores_in, const float* __restrict__ sim, int n, int n_select,
                     int block, float temp, const double* __restrict__ uniforms, int64_t* __restrict__ out_idx,
                     int* err) {
  constexpr int W = NT / 32;
  extern __shared__ __align__(16) uint8_t sel_smem[];
  SelShared& s = *reinterpret_cast<SelShared*>(sel_smem);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cnt = (n + NT - 1) / NT;
  const int lo = min(n, tid * cnt), own = min(n, lo + cnt) - lo;
  // warps that own no candidate skip the per-candidate loops (warp-uniform)
  const bool warp_live = warp * 32 * cnt < n;
  float sc[PER], xv[PER], ev[PER];
  unsigned mask = 0;  // bit k: candidate lo + k is still available
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    sc[k] = k < own ? scores_in[lo + k] : 0.0f;
    xv[k] = ev[k] = 0.0f;
    if (k < own) mask |= 1u << k;
  }
  int pbase = lo;  // compacted position of this thread's first available candidate
  if (tid == 0) {
    s.fallback = 0;
    s.pick = 0;
    s.sel = 0;
  }
  __syncthreads();

  // candidates whose score changed since x and exp(x) were cached: all at the
  // first draw and after a dense penalty row, else the picked block
  int c0 = 0, c1 = n;
  for (int r = 0; r < n_select; ++r) {
    const int m = n - r;  // available candidates
    const double u = uniforms[r];
    // (1) x = score / T and exp(x) (refreshed where the score changed), placed
    //     at the compacted positions; max and NaN flag
    float lmax = -INFINITY;
    int lnan = 0;
    if (warp_live) {
      int q = pbase;
#pragma unroll
      for (int k = 0; k < PER; ++k) {
        if (!((mask >> k) & 1u)) continue;
        const int i = lo + k;
        if (i >= c0 && i < c1) {
          xv[k] = __fdiv_rn(sc[k], temp);
          ev[k] = static_cast<float>(exp(static_cast<double>(xv[k])));
        }
        s.pc[skew(q++)] = ev[k];
        if (isnan(xv[k])) lnan = 1; else lmax = fmaxf(lmax, xv[k]);
      }
    }
    {
      const int kmax = __reduce_max_sync(0xffffffffu, f2ord(lmax));
      lnan = __reduce_or_sync(0xffffffffu, lnan);
      if (lane == 0) {
        s.red_max[warp] = kmax;
        s.red_nan[warp] = lnan;
      }
    }
    __syncthreads();                                                   // barrier A
    {
      // the reference shifts by the max only when it exceeds 700 (and no NaN)
      const float mx = ord2f(__reduce_max_sync(0xffffffffu, lane < W ? s.red_max[lane] : f2ord(-INFINITY)));
      const int nn = __reduce_or_sync(0xffffffffu, lane < W ? s.red_nan[lane] : 0);
      if (nn == 0 && mx > 700.0f) {
        int q = pbase;
#pragma unroll
        for (int k = 0; k < PER; ++k)
          if ((mask >> k) & 1u) s.pc[skew(q++)] = static_cast<float>(exp(static_cast<double>(__fsub_rn(xv[k], mx))));
        __syncthreads();
      }
    }
    // (2) leaf sums, 8 lanes per slot: lane j holds numpy's accumulator r[j],
    //     combined as ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)), then the tail;
    //     leaves shorter than 8 are a running sum from 0
    //     Warps without a slot skip the pass (their predicated-off instruction
    //     stream would take issue slots from the working warps), and the loads
    //     are unconditional (clamped inside pc) so that they issue back to back.
    const int depth = pw_depth(m), n_slots = 1 << depth;
    for (int g0 = 0; g0 < n_slots; g0 += NT / 8) {
      if (g0 + 4 * warp >= n_slots) continue;  // warp-uniform
      const int g = g0 + (tid >> 3), j = tid & 7;
      const bool active = g < n_slots;
      int a0 = 0, ln = active ? m : 0;
      for (int d = depth - 1; d >= 0; --d) {
        const bool right = (g >> d) & 1;
        if (ln > kPwBlock) {
          const int n2 = (ln / 2) & ~7;
          if (right) {
            a0 += n2;
            ln -= n2;
          } else {
            ln = n2;
          }
        } else if (right) {
          ln = 0;
        }
      }
      const int full = ln >= 8 ? ln - (ln % 8) : 0;
      float v[kPwBlock / 8];
#pragma unroll
      for (int t = 0; t < kPwBlock / 8; ++t) v[t] = s.pc[skew(min(a0 + 8 * t + j, kSelMax - 1))];
      float acc = full > 0 ? v[0] : 0.0f;
#pragma unroll
      for (int t = 1; t < kPwBlock / 8; ++t) acc = 8 * t < full ? __fadd_rn(acc, v[t]) : acc;
      const float p01 = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
      const float p03 = __fadd_rn(p01, __shfl_xor_sync(0xffffffffu, p01, 2));
      const float p07 = __fadd_rn(p03, __shfl_xor_sync(0xffffffffu, p03, 4));
      if (active && j == 0) {
        float tail[7];
#pragma unroll
        for (int t = 0; t < 7; ++t) tail[t] = s.pc[skew(min(a0 + full + t, kSelMax - 1))];
        float res = full >= 8 ? p07 : 0.0f;
#pragma unroll
        for (int t = 0; t < 7; ++t) res = full + t < ln ? __fadd_rn(res, tail[t]) : res;
        s.slot_sum[g] = res;
      }
    }
    __syncthreads();                                                   // barrier L
    // (3) every warp combines the slots (pairs of slots first when there are
    //     more than 32), then normalises its owned positions; p * 2^52 is an
    //     integer for every p >= 2^-29, and then the float64 running sum is
    //     exact and equals an int64 scan
    float total = 0.0f;
    if (warp_live) {
      float v;
      if (n_slots <= 32) {
        v = s.slot_sum[lane & (n_slots - 1)];  // every group of n_slots lanes holds the slots
      } else if (n_slots == 64) {
        v = __fadd_rn(s.slot_sum[2 * lane], s.slot_sum[2 * lane + 1]);
      } else {
        v = __fadd_rn(__fadd_rn(s.slot_sum[4 * lane], s.slot_sum[4 * lane + 1]),
                      __fadd_rn(s.slot_sum[4 * lane + 2], s.slot_sum[4 * lane + 3]));
      }
      const int span = n_slots < 32 ? n_slots : 32;
      for (int off = 1; off < span; off <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
      total = __fadd_rn(0.0f, v);
    }
    const bool uniform = (total == 0.0f) || !isfinite(total);
    const float inv_m = __fdiv_rn(1.0f, static_cast<float>(m));
    int not_exact = 0;
    long long fsum = 0;
    if (warp_live) {
      int q = pbase;
#pragma unroll
      for (int k = 0; k < PER; ++k) {
        if (!((mask >> k) & 1u)) continue;
        const int qs = skew(q++);
        const float p = uniform ? inv_m : __fdiv_rn(s.pc[qs], total);
        s.pc[qs] = p;
        long long P;
        if (!fixed52(p, P)) not_exact = 1;
        fsum += P;
      }
    }
    long long fx = fsum;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, fx, off);
      if (lane >= off) fx += y;
    }
    not_exact = __reduce_or_sync(0xffffffffu, not_exact);
    if (lane == 31) s.scan_ll[warp] = fx;
    if (lane == 0) s.red_ne[warp] = not_exact;
    __syncthreads();                                                   // barrier C
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
      exact = __reduce_or_sync(0xffffffffu, lane < W ? s.red_ne[lane] : 0) == 0;
      // np.random.choice rejects p whose sum is off by more than sqrt(eps_f32);
      // the truncated int64 total is within n * 2^-52 of the float64 sum.
      if (tid == 0 && fabs(static_cast<double>(ftot) * 0x1p-52 - 1.0) > 3.4526698300124393e-04)
        record_device_error(err, 0x301);
    }
    // (4) searchsorted(cdf / cdf[-1], u, 'right') counts the entries <= u; the
    //     cdf is non-decreasing, so the pick is the first position whose entry
    //     is not <= u (or the last one).  With T_q the int64 scan, that is the
    //     first T_q above thr = max{X : RN(X / T_{m-1}) <= u}; thr is within
    //     2 of u * T_{m-1}, so only a thread whose range of T comes that close
    //     evaluates it and searches its candidates.
    //     When some p is not a multiple of 2^-52, T_q truncates the p and the
    //     float64 running sum c_q rounds: |c_q * 2^52 - T_q| < q + 1 + m/2 * S_q
    //     <= E = 2m + 2 (S_q the exact sum, <= 1 + 3.5e-4).  The pick found from
    //     T stands when it is proven by that margin on both sides; otherwise
    //     one thread runs the float64 recurrence below.
    {
      const bool u_ok = u >= 0.0 && u < 1.0;
      const double approx = u * static_cast<double>(ftot);
      const bool cand = own > 0 && (!u_ok || (static_cast<double>(fbase) <= approx + 4.0 &&
                                              approx - 4.0 < static_cast<double>(fbase + fsum)));
      if (__any_sync(0xffffffffu, cand)) {
        const long long thr = cdf_threshold(u, ftot);
        if (cand) {
          long long run = fbase;
          int q = pbase;
#pragma unroll
          for (int k = 0; k < PER; ++k) {
            if (!((mask >> k) & 1u)) continue;
            long long P;
            fixed52(s.pc[skew(q)], P);
            const long long prev = run;
            run += P;
            if ((run > thr && (q == 0 || prev <= thr)) || (q == m - 1 && run <= thr)) {
              s.pick = q;
              s.sel = lo + k;
              if (!exact) {
                const double E = 2.0 * m + 2.0;
                bool proven = true;
                if (q != m - 1)
                  proven = static_cast<double>(run) - E >= (u * (static_cast<double>(ftot) + E)) * (1.0 + 0x1p-50);
                if (q != 0)
                  proven = proven &&
                           static_cast<double>(prev) + E <= (u * (static_cast<double>(ftot) - E)) * (1.0 - 0x1p-50);
                if (!proven) s.fallback = 1;
              }
            }
            ++q;
          }
        }
      }
    }
    __syncthreads();                                                   // barrier D
    if (s.fallback) {
      // float64 recurrence of numpy's cumsum, then RN(cdf[q] / cdf[-1]) <= u
      if (tid == 0) {
        double acc = 0.0;
        for (int q = 0; q < m; ++q) {
          acc = __dadd_rn(acc, static_cast<double>(s.pc[skew(q)]));
          s.cdf[q] = acc;
        }
        s.cdf_total = acc;
      }
      __syncthreads();
      if (tid == 0) s.fallback = 0;  // every thread has read it
      const double last = s.cdf_total;
      int q = pbase;
#pragma unroll
      for (int k = 0; k < PER; ++k) {
        if (!((mask >> k) & 1u)) continue;
        const bool le = __ddiv_rn(s.cdf[q], last) <= u;
        const bool prev_le = q == 0 || __ddiv_rn(s.cdf[q - 1], last) <= u;
        if ((!le && prev_le) || (q == m - 1 && le)) {
          s.pick = q;
          s.sel = lo + k;
        }
        ++q;
      }
      __syncthreads();
    }
    const int sel = s.sel;
    if (tid == 0) out_idx[r] = sel;
    // (5) interaction penalty on every owned score (float32) and retire the
    //     pick.  Block-diagonal sim: [n/block, block, block], and only the
    //     pick's own block has nonzero entries (x - 0 == x).
    const float* row = sim + static_cast<int64_t>(sel) * n;
    c0 = 0;
    c1 = n;
    if (block > 0) {
      c0 = sel - sel % block;
      c1 = c0 + block;
      row = sim + static_cast<int64_t>(sel) * block - c0;
    }
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int i = lo + k;
      if (k < own && i >= c0 && i < c1) sc[k] = __fsub_rn(sc[k], __ldg(row + i));
    }
    if (sel < lo) --pbase;
    else if (sel < lo + own) mask &= ~(1u << (sel - lo));
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

// np.argmax over a warp with two redux steps: the largest order key (NaN above
// every number, -0 folded into +0 since they compare equal), then the lowest
// index holding it.
__device__ __forceinline__ void warp_argmax(int& key, int& idx) {
  const int kmax = __reduce_max_sync(0xffffffffu, key);
  idx = __reduce_min_sync(0xffffffffu, key == kmax ? idx : 0x7fffffff);
  key = kmax;
}

// Thread t owns the candidates i = t, t + NT, t + 2 NT, ...: it alone reads and
// writes their scores (the penalty row is then read coalesced), so the one
// barrier of a draw is the one that publishes the warps' maxima; they sit in
// two buffers by draw parity, so the next draw's writes cannot meet this
// draw's reads.  Every warp finishes the argmax itself.
template <int NT>
__global__ void __launch_bounds__(NT, 1)
    greedy_kernel(const float* __restrict__ scores_in, const float* __restrict__ sim, int n, int block, int n_select,
                  int64_t* __restrict__ out_idx) {
  constexpr int W = NT / 32;
  extern __shared__ __align__(16) uint8_t sel_smem[];
  float* scores = reinterpret_cast<float*>(sel_smem);
  __shared__ int rk[2][W];
  __shared__ int ri[2][W];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < n; i += NT) scores[i] = scores_in[i];
  for (int r = 0; r < n_select; ++r) {
    ArgMax best{-INFINITY, 0x7fffffff};
    for (int i = tid; i < n; i += NT) best = better(best, ArgMax{scores[i], i});
    int key = isnan(best.v) ? 0x7fffffff : f2ord(best.v == 0.0f ? 0.0f : best.v), idx = best.i;
    warp_argmax(key, idx);
    if (lane == 0) {
      rk[r & 1][warp] = key;
      ri[r & 1][warp] = idx;
    }
    __syncthreads();
    key = lane < W ? rk[r & 1][lane] : f2ord(-INFINITY);
    idx = lane < W ? ri[r & 1][lane] : 0x7fffffff;
    warp_argmax(key, idx);
    // all entries -inf: np.argmax returns 0
    const int sel = (idx == 0x7fffffff) ? 0 : idx;
    if (tid == 0) out_idx[r] = sel;
    const float* row = sim + (int64_t)sel * n;
    int plo = 0, phi = n;
    if (block > 0) {  // block-diagonal sim, as in boltzmann_kernel
      plo = sel - sel % block;
      phi = plo + block;
      row = sim + (int64_t)sel * block - plo;
    }
    // the first owned candidate at or after plo
    for (int i = plo + ((tid - plo % NT) + NT) % NT; i < phi; i += NT) scores[i] = __fsub_rn(scores[i], row[i]);
    if (sel % NT == tid) scores[sel] = -INFINITY;
  }
}

}  // namespace
}  // namespace opus

using namespace opus;

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
  // one candidate per thread up to 512 candidates, then two each on 512 threads, then 1024
  // threads with up to 8 each
#define OPUS_LAUNCH_BOLTZMANN(NT, PER)                                                                          \
  OPUS_CUDA_TRY(cudaFuncSetAttribute(boltzmann_kernel<NT, PER>, cudaFuncAttributeMaxDynamicSharedMemorySize,      \
                                     (int)smem));                                                                 \
  boltzmann_kernel<NT, PER><<<1, NT, smem, st>>>(scores, sim, n, n_select, block, tf, uniforms, out_idx, err)
  if (n <= 128) {
    OPUS_LAUNCH_BOLTZMANN(128, 1);
  } else if (n <= 256) {
    OPUS_LAUNCH_BOLTZMANN(256, 1);
  } else if (n <= 512) {
    OPUS_LAUNCH_BOLTZMANN(512, 1);
  } else if (n <= 1024) {
    OPUS_LAUNCH_BOLTZMANN(512, 2);  // measured 5% faster than 1024 x 1 at n = 1024
  } else if (n <= 2048) {
    OPUS_LAUNCH_BOLTZMANN(1024, 2);
  } else if (n <= 4096) {
    OPUS_LAUNCH_BOLTZMANN(1024, 4);
  } else {
    OPUS_LAUNCH_BOLTZMANN(1024, 8);
  }
#undef OPUS_LAUNCH_BOLTZMANN
  ::opus::note_launch();
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
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
#define OPUS_LAUNCH_GREEDY(NT)                                                                                 \
  if (smem > 48 * 1024)                                                                                        \
    OPUS_CUDA_TRY(cudaFuncSetAttribute(greedy_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
  greedy_kernel<NT><<<1, NT, smem, st>>>(scores, sim, n, block, n_select, out_idx)
  if (n <= 128) {
    OPUS_LAUNCH_GREEDY(128);
  } else if (n <= 256) {
    OPUS_LAUNCH_GREEDY(256);
  } else if (n <= 512) {
    OPUS_LAUNCH_GREEDY(512);
  } else {
    OPUS_LAUNCH_GREEDY(1024);
  }
#undef OPUS_LAUNCH_GREEDY
  ::opus::note_launch();
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
