// Fused per-sample gradient GEMM + CountSketch scatter (stage 3 of the
// selection path), sm_100a.
//
// For candidate b and weight tile (ob, cb) the CTA computes the 128 x 256
// tile of G_b = dLdZ_b^T a_b (K = the candidate's tokens) with tcgen05.mma
// (bf16 x bf16 -> f32 in TMEM), then its epilogue multiplies every element by
// w(o,c) = s(o,c) * D(o,c) from the precomputed table and adds it into bucket
// h(o,c) of candidate b's sketch.  G_b is never written to HBM.
//
// Warp roles (64 + 32 x 8, 12 or 16 epilogue warps threads; persistent, one
// CTA per SM; in a pair the MMA warp of the second CTA issues no MMA and
// forwards its epilogue's accumulator releases to the leader):
//   warp 0      TMA producer: 3-D tile loads of dLdZ and a into a ring of
//               shared-memory stages (128-byte swizzle, MN-major operands);
//   warp 1      TMEM allocation + single-thread UMMA issue into one of two
//               256-column accumulators (double-buffered against the epilogue);
//   warps 2..   epilogue: 8, 12 or 16 warps, two to four per TMEM lane
//               quarter, dealt the tile's 32-, 16- or 8-column chunks round-robin;
//               chunks past d_in and lane quarters past d_out are skipped.
//
// Shared-memory sketch in 32-bit fixed point.  Float atomics on shared memory
// are compare-and-swap loops on this hardware, integer adds are native, so
// the CTA-private sketch of the current job holds int32 buckets at a
// power-of-two scale S chosen from a sample of the job's first tile (each
// epilogue warp's first live chunk; the sample's max |w G| maps to cap/16).  cap = 2^31 / (largest bucket load of the
// layer) bounds every admitted update, so no bucket can overflow whatever the
// data; an update above cap (or NaN/Inf, or any update before a scale could
// be chosen) goes straight to the f32 output row with a global atomic add.
// The sketch is converted back to f32 and added to the output row (vector
// reductions) whenever the candidate changes.  Quantisation error per update
// is at most (max |w G| of the sample) * 2^-(log2(cap) - 4 + 1), i.e.
// ~1e-6 of the tile maximum for the GPT-2 layer shapes.  When the k buckets
// do not fit next to two pipeline stages (k > 32768), the sketch covers the
// largest prefix of them that does (32768 buckets for one CTA, 40960 or 45056
// for a pair) and the updates of the other buckets are f32 global atomic adds.
//
// CTA pairs (sketches larger than one CTA's shared memory): a cluster of two
// CTAs computes 256 x 256 tiles with tcgen05.mma.cta_group::2.  Each CTA
// stages its own o-block's dLdZ rows and half of the activation columns (32 KB
// per 64-token stage instead of 48 KB), so the shared memory it saves holds
// more of the sketch; the leader issues the MMAs and each CTA's epilogue
// scatters the accumulator rows of its own o-block.
//
// Work: a job is a contiguous range of one candidate's tiles (in the walk
// that plan_jobs picks); jobs are numbered candidate-major and dealt to CTAs
// (or pairs) round-robin, so at any time they work on neighbouring candidates
// whose operands stay resident in L2, and each job ends with one sketch flush.
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "opus_common.cuh"
#include "sketch_layout.cuh"

namespace opus {
namespace {

// Epilogue warps: 8 (the dense epilogue), 12 or 16 (the scatter; 16 by default).
// kThreads and the dense epilogue's chunking are those of 8.
constexpr int kEpiWarps = 8;
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr int kThreads = 64 + kEpiThreads;
constexpr int kChunksPerWarp = kChunksPerTile / (kEpiWarps / 4);  // 4
constexpr int block_threads(int epi) { return 64 + 32 * epi; }

constexpr int kHeadroomLog2 = 4;                     // sampled first-tile max maps to cap / 16
constexpr int kBoxMN = 64;                           // bf16 elements per 128-byte swizzle row
constexpr int kUmmaK = 16;                           // K of one kind::f16 MMA
constexpr int kGBoxes = kTileM / kBoxMN;             // 2 boxes for the 128 weight rows
constexpr int kABoxes = kTileN / kBoxMN;             // 4 boxes for the 256 weight columns
// Pipeline stage geometry for BK tokens per stage (64: 48 KB stages; 32: 24 KB
// stages, which leave room for more of a large sketch in shared memory).  A CTA
// of a pair (PAIR) stages its own o-block's dLdZ rows and half of the tile's
// activation columns: 32 KB at BK = 64.
template <int BK, bool PAIR = false>
struct Stage {
  static constexpr int kBK = BK;
  static constexpr int kKSteps = BK / kUmmaK;                     // MMAs per stage
  static constexpr int kBoxBytes = kBoxMN * 2 * BK;               // one 64-feature box
  static constexpr int kGTileBytes = kGBoxes * kBoxBytes;
  static constexpr int kABoxesCta = PAIR ? kABoxes / 2 : kABoxes;  // activation boxes this CTA loads
  static constexpr int kATileBytes = kABoxesCta * kBoxBytes;
  static constexpr int kStageBytes = kGTileBytes + kATileBytes;   // 48 KB at BK = 64, 24 KB at 32
  static constexpr uint32_t kLBO = kBoxBytes;
};
constexpr int kStageBytes64 = Stage<64>::kStageBytes;
constexpr int kStageBytes32 = Stage<32>::kStageBytes;
constexpr int kStageBytesPair64 = Stage<64, true>::kStageBytes;
constexpr int kStageBytesPair32 = Stage<32, true>::kStageBytes;
// MN-major SW128 canonical layout: 64 contiguous MN elements x 8 K rows per
// 1024-B atom; atoms along K at SBO = 1024 B, along MN (next box) at LBO.
constexpr uint32_t kSBO = 1024;
constexpr uint32_t kKStepBytes = (kUmmaK / 8) * 1024;  // 2 atoms per MMA
constexpr uint32_t kIdesc = make_idesc(/*bf16*/ 1, /*a MN-major*/ 1, /*b MN-major*/ 1, kTileM, kTileN);
constexpr uint32_t kIdescPair = make_idesc(/*bf16*/ 1, /*a MN-major*/ 1, /*b MN-major*/ 1, 2 * kTileM, kTileN);
constexpr int kTmemCols = 2 * kTileN;  // two accumulators

struct SmemPlan {
  int stages;
  int64_t k_sm;      // buckets [0, k_sm) have a CTA-private fixed-point sketch in shared memory
  size_t bytes;      // dynamic shared memory to request
};

// Read-only table load that bypasses L1 (each entry is read once per tile).
// Not volatile: independent loads may be hoisted and kept in flight together.
// Table entries: read once per candidate tile, never kept in L1, kept in L2
// (every candidate re-reads the layer's table).
__device__ __forceinline__ uint4 ld_table(const uint4* p, uint64_t l2_policy) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p), "l"(l2_policy));
  return v;
}

// Read-only 16-byte load kept in L2 with the given policy (the dense
// epilogue's diagonal, read again by every candidate).
__device__ __forceinline__ float4 ld_f4_hint(const float* p, uint64_t l2_policy) {
  float4 v;
  asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
      : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
      : "l"(p), "l"(l2_policy));
  return v;
}

// Tile range [begin, end) of job j: each candidate's n_tiles tiles (o-block
// major) are cut into units of `unit` tiles (a whole o-block, or one tile),
// and the units into `groups` contiguous ranges.
__device__ __forceinline__ int job_tile_begin(int64_t job, int groups, int n_tiles, int unit) {
  return static_cast<int>((job % groups) * (n_tiles / unit) / groups) * unit;
}
__device__ __forceinline__ int job_tile_end(int64_t job, int groups, int n_tiles, int unit) {
  return static_cast<int>((job % groups + 1) * (n_tiles / unit) / groups) * unit;
}

// Tile `t` of a candidate's walk: o-block major (t = ob * n_cb + cb) or
// column-block major (t = cb * n_ob + ob); plan_jobs picks the walk.
struct TileWalk {
  int n_ob, n_cb, cb_major;
  __device__ __forceinline__ int ob(int t) const { return cb_major ? t % n_ob : t / n_cb; }
  __device__ __forceinline__ int cb(int t) const { return cb_major ? t / n_ob : t % n_cb; }
  // the last tile of a run that shares the outer operand
  __device__ __forceinline__ bool last_inner(int t) const {
    return cb_major ? t % n_ob == n_ob - 1 : t % n_cb == n_cb - 1;
  }
};

// Bounded barrier over the epilogue threads (an mbarrier, so that a thread
// that gave up cannot leave the others blocked forever).
__device__ __forceinline__ bool epi_sync(uint64_t* bar, uint32_t& phase, volatile int* abort_flag, int* err) {
  mbar_arrive(bar);
  const bool ok = mbar_wait(bar, phase, abort_flag, err, kDevTimeoutGroup);
  phase ^= 1;
  return ok;
}

// Add the fixed-point sketch of buckets [0, k) (scaled by 2^-scale_exp) into
// dst and clear it.
__device__ bool flush_sketch(int* sk, float* dst, int64_t k, int scale_exp, int et, int n_threads, uint64_t* bar,
                             uint32_t& phase, volatile int* abort_flag, int* err) {
  if (!epi_sync(bar, phase, abort_flag, err)) return false;
  const float inv = ldexpf(1.0f, -scale_exp);
  if ((k & 3) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
    int4* s4 = reinterpret_cast<int4*>(sk);
    for (int64_t i = et; i < k / 4; i += n_threads) {
      const int4 q = s4[i];
      if (q.x | q.y | q.z | q.w) {
        red_add_v4(dst + 4 * i, (float)q.x * inv, (float)q.y * inv, (float)q.z * inv, (float)q.w * inv);
        s4[i] = make_int4(0, 0, 0, 0);
      }
    }
  } else {
    for (int64_t i = et; i < k; i += n_threads) {
      const int q = sk[i];
      if (q != 0) {
        atomicAdd(dst + i, (float)q * inv);
        sk[i] = 0;
      }
    }
  }
  return epi_sync(bar, phase, abort_flag, err);
}

template <int BK, bool PAIR, int EPI>
__global__ void __launch_bounds__(block_threads(EPI), 1)
    sketch_gemm_kernel(const __grid_constant__ CUtensorMap tm_g, const __grid_constant__ CUtensorMap tm_a,
                       const __grid_constant__ CUtensorMap tm_out,
                       const uint4* __restrict__ table, float* __restrict__ phi, int n_rows, int seq_len, int n_tiles, int unit, int cb_major,
                       int n_cb, int groups, int64_t k, int rows_div, int stages, int64_t k_sm, float cap,
                       int cap_log2, int* err, int dense, const float* __restrict__ dense_diag, int d_out,
                       int d_in, int accumulate, float alpha) {
  using G = Stage<BK, PAIR>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* stage_mem = smem;
  int* sk = reinterpret_cast<int*>(smem + (size_t)stages * G::kStageBytes);
  const bool smem_sketch = k_sm > 0;
  uint8_t* tail = smem + (size_t)stages * G::kStageBytes + (size_t)k_sm * 4;
  tail = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tail) + 15) & ~uintptr_t(15));
  uint64_t* full = reinterpret_cast<uint64_t*>(tail);
  uint64_t* empty = full + stages;
  uint64_t* tfull = empty + stages;
  uint64_t* tempty = tfull + 2;
  uint64_t* epi_bar = tempty + 2;
  uint64_t* drain_bar = epi_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* tile_max_bits = reinterpret_cast<int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // PAIR: a cluster of two CTAs computes 256 x 256 tiles (an o-block pair by a
  // column block) with tcgen05.mma.cta_group::2.  Each CTA stages its own
  // o-block's 128 dLdZ rows and its half of the activation columns, the leader
  // (rank 0) issues the MMAs for both, and each CTA's TMEM holds the accumulator
  // rows of its own o-block, which its epilogue scatters into its own sketch.
  // The walk then runs over o-block pairs; the CTA's o-block is 2 * pair + rank.
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const int64_t worker = PAIR ? blockIdx.x / 2 : blockIdx.x;  // the CTA, or the pair, that takes jobs
  const int64_t n_workers = PAIR ? gridDim.x / 2 : gridDim.x;
  const int n_ob_real = (d_out + kTileM - 1) / kTileM;
  // Job j = (candidate j / groups, tile range j % groups); worker i takes jobs
  // i, i + workers, ..., so the CTAs work on neighbouring candidates at any time
  // and each candidate's operands stay L2-resident while they are read.
  const int64_t n_jobs = (int64_t)n_rows * groups;
  const TileWalk walk{n_tiles / n_cb, n_cb, cb_major};
  const int n_kb = (seq_len + G::kBK - 1) / G::kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      // one arrival per epilogue warp of this CTA; a pair's leader also counts the one
      // arrival that relays the second CTA's release
      mbar_init(&tempty[a], PAIR && rank == 0 ? EPI + 1 : EPI);
    }
    mbar_init(epi_bar, 32 * EPI);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    *tile_max_bits = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_g);
    prefetch_tmap(&tm_a);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, kTmemCols);
      tmem_relinquish();
    }
  }
  for (int64_t i = threadIdx.x; i < k_sm; i += block_threads(EPI)) sk[i] = 0;
  tc_fence_before();
  __syncthreads();
  // both CTAs' barriers are initialised before any load, commit or arrival crosses the pair
  if constexpr (PAIR) cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      const uint64_t pol_last = l2_policy_evict_last(), pol_first = l2_policy_evict_first();
      const uint32_t full_lead = PAIR ? mapa_shared(smem_u32(full), 0) : 0u;  // the leader's full barriers
      for (int64_t job = worker; job < n_jobs && ok; job += n_workers)
      for (int tile = job_tile_begin(job, groups, n_tiles, unit); tile < job_tile_end(job, groups, n_tiles, unit) && ok;
           ++tile) {
        const int ob = walk.ob(tile), cb = walk.cb(tile);
        const int b = static_cast<int>(job / groups);
        for (int kb = 0; kb < n_kb; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, err, kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          // a pair's stage is complete on the leader's barrier when both CTAs' bytes have landed
          if (rank == 0) mbar_arrive_expect_tx(&full[s], (PAIR ? 2 : 1) * G::kStageBytes);
          uint8_t* sg = stage_mem + (size_t)s * G::kStageBytes;
          uint8_t* sa = sg + G::kGTileBytes;
          const int t0 = kb * G::kBK;
          // L2 policy: the outer operand of the walk (dLdZ rows of an o-block, or
          // activation columns of a column block) is not read again after the
          // last tile of its run; the inner operand serves every run
          const bool drop = walk.last_inner(tile);
          const uint64_t gpol = drop && !walk.cb_major ? pol_first : pol_last;
          const uint64_t apol = drop && walk.cb_major ? pol_first : pol_last;
          if constexpr (PAIR) {
            // this CTA's o-block (zero-filled past d_out) and its half of the columns
            const uint32_t bar = full_lead + static_cast<uint32_t>(s) * 8u;
#pragma unroll
            for (int i = 0; i < kGBoxes; ++i)
              tma_load_3d_pair(sg + i * G::kBoxBytes, &tm_g, bar, (2 * ob + (int)rank) * kTileM + i * kBoxMN, t0, b,
                               gpol);
#pragma unroll
            for (int i = 0; i < G::kABoxesCta; ++i)
              tma_load_3d_pair(sa + i * G::kBoxBytes, &tm_a, bar,
                               cb * kTileN + (int)rank * (kTileN / 2) + i * kBoxMN, t0, b, apol);
          } else {
#pragma unroll
            for (int i = 0; i < kGBoxes; ++i)
              tma_load_3d_hint(sg + i * G::kBoxBytes, &tm_g, &full[s], ob * kTileM + i * kBoxMN, t0, b, gpol);
#pragma unroll
            for (int i = 0; i < kABoxes; ++i)
              tma_load_3d_hint(sa + i * G::kBoxBytes, &tm_a, &full[s], cb * kTileN + i * kBoxMN, t0, b, apol);
          }
          if (++s == stages) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // (a pair's MMAs are issued by its leader alone)
    if (lane == 0 && rank == 0) {
      int s = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t aph = 0;
      bool ok = true;
      // a commit arrives on this barrier in both CTAs of a pair (each at its own address)
      auto commit_both = [&](uint64_t* bar) {
        if constexpr (PAIR) {
          umma_commit_pair(mapa_shared(smem_u32(bar), 0));
          umma_commit_pair(mapa_shared(smem_u32(bar), 1));
        } else {
          umma_commit(bar);
        }
      };
      for (int64_t job = worker; job < n_jobs && ok; job += n_workers)
      for (int u = job_tile_begin(job, groups, n_tiles, unit); u < job_tile_end(job, groups, n_tiles, unit) && ok; ++u) {
        if (!mbar_wait(&tempty[acc], aph ^ 1, abort_flag, err, kDevTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kTileN);
        for (int kb = 0; kb < n_kb; ++kb) {
          if (!mbar_wait(&full[s], ph, abort_flag, err, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t ag = smem_u32(stage_mem + (size_t)s * G::kStageBytes);
          const uint32_t aa = ag + G::kGTileBytes;
#pragma unroll
          for (int kk = 0; kk < G::kKSteps; ++kk) {
            const uint64_t da = make_sdesc_sw128(ag + kk * kKStepBytes, G::kLBO, kSBO);
            const uint64_t db = make_sdesc_sw128(aa + kk * kKStepBytes, G::kLBO, kSBO);
            if constexpr (PAIR)
              umma_bf16_pair(d_tmem, da, db, kIdescPair, (kb | kk) != 0 ? 1u : 0u);
            else
              umma_bf16(d_tmem, da, db, kIdesc, (kb | kk) != 0 ? 1u : 0u);
          }
          commit_both(&empty[s]);
          if (++s == stages) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        commit_both(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          aph ^= 1;
        }
      }
      // Drain: every MMA issued above must be complete before TMEM is freed.
      if constexpr (PAIR)
        umma_commit_pair(mapa_shared(smem_u32(drain_bar), 0));
      else
        umma_commit(drain_bar);
      mbar_wait(drain_bar, 0, nullptr, err, kDevTimeoutDrain);
    } else if (PAIR && lane == 0) {
      // The second CTA's epilogue warps release an accumulator on this CTA's own barrier
      // (CTA-scope arrivals); this thread, which has no memory operations of its own in
      // flight, forwards each completed release to the leader with one cluster-scope arrival.
      // (Sixteen cluster-scope arrivals, one per epilogue warp, each waited for that warp's
      // L2 reductions in flight: 552 against 578 TFLOP/s at 1600 -> 6400, 128 rows.)
      const uint32_t lead = mapa_shared(smem_u32(tempty), 0);
      int acc = 0;
      uint32_t aph = 0;
      bool ok = true;
      for (int64_t job = worker; job < n_jobs && ok; job += n_workers)
      for (int u = job_tile_begin(job, groups, n_tiles, unit); u < job_tile_end(job, groups, n_tiles, unit) && ok; ++u) {
        if (!mbar_wait(&tempty[acc], aph, abort_flag, err, kDevTimeoutEpilogue)) {
          ok = false;
          break;
        }
        mbar_arrive_cluster(lead + static_cast<uint32_t>(acc) * 8u);
        if (++acc == 2) {
          acc = 0;
          aph ^= 1;
        }
      }
    }
  } else if (!PAIR && EPI == kEpiWarps && dense) {
    // ------------------------------------------------- dense epilogue
    // Per-sample gradients: element (o, c) of G_b, times dense_diag[o, c]
    // when given, goes to phi[b, o * d_in + c].  Each warp stages its 32 rows
    // x 32 columns of a chunk in shared memory, in the 128-byte-swizzled
    // layout of the output tensor map (row r's 16-byte piece u sits at
    // u ^ (r & 7): conflict-free writes), and one lane stores the box with
    // TMA (a reduce-add when accumulating), so every global write is a full
    // 128-byte line.  Two staging buffers per warp: a buffer is rewritten
    // only after the store issued from it two chunks earlier has been read.
    // Rows past d_out and columns past d_in fall outside the tensor map and
    // are not written.
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
    const uint64_t diag_policy = l2_policy_evict_last();  // every candidate re-reads the diagonal
    float* staging = reinterpret_cast<float*>(sk) + (size_t)(warp - 2) * 2 * kChunkCols * 32;
    int buf = 0;
    int acc = 0;
    uint32_t aph = 0;
    bool ok = true;
    for (int64_t job = worker; job < n_jobs && ok; job += n_workers)
    for (int tile = job_tile_begin(job, groups, n_tiles, unit); tile < job_tile_end(job, groups, n_tiles, unit) && ok; ++tile) {
      const int ob = walk.ob(tile), cb = walk.cb(tile);
      const int b = static_cast<int>(job / groups);
      const int row0 = ob * kTileM + q * 32;  // first row of this warp's block
      // the diagonal of a chunk is loaded one chunk ahead (the first one before the accumulator
      // wait), so its L2 latency hides behind the previous chunk's staging and store
      // The diagonal of the warp's 32 x 32 block of a chunk, read coalesced: load u of lane l
      // is row 4u + l / 8, columns 4 (l % 8) .. +3, so one warp load covers four whole 128-byte
      // rows.  It goes through the staging buffer to reach the thread that owns its row.  A
      // chunk's block is loaded two chunks ahead (the first two before the accumulator wait).
      float4 w_ring[3][kChunkCols / 4];
      auto load_diag = [&](float4(&w)[kChunkCols / 4], int jj) {
        const int c = cb * kTileN + (half * kChunksPerWarp + jj) * kChunkCols + (lane & 7) * 4;
#pragma unroll
        for (int u = 0; u < kChunkCols / 4; ++u) {  // d_in % 8 == 0: a piece is all in or all out
          const int orow = row0 + 4 * u + (lane >> 3);
          w[u] = (dense_diag != nullptr && orow < d_out && c < d_in)
                     ? ld_f4_hint(dense_diag + (int64_t)orow * d_in + c, diag_policy)
                     : make_float4(1.0f, 1.0f, 1.0f, 1.0f);
        }
      };
      load_diag(w_ring[0], 0);
      load_diag(w_ring[1], 1);
      if (!mbar_wait(&tfull[acc], aph, abort_flag, err, kDevTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int jj = 0; jj < kChunksPerWarp; ++jj) {
        const int j = half * kChunksPerWarp + jj;
        const int c0 = cb * kTileN + j * kChunkCols;
        if (jj + 2 < kChunksPerWarp) load_diag(w_ring[(jj + 2) % 3], jj + 2);
        const float4* w_cur = w_ring[jj % 3];
        uint32_t v[32];
        tmem_ld32(tmem_base + lane_addr + static_cast<uint32_t>(acc * kTileN) + j * kChunkCols, v);
        tmem_ld_wait();
        if (jj == kChunksPerWarp - 1) {
          // the warp's accumulator reads are done: one lane releases the buffer
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[acc]);
        }
        if (row0 >= d_out || c0 >= d_in) continue;  // the whole block lies outside the output
        if (lane == 0) bulk_wait_group_read<1>();
        __syncwarp();
        float* sbuf = staging + buf * (kChunkCols * 32);
        float4* srow = reinterpret_cast<float4*>(sbuf + lane * kChunkCols);  // this thread's row
        if (dense_diag != nullptr) {
          // the diagonal block into the buffer (row 4u + lane / 8 per load), then back out by row
#pragma unroll
          for (int u = 0; u < kChunkCols / 4; ++u) {
            const int rr = 4 * u + (lane >> 3);
            reinterpret_cast<float4*>(sbuf + rr * kChunkCols)[(lane & 7) ^ (rr & 7)] = w_cur[u];
          }
          __syncwarp();
        }
#pragma unroll
        for (int u = 0; u < kChunkCols / 4; ++u) {
          float4 x = make_float4(__uint_as_float(v[4 * u]), __uint_as_float(v[4 * u + 1]),
                                 __uint_as_float(v[4 * u + 2]), __uint_as_float(v[4 * u + 3]));
          if (dense_diag != nullptr) {  // out-of-range pieces carry weight 1 and are clipped by the store
            const float4 w = srow[u ^ (lane & 7)];
            x.x *= w.x;
            x.y *= w.y;
            x.z *= w.z;
            x.w *= w.w;
          }
          srow[u ^ (lane & 7)] = x;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (accumulate)
            tma_reduce_add_3d(&tm_out, sbuf, c0, row0, b);
          else
            tma_store_3d(&tm_out, sbuf, c0, row0, b);
          bulk_commit_group();
        }
        buf ^= 1;
      }
      if (++acc == 2) {
        acc = 0;
        aph ^= 1;
      }
    }
    if (lane == 0) bulk_wait_group<0>();  // every store has landed before the CTA exits
  } else {
    // ------------------------------------------------------------ epilogue
    // EPI / 4 warps per TMEM lane quarter share a tile's chunks round-robin: 32-column chunks
    // with 8 warps, 16-column chunks with 12 (fewer registers per thread, more warps to hide
    // the latency of the table loads and of the updates).
    constexpr int kGroups = EPI / 4;
    constexpr int kCols = EPI == 8 ? 32 : (EPI == 12 ? 16 : 8);
    constexpr int kChunks = kTileN / kCols;
    constexpr int kPairs = kCols / 2;
    const int et = threadIdx.x - 64;          // 0 .. 32 * EPI - 1
    const int q = warp & 3;                   // TMEM lane quarter this warp may access
    const int grp = (warp - 2) >> 2;          // chunks grp, grp + kGroups, ...
    const int r = q * 32 + lane;              // tile row owned by this thread
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t kk32 = static_cast<uint32_t>(k);
    const uint32_t ksm32 = static_cast<uint32_t>(k_sm);
    const uint64_t table_policy = l2_policy_evict_last();
    int acc = 0;
    uint32_t aph = 0;
    uint32_t epi_phase = 0;
    int64_t cur_job = -1;
    int scale_exp = 0;      // fixed-point scale S = 2^scale_exp of the current candidate
    bool scaled = false;    // a scale has been chosen for the current candidate
    bool bad = false;
    bool ok = true;
    // release an accumulator to the MMA issuer once the whole warp is done with it: one
    // arrival per warp on this CTA's barrier (a pair's second CTA: relayed by its MMA warp)
    auto release = [&](int a) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[a]);
    };
    for (int64_t job = worker; job < n_jobs && ok; job += n_workers)
    for (int tile = job_tile_begin(job, groups, n_tiles, unit); tile < job_tile_end(job, groups, n_tiles, unit) && ok; ++tile) {
      const int b = static_cast<int>(job / groups);
      float* out_row = phi + (int64_t)(b / rows_div) * k;
      if (smem_sketch && job != cur_job) {
        if (cur_job >= 0 && !flush_sketch(sk, phi + (cur_job / groups / rows_div) * k, k_sm, scale_exp, et, 32 * EPI,
                                          epi_bar, epi_phase, abort_flag, err)) {
          ok = false;
          break;
        }
        cur_job = job;
        scaled = false;
      }
      if (!mbar_wait(&tfull[acc], aph, abort_flag, err, kDevTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // this CTA's o-block; past d_out (the second o-block of a pair when their count is odd)
      // the accumulator rows are zeros and there is no table tile: release the accumulator only
      const int ob = PAIR ? 2 * walk.ob(tile) + (int)rank : walk.ob(tile);
      if (PAIR && ob >= n_ob_real) {
        release(acc);
        if (++acc == 2) {
          acc = 0;
          aph ^= 1;
        }
        continue;
      }
      const int cb = walk.cb(tile);
      const uint4* tp = table + ((int64_t)ob * n_cb + cb) * kEntriesPerTile + r;
      const uint32_t col0 = static_cast<uint32_t>(acc * kTileN);
      // chunks that hold a column below d_in, none if this warp's 32 rows lie past d_out: the
      // table pads the rest with bucket 0 and weight 0, whose updates add nothing
      const int n_live = ob * kTileM + q * 32 >= d_out ? 0 : min(kChunks, ceil_div(d_in - cb * kTileN, kCols));
      // chunk j: its table entries (column pairs j * kPairs ..) in flight, then its accumulator columns
      auto load_chunk = [&](int j, uint4(&ent)[kPairs], uint32_t(&v)[kCols]) {
#pragma unroll
        for (int p = 0; p < kPairs; ++p) ent[p] = ld_table(tp + (j * kPairs + p) * kTileM, table_policy);
        if constexpr (kCols == 32)
          tmem_ld32(tmem_base + lane_addr + col0 + j * kCols, v);
        else if constexpr (kCols == 16)
          tmem_ld16(tmem_base + lane_addr + col0 + j * kCols, v);
        else
          tmem_ld8(tmem_base + lane_addr + col0 + j * kCols, v);
        tmem_ld_wait();
      };
      if (smem_sketch && !scaled) {
        // First tile of this job: scale from max |w G| over a sample of the tile, the first
        // live chunk of every warp (1/8 of the tile with 16 warps).  The sample's maximum is at
        // most the tile's, so the scale is at least as fine as a whole-tile one; a value more
        // than 16 times the sample's maximum takes the exact f32 path.
        float m = 0.0f;
        if (grp < n_live) {
          const int j = grp;
          uint4 ent[kPairs];
          uint32_t v[kCols];
          load_chunk(j, ent, v);
#pragma unroll
          for (int p = 0; p < kPairs; ++p) {
            const uint4 e = ent[p];
            const float x0 = fabsf(__uint_as_float(v[2 * p]) * __uint_as_float(e.z) * alpha);
            const float x1 = fabsf(__uint_as_float(v[2 * p + 1]) * __uint_as_float(e.w) * alpha);
            if (x0 <= 3.0e38f) m = fmaxf(m, x0);   // finite values only
            if (x1 <= 3.0e38f) m = fmaxf(m, x1);
          }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        if (lane == 0) atomicMax(tile_max_bits, __float_as_int(m));
        if (!epi_sync(epi_bar, epi_phase, abort_flag, err)) {
          ok = false;
          break;
        }
        const float tmax = __int_as_float(*const_cast<volatile int*>(tile_max_bits));
        if (tmax > 0.0f) {
          int e2;
          frexpf(tmax, &e2);                       // tmax < 2^e2
          int se = cap_log2 - kHeadroomLog2 - e2;  // tmax * 2^se < cap / 16
          se = max(-120, min(120, se));
          scale_exp = se;
          scaled = true;
        }
        if (!epi_sync(epi_bar, epi_phase, abort_flag, err)) {  // everyone has read the maximum
          ok = false;
          break;
        }
        if (et == 0) *tile_max_bits = 0;
      }
      const float S = ldexpf(1.0f, scale_exp);
      const bool use_int = smem_sketch && scaled;
      if (grp >= n_live) release(acc);  // nothing of this tile to scatter for this warp
#pragma unroll 1
      for (int j = grp; j < n_live; j += kGroups) {
        uint4 ent[kPairs];
        uint32_t v[kCols];
        load_chunk(j, ent, v);
        if (j + kGroups >= n_live) release(acc);  // the warp's accumulator reads are done
#pragma unroll
        for (int p = 0; p < kPairs; ++p) {
          const uint4 e = ent[p];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t bucket = h ? e.y : e.x;
            const float x = __uint_as_float(v[2 * p + h]) * __uint_as_float(h ? e.w : e.z) * alpha;
            if (bucket >= kk32) {
              bad = true;
              continue;
            }
            const float y = x * S;
            if (use_int && bucket < ksm32 && fabsf(y) < cap) {
              atomicAdd(sk + bucket, __float2int_rn(y));
            } else if (x != 0.0f) {
              atomicAdd(out_row + bucket, x);   // outlier, non-finite, unscaled or no shared sketch
            }
          }
        }
      }
      if (++acc == 2) {
        acc = 0;
        aph ^= 1;
      }
    }
    if (ok && smem_sketch && cur_job >= 0)
      flush_sketch(sk, phi + (cur_job / groups / rows_div) * k, k_sm, scale_exp, et, 32 * EPI, epi_bar, epi_phase,
                   abort_flag, err);
    if (bad) record_device_error(err, kDevBadBucket);
  }

  tc_fence_before();
  __syncthreads();
  // a pair: the leader's MMAs are drained, both epilogues are done with TMEM and every
  // arrival that crosses the pair has landed before either CTA frees TMEM or exits
  if constexpr (PAIR) cluster_sync();
  tc_fence_after();
  if (warp == 1) {
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, kTmemCols);
    else
      tmem_dealloc(tmem_base, kTmemCols);
  }
}

SmemPlan plan_smem(int64_t k, int kStageBytes = kStageBytes64) {
  const size_t limit = static_cast<size_t>(max_smem_optin());
  const size_t fixed = 1024 /*alignment slack*/ + 16 + 8 * (2 * 8 + 6) + 32;
  SmemPlan p{0, 0, 0};
  for (int st = 6; st >= 2; --st) {
    const size_t need = fixed + (size_t)st * kStageBytes + (size_t)k * 4;
    if (need <= limit) {
      p = {st, k, need};
      return p;
    }
  }
  // The whole sketch does not fit next to two stages.  Keep the largest
  // prefix of the buckets (a multiple of 1024) that does: updates of those
  // buckets stay in shared memory, the rest go to L2 atomics, whose rate
  // bounds the kernel at this size, so coverage beats a third stage.
  if (fixed + 2 * (size_t)kStageBytes < limit) {
    const int64_t k_sm = static_cast<int64_t>((limit - fixed - 2 * (size_t)kStageBytes) / 4) & ~int64_t(1023);
    if (k_sm >= 4096) return {2, k_sm < k ? k_sm : k, fixed + 2 * (size_t)kStageBytes + (size_t)k_sm * 4};
  }
  // No room for a useful prefix: scatter straight into HBM/L2.
  for (int st = 4; st >= 2; --st) {
    const size_t need = fixed + (size_t)st * kStageBytes;
    if (need <= limit) return {st, 0, need};
  }
  return p;
}

// TMA maps of the two operands: dLdZ [n_rows, seq_len, d_out] and
// a [n_rows, seq_len, d_in], bf16, boxes of 64 features x bk tokens.
int encode_operands(const void* dLdZ, const void* a, int n_rows, int seq_len, int d_out, int d_in, CUtensorMap* tm_g,
                    CUtensorMap* tm_a, int bk = 64) {
  {
    const uint64_t dims[3] = {(uint64_t)d_out, (uint64_t)seq_len, (uint64_t)n_rows};
    const uint64_t strides[2] = {(uint64_t)d_out * 2, (uint64_t)seq_len * d_out * 2};
    const uint32_t box[3] = {kBoxMN, (uint32_t)bk, 1};
    int rc = encode_tmap(tm_g, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, dLdZ, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  const uint64_t dims[3] = {(uint64_t)d_in, (uint64_t)seq_len, (uint64_t)n_rows};
  const uint64_t strides[2] = {(uint64_t)d_in * 2, (uint64_t)seq_len * d_in * 2};
  const uint32_t box[3] = {kBoxMN, (uint32_t)bk, 1};
  return encode_tmap(tm_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

struct JobPlan {
  int groups;
  int unit;      // tiles per unit of a job range: 1, or a whole run of the outer index
  int cb_major;  // tile walk (TileWalk)
  int64_t n_jobs;
  int grid;
};

// Walk and job cut, from measurements on the GPT-2-XL and Qwen3 layer shapes
// (k = 65536 / 131072):
//  - d_in <= d_out, or many rows: o-block major, jobs of single tiles, so a
//    launch with few rows (a pass of the whole path, proxies merged into long
//    rows) still fills every SM;
//  - d_in > d_out with up to 64 rows (the passes of the whole path): column
//    block major, jobs cut at whole columns while the rows have enough columns
//    to fill every worker (tiles otherwise: one merged proxy row of 4096 ->
//    1024 has 16 columns, 93 against 492 TFLOP/s).  Each job then loads each
//    of its wide activation tiles once and re-reads only the narrow dLdZ
//    tiles, which every candidate in flight keeps in L2 (6400 -> 1600 at 24
//    rows: 418 against 348 TFLOP/s).
// Each candidate's walk is split into `groups` jobs so that the rounds of jobs
// over the SMs waste the least time: minimise ceil(jobs / SMs) x (tiles per
// job + 1), the 1 standing for a job's fixed cost (its sketch flush and the
// scale pass over a sample of its first tile), preferring larger jobs on ties.
// OPUS_SKETCH_ORDER=ob|cb and OPUS_SKETCH_JOBS=tiles|lines force either choice.
JobPlan plan_jobs(int n_rows, int d_out, int d_in, int n_ob, int workers) {
  const int sms = workers;  // CTAs, or CTA pairs, that take jobs
  const int n_cb = ceil_div(d_in, kTileN);
  const int64_t n_tiles = (int64_t)n_ob * n_cb;
  int cb_major = d_in > d_out && n_rows <= 64 ? 1 : 0;
  if (const char* env = getenv("OPUS_SKETCH_ORDER")) {
    if (strcmp(env, "cb") == 0) cb_major = 1;
    if (strcmp(env, "ob") == 0) cb_major = 0;
  }
  bool lines = cb_major != 0 && (int64_t)n_rows * n_cb >= sms;
  if (const char* env = getenv("OPUS_SKETCH_JOBS")) {
    if (strcmp(env, "lines") == 0) lines = true;
    if (strcmp(env, "tiles") == 0) lines = false;
  }
  const int unit = lines ? (cb_major ? n_ob : n_cb) : 1;
  const int64_t n_units = n_tiles / unit;
  int groups = 1;
  int64_t best = -1;
  for (int64_t q = 1; q <= n_units; ++q) {
    const int64_t jobs = (int64_t)n_rows * q;
    const int64_t cost = ((jobs + sms - 1) / sms) * (((n_units + q - 1) / q) * unit + 1);
    if (best < 0 || cost < best) {
      best = cost;
      groups = static_cast<int>(q);
    }
  }
  const int64_t n_jobs = (int64_t)n_rows * groups;
  return {groups, unit, cb_major, n_jobs, static_cast<int>(n_jobs < sms ? n_jobs : sms)};
}

}  // namespace
}  // namespace opus

using namespace opus;

// Epilogue warps of the scatter launches.  The epilogue is latency-bound (table
// loads and update issue), and more warps on narrower chunks hide more of it
// (interleaved launches at 24 and 128 rows, TFLOP/s for 8 / 12 / 16 warps):
//   pairs on 64-token stages, k = 65536: 1600 -> 6400 at 24 rows 459 / 495 / 521,
//     6400 -> 1600 432 / 473 / 511: 16 warps (8-column chunks);
//   one CTA with the whole sketch next to three stages or more (k <= 16384): 768 -> 3072
//     at 64 rows 734 / 799 / 815, 768 -> 768 486 / 531 / 545: 16 warps; with two stages
//     next to the sketch (1024 -> 4096 at k = 32768, 128 rows 752 / 749 / 719): 12;
//   pairs on 32-token stages (k > 65536): 2048 -> 6144 at 24 rows 450 / 438 / 429: 8.
// OPUS_SKETCH_EPI_WARPS (8, 12 or 16) forces one.
int epilogue_warps(bool pair, bool short_stages, bool deep_pipeline) {
  if (const char* env = getenv("OPUS_SKETCH_EPI_WARPS")) {
    const int w = atoi(env);
    return w == 12 || w == 16 ? w : 8;
  }
  if (!pair) return deep_pipeline ? 16 : 12;
  return short_stages ? 8 : 16;
}

// Shared memory of one CTA of a pair: stages of `stage` bytes (32 KB at 64
// tokens, 16 KB at 32).  The whole sketch with as many stages (3 to 6) as fit;
// otherwise `pref_stages` stages and the largest prefix of the buckets next to them.
SmemPlan plan_smem_pair(int64_t k, bool sketch_on_chip, size_t stage, int pref_stages) {
  const size_t limit = static_cast<size_t>(max_smem_optin());
  const size_t fixed = 1024 /*alignment slack*/ + 16 + 8 * (2 * 8 + 6) + 32;
  if (!sketch_on_chip) {
    for (int st = 6; st >= 2; --st)
      if (fixed + st * stage <= limit) return {st, 0, fixed + st * stage};
    return {0, 0, 0};
  }
  for (int st = 6; st >= 3; --st)
    if (fixed + st * stage + (size_t)k * 4 <= limit) return {st, k, fixed + st * stage + (size_t)k * 4};
  const int st = pref_stages;
  if (fixed + st * stage >= limit) return {0, 0, 0};
  int64_t k_sm = static_cast<int64_t>((limit - fixed - st * stage) / 4) & ~int64_t(1023);
  if (k_sm > k) k_sm = k;
  if (k_sm < 4096) k_sm = 0;
  return {st, k_sm, fixed + st * stage + (size_t)k_sm * 4};
}

// The CTA-pair launch of opus_sketch_gemm (OPUS_SKETCH_PAIR=1): clusters of two
// CTAs, as many as the device keeps resident, each pair taking jobs over
// o-block pairs x column blocks.
int launch_pair(const void* dLdZ, const void* a, const void* table, float* phi, int n_rows, int seq_len,
                int d_out, int d_in, int64_t k, int max_bucket_load, int rows_div, float cap, int cap_log2,
                int accumulate, float alpha, cudaStream_t st) {
  // Pipeline, measured with interleaved launches at 24 and 128 rows: up to k = 65536 two
  // 64-token stages (32 KB) next to 40960 buckets beat three stages next to 32768 (1600 -> 6400:
  // 491 against 470 TFLOP/s at 24 rows); at k = 131072 three 32-token stages (16 KB) next to
  // 45056 buckets win (2048 -> 6144: 459 against 426).  OPUS_SKETCH_PAIR_STAGE_TOKENS (64 or
  // 32) and OPUS_SKETCH_PAIR_STAGES force either.
  int bk = k > 65536 ? 32 : 64;
  if (const char* env = getenv("OPUS_SKETCH_PAIR_STAGE_TOKENS")) bk = atoi(env) == 32 ? 32 : 64;
  int pref = bk == 32 ? 3 : 2;
  if (const char* env = getenv("OPUS_SKETCH_PAIR_STAGES")) pref = atoi(env) >= 2 && atoi(env) <= 6 ? atoi(env) : pref;
  const SmemPlan plan = plan_smem_pair(k, max_bucket_load > 0, bk == 32 ? kStageBytesPair32 : kStageBytesPair64,
                                       pref);
  if (plan.stages == 0) return set_error(OPUS_ERR_UNSUPPORTED, "sketch_gemm: shared memory too small for CTA pairs");
  CUtensorMap tm_g, tm_a;
  if (int rc = encode_operands(dLdZ, a, n_rows, seq_len, d_out, d_in, &tm_g, &tm_a, bk)) return rc;
  const int epi = epilogue_warps(true, bk == 32, plan.stages >= 3);
  auto kernel = bk == 32 ? (epi == 16 ? sketch_gemm_kernel<32, true, 16>
                             : epi == 12 ? sketch_gemm_kernel<32, true, 12> : sketch_gemm_kernel<32, true, 8>)
                         : (epi == 16 ? sketch_gemm_kernel<64, true, 16>
                             : epi == 12 ? sketch_gemm_kernel<64, true, 12> : sketch_gemm_kernel<64, true, 8>);
  OPUS_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(plan.bytes)));
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * (sm_count() / 2), 1, 1);
  cfg.blockDim = dim3(block_threads(epi), 1, 1);
  cfg.dynamicSmemBytes = plan.bytes;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int pairs = 0;
  OPUS_CUDA_TRY(cudaOccupancyMaxActiveClusters(&pairs, kernel, &cfg));
  if (pairs <= 0) return set_error(OPUS_ERR_UNSUPPORTED, "sketch_gemm: no CTA pair fits on the device");
  const int n_op = ceil_div(ceil_div(d_out, kTileM), 2), n_cb = ceil_div(d_in, kTileN);
  const JobPlan jp = plan_jobs(n_rows, d_out, d_in, n_op, pairs);
  cfg.gridDim = dim3(2 * jp.grid, 1, 1);
  int* err = device_error_word();
  OPUS_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, tm_g, tm_a, tm_g /*no dense output*/,
                                   reinterpret_cast<const uint4*>(table), phi, n_rows, seq_len, n_op * n_cb, jp.unit,
                                   jp.cb_major, n_cb, jp.groups, k, rows_div, plan.stages, plan.k_sm, cap, cap_log2,
                                   err, /*dense*/ 0, static_cast<const float*>(nullptr), d_out, d_in, accumulate,
                                   alpha));
  ::opus::note_launch();
  return OPUS_OK;
}

// CTA pairs, on layers of two o-blocks or more with a fixed-point bound: each
// CTA stages half of a tile's activation columns (a third less operand traffic
// per SM), and for sketches larger than one CTA's shared memory (k > 32768) the
// memory saved holds more of the sketch (40960 or 45056 buckets against
// 32768), so fewer updates go to L2.  With 16 epilogue warps they also win
// where the whole sketch fits (k = 32768, 64 rows: 1024 -> 1024 659 against 530
// TFLOP/s, 1024 -> 4096 850 against 735); at k = 16384 only with many rows
// (768 -> 3072: 931 against 897 at 256 rows, 739 against 801 at 64).
// OPUS_SKETCH_PAIR=1 or 0 forces either.
bool use_pairs(int d_out, int64_t k, int max_bucket_load, int n_rows) {
  if (ceil_div(d_out, kTileM) < 2) return false;
  if (const char* env = getenv("OPUS_SKETCH_PAIR")) return strcmp(env, "1") == 0;
  return max_bucket_load > 0 && (k > 16384 || n_rows >= 256);
}

extern "C" int opus_sketch_gemm(const void* dLdZ, const void* a, int dtype, int n_rows, int seq_len, int d_out,
                                int d_in, const void* table, int64_t table_entries_given, int64_t k,
                                int max_bucket_load, int rows_div, float* phi, int accumulate, float alpha,
                                void* stream) {
  if (dtype != OPUS_DTYPE_BF16)
    return set_error(OPUS_ERR_UNSUPPORTED,
                     "sketch_gemm: operands must be bf16 (split f32 operands into bf16 hi/lo with opus_split_bf16)");
  if (n_rows < 0 || seq_len < 0 || d_out <= 0 || d_in <= 0 || k <= 0 || k > 0x7FFFFFFF || rows_div <= 0)
    return set_error(OPUS_ERR_INVALID, "sketch_gemm: bad sizes (n=%d T=%d d_out=%d d_in=%d k=%lld rows_div=%d)",
                     n_rows, seq_len, d_out, d_in, (long long)k, rows_div);
  if (!table || (n_rows > 0 && !phi) || (n_rows > 0 && seq_len > 0 && (!dLdZ || !a)))
    return set_error(OPUS_ERR_INVALID, "sketch_gemm: NULL pointer");
  if (table_entries_given < table_entries(d_out, d_in))
    return set_error(OPUS_ERR_INVALID, "sketch_gemm: table holds %lld entries, need %lld",
                     (long long)table_entries_given, (long long)table_entries(d_out, d_in));
  if (d_out % 8 != 0 || d_in % 8 != 0)
    return set_error(OPUS_ERR_UNSUPPORTED, "sketch_gemm: d_out and d_in must be multiples of 8 (got %d, %d)", d_out,
                     d_in);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t out_rows = n_rows == 0 ? 0 : (n_rows + rows_div - 1) / rows_div;
  if (!accumulate && out_rows > 0) OPUS_CUDA_TRY(cudaMemsetAsync(phi, 0, (size_t)out_rows * k * sizeof(float), st));
  if (n_rows == 0 || seq_len == 0) return OPUS_OK;

  SmemPlan plan = plan_smem(k);
  if (plan.stages == 0) return set_error(OPUS_ERR_UNSUPPORTED, "sketch_gemm: shared memory too small");
  // Fixed-point cap: max_bucket_load admitted updates of magnitude <= cap sum to < 2^31.
  float cap = 0.0f;
  int cap_log2 = 0;
  if (max_bucket_load > 0) {
    const int64_t cap_int = 0x7FFFFFFFll / max_bucket_load;
    cap = static_cast<float>(cap_int);
    if (static_cast<double>(cap) > static_cast<double>(cap_int)) cap = nextafterf(cap, 0.0f);
    while ((int64_t(1) << (cap_log2 + 1)) <= cap_int) ++cap_log2;
    if (cap_log2 < 2 * kHeadroomLog2) max_bucket_load = 0;  // too little range left for fixed point
  }
  // A sketch larger than shared memory sends the updates of the buckets outside the shared
  // prefix to L2 reductions.  32-token stages (24 KB) leave room for 45056 buckets instead of
  // 32768 but feed the MMAs from a shorter pipeline: measured at 128 candidates, they lose at
  // k = 65536 (445 against 462 TFLOP/s at 1600 -> 6400) and win at k = 131072 (469 against
  // 391 at 2048 -> 6144), so they are taken when less than half of the sketch fits with
  // 64-token stages.  OPUS_SKETCH_STAGE_TOKENS=64 or 32 forces one depth.
  int bk = 64;
  if (max_bucket_load > 0 && plan.k_sm * 2 < k) {
    const SmemPlan p32 = plan_smem(k, kStageBytes32);
    if (p32.stages > 0 && p32.k_sm > plan.k_sm) {
      plan = p32;
      bk = 32;
    }
  }
  if (const char* env = getenv("OPUS_SKETCH_STAGE_TOKENS")) {
    const int want = atoi(env);
    if ((want == 32 || want == 64) && want != bk) {
      const SmemPlan pf = plan_smem(k, want == 32 ? kStageBytes32 : kStageBytes64);
      if (pf.stages > 0) {
        plan = pf;
        bk = want;
      }
    }
  }
  if (use_pairs(d_out, k, max_bucket_load, n_rows))
    return launch_pair(dLdZ, a, table, phi, n_rows, seq_len, d_out, d_in, k, max_bucket_load, rows_div, cap,
                       cap_log2, accumulate, alpha, st);
  const int stage_bytes = bk == 32 ? kStageBytes32 : kStageBytes64;
  if (max_bucket_load <= 0 && plan.k_sm > 0) {
    // No usable bound: every update goes to global f32 atomics; use the smem for stages.
    for (int stg = 4; stg >= 2; --stg) {
      const size_t need =
          plan.bytes - (size_t)plan.stages * stage_bytes - (size_t)plan.k_sm * 4 + (size_t)stg * stage_bytes;
      if (need <= static_cast<size_t>(max_smem_optin())) {
        plan = {stg, 0, need};
        break;
      }
    }
  }
  CUtensorMap tm_g, tm_a;
  if (int rc = encode_operands(dLdZ, a, n_rows, seq_len, d_out, d_in, &tm_g, &tm_a, bk)) return rc;
  const int epi = epilogue_warps(false, false, plan.stages >= 3 && plan.k_sm >= k);
  auto kernel = bk == 32 ? (epi == 16 ? sketch_gemm_kernel<32, false, 16>
                             : epi == 12 ? sketch_gemm_kernel<32, false, 12> : sketch_gemm_kernel<32, false, 8>)
                         : (epi == 16 ? sketch_gemm_kernel<64, false, 16>
                             : epi == 12 ? sketch_gemm_kernel<64, false, 12> : sketch_gemm_kernel<64, false, 8>);
  OPUS_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(plan.bytes)));
  const int n_cb = ceil_div(d_in, kTileN), n_tiles = ceil_div(d_out, kTileM) * n_cb;
  const JobPlan jp = plan_jobs(n_rows, d_out, d_in, ceil_div(d_out, kTileM), sm_count());
  int* err = device_error_word();
  kernel<<<jp.grid, block_threads(epi), plan.bytes, st>>>(
      tm_g, tm_a, tm_g /*no dense output*/, reinterpret_cast<const uint4*>(table), phi, n_rows, seq_len, n_tiles,
      jp.unit, jp.cb_major, n_cb, jp.groups, k, rows_div, plan.stages, plan.k_sm, cap, cap_log2, err, /*dense*/ 0,
      nullptr, d_out, d_in, accumulate, alpha);
  ::opus::note_launch();
  OPUS_CUDA_TRY(cudaGetLastError());
  return OPUS_OK;
}

extern "C" int opus_per_sample_grad(const void* dLdZ, const void* a, int dtype, int n_rows, int seq_len, int d_out,
                                    int d_in, const float* diag, float* out, int accumulate, void* stream) {
  if (dtype != OPUS_DTYPE_BF16)
    return set_error(OPUS_ERR_UNSUPPORTED,
                     "per_sample_grad: operands must be bf16 (split f32 operands into bf16 hi/lo with opus_split_bf16)");
  if (n_rows < 0 || seq_len < 0 || d_out <= 0 || d_in <= 0)
    return set_error(OPUS_ERR_INVALID, "per_sample_grad: bad sizes (n=%d T=%d d_out=%d d_in=%d)", n_rows, seq_len,
                     d_out, d_in);
  if (d_out % 8 != 0 || d_in % 8 != 0)
    return set_error(OPUS_ERR_UNSUPPORTED, "per_sample_grad: d_out and d_in must be multiples of 8 (got %d, %d)",
                     d_out, d_in);
  if ((n_rows > 0 && !out) || (n_rows > 0 && seq_len > 0 && (!dLdZ || !a)))
    return set_error(OPUS_ERR_INVALID, "per_sample_grad: NULL pointer");
  if (n_rows == 0) return OPUS_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t numel = (int64_t)d_out * d_in;
  if (seq_len == 0) {  // no tokens: every gradient is zero
    if (!accumulate) OPUS_CUDA_TRY(cudaMemsetAsync(out, 0, (size_t)n_rows * numel * sizeof(float), st));
    return OPUS_OK;
  }
  CUtensorMap tm_g, tm_a;
  if (int rc = encode_operands(dLdZ, a, n_rows, seq_len, d_out, d_in, &tm_g, &tm_a)) return rc;
  // the output as [n_rows][d_out][d_in] f32, 32 x 32 boxes, 128-byte swizzle
  CUtensorMap tm_out;
  {
    const uint64_t dims[3] = {(uint64_t)d_in, (uint64_t)d_out, (uint64_t)n_rows};
    const uint64_t strides[2] = {(uint64_t)d_in * 4, (uint64_t)numel * 4};
    const uint32_t box[3] = {kChunkCols, 32, 1};
    if (int rc = encode_tmap(&tm_out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, out, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  }
  // the epilogue's staging (two 32 x 32 f32 boxes per epilogue warp) takes the place of the sketch
  constexpr int64_t kStagingWords = (int64_t)kEpiWarps * 2 * kChunkCols * 32;
  const SmemPlan plan = plan_smem(kStagingWords);
  if (plan.stages == 0 || plan.k_sm < kStagingWords)
    return set_error(OPUS_ERR_UNSUPPORTED, "per_sample_grad: shared memory too small");
  OPUS_CUDA_TRY(cudaFuncSetAttribute(sketch_gemm_kernel<64, false, kEpiWarps>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(plan.bytes)));
  const int n_cb = ceil_div(d_in, kTileN), n_tiles = ceil_div(d_out, kTileM) * n_cb;
  const JobPlan jp = plan_jobs(n_rows, d_out, d_in, ceil_div(d_out, kTileM), sm_count());
  int* err = device_error_word();
  sketch_gemm_kernel<64, false, kEpiWarps><<<jp.grid, kThreads, plan.bytes, st>>>(
      tm_g, tm_a, tm_out, nullptr, out, n_rows, seq_len, n_tiles, jp.unit, jp.cb_major, n_cb, jp.groups, numel, 1,
      plan.stages, plan.k_sm, 0.0f, 0, err, /*dense*/ 1, diag, d_out, d_in, accumulate, 1.0f);
  ::opus::note_launch();
  OPUS_CUDA_TRY(cudaGetLastError());
  return OPUS_OK;
}
