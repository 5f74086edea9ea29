// Tile geometry shared by the epilogue-table builder and the fused
// per-sample sketch GEMM.
//
// A layer's [d_out, d_in] weight grid is cut into kTileM x kTileN tiles
// (tile index = ob * n_cb + cb).  Inside a tile, the sketch epilogue thread
// that owns TMEM lane r (= tile row r) walks the 256 columns in 8 chunks of
// 32; for column pair p of chunk j it reads one 16-byte entry
//   {bucket(c), bucket(c+1), w(c), w(c+1)},  c = 32 j + 2 p,
// stored at ((tile * 8 + j) * 16 + p) * 128 + r, so the 32 lanes of a warp
// read 512 contiguous bytes per load.  w = sign * preconditioner as f32 bits;
// elements outside [d_out, d_in] carry bucket 0 and weight 0.
#pragma once
#include <stdint.h>

namespace opus {

constexpr int kTileM = 128;  // weight rows (d_out) per tile = UMMA M = TMEM lanes
constexpr int kTileN = 256;  // weight columns (d_in) per tile = UMMA N = TMEM columns
constexpr int kChunkCols = 32;
constexpr int kChunksPerTile = kTileN / kChunkCols;     // 8
constexpr int kPairsPerChunk = kChunkCols / 2;          // 16
constexpr int64_t kEntriesPerTile = (int64_t)kChunksPerTile * kPairsPerChunk * kTileM;  // 16384

__host__ __device__ inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

__host__ __device__ inline int64_t table_entries(int d_out, int d_in) {
  return (int64_t)ceil_div(d_out, kTileM) * ceil_div(d_in, kTileN) * kEntriesPerTile;
}

}  // namespace opus
