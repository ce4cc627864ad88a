// nq8_layout.h -- packed Q8_0 weight layout shared by host and device code.
//
//   tiles[n_tiles = ceil(N/128)][kc = ceil(K/64)], each kTileBytes = 8704 B:
//     [0, 8192)    int8 qs[128 rows][64 k]  (row-major, 64 B per row)
//     [8192, 8704) f16  d [128 rows][2]     (the two Q8_0 scales of the row)
//   One contiguous chunk per tile, so one cp.async.bulk moves it to shared
//   memory.  Rows beyond N and k beyond K are zero blocks (d = 0).
//   NQ_PACK_GLU weights hold 64 value rows and their 64 gate rows per tile.
#pragma once

namespace nq {
constexpr int kPackRows = 128;
constexpr int kPackK = 64;
constexpr int kTileQsBytes = kPackRows * kPackK;         // 8192
constexpr int kTileScaleBytes = kPackRows * 2 * 2;       // 512
constexpr int kTileBytes = kTileQsBytes + kTileScaleBytes;  // 8704
}  // namespace nq
