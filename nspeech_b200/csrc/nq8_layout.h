// nq8_layout.h -- packed Q8_0 weight layout shared by host and device code.
//
//   tiles[n_tiles = ceil(N/128)][kc = ceil(K/64)], each kTileBytes = 8704 B:
//     [0, 8192)    int8 qs as [4 chunks of 16 k][128 rows][16 B]
//     [8192, 8704) f16  d  as [2 Q8_0 blocks][128 rows]
//   so that 32 consecutive rows of one 16-k chunk (or one scale) are one
//   contiguous, coalesced warp access.  One contiguous 8704-byte tile per
//   (row tile, k chunk): a single cp.async.bulk moves it to shared memory.
//   Rows beyond N and k beyond K are zero blocks (d = 0).
//   NQ_PACK_GLU weights hold 64 value rows and their 64 gate rows per tile.
#pragma once

namespace nq {
constexpr int kPackRows = 128;
constexpr int kPackK = 64;
constexpr int kTileQsBytes = kPackRows * kPackK;         // 8192
constexpr int kTileScaleBytes = kPackRows * 2 * 2;       // 512
constexpr int kTileBytes = kTileQsBytes + kTileScaleBytes;  // 8704

// Byte offset of row `r`'s 16-k chunk `c` (0..3), and of its Q8_0 scale `h`.
constexpr int qs_offset(int r, int c) { return (c * kPackRows + r) * 16; }
constexpr int scale_offset(int r, int h) { return kTileQsBytes + (h * kPackRows + r) * 2; }
}  // namespace nq
