// Unit-tiled W4A16 weight format (an offline re-layout of the reference's
// [N, K/8] int32 packing plus its fp16 scales / zeros [N, K/128]).
//
// Unit u = rb * (K / 256) + st covers weight rows 64 rb .. 64 rb + 63 and K
// values 256 st .. 256 st + 255, and is one contiguous chunk of kTileBytes:
//   [0, 8192)      the 64 rows x 32 packed words, row r at byte 128 r, its
//                  16-byte chunk c (words 4c .. 4c + 3) at chunk position
//                  c ^ (r & 7) — the image a 128-byte-swizzled TMA box of the
//                  reference layout leaves in shared memory;
//   [8192, 8448)   scales, row r at 8192 + 4 r: groups 2 st, 2 st + 1 (fp16);
//   [8448, 8704)   zeros, same arrangement.
// Units follow each other in u order, so a run of units is one contiguous
// stream and a unit arrives with two 1-D bulk copies.
#pragma once

#include <cstddef>
#include <cstdint>

namespace focal {
namespace tiles {

constexpr int kUnitRows = 64;
constexpr int kUnitK = 256;
constexpr uint32_t kWeightBytes = kUnitRows * 128;           // 8192
constexpr uint32_t kScalesOffset = kWeightBytes;             // 8192
constexpr uint32_t kZerosOffset = kWeightBytes + kUnitRows * 4;  // 8448
constexpr uint32_t kGroupBytes = 2 * kUnitRows * 4;          // scales + zeros, 512
constexpr uint32_t kTileBytes = kWeightBytes + kGroupBytes;  // 8704

inline size_t tiles_bytes(int K, int N) { return (size_t)(N / kUnitRows) * (K / kUnitK) * kTileBytes; }

}  // namespace tiles
}  // namespace focal
