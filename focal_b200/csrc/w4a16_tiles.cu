// Offline re-layout of W4A16 weights into the unit-tiled format of
// w4a16_tiles.h, and its inverse.  Replaces no reference code: the reference
// keeps the [N, K/8] packing (focal_w4a16/__init__.py:38-54) and lists a
// tensor-core-friendly re-layout as next work.  The inverse proves that the
// format round-trips to the reference packing bit for bit.
//
// One thread per 16-byte chunk of a tile: 512 weight chunks (a 16-byte load
// of four packed words, stored at its swizzled position) and 32 scale / zero
// chunks (four rows' group pairs, gathered with 4-byte loads).
#include "common.cuh"
#include "host_common.h"
#include "w4a16_tiles.h"

namespace focal {
namespace tiles {

constexpr int kChunksPerTile = kTileBytes / 16;  // 544

// Byte offsets of chunk ci of unit (rb, st) in the reference arrays: a weight
// chunk maps to 16 bytes of wq, a scale / zero chunk to four 4-byte pieces.
template <bool kToTiles>
__global__ void relayout_kernel(uint8_t* __restrict__ tiles, uint32_t* __restrict__ wq, uint32_t* __restrict__ sc,
                                uint32_t* __restrict__ ze, int K, int N, long long chunks) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= chunks) return;
  const int TS = K / kUnitK;
  const long long u = i / kChunksPerTile;
  const int ci = (int)(i - u * kChunksPerTile);
  const int rb = (int)(u / TS), st = (int)(u - (long long)rb * TS);
  uint4* t = reinterpret_cast<uint4*>(tiles + u * kTileBytes) + ci;
  if (ci < 512) {
    const int r = ci >> 3, c = (ci & 7) ^ (r & 7);  // chunk position ci holds chunk c of row r
    uint4* w = reinterpret_cast<uint4*>(wq + ((size_t)rb * kUnitRows + r) * (K / 8) + st * 32 + 4 * c);
    if (kToTiles)
      *t = *w;
    else
      *w = *t;
  } else {
    const int k = ci - 512;                // 0..15 scales, 16..31 zeros
    uint32_t* arr = k < 16 ? sc : ze;      // [N, K/128] fp16, two groups per 4 bytes
    const int r0 = 4 * (k & 15);
    const int G2 = K / kUnitK;             // 4-byte group pairs per row
    uint32_t* src = arr + ((size_t)rb * kUnitRows + r0) * G2 + st;
    if (kToTiles) {
      *t = make_uint4(src[0], src[G2], src[2 * G2], src[3 * G2]);
    } else {
      const uint4 v = *t;
      src[0] = v.x;
      src[G2] = v.y;
      src[2 * G2] = v.z;
      src[3 * G2] = v.w;
    }
  }
}

int check(int K, int N, const void* tiles, const void* wq, const void* s, const void* z) {
  if (N <= 0 || N % kUnitRows != 0 || K <= 0 || K % kUnitK != 0)
    return set_error(FOCAL_ERR_UNSUPPORTED, "unsupported K/N");
  if (!tiles || !wq || !s || !z) return set_error(FOCAL_ERR_INVALID_VALUE, "null pointer");
  if (!aligned(tiles, 16) || !aligned(wq, 16) || !aligned(s, 4) || !aligned(z, 4))
    return set_error(FOCAL_ERR_INVALID_VALUE, "tiles and wq must be 16-byte, scales and zeros 4-byte aligned");
  return FOCAL_OK;
}

template <bool kToTiles>
int launch(uint8_t* t, uint32_t* wq, uint32_t* s, uint32_t* z, int K, int N, cudaStream_t stream) {
  const long long chunks = (long long)(N / kUnitRows) * (K / kUnitK) * kChunksPerTile;
  const int threads = 256;
  const long long blocks = (chunks + threads - 1) / threads;
  relayout_kernel<kToTiles><<<(unsigned)blocks, threads, 0, stream>>>(t, wq, s, z, K, N, chunks);
  return check_cuda(cudaGetLastError(), "relayout_kernel launch");
}

}  // namespace tiles
}  // namespace focal

using namespace focal;

extern "C" {

size_t focal_w4a16_tiles_size(int K, int N) {
  if (N <= 0 || N % tiles::kUnitRows != 0 || K <= 0 || K % tiles::kUnitK != 0) return 0;
  return tiles::tiles_bytes(K, N);
}

int focal_w4a16_tile_pack(const int32_t* wq, const void* scales, const void* zeros, void* tiles, int K, int N,
                          cudaStream_t stream) {
  clear_error();
  int rc = tiles::check(K, N, tiles, wq, scales, zeros);
  if (rc) return rc;
  return tiles::launch<true>(static_cast<uint8_t*>(tiles), (uint32_t*)wq, (uint32_t*)scales, (uint32_t*)zeros, K,
                             N, stream);
}

int focal_w4a16_tile_unpack(const void* tiles, int32_t* wq, void* scales, void* zeros, int K, int N,
                            cudaStream_t stream) {
  clear_error();
  int rc = tiles::check(K, N, tiles, wq, scales, zeros);
  if (rc) return rc;
  return tiles::launch<false>((uint8_t*)tiles, (uint32_t*)wq, (uint32_t*)scales, (uint32_t*)zeros, K, N, stream);
}

}  // extern "C"
