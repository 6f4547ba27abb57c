// Contiguous-KV GQA decode attention for B200 (sm_100a), split-KV
// ("flash-decoding") with a log-sum-exp combine.
//
//   o[b, h, :] = softmax(q[b, h, :] . K[b, g]^T * scale) . V[b, g],   g = h / (Hq / Hkv)
//
// New component (the reference has no attention code).  One CTA handles one
// (batch, KV head) and a contiguous range of 64-position tiles:
//  * warp 4 (producer) streams K and V tiles (64 positions x 128 dims, bf16)
//    with 3-D TMA boxes (64 dims x 64 positions x 1 head, 128-byte swizzle)
//    into a 3-stage ring; positions past L are zero-filled by TMA and masked;
//  * warps 0-3 (consumers) each take 16 positions of every tile and serve all
//    q heads of the KV head at once: the group's q heads are the M side of
//    mma.sync m16n8k16 (bf16 in, fp32 accumulate), so each K/V element is
//    read from shared memory once per CTA for every head that uses it;
//    S = Q K^T uses ldmatrix fragments of K, P V uses ldmatrix.trans of V with
//    P kept in registers;
//  * online softmax in the log2 domain per warp, merged across the four warps
//    in shared memory, then across splits by the last CTA to finish (an
//    arrival counter per (b, kv head) in the caller's workspace).
//
// Paged variant (PAGED = true): the caches are pages [num_pages, Hkv,
// page_size, 128] shared by all sequences, a block table maps page j of
// sequence b to its page, and each sequence has its own length.  The
// producer warp looks the pages up (32 block-table entries per warp-wide
// load) and loads each tile with 4-D TMA boxes of min(page_size, 64) rows,
// so shared memory holds the same swizzled tile as in the contiguous case
// (16-row pages need 16 boxes per tile and run about 21% below contiguous
// speed; 64-row and larger pages match it).  Rows past a sequence's end are
// masked in S; their V rows are zeroed in shared memory before P V (a stale
// NaN times p = 0 would still be NaN).  A sequence uses only the splits its
// length needs; block-table entries or lengths out of range set the device
// status (kDevBadIndex) and are clamped.
#include <cmath>
#include <cstdlib>

#include "common.cuh"
#include "host_common.h"

namespace focal {
namespace attn {

constexpr int kD = 128;
constexpr int kTile = 64;              // positions per stage
constexpr int kConsumerWarps = 4;      // 16 positions each
constexpr int kThreads = 32 * (kConsumerWarps + 1);
constexpr int kStages = 3;       // ring stages at two CTAs per SM
constexpr int kStagesDeep = 6;   // ring stages when a plan gives each SM one CTA
constexpr int kHalfBytes = kTile * 128;        // 64 positions x 64 dims x 2 B
constexpr int kKVStageBytes = 4 * kHalfBytes;  // K lo/hi + V lo/hi
constexpr int kMaxGroup = 16;
constexpr int kMaxSplits = 128;
constexpr int kCounterBytes = 256;     // counters region granularity
constexpr int kCombineBatch = 8;      // split partials loaded together by the combining CTA

struct Params {
  const int32_t* block_table;  // paged: [B, max_pages]
  const int32_t* seq_lens;     // paged: [B], 1 .. L
  int page_size, max_pages, num_pages;
  const __nv_bfloat16* q;
  __nv_bfloat16* o;
  float* part_o;   // [BH][S][grp][128]
  float* part_ml;  // [BH][S][grp][2]  (max in log2 domain, sum)
  unsigned int* counters;  // [BH]
  int* status;
  int Hq, Hkv, grp, L, tiles, tiles_per_split, splits;  // paged: L is the longest allowed sequence
  float scale_log2;
};

// smem: ring (re-used for the warp partials O [4][16][128] f32 after the last
// stage) | m,l [4][16][2] | flag | barriers.  About 98 KB: two CTAs per SM.
constexpr int kRingBytes = kStages * kKVStageBytes;
constexpr int kWarpOBytes = kConsumerWarps * kMaxGroup * kD * 4;
constexpr int kWarpMLBytes = kConsumerWarps * kMaxGroup * 2 * 4;
__host__ __device__ constexpr int smem_bytes(int st) { return 1024 + st * kKVStageBytes + kWarpMLBytes + 16 + 2 * st * 8; }
static_assert(kWarpOBytes <= kRingBytes, "warp partials alias the K/V ring");

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// byte offset of 16-byte chunk `c` (0..15 across the 128 dims) of position row `p` in a tile
__device__ __forceinline__ uint32_t tile_off(int p, int c) {
  return (c >> 3) * kHalfBytes + p * 128 + (((c & 7) ^ (p & 7)) << 4);
}

template <bool PAGED, int ST>
__global__ void __launch_bounds__(kThreads, 1)
    gqa_decode_kernel(const __grid_constant__ CUtensorMap tmap_k,
                      const __grid_constant__ CUtensorMap tmap_v, const Params p) {
  constexpr int kStages = ST;  // ring depth of this instantiation
  constexpr int kRingBytes = ST * kKVStageBytes;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw);
  const uint32_t ring = base;
  float* warp_o = reinterpret_cast<float*>(base_ptr);  // aliases the ring once it is drained
  float* warp_ml = reinterpret_cast<float*>(base_ptr + kRingBytes);
  int* last_flag = reinterpret_cast<int*>(base_ptr + kRingBytes + kWarpMLBytes);
  const uint32_t full_bar = base + kRingBytes + kWarpMLBytes + 16;
  const uint32_t empty_bar = full_bar + kStages * 8;

  const int split = blockIdx.x;
  const int bh = blockIdx.y;  // b * Hkv + kv head
  const int b = bh / p.Hkv;
  const int kvh = bh - b * p.Hkv;
  const int t0 = split * p.tiles_per_split;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full_bar + 8 * s, 1);
      mbar_init(empty_bar + 8 * s, kConsumerWarps);
    }
    fence_barrier_init();
    griddep_launch_dependents();
  }
  __syncthreads();
  // Launched with programmatic dependent launch: the set-up above overlaps the
  // previous kernel; q, the caches and the workspace are touched only after it.
  if (warp == kConsumerWarps && lane == 0) {
    prefetch_tensormap(&tmap_k);
    prefetch_tensormap(&tmap_v);
  }
  griddep_wait();

  // this sequence's length, tiles and splits (all of the grid's for contiguous caches)
  int L = p.L;
  if (PAGED) {
    L = p.seq_lens[b];
    if (L < 1 || L > p.L) {
      if (threadIdx.x == 0 && split == 0) set_status(p.status, kDevBadIndex);
      L = L < 1 ? 1 : p.L;
    }
  }
  const int tiles = PAGED ? (L + kTile - 1) / kTile : p.tiles;
  const int splits = PAGED ? (tiles + p.tiles_per_split - 1) / p.tiles_per_split : p.splits;
  const int nt = min(tiles, t0 + p.tiles_per_split) - t0;
  if (nt <= 0) return;  // a split past this sequence's end: nothing to do, no arrival

  if (PAGED && warp == kConsumerWarps) {
    // ------------------------------------------------------ paged producer
    const int rows = p.page_size >= kTile ? kTile : p.page_size;  // rows per box
    const int32_t* bt = p.block_table + (size_t)b * p.max_pages;
    const int first_page = (t0 * kTile) / p.page_size;
    const int last_page = (L - 1) / p.page_size;
    int chunk = -1, my_id = 0;
    // page id of page `pj` of the sequence (warp-uniform pj >= first_page),
    // from 32 block-table entries loaded by the warp at a time
    auto page_id = [&](int pj) {
      const int c = (pj - first_page) >> 5;
      if (c != chunk) {
        chunk = c;
        const int q = first_page + 32 * c + lane;
        my_id = q <= last_page ? bt[q] : 0;
        if (my_id < 0 || my_id >= p.num_pages) {
          set_status(p.status, kDevBadIndex);
          my_id = 0;
        }
      }
      return __shfl_sync(0xffffffffu, my_id, (pj - first_page) & 31);
    };
    const uint64_t pol = l2_policy_evict_first();
    bool ok = true;
    for (int i = 0; i < nt; ++i) {
      const int slot = i % kStages;
      if (i >= kStages) {
        bool w = true;
        if (lane == 0) w = mbar_wait_bounded(empty_bar + 8 * slot, ((i / kStages) - 1) & 1);
        if (!__shfl_sync(0xffffffffu, w ? 1 : 0, 0)) {
          ok = false;
          break;
        }
      }
      const uint32_t fb = full_bar + 8 * slot;
      const uint32_t dst = ring + slot * kKVStageBytes;
      const int pos = (t0 + i) * kTile;
      // pages of this tile that hold positions < L (boxes past the end are not loaded)
      const int npg = rows == kTile ? 1 : min(kTile / rows, (L - pos + rows - 1) / rows);
      const int row0 = rows == kTile ? pos % p.page_size : 0;
      if (lane == 0) mbar_arrive_expect_tx(fb, npg * 4 * rows * 128);
      for (int j = 0; j < npg; ++j) {
        const int id = page_id(pos / p.page_size + j);
        if (lane == 0) {
          const uint32_t dj = dst + j * rows * 128;
          tma_load_4d(dj + 0 * kHalfBytes, &tmap_k, 0, row0, kvh, id, fb, pol);
          tma_load_4d(dj + 1 * kHalfBytes, &tmap_k, 64, row0, kvh, id, fb, pol);
          tma_load_4d(dj + 2 * kHalfBytes, &tmap_v, 0, row0, kvh, id, fb, pol);
          tma_load_4d(dj + 3 * kHalfBytes, &tmap_v, 64, row0, kvh, id, fb, pol);
        }
      }
    }
    if (!ok && lane == 0 && p.status) set_status(p.status, kDevWaitTimeout);
    return;
  }
  if (!PAGED && warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    bool ok = true;
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      for (int i = 0; i < nt; ++i) {
        const int slot = i % kStages;
        if (i >= kStages && !mbar_wait_bounded(empty_bar + 8 * slot, ((i / kStages) - 1) & 1)) {
          ok = false;
          break;
        }
        const uint32_t fb = full_bar + 8 * slot;
        const uint32_t dst = ring + slot * kKVStageBytes;
        const int pos = (t0 + i) * kTile;
        mbar_arrive_expect_tx(fb, kKVStageBytes);
        tma_load_3d(dst + 0 * kHalfBytes, &tmap_k, 0, pos, bh, fb, pol);
        tma_load_3d(dst + 1 * kHalfBytes, &tmap_k, 64, pos, bh, fb, pol);
        tma_load_3d(dst + 2 * kHalfBytes, &tmap_v, 0, pos, bh, fb, pol);
        tma_load_3d(dst + 3 * kHalfBytes, &tmap_v, 64, pos, bh, fb, pol);
      }
      if (!ok && p.status) set_status(p.status, kDevWaitTimeout);
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int g = lane >> 2, t = lane & 3;
  const int grp = p.grp;
  const __nv_bfloat16* qb = p.q + ((size_t)b * p.Hq + (size_t)kvh * grp) * kD;

  // Q as the A operand: rows = the group's q heads (zero beyond grp), k = dims
  uint32_t qa[8][4];
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const int d0 = 16 * kk + 2 * t;
    qa[kk][0] = g < grp ? *reinterpret_cast<const uint32_t*>(qb + g * kD + d0) : 0u;
    qa[kk][1] = g + 8 < grp ? *reinterpret_cast<const uint32_t*>(qb + (g + 8) * kD + d0) : 0u;
    qa[kk][2] = g < grp ? *reinterpret_cast<const uint32_t*>(qb + g * kD + d0 + 8) : 0u;
    qa[kk][3] = g + 8 < grp ? *reinterpret_cast<const uint32_t*>(qb + (g + 8) * kD + d0 + 8) : 0u;
  }

  float oacc[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) oacc[j][0] = oacc[j][1] = oacc[j][2] = oacc[j][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY};  // running max (log2 domain) for rows g, g+8
  float lrow[2] = {0.f, 0.f};              // this thread's partial row sums

  const int pw = 16 * warp;  // first position of this warp inside a tile
  // ldmatrix row addresses: lane supplies row (lane & 7) of matrix (lane >> 3)
  const int lm = lane >> 3, lr = lane & 7;
  bool ok = true;

  for (int i = 0; i < nt; ++i) {
    const int slot = i % kStages;
    if (!mbar_wait_bounded(full_bar + 8 * slot, (i / kStages) & 1)) {
      ok = false;
      break;
    }
    const uint32_t kt = ring + slot * kKVStageBytes;
    const uint32_t vt = kt + 2 * kHalfBytes;
    if (PAGED && (t0 + i) * kTile + pw + 15 >= L) {
      // zero this warp's V rows past the sequence's end (loaded from the rest
      // of a page, or left from an earlier tile when their page was skipped)
      const int p0 = (t0 + i) * kTile + pw;
      for (int e = lane; e < 16 * 16; e += 32) {
        const int r = e >> 4, c = e & 15;
        if (p0 + r >= L) sts128(vt + tile_off(pw + r, c), make_uint4(0u, 0u, 0u, 0u));
      }
      __syncwarp();
    }

    // ---- S = Q K^T for positions pw .. pw+15 (two n-tiles of 8)
    float sacc[2][4];
#pragma unroll
    for (int n2 = 0; n2 < 2; ++n2) {
      sacc[n2][0] = sacc[n2][1] = sacc[n2][2] = sacc[n2][3] = 0.f;
      const int prow = pw + 8 * n2 + lr;
#pragma unroll
      for (int kk = 0; kk < 8; kk += 2) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(kt + tile_off(prow, 2 * kk + lm), b0, b1, b2, b3);
        mma_bf16_16816(sacc[n2], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
        mma_bf16_16816(sacc[n2], qa[kk + 1][0], qa[kk + 1][1], qa[kk + 1][2], qa[kk + 1][3], b2, b3);
      }
    }
    // ---- scale, mask, online softmax (rows g and g+8)
    const int pos0 = (t0 + i) * kTile + pw;
    float mt[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n2 = 0; n2 < 2; ++n2) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int pos = pos0 + 8 * n2 + 2 * t + (j & 1);
        const float s = pos < L ? sacc[n2][j] * p.scale_log2 : -INFINITY;
        sacc[n2][j] = s;
        mt[j >> 1] = fmaxf(mt[j >> 1], s);
      }
    }
    float alpha[2], mref[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mt[r] = fmaxf(mt[r], __shfl_xor_sync(0xffffffffu, mt[r], 1));
      mt[r] = fmaxf(mt[r], __shfl_xor_sync(0xffffffffu, mt[r], 2));
      const float mnew = fmaxf(mrow[r], mt[r]);
      mref[r] = mnew == -INFINITY ? 0.f : mnew;
      alpha[r] = fast_exp2(mrow[r] - mref[r]);
      mrow[r] = mnew;
      lrow[r] *= alpha[r];
    }
    uint32_t pa[4];
#pragma unroll
    for (int n2 = 0; n2 < 2; ++n2) {
      const float p0 = fast_exp2(sacc[n2][0] - mref[0]);
      const float p1 = fast_exp2(sacc[n2][1] - mref[0]);
      const float p2 = fast_exp2(sacc[n2][2] - mref[1]);
      const float p3 = fast_exp2(sacc[n2][3] - mref[1]);
      lrow[0] += p0 + p1;
      lrow[1] += p2 + p3;
      pa[2 * n2 + 0] = pack_bf16x2(p0, p1);  // row g,   positions 8*n2 + 2t, +1
      pa[2 * n2 + 1] = pack_bf16x2(p2, p3);  // row g+8
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      oacc[j][0] *= alpha[0];
      oacc[j][1] *= alpha[0];
      oacc[j][2] *= alpha[1];
      oacc[j][3] *= alpha[1];
    }
    // ---- O += P V : A = P (rows x 16 positions), B = V^T fragments via ldmatrix.trans
    const int vrow = pw + 8 * (lm & 1) + lr;
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      uint32_t b0, b1, b2, b3;
      ldmatrix_x4_trans(vt + tile_off(vrow, j + (lm >> 1)), b0, b1, b2, b3);
      mma_bf16_16816(oacc[j], pa[0], pa[1], pa[2], pa[3], b0, b1);
      mma_bf16_16816(oacc[j + 1], pa[0], pa[1], pa[2], pa[3], b2, b3);
    }
    fence_proxy_async_smem();  // our ldmatrix reads of this slot precede its TMA refill
    __syncwarp();
    if (lane == 0) mbar_arrive(empty_bar + 8 * slot);
  }
  if (!ok && p.status) set_status(p.status, kDevWaitTimeout);

  // ---- per-warp state -> shared memory (over the drained ring: wait for all warps)
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
  }
  named_barrier(1, kConsumerWarps * 32);
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = g + 8 * r;
    if (row < grp) {
      float* wo = warp_o + (warp * kMaxGroup + row) * kD;
#pragma unroll
      for (int j = 0; j < 16; ++j)
        *reinterpret_cast<float2*>(wo + 8 * j + 2 * t) = make_float2(oacc[j][2 * r], oacc[j][2 * r + 1]);
      if (t == 0) {
        warp_ml[(warp * kMaxGroup + row) * 2 + 0] = mrow[r];
        warp_ml[(warp * kMaxGroup + row) * 2 + 1] = lrow[r];
      }
    }
  }
  named_barrier(1, kConsumerWarps * 32);

  // ---- merge the four warps; each thread owns (row, 4 dims)
  const int ctid = threadIdx.x;  // 0..127
  const int nvals = grp * (kD / 4);
  for (int e = ctid; e < nvals; e += kConsumerWarps * 32) {
    const int row = e / (kD / 4);
    const int d = (e - row * (kD / 4)) * 4;
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) mm = fmaxf(mm, warp_ml[(w * kMaxGroup + row) * 2]);
    const float mu = mm == -INFINITY ? 0.f : mm;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float l = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      const float wgt = fast_exp2(warp_ml[(w * kMaxGroup + row) * 2] - mu);
      const float4 v = *reinterpret_cast<const float4*>(warp_o + (w * kMaxGroup + row) * kD + d);
      acc.x += wgt * v.x;
      acc.y += wgt * v.y;
      acc.z += wgt * v.z;
      acc.w += wgt * v.w;
      l += wgt * warp_ml[(w * kMaxGroup + row) * 2 + 1];
    }
    if (splits == 1) {
      const float inv = 1.0f / l;
      __nv_bfloat16* dst = p.o + ((size_t)b * p.Hq + (size_t)kvh * grp + row) * kD + d;
      *reinterpret_cast<uint2*>(dst) =
          make_uint2(pack_bf16x2(acc.x * inv, acc.y * inv), pack_bf16x2(acc.z * inv, acc.w * inv));
    } else {
      const size_t rec = ((size_t)bh * p.splits + split) * grp + row;
      *reinterpret_cast<float4*>(p.part_o + rec * kD + d) = acc;
      if (d == 0) *reinterpret_cast<float2*>(p.part_ml + rec * 2) = make_float2(mm, l);
    }
  }
  if (splits == 1) return;

  // ---- split combine by the last CTA of this (b, kv head)
  named_barrier(1, kConsumerWarps * 32);
  // The barrier orders this CTA's partial stores before thread 0's
  // acquire-release increment, which publishes them at GPU scope; in the last
  // CTA the same increment and the barrier after it order its loads.
  if (ctid == 0) {
    const unsigned int prev = atom_add_acq_rel_gpu(p.counters + bh, 1u);
    *last_flag = (prev == (unsigned int)(splits - 1));
  }
  named_barrier(1, kConsumerWarps * 32);
  if (!*last_flag) return;
  for (int e = ctid; e < nvals; e += kConsumerWarps * 32) {
    const int row = e / (kD / 4);
    const int d = (e - row * (kD / 4)) * 4;
    const size_t rec0 = (size_t)bh * p.splits * grp + row;
    // One pass in split order, kCombineBatch splits' partials loaded together
    // (one L2 round trip per batch), merged online: the running sums are
    // rescaled when a batch raises the running maximum.
    float mu = -INFINITY;  // running maximum (log2 domain)
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float l = 0.f;
    for (int s0 = 0; s0 < splits; s0 += kCombineBatch) {
      float2 ml[kCombineBatch];
      float4 v[kCombineBatch];
#pragma unroll
      for (int u = 0; u < kCombineBatch; ++u) {
        ml[u] = make_float2(-INFINITY, 0.f);
        v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (s0 + u < splits) {
          const size_t rec = rec0 + (size_t)(s0 + u) * grp;
          ml[u] = __ldcg(reinterpret_cast<const float2*>(p.part_ml + rec * 2));
          v[u] = __ldcg(reinterpret_cast<const float4*>(p.part_o + rec * kD + d));
        }
      }
      float nm = mu;
#pragma unroll
      for (int u = 0; u < kCombineBatch; ++u) nm = fmaxf(nm, ml[u].x);
      if (nm == -INFINITY) continue;  // nothing but empty splits so far
      const float r = fast_exp2(mu - nm);  // 0 while mu is still -inf
      acc.x *= r;
      acc.y *= r;
      acc.z *= r;
      acc.w *= r;
      l *= r;
#pragma unroll
      for (int u = 0; u < kCombineBatch; ++u) {
        const float wgt = fast_exp2(ml[u].x - nm);
        acc.x += wgt * v[u].x;
        acc.y += wgt * v[u].y;
        acc.z += wgt * v[u].z;
        acc.w += wgt * v[u].w;
        l += wgt * ml[u].y;
      }
      mu = nm;
    }
    const float inv = 1.0f / l;
    __nv_bfloat16* dst = p.o + ((size_t)b * p.Hq + (size_t)kvh * grp + row) * kD + d;
    *reinterpret_cast<uint2*>(dst) =
        make_uint2(pack_bf16x2(acc.x * inv, acc.y * inv), pack_bf16x2(acc.z * inv, acc.w * inv));
  }
  if (ctid == 0) p.counters[bh] = 0u;  // leave the counter zeroed for the next call
}

// ----------------------------------------------------------------- host side
struct Plan {
  int tiles, tiles_per_split, splits;
};

Plan make_plan(int B, int Hkv, int L, int sm_count) {
  Plan pl;
  pl.tiles = (L + kTile - 1) / kTile;
  const int bhn = B * Hkv;
  // Two CTAs per SM fit in shared memory; stay within one resident wave so
  // every CTA streams the same number of tiles at the same time.
  // One CTA per SM (launched with the 6-stage ring) when the (sequence, KV
  // head) pairs times their splits still cover 90 % of the SMs, or when the
  // sequence is short (at most four tiles per split at one CTA per SM): fewer,
  // longer splits with a deeper ring then beat more, shorter ones (B=1,
  // L=4096: 9.1 -> 7.7 us; B=4, L=512: 5.7 -> 5.4 us).  Otherwise two CTAs per
  // SM, so more splits start at once.  FOCAL_ATTN_CTAS_PER_SM forces either (tuning).
  static const int per_sm_env = [] {
    const char* e = getenv("FOCAL_ATTN_CTAS_PER_SM");
    return e && atoi(e) > 0 ? atoi(e) : 0;
  }();
  static const int min_tiles = [] {  // tuning override
    const char* e = getenv("FOCAL_ATTN_MIN_TILES");
    return e && atoi(e) > 0 ? atoi(e) : 1;
  }();
  int per_sm = per_sm_env;
  if (per_sm == 0) {
    const int s1 = sm_count / bhn;
    const bool covers = s1 >= 1 && 10 * bhn * s1 >= 9 * sm_count;
    const bool short_seq = s1 >= 1 && pl.tiles <= 4 * s1;
    per_sm = (covers || short_seq) ? 1 : 2;
  }
  const int target = per_sm * sm_count;
  int s = target / bhn;
  s = s < 1 ? 1 : s;
  s = s > pl.tiles ? pl.tiles : s;
  if (min_tiles > 1 && s > 1 && pl.tiles / s < min_tiles) s = pl.tiles / min_tiles > 1 ? pl.tiles / min_tiles : 1;
  s = s > kMaxSplits ? kMaxSplits : s;
  pl.tiles_per_split = (pl.tiles + s - 1) / s;
  pl.splits = (pl.tiles + pl.tiles_per_split - 1) / pl.tiles_per_split;
  return pl;
}

size_t workspace_size(int B, int Hq, int Hkv, int L) {
  const int bhn = B * Hkv;
  const int tiles = (L + kTile - 1) / kTile;
  const int smax = tiles < kMaxSplits ? tiles : kMaxSplits;
  const int grp = Hq / Hkv;
  const size_t counters = ((size_t)bhn * 4 + kCounterBytes - 1) / kCounterBytes * kCounterBytes;
  const size_t recs = (size_t)bhn * smax * grp;
  return counters + recs * kD * 4 + recs * 2 * 4;
}

int check(int B, int Hq, int Hkv, int L, int D) {
  if (B < 1 || Hq < 1 || Hkv < 1 || L < 1) return set_error(FOCAL_ERR_UNSUPPORTED, "B, Hq, Hkv and L must be positive");
  if (D != kD) return set_error(FOCAL_ERR_UNSUPPORTED, "unsupported head_dim (must be 128)");
  if (Hq % Hkv != 0) return set_error(FOCAL_ERR_UNSUPPORTED, "Hq must be a multiple of Hkv");
  if (Hq / Hkv > kMaxGroup) return set_error(FOCAL_ERR_UNSUPPORTED, "Hq / Hkv must be <= 16");
  if ((long long)B * Hkv > 65535) return set_error(FOCAL_ERR_UNSUPPORTED, "B * Hkv too large");
  return FOCAL_OK;
}

// Parameters common to both layouts; the split partials and counters come
// from the workspace when the plan splits the sequence.
int fill_params(Params* pp, const void* q, void* o, int B, int Hq, int Hkv, int L, float scale, const Plan& pl,
                void* workspace, size_t ws_bytes, const DeviceInfo& dev) {
  Params& p = *pp;
  p = Params{};
  const int grp = Hq / Hkv;
  const int bhn = B * Hkv;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.o = static_cast<__nv_bfloat16*>(o);
  if (pl.splits > 1) {
    const size_t need = workspace_size(B, Hq, Hkv, L);
    if (!workspace || ws_bytes < need)
      return set_error(FOCAL_ERR_WORKSPACE, "workspace too small: need %zu bytes, got %zu", need, ws_bytes);
    if (!aligned(workspace, 256)) return set_error(FOCAL_ERR_INVALID_VALUE, "workspace must be 256-byte aligned");
    const size_t counters = ((size_t)bhn * 4 + kCounterBytes - 1) / kCounterBytes * kCounterBytes;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    p.counters = reinterpret_cast<unsigned int*>(ws);
    p.part_o = reinterpret_cast<float*>(ws + counters);
    p.part_ml = p.part_o + (size_t)bhn * pl.splits * grp * kD;
  }
  p.status = dev.status;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.grp = grp;
  p.L = L;
  p.tiles = pl.tiles;
  p.tiles_per_split = pl.tiles_per_split;
  p.splits = pl.splits;
  p.scale_log2 = scale * 1.4426950408889634f;
  return FOCAL_OK;
}

template <bool PAGED, int ST>
int launch_st(const CUtensorMap& mk, const CUtensorMap& mv, const Params& p, int bhn, cudaStream_t stream) {
  auto kern = gqa_decode_kernel<PAGED, ST>;
  constexpr int kSmemBytes = smem_bytes(ST);
  static_assert(smem_bytes(ST) <= 227 * 1024, "shared memory per CTA");
  int rc = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), (PAGED ? 41 : 40) + (ST == kStages ? 0 : 2),
                               kSmemBytes);
  if (rc) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.splits, bhn, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, mk, mv, p), "gqa_decode_kernel launch");
}

// Two CTAs per SM use the 3-stage ring; a plan whose grid fits one CTA per SM
// gets the 6-stage ring (twice the bytes in flight per SM).
template <bool PAGED>
int launch(const CUtensorMap& mk, const CUtensorMap& mv, const Params& p, int bhn, cudaStream_t stream,
           int sm_count) {
  if (p.splits * bhn <= sm_count) return launch_st<PAGED, kStagesDeep>(mk, mv, p, bhn, stream);
  return launch_st<PAGED, kStages>(mk, mv, p, bhn, stream);
}

}  // namespace attn
}  // namespace focal

using namespace focal;

extern "C" {

size_t focal_gqa_decode_workspace_size(int B, int Hq, int Hkv, int L, int D) {
  if (attn::check(B, Hq, Hkv, L, D)) return 0;
  return attn::workspace_size(B, Hq, Hkv, L);
}

int focal_gqa_decode_attn(const void* q, const void* k, const void* v, void* o, int B, int Hq,
                          int Hkv, int L, int D, float scale, void* workspace, size_t ws_bytes,
                          cudaStream_t stream) {
  clear_error();
  int rc = attn::check(B, Hq, Hkv, L, D);
  if (rc) return rc;
  if (!q || !k || !v || !o) return set_error(FOCAL_ERR_INVALID_VALUE, "null pointer");
  if (!aligned(q, 4) || !aligned(o, 8) || !aligned(k, 16) || !aligned(v, 16))
    return set_error(FOCAL_ERR_INVALID_VALUE, "q/o must be 8-byte and k/v 16-byte aligned");
  if (!(scale > 0.f) || !std::isfinite(scale))
    return set_error(FOCAL_ERR_INVALID_VALUE, "scale must be positive and finite");
  DeviceInfo dev;
  rc = current_device_info(&dev);
  if (rc) return rc;
  const attn::Plan pl = attn::make_plan(B, Hkv, L, dev.sm_count);
  const int bhn = B * Hkv;
  attn::Params p;
  rc = attn::fill_params(&p, q, o, B, Hq, Hkv, L, scale, pl, workspace, ws_bytes, dev);
  if (rc) return rc;

  CUtensorMap mk, mv;
  const uint64_t dims[3] = {(uint64_t)attn::kD, (uint64_t)L, (uint64_t)bhn};
  const uint64_t strides[2] = {(uint64_t)attn::kD * 2, (uint64_t)L * attn::kD * 2};
  const uint32_t box[3] = {64, attn::kTile, 1};
  rc = encode_tensor_map(&mk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, k, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_tensor_map(&mv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, v, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;

  return attn::launch<false>(mk, mv, p, bhn, stream, dev.sm_count);
}

int focal_gqa_decode_paged(const void* q, const void* k_pages, const void* v_pages, const int32_t* block_table,
                           const int32_t* seq_lens, void* o, int B, int Hq, int Hkv, int D, int num_pages,
                           int page_size, int max_pages_per_seq, int max_seq_len, float scale, void* workspace,
                           size_t ws_bytes, cudaStream_t stream) {
  clear_error();
  int rc = attn::check(B, Hq, Hkv, max_seq_len, D);
  if (rc) return rc;
  if (page_size < 16 || page_size % 16 != 0 || (attn::kTile % page_size != 0 && page_size % attn::kTile != 0))
    return set_error(FOCAL_ERR_UNSUPPORTED, "page_size must be 16, 32 or a multiple of 64");
  if (num_pages < 1 || max_pages_per_seq < 1)
    return set_error(FOCAL_ERR_UNSUPPORTED, "num_pages and max_pages_per_seq must be positive");
  if ((long long)max_pages_per_seq * page_size < max_seq_len)
    return set_error(FOCAL_ERR_UNSUPPORTED, "max_seq_len exceeds max_pages_per_seq * page_size");
  if (!q || !k_pages || !v_pages || !block_table || !seq_lens || !o)
    return set_error(FOCAL_ERR_INVALID_VALUE, "null pointer");
  if (!aligned(q, 4) || !aligned(o, 8) || !aligned(k_pages, 16) || !aligned(v_pages, 16) ||
      !aligned(block_table, 4) || !aligned(seq_lens, 4))
    return set_error(FOCAL_ERR_INVALID_VALUE, "q/o must be 8-byte, pages 16-byte, tables 4-byte aligned");
  if (!(scale > 0.f) || !std::isfinite(scale))
    return set_error(FOCAL_ERR_INVALID_VALUE, "scale must be positive and finite");
  DeviceInfo dev;
  rc = current_device_info(&dev);
  if (rc) return rc;
  const attn::Plan pl = attn::make_plan(B, Hkv, max_seq_len, dev.sm_count);
  const int bhn = B * Hkv;
  attn::Params p;
  rc = attn::fill_params(&p, q, o, B, Hq, Hkv, max_seq_len, scale, pl, workspace, ws_bytes, dev);
  if (rc) return rc;
  p.block_table = block_table;
  p.seq_lens = seq_lens;
  p.page_size = page_size;
  p.max_pages = max_pages_per_seq;
  p.num_pages = num_pages;

  // [num_pages, Hkv, page_size, 128] pages; boxes of 64 dims x min(page_size, 64) rows
  CUtensorMap mk, mv;
  const uint64_t dims[4] = {(uint64_t)attn::kD, (uint64_t)page_size, (uint64_t)Hkv, (uint64_t)num_pages};
  const uint64_t strides[3] = {(uint64_t)attn::kD * 2, (uint64_t)page_size * attn::kD * 2,
                               (uint64_t)Hkv * page_size * attn::kD * 2};
  const uint32_t box[4] = {64, (uint32_t)(page_size < attn::kTile ? page_size : attn::kTile), 1, 1};
  rc = encode_tensor_map(&mk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, k_pages, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_tensor_map(&mv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, v_pages, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  return attn::launch<true>(mk, mv, p, bhn, stream, dev.sm_count);
}

}  // extern "C"
