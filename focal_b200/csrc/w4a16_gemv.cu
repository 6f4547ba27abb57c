// W4A16 small-M linear for B200 (sm_100a).
//
//   y[m, n] = bf16( sum_k x[m, k] * (q[n, k] - z[n, k/128]) * s[n, k/128] ),  M <= 8
//
// Replaces the reference's SIMT kernel and launcher (csrc/w4a16_gemv.cu:33-116,
// :152-223) behind the same packing and dequant semantics (README.md:66-73).
//
// Two kernels per call, chained with programmatic dependent launch:
//
// 1. x_prepare (O(M*K) work, once per call): the activations in the order of
//    the tensor core's B fragments plus their fp32 sums per 128-wide group,
//    one 16-byte-aligned record per 256 K values, into the caller's
//    workspace; it also clears the row-block arrival counters.
//
// 2. w4a16_gemv, stream-K over units of (64 weight rows x 256 K values):
//    the grid is exactly the number of CTAs that are resident at once, and
//    CTA c takes the contiguous unit range [c*U/P, (c+1)*U/P) in row-block-
//    major order, so every CTA streams the same number of bytes in a single
//    wave.  Inside a CTA:
//    * warp 8 (loader) fills a ring of 12 (gate/up: 8) slots.  Per unit: the packed
//      weights as one 2-D TMA box of 64 rows x 128 bytes (128-byte swizzle),
//      the unit's activation record as one bulk copy, and the fp16 scales and
//      zeros: when K % 1024 == 0, one 2-D TMA box each of 64 rows x 8 groups
//      per four units (a "quad", kept in its own 5-slot ring), otherwise the
//      unit's two groups per row with 4-byte cp.async.  All complete on the
//      slot's mbarrier.  Weight and scale/zero boxes of the first ring-full
//      start streaming before the previous kernel has finished (weights,
//      scales and zeros must not be written by a kernel that triggers
//      programmatic launch early); only the activation copies wait for it.
//    * warps 0-7 (consumers), in four pairs: pair p takes the CTA's units
//      i with i % 4 == p, so four units are consumed at once; the pair's two
//      warps take one quantisation group each, over all 64 rows (four 16-row
//      MMA tiles sharing one load of the group's activation fragments).  The
//      slot's empty barrier waits for those two warps.  A packed word becomes bf16
//      (128 + q) pairs with one shift and one LOP3 per pair, fed as the A
//      fragment of mma.sync m16n8k16 (bf16 in, fp32 accumulate); the <= 8
//      tokens are the n = 8 side.  Zero point and +128 factor out per group:
//          sum_k x (q - z) s = s * (sum_k x (128 + q) - (z + 128) sum_k x)
//      so the tensor core only sees exact small integers and x.
//    * at the end of each row block's run of units the eight warps' shares are
//      added in a fixed order, and the CTA either writes y
//      (it had the whole row block) or stores its fp32 partial; the last CTA
//      to arrive on the row block's counter adds all partials in CTA order
//      (deterministic, no waiting) and writes y.
//    No TMA multicast is used.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "host_common.h"

namespace focal {
namespace gemv {

constexpr int kStageK = 256;            // K values per unit / pipeline stage (two groups)
constexpr int kWordsPerStage = 32;      // int32 words per row per stage (128 B)
constexpr int kRowTiles = 4;            // 16-row MMA tiles per unit
constexpr int kRows = 16 * kRowTiles;   // weight rows per unit
constexpr int kPairs = 4;               // consumer warp pairs; pair p takes every 4th unit
constexpr int kConsumerWarps = 2 * kPairs;  // one warp per (pair, group of the unit)
constexpr int kConsumerThreads = 32 * kConsumerWarps;
constexpr int kLoaderWarp = kConsumerWarps;
constexpr int kThreads = 32 * (kConsumerWarps + 1);
// Ring slots: one resident CTA per SM (the 288-thread CTA is allocated as 12
// warps, so its registers fill the SM), holding 96 KB (12 x 8 KB) or, for the
// gate/up pair, 128 KB (8 x 16 KB) of weights in flight.
__host__ __device__ constexpr int stages_of(int NW) { return NW == 1 ? 12 : 8; }
constexpr int kMaxStages = 12;
constexpr int kMaxCtasPerSm = 4;        // occupancy bound used to size the workspace
constexpr int kSumBatch = 8;            // partial sums loaded together by a finishing CTA
constexpr int kMinUnitsPerCta = 4;      // below this, fewer CTAs beat more split overhead
// Scale/zero quad slots when they arrive by TMA.  Pairs consume units out of
// order, so a quad slot may only be refilled once every unit of the quad it
// held is known consumed: the loader knows that of unit u once it has issued
// unit u + stages.  With quads of four units (the first may have one) that
// takes ceil((stages + 7) / 4) slots: 5 for 12 stages, 4 for 8.
constexpr int kSzSlotsTma = 5;
static_assert(4 * kSzSlotsTma >= kMaxStages + 7, "too few scale/zero quad slots for the ring depth");
constexpr int kSzQuadGroups = 8;        // groups per scale/zero TMA box (16 bytes of fp16)
// bytes of scale/zero staging per weight matrix: the larger of the two modes
constexpr uint32_t kSzSlotBytes =
    (kSzSlotsTma * 2 * kRows * 16 > kMaxStages * 2 * kRows * 4) ? kSzSlotsTma * 2 * kRows * 16
                                                                : kMaxStages * 2 * kRows * 4;

enum Epi : int { kEpiBf16 = 0, kEpiF32 = 1, kEpiSiluMul = 2 };

// ---------------------------------------------------- activation records
// One record per unit column: [group G][token m][t][4 x 16 B] B fragments, then
// the fp32 group sums [G][MTp].  The fragment of lane 4g+t for chunk qq holds
// the pairs (x_j, x_{j+4}), j = 0..3, of K values 128G + 32t + 8qq + j, matching
// the nibble pairs (q_j, q_{j+4}) that one packed word yields.
__host__ __device__ constexpr int mtp_of(int MT) { return MT < 2 ? 2 : MT; }
__host__ __device__ constexpr uint32_t rec_frag_bytes(int MT) { return MT * 2 * 256; }
__host__ __device__ constexpr uint32_t rec_bytes(int MT) {
  return rec_frag_bytes(MT) + ((2 * mtp_of(MT) * 4 + 15) / 16) * 16;
}

// Byte offset of chunk qq of lane (g, t), group G, inside a record.  Rotating
// a lane's four chunks by (lane >> 1) keeps each 8-lane LDS.128 phase
// conflict-free.
__host__ __device__ constexpr uint32_t frag_offset(int MT, int G, int g, int t, int qq) {
  return ((G * MT + g) * 4 + t) * 64 + (((qq + ((4 * g + t) >> 1)) & 3) << 4);
}

// ------------------------------------------------- workspace layout
// [records: TS x rec_bytes][counters: RB x 4, padded to 256][partials: 2P slots]
struct WsLayout {
  size_t rec, counters, partials, total;
};

__host__ __device__ inline size_t slot_floats(int MT, int NW) { return (size_t)NW * MT * kRows; }

inline WsLayout ws_layout(int MT, int NW, int TS, int RB, int P) {
  WsLayout w;
  w.rec = 0;
  w.counters = (size_t)TS * rec_bytes(MT);
  w.partials = w.counters + ((size_t)RB * 4 + 255) / 256 * 256;
  w.total = w.partials + 2 * (size_t)P * slot_floats(MT, NW) * 4;
  return w;
}

struct PrepParams {
  const __nv_bfloat16* x;
  uint8_t* rec;
  unsigned int* counters;
  int M, K, stages, RB;
};

// One warp per (unit column, token): lane l takes K values 8l..8l+7.
template <int MT>
__global__ void __launch_bounds__(128) x_prepare_kernel(const PrepParams p) {
  griddep_launch_dependents();
  griddep_wait();  // x may be the previous kernel's output; the workspace may still be read by it
  constexpr int MTp = mtp_of(MT);
  if (blockIdx.x == 0)
    for (int r = threadIdx.x; r < p.RB; r += blockDim.x) p.counters[r] = 0u;
  const int lane = threadIdx.x & 31;
  const int item = blockIdx.x * 4 + (threadIdx.x >> 5);
  if (item >= p.stages * MTp) return;
  const int st = item / MTp, m = item - st * MTp;
  uint8_t* rec = p.rec + (size_t)st * rec_bytes(MT);
  uint4 v = make_uint4(0u, 0u, 0u, 0u);
  if (m < p.M)
    v = __ldg(reinterpret_cast<const uint4*>(p.x + (size_t)m * p.K + (size_t)st * kStageK) + lane);
  float sum = bf16_lo(v.x) + bf16_hi(v.x) + bf16_lo(v.y) + bf16_hi(v.y) + bf16_lo(v.z) + bf16_hi(v.z) +
              bf16_lo(v.w) + bf16_hi(v.w);
  sum += __shfl_xor_sync(0xffffffffu, sum, 1);
  sum += __shfl_xor_sync(0xffffffffu, sum, 2);
  sum += __shfl_xor_sync(0xffffffffu, sum, 4);
  sum += __shfl_xor_sync(0xffffffffu, sum, 8);
  const int G = lane >> 4, c = lane & 15;
  if (c == 0) reinterpret_cast<float*>(rec + rec_frag_bytes(MT))[G * MTp + m] = sum;
  if (m < MT) {
    uint4 pv;
    pv.x = prmt(v.x, v.z, 0x5410);
    pv.y = prmt(v.x, v.z, 0x7632);
    pv.z = prmt(v.y, v.w, 0x5410);
    pv.w = prmt(v.y, v.w, 0x7632);
    *reinterpret_cast<uint4*>(rec + frag_offset(MT, G, m, c >> 2, c & 3)) = pv;
  }
}

// ------------------------------------------------------------------ GEMV
struct Params {
  const uint8_t* rec;      // activation records (x_prepare output)
  unsigned int* counters;  // per row block arrivals (cleared by x_prepare)
  float* partials;         // [2P][NW][MT][64] split row-block partial sums
  const __half* scales0;
  const __half* zeros0;
  const __half* scales1;
  const __half* zeros1;
  void* y;
  int* status;
  int M, K, N, G, TS, RB, P;
  int sz_tma;   // scales / zeros by TMA quads (needs G % 8 == 0 and 16-byte aligned bases)
  long long U;  // units = RB * TS
};

struct Layout {
  uint32_t w, x, sz, red, flag, bars, total;
};

__host__ __device__ constexpr uint32_t round_up(uint32_t a, uint32_t b) { return (a + b - 1) / b * b; }

// Shared-memory carve-up, identical on host (sizing) and device (addressing).
template <int MT, int NW>
__host__ __device__ constexpr Layout make_layout() {
  Layout L{};
  uint32_t off = 0;
  L.w = off;  // [slot][mat][64 rows][128 B], 1024-aligned (swizzle atom)
  off += stages_of(NW) * NW * kRows * 128;
  L.x = off;  // [slot] activation record
  off += stages_of(NW) * rec_bytes(MT);
  // scale / zero slots, [slot][mat][scale|zero][64 rows][row bytes]: either
  // kSzSlotsTma slots of 16-byte rows (eight groups = four units, by TMA) or
  // one slot per ring slot of 4-byte rows (the unit's two groups, by cp.async)
  off = round_up(off, 128);
  L.sz = off;
  off += NW * kSzSlotBytes;
  L.red = off;  // [pair][mat][group][token][64 rows] fp32 shares of the current row block
  off += kPairs * NW * 2 * MT * kRows * 4;
  L.flag = off;  // "this CTA finishes the row block" broadcast
  off += 16;
  L.bars = round_up(off, 8);  // full[stages], empty[stages]
  off = L.bars + 2 * stages_of(NW) * 8;
  L.total = off + 1024;  // slack for aligning the base to 1024 B
  return L;
}

// CTA whose unit range contains unit x (ranges are [c*U/P, (c+1)*U/P)).
__host__ __device__ inline int unit_owner(long long x, long long U, int P) {
  return (int)(((x + 1) * P - 1) / U);
}

__host__ __device__ inline long long unit_begin(int c, long long U, int P) { return (U * c) / P; }

// Partial-sum slots: CTA c writes its first row block's partial to slot 2c and
// any later one to 2c + 1 (only the first and last can be partial).

template <int EPI, int NW>
__device__ __forceinline__ void store_out(void* y, size_t yi, const float (&v)[NW]) {
  if (EPI == kEpiBf16) {
    static_cast<__nv_bfloat16*>(y)[yi] = __float2bfloat16_rn(v[0]);
  } else if (EPI == kEpiF32) {
    static_cast<float*>(y)[yi] = v[0];
  } else {
    // silu(gate) * up with the roundings of the unfused bf16 path
    const float gt = __bfloat162float(__float2bfloat16_rn(v[0]));
    const float up = __bfloat162float(__float2bfloat16_rn(v[NW - 1]));
    const float sg = __bfloat162float(__float2bfloat16_rn(gt / (1.0f + expf(-gt))));
    static_cast<__nv_bfloat16*>(y)[yi] = __float2bfloat16_rn(sg * up);
  }
}

template <int MT, int NW, int EPI>
__global__ void __maxnreg__(160)
    w4a16_gemv_kernel(const __grid_constant__ CUtensorMap tmap0, const __grid_constant__ CUtensorMap tmap1,
                      const __grid_constant__ CUtensorMap tms0, const __grid_constant__ CUtensorMap tmz0,
                      const __grid_constant__ CUtensorMap tms1, const __grid_constant__ CUtensorMap tmz1,
                      const Params p) {
  constexpr int MTp = mtp_of(MT);
  constexpr Layout L = make_layout<MT, NW>();
  constexpr uint32_t kRec = rec_bytes(MT);
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* sm = smem_raw + (base - raw);  // generic pointer to the aligned base

  const int cta = blockIdx.x;
  const long long u0 = unit_begin(cta, p.U, p.P);
  const long long u1 = unit_begin(cta + 1, p.U, p.P);
  const int nu = (int)(u1 - u0);

  const uint32_t full_bar = base + L.bars;
  constexpr int kStages = stages_of(NW);
  const uint32_t empty_bar = full_bar + kStages * 8;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) {
      // the loader's expect_tx, plus 32 cp.async arrivals when scales / zeros use cp.async
      mbar_init(full_bar + 8 * s, p.sz_tma ? 1 : 1 + 32);
      mbar_init(empty_bar + 8 * s, 2);  // the two warps of the unit's pair
    }
    fence_barrier_init();
    griddep_launch_dependents();
  }
  __syncthreads();

  bool ok = true;
  if (warp == kLoaderWarp) {
    // -------------------------------------------------------------- loader
    if (lane == 0) {
      prefetch_tensormap(&tmap0);
      if (NW == 2) prefetch_tensormap(&tmap1);
      if (p.sz_tma) {
        prefetch_tensormap(&tms0);
        prefetch_tensormap(&tmz0);
        if (NW == 2) {
          prefetch_tensormap(&tms1);
          prefetch_tensormap(&tmz1);
        }
      }
    }
    const uint64_t pol = l2_policy_evict_first();
    const uint64_t pol_sz = l2_policy_evict_normal();
    // Unit (slot, rb, st): its weight boxes and, when it opens a scale/zero
    // quad (sz_slot >= 0), the quad's scale and zero boxes, all on the slot's
    // full barrier.  The activation record is added after griddep_wait.
    auto issue_unit = [&](int slot, int rb, int st, int sz_slot) {
      const uint32_t fb = full_bar + 8 * slot;
      mbar_arrive_expect_tx(fb, NW * kRows * 128 + kRec + (sz_slot >= 0 ? NW * 2 * kRows * 16 : 0));
      tma_load_2d(base + L.w + (slot * NW + 0) * kRows * 128, &tmap0, st * kWordsPerStage, rb * kRows, fb, pol);
      if (NW == 2)
        tma_load_2d(base + L.w + (slot * NW + 1) * kRows * 128, &tmap1, st * kWordsPerStage, rb * kRows, fb,
                    pol);
      if (sz_slot >= 0) {
        const uint32_t d = base + L.sz + sz_slot * NW * (2 * kRows * 16);
        const int gx = kSzQuadGroups * (st >> 2), gy = rb * kRows;
        tma_load_2d(d, &tms0, gx, gy, fb, pol_sz);
        tma_load_2d(d + kRows * 16, &tmz0, gx, gy, fb, pol_sz);
        if (NW == 2) {
          tma_load_2d(d + 2 * kRows * 16, &tms1, gx, gy, fb, pol_sz);
          tma_load_2d(d + 3 * kRows * 16, &tmz1, gx, gy, fb, pol_sz);
        }
      }
    };
    // A unit opens a quad when it is the CTA's first or starts a group of four
    // stages (quads never straddle row blocks: TS % 4 == 0 in this mode).
    int sz_next = 0;  // next quad slot
    auto quad_slot = [&](int i, int st) -> int {
      if (!p.sz_tma || (i != 0 && (st & 3) != 0)) return -1;
      const int q = sz_next;
      sz_next = (sz_next + 1 == kSzSlotsTma) ? 0 : sz_next + 1;
      return q;
    };
    // weights (and quads) of the first ring-full of units do not depend on the previous kernel
    {
      int rb = (int)(u0 / p.TS), st = (int)(u0 - (long long)rb * p.TS);
      for (int i = 0; i < min(nu, kStages); ++i) {
        const int q = quad_slot(i, st);
        if (lane == 0) issue_unit(i, rb, st, q);
        if (++st == p.TS) {
          st = 0;
          ++rb;
        }
      }
    }
    griddep_wait();  // the activation records come from the x_prepare kernel
    fence_proxy_async_global();
    int slot = 0;
    uint32_t phase = 0;  // phase of the empty barrier awaited on this lap of the ring
    int rb = (int)(u0 / p.TS), st = (int)(u0 - (long long)rb * p.TS);  // stepped per unit
    for (int i = 0; i < nu; ++i) {
      const uint32_t fb = full_bar + 8 * slot;
      if (i >= kStages) {
        if (!mbar_wait_bounded(empty_bar + 8 * slot, phase)) {
          ok = false;
          break;
        }
        const int q = quad_slot(i, st);
        if (lane == 0) issue_unit(slot, rb, st, q);
      }
      if (lane == 0) bulk_load(base + L.x + slot * kRec, p.rec + (size_t)st * kRec, kRec, fb);
      if (!p.sz_tma) {
        // scale / zero pairs (groups 2st, 2st+1) of the 64 rows: 4 bytes each
        const int row0 = rb * kRows;
#pragma unroll
        for (int j = lane; j < NW * 2 * kRows; j += 32) {
          const int mat = j / (2 * kRows);
          const int arr = (j / kRows) & 1;
          const int r = j % kRows;
          const __half* src = mat == 0 ? (arr ? p.zeros0 : p.scales0) : (arr ? p.zeros1 : p.scales1);
          src += (size_t)(row0 + r) * p.G + 2 * st;
          cp_async_4(base + L.sz + (((slot * NW + mat) * 2 + arr) * kRows + r) * 4, src);
        }
        cp_async_arrive_noinc(fb);
      }
      if (++slot == kStages) {
        slot = 0;
        if (i >= kStages) phase ^= 1u;  // laps after the first wait on alternating phases
      }
      if (++st == p.TS) {
        st = 0;
        ++rb;
      }
    }
    cp_async_wait<0>();  // no copy may land after this CTA exits
  } else {
    // ------------------------------------------------------------ consumers
    griddep_wait();  // the row-block counters are cleared by x_prepare
    const int tid = threadIdx.x;  // 0 .. kConsumerThreads-1
    const int g = lane >> 2, t = lane & 3;
    const int pair = warp >> 1;  // takes the units i of this CTA with i % kPairs == pair
    const int G = warp & 1;      // which quantisation group of those units this warp takes
    // Lane (g, t) covers rows pg + 8h, h = 0..7 (tile h/2, MMA row g or g+8): the
    // permutation keeps the swizzled reads conflict-free, and because every such
    // row is pg mod 8 the 128-byte swizzle maps chunk 4G+t to one column for all.
    const int pg = (g >> 1) + ((g & 1) << 2);
    const bool has_token = g < p.M;
    const int gc = g < MT ? g : 0;
    const int tok2 = 2 * t < MTp ? 2 * t : 0;
    const uint32_t kMask = 0x000F000Fu, kMagic = 0x43004300u;  // held in registers
    const uint32_t w_lane = L.w + pg * 128 + ((uint32_t)((4 * G + t) ^ pg) << 4);
    uint32_t x_off[4];
#pragma unroll
    for (int qq = 0; qq < 4; ++qq) x_off[qq] = L.x + frag_offset(MT, G, gc, t, qq);
    const uint32_t xs_off = L.x + rec_frag_bytes(MT) + (G * MTp + tok2) * 4;
    // scale/zero staging: 16-byte rows (quad of four units) or 4-byte rows (one unit)
    const uint32_t rs = p.sz_tma ? 16u : 4u;
    const uint32_t sz_mat = 2 * kRows * rs;  // bytes per (slot, mat)
    const uint32_t sz_lane = L.sz + pg * rs;
    const int half_shift = 16 * G;  // this group's fp16 within a scale/zero pair
    int sz_slot = -1;
    float acc[NW][kRowTiles][4];
#pragma unroll
    for (int mat = 0; mat < NW; ++mat)
#pragma unroll
      for (int tl = 0; tl < kRowTiles; ++tl)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[mat][tl][j] = 0.f;

    int slot = 0;
    uint32_t phase = 0;
    const int rb0 = (int)(u0 / p.TS);
    int rb = rb0, st = (int)(u0 - (long long)rb0 * p.TS);  // stepped per unit
    for (int i = 0; i < nu; ++i) {
      // the scale/zero slot of unit i (same sequence as the loader's)
      if (!p.sz_tma) {
        sz_slot = slot;
      } else if (i == 0 || (st & 3) == 0) {
        sz_slot = (sz_slot + 1 == kSzSlotsTma) ? 0 : sz_slot + 1;
      }
      if ((i & (kPairs - 1)) == pair) {
        // After a wait gives up, later waits are skipped (the result is garbage
        // and the status word is set) but every warp still takes the same path
        // through the row-block barriers below, so none of them can hang.
        if (ok && !mbar_wait_bounded(full_bar + 8 * slot, phase)) ok = false;
        const uint32_t xso = slot * kRec;                // this slot's activation record
        const uint32_t wso = slot * (NW * kRows * 128);  // this slot's weight boxes
        // B fragments: token g, K values 128G + 32t + 8qq + {j, j+4}
        uint32_t xb[16];
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          uint4 v = make_uint4(0u, 0u, 0u, 0u);
          if (has_token) v = ld_smem<uint4>(sm, x_off[qq] + xso);
          xb[4 * qq + 0] = v.x;
          xb[4 * qq + 1] = v.y;
          xb[4 * qq + 2] = v.z;
          xb[4 * qq + 3] = v.w;
        }
        // group sums of x for tokens 2t and 2t+1
        const float2 xs = ld_smem<float2>(sm, xs_off + xso);
        const uint32_t sz_col = p.sz_tma ? (uint32_t)(st & 3) * 4u : 0u;
#pragma unroll
        for (int mat = 0; mat < NW; ++mat) {
          const uint32_t sb = sz_lane + (sz_slot * NW + mat) * sz_mat + sz_col;
          const uint32_t wb = w_lane + wso + mat * kRows * 128;
          // every load of the unit first (one shared-memory latency), then the
          // four tiles' MMA chains interleaved
          uint4 wv[kRowTiles][2];
          uint32_t sv[kRowTiles][2], zv[kRowTiles][2];
#pragma unroll
          for (int tl = 0; tl < kRowTiles; ++tl) {
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
              const uint32_t r = 16 * tl + 8 * hf;  // rows beyond pg
              wv[tl][hf] = ld_smem<uint4>(sm, wb + r * 128);
              sv[tl][hf] = ld_smem<uint32_t>(sm, sb + r * rs) >> half_shift;
              zv[tl][hf] = ld_smem<uint32_t>(sm, sb + (kRows + r) * rs) >> half_shift;
            }
          }
          float d[kRowTiles][4];
#pragma unroll
          for (int tl = 0; tl < kRowTiles; ++tl)
#pragma unroll
            for (int j = 0; j < 4; ++j) d[tl][j] = 0.f;
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
#pragma unroll
              for (int tl = 0; tl < kRowTiles; ++tl) {
                const uint32_t wa = qq == 0 ? wv[tl][0].x : qq == 1 ? wv[tl][0].y : qq == 2 ? wv[tl][0].z : wv[tl][0].w;
                const uint32_t wr = qq == 0 ? wv[tl][1].x : qq == 1 ? wv[tl][1].y : qq == 2 ? wv[tl][1].z : wv[tl][1].w;
                mma_bf16_16816(d[tl], nib_pair_bf16(wa, 2 * h, kMask, kMagic), nib_pair_bf16(wr, 2 * h, kMask, kMagic),
                               nib_pair_bf16(wa, 2 * h + 1, kMask, kMagic),
                               nib_pair_bf16(wr, 2 * h + 1, kMask, kMagic), xb[4 * qq + 2 * h],
                               xb[4 * qq + 2 * h + 1]);
              }
            }
          }
#pragma unroll
          for (int tl = 0; tl < kRowTiles; ++tl) {
            const float s0 = half_lo(sv[tl][0]), s1 = half_lo(sv[tl][1]);
            const float z0 = half_lo(zv[tl][0]) + 128.0f, z1 = half_lo(zv[tl][1]) + 128.0f;
            acc[mat][tl][0] = fmaf(s0, fmaf(-z0, xs.x, d[tl][0]), acc[mat][tl][0]);
            acc[mat][tl][1] = fmaf(s0, fmaf(-z0, xs.y, d[tl][1]), acc[mat][tl][1]);
            acc[mat][tl][2] = fmaf(s1, fmaf(-z1, xs.x, d[tl][2]), acc[mat][tl][2]);
            acc[mat][tl][3] = fmaf(s1, fmaf(-z1, xs.y, d[tl][3]), acc[mat][tl][3]);
          }
        }
        fence_proxy_async_smem();  // our loads of this slot precede its TMA / bulk refill
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar + 8 * slot);
      }
      if (++slot == kStages) {
        slot = 0;
        phase ^= 1u;
      }

      // ------------------------------------------- end of a row-block run
      const bool run_ends = (i + 1 == nu) || (st + 1 == p.TS);
      if (run_ends) {
        // every warp's share: red[pair][mat][G][token][row]
#pragma unroll
        for (int mat = 0; mat < NW; ++mat) {
#pragma unroll
          for (int tl = 0; tl < kRowTiles; ++tl) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int tok = 2 * t + (j & 1);
              const int row = 16 * tl + pg + ((j < 2) ? 0 : 8);
              if (tok < MT)
                *reinterpret_cast<float*>(sm + L.red + ((((pair * NW + mat) * 2 + G) * MT + tok) * kRows + row) * 4) =
                    acc[mat][tl][j];
              acc[mat][tl][j] = 0.f;
            }
          }
        }
        named_barrier(1, kConsumerThreads);
        const long long rb_lo = (long long)rb * p.TS, rb_hi = rb_lo + p.TS;
        const int nout = p.M * kRows;
        // the eight shares of an output, added in a fixed order
        auto reduced = [&](int mat, int tok, int row) {
          float v = 0.f;
#pragma unroll
          for (int q = 0; q < kPairs * 2; ++q)
            v += ld_smem<float>(sm, L.red + ((((q >> 1) * NW + mat) * 2 + (q & 1)) * MT + tok) * kRows * 4 + row * 4);
          return v;
        };
        if (u0 <= rb_lo && u1 >= rb_hi) {
          // the whole row block was ours
          for (int o = tid; o < nout; o += kConsumerThreads) {
            const int tok = o / kRows, row = o - tok * kRows;
            float v[NW];
#pragma unroll
            for (int mat = 0; mat < NW; ++mat) v[mat] = reduced(mat, tok, row);
            store_out<EPI, NW>(p.y, (size_t)tok * p.N + (size_t)rb * kRows + row, v);
          }
        } else {
          // publish this CTA's partial; the last of the row block's CTAs finishes it
          float* mine = p.partials + (2LL * cta + (rb == rb0 ? 0 : 1)) * slot_floats(MT, NW);
          for (int o = tid; o < nout; o += kConsumerThreads) {
            const int tok = o / kRows, row = o - tok * kRows;
#pragma unroll
            for (int mat = 0; mat < NW; ++mat) mine[(mat * MT + tok) * kRows + row] = reduced(mat, tok, row);
          }
          __threadfence();
          named_barrier(1, kConsumerThreads);
          const int c_first = unit_owner(rb_lo, p.U, p.P), c_last = unit_owner(rb_hi - 1, p.U, p.P);
          if (tid == 0) {
            const unsigned int prev = atomicAdd(p.counters + rb, 1u);
            *reinterpret_cast<int*>(sm + L.flag) = (prev == (unsigned int)(c_last - c_first));
          }
          named_barrier(1, kConsumerThreads);
          if (ld_smem<int>(sm, L.flag)) {
            __threadfence();
            // Partial slots: a CTA after c_first began inside this row block (slot
            // 2c); c_first used slot 2c + 1 unless it began exactly at rb_lo.
            const long long first_slot = 2LL * c_first + (unit_begin(c_first, p.U, p.P) == rb_lo ? 0 : 1);
            for (int o = tid; o < nout; o += kConsumerThreads) {
              const int tok = o / kRows, row = o - tok * kRows;
              float v[NW];
#pragma unroll
              for (int mat = 0; mat < NW; ++mat) v[mat] = 0.f;
              // fixed order (deterministic sums); loads issued a batch at a time
              for (int cb = c_first; cb <= c_last; cb += kSumBatch) {
                float part[kSumBatch][NW];
#pragma unroll
                for (int j = 0; j < kSumBatch; ++j) {
                  const int c = cb + j;
                  const long long ps = c == c_first ? first_slot : 2LL * (c <= c_last ? c : cb);
                  const float* src = p.partials + ps * slot_floats(MT, NW);
#pragma unroll
                  for (int mat = 0; mat < NW; ++mat)
                    part[j][mat] = c <= c_last ? __ldcg(src + (mat * MT + tok) * kRows + row) : 0.f;
                }
#pragma unroll
                for (int j = 0; j < kSumBatch; ++j)
#pragma unroll
                  for (int mat = 0; mat < NW; ++mat) v[mat] += part[j][mat];
              }
              store_out<EPI, NW>(p.y, (size_t)tok * p.N + (size_t)rb * kRows + row, v);
            }
            if (tid == 0) p.counters[rb] = 0u;
          }
        }
        named_barrier(1, kConsumerThreads);  // red is rewritten by the next run
      }
      if (++st == p.TS) {
        st = 0;
        ++rb;
      }
    }
  }

  if (!ok && p.status) atomicExch(p.status, kDevWaitTimeout);
}

// ----------------------------------------------------------------- host side
enum TmapKind : int { kTmapWeights = 0, kTmapGroups = 1 };

struct TmapEntry {
  const void* ptr = nullptr;
  int kind = -1, K = 0, N = 0, dev = -1;
  CUtensorMap map;
};

thread_local TmapEntry t_tmap_cache[32];
thread_local int t_tmap_next = 0;

// Tensor map over packed weights [N, K/8] int32 (box 32 words x 64 rows,
// 128-byte swizzle) or over a scale / zero matrix [N, K/128] fp16 (box 8
// groups x 64 rows), cached per thread.
int tensor_map(int kind, const void* ptr, int K, int N, int dev, CUtensorMap* out) {
  for (auto& e : t_tmap_cache) {
    if (e.ptr == ptr && e.kind == kind && e.K == K && e.N == N && e.dev == dev) {
      *out = e.map;
      return FOCAL_OK;
    }
  }
  TmapEntry& e = t_tmap_cache[t_tmap_next];
  int rc;
  if (kind == kTmapWeights) {
    const uint64_t dims[2] = {(uint64_t)(K / 8), (uint64_t)N};
    const uint64_t strides[1] = {(uint64_t)K / 2};
    const uint32_t box[2] = {kWordsPerStage, kRows};
    rc = encode_tensor_map(&e.map, CU_TENSOR_MAP_DATA_TYPE_INT32, 2, ptr, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    const uint64_t dims[2] = {(uint64_t)(K / 128), (uint64_t)N};
    const uint64_t strides[1] = {(uint64_t)(K / 128) * 2};
    const uint32_t box[2] = {kSzQuadGroups, kRows};
    rc = encode_tensor_map(&e.map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, ptr, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_NONE);
  }
  if (rc) {
    e.ptr = nullptr;
    return rc;
  }
  e.ptr = ptr;
  e.kind = kind;
  e.K = K;
  e.N = N;
  e.dev = dev;
  t_tmap_next = (t_tmap_next + 1) % 32;
  *out = e.map;
  return FOCAL_OK;
}

int mt_for(int M) { return M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8; }

int check_shape(int M, int K, int N) {
  if (M < 1 || M > 8) return set_error(FOCAL_ERR_UNSUPPORTED, "unsupported M");
  if (N <= 0 || N % 64 != 0) return set_error(FOCAL_ERR_UNSUPPORTED, "unsupported N");
  // The reference accepts only a whitelist (csrc/w4a16_gemv.cu:135-143); this
  // contract is rule-based but keeps its deliberate K = N = 11008 rejection.
  if (K <= 0 || K % kStageK != 0 || K > (1 << 24) || (K == 11008 && N == 11008))
    return set_error(FOCAL_ERR_UNSUPPORTED, "unsupported K/N");
  if ((long long)N * K / 8 > (1LL << 40)) return set_error(FOCAL_ERR_UNSUPPORTED, "unsupported K/N");
  return FOCAL_OK;
}

// Workspace bound for (M, K, N) on a device with `sm_count` SMs: room for the
// gate/up variant's partial slots and the largest grid the kernels can have.
size_t workspace_bound(int M, int K, int N, int sm_count) {
  const int TS = K / kStageK, RB = N / kRows;
  const long long U = (long long)TS * RB;
  const int P = (int)std::min<long long>(U, (long long)kMaxCtasPerSm * sm_count);
  return ws_layout(mt_for(M), 2, TS, RB, P).total;
}

cudaLaunchAttribute pdl_attribute() {
  cudaLaunchAttribute a;
  a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  a.val.programmaticStreamSerializationAllowed = 1;
  return a;
}

// Resident CTAs per SM for one kernel instantiation (cached per device).
std::mutex g_occ_mutex;
int g_occ[64][12];

int ctas_per_sm(const void* kern, int slot, int smem, int dev, int* out) {
  std::lock_guard<std::mutex> lock(g_occ_mutex);
  if (dev < 0 || dev >= 64 || slot < 0 || slot >= 12) return set_error(FOCAL_ERR_INVALID_VALUE, "bad slot");
  if (!g_occ[dev][slot]) {
    int n = 0;
    int rc = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kThreads, smem),
                        "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    if (rc) return rc;
    g_occ[dev][slot] = std::max(1, std::min(n, kMaxCtasPerSm));
  }
  *out = g_occ[dev][slot];
  return FOCAL_OK;
}

template <int MT>
int launch_prepare(const __nv_bfloat16* x, uint8_t* rec, unsigned int* counters, int M, int K, int RB,
                   cudaStream_t stream) {
  PrepParams pp{x, rec, counters, M, K, K / kStageK, RB};
  const int items = pp.stages * mtp_of(MT);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((items + 3) / 4, 1, 1);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1] = {pdl_attribute()};
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, x_prepare_kernel<MT>, pp), "x_prepare_kernel launch");
}

template <int MT, int NW, int EPI>
int launch_t(const CUtensorMap* maps, Params p, const __nv_bfloat16* x,
             uint8_t* workspace, size_t ws_bytes, const DeviceInfo& dev, cudaStream_t stream) {
  constexpr Layout L = make_layout<MT, NW>();
  static_assert(L.total <= 227 * 1024, "shared-memory carve-up exceeds the per-CTA limit");
  auto kern = w4a16_gemv_kernel<MT, NW, EPI>;
  constexpr int slot = (MT == 1 ? 0 : MT == 2 ? 1 : MT == 4 ? 2 : 3) + 4 * EPI;
  int rc = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), slot, (int)L.total);
  if (rc) return rc;
  int occ = 0;
  rc = ctas_per_sm(reinterpret_cast<const void*>(kern), slot, (int)L.total, dev.device, &occ);
  if (rc) return rc;
  static const int min_units = [] {
    const char* e = getenv("FOCAL_W4A16_MIN_UNITS");  // tuning override
    return e && atoi(e) > 0 ? atoi(e) : kMinUnitsPerCta;
  }();
  static const int waves = [] {
    const char* e = getenv("FOCAL_W4A16_WAVES");  // tuning override: CTAs per resident slot
    return e && atoi(e) > 0 ? std::min(atoi(e), kMaxCtasPerSm) : 1;
  }();
  p.P = (int)std::min<long long>((p.U + min_units - 1) / min_units,
                                 (long long)std::min(occ * waves, kMaxCtasPerSm) * dev.sm_count);
  p.P = std::max(p.P, 1);
  const WsLayout W = ws_layout(MT, NW, p.TS, p.RB, p.P);
  if (ws_bytes < W.total)
    return set_error(FOCAL_ERR_WORKSPACE, "workspace too small: need %zu bytes, got %zu", W.total, ws_bytes);
  p.rec = workspace + W.rec;
  p.counters = reinterpret_cast<unsigned int*>(workspace + W.counters);
  p.partials = reinterpret_cast<float*>(workspace + W.partials);
  rc = launch_prepare<MT>(x, workspace + W.rec, p.counters, p.M, p.K, p.RB, stream);
  if (rc) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.P, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1] = {pdl_attribute()};
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, maps[0], maps[1], maps[2], maps[3], maps[4], maps[5], p),
                    "w4a16_gemv_kernel launch");
}

template <int NW, int EPI>
int dispatch_mt(int MT, const CUtensorMap* maps, const Params& p, const __nv_bfloat16* x, uint8_t* ws,
                size_t ws_bytes, const DeviceInfo& dev, cudaStream_t stream) {
  switch (MT) {
    case 1: return launch_t<1, NW, EPI>(maps, p, x, ws, ws_bytes, dev, stream);
    case 2: return launch_t<2, NW, EPI>(maps, p, x, ws, ws_bytes, dev, stream);
    case 4: return launch_t<4, NW, EPI>(maps, p, x, ws, ws_bytes, dev, stream);
    default: return launch_t<8, NW, EPI>(maps, p, x, ws, ws_bytes, dev, stream);
  }
}

int run(int epi, const void* x, const int32_t* wq0, const void* s0, const void* z0,
        const int32_t* wq1, const void* s1, const void* z1, void* y, int M, int K, int N,
        void* workspace, size_t ws_bytes, cudaStream_t stream) {
  clear_error();
  int rc = check_shape(M, K, N);
  if (rc) return rc;
  const int NW = epi == kEpiSiluMul ? 2 : 1;
  if (!x || !wq0 || !s0 || !z0 || !y || (NW == 2 && (!wq1 || !s1 || !z1)))
    return set_error(FOCAL_ERR_INVALID_VALUE, "null pointer");
  if (!aligned(x, 16)) return set_error(FOCAL_ERR_INVALID_VALUE, "x must be 16-byte aligned");
  if (!aligned(wq0, 16) || (NW == 2 && !aligned(wq1, 16)))
    return set_error(FOCAL_ERR_INVALID_VALUE, "wq must be 16-byte aligned");
  if (!aligned(s0, 4) || !aligned(z0, 4) || (NW == 2 && (!aligned(s1, 4) || !aligned(z1, 4))))
    return set_error(FOCAL_ERR_INVALID_VALUE, "scales and zeros must be 4-byte aligned");
  if (!aligned(y, epi == kEpiF32 ? 4 : 2)) return set_error(FOCAL_ERR_INVALID_VALUE, "y is misaligned");
  if (!workspace) return set_error(FOCAL_ERR_WORKSPACE, "workspace missing");
  if (!aligned(workspace, 256)) return set_error(FOCAL_ERR_INVALID_VALUE, "workspace must be 256-byte aligned");

  DeviceInfo dev;
  rc = current_device_info(&dev);
  if (rc) return rc;
  const int MT = mt_for(M);

  // maps: weights 0 / 1, then scales 0, zeros 0, scales 1, zeros 1
  CUtensorMap maps[6];
  const int32_t* wqs[2] = {wq0, NW == 2 ? wq1 : wq0};
  const void* szs[4] = {s0, z0, NW == 2 ? s1 : s0, NW == 2 ? z1 : z0};
  for (int m = 0; m < 2; ++m) {
    rc = tensor_map(kTmapWeights, wqs[m], K, N, dev.device, &maps[m]);
    if (rc) return rc;
  }
  // Scales and zeros come in by TMA when each row's groups form 16-byte
  // multiples (K % 1024 == 0) and the bases are 16-byte aligned; otherwise
  // by 4-byte cp.async.
  bool sz_tma = (K / 128) % kSzQuadGroups == 0;
  for (int j = 0; j < 4; ++j) sz_tma = sz_tma && aligned(szs[j], 16);
  for (int j = 0; j < 4; ++j) {
    if (sz_tma) {
      rc = tensor_map(kTmapGroups, szs[j], K, N, dev.device, &maps[2 + j]);
      if (rc) return rc;
    } else {
      maps[2 + j] = maps[0];  // unused
    }
  }
  Params p{};
  p.scales0 = static_cast<const __half*>(s0);
  p.zeros0 = static_cast<const __half*>(z0);
  p.scales1 = static_cast<const __half*>(NW == 2 ? s1 : s0);
  p.zeros1 = static_cast<const __half*>(NW == 2 ? z1 : z0);
  p.y = y;
  p.status = dev.status;
  p.M = M;
  p.K = K;
  p.N = N;
  p.G = K / 128;
  p.TS = K / kStageK;
  p.RB = N / kRows;
  p.U = (long long)p.TS * p.RB;
  p.sz_tma = sz_tma ? 1 : 0;
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  auto* ws = static_cast<uint8_t*>(workspace);
  if (epi == kEpiBf16) return dispatch_mt<1, kEpiBf16>(MT, maps, p, xb, ws, ws_bytes, dev, stream);
  if (epi == kEpiF32) return dispatch_mt<1, kEpiF32>(MT, maps, p, xb, ws, ws_bytes, dev, stream);
  return dispatch_mt<2, kEpiSiluMul>(MT, maps, p, xb, ws, ws_bytes, dev, stream);
}

}  // namespace gemv
}  // namespace focal

using namespace focal;

extern "C" {

int focal_w4a16_check_shape(int M, int K, int N) {
  clear_error();
  return gemv::check_shape(M, K, N);
}

size_t focal_w4a16_workspace_size(int M, int K, int N) {
  if (gemv::check_shape(M, K, N)) return 0;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    sms = 256;  // no device visible: the bound for the largest GPUs
  return gemv::workspace_bound(M, K, N, sms);
}

int focal_w4a16_gemv(const void* x, const int32_t* wq, const void* scales, const void* zeros,
                     void* y, int M, int K, int N, void* workspace, size_t ws_bytes,
                     cudaStream_t stream) {
  return gemv::run(gemv::kEpiBf16, x, wq, scales, zeros, nullptr, nullptr, nullptr, y, M, K, N,
                   workspace, ws_bytes, stream);
}

int focal_w4a16_gemv_f32(const void* x, const int32_t* wq, const void* scales, const void* zeros,
                         float* y, int M, int K, int N, void* workspace, size_t ws_bytes,
                         cudaStream_t stream) {
  return gemv::run(gemv::kEpiF32, x, wq, scales, zeros, nullptr, nullptr, nullptr, y, M, K, N,
                   workspace, ws_bytes, stream);
}

int focal_w4a16_gate_up_silu(const void* x, const int32_t* wq_gate, const void* scales_gate,
                             const void* zeros_gate, const int32_t* wq_up, const void* scales_up,
                             const void* zeros_up, void* h, int M, int K, int N, void* workspace,
                             size_t ws_bytes, cudaStream_t stream) {
  return gemv::run(gemv::kEpiSiluMul, x, wq_gate, scales_gate, zeros_gate, wq_up, scales_up,
                   zeros_up, h, M, K, N, workspace, ws_bytes, stream);
}

}  // extern "C"
