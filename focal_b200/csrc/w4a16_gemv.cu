// W4A16 small-M linear for B200 (sm_100a).
//
//   y[m, n] = bf16( sum_k x[m, k] * (q[n, k] - z[n, k/128]) * s[n, k/128] ),  M <= 8
//
// Replaces the reference's SIMT kernel and launcher (csrc/w4a16_gemv.cu:33-116,
// :152-223) behind the same packing and dequant semantics (README.md:66-73).
//
// Design (one CTA = 64 weight rows x one K slice; a cluster of S CTAs = the S
// K slices of the same 64 rows):
//  * warp 4 (producer) streams the packed weights with 2-D TMA boxes of
//    64 rows x 128 bytes (256 K values, two quantisation groups) into a
//    4-stage shared-memory ring with the 128-byte swizzle, and the matching
//    fp16 scale/zero pairs with 4-byte cp.async, all completing on one
//    mbarrier per stage;
//  * warps 0-3 (consumers) each own 16 rows.  A packed word is turned into
//    bf16 (128 + q) pairs with one shift and one LOP3 per pair and fed as the
//    A fragment of mma.sync m16n8k16 (bf16 in, fp32 accumulate); the <= 8
//    tokens are the n = 8 side.  The zero point and the +128 are factored
//    out per group:  sum_k x (q - z) s = s * (sum_k x (128 + q) - (z + 128) sum_k x)
//    so the tensor core only sees exact small integers and x;
//  * the activation slice of this CTA sits in shared memory for the whole
//    CTA, pre-permuted into the MMA's B-fragment order together with its
//    per-group sums, so each B fragment is one conflict-free 16-byte load;
//  * split-K partials are reduced through distributed shared memory
//    (ld.shared::cluster) in rank order — deterministic, no global
//    workspace, no atomics.  No TMA multicast is used.
#include <cmath>
#include <cstdlib>

#include "common.cuh"
#include "host_common.h"

namespace focal {
namespace gemv {

constexpr int kStageK = 256;            // K values per pipeline stage
constexpr int kWordsPerStage = 32;      // int32 words per row per stage (128 B)
constexpr int kConsumerWarps = 4;
constexpr int kRows = 16 * kConsumerWarps;  // weight rows per CTA
constexpr int kThreads = 32 * (kConsumerWarps + 1);
constexpr int kStages = 4;
constexpr int kXsMaxBytes = 64 * 1024;  // activation slice budget in shared memory
constexpr int kMaxSplits = 8;           // portable cluster size

enum Epi : int { kEpiBf16 = 0, kEpiF32 = 1, kEpiSiluMul = 2 };

struct Params {
  const __nv_bfloat16* x;
  const __half* scales0;
  const __half* zeros0;
  const __half* scales1;
  const __half* zeros1;
  void* y;
  int* status;
  int M, K, N, G, total_stages, splits;
};

struct Layout {
  uint32_t w, sz, xs, xsum, red, bars, total;
};

__host__ __device__ constexpr int round_up(int a, int b) { return (a + b - 1) / b * b; }

// Shared-memory carve-up, identical on host (sizing) and device (addressing).
template <int MT, int NW>
__host__ __device__ inline Layout make_layout(int slice_stages_max) {
  constexpr int MTp = MT < 2 ? 2 : MT;
  Layout L{};
  uint32_t off = 0;
  L.w = off;
  off += kStages * NW * kRows * 128;
  L.sz = off;
  off += kStages * NW * 2 * kRows * 4;
  L.xs = off;
  off += slice_stages_max * 2 * MT * 256;
  L.xsum = off;
  off += round_up(slice_stages_max * 2 * MTp * 4, 16);
  L.red = off;
  off += NW * MT * kRows * 4;
  L.bars = round_up(off, 8);
  off = L.bars + 2 * kStages * 8;
  L.total = off + 1024;  // slack for aligning the base to 1024 B (128-byte swizzle atom)
  return L;
}

template <int MT, int NW, int EPI>
__global__ void __launch_bounds__(kThreads, 2)
    w4a16_gemv_kernel(const __grid_constant__ CUtensorMap tmap0,
                      const __grid_constant__ CUtensorMap tmap1, const Params p) {
  constexpr int MTp = MT < 2 ? 2 : MT;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;

  const int S = p.splits;
  const int split = blockIdx.x;  // the cluster spans gridDim.x, so this is the cluster rank
  const int rb = blockIdx.y;
  const int per = p.total_stages / S, rem = p.total_stages % S;
  const int st0 = split * per + min(split, rem);
  const int nst = per + (split < rem ? 1 : 0);
  const Layout L = make_layout<MT, NW>(per + (rem ? 1 : 0));

  const uint32_t w_base = base + L.w;
  const uint32_t sz_base = base + L.sz;
  const uint32_t xs_base = base + L.xs;
  const uint32_t xsum_base = base + L.xsum;
  const uint32_t red_base = base + L.red;
  const uint32_t full_bar = base + L.bars;
  const uint32_t empty_bar = full_bar + kStages * 8;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full_bar + 8 * s, 1 + 32);  // producer expect_tx + 32 cp.async arrivals
      mbar_init(empty_bar + 8 * s, kConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  bool ok = true;
  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tensormap(&tmap0);
      if (NW == 2) prefetch_tensormap(&tmap1);
    }
    const uint64_t pol = l2_policy_evict_first();
    const int row0 = rb * kRows;
    for (int i = 0; i < nst; ++i) {
      const int slot = i % kStages;
      if (i >= kStages) {
        if (!mbar_wait_bounded(empty_bar + 8 * slot, ((i / kStages) - 1) & 1)) {
          ok = false;
          break;
        }
      }
      const int gs = st0 + i;
      const uint32_t fb = full_bar + 8 * slot;
      if (lane == 0) {
        mbar_arrive_expect_tx(fb, NW * kRows * 128);
        tma_load_2d(w_base + (slot * NW + 0) * kRows * 128, &tmap0, gs * kWordsPerStage, row0, fb, pol);
        if (NW == 2)
          tma_load_2d(w_base + (slot * NW + 1) * kRows * 128, &tmap1, gs * kWordsPerStage, row0, fb,
                      pol);
      }
      // scale / zero pairs (groups 2gs, 2gs+1) of the 64 rows: 4 bytes each
#pragma unroll
      for (int j = lane; j < NW * 2 * kRows; j += 32) {
        const int mat = j / (2 * kRows);
        const int arr = (j / kRows) & 1;
        const int r = j % kRows;
        const __half* src = mat == 0 ? (arr ? p.zeros0 : p.scales0) : (arr ? p.zeros1 : p.scales1);
        src += (size_t)(row0 + r) * p.G + 2 * gs;
        cp_async_4(sz_base + (((slot * NW + mat) * 2 + arr) * kRows + r) * 4, src);
      }
      cp_async_arrive_noinc(fb);
    }
  } else {
    // ------------------------------------------------------------ consumers
    // 1. activation slice -> shared memory in B-fragment order, plus group sums
    {
      const int k0 = st0 * kStageK;
      const int nchunks = 2 * nst * MT * 16;  // 16-byte chunks (8 values) of x
      for (int ib = 0; ib < nchunks; ib += kConsumerWarps * 32) {
        const int idx = ib + threadIdx.x;
        const bool active = idx < nchunks;
        const int c = idx & 15;  // chunk within the 128-wide group
        const int gm = idx >> 4;
        const int m = gm % MT;
        const int gl = gm / MT;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (active && m < p.M)
          v = __ldg(reinterpret_cast<const uint4*>(p.x + (size_t)m * p.K + k0 + gl * 128 + c * 8));
        float sum = bf16_lo(v.x) + bf16_hi(v.x) + bf16_lo(v.y) + bf16_hi(v.y) + bf16_lo(v.z) +
                    bf16_hi(v.z) + bf16_lo(v.w) + bf16_hi(v.w);
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        sum += __shfl_xor_sync(0xffffffffu, sum, 4);
        sum += __shfl_xor_sync(0xffffffffu, sum, 8);
        if (active) {
          // pairs (x_j, x_{j+4}) match the nibble pairs (q_j, q_{j+4}) of a word
          uint4 pv;
          pv.x = prmt(v.x, v.z, 0x5410);
          pv.y = prmt(v.x, v.z, 0x7632);
          pv.z = prmt(v.y, v.w, 0x5410);
          pv.w = prmt(v.y, v.w, 0x7632);
          const int tt = c >> 2, qq = c & 3;
          const int reader_lane = 4 * m + tt;
          sts128(xs_base + ((gl * MT + m) * 4 + tt) * 64 + (((qq + (reader_lane >> 1)) & 3) << 4), pv);
          if (c == 0) {
            asm volatile("st.shared.f32 [%0], %1;" ::"r"(xsum_base + (gl * MTp + m) * 4), "f"(sum)
                         : "memory");
          }
        }
      }
      if (MT == 1) {  // token 1 of the padded pair reads as zero
        for (int gl = threadIdx.x; gl < 2 * nst; gl += kConsumerWarps * 32)
          asm volatile("st.shared.f32 [%0], %1;" ::"r"(xsum_base + (gl * MTp + 1) * 4), "f"(0.0f)
                       : "memory");
      }
      named_barrier(1, kConsumerWarps * 32);
    }

    // 2. main loop
    const int g = lane >> 2, t = lane & 3;
    const int pg = (g >> 1) + ((g & 1) << 2);  // row permutation: conflict-free 128B-swizzled reads
    const int r0 = warp * 16 + pg, r1 = r0 + 8;
    const int rot = (lane >> 1) & 3;
    float acc[NW][4];
#pragma unroll
    for (int mat = 0; mat < NW; ++mat)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[mat][j] = 0.f;

    for (int i = 0; i < nst; ++i) {
      const int slot = i % kStages;
      if (!mbar_wait_bounded(full_bar + 8 * slot, (i / kStages) & 1)) {
        ok = false;
        break;
      }
      uint32_t sv[NW][2], zv[NW][2];
#pragma unroll
      for (int mat = 0; mat < NW; ++mat) {
        const uint32_t sb = sz_base + ((slot * NW + mat) * 2) * kRows * 4;
        sv[mat][0] = lds32(sb + r0 * 4);
        sv[mat][1] = lds32(sb + r1 * 4);
        zv[mat][0] = lds32(sb + (kRows + r0) * 4);
        zv[mat][1] = lds32(sb + (kRows + r1) * 4);
      }
#pragma unroll
      for (int G = 0; G < 2; ++G) {
        const int gl = 2 * i + G;
        uint32_t xb[16];
        if (g < MT) {
          const uint32_t xa = xs_base + ((gl * MT + g) * 4 + t) * 64;
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) {
            const uint4 v = lds128(xa + (((qq + rot) & 3) << 4));
            xb[4 * qq + 0] = v.x;
            xb[4 * qq + 1] = v.y;
            xb[4 * qq + 2] = v.z;
            xb[4 * qq + 3] = v.w;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) xb[j] = 0u;
        }
        const float2 xsv = lds_f2(xsum_base + (gl * MTp + (2 * t < MT ? 2 * t : 0)) * 4);
#pragma unroll
        for (int mat = 0; mat < NW; ++mat) {
          const uint32_t wb = w_base + (slot * NW + mat) * kRows * 128;
          const uint4 wa4 = lds128(wb + r0 * 128 + (((4 * G + t) ^ (r0 & 7)) << 4));
          const uint4 wb4 = lds128(wb + r1 * 128 + (((4 * G + t) ^ (r1 & 7)) << 4));
          const uint32_t wa[4] = {wa4.x, wa4.y, wa4.z, wa4.w};
          const uint32_t wr[4] = {wb4.x, wb4.y, wb4.z, wb4.w};
          float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              mma_bf16_16816(d, nib_pair_bf16(wa[qq], 2 * h), nib_pair_bf16(wr[qq], 2 * h),
                             nib_pair_bf16(wa[qq], 2 * h + 1), nib_pair_bf16(wr[qq], 2 * h + 1),
                             xb[4 * qq + 2 * h], xb[4 * qq + 2 * h + 1]);
            }
          }
          const float s0 = G ? half_hi(sv[mat][0]) : half_lo(sv[mat][0]);
          const float s1 = G ? half_hi(sv[mat][1]) : half_lo(sv[mat][1]);
          const float z0 = (G ? half_hi(zv[mat][0]) : half_lo(zv[mat][0])) + 128.0f;
          const float z1 = (G ? half_hi(zv[mat][1]) : half_lo(zv[mat][1])) + 128.0f;
          acc[mat][0] = fmaf(s0, fmaf(-z0, xsv.x, d[0]), acc[mat][0]);
          acc[mat][1] = fmaf(s0, fmaf(-z0, xsv.y, d[1]), acc[mat][1]);
          acc[mat][2] = fmaf(s1, fmaf(-z1, xsv.x, d[2]), acc[mat][2]);
          acc[mat][3] = fmaf(s1, fmaf(-z1, xsv.y, d[3]), acc[mat][3]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_bar + 8 * slot);
    }

    // 3. this CTA's partial sums -> shared memory [mat][token][row]
#pragma unroll
    for (int mat = 0; mat < NW; ++mat) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int tok = 2 * t + (j & 1);
        const int row = (j < 2) ? r0 : r1;
        if (tok < MT)
          asm volatile("st.shared.f32 [%0], %1;" ::"r"(red_base + ((mat * MT + tok) * kRows + row) * 4),
                       "f"(acc[mat][j])
                       : "memory");
      }
    }
  }

  if (!ok && p.status) atomicExch(p.status, kDevWaitTimeout);

  // 4. split-K reduction across the cluster, in rank order
  cluster_sync_all();
  {
    const int total = p.M * kRows;
    const int chunk = (total + S - 1) / S;
    const int o_end = min(total, (split + 1) * chunk);
    for (int o = split * chunk + threadIdx.x; o < o_end; o += kThreads) {
      const int tok = o / kRows, row = o - tok * kRows;
      float v[NW];
#pragma unroll
      for (int mat = 0; mat < NW; ++mat) {
        const uint32_t a = red_base + ((mat * MT + tok) * kRows + row) * 4;
        float sacc = 0.f;
        for (int s = 0; s < S; ++s) sacc += ld_shared_cluster_f32(mapa_shared(a, s));
        v[mat] = sacc;
      }
      const size_t yi = (size_t)tok * p.N + (size_t)rb * kRows + row;
      if (EPI == kEpiBf16) {
        static_cast<__nv_bfloat16*>(p.y)[yi] = __float2bfloat16_rn(v[0]);
      } else if (EPI == kEpiF32) {
        static_cast<float*>(p.y)[yi] = v[0];
      } else {
        // silu(gate) * up with the roundings of the unfused bf16 path
        const float gt = __bfloat162float(__float2bfloat16_rn(v[0]));
        const float up = __bfloat162float(__float2bfloat16_rn(v[NW - 1]));
        const float sg = __bfloat162float(__float2bfloat16_rn(gt / (1.0f + expf(-gt))));
        static_cast<__nv_bfloat16*>(p.y)[yi] = __float2bfloat16_rn(sg * up);
      }
    }
  }
  cluster_sync_all();  // peers may still be reading this CTA's partials
}

// ----------------------------------------------------------------- host side
struct TmapEntry {
  const void* ptr = nullptr;
  int K = 0, N = 0, dev = -1;
  CUtensorMap map;
};

thread_local TmapEntry t_tmap_cache[16];
thread_local int t_tmap_next = 0;

int weight_tensor_map(const int32_t* wq, int K, int N, int dev, CUtensorMap* out) {
  for (auto& e : t_tmap_cache) {
    if (e.ptr == wq && e.K == K && e.N == N && e.dev == dev) {
      *out = e.map;
      return FOCAL_OK;
    }
  }
  const uint64_t dims[2] = {(uint64_t)(K / 8), (uint64_t)N};
  const uint64_t strides[1] = {(uint64_t)K / 2};
  const uint32_t box[2] = {kWordsPerStage, kRows};
  TmapEntry& e = t_tmap_cache[t_tmap_next];
  int rc = encode_tensor_map(&e.map, CU_TENSOR_MAP_DATA_TYPE_INT32, 2, wq, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) {
    e.ptr = nullptr;
    return rc;
  }
  e.ptr = wq;
  e.K = K;
  e.N = N;
  e.dev = dev;
  t_tmap_next = (t_tmap_next + 1) % 16;
  *out = e.map;
  return FOCAL_OK;
}

int mt_for(int M) { return M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8; }

int xs_bytes(int MT, int slice_stages) { return slice_stages * 2 * MT * 256; }

// Splits S (cluster size) for a (row blocks, stages) problem: the smallest S
// that puts at least two CTAs per SM in flight, within the activation budget.
int choose_splits(int MT, int RB, int TS, int sm_count) {
  static const int forced = [] {
    const char* e = getenv("FOCAL_W4A16_SPLITS");
    return e ? atoi(e) : 0;
  }();
  int best = 0;
  for (int S = 1; S <= kMaxSplits && S <= TS; ++S) {
    const int sl = (TS + S - 1) / S;
    if (xs_bytes(MT, sl) > kXsMaxBytes) continue;
    if (forced > 0) {
      if (S == forced) return S;
      continue;
    }
    best = S;
    if (RB * S >= 2 * sm_count) return S;
  }
  return best;  // 0 = no feasible split
}

int check_shape(int M, int K, int N) {
  if (M < 1 || M > 8) return set_error(FOCAL_ERR_UNSUPPORTED, "unsupported M");
  if (N <= 0 || N % 64 != 0 || N / kRows > 65535) return set_error(FOCAL_ERR_UNSUPPORTED, "unsupported N");
  // The reference accepts only a whitelist (csrc/w4a16_gemv.cu:135-143); this
  // contract is rule-based but keeps its deliberate K = N = 11008 rejection.
  if (K <= 0 || K % kStageK != 0 || (K == 11008 && N == 11008))
    return set_error(FOCAL_ERR_UNSUPPORTED, "unsupported K/N");
  const int MT = mt_for(M);
  const int TS = K / kStageK;
  bool fits = false;
  for (int S = 1; S <= kMaxSplits && S <= TS; ++S)
    fits = fits || xs_bytes(MT, (TS + S - 1) / S) <= kXsMaxBytes;
  if (!fits) return set_error(FOCAL_ERR_UNSUPPORTED, "unsupported K/N");
  return FOCAL_OK;
}

template <int MT, int NW, int EPI>
int launch_t(const CUtensorMap& m0, const CUtensorMap& m1, const Params& p, int S, cudaStream_t stream) {
  const int TS = p.total_stages;
  const Layout L = make_layout<MT, NW>((TS + S - 1) / S);
  auto kern = w4a16_gemv_kernel<MT, NW, EPI>;
  constexpr int slot = (MT == 1 ? 0 : MT == 2 ? 1 : MT == 4 ? 2 : 3) + 4 * (NW - 1) + 8 * EPI;
  int rc = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), slot, (int)L.total);
  if (rc) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(S, p.N / kRows, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, m0, m1, p), "w4a16_gemv_kernel launch");
}

template <int NW, int EPI>
int dispatch_mt(int MT, const CUtensorMap& m0, const CUtensorMap& m1, const Params& p, int S,
                cudaStream_t stream) {
  switch (MT) {
    case 1: return launch_t<1, NW, EPI>(m0, m1, p, S, stream);
    case 2: return launch_t<2, NW, EPI>(m0, m1, p, S, stream);
    case 4: return launch_t<4, NW, EPI>(m0, m1, p, S, stream);
    default: return launch_t<8, NW, EPI>(m0, m1, p, S, stream);
  }
}

int run(int epi, const void* x, const int32_t* wq0, const void* s0, const void* z0,
        const int32_t* wq1, const void* s1, const void* z1, void* y, int M, int K, int N,
        cudaStream_t stream) {
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

  DeviceInfo dev;
  rc = current_device_info(&dev);
  if (rc) return rc;
  const int MT = mt_for(M);
  const int TS = K / kStageK;
  const int S = choose_splits(MT, N / kRows, TS, dev.sm_count);
  if (S <= 0) return set_error(FOCAL_ERR_UNSUPPORTED, "unsupported K/N");

  CUtensorMap m0, m1;
  rc = weight_tensor_map(wq0, K, N, dev.device, &m0);
  if (rc) return rc;
  if (NW == 2) {
    rc = weight_tensor_map(wq1, K, N, dev.device, &m1);
    if (rc) return rc;
  } else {
    m1 = m0;
  }
  Params p;
  p.x = static_cast<const __nv_bfloat16*>(x);
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
  p.total_stages = TS;
  p.splits = S;
  if (epi == kEpiBf16) return dispatch_mt<1, kEpiBf16>(MT, m0, m1, p, S, stream);
  if (epi == kEpiF32) return dispatch_mt<1, kEpiF32>(MT, m0, m1, p, S, stream);
  return dispatch_mt<2, kEpiSiluMul>(MT, m0, m1, p, S, stream);
}

}  // namespace gemv
}  // namespace focal

using namespace focal;

extern "C" {

int focal_w4a16_check_shape(int M, int K, int N) {
  clear_error();
  return gemv::check_shape(M, K, N);
}

int focal_w4a16_gemv(const void* x, const int32_t* wq, const void* scales, const void* zeros,
                     void* y, int M, int K, int N, cudaStream_t stream) {
  return gemv::run(gemv::kEpiBf16, x, wq, scales, zeros, nullptr, nullptr, nullptr, y, M, K, N,
                   stream);
}

int focal_w4a16_gemv_f32(const void* x, const int32_t* wq, const void* scales, const void* zeros,
                         float* y, int M, int K, int N, cudaStream_t stream) {
  return gemv::run(gemv::kEpiF32, x, wq, scales, zeros, nullptr, nullptr, nullptr, y, M, K, N,
                   stream);
}

int focal_w4a16_gate_up_silu(const void* x, const int32_t* wq_gate, const void* scales_gate,
                             const void* zeros_gate, const int32_t* wq_up, const void* scales_up,
                             const void* zeros_up, void* h, int M, int K, int N,
                             cudaStream_t stream) {
  return gemv::run(gemv::kEpiSiluMul, x, wq_gate, scales_gate, zeros_gate, wq_up, scales_up,
                   zeros_up, h, M, K, N, stream);
}

}  // extern "C"
