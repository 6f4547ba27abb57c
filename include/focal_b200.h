/*
 * focal_b200 — C ABI of the B200-native (sm_100a) decode hot paths.
 *
 * Plain pointers, sizes and a CUDA stream; no framework types.  Every entry
 * point is asynchronous on `stream`, returns FOCAL_OK (0) or a focal_status
 * code, and leaves a message for focal_last_error() on failure.  Pointers are
 * device pointers unless stated otherwise.  Shape errors use the reference's
 * exact messages ("unsupported M", "unsupported K/N", ...).
 *
 * Reference interfaces replaced (paths within the reference project):
 *   csrc/bindings.cpp:4-16        pybind11 module exporting w4a16_linear
 *   csrc/w4a16_gemv.cu:119-235    check_tensor / check_shape / launch_w4a16
 *   focal_w4a16/__init__.py:38-91 pack_int4_weight / dequant_ref
 */
#ifndef FOCAL_B200_H_
#define FOCAL_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same typedef as the CUDA runtime's (driver_types.h); a NULL stream is the
 * legacy default stream. */
typedef struct CUstream_st* cudaStream_t;

typedef enum focal_status {
  FOCAL_OK = 0,
  FOCAL_ERR_INVALID_VALUE = 1, /* null/misaligned pointer, bad argument        */
  FOCAL_ERR_UNSUPPORTED = 2,   /* shape outside the contract                   */
  FOCAL_ERR_WORKSPACE = 3,     /* workspace missing or too small               */
  FOCAL_ERR_CUDA = 4,          /* CUDA runtime / driver error at launch        */
  FOCAL_ERR_DEVICE = 5         /* a kernel reported a device-side failure      */
} focal_status;

/* Message of the last failing call on this host thread ("" if none). */
const char* focal_last_error(void);

/* ABI version of this library (bumped on any signature change). */
int focal_abi_version(void);

/* ---------------------------------------------------------------- W4A16 ---
 * y[M,N] = bf16( x[M,K] . dequant(wq)[N,K]^T ), fp32 accumulation.
 *   x      bf16  [M, K]      row-major, 16-byte aligned
 *   wq     int32 [N, K/8]    eight uint4 per word, value k at bits 4*(k%8)
 *   scales fp16  [N, K/128]  4-byte aligned
 *   zeros  fp16  [N, K/128]  4-byte aligned
 *   dequant: w[n,k] = (float(q) - float(zeros[n,k/128])) * float(scales[n,k/128])
 * Contract: 1 <= M <= 8; N % 64 == 0, N <= 262144; 0 < K <= 2^24 with K % 256 == 0;
 * K = N = 11008 is rejected ("unsupported K/N") as the reference does.
 */

/* Host-only shape check; FOCAL_OK or FOCAL_ERR_UNSUPPORTED with the
 * reference's message.  Replaces check_shape, csrc/w4a16_gemv.cu:129-149. */
int focal_w4a16_check_shape(int M, int K, int N);

/* Bytes of device workspace the linear entry points below need for (M, K, N)
 * on the current device: the partial sums of 64-row blocks whose K is split
 * across CTAs, as 64-bit {fp32 bits, ready} words.  0 if the shape is outside
 * the contract.  The workspace needs 256-byte alignment and must be zeroed once
 * before its first call; every call that returns FOCAL_OK leaves every word at
 * zero again, so one workspace can serve calls of any shape (zero it again
 * after a call that failed on the device).  Calls that share a workspace must
 * be ordered on one stream. */
size_t focal_w4a16_workspace_size(int M, int K, int N);

/* The linear layer.  Replaces launch_w4a16 / w4a16_gemv_kernel,
 * csrc/w4a16_gemv.cu:33-116 and :152-223; y is written, never read. */
int focal_w4a16_gemv(const void* x, const int32_t* wq, const void* scales, const void* zeros,
                     void* y, int M, int K, int N, void* workspace, size_t ws_bytes,
                     cudaStream_t stream);

/* The linear layer without a caller workspace.  No reference counterpart: for
 * callers that cannot allocate device memory where they call it (a host
 * callback, or a runtime whose device memory is planned up front), it uses a
 * fixed 8 MiB scratch array per device instead.
 *  - Shapes whose focal_w4a16_workspace_size() exceeds 8 MiB are rejected with
 *    FOCAL_ERR_UNSUPPORTED (on a 148-SM B200 every shape of the contract fits;
 *    the check guards devices with many more SMs).
 *  - The first call on a device resolves the scratch's address
 *    (cudaGetSymbolAddress); make it before any stream capture.
 *  - The scratch starts at zero when the library loads and every successful
 *    call leaves it at zero; after a call that failed on the device
 *    (focal_device_status nonzero) it may not be: focal_reset_device_status
 *    zeroes it again (a memset, no allocation).
 *  - All calls on one device share the scratch, so calls that may overlap
 *    (different streams, or host threads without ordering) race; order them on
 *    one stream. */
int focal_w4a16_gemv_noalloc(const void* x, const int32_t* wq, const void* scales, const void* zeros,
                             void* y, int M, int K, int N, cudaStream_t stream);

/* Diagnostic: the no-allocation scratch of the current device (its device
 * address, resolved on first use, and its size in bytes).  No reference
 * counterpart. */
int focal_w4a16_noalloc_scratch(void** scratch, size_t* bytes);

/* Same product with an fp32 output (no bf16 rounding): the partial sum of a
 * K-sharded (row-parallel) projection before its all-reduce.  New entry point;
 * the reference has no multi-GPU path. */
int focal_w4a16_gemv_f32(const void* x, const int32_t* wq, const void* scales, const void* zeros,
                         float* y, int M, int K, int N, void* workspace, size_t ws_bytes,
                         cudaStream_t stream);

/* Fused decode MLP front half: h = bf16( silu(x.Wg^T) * (x.Wu^T) ), with Wg and
 * Wu two W4A16 weights of identical shape [N, K/8] (gate and up projections).
 * The reference times these as separate projections
 * (bench/bench_decode_bundle.py:19-27); this entry point is new. */
int focal_w4a16_gate_up_silu(const void* x, const int32_t* wq_gate, const void* scales_gate,
                             const void* zeros_gate, const int32_t* wq_up, const void* scales_up,
                             const void* zeros_up, void* h, int M, int K, int N, void* workspace,
                             size_t ws_bytes, cudaStream_t stream);

/* ------------------------------------------------- unit-tiled weights ---
 * An offline re-layout of (wq, scales, zeros) for the linears below (the
 * reference lists a tensor-core-friendly re-layout as next work and has no
 * counterpart).  Unit u = rb * (K/256) + st (64 weight rows x 256 K values)
 * is one contiguous 8704-byte chunk: its 64 x 32 packed words in the order a
 * 128-byte-swizzled copy leaves them in shared memory (row r at byte 128 r,
 * 16-byte chunk c at position c ^ (r & 7)), then the rows' two scales
 * (4 bytes a row), then their two zeros.  Each unit of the GEMV is then one
 * contiguous read.  Contract: N % 64 == 0, K % 256 == 0; tiles 16-byte
 * aligned, wq 16-byte, scales and zeros 4-byte aligned.
 */
size_t focal_w4a16_tiles_size(int K, int N);   /* bytes; 0 outside the contract */
int focal_w4a16_tile_pack(const int32_t* wq, const void* scales, const void* zeros, void* tiles, int K, int N,
                          cudaStream_t stream);
/* The inverse: recovers the reference packing bit for bit. */
int focal_w4a16_tile_unpack(const void* tiles, int32_t* wq, void* scales, void* zeros, int K, int N,
                            cudaStream_t stream);

/* The linear layer, its fp32-output form and the fused gate/up/SiLU on
 * unit-tiled weights: the same results, bit for bit, as focal_w4a16_gemv,
 * focal_w4a16_gemv_f32 and focal_w4a16_gate_up_silu on the weights the tiles
 * were packed from.  Same shape contract and workspace rules. */
int focal_w4a16_gemv_tiled(const void* x, const void* tiles, void* y, int M, int K, int N, void* workspace,
                           size_t ws_bytes, cudaStream_t stream);
int focal_w4a16_gemv_tiled_f32(const void* x, const void* tiles, float* y, int M, int K, int N, void* workspace,
                               size_t ws_bytes, cudaStream_t stream);
int focal_w4a16_gate_up_silu_tiled(const void* x, const void* tiles_gate, const void* tiles_up, void* h, int M,
                                   int K, int N, void* workspace, size_t ws_bytes, cudaStream_t stream);

/* ---------------------------------------- tensor-parallel fused linears ---
 * New entry points (the reference has no multi-GPU code): the linear layer
 * with its collective in the same kernel.  Each 64-row block, once finished,
 * is stored into every other rank's buffer over NVLink peer memory, every
 * value in one 64-bit store together with the call's epoch, and completed
 * once the same block's words from every rank have arrived (a bounded poll of
 * the epochs; no fences or separate flags).  No TMA or library kernel touches
 * peer memory, and nothing uses multicast.
 *
 * The group: one buffer per rank, all of focal_tp_buffer_size() bytes or more,
 * zero-filled before the first call, 256-byte aligned, and mapped into every
 * rank's process for its own device (peer[q] is rank q's buffer as seen
 * here, peer[rank] the local one; focal_tp_buffer_create / _open below make
 * and map them).  Every rank must make the same sequence
 * of fused calls on its group, with the same M and N, each rank on its own
 * GPU; all CTAs of a call wait for the other ranks' blocks, so a rank that
 * does not make the call makes the others give up after about a second and
 * set focal_device_status to 2 (the group must then be rebuilt: zero the
 * buffers on every rank).  Calls on one group must be ordered on one stream
 * per rank; the buffers hold per-call state, so a group serves one stream. */
typedef struct focal_tp_comm {
  void* peer[8];  /* rank q's buffer as mapped in this process            */
  size_t bytes;   /* usable bytes of each buffer (the smallest of them)   */
  int world;      /* ranks, 1..8                                           */
  int rank;       /* this process's rank                                   */
} focal_tp_comm;

/* Bytes of each rank's buffer for fused calls with M <= max_m, N <= max_n
 * (per-rank N); 0 if world or the shape is outside the contract. */
size_t focal_tp_buffer_size(int world, int max_m, int max_n);

/* This rank's buffer: cudaMalloc'd on the current device, zero-filled (the
 * call waits for the fill), and exported as a 64-byte CUDA IPC handle
 * (`handle`) to send to every other rank. */
int focal_tp_buffer_create(size_t bytes, void** buffer, uint8_t* handle);

/* Maps another rank's buffer, given its handle, for kernels on the current
 * device (which must be this rank's GPU), enabling peer access as needed.
 * A mapping made in another device's context (for instance by a framework
 * that opens the handle on its owner's device) is not usable by the fused
 * kernels on this device. */
int focal_tp_buffer_open(const uint8_t* handle, void** peer);

/* Unmaps a buffer opened with focal_tp_buffer_open. */
int focal_tp_buffer_close(void* peer);

/* Frees this rank's buffer, once no rank uses it any more. */
int focal_tp_buffer_destroy(void* buffer);

/* Column-parallel linear + all-gather: this rank holds rows
 * [rank*N, (rank+1)*N) of a [world*N, K] weight (wq [N, K/8], scales and
 * zeros [N, K/128]) and the full x [M, K]; y is bf16 [M, world*N], every
 * rank's block in its columns, identical on every rank. */
int focal_w4a16_gemv_allgather(const void* x, const int32_t* wq, const void* scales, const void* zeros,
                               void* y, int M, int K, int N, const focal_tp_comm* comm, void* workspace,
                               size_t ws_bytes, cudaStream_t stream);

/* Row-parallel linear + all-reduce: this rank holds K columns
 * [rank*K, (rank+1)*K) of a [N, world*K] weight (wq [N, K/8], scales and
 * zeros [N, K/128]) and the matching x slice [M, K]; y is bf16 [M, N] =
 * bf16(sum over ranks, in rank order, of the fp32 partial products),
 * bit-identical on every rank. */
int focal_w4a16_gemv_allreduce(const void* x, const int32_t* wq, const void* scales, const void* zeros,
                               void* y, int M, int K, int N, const focal_tp_comm* comm, void* workspace,
                               size_t ws_bytes, cudaStream_t stream);

/* fp32 [N, K] dequantized weights, bit-identical to dequant_ref
 * (focal_w4a16/__init__.py:57-91); exposes the kernels' int4 unpacking. */
int focal_w4a16_dequant(const int32_t* wq, const void* scales, const void* zeros, float* w,
                        int K, int N, cudaStream_t stream);

/* uint8 [N, K] (low nibble used) -> int32 [N, K/8]; replaces pack_int4_weight,
 * focal_w4a16/__init__.py:38-54.  K % 8 == 0. */
int focal_pack_int4(const uint8_t* q, int32_t* wq, int N, int K, cudaStream_t stream);

/* ------------------------------------------------- GQA decode attention ---
 * o[b,h,:] = softmax( q[b,h,:] . k[b,g,:,:]^T * scale ) . v[b,g,:,:],  g = h / (Hq/Hkv)
 *   q bf16 [B, Hq, D]; k, v bf16 [B, Hkv, L, D] contiguous; o bf16 [B, Hq, D]
 * fp32 scores, softmax and accumulation; split-KV with a log-sum-exp combine.
 * Contract: D == 128; Hq % Hkv == 0; Hq / Hkv <= 16; L >= 1.
 * New component: the reference contains no attention code.
 *
 * Workspace (device memory, ws_bytes >= focal_gqa_decode_workspace_size(...)):
 * split partials plus one arrival counter per (b, kv head).  The counters must
 * be zero before the first call on a workspace; every call that returns
 * FOCAL_OK leaves them zero again.  Calls sharing a workspace must be ordered
 * on one stream.
 */
size_t focal_gqa_decode_workspace_size(int B, int Hq, int Hkv, int L, int D);

int focal_gqa_decode_attn(const void* q, const void* k, const void* v, void* o, int B, int Hq,
                          int Hkv, int L, int D, float scale, void* workspace, size_t ws_bytes,
                          cudaStream_t stream);

/* Paged (variable-length) form, new as well: the caches are pages shared by
 * all sequences, k_pages / v_pages bf16 [num_pages, Hkv, page_size, D]; page j
 * of sequence b is block_table[b * max_pages_per_seq + j] (int32), and
 * sequence b has seq_lens[b] positions (int32, 1 .. max_seq_len; entries of
 * the block table past a sequence's last page are not read).  page_size is
 * 16, 32 or a multiple of 64; max_seq_len <= max_pages_per_seq * page_size.
 * Workspace: focal_gqa_decode_workspace_size(B, Hq, Hkv, max_seq_len, D)
 * bytes, same rules as above.  A page id or length out of range sets device
 * status 3 and is clamped (the output is then not meaningful).  With every
 * seq_lens[b] == max_seq_len and the pages holding the contiguous caches, the
 * result is bit-identical to focal_gqa_decode_attn's. */
int focal_gqa_decode_paged(const void* q, const void* k_pages, const void* v_pages, const int32_t* block_table,
                           const int32_t* seq_lens, void* o, int B, int Hq, int Hkv, int D, int num_pages,
                           int page_size, int max_pages_per_seq, int max_seq_len, float scale, void* workspace,
                           size_t ws_bytes, cudaStream_t stream);

/* ------------------------------------------------------------ diagnostics ---
 * Device-side status word of the current device: 0 while every kernel's
 * bounded waits have completed; otherwise 1 (a pipeline wait gave up), 2 (a
 * tensor-parallel peer did not deliver in time) or 3 (a paged-KV page id or
 * sequence length out of range).
 * The word lives in mapped pinned host memory, one per device.
 * focal_device_status synchronizes the device first, so it covers every call
 * made before it; focal_device_status_peek reads the word as it stands (calls
 * that have finished), with no synchronization, so a caller can check it
 * before each launch (the PyTorch wrapper does, and on a nonzero word re-zeroes
 * its cached workspaces and raises).  focal_reset_device_status clears it.
 * (No counterpart in the reference, which has no bounded device waits.) */
int focal_device_status(int* status_out);
int focal_device_status_peek(int* status_out);
int focal_reset_device_status(void);

#ifdef __cplusplus
}
#endif

#endif /* FOCAL_B200_H_ */
