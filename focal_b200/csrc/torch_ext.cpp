// Thin PyTorch extension over the focal_b200 C ABI; the replacement for the
// reference's pybind11 binding (csrc/bindings.cpp:4-16) and its tensor-level
// launcher (csrc/w4a16_gemv.cu:119-235).
//
// It keeps the reference's contract at the tensor level: inputs are CUDA,
// contiguous and of the exact dtype; the output is allocated here with
// torch::empty on x's device; work is queued on PyTorch's current stream under
// a device guard; failures raise RuntimeError with the reference's messages.
// All arithmetic happens in libfocal_b200.so behind include/focal_b200.h.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <algorithm>
#include <cmath>
#include <map>
#include <mutex>
#include <tuple>
#include <utility>
#include <vector>

#include "focal_b200.h"

namespace {

void check_tensor(const torch::Tensor& t, const char* name, c10::ScalarType dtype) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
  TORCH_CHECK(t.scalar_type() == dtype, name, " has wrong dtype");
}

void raise_on(int rc) {
  if (rc != FOCAL_OK) TORCH_CHECK(false, focal_last_error());
}

cudaStream_t current_stream() {
  return reinterpret_cast<cudaStream_t>(at::cuda::getCurrentCUDAStream().stream());
}

// Device workspaces, one per (kind, device, stream), zeroed when allocated.
// Their partial words start at zero and every successful call leaves them at zero,
// and calls on one stream are ordered, so reuse is safe.  A workspace that is
// outgrown stays allocated (a CUDA graph captured earlier may still use it).
enum WsKind { kWsLinear = 0, kWsAttention = 1 };
std::mutex g_ws_mutex;
std::map<std::tuple<int, int, cudaStream_t>, torch::Tensor> g_ws;
std::vector<torch::Tensor> g_ws_retired;

// A kernel that gave up a bounded device-side wait (a timed-out pipeline or
// tensor-parallel peer) wrote a nonzero status word and may have left row-block
// partial words in a workspace set.  Before every call that uses a workspace the
// word is read (mapped host memory, no device sync); when it is set, every
// cached workspace of the device is zeroed again on its own stream, the word is
// cleared and the call raises, so the failure is reported once and later calls
// are valid.  Called with g_ws_mutex held.
void check_device_status_locked(const torch::Device& dev) {
  int st = 0;
  raise_on(focal_device_status_peek(&st));
  if (st == 0) return;
  for (auto& kv : g_ws)
    if (std::get<1>(kv.first) == (int)dev.index()) {
      const cudaError_t e =
          cudaMemsetAsync(kv.second.data_ptr(), 0, (size_t)kv.second.numel(), std::get<2>(kv.first));
      TORCH_CHECK(e == cudaSuccess, "cudaMemsetAsync (workspace reset): ", cudaGetErrorString(e));
    }
  raise_on(focal_reset_device_status());
  TORCH_CHECK(false, "focal_b200: an earlier call on cuda:", (int)dev.index(),
              " gave up a bounded device-side wait (status ", st,
              st == 2 ? ": a tensor-parallel peer did not deliver" : st == 3 ? ": bad paged-KV index" : ": pipeline wait",
              "); its output is invalid.  The cached workspaces were zeroed again and the status cleared; "
              "later calls are valid.");
}

torch::Tensor workspace_for(WsKind kind, const torch::Device& dev, cudaStream_t stream, size_t bytes) {
  std::lock_guard<std::mutex> lock(g_ws_mutex);
  check_device_status_locked(dev);
  auto key = std::make_tuple((int)kind, (int)dev.index(), stream);
  auto it = g_ws.find(key);
  if (it == g_ws.end() || (size_t)it->second.numel() < bytes) {
    if (it != g_ws.end()) g_ws_retired.push_back(it->second);
    auto t = torch::zeros({(int64_t)bytes}, torch::TensorOptions().dtype(torch::kUInt8).device(dev));
    g_ws[key] = t;
    return t;
  }
  return it->second;
}

torch::Tensor w4a16_workspace(const torch::Tensor& x, int64_t N) {
  const size_t n = focal_w4a16_workspace_size((int)x.size(0), (int)x.size(1), (int)N);
  return workspace_for(kWsLinear, x.device(), current_stream(), std::max<size_t>(n, 256));
}

// Validation in the reference's order and wording (csrc/w4a16_gemv.cu:157-177).
void check_w4a16(const torch::Tensor& x, const torch::Tensor& wq, const torch::Tensor& scales,
                 const torch::Tensor& zeros) {
  check_tensor(x, "x", at::kBFloat16);
  check_tensor(wq, "wq", at::kInt);
  check_tensor(scales, "scales", at::kHalf);
  check_tensor(zeros, "zeros", at::kHalf);
  TORCH_CHECK(x.dim() == 2, "x must have shape [M, K]");
  TORCH_CHECK(wq.dim() == 2, "wq must have shape [N, K / 8]");
  TORCH_CHECK(scales.dim() == 2, "scales must have shape [N, K / 128]");
  TORCH_CHECK(zeros.dim() == 2, "zeros must have shape [N, K / 128]");
  TORCH_CHECK(wq.device() == x.device(), "wq must be on the same device as x");
  TORCH_CHECK(scales.device() == x.device(), "scales must be on the same device as x");
  TORCH_CHECK(zeros.device() == x.device(), "zeros must be on the same device as x");
  const int64_t M = x.size(0), K = x.size(1), N = wq.size(0);
  TORCH_CHECK(M <= INT32_MAX && K <= INT32_MAX && N <= INT32_MAX, "unsupported K/N");
  raise_on(focal_w4a16_check_shape((int)M, (int)K, (int)N));
  TORCH_CHECK(wq.size(1) == K / 8, "wq must have shape [N, K / 8]");
  TORCH_CHECK(scales.size(0) == N && scales.size(1) == K / 128,
              "scales must have shape [N, K / 128]");
  TORCH_CHECK(zeros.size(0) == N && zeros.size(1) == K / 128,
              "zeros must have shape [N, K / 128]");
}

torch::Tensor w4a16_linear(torch::Tensor x, torch::Tensor wq, torch::Tensor scales,
                           torch::Tensor zeros) {
  check_w4a16(x, wq, scales, zeros);
  const c10::cuda::CUDAGuard guard(x.device());
  const int M = (int)x.size(0), K = (int)x.size(1), N = (int)wq.size(0);
  auto y = torch::empty({M, N}, x.options());
  auto ws = w4a16_workspace(x, N);
  raise_on(focal_w4a16_gemv(x.data_ptr(), wq.data_ptr<int32_t>(), scales.data_ptr(),
                            zeros.data_ptr(), y.data_ptr(), M, K, N, ws.data_ptr(), ws.numel(),
                            current_stream()));
  return y;
}

torch::Tensor w4a16_linear_f32(torch::Tensor x, torch::Tensor wq, torch::Tensor scales,
                               torch::Tensor zeros) {
  check_w4a16(x, wq, scales, zeros);
  const c10::cuda::CUDAGuard guard(x.device());
  const int M = (int)x.size(0), K = (int)x.size(1), N = (int)wq.size(0);
  auto y = torch::empty({M, N}, x.options().dtype(torch::kFloat32));
  auto ws = w4a16_workspace(x, N);
  raise_on(focal_w4a16_gemv_f32(x.data_ptr(), wq.data_ptr<int32_t>(), scales.data_ptr(),
                                zeros.data_ptr(), y.data_ptr<float>(), M, K, N, ws.data_ptr(),
                                ws.numel(), current_stream()));
  return y;
}

torch::Tensor w4a16_gate_up_silu(torch::Tensor x, torch::Tensor wq_gate, torch::Tensor scales_gate,
                                 torch::Tensor zeros_gate, torch::Tensor wq_up,
                                 torch::Tensor scales_up, torch::Tensor zeros_up) {
  check_w4a16(x, wq_gate, scales_gate, zeros_gate);
  check_w4a16(x, wq_up, scales_up, zeros_up);
  TORCH_CHECK(wq_up.sizes() == wq_gate.sizes(), "gate and up weights must have the same shape");
  const c10::cuda::CUDAGuard guard(x.device());
  const int M = (int)x.size(0), K = (int)x.size(1), N = (int)wq_gate.size(0);
  auto h = torch::empty({M, N}, x.options());
  auto ws = w4a16_workspace(x, N);
  raise_on(focal_w4a16_gate_up_silu(x.data_ptr(), wq_gate.data_ptr<int32_t>(),
                                    scales_gate.data_ptr(), zeros_gate.data_ptr(),
                                    wq_up.data_ptr<int32_t>(), scales_up.data_ptr(),
                                    zeros_up.data_ptr(), h.data_ptr(), M, K, N, ws.data_ptr(),
                                    ws.numel(), current_stream()));
  return h;
}

// Unit-tiled weights (include/focal_b200.h): tiles is a uint8 tensor of
// focal_w4a16_tiles_size(K, N) bytes made by tile_pack.
torch::Tensor tile_pack(torch::Tensor wq, torch::Tensor scales, torch::Tensor zeros) {
  check_tensor(wq, "wq", at::kInt);
  check_tensor(scales, "scales", at::kHalf);
  check_tensor(zeros, "zeros", at::kHalf);
  TORCH_CHECK(wq.dim() == 2, "wq must have shape [N, K / 8]");
  const int64_t N = wq.size(0), K = wq.size(1) * 8;
  TORCH_CHECK(scales.dim() == 2 && scales.size(0) == N && scales.size(1) == K / 128,
              "scales must have shape [N, K / 128]");
  TORCH_CHECK(zeros.dim() == 2 && zeros.size(0) == N && zeros.size(1) == K / 128,
              "zeros must have shape [N, K / 128]");
  TORCH_CHECK(K <= INT32_MAX && N <= INT32_MAX, "unsupported K/N");
  const size_t n = focal_w4a16_tiles_size((int)K, (int)N);
  TORCH_CHECK(n > 0, "unsupported K/N");
  const c10::cuda::CUDAGuard guard(wq.device());
  auto t = torch::empty({(int64_t)n}, wq.options().dtype(torch::kUInt8));
  raise_on(focal_w4a16_tile_pack(wq.data_ptr<int32_t>(), scales.data_ptr(), zeros.data_ptr(), t.data_ptr(),
                                 (int)K, (int)N, current_stream()));
  return t;
}

void check_tiled(const torch::Tensor& x, const torch::Tensor& tiles, int64_t N) {
  check_tensor(x, "x", at::kBFloat16);
  check_tensor(tiles, "tiles", at::kByte);
  TORCH_CHECK(x.dim() == 2, "x must have shape [M, K]");
  TORCH_CHECK(tiles.device() == x.device(), "tiles must be on the same device as x");
  const int64_t M = x.size(0), K = x.size(1);
  TORCH_CHECK(M <= INT32_MAX && K <= INT32_MAX && N > 0 && N <= INT32_MAX, "unsupported K/N");
  raise_on(focal_w4a16_check_shape((int)M, (int)K, (int)N));
  TORCH_CHECK(tiles.dim() == 1 && (size_t)tiles.numel() == focal_w4a16_tiles_size((int)K, (int)N),
              "tiles must hold focal_w4a16_tiles_size(K, N) bytes");
}

torch::Tensor w4a16_linear_tiled(torch::Tensor x, torch::Tensor tiles, int64_t N) {
  check_tiled(x, tiles, N);
  const c10::cuda::CUDAGuard guard(x.device());
  const int M = (int)x.size(0), K = (int)x.size(1);
  auto y = torch::empty({M, N}, x.options());
  auto ws = w4a16_workspace(x, N);
  raise_on(focal_w4a16_gemv_tiled(x.data_ptr(), tiles.data_ptr(), y.data_ptr(), M, K, (int)N, ws.data_ptr(),
                                  ws.numel(), current_stream()));
  return y;
}

torch::Tensor w4a16_linear_tiled_f32(torch::Tensor x, torch::Tensor tiles, int64_t N) {
  check_tiled(x, tiles, N);
  const c10::cuda::CUDAGuard guard(x.device());
  const int M = (int)x.size(0), K = (int)x.size(1);
  auto y = torch::empty({M, N}, x.options().dtype(torch::kFloat32));
  auto ws = w4a16_workspace(x, N);
  raise_on(focal_w4a16_gemv_tiled_f32(x.data_ptr(), tiles.data_ptr(), y.data_ptr<float>(), M, K, (int)N,
                                      ws.data_ptr(), ws.numel(), current_stream()));
  return y;
}

torch::Tensor w4a16_gate_up_silu_tiled(torch::Tensor x, torch::Tensor tiles_gate, torch::Tensor tiles_up,
                                       int64_t N) {
  check_tiled(x, tiles_gate, N);
  check_tiled(x, tiles_up, N);
  const c10::cuda::CUDAGuard guard(x.device());
  const int M = (int)x.size(0), K = (int)x.size(1);
  auto h = torch::empty({M, N}, x.options());
  auto ws = w4a16_workspace(x, N);
  raise_on(focal_w4a16_gate_up_silu_tiled(x.data_ptr(), tiles_gate.data_ptr(), tiles_up.data_ptr(), h.data_ptr(),
                                          M, K, (int)N, ws.data_ptr(), ws.numel(), current_stream()));
  return h;
}

torch::Tensor dequant(torch::Tensor wq, torch::Tensor scales, torch::Tensor zeros, int64_t K) {
  check_tensor(wq, "wq", at::kInt);
  check_tensor(scales, "scales", at::kHalf);
  check_tensor(zeros, "zeros", at::kHalf);
  TORCH_CHECK(wq.dim() == 2, "wq must have shape [N, K / 8]");
  TORCH_CHECK(K % 128 == 0, "K must be divisible by 128");
  const int64_t N = wq.size(0);
  TORCH_CHECK(wq.size(1) * 8 == K, "wq shape does not match K");
  TORCH_CHECK(scales.dim() == 2 && scales.size(0) == N && scales.size(1) == K / 128,
              "scales must have shape [N, K / 128]");
  TORCH_CHECK(zeros.dim() == 2 && zeros.size(0) == N && zeros.size(1) == K / 128,
              "zeros must have shape [N, K / 128]");
  const c10::cuda::CUDAGuard guard(wq.device());
  auto w = torch::empty({N, K}, wq.options().dtype(torch::kFloat32));
  raise_on(focal_w4a16_dequant(wq.data_ptr<int32_t>(), scales.data_ptr(), zeros.data_ptr(),
                               w.data_ptr<float>(), (int)K, (int)N, current_stream()));
  return w;
}

torch::Tensor pack_int4(torch::Tensor q) {
  check_tensor(q, "w_q_uint8", at::kByte);
  TORCH_CHECK(q.dim() == 2, "w_q_uint8 must have shape [N, K]");
  const int64_t N = q.size(0), K = q.size(1);
  TORCH_CHECK(K % 8 == 0, "K must be divisible by 8");
  const c10::cuda::CUDAGuard guard(q.device());
  auto wq = torch::empty({N, K / 8}, q.options().dtype(torch::kInt32));
  raise_on(focal_pack_int4(q.data_ptr<uint8_t>(), wq.data_ptr<int32_t>(), (int)N, (int)K,
                           current_stream()));
  return wq;
}

torch::Tensor gqa_decode_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                                   c10::optional<double> scale) {
  check_tensor(q, "q", at::kBFloat16);
  check_tensor(k_cache, "k_cache", at::kBFloat16);
  check_tensor(v_cache, "v_cache", at::kBFloat16);
  TORCH_CHECK(q.dim() == 3, "q must have shape [B, Hq, D]");
  TORCH_CHECK(k_cache.dim() == 4, "k_cache must have shape [B, Hkv, L, D]");
  TORCH_CHECK(v_cache.sizes() == k_cache.sizes(), "v_cache must have the shape of k_cache");
  TORCH_CHECK(k_cache.device() == q.device(), "k_cache must be on the same device as q");
  TORCH_CHECK(v_cache.device() == q.device(), "v_cache must be on the same device as q");
  const int64_t B = q.size(0), Hq = q.size(1), D = q.size(2);
  const int64_t Hkv = k_cache.size(1), L = k_cache.size(2);
  TORCH_CHECK(k_cache.size(0) == B && k_cache.size(3) == D, "k_cache must have shape [B, Hkv, L, D]");
  TORCH_CHECK(B <= INT32_MAX && L <= INT32_MAX, "unsupported size");
  const double sc = scale.has_value() ? *scale : 1.0 / std::sqrt((double)D);
  const c10::cuda::CUDAGuard guard(q.device());
  auto o = torch::empty({B, Hq, D}, q.options());
  const cudaStream_t stream = current_stream();
  const size_t ws_bytes = focal_gqa_decode_workspace_size((int)B, (int)Hq, (int)Hkv, (int)L, (int)D);
  void* ws = nullptr;
  torch::Tensor ws_t;
  if (ws_bytes > 0) {
    ws_t = workspace_for(kWsAttention, q.device(), stream, ws_bytes);
    ws = ws_t.data_ptr();
  }
  raise_on(focal_gqa_decode_attn(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), o.data_ptr(),
                                 (int)B, (int)Hq, (int)Hkv, (int)L, (int)D, (float)sc, ws, ws_bytes,
                                 stream));
  return o;
}

torch::Tensor gqa_decode_attention_paged(torch::Tensor q, torch::Tensor k_pages, torch::Tensor v_pages,
                                         torch::Tensor block_table, torch::Tensor seq_lens, int64_t max_seq_len,
                                         c10::optional<double> scale) {
  check_tensor(q, "q", at::kBFloat16);
  check_tensor(k_pages, "k_pages", at::kBFloat16);
  check_tensor(v_pages, "v_pages", at::kBFloat16);
  check_tensor(block_table, "block_table", at::kInt);
  check_tensor(seq_lens, "seq_lens", at::kInt);
  TORCH_CHECK(q.dim() == 3, "q must have shape [B, Hq, D]");
  TORCH_CHECK(k_pages.dim() == 4, "k_pages must have shape [num_pages, Hkv, page_size, D]");
  TORCH_CHECK(v_pages.sizes() == k_pages.sizes(), "v_pages must have the shape of k_pages");
  const int64_t B = q.size(0), Hq = q.size(1), D = q.size(2);
  TORCH_CHECK(block_table.dim() == 2 && block_table.size(0) == B, "block_table must have shape [B, max_pages]");
  TORCH_CHECK(seq_lens.dim() == 1 && seq_lens.size(0) == B, "seq_lens must have shape [B]");
  for (const auto* t : {&k_pages, &v_pages, &block_table, &seq_lens})
    TORCH_CHECK(t->device() == q.device(), "all tensors must be on q's device");
  TORCH_CHECK(k_pages.size(3) == D, "k_pages must have shape [num_pages, Hkv, page_size, D]");
  TORCH_CHECK(k_pages.size(0) <= INT32_MAX && max_seq_len <= INT32_MAX && max_seq_len >= 1, "unsupported size");
  const double sc = scale.has_value() ? *scale : 1.0 / std::sqrt((double)D);
  const c10::cuda::CUDAGuard guard(q.device());
  auto o = torch::empty({B, Hq, D}, q.options());
  const cudaStream_t stream = current_stream();
  const int Hkv = (int)k_pages.size(1);
  const size_t ws_bytes = focal_gqa_decode_workspace_size((int)B, (int)Hq, Hkv, (int)max_seq_len, (int)D);
  void* ws = nullptr;
  torch::Tensor ws_t;
  if (ws_bytes > 0) {
    ws_t = workspace_for(kWsAttention, q.device(), stream, ws_bytes);
    ws = ws_t.data_ptr();
  }
  raise_on(focal_gqa_decode_paged(q.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(),
                                  block_table.data_ptr<int32_t>(), seq_lens.data_ptr<int32_t>(), o.data_ptr(),
                                  (int)B, (int)Hq, Hkv, (int)D, (int)k_pages.size(0), (int)k_pages.size(2),
                                  (int)block_table.size(1), (int)max_seq_len, (float)sc, ws, ws_bytes, stream));
  return o;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("w4a16_linear", &w4a16_linear, "W4A16 small-M linear (B200 sm_100a)");
  m.def("w4a16_linear_f32", &w4a16_linear_f32, "W4A16 small-M linear, fp32 output");
  m.def("w4a16_gate_up_silu", &w4a16_gate_up_silu, "fused gate/up projections with SiLU(gate)*up");
  m.def("tile_pack", &tile_pack, "re-layout W4A16 weights into the unit-tiled format");
  m.def("w4a16_linear_tiled", &w4a16_linear_tiled, "W4A16 small-M linear on unit-tiled weights");
  m.def("w4a16_linear_tiled_f32", &w4a16_linear_tiled_f32, "as w4a16_linear_tiled, fp32 output");
  m.def("w4a16_gate_up_silu_tiled", &w4a16_gate_up_silu_tiled, "fused gate/up/SiLU on unit-tiled weights");
  m.def("dequant", &dequant, "fp32 dequantized weights (bit-identical to dequant_ref)");
  m.def("pack_int4", &pack_int4, "pack uint8 [N,K] nibbles into int32 [N,K/8]");
  m.def("gqa_decode_attention_paged", &gqa_decode_attention_paged, "paged variable-length GQA decode attention",
        pybind11::arg("q"), pybind11::arg("k_pages"), pybind11::arg("v_pages"), pybind11::arg("block_table"),
        pybind11::arg("seq_lens"), pybind11::arg("max_seq_len"), pybind11::arg("scale") = pybind11::none());
  m.def("gqa_decode_attention", &gqa_decode_attention, "contiguous GQA decode attention",
        pybind11::arg("q"), pybind11::arg("k_cache"), pybind11::arg("v_cache"),
        pybind11::arg("scale") = pybind11::none());
}
