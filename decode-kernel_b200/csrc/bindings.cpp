// bindings.cpp -- torch extension `decode_kernel._cuda`, a thin layer over the
// C ABI in include/dk_w4a16.h.
//
// Keeps the reference module's exports, argument names, defaults and error
// messages (RohanDisa/decode-kernel csrc/bindings.cpp:10-48, 114-129) so code
// and tests written against the reference run unchanged:
//   w4a16_gemv(packed, scales, x, version=5, split_k=4, reuse_weights=False,
//              warps_per_row=1) -> fp16 [B, M]
//   d2d_copy(src, dst), stream_read(src, partials), stream_write(dst),
//   stream_recommended_blocks(), last_kernel_stamp()
// and adds: w4a16_gemv_out (caller-provided y, optional PDL launch),
// workspace_bytes, quantize_pack / unpack_to_int / dequantize on the GPU,
// device_error.  Every C-ABI status other than DK_OK becomes a RuntimeError.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstdint>
#include <string>

#include "dk_w4a16.h"

namespace {

void check_status(dk_status s, const char* what) {
  if (s == DK_OK) return;
  std::string msg = std::string(what) + ": " + dk_status_string(s);
  if (s == DK_ERR_LAUNCH || s == DK_ERR_CUDA) msg += std::string(" [") + dk_last_cuda_error() + "]";
  TORCH_CHECK(false, msg);
}

bool aligned16(const torch::Tensor& t) {
  return (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15u) == 0;
}

// bindings.cpp:10-33
void check_gemv_inputs(const torch::Tensor& packed, const torch::Tensor& scales,
                       const torch::Tensor& x) {
  TORCH_CHECK(packed.is_cuda() && scales.is_cuda() && x.is_cuda(),
              "packed, scales, and x must be CUDA tensors");
  TORCH_CHECK(packed.scalar_type() == torch::kInt32, "packed must be int32 (uint32 bit pattern)");
  TORCH_CHECK(scales.scalar_type() == torch::kFloat16, "scales must be fp16");
  TORCH_CHECK(x.scalar_type() == torch::kFloat16, "x must be fp16");
  TORCH_CHECK(packed.dim() == 2 && scales.dim() == 2 && x.dim() == 2,
              "packed [M,K/8], scales [M,K/128], x [B,K]");
  TORCH_CHECK(packed.is_contiguous() && scales.is_contiguous() && x.is_contiguous(),
              "packed, scales, and x must be contiguous");
  const int64_t M = packed.size(0);
  const int64_t K = packed.size(1) * DK_NIBBLES_PER_WORD;
  TORCH_CHECK(K % DK_GROUP_SIZE == 0, "K must be divisible by group size 128");
  TORCH_CHECK(scales.size(0) == M && scales.size(1) == K / DK_GROUP_SIZE,
              "scales shape must be [M, K/128]");
  TORCH_CHECK(x.size(1) == K, "x.shape[1] must equal K");
  TORCH_CHECK(packed.device() == scales.device() && packed.device() == x.device(),
              "packed, scales, and x must be on the same device");
  TORCH_CHECK(M <= INT32_MAX && K <= INT32_MAX && x.size(0) <= INT32_MAX,
              "dimensions must fit in int32");
}

// bindings.cpp:41-48
dk_gemv_config make_config(int version, int split_k, bool reuse_weights, int warps_per_row,
                           bool pdl) {
  TORCH_CHECK(version >= 0 && version <= 5, "version must be 0..5");
  TORCH_CHECK(split_k >= 1 && split_k <= 32, "split_k must be in [1, 32]");
  TORCH_CHECK(warps_per_row >= 1 && warps_per_row <= 8, "warps_per_row must be in [1, 8]");
  if (warps_per_row > 1) {
    TORCH_CHECK(version == 1 && !reuse_weights,
                "warps_per_row > 1 is implemented for streaming v1 only");
  }
  dk_gemv_config cfg;
  dk_gemv_config_init(&cfg);
  cfg.version = version;
  cfg.split_k = split_k;
  cfg.reuse_weights = reuse_weights ? 1 : 0;
  cfg.warps_per_row = warps_per_row;
  cfg.flags = pdl ? DK_FLAG_PDL : 0u;
  return cfg;
}

void run_gemv(const torch::Tensor& packed_in, const torch::Tensor& scales,
              const torch::Tensor& x_in, torch::Tensor& y, const dk_gemv_config& cfg) {
  // The kernels stream with 128-bit loads: re-home a (rare) misaligned view.
  const torch::Tensor packed = aligned16(packed_in) ? packed_in : packed_in.clone();
  const torch::Tensor x = aligned16(x_in) ? x_in : x_in.clone();
  const int M = static_cast<int>(packed.size(0));
  const int K = static_cast<int>(packed.size(1) * DK_NIBBLES_PER_WORD);
  const int B = static_cast<int>(x.size(0));
  const size_t ws_bytes = dk_w4a16_workspace_bytes(M, K, B, &cfg);
  torch::Tensor ws;
  if (ws_bytes) ws = torch::empty({static_cast<int64_t>(ws_bytes)}, x.options().dtype(torch::kUInt8));
  check_status(
      dk_w4a16_gemv(packed.data_ptr<int32_t>(),
                    reinterpret_cast<const uint16_t*>(scales.data_ptr<at::Half>()),
                    reinterpret_cast<const uint16_t*>(x.data_ptr<at::Half>()),
                    reinterpret_cast<uint16_t*>(y.data_ptr<at::Half>()), M, K, B, &cfg,
                    ws_bytes ? ws.data_ptr() : nullptr, ws_bytes,
                    at::cuda::getCurrentCUDAStream().stream()),
      "w4a16_gemv");
}

torch::Tensor w4a16_gemv(torch::Tensor packed, torch::Tensor scales, torch::Tensor x,
                         int version, int split_k, bool reuse_weights, int warps_per_row) {
  check_gemv_inputs(packed, scales, x);
  const dk_gemv_config cfg = make_config(version, split_k, reuse_weights, warps_per_row, false);
  const c10::cuda::CUDAGuard guard(x.device());
  auto y = torch::empty({x.size(0), packed.size(0)}, x.options());
  run_gemv(packed, scales, x, y, cfg);
  return y;
}

void w4a16_gemv_out(torch::Tensor packed, torch::Tensor scales, torch::Tensor x, torch::Tensor y,
                    int version, int split_k, bool reuse_weights, int warps_per_row, bool pdl) {
  check_gemv_inputs(packed, scales, x);
  TORCH_CHECK(y.is_cuda() && y.device() == x.device(), "y must be on x's device");
  TORCH_CHECK(y.scalar_type() == torch::kFloat16 && y.is_contiguous(), "y must be contiguous fp16");
  TORCH_CHECK(y.dim() == 2 && y.size(0) == x.size(0) && y.size(1) == packed.size(0),
              "y must be [B, M]");
  const dk_gemv_config cfg = make_config(version, split_k, reuse_weights, warps_per_row, pdl);
  const c10::cuda::CUDAGuard guard(x.device());
  run_gemv(packed, scales, x, y, cfg);
}

int64_t workspace_bytes(int64_t M, int64_t K, int64_t B, int version, int split_k,
                        bool reuse_weights) {
  const dk_gemv_config cfg = make_config(version, split_k, reuse_weights, 1, false);
  return static_cast<int64_t>(dk_w4a16_workspace_bytes(static_cast<int>(M), static_cast<int>(K),
                                                       static_cast<int>(B), &cfg));
}

// bindings.cpp:80-110
void d2d_copy(torch::Tensor src, torch::Tensor dst) {
  TORCH_CHECK(src.is_cuda() && dst.is_cuda(), "src and dst must be CUDA");
  TORCH_CHECK(src.nbytes() == dst.nbytes(), "src/dst size mismatch");
  TORCH_CHECK(src.nbytes() % 16 == 0, "copy size must be a multiple of 16");
  const c10::cuda::CUDAGuard guard(src.device());
  check_status(dk_d2d_copy(src.data_ptr(), dst.data_ptr(), src.nbytes(),
                           at::cuda::getCurrentCUDAStream().stream()),
               "d2d_copy");
}

void stream_read(torch::Tensor src, torch::Tensor partials) {
  TORCH_CHECK(src.is_cuda() && partials.is_cuda(), "src and partials must be CUDA");
  TORCH_CHECK(src.nbytes() % 16 == 0, "buffer size must be a multiple of 16");
  TORCH_CHECK(partials.scalar_type() == torch::kFloat32, "partials must be fp32");
  TORCH_CHECK(partials.is_contiguous(), "partials must be contiguous");
  const int blocks = static_cast<int>(partials.numel());
  TORCH_CHECK(blocks >= 1, "partials must have one float per block");
  const c10::cuda::CUDAGuard guard(src.device());
  check_status(dk_stream_read(src.data_ptr(), partials.data_ptr<float>(), src.nbytes(), blocks,
                              at::cuda::getCurrentCUDAStream().stream()),
               "stream_read");
}

void stream_write(torch::Tensor dst) {
  TORCH_CHECK(dst.is_cuda(), "dst must be CUDA");
  TORCH_CHECK(dst.nbytes() % 16 == 0, "buffer size must be a multiple of 16");
  const c10::cuda::CUDAGuard guard(dst.device());
  check_status(dk_stream_write(dst.data_ptr(), dst.nbytes(), dk_stream_recommended_blocks(-1),
                               at::cuda::getCurrentCUDAStream().stream()),
               "stream_write");
}

int stream_recommended_blocks() { return dk_stream_recommended_blocks(-1); }

int last_kernel_stamp() { return dk_last_kernel_stamp(-1); }

int device_error(bool clear) { return dk_device_error(-1, clear ? 1 : 0); }

std::vector<torch::Tensor> quantize_pack(torch::Tensor w, bool torch_cuda_scale) {
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == torch::kFloat32 && w.dim() == 2,
              "weight must be a 2-D fp32 CUDA tensor");
  const int64_t M = w.size(0), K = w.size(1);
  TORCH_CHECK(K % DK_GROUP_SIZE == 0, "K=", K, " is not divisible by group_size=", DK_GROUP_SIZE);
  TORCH_CHECK(M <= INT32_MAX && K <= INT32_MAX, "dimensions must fit in int32");
  const c10::cuda::CUDAGuard guard(w.device());
  torch::Tensor wc = w.contiguous();
  if (!aligned16(wc)) wc = wc.clone();
  auto packed = torch::empty({M, K / DK_NIBBLES_PER_WORD}, w.options().dtype(torch::kInt32));
  auto scales = torch::empty({M, K / DK_GROUP_SIZE}, w.options().dtype(torch::kFloat16));
  check_status(dk_quantize_pack(wc.data_ptr<float>(), static_cast<int>(M), static_cast<int>(K),
                                packed.data_ptr<int32_t>(),
                                reinterpret_cast<uint16_t*>(scales.data_ptr<at::Half>()),
                                torch_cuda_scale ? DK_QUANT_TORCH_CUDA_SCALE : 0u,
                                at::cuda::getCurrentCUDAStream().stream()),
               "quantize_pack");
  return {packed, scales};
}

torch::Tensor unpack_to_int(torch::Tensor packed) {
  TORCH_CHECK(packed.is_cuda() && packed.scalar_type() == torch::kInt32 && packed.dim() == 2,
              "packed must be a 2-D int32 CUDA tensor");
  const int64_t M = packed.size(0), K = packed.size(1) * DK_NIBBLES_PER_WORD;
  TORCH_CHECK(K % DK_GROUP_SIZE == 0, "K must be divisible by group size 128");
  const c10::cuda::CUDAGuard guard(packed.device());
  auto pc = packed.contiguous();
  auto q = torch::empty({M, K}, packed.options());
  check_status(dk_unpack_to_int(pc.data_ptr<int32_t>(), static_cast<int>(M), static_cast<int>(K),
                                q.data_ptr<int32_t>(), at::cuda::getCurrentCUDAStream().stream()),
               "unpack_to_int");
  return q;
}

torch::Tensor dequantize(torch::Tensor packed, torch::Tensor scales) {
  TORCH_CHECK(packed.is_cuda() && scales.is_cuda(), "packed and scales must be CUDA tensors");
  TORCH_CHECK(packed.scalar_type() == torch::kInt32 && scales.scalar_type() == torch::kFloat16,
              "packed int32, scales fp16");
  const int64_t M = packed.size(0), K = packed.size(1) * DK_NIBBLES_PER_WORD;
  TORCH_CHECK(K % DK_GROUP_SIZE == 0 && scales.size(0) == M && scales.size(1) == K / DK_GROUP_SIZE,
              "scales shape must be [M, K/128]");
  const c10::cuda::CUDAGuard guard(packed.device());
  auto pc = packed.contiguous();
  auto sc = scales.contiguous();
  auto w = torch::empty({M, K}, packed.options().dtype(torch::kFloat32));
  check_status(dk_dequantize(pc.data_ptr<int32_t>(),
                             reinterpret_cast<const uint16_t*>(sc.data_ptr<at::Half>()),
                             static_cast<int>(M), static_cast<int>(K), w.data_ptr<float>(),
                             at::cuda::getCurrentCUDAStream().stream()),
               "dequantize");
  return w;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("w4a16_gemv", &w4a16_gemv, "W4A16 GEMV", py::arg("packed"), py::arg("scales"),
        py::arg("x"), py::arg("version") = 5, py::arg("split_k") = 4,
        py::arg("reuse_weights") = false, py::arg("warps_per_row") = 1);
  m.def("w4a16_gemv_out", &w4a16_gemv_out, "W4A16 GEMV into a caller-provided y",
        py::arg("packed"), py::arg("scales"), py::arg("x"), py::arg("y"), py::arg("version") = 5,
        py::arg("split_k") = 4, py::arg("reuse_weights") = false, py::arg("warps_per_row") = 1,
        py::arg("pdl") = false);
  m.def("workspace_bytes", &workspace_bytes, "Workspace bytes for a GEMV", py::arg("M"),
        py::arg("K"), py::arg("B"), py::arg("version") = 5, py::arg("split_k") = 4,
        py::arg("reuse_weights") = false);
  m.def("d2d_copy", &d2d_copy, "Aligned device-to-device copy", py::arg("src"), py::arg("dst"));
  m.def("stream_read", &stream_read, "Read-only STREAM sum-reduction (one float partial per block)",
        py::arg("src"), py::arg("partials"));
  m.def("stream_write", &stream_write, "Write-only STREAM fill", py::arg("dst"));
  m.def("stream_recommended_blocks", &stream_recommended_blocks,
        "Block count used by STREAM probes");
  m.def("last_kernel_stamp", &last_kernel_stamp,
        "Stage stamp written by the GEMV that actually launched");
  m.def("device_error", &device_error, "Device-side error word (1 = bounded wait timed out)",
        py::arg("clear") = false);
  m.def("quantize_pack", &quantize_pack, "GPU quantize_and_pack (bit-exact)", py::arg("weight"),
        py::arg("torch_cuda_scale") = false);
  m.def("unpack_to_int", &unpack_to_int, "GPU unpack_to_int", py::arg("packed"));
  m.def("dequantize", &dequantize, "GPU dequantize to fp32", py::arg("packed"), py::arg("scales"));
  m.def("version", []() { return std::string(dk_version()); });
}
