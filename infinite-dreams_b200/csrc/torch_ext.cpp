// Native torch binding of the kernel bank's C ABI: the reference shipped its
// op as a pybind11/torch C++ extension (src/gemm_ext.cpp:22-132), and so does
// this build.  The ctypes path in infinite_dreams_ext.py reaches the same C
// ABI; this module removes the Python work around each call (argument checks,
// allocation of C, stream lookup, workspace lookup), which dominates the cost
// of a small GEMM launched back to back.
//
// Exported (all asynchronous on the current stream of A's device):
//   gemm_forward_cfg(A, B, cfg_id, out=None) -> C             (gemm_ext.cpp:95-106)
//   gemm_ex(A, B, cfg_id, alpha, beta, C, bias, act, out) -> out
//   reset_workspaces()
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <map>
#include <mutex>
#include <utility>

#include "../../include/gemm_sm100.h"

namespace {

// Split-K / repack workspace per (device, stream), zero-initialised once as
// the C ABI requires; grows geometrically.  Leaked on purpose: freeing CUDA
// memory from a static destructor at exit would race the context teardown.
std::mutex g_ws_mu;
std::map<std::pair<int, cudaStream_t>, at::Tensor>* g_ws = new std::map<std::pair<int, cudaStream_t>, at::Tensor>();

void* workspace(const at::Device& dev, cudaStream_t stream, size_t nbytes, size_t* len) {
  std::lock_guard<std::mutex> lock(g_ws_mu);
  at::Tensor& ws = (*g_ws)[{dev.index(), stream}];
  if (!ws.defined() || static_cast<size_t>(ws.numel()) < nbytes) {
    const int64_t grown = ws.defined() ? 2 * ws.numel() : 0;
    const int64_t size = std::max<int64_t>(static_cast<int64_t>(nbytes), grown);
    ws = at::zeros({size}, at::TensorOptions().dtype(at::kByte).device(dev));
  }
  *len = static_cast<size_t>(ws.numel());
  return ws.data_ptr();
}

void check_inputs(const at::Tensor& A, const at::Tensor& B) {
  // Same checks and messages as src/gemm_ext.cpp:66-73,86.
  TORCH_CHECK(A.is_cuda(), "A must be CUDA tensor");
  TORCH_CHECK(B.is_cuda(), "B must be CUDA tensor");
  TORCH_CHECK(A.scalar_type() == at::kHalf, "A must be float16");
  TORCH_CHECK(B.scalar_type() == at::kHalf, "B must be float16");
  TORCH_CHECK(A.dim() == 2, "A must be 2D (M x K)");
  TORCH_CHECK(B.dim() == 2, "B must be 2D (K x N)");
  TORCH_CHECK(A.size(1) == B.size(0), "Inner dimensions must match: A is (M x K), B is (K x N)");
  TORCH_CHECK(A.get_device() == B.get_device(), "A and B must be on the same CUDA device");
}

void check_status(int st, const char* what) {
  TORCH_CHECK(st == GEMM_OK, what, ": ", gemm_status_string(st), ": ", gemm_last_error());
}

at::Tensor output(const c10::optional<at::Tensor>& out, int64_t M, int64_t N, const at::Tensor& A) {
  if (!out.has_value()) return at::empty({M, N}, A.options());
  const at::Tensor& C = *out;
  TORCH_CHECK(C.scalar_type() == at::kHalf && C.dim() == 2 && C.size(0) == M && C.size(1) == N &&
                  C.device() == A.device() && (C.stride(1) == 1 || N <= 1),
              "out must be a float16 (M x N) tensor with unit column stride on A's device");
  return C;
}

at::Tensor gemm_forward_cfg(at::Tensor A, at::Tensor B, int64_t cfg_id, c10::optional<at::Tensor> out) {
  check_inputs(A, B);
  TORCH_CHECK(cfg_id >= 0, "cfg_id must be >= 0");
  TORCH_CHECK(cfg_id < gemm_num_cfgs(), "cfg_id out of range");
  const c10::cuda::CUDAGuard guard(A.device());
  A = A.contiguous();
  B = B.contiguous();
  const int64_t M = A.size(0), K = A.size(1), N = B.size(1);
  at::Tensor C = output(out, M, N, A);
  TORCH_CHECK(C.is_contiguous(), "out must be contiguous");
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(A.device().index()).stream();
  const size_t need = gemm_workspace_bytes(A.data_ptr(), B.data_ptr(), M, N, K, K, N, static_cast<int>(cfg_id));
  size_t len = 0;
  void* ws = need ? workspace(A.device(), stream, need, &len) : nullptr;
  check_status(gemm_launch(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, K, N, N, static_cast<int>(cfg_id),
                           ws, len, stream),
               "gemm_launch");
  return C;
}

// (tensor, trans, pitch) of a logical [R, C] operand read in place: a
// row-major view as stored, a transposed view (unit row stride) as its
// transposed storage, anything else copied contiguous.
std::tuple<at::Tensor, int, int64_t> operand(const at::Tensor& X) {
  const int64_t R = X.size(0), Cc = X.size(1), s0 = X.stride(0), s1 = X.stride(1);
  if ((s1 == 1 || Cc <= 1) && s0 >= std::max<int64_t>(Cc, 1)) return {X, 0, s0};
  if ((s0 == 1 || R <= 1) && s1 >= std::max<int64_t>(R, 1)) return {X, 1, s1};
  return {X.contiguous(), 0, std::max<int64_t>(Cc, 1)};
}

at::Tensor gemm_ex(const at::Tensor& A, const at::Tensor& B, int64_t cfg_id, double alpha, double beta,
                   c10::optional<at::Tensor> Cin, c10::optional<at::Tensor> bias, int64_t act,
                   c10::optional<at::Tensor> out) {
  check_inputs(A, B);
  TORCH_CHECK(cfg_id >= 0 && cfg_id < gemm_num_cfgs(), "cfg_id out of range");
  const c10::cuda::CUDAGuard guard(A.device());
  const int64_t M = A.size(0), K = A.size(1), N = B.size(1);
  at::Tensor D;
  if (beta != 0.0) {
    TORCH_CHECK(Cin.has_value(), "beta != 0 needs C");
    D = *Cin;
    TORCH_CHECK(D.scalar_type() == at::kHalf && D.dim() == 2 && D.size(0) == M && D.size(1) == N &&
                    D.device() == A.device(),
                "C must be a float16 (M x N) tensor on A's device");
    if (D.stride(1) != 1 && N > 1) D = D.contiguous();
  }
  at::Tensor bvec;
  if (bias.has_value()) {
    bvec = *bias;
    TORCH_CHECK(bvec.scalar_type() == at::kHalf && bvec.numel() == N && bvec.device() == A.device(),
                "bias must be a float16 tensor of N elements on A's device");
    bvec = bvec.reshape({N}).contiguous();
  }
  auto [As, ta, lda] = operand(A);
  auto [Bs, tb, ldb] = operand(B);
  at::Tensor C = output(out, M, N, A);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(A.device().index()).stream();
  const size_t need = gemm_workspace_bytes_ex(As.data_ptr(), Bs.data_ptr(), M, N, K, lda, ldb, ta, tb,
                                              static_cast<int>(cfg_id));
  size_t len = 0;
  void* ws = need ? workspace(A.device(), stream, need, &len) : nullptr;
  check_status(gemm_launch_ex(As.data_ptr(), Bs.data_ptr(), C.data_ptr(), M, N, K, lda, ldb,
                              std::max<int64_t>(C.stride(0), N), ta, tb, static_cast<float>(alpha),
                              static_cast<float>(beta), D.defined() ? D.data_ptr() : nullptr,
                              D.defined() ? std::max<int64_t>(D.stride(0), N) : 0,
                              bvec.defined() ? bvec.data_ptr() : nullptr, static_cast<int>(act),
                              static_cast<int>(cfg_id), ws, len, stream),
               "gemm_launch_ex");
  return C;
}

void reset_workspaces() {
  std::lock_guard<std::mutex> lock(g_ws_mu);
  g_ws->clear();
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "torch binding of the sm_100a FP16 GEMM kernel bank (C ABI in gemm_sm100.h)";
  m.def("gemm_forward_cfg", &gemm_forward_cfg, "C = A @ B with menu configuration cfg_id", py::arg("A"),
        py::arg("B"), py::arg("cfg_id"), py::arg("out") = py::none());
  m.def("gemm_ex", &gemm_ex, "out = act(alpha * A @ B + beta * C + bias)", py::arg("A"), py::arg("B"),
        py::arg("cfg_id"), py::arg("alpha") = 1.0, py::arg("beta") = 0.0, py::arg("C") = py::none(),
        py::arg("bias") = py::none(), py::arg("act") = 0, py::arg("out") = py::none());
  m.def("reset_workspaces", &reset_workspaces, "drop the cached split-K / repack workspaces");
}
