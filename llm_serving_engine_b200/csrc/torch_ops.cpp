// torch.library operators over the C ABI (liblse_int8.so): the calls the engine-facing
// modules make, as one dispatcher call each (host checks in C++, output and workspace from the
// caching allocator on the current stream, launch on that stream, no sync).
//
//   lse::int8_linear(Tensor x, Tensor w_packed, Tensor scale, int N, int K,
//                    Tensor? residual=None, int algo=0) -> Tensor
//       y[..., N] = x[..., K] @ (W * s)^T (+ residual), W in the packed layout
//       (lse_int8_linear_packed_dt); x bf16 or fp16, y of x's dtype
//   lse::gate_up_silu(Tensor x, Tensor w_packed, Tensor scale, int I, int K) -> Tensor
//       silu(x @ Wg^T * sg) * (x @ Wu^T * su), [..., I] (lse_int8_gate_up_silu_packed_dt)
//
// Errors come back as c10::Error (RuntimeError in Python) before any launch when an argument
// is wrong, and with the library's status text when a launch is refused.  CUDA tensors only:
// there is no CPU implementation.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <mutex>

#include "../../include/lse_int8.h"

namespace {

int dtype_code(const at::Tensor &x) {
    if (x.scalar_type() == at::kBFloat16) return LSE_BF16;
    if (x.scalar_type() == at::kHalf) return LSE_F16;
    TORCH_CHECK(false, "lse: x must be bfloat16 or float16, got ", x.scalar_type());
    return -1;
}

void init_device(int index) {
    static std::once_flag once[64];
    TORCH_CHECK(index >= 0 && index < 64, "lse: device index ", index, " out of range");
    std::call_once(once[index], [index] {
        const int rc = lse_init(index);
        TORCH_CHECK(rc == LSE_OK, "lse_init(cuda:", index, "): ", lse_status_string(rc), " ", lse_last_cuda_error());
    });
}

void check_common(const at::Tensor &x, const at::Tensor &w_packed, const at::Tensor &scale, int64_t rows, int64_t K,
                  const char *what) {
    TORCH_CHECK(x.is_cuda() && w_packed.is_cuda() && scale.is_cuda(), what, ": CUDA tensors only (no CPU fallback)");
    TORCH_CHECK(w_packed.device() == x.device() && scale.device() == x.device(), what, ": tensors on different devices");
    TORCH_CHECK(x.dim() >= 1 && x.size(-1) == K, what, ": x last dim ", x.size(-1), " != K ", K);
    TORCH_CHECK(K % 16 == 0, what, ": K must be a multiple of 16, got ", K);
    TORCH_CHECK(w_packed.scalar_type() == at::kChar && w_packed.is_contiguous() &&
                    w_packed.numel() == static_cast<int64_t>(lse_int8_packed_weight_bytes(rows, K)),
                what, ": w_packed must be the packed int8 buffer of [", rows, ", ", K, "]");
    TORCH_CHECK(scale.scalar_type() == at::kFloat && scale.dim() == 1 && scale.size(0) == rows && scale.is_contiguous(),
                what, ": scale must be float32 [", rows, "]");
}

// x as [M, K] with unit column stride, row stride a multiple of 8 and a 16-byte aligned start
at::Tensor rows_of(const at::Tensor &x, int64_t K) {
    at::Tensor x2 = x.reshape({-1, K});
    if (x2.stride(1) != 1 || x2.stride(0) % 8 != 0 || reinterpret_cast<uintptr_t>(x2.data_ptr()) % 16 != 0)
        x2 = x2.contiguous();
    return x2;
}

at::Tensor workspace(size_t bytes, const at::Tensor &like) {
    if (bytes == 0) return at::Tensor();
    return at::empty({static_cast<int64_t>(bytes)}, like.options().dtype(at::kByte));
}

at::Tensor int8_linear(const at::Tensor &x, const at::Tensor &w_packed, const at::Tensor &scale, int64_t N, int64_t K,
                       const c10::optional<at::Tensor> &residual, int64_t algo) {
    check_common(x, w_packed, scale, N, K, "lse::int8_linear");
    const int dt = dtype_code(x);
    c10::cuda::CUDAGuard guard(x.device());
    init_device(x.get_device());
    const at::Tensor x2 = rows_of(x, K);
    const int64_t M = x2.size(0);
    std::vector<int64_t> shape(x.sizes().begin(), x.sizes().end());
    shape.back() = N;
    at::Tensor y = at::empty(shape, x.options());
    if (M == 0 || N == 0) return y;
    const void *res = nullptr;
    int64_t ldr = 0;
    at::Tensor r2;
    if (residual.has_value() && residual->defined()) {
        const at::Tensor &r = *residual;
        TORCH_CHECK(r.is_cuda() && r.device() == x.device() && r.scalar_type() == x.scalar_type() &&
                        r.sizes() == y.sizes() && r.stride(-1) == 1,
                    "lse::int8_linear: residual must match the output's shape and dtype with a contiguous last dim");
        r2 = r.reshape({-1, N});
        res = r2.data_ptr();
        ldr = r2.stride(0);
    }
    const size_t ws_bytes = lse_int8_linear_workspace_for(M, K, N, static_cast<int>(algo), 1);
    const at::Tensor ws = workspace(ws_bytes, x);
    const cudaStream_t st = at::cuda::getCurrentCUDAStream(x.get_device()).stream();
    const int rc = lse_int8_linear_packed_dt(x2.data_ptr(), dt, M, K, x2.stride(0),
                                             static_cast<const int8_t *>(w_packed.data_ptr()),
                                             scale.data_ptr<float>(), N, res, ldr, y.data_ptr(), N,
                                             ws.defined() ? ws.data_ptr() : nullptr, ws_bytes, static_cast<int>(algo), st);
    TORCH_CHECK(rc == LSE_OK, "lse_int8_linear_packed_dt: ", lse_status_string(rc), " ", lse_last_cuda_error());
    return y;
}

at::Tensor gate_up_silu(const at::Tensor &x, const at::Tensor &w_packed, const at::Tensor &scale, int64_t I, int64_t K) {
    check_common(x, w_packed, scale, 2 * I, K, "lse::gate_up_silu");
    TORCH_CHECK(I % 8 == 0, "lse::gate_up_silu: the intermediate size must be a multiple of 8, got ", I);
    const int dt = dtype_code(x);
    c10::cuda::CUDAGuard guard(x.device());
    init_device(x.get_device());
    const at::Tensor x2 = rows_of(x, K);
    const int64_t M = x2.size(0);
    std::vector<int64_t> shape(x.sizes().begin(), x.sizes().end());
    shape.back() = I;
    at::Tensor y = at::empty(shape, x.options());
    if (M == 0 || I == 0) return y;
    const size_t ws_bytes = M <= 16 ? 0 : lse_int8_linear_workspace_for(M, K, 2 * I, LSE_ALGO_TCGEN05, 1);
    const at::Tensor ws = workspace(ws_bytes, x);
    const cudaStream_t st = at::cuda::getCurrentCUDAStream(x.get_device()).stream();
    const int rc = lse_int8_gate_up_silu_packed_dt(x2.data_ptr(), dt, M, K, x2.stride(0),
                                                   static_cast<const int8_t *>(w_packed.data_ptr()),
                                                   scale.data_ptr<float>(), I, y.data_ptr(), I,
                                                   ws.defined() ? ws.data_ptr() : nullptr, ws_bytes, st);
    TORCH_CHECK(rc == LSE_OK, "lse_int8_gate_up_silu_packed_dt: ", lse_status_string(rc), " ", lse_last_cuda_error());
    return y;
}

}  // namespace

TORCH_LIBRARY(lse, m) {
    m.def("int8_linear(Tensor x, Tensor w_packed, Tensor scale, int N, int K, Tensor? residual=None, int algo=0) -> Tensor");
    m.def("gate_up_silu(Tensor x, Tensor w_packed, Tensor scale, int I, int K) -> Tensor");
}

TORCH_LIBRARY_IMPL(lse, CUDA, m) {
    m.impl("int8_linear", &int8_linear);
    m.impl("gate_up_silu", &gate_up_silu);
}
