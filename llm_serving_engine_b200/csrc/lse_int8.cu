// C-ABI entry points of liblse_int8.so (declared in include/lse_int8.h).
//
// Host-side responsibilities: argument/alignment validation before any launch (errors come
// back as lse_status codes, nothing aborts), per-device one-time set-up, TMA tensor-map
// encoding (driver entry point fetched through the runtime, so the library has no link-time
// libcuda dependency and loads on machines without a driver), and kernel selection by M.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/lse_int8.h"
#include "gemv_i8.cuh"
#include "quantize.cuh"
#include "tc_gemm_i8.cuh"

namespace lse {

namespace {

constexpr int kMaxDevices = 64;
// Largest grid the tensor-core kernel launches (one CTA per SM); sizes the partial-tile
// region of the workspace.  B200 has 148 SMs.
constexpr int kMaxGridForWorkspace = 160;

thread_local char t_last_error[256] = "";

void set_cuda_error(cudaError_t e, const char *where) {
    std::snprintf(t_last_error, sizeof(t_last_error), "%s: %s (%s)", where, cudaGetErrorName(e),
                  cudaGetErrorString(e));
}

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct DeviceState {
    std::once_flag once;
    int status = LSE_ERR_CUDA;
    int num_sms = 0;
};
DeviceState g_dev[kMaxDevices];
std::once_flag g_encode_once;
EncodeTiledFn g_encode = nullptr;

template <int NT>
cudaError_t set_tc_attrs() {
    return cudaFuncSetAttribute(tc::tc_gemm_i8_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                tc::Cfg<NT>::SMEM_BYTES);
}

int init_device(int device) {
    if (device < 0 || device >= kMaxDevices) return LSE_ERR_INVALID_ARG;
    DeviceState &d = g_dev[device];
    std::call_once(d.once, [&] {
        int prev = -1;
        cudaError_t e = cudaGetDevice(&prev);
        if (e != cudaSuccess) { set_cuda_error(e, "cudaGetDevice"); return; }
        if (prev != device && (e = cudaSetDevice(device)) != cudaSuccess) { set_cuda_error(e, "cudaSetDevice"); return; }
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
        if (e == cudaSuccess) e = set_tc_attrs<16>();
        if (e == cudaSuccess) e = set_tc_attrs<32>();
        if (e == cudaSuccess) e = set_tc_attrs<64>();
        if (e == cudaSuccess) e = set_tc_attrs<128>();
        if (e != cudaSuccess) set_cuda_error(e, "device set-up");
        std::call_once(g_encode_once, [] {
            void *fn = nullptr;
            cudaDriverEntryPointQueryResult q;
            if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
                q == cudaDriverEntryPointSuccess)
                g_encode = reinterpret_cast<EncodeTiledFn>(fn);
        });
        if (prev != device) cudaSetDevice(prev);
        if (e == cudaSuccess && g_encode == nullptr) {
            std::snprintf(t_last_error, sizeof(t_last_error), "cuTensorMapEncodeTiled unavailable");
            return;
        }
        if (e == cudaSuccess) {
            d.num_sms = sms;
            d.status = LSE_OK;
        }
    });
    return d.status;
}

int current_device(int *dev) {
    cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) { set_cuda_error(e, "cudaGetDevice"); return LSE_ERR_CUDA; }
    return init_device(*dev);
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int token_tile(int64_t M) {
    if (M <= 16) return 16;
    if (M <= 32) return 32;
    if (M <= 64) return 64;
    return 128;
}

// Tensor-core kernel schedule: full waves data-parallel, the last one-to-two waves stream-K.
struct TcPlan {
    int nt, m_tiles, n_tiles, tiles, kb, dp_tiles, grid;
    long long sk_units;
};

TcPlan plan_tc(int64_t M, int64_t K, int64_t N, int num_sms) {
    TcPlan t{};
    t.nt = token_tile(M);
    t.m_tiles = static_cast<int>((M + t.nt - 1) / t.nt);
    t.n_tiles = static_cast<int>((N + tc::BN - 1) / tc::BN);
    t.tiles = t.m_tiles * t.n_tiles;
    t.kb = static_cast<int>((K + tc::BK - 1) / tc::BK);
    int G = num_sms;
    if (t.tiles % G == 0) t.dp_tiles = t.tiles;
    else if (t.tiles < G) t.dp_tiles = 0;
    else t.dp_tiles = (t.tiles / G - 1) * G;
    t.sk_units = static_cast<long long>(t.tiles - t.dp_tiles) * t.kb;
    if (t.dp_tiles == 0) G = static_cast<int>(std::min<long long>(G, t.sk_units));
    t.grid = G;
    return t;
}

size_t tc_workspace_bytes(int nt, int grid) {
    return LSE_WS_COUNTER_BYTES + static_cast<size_t>(2) * grid * nt * tc::BN * sizeof(float);
}

int encode_2d(CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t inner, uint64_t outer,
              uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer) {
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(m, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        std::snprintf(t_last_error, sizeof(t_last_error), "cuTensorMapEncodeTiled failed (%d)", (int)r);
        return LSE_ERR_CUDA;
    }
    return LSE_OK;
}

template <int NT>
int launch_tc(const TcPlan &pl, const void *x, int64_t M, int64_t K, int64_t ldx, const int8_t *w,
              const float *scale, int64_t N, void *y, int64_t ldy, void *ws, cudaStream_t st) {
    CUtensorMap tw, tx;
    int rc = encode_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, K, N, K, tc::BK, tc::BN);
    if (rc) return rc;
    rc = encode_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, K, M, ldx * 2, 64, NT);
    if (rc) return rc;
    tc::Params p{};
    p.M = static_cast<int>(M);
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(K);
    p.y = static_cast<__nv_bfloat16 *>(y);
    p.ldy = ldy;
    p.scale = scale;
    p.counters = static_cast<int *>(ws);
    p.partials = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + LSE_WS_COUNTER_BYTES);
    p.m_tiles = pl.m_tiles;
    p.tiles = pl.tiles;
    p.kb = pl.kb;
    p.dp_tiles = pl.dp_tiles;
    p.grid = pl.grid;
    p.sk_units = pl.sk_units;
    tc::tc_gemm_i8_kernel<NT><<<pl.grid, tc::NUM_THREADS, tc::Cfg<NT>::SMEM_BYTES, st>>>(tw, tx, p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { set_cuda_error(e, "tc_gemm_i8 launch"); return LSE_ERR_CUDA; }
    return LSE_OK;
}

template <int MT, int ROWS>
void launch_gemv(const void *x, int64_t M, int64_t K, int64_t ldx, const int8_t *w, const float *scale,
                 int64_t N, void *y, int64_t ldy, cudaStream_t st) {
    dim3 grid(static_cast<unsigned>((N + ROWS - 1) / ROWS), static_cast<unsigned>((M + MT - 1) / MT));
    gemv_i8_kernel<MT, ROWS><<<grid, kGemvThreads, 0, st>>>(static_cast<const __nv_bfloat16 *>(x), ldx,
                                                           static_cast<int>(M), static_cast<int>(K), w, scale,
                                                           static_cast<int>(N),
                                                           static_cast<__nv_bfloat16 *>(y), ldy);
}

int run_gemv(const void *x, int64_t M, int64_t K, int64_t ldx, const int8_t *w, const float *scale, int64_t N,
             void *y, int64_t ldy, cudaStream_t st) {
    switch (M) {
        case 1: launch_gemv<1, 4>(x, M, K, ldx, w, scale, N, y, ldy, st); break;
        case 2: launch_gemv<2, 4>(x, M, K, ldx, w, scale, N, y, ldy, st); break;
        case 3: launch_gemv<3, 4>(x, M, K, ldx, w, scale, N, y, ldy, st); break;
        default: launch_gemv<4, 4>(x, M, K, ldx, w, scale, N, y, ldy, st); break;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { set_cuda_error(e, "gemv_i8 launch"); return LSE_ERR_CUDA; }
    return LSE_OK;
}

// Auto policy: the CUDA-core GEMV while its FMA work stays under the HBM stream
// (M <= 2), the tensor-core kernel from there on.
int auto_algo(int64_t M) { return M <= 2 ? LSE_ALGO_GEMV : LSE_ALGO_TCGEN05; }

}  // namespace
}  // namespace lse

using namespace lse;

extern "C" {

int lse_abi_version(void) { return LSE_ABI_VERSION; }

const char *lse_status_string(int status) {
    switch (status) {
        case LSE_OK: return "ok";
        case LSE_ERR_INVALID_ARG: return "invalid argument";
        case LSE_ERR_ALIGNMENT: return "unsupported alignment (need K%16==0, ldx%8==0, 16-byte aligned x/w)";
        case LSE_ERR_UNSUPPORTED: return "unsupported shape or algorithm";
        case LSE_ERR_WORKSPACE: return "workspace missing or too small";
        case LSE_ERR_CUDA: return "CUDA error";
        case LSE_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
        default: return "unknown status";
    }
}

const char *lse_last_cuda_error(void) { return t_last_error; }

int lse_init(int device) { return init_device(device); }

size_t lse_int8_linear_workspace(int64_t M, int64_t K, int64_t N) {
    (void)K;
    (void)N;
    if (M <= 0) return LSE_WS_COUNTER_BYTES;
    return tc_workspace_bytes(token_tile(M), kMaxGridForWorkspace);
}

int lse_int8_linear_ex(const void *x, int64_t M, int64_t K, int64_t ldx, const int8_t *w, const float *scale,
                       int64_t N, void *y, int64_t ldy, void *workspace, size_t workspace_bytes, int algo,
                       void *stream) {
    if (M < 0 || N < 0 || K < 0) return LSE_ERR_INVALID_ARG;
    if (M == 0 || N == 0) return LSE_OK;
    if (!x || !w || !scale || !y) return LSE_ERR_INVALID_ARG;
    if (ldx < K || ldy < N) return LSE_ERR_INVALID_ARG;
    if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return LSE_ERR_UNSUPPORTED;
    if ((K & 15) || (ldx & 7) || !aligned16(x) || !aligned16(w)) return LSE_ERR_ALIGNMENT;
    if ((reinterpret_cast<uintptr_t>(y) & 1u) || (reinterpret_cast<uintptr_t>(scale) & 3u)) return LSE_ERR_ALIGNMENT;
    if (algo < LSE_ALGO_AUTO || algo > LSE_ALGO_TCGEN05) return LSE_ERR_INVALID_ARG;
    int dev = 0;
    int rc = current_device(&dev);
    if (rc) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (K == 0) {
        cudaError_t e = cudaMemset2DAsync(y, static_cast<size_t>(ldy) * 2, 0, static_cast<size_t>(N) * 2,
                                          static_cast<size_t>(M), st);
        if (e != cudaSuccess) { set_cuda_error(e, "cudaMemset2DAsync"); return LSE_ERR_CUDA; }
        return LSE_OK;
    }
    if (algo == LSE_ALGO_AUTO) algo = auto_algo(M);
    if (algo == LSE_ALGO_GEMV) return run_gemv(x, M, K, ldx, w, scale, N, y, ldy, st);

    const TcPlan pl = plan_tc(M, K, N, g_dev[dev].num_sms);
    if (!workspace || !aligned16(workspace) || workspace_bytes < tc_workspace_bytes(pl.nt, pl.grid))
        return LSE_ERR_WORKSPACE;
    switch (pl.nt) {
        case 16: return launch_tc<16>(pl, x, M, K, ldx, w, scale, N, y, ldy, workspace, st);
        case 32: return launch_tc<32>(pl, x, M, K, ldx, w, scale, N, y, ldy, workspace, st);
        case 64: return launch_tc<64>(pl, x, M, K, ldx, w, scale, N, y, ldy, workspace, st);
        default: return launch_tc<128>(pl, x, M, K, ldx, w, scale, N, y, ldy, workspace, st);
    }
}

int lse_int8_linear(const void *x, int64_t M, int64_t K, int64_t ldx, const int8_t *w, const float *scale,
                    int64_t N, void *y, int64_t ldy, void *workspace, size_t workspace_bytes, void *stream) {
    return lse_int8_linear_ex(x, M, K, ldx, w, scale, N, y, ldy, workspace, workspace_bytes, LSE_ALGO_AUTO,
                              stream);
}

int lse_int8_quantize(const void *w, int dtype, int64_t N, int64_t K, int64_t ldw, int8_t *q_out, float *s_out,
                      void *stream) {
    if (N < 0 || K < 0 || ldw < K) return LSE_ERR_INVALID_ARG;
    if (N == 0) return LSE_OK;
    if (!w || !q_out || !s_out) return LSE_ERR_INVALID_ARG;
    if (N > INT32_MAX) return LSE_ERR_UNSUPPORTED;
    int dev = 0;
    int rc = current_device(&dev);
    if (rc) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const unsigned grid = static_cast<unsigned>(N);
    switch (dtype) {
        case LSE_BF16:
            quantize_rows_kernel<__nv_bfloat16><<<grid, kQuantThreads, 0, st>>>(
                static_cast<const __nv_bfloat16 *>(w), ldw, K, q_out, s_out);
            break;
        case LSE_F16:
            quantize_rows_kernel<__half><<<grid, kQuantThreads, 0, st>>>(static_cast<const __half *>(w), ldw, K,
                                                                         q_out, s_out);
            break;
        case LSE_F32:
            quantize_rows_kernel<float><<<grid, kQuantThreads, 0, st>>>(static_cast<const float *>(w), ldw, K,
                                                                        q_out, s_out);
            break;
        default: return LSE_ERR_INVALID_ARG;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { set_cuda_error(e, "quantize launch"); return LSE_ERR_CUDA; }
    return LSE_OK;
}

int lse_device_status(int device, int reset) {
    int prev = -1;
    cudaError_t e = cudaGetDevice(&prev);
    if (e != cudaSuccess) { set_cuda_error(e, "cudaGetDevice"); return LSE_ERR_CUDA; }
    if (prev != device && (e = cudaSetDevice(device)) != cudaSuccess) {
        set_cuda_error(e, "cudaSetDevice");
        return LSE_ERR_CUDA;
    }
    int status = LSE_OK;
    e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&status, g_device_status, sizeof(int));
    if (e == cudaSuccess && reset) {
        const int zero = LSE_OK;
        e = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int));
    }
    if (prev != device) cudaSetDevice(prev);
    if (e != cudaSuccess) { set_cuda_error(e, "lse_device_status"); return LSE_ERR_CUDA; }
    return status;
}

}  // extern "C"
