// C-ABI entry points of liblse_int8.so (declared in include/lse_int8.h).
//
// Host-side responsibilities: argument/alignment validation before any launch (errors come
// back as lse_status codes, nothing aborts), per-device one-time set-up, TMA tensor-map
// encoding (driver entry point fetched through the runtime, so the library has no link-time
// libcuda dependency and loads on machines without a driver), and kernel selection by M.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "../../include/lse_int8.h"
#include "decode_attn.cuh"
#include "paged_attn.cuh"
#include "rope_kv.cuh"
#include "rms_norm.cuh"
#include "gemv_i8.cuh"
#include "pack_w.cuh"
#include "quantize.cuh"
#include "skinny_mma.cuh"
#include "act_split.cuh"
#include "tc_i8.cuh"

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

template <int NT, int S, bool SILU, bool WPACK, bool CLUSTER>
cudaError_t set_tci8_attrs() {
    return cudaFuncSetAttribute(tci8::tc_i8_kernel<NT, S, SILU, WPACK, CLUSTER>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, tci8::Cfg<NT, S>::SMEM_BYTES);
}

template <bool SILU, bool WPACK>
cudaError_t set_tci8_attrs_all() {
    cudaError_t e = set_tci8_attrs<64, 3, SILU, WPACK, false>();
    if (e == cudaSuccess) e = set_tci8_attrs<128, 2, SILU, WPACK, false>();
    if (e == cudaSuccess) e = set_tci8_attrs<64, 3, SILU, WPACK, true>();
    if (e == cudaSuccess) e = set_tci8_attrs<128, 2, SILU, WPACK, true>();
#ifdef LSE_TUNING
    if (e == cudaSuccess) e = set_tci8_attrs<64, 2, SILU, WPACK, false>();
    if (e == cudaSuccess) e = set_tci8_attrs<64, 2, SILU, WPACK, true>();
#endif
    return e;
}

// How many thread-block clusters of c CTAs of a token-tile configuration can be resident at
// once on the current device (the cluster plan needs all of its clusters resident in one
// wave; how many fit depends on how the SMs are grouped, not only on their number).
constexpr int kMaxCluster = 8;  // portable cluster size
int g_max_clusters[kMaxDevices][2][kMaxCluster + 1];

template <int NT, int S>
int query_max_clusters(int c) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c * 16);
    cfg.blockDim = dim3(tci8::NUM_THREADS);
    cfg.dynamicSmemBytes = tci8::Cfg<NT, S>::SMEM_BYTES;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = c;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, tci8::tc_i8_kernel<NT, S, false, true, true>, &cfg) != cudaSuccess) {
        (void)cudaGetLastError();  // not fatal: the plan then splits through global memory
        return 0;
    }
    return n;
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
        if (e == cudaSuccess) e = set_tci8_attrs_all<false, false>();
        if (e == cudaSuccess) e = set_tci8_attrs_all<false, true>();
        if (e == cudaSuccess) e = set_tci8_attrs_all<true, true>();
        if (e == cudaSuccess)
            for (int c = 2; c <= kMaxCluster; ++c) {
                g_max_clusters[device][0][c] = query_max_clusters<64, 3>(c);
                g_max_clusters[device][1][c] = query_max_clusters<128, 2>(c);
            }
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

// Tuning knobs.  The shipped library uses the constant given at each call site; a build with
// -DLSE_TUNING (parameter sweeps only, never the shipped library) lets an environment
// variable of the same name override it.
int tuning_knob(const char *name, int value) {
#ifdef LSE_TUNING
    const char *e = std::getenv(name);
    if (e) value = std::atoi(e);
#else
    (void)name;
#endif
    return value;
}

// Programmatic dependent launch: both kernels start their weight streams before waiting on
// the previous kernel in the stream (griddepcontrol.wait), which hides launch latency and
// pipeline fill between back-to-back projections.
bool pdl_enabled() {
    static const bool on = tuning_knob("LSE_DISABLE_PDL", 0) != 1;
    return on;
}

// How many 16 KB weight tiles the kernel's prefetch warp keeps in flight to L2 ahead of the
// data that has landed in shared memory (0 disables).
int prefetch_stages() {
    static const int v = tuning_knob("LSE_PF_STAGES", 12);
    return v;
}

void launch_config(cudaLaunchConfig_t &cfg, cudaLaunchAttribute (&attr)[1], dim3 grid, dim3 block, size_t smem,
                   cudaStream_t st) {
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Token tile of the tensor-core kernel: 64 up to 64 tokens, 128 above.  A tcgen05.mma costs
// the same issue time at N = 16, 32 or 64, so smaller tiles only add instructions per weight
// byte (measured on B200: gate_up at M <= 32 runs 35 us with 64-token tiles, 52 us with
// 16/32-token tiles).
int token_tile(int64_t M) { return M <= 64 ? 64 : 128; }

// -1: the plan's rule below; 0 / 1 force the even spread / the aligned grid (sweeps only).
int tc_split_align() {
    static const int v = tuning_knob("LSE_TC_SPLIT_ALIGN", -1);
    return v;
}

// Tensor-core kernel schedule: full waves data-parallel, the last one-to-two waves stream-K.
struct TcPlan {
    int nt, m_tiles, n_tiles, tiles, kb, dp_tiles, grid;
    long long sk_units;
    int cluster;  // >= 2: every tile split over the CTAs of one thread-block cluster
};

TcPlan plan_tc(int64_t M, int64_t K, int64_t N, int num_sms, int dev) {
    TcPlan t{};
    t.nt = token_tile(M);
    t.m_tiles = static_cast<int>((M + t.nt - 1) / t.nt);
    t.n_tiles = static_cast<int>((N + tci8::BN - 1) / tci8::BN);
    t.tiles = t.m_tiles * t.n_tiles;
    t.kb = static_cast<int>((K + tci8::BK - 1) / tci8::BK);
    int G = num_sms;
    // Few tiles (decode): split every tile's K range evenly over the c CTAs of one cluster,
    // reduced through distributed shared memory, with c as large as the SMs allow while all
    // tiles x c CTAs stay resident together (and every CTA gets at least one 128-K stage).
    // Measured on B200 at M = 64 (globaltimer trace of the global-memory split): the weight
    // stream ran at the HBM rate, and the partial publication plus the last arriver's sum
    // added 6-9 us after the last MMA.
    if (t.tiles <= G / 2 && dev >= 0) {
        static const int cmax = tuning_knob("LSE_TC_CMAX", kMaxCluster);
        int c = std::min(std::min(G / t.tiles, cmax), t.kb);
        while (c >= 2 && g_max_clusters[dev][t.nt == 128 ? 1 : 0][c] < t.tiles) --c;
        if (c >= 2) {
            t.cluster = c;
            t.dp_tiles = 0;
            t.grid = t.tiles * c;
            t.sk_units = static_cast<long long>(t.tiles) * t.kb;
            return t;
        }
    }
    // Prefill-sized tiles (tensor-bound), more than half a wave but less than a whole one: every
    // tile whole on its own CTA, the remaining SMs idle.  Measured on B200 (Llama-3-8B shapes at
    // M = 512, 128 tiles): O 33.3 -> 27.0 us and down 72.9 -> 56.3 us against stream-K over all
    // SMs, whose every tile then has two segments and a partial-sum reduction.
    // Decode-sized tiles (64 tokens) over more than one wave whose last wave is at least half
    // full: whole tiles too, dealt round-robin (the first tiles % G CTAs take one more).
    // Measured on B200 (us per launch, 32 or 16 weights per CUDA graph, stream-K -> whole):
    // Llama-3-8B gate_up (224 tiles) at M = 64 35.2 -> 31.6, with SiLU * mul 38.7 -> 33.5, at
    // M = 48 33.6 -> 31.1, at M = 33 32.2 -> 30.6; the Llama-3 lm_head shape (N = 128256, 1002
    // tiles) at M = 64 118.8 -> 114.3.  With a nearly empty last wave stream-K stays ahead
    // (Llama-3-70B gate_up, 448 tiles: 105.1 against 110.3 at M = 64), and so does a single
    // partial wave (70B QKV, 80 tiles: 26.1 against 27.4 at M = 32).
    const bool dp_decode = t.nt == 64 && t.tiles > G && 2 * (t.tiles % G) >= G;
    if (dp_decode || t.tiles % G == 0 || (t.nt == 128 && t.tiles > G / 2 && t.tiles < G)) t.dp_tiles = t.tiles;
    else if (t.tiles < G) t.dp_tiles = 0;
    else {
        static const int sk_waves = tuning_knob("LSE_TC_SK_WAVES", 2);  // waves left to stream-K: 1 or 2
        t.dp_tiles = (t.tiles / G - (sk_waves >= 2 ? 1 : 0)) * G;
    }
    // At most half a wave of tiles (decode shapes): split every tile's K range over the same
    // number s of CTAs (grid tiles * s, s = num_sms / tiles), so that each CTA works on one
    // tile and each tile's last arriver sums s partials.  Spreading the units evenly over all
    // SMs instead lets segments straddle tiles: some CTAs then publish two partials and sum
    // two tiles, one after the other, and they set the launch's tail (a globaltimer trace of
    // O at M = 64: 7.8 us from the last MMA issue to the last reduction, 6.4 us aligned).  The
    // aligned grid leaves SMs idle, so it is taken only while it costs at most two more
    // 128-K stages per CTA.  Measured (24 launches per CUDA graph, even -> aligned): Llama-3-8B
    // at M = 64 O 15.45 -> 13.77 us (8 stages per CTA instead of 7), QKV 16.62 -> 15.62 (11
    // either way), down 24.90 -> 24.83 (28 instead of 25); at M = 32 O 14.03 -> 12.68, QKV
    // 15.30 -> 14.61, down 23.51 -> 23.76; Llama-3-70B at M = 32 O 24.69 -> 25.97 (32 instead
    // of 28), down 61.36 -> 68.55 (112 instead of 97).
    if (t.tiles <= G / 2) {
        const int s = G / t.tiles;
        const long long even = (static_cast<long long>(t.tiles) * t.kb + G - 1) / G;
        const long long aligned = (t.kb + s - 1) / s;
        const int force = tc_split_align();
        if (force == 1 || (force < 0 && aligned <= even + 2)) G = t.tiles * s;
    }
    t.sk_units = static_cast<long long>(t.tiles - t.dp_tiles) * t.kb;
    if (t.dp_tiles == 0) G = static_cast<int>(std::min<long long>(G, t.sk_units));
    if (t.sk_units == 0) G = std::min(G, t.dp_tiles);  // whole tiles only: no idle CTAs
    t.grid = G;
    return t;
}


int encode_2d(CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t inner, uint64_t outer,
              uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
              CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(m, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        std::snprintf(t_last_error, sizeof(t_last_error), "cuTensorMapEncodeTiled failed (%d)", (int)r);
        return LSE_ERR_CUDA;
    }
    return LSE_OK;
}

int encode_3d(CUtensorMap *m, const void *base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1_bytes,
              uint64_t s2_bytes, uint32_t b0, uint32_t b1, uint32_t b2) {
    cuuint64_t dims[3] = {d0, d1, d2};
    cuuint64_t strides[2] = {s1_bytes, s2_bytes};
    cuuint32_t box[3] = {b0, b1, b2};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        std::snprintf(t_last_error, sizeof(t_last_error), "cuTensorMapEncodeTiled (3-D) failed (%d)", (int)r);
        return LSE_ERR_CUDA;
    }
    return LSE_OK;
}

// Digit planes of the int8 tensor-core path: 3 (24-bit activations) up to 64 tokens, where the
// MMA's N = 3 x 64 costs nothing against the weight stream, 2 (16-bit) above.
int digit_planes(int64_t M) {
    static const int s64 = tuning_knob("LSE_TC_S64", 3);
    return M <= 64 ? s64 : 2;
}

size_t tci8_partial_bytes(int nt, int grid) { return static_cast<size_t>(2) * grid * nt * tci8::BN * sizeof(float); }

// Workspace of one tensor-core call: stream-K counters, partial tiles, S digit planes of
// M x Kp bytes and M row scales.
size_t tci8_workspace_bytes(int nt, int S, int grid, int64_t M, int64_t K) {
    const size_t planes = static_cast<size_t>(S) * M * packed_cols(K);
    return LSE_WS_COUNTER_BYTES + tci8_partial_bytes(nt, grid) + planes + (static_cast<size_t>(M) * 4 + 15) / 16 * 16;
}

template <int NT, int S, bool SILU>
int launch_tc_i8(const TcPlan &pl, const void *x, int64_t M, int64_t K, int64_t ldx, const int8_t *w,
                 const float *scale, int64_t N, void *y, int64_t ldy, const void *res, int64_t ldr, void *ws,
                 bool packed, cudaStream_t st, bool xf16, const void *norm_w, float eps) {
    const int64_t Kp = packed_cols(K);
    uint8_t *wsb = static_cast<uint8_t *>(ws);
    int *counters = reinterpret_cast<int *>(wsb);
    float *partials = reinterpret_cast<float *>(wsb + LSE_WS_COUNTER_BYTES);
    int8_t *planes = reinterpret_cast<int8_t *>(wsb + LSE_WS_COUNTER_BYTES + tci8_partial_bytes(NT, pl.grid));
    const int64_t plane_stride = M * Kp;
    float *rscale = reinterpret_cast<float *>(planes + S * plane_stride);
    // 1) activations -> digit planes + row scales (also clears this launch's stream-K counters);
    //    with norm_w, of the RMSNorm of the activations (bf16)
    {
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        launch_config(cfg, attr, dim3(static_cast<unsigned>(M)), dim3(split::THREADS), 0, st);
        const int n_counters = pl.cluster >= 2 ? 0 : static_cast<int>(pl.tiles - pl.dp_tiles);
        cudaError_t e = norm_w ? cudaLaunchKernelEx(&cfg, split::rms_norm_split_kernel<S>,
                                                    static_cast<const __nv_bfloat16 *>(x), ldx,
                                                    static_cast<const __nv_bfloat16 *>(norm_w), eps, static_cast<int>(K),
                                                    static_cast<int>(Kp), planes, plane_stride, rscale, counters,
                                                    n_counters)
                      : xf16 ? cudaLaunchKernelEx(&cfg, split::act_split_kernel<S, __half>, static_cast<const __half *>(x),
                                                  ldx, static_cast<int>(K), static_cast<int>(Kp), planes, plane_stride,
                                                  rscale, counters, n_counters)
                             : cudaLaunchKernelEx(&cfg, split::act_split_kernel<S, __nv_bfloat16>,
                                                  static_cast<const __nv_bfloat16 *>(x), ldx, static_cast<int>(K),
                                                  static_cast<int>(Kp), planes, plane_stride, rscale, counters,
                                                  n_counters);
        if (e == cudaSuccess) e = cudaGetLastError();
        if (e != cudaSuccess) { set_cuda_error(e, "act_split launch"); return LSE_ERR_CUDA; }
    }
    // 2) the projection
    CUtensorMap tw, tx;
    int rc = packed ? encode_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT64, w, static_cast<uint64_t>(2 * Kp),
                                static_cast<uint64_t>(packed_rows(N) / 16), static_cast<uint64_t>(16 * Kp), 256, 8,
                                CU_TENSOR_MAP_SWIZZLE_NONE)
                    : encode_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, K, N, K, tci8::BK, tci8::BN);
    if (rc) return rc;
    rc = encode_3d(&tx, planes, static_cast<uint64_t>(Kp), static_cast<uint64_t>(M), S, static_cast<uint64_t>(Kp),
                   static_cast<uint64_t>(plane_stride), tci8::BK, NT, S);
    if (rc) return rc;
    tci8::Params p{};
    p.M = static_cast<int>(M);
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(K);
    p.y = static_cast<uint16_t *>(y);
    p.y_f16 = xf16 ? 1 : 0;
    p.ldy = ldy;
    p.res = static_cast<const uint16_t *>(res);
    p.ldr = ldr;
    p.scale = scale;
    p.row_scale = rscale;
    p.counters = counters;
    p.partials = partials;
    p.m_tiles = pl.m_tiles;
    p.tiles = pl.tiles;
    p.kb = pl.kb;
    p.dp_tiles = pl.dp_tiles;
    p.grid = pl.grid;
    p.sk_units = pl.sk_units;
    p.cluster = pl.cluster;
    p.w = w;
    p.kp = Kp;
    p.pf_stages = prefetch_stages();
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    cudaLaunchAttribute attr1[1];
    launch_config(cfg, attr1, dim3(pl.grid), dim3(tci8::NUM_THREADS), tci8::Cfg<NT, S>::SMEM_BYTES, st);
    attr[0] = attr1[0];
    cfg.attrs = attr;
    cudaError_t e;
    if (pl.cluster >= 2) {
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = static_cast<unsigned>(pl.cluster);
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        cfg.numAttrs = 2;
        e = packed ? cudaLaunchKernelEx(&cfg, tci8::tc_i8_kernel<NT, S, SILU, true, true>, tw, tx, p)
                   : cudaLaunchKernelEx(&cfg, tci8::tc_i8_kernel<NT, S, SILU, false, true>, tw, tx, p);
    } else {
        cfg.numAttrs = 1;
        e = packed ? cudaLaunchKernelEx(&cfg, tci8::tc_i8_kernel<NT, S, SILU, true, false>, tw, tx, p)
                   : cudaLaunchKernelEx(&cfg, tci8::tc_i8_kernel<NT, S, SILU, false, false>, tw, tx, p);
    }
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) { set_cuda_error(e, "tc_i8 launch"); return LSE_ERR_CUDA; }
    return LSE_OK;
}

// The token tile and digit planes go together: 64-token tiles with 3 planes (M <= 64),
// 128-token tiles with 2 planes above.
template <bool SILU>
int run_tc_i8(const TcPlan &pl, const void *x, int64_t M, int64_t K, int64_t ldx, const int8_t *w,
              const float *scale, int64_t N, void *y, int64_t ldy, const void *res, int64_t ldr, void *ws, bool packed,
              cudaStream_t st, bool xf16 = false, const void *norm_w = nullptr, float eps = 0.f) {
#ifdef LSE_TUNING
    if (pl.nt == 64 && digit_planes(M) == 2)
        return launch_tc_i8<64, 2, SILU>(pl, x, M, K, ldx, w, scale, N, y, ldy, res, ldr, ws, packed, st, xf16, norm_w, eps);
#endif
    if (pl.nt == 64)
        return launch_tc_i8<64, 3, SILU>(pl, x, M, K, ldx, w, scale, N, y, ldy, res, ldr, ws, packed, st, xf16, norm_w, eps);
    return launch_tc_i8<128, 2, SILU>(pl, x, M, K, ldx, w, scale, N, y, ldy, res, ldr, ws, packed, st, xf16, norm_w, eps);
}

template <int MT, int ROWS>
cudaError_t launch_gemv(const void *x, int64_t M, int64_t K, int64_t ldx, const int8_t *w, const float *scale,
                 int64_t N, void *y, int64_t ldy, cudaStream_t st) {
    dim3 grid(static_cast<unsigned>((N + ROWS - 1) / ROWS), static_cast<unsigned>((M + MT - 1) / MT));
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    launch_config(cfg, attr, grid, dim3(kGemvThreads), 0, st);
    return cudaLaunchKernelEx(&cfg, gemv_i8_kernel<MT, ROWS>, static_cast<const __nv_bfloat16 *>(x), ldx,
                              static_cast<int>(M), static_cast<int>(K), w, scale, static_cast<int>(N),
                              static_cast<__nv_bfloat16 *>(y), ldy);
}

int run_gemv(const void *x, int64_t M, int64_t K, int64_t ldx, const int8_t *w, const float *scale, int64_t N,
             void *y, int64_t ldy, cudaStream_t st) {
    cudaError_t e;
    switch (M) {
        case 1: e = launch_gemv<1, 4>(x, M, K, ldx, w, scale, N, y, ldy, st); break;
        case 2: e = launch_gemv<2, 4>(x, M, K, ldx, w, scale, N, y, ldy, st); break;
        case 3: e = launch_gemv<3, 4>(x, M, K, ldx, w, scale, N, y, ldy, st); break;
        default: e = launch_gemv<4, 4>(x, M, K, ldx, w, scale, N, y, ldy, st); break;
    }
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) { set_cuda_error(e, "gemv_i8 launch"); return LSE_ERR_CUDA; }
    return LSE_OK;
}

// Groups per row block the decode kernel prefetches into L2 ahead of its register loads, for
// M <= 8 (one group measured best on B200: 5-14% faster at M = 1 and 4; at M = 9..16, where
// the activation loads weigh more, prefetching measured 3-5% slower and is off)
// (0 disables).
int skinny_prefetch_groups() {
    static const int v = std::max(0, tuning_knob("LSE_SKINNY_PF", 1));
    return v;
}

template <int MT, int KW, int R, int U, bool BF16, int MINB, bool SILU_MUL = false, typename XT = __nv_bfloat16>
cudaError_t launch_skinny(const void *x, int64_t M, int64_t K, int64_t ldx, const int8_t *wp, const float *scale,
                          int64_t N, void *y, int64_t ldy, const void *res, int64_t ldr, cudaStream_t st) {
    const int64_t row_blocks = SILU_MUL ? N / 8 : (N + 15) / 16;  // weight row blocks (SILU_MUL: 2N rows)
    dim3 grid(static_cast<unsigned>((row_blocks + R - 1) / R), static_cast<unsigned>((M + 8 * MT - 1) / (8 * MT)));
    auto kernel = skinny_i8_kernel<MT, KW, R, U, BF16, MINB, SILU_MUL, XT>;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    launch_config(cfg, attr, grid, dim3(KW * 32), 0, st);
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<const XT *>(x), ldx,
                              static_cast<int>(M), static_cast<int>(K), wp, scale, static_cast<int>(N),
                              static_cast<XT *>(y), ldy, static_cast<const XT *>(res), ldr,
                              static_cast<int>(packed_cols(K)),
                              MT == 1 ? skinny_prefetch_groups() : 0);
}

// Decode-kernel configuration by shape (measured on B200, Llama-3 projection shapes; variant
// sweeps of 32 layers' weights per CUDA graph, the winners below):
//   * very many row blocks (N/16 >= 4 x SMs: gate_up): CTAs of 8 warps on one row block, four
//     CTAs per SM (M <= 8; above that, four row blocks per CTA, so that each activation load,
//     which costs eight L1 wavefronts, serves 64 weight rows);
//   * many row blocks (N/16 >= 2 x SMs: QKV): CTAs of 8 warps on two row blocks, so every
//     activation load serves 32 weight rows, eight chunks per row block in registers (a warp's
//     K slice is then one or two register groups deep at K = 4096): M <= 8 at 4519 GB/s against
//     3884 with four chunks; M = 9..16 three CTAs per SM, one row block (3286 against 3227);
//   * few row blocks (O, down): CTAs of 16 warps, one row block (two for M > 8, where the
//     activation loads, not the weight stream, would otherwise saturate L1, and for a long K
//     at M <= 8: down 5257 GB/s against 4940);
//   * fp16 MMA for M <= 8 (cheapest widening), bf16 MMA for M > 8 (activations used as they
//     are).
// -1 selects by shape as above; 0..17 pin one configuration in sweeps.
int skinny_variant() {
    static const int v = tuning_knob("LSE_SKINNY_VARIANT", -1);
    return v;
}

// SILU (the fused gate_up + SiLU * mul): N is the intermediate size and the weight has 2N
// rows, which set the shape tier.
template <int MT, bool SILU = false>
cudaError_t launch_skinny_mt(int variant, const void *x, int64_t M, int64_t K, int64_t ldx, const int8_t *wp,
                             const float *scale, int64_t N, void *y, int64_t ldy, const void *res, int64_t ldr,
                             int num_sms, cudaStream_t st) {
    if (variant < 0) {
        const int64_t rb_per_sm = (SILU ? N / 8 : (N + 15) / 16) / num_sms;
        if (rb_per_sm >= 4) variant = MT == 1 ? 7 : 1;
        else if (SILU || MT == 4) variant = rb_per_sm >= 2 ? 1 : 0;
        else if (rb_per_sm >= 2) variant = MT == 1 ? 15 : 17;
        else variant = (MT == 1 && K >= 8192) ? 4 : 0;
    }
    if constexpr (MT == 4) {
        // 17..32 tokens: bf16 MMA, two row blocks per CTA so each activation load serves 32 rows
        switch (variant) {
            case 1: return launch_skinny<4, 8, 2, 4, true, 2, SILU>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
            case 2: return launch_skinny<4, 16, 1, 4, true, 1, SILU>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
            default: return launch_skinny<4, 8, 1, 4, true, 2, SILU>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
        }
    } else {
        constexpr bool BF = MT == 2;
        switch (variant) {
            case 1: return launch_skinny<MT, 8, 2, 4, BF, 2, SILU>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
            case 2: return launch_skinny<MT, 16, 1, 4, !BF, 2, SILU>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
            case 3: return launch_skinny<MT, 8, 2, 4, !BF, 2, SILU>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
            case 4: return launch_skinny<MT, 16, 2, 4, BF, 1, SILU>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
            case 5: return launch_skinny<MT, 8, 2, 2, BF, 3, SILU>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
            case 6: return launch_skinny<MT, 8, 2, 4, BF, 3, SILU>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
            case 7: return launch_skinny<MT, 8, 1, 4, BF, 4, SILU>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
            case 8: return launch_skinny<MT, 16, 1, 2, BF, 2, SILU>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
            case 9: return launch_skinny<MT, 8, 1, 8, BF, 4, SILU>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
            case 10: return launch_skinny<MT, 16, 1, 8, BF, 2, SILU>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
            // four row blocks per CTA: each activation load serves 64 weight rows
            case 11: return launch_skinny<MT, 8, 4, 2, BF, 2, SILU>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
            case 12: return launch_skinny<MT, 4, 4, 2, BF, 4, SILU>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
            case 13: return launch_skinny<MT, 4, 4, 2, BF, 3, SILU>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
            case 14: return launch_skinny<MT, 8, 4, 1, BF, 2, SILU>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
            // eight chunks per row block in registers: a short K slice (O, QKV at K = 4096) is
            // one or two register groups deep instead of two to four
            case 15: return launch_skinny<MT, 8, 2, 8, BF, 2, SILU>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
            case 16: return launch_skinny<MT, 16, 1, 8, BF, 1, SILU>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
            case 17: return launch_skinny<MT, 8, 1, 8, BF, 3, SILU>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
            default:
                if constexpr (MT == 1) return launch_skinny<1, 16, 1, 4, false, 2, SILU>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
                else return launch_skinny<2, 16, 2, 4, true, 1, SILU>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
        }
    }
}

// fp16 activations: the fp16 MMA at every token count, in the shapes the bf16 policy above
// picks for the same weight (the activations enter the MMA as they are).
template <int MT, bool SILU = false>
cudaError_t launch_skinny_f16(const void *x, int64_t M, int64_t K, int64_t ldx, const int8_t *wp, const float *scale,
                              int64_t N, void *y, int64_t ldy, const void *res, int64_t ldr, int num_sms,
                              cudaStream_t st) {
    const int64_t rb_per_sm = (SILU ? N / 8 : (N + 15) / 16) / num_sms;
    if (rb_per_sm >= 4) {
        if constexpr (MT == 1) return launch_skinny<1, 8, 1, 4, false, 4, SILU, __half>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
        else return launch_skinny<MT, 8, 2, 4, false, 2, SILU, __half>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
    }
    if (rb_per_sm >= 2) {
        if (SILU || MT == 4) return launch_skinny<MT, 8, 2, 4, false, 2, SILU, __half>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
        if constexpr (MT == 1) return launch_skinny<1, 8, 2, 8, false, 2, SILU, __half>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
        else return launch_skinny<MT, 8, 1, 8, false, 3, SILU, __half>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
    }
    if constexpr (MT == 1) {
        if (!SILU && K >= 8192) return launch_skinny<1, 16, 2, 4, false, 1, SILU, __half>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
        return launch_skinny<1, 16, 1, 4, false, 2, SILU, __half>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
    } else if constexpr (MT == 2) {
        return launch_skinny<2, 16, 2, 4, false, 1, SILU, __half>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
    } else {
        return launch_skinny<4, 8, 1, 4, false, 2, SILU, __half>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, st);
    }
}

constexpr int64_t kSkinnyMaxM = 32;  // the decode kernel's token range (four 8-token tiles)

int run_skinny(const void *x, int64_t M, int64_t K, int64_t ldx, const int8_t *wp, const float *scale, int64_t N,
               void *y, int64_t ldy, const void *res, int64_t ldr, int num_sms, cudaStream_t st, bool xf16 = false) {
    if (M > kSkinnyMaxM) return LSE_ERR_UNSUPPORTED;
    const int variant = skinny_variant();
    cudaError_t e;
    if (xf16)
        e = M <= 8    ? launch_skinny_f16<1>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, num_sms, st)
            : M <= 16 ? launch_skinny_f16<2>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, num_sms, st)
                      : launch_skinny_f16<4>(x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, num_sms, st);
    else
        e = M <= 8    ? launch_skinny_mt<1>(variant, x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, num_sms, st)
            : M <= 16 ? launch_skinny_mt<2>(variant, x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, num_sms, st)
                      : launch_skinny_mt<4>(variant, x, M, K, ldx, wp, scale, N, y, ldy, res, ldr, num_sms, st);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) { set_cuda_error(e, "skinny_i8 launch"); return LSE_ERR_CUDA; }
    return LSE_OK;
}

// Auto policy.  Row-major W: the CUDA-core GEMV while its FMA work stays under the HBM
// stream (M <= 2), the tensor-core kernel from there on.  Packed W: the warp-MMA skinny
// kernel while the weight stream, not MMA issue, is the bound (M <= 16); from 17 to 32 tokens
// still the skinny kernel for a weight of at most kSkinnySmallWeight bytes, where the
// tensor-core kernel's fixed cost per launch (the split launch in front of it, the first stage,
// the cluster reduction) outweighs its faster stream; the tcgen05 kernel otherwise.  Measured
// on B200 (32 layers' weights per CUDA graph, us per launch, skinny against tcgen05) at
// M = 17 / 32: QKV 4096 x 6144 11.7 / 12.4 against 13.2 / 13.6, O 4096 x 4096 7.3 / 8.4
// against 10.7 / 11.2, down 14336 x 4096 20.8 / 23.1 against 17.3 / 19.4, gate_up
// 4096 x 28672 37.3 / 41.3 against 28.8 / 30.1: the two lines cross near 32 MB.
constexpr int64_t kSkinnySmallWeight = int64_t(32) << 20;
int auto_algo(int64_t M, int64_t K, int64_t N, bool packed) {
    if (packed)
        return (M <= 16 || (M <= kSkinnyMaxM && N * K <= kSkinnySmallWeight)) ? LSE_ALGO_SKINNY : LSE_ALGO_TCGEN05;
    return M <= 2 ? LSE_ALGO_GEMV : LSE_ALGO_TCGEN05;
}

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
    (void)N;
    if (M <= 0 || K < 0) return LSE_WS_COUNTER_BYTES;
    return tci8_workspace_bytes(token_tile(M), digit_planes(M), kMaxGridForWorkspace, M, K);
}

size_t lse_int8_linear_workspace_for(int64_t M, int64_t K, int64_t N, int algo, int packed) {
    if (algo == LSE_ALGO_AUTO) algo = auto_algo(M, K, N, packed != 0);
    if (algo != LSE_ALGO_TCGEN05) return 0;
    return lse_int8_linear_workspace(M, K, N);
}

}  // extern "C"

namespace lse {
namespace {
// res (may be null): y = bf16(res + s * acc), res bf16 [M, N] with row stride ldr; res may be
// y itself (same pointer and stride): every element is read before it is written, by the
// same thread.
int linear_impl(const void *x, int64_t M, int64_t K, int64_t ldx, const int8_t *w, const float *scale, int64_t N,
                void *y, int64_t ldy, void *workspace, size_t workspace_bytes, int algo, bool packed, void *stream,
                const void *res = nullptr, int64_t ldr = 0, bool xf16 = false) {
    if (M < 0 || N < 0 || K < 0) return LSE_ERR_INVALID_ARG;
    if (M == 0 || N == 0) return LSE_OK;
    if (!x || !w || !scale || !y) return LSE_ERR_INVALID_ARG;
    if (ldx < K || ldy < N) return LSE_ERR_INVALID_ARG;
    if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return LSE_ERR_UNSUPPORTED;
    if ((K & 15) || (ldx & 7) || !aligned16(x) || !aligned16(w)) return LSE_ERR_ALIGNMENT;
    if ((reinterpret_cast<uintptr_t>(y) & 1u) || (reinterpret_cast<uintptr_t>(scale) & 3u)) return LSE_ERR_ALIGNMENT;
    if (res && (ldr < N || (reinterpret_cast<uintptr_t>(res) & 1u))) return ldr < N ? LSE_ERR_INVALID_ARG : LSE_ERR_ALIGNMENT;
    if (res == y && ldr != ldy) return LSE_ERR_INVALID_ARG;  // in place only element for element
    if (algo < LSE_ALGO_AUTO || algo > LSE_ALGO_SKINNY) return LSE_ERR_INVALID_ARG;
    if ((algo == LSE_ALGO_GEMV && packed) || (algo == LSE_ALGO_SKINNY && !packed)) return LSE_ERR_UNSUPPORTED;
    int dev = 0;
    int rc = current_device(&dev);
    if (rc) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (K == 0) {  // y = 0, or y = res
        cudaError_t e = cudaSuccess;
        if (!res) e = cudaMemset2DAsync(y, static_cast<size_t>(ldy) * 2, 0, static_cast<size_t>(N) * 2,
                                        static_cast<size_t>(M), st);
        else if (res != y)
            e = cudaMemcpy2DAsync(y, static_cast<size_t>(ldy) * 2, res, static_cast<size_t>(ldr) * 2,
                                  static_cast<size_t>(N) * 2, static_cast<size_t>(M), cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) { set_cuda_error(e, "K == 0 output"); return LSE_ERR_CUDA; }
        return LSE_OK;
    }
    if (algo == LSE_ALGO_AUTO) algo = auto_algo(M, K, N, packed);
    if (xf16 && !packed) return LSE_ERR_UNSUPPORTED;  // fp16 activations: packed weights only
    if (algo == LSE_ALGO_GEMV) return run_gemv(x, M, K, ldx, w, scale, N, y, ldy, st);  // row-major: no res
    if (algo == LSE_ALGO_SKINNY)
        return run_skinny(x, M, K, ldx, w, scale, N, y, ldy, res, ldr, g_dev[dev].num_sms, st, xf16);

    const TcPlan pl = plan_tc(M, K, N, g_dev[dev].num_sms, dev);
    if (!workspace || !aligned16(workspace) ||
        workspace_bytes < tci8_workspace_bytes(pl.nt, digit_planes(M), pl.grid, M, K))
        return LSE_ERR_WORKSPACE;
    return run_tc_i8<false>(pl, x, M, K, ldx, w, scale, N, y, ldy, res, ldr, workspace, packed, st, xf16);
}
}  // namespace
}  // namespace lse

extern "C" {

int lse_int8_linear_ex(const void *x, int64_t M, int64_t K, int64_t ldx, const int8_t *w, const float *scale,
                       int64_t N, void *y, int64_t ldy, void *workspace, size_t workspace_bytes, int algo,
                       void *stream) {
    return linear_impl(x, M, K, ldx, w, scale, N, y, ldy, workspace, workspace_bytes, algo, false, stream);
}

int lse_int8_linear(const void *x, int64_t M, int64_t K, int64_t ldx, const int8_t *w, const float *scale,
                    int64_t N, void *y, int64_t ldy, void *workspace, size_t workspace_bytes, void *stream) {
    return linear_impl(x, M, K, ldx, w, scale, N, y, ldy, workspace, workspace_bytes, LSE_ALGO_AUTO, false,
                       stream);
}

int lse_int8_linear_packed(const void *x, int64_t M, int64_t K, int64_t ldx, const int8_t *w_packed,
                           const float *scale, int64_t N, void *y, int64_t ldy, void *workspace,
                           size_t workspace_bytes, int algo, void *stream) {
    return linear_impl(x, M, K, ldx, w_packed, scale, N, y, ldy, workspace, workspace_bytes, algo, true, stream);
}

int lse_int8_linear_packed_residual(const void *x, int64_t M, int64_t K, int64_t ldx, const int8_t *w_packed,
                                    const float *scale, int64_t N, const void *residual, int64_t ldr, void *y,
                                    int64_t ldy, void *workspace, size_t workspace_bytes, int algo, void *stream) {
    if (!residual) return LSE_ERR_INVALID_ARG;
    return linear_impl(x, M, K, ldx, w_packed, scale, N, y, ldy, workspace, workspace_bytes, algo, true, stream,
                       residual, ldr);
}

size_t lse_int8_packed_weight_bytes(int64_t N, int64_t K) {
    if (N <= 0 || K <= 0) return 0;
    return static_cast<size_t>(packed_weight_bytes(N, K));
}

int lse_int8_pack_weight(const int8_t *w, int64_t N, int64_t K, int64_t ldw, int8_t *w_packed, void *stream) {
    if (N < 0 || K < 0 || ldw < K) return LSE_ERR_INVALID_ARG;
    if (N == 0 || K == 0) return LSE_OK;
    if (!w || !w_packed) return LSE_ERR_INVALID_ARG;
    if (!aligned16(w_packed)) return LSE_ERR_ALIGNMENT;
    int dev = 0;
    int rc = current_device(&dev);
    if (rc) return rc;
    const int64_t runs = packed_weight_bytes(N, K) / 16;
    pack_weight_kernel<<<static_cast<unsigned>((runs + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        w, N, K, ldw, w_packed, packed_cols(K), runs);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { set_cuda_error(e, "pack launch"); return LSE_ERR_CUDA; }
    return LSE_OK;
}

int lse_int8_unpack_weight(const int8_t *w_packed, int64_t N, int64_t K, int8_t *w, void *stream) {
    if (N < 0 || K < 0) return LSE_ERR_INVALID_ARG;
    if (N == 0 || K == 0) return LSE_OK;
    if (!w || !w_packed) return LSE_ERR_INVALID_ARG;
    int dev = 0;
    int rc = current_device(&dev);
    if (rc) return rc;
    const int64_t total = N * K;
    unpack_weight_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        w_packed, N, K, w, packed_cols(K));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { set_cuda_error(e, "unpack launch"); return LSE_ERR_CUDA; }
    return LSE_OK;
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

}  // extern "C"

namespace lse {
namespace {

template <int D, int G, typename T>
cudaError_t launch_pattn(const pattn::Params &p, int64_t E, int64_t max_q_len, cudaStream_t st) {
    constexpr int smem = pattn::smem_bytes<D>();
    auto kernel = pattn::paged_attn_kernel<D, G, T>;
    {  // opt in to more than 48 KB of dynamic shared memory, once per device
        static std::once_flag once[kMaxDevices];
        static cudaError_t set_err[kMaxDevices];
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
        std::call_once(once[dev], [&] {
            set_err[dev] = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        });
        if (set_err[dev] != cudaSuccess) return set_err[dev];
    }
    constexpr int toks = pattn::ROWS / G;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    launch_config(cfg, attr, dim3(static_cast<unsigned>((max_q_len + toks - 1) / toks), static_cast<unsigned>(E),
                                  static_cast<unsigned>(p.H_kv)),
                  dim3(pattn::THREADS), smem, st);
    return cudaLaunchKernelEx(&cfg, kernel, p);
}

template <int D, typename T>
cudaError_t launch_pattn_g(int64_t G, const pattn::Params &p, int64_t E, int64_t max_q_len, cudaStream_t st) {
    switch (G) {
        case 1: return launch_pattn<D, 1, T>(p, E, max_q_len, st);
        case 2: return launch_pattn<D, 2, T>(p, E, max_q_len, st);
        case 4: return launch_pattn<D, 4, T>(p, E, max_q_len, st);
        default: return launch_pattn<D, 8, T>(p, E, max_q_len, st);
    }
}

}  // namespace
}  // namespace lse

extern "C" int lse_paged_attention(const void *q, int dtype, int64_t H, int64_t D, int64_t q_stride_h,
                                   int64_t q_stride_m, const void *k_pool, const void *v_pool, int64_t num_blocks,
                                   int64_t block_size, int64_t H_kv, const int32_t *block_table, int64_t bt_stride,
                                   const int32_t *context_len, const int32_t *query_offset, const int32_t *q_start,
                                   const int32_t *q_len, int64_t E, int64_t max_q_len, float scale, void *o,
                                   int64_t o_stride_h, int64_t o_stride_m, void *stream) {
    if (E < 0 || H <= 0 || H_kv <= 0 || D <= 0 || num_blocks <= 0 || block_size <= 0 || max_q_len < 0)
        return LSE_ERR_INVALID_ARG;
    if (E == 0 || max_q_len == 0) return LSE_OK;
    if (!q || !k_pool || !v_pool || !block_table || !context_len || !query_offset || !q_start || !q_len || !o)
        return LSE_ERR_INVALID_ARG;
    if (H % H_kv) return LSE_ERR_INVALID_ARG;
    if (dtype != LSE_BF16 && dtype != LSE_F16) return LSE_ERR_UNSUPPORTED;
    const int64_t G = H / H_kv;
    if ((D != 64 && D != 128) || (G != 1 && G != 2 && G != 4 && G != 8)) return LSE_ERR_UNSUPPORTED;
    if (E > 65535 || H_kv > 65535 || num_blocks * block_size > INT32_MAX / 2 || bt_stride < 0 ||
        max_q_len > INT32_MAX / 2)
        return LSE_ERR_UNSUPPORTED;
    if ((q_stride_h & 1) || (q_stride_m & 1) || (o_stride_h & 1) || (o_stride_m & 1) || !aligned16(q) || !aligned16(o) ||
        !aligned16(k_pool) || !aligned16(v_pool))
        return LSE_ERR_ALIGNMENT;
    int dev = 0;
    int rc = current_device(&dev);
    if (rc) return rc;
    pattn::Params p{};
    p.q = q;
    p.q_sh = q_stride_h;
    p.q_sm = q_stride_m;
    p.k_pool = k_pool;
    p.v_pool = v_pool;
    p.block_table = block_table;
    p.bt_stride = bt_stride;
    p.context_len = context_len;
    p.query_offset = query_offset;
    p.q_start = q_start;
    p.q_len = q_len;
    p.o = o;
    p.o_sh = o_stride_h;
    p.o_sm = o_stride_m;
    p.H_kv = static_cast<int>(H_kv);
    p.block_size = static_cast<int>(block_size);
    p.num_blocks = static_cast<int>(num_blocks);
    p.scale_log2 = scale * 1.4426950408889634f;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e;
    if (dtype == LSE_BF16)
        e = D == 128 ? launch_pattn_g<128, __nv_bfloat16>(G, p, E, max_q_len, st)
                     : launch_pattn_g<64, __nv_bfloat16>(G, p, E, max_q_len, st);
    else
        e = D == 128 ? launch_pattn_g<128, __half>(G, p, E, max_q_len, st) : launch_pattn_g<64, __half>(G, p, E, max_q_len, st);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) { set_cuda_error(e, "paged_attn launch"); return LSE_ERR_CUDA; }
    return LSE_OK;
}

extern "C" {

int lse_set_wait_limit(int device, long long cycles) {
    int rc = init_device(device);
    if (rc) return rc;
    int prev = -1;
    cudaError_t e = cudaGetDevice(&prev);
    if (e != cudaSuccess) { set_cuda_error(e, "cudaGetDevice"); return LSE_ERR_CUDA; }
    if (prev != device && (e = cudaSetDevice(device)) != cudaSuccess) {
        set_cuda_error(e, "cudaSetDevice");
        return LSE_ERR_CUDA;
    }
    const long long v = cycles > 0 ? cycles : kWaitLimitCycles;
    e = cudaMemcpyToSymbol(g_wait_limit, &v, sizeof(v));
    if (prev != device) cudaSetDevice(prev);
    if (e != cudaSuccess) { set_cuda_error(e, "lse_set_wait_limit"); return LSE_ERR_CUDA; }
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

// ---------------------------------------------------------------------------------------
// lse_int8_linear_packed_noalloc: the tensor-core path with its scratch in a static device
// array instead of a caller workspace, for callers that cannot allocate one (a binding of
// the engine's x, W, s -> y call has no workspace argument, and the engine gives the HBM
// left after loading to its KV-cache pool).  Allocates nothing.
// ---------------------------------------------------------------------------------------
namespace lse {
namespace {

// One array per device (module globals live in each device's context).  Without an
// initializer it takes no space in the library file; its contents are never assumed: the
// counters a call needs are cleared by that call, partial tiles are written before read.
static __device__ __align__(256) uint8_t g_noalloc_scratch[LSE_NOALLOC_SCRATCH_BYTES];

struct NoAllocState {
    std::once_flag once;
    int status = LSE_ERR_CUDA;
    void *ptr = nullptr;
};
NoAllocState g_noalloc[kMaxDevices];

// Device address of g_noalloc_scratch, looked up once per device with that device current
// (the caller's current device: lse_int8_linear_packed_noalloc runs on it).
int noalloc_scratch(int device, void **ptr) {
    NoAllocState &s = g_noalloc[device];
    std::call_once(s.once, [&] {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) { set_cuda_error(e, "cudaGetSymbolAddress(no-alloc scratch)"); return; }
        if (!aligned16(p)) {
            std::snprintf(t_last_error, sizeof(t_last_error), "no-alloc scratch at %p is not 16-byte aligned", p);
            return;
        }
        s.ptr = p;
        s.status = LSE_OK;
    });
    *ptr = s.ptr;
    return s.status;
}

}  // namespace
}  // namespace lse

extern "C" int lse_int8_linear_packed_noalloc(const void *x, int64_t M, int64_t K, int64_t ldx,
                                              const int8_t *w_packed, const float *scale, int64_t N, void *y,
                                              int64_t ldy, void *stream) {
    // Host-side checks first (nothing touches the GPU before they pass): the same ones
    // linear_impl makes, plus the token limit of the fixed scratch.
    if (M > LSE_NOALLOC_MAX_M) {
        std::snprintf(t_last_error, sizeof(t_last_error),
                      "lse_int8_linear_packed_noalloc: M=%lld exceeds LSE_NOALLOC_MAX_M=%d (its fixed %d-byte "
                      "scratch); use lse_int8_linear_packed with a workspace",
                      static_cast<long long>(M), LSE_NOALLOC_MAX_M, LSE_NOALLOC_SCRATCH_BYTES);
        return LSE_ERR_WORKSPACE;
    }
    if (M < 0 || N < 0 || K < 0) return LSE_ERR_INVALID_ARG;
    if (M == 0 || N == 0) return LSE_OK;
    if (!x || !w_packed || !scale || !y) return LSE_ERR_INVALID_ARG;
    if (ldx < K || ldy < N) return LSE_ERR_INVALID_ARG;
    if (N > INT32_MAX || K > INT32_MAX) return LSE_ERR_UNSUPPORTED;
    if ((K & 15) || (ldx & 7) || !aligned16(x) || !aligned16(w_packed)) return LSE_ERR_ALIGNMENT;
    if ((reinterpret_cast<uintptr_t>(y) & 1u) || (reinterpret_cast<uintptr_t>(scale) & 3u)) return LSE_ERR_ALIGNMENT;
    int dev = 0;
    int rc = current_device(&dev);
    if (rc) return rc;
    void *scratch = nullptr;
    rc = noalloc_scratch(dev, &scratch);
    if (rc) return rc;
    if (K > 0) {
        // 64 KB of counters + 2 * grid * 64 * 128 * 4 bytes of partial tiles (9.7 MB for 148
        // SMs) + 3 digit planes of M x Kp bytes + M row scales: for M = 64 the array holds K up
        // to about 36,000 on a 148-SM part.
        const TcPlan pl = plan_tc(M, K, N, g_dev[dev].num_sms, dev);
        const size_t need = tci8_workspace_bytes(pl.nt, digit_planes(M), pl.grid, M, K);
        if (need > static_cast<size_t>(LSE_NOALLOC_SCRATCH_BYTES)) {
            std::snprintf(t_last_error, sizeof(t_last_error),
                          "lse_int8_linear_packed_noalloc: this shape needs %zu scratch bytes, the fixed array "
                          "holds %d",
                          need, LSE_NOALLOC_SCRATCH_BYTES);
            return LSE_ERR_WORKSPACE;
        }
    }
    // The split kernel that precedes the projection clears the stream-K counters it uses, so
    // nothing of an earlier call's contents is relied upon.
    return linear_impl(x, M, K, ldx, w_packed, scale, N, y, ldy, scratch, LSE_NOALLOC_SCRATCH_BYTES,
                       LSE_ALGO_TCGEN05, true, stream);
}

// ---------------------------------------------------------------------------------------
// The MLP's gate and up projections and SiLU * mul in one projection launch: M <= 16 on the
// decode kernel (workspace unused), larger M on the tensor-core kernel with SiLU * mul in its
// epilogue (tc_i8.cuh, SILU = true), after the activation split.
// ---------------------------------------------------------------------------------------
namespace lse {
namespace {
int gate_up_impl(const void *x, int64_t M, int64_t K, int64_t ldx, const int8_t *w_packed, const float *scale,
                 int64_t I, void *y, int64_t ldy, void *workspace, size_t workspace_bytes, void *stream, bool xf16,
                 bool decode_only) {
    if (M < 0 || I < 0 || K < 0) return LSE_ERR_INVALID_ARG;
    if (M == 0 || I == 0) return LSE_OK;
    if (!x || !w_packed || !scale || !y) return LSE_ERR_INVALID_ARG;
    if (ldx < K || ldy < I) return LSE_ERR_INVALID_ARG;
    if (I % 8) return LSE_ERR_UNSUPPORTED;
    if ((decode_only && M > 16) || M > INT32_MAX || 2 * I > INT32_MAX || K > INT32_MAX) return LSE_ERR_UNSUPPORTED;
    if ((K & 15) || (ldx & 7) || !aligned16(x) || !aligned16(w_packed)) return LSE_ERR_ALIGNMENT;
    if ((reinterpret_cast<uintptr_t>(y) & 1u) || (reinterpret_cast<uintptr_t>(scale) & 3u)) return LSE_ERR_ALIGNMENT;
    int dev = 0;
    int rc = current_device(&dev);
    if (rc) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (K == 0) {  // silu(0) * 0
        const cudaError_t e = cudaMemset2DAsync(y, static_cast<size_t>(ldy) * 2, 0, static_cast<size_t>(I) * 2,
                                                static_cast<size_t>(M), st);
        if (e != cudaSuccess) { set_cuda_error(e, "cudaMemset2DAsync"); return LSE_ERR_CUDA; }
        return LSE_OK;
    }
    const int num_sms = g_dev[dev].num_sms;
    if (M <= 16) {
        const int variant = skinny_variant();
        cudaError_t e;
        if (xf16)
            e = M <= 8 ? launch_skinny_f16<1, true>(x, M, K, ldx, w_packed, scale, I, y, ldy, nullptr, 0, num_sms, st)
                       : launch_skinny_f16<2, true>(x, M, K, ldx, w_packed, scale, I, y, ldy, nullptr, 0, num_sms, st);
        else
            e = M <= 8 ? launch_skinny_mt<1, true>(variant, x, M, K, ldx, w_packed, scale, I, y, ldy, nullptr, 0, num_sms, st)
                       : launch_skinny_mt<2, true>(variant, x, M, K, ldx, w_packed, scale, I, y, ldy, nullptr, 0, num_sms, st);
        if (e == cudaSuccess) e = cudaGetLastError();
        if (e != cudaSuccess) { set_cuda_error(e, "skinny_i8 gate_up launch"); return LSE_ERR_CUDA; }
        return LSE_OK;
    }
    const int64_t N = 2 * I;
    const TcPlan pl = plan_tc(M, K, N, num_sms, dev);
    if (!workspace || !aligned16(workspace) ||
        workspace_bytes < tci8_workspace_bytes(pl.nt, digit_planes(M), pl.grid, M, K))
        return LSE_ERR_WORKSPACE;
    return run_tc_i8<true>(pl, x, M, K, ldx, w_packed, scale, N, y, ldy, nullptr, 0, workspace, true, st, xf16);
}

int activation_type(int dtype, bool *xf16) {
    if (dtype == LSE_BF16) *xf16 = false;
    else if (dtype == LSE_F16) *xf16 = true;
    else return LSE_ERR_UNSUPPORTED;
    return LSE_OK;
}
}  // namespace
}  // namespace lse

extern "C" {

int lse_int8_gate_up_silu_packed(const void *x, int64_t M, int64_t K, int64_t ldx, const int8_t *w_packed,
                                 const float *scale, int64_t I, void *y, int64_t ldy, void *stream) {
    return gate_up_impl(x, M, K, ldx, w_packed, scale, I, y, ldy, nullptr, 0, stream, false, true);
}

int lse_int8_gate_up_silu_packed_ws(const void *x, int64_t M, int64_t K, int64_t ldx, const int8_t *w_packed,
                                    const float *scale, int64_t I, void *y, int64_t ldy, void *workspace,
                                    size_t workspace_bytes, void *stream) {
    return gate_up_impl(x, M, K, ldx, w_packed, scale, I, y, ldy, workspace, workspace_bytes, stream, false, false);
}

int lse_int8_gate_up_silu_packed_dt(const void *x, int dtype, int64_t M, int64_t K, int64_t ldx,
                                    const int8_t *w_packed, const float *scale, int64_t I, void *y, int64_t ldy,
                                    void *workspace, size_t workspace_bytes, void *stream) {
    bool xf16 = false;
    const int rc = activation_type(dtype, &xf16);
    if (rc) return rc;
    return gate_up_impl(x, M, K, ldx, w_packed, scale, I, y, ldy, workspace, workspace_bytes, stream, xf16, false);
}

int lse_int8_linear_packed_dt(const void *x, int dtype, int64_t M, int64_t K, int64_t ldx, const int8_t *w_packed,
                              const float *scale, int64_t N, const void *residual, int64_t ldr, void *y, int64_t ldy,
                              void *workspace, size_t workspace_bytes, int algo, void *stream) {
    bool xf16 = false;
    const int rc = activation_type(dtype, &xf16);
    if (rc) return rc;
    return linear_impl(x, M, K, ldx, w_packed, scale, N, y, ldy, workspace, workspace_bytes, algo, true, stream,
                       residual, residual ? ldr : 0, xf16);
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// lse_paged_decode_attention: decode attention over the paged K/V pool (decode_attn.cuh).
// ---------------------------------------------------------------------------------------
namespace lse {
namespace {

struct AttnPlan {
    int splits, chunk;
};

// Workspace of a split launch: a fixed region of arrival counters (one per (sequence, KV
// head) pair; splits happen only for fewer pairs than this), then the fp32 partials.  The
// counters sit at the same place for every launch shape, so one zero-initialised buffer
// serves every shape on a stream.
constexpr int64_t kAttnMaxSplitPairs = 1024;
constexpr size_t kAttnCounterBytes = kAttnMaxSplitPairs * sizeof(int);

// Split the positions of a (sequence, KV head) pair only when there are too few pairs to fill
// the GPU, and only into as many splits as leave the launch at about one and a half CTAs per
// SM, with at least 128 positions per split.  A CTA pays a few microseconds before its stream
// is full (context length and block-table loads, pipeline fill) and again at the end (warp
// merge, partials), so small batches want splits; but residency is two CTAs per SM (184
// registers x 128 threads, 104 KB of shared memory), a second wave pays the fixed costs twice,
// and in a decode step the next projection's CTAs start their weight streams under this
// kernel (programmatic dependent launch) only where an SM has room left.  Measured on B200 at
// 1025 positions, the kernel alone (32 layers' pools per CUDA graph): 1 sequence 8.9 us in 5
// splits of >= 256 positions, 8.0 us in 9 of >= 128, 8.9 us in 17; 4 sequences 10.7 us in 5
// splits, 10.3 us in 7, 9.8 us in 9; 8 sequences 12.8 us in 3 splits, 12.5 us in 4, 16.6 us in
// 5 (two waves); 16 sequences 19.3 us unsplit, 17.4 us in 2 splits, 22.9 us in 3.  In the
// Llama-3-8B decode step (llama_decode.py, 1024-token context, CUDA graph): 8 sequences
// 2.738 ms/step in 3 splits, 2.760 in 4, 2.774 in 2; 16 sequences 3.384 ms unsplit, 3.460 in 2
// splits.
//
// Fewest positions per split, and the CTAs a split launch may reach (0: 1.5 per SM).
int attn_min_chunk() {
    static const int v = [] {
        const int c = tuning_knob("LSE_ATTN_MIN_CHUNK", 128);
        return c > 0 ? c : 128;
    }();
    return v;
}
int attn_target_ctas(int num_sms) {
    static const int v = std::max(0, tuning_knob("LSE_ATTN_TARGET_CTAS", 0));
    return v > 0 ? v : 3 * num_sms / 2;
}

AttnPlan plan_attn(int64_t E, int64_t H_kv, int64_t max_context, int64_t block_size, int num_sms,
                   bool unsplit = false) {
    const int64_t pairs = std::max<int64_t>(1, E * H_kv);
    const int64_t min_chunk = attn_min_chunk();
    const int64_t target = attn_target_ctas(num_sms);
    const int64_t cap = std::max<int64_t>(1, (max_context + min_chunk - 1) / min_chunk);
    if (unsplit)  // one CTA per (sequence, KV head) over all of max_context (the kernel stages
                  // at most attn::MAX_TABLE block ids and reports a longer context)
        return {1, static_cast<int>(std::max<int64_t>(32, (max_context + 31) / 32 * 32))};
    int64_t splits = 1;
    if (2 * pairs <= target && pairs <= kAttnMaxSplitPairs) splits = std::min<int64_t>(target / pairs, cap);
    // a CTA stages at most attn::MAX_TABLE block-table entries (chunk / block_size + 1)
    const int64_t max_chunk = (attn::MAX_TABLE - 1) * block_size / 32 * 32;
    splits = std::max<int64_t>(splits, (max_context + max_chunk - 1) / max_chunk);
    int64_t chunk = (max_context + splits - 1) / splits;
    chunk = std::max<int64_t>(32, (chunk + 31) / 32 * 32);
    splits = std::max<int64_t>(1, (max_context + chunk - 1) / chunk);
    return {static_cast<int>(splits), static_cast<int>(chunk)};
}

size_t attn_workspace_bytes(const AttnPlan &pl, int64_t E, int64_t H, int64_t H_kv, int64_t D) {
    if (pl.splits <= 1) return 0;
    const int64_t G = H / H_kv;
    return kAttnCounterBytes + static_cast<size_t>(E * H_kv) * pl.splits * G * (D + 2) * sizeof(float);
}

template <int D, int G, typename T>
cudaError_t launch_attn(const attn::Params &p, int64_t E, cudaStream_t st) {
    constexpr int smem = attn::attn_smem_bytes<D>();
    auto kernel = attn::paged_decode_kernel<D, G, T>;
    {  // opt in to the ring's shared memory (with the static part it exceeds 48 KB), once per device
        static std::once_flag once[kMaxDevices];
        static cudaError_t set_err[kMaxDevices];
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
        std::call_once(once[dev], [&] {
            set_err[dev] = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        });
        if (set_err[dev] != cudaSuccess) return set_err[dev];
    }
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    launch_config(cfg, attr, dim3(p.splits, p.H_kv, static_cast<unsigned>(E)), dim3(attn::THREADS), smem, st);
    return cudaLaunchKernelEx(&cfg, kernel, p);
}

// The kernel instance for head_dim D (64 or 128) and group size G (1, 2, 4, 8).
template <typename T>
cudaError_t launch_attn_dg(const attn::Params &p, int64_t D, int64_t G, int64_t E, cudaStream_t st) {
    cudaError_t e;
    if (D == 128) {
        switch (G) {
            case 1: e = launch_attn<128, 1, T>(p, E, st); break;
            case 2: e = launch_attn<128, 2, T>(p, E, st); break;
            case 4: e = launch_attn<128, 4, T>(p, E, st); break;
            default: e = launch_attn<128, 8, T>(p, E, st); break;
        }
    } else {
        switch (G) {
            case 1: e = launch_attn<64, 1, T>(p, E, st); break;
            case 2: e = launch_attn<64, 2, T>(p, E, st); break;
            case 4: e = launch_attn<64, 4, T>(p, E, st); break;
            default: e = launch_attn<64, 8, T>(p, E, st); break;
        }
    }
    return e == cudaSuccess ? cudaGetLastError() : e;
}

}  // namespace
}  // namespace lse

extern "C" size_t lse_paged_decode_attention_workspace(int64_t E, int64_t H, int64_t H_kv, int64_t D,
                                                       int64_t max_context, int64_t block_size) {
    if (E <= 0 || H <= 0 || H_kv <= 0 || D <= 0 || max_context <= 0 || block_size <= 0 || H % H_kv) return 0;
    int dev = 0;
    if (current_device(&dev)) return 0;
    return attn_workspace_bytes(plan_attn(E, H_kv, max_context, block_size, g_dev[dev].num_sms), E, H, H_kv, D);
}

extern "C" int lse_paged_decode_attention_dt(const void *q, int dtype, int64_t E, int64_t H, int64_t D,
                                             int64_t q_stride_e, int64_t q_stride_h, const void *k_pool,
                                             const void *v_pool, int64_t num_blocks, int64_t block_size, int64_t H_kv,
                                             const int32_t *block_table, int64_t bt_stride,
                                             const int32_t *context_len, int64_t max_context, float scale, void *o,
                                             int64_t o_stride_e, int64_t o_stride_h, void *workspace,
                                             size_t workspace_bytes, void *stream) {
    if (E < 0 || H <= 0 || H_kv <= 0 || D <= 0 || num_blocks <= 0 || block_size <= 0 || max_context < 0)
        return LSE_ERR_INVALID_ARG;
    if (dtype != LSE_BF16 && dtype != LSE_F16) return LSE_ERR_UNSUPPORTED;
    if (E == 0) return LSE_OK;
    if (!q || !k_pool || !v_pool || !block_table || !context_len || !o) return LSE_ERR_INVALID_ARG;
    if (H % H_kv) return LSE_ERR_INVALID_ARG;
    const int64_t G = H / H_kv;
    if ((D != 64 && D != 128) || (G != 1 && G != 2 && G != 4 && G != 8)) return LSE_ERR_UNSUPPORTED;
    if (E > 65535 || H_kv > 65535 || num_blocks * block_size > INT32_MAX / 2 || max_context > INT32_MAX / 2)
        return LSE_ERR_UNSUPPORTED;
    if (bt_stride < (max_context + block_size - 1) / block_size) return LSE_ERR_INVALID_ARG;
    // K/V rows are copied in 16-byte chunks; q is read as bf16 pairs
    if ((reinterpret_cast<uintptr_t>(q) & 3u) || (reinterpret_cast<uintptr_t>(k_pool) & 15u) ||
        (reinterpret_cast<uintptr_t>(v_pool) & 15u) || (q_stride_e % 2) || (q_stride_h % 2) ||
        (reinterpret_cast<uintptr_t>(o) & 1u) || (reinterpret_cast<uintptr_t>(block_table) & 3u) ||
        (reinterpret_cast<uintptr_t>(context_len) & 3u))
        return LSE_ERR_ALIGNMENT;
    int dev = 0;
    int rc = current_device(&dev);
    if (rc) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (max_context == 0) {  // no positions: softmax over nothing is 0 here
        for (int64_t e = 0; e < E; ++e) {
            const cudaError_t e2 = cudaMemset2DAsync(static_cast<__nv_bfloat16 *>(o) + e * o_stride_e,
                                                     static_cast<size_t>(o_stride_h) * 2, 0,
                                                     static_cast<size_t>(D) * 2, static_cast<size_t>(H), st);
            if (e2 != cudaSuccess) { set_cuda_error(e2, "cudaMemset2DAsync"); return LSE_ERR_CUDA; }
        }
        return LSE_OK;
    }
    // No workspace at all: one CTA per (sequence, KV head) wherever the context allows.
    const AttnPlan pl = plan_attn(E, H_kv, max_context, block_size, g_dev[dev].num_sms,
                                  workspace == nullptr && workspace_bytes == 0);
    if (pl.splits > attn::MAX_SPLITS) return LSE_ERR_UNSUPPORTED;  // a very long context at block_size < 16
    const size_t need = attn_workspace_bytes(pl, E, H, H_kv, D);
    if (need && (!workspace || workspace_bytes < need || !aligned16(workspace))) return LSE_ERR_WORKSPACE;
    attn::Params p{};
    p.q = q;
    p.q_stride_e = q_stride_e;
    p.q_stride_h = q_stride_h;
    p.k_pool = k_pool;
    p.v_pool = v_pool;
    p.block_table = block_table;
    p.bt_stride = bt_stride;
    p.context_len = context_len;
    p.o = o;
    p.o_stride_e = o_stride_e;
    p.o_stride_h = o_stride_h;
    p.E = static_cast<int>(E);
    p.H_kv = static_cast<int>(H_kv);
    p.block_size = static_cast<int>(block_size);
    p.num_blocks = static_cast<int>(num_blocks);
    p.chunk = pl.chunk;
    p.splits = pl.splits;
    p.max_ctx = static_cast<int>(max_context);
    p.scale_log2 = scale * 1.4426950408889634f;  // log2(e): softmax in base 2
    p.counters = static_cast<int *>(workspace);
    p.part = need ? reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + kAttnCounterBytes) : nullptr;
    const cudaError_t e = dtype == LSE_F16 ? launch_attn_dg<__half>(p, D, G, E, st)
                                           : launch_attn_dg<__nv_bfloat16>(p, D, G, E, st);
    if (e != cudaSuccess) { set_cuda_error(e, "paged_decode_attention launch"); return LSE_ERR_CUDA; }
    return LSE_OK;
}

extern "C" int lse_paged_decode_attention(const void *q, int64_t E, int64_t H, int64_t D, int64_t q_stride_e,
                                          int64_t q_stride_h, const void *k_pool, const void *v_pool,
                                          int64_t num_blocks, int64_t block_size, int64_t H_kv,
                                          const int32_t *block_table, int64_t bt_stride, const int32_t *context_len,
                                          int64_t max_context, float scale, void *o, int64_t o_stride_e,
                                          int64_t o_stride_h, void *workspace, size_t workspace_bytes,
                                          void *stream) {
    return lse_paged_decode_attention_dt(q, LSE_BF16, E, H, D, q_stride_e, q_stride_h, k_pool, v_pool, num_blocks,
                                         block_size, H_kv, block_table, bt_stride, context_len, max_context, scale, o,
                                         o_stride_e, o_stride_h, workspace, workspace_bytes, stream);
}

// ---------------------------------------------------------------------------------------
// lse_rope_kv_write: RoPE on q and k of the fused QKV output, q transposed to
// (heads, tokens, head_dim), k and v written to their per-token slots (rope_kv.cuh).
// ---------------------------------------------------------------------------------------
namespace lse {
namespace {
template <typename T>
int launch_rope(const void *qkv, int64_t M, int64_t ld_qkv, int64_t H, int64_t H_kv, int64_t D, const void *cos,
                const void *sin, int64_t ld_cs, int cs_dtype, void *q_out, void *k_dst, void *v_dst,
                const int64_t *kv_offset, int64_t kv_head_stride, int num_sms, cudaStream_t st) {
    rope::Params<T> p{};
    p.qkv = static_cast<const T *>(qkv);
    p.ld_qkv = ld_qkv;
    p.cos = cos;
    p.sin = sin;
    p.ld_cs = ld_cs;
    p.cs_type = cs_dtype == LSE_BF16 ? 1 : cs_dtype == LSE_F16 ? 2 : 0;
    p.q_out = static_cast<T *>(q_out);
    p.k_dst = static_cast<T *>(k_dst);
    p.v_dst = static_cast<T *>(v_dst);
    p.kv_off = kv_offset;
    p.kv_head_stride = kv_head_stride;
    p.M = static_cast<int>(M);
    p.H = static_cast<int>(H);
    p.H_kv = static_cast<int>(H_kv);
    p.D = static_cast<int>(D);
    const int64_t total = M * (H + 2 * H_kv) * (D / 2);
    const int64_t blocks = std::min<int64_t>((total + 255) / 256, 8LL * num_sms);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    launch_config(cfg, attr, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, st);
    cudaError_t e = cudaLaunchKernelEx(&cfg, rope::rope_kv_kernel<T>, p);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) { set_cuda_error(e, "rope_kv_write launch"); return LSE_ERR_CUDA; }
    return LSE_OK;
}
}  // namespace
}  // namespace lse

extern "C" int lse_rope_kv_write_dt(const void *qkv, int dtype, int64_t M, int64_t ld_qkv, int64_t H, int64_t H_kv,
                                    int64_t D, const void *cos, const void *sin, int64_t ld_cs, int cs_dtype,
                                    void *q_out, void *k_dst, void *v_dst, const int64_t *kv_offset,
                                    int64_t kv_head_stride, void *stream) {
    if (M < 0 || H <= 0 || H_kv <= 0 || D <= 0 || (D & 1)) return LSE_ERR_INVALID_ARG;
    if (dtype != LSE_BF16 && dtype != LSE_F16) return LSE_ERR_UNSUPPORTED;
    if (M == 0) return LSE_OK;
    if (!qkv || !cos || !sin || !q_out || !k_dst || !v_dst || !kv_offset) return LSE_ERR_INVALID_ARG;
    if (ld_qkv < (H + 2 * H_kv) * D || ld_cs < D) return LSE_ERR_INVALID_ARG;
    if (cs_dtype != LSE_F32 && cs_dtype != LSE_BF16 && cs_dtype != LSE_F16) return LSE_ERR_INVALID_ARG;
    if (M > INT32_MAX || (H + 2 * H_kv) * D > INT32_MAX) return LSE_ERR_UNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(qkv) & 1u) || (reinterpret_cast<uintptr_t>(q_out) & 1u) ||
        (reinterpret_cast<uintptr_t>(k_dst) & 1u) || (reinterpret_cast<uintptr_t>(v_dst) & 1u) ||
        (reinterpret_cast<uintptr_t>(kv_offset) & 7u) ||
        (reinterpret_cast<uintptr_t>(cos) & (cs_dtype == LSE_F32 ? 3u : 1u)) ||
        (reinterpret_cast<uintptr_t>(sin) & (cs_dtype == LSE_F32 ? 3u : 1u)))
        return LSE_ERR_ALIGNMENT;
    int dev = 0;
    int rc = current_device(&dev);
    if (rc) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int cs = cs_dtype;
    return dtype == LSE_F16 ? launch_rope<__half>(qkv, M, ld_qkv, H, H_kv, D, cos, sin, ld_cs, cs, q_out, k_dst, v_dst,
                                                  kv_offset, kv_head_stride, g_dev[dev].num_sms, st)
                            : launch_rope<__nv_bfloat16>(qkv, M, ld_qkv, H, H_kv, D, cos, sin, ld_cs, cs, q_out, k_dst,
                                                         v_dst, kv_offset, kv_head_stride, g_dev[dev].num_sms, st);
}

extern "C" int lse_rope_kv_write(const void *qkv, int64_t M, int64_t ld_qkv, int64_t H, int64_t H_kv, int64_t D,
                                 const void *cos, const void *sin, int64_t ld_cs, int cs_dtype, void *q_out,
                                 void *k_dst, void *v_dst, const int64_t *kv_offset, int64_t kv_head_stride,
                                 void *stream) {
    return lse_rope_kv_write_dt(qkv, LSE_BF16, M, ld_qkv, H, H_kv, D, cos, sin, ld_cs, cs_dtype, q_out, k_dst, v_dst,
                                kv_offset, kv_head_stride, stream);
}

// ---------------------------------------------------------------------------------------
// lse_rms_norm(_dt): RMSNorm of bf16 or fp16 rows (rms_norm.cuh).
// ---------------------------------------------------------------------------------------
extern "C" int lse_rms_norm_dt(const void *x, int dtype, int64_t M, int64_t N, int64_t ldx, const void *weight,
                               float eps, void *y, int64_t ldy, void *stream) {
    if (M < 0 || N <= 0 || ldx < N || ldy < N || !(eps >= 0.f)) return LSE_ERR_INVALID_ARG;
    if (dtype != LSE_BF16 && dtype != LSE_F16) return LSE_ERR_UNSUPPORTED;
    if (M == 0) return LSE_OK;
    if (!x || !weight || !y) return LSE_ERR_INVALID_ARG;
    if (M > INT32_MAX || N > INT32_MAX) return LSE_ERR_UNSUPPORTED;
    if ((N & 7) || (ldx & 7) || (ldy & 7) || !aligned16(x) || !aligned16(weight) || !aligned16(y))
        return LSE_ERR_ALIGNMENT;
    int dev = 0;
    int rc = current_device(&dev);
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    launch_config(cfg, attr, dim3(static_cast<unsigned>(M)), dim3(norm::THREADS), 0, static_cast<cudaStream_t>(stream));
    cudaError_t e =
        dtype == LSE_F16
            ? cudaLaunchKernelEx(&cfg, norm::rms_norm_kernel<__half>, static_cast<const __half *>(x), ldx,
                                 static_cast<const __half *>(weight), static_cast<int>(N), eps, static_cast<__half *>(y), ldy)
            : cudaLaunchKernelEx(&cfg, norm::rms_norm_kernel<__nv_bfloat16>, static_cast<const __nv_bfloat16 *>(x), ldx,
                                 static_cast<const __nv_bfloat16 *>(weight), static_cast<int>(N), eps,
                                 static_cast<__nv_bfloat16 *>(y), ldy);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) { set_cuda_error(e, "rms_norm launch"); return LSE_ERR_CUDA; }
    return LSE_OK;
}

extern "C" int lse_rms_norm(const void *x, int64_t M, int64_t N, int64_t ldx, const void *weight, float eps, void *y,
                            int64_t ldy, void *stream) {
    return lse_rms_norm_dt(x, LSE_BF16, M, N, ldx, weight, eps, y, ldy, stream);
}

// ---------------------------------------------------------------------------------------
// RMSNorm fused with the projection that consumes it (bf16): the decoder layer's
// q/k/v(input_layernorm(h)) and mlp.gate_up(post_attention_layernorm(h)).  Wherever the
// projection alone would take the decode kernel (lse_int8_linear_packed's and
// lse_int8_gate_up_silu_packed's automatic choice) the normalised rows go through the
// workspace to it; otherwise the digit planes are written straight from the normalisation
// (split::rms_norm_split_kernel) and the separate split launch disappears.
// ---------------------------------------------------------------------------------------
namespace lse {
namespace {
size_t norm_proj_workspace(int64_t M, int64_t K) {
    if (M <= 0 || K < 0) return 0;
    const size_t rows = (static_cast<size_t>(M) * K * 2 + 15) / 16 * 16;  // the normalised rows
    if (M <= 16) return rows;
    // 17..32 tokens take either route, by the weight's size
    return std::max(rows, tci8_workspace_bytes(token_tile(M), digit_planes(M), kMaxGridForWorkspace, M, K));
}

int norm_proj_impl(const void *x, int64_t M, int64_t K, int64_t ldx, const void *norm_w, float eps,
                   const int8_t *w_packed, const float *scale, int64_t N_out, bool silu, void *y, int64_t ldy,
                   void *workspace, size_t workspace_bytes, void *stream) {
    if (M < 0 || N_out < 0 || K < 0 || !(eps >= 0.f)) return LSE_ERR_INVALID_ARG;
    if (M == 0 || N_out == 0) return LSE_OK;
    if (!x || !norm_w || !w_packed || !scale || !y) return LSE_ERR_INVALID_ARG;
    if (ldx < K || ldy < N_out || K == 0) return LSE_ERR_INVALID_ARG;
    if (silu && (N_out % 8)) return LSE_ERR_UNSUPPORTED;
    const int64_t N = silu ? 2 * N_out : N_out;
    if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return LSE_ERR_UNSUPPORTED;
    if ((K & 15) || (ldx & 7) || !aligned16(x) || !aligned16(w_packed) || !aligned16(norm_w)) return LSE_ERR_ALIGNMENT;
    if ((reinterpret_cast<uintptr_t>(y) & 1u) || (reinterpret_cast<uintptr_t>(scale) & 3u)) return LSE_ERR_ALIGNMENT;
    if (!workspace || !aligned16(workspace) || workspace_bytes < norm_proj_workspace(M, K)) return LSE_ERR_WORKSPACE;
    int dev = 0;
    int rc = current_device(&dev);
    if (rc) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (M <= 16 || (!silu && auto_algo(M, K, N, true) == LSE_ALGO_SKINNY)) {
        rc = lse_rms_norm(x, M, K, ldx, norm_w, eps, workspace, K, stream);
        if (rc) return rc;
        return silu ? gate_up_impl(workspace, M, K, K, w_packed, scale, N_out, y, ldy, nullptr, 0, stream, false, true)
                    : linear_impl(workspace, M, K, K, w_packed, scale, N, y, ldy, nullptr, 0, LSE_ALGO_SKINNY, true,
                                  stream);
    }
    const TcPlan pl = plan_tc(M, K, N, g_dev[dev].num_sms, dev);
    if (workspace_bytes < tci8_workspace_bytes(pl.nt, digit_planes(M), pl.grid, M, K)) return LSE_ERR_WORKSPACE;
    return silu ? run_tc_i8<true>(pl, x, M, K, ldx, w_packed, scale, N, y, ldy, nullptr, 0, workspace, true, st, false,
                                  norm_w, eps)
                : run_tc_i8<false>(pl, x, M, K, ldx, w_packed, scale, N, y, ldy, nullptr, 0, workspace, true, st,
                                   false, norm_w, eps);
}
}  // namespace
}  // namespace lse

extern "C" size_t lse_int8_rms_norm_proj_workspace(int64_t M, int64_t K) { return norm_proj_workspace(M, K); }

extern "C" int lse_int8_rms_norm_linear_packed(const void *x, int64_t M, int64_t K, int64_t ldx, const void *norm_weight,
                                               float eps, const int8_t *w_packed, const float *scale, int64_t N, void *y,
                                               int64_t ldy, void *workspace, size_t workspace_bytes, void *stream) {
    return norm_proj_impl(x, M, K, ldx, norm_weight, eps, w_packed, scale, N, false, y, ldy, workspace,
                          workspace_bytes, stream);
}

extern "C" int lse_int8_rms_norm_gate_up_silu_packed(const void *x, int64_t M, int64_t K, int64_t ldx,
                                                     const void *norm_weight, float eps, const int8_t *w_packed,
                                                     const float *scale, int64_t I, void *y, int64_t ldy,
                                                     void *workspace, size_t workspace_bytes, void *stream) {
    return norm_proj_impl(x, M, K, ldx, norm_weight, eps, w_packed, scale, I, true, y, ldy, workspace,
                          workspace_bytes, stream);
}
