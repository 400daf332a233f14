// libdotl: host side of the C ABI declared in include/dotl.h.
//
// One translation unit: the kernel headers are included here so the device
// error word has a single definition and nvcc sees every launcher with its
// kernel. Argument checks mirror the reference's TORCH_CHECKs
// (attention_dispatch.cuh:351-369, linear_gelu.cuh:606-625,
// add_layernorm.cuh:500-552): a rejected call returns a code and a message
// and enqueues nothing. Nothing on the forward path allocates device memory;
// only the peer-memory setup calls (dotl_peer_alloc, dotl_ipc_open) do.

#include "../../include/dotl.h"
#include "attention.cuh"
#include "attn_generic.cuh"
#include "gemm.cuh"
#include "gemm_ln.cuh"
#include "ffn.cuh"
#include "layernorm.cuh"
#include "peer_ln.cuh"

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <algorithm>
#include <atomic>
#include <utility>

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int check_launch(const char* who) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(DOTL_ECUDA, "%s: kernel launch failed: %s", who, cudaGetErrorString(e));
    return DOTL_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int current_device(int* dev) {
    const cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) return fail(DOTL_ECUDA, "cudaGetDevice failed: %s", cudaGetErrorString(e));
    return DOTL_OK;
}

constexpr int kMaxDevices = 64;

// Per-device caches below are filled on first use from whichever host thread
// gets there first. They hold atomics: two threads may both miss and both
// fill an entry (each writes the same value; the CUDA calls behind them are
// idempotent), but no thread reads a torn or racy value.
using DeviceFlags = std::atomic<bool>[kMaxDevices];

int sm_count(int dev) {
    static std::atomic<int> counts[kMaxDevices];
    if (dev < 0 || dev >= kMaxDevices) return 148;
    int n = counts[dev].load(std::memory_order_relaxed);
    if (n == 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        counts[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

// Raises a kernel's dynamic shared memory limit, once per device.
template <typename Kernel>
int ensure_smem(Kernel kernel, uint32_t bytes, int dev, DeviceFlags& done_flags) {
    if (dev >= 0 && dev < kMaxDevices && done_flags[dev].load(std::memory_order_acquire)) return DOTL_OK;
    const cudaError_t e =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
    if (e != cudaSuccess)
        return fail(DOTL_ECUDA, "cudaFuncSetAttribute(%u bytes of shared memory) failed: %s", bytes,
                    cudaGetErrorString(e));
    if (dev >= 0 && dev < kMaxDevices) done_flags[dev].store(true, std::memory_order_release);
    return DOTL_OK;
}

// Kernels that move registers between warpgroups (setmaxnreg) need their
// launch to grant at least `needed` registers in total; a raise that the
// launch cannot cover would wait forever, so such a build refuses to launch.
template <typename Kernel>
int check_regs(Kernel kernel, int threads, int needed, DeviceFlags& done_flags, int dev, const char* who) {
    if (dev >= 0 && dev < kMaxDevices && done_flags[dev].load(std::memory_order_acquire)) return DOTL_OK;
    cudaFuncAttributes fa;
    const cudaError_t e = cudaFuncGetAttributes(&fa, kernel);
    if (e != cudaSuccess) return fail(DOTL_ECUDA, "%s: cudaFuncGetAttributes failed: %s", who, cudaGetErrorString(e));
    if (fa.numRegs * threads < needed)
        return fail(DOTL_EUNSUPPORTED, "%s: kernel built with %d registers per thread, its warpgroup split needs %d in total",
                    who, fa.numRegs, needed);
    if (dev >= 0 && dev < kMaxDevices) done_flags[dev].store(true, std::memory_order_release);
    return DOTL_OK;
}

// Launches with programmatic stream serialization, so the kernel's prologue
// can overlap the previous kernel's tail (each kernel starts with
// griddepcontrol.wait before it touches its inputs).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ------------------------------------------------------------ tensor maps --

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// fp16 tensor map of rank 2 or 4 with a 128-row box (box_rows) and
// box_cols fp16 columns, swizzled to the box row width.
int encode_f16_map(CUtensorMap* map, const void* base, int rank, const cuuint64_t* dims,
                   const cuuint64_t* strides_bytes, uint32_t box_cols, uint32_t box_rows, const char* who) {
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return fail(DOTL_ECUDA, "%s: cuTensorMapEncodeTiled is unavailable from the driver", who);
    cuuint32_t box[4] = {box_cols, box_rows, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUtensorMapSwizzle swz = box_cols * 2 == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                   : box_cols * 2 == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                        : CU_TENSOR_MAP_SWIZZLE_32B;
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, static_cast<cuuint32_t>(rank),
                          const_cast<void*>(base), dims, strides_bytes, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(DOTL_ECUDA, "%s: cuTensorMapEncodeTiled failed (CUresult %d)", who, (int)r);
    return DOTL_OK;
}

// ------------------------------------------------------------------ GEMM --

template <int BN, int STAGES, bool OUT_F16, bool SPLIT2 = false, bool PEER = false, bool PAIR = false>
int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& to, const CUtensorMap& tr,
                const dotl::GemmParams& p, int dev, cudaStream_t stream, const dotl::GemmPeerOut* po_in = nullptr) {
    using L = dotl::GemmSmem<BN, STAGES, PAIR ? BN / 2 : BN>;
    auto kernel = dotl::gemm_tc_kernel<BN, STAGES, OUT_F16, SPLIT2, PEER, PAIR>;
    static const dotl::GemmPeerOut kNoPeers = {};
    const dotl::GemmPeerOut& po = po_in != nullptr ? *po_in : kNoPeers;
    static DeviceFlags done;
    if (int rc = ensure_smem(kernel, L::kAlloc, dev, done)) return rc;
    const int tiles = p.num_m_tiles * p.num_n_tiles;
    cudaError_t e;
    if constexpr (SPLIT2 || PAIR) {
        // split-K: one cluster of two CTAs per tile (the exchange buffer reuses
        // the stage ring, so no CTA may own a second tile); pair: persistent
        // clusters of two, at most one CTA per SM
        const int pairs = PAIR ? (tiles < sm_count(dev) / 2 ? tiles : sm_count(dev) / 2) : tiles;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
        cfg.blockDim = dim3(dotl::kGemmThreads);
        cfg.dynamicSmemBytes = L::kAlloc;
        cfg.stream = stream;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = 2;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 2;
        e = cudaLaunchKernelEx(&cfg, kernel, ta, tw, to, tr, p, po);
    } else {
        const int grid = tiles < sm_count(dev) ? tiles : sm_count(dev);
        e = launch_pdl(kernel, dim3(grid), dim3(dotl::kGemmThreads), L::kAlloc, stream, ta, tw, to, tr, p, po);
    }
    if (e != cudaSuccess) return fail(DOTL_ECUDA, "dotl_linear: launch failed: %s", cudaGetErrorString(e));
    return check_launch("dotl_linear");
}

// N tile for an [M,N,K] problem.
int pick_tile_n(int64_t M, int64_t N, int64_t K, int sms) {
    // The widest tile that still gives most SMs a tile: wide tiles read each
    // operand byte into fewer CTAs (A is read once per N tile, W once per M
    // tile), narrow ones only pay off when wide ones would leave SMs idle.
    // Measured on B200 over the five BASELINE configs' GEMMs.
    (void)K;
    const int64_t mt = (M + dotl::kGemmBM - 1) / dotl::kGemmBM;
    for (int bn : {256, 128}) {
        const int64_t tiles = mt * ((N + bn - 1) / bn);
        if (tiles * 5 >= static_cast<int64_t>(sms) * 3) return bn;
    }
    return 64;
}

// A [rows, cols] fp32 or fp16 output written by 32 x 32 TMA store boxes (128 B
// fp32 rows with 128B swizzle, 64 B fp16 rows with 64B swizzle).
int encode_out_map(CUtensorMap* map, void* base, int64_t rows, int64_t cols, int64_t ld, int dtype, const char* who) {
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return fail(DOTL_ECUDA, "%s: cuTensorMapEncodeTiled is unavailable from the driver", who);
    const cuuint64_t odims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t ostr[1] = {static_cast<cuuint64_t>(ld) * (dtype == DOTL_F16 ? 2 : 4)};
    const cuuint32_t obox[2] = {32u, 32u};
    const cuuint32_t oes[2] = {1, 1};
    const CUresult r = fn(map, dtype == DOTL_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                          base, odims, ostr, obox, oes, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          dtype == DOTL_F16 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(DOTL_ECUDA, "%s: cuTensorMapEncodeTiled (output) failed (CUresult %d)", who, (int)r);
    return DOTL_OK;
}

// ------------------------------------------------- GEMM + LayerNorm epilogue --

// Clusters of `cs` CTAs of this kernel that fit on the device at once.
template <typename Kernel>
int max_clusters(Kernel kernel, int cs, uint32_t smem, int* out) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(cs));
    cfg.blockDim = dim3(dotl::kGemmThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(cs);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    const cudaError_t e = cudaOccupancyMaxActiveClusters(&n, kernel, &cfg);
    if (e != cudaSuccess || n <= 0)
        return fail(DOTL_ECUDA, "cudaOccupancyMaxActiveClusters(cluster %d) failed: %s", cs,
                    e != cudaSuccess ? cudaGetErrorString(e) : "no cluster fits");
    *out = n;
    return DOTL_OK;
}

template <int BN, int STAGES, bool NORM_F16>
int launch_gemm_ln(const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& tx, const CUtensorMap& tn,
                   const CUtensorMap& tr, const CUtensorMap& tnl, const dotl::GemmLnParams& p, int dev,
                   cudaStream_t stream) {
    using L = dotl::GemmLnSmem<BN, STAGES>;
    auto kernel = dotl::gemm_ln_kernel<BN, STAGES, NORM_F16>;
    static DeviceFlags done;
    static std::atomic<int> fit[kMaxDevices][dotl::kLnMaxCluster + 1];
    if (int rc = ensure_smem(kernel, L::kAlloc, dev, done)) return rc;
    int clusters = (dev >= 0 && dev < kMaxDevices) ? fit[dev][p.cs].load(std::memory_order_relaxed) : 0;
    if (clusters == 0) {
        if (int rc = max_clusters(kernel, p.cs, L::kAlloc, &clusters)) return rc;
        if (dev >= 0 && dev < kMaxDevices) fit[dev][p.cs].store(clusters, std::memory_order_relaxed);
    }
    if (clusters > p.num_m_tiles) clusters = p.num_m_tiles;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(clusters * p.cs));
    cfg.blockDim = dim3(dotl::kGemmThreads);
    cfg.dynamicSmemBytes = L::kAlloc;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = static_cast<unsigned>(p.cs);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, ta, tw, tx, tn, tr, tnl, p);
    if (e != cudaSuccess) return fail(DOTL_ECUDA, "dotl_linear_ln: launch failed: %s", cudaGetErrorString(e));
    return check_launch("dotl_linear_ln");
}

// N tile for the LayerNorm epilogue: N = cs * BN with cs <= 8; the widest
// tile that still gives most SMs work, else the narrowest (most CTAs).
int pick_tile_n_ln(int64_t M, int64_t N, int sms) {
    const int64_t mt = (M + dotl::kGemmBM - 1) / dotl::kGemmBM;
    int narrowest = 0;
    for (int bn : {256, 128, 64}) {
        if (N % bn != 0 || N / bn > dotl::kLnMaxCluster) continue;
        if (mt * (N / bn) * 5 >= static_cast<int64_t>(sms) * 3) return bn;
        narrowest = bn;
    }
    return narrowest;
}

// ------------------------------------------------------------- attention --

// single: every item has one key tile (the host's test in dotl_attention).
template <int HD, int STAGES>
int launch_attn(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const dotl::AttnParams& p,
                bool single, int dev, cudaStream_t stream) {
    using L = dotl::AttnSmem<HD, STAGES>;
    const int items = p.num_streams * p.num_q_tiles * p.splits;
    const int grid = items < sm_count(dev) ? items : sm_count(dev);
    // The overlapped order only pays when a CTA has a next item; with one
    // item per CTA the plain kernel (smaller code) runs.
    const bool overlap = single && items > grid;
    auto kernel = overlap ? dotl::attn_tc_kernel<HD, STAGES, true> : dotl::attn_tc_kernel<HD, STAGES, false>;
    static DeviceFlags done[2];
    static DeviceFlags regs_ok[2];
    if (int rc = ensure_smem(kernel, L::kAlloc, dev, done[overlap])) return rc;
    if (int rc = check_regs(kernel, dotl::kAttnThreads, dotl::kAttnRegSplit, regs_ok[overlap], dev, "dotl_attention"))
        return rc;
    cudaError_t e = launch_pdl(kernel, dim3(grid), dim3(dotl::kAttnThreads), L::kAlloc, stream, tq, tk, tv, p);
    if (e != cudaSuccess) return fail(DOTL_ECUDA, "dotl_attention: launch failed: %s", cudaGetErrorString(e));
    if (p.splits > 1) {
        // fold each query tile's key runs (workspace -> out)
        const int64_t rows = static_cast<int64_t>(p.num_streams) * p.num_q_tiles * dotl::kAttnTile;
        const dim3 cgrid(static_cast<unsigned>((rows + dotl::kCombineWarps - 1) / dotl::kCombineWarps));
        e = launch_pdl(dotl::attn_combine_kernel<HD>, cgrid, dim3(dotl::kCombineWarps * 32), 0, stream, p);
        if (e != cudaSuccess) return fail(DOTL_ECUDA, "dotl_attention: combine launch failed: %s", cudaGetErrorString(e));
    }
    return check_launch("dotl_attention");
}

// Split-KV plan for the tcgen05 attention: key runs per query tile and key
// tiles per run. Each work item pays a fixed cost (its Q tile, the pipeline
// fill, the epilogue) and the runs a combine pass, which measured on B200 as
// a loss whenever the items already came near the SM count (config 2's 128
// items of at most 4 key tiles: 10.3 -> 19.8 us; 128 items of 32 key tiles:
// 44 -> 65 us). So split only when the items fill at most a quarter of the
// SMs and a tile sees at least 8 key tiles, in runs of at least 4 key tiles
// (about one SM's fair share of all key tiles when that is more).
int attn_split_plan(int streams, int q_tiles, int max_kt, bool causal, int sms, int* kt_per_split) {
    *kt_per_split = max_kt;
    const int64_t items = static_cast<int64_t>(streams) * q_tiles;
    if (items * 4 > sms || max_kt < 8) return 1;
    const int64_t total_kt = causal ? static_cast<int64_t>(streams) * q_tiles * (q_tiles + 1) / 2
                                    : items * max_kt;
    int64_t kt = (total_kt + sms - 1) / sms;
    if (kt < 4) kt = 4;
    const int splits = static_cast<int>((max_kt + kt - 1) / kt);
    if (splits < 2) return 1;
    *kt_per_split = static_cast<int>(kt);
    return splits;
}

// Workspace of a split-KV plan: per slot, 128 rows of head_dim fp32 values
// and a (max, sum) pair.
int64_t attn_split_bytes(int streams, int q_tiles, int splits, int head_dim) {
    return static_cast<int64_t>(streams) * q_tiles * splits * dotl::kAttnTile * (head_dim * 4 + 8);
}

// ------------------------------------------------------------- fused MLP --

template <int D, bool NF16>
int launch_ffn(const CUtensorMap& ta, const CUtensorMap& tw1, const CUtensorMap& tw2, const CUtensorMap& tr,
               const CUtensorMap& tx, const CUtensorMap& tn, const dotl::FfnParams& p, int dev, cudaStream_t stream) {
    using L = dotl::FfnSmem<D>;
    auto kernel = dotl::ffn_kernel<D, NF16>;
    static DeviceFlags done;
    if (int rc = ensure_smem(kernel, L::kAlloc, dev, done)) return rc;
    const int grid = p.num_m_tiles < sm_count(dev) ? p.num_m_tiles : sm_count(dev);
    const cudaError_t e =
        launch_pdl(kernel, dim3(grid), dim3(dotl::kFfnThreads), L::kAlloc, stream, ta, tw1, tw2, tr, tx, tn, p);
    if (e != cudaSuccess) return fail(DOTL_ECUDA, "dotl_ffn: launch failed: %s", cudaGetErrorString(e));
    return check_launch("dotl_ffn");
}

}  // namespace

extern "C" {

int dotl_abi_version(void) { return DOTL_ABI_VERSION; }

const char* dotl_last_error(void) { return g_last_error.c_str(); }

int dotl_num_sms(int* out) {
    if (out == nullptr) return fail(DOTL_EINVAL, "dotl_num_sms: out is NULL");
    int dev;
    if (int rc = current_device(&dev)) return rc;
    *out = sm_count(dev);
    return DOTL_OK;
}

int dotl_device_error(int clear, unsigned int* word) {
    unsigned int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, dotl::g_dotl_dev_error, sizeof(v));
    if (e != cudaSuccess) return fail(DOTL_ECUDA, "dotl_device_error: %s", cudaGetErrorString(e));
    if (clear) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbol(dotl::g_dotl_dev_error, &zero, sizeof(zero));
        if (e != cudaSuccess) return fail(DOTL_ECUDA, "dotl_device_error: %s", cudaGetErrorString(e));
    }
    if (word != nullptr) *word = v;
    return DOTL_OK;
}

int dotl_identity_f32(const float* in, float* out, int64_t n, void* stream) {
    if (n < 0) return fail(DOTL_EINVAL, "smoke_test_identity: negative size");
    if (n == 0) return DOTL_OK;
    if (in == nullptr || out == nullptr) return fail(DOTL_EINVAL, "smoke_test_identity: NULL pointer");
    const int threads = 256;
    const int64_t blocks = (n + threads - 1) / threads;
    dotl::identity_f32_kernel<<<static_cast<unsigned>(blocks), threads, 0, static_cast<cudaStream_t>(stream)>>>(
        in, out, n);
    return check_launch("smoke_test_identity");
}

int dotl_cast_f32_f16(const float* in, void* out, int64_t n, void* stream) {
    if (n < 0) return fail(DOTL_EINVAL, "dotl_cast_f32_f16: negative size");
    if (n == 0) return DOTL_OK;
    if (in == nullptr || out == nullptr) return fail(DOTL_EINVAL, "dotl_cast_f32_f16: NULL pointer");
    if (!aligned16(in) || !aligned16(out))
        return fail(DOTL_EINVAL, "dotl_cast_f32_f16: pointers must be 16-byte aligned");
    const int threads = 256;
    const int64_t blocks = ((n + 3) / 4 + threads - 1) / threads;
    dotl::cast_f32_f16_kernel<<<static_cast<unsigned>(blocks), threads, 0, static_cast<cudaStream_t>(stream)>>>(
        in, static_cast<__half*>(out), n);
    return check_launch("dotl_cast_f32_f16");
}

int dotl_cast_f16_f32(const void* in, float* out, int64_t n, void* stream) {
    if (n < 0) return fail(DOTL_EINVAL, "dotl_cast_f16_f32: negative size");
    if (n == 0) return DOTL_OK;
    if (in == nullptr || out == nullptr) return fail(DOTL_EINVAL, "dotl_cast_f16_f32: NULL pointer");
    const int threads = 256;
    const int64_t blocks = (n + threads - 1) / threads;
    dotl::cast_f16_f32_kernel<<<static_cast<unsigned>(blocks), threads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __half*>(in), out, n);
    return check_launch("dotl_cast_f16_f32");
}

int dotl_layernorm(const float* x, const float* sub, const float* weight, const float* bias, float* x_new,
                   void* normed, int normed_dtype, const uint8_t* row_valid, int64_t rows, int64_t D, float eps,
                   void* stream) {
    const char* who = sub ? "fused_add_layernorm" : "fused_layernorm";
    if (rows < 0 || D <= 0) return fail(DOTL_EINVAL, "%s: bad shape rows=%lld D=%lld", who, (long long)rows, (long long)D);
    if (D > 2048) return fail(DOTL_EUNSUPPORTED, "%s: last dimension %lld is over the 2048 this kernel holds in registers", who, (long long)D);
    if (normed_dtype != DOTL_F32 && normed_dtype != DOTL_F16 && normed_dtype != DOTL_F16X2)
        return fail(DOTL_EINVAL, "%s: normed dtype must be DOTL_F32, DOTL_F16 or DOTL_F16X2", who);
    if (rows == 0) return DOTL_OK;
    if (x == nullptr || weight == nullptr || bias == nullptr || normed == nullptr)
        return fail(DOTL_EINVAL, "%s: NULL pointer", who);
    // DOTL_F16X2: the lo plane follows the hi plane ([rows, D] each)
    const int64_t lo_plane = normed_dtype == DOTL_F16X2 ? rows * D : 0;
    if (sub != nullptr && x_new == nullptr) return fail(DOTL_EINVAL, "%s: sub given without x_new", who);
    const bool vec = (D % 128 == 0) && aligned16(x) && aligned16(weight) && aligned16(bias) && aligned16(normed) &&
                     (sub == nullptr || (aligned16(sub) && aligned16(x_new)));
    const int64_t blocks = (rows + dotl::kLnWarpsPerBlock - 1) / dotl::kLnWarpsPerBlock;
    const dim3 grid(static_cast<unsigned>(blocks));
    const dim3 block(dotl::kLnWarpsPerBlock * 32);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int Di = static_cast<int>(D);

    cudaError_t le = cudaSuccess;
#define DOTL_LN(EPL, VEC)                                                                                      \
    do {                                                                                                       \
        if (normed_dtype != DOTL_F32)                                                                          \
            le = launch_pdl(dotl::ln_rows_kernel<EPL, VEC, __half>, grid, block, 0, s, x, sub, weight, bias,  \
                            x_new, static_cast<__half*>(normed), row_valid, rows, Di, eps, lo_plane);          \
        else                                                                                                   \
            le = launch_pdl(dotl::ln_rows_kernel<EPL, VEC, float>, grid, block, 0, s, x, sub, weight, bias,   \
                            x_new, static_cast<float*>(normed), row_valid, rows, Di, eps, int64_t{0});         \
    } while (0)

    if (vec) {
        if (D <= 128) DOTL_LN(4, true);
        else if (D <= 256) DOTL_LN(8, true);
        else if (D <= 512) DOTL_LN(16, true);
        else if (D <= 1024) DOTL_LN(32, true);
        else DOTL_LN(64, true);
    } else {
        if (D <= 32) DOTL_LN(1, false);
        else if (D <= 64) DOTL_LN(2, false);
        else if (D <= 128) DOTL_LN(4, false);
        else if (D <= 256) DOTL_LN(8, false);
        else if (D <= 512) DOTL_LN(16, false);
        else if (D <= 1024) DOTL_LN(32, false);
        else DOTL_LN(64, false);
    }
#undef DOTL_LN
    if (le != cudaSuccess) return fail(DOTL_ECUDA, "%s: launch failed: %s", who, cudaGetErrorString(le));
    return check_launch(who);
}

int dotl_linear(const void* a, int64_t M, int64_t K, int64_t lda, const void* w, int64_t N, int64_t ldw,
                const float* bias, int act, const float* resid, int64_t ldr, const uint8_t* row_valid, int resid_mode,
                void* out, int out_dtype, int64_t ldo, int tile_n, int operands, void* stream) {
    const char* who = act ? "linear_gelu" : "linear_bias";
    if (M < 0 || N <= 0 || K <= 0) return fail(DOTL_EINVAL, "%s: bad shape M=%lld N=%lld K=%lld", who, (long long)M, (long long)N, (long long)K);
    if (M > (int64_t)0x7fffffff - 256 || N > 0x7fffffff || K > 0x7fffffff)
        return fail(DOTL_EUNSUPPORTED, "%s: dimensions must fit in 31 bits", who);
    if (act != 0 && act != 1) return fail(DOTL_EINVAL, "%s: act must be 0 (none) or 1 (GELU)", who);
    if (resid_mode < DOTL_RESID_NONE || resid_mode > DOTL_MASK_ROWS)
        return fail(DOTL_EINVAL, "%s: unknown residual mode %d", who, resid_mode);
    if (out_dtype != DOTL_F32 && out_dtype != DOTL_F16 && out_dtype != DOTL_F16X2)
        return fail(DOTL_EINVAL, "%s: out dtype must be DOTL_F32, DOTL_F16 or DOTL_F16X2", who);
    if (operands != DOTL_F16 && operands != DOTL_F16X2)
        return fail(DOTL_EINVAL, "%s: operands must be DOTL_F16 or DOTL_F16X2", who);
    const bool x3 = operands == DOTL_F16X2;
    if (M == 0) return DOTL_OK;
    if (a == nullptr || w == nullptr || bias == nullptr || out == nullptr) return fail(DOTL_EINVAL, "%s: NULL pointer", who);
    if (K % 8 != 0 || lda % 8 != 0 || ldw % 8 != 0 || lda < K || ldw < K)
        return fail(DOTL_EUNSUPPORTED, "%s: K, lda and ldw must be multiples of 8 (16-byte fp16 rows for TMA), got K=%lld lda=%lld ldw=%lld", who, (long long)K, (long long)lda, (long long)ldw);
    if (!aligned16(a) || !aligned16(w)) return fail(DOTL_EUNSUPPORTED, "%s: a and w must be 16-byte aligned", who);
    if (N % 8 != 0) return fail(DOTL_EUNSUPPORTED, "%s: N=%lld must be a multiple of 8", who, (long long)N);
    if (ldo < N || !aligned16(out) || ldo % 8 != 0) return fail(DOTL_EUNSUPPORTED, "%s: out must be 16-byte aligned with ldo >= N, ldo %% 8 == 0", who);
    if (resid_mode != DOTL_RESID_NONE && resid_mode != DOTL_MASK_ROWS) {
        if (resid == nullptr) return fail(DOTL_EINVAL, "%s: residual mode %d needs resid", who, resid_mode);
        if (!aligned16(resid) || ldr % 4 != 0 || ldr < N) return fail(DOTL_EUNSUPPORTED, "%s: resid must be 16-byte aligned with ldr >= N, ldr %% 4 == 0", who);
    }
    if ((resid_mode == DOTL_RESID_ADD_MASKSUB || resid_mode == DOTL_RESID_ADD_MASKALL || resid_mode == DOTL_MASK_ROWS) &&
        row_valid == nullptr)
        return fail(DOTL_EINVAL, "%s: masked residual mode needs row_valid", who);
    if (!aligned16(bias)) return fail(DOTL_EUNSUPPORTED, "%s: bias must be 16-byte aligned", who);
    if (resid_mode != DOTL_RESID_NONE && resid_mode != DOTL_MASK_ROWS && out_dtype != DOTL_F32)
        return fail(DOTL_EUNSUPPORTED, "%s: residual epilogues write the fp32 residual stream (out dtype DOTL_F32)", who);

    int dev;
    if (int rc = current_device(&dev)) return rc;
    // the k loop's length; the three-product mode runs three passes of K
    const int64_t nkb = (x3 ? 3 : 1) * ((K + dotl::kGemmBK - 1) / dotl::kGemmBK);
    const int64_t mt = (M + dotl::kGemmBM - 1) / dotl::kGemmBM;
    int bn = tile_n;
    bool split2 = false, pair = false;
    if (bn == -256) {
        // CTA pairs on 256 x 256 tiles (M = 256 MMAs over two SMs)
        bn = 256;
        pair = true;
    } else if (bn == 0) {
        bn = pick_tile_n(M, N, K, sm_count(dev));
        // Too few tiles for the SMs even at width 64, and a long K: split K
        // between the two CTAs of a cluster at width 128 instead (each CTA
        // streams half the k-blocks of a tile twice as wide).
        // (below ~24 k-blocks the pair's exchange costs more than it saves)
        if (bn == 64 && nkb >= 24 && 2 * mt * ((N + 127) / 128) <= sm_count(dev)) {
            bn = 128;
            split2 = true;
        }
        // Large fp32 residual-stream GEMMs (out_proj, ffn_out of a wide layer)
        // on CTA pairs: measured on B200 (interleaved medians, L2 flushed) at
        // M=16384 N=2048: K=8192 450 -> 405 us, K=2048 124 -> 116 us, same
        // bits; fp16-output GEMMs and shapes with fewer than four pair tiles
        // per CTA pair gained nothing or lost (up to 16 %).
        const bool resid_out = out_dtype == DOTL_F32 && resid_mode != DOTL_RESID_NONE && resid_mode != DOTL_MASK_ROWS;
        const int64_t pair_tiles = ((M + 2 * dotl::kGemmBM - 1) / (2 * dotl::kGemmBM)) * (N / 256);
        if (bn == 256 && resid_out && N >= 2048 && N % 256 == 0 && K >= 2048 &&
            pair_tiles >= 4 * static_cast<int64_t>(sm_count(dev) / 2)) {
            pair = true;
        }
    } else if (bn == -128) {
        if (nkb < 2) return fail(DOTL_EINVAL, "%s: split-K needs at least two k-blocks (K > 64)", who);
        bn = 128;
        split2 = true;
    }
    if (bn != 64 && bn != 128 && bn != 160 && bn != 192 && bn != 224 && bn != 256)
        return fail(DOTL_EINVAL,
                    "%s: tile_n must be 0, 64, 128, 160, 192, 224, 256, -128 (split K) or -256 (CTA pairs)", who);

    // DOTL_F16X2 operands: one map over both planes of each (lo rows below hi)
    CUtensorMap ta, tw;
    const cuuint64_t adims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(x3 ? 2 * M : M)};
    const cuuint64_t astr[1] = {static_cast<cuuint64_t>(lda) * 2};
    if (int rc = encode_f16_map(&ta, a, 2, adims, astr, dotl::kGemmBK, dotl::kGemmBM, who)) return rc;
    const cuuint64_t wdims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(x3 ? 2 * N : N)};
    const cuuint64_t wstr[1] = {static_cast<cuuint64_t>(ldw) * 2};
    if (int rc = encode_f16_map(&tw, w, 2, wdims, wstr, dotl::kGemmBK, static_cast<uint32_t>(pair ? bn / 2 : bn), who))
        return rc;
    CUtensorMap to;
    const int store_dtype = out_dtype == DOTL_F16X2 ? DOTL_F16 : out_dtype;
    if (int rc = encode_out_map(&to, out, M, N, ldo, store_dtype, who)) return rc;
    // the residual in as 32 x 32 fp32 blocks (fp32 out); without one the map is unused
    CUtensorMap tr = to;
    if (resid_mode != DOTL_RESID_NONE && resid_mode != DOTL_MASK_ROWS)
        if (int rc = encode_out_map(&tr, const_cast<float*>(resid), M, N, ldr, DOTL_F32, who)) return rc;
    // DOTL_F16X2 out: the lo plane, M rows of ldo below the hi plane
    dotl::GemmPeerOut lo_out = {};
    if (out_dtype == DOTL_F16X2)
        if (int rc = encode_out_map(&lo_out.map[0], static_cast<__half*>(out) + M * ldo, M, N, ldo, DOTL_F16, who))
            return rc;

    dotl::GemmParams p;
    p.M = static_cast<int>(M);
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(K);
    p.num_m_tiles = static_cast<int>((M + (pair ? 2 : 1) * dotl::kGemmBM - 1) / ((pair ? 2 : 1) * dotl::kGemmBM));
    p.num_n_tiles = static_cast<int>((N + bn - 1) / bn);
    p.bias = bias;
    p.resid = resid;
    p.ldr = ldr;
    p.row_valid = row_valid;
    p.resid_mode = resid_mode;
    p.act = act;
    p.out = out;
    p.ldo = ldo;
    p.x3_nkb = x3 ? static_cast<int>((K + dotl::kGemmBK - 1) / dotl::kGemmBK) : 0;
    p.a_lo_row = x3 ? static_cast<int>(M) : 0;
    p.w_lo_row = x3 ? static_cast<int>(N) : 0;
    p.out_lo = out_dtype == DOTL_F16X2 ? 1 : 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool f16 = store_dtype == DOTL_F16;
    const dotl::GemmPeerOut* po = &lo_out;
    if (pair)
        return f16 ? launch_gemm<256, 6, true, false, false, true>(ta, tw, to, tr, p, dev, s, po)
                   : launch_gemm<256, 6, false, false, false, true>(ta, tw, to, tr, p, dev, s, po);
    if (split2)
        return f16 ? launch_gemm<128, 5, true, true>(ta, tw, to, tr, p, dev, s, po)
                   : launch_gemm<128, 5, false, true>(ta, tw, to, tr, p, dev, s, po);
    if (bn == 256)
        return f16 ? launch_gemm<256, 4, true>(ta, tw, to, tr, p, dev, s, po)
                   : launch_gemm<256, 4, false>(ta, tw, to, tr, p, dev, s, po);
    if (bn == 224)
        return f16 ? launch_gemm<224, 4, true>(ta, tw, to, tr, p, dev, s, po)
                   : launch_gemm<224, 4, false>(ta, tw, to, tr, p, dev, s, po);
    if (bn == 192)
        return f16 ? launch_gemm<192, 4, true>(ta, tw, to, tr, p, dev, s, po)
                   : launch_gemm<192, 4, false>(ta, tw, to, tr, p, dev, s, po);
    if (bn == 160)
        return f16 ? launch_gemm<160, 5, true>(ta, tw, to, tr, p, dev, s, po)
                   : launch_gemm<160, 5, false>(ta, tw, to, tr, p, dev, s, po);
    if (bn == 64)
        return f16 ? launch_gemm<64, 7, true>(ta, tw, to, tr, p, dev, s, po)
                   : launch_gemm<64, 7, false>(ta, tw, to, tr, p, dev, s, po);
    return f16 ? launch_gemm<128, 5, true>(ta, tw, to, tr, p, dev, s, po)
               : launch_gemm<128, 5, false>(ta, tw, to, tr, p, dev, s, po);
}

int dotl_linear_peer(const void* a, int64_t M, int64_t K, int64_t lda, const void* w, int64_t N, int64_t ldw,
                     const float* bias, int world, void* const* outs, int64_t rows_per_rank, int64_t ldo,
                     void* stream) {
    const char* who = "dotl_linear_peer";
    if (world < 1 || world > dotl::kGemmPeerMax) return fail(DOTL_EINVAL, "%s: world %d outside 1..%d", who, world, dotl::kGemmPeerMax);
    if (M < 0 || N <= 0 || K <= 0 || M > (int64_t)0x7fffffff - 256 || N > 0x7fffffff || K > 0x7fffffff)
        return fail(DOTL_EINVAL, "%s: bad shape M=%lld N=%lld K=%lld", who, (long long)M, (long long)N, (long long)K);
    if (rows_per_rank <= 0 || rows_per_rank % dotl::kGemmBM != 0 || M != rows_per_rank * world)
        return fail(DOTL_EUNSUPPORTED, "%s: M=%lld must be world x rows_per_rank with rows_per_rank a multiple of 128",
                    who, (long long)M);
    if (a == nullptr || w == nullptr || outs == nullptr) return fail(DOTL_EINVAL, "%s: NULL pointer", who);
    if (K % 8 != 0 || lda % 8 != 0 || ldw % 8 != 0 || lda < K || ldw < K)
        return fail(DOTL_EUNSUPPORTED, "%s: K, lda and ldw must be multiples of 8", who);
    if (!aligned16(a) || !aligned16(w) || !aligned16(bias)) return fail(DOTL_EUNSUPPORTED, "%s: a, w and bias must be 16-byte aligned", who);
    if (N % 8 != 0 || ldo < N || ldo % 4 != 0) return fail(DOTL_EUNSUPPORTED, "%s: N %% 8 == 0 and ldo >= N, ldo %% 4 == 0", who);
    dotl::GemmPeerOut po = {};
    po.rows = static_cast<int>(rows_per_rank);
    for (int r = 0; r < world; ++r) {
        if (outs[r] == nullptr || !aligned16(outs[r])) return fail(DOTL_EINVAL, "%s: outs[%d] NULL or unaligned", who, r);
        if (int rc = encode_out_map(&po.map[r], outs[r], rows_per_rank, N, ldo, DOTL_F32, who)) return rc;
    }
    int dev;
    if (int rc = current_device(&dev)) return rc;
    const int bn = pick_tile_n(M, N, K, sm_count(dev));
    CUtensorMap ta, tw;
    const cuuint64_t adims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
    const cuuint64_t astr[1] = {static_cast<cuuint64_t>(lda) * 2};
    if (int rc = encode_f16_map(&ta, a, 2, adims, astr, dotl::kGemmBK, dotl::kGemmBM, who)) return rc;
    const cuuint64_t wdims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(N)};
    const cuuint64_t wstr[1] = {static_cast<cuuint64_t>(ldw) * 2};
    if (int rc = encode_f16_map(&tw, w, 2, wdims, wstr, dotl::kGemmBK, static_cast<uint32_t>(bn), who)) return rc;
    dotl::GemmParams p = {};
    p.M = static_cast<int>(M);
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(K);
    p.num_m_tiles = static_cast<int>(M / dotl::kGemmBM);
    p.num_n_tiles = static_cast<int>((N + bn - 1) / bn);
    p.bias = bias;
    p.resid_mode = DOTL_RESID_NONE;
    p.act = 0;
    p.out = outs[0];
    p.ldo = ldo;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (bn == 256) return launch_gemm<256, 4, false, false, true>(ta, tw, po.map[0], po.map[0], p, dev, s, &po);
    if (bn == 64) return launch_gemm<64, 7, false, false, true>(ta, tw, po.map[0], po.map[0], p, dev, s, &po);
    return launch_gemm<128, 5, false, false, true>(ta, tw, po.map[0], po.map[0], p, dev, s, &po);
}

int dotl_linear_ln(const void* a, int64_t M, int64_t K, int64_t lda, const void* w, int64_t N, int64_t ldw,
                   const float* bias, const float* resid, int64_t ldr, const uint8_t* row_valid, int resid_mode,
                   float* out, int64_t ldo, const float* ln_weight, const float* ln_bias, float eps, void* normed,
                   int normed_dtype, int64_t ldn, const uint8_t* normed_row_valid, int tile_n, int operands,
                   void* stream) {
    const char* who = "linear_add_layernorm";
    if (M < 0 || N <= 0 || K <= 0) return fail(DOTL_EINVAL, "%s: bad shape M=%lld N=%lld K=%lld", who, (long long)M, (long long)N, (long long)K);
    if (M > (int64_t)0x7fffffff - 256 || N > 0x7fffffff || K > 0x7fffffff)
        return fail(DOTL_EUNSUPPORTED, "%s: dimensions must fit in 31 bits", who);
    if (resid_mode != DOTL_RESID_NONE && resid_mode != DOTL_RESID_ADD && resid_mode != DOTL_RESID_ADD_MASKSUB &&
        resid_mode != DOTL_RESID_ADD_MASKALL)
        return fail(DOTL_EINVAL, "%s: residual mode %d is not one of NONE, ADD, ADD_MASKSUB, ADD_MASKALL", who, resid_mode);
    if (normed_dtype != DOTL_F32 && normed_dtype != DOTL_F16 && normed_dtype != DOTL_F16X2)
        return fail(DOTL_EINVAL, "%s: normed dtype must be DOTL_F32, DOTL_F16 or DOTL_F16X2", who);
    if (operands != DOTL_F16 && operands != DOTL_F16X2)
        return fail(DOTL_EINVAL, "%s: operands must be DOTL_F16 or DOTL_F16X2", who);
    const bool x3 = operands == DOTL_F16X2;
    if (!(eps >= 0.0f)) return fail(DOTL_EINVAL, "%s: eps must be >= 0", who);
    if (M == 0) return DOTL_OK;
    if (a == nullptr || w == nullptr || bias == nullptr || ln_weight == nullptr || ln_bias == nullptr || normed == nullptr)
        return fail(DOTL_EINVAL, "%s: NULL pointer", who);
    if (K % 8 != 0 || lda % 8 != 0 || ldw % 8 != 0 || lda < K || ldw < K)
        return fail(DOTL_EUNSUPPORTED, "%s: K, lda and ldw must be multiples of 8 (16-byte fp16 rows for TMA), got K=%lld lda=%lld ldw=%lld", who, (long long)K, (long long)lda, (long long)ldw);
    if (!aligned16(a) || !aligned16(w)) return fail(DOTL_EUNSUPPORTED, "%s: a and w must be 16-byte aligned", who);
    if (!aligned16(bias) || !aligned16(ln_weight) || !aligned16(ln_bias))
        return fail(DOTL_EUNSUPPORTED, "%s: bias, ln_weight and ln_bias must be 16-byte aligned", who);
    if (out != nullptr && (ldo < N || !aligned16(out) || ldo % 4 != 0))
        return fail(DOTL_EUNSUPPORTED, "%s: out must be 16-byte aligned with ldo >= N, ldo %% 4 == 0", who);
    if (ldn < N || !aligned16(normed) || ldn % 8 != 0)
        return fail(DOTL_EUNSUPPORTED, "%s: normed must be 16-byte aligned with ldn >= N, ldn %% 8 == 0", who);
    if (resid_mode != DOTL_RESID_NONE) {
        if (resid == nullptr) return fail(DOTL_EINVAL, "%s: residual mode %d needs resid", who, resid_mode);
        if (!aligned16(resid) || ldr % 4 != 0 || ldr < N) return fail(DOTL_EUNSUPPORTED, "%s: resid must be 16-byte aligned with ldr >= N, ldr %% 4 == 0", who);
    }
    if ((resid_mode == DOTL_RESID_ADD_MASKSUB || resid_mode == DOTL_RESID_ADD_MASKALL) && row_valid == nullptr)
        return fail(DOTL_EINVAL, "%s: masked residual mode needs row_valid", who);

    int dev;
    if (int rc = current_device(&dev)) return rc;
    int bn = tile_n;
    if (bn == 0) bn = pick_tile_n_ln(M, N, sm_count(dev));
    if (bn != 64 && bn != 128 && bn != 256)
        return fail(DOTL_EUNSUPPORTED, "%s: N=%lld must be 64, 128 or 256 times a cluster size of at most %d", who,
                    (long long)N, dotl::kLnMaxCluster);
    if (N % bn != 0 || N / bn > dotl::kLnMaxCluster)
        return fail(DOTL_EUNSUPPORTED, "%s: N=%lld is not tile_n=%d times a cluster size of at most %d", who,
                    (long long)N, bn, dotl::kLnMaxCluster);

    CUtensorMap ta, tw, tx, tn, tnl;
    const cuuint64_t adims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(x3 ? 2 * M : M)};
    const cuuint64_t astr[1] = {static_cast<cuuint64_t>(lda) * 2};
    if (int rc = encode_f16_map(&ta, a, 2, adims, astr, dotl::kGemmBK, dotl::kGemmBM, who)) return rc;
    const cuuint64_t wdims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(x3 ? 2 * N : N)};
    const cuuint64_t wstr[1] = {static_cast<cuuint64_t>(ldw) * 2};
    if (int rc = encode_f16_map(&tw, w, 2, wdims, wstr, dotl::kGemmBK, static_cast<uint32_t>(bn), who)) return rc;
    const int nstore = normed_dtype == DOTL_F16X2 ? DOTL_F16 : normed_dtype;
    // with out == NULL the x map points at `normed` and is never used
    if (int rc = encode_out_map(&tx, out != nullptr ? static_cast<void*>(out) : normed, M, N,
                                out != nullptr ? ldo : ldn, out != nullptr ? DOTL_F32 : nstore, who))
        return rc;
    if (int rc = encode_out_map(&tn, normed, M, N, ldn, nstore, who)) return rc;
    // DOTL_F16X2 normed: the lo plane, M rows of ldn below the hi plane
    tnl = tn;
    if (normed_dtype == DOTL_F16X2)
        if (int rc = encode_out_map(&tnl, static_cast<__half*>(normed) + M * ldn, M, N, ldn, DOTL_F16, who)) return rc;
    // residual in as 32 x 32 fp32 blocks (without a residual the map is unused)
    CUtensorMap tr = tn;
    if (resid_mode != DOTL_RESID_NONE)
        if (int rc = encode_out_map(&tr, const_cast<float*>(resid), M, N, ldr, DOTL_F32, who)) return rc;

    dotl::GemmLnParams p;
    p.M = static_cast<int>(M);
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(K);
    p.num_m_tiles = static_cast<int>((M + dotl::kGemmBM - 1) / dotl::kGemmBM);
    p.cs = static_cast<int>(N / bn);
    p.bias = bias;
    p.resid = resid;
    p.ldr = ldr;
    p.row_valid = row_valid;
    p.resid_mode = resid_mode;
    p.store_x = out != nullptr ? 1 : 0;
    p.ln_w = ln_weight;
    p.ln_b = ln_bias;
    p.eps = eps;
    p.norm_row_valid = normed_row_valid;
    p.x3_nkb = x3 ? static_cast<int>((K + dotl::kGemmBK - 1) / dotl::kGemmBK) : 0;
    p.a_lo_row = x3 ? static_cast<int>(M) : 0;
    p.w_lo_row = x3 ? static_cast<int>(N) : 0;
    p.norm_lo = normed_dtype == DOTL_F16X2 ? 1 : 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool f16 = nstore == DOTL_F16;
    if (bn == 256)
        return f16 ? launch_gemm_ln<256, 3, true>(ta, tw, tx, tn, tr, tnl, p, dev, s)
                   : launch_gemm_ln<256, 3, false>(ta, tw, tx, tn, tr, tnl, p, dev, s);
    if (bn == 128)
        return f16 ? launch_gemm_ln<128, 4, true>(ta, tw, tx, tn, tr, tnl, p, dev, s)
                   : launch_gemm_ln<128, 4, false>(ta, tw, tx, tn, tr, tnl, p, dev, s);
    return f16 ? launch_gemm_ln<64, 6, true>(ta, tw, tx, tn, tr, tnl, p, dev, s)
               : launch_gemm_ln<64, 6, false>(ta, tw, tx, tn, tr, tnl, p, dev, s);
}

}  // extern "C"

namespace {

// dotl_attention's body. workspace / workspace_bytes: where the split-KV
// partial rows may go (NULL or too small: no split-KV).
int attention_run(const void* q, const void* k, const void* v, int B, int H, int S, int head_dim,
                  const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides, const uint8_t* mask,
                  int mask_kind, const int64_t* mask_strides, int causal, float scale, void* out, int out_layout,
                  int out_dtype, void* workspace, int64_t workspace_bytes, void* stream) {
    const char* who = "fused_attention_forward";
    if (B < 0 || H < 0 || S < 0) return fail(DOTL_EINVAL, "%s: negative shape", who);
    if (out_layout != 0 && out_layout != 1)
        return fail(DOTL_EINVAL, "%s: out_layout must be 0 ([B,H,S,head_dim]) or 1 ([B,S,H*head_dim])", who);
    if (mask_kind < DOTL_MASK_NONE || mask_kind > DOTL_MASK_FULL) return fail(DOTL_EINVAL, "%s: unknown mask kind %d", who, mask_kind);
    if (out_dtype != DOTL_F16 && out_dtype != DOTL_F16X2)
        return fail(DOTL_EINVAL, "%s: out dtype must be DOTL_F16 or DOTL_F16X2", who);
    // DOTL_F16X2: the lo plane follows the hi plane (B*H*S*head_dim elements each)
    const int64_t out_lo = out_dtype == DOTL_F16X2 ? static_cast<int64_t>(B) * H * S * head_dim : 0;
    const bool tc = head_dim == 32 || head_dim == 64 || head_dim == 128;
    if (!tc && (head_dim < 8 || head_dim > 256 || head_dim % 8 != 0))
        return fail(DOTL_EUNSUPPORTED, "%s: head_dim must be a multiple of 8 up to 256, got %d", who, head_dim);
    if (B == 0 || H == 0 || S == 0) return DOTL_OK;
    if (q == nullptr || k == nullptr || v == nullptr || out == nullptr || q_strides == nullptr ||
        k_strides == nullptr || v_strides == nullptr)
        return fail(DOTL_EINVAL, "%s: NULL pointer", who);
    if (mask_kind != DOTL_MASK_NONE && (mask == nullptr || mask_strides == nullptr))
        return fail(DOTL_EINVAL, "%s: mask kind %d needs mask and mask_strides", who, mask_kind);
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
        return fail(DOTL_EUNSUPPORTED, "%s: q, k, v and out must be 16-byte aligned", who);
    const int64_t* st[3] = {q_strides, k_strides, v_strides};
    for (int t = 0; t < 3; ++t)
        for (int d = 0; d < 3; ++d)
            if (st[t][d] % 8 != 0 || st[t][d] < 0)
                return fail(DOTL_EUNSUPPORTED, "%s: q/k/v strides must be non-negative multiples of 8 elements (16 bytes)", who);
    if (static_cast<int64_t>(B) * S > 0x7fffff00LL) return fail(DOTL_EUNSUPPORTED, "%s: B*S must fit in 31 bits", who);
    if (!tc) {
        // head dims outside the tcgen05 kernel's tiles: the CUDA-core kernel
        if (static_cast<int64_t>(B) * H > 65535)
            return fail(DOTL_EUNSUPPORTED, "%s: B*H=%lld is over the 65535 (batch, head) pairs of the head_dim %d kernel's grid", who,
                        static_cast<long long>(B) * H, head_dim);
        dotl::AttnGenericParams g;
        g.q = static_cast<const __half*>(q);
        g.k = static_cast<const __half*>(k);
        g.v = static_cast<const __half*>(v);
        for (int d = 0; d < 3; ++d) {
            g.qs[d] = q_strides[d];
            g.ks[d] = k_strides[d];
            g.vs[d] = v_strides[d];
        }
        g.B = B;
        g.H = H;
        g.S = S;
        g.hd = head_dim;
        g.causal = causal ? 1 : 0;
        g.scale = scale;
        g.mask_kind = mask_kind;
        g.mask = mask;
        g.ms0 = mask_strides ? mask_strides[0] : 0;
        g.ms1 = mask_strides ? mask_strides[1] : 0;
        g.ms2 = mask_strides ? mask_strides[2] : 0;
        g.ms3 = mask_strides ? mask_strides[3] : 0;
        g.out = static_cast<__half*>(out);
        g.out_layout = out_layout;
        g.out_lo = out_lo;
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        cudaError_t e;
        if (head_dim <= 24) {
            // a thread per query row
            const dim3 rgrid(static_cast<unsigned>((S + dotl::kRowsBlock - 1) / dotl::kRowsBlock),
                             static_cast<unsigned>(B * H));
            const dim3 rblock(dotl::kRowsBlock);
            if (head_dim == 8) e = launch_pdl(dotl::attn_rows_kernel<8>, rgrid, rblock, 0, s, g);
            else if (head_dim == 16) e = launch_pdl(dotl::attn_rows_kernel<16>, rgrid, rblock, 0, s, g);
            else e = launch_pdl(dotl::attn_rows_kernel<24>, rgrid, rblock, 0, s, g);
            if (e != cudaSuccess) return fail(DOTL_ECUDA, "%s: launch failed: %s", who, cudaGetErrorString(e));
            return check_launch(who);
        }
        const dim3 grid(static_cast<unsigned>((S + dotl::kGenRows - 1) / dotl::kGenRows),
                        static_cast<unsigned>(B * H));
        const dim3 block(dotl::kGenRows * 32);
        if (head_dim <= 64) e = launch_pdl(dotl::attn_generic_kernel<2>, grid, block, 0, s, g);
        else if (head_dim <= 128) e = launch_pdl(dotl::attn_generic_kernel<4>, grid, block, 0, s, g);
        else e = launch_pdl(dotl::attn_generic_kernel<8>, grid, block, 0, s, g);
        if (e != cudaSuccess) return fail(DOTL_ECUDA, "%s: launch failed: %s", who, cudaGetErrorString(e));
        return check_launch(who);
    }

    // Packed tiles run over the flat token axis: every tensor must step from
    // one batch to the next exactly one sequence length further on. Only
    // sequences shorter than a tile are packed; longer ones get tiles of their
    // own, so a row's key tiles start at its sequence's first key whatever the
    // batch size, and a batch row gives the same bits alone or in a batch.
    bool packed = S < dotl::kAttnTile;
    for (int t = 0; t < 3; ++t) packed = packed && (st[t][0] == static_cast<int64_t>(S) * st[t][2]);

    dotl::AttnParams p;
    p.B = B;
    p.H = H;
    p.S = S;
    p.packed = packed ? 1 : 0;
    p.rows_total = packed ? B * S : S;
    p.num_q_tiles = (p.rows_total + dotl::kAttnTile - 1) / dotl::kAttnTile;
    p.num_streams = packed ? H : B * H;
    p.causal = causal ? 1 : 0;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.mask_kind = mask_kind;
    p.mask = mask;
    p.ms0 = mask_strides ? mask_strides[0] : 0;
    p.ms1 = mask_strides ? mask_strides[1] : 0;
    p.ms2 = mask_strides ? mask_strides[2] : 0;
    p.ms3 = mask_strides ? mask_strides[3] : 0;
    p.out = out;
    p.out_layout = out_layout;
    p.out_lo = out_lo;
    p.splits = 1;
    p.kt_per_split = 0;
    p.ws_o = nullptr;
    p.ws_ml = nullptr;

    const uint32_t box_cols = head_dim < 64 ? static_cast<uint32_t>(head_dim) : 64u;
    const void* bases[3] = {q, k, v};
    CUtensorMap maps[3];
    p.head_inner = 0;
    for (int t = 0; t < 3; ++t) {
        if (st[t][1] == 0 || st[t][2] == 0)
            return fail(DOTL_EUNSUPPORTED, "%s: zero sequence/head strides are not supported", who);
        // Dimensions in memory order: the head axis goes inside the row axis
        // when heads are closer together than rows (the fused QKV buffer).
        const bool head_inner = st[t][1] < st[t][2];
        const cuuint64_t rows = static_cast<cuuint64_t>(p.rows_total);
        const cuuint64_t row_stride = static_cast<cuuint64_t>(st[t][2]) * 2;
        const cuuint64_t head_stride = static_cast<cuuint64_t>(st[t][1]) * 2;
        cuuint64_t batch_stride = packed ? row_stride * rows : static_cast<cuuint64_t>(st[t][0]) * 2;
        if (batch_stride == 0) batch_stride = 16;
        const cuuint64_t batches = packed ? 1 : static_cast<cuuint64_t>(B);
        cuuint64_t dims[4], strides[3];
        dims[0] = static_cast<cuuint64_t>(head_dim);
        if (head_inner) {
            dims[1] = static_cast<cuuint64_t>(H); dims[2] = rows;
            strides[0] = head_stride; strides[1] = row_stride;
        } else {
            dims[1] = rows; dims[2] = static_cast<cuuint64_t>(H);
            strides[0] = row_stride; strides[1] = head_stride;
        }
        dims[3] = batches;
        strides[2] = batch_stride;
        CUtensorMap* m = &maps[t];
        EncodeTiledFn fn = encode_fn();
        if (fn == nullptr) return fail(DOTL_ECUDA, "%s: cuTensorMapEncodeTiled is unavailable from the driver", who);
        cuuint32_t box[4] = {box_cols, head_inner ? 1u : static_cast<cuuint32_t>(dotl::kAttnTile),
                             head_inner ? static_cast<cuuint32_t>(dotl::kAttnTile) : 1u, 1u};
        cuuint32_t estr[4] = {1, 1, 1, 1};
        const CUtensorMapSwizzle swz = box_cols == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
        const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(bases[t]), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return fail(DOTL_ECUDA, "%s: cuTensorMapEncodeTiled failed (CUresult %d)", who, (int)r);
        if (head_inner) p.head_inner |= (1 << t);
    }
    int dev;
    if (int rc = current_device(&dev)) return rc;
    if (!packed && workspace != nullptr) {
        int kt = 0;
        const int splits = attn_split_plan(p.num_streams, p.num_q_tiles, (S + dotl::kAttnTile - 1) / dotl::kAttnTile,
                                           causal != 0, sm_count(dev), &kt);
        const int64_t need = attn_split_bytes(p.num_streams, p.num_q_tiles, splits, head_dim);
        if (splits > 1 && workspace_bytes >= need && aligned16(workspace)) {
            p.splits = splits;
            p.kt_per_split = kt;
            p.ws_o = static_cast<float*>(workspace);
            p.ws_ml = reinterpret_cast<float2*>(static_cast<uint8_t*>(workspace) +
                                                static_cast<int64_t>(p.num_streams) * p.num_q_tiles * splits *
                                                    dotl::kAttnTile * head_dim * 4);
        }
    }
    // One key tile per item: a query tile's keys are its own sequence's (at
    // most 128 of them), or, packed, those of the sequences that fill it.
    const bool single = p.splits == 1 && (packed ? dotl::kAttnTile % S == 0 : S <= dotl::kAttnTile);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (head_dim) {
        case 32: return launch_attn<32, 4>(maps[0], maps[1], maps[2], p, single, dev, s);
        case 64: return launch_attn<64, 3>(maps[0], maps[1], maps[2], p, single, dev, s);
        default: return launch_attn<128, 2>(maps[0], maps[1], maps[2], p, single, dev, s);
    }
}

}  // namespace

extern "C" {

int dotl_attention(const void* q, const void* k, const void* v, int B, int H, int S, int head_dim,
                   const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides, const uint8_t* mask,
                   int mask_kind, const int64_t* mask_strides, int causal, float scale, void* out, int out_layout,
                   int out_dtype, void* workspace, int64_t workspace_bytes, void* stream) {
    return attention_run(q, k, v, B, H, S, head_dim, q_strides, k_strides, v_strides, mask, mask_kind, mask_strides,
                         causal, scale, out, out_layout, out_dtype, workspace, workspace_bytes, stream);
}

// ---------------------------------------------- attention without allocation --
//
// For callers that cannot allocate device memory on their own: a caller whose
// host side has no CUDA allocator it may use (a binding that can only hand
// over the pointers it already owns), or one running while allocation is off
// limits to it (inside a memory pool it must not grow). The split-KV scratch
// lives in one static device array of kStaticScratchBytes instead of a
// caller workspace. The array is per device and per process, held from the
// library's load until exit, and shared by every call.

}  // extern "C"

namespace {

constexpr int64_t kStaticScratchBytes = int64_t{16} << 20;
static_assert(kStaticScratchBytes == DOTL_ATTENTION_STATIC_SCRATCH_BYTES, "the header states the array's size");
static __device__ __align__(256) uint8_t g_attn_static_scratch[kStaticScratchBytes];

// The array's device address on device `dev` (the current device). The name
// in host code only stands in for the symbol; the address comes from
// cudaGetSymbolAddress, once per device, with that device current.
int static_scratch_address(int dev, void** out) {
    static std::atomic<void*> addr[kMaxDevices];
    if (dev < 0 || dev >= kMaxDevices) return fail(DOTL_EUNSUPPORTED, "dotl_attention_static_scratch: device %d", dev);
    void* p = addr[dev].load(std::memory_order_acquire);
    if (p == nullptr) {
        const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_static_scratch);
        if (e != cudaSuccess || p == nullptr)
            return fail(DOTL_ECUDA, "dotl_attention_static_scratch: cudaGetSymbolAddress failed: %s",
                        cudaGetErrorString(e));
        addr[dev].store(p, std::memory_order_release);
    }
    *out = p;
    return DOTL_OK;
}

}  // namespace

extern "C" {

int dotl_attention_static_scratch(const void* q, const void* k, const void* v, int B, int H, int S, int head_dim,
                                  const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                                  const uint8_t* mask, int mask_kind, const int64_t* mask_strides, int causal,
                                  float scale, void* out, int out_layout, int out_dtype, void* stream) {
    int64_t need = 0;
    if (int rc = dotl_attention_workspace_bytes(B, H, S, head_dim, causal, &need)) return rc;
    if (need > kStaticScratchBytes)
        return fail(DOTL_EUNSUPPORTED,
                    "dotl_attention_static_scratch: B=%d H=%d S=%d head_dim=%d needs %lld bytes of split-KV scratch, "
                    "over the %lld-byte static array; call dotl_attention with a workspace instead",
                    B, H, S, head_dim, (long long)need, (long long)kStaticScratchBytes);
    void* scratch = nullptr;
    if (need > 0) {
        int dev;
        if (int rc = current_device(&dev)) return rc;
        if (int rc = static_scratch_address(dev, &scratch)) return rc;
    }
    return attention_run(q, k, v, B, H, S, head_dim, q_strides, k_strides, v_strides, mask, mask_kind, mask_strides,
                         causal, scale, out, out_layout, out_dtype, scratch, need > 0 ? kStaticScratchBytes : 0,
                         stream);
}

int dotl_attention_workspace_bytes(int B, int H, int S, int head_dim, int causal, int64_t* bytes) {
    if (bytes == nullptr || B < 0 || H < 0 || S < 0) return fail(DOTL_EINVAL, "dotl_attention_workspace_bytes: bad arguments");
    *bytes = 0;
    const bool tc = head_dim == 32 || head_dim == 64 || head_dim == 128;
    if (!tc || B == 0 || H == 0 || S < dotl::kAttnTile) return DOTL_OK;   // no split-KV there
    int dev;
    if (int rc = current_device(&dev)) return rc;
    const int streams = B * H, q_tiles = (S + dotl::kAttnTile - 1) / dotl::kAttnTile;
    int kt = 0;
    const int splits = attn_split_plan(streams, q_tiles, q_tiles, causal != 0, sm_count(dev), &kt);
    if (splits > 1) *bytes = attn_split_bytes(streams, q_tiles, splits, head_dim);
    return DOTL_OK;
}

int dotl_ffn(const void* a, int64_t M, int64_t D, int64_t lda, const void* w1, int64_t F, int64_t ldw1,
             const float* b1, const void* w2, int64_t ldw2, const float* b2, const float* resid, int64_t ldr,
             const uint8_t* row_valid, int resid_mode, float* x_out, int64_t ldx, const float* ln_weight,
             const float* ln_bias, float eps, void* normed, int normed_dtype, int64_t ldn,
             const uint8_t* normed_row_valid, void* stream) {
    const char* who = "dotl_ffn";
    if (M < 0 || M > (int64_t)0x7fffffff - 256) return fail(DOTL_EINVAL, "%s: bad M=%lld", who, (long long)M);
    if (D != 128 && D != 256) return fail(DOTL_EUNSUPPORTED, "%s: D=%lld (d_model) must be 128 or 256", who, (long long)D);
    if (F <= 0 || F % dotl::kFfnChunk != 0 || F > 0x7fffffff)
        return fail(DOTL_EUNSUPPORTED, "%s: F=%lld (ffn_dim) must be a positive multiple of 128", who, (long long)F);
    if (resid_mode != DOTL_RESID_NONE && resid_mode != DOTL_RESID_ADD && resid_mode != DOTL_RESID_ADD_MASKSUB &&
        resid_mode != DOTL_RESID_ADD_MASKALL)
        return fail(DOTL_EINVAL, "%s: residual mode %d is not one of NONE, ADD, ADD_MASKSUB, ADD_MASKALL", who, resid_mode);
    if (normed_dtype != DOTL_F32 && normed_dtype != DOTL_F16) return fail(DOTL_EINVAL, "%s: normed dtype must be DOTL_F32 or DOTL_F16", who);
    if (!(eps >= 0.0f)) return fail(DOTL_EINVAL, "%s: eps must be >= 0", who);
    if (M == 0) return DOTL_OK;
    if (a == nullptr || w1 == nullptr || w2 == nullptr || b1 == nullptr || b2 == nullptr || ln_weight == nullptr ||
        ln_bias == nullptr || normed == nullptr)
        return fail(DOTL_EINVAL, "%s: NULL pointer", who);
    if (lda < D || ldw1 < D || ldw2 < F || lda % 8 != 0 || ldw1 % 8 != 0 || ldw2 % 8 != 0)
        return fail(DOTL_EUNSUPPORTED, "%s: lda, ldw1 >= D and ldw2 >= F must be multiples of 8", who);
    if (!aligned16(a) || !aligned16(w1) || !aligned16(w2) || !aligned16(b1) || !aligned16(b2) ||
        !aligned16(ln_weight) || !aligned16(ln_bias))
        return fail(DOTL_EUNSUPPORTED, "%s: operands, biases and LayerNorm parameters must be 16-byte aligned", who);
    if (resid_mode != DOTL_RESID_NONE) {
        if (resid == nullptr) return fail(DOTL_EINVAL, "%s: residual mode %d needs resid", who, resid_mode);
        if (!aligned16(resid) || ldr % 4 != 0 || ldr < D) return fail(DOTL_EUNSUPPORTED, "%s: resid must be 16-byte aligned with ldr >= D, ldr %% 4 == 0", who);
    }
    if ((resid_mode == DOTL_RESID_ADD_MASKSUB || resid_mode == DOTL_RESID_ADD_MASKALL) && row_valid == nullptr)
        return fail(DOTL_EINVAL, "%s: masked residual mode needs row_valid", who);
    if (x_out != nullptr && (!aligned16(x_out) || ldx % 4 != 0 || ldx < D))
        return fail(DOTL_EUNSUPPORTED, "%s: x_out must be 16-byte aligned with ldx >= D, ldx %% 4 == 0", who);
    if (!aligned16(normed) || ldn % 8 != 0 || ldn < D)
        return fail(DOTL_EUNSUPPORTED, "%s: normed must be 16-byte aligned with ldn >= D, ldn %% 8 == 0", who);

    CUtensorMap ta, tw1, tw2;
    const cuuint64_t adims[2] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(M)};
    const cuuint64_t astr[1] = {static_cast<cuuint64_t>(lda) * 2};
    if (int rc = encode_f16_map(&ta, a, 2, adims, astr, dotl::kGemmBK, dotl::kGemmBM, who)) return rc;
    const cuuint64_t w1dims[2] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(F)};
    const cuuint64_t w1str[1] = {static_cast<cuuint64_t>(ldw1) * 2};
    if (int rc = encode_f16_map(&tw1, w1, 2, w1dims, w1str, dotl::kGemmBK, 128, who)) return rc;
    const cuuint64_t w2dims[2] = {static_cast<cuuint64_t>(F), static_cast<cuuint64_t>(D)};
    const cuuint64_t w2str[1] = {static_cast<cuuint64_t>(ldw2) * 2};
    if (int rc = encode_f16_map(&tw2, w2, 2, w2dims, w2str, dotl::kGemmBK, 128, who)) return rc;
    // residual in, x_new and normed out: 32 x 32 blocks (unused maps describe `normed`)
    CUtensorMap tr, tx, tn;
    if (int rc = encode_out_map(&tn, normed, M, D, ldn, normed_dtype, who)) return rc;
    tr = tn;
    tx = tn;
    if (resid_mode != DOTL_RESID_NONE)
        if (int rc = encode_out_map(&tr, const_cast<float*>(resid), M, D, ldr, DOTL_F32, who)) return rc;
    if (x_out != nullptr)
        if (int rc = encode_out_map(&tx, x_out, M, D, ldx, DOTL_F32, who)) return rc;

    dotl::FfnParams p;
    p.M = static_cast<int>(M);
    p.D = static_cast<int>(D);
    p.F = static_cast<int>(F);
    p.num_m_tiles = static_cast<int>((M + dotl::kGemmBM - 1) / dotl::kGemmBM);
    p.b1 = b1;
    p.b2 = b2;
    p.resid = resid;
    p.ldr = ldr;
    p.row_valid = row_valid;
    p.resid_mode = resid_mode;
    p.x_out = x_out;
    p.ldx = ldx;
    p.ln_w = ln_weight;
    p.ln_b = ln_bias;
    p.eps = eps;
    p.normed = normed;
    p.ldn = ldn;
    p.norm_row_valid = normed_row_valid;
    int dev;
    if (int rc = current_device(&dev)) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (D == 128)
        return normed_dtype == DOTL_F16 ? launch_ffn<128, true>(ta, tw1, tw2, tr, tx, tn, p, dev, s)
                                        : launch_ffn<128, false>(ta, tw1, tw2, tr, tx, tn, p, dev, s);
    return normed_dtype == DOTL_F16 ? launch_ffn<256, true>(ta, tw1, tw2, tr, tx, tn, p, dev, s)
                                    : launch_ffn<256, false>(ta, tw1, tw2, tr, tx, tn, p, dev, s);
}

// ------------------------------------------------------------ peer memory --

int dotl_peer_alloc(int64_t bytes, void** ptr) {
    if (ptr == nullptr || bytes <= 0) return fail(DOTL_EINVAL, "dotl_peer_alloc: bad arguments");
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, static_cast<size_t>(bytes));
    if (e != cudaSuccess) return fail(DOTL_ECUDA, "dotl_peer_alloc(%lld bytes): %s", (long long)bytes, cudaGetErrorString(e));
    e = cudaMemset(p, 0, static_cast<size_t>(bytes));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(p);
        return fail(DOTL_ECUDA, "dotl_peer_alloc: zeroing failed: %s", cudaGetErrorString(e));
    }
    *ptr = p;
    return DOTL_OK;
}

int dotl_peer_free(void* ptr) {
    if (ptr == nullptr) return DOTL_OK;
    const cudaError_t e = cudaFree(ptr);
    if (e != cudaSuccess) return fail(DOTL_ECUDA, "dotl_peer_free: %s", cudaGetErrorString(e));
    return DOTL_OK;
}

int dotl_ipc_handle(const void* ptr, void* handle) {
    if (ptr == nullptr || handle == nullptr) return fail(DOTL_EINVAL, "dotl_ipc_handle: NULL pointer");
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
    if (e != cudaSuccess) return fail(DOTL_ECUDA, "dotl_ipc_handle: %s", cudaGetErrorString(e));
    static_assert(sizeof(h) == DOTL_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof(h));
    return DOTL_OK;
}

int dotl_ipc_open(const void* handle, void** ptr) {
    if (ptr == nullptr || handle == nullptr) return fail(DOTL_EINVAL, "dotl_ipc_open: NULL pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return fail(DOTL_ECUDA, "dotl_ipc_open: %s", cudaGetErrorString(e));
    *ptr = p;
    return DOTL_OK;
}

int dotl_ipc_close(void* ptr) {
    if (ptr == nullptr) return DOTL_OK;
    const cudaError_t e = cudaIpcCloseMemHandle(ptr);
    if (e != cudaSuccess) return fail(DOTL_ECUDA, "dotl_ipc_close: %s", cudaGetErrorString(e));
    return DOTL_OK;
}

int dotl_peer_blocks(int* blocks) {
    if (blocks == nullptr) return fail(DOTL_EINVAL, "dotl_peer_blocks: out is NULL");
    int dev;
    if (int rc = current_device(&dev)) return rc;
    *blocks = sm_count(dev) * dotl::kPeerBlocksPerSm;
    return DOTL_OK;
}

int dotl_peer_signal_bytes(int blocks, int64_t* bytes) {
    if (bytes == nullptr || blocks <= 0) return fail(DOTL_EINVAL, "dotl_peer_signal_bytes: bad arguments");
    *bytes = dotl::peer_signal_words(blocks) * 4;
    return DOTL_OK;
}

int dotl_allreduce_ln(int world, int rank, const float* const* parts, void* const* signals, float* const* x_new,
                      void* const* normed, int normed_dtype, int push, int parts_local, const float* x, const float* bias,
                      const uint8_t* sum_row_valid, const float* ln_weight, const float* ln_bias, float eps,
                      const uint8_t* normed_row_valid, int64_t rows, int64_t D, int blocks, int64_t signal_bytes,
                      unsigned int* status, int timeout_ms, void* stream) {
    const char* who = "dotl_allreduce_ln";
    if (world < 1 || world > dotl::kPeerMax || rank < 0 || rank >= world)
        return fail(DOTL_EINVAL, "%s: world %d / rank %d outside 1..%d", who, world, rank, dotl::kPeerMax);
    if (rows < 0 || D <= 0 || D % 4 != 0 || D > 2048)
        return fail(DOTL_EINVAL, "%s: rows=%lld, D=%lld (D must be a multiple of 4 up to 2048)", who, (long long)rows,
                    (long long)D);
    if (normed_dtype != DOTL_F32 && normed_dtype != DOTL_F16)
        return fail(DOTL_EINVAL, "%s: normed dtype must be DOTL_F32 or DOTL_F16", who);
    if (timeout_ms < 1 || timeout_ms > 60000) return fail(DOTL_EINVAL, "%s: timeout_ms must be in 1..60000", who);
    if (parts_local && !push) return fail(DOTL_EINVAL, "%s: parts_local needs push mode (each rank reduces its own rows)", who);
    if (parts == nullptr || signals == nullptr || normed == nullptr || x == nullptr || ln_weight == nullptr ||
        ln_bias == nullptr)
        return fail(DOTL_EINVAL, "%s: NULL pointer", who);
    // The signal layout depends on the grid (counters, then flags at offset
    // blocks): a grid other than the one the areas were sized for would write
    // past them or overlap counters with flags.
    if (signal_bytes != dotl::peer_signal_words(blocks) * 4)
        return fail(DOTL_EINVAL,
                    "%s: signal areas of %lld bytes do not match blocks=%d (dotl_peer_signal_bytes gives %lld); "
                    "blocks must be the value the areas were allocated for, on every call and every rank",
                    who, (long long)signal_bytes, blocks, (long long)(dotl::peer_signal_words(blocks) * 4));
    if (status != nullptr && (reinterpret_cast<uintptr_t>(status) & 3u) != 0)
        return fail(DOTL_EINVAL, "%s: status word must be 4-byte aligned", who);
    dotl::PeerLnParams p = {};
    const int d0 = push ? 0 : rank, d1 = push ? world : rank + 1;
    for (int i = 0; i < world; ++i) {
        if (parts[i] == nullptr || signals[i] == nullptr) return fail(DOTL_EINVAL, "%s: rank %d buffer is NULL", who, i);
        if (!aligned16(parts[i]) || !aligned16(signals[i]))
            return fail(DOTL_EINVAL, "%s: rank %d buffers must be 16-byte aligned", who, i);
        p.part[i] = parts[i];
        p.signal[i] = static_cast<unsigned int*>(signals[i]);
        if (i >= d0 && i < d1) {
            if (normed[i] == nullptr) return fail(DOTL_EINVAL, "%s: normed output of rank %d is NULL", who, i);
            p.normed[i] = normed[i];
            p.x_new[i] = x_new != nullptr ? x_new[i] : nullptr;
            if (!aligned16(p.normed[i]) || !aligned16(p.x_new[i]))
                return fail(DOTL_EINVAL, "%s: outputs must be 16-byte aligned", who);
        }
    }
    if (!aligned16(x) || !aligned16(bias) || !aligned16(ln_weight) || !aligned16(ln_bias))
        return fail(DOTL_EINVAL, "%s: x, bias and LayerNorm parameters must be 16-byte aligned", who);
    int dev;
    if (int rc = current_device(&dev)) return rc;
    const int cap = sm_count(dev) * dotl::kPeerBlocksPerSm;
    if (blocks < 1 || blocks > cap)
        return fail(DOTL_EINVAL, "%s: blocks %d outside 1..%d (every CTA must be resident at once)", who, blocks, cap);
    if (rows == 0) return DOTL_OK;
    p.x = x;
    p.bias = bias;
    p.sum_row_valid = sum_row_valid;
    p.ln_w = ln_weight;
    p.ln_b = ln_bias;
    p.normed_row_valid = normed_row_valid;
    p.rows = rows;
    p.D = static_cast<int>(D);
    p.eps = eps;
    p.world = world;
    p.rank = rank;
    p.push = push ? 1 : 0;
    p.parts_local = parts_local ? 1 : 0;
    p.timeout_ns = static_cast<unsigned long long>(timeout_ms) * 1000000ull;
    p.status = status;
    const dim3 grid(static_cast<unsigned>(blocks)), block(dotl::kPeerWarps * 32);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t le;
#define DOTL_ARLN(EPL)                                                                                   \
    le = normed_dtype == DOTL_F16 ? launch_pdl(dotl::allreduce_ln_kernel<EPL, __half>, grid, block, 0, s, p) \
                                  : launch_pdl(dotl::allreduce_ln_kernel<EPL, float>, grid, block, 0, s, p)
    if (D <= 128) DOTL_ARLN(4);
    else if (D <= 256) DOTL_ARLN(8);
    else if (D <= 512) DOTL_ARLN(16);
    else if (D <= 1024) DOTL_ARLN(32);
    else DOTL_ARLN(64);
#undef DOTL_ARLN
    if (le != cudaSuccess) return fail(DOTL_ECUDA, "%s: launch failed: %s", who, cudaGetErrorString(le));
    return check_launch(who);
}

}  // extern "C"
