// extern "C" entry points of libgptoss_moe.so (declared in include/gptoss_moe.h).
// Validation mirrors the reference's CHECK_* macros (kernels/matmul_mxfp4_cutlass.cu:
// 1107-1116): every failure becomes a status code plus a thread-local message.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>
#include <string>
#include <utility>

#include "gptoss_moe.h"
#include "ptx.cuh"
#include "numerics.cuh"
#include "routing.cuh"
#include "gemm.cuh"
#include "prologue.cuh"
#include "ep_p2p.cuh"
#include "decode_layer.cuh"
#include "mma_peak.cuh"

using namespace gptoss;

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

#define GPTOSS_CUDA(call)                                                                    \
  do {                                                                                       \
    cudaError_t e_ = (call);                                                                 \
    if (e_ != cudaSuccess)                                                                   \
      return fail(GPTOSS_ERR_CUDA, "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_),   \
                  __FILE__, __LINE__);                                                       \
  } while (0)

#define GPTOSS_CHECK(cond, ...)                                                              \
  do {                                                                                       \
    if (!(cond)) return fail(GPTOSS_ERR_INVALID_ARGUMENT, __VA_ARGS__);                      \
  } while (0)

#define GPTOSS_TRY(expr)                                                                     \
  do {                                                                                       \
    int rc_ = (expr);                                                                        \
    if (rc_ != GPTOSS_OK) return rc_;                                                        \
  } while (0)

constexpr int kMaxDevices = 64;

// NVTX range around one entry point (visible in Nsight timelines and `ncu --nvtx`; the
// calls are no-ops while no tool is attached).
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

// Kernels this library launched in this process (every device), for launch accounting.
std::atomic<uint64_t> g_kernel_launches{0};

struct DeviceInfo {
  int sms = 0;
  int major = 0;
  int minor = 0;
  int* status_sink = nullptr;
};

__device__ int g_status_sink[kMaxDevices];

std::mutex g_dev_mu;
DeviceInfo g_dev[kMaxDevices];
bool g_dev_ready[kMaxDevices] = {};

// Makes the device that owns `ptr` current for this runtime and returns its info.
int bind_device(const void* ptr, const char* name, DeviceInfo* info) {
  if (ptr == nullptr) return fail(GPTOSS_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  cudaPointerAttributes at{};
  cudaError_t e = cudaPointerGetAttributes(&at, ptr);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(GPTOSS_ERR_INVALID_ARGUMENT, "%s: not a CUDA pointer (%s)", name, cudaGetErrorString(e));
  }
  if (at.type != cudaMemoryTypeDevice && at.type != cudaMemoryTypeManaged)
    return fail(GPTOSS_ERR_INVALID_ARGUMENT, "%s: must be a CUDA tensor", name);
  const int dev = at.device;
  if (dev < 0 || dev >= kMaxDevices) return fail(GPTOSS_ERR_INVALID_ARGUMENT, "%s: bad device %d", name, dev);
  int cur = -1;
  GPTOSS_CUDA(cudaGetDevice(&cur));
  if (cur != dev) GPTOSS_CUDA(cudaSetDevice(dev));
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (!g_dev_ready[dev]) {
    cudaDeviceProp prop{};
    GPTOSS_CUDA(cudaGetDeviceProperties(&prop, dev));
    g_dev[dev].sms = prop.multiProcessorCount;
    g_dev[dev].major = prop.major;
    g_dev[dev].minor = prop.minor;
    void* sink = nullptr;
    GPTOSS_CUDA(cudaGetSymbolAddress(&sink, g_status_sink));
    g_dev[dev].status_sink = static_cast<int*>(sink) + dev;
    g_dev_ready[dev] = true;
  }
  *info = g_dev[dev];
  if (info->major != 10)
    return fail(GPTOSS_ERR_UNSUPPORTED_DEVICE,
                "requires an sm_100 (B200-class) GPU, device %d is sm_%d%d", dev, info->major, info->minor);
  return GPTOSS_OK;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int64_t pad128(int64_t k) { return (k + 127) / 128 * 128; }

// Launch with programmatic stream serialisation: the kernel may be scheduled while the
// previous kernel on the stream drains; every kernel of this library waits
// (griddepcontrol.wait) before touching global memory, so ordering is unchanged.
template <typename... KArgs, typename... Args>
int launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       dim3 cluster, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  int n = 1;
  if (cluster.x * cluster.y * cluster.z > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster.x;
    attr[1].val.clusterDim.y = cluster.y;
    attr[1].val.clusterDim.z = cluster.z;
    n = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  GPTOSS_CUDA(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
  return GPTOSS_OK;
}

template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  return launch_pdl_cluster(kernel, grid, block, smem, st, dim3(1, 1, 1), std::forward<Args>(args)...);
}

// ---------------------------------------------------------------- TMA descriptors
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int get_encode_fn(EncodeTiledFn* out) {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (err == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (fn == nullptr) return fail(GPTOSS_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (%s)", cudaGetErrorString(err));
  *out = fn;
  return GPTOSS_OK;
}

// Activations: 2-D [rows, lda] bytes (e4m3), box [box_rows, 128], 128B swizzle.
int make_act_map(CUtensorMap* m, const void* base, int64_t rows, int64_t lda, int box_rows) {
  EncodeTiledFn enc;
  GPTOSS_TRY(get_encode_fn(&enc));
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(lda), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(lda)};
  cuuint32_t box[2] = {128u, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(GPTOSS_ERR_CUDA, "cuTensorMapEncodeTiled(activations) failed: %d", (int)r);
  return GPTOSS_OK;
}

// Weights: 3-D [E, N, K] packed E2M1 (K/2 bytes per row); the TMA unit expands each
// 8-byte group of 16 codes into a 16-byte slot (the 8-bit container kind::mxf8f6f4 reads).
// packed: the W4A4 mode, whose MMA reads the packed bytes themselves (a 128-byte box of
// K/2-byte rows).
int make_wgt_map(CUtensorMap* m, const void* base, int E, int64_t N, int64_t K, int box_rows, bool packed = false) {
  EncodeTiledFn enc;
  GPTOSS_TRY(get_encode_fn(&enc));
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(packed ? K / 2 : K), static_cast<cuuint64_t>(N),
                        static_cast<cuuint64_t>(E)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(K / 2), static_cast<cuuint64_t>(N * (K / 2))};
  cuuint32_t box[3] = {128u, static_cast<cuuint32_t>(box_rows), 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = enc(m, packed ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 3,
                   const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(GPTOSS_ERR_CUDA, "cuTensorMapEncodeTiled(weights) failed: %d", (int)r);
  return GPTOSS_OK;
}

// Blocked scale buffer as rows of 256 bytes; a 512-byte chunk (one 128-row x 4-group
// atom) is a 2-row box. Used by the CTA-pair GEMM, whose loads all complete on one barrier.
int make_sf_map(CUtensorMap* m, const void* base, int64_t bytes) {
  EncodeTiledFn enc;
  GPTOSS_TRY(get_encode_fn(&enc));
  GPTOSS_CHECK(bytes >= 512 && bytes % 256 == 0, "scale buffer of %lld bytes", (long long)bytes);
  cuuint64_t dims[2] = {256u, static_cast<cuuint64_t>(bytes / 256)};
  cuuint64_t strides[1] = {256u};
  cuuint32_t box[2] = {256u, 2u};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(GPTOSS_ERR_CUDA, "cuTensorMapEncodeTiled(scales) failed: %d", (int)r);
  return GPTOSS_OK;
}

// ---------------------------------------------------------------- GEMM launch
struct GemmJob {
  const uint8_t* act;   // [act_rows, lda] e4m3
  int64_t act_rows;
  int64_t lda;
  const uint8_t* wgt;   // [E, N, K/2]
  GemmParams p;
  int64_t sfa_bytes;    // sizes of the scale buffers (0: unknown -> no CTA-pair tiles)
  int64_t sfb_bytes;
};

template <bool SWAP, bool SPREAD, int EPI, bool PAIR = false, bool NVF4 = false>
int launch_gemm(const GemmJob& job, const DeviceInfo& di, int dev, cudaStream_t st) {
  using C = GemmConfig<SWAP, SPREAD, PAIR, NVF4>;
  if (job.act_rows <= 0) return GPTOSS_OK;
  CUtensorMap ta, ta32, ta16, tw;
  GPTOSS_TRY(make_act_map(&ta, job.act, job.act_rows, job.lda, C::kActRows));
  if (SWAP) {
    GPTOSS_TRY(make_act_map(&ta32, job.act, job.act_rows, job.lda, 32));
    GPTOSS_TRY(make_act_map(&ta16, job.act, job.act_rows, job.lda, 16));
  } else if (PAIR) {
    GPTOSS_TRY(make_sf_map(&ta32, job.p.sfa, job.sfa_bytes));
    GPTOSS_TRY(make_sf_map(&ta16, job.p.sfb, job.sfb_bytes));
  } else {
    ta32 = ta;
    ta16 = ta;
  }
  GPTOSS_TRY(make_wgt_map(&tw, job.wgt, job.p.num_experts, job.p.N, job.p.K, C::kWgtRowsCta, NVF4));
  static uint64_t attr_done = 0;   // one bit per device
  static std::mutex mu;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!(attr_done & (1ull << dev))) {
      GPTOSS_CUDA(cudaFuncSetAttribute(moe_gemm_kernel<SWAP, SPREAD, EPI, PAIR, NVF4>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(C::kSmemBytes)));
      attr_done |= (1ull << dev);
    }
  }
  GemmParams p = job.p;
  p.n_tiles = static_cast<int>((p.N + C::kWgtRows - 1) / C::kWgtRows);
  const int64_t tiles_ub = (job.act_rows / C::kTileM + p.num_experts) * static_cast<int64_t>(p.n_tiles);
  const int grid = PAIR ? 2 * static_cast<int>(std::min<int64_t>(di.sms / 2, tiles_ub))
                        : static_cast<int>(std::min<int64_t>(di.sms, tiles_ub));
  if (grid <= 0) return GPTOSS_OK;
  return launch_pdl_cluster(moe_gemm_kernel<SWAP, SPREAD, EPI, PAIR, NVF4>, dim3(grid), dim3(C::kThreads), C::kSmemBytes,
                            st, PAIR ? dim3(2, 1, 1) : dim3(1, 1, 1), ta, ta32, ta16, tw, p);
}

// GEMM orientation of one call (pick_layout for the fused forwards; the reference-layout
// group GEMM uses 64-row chunks up to 48 rows per expert).
bool pick_swap(int mode, int64_t rows, int experts, int64_t max_avg) {
  if (mode == GPTOSS_GEMM_SWAP || mode == GPTOSS_GEMM_SWAP_WIDE) return true;
  if (mode == GPTOSS_GEMM_TOKENS_M) return false;
  return rows <= max_avg * experts;
}

// Tile orientation and activation-scale row layout of one expert forward. Weights-on-M
// tiles multiply 16-row activation chunks (SPREAD scale rows) while experts hold few rows:
// every chunk re-streams the expert's weight tiles, so an expert of 17..32 rows reads its
// weights twice. Past kSpreadMaxAvg rows per expert on average the 64-row chunks
// (reference scale rows; 16/32/64-row loads) take over, and past kSwapMaxAvg the
// tokens-on-M tiles. Crossovers measured on B200 for H = I = 2880, E = 16 and 32.
constexpr int64_t kSpreadMaxAvg = 12;
constexpr int64_t kSwapMaxAvg = 80;

struct GemmLayout {
  bool swap;
  bool spread;
};

GemmLayout pick_layout(int mode, int64_t rows, int experts) {
  if (mode == GPTOSS_GEMM_TOKENS_M) return {false, false};
  if (mode == GPTOSS_GEMM_SWAP) return {true, true};
  if (mode == GPTOSS_GEMM_SWAP_WIDE) return {true, false};
  if (rows > kSwapMaxAvg * experts) return {false, false};
  return {true, rows <= kSpreadMaxAvg * experts};
}

template <int EPI>
int run_gemm(const GemmJob& job, bool swap, bool spread, const DeviceInfo& di, int dev, cudaStream_t st) {
  if (!swap) {
    // CTA-pair tiles when the scale buffers can be described as 256-byte rows
    const bool pair = job.sfa_bytes > 0 && job.sfb_bytes > 0 && job.p.sfb_stride % 256 == 0 && di.sms >= 2;
    return pair ? launch_gemm<false, false, EPI, true>(job, di, dev, st) : launch_gemm<false, false, EPI>(job, di, dev, st);
  }
  return spread ? launch_gemm<true, true, EPI>(job, di, dev, st) : launch_gemm<true, false, EPI>(job, di, dev, st);
}

// ---------------------------------------------------------------- workspace layout
struct Workspace {
  size_t sorted_token, sorted_expert, sorted_weight, counts, offsets, sfoff_a, sfoff_b;
  size_t act_codes, act_sf, inter_codes, inter_sf, router_idx, router_w;
  size_t dl_logits, dl_sync;   // decode_layer_kernel: router logits, synchronisation words
  size_t total;
  int64_t act_sf_cap, inter_sf_cap;
};

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

Workspace plan_workspace(int64_t T, int k, int E, int64_t H, int64_t I) {
  Workspace w{};
  const int64_t A = T * k;
  // upper bound of the 128-row scale blocks of all experts, either scale row layout
  // (reference: sum ceil(m/128) <= A/128 + E; SPREAD: sum ceil(64 ceil(m/16) / 128) <= A/32 + E)
  const int64_t blocks = (A + 31) / 32 + E;
  w.act_sf_cap = blocks * (pad128(H) / 128) * 512;
  w.inter_sf_cap = blocks * (pad128(I) / 128) * 512;
  size_t o = 0;
  auto take = [&](size_t bytes) { size_t r = o; o = align256(o + bytes); return r; };
  w.sorted_token = take(sizeof(int64_t) * A);
  w.sorted_expert = take(sizeof(int64_t) * A);
  w.sorted_weight = take(sizeof(float) * A);
  w.counts = take(sizeof(int32_t) * E);
  w.offsets = take(sizeof(int32_t) * E);
  w.sfoff_a = take(sizeof(int32_t) * E);
  w.sfoff_b = take(sizeof(int32_t) * E);
  w.act_codes = take(static_cast<size_t>(A * H));
  w.act_sf = take(static_cast<size_t>(w.act_sf_cap));
  w.inter_codes = take(static_cast<size_t>(A * I));
  w.inter_sf = take(static_cast<size_t>(w.inter_sf_cap));
  w.router_idx = take(sizeof(int64_t) * A);
  w.router_w = take(sizeof(float) * A);
  w.dl_logits = take(sizeof(float) * T * E);
  w.dl_sync = take(sizeof(int32_t) * dl_sync_words(E));
  w.total = o;
  return w;
}

int router_launch(const void* hidden, const void* weight, const void* bias, int64_t T, int64_t H, int E,
                  int k, int64_t* idx, void* scores, float* wf32, void* logits, void* zero_rows,
                  int64_t zero_elems, int sms, int dev, cudaStream_t st) {
  const int64_t nblocks = (T + kRtTok - 1) / kRtTok;
  GPTOSS_CHECK(nblocks < (1LL << 31), "router: too many tokens");
  const int nchunks = static_cast<int>((H + kRtKc - 1) / kRtKc);
  const int tiles = (E + 7) / 8;                 // n-tiles of 8 experts over 4 warps
  const int nt = tiles <= 4 ? 1 : (tiles <= 8 ? 2 : (tiles <= 16 ? 4 : 8));
  // Split K over a cluster when the token blocks alone would leave SMs idle.
  int S = 1;
  if (nblocks < sms)
    S = static_cast<int>(std::min<int64_t>({router_max_split(nt), nchunks, (sms + nblocks - 1) / nblocks}));
  const int cpc = (nchunks + S - 1) / S;
  const size_t smem = router_smem_bytes(nt);
  auto go = [&](auto kern, int slot) -> int {
    static uint64_t attr_done[4] = {0, 0, 0, 0};   // one bit per device and instance
    static std::mutex mu;
    {
      std::lock_guard<std::mutex> lk(mu);
      if (!(attr_done[slot] & (1ull << dev))) {
        GPTOSS_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
        attr_done[slot] |= (1ull << dev);
      }
    }
    return launch_pdl_cluster(kern, dim3(static_cast<unsigned>(nblocks), S), dim3(128), smem, st, dim3(1, S, 1),
                              static_cast<const __nv_bfloat16*>(hidden), static_cast<const __nv_bfloat16*>(weight),
                              static_cast<const __nv_bfloat16*>(bias), static_cast<int>(T), static_cast<int>(H), E, k,
                              cpc, idx, static_cast<__nv_bfloat16*>(scores), wf32, static_cast<__nv_bfloat16*>(logits),
                              static_cast<__nv_bfloat16*>(zero_rows), zero_elems);
  };
  if (nt == 1) return go(router_mma_kernel<1>, 0);
  if (nt == 2) return go(router_mma_kernel<2>, 1);
  if (nt == 4) return go(router_mma_kernel<4>, 2);
  return go(router_mma_kernel<8>, 3);
}

struct ExpertWeights {
  const uint8_t* gu_data; const uint8_t* gu_scales; int64_t ldb_gu; const float* gu_bias;
  const uint8_t* dn_data; const uint8_t* dn_scales; int64_t ldb_dn; const float* dn_bias;
};

int check_expert_weights(const ExpertWeights& w, int64_t H, int64_t I, int E) {
  GPTOSS_CHECK(w.gu_data && w.gu_scales && w.gu_bias && w.dn_data && w.dn_scales && w.dn_bias,
               "expert weights: null pointer");
  GPTOSS_CHECK(aligned(w.gu_data, 32) && aligned(w.dn_data, 32), "weight data must be 32-byte aligned");
  GPTOSS_CHECK(aligned(w.gu_scales, 16) && aligned(w.dn_scales, 16), "weight scales must be 16-byte aligned");
  GPTOSS_CHECK(w.ldb_gu % 16 == 0 && w.ldb_dn % 16 == 0, "weight scale strides must be multiples of 16");
  GPTOSS_CHECK(w.ldb_gu >= blocked_sf_cosize(2 * I, static_cast<int>(pad128(H) / 32)),
               "gate_up scales: %lld bytes per expert, need %lld", (long long)w.ldb_gu,
               (long long)blocked_sf_cosize(2 * I, static_cast<int>(pad128(H) / 32)));
  GPTOSS_CHECK(w.ldb_dn >= blocked_sf_cosize(H, static_cast<int>(pad128(I) / 32)),
               "down scales: %lld bytes per expert, need %lld", (long long)w.ldb_dn,
               (long long)blocked_sf_cosize(H, static_cast<int>(pad128(I) / 32)));
  (void)E;
  return GPTOSS_OK;
}

struct WsPtrs {
  int64_t* sorted_token; int64_t* sorted_expert; float* sorted_weight;
  int32_t* counts; int32_t* offsets; int32_t* sfoff_a; int32_t* sfoff_b;
  uint8_t* act_codes; uint8_t* act_sf; uint8_t* inter_codes; uint8_t* inter_sf;
  int64_t act_sf_cap, inter_sf_cap;
};

WsPtrs ws_ptrs(uint8_t* ws, const Workspace& L) {
  WsPtrs w;
  w.sorted_token = reinterpret_cast<int64_t*>(ws + L.sorted_token);
  w.sorted_expert = reinterpret_cast<int64_t*>(ws + L.sorted_expert);
  w.sorted_weight = reinterpret_cast<float*>(ws + L.sorted_weight);
  w.counts = reinterpret_cast<int32_t*>(ws + L.counts);
  w.offsets = reinterpret_cast<int32_t*>(ws + L.offsets);
  w.sfoff_a = reinterpret_cast<int32_t*>(ws + L.sfoff_a);
  w.sfoff_b = reinterpret_cast<int32_t*>(ws + L.sfoff_b);
  w.act_codes = ws + L.act_codes;
  w.act_sf = ws + L.act_sf;
  w.inter_codes = ws + L.inter_codes;
  w.inter_sf = ws + L.inter_sf;
  w.act_sf_cap = L.act_sf_cap;
  w.inter_sf_cap = L.inter_sf_cap;
  return w;
}

// Stage 1: stable counting sort + gather + FP8 quantisation (blocked scales).
int stage_route_quant(const void* hidden, const int64_t* ridx, const float* rw, int64_t T, int k, int E, int64_t H,
                      int64_t I, const WsPtrs& w, bool spread, int* status, cudaStream_t st) {
  const int64_t A = T * k;
  const int64_t Kh = pad128(H), Ki = pad128(I);
  RouteSortParams rp{};
  rp.router_indices = ridx; rp.routing_weights = rw;
  rp.A = static_cast<int>(A); rp.K = k; rp.E = E;
  rp.sorted_token = w.sorted_token; rp.sorted_expert = w.sorted_expert; rp.sorted_weight = w.sorted_weight;
  rp.counts = w.counts; rp.offsets = w.offsets;
  rp.sf_offsets_a = w.sfoff_a; rp.g4_a = static_cast<int>(Kh / 128); rp.groups_a = static_cast<int>(H / 32); rp.sf_a = w.act_sf;
  rp.sf_offsets_b = w.sfoff_b; rp.g4_b = static_cast<int>(Ki / 128); rp.groups_b = static_cast<int>(I / 32); rp.sf_b = w.inter_sf;
  rp.spread = spread ? 1 : 0;
  rp.err = status;
  GPTOSS_TRY(launch_pdl(route_sort_kernel, dim3(E), dim3(1024), 0, st, rp));
  return launch_pdl(gather_quant_rows_kernel, dim3(static_cast<unsigned>((A + 7) / 8)), dim3(256), 0, st,
                    static_cast<const __nv_bfloat16*>(hidden), A, static_cast<int>(H),
                    static_cast<const int64_t*>(w.sorted_token), static_cast<const int64_t*>(w.sorted_expert),
                    static_cast<const int32_t*>(w.offsets), static_cast<const int32_t*>(w.sfoff_a),
                    static_cast<int>(Kh / 128), spread ? 1 : 0, w.act_codes, w.act_sf);
}

// Stage 2: GEMM1 + bias + SwiGLU + FP8 requantisation.
int stage_gemm1(int64_t A, int E, int64_t H, int64_t I, const ExpertWeights& wt, float sw_alpha, float sw_limit,
                const WsPtrs& w, GemmLayout lay, int* status, const DeviceInfo& di, int dev, cudaStream_t st,
                int prefetch_tiles = 0) {
  const int64_t Kh = pad128(H), Ki = pad128(I);
  GemmJob g1{};
  g1.act = w.act_codes; g1.act_rows = A; g1.lda = H; g1.wgt = wt.gu_data;
  g1.p.num_experts = E; g1.p.N = static_cast<int>(2 * I); g1.p.K = static_cast<int>(Kh); g1.p.num_kb = static_cast<int>(Kh / 128);
  g1.p.m_sizes = w.counts; g1.p.m_stride = 1; g1.p.row_offsets = w.offsets; g1.p.sfa_offsets = w.sfoff_a;
  g1.p.sfa = w.act_sf; g1.p.sfb = wt.gu_scales; g1.p.sfb_stride = wt.ldb_gu; g1.p.err = status;
  g1.p.out = w.inter_codes; g1.p.ld_out = I; g1.p.bias = wt.gu_bias; g1.p.out_sf = w.inter_sf;
  g1.p.out_sf_offsets = w.sfoff_b; g1.p.out_g4 = static_cast<int>(Ki / 128); g1.p.out_features = static_cast<int>(I);
  g1.p.swiglu_alpha = sw_alpha; g1.p.swiglu_limit = sw_limit;
  g1.p.prefetch_tiles = lay.swap ? prefetch_tiles : 0;
  g1.sfa_bytes = w.act_sf_cap;
  g1.sfb_bytes = wt.ldb_gu * E;
  return run_gemm<kEpiGemm1>(g1, lay.swap, lay.spread, di, dev, st);
}

// Stage 3: GEMM2 + bias, x routing weight, bf16 scatter-add into out (accumulates).
// Peer-memory return of the expert-parallel GEMM2 (see GemmParams::ep_*).
struct EpReturn {
  const uint64_t* peer_bases;
  int64_t ret_off, cap;
  int32_t* counter;
  int world, rank;
  int32_t epoch;
};

int stage_gemm2(int64_t A, int E, int64_t H, int64_t I, const ExpertWeights& wt, void* out, const WsPtrs& w,
                GemmLayout lay, int* status, const DeviceInfo& di, int dev, cudaStream_t st,
                const EpReturn* ep = nullptr) {
  const int64_t Ki = pad128(I);
  GemmJob g2{};
  g2.act = w.inter_codes; g2.act_rows = A; g2.lda = I; g2.wgt = wt.dn_data;
  g2.p.num_experts = E; g2.p.N = static_cast<int>(H); g2.p.K = static_cast<int>(Ki); g2.p.num_kb = static_cast<int>(Ki / 128);
  g2.p.m_sizes = w.counts; g2.p.m_stride = 1; g2.p.row_offsets = w.offsets; g2.p.sfa_offsets = w.sfoff_b;
  g2.p.sfa = w.inter_sf; g2.p.sfb = wt.dn_scales; g2.p.sfb_stride = wt.ldb_dn; g2.p.err = status;
  g2.p.out = out; g2.p.ld_out = H; g2.p.bias = wt.dn_bias; g2.p.token_idx = w.sorted_token; g2.p.row_weights = w.sorted_weight;
  g2.sfa_bytes = w.inter_sf_cap;
  g2.sfb_bytes = wt.ldb_dn * E;
  if (ep != nullptr) {
    GPTOSS_CHECK(lay.swap, "peer-memory GEMM2 return needs weights-on-M tiles");
    g2.p.ep_peer_bases = ep->peer_bases; g2.p.ep_ret_off = ep->ret_off; g2.p.ep_cap = ep->cap;
    g2.p.ep_counter = ep->counter; g2.p.ep_world = ep->world; g2.p.ep_rank = ep->rank; g2.p.ep_epoch = ep->epoch;
  }
  return run_gemm<kEpiGemm2>(g2, lay.swap, lay.spread, di, dev, st);
}

// ---------------------------------------------------------------- decode-sized prologue
// Router (optional) + counting sort + quantisation in one cluster launch
// (decode_prologue_kernel) for batches of at most kDpMaxTokens tokens.
// Weight tiles per CTA that GEMM1 pulls into L2 while the decode prologue runs (three
// measured best on B200 at T = 32: ~4 us off the layer; six thrash L2).
constexpr int kPrefetchTilesAfterPrologue = 3;

struct RouterArgs {
  const void* weight; const void* bias; int64_t* ridx_out; void* scores_out; float* rw_out;
};

bool decode_prologue_fits(int64_t T, int k, int E, int64_t H, bool router, size_t* smem, int* slice) {
  if (T < 1 || T > kDpMaxTokens || T * k > kDpMaxAssign || H % 8 != 0) return false;
  const int nchunks = static_cast<int>((H + 63) / 64);
  *slice = (nchunks + kDpCluster - 1) / kDpCluster;
  *slice += *slice & 1;                       // whole 128-wide k-atoms per rank
  const DpLayout Ld = dp_layout(static_cast<int>(T), E, k, *slice, router);
  *smem = Ld.total;
  return Ld.total <= kDpMaxSmem;
}

int run_decode_prologue(const void* hidden, const RouterArgs* ra, const int64_t* ridx, const float* rw, int64_t T,
                        int k, int E, int64_t H, int64_t I, const WsPtrs& w, bool spread, void* zero_out,
                        int* status, size_t smem, int slice, int dev, cudaStream_t st) {
  static uint64_t attr_done = 0;   // one bit per device
  static std::mutex mu;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!(attr_done & (1ull << dev))) {
      GPTOSS_CUDA(cudaFuncSetAttribute(decode_prologue_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(kDpMaxSmem)));
      attr_done |= (1ull << dev);
    }
  }
  DecodePrologueParams p{};
  p.x = static_cast<const __nv_bfloat16*>(hidden);
  if (ra != nullptr) {
    p.w = static_cast<const __nv_bfloat16*>(ra->weight);
    p.bias = static_cast<const __nv_bfloat16*>(ra->bias);
    p.ridx_out = ra->ridx_out;
    p.scores_out = static_cast<__nv_bfloat16*>(ra->scores_out);
    p.rw_out = ra->rw_out;
  } else {
    p.ridx_in = ridx;
    p.rw_in = rw;
  }
  p.T = static_cast<int>(T); p.H = static_cast<int>(H); p.E = E; p.K = k;
  p.slice_chunks = slice;
  p.sorted_token = w.sorted_token; p.sorted_expert = w.sorted_expert; p.sorted_weight = w.sorted_weight;
  p.counts = w.counts; p.offsets = w.offsets; p.sf_offsets_a = w.sfoff_a; p.sf_offsets_b = w.sfoff_b;
  p.act_codes = w.act_codes; p.act_sf = w.act_sf; p.inter_sf = w.inter_sf;
  p.g4_a = static_cast<int>(pad128(H) / 128); p.g4_b = static_cast<int>(pad128(I) / 128);
  p.spread = spread ? 1 : 0;
  p.zero_out = static_cast<__nv_bfloat16*>(zero_out);
  p.err = status;
  return launch_pdl_cluster(decode_prologue_kernel, dim3(kDpCluster), dim3(kDpThreads), smem, st,
                            dim3(kDpCluster, 1, 1), p);
}

// ---------------------------------------------------------------- one-launch decode layer
// decode_layer_kernel runs the whole layer (router or given routing, sort, quantisation,
// GEMM1, GEMM2) as one persistent launch behind a one-CTA reset of its synchronisation
// words. It serves batches on the 16-row-chunk weights-on-M layout (SPREAD) that fit its
// shared-memory routing state; gptoss_set_decode_layer_kernel(0) turns it off (the
// three-launch path then runs).
std::atomic<int> g_decode_layer_enabled{1};

bool decode_layer_fits(int64_t T, int k, int E, int64_t H, int64_t I, GemmLayout lay, int sms) {
  return g_decode_layer_enabled.load(std::memory_order_relaxed) != 0 && lay.swap && lay.spread && T >= 1 &&
         T <= kDlMaxTokens && T * k <= kDlMaxAssign && E <= kDlMaxExperts && H % 32 == 0 && I % 32 == 0 &&
         static_cast<size_t>(T) * (2 * E + k) * sizeof(float) <= (DlCfg::kStages - kDlPreStages) * DlCfg::kStageBytes &&
         sms >= 1;
}

int run_decode_layer(const void* hidden, const RouterArgs* ra, const int64_t* ridx, const float* rw, int64_t T, int k,
                     int E, int64_t H, int64_t I, const ExpertWeights& wt, float sw_alpha, float sw_limit, void* out,
                     uint8_t* ws, const Workspace& L, int* status, const DeviceInfo& di, int dev, cudaStream_t st,
                     bool out_prefilled = false) {
  const WsPtrs w = ws_ptrs(ws, L);
  const int64_t A = T * k, Kh = pad128(H), Ki = pad128(I);
  CUtensorMap ta, ti, tgu, tdn;
  GPTOSS_TRY(make_act_map(&ta, w.act_codes, A, H, DlCfg::kActRows));
  GPTOSS_TRY(make_act_map(&ti, w.inter_codes, A, I, DlCfg::kActRows));
  GPTOSS_TRY(make_wgt_map(&tgu, wt.gu_data, E, 2 * I, Kh, DlCfg::kWgtRowsCta));
  GPTOSS_TRY(make_wgt_map(&tdn, wt.dn_data, E, H, Ki, DlCfg::kWgtRowsCta));
  static uint64_t attr_done = 0;   // one bit per device
  static std::mutex mu;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!(attr_done & (1ull << dev))) {
      GPTOSS_CUDA(cudaFuncSetAttribute(decode_layer_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(dl_smem_bytes())));
      attr_done |= (1ull << dev);
    }
  }
  DecodeLayerParams p{};
  p.x = static_cast<const __nv_bfloat16*>(hidden);
  if (ra != nullptr) {
    p.router_w = static_cast<const __nv_bfloat16*>(ra->weight);
    p.router_b = static_cast<const __nv_bfloat16*>(ra->bias);
    p.ridx_out = ra->ridx_out;
    p.scores_out = static_cast<__nv_bfloat16*>(ra->scores_out);
    p.rw_out = ra->rw_out;
  } else {
    p.ridx_in = ridx;
    p.rw_in = rw;
  }
  p.T = static_cast<int>(T); p.H = static_cast<int>(H); p.I = static_cast<int>(I); p.E = E; p.K = k;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_prefilled = out_prefilled ? 1 : 0;
  p.logits = reinterpret_cast<float*>(ws + L.dl_logits);
  p.sorted_token = w.sorted_token; p.sorted_expert = w.sorted_expert; p.sorted_weight = w.sorted_weight;
  p.counts = w.counts; p.offsets = w.offsets; p.sf_offsets_a = w.sfoff_a; p.sf_offsets_b = w.sfoff_b;
  p.act_codes = w.act_codes; p.act_sf = w.act_sf; p.inter_codes = w.inter_codes; p.inter_sf = w.inter_sf;
  p.sync = reinterpret_cast<int32_t*>(ws + L.dl_sync);
  p.sfb_gu = wt.gu_scales; p.sfb_stride_gu = wt.ldb_gu; p.bias_gu = wt.gu_bias;
  p.sfb_dn = wt.dn_scales; p.sfb_stride_dn = wt.ldb_dn; p.bias_dn = wt.dn_bias;
  p.swiglu_alpha = sw_alpha; p.swiglu_limit = sw_limit;
  p.kb1 = static_cast<int>(Kh / 128); p.kb2 = static_cast<int>(Ki / 128);
  p.n_tiles1 = static_cast<int>((2 * I + DlCfg::kWgtRows - 1) / DlCfg::kWgtRows);
  p.n_tiles2 = static_cast<int>((H + DlCfg::kWgtRows - 1) / DlCfg::kWgtRows);
  p.err = status;
  // the epilogue parameters of the two GEMMs (shared-memory tables are filled in on the GPU)
  GemmParams g1{};
  g1.num_experts = E; g1.N = static_cast<int>(2 * I); g1.K = static_cast<int>(Kh); g1.num_kb = p.kb1;
  g1.err = status; g1.out = w.inter_codes; g1.ld_out = I; g1.bias = wt.gu_bias; g1.out_sf = w.inter_sf;
  g1.out_g4 = p.kb2; g1.out_features = static_cast<int>(I);
  g1.swiglu_alpha = sw_alpha; g1.swiglu_limit = sw_limit;
  GemmParams g2{};
  g2.num_experts = E; g2.N = static_cast<int>(H); g2.K = static_cast<int>(Ki); g2.num_kb = p.kb2;
  g2.err = status; g2.out = out; g2.ld_out = H; g2.bias = wt.dn_bias;
  g2.swiglu_alpha = sw_alpha; g2.swiglu_limit = sw_limit;
  GPTOSS_TRY(launch_pdl(decode_reset_kernel, dim3(1), dim3(256), 0, st, p.sync, dl_sync_words(E)));
  return launch_pdl(decode_layer_kernel<false>, dim3(di.sms), dim3(DlCfg::kThreads), dl_smem_bytes(), st, ta, ti, tgu, tdn,
                    p, g1, g2);
}

// route -> gather/quant -> GEMM1 -> GEMM2 on a routed batch. With `ra` the router runs
// first (inside the decode prologue, or as router_launch, which also zeroes `out`).
int experts_pipeline(const void* hidden, const int64_t* ridx, const float* rw, int64_t T, int k, int E,
                     int64_t H, int64_t I, const ExpertWeights& wt, float sw_alpha, float sw_limit, void* out,
                     uint8_t* ws, const Workspace& L, int mode, int* status, const DeviceInfo& di, int dev,
                     cudaStream_t st, const RouterArgs* ra = nullptr, bool out_prefilled = false) {
  const WsPtrs w = ws_ptrs(ws, L);
  const GemmLayout lay = pick_layout(mode, T * k, E);
  if (decode_layer_fits(T, k, E, H, I, lay, di.sms))
    return run_decode_layer(hidden, ra, ridx, rw, T, k, E, H, I, wt, sw_alpha, sw_limit, out, ws, L, status, di, dev,
                            st, out_prefilled);
  size_t smem = 0;
  int slice = 0;
  // While the one-launch decode prologue runs on kDpCluster SMs, GEMM1 (launched behind it
  // with programmatic serialisation) pulls its first weight tiles into L2.
  int prefetch = 0;
  if (decode_prologue_fits(T, k, E, H, ra != nullptr, &smem, &slice)) {
    GPTOSS_TRY(run_decode_prologue(hidden, ra, ridx, rw, T, k, E, H, I, w, lay.spread, out_prefilled ? nullptr : out,
                                   status, smem, slice, dev, st));
    prefetch = kPrefetchTilesAfterPrologue;
  } else {
    if (ra != nullptr) {
      GPTOSS_TRY(router_launch(hidden, ra->weight, ra->bias, T, H, E, k, ra->ridx_out, ra->scores_out, ra->rw_out,
                               nullptr, out_prefilled ? nullptr : out, H, di.sms, dev, st));
      ridx = ra->ridx_out;
      rw = ra->rw_out;
    }
    GPTOSS_TRY(stage_route_quant(hidden, ridx, rw, T, k, E, H, I, w, lay.spread, status, st));
    if (ra == nullptr && !out_prefilled)
      GPTOSS_CUDA(cudaMemsetAsync(out, 0, static_cast<size_t>(T * H) * sizeof(__nv_bfloat16), st));
  }
  GPTOSS_TRY(stage_gemm1(T * k, E, H, I, wt, sw_alpha, sw_limit, w, lay, status, di, dev, st, prefetch));
  return stage_gemm2(T * k, E, H, I, wt, out, w, lay, status, di, dev, st);
}

int check_dims(int64_t T, int k, int E, int64_t H, int64_t I) {
  GPTOSS_CHECK(T >= 0, "num_tokens must be >= 0");
  GPTOSS_CHECK(k >= 1 && k <= kMaxTopK, "top_k must be in [1, %d]", kMaxTopK);
  GPTOSS_CHECK(E >= 1 && E <= kMaxExperts, "num_experts must be in [1, %d]", kMaxExperts);
  GPTOSS_CHECK(k <= E, "top_k > num_experts");
  GPTOSS_CHECK(H > 0 && H % 32 == 0 && I > 0 && I % 32 == 0, "hidden/intermediate sizes must be multiples of 32");
  GPTOSS_CHECK(T * k < (1LL << 31), "too many assignments");
  return GPTOSS_OK;
}

// ---------------------------------------------------------------- no-allocation forward
// Scratch of gptoss_moe_experts_forward_noalloc. It is a module global, so every GPU
// that loads this library holds GPTOSS_NOALLOC_SCRATCH_BYTES of it until the process
// exits. Host code cannot use the symbol as a device address: the address is looked up
// once per device with cudaGetSymbolAddress while that device is current.
static __device__ __align__(256) uint8_t g_noalloc_scratch[GPTOSS_NOALLOC_SCRATCH_BYTES];

std::mutex g_noalloc_mu;
uint8_t* g_noalloc_ptr[kMaxDevices] = {};

int noalloc_scratch(int dev, uint8_t** out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess)
      return fail(GPTOSS_ERR_CUDA, "cudaGetSymbolAddress(no-alloc scratch) failed on device %d: %s", dev,
                  cudaGetErrorString(e));
    g_noalloc_ptr[dev] = static_cast<uint8_t*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return GPTOSS_OK;
}

}  // namespace

// ======================================================================= C ABI
extern "C" {

const char* gptoss_last_error(void) { return g_last_error.c_str(); }

int gptoss_abi_version(void) { return 2; }

int gptoss_set_decode_layer_kernel(int enable) {
  return g_decode_layer_enabled.exchange(enable != 0 ? 1 : 0, std::memory_order_relaxed);
}

uint64_t gptoss_kernel_launch_count(void) { return g_kernel_launches.load(std::memory_order_relaxed); }

int gptoss_moe_gemm_layout(int gemm_mode, int64_t rows, int num_experts) {
  if (gemm_mode < 0 || gemm_mode > 3 || rows < 0 || num_experts < 1) return -1;
  const GemmLayout lay = pick_layout(gemm_mode, rows, num_experts);
  return !lay.swap ? GPTOSS_GEMM_TOKENS_M : (lay.spread ? GPTOSS_GEMM_SWAP : GPTOSS_GEMM_SWAP_WIDE);
}

int gptoss_read_status(int32_t* status_dev, int32_t* status_host, void* stream) {
  GPTOSS_CHECK(status_host != nullptr, "status_host is null");
  DeviceInfo di;
  GPTOSS_TRY(bind_device(status_dev, "status", &di));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  GPTOSS_CUDA(cudaMemcpyAsync(status_host, status_dev, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
  GPTOSS_CUDA(cudaMemsetAsync(status_dev, 0, sizeof(int32_t), st));
  GPTOSS_CUDA(cudaStreamSynchronize(st));
  return GPTOSS_OK;
}

int gptoss_fused_moe_routing(const int64_t* router_indices, const float* routing_weights, int64_t num_tokens,
                             int top_k, int num_experts, int64_t* sorted_token_idx, int64_t* sorted_expert_idx,
                             float* sorted_weights, int32_t* expert_counts, int32_t* expert_offsets,
                             int32_t* status_dev, void* stream) {
  NvtxRange nvtx_range("gptoss_fused_moe_routing");
  GPTOSS_CHECK(num_tokens >= 0 && top_k >= 1 && num_experts >= 1 && num_experts <= kMaxExperts,
               "fused_moe_routing: bad sizes (T=%lld k=%d E=%d)", (long long)num_tokens, top_k, num_experts);
  GPTOSS_CHECK(num_tokens * top_k < (1LL << 31), "fused_moe_routing: too many assignments");
  DeviceInfo di;
  GPTOSS_TRY(bind_device(expert_counts, "expert_counts", &di));
  GPTOSS_CHECK(expert_offsets != nullptr, "expert_offsets is null");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t A = num_tokens * top_k;
  if (A > 0) {
    GPTOSS_CHECK(router_indices && routing_weights && sorted_token_idx && sorted_expert_idx && sorted_weights,
                 "fused_moe_routing: null pointer");
  }
  RouteSortParams rp{};
  rp.router_indices = router_indices; rp.routing_weights = routing_weights;
  rp.A = static_cast<int>(A); rp.K = top_k; rp.E = num_experts;
  rp.sorted_token = sorted_token_idx; rp.sorted_expert = sorted_expert_idx; rp.sorted_weight = sorted_weights;
  rp.counts = expert_counts; rp.offsets = expert_offsets;
  rp.err = status_dev ? status_dev : di.status_sink;
  return launch_pdl(route_sort_kernel, dim3(num_experts), dim3(1024), 0, st, rp);
}

int gptoss_router_topk(const void* hidden, const void* weight, const void* bias, int64_t num_tokens,
                       int64_t hidden_size, int num_experts, int top_k, int64_t* router_indices, void* router_scores,
                       float* routing_weights_f32, void* logits, void* stream) {
  NvtxRange nvtx_range("gptoss_router_topk");
  GPTOSS_CHECK(num_tokens >= 0, "router: num_tokens < 0");
  GPTOSS_CHECK(hidden_size > 0 && hidden_size % 8 == 0, "router: hidden_size must be a positive multiple of 8");
  GPTOSS_CHECK(num_experts >= 1 && num_experts <= kMaxExperts, "router: num_experts must be in [1, %d]", kMaxExperts);
  GPTOSS_CHECK(top_k >= 1 && top_k <= kMaxTopK && top_k <= num_experts, "router: bad top_k %d", top_k);
  DeviceInfo di;
  GPTOSS_TRY(bind_device(weight, "router weight", &di));
  GPTOSS_CHECK(bias != nullptr && router_indices != nullptr, "router: null pointer");
  if (num_tokens == 0) return GPTOSS_OK;
  GPTOSS_CHECK(hidden != nullptr && aligned(hidden, 16) && aligned(weight, 16), "router: inputs must be 16-byte aligned");
  int dev = 0;
  GPTOSS_CUDA(cudaGetDevice(&dev));
  return router_launch(hidden, weight, bias, num_tokens, hidden_size, num_experts, top_k, router_indices,
                       router_scores, routing_weights_f32, logits, nullptr, 0, di.sms, dev,
                       static_cast<cudaStream_t>(stream));
}

}  // extern "C"

namespace {
template <bool PAIR, bool NVF4>
int launch_mma_peak(int n, int iters, int* err, const DeviceInfo& di, int dev, cudaStream_t st) {
  // more than half of the shared memory per CTA: one CTA (and one 512-column TMEM
  // allocation) per SM
  const size_t smem = 120u * 1024u;
  static_assert(kMpSmemBytes <= 120u * 1024u, "peak kernel operands");
  static uint64_t attr_done = 0;   // one bit per device
  static std::mutex mu;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!(attr_done & (1ull << dev))) {
      GPTOSS_CUDA(cudaFuncSetAttribute(mma_peak_kernel<PAIR, NVF4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem)));
      attr_done |= (1ull << dev);
    }
  }
  if (PAIR)
    return launch_pdl_cluster(mma_peak_kernel<PAIR, NVF4>, dim3(2 * (di.sms / 2)), dim3(128), smem, st,
                              dim3(2, 1, 1), n, iters, err);
  return launch_pdl(mma_peak_kernel<PAIR, NVF4>, dim3(di.sms), dim3(128), smem, st, n, iters, err);
}
}  // namespace

extern "C" {

int gptoss_mma_peak(int kind, int pair, int n, int iters, int32_t* status_dev, void* stream) {
  NvtxRange nvtx_range("gptoss_mma_peak");
  GPTOSS_CHECK(kind == 0 || kind == 1, "mma_peak: kind must be 0 (mxf8f6f4) or 1 (mxf4nvf4)");
  GPTOSS_CHECK(n >= 16 && n <= 256 && n % 16 == 0, "mma_peak: n must be a multiple of 16 in [16, 256]");
  GPTOSS_CHECK(iters >= 1, "mma_peak: iters must be >= 1");
  int dev = 0;
  GPTOSS_CUDA(cudaGetDevice(&dev));
  DeviceInfo di;
  {
    // bind_device needs a device pointer; the status sink of the current device is one
    void* sink = nullptr;
    GPTOSS_CUDA(cudaGetSymbolAddress(&sink, g_status_sink));
    GPTOSS_TRY(bind_device(sink, "status sink", &di));
  }
  int* err = status_dev ? status_dev : di.status_sink;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (kind == 1)
    return pair ? launch_mma_peak<true, true>(n, iters, err, di, dev, st)
                : launch_mma_peak<false, true>(n, iters, err, di, dev, st);
  return pair ? launch_mma_peak<true, false>(n, iters, err, di, dev, st)
              : launch_mma_peak<false, false>(n, iters, err, di, dev, st);
}

int gptoss_router_topk_from_logits(const void* logits, int64_t num_tokens, int num_experts, int top_k,
                                   int64_t* router_indices, void* router_scores, float* routing_weights_f32,
                                   void* stream) {
  NvtxRange nvtx_range("gptoss_router_topk_from_logits");
  GPTOSS_CHECK(num_tokens >= 0 && num_tokens < (1LL << 31), "router_topk_from_logits: bad num_tokens");
  GPTOSS_CHECK(num_experts >= 1 && num_experts <= kMaxExperts, "router_topk_from_logits: num_experts must be in [1, %d]",
               kMaxExperts);
  GPTOSS_CHECK(top_k >= 1 && top_k <= kMaxTopK && top_k <= num_experts, "router_topk_from_logits: bad top_k %d", top_k);
  if (num_tokens == 0) return GPTOSS_OK;
  DeviceInfo di;
  GPTOSS_TRY(bind_device(logits, "logits", &di));
  GPTOSS_CHECK(router_indices != nullptr, "router_topk_from_logits: null router_indices");
  const size_t smem = 32u * static_cast<size_t>(num_experts + 1) * sizeof(float);
  return launch_pdl(router_topk_logits_kernel, dim3(static_cast<unsigned>((num_tokens + 31) / 32)), dim3(32), smem,
                    static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(logits),
                    static_cast<int>(num_tokens), num_experts, top_k, router_indices,
                    static_cast<__nv_bfloat16*>(router_scores), routing_weights_f32);
}

int gptoss_quantize_fp8(const void* x, int dtype, int64_t rows, int64_t cols, uint8_t* codes, uint8_t* scales,
                        void* stream) {
  NvtxRange nvtx_range("gptoss_quantize_fp8");
  GPTOSS_CHECK(rows >= 0 && cols > 0 && cols % 32 == 0, "quantize: K=%lld must be a positive multiple of 32",
               (long long)cols);
  GPTOSS_CHECK(dtype == GPTOSS_DTYPE_BF16 || dtype == GPTOSS_DTYPE_F32, "quantize: dtype must be bf16 or f32");
  if (rows == 0) return GPTOSS_OK;
  DeviceInfo di;
  GPTOSS_TRY(bind_device(x, "x", &di));
  GPTOSS_CHECK(codes && scales && aligned(x, 16) && aligned(codes, 16), "quantize: null or misaligned pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int tpr = quant_threads_per_row(static_cast<int>(cols));
  const int rpb = 256 / tpr;
  const int blocks = static_cast<int>((rows + rpb - 1) / rpb);
  const int64_t* no_i64 = nullptr;
  const int32_t* no_i32 = nullptr;
  uint8_t* no_u8 = nullptr;
  if (dtype == GPTOSS_DTYPE_BF16)
    return launch_pdl(gather_quant_kernel<__nv_bfloat16>, dim3(blocks), dim3(tpr * rpb), 0, st,
                      static_cast<const __nv_bfloat16*>(x), rows, static_cast<int>(cols), tpr, no_i64, no_i64, no_i32,
                      no_i32, 0, 0, codes, no_u8, scales);
  return launch_pdl(gather_quant_kernel<float>, dim3(blocks), dim3(tpr * rpb), 0, st, static_cast<const float*>(x), rows,
                    static_cast<int>(cols), tpr, no_i64, no_i64, no_i32, no_i32, 0, 0, codes, no_u8, scales);
}

int gptoss_swiglu(const void* x, int dtype, int64_t rows, int64_t cols, void* out, float alpha, float limit,
                  void* stream) {
  NvtxRange nvtx_range("gptoss_swiglu");
  GPTOSS_CHECK(rows >= 0 && cols > 0 && cols % 2 == 0, "swiglu: last dimension must be even");
  GPTOSS_CHECK(dtype == GPTOSS_DTYPE_BF16 || dtype == GPTOSS_DTYPE_F32, "swiglu: dtype must be bf16 or f32");
  if (rows == 0) return GPTOSS_OK;
  DeviceInfo di;
  GPTOSS_TRY(bind_device(x, "x", &di));
  GPTOSS_CHECK(out != nullptr, "swiglu: null output");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t n = cols / 2;
  const int blocks = static_cast<int>(std::min<int64_t>((rows * n + 255) / 256, 8192));
  if (dtype == GPTOSS_DTYPE_F32)
    swiglu_kernel<float><<<blocks, 256, 0, st>>>(static_cast<const float*>(x), rows, n, static_cast<float*>(out),
                                                 alpha, limit);
  else
    swiglu_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), rows, n,
                                                         static_cast<__nv_bfloat16*>(out), alpha, limit);
  GPTOSS_CUDA(cudaGetLastError());
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
  return GPTOSS_OK;
}

int64_t gptoss_blocked_scales_bytes(int64_t rows, int64_t k) {
  if (rows < 0 || k <= 0) return -1;
  return blocked_sf_cosize(rows, static_cast<int>(k / 32));
}

int gptoss_convert_scales_blocked(const uint8_t* scales_rowmajor, int64_t rows, int64_t k, uint8_t* blocked,
                                  int64_t blocked_bytes, void* stream) {
  GPTOSS_CHECK(rows >= 0 && k > 0 && k % 32 == 0, "convert_scales: K=%lld must be a multiple of 32", (long long)k);
  const int G = static_cast<int>(k / 32);
  const int64_t need = blocked_sf_cosize(rows, G);
  GPTOSS_CHECK(blocked_bytes >= need, "convert_scales: output holds %lld bytes, need %lld", (long long)blocked_bytes,
               (long long)need);
  if (need == 0) return GPTOSS_OK;
  DeviceInfo di;
  GPTOSS_TRY(bind_device(blocked, "blocked", &di));
  GPTOSS_CHECK(scales_rowmajor != nullptr, "convert_scales: null input");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int g4 = (G + 3) / 4;
  const int64_t total = ((rows + 127) / 128 * 128) * g4 * 4;
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 4096));
  convert_scales_kernel<<<blocks, 256, 0, st>>>(scales_rowmajor, rows, G, g4, blocked);
  GPTOSS_CUDA(cudaGetLastError());
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
  return GPTOSS_OK;
}

int64_t gptoss_batch_blocked_scales_capacity(int64_t total_rows, int num_experts, int64_t k) {
  if (total_rows < 0 || num_experts < 1 || k <= 0) return -1;
  return ((total_rows + 127) / 128 + num_experts) * ((k / 32 + 3) / 4) * 512;
}

int gptoss_batch_convert_a_scales(const uint8_t* scales_rowmajor, const int32_t* expert_counts,
                                  const int32_t* expert_offsets, int num_experts, int64_t k, uint8_t* blocked,
                                  int64_t capacity, int32_t* sf_offsets, void* stream) {
  GPTOSS_CHECK(num_experts >= 1 && num_experts <= kMaxExperts, "batch_convert: bad num_experts");
  GPTOSS_CHECK(k > 0 && k % 32 == 0, "batch_convert: K must be a multiple of 32");
  DeviceInfo di;
  GPTOSS_TRY(bind_device(sf_offsets, "sf_offsets", &di));
  GPTOSS_CHECK(expert_counts && expert_offsets && blocked && capacity >= 0, "batch_convert: null pointer");
  const int G = static_cast<int>(k / 32);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  batch_convert_scales_kernel<<<num_experts, 256, 0, st>>>(scales_rowmajor, expert_counts, expert_offsets, num_experts,
                                                           G, (G + 3) / 4, blocked, sf_offsets);
  GPTOSS_CUDA(cudaGetLastError());
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
  return GPTOSS_OK;
}

int gptoss_fp4_group_mm(void* out, const uint8_t* a, int64_t m_total, int64_t lda, const uint8_t* b, int num_experts,
                        int64_t n, int64_t k, const uint8_t* a_blockscale, const uint8_t* b_blockscales,
                        int64_t ldb_blockscale, const float* alphas, const int32_t* problem_sizes,
                        const int32_t* expert_offsets, const int32_t* sf_offsets, int gemm_mode, int32_t* status_dev,
                        void* stream) {
  NvtxRange nvtx_range("gptoss_fp4_group_mm");
  GPTOSS_CHECK(num_experts >= 1 && num_experts <= kMaxExpertsGemm, "fp4_group_mm: num_experts must be in [1, %d]",
               kMaxExpertsGemm);
  GPTOSS_CHECK(k > 0 && k % 128 == 0, "fp4_group_mm: K=%lld must be a multiple of 128 (pad with pad_k_to_tile)",
               (long long)k);
  GPTOSS_CHECK(n > 0 && n % 8 == 0 && n < (1LL << 31), "fp4_group_mm: N=%lld must be a positive multiple of 8",
               (long long)n);
  GPTOSS_CHECK(m_total >= 0 && lda > 0 && lda <= k && lda % 16 == 0, "fp4_group_mm: a must be [M, lda<=K], lda %% 16 == 0");
  GPTOSS_CHECK(gemm_mode >= 0 && gemm_mode <= 3, "fp4_group_mm: bad gemm_mode");
  DeviceInfo di;
  GPTOSS_TRY(bind_device(b, "b", &di));
  GPTOSS_CHECK(aligned(b, 32), "fp4_group_mm: b must be 32-byte aligned");
  GPTOSS_CHECK(ldb_blockscale >= blocked_sf_cosize(n, static_cast<int>(k / 32)) && ldb_blockscale % 16 == 0,
               "fp4_group_mm: b_blockscales holds %lld bytes per expert, need %lld (multiple of 16)",
               (long long)ldb_blockscale, (long long)blocked_sf_cosize(n, static_cast<int>(k / 32)));
  GPTOSS_CHECK(problem_sizes && expert_offsets && sf_offsets && b_blockscales, "fp4_group_mm: null pointer");
  if (m_total == 0) return GPTOSS_OK;
  GPTOSS_CHECK(a && out && a_blockscale && aligned(a, 16) && aligned(out, 16) && aligned(a_blockscale, 16) &&
                   aligned(b_blockscales, 16),
               "fp4_group_mm: null or misaligned pointer");
  int dev = 0;
  GPTOSS_CUDA(cudaGetDevice(&dev));
  GemmJob job{};
  job.act = a; job.act_rows = m_total; job.lda = lda; job.wgt = b;
  job.p.num_experts = num_experts; job.p.N = static_cast<int>(n); job.p.K = static_cast<int>(k);
  job.p.num_kb = static_cast<int>(k / 128); job.p.m_sizes = problem_sizes; job.p.m_stride = 3;
  job.p.row_offsets = expert_offsets; job.p.sfa_offsets = sf_offsets; job.p.sfa = a_blockscale;
  job.p.sfb = b_blockscales; job.p.sfb_stride = ldb_blockscale;
  job.p.err = status_dev ? status_dev : di.status_sink;
  job.p.out = out; job.p.ld_out = n; job.p.alphas = alphas;
  return run_gemm<kEpiPlain>(job, pick_swap(gemm_mode, m_total, num_experts, 48), false, di, dev,
                             static_cast<cudaStream_t>(stream));
}

int gptoss_fp4_group_mm_w4a4(void* out, const uint8_t* a, int64_t m_total, int64_t lda, const uint8_t* b,
                             int num_experts, int64_t n, int64_t k, const uint8_t* a_blockscale,
                             const uint8_t* b_blockscales, int64_t ldb_blockscale, const float* alphas,
                             const int32_t* problem_sizes, const int32_t* expert_offsets, const int32_t* sf_offsets,
                             int gemm_mode, int32_t* status_dev, void* stream) {
  NvtxRange nvtx_range("gptoss_fp4_group_mm_w4a4");
  GPTOSS_CHECK(num_experts >= 1 && num_experts <= kMaxExpertsGemm,
               "fp4_group_mm_w4a4: num_experts must be in [1, %d]", kMaxExpertsGemm);
  GPTOSS_CHECK(k > 0 && k % 64 == 0 && k < (1LL << 30),
               "fp4_group_mm_w4a4: K=%lld must be a positive multiple of 64 (one 16-code scale atom)", (long long)k);
  GPTOSS_CHECK(n > 0 && n % 8 == 0 && n < (1LL << 31), "fp4_group_mm_w4a4: N=%lld must be a positive multiple of 8",
               (long long)n);
  GPTOSS_CHECK(m_total >= 0 && lda == k / 2, "fp4_group_mm_w4a4: a must be [M, K/2] packed E2M1");
  GPTOSS_CHECK(gemm_mode >= 0 && gemm_mode <= 3, "fp4_group_mm_w4a4: bad gemm_mode");
  DeviceInfo di;
  GPTOSS_TRY(bind_device(b, "b", &di));
  GPTOSS_CHECK(aligned(b, 16), "fp4_group_mm_w4a4: b must be 16-byte aligned");
  GPTOSS_CHECK(ldb_blockscale >= blocked_sf_cosize(n, static_cast<int>(k / 16)) && ldb_blockscale % 16 == 0,
               "fp4_group_mm_w4a4: b_blockscales holds %lld bytes per expert, need %lld (multiple of 16)",
               (long long)ldb_blockscale, (long long)blocked_sf_cosize(n, static_cast<int>(k / 16)));
  GPTOSS_CHECK(problem_sizes && expert_offsets && sf_offsets && b_blockscales, "fp4_group_mm_w4a4: null pointer");
  if (m_total == 0) return GPTOSS_OK;
  GPTOSS_CHECK(a && out && a_blockscale && aligned(a, 16) && aligned(out, 16) && aligned(a_blockscale, 16) &&
                   aligned(b_blockscales, 16),
               "fp4_group_mm_w4a4: null or misaligned pointer");
  int dev = 0;
  GPTOSS_CUDA(cudaGetDevice(&dev));
  GemmJob job{};
  job.act = a; job.act_rows = m_total; job.lda = lda; job.wgt = b;
  job.p.num_experts = num_experts; job.p.N = static_cast<int>(n); job.p.K = static_cast<int>(k);
  job.p.num_kb = static_cast<int>((k + 255) / 256); job.p.m_sizes = problem_sizes; job.p.m_stride = 3;
  job.p.row_offsets = expert_offsets; job.p.sfa_offsets = sf_offsets; job.p.sfa = a_blockscale;
  job.p.sfb = b_blockscales; job.p.sfb_stride = ldb_blockscale;
  job.p.err = status_dev ? status_dev : di.status_sink;
  job.p.out = out; job.p.ld_out = n; job.p.alphas = alphas;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (pick_swap(gemm_mode, m_total, num_experts, 48))
    return launch_gemm<true, false, kEpiPlain, false, true>(job, di, dev, st);
  return launch_gemm<false, false, kEpiPlain, false, true>(job, di, dev, st);
}

size_t gptoss_moe_workspace_bytes(int64_t num_tokens, int top_k, int num_experts, int64_t hidden_size,
                                  int64_t intermediate_size) {
  if (num_tokens < 0 || top_k < 1 || num_experts < 1 || hidden_size <= 0 || intermediate_size <= 0) return 0;
  return plan_workspace(num_tokens, top_k, num_experts, hidden_size, intermediate_size).total;
}

int gptoss_moe_experts_forward(const void* hidden, const int64_t* router_indices, const float* routing_weights,
                               int64_t num_tokens, int top_k, int num_experts, int64_t hidden_size,
                               int64_t intermediate_size, const uint8_t* gate_up_data, const uint8_t* gate_up_scales,
                               int64_t ldb_gate_up, const float* gate_up_bias, const uint8_t* down_data,
                               const uint8_t* down_scales, int64_t ldb_down, const float* down_bias,
                               float swiglu_alpha, float swiglu_limit, void* out, void* workspace,
                               size_t workspace_bytes, int gemm_mode, int32_t* status_dev, void* stream) {
  NvtxRange nvtx_range("gptoss_moe_experts_forward");
  GPTOSS_TRY(check_dims(num_tokens, top_k, num_experts, hidden_size, intermediate_size));
  GPTOSS_CHECK(gemm_mode >= 0 && gemm_mode <= 3, "bad gemm_mode");
  DeviceInfo di;
  GPTOSS_TRY(bind_device(gate_up_data, "gate_up_proj_data", &di));
  ExpertWeights w{gate_up_data, gate_up_scales, ldb_gate_up, gate_up_bias,
                  down_data, down_scales, ldb_down, down_bias};
  GPTOSS_TRY(check_expert_weights(w, hidden_size, intermediate_size, num_experts));
  if (num_tokens == 0) return GPTOSS_OK;
  GPTOSS_CHECK(hidden && router_indices && routing_weights && out && workspace, "experts_forward: null pointer");
  GPTOSS_CHECK(aligned(hidden, 16) && aligned(out, 16) && aligned(workspace, 256), "experts_forward: misaligned pointer");
  const Workspace L = plan_workspace(num_tokens, top_k, num_experts, hidden_size, intermediate_size);
  if (workspace_bytes < L.total)
    return fail(GPTOSS_ERR_WORKSPACE, "workspace has %zu bytes, need %zu", workspace_bytes, L.total);
  int dev = 0;
  GPTOSS_CUDA(cudaGetDevice(&dev));
  return experts_pipeline(hidden, router_indices, routing_weights, num_tokens, top_k, num_experts, hidden_size,
                          intermediate_size, w, swiglu_alpha, swiglu_limit, out, static_cast<uint8_t*>(workspace), L,
                          gemm_mode, status_dev ? status_dev : di.status_sink, di, dev,
                          static_cast<cudaStream_t>(stream));
}

int gptoss_moe_layer_forward(const void* hidden, const void* router_weight, const void* router_bias,
                             int64_t num_tokens, int top_k, int num_experts, int64_t hidden_size,
                             int64_t intermediate_size, const uint8_t* gate_up_data, const uint8_t* gate_up_scales,
                             int64_t ldb_gate_up, const float* gate_up_bias, const uint8_t* down_data,
                             const uint8_t* down_scales, int64_t ldb_down, const float* down_bias, float swiglu_alpha,
                             float swiglu_limit, void* out, int64_t* router_indices_out, void* router_scores_out,
                             void* workspace, size_t workspace_bytes, int gemm_mode, int32_t* status_dev,
                             void* stream) {
  NvtxRange nvtx_range("gptoss_moe_layer_forward");
  GPTOSS_TRY(check_dims(num_tokens, top_k, num_experts, hidden_size, intermediate_size));
  GPTOSS_CHECK(gemm_mode >= 0 && gemm_mode <= 3, "bad gemm_mode");
  GPTOSS_CHECK(hidden_size % 8 == 0, "hidden size must be a multiple of 8");
  DeviceInfo di;
  GPTOSS_TRY(bind_device(gate_up_data, "gate_up_proj_data", &di));
  ExpertWeights w{gate_up_data, gate_up_scales, ldb_gate_up, gate_up_bias,
                  down_data, down_scales, ldb_down, down_bias};
  GPTOSS_TRY(check_expert_weights(w, hidden_size, intermediate_size, num_experts));
  if (num_tokens == 0) return GPTOSS_OK;
  GPTOSS_CHECK(hidden && router_weight && router_bias && out && workspace, "layer_forward: null pointer");
  GPTOSS_CHECK(aligned(hidden, 16) && aligned(router_weight, 16) && aligned(out, 16) && aligned(workspace, 256),
               "layer_forward: misaligned pointer");
  const Workspace L = plan_workspace(num_tokens, top_k, num_experts, hidden_size, intermediate_size);
  if (workspace_bytes < L.total)
    return fail(GPTOSS_ERR_WORKSPACE, "workspace has %zu bytes, need %zu", workspace_bytes, L.total);
  int dev = 0;
  GPTOSS_CUDA(cudaGetDevice(&dev));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int64_t* ridx = router_indices_out ? router_indices_out : reinterpret_cast<int64_t*>(ws + L.router_idx);
  float* rw = reinterpret_cast<float*>(ws + L.router_w);
  const RouterArgs ra{router_weight, router_bias, ridx, router_scores_out, rw};
  return experts_pipeline(hidden, nullptr, nullptr, num_tokens, top_k, num_experts, hidden_size, intermediate_size,
                          w, swiglu_alpha, swiglu_limit, out, ws, L, gemm_mode,
                          status_dev ? status_dev : di.status_sink, di, dev, st, &ra);
}


size_t gptoss_moe_block_workspace_bytes(int64_t num_tokens, int top_k, int num_experts, int64_t hidden_size,
                                        int64_t intermediate_size) {
  if (num_tokens < 0 || top_k < 1 || num_experts < 1 || hidden_size <= 0 || intermediate_size <= 0) return 0;
  return plan_workspace(num_tokens, top_k, num_experts, hidden_size, intermediate_size).total +
         align256(static_cast<size_t>(num_tokens * hidden_size) * sizeof(__nv_bfloat16));
}

int gptoss_rmsnorm_residual(const void* x, const void* weight, float eps, int64_t num_tokens, int64_t hidden_size,
                            void* xn, void* residual_out, void* stream) {
  NvtxRange nvtx_range("gptoss_rmsnorm_residual");
  GPTOSS_CHECK(num_tokens >= 0 && num_tokens < (1LL << 31), "rmsnorm: bad num_tokens");
  GPTOSS_CHECK(hidden_size > 0 && hidden_size % 8 == 0, "rmsnorm: hidden size must be a multiple of 8");
  if (num_tokens == 0) return GPTOSS_OK;
  GPTOSS_CHECK(x && weight && xn, "rmsnorm: null pointer");
  GPTOSS_CHECK(aligned(x, 16) && aligned(weight, 16) && aligned(xn, 16) && (!residual_out || aligned(residual_out, 16)),
               "rmsnorm: misaligned pointer");
  return launch_pdl(rmsnorm_residual_kernel, dim3(static_cast<unsigned>((num_tokens + 7) / 8)), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(x),
                    static_cast<const __nv_bfloat16*>(weight), eps, static_cast<int>(num_tokens),
                    static_cast<int>(hidden_size), static_cast<__nv_bfloat16*>(xn),
                    static_cast<__nv_bfloat16*>(residual_out));
}

int gptoss_moe_block_forward(const void* hidden, const void* norm_weight, float norm_eps, const void* router_weight,
                             const void* router_bias, int64_t num_tokens, int top_k, int num_experts, int64_t hidden_size,
                             int64_t intermediate_size, const uint8_t* gate_up_data, const uint8_t* gate_up_scales,
                             int64_t ldb_gate_up, const float* gate_up_bias, const uint8_t* down_data,
                             const uint8_t* down_scales, int64_t ldb_down, const float* down_bias, float swiglu_alpha,
                             float swiglu_limit, void* out, int64_t* router_indices_out, void* router_scores_out,
                             void* workspace, size_t workspace_bytes, int gemm_mode, int32_t* status_dev,
                             void* stream) {
  NvtxRange nvtx_range("gptoss_moe_block_forward");
  GPTOSS_TRY(check_dims(num_tokens, top_k, num_experts, hidden_size, intermediate_size));
  GPTOSS_CHECK(gemm_mode >= 0 && gemm_mode <= 3, "bad gemm_mode");
  GPTOSS_CHECK(hidden_size % 8 == 0, "hidden size must be a multiple of 8");
  DeviceInfo di;
  GPTOSS_TRY(bind_device(gate_up_data, "gate_up_proj_data", &di));
  ExpertWeights w{gate_up_data, gate_up_scales, ldb_gate_up, gate_up_bias,
                  down_data, down_scales, ldb_down, down_bias};
  GPTOSS_TRY(check_expert_weights(w, hidden_size, intermediate_size, num_experts));
  if (num_tokens == 0) return GPTOSS_OK;
  GPTOSS_CHECK(hidden && norm_weight && router_weight && router_bias && out && workspace, "block_forward: null pointer");
  GPTOSS_CHECK(aligned(hidden, 16) && aligned(norm_weight, 16) && aligned(router_weight, 16) && aligned(out, 16) &&
                   aligned(workspace, 256),
               "block_forward: misaligned pointer");
  const Workspace L = plan_workspace(num_tokens, top_k, num_experts, hidden_size, intermediate_size);
  const size_t need = gptoss_moe_block_workspace_bytes(num_tokens, top_k, num_experts, hidden_size, intermediate_size);
  if (workspace_bytes < need) return fail(GPTOSS_ERR_WORKSPACE, "workspace has %zu bytes, need %zu", workspace_bytes, need);
  int dev = 0;
  GPTOSS_CUDA(cudaGetDevice(&dev));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* xn = ws + L.total;   // the normalised rows, behind the layer's workspace
  // out = hidden (the residual GEMM2 adds into), xn = RMSNorm(hidden)
  GPTOSS_TRY(gptoss_rmsnorm_residual(hidden, norm_weight, norm_eps, num_tokens, hidden_size, xn, out, stream));
  int64_t* ridx = router_indices_out ? router_indices_out : reinterpret_cast<int64_t*>(ws + L.router_idx);
  float* rw = reinterpret_cast<float*>(ws + L.router_w);
  const RouterArgs ra{router_weight, router_bias, ridx, router_scores_out, rw};
  return experts_pipeline(xn, nullptr, nullptr, num_tokens, top_k, num_experts, hidden_size, intermediate_size,
                          w, swiglu_alpha, swiglu_limit, out, ws, L, gemm_mode,
                          status_dev ? status_dev : di.status_sink, di, dev, st, &ra, true);
}

int gptoss_moe_workspace_layout(int64_t num_tokens, int top_k, int num_experts, int64_t hidden_size,
                                int64_t intermediate_size, int64_t* offsets_out) {
  GPTOSS_TRY(check_dims(num_tokens, top_k, num_experts, hidden_size, intermediate_size));
  GPTOSS_CHECK(offsets_out != nullptr, "offsets_out is null");
  const Workspace L = plan_workspace(num_tokens, top_k, num_experts, hidden_size, intermediate_size);
  const size_t v[GPTOSS_WS_NUM_REGIONS] = {L.sorted_token, L.sorted_expert, L.sorted_weight, L.counts, L.offsets,
                                           L.sfoff_a, L.sfoff_b, L.act_codes, L.act_sf, L.inter_codes, L.inter_sf,
                                           L.router_idx, L.router_w, L.total};
  for (int i = 0; i < GPTOSS_WS_NUM_REGIONS; ++i) offsets_out[i] = static_cast<int64_t>(v[i]);
  return GPTOSS_OK;
}

int gptoss_moe_route_quant(const void* hidden, const int64_t* router_indices, const float* routing_weights,
                           int64_t num_tokens, int top_k, int num_experts, int64_t hidden_size,
                           int64_t intermediate_size, void* workspace, size_t workspace_bytes, int gemm_mode,
                           int32_t* status_dev, void* stream) {
  NvtxRange nvtx_range("gptoss_moe_route_quant");
  GPTOSS_TRY(check_dims(num_tokens, top_k, num_experts, hidden_size, intermediate_size));
  DeviceInfo di;
  GPTOSS_TRY(bind_device(workspace, "workspace", &di));
  if (num_tokens == 0) return GPTOSS_OK;
  GPTOSS_CHECK(hidden && router_indices && routing_weights && aligned(hidden, 16) && aligned(workspace, 256),
               "route_quant: null or misaligned pointer");
  const Workspace L = plan_workspace(num_tokens, top_k, num_experts, hidden_size, intermediate_size);
  if (workspace_bytes < L.total) return fail(GPTOSS_ERR_WORKSPACE, "workspace has %zu bytes, need %zu", workspace_bytes, L.total);
  return stage_route_quant(hidden, router_indices, routing_weights, num_tokens, top_k, num_experts, hidden_size,
                           intermediate_size, ws_ptrs(static_cast<uint8_t*>(workspace), L),
                           pick_layout(gemm_mode, num_tokens * top_k, num_experts).spread,
                           status_dev ? status_dev : di.status_sink, static_cast<cudaStream_t>(stream));
}

int gptoss_moe_gemm1(int64_t num_tokens, int top_k, int num_experts, int64_t hidden_size, int64_t intermediate_size,
                     const uint8_t* gate_up_data, const uint8_t* gate_up_scales, int64_t ldb_gate_up,
                     const float* gate_up_bias, float swiglu_alpha, float swiglu_limit, void* workspace,
                     size_t workspace_bytes, int gemm_mode, int32_t* status_dev, void* stream) {
  NvtxRange nvtx_range("gptoss_moe_gemm1");
  GPTOSS_TRY(check_dims(num_tokens, top_k, num_experts, hidden_size, intermediate_size));
  GPTOSS_CHECK(gemm_mode >= 0 && gemm_mode <= 3, "bad gemm_mode");
  DeviceInfo di;
  GPTOSS_TRY(bind_device(gate_up_data, "gate_up_proj_data", &di));
  GPTOSS_CHECK(gate_up_scales && gate_up_bias && aligned(gate_up_data, 32) && aligned(gate_up_scales, 16) &&
                   ldb_gate_up % 16 == 0 &&
                   ldb_gate_up >= blocked_sf_cosize(2 * intermediate_size, static_cast<int>(pad128(hidden_size) / 32)),
               "gemm1: bad gate_up weights");
  if (num_tokens == 0) return GPTOSS_OK;
  GPTOSS_CHECK(workspace && aligned(workspace, 256), "gemm1: null or misaligned workspace");
  const Workspace L = plan_workspace(num_tokens, top_k, num_experts, hidden_size, intermediate_size);
  if (workspace_bytes < L.total) return fail(GPTOSS_ERR_WORKSPACE, "workspace has %zu bytes, need %zu", workspace_bytes, L.total);
  int dev = 0;
  GPTOSS_CUDA(cudaGetDevice(&dev));
  ExpertWeights w{gate_up_data, gate_up_scales, ldb_gate_up, gate_up_bias, nullptr, nullptr, 0, nullptr};
  return stage_gemm1(num_tokens * top_k, num_experts, hidden_size, intermediate_size, w, swiglu_alpha, swiglu_limit,
                     ws_ptrs(static_cast<uint8_t*>(workspace), L),
                     pick_layout(gemm_mode, num_tokens * top_k, num_experts),
                     status_dev ? status_dev : di.status_sink, di, dev, static_cast<cudaStream_t>(stream));
}

int gptoss_moe_gemm2(int64_t num_tokens, int top_k, int num_experts, int64_t hidden_size, int64_t intermediate_size,
                     const uint8_t* down_data, const uint8_t* down_scales, int64_t ldb_down, const float* down_bias,
                     void* out, void* workspace, size_t workspace_bytes, int gemm_mode, int32_t* status_dev,
                     void* stream) {
  NvtxRange nvtx_range("gptoss_moe_gemm2");
  GPTOSS_TRY(check_dims(num_tokens, top_k, num_experts, hidden_size, intermediate_size));
  GPTOSS_CHECK(gemm_mode >= 0 && gemm_mode <= 3, "bad gemm_mode");
  DeviceInfo di;
  GPTOSS_TRY(bind_device(down_data, "down_proj_data", &di));
  GPTOSS_CHECK(down_scales && down_bias && aligned(down_data, 32) && aligned(down_scales, 16) && ldb_down % 16 == 0 &&
                   ldb_down >= blocked_sf_cosize(hidden_size, static_cast<int>(pad128(intermediate_size) / 32)),
               "gemm2: bad down weights");
  if (num_tokens == 0) return GPTOSS_OK;
  GPTOSS_CHECK(out && workspace && aligned(out, 16) && aligned(workspace, 256), "gemm2: null or misaligned pointer");
  const Workspace L = plan_workspace(num_tokens, top_k, num_experts, hidden_size, intermediate_size);
  if (workspace_bytes < L.total) return fail(GPTOSS_ERR_WORKSPACE, "workspace has %zu bytes, need %zu", workspace_bytes, L.total);
  int dev = 0;
  GPTOSS_CUDA(cudaGetDevice(&dev));
  ExpertWeights w{nullptr, nullptr, 0, nullptr, down_data, down_scales, ldb_down, down_bias};
  return stage_gemm2(num_tokens * top_k, num_experts, hidden_size, intermediate_size, w, out,
                     ws_ptrs(static_cast<uint8_t*>(workspace), L),
                     pick_layout(gemm_mode, num_tokens * top_k, num_experts),
                     status_dev ? status_dev : di.status_sink, di, dev, static_cast<cudaStream_t>(stream));
}

int gptoss_moe_experts_forward_noalloc(const void* hidden, const int64_t* router_indices,
                                       const float* routing_weights, int64_t num_tokens, int top_k, int num_experts,
                                       int64_t hidden_size, int64_t intermediate_size, const uint8_t* gate_up_data,
                                       const uint8_t* gate_up_scales, int64_t ldb_gate_up, const float* gate_up_bias,
                                       const uint8_t* down_data, const uint8_t* down_scales, int64_t ldb_down,
                                       const float* down_bias, float swiglu_alpha, float swiglu_limit, void* out,
                                       int gemm_mode, int32_t* status_dev, void* stream) {
  NvtxRange nvtx_range("gptoss_moe_experts_forward_noalloc");
  GPTOSS_TRY(check_dims(num_tokens, top_k, num_experts, hidden_size, intermediate_size));
  GPTOSS_CHECK(gemm_mode >= 0 && gemm_mode <= 3, "bad gemm_mode");
  DeviceInfo di;
  GPTOSS_TRY(bind_device(gate_up_data, "gate_up_proj_data", &di));
  ExpertWeights w{gate_up_data, gate_up_scales, ldb_gate_up, gate_up_bias,
                  down_data, down_scales, ldb_down, down_bias};
  GPTOSS_TRY(check_expert_weights(w, hidden_size, intermediate_size, num_experts));
  const Workspace L = plan_workspace(num_tokens, top_k, num_experts, hidden_size, intermediate_size);
  if (L.total > static_cast<size_t>(GPTOSS_NOALLOC_SCRATCH_BYTES))
    return fail(GPTOSS_ERR_INVALID_ARGUMENT,
                "experts_forward_noalloc: this batch needs %zu bytes of scratch but the library's static "
                "scratch holds %zu (GPTOSS_NOALLOC_SCRATCH_BYTES); use gptoss_moe_experts_forward with a "
                "caller workspace or fewer tokens",
                L.total, static_cast<size_t>(GPTOSS_NOALLOC_SCRATCH_BYTES));
  if (num_tokens == 0) return GPTOSS_OK;
  GPTOSS_CHECK(hidden && router_indices && routing_weights && out, "experts_forward_noalloc: null pointer");
  GPTOSS_CHECK(aligned(hidden, 16) && aligned(out, 16), "experts_forward_noalloc: misaligned pointer");
  int dev = 0;
  GPTOSS_CUDA(cudaGetDevice(&dev));
  uint8_t* ws = nullptr;
  GPTOSS_TRY(noalloc_scratch(dev, &ws));
  return experts_pipeline(hidden, router_indices, routing_weights, num_tokens, top_k, num_experts, hidden_size,
                          intermediate_size, w, swiglu_alpha, swiglu_limit, out, ws, L, gemm_mode,
                          status_dev ? status_dev : di.status_sink, di, dev, static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------- expert parallelism
int64_t gptoss_ep_row_bytes(int64_t hidden_size) {
  if (hidden_size <= 0 || hidden_size % 32 != 0) return 0;
  return ep_row_bytes(static_cast<int>(hidden_size));
}

size_t gptoss_ep_dispatch_workspace_bytes(int64_t num_tokens, int top_k, int world_size) {
  if (num_tokens < 0 || top_k < 1 || world_size < 1) return 0;
  const size_t A = static_cast<size_t>(num_tokens) * top_k;
  return align256(sizeof(int64_t) * A) * 2 + align256(sizeof(float) * A) + align256(sizeof(int32_t) * A) +
         align256(sizeof(int32_t) * world_size);
}

int gptoss_ep_dispatch(const void* hidden, const int64_t* router_indices, const float* routing_weights,
                       int64_t num_tokens, int top_k, int num_experts, int world_size, int64_t hidden_size,
                       int64_t capacity, uint8_t* send_rows, int32_t* send_counts, int32_t* pos_of,
                       void* workspace, size_t workspace_bytes, int32_t* status_dev, void* stream) {
  NvtxRange nvtx_range("gptoss_ep_dispatch");
  GPTOSS_CHECK(world_size >= 1 && world_size <= kMaxExperts, "ep_dispatch: world_size must be in [1, %d]", kMaxExperts);
  GPTOSS_CHECK(num_experts >= world_size && num_experts % world_size == 0,
               "ep_dispatch: num_experts (%d) must be a multiple of world_size (%d)", num_experts, world_size);
  GPTOSS_CHECK(num_tokens >= 0 && top_k >= 1 && top_k <= kMaxTopK && top_k <= num_experts,
               "ep_dispatch: bad sizes (T=%lld k=%d)", (long long)num_tokens, top_k);
  GPTOSS_CHECK(hidden_size > 0 && hidden_size % 32 == 0, "ep_dispatch: hidden size must be a multiple of 32");
  GPTOSS_CHECK(num_tokens * top_k < (1LL << 31), "ep_dispatch: too many assignments");
  GPTOSS_CHECK(capacity == 0 || capacity >= num_tokens * top_k,
               "ep_dispatch: capacity %lld must be 0 (compact rows) or >= num_tokens * top_k (%lld)",
               (long long)capacity, (long long)(num_tokens * top_k));
  GPTOSS_CHECK(capacity * world_size < (1LL << 31), "ep_dispatch: capacity * world_size too large");
  DeviceInfo di;
  GPTOSS_TRY(bind_device(send_counts, "send_counts", &di));
  const size_t need = gptoss_ep_dispatch_workspace_bytes(num_tokens, top_k, world_size);
  if (workspace_bytes < need) return fail(GPTOSS_ERR_WORKSPACE, "workspace has %zu bytes, need %zu", workspace_bytes, need);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t A = num_tokens * top_k;
  if (A == 0 && capacity == 0) {
    GPTOSS_CUDA(cudaMemsetAsync(send_counts, 0, sizeof(int32_t) * world_size, st));
    return GPTOSS_OK;
  }
  GPTOSS_CHECK(send_rows && workspace && (A == 0 || (hidden && router_indices && routing_weights && pos_of)),
               "ep_dispatch: null pointer");
  GPTOSS_CHECK(aligned(hidden, 16) && aligned(send_rows, 16) && aligned(workspace, 256),
               "ep_dispatch: misaligned pointer");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  size_t o = 0;
  auto take = [&](size_t bytes) { uint8_t* r = ws + o; o += align256(bytes); return r; };
  RouteSortParams rp{};
  rp.router_indices = router_indices; rp.routing_weights = routing_weights;
  rp.A = static_cast<int>(A); rp.K = top_k; rp.E = world_size;
  rp.sorted_token = reinterpret_cast<int64_t*>(take(sizeof(int64_t) * A));
  rp.sorted_expert = reinterpret_cast<int64_t*>(take(sizeof(int64_t) * A));
  rp.sorted_weight = reinterpret_cast<float*>(take(sizeof(float) * A));
  rp.sorted_src = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * A));
  rp.offsets = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * world_size));
  rp.counts = send_counts;
  rp.divisor = num_experts / world_size;
  rp.err = status_dev ? status_dev : di.status_sink;
  GPTOSS_TRY(launch_pdl(route_sort_kernel, dim3(world_size), dim3(1024), 0, st, rp));
  const int tpr = quant_threads_per_row(static_cast<int>(hidden_size));
  const int rpb = 256 / tpr;
  const int64_t rows = capacity > 0 ? capacity * world_size : A;
  return launch_pdl(ep_pack_kernel, dim3(static_cast<unsigned>((rows + rpb - 1) / rpb)), dim3(tpr * rpb), 0, st,
                    static_cast<const __nv_bfloat16*>(hidden), static_cast<int>(hidden_size), top_k,
                    num_experts / world_size, A, router_indices, routing_weights,
                    static_cast<const int32_t*>(rp.sorted_src), capacity, world_size,
                    static_cast<const int32_t*>(send_counts), static_cast<const int32_t*>(rp.offsets), tpr,
                    send_rows, pos_of);
}

int gptoss_ep_expert_forward(const uint8_t* recv_rows, int64_t num_rows, int num_local_experts, int64_t hidden_size,
                             int64_t intermediate_size, const uint8_t* gate_up_data, const uint8_t* gate_up_scales,
                             int64_t ldb_gate_up, const float* gate_up_bias, const uint8_t* down_data,
                             const uint8_t* down_scales, int64_t ldb_down, const float* down_bias,
                             float swiglu_alpha, float swiglu_limit, void* back_rows, void* workspace,
                             size_t workspace_bytes, int gemm_mode, int32_t* status_dev, void* stream) {
  NvtxRange nvtx_range("gptoss_ep_expert_forward");
  GPTOSS_TRY(check_dims(num_rows, 1, num_local_experts, hidden_size, intermediate_size));
  GPTOSS_CHECK(gemm_mode >= 0 && gemm_mode <= 3, "bad gemm_mode");
  DeviceInfo di;
  GPTOSS_TRY(bind_device(gate_up_data, "gate_up_proj_data", &di));
  ExpertWeights w{gate_up_data, gate_up_scales, ldb_gate_up, gate_up_bias,
                  down_data, down_scales, ldb_down, down_bias};
  GPTOSS_TRY(check_expert_weights(w, hidden_size, intermediate_size, num_local_experts));
  if (num_rows == 0) return GPTOSS_OK;
  GPTOSS_CHECK(recv_rows && back_rows && workspace, "ep_expert_forward: null pointer");
  GPTOSS_CHECK(aligned(recv_rows, 16) && aligned(back_rows, 16) && aligned(workspace, 256),
               "ep_expert_forward: misaligned pointer");
  const Workspace L = plan_workspace(num_rows, 1, num_local_experts, hidden_size, intermediate_size);
  if (workspace_bytes < L.total) return fail(GPTOSS_ERR_WORKSPACE, "workspace has %zu bytes, need %zu", workspace_bytes, L.total);
  int dev = 0;
  GPTOSS_CUDA(cudaGetDevice(&dev));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const WsPtrs p = ws_ptrs(ws, L);
  int* status = status_dev ? status_dev : di.status_sink;
  int64_t* lexp = reinterpret_cast<int64_t*>(ws + L.router_idx);
  float* lw = reinterpret_cast<float*>(ws + L.router_w);
  const GemmLayout lay = pick_layout(gemm_mode, num_rows, num_local_experts);
  const int H = static_cast<int>(hidden_size);
  const int64_t Kh = pad128(hidden_size), Ki = pad128(intermediate_size);
  const int ublocks = static_cast<int>(std::min<int64_t>((num_rows + 255) / 256, 4 * di.sms));
  GPTOSS_TRY(launch_pdl(ep_unpack_meta_kernel, dim3(ublocks), dim3(256), 0, st, recv_rows, num_rows, H, lexp, lw));
  RouteSortParams rp{};
  rp.router_indices = lexp; rp.routing_weights = lw;
  rp.A = static_cast<int>(num_rows); rp.K = 1; rp.E = num_local_experts;
  rp.sorted_token = p.sorted_token; rp.sorted_expert = p.sorted_expert; rp.sorted_weight = p.sorted_weight;
  rp.counts = p.counts; rp.offsets = p.offsets;
  rp.sf_offsets_a = p.sfoff_a; rp.g4_a = static_cast<int>(Kh / 128); rp.groups_a = H / 32; rp.sf_a = p.act_sf;
  rp.sf_offsets_b = p.sfoff_b; rp.g4_b = static_cast<int>(Ki / 128);
  rp.groups_b = static_cast<int>(intermediate_size / 32); rp.sf_b = p.inter_sf;
  rp.spread = lay.spread ? 1 : 0;
  rp.allow_empty = 1;
  rp.err = status;
  GPTOSS_TRY(launch_pdl(route_sort_kernel, dim3(num_local_experts), dim3(1024), 0, st, rp));
  GPTOSS_TRY(launch_pdl(ep_gather_kernel, dim3(static_cast<unsigned>(num_rows)), dim3(256), 0, st, recv_rows,
                        num_rows, H, static_cast<const int64_t*>(p.sorted_token),
                        static_cast<const int64_t*>(p.sorted_expert), static_cast<const int32_t*>(p.offsets),
                        static_cast<const int32_t*>(p.sfoff_a), static_cast<int>(Kh / 128), lay.spread ? 1 : 0,
                        p.act_codes, p.act_sf));
  GPTOSS_CUDA(cudaMemsetAsync(back_rows, 0, static_cast<size_t>(num_rows * hidden_size) * sizeof(__nv_bfloat16), st));
  GPTOSS_TRY(stage_gemm1(num_rows, num_local_experts, hidden_size, intermediate_size, w, swiglu_alpha, swiglu_limit, p,
                         lay, status, di, dev, st));
  return stage_gemm2(num_rows, num_local_experts, hidden_size, intermediate_size, w, back_rows, p, lay, status, di,
                     dev, st);
}

int gptoss_ep_combine(const void* back_rows, int64_t num_back_rows, const int32_t* pos_of,
                      const int64_t* router_indices, int64_t num_tokens, int top_k, int64_t hidden_size, void* out,
                      void* stream) {
  NvtxRange nvtx_range("gptoss_ep_combine");
  GPTOSS_CHECK(num_tokens >= 0 && top_k >= 1 && top_k <= kMaxTopK, "ep_combine: bad sizes");
  GPTOSS_CHECK(hidden_size > 0 && hidden_size % 2 == 0, "ep_combine: hidden size must be even");
  DeviceInfo di;
  GPTOSS_TRY(bind_device(out, "out", &di));
  if (num_tokens == 0) return GPTOSS_OK;
  GPTOSS_CHECK(back_rows && pos_of && router_indices, "ep_combine: null pointer");
  GPTOSS_CHECK(aligned(back_rows, 4) && aligned(out, 4), "ep_combine: misaligned pointer");
  return launch_pdl(ep_combine_kernel, dim3(static_cast<unsigned>(num_tokens)), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(back_rows), pos_of,
                    router_indices, num_tokens, top_k, static_cast<int>(hidden_size), num_back_rows,
                    static_cast<__nv_bfloat16*>(out));
}

// ---------------------------------------------------------------- peer memory (one node)
int gptoss_ipc_handle_bytes(void) { return static_cast<int>(sizeof(cudaIpcMemHandle_t)); }

int gptoss_ipc_alloc(size_t bytes, void** ptr, void* handle_out) {
  GPTOSS_CHECK(ptr != nullptr && handle_out != nullptr && bytes > 0, "ipc_alloc: bad arguments");
  void* p = nullptr;
  GPTOSS_CUDA(cudaMalloc(&p, bytes));
  cudaError_t e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) {
    cudaIpcMemHandle_t h;
    e = cudaIpcGetMemHandle(&h, p);
    if (e == cudaSuccess) {
      std::memcpy(handle_out, &h, sizeof(h));
      *ptr = p;
      return GPTOSS_OK;
    }
  }
  cudaFree(p);
  return fail(GPTOSS_ERR_CUDA, "ipc_alloc: %s", cudaGetErrorString(e));
}

int gptoss_ipc_open(const void* handle, void** ptr) {
  GPTOSS_CHECK(handle != nullptr && ptr != nullptr, "ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  GPTOSS_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return GPTOSS_OK;
}

int gptoss_ipc_close(void* ptr) {
  GPTOSS_CHECK(ptr != nullptr, "ipc_close: null pointer");
  GPTOSS_CUDA(cudaIpcCloseMemHandle(ptr));
  return GPTOSS_OK;
}

int gptoss_ipc_free(void* ptr) {
  GPTOSS_CHECK(ptr != nullptr, "ipc_free: null pointer");
  GPTOSS_CUDA(cudaFree(ptr));
  return GPTOSS_OK;
}

size_t gptoss_ep_p2p_buffer_bytes(int world_size, int64_t capacity, int64_t hidden_size) {
  if (world_size < 1 || world_size > kP2pMaxWorld || capacity < 1 || hidden_size <= 0 || hidden_size % 32) return 0;
  return static_cast<size_t>(p2p_buffer_bytes(world_size, capacity, static_cast<int>(hidden_size)));
}

}  // extern "C"

// Peer-memory dispatch (routing given, or computed first when `ra` is set). Decode-sized
// batches run as one cluster launch (decode_prologue_kernel in dispatch mode); larger ones
// as route_sort_kernel (by owning rank) + ep_pack_p2p_kernel, after router_launch if `ra`.
int ep_p2p_dispatch_impl(const void* hidden, const RouterArgs* ra, const int64_t* router_indices,
                         const float* routing_weights, int64_t num_tokens, int top_k, int num_experts,
                         int world_size, int rank, int64_t hidden_size, int64_t capacity, void* local_base,
                         const uint64_t* peer_bases, int32_t epoch, int32_t* send_counts, int32_t* pos_of,
                         void* workspace, size_t workspace_bytes, int32_t* status_dev, void* stream) {
  GPTOSS_CHECK(world_size >= 1 && world_size <= kP2pMaxWorld && rank >= 0 && rank < world_size,
               "ep_p2p_dispatch: bad world_size / rank");
  GPTOSS_CHECK(num_experts % world_size == 0, "ep_p2p_dispatch: num_experts must be a multiple of world_size");
  GPTOSS_CHECK(num_tokens >= 0 && top_k >= 1 && top_k <= kMaxTopK && top_k <= num_experts,
               "ep_p2p_dispatch: bad sizes");
  GPTOSS_CHECK(hidden_size > 0 && hidden_size % 32 == 0, "ep_p2p_dispatch: hidden size must be a multiple of 32");
  GPTOSS_CHECK(capacity >= num_tokens * top_k && capacity > 0, "ep_p2p_dispatch: capacity below num_tokens * top_k");
  DeviceInfo di;
  GPTOSS_TRY(bind_device(send_counts, "send_counts", &di));
  GPTOSS_CHECK(local_base && peer_bases && workspace &&
                   (num_tokens == 0 || (hidden && (ra != nullptr || (router_indices && routing_weights)) && pos_of)),
               "ep_p2p_dispatch: null pointer");
  const size_t need = gptoss_ep_dispatch_workspace_bytes(num_tokens, top_k, world_size);
  if (workspace_bytes < need) return fail(GPTOSS_ERR_WORKSPACE, "workspace has %zu bytes, need %zu", workspace_bytes, need);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int* status = status_dev ? status_dev : di.status_sink;
  int dev = 0;
  GPTOSS_CUDA(cudaGetDevice(&dev));
  size_t smem = 0;
  int slice = 0;
  if (num_tokens > 0 && decode_prologue_fits(num_tokens, top_k, num_experts, hidden_size, ra != nullptr, &smem, &slice)) {
    static uint64_t attr_done = 0;   // one bit per device
    static std::mutex mu;
    {
      std::lock_guard<std::mutex> lk(mu);
      if (!(attr_done & (1ull << dev))) {
        GPTOSS_CUDA(cudaFuncSetAttribute(decode_prologue_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kDpMaxSmem)));
        attr_done |= (1ull << dev);
      }
    }
    DecodePrologueParams p{};
    p.x = static_cast<const __nv_bfloat16*>(hidden);
    if (ra != nullptr) {
      p.w = static_cast<const __nv_bfloat16*>(ra->weight);
      p.bias = static_cast<const __nv_bfloat16*>(ra->bias);
      p.ridx_out = ra->ridx_out;
      p.scores_out = static_cast<__nv_bfloat16*>(ra->scores_out);
      p.rw_out = ra->rw_out;
    } else {
      p.ridx_in = router_indices;
      p.rw_in = routing_weights;
    }
    p.T = static_cast<int>(num_tokens); p.H = static_cast<int>(hidden_size); p.E = num_experts; p.K = top_k;
    p.slice_chunks = slice;
    p.err = status;
    p.ep_world = world_size; p.ep_rank = rank; p.ep_epr = num_experts / world_size;
    p.ep_rb = static_cast<int>(ep_row_bytes(static_cast<int>(hidden_size)));
    p.ep_cap = capacity;
    p.peer_bases = peer_bases;
    p.send_counts = send_counts;
    p.pos_of = pos_of;
    p.epoch = epoch;
    return launch_pdl_cluster(decode_prologue_kernel, dim3(kDpCluster), dim3(kDpThreads), smem, st,
                              dim3(kDpCluster, 1, 1), p);
  }
  if (ra != nullptr && num_tokens > 0) {
    GPTOSS_TRY(router_launch(hidden, ra->weight, ra->bias, num_tokens, hidden_size, num_experts, top_k, ra->ridx_out,
                             ra->scores_out, ra->rw_out, nullptr, nullptr, 0, di.sms, dev, st));
    router_indices = ra->ridx_out;
    routing_weights = ra->rw_out;
  }
  const int64_t A = num_tokens * top_k;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  size_t o = 0;
  auto take = [&](size_t bytes) { uint8_t* r = ws + o; o += align256(bytes); return r; };
  RouteSortParams rp{};
  rp.router_indices = router_indices; rp.routing_weights = routing_weights;
  rp.A = static_cast<int>(A); rp.K = top_k; rp.E = world_size;
  rp.sorted_token = reinterpret_cast<int64_t*>(take(sizeof(int64_t) * A));
  rp.sorted_expert = reinterpret_cast<int64_t*>(take(sizeof(int64_t) * A));
  rp.sorted_weight = reinterpret_cast<float*>(take(sizeof(float) * A));
  rp.sorted_src = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * A));
  rp.offsets = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * world_size));
  rp.counts = send_counts;
  rp.divisor = num_experts / world_size;
  rp.err = status;
  GPTOSS_TRY(launch_pdl(route_sort_kernel, dim3(world_size), dim3(1024), 0, st, rp));
  const int tpr = quant_threads_per_row(static_cast<int>(hidden_size));
  const int rpb = 256 / tpr;
  const int64_t rows = capacity * world_size;
  GPTOSS_TRY(launch_pdl(ep_pack_p2p_kernel, dim3(static_cast<unsigned>((rows + rpb - 1) / rpb)), dim3(tpr * rpb), 0,
                        st, static_cast<const __nv_bfloat16*>(hidden), static_cast<int>(hidden_size), top_k,
                        num_experts / world_size, A, router_indices, routing_weights,
                        static_cast<const int32_t*>(rp.sorted_src), capacity, world_size, rank,
                        static_cast<const int32_t*>(send_counts), static_cast<const int32_t*>(rp.offsets), tpr,
                        peer_bases, pos_of, static_cast<int32_t*>(local_base) + kP2pCounterDispatch, epoch));
  return GPTOSS_OK;
}

extern "C" {

int gptoss_ep_p2p_dispatch(const void* hidden, const int64_t* router_indices, const float* routing_weights,
                           int64_t num_tokens, int top_k, int num_experts, int world_size, int rank,
                           int64_t hidden_size, int64_t capacity, void* local_base, const uint64_t* peer_bases,
                           int32_t epoch, int32_t* send_counts, int32_t* pos_of, void* workspace,
                           size_t workspace_bytes, int32_t* status_dev, void* stream) {
  NvtxRange nvtx_range("gptoss_ep_p2p_dispatch");
  return ep_p2p_dispatch_impl(hidden, nullptr, router_indices, routing_weights, num_tokens, top_k, num_experts,
                              world_size, rank, hidden_size, capacity, local_base, peer_bases, epoch, send_counts,
                              pos_of, workspace, workspace_bytes, status_dev, stream);
}

int gptoss_ep_p2p_route_dispatch(const void* hidden, const void* router_weight, const void* router_bias,
                                 int64_t num_tokens, int top_k, int num_experts, int world_size, int rank,
                                 int64_t hidden_size, int64_t capacity, void* local_base, const uint64_t* peer_bases,
                                 int32_t epoch, int64_t* router_indices_out, void* router_scores_out,
                                 float* routing_weights_out, int32_t* send_counts, int32_t* pos_of, void* workspace,
                                 size_t workspace_bytes, int32_t* status_dev, void* stream) {
  NvtxRange nvtx_range("gptoss_ep_p2p_route_dispatch");
  GPTOSS_CHECK(num_tokens == 0 || (router_weight && router_bias && router_indices_out && routing_weights_out),
               "ep_p2p_route_dispatch: null pointer");
  GPTOSS_CHECK(hidden_size % 8 == 0, "ep_p2p_route_dispatch: hidden size must be a multiple of 8");
  const RouterArgs ra{router_weight, router_bias, router_indices_out, router_scores_out, routing_weights_out};
  return ep_p2p_dispatch_impl(hidden, &ra, nullptr, nullptr, num_tokens, top_k, num_experts, world_size, rank,
                              hidden_size, capacity, local_base, peer_bases, epoch, send_counts, pos_of, workspace,
                              workspace_bytes, status_dev, stream);
}

int gptoss_ep_p2p_expert_forward(void* local_base, int world_size, int rank, int64_t capacity, int32_t epoch,
                                 int num_local_experts, int64_t hidden_size, int64_t intermediate_size,
                                 const uint8_t* gate_up_data, const uint8_t* gate_up_scales, int64_t ldb_gate_up,
                                 const float* gate_up_bias, const uint8_t* down_data, const uint8_t* down_scales,
                                 int64_t ldb_down, const float* down_bias, float swiglu_alpha, float swiglu_limit,
                                 void* back_rows, const uint64_t* peer_bases, void* workspace, size_t workspace_bytes,
                                 int gemm_mode, int32_t* status_dev, void* stream) {
  NvtxRange nvtx_range("gptoss_ep_p2p_expert_forward");
  GPTOSS_CHECK(world_size >= 1 && world_size <= kP2pMaxWorld && rank >= 0 && rank < world_size,
               "ep_p2p_expert_forward: bad world_size / rank");
  const int64_t R = capacity * world_size;
  GPTOSS_TRY(check_dims(R, 1, num_local_experts, hidden_size, intermediate_size));
  GPTOSS_CHECK(gemm_mode >= 0 && gemm_mode <= 3, "bad gemm_mode");
  DeviceInfo di;
  GPTOSS_TRY(bind_device(gate_up_data, "gate_up_proj_data", &di));
  ExpertWeights w{gate_up_data, gate_up_scales, ldb_gate_up, gate_up_bias,
                  down_data, down_scales, ldb_down, down_bias};
  GPTOSS_TRY(check_expert_weights(w, hidden_size, intermediate_size, num_local_experts));
  GPTOSS_CHECK(local_base && back_rows && peer_bases && workspace, "ep_p2p_expert_forward: null pointer");
  GPTOSS_CHECK(aligned(local_base, 256) && aligned(back_rows, 16) && aligned(workspace, 256),
               "ep_p2p_expert_forward: misaligned pointer");
  const Workspace L = plan_workspace(R, 1, num_local_experts, hidden_size, intermediate_size);
  if (workspace_bytes < L.total) return fail(GPTOSS_ERR_WORKSPACE, "workspace has %zu bytes, need %zu", workspace_bytes, L.total);
  int dev = 0;
  GPTOSS_CUDA(cudaGetDevice(&dev));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const WsPtrs p = ws_ptrs(ws, L);
  int* status = status_dev ? status_dev : di.status_sink;
  int64_t* lexp = reinterpret_cast<int64_t*>(ws + L.router_idx);
  float* lw = reinterpret_cast<float*>(ws + L.router_w);
  // rows expected here under balanced routing: W sources x capacity / W
  const GemmLayout lay = pick_layout(gemm_mode, capacity, num_local_experts);
  const int H = static_cast<int>(hidden_size);
  const int64_t rb = ep_row_bytes(H);
  const int64_t Kh = pad128(hidden_size), Ki = pad128(intermediate_size);
  const uint8_t* recv = static_cast<const uint8_t*>(local_base) + p2p_recv_offset(0, capacity, rb);
  const int32_t* flags = static_cast<const int32_t*>(local_base);
  int32_t* ret_counter = static_cast<int32_t*>(local_base) + kP2pCounterReturn;
  const size_t rp_smem = recv_prologue_smem(R, num_local_experts);
  int prefetch = 0;
  bool fused_return = false;
  if (R <= kRpMaxRows && rp_smem <= 200 * 1024) {
    // one launch: flag wait, sort by local expert, gather into the blocked layout, zero back_rows
    static uint64_t attr_done = 0;   // one bit per device
    static std::mutex mu;
    {
      std::lock_guard<std::mutex> lk(mu);
      if (!(attr_done & (1ull << dev))) {
        GPTOSS_CUDA(cudaFuncSetAttribute(ep_recv_prologue_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         200 * 1024));
        attr_done |= (1ull << dev);
      }
    }
    RecvPrologueParams rq{};
    rq.recv = recv; rq.R = R; rq.H = H; rq.E = num_local_experts; rq.world = world_size; rq.epoch = epoch;
    rq.flags = flags; rq.err = status; rq.lexp = lexp; rq.lw = lw;
    rq.sorted_token = p.sorted_token; rq.sorted_expert = p.sorted_expert; rq.sorted_weight = p.sorted_weight;
    rq.counts = p.counts; rq.offsets = p.offsets; rq.sf_offsets_a = p.sfoff_a; rq.sf_offsets_b = p.sfoff_b;
    rq.g4_a = static_cast<int>(Kh / 128); rq.g4_b = static_cast<int>(Ki / 128); rq.spread = lay.spread ? 1 : 0;
    // weights-on-M GEMM2 stores the rows straight into the sources' return rows
    rq.act_codes = p.act_codes; rq.act_sf = p.act_sf;
    rq.back_rows = lay.swap ? nullptr : static_cast<__nv_bfloat16*>(back_rows);
    const int grid = static_cast<int>(std::min<int64_t>(di.sms, std::max<int64_t>(R, 1)));
    GPTOSS_TRY(launch_pdl(ep_recv_prologue_kernel, dim3(grid), dim3(256), rp_smem, st, rq));
    prefetch = kPrefetchTilesAfterPrologue;
    fused_return = lay.swap;
  } else {
    const int ublocks = static_cast<int>(std::min<int64_t>((R + 255) / 256, 4 * di.sms));
    GPTOSS_TRY(launch_pdl(ep_unpack_meta_p2p_kernel, dim3(ublocks), dim3(256), 0, st, recv, R, H, flags, world_size,
                          epoch, status, lexp, lw));
    RouteSortParams rp{};
    rp.router_indices = lexp; rp.routing_weights = lw;
    rp.A = static_cast<int>(R); rp.K = 1; rp.E = num_local_experts;
    rp.sorted_token = p.sorted_token; rp.sorted_expert = p.sorted_expert; rp.sorted_weight = p.sorted_weight;
    rp.counts = p.counts; rp.offsets = p.offsets;
    rp.sf_offsets_a = p.sfoff_a; rp.g4_a = static_cast<int>(Kh / 128); rp.groups_a = H / 32; rp.sf_a = p.act_sf;
    rp.sf_offsets_b = p.sfoff_b; rp.g4_b = static_cast<int>(Ki / 128);
    rp.groups_b = static_cast<int>(intermediate_size / 32); rp.sf_b = p.inter_sf;
    rp.spread = lay.spread ? 1 : 0;
    rp.allow_empty = 1;
    rp.err = status;
    GPTOSS_TRY(launch_pdl(route_sort_kernel, dim3(num_local_experts), dim3(1024), 0, st, rp));
    GPTOSS_TRY(launch_pdl(ep_gather_kernel, dim3(static_cast<unsigned>(R)), dim3(256), 0, st, recv, R, H,
                          static_cast<const int64_t*>(p.sorted_token), static_cast<const int64_t*>(p.sorted_expert),
                          static_cast<const int32_t*>(p.offsets), static_cast<const int32_t*>(p.sfoff_a),
                          static_cast<int>(Kh / 128), lay.spread ? 1 : 0, p.act_codes, p.act_sf));
    GPTOSS_CUDA(cudaMemsetAsync(back_rows, 0, static_cast<size_t>(R * hidden_size) * sizeof(__nv_bfloat16), st));
  }
  GPTOSS_TRY(stage_gemm1(R, num_local_experts, hidden_size, intermediate_size, w, swiglu_alpha, swiglu_limit, p, lay,
                         status, di, dev, st, prefetch));
  if (fused_return) {
    const EpReturn er{peer_bases, p2p_ret_offset(world_size, rank, capacity, rb, H), capacity, ret_counter,
                      world_size, rank, epoch};
    return stage_gemm2(R, num_local_experts, hidden_size, intermediate_size, w, back_rows, p, lay, status, di, dev,
                       st, &er);
  }
  GPTOSS_TRY(stage_gemm2(R, num_local_experts, hidden_size, intermediate_size, w, back_rows, p, lay, status, di,
                         dev, st));
  return launch_pdl(ep_return_p2p_kernel, dim3(static_cast<unsigned>(R)), dim3(256), 0, st,
                    static_cast<const __nv_bfloat16*>(back_rows), static_cast<const int64_t*>(lexp), capacity,
                    world_size, rank, H, peer_bases, ret_counter, epoch);
}

int gptoss_ep_p2p_combine(const void* local_base, int world_size, int64_t capacity, int32_t epoch,
                          const int32_t* pos_of, const int64_t* router_indices, int64_t num_tokens, int top_k,
                          int64_t hidden_size, void* out, int32_t* status_dev, void* stream) {
  NvtxRange nvtx_range("gptoss_ep_p2p_combine");
  GPTOSS_CHECK(world_size >= 1 && world_size <= kP2pMaxWorld, "ep_p2p_combine: bad world_size");
  GPTOSS_CHECK(num_tokens >= 0 && top_k >= 1 && top_k <= kMaxTopK, "ep_p2p_combine: bad sizes");
  GPTOSS_CHECK(hidden_size > 0 && hidden_size % 32 == 0, "ep_p2p_combine: hidden size must be a multiple of 32");
  DeviceInfo di;
  GPTOSS_TRY(bind_device(local_base, "local_base", &di));
  GPTOSS_CHECK(out != nullptr || num_tokens == 0, "ep_p2p_combine: null output");
  const int64_t rb = ep_row_bytes(static_cast<int>(hidden_size));
  const uint8_t* base = static_cast<const uint8_t*>(local_base);
  const int32_t* flags = reinterpret_cast<const int32_t*>(base);
  // With no tokens the kernel still runs one CTA: it consumes this call's return flags.
  return launch_pdl(ep_combine_p2p_kernel, dim3(static_cast<unsigned>(std::max<int64_t>(num_tokens, 1))), dim3(256),
                    0, static_cast<cudaStream_t>(stream),
                    reinterpret_cast<const __nv_bfloat16*>(base + p2p_ret_offset(world_size, 0, capacity, rb,
                                                                                  static_cast<int>(hidden_size))),
                    flags, world_size, epoch, status_dev ? status_dev : di.status_sink, pos_of, router_indices,
                    num_tokens, top_k, static_cast<int>(hidden_size), capacity * world_size,
                    static_cast<__nv_bfloat16*>(out));
}

}  // extern "C"

// ---------------------------------------------------------------- one-launch expert-parallel layer
// decode_layer_kernel<true>: router (or given routing) on this rank's tokens, dispatch into
// the owners' receive rows, the local experts' GEMMs on the received rows with GEMM2 storing
// into the sources' return rows, and the combine, in one persistent launch behind a one-CTA
// reset of its synchronisation words. Serves decode-sized steps: the received rows (W x cap)
// fit the kernel's shared-memory routing state and the local experts hold few rows each
// (16-row chunks); gptoss_set_ep_layer_kernel(0) turns it off.
// The kernel's tiles multiply 16-row activation chunks, so an expert of m rows streams its
// weight tiles ceil(m / 16) times -- concurrently, from neighbouring CTAs (chunks are the
// innermost tile index), so mostly out of L2. Up to kEpLayerMaxRowsPerExpert rows per local
// expert under balanced routing (capacity / local experts: 32 at 8 ranks x 32 tokens x top-4
// on 32 experts) the one launch wins; above it the five-launch path picks its own layout.
constexpr int64_t kEpLayerMaxRowsPerExpert = 64;
// Expert weights the one-launch kernel pulls into L2 under its routing and exchange phases
// (about half of the 126 MB L2: all of a rank's experts at 8 ranks of GPT-OSS-20B, 53 MB).
constexpr int64_t kEpLayerL2PrefetchBytes = 64ll << 20;
std::atomic<int> g_ep_layer_enabled{1};

bool ep_layer_fits(int64_t T, int k, int E, int world, int64_t H, int64_t I, int64_t cap) {
  if (g_ep_layer_enabled.load(std::memory_order_relaxed) == 0) return false;
  if (world < 1 || world > kP2pMaxWorld || E % world != 0) return false;
  const int epr = E / world;
  return cap <= kEpLayerMaxRowsPerExpert * epr && T >= 0 && T <= kDlMaxTokens && T * k <= kDlMaxAssign &&
         epr <= kDlMaxExperts &&
         H % 32 == 0 && I % 32 == 0 && cap >= T * k && world * cap <= kEpMaxRecv &&
         static_cast<size_t>(T) * (2 * E + k) * sizeof(float) <= (DlCfg::kStages - kDlPreStages) * DlCfg::kStageBytes;
}

extern "C" {

int gptoss_set_ep_layer_kernel(int enable) {
  return g_ep_layer_enabled.exchange(enable != 0 ? 1 : 0, std::memory_order_relaxed);
}

int gptoss_ep_p2p_layer_fits(int64_t num_tokens, int top_k, int num_experts, int world_size, int64_t hidden_size,
                             int64_t intermediate_size, int64_t capacity) {
  return ep_layer_fits(num_tokens, top_k, num_experts, world_size, hidden_size, intermediate_size, capacity) ? 1 : 0;
}

int gptoss_ep_p2p_layer_forward(const void* hidden, const void* router_weight, const void* router_bias,
                                const int64_t* router_indices, const float* routing_weights, int64_t num_tokens,
                                int top_k, int num_experts, int world_size, int rank, int64_t hidden_size,
                                int64_t intermediate_size, const uint8_t* gate_up_data, const uint8_t* gate_up_scales,
                                int64_t ldb_gate_up, const float* gate_up_bias, const uint8_t* down_data,
                                const uint8_t* down_scales, int64_t ldb_down, const float* down_bias,
                                float swiglu_alpha, float swiglu_limit, int64_t capacity, void* local_base,
                                const uint64_t* peer_bases, int32_t epoch, void* out, int64_t* router_indices_out,
                                void* router_scores_out, float* routing_weights_out, int32_t* send_counts,
                                int32_t* pos_of, void* workspace, size_t workspace_bytes, int32_t* status_dev,
                                void* stream) {
  NvtxRange nvtx_range("gptoss_ep_p2p_layer_forward");
  GPTOSS_CHECK(world_size >= 1 && world_size <= kP2pMaxWorld && rank >= 0 && rank < world_size,
               "ep_p2p_layer_forward: bad world_size / rank");
  GPTOSS_CHECK(num_experts % world_size == 0, "ep_p2p_layer_forward: num_experts must be a multiple of world_size");
  GPTOSS_TRY(check_dims(num_tokens, top_k, num_experts, hidden_size, intermediate_size));
  const int epr = num_experts / world_size;
  GPTOSS_CHECK(ep_layer_fits(num_tokens, top_k, num_experts, world_size, hidden_size, intermediate_size, capacity),
               "ep_p2p_layer_forward: T=%lld, top_k=%d, E=%d, W=%d, capacity=%lld do not fit the one-launch kernel "
               "(gptoss_ep_p2p_layer_fits) or it is turned off",
               (long long)num_tokens, top_k, num_experts, world_size, (long long)capacity);
  const bool router = router_weight != nullptr;
  // a rank without tokens still takes part in the exchange (its peers wait for its flags)
  GPTOSS_CHECK(local_base && peer_bases && send_counts && workspace &&
                   (num_tokens == 0 ||
                    (hidden && out && pos_of &&
                     (router ? (router_bias && router_indices_out && routing_weights_out)
                             : (router_indices && routing_weights)))),
               "ep_p2p_layer_forward: null pointer");
  GPTOSS_CHECK(aligned(hidden, 16) && aligned(out, 16) && aligned(local_base, 256) && aligned(workspace, 256) &&
                   (!router || aligned(router_weight, 16)),
               "ep_p2p_layer_forward: misaligned pointer");
  DeviceInfo di;
  GPTOSS_TRY(bind_device(gate_up_data, "gate_up_proj_data", &di));
  const ExpertWeights wt{gate_up_data, gate_up_scales, ldb_gate_up, gate_up_bias,
                         down_data, down_scales, ldb_down, down_bias};
  GPTOSS_TRY(check_expert_weights(wt, hidden_size, intermediate_size, epr));
  const int64_t R = capacity * world_size;
  const Workspace L = plan_workspace(R, 1, epr, hidden_size, intermediate_size);
  if (workspace_bytes < L.total) return fail(GPTOSS_ERR_WORKSPACE, "workspace has %zu bytes, need %zu", workspace_bytes, L.total);
  int dev = 0;
  GPTOSS_CUDA(cudaGetDevice(&dev));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int* status = status_dev ? status_dev : di.status_sink;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const WsPtrs w = ws_ptrs(ws, L);
  const int H = static_cast<int>(hidden_size);
  const int64_t I = intermediate_size, Kh = pad128(hidden_size), Ki = pad128(intermediate_size);
  const int rb = static_cast<int>(ep_row_bytes(H));
  CUtensorMap ta, ti, tgu, tdn;
  GPTOSS_TRY(make_act_map(&ta, w.act_codes, R, hidden_size, DlCfg::kActRows));
  GPTOSS_TRY(make_act_map(&ti, w.inter_codes, R, I, DlCfg::kActRows));
  GPTOSS_TRY(make_wgt_map(&tgu, wt.gu_data, epr, 2 * I, Kh, DlCfg::kWgtRowsCta));
  GPTOSS_TRY(make_wgt_map(&tdn, wt.dn_data, epr, hidden_size, Ki, DlCfg::kWgtRowsCta));
  static uint64_t attr_done = 0;   // one bit per device
  static std::mutex mu;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!(attr_done & (1ull << dev))) {
      GPTOSS_CUDA(cudaFuncSetAttribute(decode_layer_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(dl_smem_bytes<true>())));
      attr_done |= (1ull << dev);
    }
  }
  DecodeLayerParams p{};
  p.x = static_cast<const __nv_bfloat16*>(hidden);
  if (router) {
    p.router_w = static_cast<const __nv_bfloat16*>(router_weight);
    p.router_b = static_cast<const __nv_bfloat16*>(router_bias);
    p.ridx_out = router_indices_out;
    p.scores_out = static_cast<__nv_bfloat16*>(router_scores_out);
    p.rw_out = routing_weights_out;
  } else {
    p.ridx_in = router_indices;
    p.rw_in = routing_weights;
  }
  p.T = static_cast<int>(num_tokens); p.H = H; p.I = static_cast<int>(I); p.E = num_experts; p.K = top_k;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.logits = reinterpret_cast<float*>(ws + L.dl_logits);
  p.sorted_token = w.sorted_token; p.sorted_expert = w.sorted_expert; p.sorted_weight = w.sorted_weight;
  p.counts = w.counts; p.offsets = w.offsets; p.sf_offsets_a = w.sfoff_a; p.sf_offsets_b = w.sfoff_b;
  p.act_codes = w.act_codes; p.act_sf = w.act_sf; p.inter_codes = w.inter_codes; p.inter_sf = w.inter_sf;
  p.sync = reinterpret_cast<int32_t*>(ws + L.dl_sync);
  p.sfb_gu = wt.gu_scales; p.sfb_stride_gu = wt.ldb_gu; p.bias_gu = wt.gu_bias;
  p.sfb_dn = wt.dn_scales; p.sfb_stride_dn = wt.ldb_dn; p.bias_dn = wt.dn_bias;
  p.swiglu_alpha = swiglu_alpha; p.swiglu_limit = swiglu_limit;
  p.kb1 = static_cast<int>(Kh / 128); p.kb2 = static_cast<int>(Ki / 128);
  p.n_tiles1 = static_cast<int>((2 * I + DlCfg::kWgtRows - 1) / DlCfg::kWgtRows);
  p.n_tiles2 = static_cast<int>((hidden_size + DlCfg::kWgtRows - 1) / DlCfg::kWgtRows);
  p.err = status;
  p.ep_world = world_size; p.ep_rank = rank; p.ep_epr = epr; p.ep_rb = rb; p.ep_cap = capacity;
  p.ep_local = static_cast<uint8_t*>(local_base); p.ep_peer_bases = peer_bases; p.ep_epoch = epoch;
  p.ep_send_counts = send_counts; p.ep_pos_of = pos_of;
  p.wgu = wt.gu_data; p.wdn = wt.dn_data;
  p.wgu_bytes = static_cast<int64_t>(epr) * 2 * I * (Kh / 2);
  p.wdn_bytes = static_cast<int64_t>(epr) * hidden_size * (Ki / 2);
  // only when all of this rank's weights fit: a partial warm-up measured no gain at 2 ranks
  p.l2_prefetch_bytes = p.wgu_bytes + p.wdn_bytes <= kEpLayerL2PrefetchBytes ? kEpLayerL2PrefetchBytes : 0;
  GemmParams g1{};
  g1.num_experts = epr; g1.N = static_cast<int>(2 * I); g1.K = static_cast<int>(Kh); g1.num_kb = p.kb1;
  g1.err = status; g1.out = w.inter_codes; g1.ld_out = I; g1.bias = wt.gu_bias; g1.out_sf = w.inter_sf;
  g1.out_g4 = p.kb2; g1.out_features = static_cast<int>(I);
  g1.swiglu_alpha = swiglu_alpha; g1.swiglu_limit = swiglu_limit;
  GemmParams g2{};
  g2.num_experts = epr; g2.N = H; g2.K = static_cast<int>(Ki); g2.num_kb = p.kb2;
  g2.err = status; g2.out = out; g2.ld_out = H; g2.bias = wt.dn_bias;
  g2.swiglu_alpha = swiglu_alpha; g2.swiglu_limit = swiglu_limit;
  g2.ep_world = world_size; g2.ep_rank = rank; g2.ep_peer_bases = peer_bases; g2.ep_cap = capacity;
  g2.ep_ret_off = p2p_ret_offset(world_size, rank, capacity, rb, H); g2.ep_epoch = epoch;
  GPTOSS_TRY(launch_pdl(decode_reset_kernel, dim3(1), dim3(256), 0, st, p.sync, dl_sync_words(epr)));
  return launch_pdl(decode_layer_kernel<true>, dim3(di.sms), dim3(DlCfg::kThreads), dl_smem_bytes<true>(), st, ta, ti,
                    tgu, tdn, p, g1, g2);
}

}  // extern "C"
