// fqkv_api.cu -- the extern "C" boundary of the library (include/fused_rmsnorm_qkv.h).
//
// Validation happens before any CUDA call, so an invalid argument returns its error
// code even on a machine without a GPU.  The library allocates nothing: schedules that
// need scratch take it from the caller (fqkv_workspace_bytes).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>

#include "fqkv_kernels.cuh"

namespace fqkv {

__device__ int g_status = 0;
__device__ unsigned long long g_wait_limit_ns = kWaitLimitNs;

namespace {

thread_local std::string t_last_error;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  t_last_error = std::string(what) + ": " + cudaGetErrorString(e);
  return -static_cast<int>(e);
}

constexpr int kMaxDevices = 64;
struct DeviceInfo {
  bool init = false;
  int major = 0, minor = 0, sms = 0;
};
DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

int device_info(DeviceInfo* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(FQKV_ERR_DEVICE, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.init) {
    if ((e = cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess)
      return cuda_fail(e, "cudaDeviceGetAttribute");
    if ((e = cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess)
      return cuda_fail(e, "cudaDeviceGetAttribute");
    if ((e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
      return cuda_fail(e, "cudaDeviceGetAttribute");
    d.init = true;
  }
  *out = d;
  return 0;
}

// cuTensorMapEncodeTiled, reached through the runtime so the library does not link libcuda.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
std::once_flag g_encode_once;

int get_encode(EncodeTiledFn* fn) {
  std::call_once(g_encode_once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (!g_encode) return fail(FQKV_ERR_DEVICE, "cuTensorMapEncodeTiled is not available from the driver");
  *fn = g_encode;
  return 0;
}

// Element kinds of make_map: the dtype codes FQKV_F16 / FQKV_BF16, and e4m3 bytes.
constexpr int kMapBF16 = FQKV_BF16, kMapE4M3 = 2;

// 2-D K-major tensor map over a [rows, cols] matrix with row stride ld (elements), 128-byte
// swizzle: 16-bit elements with box {64, box_rows}, or one-byte e4m3 elements with box
// {128, box_rows} -- 128-byte box rows either way.
// Encoded maps are cached by (address, shape, stride, box, dtype): a model calls the op
// with the same weight (and often the same activation buffers) every step, and a map
// holds only the address and the layout.
using MapKey = std::tuple<const void*, int64_t, int64_t, int64_t, int, int>;
std::mutex g_map_mu;
std::map<MapKey, CUtensorMap> g_map_cache;
constexpr size_t kMapCacheMax = 1024;

int make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows, int kind) {
  const MapKey key{base, rows, cols, ld, box_rows, kind};
  {
    std::lock_guard<std::mutex> lk(g_map_mu);
    auto it = g_map_cache.find(key);
    if (it != g_map_cache.end()) {
      *map = it->second;
      return 0;
    }
  }
  EncodeTiledFn enc;
  if (int rc = get_encode(&enc)) return rc;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const bool e4m3 = kind == kMapE4M3;
  const cuuint64_t strides[1] = {(cuuint64_t)(ld * (e4m3 ? 1 : 2))};
  const cuuint32_t box[2] = {e4m3 ? 128u : 64u, (cuuint32_t)box_rows};  // 128-byte box rows either way
  const cuuint32_t estr[2] = {1u, 1u};
  const CUtensorMapDataType dt = e4m3 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                      : kind == kMapBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                         : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(FQKV_ERR_ALIGN, "cuTensorMapEncodeTiled failed (%d) for a [%lld, %lld] matrix, ld %lld", (int)r,
                (long long)rows, (long long)cols, (long long)ld);
  std::lock_guard<std::mutex> lk(g_map_mu);
  if (g_map_cache.size() >= kMapCacheMax) g_map_cache.clear();
  g_map_cache.emplace(key, *map);
  return 0;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool overlaps(const void* a, int64_t a_bytes, const void* b, int64_t b_bytes) {
  if (!a || !b) return false;
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(a), b0 = reinterpret_cast<uintptr_t>(b);
  return a0 < b0 + (uintptr_t)b_bytes && b0 < a0 + (uintptr_t)a_bytes;
}

int64_t mat_bytes(int64_t rows, int64_t cols, int64_t ld) { return ((rows - 1) * ld + cols) * 2; }

// Bounds of the size-based automatic choice (M = tokens).
constexpr int64_t kDecodeMaxM = 64;   // automatic choice of the fused decode kernel
constexpr int64_t kFusedMaxM = 64;    // the fused kernel's limit when forced
constexpr int64_t kSplitMaxM = 128;   // pre-pass + swap-AB GEMM
constexpr int64_t kPrepassMaxH = 16384;

struct Problem {
  int64_t M, H, N, ldx, ldr, ldw, ldo, ldro;
  const void *x, *r, *g, *w;
  void *out, *rout;
  int dtype, gdt, schedule, flags;
  bool w16 = true;  // w is a 16-bit weight; false: the caller checks its own weight layout
};

bool tma_eligible(const Problem& p) {
  if (p.H % 8 || p.ldx % 8 || (p.w16 && p.ldw % 8)) return false;
  if (p.r && p.ldr % 8) return false;
  if (p.rout && p.ldro % 8) return false;
  if (!aligned16(p.x) || (p.w16 && !aligned16(p.w)) || !aligned16(p.g) || (p.r && !aligned16(p.r)) ||
      (p.rout && !aligned16(p.rout)))
    return false;
  if (p.H > kPrepassMaxH) return false;
  return true;
}

int auto_schedule_for(int64_t M, int64_t H, int64_t N, const DeviceInfo* dev);

// The current device's description, or nullptr (recording no error) when there is none.
const DeviceInfo* current_device_or_null(DeviceInfo* buf) {
  const std::string saved = t_last_error;
  if (device_info(buf) == 0) return buf;
  t_last_error = saved;
  cudaGetLastError();
  return nullptr;
}

int choose_schedule(const Problem& p) {
  if (p.schedule != FQKV_SCHED_AUTO) return p.schedule;
  if (!tma_eligible(p)) return FQKV_SCHED_SIMT;
  DeviceInfo d;
  return auto_schedule_for(p.M, p.H, p.N, current_device_or_null(&d));
}

int64_t align256(int64_t b) { return (b + 255) / 256 * 256; }

// Workspace layout: [normalised rows M x H][stream-K partial slots][stream-K counters].
int64_t workspace_for(int sched, int64_t M, int64_t H, int64_t N) {
  if (sched == FQKV_SCHED_PREFILL) return align256(M * H * 2);
  if (sched == FQKV_SCHED_SPLIT)
    return align256(M * H * 2) + align256(streamk_partials_bytes((int)M)) + align256(streamk_counters_bytes((int)N));
  if (sched == FQKV_SCHED_GRID) return align256(decode_grid_workspace_bytes(M, N));
  return 0;
}

// Measured on B200 (Llama-3-8B layer): the fused decode kernel beats the pre-pass
// schedules up to M = 64 (M = 64: 21 us against 27 us prefill, 30 us split), and the
// prefill GEMM beats the split schedule above that.  Decode is chosen only when one of its
// configurations fits the device (every cluster resident at once); otherwise the split
// schedule, which has no such limit, takes its place.  Without a device to ask (workspace
// queries on a machine with no GPU) the decode configuration is assumed to fit.
int auto_schedule_for(int64_t M, int64_t H, int64_t N, const DeviceInfo* dev) {
  if (H % 8 || H > kPrepassMaxH) return FQKV_SCHED_SIMT;
  if (M > kDecodeMaxM) return FQKV_SCHED_PREFILL;
  DecodeConfig c;
  if (!dev || dev->major != 10 || decode_pick_config((int)M, (int)H, (int)N, dev->sms, &c) == 0)
    return FQKV_SCHED_DECODE;
  return FQKV_SCHED_SPLIT;
}

int validate(const Problem& p) {
  if (!p.x || !p.g || (p.w16 && !p.w) || !p.out)
    return fail(FQKV_ERR_NULL, "x, rms_weight, weight and out must be non-null");
  if (p.dtype != FQKV_F16 && p.dtype != FQKV_BF16)
    return fail(FQKV_ERR_DTYPE, "dtype %d is not supported (fp16 = 0, bf16 = 1)", p.dtype);
  if (p.gdt != FQKV_F16 && p.gdt != FQKV_BF16 && p.gdt != FQKV_F32)
    return fail(FQKV_ERR_DTYPE, "rms_weight dtype %d is not supported", p.gdt);
  if (p.M <= 0 || p.H <= 0 || p.N <= 0)
    return fail(FQKV_ERR_SHAPE, "M, H and N must be positive (got %lld, %lld, %lld)", (long long)p.M,
                (long long)p.H, (long long)p.N);
  if (p.M > INT32_MAX || p.H > INT32_MAX || p.N > INT32_MAX)
    return fail(FQKV_ERR_SHAPE, "M, H and N must be below 2^31");
  if (p.ldx < p.H || p.ldw < p.H || p.ldo < p.N || (p.r && p.ldr < p.H) || (p.rout && p.ldro < p.H))
    return fail(FQKV_ERR_SHAPE, "a row stride is smaller than its row length");
  if (p.schedule < FQKV_SCHED_AUTO || p.schedule > FQKV_SCHED_GRID)
    return fail(FQKV_ERR_SCHEDULE, "unknown schedule %d", p.schedule);
  if (p.flags & ~(FQKV_FLAG_PDL | FQKV_FLAG_STATIC_WEIGHTS | FQKV_FLAG_TEST_WITHHOLD))
    return fail(FQKV_ERR_SCHEDULE, "unknown flag bits 0x%x", p.flags);
  const int64_t xb = mat_bytes(p.M, p.H, p.ldx), ob = mat_bytes(p.M, p.N, p.ldo);
  const int64_t wb = p.w16 ? mat_bytes(p.N, p.H, p.ldw) : 0;  // 0: overlaps() ignores it
  const int64_t rb = p.r ? mat_bytes(p.M, p.H, p.ldr) : 0, rob = p.rout ? mat_bytes(p.M, p.H, p.ldro) : 0;
  if (overlaps(p.out, ob, p.x, xb) || overlaps(p.out, ob, p.r, rb) || overlaps(p.out, ob, p.w, wb) ||
      overlaps(p.out, ob, p.rout, rob))
    return fail(FQKV_ERR_ALIAS, "out overlaps an input or residual_out");
  if (overlaps(p.rout, rob, p.x, xb) || overlaps(p.rout, rob, p.r, rb) || overlaps(p.rout, rob, p.w, wb))
    return fail(FQKV_ERR_ALIAS, "residual_out overlaps an input (in-place update is not supported)");
  const int sched = choose_schedule(p);
  if (sched == FQKV_SCHED_SIMT && (p.flags & FQKV_FLAG_TEST_WITHHOLD))
    return fail(FQKV_ERR_SCHEDULE, "FQKV_FLAG_TEST_WITHHOLD applies to the decode and grid schedules only");
  if (sched != FQKV_SCHED_SIMT) {
    if (!tma_eligible(p))
      return fail(FQKV_ERR_ALIGN,
                  "schedule %d needs H %% 8 == 0, H <= %lld, row strides %% 8 == 0 and 16-byte aligned x, "
                  "residual, rms_weight, weight and residual_out",
                  sched, (long long)kPrepassMaxH);
    if ((p.flags & FQKV_FLAG_TEST_WITHHOLD) && sched != FQKV_SCHED_DECODE && sched != FQKV_SCHED_GRID)
      return fail(FQKV_ERR_SCHEDULE, "FQKV_FLAG_TEST_WITHHOLD applies to the decode and grid schedules only");
    if (sched == FQKV_SCHED_DECODE && p.M > kFusedMaxM)
      return fail(FQKV_ERR_SCHEDULE, "the decode schedule takes at most %lld rows (M = %lld)",
                  (long long)kFusedMaxM, (long long)p.M);
    if (sched == FQKV_SCHED_GRID && (p.M > kGridMaxM || (p.N + 127) / 128 > kGridMaxTiles))
      return fail(FQKV_ERR_SCHEDULE, "the grid schedule takes at most %d rows and %d output features "
                  "(M = %lld, N = %lld)", kGridMaxM, kGridMaxTiles * 128, (long long)p.M, (long long)p.N);
    if (sched == FQKV_SCHED_SPLIT && p.M > kSplitMaxM)
      return fail(FQKV_ERR_SCHEDULE, "the split schedule takes at most %lld rows (M = %lld)",
                  (long long)kSplitMaxM, (long long)p.M);
  }
  return 0;
}

}  // namespace

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device) and size:
// the attribute only has to cover the largest request seen.
cudaError_t ensure_smem_attr(const void* func, size_t bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const auto key = std::make_pair(func, dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = done.find(key);
    if (it != done.end() && it->second >= bytes) return cudaSuccess;
  }
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(mu);
  size_t& v = done[key];
  if (bytes > v) v = bytes;
  return cudaSuccess;
}

}  // namespace fqkv

using namespace fqkv;

extern "C" FQKV_API int fqkv_version(void) { return 102; }

#ifdef FQKV_TRACE
// Profiling builds only: the timeline buffer the kernels' trace points write to
// (fqkv_device.cuh), kTraceSlots 64-bit words per CTA record.
namespace fqkv {
__device__ unsigned long long* g_trace_buf = nullptr;
__device__ unsigned int g_trace_cap = 0;
__device__ unsigned int g_trace_ctr = 0;
}  // namespace fqkv

extern "C" FQKV_API int fqkv_trace_attach(void* buf, unsigned int records) {
  unsigned long long* b = static_cast<unsigned long long*>(buf);
  const unsigned int zero = 0;
  cudaError_t e = cudaMemcpyToSymbol(g_trace_buf, &b, sizeof(b));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_trace_cap, &records, sizeof(records));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_trace_ctr, &zero, sizeof(zero));
  return e == cudaSuccess ? 0 : cuda_fail(e, "fqkv_trace_attach");
}
#endif

// The projection's [M, (n_q + 2 n_kv) d] output to head-major Q, K, V with the rotary
// embedding on Q and K (fqkv_rope.cu): what llama3_patch.py:156-168 does in PyTorch after
// the fused call (split, view as heads, transpose, apply_rotary_pos_emb).
// The op with e4m3 weights and an fp32 scale per weight row: the fused decode kernel
// streams the one-byte weight into e4m3 x e4m3 tensor-core MMAs against the normalised
// activations split exactly into e4m3 terms (a power-of-two scale per token), and the row
// scale multiplies the k-summed value once.  Decode schedule only (M <= 64 with a fitting
// configuration).
extern "C" FQKV_API int fqkv_launch_fp8w(const void* x, const void* residual, const void* rms_weight,
                                         int rms_weight_dtype, const void* weight, const float* weight_scale,
                                         void* out, void* residual_out, int64_t M, int64_t H, int64_t N, int64_t ldx,
                                         int64_t ldr, int64_t ldw, int64_t ldo, int64_t ldro, float eps, int dtype,
                                         int flags, void* stream) {
  if (!weight || !weight_scale) return fail(FQKV_ERR_NULL, "weight and weight_scale must be non-null");
  if (flags & FQKV_FLAG_TEST_WITHHOLD)
    return fail(FQKV_ERR_SCHEDULE, "FQKV_FLAG_TEST_WITHHOLD applies to fqkv_launch only");
  // The rest is checked as fqkv_launch checks it, on the decode schedule; the one-byte
  // weight's layout and aliasing are checked here.
  Problem p{M, H, N, ldx, ldr, ldw, ldo, ldro, x, residual, rms_weight, nullptr, out, residual_out,
            dtype, rms_weight_dtype, FQKV_SCHED_DECODE, flags, false};
  if (int rc = validate(p)) return rc;
  if (ldw < H) return fail(FQKV_ERR_SHAPE, "ldw %lld is smaller than H = %lld", (long long)ldw, (long long)H);
  if (!aligned16(weight) || ldw % 16)
    return fail(FQKV_ERR_ALIGN, "the e4m3 weight needs a 16-byte aligned address and a row pitch of 16-byte multiples");
  if (reinterpret_cast<uintptr_t>(weight_scale) & 3u) return fail(FQKV_ERR_ALIGN, "weight_scale must be 4-byte aligned");
  const int64_t wb = (N - 1) * ldw + H, sb = N * 4;
  const int64_t ob = mat_bytes(M, N, ldo), rob = residual_out ? mat_bytes(M, H, ldro) : 0;
  if (overlaps(out, ob, weight, wb) || overlaps(out, ob, weight_scale, sb) || overlaps(residual_out, rob, weight, wb) ||
      overlaps(residual_out, rob, weight_scale, sb))
    return fail(FQKV_ERR_ALIAS, "out or residual_out overlaps the weight or its scale");
  DeviceInfo d;
  if (int rc = device_info(&d)) return rc;
  if (d.major != 10) return fail(FQKV_ERR_DEVICE, "compute capability %d.%d is not sm_100", d.major, d.minor);
  DecodeConfig c;
  if (decode_pick_config((int)M, (int)H, (int)N, d.sms, &c, decode_f8_terms(dtype == FQKV_BF16))) {
    // More than 32 rows: the activations' e4m3 terms of a K slice may not fit beside the
    // ring (fp16 takes three terms per value).  The rows are independent, so the first 32
    // and the rest run as two launches (each streams the weight once).
    if (M > 32 && decode_pick_config(32, (int)H, (int)N, d.sms, &c, decode_f8_terms(dtype == FQKV_BF16)) == 0) {
      const char* xb = static_cast<const char*>(x);
      const char* rb = static_cast<const char*>(residual);
      char* ob2 = static_cast<char*>(out);
      char* rob2 = static_cast<char*>(residual_out);
      if (int rc = fqkv_launch_fp8w(x, residual, rms_weight, rms_weight_dtype, weight, weight_scale, out,
                                    residual_out, 32, H, N, ldx, ldr, ldw, ldo, ldro, eps, dtype, flags, stream))
        return rc;
      return fqkv_launch_fp8w(xb + 32 * ldx * 2, rb ? rb + 32 * ldr * 2 : nullptr, rms_weight, rms_weight_dtype, weight,
                              weight_scale, ob2 + 32 * ldo * 2, rob2 ? rob2 + 32 * ldro * 2 : nullptr, M - 32, H, N,
                              ldx, ldr, ldw, ldo, ldro, eps, dtype, flags, stream);
    }
    return fail(FQKV_ERR_SCHEDULE,
                "no fused decode configuration takes M = %lld, H = %lld, N = %lld with e4m3 weights (M <= 64)",
                (long long)M, (long long)H, (long long)N);
  }
  CUtensorMap tmW;
  if (int rc = make_map(&tmW, weight, N, H, ldw, 128 * decode_box_tiles(c.nt), kMapE4M3)) return rc;
  DecodeParams dp{static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(residual), rms_weight,
                  rms_weight_dtype, static_cast<uint16_t*>(out), static_cast<uint16_t*>(residual_out), (int)M,
                  (int)H, (int)N, ldx, ldr, ldo, ldro, eps, (int)((H + 63) / 64), 0, flags, 0, 0, weight_scale};
  dp.nkb_max = decode_slice_max(c.cluster, dp.kb_total, true);
  // Rings of two stages skip programmatic dependent launch (as on the 16-bit path; here at
  // every M: the N = 28672 configuration measured 65.9 us at M = 1 with it).
  const bool pdl = (flags & FQKV_FLAG_PDL) != 0 && c.stages > 2;
  const cudaError_t e = launch_decode(c, tmW, dp, dtype == FQKV_BF16, pdl, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? 0 : cuda_fail(e, "decode kernel launch (e4m3 weights)");
}

extern "C" FQKV_API int fqkv_rope_split(const void* qkv, int64_t ldq, const void* cos, const void* sin,
                                        int64_t cos_batch, void* q, void* k, void* v, int64_t B, int64_t S,
                                        int n_q_heads, int n_kv_heads, int head_dim, int dtype, void* stream) {
  if (dtype != FQKV_F16 && dtype != FQKV_BF16)
    return fail(FQKV_ERR_DTYPE, "dtype %d is not supported (fp16 = 0, bf16 = 1)", dtype);
  if (!qkv || !cos || !sin || !q || !k || !v) return fail(FQKV_ERR_NULL, "qkv, cos, sin, q, k and v must be non-null");
  if (B <= 0 || S <= 0 || n_q_heads <= 0 || n_kv_heads <= 0)
    return fail(FQKV_ERR_SHAPE, "B, S and the head counts must be positive");
  if (head_dim <= 0 || head_dim % 16)
    return fail(FQKV_ERR_SHAPE, "head_dim %d must be a positive multiple of 16", head_dim);
  const int64_t width = (int64_t)(n_q_heads + 2 * n_kv_heads) * head_dim;
  if (ldq < width) return fail(FQKV_ERR_SHAPE, "ldq %lld is smaller than the row (%lld)", (long long)ldq, (long long)width);
  if (cos_batch != 1 && cos_batch != B)
    return fail(FQKV_ERR_SHAPE, "cos / sin must hold 1 or B = %lld batch rows (got %lld)", (long long)B,
                (long long)cos_batch);
  if (!aligned16(qkv) || !aligned16(cos) || !aligned16(sin) || !aligned16(q) || !aligned16(k) || !aligned16(v) ||
      ldq % 8)
    return fail(FQKV_ERR_ALIGN, "every pointer must be 16-byte aligned and ldq a multiple of 8");
  const int64_t M = B * S;
  const int64_t qkv_b = mat_bytes(M, width, ldq), cs_b = cos_batch * S * head_dim * 2;
  const int64_t q_b = M * n_q_heads * head_dim * 2, kv_b = M * n_kv_heads * head_dim * 2;
  const void* ins[3] = {qkv, cos, sin};
  const int64_t in_b[3] = {qkv_b, cs_b, cs_b};
  void* outs[3] = {q, k, v};
  const int64_t out_b[3] = {q_b, kv_b, kv_b};
  for (int i = 0; i < 3; ++i) {
    for (int j = 0; j < 3; ++j)
      if (overlaps(outs[i], out_b[i], ins[j], in_b[j]))
        return fail(FQKV_ERR_ALIAS, "q, k and v must not overlap qkv, cos or sin");
    for (int j = i + 1; j < 3; ++j)
      if (overlaps(outs[i], out_b[i], outs[j], out_b[j])) return fail(FQKV_ERR_ALIAS, "q, k and v must not overlap");
  }
  DeviceInfo d;
  if (int rc = device_info(&d)) return rc;
  if (d.major != 10) return fail(FQKV_ERR_DEVICE, "compute capability %d.%d is not sm_100", d.major, d.minor);
  RopeParams rp{static_cast<const uint16_t*>(qkv), static_cast<const uint16_t*>(cos), static_cast<const uint16_t*>(sin),
                static_cast<uint16_t*>(q), static_cast<uint16_t*>(k), static_cast<uint16_t*>(v), M, S, ldq,
                cos_batch == 1 ? 0 : S * head_dim, n_q_heads, n_kv_heads, head_dim};
  const cudaError_t e = launch_rope_split(rp, dtype == FQKV_BF16, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? 0 : cuda_fail(e, "rope split kernel launch");
}

// The op with the Q/K/V split and the rotary embedding in its epilogue: each CTA of the
// fused decode kernel reduces whole 128-row blocks of the output and writes them head-major
// (Q and K rotated) instead of the packed output.  Replaces fqkv_launch followed by
// fqkv_rope_split (the llama3_patch.py:148-168 sequence) with one launch, bit-identical to
// the two.
extern "C" FQKV_API int fqkv_launch_rope(const void* x, const void* residual, const void* rms_weight,
                                         int rms_weight_dtype, const void* weight, void* q, void* k, void* v,
                                         void* residual_out, int64_t B, int64_t S, int64_t H, int64_t ldx,
                                         int64_t ldr, int64_t ldw, int64_t ldro, const void* cos, const void* sin,
                                         int64_t cos_batch, int n_q_heads, int n_kv_heads, int head_dim, float eps,
                                         int dtype, int flags, void* stream) {
  if (!x || !rms_weight || !weight || !q || !k || !v || !cos || !sin)
    return fail(FQKV_ERR_NULL, "x, rms_weight, weight, q, k, v, cos and sin must be non-null");
  if (dtype != FQKV_F16 && dtype != FQKV_BF16)
    return fail(FQKV_ERR_DTYPE, "dtype %d is not supported (fp16 = 0, bf16 = 1)", dtype);
  if (rms_weight_dtype != FQKV_F16 && rms_weight_dtype != FQKV_BF16 && rms_weight_dtype != FQKV_F32)
    return fail(FQKV_ERR_DTYPE, "rms_weight dtype %d is not supported", rms_weight_dtype);
  if (B <= 0 || S <= 0 || H <= 0 || n_q_heads <= 0 || n_kv_heads <= 0)
    return fail(FQKV_ERR_SHAPE, "B, S, H and the head counts must be positive");
  if (head_dim != 64 && head_dim != 128)
    return fail(FQKV_ERR_SHAPE, "head_dim %d: the fused rotary epilogue takes 64 or 128", head_dim);
  if (cos_batch != 1 && cos_batch != B)
    return fail(FQKV_ERR_SHAPE, "cos / sin must hold 1 or B = %lld batch rows (got %lld)", (long long)B,
                (long long)cos_batch);
  if (flags & ~(FQKV_FLAG_PDL | FQKV_FLAG_STATIC_WEIGHTS))
    return fail(FQKV_ERR_SCHEDULE, "unknown flag bits 0x%x", flags);
  const int64_t M = B * S, N = (int64_t)(n_q_heads + 2 * n_kv_heads) * head_dim;
  if (M > kDecodeRopeMaxM)
    return fail(FQKV_ERR_SCHEDULE, "the fused rotary epilogue takes at most %d tokens (M = %lld); use fqkv_launch "
                "and fqkv_rope_split", kDecodeRopeMaxM, (long long)M);
  if (H > INT32_MAX || N > INT32_MAX) return fail(FQKV_ERR_SHAPE, "H and N must be below 2^31");
  if (ldx < H || ldw < H || (residual && ldr < H) || (residual_out && ldro < H))
    return fail(FQKV_ERR_SHAPE, "a row stride is smaller than its row length");
  Problem p{M, H, N, ldx, ldr, ldw, N, ldro, x, residual, rms_weight, weight, q, residual_out,
            dtype, rms_weight_dtype, FQKV_SCHED_DECODE, flags};
  if (!tma_eligible(p) || !aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(cos) || !aligned16(sin))
    return fail(FQKV_ERR_ALIGN, "the fused rotary epilogue needs H %% 8 == 0, H <= %lld, row strides %% 8 == 0 and "
                "16-byte aligned tensors", (long long)kPrepassMaxH);
  const int64_t xb = mat_bytes(M, H, ldx), wb = mat_bytes(N, H, ldw);
  const int64_t rb = residual ? mat_bytes(M, H, ldr) : 0, rob = residual_out ? mat_bytes(M, H, ldro) : 0;
  const int64_t qb = M * n_q_heads * head_dim * 2, kvb = M * n_kv_heads * head_dim * 2;
  const int64_t csb = cos_batch * S * head_dim * 2;
  const void* ins[5] = {x, residual, weight, cos, sin};
  const int64_t in_b[5] = {xb, rb, wb, csb, csb};
  void* outs[4] = {q, k, v, residual_out};
  const int64_t out_b[4] = {qb, kvb, kvb, rob};
  for (int i = 0; i < 4; ++i) {
    for (int j = 0; j < 5; ++j)
      if (overlaps(outs[i], out_b[i], ins[j], in_b[j]))
        return fail(FQKV_ERR_ALIAS, "q, k, v and residual_out must not overlap an input");
    for (int j = i + 1; j < 4; ++j)
      if (overlaps(outs[i], out_b[i], outs[j], out_b[j]))
        return fail(FQKV_ERR_ALIAS, "q, k, v and residual_out must not overlap each other");
  }
  DeviceInfo d;
  if (int rc = device_info(&d)) return rc;
  if (d.major != 10) return fail(FQKV_ERR_DEVICE, "compute capability %d.%d is not sm_100", d.major, d.minor);
  DecodeConfig c;
  if (decode_pick_config((int)M, (int)H, (int)N, d.sms, &c) || c.recv_in_normed != kDecodeRecvOwn || c.grid || c.f8)
    return fail(FQKV_ERR_SCHEDULE, "no decode configuration with the rotary epilogue takes M = %lld, H = %lld, "
                "N = %lld; use fqkv_launch and fqkv_rope_split", (long long)M, (long long)H, (long long)N);
  const bool bf16 = dtype == FQKV_BF16;
  CUtensorMap tmW;
  if (int rc = make_map(&tmW, weight, N, H, ldw, 128 * decode_box_tiles(c.nt), bf16)) return rc;
  DecodeParams dp{static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(residual), rms_weight,
                  rms_weight_dtype, nullptr, static_cast<uint16_t*>(residual_out), (int)M, (int)H, (int)N, ldx, ldr,
                  N, ldro, eps, (int)((H + 63) / 64), 0, flags, 0, 0, nullptr};
  dp.nkb_max = (dp.kb_total + c.cluster - 1) / c.cluster;
  dp.q = static_cast<uint16_t*>(q);
  dp.k = static_cast<uint16_t*>(k);
  dp.v = static_cast<uint16_t*>(v);
  dp.cos = static_cast<const uint16_t*>(cos);
  dp.sin = static_cast<const uint16_t*>(sin);
  dp.S = S;
  dp.cs_batch_stride = cos_batch == 1 ? 0 : S * head_dim;
  dp.n_q = n_q_heads;
  dp.n_kv = n_kv_heads;
  dp.head_dim = head_dim;
  const bool pdl = (flags & FQKV_FLAG_PDL) != 0 && (c.stages > 2 || M == 1);
  const cudaError_t e = launch_decode(c, tmW, dp, bf16, pdl, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? 0 : cuda_fail(e, "decode kernel launch (rotary epilogue)");
}

extern "C" FQKV_API const char* fqkv_last_error(void) { return t_last_error.c_str(); }

extern "C" FQKV_API int64_t fqkv_workspace_bytes(int64_t M, int64_t H, int64_t N, int dtype, int schedule) {
  if (M <= 0 || H <= 0 || N <= 0) return -fail(FQKV_ERR_SHAPE, "M, H and N must be positive");
  if (dtype != FQKV_F16 && dtype != FQKV_BF16) return -fail(FQKV_ERR_DTYPE, "unsupported dtype %d", dtype);
  if (schedule < FQKV_SCHED_AUTO || schedule > FQKV_SCHED_GRID)
    return -fail(FQKV_ERR_SCHEDULE, "unknown schedule %d", schedule);
  DeviceInfo d;
  const int sched = schedule == FQKV_SCHED_AUTO ? auto_schedule_for(M, H, N, current_device_or_null(&d)) : schedule;
  return workspace_for(sched, M, H, N);
}

extern "C" FQKV_API int fqkv_query_schedule(int64_t M, int64_t H, int64_t N, int dtype, int schedule,
                                   fqkv_schedule_info* info) {
  if (!info) return fail(FQKV_ERR_NULL, "info must be non-null");
  if (M <= 0 || H <= 0 || N <= 0) return fail(FQKV_ERR_SHAPE, "M, H and N must be positive");
  if (dtype != FQKV_F16 && dtype != FQKV_BF16) return fail(FQKV_ERR_DTYPE, "unsupported dtype %d", dtype);
  if (schedule < FQKV_SCHED_AUTO || schedule > FQKV_SCHED_GRID)
    return fail(FQKV_ERR_SCHEDULE, "unknown schedule %d", schedule);
  DeviceInfo d;
  if (int rc = device_info(&d)) return rc;
  const int sched = schedule == FQKV_SCHED_AUTO ? auto_schedule_for(M, H, N, &d) : schedule;
  std::memset(info, 0, sizeof(*info));
  info->schedule = sched;
  if (sched == FQKV_SCHED_SIMT) {
    info->block_m = 8;
    info->block_n = 64;
    info->block_k = 64;
    info->stages = 1;
    info->split_k = 1;
    info->grid = (int)(((N + 63) / 64) * ((M + 7) / 8));
    info->threads = 256;
    info->smem_bytes = (int)(sizeof(float) * (8 + 8 * 64 + 64 * 65));
    return 0;
  }
  if (sched == FQKV_SCHED_DECODE) {
    DecodeConfig c;
    if (int rc = decode_pick_config((int)M, (int)H, (int)N, d.sms, &c)) return rc;
    info->block_m = c.mpad;
    info->block_n = 128 * c.nt;
    info->block_k = 64;
    info->stages = c.stages;
    info->split_k = c.cluster;
    info->grid = (int)(((N + 128 * c.nt - 1) / (128 * c.nt)) * c.cluster);
    info->threads = kDecodeThreads;
    info->smem_bytes = (int)c.smem;
    info->uses_prepass = 0;
    return 0;
  }
  if (sched == FQKV_SCHED_GRID) {
    if (M > kGridMaxM) return fail(FQKV_ERR_SCHEDULE, "the grid schedule takes at most %d rows", kGridMaxM);
    DecodeConfig c;
    if (int rc = decode_grid_pick_config((int)M, (int)H, (int)N, d.sms, &c))
      return fail(rc, "no grid configuration fits H=%lld N=%lld", (long long)H, (long long)N);
    info->block_m = c.mpad;
    info->block_n = 128 * c.nt;
    info->block_k = 64;
    info->stages = c.stages;
    info->split_k = c.cluster;
    info->grid = (int)(((N + 128 * c.nt - 1) / (128 * c.nt)) * c.cluster);
    info->threads = kDecodeThreads;
    info->smem_bytes = (int)c.smem;
    info->uses_prepass = 0;
    return 0;
  }
  if (sched == FQKV_SCHED_SPLIT) {
    StreamKConfig c;
    if (int rc = streamk_pick_config((int)M, (int)H, (int)N, d.sms, &c)) return rc;
    info->block_m = c.mpad;
    info->block_n = 128;
    info->block_k = 64;
    info->stages = c.stages;
    info->split_k = 0;  // stream-K: ranges of (tile, k-block) units, not a fixed split
    info->grid = c.grid;
    info->threads = 192;
    info->smem_bytes = (int)c.smem;
    info->uses_prepass = 1;
    return 0;
  }
  GemmConfig g;
  if (int rc = gemm_pick_config((int)M, (int)H, (int)N, d.sms, &g)) return rc;
  info->block_m = g.pair ? 256 : 128;
  info->block_n = g.bn;
  info->block_k = 64;
  info->stages = g.stages;
  info->split_k = 1;
  info->grid = g.grid;
  info->threads = 192;
  info->smem_bytes = (int)g.smem;
  info->uses_prepass = 1;
  return 0;
}

extern "C" FQKV_API int fqkv_device_status(void* stream, int* status) {
  if (!status) return fail(FQKV_ERR_NULL, "status must be non-null");
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  int v = 0, zero = 0;
  if ((e = cudaMemcpyFromSymbol(&v, g_status, sizeof(int))) != cudaSuccess)
    return cuda_fail(e, "cudaMemcpyFromSymbol");
  if ((e = cudaMemcpyToSymbol(g_status, &zero, sizeof(int))) != cudaSuccess)
    return cuda_fail(e, "cudaMemcpyToSymbol");
  *status = v;
  return 0;
}

extern "C" FQKV_API int fqkv_test_set_wait_limit_ns(unsigned long long ns) {
  const unsigned long long v = ns ? ns : kWaitLimitNs;
  const cudaError_t e = cudaMemcpyToSymbol(g_wait_limit_ns, &v, sizeof(v));
  return e == cudaSuccess ? 0 : cuda_fail(e, "cudaMemcpyToSymbol(wait limit)");
}

extern "C" FQKV_API int fqkv_stream_capture_id(void* stream, unsigned long long* id) {
  if (!id) return fail(FQKV_ERR_NULL, "id must be non-null");
  cudaStreamCaptureStatus status = cudaStreamCaptureStatusNone;
  unsigned long long cid = 0;
  const cudaError_t e = cudaStreamGetCaptureInfo(static_cast<cudaStream_t>(stream), &status, &cid);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamGetCaptureInfo");
  *id = status == cudaStreamCaptureStatusActive ? cid : 0ull;
  return 0;
}

extern "C" FQKV_API int fqkv_launch(const void* x, const void* residual, const void* rms_weight, int rms_weight_dtype,
                           const void* weight, void* out, void* residual_out, int64_t M, int64_t H, int64_t N,
                           int64_t ldx, int64_t ldr, int64_t ldw, int64_t ldo, int64_t ldro, float eps, int dtype,
                           int schedule, int flags, void* workspace, int64_t workspace_bytes, void* stream) {
  Problem p{M, H, N, ldx, ldr, ldw, ldo, ldro, x, residual, rms_weight, weight, out, residual_out,
            dtype, rms_weight_dtype, schedule, flags};
  if (int rc = validate(p)) return rc;
  const int sched = choose_schedule(p);
  const int64_t need = workspace_for(sched, M, H, N);
  if (need > 0) {
    if (!workspace || workspace_bytes < need)
      return fail(FQKV_ERR_WORKSPACE, "schedule %d needs %lld bytes of workspace (got %lld)", sched,
                  (long long)need, (long long)(workspace ? workspace_bytes : 0));
    if (reinterpret_cast<uintptr_t>(workspace) & 255u)
      return fail(FQKV_ERR_ALIGN, "workspace must be 256-byte aligned");
  }
  DeviceInfo d;
  if (int rc = device_info(&d)) return rc;
  if (d.major != 10) return fail(FQKV_ERR_DEVICE, "compute capability %d.%d is not sm_100", d.major, d.minor);

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf16 = dtype == FQKV_BF16;
  const bool pdl = (flags & FQKV_FLAG_PDL) != 0;
  const auto* xs = static_cast<const uint16_t*>(x);
  const auto* rs = static_cast<const uint16_t*>(residual);
  cudaError_t e = cudaSuccess;

  if (sched == FQKV_SCHED_SIMT) {
    SimtParams sp{xs, rs, rms_weight, rms_weight_dtype, static_cast<const uint16_t*>(weight),
                  static_cast<uint16_t*>(out), static_cast<uint16_t*>(residual_out), M, H, N, ldx, ldr, ldw,
                  ldo, ldro, eps};
    e = launch_simt(sp, bf16, pdl, st);
    return e == cudaSuccess ? 0 : cuda_fail(e, "simt kernel launch");
  }

  uint16_t* normed = static_cast<uint16_t*>(workspace);
  if (sched == FQKV_SCHED_DECODE) {
    DecodeConfig c;
    if (int rc = decode_pick_config((int)M, (int)H, (int)N, d.sms, &c)) return rc;
    CUtensorMap tmW;
    if (int rc = make_map(&tmW, weight, N, H, ldw, 128 * decode_box_tiles(c.nt), bf16)) return rc;
    DecodeParams dp{xs, rs, rms_weight, rms_weight_dtype, static_cast<uint16_t*>(out),
                    static_cast<uint16_t*>(residual_out), (int)M, (int)H, (int)N, ldx, ldr, ldo, ldro, eps,
                    (int)((H + 63) / 64), 0, flags, 0, 0, nullptr};
    dp.nkb_max = (dp.kb_total + c.cluster - 1) / c.cluster;
    // A ring of two stages (the wide-weight configurations, 64-80 KB stages) is filled
    // entirely by the stages issued ahead of the preceding grid, and then the stream
    // waits for that grid and the whole norm phase.  Measured on B200 (graph-timed, H =
    // 4096): with programmatic dependent launch N = 28672 took 62.6 us at M = 16 against
    // 48.6 us without it, and N = 22528 45.9 against 40.2 us; at M = 1 the two are within
    // 2 us.  Rings of 3 or more stages gain 1.4-2.5 us from it at every M.
    const bool decode_pdl = pdl && (c.stages > 2 || M == 1);
    e = launch_decode(c, tmW, dp, bf16, decode_pdl, st);
    return e == cudaSuccess ? 0 : cuda_fail(e, "decode kernel launch");
  }

  if (sched == FQKV_SCHED_GRID) {
    DecodeConfig c;
    if (int rc = decode_grid_pick_config((int)M, (int)H, (int)N, d.sms, &c))
      return fail(rc, "no grid configuration fits H=%lld N=%lld", (long long)H, (long long)N);
    CUtensorMap tmW;
    if (int rc = make_map(&tmW, weight, N, H, ldw, 128 * decode_box_tiles(c.nt), bf16)) return rc;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    DecodeParams dp{xs, rs, rms_weight, rms_weight_dtype, static_cast<uint16_t*>(out),
                    static_cast<uint16_t*>(residual_out), (int)M, (int)H, (int)N, ldx, ldr, ldo, ldro, eps,
                    (int)((H + 63) / 64), 0, flags, 0, 0, nullptr,
                    reinterpret_cast<float*>(ws + decode_grid_counter_bytes()),
                    reinterpret_cast<int*>(ws)};
    dp.nkb_max = (dp.kb_total + c.cluster - 1) / c.cluster;
    e = launch_decode(c, tmW, dp, bf16, pdl && (c.stages > 2 || M == 1), st);
    return e == cudaSuccess ? 0 : cuda_fail(e, "grid decode kernel launch");
  }

  // Pre-pass: updated residual + normalised rows (+ zeroed stream-K counters).
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const int64_t normed_bytes = align256(M * H * 2);
  float* partials = reinterpret_cast<float*>(ws + normed_bytes);
  int* counters = reinterpret_cast<int*>(ws + normed_bytes + align256(streamk_partials_bytes((int)M)));
  const int tiles128 = (int)((N + 127) / 128);
  {
    PrepassParams pp{xs, rs, rms_weight, rms_weight_dtype, static_cast<uint16_t*>(residual_out), normed, M, H,
                     ldx, ldr, ldro, eps, sched == FQKV_SCHED_SPLIT ? counters : nullptr,
                     sched == FQKV_SCHED_SPLIT ? tiles128 : 0};
    e = launch_prepass(pp, bf16, pdl, st);
    if (e != cudaSuccess) return cuda_fail(e, "norm pre-pass launch");
  }

  if (sched == FQKV_SCHED_SPLIT) {
    StreamKConfig c;
    if (int rc = streamk_pick_config((int)M, (int)H, (int)N, d.sms, &c)) return rc;
    CUtensorMap tmW, tmB;
    if (int rc = make_map(&tmW, weight, N, H, ldw, 128, bf16)) return rc;
    if (int rc = make_map(&tmB, normed, M, H, H, c.mpad, bf16)) return rc;
    StreamKParams sp{static_cast<uint16_t*>(out), partials, counters, (int)M, (int)N, (int)H, ldo,
                     (int)((H + 63) / 64), tiles128, flags, c.b_slots, c.w_evict_first};
    // Chained to the pre-pass: the GEMM may start streaming the weight before the
    // pre-pass finishes only if the caller declared the weight static.
    e = launch_streamk(c, tmW, tmB, sp, bf16, true, st);
    return e == cudaSuccess ? 0 : cuda_fail(e, "stream-K GEMM launch");
  }

  GemmConfig g;
  if (int rc = gemm_pick_config((int)M, (int)H, (int)N, d.sms, &g)) return rc;
  CUtensorMap tmA, tmB, tmO;
  if (int rc = make_map(&tmA, normed, M, H, H, 128, bf16)) return rc;
  if (int rc = make_map(&tmB, weight, N, H, ldw, g.pair ? g.bn / 2 : g.bn, bf16)) return rc;
  // The CTA-pair kernel stores its tiles through a map of `out` (128 x 64 boxes) when the
  // output's address and row pitch are 16-byte multiples.
  const bool out_tma = g.pair && aligned16(out) && (ldo % 8) == 0;
  if (out_tma) {
    if (int rc = make_map(&tmO, out, M, N, ldo, 128, bf16)) return rc;
  } else {
    std::memset(&tmO, 0, sizeof(tmO));
  }
  const int64_t bm = g.pair ? 256 : 128;
  GemmParams gp{static_cast<uint16_t*>(out), (int)M, (int)N, (int)H, ldo, (int)((H + 63) / 64),
                (int)((M + bm - 1) / bm), (int)((N + g.bn - 1) / g.bn), flags, out_tma ? 1 : 0};
  e = launch_gemm(g, tmA, tmB, tmO, gp, bf16, true, st);
  return e == cudaSuccess ? 0 : cuda_fail(e, "prefill GEMM launch");
}

// ---------------------------------------------------------------------------
// Allocation-free entry point.
//
// Some callers cannot allocate device memory when they run the op: an inference
// engine's plugin whose enqueue step must not allocate (the engine owns all memory and
// forbids the implicit device synchronisation cudaMalloc can cause), or a runtime with a
// fixed memory budget that allocates nothing after start-up.  They cannot hand
// fqkv_launch the workspace its pre-pass
// schedule needs, so fqkv_launch_noalloc runs that schedule (norm pre-pass + stream-K
// GEMM) on a fixed array of device memory that belongs to the library.
//
// The array is a file-scope __device__ variable: every GPU that loads the library holds
// its own copy (kNoAllocScratchBytes, about 5.5 MB) until the process exits.  Its
// device address is looked up with cudaGetSymbolAddress the first time the entry point
// runs on a device in a CUDA context (with that device and context current); make that
// first call before capturing a stream.  All calls on a device share the array and it keeps the last call's contents:
// the pre-pass zeroes the arrival counters each call, the other regions are fully
// rewritten before they are read.  Calls whose kernels overlap on the GPU (e.g. issued
// on two streams at once) race on the array and must be serialised by the caller.
// ---------------------------------------------------------------------------
namespace fqkv {
namespace {

constexpr int64_t kNoAllocMaxM = 16;
constexpr int64_t kNoAllocMaxH = 8192;
constexpr int64_t kNoAllocMaxN = 16384;
constexpr size_t kNoAllocNormedBytes = (size_t)kNoAllocMaxM * kNoAllocMaxH * 2;           // 256 KiB
constexpr size_t kNoAllocPartialBytes = (size_t)kStreamKMaxGrid * 2 * 16 * 128 * 4;       // 5 MiB (MPAD 16)
constexpr size_t kNoAllocCounterBytes = (size_t)((kNoAllocMaxN + 127) / 128) * 4;         // 512 B
constexpr size_t kNoAllocScratchBytes = kNoAllocNormedBytes + kNoAllocPartialBytes + kNoAllocCounterBytes;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Symbol addresses belong to a CUDA context: the address is cached per (device, context),
// so a caller that makes another context current on the same device gets that context's
// copy of the array.  The current context comes from the driver (cuCtxGetCurrent, reached
// through the runtime so the library does not link libcuda).
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
std::mutex g_noalloc_mu;
std::map<std::pair<int, CUcontext>, void*> g_noalloc_ptr;
CtxGetCurrentFn g_ctx_get_current = nullptr;
std::once_flag g_ctx_once;

// Device address of this device's (and context's) copy of g_noalloc_scratch, looked up once.
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(FQKV_ERR_DEVICE, "device ordinal %d out of range", dev);
  std::call_once(g_ctx_once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  if (!g_ctx_get_current) return fail(FQKV_ERR_DEVICE, "cuCtxGetCurrent is not available from the driver");
  CUcontext ctx = nullptr;
  if (g_ctx_get_current(&ctx) != CUDA_SUCCESS || !ctx)
    return fail(FQKV_ERR_DEVICE, "no current CUDA context on device %d", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  const auto key = std::make_pair(dev, ctx);
  auto it = g_noalloc_ptr.find(key);
  if (it == g_noalloc_ptr.end()) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(scratch)");
    it = g_noalloc_ptr.emplace(key, p).first;
  }
  *out = it->second;
  return 0;
}

}  // namespace
}  // namespace fqkv

extern "C" FQKV_API int fqkv_launch_noalloc(const void* x, const void* residual, const void* rms_weight,
                                            int rms_weight_dtype, const void* weight, void* out, void* residual_out,
                                            int64_t M, int64_t H, int64_t N, int64_t ldx, int64_t ldr, int64_t ldw,
                                            int64_t ldo, int64_t ldro, float eps, int dtype, int flags,
                                            void* stream) {
  Problem p{M, H, N, ldx, ldr, ldw, ldo, ldro, x, residual, rms_weight, weight, out, residual_out,
            dtype, rms_weight_dtype, FQKV_SCHED_SPLIT, flags};
  if (int rc = validate(p)) return rc;
  if (M > kNoAllocMaxM || H > kNoAllocMaxH || N > kNoAllocMaxN)
    return fail(FQKV_ERR_SHAPE,
                "fqkv_launch_noalloc takes M <= %lld, H <= %lld, N <= %lld (its scratch is a fixed %zu-byte "
                "device array); got M=%lld H=%lld N=%lld -- use fqkv_launch with a workspace",
                (long long)kNoAllocMaxM, (long long)kNoAllocMaxH, (long long)kNoAllocMaxN, kNoAllocScratchBytes,
                (long long)M, (long long)H, (long long)N);
  DeviceInfo d;
  if (int rc = device_info(&d)) return rc;
  if (d.major != 10) return fail(FQKV_ERR_DEVICE, "compute capability %d.%d is not sm_100", d.major, d.minor);
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;

  uint8_t* base = static_cast<uint8_t*>(scratch);
  uint16_t* normed = reinterpret_cast<uint16_t*>(base);
  float* partials = reinterpret_cast<float*>(base + kNoAllocNormedBytes);
  int* counters = reinterpret_cast<int*>(base + kNoAllocNormedBytes + kNoAllocPartialBytes);
  const int tiles128 = (int)((N + 127) / 128);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf16 = dtype == FQKV_BF16;

  StreamKConfig c;
  if (int rc = streamk_pick_config((int)M, (int)H, (int)N, d.sms, &c)) return rc;
  if (c.mpad != 16) return fail(FQKV_ERR_SHAPE, "internal: unexpected tile width %d", c.mpad);
  CUtensorMap tmW, tmB;
  if (int rc = make_map(&tmW, weight, N, H, ldw, 128, bf16)) return rc;
  if (int rc = make_map(&tmB, normed, M, H, H, c.mpad, bf16)) return rc;

  PrepassParams pp{static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(residual), rms_weight,
                   rms_weight_dtype, static_cast<uint16_t*>(residual_out), normed, M, H, ldx, ldr, ldro, eps,
                   counters, tiles128};
  cudaError_t e = launch_prepass(pp, bf16, (flags & FQKV_FLAG_PDL) != 0, st);
  if (e != cudaSuccess) return cuda_fail(e, "norm pre-pass launch");
  StreamKParams sp{static_cast<uint16_t*>(out), partials, counters, (int)M, (int)N, (int)H, ldo,
                   (int)((H + 63) / 64), tiles128, flags, c.b_slots, c.w_evict_first};
  e = launch_streamk(c, tmW, tmB, sp, bf16, true, st);
  return e == cudaSuccess ? 0 : cuda_fail(e, "stream-K GEMM launch");
}
