// extern "C" entry points of libesa_b200.so (declared in include/esa_b200.h).
//
// Host-side validation, workspace layout, kernel selection and launch.  No
// entry point allocates device memory: outputs and workspace come from the
// caller (the Python module takes them from torch's caching allocator).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <mutex>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "esa_b200.h"
#include "esa_layer.h"
#include "esa_decode.cuh"
#include "esa_gather.cuh"
#include "esa_keymma.cuh"
#include "esa_layer.cuh"
#include "esa_pattern.cuh"
#include "esa_keyplan.cuh"
#include "esa_probe.cuh"
#include "esa_rows.cuh"
#include "esa_window_tc.cuh"
#include "esa_window_bwd.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(ESA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return ESA_OK;
}

constexpr int64_t kMaxPosition = int64_t(1) << 24;  // float32 index math is exact below 2^24
constexpr int kMaxAttnLength = 2048;

esa::Pattern make_pattern(int num_heads, int w, int layer_idx, int num_hidden_layers,
                          int head_offset = 0) {
  esa::Pattern P;
  const int denominator = num_hidden_layers > 1 ? num_hidden_layers - 1 : 1;   // :488
  const double alpha = (double)layer_idx / (double)denominator;                // :489
  P.w = w;
  P.num_heads = num_heads;
  P.a = (float)alpha;
  P.c = (float)((double)w * (1.0 - alpha));                                    // :496
  P.head_offset = head_offset;
  return P;
}

// Query heads of the pattern a problem's heads belong to.
int pattern_heads(const esa_problem_t* pb) {
  return pb->pattern_heads > 0 ? pb->pattern_heads : pb->num_heads;
}

// ---- launch trace ----------------------------------------------------------
// While enabled, every launch below is bracketed by two events recorded on its
// stream (esa_trace_* in include/esa_b200.h).
struct TraceRec {
  const char* name;
  cudaEvent_t a, b;
};
std::mutex g_trace_mu;
std::atomic<bool> g_trace_on{false};
std::vector<TraceRec> g_trace;

class LaunchTrace {
 public:
  LaunchTrace(const char* name, cudaStream_t s) : s_(s) {
    if (!g_trace_on.load(std::memory_order_relaxed)) return;
    TraceRec r{name, nullptr, nullptr};
    if (cudaEventCreate(&r.a) != cudaSuccess) return;
    if (cudaEventCreate(&r.b) != cudaSuccess) {
      cudaEventDestroy(r.a);
      return;
    }
    cudaEventRecord(r.a, s);
    std::lock_guard<std::mutex> lock(g_trace_mu);
    g_trace.push_back(r);
    end_ = r.b;
  }
  ~LaunchTrace() {
    if (end_) cudaEventRecord(end_, s_);
  }
  LaunchTrace(const LaunchTrace&) = delete;
  LaunchTrace& operator=(const LaunchTrace&) = delete;

 private:
  cudaStream_t s_;
  cudaEvent_t end_ = nullptr;
};

void trace_clear() {
  std::lock_guard<std::mutex> lock(g_trace_mu);
  for (auto& r : g_trace) {
    cudaEventDestroy(r.a);
    cudaEventDestroy(r.b);
  }
  g_trace.clear();
}

int elem_size(int dtype) { return dtype == ESA_DTYPE_F32 ? 4 : 2; }

bool head_dim_supported(int dtype, int d) {
  if (dtype == ESA_DTYPE_F32) return d == 8 || d == 16 || d == 32 || d == 64 || d == 128;
  return d == 8 || d == 16 || d == 32 || d == 64 || d == 128 || d == 256;
}

int check_tensor(const char* name, const esa_tensor_t& t, int esize) {
  if (!t.data) return fail(ESA_ERR_INVALID, "%s: null data pointer", name);
  if (reinterpret_cast<uintptr_t>(t.data) % 16)
    return fail(ESA_ERR_INVALID, "%s: data pointer must be 16-byte aligned", name);
  if ((t.stride_b * esize) % 16 || (t.stride_h * esize) % 16 || (t.stride_s * esize) % 16)
    return fail(ESA_ERR_INVALID,
                "%s: strides (%lld, %lld, %lld) elements must be multiples of 16 bytes",
                name, (long long)t.stride_b, (long long)t.stride_h, (long long)t.stride_s);
  return ESA_OK;
}

int check_problem(const esa_problem_t* pb) {
  if (!pb) return fail(ESA_ERR_INVALID, "null problem");
  if (pb->dtype < 0 || pb->dtype > 2) return fail(ESA_ERR_INVALID, "unknown dtype %d", pb->dtype);
  if (pb->batch < 0 || pb->num_heads < 1 || pb->num_kv_heads < 1)
    return fail(ESA_ERR_INVALID, "batch/num_heads/num_kv_heads out of range");
  if (pb->num_heads % pb->num_kv_heads)
    return fail(ESA_ERR_INVALID, "num_heads (%d) must be divisible by num_kv_heads (%d)",
                pb->num_heads, pb->num_kv_heads);
  if (!head_dim_supported(pb->dtype, pb->head_dim))
    return fail(ESA_ERR_UNSUPPORTED, "head_dim %d not supported for dtype %d", pb->head_dim,
                pb->dtype);
  if (pb->attn_length < 1 || pb->attn_length > kMaxAttnLength)
    return fail(ESA_ERR_UNSUPPORTED, "attention_length %d outside [1, %d]", pb->attn_length,
                kMaxAttnLength);
  if (pb->num_hidden_layers < 1) return fail(ESA_ERR_INVALID, "num_hidden_layers must be >= 1");
  if (pb->q_len < 0 || pb->q_len >= kMaxPosition)
    return fail(ESA_ERR_INVALID, "q_len %lld out of range", (long long)pb->q_len);
  if (pb->q_len > 0 && pb->kv_len < 1) return fail(ESA_ERR_INVALID, "kv_len must be >= 1");
  if (pb->kv_len > kMaxPosition)
    return fail(ESA_ERR_UNSUPPORTED, "kv_len %lld above 2^24", (long long)pb->kv_len);
  if (pb->kv_offset < 0 || pb->kv_rows < 1 || pb->kv_offset + pb->kv_rows > kMaxPosition)
    return fail(ESA_ERR_INVALID, "kv_offset/kv_rows out of range");
  if (pb->row_offset < 0 || pb->row_offset + pb->q_len > kMaxPosition)
    return fail(ESA_ERR_INVALID, "row_offset out of range");
  if (!std::isfinite(pb->scale)) return fail(ESA_ERR_INVALID, "scale must be finite");
  if (!(pb->dropout_p >= 0.f && pb->dropout_p <= 1.f))
    return fail(ESA_ERR_INVALID, "dropout_p must be in [0, 1]");
  if (pb->weights && reinterpret_cast<uintptr_t>(pb->weights) % 4)
    return fail(ESA_ERR_INVALID, "weights must be 4-byte aligned");
  if (pb->probs && reinterpret_cast<uintptr_t>(pb->probs) % 16)
    return fail(ESA_ERR_INVALID, "probs must be 16-byte aligned");
  if (pb->head_offset < 0 || pb->pattern_heads < 0 ||
      (int64_t)pb->head_offset + pb->num_heads > pattern_heads(pb) || pattern_heads(pb) > 65535)
    return fail(ESA_ERR_INVALID,
                "head_offset %d + num_heads %d must be <= pattern_heads %d (<= 65535)",
                pb->head_offset, pb->num_heads, pattern_heads(pb));
  return ESA_OK;
}

esa::AttnParams base_params(const esa_problem_t* pb) {
  esa::AttnParams p{};
  p.B = pb->batch;
  p.Hq = pb->num_heads;
  p.Hkv = pb->num_kv_heads;
  p.G = pb->num_heads / pb->num_kv_heads;
  p.D = pb->head_dim;
  p.n_rows = (int)pb->q_len;
  p.kv_len = (int)pb->kv_len;
  p.kv_offset = (int)pb->kv_offset;
  p.kv_rows = (int)pb->kv_rows;
  p.row_offset = (int)pb->row_offset;
  p.rows = pb->rows;
  p.pat = make_pattern(pattern_heads(pb), pb->attn_length, pb->layer_idx, pb->num_hidden_layers,
                       pb->head_offset);
  p.scale = pb->scale;
  p.scale_log2 = pb->scale * esa::kLog2e;
  p.alpha_zero = pb->layer_idx == 0;   // alpha = layer_idx / max(nl - 1, 1) == 0
  p.flags = pb->flags;
  if (pb->dropout_p > 0.f) {
    const double t = (double)pb->dropout_p * 4294967296.0;
    p.drop_threshold = t >= 4294967295.0 ? 0xFFFFFFFFu : (uint32_t)t;
    p.keep_scale = pb->dropout_p < 1.f ? 1.f / (1.f - pb->dropout_p) : 0.f;
  }
  p.seed = pb->dropout_seed;
  p.weights = pb->weights;
  p.probs = static_cast<float*>(pb->probs);
  return p;
}

void set_tensor(const esa_tensor_t& t, const void*& ptr, int64_t& sb, int64_t& sh, int64_t& ss) {
  ptr = t.data; sb = t.stride_b; sh = t.stride_h; ss = t.stride_s;
}
void set_tensor_mut(const esa_tensor_t& t, void*& ptr, int64_t& sb, int64_t& sh, int64_t& ss) {
  ptr = t.data; sb = t.stride_b; sh = t.stride_h; ss = t.stride_s;
}

constexpr int kFwdWarps = 8;
constexpr int kKeyWarps = 8;
constexpr int kKeyRowsPerWarp = 16;

int rows_per_cta(int G) { return G >= 64 ? 1 : 64 / G; }

// Number of SMs of the current device (persistent kernels launch one CTA per SM).
int sm_count(int* out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(out, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess || *out < 1)
    return fail(ESA_ERR_CUDA, "cannot read the SM count: %s", cudaGetErrorString(e));
  return ESA_OK;
}

// Per-device addresses of a __device__ variable of this library, looked up
// once per device (cudaGetSymbolAddress with that device current) and cached.
constexpr int kMaxDevices = 64;
struct SymbolAddresses {
  std::mutex mu;
  void* addr[kMaxDevices] = {};
};

int symbol_address(const void* symbol, SymbolAddresses& cache, const char* what, void** out) {
  int dev = -1;
  const cudaError_t de = cudaGetDevice(&dev);
  if (de != cudaSuccess) return fail(ESA_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(de));
  if (dev < 0 || dev >= kMaxDevices)
    return fail(ESA_ERR_UNSUPPORTED, "%s: device ordinal %d above %d", what, dev, kMaxDevices - 1);
  std::lock_guard<std::mutex> lock(cache.mu);
  if (!cache.addr[dev]) {
    void* addr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&addr, symbol);
    if (e != cudaSuccess || !addr)
      return fail(ESA_ERR_CUDA, "%s: cudaGetSymbolAddress failed: %s", what, cudaGetErrorString(e));
    cache.addr[dev] = addr;
  }
  *out = cache.addr[dev];
  return ESA_OK;
}

// The error word the kernels of a call record ESA_DEVERR_* bits in (one per
// device; sticky until esa_device_errors resets it).
static __device__ int g_device_errors;

int device_error_word(int** out) {
  static SymbolAddresses cache;
  void* a = nullptr;
  if (int rc = symbol_address(&g_device_errors, cache, "device error word", &a)) return rc;
  *out = static_cast<int*>(a);
  return ESA_OK;
}

// Up to this many (batch, head, row) pairs the forward runs the latency kernel
// (one CTA per pair, slots split over warps) instead of a throughput kernel.
constexpr int64_t kDecodeMaxPairs = 4096;

template <typename K>
int prepare_smem(K kernel, size_t bytes) {
  if (bytes > 48 * 1024) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) !=
        cudaSuccess)
      return fail(ESA_ERR_CUDA, "cannot reserve %zu bytes of shared memory", bytes);
  }
  return ESA_OK;
}

// Dropout and the weights output are implemented in the per-pair gather kernels.
bool needs_gather(const esa::AttnParams& p) {
  return p.drop_threshold || p.weights || (p.flags & ESA_FLAG_GATHER_ONLY);
}

// ---- tensor-core sliding-window path (alpha == 0) -------------------------
PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// 4-D map {D, rows, heads, batch} of a 16-bit operand, box {64, box_rows, 1, 1},
// 128-byte swizzle, zero fill outside the tensor.
bool encode_map(CUtensorMap* m, const void* ptr, bool fp16, int64_t D, int64_t rows,
                int64_t heads, int64_t batch, int64_t s_row, int64_t s_head, int64_t s_batch,
                int box_rows) {
  auto enc = tmap_encoder();
  if (!enc) return false;
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)rows, (cuuint64_t)heads,
                              (cuuint64_t)batch};
  const cuuint64_t strides[3] = {(cuuint64_t)s_row * 2, (cuuint64_t)s_head * 2,
                                 (cuuint64_t)s_batch * 2};
  const cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(m, fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4,
             const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Heads per UMMA tile for the window path, 0 when the call is not eligible.
template <typename T, int D>
int window_heads_for_problem(const esa::AttnParams& p) {
  if (std::is_same<T, float>::value || D != esa::kWinHeadDim) return 0;
  if (!p.alpha_zero || needs_gather(p) || p.rows) return 0;
  const int ht = (p.G % 4 == 0) ? 4 : (p.G == 2 ? 2 : 0);
  if (!ht) return 0;
  const int qt = esa::kWinRows / ht;
  const int nk = (qt + p.pat.w - 1 + 15) / 16 * 16;
  if (nk > esa::kWinMaxKeys) return 0;
  const int64_t last = (int64_t)p.row_offset + p.n_rows;   // one past the last position
  if (last > p.kv_len || last > (int64_t(1) << 21)) return 0;
  if (p.kv_offset > std::max(0, p.row_offset - p.pat.w + 1) ||
      (int64_t)p.kv_offset + p.kv_rows < last)
    return 0;
  return ht;
}

// The window kernel also needs positive strides (tensor maps) and the driver's
// tensor-map encoder.
template <typename T, int D>
int window_heads(const esa::AttnParams& p, bool, int) {
  const int ht = window_heads_for_problem<T, D>(p);
  if (!ht) return 0;
  if (p.sqb <= 0 || p.sqh <= 0 || p.sqs <= 0 || p.skb <= 0 || p.skh <= 0 || p.sks <= 0 ||
      p.svb <= 0 || p.svh <= 0 || p.svs <= 0)
    return 0;
  return tmap_encoder() ? ht : 0;
}

// The slot-major tile forward / query-side backward apply (16-bit data,
// head_dim 64 or 128, w <= 64, G divides 128, consecutive positions, at least
// 256 rows, no dropout / weights output, more pairs than the latency kernel
// takes).  Only this forward writes `probs`.
template <typename T, int D>
bool tile_path(const esa::AttnParams& p) {
  if constexpr (std::is_same<T, float>::value || !(D == 64 || D == 128)) {
    return false;
  } else {
    return p.pat.w <= esa::kTileMaxW && p.G <= esa::kTilePairs && esa::kTilePairs % p.G == 0 &&
           !p.rows && p.n_rows >= 256 && p.kv_rows >= 1 && !needs_gather(p);
  }
}

// The tensor-core key side: 16-bit types, D = 64 / 128, contiguous query
// positions (no explicit rows), all G heads' columns in one warp's cursors.
template <typename T, int D>
bool key_mma_path(const esa::AttnParams& p) {
  if constexpr (std::is_same<T, float>::value || !(D == 64 || D == 128)) {
    return false;
  } else {
    using KM = esa::KeyMma<T, D>;
    constexpr int64_t per16 = 16 / sizeof(T);
    // q / dO rows are copied in 16-byte units addressed by 32-bit offsets
    auto rows_ok = [&](const void* base, int64_t srow, int64_t shead, int64_t sbatch) {
      if (reinterpret_cast<uintptr_t>(base) % 16 || srow % per16 || shead % per16 ||
          sbatch % per16 || srow < 0 || shead < 0)
        return false;
      const int64_t last = (int64_t)(p.G - 1) * shead + (int64_t)(p.n_rows - 1) * srow;
      return last / per16 < (int64_t(1) << 32);
    };
    return !p.rows && !p.sorted_rows && !p.row_perm && p.G <= KM::kMaxGroup &&
           p.G * p.pat.w <= KM::kMaxCols && p.kv_rows >= 1 && p.n_rows >= 1 &&
           !(p.flags & ESA_FLAG_GATHER_ONLY) && rows_ok(p.q, p.sqs, p.sqh, p.sqb) &&
           rows_ok(p.dout, p.sdos, p.sdoh, p.sdob);
  }
}

bool decode_path(const esa::AttnParams& p) {
  return (int64_t)p.B * p.Hq * p.n_rows <= kDecodeMaxPairs && !needs_gather(p);
}

template <typename T, int HT>
int launch_window(const esa::AttnParams& p, cudaStream_t s) {
  constexpr int QT = esa::kWinRows / HT;
  const int nk = (QT + p.pat.w - 1 + 15) / 16 * 16;
  const bool fp16 = std::is_same<T, __half>::value;
  esa::WindowTmaps maps;
  if (!encode_map(&maps.q, p.q, fp16, p.D, p.n_rows, p.Hq, p.B, p.sqs, p.sqh, p.sqb, QT) ||
      !encode_map(&maps.k, p.k, fp16, p.D, p.kv_rows, p.Hkv, p.B, p.sks, p.skh, p.skb, nk) ||
      !encode_map(&maps.v, p.v, fp16, p.D, p.kv_rows, p.Hkv, p.B, p.svs, p.svh, p.svb, nk))
    return fail(ESA_ERR_CUDA, "cuTensorMapEncodeTiled failed for the window path");
  auto kern = esa::window_fwd_tc_kernel<T, HT>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           esa::kWinSmemBytes) != cudaSuccess)
    return fail(ESA_ERR_CUDA, "cannot reserve shared memory for the window path");
  // persistent: one CTA per SM walks the (query tile, head group, batch) tiles
  const int64_t tiles = (int64_t)((p.n_rows + QT - 1) / QT) * (p.Hkv * (p.G / HT)) * p.B;
  if (tiles > INT32_MAX) return fail(ESA_ERR_UNSUPPORTED, "window path: too many tiles");
  int sms = 0;
  if (int rc = sm_count(&sms)) return rc;
  const int grid = (int)std::min<int64_t>(tiles, sms);
  LaunchTrace tr("window_fwd_tc", s);
  kern<<<grid, esa::kWinThreads, esa::kWinSmemBytes, s>>>(maps, p, nk, (int)tiles);
  return check_launch("forward (tensor-core window)");
}

// Tensor-core backward of a sliding-window layer: dQ (query-major, also the
// row values delta = rowsum(dO o O), kept in the workspace) then dK / dV
// (key-major, all heads of a group in one CTA).
template <typename T, int HT>
int launch_window_bwd(const esa::AttnParams& p, cudaStream_t s) {
  constexpr int QT = esa::kWinRows / HT;
  const int nk = (QT + p.pat.w - 1 + 15) / 16 * 16;
  const bool fp16 = std::is_same<T, __half>::value;
  float* delta = reinterpret_cast<float*>(p.pds);   // [B, Hq, n_rows] in the workspace
  esa::WindowBwdTmaps a, b;
  if (!encode_map(&a.q, p.q, fp16, p.D, p.n_rows, p.Hq, p.B, p.sqs, p.sqh, p.sqb, QT) ||
      !encode_map(&a.dout, p.dout, fp16, p.D, p.n_rows, p.Hq, p.B, p.sdos, p.sdoh, p.sdob, QT) ||
      !encode_map(&a.k, p.k, fp16, p.D, p.kv_rows, p.Hkv, p.B, p.sks, p.skh, p.skb, nk) ||
      !encode_map(&a.v, p.v, fp16, p.D, p.kv_rows, p.Hkv, p.B, p.svs, p.svh, p.svb, nk) ||
      !encode_map(&b.q, p.q, fp16, p.D, p.n_rows, p.Hq, p.B, p.sqs, p.sqh, p.sqb, esa::kWbkQC) ||
      !encode_map(&b.dout, p.dout, fp16, p.D, p.n_rows, p.Hq, p.B, p.sdos, p.sdoh, p.sdob,
                  esa::kWbkQC) ||
      !encode_map(&b.k, p.k, fp16, p.D, p.kv_rows, p.Hkv, p.B, p.sks, p.skh, p.skb, esa::kWbkKeys) ||
      !encode_map(&b.v, p.v, fp16, p.D, p.kv_rows, p.Hkv, p.B, p.svs, p.svh, p.svb, esa::kWbkKeys))
    return fail(ESA_ERR_CUDA, "cuTensorMapEncodeTiled failed for the window backward");
  auto kq = esa::window_bwd_dq_tc_kernel<T, HT>;
  auto kkv = esa::window_bwd_dkv_tc_kernel<T>;
  if (cudaFuncSetAttribute(kq, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           esa::kWbqSmemBytes) != cudaSuccess ||
      cudaFuncSetAttribute(kkv, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           esa::kWbkSmemBytes) != cudaSuccess)
    return fail(ESA_ERR_CUDA, "cannot reserve shared memory for the window backward");
  // dQ: persistent, one CTA per SM over the (query tile, head group, batch) tiles
  const int64_t tiles = (int64_t)((p.n_rows + QT - 1) / QT) * (p.Hkv * (p.G / HT)) * p.B;
  if (tiles > INT32_MAX) return fail(ESA_ERR_UNSUPPORTED, "window backward: too many tiles");
  int sms = 0;
  if (int rc = sm_count(&sms)) return rc;
  const int gq = (int)std::min<int64_t>(tiles, sms);
  {
    LaunchTrace tr("window_bwd_dq_tc", s);
    kq<<<gq, esa::kWbqThreads, esa::kWbqSmemBytes, s>>>(a, p, nk, (int)tiles, delta);
  }
  if (int rc = check_launch("backward (tensor-core window, dQ)")) return rc;
  dim3 gk((p.kv_rows + esa::kWbkKeys - 1) / esa::kWbkKeys, p.Hkv, p.B);
  {
    LaunchTrace tr("window_bwd_dkv_tc", s);
    kkv<<<gk, esa::kWinBwdThreads, esa::kWbkSmemBytes, s>>>(b, p, delta);
  }
  return check_launch("backward (tensor-core window, dK dV)");
}

// Whether esa_forward for this call runs the tile kernel, the only one that
// writes `probs` (and so whether the backward may read them).
template <typename T, int D>
bool forward_writes_probs(const esa::AttnParams& p) {
  if (window_heads<T, D>(p, p.alpha_zero, p.flags)) return false;
  if (decode_path(p)) return false;
  return tile_path<T, D>(p);
}

template <typename T, int D>
int launch_forward(const esa::AttnParams& p, cudaStream_t s) {
  if constexpr (!std::is_same<T, float>::value && D == esa::kWinHeadDim) {
    const int ht = window_heads<T, D>(p, p.alpha_zero, p.flags);
    if (ht == 4) return launch_window<T, 4>(p, s);
    if (ht == 2) return launch_window<T, 2>(p, s);
  }
  if (decode_path(p)) {
    const int nw = std::min((p.pat.w + 31) >> 5, esa::kDecodeMaxWarps);
    LaunchTrace tr("fwd_decode", s);
    esa::fwd_decode_kernel<T, D><<<dim3(p.n_rows, p.Hq, p.B), nw * 32, 0, s>>>(p);
    return check_launch("forward (decode)");
  }
  if constexpr (!std::is_same<T, float>::value && (D == 64 || D == 128)) {
    // slot-major tile kernel: 128 pairs per CTA share their K/V rows through L1
    if (tile_path<T, D>(p)) {
      const int tq = esa::kTilePairs / p.G;
      dim3 grid((p.n_rows + tq - 1) / tq, p.Hkv, p.B);
      auto kern = esa::fwd_tile_kernel<T, D>;
      if (int rc = prepare_smem(kern, esa::kTileSmemBytes)) return rc;
      LaunchTrace tr("fwd_tile", s);
      kern<<<grid, 256, esa::kTileSmemBytes, s>>>(p);
      return check_launch("forward (tile)");
    }
  }
  const int rpc = rows_per_cta(p.G);
  const int wpad = (p.pat.w + 31) & ~31;
  const size_t smem = (size_t)kFwdWarps * 3 * wpad * sizeof(int);
  auto kern = esa::fwd_gather_kernel<T, D, kFwdWarps>;
  if (int rc = prepare_smem(kern, smem)) return rc;
  dim3 grid((p.n_rows + rpc - 1) / rpc, p.Hkv, p.B);
  LaunchTrace tr("fwd_gather", s);
  kern<<<grid, kFwdWarps * 32, smem, s>>>(p, rpc);
  return check_launch("forward");
}

template <typename T, int D>
int launch_backward(const esa::AttnParams& p_in, cudaStream_t s) {
  // probabilities from the forward only where that forward wrote them
  esa::AttnParams p = p_in;
  if (p.probs && !forward_writes_probs<T, D>(p)) p.probs = nullptr;
  if constexpr (!std::is_same<T, float>::value && D == esa::kWinHeadDim) {
    if (p.n_rows > 0 && !(p.flags & ESA_FLAG_GATHER_ONLY) && p.sdob > 0 && p.sdoh > 0 &&
        p.sdos > 0) {
      // the tensor-core backward takes up to kWbqMaxKeys keys per tile
      const int ht = window_heads<T, D>(p, p.alpha_zero, p.flags);
      const int nk = ht ? (esa::kWinRows / ht + p.pat.w - 1 + 15) / 16 * 16 : 0;
      if (ht == 4 && nk <= esa::kWbqMaxKeys) return launch_window_bwd<T, 4>(p, s);
      if (ht == 2 && nk <= esa::kWbqMaxKeys) return launch_window_bwd<T, 2>(p, s);
    }
  }
  bool query_done = false;
  if constexpr (!std::is_same<T, float>::value && (D == 64 || D == 128)) {
    if (p.n_rows > 0 && tile_path<T, D>(p)) {
      const int tq = esa::kTilePairs / p.G;
      dim3 grid((p.n_rows + tq - 1) / tq, p.Hkv, p.B);
      auto kern = esa::bwd_query_tile_kernel<T, D>;
      if (int rc = prepare_smem(kern, esa::kTileBwdSmemBytes)) return rc;
      {
        LaunchTrace tr("bwd_query_tile", s);
        kern<<<grid, 256, esa::kTileBwdSmemBytes, s>>>(p);
      }
      if (int rc = check_launch("backward (query side, tile)")) return rc;
      query_done = true;
    }
  }
  if (p.n_rows > 0 && !query_done) {
    const int rpc = rows_per_cta(p.G);
    const int wpad = (p.pat.w + 31) & ~31;
    const size_t smem = (size_t)kFwdWarps * 3 * wpad * sizeof(int);
    auto kern = esa::bwd_query_kernel<T, D, kFwdWarps>;
    if (int rc = prepare_smem(kern, smem)) return rc;
    dim3 grid((p.n_rows + rpc - 1) / rpc, p.Hkv, p.B);
    {
      LaunchTrace tr("bwd_query", s);
      kern<<<grid, kFwdWarps * 32, smem, s>>>(p, rpc);
    }
    if (int rc = check_launch("backward (query side)")) return rc;
  }
  if (p.heavy_chunks > 0) {
    // partial sums of query chunks that all use one key (long runs)
    {
      LaunchTrace tr("bwd_heavy", s);
      esa::bwd_heavy_kernel<T, D><<<dim3(p.heavy_chunks, p.Hq, p.B), 256, 0, s>>>(p);
    }
    if (int rc = check_launch("backward (key side, long runs)")) return rc;
  }
  if constexpr (!std::is_same<T, float>::value && (D == 64 || D == 128)) {
    if (key_mma_path<T, D>(p)) {
      using KM = esa::KeyMma<T, D>;
      // kHeadsPerLaunch query heads of each group per launch: a launch's
      // working set (q / dO rows and the (p, dS) workspace of its heads)
      // stays within a few L2 sizes; the launches add up in the fp32
      // workspace, the last writes dK / dV
      const int gs = p.acc ? KM::kHeadsPerLaunch : p.G;
      const size_t smem = KM::smem_bytes(gs * p.pat.w);
      // with a key plan (built for this problem with the same launch split)
      // the tiles read their user records instead of searching the columns
      const bool planned = p.plan_header && p.plan_nlaunch == (p.G + gs - 1) / gs;
      auto kern = planned ? esa::bwd_key_mma_kernel<T, D, true> : esa::bwd_key_mma_kernel<T, D, false>;
      if (int rc = prepare_smem(kern, smem)) return rc;
      const int tile = KM::kWarps * KM::kTiles * KM::kKeys;
      dim3 grid((p.kv_rows + tile - 1) / tile, p.Hkv, p.B);
      for (int h0 = 0; h0 < p.G; h0 += gs) {
        esa::AttnParams pk = p;
        pk.head_in_group = h0;
        pk.key_heads = std::min(gs, p.G - h0);
        {
          LaunchTrace tr(planned ? "bwd_key_plan" : "bwd_key_mma", s);
          kern<<<grid, KM::kWarps * 32, smem, s>>>(pk);
        }
        if (int rc = check_launch("backward (key side, tensor cores)")) return rc;
      }
      return ESA_OK;
    }
  }
  {
    const int ncol = (p.pat.w + 31) >> 5;
    const size_t smem = (size_t)kKeyWarps * (esa::KeyStage<T, D>::kWarpBytes + ncol * 64 * sizeof(int));
    auto kern = esa::bwd_key_kernel<T, D, kKeyWarps, kKeyRowsPerWarp>;
    if (int rc = prepare_smem(kern, smem)) return rc;
    const int tile = kKeyWarps * kKeyRowsPerWarp;
    dim3 grid((p.kv_rows + tile - 1) / tile, p.Hkv, p.B);
    for (int gi = 0; gi < p.G; ++gi) {
      esa::AttnParams pk = p;
      pk.head_in_group = gi;
      {
        LaunchTrace tr("bwd_key", s);
        kern<<<grid, kKeyWarps * 32, smem, s>>>(pk);
      }
      if (int rc = check_launch("backward (key side)")) return rc;
    }
  }
  return ESA_OK;
}

struct ProbsQuery {
  template <typename T, int D>
  static int run(const esa::AttnParams& p, cudaStream_t) {
    if (window_heads_for_problem<T, D>(p)) return 0;
    if (decode_path(p)) return 0;
    return tile_path<T, D>(p) ? 1 : 0;
  }
};
struct FwdOp {
  template <typename T, int D>
  static int run(const esa::AttnParams& p, cudaStream_t s) { return launch_forward<T, D>(p, s); }
};
struct BwdOp {
  template <typename T, int D>
  static int run(const esa::AttnParams& p, cudaStream_t s) { return launch_backward<T, D>(p, s); }
};

template <typename Op>
int dispatch_op(int dtype, int d, const esa::AttnParams& p, cudaStream_t s) {
  switch (dtype) {
    case ESA_DTYPE_F32:
      switch (d) {
        case 8: return Op::template run<float, 8>(p, s);
        case 16: return Op::template run<float, 16>(p, s);
        case 32: return Op::template run<float, 32>(p, s);
        case 64: return Op::template run<float, 64>(p, s);
        case 128: return Op::template run<float, 128>(p, s);
      }
      break;
    case ESA_DTYPE_BF16:
      switch (d) {
        case 8: return Op::template run<__nv_bfloat16, 8>(p, s);
        case 16: return Op::template run<__nv_bfloat16, 16>(p, s);
        case 32: return Op::template run<__nv_bfloat16, 32>(p, s);
        case 64: return Op::template run<__nv_bfloat16, 64>(p, s);
        case 128: return Op::template run<__nv_bfloat16, 128>(p, s);
        case 256: return Op::template run<__nv_bfloat16, 256>(p, s);
      }
      break;
    case ESA_DTYPE_F16:
      switch (d) {
        case 8: return Op::template run<__half, 8>(p, s);
        case 16: return Op::template run<__half, 16>(p, s);
        case 32: return Op::template run<__half, 32>(p, s);
        case 64: return Op::template run<__half, 64>(p, s);
        case 128: return Op::template run<__half, 128>(p, s);
        case 256: return Op::template run<__half, 256>(p, s);
      }
      break;
  }
  return fail(ESA_ERR_UNSUPPORTED, "dtype %d with head_dim %d not built", dtype, d);
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

size_t pds_bytes(const esa_problem_t* pb) {
  return align256((size_t)pb->batch * pb->num_heads * pb->attn_length * pb->q_len * sizeof(float2));
}
size_t heavy_bytes(const esa_problem_t* pb) {
  const int64_t chunks = pb->q_len / esa::kHeavyChunk;
  return align256((size_t)pb->batch * pb->num_heads * pb->attn_length * chunks * 2 *
                  pb->head_dim * sizeof(float));
}

size_t acc_bytes(const esa_problem_t* pb) {
  if (pb->num_heads == pb->num_kv_heads) return 0;
  return align256((size_t)2 * pb->batch * pb->num_kv_heads * pb->kv_rows * pb->head_dim *
                  sizeof(float));
}

// Key plan geometry (esa_keyplan.cuh) of a problem.
struct PlanGeom {
  int gs = 0, nlaunch = 0, ntiles = 0;
  int64_t seg_users = 0, seg_heavy = 0;
  size_t off_ustart = 0, off_hstart = 0, off_users = 0, off_heavy = 0, total = 0;
};

// Query heads per key-side launch when the backward of this problem runs the
// tensor-core key side and a plan can describe it (as far as the problem
// alone decides: tensor strides are checked at the call), else 0.
struct PlanQuery {
  template <typename T, int D>
  static int run(const esa::AttnParams& p, cudaStream_t) {
    if constexpr (std::is_same<T, float>::value || !(D == 64 || D == 128)) {
      return 0;
    } else {
      using KM = esa::KeyMma<T, D>;
      if (const int ht = window_heads_for_problem<T, D>(p)) {
        const int nk = (esa::kWinRows / ht + p.pat.w - 1 + 15) / 16 * 16;
        if (!(p.flags & ESA_FLAG_GATHER_ONLY) && nk <= esa::kWbqMaxKeys) return 0;
      }
      const int gs = p.G > 1 ? KM::kHeadsPerLaunch : 1;
      const bool ok = !p.rows && p.G <= KM::kMaxGroup && p.G * p.pat.w <= KM::kMaxCols &&
                      gs * p.pat.w <= esa::kPlanMaxCols && p.n_rows >= 1 &&
                      p.n_rows <= (1 << esa::kPlanSlotBits) && p.kv_rows >= 1 &&
                      !(p.flags & ESA_FLAG_GATHER_ONLY);
      return ok ? gs : 0;
    }
  }
};

PlanGeom plan_geom(const esa_problem_t* pb, const esa::AttnParams& p) {
  PlanGeom g;
  g.gs = dispatch_op<PlanQuery>(pb->dtype, pb->head_dim, p, nullptr);
  if (g.gs <= 0) {
    g.gs = 0;
    return g;
  }
  g.nlaunch = (p.G + g.gs - 1) / g.gs;
  g.ntiles = (p.kv_rows + esa::kKeyPlanKeys - 1) / esa::kKeyPlanKeys;
  const int64_t segs = (int64_t)p.Hkv * g.nlaunch;
  g.seg_users = (int64_t)g.gs * p.pat.w * p.n_rows;
  g.seg_heavy = (int64_t)g.gs * p.pat.w * (p.n_rows / esa::kHeavyChunk);
  size_t off = align256(esa::kKeyPlanHeaderWords * sizeof(uint64_t));
  g.off_ustart = off;
  off += align256((size_t)segs * (g.ntiles + 1) * sizeof(int));
  g.off_hstart = off;
  off += align256((size_t)segs * (g.ntiles + 1) * sizeof(int));
  g.off_users = off;
  off += align256((size_t)segs * g.seg_users * sizeof(uint32_t));
  g.off_heavy = off;
  off += align256((size_t)segs * g.seg_heavy * sizeof(uint32_t));
  g.total = off;
  return g;
}

// FNV-1a over everything the plan depends on.
uint64_t plan_fingerprint(const esa::AttnParams& p, const PlanGeom& g) {
  uint64_t h = 0xcbf29ce484222325ull;
  auto mix = [&](uint64_t v) {
    for (int i = 0; i < 8; ++i) {
      h ^= (v >> (8 * i)) & 0xff;
      h *= 0x100000001b3ull;
    }
  };
  uint32_t a, c;
  std::memcpy(&a, &p.pat.a, 4);
  std::memcpy(&c, &p.pat.c, 4);
  const int64_t f[] = {p.pat.w, p.pat.num_heads, a, c, p.pat.head_offset, p.Hq, p.Hkv,
                       p.n_rows, p.row_offset, p.kv_len, p.kv_offset, p.kv_rows,
                       p.n_rows / esa::kHeavyChunk, g.gs, esa::kKeyPlanKeys};
  for (int64_t v : f) mix((uint64_t)v);
  return h;
}

void set_plan(esa::AttnParams& p, const void* plan, const PlanGeom& g) {
  const unsigned char* b = static_cast<const unsigned char*>(plan);
  p.plan_header = reinterpret_cast<const uint64_t*>(b);
  p.plan_fp = plan_fingerprint(p, g);
  p.plan_ustart = reinterpret_cast<const int*>(b + g.off_ustart);
  p.plan_hstart = reinterpret_cast<const int*>(b + g.off_hstart);
  p.plan_users = reinterpret_cast<const uint32_t*>(b + g.off_users);
  p.plan_heavy = reinterpret_cast<const uint32_t*>(b + g.off_heavy);
  p.plan_seg_users = g.seg_users;
  p.plan_seg_heavy = g.seg_heavy;
  p.plan_ntiles = g.ntiles;
  p.plan_nlaunch = g.nlaunch;
  p.plan_gs = g.gs;
}

}  // namespace

extern "C" {

int esa_version(void) { return 130; }

const char* esa_last_error(void) { return g_last_error.c_str(); }

int esa_pattern(int32_t num_heads, int32_t attn_length, int32_t layer_idx,
                int32_t num_hidden_layers, int64_t n_rows, const int64_t* rows,
                int64_t row_offset, int64_t clamp_len, int64_t* idx, int64_t* mask,
                void* stream) {
  if (num_heads < 1 || attn_length < 1 || attn_length > kMaxAttnLength || num_hidden_layers < 1)
    return fail(ESA_ERR_INVALID, "esa_pattern: bad pattern arguments");
  if (n_rows < 0 || row_offset < 0 || row_offset + n_rows > kMaxPosition ||
      clamp_len > kMaxPosition)
    return fail(ESA_ERR_INVALID, "esa_pattern: rows out of range (positions must be < 2^24)");
  if (n_rows == 0) return ESA_OK;
  if (!idx || !mask) return fail(ESA_ERR_INVALID, "esa_pattern: null output");
  const esa::Pattern P = make_pattern(num_heads, attn_length, layer_idx, num_hidden_layers);
  const int64_t total = (int64_t)num_heads * n_rows * attn_length;
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((total + threads - 1) / threads, 148 * 64);
  LaunchTrace tr("pattern", (cudaStream_t)stream);
  esa::pattern_kernel<<<(unsigned)blocks, threads, 0, (cudaStream_t)stream>>>(
      P, (int)n_rows, rows, (int)row_offset, (int)(clamp_len > 0 ? clamp_len : 0), idx, mask);
  return check_launch("esa_pattern");
}

int esa_pattern_audit(int32_t num_heads, int32_t attn_length, int32_t layer_idx,
                      int32_t num_hidden_layers, int64_t seq_len, unsigned long long* d_count,
                      void* stream) {
  if (num_heads < 1 || attn_length < 1 || attn_length > kMaxAttnLength || num_hidden_layers < 1 ||
      seq_len < 0 || seq_len > kMaxPosition || !d_count)
    return fail(ESA_ERR_INVALID, "esa_pattern_audit: bad arguments");
  if (seq_len < 2) return ESA_OK;
  const esa::Pattern P = make_pattern(num_heads, attn_length, layer_idx, num_hidden_layers);
  const int64_t total = (int64_t)num_heads * seq_len * attn_length;
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((total + threads - 1) / threads, 148 * 32);
  LaunchTrace tr("pattern_audit", (cudaStream_t)stream);
  esa::audit_kernel<<<(unsigned)blocks, threads, 0, (cudaStream_t)stream>>>(P, (int)seq_len,
                                                                            d_count);
  return check_launch("esa_pattern_audit");
}

int esa_forward_writes_probs(const esa_problem_t* pb) {
  if (int rc = check_problem(pb)) return rc;
  if (pb->q_len == 0 || pb->batch == 0) return 0;
  const esa::AttnParams p = base_params(pb);
  return dispatch_op<ProbsQuery>(pb->dtype, pb->head_dim, p, nullptr);
}

int esa_device_errors(int32_t clear, int32_t* flags, void* stream) {
  if (!flags) return fail(ESA_ERR_INVALID, "esa_device_errors: null flags pointer");
  int* word = nullptr;
  if (int rc = device_error_word(&word)) return rc;
  int32_t host = 0;
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemcpyAsync(&host, word, sizeof(int32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess && clear) e = cudaMemsetAsync(word, 0, sizeof(int32_t), s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return fail(ESA_ERR_CUDA, "esa_device_errors: %s", cudaGetErrorString(e));
  *flags = host;
  return ESA_OK;
}

int esa_forward(const esa_problem_t* pb, esa_tensor_t q, esa_tensor_t k, esa_tensor_t v,
                esa_tensor_t o, float* lse, void* stream) {
  if (int rc = check_problem(pb)) return rc;
  if (pb->q_len == 0 || pb->batch == 0) return ESA_OK;
  const int es = elem_size(pb->dtype);
  if (int rc = check_tensor("q", q, es)) return rc;
  if (int rc = check_tensor("k", k, es)) return rc;
  if (int rc = check_tensor("v", v, es)) return rc;
  if (int rc = check_tensor("o", o, es)) return rc;
  if (!lse) return fail(ESA_ERR_INVALID, "lse: null pointer");
  esa::AttnParams p = base_params(pb);
  if (int rc = device_error_word(&p.err)) return rc;
  set_tensor(q, p.q, p.sqb, p.sqh, p.sqs);
  set_tensor(k, p.k, p.skb, p.skh, p.sks);
  set_tensor(v, p.v, p.svb, p.svh, p.svs);
  set_tensor_mut(o, p.o, p.sob, p.soh, p.sos);
  p.lse = lse;
  return dispatch_op<FwdOp>(pb->dtype, pb->head_dim, p, (cudaStream_t)stream);
}

size_t esa_key_plan_size(const esa_problem_t* pb) {
  if (check_problem(pb) || pb->q_len == 0) return 0;
  return plan_geom(pb, base_params(pb)).total;
}

int esa_key_plan_build(const esa_problem_t* pb, void* plan, size_t plan_bytes, void* stream) {
  if (int rc = check_problem(pb)) return rc;
  esa::AttnParams p = base_params(pb);
  // the chunks the backward sums separately (bwd_heavy_kernel) are left out
  // of the user lists, exactly as the backward's own key side leaves them
  p.heavy_chunks = (int)(pb->q_len / esa::kHeavyChunk);
  const PlanGeom g = pb->q_len > 0 ? plan_geom(pb, p) : PlanGeom{};
  if (!g.total)
    return fail(ESA_ERR_UNSUPPORTED, "esa_key_plan_build: this problem takes no key plan");
  if (!plan || plan_bytes < g.total)
    return fail(ESA_ERR_INVALID, "esa_key_plan_build: %zu bytes given, %zu needed", plan_bytes,
                g.total);
  if (reinterpret_cast<uintptr_t>(plan) % 256)
    return fail(ESA_ERR_INVALID, "esa_key_plan_build: plan must be 256-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  unsigned char* b = static_cast<unsigned char*>(plan);
  esa::KeyPlanBuild kb;
  kb.gs = g.gs;
  kb.nlaunch = g.nlaunch;
  kb.ntiles = g.ntiles;
  kb.seg_users = g.seg_users;
  kb.seg_heavy = g.seg_heavy;
  kb.ustart = reinterpret_cast<int*>(b + g.off_ustart);
  kb.hstart = reinterpret_cast<int*>(b + g.off_hstart);
  kb.users = reinterpret_cast<uint32_t*>(b + g.off_users);
  kb.heavy = reinterpret_cast<uint32_t*>(b + g.off_heavy);
  const int per_cta = esa::kKeyPlanWarps * esa::kKeyPlanTiles * esa::kKeyPlanKeys;
  const dim3 grid((p.kv_rows + per_cta - 1) / per_cta, p.Hkv, g.nlaunch);
  const size_t smem = (size_t)esa::kKeyPlanWarps * 2 * g.gs * p.pat.w * sizeof(int);
  LaunchTrace tr("key_plan", s);
  esa::key_plan_header_kernel<<<1, 32, 0, s>>>(reinterpret_cast<uint64_t*>(b),
                                               plan_fingerprint(p, g));
  esa::key_plan_kernel<false><<<grid, esa::kKeyPlanWarps * 32, smem, s>>>(p, kb);
  esa::key_plan_scan_kernel<<<dim3((unsigned)(p.Hkv * g.nlaunch), 2), 1024, 0, s>>>(kb);
  esa::key_plan_kernel<true><<<grid, esa::kKeyPlanWarps * 32, smem, s>>>(p, kb);
  return check_launch("esa_key_plan_build");
}

size_t esa_backward_workspace_size(const esa_problem_t* pb) {

  if (!pb || pb->batch < 0 || pb->q_len < 0 || pb->attn_length < 0) return 0;
  return pds_bytes(pb) + acc_bytes(pb) + heavy_bytes(pb);
}

int esa_backward(const esa_problem_t* pb, esa_tensor_t q, esa_tensor_t k, esa_tensor_t v,
                 esa_tensor_t o, const float* lse, esa_tensor_t dout, esa_tensor_t dq,
                 esa_tensor_t dk, esa_tensor_t dv, const int64_t* sorted_rows,
                 const int64_t* row_perm, void* workspace, size_t workspace_bytes,
                 void* stream) {
  if (int rc = check_problem(pb)) return rc;
  if (pb->batch == 0) return ESA_OK;
  const int es = elem_size(pb->dtype);
  static_assert(ESA_FLAG_F32_DKV == esa::kFlagF32Dkv, "flag values");
  const int es_dkv = (pb->flags & ESA_FLAG_F32_DKV) ? 4 : es;
  if (int rc = check_tensor("k", k, es)) return rc;
  if (int rc = check_tensor("v", v, es)) return rc;
  if (int rc = check_tensor("dk", dk, es_dkv)) return rc;
  if (int rc = check_tensor("dv", dv, es_dkv)) return rc;
  if (pb->q_len > 0) {
    if (int rc = check_tensor("q", q, es)) return rc;
    if (int rc = check_tensor("o", o, es)) return rc;
    if (int rc = check_tensor("dout", dout, es)) return rc;
    if (int rc = check_tensor("dq", dq, es)) return rc;
    if (!lse) return fail(ESA_ERR_INVALID, "lse: null pointer");
  }
  if ((sorted_rows == nullptr) != (row_perm == nullptr))
    return fail(ESA_ERR_INVALID, "sorted_rows and row_perm must be given together");
  const size_t need = esa_backward_workspace_size(pb);
  if (workspace_bytes < need || (need && !workspace))
    return fail(ESA_ERR_WORKSPACE, "workspace of %zu bytes given, %zu needed", workspace_bytes,
                need);
  if (reinterpret_cast<uintptr_t>(workspace) % 256)
    return fail(ESA_ERR_INVALID, "workspace must be 256-byte aligned");
  esa::AttnParams p = base_params(pb);
  if (pb->key_plan && pb->q_len > 0) {
    const PlanGeom g = plan_geom(pb, p);
    if (!g.total || pb->key_plan_bytes != g.total)
      return fail(ESA_ERR_INVALID, "key_plan of %llu bytes given, this problem's plan has %zu",
                  (unsigned long long)pb->key_plan_bytes, g.total);
    if (reinterpret_cast<uintptr_t>(pb->key_plan) % 256)
      return fail(ESA_ERR_INVALID, "key_plan must be 256-byte aligned");
    set_plan(p, pb->key_plan, g);
  }
  if (int rc = device_error_word(&p.err)) return rc;
  set_tensor(q, p.q, p.sqb, p.sqh, p.sqs);
  set_tensor(k, p.k, p.skb, p.skh, p.sks);
  set_tensor(v, p.v, p.svb, p.svh, p.svs);
  set_tensor_mut(o, p.o, p.sob, p.soh, p.sos);
  set_tensor(dout, p.dout, p.sdob, p.sdoh, p.sdos);
  set_tensor_mut(dq, p.dq, p.sdqb, p.sdqh, p.sdqs);
  set_tensor_mut(dk, p.dk, p.sdkb, p.sdkh, p.sdks);
  set_tensor_mut(dv, p.dv, p.sdvb, p.sdvh, p.sdvs);
  p.lse = const_cast<float*>(lse);
  p.sorted_rows = sorted_rows;
  p.row_perm = row_perm;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  p.pds = reinterpret_cast<float2*>(ws);
  p.acc = acc_bytes(pb) ? reinterpret_cast<float*>(ws + pds_bytes(pb)) : nullptr;
  p.heavy_chunks = (int)(pb->q_len / esa::kHeavyChunk);
  p.heavy = p.heavy_chunks ? reinterpret_cast<float*>(ws + pds_bytes(pb) + acc_bytes(pb)) : nullptr;
  return dispatch_op<BwdOp>(pb->dtype, pb->head_dim, p, (cudaStream_t)stream);
}

int esa_trace_enable(int32_t on) {
  if (on) {
    trace_clear();
    g_trace_on.store(true);
  } else {
    g_trace_on.store(false);
  }
  return ESA_OK;
}

int esa_trace_count(void) {
  std::lock_guard<std::mutex> lock(g_trace_mu);
  return (int)g_trace.size();
}

int esa_trace_read(int32_t i, const char** name, float* ms) {
  TraceRec r;
  {
    std::lock_guard<std::mutex> lock(g_trace_mu);
    if (i < 0 || i >= (int32_t)g_trace.size()) return fail(ESA_ERR_INVALID, "esa_trace_read: no record %d", i);
    r = g_trace[i];
  }
  if (name) *name = r.name;
  if (ms) {
    cudaError_t e = cudaEventSynchronize(r.b);
    if (e == cudaSuccess) e = cudaEventElapsedTime(ms, r.a, r.b);
    if (e != cudaSuccess) return fail(ESA_ERR_CUDA, "esa_trace_read: %s", cudaGetErrorString(e));
  }
  return ESA_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// esa_probe_gather: the tile forward's row loads alone (esa_probe.cuh).
// ---------------------------------------------------------------------------
namespace {

struct ProbeOp {
  template <typename T, int D>
  static int run(const esa::AttnParams& p, cudaStream_t s, int mode, uint32_t* sink) {
    if constexpr (std::is_same<T, float>::value || !(D == 64 || D == 128)) {
      return fail(ESA_ERR_UNSUPPORTED, "esa_probe_gather: 16-bit data with head_dim 64 or 128 only");
    } else {
      if (!tile_path<T, D>(p))
        return fail(ESA_ERR_UNSUPPORTED, "esa_probe_gather: the problem is not a tile-kernel problem");
      if (mode == esa::kProbeL1Window && p.kv_rows < esa::kProbeWindowRows)
        return fail(ESA_ERR_INVALID, "esa_probe_gather: the L1 window needs %d kv rows",
                    esa::kProbeWindowRows);
      const int tq = esa::kTilePairs / p.G;
      dim3 grid((p.n_rows + tq - 1) / tq, p.Hkv, p.B);
      auto kern = mode == esa::kProbePattern    ? esa::gather_probe_kernel<T, D, esa::kProbePattern>
                  : mode == esa::kProbeL2Random ? esa::gather_probe_kernel<T, D, esa::kProbeL2Random>
                  : mode == esa::kProbeL1Window ? esa::gather_probe_kernel<T, D, esa::kProbeL1Window>
                                                : esa::gather_probe_kernel<T, D, esa::kProbeL2Stream>;
      if (int rc = prepare_smem(kern, esa::kTileSmemBytes)) return rc;
      LaunchTrace tr("gather_probe", s);
      kern<<<grid, 256, esa::kTileSmemBytes, s>>>(p, sink);
      return check_launch("esa_probe_gather");
    }
  }
};

}  // namespace

extern "C" int esa_probe_gather(int32_t mode, const esa_problem_t* pb, esa_tensor_t k,
                                esa_tensor_t v, uint32_t* sink, void* stream) {
  if (int rc = check_problem(pb)) return rc;
  if (mode < ESA_PROBE_PATTERN || mode > ESA_PROBE_L2_STREAM)
    return fail(ESA_ERR_INVALID, "esa_probe_gather: unknown mode %d", mode);
  if (!sink) return fail(ESA_ERR_INVALID, "esa_probe_gather: null sink");
  if (pb->q_len == 0 || pb->batch == 0) return ESA_OK;
  const int es = elem_size(pb->dtype);
  if (int rc = check_tensor("k", k, es)) return rc;
  if (int rc = check_tensor("v", v, es)) return rc;
  esa::AttnParams p = base_params(pb);
  if (int rc = device_error_word(&p.err)) return rc;
  set_tensor(k, p.k, p.skb, p.skh, p.sks);
  set_tensor(v, p.v, p.svb, p.svh, p.svs);
  cudaStream_t s = (cudaStream_t)stream;
  switch (pb->dtype) {
    case ESA_DTYPE_BF16:
      if (pb->head_dim == 64) return ProbeOp::run<__nv_bfloat16, 64>(p, s, mode, sink);
      if (pb->head_dim == 128) return ProbeOp::run<__nv_bfloat16, 128>(p, s, mode, sink);
      break;
    case ESA_DTYPE_F16:
      if (pb->head_dim == 64) return ProbeOp::run<__half, 64>(p, s, mode, sink);
      if (pb->head_dim == 128) return ProbeOp::run<__half, 128>(p, s, mode, sink);
      break;
  }
  return fail(ESA_ERR_UNSUPPORTED, "esa_probe_gather: 16-bit data with head_dim 64 or 128 only");
}

// ---------------------------------------------------------------------------
// esa_backward_noalloc: the backward with its workspace in a fixed array that
// is part of the library, for callers that cannot allocate device memory (see
// include/esa_b200.h).  It forwards to esa_backward with that array as the
// workspace; nothing else about the backward differs.
// ---------------------------------------------------------------------------
namespace {

// The workspace itself.  Every GPU on which this library's kernels are loaded
// holds these ESA_NOALLOC_WORKSPACE_BYTES until the process exits.  Host code
// must not pass the symbol itself to a kernel (on the host it names a shadow
// variable, not device memory); it uses the device address looked up below.
static __device__ __align__(256) unsigned char g_noalloc_workspace[ESA_NOALLOC_WORKSPACE_BYTES];

// Device address of g_noalloc_workspace on the current device.
int noalloc_workspace_address(void** out) {
  static SymbolAddresses cache;
  return symbol_address(g_noalloc_workspace, cache, "esa_backward_noalloc", out);
}

}  // namespace

extern "C" int esa_backward_noalloc(const esa_problem_t* pb, esa_tensor_t q, esa_tensor_t k,
                                    esa_tensor_t v, esa_tensor_t o, const float* lse,
                                    esa_tensor_t dout, esa_tensor_t dq, esa_tensor_t dk,
                                    esa_tensor_t dv, const int64_t* sorted_rows,
                                    const int64_t* row_perm, void* stream) {
  if (int rc = check_problem(pb)) return rc;
  const size_t need = esa_backward_workspace_size(pb);
  if (need > ESA_NOALLOC_WORKSPACE_BYTES)
    return fail(ESA_ERR_WORKSPACE,
                "esa_backward_noalloc: this problem needs %zu bytes of workspace, more than the "
                "%zu-byte array built into the library; call esa_backward with a workspace",
                need, (size_t)ESA_NOALLOC_WORKSPACE_BYTES);
  void* ws = nullptr;
  if (int rc = noalloc_workspace_address(&ws)) return rc;
  // Every workspace byte the backward reads is written earlier in the same
  // call, so the array needs no clearing between calls.
  return esa_backward(pb, q, k, v, o, lse, dout, dq, dk, dv, sorted_rows, row_perm, ws,
                      ESA_NOALLOC_WORKSPACE_BYTES, stream);
}

// ---------------------------------------------------------------------------
// Decoder-layer harness entry points (include/esa_layer.h).
// ---------------------------------------------------------------------------
namespace {

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

int check_rows_op(const char* what, int32_t dtype, int64_t n_rows, int32_t dim) {
  if (dtype != ESA_DTYPE_F32 && dtype != ESA_DTYPE_BF16 && dtype != ESA_DTYPE_F16)
    return fail(ESA_ERR_INVALID, "%s: unknown dtype %d", what, dtype);
  if (n_rows < 0 || dim < 1) return fail(ESA_ERR_INVALID, "%s: bad shape", what);
  const int es = elem_size(dtype);
  if ((dim * es) % 16) return fail(ESA_ERR_INVALID, "%s: dim * element size must be a multiple of 16 bytes", what);
  return ESA_OK;
}

template <typename F>
int by_dtype(int32_t dtype, F&& f) {
  switch (dtype) {
    case ESA_DTYPE_F32: return f(float{});
    case ESA_DTYPE_BF16: return f(__nv_bfloat16{});
    default: return f(__half{});
  }
}

int norm_threads(int32_t dtype, int32_t dim) {
  const int vecs = dim / (16 / elem_size(dtype));
  return (vecs + 31) / 32 * 32;
}

int64_t norm_grid(int64_t n_rows) {
  const int64_t need = (n_rows + esa::layer::kNormRows - 1) / esa::layer::kNormRows;
  return std::max<int64_t>(1, std::min<int64_t>(need, esa::layer::kNormBwdCtas));
}

}  // namespace

extern "C" {

int esa_rmsnorm_forward(int32_t dtype, int64_t n_rows, int32_t dim, const void* x,
                        const void* residual, void* h_out, const void* weight, float eps,
                        void* y, float* rstd, void* stream) {
  if (int rc = check_rows_op("esa_rmsnorm_forward", dtype, n_rows, dim)) return rc;
  if (norm_threads(dtype, dim) > 1024)
    return fail(ESA_ERR_UNSUPPORTED, "esa_rmsnorm_forward: dim %d too large", dim);
  if (n_rows == 0) return ESA_OK;
  if (!x || !weight || !y || !rstd || (residual && !h_out))
    return fail(ESA_ERR_INVALID, "esa_rmsnorm_forward: null pointer");
  if (!aligned16(x) || !aligned16(weight) || !aligned16(y) || (residual && !aligned16(residual)) ||
      (h_out && !aligned16(h_out)))
    return fail(ESA_ERR_INVALID, "esa_rmsnorm_forward: pointers must be 16-byte aligned");
  const int threads = norm_threads(dtype, dim);
  const int64_t grid = std::min<int64_t>((n_rows + esa::layer::kNormRows - 1) / esa::layer::kNormRows,
                                         148 * 8);
  return by_dtype(dtype, [&](auto tag) {
    using T = decltype(tag);
    esa::layer::rmsnorm_fwd_kernel<T><<<(unsigned)grid, threads, 0, (cudaStream_t)stream>>>(
        n_rows, dim, static_cast<const T*>(x), static_cast<const T*>(residual),
        static_cast<T*>(h_out), static_cast<const T*>(weight), eps, static_cast<T*>(y), rstd);
    return check_launch("esa_rmsnorm_forward");
  });
}

size_t esa_rmsnorm_backward_workspace_size(int64_t n_rows, int32_t dim) {
  if (n_rows <= 0 || dim <= 0) return 0;
  return (size_t)norm_grid(n_rows) * dim * sizeof(float);
}

int esa_rmsnorm_backward(int32_t dtype, int64_t n_rows, int32_t dim, const void* h,
                         const void* weight, const float* rstd, const void* dy,
                         const void* dh_in, void* dh, void* dweight, void* workspace,
                         size_t workspace_bytes, void* stream) {
  if (int rc = check_rows_op("esa_rmsnorm_backward", dtype, n_rows, dim)) return rc;
  if (norm_threads(dtype, dim) > 1024)
    return fail(ESA_ERR_UNSUPPORTED, "esa_rmsnorm_backward: dim %d too large", dim);
  if (n_rows == 0) return ESA_OK;
  if (!h || !weight || !rstd || !dy || !dh || !dweight)
    return fail(ESA_ERR_INVALID, "esa_rmsnorm_backward: null pointer");
  if (!aligned16(h) || !aligned16(weight) || !aligned16(dy) || !aligned16(dh) ||
      (dh_in && !aligned16(dh_in)))
    return fail(ESA_ERR_INVALID, "esa_rmsnorm_backward: pointers must be 16-byte aligned");
  const size_t need = esa_rmsnorm_backward_workspace_size(n_rows, dim);
  if (!workspace || workspace_bytes < need)
    return fail(ESA_ERR_WORKSPACE, "esa_rmsnorm_backward: workspace of %zu bytes given, %zu needed",
                workspace_bytes, need);
  const int threads = norm_threads(dtype, dim);
  const int grid = (int)norm_grid(n_rows);
  float* part = static_cast<float*>(workspace);
  return by_dtype(dtype, [&](auto tag) {
    using T = decltype(tag);
    cudaStream_t s = (cudaStream_t)stream;
    esa::layer::rmsnorm_bwd_kernel<T><<<grid, threads, 0, s>>>(
        n_rows, dim, static_cast<const T*>(h), static_cast<const T*>(weight), rstd,
        static_cast<const T*>(dy), static_cast<const T*>(dh_in), static_cast<T*>(dh), part);
    if (int rc = check_launch("esa_rmsnorm_backward")) return rc;
    esa::layer::sum_partials_kernel<T><<<(dim + 255) / 256, 256, 0, s>>>(
        grid, dim, part, static_cast<T*>(dweight));
    return check_launch("esa_rmsnorm_backward (weight sum)");
  });
}

int esa_rope_apply(int32_t dtype, int32_t batch, int64_t seq_len, int32_t head_dim,
                   esa_tensor_t q, int32_t num_q_heads, esa_tensor_t k, int32_t num_k_heads,
                   const int64_t* positions, const float* inv_freq, int32_t inverse,
                   void* stream) {
  if (dtype != ESA_DTYPE_F32 && dtype != ESA_DTYPE_BF16 && dtype != ESA_DTYPE_F16)
    return fail(ESA_ERR_INVALID, "esa_rope_apply: unknown dtype %d", dtype);
  const int es = elem_size(dtype);
  if (batch < 0 || seq_len < 0 || num_q_heads < 0 || num_k_heads < 0 || head_dim < 2 ||
      ((head_dim / 2) * es) % 16 || head_dim % 2)
    return fail(ESA_ERR_INVALID, "esa_rope_apply: bad shape (head_dim / 2 * element size must "
                "be a multiple of 16 bytes)");
  if (batch > 65535 || seq_len > kMaxPosition)
    return fail(ESA_ERR_UNSUPPORTED, "esa_rope_apply: batch or seq_len too large");
  if (batch == 0 || seq_len == 0 || num_q_heads + (k.data ? num_k_heads : 0) == 0) return ESA_OK;
  if (!q.data || !inv_freq) return fail(ESA_ERR_INVALID, "esa_rope_apply: null pointer");
  if (int rc = check_tensor("q", q, es)) return rc;
  if (k.data)
    if (int rc = check_tensor("k", k, es)) return rc;
  const int nk = k.data ? num_k_heads : 0;
  const size_t smem = (size_t)head_dim * sizeof(float);
  dim3 grid((unsigned)seq_len, (unsigned)batch);
  return by_dtype(dtype, [&](auto tag) {
    using T = decltype(tag);
    esa::layer::rope_kernel<T><<<grid, 256, smem, (cudaStream_t)stream>>>(
        head_dim, static_cast<T*>(q.data), q.stride_b, q.stride_h, q.stride_s, num_q_heads,
        static_cast<T*>(k.data), k.stride_b, k.stride_h, k.stride_s, nk, positions, inv_freq,
        inverse ? -1.f : 1.f);
    return check_launch("esa_rope_apply");
  });
}

int esa_swiglu_forward(int32_t dtype, int64_t n_rows, int32_t ffn, const void* gate_up,
                       void* out, void* stream) {
  if (int rc = check_rows_op("esa_swiglu_forward", dtype, n_rows, ffn)) return rc;
  if (n_rows == 0) return ESA_OK;
  if (!gate_up || !out || !aligned16(gate_up) || !aligned16(out))
    return fail(ESA_ERR_INVALID, "esa_swiglu_forward: null or misaligned pointer");
  const unsigned grid = (unsigned)std::min<int64_t>(n_rows, 148 * 16);
  return by_dtype(dtype, [&](auto tag) {
    using T = decltype(tag);
    esa::layer::swiglu_fwd_kernel<T><<<grid, 256, 0, (cudaStream_t)stream>>>(
        n_rows, ffn, static_cast<const T*>(gate_up), static_cast<T*>(out));
    return check_launch("esa_swiglu_forward");
  });
}

int esa_swiglu_backward(int32_t dtype, int64_t n_rows, int32_t ffn, const void* gate_up,
                        const void* dout, void* dgate_up, void* out_recomputed, void* stream) {
  if (int rc = check_rows_op("esa_swiglu_backward", dtype, n_rows, ffn)) return rc;
  if (n_rows == 0) return ESA_OK;
  if (!gate_up || !dout || !dgate_up || !aligned16(gate_up) || !aligned16(dout) ||
      !aligned16(dgate_up) || (out_recomputed && !aligned16(out_recomputed)))
    return fail(ESA_ERR_INVALID, "esa_swiglu_backward: null or misaligned pointer");
  const unsigned grid = (unsigned)std::min<int64_t>(n_rows, 148 * 16);
  return by_dtype(dtype, [&](auto tag) {
    using T = decltype(tag);
    esa::layer::swiglu_bwd_kernel<T><<<grid, 256, 0, (cudaStream_t)stream>>>(
        n_rows, ffn, static_cast<const T*>(gate_up), static_cast<const T*>(dout),
        static_cast<T*>(dgate_up), static_cast<T*>(out_recomputed));
    return check_launch("esa_swiglu_backward");
  });
}

}  // extern "C"

// ---------------------------------------------------------------------------
// esa_copy_rows: the sequence split's layout copies (esa_rows.cuh).
// ---------------------------------------------------------------------------
extern "C" int esa_copy_rows(const esa_rows_t* r, void* stream) {
  if (!r) return fail(ESA_ERR_INVALID, "esa_copy_rows: null descriptor");
  const bool copy16 = r->src_dtype == r->dst_dtype &&
                      (r->src_dtype == ESA_DTYPE_BF16 || r->src_dtype == ESA_DTYPE_F16);
  const bool cast = r->src_dtype == ESA_DTYPE_F32 &&
                    (r->dst_dtype == ESA_DTYPE_BF16 || r->dst_dtype == ESA_DTYPE_F16);
  if (!copy16 && !cast)
    return fail(ESA_ERR_UNSUPPORTED, "esa_copy_rows: dtypes %d -> %d (a 16-bit copy or fp32 -> "
                "16-bit only)", r->src_dtype, r->dst_dtype);
  if (r->row_elems <= 0 || r->row_elems % 8 || r->row_elems / 8 > INT32_MAX)
    return fail(ESA_ERR_INVALID, "esa_copy_rows: row_elems %lld is not a positive multiple of 8",
                (long long)r->row_elems);
  const int64_t es = cast ? 4 : 2;
  int64_t rows = 1;
  for (int k = 0; k < 3; ++k) {
    if (r->count[k] < 0 || r->src_stride[k] < 0 || r->dst_stride[k] < 0)
      return fail(ESA_ERR_INVALID, "esa_copy_rows: negative count or stride at level %d", k);
    if ((r->src_stride[k] * es) % 16 || (r->dst_stride[k] * 2) % 16)
      return fail(ESA_ERR_INVALID, "esa_copy_rows: strides of level %d are not 16-byte multiples",
                  k);
    if (r->count[k] == 0) return ESA_OK;
    if (rows > INT64_MAX / r->count[k])
      return fail(ESA_ERR_INVALID, "esa_copy_rows: too many rows");
    rows *= r->count[k];
  }
  if (!r->src || !r->dst || !aligned16(r->src) || !aligned16(r->dst))
    return fail(ESA_ERR_INVALID, "esa_copy_rows: null or misaligned pointer");
  esa::RowCopyParams p;
  p.src = r->src;
  p.dst = r->dst;
  p.n0 = r->count[0];
  p.n1 = r->count[1];
  p.n2 = r->count[2];
  p.s0 = r->src_stride[0];
  p.s1 = r->src_stride[1];
  p.s2 = r->src_stride[2];
  p.d0 = r->dst_stride[0];
  p.d1 = r->dst_stride[1];
  p.d2 = r->dst_stride[2];
  p.rows = rows;
  p.row_vecs = (int32_t)(r->row_elems / 8);
  int sms = 0;
  if (int rc = sm_count(&sms)) return rc;
  // whole waves of 8-warp CTAs, 8 per SM (64 warps), each warp striding over rows
  const int64_t ctas = std::min<int64_t>((rows + esa::kRowCopyWarps - 1) / esa::kRowCopyWarps,
                                         (int64_t)sms * 8);
  cudaStream_t s = (cudaStream_t)stream;
  LaunchTrace tr("copy_rows", s);
  const dim3 grid((unsigned)ctas), block(esa::kRowCopyWarps * 32);
  if (copy16) {
    if (r->src_dtype == ESA_DTYPE_BF16)
      esa::copy_rows_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, block, 0, s>>>(p);
    else
      esa::copy_rows_kernel<__half, __half><<<grid, block, 0, s>>>(p);
  } else if (r->dst_dtype == ESA_DTYPE_BF16) {
    esa::copy_rows_kernel<float, __nv_bfloat16><<<grid, block, 0, s>>>(p);
  } else {
    esa::copy_rows_kernel<float, __half><<<grid, block, 0, s>>>(p);
  }
  return check_launch("esa_copy_rows");
}
