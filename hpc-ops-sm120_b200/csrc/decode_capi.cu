// decode_capi.cu -- host side of libattention_decode_b200.so: argument
// checks, the split plan, TMA descriptor encoding, kernel launches and the
// extern "C" entry points declared in include/attention_decode_b200.h.
//
// The reference does all of this inside attention_decode_cuda
// (csrc/decode.cu:193-258) with ATen types; here the boundary takes plain
// pointers and sizes, the caller owns every buffer (output and workspace),
// and nothing synchronises the host.
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "attention_decode_b200.h"
#include "decode_kernels.cuh"

namespace {

thread_local std::string t_last_error;
std::atomic<int64_t> g_launches{0};

// Per-thread diagnostic timing of the streaming kernel (adb_timing_*).
struct Timing {
  bool enabled = false;
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> events;
};
thread_local Timing t_timing;

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
  return fail(ADB_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

// ------------------------------------------------------------ kernel table
struct Variant {
  const char* name;
  int head_dim;
  int tile_tokens;
  int threads;
  int smem_bytes;
  bool tma;
  const void* fn;     // ordinary decode / partial decode
  const void* fn_x;   // partial decode into peer exchange buffers
  const void* fn_a;   // decode with an appended token
  bool fp8;           // K/V are e4m3 (fn only)
};

template <int D, int W, int MB, int ST, bool TMA>
constexpr Variant make_variant(const char* name) {
  using C = adb::StreamCfg<D, W, MB, ST, TMA>;
  return Variant{name,
                 D,
                 C::kTT,
                 C::kThreads,
                 C::kSmemBytes,
                 TMA,
                 reinterpret_cast<const void*>(&adb::decode_stream_kernel<D, W, MB, ST, TMA, adb::kModeDecode>),
                 reinterpret_cast<const void*>(&adb::decode_stream_kernel<D, W, MB, ST, TMA, adb::kModeExchange>),
                 reinterpret_cast<const void*>(&adb::decode_stream_kernel<D, W, MB, ST, TMA, adb::kModeAppend>),
                 false};
}

template <int W, int MB, int ST>
constexpr Variant make_fp8_variant(const char* name) {
  using C = adb::StreamCfg<128, W, MB, ST, true, 1>;
  return Variant{name, 128, C::kTT, C::kThreads, C::kSmemBytes, true,
                 reinterpret_cast<const void*>(&adb::decode_stream_kernel<128, W, MB, ST, true, adb::kModeFp8>),
                 nullptr, nullptr, true};
}

// Name format: d<head_dim>_<tma|generic>_tt<tile tokens>_s<stages>.
const Variant kVariants[] = {
    make_variant<128, 4, 2, 3, true>("d128_tma_tt128_s3"),
    make_variant<128, 4, 1, 6, true>("d128_tma_tt64_s6"),
    make_variant<128, 4, 1, 3, true>("d128_tma_tt64_s3"),
    make_variant<64, 4, 2, 6, true>("d64_tma_tt128_s6"),
    make_variant<64, 4, 1, 6, true>("d64_tma_tt64_s6"),
    make_variant<128, 4, 1, 1, false>("d128_generic_tt64"),
    make_variant<64, 4, 1, 1, false>("d64_generic_tt64"),
    make_fp8_variant<4, 2, 6>("d128_fp8_tt128_s6"),
    make_fp8_variant<4, 1, 8>("d128_fp8_tt64_s8"),
    make_fp8_variant<8, 1, 5>("d128_fp8_w8_tt128_s5"),
    make_variant<128, 8, 1, 3, true>("d128_tma_w8_tt128_s3"),
    make_fp8_variant<8, 1, 6>("d128_fp8_w8_tt128_s6"),
};
constexpr int kNumVariants = sizeof(kVariants) / sizeof(kVariants[0]);
constexpr int kDefaultTma128 = 0, kSmallTma128 = 1, kDefaultTma64 = 3, kSmallTma64 = 4;
constexpr int kGeneric128 = 5, kGeneric64 = 6, kDefaultFp8 = 11, kSmallFp8 = 8, kLongFp8 = 7;

// ------------------------------------------------------------ device cache
struct DeviceState {
  bool probed = false;
  int sms = 0;
  int major = 0;
  int minor = 0;
  bool prepared[kNumVariants] = {};
  int blocks_per_sm[kNumVariants] = {};
};
constexpr int kMaxDevices = 64;
std::mutex g_mutex;
DeviceState g_devices[kMaxDevices];

int forced_variant() {
  static int forced = [] {
    const char* name = std::getenv("ADB_KERNEL_VARIANT");
    if (name == nullptr || *name == 0) return -1;
    for (int i = 0; i < kNumVariants; ++i)
      if (std::strcmp(name, kVariants[i].name) == 0) return i;
    return -1;
  }();
  return forced;
}

// ADB_DETERMINISTIC=1 turns off dynamic load balancing: every CTA processes
// exactly its static range, so repeated calls give bit-identical results.
// Tuning knobs read once from the environment (for measurement sweeps):
// ADB_MAX_STEALS (default by problem size) and ADB_CLAIM_DIVISOR (default 4).
int env_int(const char* name, int fallback) {
  const char* v = std::getenv(name);
  if (v == nullptr || *v == 0) return fallback;
  return std::atoi(v);
}

bool deterministic_mode() {
  static bool on = [] {
    const char* v = std::getenv("ADB_DETERMINISTIC");
    return v != nullptr && *v != 0 && std::strcmp(v, "0") != 0;
  }();
  return on;
}

int probe_device(int device, DeviceState** out) {
  if (device < 0 || device >= kMaxDevices)
    return fail(ADB_ERR_INVALID_ARGUMENT, "device index %d out of range", device);
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceState& st = g_devices[device];
  if (!st.probed) {
    cudaError_t e = cudaDeviceGetAttribute(&st.sms, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
    e = cudaDeviceGetAttribute(&st.major, cudaDevAttrComputeCapabilityMajor, device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(major)");
    e = cudaDeviceGetAttribute(&st.minor, cudaDevAttrComputeCapabilityMinor, device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(minor)");
    st.probed = true;
  }
  if (st.major != 10)
    return fail(ADB_ERR_DEVICE,
                "this library requires an sm_100 GPU (compute capability 10.x); device %d is "
                "%d.%d",
                device, st.major, st.minor);
  *out = &st;
  return ADB_OK;
}

// Sets the dynamic shared-memory limit of a variant on the current device and
// caches how many CTAs of it fit on one SM.
int prepare_variant(DeviceState* st, int vi) {
  std::lock_guard<std::mutex> lock(g_mutex);
  if (st->prepared[vi]) return ADB_OK;
  const Variant& v = kVariants[vi];
  cudaError_t e =
      cudaFuncSetAttribute(v.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, v.smem_bytes);
  if (e == cudaSuccess && v.fn_x != nullptr)
    e = cudaFuncSetAttribute(v.fn_x, cudaFuncAttributeMaxDynamicSharedMemorySize, v.smem_bytes);
  if (e == cudaSuccess && v.fn_a != nullptr)
    e = cudaFuncSetAttribute(v.fn_a, cudaFuncAttributeMaxDynamicSharedMemorySize, v.smem_bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(max dynamic smem)");
  int blocks = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, v.fn, v.threads, v.smem_bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
  if (blocks < 1) return fail(ADB_ERR_CUDA, "kernel %s does not fit on an SM", v.name);
  st->blocks_per_sm[vi] = blocks;
  st->prepared[vi] = true;
  return ADB_OK;
}

// ------------------------------------------------------------ TMA encode
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
cudaError_t g_encode_error = cudaSuccess;

int get_encoder(PFN_cuTensorMapEncodeTiled_v12000* fn) {
  std::call_once(g_encode_once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    g_encode_error =
        cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q);
    if (g_encode_error == cudaSuccess && q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  if (g_encode == nullptr) {
    if (g_encode_error != cudaSuccess) return cuda_fail(g_encode_error, "cuTensorMapEncodeTiled lookup");
    return fail(ADB_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  }
  *fn = g_encode;
  return ADB_OK;
}

// 3-D map over one KV tensor viewed as [pairs][S][D] bf16; a box is
// 64 columns (128 bytes, swizzled) x tile_tokens rows x 1 pair.  Rows past S
// are outside the tensor and read as zeros.
int encode_kv_map(CUtensorMap* map, const void* base, int64_t pairs, int64_t S, int64_t D,
                  int tile_tokens, int elem_bytes = 2) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  int rc = get_encoder(&encode);
  if (rc != ADB_OK) return rc;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(S),
                        static_cast<cuuint64_t>(pairs)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(D * elem_bytes),
                           static_cast<cuuint64_t>(S * D * elem_bytes)};
  // one box row is 128 bytes (the swizzle span): 64 bf16 or 128 e4m3 values
  cuuint32_t box[3] = {static_cast<cuuint32_t>(128 / elem_bytes), static_cast<cuuint32_t>(tile_tokens), 1u};
  cuuint32_t elem[3] = {1u, 1u, 1u};
  const CUtensorMapDataType dtype =
      elem_bytes == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUresult r = encode(map, dtype, 3, const_cast<void*>(base), dims,
                      strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ADB_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", int(r));
  return ADB_OK;
}

// 4-D map over a paged pool laid out [blocks][page][kv_heads][D] bf16 (NHD);
// a box is 64 columns x 1 head x `rows` tokens x 1 block.
int encode_nhd_map(CUtensorMap* map, const void* base, int64_t blocks, int64_t page,
                   int64_t heads, int64_t D, int rows) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  int rc = get_encoder(&encode);
  if (rc != ADB_OK) return rc;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(heads),
                        static_cast<cuuint64_t>(page), static_cast<cuuint64_t>(blocks)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(D * 2), static_cast<cuuint64_t>(heads * D * 2),
                           static_cast<cuuint64_t>(page * heads * D * 2)};
  cuuint32_t box[4] = {64u, 1u, static_cast<cuuint32_t>(rows), 1u};
  cuuint32_t elem[4] = {1u, 1u, 1u, 1u};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims,
                      strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ADB_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", int(r));
  return ADB_OK;
}

// Encoded descriptors of the last few K/V tensors this thread used: a decode
// loop passes the same cache buffers every step, and re-encoding costs host
// time on every call.
struct MapCacheEntry {
  const void* base = nullptr;
  int64_t pairs = 0, S = 0, D = 0, heads = 0;
  int tile_tokens = 0;
  int layout = 0;  // 0: 3-D [rows][S][D] bf16; 1: 4-D NHD pages (pairs = blocks, S = page); 2: 3-D e4m3
  CUtensorMap map;
};
constexpr int kMapCacheEntries = 8;
thread_local MapCacheEntry t_map_cache[kMapCacheEntries];
thread_local int t_map_cache_next = 0;

int kv_map(CUtensorMap* map, const void* base, int64_t pairs, int64_t S, int64_t D,
           int tile_tokens, int layout = 0, int64_t heads = 0) {
  for (const MapCacheEntry& e : t_map_cache)
    if (e.base == base && e.pairs == pairs && e.S == S && e.D == D &&
        e.tile_tokens == tile_tokens && e.layout == layout && e.heads == heads) {
      *map = e.map;
      return ADB_OK;
    }
  const int rc = layout == 0   ? encode_kv_map(map, base, pairs, S, D, tile_tokens)
                 : layout == 2 ? encode_kv_map(map, base, pairs, S, D, tile_tokens, 1)
                               : encode_nhd_map(map, base, pairs, S, heads, D, tile_tokens);
  if (rc != ADB_OK) return rc;
  MapCacheEntry& e = t_map_cache[t_map_cache_next];
  t_map_cache_next = (t_map_cache_next + 1) % kMapCacheEntries;
  e.base = base;
  e.pairs = pairs;
  e.S = S;
  e.D = D;
  e.heads = heads;
  e.tile_tokens = tile_tokens;
  e.layout = layout;
  e.map = *map;
  return ADB_OK;
}

// ------------------------------------------------------------ plan
struct Shape {
  int64_t B, Hq, Hkv, S, D, G, P;
};

int check_shape(int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t kv_len,
                int64_t head_dim, Shape* s) {
  if (batch <= 0 || q_heads <= 0 || kv_heads <= 0 || kv_len <= 0 || head_dim <= 0)
    return fail(ADB_ERR_INVALID_ARGUMENT,
                "all dimensions must be positive (empty tensors are unsupported): batch=%lld "
                "q_heads=%lld kv_heads=%lld kv_len=%lld head_dim=%lld",
                (long long)batch, (long long)q_heads, (long long)kv_heads, (long long)kv_len,
                (long long)head_dim);
  if (q_heads % kv_heads != 0)
    return fail(ADB_ERR_INVALID_ARGUMENT, "query heads (%lld) must be divisible by KV heads (%lld)",
                (long long)q_heads, (long long)kv_heads);
  const int64_t G = q_heads / kv_heads;
  if (G != 1 && G != 4 && G != 8)
    return fail(ADB_ERR_UNSUPPORTED, "supported GQA group sizes are 1, 4 and 8 (got %lld)",
                (long long)G);
  if (head_dim != 64 && head_dim != 128)
    return fail(ADB_ERR_UNSUPPORTED, "head dimension must be 64 or 128 (got %lld)",
                (long long)head_dim);
  if (kv_len > INT32_MAX)
    return fail(ADB_ERR_INVALID_ARGUMENT, "kv_len %lld exceeds 2^31-1", (long long)kv_len);
  if (batch * kv_heads > INT32_MAX)
    return fail(ADB_ERR_INVALID_ARGUMENT, "batch*kv_heads exceeds 2^31-1");
  *s = Shape{batch, q_heads, kv_heads, kv_len, head_dim, G, batch * kv_heads};
  return ADB_OK;
}

// Workspace layout (offsets 256-byte aligned):
//   header, zero on entry and left zero by every completed call:
//     claims u64[Nc] | counters u32[2] | done u64[P] (8-aligned) | slot_pair u32[dyn]
//   acc f32[(Nc+P+dyn)*G*D] | ml f32[(Nc+P+dyn)*G*2]
struct Plan {
  int variant;
  int64_t num_ctas;
  int64_t dyn_slots;
  size_t off_claims, off_counters, off_done, off_slot_pair, header_bytes;
  size_t off_acc, off_ml, bytes;
};

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

int choose_variant(const Shape& s, bool tma, bool fp8 = false) {
  const int forced = forced_variant();
  if (fp8) return forced >= 0 && kVariants[forced].fp8 ? forced : kDefaultFp8;
  if (!tma) return s.D == 128 ? kGeneric128 : kGeneric64;
  if (forced >= 0 && kVariants[forced].head_dim == s.D && kVariants[forced].tma && !kVariants[forced].fp8)
    return forced;
  return s.D == 128 ? kDefaultTma128 : kDefaultTma64;
}

int make_plan(const Shape& s, bool varlen, bool tma, DeviceState* st, Plan* plan,
              bool allow_steal = true, bool fp8 = false) {
  int vi = choose_variant(s, tma, fp8);
  // Small problems: prefer the 64-token tile so more SMs get work.
  if (tma && forced_variant() < 0) {
    const int64_t tiles = s.P * ((s.S + kVariants[vi].tile_tokens - 1) / kVariants[vi].tile_tokens);
    if (tiles < 2LL * st->sms) vi = fp8 ? kSmallFp8 : (s.D == 128 ? kSmallTma128 : kSmallTma64);
    // FP8, long ranges per CTA (>= 192 tiles): the 4-warp variant streams
    // faster once start-up and tail no longer dominate (measured on cfg5:
    // 817 against 842 us; on cfg2-sized problems 8 warps win, 61.5 against 63.7 us).
    if (fp8 && tiles >= 192LL * st->sms) vi = kLongFp8;
  }
  int rc = prepare_variant(st, vi);
  if (rc != ADB_OK) return rc;
  const Variant& v = kVariants[vi];
  const int64_t nt_max = s.P * ((s.S + v.tile_tokens - 1) / v.tile_tokens);
  int64_t nc = static_cast<int64_t>(st->sms) * st->blocks_per_sm[vi];
  if (nc > nt_max) nc = nt_max;
  if (nc < 1) nc = 1;
  plan->variant = vi;
  plan->num_ctas = nc;
  plan->dyn_slots = (v.tma && allow_steal) ? adb::dynamic_slot_capacity(nc) : 0;
  const size_t slots = static_cast<size_t>(nc + s.P + plan->dyn_slots);
  plan->off_claims = 0;
  plan->off_counters = static_cast<size_t>(nc) * 8;
  plan->off_done = plan->off_counters + 8;
  plan->off_slot_pair = plan->off_done + static_cast<size_t>(s.P) * 8;
  plan->header_bytes = plan->off_slot_pair + static_cast<size_t>(plan->dyn_slots) * 4;
  plan->off_acc = align256(plan->header_bytes);
  plan->off_ml = plan->off_acc + align256(slots * s.G * s.D * sizeof(float));
  plan->bytes = plan->off_ml + align256(slots * s.G * 2 * sizeof(float));
  return ADB_OK;
}

struct DeviceGuard {
  int previous = -1;
  bool switched = false;
  cudaError_t error = cudaSuccess;
  explicit DeviceGuard(int device) {
    error = cudaGetDevice(&previous);
    if (error == cudaSuccess && previous != device) {
      error = cudaSetDevice(device);
      switched = error == cudaSuccess;
    }
  }
  ~DeviceGuard() {
    if (switched) cudaSetDevice(previous);
  }
};

bool is_aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// A paged K/V cache (adb_decode_paged): pools of 2^page_shift-token pages.
struct PagedArgs {
  const int32_t* block_table;
  int64_t bt_stride;
  int64_t num_blocks;
  int page_shift;
  int layout;  // ADB_PAGED_HND or ADB_PAGED_NHD
};

// Dequantisation scales of an e4m3 K/V cache (adb_decode_fp8).
struct Fp8Args {
  float k_scale;
  float v_scale;
};

// The new token of an appending decode (adb_decode_append): K/V rows [pairs][D].
struct AppendArgs {
  const void* k_new;
  const void* v_new;
};

// Destinations of a decode whose partial states go to every rank's exchange
// buffer (adb_decode_exchange).
struct ExchangeArgs {
  uint8_t* base[adb::kMaxRanks];
  int world;
  int rank;
  void* out = nullptr;      // fused merge: BF16 [rows][D] (nullptr: states only)
  int64_t timeout_us = 0;   // fused merge: bound of the wait for the peers' flags
};

int run_decode(const void* q, const void* k, const void* v, const int32_t* seqlens, void* out,
               float* state_acc, float* state_ml, int64_t batch, int64_t q_heads, int64_t kv_heads,
               int64_t kv_len, int64_t head_dim, void* workspace, size_t workspace_bytes,
               unsigned flags, int device, void* stream_ptr, bool allow_steal = true,
               const ExchangeArgs* exchange = nullptr, const PagedArgs* paged = nullptr,
               const AppendArgs* append = nullptr, const Fp8Args* fp8 = nullptr) {
  Shape s;
  int rc = check_shape(batch, q_heads, kv_heads, kv_len, head_dim, &s);
  if (rc != ADB_OK) return rc;
  const bool partial = state_acc != nullptr || exchange != nullptr;
  if (q == nullptr || k == nullptr || v == nullptr)
    return fail(ADB_ERR_INVALID_ARGUMENT, "Q, K and V pointers must be non-null");
  if (!partial && out == nullptr) return fail(ADB_ERR_INVALID_ARGUMENT, "output pointer is null");
  if (partial && exchange == nullptr && state_ml == nullptr)
    return fail(ADB_ERR_INVALID_ARGUMENT, "partial-state pointers must be non-null");
  DeviceGuard guard(device);
  if (guard.error != cudaSuccess) return cuda_fail(guard.error, "cudaSetDevice");
  DeviceState* st = nullptr;
  rc = probe_device(device, &st);
  if (rc != ADB_OK) return rc;
  const bool tma = is_aligned(k, 16) && is_aligned(v, 16);
  if (paged != nullptr && !tma)
    return fail(ADB_ERR_INVALID_ARGUMENT, "paged K/V caches must be 16-byte aligned");
  if (fp8 != nullptr && !tma)
    return fail(ADB_ERR_INVALID_ARGUMENT, "FP8 K/V caches must be 16-byte aligned");
  if (fp8 != nullptr && s.D != 128)
    return fail(ADB_ERR_UNSUPPORTED, "FP8 K/V supports head dimension 128 only (got %lld)",
                (long long)s.D);
  Plan plan;
  rc = make_plan(s, seqlens != nullptr, tma, st, &plan, allow_steal, fp8 != nullptr);
  if (rc != ADB_OK) return rc;
  if (workspace == nullptr || !is_aligned(workspace, 256))
    return fail(ADB_ERR_WORKSPACE, "workspace must be a non-null 256-byte aligned device buffer");
  if (workspace_bytes < plan.bytes)
    return fail(ADB_ERR_WORKSPACE, "workspace too small: %zu bytes given, %zu needed",
                workspace_bytes, plan.bytes);
  const Variant& var = kVariants[plan.variant];

  CUtensorMap tm_k, tm_v;
  std::memset(&tm_k, 0, sizeof(tm_k));
  std::memset(&tm_v, 0, sizeof(tm_v));
  if (var.tma && paged != nullptr) {
    // One box is a page-sized part of a tile: min(tile, page) tokens.
    const int64_t page = int64_t(1) << paged->page_shift;
    const int rows = static_cast<int>(page < var.tile_tokens ? page : var.tile_tokens);
    if (paged->layout == ADB_PAGED_HND) {  // [blocks * kv_heads][page][D]
      rc = kv_map(&tm_k, k, paged->num_blocks * s.Hkv, page, s.D, rows);
      if (rc == ADB_OK) rc = kv_map(&tm_v, v, paged->num_blocks * s.Hkv, page, s.D, rows);
    } else {  // [blocks][page][kv_heads][D]
      rc = kv_map(&tm_k, k, paged->num_blocks, page, s.D, rows, 1, s.Hkv);
      if (rc == ADB_OK) rc = kv_map(&tm_v, v, paged->num_blocks, page, s.D, rows, 1, s.Hkv);
    }
    if (rc != ADB_OK) return rc;
  } else if (var.tma) {
    const int layout = var.fp8 ? 2 : 0;
    rc = kv_map(&tm_k, k, s.P, s.S, s.D, var.tile_tokens, layout);
    if (rc != ADB_OK) return rc;
    rc = kv_map(&tm_v, v, s.P, s.S, s.D, var.tile_tokens, layout);
    if (rc != ADB_OK) return rc;
  }

  uint8_t* ws = static_cast<uint8_t*>(workspace);
  adb::DecodeParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.seqlens = seqlens;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.state_acc = state_acc;
  p.state_ml = state_ml;
  p.ws_acc = reinterpret_cast<float*>(ws + plan.off_acc);
  p.ws_ml = reinterpret_cast<float*>(ws + plan.off_ml);
  p.ws_claims = reinterpret_cast<unsigned long long*>(ws + plan.off_claims);
  p.ws_counters = reinterpret_cast<uint32_t*>(ws + plan.off_counters);
  p.ws_done = reinterpret_cast<unsigned long long*>(ws + plan.off_done);
  p.ws_slot_pair = reinterpret_cast<uint32_t*>(ws + plan.off_slot_pair);
  p.batch = s.B;
  p.kv_heads = s.Hkv;
  p.kv_len = s.S;
  p.group = static_cast<int>(s.G);
  p.partial_mode = partial ? 1 : 0;
  // Stealing pays for itself when each CTA streams long enough for the SMs'
  // unequal HBM shares to spread their finish times by more than the cost of
  // the extra segments it creates (about 192 tiles per CTA).
  static const int forced_steals = env_int("ADB_MAX_STEALS", -1);
  static const int claim_divisor = env_int("ADB_CLAIM_DIVISOR", 4);
  static const int steal_min_tiles = env_int("ADB_STEAL_MIN_TILES", 192);
  const int64_t tiles_per_cta =
      s.P * ((s.S + var.tile_tokens - 1) / var.tile_tokens) / plan.num_ctas;
  p.max_steals = forced_steals >= 0 ? forced_steals : (tiles_per_cta >= steal_min_tiles ? adb::kMaxSteals : 0);
  p.claim_divisor = claim_divisor >= 2 ? claim_divisor : 2;
  p.steal = (allow_steal && var.tma && !deterministic_mode() && p.max_steals > 0) ? 1 : 0;
  p.dyn_capacity = plan.dyn_slots;
  // FP8: the kernel's f16 operands hold the e4m3 values themselves; K's
  // scale multiplies the scores and V's the output.
  p.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(s.D)) *
                                    (fp8 != nullptr ? static_cast<double>(fp8->k_scale) : 1.0));
  p.v_scale = fp8 != nullptr ? fp8->v_scale : 1.f;
  p.k_new = append != nullptr ? static_cast<const __nv_bfloat16*>(append->k_new) : nullptr;
  p.v_new = append != nullptr ? static_cast<const __nv_bfloat16*>(append->v_new) : nullptr;
  p.k_cache = append != nullptr ? static_cast<__nv_bfloat16*>(const_cast<void*>(k)) : nullptr;
  p.v_cache = append != nullptr ? static_cast<__nv_bfloat16*>(const_cast<void*>(v)) : nullptr;
  p.block_table = paged != nullptr ? paged->block_table : nullptr;
  p.bt_stride = paged != nullptr ? paged->bt_stride : 0;
  p.paged = paged != nullptr ? (paged->layout == ADB_PAGED_HND ? 1 : 2) : 0;
  p.page_shift = paged != nullptr ? paged->page_shift : 0;
  for (int r = 0; r < adb::kMaxRanks; ++r) p.x_base[r] = nullptr;
  p.x_world = 0;
  p.x_rank = 0;
  p.x_out = nullptr;
  p.x_mergers = 0;
  p.x_timeout_ns = 0;
  if (exchange != nullptr) {
    for (int r = 0; r < exchange->world; ++r) p.x_base[r] = exchange->base[r];
    p.x_world = exchange->world;
    p.x_rank = exchange->rank;
    if (exchange->out != nullptr) {
      // one warp per row over the first CTAs: rows / 4 mergers at most
      const int64_t rows = s.B * s.Hq;
      const int64_t mergers = (rows + 3) / 4;
      p.x_out = static_cast<__nv_bfloat16*>(exchange->out);
      p.x_mergers = static_cast<int>(mergers < plan.num_ctas ? mergers : plan.num_ctas);
      p.x_timeout_ns = static_cast<uint64_t>(exchange->timeout_us) * 1000ull;
    }
  }

  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (!(flags & ADB_FLAG_HEADER_ZEROED)) {
    cudaError_t me = cudaMemsetAsync(ws, 0, plan.header_bytes, stream);
    if (me != cudaSuccess) return cuda_fail(me, "workspace header memset");
  }
  cudaEvent_t ev_start = nullptr, ev_stop = nullptr;
  if (t_timing.enabled) {
    cudaError_t te = cudaEventCreate(&ev_start);
    if (te == cudaSuccess) te = cudaEventCreate(&ev_stop);
    if (te == cudaSuccess) te = cudaEventRecord(ev_start, stream);
    if (te != cudaSuccess) return cuda_fail(te, "timing event");
  }
  // Programmatic stream serialisation: the kernel may launch while the
  // previous kernel in the stream drains; it waits (griddepcontrol.wait)
  // before touching global memory.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(plan.num_ctas));
  cfg.blockDim = dim3(var.threads);
  cfg.dynamicSmemBytes = static_cast<size_t>(var.smem_bytes);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {&tm_k, &tm_v, &p};
  const void* fn = exchange != nullptr ? var.fn_x : (append != nullptr ? var.fn_a : var.fn);
  cudaError_t e = cudaLaunchKernelExC(&cfg, fn, args);
  if (e != cudaSuccess) return cuda_fail(e, "decode kernel launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  if (t_timing.enabled) {
    e = cudaEventRecord(ev_stop, stream);
    if (e != cudaSuccess) return cuda_fail(e, "timing event");
    t_timing.events.emplace_back(ev_start, ev_stop);
  }
  return ADB_OK;
}

// ------------------------------------------------------------ fixed workspace
// Scratch for adb_decode_no_alloc: one array in the module's global memory,
// so that decoding needs no device allocation at all.  Every GPU that loads
// the library holds ADB_NO_ALLOC_WORKSPACE_BYTES of it until the process
// exits.  Host code cannot use the array's name as a device address; its
// address on each device comes from cudaGetSymbolAddress (below).
static __device__ __align__(256) unsigned char g_adb_fixed_workspace[ADB_NO_ALLOC_WORKSPACE_BYTES];

std::mutex g_fixed_mutex;
void* g_fixed_address[kMaxDevices] = {};

// Device address of g_adb_fixed_workspace on `device`, which must be the
// current device; looked up on the first call per device and kept (so it is
// stale after cudaDeviceReset reloads the module: the header says not to
// call the entry point again in that process).
int fixed_workspace(int device, void** address) {
  std::lock_guard<std::mutex> lock(g_fixed_mutex);
  if (g_fixed_address[device] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_adb_fixed_workspace);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(fixed workspace)");
    if (ptr == nullptr) return fail(ADB_ERR_CUDA, "fixed workspace has no device address");
    g_fixed_address[device] = ptr;
  }
  *address = g_fixed_address[device];
  return ADB_OK;
}

}  // namespace

extern "C" {

const char* adb_version(void) { return "attention_decode_b200 0.1.0 sm_100a"; }

const char* adb_last_error(void) { return t_last_error.c_str(); }

int adb_check_device(int device) {
  DeviceState* st = nullptr;
  return probe_device(device, &st);
}

int adb_decode_workspace_size(int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t kv_len,
                              int64_t head_dim, int has_seqlens, int device, size_t* bytes,
                              size_t* header_bytes) {
  if (bytes == nullptr) return fail(ADB_ERR_INVALID_ARGUMENT, "bytes pointer is null");
  Shape s;
  int rc = check_shape(batch, q_heads, kv_heads, kv_len, head_dim, &s);
  if (rc != ADB_OK) return rc;
  DeviceGuard guard(device);
  if (guard.error != cudaSuccess) return cuda_fail(guard.error, "cudaSetDevice");
  DeviceState* st = nullptr;
  rc = probe_device(device, &st);
  if (rc != ADB_OK) return rc;
  Plan a, b, f;
  rc = make_plan(s, has_seqlens != 0, true, st, &a);
  if (rc != ADB_OK) return rc;
  rc = make_plan(s, has_seqlens != 0, false, st, &b);
  if (rc != ADB_OK) return rc;
  f = a;
  if (s.D == 128) {  // the FP8 kernels (adb_decode_fp8) may plan differently
    rc = make_plan(s, has_seqlens != 0, true, st, &f, true, true);
    if (rc != ADB_OK) return rc;
  }
  *bytes = std::max({a.bytes, b.bytes, f.bytes});
  if (header_bytes != nullptr) *header_bytes = std::max({a.header_bytes, b.header_bytes, f.header_bytes});
  return ADB_OK;
}

int adb_decode(const void* q, const void* k, const void* v, const int32_t* seqlens, void* out,
               int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t kv_len, int64_t head_dim,
               void* workspace, size_t workspace_bytes, unsigned flags, int device, void* stream) {
  return run_decode(q, k, v, seqlens, out, nullptr, nullptr, batch, q_heads, kv_heads, kv_len,
                    head_dim, workspace, workspace_bytes, flags, device, stream);
}

int adb_decode_partial(const void* q, const void* k, const void* v, const int32_t* seqlens,
                       float* acc, float* ml, int64_t batch, int64_t q_heads, int64_t kv_heads,
                       int64_t kv_len, int64_t head_dim, void* workspace, size_t workspace_bytes,
                       unsigned flags, int device, void* stream) {
  if (acc == nullptr || ml == nullptr)
    return fail(ADB_ERR_INVALID_ARGUMENT, "partial-state pointers must be non-null");
  return run_decode(q, k, v, seqlens, nullptr, acc, ml, batch, q_heads, kv_heads, kv_len, head_dim,
                    workspace, workspace_bytes, flags, device, stream);
}

int adb_decode_fp8(const void* q, const void* k, const void* v, const int32_t* seqlens, void* out,
                   int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t kv_len,
                   int64_t head_dim, float k_scale, float v_scale, void* workspace,
                   size_t workspace_bytes, unsigned flags, int device, void* stream) {
  if (!(k_scale > 0.f) || !(v_scale > 0.f) || !std::isfinite(k_scale) || !std::isfinite(v_scale))
    return fail(ADB_ERR_INVALID_ARGUMENT, "FP8 scales must be positive and finite");
  Fp8Args fa{k_scale, v_scale};
  return run_decode(q, k, v, seqlens, out, nullptr, nullptr, batch, q_heads, kv_heads, kv_len,
                    head_dim, workspace, workspace_bytes, flags, device, stream, true, nullptr,
                    nullptr, nullptr, &fa);
}

int adb_decode_append(const void* q, const void* k_new, const void* v_new, void* k_cache,
                      void* v_cache, const int32_t* seqlens, void* out, int64_t batch,
                      int64_t q_heads, int64_t kv_heads, int64_t kv_capacity, int64_t head_dim,
                      void* workspace, size_t workspace_bytes, unsigned flags, int device,
                      void* stream) {
  if (k_new == nullptr || v_new == nullptr || seqlens == nullptr)
    return fail(ADB_ERR_INVALID_ARGUMENT,
                "append needs the new token's K and V rows and the sequence lengths");
  AppendArgs ap{k_new, v_new};
  return run_decode(q, k_cache, v_cache, seqlens, out, nullptr, nullptr, batch, q_heads, kv_heads,
                    kv_capacity, head_dim, workspace, workspace_bytes, flags, device, stream, true,
                    nullptr, nullptr, &ap);
}

int adb_decode_paged(const void* q, const void* k_cache, const void* v_cache,
                     const int32_t* block_table, int64_t block_table_stride,
                     const int32_t* seqlens, void* out, int64_t batch, int64_t q_heads,
                     int64_t kv_heads, int64_t head_dim, int64_t num_blocks, int64_t page_size,
                     int64_t max_blocks_per_seq, int layout, void* workspace,
                     size_t workspace_bytes, unsigned flags, int device, void* stream) {
  if (block_table == nullptr || seqlens == nullptr)
    return fail(ADB_ERR_INVALID_ARGUMENT, "paged decode needs a block table and sequence lengths");
  if (layout != ADB_PAGED_HND && layout != ADB_PAGED_NHD)
    return fail(ADB_ERR_INVALID_ARGUMENT, "unknown paged layout %d (ADB_PAGED_HND or ADB_PAGED_NHD)",
                layout);
  if (page_size < 8 || page_size > (1 << 20) || (page_size & (page_size - 1)) != 0)
    return fail(ADB_ERR_UNSUPPORTED, "page size must be a power of two from 8 to 2^20 (got %lld)",
                (long long)page_size);
  if (num_blocks <= 0 || max_blocks_per_seq <= 0)
    return fail(ADB_ERR_INVALID_ARGUMENT, "num_blocks and max_blocks_per_seq must be positive");
  if (block_table_stride < max_blocks_per_seq)
    return fail(ADB_ERR_INVALID_ARGUMENT, "block table row stride %lld is below max_blocks_per_seq %lld",
                (long long)block_table_stride, (long long)max_blocks_per_seq);
  if (num_blocks * kv_heads > INT32_MAX)
    return fail(ADB_ERR_INVALID_ARGUMENT, "num_blocks * kv_heads exceeds 2^31-1");
  int shift = 0;
  while ((int64_t(1) << shift) < page_size) ++shift;
  PagedArgs pa{block_table, block_table_stride, num_blocks, shift, layout};
  // The sequence capacity (max_blocks_per_seq pages) plays the role of kv_len:
  // lengths are clamped to it, and the workspace is sized for it.
  return run_decode(q, k_cache, v_cache, seqlens, out, nullptr, nullptr, batch, q_heads, kv_heads,
                    max_blocks_per_seq * page_size, head_dim, workspace, workspace_bytes, flags,
                    device, stream, true, nullptr, &pa);
}

int adb_decode_no_alloc(const void* q, const void* k, const void* v, const int32_t* seqlens,
                        void* out, int64_t batch, int64_t q_heads, int64_t kv_heads,
                        int64_t kv_len, int64_t head_dim, int device, void* stream) {
  Shape s;
  int rc = check_shape(batch, q_heads, kv_heads, kv_len, head_dim, &s);
  if (rc != ADB_OK) return rc;
  if (device < 0 || device >= kMaxDevices)
    return fail(ADB_ERR_INVALID_ARGUMENT, "device index %d out of range", device);
  DeviceGuard guard(device);
  if (guard.error != cudaSuccess) return cuda_fail(guard.error, "cudaSetDevice");
  DeviceState* st = nullptr;
  rc = probe_device(device, &st);
  if (rc != ADB_OK) return rc;
  // Size the scratch exactly as the launch will (no work stealing here, so
  // no thief slots), and refuse problems that do not fit.
  const bool tma = is_aligned(k, 16) && is_aligned(v, 16);
  Plan plan;
  rc = make_plan(s, seqlens != nullptr, tma, st, &plan, false);
  if (rc != ADB_OK) return rc;
  if (plan.bytes > ADB_NO_ALLOC_WORKSPACE_BYTES)
    return fail(ADB_ERR_WORKSPACE,
                "problem needs %zu bytes of scratch; the fixed workspace of adb_decode_no_alloc "
                "holds %zu bytes (use adb_decode with a caller-provided workspace)",
                plan.bytes, static_cast<size_t>(ADB_NO_ALLOC_WORKSPACE_BYTES));
  void* ws = nullptr;
  rc = fixed_workspace(device, &ws);
  if (rc != ADB_OK) return rc;
  // flags = 0: the scheduler header of the shared array is zeroed with one
  // cudaMemsetAsync on `stream` before the kernel.
  return run_decode(q, k, v, seqlens, out, nullptr, nullptr, batch, q_heads, kv_heads, kv_len,
                    head_dim, ws, ADB_NO_ALLOC_WORKSPACE_BYTES, 0u, device, stream, false);
}

int adb_combine(const float* acc, int64_t acc_part_stride, const float* ml, int64_t ml_part_stride,
                int64_t parts, int64_t rows, int64_t head_dim, void* out, int device, void* stream) {
  if (acc == nullptr || ml == nullptr || out == nullptr)
    return fail(ADB_ERR_INVALID_ARGUMENT, "combine pointers must be non-null");
  if (parts <= 0 || rows <= 0)
    return fail(ADB_ERR_INVALID_ARGUMENT, "parts and rows must be positive");
  if (head_dim != 64 && head_dim != 128)
    return fail(ADB_ERR_UNSUPPORTED, "head dimension must be 64 or 128 (got %lld)",
                (long long)head_dim);
  if (parts > 1 && (acc_part_stride < rows * head_dim || ml_part_stride < rows * 2))
    return fail(ADB_ERR_INVALID_ARGUMENT,
                "part strides (%lld, %lld) are smaller than one part (%lld, %lld floats)",
                (long long)acc_part_stride, (long long)ml_part_stride, (long long)(rows * head_dim),
                (long long)(rows * 2));
  DeviceGuard guard(device);
  if (guard.error != cudaSuccess) return cuda_fail(guard.error, "cudaSetDevice");
  DeviceState* st = nullptr;
  int rc = probe_device(device, &st);
  if (rc != ADB_OK) return rc;
  const int warps = 8;
  const dim3 grid(static_cast<unsigned>((rows + warps - 1) / warps));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out);
  if (head_dim == 128)
    adb::merge_states_kernel<128><<<grid, warps * 32, 0, s>>>(acc, acc_part_stride, ml,
                                                            ml_part_stride, parts, rows, o);
  else
    adb::merge_states_kernel<64><<<grid, warps * 32, 0, s>>>(acc, acc_part_stride, ml,
                                                           ml_part_stride, parts, rows, o);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "combine kernel launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return ADB_OK;
}

int adb_exchange_size(int64_t rows, int64_t head_dim, int world, size_t* bytes) {
  if (bytes == nullptr) return fail(ADB_ERR_INVALID_ARGUMENT, "bytes pointer is null");
  if (rows <= 0) return fail(ADB_ERR_INVALID_ARGUMENT, "rows must be positive");
  if (world < 1 || world > adb::kMaxRanks)
    return fail(ADB_ERR_UNSUPPORTED, "world size must be 1..%d (got %d)", adb::kMaxRanks, world);
  if (head_dim != 64 && head_dim != 128)
    return fail(ADB_ERR_UNSUPPORTED, "head dimension must be 64 or 128 (got %lld)",
                (long long)head_dim);
  *bytes = adb::x_bytes(world, rows, static_cast<int>(head_dim));
  return ADB_OK;
}

int adb_exchange_alloc(size_t bytes, int device, void** buffer) {
  if (buffer == nullptr || bytes == 0)
    return fail(ADB_ERR_INVALID_ARGUMENT, "buffer pointer is null or size is zero");
  *buffer = nullptr;
  DeviceGuard guard(device);
  if (guard.error != cudaSuccess) return cuda_fail(guard.error, "cudaSetDevice");
  void* ptr = nullptr;
  cudaError_t e = cudaMalloc(&ptr, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(exchange buffer)");
  e = cudaMemset(ptr, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(ptr);
    return cuda_fail(e, "zeroing the exchange buffer");
  }
  *buffer = ptr;
  return ADB_OK;
}

int adb_exchange_free(void* buffer, int device) {
  if (buffer == nullptr) return ADB_OK;
  DeviceGuard guard(device);
  if (guard.error != cudaSuccess) return cuda_fail(guard.error, "cudaSetDevice");
  const cudaError_t e = cudaFree(buffer);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFree(exchange buffer)");
  return ADB_OK;
}

int adb_ipc_handle(void* buffer, int device, unsigned char* handle) {
  if (buffer == nullptr || handle == nullptr)
    return fail(ADB_ERR_INVALID_ARGUMENT, "buffer and handle pointers must be non-null");
  static_assert(sizeof(cudaIpcMemHandle_t) == ADB_IPC_HANDLE_BYTES, "IPC handle size");
  DeviceGuard guard(device);
  if (guard.error != cudaSuccess) return cuda_fail(guard.error, "cudaSetDevice");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, buffer);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  std::memcpy(handle, &h, sizeof(h));
  return ADB_OK;
}

int adb_ipc_open(const unsigned char* handle, int device, void** buffer) {
  if (buffer == nullptr || handle == nullptr)
    return fail(ADB_ERR_INVALID_ARGUMENT, "buffer and handle pointers must be non-null");
  *buffer = nullptr;
  DeviceGuard guard(device);
  if (guard.error != cudaSuccess) return cuda_fail(guard.error, "cudaSetDevice");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(buffer, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  return ADB_OK;
}

int adb_ipc_close(void* buffer, int device) {
  if (buffer == nullptr) return ADB_OK;
  DeviceGuard guard(device);
  if (guard.error != cudaSuccess) return cuda_fail(guard.error, "cudaSetDevice");
  const cudaError_t e = cudaIpcCloseMemHandle(buffer);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
  return ADB_OK;
}

int adb_decode_exchange(const void* q, const void* k, const void* v, const int32_t* seqlens,
                        int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t kv_len,
                        int64_t head_dim, void* const* exchange, int world, int rank,
                        void* workspace, size_t workspace_bytes, unsigned flags, int device,
                        void* stream) {
  if (exchange == nullptr) return fail(ADB_ERR_INVALID_ARGUMENT, "exchange array is null");
  if (world < 1 || world > adb::kMaxRanks)
    return fail(ADB_ERR_UNSUPPORTED, "world size must be 1..%d (got %d)", adb::kMaxRanks, world);
  if (rank < 0 || rank >= world)
    return fail(ADB_ERR_INVALID_ARGUMENT, "rank %d is outside 0..%d", rank, world - 1);
  ExchangeArgs x;
  for (int r = 0; r < adb::kMaxRanks; ++r) x.base[r] = nullptr;
  for (int r = 0; r < world; ++r) {
    if (exchange[r] == nullptr || !is_aligned(exchange[r], 256))
      return fail(ADB_ERR_INVALID_ARGUMENT, "exchange buffer of rank %d is null or misaligned", r);
    x.base[r] = static_cast<uint8_t*>(exchange[r]);
  }
  x.world = world;
  x.rank = rank;
  return run_decode(q, k, v, seqlens, nullptr, nullptr, nullptr, batch, q_heads, kv_heads, kv_len,
                    head_dim, workspace, workspace_bytes, flags, device, stream, true, &x);
}

int adb_decode_exchange_merged(const void* q, const void* k, const void* v, const int32_t* seqlens,
                               int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t kv_len,
                               int64_t head_dim, void* const* exchange, int world, int rank, void* out,
                               int64_t timeout_us, void* workspace, size_t workspace_bytes,
                               unsigned flags, int device, void* stream) {
  if (exchange == nullptr || out == nullptr)
    return fail(ADB_ERR_INVALID_ARGUMENT, "exchange array and output pointer must be non-null");
  if (world < 1 || world > adb::kMaxRanks)
    return fail(ADB_ERR_UNSUPPORTED, "world size must be 1..%d (got %d)", adb::kMaxRanks, world);
  if (rank < 0 || rank >= world)
    return fail(ADB_ERR_INVALID_ARGUMENT, "rank %d is outside 0..%d", rank, world - 1);
  if (timeout_us <= 0) return fail(ADB_ERR_INVALID_ARGUMENT, "timeout must be positive");
  ExchangeArgs x;
  for (int r = 0; r < adb::kMaxRanks; ++r) x.base[r] = nullptr;
  for (int r = 0; r < world; ++r) {
    if (exchange[r] == nullptr || !is_aligned(exchange[r], 256))
      return fail(ADB_ERR_INVALID_ARGUMENT, "exchange buffer of rank %d is null or misaligned", r);
    x.base[r] = static_cast<uint8_t*>(exchange[r]);
  }
  x.world = world;
  x.rank = rank;
  x.out = out;
  x.timeout_us = timeout_us;
  return run_decode(q, k, v, seqlens, nullptr, nullptr, nullptr, batch, q_heads, kv_heads, kv_len,
                    head_dim, workspace, workspace_bytes, flags, device, stream, true, &x);
}

int adb_exchange_merge(const void* exchange, int world, int64_t rows, int64_t head_dim, void* out,
                       int64_t timeout_us, int device, void* stream) {
  if (exchange == nullptr || out == nullptr)
    return fail(ADB_ERR_INVALID_ARGUMENT, "exchange and output pointers must be non-null");
  if (world < 1 || world > adb::kMaxRanks)
    return fail(ADB_ERR_UNSUPPORTED, "world size must be 1..%d (got %d)", adb::kMaxRanks, world);
  if (rows <= 0) return fail(ADB_ERR_INVALID_ARGUMENT, "rows must be positive");
  if (head_dim != 64 && head_dim != 128)
    return fail(ADB_ERR_UNSUPPORTED, "head dimension must be 64 or 128 (got %lld)",
                (long long)head_dim);
  if (timeout_us <= 0) return fail(ADB_ERR_INVALID_ARGUMENT, "timeout must be positive");
  DeviceGuard guard(device);
  if (guard.error != cudaSuccess) return cuda_fail(guard.error, "cudaSetDevice");
  DeviceState* st = nullptr;
  int rc = probe_device(device, &st);
  if (rc != ADB_OK) return rc;
  const int warps = 8;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((rows + warps - 1) / warps));
  cfg.blockDim = dim3(warps * 32);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const uint8_t* xb = static_cast<const uint8_t*>(exchange);
  __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out);
  const uint64_t timeout_ns = static_cast<uint64_t>(timeout_us) * 1000ull;
  cudaError_t e;
  if (head_dim == 128)
    e = cudaLaunchKernelEx(&cfg, adb::exchange_merge_kernel<128>, xb, world, rows, o, timeout_ns);
  else
    e = cudaLaunchKernelEx(&cfg, adb::exchange_merge_kernel<64>, xb, world, rows, o, timeout_ns);
  if (e != cudaSuccess) return cuda_fail(e, "exchange merge kernel launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return ADB_OK;
}

int adb_read_error_flag(int device, int* flag, int reset) {
  if (flag == nullptr) return fail(ADB_ERR_INVALID_ARGUMENT, "flag pointer is null");
  DeviceGuard guard(device);
  if (guard.error != cudaSuccess) return cuda_fail(guard.error, "cudaSetDevice");
  cudaError_t e = cudaMemcpyFromSymbol(flag, adb::g_adb_error_flag, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "reading the device error flag");
  if (reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(adb::g_adb_error_flag, &zero, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "clearing the device error flag");
  }
  return ADB_OK;
}

int adb_launch_count(int64_t* launches) {
  if (launches == nullptr) return fail(ADB_ERR_INVALID_ARGUMENT, "launches pointer is null");
  *launches = g_launches.load(std::memory_order_relaxed);
  return ADB_OK;
}

int adb_timing_enable(int enable) {
  t_timing.enabled = enable != 0;
  return ADB_OK;
}

#ifdef ADB_TRACE
// Diagnostic build only: copies the per-CTA timeline of launch slot `slot`
// (0 or 1) into `host` (adb::kTraceCtas * 16 u64) and returns the slot the
// next launch will write.
__attribute__((visibility("default"))) int adb_trace_read(unsigned long long* host, int slot) {
  cudaError_t e = cudaMemcpyFromSymbol(host, adb::g_adb_trace, sizeof(unsigned long long) * adb::kTraceCtas * 16,
                                       sizeof(unsigned long long) * adb::kTraceCtas * 16 * (slot & 1));
  if (e != cudaSuccess) return cuda_fail(e, "reading the trace");
  unsigned int next = 0;
  e = cudaMemcpyFromSymbol(&next, adb::g_adb_trace_launch, sizeof(next));
  if (e != cudaSuccess) return cuda_fail(e, "reading the trace");
  return static_cast<int>(next & 1u);
}

// Diagnostic build only: the per-launch log (256 x 4 u64, then the merge log
// 256 x 3 u64) and the number of
// launches so far.
__attribute__((visibility("default"))) int adb_launch_log_read(unsigned long long* host, unsigned* launches) {
  cudaError_t e = cudaMemcpyFromSymbol(host, adb::g_adb_launch_log, sizeof(unsigned long long) * 1024);
  if (e == cudaSuccess)
    e = cudaMemcpyFromSymbol(host + 1024, adb::g_adb_merge_log, sizeof(unsigned long long) * 768);
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(launches, adb::g_adb_trace_launch, sizeof(unsigned));
  if (e != cudaSuccess) return cuda_fail(e, "reading the launch log");
  return ADB_OK;
}
#endif

int adb_timing_read(double* total_ms, int64_t* launches) {
  if (total_ms == nullptr || launches == nullptr)
    return fail(ADB_ERR_INVALID_ARGUMENT, "output pointers must be non-null");
  double sum = 0.0;
  int64_t n = 0;
  cudaError_t first_error = cudaSuccess;
  for (auto& pr : t_timing.events) {
    float ms = 0.f;
    cudaError_t e = cudaEventSynchronize(pr.second);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, pr.first, pr.second);
    if (e == cudaSuccess) {
      sum += ms;
      ++n;
    } else if (first_error == cudaSuccess) {
      first_error = e;
    }
    cudaEventDestroy(pr.first);
    cudaEventDestroy(pr.second);
  }
  t_timing.events.clear();
  *total_ms = sum;
  *launches = n;
  if (first_error != cudaSuccess) return cuda_fail(first_error, "reading timing events");
  return ADB_OK;
}

}  // extern "C"
