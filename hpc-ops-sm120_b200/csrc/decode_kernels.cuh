// decode_kernels.cuh -- BF16 split-K attention-decode kernels for sm_100a.
//
// One decode call is ONE kernel launch (replaces the reference's partial
// kernel + merge kernel pair and its fixed 256-token split grid,
// csrc/decode.cu:193-211).
//
// Work decomposition:
//   * A "pair" is one (batch, kv_head); its KV rows are contiguous in HBM at
//     row offset pair * S of the [B*Hkv*S, D] view.  Pair p has L_p valid
//     tokens (S, or seqlens[b]) cut into nt_p = ceil(L_p / TT) tiles of TT
//     tokens.  All tiles of all pairs form one flattened tile space of NT
//     tiles, and persistent CTA c of Nc owns the contiguous range
//     [c*NT/Nc, (c+1)*NT/Nc).
//   * Load balancing: SMs do not stream HBM at equal rates (their finish
//     times spread by ~20% under a static split), so a CTA whose range is
//     exhausted becomes a thief and takes unclaimed tiles from the CTA with
//     the most left.  Softmax state does not depend on tile order, so an
//     owner folds every tile of a pair it processed into one state whatever
//     was stolen in between.
//   * The part of a pair one CTA processed is a "segment".  An owner that
//     processed all of a pair's tiles writes the normalised BF16 output (or,
//     in partial mode, the state) directly.  Any other segment is written to
//     a workspace slot -- owners to slot (c + p), which is unique because c
//     and p are both non-decreasing along the flattened space (an owner whose
//     tiles of p were all stolen writes an empty state there), thieves to a
//     dynamically allocated slot tagged with its pair -- and then committed
//     by adding (owner ? 2^48 : 2^32) + tiles to the pair's counter.  The
//     committer that brings the owner and tile fields to (owners(p), nt_p)
//     merges all segments of p and writes the output: the split-K reduction
//     happens inside the same kernel, by whichever CTA finishes the pair last.
//   * Processing order: a CTA first processes its part of the pair it shares
//     with the next CTA, so the merges of pairs split between owners happen
//     early and overlap the stream; the last 1/claim_divisor of its range is
//     claimable, one tile at a time by the owner and in chunks of up to
//     kStealChunk tiles (from the back) by thieves.
//   * Scheduler state (claim counters, pair counters, slot tags) lives in a
//     workspace header that must be zero on entry; the last CTA to finish
//     resets it, so a workspace reused by stream-ordered calls is zeroed
//     once.
//
// Streaming (replaces decode_bf16_mma, csrc/decode.cu:70-167):
//   * one producer warp issues 3-D TMA tiled loads (cp.async.bulk.tensor,
//     128-byte swizzle, no multicast) of the K and V tiles into a kStages
//     deep shared-memory ring with full/empty mbarriers; a 32-byte record per
//     stage tells the consumers which tile it holds;
//   * kWarps consumer warps each own 16*kMB tokens of every tile and keep an
//     independent online-softmax state; Q.K^T and P.V run on the tensor
//     cores as m16n8k16 BF16 MMAs with the tokens as M and the GQA query
//     group (G <= 8) as N, so G = 8 fills the MMA exactly.  The score
//     fragment becomes the P.V B-operand with one movmatrix per 8x8 block,
//     without a shared-memory round trip;
//   * softmax is FP32 in the log2 domain (scores pre-scaled by
//     log2(e)/sqrt(D), exp2 on the SFU), the FlashAttention online
//     rescaling method.
#pragma once

#include "device_primitives.cuh"

namespace adb {

constexpr int kMaxGroup = 8;
constexpr float kLn2 = 0.693147180559945309f;
constexpr int kMaxSteals = 16;          // most steals one thief CTA may make (sizes the workspace)
constexpr int kMaxTableBatches = 1024;  // varlen: per-batch tile table kept in shared memory
constexpr int kStealChunk = 4;          // most tiles one steal takes
constexpr int kStealMinRemaining = 4;   // a victim with fewer claimable tiles is left alone
constexpr int kPrefetchTiles = 6;       // tiles warmed in L2 before the previous grid is done

#ifdef ADB_TRACE
// Diagnostic build only (-DADB_TRACE): per-CTA timeline of the last two
// launches, read back with adb_trace_read.  Per CTA: [0] smid | cta << 32,
// [1] entry, [2] after the grid dependency wait, [3] first tile arrived,
// [4] own range done, [5] exit (globaltimer ns), [6] own tiles | other tiles
// << 32, [7] merges | merge ns << 16, [8] producer's first load issued,
// [9] producer done, [10] producer ns waiting for free stages, [11] consumer
// (warp 0) ns waiting for full stages, [12] consumer ns from a full stage to
// its release.
constexpr int kTraceCtas = 1024;
__device__ unsigned long long g_adb_trace[2][kTraceCtas][16];
__device__ unsigned int g_adb_trace_launch = 0;
// Per launch (ring of 256): [0] earliest return from the grid dependency wait,
// [1] exit of the last CTA, [2] / [3] before the exchange publication's
// system fence / after its flag stores.  Per exchange merge (by call number):
// [0] after the grid dependency wait, [1] all flags seen, [2] CTA 0 done.
__device__ unsigned long long g_adb_launch_log[256][4];
__device__ unsigned long long g_adb_merge_log[256][3];
#define ADB_TRACE_ONLY(...) __VA_ARGS__
#else
#define ADB_TRACE_ONLY(...)
#endif

// ---------------------------------------------------------------- exchange
// Sequence sharding over NVLink peer memory.  Every rank owns one exchange
// buffer in its own HBM, mapped into every other rank's process (CUDA IPC):
//   [0, 64)     u32 flags[kMaxRanks]: the last call number rank s delivered
//   [64, 68)    u32 epoch: decode calls this rank has completed
//   [256, ...)  acc f32[2][world][rows][D]   partial states, by call parity,
//   then        ml  f32[2][world][rows][2]   then by the sending rank
// A rank's decode stores its states into its slot of every buffer (parity of
// its next call number), fences at system scope, and raises its flag in
// every buffer; the merge on each rank waits for all flags to reach the
// call number and merges the `world` slots of that parity.  A rank can run
// at most one call ahead of another (its next merge needs the other's
// states), so two parities never collide.
constexpr int kMaxRanks = 8;
constexpr size_t kXFlagsOffset = 0;
constexpr size_t kXEpochOffset = 64;
constexpr size_t kXAccOffset = 256;

__host__ __device__ constexpr size_t x_align256(size_t x) { return (x + 255) & ~size_t(255); }
__host__ __device__ constexpr size_t x_ml_offset(int world, int64_t rows, int d) {
  return kXAccOffset + x_align256(size_t(2) * world * rows * d * sizeof(float));
}
__host__ __device__ constexpr size_t x_bytes(int world, int64_t rows, int d) {
  return x_ml_offset(world, rows, d) + x_align256(size_t(2) * world * rows * 2 * sizeof(float));
}

// Dynamic (thief) segment slots a launch of `nc` CTAs can create: each steal
// takes at most kStealChunk tiles, so it adds at most that many segments.
__host__ __device__ constexpr int64_t dynamic_slot_capacity(int64_t nc) {
  return nc * (kStealChunk * kMaxSteals + 2);
}

struct DecodeParams {
  const __nv_bfloat16* q;  // [B*Hq, D]
  const __nv_bfloat16* k;  // [B*Hkv*S, D]
  const __nv_bfloat16* v;  // [B*Hkv*S, D]
  const int32_t* seqlens;  // [B] or nullptr (all sequences have S tokens)
  __nv_bfloat16* out;      // final mode: [B*Hq, D]
  float* state_acc;        // partial mode: [B*Hq, D]
  float* state_ml;         // partial mode: [B*Hq, 2]  (m natural units, l)
  float* ws_acc;           // [(Nc + P + dyn) * G, D]   segment accumulators
  float* ws_ml;            // [(Nc + P + dyn) * G, 2]   (m log2 units, l)
  // workspace header: zero on entry and on exit
  // [Nc] claims on each CTA's claimable positions: owner count from the
  // front in the low 32 bits, thief count from the back in the high 32 bits
  unsigned long long* ws_claims;
  uint32_t* ws_counters;           // [0] dynamic slots handed out, [1] CTAs finished
  // [P] per pair: (owner segments << 48) + (thief segments << 32) + tiles
  unsigned long long* ws_done;
  uint32_t* ws_slot_pair;          // [dyn] pair + 1 of each dynamic (thief) slot
  int64_t batch;
  int64_t kv_heads;
  int64_t kv_len;
  int group;
  int partial_mode;
  int steal;         // 1: dynamic load balancing enabled
  int max_steals;    // steals per thief CTA (<= kMaxSteals)
  int claim_divisor; // the last 1/claim_divisor of each range is claimable
  int64_t dyn_capacity;  // dynamic slots the workspace holds
  float scale_log2;  // log2(e) / sqrt(D)
  // Paged K/V cache (paged != 0): K and V are pools of pages of 2^page_shift
  // tokens, HND ([blocks][kv_heads][page][D], paged == 1) or NHD
  // ([blocks][page][kv_heads][D], paged == 2); page j of sequence b is
  // block_table[b * bt_stride + j].  A tile is loaded as TT / rows sub-boxes
  // of rows = min(TT, page) tokens, each from its own page.
  const int32_t* block_table;
  int64_t bt_stride;
  int paged;
  int page_shift;
  // Append (kModeAppend): the new token's K/V rows ([pairs][D]); they are
  // folded into each output row and written into the cache (k_cache /
  // v_cache, the same tensors as k / v) at position seqlens[b].
  const __nv_bfloat16* k_new;
  const __nv_bfloat16* v_new;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  // FP8 K/V (kModeFp8): V's dequantisation scale, applied to every output
  // (K's is folded into scale_log2).
  float v_scale;
  // Peer exchange (kernel instantiated with kExchange): the partial states
  // go to slot x_rank of every rank's exchange buffer, not state_acc/ml.
  uint8_t* x_base[kMaxRanks];  // each rank's exchange buffer as mapped here
  int x_world;
  int x_rank;
  // Fused merge (x_mergers > 0, ranks on distinct GPUs only): CTAs
  // 0..x_mergers-1 wait, bounded by x_timeout_ns, for every rank's flag of
  // this call and merge the rows into x_out (no separate merge launch).
  __nv_bfloat16* x_out;
  int x_mergers;
  uint64_t x_timeout_ns;
};

// Number of copies of each partial state a decode stores (one per rank).
template <bool kExchange>
__device__ __forceinline__ int partial_copies(const DecodeParams& p) {
  if constexpr (kExchange) return p.x_world; else return 1;
}

// This rank's call counter (it only changes when the last CTA finishes,
// after every store of the call).
__device__ __forceinline__ uint32_t x_epoch(const DecodeParams& p) {
  return *reinterpret_cast<const volatile uint32_t*>(p.x_base[p.x_rank] + kXEpochOffset);
}

// Destination of copy s of the partial states: the local arrays, or slot
// `p.x_rank` of rank s's exchange buffer at parity `par` (of the call being
// produced).
template <bool kExchange>
__device__ __forceinline__ float* partial_acc(const DecodeParams& p, int s, int64_t par,
                                              int64_t rows, int d) {
  if constexpr (!kExchange) return p.state_acc;
  return reinterpret_cast<float*>(p.x_base[s] + kXAccOffset) + (par * p.x_world + p.x_rank) * rows * d;
}
template <bool kExchange>
__device__ __forceinline__ float* partial_ml(const DecodeParams& p, int s, int64_t par,
                                             int64_t rows, int d) {
  if constexpr (!kExchange) return p.state_ml;
  return reinterpret_cast<float*>(p.x_base[s] + x_ml_offset(p.x_world, rows, d)) +
         (par * p.x_world + p.x_rank) * rows * 2;
}

__device__ __forceinline__ float neg_inf() { return __int_as_float(0xff800000); }

// Merges parts <= kMaxRanks partial states (m in natural units) of one row
// into BF16; called by one warp.  Every part's (m, l) and accumulator row are
// requested together (lane r reads part r's (m, l); each lane its dims of
// every part), so the merge is one round trip of loads.  Empty parts (l = 0)
// weigh zero.  The cross-GPU merge of sequence shards (the reference's
// merge_splits, csrc/decode.cu:169-184, over ranks).
template <int D>
__device__ __forceinline__ void merge_row_few(const float* __restrict__ acc, int64_t acc_stride,
                                              const float* __restrict__ ml, int64_t ml_stride,
                                              int parts, int64_t row, __nv_bfloat16* __restrict__ out,
                                              int lane) {
  constexpr int kPer = D / 32;
  constexpr float kLog2e = 1.4426950408889634f;
  float m = neg_inf(), l = 0.f;
  if (lane < parts) {
    const float2 v = __ldcg(reinterpret_cast<const float2*>(ml + lane * ml_stride + 2 * row));
    m = v.x;
    l = v.y;
  }
  float x[kMaxRanks][kPer];
#pragma unroll
  for (int r = 0; r < kMaxRanks; ++r) {
#pragma unroll
    for (int i = 0; i < kPer; ++i) x[r][i] = 0.f;
    if (r < parts) {
      const float* src = acc + r * acc_stride + row * D + lane * kPer;
      if constexpr (kPer == 4) {
        const float4 v4 = __ldcg(reinterpret_cast<const float4*>(src));
        x[r][0] = v4.x; x[r][1] = v4.y; x[r][2] = v4.z; x[r][3] = v4.w;
      } else {
        const float2 v2 = __ldcg(reinterpret_cast<const float2*>(src));
        x[r][0] = v2.x; x[r][1] = v2.y;
      }
    }
  }
  float M = l > 0.f ? m : neg_inf();
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  const float Mu = M == neg_inf() ? 0.f : M;
  const float w = l > 0.f ? fast_exp2((m - Mu) * kLog2e) : 0.f;
  float L = w * l;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
  float O[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) O[i] = 0.f;
#pragma unroll
  for (int r = 0; r < kMaxRanks; ++r) {
    const float wr = __shfl_sync(0xffffffffu, w, r);
#pragma unroll
    for (int i = 0; i < kPer; ++i) O[i] += wr > 0.f ? wr * x[r][i] : 0.f;
  }
  __nv_bfloat16* dst = out + row * D + lane * kPer;
#pragma unroll
  for (int i = 0; i < kPer; ++i) dst[i] = __float2bfloat16_rn(L > 0.f ? O[i] / L : 0.f);
}

__device__ __forceinline__ int32_t clamped_len(const DecodeParams& p, int64_t b) {
  if (p.seqlens == nullptr) return static_cast<int32_t>(p.kv_len);
  int32_t len = __ldg(p.seqlens + b);
  if (len < 0) len = 0;
  if (len > p.kv_len) len = static_cast<int32_t>(p.kv_len);
  return len;
}

__device__ __forceinline__ int64_t tiles_of(int32_t len, int tt) {
  return (static_cast<int64_t>(len) + tt - 1) / tt;
}

// CTA whose tile range [c*NT/Nc, (c+1)*NT/Nc) contains tile t.
__device__ __forceinline__ int64_t cta_of_tile(int64_t t, int64_t nt_total, int64_t nc) {
  return ((t + 1) * nc + nt_total - 1) / nt_total - 1;
}

// Position in the flattened tile space.
struct Walk {
  int64_t b;     // batch
  int64_t h;     // kv head
  int64_t tile;  // tile index inside the pair
  int64_t nt;    // tiles in the current pair
  int32_t len;   // valid tokens in the current pair
};

__device__ __forceinline__ void walk_set_batch(Walk& w, const DecodeParams& p, int64_t b,
                                               int tt) {
  w.b = b;
  w.len = clamped_len(p, b);
  w.nt = tiles_of(w.len, tt);
}

__device__ __forceinline__ void walk_next(Walk& w, const DecodeParams& p, int tt) {
  if (++w.tile < w.nt) return;
  w.tile = 0;
  if (++w.h < p.kv_heads) return;  // same batch: same length, nt > 0
  w.h = 0;
  for (int64_t b = w.b + 1; b < p.batch; ++b) {
    walk_set_batch(w, p, b, tt);
    if (w.nt > 0) return;
  }
  w.b = p.batch;  // past the end; never dereferenced
  w.nt = 0;
}

// Tile t of batch b whose tiles start at flattened index `base`.
__device__ __forceinline__ void walk_locate(Walk& w, const DecodeParams& p, int64_t b,
                                            int64_t base, int64_t t, int tt) {
  walk_set_batch(w, p, b, tt);
  const int64_t r = t - base;
  w.h = r / w.nt;
  w.tile = r - w.h * w.nt;
}

// Inclusive block-wide scan of one int64 per thread.  `scratch` holds >= 33
// int64 in shared memory.  All threads of the block must call it.
__device__ __forceinline__ int64_t block_inclusive_scan(int64_t x, int64_t* scratch,
                                                        int64_t& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) scratch[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int64_t s = lane < nwarps ? scratch[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    scratch[lane] = s;
  }
  __syncthreads();
  const int64_t prefix = warp > 0 ? scratch[warp - 1] : 0;
  total = scratch[nwarps - 1];
  __syncthreads();
  return x + prefix;
}

enum : int32_t { kMetaOwn = 0, kMetaStolen = 1, kMetaEndOwn = 2, kMetaEndAll = 3 };

// What one ring stage holds (written by the producer before the stage's
// full-barrier arrive, read by the consumers after their wait).
struct TileMeta {
  int64_t tile;  // flattened tile index
  int32_t b, h, tile_in_pair, len, nt, kind;
};
static_assert(sizeof(TileMeta) == 32, "stage record");

__device__ __forceinline__ TileMeta meta_of(const Walk& w, int64_t t, int32_t kind) {
  TileMeta m;
  m.tile = t;
  m.b = static_cast<int32_t>(w.b);
  m.h = static_cast<int32_t>(w.h);
  m.tile_in_pair = static_cast<int32_t>(w.tile);
  m.len = w.len;
  m.nt = static_cast<int32_t>(w.nt);
  m.kind = kind;
  return m;
}

__device__ __forceinline__ TileMeta meta_marker(int32_t kind) {
  TileMeta m;
  m.tile = -1;
  m.b = m.h = m.tile_in_pair = m.len = m.nt = 0;
  m.kind = kind;
  return m;
}

template <int D, int kWarps, int kMB, int kStages, bool kTma, int kElem = 2>
struct StreamCfg {
  static constexpr int kTT = 16 * kWarps * kMB;  // tokens per tile
  static constexpr int kHalves = D * kElem / 128;  // 128-byte swizzle atoms per K/V row
  static constexpr int kBoxCols = 128 / kElem;     // elements per box row
  static constexpr int kBoxBytes = kTT * 128;    // one TMA box: kTT rows x 128 B
  static constexpr int kStageBytes = 2 * kHalves * kBoxBytes;  // K and V
  static constexpr int kRingStages = kTma ? kStages : 1;
  static constexpr int kThreads = (kWarps + (kTma ? 1 : 0)) * 32;
  static constexpr int kConsumerThreads = kWarps * 32;
  static constexpr int kRingBytes = kRingStages * kStageBytes;
  // Warps whose states meet in shared memory when a segment is flushed; with
  // more consumer warps, warp w + kFlushWarps first folds its state into
  // warp w's registers through the same buffer.
  static constexpr int kFlushWarps = kWarps < 4 ? kWarps : 4;
  static constexpr int kFlushAccBytes = kFlushWarps * kMaxGroup * D * 4;
  static constexpr int kFlushMlBytes = kFlushWarps * kMaxGroup * 2 * 4;
  static constexpr int kBarBytes = 2 * kRingStages * 8;
  static constexpr int kMetaBytes = kRingStages * 32;
  static constexpr int kTableBytes = (kMaxTableBatches + 1) * 8;
  static constexpr int kMiscBytes = 64 * 8;
  static constexpr int kSmemBytes = 1024 + kRingBytes + kFlushAccBytes + kFlushMlBytes +
                                    kBarBytes + kMetaBytes + kTableBytes + kMiscBytes;
  // Heads one consumer warp merges (warp w takes heads w, w + kWarps, ...).
  static constexpr int kHeadsPerWarp = (kMaxGroup + kWarps - 1) / kWarps;
  static_assert(D == 64 || D == 128, "head_dim");
  static_assert(kTT <= 256, "TMA box rows");
  static_assert(kBoxBytes % 1024 == 0, "128B-swizzle boxes must stay 1024-byte aligned");
  // The merge's slot list reuses the flush accumulator region.
  static constexpr int kMergeList = kFlushAccBytes / 4;
};

// Byte offset of the 16-byte chunk `chunk` (0..7) of row `row` inside a
// 128-byte-swizzled box (the layout CU_TENSOR_MAP_SWIZZLE_128B writes).
__device__ __forceinline__ uint32_t swz128(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// Appended token: score of query row `row` against the new key of `pair`
// (log2 domain), one warp; every lane gets the sum.
template <int D>
__device__ __forceinline__ float append_score(const DecodeParams& p, int64_t row, int64_t pair,
                                              int lane) {
  constexpr int kPer = D / 32;
  float dot = 0.f;
#pragma unroll
  for (int i = 0; i < kPer; ++i)
    dot += __bfloat162float(p.q[row * D + lane * kPer + i]) *
           __bfloat162float(p.k_new[pair * D + lane * kPer + i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
  return dot * p.scale_log2;
}

// Writes the new token's K and V rows into the cache at position `len` of
// `pair` (threads tid, tid + nthreads, ...); a full cache gets no write and
// sets the device error word.
template <int D>
__device__ __forceinline__ void append_store(const DecodeParams& p, int64_t pair, int32_t len,
                                             int tid, int nthreads) {
  if (len >= p.kv_len) {
    if (tid == 0) atomicOr(&g_adb_error_flag, kErrAppendFull);
    return;
  }
  const int64_t dst = (pair * p.kv_len + len) * D;
  for (int d = tid; d < D; d += nthreads) {
    p.k_cache[dst + d] = p.k_new[pair * D + d];
    p.v_cache[dst + d] = p.v_new[pair * D + d];
  }
}

// Kernel modes, each its own instantiation so that the extra work of one
// costs the others nothing (registers and code of the shared paths):
//   kModeDecode    decode / partial decode (local state arrays)
//   kModeExchange  partial states go to every rank's exchange buffer
//   kModeAppend    decode over the cache plus one new token, which is also
//                  written into the cache
//   kModeFp8       decode / partial decode of an FP8 (e4m3) K/V cache
constexpr int kModeDecode = 0, kModeExchange = 1, kModeAppend = 2, kModeFp8 = 3;

template <int D, int kWarps, int kMB, int kStages, bool kTma, int kMode>
__global__ void __launch_bounds__(StreamCfg<D, kWarps, kMB, kStages, kTma>::kThreads, 1)
    decode_stream_kernel(const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const DecodeParams p) {
  constexpr bool kFp8 = kMode == kModeFp8;
  using C = StreamCfg<D, kWarps, kMB, kStages, kTma, kFp8 ? 1 : 2>;
  constexpr bool kExchange = kMode == kModeExchange;
  constexpr bool kAppend = kMode == kModeAppend;
  static_assert(!kFp8 || (D == 128 && kTma), "FP8 K/V: head_dim 128, TMA path");
  constexpr int TT = C::kTT;
  constexpr int kTTShift = TT == 128 ? 7 : 6;
  static_assert(TT == 64 || TT == 128, "tile tokens");
  constexpr int kSlabs = D / 16;
  constexpr int kCT = C::kConsumerThreads;

  extern __shared__ uint8_t smem_raw[];
  // 128-byte-swizzled TMA boxes need 1024-byte aligned shared addresses.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* ring = smem;
  constexpr int kFW = C::kFlushWarps;
  float* fl_acc = reinterpret_cast<float*>(smem + C::kRingBytes);  // [kFW][8][D]
  float* fl_m = fl_acc + kFW * kMaxGroup * D;                       // [kFW][8]
  float* fl_l = fl_m + kFW * kMaxGroup;                             // [kFW][8]
  uint64_t* bars = reinterpret_cast<uint64_t*>(fl_l + kFW * kMaxGroup);
  TileMeta* meta = reinterpret_cast<TileMeta*>(bars + 2 * C::kRingStages);
  int64_t* table = reinterpret_cast<int64_t*>(meta + C::kRingStages);  // [B+1] varlen
  int64_t* misc = table + kMaxTableBatches + 1;
  // misc[0..32]: scan scratch; misc[40..43]: batches / bases of the first and
  // last tile; misc[44]: dynamic slot of a thief flush; misc[46]: broadcast
  // flag; misc[47]: dynamic slots in use; misc[48]: merge segment count;
  // misc[50]: abort flag; misc[52] / misc[53]: parity of the exchange slots
  // written / this call's number; misc[54]: peers' flags seen (fused merge)
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 50);
  // merge slot list, aliased on fl_acc (see StreamCfg)
  int32_t* mg_list = reinterpret_cast<int32_t*>(fl_acc);

  // Let the next kernel in the stream launch early; it must wait for this
  // grid (griddepcontrol.wait) before touching memory, as this one does.
  griddep_launch_dependents();
  ADB_TRACE_ONLY(const uint64_t tr_entry = global_timer_ns(); uint64_t tr_wait = 0, tr_first = 0, tr_own = 0, tr_merge_ns = 0; uint32_t tr_merges = 0, tr_own_tiles = 0, tr_other_tiles = 0; uint64_t tr_c1 = 0, tr_cwait = 0, tr_cbusy = 0;)

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t B = p.batch, Hkv = p.kv_heads, S = p.kv_len;
  const int64_t nc = gridDim.x, c = blockIdx.x;
  const int64_t P = B * Hkv;
  const int G = p.group;

  // ------------------------------------------------------------ barriers
  const uint32_t bar_base = smem_u32(bars);
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (C::kRingStages + s); };
  if (tid == 0) {
    *abort_flag = 0;
    if constexpr (kTma) {
      for (int s = 0; s < C::kRingStages; ++s) {
        mbar_init(full_bar(s), 1);
        mbar_init(empty_bar(s), kWarps);
      }
      fence_barrier_init();
      prefetch_tensormap(&tm_k);
      prefetch_tensormap(&tm_v);
    }
  }
  // ------------------------------------------------------------ uniform range
  // With one length for every sequence the CTA's tile range follows from the
  // parameters alone, so it is computed before the grid dependency wait and
  // the first loads go out as soon as the previous grid is done.
  const int64_t nt_uniform = (S + TT - 1) / TT;
  int64_t nt_total = 0, t0 = 0, t1 = 0;
  Walk first_w, last_w;  // tiles t0 and t1 - 1 (valid when t0 < t1)
  first_w = Walk{0, 0, 0, 0, 0};
  last_w = first_w;
  bool have_table = false;
  if (p.seqlens == nullptr) {
    nt_total = P * nt_uniform;
    t0 = c * nt_total / nc;
    t1 = (c + 1) * nt_total / nc;
    if (t0 < t1) {
      const int64_t b0 = t0 / nt_uniform / Hkv, b1 = (t1 - 1) / nt_uniform / Hkv;
      walk_locate(first_w, p, b0, b0 * Hkv * nt_uniform, t0, TT);
      walk_locate(last_w, p, b1, b1 * Hkv * nt_uniform, t1 - 1, TT);
    }
  }
  // While the previous grid in the stream drains, warm L2 with the first
  // tiles this CTA will stream (uniform layout: the range follows from the
  // parameters alone).  A prefetch reads nothing into the CTA and L2 is the
  // coherence point, so later loads still see whatever the previous grid
  // writes.  These first positions are never claimable by other CTAs unless
  // the range is shorter than kPrefetchTiles, where a stolen tile only costs
  // one wasted prefetch.
  if constexpr (kTma) {
    if (warp == kWarps && lane == 0 && p.seqlens == nullptr && p.paged == 0) {
      const int64_t ntu = nt_uniform;
      const int64_t a = t0, e = t1, n = e - a;
      if (n > 0) {
        // processing order: the part of the last pair that continues into
        // the next CTA's range first, then the range in order
        const int64_t last_tile = last_w.tile;
        int64_t rot = last_tile + 1 < ntu ? (last_tile + 1 < n ? last_tile + 1 : n) : 0;
        if (rot == n) rot = 0;
        const int64_t count = n < kPrefetchTiles ? n : kPrefetchTiles;
        for (int64_t i = 0; i < count; ++i) {
          const int64_t t = i < rot ? e - rot + i : a + i - rot;
          const int64_t pr = t / ntu;
          const int y = static_cast<int>((t - pr * ntu) * TT);
          const int z = static_cast<int>(pr);
#pragma unroll
          for (int h = 0; h < C::kHalves; ++h) {
            tma_prefetch_3d(&tm_k, h * C::kBoxCols, y, z);
            tma_prefetch_3d(&tm_v, h * C::kBoxCols, y, z);
          }
        }
      }
    }
  }
  __syncthreads();
  // No global memory is touched before the previous grid in the stream is done.
  griddep_wait();
#ifdef ADB_TRACE
  tr_wait = global_timer_ns();
  if (tid == 0) atomicMin(&g_adb_launch_log[g_adb_trace_launch & 255u][0], tr_wait);
#endif

  // Partial-state stores go to the local arrays, or (peer exchange) to this
  // rank's slot in every rank's exchange buffer, at the parity of the call
  // being produced (read once here and kept in shared memory, misc[52]).
  // Only the consumer warps wait for that read (they wait for the first tile
  // anyway); the producer goes straight to its first loads.  The varlen
  // set-up below passes __syncthreads before any thread uses the value.
  if constexpr (kExchange) {
    if (tid == 0) {
      const uint32_t call = x_epoch(p) + 1u;  // the call this launch produces
      misc[52] = call & 1u;
      misc[53] = call;
    }
    if (warp < kWarps) named_barrier_sync(1, C::kConsumerThreads);
  }
  auto acc_dest = [&](int s) -> float* {
    return partial_acc<kExchange>(p, s, kExchange ? misc[52] : 0, P * G, D);
  };
  auto ml_dest = [&](int s) -> float* {
    return partial_ml<kExchange>(p, s, kExchange ? misc[52] : 0, P * G, D);
  };

  // ------------------------------------------------------------ tile range
  // (varlen: computed after the wait below, from the sequence lengths)
  if (p.seqlens != nullptr) {
    // A batch that fits the block: one load of the lengths and one scan give
    // the total, the per-batch tile prefix (kept in shared memory) and the
    // batches holding tiles t0 and t1 - 1.
    if (B <= static_cast<int64_t>(blockDim.x)) {
      if (tid == 0) misc[40] = misc[42] = -1;  // ordered by the scan's barriers
      const int64_t x = tid < B ? Hkv * tiles_of(clamped_len(p, tid), TT) : 0;
      int64_t total = 0;
      const int64_t incl = block_inclusive_scan(x, misc, total);
      nt_total = total;
      have_table = true;
      t0 = nt_total > 0 ? c * nt_total / nc : 0;
      t1 = nt_total > 0 ? (c + 1) * nt_total / nc : 0;
      const int64_t excl = incl - x;
      if (tid < B) {
        table[tid] = excl;
        if (x > 0 && excl <= t0 && t0 < excl + x) {
          misc[40] = tid;
          misc[41] = excl;
        }
        if (x > 0 && excl <= t1 - 1 && t1 - 1 < excl + x) {
          misc[42] = tid;
          misc[43] = excl;
        }
      }
      if (tid == 0) table[B] = total;
    } else {
    // Pass 1: total tiles.  Pass 2: per-batch tile prefix (kept in shared
    // memory when the batch is small) and the batches holding tiles t0 and
    // t1 - 1.
    int64_t local = 0;
    for (int64_t b = tid; b < B; b += blockDim.x) local += Hkv * tiles_of(clamped_len(p, b), TT);
    int64_t total = 0;
    block_inclusive_scan(local, misc, total);
    nt_total = total;
    t0 = nt_total > 0 ? c * nt_total / nc : 0;
    t1 = nt_total > 0 ? (c + 1) * nt_total / nc : 0;
    have_table = B <= kMaxTableBatches;
    if (tid == 0) misc[40] = misc[42] = -1;
    __syncthreads();
    if (have_table || t0 < t1) {
      int64_t running = 0;
      for (int64_t base = 0; base < B; base += blockDim.x) {
        const int64_t b = base + tid;
        const int64_t x = b < B ? Hkv * tiles_of(clamped_len(p, b), TT) : 0;
        int64_t chunk_total = 0;
        const int64_t incl = block_inclusive_scan(x, misc, chunk_total);
        const int64_t excl = running + incl - x;
        if (b < B) {
          if (have_table) table[b] = excl;
          if (x > 0 && excl <= t0 && t0 < excl + x) {
            misc[40] = b;
            misc[41] = excl;
          }
          if (x > 0 && excl <= t1 - 1 && t1 - 1 < excl + x) {
            misc[42] = b;
            misc[43] = excl;
          }
        }
        running += chunk_total;
        __syncthreads();
        if (!have_table && misc[40] >= 0 && misc[42] >= 0) break;
      }
      if (tid == 0 && have_table) table[B] = running;
    }
    }
    __syncthreads();
    if (t0 < t1) {
      walk_locate(first_w, p, misc[40], misc[41], t0, TT);
      walk_locate(last_w, p, misc[42], misc[43], t1 - 1, TT);
    }
    if (c == 0) {  // CTA 0 writes the rows of empty sequences (zero output / empty states)
      const int64_t Hq = Hkv * G;
      for (int64_t b = tid; b < B; b += blockDim.x) {
        if (clamped_len(p, b) != 0) continue;
        if constexpr (kAppend) {  // only the new token: O = its V row, exactly
          for (int64_t h = 0; h < Hkv; ++h) {
            const int64_t pair = b * Hkv + h;
            for (int64_t row = pair * G; row < (pair + 1) * G; ++row)
              for (int d = 0; d < D; ++d) p.out[row * D + d] = p.v_new[pair * D + d];
            append_store<D>(p, pair, 0, 0, 1);
          }
        } else {
          for (int64_t row = b * Hq; row < (b + 1) * Hq; ++row) {
            if (!p.partial_mode) {
              for (int d = 0; d < D; ++d) p.out[row * D + d] = __float2bfloat16_rn(0.f);
              continue;
            }
            for (int s = 0; s < partial_copies<kExchange>(p); ++s) {
              float* a = acc_dest(s);
              float* ml = ml_dest(s);
              for (int d = 0; d < D; ++d) a[row * D + d] = 0.f;
              ml[2 * row] = neg_inf();
              ml[2 * row + 1] = 0.f;
            }
          }
        }
      }
    }
  }
  // Thieves decode arbitrary tiles, which needs the uniform layout or the table.
  const bool steal = kTma && p.steal && (p.seqlens == nullptr || have_table) && nt_total > 0;
  auto steal_on = [&](int64_t) { return steal; };
  // Processing order of a CTA's range [s, e) of n tiles: when the last pair
  // of the range continues into the next CTA's range, its part ("rot"
  // tiles) comes first, so both CTAs sharing the pair commit it early and
  // its merge overlaps the stream; then [s, e - rot) in order.  Positions
  // [0, n - n/claim_divisor) are static; with stealing the remaining
  // positions are claimed through the CTA's counter, by the owner or by
  // thieves.
  auto rot_of = [&](int64_t n, const Walk& lw) -> int64_t {
    const int64_t r = (lw.tile + 1 < lw.nt) ? (lw.tile + 1 < n ? lw.tile + 1 : n) : 0;
    return r == n ? 0 : r;
  };
  auto dyn_size_of = [&](int64_t n) -> int64_t { return steal_on(n) ? n / p.claim_divisor : 0; };
  auto tile_at = [&](int64_t s_v, int64_t e_v, int64_t rot, int64_t pos) -> int64_t {
    return pos < rot ? e_v - rot + pos : s_v + pos - rot;
  };

  // Decode any tile t (uniform layout or varlen table).
  auto locate = [&](int64_t t, Walk& w) {
    if (p.seqlens == nullptr) {
      const int64_t b = t / nt_uniform / Hkv;
      walk_locate(w, p, b, b * Hkv * nt_uniform, t, TT);
    } else {
      int64_t lo = 0, hi = B;  // table[lo] <= t < table[hi]
      while (hi - lo > 1) {
        const int64_t mid = (lo + hi) >> 1;
        if (table[mid] <= t)
          lo = mid;
        else
          hi = mid;
      }
      walk_locate(w, p, lo, table[lo], t, TT);
    }
  };

  // ------------------------------------------------------------ producer
  if constexpr (kTma) {
    if (warp == kWarps) {
      // K/V tiles are read exactly once: mark them first to leave L2, so the
      // segment states that other CTAs merge later stay resident.
      const uint64_t policy = l2_policy_evict_first();
      ADB_TRACE_ONLY(uint64_t tr_pwait = 0, tr_pfirst = 0;)
      int64_t k = 0;  // stage sequence number (lane 0)
      bool ok = true;
      // The whole producer warp runs the same control flow (the tile walks
      // are deterministic, so every lane holds the same cursors); side
      // effects belong to one lane -- lane 0 claims, writes the stage record
      // and arrives on the barriers -- except a paged tile's sub-boxes, which
      // lane j looks up and loads (one page each), so that small pages do not
      // serialise on one thread.
      const int sub_shift = p.paged != 0 && p.page_shift < kTTShift ? p.page_shift : kTTShift;
      const int n_sub = TT >> sub_shift;  // <= TT / 8 <= 32
      // Fill stage k with `m` (and its tile, if it is one); called by all lanes.
      auto issue = [&](const TileMeta& m) -> bool {
        const int s = static_cast<int>(k % kStages);
        const bool is_tile = m.kind == kMetaOwn || m.kind == kMetaStolen;
        // Paged: lane j looks its page up before waiting for the stage, so the
        // block-table read overlaps the wait.  Sub-boxes past the sequence's
        // last page reuse that page (their rows are masked as past the end).
        int32_t blk = 0;
        if (p.paged != 0 && is_tile && lane < n_sub) {
          const int64_t tok0 = static_cast<int64_t>(m.tile_in_pair) * TT;
          const int64_t last_page = m.len > 0 ? (static_cast<int64_t>(m.len) - 1) >> p.page_shift : 0;
          int64_t pg = (tok0 + (static_cast<int64_t>(lane) << sub_shift)) >> p.page_shift;
          if (pg > last_page) pg = last_page;
          blk = __ldg(p.block_table + static_cast<int64_t>(m.b) * p.bt_stride + pg);
        }
        bool waited = true;
        ADB_TRACE_ONLY(const uint64_t tr_p0 = global_timer_ns();)
        if (k >= kStages)
          waited = mbar_wait(empty_bar(s), static_cast<uint32_t>((k / kStages) - 1) & 1u, abort_flag);
        ADB_TRACE_ONLY(tr_pwait += global_timer_ns() - tr_p0; if (k == 0) tr_pfirst = global_timer_ns();)
        if (!__all_sync(0xffffffffu, waited)) return false;
        if (lane == 0) meta[s] = m;
        if (is_tile) {
          if (lane == 0) mbar_arrive_expect_tx(full_bar(s), C::kStageBytes);
          __syncwarp();
          uint8_t* st = ring + static_cast<size_t>(s) * C::kStageBytes;
          if (p.paged == 0) {
            if (lane == 0) {
              const int y = m.tile_in_pair * TT;
              const int z = static_cast<int>(m.b * Hkv + m.h);
#pragma unroll
              for (int h = 0; h < C::kHalves; ++h)
                tma_load_3d(smem_u32(st + h * C::kBoxBytes), &tm_k, h * C::kBoxCols, y, z, full_bar(s), policy);
#pragma unroll
              for (int h = 0; h < C::kHalves; ++h)
                tma_load_3d(smem_u32(st + (C::kHalves + h) * C::kBoxBytes), &tm_v, h * C::kBoxCols, y, z,
                            full_bar(s), policy);
            }
          } else if (lane < n_sub) {
            // Sub-box `lane` lands at row lane * rows of the stage's boxes;
            // rows is a multiple of 8, so every sub-box starts on a 1024-byte
            // swizzle atom and the layout equals one whole-tile load.
            const int64_t tok0 = static_cast<int64_t>(m.tile_in_pair) * TT;
            const int page_mask = (1 << p.page_shift) - 1;
            const int y = static_cast<int>((tok0 + (static_cast<int64_t>(lane) << sub_shift)) & page_mask);
            const uint32_t off = static_cast<uint32_t>(lane << sub_shift) * 128u;
#pragma unroll
            for (int h = 0; h < C::kHalves; ++h) {
              const uint32_t dk = smem_u32(st + h * C::kBoxBytes) + off;
              const uint32_t dv = smem_u32(st + (C::kHalves + h) * C::kBoxBytes) + off;
              if (p.paged == 1) {
                const int z = blk * static_cast<int>(Hkv) + m.h;
                tma_load_3d(dk, &tm_k, h * C::kBoxCols, y, z, full_bar(s), policy);
                tma_load_3d(dv, &tm_v, h * C::kBoxCols, y, z, full_bar(s), policy);
              } else {
                tma_load_4d(dk, &tm_k, h * C::kBoxCols, m.h, y, blk, full_bar(s), policy);
                tma_load_4d(dv, &tm_v, h * C::kBoxCols, m.h, y, blk, full_bar(s), policy);
              }
            }
          }
        } else if (lane == 0) {
          mbar_arrive(full_bar(s));
        }
        ++k;
        return true;
      };

      // Own phase: the static positions in order, then the claimable ones one
      // claim at a time (the next claim is in flight while the current tile
      // is issued).  One walk cursor per contiguous part of the order.
      {
        if (t0 < t1) {
          const int64_t n = t1 - t0;
          const int64_t rot = rot_of(n, last_w);
          const int64_t n_dyn = dyn_size_of(n);
          const int64_t n_stat = n - n_dyn;
          Walk rw = last_w;  // rotated part [t1 - rot, t1)
          rw.tile -= rot > 0 ? rot - 1 : 0;
          int64_t rw_t = t1 - (rot > 0 ? rot : 1);
          Walk nw = first_w;  // in-order part [t0, t1 - rot)
          int64_t nw_t = t0;
          auto issue_pos = [&](int64_t pos) -> bool {
            const int64_t tt = tile_at(t0, t1, rot, pos);
            Walk* cur = pos < rot ? &rw : &nw;
            int64_t* cur_t = pos < rot ? &rw_t : &nw_t;
            while (*cur_t < tt) {
              walk_next(*cur, p, TT);
              ++*cur_t;
            }
            return issue(meta_of(*cur, tt, kMetaOwn));
          };
          // A claim is valid while front + back < n_dyn (same atomic word).
          auto valid = [&](unsigned long long w) {
            return static_cast<int64_t>(w & 0xffffffffull) + static_cast<int64_t>(w >> 32) < n_dyn;
          };
          // Two claims are kept in flight: lane 0 issues the atomic one
          // tile ahead and the warp reads its result a tile later, so the
          // claim's round trip overlaps the wait for a free stage.  A claim
          // is never wasted: once one is invalid every later one is too.
          auto claim_issue = [&]() -> unsigned long long {
            return lane == 0 ? atomicAdd(p.ws_claims + c, 1ull) : 0ull;
          };
          unsigned long long c1 = 0ull, c2 = 0ull;
          if (n_dyn > 0) {
            c1 = claim_issue();
            c2 = claim_issue();
          }
          for (int64_t pos = 0; pos < n_stat && ok; ++pos) ok = issue_pos(pos);
          while (ok && n_dyn > 0) {
            const unsigned long long claim = __shfl_sync(0xffffffffu, c1, 0);
            if (!valid(claim)) break;
            c1 = c2;
            c2 = claim_issue();
            ok = issue_pos(n_stat + static_cast<int64_t>(claim & 0xffffffffull));
          }
        }
        if (ok) ok = issue(meta_marker(kMetaEndOwn));
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);

      // Steal phase: take up to kStealChunk positions from the back of the
      // claimable part of the CTA with the most unclaimed positions.
      if (steal && ok) {
        int steals = 0;
        const int max_steals = p.max_steals < kMaxSteals ? p.max_steals : kMaxSteals;
        for (int attempt = 0; attempt < 4 * nc + 8 && steals < max_steals; ++attempt) {
          int64_t best_rem = 0;
          int64_t best_v = -1;
          for (int64_t v = lane; v < nc; v += 32) {
            const int64_t s_v = v * nt_total / nc, e_v = (v + 1) * nt_total / nc;
            const int64_t size_v = dyn_size_of(e_v - s_v);
            const unsigned long long w = __ldcv(p.ws_claims + v);
            const int64_t rem = size_v - static_cast<int64_t>(w & 0xffffffffull) -
                                static_cast<int64_t>(w >> 32);
            if (rem > best_rem) {
              best_rem = rem;
              best_v = v;
            }
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            const int64_t r2 = __shfl_xor_sync(0xffffffffu, best_rem, o);
            const int64_t v2 = __shfl_xor_sync(0xffffffffu, best_v, o);
            if (r2 > best_rem || (r2 == best_rem && v2 > best_v)) {
              best_rem = r2;
              best_v = v2;
            }
          }
          if (best_rem < kStealMinRemaining) break;
          const int64_t s_v = best_v * nt_total / nc, e_v = (best_v + 1) * nt_total / nc;
          const int64_t n_v = e_v - s_v;
          const int64_t size_v = dyn_size_of(n_v);
          int64_t got = 0, back = 0;  // positions [n_v - back - got, n_v - back)
          if (lane == 0) {
            unsigned long long cur = __ldcv(p.ws_claims + best_v);
            for (int tries = 0; tries < 8; ++tries) {
              const int64_t f = static_cast<int64_t>(cur & 0xffffffffull);
              const int64_t bk = static_cast<int64_t>(cur >> 32);
              const int64_t rem = size_v - f - bk;
              if (rem < kStealMinRemaining) break;
              int64_t take = rem / 2;
              take = take > kStealChunk ? kStealChunk : take;
              const unsigned long long want = cur + (static_cast<unsigned long long>(take) << 32);
              const unsigned long long seen = atomicCAS(p.ws_claims + best_v, cur, want);
              if (seen == cur) {
                got = take;
                back = bk;
                break;
              }
              cur = seen;
            }
          }
          got = __shfl_sync(0xffffffffu, got, 0);
          back = __shfl_sync(0xffffffffu, back, 0);
          if (got == 0) continue;
          ++steals;
          {
            Walk lw;
            locate(e_v - 1, lw);
            const int64_t rot_v = rot_of(n_v, lw);
            for (int64_t i = 0; i < got && ok; ++i) {
              const int64_t tt = tile_at(s_v, e_v, rot_v, n_v - back - got + i);
              Walk w;
              locate(tt, w);
              ok = issue(meta_of(w, tt, kMetaStolen));
            }
          }
          if (!ok) break;
        }
      }
      if (ok) issue(meta_marker(kMetaEndAll));
#ifdef ADB_TRACE
      if (lane == 0 && c < kTraceCtas) {
        unsigned long long* r = g_adb_trace[g_adb_trace_launch & 1u][c];
        r[8] = tr_pfirst;
        r[9] = global_timer_ns();
        r[10] = tr_pwait;
      }
#endif
      return;
    }
  }

  // ------------------------------------------------------------ consumers
  const int g = lane >> 2, t = lane & 3;
  const uint16_t* q16 = reinterpret_cast<const uint16_t*>(p.q);
  const uint16_t* k16 = reinterpret_cast<const uint16_t*>(p.k);
  const uint16_t* v16 = reinterpret_cast<const uint16_t*>(p.v);

  uint32_t qf[kSlabs][2];
  auto load_q = [&](int64_t pair) {
    if (g < G) {
      const uint16_t* row = q16 + (pair * G + g) * D;
#pragma unroll
      for (int j = 0; j < kSlabs; ++j) {
        if constexpr (kFp8) {
          // f16, reduction index k of slab j = dims 16j + {4t, 4t+1} (k = 2t,
          // 2t+1) and 16j + {4t+2, 4t+3} (k = 2t+8, 2t+9): the order in which
          // a 16-bit ldmatrix delivers the FP8 K row (the dot product is the
          // same under any common permutation of its index)
          const uint16_t* r4 = row + 16 * j + 4 * t;
          qf[j][0] = pack_f16x2(__bfloat162float(__ushort_as_bfloat16(__ldg(r4))),
                                __bfloat162float(__ushort_as_bfloat16(__ldg(r4 + 1))));
          qf[j][1] = pack_f16x2(__bfloat162float(__ushort_as_bfloat16(__ldg(r4 + 2))),
                                __bfloat162float(__ushort_as_bfloat16(__ldg(r4 + 3))));
        } else {
          qf[j][0] = pack_u16x2(__ldg(row + 16 * j + 2 * t), __ldg(row + 16 * j + 2 * t + 1));
          qf[j][1] =
              pack_u16x2(__ldg(row + 16 * j + 8 + 2 * t), __ldg(row + 16 * j + 8 + 2 * t + 1));
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < kSlabs; ++j) qf[j][0] = qf[j][1] = 0u;
    }
  };

  float acc[kSlabs][4];
  float m_run[2], l_run[2];
  auto reset_state = [&]() {
#pragma unroll
    for (int j = 0; j < kSlabs; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    m_run[0] = m_run[1] = neg_inf();
    l_run[0] = l_run[1] = 0.f;
  };

  auto bar = [&]() { named_barrier_sync(1, kCT); };
  // Dynamic slots handed out so far, never more than the workspace holds.
  auto dyn_in_use = [&]() -> int64_t {
    const int64_t n = static_cast<int64_t>(__ldcg(p.ws_counters));
    return n < p.dyn_capacity ? n : p.dyn_capacity;
  };

  // Merge every committed segment of pair q and write its output.  Called by
  // all consumer threads of the CTA whose commit completed the pair.  The
  // segment slots (owners first_cta..last_cta, then every dynamic slot
  // tagged with q, found by a scan shared by all threads) are listed in
  // shared memory.  Each warp merges its heads 32 segments at a time: lane j
  // loads segment j's (m, l) of every head (one round trip for all the
  // weights), then the accumulator rows of several segments and of all its
  // heads are loaded together and folded in.
  auto merge_pair = [&](int64_t q, int64_t first, int64_t last, int64_t n_thieves) {
    __threadfence();
    ADB_TRACE_ONLY(const uint64_t tr_m0 = global_timer_ns();)
    constexpr int kPer = D / 32;
    float mrun[C::kHeadsPerWarp], lrun[C::kHeadsPerWarp], o[C::kHeadsPerWarp][kPer];
#pragma unroll
    for (int hi = 0; hi < C::kHeadsPerWarp; ++hi) {
      mrun[hi] = neg_inf();
      lrun[hi] = 0.f;
#pragma unroll
      for (int i = 0; i < kPer; ++i) o[hi][i] = 0.f;
    }
    // Thief segments are found by their tags; without thieves no scan is needed.
    if (n_thieves > 0) {
      if (tid == 0) misc[47] = dyn_in_use();
      bar();
    }
    const int64_t n_tag = n_thieves > 0 ? misc[47] : 0;
    const int64_t n_owner = last - first + 1;  // <= Nc
    const int64_t per_pass = C::kMergeList - n_owner;
    const int64_t passes = n_tag > 0 ? (n_tag + per_pass - 1) / per_pass : 1;
    for (int64_t r = 0; r < passes; ++r) {
      if (warp == 0) {
        // Owner slots first..last in order (warp-parallel, order kept with a
        // ballot); with at least as many tiles as CTAs every range is
        // non-empty and no division is needed.
        int n = 0;
        if (r == 0) {
          const bool all_owned = nc <= nt_total;
          for (int64_t base = first; base <= last; base += 32) {
            const int64_t cc = base + lane;
            const bool take =
                cc <= last && (all_owned || cc * nt_total / nc != (cc + 1) * nt_total / nc);
            const unsigned bal = __ballot_sync(0xffffffffu, take);
            if (take) mg_list[n + __popc(bal & ((1u << lane) - 1u))] = static_cast<int32_t>(cc + q);
            n += __popc(bal);
          }
        }
        if (lane == 0) misc[48] = n;
      }
      bar();
      const int64_t d_end = (r + 1) * per_pass < n_tag ? (r + 1) * per_pass : n_tag;
      for (int64_t d = r * per_pass + tid; d < d_end; d += kCT)
        if (__ldcg(p.ws_slot_pair + d) == static_cast<uint32_t>(q + 1))
          mg_list[atomicAdd(reinterpret_cast<int*>(misc + 48), 1)] = static_cast<int32_t>(nc + P + d);
      bar();
      const int n = static_cast<int>(misc[48]);
      constexpr int H = C::kHeadsPerWarp;
      constexpr int kU = 8;  // segments whose rows are in flight together
      for (int c0 = 0; c0 < n; c0 += 32) {
        const int cn = n - c0 < 32 ? n - c0 : 32;
        // Lane j holds segment c0 + j's (m, l) of each of this warp's heads:
        // one round trip for the chunk's weights.
        float w[H];
        {
          float mj[H], lj[H];
          const int64_t sb = lane < cn ? static_cast<int64_t>(mg_list[c0 + lane]) * G : 0;
#pragma unroll
          for (int hi = 0; hi < H; ++hi) {
            const int hd = warp + hi * kWarps;
            mj[hi] = neg_inf();
            lj[hi] = 0.f;
            if (hd < G && lane < cn) {
              const float2 ml2 = __ldcg(reinterpret_cast<const float2*>(p.ws_ml + 2 * (sb + hd)));
              mj[hi] = ml2.x;
              lj[hi] = ml2.y;
            }
          }
#pragma unroll
          for (int hi = 0; hi < H; ++hi) {
            // empty owner states (l = 0) hold no accumulator: weight 0
            float cm = lj[hi] > 0.f ? mj[hi] : neg_inf();
#pragma unroll
            for (int o2 = 16; o2 > 0; o2 >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o2));
            const float mnew = fmaxf(mrun[hi], cm);
            const float mu = mnew == neg_inf() ? 0.f : mnew;
            const float alpha = fast_exp2(mrun[hi] - mu);
            w[hi] = lj[hi] > 0.f ? fast_exp2(mj[hi] - mu) : 0.f;
            float ls = w[hi] * lj[hi];
#pragma unroll
            for (int o2 = 16; o2 > 0; o2 >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o2);
            lrun[hi] = lrun[hi] * alpha + ls;
#pragma unroll
            for (int i = 0; i < kPer; ++i) o[hi][i] *= alpha;
            mrun[hi] = mnew;
          }
        }
        // Accumulator rows: kU segments of every head of this warp at once.
        for (int j0 = 0; j0 < cn; j0 += kU) {
          float x[kU][H][kPer], wj[kU][H];
#pragma unroll
          for (int u = 0; u < kU; ++u) {
            const int j = j0 + u;
            const int64_t sb = static_cast<int64_t>(mg_list[c0 + (j < cn ? j : 0)]) * G;
#pragma unroll
            for (int hi = 0; hi < H; ++hi) {
              const int hd = warp + hi * kWarps;
              wj[u][hi] = __shfl_sync(0xffffffffu, w[hi], j & 31);
#pragma unroll
              for (int i = 0; i < kPer; ++i) x[u][hi][i] = 0.f;
              if (j < cn && hd < G && wj[u][hi] > 0.f) {
                const float* row = p.ws_acc + (sb + hd) * D + lane * kPer;
                if constexpr (kPer == 4) {
                  const float4 v4 = __ldcg(reinterpret_cast<const float4*>(row));
                  x[u][hi][0] = v4.x; x[u][hi][1] = v4.y; x[u][hi][2] = v4.z; x[u][hi][3] = v4.w;
                } else {
                  const float2 v2 = __ldcg(reinterpret_cast<const float2*>(row));
                  x[u][hi][0] = v2.x; x[u][hi][1] = v2.y;
                }
              }
            }
          }
#pragma unroll
          for (int u = 0; u < kU; ++u)
#pragma unroll
            for (int hi = 0; hi < H; ++hi)
#pragma unroll
              for (int i = 0; i < kPer; ++i) o[hi][i] += wj[u][hi] * x[u][hi][i];
        }
      }
      bar();  // the list is refilled next pass
    }
#pragma unroll
    for (int hi = 0; hi < C::kHeadsPerWarp; ++hi) {
      const int hd = warp + hi * kWarps;
      if (hd >= G) break;
      const int64_t row = q * G + hd;
      const float L = lrun[hi];
      const float vs = kFp8 ? p.v_scale : 1.f;
      if (p.partial_mode) {
        for (int s = 0; s < partial_copies<kExchange>(p); ++s) {
          float* a = acc_dest(s) + row * D + lane * kPer;
#pragma unroll
          for (int i = 0; i < kPer; ++i) a[i] = o[hi][i] * vs;
          if (lane == 0) {
            float* ml = ml_dest(s);
            ml[2 * row] = mrun[hi] * kLn2;
            ml[2 * row + 1] = L;
          }
        }
      } else if constexpr (kAppend) {
        // fold the new token into the row: online-softmax update by one key
        const float sn = append_score<D>(p, row, q, lane);
        const float mn = fmaxf(mrun[hi], sn);
        const float a = fast_exp2(mrun[hi] - mn), wn = fast_exp2(sn - mn);
        const float La = L * a + wn;
#pragma unroll
        for (int i = 0; i < kPer; ++i)
          p.out[row * D + lane * kPer + i] = __float2bfloat16_rn(
              (o[hi][i] * a + wn * __bfloat162float(p.v_new[q * D + lane * kPer + i])) / La);
      } else {
#pragma unroll
        for (int i = 0; i < kPer; ++i)
          p.out[row * D + lane * kPer + i] = __float2bfloat16_rn(L > 0.f ? o[hi][i] / L * vs : 0.f);
      }
    }
    if constexpr (kAppend) append_store<D>(p, q, clamped_len(p, q / Hkv), tid, kCT);
    ADB_TRACE_ONLY(tr_merge_ns += global_timer_ns() - tr_m0; ++tr_merges;)
  };

  // Commit `add` for pair q (after this CTA's segment of q is written) and
  // merge the pair if this commit completes it.
  auto commit = [&](int64_t q, int64_t toff, int64_t nt_q, unsigned long long add) {
    __threadfence();
    bar();
    const int64_t first = cta_of_tile(toff, nt_total, nc);
    const int64_t last = cta_of_tile(toff + nt_q - 1, nt_total, nc);
    if (tid == 0) {
      int64_t owners = last - first + 1;
      if (nc > nt_total) {  // some CTAs have an empty range
        owners = 0;
        for (int64_t cc = first; cc <= last; ++cc)
          owners += (cc * nt_total / nc != (cc + 1) * nt_total / nc);
      }
      const unsigned long long expected =
          (static_cast<unsigned long long>(owners) << 48) + static_cast<unsigned long long>(nt_q);
      const unsigned long long now = atomicAdd(p.ws_done + q, add) + add;
      const unsigned long long thieves = (now >> 32) & 0xffffull;
      misc[46] = ((now & ~(0xffffull << 32)) == expected) ? static_cast<int64_t>(thieves) + 1 : 0;
    }
    bar();
    const int64_t done = misc[46];  // 0: not complete; else 1 + thief segments
    if (done) {
      merge_pair(q, first, last, done - 1);
      // the completing commit is the last to touch q's counter in this call:
      // leave it zero for the next call
      if (tid == 0) p.ws_done[q] = 0ull;
    }
  };

  // Owner slots of pairs [q0, q1] whose tiles were all stolen: empty states,
  // committed as owners with no tiles.
  auto flush_empty = [&](int64_t q0, int64_t q1) {
    for (int64_t q = q0; q <= q1; ++q) {
      const int64_t b = q / Hkv, h = q - b * Hkv;
      const int64_t nt_q = tiles_of(clamped_len(p, b), TT);
      // Empty sequences have no tiles and no owner (CTA 0 wrote their rows);
      // pairs are skipped only when stealing is on, which implies the table.
      if (nt_q == 0 || (p.seqlens != nullptr && !have_table)) continue;
      if (tid < G) {
        const int64_t srow = (c + q) * G + tid;
        p.ws_ml[2 * srow] = neg_inf();
        p.ws_ml[2 * srow + 1] = 0.f;
      }
      const int64_t toff = p.seqlens == nullptr ? q * nt_uniform : table[b] + h * nt_q;
      commit(q, toff, nt_q, 1ull << 48);
    }
  };

  // Merge the kWarps states of `pair` and write them: directly when this
  // owner processed the whole pair, else to a slot followed by a commit.
  auto flush = [&](int64_t pair, bool thief, int64_t toff, int64_t nt_q, int64_t tiles) {
    const bool complete = !thief && tiles == nt_q;
    float lr0 = l_run[0], lr1 = l_run[1];
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      lr0 += __shfl_xor_sync(0xffffffffu, lr0, o);
      lr1 += __shfl_xor_sync(0xffffffffu, lr1, o);
    }
    // accumulator row -> dim: g and 8 + g (BF16), 2g and 2g + 1 (FP8 V order)
    constexpr int kRowB = kFp8 ? 1 : 8;
    const int da = kFp8 ? 2 * g : g;
    auto publish = [&](int slot_w) {
      if (g == 0) {
        fl_m[slot_w * kMaxGroup + 2 * t] = m_run[0];
        fl_m[slot_w * kMaxGroup + 2 * t + 1] = m_run[1];
        fl_l[slot_w * kMaxGroup + 2 * t] = lr0;
        fl_l[slot_w * kMaxGroup + 2 * t + 1] = lr1;
      }
      float* wa = fl_acc + slot_w * kMaxGroup * D;
#pragma unroll
      for (int j = 0; j < kSlabs; ++j) {
        wa[(2 * t) * D + 16 * j + da] = acc[j][0];
        wa[(2 * t + 1) * D + 16 * j + da] = acc[j][1];
        wa[(2 * t) * D + 16 * j + da + kRowB] = acc[j][2];
        wa[(2 * t + 1) * D + 16 * j + da + kRowB] = acc[j][3];
      }
    };
    if constexpr (kWarps > kFW) {
      // Warp w + kFW hands its state to warp w (same lane layout, so each
      // lane reads back exactly the values its counterpart wrote) ...
      if (warp >= kFW) publish(warp - kFW);
      bar();
      if (warp < kFW) {
        const float mo0 = fl_m[warp * kMaxGroup + 2 * t], mo1 = fl_m[warp * kMaxGroup + 2 * t + 1];
        const float lo0 = fl_l[warp * kMaxGroup + 2 * t], lo1 = fl_l[warp * kMaxGroup + 2 * t + 1];
        const float M0 = fmaxf(m_run[0], mo0), M1 = fmaxf(m_run[1], mo1);
        const float u0 = M0 == neg_inf() ? 0.f : M0, u1 = M1 == neg_inf() ? 0.f : M1;
        const float a0 = fast_exp2(m_run[0] - u0), b0 = fast_exp2(mo0 - u0);
        const float a1 = fast_exp2(m_run[1] - u1), b1 = fast_exp2(mo1 - u1);
        const float* wa = fl_acc + warp * kMaxGroup * D;
#pragma unroll
        for (int j = 0; j < kSlabs; ++j) {
          acc[j][0] = acc[j][0] * a0 + wa[(2 * t) * D + 16 * j + da] * b0;
          acc[j][1] = acc[j][1] * a1 + wa[(2 * t + 1) * D + 16 * j + da] * b1;
          acc[j][2] = acc[j][2] * a0 + wa[(2 * t) * D + 16 * j + da + kRowB] * b0;
          acc[j][3] = acc[j][3] * a1 + wa[(2 * t + 1) * D + 16 * j + da + kRowB] * b1;
        }
        lr0 = lr0 * a0 + lo0 * b0;
        lr1 = lr1 * a1 + lo1 * b1;
        m_run[0] = M0;
        m_run[1] = M1;
      }
      bar();
    }
    // ... and warps 0..kFW-1 meet in shared memory.
    if (warp < kFW) publish(warp);
    if (thief && tid == 0) {
      const uint32_t d = atomicAdd(p.ws_counters, 1u);
      if (d < p.dyn_capacity) {
        p.ws_slot_pair[d] = static_cast<uint32_t>(pair + 1);
        misc[44] = nc + P + d;
      } else {  // cannot happen with a zeroed header (the capacity bounds the claims)
        atomicOr(&g_adb_error_flag, kErrWorkspace);
        misc[44] = -1;
      }
    }
    bar();
    const int64_t slot = thief ? misc[44] : c + pair;
    if (slot < 0) {  // uniform: every thread read the same value
      bar();
      reset_state();
      return;
    }
    if constexpr (kAppend) {
      // new-token scores of the pair's heads, for the output below
      if (complete) {
        for (int hd = warp; hd < G; hd += kWarps) {
          const float sn = append_score<D>(p, pair * G + hd, pair, lane);
          if (lane == 0) misc[56 + hd] = __float_as_int(sn);
        }
        bar();
      }
    }
    for (int e = tid; e < G * D; e += kCT) {
      const int hd = e / D, d = e - hd * D;
      float M = neg_inf();
#pragma unroll
      for (int ww = 0; ww < kFW; ++ww) M = fmaxf(M, fl_m[ww * kMaxGroup + hd]);
      const float Mu = M == neg_inf() ? 0.f : M;
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int ww = 0; ww < kFW; ++ww) {
        const float f = fast_exp2(fl_m[ww * kMaxGroup + hd] - Mu);
        L += f * fl_l[ww * kMaxGroup + hd];
        O += f * fl_acc[(ww * kMaxGroup + hd) * D + d];
      }
      const int64_t row = pair * G + hd;
      if (kAppend && complete) {
        const float sn = __int_as_float(static_cast<int>(misc[56 + hd]));
        const float mn = fmaxf(M, sn);
        const float a = fast_exp2(M - mn), wn = fast_exp2(sn - mn);
        p.out[row * D + d] = __float2bfloat16_rn(
            (O * a + wn * __bfloat162float(p.v_new[pair * D + d])) / (L * a + wn));
      } else if (complete && !p.partial_mode) {
        p.out[row * D + d] = __float2bfloat16_rn(L > 0.f ? O / L * (kFp8 ? p.v_scale : 1.f) : 0.f);
      } else if (complete) {
        for (int s = 0; s < partial_copies<kExchange>(p); ++s) {
          acc_dest(s)[row * D + d] = O * (kFp8 ? p.v_scale : 1.f);
          if (d == 0) {
            float* ml = ml_dest(s);
            ml[2 * row] = M * kLn2;
            ml[2 * row + 1] = L;
          }
        }
      } else {
        const int64_t srow = slot * G + hd;
        p.ws_acc[srow * D + d] = O;
        if (d == 0) {
          p.ws_ml[2 * srow] = M;
          p.ws_ml[2 * srow + 1] = L;
        }
      }
    }
    if constexpr (kAppend) {
      if (complete) append_store<D>(p, pair, clamped_len(p, pair / Hkv), tid, kCT);
    }
    bar();  // fl_* reads done before the merge scratch (aliased) is used
    if (!complete)
      commit(pair, toff, nt_q,
             (thief ? (1ull << 32) : (1ull << 48)) + static_cast<unsigned long long>(tiles));
    reset_state();
  };

  const int64_t pair_first = t0 < t1 ? first_w.b * Hkv + first_w.h : 0;
  const int64_t pair_last = t0 < t1 ? last_w.b * Hkv + last_w.h : -1;
  // The own phase visits the rotated pair (if any) first, then pairs in
  // increasing order; owner slots of pairs it never saw get empty states.
  const int64_t rot_pair = (t0 < t1 && rot_of(t1 - t0, last_w) > 0) ? pair_last : -1;
  int64_t inc_next = pair_first;
  const int64_t inc_last = rot_pair >= 0 ? pair_last - 1 : pair_last;
  int64_t cur_pair = -1, cur_count = 0, cur_nt = 0, cur_toff = 0;
  bool thief_phase = false;
  Walk gen = first_w;  // generic path: next own tile
  int64_t gen_t = t0;
  bool gen_end_own = false;
  reset_state();

  for (int64_t k = 0;; ++k) {
    const int s = kTma ? static_cast<int>(k % kStages) : 0;
    const uint8_t* st = ring + static_cast<size_t>(s) * C::kStageBytes;
    TileMeta m;
    if constexpr (kTma) {
      ADB_TRACE_ONLY(const uint64_t tr_c0 = global_timer_ns();)
      if (!mbar_wait(full_bar(s), static_cast<uint32_t>(k / kStages) & 1u, abort_flag)) break;
      m = meta[s];
      ADB_TRACE_ONLY(tr_c1 = global_timer_ns(); tr_cwait += tr_c1 - tr_c0; if (k == 0) tr_first = tr_c1;)
    } else {
      // Generic path (K/V not 16-byte aligned): no producer and no stealing;
      // every warp copies its own rows with 2-byte loads into the same
      // swizzled layout.
      if (gen_t < t1) {
        m = meta_of(gen, gen_t, kMetaOwn);
        __syncwarp();
        uint8_t* dst = ring;
        const int64_t row0 = (gen.b * Hkv + gen.h) * S + gen.tile * TT;
        const int valid_rows =
            static_cast<int>(min(static_cast<int64_t>(TT), gen.len - gen.tile * TT));
        for (int e = lane; e < 16 * kMB * D; e += 32) {
          const int r = warp * 16 * kMB + e / D, col = e % D;
          uint16_t kx = 0, vx = 0;
          if (r < valid_rows) {
            kx = __ldg(k16 + (row0 + r) * D + col);
            vx = __ldg(v16 + (row0 + r) * D + col);
          }
          const uint32_t off = swz128(r, (col & 63) >> 3) + (col & 7) * 2;
          const int h = col >> 6;
          *reinterpret_cast<uint16_t*>(dst + h * C::kBoxBytes + off) = kx;
          *reinterpret_cast<uint16_t*>(dst + (C::kHalves + h) * C::kBoxBytes + off) = vx;
        }
        __syncwarp();
        ++gen_t;
        if (gen_t < t1) walk_next(gen, p, TT);
      } else {
        m = meta_marker(gen_end_own ? kMetaEndAll : kMetaEndOwn);
        gen_end_own = true;
      }
    }
    auto release = [&]() {
      if constexpr (kTma) {
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar(s));
      }
    };

    if (m.kind == kMetaEndOwn) {
      release();
      ADB_TRACE_ONLY(tr_own = global_timer_ns();)
      if (cur_pair >= 0) flush(cur_pair, false, cur_toff, cur_nt, cur_count);
      flush_empty(inc_next, inc_last);
      cur_pair = -1;
      thief_phase = true;
      continue;
    }
    if (m.kind == kMetaEndAll) {
      release();
      if (cur_pair >= 0) flush(cur_pair, true, cur_toff, cur_nt, cur_count);
      break;
    }
    const int64_t pair = static_cast<int64_t>(m.b) * Hkv + m.h;
    if (pair != cur_pair) {
      if (cur_pair >= 0) flush(cur_pair, thief_phase, cur_toff, cur_nt, cur_count);
      if (!thief_phase && pair != rot_pair) {
        flush_empty(inc_next, pair - 1);
        inc_next = pair + 1;
      }
      cur_pair = pair;
      cur_count = 0;
      cur_nt = m.nt;
      cur_toff = m.tile - m.tile_in_pair;
      load_q(pair);
    }
    const int valid = static_cast<int>(
        min(static_cast<int64_t>(TT),
            static_cast<int64_t>(m.len) - static_cast<int64_t>(m.tile_in_pair) * TT));
    {
      const uint32_t kbase = smem_u32(st);
      const uint32_t vbase = kbase + C::kHalves * C::kBoxBytes;
      // ---- S^T = K . Q^T  (tokens x heads), two accumulation chains
      float sc[kMB][4];
#pragma unroll
      for (int mb = 0; mb < kMB; ++mb) {
        const int tok0 = (warp * kMB + mb) * 16;
        const int row = tok0 + (lane & 7) + ((lane >> 3) & 1) * 8;
        float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
        if constexpr (kFp8) {
          // one 16-byte chunk of an FP8 row is a 16-dim slab: an x4 load
          // covers slabs 2*s2 and 2*s2 + 1 of 16 tokens; each register holds
          // 4 dims of one token, turned into two f16 pairs (exact values;
          // the K and V scales are applied to the scores and the output)
#pragma unroll
          for (int s2 = 0; s2 < kSlabs / 2; ++s2) {
            uint32_t r[4];
            ldsm_x4(kbase + swz128(row, 2 * s2 + (lane >> 4)), r);
            const uint32_t a0[4] = {e4m3_01(r[0]), e4m3_01(r[1]), e4m3_23(r[0]), e4m3_23(r[1])};
            const uint32_t a1[4] = {e4m3_01(r[2]), e4m3_01(r[3]), e4m3_23(r[2]), e4m3_23(r[3])};
            mma_f16_16816(c0, a0, qf[2 * s2][0], qf[2 * s2][1]);
            mma_f16_16816(c1, a1, qf[2 * s2 + 1][0], qf[2 * s2 + 1][1]);
          }
        } else {
#pragma unroll
          for (int j = 0; j < kSlabs; ++j) {
            const int chunk = (j & 3) * 2 + (lane >> 4);
            uint32_t a[4];
            ldsm_x4(kbase + (j >> 2) * C::kBoxBytes + swz128(row, chunk), a);
            if (j & 1)
              mma_bf16_16816(c1, a, qf[j][0], qf[j][1]);
            else
              mma_bf16_16816(c0, a, qf[j][0], qf[j][1]);
          }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int tok = tok0 + g + ((i >> 1) << 3);
          sc[mb][i] = tok < valid ? (c0[i] + c1[i]) * p.scale_log2 : neg_inf();
        }
      }
      // ---- online softmax (per head column 2t and 2t+1)
      float mx0 = neg_inf(), mx1 = neg_inf();
#pragma unroll
      for (int mb = 0; mb < kMB; ++mb) {
        mx0 = fmaxf(mx0, fmaxf(sc[mb][0], sc[mb][2]));
        mx1 = fmaxf(mx1, fmaxf(sc[mb][1], sc[mb][3]));
      }
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
      }
      const float mn0 = fmaxf(m_run[0], mx0), mn1 = fmaxf(m_run[1], mx1);
      const float mu0 = mn0 == neg_inf() ? 0.f : mn0;
      const float mu1 = mn1 == neg_inf() ? 0.f : mn1;
      const float al0 = fast_exp2(m_run[0] - mu0), al1 = fast_exp2(m_run[1] - mu1);
      m_run[0] = mn0;
      m_run[1] = mn1;
      float ps0 = 0.f, ps1 = 0.f;
      uint32_t pb[kMB][2];
#pragma unroll
      for (int mb = 0; mb < kMB; ++mb) {
        const float p0 = fast_exp2(sc[mb][0] - mu0), p1 = fast_exp2(sc[mb][1] - mu1);
        const float p2 = fast_exp2(sc[mb][2] - mu0), p3 = fast_exp2(sc[mb][3] - mu1);
        ps0 += p0 + p2;
        ps1 += p1 + p3;
        if constexpr (kFp8) {
          pb[mb][0] = movmatrix_trans(pack_f16x2(p0, p1));
          pb[mb][1] = movmatrix_trans(pack_f16x2(p2, p3));
        } else {
          pb[mb][0] = movmatrix_trans(pack_bf16x2(p0, p1));
          pb[mb][1] = movmatrix_trans(pack_bf16x2(p2, p3));
        }
      }
      l_run[0] = l_run[0] * al0 + ps0;
      l_run[1] = l_run[1] * al1 + ps1;
#pragma unroll
      for (int j = 0; j < kSlabs; ++j) {
        acc[j][0] *= al0;
        acc[j][1] *= al1;
        acc[j][2] *= al0;
        acc[j][3] *= al1;
      }
      // ---- O^T += V^T . P^T  (dims x heads)
#pragma unroll
      for (int mb = 0; mb < kMB; ++mb) {
        const int tok0 = (warp * kMB + mb) * 16;
        const int row = tok0 + (lane & 7) + (lane >> 4) * 8;
        uint32_t keep01 = 0xffffffffu, keep23 = 0xffffffffu;
        if (valid < TT) {  // zero V of tokens past the end (may be stale or NaN padding)
          const int ta = tok0 + 2 * t, tb = tok0 + 8 + 2 * t;
          keep01 = (ta < valid ? 0x0000ffffu : 0u) | (ta + 1 < valid ? 0xffff0000u : 0u);
          keep23 = (tb < valid ? 0x0000ffffu : 0u) | (tb + 1 < valid ? 0xffff0000u : 0u);
        }
        if constexpr (kFp8) {
          // transposed 16-bit loads of the FP8 V tile: a register holds
          // dims (2g, 2g+1) of tokens (2t, 2t+1); regrouped by token pair per
          // dim, MMA row g of slab j is dim 16j + 2g and row g + 8 is
          // 16j + 2g + 1 (the flush writes the accumulator back that way)
          const int rowk = tok0 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
          for (int s2 = 0; s2 < kSlabs / 2; ++s2) {
            uint32_t r[4];
            ldsm_x4_trans(vbase + swz128(rowk, 2 * s2 + (lane >> 4)), r);
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
              uint32_t a[4] = {e4m3_02(r[2 * h2]), e4m3_13(r[2 * h2]), e4m3_02(r[2 * h2 + 1]),
                               e4m3_13(r[2 * h2 + 1])};
              a[0] &= keep01;
              a[1] &= keep01;
              a[2] &= keep23;
              a[3] &= keep23;
              mma_f16_16816(acc[2 * s2 + h2], a, pb[mb][0], pb[mb][1]);
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < kSlabs; ++j) {
            const int chunk = (j & 3) * 2 + ((lane >> 3) & 1);
            uint32_t a[4];
            ldsm_x4_trans(vbase + (j >> 2) * C::kBoxBytes + swz128(row, chunk), a);
            a[0] &= keep01;
            a[1] &= keep01;
            a[2] &= keep23;
            a[3] &= keep23;
            mma_bf16_16816(acc[j], a, pb[mb][0], pb[mb][1]);
          }
        }
      }
    }
    release();
    ++cur_count;
    ADB_TRACE_ONLY(if (thief_phase) ++tr_other_tiles; else ++tr_own_tiles; tr_cbusy += global_timer_ns() - tr_c1;)
  }

  // ------------------------------------------------------------ exit
  // Without work stealing and without a peer exchange the only header state
  // a call touches is the per-pair commit counters, which their completing
  // commits zero (above), so a CTA just exits.  Otherwise the last CTA to
  // finish resets the scheduler header for the next call and, with a peer
  // exchange, publishes this call's states to every rank: each CTA's stores
  // (peer ones included) are released at GPU scope before it counts itself
  // finished; the last CTA, having observed every count, fences at system
  // scope and raises the flags, which releases them all.  (The diagnostic
  // build always counts, to number its launches.)
#ifdef ADB_TRACE
  if (tid == 0 && c < kTraceCtas) {
    unsigned long long* r = g_adb_trace[g_adb_trace_launch & 1u][c];
    r[0] = static_cast<unsigned long long>(smid()) | (static_cast<unsigned long long>(c) << 32);
    r[1] = tr_entry;
    r[2] = tr_wait;
    r[3] = tr_first;
    r[4] = tr_own;
    r[5] = global_timer_ns();
    r[6] = tr_own_tiles | (static_cast<unsigned long long>(tr_other_tiles) << 32);
    r[7] = tr_merges | (tr_merge_ns << 16);
    r[11] = tr_cwait;
    r[12] = tr_cbusy;
  }
#endif
#ifdef ADB_TRACE
  constexpr bool kCountAlways = true;
#else
  constexpr bool kCountAlways = false;
#endif
  if (!(kExchange || kCountAlways || steal)) return;
  __threadfence();
  bar();
  if (tid == 0) misc[46] = atomicAdd(p.ws_counters + 1, 1u) == static_cast<uint32_t>(nc - 1);
  bar();
  if (misc[46]) {
    __threadfence();
    if (tid == 0) misc[47] = dyn_in_use();
    bar();
    const int64_t n_dyn = misc[47];
    for (int64_t i = tid; i < nc; i += kCT) p.ws_claims[i] = 0ull;
    for (int64_t i = tid; i < P; i += kCT) p.ws_done[i] = 0ull;
    for (int64_t i = tid; i < n_dyn; i += kCT) p.ws_slot_pair[i] = 0u;
    bar();
    if (tid == 0) {
      p.ws_counters[0] = 0u;
      p.ws_counters[1] = 0u;
#ifdef ADB_TRACE
      g_adb_launch_log[g_adb_trace_launch & 255u][1] = global_timer_ns();
      g_adb_launch_log[(g_adb_trace_launch + 1u) & 255u][0] = ~0ull;
      g_adb_trace_launch += 1u;
#endif
      if constexpr (kExchange) {
        ADB_TRACE_ONLY(const unsigned tr_l = (g_adb_trace_launch - 1u) & 255u; g_adb_launch_log[tr_l][2] = global_timer_ns();)
        // release pattern: one system-scope fence, then the flags
        fence_acq_rel_sys();
        const uint32_t call = x_epoch(p) + 1u;
        for (int s = 0; s < p.x_world; ++s)
          st_relaxed_sys_u32(
              reinterpret_cast<uint32_t*>(p.x_base[s] + kXFlagsOffset) + p.x_rank, call);
        *reinterpret_cast<volatile uint32_t*>(p.x_base[p.x_rank] + kXEpochOffset) = call;
        ADB_TRACE_ONLY(g_adb_launch_log[tr_l][3] = global_timer_ns();)
      }
    }
  }
  // Fused merge: CTAs 0..x_mergers-1 (each a share of the rows) wait for
  // every rank's flag of this call in this rank's buffer -- this rank's own
  // flag is raised by its last CTA above -- and merge the `world` states of
  // each row.  Ranks run on distinct GPUs (the host guarantees it), and every
  // CTA of this persistent grid is resident, so each wait ends; it is also
  // bounded by x_timeout_ns (zero rows and the device error bit after it).
  if constexpr (kExchange) {
    if (p.x_mergers > 0 && c < p.x_mergers) {
      const uint32_t call = static_cast<uint32_t>(misc[53]);
      const uint8_t* xbuf = p.x_base[p.x_rank];
      if (tid == 0) {
        const uint32_t* flags = reinterpret_cast<const uint32_t*>(xbuf + kXFlagsOffset);
        int ok = 1;
        const uint64_t start = global_timer_ns();
        for (int s = 0; s < p.x_world && ok; ++s) {
          // flags only grow; a rank one call ahead has already passed `call`
          while (static_cast<int32_t>(ld_relaxed_sys_u32(flags + s) - call) < 0) {
            if (global_timer_ns() - start > p.x_timeout_ns) {
              ok = 0;
              atomicOr(&g_adb_error_flag, kErrPeerTimeout);
              break;
            }
            __nanosleep(32);
          }
        }
        if (ok) fence_acq_rel_sys();  // acquire pattern: the flags, then one fence
        misc[54] = ok;
      }
      bar();
      const int64_t rows = P * G;
      const int64_t r0 = c * rows / p.x_mergers, r1 = (c + 1) * rows / p.x_mergers;
      const int64_t par = call & 1u;
      const float* xacc = reinterpret_cast<const float*>(xbuf + kXAccOffset) + par * p.x_world * rows * D;
      const float* xml = reinterpret_cast<const float*>(xbuf + x_ml_offset(p.x_world, rows, D)) +
                         par * p.x_world * rows * 2;
      for (int64_t row = r0 + warp; row < r1; row += kWarps) {
        if (misc[54]) {
          merge_row_few<D>(xacc, rows * D, xml, rows * 2, p.x_world, row, p.x_out, lane);
        } else {
          for (int d = lane; d < D; d += 32) p.x_out[row * D + d] = __float2bfloat16_rn(0.f);
        }
      }
    }
  }
}

// Merges `parts` partial states (m in natural units) of one row into BF16;
// called by one warp.  Replaces merge_splits (csrc/decode.cu:169-184) for the
// cross-GPU merge of sequence shards.
template <int D>
__device__ __forceinline__ void merge_row(const float* __restrict__ acc, int64_t acc_stride,
                                          const float* __restrict__ ml, int64_t ml_stride,
                                          int64_t parts, int64_t row, __nv_bfloat16* __restrict__ out,
                                          int lane) {
  constexpr int kPer = D / 32;
  constexpr float kLog2e = 1.4426950408889634f;
  float M = neg_inf();
  for (int64_t r = lane; r < parts; r += 32)
    if (__ldcg(ml + r * ml_stride + 2 * row + 1) > 0.f) M = fmaxf(M, __ldcg(ml + r * ml_stride + 2 * row));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  const float Mu = M == neg_inf() ? 0.f : M;
  float L = 0.f, O[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) O[i] = 0.f;
  for (int64_t r = 0; r < parts; ++r) {
    const float m = __ldcg(ml + r * ml_stride + 2 * row);
    const float l = __ldcg(ml + r * ml_stride + 2 * row + 1);
    if (!(l > 0.f)) continue;  // empty part: contributes nothing
    const float f = fast_exp2((m - Mu) * kLog2e);
    L += f * l;
    const float* src = acc + r * acc_stride + row * D + lane * kPer;
#pragma unroll
    for (int i = 0; i < kPer; ++i) O[i] += f * __ldcg(src + i);
  }
  __nv_bfloat16* dst = out + row * D + lane * kPer;
#pragma unroll
  for (int i = 0; i < kPer; ++i) dst[i] = __float2bfloat16_rn(L > 0.f ? O[i] / L : 0.f);
}

// Merges `parts` partial states per row.  One warp per row.
template <int D>
__global__ void __launch_bounds__(256)
    merge_states_kernel(const float* __restrict__ acc, int64_t acc_stride,
                        const float* __restrict__ ml, int64_t ml_stride, int64_t parts,
                        int64_t rows, __nv_bfloat16* __restrict__ out) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  if (parts <= kMaxRanks)
    merge_row_few<D>(acc, acc_stride, ml, ml_stride, static_cast<int>(parts), row, out, threadIdx.x & 31);
  else
    merge_row<D>(acc, acc_stride, ml, ml_stride, parts, row, out, threadIdx.x & 31);
}

// The merge step of a peer exchange (see the layout above), on one rank:
// waits, bounded by `timeout_ns`, until every rank has delivered the call
// this rank's decode just completed, then merges the `world` slots of that
// call's parity per row.  Launched behind the decode kernel with
// programmatic serialisation; nothing is read before that grid is done.  If
// the wait gives up, the device error word gets kErrPeerTimeout and the rows
// are written as zeros.
template <int D>
__global__ void __launch_bounds__(256)
    exchange_merge_kernel(const uint8_t* __restrict__ xbuf, int world, int64_t rows,
                          __nv_bfloat16* __restrict__ out, uint64_t timeout_ns) {
  griddep_launch_dependents();
  griddep_wait();
  __shared__ int ready;
  const uint32_t call = *reinterpret_cast<const volatile uint32_t*>(xbuf + kXEpochOffset);
  ADB_TRACE_ONLY(if (blockIdx.x == 0 && threadIdx.x == 0) g_adb_merge_log[call & 255u][0] = global_timer_ns();)
  if (threadIdx.x == 0) {
    const uint32_t* flags = reinterpret_cast<const uint32_t*>(xbuf + kXFlagsOffset);
    int ok = 1;
    const uint64_t start = global_timer_ns();
    for (int s = 0; s < world && ok; ++s) {
      // Flags only grow; a rank one call ahead has already passed `call`.
      while (static_cast<int32_t>(ld_relaxed_sys_u32(flags + s) - call) < 0) {
        if (global_timer_ns() - start > timeout_ns) {
          ok = 0;
          atomicOr(&g_adb_error_flag, kErrPeerTimeout);
          break;
        }
        __nanosleep(64);
      }
    }
    if (ok) fence_acq_rel_sys();  // acquire pattern: the flags, then one fence
    ready = ok;
    ADB_TRACE_ONLY(if (blockIdx.x == 0) g_adb_merge_log[call & 255u][1] = global_timer_ns();)
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  if (!ready) {
    for (int d = lane; d < D; d += 32) out[row * D + d] = __float2bfloat16_rn(0.f);
    return;
  }
  const int64_t par = call & 1u;
  const float* acc = reinterpret_cast<const float*>(xbuf + kXAccOffset) + par * world * rows * D;
  const float* ml = reinterpret_cast<const float*>(xbuf + x_ml_offset(world, rows, D)) + par * world * rows * 2;
  merge_row_few<D>(acc, rows * D, ml, rows * 2, world, row, out, lane);
  ADB_TRACE_ONLY(if (blockIdx.x == 0 && threadIdx.x == 0) g_adb_merge_log[call & 255u][2] = global_timer_ns();)
}

}  // namespace adb
