// decode_kernels.cuh -- BF16 split-K attention-decode kernels for sm_100a.
//
// Work decomposition (replaces the reference's fixed 256-token split grid,
// csrc/decode.cu:193-211):
//   * A "pair" is one (batch, kv_head); its KV rows are contiguous in HBM at
//     row offset pair * S of the [B*Hkv*S, D] view.  Pair p has L_p valid
//     tokens (S, or seqlens[b]) cut into nt_p = ceil(L_p / TT) tiles of TT
//     tokens.  All tiles of all pairs form one flattened tile space of NT
//     tiles, and persistent CTA c of Nc streams the contiguous range
//     [c*NT/Nc, (c+1)*NT/Nc).  Every CTA therefore moves the same number of
//     bytes (+-1 tile) whatever B, Hkv and S are.
//   * The part of a pair covered by one CTA is a "segment".  A segment that
//     covers its whole pair is normalised and written as BF16 directly; any
//     other segment writes an FP32 state (acc[G][D], m, l) into workspace
//     slot (c + p) -- unique because both c and p are non-decreasing along
//     the flattened space -- and the combine kernel merges the slots
//     first_cta(p)+p .. last_cta(p)+p of each split pair.
//
// Partial kernel (replaces decode_bf16_mma, csrc/decode.cu:70-167):
//   * one producer warp issues 3-D TMA tiled loads (cp.async.bulk.tensor,
//     128-byte swizzle, no multicast) of the K and V tiles into a kStages
//     deep shared-memory ring with full/empty mbarriers;
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

struct DecodeParams {
  const __nv_bfloat16* q;  // [B*Hq, D]
  const __nv_bfloat16* k;  // [B*Hkv*S, D]
  const __nv_bfloat16* v;  // [B*Hkv*S, D]
  const int32_t* seqlens;  // [B] or nullptr (all sequences have S tokens)
  __nv_bfloat16* out;      // final mode: [B*Hq, D]
  float* state_acc;        // partial mode: [B*Hq, D]
  float* state_ml;         // partial mode: [B*Hq, 2]  (m natural units, l)
  float* ws_acc;           // [(Nc + P) * G, D]
  float* ws_ml;            // [(Nc + P) * G, 2]        (m log2 units, l)
  int64_t* ws_cum;         // varlen: [B + 1] exclusive tile prefix per batch, [B] = NT
  int64_t batch;
  int64_t kv_heads;
  int64_t kv_len;
  int group;
  int partial_mode;
  int num_ctas;
  int tile_tokens;
  float scale_log2;  // log2(e) / sqrt(D)
};

__device__ __forceinline__ float neg_inf() { return __int_as_float(0xff800000); }

__device__ __forceinline__ int32_t clamped_len(const DecodeParams& p, int64_t b) {
  if (p.seqlens == nullptr) return static_cast<int32_t>(p.kv_len);
  int32_t len = __ldg(p.seqlens + b);
  if (len < 0) len = 0;
  if (len > p.kv_len) len = static_cast<int32_t>(p.kv_len);
  return len;
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
  w.nt = (static_cast<int64_t>(w.len) + tt - 1) / tt;
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

template <int D, int kWarps, int kMB, int kStages, bool kTma>
struct StreamCfg {
  static constexpr int kTT = 16 * kWarps * kMB;  // tokens per tile
  static constexpr int kHalves = D / 64;         // 64-column (128-byte) swizzle atoms per row
  static constexpr int kBoxBytes = kTT * 128;    // one TMA box: kTT rows x 128 B
  static constexpr int kStageBytes = 2 * kHalves * kBoxBytes;  // K and V
  static constexpr int kRingStages = kTma ? kStages : 1;
  static constexpr int kThreads = (kWarps + (kTma ? 1 : 0)) * 32;
  static constexpr int kConsumerThreads = kWarps * 32;
  static constexpr int kRingBytes = kRingStages * kStageBytes;
  static constexpr int kFlushAccBytes = kWarps * kMaxGroup * D * 4;
  static constexpr int kFlushMlBytes = kWarps * kMaxGroup * 2 * 4;
  static constexpr int kBarBytes = 2 * kRingStages * 8;
  static constexpr int kMiscBytes = 48 * 8;
  static constexpr int kSmemBytes =
      1024 + kRingBytes + kFlushAccBytes + kFlushMlBytes + kBarBytes + kMiscBytes;
  static_assert(D == 64 || D == 128, "head_dim");
  static_assert(kTT <= 256, "TMA box rows");
  static_assert(kBoxBytes % 1024 == 0, "128B-swizzle boxes must stay 1024-byte aligned");
};

// Byte offset of the 16-byte chunk `chunk` (0..7) of row `row` inside a
// 128-byte-swizzled box (the layout CU_TENSOR_MAP_SWIZZLE_128B writes).
__device__ __forceinline__ uint32_t swz128(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

template <int D, int kWarps, int kMB, int kStages, bool kTma>
__global__ void __launch_bounds__(StreamCfg<D, kWarps, kMB, kStages, kTma>::kThreads, 1)
    decode_stream_kernel(const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const DecodeParams p) {
  using C = StreamCfg<D, kWarps, kMB, kStages, kTma>;
  constexpr int TT = C::kTT;
  constexpr int kSlabs = D / 16;

  extern __shared__ uint8_t smem_raw[];
  // 128-byte-swizzled TMA boxes need 1024-byte aligned shared addresses.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* ring = smem;
  float* fl_acc = reinterpret_cast<float*>(smem + C::kRingBytes);  // [kWarps][8][D]
  float* fl_m = fl_acc + kWarps * kMaxGroup * D;                    // [kWarps][8]
  float* fl_l = fl_m + kWarps * kMaxGroup;                          // [kWarps][8]
  uint64_t* bars = reinterpret_cast<uint64_t*>(fl_l + kWarps * kMaxGroup);
  int64_t* misc = reinterpret_cast<int64_t*>(bars + 2 * C::kRingStages);
  // misc[0..32]: scan scratch; misc[40]: start batch; misc[41]: its tile base;
  // misc[42]: abort flag (int)
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 42);

  // The combine kernel is launched with programmatic stream serialisation;
  // it blocks in griddepcontrol.wait until this grid has completed.
  griddep_launch_dependents();

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t B = p.batch, Hkv = p.kv_heads, S = p.kv_len;
  const int64_t nc = gridDim.x, c = blockIdx.x;

  // ------------------------------------------------------------ tile range
  int64_t nt_total, t0, t1;
  Walk start;
  start.tile = 0;
  if (p.seqlens == nullptr) {
    const int64_t nt = (S + TT - 1) / TT;
    nt_total = B * Hkv * nt;
    t0 = c * nt_total / nc;
    t1 = (c + 1) * nt_total / nc;
    if (t0 >= t1) return;
    const int64_t pair = t0 / nt;
    start.b = pair / Hkv;
    start.h = pair - start.b * Hkv;
    start.tile = t0 - pair * nt;
    start.nt = nt;
    start.len = static_cast<int32_t>(S);
  } else {
    // Pass 1: total tiles.  Pass 2: the batch holding tile t0 (and, in CTA 0,
    // the per-batch tile prefix the combine kernel reads).
    int64_t local = 0;
    for (int64_t b = tid; b < B; b += blockDim.x)
      local += Hkv * ((static_cast<int64_t>(clamped_len(p, b)) + TT - 1) / TT);
    int64_t total = 0;
    block_inclusive_scan(local, misc, total);
    nt_total = total;
    t0 = nt_total > 0 ? c * nt_total / nc : 0;
    t1 = nt_total > 0 ? (c + 1) * nt_total / nc : 0;
    if (tid == 0) misc[40] = -1;
    __syncthreads();
    const bool writer = (c == 0);
    if (t0 < t1 || writer) {
      int64_t running = 0;
      for (int64_t base = 0; base < B; base += blockDim.x) {
        const int64_t b = base + tid;
        const int64_t x =
            b < B ? Hkv * ((static_cast<int64_t>(clamped_len(p, b)) + TT - 1) / TT) : 0;
        int64_t chunk_total = 0;
        const int64_t incl = block_inclusive_scan(x, misc, chunk_total);
        const int64_t excl = running + incl - x;
        if (b < B) {
          if (writer) p.ws_cum[b] = excl;
          if (x > 0 && excl <= t0 && t0 < excl + x) {
            misc[40] = b;
            misc[41] = excl;
          }
        }
        running += chunk_total;
        __syncthreads();
        if (!writer && misc[40] >= 0) break;
      }
      if (writer && tid == 0) p.ws_cum[B] = running;
    }
    if (t0 >= t1) return;
    const int64_t b0 = misc[40];
    const int64_t base0 = misc[41];
    walk_set_batch(start, p, b0, TT);
    const int64_t r = t0 - base0;
    start.h = r / start.nt;
    start.tile = r - start.h * start.nt;
  }
  const int64_t n_tiles = t1 - t0;

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
  __syncthreads();

  // ------------------------------------------------------------ producer
  if constexpr (kTma) {
    if (warp == kWarps) {
      if (lane == 0) {
        Walk w = start;
        for (int64_t k = 0; k < n_tiles; ++k) {
          const int s = static_cast<int>(k % kStages);
          if (k >= kStages) {
            if (!mbar_wait(empty_bar(s), static_cast<uint32_t>((k / kStages) - 1) & 1u,
                           abort_flag))
              break;
          }
          mbar_arrive_expect_tx(full_bar(s), C::kStageBytes);
          uint8_t* st = ring + static_cast<size_t>(s) * C::kStageBytes;
          const int y = static_cast<int>(w.tile * TT);
          const int z = static_cast<int>(w.b * Hkv + w.h);
#pragma unroll
          for (int h = 0; h < C::kHalves; ++h)
            tma_load_3d(smem_u32(st + h * C::kBoxBytes), &tm_k, h * 64, y, z, full_bar(s));
#pragma unroll
          for (int h = 0; h < C::kHalves; ++h)
            tma_load_3d(smem_u32(st + (C::kHalves + h) * C::kBoxBytes), &tm_v, h * 64, y, z,
                        full_bar(s));
          walk_next(w, p, TT);
        }
      }
      return;
    }
  }

  // ------------------------------------------------------------ consumers
  const int g = lane >> 2, t = lane & 3;
  const int G = p.group;
  const uint16_t* q16 = reinterpret_cast<const uint16_t*>(p.q);
  const uint16_t* k16 = reinterpret_cast<const uint16_t*>(p.k);
  const uint16_t* v16 = reinterpret_cast<const uint16_t*>(p.v);

  uint32_t qf[kSlabs][2];
  auto load_q = [&](int64_t pair) {
    if (g < G) {
      const uint16_t* row = q16 + (pair * G + g) * D;
#pragma unroll
      for (int j = 0; j < kSlabs; ++j) {
        qf[j][0] = pack_u16x2(__ldg(row + 16 * j + 2 * t), __ldg(row + 16 * j + 2 * t + 1));
        qf[j][1] =
            pack_u16x2(__ldg(row + 16 * j + 8 + 2 * t), __ldg(row + 16 * j + 8 + 2 * t + 1));
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

  Walk w = start;
  int64_t seg_first_tile = w.tile;
  load_q(w.b * Hkv + w.h);
  reset_state();

  for (int64_t k = 0; k < n_tiles; ++k) {
    const int s = kTma ? static_cast<int>(k % kStages) : 0;
    const uint8_t* st = ring + static_cast<size_t>(s) * C::kStageBytes;
    const int64_t tile_tok0 = w.tile * TT;
    const int valid =
        static_cast<int>(min(static_cast<int64_t>(TT), static_cast<int64_t>(w.len) - tile_tok0));
    bool have_data = true;
    if constexpr (kTma) {
      have_data = mbar_wait(full_bar(s), static_cast<uint32_t>(k / kStages) & 1u, abort_flag);
    } else {
      // Generic path for K/V that are not 16-byte aligned: every warp copies
      // its own rows with 2-byte loads into the same swizzled layout.
      __syncwarp();
      uint8_t* dst = ring;
      const int64_t row0 = (w.b * Hkv + w.h) * S + tile_tok0;
      for (int e = lane; e < 16 * kMB * D; e += 32) {
        const int r = warp * 16 * kMB + e / D, col = e % D;
        uint16_t kx = 0, vx = 0;
        if (r < valid) {
          kx = __ldg(k16 + (row0 + r) * D + col);
          vx = __ldg(v16 + (row0 + r) * D + col);
        }
        const uint32_t off = swz128(r, (col & 63) >> 3) + (col & 7) * 2;
        const int h = col >> 6;
        *reinterpret_cast<uint16_t*>(dst + h * C::kBoxBytes + off) = kx;
        *reinterpret_cast<uint16_t*>(dst + (C::kHalves + h) * C::kBoxBytes + off) = vx;
      }
      __syncwarp();
    }

    if (have_data) {
      const uint32_t kbase = smem_u32(st);
      const uint32_t vbase = kbase + C::kHalves * C::kBoxBytes;
      // ---- S^T = K . Q^T  (tokens x heads), two accumulation chains
      float sc[kMB][4];
#pragma unroll
      for (int mb = 0; mb < kMB; ++mb) {
        const int tok0 = (warp * kMB + mb) * 16;
        const int row = tok0 + (lane & 7) + ((lane >> 3) & 1) * 8;
        float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
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
        pb[mb][0] = movmatrix_trans(pack_bf16x2(p0, p1));
        pb[mb][1] = movmatrix_trans(pack_bf16x2(p2, p3));
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
    if constexpr (kTma) {
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_bar(s));
    }

    // ---- segment end: merge the kWarps states and write the result
    const bool last_in_pair = (w.tile == w.nt - 1);
    if (last_in_pair || k == n_tiles - 1) {
      const bool complete = (seg_first_tile == 0) && last_in_pair;
      const int64_t pair = w.b * Hkv + w.h;
      float lr0 = l_run[0], lr1 = l_run[1];
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        lr0 += __shfl_xor_sync(0xffffffffu, lr0, o);
        lr1 += __shfl_xor_sync(0xffffffffu, lr1, o);
      }
      if (g == 0) {
        fl_m[warp * kMaxGroup + 2 * t] = m_run[0];
        fl_m[warp * kMaxGroup + 2 * t + 1] = m_run[1];
        fl_l[warp * kMaxGroup + 2 * t] = lr0;
        fl_l[warp * kMaxGroup + 2 * t + 1] = lr1;
      }
      float* wa = fl_acc + warp * kMaxGroup * D;
#pragma unroll
      for (int j = 0; j < kSlabs; ++j) {
        wa[(2 * t) * D + 16 * j + g] = acc[j][0];
        wa[(2 * t + 1) * D + 16 * j + g] = acc[j][1];
        wa[(2 * t) * D + 16 * j + 8 + g] = acc[j][2];
        wa[(2 * t + 1) * D + 16 * j + 8 + g] = acc[j][3];
      }
      named_barrier_sync(1, C::kConsumerThreads);
      for (int e = tid; e < G * D; e += C::kConsumerThreads) {
        const int hd = e / D, d = e - hd * D;
        float M = neg_inf();
#pragma unroll
        for (int ww = 0; ww < kWarps; ++ww) M = fmaxf(M, fl_m[ww * kMaxGroup + hd]);
        const float Mu = M == neg_inf() ? 0.f : M;
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int ww = 0; ww < kWarps; ++ww) {
          const float f = fast_exp2(fl_m[ww * kMaxGroup + hd] - Mu);
          L += f * fl_l[ww * kMaxGroup + hd];
          O += f * fl_acc[(ww * kMaxGroup + hd) * D + d];
        }
        const int64_t row = pair * G + hd;
        if (complete && !p.partial_mode) {
          p.out[row * D + d] = __float2bfloat16_rn(L > 0.f ? O / L : 0.f);
        } else if (complete) {
          p.state_acc[row * D + d] = O;
          if (d == 0) {
            p.state_ml[2 * row] = M * kLn2;
            p.state_ml[2 * row + 1] = L;
          }
        } else {
          const int64_t srow = (c + pair) * G + hd;
          p.ws_acc[srow * D + d] = O;
          if (d == 0) {
            p.ws_ml[2 * srow] = M;
            p.ws_ml[2 * srow + 1] = L;
          }
        }
      }
      named_barrier_sync(1, C::kConsumerThreads);
      reset_state();
    }
    if (k + 1 < n_tiles) {
      const int64_t old_pair = w.b * Hkv + w.h;
      walk_next(w, p, TT);
      const int64_t new_pair = w.b * Hkv + w.h;
      if (new_pair != old_pair) {
        load_q(new_pair);
        seg_first_tile = w.tile;
      }
    }
  }
}

// Merges the workspace segments of every split (pair, head) row.  One warp
// per output row; rows whose pair lies inside one CTA were written by the
// partial kernel and are skipped.  Replaces merge_splits
// (csrc/decode.cu:169-184).
template <int D>
__global__ void __launch_bounds__(256) combine_segments_kernel(const DecodeParams p) {
  griddep_wait();
  constexpr int kPer = D / 32;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int G = p.group;
  const int64_t Hkv = p.kv_heads;
  const int64_t P = p.batch * Hkv;
  if (row >= P * G) return;
  const int64_t pair = row / G;
  const int hd = static_cast<int>(row - pair * G);
  const int64_t b = pair / Hkv, h = pair - b * Hkv;
  const int tt = p.tile_tokens;
  int64_t nt, toff, nt_total;
  if (p.seqlens == nullptr) {
    nt = (p.kv_len + tt - 1) / tt;
    toff = pair * nt;
    nt_total = P * nt;
  } else {
    nt = (static_cast<int64_t>(clamped_len(p, b)) + tt - 1) / tt;
    toff = p.ws_cum[b] + h * nt;
    nt_total = p.ws_cum[p.batch];
  }
  float* out_acc = p.partial_mode ? p.state_acc + row * D : nullptr;
  if (nt == 0) {  // empty sequence: zero output / empty state
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int d = lane * kPer + i;
      if (p.partial_mode)
        out_acc[d] = 0.f;
      else
        p.out[row * D + d] = __float2bfloat16_rn(0.f);
    }
    if (p.partial_mode && lane == 0) {
      p.state_ml[2 * row] = neg_inf();
      p.state_ml[2 * row + 1] = 0.f;
    }
    return;
  }
  const int64_t nc = p.num_ctas;
  const int64_t first = cta_of_tile(toff, nt_total, nc);
  const int64_t last = cta_of_tile(toff + nt - 1, nt_total, nc);
  if (first == last) return;
  // With variable lengths there can be more CTAs than tiles; CTAs with an
  // empty range wrote no segment and are skipped.
  auto empty_cta = [&](int64_t cc) { return cc * nt_total / nc == (cc + 1) * nt_total / nc; };
  float M = neg_inf();
  for (int64_t cc = first; cc <= last; ++cc)
    if (!empty_cta(cc)) M = fmaxf(M, p.ws_ml[2 * ((cc + pair) * G + hd)]);
  const float Mu = M == neg_inf() ? 0.f : M;
  float L = 0.f, O[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) O[i] = 0.f;
  for (int64_t cc = first; cc <= last; ++cc) {
    if (empty_cta(cc)) continue;
    const int64_t srow = (cc + pair) * G + hd;
    const float f = fast_exp2(p.ws_ml[2 * srow] - Mu);
    L += f * p.ws_ml[2 * srow + 1];
    const float* src = p.ws_acc + srow * D + lane * kPer;
    if constexpr (kPer == 4) {
      const float4 x = *reinterpret_cast<const float4*>(src);
      O[0] += f * x.x;
      O[1] += f * x.y;
      O[2] += f * x.z;
      O[3] += f * x.w;
    } else {
      const float2 x = *reinterpret_cast<const float2*>(src);
      O[0] += f * x.x;
      O[1] += f * x.y;
    }
  }
  if (p.partial_mode) {
#pragma unroll
    for (int i = 0; i < kPer; ++i) out_acc[lane * kPer + i] = O[i];
    if (lane == 0) {
      p.state_ml[2 * row] = M * kLn2;
      p.state_ml[2 * row + 1] = L;
    }
  } else {
    __nv_bfloat16* dst = p.out + row * D + lane * kPer;
#pragma unroll
    for (int i = 0; i < kPer; ++i) dst[i] = __float2bfloat16_rn(L > 0.f ? O[i] / L : 0.f);
  }
}

// Merges `parts` public partial states (m in natural units) per row into
// BF16.  One warp per row.
template <int D>
__global__ void __launch_bounds__(256)
    merge_states_kernel(const float* __restrict__ acc, int64_t acc_stride,
                        const float* __restrict__ ml, int64_t ml_stride, int64_t parts,
                        int64_t rows, __nv_bfloat16* __restrict__ out) {
  constexpr int kPer = D / 32;
  constexpr float kLog2e = 1.4426950408889634f;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  float M = neg_inf();
  for (int64_t r = 0; r < parts; ++r) M = fmaxf(M, ml[r * ml_stride + 2 * row]);
  const float Mu = M == neg_inf() ? 0.f : M;
  float L = 0.f, O[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) O[i] = 0.f;
  for (int64_t r = 0; r < parts; ++r) {
    const float m = ml[r * ml_stride + 2 * row];
    const float l = ml[r * ml_stride + 2 * row + 1];
    if (!(l > 0.f)) continue;  // empty part: contributes nothing
    const float f = fast_exp2((m - Mu) * kLog2e);
    L += f * l;
    const float* src = acc + r * acc_stride + row * D + lane * kPer;
#pragma unroll
    for (int i = 0; i < kPer; ++i) O[i] += f * src[i];
  }
  __nv_bfloat16* dst = out + row * D + lane * kPer;
#pragma unroll
  for (int i = 0; i < kPer; ++i) dst[i] = __float2bfloat16_rn(L > 0.f ? O[i] / L : 0.f);
}

}  // namespace adb
