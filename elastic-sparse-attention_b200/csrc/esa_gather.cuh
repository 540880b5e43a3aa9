// Gather kernels (CUDA cores) for elastic sparse attention on sm_100a.
//
// Every (query row, head) pair attends to exactly w keys whose positions are
// computed on the fly from the pattern (no index buffers in HBM).  One warp
// owns one pair at a time.  A key/value row of D elements is read as 16-byte
// vectors by a group of LPR lanes (RPW = 32 / LPR rows per warp load), so
// every load instruction touches whole 128-byte lines.  Dot products are
// finished with a butterfly transpose-reduce that leaves one slot's score per
// lane after LPR - 1 shuffles for a sub-chunk of 32 slots.
//
// Forward   (reference kernel :117-166):  O = softmax(s) V,  s = q.k * scale,
//           plus the base-2 log-sum-exp per row (replaces the reference's
//           separate L = sum exp and M = max outputs, :165-166).
// Backward, query side (reference :169-233 without the atomics): recompute
//           s, p = exp(s - lse), dp = dO.v, dS = p (dp - dO.o); write
//           (p, dS*scale) per (row, slot) to a workspace and dQ = scale dS K.
// Backward, key side: dK_j = sum dS*scale q_i, dV_j = sum p dO_i over the
//           (row i, slot k) users of key j, enumerated through the transposed
//           index: for a fixed head and slot, the key index is non-decreasing
//           in the query position, so the users of key j in one slot column
//           are one contiguous run of query rows, found by binary / galloping
//           search.  No atomics: each key row is owned by one warp.
#pragma once
#include "esa_params.h"

namespace esa {

template <typename T, int D>
struct Layout {
  static constexpr int EPL = Vec<T>::kElems;  // elements per 16-byte vector
  static constexpr int LPR = D / EPL;         // lanes per row
  static constexpr int RPW = 32 / LPR;        // rows per warp load
  static_assert(D % EPL == 0, "head_dim must fill whole 16-byte vectors");
  static_assert(LPR >= 1 && LPR <= 32 && (32 % LPR) == 0, "unsupported head_dim");
};

// Position of query row j: rows[j] (negative entries count back from kv_len,
// like torch indexing of the reference's [:kv_len] slice), or row_offset + j.
// -1 for an entry outside [-kv_len, kv_len): callers mask every slot of it.
__device__ __forceinline__ int query_pos(const AttnParams& p, int j) {
  if (!p.rows) return p.row_offset + j;
  int64_t r = p.rows[j];
  if (r < 0) r += p.kv_len;
  if (r < 0 || r >= p.kv_len) {
    if (p.err) atomicOr(p.err, kErrQueryRange);
    return -1;
  }
  return (int)r;
}

// Fills sidx[0..wpad) with the k/v buffer row of each slot of a pair, -1 for
// masked slots (reference :126-131: causal mask and bounds) and padding.
__device__ __forceinline__ void fill_slot_rows(const AttnParams& p, int pos, int h, int wpad,
                                               int lane, int* sidx) {
  const RowWin rw = row_window(p.pat, pos);
  const float t = head_weight(p.pat, h);
  const float omt = __fsub_rn(1.f, t);
  for (int k = lane; k < wpad; k += 32) {
    int row = -1;
    if (k < p.pat.w && pos >= 0) {
      const int raw = raw_index(rw, k, t, omt);
      if (raw <= pos) {                              // causal mask (:532)
        const int c = min(raw, p.kv_len - 1);        // clamp (:615)
        row = c - p.kv_offset;
        if (row < 0 || row >= p.kv_rows) {
          if (p.err) atomicOr(p.err, kErrKvRange);
          row = -1;
        }
      }
    }
    sidx[k] = row;
  }
}

// ---------------------------------------------------------------------------
// Forward.
// grid = (ceil(n_rows / rows_per_cta), Hkv, B); block = NW warps; the pairs of
// a CTA are its rows x the G query heads of one KV head, head-minor, so the
// warps running together read neighbouring rows of the same K/V head.
// ---------------------------------------------------------------------------
template <typename T, int D, int NW>
__global__ void __launch_bounds__(NW * 32, 2)
fwd_gather_kernel(const AttnParams p, int rows_per_cta) {
  using L = Layout<T, D>;
  using V = Vec<T>;
  using M = Mix<T>;
  using Sc = typename M::Scalar;
  constexpr int EPL = L::EPL, LPR = L::LPR, RPW = L::RPW;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int w = p.pat.w;
  const int wpad = (w + 31) & ~31;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* sidx = reinterpret_cast<int*>(smem_raw) + warp * 3 * wpad;
  float* ssc = reinterpret_cast<float*>(sidx + wpad);
  Sc* sps = reinterpret_cast<Sc*>(ssc + wpad);    // softmax weights in the input type
  const int g = lane / LPR, r = lane % LPR;
  const int hkv = blockIdx.y, b = blockIdx.z;
  const int row0 = blockIdx.x * rows_per_cta;
  const int n_pairs = rows_per_cta * p.G;
  const T* Kb = reinterpret_cast<const T*>(p.k) + b * p.skb + hkv * p.skh + r * EPL;
  const T* Vb = reinterpret_cast<const T*>(p.v) + b * p.svb + hkv * p.svh + r * EPL;

  for (int pr = warp; pr < n_pairs; pr += NW) {
    const int j = row0 + pr / p.G;
    if (j >= p.n_rows) break;
    const int h = hkv * p.G + pr % p.G;
    const int pos = query_pos(p, j);
    fill_slot_rows(p, pos, h, wpad, lane, sidx);

    const uint4 qv = ldg16_stream(reinterpret_cast<const T*>(p.q) + b * p.sqb + h * p.sqh +
                                  (int64_t)j * p.sqs + r * EPL);
    __syncwarp();

    // Scores (base-2 scaled), one slot per lane per sub-chunk of 32 slots.  All
    // LPR row loads of a sub-chunk are issued before the first use.
    float mloc = -INFINITY;
    for (int s0 = 0; s0 < wpad; s0 += 32) {
      uint4 kb[LPR];
#pragma unroll
      for (int m = 0; m < LPR; ++m) {
        const int row = sidx[s0 + m * RPW + g];
        kb[m] = row >= 0 ? ldg16(Kb + (int64_t)row * p.sks) : make_uint4(0, 0, 0, 0);
      }
      float part[LPR];
#pragma unroll
      for (int m = 0; m < LPR; ++m) part[m] = M::dot(qv, kb[m], 0.f);
      transpose_reduce<LPR>(part, lane);
      const int k = s0 + r * RPW + g;
      const float s = sidx[k] >= 0 ? part[0] * p.scale_log2 : -INFINITY;
      ssc[k] = s;
      mloc = fmaxf(mloc, s);
    }
    float mx = warp_max(mloc);
    mx = mx == -INFINITY ? 0.f : mx;
    __syncwarp();
    // Weights rounded to the input type once; the normaliser sums the rounded
    // values so that they add up to one exactly as used.
    float lsum = 0.f;
    for (int k = lane; k < wpad; k += 32) {
      Sc e = M::scalar(exp2f(ssc[k] - mx));
      lsum += M::to_float(e);
      if (p.drop_threshold && k < w)   // dropout acts on the normalised weights (ref :674)
        e = dropout_keep(p, pos, b, h, k) ? M::scalar(M::to_float(e) * p.keep_scale)
                                                   : M::scalar(0.f);
      sps[k] = e;
    }
    const float l = warp_sum(lsum);
    if (p.weights) {   // the naive path's attn_weights (ref :673-674)
      T* wrow = reinterpret_cast<T*>(p.weights) + (((int64_t)b * p.Hq + h) * p.n_rows + j) * w;
      const float inv = l > 0.f ? 1.f / l : 0.f;
      for (int k = lane; k < w; k += 32) wrow[k] = from_f32<T>(M::to_float(sps[k]) * inv);
    }
    __syncwarp();

    float acc[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[e] = 0.f;
    for (int s0 = 0; s0 < wpad; s0 += 32) {
      uint4 vb[LPR];
#pragma unroll
      for (int m = 0; m < LPR; ++m) {
        const int row = sidx[s0 + m * RPW + g];
        vb[m] = row >= 0 ? ldg16(Vb + (int64_t)row * p.svs) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int m = 0; m < LPR; ++m) M::axpy(sps[s0 + m * RPW + g], vb[m], acc);   // 0 when masked
    }
#pragma unroll
    for (int o = LPR; o < 32; o <<= 1)
#pragma unroll
      for (int e = 0; e < EPL; ++e) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], o);
    if (g == 0) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) acc[e] *= inv;
      T* orow = reinterpret_cast<T*>(p.o) + b * p.sob + h * p.soh + (int64_t)j * p.sos + r * EPL;
      stg16(orow, V::from_float(acc));
    }
    if (lane == 0) p.lse[((int64_t)b * p.Hq + h) * p.n_rows + j] = mx + log2f(l);
    __syncwarp();
  }
}

// Rows of slots [kbeg, kbeg + half) of the pair (row j, head h) for the tile
// kernels: the k/v buffer row of a valid slot; for a masked slot (and every
// slot of a padding row j >= n_rows) the pair's slot-0 row, or row 0 when that
// is masked too, with the sign bit set.  The tile kernels then load every
// slot unconditionally from `row & kRowMask` (always inside the buffer) and
// take the sign bit as the mask; a masked slot's weight is 0, and its row is
// one the pair reads anyway, so no value it could not see enters the sums.
constexpr int kMaskBit = int(0x80000000u);
constexpr int kRowMask = 0x7fffffff;

__device__ __forceinline__ void tile_slot_rows(const AttnParams& p, int j, int h, int kbeg,
                                               int half, int* out) {
  if (j >= p.n_rows) {
    for (int k = kbeg; k < kbeg + half; ++k) out[k] = kMaskBit;
    return;
  }
  const int w = p.pat.w;
  const int pos = query_pos(p, j);
  const RowWin rw = row_window(p.pat, pos);
  const float t = head_weight(p.pat, h);
  const float omt = __fsub_rn(1.f, t);
  auto row_of = [&](int k) -> int {   // -1 when masked or outside the buffer
    const int raw = raw_index(rw, k, t, omt);
    if (pos < 0 || raw > pos) return -1;   // causal mask (:532)
    const int row = min(raw, p.kv_len - 1) - p.kv_offset;   // clamp (:615)
    if (row < 0 || row >= p.kv_rows) {
      if (p.err) atomicOr(p.err, kErrKvRange);
      return -1;
    }
    return row;
  };
  const int r0 = row_of(0);
  const int fallback = kMaskBit | (r0 >= 0 ? r0 : 0);
  for (int k = kbeg; k < kbeg + half; ++k) {
    const int row = k < w ? (k == 0 ? r0 : row_of(k)) : -1;
    out[k] = row >= 0 ? row : fallback;
  }
}

// ---------------------------------------------------------------------------
// Forward, slot-major tile variant (16-bit types, w <= 64, G divides 128).
//
// A CTA owns a tile of 128 (query, head) pairs of one KV head: 128/G
// consecutive queries x the G heads.  Warp w owns pairs [16w, 16w + 16); half
// of a warp load serves one pair (RPW = 2 for D = 128).  Unlike
// fwd_gather_kernel, all warps walk the slots together (two slots per
// butterfly), so at any moment the CTA reads the K (then V) rows of the same
// few slots for all 128 pairs: the rows several pairs share (neighbouring
// queries at small dilation, neighbouring heads at any dilation) are served
// from L1 after the first miss.  Scores stay in registers (one pair's 64
// scores live in two lanes), softmax weights go to shared memory in the input
// type, and each half-warp writes its pair's output row without a reduction.
// ---------------------------------------------------------------------------
constexpr int kTilePairs = 128;
constexpr int kTileMaxW = 64;
// Per-pair shared arrays.  The row indices (int) and the 16-bit weights are
// read 2 slots at a time (8-byte / 4-byte loads), so their rows are 68
// elements long: 16- resp. 8-byte aligned, and the two pairs one warp load
// reads (neighbouring pairs) start 4 (2) banks apart, clear of each other.
// The fp32 score rows keep an odd stride of 65 words (read one slot at a
// time by one thread per pair).
constexpr int kTileRowStride = kTileMaxW + 4;
constexpr int kTileIdxStride = kTileMaxW + 1;
constexpr int kTileSpStride = kTileMaxW + 4;
constexpr int kTileSidxBytes = kTilePairs * kTileRowStride * 4;
constexpr int kTileScoreBytes = kTilePairs * kTileIdxStride * 4;
// sidx, fp32 scores (later the weights in the input type), per-pair 1 / sum.
// Kept small: shared memory comes out of the same 256 KB per SM as the L1
// that serves the shared K / V rows.
constexpr int kTileSmemBytes = kTileSidxBytes + kTileScoreBytes + kTilePairs * 4;
static_assert(kTilePairs * kTileSpStride * 2 <= kTileScoreBytes, "weights alias the scores");

// Lane layout of the tile kernels: a 16-bit row of D elements is read by
// LPR = 8 lanes, each taking CPL 16-byte chunks (chunks r and r + 8 of the
// row for lane r of its group): a warp load instruction then covers RPW = 4
// whole 128-byte segments of 4 rows (4 L1 wavefronts for 512 bytes, as with
// one chunk per lane), while a dot product is finished by a butterfly over 8
// lanes (7 shuffles for two slots of the warp's 16 pairs) instead of 16.
template <typename T, int D>
struct TileLayout {
  static constexpr int EPL = Vec<T>::kElems;   // elements per 16-byte chunk
  static constexpr int LPR = 8;                // lanes per row
  static constexpr int CPL = D / (EPL * LPR);  // chunks per lane
  static constexpr int RPW = 32 / LPR;         // rows per warp load
  static_assert(CPL >= 1 && CPL * EPL * LPR == D, "tile kernels take D = 64 or 128 (16-bit)");
};

// Rows of 2 consecutive slots of one pair (one 8-byte shared load).
__device__ __forceinline__ int2 slot_rows2(const int (*sidx)[kTileRowStride], int pi, int k0) {
  return *reinterpret_cast<const int2*>(&sidx[pi][k0]);
}
__device__ __forceinline__ int row2_at(const int2& r, int i) { return i ? r.y : r.x; }
// 2 consecutive 16-bit weights of one pair (one 4-byte shared load).
__device__ __forceinline__ uint32_t weights2(const uint16_t* row, int k0) {
  return *reinterpret_cast<const uint32_t*>(row + k0);
}
__device__ __forceinline__ uint16_t weight2_at(uint32_t u, int i) {
  return static_cast<uint16_t>(i ? (u >> 16) : (u & 0xffffu));
}

template <typename T, int D>
__global__ void __launch_bounds__(256, 2)
fwd_tile_kernel(const AttnParams p) {
  using L = TileLayout<T, D>;
  using V = Vec<T>;
  using M = Mix<T>;
  using Sc = typename M::Scalar;
  constexpr int EPL = L::EPL, LPR = L::LPR, RPW = L::RPW, CPL = L::CPL;
  constexpr int PPW = kTilePairs / 8;      // pairs per warp
  constexpr int MI = PPW / RPW;            // warp loads per slot
  static_assert(MI * 2 == LPR, "two slots per transpose-reduce");
  constexpr int HALF = kTileMaxW / 2;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int(*sidx)[kTileRowStride] = reinterpret_cast<int(*)[kTileRowStride]>(smem_raw);
  // fp32 scores; after the softmax the same bytes hold the weights in the
  // input type, laid out as Sc[kTilePairs][kTileSpStride]
  float(*sbuf)[kTileIdxStride] =
      reinterpret_cast<float(*)[kTileIdxStride]>(smem_raw + kTileSidxBytes);
  Sc(*sp)[kTileSpStride] = reinterpret_cast<Sc(*)[kTileSpStride]>(&sbuf[0][0]);
  float* sl = reinterpret_cast<float*>(smem_raw + kTileSidxBytes + kTileScoreBytes);
  const int w = p.pat.w;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane / LPR, r = lane % LPR;
  const int G = p.G;
  const int TQ = kTilePairs / G;
  const int hkv = blockIdx.y, b = blockIdx.z;
  const int j0 = blockIdx.x * TQ;

  // ---- indices: thread t fills pair t / 2, slots [(t & 1) * 32, +32) ------
  {
    const int pi = threadIdx.x >> 1;
    const int j = j0 + pi / G;
    const int h = hkv * G + pi % G;
    const int kbeg = (threadIdx.x & 1) * HALF;
    tile_slot_rows(p, j, h, kbeg, HALF, &sidx[pi][0]);
  }
  __syncthreads();

  const int pw0 = warp * PPW;   // first pair of this warp
  // lane r of a group reads chunks r, r + LPR, ... of a row
  const T* Kb = reinterpret_cast<const T*>(p.k) + b * p.skb + hkv * p.skh + r * EPL;
  const T* Vb = reinterpret_cast<const T*>(p.v) + b * p.svb + hkv * p.svh + r * EPL;

  {
    // q chunks of this lane's pairs (pair pw0 + m * RPW + g, m < MI)
    uint4 qv[MI][CPL];
#pragma unroll
    for (int m = 0; m < MI; ++m) {
      const int pi = pw0 + m * RPW + g;
      const int j = j0 + pi / G;
      const int h = hkv * G + pi % G;
      const T* qrow = reinterpret_cast<const T*>(p.q) + b * p.sqb + h * p.sqh + (int64_t)j * p.sqs +
                      r * EPL;
#pragma unroll
      for (int c = 0; c < CPL; ++c)
        qv[m][c] = j < p.n_rows ? ldg16_stream(qrow + c * LPR * EPL) : make_uint4(0, 0, 0, 0);
    }
    // ---- scores, two slots per butterfly (their rows in one shared load per
    // pair): lane r ends with slot k0 + r / MI of pair pw0 + (r % MI) * RPW + g.
    // A slot past w (odd w) holds a masked row (tile_slot_rows) ----------------
    const int my_pi = pw0 + (r % MI) * RPW + g;
    for (int k0 = 0; k0 < w; k0 += 2) {
      int2 rows[MI];
#pragma unroll
      for (int m = 0; m < MI; ++m) rows[m] = slot_rows2(sidx, pw0 + m * RPW + g, k0);
      float part[LPR];
#pragma unroll
      for (int s2 = 0; s2 < 2; ++s2) {
        uint4 kb[MI][CPL];
#pragma unroll
        for (int m = 0; m < MI; ++m) {
          const T* krow = Kb + (int64_t)(row2_at(rows[m], s2) & kRowMask) * p.sks;
#pragma unroll
          for (int c = 0; c < CPL; ++c) kb[m][c] = ldg16(krow + c * LPR * EPL);
        }
#pragma unroll
        for (int m = 0; m < MI; ++m) {
          float d = 0.f;
#pragma unroll
          for (int c = 0; c < CPL; ++c) d = M::dot(qv[m][c], kb[m][c], d);
          part[s2 * MI + m] = d;
        }
      }
      transpose_reduce<LPR>(part, lane);
      const int k = k0 + r / MI;
      sbuf[my_pi][k] = sidx[my_pi][k] >= 0 ? part[0] * p.scale_log2 : -INFINITY;
    }
  }
  __syncthreads();

  // ---- softmax: thread t takes pair t / 2, slots [(t & 1) * 32, +32) ------
  {
    const int pi = threadIdx.x >> 1;
    const int kbeg = (threadIdx.x & 1) * HALF;
    float v[HALF];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < HALF; ++i) {
      v[i] = kbeg + i < w ? sbuf[pi][kbeg + i] : -INFINITY;
      mx = fmaxf(mx, v[i]);
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = mx == -INFINITY ? 0.f : mx;
    __syncthreads();   // every score is in registers before the weights overwrite them
    float l = 0.f;
#pragma unroll
    for (int i = 0; i < HALF; ++i) {
      const Sc e = M::scalar(exp2f(v[i] - mx));
      sp[pi][kbeg + i] = e;
      l += M::to_float(e);
    }
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const int j = j0 + pi / G;
    const int h = hkv * G + pi % G;
    if ((threadIdx.x & 1) == 0) {
      sl[pi] = inv;
      if (j < p.n_rows) p.lse[((int64_t)b * p.Hq + h) * p.n_rows + j] = mx + log2f(l);
    }
    // optional: the normalised probabilities for the backward, fp32 from the
    // fp32 scores (what the backward would recompute from lse), slot-major
    // [B, Hq, w, n]; the 4 bytes of neighbouring queries come from
    // neighbouring warps and merge in L2
    if (p.probs && j < p.n_rows) {
      const uint64_t pol = l2_evict_first_policy();   // read once, by the backward
      float* dst = p.probs + ((int64_t)(b * p.Hq + h) * w + kbeg) * p.n_rows + j;
#pragma unroll
      for (int i = 0; i < HALF; ++i)
        if (kbeg + i < w) stg_f32_hint(dst + (int64_t)i * p.n_rows, exp2f(v[i] - mx) * inv, pol);
    }
  }
  __syncthreads();

  // ---- O = P V: lane keeps dims (r + c * LPR) * EPL .. of its MI pairs ----
  float acc[MI][CPL * EPL];
#pragma unroll
  for (int m = 0; m < MI; ++m)
#pragma unroll
    for (int e = 0; e < CPL * EPL; ++e) acc[m][e] = 0.f;
  // 2 slots per shared load of rows and weights; a slot past w (odd w) has
  // weight 0 (written by the softmax) and a masked in-bounds row
  for (int k0 = 0; k0 < w; k0 += 2) {
    int2 rows[MI];
    uint32_t wts[MI];
#pragma unroll
    for (int m = 0; m < MI; ++m) {
      rows[m] = slot_rows2(sidx, pw0 + m * RPW + g, k0);
      wts[m] = weights2(&sp[pw0 + m * RPW + g][0], k0);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      uint4 vb[MI][CPL];
#pragma unroll
      for (int m = 0; m < MI; ++m) {
        const T* vrow = Vb + (int64_t)(row2_at(rows[m], i) & kRowMask) * p.svs;
#pragma unroll
        for (int c = 0; c < CPL; ++c) vb[m][c] = ldg16(vrow + c * LPR * EPL);
      }
#pragma unroll
      for (int m = 0; m < MI; ++m)
#pragma unroll
        for (int c = 0; c < CPL; ++c) M::axpy(weight2_at(wts[m], i), vb[m][c], acc[m] + c * EPL);
    }
  }
#pragma unroll
  for (int m = 0; m < MI; ++m) {
    const int pi = pw0 + m * RPW + g;
    const int j = j0 + pi / G;
    const int h = hkv * G + pi % G;
    if (j < p.n_rows) {
      const float inv = sl[pi];
#pragma unroll
      for (int e = 0; e < CPL * EPL; ++e) acc[m][e] *= inv;
      T* orow = reinterpret_cast<T*>(p.o) + b * p.sob + h * p.soh + (int64_t)j * p.sos + r * EPL;
#pragma unroll
      for (int c = 0; c < CPL; ++c) stg16(orow + c * LPR * EPL, V::from_float(acc[m] + c * EPL));
    }
  }
}

// ---------------------------------------------------------------------------
// Backward, query side, slot-major tile variant (same tiling as
// fwd_tile_kernel): pass 1a scores -> p = exp2(s - lse) (fp32, shared), or the
// forward's probabilities; pass 1b dp = dO.v (V gather, fp32, shared) and the
// row value delta = sum_k p_k dp_k, which equals rowsum(dO o O) for the exact
// O = sum_k p_k v_k (computed this way it needs no O read and carries no
// rounding of the stored 16-bit O: a key with ~1e5 users sums that rounding
// into its dK otherwise); then dS = p (dp - delta), written to the (p,
// dS*scale) workspace and kept in shared memory; pass 2 dQ = sum dS k.
// Every pass walks the slots with all warps together, so the K / V rows the
// tile's pairs share come from L1.
// ---------------------------------------------------------------------------
constexpr int kTileBwdSmemBytes = kTileSidxBytes + 2 * kTileScoreBytes;   // sidx, p, dp / dS

template <typename T, int D>
__global__ void __launch_bounds__(256, 2)
bwd_query_tile_kernel(const AttnParams p) {
  using L = TileLayout<T, D>;
  using V = Vec<T>;
  using M = Mix<T>;
  using Sc = typename M::Scalar;
  constexpr int EPL = L::EPL, LPR = L::LPR, RPW = L::RPW, CPL = L::CPL;
  constexpr int PPW = kTilePairs / 8;
  constexpr int MI = PPW / RPW;
  static_assert(MI * 2 == LPR, "two slots per transpose-reduce");
  constexpr int HALF = kTileMaxW / 2;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int(*sidx)[kTileRowStride] = reinterpret_cast<int(*)[kTileRowStride]>(smem_raw);
  float(*sprob)[kTileIdxStride] =
      reinterpret_cast<float(*)[kTileIdxStride]>(smem_raw + kTileSidxBytes);
  // dp per (pair, slot), then dS * scale in place
  float(*sdp)[kTileIdxStride] =
      reinterpret_cast<float(*)[kTileIdxStride]>(smem_raw + kTileSidxBytes + kTileScoreBytes);
  const int w = p.pat.w;
  const int n = p.n_rows;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane / LPR, r = lane % LPR;
  const int G = p.G;
  const int TQ = kTilePairs / G;
  const int hkv = blockIdx.y, b = blockIdx.z;
  const int j0 = blockIdx.x * TQ;

  {
    const int pi = threadIdx.x >> 1;
    const int j = j0 + pi / G;
    const int h = hkv * G + pi % G;
    const int kbeg = (threadIdx.x & 1) * HALF;
    tile_slot_rows(p, j, h, kbeg, HALF, &sidx[pi][0]);
  }
  __syncthreads();

  const int pw0 = warp * PPW;
  const int my_pi = pw0 + (r % MI) * RPW + g;   // pair whose totals this lane ends with
  const int my_j = j0 + my_pi / G;
  const int my_h = hkv * G + my_pi % G;
  const bool my_live = my_j < n;
  // lane r of a group reads chunks r, r + LPR, ... of a row
  const T* Kb = reinterpret_cast<const T*>(p.k) + b * p.skb + hkv * p.skh + r * EPL;
  const T* Vb = reinterpret_cast<const T*>(p.v) + b * p.svb + hkv * p.svh + r * EPL;
  // the CPL chunks of this lane of row j of pair m's head in a [B, Hq, n, D] tensor
  auto row_of = [&](const void* base, int64_t sb, int64_t sh, int64_t ss, int m, uint4 (&out)[CPL]) {
    const int pi = pw0 + m * RPW + g;
    const int j = j0 + pi / G;
    const int h = hkv * G + pi % G;
    const T* row = reinterpret_cast<const T*>(base) + b * sb + h * sh + (int64_t)j * ss + r * EPL;
#pragma unroll
    for (int c = 0; c < CPL; ++c)
      out[c] = j < n ? ldg16_stream(row + c * LPR * EPL) : make_uint4(0, 0, 0, 0);
  };

  // ---- pass 1a: p = exp2(s * scale_log2 - lse), or the forward's p --------
  if (p.probs) {
    const int lg = __ffs(G) - 1;   // same lane order as the forward's write
    const uint64_t pol = l2_evict_first_policy();
    for (int k = warp; k < w; k += 8) {
      for (int pi = lane; pi < kTilePairs; pi += 32) {
        const int j = j0 + (pi >> lg);
        if (j >= n) break;
        const int h = hkv * G + (pi & (G - 1));
        sprob[pi][k] = ldg_f32_hint(p.probs + (((int64_t)b * p.Hq + h) * w + k) * n + j, pol);
      }
    }
    __syncthreads();
  } else {
    const float lse2 = my_live ? p.lse[((int64_t)b * p.Hq + my_h) * n + my_j] : 0.f;
    uint4 qv[MI][CPL];
#pragma unroll
    for (int m = 0; m < MI; ++m) row_of(p.q, p.sqb, p.sqh, p.sqs, m, qv[m]);
    for (int k0 = 0; k0 < w; k0 += 2) {
      int2 rows[MI];
#pragma unroll
      for (int m = 0; m < MI; ++m) rows[m] = slot_rows2(sidx, pw0 + m * RPW + g, k0);
      float part[LPR];
#pragma unroll
      for (int s2 = 0; s2 < 2; ++s2) {
        uint4 kb[MI][CPL];
#pragma unroll
        for (int m = 0; m < MI; ++m) {
          const T* krow = Kb + (int64_t)(row2_at(rows[m], s2) & kRowMask) * p.sks;
#pragma unroll
          for (int c = 0; c < CPL; ++c) kb[m][c] = ldg16(krow + c * LPR * EPL);
        }
#pragma unroll
        for (int m = 0; m < MI; ++m) {
          float d = 0.f;
#pragma unroll
          for (int c = 0; c < CPL; ++c) d = M::dot(qv[m][c], kb[m][c], d);
          part[s2 * MI + m] = d;
        }
      }
      transpose_reduce<LPR>(part, lane);
      const int k = k0 + r / MI;
      sprob[my_pi][k] = sidx[my_pi][k] >= 0 ? exp2f(part[0] * p.scale_log2 - lse2) : 0.f;
    }
  }

  // ---- pass 1b: dp = dO.v and delta = sum_k p_k dp_k ---------------------
  {
    uint4 dv[MI][CPL];
#pragma unroll
    for (int m = 0; m < MI; ++m) row_of(p.dout, p.sdob, p.sdoh, p.sdos, m, dv[m]);
    float dpart = 0.f;   // this lane's slots of pair my_pi
    for (int k0 = 0; k0 < w; k0 += 2) {
      int2 rows[MI];
#pragma unroll
      for (int m = 0; m < MI; ++m) rows[m] = slot_rows2(sidx, pw0 + m * RPW + g, k0);
      float part[LPR];
#pragma unroll
      for (int s2 = 0; s2 < 2; ++s2) {
        uint4 vb[MI][CPL];
#pragma unroll
        for (int m = 0; m < MI; ++m) {
          const T* vrow = Vb + (int64_t)(row2_at(rows[m], s2) & kRowMask) * p.svs;
#pragma unroll
          for (int c = 0; c < CPL; ++c) vb[m][c] = ldg16(vrow + c * LPR * EPL);
        }
#pragma unroll
        for (int m = 0; m < MI; ++m) {
          float d = 0.f;
#pragma unroll
          for (int c = 0; c < CPL; ++c) d = M::dot(dv[m][c], vb[m][c], d);
          part[s2 * MI + m] = d;
        }
      }
      transpose_reduce<LPR>(part, lane);
      const int k = k0 + r / MI;
      // a slot past w (odd w) and masked slots have p = 0
      const float pk = k < w ? sprob[my_pi][k] : 0.f;
      sdp[my_pi][k] = part[0];
      dpart += pk * part[0];
    }
    // lanes r and r ^ MI hold the even / odd slots of the same pair
    const float delta = dpart + __shfl_xor_sync(0xffffffffu, dpart, MI);
    // dS = p (dp - delta), the (p, dS * scale) workspace, dS * scale in place of dp
    float2* pds_pair = p.pds + ((int64_t)(b * p.Hq + my_h) * w) * n + my_j;
    const uint64_t pol_ws = l2_evict_first_policy();   // read once, by the key side
    for (int k = r / MI; k < w + 1; k += 2) {
      if (k >= kTileMaxW) break;
      const float pk = k < w ? sprob[my_pi][k] : 0.f;
      const float dsk = pk * (sdp[my_pi][k] - delta) * p.scale;   // 0 for masked slots
      if (my_live && k < w) stg_f2_hint(pds_pair + (int64_t)k * n, make_float2(pk, dsk), pol_ws);
      sdp[my_pi][k] = dsk;
    }
  }
  __syncthreads();

  // ---- pass 2: dQ = sum dS k ------------------------------------------------
  float acc[MI][CPL * EPL];
#pragma unroll
  for (int m = 0; m < MI; ++m)
#pragma unroll
    for (int e = 0; e < CPL * EPL; ++e) acc[m][e] = 0.f;
  // dS * scale of 2 slots per shared load (fp32, rounded to the input type
  // for the mixed-precision FMA); a slot past w (odd w) has dS = 0
  for (int k0 = 0; k0 < w; k0 += 2) {
    int2 rows[MI];
    float2 wts[MI];
#pragma unroll
    for (int m = 0; m < MI; ++m) {
      rows[m] = slot_rows2(sidx, pw0 + m * RPW + g, k0);
      wts[m] = make_float2(sdp[pw0 + m * RPW + g][k0], sdp[pw0 + m * RPW + g][k0 + 1]);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      uint4 kb[MI][CPL];
#pragma unroll
      for (int m = 0; m < MI; ++m) {
        const T* krow = Kb + (int64_t)(row2_at(rows[m], i) & kRowMask) * p.sks;
#pragma unroll
        for (int c = 0; c < CPL; ++c) kb[m][c] = ldg16(krow + c * LPR * EPL);
      }
#pragma unroll
      for (int m = 0; m < MI; ++m) {
        const Sc wt = M::scalar(i ? wts[m].y : wts[m].x);
#pragma unroll
        for (int c = 0; c < CPL; ++c) M::axpy(wt, kb[m][c], acc[m] + c * EPL);
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MI; ++m) {
    const int pi = pw0 + m * RPW + g;
    const int j = j0 + pi / G;
    const int h = hkv * G + pi % G;
    if (j < n) {
      T* dqrow = reinterpret_cast<T*>(p.dq) + b * p.sdqb + h * p.sdqh + (int64_t)j * p.sdqs + r * EPL;
#pragma unroll
      for (int c = 0; c < CPL; ++c) stg16(dqrow + c * LPR * EPL, V::from_float(acc[m] + c * EPL));
    }
  }
}

// ---------------------------------------------------------------------------
// Backward, query side: dQ and the (p, dS*scale) workspace.
// Same grid and pair order as the forward.
// ---------------------------------------------------------------------------
template <typename T, int D, int NW>
__global__ void __launch_bounds__(NW * 32, 2)
bwd_query_kernel(const AttnParams p, int rows_per_cta) {
  using L = Layout<T, D>;
  using V = Vec<T>;
  using M = Mix<T>;
  using Sc = typename M::Scalar;
  constexpr int EPL = L::EPL, LPR = L::LPR, RPW = L::RPW;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int w = p.pat.w;
  const int wpad = (w + 31) & ~31;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* sidx = reinterpret_cast<int*>(smem_raw) + warp * 3 * wpad;
  // per slot: p (the sign bit set when dropout drops the slot), and dP (after
  // dropout), then dS * scale in its place
  float* spk = reinterpret_cast<float*>(sidx + wpad);
  float* sdp = spk + wpad;
  const int g = lane / LPR, r = lane % LPR;
  const int hkv = blockIdx.y, b = blockIdx.z;
  const int row0 = blockIdx.x * rows_per_cta;
  const int n_pairs = rows_per_cta * p.G;
  const int n = p.n_rows;
  const T* Kb = reinterpret_cast<const T*>(p.k) + b * p.skb + hkv * p.skh + r * EPL;
  const T* Vb = reinterpret_cast<const T*>(p.v) + b * p.svb + hkv * p.svh + r * EPL;

  for (int pr = warp; pr < n_pairs; pr += NW) {
    const int j = row0 + pr / p.G;
    if (j >= n) break;
    const int h = hkv * p.G + pr % p.G;
    const int pos = query_pos(p, j);
    fill_slot_rows(p, pos, h, wpad, lane, sidx);

    uint4 qv, dv;
    {
      const int64_t jr = (int64_t)j;
      const T* qrow = reinterpret_cast<const T*>(p.q) + b * p.sqb + h * p.sqh + jr * p.sqs + r * EPL;
      const T* drow = reinterpret_cast<const T*>(p.dout) + b * p.sdob + h * p.sdoh + jr * p.sdos + r * EPL;
      qv = ldg16_stream(qrow);
      dv = ldg16_stream(drow);
    }
    const float lse2 = p.lse[((int64_t)b * p.Hq + h) * n + j];
    float2* pds_row = p.pds + ((int64_t)(b * p.Hq + h) * w) * n + j;
    __syncwarp();

    float dpart = 0.f;
    for (int s0 = 0; s0 < wpad; s0 += 32) {
      float ps[LPR], pp[LPR];
      {
        uint4 kb[LPR];
#pragma unroll
        for (int m = 0; m < LPR; ++m) {
          const int row = sidx[s0 + m * RPW + g];
          kb[m] = row >= 0 ? ldg16(Kb + (int64_t)row * p.sks) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int m = 0; m < LPR; ++m) ps[m] = M::dot(qv, kb[m], 0.f);
      }
      {
        uint4 vb[LPR];
#pragma unroll
        for (int m = 0; m < LPR; ++m) {
          const int row = sidx[s0 + m * RPW + g];
          vb[m] = row >= 0 ? ldg16(Vb + (int64_t)row * p.svs) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int m = 0; m < LPR; ++m) pp[m] = M::dot(dv, vb[m], 0.f);
      }
      transpose_reduce<LPR>(ps, lane);
      transpose_reduce<LPR>(pp, lane);
      const int k = s0 + r * RPW + g;
      float pk = 0.f, dpk = 0.f;
      bool keep = true;
      if (sidx[k] >= 0) {
        pk = exp2f(ps[0] * p.scale_log2 - lse2);
        dpk = pp[0];
        if (p.drop_threshold) {
          // the same keep mask as the forward: dP = mask / (1 - p) * dO.v and
          // the weight used for dV is the kept, rescaled one
          keep = dropout_keep(p, pos, b, h, k);
          dpk = keep ? dpk * p.keep_scale : 0.f;
        }
      }
      spk[k] = keep ? pk : -pk;
      sdp[k] = dpk;
      dpart += pk * dpk;
    }
    // delta = sum_k p_k dP_k = rowsum(dO o O) for the exact O (with dropout:
    // the O of the kept, rescaled weights), without the stored O's rounding
    const float delta = warp_sum(dpart);
    __syncwarp();
    for (int k = lane; k < wpad; k += 32) {
      const float v = spk[k];
      const float pk = fabsf(v);
      const float dsk = pk * (sdp[k] - delta) * p.scale;   // 0 for masked slots
      const float pw = signbit(v) ? 0.f : (p.drop_threshold ? pk * p.keep_scale : pk);
      if (k < w) pds_row[(int64_t)k * n] = make_float2(pw, dsk);
      sdp[k] = dsk;
    }
    __syncwarp();

    float acc[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[e] = 0.f;
    for (int s0 = 0; s0 < wpad; s0 += 32) {
      uint4 kb[LPR];
#pragma unroll
      for (int m = 0; m < LPR; ++m) {
        const int row = sidx[s0 + m * RPW + g];
        kb[m] = row >= 0 ? ldg16(Kb + (int64_t)row * p.sks) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int m = 0; m < LPR; ++m) M::axpy(M::scalar(sdp[s0 + m * RPW + g]), kb[m], acc);   // 0 when masked
    }
#pragma unroll
    for (int o = LPR; o < 32; o <<= 1)
#pragma unroll
      for (int e = 0; e < EPL; ++e) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], o);
    if (g == 0) {
      T* dqrow = reinterpret_cast<T*>(p.dq) + b * p.sdqb + h * p.sdqh + (int64_t)j * p.sdqs + r * EPL;
      stg16(dqrow, V::from_float(acc));
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Backward, key side, long runs: for every chunk of kHeavyChunk consecutive
// query slots whose users all use one key in a (head, slot) column (with the
// per-slot index monotone in position, the first and the last slot decide),
// the sums of dS*scale q and p dO over the chunk, into
// heavy[b, h, slot, chunk, {dK, dV}, D] (fp32).  bwd_key_kernel skips those
// chunks and adds the partials, so a key that receives a whole column's
// queries (alpha = 1, head 0, slot 0: every query uses key 0) is summed by
// many warps instead of one.  grid = (n_rows / kHeavyChunk, Hq, B).
// ---------------------------------------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(256)
bwd_heavy_kernel(const AttnParams p) {
  using L = Layout<T, D>;
  constexpr int EPL = L::EPL, LPR = L::LPR, RPW = L::RPW;
  constexpr int UNROLL = 4;
  static_assert(kHeavyChunk % (RPW * UNROLL) == 0, "chunk must split into whole steps");
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane / LPR, r = lane % LPR;
  const int n = p.n_rows, w = p.pat.w;
  const int j0 = c * kHeavyChunk;
  const float t = head_weight(p.pat, h);
  const float omt = __fsub_rn(1.f, t);
  const int64_t* srows = p.sorted_rows ? p.sorted_rows : p.rows;
  const int kvmax = p.kv_len - 1;
  auto cidx = [&](int jq, int k) -> int {
    const int pos = srows ? (int)srows[jq] : p.row_offset + jq;
    return min(raw_index(row_window(p.pat, pos), k, t, omt), kvmax);
  };
  const float2* pdsb = p.pds + (int64_t)(b * p.Hq + h) * w * n;
  const T* qb = reinterpret_cast<const T*>(p.q) + b * p.sqb + h * p.sqh + r * EPL;
  const T* db = reinterpret_cast<const T*>(p.dout) + b * p.sdob + h * p.sdoh + r * EPL;
  for (int k = warp; k < w; k += blockDim.x >> 5) {
    int constant = 0;
    if (lane == 0) constant = cidx(j0, k) == cidx(j0 + kHeavyChunk - 1, k);
    if (!__shfl_sync(0xffffffffu, constant, 0)) continue;
    float adk[EPL], adv[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) { adk[e] = 0.f; adv[e] = 0.f; }
    const float2* pk = pdsb + (int64_t)k * n;
    for (int u = g; u < kHeavyChunk; u += RPW * UNROLL) {
      int qi[UNROLL];
      float2 pd[UNROLL];
      uint4 qv[UNROLL], dv[UNROLL];
#pragma unroll
      for (int x = 0; x < UNROLL; ++x) {
        const int jq = j0 + u + x * RPW;
        qi[x] = p.row_perm ? (int)p.row_perm[jq] : jq;
      }
#pragma unroll
      for (int x = 0; x < UNROLL; ++x) {
        pd[x] = pk[qi[x]];
        qv[x] = ldg16_stream(qb + (int64_t)qi[x] * p.sqs);
        dv[x] = ldg16_stream(db + (int64_t)qi[x] * p.sdos);
      }
#pragma unroll
      for (int x = 0; x < UNROLL; ++x) {
        axpy_f32<T>(pd[x].y, qv[x], adk);
        axpy_f32<T>(pd[x].x, dv[x], adv);
      }
    }
#pragma unroll
    for (int o = LPR; o < 32; o <<= 1)
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        adk[e] += __shfl_xor_sync(0xffffffffu, adk[e], o);
        adv[e] += __shfl_xor_sync(0xffffffffu, adv[e], o);
      }
    if (g == 0) {
      float* part = p.heavy + ((((int64_t)b * p.Hq + h) * w + k) * p.heavy_chunks + c) * (2 * D) +
                    r * EPL;
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        part[e] = adk[e];
        part[D + e] = adv[e];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Backward, key side, for query head (hkv * G + head_in_group) of every group.
// grid = (ceil(kv_rows / (NW * RW)), Hkv, B); warp owns RW consecutive key
// rows; lanes own slot columns k = lane + 32 * cc.  With G > 1 the G launches
// run in order on one stream and accumulate into the fp32 workspace; the last
// one writes dK / dV in the input dtype.
//
// The q / dO rows of a key row's users are copied with cp.async (16 bytes per
// lane, L1 bypassed) into a per-warp ring of two shared-memory stages of UB
// users each, so the warp computes one stage while the next is in flight.
// ---------------------------------------------------------------------------
template <typename T, int D>
struct KeyStage {
  static constexpr int kRowBytes = D * (int)sizeof(T);
  static constexpr int kUsers = (2048 / kRowBytes) < 32 ? (2048 / kRowBytes) : 32;  // per stage
  static constexpr int kStageBytes = kUsers * 2 * kRowBytes;                       // q + dO rows
  static constexpr int kWarpBytes = 2 * kStageBytes;
};

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src, bool valid) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(gmem_src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <typename T, int D, int NW, int RW>
__global__ void __launch_bounds__(NW * 32, 3)
bwd_key_kernel(const AttnParams p) {
  using L = Layout<T, D>;
  using V = Vec<T>;
  using S = KeyStage<T, D>;
  constexpr int EPL = L::EPL, LPR = L::LPR, RPW = L::RPW;
  constexpr int UB = S::kUsers;
  static_assert(UB % RPW == 0 && UB <= 32, "stage size must hold whole warp loads");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int w = p.pat.w;
  const int ncol = (w + 31) >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned char* ring = smem_raw + warp * S::kWarpBytes;
  // per column: cursor (first query slot not yet assigned to a key) and the
  // key index at the cursor (so a column with no user for a key costs no
  // index computation)
  int* scur = reinterpret_cast<int*>(smem_raw + NW * S::kWarpBytes) + warp * ncol * 64;
  int* sval = scur + ncol * 32;
  const int g = lane / LPR, r = lane % LPR;
  const int hkv = blockIdx.y, b = blockIdx.z;
  const int h = hkv * p.G + p.head_in_group;
  const int lr0 = (blockIdx.x * NW + warp) * RW;
  if (lr0 >= p.kv_rows) return;
  const int lr1 = min(lr0 + RW, p.kv_rows);
  const int n = p.n_rows;
  const float t = head_weight(p.pat, h);
  const float omt = __fsub_rn(1.f, t);
  const int64_t* srows = p.sorted_rows ? p.sorted_rows : p.rows;
  const int kvmax = p.kv_len - 1;
  auto cidx = [&](int jq, int k) -> int {
    const int pos = srows ? (int)srows[jq] : p.row_offset + jq;
    return min(raw_index(row_window(p.pat, pos), k, t, omt), kvmax);
  };

  // Cursor of each owned column: first query slot whose key is >= row lr0.
  {
    const int P0 = p.kv_offset + lr0;
    for (int cc = 0; cc < ncol; ++cc) {
      const int k = lane + 32 * cc;
      int lo = n;
      if (k < w) {
        int a = 0, e = n;
        while (a < e) {
          const int mid = (a + e) >> 1;
          if (cidx(mid, k) < P0) a = mid + 1; else e = mid;
        }
        lo = a;
      }
      scur[cc * 32 + lane] = lo;
      sval[cc * 32 + lane] = (k < w && lo < n) ? cidx(lo, k) : 0x7fffffff;
    }
  }

  const unsigned char* qbase = reinterpret_cast<const unsigned char*>(
      reinterpret_cast<const T*>(p.q) + b * p.sqb + h * p.sqh);
  const unsigned char* dbase = reinterpret_cast<const unsigned char*>(
      reinterpret_cast<const T*>(p.dout) + b * p.sdob + h * p.sdoh);
  const int64_t qrow_bytes = p.sqs * (int64_t)sizeof(T);
  const int64_t drow_bytes = p.sdos * (int64_t)sizeof(T);
  const float2* pdsb = p.pds + (int64_t)(b * p.Hq + h) * w * n;

  float adk[EPL], adv[EPL];
  // Streams the users of the lanes' runs [start, start + len) of column chunk
  // cc: flattened over lanes, moved with cp.async into two shared-memory
  // stages of UB users, accumulated into adk / adv.
  auto stream_runs = [&](const int start, const int len, const int cc) {
      // Flatten the lanes' runs: exclusive prefix of run lengths.
      int off = len;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, off, o);
        if (lane >= o) off += y;
      }
      const int total = __shfl_sync(0xffffffffu, off, 31);
      off -= len;
      if (total == 0) return;
      // Resolve users u0 + lane (lane < UB) and start their row copies into
      // stage `st`; returns this lane's (p, dS) of its user (0 when none).
      // They stay fp32: a key row can have ~1e5 users (alpha = 1, head 0,
      // slot 0 sends every query to key 0), too many to sum rounded terms.
      auto issue = [&](int u0, int st, float& my_p, float& my_ds) {
        const int u = u0 + lane;
        int o = 0;
#pragma unroll
        for (int sh = 16; sh >= 1; sh >>= 1) {
          const int c = o + sh;
          if (__shfl_sync(0xffffffffu, off, c) <= u) o = c;
        }
        const int o_start = __shfl_sync(0xffffffffu, start, o);
        const int o_off = __shfl_sync(0xffffffffu, off, o);
        int my_qi = 0;
        my_p = 0.f;
        my_ds = 0.f;
        if (lane < UB && u < total) {
          const int jq = o_start + (u - o_off);
          my_qi = p.row_perm ? (int)p.row_perm[jq] : jq;
          const float2 pd = pdsb[(int64_t)(o + 32 * cc) * n + my_qi];
          my_p = pd.x;
          my_ds = pd.y;
        }
        unsigned char* stage = ring + st * S::kStageBytes;
#pragma unroll
        for (int m = 0; m < UB / RPW; ++m) {
          const int x = m * RPW + g;   // user slot in the stage
          const int qi = __shfl_sync(0xffffffffu, my_qi, x);
          const bool valid = u0 + x < total;
          unsigned char* dst = stage + x * 2 * S::kRowBytes + r * 16;
          cp_async16(dst, qbase + qi * qrow_bytes + r * 16, valid);
          cp_async16(dst + S::kRowBytes, dbase + qi * drow_bytes + r * 16, valid);
        }
        cp_async_commit();
      };

      float p_cur, s_cur, p_nxt = 0.f, s_nxt = 0.f;
      issue(0, 0, p_cur, s_cur);
      int st = 0;
      for (int u0 = 0; u0 < total; u0 += UB) {
        const bool more = u0 + UB < total;
        if (more) {
          issue(u0 + UB, st ^ 1, p_nxt, s_nxt);
          cp_async_wait<1>();
        } else {
          cp_async_wait<0>();
        }
        __syncwarp();
        const unsigned char* stage = ring + st * S::kStageBytes;
#pragma unroll
        for (int m = 0; m < UB / RPW; ++m) {
          const int x = m * RPW + g;
          const float pm = __shfl_sync(0xffffffffu, p_cur, x);
          const float sm = __shfl_sync(0xffffffffu, s_cur, x);
          const unsigned char* src = stage + x * 2 * S::kRowBytes + r * 16;
          axpy_f32<T>(sm, *reinterpret_cast<const uint4*>(src), adk);
          axpy_f32<T>(pm, *reinterpret_cast<const uint4*>(src + S::kRowBytes), adv);
        }
        __syncwarp();   // every lane is done with this stage before it is refilled
        p_cur = p_nxt;
        s_cur = s_nxt;
        st ^= 1;
      }
  };
  for (int lr = lr0; lr < lr1; ++lr) {
    const int P = p.kv_offset + lr;
#pragma unroll
    for (int e = 0; e < EPL; ++e) { adk[e] = 0.f; adv[e] = 0.f; }

    for (int cc = 0; cc < ncol; ++cc) {
      const int k = lane + 32 * cc;
      const int start = scur[cc * 32 + lane];
      int len = 0;
      if (sval[cc * 32 + lane] == P) {   // the column's next users are key P's
        // Gallop to the end of the run of query slots that use key P; hv is
        // the key at hi once known (hi = n: none).
        int lo = start, step = 1, hv = 0x7fffffff;
        while (lo + step < n) {
          const int c = cidx(lo + step, k);
          if (c != P) { hv = c; break; }
          lo += step;
          step <<= 1;
        }
        int hi = min(lo + step, n);
        while (hi - lo > 1) {
          const int mid = (lo + hi) >> 1;
          const int c = cidx(mid, k);
          if (c == P) lo = mid; else { hi = mid; hv = c; }
        }
        len = hi - start;
        scur[cc * 32 + lane] = hi;
        sval[cc * 32 + lane] = hi < n ? hv : 0x7fffffff;
      }
      // Full kHeavyChunk-aligned chunks inside a long run were summed by
      // bwd_heavy_kernel; stream only the pieces before and after them.
      int hc0 = 0, hc1 = 0, start2 = 0, len2 = 0, len1 = len;
      if (p.heavy_chunks > 0 && len >= kHeavyChunk) {
        const int e = start + len;
        const int c0 = (start + kHeavyChunk - 1) / kHeavyChunk;
        const int c1 = min(e / kHeavyChunk, p.heavy_chunks);
        if (c1 > c0) {
          hc0 = c0;
          hc1 = c1;
          len1 = c0 * kHeavyChunk - start;
          start2 = c1 * kHeavyChunk;
          len2 = e - start2;
        }
      }
      stream_runs(start, len1, cc);
      if (__any_sync(0xffffffffu, len2 > 0)) stream_runs(start2, len2, cc);
      // add the chunk partials (each lane of row group 0 its D slice)
      unsigned hm = __ballot_sync(0xffffffffu, hc1 > hc0);
      while (hm) {
        const int src = __ffs(hm) - 1;
        hm &= hm - 1;
        const int ck = __shfl_sync(0xffffffffu, k, src);
        const int a = __shfl_sync(0xffffffffu, hc0, src);
        const int z = __shfl_sync(0xffffffffu, hc1, src);
        if (g == 0) {
          const float* part = p.heavy + ((((int64_t)b * p.Hq + h) * w + ck) * p.heavy_chunks + a) *
                                            (2 * D) + r * EPL;
          for (int c = a; c < z; ++c, part += 2 * D) {
#pragma unroll
            for (int e = 0; e < EPL; ++e) {
              adk[e] += part[e];
              adv[e] += part[D + e];
            }
          }
        }
      }
    }

#pragma unroll
    for (int o = LPR; o < 32; o <<= 1)
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        adk[e] += __shfl_xor_sync(0xffffffffu, adk[e], o);
        adv[e] += __shfl_xor_sync(0xffffffffu, adv[e], o);
      }
    if (g == 0) {
      const int64_t ok_ = b * p.sdkb + hkv * p.sdkh + (int64_t)lr * p.sdks + r * EPL;
      const int64_t ov_ = b * p.sdvb + hkv * p.sdvh + (int64_t)lr * p.sdvs + r * EPL;
      // the final dK / dV row piece: input dtype, or fp32 with ESA_FLAG_F32_DKV
      auto store = [&]() {
        if (p.flags & kFlagF32Dkv) {
          float* fk = reinterpret_cast<float*>(p.dk) + ok_;
          float* fv = reinterpret_cast<float*>(p.dv) + ov_;
#pragma unroll
          for (int e = 0; e < EPL; e += 4) {
            *reinterpret_cast<float4*>(fk + e) = make_float4(adk[e], adk[e + 1], adk[e + 2], adk[e + 3]);
            *reinterpret_cast<float4*>(fv + e) = make_float4(adv[e], adv[e + 1], adv[e + 2], adv[e + 3]);
          }
        } else {
          stg16(reinterpret_cast<T*>(p.dk) + ok_, V::from_float(adk));
          stg16(reinterpret_cast<T*>(p.dv) + ov_, V::from_float(adv));
        }
      };
      if (p.G == 1) {
        store();
      } else {
        const int64_t plane = (int64_t)p.B * p.Hkv * p.kv_rows * D;
        float* ak = p.acc + (((int64_t)b * p.Hkv + hkv) * p.kv_rows + lr) * D + r * EPL;
        float* av = ak + plane;
        if (p.head_in_group > 0) {
#pragma unroll
          for (int e = 0; e < EPL; e += 4) {
            const float4 x = *reinterpret_cast<const float4*>(ak + e);
            const float4 y = *reinterpret_cast<const float4*>(av + e);
            adk[e] += x.x; adk[e + 1] += x.y; adk[e + 2] += x.z; adk[e + 3] += x.w;
            adv[e] += y.x; adv[e + 1] += y.y; adv[e + 2] += y.z; adv[e + 3] += y.w;
          }
        }
        if (p.head_in_group == p.G - 1) {
          store();
        } else {
#pragma unroll
          for (int e = 0; e < EPL; e += 4) {
            *reinterpret_cast<float4*>(ak + e) = make_float4(adk[e], adk[e + 1], adk[e + 2], adk[e + 3]);
            *reinterpret_cast<float4*>(av + e) = make_float4(adv[e], adv[e + 1], adv[e + 2], adv[e + 3]);
          }
        }
      }
    }
  }
}

}  // namespace esa
