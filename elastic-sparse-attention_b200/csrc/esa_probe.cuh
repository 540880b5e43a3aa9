// Gather probe: the row loads of the slot-major tile forward without its
// arithmetic, for measuring the row-gather bandwidth that bounds the gather
// kernels (esa_probe_gather in include/esa_b200.h).
//
// Same grid, CTA shape and load order as fwd_tile_kernel: a CTA owns 128
// (query, head) pairs of one KV head (128 / G queries x G heads), warp w owns
// pairs [16w, 16w + 16), 8 lanes read a row (D / 64 16-byte chunks each, so
// one warp load covers 4 rows); all warps walk the slots together, K rows
// first (the score pass), then V rows (the P V pass), two slots per step
// with their rows in one shared load.  The rows come from the elastic
// pattern (the
// tile kernels' exact stream), uniformly at random over the KV head's rows
// (an L2-resident random gather), or at random within 64 rows per CTA (an
// L1-resident gather), or as runs of consecutive rows that no CTA reads
// twice (L2 streaming).  The loaded words are folded into an xor checksum
// that is stored only when it equals an improbable constant.
#pragma once
#include "esa_gather.cuh"

namespace esa {

enum ProbeMode : int { kProbePattern = 0, kProbeL2Random = 1, kProbeL1Window = 2, kProbeL2Stream = 3 };
constexpr int kProbeWindowRows = 64;

// 32-bit integer mix (xor-shift / multiply rounds) for the random row choices.
__device__ __forceinline__ uint32_t probe_mix(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

template <typename T, int D, int MODE>
__global__ void __launch_bounds__(256, 2)
gather_probe_kernel(const AttnParams p, uint32_t* sink) {
  using L = TileLayout<T, D>;
  constexpr int EPL = L::EPL, LPR = L::LPR, RPW = L::RPW, CPL = L::CPL;
  constexpr int PPW = kTilePairs / 8;      // pairs per warp
  constexpr int MI = PPW / RPW;            // warp loads per slot
  constexpr int HALF = kTileMaxW / 2;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int(*sidx)[kTileRowStride] = reinterpret_cast<int(*)[kTileRowStride]>(smem_raw);
  const int w = p.pat.w;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane / LPR, r = lane % LPR;
  const int G = p.G;
  const int TQ = kTilePairs / G;
  const int hkv = blockIdx.y, b = blockIdx.z;
  const int j0 = blockIdx.x * TQ;
  if (MODE == kProbePattern) {
    const int pi = threadIdx.x >> 1;
    tile_slot_rows(p, j0 + pi / G, hkv * G + pi % G, (threadIdx.x & 1) * HALF, HALF, &sidx[pi][0]);
    __syncthreads();
  }
  const uint32_t cta = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
  // L1 window: rows [win0, win0 + kProbeWindowRows), inside the buffer (the
  // host requires kv_rows >= kProbeWindowRows)
  const int win0 = MODE == kProbeL1Window
                       ? (int)(probe_mix(cta) % (uint32_t)(p.kv_rows - kProbeWindowRows + 1))
                       : 0;
  // rows of 2 slots of pair pi (a slot past w: the masked in-bounds row)
  auto rows_at = [&](int pi, int k0) -> int2 {
    if constexpr (MODE == kProbePattern) {
      return slot_rows2(sidx, pi, k0);
    } else {
      int v[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        if constexpr (MODE == kProbeL2Stream) {
          // CTA c, pair pi, slot k: row (c * 128 * 64 + pi * 64 + k) mod kv_rows
          const uint32_t r = (cta * (uint32_t)kTilePairs + (uint32_t)pi) * (uint32_t)kTileMaxW +
                             (uint32_t)(k0 + i);
          v[i] = (int)(r % (uint32_t)p.kv_rows);
        } else {
          const uint32_t hsh = probe_mix(cta * 8192u + (uint32_t)(pi * kTileMaxW + k0 + i));
          v[i] = MODE == kProbeL2Random ? (int)(hsh % (uint32_t)p.kv_rows)
                                        : win0 + (int)(hsh & (kProbeWindowRows - 1));
        }
      }
      return make_int2(v[0], v[1]);
    }
  };
  const int pw0 = warp * PPW;
  const T* Kb = reinterpret_cast<const T*>(p.k) + b * p.skb + hkv * p.skh + r * EPL;
  const T* Vb = reinterpret_cast<const T*>(p.v) + b * p.svb + hkv * p.svh + r * EPL;
  uint32_t acc = 0;
#pragma unroll 1
  for (int pass = 0; pass < 2; ++pass) {
    const T* base = pass ? Vb : Kb;
    const int64_t stride = pass ? p.svs : p.sks;
    for (int k0 = 0; k0 < w; k0 += 2) {
      int2 rows[MI];
#pragma unroll
      for (int m = 0; m < MI; ++m) rows[m] = rows_at(pw0 + m * RPW + g, k0);
#pragma unroll
      for (int s2 = 0; s2 < 2; ++s2) {
        uint4 x[MI][CPL];
#pragma unroll
        for (int m = 0; m < MI; ++m) {
          const T* row = base + (int64_t)(row2_at(rows[m], s2) & kRowMask) * stride;
#pragma unroll
          for (int c = 0; c < CPL; ++c) x[m][c] = ldg16(row + c * LPR * EPL);
        }
#pragma unroll
        for (int m = 0; m < MI; ++m)
#pragma unroll
          for (int c = 0; c < CPL; ++c) acc ^= x[m][c].x ^ x[m][c].y ^ x[m][c].z ^ x[m][c].w;
      }
    }
  }
  if (acc == 0x9E3779B9u) *sink = acc;
}

}  // namespace esa
