// Latency kernel for few query rows (decode with cache_position, short
// prompts): the forward of reference :117-166 with the w slots of one
// (row, head) pair split across the warps of a CTA.
//
// The throughput kernels give a warp a whole pair and walk its slots in
// sub-chunks of 32 (scores of every sub-chunk, then the values), which costs
// 2 * w / 32 dependent round trips to memory per pair.  With a handful of
// pairs nothing hides those round trips, so here each warp owns one sub-chunk
// of 32 slots and issues the K and V loads of all its slots at once: one
// round trip for the whole pair (two for 32-lane rows, whose 2 x 32 vectors
// per lane would not fit in registers together).  Warps merge their partial
// softmax states (max, sum, weighted V) through shared memory.
//
// grid = (n_rows, Hq, B); block = NW = min(ceil(w / 32), kDecodeMaxWarps)
// warps; warp i handles sub-chunks i, i + NW, ... with an online softmax.
#pragma once
#include "esa_gather.cuh"

namespace esa {

constexpr int kDecodeMaxWarps = 8;

template <typename T, int D>
__global__ void __launch_bounds__(kDecodeMaxWarps * 32)
fwd_decode_kernel(const AttnParams p) {
  using L = Layout<T, D>;
  using V = Vec<T>;
  using M = Mix<T>;
  constexpr int EPL = L::EPL, LPR = L::LPR, RPW = L::RPW;
  constexpr bool kKvTogether = LPR <= 16;
  __shared__ float s_ml[kDecodeMaxWarps][2];
  __shared__ __align__(16) float s_acc[kDecodeMaxWarps][D];

  const int w = p.pat.w;
  const int nchunks = (w + 31) >> 5;
  const int nw = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane / LPR, r = lane % LPR;
  const int j = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hkv = h / p.G;
  const int pos = query_pos(p, j);
  const RowWin rw = row_window(p.pat, pos);
  const float t = head_weight(p.pat, h);
  const float omt = __fsub_rn(1.f, t);
  const T* Kb = reinterpret_cast<const T*>(p.k) + b * p.skb + hkv * p.skh + r * EPL;
  const T* Vb = reinterpret_cast<const T*>(p.v) + b * p.svb + hkv * p.svh + r * EPL;
  const uint4 qv = ldg16(reinterpret_cast<const T*>(p.q) + b * p.sqb + h * p.sqh +
                         (int64_t)j * p.sqs + r * EPL);

  float m_run = -INFINITY, l_run = 0.f;
  float acc[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) acc[e] = 0.f;

  for (int c = warp; c < nchunks; c += nw) {
    const int s0 = c << 5;
    // lane l computes the buffer row of slot s0 + l (-1: masked or padding)
    int myrow = -1;
    if (s0 + lane < w && pos >= 0) {
      const int raw = raw_index(rw, s0 + lane, t, omt);
      if (raw <= pos) {                                  // causal mask (:532)
        const int row = min(raw, p.kv_len - 1) - p.kv_offset;   // clamp (:615)
        if (row >= 0 && row < p.kv_rows) {
          myrow = row;
        } else if (p.err) {
          atomicOr(p.err, kErrKvRange);
        }
      }
    }
    int rows[LPR];
    uint4 kb[LPR], vb[LPR];
#pragma unroll
    for (int m = 0; m < LPR; ++m) {
      rows[m] = __shfl_sync(0xffffffffu, myrow, m * RPW + g);
      kb[m] = rows[m] >= 0 ? ldg16(Kb + (int64_t)rows[m] * p.sks) : make_uint4(0, 0, 0, 0);
      if constexpr (kKvTogether)
        vb[m] = rows[m] >= 0 ? ldg16(Vb + (int64_t)rows[m] * p.svs) : make_uint4(0, 0, 0, 0);
    }
    float part[LPR];
#pragma unroll
    for (int m = 0; m < LPR; ++m) part[m] = M::dot(qv, kb[m], 0.f);
    if constexpr (!kKvTogether) {
#pragma unroll
      for (int m = 0; m < LPR; ++m)
        vb[m] = rows[m] >= 0 ? ldg16(Vb + (int64_t)rows[m] * p.svs) : make_uint4(0, 0, 0, 0);
    }
    transpose_reduce<LPR>(part, lane);
    // this lane now holds the score of slot s0 + r * RPW + g
    const bool valid = __shfl_sync(0xffffffffu, myrow, r * RPW + g) >= 0;
    const float s = valid ? part[0] * p.scale_log2 : -INFINITY;
    const float mn = fmaxf(m_run, warp_max(s));
    if (mn == -INFINITY) continue;                      // whole sub-chunk masked
    const float corr = exp2f(m_run - mn);               // 0 on the first valid chunk
    const float e = exp2f(s - mn);
    l_run = l_run * corr + warp_sum(e);
    m_run = mn;
#pragma unroll
    for (int i = 0; i < EPL; ++i) acc[i] *= corr;
#pragma unroll
    for (int m = 0; m < LPR; ++m) {
      // the weight of slot s0 + m * RPW + g sits in lane g * LPR + m
      const float pm = __shfl_sync(0xffffffffu, e, g * LPR + m);
      axpy_f32<T>(pm, vb[m], acc);                      // pm = 0 for masked slots
    }
  }
  // sum the RPW row groups of the warp: lanes 0..LPR-1 hold D / LPR columns each
#pragma unroll
  for (int o = LPR; o < 32; o <<= 1)
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], o);

  T* orow = reinterpret_cast<T*>(p.o) + b * p.sob + h * p.soh + (int64_t)j * p.sos + r * EPL;
  float* lse = p.lse + ((int64_t)b * p.Hq + h) * p.n_rows + j;
  if (nw == 1) {
    if (lane < LPR) {
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) acc[e] *= inv;
      stg16(orow, V::from_float(acc));
    }
    if (lane == 0) *lse = (m_run == -INFINITY ? 0.f : m_run) + log2f(l_run);
    return;
  }
  if (lane < LPR) {
#pragma unroll
    for (int e = 0; e < EPL; ++e) s_acc[warp][r * EPL + e] = acc[e];
  }
  if (lane == 0) {
    s_ml[warp][0] = m_run;
    s_ml[warp][1] = l_run;
  }
  __syncthreads();
  if (warp != 0) return;
  const float mi = lane < nw ? s_ml[lane][0] : -INFINITY;
  const float mx = warp_max(mi);
  const float sc = (mi == -INFINITY) ? 0.f : exp2f(mi - mx);
  const float l = warp_sum(lane < nw ? s_ml[lane][1] * sc : 0.f);
  float out[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) out[e] = 0.f;
  for (int wi = 0; wi < nw; ++wi) {
    const float f = __shfl_sync(0xffffffffu, sc, wi);
    if (lane < LPR) {
#pragma unroll
      for (int e = 0; e < EPL; ++e) out[e] = fmaf(s_acc[wi][r * EPL + e], f, out[e]);
    }
  }
  if (lane < LPR) {
    const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) out[e] *= inv;
    stg16(orow, V::from_float(out));
  }
  if (lane == 0) *lse = (mx == -INFINITY ? 0.f : mx) + log2f(l);
}

}  // namespace esa
