// Decoder-layer harness kernels (include/esa_layer.h): RMSNorm with a fused
// residual add, rotary position embedding in place, SwiGLU.  All of them move
// a few bytes per element and do little arithmetic, so they are written for
// HBM bandwidth: 16-byte vector loads and stores, one vector per thread per
// row, several rows in flight per CTA, float32 arithmetic and one rounding of
// each output to the storage type.
#pragma once
#include "esa_common.cuh"

namespace esa {
namespace layer {

constexpr int kNormRows = 2;       // rows per CTA iteration (loads in flight)
constexpr int kNormBwdCtas = 296;  // CTAs of the norm backward (2 per SM on B200)

// Sums v[0..R) over the CTA; red holds 32 * R floats.  Every thread returns
// the totals.  One barrier; callers alternate two red buffers between calls.
template <int R>
__device__ __forceinline__ void block_sum(float (&v)[R], float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int r = 0; r < R; ++r) v[r] = warp_sum(v[r]);
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < R; ++r) red[warp * R + r] = v[r];
  }
  __syncthreads();
  const int nw = blockDim.x >> 5;
#pragma unroll
  for (int r = 0; r < R; ++r) v[r] = 0.f;
  for (int wi = 0; wi < nw; ++wi) {
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] += red[wi * R + r];
  }
}

__device__ __forceinline__ uint4 ld16(const void* p) {
  return *reinterpret_cast<const uint4*>(p);
}

// y = (x [+ res]) * rstd * w; thread t owns elements [t*E, t*E + E) of each row.
template <typename T>
__global__ void __launch_bounds__(1024)
rmsnorm_fwd_kernel(int64_t n_rows, int dim, const T* __restrict__ x, const T* __restrict__ res,
                   T* __restrict__ h_out, const T* __restrict__ w, float eps, T* __restrict__ y,
                   float* __restrict__ rstd_out) {
  using V = Vec<T>;
  constexpr int E = V::kElems;
  constexpr int R = kNormRows;
  __shared__ float red[2][32 * R];
  const int t = threadIdx.x;
  const bool active = t * E < dim;
  const int64_t c = (int64_t)t * E;
  float wv[E];
  if (active) V::to_float(ldg16(w + c), wv);
  const float inv_dim = 1.f / (float)dim;
  int buf = 0;
  for (int64_t r0 = (int64_t)blockIdx.x * R; r0 < n_rows; r0 += (int64_t)gridDim.x * R) {
    float hv[R][E], ss[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int64_t row = r0 + r;
      ss[r] = 0.f;
      if (active && row < n_rows) {
        V::to_float(ldg16(x + row * dim + c), hv[r]);
        if (res) {
          float rv[E];
          V::to_float(ldg16(res + row * dim + c), rv);
#pragma unroll
          for (int e = 0; e < E; ++e) hv[r][e] += rv[e];
          const uint4 hq = V::from_float(hv[r]);   // the stored h is what the norm sees
          stg16(h_out + row * dim + c, hq);
          V::to_float(hq, hv[r]);
        }
#pragma unroll
        for (int e = 0; e < E; ++e) ss[r] = fmaf(hv[r][e], hv[r][e], ss[r]);
      }
    }
    block_sum<R>(ss, red[buf]);
    buf ^= 1;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int64_t row = r0 + r;
      if (row >= n_rows) break;
      const float rs = rsqrtf(ss[r] * inv_dim + eps);
      if (active) {
        float o[E];
#pragma unroll
        for (int e = 0; e < E; ++e) o[e] = hv[r][e] * rs * wv[e];
        stg16(y + row * dim + c, V::from_float(o));
      }
      if (t == 0) rstd_out[row] = rs;
    }
  }
}

// dh = dh_in + rstd (w dy - xhat mean(xhat w dy)); per-CTA partial dw.
template <typename T>
__global__ void __launch_bounds__(1024)
rmsnorm_bwd_kernel(int64_t n_rows, int dim, const T* __restrict__ h, const T* __restrict__ w,
                   const float* __restrict__ rstd, const T* __restrict__ dy, const T* dh_in,
                   T* dh, float* __restrict__ dw_part) {
  using V = Vec<T>;
  constexpr int E = V::kElems;
  constexpr int R = kNormRows;
  __shared__ float red[2][32 * R];
  const int t = threadIdx.x;
  const bool active = t * E < dim;
  const int64_t c = (int64_t)t * E;
  float wv[E], dwacc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) dwacc[e] = 0.f;
  if (active) V::to_float(ldg16(w + c), wv);
  const float inv_dim = 1.f / (float)dim;
  int buf = 0;
  for (int64_t r0 = (int64_t)blockIdx.x * R; r0 < n_rows; r0 += (int64_t)gridDim.x * R) {
    float xh[R][E], gv[R][E], s[R], rs[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int64_t row = r0 + r;
      s[r] = 0.f;
      rs[r] = row < n_rows ? rstd[row] : 0.f;
      if (active && row < n_rows) {
        V::to_float(ldg16(h + row * dim + c), xh[r]);
        V::to_float(ldg16(dy + row * dim + c), gv[r]);
#pragma unroll
        for (int e = 0; e < E; ++e) {
          xh[r][e] *= rs[r];
          s[r] = fmaf(xh[r][e] * wv[e], gv[r][e], s[r]);
        }
      }
    }
    block_sum<R>(s, red[buf]);
    buf ^= 1;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int64_t row = r0 + r;
      if (!active || row >= n_rows) continue;
      const float m = s[r] * inv_dim;
      float o[E];
      if (dh_in) {
        V::to_float(ld16(dh_in + row * dim + c), o);   // may alias dh: plain load
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) o[e] = 0.f;
      }
#pragma unroll
      for (int e = 0; e < E; ++e) {
        o[e] += rs[r] * (wv[e] * gv[r][e] - xh[r][e] * m);
        dwacc[e] = fmaf(gv[r][e], xh[r][e], dwacc[e]);
      }
      stg16(dh + row * dim + c, V::from_float(o));
    }
  }
  if (active) {
    float* part = dw_part + (int64_t)blockIdx.x * dim + c;
#pragma unroll
    for (int e = 0; e < E; ++e) part[e] = dwacc[e];
  }
}

// dw[c] = sum over CTAs of the partials (column per thread).
template <typename T>
__global__ void sum_partials_kernel(int parts, int dim, const float* __restrict__ part,
                                    T* __restrict__ out) {
  const int cidx = blockIdx.x * blockDim.x + threadIdx.x;
  if (cidx >= dim) return;
  float acc = 0.f;
  for (int b = 0; b < parts; ++b) acc += part[(int64_t)b * dim + cidx];
  out[cidx] = from_f32<T>(acc);
}

// In-place rotary embedding of the q and k rows of one (position, batch).
// grid = (L, B); smem = D floats: cos for i < D/2, then sign * sin.
template <typename T>
__global__ void __launch_bounds__(256)
rope_kernel(int D, T* q, int64_t sqb, int64_t sqh, int64_t sqs, int Hq, T* k, int64_t skb,
            int64_t skh, int64_t sks, int Hk, const int64_t* __restrict__ pos,
            const float* __restrict__ inv_freq, float sign) {
  using V = Vec<T>;
  constexpr int E = V::kElems;
  extern __shared__ float cs[];
  const int half = D >> 1;
  const int64_t l = blockIdx.x;
  const int b = blockIdx.y;
  const int64_t p = pos ? pos[l] : l;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float a = __fmul_rn((float)p, inv_freq[i]);
    float sn, cn;
    sincosf(a, &sn, &cn);
    cs[i] = cn;
    cs[half + i] = sign * sn;
  }
  __syncthreads();
  const int vph = half / E;
  const int total = (Hq + Hk) * vph;
  for (int tt = threadIdx.x; tt < total; tt += blockDim.x) {
    const int hh = tt / vph;
    const int i0 = (tt - hh * vph) * E;
    T* row = hh < Hq ? q + b * sqb + hh * sqh + l * sqs
                     : k + b * skb + (int64_t)(hh - Hq) * skh + l * sks;
    float x1[E], x2[E], o1[E], o2[E];
    V::to_float(ld16(row + i0), x1);
    V::to_float(ld16(row + half + i0), x2);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float cn = cs[i0 + e], sn = cs[half + i0 + e];
      o1[e] = x1[e] * cn - x2[e] * sn;
      o2[e] = x2[e] * cn + x1[e] * sn;
    }
    stg16(row + i0, V::from_float(o1));
    stg16(row + half + i0, V::from_float(o2));
  }
}

__device__ __forceinline__ float sigmoid_f(float g) { return 1.f / (1.f + expf(-g)); }

// out = silu(gate) * up; rows strided over the grid, vectors over the block.
template <typename T>
__global__ void __launch_bounds__(256)
swiglu_fwd_kernel(int64_t n_rows, int ffn, const T* __restrict__ gu, T* __restrict__ out) {
  using V = Vec<T>;
  constexpr int E = V::kElems;
  const int vpr = ffn / E;
  for (int64_t r = blockIdx.x; r < n_rows; r += gridDim.x) {
    const T* g_row = gu + r * 2 * ffn;
    for (int v = threadIdx.x; v < vpr; v += blockDim.x) {
      float g[E], u[E], o[E];
      V::to_float(ldg16_stream(g_row + v * E), g);
      V::to_float(ldg16_stream(g_row + ffn + v * E), u);
#pragma unroll
      for (int e = 0; e < E; ++e) o[e] = g[e] * sigmoid_f(g[e]) * u[e];
      stg16(out + r * ffn + v * E, V::from_float(o));
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
swiglu_bwd_kernel(int64_t n_rows, int ffn, const T* __restrict__ gu, const T* __restrict__ dout,
                  T* __restrict__ dgu, T* __restrict__ out_re) {
  using V = Vec<T>;
  constexpr int E = V::kElems;
  const int vpr = ffn / E;
  for (int64_t r = blockIdx.x; r < n_rows; r += gridDim.x) {
    const T* g_row = gu + r * 2 * ffn;
    T* d_row = dgu + r * 2 * ffn;
    for (int v = threadIdx.x; v < vpr; v += blockDim.x) {
      float g[E], u[E], d[E], dg[E], du[E], o[E];
      V::to_float(ldg16_stream(g_row + v * E), g);
      V::to_float(ldg16_stream(g_row + ffn + v * E), u);
      V::to_float(ldg16_stream(dout + r * ffn + v * E), d);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float s = sigmoid_f(g[e]);
        const float silu = g[e] * s;
        dg[e] = d[e] * u[e] * (s * (1.f + g[e] * (1.f - s)));
        du[e] = d[e] * silu;
        o[e] = silu * u[e];
      }
      stg16(d_row + v * E, V::from_float(dg));
      stg16(d_row + ffn + v * E, V::from_float(du));
      if (out_re) stg16(out_re + r * ffn + v * E, V::from_float(o));
    }
  }
}

}  // namespace layer
}  // namespace esa
