// Strided row copies for the sequence split's buffer layouts.
//
// No reference counterpart: the reference runs on one device.  The sequence
// split keeps each KV-head group's K / V rows in a [rows, B, heads, D] buffer
// (contiguous slices for the NCCL transfers) and its partial dK / dV in fp32
// in the same layout; the caller's tensors are [B, S, H, D].  Moving between
// the two is a copy of "rows" of row_elems contiguous elements laid out on a
// 3-level grid (n0, n1, n2) with their own element strides on each side.
//
// One warp copies one row at a time, each lane 16 bytes of output per step
// (8 16-bit elements), read as 16 bytes (same type) or 32 bytes (fp32,
// rounded to nearest even, as torch's casts round); the row's grid position is
// divided out once per row.  HBM-bound: 4 (16-bit copy) or 6 (fp32 -> 16-bit)
// bytes per element.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace esa {

struct RowCopyParams {
  const void* src;
  void* dst;
  int64_t n0, n1, n2;   // grid of rows
  int64_t s0, s1, s2;   // source strides, elements
  int64_t d0, d1, d2;   // destination strides, elements
  int64_t rows;         // n0 * n1 * n2
  int32_t row_vecs;     // 8-element vectors per row
};

constexpr int kRowCopyWarps = 8;

template <typename Tout>
__device__ __forceinline__ uint4 pack8(const float4& a, const float4& b);

template <>
__device__ __forceinline__ uint4 pack8<__nv_bfloat16>(const float4& a, const float4& b) {
  __nv_bfloat162 h[4] = {__floats2bfloat162_rn(a.x, a.y), __floats2bfloat162_rn(a.z, a.w),
                         __floats2bfloat162_rn(b.x, b.y), __floats2bfloat162_rn(b.z, b.w)};
  return *reinterpret_cast<const uint4*>(h);
}

template <>
__device__ __forceinline__ uint4 pack8<__half>(const float4& a, const float4& b) {
  __half2 h[4] = {__floats2half2_rn(a.x, a.y), __floats2half2_rn(a.z, a.w),
                  __floats2half2_rn(b.x, b.y), __floats2half2_rn(b.z, b.w)};
  return *reinterpret_cast<const uint4*>(h);
}

// Tin == Tout: a 16-bit copy; Tin == float: fp32 rounded to Tout.
template <typename Tin, typename Tout>
__global__ void __launch_bounds__(kRowCopyWarps * 32) copy_rows_kernel(const RowCopyParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (int64_t)blockIdx.x * kRowCopyWarps + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * kRowCopyWarps;
  for (int64_t r = warp0; r < p.rows; r += nwarps) {
    const int64_t i2 = r % p.n2;
    const int64_t r1 = r / p.n2;
    const int64_t i1 = r1 % p.n1;
    const int64_t i0 = r1 / p.n1;
    const Tin* __restrict__ src =
        reinterpret_cast<const Tin*>(p.src) + i0 * p.s0 + i1 * p.s1 + i2 * p.s2;
    Tout* __restrict__ dst = reinterpret_cast<Tout*>(p.dst) + i0 * p.d0 + i1 * p.d1 + i2 * p.d2;
    for (int v = lane; v < p.row_vecs; v += 32) {
      uint4 out;
      if constexpr (sizeof(Tin) == 4) {
        const float4* s4 = reinterpret_cast<const float4*>(src + v * 8);
        out = pack8<Tout>(__ldcs(s4), __ldcs(s4 + 1));
      } else {
        out = __ldcs(reinterpret_cast<const uint4*>(src + v * 8));
      }
      __stcs(reinterpret_cast<uint4*>(dst + v * 8), out);
    }
  }
}

}  // namespace esa
