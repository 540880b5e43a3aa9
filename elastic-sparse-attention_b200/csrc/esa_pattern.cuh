// Pattern kernels: materialise the reference's (indices, causal mask) buffers
// and audit the per-slot monotonicity that the backward's key-side
// enumeration relies on.
#pragma once
#include "esa_common.cuh"

namespace esa {

// idx/mask [H, n, w] int64 (reference layout, :524-535).  Row r holds position
// rows[r] (or row_offset + r).  When kv_len > 0 the indices are clamped to
// [0, kv_len - 1] as _triton_forward does (:615); masked slots carry index 0
// before the clamp, exactly like the reference buffers (:533).
__global__ void pattern_kernel(Pattern P, int n, const int64_t* __restrict__ rows,
                               int row_offset, int kv_len, int64_t* __restrict__ idx_out,
                               int64_t* __restrict__ mask_out) {
  const int64_t total = (int64_t)P.num_heads * n * P.w;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int k = (int)(e % P.w);
    const int64_t hr = e / P.w;
    const int r = (int)(hr % n);
    const int h = (int)(hr / n);
    const int pos = rows ? (int)rows[r] : row_offset + r;
    const RowWin rw = row_window(P, pos);
    const float t = head_weight(P, h);
    const float omt = __fsub_rn(1.f, t);
    int id = raw_index(rw, k, t, omt);
    const bool ok = id <= pos;                                   // :532
    id = ok ? id : 0;                                            // :533
    if (kv_len > 0) id = min(max(id, 0), kv_len - 1);            // :615
    idx_out[e] = id;
    mask_out[e] = ok ? 1 : 0;
  }
}

// Counts (h, r, k) with raw_index(r) < raw_index(r - 1), r in [1, n): zero
// means every per-slot column is sorted along the query positions.
__global__ void audit_kernel(Pattern P, int n, unsigned long long* __restrict__ bad) {
  const int64_t total = (int64_t)P.num_heads * n * P.w;
  unsigned long long local = 0;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int k = (int)(e % P.w);
    const int64_t hr = e / P.w;
    const int r = (int)(hr % n);
    const int h = (int)(hr / n);
    if (r == 0) continue;
    const float t = head_weight(P, h);
    const float omt = __fsub_rn(1.f, t);
    const int a = raw_index(row_window(P, r - 1), k, t, omt);
    const int b = raw_index(row_window(P, r), k, t, omt);
    local += (b < a) ? 1ull : 0ull;
  }
  if (local) atomicAdd(bad, local);
}

}  // namespace esa
