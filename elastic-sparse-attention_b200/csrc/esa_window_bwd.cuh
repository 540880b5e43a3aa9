// Tensor-core (tcgen05) backward for sliding-window layers (alpha == 0): the
// backward of reference :169-233 / :300-339 for layer_idx 0, where every query
// i attends the causal window [max(0, i - w + 1), i] (see esa_window_tc.cuh).
// Two kernels, no atomics:
//
// window_bwd_dq_tc_kernel (query-major, the forward's tiling: HT heads x QT
// queries = 128 UMMA rows, NK = QT + w - 1 keys rounded up to 16):
//   TMA      Q, dO [128 rows], K, V [NK rows] -> SMEM (128B swizzle)
//   UMMA 1   S  = Q K^T                    TMEM [0, NK)
//   UMMA 2   dP = dO V^T                   TMEM [192, 192 + NK)
//   threads  P = exp2(S * scale_log2 - lse), dS = P (dP - delta) * scale with
//            delta = rowsum(dO o O) (computed from global while the MMAs run
//            and stored for the second kernel); dS (input type) into the Q
//            buffer, K-major over keys
//   UMMA 3   dQ = dS K                     TMEM [384, 512) -> global
//
// window_bwd_dkv_tc_kernel (key-major: 128 keys of one KV head; the queries
// that see them are positions [k0, k0 + 127 + w - 1], taken in chunks of 64
// for each of the G query heads of the group):
//   TMA      K, V [128 rows] once; Q, dO chunks [64 rows], double-buffered
//   UMMA 1   S^T  = K Q^T                  TMEM [0, 64)
//   UMMA 2   dP^T = V dO^T                 TMEM [64, 128)
//   threads  P^T, dS^T (input type) -> SMEM, K-major over queries (double-buffered)
//   UMMA 3   dV += P^T dO                  TMEM [128, 256)
//   UMMA 4   dK += dS^T Q                  TMEM [256, 384), summed over heads
//   epilogue dK, dV rows -> global in the input type
//
// One elected thread of warp 4 issues TMA and UMMA; warps 0-3 own one TMEM
// lane (row) each.  Every mbarrier wait is bounded; on a timeout the kernel
// records ESA_DEVERR_TIMEOUT, drains its copies, frees TMEM and returns.
#pragma once
#include "esa_window_tc.cuh"

namespace esa {

struct WindowBwdTmaps {
  CUtensorMap q, k, v, dout;
};

constexpr int kWinBwdThreads = 160;
constexpr int kWinBwdTmemCols = 512;
constexpr int kWinBwdMaxKeys = 192;

// ---- dQ kernel --------------------------------------------------------------
constexpr int kWbqSmemQ = 3 * kWinRows * 128;          // Q (2 chunks), later dS (3 chunks)
constexpr int kWbqSmemDO = 2 * kWinRows * 128;
constexpr int kWbqSmemKV = 2 * kWinBwdMaxKeys * 128;   // K, V: 2 chunks of nk rows each
constexpr int kWbqSmemBytes = kWbqSmemQ + kWbqSmemDO + 2 * kWbqSmemKV + 1024 + 256;

template <typename T, int HT>
__global__ void __launch_bounds__(kWinBwdThreads, 1)
window_bwd_dq_tc_kernel(const __grid_constant__ WindowBwdTmaps maps, const AttnParams p, int nk,
                        float* delta_out) {
  constexpr int QT = kWinRows / HT;
  constexpr uint32_t kFmt = std::is_same<T, __half>::value ? 0u : 1u;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sQ = base;   // Q, then dS
  unsigned char* sDO = sQ + kWbqSmemQ;
  unsigned char* sK = sDO + kWbqSmemDO;
  unsigned char* sV = sK + kWbqSmemKV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kWbqSmemKV);
  uint64_t* bar_qk = bars + 0;   // Q + K landed
  uint64_t* bar_dv = bars + 1;   // dO + V landed
  uint64_t* bar_s = bars + 2;    // UMMA 1 and 2 done
  uint64_t* bar_ds = bars + 3;   // dS written (128 arrivals)
  uint64_t* bar_dq = bars + 4;   // UMMA 3 done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 5);
  volatile int* failed = reinterpret_cast<volatile int*>(bars + 6);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups_per_kv = p.G / HT;
  const int hkv = blockIdx.y / groups_per_kv;
  const int h0 = hkv * p.G + (blockIdx.y % groups_per_kv) * HT;
  const int b = blockIdx.z;
  const int j0 = blockIdx.x * QT;
  const int i0 = p.row_offset + j0;
  const int ks = i0 - (p.pat.w - 1);   // position of key column 0
  const uint32_t kv_bytes = 2u * nk * 128u;
  const uint32_t q_bytes = 2u * kWinRows * 128u;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 5; ++i) sm100::mbar_init(bars + i, i == 3 ? 128 : 1);
    *failed = 0;
    sm100::fence_mbar_init();
  }
  if (warp == 4) {
    sm100::tmem_alloc(tmem_slot, kWinBwdTmemCols);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tP = tmem + 192, tQ = tmem + 384;

  if (warp == 4) {
    if (lane == 0) {
      sm100::prefetch_tmap(&maps.q);
      sm100::prefetch_tmap(&maps.k);
      sm100::prefetch_tmap(&maps.v);
      sm100::prefetch_tmap(&maps.dout);
      sm100::mbar_expect_tx(bar_qk, q_bytes + kv_bytes);
      for (int c = 0; c < 2; ++c) {
        for (int ht = 0; ht < HT; ++ht)
          sm100::tma_load_4d(sQ + c * (kWinRows * 128) + ht * QT * 128, &maps.q, bar_qk, c * 64,
                             j0, h0 + ht, b);
        sm100::tma_load_4d(sK + c * (nk * 128), &maps.k, bar_qk, c * 64, ks - p.kv_offset, hkv, b);
      }
      sm100::mbar_expect_tx(bar_dv, q_bytes + kv_bytes);
      for (int c = 0; c < 2; ++c) {
        for (int ht = 0; ht < HT; ++ht)
          sm100::tma_load_4d(sDO + c * (kWinRows * 128) + ht * QT * 128, &maps.dout, bar_dv,
                             c * 64, j0, h0 + ht, b);
        sm100::tma_load_4d(sV + c * (nk * 128), &maps.v, bar_dv, c * 64, ks - p.kv_offset, hkv, b);
      }
      const uint32_t idesc_s = sm100::instr_desc_f16(kWinRows, nk, kFmt, 0);
      bool ok = sm100::mbar_wait(bar_qk, 0, kWinWaitIters);
      if (ok) {
        sm100::tc_fence_after();
        const uint32_t a = sm100::smem_u32(sQ), bk = sm100::smem_u32(sK);
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const uint32_t off = (s >> 2) * (kWinRows * 128) + (s & 3) * 32;
          const uint32_t koff = (s >> 2) * (nk * 128) + (s & 3) * 32;
          sm100::umma_f16(tS, sm100::smem_desc_sw128(a + off, 16, 1024),
                          sm100::smem_desc_sw128(bk + koff, 16, 1024), idesc_s, s > 0);
        }
      }
      ok = ok && sm100::mbar_wait(bar_dv, 0, kWinWaitIters);
      if (ok) {
        sm100::tc_fence_after();
        const uint32_t a = sm100::smem_u32(sDO), bv = sm100::smem_u32(sV);
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const uint32_t off = (s >> 2) * (kWinRows * 128) + (s & 3) * 32;
          const uint32_t voff = (s >> 2) * (nk * 128) + (s & 3) * 32;
          sm100::umma_f16(tP, sm100::smem_desc_sw128(a + off, 16, 1024),
                          sm100::smem_desc_sw128(bv + voff, 16, 1024), idesc_s, s > 0);
        }
      } else {
        *failed = 1;
      }
      sm100::umma_commit(bar_s);   // arrives even when nothing was issued
      // UMMA 3: dQ = dS K; dS K-major over keys in the Q buffer, K stored
      // [keys][dims] = N-contiguous for this product.
      ok = ok && !*failed && sm100::mbar_wait(bar_ds, 0, kWinWaitIters);
      if (ok && !*failed) {
        sm100::tc_fence_after();
        const uint32_t idesc = sm100::instr_desc_f16(kWinRows, kWinHeadDim, kFmt, 1);
        const uint32_t a = sm100::smem_u32(sQ), bk = sm100::smem_u32(sK);
        for (int s = 0; s < nk / 16; ++s) {
          const uint32_t off = (s >> 2) * (kWinRows * 128) + (s & 3) * 32;
          sm100::umma_f16(tQ, sm100::smem_desc_sw128(a + off, 16, 1024),
                          sm100::smem_desc_sw128(bk + s * 16 * 128, nk * 128, 1024), idesc, s > 0);
        }
      } else {
        *failed = 1;
      }
      sm100::umma_commit(bar_dq);
      if (*failed) {
        sm100::mbar_wait(bar_qk, 0, kWinWaitIters);
        sm100::mbar_wait(bar_dv, 0, kWinWaitIters);
        if (p.err) atomicOr(p.err, kErrTimeout);
      }
    }
    __syncwarp();
  } else {
    // ---- warps 0..3: thread t owns row t = (ht, qi) -------------------------
    const int t = threadIdx.x;
    const int ht = t / QT, qi = t % QT;
    const int j = j0 + qi;
    const int h = h0 + ht;
    const bool live = j < p.n_rows;
    const int pos = p.row_offset + j;
    const int lo = max(0, pos - p.pat.w + 1) - ks;   // valid key columns [lo, hi]
    const int hi = pos - ks;
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    // delta = rowsum(dO o O) and lse while the loads and UMMAs run
    float delta = 0.f, lse = 0.f;
    if (live) {
      const T* orow = reinterpret_cast<const T*>(p.o) + b * p.sob + h * p.soh + (int64_t)j * p.sos;
      const T* drow =
          reinterpret_cast<const T*>(p.dout) + b * p.sdob + h * p.sdoh + (int64_t)j * p.sdos;
#pragma unroll 4
      for (int c = 0; c < kWinHeadDim / 8; ++c) delta = Mix<T>::dot(ldg16(orow + c * 8), ldg16(drow + c * 8), delta);
      lse = p.lse[((int64_t)b * p.Hq + h) * p.n_rows + j];
      delta_out[((int64_t)b * p.Hq + h) * p.n_rows + j] = delta;
    }
    const bool ok = __all_sync(0xffffffffu, sm100::mbar_wait(bar_s, 0, kWinWaitIters)) && !*failed;
    sm100::tc_fence_after();
    if (ok) {
      const int nch = (nk + 31) / 32;
      for (int cc = 0; cc < nch; ++cc) {
        float s[32], dp[32];
        sm100::tmem_ld_x32(tS + lane_base + cc * 32, s);
        sm100::tmem_ld_x32(tP + lane_base + cc * 32, dp);
#pragma unroll
        for (int u8 = 0; u8 < 4; ++u8) {
          const int c8 = cc * 4 + u8;   // 8-key unit
          if (c8 * 8 >= nk) break;
          float ds[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int c = c8 * 8 + u;
            const bool valid = live && c >= lo && c <= hi;
            const float pr = valid ? exp2f(s[u8 * 8 + u] * p.scale_log2 - lse) : 0.f;
            ds[u] = pr * (dp[u8 * 8 + u] - delta) * p.scale;
          }
          const int chunk = c8 >> 3, unit = c8 & 7;
          unsigned char* dst = sQ + chunk * (kWinRows * 128) + t * 128 + ((unit ^ (t & 7)) << 4);
          *reinterpret_cast<uint4*>(dst) = Vec<T>::from_float(ds);
        }
      }
    }
    sm100::fence_async_smem();
    sm100::mbar_arrive(bar_ds);

    const bool ok_q =
        __all_sync(0xffffffffu, sm100::mbar_wait(bar_dq, 0, kWinWaitIters)) && ok && !*failed;
    sm100::tc_fence_after();
    if (ok_q) {
      T* dqrow = reinterpret_cast<T*>(p.dq) + b * p.sdqb + h * p.sdqh + (int64_t)j * p.sdqs;
#pragma unroll
      for (int c = 0; c < kWinHeadDim / 32; ++c) {
        float o[32];
        sm100::tmem_ld_x32(tQ + lane_base + c * 32, o);
        if (live) {
#pragma unroll
          for (int u = 0; u < 4; ++u) stg16(dqrow + c * 32 + u * 8, Vec<T>::from_float(o + u * 8));
        }
      }
    } else if (p.err) {
      atomicOr(p.err, kErrTimeout);
    }
  }

  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, kWinBwdTmemCols);
  }
}

// ---- dK / dV kernel -----------------------------------------------------------
constexpr int kWbkKeys = 128;    // keys per CTA (UMMA M)
constexpr int kWbkQC = 64;       // queries per chunk (UMMA N of S^T, K of dV / dK)
constexpr int kWbkSmemKV = 2 * kWbkKeys * 128;     // K or V: 2 chunks x 128 rows x 128 B
constexpr int kWbkSmemQC = 2 * kWbkQC * 128;       // a Q or dO chunk: 2 chunks x 64 rows
constexpr int kWbkSmemPT = kWbkKeys * 128;         // P^T or dS^T: 128 rows x 64 queries
constexpr int kWbkSmemBytes = 2 * kWbkSmemKV + 4 * kWbkSmemQC + 4 * kWbkSmemPT + 1024 +
                              2 * 2 * kWbkQC * 4 + 256;

__device__ __forceinline__ void named_sync_compute() {
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

template <typename T>
__global__ void __launch_bounds__(kWinBwdThreads, 1)
window_bwd_dkv_tc_kernel(const __grid_constant__ WindowBwdTmaps maps, const AttnParams p,
                         const float* delta_in) {
  constexpr uint32_t kFmt = std::is_same<T, __half>::value ? 0u : 1u;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sK = base;
  unsigned char* sV = sK + kWbkSmemKV;
  unsigned char* sQc = sV + kWbkSmemKV;      // [2] chunks of Q
  unsigned char* sDOc = sQc + 2 * kWbkSmemQC;  // [2] chunks of dO
  unsigned char* sPT = sDOc + 2 * kWbkSmemQC;  // [2] P^T
  unsigned char* sDST = sPT + 2 * kWbkSmemPT;  // [2] dS^T
  float* sLse = reinterpret_cast<float*>(sDST + 2 * kWbkSmemPT);   // [2][64]
  float* sDel = sLse + 2 * kWbkQC;                                  // [2][64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDel + 2 * kWbkQC);
  uint64_t* bar_kv = bars + 0;
  uint64_t* bar_ld = bars + 1;     // [2]: Q + dO chunk landed in slot
  uint64_t* bar_s = bars + 3;      // UMMA 1 and 2 of the iteration done
  uint64_t* bar_p = bars + 4;      // P^T / dS^T written, S^T / dP^T read (128 arrivals)
  uint64_t* bar_free = bars + 5;   // [2]: UMMA 3 and 4 of the slot done
  uint64_t* bar_done = bars + 7;   // every UMMA done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);
  volatile int* failed = reinterpret_cast<volatile int*>(bars + 9);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hkv = blockIdx.y, b = blockIdx.z;
  const int kr0 = blockIdx.x * kWbkKeys;       // first key row of the tile
  const int kp0 = p.kv_offset + kr0;           // its position
  const int w = p.pat.w;
  const int nch = (kWbkKeys - 1 + w + kWbkQC - 1) / kWbkQC;   // query chunks per head
  const int nit = p.G * nch;
  const uint32_t chunk_bytes = 2u * kWbkSmemQC;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 8; ++i) sm100::mbar_init(bars + i, i == 4 ? 128 : 1);
    *failed = 0;
    sm100::fence_mbar_init();
  }
  if (warp == 4) {
    sm100::tmem_alloc(tmem_slot, kWinBwdTmemCols);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tST = tmem, tDP = tmem + 64, tDV = tmem + 128, tDK = tmem + 256;

  // iteration it -> (query head, chunk)
  auto chunk_row = [&](int it) { return kp0 + (it % nch) * kWbkQC - p.row_offset; };
  auto chunk_head = [&](int it) { return hkv * p.G + it / nch; };

  if (warp == 4) {
    if (lane == 0) {
      sm100::prefetch_tmap(&maps.q);
      sm100::prefetch_tmap(&maps.k);
      sm100::prefetch_tmap(&maps.v);
      sm100::prefetch_tmap(&maps.dout);
      sm100::mbar_expect_tx(bar_kv, 2u * kWbkSmemKV);
      for (int c = 0; c < 2; ++c) {
        sm100::tma_load_4d(sK + c * (kWbkKeys * 128), &maps.k, bar_kv, c * 64, kr0, hkv, b);
        sm100::tma_load_4d(sV + c * (kWbkKeys * 128), &maps.v, bar_kv, c * 64, kr0, hkv, b);
      }
      auto load_chunk = [&](int it) {
        const int slot = it & 1;
        sm100::mbar_expect_tx(bar_ld + slot, chunk_bytes);
        for (int c = 0; c < 2; ++c) {
          sm100::tma_load_4d(sQc + slot * kWbkSmemQC + c * (kWbkQC * 128), &maps.q, bar_ld + slot,
                             c * 64, chunk_row(it), chunk_head(it), b);
          sm100::tma_load_4d(sDOc + slot * kWbkSmemQC + c * (kWbkQC * 128), &maps.dout,
                             bar_ld + slot, c * 64, chunk_row(it), chunk_head(it), b);
        }
      };
      load_chunk(0);
      const uint32_t idesc_s = sm100::instr_desc_f16(kWbkKeys, kWbkQC, kFmt, 0);
      const uint32_t idesc_g = sm100::instr_desc_f16(kWbkKeys, kWinHeadDim, kFmt, 1);
      bool ok = sm100::mbar_wait(bar_kv, 0, kWinWaitIters);
      int issued_loads = 1;   // chunks whose copies were started
      for (int it = 0; it < nit && ok; ++it) {
        const int slot = it & 1;
        if (it + 1 < nit) {
          // slot^1 was last used by iteration it-1: its UMMA 3/4 must be done
          if (it >= 1) ok = sm100::mbar_wait(bar_free + (slot ^ 1), ((it - 1) >> 1) & 1, kWinWaitIters);
          if (!ok) break;
          load_chunk(it + 1);
          ++issued_loads;
        }
        ok = sm100::mbar_wait(bar_ld + slot, (it >> 1) & 1, kWinWaitIters);
        if (!ok) break;
        sm100::tc_fence_after();
        {
          const uint32_t ak = sm100::smem_u32(sK), av = sm100::smem_u32(sV);
          const uint32_t bq = sm100::smem_u32(sQc + slot * kWbkSmemQC);
          const uint32_t bd = sm100::smem_u32(sDOc + slot * kWbkSmemQC);
#pragma unroll
          for (int s = 0; s < 8; ++s) {
            const uint32_t aoff = (s >> 2) * (kWbkKeys * 128) + (s & 3) * 32;
            const uint32_t boff = (s >> 2) * (kWbkQC * 128) + (s & 3) * 32;
            sm100::umma_f16(tST, sm100::smem_desc_sw128(ak + aoff, 16, 1024),
                            sm100::smem_desc_sw128(bq + boff, 16, 1024), idesc_s, s > 0);
            sm100::umma_f16(tDP, sm100::smem_desc_sw128(av + aoff, 16, 1024),
                            sm100::smem_desc_sw128(bd + boff, 16, 1024), idesc_s, s > 0);
          }
        }
        sm100::umma_commit(bar_s);
        ok = sm100::mbar_wait(bar_p, it & 1, kWinWaitIters) && !*failed;
        if (!ok) break;
        sm100::tc_fence_after();
        {
          const uint32_t apt = sm100::smem_u32(sPT + slot * kWbkSmemPT);
          const uint32_t adst = sm100::smem_u32(sDST + slot * kWbkSmemPT);
          const uint32_t bq = sm100::smem_u32(sQc + slot * kWbkSmemQC);
          const uint32_t bd = sm100::smem_u32(sDOc + slot * kWbkSmemQC);
#pragma unroll
          for (int s = 0; s < kWbkQC / 16; ++s) {
            const uint32_t acc = (it > 0 || s > 0) ? 1u : 0u;
            sm100::umma_f16(tDV, sm100::smem_desc_sw128(apt + s * 32, 16, 1024),
                            sm100::smem_desc_sw128(bd + s * 16 * 128, kWbkQC * 128, 1024),
                            idesc_g, acc);
            sm100::umma_f16(tDK, sm100::smem_desc_sw128(adst + s * 32, 16, 1024),
                            sm100::smem_desc_sw128(bq + s * 16 * 128, kWbkQC * 128, 1024),
                            idesc_g, acc);
          }
        }
        sm100::umma_commit(bar_free + slot);
      }
      if (!ok) *failed = 1;
      sm100::umma_commit(bar_done);   // arrives once everything issued has completed
      if (*failed) {
        // unblock the compute warps (they wait on bar_s / bar_free with bounds
        // anyway) and drain the copies still in flight
        sm100::mbar_wait(bar_kv, 0, kWinWaitIters);
        for (int it = 0; it < issued_loads; ++it)
          sm100::mbar_wait(bar_ld + (it & 1), (it >> 1) & 1, kWinWaitIters);
        if (p.err) atomicOr(p.err, kErrTimeout);
      }
    }
    __syncwarp();
  } else {
    // ---- warps 0..3: thread t owns key row kr0 + t ---------------------------
    const int t = threadIdx.x;
    const int kpos = kp0 + t;
    const bool live_k = kr0 + t < p.kv_rows;
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    bool ok = true;
    for (int it = 0; it < nit; ++it) {
      const int slot = it & 1;
      const int h = chunk_head(it);
      const int jq0 = chunk_row(it);   // query row of chunk column 0
      // stage lse and delta of the chunk's 64 queries (0 outside [0, n_rows))
      named_sync_compute();            // everyone is done with this slot's stage (it - 2)
      {
        const int qc = t & (kWbkQC - 1);
        const int jq = jq0 + qc;
        const bool in = jq >= 0 && jq < p.n_rows;
        const int64_t ix = ((int64_t)b * p.Hq + h) * p.n_rows + jq;
        if (t < kWbkQC) sLse[slot * kWbkQC + qc] = in ? p.lse[ix] : 0.f;
        else sDel[slot * kWbkQC + qc] = in ? delta_in[ix] : 0.f;
      }
      named_sync_compute();
      ok = ok && __all_sync(0xffffffffu, sm100::mbar_wait(bar_s, it & 1, kWinWaitIters)) &&
           !*failed;
      // the slot's P^T / dS^T buffers were read by UMMA 3/4 of iteration it - 2
      if (it >= 2)
        ok = ok && __all_sync(0xffffffffu, sm100::mbar_wait(bar_free + slot, ((it - 2) >> 1) & 1,
                                                            kWinWaitIters));
      sm100::tc_fence_after();
      if (ok) {
        unsigned char* pt_row = sPT + slot * kWbkSmemPT + t * 128;
        unsigned char* dst_row = sDST + slot * kWbkSmemPT + t * 128;
        const float* lse = sLse + slot * kWbkQC;
        const float* del = sDel + slot * kWbkQC;
#pragma unroll
        for (int cc = 0; cc < kWbkQC / 32; ++cc) {
          float s[32], dp[32];
          sm100::tmem_ld_x32(tST + lane_base + cc * 32, s);
          sm100::tmem_ld_x32(tDP + lane_base + cc * 32, dp);
#pragma unroll
          for (int u8 = 0; u8 < 4; ++u8) {
            float pr[8], ds[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              const int qc = cc * 32 + u8 * 8 + u;
              const int jq = jq0 + qc;
              const int qpos = p.row_offset + jq;
              const bool valid = live_k && jq >= 0 && jq < p.n_rows && qpos >= kpos &&
                                 qpos <= kpos + w - 1;
              pr[u] = valid ? exp2f(s[u8 * 8 + u] * p.scale_log2 - lse[qc]) : 0.f;
              ds[u] = pr[u] * (dp[u8 * 8 + u] - del[qc]) * p.scale;
            }
            const int unit = cc * 4 + u8;   // 16-byte unit of the 128-byte row
            const int sw = (unit ^ (t & 7)) << 4;
            *reinterpret_cast<uint4*>(pt_row + sw) = Vec<T>::from_float(pr);
            *reinterpret_cast<uint4*>(dst_row + sw) = Vec<T>::from_float(ds);
          }
        }
      }
      sm100::tc_fence_before();
      sm100::fence_async_smem();
      sm100::mbar_arrive(bar_p);
    }
    const bool ok_o =
        __all_sync(0xffffffffu, sm100::mbar_wait(bar_done, 0, kWinWaitIters)) && ok && !*failed;
    sm100::tc_fence_after();
    if (ok_o) {
      T* dkrow = reinterpret_cast<T*>(p.dk) + b * p.sdkb + hkv * p.sdkh + (int64_t)(kr0 + t) * p.sdks;
      T* dvrow = reinterpret_cast<T*>(p.dv) + b * p.sdvb + hkv * p.sdvh + (int64_t)(kr0 + t) * p.sdvs;
#pragma unroll
      for (int c = 0; c < kWinHeadDim / 32; ++c) {
        float o[32];
        sm100::tmem_ld_x32(tDK + lane_base + c * 32, o);
        if (live_k) {
#pragma unroll
          for (int u = 0; u < 4; ++u) stg16(dkrow + c * 32 + u * 8, Vec<T>::from_float(o + u * 8));
        }
        sm100::tmem_ld_x32(tDV + lane_base + c * 32, o);
        if (live_k) {
#pragma unroll
          for (int u = 0; u < 4; ++u) stg16(dvrow + c * 32 + u * 8, Vec<T>::from_float(o + u * 8));
        }
      }
    } else if (p.err) {
      atomicOr(p.err, kErrTimeout);
    }
  }

  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, kWinBwdTmemCols);
  }
}

}  // namespace esa
