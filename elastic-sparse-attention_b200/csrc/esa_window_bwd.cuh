// Tensor-core (tcgen05) backward for sliding-window layers (alpha == 0): the
// backward of reference :169-233 / :300-339 for layer_idx 0, where every query
// i attends the causal window [max(0, i - w + 1), i] (see esa_window_tc.cuh).
// Two kernels, no atomics:
//
// window_bwd_dq_tc_kernel (query-major, the forward's tiling: HT heads x QT
// queries = 128 UMMA rows, NK = QT + w - 1 keys rounded up to 16, NK <= 96),
// persistent and warp-specialised like the forward (one CTA per SM, tiles
// blockIdx.x, blockIdx.x + gridDim.x, ...; 2 stages of Q/dS, dO, K, V in
// shared memory and of S, dP / dQ in TMEM; local tile i uses stage i & 1):
//   warp 8   TMA     Q, K (one barrier), dO, V (another) -> SMEM (128B swizzle)
//   warp 9   UMMA 1  S  = Q K^T                TMEM stage [0, NK)
//            UMMA 2  dP = dO V^T               TMEM stage [128, 128 + NK)
//            UMMA 3  dQ = dS K                 TMEM stage [0, 128) (S is read by then)
//            issued in whichever order their inputs become ready (polling)
//   warps 0-3 / 4-7 (one warpgroup per stage, one row per thread): P =
//            exp2(S * scale_log2 - lse) from TMEM, delta = sum_k P_k dP_k (equal
//            to rowsum(dO o O) for the exact O; stored for the second kernel),
//            dS = P (dP - delta) * scale, dS (input type) over the tile's Q in
//            SMEM, K-major over keys; then the tile's epilogue (dQ -> global).
//
// window_bwd_dkv_tc_kernel (key-major: 128 keys of one KV head; the queries
// that see them are positions [k0, k0 + 127 + w - 1], taken in chunks of 64
// for each of the G query heads of the group):
//   TMA      K, V [128 rows] once; Q, dO chunks [64 rows], double-buffered
//   UMMA 1   S^T  = K Q^T                  TMEM [0, 64) or [64, 128) (2 stages)
//   UMMA 2   dP^T = V dO^T                 TMEM [128, 192) or [192, 256)
//   threads  P^T, dS^T (input type) -> SMEM, K-major over queries (double-buffered)
//   UMMA 3   dV += P^T dO                  TMEM [256, 384)
//   UMMA 4   dK += dS^T Q                  TMEM [384, 512), summed over heads
//   epilogue dK, dV rows -> global in the input type
// The MMA thread issues UMMA 1/2 of chunk i + 1 before it waits for the
// threads' P^T / dS^T of chunk i, so the tensor core and the threads overlap.
// P^T and dS^T enter UMMA 3/4 rounded to the input type.  Queries near
// position 0 have fewer than w keys, so the weights of the first keys are
// large (up to 1) and their rounding error shows in dK / dV; a tile holding a
// key below w - 1 therefore makes a second pass over its chunks that adds the
// products of the rounding remainders (P^T - round(P^T), dS^T - round(dS^T)),
// which gives those sums ~16-bit weights.
//
// Every mbarrier wait is bounded; on a timeout the kernels record
// ESA_DEVERR_TIMEOUT, drain their copies and MMAs, free TMEM and return.
#pragma once
#include "esa_window_tc.cuh"

namespace esa {

struct WindowBwdTmaps {
  CUtensorMap q, k, v, dout;
};

constexpr int kWinBwdThreads = 160;
constexpr int kWinBwdTmemCols = 512;

// ---- dQ kernel (persistent) -------------------------------------------------
constexpr int kWbqMaxKeys = 96;                        // NK bound: two stages fit
constexpr int kWbqThreads = 320;
constexpr int kWbqStageQ = 2 * kWinRows * 128;         // Q, later dS (2 chunks of 64 keys)
constexpr int kWbqStageDO = 2 * kWinRows * 128;
constexpr int kWbqStageKV = 2 * kWbqMaxKeys * 128;     // K or V: 2 chunks of nk rows
constexpr int kWbqStageBytes = kWbqStageQ + kWbqStageDO + 2 * kWbqStageKV;
constexpr int kWbqSmemBytes = 2 * kWbqStageBytes + 1024 + 256;

template <typename T, int HT>
__global__ void __launch_bounds__(kWbqThreads, 1)
window_bwd_dq_tc_kernel(const __grid_constant__ WindowBwdTmaps maps, const AttnParams p, int nk,
                        int num_tiles, float* delta_out) {
  constexpr int QT = kWinRows / HT;
  constexpr uint32_t kFmt = std::is_same<T, __half>::value ? 0u : 1u;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  auto sQ = [&](int s) { return base + s * kWbqStageBytes; };   // Q, then dS
  auto sDO = [&](int s) { return base + s * kWbqStageBytes + kWbqStageQ; };
  auto sK = [&](int s) { return base + s * kWbqStageBytes + kWbqStageQ + kWbqStageDO; };
  auto sV = [&](int s) {
    return base + s * kWbqStageBytes + kWbqStageQ + kWbqStageDO + kWbqStageKV;
  };
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + 2 * kWbqStageBytes);
  uint64_t* full_a = bars + 0;     // [2] Q + K landed
  uint64_t* full_b = bars + 2;     // [2] dO + V landed
  uint64_t* sd_ready = bars + 4;   // [2] S and dP done
  uint64_t* ds_ready = bars + 6;   // [2] dS written, S / dP read (128 arrivals)
  uint64_t* dq_ready = bars + 8;   // [2] dQ done (the stage's SMEM is free)
  uint64_t* dq_free = bars + 10;   // [2] dQ read out of TMEM (128 arrivals)
  uint64_t* mma_done = bars + 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  volatile int* failed = reinterpret_cast<volatile int*>(bars + 14);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qtiles = (p.n_rows + QT - 1) / QT;
  const int groups_per_kv = p.G / HT;
  const int ygroups = p.Hkv * groups_per_kv;
  const int n_local =
      (int)blockIdx.x < num_tiles ? (num_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const uint32_t kv_bytes = 2u * nk * 128u;
  const uint32_t q_bytes = 2u * kWinRows * 128u;

  struct Tile {
    int j0, h0, hkv, b, ks;
  };
  auto tile_of = [&](int i) {
    const int tau = (int)blockIdx.x + i * (int)gridDim.x;
    const int qt = tau % qtiles;
    const int r = tau / qtiles;
    const int yg = r % ygroups;
    Tile t;
    t.b = r / ygroups;
    t.hkv = yg / groups_per_kv;
    t.h0 = t.hkv * p.G + (yg % groups_per_kv) * HT;
    t.j0 = qt * QT;
    t.ks = p.row_offset + t.j0 - (p.pat.w - 1);
    return t;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < 13; ++i) {
      const bool many = (i >= 6 && i < 8) || (i >= 10 && i < 12);
      sm100::mbar_init(bars + i, many ? 128 : 1);
    }
    *failed = 0;
    sm100::fence_mbar_init();
  }
  if (warp == 9) {
    sm100::tmem_alloc(tmem_slot, kWinBwdTmemCols);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ---- TMA producer ------------------------------------------------------
    if (lane == 0) {
      sm100::prefetch_tmap(&maps.q);
      sm100::prefetch_tmap(&maps.k);
      sm100::prefetch_tmap(&maps.v);
      sm100::prefetch_tmap(&maps.dout);
      int issued = 0;
      for (int i = 0; i < n_local; ++i) {
        const int s = i & 1;
        // stage s held tile i - 2: its dQ product (the last reader) must be done
        if (i >= 2 && !sm100::mbar_wait(dq_ready + s, ((i - 2) >> 1) & 1, kWinWaitIters)) {
          *failed = 1;
          break;
        }
        if (*failed) break;
        const Tile t = tile_of(i);
        const int kr = t.ks - p.kv_offset;
        sm100::mbar_expect_tx(full_a + s, q_bytes + kv_bytes);
        for (int c = 0; c < 2; ++c) {
          for (int ht = 0; ht < HT; ++ht)
            sm100::tma_load_4d(sQ(s) + c * (kWinRows * 128) + ht * QT * 128, &maps.q, full_a + s,
                               c * 64, t.j0, t.h0 + ht, t.b);
          sm100::tma_load_4d(sK(s) + c * (nk * 128), &maps.k, full_a + s, c * 64, kr, t.hkv, t.b);
        }
        sm100::mbar_expect_tx(full_b + s, q_bytes + kv_bytes);
        for (int c = 0; c < 2; ++c) {
          for (int ht = 0; ht < HT; ++ht)
            sm100::tma_load_4d(sDO(s) + c * (kWinRows * 128) + ht * QT * 128, &maps.dout,
                               full_b + s, c * 64, t.j0, t.h0 + ht, t.b);
          sm100::tma_load_4d(sV(s) + c * (nk * 128), &maps.v, full_b + s, c * 64, kr, t.hkv, t.b);
        }
        ++issued;
      }
      for (int i = issued > 2 ? issued - 2 : 0; i < issued; ++i) {
        sm100::mbar_wait(full_a + (i & 1), (i >> 1) & 1, kWinWaitIters);
        sm100::mbar_wait(full_b + (i & 1), (i >> 1) & 1, kWinWaitIters);
      }
    }
    __syncwarp();
  } else if (warp == 9) {
    // ---- MMA issuer: S(ns) / dP(ns) or dQ(no), whichever is ready -----------
    if (lane == 0) {
      const uint32_t idesc_s = sm100::instr_desc_f16(kWinRows, nk, kFmt, 0);
      const uint32_t idesc_q = sm100::instr_desc_f16(kWinRows, kWinHeadDim, kFmt, 1);
      int ns = 0, no = 0;
      uint32_t idle = 0;
      bool ok = true;
      while (no < n_local) {
        if (*failed) {
          ok = false;
          break;
        }
        bool progress = false;
        // S / dP of tile ns overwrite the TMEM columns dQ(ns - 2) was read from
        // and dP(ns - 2) (read before dS(ns - 2), which dQ(ns - 2) waited for)
        if (ns < n_local) {
          const int st = ns & 1, ph = (ns >> 1) & 1;
          if (sm100::mbar_test(full_a + st, ph) && sm100::mbar_test(full_b + st, ph) &&
              (ns < 2 || sm100::mbar_test(dq_free + st, ((ns - 2) >> 1) & 1))) {
            sm100::tc_fence_after();
            const uint32_t a = sm100::smem_u32(sQ(st)), bk = sm100::smem_u32(sK(st));
            const uint32_t ad = sm100::smem_u32(sDO(st)), bv = sm100::smem_u32(sV(st));
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const uint32_t off = (k >> 2) * (kWinRows * 128) + (k & 3) * 32;
              const uint32_t koff = (k >> 2) * (nk * 128) + (k & 3) * 32;
              sm100::umma_f16(tmem + st * 256, sm100::smem_desc_sw128(a + off, 16, 1024),
                              sm100::smem_desc_sw128(bk + koff, 16, 1024), idesc_s, k > 0);
              sm100::umma_f16(tmem + st * 256 + 128, sm100::smem_desc_sw128(ad + off, 16, 1024),
                              sm100::smem_desc_sw128(bv + koff, 16, 1024), idesc_s, k > 0);
            }
            sm100::umma_commit(sd_ready + st);
            ++ns;
            progress = true;
          }
        }
        // dQ(no) = dS K: dS K-major over keys in the Q buffer, K stored
        // [keys][dims] = N-contiguous for this product
        if (no < ns && sm100::mbar_test(ds_ready + (no & 1), (no >> 1) & 1)) {
          const int st = no & 1;
          sm100::tc_fence_after();
          const uint32_t a = sm100::smem_u32(sQ(st)), bk = sm100::smem_u32(sK(st));
          for (int k = 0; k < nk / 16; ++k) {
            const uint32_t off = (k >> 2) * (kWinRows * 128) + (k & 3) * 32;
            sm100::umma_f16(tmem + st * 256, sm100::smem_desc_sw128(a + off, 16, 1024),
                            sm100::smem_desc_sw128(bk + k * 16 * 128, nk * 128, 1024), idesc_q,
                            k > 0);
          }
          sm100::umma_commit(dq_ready + st);
          ++no;
          progress = true;
        }
        if (progress) {
          idle = 0;
        } else if (++idle > kWinPollIters) {
          ok = false;
          break;
        }
      }
      if (!ok) *failed = 1;
      sm100::umma_commit(mma_done);
      sm100::mbar_wait(mma_done, 0, kWinWaitIters);
    }
    __syncwarp();
  } else {
    // ---- warpgroup wg (warps 4 wg .. 4 wg + 3) takes the local tiles wg, wg + 2,
    // ... (stage wg); thread t owns row t = (ht, qi) ---------------------------
    const int wg = warp >> 2;
    const int t = threadIdx.x & 127;
    const int ht = t / QT, qi = t % QT;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int s = wg;
    bool ok = true;
    for (int i = wg; i < n_local; i += 2) {
      const int ph = (i >> 1) & 1;
      const Tile tl = tile_of(i);
      const int j = tl.j0 + qi;
      const int h = tl.h0 + ht;
      const bool live = j < p.n_rows;
      const int pos = p.row_offset + j;
      const int lo = max(0, pos - p.pat.w + 1) - tl.ks;   // valid key columns [lo, hi]
      const int hi = pos - tl.ks;
      const int64_t ix = ((int64_t)tl.b * p.Hq + h) * p.n_rows + j;
      const float lse = live ? p.lse[ix] : 0.f;
      ok = ok && __all_sync(0xffffffffu, sm100::mbar_wait(sd_ready + s, ph, kWinWaitIters)) &&
           !*failed;
      sm100::tc_fence_after();
      if (ok) {
        // two passes over the row's S / dP in TMEM, 32 keys at a time: the row
        // value delta = sum_k P_k dP_k with P = exp2(S * scale_log2 - lse)
        // (rowsum(dO o O) for the exact O: no O read, and no rounding of the
        // stored 16-bit O, which shows in dK of keys with few users), then
        // dS = P (dP - delta) * scale
        constexpr int kCh = kWbqMaxKeys / 32;
        float delta = 0.f;
#pragma unroll
        for (int pass = 0; pass < 2; ++pass) {
#pragma unroll
          for (int cc = 0; cc < kCh; ++cc) {
            if (cc * 32 < nk) {
              float sc[32], dp[32];
              sm100::tmem_ld_x32(tmem + s * 256 + lane_base + cc * 32, sc);
              sm100::tmem_ld_x32(tmem + s * 256 + 128 + lane_base + cc * 32, dp);
#pragma unroll
              for (int u8 = 0; u8 < 4; ++u8) {
                const int c8 = cc * 4 + u8;   // 8-key unit
                float ds[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                  const int c = c8 * 8 + u;
                  const bool valid = live && c < nk && c >= lo && c <= hi;
                  const float pr = valid ? exp2f(sc[u8 * 8 + u] * p.scale_log2 - lse) : 0.f;
                  if (pass == 0) delta += pr * dp[u8 * 8 + u];
                  else ds[u] = pr * (dp[u8 * 8 + u] - delta) * p.scale;
                }
                if (pass == 1 && c8 * 8 < nk) {
                  const int chunk = c8 >> 3, unit = c8 & 7;
                  unsigned char* dst =
                      sQ(s) + chunk * (kWinRows * 128) + t * 128 + ((unit ^ (t & 7)) << 4);
                  *reinterpret_cast<uint4*>(dst) = Vec<T>::from_float(ds);
                }
              }
            }
          }
          if (pass == 0 && live) delta_out[ix] = delta;
        }
      }
      sm100::fence_async_smem();
      sm100::tc_fence_before();
      sm100::mbar_arrive(ds_ready + s);

      // epilogue: dQ -> global
      ok = ok && __all_sync(0xffffffffu, sm100::mbar_wait(dq_ready + s, ph, kWinWaitIters)) &&
           !*failed;
      sm100::tc_fence_after();
      if (ok) {
        T* dqrow = reinterpret_cast<T*>(p.dq) + tl.b * p.sdqb + h * p.sdqh + (int64_t)j * p.sdqs;
#pragma unroll
        for (int c = 0; c < kWinHeadDim / 32; ++c) {
          float o[32];
          sm100::tmem_ld_x32(tmem + s * 256 + lane_base + c * 32, o);
          if (live) {
#pragma unroll
            for (int u = 0; u < 4; ++u) stg16(dqrow + c * 32 + u * 8, Vec<T>::from_float(o + u * 8));
          }
        }
      }
      sm100::tc_fence_before();
      sm100::mbar_arrive(dq_free + s);
    }
    if (!ok && p.err) atomicOr(p.err, kErrTimeout);
  }

  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, kWinBwdTmemCols);
  }
}

// ---- dK / dV kernel -----------------------------------------------------------
constexpr int kWbkKeys = 128;    // keys per CTA (UMMA M)
constexpr int kWbkQC = 64;       // queries per chunk (UMMA N of S^T, K of dV / dK)
constexpr int kWbkSlots = 3;     // Q / dO chunk ring: chunk i in use, i + 1 ready, i + 2 loading
constexpr int kWbkSmemKV = 2 * kWbkKeys * 128;     // K or V: 2 chunks x 128 rows x 128 B
constexpr int kWbkSmemQC = 2 * kWbkQC * 128;       // a Q or dO chunk: 2 chunks x 64 rows
constexpr int kWbkSmemPT = kWbkKeys * 128;         // P^T or dS^T: 128 rows x 64 queries
constexpr int kWbkSmemBytes = 2 * kWbkSmemKV + 2 * kWbkSlots * kWbkSmemQC + 4 * kWbkSmemPT +
                              1024 + 2 * kWbkSlots * kWbkQC * 4 + 128;

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
  unsigned char* sQc = sV + kWbkSmemKV;                 // [3] chunks of Q
  unsigned char* sDOc = sQc + kWbkSlots * kWbkSmemQC;   // [3] chunks of dO
  unsigned char* sPT = sDOc + kWbkSlots * kWbkSmemQC;   // [2] P^T
  unsigned char* sDST = sPT + 2 * kWbkSmemPT;           // [2] dS^T
  float* sLse = reinterpret_cast<float*>(sDST + 2 * kWbkSmemPT);   // [3][64]
  float* sDel = sLse + kWbkSlots * kWbkQC;                          // [3][64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDel + kWbkSlots * kWbkQC);
  uint64_t* bar_kv = bars + 0;
  uint64_t* bar_ld = bars + 1;       // [3] Q + dO chunk landed in slot
  uint64_t* s_ready = bars + 4;      // [2] S^T / dP^T of the stage done
  uint64_t* p_ready = bars + 6;      // [2] P^T / dS^T written, S^T / dP^T read (128 arrivals)
  uint64_t* chunk_free = bars + 8;   // [3] dV / dK products of the chunk slot done
  uint64_t* pt_free = bars + 11;     // [2] dV / dK products of the P^T stage done
  uint64_t* bar_done = bars + 13;    // every UMMA done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  volatile int* failed = reinterpret_cast<volatile int*>(bars + 15);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hkv = blockIdx.y, b = blockIdx.z;
  const int kr0 = blockIdx.x * kWbkKeys;       // first key row of the tile
  const int kp0 = p.kv_offset + kr0;           // its position
  const int w = p.pat.w;
  const int nch = (kWbkKeys - 1 + w + kWbkQC - 1) / kWbkQC;   // query chunks per head
  const int npass = p.G * nch;                                  // chunks per pass
  const int nit = npass * (kp0 < w - 1 ? 2 : 1);                // second pass: remainders
  const uint32_t chunk_bytes = 2u * kWbkSmemQC;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 14; ++i) sm100::mbar_init(bars + i, (i == 6 || i == 7) ? 128 : 1);
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
  // S^T of stage st at [64 st, 64 st + 64), dP^T at [128 + 64 st, ...)
  const uint32_t tDV = tmem + 256, tDK = tmem + 384;

  // iteration it -> (query head, chunk)
  auto chunk_row = [&](int it) { return kp0 + ((it % npass) % nch) * kWbkQC - p.row_offset; };
  auto chunk_head = [&](int it) { return hkv * p.G + (it % npass) / nch; };

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
        const int slot = it % kWbkSlots;
        sm100::mbar_expect_tx(bar_ld + slot, chunk_bytes);
        for (int c = 0; c < 2; ++c) {
          sm100::tma_load_4d(sQc + slot * kWbkSmemQC + c * (kWbkQC * 128), &maps.q, bar_ld + slot,
                             c * 64, chunk_row(it), chunk_head(it), b);
          sm100::tma_load_4d(sDOc + slot * kWbkSmemQC + c * (kWbkQC * 128), &maps.dout,
                             bar_ld + slot, c * 64, chunk_row(it), chunk_head(it), b);
        }
      };
      const uint32_t idesc_s = sm100::instr_desc_f16(kWbkKeys, kWbkQC, kFmt, 0);
      const uint32_t idesc_g = sm100::instr_desc_f16(kWbkKeys, kWinHeadDim, kFmt, 1);
      // S^T(it) = K Q^T and dP^T(it) = V dO^T into TMEM stage it & 1
      auto issue_s = [&](int it) {
        const int slot = it % kWbkSlots, st = it & 1;
        const uint32_t ak = sm100::smem_u32(sK), av = sm100::smem_u32(sV);
        const uint32_t bq = sm100::smem_u32(sQc + slot * kWbkSmemQC);
        const uint32_t bd = sm100::smem_u32(sDOc + slot * kWbkSmemQC);
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const uint32_t aoff = (s >> 2) * (kWbkKeys * 128) + (s & 3) * 32;
          const uint32_t boff = (s >> 2) * (kWbkQC * 128) + (s & 3) * 32;
          sm100::umma_f16(tmem + st * 64, sm100::smem_desc_sw128(ak + aoff, 16, 1024),
                          sm100::smem_desc_sw128(bq + boff, 16, 1024), idesc_s, s > 0);
          sm100::umma_f16(tmem + 128 + st * 64, sm100::smem_desc_sw128(av + aoff, 16, 1024),
                          sm100::smem_desc_sw128(bd + boff, 16, 1024), idesc_s, s > 0);
        }
        sm100::umma_commit(s_ready + st);
      };
      load_chunk(0);
      int issued_loads = 1;
      if (nit > 1) {
        load_chunk(1);
        issued_loads = 2;
      }
      bool ok = sm100::mbar_wait(bar_kv, 0, kWinWaitIters) &&
                sm100::mbar_wait(bar_ld + 0, 0, kWinWaitIters);
      if (ok) {
        sm100::tc_fence_after();
        issue_s(0);
      }
      for (int it = 0; it < nit && ok; ++it) {
        const int slot = it % kWbkSlots, st = it & 1;
        // the next chunk's products first, so the tensor core works while the
        // threads turn S^T(it) into P^T(it); its TMEM stage held S^T(it - 1),
        // read by the threads before the p_ready(it - 1) waited for below
        if (it + 1 < nit) {
          const int n1 = it + 1;
          ok = sm100::mbar_wait(bar_ld + n1 % kWbkSlots, (n1 / kWbkSlots) & 1, kWinWaitIters) &&
               !*failed;
          if (!ok) break;
          sm100::tc_fence_after();
          issue_s(n1);
        }
        // chunk it + 2 into the slot chunk it - 1 used
        if (it + 2 < nit) {
          const int n2 = it + 2;
          if (it >= 1) {
            ok = sm100::mbar_wait(chunk_free + n2 % kWbkSlots, ((it - 1) / kWbkSlots) & 1,
                                  kWinWaitIters);
            if (!ok) break;
          }
          load_chunk(n2);
          ++issued_loads;
        }
        ok = sm100::mbar_wait(p_ready + st, (it >> 1) & 1, kWinWaitIters) && !*failed;
        if (!ok) break;
        sm100::tc_fence_after();
        {
          const uint32_t apt = sm100::smem_u32(sPT + st * kWbkSmemPT);
          const uint32_t adst = sm100::smem_u32(sDST + st * kWbkSmemPT);
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
        sm100::umma_commit(chunk_free + slot);
        sm100::umma_commit(pt_free + st);
      }
      if (!ok) *failed = 1;
      sm100::umma_commit(bar_done);   // arrives once everything issued has completed
      sm100::mbar_wait(bar_done, 0, kWinWaitIters);
      if (*failed) {
        // the copies still in flight: at most the last kWbkSlots chunks and K / V
        sm100::mbar_wait(bar_kv, 0, kWinWaitIters);
        for (int it = issued_loads > kWbkSlots ? issued_loads - kWbkSlots : 0; it < issued_loads; ++it)
          sm100::mbar_wait(bar_ld + it % kWbkSlots, (it / kWbkSlots) & 1, kWinWaitIters);
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
      const int slot = it % kWbkSlots, st = it & 1;
      const int h = chunk_head(it);
      const int jq0 = chunk_row(it);   // query row of chunk column 0
      // stage lse and delta of the chunk's 64 queries (0 outside [0, n_rows));
      // the slot's previous chunk (it - 3) is done with them
      named_sync_compute();
      {
        const int qc = t & (kWbkQC - 1);
        const int jq = jq0 + qc;
        const bool in = jq >= 0 && jq < p.n_rows;
        const int64_t ix = ((int64_t)b * p.Hq + h) * p.n_rows + jq;
        if (t < kWbkQC) sLse[slot * kWbkQC + qc] = in ? p.lse[ix] : 0.f;
        else sDel[slot * kWbkQC + qc] = in ? delta_in[ix] : 0.f;
      }
      named_sync_compute();
      ok = ok && __all_sync(0xffffffffu,
                            sm100::mbar_wait(s_ready + st, (it >> 1) & 1, kWinWaitIters)) &&
           !*failed;
      // the stage's P^T / dS^T buffers were read by UMMA 3/4 of iteration it - 2
      if (it >= 2)
        ok = ok && __all_sync(0xffffffffu, sm100::mbar_wait(pt_free + st, ((it - 2) >> 1) & 1,
                                                            kWinWaitIters));
      sm100::tc_fence_after();
      if (ok) {
        unsigned char* pt_row = sPT + st * kWbkSmemPT + t * 128;
        unsigned char* dst_row = sDST + st * kWbkSmemPT + t * 128;
        const float* lse = sLse + slot * kWbkQC;
        const float* del = sDel + slot * kWbkQC;
        const bool remainder = it >= npass;   // second pass: the rounding remainders
#pragma unroll
        for (int cc = 0; cc < kWbkQC / 32; ++cc) {
          float sc[32], dp[32];
          sm100::tmem_ld_x32(tmem + st * 64 + lane_base + cc * 32, sc);
          sm100::tmem_ld_x32(tmem + 128 + st * 64 + lane_base + cc * 32, dp);
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
              pr[u] = valid ? exp2f(sc[u8 * 8 + u] * p.scale_log2 - lse[qc]) : 0.f;
              ds[u] = pr[u] * (dp[u8 * 8 + u] - del[qc]) * p.scale;
              if (remainder) {
                pr[u] -= static_cast<float>(from_f32<T>(pr[u]));
                ds[u] -= static_cast<float>(from_f32<T>(ds[u]));
              }
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
      sm100::mbar_arrive(p_ready + st);
    }
    const bool ok_o =
        __all_sync(0xffffffffu, sm100::mbar_wait(bar_done, 0, kWinWaitIters)) && ok && !*failed;
    sm100::tc_fence_after();
    if (ok_o) {
      const int64_t ok_ = b * p.sdkb + hkv * p.sdkh + (int64_t)(kr0 + t) * p.sdks;
      const int64_t ov_ = b * p.sdvb + hkv * p.sdvh + (int64_t)(kr0 + t) * p.sdvs;
      const bool f32 = p.flags & kFlagF32Dkv;   // unrounded sums (ESA_FLAG_F32_DKV)
      // 32 columns of a dK or dV row: input dtype, or fp32
      auto store32 = [&](void* base, int64_t off, const float* o) {
        if (f32) {
          float* dst = reinterpret_cast<float*>(base) + off;
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<float4*>(dst + 4 * u) = make_float4(o[4 * u], o[4 * u + 1],
                                                                  o[4 * u + 2], o[4 * u + 3]);
        } else {
          T* dst = reinterpret_cast<T*>(base) + off;
#pragma unroll
          for (int u = 0; u < 4; ++u) stg16(dst + u * 8, Vec<T>::from_float(o + u * 8));
        }
      };
#pragma unroll
      for (int c = 0; c < kWinHeadDim / 32; ++c) {
        float o[32];
        sm100::tmem_ld_x32(tDK + lane_base + c * 32, o);
        if (live_k) store32(p.dk, ok_ + c * 32, o);
        sm100::tmem_ld_x32(tDV + lane_base + c * 32, o);
        if (live_k) store32(p.dv, ov_ + c * 32, o);
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
