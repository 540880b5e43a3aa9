// Tensor-core (tcgen05) forward for sliding-window layers (alpha == 0).
//
// For layer_idx 0 the elastic pattern degenerates to the causal window
// {j : max(0, i - w + 1) <= j <= i} for every head (reference :496-526 with
// alpha = 0: spacing 1, base == shifted), exactly for positions < 2^21
// (the float32 head interpolation is then exact to well under 0.5).  All the
// query heads of a KV head read the same keys, so one tile is HT heads x QT
// consecutive queries as the M = 128 rows of a UMMA, and the NK = QT + w - 1
// (rounded up to 16) keys they need as N:
//
//   TMA:     Q [HT x QT rows, 128], K/V [NK rows, 128] -> SMEM (128B swizzle);
//            key rows before position 0 are zero-filled by the tensor map
//   UMMA 1:  S[128 x NK] = Q K^T             (TMEM)
//   softmax: one TMEM lane (row) per thread: mask, base-2 exp, row sums;
//            P (bf16/f16) written over the tile's Q in SMEM (128B swizzle)
//   UMMA 2:  O[128 x 128] = P V              (TMEM)
//   epilogue: O / rowsum -> global (o strides), base-2 LSE.
//
// The kernel is persistent and warp-specialised: one CTA per SM walks the
// tiles blockIdx.x, blockIdx.x + gridDim.x, ... with a 2-stage shared-memory
// ring (Q/P, K, V per stage) and two TMEM stages (S and O each); local tile i
// uses stage i & 1:
//   warp 8 (one thread)   TMA producer: stage s is reloaded for tile i once
//                         tile i-2's P V has completed;
//   warp 9 (one thread)   MMA issuer: polls for whichever is ready first,
//                         S(i) (its Q and K landed) or O(t) (P(t) written,
//                         O(t-2) read out of the TMEM stage), so a late load
//                         never holds back another tile's P V;
//   warps 0-3 / 4-7       two softmax + epilogue warpgroups, one per stage
//                         (the even / odd local tiles): softmax of tile i,
//                         then its epilogue once P V is done.
// So the loads of tile i+1, the QK^T of one tile, the softmax of the other,
// the P V and the epilogues overlap.  Every mbarrier wait is bounded; a
// timeout sets an error bit, each role stops, the CTA waits for its copies and
// MMAs in flight, frees TMEM and exits.
#pragma once
#include "esa_params.h"
#include "esa_sm100.cuh"

namespace esa {

struct WindowTmaps {
  CUtensorMap q;  // dims {D, n_rows, Hq, B},   box {64, QT, 1, 1}
  CUtensorMap k;  // dims {D, kv_rows, Hkv, B}, box {64, NK, 1, 1}
  CUtensorMap v;  // same as k
};

constexpr int kWinHeadDim = 128;
constexpr int kWinRows = 128;           // UMMA M
constexpr int kWinMaxKeys = 128;        // NK upper bound (w <= 129 - QT)
constexpr uint32_t kWinWaitIters = 1u << 22;
constexpr int kErrTimeout = 2;

// Persistent forward: 10 warps, 2 stages of Q/P (32 KB), K and V (32 KB each,
// room for kWinMaxKeys rows), TMEM stage s = S at [256 s, 256 s + NK), O at
// [256 s + 128, 256 s + 256).  One CTA per SM (the ring takes 192 KB).
constexpr int kWinThreads = 320;
constexpr uint32_t kWinPollIters = 1u << 26;   // bound of the MMA thread's polling loop
constexpr int kWinStages = 2;
constexpr int kWinTmemCols = 512;
constexpr int kWinStageQ = 2 * kWinRows * 128;
constexpr int kWinStageKV = 2 * kWinMaxKeys * 128;
constexpr int kWinStageBytes = kWinStageQ + 2 * kWinStageKV;
constexpr int kWinSmemBytes = kWinStages * kWinStageBytes + 1024 + 256;

template <typename T, int HT>
__global__ void __launch_bounds__(kWinThreads, 1)
window_fwd_tc_kernel(const __grid_constant__ WindowTmaps maps, const AttnParams p, int nk,
                     int num_tiles) {
  constexpr int QT = kWinRows / HT;
  constexpr uint32_t kFmt = std::is_same<T, __half>::value ? 0u : 1u;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  auto sQ = [&](int s) { return base + s * kWinStageBytes; };   // Q, then P
  auto sK = [&](int s) { return base + s * kWinStageBytes + kWinStageQ; };
  auto sV = [&](int s) { return base + s * kWinStageBytes + kWinStageQ + kWinStageKV; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + kWinStages * kWinStageBytes);
  uint64_t* full_qk = bars + 0;    // [2] Q + K of the stage landed
  uint64_t* full_v = bars + 2;     // [2] V landed
  uint64_t* s_ready = bars + 4;    // [2] S = Q K^T done
  uint64_t* p_ready = bars + 6;    // [2] P written, S read (128 arrivals)
  uint64_t* o_ready = bars + 8;    // [2] O = P V done (the stage's SMEM is free)
  uint64_t* o_free = bars + 10;    // [2] O read out of TMEM (128 arrivals)
  uint64_t* mma_done = bars + 12;  // every UMMA issued has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  volatile int* failed = reinterpret_cast<volatile int*>(bars + 14);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qtiles = (p.n_rows + QT - 1) / QT;
  const int groups_per_kv = p.G / HT;
  const int ygroups = p.Hkv * groups_per_kv;
  const int n_local =
      (int)blockIdx.x < num_tiles ? (num_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const uint32_t kv_bytes = 2u * nk * 128u;

  struct Tile {
    int j0, h0, hkv, b, ks;
  };
  // local tile i -> its queries, heads and first key position; consecutive
  // CTAs take consecutive query tiles of one head group (shared K/V in L2)
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
    sm100::tmem_alloc(tmem_slot, kWinTmemCols);
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
      int issued = 0;
      for (int i = 0; i < n_local; ++i) {
        const int s = i & 1;
        // stage s held tile i - 2: its P V (the last reader) must be done
        if (i >= 2 && !sm100::mbar_wait(o_ready + s, ((i - 2) >> 1) & 1, kWinWaitIters)) {
          *failed = 1;
          break;
        }
        if (*failed) break;
        const Tile t = tile_of(i);
        sm100::mbar_expect_tx(full_qk + s, kWinStageQ + kv_bytes);
        for (int c = 0; c < 2; ++c) {
          for (int ht = 0; ht < HT; ++ht)
            sm100::tma_load_4d(sQ(s) + c * (kWinRows * 128) + ht * QT * 128, &maps.q, full_qk + s,
                               c * 64, t.j0, t.h0 + ht, t.b);
          sm100::tma_load_4d(sK(s) + c * (nk * 128), &maps.k, full_qk + s, c * 64,
                             t.ks - p.kv_offset, t.hkv, t.b);
        }
        sm100::mbar_expect_tx(full_v + s, kv_bytes);
        for (int c = 0; c < 2; ++c)
          sm100::tma_load_4d(sV(s) + c * (nk * 128), &maps.v, full_v + s, c * 64,
                             t.ks - p.kv_offset, t.hkv, t.b);
        ++issued;
      }
      // only the last two tiles' copies can still be in flight (each earlier
      // stage reuse waited for its tile's MMAs, which waited for its copies)
      for (int i = issued > 2 ? issued - 2 : 0; i < issued; ++i) {
        sm100::mbar_wait(full_qk + (i & 1), (i >> 1) & 1, kWinWaitIters);
        sm100::mbar_wait(full_v + (i & 1), (i >> 1) & 1, kWinWaitIters);
      }
    }
    __syncwarp();
  } else if (warp == 9) {
    // ---- MMA issuer: issue S(ns) or O(no), whichever is ready ----------------
    if (lane == 0) {
      const uint32_t idesc_s = sm100::instr_desc_f16(kWinRows, nk, kFmt, 0);
      const uint32_t idesc_o = sm100::instr_desc_f16(kWinRows, kWinHeadDim, kFmt, 1);
      int ns = 0, no = 0;   // next tile whose S / O is issued
      uint32_t idle = 0;
      bool ok = true;
      while (no < n_local) {
        if (*failed) {
          ok = false;
          break;
        }
        bool progress = false;
        // S(ns) = Q K^T, K = 128 in 8 steps of 16 (32 bytes of a 128-byte row).
        // Its TMEM stage held S(ns - 2): read by the softmax before P(ns - 2),
        // which O(ns - 2) waited for, and tile ns's loads waited for O(ns - 2)
        if (ns < n_local && sm100::mbar_test(full_qk + (ns & 1), (ns >> 1) & 1)) {
          const int st = ns & 1;
          sm100::tc_fence_after();
          const uint32_t q_addr = sm100::smem_u32(sQ(st)), k_addr = sm100::smem_u32(sK(st));
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint32_t off = (k >> 2) * (kWinRows * 128) + (k & 3) * 32;
            const uint32_t koff = (k >> 2) * (nk * 128) + (k & 3) * 32;
            sm100::umma_f16(tmem + st * 256, sm100::smem_desc_sw128(q_addr + off, 16, 1024),
                            sm100::smem_desc_sw128(k_addr + koff, 16, 1024), idesc_s, k > 0);
          }
          sm100::umma_commit(s_ready + st);
          ++ns;
          progress = true;
        }
        // O(no) = P V, K = nk keys in steps of 16; V is N-major (dims contiguous)
        if (no < ns) {
          const int st = no & 1, ph = (no >> 1) & 1;
          if (sm100::mbar_test(p_ready + st, ph) && sm100::mbar_test(full_v + st, ph) &&
              (no < 2 || sm100::mbar_test(o_free + st, ((no - 2) >> 1) & 1))) {
            sm100::tc_fence_after();
            const uint32_t p_addr = sm100::smem_u32(sQ(st)), v_addr = sm100::smem_u32(sV(st));
            for (int k = 0; k < nk / 16; ++k) {
              const uint32_t poff = (k >> 2) * (kWinRows * 128) + (k & 3) * 32;
              sm100::umma_f16(tmem + st * 256 + 128,
                              sm100::smem_desc_sw128(p_addr + poff, 16, 1024),
                              sm100::smem_desc_sw128(v_addr + k * 16 * 128, nk * 128, 1024),
                              idesc_o, k > 0);
            }
            sm100::umma_commit(o_ready + st);
            ++no;
            progress = true;
          }
        }
        if (progress) {
          idle = 0;
        } else if (++idle > kWinPollIters) {
          ok = false;
          break;
        }
      }
      if (!ok) *failed = 1;
      sm100::umma_commit(mma_done);   // arrives once every UMMA issued has completed
      sm100::mbar_wait(mma_done, 0, kWinWaitIters);
    }
    __syncwarp();
  } else {
    // ---- softmax + epilogue: warpgroup wg (warps 4 wg .. 4 wg + 3) takes the
    // local tiles i = wg, wg + 2, ... (stage wg); thread t owns row t = (ht, qi)
    const int wg = warp >> 2;
    const int t = threadIdx.x & 127;
    const int ht = t / QT, qi = t % QT;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int s = wg;
    bool ok = true;
    for (int i = wg; i < n_local; i += 2) {
      const int ph = (i >> 1) & 1;
      const Tile tl = tile_of(i);
      const int pos = p.row_offset + tl.j0 + qi;
      const int lo = max(0, pos - p.pat.w + 1) - tl.ks;   // valid columns [lo, hi]
      const int hi = pos - tl.ks;
      // tcgen05.ld is warp-collective: every branch around it is warp-uniform
      ok = ok && __all_sync(0xffffffffu, sm100::mbar_wait(s_ready + s, ph, kWinWaitIters)) &&
           !*failed;
      sm100::tc_fence_after();
      float mx = -INFINITY, l = 0.f;
      if (ok) {
        // the maximum over the whole S row (kWinMaxKeys columns of the stage,
        // those past nk masked) with one TMEM wait; then P from two reloads of
        // half the row (a whole row held across the exponentials would spill)
        {
          float sc[kWinMaxKeys];
          sm100::tmem_ld_cols<kWinMaxKeys / 32>(tmem + s * 256 + lane_base, sc);
#pragma unroll
          for (int col = 0; col < kWinMaxKeys; ++col)
            if (col < nk && col >= lo && col <= hi) mx = fmaxf(mx, sc[col] * p.scale_log2);
        }
        const float m = mx == -INFINITY ? 0.f : mx;
        // P row over the tile's Q: K-major, 128B swizzle, 64 keys per chunk
#pragma unroll
        for (int hf = 0; hf < kWinMaxKeys / 64; ++hf) {
          if (hf * 64 < nk) {
            float sc[64];
            sm100::tmem_ld_cols<2>(tmem + s * 256 + lane_base + hf * 64, sc);
#pragma unroll
            for (int u8 = 0; u8 < 8; ++u8) {
              const int c8 = hf * 8 + u8;
              if (c8 * 8 < nk) {
                float e[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                  const int col = c8 * 8 + u;
                  const bool valid = col >= lo && col <= hi;
                  e[u] = valid ? exp2f(sc[u8 * 8 + u] * p.scale_log2 - m) : 0.f;
                  l += e[u];
                }
                const int chunk = c8 >> 3, unit = c8 & 7;
                unsigned char* dst =
                    sQ(s) + chunk * (kWinRows * 128) + t * 128 + ((unit ^ (t & 7)) << 4);
                *reinterpret_cast<uint4*>(dst) = Vec<T>::from_float(e);
              }
            }
          }
        }
        mx = m;
      }
      sm100::fence_async_smem();
      sm100::tc_fence_before();
      sm100::mbar_arrive(p_ready + s);

      // epilogue: O / l -> global, LSE
      ok = ok && __all_sync(0xffffffffu, sm100::mbar_wait(o_ready + s, ph, kWinWaitIters)) &&
           !*failed;
      sm100::tc_fence_after();
      if (ok) {
        const int j = tl.j0 + qi;
        const bool store = j < p.n_rows;
        const int h = tl.h0 + ht;
        const float inv = l > 0.f ? 1.f / l : 0.f;
        T* orow = reinterpret_cast<T*>(p.o) + tl.b * p.sob + h * p.soh + (int64_t)j * p.sos;
#pragma unroll
        for (int hf = 0; hf < kWinHeadDim / 64; ++hf) {
          float o[64];
          sm100::tmem_ld_cols<2>(tmem + s * 256 + 128 + lane_base + hf * 64, o);
#pragma unroll
          for (int u = 0; u < 64; ++u) o[u] *= inv;
          if (store) {
#pragma unroll
            for (int u = 0; u < 8; ++u) stg16(orow + hf * 64 + u * 8, Vec<T>::from_float(o + u * 8));
          }
        }
        if (store) p.lse[((int64_t)tl.b * p.Hq + h) * p.n_rows + j] = mx + log2f(l);
      }
      sm100::tc_fence_before();
      sm100::mbar_arrive(o_free + s);
    }
    if (!ok && p.err) atomicOr(p.err, kErrTimeout);
  }

  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, kWinTmemCols);
  }
}

}  // namespace esa
