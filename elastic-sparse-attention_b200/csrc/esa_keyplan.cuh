// Key plan: the tensor-core key side's user lists, built once per pattern.
//
// The key side (esa_keymma.cuh) finds, for every tile of 4 keys, the users
// of each (query head, slot) column by searching the column and evaluating
// the pattern's index for every user.  None of that depends on the data:
// it is a function of the pattern, the shapes and the offsets only, like the
// reference's index buffers built at module construction (reference
// :454-468).  key_plan_kernel runs the same searches once and stores the
// result; a backward given the plan reads, per tile, its user records and
// summed-chunk records instead.
//
// Layout of a plan (one device buffer, esa_key_plan_size bytes):
//   header   uint64 [32]: magic, fingerprint of the problem it was built for
//   ustart   int32 [S][ntiles + 1]: per segment, the first user record of
//            each tile (exclusive prefix; entry ntiles = the segment's total)
//   hstart   int32 [S][ntiles + 1]: likewise for summed-chunk records
//   users    uint32 [S][seg_users]: column << 25 | (key - P0) << 23 | slot
//   heavy    uint32 [S][seg_heavy]: column << 25 | (key - P0) << 23 | chunk
// with S = Hkv * nlaunch segments (KV head, launch of the key side's query
// heads), ntiles = ceil(kv_rows / 4), seg_users = gs * w * n_rows (every
// (query, head, slot) is at most one user) and seg_heavy = gs * w *
// heavy_chunks.  Within a tile the records follow the key kernel's own
// order: the columns without summed chunks in column order (slots
// ascending), then the pieces and chunks of the others, column by column.
//
// Build: key_plan_kernel<false> counts each tile's records into ustart /
// hstart, key_plan_scan_kernel turns the counts into starts, and
// key_plan_kernel<true> writes the records.
#pragma once
#include "esa_keymma.cuh"

namespace esa {

constexpr uint64_t kKeyPlanMagic = 0x314e414c504b5345ull;   // "ESKPLAN1"
constexpr int kKeyPlanHeaderWords = 32;
constexpr int kKeyPlanWarps = 4;
constexpr int kKeyPlanTiles = 4;      // tiles of 4 keys per warp (as the key kernel)
constexpr int kKeyPlanKeys = 4;

struct KeyPlanBuild {
  int gs, nlaunch, ntiles;
  int64_t seg_users, seg_heavy;
  int* ustart;
  int* hstart;
  uint32_t* users;
  uint32_t* heavy;
};

template <bool EMIT>
__global__ void __launch_bounds__(kKeyPlanWarps * 32)
key_plan_kernel(const AttnParams p, const KeyPlanBuild kb) {
  constexpr unsigned kAll = 0xffffffffu;
  extern __shared__ __align__(16) int plan_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int w = p.pat.w, G = p.G, hh0 = blockIdx.z * kb.gs, GS = min(kb.gs, G - hh0);
  const int ncols = GS * w, nrounds = (ncols + 31) >> 5;
  // per column: the cursor, and the start of the current tile's range
  // (bit-inverted when the column holds summed chunks in this tile)
  int* scur = plan_smem + warp * 2 * ncols;
  int* sbeg = scur + ncols;
  const int hkv = blockIdx.y;
  const int lr0 = (blockIdx.x * kKeyPlanWarps + warp) * (kKeyPlanTiles * kKeyPlanKeys);
  if (lr0 >= p.kv_rows) return;
  const KeyColumns kc(p);
  const unsigned long long wmagic = 0xffffffffull / (unsigned)w + 1ull;
  const float lane_t = head_weight(p.pat, hkv * G + hh0 + (lane < GS ? lane : 0));
  auto col_kt = [&](int col, int& k, float& t) {   // every lane calls it (shuffle inside)
    const int j = (int)(((unsigned long long)(unsigned)col * wmagic) >> 32);
    k = col - j * w;
    t = __shfl_sync(kAll, lane_t, j & 31);
  };
  const int sg = hkv * kb.nlaunch + blockIdx.z;
  int* us = kb.ustart + (int64_t)sg * (kb.ntiles + 1);
  int* hs = kb.hstart + (int64_t)sg * (kb.ntiles + 1);
  uint32_t* ur = kb.users + (int64_t)sg * kb.seg_users;
  uint32_t* hr = kb.heavy + (int64_t)sg * kb.seg_heavy;

  for (int cc = 0; cc < nrounds; ++cc) {
    const int col = cc * 32 + lane;
    int k;
    float t;
    col_kt(col < ncols ? col : 0, k, t);
    if (col < ncols) scur[col] = kc.first_user(p.kv_offset + lr0, k, t);
  }
  __syncwarp();

  for (int tile = 0; tile < kKeyPlanTiles; ++tile) {
    const int lt = lr0 + tile * kKeyPlanKeys;
    if (lt >= p.kv_rows) break;
    const int P0 = p.kv_offset + lt, P1 = P0 + kKeyPlanKeys;
    const int ti = lt / kKeyPlanKeys;
    const int ubase = EMIT ? us[ti] : 0, hbase = EMIT ? hs[ti] : 0;
    int un = 0, hn = 0;   // records of the tile so far (warp-uniform)
    // exclusive prefix of v over the lanes; total over the warp in tot
    auto lane_scan = [&](int v, int& tot) {
      int off = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(kAll, off, o);
        if (lane >= o) off += y;
      }
      tot = __shfl_sync(kAll, off, 31);
      return off - v;
    };
    auto user_rec = [&](int col, int q, int k, float t) {
      return ((uint32_t)col << kPlanColShift) |
             ((uint32_t)(kc.cidx(q, k, t) - P0) << kPlanSlotBits) | (uint32_t)q;
    };

    // columns without summed chunks: their whole range
    for (int cc = 0; cc < nrounds; ++cc) {
      const int col = cc * 32 + lane;
      const bool ok = col < ncols;
      int k;
      float t;
      col_kt(ok ? col : 0, k, t);
      int s = 0, e = 0;
      bool heavy = false;
      if (ok) {
        s = scur[col];
        e = s;
        const int ev = s < p.n_rows ? kc.cidx(s, k, t) : 0x7fffffff;   // key at the cursor
        if (ev < P1) {
          const float steps = (float)(P1 - ev) / kc.slope(k, t);
          const int g = s + (int)fminf(ceilf(steps), (float)p.n_rows);
          int v;
          e = kc.find_first(s + 1, g, P1, k, t, v);
        }
        scur[col] = e;
        if (p.heavy_chunks > 0 && e - s >= kHeavyChunk) {
          const int cend = min(e / kHeavyChunk, p.heavy_chunks);
          for (int ch = (s + kHeavyChunk - 1) / kHeavyChunk; ch < cend && !heavy; ++ch)
            heavy = kc.constant_chunk(ch, k, t);
        }
        sbeg[col] = heavy ? ~s : s;
      }
      const int len = heavy ? 0 : e - s;
      int tot;
      const int off = lane_scan(len, tot);
      if (EMIT)
        for (int q = s; q < s + len; ++q) ur[ubase + un + off + (q - s)] = user_rec(col, q, k, t);
      un += tot;
    }
    __syncwarp();

    // columns with summed chunks: the pieces between the chunks (users) and
    // the chunks themselves; counted first, then written at their offsets
    for (int cc = 0; cc < nrounds; ++cc) {
      const int col = cc * 32 + lane;
      const bool ok = col < ncols;
      int k;
      float t;
      col_kt(ok ? col : 0, k, t);
      const int sb = ok ? sbeg[col] : 0;
      const bool heavy = ok && sb < 0;
      const int s = heavy ? ~sb : 0, e = heavy ? scur[col] : 0;
      // visit(piece(a, b), chunk(c)) over the column's range
      auto walk = [&](auto&& piece, auto&& chunk) {
        int cur = s;
        while (cur < e) {
          int seg_e = e, hc0 = 0, hc1 = 0;
          if (e - cur >= kHeavyChunk) {
            int ch = (cur + kHeavyChunk - 1) / kHeavyChunk;
            const int cend = min(e / kHeavyChunk, p.heavy_chunks);
            while (ch < cend && !kc.constant_chunk(ch, k, t)) ++ch;
            if (ch < cend) {
              int ch2 = ch + 1;
              while (ch2 < cend && kc.constant_chunk(ch2, k, t)) ++ch2;
              seg_e = ch * kHeavyChunk;
              hc0 = ch;
              hc1 = ch2;
            }
          }
          piece(cur, seg_e);
          for (int chk = hc0; chk < hc1; ++chk) chunk(chk);
          cur = hc1 > hc0 ? hc1 * kHeavyChunk : e;
        }
      };
      int nu = 0, nh = 0;
      if (heavy) walk([&](int a, int b) { nu += b - a; }, [&](int) { ++nh; });
      int tu, th;
      const int ou = lane_scan(nu, tu), oh = lane_scan(nh, th);
      if (EMIT && heavy) {
        int iu = ubase + un + ou, ih = hbase + hn + oh;
        walk(
            [&](int a, int b) {
              for (int q = a; q < b; ++q) ur[iu++] = user_rec(col, q, k, t);
            },
            [&](int chk) {
              const int kk = kc.cidx(chk * kHeavyChunk, k, t) - P0;
              hr[ih++] = ((uint32_t)col << kPlanColShift) | ((uint32_t)kk << kPlanSlotBits) |
                         (uint32_t)chk;
            });
      }
      un += tu;
      hn += th;
    }
    __syncwarp();
    if (!EMIT && lane == 0) {
      us[ti] = un;
      hs[ti] = hn;
    }
  }
}

// Per segment (blockIdx.x): counts [0, ntiles) -> exclusive starts, entry
// ntiles = total; for ustart and hstart (blockIdx.y).
__global__ void __launch_bounds__(1024) key_plan_scan_kernel(KeyPlanBuild kb) {
  __shared__ int part[1024];
  int* a = (blockIdx.y ? kb.hstart : kb.ustart) + (int64_t)blockIdx.x * (kb.ntiles + 1);
  const int n = kb.ntiles;
  const int per = (n + 1023) / 1024;
  const int i0 = min(n, (int)threadIdx.x * per), i1 = min(n, i0 + per);
  int sum = 0;
  for (int i = i0; i < i1; ++i) sum += a[i];
  part[threadIdx.x] = sum;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {   // inclusive scan of the per-thread sums
    const int v = threadIdx.x >= o ? part[threadIdx.x - o] : 0;
    __syncthreads();
    part[threadIdx.x] += v;
    __syncthreads();
  }
  int run = part[threadIdx.x] - sum;
  for (int i = i0; i < i1; ++i) {
    const int c = a[i];
    a[i] = run;
    run += c;
  }
  if (threadIdx.x == 1023) a[n] = part[1023];
}

__global__ void key_plan_header_kernel(uint64_t* header, uint64_t fingerprint) {
  if (threadIdx.x < kKeyPlanHeaderWords)
    header[threadIdx.x] = threadIdx.x == 0 ? kKeyPlanMagic : threadIdx.x == 1 ? fingerprint : 0ull;
}

}  // namespace esa
