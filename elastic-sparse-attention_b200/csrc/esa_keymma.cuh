// Backward, key side, on the tensor cores (bf16 / fp16, D = 64 or 128).
//
// dK[key] = sum over the key's users u of dS_u * q_u and dV[key] = sum of
// p_u * dO_u, where a user is a (query, head, slot) whose gathered index is
// the key (reference elastic_sparse_attention.py:535-545, the take_along_dim
// gather whose autograd backward is this scatter-add).  Every user belongs to
// exactly one key, so for a tile of 4 consecutive keys and a batch of 16
// users the sums are one mma.sync m16n8k16 per 16 dims and tensor:
//
//     D[dim, n] += Q^T[dim, user] * S[user, n],   n = part * 4 + key
//
// S[u, key] = hi(dS_u) and S[u, 4 + key] = lo(dS_u) for the user's key, 0
// elsewhere, with hi = round(x) and lo = round(x - hi) in the input type: the
// fp32 weights (p, dS from the workspace) enter with ~16 significant bits
// instead of the 8 (bf16) one rounding keeps, and dK[key] = D[:, key] +
// D[:, 4 + key] at the end.  Two non-zeros per row of S: 32 of the 128
// products of a (16 dims x 8 columns) output step are real work, still far
// cheaper per user than the FMA path's conversions, shuffles and bookkeeping.
// The q and dO rows of a batch's users are copied with cp.async into a
// swizzled shared-memory stage (16-byte chunk c of user x at chunk c ^ (x & 7),
// so the eight rows an ldmatrix phase reads sit in distinct banks) and read
// back transposed with ldmatrix.x4.trans, which yields the A fragments.
//
// Users are found per (head, slot) column: the index is non-decreasing along
// query positions, so a column's users of the keys [P0, P0 + 4) are one
// contiguous query range [a, b); a is the cursor left by the previous tile
// and b is found by galloping from a slope-based guess.  A launch covers
// kHeadsPerLaunch query heads of every group (its working set of q / dO rows
// and (p, dS) columns stays within a few L2 sizes); with more heads per
// group the launches add up in the fp32 workspace and the last one writes
// dK / dV in the input type.  Query chunks that use one key throughout (long
// runs, summed by bwd_heavy_kernel) are skipped and their partial sums added.
//
// Per tile: (A) every column's user range and a flat prefix of the counts,
// (B) all those users in one software pipeline, 32 per trip (user u ->
// column by a binary search over a 32-column window of the prefix), (C) the
// rare columns holding summed chunks.  With a key plan (PLANNED, built once
// per pattern by esa_keyplan.cuh) A-C are replaced by the tile's precomputed
// user records and summed-chunk records: no searches and no index
// arithmetic per user.  Warp = kTiles consecutive tiles of 4 keys; CTA =
// kWarps warps.
#pragma once
#include "esa_common.cuh"
#include "esa_params.h"

namespace esa {

template <typename T, int D>
struct KeyMma {
  static constexpr int kWarps = 4;
  static constexpr int kMinBlocks = 3;
  static constexpr int kKeys = 4;                         // keys per tile (MMA N = 2 x 4)
  static constexpr int kUsers = 16;                       // MMA K
  static constexpr int kTiles = 4;                        // key tiles per warp
  static constexpr int kRowBytes = D * (int)sizeof(T);
  static constexpr int kChunks = kRowBytes / 16;          // 16-byte chunks per row
  static constexpr int kUsersPerCopy = 32 / kChunks;      // users one cp.async step covers
  static constexpr int kUserBytes = 2 * kRowBytes;        // q row, then dO row
  static constexpr int kStageBytes = kUsers * kUserBytes;
  static constexpr int kRingBytes = 2 * kStageBytes;
  static constexpr int kEpRow = D + 4;                    // epilogue row (fp32), padded
  static constexpr int kMaxCols = 512;                    // G * w
  static constexpr int kMaxGroup = 16;                    // G (4 bits in the user word)
  static constexpr int kHeadsPerLaunch = 2;               // with an fp32 workspace (G > 1)
  static_assert(D == 64 || D == 128, "tensor-core key side is built for D = 64 and 128");
  static_assert(2 * kKeys * kEpRow * (int)sizeof(float) <= kRingBytes, "epilogue must fit the ring");
  // ints of per-column state per warp (2 arrays), a multiple of 4
  __host__ __device__ static constexpr int arrays(int cols) { return (2 * cols + 3) & ~3; }
  static size_t smem_bytes(int cols) {
    return (size_t)kWarps * (kRingBytes + arrays(cols) * sizeof(int));
  }
};

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&a)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
               : "r"(addr));
}

// d += a * b (m16n8k16, fp32 accumulate).  Not volatile: a pure function of
// its registers, so the compiler may interleave it with independent work.
template <typename T>
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// (lo, hi) rounded to T and packed, lo in the low half.
template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return Vec<T>::pack(lo, hi);
}
// One 16-bit value (low half of u) of type T as float.
template <typename T>
__device__ __forceinline__ float widen(uint32_t u) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return __uint_as_float(u << 16);
  else return __half2float(__ushort_as_half(static_cast<unsigned short>(u)));
}
template <typename T>
__device__ __forceinline__ T round_to(float x) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return __float2bfloat16_rn(x);
  else return __float2half_rn(x);
}

__device__ __forceinline__ void km_cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
// 16-byte copy global -> shared (L1 bypassed), zero-filled when !valid, with
// an L2 eviction policy for the source line.
__device__ __forceinline__ void km_cp_async16s(uint32_t smem_dst, const void* gmem_src, bool valid,
                                               uint64_t pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;" ::"r"(smem_dst),
               "l"(gmem_src), "r"(valid ? 16 : 0), "l"(pol)
               : "memory");
}
template <int N>
__device__ __forceinline__ void km_cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Column geometry of the key side.  A column is one (query head, slot) pair;
// its index is non-decreasing along query slots, so the users of a key range
// are one query range, found by searching the column.
struct KeyColumns {
  const AttnParams& p;
  int n, kvmax, w;
  __device__ __forceinline__ explicit KeyColumns(const AttnParams& pp)
      : p(pp), n(pp.n_rows), kvmax(pp.kv_len - 1), w(pp.pat.w) {}
  // key of query slot jq in column (k, t) (clamped like the forward, :615)
  __device__ __forceinline__ int cidx(int jq, int k, float t) const {
    return min(raw_index(row_window(p.pat, p.row_offset + jq), k, t, __fsub_rn(1.f, t)), kvmax);
  }
  // Approximate keys per query slot along a column (the index grows by
  // (1 - alpha) + (k + t) * alpha / w per position), for first guesses.
  __device__ __forceinline__ float slope(int k, float t) const {
    return fmaxf((1.f - p.pat.a) + (k + t) * p.pat.a / (float)w, 1e-6f);
  }
  // First slot q in [lo0, n) of column (k, t) whose key is >= target, given
  // that slot lo0 - 1 (if any) is below it; starts at the guess g and
  // gallops from there (down if g is already at or above the target, up
  // otherwise), then bisects.  val = the key at the result (or INT_MAX at n).
  __device__ __forceinline__ int find_first(int lo0, int g, int target, int k, float t,
                                            int& val) const {
    int lo = lo0 - 1, hi = n, hv = 0x7fffffff;
    if (lo0 < n) {
      g = min(max(g, lo0), n - 1);
      const int x = cidx(g, k, t);
      if (x >= target) {
        hi = g;
        hv = x;
        for (int step = 1; hi - step > lo; step <<= 1) {
          const int y = cidx(hi - step, k, t);
          if (y < target) { lo = hi - step; break; }
          hi -= step;
          hv = y;
        }
      } else {
        lo = g;
        for (int step = 1; lo + step < hi; step <<= 1) {
          const int y = cidx(lo + step, k, t);
          if (y >= target) { hi = lo + step; hv = y; break; }
          lo += step;
        }
      }
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        const int y = cidx(mid, k, t);
        if (y >= target) { hi = mid; hv = y; } else lo = mid;
      }
    }
    val = hi < n ? hv : 0x7fffffff;
    return hi;
  }
  // first query slot of column (k, t) whose key is >= P, searched from a guess:
  // the position whose key is about P, st + (k + t) * sp - t = P with
  // st = E (1 - alpha) - c and sp = (E alpha + c) / w, E = position + 1
  __device__ __forceinline__ int first_user(int P, int k, float t) const {
    const float num = (float)P + p.pat.c + t - (k + t) * p.pat.c / (float)w;
    const float gq = num / slope(k, t) - 1.f - (float)p.row_offset;
    const int g = (int)fminf(fmaxf(gq, 0.f), (float)n);
    int v;
    return find_first(0, g, P, k, t, v);
  }
  // is chunk ch of column (k, t) one key throughout (summed by bwd_heavy_kernel)?
  __device__ __forceinline__ bool constant_chunk(int ch, int k, float t) const {
    return cidx(ch * kHeavyChunk, k, t) == cidx(ch * kHeavyChunk + kHeavyChunk - 1, k, t);
  }
};

// Key plan records (esa_keyplan.cuh): user = column << 25 | (key - tile
// start) << 23 | query slot; summed chunk = column << 25 | (key - tile
// start) << 23 | chunk.  So a plan covers at most 2^23 query slots and 128
// columns per launch.
constexpr int kPlanSlotBits = 23;
constexpr uint32_t kPlanSlotMask = (1u << kPlanSlotBits) - 1u;
constexpr int kPlanColShift = 25;
constexpr int kPlanMaxCols = 1 << (32 - kPlanColShift);

template <typename T, int D, bool PLANNED>
__global__ void __launch_bounds__(KeyMma<T, D>::kWarps * 32, KeyMma<T, D>::kMinBlocks)
bwd_key_mma_kernel(const AttnParams p) {
  using C = KeyMma<T, D>;
  constexpr int MT = D / 16;                      // 16-dim MMA row tiles
  constexpr int UB = C::kUsers;
  constexpr int NK = C::kKeys;
  constexpr unsigned kAll = 0xffffffffu;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // this launch: query heads hh0 .. hh0 + GS - 1 of every group
  const int w = p.pat.w, G = p.G, GS = p.key_heads, hh0 = p.head_in_group;
  const int ncols = GS * w, nrounds = (ncols + 31) >> 5;
  unsigned char* ring = smem_raw + warp * C::kRingBytes;
  // per column: the cursor (first query slot whose key is >= the current
  // tile's first key; after step A of a tile, >= the next tile's) and the
  // exclusive prefix of the tile's streamed user counts
  int* scur = reinterpret_cast<int*>(smem_raw + C::kWarps * C::kRingBytes) + warp * C::arrays(ncols);
  int* soff = scur + ncols;
  const int hkv = blockIdx.y, b = blockIdx.z;
  const int lr0 = (blockIdx.x * C::kWarps + warp) * (C::kTiles * NK);
  if (lr0 >= p.kv_rows) return;
  if constexpr (PLANNED) {
    // a plan built for another problem: record it, write nothing
    if (p.plan_header[1] != p.plan_fp) {
      if (lane == 0 && p.err) atomicOr(p.err, kErrPlan);
      return;
    }
  }
  const int n = p.n_rows;
  // L2: the users' q / dO rows are re-read (a query row serves 64 keys spread
  // over the sweep); the (p, dS) workspace passes once
  const uint64_t pol_rows = l2_evict_last_policy();
  const uint64_t pol_stream = l2_evict_first_policy();
  // col -> (hh, k) with hh = col / w by a multiply-high (exact for col < 2^14, w <= 1024)
  const unsigned long long wmagic = 0xffffffffull / (unsigned)w + 1ull;
  // lane j (< GS) holds the head weight of query head hkv * G + hh0 + j
  const float lane_t = head_weight(p.pat, hkv * G + hh0 + (lane < GS ? lane : 0));
  const KeyColumns kc(p);
  // (hh, k, t, workspace column) of column col; every lane calls it (shuffle inside)
  struct Col {
    int hh, k, base;
    float t;
  };
  auto column = [&](int col) {
    Col c;
    const int j = (int)(((unsigned long long)(unsigned)col * wmagic) >> 32);
    c.hh = hh0 + j;
    c.k = col - j * w;
    c.t = __shfl_sync(kAll, lane_t, j & 31);
    c.base = (b * p.Hq + hkv * G + c.hh) * w + c.k;
    return c;
  };

  // Cursors: first query slot of each column whose key is >= the warp's first key.
  if constexpr (!PLANNED) {
    for (int cc = 0; cc < nrounds; ++cc) {
      const int col = cc * 32 + lane;
      const Col c = column(col < ncols ? col : 0);
      if (col < ncols) scur[col] = kc.first_user(p.kv_offset + lr0, c.k, c.t);
    }
  }

  const unsigned char* qbytes = reinterpret_cast<const unsigned char*>(
      reinterpret_cast<const T*>(p.q) + b * p.sqb + (int64_t)hkv * G * p.sqh);
  const unsigned char* dbytes = reinterpret_cast<const unsigned char*>(
      reinterpret_cast<const T*>(p.dout) + b * p.sdob + (int64_t)hkv * G * p.sdoh);
  // row strides in 16-byte units (the host checks the rows read stay below 2^32 units)
  constexpr int kPer16 = 16 / (int)sizeof(T);
  const uint32_t qs16 = (uint32_t)(p.sqs / kPer16), qh16 = (uint32_t)(p.sqh / kPer16);
  const uint32_t ds16 = (uint32_t)(p.sdos / kPer16), dh16 = (uint32_t)(p.sdoh / kPer16);
  // copy lanes: chunk cp_chunk of user m * kUsersPerCopy + cp_user
  const int cp_chunk = lane % C::kChunks, cp_user = lane / C::kChunks;
  const uint32_t cp_dst = (uint32_t)cp_user * C::kUserBytes;
  const unsigned char* qlane = qbytes + cp_chunk * 16;
  const unsigned char* dlane = dbytes + cp_chunk * 16;
  const int g4 = lane >> 2, t4 = lane & 3;           // MMA fragment coordinates
  const int lj = lane >> 3, lr = lane & 7;           // ldmatrix address coordinates
  const uint32_t ring_s = static_cast<uint32_t>(__cvta_generic_to_shared(ring));
  // this lane's ldmatrix row: user lr + 8 * (lj >> 1) of a stage
  const uint32_t lm_user = (uint32_t)(lr + ((lj >> 1) << 3)) * C::kUserBytes;
  // B-fragment column g4 = part * 4 + key (part 0: hi terms, 1: lo terms)
  const int bkey = g4 & 3;
  float acck[MT][4], accv[MT][4];

  for (int tile = 0; tile < C::kTiles; ++tile) {
    const int lt = lr0 + tile * NK;
    if (lt >= p.kv_rows) break;
    const int P0 = p.kv_offset + lt, P1 = P0 + NK;
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) { acck[i][e] = 0.f; accv[i][e] = 0.f; }
    // adds the partial sums of summed chunk chk of workspace column sbase
    // (heavy[(b * Hq + h) * w + k][chunk][{dK, dV}][D]) to key kk of the tile
    auto add_partials = [&](int sbase, int chk, int kk) {
      if (t4 != (kk >> 1)) return;
      const float* part = p.heavy + ((int64_t)sbase * p.heavy_chunks + chk) * (2 * D);
      const bool odd = kk & 1;
#pragma unroll
      for (int i = 0; i < MT; ++i) {
        const float k0 = part[16 * i + g4], k1 = part[16 * i + g4 + 8];
        const float v0 = part[D + 16 * i + g4], v1 = part[D + 16 * i + g4 + 8];
        if (odd) {
          acck[i][1] += k0; acck[i][3] += k1; accv[i][1] += v0; accv[i][3] += v1;
        } else {
          acck[i][0] += k0; acck[i][2] += k1; accv[i][0] += v0; accv[i][2] += v1;
        }
      }
    };

    // Streams `total` users through the MMAs.  resolve(t0, qi, key) -> Col of
    // user t0 + lane (and its query slot qi; with a plan also its key - P0);
    // every lane calls it, once per trip of 32 users, t0 = 0, 32, 64, ...  The
    // rows of a batch are in flight while the previous batch is multiplied.
    auto stream = [&](const int total, auto&& resolve) {
      if (total <= 0) return;
      // One trip = 32 users (lane l: user t0 + l) = two batches of UB: users
      // of lanes 0-15 (half 0) and 16-31 (half 1).  Per lane: its user's
      // (p, dS), key - P0 and q / dO rows in 16-byte units.
      struct U {
        float2 pd;
        int key;
        uint32_t oq, od;
      };
      int qi_f, key_f = 0;
      Col c_f;
      auto fetch = [&](int t0, U& r) {   // resolve, start the (p, dS) load
        const bool valid = t0 + lane < total;
        c_f = resolve(t0, qi_f, key_f);
        // past the end: slot 0 of column base 0 (in bounds), weights zeroed
        if (!valid) { qi_f = 0; c_f.hh = 0; c_f.base = 0; }
        const float2 pd = ldg_f2_hint(p.pds + (int64_t)c_f.base * n + qi_f, pol_stream);
        r.pd = valid ? pd : make_float2(0.f, 0.f);
        r.oq = (uint32_t)c_f.hh * qh16 + (uint32_t)qi_f * qs16;
        r.od = (uint32_t)c_f.hh * dh16 + (uint32_t)qi_f * ds16;
      };
      auto key_of = [&](int t0) {
        int key;
        if constexpr (PLANNED) key = key_f;
        else key = kc.cidx(qi_f, c_f.k, c_f.t) - P0;
        return t0 + lane < total ? key : 0;
      };
      // start the row copies of half h of trip t0 into stage st
      auto copies = [&](int t0, int h, int st, const U& r) {
        const uint32_t stage = ring_s + st * C::kStageBytes + cp_dst;
#pragma unroll
        for (int m = 0; m < UB / C::kUsersPerCopy; ++m) {
          const int x = m * C::kUsersPerCopy + cp_user;
          const uint32_t oq = __shfl_sync(kAll, r.oq, 16 * h + x);
          const uint32_t od = __shfl_sync(kAll, r.od, 16 * h + x);
          const bool ok = t0 + 16 * h + x < total;
          const uint32_t dst = stage + m * C::kUsersPerCopy * C::kUserBytes +
                               (((uint32_t)cp_chunk ^ (uint32_t)(x & 7)) << 4);
          km_cp_async16s(dst, qlane + (size_t)oq * 16u, ok, pol_rows);
          km_cp_async16s(dst + C::kRowBytes, dlane + (size_t)od * 16u, ok, pol_rows);
        }
        km_cp_async_commit();
      };
      // multiply half h of a trip, its rows in stage st
      auto compute = [&](int st, int h, const U& r) {
        const uint32_t hi = pack2<T>(r.pd.y, r.pd.x);
        const uint32_t lo = pack2<T>(r.pd.y - widen<T>(hi & 0xffffu), r.pd.x - widen<T>(hi >> 16));
        const unsigned c0 = __ballot_sync(kAll, r.key & 1);
        const unsigned c1 = __ballot_sync(kAll, r.key & 2);
        const unsigned mk = (((bkey & 1) ? c0 : ~c0) & ((bkey & 2) ? c1 : ~c1)) >> (16 * h + 2 * t4);
        const uint32_t m0 = ((mk & 1u) ? 0x0000ffffu : 0u) | ((mk & 2u) ? 0xffff0000u : 0u);
        const uint32_t m1 = ((mk & 0x100u) ? 0x0000ffffu : 0u) | ((mk & 0x200u) ? 0xffff0000u : 0u);
        const int src = 16 * h + 2 * t4;
        const bool lopart = g4 >= 4;
        const uint32_t h0 = __shfl_sync(kAll, hi, src), h1 = __shfl_sync(kAll, hi, src + 1);
        const uint32_t h2 = __shfl_sync(kAll, hi, src + 8), h3 = __shfl_sync(kAll, hi, src + 9);
        const uint32_t l0 = __shfl_sync(kAll, lo, src), l1 = __shfl_sync(kAll, lo, src + 1);
        const uint32_t l2 = __shfl_sync(kAll, lo, src + 8), l3 = __shfl_sync(kAll, lo, src + 9);
        const uint32_t v0 = lopart ? l0 : h0, v1 = lopart ? l1 : h1;
        const uint32_t v2 = lopart ? l2 : h2, v3 = lopart ? l3 : h3;
        const uint32_t bk0 = __byte_perm(v0, v1, 0x5410) & m0, bk1 = __byte_perm(v2, v3, 0x5410) & m1;
        const uint32_t bv0 = __byte_perm(v0, v1, 0x7632) & m0, bv1 = __byte_perm(v2, v3, 0x7632) & m1;
        const uint32_t sb = ring_s + st * C::kStageBytes + lm_user;
#pragma unroll
        for (int i = 0; i < MT; ++i) {
          const uint32_t co = (uint32_t)(((2 * i + (lj & 1)) ^ lr) << 4);
          uint32_t aq[4], ad[4];
          ldsm_x4_trans(sb + co, aq);
          ldsm_x4_trans(sb + C::kRowBytes + co, ad);
          mma_16816<T>(acck[i], aq, bk0, bk1);
          mma_16816<T>(accv[i], ad, bv0, bv1);
        }
      };
      // Trip t0 (state rc, its half 0 already copying into stage 0): copy
      // half 1, resolve trip t0 + 32 into rn, multiply both halves; returns
      // whether trip t0 + 32 has users.  Nothing in flight is moved between
      // registers: the two state sets alternate.
      auto trip = [&](const int t0, const U& rc, U& rn) {
        copies(t0, 1, 1, rc);                  // past the end: zero-filled, never read
        fetch(t0 + 32, rn);
        km_cp_async_wait<1>();
        __syncwarp();
        compute(0, 0, rc);
        __syncwarp();                          // stage 0 consumed before it is refilled
        copies(t0 + 32, 0, 0, rn);
        km_cp_async_wait<1>();
        __syncwarp();
        if (t0 + 16 < total) compute(1, 1, rc);
        rn.key = key_of(t0 + 32);
        __syncwarp();
        return t0 + 32 < total;
      };

      U r0, r1;
      fetch(0, r0);
      r0.key = key_of(0);
      copies(0, 0, 0, r0);
      for (int t0 = 0;; t0 += 64) {
        if (!trip(t0, r0, r1)) break;
        if (!trip(t0 + 32, r1, r0)) break;
      }
      km_cp_async_wait<0>();   // the zero-filled batches past the end
      __syncwarp();
    };

    if constexpr (PLANNED) {
      // the tile's users and summed chunks from the plan
      const int sg = hkv * p.plan_nlaunch + hh0 / p.plan_gs;
      const int ti = lt / NK;
      const int* us = p.plan_ustart + (int64_t)sg * (p.plan_ntiles + 1);
      const uint32_t* ur = p.plan_users + (int64_t)sg * p.plan_seg_users;
      // (every value read from the plan is clamped to its range, so even a
      // damaged plan cannot make an access leave the buffers)
      const int ub = min(max(us[ti], 0), (int)p.plan_seg_users);
      const int nu = min(max(us[ti + 1], ub), (int)p.plan_seg_users) - ub;
      stream(nu, [&](int t0, int& qi, int& key) {
        const int u = t0 + lane;
        const uint32_t rec = u < nu ? __ldg(ur + ub + u) : 0u;
        qi = min((int)(rec & kPlanSlotMask), n - 1);
        key = (int)((rec >> kPlanSlotBits) & 3u);
        return column(min((int)(rec >> kPlanColShift), ncols - 1));
      });
      const int* hs = p.plan_hstart + (int64_t)sg * (p.plan_ntiles + 1);
      const uint32_t* hr = p.plan_heavy + (int64_t)sg * p.plan_seg_heavy;
      const int hb = min(max(hs[ti], 0), (int)p.plan_seg_heavy);
      const int he = min(max(hs[ti + 1], hb), (int)p.plan_seg_heavy);
      for (int e = hb; e < he; ++e) {
        const uint32_t rec = __ldg(hr + e);
        const Col c = column(min((int)(rec >> kPlanColShift), ncols - 1));
        add_partials(c.base, min((int)(rec & kPlanSlotMask), p.heavy_chunks - 1),
                     (int)((rec >> kPlanSlotBits) & 3u));
      }
    } else {
      // ---- A: each column's users of [P0, P1): [scur_old, scur_new); flat
      // prefix of the counts streamed in B.  A column whose range holds a chunk
      // bwd_heavy_kernel summed streams nothing here (handled in C).
      int run = 0;
      bool any_heavy = false;
      for (int cc = 0; cc < nrounds; ++cc) {
        const int col = cc * 32 + lane;
        const bool ok = col < ncols;
        const Col c = column(ok ? col : 0);
        int s = 0, e = 0;
        bool heavy = false;
        if (ok) {
          s = scur[col];
          e = s;
          const int ev = s < n ? kc.cidx(s, c.k, c.t) : 0x7fffffff;   // key at the cursor
          if (ev < P1) {
            // first slot after s whose key is >= P1, from the slope's guess
            const float steps = (float)(P1 - ev) / kc.slope(c.k, c.t);
            const int g = s + (int)fminf(ceilf(steps), (float)n);
            int v;
            e = kc.find_first(s + 1, g, P1, c.k, c.t, v);
          }
          scur[col] = e;
          if (p.heavy_chunks > 0 && e - s >= kHeavyChunk) {
            const int cend = min(e / kHeavyChunk, p.heavy_chunks);
            for (int ch = (s + kHeavyChunk - 1) / kHeavyChunk; ch < cend && !heavy; ++ch)
              heavy = kc.constant_chunk(ch, c.k, c.t);
          }
        }
        const int len = heavy ? 0 : e - s;
        int off = len;
  #pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(kAll, off, o);
          if (lane >= o) off += y;
        }
        if (ok) soff[col] = run + off - len;
        run += __shfl_sync(kAll, off, 31);
        any_heavy |= __any_sync(kAll, heavy);
      }
      __syncwarp();

      // ---- B: the flat stream; user u -> the last column whose prefix is <= u.
      // Per trip (users t0 .. t0 + 31) the lanes load the prefixes of the 32
      // columns after an anchor column c0 (prefix <= t0) and each lane counts,
      // by a binary search over the lanes, those at or before its user.
      {
        int c0 = 0;
        // anchor c0: soff[c0] <= t0 at every trip
        stream(run, [&](int t0, int& qi, int&) {
          const int u = t0 + lane;
          const int cl = c0 + 1 + lane;
          const int bl = cl < ncols ? soff[cl] : 0x7fffffff;
          int col, nxt;   // nxt: prefix of the column after col
          if (__ballot_sync(kAll, bl <= t0 + 31) != kAll) {
            int pos = 0;   // window columns starting at or before u (bl is non-decreasing)
  #pragma unroll
            for (int sh = 16; sh >= 1; sh >>= 1) {
              const int v = __shfl_sync(kAll, bl, pos + sh - 1);
              if (v <= u) pos += sh;
            }
            col = c0 + pos;
            nxt = min(__shfl_sync(kAll, bl, pos), run);   // soff[col + 1], run past the end
            c0 += __popc(__ballot_sync(kAll, bl <= t0 + 32));
          } else {
            // more than 32 columns start inside the trip (empty columns): search
            int lo = c0, hi = ncols;   // soff[lo] <= u < soff[hi] (hi = ncols: end)
            while (hi - lo > 1) {
              const int mid = (lo + hi) >> 1;
              if (soff[mid] <= u) lo = mid; else hi = mid;
            }
            col = lo;
            nxt = col + 1 < ncols ? soff[col + 1] : run;
            c0 = __shfl_sync(kAll, col, 31);
          }
          // the column's users of this tile end at its cursor: [scur - len, scur)
          qi = scur[col] - nxt + u;
          return column(col);
        });
      }

      // ---- C: columns with summed chunks: the pieces between those chunks, then
      // the chunks' partial sums
      if (any_heavy) {
        for (int cc = 0; cc < nrounds; ++cc) {
          const int col = cc * 32 + lane;
          const bool ok = col < ncols;
          const Col c = column(ok ? col : 0);
          int cur = 0, e = 0;
          if (ok) {
            const int nxt = col + 1 < ncols ? soff[col + 1] : run;
            e = scur[col];
            if (nxt == soff[col] && e > 0)   // nothing streamed in B: empty or heavy
              cur = kc.first_user(P0, c.k, c.t);
            else
              cur = e;
          }
          while (__any_sync(kAll, cur < e)) {
            int seg_e = e, hc0 = 0, hc1 = 0;
            if (cur < e && p.heavy_chunks > 0 && e - cur >= kHeavyChunk) {
              int ch = (cur + kHeavyChunk - 1) / kHeavyChunk;
              const int cend = min(e / kHeavyChunk, p.heavy_chunks);
              while (ch < cend && !kc.constant_chunk(ch, c.k, c.t)) ++ch;
              if (ch < cend) {
                int ch2 = ch + 1;
                while (ch2 < cend && kc.constant_chunk(ch2, c.k, c.t)) ++ch2;
                seg_e = ch * kHeavyChunk;
                hc0 = ch;
                hc1 = ch2;
              }
            }
            const int len = cur < e ? seg_e - cur : 0;
            int off = len;
  #pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
              const int y = __shfl_up_sync(kAll, off, o);
              if (lane >= o) off += y;
            }
            const int total = __shfl_sync(kAll, off, 31);
            off -= len;
            stream(total, [&](int t0, int& qi, int&) {
              const int u = t0 + lane;
              int o = 0;
  #pragma unroll
              for (int sh = 16; sh >= 1; sh >>= 1) {
                const int cand = o + sh;
                if (__shfl_sync(kAll, off, cand) <= u) o = cand;
              }
              qi = __shfl_sync(kAll, cur, o) + (u - __shfl_sync(kAll, off, o));
              const int oc = cc * 32 + o;
              return column(oc < ncols ? oc : 0);
            });
            // partial sums of the skipped chunks, added to their key's hi column
            unsigned hm = __ballot_sync(kAll, hc1 > hc0);
            while (hm) {
              const int src = __ffs(hm) - 1;
              hm &= hm - 1;
              const int a = __shfl_sync(kAll, hc0, src);
              const int z = __shfl_sync(kAll, hc1, src);
              const int sk = __shfl_sync(kAll, c.k, src);
              const int sbase = __shfl_sync(kAll, c.base, src);
              const float stt = __shfl_sync(kAll, c.t, src);
              for (int chk = a; chk < z; ++chk)   // the key is the same on every lane
                add_partials(sbase, chk, kc.cidx(chk * kHeavyChunk, sk, stt) - P0);
            }
            cur = hc1 > hc0 ? hc1 * kHeavyChunk : e;
          }
        }
      }

    }

    // ---- epilogue: hi + lo columns (lanes t4 and t4 ^ 2) -> fp32 [2][4 keys][D]
    // in the ring (drained) -> global: dK / dV in T by the launch holding the
    // group's last heads, the fp32 sum of the heads so far otherwise
    {
#pragma unroll
      for (int i = 0; i < MT; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          acck[i][e] += __shfl_xor_sync(kAll, acck[i][e], 2);
          accv[i][e] += __shfl_xor_sync(kAll, accv[i][e], 2);
        }
      float* ep = reinterpret_cast<float*>(ring);
      if (t4 < 2) {
        const int k0 = 2 * t4;
#pragma unroll
        for (int i = 0; i < MT; ++i) {
          const int d0 = 16 * i + g4;
          ep[k0 * C::kEpRow + d0] = acck[i][0];
          ep[(k0 + 1) * C::kEpRow + d0] = acck[i][1];
          ep[k0 * C::kEpRow + d0 + 8] = acck[i][2];
          ep[(k0 + 1) * C::kEpRow + d0 + 8] = acck[i][3];
          ep[(NK + k0) * C::kEpRow + d0] = accv[i][0];
          ep[(NK + k0 + 1) * C::kEpRow + d0] = accv[i][1];
          ep[(NK + k0) * C::kEpRow + d0 + 8] = accv[i][2];
          ep[(NK + k0 + 1) * C::kEpRow + d0 + 8] = accv[i][3];
        }
      }
      __syncwarp();
      const bool first = hh0 == 0, last = hh0 + GS == G;
      const int64_t plane = (int64_t)p.B * p.Hkv * p.kv_rows * D;
      constexpr int kQuads = D / 4;
      constexpr int kOut = 2 * NK * kQuads;   // float4 pieces
#pragma unroll
      for (int idx = lane; idx < kOut; idx += 32) {
        const int tensor = idx / (NK * kQuads);
        const int rem = idx - tensor * (NK * kQuads);
        const int kr = rem / kQuads, qd = rem % kQuads;
        const int row = lt + kr;
        if (row < p.kv_rows) {
          float4 v = *reinterpret_cast<const float4*>(ep + (tensor * NK + kr) * C::kEpRow + 4 * qd);
          float* acc = p.acc + tensor * plane + (((int64_t)b * p.Hkv + hkv) * p.kv_rows + row) * D + 4 * qd;
          if (!first) {
            const float4 x = *reinterpret_cast<const float4*>(acc);
            v.x += x.x; v.y += x.y; v.z += x.z; v.w += x.w;
          }
          if (last) {
            const int64_t off = tensor == 0
                                    ? b * p.sdkb + hkv * p.sdkh + (int64_t)row * p.sdks + 4 * qd
                                    : b * p.sdvb + hkv * p.sdvh + (int64_t)row * p.sdvs + 4 * qd;
            void* base = tensor == 0 ? p.dk : p.dv;
            if (p.flags & kFlagF32Dkv)   // unrounded sums (ESA_FLAG_F32_DKV)
              *reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + off) = v;
            else
              *reinterpret_cast<uint2*>(reinterpret_cast<T*>(base) + off) =
                  make_uint2(pack2<T>(v.x, v.y), pack2<T>(v.z, v.w));
          } else {
            *reinterpret_cast<float4*>(acc) = v;
          }
        }
      }
      __syncwarp();
    }
  }
}

}  // namespace esa
