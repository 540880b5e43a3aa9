// Shared device code for the elastic sparse attention kernels (sm_100a).
//
// Index math: bit-exact restatement of the reference's pattern generator
// (elastic_sparse_attention.py:470-535).  torch evaluates that function in
// float32 with one rounding per operation and rounds half to even; the device
// code does the same with __fmul_rn / __fadd_rn / __fsub_rn / __fdiv_rn (never
// contracted into an FMA) and rintf (round to nearest even).  All integer <->
// float conversions are exact because positions are below 2^24 (checked by the
// host entry points).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <type_traits>

namespace esa {

constexpr float kLog2e = 1.4426950408889634f;

// Per-layer constants of the pattern (reference :476-499).
struct Pattern {
  int w;            // attention_length
  int num_heads;    // query heads H of the pattern (it is defined per query head)
  float a;          // f32(alpha), alpha = layer_idx / max(nl - 1, 1)          :488-489
  float c;          // f32(w * (1 - alpha)), the product taken in double        :496
  int head_offset;  // a launch's head h is pattern head head_offset + h (0 unless the
                    // caller runs a subset of the heads, e.g. one GPU's share)
};

// Start and spacing of the window of one query position (reference :482-499).
struct RowWin {
  int st;    // start_ids_base                                                :497
  float sp;  // spacing_base                                                  :498-499
};

__device__ __forceinline__ RowWin row_window(const Pattern& P, int pos) {
  const int end = pos > P.w - 1 ? pos : P.w - 1;                            // :483
  const float E = __int2float_rn(end + 1);                                  // :495
  const float pd = __fadd_rn(P.c, __fmul_rn(E, P.a));                       // :496
  float s = rintf(__fsub_rn(E, pd));                                        // :497 round
  s = s < 0.f ? 0.f : s;                                                    // :497 clamp
  RowWin r;
  r.st = __float2int_rz(s);
  r.sp = __fdiv_rn(__int2float_rn(end + 1 - r.st), __int2float_rn(P.w));    // :498-499
  return r;
}

// attention_indices_oversized[:, k] (reference :503-506)
__device__ __forceinline__ int oversized(const RowWin& r, int k) {
  return r.st + __float2int_rz(rintf(__fmul_rn(__int2float_rn(k), r.sp)));
}

// Head interpolation weight t = h / (H - 1) (reference :515-516) of the
// launch's head h, i.e. pattern head head_offset + h.
__device__ __forceinline__ float head_weight(const Pattern& P, int h) {
  return P.num_heads > 1
             ? __fdiv_rn(__int2float_rn(h + P.head_offset), __int2float_rn(P.num_heads - 1))
             : 0.f;
}

// Raw (unmasked, unclamped) index of slot k for a head with weight t:
// round(base * (1 - t) + shifted * t) with base = ov[k], shifted = ov[k+1] - 1
// (reference :510-511, :521-526).
__device__ __forceinline__ int raw_index(const RowWin& r, int k, float t, float omt) {
  const int ov0 = oversized(r, k);
  const int ov1 = oversized(r, k + 1);
  const float x = __fmul_rn(__int2float_rn(ov0), omt);
  const float y = __fmul_rn(__int2float_rn(ov1 - 1), t);
  return __float2int_rz(rintf(__fadd_rn(x, y)));
}

// ---------------------------------------------------------------------------
// 16-byte vector <-> float conversions for the three supported element types.
// ---------------------------------------------------------------------------
template <typename T> struct Vec;

template <> struct Vec<float> {
  static constexpr int kElems = 4;
  __device__ __forceinline__ static void to_float(const uint4& u, float* f) {
    f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
  }
  __device__ __forceinline__ static uint4 from_float(const float* f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]),
                      __float_as_uint(f[2]), __float_as_uint(f[3]));
  }
};

__device__ __forceinline__ void bf16x2_to_float(uint32_t u, float& lo, float& hi) {
  lo = __uint_as_float(u << 16);
  hi = __uint_as_float(u & 0xffff0000u);
}

template <> struct Vec<__nv_bfloat16> {
  static constexpr int kElems = 8;
  __device__ __forceinline__ static void to_float(const uint4& u, float* f) {
    bf16x2_to_float(u.x, f[0], f[1]); bf16x2_to_float(u.y, f[2], f[3]);
    bf16x2_to_float(u.z, f[4], f[5]); bf16x2_to_float(u.w, f[6], f[7]);
  }
  __device__ __forceinline__ static uint32_t pack(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static uint4 from_float(const float* f) {
    return make_uint4(pack(f[0], f[1]), pack(f[2], f[3]), pack(f[4], f[5]), pack(f[6], f[7]));
  }
};

template <> struct Vec<__half> {
  static constexpr int kElems = 8;
  __device__ __forceinline__ static void cvt2(uint32_t u, float& lo, float& hi) {
    __half2 h = *reinterpret_cast<__half2*>(&u);
    float2 f = __half22float2(h);
    lo = f.x; hi = f.y;
  }
  __device__ __forceinline__ static void to_float(const uint4& u, float* f) {
    cvt2(u.x, f[0], f[1]); cvt2(u.y, f[2], f[3]); cvt2(u.z, f[4], f[5]); cvt2(u.w, f[6], f[7]);
  }
  __device__ __forceinline__ static uint32_t pack(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static uint4 from_float(const float* f) {
    return make_uint4(pack(f[0], f[1]), pack(f[2], f[3]), pack(f[4], f[5]), pack(f[6], f[7]));
  }
};

// ---------------------------------------------------------------------------
// Arithmetic on one 16-byte vector with fp32 accumulation.  For bf16 / fp16
// data the products use the mixed-precision FMA (16-bit x 16-bit + fp32 ->
// fp32, full rate on sm_100), so no conversion instructions are issued; for
// fp32 data it is plain FFMA.
//   dot(a, b, acc)      -> acc + sum_e a[e] * b[e]
//   axpy(s, b, acc[])   -> acc[e] += s * b[e]   (s as from scalar(): rounded
//                          to the vector's type for 16-bit data)
// ---------------------------------------------------------------------------
template <typename T> struct Mix;

template <> struct Mix<float> {
  using Scalar = float;
  __device__ __forceinline__ static Scalar scalar(float s) { return s; }
  __device__ __forceinline__ static float to_float(Scalar s) { return s; }
  __device__ __forceinline__ static float dot(const uint4& a, const uint4& b, float acc) {
    acc = fmaf(__uint_as_float(a.x), __uint_as_float(b.x), acc);
    acc = fmaf(__uint_as_float(a.y), __uint_as_float(b.y), acc);
    acc = fmaf(__uint_as_float(a.z), __uint_as_float(b.z), acc);
    acc = fmaf(__uint_as_float(a.w), __uint_as_float(b.w), acc);
    return acc;
  }
  __device__ __forceinline__ static void axpy(Scalar s, const uint4& b, float* acc) {
    acc[0] = fmaf(s, __uint_as_float(b.x), acc[0]);
    acc[1] = fmaf(s, __uint_as_float(b.y), acc[1]);
    acc[2] = fmaf(s, __uint_as_float(b.z), acc[2]);
    acc[3] = fmaf(s, __uint_as_float(b.w), acc[3]);
  }
};

#define ESA_MIX16(NAME, PTXTYPE)                                                                  \
  __device__ __forceinline__ void NAME##_fma2(uint32_t a, uint32_t b, float& c0, float& c1) {     \
    asm("{\n\t.reg .b16 a0, a1, b0, b1;\n\t"                                                      \
        "mov.b32 {a0, a1}, %2;\n\tmov.b32 {b0, b1}, %3;\n\t"                                     \
        "fma.rn.f32." PTXTYPE " %0, a0, b0, %0;\n\t"                                             \
        "fma.rn.f32." PTXTYPE " %1, a1, b1, %1;\n\t}"                                            \
        : "+f"(c0), "+f"(c1)                                                                      \
        : "r"(a), "r"(b));                                                                        \
  }                                                                                               \
  __device__ __forceinline__ void NAME##_axpy2(uint16_t s, uint32_t b, float& c0, float& c1) {    \
    asm("{\n\t.reg .b16 b0, b1;\n\t"                                                            \
        "mov.b32 {b0, b1}, %3;\n\t"                                                               \
        "fma.rn.f32." PTXTYPE " %0, %2, b0, %0;\n\t"                                             \
        "fma.rn.f32." PTXTYPE " %1, %2, b1, %1;\n\t}"                                            \
        : "+f"(c0), "+f"(c1)                                                                      \
        : "h"(s), "r"(b));                                                                        \
  }
ESA_MIX16(bf16, "bf16")
ESA_MIX16(f16, "f16")
#undef ESA_MIX16

template <> struct Mix<__nv_bfloat16> {
  using Scalar = uint16_t;
  __device__ __forceinline__ static Scalar scalar(float s) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(s));
  }
  __device__ __forceinline__ static float to_float(Scalar s) {
    return __uint_as_float(static_cast<uint32_t>(s) << 16);
  }
  __device__ __forceinline__ static float dot(const uint4& a, const uint4& b, float acc) {
    float c1 = 0.f;
    bf16_fma2(a.x, b.x, acc, c1);
    bf16_fma2(a.y, b.y, acc, c1);
    bf16_fma2(a.z, b.z, acc, c1);
    bf16_fma2(a.w, b.w, acc, c1);
    return acc + c1;
  }
  __device__ __forceinline__ static void axpy(Scalar s, const uint4& b, float* acc) {
    bf16_axpy2(s, b.x, acc[0], acc[1]);
    bf16_axpy2(s, b.y, acc[2], acc[3]);
    bf16_axpy2(s, b.z, acc[4], acc[5]);
    bf16_axpy2(s, b.w, acc[6], acc[7]);
  }
};

template <> struct Mix<__half> {
  using Scalar = uint16_t;
  __device__ __forceinline__ static Scalar scalar(float s) {
    return __half_as_ushort(__float2half_rn(s));
  }
  __device__ __forceinline__ static float to_float(Scalar s) {
    return __half2float(__ushort_as_half(s));
  }
  __device__ __forceinline__ static float dot(const uint4& a, const uint4& b, float acc) {
    float c1 = 0.f;
    f16_fma2(a.x, b.x, acc, c1);
    f16_fma2(a.y, b.y, acc, c1);
    f16_fma2(a.z, b.z, acc, c1);
    f16_fma2(a.w, b.w, acc, c1);
    return acc + c1;
  }
  __device__ __forceinline__ static void axpy(Scalar s, const uint4& b, float* acc) {
    f16_axpy2(s, b.x, acc[0], acc[1]);
    f16_axpy2(s, b.y, acc[2], acc[3]);
    f16_axpy2(s, b.z, acc[4], acc[5]);
    f16_axpy2(s, b.w, acc[6], acc[7]);
  }
};

// acc[e] += s * b[e] with s in fp32 and the 16-byte vector b converted to
// fp32 (exact for every input type); for 16-bit data the products use the
// packed fma.rn.f32x2 (two lanes per instruction).  Used where many terms
// are summed (the key side of the backward), so s keeps full precision.
__device__ __forceinline__ void ffma2(float& c0, float& c1, float a0, float a1, float b0,
                                      float b1) {
  asm("{\n\t.reg .b64 ra, rb, rc;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%0, %1};\n\t"
      "fma.rn.f32x2 rc, ra, rb, rc;\n\tmov.b64 {%0, %1}, rc;\n\t}"
      : "+f"(c0), "+f"(c1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// Low bf16 half of a 32-bit word to fp32 on the FMA pipe: lo * 1 + (-0) is
// exact (and keeps the sign of zero), so half of a vector's conversions leave
// the integer pipe, which the shift / mask forms of the other half use.
__device__ __forceinline__ float bf16_lo_to_f32_fma(uint32_t u) {
  float f;
  asm("{\n\t.reg .b16 l, h, one;\n\t"
      "mov.b32 {l, h}, %1;\n\tmov.b16 one, 0x3F80;\n\t"
      "fma.rn.f32.bf16 %0, l, one, %2;\n\t}"
      : "=f"(f)
      : "r"(u), "f"(-0.0f));
  return f;
}

template <typename T>
__device__ __forceinline__ void axpy_f32(float s, const uint4& b, float* acc) {
  if constexpr (sizeof(T) == 4) {
    Mix<float>::axpy(s, b, acc);
  } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    const uint32_t w[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float lo = bf16_lo_to_f32_fma(w[i]);
      const float hi = __uint_as_float(w[i] & 0xffff0000u);
      ffma2(acc[2 * i], acc[2 * i + 1], s, s, lo, hi);
    }
  } else {
    float f[8];
    Vec<T>::to_float(b, f);
#pragma unroll
    for (int e = 0; e < 8; e += 2) ffma2(acc[e], acc[e + 1], s, s, f[e], f[e + 1]);
  }
}

// ---------------------------------------------------------------------------
// Counter-based random numbers for dropout: Philox4x32 with 10 rounds, as
// published by Salmon, Moraes, Dror and Shaw ("Parallel random numbers: as
// easy as 1, 2, 3", SC 2011): per round two 32x32->64 multiplications by the
// paper's constants and a xor with the key; the key advances by the paper's
// Weyl increments between rounds.  Pure function of (counter, key).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
#pragma unroll
  for (int i = 0; i < 10; ++i) {
    if (i) { k.x += 0x9E3779B9u; k.y += 0xBB67AE85u; }
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
  }
  return c;
}

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

__device__ __forceinline__ uint4 ldg16(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

// Read-only load that is not kept in L1 (streamed operands such as Q rows of
// the query being processed, or the output/gradient rows).
__device__ __forceinline__ uint4 ldg16_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

__device__ __forceinline__ void stg16(void* p, const uint4& v) {
  *reinterpret_cast<uint4*>(p) = v;
}

// L2 eviction-priority policies (createpolicy) for accesses that carry an
// L2::cache_hint: evict_last for data a kernel re-reads from L2 many times
// (the key side's q / dO rows), evict_first for data that passes once (the
// (p, dS) workspace, the forward's probabilities), so the streams do not push
// the re-read rows out.
__device__ __forceinline__ uint64_t l2_evict_last_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ float2 ldg_f2_hint(const float2* p, uint64_t pol) {
  float2 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.f32 {%0, %1}, [%2], %3;"
               : "=f"(r.x), "=f"(r.y)
               : "l"(p), "l"(pol));
  return r;
}
__device__ __forceinline__ float ldg_f32_hint(const float* p, uint64_t pol) {
  float r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.f32 %0, [%1], %2;"
               : "=f"(r)
               : "l"(p), "l"(pol));
  return r;
}
__device__ __forceinline__ void stg_f2_hint(float2* p, float2 v, uint64_t pol) {
  asm volatile("st.global.L1::no_allocate.L2::cache_hint.v2.f32 [%0], {%1, %2}, %3;" ::"l"(p),
               "f"(v.x), "f"(v.y), "l"(pol)
               : "memory");
}
__device__ __forceinline__ void stg_f32_hint(float* p, float v, uint64_t pol) {
  asm volatile("st.global.L1::no_allocate.L2::cache_hint.f32 [%0], %1, %2;" ::"l"(p), "f"(v),
               "l"(pol)
               : "memory");
}

// Butterfly "transpose-reduce": every lane of an aligned group of LPR lanes
// holds LPR partial sums v[0..LPR); afterwards lane r of the group holds in
// v[0] the total of index r over the group.  Costs LPR-1 shuffles per lane.
template <int LPR>
__device__ __forceinline__ void transpose_reduce(float* v, int lane) {
#pragma unroll
  for (int o = LPR / 2, n = LPR; o >= 1; o >>= 1, n >>= 1) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float send = upper ? v[i] : v[i + n / 2];
      const float keep = upper ? v[i + n / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
}

template <int LPR>
__device__ __forceinline__ float group_allreduce_sum(float x) {
#pragma unroll
  for (int o = LPR / 2; o >= 1; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

}  // namespace esa
