// Launch parameters shared by the host entry points and the kernels.
#pragma once
#include <stdint.h>

#include "esa_common.cuh"

namespace esa {

struct AttnParams {
  // Shapes.
  int B, Hq, Hkv, G, D;
  int n_rows;     // query rows handed to the launch (Lq, or len(cache_position))
  int kv_len;     // kv_seq_len of the call: indices are clamped to kv_len - 1 (reference :615)
  int kv_offset;  // absolute position held by row 0 of the k/v (and dk/dv) buffers
  int kv_rows;    // rows present in the k/v buffers
  int row_offset; // position of query row j is row_offset + j when rows == nullptr
  const int64_t* rows;  // optional explicit positions [n_rows] (decode: cache_position)
  Pattern pat;
  float scale;       // softmax scale (reference self.scaling = head_dim ** -0.5, :444)
  float scale_log2;  // scale * log2(e)

  // Forward operands; strides are in elements, the head_dim axis is contiguous.
  const void* q; int64_t sqb, sqh, sqs;
  const void* k; int64_t skb, skh, sks;
  const void* v; int64_t svb, svh, svs;
  void* o;       int64_t sob, soh, sos;
  float* lse;    // [B, Hq, n_rows] base-2 log-sum-exp of the scaled scores

  // Backward operands.
  const void* dout; int64_t sdob, sdoh, sdos;
  void* dq;         int64_t sdqb, sdqh, sdqs;
  void* dk;         int64_t sdkb, sdkh, sdks;
  void* dv;         int64_t sdvb, sdvh, sdvs;
  float2* pds;      // workspace [B, Hq, w, n_rows]: (p, dS * scale) per (row, slot)
  float* acc;       // workspace fp32 [2, B, Hkv, kv_rows, D] (only when G > 1)
  const int64_t* sorted_rows;  // optional positions sorted ascending (key side)
  const int64_t* row_perm;     // optional: sorted slot -> query row of the tensors
  int head_in_group;           // key-side launch: (first) query head of each group
  int key_heads;               // tensor-core key side: query heads per launch
  int* err;                    // optional device error word (bit flags)
  bool alpha_zero;             // layer_idx == 0: the pattern is a causal window of w keys
  int flags;                   // ESA_FLAG_* of the call
  // Dropout of the softmax weights: keep when the Philox word of
  // (position, batch * H + pattern head, slot / 4) under key `seed` is >= threshold.
  uint32_t drop_threshold;     // 0 = no dropout
  float keep_scale;            // 1 / (1 - dropout_p)
  uint64_t seed;
  void* weights;               // optional [B, Hq, n_rows, w] weights output (input dtype)
  float* probs;                // optional fp32 [B, Hq, w, n_rows] probabilities (tile path)
  // Key side: partial dK / dV sums of "constant" query chunks (kHeavyChunk
  // consecutive query slots that all use one key in a (head, slot) column),
  // fp32 [B, Hq, w, heavy_chunks, 2, D]; heavy_chunks = n_rows / kHeavyChunk.
  float* heavy;
  int heavy_chunks;
  // Key plan (optional): the tensor-core key side's user lists, precomputed
  // from the pattern (esa_keyplan.cuh).  Segment sg = hkv * plan_nlaunch +
  // launch holds, per tile of 4 keys, its users as packed records
  // (column << 25 | key - tile start << 23 | query slot) in
  // [plan_ustart[sg][tile], plan_ustart[sg][tile + 1]) of plan_users + sg *
  // plan_seg_users, and its summed long-run chunks (column << 25 | key << 23 |
  // chunk) likewise in plan_hstart / plan_heavy.
  const uint64_t* plan_header;  // nullptr = no plan
  uint64_t plan_fp;             // fingerprint of the problem the plan must match
  const int* plan_ustart;
  const int* plan_hstart;
  const uint32_t* plan_users;
  const uint32_t* plan_heavy;
  int64_t plan_seg_users, plan_seg_heavy;
  int plan_ntiles, plan_nlaunch, plan_gs;   // plan_gs: query heads per launch
};

constexpr int kHeavyChunk = 1024;

// Keep decision of slot k of (position pos, batch b, launch head h); the
// counter uses the pattern head, so a head split reproduces the same mask.
__device__ __forceinline__ bool dropout_keep(const AttnParams& p, int pos, int b, int h, int k) {
  const uint32_t bh = (uint32_t)(b * p.pat.num_heads + p.pat.head_offset + h);
  const uint4 r = philox4x32_10(make_uint4((uint32_t)pos, bh, (uint32_t)(k >> 2), 0u),
                                make_uint2((uint32_t)p.seed, (uint32_t)(p.seed >> 32)));
  const uint32_t word = (k & 3) == 0 ? r.x : (k & 3) == 1 ? r.y : (k & 3) == 2 ? r.z : r.w;
  return word >= p.drop_threshold;
}

// AttnParams::flags bit (ESA_FLAG_F32_DKV): dk / dv are float32 buffers.
constexpr int kFlagF32Dkv = 2;

enum ErrBits : int {
  kErrKvRange = 1,     // an index fell outside the k/v rows handed to the launch
  kErrQueryRange = 4,  // a rows[] entry outside [-kv_len, kv_len)
  kErrPlan = 8,        // the key plan was built for another problem
};

}  // namespace esa
