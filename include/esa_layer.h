/*
 * esa_layer.h -- decoder-layer harness kernels of libesa_b200.so: the
 * memory-bound operations of a pre-norm decoder layer (RMSNorm with a fused
 * residual add, rotary position embedding, SwiGLU) that surround elastic
 * sparse attention in the C4 decoder-stack configuration.  The reference
 * ships no model code (its module is used inside external decoder layers), so
 * these entry points replace no reference interface; they exist so that the
 * layer around the attention runs without layout copies: RoPE rotates q and k
 * in place inside the QKV projection's output buffer, which the attention
 * kernels then read through strides.
 *
 * Same conventions as esa_b200.h: device pointers owned by the caller, no
 * allocation, launches on `stream`, ESA_OK or a negative code with
 * esa_last_error() describing the failure.  dtype is an esa_dtype_t value
 * (ESA_DTYPE_F32 / _BF16 / _F16); rows are contiguous vectors of `dim`
 * elements (row stride = dim) unless stated otherwise; every pointer is
 * 16-byte aligned and dim * element size is a multiple of 16 bytes.
 * Arithmetic is float32; each output is rounded once to dtype.
 */
#ifndef ESA_LAYER_H
#define ESA_LAYER_H

#include <stddef.h>
#include <stdint.h>

#include "esa_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/*
 * RMSNorm with an optional residual add:
 *   h = x + residual (residual may be NULL: h = x; h_out may be NULL when
 *       residual is NULL), rounded to dtype and written to h_out;
 *   y = h * rstd * weight,  rstd = 1 / sqrt(mean(h^2) + eps)  (float32,
 *       written to rstd[n_rows]).
 * dim <= 1024 * (16 / element size).
 */
int esa_rmsnorm_forward(int32_t dtype, int64_t n_rows, int32_t dim, const void* x,
                        const void* residual, void* h_out, const void* weight, float eps,
                        void* y, float* rstd, void* stream);

/* Bytes of float32 workspace esa_rmsnorm_backward needs (per-CTA partial
 * sums of the weight gradient). */
size_t esa_rmsnorm_backward_workspace_size(int64_t n_rows, int32_t dim);

/*
 * Backward of esa_rmsnorm_forward given the saved h and rstd:
 *   dh = dh_in + rstd * (weight * dy - xhat * mean(xhat * weight * dy)),
 *        xhat = h * rstd (dh_in, the gradient reaching h from its other
 *        uses, may be NULL);
 *   dweight = sum over rows of dy * xhat (written in dtype).
 * dh may alias dh_in.
 */
int esa_rmsnorm_backward(int32_t dtype, int64_t n_rows, int32_t dim, const void* h,
                         const void* weight, const float* rstd, const void* dy,
                         const void* dh_in, void* dh, void* dweight, void* workspace,
                         size_t workspace_bytes, void* stream);

/*
 * Rotary position embedding, in place, on q [B, Hq, L, D] and k [B, Hk, L, D]
 * (esa_tensor_t strides, D contiguous; k.data may be NULL).  For i < D/2 the
 * pair (x[i], x[i + D/2]) of the row at position p is rotated by
 * angle = f32(p) * inv_freq[i] (one float32 rounding; cos and sin in float32):
 *   x'[i] = x[i] cos - x[i + D/2] sin,  x'[i + D/2] = x[i + D/2] cos + x[i] sin
 * ("rotate half" convention).  inverse != 0 rotates by -angle (the backward:
 * applied to the gradients of the rotated q and k).  positions: device int64
 * [L] shared by the batch, or NULL for 0..L-1.  inv_freq: device float32
 * [D/2], e.g. 1 / base^(2i/D) computed by the caller.
 */
int esa_rope_apply(int32_t dtype, int32_t batch, int64_t seq_len, int32_t head_dim,
                   esa_tensor_t q, int32_t num_q_heads, esa_tensor_t k, int32_t num_k_heads,
                   const int64_t* positions, const float* inv_freq, int32_t inverse,
                   void* stream);

/*
 * SwiGLU on a fused gate/up projection: gate_up rows are [gate (ffn) | up
 * (ffn)] (row stride 2 * ffn); out[r, f] = silu(gate) * up with
 * silu(g) = g / (1 + exp(-g)).  ffn * element size is a multiple of 16 bytes.
 */
int esa_swiglu_forward(int32_t dtype, int64_t n_rows, int32_t ffn, const void* gate_up,
                       void* out, void* stream);

/*
 * Backward of esa_swiglu_forward: dgate_up rows = [dout * up * silu'(gate) |
 * dout * silu(gate)]; out_recomputed (may be NULL) receives the forward
 * output again, for the down projection's weight gradient, in the same pass.
 */
int esa_swiglu_backward(int32_t dtype, int64_t n_rows, int32_t ffn, const void* gate_up,
                        const void* dout, void* dgate_up, void* out_recomputed, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ESA_LAYER_H */
