// kb_kda_prep.cuh - the arithmetic of the KDA decode preparation shared by the
// preparation kernel and the fused preparation + step kernel, so both compute
// the same operations in the same order (engine/kernels/kda_prepare.py:426-472
// for the short convolution, :581-615 for the gates).
#pragma once

#include "kb_common.cuh"

namespace kb {

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

__device__ __forceinline__ float softplus_f(float x) {
  return x > 20.0f ? x : log1pf(expf(x));
}

// One channel's width-4 convolution from its state (4 bf16: s0 s1 s2 s3),
// weights (4 bf16) and new token: the state shifts left by one and takes the
// token last (returned in new_st); the output is silu(sum) rounded to bf16.
__device__ __forceinline__ float conv_regs(uint2 st, uint2 wv, uint16_t tok, uint2& new_st) {
  const float s1 = bf16_bits_to_float((uint16_t)(st.x >> 16));
  const float s2 = bf16_bits_to_float((uint16_t)(st.y & 0xffffu));
  const float s3 = bf16_bits_to_float((uint16_t)(st.y >> 16));
  const float t = bf16_bits_to_float(tok);
  float acc = s1 * bf16_bits_to_float((uint16_t)(wv.x & 0xffffu));
  acc += s2 * bf16_bits_to_float((uint16_t)(wv.x >> 16));
  acc += s3 * bf16_bits_to_float((uint16_t)(wv.y & 0xffffu));
  acc += t * bf16_bits_to_float((uint16_t)(wv.y >> 16));
  new_st = make_uint2(st.x >> 16 | (st.y << 16), (st.y >> 16) | ((uint32_t)tok << 16));
  return round_bf16(silu_f(acc));
}

// decay = -exp(A_log) * softplus(raw + dt_bias), fp32.
__device__ __forceinline__ float kda_decay(float a_log, uint16_t raw, float dt_bias) {
  const float rate = expf(a_log);
  const float biased = bf16_bits_to_float(raw) + dt_bias;
  return -rate * softplus_f(biased);
}

__device__ __forceinline__ float kda_beta(uint16_t raw) {
  return 1.0f / (1.0f + expf(-bf16_bits_to_float(raw)));
}

}  // namespace kb
