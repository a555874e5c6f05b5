// kb_kda_prep.cu - KDA decode preparation in one launch.
//
// Between the q/k/v projections and the KDA recurrent step a decode token goes
// through (engine/klinear/attention.py:192-230, the fused path):
//   * the width-4 depthwise causal convolution of each of q, k and v
//     (engine/kernels/kda_prepare.py:426-472): the state [B, C, 4] shifts left
//     by one and takes the new token last (updated in place); the output is
//     silu(sum_w float(state'[w]) * float(weight[w])) rounded to bf16;
//   * the gates (kda_prepare.py:581-615): decay = -exp(A_log[h]) *
//     softplus(raw_decay + dt_bias) in fp32 (softplus(x) = x above 20, else
//     log(1 + exp(x))), beta = sigmoid(raw_beta), q and k of each head times
//     rsqrt(sum of squares + eps).
// The reference runs these as two launches (a convolution launch and a gate
// launch); here one CTA per (sequence, head) does both, one thread per channel
// of the head: the convolution outputs never leave the SM.  Memory-bound
// elementwise work: bytes = the three projections in, the three states read
// and written, decay/beta inputs, the fp32 outputs.
#include "kb_kda_prep.cuh"

namespace kb {

constexpr int KP_MAX_DIM = 256;

// Convolution of one channel in memory: returns the bf16-rounded output as
// float and writes the shifted state back.
__device__ __forceinline__ float conv_channel(const uint16_t* in, uint16_t* state,
                                              const uint16_t* w) {
  uint2 ns;
  const float y = conv_regs(*reinterpret_cast<const uint2*>(state),
                            *reinterpret_cast<const uint2*>(w), *in, ns);
  *reinterpret_cast<uint2*>(state) = ns;
  return y;
}

__device__ __forceinline__ float block_sum(float v, float* red, int D) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
  for (int w = 0; w < (D + 31) / 32; ++w) s += red[w];
  __syncthreads();
  return s;
}

__global__ void kda_prepare_kernel(const uint16_t* __restrict__ q_in,
                                   const uint16_t* __restrict__ k_in,
                                   const uint16_t* __restrict__ v_in, int64_t in_stride,
                                   uint16_t* __restrict__ q_state, uint16_t* __restrict__ k_state,
                                   uint16_t* __restrict__ v_state,
                                   const uint16_t* __restrict__ q_w,
                                   const uint16_t* __restrict__ k_w,
                                   const uint16_t* __restrict__ v_w,
                                   const uint16_t* __restrict__ raw_decay, int64_t rd_stride,
                                   const float* __restrict__ dt_bias,
                                   const float* __restrict__ a_log,
                                   const uint16_t* __restrict__ raw_beta, int64_t rb_stride,
                                   int H, int D, float eps, float* __restrict__ q_out,
                                   float* __restrict__ k_out, float* __restrict__ v_out,
                                   float* __restrict__ decay_out, float* __restrict__ beta_out) {
  __shared__ float red[KP_MAX_DIM / 32];
  const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const int C = H * D;
  const int c = h * D + d;
  pdl_wait();
  const size_t si = ((size_t)b * C + c) * 4;
  const size_t ii = (size_t)b * in_stride + c;
  const float q = conv_channel(q_in + ii, q_state + si, q_w + (size_t)c * 4);
  const float k = conv_channel(k_in + ii, k_state + si, k_w + (size_t)c * 4);
  const float v = conv_channel(v_in + ii, v_state + si, v_w + (size_t)c * 4);
  const size_t oi = (size_t)b * C + c;
  decay_out[oi] = kda_decay(a_log[h], raw_decay[(size_t)b * rd_stride + c], dt_bias[c]);
  v_out[oi] = v;
  const float qs = rsqrtf(block_sum(q * q, red, D) + eps);
  const float ks = rsqrtf(block_sum(k * k, red, D) + eps);
  q_out[oi] = q * qs;
  k_out[oi] = k * ks;
  if (d == 0) {
    beta_out[(size_t)b * H + h] = kda_beta(raw_beta[(size_t)b * rb_stride + h]);
  }
  pdl_launch_dependents();
}

}  // namespace kb

extern "C" int kb_kda_prepare(const uint16_t* q_in, const uint16_t* k_in, const uint16_t* v_in,
                              int64_t in_stride, uint16_t* q_state, uint16_t* k_state,
                              uint16_t* v_state, const uint16_t* q_weight,
                              const uint16_t* k_weight, const uint16_t* v_weight,
                              const uint16_t* raw_decay, int64_t raw_decay_stride,
                              const float* dt_bias, const float* a_log,
                              const uint16_t* raw_beta, int64_t raw_beta_stride, int64_t B,
                              int64_t H, int64_t D, float eps, float* q_out, float* k_out,
                              float* v_out, float* decay_out, float* beta_out, void* stream) {
  kb::clear_error();
  KB_REQUIRE(B >= 0 && H > 0 && D > 0, KB_ERR_BAD_SHAPE, "KDA prepare: bad shape");
  if (B == 0) return KB_OK;
  KB_REQUIRE(D % 32 == 0 && D <= kb::KP_MAX_DIM && B <= 65535 && H <= 65535,
             KB_ERR_UNSUPPORTED, "KDA prepare supports head_dim a multiple of 32 up to %d",
             kb::KP_MAX_DIM);
  KB_REQUIRE(in_stride >= H * D && raw_decay_stride >= H * D && raw_beta_stride >= H,
             KB_ERR_BAD_SHAPE, "KDA prepare: row strides too small");
  KB_REQUIRE(eps > 0.f, KB_ERR_BAD_SHAPE, "KDA prepare: eps must be positive");
  KB_REQUIRE(q_in && k_in && v_in && q_state && k_state && v_state && q_weight && k_weight &&
                 v_weight && raw_decay && dt_bias && a_log && raw_beta && q_out && k_out &&
                 v_out && decay_out && beta_out,
             KB_ERR_NULL_POINTER, "KDA prepare: NULL pointer");
  auto a8 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7) == 0; };
  KB_REQUIRE(a8(q_state) && a8(k_state) && a8(v_state) && a8(q_weight) && a8(k_weight) &&
                 a8(v_weight),
             KB_ERR_ALIGNMENT, "KDA prepare: states and weights must be 8-byte aligned");
  return kb::launch(kb::kda_prepare_kernel, dim3((unsigned)H, (unsigned)B), dim3((unsigned)D),
                    0, stream, q_in, k_in, v_in, in_stride, q_state, k_state, v_state, q_weight,
                    k_weight, v_weight, raw_decay, raw_decay_stride, dt_bias, a_log, raw_beta,
                    raw_beta_stride, (int)H, (int)D, eps, q_out, k_out, v_out, decay_out,
                    beta_out);
}
