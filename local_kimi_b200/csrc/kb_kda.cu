// kb_kda.cu - Kimi Delta Attention recurrent decode step for sm_100a.
//
// Reference: engine/kernels/kda_step.py:173-196 (kda_decode_step_reference)
// and the fused Triton kernel at :21-134.  For one (batch, head) the state S
// is a [Dk, Dv] fp32 matrix updated in place:
//   C  = S * exp(decay)[:, None]          (row i scaled by exp(decay_i))
//   p  = C^T k                            (sum over rows)
//   d  = v - p
//   S' = C + (beta * k)[:, None] * d[None, :]
//   o  = S'^T (q * scale)
// Columns of S are independent, so a CTA owns one (batch, head) and a slice of
// 32 columns: lane = column, the sixteen warps split the rows, the state slice
// is read from HBM once into registers and written once.  Row-wise factors
// (exp(decay), k, beta*k, q*scale) are computed once per CTA in shared memory.
// Products and sums are kept as separate rounded fp32 operations in the order
// of the reference expression so the result tracks it closely.
#include "kb_common.cuh"

namespace kb {

constexpr int KDA_WARPS = 16;
constexpr int KDA_COLS = 32;

template <int RPW>
__global__ void __launch_bounds__(KDA_WARPS * 32)
    kda_step_kernel(float* __restrict__ state, int64_t sb, int64_t sh, int64_t sk,
                    const float* __restrict__ q, const float* __restrict__ k,
                    const float* __restrict__ v, const float* __restrict__ decay,
                    const float* __restrict__ beta, int H, int Dk, int Dv, float scale,
                    float* __restrict__ out, uint16_t* __restrict__ out_bf16) {
  __shared__ float s_ed[RPW * KDA_WARPS];
  __shared__ float s_k[RPW * KDA_WARPS];
  __shared__ float s_bk[RPW * KDA_WARPS];
  __shared__ float s_q[RPW * KDA_WARPS];
  __shared__ float s_red[KDA_WARPS][KDA_COLS];

  const int bh = blockIdx.x;
  const int b = bh / H, h = bh - b * H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int col = blockIdx.y * KDA_COLS + lane;
  const bool col_ok = col < Dv;

  pdl_wait();
  pdl_launch_dependents();

  const size_t vec = (size_t)bh * Dk;
  const float bt = beta[bh];
  for (int i = threadIdx.x; i < Dk; i += KDA_WARPS * 32) {
    const float kv = k[vec + i];
    s_ed[i] = expf(decay[vec + i]);
    s_k[i] = kv;
    s_bk[i] = __fmul_rn(bt, kv);
    s_q[i] = __fmul_rn(q[vec + i], scale);
  }

  float* base = state + (size_t)b * sb + (size_t)h * sh + col;
  float c[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const int i = r * KDA_WARPS + warp;
    c[r] = (col_ok && i < Dk) ? base[(size_t)i * sk] : 0.f;
  }
  __syncthreads();

  float part = 0.f;
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const int i = r * KDA_WARPS + warp;
    if (i < Dk) {
      c[r] = __fmul_rn(c[r], s_ed[i]);
      part = __fadd_rn(part, __fmul_rn(c[r], s_k[i]));
    }
  }
  s_red[warp][lane] = part;
  __syncthreads();
  float pred = 0.f;
#pragma unroll
  for (int w = 0; w < KDA_WARPS; ++w) pred = __fadd_rn(pred, s_red[w][lane]);
  const float delta = col_ok ? __fsub_rn(v[(size_t)bh * Dv + col], pred) : 0.f;
  __syncthreads();

  float opart = 0.f;
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const int i = r * KDA_WARPS + warp;
    if (i < Dk) {
      c[r] = __fadd_rn(c[r], __fmul_rn(s_bk[i], delta));
      opart = __fadd_rn(opart, __fmul_rn(c[r], s_q[i]));
      if (col_ok) base[(size_t)i * sk] = c[r];
    }
  }
  s_red[warp][lane] = opart;
  __syncthreads();
  if (warp == 0 && col_ok) {
    float o = 0.f;
#pragma unroll
    for (int w = 0; w < KDA_WARPS; ++w) o = __fadd_rn(o, s_red[w][lane]);
    out[(size_t)bh * Dv + col] = o;
    if (out_bf16) out_bf16[(size_t)bh * Dv + col] = float_to_bf16_bits(o);
  }
}

}  // namespace kb

extern "C" int kb_kda_decode_step(float* state, int64_t sb, int64_t sh, int64_t sk,
                                  const float* q, const float* k, const float* v,
                                  const float* decay, const float* beta, int64_t B, int64_t H,
                                  int64_t Dk, int64_t Dv, float scale, float* out,
                                  uint16_t* out_bf16, void* stream) {
  kb::clear_error();
  KB_REQUIRE(B > 0 && H > 0 && Dk > 0 && Dv > 0, KB_ERR_BAD_SHAPE,
             "KDA dimensions must be positive (B=%lld H=%lld Dk=%lld Dv=%lld)", (long long)B,
             (long long)H, (long long)Dk, (long long)Dv);
  KB_REQUIRE(Dk <= 256 && Dv <= 4096 && B * H <= (int64_t(1) << 30), KB_ERR_UNSUPPORTED,
             "KDA step supports Dk <= 256 and Dv <= 4096");
  KB_REQUIRE(state && q && k && v && decay && beta && out, KB_ERR_NULL_POINTER,
             "NULL KDA pointer");
  KB_REQUIRE(sk >= Dv && sh >= Dk * sk && sb >= H * sh, KB_ERR_BAD_SHAPE,
             "state strides (%lld, %lld, %lld) overlap rows", (long long)sb, (long long)sh,
             (long long)sk);
  const dim3 grid((unsigned)(B * H), (unsigned)((Dv + kb::KDA_COLS - 1) / kb::KDA_COLS));
  const dim3 block(kb::KDA_WARPS * 32);
  if (Dk <= 128)
    return kb::launch(kb::kda_step_kernel<8>, grid, block, 0, stream, state, sb, sh, sk, q, k,
                      v, decay, beta, (int)H, (int)Dk, (int)Dv, scale, out, out_bf16);
  return kb::launch(kb::kda_step_kernel<16>, grid, block, 0, stream, state, sb, sh, sk, q, k, v,
                    decay, beta, (int)H, (int)Dk, (int)Dv, scale, out, out_bf16);
}
