// kb_router.cu - sigmoid top-k router for sm_100a.
//
// Reference: engine/klinear/router.py:47-85 (sigmoid activation, one expert
// group, so the group mask selects every expert).  Logits are fp32 dot
// products of bf16 hidden states and bf16 router rows; scores are
// sigmoid(logit); the choice score adds the correction bias; the top_k
// choices are taken in (choice desc, expert index asc) order, which breaks
// ties by the lower index; the returned weights are the unbiased scores of the
// chosen experts, renormalised by (sum + 1e-20) and multiplied by the scaling
// factor.
//
// Phase 1: CTA (expert block, token block) computes 8 experts x up to 8
// tokens of logits, one warp per expert, with a fixed reduction order (each
// lane sums its strided 8-element pieces in order, then a xor butterfly), so
// logits are identical run to run.  Phase 2: the CTA that completes a token
// block (arrival counter) selects the top_k for its tokens, one warp per
// token, and resets the counter.
#include "kb_common.cuh"

namespace kb {

constexpr int RT_WARPS = 8;      // experts per CTA
constexpr int RT_TOK = 8;        // tokens per CTA

__device__ __forceinline__ bool choice_better(float a, int ia, float b, int ib) {
  // NaN ranks below every number; ties go to the lower index.
  const bool an = a != a, bn = b != b;
  if (an != bn) return bn;
  if (!an && a != b) return a > b;
  return ia < ib;
}

__global__ void __launch_bounds__(RT_WARPS * 32)
    router_kernel(const uint16_t* __restrict__ hidden, int64_t hs, int T, int K,
                  const uint16_t* __restrict__ weight, const float* __restrict__ bias, int E,
                  int top_k, int renorm, float scaling, int64_t* __restrict__ idx_out,
                  float* __restrict__ w_out, float* __restrict__ logits,
                  int* __restrict__ counters) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint16_t* hsm = reinterpret_cast<uint16_t*>(smem);  // [RT_TOK][K]
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.y * RT_TOK;
  const int nt = min(RT_TOK, T - t0);
  const int words = K >> 3;

  pdl_wait();
  pdl_launch_dependents();

  for (int e = threadIdx.x; e < nt * words; e += RT_WARPS * 32) {
    const int m = e / words, w = e - m * words;
    reinterpret_cast<uint4*>(hsm + (size_t)m * K)[w] =
        *reinterpret_cast<const uint4*>(hidden + (size_t)(t0 + m) * hs + (size_t)w * 8);
  }
  __syncthreads();

  const int expert = blockIdx.x * RT_WARPS + warp;
  if (expert < E) {
    float acc[RT_TOK];
#pragma unroll
    for (int m = 0; m < RT_TOK; ++m) acc[m] = 0.f;
    const uint16_t* wrow = weight + (size_t)expert * K;
    for (int w = lane; w < words; w += 32) {
      const uint4 wv = *reinterpret_cast<const uint4*>(wrow + (size_t)w * 8);
      const uint32_t wr[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int m = 0; m < RT_TOK; ++m) {
        if (m < nt) {
          const uint4 hv = reinterpret_cast<const uint4*>(hsm + (size_t)m * K)[w];
          const uint32_t hr[4] = {hv.x, hv.y, hv.z, hv.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float w_lo = __uint_as_float(wr[j] << 16);
            const float w_hi = __uint_as_float(wr[j] & 0xFFFF0000u);
            const float h_lo = __uint_as_float(hr[j] << 16);
            const float h_hi = __uint_as_float(hr[j] & 0xFFFF0000u);
            acc[m] = __fmaf_rn(h_lo, w_lo, acc[m]);
            acc[m] = __fmaf_rn(h_hi, w_hi, acc[m]);
          }
        }
      }
    }
#pragma unroll
    for (int m = 0; m < RT_TOK; ++m) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
      if (lane == 0 && m < nt) logits[(size_t)(t0 + m) * E + expert] = acc[m];
    }
  }

  // Arrival: the last expert block of this token block runs the selection.
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int old = atomicAdd(&counters[blockIdx.y], 1);
    s_last = (old == (int)gridDim.x - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  for (int m = warp; m < nt; m += RT_WARPS) {
    const int tok = t0 + m;
    const float* lrow = logits + (size_t)tok * E;
    // Selection by repeated warp argmax over (choice desc, index asc).
    unsigned taken_mask_local = 0;  // bit j: expert lane + 32*j already taken
    float wsum = 0.f;
    float picked_score[32];
    int picked_idx[32];
    for (int sel = 0; sel < top_k; ++sel) {
      float best = 0.f;
      int bidx = 0x7fffffff;
      bool have = false;
      for (int j = 0; lane + 32 * j < E; ++j) {
        const int e = lane + 32 * j;
        if (taken_mask_local & (1u << j)) continue;
        const float lg = __ldcg(&lrow[e]);
        const float sc = 1.0f / (1.0f + expf(-lg));
        const float ch = sc + (bias ? bias[e] : 0.f);
        if (!have || choice_better(ch, e, best, bidx)) {
          best = ch;
          bidx = e;
          have = true;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
        const int oh = __shfl_xor_sync(0xffffffffu, (int)have, o);
        if (oh && (!have || choice_better(ob, oi, best, bidx))) {
          best = ob;
          bidx = oi;
          have = true;
        }
      }
      if ((bidx & 31) == lane) taken_mask_local |= 1u << (bidx >> 5);
      const float lg = __ldcg(&lrow[bidx]);
      const float sc = 1.0f / (1.0f + expf(-lg));
      picked_score[sel] = sc;
      picked_idx[sel] = bidx;
    }
    for (int sel = 0; sel < top_k; ++sel) wsum += picked_score[sel];
    const float denom = wsum + 1e-20f;
    if (lane == 0) {
      for (int sel = 0; sel < top_k; ++sel) {
        float wv = picked_score[sel];
        if (renorm && top_k > 1) wv = wv / denom;
        idx_out[(size_t)tok * top_k + sel] = picked_idx[sel];
        w_out[(size_t)tok * top_k + sel] = wv * scaling;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) counters[blockIdx.y] = 0;
}

}  // namespace kb

extern "C" size_t kb_router_workspace_size(int64_t T, int64_t E) {
  if (T <= 0 || E <= 0) return 0;
  const size_t lbytes = ((size_t)T * E * sizeof(float) + 255) / 256 * 256;
  const size_t nblk = (size_t)(T + kb::RT_TOK - 1) / kb::RT_TOK;
  return lbytes + (nblk * sizeof(int) + 255) / 256 * 256;
}

extern "C" int kb_router_topk(const uint16_t* hidden, int64_t h_stride, int64_t T, int64_t K,
                              const uint16_t* weight, const float* bias, int64_t E,
                              int64_t top_k, int renormalize, float scaling, int64_t* idx_out,
                              float* w_out, void* workspace, size_t workspace_bytes,
                              void* stream) {
  kb::clear_error();
  KB_REQUIRE(T >= 0 && K > 0 && E > 0 && top_k > 0, KB_ERR_BAD_SHAPE,
             "router needs T >= 0 and K, E, top_k > 0");
  KB_REQUIRE(top_k <= E, KB_ERR_BAD_SHAPE, "top_k %lld exceeds E %lld", (long long)top_k,
             (long long)E);
  KB_REQUIRE(E <= 1024 && top_k <= 32 && K <= 8192 && K % 8 == 0, KB_ERR_UNSUPPORTED,
             "router supports E <= 1024, top_k <= 32, K <= 8192 with K %% 8 == 0");
  if (T == 0) return KB_OK;
  KB_REQUIRE(hidden && weight && idx_out && w_out, KB_ERR_NULL_POINTER, "NULL router pointer");
  KB_REQUIRE(reinterpret_cast<uintptr_t>(hidden) % 16 == 0 && h_stride % 8 == 0 &&
                 reinterpret_cast<uintptr_t>(weight) % 16 == 0,
             KB_ERR_ALIGNMENT, "hidden/weight must be 16-byte aligned with row stride %% 8 == 0");
  const size_t need = kb_router_workspace_size(T, E);
  KB_REQUIRE(workspace && workspace_bytes >= need, KB_ERR_WORKSPACE,
             "router workspace of %zu bytes is smaller than the %zu required", workspace_bytes,
             need);
  float* logits = reinterpret_cast<float*>(workspace);
  const size_t lbytes = ((size_t)T * E * sizeof(float) + 255) / 256 * 256;
  int* counters = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(workspace) + lbytes);
  const size_t smem = (size_t)kb::RT_TOK * K * sizeof(uint16_t);
  static bool attr_done = false;
  if (!attr_done) {
    cudaFuncSetAttribute(kb::router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)(kb::RT_TOK * 8192 * sizeof(uint16_t)));
    attr_done = true;
  }
  const dim3 grid((unsigned)((E + kb::RT_WARPS - 1) / kb::RT_WARPS),
                  (unsigned)((T + kb::RT_TOK - 1) / kb::RT_TOK));
  return kb::launch(kb::router_kernel, grid, dim3(kb::RT_WARPS * 32), smem, stream, hidden,
                    h_stride, (int)T, (int)K, weight, bias, (int)E, (int)top_k, renormalize,
                    scaling, idx_out, w_out, logits, counters);
}
