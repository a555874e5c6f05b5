// kb_topk.cuh - warp-wide biased top-k selection of the sigmoid router,
// shared by the router kernel (kb_router.cu) and the decode-step executor
// (kb_step.cu).  Reference: engine/klinear/router.py:47-85.
#pragma once

#include "kb_common.cuh"

namespace kb {

// Order-preserving map of a choice score to uint32 (larger is better); NaN
// maps to 0, below every number, and -0 is folded into +0.
__device__ __forceinline__ uint32_t choice_key(float x) {
  if (x != x) return 0u;
  const uint32_t b = __float_as_uint(x + 0.0f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ bool choice_better(uint32_t ka, int ia, uint32_t kb, int ib) {
  return ka > kb || (ka == kb && ia < ib);
}

template <int N>
__device__ __forceinline__ void cswap(uint32_t (&k)[N], int (&id)[N], float (&sc)[N], int i,
                                      int j) {
  if (choice_better(k[j], id[j], k[i], id[i])) {
    const uint32_t tk = k[i];
    k[i] = k[j];
    k[j] = tk;
    const int ti = id[i];
    id[i] = id[j];
    id[j] = ti;
    const float ts = sc[i];
    sc[i] = sc[j];
    sc[j] = ts;
  }
}

// Router dot products: one lane accumulates its 16-byte words of bf16
// weights times bf16 activations (fp32 products, fused adds) into four
// partial sums, one per element pair j of the word; router_lane_sum joins
// them as (a0 + a1) + (a2 + a3) before the warp's xor butterfly.  Both router
// implementations use this order, so their logits agree bit for bit.
__device__ __forceinline__ void router_word_fma(uint4 wv, uint4 hv, float (&a)[4]) {
  const uint32_t wr[4] = {wv.x, wv.y, wv.z, wv.w};
  const uint32_t hr[4] = {hv.x, hv.y, hv.z, hv.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    a[j] = __fmaf_rn(__uint_as_float(hr[j] << 16), __uint_as_float(wr[j] << 16), a[j]);
    a[j] = __fmaf_rn(__uint_as_float(hr[j] & 0xFFFF0000u), __uint_as_float(wr[j] & 0xFFFF0000u),
                     a[j]);
  }
}

__device__ __forceinline__ float router_lane_sum(const float (&a)[4]) {
  return __fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3]));
}

// Top-k of one token over E <= 256 experts, one warp.  lrow holds the fp32
// logits (read with L2-only loads: another CTA may have written them in the
// same kernel).  scores = sigmoid(logit); choice = score + bias; the k picks
// are made in (choice desc, index asc) order.  Lane r < top_k receives pick r
// (my_idx, my_score = unbiased score); every lane receives wsum, the sum of
// the picked scores in pick order.
__device__ __forceinline__ void warp_topk256(const float* lrow, const float* bias, int E,
                                             int top_k, int lane, int& my_idx, float& my_score,
                                             float& wsum) {
  uint32_t key[8];
  int id[8];
  float sc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int e = lane + 32 * j;
    if (e < E) {
      const float lg = __ldcg(&lrow[e]);
      sc[j] = 1.0f / (1.0f + expf(-lg));
      key[j] = choice_key(sc[j] + (bias ? bias[e] : 0.f));
      id[j] = e;
    } else {
      sc[j] = 0.f;
      key[j] = 0u;
      id[j] = 0x7fffffff;
    }
  }
  // Sort descending by (key, -index): optimal 19-comparator network.
  cswap(key, id, sc, 0, 2);
  cswap(key, id, sc, 1, 3);
  cswap(key, id, sc, 4, 6);
  cswap(key, id, sc, 5, 7);
  cswap(key, id, sc, 0, 4);
  cswap(key, id, sc, 1, 5);
  cswap(key, id, sc, 2, 6);
  cswap(key, id, sc, 3, 7);
  cswap(key, id, sc, 0, 1);
  cswap(key, id, sc, 2, 3);
  cswap(key, id, sc, 4, 5);
  cswap(key, id, sc, 6, 7);
  cswap(key, id, sc, 2, 4);
  cswap(key, id, sc, 3, 5);
  cswap(key, id, sc, 1, 4);
  cswap(key, id, sc, 3, 6);
  cswap(key, id, sc, 1, 2);
  cswap(key, id, sc, 3, 4);
  cswap(key, id, sc, 5, 6);
  // Each pick: the best head over the lanes (one max-reduction); the lane
  // holding it is found with a ballot, and only exact key ties fall back to
  // the lower expert index.
  for (int sel = 0; sel < top_k; ++sel) {
    const uint32_t best = __reduce_max_sync(0xffffffffu, key[0]);
    const unsigned holders = __ballot_sync(0xffffffffu, key[0] == best);
    int win;
    if ((holders & (holders - 1u)) == 0u) {
      win = __ffs(holders) - 1;
    } else {
      const uint32_t cand = (key[0] == best) ? (uint32_t)id[0] : 0xffffffffu;
      const uint32_t lowest = __reduce_min_sync(0xffffffffu, cand);
      win = __ffs(__ballot_sync(0xffffffffu, cand == lowest)) - 1;
    }
    const float s = __shfl_sync(0xffffffffu, sc[0], win);
    const int wid = __shfl_sync(0xffffffffu, id[0], win);
    if (lane == win) {
#pragma unroll
      for (int j = 0; j < 7; ++j) {
        key[j] = key[j + 1];
        id[j] = id[j + 1];
        sc[j] = sc[j + 1];
      }
      key[7] = 0u;
      id[7] = 0x7fffffff;
      sc[7] = 0.f;
    }
    wsum += s;
    if (lane == sel) {
      my_score = s;
      my_idx = wid;
    }
  }
}

// Router word of one (token, expert): choice key + 1 in the high half (zero
// means "not yet written"; keys stay below 0xff800001, so the sum does not
// wrap) and the fp32 logit in the low half, published with one 64-bit store
// so that a reader sees both or neither.
__device__ __forceinline__ unsigned long long router_word(uint32_t key, float logit) {
  return ((unsigned long long)(key + 1u) << 32) | __float_as_uint(logit);
}

__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

}  // namespace kb
