// kb_w4a16.cu - W4A16 projection engine for sm_100a.
//
// One persistent kernel serves every INT4-weight projection of the decode hot
// path: dense (w4a16_dense, fused QKV), expert-grouped (w4a16_grouped), fused
// gate/up + SwiGLU (w4a16_swiglu) and down projection + weighted combine
// (fused_w2_combine).  Work is split into items; an item is a group of 16-row
// blocks of one weight matrix (or of the w1/w3 pair) over the full reduction
// axis, for up to 8*NSUB tokens that use that matrix.
//
// Inside an item each warp owns one 16-row block and one slice of the
// reduction axis.  A lane streams 16-byte pieces of packed codes for two rows
// straight from HBM (ld.global.nc, L1 bypass), decodes them in registers to
// bf16(code * scale) with bf16x2 arithmetic (decode_word), and feeds the
// tensor core through mma.m16n8k16 with the weights as the 16x16 A operand
// and up to 8 tokens of activations (staged once per item in shared memory in
// decode pair order) as the B operand, accumulating in fp32.  Slices of the
// reduction axis are summed in a fixed order through shared memory, so every
// output is deterministic run to run.
//
// Reference semantics (engine/kernels/w4a16_gemv.py:56-174, :224-392,
// engine/kernels/moe_combine.py:209-261): decoded weight bf16(code*scale),
// fp32 products and sums, bf16 projection outputs, SwiGLU rounding contract
// silu(bf16 g) -> bf16, times bf16 u -> bf16, combine = bf16(fp32 sum of the
// routed outputs times fp32 weights) + shared output (bf16 add).
#include "kb_common.cuh"

#include <algorithm>
#include <mutex>

namespace kb {

constexpr int NW = 8;               // warps per CTA
constexpr int NTHREADS = NW * 32;
constexpr int KCH = 4;              // 128-wide reduction blocks loaded per batch
constexpr int MAX_SMEM = 200 * 1024;

enum : int { MODE_DENSE = 0, MODE_GROUPED = 1, MODE_SWIGLU = 2, MODE_W2C = 3 };

struct DenseProb {
  const uint16_t* x;
  int64_t xs;
  const uint8_t* w;
  const uint16_t* s;
  uint16_t* y;
  int64_t ys;
  int M, K, N, gshift;
  int KS, RBc, items_rb, tok_groups;
  int item_begin;
};

struct GroupedArgs {
  const uint16_t* x;
  int64_t xs;
  const int64_t* idx;
  const uint8_t* w0;
  const uint16_t* s0;
  const uint8_t* w1;
  const uint16_t* s1;
  int64_t wse, sse;
  uint16_t* y;
  const float* cw;
  int64_t cws;
  uint16_t* out;
  uint16_t* wsy;
  int* counters;
  int T, R, K, N, E, gshift;
  int KS, RBc, items_rb;
};

struct EngineParams {
  int mode;
  int tok_cap;
  int tstride;
  int red_off;
  int plan_off;
  int total_items;
  int nprob;
  uint32_t* err;
  DenseProb prob[KB_MAX_DENSE_PROBLEMS];
  GroupedArgs g;
};

// ---------------------------------------------------------------------------
// Device side.
// ---------------------------------------------------------------------------

// Stage one activation row (K bf16, 16-byte aligned) into shared memory in the
// layout the B fragments read: token row m, word j of chunk c at byte offset
// m*tstride + (j*NC + c)*16, each word in pair order (x0,x4),(x1,x5),...
__device__ __forceinline__ void stage_row(uint8_t* xs_row, const uint16_t* src, int K,
                                          int first, int step) {
  const int NC = K >> 5;
  const int words = K >> 3;
  for (int w = first; w < words; w += step) {
    const uint4 v = *reinterpret_cast<const uint4*>(src + (size_t)w * 8);
    const int c = w >> 2, j = w & 3;
    *reinterpret_cast<uint4*>(xs_row + (j * NC + c) * 16) = permute_pairs(v);
  }
}

// Accumulate the 16-row block [r0, r0+16) of matrix (w, s) over reduction
// blocks [kb0, kb1) into acc[p] for token sub-pass p (tokens 8p..8p+7).
// D fragment: acc[p][0] = (row g, token 2t), [1] = (row g, token 2t+1),
// [2] = (row g+8, token 2t), [3] = (row g+8, token 2t+1).
template <int NSUB>
__device__ __forceinline__ void rowblock_mma(const uint8_t* __restrict__ w,
                                             const uint16_t* __restrict__ s, int N, int K,
                                             int gshift, int r0, int kb0, int kb1,
                                             const uint8_t* xs, int tstride, int ntok,
                                             float (&acc)[NSUB][4]) {
  const int nact = (ntok + 7) >> 3;  // sub-passes holding at least one token
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int NC = K >> 5;
  const int rowA = min(r0 + g, N - 1);
  const int rowB = min(r0 + g + 8, N - 1);
  const uint8_t* wA = w + (size_t)rowA * (size_t)(K >> 1);
  const uint8_t* wB = w + (size_t)rowB * (size_t)(K >> 1);
  const int ng = K >> (5 + gshift);
  const uint16_t* sA = s + (size_t)rowA * ng;
  const uint16_t* sB = s + (size_t)rowB * ng;
  const uint8_t* xrow[NSUB];
#pragma unroll
  for (int p = 0; p < NSUB; ++p) xrow[p] = xs + min(p * 8 + g, ntok - 1) * tstride;

  for (int kb = kb0; kb < kb1; kb += KCH) {
    uint4 WA[KCH], WB[KCH];
    uint32_t SA[KCH], SB[KCH];
#pragma unroll
    for (int i = 0; i < KCH; ++i) {
      const int c = (kb + i) * 4 + t;
      if (kb + i < kb1 && c < NC) {
        WA[i] = ldg_stream_v4(wA + (size_t)c * 16);
        WB[i] = ldg_stream_v4(wB + (size_t)c * 16);
        SA[i] = ldg_u16(sA + (c >> gshift));
        SB[i] = ldg_u16(sB + (c >> gshift));
      } else {
        WA[i] = make_uint4(0, 0, 0, 0);
        WB[i] = make_uint4(0, 0, 0, 0);
        SA[i] = 0;
        SB[i] = 0;
      }
    }
#pragma unroll
    for (int i = 0; i < KCH; ++i) {
      if (kb + i < kb1) {
        const int c = min((kb + i) * 4 + t, NC - 1);
        const uint32_t sa2 = SA[i] | (SA[i] << 16);
        const uint32_t sb2 = SB[i] | (SB[i] << 16);
        const uint32_t wa[4] = {WA[i].x, WA[i].y, WA[i].z, WA[i].w};
        const uint32_t wb[4] = {WB[i].x, WB[i].y, WB[i].z, WB[i].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
          decode_word(wa[j], sa2, a0, a1, a2, a3);
          decode_word(wb[j], sb2, b0, b1, b2, b3);
#pragma unroll
          for (int p = 0; p < NSUB; ++p) {
            if (p < nact) {
              const uint4 xv = lds_v4(xrow[p] + (j * NC + c) * 16);
              mma_bf16_16816(acc[p], a0, b0, a1, b1, xv.x, xv.y);
              mma_bf16_16816(acc[p], a2, b2, a3, b3, xv.z, xv.w);
            }
          }
        }
      }
    }
  }
}

__device__ __forceinline__ int clamp_expert(int64_t v, int E, uint32_t* err) {
  if (v < 0 || v >= E) {
    atomicOr(err, 1u);
    return 0;
  }
  return static_cast<int>(v);
}

__device__ __forceinline__ float swiglu_contract(float gate, float up) {
  // F.silu(gate_bf16) * up_bf16 in bf16 (engine/kernels/__init__.py:182-197).
  const float g = round_bf16(gate);
  const float u = round_bf16(up);
  const float sl = round_bf16(g / (1.0f + expf(-g)));
  return sl * u;
}

template <int NSUB>
__device__ void dense_loop(const EngineParams& P, uint8_t* xs, float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  int staged_p = -1, staged_gb = -1;
  for (int item = blockIdx.x; item < P.total_items; item += gridDim.x) {
    int p = 0;
    while (p + 1 < P.nprob && item >= P.prob[p + 1].item_begin) ++p;
    const DenseProb& D = P.prob[p];
    const int local = item - D.item_begin;
    const int gb = local / D.items_rb;
    const int rbg = local - gb * D.items_rb;
    const int tok0 = gb * P.tok_cap;
    const int ntok = min(P.tok_cap, D.M - tok0);
    if (p != staged_p || gb != staged_gb) {
      __syncthreads();
      for (int m = 0; m < ntok; ++m)
        stage_row(xs + m * P.tstride, D.x + (size_t)(tok0 + m) * D.xs, D.K, threadIdx.x,
                  NTHREADS);
      __syncthreads();
      staged_p = p;
      staged_gb = gb;
    }
    const int ks = warp % D.KS;
    const int rb = warp / D.KS;
    const int KB = (D.K + 127) >> 7;
    const int kb0 = KB * ks / D.KS, kb1 = KB * (ks + 1) / D.KS;
    const int r0 = (rbg * D.RBc + rb) * 16;
    float acc[NSUB][4];
#pragma unroll
    for (int q = 0; q < NSUB; ++q)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[q][i] = 0.f;
    if (r0 < D.N)
      rowblock_mma<NSUB>(D.w, D.s, D.N, D.K, D.gshift, r0, kb0, kb1, xs, P.tstride, ntok, acc);
#pragma unroll
    for (int q = 0; q < NSUB; ++q)
      *reinterpret_cast<float4*>(red + ((warp * NSUB + q) * 32 + lane) * 4) =
          make_float4(acc[q][0], acc[q][1], acc[q][2], acc[q][3]);
    __syncthreads();
    if (ks == 0 && r0 < D.N) {
#pragma unroll
      for (int q = 0; q < NSUB; ++q) {
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        for (int k2 = 0; k2 < D.KS; ++k2) {
          const float4 pv =
              *reinterpret_cast<const float4*>(red + (((warp + k2) * NSUB + q) * 32 + lane) * 4);
          v[0] += pv.x;
          v[1] += pv.y;
          v[2] += pv.z;
          v[3] += pv.w;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = r0 + g + ((i >> 1) << 3);
          const int tok = q * 8 + 2 * t + (i & 1);
          if (row < D.N && tok < ntok)
            D.y[(size_t)(tok0 + tok) * D.ys + row] = float_to_bf16_bits(v[i]);
        }
      }
    }
    __syncthreads();
  }
}

// Build the expert-major assignment plan in shared memory: the used experts in
// ascending order (slot_expert), the start of each slot's assignments
// (slot_start) and the assignment ids ordered by (expert, id) (assign).
__device__ int build_plan(const GroupedArgs& G, uint32_t* err, int* cnt, int* slot_expert,
                          int* slot_start, int* assign) {
  __shared__ int s_nslots;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int TR = G.T * G.R;
  const int E = G.E;
  for (int e = threadIdx.x; e <= E; e += NTHREADS) cnt[e] = 0;
  __syncthreads();
  for (int a = threadIdx.x; a < TR; a += NTHREADS) {
    const int e = clamp_expert(G.idx[a], E, err);
    atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (warp == 0) {
    int running = 0, nslots = 0;
    for (int base = 0; base < E; base += 32) {
      const int e = base + lane;
      const int c = (e < E) ? cnt[e] : 0;
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      const int excl = running + incl - c;
      const unsigned used = __ballot_sync(0xffffffffu, c > 0);
      const int rank = nslots + __popc(used & ((1u << lane) - 1u));
      if (c > 0) {
        slot_expert[rank] = e;
        slot_start[rank] = excl;
      }
      if (e < E) cnt[e] = excl;
      running += __shfl_sync(0xffffffffu, incl, 31);
      nslots += __popc(used);
    }
    if (lane == 0) {
      slot_start[nslots] = running;
      s_nslots = nslots;
    }
    __syncwarp();
    for (int base = 0; base < TR; base += 32) {
      const int a = base + lane;
      const bool valid = a < TR;
      int e = -1 - lane;
      if (valid) {
        const int64_t v = G.idx[a];
        e = (v < 0 || v >= E) ? 0 : static_cast<int>(v);
      }
      const unsigned peers = __match_any_sync(0xffffffffu, e);
      const int rank = __popc(peers & ((1u << lane) - 1u));
      int pos = 0;
      if (valid) pos = cnt[e] + rank;
      __syncwarp();
      if (valid) {
        assign[pos] = a;
        if (lane == __ffs(peers) - 1) cnt[e] += __popc(peers);
      }
      __syncwarp();
    }
  }
  __syncthreads();
  return s_nslots;
}

template <int NSUB>
__device__ void grouped_loop(const EngineParams& P, uint8_t* xs, float* red, uint8_t* plan) {
  const GroupedArgs& G = P.g;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  int* cnt = reinterpret_cast<int*>(plan);
  int* slot_expert = cnt + (G.E + 1);
  int* slot_start = slot_expert + G.E;
  int* assign = slot_start + (G.E + 1);
  __shared__ int s_done[16];

  const int nslots = build_plan(G, P.err, cnt, slot_expert, slot_start, assign);
  const int mats = (P.mode == MODE_SWIGLU) ? 2 : 1;
  const int per_mat = G.RBc * G.KS;
  const int mat = warp / per_mat;
  const int rem = warp - mat * per_mat;
  const int rb = rem / G.KS;
  const int ks = rem - rb * G.KS;
  const int KB = (G.K + 127) >> 7;
  const int kb0 = KB * ks / G.KS, kb1 = KB * (ks + 1) / G.KS;
  const int nitems = nslots * G.items_rb;
  (void)mats;

  for (int item = blockIdx.x; item < nitems; item += gridDim.x) {
    const int slot = item / G.items_rb;
    const int rbg = item - slot * G.items_rb;
    const int e = slot_expert[slot];
    const int abase = slot_start[slot];
    const int count = slot_start[slot + 1] - abase;
    const int r0 = (rbg * G.RBc + rb) * 16;
    for (int gb = 0; gb < count; gb += P.tok_cap) {
      const int ntok = min(P.tok_cap, count - gb);
      __syncthreads();
      for (int m = 0; m < ntok; ++m) {
        const int a = assign[abase + gb + m];
        const uint16_t* src = (P.mode == MODE_W2C) ? G.x + (size_t)a * G.xs
                                                   : G.x + (size_t)(a / G.R) * G.xs;
        stage_row(xs + m * P.tstride, src, G.K, threadIdx.x, NTHREADS);
      }
      __syncthreads();
      float acc[NSUB][4];
#pragma unroll
      for (int q = 0; q < NSUB; ++q)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[q][i] = 0.f;
      if (r0 < G.N) {
        const uint8_t* wbase = (mat ? G.w1 : G.w0) + (size_t)e * (size_t)G.wse;
        const uint16_t* sbase = (mat ? G.s1 : G.s0) + (size_t)e * (size_t)G.sse;
        rowblock_mma<NSUB>(wbase, sbase, G.N, G.K, G.gshift, r0, kb0, kb1, xs, P.tstride, ntok,
                           acc);
      }
#pragma unroll
      for (int q = 0; q < NSUB; ++q)
        *reinterpret_cast<float4*>(red + ((warp * NSUB + q) * 32 + lane) * 4) =
            make_float4(acc[q][0], acc[q][1], acc[q][2], acc[q][3]);
      __syncthreads();
      if (mat == 0 && ks == 0 && r0 < G.N) {
#pragma unroll
        for (int q = 0; q < NSUB; ++q) {
          float v0[4] = {0.f, 0.f, 0.f, 0.f};
          float v1[4] = {0.f, 0.f, 0.f, 0.f};
          for (int k2 = 0; k2 < G.KS; ++k2) {
            const float4 pv = *reinterpret_cast<const float4*>(
                red + (((warp + k2) * NSUB + q) * 32 + lane) * 4);
            v0[0] += pv.x;
            v0[1] += pv.y;
            v0[2] += pv.z;
            v0[3] += pv.w;
            if (P.mode == MODE_SWIGLU) {
              const float4 uv = *reinterpret_cast<const float4*>(
                  red + (((warp + per_mat + k2) * NSUB + q) * 32 + lane) * 4);
              v1[0] += uv.x;
              v1[1] += uv.y;
              v1[2] += uv.z;
              v1[3] += uv.w;
            }
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int row = r0 + g + ((i >> 1) << 3);
            const int tok = q * 8 + 2 * t + (i & 1);
            if (row < G.N && tok < ntok) {
              const int a = assign[abase + gb + tok];
              const size_t o = (size_t)a * G.N + row;
              if (P.mode == MODE_GROUPED) {
                G.y[o] = float_to_bf16_bits(v0[i]);
              } else if (P.mode == MODE_SWIGLU) {
                G.y[o] = float_to_bf16_bits(swiglu_contract(v0[i], v1[i]));
              } else {
                G.wsy[o] = float_to_bf16_bits(v0[i]);
              }
            }
          }
        }
      }
      if (P.mode == MODE_W2C) {
        // Arrival: once all R routes of a token have written this row group,
        // the CTA that arrives last combines them (fixed route order).
        __threadfence();
        __syncthreads();
        if (threadIdx.x < ntok) {
          const int a = assign[abase + gb + threadIdx.x];
          const int tok = a / G.R;
          const int old = atomicAdd(&G.counters[tok * G.items_rb + rbg], 1);
          s_done[threadIdx.x] = (old == G.R - 1) ? tok : -1;
        }
        __syncthreads();
        const int rstart = rbg * G.RBc * 16;
        const int rend = min(G.N, rstart + G.RBc * 16);
        for (int m = 0; m < ntok; ++m) {
          const int tok = s_done[m];
          if (tok < 0) continue;
          __threadfence();
          for (int row = rstart + threadIdx.x; row < rend; row += NTHREADS) {
            float accum = 0.f;
            for (int r = 0; r + 1 < G.R; ++r) {
              const uint16_t ov = __ldcg(&G.wsy[((size_t)tok * G.R + r) * G.N + row]);
              accum += bf16_bits_to_float(ov) * G.cw[(size_t)tok * G.cws + r];
            }
            const uint16_t sv = __ldcg(&G.wsy[((size_t)tok * G.R + G.R - 1) * G.N + row]);
            const float routed = round_bf16(accum);
            G.out[(size_t)tok * G.N + row] = float_to_bf16_bits(routed + bf16_bits_to_float(sv));
          }
          if (threadIdx.x == 0) G.counters[tok * G.items_rb + rbg] = 0;
        }
      }
      __syncthreads();
    }
  }
}

template <int NSUB>
__global__ void __launch_bounds__(NTHREADS, 1) w4a16_engine(const __grid_constant__ EngineParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  pdl_wait();
  pdl_launch_dependents();
  float* red = reinterpret_cast<float*>(smem + P.red_off);
  if (P.mode == MODE_DENSE)
    dense_loop<NSUB>(P, smem, red);
  else
    grouped_loop<NSUB>(P, smem, red, smem + P.plan_off);
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------

static int ilog2_exact(int64_t v) {
  int s = 0;
  while ((int64_t(1) << s) < v) ++s;
  return ((int64_t(1) << s) == v) ? s : -1;
}

static int check_group(int64_t K, int64_t group, int* gshift) {
  KB_REQUIRE(group >= 32 && group % 32 == 0, KB_ERR_BAD_GROUP,
             "group size %lld must be a positive multiple of 32", (long long)group);
  const int s = ilog2_exact(group / 32);
  KB_REQUIRE(s >= 0, KB_ERR_BAD_GROUP, "group size %lld must be 32 times a power of two",
             (long long)group);
  KB_REQUIRE(K % group == 0, KB_ERR_BAD_GROUP,
             "reduction width %lld is not divisible by group size %lld", (long long)K,
             (long long)group);
  *gshift = s;
  return KB_OK;
}

// Warp split for a reduction width: KS warps share a 16-row block, each
// covering at least four 128-wide blocks when possible; RBc row blocks per
// item so that mats * RBc * KS == NW.
static void choose_split(int K, int mats, int* KS, int* RBc) {
  const int KB = (K + 127) / 128;
  const int maxks = NW / mats;
  int ks = 1;
  while (ks * 2 <= maxks && KB / (ks * 2) >= 4) ks *= 2;
  *KS = ks;
  *RBc = maxks / ks;
}

static inline bool aligned(const void* p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

static int token_stride(int K) {
  const int bytes = 2 * K;
  const int pad = (64 - (bytes % 128) + 128) % 128;
  return bytes + pad;
}

template <int NSUB>
static int engine_launch(EngineParams& P, int grid_items, size_t smem, void* stream) {
  static std::once_flag once[2];
  static cudaError_t attr_err[2] = {cudaSuccess, cudaSuccess};
  std::call_once(once[NSUB - 1], [] {
    attr_err[NSUB - 1] = cudaFuncSetAttribute(
        w4a16_engine<NSUB>, cudaFuncAttributeMaxDynamicSharedMemorySize, MAX_SMEM);
  });
  KB_REQUIRE(attr_err[NSUB - 1] == cudaSuccess, KB_ERR_LAUNCH,
             "cudaFuncSetAttribute failed: %s", cudaGetErrorString(attr_err[NSUB - 1]));
  KB_REQUIRE(smem <= (size_t)MAX_SMEM, KB_ERR_UNSUPPORTED,
             "shared memory need %zu bytes exceeds %d (reduce K or tokens)", smem, MAX_SMEM);
  const int dev = bind_stream_device(stream);
  int occ = 1;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, w4a16_engine<NSUB>, NTHREADS, smem);
  if (occ < 1) occ = 1;
  const int grid = std::max(1, std::min(grid_items, num_sms(dev) * occ));
  P.err = device_error_word(dev);
  return launch(w4a16_engine<NSUB>, dim3(grid), dim3(NTHREADS), smem, stream, P);
}

static int dense_multi_impl(const kb_dense_problem* probs, int count, void* stream) {
  KB_REQUIRE(count >= 0 && count <= KB_MAX_DENSE_PROBLEMS, KB_ERR_UNSUPPORTED,
             "problem count %d outside [0, %d]", count, KB_MAX_DENSE_PROBLEMS);
  KB_REQUIRE(count == 0 || probs != nullptr, KB_ERR_NULL_POINTER, "problems is NULL");
  EngineParams P = {};
  P.mode = MODE_DENSE;
  int maxM = 0, maxK = 0;
  for (int i = 0; i < count; ++i) {
    const kb_dense_problem& q = probs[i];
    KB_REQUIRE(q.M >= 0 && q.K > 0 && q.N > 0, KB_ERR_BAD_SHAPE,
               "problem %d: need M >= 0, K > 0, N > 0 (got M=%lld K=%lld N=%lld)", i,
               (long long)q.M, (long long)q.K, (long long)q.N);
    KB_REQUIRE(q.K % 32 == 0, KB_ERR_BAD_SHAPE,
               "problem %d: reduction width %lld is not divisible by 32", i, (long long)q.K);
    KB_REQUIRE(q.K <= 65536 && q.N <= (int64_t(1) << 30) && q.M <= (int64_t(1) << 30),
               KB_ERR_UNSUPPORTED, "problem %d: size above the supported range", i);
    int gs = 0;
    int rc = check_group(q.K, q.group, &gs);
    if (rc) return rc;
    if (q.M == 0) continue;
    KB_REQUIRE(q.x && q.packed && q.scales && q.y, KB_ERR_NULL_POINTER,
               "problem %d: NULL pointer", i);
    KB_REQUIRE(aligned(q.x, 16) && q.x_stride % 8 == 0 && q.x_stride >= q.K, KB_ERR_ALIGNMENT,
               "problem %d: activations must be 16-byte aligned with a row stride that is a "
               "multiple of 8 elements and >= K",
               i);
    KB_REQUIRE(aligned(q.packed, 16), KB_ERR_ALIGNMENT,
               "problem %d: packed weights must be 16-byte aligned", i);
    KB_REQUIRE(aligned(q.scales, 2) && aligned(q.y, 2) && q.y_stride >= q.N, KB_ERR_ALIGNMENT,
               "problem %d: scales/output misaligned or output stride < N", i);
    DenseProb& D = P.prob[P.nprob];
    D.x = q.x;
    D.xs = q.x_stride;
    D.w = q.packed;
    D.s = q.scales;
    D.y = q.y;
    D.ys = q.y_stride;
    D.M = (int)q.M;
    D.K = (int)q.K;
    D.N = (int)q.N;
    D.gshift = gs;
    choose_split(D.K, 1, &D.KS, &D.RBc);
    maxM = std::max(maxM, D.M);
    maxK = std::max(maxK, D.K);
    P.nprob++;
  }
  if (P.nprob == 0) return KB_OK;
  const int nsub = (maxM > 8) ? 2 : 1;
  P.tok_cap = 8 * nsub;
  int items = 0;
  for (int i = 0; i < P.nprob; ++i) {
    DenseProb& D = P.prob[i];
    D.items_rb = (D.N + 16 * D.RBc - 1) / (16 * D.RBc);
    D.tok_groups = (D.M + P.tok_cap - 1) / P.tok_cap;
    D.item_begin = items;
    items += D.items_rb * D.tok_groups;
  }
  P.total_items = items;
  P.tstride = token_stride(maxK);
  const int staged = std::min(P.tok_cap, maxM);
  P.red_off = ((staged * P.tstride) + 127) / 128 * 128;
  const size_t smem = (size_t)P.red_off + (size_t)NW * nsub * 32 * 4 * sizeof(float);
  P.plan_off = 0;
  return nsub == 2 ? engine_launch<2>(P, items, smem, stream)
                   : engine_launch<1>(P, items, smem, stream);
}

static int grouped_impl(int mode, const uint16_t* x, int64_t x_stride, int64_t T, int64_t K,
                        const int64_t* idx, int64_t R, const uint8_t* w0, const uint16_t* s0,
                        const uint8_t* w1, const uint16_t* s1, int64_t E, int64_t N,
                        int64_t group, uint16_t* y, const float* cw, int64_t cws, uint16_t* out,
                        void* workspace, size_t ws_bytes, void* stream) {
  KB_REQUIRE(T >= 0 && R > 0 && K > 0 && E > 0 && N > 0, KB_ERR_BAD_SHAPE,
             "need T >= 0 and R, K, E, N > 0 (got T=%lld R=%lld K=%lld E=%lld N=%lld)",
             (long long)T, (long long)R, (long long)K, (long long)E, (long long)N);
  KB_REQUIRE(K % 32 == 0, KB_ERR_BAD_SHAPE, "reduction width %lld is not divisible by 32",
             (long long)K);
  int gs = 0;
  int rc = check_group(K, group, &gs);
  if (rc) return rc;
  if (T == 0) return KB_OK;
  KB_REQUIRE(T * R <= KB_MAX_ASSIGNMENTS, KB_ERR_UNSUPPORTED,
             "T*R = %lld exceeds the limit of %d assignments per call", (long long)(T * R),
             KB_MAX_ASSIGNMENTS);
  KB_REQUIRE(E <= 4096 && K <= 65536 && N <= (int64_t(1) << 24), KB_ERR_UNSUPPORTED,
             "E, K or N above the supported range");
  KB_REQUIRE(x && idx && w0 && s0, KB_ERR_NULL_POINTER, "NULL input pointer");
  KB_REQUIRE(mode != MODE_SWIGLU || (w1 && s1), KB_ERR_NULL_POINTER, "NULL w3 pointer");
  KB_REQUIRE(aligned(x, 16) && x_stride % 8 == 0 && x_stride >= K, KB_ERR_ALIGNMENT,
             "activations must be 16-byte aligned with a row stride that is a multiple of 8 "
             "elements and >= K");
  KB_REQUIRE(aligned(w0, 16) && (!w1 || aligned(w1, 16)), KB_ERR_ALIGNMENT,
             "packed weights must be 16-byte aligned");
  KB_REQUIRE(aligned(idx, 8), KB_ERR_ALIGNMENT, "expert indices must be 8-byte aligned");
  EngineParams P = {};
  P.mode = mode;
  GroupedArgs& G = P.g;
  G.x = x;
  G.xs = x_stride;
  G.idx = idx;
  G.w0 = w0;
  G.s0 = s0;
  G.w1 = w1;
  G.s1 = s1;
  G.wse = N * (K / 2);
  G.sse = N * (K / group);
  G.y = y;
  G.cw = cw;
  G.cws = cws;
  G.out = out;
  G.T = (int)T;
  G.R = (int)R;
  G.K = (int)K;
  G.N = (int)N;
  G.E = (int)E;
  G.gshift = gs;
  const int mats = (mode == MODE_SWIGLU) ? 2 : 1;
  choose_split(G.K, mats, &G.KS, &G.RBc);
  G.items_rb = (G.N + 16 * G.RBc - 1) / (16 * G.RBc);
  if (mode == MODE_W2C) {
    KB_REQUIRE(out && cw, KB_ERR_NULL_POINTER, "NULL output or weights pointer");
    const size_t need = kb_w4a16_w2_combine_workspace_size(T, R, N);
    KB_REQUIRE(workspace && ws_bytes >= need, KB_ERR_WORKSPACE,
               "workspace of %zu bytes is smaller than the %zu required", ws_bytes, need);
    KB_REQUIRE(aligned(workspace, 16), KB_ERR_ALIGNMENT, "workspace must be 16-byte aligned");
    G.wsy = reinterpret_cast<uint16_t*>(workspace);
    const size_t ybytes = ((size_t)T * R * N * 2 + 255) / 256 * 256;
    G.counters = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(workspace) + ybytes);
  } else {
    KB_REQUIRE(y, KB_ERR_NULL_POINTER, "NULL output pointer");
  }
  const int64_t TR = T * R;
  const int maxtok = (int)std::min<int64_t>(TR, 16);
  const int nsub = (maxtok > 8) ? 2 : 1;
  P.tok_cap = 8 * nsub;
  P.tstride = token_stride(G.K);
  const int staged = std::min(P.tok_cap, maxtok);
  P.red_off = ((staged * P.tstride) + 127) / 128 * 128;
  P.plan_off = P.red_off + NW * nsub * 32 * 4 * (int)sizeof(float);
  const size_t smem = (size_t)P.plan_off + (size_t)(3 * E + 2 + TR) * sizeof(int);
  const int64_t max_slots = std::min<int64_t>(E, TR);
  const int grid_items = (int)std::min<int64_t>(max_slots * G.items_rb, 1 << 20);
  return nsub == 2 ? engine_launch<2>(P, grid_items, smem, stream)
                   : engine_launch<1>(P, grid_items, smem, stream);
}

}  // namespace kb

// ---------------------------------------------------------------------------
// C ABI.
// ---------------------------------------------------------------------------
extern "C" {

int kb_w4a16_dense(const uint16_t* x, int64_t x_stride, int64_t M, int64_t K,
                   const uint8_t* packed, const uint16_t* scales, int64_t N, int64_t group,
                   uint16_t* y, int64_t y_stride, void* stream) {
  kb::clear_error();
  kb_dense_problem p = {x, x_stride, M, K, packed, scales, N, group, y, y_stride};
  return kb::dense_multi_impl(&p, 1, stream);
}

int kb_w4a16_dense_multi(const kb_dense_problem* problems, int count, void* stream) {
  kb::clear_error();
  return kb::dense_multi_impl(problems, count, stream);
}

int kb_w4a16_grouped(const uint16_t* x, int64_t x_stride, int64_t T, int64_t K,
                     const int64_t* idx, int64_t R, const uint8_t* packed,
                     const uint16_t* scales, int64_t E, int64_t N, int64_t group, uint16_t* y,
                     void* stream) {
  kb::clear_error();
  return kb::grouped_impl(kb::MODE_GROUPED, x, x_stride, T, K, idx, R, packed, scales, nullptr,
                          nullptr, E, N, group, y, nullptr, 0, nullptr, nullptr, 0, stream);
}

int kb_w4a16_swiglu(const uint16_t* x, int64_t x_stride, int64_t T, int64_t K,
                    const int64_t* idx, int64_t R, const uint8_t* w1_packed,
                    const uint16_t* w1_scales, const uint8_t* w3_packed,
                    const uint16_t* w3_scales, int64_t E, int64_t N, int64_t group,
                    uint16_t* y, void* stream) {
  kb::clear_error();
  return kb::grouped_impl(kb::MODE_SWIGLU, x, x_stride, T, K, idx, R, w1_packed, w1_scales,
                          w3_packed, w3_scales, E, N, group, y, nullptr, 0, nullptr, nullptr, 0,
                          stream);
}

size_t kb_w4a16_w2_combine_workspace_size(int64_t T, int64_t R, int64_t N) {
  if (T <= 0 || R <= 0 || N <= 0) return 0;
  // Per-route outputs, then one arrival counter per (token, row group).  The
  // smallest row group is 16 rows, so N/16 + 1 counters per token suffice.
  const size_t ybytes = ((size_t)T * R * N * 2 + 255) / 256 * 256;
  const size_t cbytes = (size_t)T * ((size_t)N / 16 + 1) * sizeof(int);
  return ybytes + (cbytes + 255) / 256 * 256;
}

int kb_w4a16_w2_combine(const uint16_t* activated, int64_t T, int64_t R, int64_t K,
                        const int64_t* idx, const float* weights, int64_t w_stride,
                        const uint8_t* w2_packed, const uint16_t* w2_scales, int64_t E,
                        int64_t N, int64_t group, uint16_t* out, void* workspace,
                        size_t workspace_bytes, void* stream) {
  kb::clear_error();
  if (T > 0) {
    KB_REQUIRE(w_stride >= R - 1, KB_ERR_BAD_SHAPE, "weights row stride %lld < R-1",
               (long long)w_stride);
  }
  return kb::grouped_impl(kb::MODE_W2C, activated, K, T, K, idx, R, w2_packed, w2_scales,
                          nullptr, nullptr, E, N, group, nullptr, weights, w_stride, out,
                          workspace, workspace_bytes, stream);
}

}  // extern "C"
