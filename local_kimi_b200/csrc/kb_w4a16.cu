// kb_w4a16.cu - W4A16 projection engine for sm_100a.
//
// One persistent kernel serves every INT4-weight projection of the decode hot
// path: dense (w4a16_dense, fused QKV), expert-grouped (w4a16_grouped), fused
// gate/up + SwiGLU (w4a16_swiglu) and down projection + weighted combine
// (fused_w2_combine).  Work is split into items: an item is RBc 16-row blocks
// of one weight matrix (or of the w1/w3 pair) over the full reduction axis,
// for all tokens that use that matrix.
//
// Data movement.  A producer warp streams each item's packed codes (one
// cp.async.bulk per weight row, L2 evict-first) and its bf16 scales (one bulk
// copy per matrix and item) from HBM into a ring of shared-memory stages
// guarded by mbarriers (full: transaction bytes; empty: one arrival per
// consumer warp).  Rows land with a padded stride (K/2 + pad, the pad making
// the stride 64 mod 128 bytes) so the consumers' 16-byte fragment loads are
// bank-conflict free.  For dense problems the producer starts streaming before
// the programmatic-dependent-launch wait: no kernel of this library that lets
// its successor start early writes packed weights or scales, so their fetch
// overlaps the tail of the kernel in front.
//
// Compute.  Eight consumer warps each own one 16-row block and one slice of
// the reduction axis of the item.  A lane decodes 16-byte pieces of two rows
// to bf16(code * scale) with bf16x2 arithmetic (decode_word) and feeds the
// tensor core through mma.m16n8k16: weights are the 16x16 A operand, eight
// tokens of activations (staged in shared memory in decode pair order) are the
// B operand, fp32 accumulation in two independent accumulator sets.
// Reduction-axis slices are summed in a fixed order through shared memory, so
// every output is deterministic run to run.
//
// Reference semantics (engine/kernels/w4a16_gemv.py:56-174, :224-392,
// engine/kernels/moe_combine.py:209-261): decoded weight bf16(code*scale),
// fp32 products and sums, bf16 projection outputs, SwiGLU rounding contract
// silu(bf16 g) -> bf16, times bf16 u -> bf16, combine = bf16(fp32 sum of the
// routed outputs times fp32 weights) + shared output (bf16 add).
#include "kb_engine.cuh"

#include <algorithm>
#include <mutex>

namespace kb {

struct DenseProb {
  const uint16_t* x;
  int64_t xs;
  const uint8_t* w;
  const uint16_t* s;
  uint16_t* y;
  int64_t ys;
  int M, K, N, gshift;
  int KS, RBc, items;
  int item_begin;
  int x_off;  // resident activations: byte offset of token 0 (-1: streamed per group)
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
  int x_rows;  // resident activation rows (T, or T*R for W2C); 0: streamed per group
};

struct EngineParams {
  int mode;
  int tok_cap;      // tokens per compute group (8 * NSUB)
  int tstride;      // bytes per staged token row
  int x_bytes;      // bytes of the activation region
  int stage_bytes;  // bytes per ring stage
  int stages;
  int ring_off, red_off, plan_off, bar_off;
  int total_items;  // dense
  int nprob;
  uint32_t* err;
  DenseProb prob[KB_MAX_DENSE_PROBLEMS];
  GroupedArgs g;
};

__device__ __forceinline__ void describe_dense(const EngineParams& P, int item, Item& it) {
  int p = 0;
  while (p + 1 < P.nprob && item >= P.prob[p + 1].item_begin) ++p;
  const DenseProb& D = P.prob[p];
  const int rbg = item - D.item_begin;
  it.mats = 1;
  it.w[0] = D.w;
  it.s[0] = D.s;
  it.w[1] = nullptr;
  it.s[1] = nullptr;
  it.K = D.K;
  it.N = D.N;
  it.gshift = D.gshift;
  it.KS = D.KS;
  it.RBc = D.RBc;
  it.r0 = rbg * D.RBc * 16;
  it.rows = min(D.RBc * 16, D.N - it.r0);
  it.RS = row_stride_bytes(D.K);
  it.ng = D.K >> (5 + D.gshift);
  it.scale_bulk = scale_bulk_ok(D.s, it.r0, it.rows, it.ng);
  it.p = p;
  it.abase = 0;
  it.count = D.M;
}

__device__ __forceinline__ void describe_grouped(const EngineParams& P, int item,
                                                 const int* slot_expert, const int* slot_start,
                                                 Item& it) {
  const GroupedArgs& G = P.g;
  const int slot = item / G.items_rb;
  const int rbg = item - slot * G.items_rb;
  const int e = slot_expert[slot];
  it.mats = (P.mode == MODE_SWIGLU) ? 2 : 1;
  it.w[0] = G.w0 + (size_t)e * (size_t)G.wse;
  it.s[0] = G.s0 + (size_t)e * (size_t)G.sse;
  it.w[1] = (it.mats == 2) ? G.w1 + (size_t)e * (size_t)G.wse : nullptr;
  it.s[1] = (it.mats == 2) ? G.s1 + (size_t)e * (size_t)G.sse : nullptr;
  it.K = G.K;
  it.N = G.N;
  it.gshift = G.gshift;
  it.KS = G.KS;
  it.RBc = G.RBc;
  it.r0 = rbg * G.RBc * 16;
  it.rows = min(G.RBc * 16, G.N - it.r0);
  it.RS = row_stride_bytes(G.K);
  it.ng = G.K >> (5 + G.gshift);
  it.scale_bulk = scale_bulk_ok(it.s[0], it.r0, it.rows, it.ng) &&
                  (it.mats == 1 || scale_bulk_ok(it.s[1], it.r0, it.rows, it.ng));
  it.p = slot;
  it.abase = slot_start[slot];
  it.count = slot_start[slot + 1] - it.abase;
}

// Build the expert-major assignment plan in shared memory: used experts in
// ascending order (slot_expert), the start of each slot's assignments
// (slot_start) and assignment ids ordered by (expert, id) (assign).  All
// NTHREADS threads take part.
__device__ int build_plan(const GroupedArgs& G, uint32_t* err, int* cnt, int* slot_expert,
                          int* slot_start, int* assign) {
  __shared__ int s_nslots;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int TR = G.T * G.R;
  const int E = G.E;
  for (int e = threadIdx.x; e <= E; e += NTHREADS) cnt[e] = 0;
  __syncthreads();
  for (int a = threadIdx.x; a < TR; a += NTHREADS) {
    const int64_t v = G.idx[a];
    if (v == EXPERT_NONE) continue;  // empty slot: no weights read, no output written
    atomicAdd(&cnt[clamp_expert(v, E, err)], 1);
  }
  __syncthreads();
  if (warp == 0) {
    // Each lane scans a contiguous run of experts; one warp-wide scan joins
    // the runs, so the pass over E experts takes ceil(E/32) steps per lane.
    const int per = (E + 31) / 32;
    const int e0 = lane * per, e1 = min(E, e0 + per);
    int tot = 0, used_cnt = 0;
    for (int e = e0; e < e1; ++e) {
      const int c = cnt[e];
      tot += c;
      used_cnt += (c > 0);
    }
    int incl = tot, uincl = used_cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, incl, o);
      const int un = __shfl_up_sync(0xffffffffu, uincl, o);
      if (lane >= o) {
        incl += n;
        uincl += un;
      }
    }
    int running = incl - tot, rank = uincl - used_cnt;
    for (int e = e0; e < e1; ++e) {
      const int c = cnt[e];
      if (c > 0) {
        slot_expert[rank] = e;
        slot_start[rank] = running;
        ++rank;
      }
      cnt[e] = running;
      running += c;
    }
    const int nslots = __shfl_sync(0xffffffffu, uincl, 31);
    running = __shfl_sync(0xffffffffu, incl, 31);
    if (lane == 0) {
      slot_start[nslots] = running;
      s_nslots = nslots;
    }
    __syncwarp();
    for (int base = 0; base < TR; base += 32) {
      const int a = base + lane;
      const int64_t v = a < TR ? G.idx[a] : EXPERT_NONE;
      const bool valid = v != EXPERT_NONE;
      int e = -1 - lane;
      if (valid) e = (v < 0 || v >= E) ? 0 : static_cast<int>(v);
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

// Global source row of the activations of token slot m of an item.
__device__ __forceinline__ const uint16_t* token_src(const EngineParams& P, const Item& it,
                                                     const int* assign, int m) {
  if (P.mode == MODE_DENSE) {
    const DenseProb& D = P.prob[it.p];
    return D.x + (size_t)m * D.xs;
  }
  const int a = assign[it.abase + m];
  return (P.mode == MODE_W2C) ? P.g.x + (size_t)a * P.g.xs
                              : P.g.x + (size_t)(a / P.g.R) * P.g.xs;
}

// Byte offset of token slot m's row inside the resident activation region.
__device__ __forceinline__ int resident_off(const EngineParams& P, const Item& it,
                                            const int* assign, int m) {
  if (P.mode == MODE_DENSE) return P.prob[it.p].x_off + m * P.tstride;
  const int a = assign[it.abase + m];
  return ((P.mode == MODE_W2C) ? a : a / P.g.R) * P.tstride;
}

template <int NSUB>
__global__ void __launch_bounds__(NTHREADS, 1)
    w4a16_engine(const __grid_constant__ EngineParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_done[16];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool producer = warp == NCW;
  uint8_t* xs = smem;
  uint8_t* ring = smem + P.ring_off;
  float* red = reinterpret_cast<float*>(smem + P.red_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + P.bar_off);
  uint64_t* empty = full + P.stages;
  int* cnt = reinterpret_cast<int*>(smem + P.plan_off);

  if (threadIdx.x == 0) {
    for (int s = 0; s < P.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NCW);
    }
    mbar_fence_init();
  }
  __syncthreads();

  const bool dense = P.mode == MODE_DENSE;
  int nitems = 0;
  int* slot_expert = nullptr;
  int* slot_start = nullptr;
  int* assign = nullptr;
  bool x_resident = false;

  if (dense) {
    nitems = P.total_items;
    x_resident = P.prob[0].x_off >= 0;
    if (producer) {
      // Weights never depend on the previous kernel: start streaming at once
      // and wait for that kernel only when the ring is full.
      const uint64_t pol = l2_evict_first_policy();
      int use = 0;
      bool waited = false;
      for (int item = blockIdx.x; item < nitems; item += gridDim.x, ++use) {
        if (!waited && use >= P.stages) {
          pdl_wait();
          waited = true;
        }
        const int s = use % P.stages;
        const uint32_t ph = (use / P.stages) & 1;
        if (!mbar_wait_bounded(&empty[s], ph ^ 1)) {
          if (lane == 0) atomicOr(P.err, ERR_TIMEOUT);
          break;
        }
        Item it;
        describe_dense(P, item, it);
        produce_item(it, ring + (size_t)s * P.stage_bytes, &full[s], pol);
      }
      if (!waited) pdl_wait();
      return;
    }
    pdl_wait();
    pdl_launch_dependents();
    if (x_resident) {
      for (int p = 0; p < P.nprob; ++p) {
        const DenseProb& D = P.prob[p];
        bool dup = false;
        for (int q = 0; q < p; ++q) dup |= (P.prob[q].x_off == D.x_off);
        if (dup) continue;
        for (int m = 0; m < D.M; ++m)
          stage_row(xs + D.x_off + m * P.tstride, D.x + (size_t)m * D.xs, D.K, threadIdx.x, NCT);
      }
    }
    named_barrier(CBAR, NCT);
  } else {
    pdl_wait();
    pdl_launch_dependents();
    const GroupedArgs& G = P.g;
    slot_expert = cnt + (G.E + 1);
    slot_start = slot_expert + G.E;
    assign = slot_start + (G.E + 1);
    const int nslots = build_plan(G, P.err, cnt, slot_expert, slot_start, assign);
    nitems = nslots * G.items_rb;
    x_resident = G.x_rows > 0;
    if (x_resident) {
      for (int r = 0; r < G.x_rows; ++r)
        stage_row(xs + r * P.tstride, G.x + (size_t)r * G.xs, G.K, threadIdx.x, NTHREADS);
    }
    __syncthreads();
    if (producer) {
      const uint64_t pol = l2_evict_first_policy();
      int use = 0;
      for (int item = blockIdx.x; item < nitems; item += gridDim.x, ++use) {
        const int s = use % P.stages;
        const uint32_t ph = (use / P.stages) & 1;
        if (!mbar_wait_bounded(&empty[s], ph ^ 1)) {
          if (lane == 0) atomicOr(P.err, ERR_TIMEOUT);
          break;
        }
        Item it;
        describe_grouped(P, item, slot_expert, slot_start, it);
        produce_item(it, ring + (size_t)s * P.stage_bytes, &full[s], pol);
      }
      return;
    }
  }

  // ---------------- consumers ----------------
  const int g = lane >> 2, t = lane & 3;
  int rslot = 0;
  int use = 0;
  for (int item = blockIdx.x; item < nitems; item += gridDim.x, ++use) {
    Item it;
    if (dense)
      describe_dense(P, item, it);
    else
      describe_grouped(P, item, slot_expert, slot_start, it);
    const int s = use % P.stages;
    const uint32_t ph = (use / P.stages) & 1;
    if (!mbar_wait_bounded(&full[s], ph)) {
      if (lane == 0) atomicOr(P.err, ERR_TIMEOUT);
      break;
    }
    uint8_t* stage = ring + (size_t)s * P.stage_bytes;
    const int per_mat = it.RBc * it.KS;
    const int mat = warp / per_mat;
    const int rem = warp - mat * per_mat;
    const int rb = rem / it.KS;
    const int ks = rem - rb * it.KS;
    const int KB = (it.K + 127) >> 7;
    const int kb0 = KB * ks / it.KS, kb1 = KB * (ks + 1) / it.KS;
    const int rb_rows = min(16, it.rows - rb * 16);
    const uint8_t* wtile = stage + (mat * it.RBc * 16 + rb * 16) * it.RS;
    const uint16_t* srow =
        it.scale_bulk ? reinterpret_cast<const uint16_t*>(stage + stage_scale_offset(it) +
                                                          mat * stage_scale_stride(it)) +
                            rb * 16 * it.ng
                      : (mat ? it.s[1] : it.s[0]) + (size_t)(it.r0 + rb * 16) * it.ng;

    for (int gb = 0; gb < it.count; gb += P.tok_cap) {
      const int ntok = min(P.tok_cap, it.count - gb);
      const uint8_t* xrow[NSUB];
      if (x_resident) {
#pragma unroll
        for (int q = 0; q < NSUB; ++q)
          xrow[q] = xs + resident_off(P, it, assign, gb + min(q * 8 + g, ntok - 1));
      } else {
        named_barrier(CBAR, NCT);
        for (int m = 0; m < ntok; ++m)
          stage_row(xs + m * P.tstride, token_src(P, it, assign, gb + m), it.K, threadIdx.x,
                    NCT);
        named_barrier(CBAR, NCT);
#pragma unroll
        for (int q = 0; q < NSUB; ++q) xrow[q] = xs + min(q * 8 + g, ntok - 1) * P.tstride;
      }
      float acc[NSUB][4];
#pragma unroll
      for (int q = 0; q < NSUB; ++q)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[q][i] = 0.f;
      if (rb_rows > 0)
        rowblock_compute<NSUB>(wtile, it.RS, srow, it.ng, rb_rows, it.K, it.gshift, kb0, kb1,
                               xrow, (ntok + 7) >> 3, acc);
      float* rbuf = red + rslot * (NCW * NSUB * 128);
#pragma unroll
      for (int q = 0; q < NSUB; ++q)
        *reinterpret_cast<float4*>(rbuf + ((warp * NSUB + q) * 32 + lane) * 4) =
            make_float4(acc[q][0], acc[q][1], acc[q][2], acc[q][3]);
      named_barrier(CBAR, NCT);
      if (mat == 0 && ks == 0 && rb_rows > 0) {
#pragma unroll
        for (int q = 0; q < NSUB; ++q) {
          float v0[4] = {0.f, 0.f, 0.f, 0.f};
          float v1[4] = {0.f, 0.f, 0.f, 0.f};
          for (int k2 = 0; k2 < it.KS; ++k2) {
            const float4 pv = *reinterpret_cast<const float4*>(
                rbuf + (((warp + k2) * NSUB + q) * 32 + lane) * 4);
            v0[0] += pv.x;
            v0[1] += pv.y;
            v0[2] += pv.z;
            v0[3] += pv.w;
            if (P.mode == MODE_SWIGLU) {
              const float4 uv = *reinterpret_cast<const float4*>(
                  rbuf + (((warp + per_mat + k2) * NSUB + q) * 32 + lane) * 4);
              v1[0] += uv.x;
              v1[1] += uv.y;
              v1[2] += uv.z;
              v1[3] += uv.w;
            }
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int rloc = rb * 16 + g + ((i >> 1) << 3);
            const int tok = q * 8 + 2 * t + (i & 1);
            if (rloc < it.rows && tok < ntok) {
              const int row = it.r0 + rloc;
              if (dense) {
                const DenseProb& D = P.prob[it.p];
                D.y[(size_t)(gb + tok) * D.ys + row] = float_to_bf16_bits(v0[i]);
              } else {
                const int a = assign[it.abase + gb + tok];
                const size_t o = (size_t)a * P.g.N + row;
                if (P.mode == MODE_GROUPED)
                  P.g.y[o] = float_to_bf16_bits(v0[i]);
                else if (P.mode == MODE_SWIGLU)
                  P.g.y[o] = float_to_bf16_bits(swiglu_contract(v0[i], v1[i]));
                else
                  P.g.wsy[o] = float_to_bf16_bits(v0[i]);
              }
            }
          }
        }
      }
      rslot ^= 1;
      if (P.mode == MODE_W2C) {
        // Arrival: once all R routes of a token have written this row group,
        // the CTA that arrives last combines them in fixed route order.
        const GroupedArgs& G = P.g;
        const int rbg = it.r0 / (G.RBc * 16);
        // One thread publishes the group: the barrier orders every consumer's
        // stores before its release fence, and the fence before the counters.
        named_barrier(CBAR, NCT);
        if (threadIdx.x == 0) {
          __threadfence();
          for (int m = 0; m < ntok; ++m) {
            const int a = assign[it.abase + gb + m];
            const int tok = a / G.R;
            const int old = atomicAdd(&G.counters[tok * G.items_rb + rbg], 1);
            s_done[m] = (old == G.R - 1) ? tok : -1;
          }
          __threadfence();  // acquire side for the combine below
        }
        named_barrier(CBAR, NCT);
        for (int m = 0; m < ntok; ++m) {
          const int tok = s_done[m];
          if (tok < 0) continue;
          for (int rl = threadIdx.x; rl < it.rows; rl += NCT) {
            const int row = it.r0 + rl;
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
        // s_done is rewritten by the next group only after its barriers.
      }
    }
    // This warp has finished reading stage s.
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------

// Warp split for a reduction width: KS warps share a 16-row block and RBc row
// blocks make an item, mats * RBc * KS == NCW.  KS starts where every warp
// covers at least four 128-wide blocks; while the problem yields fewer than
// two items per SM it doubles (smaller items), as long as each warp keeps two
// blocks.  `row_blocks` is the number of 16-row blocks of all matrices the
// launch covers.
static void choose_split(int K, int mats, int64_t row_blocks, int sms, int* KS, int* RBc) {
  const int KB = (K + 127) / 128;
  const int maxks = NCW / mats;
  int ks = 1;
  while (ks * 2 <= maxks && KB / (ks * 2) >= 4) ks *= 2;
  while (ks * 2 <= maxks && KB / (ks * 2) >= 2 &&
         row_blocks / (maxks / ks) < 2 * (int64_t)sms)
    ks *= 2;
  *KS = ks;
  *RBc = maxks / ks;
}

template <int NSUB>
static int engine_launch(EngineParams& P, int grid_items, size_t fixed_smem, void* stream) {
  static std::once_flag once[2];
  static cudaError_t attr_err[2] = {cudaSuccess, cudaSuccess};
  std::call_once(once[NSUB - 1], [] {
    attr_err[NSUB - 1] = cudaFuncSetAttribute(
        w4a16_engine<NSUB>, cudaFuncAttributeMaxDynamicSharedMemorySize, MAX_SMEM);
  });
  KB_REQUIRE(attr_err[NSUB - 1] == cudaSuccess, KB_ERR_LAUNCH,
             "cudaFuncSetAttribute failed: %s", cudaGetErrorString(attr_err[NSUB - 1]));
  // The ring takes what the fixed regions (activations, reduction, plan) leave.
  const size_t reserve = SMEM_RESERVE;
  KB_REQUIRE(fixed_smem + reserve + 2 * (size_t)P.stage_bytes <= (size_t)MAX_SMEM,
             KB_ERR_UNSUPPORTED,
             "shared memory: %zu bytes of fixed regions leave no room for two %d-byte stages",
             fixed_smem, P.stage_bytes);
  const size_t avail = (size_t)MAX_SMEM - reserve - fixed_smem;
  P.stages = (int)std::min<size_t>(MAX_STAGES, avail / P.stage_bytes);
  P.ring_off = (int)((fixed_smem + 127) / 128 * 128);
  P.bar_off = P.ring_off + P.stages * P.stage_bytes;
  const size_t smem = (size_t)P.bar_off + 2 * P.stages * sizeof(uint64_t);
  KB_REQUIRE(smem + 256 <= (size_t)MAX_SMEM, KB_ERR_UNSUPPORTED, "shared memory plan overflow");
  const int dev = bind_stream_device(stream);
  P.err = device_error_word(dev);
  KB_REQUIRE(P.err != nullptr, KB_ERR_LAUNCH, "device error word unavailable");
  const int grid = std::max(1, std::min(grid_items, num_sms(dev)));
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
    KB_REQUIRE(q.K <= 16384 && q.N <= (int64_t(1) << 30) && q.M <= (int64_t(1) << 30),
               KB_ERR_UNSUPPORTED, "problem %d: size above the supported range (K <= 16384)",
               i);
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
    maxM = std::max(maxM, D.M);
    maxK = std::max(maxK, D.K);
    P.nprob++;
  }
  if (P.nprob == 0) return KB_OK;
  {
    int64_t row_blocks = 0;
    for (int i = 0; i < P.nprob; ++i) row_blocks += (P.prob[i].N + 15) / 16;
    const int sms = num_sms(bind_stream_device(stream));
    for (int i = 0; i < P.nprob; ++i)
      choose_split(P.prob[i].K, 1, row_blocks, sms, &P.prob[i].KS, &P.prob[i].RBc);
  }
  const int nsub = (maxM > 8) ? 2 : 1;
  P.tok_cap = 8 * nsub;
  P.tstride = token_stride(maxK);
  const int red_bytes = 2 * NCW * nsub * 128 * (int)sizeof(float);
  // Resident activations: every distinct x, all of its tokens.
  int xneed = 0;
  for (int i = 0; i < P.nprob; ++i) {
    DenseProb& D = P.prob[i];
    D.x_off = -1;
    for (int j = 0; j < i; ++j)
      if (P.prob[j].x == D.x && P.prob[j].xs == D.xs && P.prob[j].K == D.K &&
          P.prob[j].M == D.M)
        D.x_off = P.prob[j].x_off;
    if (D.x_off < 0) {
      D.x_off = xneed;
      xneed += D.M * P.tstride;
    }
  }
  auto max_stage = [&P]() {
    int st = 0;
    for (int i = 0; i < P.nprob; ++i) {
      const DenseProb& D = P.prob[i];
      st = std::max(st, item_stage_bytes(D.K, 1, D.RBc, D.K >> (5 + D.gshift)));
    }
    return st;
  };
  // Room for activations beside the reduction buffers and two stages.
  auto room = [&](int st) { return MAX_SMEM - SMEM_RESERVE - red_bytes - 2 * st - 128; };
  // More tokens than the resident budget allows: smaller items (fewer rows,
  // more reduction slices) when that lets every token stay resident, since
  // otherwise each item restages its activations for every token group.
  if (xneed > std::min(X_RESIDENT_BUDGET, room(max_stage()))) {
    int ks[KB_MAX_DENSE_PROBLEMS], rbc[KB_MAX_DENSE_PROBLEMS];
    for (int i = 0; i < P.nprob; ++i) {
      ks[i] = P.prob[i].KS;
      rbc[i] = P.prob[i].RBc;
    }
    bool shrunk = true;
    while (xneed > room(max_stage()) && shrunk) {
      shrunk = false;
      for (int i = 0; i < P.nprob; ++i) {
        DenseProb& D = P.prob[i];
        if (D.RBc > 1 && D.KS * 2 <= (D.K + 127) / 128) {
          D.RBc /= 2;
          D.KS *= 2;
          shrunk = true;
        }
      }
    }
    if (xneed > room(max_stage())) {
      for (int i = 0; i < P.nprob; ++i) {
        P.prob[i].KS = ks[i];
        P.prob[i].RBc = rbc[i];
      }
    }
  }
  int items = 0;
  for (int i = 0; i < P.nprob; ++i) {
    DenseProb& D = P.prob[i];
    D.items = (D.N + 16 * D.RBc - 1) / (16 * D.RBc);
    D.item_begin = items;
    items += D.items;
  }
  const int stage = max_stage();
  KB_REQUIRE(room(stage) >= P.tstride, KB_ERR_UNSUPPORTED,
             "shared memory cannot hold one activation row of K=%d next to two stages", maxK);
  int xbytes = xneed;
  if (xneed > room(stage)) {
    const int cap = std::min(X_RESIDENT_BUDGET, room(stage));
    for (int i = 0; i < P.nprob; ++i) P.prob[i].x_off = -1;
    P.tok_cap = std::min(P.tok_cap, std::max(1, cap / P.tstride));
    xbytes = P.tok_cap * P.tstride;
  }
  P.total_items = items;
  P.x_bytes = (xbytes + 127) / 128 * 128;
  P.red_off = P.x_bytes;
  P.plan_off = P.red_off + red_bytes;
  P.stage_bytes = stage;
  const size_t fixed = (size_t)P.plan_off;
  return nsub == 2 ? engine_launch<2>(P, items, fixed, stream)
                   : engine_launch<1>(P, items, fixed, stream);
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
  KB_REQUIRE(E <= 4096 && K <= 16384 && N <= (int64_t(1) << 24), KB_ERR_UNSUPPORTED,
             "E, K or N above the supported range (E <= 4096, K <= 16384)");
  KB_REQUIRE(x && idx && w0 && s0, KB_ERR_NULL_POINTER, "NULL input pointer");
  KB_REQUIRE(mode != MODE_SWIGLU || (w1 && s1), KB_ERR_NULL_POINTER, "NULL w3 pointer");
  KB_REQUIRE(aligned(x, 16) && x_stride % 8 == 0 && x_stride >= K, KB_ERR_ALIGNMENT,
             "activations must be 16-byte aligned with a row stride that is a multiple of 8 "
             "elements and >= K");
  KB_REQUIRE(aligned(w0, 16) && (!w1 || aligned(w1, 16)), KB_ERR_ALIGNMENT,
             "packed weights must be 16-byte aligned");
  KB_REQUIRE(aligned(s0, 2) && (!s1 || aligned(s1, 2)), KB_ERR_ALIGNMENT,
             "scales must be 2-byte aligned");
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
  const int64_t slots = std::min<int64_t>(E, T * R);
  choose_split(G.K, mats, slots * ((N + 15) / 16), num_sms(bind_stream_device(stream)), &G.KS,
               &G.RBc);
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
  // An expert serves at most T assignments when each token routes to distinct
  // experts; more (repeated experts within a token) still works through
  // several token groups.
  const int nsub = (T > 8) ? 2 : 1;
  P.tok_cap = 8 * nsub;
  P.tstride = token_stride(G.K);
  P.stage_bytes = item_stage_bytes(G.K, mats, G.RBc, G.K >> (5 + gs));
  const int red_bytes = 2 * NCW * nsub * 128 * (int)sizeof(float);
  const size_t plan_bytes = ((size_t)(3 * E + 2 + TR) * sizeof(int) + 127) / 128 * 128;
  const int x_budget = std::min<int>(
      X_RESIDENT_BUDGET,
      MAX_SMEM - SMEM_RESERVE - red_bytes - (int)plan_bytes - 2 * P.stage_bytes - 128);
  KB_REQUIRE(x_budget >= P.tstride, KB_ERR_UNSUPPORTED,
             "shared memory cannot hold one activation row of K=%d next to two stages", G.K);
  const int64_t xrows = (mode == MODE_W2C) ? TR : T;
  if (xrows * P.tstride <= x_budget) {
    G.x_rows = (int)xrows;
    P.x_bytes = (int)xrows * P.tstride;
  } else {
    G.x_rows = 0;
    P.tok_cap = std::min(P.tok_cap, x_budget / P.tstride);
    P.x_bytes = P.tok_cap * P.tstride;
  }
  P.x_bytes = (P.x_bytes + 127) / 128 * 128;
  P.red_off = P.x_bytes;
  P.plan_off = P.red_off + red_bytes;
  const size_t fixed = (size_t)P.plan_off + plan_bytes;
  const int64_t max_slots = std::min<int64_t>(E, TR);
  const int grid_items = (int)std::min<int64_t>(max_slots * G.items_rb, 1 << 20);
  return nsub == 2 ? engine_launch<2>(P, grid_items, fixed, stream)
                   : engine_launch<1>(P, grid_items, fixed, stream);
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
