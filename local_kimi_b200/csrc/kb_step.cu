// kb_step.cu - decode-step executor for sm_100a: one persistent launch runs a
// whole program of hot-path operations.
//
// A decode step of the hot path is ~150 dependent operations (per layer: the
// attention projections, the KDA state step, the router, the expert gate/up
// and down+combine; then the lm_head), each of which moves a few MB.  Issued
// as separate kernels every operation pays launch, ramp-up, DRAM latency and
// drain (several microseconds) although its data takes well under one at HBM
// rate.  This executor keeps one CTA per SM resident for the whole step:
//
//  * The producer warp of every CTA walks the program and streams the weights
//    of every item assigned to its CTA (plain cp.async.bulk, L2 evict-first)
//    into a ring of shared-memory stages, as far ahead as the ring allows.
//    Weights never depend on the step's activations, so the stream runs across
//    the dependencies between operations; only the routed experts wait for
//    the routing of their layer.
//  * The consumer warps walk the same program.  Before an operation reads its
//    inputs they wait on device completion counters of the operations that
//    produce them (published with a release fence + atomic add by the warps
//    that wrote them, observed with acquire loads; every wait is bounded in
//    time and a shared abort flag ends the launch on any failure).
//  * Item arithmetic is the projection engine's (kb_engine.cuh): bf16(code *
//    scale) decode, mma.sync m16n8k16, fp32 sums in a fixed order.
//
// Operations: OP_DENSE (up to three INT4 projections), OP_ROUTER (fp32 router
// logits of eight experts per item), OP_MOE_UP (top-k selection and expert
// plan, then gate/up + SwiGLU of the shared expert and the routed experts),
// OP_MOE_DOWN (down projection of every route, then the weighted combine by
// the CTA that completes a (token, row group)), OP_KDA (recurrent state step).
// Results equal those of the per-operation kernels up to fp32 summation order
// (KDA row partials, router logits).
//
// Reference semantics: engine/kernels/w4a16_gemv.py:56-174 (decode and
// projections), engine/kernels/__init__.py:182-218 (SwiGLU contract),
// engine/klinear/router.py:47-85 (router), engine/klinear/moe.py:278-334 and
// engine/kernels/moe_combine.py:209-261 (expert dispatch and combine),
// engine/kernels/kda_step.py:173-196 (KDA step).
#include "kb_engine.cuh"
#include "kb_topk.cuh"

#include <cstring>
#include <mutex>
#include <new>
#include <vector>

namespace kb {

enum : int { OP_DENSE = 0, OP_ROUTER = 1, OP_MOE_UP = 2, OP_MOE_DOWN = 3, OP_KDA = 4 };

constexpr int ST_MAX_DEPS = KB_STEP_MAX_DEPS;
constexpr int ST_MAX_PROB = 3;
constexpr int ST_MAX_T = KB_STEP_MAX_TOKENS;
constexpr int ST_MAX_TOPK = 8;
constexpr int ST_MAX_R = ST_MAX_TOPK + 1;
constexpr int ST_MAX_E = 256;
constexpr int ST_MAX_SLOTS = 1 + ST_MAX_T * ST_MAX_TOPK;
constexpr int ST_RT_EXPERTS = 8;          // router experts per item (two warps each)
constexpr int ST_KDA_COLS = 32;
constexpr int ST_STAGE_TARGET = 40 * 1024;  // preferred bytes per item
constexpr long long ST_WAIT_NS = 2000000000LL;  // 2 s per wait
// Timeline fields per (CTA, operation): consumers start, inputs ready,
// routing built (expert blocks), end; producer done issuing; reducer done;
// shared-expert items done (expert gate/up); spare.
constexpr int ST_TRACE_FIELDS = 8;
constexpr int ST_REDUCERS = 2;        // reducer warps, alternating over the items
constexpr int ST_THREADS = NCT + 32 * (2 + ST_REDUCERS);  // consumers, producer (warp NCW),
                                      // reducers (NCW+1 ..), stager (last warp)
constexpr int ST_NB = 4;              // partial-sum buffers between consumers and reducer
constexpr int ST_DNB = 4;             // down-projection input buffers (stager to consumers)
constexpr int EXIT_BAR = 2;           // named barrier: consumers + reducers

struct StDense {
  const uint16_t* x;
  int64_t xs;
  const uint8_t* w;
  const uint16_t* s;
  const uint8_t* w3;   // gate/up pair: up matrix (mats == 2), SwiGLU epilogue
  const uint16_t* s3;
  uint16_t* y;
  int64_t ys;
  int K, N, gshift, KS, RBc, nchunk, mats;
  int items, item_begin, x_off;
  int xcomb;  // x is the output of the down operation just before: staged as its combine
  uint32_t* ytag;        // tagged copy of y ([T][N] words), read by the next operation
  uint32_t* xtag;        // x read from the previous operation's tagged copy ([T][K] words)
};

struct StOp {
  int type;
  int ndeps;
  int dep[ST_MAX_DEPS];
  int done;    // sync index of the completion counter
  int target;  // completion count (every op but OP_MOE_UP)
  int rot;     // item i runs on CTA (i + rot) % grid
  int T;
  int items;   // static items (dense, router, KDA)
  int cstage;  // dense/router: the consumers stage the activations (input of the previous operation)
  int comb_src;  // dense: down operation whose combine the consumers compute while staging, or -1
  int tag_src;   // operation whose output this one reads as tagged words (no counter wait), or -1
  uint32_t* rxtag;        // router: hidden rows read from a tagged copy ([T][K] words)
  uint32_t* ktag;         // KDA: tagged copy of the bf16 output ([B][H*Dv] words)
  uint32_t* wtag;         // down: tagged copy of the per-route outputs ([T*R][N] words)
  // dense
  int nprob;
  StDense p[ST_MAX_PROB];
  // router
  const uint16_t* rx;
  int64_t rxs;
  const uint16_t* rw;
  const float* rbias;
  int E, K, top_k, renorm;
  float scaling;
  unsigned long long* rwords;  // router words [2 parities][T][E]
  int64_t* idx_out;
  float* w_out;
  // experts (up and down)
  int router_op;
  int slot_cnt;    // sync index of the up op's per-slot counters
  int items_done;  // down: sync index of the count of finished down items
  const uint16_t* mx;
  int64_t mxs;
  const uint8_t* w0;
  const uint16_t* s0;
  const uint8_t* w1;
  const uint16_t* s1;
  int64_t wse, sse;
  int N, gshift, KS, RBc, items_rb, R, up_rb;
  int sbulk;  // expert scale banks 16-byte aligned per expert: items stage their scales
  uint16_t* y;
  uint16_t* out;
  uint16_t* wsy;
  // KDA
  float* state;
  int64_t sb, sh, sk;
  const float* q;
  const float* k;
  const float* v;
  const float* decay;
  const float* beta;
  int B, H, Dk, Dv;
  float scale;
  float* kout;
  uint16_t* kout_bf16;
};

struct StepParams {
  const StOp* ops;
  int nops;
  int* sync;
  int nsync;
  int exit_idx, abort_idx;
  int parity_idx;    // launch count (its parity selects the router words of this launch)
  uint32_t* err;
  int stages, stage_bytes;
  int ring_off, red_off, scr_off, bar_off;
  int part_bytes;  // partial-sum buffers at red_off
  int T;
  int x_bytes, nxb;  // activation buffers at 0 (nxb of x_bytes)
  int dnb, drow_bytes;  // down inputs: dnb buffers of drow_bytes inside the op's activation buffer
  int desc_off;      // nxb operation descriptor copies
  long long* trace;  // optional timeline [grid][nops][ST_TRACE_FIELDS] of %globaltimer ns
};

// Per-CTA routing state and plan (shared memory scratch).
struct StPlan {
  int route_e[ST_MAX_T * ST_MAX_R];     // expert of assignment t*R + r
  float route_w[ST_MAX_T * ST_MAX_TOPK];
  int slot_expert[ST_MAX_SLOTS];
  int slot_start[ST_MAX_SLOTS + 1];
  int assign[ST_MAX_T * ST_MAX_R];
  int slot_id[ST_MAX_T * ST_MAX_TOPK];
  int slot_of[ST_MAX_E + 1];
  int nslots;
  // Selection scratch, two tokens at a time: 8 candidates per warp of 32
  // experts (choice key, expert, sigmoid score), then the picks in choice
  // order.  A single token's routing (route_one) uses row 0 for the
  // candidates at or above its threshold.
  uint32_t cand_k[2][64];
  int cand_e[2][64];
  float cand_l[2][64];
  int pick_e[2][ST_MAX_TOPK];
  float pick_l[2][ST_MAX_TOPK];
  int done_tok[ST_MAX_T];
  int abort;
  int last;
  int parity;  // launch parity
  uint32_t launch;  // launches of this program before this one
  int cur_op;  // operation the consumers are in (timeline)
};

struct StKda {
  float ed[256], k[256], bk[256], q[256];
  float red[NCW][32];
};

// ---------------------------------------------------------------------------
// Device-side synchronisation.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ long long now_ns() {
  long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void trace_mark(const StepParams& P, int op, int field) {
  if (P.trace)
    P.trace[((size_t)blockIdx.x * P.nops + op) * ST_TRACE_FIELDS + field] = now_ns();
}

__device__ __forceinline__ void raise_abort(const StepParams& P, StPlan* pl, uint32_t bits) {
  atomicOr(P.err, bits);
  atomicExch(&P.sync[P.abort_idx], 1);
  pl->abort = 1;
}

// Thread 0 of the consumers waits until sync[idx] >= target (bounded), then
// all consumers pass a barrier.  Consumers never leave the common sequence of
// barriers early: after a failure every later wait returns at once and the
// launch runs to its end with the error recorded.
__device__ void consumers_wait(const StepParams& P, StPlan* pl, int idx, int target) {
  if (threadIdx.x == 0 && !pl->abort && target > 0) {
    const long long t0 = now_ns();
    int spins = 0;
    while (ld_acquire(&P.sync[idx]) < target) {
      __nanosleep(64);
      if (((++spins) & 15) == 0) {
        if (*((volatile int*)&P.sync[P.abort_idx]) != 0) {
          pl->abort = 1;
          break;
        }
        if (now_ns() - t0 > ST_WAIT_NS) {
          raise_abort(P, pl, ERR_TIMEOUT);
          break;
        }
      }
    }
  }
  named_barrier(CBAR, NCT);
}

__device__ void wait_deps(const StepParams& P, StPlan* pl, const StOp& op) {
  for (int d = 0; d < op.ndeps; ++d) {
    const StOp& dop = P.ops[op.dep[d]];
    consumers_wait(P, pl, dop.done, dop.target);
  }
  if (op.ndeps == 0) named_barrier(CBAR, NCT);
  if (threadIdx.x == 0) trace_mark(P, pl->cur_op, 1);
}

// Release reduction at GPU scope: the add becomes visible after every write
// that happens before it (cumulative release).
__device__ __forceinline__ void red_release(int* counter, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(counter), "r"(v) : "memory");
}

// Release: the writes of this warp (ordered by __syncwarp) before the add.
__device__ __forceinline__ void warp_signal(int* counter, int v) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) red_release(counter, v);
}

// Bounded mbarrier wait that also gives up when the CTA is aborting.
__device__ bool stage_wait(uint64_t* bar, uint32_t parity, const StPlan* pl) {
  if (mbar_test_wait(bar, parity)) return true;
  const long long t0 = now_ns();
  int spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if (((++spins) & 15) == 0) {
      if (*((volatile const int*)&pl->abort) != 0) return false;
      if (now_ns() - t0 > ST_WAIT_NS) return false;
    }
  }
  return true;
}

__device__ __forceinline__ int first_item(int rot) {
  const int G = gridDim.x;
  return ((int)blockIdx.x - rot % G + G) % G;
}

// Activation row into the B-fragment layout, read with L2-only loads (the row
// may have been written by another CTA of this launch); B loads per thread in
// flight before the stores.
template <int B = 1>
__device__ __forceinline__ void stage_row_cg(uint8_t* xs_row, const uint16_t* src, int K,
                                             int first, int step) {
  const int NC = K >> 5;
  const int words = K >> 3;
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
  for (int w0 = first; w0 < words; w0 += B * step) {
    uint4 v[B];
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const int w = w0 + b * step;
      if (w < words) v[b] = __ldcg(s4 + w);
    }
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const int w = w0 + b * step;
      if (w < words)
        *reinterpret_cast<uint4*>(xs_row + ((w & 3) * NC + (w >> 2)) * 16) = permute_pairs(v[b]);
    }
  }
}

// Tagged activations.  An operation whose output feeds the one right after it
// also writes each bf16 value as a 32-bit word with a tag in the high half:
// (launch * nops + op + 1) mod 2^16, distinct for every writer of a launch and
// from every word of the previous launch (2 * nops < 2^16), and never 0 in the
// first launch (the buffers start zeroed).  The reader polls the words
// themselves instead of a completion counter followed by the load: one L2
// round trip instead of two.  A word is one 32-bit store, so a reader sees
// the value and its tag together.  pl->launch is set by consumer thread 0
// before the first consumer barrier.
__device__ __forceinline__ uint32_t op_tag(const StPlan* pl, int nops, int o) {
  return (pl->launch * (uint32_t)nops + (uint32_t)o + 1u) & 0xffffu;
}

__device__ __forceinline__ void st_tag(uint32_t* p, uint16_t v, uint32_t tag) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"((uint32_t)v | (tag << 16))
               : "memory");
}

__device__ __forceinline__ uint4 ld_tags4(const uint32_t* p) {
  uint4 v;
  asm volatile("ld.relaxed.gpu.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__device__ __forceinline__ uint2 ld_tags2(const uint32_t* p) {
  uint2 v;
  asm volatile("ld.relaxed.gpu.global.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ bool tags_ok4(uint4 v, uint32_t tag) {
  return ((v.x >> 16) == tag) & ((v.y >> 16) == tag) & ((v.z >> 16) == tag) & ((v.w >> 16) == tag);
}

// Eight tagged values (8 consecutive elements from p, 16-byte aligned) as
// bf16x8 in natural order, once all carry `tag` (bounded wait).
__device__ uint4 poll_tagged8(const StepParams& P, StPlan* pl, const uint32_t* p, uint32_t tag) {
  uint4 a = ld_tags4(p), b = ld_tags4(p + 4);
  if (!(tags_ok4(a, tag) && tags_ok4(b, tag))) {
    const long long t0 = now_ns();
    for (int spins = 1;; ++spins) {
      __nanosleep(32);
      a = ld_tags4(p);
      b = ld_tags4(p + 4);
      if (tags_ok4(a, tag) && tags_ok4(b, tag)) break;
      if ((spins & 15) == 0) {
        if (*((volatile int*)&P.sync[P.abort_idx]) != 0 || *((volatile int*)&pl->abort) != 0) {
          pl->abort = 1;
          break;
        }
        if (now_ns() - t0 > ST_WAIT_NS) {
          raise_abort(P, pl, ERR_TIMEOUT);
          break;
        }
      }
    }
  }
  return make_uint4(prmt(a.x, a.y, 0x5410), prmt(a.z, a.w, 0x5410), prmt(b.x, b.y, 0x5410),
                    prmt(b.z, b.w, 0x5410));
}

// One combined value: bf16(sum_r routed_r * w_r, fp32 in route order) +
// shared (engine/kernels/moe_combine.py:209-261).
__device__ __forceinline__ uint16_t combine_value(const uint16_t (&rv)[ST_MAX_TOPK],
                                                  const float* rw, int top_k, uint16_t sv) {
  float accum = 0.f;
#pragma unroll
  for (int r = 0; r < ST_MAX_TOPK; ++r)
    if (r < top_k) accum = fmaf(bf16_bits_to_float(rv[r]), rw[r], accum);
  return float_to_bf16_bits(round_bf16(accum) + bf16_bits_to_float(sv));
}

// ---------------------------------------------------------------------------
// Item descriptions (identical on the producer and consumer side).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void st_describe_dense(const StOp& op, int item, Item& it) {
  int p = 0;
  while (p + 1 < op.nprob && item >= op.p[p + 1].item_begin) ++p;
  const StDense& D = op.p[p];
  const int rbg = item - D.item_begin;
  it.mats = D.mats;
  it.w[0] = D.w;
  it.s[0] = D.s;
  it.w[1] = D.w3;
  it.s[1] = D.s3;
  it.K = D.K;
  it.N = D.N;
  it.gshift = D.gshift;
  it.KS = D.KS;
  it.RBc = D.RBc;
  it.r0 = rbg * D.RBc * 16;
  it.rows = min(D.RBc * 16, D.N - it.r0);
  it.ng = D.K >> (5 + D.gshift);
  it.RS = (D.nchunk > 1) ? D.K / (2 * D.nchunk) : row_stride_bytes(D.K);
  it.scale_bulk = D.nchunk == 1 && scale_bulk_ok(D.s, it.r0, it.rows, it.ng) &&
                  (D.mats == 1 || scale_bulk_ok(D.s3, it.r0, it.rows, it.ng));
  it.p = p;
  it.abase = 0;
  it.count = op.T;
}

// Scales of an expert item are staged with its weights when every expert's
// scale rows start 16-byte aligned (host-checked) and the item's scale block
// is a whole number of 16-byte units (row offsets are multiples of 16 rows).
__device__ __forceinline__ bool expert_scale_bulk(const StOp& op, int rows) {
  return op.sbulk && ((rows * (op.K >> (5 + op.gshift)) * 2) & 15) == 0;
}

// Slot s of the plan: expert slot_expert[s], assignments assign[start..end).
__device__ __forceinline__ void st_describe_moe(const StOp& op, const StPlan* pl, int item,
                                                Item& it) {
  const int slot = item / op.items_rb;
  const int rbg = item - slot * op.items_rb;
  const int e = pl->slot_expert[slot];
  it.mats = (op.type == OP_MOE_UP) ? 2 : 1;
  it.w[0] = op.w0 + (size_t)e * (size_t)op.wse;
  it.s[0] = op.s0 + (size_t)e * (size_t)op.sse;
  it.w[1] = (it.mats == 2) ? op.w1 + (size_t)e * (size_t)op.wse : nullptr;
  it.s[1] = (it.mats == 2) ? op.s1 + (size_t)e * (size_t)op.sse : nullptr;
  it.K = op.K;
  it.N = op.N;
  it.gshift = op.gshift;
  it.KS = op.KS;
  it.RBc = op.RBc;
  it.r0 = rbg * op.RBc * 16;
  it.rows = min(op.RBc * 16, op.N - it.r0);
  it.RS = row_stride_bytes(op.K);
  it.ng = op.K >> (5 + op.gshift);
  it.scale_bulk = expert_scale_bulk(op, it.rows);
  it.p = slot;
  it.abase = pl->slot_start[slot];
  it.count = pl->slot_start[slot + 1] - it.abase;
}

// Shared slot 0 (the shared expert, every token) before the plan exists.
__device__ __forceinline__ void st_describe_shared(const StOp& op, int item, Item& it) {
  const int rbg = item;
  const int e = op.E;
  it.mats = (op.type == OP_MOE_UP) ? 2 : 1;
  it.w[0] = op.w0 + (size_t)e * (size_t)op.wse;
  it.s[0] = op.s0 + (size_t)e * (size_t)op.sse;
  it.w[1] = (it.mats == 2) ? op.w1 + (size_t)e * (size_t)op.wse : nullptr;
  it.s[1] = (it.mats == 2) ? op.s1 + (size_t)e * (size_t)op.sse : nullptr;
  it.K = op.K;
  it.N = op.N;
  it.gshift = op.gshift;
  it.KS = op.KS;
  it.RBc = op.RBc;
  it.r0 = rbg * op.RBc * 16;
  it.rows = min(op.RBc * 16, op.N - it.r0);
  it.RS = row_stride_bytes(op.K);
  it.ng = op.K >> (5 + op.gshift);
  it.scale_bulk = expert_scale_bulk(op, it.rows);
  it.p = 0;
  it.abase = 0;
  it.count = op.T;
}

// One reduction chunk of a chunked dense item: rows copied one by one.
__device__ __forceinline__ void produce_chunk(const Item& it, int nchunk, int ci, uint8_t* stage,
                                              uint64_t* full, uint64_t policy) {
  const int lane = threadIdx.x & 31;
  const uint32_t cbytes = (uint32_t)(it.K / (2 * nchunk));
  if (lane == 0) mbar_arrive_expect_tx(full, (uint32_t)it.rows * cbytes);
  __syncwarp();
  for (int r = lane; r < it.rows; r += 32)
    bulk_g2s(stage + (size_t)r * cbytes,
             it.w[0] + (size_t)(it.r0 + r) * (it.K / 2) + (size_t)ci * cbytes, cbytes, full,
             policy);
}

// ---------------------------------------------------------------------------
// Producer warp.
// ---------------------------------------------------------------------------
struct Ring {
  uint8_t* base;
  uint64_t* full;
  uint64_t* empty;
  int stages, stage_bytes;
  int use;     // stages used so far
  int slot;    // use % stages
  uint32_t phase;  // (use / stages) & 1
  __device__ __forceinline__ void advance() {
    ++use;
    if (++slot == stages) {
      slot = 0;
      phase ^= 1u;
    }
  }
};

__device__ bool ring_acquire(Ring& R, const StPlan* pl, uint8_t** stage, uint64_t** full) {
  const int s = R.slot;
  if (!stage_wait(&R.empty[s], R.phase ^ 1u, pl)) return false;
  *stage = R.base + (size_t)s * R.stage_bytes;
  *full = &R.full[s];
  R.advance();
  return true;
}

__device__ void producer_main(const StepParams& P, StPlan* pl, Ring& R, uint64_t* plan_bar,
                              uint64_t* plan_ack) {
  const int lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const uint64_t pol = l2_evict_first_policy();
  uint32_t plan_phase = 0;
  bool ok = true;
  for (int o = 0; o < P.nops && ok; ++o) {
    const StOp& op = P.ops[o];
    uint8_t* stage;
    uint64_t* full;
    if (o > 0 && lane == 0) trace_mark(P, o - 1, 4);
    if (op.type == OP_DENSE) {
      const int n = op.p[op.nprob - 1].item_begin + op.p[op.nprob - 1].items;
      for (int i = first_item(op.rot); i < n && ok; i += G) {
        Item it;
        st_describe_dense(op, i, it);
        const int nchunk = op.p[it.p].nchunk;
        for (int ci = 0; ci < nchunk && ok; ++ci) {
          ok = ring_acquire(R, pl, &stage, &full);
          if (!ok) break;
          if (nchunk == 1)
            produce_item(it, stage, full, pol);
          else
            produce_chunk(it, nchunk, ci, stage, full, pol);
        }
      }
    } else if (op.type == OP_ROUTER) {
      for (int i = first_item(op.rot); i < op.items && ok; i += G) {
        ok = ring_acquire(R, pl, &stage, &full);
        if (!ok) break;
        const int e0 = i * ST_RT_EXPERTS;
        const int ne = min(ST_RT_EXPERTS, op.E - e0);
        const uint32_t bytes = (uint32_t)ne * op.K * 2;
        if (lane == 0) {
          mbar_arrive_expect_tx(full, bytes);
          bulk_g2s(stage, op.rw + (size_t)e0 * op.K, bytes, full, pol);
        }
        __syncwarp();
      }
    } else if (op.type == OP_MOE_UP) {
      int i = first_item(op.rot);
      for (; i < op.items_rb && ok; i += G) {
        ok = ring_acquire(R, pl, &stage, &full);
        if (!ok) break;
        Item it;
        st_describe_shared(op, i, it);
        produce_item(it, stage, full, pol);
      }
      if (!ok) break;
      ok = stage_wait(plan_bar, plan_phase, pl);
      if (!ok) break;
      const int n = pl->nslots * op.items_rb;
      for (; i < n && ok; i += G) {
        ok = ring_acquire(R, pl, &stage, &full);
        if (!ok) break;
        Item it;
        st_describe_moe(op, pl, i, it);
        produce_item(it, stage, full, pol);
      }
    } else if (op.type == OP_KDA) {
      // The consumers read their state slices as soon as the inputs are ready:
      // bring the slices of this CTA's items into L2 now (the state is read
      // only by this operation; a prefetch moves no data to the SM).
      const int nsl = (op.Dv + ST_KDA_COLS - 1) / ST_KDA_COLS;
      for (int u = first_item(op.rot); u < op.items; u += G) {
        const int bh = u / nsl, sl = u - bh * nsl;
        const int b = bh / op.H, h = bh - b * op.H;
        const int cols = min(ST_KDA_COLS, op.Dv - sl * ST_KDA_COLS);
        const float* base = op.state + (size_t)b * op.sb + (size_t)h * op.sh + sl * ST_KDA_COLS;
        for (int i = lane; i < op.Dk; i += 32) {
          const float* row = base + (size_t)i * op.sk;
          if ((reinterpret_cast<uintptr_t>(row) & 15) == 0 && (cols & 3) == 0)
            l2_prefetch_bulk(row, (uint32_t)cols * 4);
        }
      }
    } else if (op.type == OP_MOE_DOWN) {
      const int n = pl->nslots * op.items_rb;
      for (int i = first_item(op.rot); i < n && ok; i += G) {
        ok = ring_acquire(R, pl, &stage, &full);
        if (!ok) break;
        Item it;
        st_describe_moe(op, pl, i, it);
        produce_item(it, stage, full, pol);
      }
      // The plan of this router may now be replaced by the consumers.
      __syncwarp();
      if (lane == 0) mbar_arrive(plan_ack);
      plan_phase ^= 1;
    }
  }
  if (!ok && lane == 0 && !pl->abort) raise_abort(P, pl, ERR_TIMEOUT);
  // Every copy this warp issued must land before the CTA may exit.
  const int outstanding = min(R.use, R.stages);
  for (int u = R.use - outstanding; u < R.use; ++u) {
    const int s = u % R.stages;
    const uint32_t ph = (u / R.stages) & 1;
    const long long t0 = now_ns();
    while (!mbar_try_wait(&R.full[s], ph))
      if (now_ns() - t0 > ST_WAIT_NS) break;
  }
}

// ---------------------------------------------------------------------------
// Consumers: projection items.
// ---------------------------------------------------------------------------
struct Split {
  int mat, rb, ks, rb_rows;  // ks: the reduction slice this warp computes
  int slot;                 // partial slot mat*RBc*KS + rb*KS + ks
  const uint8_t* wtile;
  const uint16_t* srow;
};

// rot rotates the reduction slices over the KS warps of a row block (KS is a
// power of two); every consumer passes the same value for an item.
__device__ __forceinline__ Split split_of(const Item& it, const uint8_t* stage, int rot = 0) {
  const int warp = threadIdx.x >> 5;
  Split sp;
  const int per_mat = it.RBc * it.KS;
  sp.mat = warp / per_mat;
  const int rem = warp - sp.mat * per_mat;
  sp.rb = rem / it.KS;
  sp.ks = ((rem - sp.rb * it.KS) + rot) & (it.KS - 1);
  sp.rb_rows = min(16, it.rows - sp.rb * 16);
  sp.slot = sp.mat * per_mat + sp.rb * it.KS + sp.ks;
  sp.wtile = stage + (sp.mat * it.RBc * 16 + sp.rb * 16) * it.RS;
  sp.srow = it.scale_bulk
                ? reinterpret_cast<const uint16_t*>(stage + stage_scale_offset(it) +
                                                    sp.mat * stage_scale_stride(it)) +
                      sp.rb * 16 * it.ng
                : (sp.mat ? it.s[1] : it.s[0]) + (size_t)(it.r0 + sp.rb * 16) * it.ng;
  return sp;
}

// Partial sums of this warp's row block over the kblocks [kb_lo, kb_hi) of
// the item split among its KS warps.
__device__ __forceinline__ void split_compute(const Item& it, const Split& sp,
                                              const uint8_t* wtile, int kb_lo, int kb_hi,
                                              const uint8_t* (&xrow)[1], float (&acc)[1][4]) {
  const int n = kb_hi - kb_lo;
  const int kb0 = kb_lo + n * sp.ks / it.KS, kb1 = kb_lo + n * (sp.ks + 1) / it.KS;
  if (sp.rb_rows > 0 && kb1 > kb0) {
    if (it.scale_bulk)  // scales staged with the weights: explicit shared loads
      rowblock_compute<1, true, true>(wtile, it.RS, sp.srow, it.ng, sp.rb_rows, it.K, it.gshift, kb0,
                                kb1, xrow, 1, acc);
    else
      rowblock_compute<1, false, true>(wtile, it.RS, sp.srow, it.ng, sp.rb_rows, it.K, it.gshift, kb0, kb1,
                          xrow, 1, acc);
  }
}

// Partial sums of an item's warps are handed to the reducer warps through a
// small ring of shared-memory buffers: every consumer warp stores the partial
// of its (matrix, row block, reduction slice) and arrives on the buffer's
// `done` mbarrier (count NCW); the reducer that owns the item (items
// alternate between the ST_REDUCERS reducer warps) waits for it, sums the
// slices of each row block in fixed order (so results do not depend on
// timing), writes the outputs and arrives on the buffer's `free` mbarrier
// (count 1) so it can be refilled.
struct Partials {
  float* buf;      // [ST_NB][NCW slots][16 rows][T tokens]
  uint64_t* done;  // [ST_NB] count NCW
  uint64_t* free;  // [ST_NB] count 1
  int T;
  int count;       // items published (consumers) or seen (reducers) so far
  __device__ __forceinline__ int slot() const { return count & (ST_NB - 1); }
  __device__ __forceinline__ uint32_t phase() const { return (uint32_t)(count / ST_NB) & 1u; }
  __device__ __forceinline__ const float* cur() const {
    return buf + (size_t)slot() * NCW * 16 * T;
  }
  // Reducer r owns the items whose sequence number is r modulo ST_REDUCERS.
  __device__ __forceinline__ bool mine(int r) const { return count % ST_REDUCERS == r; }
};

// Consumer side: store this warp's partial in slot `pslot` (matrix*RBc*KS +
// rb*KS + reduction slice) and arrive.  D fragment element e is row
// g + 8*(e>>1), token 2t + (e&1).
__device__ __forceinline__ void partial_publish(const StepParams& P, Partials& pa, StPlan* pl,
                                                int pslot, int ntok, const float (&acc)[1][4]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int s = pa.slot();
  // The buffer is free once its reducer has read the item published ST_NB ago.
  if (pa.count >= ST_NB && !stage_wait(&pa.free[s], pa.phase() ^ 1u, pl) && lane == 0 &&
      !pl->abort)
    raise_abort(P, pl, ERR_TIMEOUT);
  float* base = pa.buf + ((size_t)s * NCW + pslot) * 16 * pa.T;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int row = g + ((e >> 1) << 3), tok = 2 * t + (e & 1);
    if (tok < ntok) base[row * pa.T + tok] = acc[0][e];
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(&pa.done[s]);
  ++pa.count;
}

// Reducer side: wait for the next item's partials (false when aborting).
__device__ __forceinline__ bool partial_take(Partials& pa, const StPlan* pl) {
  return stage_wait(&pa.done[pa.slot()], pa.phase(), pl);
}

__device__ __forceinline__ void partial_release(Partials& pa) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&pa.free[pa.slot()]);
  ++pa.count;
}

// Sum of the KS slices of row block rb (matrix m) at (row, tok).
__device__ __forceinline__ float partial_sum(const Partials& pa, int m, int RBc, int KS, int rb,
                                             int row, int tok) {
  const float* base = pa.cur() + ((size_t)(m * RBc * KS + rb * KS) * 16 + row) * pa.T + tok;
  float v = 0.f;
  for (int k2 = 0; k2 < KS; ++k2) v += base[(size_t)k2 * 16 * pa.T];
  return v;
}

// Waits for the next ring stage.  A failed wait records the error and the
// consumers carry on with the stage as it is (its contents are then unused
// garbage), so every warp keeps the same sequence of barriers.
__device__ __forceinline__ const uint8_t* consume_stage(const StepParams& P, Ring& R,
                                                        StPlan* pl, int* slot) {
  const int s = R.slot;
  const uint32_t ph = R.phase;
  R.advance();
  *slot = s;
  if (!stage_wait(&R.full[s], ph, pl) && (threadIdx.x & 31) == 0 && !pl->abort)
    raise_abort(P, pl, ERR_TIMEOUT);
  return R.base + (size_t)s * R.stage_bytes;
}

__device__ __forceinline__ void release_stage(Ring& R, int s) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&R.empty[s]);
}

// ---------------------------------------------------------------------------
// Consumer operations.
// ---------------------------------------------------------------------------
// A consumer warp waits until the stager has copied the operation's
// descriptor, seen its dependencies complete and staged its activations.
__device__ __forceinline__ void consumer_op_wait(const StepParams& P, StPlan* pl,
                                                 uint64_t* xready, uint32_t xphase) {
  if (!stage_wait(xready, xphase, pl) && (threadIdx.x & 31) == 0 && !pl->abort)
    raise_abort(P, pl, ERR_TIMEOUT);
  if (threadIdx.x == 0) trace_mark(P, pl->cur_op, 1);
}

// ---------------------------------------------------------------------------
// Stager warp: runs one operation ahead of the consumers.  Per operation it
// waits until the consumers released the activation buffer it will use,
// copies the descriptor into shared memory, waits for the operation's
// dependencies (acquire polls of their completion counters), stages the
// activations and arrives on the buffer's `ready` mbarrier.
// ---------------------------------------------------------------------------
struct XBufs {
  uint8_t* base;   // nxb buffers of x_bytes
  int x_bytes, nxb;
  StOp* desc;      // nxb descriptor copies
  uint64_t* ready; // [nxb] count 1 (stager): dependencies complete, activations staged
  uint64_t* free;  // [nxb] count NCW (consumer warps)
  uint64_t* dsc;   // [nxb] count 1 (stager): descriptor copied
  uint64_t* dready;  // [ST_DNB] down inputs staged, count 1 (stager)
  uint64_t* dfree;   // [ST_DNB] down inputs consumed, count NCW
  int dnb, drow_bytes;
};

// Down-projection input buffer use u (the same sequence on the stager and the
// consumers): buffer u % dnb, phase (u / dnb) & 1.
struct DUse {
  int u = 0;
  __device__ __forceinline__ int buf(int dnb) const { return u % dnb; }
  __device__ __forceinline__ uint32_t phase(int dnb) const { return (uint32_t)(u / dnb) & 1u; }
};

__device__ bool stager_poll(const StepParams& P, StPlan* pl, int idx, int target) {
  const int lane = threadIdx.x & 31;
  int ok = 1;
  if (lane == 0 && target > 0) {
    const long long t0 = now_ns();
    int spins = 0;
    while (ld_acquire(&P.sync[idx]) < target) {
      __nanosleep(32);
      if (((++spins) & 15) == 0) {
        if (*((volatile int*)&P.sync[P.abort_idx]) != 0 || pl->abort) {
          pl->abort = 1;
          ok = 0;
          break;
        }
        if (now_ns() - t0 > ST_WAIT_NS) {
          raise_abort(P, pl, ERR_TIMEOUT);
          ok = 0;
          break;
        }
      }
    }
  }
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

__device__ bool route_one(const StepParams& P, const StOp& up, StPlan* pl);

__device__ void stager_main(const StepParams& P, StPlan* pl, const XBufs& X, uint64_t* plan_bar,
                            uint64_t* plan_ack) {
  const int lane = threadIdx.x & 31;
  const int G = gridDim.x;
  int b = 0;
  uint32_t ph = 0;
  uint32_t plan_phase = 0;
  uint32_t route_round = 0;
  DUse du;
  int o = 0;
  for (; o < P.nops; ++o) {
    if (o >= X.nxb && !stage_wait(&X.free[b], ph ^ 1u, pl)) break;
    StOp* dst = X.desc + b;
    const int* src = reinterpret_cast<const int*>(P.ops + o);
    for (int w = lane; w < (int)(sizeof(StOp) / sizeof(int)); w += 32)
      reinterpret_cast<int*>(dst)[w] = src[w];
    __syncwarp();
    const StOp& op = *dst;
    if (lane == 0) mbar_arrive(&X.dsc[b]);
    bool ok = true;
    for (int d = 0; d < op.ndeps && ok; ++d) {
      // The consumers wait for the items of a combine source and poll the
      // words of a tagged source.
      if (op.dep[d] == op.comb_src || op.dep[d] == op.tag_src) continue;
      const StOp& dop = P.ops[op.dep[d]];
      ok = stager_poll(P, pl, dop.done, dop.target);
    }
    if (!ok) break;
    uint8_t* xs = X.base + (size_t)b * X.x_bytes;
    if (op.cstage) {
      // Staged by the consumers, which are waiting for this input anyway.
    } else if (op.type == OP_DENSE) {
      for (int p = 0; p < op.nprob; ++p) {
        const StDense& D = op.p[p];
        if (D.nchunk > 1) continue;  // staged chunk by chunk by the consumers
        bool dup = false;
        for (int q = 0; q < p; ++q) dup |= (op.p[q].x_off == D.x_off);
        if (dup) continue;
        const int ts = token_stride(D.K);
        for (int m = 0; m < op.T; ++m)
          stage_row_cg<1>(xs + D.x_off + m * ts, D.x + (size_t)m * D.xs, D.K, lane, 32);
      }
    } else if (op.type == OP_ROUTER) {
      const int words = op.K >> 3;
      for (int m = 0; m < op.T; ++m) {
        const uint4* s4 = reinterpret_cast<const uint4*>(op.rx + (size_t)m * op.rxs);
        uint4* d4 = reinterpret_cast<uint4*>(xs + (size_t)m * op.K * 2);
        for (int w = lane; w < words; w += 32) d4[w] = __ldcg(s4 + w);
      }
    } else if (op.type == OP_MOE_UP) {
      const int ts = token_stride(op.K);
      for (int m = 0; m < op.T; ++m)
        stage_row_cg<1>(xs + m * ts, op.mx + (size_t)m * op.mxs, op.K, lane, 32);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&X.ready[b]);
    if (op.type == OP_MOE_UP && op.T == 1) {
      // One token: this warp builds the routing and the plan while the
      // consumers compute the shared expert, once the producer and the
      // reducers are done with the previous plan.
      if (route_round > 0 && !stage_wait(plan_ack, (route_round - 1) & 1u, pl)) break;
      ++route_round;
      if (!route_one(P, op, pl)) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(plan_bar);
    }
    if (op.type == OP_MOE_DOWN) {
      // Inputs of each down item of this CTA, in item order, as soon as the
      // gate/up of its slot is complete: the activated rows of the slot's
      // assignments, into the next of dnb buffers inside this operation's
      // activation buffer.
      if (!stage_wait(plan_bar, plan_phase, pl)) break;
      plan_phase ^= 1u;
      const int n = pl->nslots * op.items_rb;
      const int ts = token_stride(op.K);
      for (int i = first_item(op.rot); i < n && ok; i += G, ++du.u) {
        const int j = du.buf(X.dnb);
        if (du.u >= X.dnb && !stage_wait(&X.dfree[j], du.phase(X.dnb) ^ 1u, pl)) {
          ok = false;
          break;
        }
        const int slot = i / op.items_rb;
        ok = stager_poll(P, pl, op.slot_cnt + slot, op.up_rb);
        if (!ok) break;
        const int a0 = pl->slot_start[slot], cnt = pl->slot_start[slot + 1] - a0;
        uint8_t* dst = xs + (size_t)j * X.drow_bytes;
        for (int m = 0; m < cnt; ++m)
          stage_row_cg<4>(dst + m * ts, op.mx + (size_t)pl->assign[a0 + m] * op.mxs, op.K, lane,
                          32);
        __syncwarp();
        if (lane == 0) mbar_arrive(&X.dready[j]);
      }
      if (!ok) break;
    }
    if (++b == X.nxb) {
      b = 0;
      ph ^= 1u;
    }
  }
  // A wait that gave up ends the launch (the consumers' waits are bounded too).
  if (o < P.nops && lane == 0 && !pl->abort) raise_abort(P, pl, ERR_TIMEOUT);
}

// Row of the combined output of a down operation (routes of one token at
// wrows + r*N, r < R; weights rw) computed from the per-route outputs and
// staged in the B-fragment layout: what staging the combine's output row
// would give, without waiting for the combine.  Each lane combines one
// 8-byte half of a 16-byte word (few registers: this runs inside the
// consumer loop) and trades a pair of values with its neighbour lane, which
// holds the other half.  first/step: a warp-aligned thread index and stride.
// TAGGED: the per-route outputs are read from their tagged copy (wtags, same
// layout in 32-bit words), polling until every word carries `tag`.
template <bool TAGGED>
__device__ __forceinline__ void stage_combined(uint8_t* xs_row, const uint16_t* wrows,
                                               const uint32_t* wtags, uint32_t tag,
                                               const StepParams& P, StPlan* pl,
                                               const float* rw, int top_k, int R, int N,
                                               int first, int step) {
  const int NC = N >> 5;
  const int halves = N >> 2;
  for (int h = first; h - (first & 31) < halves; h += step) {
    const bool valid = h < halves;
    const int part = h & 1, w = h >> 1;
    uint2 v[ST_MAX_TOPK];
    uint2 sv;
    if constexpr (TAGGED) {
      const uint32_t f = tag << 16;
      uint4 t[ST_MAX_TOPK], ts;
      const long long t0 = now_ns();
      for (int spins = 0;; ++spins) {
        bool ok = true;
#pragma unroll
        for (int r = 0; r < ST_MAX_TOPK; ++r) {
          t[r] = (valid && r < top_k) ? ld_tags4(wtags + (size_t)r * N + 4 * h)
                                      : make_uint4(f, f, f, f);
          ok &= tags_ok4(t[r], tag);
        }
        ts = valid ? ld_tags4(wtags + (size_t)(R - 1) * N + 4 * h) : make_uint4(f, f, f, f);
        ok &= tags_ok4(ts, tag);
        if (ok) break;
        __nanosleep(32);
        if ((spins & 15) == 15) {
          if (*((volatile int*)&P.sync[P.abort_idx]) != 0 || *((volatile int*)&pl->abort) != 0) {
            pl->abort = 1;
            break;
          }
          if (now_ns() - t0 > ST_WAIT_NS) {
            raise_abort(P, pl, ERR_TIMEOUT);
            break;
          }
        }
      }
#pragma unroll
      for (int r = 0; r < ST_MAX_TOPK; ++r)
        v[r] = make_uint2(prmt(t[r].x, t[r].y, 0x5410), prmt(t[r].z, t[r].w, 0x5410));
      sv = make_uint2(prmt(ts.x, ts.y, 0x5410), prmt(ts.z, ts.w, 0x5410));
    } else {
#pragma unroll
      for (int r = 0; r < ST_MAX_TOPK; ++r)
        v[r] = (valid && r < top_k)
                   ? __ldcg(reinterpret_cast<const uint2*>(wrows + (size_t)r * N) + h)
                   : make_uint2(0u, 0u);
      sv = valid ? __ldcg(reinterpret_cast<const uint2*>(wrows + (size_t)(R - 1) * N) + h)
                 : make_uint2(0u, 0u);
    }
    uint32_t c[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      uint16_t lo[ST_MAX_TOPK], hi[ST_MAX_TOPK];
#pragma unroll
      for (int r = 0; r < ST_MAX_TOPK; ++r) {
        const uint32_t x = q ? v[r].y : v[r].x;
        lo[r] = (uint16_t)(x & 0xffffu);
        hi[r] = (uint16_t)(x >> 16);
      }
      const uint32_t sx = q ? sv.y : sv.x;
      c[q] = (uint32_t)combine_value(lo, rw, top_k, (uint16_t)(sx & 0xffffu)) |
             ((uint32_t)combine_value(hi, rw, top_k, (uint16_t)(sx >> 16)) << 16);
    }
    // Half 0 holds elements 0-3 of the word, half 1 elements 4-7; the pair
    // order (0,4),(1,5) | (2,6),(3,7) needs one value of the other half.
    const uint32_t got = __shfl_xor_sync(0xffffffffu, part ? c[0] : c[1], 1);
    if (valid) {
      const uint32_t a = part ? got : c[0], b2 = part ? c[1] : got;
      *reinterpret_cast<uint2*>(xs_row + ((w & 3) * NC + (w >> 2)) * 16 + part * 8) =
          make_uint2(prmt(a, b2, 0x5410), prmt(a, b2, 0x7632));
    }
  }
}

// Activations of a dense or router operation whose input comes from the
// operation just before it: staged by all consumer threads (one L2 round
// trip) once the stager has seen the input complete.
__device__ void consumer_stage(const StepParams& P, StPlan* pl, const StOp& op, uint8_t* xs) {
  const uint32_t tag = op.tag_src >= 0 ? op_tag(pl, P.nops, op.tag_src) : 0u;
  if (op.type == OP_DENSE) {
    int comb_off = -1, comb_k = 0;
    for (int p = 0; p < op.nprob; ++p) {
      const StDense& D = op.p[p];
      if (D.nchunk > 1) continue;  // staged chunk by chunk
      bool dup = false;
      for (int q = 0; q < p; ++q) dup |= (op.p[q].x_off == D.x_off);
      if (dup) continue;
      if (D.xcomb) {
        comb_off = D.x_off;
        comb_k = D.K;
        continue;
      }
      const int ts = token_stride(D.K);
      if (D.xtag) {
        const int NC = D.K >> 5, words = D.K >> 3;
        for (int m = 0; m < op.T; ++m) {
          uint8_t* const row = xs + D.x_off + m * ts;
          for (int w = threadIdx.x; w < words; w += NCT)
            *reinterpret_cast<uint4*>(row + ((w & 3) * NC + (w >> 2)) * 16) =
                permute_pairs(poll_tagged8(P, pl, D.xtag + (size_t)m * D.K + 8 * w, tag));
        }
      } else {
        for (int m = 0; m < op.T; ++m)
          stage_row_cg(xs + D.x_off + m * ts, D.x + (size_t)m * D.xs, D.K, threadIdx.x, NCT);
      }
    }
    if (comb_off >= 0) {
      const StOp& dop = P.ops[op.comb_src];
      const int R = dop.R, N = dop.N;
      const int ts = token_stride(comb_k);
      if (dop.wtag) {
        // Tagged per-route outputs: polled word by word.
        for (int m = 0; m < op.T; ++m)
          stage_combined<true>(xs + comb_off + m * ts, nullptr, dop.wtag + (size_t)m * R * N,
                               tag, P, pl, pl->route_w + m * (R - 1), R - 1, R, N,
                               threadIdx.x, NCT);
      } else {
        // The down operation's per-route outputs are complete once all of its
        // items are (the plan in shared memory is still this layer's).
        consumers_wait(P, pl, dop.items_done, pl->nslots * dop.items_rb);
        for (int m = 0; m < op.T; ++m)
          stage_combined<false>(xs + comb_off + m * ts, dop.wsy + (size_t)m * R * N, nullptr, 0u,
                                P, pl, pl->route_w + m * (R - 1), R - 1, R, N, threadIdx.x,
                                NCT);
      }
    }
  } else {
    const int words = op.K >> 3;
    for (int m = 0; m < op.T; ++m) {
      uint4* d4 = reinterpret_cast<uint4*>(xs + (size_t)m * op.K * 2);
      if (op.rxtag) {
        for (int w = threadIdx.x; w < words; w += NCT)
          d4[w] = poll_tagged8(P, pl, op.rxtag + (size_t)m * op.K + 8 * w, tag);
      } else {
        const uint4* s4 = reinterpret_cast<const uint4*>(op.rx + (size_t)m * op.rxs);
        for (int w = threadIdx.x; w < words; w += NCT) d4[w] = __ldcg(s4 + w);
      }
    }
  }
  named_barrier(CBAR, NCT);
}

// A dense operation of one problem whose rows are split into reduction
// chunks (one stage each): the consumers stage the activations chunk by chunk.
__device__ void run_dense_chunked(const StepParams& P, const StOp& op, StPlan* pl, Ring& R,
                                  uint8_t* xs, Partials& pa) {
  const int g = (threadIdx.x & 31) >> 2;
  const int G = gridDim.x;
  const StDense& D = op.p[0];
  const int n = D.items;
  for (int i = first_item(op.rot); i < n; i += G) {
    Item it;
    st_describe_dense(op, i, it);
    float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
    Split sp;
    // Reduction chunks of kc columns: each stage holds kc/2 bytes of every
    // row; the activations of the chunk are staged in a chunk-local layout
    // and the chunk is contracted as a problem of width kc.
    const int kc = D.K / D.nchunk;
    const int tsc = token_stride(kc);
    const int gpc = kc >> (5 + D.gshift);  // scale groups per chunk
    Item ic = it;
    ic.K = kc;
    const uint8_t* xrow[1] = {xs + min(g, op.T - 1) * tsc};
    const int crot = (i / G) & (D.KS - 1);
    for (int ci = 0; ci < D.nchunk; ++ci) {
      named_barrier(CBAR, NCT);
      for (int m = 0; m < op.T; ++m)
        stage_row_cg(xs + m * tsc, D.x + (size_t)m * D.xs + (size_t)ci * kc, kc, threadIdx.x,
                     NCT);
      named_barrier(CBAR, NCT);
      int st;
      const uint8_t* stage = consume_stage(P, R, pl, &st);
      sp = split_of(ic, stage, crot);
      sp.srow += ci * gpc;
      split_compute(ic, sp, sp.wtile, 0, (kc + 127) >> 7, xrow, acc);
      release_stage(R, st);
    }
    partial_publish(P, pa, pl, sp.slot, op.T, acc);
  }
}

// xready/xphase: the operation's inputs; the per-warp setup of the first
// item is done before waiting for them.
__device__ void run_dense(const StepParams& P, const StOp& op, StPlan* pl, Ring& R, uint8_t* xs,
                          Partials& pa, uint64_t* xready, uint32_t xphase) {
  const int lane = threadIdx.x & 31, g = lane >> 2;
  const int G = gridDim.x;
  const int warp = threadIdx.x >> 5;
  const int nprob = op.nprob;
  const int n = op.p[nprob - 1].item_begin + op.p[nprob - 1].items;
  if (op.p[0].nchunk > 1) {
    consumer_op_wait(P, pl, xready, xphase);
    if (op.cstage) consumer_stage(P, pl, op, xs);
    run_dense_chunked(P, op, pl, R, xs, pa);
    return;
  }
  // This warp's part of an item of the current problem (reloaded when the
  // item sequence i = first, first + G, ... enters another problem).  KS and
  // RBc are powers of two.
  int p = -1, pend = 0, ib = 0;
  int K = 0, N = 0, gshift = 0, ng = 0, KB = 0, KS = 1, kslog = 0, item_rows = 0;
  int rb = 0, ks = 0, pslot_base = 0, wt_off = 0, sc_off = 0;
  bool base_ok = false;
  const uint16_t* sglob = nullptr;
  const uint8_t* xrow0 = xs;
  int rot = 0;  // reduction slice of this warp = (ks + rot) % KS, rot advancing per item
  bool waited = false;
  for (int i = first_item(op.rot);; i += G) {
    if (i < n && i >= pend) {
      do {
        ++p;
        pend = op.p[p].item_begin + op.p[p].items;
      } while (i >= pend);
      const StDense& D = op.p[p];
      ib = D.item_begin;
      K = D.K;
      N = D.N;
      gshift = D.gshift;
      ng = K >> (5 + gshift);
      KB = K >> 7;
      KS = D.KS;
      kslog = __ffs(KS) - 1;
      item_rows = D.RBc * 16;
      const int mats = D.mats;
      const int pmlog = kslog + __ffs(D.RBc) - 1;  // log2(RBc * KS)
      const int mat = warp >> pmlog;
      const int rem = warp - (mat << pmlog);
      rb = rem >> kslog;
      ks = rem & (KS - 1);
      pslot_base = (mat << pmlog) + (rb << kslog);
      const int RS = K >> 1;
      wt_off = (mat * item_rows + rb * 16) * RS;
      sc_off = mats * item_rows * RS + mat * ((item_rows * ng * 2 + 15) / 16 * 16) +
               rb * 16 * ng * 2;
      sglob = mat ? D.s3 : D.s;
      xrow0 = xs + D.x_off + min(g, op.T - 1) * token_stride(K);
      base_ok = (reinterpret_cast<uintptr_t>(D.s) % 16 == 0) &&
                (mats == 1 || reinterpret_cast<uintptr_t>(D.s3) % 16 == 0);
    }
    if (!waited) {
      // Inputs: wait for them (and stage them) once the first item's setup
      // is done; every consumer thread passes here, with or without items.
      consumer_op_wait(P, pl, xready, xphase);
      if (op.cstage) consumer_stage(P, pl, op, xs);
      waited = true;
    }
    if (i >= n) break;
    const int r0 = (i - ib) * item_rows;
    const int rows = min(item_rows, N - r0);
    const int rb_rows = min(16, rows - rb * 16);
    const bool bulk = base_ok && ((rows * ng * 2) % 16 == 0);
    // Slices of unequal length rotate over the warps from item to item, so
    // the ring's slack evens the load out.
    const int ksr = (ks + rot) & (KS - 1);
    rot = (rot + 1) & (KS - 1);
    const int kb0 = (KB * ksr) >> kslog, kb1 = (KB * (ksr + 1)) >> kslog;
    const uint8_t* xrow[1] = {xrow0};
    float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
    int st;
    const uint8_t* stage = consume_stage(P, R, pl, &st);
    if (rb_rows > 0 && kb1 > kb0) {
      if (bulk)
        rowblock_compute<1, true, true>(stage + wt_off, K >> 1,
                                  reinterpret_cast<const uint16_t*>(stage + sc_off), ng,
                                  rb_rows, K, gshift, kb0, kb1, xrow, 1, acc);
      else
        rowblock_compute<1, false, true>(stage + wt_off, K >> 1, sglob + (size_t)(r0 + rb * 16) * ng, ng,
                            rb_rows, K, gshift, kb0, kb1, xrow, 1, acc);
    }
    release_stage(R, st);
    partial_publish(P, pa, pl, pslot_base + ksr, op.T, acc);
  }
}

__device__ void run_router(const StepParams& P, const StOp& op, StPlan* pl, Ring& R,
                           uint8_t* xs) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;
  // Descriptor fields in registers: the loops below must not re-read them.
  const int K = op.K, words = K >> 3, T = op.T, E = op.E, items = op.items;
  const float* rbias = op.rbias;
  // Router words of this launch and of the next (cleared here for it).
  unsigned long long* rwords = op.rwords + (size_t)pl->parity * T * E;
  unsigned long long* next_rwords = op.rwords + (size_t)(pl->parity ^ 1) * T * E;
  int* done = &P.sync[op.done];
  const uint32_t xs_s = smem_addr(xs);
  // Warp j < 8 computes expert i*8 + j over the whole row in the order of the
  // router kernel (lane-strided 16-byte words, router_word_fma, a xor
  // butterfly), so logits equal kb_router_topk's bit for bit; warps 8..15
  // only release the stages.
  int experts = 0;
  for (int i = first_item(op.rot); i < items; i += G) {
    const int e = i * ST_RT_EXPERTS + warp;
    // The bias is read from memory; its load goes out before the stage wait
    // and the dot product, which hide its latency.
    const float be = (rbias && warp < ST_RT_EXPERTS && e < E) ? __ldg(rbias + e) : 0.f;
    int s;
    const uint8_t* stage = consume_stage(P, R, pl, &s);
    if (warp < ST_RT_EXPERTS && e < E && T == 1) {
      // One token: a branch-free loop and a four-register accumulator (the
      // general path below keeps eight tokens' accumulators live).
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      const uint4* wp = reinterpret_cast<const uint4*>(stage + warp * K * 2) + lane;
      const uint4* hp = reinterpret_cast<const uint4*>(xs) + lane;
#pragma unroll 3
      for (int w = lane; w < words; w += 32, wp += 32, hp += 32) router_word_fma(*wp, *hp, acc);
      float v = router_lane_sum(acc);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      // Lane 0 publishes the word: the choice key of sigmoid + bias (plus
      // one, so that zero means "not written") and the sigmoid score.
      if (lane == 0) {
        const float sc = 1.0f / (1.0f + expf(-v));
        st_relaxed_u64(rwords + e, router_word(choice_key(sc + be), sc));
        next_rwords[e] = 0ull;
      }
    } else if (warp < ST_RT_EXPERTS && e < E) {
      float acc[ST_MAX_T][4];
#pragma unroll
      for (int m = 0; m < ST_MAX_T; ++m)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[m][j] = 0.f;
      uint32_t wa = smem_addr(stage) + (uint32_t)(warp * K * 2 + lane * 16);
      const uint32_t ha = xs_s + (uint32_t)(lane * 16);
      for (int w = lane; w < words; w += 32, wa += 512) {
        uint4 wv;
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(wv.x), "=r"(wv.y), "=r"(wv.z), "=r"(wv.w)
                     : "r"(wa));
#pragma unroll
        for (int m = 0; m < ST_MAX_T; ++m) {
          if (m < T) {
            uint4 hv;
            asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(hv.x), "=r"(hv.y), "=r"(hv.z), "=r"(hv.w)
                         : "r"(ha + (uint32_t)(m * K * 2 + (w - lane) * 16)));
            router_word_fma(wv, hv, acc[m]);
          }
        }
      }
      // Lane m publishes token m's word.
#pragma unroll
      for (int m = 0; m < ST_MAX_T; ++m) {
        if (m < T) {
          float v = router_lane_sum(acc[m]);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
          if (lane == m) {
            const float sc = 1.0f / (1.0f + expf(-v));
            st_relaxed_u64(rwords + (size_t)m * E + e, router_word(choice_key(sc + be), sc));
            next_rwords[(size_t)m * E + e] = 0ull;
          }
        }
      }
    }
    release_stage(R, s);
    experts += min(ST_RT_EXPERTS, E - i * ST_RT_EXPERTS);
  }
  named_barrier(CBAR, NCT);
  if (threadIdx.x == 0 && experts > 0) red_release(done, experts);
}

// Waits (bounded) until a router word is written and returns it; zero when
// the wait gave up (then the launch is aborting).
__device__ unsigned long long poll_router_word(const StepParams& P, StPlan* pl,
                                               const unsigned long long* word) {
  unsigned long long w = ld_relaxed_u64(word);
  if ((w >> 32) != 0ull) return w;
  const long long t0 = now_ns();
  for (int spins = 1;; ++spins) {
    __nanosleep(32);
    w = ld_relaxed_u64(word);
    if ((w >> 32) != 0ull) return w;
    if ((spins & 15) == 0) {
      if (*((volatile int*)&P.sync[P.abort_idx]) != 0 || *((volatile int*)&pl->abort) != 0) {
        pl->abort = 1;
        return 0ull;
      }
      if (now_ns() - t0 > ST_WAIT_NS) {
        raise_abort(P, pl, ERR_TIMEOUT);
        return 0ull;
      }
    }
  }
}

// (key, expert) a precedes (key, expert) b in choice order: larger key, then
// lower expert index.
__device__ __forceinline__ bool choice_before(uint32_t ka, int ea, uint32_t kb, int eb) {
  return ka > kb || (ka == kb && ea < eb);
}

// Routing weight of a pick: unbiased sigmoid score renormalised over the
// picks in pick order, scaled (lane r < top_k holds pick r's score).
__device__ __forceinline__ float route_weight(const StOp& rop, float score, int lane) {
  const int top_k = rop.top_k;
  const float sc = lane < top_k ? score : 0.f;
  float v[ST_MAX_TOPK];
#pragma unroll
  for (int r = 0; r < ST_MAX_TOPK; ++r) v[r] = __shfl_sync(0xffffffffu, sc, r);
  float wsum = 0.f;
#pragma unroll
  for (int r = 0; r < ST_MAX_TOPK; ++r)
    if (r < top_k) wsum += v[r];
  float wv = sc;
  if (rop.renorm && top_k > 1) wv = wv / (wsum + 1e-20f);
  return wv * rop.scaling;
}

// Routing and plan of a single token by one warp (the stager), the same as
// build_routing computes them.  Lane l holds experts l + 32 j (j < 8).  The
// lane bests ranked among themselves give a threshold H (the top_k-th best
// of the lane bests): every pick is >= H in choice order, and the candidates
// >= H (at most 8 * top_k, from top_k lanes) are ranked against each other
// in shared memory.  Returns false when a word wait gave up.
__device__ bool route_one(const StepParams& P, const StOp& up, StPlan* pl) {
  const int lane = threadIdx.x & 31;
  const StOp& rop = P.ops[up.router_op];
  const int R = up.R, top_k = rop.top_k, E = rop.E;
  const unsigned long long* words = rop.rwords + (size_t)pl->parity * E;
  // All eight words of a lane in flight at once, re-read together until all
  // are written (bounded).
  unsigned long long wd[8];
  uint32_t missing = 0u;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    if (lane + 32 * j < E) missing |= 1u << j;
  bool ok = true;
  const long long t0 = now_ns();
  for (int spins = 0; missing != 0u; ++spins) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if ((missing >> j) & 1u) wd[j] = ld_relaxed_u64(words + lane + 32 * j);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (((missing >> j) & 1u) && (wd[j] >> 32) != 0ull) missing &= ~(1u << j);
    if (missing == 0u) break;
    __nanosleep(32);
    if ((spins & 15) == 15) {
      if (*((volatile int*)&P.sync[P.abort_idx]) != 0 || *((volatile int*)&pl->abort) != 0) {
        pl->abort = 1;
        ok = false;
        break;
      }
      if (now_ns() - t0 > ST_WAIT_NS) {
        raise_abort(P, pl, ERR_TIMEOUT);
        ok = false;
        break;
      }
    }
  }
  if (!__all_sync(0xffffffffu, ok)) return false;
  // Choice order as one 64-bit value: key << 32 | ~expert (absent: 0).
  unsigned long long c[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int e = lane + 32 * j;
    c[j] = e < E ? ((wd[j] >> 32) - 1ull) << 32 | (uint32_t)~e : 0ull;
  }
  unsigned long long b = c[0];
#pragma unroll
  for (int j = 1; j < 8; ++j) b = c[j] > b ? c[j] : b;
  int rank = 0;
#pragma unroll
  for (int sl = 0; sl < 32; ++sl) rank += __shfl_sync(0xffffffffu, b, sl) > b ? 1 : 0;
  const unsigned at = __ballot_sync(0xffffffffu, rank == top_k - 1);
  const unsigned long long H = __shfl_sync(0xffffffffu, b, __ffs(at) - 1);
  int cnt = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) cnt += c[j] >= H ? 1 : 0;
  int incl = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  const int total = __shfl_sync(0xffffffffu, incl, 31);
  int w = incl - cnt;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (c[j] >= H) {
      pl->cand_k[0][w] = (uint32_t)(c[j] >> 32);
      pl->cand_e[0][w] = lane + 32 * j;
      pl->cand_l[0][w] = __uint_as_float((uint32_t)wd[j]);
      ++w;
    }
  }
  __syncwarp();
  for (int t = lane; t < total; t += 32) {
    const uint32_t kt = pl->cand_k[0][t];
    const int et = pl->cand_e[0][t];
    int r = 0;
#pragma unroll 1
    for (int u = 0; u < total; ++u) r += choice_before(pl->cand_k[0][u], pl->cand_e[0][u], kt, et);
    if (r < top_k) {
      pl->pick_e[0][r] = et;
      pl->pick_l[0][r] = pl->cand_l[0][t];
    }
  }
  __syncwarp();
  const int my_e = lane < top_k ? min(max(pl->pick_e[0][lane], 0), E - 1) : 0;
  const float my_l = lane < top_k ? pl->pick_l[0][lane] : 0.f;
  const float wv = route_weight(rop, my_l, lane);
  if (lane < top_k) {
    pl->route_e[lane] = my_e;
    pl->route_w[lane] = wv;
    pl->slot_expert[1 + lane] = my_e;
    pl->slot_start[1 + lane] = 1 + lane;
    pl->assign[1 + lane] = lane;
    if (blockIdx.x == 0) {
      rop.idx_out[lane] = my_e;
      rop.w_out[lane] = wv;
    }
  }
  if (lane == top_k) pl->slot_start[1 + top_k] = 1 + top_k;
  if (lane == 0) {
    pl->route_e[R - 1] = E;
    pl->assign[0] = R - 1;
    pl->slot_expert[0] = E;
    pl->slot_start[0] = 0;
    pl->nslots = 1 + top_k;
    if (blockIdx.x == 0) rop.idx_out[top_k] = E;
  }
  return true;
}

// Top-k of every token and the expert plan (warp 0) for two or more tokens
// (route_one builds a single token's), in every CTA from the same router
// words, so every CTA holds the same plan.  The words are read as
// soon as the router has written them (no completion counter between).  Two
// tokens at a time, 256 consumer threads per token, one expert each: every
// warp ranks its 32 experts with shuffles and keeps its best 8 (a superset
// of the token's top-k among them), then 64 threads rank those 64
// candidates.  The picks come out in choice order (largest choice key, ties
// to the lower index), the order of the per-operation router.  Slot 0 is the
// shared expert (bank slot E, every token, route R-1); routed experts follow
// in order of first use (token-major, then route order).  Indices are always
// in [0, E), whatever the words hold.
__device__ void build_routing(const StepParams& P, const StOp& up, StPlan* pl,
                              uint64_t* plan_bar) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const StOp& rop = P.ops[up.router_op];
  const int T = up.T, R = up.R, top_k = rop.top_k, E = rop.E;
  const unsigned long long* words = rop.rwords + (size_t)pl->parity * T * E;
  const int half = threadIdx.x >> 8;        // token t0 + half
  const int e = threadIdx.x & 255;          // expert of this thread
  const int w8 = warp & 7;                  // warp within the token's eight
  for (int t0 = 0; t0 < T; t0 += 2) {
    const int t = t0 + half;
    const bool valid = t < T && e < E;
    uint32_t key = 0u;
    float lg = 0.f;
    if (valid) {
      const unsigned long long w = poll_router_word(P, pl, words + (size_t)t * E + e);
      key = (uint32_t)(w >> 32) - 1u;
      lg = __uint_as_float((uint32_t)w);
    }
    if (t0 == 0 && threadIdx.x == 0) trace_mark(P, pl->cur_op, 7);
    // Rank among the warp's valid experts (lane order = index order).
    int rank = 0;
#pragma unroll
    for (int sl = 0; sl < 32; ++sl) {
      const uint32_t ks = __shfl_sync(0xffffffffu, key, sl);
      const bool vs = __shfl_sync(0xffffffffu, valid, sl);
      rank += (vs && (ks > key || (ks == key && sl < lane))) ? 1 : 0;
    }
    if (lane < 8) pl->cand_e[half][w8 * 8 + lane] = 0x7fffffff;  // empty candidate slot
    __syncwarp();
    if (valid && rank < 8) {
      pl->cand_k[half][w8 * 8 + rank] = key;
      pl->cand_e[half][w8 * 8 + rank] = e;
      pl->cand_l[half][w8 * 8 + rank] = lg;
    }
    named_barrier(CBAR, NCT);
    // Rank of candidate e >> 2 among the 64, four threads (a quarter of the
    // candidates each) per candidate.
    {
      const int c = e >> 2, q = e & 3;
      const int ec = pl->cand_e[half][c];
      const uint32_t kc = pl->cand_k[half][c];
      int r2 = 0;
#pragma unroll 4
      for (int j = q * 16; j < q * 16 + 16; ++j) {
        const int ej = pl->cand_e[half][j];
        r2 += (ej < E && choice_before(pl->cand_k[half][j], ej, kc, ec)) ? 1 : 0;
      }
      r2 += __shfl_xor_sync(0xffffffffu, r2, 1);
      r2 += __shfl_xor_sync(0xffffffffu, r2, 2);
      if (q == 0 && t < T && ec < E && r2 < top_k) {
        pl->pick_e[half][r2] = ec;
        pl->pick_l[half][r2] = pl->cand_l[half][c];
      }
    }
    named_barrier(CBAR, NCT);
    // Weights of token t0 + warp (warps 0 and 1): unbiased sigmoid scores,
    // renormalised in pick order, scaled.
    if (warp < 2 && t0 + warp < T) {
      const int tt = t0 + warp;
      const int my_idx = lane < top_k ? min(max(pl->pick_e[warp][lane], 0), E - 1) : 0;
      const float wv = route_weight(rop, lane < top_k ? pl->pick_l[warp][lane] : 0.f, lane);
      if (lane < top_k) {
        pl->route_e[tt * R + lane] = my_idx;
        pl->route_w[tt * top_k + lane] = wv;
        if (blockIdx.x == 0) {
          rop.idx_out[(size_t)tt * (top_k + 1) + lane] = my_idx;
          rop.w_out[(size_t)tt * top_k + lane] = wv;
        }
      }
      if (lane == 0) {
        pl->route_e[tt * R + R - 1] = E;
        if (blockIdx.x == 0) rop.idx_out[(size_t)tt * (top_k + 1) + top_k] = E;
      }
    }
  }
  named_barrier(CBAR, NCT);  // the plan below reads every token's routes
  if (warp == 0) {
    if (lane < T) pl->assign[lane] = lane * R + R - 1;
    if (lane == 0) {
      pl->slot_expert[0] = E;
      pl->slot_start[0] = 0;
    }
    const int n = T * top_k;
    int nslot = 1;
    for (int base = 0; base < n; base += 32) {
      const int a = base + lane;
      const bool valid = a < n;
      const int e = valid ? pl->route_e[(a / top_k) * R + (a % top_k)] : -1 - lane;
      const unsigned peers = __match_any_sync(0xffffffffu, e);
      const int leader = __ffs(peers) - 1;
      const int known = valid ? pl->slot_of[e] : 0;
      __syncwarp();
      const bool fresh = valid && known < 0 && lane == leader;
      const unsigned nb = __ballot_sync(0xffffffffu, fresh);
      if (fresh) {
        const int sl = nslot + __popc(nb & ((1u << lane) - 1u));
        pl->slot_of[e] = sl;
        pl->slot_expert[sl] = e;
      }
      nslot += __popc(nb);
      __syncwarp();
      if (valid) pl->slot_id[a] = pl->slot_of[e];
      __syncwarp();
    }
    // Counts per routed slot, exclusive prefix after the T shared assignments.
    int running = T;
    for (int sb = 1; sb < nslot; sb += 32) {
      const int sl = sb + lane;
      int c = 0;
      if (sl < nslot)
        for (int a = 0; a < n; ++a) c += (pl->slot_id[a] == sl);
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      if (sl < nslot) pl->slot_start[sl] = running + incl - c;
      running += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      pl->slot_start[nslot] = running;
      pl->nslots = nslot;
    }
    __syncwarp();
    // Stable scatter of the routed assignments.
    for (int a = lane; a < n; a += 32) {
      const int sl = pl->slot_id[a];
      int rank = 0;
      for (int b = 0; b < a; ++b) rank += (pl->slot_id[b] == sl);
      pl->assign[pl->slot_start[sl] + rank] = (a / top_k) * R + (a % top_k);
    }
    __syncwarp();
    for (int sl = 1 + lane; sl < nslot; sl += 32) pl->slot_of[pl->slot_expert[sl]] = -1;
    __syncwarp();
    if (lane == 0) mbar_arrive(plan_bar);
  }
  if (threadIdx.x == 0) trace_mark(P, pl->cur_op, 2);
  named_barrier(CBAR, NCT);
}

// Item-invariant part of an expert operation's items for one consumer warp
// (read once per operation; per item only the slot, row group and token rows
// change).  KS and RBc are powers of two.
struct ExpertWarp {
  int K, N, gshift, ng, KB, KS, kslog, item_rows, items_rb;
  int pslot_base;      // partial slot of this warp's (matrix, row block), + slice
  int rb;              // row block within the item
  int ks;              // reduction slice before rotation
  int wt_off, sc_off;  // stage offsets of this warp's weight tile and scale rows
  int64_t sse;         // scale elements per expert
  const uint16_t* s;   // scales of this warp's matrix, expert 0
  int sbulk;
};

__device__ __forceinline__ ExpertWarp expert_warp(const StOp& op) {
  const int warp = threadIdx.x >> 5;
  ExpertWarp w;
  w.K = op.K;
  w.N = op.N;
  w.gshift = op.gshift;
  w.ng = op.K >> (5 + op.gshift);
  w.KB = (op.K + 127) >> 7;
  w.KS = op.KS;
  w.kslog = __ffs(op.KS) - 1;
  w.item_rows = op.RBc * 16;
  w.items_rb = op.items_rb;
  const int per_mat = op.RBc * op.KS;
  const int mat = warp / per_mat;
  const int rem = warp - mat * per_mat;
  w.rb = rem >> w.kslog;
  w.ks = rem & (op.KS - 1);
  w.pslot_base = mat * per_mat + w.rb * op.KS;
  const int RS = op.K >> 1;
  const int mats = (op.type == OP_MOE_UP) ? 2 : 1;
  w.wt_off = (mat * w.item_rows + w.rb * 16) * RS;
  w.sc_off = mats * w.item_rows * RS + mat * ((w.item_rows * w.ng * 2 + 15) / 16 * 16) +
             w.rb * 16 * w.ng * 2;
  w.sse = op.sse;
  w.s = mat ? op.s1 : op.s0;
  w.sbulk = op.sbulk;
  return w;
}

// Item i = slot * items_rb + row group, advanced by the grid without divisions.
struct ExpertIter {
  int i, slot, rbg;
  __device__ __forceinline__ void start(int first, int items_rb) {
    i = first;
    slot = first / items_rb;
    rbg = first - slot * items_rb;
  }
  __device__ __forceinline__ void next(int G, int items_rb) {
    i += G;
    rbg += G;
    while (rbg >= items_rb) {
      rbg -= items_rb;
      ++slot;
    }
  }
};

// One expert item (row group rbg of expert e, cnt token rows; xrow0: this
// lane's activation row): the warp's row block over its rotated reduction
// slice, partial to the reducer.
__device__ __forceinline__ void expert_item(const StepParams& P, const ExpertWarp& w, StPlan* pl,
                                            Ring& R, Partials& pa, int e, int rbg, int cnt,
                                            const uint8_t* xrow0, int& rot) {
  const int r0 = rbg * w.item_rows;
  const int rows = min(w.item_rows, w.N - r0);
  const int rb_rows = min(16, rows - w.rb * 16);
  const bool bulk = w.sbulk && ((rows * w.ng * 2) & 15) == 0;
  const int ksr = (w.ks + rot) & (w.KS - 1);
  rot = (rot + 1) & (w.KS - 1);
  const int kb0 = (w.KB * ksr) >> w.kslog, kb1 = (w.KB * (ksr + 1)) >> w.kslog;
  const uint8_t* xrow[1] = {xrow0};
  float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
  int st;
  const uint8_t* stage = consume_stage(P, R, pl, &st);
  if (rb_rows > 0 && kb1 > kb0) {
    if (bulk)
      rowblock_compute<1, true, true>(stage + w.wt_off, w.K >> 1,
                                reinterpret_cast<const uint16_t*>(stage + w.sc_off), w.ng,
                                rb_rows, w.K, w.gshift, kb0, kb1, xrow, 1, acc);
    else
      rowblock_compute<1, false, true>(stage + w.wt_off, w.K >> 1,
                          w.s + (size_t)e * w.sse + (size_t)(r0 + w.rb * 16) * w.ng, w.ng,
                          rb_rows, w.K, w.gshift, kb0, kb1, xrow, 1, acc);
  }
  release_stage(R, st);
  partial_publish(P, pa, pl, w.pslot_base + ksr, cnt, acc);
}

// Gate/up + SwiGLU of the shared expert, then (after the routing) of every
// routed expert; the reducer applies SwiGLU, writes and signals per slot.
__device__ void run_moe_up(const StepParams& P, const StOp& op, StPlan* pl, Ring& R,
                           uint64_t* plan_bar, uint64_t* plan_ack, uint32_t& plan_round,
                           uint8_t* xs, Partials& pa) {
  const int G = gridDim.x, g = (threadIdx.x & 31) >> 2;
  const ExpertWarp w = expert_warp(op);
  const int T = op.T, Rr = op.R, E = op.E;
  const int ts = token_stride(op.K);
  // Token of assignment a = t*R + r without a division (a < 2^16 / R).
  const uint32_t rinv = (65536u + (uint32_t)Rr - 1u) / (uint32_t)Rr;
  // The shared slot needs no routing: its assignments are t*R + R-1 (the
  // producer may still be reading the previous plan, which holds the same
  // values for slot 0).
  if (threadIdx.x < T) pl->assign[threadIdx.x] = threadIdx.x * Rr + Rr - 1;
  if (threadIdx.x == 0) {
    pl->slot_start[0] = 0;
    pl->slot_start[1] = T;
    pl->slot_expert[0] = E;
  }
  named_barrier(CBAR, NCT);
  ExpertIter it;
  it.start(first_item(op.rot), w.items_rb);
  int rot = 0;
  const uint8_t* xshared = xs + min(g, T - 1) * ts;
  for (; it.i < w.items_rb; it.next(G, w.items_rb))
    expert_item(P, w, pl, R, pa, E, it.rbg, T, xshared, rot);
  if (threadIdx.x == 0) trace_mark(P, pl->cur_op, 6);
  if (T == 1) {
    // The stager builds a single token's plan (route_one).
    if (threadIdx.x == 0 && !stage_wait(plan_bar, plan_round & 1u, pl) && !pl->abort)
      raise_abort(P, pl, ERR_TIMEOUT);
    if (threadIdx.x == 0) trace_mark(P, pl->cur_op, 2);
    named_barrier(CBAR, NCT);
  } else {
    // The producer must be done with the previous plan before it is replaced.
    if (plan_round > 0) {
      if (threadIdx.x == 0 && !stage_wait(plan_ack, (plan_round - 1) & 1, pl) && !pl->abort)
        raise_abort(P, pl, ERR_TIMEOUT);
      named_barrier(CBAR, NCT);
    }
    build_routing(P, op, pl, plan_bar);
  }
  ++plan_round;
  const int n = pl->nslots * w.items_rb;
  for (; it.i < n; it.next(G, w.items_rb)) {
    const int abase = pl->slot_start[it.slot];
    const int cnt = pl->slot_start[it.slot + 1] - abase;
    const int a = pl->assign[abase + min(g, cnt - 1)];
    const int tok = (int)(((uint32_t)a * rinv) >> 16);
    expert_item(P, w, pl, R, pa, pl->slot_expert[it.slot], it.rbg, cnt, xs + tok * ts, rot);
  }
}

// Down projection of every route (consumer side).  The stager stages each
// item's inputs (the activated rows of its slot) into one of dnb buffers once
// the slot's gate/up is complete; the reducer writes the per-route outputs,
// and the combine follows once every item of the operation is done.
__device__ void run_moe_down(const StepParams& P, const StOp& op, StPlan* pl, Ring& R,
                             const XBufs& X, uint8_t* xs, Partials& pa, DUse& du) {
  const int lane = threadIdx.x & 31, g = lane >> 2;
  const int G = gridDim.x;
  const ExpertWarp w = expert_warp(op);
  const int n = pl->nslots * w.items_rb;
  const int ts = token_stride(op.K);
  const int dnb = X.dnb, drow = X.drow_bytes;
  int rot = 0;
  ExpertIter it;
  for (it.start(first_item(op.rot), w.items_rb); it.i < n; it.next(G, w.items_rb), ++du.u) {
    const int abase = pl->slot_start[it.slot];
    const int cnt = pl->slot_start[it.slot + 1] - abase;
    const int j = du.buf(dnb);
    if (!stage_wait(&X.dready[j], du.phase(dnb), pl) && lane == 0 && !pl->abort)
      raise_abort(P, pl, ERR_TIMEOUT);
    if (threadIdx.x == 0 && it.i < G) trace_mark(P, pl->cur_op, 1);
    // The input buffer is freed once every warp has published its part (the
    // publish synchronizes the warp after its last read of the buffer).
    expert_item(P, w, pl, R, pa, pl->slot_expert[it.slot], it.rbg, cnt,
                xs + (size_t)j * drow + min(g, cnt - 1) * ts, rot);
    if (lane == 0) mbar_arrive(&X.dfree[j]);
  }
}

// Warp w owns rows i = r*16 + w (r < 8) of a 32-column slice, as the KDA
// kernel does, so the arithmetic (and its rounding) is the same.
__device__ void run_kda(const StepParams& P, const StOp& op, int o, StPlan* pl, StKda* kd,
                        uint64_t* xready, uint32_t xphase) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;
  constexpr int KW = NCW;  // computing warps
  constexpr int RPW = 8;   // rows per warp (Dk <= 128)
  const bool worker = warp < KW;
  // Descriptor fields in registers: the loops below store to global memory
  // and must not re-read them.
  const int Dk = op.Dk, Dv = op.Dv, H = op.H, items = op.items;
  const int64_t sb = op.sb, sh = op.sh, sk = op.sk;
  float* const state = op.state;
  const float* const qp = op.q;
  const float* const kp = op.k;
  const float* const vp = op.v;
  const float* const dp = op.decay;
  const float* const bp = op.beta;
  const float scale = op.scale;
  float* const kout = op.kout;
  uint16_t* const kout16 = op.kout_bf16;
  uint32_t* const ktag = op.ktag;
  const uint32_t tag = op_tag(pl, P.nops, o);
  int* const done = &P.sync[op.done];
  const int nsl = (Dv + ST_KDA_COLS - 1) / ST_KDA_COLS;
  bool waited = false;
  for (int u = first_item(op.rot); u < items; u += G) {
    const int bh = u / nsl, sl = u - bh * nsl;
    const int b = bh / H, h = bh - b * H;
    const int col = sl * ST_KDA_COLS + lane;
    const bool col_ok = worker && col < Dv;
    float* base = state + (size_t)b * sb + (size_t)h * sh + col;
    // The state depends on no operation of this launch: read it before the
    // wait for the inputs.
    float c[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const int i = r * KW + warp;
      c[r] = (col_ok && i < Dk) ? base[(size_t)i * sk] : 0.f;
    }
    if (!waited) {
      consumer_op_wait(P, pl, xready, xphase);
      waited = true;
    }
    const size_t vec = (size_t)bh * Dk;
    const float bt = __ldcg(&bp[bh]);
    const float vcol = col_ok ? __ldcg(&vp[(size_t)bh * Dv + col]) : 0.f;
    for (int i = threadIdx.x; i < Dk; i += NCT) {
      const float kv = __ldcg(&kp[vec + i]);
      kd->ed[i] = expf(__ldcg(&dp[vec + i]));
      kd->k[i] = kv;
      kd->bk[i] = __fmul_rn(bt, kv);
      kd->q[i] = __fmul_rn(__ldcg(&qp[vec + i]), scale);
    }
    named_barrier(CBAR, NCT);
    if (worker) {
      float part = 0.f;
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        const int i = r * KW + warp;
        if (i < Dk) {
          c[r] = __fmul_rn(c[r], kd->ed[i]);
          part = __fadd_rn(part, __fmul_rn(c[r], kd->k[i]));
        }
      }
      kd->red[warp][lane] = part;
    }
    named_barrier(CBAR, NCT);
    float pred = 0.f;
#pragma unroll
    for (int w = 0; w < KW; ++w) pred = __fadd_rn(pred, kd->red[w][lane]);
    const float delta = col_ok ? __fsub_rn(vcol, pred) : 0.f;
    named_barrier(CBAR, NCT);
    if (worker) {
      float opart = 0.f;
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        const int i = r * KW + warp;
        if (i < Dk) {
          c[r] = __fadd_rn(c[r], __fmul_rn(kd->bk[i], delta));
          opart = __fadd_rn(opart, __fmul_rn(c[r], kd->q[i]));
        }
      }
      kd->red[warp][lane] = opart;
    }
    named_barrier(CBAR, NCT);
    if (warp == 0) {
      if (sl * ST_KDA_COLS + lane < Dv) {
        float o = 0.f;
#pragma unroll
        for (int w = 0; w < KW; ++w) o = __fadd_rn(o, kd->red[w][lane]);
        if (kout) kout[(size_t)bh * Dv + col] = o;
        if (kout16) kout16[(size_t)bh * Dv + col] = float_to_bf16_bits(o);
        if (ktag) st_tag(ktag + (size_t)bh * Dv + col, float_to_bf16_bits(o), tag);
      }
      // The outputs are published before the state is written back: only
      // the next launch reads the state, so its stores need not complete
      // before the signal.
      warp_signal(done, 1);
    }
    if (worker && col_ok) {
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        const int i = r * KW + warp;
        if (i < Dk) base[(size_t)i * sk] = c[r];
      }
    }
    named_barrier(CBAR, NCT);
  }
  if (!waited) consumer_op_wait(P, pl, xready, xphase);
}

// ---------------------------------------------------------------------------
// Reducer warp: the epilogue of every projection item, in the consumers'
// item order (dense outputs and SwiGLU; gate/up slot signals; down
// projection per-route outputs, arrivals and the routing-weighted combine).
// ---------------------------------------------------------------------------
// Expert-block fields the reducer needs, read once per operation (the
// epilogues store to global memory, so fields read through the descriptor
// would be re-read after every store).
struct MoeEpi {
  uint16_t* y;     // gate/up: activated rows
  uint16_t* wsy;   // down: per-route outputs
  uint32_t* wtag;  // down: tagged copy of the per-route outputs (or null)
  uint16_t* out;   // down: combined rows
  int* slot_cnt;    // gate/up: per-slot counters
  int* items_done;  // down: finished items
  int* done;        // down: combined blocks
  int N, R, KS, RBc, items_rb, item_rows;
};

__device__ __forceinline__ MoeEpi moe_epi(const StepParams& P, const StOp& op) {
  MoeEpi m;
  m.y = op.y;
  m.wsy = op.wsy;
  m.wtag = op.wtag;
  m.out = op.out;
  m.slot_cnt = &P.sync[op.slot_cnt];
  m.items_done = &P.sync[op.items_done];
  m.done = &P.sync[op.done];
  m.N = op.N;
  m.R = op.R;
  m.KS = op.KS;
  m.RBc = op.RBc;
  m.items_rb = op.items_rb;
  m.item_rows = op.RBc * 16;
  return m;
}

// Epilogue of one gate/up item (slot ei.slot, row group ei.rbg; assignments
// assign[abase .. abase+cnt)): SwiGLU of the summed slices into the activated
// rows, then the slot's counter.
__device__ bool reduce_up_item(const MoeEpi& m, StPlan* pl, Partials& pa, int abase, int cnt,
                               const ExpertIter& ei) {
  const int lane = threadIdx.x & 31;
  if (!partial_take(pa, pl)) return false;
  const int* assign = pl->assign + abase;
  const int r0 = ei.rbg * m.item_rows;
  const int rows = min(m.item_rows, m.N - r0);
  uint16_t* const y = m.y;
  const int N = m.N;
  if (cnt == 1 && rows <= 16) {
    // One token, one row block: lanes 0-15 sum the gate slices of row
    // `lane`, lanes 16-31 the up slices of row `lane - 16`.
    uint16_t* const yrow = y + (size_t)assign[0] * N + r0;
    const int r = lane & 15, mat = lane >> 4;
    const float v = r < rows ? partial_sum(pa, mat, m.RBc, m.KS, 0, r, 0) : 0.f;
    const float uv = __shfl_down_sync(0xffffffffu, v, 16);
    if (lane < rows) yrow[lane] = float_to_bf16_bits(swiglu_contract(v, uv));
  } else if (cnt == 1) {
    uint16_t* const yrow = y + (size_t)assign[0] * N + r0;
    for (int r = lane; r < rows; r += 32) {
      const float gv = partial_sum(pa, 0, m.RBc, m.KS, r >> 4, r & 15, 0);
      const float uv = partial_sum(pa, 1, m.RBc, m.KS, r >> 4, r & 15, 0);
      yrow[r] = float_to_bf16_bits(swiglu_contract(gv, uv));
    }
  } else {
    const int n = rows * cnt;
    for (int idx = lane; idx < n; idx += 32) {
      const int r = idx / cnt, tok = idx - r * cnt;
      const float gv = partial_sum(pa, 0, m.RBc, m.KS, r >> 4, r & 15, tok);
      const float uv = partial_sum(pa, 1, m.RBc, m.KS, r >> 4, r & 15, tok);
      y[(size_t)assign[tok] * N + r0 + r] = float_to_bf16_bits(swiglu_contract(gv, uv));
    }
  }
  partial_release(pa);
  if (lane == 0) red_release(m.slot_cnt + ei.slot, (rows + 15) >> 4);
  return true;
}

// Epilogue of one down item: the per-route outputs.
__device__ bool reduce_down_item(const MoeEpi& m, StPlan* pl, Partials& pa, int abase, int cnt,
                                 const ExpertIter& ei, uint32_t tag) {
  const int lane = threadIdx.x & 31;
  if (!partial_take(pa, pl)) return false;
  const int* assign = pl->assign + abase;
  const int r0 = ei.rbg * m.item_rows;
  const int rows = min(m.item_rows, m.N - r0);
  const int N = m.N;
  uint16_t* const wsy = m.wsy;
  uint32_t* const wtag = m.wtag;
  if (cnt == 1) {
    const size_t row0 = (size_t)assign[0] * N + r0;
    for (int r = lane; r < rows; r += 32) {
      const uint16_t b = float_to_bf16_bits(partial_sum(pa, 0, m.RBc, m.KS, r >> 4, r & 15, 0));
      wsy[row0 + r] = b;
      if (wtag) st_tag(wtag + row0 + r, b, tag);
    }
  } else {
    const int n = rows * cnt;
    for (int idx = lane; idx < n; idx += 32) {
      const int r = idx / cnt, tok = idx - r * cnt;
      const float v = partial_sum(pa, 0, m.RBc, m.KS, r >> 4, r & 15, tok);
      const size_t at = (size_t)assign[tok] * N + r0 + r;
      const uint16_t b = float_to_bf16_bits(v);
      wsy[at] = b;
      if (wtag) st_tag(wtag + at, b, tag);
    }
  }
  partial_release(pa);
  return true;
}

// Combine of the (token, 16-row block) pairs p = first_item(rot) + k*grid
// once every down item of the operation is done: out = bf16(sum_r
// routed_r * w_r in route order) + shared, two pairs per pass (lanes 0-15 and
// 16-31, one row each).  Returns false when the wait gave up.
__device__ bool combine_pairs(const StepParams& P, const MoeEpi& m, StPlan* pl, int T, int rot,
                              int total_items) {
  const int lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const int N = m.N, R = m.R, top_k = R - 1;
  const int nrb = (N + 15) >> 4;
  const int npairs = T * nrb;
  const int p0 = first_item(rot);
  if (p0 >= npairs) return true;
  if (!stager_poll(P, pl, (int)(m.items_done - P.sync), total_items)) return false;
  const uint16_t* const wsy = m.wsy;
  uint16_t* const out = m.out;
  int combined = 0;
  for (int p = p0; p < npairs; p += 2 * G) {
    const int mine = (lane < 16) ? p : p + G;
    if (mine < npairs) {
      const int tok = mine / nrb, rb = mine - tok * nrb;
      const int row = rb * 16 + (lane & 15);
      if (row < N) {
        const uint16_t* ws = wsy + (size_t)tok * R * N + row;
        const float* rw = pl->route_w + tok * top_k;
        // Every route's value in flight at once, then the sum in route order.
        uint16_t rv[ST_MAX_TOPK];
#pragma unroll
        for (int r = 0; r < ST_MAX_TOPK; ++r) rv[r] = r < top_k ? __ldcg(ws + (size_t)r * N) : 0;
        const uint16_t sv = __ldcg(ws + (size_t)(R - 1) * N);
        out[(size_t)tok * N + row] = combine_value(rv, rw, top_k, sv);
      }
    }
    combined += (p + G < npairs) ? 2 : 1;
  }
  warp_signal(m.done, combined);
  return true;
}

// Reducer `rid` walks the consumers' item sequence and takes its own items.
__device__ void reducer_main(const StepParams& P, StPlan* pl, Partials& pa, uint64_t* plan_bar,
                             uint64_t* plan_ack, int rid) {
  const int lane = threadIdx.x & 31;
  const int G = gridDim.x;
  uint32_t plan_phase = 0;
  bool ok = true;
  for (int o = 0; o < P.nops && ok; ++o) {
    const StOp& op = P.ops[o];
    if (o > 0 && lane == 0) trace_mark(P, o - 1, 5);
    if (op.type == OP_DENSE) {
      const int T = op.T, nprob = op.nprob;
      const int n = op.p[nprob - 1].item_begin + op.p[nprob - 1].items;
      int blocks = 0;
      int p = -1, pend = 0, ib = 0, RBc = 1, KS = 1, N = 0, item_rows = 0;
      bool pair = false;
      uint16_t* y = nullptr;
      uint32_t* ytag = nullptr;
      int64_t ys = 0;
      for (int i = first_item(op.rot); i < n && ok; i += G) {
        if (i >= pend) {
          do {
            ++p;
            pend = op.p[p].item_begin + op.p[p].items;
          } while (i >= pend);
          const StDense& Dg = op.p[p];
          ib = Dg.item_begin;
          RBc = Dg.RBc;
          KS = Dg.KS;
          N = Dg.N;
          item_rows = RBc * 16;
          pair = Dg.mats == 2;
          y = Dg.y;
          ytag = Dg.ytag;
          ys = Dg.ys;
        }
        if (!pa.mine(rid)) {
          ++pa.count;
          continue;
        }
        if (!partial_take(pa, pl)) {
          ok = false;
          break;
        }
        const int r0 = (i - ib) * item_rows;
        const int rows = min(item_rows, N - r0);
        blocks += (rows + 15) >> 4;
        if (T == 1) {
          for (int r = lane; r < rows; r += 32) {
            const float v0 = partial_sum(pa, 0, RBc, KS, r >> 4, r & 15, 0);
            const float val =
                pair ? swiglu_contract(v0, partial_sum(pa, 1, RBc, KS, r >> 4, r & 15, 0)) : v0;
            const uint16_t b = float_to_bf16_bits(val);
            y[r0 + r] = b;
            if (ytag) st_tag(ytag + r0 + r, b, op_tag(pl, P.nops, o));
          }
        } else {
          for (int idx = lane; idx < rows * T; idx += 32) {
            const int r = idx / T, tok = idx - r * T;
            const float v0 = partial_sum(pa, 0, RBc, KS, r >> 4, r & 15, tok);
            const float val =
                pair ? swiglu_contract(v0, partial_sum(pa, 1, RBc, KS, r >> 4, r & 15, tok)) : v0;
            const uint16_t b = float_to_bf16_bits(val);
            y[(size_t)tok * ys + r0 + r] = b;
            if (ytag) st_tag(ytag + (size_t)tok * N + r0 + r, b, op_tag(pl, P.nops, o));
          }
        }
        partial_release(pa);
      }
      __syncwarp();
      if (lane == 0 && blocks > 0) red_release(&P.sync[op.done], blocks);
    } else if (op.type == OP_MOE_UP) {
      const MoeEpi m = moe_epi(P, op);
      ExpertIter ei;
      ei.start(first_item(op.rot), m.items_rb);
      for (; ei.i < m.items_rb && ok; ei.next(G, m.items_rb)) {
        if (pa.mine(rid))
          ok = reduce_up_item(m, pl, pa, 0, op.T, ei);
        else
          ++pa.count;
      }
      if (!ok) break;
      if (!stage_wait(plan_bar, plan_phase, pl)) break;
      const int n = pl->nslots * m.items_rb;
      for (; ei.i < n && ok; ei.next(G, m.items_rb)) {
        if (!pa.mine(rid)) {
          ++pa.count;
          continue;
        }
        const int abase = pl->slot_start[ei.slot];
        ok = reduce_up_item(m, pl, pa, abase, pl->slot_start[ei.slot + 1] - abase, ei);
      }
    } else if (op.type == OP_MOE_DOWN) {
      const MoeEpi m = moe_epi(P, op);
      const int n = pl->nslots * m.items_rb;
      int items = 0;
      ExpertIter ei;
      for (ei.start(first_item(op.rot), m.items_rb); ei.i < n && ok; ei.next(G, m.items_rb)) {
        if (!pa.mine(rid)) {
          ++pa.count;
          continue;
        }
        const int abase = pl->slot_start[ei.slot];
        ok = reduce_down_item(m, pl, pa, abase, pl->slot_start[ei.slot + 1] - abase, ei,
                              op_tag(pl, P.nops, o));
        ++items;
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0 && items > 0) red_release(m.items_done, items);
      // One reducer writes the combine output.
      if (rid == 0) ok = combine_pairs(P, m, pl, op.T, op.rot, n);
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(plan_ack);
      plan_phase ^= 1;
    }
  }
  if (!ok && lane == 0 && !pl->abort) raise_abort(P, pl, ERR_TIMEOUT);
}

// ---------------------------------------------------------------------------
// The kernel.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(ST_THREADS, 1) step_kernel(const __grid_constant__ StepParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5;
  StPlan* pl = reinterpret_cast<StPlan*>(smem + P.scr_off);
  StKda* kd = reinterpret_cast<StKda*>(smem + P.scr_off + sizeof(StPlan));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P.bar_off);
  Ring R;
  R.base = smem + P.ring_off;
  R.full = bars;
  R.empty = bars + P.stages;
  R.stages = P.stages;
  R.stage_bytes = P.stage_bytes;
  R.use = 0;
  R.slot = 0;
  R.phase = 0;
  uint64_t* plan_bar = bars + 2 * P.stages;
  uint64_t* plan_ack = plan_bar + 1;
  Partials pa;
  pa.buf = reinterpret_cast<float*>(smem + P.red_off);
  pa.done = plan_ack + 1;
  pa.free = pa.done + ST_NB;
  pa.T = P.T;
  pa.count = 0;
  XBufs X;
  X.base = smem;
  X.x_bytes = P.x_bytes;
  X.nxb = P.nxb;
  X.desc = reinterpret_cast<StOp*>(smem + P.desc_off);
  X.ready = pa.free + ST_NB;
  X.free = X.ready + 2;
  X.dsc = X.free + 2;
  X.dready = X.dsc + 2;
  X.dfree = X.dready + ST_DNB;
  X.dnb = P.dnb;
  X.drow_bytes = P.drow_bytes;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P.stages; ++s) {
      mbar_init(&R.full[s], 1);
      mbar_init(&R.empty[s], NCW);
    }
    mbar_init(plan_bar, 1);
    mbar_init(plan_ack, 1 + ST_REDUCERS);  // producer and reducers
    for (int b = 0; b < ST_NB; ++b) {
      mbar_init(&pa.done[b], NCW);
      mbar_init(&pa.free[b], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&X.ready[b], 1);
      mbar_init(&X.dsc[b], 1);
      mbar_init(&X.free[b], NCW);
    }
    for (int b = 0; b < ST_DNB; ++b) {
      mbar_init(&X.dready[b], 1);
      mbar_init(&X.dfree[b], NCW);
    }
    mbar_fence_init();
    pl->abort = 0;
    pl->nslots = 0;
  }
  for (int e = threadIdx.x; e <= ST_MAX_E; e += ST_THREADS) pl->slot_of[e] = -1;
  __syncthreads();

  if (warp == NCW) {
    // Weights are constant: stream them at once; only the routed experts
    // wait for the consumers' plan.
    producer_main(P, pl, R, plan_bar, plan_ack);
    return;
  }
  if (warp > NCW && warp <= NCW + ST_REDUCERS) {
    reducer_main(P, pl, pa, plan_bar, plan_ack, warp - NCW - 1);
    named_barrier(EXIT_BAR, NCT + 32 * ST_REDUCERS);
    return;
  }
  if (warp == NCW + 1 + ST_REDUCERS) {
    pdl_wait();
    stager_main(P, pl, X, plan_bar, plan_ack);
    return;
  }

  // Counters are reset by the previous launch; wait for it to finish.
  pdl_wait();
  if (threadIdx.x == 0) {
    pl->launch = (uint32_t)*((volatile int*)&P.sync[P.parity_idx]);
    pl->parity = (int)(pl->launch & 1u);
  }
  named_barrier(CBAR, NCT);
  uint32_t plan_round = 0;
  DUse du;
  int xb = 0;
  uint32_t xph = 0;
  for (int o = 0; o < P.nops; ++o) {
    if (threadIdx.x == 0) {
      pl->cur_op = o;
      trace_mark(P, o, 0);
    }
    const int type = P.ops[o].type;
    uint8_t* xs = X.base + (size_t)xb * X.x_bytes;
    // The descriptor copy is available before the operation's inputs are:
    // work that needs only the descriptor goes before the input wait.
    if (!stage_wait(&X.dsc[xb], xph, pl) && (threadIdx.x & 31) == 0 && !pl->abort)
      raise_abort(P, pl, ERR_TIMEOUT);
    if (type == OP_KDA) {
      // The KDA state does not depend on this launch: its loads are issued
      // before the wait for the inputs (inside run_kda).
      run_kda(P, P.ops[o], o, pl, kd, &X.ready[xb], xph);
    } else if (type == OP_DENSE) {
      run_dense(P, X.desc[xb], pl, R, xs, pa, &X.ready[xb], xph);
    } else {
      consumer_op_wait(P, pl, &X.ready[xb], xph);
      const StOp& op = X.desc[xb];
      if (op.cstage) consumer_stage(P, pl, op, xs);
      switch (type) {
        case OP_ROUTER:
          run_router(P, op, pl, R, xs);
          break;
        case OP_MOE_UP:
          run_moe_up(P, op, pl, R, plan_bar, plan_ack, plan_round, xs, pa);
          break;
        case OP_MOE_DOWN:
          run_moe_down(P, op, pl, R, X, xs, pa, du);
          break;
        default:
          break;
      }
    }
    // This warp is done with the buffer and the descriptor copy.
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&X.free[xb]);
    if (++xb == X.nxb) {
      xb = 0;
      xph ^= 1u;
    }
    if (threadIdx.x == 0) trace_mark(P, o, 3);
  }
  // Exit: once the reducer is done too, the last CTA resets every counter for
  // the next launch (all of its consumer threads; the exit counter last).
  named_barrier(EXIT_BAR, NCT + 32 * ST_REDUCERS);
  if (threadIdx.x == 0) {
    __threadfence();
    const int old = atomicAdd(&P.sync[P.exit_idx], 1);
    pl->last = (old == (int)gridDim.x - 1);
    if (pl->last) __threadfence();
  }
  named_barrier(CBAR, NCT);
  if (pl->last) {
    for (int i = threadIdx.x; i < P.nsync; i += NCT)
      if (i != P.exit_idx && i != P.parity_idx) P.sync[i] = 0;
    if (threadIdx.x == 0) P.sync[P.parity_idx] = (int)(pl->launch + 1u);
    __threadfence();
    named_barrier(CBAR, NCT);
    if (threadIdx.x == 0) P.sync[P.exit_idx] = 0;
  }
}

// ---------------------------------------------------------------------------
// Host side: program construction.
// ---------------------------------------------------------------------------
struct StepProgram {
  int T = 0;
  std::vector<StOp> ops;
  int nsync = 0;
  bool finalized = false;
  int device = -1;
  StOp* d_ops = nullptr;
  int* d_sync = nullptr;
  uint32_t* d_tags = nullptr;  // tagged activation copies
  StepParams params = {};
  size_t smem = 0;
  int grid = 0;
};

// Counters are allocated in whole 128-byte lines, so that polls of one
// operation's counter do not share a line with another's atomics.
static int add_sync(StepProgram* pr, int n) {
  const int at = pr->nsync;
  pr->nsync += (n + 31) / 32 * 32;
  return at;
}

static int check_deps(StepProgram* pr, const int* deps, int ndeps, StOp& op) {
  KB_REQUIRE(ndeps >= 0 && ndeps <= ST_MAX_DEPS, KB_ERR_UNSUPPORTED,
             "at most %d dependencies per operation", ST_MAX_DEPS);
  KB_REQUIRE(ndeps == 0 || deps, KB_ERR_NULL_POINTER, "deps is NULL");
  op.ndeps = ndeps;
  for (int d = 0; d < ndeps; ++d) {
    KB_REQUIRE(deps[d] >= 0 && deps[d] < (int)pr->ops.size(), KB_ERR_BAD_SHAPE,
               "dependency %d is not an earlier operation", deps[d]);
    KB_REQUIRE(pr->ops[deps[d]].type != OP_MOE_UP, KB_ERR_BAD_SHAPE,
               "depend on the expert block's down operation, not its gate/up");
    op.dep[d] = deps[d];
  }
  return KB_OK;
}

// Warp split for the executor: items of at most ST_STAGE_TARGET bytes (dense
// rows longer than that are split into reduction chunks, one stage each),
// smaller items while the operation has fewer items than CTAs, and at least
// one 128-wide block per warp.
static void step_split(int K, int mats, int64_t row_blocks, int grid, int* KS, int* RBc,
                       int* nchunk) {
  const int KB = (K + 127) / 128;
  const int maxks = NCW / mats;
  int chunks = 1;
  if (mats == 1)
    while ((int64_t)16 * (K / chunks) / 2 > ST_STAGE_TARGET && KB % (chunks * 2) == 0)
      chunks *= 2;
  const int KBc = KB / chunks;
  int rbc = maxks;
  while (rbc > 1 && (int64_t)rbc * 16 * (K / chunks) / 2 * mats > ST_STAGE_TARGET) rbc /= 2;
  while (rbc > 1 && (row_blocks + rbc - 1) / rbc < grid && KBc >= maxks / (rbc / 2)) rbc /= 2;
  int ks = maxks / rbc;
  while (ks > 1 && KBc < ks) {
    ks /= 2;
    rbc *= 2;
  }
  *KS = ks;
  *RBc = rbc;
  *nchunk = chunks;
}

static int current_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  const int n = num_sms(dev);
  return n > 0 ? n : 148;
}

// Tag field of the writer in `src` of the rows x[t * stride + k] (t < T,
// k < K) as complete bf16 rows, or null: a dense problem's y or a KDA step's
// bf16 output.
static uint32_t** tag_writer(StOp& src, const uint16_t* x, int K, int64_t stride, int T) {
  if (src.type == OP_DENSE) {
    for (int q = 0; q < src.nprob; ++q) {
      StDense& Q = src.p[q];
      if (Q.y == x && Q.N == K && Q.ys == stride) return &Q.ytag;
    }
  } else if (src.type == OP_KDA) {
    if (src.kout_bf16 == x && src.H * src.Dv == K && stride == K && src.B == T)
      return &src.ktag;
  }
  return nullptr;
}

// Tagged activations: operation o reads the output of operation o - 1 as
// tagged words (no wait for o - 1's completion counter) when every input it
// stages comes from a writer that can keep a tagged copy.  Records (field,
// word offset) pairs for the arena and sets op.tag_src.
static void plan_tags(StepProgram* pr, size_t o, std::vector<std::pair<uint32_t**, size_t>>& fields,
                      size_t& words) {
  StOp& op = pr->ops[o];
  op.tag_src = -1;
  if (!op.cstage || o == 0) return;
  StOp& src = pr->ops[o - 1];
  const int T = pr->T;
  auto offset_of = [&](uint32_t** writer, size_t n) {
    for (const auto& f : fields)
      if (f.first == writer) return f.second;
    const size_t at = words;
    words += (n + 31) / 32 * 32;
    fields.emplace_back(writer, at);
    return at;
  };
  if (op.type == OP_ROUTER) {
    uint32_t** w = tag_writer(src, op.rx, op.K, op.rxs, T);
    if (!w) return;
    fields.emplace_back(&op.rxtag, offset_of(w, (size_t)T * op.K));
    op.tag_src = (int)o - 1;
    return;
  }
  if (op.type != OP_DENSE) return;
  uint32_t** wr[ST_MAX_PROB] = {};
  bool comb = false;
  for (int i = 0; i < op.nprob; ++i) {
    const StDense& D = op.p[i];
    if (D.nchunk > 1) return;
    bool dup = false;
    for (int q = 0; q < i; ++q) dup |= (op.p[q].x_off == D.x_off);
    if (dup) continue;
    if (D.xcomb) {
      comb = true;
      continue;
    }
    wr[i] = tag_writer(src, D.x, D.K, D.xs, T);
    if (!wr[i]) return;
  }
  for (int i = 0; i < op.nprob; ++i)
    if (wr[i]) fields.emplace_back(&op.p[i].xtag, offset_of(wr[i], (size_t)T * op.p[i].K));
  if (comb) offset_of(&src.wtag, (size_t)T * src.R * src.N);
  op.tag_src = (int)o - 1;
}

}  // namespace kb

using kb::StepProgram;

extern "C" {

int kb_step_create(int64_t tokens, kb_step** out) {
  kb::clear_error();
  KB_REQUIRE(out, KB_ERR_NULL_POINTER, "out is NULL");
  *out = nullptr;
  KB_REQUIRE(tokens >= 1 && tokens <= kb::ST_MAX_T, KB_ERR_UNSUPPORTED,
             "the step executor supports 1 to %d tokens", kb::ST_MAX_T);
  StepProgram* pr = new (std::nothrow) StepProgram();
  KB_REQUIRE(pr, KB_ERR_DEVICE, "out of host memory");
  pr->T = (int)tokens;
  *out = reinterpret_cast<kb_step*>(pr);
  return KB_OK;
}

void kb_step_destroy(kb_step* step) {
  StepProgram* pr = reinterpret_cast<StepProgram*>(step);
  if (!pr) return;
  if (pr->d_ops || pr->d_sync || pr->d_tags) {
    int cur = -1;
    cudaGetDevice(&cur);
    if (pr->device >= 0) cudaSetDevice(pr->device);
    cudaFree(pr->d_ops);
    cudaFree(pr->d_sync);
    cudaFree(pr->d_tags);
    if (cur >= 0) cudaSetDevice(cur);
  }
  delete pr;
}

int kb_step_add_dense(kb_step* step, const kb_dense_problem* problems, int count,
                      const int* deps, int ndeps, int* op_out) {
  kb::clear_error();
  StepProgram* pr = reinterpret_cast<StepProgram*>(step);
  KB_REQUIRE(pr && problems && op_out, KB_ERR_NULL_POINTER, "NULL argument");
  KB_REQUIRE(!pr->finalized, KB_ERR_UNSUPPORTED, "program already finalized");
  KB_REQUIRE(count >= 1 && count <= kb::ST_MAX_PROB, KB_ERR_UNSUPPORTED,
             "1 to %d problems per dense operation", kb::ST_MAX_PROB);
  kb::StOp op = {};
  op.type = kb::OP_DENSE;
  op.T = pr->T;
  int rc = kb::check_deps(pr, deps, ndeps, op);
  if (rc) return rc;
  int64_t row_blocks = 0;
  for (int i = 0; i < count; ++i) row_blocks += (problems[i].N + 15) / 16;
  int items = 0, xbytes = 0;
  for (int i = 0; i < count; ++i) {
    const kb_dense_problem& q = problems[i];
    KB_REQUIRE(q.M == pr->T, KB_ERR_BAD_SHAPE, "problem %d: M=%lld differs from the step's %d",
               i, (long long)q.M, pr->T);
    KB_REQUIRE(q.K > 0 && q.K % 128 == 0 && q.K <= 16384 && q.N > 0 && q.N < (1 << 24),
               KB_ERR_UNSUPPORTED, "problem %d: need K %% 128 == 0, K <= 16384", i);
    int gs = 0;
    rc = kb::check_group(q.K, q.group, &gs);
    if (rc) return rc;
    KB_REQUIRE(q.x && q.packed && q.scales && q.y, KB_ERR_NULL_POINTER,
               "problem %d: NULL pointer", i);
    KB_REQUIRE(kb::aligned(q.x, 16) && q.x_stride % 8 == 0 && kb::aligned(q.packed, 16) &&
                   kb::aligned(q.scales, 2) && q.y_stride >= q.N,
               KB_ERR_ALIGNMENT, "problem %d: misaligned operand", i);
    kb::StDense& D = op.p[i];
    D.x = q.x;
    D.xs = q.x_stride;
    D.w = q.packed;
    D.s = q.scales;
    D.y = q.y;
    D.ys = q.y_stride;
    D.K = (int)q.K;
    D.N = (int)q.N;
    D.gshift = gs;
    kb::step_split(D.K, 1, row_blocks, kb::current_sms(), &D.KS, &D.RBc, &D.nchunk);
    D.mats = 1;
    KB_REQUIRE(D.nchunk == 1 || count == 1, KB_ERR_UNSUPPORTED,
               "problem %d: a reduction width of %lld needs an operation of its own", i,
               (long long)q.K);
    D.items = (D.N + 16 * D.RBc - 1) / (16 * D.RBc);
    D.item_begin = items;
    items += D.items;
    D.x_off = -1;
    for (int j = 0; j < i; ++j)
      if (op.p[j].x == D.x && op.p[j].K == D.K) D.x_off = op.p[j].x_off;
    if (D.x_off < 0) {
      D.x_off = xbytes;
      xbytes += pr->T * kb::token_stride(D.K);
    }
    op.target += (D.N + 15) / 16;
  }
  op.nprob = count;
  op.items = items;
  op.done = kb::add_sync(pr, 1);
  *op_out = (int)pr->ops.size();
  pr->ops.push_back(op);
  return KB_OK;
}

int kb_step_add_swiglu(kb_step* step, const uint16_t* x, int64_t x_stride, int64_t K,
                       const uint8_t* w1_packed, const uint16_t* w1_scales,
                       const uint8_t* w3_packed, const uint16_t* w3_scales, int64_t N,
                       int64_t group, uint16_t* y, int64_t y_stride, const int* deps, int ndeps,
                       int* op_out) {
  kb::clear_error();
  StepProgram* pr = reinterpret_cast<StepProgram*>(step);
  KB_REQUIRE(pr && x && w1_packed && w1_scales && w3_packed && w3_scales && y && op_out,
             KB_ERR_NULL_POINTER, "NULL argument");
  KB_REQUIRE(!pr->finalized, KB_ERR_UNSUPPORTED, "program already finalized");
  KB_REQUIRE(K > 0 && K % 128 == 0 && K <= 16384 && N > 0 && N < (1 << 24),
             KB_ERR_UNSUPPORTED, "need K %% 128 == 0, K <= 16384");
  int gs = 0;
  int rc = kb::check_group(K, group, &gs);
  if (rc) return rc;
  KB_REQUIRE(kb::aligned(x, 16) && x_stride % 8 == 0 && kb::aligned(w1_packed, 16) &&
                 kb::aligned(w3_packed, 16) && kb::aligned(w1_scales, 2) &&
                 kb::aligned(w3_scales, 2) && y_stride >= N,
             KB_ERR_ALIGNMENT, "misaligned operand");
  kb::StOp op = {};
  op.type = kb::OP_DENSE;
  op.T = pr->T;
  rc = kb::check_deps(pr, deps, ndeps, op);
  if (rc) return rc;
  kb::StDense& D = op.p[0];
  D.x = x;
  D.xs = x_stride;
  D.w = w1_packed;
  D.s = w1_scales;
  D.w3 = w3_packed;
  D.s3 = w3_scales;
  D.y = y;
  D.ys = y_stride;
  D.K = (int)K;
  D.N = (int)N;
  D.gshift = gs;
  D.mats = 2;
  kb::step_split(D.K, 2, (N + 15) / 16, kb::current_sms(), &D.KS, &D.RBc, &D.nchunk);
  D.items = (D.N + 16 * D.RBc - 1) / (16 * D.RBc);
  D.item_begin = 0;
  D.x_off = 0;
  op.nprob = 1;
  op.items = D.items;
  op.target = (D.N + 15) / 16;
  op.done = kb::add_sync(pr, 1);
  *op_out = (int)pr->ops.size();
  pr->ops.push_back(op);
  return KB_OK;
}

int kb_step_add_router(kb_step* step, const uint16_t* hidden, int64_t h_stride, int64_t K,
                       const uint16_t* weight, const float* bias, int64_t E, int64_t top_k,
                       int renormalize, float scaling, void* scratch, int64_t* idx_out,
                       float* w_out, const int* deps, int ndeps, int* op_out) {
  kb::clear_error();
  StepProgram* pr = reinterpret_cast<StepProgram*>(step);
  KB_REQUIRE(pr && hidden && weight && scratch && idx_out && w_out && op_out,
             KB_ERR_NULL_POINTER, "NULL argument");
  KB_REQUIRE(!pr->finalized, KB_ERR_UNSUPPORTED, "program already finalized");
  KB_REQUIRE(E >= 1 && E <= kb::ST_MAX_E && top_k >= 1 && top_k <= kb::ST_MAX_TOPK &&
                 top_k <= E && K > 0 && K % 8 == 0 && K <= 8192,
             KB_ERR_UNSUPPORTED, "step router supports E <= %d, top_k <= %d, K %% 8 == 0",
             kb::ST_MAX_E, kb::ST_MAX_TOPK);
  KB_REQUIRE(kb::aligned(hidden, 16) && h_stride % 8 == 0 && kb::aligned(weight, 16) &&
                 kb::aligned(scratch, 8),
             KB_ERR_ALIGNMENT, "hidden/weight must be 16-byte aligned, scratch 8-byte aligned");
  kb::StOp op = {};
  op.type = kb::OP_ROUTER;
  op.T = pr->T;
  int rc = kb::check_deps(pr, deps, ndeps, op);
  if (rc) return rc;
  op.rx = hidden;
  op.rxs = h_stride;
  op.rw = weight;
  op.rbias = bias;
  op.E = (int)E;
  op.K = (int)K;
  op.top_k = (int)top_k;
  op.renorm = renormalize;
  op.scaling = scaling;
  op.rwords = static_cast<unsigned long long*>(scratch);
  op.idx_out = idx_out;
  op.w_out = w_out;
  op.items = (int)((E + kb::ST_RT_EXPERTS - 1) / kb::ST_RT_EXPERTS);
  op.target = (int)E;
  op.done = kb::add_sync(pr, 1);
  *op_out = (int)pr->ops.size();
  pr->ops.push_back(op);
  return KB_OK;
}

int kb_step_add_moe(kb_step* step, int router_op, const uint16_t* hidden, int64_t h_stride,
                    int64_t H, const uint8_t* w1_packed, const uint16_t* w1_scales,
                    const uint8_t* w3_packed, const uint16_t* w3_scales,
                    const uint8_t* w2_packed, const uint16_t* w2_scales, int64_t I,
                    int64_t group, uint16_t* activated, uint16_t* routed_out, uint16_t* out,
                    const int* deps, int ndeps, int* op_out) {
  kb::clear_error();
  StepProgram* pr = reinterpret_cast<StepProgram*>(step);
  KB_REQUIRE(pr && hidden && w1_packed && w1_scales && w3_packed && w3_scales && w2_packed &&
                 w2_scales && activated && routed_out && out && op_out,
             KB_ERR_NULL_POINTER, "NULL argument");
  KB_REQUIRE(!pr->finalized, KB_ERR_UNSUPPORTED, "program already finalized");
  KB_REQUIRE(router_op >= 0 && router_op < (int)pr->ops.size() &&
                 pr->ops[router_op].type == kb::OP_ROUTER,
             KB_ERR_BAD_SHAPE, "router_op %d is not a router operation", router_op);
  const kb::StOp& rop = pr->ops[router_op];
  KB_REQUIRE(rop.K == H, KB_ERR_BAD_SHAPE, "hidden width %lld differs from the router's %d",
             (long long)H, rop.K);
  KB_REQUIRE(H % 128 == 0 && I % 128 == 0 && H <= 16384 && I <= 16384, KB_ERR_UNSUPPORTED,
             "hidden and intermediate widths must be multiples of 128");
  int gs_up = 0, gs_dn = 0;
  int rc = kb::check_group(H, group, &gs_up);
  if (rc) return rc;
  rc = kb::check_group(I, group, &gs_dn);
  if (rc) return rc;
  KB_REQUIRE(kb::aligned(hidden, 16) && h_stride % 8 == 0 && kb::aligned(w1_packed, 16) &&
                 kb::aligned(w3_packed, 16) && kb::aligned(w2_packed, 16) &&
                 kb::aligned(activated, 16),
             KB_ERR_ALIGNMENT, "misaligned expert operand");
  const int T = pr->T, E = rop.E, R = rop.top_k + 1;
  kb::StOp up = {};
  up.type = kb::OP_MOE_UP;
  up.T = T;
  rc = kb::check_deps(pr, deps, ndeps, up);
  if (rc) return rc;
  up.router_op = router_op;
  up.E = E;
  up.R = R;
  up.mx = hidden;
  up.mxs = h_stride;
  up.w0 = w1_packed;
  up.s0 = w1_scales;
  up.w1 = w3_packed;
  up.s1 = w3_scales;
  up.wse = I * (H / 2);
  up.sse = I * (H / group);
  up.K = (int)H;
  up.N = (int)I;
  up.gshift = gs_up;
  int nchunk = 1;
  kb::step_split(up.K, 2, (int64_t)(1 + T * rop.top_k) * ((I + 15) / 16), kb::current_sms(),
                 &up.KS, &up.RBc, &nchunk);
  up.items_rb = (int)((I + 16 * up.RBc - 1) / (16 * up.RBc));
  up.y = activated;
  up.sbulk = kb::aligned(w1_scales, 16) && kb::aligned(w3_scales, 16) && (up.sse * 2) % 16 == 0;
  up.rot = ((int)pr->ops.size() * 37) % kb::current_sms();
  up.done = kb::add_sync(pr, 1);
  up.slot_cnt = kb::add_sync(pr, kb::ST_MAX_SLOTS);
  up.target = 0;
  const int up_index = (int)pr->ops.size();
  pr->ops.push_back(up);

  kb::StOp dn = {};
  dn.type = kb::OP_MOE_DOWN;
  dn.T = T;
  dn.ndeps = 0;
  dn.router_op = router_op;
  dn.E = E;
  dn.R = R;
  dn.mx = activated;
  dn.mxs = I;
  dn.w0 = w2_packed;
  dn.s0 = w2_scales;
  dn.wse = H * (I / 2);
  dn.sse = H * (I / group);
  dn.K = (int)I;
  dn.N = (int)H;
  dn.gshift = gs_dn;
  kb::step_split(dn.K, 1, (int64_t)(1 + T * rop.top_k) * ((H + 15) / 16), kb::current_sms(),
                 &dn.KS, &dn.RBc, &nchunk);
  dn.items_rb = (int)((H + 16 * dn.RBc - 1) / (16 * dn.RBc));
  dn.up_rb = (int)((I + 15) / 16);
  dn.slot_cnt = pr->ops[up_index].slot_cnt;
  dn.wsy = routed_out;
  dn.out = out;
  dn.sbulk = kb::aligned(w2_scales, 16) && (dn.sse * 2) % 16 == 0;
  dn.rot = ((up_index + 1) * 37) % kb::current_sms();
  dn.done = kb::add_sync(pr, 1);
  dn.items_done = kb::add_sync(pr, 1);
  dn.target = T * (int)((H + 15) / 16);
  *op_out = (int)pr->ops.size();
  pr->ops.push_back(dn);
  return KB_OK;
}

int kb_step_add_kda(kb_step* step, float* state, int64_t sb, int64_t sh, int64_t sk,
                    const float* q, const float* k, const float* v, const float* decay,
                    const float* beta, int64_t B, int64_t H, int64_t Dk, int64_t Dv,
                    float scale, float* out, uint16_t* out_bf16, const int* deps, int ndeps,
                    int* op_out) {
  kb::clear_error();
  StepProgram* pr = reinterpret_cast<StepProgram*>(step);
  KB_REQUIRE(pr && state && q && k && v && decay && beta && op_out && (out || out_bf16),
             KB_ERR_NULL_POINTER, "NULL argument");
  KB_REQUIRE(!pr->finalized, KB_ERR_UNSUPPORTED, "program already finalized");
  KB_REQUIRE(B >= 1 && H >= 1 && Dk >= 1 && Dk <= 128 && Dv >= 1 && Dv <= 4096,
             KB_ERR_UNSUPPORTED, "step KDA supports Dk <= 128, Dv <= 4096");
  KB_REQUIRE(sk >= Dv && sh >= Dk * sk && sb >= H * sh, KB_ERR_BAD_SHAPE,
             "state strides overlap rows");
  kb::StOp op = {};
  op.type = kb::OP_KDA;
  op.T = pr->T;
  int rc = kb::check_deps(pr, deps, ndeps, op);
  if (rc) return rc;
  op.state = state;
  op.sb = sb;
  op.sh = sh;
  op.sk = sk;
  op.q = q;
  op.k = k;
  op.v = v;
  op.decay = decay;
  op.beta = beta;
  op.B = (int)B;
  op.H = (int)H;
  op.Dk = (int)Dk;
  op.Dv = (int)Dv;
  op.scale = scale;
  op.kout = out;
  op.kout_bf16 = out_bf16;
  op.items = (int)(B * H * ((Dv + kb::ST_KDA_COLS - 1) / kb::ST_KDA_COLS));
  op.target = op.items;
  op.done = kb::add_sync(pr, 1);
  *op_out = (int)pr->ops.size();
  pr->ops.push_back(op);
  return KB_OK;
}

int kb_step_finalize(kb_step* step) {
  kb::clear_error();
  StepProgram* pr = reinterpret_cast<StepProgram*>(step);
  KB_REQUIRE(pr, KB_ERR_NULL_POINTER, "step is NULL");
  KB_REQUIRE(!pr->finalized, KB_ERR_UNSUPPORTED, "program already finalized");
  KB_REQUIRE(!pr->ops.empty(), KB_ERR_BAD_SHAPE, "empty program");
  int dev = 0;
  KB_REQUIRE(cudaGetDevice(&dev) == cudaSuccess, KB_ERR_DEVICE, "no current CUDA device");
  const int G = kb::num_sms(dev);
  KB_REQUIRE(G > 0, KB_ERR_DEVICE, "cannot query the SM count");
  const int T = pr->T;
  // Rotations and the largest stage and activation regions.
  int stage = 0, xbytes = 0, cum = 0, drow = 0;
  std::vector<std::pair<uint32_t**, size_t>> tag_fields;
  size_t tag_words = 0;
  for (size_t o = 0; o < pr->ops.size(); ++o) {
    kb::StOp& op = pr->ops[o];
    // Inputs produced by the operation just before are staged by the
    // consumers (they wait for them in any case); others by the stager,
    // ahead of the consumers.
    op.cstage = 0;
    op.comb_src = -1;
    if (op.type == kb::OP_DENSE || op.type == kb::OP_ROUTER)
      for (int d = 0; d < op.ndeps; ++d) op.cstage |= (op.dep[d] == (int)o - 1);
    // An activation row that is the combine output of the down operation just
    // before is computed from its per-route outputs by the consumers.
    if (op.type == kb::OP_DENSE && op.cstage && o > 0 &&
        pr->ops[o - 1].type == kb::OP_MOE_DOWN) {
      const kb::StOp& dop = pr->ops[o - 1];
      for (int i = 0; i < op.nprob; ++i) {
        kb::StDense& D = op.p[i];
        D.xcomb = D.nchunk == 1 && D.x == dop.out && D.xs == dop.N && D.K == dop.N &&
                  dop.R - 1 <= kb::ST_MAX_TOPK;
        if (D.xcomb) op.comb_src = (int)o - 1;
      }
    }
    kb::plan_tags(pr, o, tag_fields, tag_words);
    switch (op.type) {
      case kb::OP_DENSE: {
        op.rot = cum % G;
        cum += op.items;
        int xb = 0;
        for (int i = 0; i < op.nprob; ++i) {
          const kb::StDense& D = op.p[i];
          const int ng = D.K >> (5 + D.gshift);
          const int sb = (D.nchunk > 1) ? D.RBc * 16 * (D.K / (2 * D.nchunk))
                                        : kb::item_stage_bytes(D.K, D.mats, D.RBc, ng);
          stage = std::max(stage, sb);
          xb = std::max(xb, (D.nchunk > 1) ? T * kb::token_stride(D.K / D.nchunk)
                                           : D.x_off + T * kb::token_stride(D.K));
        }
        xbytes = std::max(xbytes, xb);
        break;
      }
      case kb::OP_ROUTER:
        op.rot = cum % G;
        cum += op.items;
        stage = std::max(stage, kb::ST_RT_EXPERTS * op.K * 2);
        xbytes = std::max(xbytes, T * op.K * 2);
        break;
      case kb::OP_MOE_UP:
      case kb::OP_MOE_DOWN: {
        const int mats = op.type == kb::OP_MOE_UP ? 2 : 1;
        stage = std::max(stage,
                         kb::item_stage_bytes(op.K, mats, op.RBc, op.K >> (5 + op.gshift)));
        xbytes = std::max(xbytes, T * kb::token_stride(op.K));
        if (op.type == kb::OP_MOE_DOWN) drow = std::max(drow, T * kb::token_stride(op.K));
        break;
      }
      case kb::OP_KDA:
        op.rot = cum % G;
        cum += op.items;
        break;
    }
  }
  stage = (stage + 127) / 128 * 128;
  const int exit_idx = kb::add_sync(pr, 1);
  const int abort_idx = kb::add_sync(pr, 1);
  const int parity_idx = kb::add_sync(pr, 1);
  kb::StepParams& P = pr->params;
  P = {};
  P.nops = (int)pr->ops.size();
  P.nsync = pr->nsync;
  P.exit_idx = exit_idx;
  P.abort_idx = abort_idx;
  P.parity_idx = parity_idx;
  P.stage_bytes = stage;
  P.T = T;
  const int scr = (int)(sizeof(kb::StPlan) + sizeof(kb::StKda) + 127) / 128 * 128;
  // Layout: nxb activation buffers, nxb descriptor copies, ST_NB partial-sum
  // buffers (NCW x 16 rows x T fp32 each), scratch, then the ring.  Two
  // activation buffers (the stager works one operation ahead) when at least
  // three ring stages remain, else one.
  P.part_bytes = kb::ST_NB * kb::NCW * 16 * T * (int)sizeof(float);
  P.x_bytes = (xbytes + 127) / 128 * 128;
  // Down inputs: as many item buffers as fit in one activation buffer.
  P.drow_bytes = std::max(128, (drow + 127) / 128 * 128);
  P.dnb = std::max(1, std::min(kb::ST_DNB, P.x_bytes / P.drow_bytes));
  const int desc_bytes = ((int)sizeof(kb::StOp) + 127) / 128 * 128;
  const int nbar = 2 + 2 * kb::ST_NB + 6 + 2 * kb::ST_DNB;  // plan, ack, partial done/free,
                                                           // x ready/free/desc, down ready/free
  for (int nxb = 2; nxb >= 1; --nxb) {
    P.nxb = nxb;
    P.desc_off = nxb * P.x_bytes;
    P.red_off = P.desc_off + nxb * desc_bytes;
    P.scr_off = P.red_off + (P.part_bytes + 127) / 128 * 128;
    P.ring_off = P.scr_off + scr;
    const int room = kb::MAX_SMEM - P.ring_off - nbar * 8 - 256;
    P.stages = std::min(16, room / std::max(stage + 16, 1));
    if (P.stages >= 3) break;
  }
  KB_REQUIRE(P.stages >= 2, KB_ERR_UNSUPPORTED,
             "shared memory: %d bytes of fixed regions leave room for %d stages of %d bytes",
             P.ring_off, P.stages, stage);
  P.bar_off = P.ring_off + P.stages * stage;
  pr->smem = (size_t)P.bar_off + (2 * P.stages + nbar) * sizeof(uint64_t);
  KB_REQUIRE(pr->smem <= (size_t)kb::MAX_SMEM, KB_ERR_UNSUPPORTED, "shared memory overflow");
  P.err = kb::device_error_word(dev);
  KB_REQUIRE(P.err, KB_ERR_DEVICE, "device error word unavailable");
  cudaError_t e = cudaMalloc(&pr->d_ops, pr->ops.size() * sizeof(kb::StOp));
  if (e == cudaSuccess) e = cudaMalloc(&pr->d_sync, (size_t)pr->nsync * sizeof(int));
  // Tagged copies start zeroed (tag 0 is never a first launch's tag).
  if (e == cudaSuccess && tag_words > 0) {
    e = cudaMalloc(&pr->d_tags, tag_words * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemset(pr->d_tags, 0, tag_words * sizeof(uint32_t));
    if (e == cudaSuccess)
      for (const auto& f : tag_fields) *f.first = pr->d_tags + f.second;
  }
  if (e == cudaSuccess)
    e = cudaMemcpy(pr->d_ops, pr->ops.data(), pr->ops.size() * sizeof(kb::StOp),
                   cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemset(pr->d_sync, 0, (size_t)pr->nsync * sizeof(int));
  // Router words: zero means "not written"; each launch clears the other
  // launch parity's words for the next.
  for (size_t o = 0; o < pr->ops.size() && e == cudaSuccess; ++o)
    if (pr->ops[o].type == kb::OP_ROUTER)
      e = cudaMemset(pr->ops[o].rwords, 0, (size_t)2 * T * pr->ops[o].E * sizeof(uint64_t));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(kb::step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kb::MAX_SMEM);
  KB_REQUIRE(e == cudaSuccess, KB_ERR_DEVICE, "step program upload failed: %s",
             cudaGetErrorString(e));
  P.ops = pr->d_ops;
  P.sync = pr->d_sync;
  pr->grid = G;
  pr->device = dev;
  pr->finalized = true;
  return KB_OK;
}

int kb_step_launch(kb_step* step, void* stream) {
  kb::clear_error();
  StepProgram* pr = reinterpret_cast<StepProgram*>(step);
  KB_REQUIRE(pr, KB_ERR_NULL_POINTER, "step is NULL");
  KB_REQUIRE(pr->finalized, KB_ERR_UNSUPPORTED, "program not finalized");
  int dev = -1;
  cudaGetDevice(&dev);
  KB_REQUIRE(dev == pr->device, KB_ERR_DEVICE,
             "program was finalized on device %d, current device is %d", pr->device, dev);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pr->grid);
  cfg.blockDim = dim3(kb::ST_THREADS);
  cfg.dynamicSmemBytes = pr->smem;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kb::step_kernel, pr->params);
  KB_REQUIRE(err == cudaSuccess, KB_ERR_LAUNCH, "step launch failed: %s",
             cudaGetErrorString(err));
  return KB_OK;
}

int kb_step_set_trace(kb_step* step, int64_t* trace, int64_t entries) {
  kb::clear_error();
  StepProgram* pr = reinterpret_cast<StepProgram*>(step);
  KB_REQUIRE(pr, KB_ERR_NULL_POINTER, "step is NULL");
  KB_REQUIRE(pr->finalized, KB_ERR_UNSUPPORTED, "program not finalized");
  const int64_t need = (int64_t)pr->grid * (int64_t)pr->ops.size() * kb::ST_TRACE_FIELDS;
  KB_REQUIRE(trace == nullptr || entries >= need, KB_ERR_WORKSPACE,
             "trace needs %lld entries, got %lld", (long long)need, (long long)entries);
  pr->params.trace = reinterpret_cast<long long*>(trace);
  return KB_OK;
}

int64_t kb_step_trace_entries(const kb_step* step) {
  const StepProgram* pr = reinterpret_cast<const StepProgram*>(step);
  if (!pr || !pr->finalized) return 0;
  return (int64_t)pr->grid * (int64_t)pr->ops.size() * kb::ST_TRACE_FIELDS;
}

int kb_step_info(const kb_step* step, int* n_ops, int* stages, int* stage_bytes,
                 size_t* smem_bytes) {
  kb::clear_error();
  const StepProgram* pr = reinterpret_cast<const StepProgram*>(step);
  KB_REQUIRE(pr, KB_ERR_NULL_POINTER, "step is NULL");
  if (n_ops) *n_ops = (int)pr->ops.size();
  if (stages) *stages = pr->params.stages;
  if (stage_bytes) *stage_bytes = pr->params.stage_bytes;
  if (smem_bytes) *smem_bytes = pr->smem;
  return KB_OK;
}

}  // extern "C"
