// kb_tc.cu - W4A16 projections on the 5th-generation tensor cores (tcgen05)
// for the many-token regime: dense projections of 16+ tokens and expert
// groups of many rows (batched decode, the expert-parallel expert phase, the
// shared expert over a whole batch).
//
// Reference semantics (engine/quant/triton_w4a16.py:44-124, the tl.dot W4A16
// GEMM every M > 1 dense call falls back to via
// engine/kernels/w4a16_dense_gemv.py:327-331; grouped per (t, r) as
// engine/kernels/w4a16_grouped.py:121-194; SwiGLU contract of
// engine/kernels/__init__.py:182-197): decoded weight bf16(code * scale),
// fp32 accumulation, bf16 outputs.
//
// One persistent CTA per SM (24 warps) walks work units.  A unit is two
// 128-row weight tiles -- rows [256 rt, 256 rt + 256) of one matrix (dense and
// grouped modes) or the same 128 rows of the gate and up matrices (SwiGLU
// mode) -- times up to 64 token rows (one expert's rows in the grouped modes),
// over the reduction axis (or one split of it) in 128-wide k-chunks (each
// pipeline hand-off carries a whole chunk, so the fixed cost of the barrier
// hand-offs is paid once per 32 KB of decoded weights):
//
//   warp 0 (lane 0): TMA producer.  Packed codes of both tiles, one 2-D tiled
//     bulk tensor copy of 128 rows x 64 bytes per tile and k-chunk (64-byte
//     swizzle, plain, no multicast, L2 evict-first), into a ring of SW
//     shared-memory stages; the unit's bf16 scales (rows contiguous) with one
//     bulk copy per tile into a double buffer.
//   warp 1: activation loader.  Dense mode: two 2-D tensor copies per chunk
//     (lane 0).  Grouped modes: 16-byte cp.async pieces of the unit's token
//     rows gathered through the expert plan.  Both write the
//     128-byte-swizzled K-major layout the tensor core reads as its B operand
//     (two 64-element halves per chunk), into a ring of SX stages.
//   warps 8-23: decoders, four per TMEM lane quarter (a warp reaches only the
//     32 lanes of its quarter).  A thread turns 32 packed bytes of its row into
//     64 weights bf16(code * scale) in k order (17 instructions per 8 weights:
//     one shift, four byte permutes, four LOP3s, four exact bf16x2
//     subtractions and four bf16x2 multiplies -- the one rounding of the
//     reference) and writes them with two tcgen05.st into a ring of two or
//     three decoded-weight stages held in tensor memory.
//   warps 2 and 3 (lane 0): MMA issuers, one per tile (a tcgen05.mma costs
//     its issuing thread ~110 cycles at these shapes, measured, so one thread
//     cannot keep the tensor core busy).  Per k-chunk, eight tcgen05.mma with
//     A (the decoded weights) read from TMEM and B (the activations) from
//     shared memory: M 128, N = tokens rounded up to 16, K 16, bf16 x bf16 ->
//     fp32 into the tile's TMEM accumulator; each issuer's tcgen05.commit
//     frees its share of each stage and, after the unit's last chunk,
//     publishes its accumulator (two accumulator buffers, so the next unit's
//     products overlap this unit's epilogue).
//   warps 4-7: epilogue.  tcgen05.ld of their 32 TMEM lanes (one weight row per
//     thread), bf16 rounding (or the SwiGLU contract of the gate/up pair) and
//     stores to the output rows; with a split reduction axis, fp32 partials to
//     the workspace and the last CTA of the tile sums them in split order.
//
// The decoded weights never pass through shared memory: keeping them in TMEM
// spares the 4 bytes of shared-memory traffic per weight (decoder store plus
// tensor-core read) that made the shared-memory form bandwidth-bound.
//
// Every wait is bounded (2 s); a timeout sets device error bit 1 and a shared
// abort flag, the roles leave their loops, the bulk copies and tensor-core
// operations already issued are waited for (bounded), and the TMEM is freed.
#include "kb_engine.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

namespace kb {
namespace tc {

constexpr int BM = 128;                 // weight rows per tile (MMA M)
constexpr int KC = 128;                 // reduction elements per chunk (two 128-byte swizzle rows)
constexpr int W_TILE = BM * KC / 2;     // packed bytes per tile and chunk (64 per row)
constexpr int A_COLS = KC / 2;          // TMEM columns of one decoded tile chunk (bf16 pairs)
constexpr int NT_MAX = 64;              // token rows per unit with two accumulator buffers
constexpr int NT_DENSE_MAX = 128;       // dense units of more rows: one accumulator buffer
constexpr int TMEM_COLS = 512;          // accumulators [2 buffers][2 tiles][NT], then the A ring
constexpr int SA_MAX = 3;               // decoded-weight stages in TMEM (2 at NT 64, 3 at NT 32)
constexpr int W_WARP = 0;
constexpr int X_WARP0 = 1;              // activation loaders (warps 1 and 3)
constexpr int MMA_WARP = 2;             // MMA issuer of tile 0
constexpr int X_WARP1 = 3;              // also allocates the TMEM
constexpr int EPI_WARP0 = 4;            // warps 4..7: TMEM lane quarters 0..3
constexpr int DEC_WARP0 = 8;
constexpr int NDEC_WARPS = 16;
constexpr int NWARPS = DEC_WARP0 + NDEC_WARPS;
constexpr int NTHREADS = NWARPS * 32;
constexpr int NXTHREADS = 32;
constexpr int NISSUERS = 2;             // MMA-issuing threads (one per tile)
constexpr int MAX_SMEM = 226 * 1024;   // dynamic; the static plan counters take a few bytes
constexpr int MAX_SX = 12;
constexpr int MAX_SW = 16;
constexpr int MAX_ASSIGN = 4096;        // grouped modes: T * R
constexpr int MAX_SLOTS = 520;          // grouped modes: experts in the bank
constexpr int MAX_SPLITS = 4;           // reduction-axis splits per tile
constexpr int MAX_RED = 16;             // split tiles one CTA may finish (deferred reductions)
constexpr long long WAIT_NS = 2000000000LL;
constexpr long long DRAIN_NS = 200000000LL;

enum Mode : int { DENSE = 0, GROUPED = 1, SWIGLU = 2 };

struct Args {
  int mode;
  const uint16_t* x;
  int64_t xs;             // activation row stride (elements)
  const int64_t* idx;     // grouped: [T, R]
  int T, R;               // dense: T tokens, R = 1
  int K, N, E, gshift, ng;
  const uint16_t* s0;     // scales of tile-0 matrices (bank base)
  const uint16_t* s1;     // SwiGLU: scales of the up matrices
  int64_t sse;            // scale elements per expert (N * ng)
  uint16_t* y;
  int64_t ys;             // output row stride (elements)
  int n_rt;               // row tiles per matrix
  int nt;                 // token rows per unit (MMA N bound, multiple of 16)
  int sx, sw;             // ring stages: activations, packed weights
  int off_x, off_w, off_sc, off_plan, off_bar;
  int splits;             // reduction-axis splits per tile (1: no split)
  float* ws;              // splits > 1: fp32 partials [tile][split][2][NT][BM]
  int* counters;          // splits > 1: arrival counter per tile (zero between launches)
  int x_tma;              // dense: activations by tensor copies of the map tmx
  int sa, a_base;         // decoded-weight stages in TMEM and the first column of their ring
  int nbuf;               // accumulator buffers (2: a unit's epilogue overlaps the next unit)
  uint32_t* err;
};

struct Unit {
  int e, rt, tok0, nt;
  int tile, ks, s0, s1;   // split-K: tile id, split index, k-chunk range [s0, s1)
  int rot;                // first k-chunk visited, relative to s0
};

// The k-chunks of a unit are visited from a starting point that differs from
// unit to unit (a fixed function of the unit), so that CTAs working at the
// same time read different activation lines instead of all requesting the
// same few L2 lines at once.  The order is a property of the unit, so every
// result is still the same run to run.
__device__ __forceinline__ int chunk_of(const Unit& U, int si) {
  const int n = U.s1 - U.s0;
  int c = U.rot + si;
  if (c >= n) c -= n;
  return U.s0 + c;
}

__device__ __forceinline__ long long now_ns() {
  long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait on a barrier phase; false on timeout (recorded) or abort.
// try_wait with a suspend-time hint: a waiting thread sleeps in hardware until
// the phase completes (or the hint runs out) instead of polling, so waiters
// take no issue slots or shared-memory bandwidth from the working warps.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// Bounded wait: suspends up to 0.5 ms per try, then checks the abort flag
// and the 2 s limit.
__device__ __forceinline__ bool wait_phase(uint64_t* bar, uint32_t parity, volatile int* abort_f,
                                           uint32_t* err, long long limit = WAIT_NS) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = now_ns();
  while (true) {
    if (mbar_wait_sleep(bar, parity, 500000u)) return true;
    if (*abort_f) return false;
    if (now_ns() - t0 > limit) {
      *abort_f = 1;
      atomicOr(err, ERR_TIMEOUT);
      return false;
    }
  }
}

// Drain wait (error path): no abort check, short limit, no error recorded.
__device__ __forceinline__ void drain_phase(uint64_t* bar, uint32_t parity) {
  const long long t0 = now_ns();
  while (!mbar_try_wait(bar, parity))
    if (now_ns() - t0 > DRAIN_NS) return;
}

// ---------------------------------------------------------------------------
// tcgen05 / TMA primitives (inline PTX).
// ---------------------------------------------------------------------------

// Shared-memory matrix descriptor: K-major operand in the 128-byte swizzle
// layout (8-row groups 1024 bytes apart), sm_100 descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;                 // leading byte offset (unused when K fits the swizzle row)
  d |= (uint64_t)(1024 >> 4) << 32;       // stride byte offset: next 8-row group
  d |= (uint64_t)1 << 46;                 // descriptor version
  d |= (uint64_t)2 << 61;                 // 128-byte swizzle
  return d;
}

// Instruction descriptor: bf16 A and B (K-major), fp32 D, M = 128, N = n.
__device__ __forceinline__ uint32_t idesc_bf16(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                     uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// A from tensor memory (lane = row, column = a pair of bf16 along K), B from
// shared memory.
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
        "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16};"
      ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]),
        "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]),
        "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;"
      ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y),
        "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src)
               : "memory");
}

// Arrive on `bar` once every cp.async this thread issued so far has landed;
// the arrival counts against the barrier's expected count (noinc).
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Shared-memory loads by 32-bit shared address (ordered after the barrier
// waits like the other volatile instructions).
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(a));
  return v;
}

__device__ __forceinline__ uint32_t ld_shared_u16(uint32_t a) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return v;
}

// Byte offset of 16-byte chunk c of row r in a 128-byte-swizzled K-major tile.
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + (((c ^ r) & 7) << 4));
}

// Decode one word of 8 codes (reduction indices 8w..8w+7, even index in the
// low nibble of each byte) into four bf16x2 words in k order:
// (k0,k1), (k2,k3), (k4,k5), (k6,k7), each bf16(code * scale).  The two
// nibbles of byte i land in the low and high halves through one byte
// permute; XOR with 8 and the exponent of 128 make each half 136 + code
// exactly; the exact subtraction of 136 and one multiply by the scale follow
// the reference's single rounding.
__device__ __forceinline__ uint4 decode_word_ordered(uint32_t q, uint32_t scale2) {
  const uint32_t s4 = q >> 4;
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t sel = (uint32_t)i | ((uint32_t)i << 4) | ((uint32_t)(4 + i) << 8) |
                         ((uint32_t)(4 + i) << 12);
    const uint32_t t = prmt(q, s4, sel);
    const uint32_t v = lop3_and_xor(t, 0x000F000Fu, 0x43084308u);
    o[i] = bf2_mul(bf2_fma(v, BF2_ONE, BF2_M136), scale2);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Position in a ring of n stages: the stage, the parity of its current use
// and whether this is the first pass (no earlier use to wait for).  Kept as
// running counters so that no loop divides by a runtime ring depth.
struct Ring {
  int st, n;
  uint32_t ph;
  bool first;
  __device__ __forceinline__ explicit Ring(int n_) : st(0), n(n_), ph(0), first(true) {}
  __device__ __forceinline__ void next() {
    if (++st == n) {
      st = 0;
      ph ^= 1u;
      first = false;
    }
  }
};

// ---------------------------------------------------------------------------
// Work units and the expert plan.
// ---------------------------------------------------------------------------
struct Plan {
  int* slot_expert;   // [nslots]
  int* slot_start;    // [nslots + 1]
  int* unit_prefix;   // [nslots + 1]
  int* assign;        // [T * R], assignments grouped by expert
  int nslots;
  int units;
};

__device__ __forceinline__ int tile_row(const Args& A, int rt, int m) {
  return A.mode == SWIGLU ? rt * BM : rt * 2 * BM + m * BM;
}

__device__ __forceinline__ int valid_rows(const Args& A, int rt, int m) {
  return max(0, min(BM, A.N - tile_row(A, rt, m)));
}

__device__ __forceinline__ Unit unit_of(const Args& A, const Plan& P, int uu) {
  Unit U;
  U.tile = uu / A.splits;
  U.ks = uu - U.tile * A.splits;
  const int KS = A.K / KC;
  U.s0 = U.ks * KS / A.splits;
  U.s1 = (U.ks + 1) * KS / A.splits;
  U.rot = (int)(((unsigned)uu * 7u) % (unsigned)(U.s1 - U.s0));
  const int u = U.tile;
  if (A.mode == DENSE) {
    const int nb = (A.T + A.nt - 1) / A.nt;
    U.e = 0;
    U.rt = u / nb;
    const int b = u - U.rt * nb;
    U.tok0 = b * A.nt;
    U.nt = min(A.nt, A.T - U.tok0);
    return U;
  }
  int lo = 0, hi = P.nslots - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (P.unit_prefix[mid] <= u) lo = mid; else hi = mid - 1;
  }
  const int j = lo;
  const int cnt = P.slot_start[j + 1] - P.slot_start[j];
  const int nb = (cnt + A.nt - 1) / A.nt;
  const int v = u - P.unit_prefix[j];
  U.e = P.slot_expert[j];
  U.rt = v / nb;
  const int b = v - U.rt * nb;
  U.tok0 = P.slot_start[j] + b * A.nt;
  U.nt = min(A.nt, P.slot_start[j + 1] - U.tok0);
  return U;
}

// Source activation row and destination output row of slot i of a unit.
__device__ __forceinline__ void rows_of(const Args& A, const Plan& P, const Unit& U, int i,
                                        int& xrow, int& yrow) {
  if (A.mode == DENSE) {
    xrow = yrow = U.tok0 + i;
  } else {
    const int a = P.assign[U.tok0 + i];
    xrow = a / A.R;
    yrow = a;
  }
}

// Expert-major plan of the grouped modes, built by all threads of the CTA.
// Every CTA builds the same plan (the token blocks of an expert with more
// rows than one unit takes must be the same rows in every CTA): assignments
// of an expert in ascending order.  The expert ids are staged in shared
// memory once; PLAN_WARPS warps then each take a contiguous segment of the
// assignments, count it per expert, and -- after a scan over experts and over
// the warps -- scatter it, each warp's segment after the earlier warps'.
constexpr int PLAN_WARPS = 8;

// Ints of shared memory the plan takes for E experts and TR assignments.
__host__ __device__ constexpr int plan_ints_for(int E, int TR) {
  return 4 * E + 2 + TR + (TR + 1) / 2 + (PLAN_WARPS * E + 1) / 2;
}

__device__ void build_plan(const Args& A, int* cnt, Plan& P) {
  __shared__ int s_nslots, s_units;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int TR = A.T * A.R;
  const int E = A.E;
  int16_t* eid = reinterpret_cast<int16_t*>(P.assign + TR);      // [TR]
  int16_t* wcnt = eid + ((TR + 1) & ~1);                         // [PLAN_WARPS][E]
  const int seg = ((TR + PLAN_WARPS - 1) / PLAN_WARPS + 31) & ~31;
  for (int a = tid; a < TR; a += NTHREADS) {
    const int64_t v = A.idx[a];
    eid[a] = (int16_t)(v == EXPERT_NONE ? -1 : clamp_expert(v, E, A.err));
  }
  for (int i = tid; i < PLAN_WARPS * E; i += NTHREADS) wcnt[i] = 0;
  __syncthreads();
  // Per-warp counts of each expert over the warp's segment.
  if (warp < PLAN_WARPS) {
    int16_t* wc = wcnt + warp * E;
    const int a_end = min(TR, (warp + 1) * seg);
    for (int base = warp * seg; base < a_end; base += 32) {
      const int a = base + lane;
      const int e = a < a_end ? (int)eid[a] : -1;
      const unsigned peers = __match_any_sync(0xffffffffu, e < 0 ? -1 - lane : e);
      if (e >= 0 && lane == __ffs(peers) - 1) wc[e] = (int16_t)(wc[e] + __popc(peers));
      __syncwarp();
    }
  }
  __syncthreads();
  // Expert totals; each warp's count becomes its offset within the expert.
  for (int e = tid; e < E; e += NTHREADS) {
    int run = 0;
    for (int w = 0; w < PLAN_WARPS; ++w) {
      const int c = wcnt[w * E + e];
      wcnt[w * E + e] = (int16_t)run;
      run += c;
    }
    cnt[e] = run;
  }
  __syncthreads();
  if (tid < 32) {
    const int per = (E + 31) / 32;
    const int e0 = min(E, lane * per), e1 = min(E, e0 + per);
    int tot = 0, used = 0, un = 0;
    for (int e = e0; e < e1; ++e) {
      const int c = cnt[e];
      tot += c;
      used += (c > 0);
      un += ((c + A.nt - 1) / A.nt) * A.n_rt;
    }
    int it = tot, iu = used, iun = un;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int a = __shfl_up_sync(0xffffffffu, it, o);
      const int b = __shfl_up_sync(0xffffffffu, iu, o);
      const int c = __shfl_up_sync(0xffffffffu, iun, o);
      if (lane >= o) {
        it += a;
        iu += b;
        iun += c;
      }
    }
    int run = it - tot, rank = iu - used, urun = iun - un;
    for (int e = e0; e < e1; ++e) {
      const int c = cnt[e];
      if (c > 0) {
        P.slot_expert[rank] = e;
        P.slot_start[rank] = run;
        P.unit_prefix[rank] = urun;
        ++rank;
        urun += ((c + A.nt - 1) / A.nt) * A.n_rt;
      }
      cnt[e] = run;  // the expert's first position
      run += c;
    }
    if (lane == 31) {
      P.slot_start[iu] = it;
      P.unit_prefix[iu] = iun;
      s_nslots = iu;
      s_units = iun;
    }
  }
  __syncthreads();
  // Stable scatter: position = expert start + earlier warps' count + this
  // warp's running count + the lane's rank among equal experts of the chunk.
  if (warp < PLAN_WARPS) {
    int16_t* wc = wcnt + warp * E;
    const int a_end = min(TR, (warp + 1) * seg);
    for (int base = warp * seg; base < a_end; base += 32) {
      const int a = base + lane;
      const int e = a < a_end ? (int)eid[a] : -1;
      const unsigned peers = __match_any_sync(0xffffffffu, e < 0 ? -1 - lane : e);
      if (e >= 0) {
        P.assign[cnt[e] + wc[e] + __popc(peers & ((1u << lane) - 1u))] = a;
      }
      __syncwarp();
      if (e >= 0 && lane == __ffs(peers) - 1) wc[e] = (int16_t)(wc[e] + __popc(peers));
      __syncwarp();
    }
  }
  P.nslots = s_nslots;
  P.units = s_units;
  __syncthreads();
}

// ---------------------------------------------------------------------------
// The kernel.
// ---------------------------------------------------------------------------
struct Bars {
  uint64_t w_full[MAX_SW], w_empty[MAX_SW];
  uint64_t a_full[SA_MAX], a_empty[SA_MAX];
  uint64_t x_full[MAX_SX], x_empty[MAX_SX];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t sc_full[2], sc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  int epi_last;
  // Split tiles whose last partial this CTA wrote: reduced by all threads at
  // the end of the kernel.
  int red_n;
  int red_unit[MAX_RED];
  int xoff[NT_MAX];       // grouped modes: the current unit's activation row offsets
};

// Deferred split-K reduction (dense mode): for each split tile this CTA
// finished last, every thread sums 16-byte pieces (four rows of one token of
// one tile) over the splits in split order -- the same additions, in the same
// order, as a per-row sum -- and stores four bf16 outputs; then the tile's
// arrival counter is reset for the next launch.
__device__ __forceinline__ void reduce_splits(const Args& A, const Plan& P, Bars* B) {
  const int NT = A.nt;
  for (int li = 0; li < B->red_n; ++li) {
    const Unit U = unit_of(A, P, B->red_unit[li]);
    __threadfence();
    const int items = 2 * U.nt * (BM / 4);
    const size_t split_stride = (size_t)2 * NT * BM;
    const float* base = A.ws + (size_t)U.tile * A.splits * split_stride;
    for (int e0 = threadIdx.x; e0 < items; e0 += 2 * NTHREADS) {
      float4 p[2][MAX_SPLITS];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int e = min(e0 + i * NTHREADS, items - 1);
        const int m = e / (U.nt * (BM / 4));
        const int rem = e - m * U.nt * (BM / 4);
        const int j = rem / (BM / 4), r4 = rem - j * (BM / 4);
        const float* src = base + (size_t)m * NT * BM + (size_t)j * BM + r4 * 4;
#pragma unroll
        for (int k = 0; k < MAX_SPLITS; ++k)
          p[i][k] = k < A.splits ? __ldcg(reinterpret_cast<const float4*>(src + k * split_stride))
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int e = e0 + i * NTHREADS;
        if (e >= items) break;
        const int m = e / (U.nt * (BM / 4));
        const int rem = e - m * U.nt * (BM / 4);
        const int j = rem / (BM / 4), r4 = rem - j * (BM / 4);
        float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < MAX_SPLITS; ++k) {
          if (k < A.splits) {
            t.x += p[i][k].x;
            t.y += p[i][k].y;
            t.z += p[i][k].z;
            t.w += p[i][k].w;
          }
        }
        const int row = tile_row(A, U.rt, m) + r4 * 4;
        uint16_t* y = A.y + (size_t)(U.tok0 + j) * A.ys + row;
        const float v[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (row + c < A.N) y[c] = float_to_bf16_bits(v[c]);
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) A.counters[U.tile] = 0;
  }
}

__global__ void __launch_bounds__(NTHREADS, 1)
    tc_kernel(const __grid_constant__ CUtensorMap tm0, const __grid_constant__ CUtensorMap tm1,
              const __grid_constant__ CUtensorMap tmx, const Args A) {
  extern __shared__ uint8_t smem_raw[];
  // Aligned to 1024 bytes by pointer arithmetic on the shared array, so the
  // compiler keeps the shared state space and emits shared-memory loads and
  // stores (not generic ones) for everything placed in it.
  uint8_t* smem =
      smem_raw + ((1024u - (static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw)) & 1023u)) &
                  1023u);
  Bars* B = reinterpret_cast<Bars*>(smem + A.off_bar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NT = A.nt;
  const uint32_t tmem_cols = (uint32_t)TMEM_COLS;
  volatile int* abort_f = &B->abort_flag;

  if (threadIdx.x == 0) {
    for (int i = 0; i < A.sw; ++i) {
      mbar_init(&B->w_full[i], 1);
      mbar_init(&B->w_empty[i], NDEC_WARPS);
    }
    for (int i = 0; i < A.sa; ++i) {
      mbar_init(&B->a_full[i], NDEC_WARPS);
      mbar_init(&B->a_empty[i], NISSUERS);
    }
    for (int i = 0; i < A.sx; ++i) {
      mbar_init(&B->x_full[i], A.x_tma ? 1 : NXTHREADS);
      mbar_init(&B->x_empty[i], NISSUERS);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B->acc_full[i], NISSUERS);
      mbar_init(&B->acc_empty[i], 4);
      mbar_init(&B->sc_full[i], 1);
      mbar_init(&B->sc_empty[i], NDEC_WARPS);
    }
    mbar_init(&B->drain, NISSUERS);
    B->abort_flag = 0;
    B->red_n = 0;
    mbar_fence_init();
  }
  if (warp == X_WARP1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_addr(&B->tmem_base)), "r"(tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = B->tmem_base;

  pdl_wait();
  pdl_launch_dependents();

  Plan P;
  P.nslots = 0;
  P.units = 0;
  if (A.mode != DENSE) {
    int* base = reinterpret_cast<int*>(smem + A.off_plan);
    int* cnt = base;
    P.slot_expert = cnt + A.E;
    P.slot_start = P.slot_expert + A.E;
    P.unit_prefix = P.slot_start + A.E + 1;
    P.assign = P.unit_prefix + A.E + 1;
    build_plan(A, cnt, P);
  } else {
    P.units = A.n_rt * ((A.T + NT - 1) / NT);
  }
  P.units *= A.splits;
  const int units = P.units;
  uint8_t* ring_x = smem + A.off_x;                 // [sx][2][NT * 128]
  uint8_t* ring_w = smem + A.off_w;                 // [sw][2][W_TILE]
  const int x_stage = NT * KC * 2;                  // bytes of one activation stage
  uint16_t* scl = reinterpret_cast<uint16_t*>(smem + A.off_sc);  // [2][2][BM * ng]
  const int ng = A.ng;

  if (warp == W_WARP) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      int it = 0, uc = 0;
      Ring wr(A.sw);
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++uc) {
        const Unit U = unit_of(A, P, u);
        const int sb = uc & 1;
        if (uc >= 2 && !wait_phase(&B->sc_empty[sb], ((uc >> 1) - 1) & 1, abort_f, A.err)) {
          ok = false;
          break;
        }
        uint32_t bytes = 0;
        int vr[2];
        for (int m = 0; m < 2; ++m) {
          vr[m] = valid_rows(A, U.rt, m);
          bytes += (uint32_t)(vr[m] * ng * 2);
        }
        mbar_arrive_expect_tx(&B->sc_full[sb], bytes);
        for (int m = 0; m < 2; ++m) {
          if (vr[m] == 0) continue;
          const uint16_t* src = ((A.mode == SWIGLU && m == 1) ? A.s1 : A.s0) +
                                (size_t)U.e * (size_t)A.sse +
                                (size_t)tile_row(A, U.rt, m) * ng;
          bulk_g2s(scl + (size_t)(sb * 2 + m) * BM * ng, src, (uint32_t)(vr[m] * ng * 2),
                   &B->sc_full[sb], pol);
        }
        const int row0 = U.e * A.N + tile_row(A, U.rt, 0);
        const int row1 = U.e * A.N + tile_row(A, U.rt, 1);
        const CUtensorMap* map1 = (A.mode == SWIGLU) ? &tm1 : &tm0;
        for (int si = 0; si < U.s1 - U.s0; ++si, ++it, wr.next()) {
          const int s = chunk_of(U, si);
          if (!wr.first && !wait_phase(&B->w_empty[wr.st], wr.ph ^ 1u, abort_f, A.err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&B->w_full[wr.st], 2 * W_TILE);
          tma_load_2d(ring_w + (size_t)(wr.st * 2) * W_TILE, &tm0, s * (KC / 2), row0,
                      &B->w_full[wr.st], pol);
          tma_load_2d(ring_w + (size_t)(wr.st * 2 + 1) * W_TILE, map1, s * (KC / 2), row1,
                      &B->w_full[wr.st], pol);
        }
      }
      // Copies still in flight land before the CTA may exit.
      const int first = max(0, it - A.sw);
      for (int i = first; i < it; ++i) drain_phase(&B->w_full[i % A.sw], (i / A.sw) & 1);
      for (int k = max(0, uc - 2); k < uc; ++k) drain_phase(&B->sc_full[k & 1], (k >> 1) & 1);
    }
  } else if (A.x_tma && warp == X_WARP0) {
    // ------------------------------------- activation loader (dense: tensor copies)
    // Two 2-D tensor copies per k-chunk, one per 64-element half: NT token
    // rows x 128 bytes each, written by the copy engine in the 128-byte-
    // swizzled K-major layout the MMA reads (rows past the last token are
    // zero-filled).  Asynchronous-proxy writes, so the MMA issuer needs no
    // proxy fence.
    if (warp == X_WARP0 && lane == 0) {
      const uint64_t pol = l2_evict_last_policy();
      Ring xr(A.sx);
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const Unit U = unit_of(A, P, u);
        for (int si = 0; si < U.s1 - U.s0; ++si, ++it, xr.next()) {
          const int s = chunk_of(U, si);
          if (!xr.first && !wait_phase(&B->x_empty[xr.st], xr.ph ^ 1u, abort_f, A.err)) {
            ok = false;
            break;
          }
          uint8_t* dst = ring_x + (size_t)xr.st * x_stage;
          mbar_arrive_expect_tx(&B->x_full[xr.st], (uint32_t)x_stage);
          tma_load_2d(dst, &tmx, s * KC, U.tok0, &B->x_full[xr.st], pol);
          tma_load_2d(dst + NT * 128, &tmx, s * KC + KC / 2, U.tok0, &B->x_full[xr.st], pol);
        }
      }
      const int first = max(0, it - A.sx);
      for (int i = first; i < it; ++i) drain_phase(&B->x_full[i % A.sx], (i / A.sx) & 1);
    }
  } else if (!A.x_tma && warp == X_WARP0) {
    // ------------------------------------------------------ activation loader
    const int xt = lane;
    Ring xr(A.sx);
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      const Unit U = unit_of(A, P, u);
      // The unit's source rows once (the plan lookup and the division by R),
      // then every chunk's pieces read them from shared memory.
      __syncwarp();
      for (int i = lane; i < U.nt; i += 32) {
        int xrow, yrow;
        rows_of(A, P, U, i, xrow, yrow);
        B->xoff[i] = xrow * (int)A.xs;
      }
      __syncwarp();
      bool ok = true;
      for (int si = 0; si < U.s1 - U.s0; ++si, xr.next()) {
        const int s = chunk_of(U, si);
        if (!xr.first && !wait_phase(&B->x_empty[xr.st], xr.ph ^ 1u, abort_f, A.err)) {
          ok = false;
          break;
        }
        // Sixteen 16-byte pieces per token row: pieces 0-7 go to the first
        // 64-element half, 8-15 to the second, each half in the swizzled layout.
        uint8_t* dst = ring_x + (size_t)xr.st * x_stage;
        const uint16_t* xs = A.x + s * KC;
        for (int p = xt; p < U.nt * 16; p += NXTHREADS) {
          const int i = p >> 4, c = p & 15;
          cp_async16(dst + (c >> 3) * NT * 128 + sw128_off(i, c & 7), xs + B->xoff[i] + c * 8);
        }
        // The stage's arrival is made by the copies' completion (no wait here),
        // so several stages are in flight per thread.
        cp_async_arrive_noinc(&B->x_full[xr.st]);
      }
      if (!ok) break;
    }
    cp_async_wait_all();
  } else if (warp == MMA_WARP || warp == X_WARP1) {
    // ----------------------------------------------------------- MMA issuers
    // One thread per tile: a tcgen05.mma costs its issuing thread about a
    // hundred cycles whatever its size at these shapes, so two issuers with
    // their own accumulators double the rate at which the tensor core is fed.
    // Each commits its own products to the stage barriers (count two).
    // Lane 0 of warps 2 and 3: issuers in different warps issue independently
    // (lanes of one warp share its instruction stream).
    if (lane == 0) {
      const int mt = warp == MMA_WARP ? 0 : 1;
      int uc = 0;
      bool ok = true;
      Ring ar(A.sa), xr(A.sx);
      const uint64_t xdesc0 = sw128_desc(smem_addr(ring_x));
      const uint64_t xstride = (uint64_t)(x_stage >> 4);
      const uint64_t xhalf = (uint64_t)((NT * 128) >> 4);
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++uc) {
        const Unit U = unit_of(A, P, u);
        const int b = A.nbuf == 2 ? (uc & 1) : 0;
        const int use_acc = A.nbuf == 2 ? (uc >> 1) : uc;
        if (use_acc > 0 && !wait_phase(&B->acc_empty[b], (use_acc - 1) & 1, abort_f, A.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t idesc = idesc_bf16((U.nt + 15) & ~15);
        const uint32_t dm = tmem + (uint32_t)((b * 2 + mt) * NT);
        const int nks = U.s1 - U.s0;
        for (int si = 0; si < nks; ++si, ar.next(), xr.next()) {
          if (!wait_phase(&B->a_full[ar.st], ar.ph, abort_f, A.err) ||
              !wait_phase(&B->x_full[xr.st], xr.ph, abort_f, A.err)) {
            ok = false;
            break;
          }
          if (!A.x_tma) fence_proxy_async();   // cp.async (generic-proxy) writes
          tc_fence_after();
          // Descriptors and TMEM addresses of the stage, then the eight
          // k-steps of this issuer's tile with immediate offsets.  k-step kk
          // reads activation half kk / 4 at byte offset 32 (kk % 4).
          const uint64_t bd = xdesc0 + (uint64_t)xr.st * xstride;
          const uint64_t bd1 = bd + xhalf;
          const uint32_t ta =
              tmem + (uint32_t)(A.a_base + (ar.st * 2 + mt) * A_COLS);
          const uint32_t acc0 = si > 0 ? 1u : 0u;
          umma_ts(dm, ta, bd, idesc, acc0);
#pragma unroll
          for (int kk = 1; kk < 4; ++kk)
            umma_ts(dm, ta + kk * 8, bd + (uint64_t)(kk * 2), idesc, 1u);
#pragma unroll
          for (int kk = 4; kk < KC / 16; ++kk)
            umma_ts(dm, ta + kk * 8, bd1 + (uint64_t)((kk - 4) * 2), idesc, 1u);
          umma_commit(&B->a_empty[ar.st]);
          umma_commit(&B->x_empty[xr.st]);
        }
        if (ok) umma_commit(&B->acc_full[b]);
      }
      // Every product issued has completed before the TMEM is released.
      umma_commit(&B->drain);
      drain_phase(&B->drain, 0);
    }
  } else if (warp >= EPI_WARP0 && warp < EPI_WARP0 + 4) {
    // -------------------------------------------------------------- epilogue
    const int q = warp - EPI_WARP0;
    int uc = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++uc) {
      const Unit U = unit_of(A, P, u);
      const int b = A.nbuf == 2 ? (uc & 1) : 0;
      const int use_acc = A.nbuf == 2 ? (uc >> 1) : uc;
      if (!wait_phase(&B->acc_full[b], use_acc & 1, abort_f, A.err)) break;
      tc_fence_after();
      const int r = q * 32 + lane;
      const int row0 = tile_row(A, U.rt, 0), row1 = tile_row(A, U.rt, 1);
      const bool v0 = row0 + r < A.N, v1 = row1 + r < A.N;
      const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16);
      // Split units leave fp32 partials [2][NT][BM] in the workspace.
      float* part = A.splits > 1
                        ? A.ws + (size_t)(U.tile * A.splits + U.ks) * 2 * NT * BM
                        : nullptr;
      for (int c0 = 0; c0 < U.nt; c0 += 16) {
        uint32_t d0[16], d1[16];
        tmem_ld16(lane_addr + (uint32_t)((b * 2 + 0) * NT + c0), d0);
        tmem_ld16(lane_addr + (uint32_t)((b * 2 + 1) * NT + c0), d1);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (c0 + j < U.nt) {
            const float g = __uint_as_float(d0[j]), h = __uint_as_float(d1[j]);
            if (part != nullptr) {
              part[(size_t)(c0 + j) * BM + r] = g;
              part[(size_t)(NT + c0 + j) * BM + r] = h;
            } else {
              int xr, yr;
              rows_of(A, P, U, c0 + j, xr, yr);
              uint16_t* yrow = A.y + (size_t)yr * A.ys;
              if (A.mode == SWIGLU) {
                if (v0) yrow[row0 + r] = float_to_bf16_bits(swiglu_contract(g, h));
              } else {
                if (v0) yrow[row0 + r] = float_to_bf16_bits(g);
                if (v1) yrow[row1 + r] = float_to_bf16_bits(h);
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&B->acc_empty[b]);
      if (part != nullptr) {
        // The CTA that brings the tile's counter to `splits` sums the partials
        // in split order (deterministic), writes the outputs and resets the
        // counter for the next launch.
        __threadfence();
        named_barrier(1, 128);
        if (q == 0 && lane == 0) {
          const int old = atomicAdd(&A.counters[U.tile], 1);
          B->epi_last = (old == A.splits - 1);
        }
        named_barrier(1, 128);
        if (B->epi_last && q == 0 && lane == 0) {
          // The sums run after the roles finish, on all threads (more loads
          // in flight than the four epilogue warps can keep).
          if (B->red_n < MAX_RED) {
            B->red_unit[B->red_n++] = u;
          } else {
            *abort_f = 1;
            atomicOr(A.err, ERR_TIMEOUT);
          }
        }
        named_barrier(1, 128);
      }
    }
  } else if (warp >= DEC_WARP0 && warp < DEC_WARP0 + NDEC_WARPS) {
    // -------------------------------------------------------------- decoders
    // Warp w may only reach TMEM lanes 32 (w % 4) .. + 31, so the four lane
    // quarters each get four decoder warps: one per (tile, half of the
    // 128-wide chunk).  A thread decodes 64 weights of its row per chunk: the
    // two 16-byte pieces of its half of the row's 64 packed bytes, which the
    // copy engine wrote with the 64-byte swizzle (piece p of row r at
    // p ^ ((r >> 1) & 3)), so the lanes of a quarter-warp read distinct banks.
    const int dw = warp - DEC_WARP0;
    const int quarter = warp & 3;
    const int m = (dw >> 2) >> 1, h = (dw >> 2) & 1;
    const int r = quarter * 32 + lane;
    const uint32_t lane_bits = (uint32_t)(quarter * 32) << 16;
    int uc = 0;
    bool ok = true;
    Ring wr(A.sw), ar(A.sa);
    const int swz = (r >> 1) & 3;
    const uint32_t wrow = smem_addr(ring_w) + (uint32_t)(m * W_TILE + r * 64);
    const uint32_t piece0 = (uint32_t)(((2 * h) ^ swz) << 4);
    const uint32_t piece1 = (uint32_t)(((2 * h + 1) ^ swz) << 4);
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++uc) {
      const Unit U = unit_of(A, P, u);
      const int sb = uc & 1;
      if (!wait_phase(&B->sc_full[sb], (uc >> 1) & 1, abort_f, A.err)) break;
      const bool rv = r < valid_rows(A, U.rt, m);
      const uint32_t srow = smem_addr(scl + (size_t)(sb * 2 + m) * BM * ng + (size_t)r * ng);
      for (int si = 0; si < U.s1 - U.s0; ++si, wr.next(), ar.next()) {
        const int s = chunk_of(U, si);
        const int wst = wr.st, ast = ar.st;
        if (!wait_phase(&B->w_full[wst], wr.ph, abort_f, A.err) ||
            (!ar.first && !wait_phase(&B->a_empty[ast], ar.ph ^ 1u, abort_f, A.err))) {
          ok = false;
          break;
        }
        const uint32_t wsrc = wrow + (uint32_t)(wst * 2 * W_TILE);
        const uint4 qa = ld_shared_v4(wsrc + piece0);
        const uint4 qb = ld_shared_v4(wsrc + piece1);
        const int k0 = s * KC + h * 64;   // reduction index of this thread's first weight
        const uint32_t sa = rv ? ld_shared_u16(srow + 2u * (uint32_t)(k0 >> (5 + A.gshift))) : 0u;
        const uint32_t sbv =
            rv ? ld_shared_u16(srow + 2u * (uint32_t)((k0 + 32) >> (5 + A.gshift))) : 0u;
        const uint32_t col = tmem + lane_bits + (uint32_t)(A.a_base + (ast * 2 + m) * A_COLS + h * 32);
        {
          const uint32_t sc2 = sa | (sa << 16);
          const uint32_t words[4] = {qa.x, qa.y, qa.z, qa.w};
          uint32_t o[16];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint4 v = decode_word_ordered(words[i], sc2);
            o[4 * i + 0] = v.x;
            o[4 * i + 1] = v.y;
            o[4 * i + 2] = v.z;
            o[4 * i + 3] = v.w;
          }
          tmem_st16(col, o);
        }
        {
          const uint32_t sc2 = sbv | (sbv << 16);
          const uint32_t words[4] = {qb.x, qb.y, qb.z, qb.w};
          uint32_t o[16];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint4 v = decode_word_ordered(words[i], sc2);
            o[4 * i + 0] = v.x;
            o[4 * i + 1] = v.y;
            o[4 * i + 2] = v.z;
            o[4 * i + 3] = v.w;
          }
          tmem_st16(col + 16, o);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&B->w_empty[wst]);
          mbar_arrive(&B->a_full[ast]);
        }
      }
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(&B->sc_empty[sb]);
    }
  }

  __syncthreads();
  if (warp == X_WARP1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(tmem_cols)
                 : "memory");
  }
  if (B->red_n > 0) reduce_splits(A, P, B);
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
using EncodeFn = PFN_cuTensorMapEncodeTiled_v12000;

static EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  return fn;
}

// 2-D map over packed codes viewed as [rows, K/2] bytes, box 128 rows x 64
// bytes (one k-chunk of a tile), written to shared memory with the 64-byte
// swizzle.
static int make_map(CUtensorMap* map, const uint8_t* w, int64_t rows, int64_t K) {
  EncodeFn enc = encode_fn();
  KB_REQUIRE(enc != nullptr, KB_ERR_DEVICE, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)(K / 2), (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(K / 2)};
  cuuint32_t box[2] = {(cuuint32_t)(KC / 2), (cuuint32_t)BM};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(w), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  KB_REQUIRE(r == CUDA_SUCCESS, KB_ERR_DEVICE, "tensor map encoding failed (%d)", (int)r);
  return KB_OK;
}

// 2-D map over bf16 activations [T, K] (row stride xs elements), box NT rows x
// 64 elements (one 128-byte swizzle row) with the swizzle the tensor cores
// read; a k-chunk takes two copies.
static int make_x_map(CUtensorMap* map, const uint16_t* x, int64_t T, int64_t K, int64_t xs,
                      int nt) {
  EncodeFn enc = encode_fn();
  KB_REQUIRE(enc != nullptr, KB_ERR_DEVICE, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)T};
  cuuint64_t strides[1] = {(cuuint64_t)(xs * 2)};
  cuuint32_t box[2] = {(cuuint32_t)(KC / 2), (cuuint32_t)nt};   // one 64-element half
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(x), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  KB_REQUIRE(r == CUDA_SUCCESS, KB_ERR_DEVICE, "activation tensor map encoding failed (%d)",
             (int)r);
  return KB_OK;
}

static std::mutex g_attr_mu;
static bool g_attr_done[64] = {};

static int smem_limit() {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    set_error("tcgen05 GEMM: no usable current device (%s)", cudaGetErrorString(e));
    return KB_ERR_DEVICE;
  }
  std::lock_guard<std::mutex> lock(g_attr_mu);
  if (g_attr_done[dev]) return KB_OK;
  e = cudaFuncSetAttribute(tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, MAX_SMEM);
  if (e != cudaSuccess) {
    set_error("tcgen05 GEMM: setting the shared-memory limit failed: %s", cudaGetErrorString(e));
    return KB_ERR_DEVICE;
  }
  g_attr_done[dev] = true;
  return KB_OK;
}

// Shared-memory layout and ring depths for a problem; KB_ERR_UNSUPPORTED when
// the scale buffers and plan leave no room for two stages of each ring.
static int layout(Args& A, int plan_ints) {
  const int x_stage = A.nt * KC * 2;
  // TMEM: accumulators [nbuf][2 tiles][nt] columns, then the decoded-weight
  // ring (2 tiles x A_COLS columns per stage).
  A.a_base = 2 * A.nbuf * A.nt;
  A.sa = std::min(SA_MAX, (TMEM_COLS - A.a_base) / (2 * A_COLS));
  const int sc_bytes = (2 * 2 * BM * A.ng * 2 + 1023) / 1024 * 1024;
  const int plan_bytes = (plan_ints * 4 + 127) / 128 * 128;
  const int bar_bytes = (int)((sizeof(Bars) + 127) / 128 * 128);
  const int fixed = 1024 + sc_bytes + plan_bytes + bar_bytes;
  const int avail = MAX_SMEM - fixed;
  // The decoded weights live in TMEM; shared memory holds the packed-weight
  // ring (HBM latency) and the activation ring (L2 latency), grown in turn.
  int sx = 2, sw = 4;
  auto need = [&](int x, int w) { return x * x_stage + w * 2 * W_TILE; };
  KB_REQUIRE(need(sx, sw) <= avail, KB_ERR_UNSUPPORTED,
             "tcgen05 GEMM: %d scale groups per row and %d plan entries leave no room for the "
             "stage rings",
             A.ng, plan_ints);
  bool grew = true;
  while (grew) {
    grew = false;
    if (sw < MAX_SW && need(sx, sw + 1) <= avail) { ++sw; grew = true; }
    if (sx < MAX_SX && need(sx + 1, sw) <= avail) { ++sx; grew = true; }
  }
  A.sx = sx;
  A.sw = sw;
  A.off_x = 0;
  A.off_w = A.off_x + sx * x_stage;
  A.off_sc = A.off_w + sw * 2 * W_TILE;
  A.off_plan = A.off_sc + sc_bytes;
  A.off_bar = A.off_plan + plan_bytes;
  return KB_OK;
}

static int common_checks(const uint16_t* x, int64_t xs, int64_t K, int64_t N, int64_t group,
                         int* gshift) {
  const int st = check_group(K, group, gshift);
  if (st != KB_OK) return st;
  KB_REQUIRE(K % KC == 0 && K >= KC && K <= 65536, KB_ERR_UNSUPPORTED,
             "tcgen05 GEMM needs K a multiple of %d (got %lld)", KC, (long long)K);
  KB_REQUIRE(N > 0 && N % 8 == 0, KB_ERR_UNSUPPORTED,
             "tcgen05 GEMM needs N a positive multiple of 8 (got %lld)", (long long)N);
  KB_REQUIRE(aligned(x, 16) && xs % 8 == 0 && xs >= K, KB_ERR_ALIGNMENT,
             "activations must be 16-byte aligned with row stride %% 8 == 0");
  return KB_OK;
}

static int launch_tc(Args& A, const uint8_t* w0, const uint8_t* w1, int64_t rows, int units_hint,
                     void* stream) {
  int st = smem_limit();
  if (st != KB_OK) return st;
  CUtensorMap m0, m1, mx;
  st = make_map(&m0, w0, rows, A.K);
  if (st != KB_OK) return st;
  st = make_map(&m1, w1 ? w1 : w0, rows, A.K);
  if (st != KB_OK) return st;
  if (A.x_tma) {
    st = make_x_map(&mx, A.x, A.T, A.K, A.xs, A.nt);
    if (st != KB_OK) return st;
  } else {
    mx = m0;   // unused
  }
  int dev = 0;
  cudaGetDevice(&dev);
  A.err = device_error_word(dev);
  KB_REQUIRE(A.err != nullptr, KB_ERR_LAUNCH, "device error word unavailable");
  const int sms = num_sms(dev);
  const int grid = std::max(1, std::min(sms, units_hint));
  return launch(tc_kernel, dim3(grid), dim3(NTHREADS), (size_t)MAX_SMEM, stream, m0, m1, mx, A);
}

}  // namespace tc
}  // namespace kb

using kb::tc::Args;

namespace kb {
namespace tc {

constexpr int TARGET_CTAS = 148;

// Tiles of a dense problem and the reduction-axis split that brings them to
// about one CTA per SM (each split keeps at least four 128-wide k-chunks).
static void dense_split_for(int64_t M, int64_t K, int64_t N, int nt, int* tiles, int* splits) {
  const int n_rt = (int)((N + 2 * BM - 1) / (2 * BM));
  *tiles = n_rt * (int)((M + nt - 1) / nt);
  const int ks = (int)(K / KC);
  // Splitting pays only when the tiles leave most SMs idle: each split adds
  // an fp32 partial round trip through L2 and the deferred reduction.
  int sp = 1;
  if (*tiles * 3 <= TARGET_CTAS)
    sp = std::max(1, std::min(std::min(TARGET_CTAS / *tiles, MAX_SPLITS), ks / 4));
  *splits = sp;
}

// Token rows per unit and the split: all of M up to 64 (rounded to the
// MMA's 16), or 128 (each weight decoded once per 128 tokens, one
// accumulator buffer) when that lowers the most k-chunks any CTA walks (a
// split counts four chunks for its reduction).
static void dense_split(int64_t M, int64_t K, int64_t N, int* nt, int* tiles, int* splits) {
  const int ks = (int)(K / KC);
  auto cost = [&](int n, int t, int sp) {
    const int waves = (t * sp + TARGET_CTAS - 1) / TARGET_CTAS;
    return waves * ((ks + sp - 1) / sp) + (sp > 1 ? 4 : 0);
  };
  const int small = (int)std::min<int64_t>(NT_MAX, (M + 15) / 16 * 16);
  dense_split_for(M, K, N, small, tiles, splits);
  *nt = small;
  if (M > NT_MAX) {
    int t2, s2;
    dense_split_for(M, K, N, NT_DENSE_MAX, &t2, &s2);
    if (cost(NT_DENSE_MAX, t2, s2) < cost(small, *tiles, *splits)) {
      *nt = NT_DENSE_MAX;
      *tiles = t2;
      *splits = s2;
    }
  }
}

static size_t split_ws_bytes(int tiles, int splits, int nt) {
  if (splits <= 1) return 0;
  const size_t part = (size_t)tiles * splits * 2 * nt * BM * sizeof(float);
  return (part + 255) / 256 * 256 + ((size_t)tiles * sizeof(int) + 255) / 256 * 256;
}

}  // namespace tc
}  // namespace kb

extern "C" size_t kb_w4a16_dense_tc_workspace_size(int64_t M, int64_t K, int64_t N) {
  if (M <= 0 || K < kb::tc::KC || N <= 0) return 0;
  int nt, tiles, splits;
  kb::tc::dense_split(M, K, N, &nt, &tiles, &splits);
  return kb::tc::split_ws_bytes(tiles, splits, nt);
}

extern "C" int kb_w4a16_dense_tc(const uint16_t* x, int64_t x_stride, int64_t M, int64_t K,
                                 const uint8_t* packed, const uint16_t* scales, int64_t N,
                                 int64_t group, uint16_t* y, int64_t y_stride, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  kb::clear_error();
  KB_REQUIRE(M >= 0 && K > 0 && N > 0, KB_ERR_BAD_SHAPE, "dense: bad shape");
  if (M == 0) return KB_OK;
  KB_REQUIRE(x && packed && scales && y, KB_ERR_NULL_POINTER, "dense (tcgen05): NULL pointer");
  int gshift = 0;
  int st = kb::tc::common_checks(x, x_stride, K, N, group, &gshift);
  if (st != KB_OK) return st;
  KB_REQUIRE(kb::aligned(packed, 16) && kb::aligned(scales, 16), KB_ERR_ALIGNMENT,
             "packed weights and scales must be 16-byte aligned");
  KB_REQUIRE(y_stride >= N && M <= (1 << 24), KB_ERR_BAD_SHAPE, "dense (tcgen05): bad output");
  int nt, tiles, splits;
  kb::tc::dense_split(M, K, N, &nt, &tiles, &splits);
  const size_t need = kb::tc::split_ws_bytes(tiles, splits, nt);
  KB_REQUIRE(need == 0 || (workspace && workspace_bytes >= need &&
                           kb::aligned(workspace, 256)),
             KB_ERR_WORKSPACE,
             "dense (tcgen05): workspace of %zu bytes (256-byte aligned, counters zeroed) "
             "required, %zu given",
             need, workspace_bytes);
  Args A = {};
  A.mode = kb::tc::DENSE;
  A.x_tma = 1;
  A.x = x;
  A.xs = x_stride;
  A.T = (int)M;
  A.R = 1;
  A.K = (int)K;
  A.N = (int)N;
  A.E = 1;
  A.gshift = gshift;
  A.ng = (int)(K / group);
  A.s0 = scales;
  A.s1 = scales;
  A.sse = 0;
  A.y = y;
  A.ys = y_stride;
  A.n_rt = (int)((N + 2 * kb::tc::BM - 1) / (2 * kb::tc::BM));
  A.nt = nt;
  A.nbuf = nt > kb::tc::NT_MAX ? 1 : 2;
  A.splits = splits;
  if (splits > 1) {
    const size_t part = (size_t)tiles * splits * 2 * nt * kb::tc::BM * sizeof(float);
    A.ws = static_cast<float*>(workspace);
    A.counters = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) +
                                        (part + 255) / 256 * 256);
  }
  st = kb::tc::layout(A, 0);
  if (st != KB_OK) return st;
  return kb::tc::launch_tc(A, packed, nullptr, N, tiles * splits, stream);
}

static int grouped_tc(int mode, const uint16_t* x, int64_t x_stride, int64_t T, int64_t K,
                      const int64_t* idx, int64_t R, const uint8_t* w0, const uint16_t* s0,
                      const uint8_t* w1, const uint16_t* s1, int64_t E, int64_t N,
                      int64_t group, uint16_t* y, void* stream) {
  kb::clear_error();
  KB_REQUIRE(T >= 0 && K > 0 && N > 0 && R > 0 && E > 0, KB_ERR_BAD_SHAPE,
             "grouped (tcgen05): bad shape");
  if (T == 0) return KB_OK;
  KB_REQUIRE(x && idx && w0 && s0 && y && (mode != kb::tc::SWIGLU || (w1 && s1)),
             KB_ERR_NULL_POINTER, "grouped (tcgen05): NULL pointer");
  int gshift = 0;
  int st = kb::tc::common_checks(x, x_stride, K, N, group, &gshift);
  if (st != KB_OK) return st;
  KB_REQUIRE(T * R <= kb::tc::MAX_ASSIGN && E <= kb::tc::MAX_SLOTS, KB_ERR_UNSUPPORTED,
             "grouped (tcgen05): T*R = %lld above %d or E = %lld above %d", (long long)(T * R),
             kb::tc::MAX_ASSIGN, (long long)E, kb::tc::MAX_SLOTS);
  KB_REQUIRE(kb::aligned(w0, 16) && kb::aligned(s0, 16) &&
                 (mode != kb::tc::SWIGLU || (kb::aligned(w1, 16) && kb::aligned(s1, 16))),
             KB_ERR_ALIGNMENT, "packed weights and scales must be 16-byte aligned");
  KB_REQUIRE(E * N <= (int64_t)1 << 31, KB_ERR_UNSUPPORTED, "grouped (tcgen05): bank too large");
  KB_REQUIRE(T * x_stride < (int64_t)1 << 31, KB_ERR_UNSUPPORTED,
             "grouped (tcgen05): activations too large for 32-bit row offsets");
  Args A = {};
  A.mode = mode;
  A.x = x;
  A.xs = x_stride;
  A.idx = idx;
  A.T = (int)T;
  A.R = (int)R;
  A.K = (int)K;
  A.N = (int)N;
  A.E = (int)E;
  A.gshift = gshift;
  A.ng = (int)(K / group);
  A.s0 = s0;
  A.s1 = s1 ? s1 : s0;
  A.sse = N * (K / group);
  A.y = y;
  A.ys = N;
  const int rows_per_unit = (mode == kb::tc::SWIGLU) ? kb::tc::BM : 2 * kb::tc::BM;
  A.n_rt = (int)((N + rows_per_unit - 1) / rows_per_unit);
  // Token rows per unit: 32 when experts average fewer than 48 rows (batched
  // decode spreads T * R rows over many experts; TMEM then holds three
  // decoded-weight stages), else 64 (one expert taking many rows).
  A.nt = (T * R >= 48 * E) ? kb::tc::NT_MAX : 32;
  A.nbuf = 2;
  A.splits = 1;
  const int plan_ints = kb::tc::plan_ints_for((int)E, (int)(T * R));
  st = kb::tc::layout(A, plan_ints);
  if (st != KB_OK) return st;
  return kb::tc::launch_tc(A, w0, w1, E * N, 1 << 30, stream);
}

extern "C" int kb_w4a16_grouped_tc(const uint16_t* x, int64_t x_stride, int64_t T, int64_t K,
                                   const int64_t* idx, int64_t R, const uint8_t* packed,
                                   const uint16_t* scales, int64_t E, int64_t N, int64_t group,
                                   uint16_t* y, void* stream) {
  return grouped_tc(kb::tc::GROUPED, x, x_stride, T, K, idx, R, packed, scales, nullptr, nullptr,
                    E, N, group, y, stream);
}

extern "C" int kb_w4a16_swiglu_tc(const uint16_t* x, int64_t x_stride, int64_t T, int64_t K,
                                  const int64_t* idx, int64_t R, const uint8_t* w1_packed,
                                  const uint16_t* w1_scales, const uint8_t* w3_packed,
                                  const uint16_t* w3_scales, int64_t E, int64_t N, int64_t group,
                                  uint16_t* y, void* stream) {
  return grouped_tc(kb::tc::SWIGLU, x, x_stride, T, K, idx, R, w1_packed, w1_scales, w3_packed,
                    w3_scales, E, N, group, y, stream);
}
