// kb_engine.cuh - pieces of the W4A16 projection engine shared by the
// per-operation kernels (kb_w4a16.cu) and the decode-step executor
// (kb_step.cu): thread layout, the item/stage layout of the shared-memory
// ring, the producer's bulk copies, and the consumers' decode + mma.sync
// contraction of one 16-row block over a range of 128-wide reduction blocks.
#pragma once

#include "kb_common.cuh"

#include <algorithm>

namespace kb {

constexpr int NCW = 16;                 // consumer warps
constexpr int NCT = NCW * 32;           // consumer threads
constexpr int NTHREADS = NCT + 32;      // + one producer warp
constexpr int MAX_SMEM = 225 * 1024;
constexpr int MAX_STAGES = 6;
constexpr int X_RESIDENT_BUDGET = 64 * 1024;  // bytes of activations kept resident
constexpr int CBAR = 1;                 // named barrier id of the consumer warps
constexpr int SMEM_RESERVE = 2048;      // static shared memory and barriers

enum : int { MODE_DENSE = 0, MODE_GROUPED = 1, MODE_SWIGLU = 2, MODE_W2C = 3 };
enum : uint32_t { ERR_INDEX = 1u, ERR_TIMEOUT = 2u };

// Description of one item, computed identically by producer and consumers.
struct Item {
  const uint8_t* w[2];
  const uint16_t* s[2];
  int mats;
  int K, N, gshift, KS, RBc;
  int r0;           // first row of the item
  int rows;         // valid rows (<= RBc*16)
  int RS;           // shared-memory row stride in bytes (K/2: rows land contiguously)
  int ng;           // scale groups per row
  bool scale_bulk;  // scales copied into the stage (else read from global memory)
  int p;            // dense problem index or grouped slot
  int abase, count; // grouped: assignment range; dense: 0, M
};

// An item's rows are contiguous in global memory and are copied with one bulk
// copy per matrix, so they keep their global stride in shared memory.  (Large
// copies stream at full HBM rate; per-row copies of 0.25-1 KB did not.)
__host__ __device__ __forceinline__ int row_stride_bytes(int K) { return K / 2; }

__device__ __forceinline__ bool scale_bulk_ok(const uint16_t* s, int r0, int rows, int ng) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(s + (size_t)r0 * ng);
  const uint32_t bytes = (uint32_t)rows * ng * 2;
  return (a % 16 == 0) && (bytes % 16 == 0);
}

// Stage layout of an item: mats x RBc*16 weight rows of RS bytes, then one
// 16-byte-padded block of scale rows per matrix.
__device__ __forceinline__ int stage_scale_offset(const Item& it) {
  return it.mats * it.RBc * 16 * it.RS;
}
__device__ __forceinline__ int stage_scale_stride(const Item& it) {
  return (it.RBc * 16 * it.ng * 2 + 15) / 16 * 16;
}

// ---------------------------------------------------------------------------
// Producer: stream one item into a ring stage.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void produce_item(const Item& it, uint8_t* stage, uint64_t* full,
                                             uint64_t policy) {
  const int lane = threadIdx.x & 31;
  const uint32_t wbytes = (uint32_t)(it.K / 2);
  const uint32_t sbytes = (uint32_t)it.rows * it.ng * 2;
  uint32_t total = (uint32_t)it.mats * it.rows * wbytes;
  if (it.scale_bulk) total += (uint32_t)it.mats * sbytes;
  if (lane == 0) mbar_arrive_expect_tx(full, total);
  __syncwarp();
  if (lane < it.mats) {
    const uint8_t* wm = lane ? it.w[1] : it.w[0];
    bulk_g2s(stage + lane * it.RBc * 16 * it.RS, wm + (size_t)it.r0 * wbytes,
             (uint32_t)it.rows * wbytes, full, policy);
  }
  if (it.scale_bulk && lane < it.mats) {
    const uint16_t* sm = lane ? it.s[1] : it.s[0];
    bulk_g2s(stage + stage_scale_offset(it) + lane * stage_scale_stride(it),
             sm + (size_t)it.r0 * it.ng, sbytes, full, policy);
  }
}

// ---------------------------------------------------------------------------
// Consumer: one 16-row block x one reduction slice of a staged item.
// ---------------------------------------------------------------------------
// One 128-wide reduction block for this lane: 16-byte pieces of rows g (WA)
// and g+8 (WB), their replicated scales, and the activation words at px[p]
// (token slot 8p+g; word j of the chunk at px[p] + j*NC16).
template <int NSUB>
__device__ __forceinline__ void kblock_mma(uint4 WA, uint4 WB, uint32_t sa2, uint32_t sb2,
                                           const uint8_t* const (&px)[NSUB], int NC16, int nact,
                                           float (&acc)[NSUB][4], float (&acc2)[NSUB][4]) {
  const uint32_t wa[4] = {WA.x, WA.y, WA.z, WA.w};
  const uint32_t wb[4] = {WB.x, WB.y, WB.z, WB.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
    decode_word(wa[j], sa2, a0, a1, a2, a3);
    decode_word(wb[j], sb2, b0, b1, b2, b3);
#pragma unroll
    for (int p = 0; p < NSUB; ++p) {
      if (NSUB == 1 || p < nact) {
        const uint4 xv = lds_v4(px[p] + j * NC16);
        if (j & 1) {
          mma_bf16_16816(acc2[p], a0, b0, a1, b1, xv.x, xv.y);
          mma_bf16_16816(acc2[p], a2, b2, a3, b3, xv.z, xv.w);
        } else {
          mma_bf16_16816(acc[p], a0, b0, a1, b1, xv.x, xv.y);
          mma_bf16_16816(acc[p], a2, b2, a3, b3, xv.z, xv.w);
        }
      }
    }
  }
}

// xrow[p]: this lane's activation row for token slot 8p + g (shared memory).
// srow: scale rows of this row block (shared or global memory, generic loads).
// D fragment: acc[p][0] = (row g, token 2t), [1] = (row g, token 2t+1),
// [2] = (row g+8, token 2t), [3] = (row g+8, token 2t+1).
// SMEM_SCALES: srow is known to point into shared memory (explicit shared loads).
// COMPACT: the reduction width is a multiple of 128 (no partial block) and the
// loop is not unrolled -- the decode-step executor runs many operations in one
// kernel, where instruction-cache footprint costs more than the unrolling gains.
template <int NSUB, bool SMEM_SCALES = false, bool COMPACT = false>
__device__ __forceinline__ void rowblock_compute(const uint8_t* wtile, int RS,
                                                 const uint16_t* srow, int ng, int rows_valid,
                                                 int K, int gshift, int kb0, int kb1,
                                                 const uint8_t* (&xrow)[NSUB], int nact,
                                                 float (&acc)[NSUB][4]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int NC = K >> 5;
  const int NC16 = NC * 16;
  const int rowA = min(g, rows_valid - 1);
  const int rowB = min(g + 8, rows_valid - 1);
  const uint16_t* sA = srow + rowA * ng;
  const uint16_t* sB = srow + rowB * ng;
  float acc2[NSUB][4];
#pragma unroll
  for (int p = 0; p < NSUB; ++p)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc2[p][i] = 0.f;
  // Full 128-wide blocks first (every chunk of the block exists), then the
  // partial block at the end of the reduction axis when K % 128 != 0.
  const int kbf = min(kb1, NC >> 2);
  int c = kb0 * 4 + t;
  const uint8_t* pa = wtile + rowA * RS + c * 16;
  const uint8_t* pb = wtile + rowB * RS + c * 16;
  const uint8_t* px[NSUB];
#pragma unroll
  for (int p = 0; p < NSUB; ++p) px[p] = xrow[p] + c * 16;
#pragma unroll(COMPACT ? 1 : 2)
  for (int kb = kb0; kb < kbf; ++kb) {
    const uint4 WA = lds_v4(pa);
    const uint4 WB = lds_v4(pb);
    const uint32_t sa = SMEM_SCALES ? lds_u16(sA + (c >> gshift)) : sA[c >> gshift];
    const uint32_t sb = SMEM_SCALES ? lds_u16(sB + (c >> gshift)) : sB[c >> gshift];
    kblock_mma<NSUB>(WA, WB, prmt(sa, 0, 0x1010), prmt(sb, 0, 0x1010), px, NC16, nact, acc,
                     acc2);
    pa += 64;
    pb += 64;
    c += 4;
#pragma unroll
    for (int p = 0; p < NSUB; ++p) px[p] += 64;
  }
  if (!COMPACT && kbf < kb1) {
    // Partial block: chunks at or past NC contribute zero weights.
    const bool valid = c < NC;
    const int cc = valid ? c : NC - 1;
    const int back = (c - cc) * 16;
    uint4 WA = lds_v4(pa - back);
    uint4 WB = lds_v4(pb - back);
    if (!valid) {
      WA = make_uint4(0, 0, 0, 0);
      WB = make_uint4(0, 0, 0, 0);
    }
    const uint32_t sa = sA[cc >> gshift];
    const uint32_t sb = sB[cc >> gshift];
    const uint8_t* pxc[NSUB];
#pragma unroll
    for (int p = 0; p < NSUB; ++p) pxc[p] = px[p] - back;
    kblock_mma<NSUB>(WA, WB, prmt(sa, 0, 0x1010), prmt(sb, 0, 0x1010), pxc, NC16, nact, acc,
                     acc2);
  }
#pragma unroll
  for (int p = 0; p < NSUB; ++p)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[p][i] += acc2[p][i];
}

// Stage one activation row (K bf16, 16-byte aligned) into shared memory in
// the layout the B fragments read: word j of chunk c at (j*NC + c)*16, each
// word in pair order (x0,x4),(x1,x5),(x2,x6),(x3,x7).
__device__ __forceinline__ void stage_row(uint8_t* xs_row, const uint16_t* src, int K, int first,
                                          int step) {
  const int NC = K >> 5;
  const int words = K >> 3;
  for (int w = first; w < words; w += step) {
    const uint4 v = *reinterpret_cast<const uint4*>(src + (size_t)w * 8);
    const int c = w >> 2, j = w & 3;
    *reinterpret_cast<uint4*>(xs_row + (j * NC + c) * 16) = permute_pairs(v);
  }
}

// Expert index of an empty assignment slot in the grouped and SwiGLU modes
// (fixed-capacity exchange buffers of the expert-parallel layer): the slot is
// skipped -- no weights read for it, no output row written.
constexpr int64_t EXPERT_NONE = -1;

__device__ __forceinline__ int clamp_expert(int64_t v, int E, uint32_t* err) {
  if (v < 0 || v >= E) {
    atomicOr(err, ERR_INDEX);
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


// ---------------------------------------------------------------------------
// Host helpers.
// ---------------------------------------------------------------------------
inline int ilog2_exact(int64_t v) {
  int s = 0;
  while ((int64_t(1) << s) < v) ++s;
  return ((int64_t(1) << s) == v) ? s : -1;
}

inline int check_group(int64_t K, int64_t group, int* gshift) {
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

inline bool aligned(const void* p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

__host__ __device__ inline int token_stride(int K) {
  const int bytes = 2 * K;
  const int pad = (64 - (bytes % 128) + 128) % 128;
  return bytes + pad;
}

inline int item_stage_bytes(int K, int mats, int RBc, int ng) {
  const int rows = RBc * 16;
  const int wb = mats * rows * row_stride_bytes(K);
  const int sb = mats * ((rows * ng * 2 + 15) / 16 * 16);
  return (wb + sb + 127) / 128 * 128;
}


}  // namespace kb
