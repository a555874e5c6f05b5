// kb_ep.cu - the data plane of the expert-parallel MoE layer.
//
// The experts of a layer are sharded over the ranks (expert e on rank
// e / per_rank).  The exchange uses fixed-capacity buffers so that no step
// needs a host-side count and the whole layer can be captured in a CUDA graph:
// every rank reserves `capacity` row slots for every destination rank
// (capacity = tokens * top_k, the most one destination can receive, so no
// route is ever dropped).
//
// kb_ep_dispatch: for every routed (token, route) pair -- in token-major,
// route order -- the destination rank and its position among the pairs bound
// for that rank (a stable counting scan), then the token's hidden row copied
// into the send buffer at slot destination * capacity + position.  A payload
// row is H bf16 values followed by 8 more: the owner-local expert id as an
// int64 and padding, so rows and ids travel in one exchange.  Unused slots get
// expert id -1 (the grouped kernels skip such slots).  The slot of every pair is returned for the
// combine.  Reference: the routing of engine/klinear/moe.py:278-334 (the same
// rows reach the same experts as on one GPU).
//
// kb_ep_combine: out[t] = bf16( bf16(sum_r float(y[slot[t,r]]) * w[t,r])
//                               + y_shared[t] ), fp32 sum in route order --
// the combine of engine/kernels/moe_combine.py:209-261 reading each route's
// output where the return exchange left it.
#include <algorithm>

#include "kb_common.cuh"

namespace kb {

constexpr int EP_THREADS = 256;
constexpr int EP_MAX_PAIRS = 8192;   // tokens * top_k per call
constexpr int EP_MAX_RANKS = 64;

// Stable per-destination positions of all pairs: pos[a] and the counts
// cnt[d].  All threads first stage every pair's destination in shared memory
// (coalesced loads); then warp w scans the pairs for destinations d = w, w+8,
// ...: a ballot per 32 pairs gives each match its rank among the earlier
// matches.  Every CTA computes the same table.
__device__ void ep_positions(const int64_t* idx, int64_t istride, int T, int k, int per_rank,
                             int world, int* cnt, int* pos, uint8_t* dest, uint32_t* err) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int pairs = T * k;
  // Eight ids per thread are requested before any is used (the loads are
  // independent; one round trip instead of eight).
  for (int a0 = tid; a0 < pairs; a0 += 8 * EP_THREADS) {
    int64_t ev[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int a = a0 + i * EP_THREADS;
      if (a < pairs) {
        const int t = a / k, r = a - t * k;
        ev[i] = idx[(size_t)t * istride + r];
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int a = a0 + i * EP_THREADS;
      if (a < pairs) {
        const int64_t e = ev[i];
        int d = 0;
        if (e < 0 || e >= (int64_t)per_rank * world) {
          atomicOr(err, 1u);
        } else {
          d = (int)(e / per_rank);
        }
        dest[a] = (uint8_t)d;
      }
    }
  }
  __syncthreads();
  for (int d = warp; d < world; d += EP_THREADS / 32) {
    int running = 0;
    for (int base = 0; base < pairs; base += 32) {
      const int a = base + lane;
      const bool mine = a < pairs && dest[a] == d;
      const unsigned m = __ballot_sync(0xffffffffu, mine);
      if (mine) pos[a] = running + __popc(m & ((1u << lane) - 1u));
      running += __popc(m);
    }
    if (lane == 0) cnt[d] = running;
  }
  __syncthreads();
}

// Copy of one row of `vecs` 16-byte pieces by a warp: eight pieces per lane
// are requested before any is stored, so a row costs one memory round trip
// per 4 KB instead of one per 512 bytes.
__device__ __forceinline__ void warp_copy_row(uint4* __restrict__ dst,
                                              const uint4* __restrict__ src, int vecs,
                                              int lane) {
  for (int v0 = 0; v0 < vecs; v0 += 32 * 8) {
    uint4 t[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int v = v0 + i * 32 + lane;
      if (v < vecs) t[i] = src[v];
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int v = v0 + i * 32 + lane;
      if (v < vecs) dst[v] = t[i];
    }
  }
}

__global__ void __launch_bounds__(EP_THREADS)
    ep_dispatch_kernel(const uint16_t* __restrict__ hidden, int64_t hs, int T, int H,
                       const int64_t* __restrict__ idx, int64_t istride, int k, int per_rank,
                       int world, int capacity, int64_t shared_id,
                       uint16_t* __restrict__ send_rows, int* __restrict__ slots, uint32_t* err) {
  __shared__ int cnt[EP_MAX_RANKS];
  extern __shared__ int pos[];                 // [pairs], then the destinations as bytes
  pdl_wait();
  ep_positions(idx, istride, T, k, per_rank, world, cnt, pos,
               reinterpret_cast<uint8_t*>(pos + T * k), err);
  const int pairs = T * k;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (EP_THREADS / 32) + warp, nw = gridDim.x * (EP_THREADS / 32);
  const int vecs = H >> 3;
  const int64_t ps = (int64_t)H + 8;  // payload row stride (elements)
  // Rows of the routed pairs, one warp per pair; with shared_id >= 0 also
  // every token's row once more after the world * capacity slots (the rank's
  // own rows for the shared expert, which are not exchanged).
  const int extra = shared_id >= 0 ? T : 0;
  for (int a = gw; a < pairs + extra; a += nw) {
    if (a >= pairs) {
      const int t = a - pairs;
      const uint4* src = reinterpret_cast<const uint4*>(hidden + (size_t)t * hs);
      uint4* dst = reinterpret_cast<uint4*>(send_rows + ((size_t)world * capacity + t) * ps);
      warp_copy_row(dst, src, vecs, lane);
      if (lane == 0)
        dst[vecs] = make_uint4((uint32_t)shared_id, (uint32_t)((uint64_t)shared_id >> 32), 0u, 0u);
      continue;
    }
    const int t = a / k, r = a - t * k;
    const int64_t e = idx[(size_t)t * istride + r];
    const bool ok = e >= 0 && e < (int64_t)per_rank * world;
    const int d = ok ? (int)(e / per_rank) : 0;
    const int p = pos[a];
    if (p >= capacity) {            // cannot happen with capacity = T * k
      if (lane == 0) atomicOr(err, 1u);
      continue;
    }
    const int slot = d * capacity + p;
    const uint4* src = reinterpret_cast<const uint4*>(hidden + (size_t)t * hs);
    uint4* dst = reinterpret_cast<uint4*>(send_rows + (size_t)slot * ps);
    warp_copy_row(dst, src, vecs, lane);
    if (lane == 0) {
      const int64_t id = ok ? e - (int64_t)d * per_rank : 0;
      dst[vecs] = make_uint4((uint32_t)id, (uint32_t)((uint64_t)id >> 32), 0u, 0u);
      slots[a] = slot;
    }
  }
  // Unused slots of every destination: expert id -1.
  const int total = world * capacity;
  for (int s = blockIdx.x * EP_THREADS + threadIdx.x; s < total; s += gridDim.x * EP_THREADS) {
    const int d = s / capacity;
    if (s - d * capacity >= cnt[d])
      *reinterpret_cast<uint4*>(send_rows + (size_t)s * ps + H) =
          make_uint4(0xffffffffu, 0xffffffffu, 0u, 0u);
  }
  pdl_launch_dependents();
}

__global__ void __launch_bounds__(EP_THREADS)
    ep_combine_kernel(const uint16_t* __restrict__ y, const int* __restrict__ slots, int T,
                      int k, int H, const float* __restrict__ w, int64_t wstride,
                      const uint16_t* __restrict__ shared, int64_t ss,
                      uint16_t* __restrict__ out, int64_t os) {
  pdl_wait();
  const int words = H >> 3;
  const int64_t total = (int64_t)T * words;
  for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < total;
       u += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(u / words), wd = (int)(u - (int64_t)t * words);
    float accum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    // Up to eight routes' slots, weights and rows are requested before any is
    // summed; the sums then run in route order.
    for (int r0 = 0; r0 < k; r0 += 8) {
      int sl[8];
      float wr[8];
      uint4 v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (r0 + i < k) {
          sl[i] = slots[t * k + r0 + i];
          wr[i] = w[(size_t)t * wstride + r0 + i];
        }
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (r0 + i < k)
          v[i] = *reinterpret_cast<const uint4*>(y + (size_t)sl[i] * H + (size_t)wd * 8);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (r0 + i < k) {
          const uint32_t pv[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            accum[2 * j] += bf16_bits_to_float((uint16_t)(pv[j] & 0xffffu)) * wr[i];
            accum[2 * j + 1] += bf16_bits_to_float((uint16_t)(pv[j] >> 16)) * wr[i];
          }
        }
      }
    }
    const uint4 s = *reinterpret_cast<const uint4*>(shared + (size_t)t * ss + (size_t)wd * 8);
    const uint32_t sv[4] = {s.x, s.y, s.z, s.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint16_t lo = float_to_bf16_bits(round_bf16(accum[2 * j]) +
                                             bf16_bits_to_float((uint16_t)(sv[j] & 0xffffu)));
      const uint16_t hi = float_to_bf16_bits(round_bf16(accum[2 * j + 1]) +
                                             bf16_bits_to_float((uint16_t)(sv[j] >> 16)));
      o[j] = (uint32_t)lo | ((uint32_t)hi << 16);
    }
    *reinterpret_cast<uint4*>(out + (size_t)t * os + (size_t)wd * 8) =
        make_uint4(o[0], o[1], o[2], o[3]);
  }
  pdl_launch_dependents();
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace kb

extern "C" int kb_ep_dispatch(const uint16_t* hidden, int64_t h_stride, int64_t T, int64_t H,
                              const int64_t* idx, int64_t idx_stride, int64_t k,
                              int64_t per_rank, int64_t world, int64_t capacity,
                              int64_t shared_id, uint16_t* send_rows, int32_t* slots,
                              void* stream) {
  kb::clear_error();
  KB_REQUIRE(T >= 0 && H > 0 && k > 0 && per_rank > 0 && world > 0 && capacity > 0,
             KB_ERR_BAD_SHAPE, "dispatch: bad shape");
  if (T == 0) return KB_OK;
  KB_REQUIRE(H % 8 == 0 && h_stride % 8 == 0 && h_stride >= H && idx_stride >= k,
             KB_ERR_BAD_SHAPE, "dispatch: H and the row stride must be multiples of 8");
  KB_REQUIRE(T * k <= kb::EP_MAX_PAIRS && world <= kb::EP_MAX_RANKS &&
                 world * capacity <= (int64_t)1 << 24 && capacity >= T * k,
             KB_ERR_UNSUPPORTED,
             "dispatch: needs T*k <= %d, world <= %d and capacity >= T*k (T*k = %lld, "
             "capacity = %lld)",
             kb::EP_MAX_PAIRS, kb::EP_MAX_RANKS, (long long)(T * k), (long long)capacity);
  KB_REQUIRE(hidden && idx && send_rows && slots, KB_ERR_NULL_POINTER,
             "dispatch: NULL pointer");
  KB_REQUIRE(kb::al16(hidden) && kb::al16(send_rows), KB_ERR_ALIGNMENT,
             "dispatch: hidden and send_rows must be 16-byte aligned");
  const int dev = kb::bind_stream_device(stream);
  uint32_t* err = kb::device_error_word(dev);
  KB_REQUIRE(err != nullptr, KB_ERR_LAUNCH, "device error word unavailable");
  const int sms = kb::num_sms(dev);
  const int grid = std::max(1, std::min<int>(sms, (int)((T * k + 7) / 8)));
  const size_t smem = (size_t)(T * k) * (sizeof(int) + 1);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kb::ep_dispatch_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)(kb::EP_MAX_PAIRS * (sizeof(int) + 1)));
    KB_REQUIRE(e == cudaSuccess, KB_ERR_DEVICE, "dispatch: shared-memory limit: %s",
               cudaGetErrorString(e));
  }
  return kb::launch(kb::ep_dispatch_kernel, dim3(grid), dim3(kb::EP_THREADS), smem, stream,
                    hidden, h_stride, (int)T, (int)H, idx, idx_stride, (int)k, (int)per_rank,
                    (int)world, (int)capacity, shared_id, send_rows, slots, err);
}

extern "C" int kb_ep_combine(const uint16_t* y, const int32_t* slots, int64_t T, int64_t k,
                             int64_t H, const float* weights, int64_t w_stride,
                             const uint16_t* shared, int64_t shared_stride, uint16_t* out,
                             int64_t out_stride, void* stream) {
  kb::clear_error();
  KB_REQUIRE(T >= 0 && k > 0 && H > 0, KB_ERR_BAD_SHAPE, "combine: bad shape");
  if (T == 0) return KB_OK;
  KB_REQUIRE(H % 8 == 0 && shared_stride % 8 == 0 && out_stride % 8 == 0 &&
                 shared_stride >= H && out_stride >= H && w_stride >= k,
             KB_ERR_BAD_SHAPE, "combine: widths and strides must be multiples of 8");
  KB_REQUIRE(T <= (1 << 24) && k <= 64 && H <= (1 << 20), KB_ERR_UNSUPPORTED,
             "combine supports T <= 2^24, k <= 64, H <= 2^20");
  KB_REQUIRE(y && slots && weights && shared && out, KB_ERR_NULL_POINTER,
             "combine: NULL pointer");
  KB_REQUIRE(kb::al16(y) && kb::al16(shared) && kb::al16(out), KB_ERR_ALIGNMENT,
             "combine: y, shared and out must be 16-byte aligned");
  const int sms = kb::num_sms(kb::bind_stream_device(stream));
  const int64_t work = T * (H / 8);
  const int64_t blocks =
      std::min<int64_t>((work + kb::EP_THREADS - 1) / kb::EP_THREADS, (int64_t)sms * 8);
  return kb::launch(kb::ep_combine_kernel, dim3((unsigned)std::max<int64_t>(blocks, 1)),
                    dim3(kb::EP_THREADS), 0, stream, y, slots, (int)T, (int)k, (int)H,
                    weights, w_stride, shared, shared_stride, out, out_stride);
}
