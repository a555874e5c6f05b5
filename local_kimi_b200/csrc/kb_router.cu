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
// Phase 1: CTA (expert block, token block) computes 32 experts x up to 4
// tokens of logits (small token blocks: a CTA's latency, not the machine's
// throughput, sets the kernel's time at decode sizes), each warp 4 experts x
// 4 tokens per pass (every 16-byte
// piece it loads feeds four sums), with a fixed reduction order (each lane
// sums its strided 16-byte pieces in order, then a xor butterfly), so logits
// are identical run to run.  Phase 2: the CTA that completes a token block
// (arrival counter, one publishing thread) selects the top_k of its tokens,
// one warp per token, and resets the counter.  For E <= 256 every lane sorts
// its eight candidates once with a sorting network and each pick is two
// warp reductions (max key, then min index among the lanes holding it).
#include "kb_common.cuh"
#include "kb_topk.cuh"

#include <algorithm>
#include <mutex>

namespace kb {

constexpr int RT_WARPS = 8;               // warps per CTA
constexpr int RT_EW = 4;                  // experts per warp
constexpr int RT_EXP = RT_WARPS * RT_EW;  // experts per CTA
constexpr int RT_TOK = 4;                 // tokens per CTA (one pass of each warp)
constexpr int RT_TQ = 4;                  // tokens per pass of a warp

__global__ void __launch_bounds__(RT_WARPS * 32)
    router_kernel(const uint16_t* __restrict__ hidden, int64_t hs, int T, int K,
                  const uint16_t* __restrict__ weight, const float* __restrict__ bias, int E,
                  int top_k, int renorm, float scaling, int64_t* __restrict__ idx_out,
                  int64_t append_id, float* __restrict__ w_out, float* __restrict__ logits,
                  int* __restrict__ counters) {
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.y * RT_TOK;
  const int nt = min(RT_TOK, T - t0);
  const int words = K >> 3;

  pdl_wait();
  pdl_launch_dependents();

  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint16_t* hsm = reinterpret_cast<uint16_t*>(smem_raw);  // [nt][K]
  // Warp w computes experts ebase .. ebase + 3 for the CTA's tokens, four
  // tokens per pass: each 16-byte piece of a router row (from L2) and of a
  // staged hidden row (from shared memory) feeds four (token, expert) sums.
  // Every sum keeps the stated order: lane l takes pieces l, l + 32, ... in
  // order (router_word_fma), then router_lane_sum and the xor butterfly.
  const int ebase = blockIdx.x * RT_EXP + warp * RT_EW;
  const uint16_t* wrow[RT_EW];
#pragma unroll
  for (int i = 0; i < RT_EW; ++i) wrow[i] = weight + (size_t)min(ebase + i, E - 1) * K;
  // The warp's first pieces are requested before the hidden states are
  // staged, so both fetches overlap.
  uint4 wv[RT_EW];
#pragma unroll
  for (int i = 0; i < RT_EW; ++i)
    wv[i] = lane < words ? ldg_stream_v4(wrow[i] + (size_t)lane * 8) : make_uint4(0, 0, 0, 0);
  for (int e = threadIdx.x; e < nt * words; e += RT_WARPS * 32) {
    const int m = e / words, w = e - m * words;
    reinterpret_cast<uint4*>(hsm + (size_t)m * K)[w] =
        __ldg(reinterpret_cast<const uint4*>(hidden + (size_t)(t0 + m) * hs) + w);
  }
  __syncthreads();
  if (ebase < E) {
    for (int tq = 0; tq < nt; tq += RT_TQ) {
      float acc[RT_TQ][RT_EW][4];
#pragma unroll
      for (int t = 0; t < RT_TQ; ++t)
#pragma unroll
        for (int i = 0; i < RT_EW; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[t][i][j] = 0.f;
      if (tq > 0) {
#pragma unroll
        for (int i = 0; i < RT_EW; ++i)
          wv[i] = lane < words ? ldg_stream_v4(wrow[i] + (size_t)lane * 8) : make_uint4(0, 0, 0, 0);
      }
      for (int w = lane; w < words; w += 32) {
        // Next pieces of the router rows, requested before these are used.
        uint4 wn[RT_EW];
        const int wnext = w + 32;
#pragma unroll
        for (int i = 0; i < RT_EW; ++i)
          wn[i] = wnext < words ? ldg_stream_v4(wrow[i] + (size_t)wnext * 8)
                                : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int t = 0; t < RT_TQ; ++t) {
          if (tq + t < nt) {
            const uint4 hv = reinterpret_cast<const uint4*>(hsm + (size_t)(tq + t) * K)[w];
#pragma unroll
            for (int i = 0; i < RT_EW; ++i) router_word_fma(wv[i], hv, acc[t][i]);
          }
        }
#pragma unroll
        for (int i = 0; i < RT_EW; ++i) wv[i] = wn[i];
      }
#pragma unroll
      for (int t = 0; t < RT_TQ; ++t) {
#pragma unroll
        for (int i = 0; i < RT_EW; ++i) {
          float v = router_lane_sum(acc[t][i]);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
          if (lane == 0 && tq + t < nt && ebase + i < E)
            logits[(size_t)(t0 + tq + t) * E + ebase + i] = v;
        }
      }
    }
  }

  // Arrival: the last expert block of this token block runs the selection.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int old = atomicAdd(&counters[blockIdx.y], 1);
    s_last = (old == (int)gridDim.x - 1);
    if (s_last) __threadfence();
  }
  __syncthreads();
  if (!s_last) return;

  for (int m = warp; m < nt; m += RT_WARPS) {
    const int tok = t0 + m;
    const float* lrow = logits + (size_t)tok * E;
    float my_score = 0.f, wsum = 0.f;
    int my_idx = 0;
    if (E <= 256) {
      warp_topk256(lrow, bias, E, top_k, lane, my_idx, my_score, wsum);
    } else {
      // General E <= 1024: repeated warp argmax over register-held scores.
      float score[32];
      uint32_t key[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int e = lane + 32 * j;
        if (e < E) {
          const float lg = __ldcg(&lrow[e]);
          score[j] = 1.0f / (1.0f + expf(-lg));
          key[j] = choice_key(score[j] + (bias ? bias[e] : 0.f));
        } else {
          score[j] = 0.f;
          key[j] = 0u;
        }
      }
      unsigned taken = 0;
      for (int sel = 0; sel < top_k; ++sel) {
        uint32_t bk = 0u;
        int bi = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int e = lane + 32 * j;
          if (e < E && !(taken & (1u << j)) && choice_better(key[j], e, bk, bi)) {
            bk = key[j];
            bi = e;
          }
        }
        const uint32_t best = __reduce_max_sync(0xffffffffu, bk);
        const int win =
            (int)__reduce_min_sync(0xffffffffu, (bk == best) ? (uint32_t)bi : 0xffffffffu);
        float s = 0.f;
        if ((win & 31) == lane) {
          const int jw = win >> 5;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j == jw) s = score[j];
          taken |= 1u << jw;
        }
        s = __shfl_sync(0xffffffffu, s, win & 31);
        wsum += s;
        if (lane == sel) {
          my_score = s;
          my_idx = win;
        }
      }
    }
    const float denom = wsum + 1e-20f;
    const int istride = top_k + (append_id >= 0 ? 1 : 0);
    if (lane < top_k) {
      float wv = my_score;
      if (renorm && top_k > 1) wv = wv / denom;
      idx_out[(size_t)tok * istride + lane] = my_idx;
      w_out[(size_t)tok * top_k + lane] = wv * scaling;
    }
    if (append_id >= 0 && lane == 0) idx_out[(size_t)tok * istride + top_k] = append_id;
  }
  __syncthreads();
  if (threadIdx.x == 0) counters[blockIdx.y] = 0;
}

}  // namespace kb

namespace kb {

// The router kernel stages up to RT_TOK rows of K <= 8192 bf16 activations in
// dynamic shared memory (128 KiB at the limit), above the 48 KiB a launch gets
// without opting in.  The opt-in is a per-device function attribute, so it is
// set once for each device (with that device current), under a lock, and its
// result is checked.
constexpr int RT_MAX_DEVICES = 64;
static std::mutex g_router_attr_mu;
static bool g_router_attr_done[RT_MAX_DEVICES] = {};

static int router_smem_limit() {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= RT_MAX_DEVICES) {
    set_error("router: no usable current device (%s)", cudaGetErrorString(e));
    return KB_ERR_DEVICE;
  }
  std::lock_guard<std::mutex> lock(g_router_attr_mu);
  if (g_router_attr_done[dev]) return KB_OK;
  e = cudaFuncSetAttribute(router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)(RT_TOK * 8192 * sizeof(uint16_t)));
  if (e != cudaSuccess) {
    set_error("router: setting the shared-memory limit failed: %s", cudaGetErrorString(e));
    return KB_ERR_DEVICE;
  }
  g_router_attr_done[dev] = true;
  return KB_OK;
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
                              int64_t append_id, float* w_out, void* workspace,
                              size_t workspace_bytes, void* stream) {
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
  const dim3 grid((unsigned)((E + kb::RT_EXP - 1) / kb::RT_EXP),
                  (unsigned)((T + kb::RT_TOK - 1) / kb::RT_TOK));
  const size_t smem = (size_t)std::min<int64_t>(T, kb::RT_TOK) * K * sizeof(uint16_t);
  const int attr = kb::router_smem_limit();
  if (attr != KB_OK) return attr;
  return kb::launch(kb::router_kernel, grid, dim3(kb::RT_WARPS * 32), smem, stream, hidden,
                    h_stride, (int)T, (int)K, weight, bias, (int)E, (int)top_k, renormalize,
                    scaling, idx_out, append_id, w_out, logits, counters);
}

// ---------------------------------------------------------------------------
// kb_router_topk_static: the router with its scratch in a fixed device array.
//
// For callers that cannot allocate device memory: a host that binds the C ABI
// without a device allocator of its own, or a serving loop that must not call
// cudaMalloc between steps (cudaMalloc can synchronise the device and can fail
// under memory pressure).  This entry point calls no allocating routine; its
// scratch is the file-scope array below, one copy per device.
//
// Layout of the scratch: arrival counters first, at a fixed offset, so calls of
// any shape find them where the previous call left them; logits after them.
// The counters must start at zero: device storage without an initialiser is
// zero-filled when the module loads, the set-up clears them once more on the
// caller's stream, and every launch returns them to zero.  The logits need no
// initial value (each launch writes them before it reads them).
//
// The first call on each device does the set-up (symbol address, dynamic
// shared-memory limit, counter clear) with that device current; make that first
// call before any stream capture.  All calls on one device share the one
// scratch array, so calls that overlap in time on that device (other streams,
// other host threads) race and give wrong results: serialise them.
//
// The scratch address found by the set-up is kept for the life of the process.
// It assumes the device is not reset: after cudaDeviceReset the module (and
// with it the array) is loaded again, possibly at another address, and the
// kept address is stale.  A process that resets a device must not call this
// entry point on it afterwards.
// ---------------------------------------------------------------------------
namespace kb {

constexpr size_t RT_STATIC_COUNTERS = 2048;                          // token blocks (T <= 8192)
constexpr size_t RT_STATIC_LOGITS = 131072;                          // T * E floats (512 KiB)
constexpr size_t RT_STATIC_COUNTER_BYTES = RT_STATIC_COUNTERS * sizeof(int);
constexpr size_t RT_STATIC_BYTES =
    RT_STATIC_COUNTER_BYTES + RT_STATIC_LOGITS * sizeof(float);      // 532,480 bytes

static __device__ __align__(256) uint8_t g_router_static_scratch[RT_STATIC_BYTES];

constexpr int RT_STATIC_MAX_DEVICES = 64;
static std::mutex g_router_static_mu;
static void* g_router_static_ptr[RT_STATIC_MAX_DEVICES] = {};

// Per-device set-up; returns the scratch address on the current device or NULL
// after recording the error.
static void* router_static_scratch(int* status, cudaStream_t stream) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= RT_STATIC_MAX_DEVICES) {
    set_error("router (static scratch): no usable current device (%s)", cudaGetErrorString(e));
    *status = KB_ERR_DEVICE;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_router_static_mu);
  if (g_router_static_ptr[dev]) return g_router_static_ptr[dev];
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_router_static_scratch);
  if (e != cudaSuccess || p == nullptr) {
    set_error("router (static scratch): cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    *status = KB_ERR_DEVICE;
    return nullptr;
  }
  const int attr = router_smem_limit();
  if (attr != KB_OK) {
    *status = attr;
    return nullptr;
  }
  e = cudaMemsetAsync(p, 0, RT_STATIC_COUNTER_BYTES, stream);
  if (e != cudaSuccess) {
    set_error("router (static scratch): set-up failed: %s", cudaGetErrorString(e));
    *status = KB_ERR_DEVICE;
    return nullptr;
  }
  g_router_static_ptr[dev] = p;
  return p;
}

}  // namespace kb

extern "C" size_t kb_router_static_scratch_bytes(void) { return kb::RT_STATIC_BYTES; }

extern "C" int kb_router_topk_static(const uint16_t* hidden, int64_t h_stride, int64_t T,
                                     int64_t K, const uint16_t* weight, const float* bias,
                                     int64_t E, int64_t top_k, int renormalize, float scaling,
                                     int64_t* idx_out, int64_t append_id, float* w_out,
                                     void* stream) {
  kb::clear_error();
  KB_REQUIRE(T >= 0 && K > 0 && E > 0 && top_k > 0, KB_ERR_BAD_SHAPE,
             "router needs T >= 0 and K, E, top_k > 0");
  KB_REQUIRE(top_k <= E, KB_ERR_BAD_SHAPE, "top_k %lld exceeds E %lld", (long long)top_k,
             (long long)E);
  KB_REQUIRE(E <= 1024 && top_k <= 32 && K <= 8192 && K % 8 == 0, KB_ERR_UNSUPPORTED,
             "router supports E <= 1024, top_k <= 32, K <= 8192 with K %% 8 == 0");
  KB_REQUIRE((size_t)T * (size_t)E <= kb::RT_STATIC_LOGITS, KB_ERR_WORKSPACE,
             "router (static scratch): T*E = %lld exceeds the fixed scratch of %zu logits; "
             "use kb_router_topk with a caller workspace",
             (long long)(T * E), kb::RT_STATIC_LOGITS);
  KB_REQUIRE((size_t)(T + kb::RT_TOK - 1) / kb::RT_TOK <= kb::RT_STATIC_COUNTERS,
             KB_ERR_WORKSPACE,
             "router (static scratch): T = %lld needs %lld token blocks of %d, above the "
             "fixed scratch's %zu arrival counters (T <= %zu); use kb_router_topk with a "
             "caller workspace",
             (long long)T, (long long)((T + kb::RT_TOK - 1) / kb::RT_TOK), kb::RT_TOK,
             kb::RT_STATIC_COUNTERS, kb::RT_STATIC_COUNTERS * kb::RT_TOK);
  if (T == 0) return KB_OK;
  KB_REQUIRE(hidden && weight && idx_out && w_out, KB_ERR_NULL_POINTER, "NULL router pointer");
  KB_REQUIRE(reinterpret_cast<uintptr_t>(hidden) % 16 == 0 && h_stride % 8 == 0 &&
                 reinterpret_cast<uintptr_t>(weight) % 16 == 0,
             KB_ERR_ALIGNMENT, "hidden/weight must be 16-byte aligned with row stride %% 8 == 0");
  int status = KB_OK;
  void* scratch = kb::router_static_scratch(&status, static_cast<cudaStream_t>(stream));
  if (!scratch) return status;
  int* counters = reinterpret_cast<int*>(scratch);
  float* logits =
      reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(scratch) + kb::RT_STATIC_COUNTER_BYTES);
  const dim3 grid((unsigned)((E + kb::RT_EXP - 1) / kb::RT_EXP),
                  (unsigned)((T + kb::RT_TOK - 1) / kb::RT_TOK));
  const size_t smem = (size_t)std::min<int64_t>(T, kb::RT_TOK) * K * sizeof(uint16_t);
  return kb::launch(kb::router_kernel, grid, dim3(kb::RT_WARPS * 32), smem, stream, hidden,
                    h_stride, (int)T, (int)K, weight, bias, (int)E, (int)top_k, renormalize,
                    scaling, idx_out, append_id, w_out, logits, counters);
}
