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
#include "kb_kda_prep.cuh"

#include <algorithm>
#include <mutex>

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

// Streaming form for Dk = Dv = 128 (the model's shape) with contiguous state
// rows, used when there are enough (batch, head) pairs to fill the GPU.  One
// persistent CTA per SM walks the heads u = blockIdx.x + n * gridDim.x; each
// head's state (64 KB, contiguous) and its q, k, decay and v rows arrive by
// bulk asynchronous copies into one of three shared-memory stages, two heads
// ahead of the one being updated, and the updated state leaves by one bulk
// store.  So every SM keeps about 130 KB of reads and one 64 KB write in
// flight with no thread waiting on them, and the registers hold one head's
// slice at a time: lane l owns columns 4l .. 4l+3, warp w the rows w, w+8, ...
// Column sums go through shared memory in warp order.
constexpr int KS_THREADS = 256;
constexpr int KS_WARPS = KS_THREADS / 32;
constexpr int KS_DIM = 128;
constexpr int KS_ROWS = KS_DIM / KS_WARPS;
constexpr int KS_STAGES = 3;
constexpr int KS_HEAD = KS_DIM * KS_DIM;                 // floats of one head's state
constexpr int KS_STAGE = KS_HEAD + 4 * KS_DIM;           // + q, k, decay, v
constexpr size_t KS_SMEM = (size_t)KS_STAGES * KS_STAGE * 4 + 5 * KS_DIM * 4 + 32 * 4 +
                           2 * KS_WARPS * 32 * 16 + KS_STAGES * 8 + 16;
constexpr long long KS_WAIT_NS = 2000000000LL;

__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
               "r"(smem_addr(src)), "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

__device__ __forceinline__ void bulk_wait_read_1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}

__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ long long ks_now() {
  long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Inputs of the fused form: the preparation's (kb_kda_prepare) instead of
// prepared q, k, v, decay and beta.
struct KsPrep {
  const uint16_t *q_in, *k_in, *v_in;
  int64_t in_stride;
  uint16_t *q_state, *k_state, *v_state;
  const uint16_t *q_w, *k_w, *v_w;
  const uint16_t* raw_decay;
  int64_t rd_stride;
  const float* dt_bias;
  const float* a_log;
  const uint16_t* raw_beta;
  int64_t rb_stride;
  float eps;
};

// One channel's preparation inputs, fetched one head ahead.
struct KsChan {
  uint2 qs, ks, vs, qw, kw, vw;
  uint16_t qt, kt, vt, rd, rb;
  float dtb, al;
};

// Sum over the 128 channel threads (warps 0-3) in the order of the
// preparation kernel's block sum: xor butterfly, then the warps in order.
__device__ __forceinline__ float chan_sum(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  named_barrier(1, KS_DIM);
  float s = 0.f;
  for (int w = 0; w < KS_DIM / 32; ++w) s += red[w];
  named_barrier(1, KS_DIM);
  return s;
}

template <bool FUSED>
__global__ void __launch_bounds__(KS_THREADS, 1)
    kda_stream_kernel(float* __restrict__ state, int64_t sb, int64_t sh,
                      const float* __restrict__ q, const float* __restrict__ k,
                      const float* __restrict__ v, const float* __restrict__ decay,
                      const float* __restrict__ beta, int H, int BH, float scale,
                      float* __restrict__ out, uint16_t* __restrict__ out_bf16,
                      uint32_t* __restrict__ err, const KsPrep pp) {
  extern __shared__ __align__(128) uint8_t ks_smem[];
  float* stage = reinterpret_cast<float*>(ks_smem);
  float* s_ed = stage + KS_STAGES * KS_STAGE;
  float* s_k = s_ed + KS_DIM;
  float* s_bk = s_k + KS_DIM;
  float* s_q = s_bk + KS_DIM;
  float* s_v = s_q + KS_DIM;                                   // fused form: v
  float* s_cred = s_v + KS_DIM;                                // fused form: channel sums
  float4* s_red = reinterpret_cast<float4*>(s_cred + 32);      // [2][KS_WARPS][32]
  uint64_t* full = reinterpret_cast<uint64_t*>(s_red + 2 * KS_WARPS * 32);
  int* s_ok = reinterpret_cast<int*>(full + KS_STAGES);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x;

  if (tid == 0) {
    for (int i = 0; i < KS_STAGES; ++i) mbar_init(&full[i], 1);
    mbar_fence_init();
  }
  __syncthreads();
  pdl_wait();
  pdl_launch_dependents();

  const uint64_t pol = l2_evict_first_policy();
  auto head_state = [&](int u) {
    const int b = u / H, h = u - b * H;
    return state + (size_t)b * sb + (size_t)h * sh;
  };
  auto issue = [&](int u, int s) {
    float* st = stage + (size_t)s * KS_STAGE;
    const size_t vec = (size_t)u * KS_DIM;
    if (FUSED) {
      mbar_arrive_expect_tx(&full[s], KS_HEAD * 4);
      bulk_g2s(st, head_state(u), KS_HEAD * 4, &full[s], pol);
      return;
    }
    mbar_arrive_expect_tx(&full[s], KS_STAGE * 4);
    bulk_g2s(st, head_state(u), KS_HEAD * 4, &full[s], pol);
    bulk_g2s(st + KS_HEAD, q + vec, KS_DIM * 4, &full[s], pol);
    bulk_g2s(st + KS_HEAD + KS_DIM, k + vec, KS_DIM * 4, &full[s], pol);
    bulk_g2s(st + KS_HEAD + 2 * KS_DIM, decay + vec, KS_DIM * 4, &full[s], pol);
    bulk_g2s(st + KS_HEAD + 3 * KS_DIM, v + vec, KS_DIM * 4, &full[s], pol);
  };
  if (tid == 0)
    for (int n = 0; n < KS_STAGES - 1; ++n)
      if (blockIdx.x + n * G < BH) issue(blockIdx.x + n * G, n);

  // Fused form: channel tid's preparation inputs of head u.
  const int C = H * KS_DIM;
  auto fetch = [&](int u, KsChan& ci) {
    const int b = u / H, h = u - b * H, c = h * KS_DIM + tid;
    const size_t si = ((size_t)b * C + c) * 4;
    ci.qs = *reinterpret_cast<const uint2*>(pp.q_state + si);
    ci.ks = *reinterpret_cast<const uint2*>(pp.k_state + si);
    ci.vs = *reinterpret_cast<const uint2*>(pp.v_state + si);
    ci.qw = *reinterpret_cast<const uint2*>(pp.q_w + (size_t)c * 4);
    ci.kw = *reinterpret_cast<const uint2*>(pp.k_w + (size_t)c * 4);
    ci.vw = *reinterpret_cast<const uint2*>(pp.v_w + (size_t)c * 4);
    const size_t ii = (size_t)b * pp.in_stride + c;
    ci.qt = pp.q_in[ii];
    ci.kt = pp.k_in[ii];
    ci.vt = pp.v_in[ii];
    ci.rd = pp.raw_decay[(size_t)b * pp.rd_stride + c];
    ci.dtb = pp.dt_bias[c];
    ci.al = pp.a_log[h];
    ci.rb = pp.raw_beta[(size_t)b * pp.rb_stride + h];
  };
  KsChan ci;
  if (FUSED && tid < KS_DIM) fetch(blockIdx.x, ci);
  float bt = (!FUSED && tid < KS_DIM) ? beta[blockIdx.x] : 0.f;
  int s = 0;
  uint32_t ph = 0;
  int issued = min(KS_STAGES - 1, (BH - (int)blockIdx.x + G - 1) / G);
  int done = 0;
  for (int u = blockIdx.x; u < BH; u += G, ++done) {
    // One thread waits (bounded); its outcome is shared so that every thread
    // leaves the loop together on a timeout.
    if (tid == 0) {
      int ok = 1;
      const long long t0 = ks_now();
      while (!mbar_try_wait(&full[s], ph)) {
        if (ks_now() - t0 > KS_WAIT_NS) {
          atomicOr(err, 2u);
          ok = 0;
          break;
        }
      }
      *s_ok = ok;
    }
    __syncthreads();
    if (!*s_ok) break;
    while (!mbar_try_wait(&full[s], ph)) {
    }
    float* st = stage + (size_t)s * KS_STAGE;
    const float* sq = st + KS_HEAD;
    if (FUSED) {
      if (tid < KS_DIM) {
        // The preparation of channel tid (kb_kda_prepare's operations in its
        // order), the shifted convolution states written back.
        const int b = u / H, c = (u - b * H) * KS_DIM + tid;
        const size_t si = ((size_t)b * C + c) * 4;
        uint2 nq, nk, nv;
        const float qc = conv_regs(ci.qs, ci.qw, ci.qt, nq);
        const float kc = conv_regs(ci.ks, ci.kw, ci.kt, nk);
        const float vc = conv_regs(ci.vs, ci.vw, ci.vt, nv);
        *reinterpret_cast<uint2*>(pp.q_state + si) = nq;
        *reinterpret_cast<uint2*>(pp.k_state + si) = nk;
        *reinterpret_cast<uint2*>(pp.v_state + si) = nv;
        const float dec = kda_decay(ci.al, ci.rd, ci.dtb);
        const float btv = kda_beta(ci.rb);
        const float qn = qc * rsqrtf(chan_sum(qc * qc, s_cred) + pp.eps);
        const float kn = kc * rsqrtf(chan_sum(kc * kc, s_cred) + pp.eps);
        s_ed[tid] = expf(dec);
        s_k[tid] = kn;
        s_bk[tid] = __fmul_rn(btv, kn);
        s_q[tid] = __fmul_rn(qn, scale);
        s_v[tid] = vc;
        if (u + G < BH) fetch(u + G, ci);   // next head's, used next pass
      }
    } else if (tid < KS_DIM) {
      const float kv = sq[KS_DIM + tid];
      s_ed[tid] = expf(sq[2 * KS_DIM + tid]);
      s_k[tid] = kv;
      s_bk[tid] = __fmul_rn(bt, kv);
      s_q[tid] = __fmul_rn(sq[tid], scale);
      bt = u + G < BH ? beta[u + G] : 0.f;   // next head's, consumed next pass
    }
    if (FUSED) __syncthreads();   // s_v complete before the lanes read it
    const float4 vv = FUSED ? reinterpret_cast<const float4*>(s_v)[lane]
                            : reinterpret_cast<const float4*>(sq + 3 * KS_DIM)[lane];
    __syncthreads();

    float4 c[KS_ROWS];
    float4 part = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < KS_ROWS; ++j) {
      const int i = warp + KS_WARPS * j;
      const float ed = s_ed[i], kk = s_k[i];
      c[j] = reinterpret_cast<const float4*>(st + i * KS_DIM)[lane];
      c[j].x = __fmul_rn(c[j].x, ed);
      c[j].y = __fmul_rn(c[j].y, ed);
      c[j].z = __fmul_rn(c[j].z, ed);
      c[j].w = __fmul_rn(c[j].w, ed);
      part.x = fmaf(c[j].x, kk, part.x);
      part.y = fmaf(c[j].y, kk, part.y);
      part.z = fmaf(c[j].z, kk, part.z);
      part.w = fmaf(c[j].w, kk, part.w);
    }
    s_red[warp * 32 + lane] = part;
    __syncthreads();
    float4 pred = s_red[lane];
#pragma unroll
    for (int w = 1; w < KS_WARPS; ++w) {
      const float4 p = s_red[w * 32 + lane];
      pred.x += p.x;
      pred.y += p.y;
      pred.z += p.z;
      pred.w += p.w;
    }
    const float4 d = make_float4(__fsub_rn(vv.x, pred.x), __fsub_rn(vv.y, pred.y),
                                 __fsub_rn(vv.z, pred.z), __fsub_rn(vv.w, pred.w));
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < KS_ROWS; ++j) {
      const int i = warp + KS_WARPS * j;
      const float bk = s_bk[i], qq = s_q[i];
      c[j].x = __fadd_rn(c[j].x, __fmul_rn(bk, d.x));
      c[j].y = __fadd_rn(c[j].y, __fmul_rn(bk, d.y));
      c[j].z = __fadd_rn(c[j].z, __fmul_rn(bk, d.z));
      c[j].w = __fadd_rn(c[j].w, __fmul_rn(bk, d.w));
      reinterpret_cast<float4*>(st + i * KS_DIM)[lane] = c[j];
      o.x = fmaf(c[j].x, qq, o.x);
      o.y = fmaf(c[j].y, qq, o.y);
      o.z = fmaf(c[j].z, qq, o.z);
      o.w = fmaf(c[j].w, qq, o.w);
    }
    s_red[(KS_WARPS + warp) * 32 + lane] = o;
    // The updated rows become visible to the bulk-copy engine, then one
    // thread sends the head back and refills the stage used two heads ago.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (tid == 0) {
      bulk_s2g(head_state(u), st, KS_HEAD * 4);
      const int un = u + (KS_STAGES - 1) * G;
      if (un < BH) {
        int sn = s + KS_STAGES - 1;
        if (sn >= KS_STAGES) sn -= KS_STAGES;
        bulk_wait_read_1();   // that stage's store has left shared memory
        issue(un, sn);
        ++issued;
      }
    }
    if (warp == 0) {
      float4 r = s_red[KS_WARPS * 32 + lane];
#pragma unroll
      for (int w = 1; w < KS_WARPS; ++w) {
        const float4 p = s_red[(KS_WARPS + w) * 32 + lane];
        r.x += p.x;
        r.y += p.y;
        r.z += p.z;
        r.w += p.w;
      }
      const size_t vec = (size_t)u * KS_DIM;
      reinterpret_cast<float4*>(out + vec)[lane] = r;
      if (out_bf16) {
        const uint32_t lo = (uint32_t)float_to_bf16_bits(r.x) |
                            ((uint32_t)float_to_bf16_bits(r.y) << 16);
        const uint32_t hi = (uint32_t)float_to_bf16_bits(r.z) |
                            ((uint32_t)float_to_bf16_bits(r.w) << 16);
        reinterpret_cast<uint2*>(out_bf16 + vec)[lane] = make_uint2(lo, hi);
      }
    }
    if (++s == KS_STAGES) {
      s = 0;
      ph ^= 1u;
    }
  }
  if (tid == 0) {
    // Loads still in flight after a timeout land before the CTA exits
    // (bounded); every store has completed.
    for (int n = done; n < issued; ++n) {
      const int sn = n % KS_STAGES;
      const uint32_t pn = (uint32_t)(n / KS_STAGES) & 1u;
      const long long t0 = ks_now();
      while (!mbar_try_wait(&full[sn], pn))
        if (ks_now() - t0 > KS_WAIT_NS / 10) break;
    }
    bulk_wait_all();
  }
}

static std::mutex g_ks_attr_mu;
static bool g_ks_attr_done[64] = {};

static int kda_stream_attr(int dev) {
  KB_REQUIRE(dev >= 0 && dev < 64, KB_ERR_DEVICE, "KDA step: no usable current device");
  std::lock_guard<std::mutex> lock(g_ks_attr_mu);
  if (g_ks_attr_done[dev]) return KB_OK;
  cudaError_t e = cudaFuncSetAttribute(kda_stream_kernel<false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)KS_SMEM);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(kda_stream_kernel<true>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)KS_SMEM);
  KB_REQUIRE(e == cudaSuccess, KB_ERR_DEVICE, "KDA step: setting the shared-memory limit failed: %s",
             cudaGetErrorString(e));
  g_ks_attr_done[dev] = true;
  return KB_OK;
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
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (Dk == kb::KS_DIM && Dv == kb::KS_DIM && sk == kb::KS_DIM && sh % 4 == 0 && sb % 4 == 0 &&
      B * H >= 2 * 148 && a16(state) && a16(q) && a16(k) && a16(v) && a16(decay) && a16(out) &&
      (out_bf16 == nullptr || (reinterpret_cast<uintptr_t>(out_bf16) & 7) == 0)) {
    const int dev = kb::bind_stream_device(stream);
    const int attr = kb::kda_stream_attr(dev);
    if (attr != KB_OK) return attr;
    uint32_t* err = kb::device_error_word(dev);
    KB_REQUIRE(err != nullptr, KB_ERR_LAUNCH, "device error word unavailable");
    const int grid = (int)std::min<int64_t>(B * H, kb::num_sms(dev));
    return kb::launch(kb::kda_stream_kernel<false>, dim3((unsigned)grid),
                      dim3(kb::KS_THREADS), kb::KS_SMEM, stream, state, sb, sh, q, k, v, decay,
                      beta, (int)H, (int)(B * H), scale, out, out_bf16, err, kb::KsPrep{});
  }
  const dim3 grid((unsigned)(B * H), (unsigned)((Dv + kb::KDA_COLS - 1) / kb::KDA_COLS));
  const dim3 block(kb::KDA_WARPS * 32);
  if (Dk <= 128)
    return kb::launch(kb::kda_step_kernel<8>, grid, block, 0, stream, state, sb, sh, sk, q, k,
                      v, decay, beta, (int)H, (int)Dk, (int)Dv, scale, out, out_bf16);
  return kb::launch(kb::kda_step_kernel<16>, grid, block, 0, stream, state, sb, sh, sk, q, k, v,
                    decay, beta, (int)H, (int)Dk, (int)Dv, scale, out, out_bf16);
}

// The preparation (kb_kda_prepare) and the step (kb_kda_decode_step) of the
// model's shape in one streaming launch: each head's channel threads run the
// preparation's operations in its order, so the result equals the two calls.
extern "C" int kb_kda_prepare_step(const uint16_t* q_in, const uint16_t* k_in,
                                   const uint16_t* v_in, int64_t in_stride, uint16_t* q_state,
                                   uint16_t* k_state, uint16_t* v_state,
                                   const uint16_t* q_weight, const uint16_t* k_weight,
                                   const uint16_t* v_weight, const uint16_t* raw_decay,
                                   int64_t raw_decay_stride, const float* dt_bias,
                                   const float* a_log, const uint16_t* raw_beta,
                                   int64_t raw_beta_stride, float eps, float* state, int64_t sb,
                                   int64_t sh, int64_t sk, int64_t B, int64_t H, int64_t D,
                                   float scale, float* out, uint16_t* out_bf16, void* stream) {
  kb::clear_error();
  KB_REQUIRE(B > 0 && H > 0 && D > 0, KB_ERR_BAD_SHAPE, "KDA prepare+step: bad shape");
  KB_REQUIRE(D == kb::KS_DIM && sk == kb::KS_DIM && B * H <= (int64_t(1) << 30),
             KB_ERR_UNSUPPORTED,
             "KDA prepare+step supports head_dim %d with contiguous state rows", kb::KS_DIM);
  KB_REQUIRE(sh >= D * sk && sb >= H * sh && sh % 4 == 0 && sb % 4 == 0, KB_ERR_BAD_SHAPE,
             "KDA prepare+step: state strides");
  KB_REQUIRE(in_stride >= H * D && raw_decay_stride >= H * D && raw_beta_stride >= H,
             KB_ERR_BAD_SHAPE, "KDA prepare+step: row strides too small");
  KB_REQUIRE(eps > 0.f, KB_ERR_BAD_SHAPE, "KDA prepare+step: eps must be positive");
  KB_REQUIRE(q_in && k_in && v_in && q_state && k_state && v_state && q_weight && k_weight &&
                 v_weight && raw_decay && dt_bias && a_log && raw_beta && state && out,
             KB_ERR_NULL_POINTER, "KDA prepare+step: NULL pointer");
  auto a8 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7) == 0; };
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  KB_REQUIRE(a8(q_state) && a8(k_state) && a8(v_state) && a8(q_weight) && a8(k_weight) &&
                 a8(v_weight) && a16(state) && a16(out) &&
                 (out_bf16 == nullptr || a8(out_bf16)),
             KB_ERR_ALIGNMENT,
             "KDA prepare+step: states/weights 8-byte, state/out 16-byte aligned");
  const int dev = kb::bind_stream_device(stream);
  const int attr = kb::kda_stream_attr(dev);
  if (attr != KB_OK) return attr;
  uint32_t* err = kb::device_error_word(dev);
  KB_REQUIRE(err != nullptr, KB_ERR_LAUNCH, "device error word unavailable");
  kb::KsPrep pp;
  pp.q_in = q_in;
  pp.k_in = k_in;
  pp.v_in = v_in;
  pp.in_stride = in_stride;
  pp.q_state = q_state;
  pp.k_state = k_state;
  pp.v_state = v_state;
  pp.q_w = q_weight;
  pp.k_w = k_weight;
  pp.v_w = v_weight;
  pp.raw_decay = raw_decay;
  pp.rd_stride = raw_decay_stride;
  pp.dt_bias = dt_bias;
  pp.a_log = a_log;
  pp.raw_beta = raw_beta;
  pp.rb_stride = raw_beta_stride;
  pp.eps = eps;
  const int grid = (int)std::min<int64_t>(B * H, kb::num_sms(dev));
  return kb::launch(kb::kda_stream_kernel<true>, dim3((unsigned)grid), dim3(kb::KS_THREADS),
                    kb::KS_SMEM, stream, state, sb, sh, nullptr, nullptr, nullptr, nullptr,
                    nullptr, (int)H, (int)(B * H), scale, out, out_bf16, err, pp);
}
