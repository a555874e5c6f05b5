// kb_combine.cu - routing-weighted combine of per-route expert outputs.
//
// The combine step of the MoE layer when the per-route down-projection outputs
// are already in memory (expert parallelism: they come back from the GPUs
// that own the experts).  Same arithmetic as the fused down+combine kernel
// (engine/kernels/moe_combine.py:209-261, restated in kb_w4a16.cu):
//   out[t,n] = bf16( bf16(sum_{r<R-1} float(y[t,r,n]) * w[t,r]) + y[t,R-1,n] )
// with the fp32 sum taken in route order; the last route is the shared expert
// (weight 1).  HBM-bound elementwise work: one thread per 8 output elements,
// 16-byte loads of every route, grid a multiple of the SM count.
#include <algorithm>

#include "kb_common.cuh"

namespace kb {

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

__global__ void __launch_bounds__(256)
    combine_routes_kernel(const uint16_t* __restrict__ y, int T, int R, int N,
                          const float* __restrict__ w, int64_t wstride,
                          uint16_t* __restrict__ out) {
  pdl_wait();
  const int words = N >> 3;
  const int64_t total = (int64_t)T * words;
  for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < total;
       u += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(u / words), wd = (int)(u - (int64_t)t * words);
    const uint16_t* row = y + (size_t)t * R * N + (size_t)wd * 8;
    float accum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = 0; r + 1 < R; ++r) {
      const uint4 v = *reinterpret_cast<const uint4*>(row + (size_t)r * N);
      const float wr = w[(size_t)t * wstride + r];
      const uint32_t pv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        accum[2 * j] += bf16_bits_to_float((uint16_t)(pv[j] & 0xffffu)) * wr;
        accum[2 * j + 1] += bf16_bits_to_float((uint16_t)(pv[j] >> 16)) * wr;
      }
    }
    const uint4 s = *reinterpret_cast<const uint4*>(row + (size_t)(R - 1) * N);
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
    *reinterpret_cast<uint4*>(out + (size_t)t * N + (size_t)wd * 8) =
        make_uint4(o[0], o[1], o[2], o[3]);
  }
  pdl_launch_dependents();
}

}  // namespace kb

extern "C" int kb_moe_combine_routes(const uint16_t* routes, int64_t T, int64_t R, int64_t N,
                                     const float* weights, int64_t w_stride, uint16_t* out,
                                     void* stream) {
  kb::clear_error();
  KB_REQUIRE(T >= 0 && R >= 1 && N > 0, KB_ERR_BAD_SHAPE,
             "need T >= 0, R >= 1, N > 0 (got T=%lld R=%lld N=%lld)", (long long)T,
             (long long)R, (long long)N);
  if (T == 0) return KB_OK;
  KB_REQUIRE(N % 8 == 0, KB_ERR_BAD_SHAPE, "width %lld is not a multiple of 8", (long long)N);
  KB_REQUIRE(T <= (1 << 24) && R <= 64 && N <= (1 << 20), KB_ERR_UNSUPPORTED,
             "combine supports T <= 2^24, R <= 64, N <= 2^20");
  KB_REQUIRE(routes && out && (R == 1 || weights), KB_ERR_NULL_POINTER, "NULL argument");
  KB_REQUIRE(R == 1 || w_stride >= R - 1, KB_ERR_BAD_SHAPE, "weight row stride < R-1");
  KB_REQUIRE(kb::aligned16(routes) && kb::aligned16(out), KB_ERR_ALIGNMENT,
             "routes and out must be 16-byte aligned");
  const int sms = kb::num_sms(kb::bind_stream_device(stream));
  const int64_t work = T * (N / 8);
  const int64_t blocks = std::min<int64_t>((work + 255) / 256, (int64_t)std::max(sms, 1) * 8);
  return kb::launch(kb::combine_routes_kernel, dim3((unsigned)std::max<int64_t>(blocks, 1)),
                    dim3(256), 0, stream, routes, (int)T, (int)R, (int)N, weights, w_stride,
                    out);
}
