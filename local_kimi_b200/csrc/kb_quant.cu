// kb_quant.cu - on-device W4A16 quantiser (restates engine/quant/w4a16.py:68-105).
//
// Per group of `group` consecutive reduction-axis values of one row:
//   absmax = max |w|; stored = bf16(absmax / 7)
//   scale  = 1 if absmax == 0 else bf16(max(float(stored), smallest normal))
//   code   = clamp(rint(float(w) / float(scale)), -7, 7)   (rint: ties to even)
// and the codes are packed two per byte, even index in the low nibble.
// One thread handles eight consecutive values (one packed 32-bit word); the
// group's absmax is reduced across the group/8 lanes that share it.
#include "kb_common.cuh"

namespace kb {

__global__ void __launch_bounds__(256)
    quantise_kernel(const uint16_t* __restrict__ w, int64_t ws, int N, int K, int gshift,
                    uint8_t* __restrict__ packed, uint16_t* __restrict__ scales,
                    int32_t* nonfinite) {
  const int words = K >> 3;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int lanes_per_group = 4 << gshift;  // group / 8
  const int64_t total = (int64_t)N * words;
  const bool valid = gid < total;
  const int row = valid ? (int)(gid / words) : 0;
  const int word = valid ? (int)(gid - (int64_t)row * words) : 0;

  pdl_wait();
  pdl_launch_dependents();

  float v[8];
  float amax = 0.f;
  bool finite = true;
  if (valid) {
    const uint4 raw = *reinterpret_cast<const uint4*>(w + (size_t)row * ws + (size_t)word * 8);
    const uint32_t r[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[2 * j] = __uint_as_float(r[j] << 16);
      v[2 * j + 1] = __uint_as_float(r[j] & 0xFFFF0000u);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      finite = finite && isfinite(v[j]);
      amax = fmaxf(amax, fabsf(v[j]));
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = 0.f;
  }
  if (!finite && nonfinite) atomicExch(nonfinite, 1);
  // Groups never straddle a warp: lanes_per_group divides 32 or is a multiple
  // of it, and words per row is a multiple of lanes_per_group.
  if (lanes_per_group <= 32) {
    for (int o = lanes_per_group >> 1; o > 0; o >>= 1)
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  }
  if (!valid) return;
  const float stored = round_bf16(amax / 7.0f);
  const float tiny = 1.17549435082228750797e-38f;  // smallest normal bf16 / fp32
  const float scale = (amax == 0.f) ? 1.0f : round_bf16(fmaxf(stored, tiny));
  uint32_t word_out = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float c = rintf(v[j] / scale);
    c = fminf(7.f, fmaxf(-7.f, c));
    const uint32_t nib = static_cast<uint32_t>(static_cast<int>(c)) & 0xFu;
    word_out |= nib << (4 * j);
  }
  reinterpret_cast<uint32_t*>(packed + (size_t)row * (K >> 1))[word] = word_out;
  if ((word & (lanes_per_group - 1)) == 0)
    scales[(size_t)row * (K >> (5 + gshift)) + (word >> (2 + gshift))] = float_to_bf16_bits(scale);
}

}  // namespace kb

extern "C" int kb_w4a16_quantise(const uint16_t* w, int64_t w_stride, int64_t N, int64_t K,
                                 int64_t group, uint8_t* packed, uint16_t* scales,
                                 int32_t* nonfinite_flag, void* stream) {
  kb::clear_error();
  KB_REQUIRE(N > 0 && K > 0, KB_ERR_BAD_SHAPE, "quantise needs N, K > 0");
  KB_REQUIRE(group == 32 || group == 64 || group == 128 || group == 256, KB_ERR_BAD_GROUP,
             "quantise supports group sizes 32, 64, 128 and 256 (got %lld)", (long long)group);
  KB_REQUIRE(K % group == 0, KB_ERR_BAD_GROUP, "K %lld is not divisible by group %lld",
             (long long)K, (long long)group);
  KB_REQUIRE(w && packed && scales, KB_ERR_NULL_POINTER, "NULL quantise pointer");
  KB_REQUIRE(reinterpret_cast<uintptr_t>(w) % 16 == 0 && w_stride % 8 == 0 && w_stride >= K,
             KB_ERR_ALIGNMENT, "weights must be 16-byte aligned with row stride %% 8 == 0");
  KB_REQUIRE(reinterpret_cast<uintptr_t>(packed) % 4 == 0, KB_ERR_ALIGNMENT,
             "packed output must be 4-byte aligned");
  int gshift = 0;
  while ((32 << gshift) < group) ++gshift;
  const int64_t total = N * (K / 8);
  const int64_t blocks = (total + 255) / 256;
  KB_REQUIRE(blocks < (int64_t(1) << 31), KB_ERR_UNSUPPORTED, "matrix too large");
  return kb::launch(kb::quantise_kernel, dim3((unsigned)blocks), dim3(256), 0, stream, w,
                    w_stride, (int)N, (int)K, gshift, packed, scales, nonfinite_flag);
}
