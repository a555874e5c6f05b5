// kb_common.cuh - shared device helpers and host-side plumbing for the
// B200 (sm_100a) decode hot path: error reporting, launch helpers with
// programmatic dependent launch, the INT4 -> bf16 decode used by every W4A16
// kernel, and the warp-level tensor-core step.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stddef.h>
#include <string>

#include "../../include/kimi_b200.h"

namespace kb {

// ---------------------------------------------------------------------------
// Host-side error plumbing.
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);
void clear_error();
bool pdl_enabled();
int num_sms(int device);
uint32_t* device_error_word(int device);
// Make the stream's device current for this runtime instance (the library
// links its own CUDA runtime, so it follows the stream rather than assuming
// the caller's current device).  Returns the device index.
int bind_stream_device(void* stream);

#define KB_REQUIRE(cond, code, ...)            \
  do {                                         \
    if (!(cond)) {                             \
      ::kb::set_error(__VA_ARGS__);            \
      return (code);                           \
    }                                          \
  } while (0)

// Launch `kernel` with grid/block/smem on `stream`, adding the programmatic
// stream serialization attribute when PDL is enabled.  Returns KB_OK or
// KB_ERR_LAUNCH (with the CUDA error text recorded).
template <typename... KArgs, typename... Args>
int launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
           void* stream, Args&&... args) {
  bind_stream_device(stream);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (err != cudaSuccess) {
    set_error("kernel launch failed: %s", cudaGetErrorString(err));
    return KB_ERR_LAUNCH;
  }
  return KB_OK;
}

// ---------------------------------------------------------------------------
// Device helpers.
// ---------------------------------------------------------------------------

// Wait until the grid this launch depends on (programmatic dependent launch)
// has completed and its memory is visible.  No-op without the attribute.
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
// Allow the next grid on the stream to start its prologue.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint16_t ldg_u16(const uint16_t* p) {
  uint16_t v;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ uint4 lds_v4(const void* p) {
  return *reinterpret_cast<const uint4*>(p);
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ uint32_t lop3_and_xor(uint32_t a, uint32_t mask, uint32_t x) {
  // (a & mask) ^ x in one LOP3.
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(d) : "r"(a), "r"(mask), "r"(x));
  return d;
}

__device__ __forceinline__ uint32_t bf2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint32_t bf2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// bf16x2 constants (bit patterns).
constexpr uint32_t BF2_ONE = 0x3F803F80u;     // (1, 1)
constexpr uint32_t BF2_M136 = 0xC308C308u;    // (-136, -136)
constexpr uint32_t BF2_EIGHTH = 0x3E003E00u;  // (0.125, 0.125)
constexpr uint32_t BF2_M24 = 0xC1C0C1C0u;     // (-24, -24)

// Decode one 32-bit word of packed codes (8 nibbles n0..n7, n_i = code of
// reduction index 8w+i, even index in the low nibble of each byte) into four
// bf16x2 pairs of decoded weights bf16(code * scale):
//   p0 = (k0, k4), p1 = (k1, k5), p2 = (k2, k6), p3 = (k3, k7).
// Each nibble n is turned into u = n ^ 8 = code + 8 and placed in the
// mantissa of a bf16 whose exponent encodes 128: bits 0-3 give 128 + u,
// bits 3-6 give 128 + 8u.  One exact bf16x2 FMA recovers the signed code,
// and one bf16x2 multiply by the replicated scale performs the single
// rounding the reference applies (w4a16_gemv.py:146-158).
__device__ __forceinline__ void decode_word(uint32_t w, uint32_t scale2,
                                            uint32_t& p0, uint32_t& p1,
                                            uint32_t& p2, uint32_t& p3) {
  const uint32_t a = lop3_and_xor(w, 0x000F000Fu, 0x43084308u);
  const uint32_t b = lop3_and_xor(w >> 1, 0x00780078u, 0x43404340u);
  const uint32_t c = lop3_and_xor(w >> 8, 0x000F000Fu, 0x43084308u);
  const uint32_t d = lop3_and_xor(w >> 9, 0x00780078u, 0x43404340u);
  p0 = bf2_mul(bf2_fma(a, BF2_ONE, BF2_M136), scale2);
  p1 = bf2_mul(bf2_fma(b, BF2_EIGHTH, BF2_M24), scale2);
  p2 = bf2_mul(bf2_fma(c, BF2_ONE, BF2_M136), scale2);
  p3 = bf2_mul(bf2_fma(d, BF2_EIGHTH, BF2_M24), scale2);
}

// Permute 8 bf16 activations x0..x7 (natural order, packed as 4 u32 with the
// lower index in the low half) into the decode pair order
// (x0,x4), (x1,x5), (x2,x6), (x3,x7).
__device__ __forceinline__ uint4 permute_pairs(uint4 v) {
  uint4 o;
  o.x = prmt(v.x, v.z, 0x5410);
  o.y = prmt(v.x, v.z, 0x7632);
  o.z = prmt(v.y, v.w, 0x5410);
  o.w = prmt(v.y, v.w, 0x7632);
  return o;
}

// D[16x8] += A[16x16] * B[16x8], bf16 inputs, fp32 accumulate.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------------------
// mbarrier + bulk-copy (TMA, non-multicast) primitives.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

// Make barrier initialisation visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking probe of a phase.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after `limit` polls (each poll may suspend the
// thread for a hardware-defined interval) and returns false.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint32_t limit = (1u << 22)) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// Brings [p, p + bytes) into L2 without returning data to the SM; p 16-byte
// aligned, bytes a multiple of 16.  L2 is the point of coherence, so a line
// prefetched early still reads the current value later.
__device__ __forceinline__ void l2_prefetch_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint64_t l2_evict_last_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Global -> shared bulk copy completing on `bar` (bytes % 16 == 0, both
// addresses 16-byte aligned).  Plain (non-multicast) form.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ uint16_t lds_u16(const void* p) {
  return *reinterpret_cast<const uint16_t*>(p);
}

__device__ __forceinline__ float bf16_bits_to_float(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

__device__ __forceinline__ uint16_t float_to_bf16_bits(float f) {
  __nv_bfloat16 h = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&h);
}

__device__ __forceinline__ float round_bf16(float f) {
  return bf16_bits_to_float(float_to_bf16_bits(f));
}

}  // namespace kb
