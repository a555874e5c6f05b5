// kb_capi.cu - library-wide state behind the C ABI: error messages, the
// programmatic-dependent-launch switch, SM counts and the device error word.
#include "kb_common.cuh"

#include <cstdarg>
#include <cstdio>
#include <mutex>

namespace kb {

namespace {
thread_local char g_last_error[512] = {0};
int g_pdl = 1;
constexpr int kMaxDevices = 64;
int g_sms[kMaxDevices] = {0};
uint32_t* g_err_ptr[kMaxDevices] = {nullptr};
std::mutex g_mutex;
}  // namespace

// One 32-bit error word per device, in a __device__ variable so that reading
// or clearing it never allocates.
__device__ uint32_t g_device_error_word;

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

void clear_error() { g_last_error[0] = 0; }

bool pdl_enabled() { return g_pdl != 0; }

int num_sms(int device) {
  if (device < 0 || device >= kMaxDevices) return 148;
  if (g_sms[device] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
        v <= 0)
      v = 148;
    g_sms[device] = v;
  }
  return g_sms[device];
}

uint32_t* device_error_word(int device) {
  if (device < 0 || device >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_err_ptr[device] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error_word) == cudaSuccess)
      g_err_ptr[device] = static_cast<uint32_t*>(p);
  }
  return g_err_ptr[device];
}

int bind_stream_device(void* stream) {
  // The library's runtime follows the context current on the calling thread,
  // which is the device the caller (torch) made current.  No stream query is
  // made here: stream queries are not permitted while a stream is capturing.
  (void)stream;
  int cur = 0;
  cudaGetDevice(&cur);
  return cur;
}

}  // namespace kb

extern "C" {

int kb_version(void) { return 100; }

const char* kb_last_error(void) { return kb::g_last_error; }

void kb_set_pdl(int enabled) { kb::g_pdl = enabled ? 1 : 0; }

int kb_get_pdl(void) { return kb::g_pdl; }

int kb_device_errors(void* stream, uint32_t* out_bits) {
  kb::clear_error();
  KB_REQUIRE(out_bits != nullptr, KB_ERR_NULL_POINTER, "out_bits is NULL");
  const int dev = kb::bind_stream_device(stream);
  uint32_t* p = kb::device_error_word(dev);
  KB_REQUIRE(p != nullptr, KB_ERR_LAUNCH, "device error word unavailable");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint32_t host = 0;
  cudaError_t e = cudaMemcpyAsync(&host, p, sizeof(host), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaMemsetAsync(p, 0, sizeof(uint32_t), s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  KB_REQUIRE(e == cudaSuccess, KB_ERR_LAUNCH, "reading the device error word failed: %s",
             cudaGetErrorString(e));
  *out_bits = host;
  return KB_OK;
}

}  // extern "C"
