// Library-wide entry points: error reporting, version and the device error word.
#include <atomic>
#include <string>

#include "capi_internal.h"
#include "gs_common.cuh"

namespace gs {

__device__ unsigned g_device_errors = 0u;

static thread_local std::string t_last_error;
static std::atomic<unsigned long long> g_launches{0};

void count_launches(unsigned n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int set_error(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

void clear_error() { t_last_error.clear(); }

}  // namespace gs

extern "C" const char* gs_last_error(void) { return gs::t_last_error.c_str(); }

extern "C" unsigned long long gs_kernel_launches(void) {
  return gs::g_launches.load(std::memory_order_relaxed);
}

extern "C" const char* gs_version(void) { return "gs3d_b200 0.1.0 (sm_100a)"; }

extern "C" int gs_device_error_bits(unsigned* bits) {
  GS_API_BEGIN();
  GS_REQUIRE(bits != nullptr, "null pointer");
  GS_CUDA(cudaDeviceSynchronize());
  GS_CUDA(cudaMemcpyFromSymbol(bits, gs::g_device_errors, sizeof(unsigned)));
  return GS_OK;
  GS_API_END();
}

extern "C" int gs_clear_device_errors(void) {
  GS_API_BEGIN();
  const unsigned zero = 0u;
  GS_CUDA(cudaDeviceSynchronize());
  GS_CUDA(cudaMemcpyToSymbol(gs::g_device_errors, &zero, sizeof(unsigned)));
  return GS_OK;
  GS_API_END();
}

extern "C" int gs_event_create(void** event) {
  GS_API_BEGIN();
  GS_REQUIRE(event != nullptr, "null pointer");
  cudaEvent_t ev = nullptr;
  GS_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
  *event = ev;
  return GS_OK;
  GS_API_END();
}

extern "C" int gs_event_synchronize(void* event) {
  GS_API_BEGIN();
  GS_REQUIRE(event != nullptr, "null event");
  GS_CUDA(cudaEventSynchronize((cudaEvent_t)event));
  return GS_OK;
  GS_API_END();
}

extern "C" int gs_event_destroy(void* event) {
  GS_API_BEGIN();
  if (event) GS_CUDA(cudaEventDestroy((cudaEvent_t)event));
  return GS_OK;
  GS_API_END();
}
