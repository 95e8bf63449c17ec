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

static constexpr int kMaxStageEvents = 16;
static std::atomic<int> g_stage_n{0};
static cudaEvent_t g_stage_events[kMaxStageEvents] = {};

void mark_stage(int k, cudaStream_t stream) {
  if (k < g_stage_n.load(std::memory_order_acquire) && g_stage_events[k])
    cudaEventRecord(g_stage_events[k], stream);
}

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

extern "C" int gs_set_stage_events(void* const* events, int n) {
  GS_API_BEGIN();
  GS_REQUIRE(n >= 0 && n <= gs::kMaxStageEvents, "at most 16 stage events");
  gs::g_stage_n.store(0, std::memory_order_release);
  if (events == nullptr || n == 0) return GS_OK;
  for (int k = 0; k < n; ++k) gs::g_stage_events[k] = (cudaEvent_t)events[k];
  gs::g_stage_n.store(n, std::memory_order_release);
  return GS_OK;
  GS_API_END();
}

extern "C" int gs_event_create_timed(void** event) {
  GS_API_BEGIN();
  GS_REQUIRE(event != nullptr, "null pointer");
  cudaEvent_t ev = nullptr;
  GS_CUDA(cudaEventCreate(&ev));
  *event = ev;
  return GS_OK;
  GS_API_END();
}

extern "C" int gs_event_elapsed_ms(void* start, void* end, float* ms) {
  GS_API_BEGIN();
  GS_REQUIRE(start && end && ms, "null pointer");
  GS_CUDA(cudaEventElapsedTime(ms, (cudaEvent_t)start, (cudaEvent_t)end));
  return GS_OK;
  GS_API_END();
}
