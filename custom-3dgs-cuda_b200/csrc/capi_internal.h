// Error plumbing shared by the extern "C" entry points.
#pragma once

#include <cuda_runtime.h>

#include <exception>
#include <string>

#include "gs3d_b200.h"

namespace gs {

// Counts kernel launches made by this library (read by gs_kernel_launches).
void count_launches(unsigned n);

// Records the installed stage event `k` (gs_set_stage_events) on `stream`, if any.
void mark_stage(int k, cudaStream_t stream);

// Records `msg` as the calling thread's last error and returns `code`.
int set_error(int code, const std::string& msg);
void clear_error();

}  // namespace gs

#define GS_API_BEGIN() \
  gs::clear_error();   \
  try {
#define GS_API_END()                                           \
  }                                                            \
  catch (const std::exception& e) {                            \
    return gs::set_error(GS_ERR_INVALID_ARG, e.what());        \
  }                                                            \
  catch (...) {                                                \
    return gs::set_error(GS_ERR_INVALID_ARG, "unknown error"); \
  }

#define GS_REQUIRE(cond, msg)                                    \
  do {                                                           \
    if (!(cond)) return gs::set_error(GS_ERR_INVALID_ARG, (msg)); \
  } while (0)

#define GS_CUDA(expr)                                                                 \
  do {                                                                                \
    cudaError_t gs_err__ = (expr);                                                    \
    if (gs_err__ != cudaSuccess)                                                      \
      return gs::set_error(GS_ERR_CUDA, std::string("CUDA error: ") +                 \
                                            cudaGetErrorString(gs_err__) + " (" #expr \
                                            ") at " __FILE__);                        \
  } while (0)

#define GS_CHECK_LAUNCH()       \
  do {                          \
    gs::count_launches(1u);     \
    GS_CUDA(cudaGetLastError()); \
  } while (0)
