// Tensor-memory-accelerator (TMA) tile copies global -> shared with mbarrier completion, and the
// host side that describes a tensor to the copy engine (cuTensorMapEncodeTiled, reached through
// the runtime's driver entry point, so the library still links only the CUDA runtime).
//
// Rules the callers keep: the shared destination is 128-byte aligned; the tensor's base address
// and every stride above the innermost are multiples of 16 bytes; the innermost box extent and
// the innermost start coordinate are multiples of 16 bytes (4 floats). Other coordinates may be
// negative or past the end: those elements read as zero. Each CTA copies for itself only.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "gs_common.cuh"

namespace gs {

__device__ __forceinline__ unsigned smem_u32(const void* p) {
  return (unsigned)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned arrivals) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(arrivals)
               : "memory");
  // make the initialised barrier visible to the copy engine (async proxy)
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// One arrival that also announces `bytes` of copies to come.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ unsigned long long tma_global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits for the barrier's phase `parity` to complete, for at most `limit_ns` of GPU global
// time and 2^26 polls (each poll may suspend the thread for a hardware-defined time). Returns
// false if a limit ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity,
                                          unsigned long long limit_ns) {
  const unsigned addr = smem_u32(bar);
  const unsigned long long t0 = tma_global_ns();
  for (unsigned k = 0; k < (1u << 26); ++k) {
    unsigned done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
    if (tma_global_ns() - t0 > limit_ns) return false;
  }
  return false;
}

// Tile copy of a 3-D box at (x, y, z) (innermost first) of `map` into `dst`, completing on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y,
                                            int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// Host: cuTensorMapEncodeTiled from the driver, or null where the driver does not offer it.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Describes a float32 tensor [d2][d1][d0] (d0 innermost) with row pitch `pitch0` elements and
// plane pitch `pitch1` elements, copied in boxes of b0 x b1 x b2; out-of-range elements read as
// zero. Returns false (and leaves `map` unusable) where the rules above do not hold or the
// driver refuses.
inline bool encode_f32_3d(CUtensorMap* map, const float* base, uint64_t d0, uint64_t d1,
                          uint64_t d2, uint64_t pitch0, uint64_t pitch1, unsigned b0,
                          unsigned b1, unsigned b2) {
  const EncodeTiledFn fn = encode_tiled_fn();
  if (!fn || (reinterpret_cast<uintptr_t>(base) & 15u) || (pitch0 * 4) % 16 || (pitch1 * 4) % 16 ||
      (b0 * 4) % 16 || b0 > 256 || b1 > 256 || b2 > 256)
    return false;
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {pitch0 * 4, pitch1 * 4};
  const cuuint32_t box[3] = {b0, b1, b2};
  const cuuint32_t elem[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box,
            elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

}  // namespace gs
