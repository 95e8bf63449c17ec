// The multi-GPU optimizer step of the view-parallel training step as one kernel per rank:
// reduce-scatter of the gradient bucket, Adam on this rank's shard, all-gather of the updated
// parameters, plus the SUM / MAX reductions of the densification statistics.
//
// Every rank holds the parameters, the gradient bucket and the max-statistic buffer in
// symmetric memory (the same layout on every GPU, mapped into every peer and, on NVSwitch
// systems, into one NVLink multicast range). Rank r owns elements [r S, (r + 1) S) of the
// bucket and parameter buffers (S a multiple of 4). After a barrier that makes every rank's
// bucket complete, each thread takes 16-byte groups of its rank's shard:
//   multicast: multimem.ld_reduce.add.v4.f32 sums the group over all GPUs inside the switch;
//              multimem.st.v4.f32 writes the result to every GPU;
//   peer:      plain 16-byte loads from each peer's buffer summed in rank order, and 16-byte
//              stores into each peer's buffer.
// Parameter groups get the Adam update (the same arithmetic as adam.cu, gradient scaled by
// 1 / batch) with this rank's shard of the moments; statistic groups are written back reduced.
// The max statistic (non-negative floats, ordered like their u32 bit patterns) is reduced with
// multimem.ld_reduce.max.u32 or peer loads. A closing barrier makes every rank's stores visible
// everywhere before the kernel ends. Barrier waits are bounded (gs_shard_buffers::wait_ns of
// GPU global time, 5 s by default, and an iteration cap); a timeout sets kErrPeerTimeout and
// the kernel returns.
#include <algorithm>
#include <atomic>
#include <cmath>

#include "capi_internal.h"
#include "gs_common.cuh"

namespace gs {

constexpr int kShardThreads = 256;
constexpr int kShardMaxGroups = 8;
constexpr int kShardMaxWorld = 8;
constexpr int kShardUnroll = 4;

struct ShardArgs {
  gs_shard_buffers b;
  float* exp_avg;
  float* exp_avg_sq;
  int n_groups;
  long long group_end[kShardMaxGroups];  // exclusive end of each parameter group
  float step_size[kShardMaxGroups];
  float clamp_lo[kShardMaxGroups], clamp_hi[kShardMaxGroups];
  unsigned clamp_mask;  // bit k: group k's parameters are clamped after the update
  float bc2_sqrt, beta1, beta2, one_minus_beta1, one_minus_beta2, eps, grad_scale;
};

__device__ __forceinline__ float4 mm_ld_reduce_add_v4(const float* mc) {
  float4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}

__device__ __forceinline__ void mm_st_v4(float* mc, float4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc),
               "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

__device__ __forceinline__ unsigned mm_ld_reduce_max_u32(const unsigned* mc) {
  unsigned v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.max.u32 %0, [%1];"
               : "=r"(v)
               : "l"(mc)
               : "memory");
  return v;
}

__device__ __forceinline__ void mm_st_u32(unsigned* mc, unsigned v) {
  asm volatile("multimem.st.relaxed.sys.global.b32 [%0], %1;" ::"l"(mc), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_proxy_alias() {
  asm volatile("fence.proxy.alias;" ::: "memory");
}

__device__ __forceinline__ unsigned cas_release_sys(unsigned* p, unsigned cmp, unsigned val) {
  unsigned old;
  asm volatile("atom.release.sys.global.cas.b32 %0, [%1], %2, %3;"
               : "=r"(old)
               : "l"(p), "r"(cmp), "r"(val)
               : "memory");
  return old;
}

__device__ __forceinline__ unsigned cas_acquire_sys(unsigned* p, unsigned cmp, unsigned val) {
  unsigned old;
  asm volatile("atom.acquire.sys.global.cas.b32 %0, [%1], %2, %3;"
               : "=r"(old)
               : "l"(p), "r"(cmp), "r"(val)
               : "memory");
  return old;
}

constexpr unsigned long long kPeerWaitNs = 5000000000ull;  // default limit of a barrier wait
constexpr unsigned kPeerSpinLimit = 1u << 26;                // and never more iterations

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Barrier between CTA blockIdx.x of every rank. Slot (block, src) of rank dst's signal pad
// carries src's arrival: the sender turns it 0 -> 1, the receiver 1 -> 0, so the slots are
// reusable barrier after barrier. Returns false (and raises kErrPeerTimeout) if a wait ran out.
__device__ bool peer_barrier(const ShardArgs& a) {
  __shared__ int s_ok;
  __syncthreads();
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  const int world = a.b.world, rank = a.b.rank;
  if (threadIdx.x < world) {
    const int peer = threadIdx.x;
    unsigned* const* pads = reinterpret_cast<unsigned* const*>(a.b.signal_pads);
    const long long slot = (long long)blockIdx.x * world;
    unsigned* out = pads[peer] + slot + rank;
    unsigned* in = pads[rank] + slot + peer;
    unsigned spins = 0;
    bool ok = true;
    const unsigned long long limit = a.b.wait_ns ? a.b.wait_ns : kPeerWaitNs;
    const unsigned long long t0 = global_ns();
    __threadfence_system();
    while (cas_release_sys(out, 0u, 1u) != 0u) {
      if (++spins > kPeerSpinLimit || global_ns() - t0 > limit) { ok = false; break; }
      __nanosleep(64);
    }
    while (ok && cas_acquire_sys(in, 1u, 0u) != 1u) {
      if (++spins > kPeerSpinLimit || global_ns() - t0 > limit) { ok = false; break; }
      __nanosleep(64);
    }
    if (!ok) {
      raise_device_error(kErrPeerTimeout);
      atomicAnd(&s_ok, 0);
    }
  }
  __syncthreads();
  return s_ok != 0;
}

__device__ __forceinline__ void adam_lane(const ShardArgs& a, long long idx, float g, float& p,
                                          float& m, float& v) {
  int grp = 0;
#pragma unroll
  for (int k = 0; k < kShardMaxGroups - 1; ++k)
    if (k < a.n_groups - 1 && idx >= a.group_end[k]) grp = k + 1;
  g *= a.grad_scale;
  m = m + a.one_minus_beta1 * (g - m);
  v = a.beta2 * v + a.one_minus_beta2 * g * g;
  const float denom = sqrtf(v) / a.bc2_sqrt + a.eps;
  p -= a.step_size[grp] * (m / denom);
  if ((a.clamp_mask >> grp) & 1u) p = fminf(fmaxf(p, a.clamp_lo[grp]), a.clamp_hi[grp]);
}

__device__ __forceinline__ void mark_phase(const gs_shard_buffers& b, int k) {
  if (b.phase_ns && threadIdx.x == 0) {
    const unsigned long long t = global_ns();
    if (k == 0)
      atomicMin(b.phase_ns, t);
    else
      atomicMax(b.phase_ns + k, t);
  }
}

// Two CTAs per SM: the grid is two CTAs per SM and every CTA waits at the barriers for the CTA
// of the same index on the other GPUs, so the whole grid must be resident at once; the launch
// bound keeps the registers within what two CTAs of 256 threads may use.
template <bool kMulticast>
__global__ void __launch_bounds__(kShardThreads, 2) sharded_adam_kernel(ShardArgs a) {
  const gs_shard_buffers& b = a.b;
  mark_phase(b, 0);
  if (!peer_barrier(a)) return;
  mark_phase(b, 1);
  fence_proxy_alias();
  const long long lo = (long long)b.rank * b.shard, hi = lo + b.shard;
  const long long data_end = min(hi, b.stats_offset + b.n_stats);
  const long long stride = 4ll * gridDim.x * blockDim.x;
  // kShardUnroll 16-byte groups per thread and iteration: all reductions are issued before the
  // first update so that several NVLink round trips are in flight per thread
  for (long long i0 = lo + 4ll * ((long long)blockIdx.x * blockDim.x + threadIdx.x);
       i0 < data_end; i0 += kShardUnroll * stride) {
    float4 g[kShardUnroll], pp[kShardUnroll], mm[kShardUnroll], vv[kShardUnroll];
#pragma unroll
    for (int u = 0; u < kShardUnroll; ++u) {
      const long long i = i0 + u * stride;
      g[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i >= data_end) continue;
      if (i < b.stats_offset) {  // this rank's parameters and moments, loaded alongside
        pp[u] = *reinterpret_cast<const float4*>(b.params + i);
        mm[u] = *reinterpret_cast<const float4*>(a.exp_avg + (i - lo));
        vv[u] = *reinterpret_cast<const float4*>(a.exp_avg_sq + (i - lo));
      }
      if (kMulticast) {
        g[u] = mm_ld_reduce_add_v4(b.bucket_mc + i);
      } else {
        for (int r = 0; r < b.world; ++r) {
          const float4 x = *reinterpret_cast<const float4*>(
              static_cast<const float*>(b.bucket_peers[r]) + i);
          g[u].x += x.x;
          g[u].y += x.y;
          g[u].z += x.z;
          g[u].w += x.w;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kShardUnroll; ++u) {
      const long long i = i0 + u * stride;
      if (i >= data_end) continue;
      const bool is_param = i < b.stats_offset;
      float4 out = g[u];
      if (is_param) {
        float4 p = pp[u], m = mm[u], v = vv[u];
        if (i + 0 < b.n_param) adam_lane(a, i + 0, g[u].x, p.x, m.x, v.x);
        if (i + 1 < b.n_param) adam_lane(a, i + 1, g[u].y, p.y, m.y, v.y);
        if (i + 2 < b.n_param) adam_lane(a, i + 2, g[u].z, p.z, m.z, v.z);
        if (i + 3 < b.n_param) adam_lane(a, i + 3, g[u].w, p.w, m.w, v.w);
        *reinterpret_cast<float4*>(a.exp_avg + (i - lo)) = m;
        *reinterpret_cast<float4*>(a.exp_avg_sq + (i - lo)) = v;
        out = p;
      }
      float* dst_mc = is_param ? b.params_mc : b.bucket_mc;
      void* const* dst_peers = is_param ? b.params_peers : b.bucket_peers;
      if (kMulticast) {
        mm_st_v4(dst_mc + i, out);
      } else {
        for (int r = 0; r < b.world; ++r)
          *reinterpret_cast<float4*>(static_cast<float*>(dst_peers[r]) + i) = out;
      }
    }
  }
  // max statistic
  const long long mlo = (long long)b.rank * b.max_shard;
  const long long mhi = min(mlo + b.max_shard, b.n_max);
  for (long long i = mlo + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < mhi;
       i += (long long)gridDim.x * blockDim.x) {
    unsigned m;
    if (kMulticast) {
      m = mm_ld_reduce_max_u32(reinterpret_cast<const unsigned*>(b.max_mc) + i);
      mm_st_u32(reinterpret_cast<unsigned*>(b.max_mc) + i, m);
    } else {
      m = 0u;
      for (int r = 0; r < b.world; ++r)
        m = max(m, static_cast<const unsigned*>(b.max_peers[r])[i]);
      for (int r = 0; r < b.world; ++r) static_cast<unsigned*>(b.max_peers[r])[i] = m;
    }
  }
  fence_proxy_alias();
  mark_phase(b, 2);
  peer_barrier(a);
  mark_phase(b, 3);
  fence_proxy_alias();
}

// SM count of the current device, looked up once per device ordinal.
int sm_count_cached() {
  constexpr int kMaxDevices = 64;
  static std::atomic<int> counts[kMaxDevices];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) dev = 0;
  int count = counts[dev].load(std::memory_order_relaxed);
  if (count == 0) {
    cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev);
    if (count <= 0) count = 148;
    counts[dev].store(count, std::memory_order_relaxed);
  }
  return count;
}

}  // namespace gs

using namespace gs;

extern "C" int gs_sharded_adam_step(const gs_shard_buffers* bufs, float* exp_avg,
                                    float* exp_avg_sq, int n_groups, const long long* group_sizes,
                                    const float* lrs, double beta1, double beta2, double eps,
                                    long long step, float grad_scale, const float* clamp_min,
                                    const float* clamp_max, void* stream) {
  GS_API_BEGIN();
  GS_REQUIRE(bufs, "null buffer description");
  const gs_shard_buffers& b = *bufs;
  GS_REQUIRE(b.world >= 1 && b.world <= kShardMaxWorld, "world size must be in [1, 8]");
  GS_REQUIRE(b.rank >= 0 && b.rank < b.world, "rank out of range");
  GS_REQUIRE(b.shard > 0 && b.shard % 4 == 0, "shard must be a positive multiple of 4");
  GS_REQUIRE(b.n_param >= 0 && b.stats_offset >= b.n_param && b.stats_offset % 4 == 0 &&
                 b.n_stats >= 0 && b.stats_offset + b.n_stats <= b.shard * b.world,
             "bucket layout does not fit the shards");
  GS_REQUIRE(b.n_max >= 0 && b.max_shard >= 0 && b.max_shard * b.world >= b.n_max,
             "max-statistic layout does not fit the shards");
  GS_REQUIRE(b.bucket && b.params && b.signal_pads && exp_avg && exp_avg_sq, "null pointer");
  GS_REQUIRE(b.n_max == 0 || b.maxbuf, "null max-statistic buffer");
  const bool mc = b.bucket_mc && b.params_mc && (b.n_max == 0 || b.max_mc);
  GS_REQUIRE(mc || (b.bucket_peers && b.params_peers && (b.n_max == 0 || b.max_peers)),
             "need multicast pointers or peer pointer arrays");
  GS_REQUIRE(((reinterpret_cast<uintptr_t>(b.bucket) | reinterpret_cast<uintptr_t>(b.params) |
               reinterpret_cast<uintptr_t>(exp_avg) | reinterpret_cast<uintptr_t>(exp_avg_sq)) &
              15u) == 0,
             "buffers must be 16-byte aligned");
  GS_REQUIRE(n_groups >= 1 && n_groups <= kShardMaxGroups, "n_groups must be in [1, 8]");
  GS_REQUIRE(group_sizes && lrs, "null group table");
  GS_REQUIRE(step >= 1, "step must be >= 1");
  GS_REQUIRE(beta1 >= 0.0 && beta1 < 1.0 && beta2 >= 0.0 && beta2 < 1.0,
             "betas must be in [0, 1)");
  ShardArgs a{};
  a.b = b;
  a.exp_avg = exp_avg;
  a.exp_avg_sq = exp_avg_sq;
  a.n_groups = n_groups;
  long long end = 0;
  const double bc1 = 1.0 - std::pow(beta1, (double)step);
  for (int k = 0; k < n_groups; ++k) {
    GS_REQUIRE(group_sizes[k] >= 0, "negative group size");
    end += group_sizes[k];
    a.group_end[k] = end;
    a.step_size[k] = (float)((double)lrs[k] / bc1);
    a.clamp_lo[k] = clamp_min ? clamp_min[k] : -INFINITY;
    a.clamp_hi[k] = clamp_max ? clamp_max[k] : INFINITY;
    GS_REQUIRE(!(a.clamp_lo[k] > a.clamp_hi[k]), "clamp_min above clamp_max");
    if (a.clamp_lo[k] > -INFINITY || a.clamp_hi[k] < INFINITY) a.clamp_mask |= 1u << k;
  }
  GS_REQUIRE(end == b.n_param, "group sizes must add up to n_param");
  a.bc2_sqrt = (float)std::sqrt(1.0 - std::pow(beta2, (double)step));
  a.beta1 = (float)beta1;
  a.beta2 = (float)beta2;
  a.one_minus_beta1 = (float)(1.0 - beta1);
  a.one_minus_beta2 = (float)(1.0 - beta2);
  a.eps = (float)eps;
  a.grad_scale = grad_scale;
  const int grid = (int)std::min<long long>(2ll * sm_count_cached(), b.signal_slots / b.world);
  GS_REQUIRE(grid >= 1, "signal pad too small");
  cudaStream_t st = (cudaStream_t)stream;
  if (mc)
    sharded_adam_kernel<true><<<grid, kShardThreads, 0, st>>>(a);
  else
    sharded_adam_kernel<false><<<grid, kShardThreads, 0, st>>>(a);
  GS_CHECK_LAUNCH();
  return GS_OK;
  GS_API_END();
}
