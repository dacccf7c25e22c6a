// Small-gradient all-reduce through peer-mapped memory (NVLink P2P loads), one kernel:
// copy this rank's values into its slot of a symmetric buffer, raise a flag in every
// peer's signal pad, wait (bounded) for every peer's flag, then add all ranks' slots in
// rank order. Every rank computes the same sum in the same order, so the result is
// identical on all ranks and run to run. It replaces NCCL for the buckets of small
// gradients (the reference's AllReduce node, numpy/eager/distributed.py:205-225), where a
// collective's fixed latency, not bandwidth, sets the cost.
//
// Protocol. Block b owns a chunk of the values and pad slots [b * world, (b + 1) * world)
// of every pad. Its call number e (per block, kept in `epoch`, advanced by the block
// itself) selects the half of the slot buffer (e & 1), so a rank never overwrites values a
// slower peer may still read: rank r starts call e only after it saw every peer's flag of
// call e - 1, and a peer raises that flag only after its call e - 2 (the last reader of
// this half) has finished on its stream. Flags hold the call number and only grow, so no
// reset between calls. A wait gives up after `spin_limit` polls: the block records
// B200_ERR_TIMEOUT in `status`, leaves its values unchanged and does not advance its
// call number.
#include <algorithm>

#include "common.cuh"

namespace b200 {
namespace peer {

constexpr int PT = 512;  // threads per block

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(PT) peer_allreduce_kernel(float* __restrict__ data, int64_t n, int64_t chunk,
                                                            const uint64_t* __restrict__ slots, const uint64_t* __restrict__ pads,
                                                            int rank, int world, uint32_t* __restrict__ epoch,
                                                            int* __restrict__ status, int64_t spin_limit, float scale) {
  __shared__ int s_err;
  const int b = blockIdx.x, tid = threadIdx.x;
  const int64_t lo = (int64_t)b * chunk, hi = min(n, lo + chunk);
  const uint32_t e = epoch[b] + 1u;
  const int64_t off = (int64_t)(e & 1u) * n;
  float* mine = reinterpret_cast<float*>(slots[rank]) + off;
  if (tid == 0) s_err = 0;
  for (int64_t i = lo + tid; i < hi; i += PT) mine[i] = data[i];
  __threadfence_system();
  __syncthreads();
  if (tid < world && tid != rank) {
    // tell peer `tid` that this rank's chunk b of call e is in place ...
    st_release_sys(reinterpret_cast<uint32_t*>(pads[tid]) + (size_t)b * world + rank, e);
    // ... and wait until peer `tid` has said the same to this rank
    const uint32_t* f = reinterpret_cast<const uint32_t*>(pads[rank]) + (size_t)b * world + tid;
    int64_t it = 0;
    while ((int32_t)(ld_acquire_sys(f) - e) < 0) {
      if (++it > spin_limit) {
        s_err = 1;
        atomicExch(status, B200_ERR_TIMEOUT);
        break;
      }
      __nanosleep(128);
    }
  }
  __syncthreads();
  if (s_err) return;
  for (int64_t i = lo + tid; i < hi; i += PT) {
    float s = 0.f;
#pragma unroll 8
    for (int q = 0; q < world; ++q) s += reinterpret_cast<const float*>(slots[q])[off + i];
    data[i] = s * scale;
  }
  if (tid == 0) epoch[b] = e;
}

}  // namespace peer
}  // namespace b200

using namespace b200;

extern "C" int b200_peer_allreduce_blocks(int64_t n, int world, size_t pad_bytes) {
  if (n <= 0 || world < 1) return 0;
  const int64_t by_size = ceil_div(n, (int64_t)8192);
  const int64_t by_pad = (int64_t)(pad_bytes / (sizeof(uint32_t) * (size_t)world));
  return (int)std::max<int64_t>(1, std::min<int64_t>(std::min<int64_t>(by_size, by_pad), 64));
}

extern "C" int b200_peer_allreduce_f32(float* data, int64_t n, const void* slots_dev, const void* pads_dev, int rank, int world,
                                       unsigned int* epoch, int* status, int64_t spin_limit, float scale, int blocks,
                                       void* stream) {
  B200_REQUIRE(data && slots_dev && pads_dev && epoch && status, "peer_allreduce: null pointer");
  B200_REQUIRE(n >= 0 && world >= 1 && world <= 64 && rank >= 0 && rank < world, "peer_allreduce: bad rank %d / world %d", rank,
               world);
  B200_REQUIRE(blocks >= 1 && blocks <= 64, "peer_allreduce: blocks %d not in [1, 64]", blocks);
  B200_REQUIRE(spin_limit > 0, "peer_allreduce: spin_limit must be positive");
  if (n == 0) return B200_OK;
  const int64_t chunk = ceil_div(n, (int64_t)blocks);
  peer::peer_allreduce_kernel<<<blocks, peer::PT, 0, as_stream(stream)>>>(
      data, n, chunk, reinterpret_cast<const uint64_t*>(slots_dev), reinterpret_cast<const uint64_t*>(pads_dev), rank, world,
      reinterpret_cast<uint32_t*>(epoch), status, spin_limit, scale);
  return check_launch("peer_allreduce");
}

extern "C" int b200_memset_async(void* p, int value, size_t bytes, void* stream) {
  B200_REQUIRE(p || bytes == 0, "memset: null pointer");
  if (bytes) cudaMemsetAsync(p, value, bytes, as_stream(stream));
  return check_launch("memset");
}
