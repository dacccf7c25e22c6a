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
#include "optim_math.cuh"

namespace b200 {
namespace peer {

constexpr int PT = 512;  // threads per block
constexpr int MAXS = 64;  // parameter segments of a fused optimizer epilogue

// Optional optimizer epilogue: the summed values are the gradients of `count` parameter
// tensors laid end to end, segment j covering [off[j], off[j + 1]); each summed element
// also updates its parameter and state elements in place.
struct Segs {
  int count, kind;
  opt::Consts k;
  int64_t off[MAXS + 1];
  float* p[MAXS];
  float* s1[MAXS];
  float* s2[MAXS];
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__global__ void __launch_bounds__(PT) peer_allreduce_kernel(float* __restrict__ data, int64_t n, int64_t chunk,
                                                            const uint64_t* __restrict__ slots, const uint64_t* __restrict__ pads,
                                                            int rank, int world, uint32_t* __restrict__ epoch,
                                                            int* __restrict__ status, int64_t spin_limit, float scale,
                                                            const __grid_constant__ Segs S) {
  __shared__ int s_err;
  const int b = blockIdx.x, tid = threadIdx.x;
  const int64_t lo = (int64_t)b * chunk, hi = min(n, lo + chunk);
  const uint32_t e = epoch[b] + 1u;
  const int64_t off = (int64_t)(e & 1u) * n;
  float* mine = reinterpret_cast<float*>(slots[rank]) + off;
  if (tid == 0) s_err = 0;
  for (int64_t i = lo + tid; i < hi; i += PT) mine[i] = data[i];
  // The block's slot writes are ordered before the flag by the barrier and the flag's
  // system-scope release (release is cumulative over what the releasing thread has
  // synchronised with); likewise one acquire fence after the last poll, then the barrier,
  // orders the peers' slot writes before every thread's reads.
  __syncthreads();
  if (tid < world && tid != rank) {
    // tell peer `tid` that this rank's chunk b of call e is in place ...
    st_release_sys(reinterpret_cast<uint32_t*>(pads[tid]) + (size_t)b * world + rank, e);
    // ... and wait until peer `tid` has said the same to this rank
    const uint32_t* f = reinterpret_cast<const uint32_t*>(pads[rank]) + (size_t)b * world + tid;
    int64_t it = 0;
    while ((int32_t)(ld_relaxed_sys(f) - e) < 0) {
      if (++it > spin_limit) {
        s_err = 1;
        atomicExch(status, B200_ERR_TIMEOUT);
        break;
      }
      if (it > 32) __nanosleep(it > 4096 ? 256 : 32);
    }
    fence_acq_rel_sys();
  }
  __syncthreads();
  if (s_err) return;
  for (int64_t i = lo + tid; i < hi; i += PT) {
    float s = 0.f;
#pragma unroll 8
    for (int q = 0; q < world; ++q) s += reinterpret_cast<const float*>(slots[q])[off + i];
    const float g = s * scale;
    data[i] = g;
    if (S.count > 0) {  // the parameter segment of element i (binary search), then its update
      int lo_s = 0, hi_s = S.count - 1;
      while (lo_s < hi_s) {
        const int mid = (lo_s + hi_s + 1) >> 1;
        if (S.off[mid] <= i) lo_s = mid;
        else hi_s = mid - 1;
      }
      const int64_t j = i - S.off[lo_s];
      float* p = S.p[lo_s];
      float* a = S.s1[lo_s];
      float* b = S.s2[lo_s];
      float po, ao, bo;
      opt::update(S.kind, S.k, p[j], a[j], b ? b[j] : 0.f, g, po, ao, bo);
      p[j] = po;
      a[j] = ao;
      if (b) b[j] = bo;
    }
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

static int peer_launch(float* data, int64_t n, const void* slots_dev, const void* pads_dev, int rank, int world, unsigned int* epoch,
                       int* status, int64_t spin_limit, float scale, int blocks, const peer::Segs& S, void* stream) {
  B200_REQUIRE(data && slots_dev && pads_dev && epoch && status, "peer_allreduce: null pointer");
  B200_REQUIRE(n >= 0 && world >= 1 && world <= 64 && rank >= 0 && rank < world, "peer_allreduce: bad rank %d / world %d", rank,
               world);
  B200_REQUIRE(blocks >= 1 && blocks <= 64, "peer_allreduce: blocks %d not in [1, 64]", blocks);
  B200_REQUIRE(spin_limit > 0, "peer_allreduce: spin_limit must be positive");
  if (n == 0) return B200_OK;
  const int64_t chunk = ceil_div(n, (int64_t)blocks);
  peer::peer_allreduce_kernel<<<blocks, peer::PT, 0, as_stream(stream)>>>(
      data, n, chunk, reinterpret_cast<const uint64_t*>(slots_dev), reinterpret_cast<const uint64_t*>(pads_dev), rank, world,
      reinterpret_cast<uint32_t*>(epoch), status, spin_limit, scale, S);
  return check_launch("peer_allreduce");
}

extern "C" int b200_peer_allreduce_f32(float* data, int64_t n, const void* slots_dev, const void* pads_dev, int rank, int world,
                                       unsigned int* epoch, int* status, int64_t spin_limit, float scale, int blocks,
                                       void* stream) {
  peer::Segs S;
  S.count = 0;
  return peer_launch(data, n, slots_dev, pads_dev, rank, world, epoch, status, spin_limit, scale, blocks, S, stream);
}

extern "C" int b200_peer_allreduce_apply_f32(float* data, int64_t n, const void* slots_dev, const void* pads_dev, int rank,
                                             int world, unsigned int* epoch, int* status, int64_t spin_limit, float scale,
                                             int blocks, int kind, int count, const int64_t* offsets, float* const* param,
                                             float* const* s1, float* const* s2, float lr, void* stream) {
  B200_REQUIRE(kind >= 0 && kind <= 3, "peer_allreduce_apply: kind %d not in [0, 3]", kind);
  B200_REQUIRE(count >= 1 && count <= peer::MAXS, "peer_allreduce_apply: %d segments not in [1, %d]", count, peer::MAXS);
  B200_REQUIRE(offsets && param && s1, "peer_allreduce_apply: null table");
  B200_REQUIRE(offsets[0] == 0 && offsets[count] == n, "peer_allreduce_apply: segments must cover [0, n) exactly");
  const bool two = kind != opt::ADAGRAD;
  B200_REQUIRE(!two || s2, "peer_allreduce_apply: this optimizer has a second state array");
  peer::Segs S;
  S.count = count;
  S.kind = kind;
  S.k = opt::consts_for(kind, lr);
  for (int j = 0; j < count; ++j) {
    B200_REQUIRE(offsets[j + 1] >= offsets[j], "peer_allreduce_apply: offsets must not decrease");
    B200_REQUIRE(param[j] && s1[j] && (!two || s2[j]), "peer_allreduce_apply: null pointer for segment %d", j);
    S.off[j] = offsets[j];
    S.p[j] = param[j];
    S.s1[j] = s1[j];
    S.s2[j] = two ? s2[j] : nullptr;
  }
  S.off[count] = offsets[count];
  return peer_launch(data, n, slots_dev, pads_dev, rank, world, epoch, status, spin_limit, scale, blocks, S, stream);
}

extern "C" int b200_memset_async(void* p, int value, size_t bytes, void* stream) {
  B200_REQUIRE(p || bytes == 0, "memset: null pointer");
  if (bytes) cudaMemsetAsync(p, value, bytes, as_stream(stream));
  return check_launch("memset");
}
