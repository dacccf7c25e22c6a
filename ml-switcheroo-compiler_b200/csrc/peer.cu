// Small-gradient all-reduce through peer-mapped memory over NVLink, one kernel, in the
// low-latency style: every value travels with its call number in one 64-bit word
// (call << 32 | value bits). A 64-bit store is single-copy atomic, so a receiver that sees
// the current call number in a word also sees the value written with it, with no fences
// and no separate flags. Each rank pushes its values into every peer's receive area
// (remote stores), then polls its own receive area (local loads) and adds all ranks'
// values in rank order, so every rank computes the same sum in the same order: the result
// is identical on all ranks and run to run. It replaces NCCL for the buckets of small
// gradients (the reference's AllReduce node, numpy/eager/distributed.py:205-225), where a
// collective's fixed latency, not bandwidth, sets the cost.
//
// Receive area of a rank: [2 halves][world sources][capacity] words in a symmetric buffer
// that every rank maps. Block b owns a chunk of the values and has its own call counter
// (`epoch[b]`, advanced by the block); call e writes half e & 1. A sender starts call e
// only after its call e - 1 received every peer's words, and a peer sends those only after
// its call e - 2 (the last reader of that half) has finished on its stream, so a half is
// never overwritten while it is read. Words of older calls carry older call numbers, so the
// area is cleared once at set-up and never again. A wait gives up after `spin_limit` polls
// per thread: the block records B200_ERR_TIMEOUT in `status`, leaves its values
// unchanged and does not advance its call number.
//
// A timeout is fatal for the exchange. After one, the ranks disagree on call numbers (a
// peer that received this rank's words did advance), so a later call could find a peer's
// words of the previous call under the number it expects and add stale values. Every
// block therefore reads `status` first and returns without sending, summing or advancing
// when it is non-zero: a rank that timed out stops exchanging, and its peers' next waits
// time out in turn, so every rank ends with the status set and no rank sums stale words.
// Only a collective reset (receive areas cleared, call numbers and status zeroed on every
// rank) re-opens the exchange. With the optimizer epilogue, parameters may differ across
// ranks after a timeout: the blocks that completed on one rank updated them.
#include <algorithm>

#include "common.cuh"
#include "optim_math.cuh"

namespace b200 {
namespace peer {

constexpr int PT = 512;  // threads per block
constexpr int MAXS = 64;  // parameter segments of a fused optimizer epilogue
constexpr int MAXB = 64;  // blocks (call counters) per launch

// Segments: the values are `count` tensors laid end to end, segment j covering
// [off[j], off[j + 1]); they are read from and written back to those tensors (`direct`),
// and / or, with an optimizer, they are the gradients of the parameters p[j] and each
// summed element also updates its parameter and state elements in place.
struct Segs {
  int count;   // segments; 0: one flat buffer and no optimizer
  int kind;    // optimizer kind, -1 for none
  int direct;  // the values live in the segments' own tensors d[j], not in one flat buffer
  opt::Consts k;
  int64_t off[MAXS + 1];
  float* d[MAXS];
  float* p[MAXS];
  float* s1[MAXS];
  float* s2[MAXS];
};

// the segment holding element i: the last j with off[j] <= i
__device__ __forceinline__ int seg_of(const Segs& S, int64_t i) {
  int lo = 0, hi = S.count - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (S.off[mid] <= i) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

constexpr int EPT = 8;  // values per thread: a block covers PT * EPT values

__device__ __forceinline__ void st_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(PT) peer_allreduce_kernel(float* __restrict__ data, int64_t n, const uint64_t* __restrict__ bufs,
                                                            int64_t cap, int rank, int world, uint32_t* __restrict__ epoch,
                                                            int* __restrict__ status, int64_t spin_limit, float scale,
                                                            const __grid_constant__ Segs S) {
  const int b = blockIdx.x, tid = threadIdx.x;
  // fail-stop: a rank whose exchange timed out before sends, sums and advances nothing
  if (*reinterpret_cast<volatile const int*>(status) != 0) return;
  const int64_t lo = (int64_t)b * PT * EPT;
  const uint32_t e = epoch[b] + 1u;
  const int64_t half = (int64_t)(e & 1u) * world;
  float mine[EPT];
  // push this rank's values into every peer's receive area
#pragma unroll
  for (int k = 0; k < EPT; ++k) {
    const int64_t i = lo + (int64_t)k * PT + tid;
    if (i < n) {
      if (S.direct) {
        const int j = seg_of(S, i);
        mine[k] = S.d[j][i - S.off[j]];
      } else {
        mine[k] = data[i];
      }
    } else {
      mine[k] = 0.f;
    }
    if (i < n) {
      const uint64_t w = ((uint64_t)e << 32) | (uint64_t)__float_as_uint(mine[k]);
      for (int q = 0; q < world; ++q)
        if (q != rank) st_sys_u64(reinterpret_cast<uint64_t*>(bufs[q]) + (half + rank) * cap + i, w);
    }
  }
  // receive: add all ranks' values in rank order
  const uint64_t* in = reinterpret_cast<const uint64_t*>(bufs[rank]);
  float sum[EPT];
  int64_t it = 0;
  bool err = false;
#pragma unroll
  for (int k = 0; k < EPT; ++k) {
    const int64_t i = lo + (int64_t)k * PT + tid;
    float acc = 0.f;
    if (i < n) {
      for (int q = 0; q < world && !err; ++q) {
        float v;
        if (q == rank) {
          v = mine[k];
        } else {
          const uint64_t* src = in + (half + q) * cap + i;
          uint64_t w = ld_sys_u64(src);
          while ((uint32_t)(w >> 32) != e) {
            if (++it > spin_limit) {
              err = true;
              break;
            }
            if (it > 64) __nanosleep(it > 8192 ? 256 : 32);
            w = ld_sys_u64(src);
          }
          v = __uint_as_float((uint32_t)w);
        }
        acc += v;
      }
    }
    sum[k] = acc;
  }
  if (err) atomicExch(status, B200_ERR_TIMEOUT);
  // every thread of the block learns whether any wait gave up (one barrier, no shared flag)
  if (__syncthreads_or(err ? 1 : 0)) return;
#pragma unroll
  for (int k = 0; k < EPT; ++k) {
    const int64_t i = lo + (int64_t)k * PT + tid;
    if (i >= n) continue;
    const float g = sum[k] * scale;
    const int j = S.count > 0 ? seg_of(S, i) : 0;
    const int64_t jj = S.count > 0 ? i - S.off[j] : i;
    if (S.direct) S.d[j][jj] = g;
    else data[i] = g;
    if (S.kind >= 0) {  // optimizer step on element jj of parameter tensor j
      float* p = S.p[j];
      float* a = S.s1[j];
      float* bb = S.s2[j];
      float po, ao, bo;
      opt::update(S.kind, S.k, p[jj], a[jj], bb ? bb[jj] : 0.f, g, po, ao, bo);
      p[jj] = po;
      a[jj] = ao;
      if (bb) bb[jj] = bo;
    }
  }
  if (tid == 0) epoch[b] = e;
}

}  // namespace peer
}  // namespace b200

using namespace b200;

extern "C" int b200_peer_allreduce_blocks(int64_t n) {
  return n <= 0 ? 0 : (int)ceil_div(n, (int64_t)peer::PT * peer::EPT);
}

static int peer_launch(float* data, int64_t n, const void* bufs_dev, int64_t capacity, int rank, int world, unsigned int* epoch,
                       int* status, int64_t spin_limit, float scale, const peer::Segs& S, void* stream) {
  B200_REQUIRE((data || S.direct) && bufs_dev && epoch && status, "peer_allreduce: null pointer");
  B200_REQUIRE(n >= 0 && world >= 1 && world <= 64 && rank >= 0 && rank < world, "peer_allreduce: bad rank %d / world %d", rank,
               world);
  B200_REQUIRE(n <= capacity, "peer_allreduce: %lld values above the receive capacity %lld", (long long)n, (long long)capacity);
  B200_REQUIRE(spin_limit > 0, "peer_allreduce: spin_limit must be positive");
  if (n == 0) return B200_OK;
  const int blocks = b200_peer_allreduce_blocks(n);
  B200_REQUIRE(blocks <= peer::MAXB, "peer_allreduce: %lld values need %d blocks, above %d", (long long)n, blocks, peer::MAXB);
  peer::peer_allreduce_kernel<<<blocks, peer::PT, 0, as_stream(stream)>>>(data, n, reinterpret_cast<const uint64_t*>(bufs_dev),
                                                                          capacity, rank, world, reinterpret_cast<uint32_t*>(epoch),
                                                                          status, spin_limit, scale, S);
  return check_launch("peer_allreduce");
}

extern "C" int b200_peer_allreduce_f32(float* data, int64_t n, const void* bufs_dev, int64_t capacity, int rank, int world,
                                       unsigned int* epoch, int* status, int64_t spin_limit, float scale, void* stream) {
  peer::Segs S;
  S.count = 0;
  S.kind = -1;
  S.direct = 0;
  return peer_launch(data, n, bufs_dev, capacity, rank, world, epoch, status, spin_limit, scale, S, stream);
}

extern "C" int b200_peer_allreduce_apply_f32(float* data, int64_t n, const void* bufs_dev, int64_t capacity, int rank, int world,
                                             unsigned int* epoch, int* status, int64_t spin_limit, float scale, int kind, int count,
                                             const int64_t* offsets, float* const* param, float* const* s1, float* const* s2,
                                             float lr, void* stream) {
  B200_REQUIRE(kind >= 0 && kind <= 3, "peer_allreduce_apply: kind %d not in [0, 3]", kind);
  B200_REQUIRE(count >= 1 && count <= peer::MAXS, "peer_allreduce_apply: %d segments not in [1, %d]", count, peer::MAXS);
  B200_REQUIRE(offsets && param && s1, "peer_allreduce_apply: null table");
  B200_REQUIRE(offsets[0] == 0 && offsets[count] == n, "peer_allreduce_apply: segments must cover [0, n) exactly");
  const bool two = kind != opt::ADAGRAD;
  B200_REQUIRE(!two || s2, "peer_allreduce_apply: this optimizer has a second state array");
  peer::Segs S;
  S.count = count;
  S.kind = kind;
  S.direct = 0;
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
  return peer_launch(data, n, bufs_dev, capacity, rank, world, epoch, status, spin_limit, scale, S, stream);
}

// The same exchange over `count` (<= 64) tensors laid end to end without packing them:
// values are read from and the sums written back to tensors[j], which covers
// [offsets[j], offsets[j + 1]). kind >= 0 adds the optimizer epilogue on param / s1 / s2
// (as b200_peer_allreduce_apply_f32); kind -1 is the plain sum.
extern "C" int b200_peer_allreduce_tensors_f32(int count, const int64_t* offsets, float* const* tensors, const void* bufs_dev,
                                               int64_t capacity, int rank, int world, unsigned int* epoch, int* status,
                                               int64_t spin_limit, float scale, int kind, float* const* param,
                                               float* const* s1, float* const* s2, float lr, void* stream) {
  B200_REQUIRE(count >= 1 && count <= peer::MAXS, "peer_allreduce_tensors: %d tensors not in [1, %d]", count, peer::MAXS);
  B200_REQUIRE(offsets && tensors && offsets[0] == 0, "peer_allreduce_tensors: null table or offsets[0] != 0");
  B200_REQUIRE(kind >= -1 && kind <= 3, "peer_allreduce_tensors: kind %d not in [-1, 3]", kind);
  const bool opt_on = kind >= 0, two = kind >= 0 && kind != opt::ADAGRAD;
  B200_REQUIRE(!opt_on || (param && s1 && (!two || s2)), "peer_allreduce_tensors: optimizer tables missing");
  peer::Segs S;
  S.count = count;
  S.kind = kind;
  S.direct = 1;
  S.k = opt::consts_for(opt_on ? kind : 0, lr);
  for (int j = 0; j < count; ++j) {
    B200_REQUIRE(offsets[j + 1] >= offsets[j], "peer_allreduce_tensors: offsets must not decrease");
    B200_REQUIRE(offsets[j + 1] == offsets[j] || tensors[j], "peer_allreduce_tensors: null tensor %d", j);
    B200_REQUIRE(!opt_on || (param[j] && s1[j] && (!two || s2[j])), "peer_allreduce_tensors: null pointer for tensor %d", j);
    S.off[j] = offsets[j];
    S.d[j] = tensors[j];
    S.p[j] = opt_on ? param[j] : nullptr;
    S.s1[j] = opt_on ? s1[j] : nullptr;
    S.s2[j] = two ? s2[j] : nullptr;
  }
  S.off[count] = offsets[count];
  return peer_launch(nullptr, offsets[count], bufs_dev, capacity, rank, world, epoch, status, spin_limit, scale, S, stream);
}

extern "C" int b200_memset_async(void* p, int value, size_t bytes, void* stream) {
  B200_REQUIRE(p || bytes == 0, "memset: null pointer");
  if (bytes) cudaMemsetAsync(p, value, bytes, as_stream(stream));
  return check_launch("memset");
}
