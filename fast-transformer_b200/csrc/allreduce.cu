// Tensor-parallel all-reduce producer for split-K projections (sm_100a).
//
// fb_reduce_push sums a projection's fp32 split-K partials [S, M, N] in split order (the
// projection's own arithmetic, as a single-split epilogue would see it) and stores every
// value, as one 8-byte word with the flag (uint32)(*epoch) + 1 in its high half, into slab
// `rank` of recv[use] on every rank - the low-latency push protocol that
// fb_allreduce_add_rmsnorm polls. The decode step's producer whenever the projection has K
// splits: on B200, summing the splits inside the projection (cluster reduction or the split
// fix-up) and pushing from its epilogue, or pushing from the polling kernel itself
// (fb_reduce_push_add_rmsnorm), each measured slower than split partials plus this pass.
#include "common.cuh"

namespace fb {
namespace ar {

constexpr int kThreads = 128;
constexpr int kBatch = 8;  // split slabs in flight per thread
constexpr int kMaxWorld = 8;

struct Params {
  const float* partials;  // [splits, m, n]
  int splits, m, n, world, rank, use;
  uint64_t* peer_recv[kMaxWorld];
  uint64_t* mc_recv;  // multicast address of the receive buffers (NVSwitch), or null
  const int64_t* epoch;
};

// Two values per thread, so one store instruction of a warp writes 512 contiguous bytes
// (32 lanes x one 16-byte pair of flagged words) to each peer.
__global__ void __launch_bounds__(kThreads) reduce_push_kernel(const __grid_constant__ Params p) {
  pdl_wait();
  pdl_trigger();
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) * 2;
  const int64_t count = static_cast<int64_t>(p.m) * p.n;
  if (i >= count) return;
  float2 x = make_float2(0.f, 0.f);
  for (int s0 = 0; s0 < p.splits; s0 += kBatch) {
    float2 part[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j)
      if (s0 + j < p.splits) part[j] = __ldcg(reinterpret_cast<const float2*>(p.partials + (s0 + j) * count + i));
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      if (s0 + j == 0) {
        x = part[0];
      } else if (s0 + j < p.splits) {
        x.x += part[j].x;
        x.y += part[j].y;
      }
    }
  }
  const uint64_t flag = static_cast<uint64_t>(static_cast<uint32_t>(*p.epoch) + 1u) << 32;
  const uint64_t w0 = flag | __float_as_uint(x.x), w1 = flag | __float_as_uint(x.y);
  const size_t off = (static_cast<size_t>(p.use) * p.world + p.rank) * count + i;
  if (p.mc_recv != nullptr) {
    // one store per word through the multicast address: NVSwitch delivers it to every rank
    asm volatile("multimem.st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p.mc_recv + off), "l"(w0) : "memory");
    asm volatile("multimem.st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p.mc_recv + off + 1), "l"(w1) : "memory");
  } else {
    for (int q = 0; q < p.world; ++q)
      asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p.peer_recv[q] + off), "l"(w0), "l"(w1)
                   : "memory");
  }
}

}  // namespace ar
}  // namespace fb

using namespace fb;

extern "C" int fb_reduce_push(const void* partials, int splits, int m, int n, int world, int rank, int use,
                              void* const* peer_recv, void* multicast_recv, const int64_t* epoch, void* stream) {
  if (!partials || !peer_recv || !epoch || splits <= 0 || m <= 0 || n <= 0) return FB_ERR_ARG;
  if (world < 1 || world > ar::kMaxWorld || rank < 0 || rank >= world || use < 0) return FB_ERR_ARG;
  if (n % 2 != 0) return FB_ERR_SHAPE;
  ar::Params p{};
  p.partials = static_cast<const float*>(partials);
  p.splits = splits;
  p.m = m;
  p.n = n;
  p.world = world;
  p.rank = rank;
  p.use = use;
  p.epoch = epoch;
  if (multicast_recv != nullptr && (reinterpret_cast<uintptr_t>(multicast_recv) & 15u)) return FB_ERR_ARG;
  p.mc_recv = static_cast<uint64_t*>(multicast_recv);
  for (int r = 0; r < world; ++r) {
    if (!peer_recv[r] || (reinterpret_cast<uintptr_t>(peer_recv[r]) & 15u)) return FB_ERR_ARG;
    p.peer_recv[r] = static_cast<uint64_t*>(peer_recv[r]);
  }
  const int64_t threads = (static_cast<int64_t>(m) * n + 1) / 2;
  const int64_t blocks = (threads + ar::kThreads - 1) / ar::kThreads;
  if (blocks >= (1ll << 31)) return FB_ERR_SHAPE;
  return launch_ex(ar::reduce_push_kernel, dim3(static_cast<unsigned>(blocks)), dim3(ar::kThreads), 0,
                   static_cast<cudaStream_t>(stream), 1, p);
}
