// Tensor-parallel all-reduce + add + RMSNorm over NVLink peer memory (sm_100a), owner-computes:
// a reduce-scatter of fp32 partials followed by an all-gather of the summed bf16 rows.
//
// The reference is single-GPU; this replaces the all-reduce a tensor-parallel decode step needs
// after o_proj and down_proj, and folds the residual add + RMSNorm that follows
// (engine/kernels/rmsnorm.py:75-95 arithmetic) into it.
//
// Every value travels inside an 8-byte word whose high half is the flag (uint32)(*epoch) + 1
// and is stored whole, so a reader that sees the flag sees the value: no fence, counter, reset
// or barrier sits on the step's path. Column slice q = [q*W/world, (q+1)*W/world) of the
// hidden width W is owned by rank q.
//  1. fb_reduce_scatter_push (after the projection's split-K partials): each rank sums its
//     partials in split order and stores every fp32 value, flagged, only into the owner's
//     receive slab rs[use][rank] - M*W words per rank in total.
//  2. fb_allreduce_add_rmsnorm, phase B (the owner), over (row, 512-column chunk of its slice)
//     work items so that every thread polls once whatever the slice width: polls
//     rs[use][0..world) for its pair of columns, sums the ranks in rank order (the same bits a
//     rank-order sum of whole rows gives), rounds to bf16, adds the residual (rounded again),
//     and stores the summed bf16 pairs, flagged, into ag[use] of every rank; each item also
//     stores its fp32 sum of squares into ss[use][rank][chunk] of every rank.
//     Phase C (every rank, every row): polls ag[use] for the whole row and the row's partial
//     sums of squares, adds those in rank order and chunk order (identical bits on every rank),
//     and writes the normalized row bf16(bf16(s * inv) * w) and the summed row (the next
//     residual).
// NVLink volume per use and rank: M*W*8 bytes of partials plus M*W*4 bytes of summed values
// (1/world of each stays local), against world*M*W*8 for pushing whole partials to every rank.
//
// The consumer's CTAs wait on one another's stores (phase C on other ranks' phase B), so its
// grid never exceeds the SM count: every CTA is resident, each does all its phase-B work before
// any phase-C wait, and every wait is bounded (2 s; on timeout the error word is set and zeros
// are used).
#include "common.cuh"

namespace fb {
namespace ar {

constexpr int kThreads = 256;
constexpr int kBatch = 8;  // split slabs in flight per thread
constexpr int kMaxWorld = 8;
constexpr int kChunk = 2 * kThreads;  // columns of one work item (one pair per thread)
constexpr int kMaxSliceChunks = 16;   // work items per owner slice of a row (N / world <= 8192)

struct PushParams {
  const float* partials;  // [splits, m, n]
  int splits, m, n, world, rank, use;
  uint64_t* peer_rs[kMaxWorld];
  const int64_t* epoch;
};

// One pair of columns per thread: the pair's owner gets one 16-byte store of two flagged words.
__global__ void __launch_bounds__(kThreads) reduce_scatter_push_kernel(const __grid_constant__ PushParams p) {
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
  const int m = static_cast<int>(i / p.n), col = static_cast<int>(i % p.n);
  const int slice = p.n / p.world;
  const int owner = col / slice;
  const size_t off = ((static_cast<size_t>(p.use) * p.world + p.rank) * p.m + m) * slice + (col - owner * slice);
  const uint64_t w0 = flag | __float_as_uint(x.x), w1 = flag | __float_as_uint(x.y);
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p.peer_rs[owner] + off), "l"(w0), "l"(w1)
               : "memory");
}

// The one-phase form's producer: the same split-order sum, then each pair of values, flagged,
// into slab `rank` of recv[use] on every rank (fb_allreduce_sum_add_rmsnorm, in norms.cu, polls
// all slabs and sums them in rank order).
__global__ void __launch_bounds__(kThreads) push_all_kernel(const __grid_constant__ PushParams p) {
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
  for (int q = 0; q < p.world; ++q)
    asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p.peer_rs[q] + off), "l"(w0), "l"(w1)
                 : "memory");
}

struct NormParams {
  const uint64_t* rs;             // this rank's reduce-scatter slabs, all uses
  const uint64_t* ag;             // this rank's all-gather rows, all uses
  const uint64_t* ss;             // this rank's partial sums of squares, all uses
  uint64_t* peer_ag[kMaxWorld];   // every rank's all-gather rows
  uint64_t* peer_ss[kMaxWorld];   // every rank's partial sums of squares
  const int64_t* epoch;
  const __nv_bfloat16* residual;  // [m, n]
  const __nv_bfloat16* w;         // [n]
  __nv_bfloat16* out;             // [m, n]
  __nv_bfloat16* sum;             // [m, n]
  int m, n, world, rank, use, chunks, bchunks;  // chunks of a row (phase C), of a slice (phase B)
  float eps;
  unsigned* err;
};

// Polls `count` (<= kMaxSliceChunks) flagged words at src[0], src[stride], ... until all carry `flag`;
// false after the wait budget (or at once when an earlier wait gave up).
__device__ __forceinline__ bool poll_words(const uint64_t* src, size_t stride, int count, uint32_t flag,
                                           unsigned* err, uint64_t (&words)[kMaxSliceChunks]) {
  unsigned long long start = 0;
  for (;;) {
    bool ready = true;
#pragma unroll
    for (int q = 0; q < kMaxSliceChunks; ++q)
      if (q < count) {
        asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(words[q]) : "l"(src + q * stride));
        ready = ready && static_cast<uint32_t>(words[q] >> 32) == flag;
      }
    if (ready) return true;
    if (start == 0) start = globaltimer();
    if ((err != nullptr && (*reinterpret_cast<volatile unsigned*>(err) & kErrTimeoutFull) != 0) ||
        globaltimer() - start > kWaitBudgetNs) {
      raise_error(err, kErrTimeoutFull);
      return false;
    }
  }
}

// Two consecutive values of each rank's slab (one 16-byte load per rank), summed in rank order.
__device__ __forceinline__ bool poll_pair(const uint64_t* src, size_t stride, int world, uint32_t flag,
                                          unsigned* err, float& x0, float& x1) {
  unsigned long long start = 0;
  for (;;) {
    bool ready = true;
    uint64_t a[kMaxWorld], b[kMaxWorld];
#pragma unroll
    for (int q = 0; q < kMaxWorld; ++q)
      if (q < world)
        asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a[q]), "=l"(b[q]) : "l"(src + q * stride));
#pragma unroll
    for (int q = 0; q < kMaxWorld; ++q)
      if (q < world) {
        ready = ready && static_cast<uint32_t>(a[q] >> 32) == flag && static_cast<uint32_t>(b[q] >> 32) == flag;
        const float u = __uint_as_float(static_cast<uint32_t>(a[q]));
        const float v = __uint_as_float(static_cast<uint32_t>(b[q]));
        x0 = q == 0 ? u : x0 + u;
        x1 = q == 0 ? v : x1 + v;
      }
    if (ready) return true;
    if (start == 0) start = globaltimer();
    if ((err != nullptr && (*reinterpret_cast<volatile unsigned*>(err) & kErrTimeoutFull) != 0) ||
        globaltimer() - start > kWaitBudgetNs) {
      raise_error(err, kErrTimeoutFull);
      x0 = x1 = 0.f;
      return false;
    }
  }
}

__global__ void __launch_bounds__(kThreads) allreduce_norm_kernel(const __grid_constant__ NormParams p) {
  __shared__ float scratch[kThreads / 32];
  // the gains are never written while decoding: none of this kernel's inputs before the wait
  pdl_wait();
  pdl_trigger();
  const uint32_t flag = static_cast<uint32_t>(*p.epoch) + 1u;
  const uint64_t hi = static_cast<uint64_t>(flag) << 32;
  const int W = p.world, slice = p.n / W, half = p.n / 2;
  const size_t use_rs = static_cast<size_t>(p.use) * W * p.m * slice;
  const size_t use_ag = static_cast<size_t>(p.use) * p.m * half;
  const size_t use_ss = static_cast<size_t>(p.use) * W * p.bchunks * p.m;

  // ---- phase B: (row, chunk of this rank's slice) items, every thread one pair of columns,
  // so a slice of any width is one poll per thread ----
  for (int item = blockIdx.x; item < p.m * p.bchunks; item += gridDim.x) {
    const int row = item / p.bchunks, cb = item % p.bchunks;
    float ss = 0.f;
    const int j = cb * kThreads + threadIdx.x;  // pair index within the slice
    if (2 * j < slice) {
      const int col = p.rank * slice + 2 * j;
      float x0, x1;
      poll_pair(p.rs + use_rs + static_cast<size_t>(row) * slice + 2 * j, static_cast<size_t>(p.m) * slice, W,
                flag, p.err, x0, x1);
      const uint32_t r2 = *reinterpret_cast<const uint32_t*>(p.residual + static_cast<size_t>(row) * p.n + col);
      const float s0 = bf16_round(bf16_round(x0) + bf16_lo(r2));
      const float s1 = bf16_round(bf16_round(x1) + bf16_hi(r2));
      ss += s0 * s0;
      ss += s1 * s1;
      const uint64_t word = hi | pack_bf16x2(s0, s1);
      const size_t off = use_ag + static_cast<size_t>(row) * half + col / 2;
      for (int q = 0; q < W; ++q)
        asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p.peer_ag[q] + off), "l"(word) : "memory");
    }
    ss = warp_sum(ss);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) scratch[warp] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      float total = 0.f;
      for (int i = 0; i < kThreads / 32; ++i) total += scratch[i];
      const uint64_t word = hi | __float_as_uint(total);
      const size_t off = use_ss + (static_cast<size_t>(p.rank) * p.bchunks + cb) * p.m + row;
      for (int q = 0; q < W; ++q)
        asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p.peer_ss[q] + off), "l"(word) : "memory");
    }
    __syncthreads();
  }

  // ---- phase C: (row, chunk) items; every thread one pair of columns ----
  for (int item = blockIdx.x; item < p.m * p.chunks; item += gridDim.x) {
    const int row = item / p.chunks, chunk = item % p.chunks;
    const int col = chunk * kChunk + 2 * threadIdx.x;
    if (col >= p.n) continue;
    // the row's partial sums of squares (per rank, per slice chunk), added in rank order and
    // chunk order (the same bits on every rank)
    float total = 0.f;
    for (int q = 0; q < W; ++q) {
      uint64_t words[kMaxSliceChunks];
      if (poll_words(p.ss + use_ss + static_cast<size_t>(q) * p.bchunks * p.m + row, p.m, p.bchunks, flag, p.err,
                     words)) {
#pragma unroll
        for (int c = 0; c < kMaxSliceChunks; ++c)
          if (c < p.bchunks) total += __uint_as_float(static_cast<uint32_t>(words[c]));
      }
    }
    uint64_t pair[kMaxSliceChunks];
    float s0 = 0.f, s1 = 0.f;
    if (poll_words(p.ag + use_ag + static_cast<size_t>(row) * half + col / 2, 0, 1, flag, p.err, pair)) {
      s0 = bf16_lo(static_cast<uint32_t>(pair[0]));
      s1 = bf16_hi(static_cast<uint32_t>(pair[0]));
    }
    const float inv = 1.0f / sqrtf(total / static_cast<float>(p.n) + p.eps);
    const uint32_t w2 = __ldg(reinterpret_cast<const uint32_t*>(p.w + col));
    const size_t o = static_cast<size_t>(row) * p.n + col;
    *reinterpret_cast<uint32_t*>(p.sum + o) = pack_bf16x2(s0, s1);
    *reinterpret_cast<uint32_t*>(p.out + o) =
        pack_bf16x2(bf16_round(s0 * inv) * bf16_lo(w2), bf16_round(s1 * inv) * bf16_hi(w2));
  }
}

}  // namespace ar
}  // namespace fb

using namespace fb;

extern "C" int fb_reduce_scatter_push(const void* partials, int splits, int m, int n, int world, int rank, int use,
                                      void* const* peer_rs, const int64_t* epoch, void* stream) {
  if (!partials || !peer_rs || !epoch || splits <= 0 || m <= 0 || n <= 0) return FB_ERR_ARG;
  if (world < 1 || world > ar::kMaxWorld || rank < 0 || rank >= world || use < 0) return FB_ERR_ARG;
  if (n % (2 * world) != 0) return FB_ERR_SHAPE;
  ar::PushParams p{};
  p.partials = static_cast<const float*>(partials);
  p.splits = splits;
  p.m = m;
  p.n = n;
  p.world = world;
  p.rank = rank;
  p.use = use;
  p.epoch = epoch;
  for (int r = 0; r < world; ++r) {
    if (!peer_rs[r] || (reinterpret_cast<uintptr_t>(peer_rs[r]) & 15u)) return FB_ERR_ARG;
    p.peer_rs[r] = static_cast<uint64_t*>(peer_rs[r]);
  }
  const int64_t threads = static_cast<int64_t>(m) * n / 2;
  const int64_t blocks = (threads + ar::kThreads - 1) / ar::kThreads;
  if (blocks >= (1ll << 31)) return FB_ERR_SHAPE;
  return launch_ex(ar::reduce_scatter_push_kernel, dim3(static_cast<unsigned>(blocks)), dim3(ar::kThreads), 0,
                   static_cast<cudaStream_t>(stream), 1, p);
}

extern "C" int fb_allreduce_add_rmsnorm(const void* rs, const void* ag, const void* ss, void* const* peer_ag,
                                        void* const* peer_ss, int use, int world, int rank, const int64_t* epoch,
                                        const void* residual, const void* w, void* out, void* sum, int rows,
                                        int width, float eps, void* stream) {
  if (!rs || !ag || !ss || !peer_ag || !peer_ss || !epoch || !residual || !w || !out || !sum) return FB_ERR_ARG;
  if (use < 0 || world < 1 || world > ar::kMaxWorld || rank < 0 || rank >= world || rows <= 0 || width <= 0)
    return FB_ERR_ARG;
  if (width % (2 * world) != 0 || width % 8 != 0) return FB_ERR_SHAPE;
  ar::NormParams p{};
  p.rs = static_cast<const uint64_t*>(rs);
  p.ag = static_cast<const uint64_t*>(ag);
  p.ss = static_cast<const uint64_t*>(ss);
  for (int r = 0; r < world; ++r) {
    if (!peer_ag[r] || !peer_ss[r] || (reinterpret_cast<uintptr_t>(peer_ag[r]) & 7u) ||
        (reinterpret_cast<uintptr_t>(peer_ss[r]) & 7u))
      return FB_ERR_ARG;
    p.peer_ag[r] = static_cast<uint64_t*>(peer_ag[r]);
    p.peer_ss[r] = static_cast<uint64_t*>(peer_ss[r]);
  }
  p.epoch = epoch;
  p.residual = static_cast<const __nv_bfloat16*>(residual);
  p.w = static_cast<const __nv_bfloat16*>(w);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.sum = static_cast<__nv_bfloat16*>(sum);
  p.m = rows;
  p.n = width;
  p.world = world;
  p.rank = rank;
  p.use = use;
  p.chunks = (width + ar::kChunk - 1) / ar::kChunk;
  p.bchunks = (width / world + ar::kChunk - 1) / ar::kChunk;
  if (p.bchunks > ar::kMaxSliceChunks) return FB_ERR_SHAPE;
  p.eps = eps;
  p.err = error_word();
  // every CTA resident at once (phase C waits on phase B of other CTAs, here and on the peers)
  long long grid = static_cast<long long>(rows) * (p.chunks > p.bchunks ? p.chunks : p.bchunks);
  if (grid > sm_count()) grid = sm_count();
  return launch_ex(ar::allreduce_norm_kernel, dim3(static_cast<unsigned>(grid)), dim3(ar::kThreads), 0,
                   static_cast<cudaStream_t>(stream), 1, p);
}

extern "C" int fb_allreduce_push(const void* partials, int splits, int m, int n, int world, int rank, int use,
                                 void* const* peer_recv, const int64_t* epoch, void* stream) {
  if (!partials || !peer_recv || !epoch || splits <= 0 || m <= 0 || n <= 0) return FB_ERR_ARG;
  if (world < 1 || world > ar::kMaxWorld || rank < 0 || rank >= world || use < 0) return FB_ERR_ARG;
  if (n % 2 != 0) return FB_ERR_SHAPE;
  ar::PushParams p{};
  p.partials = static_cast<const float*>(partials);
  p.splits = splits;
  p.m = m;
  p.n = n;
  p.world = world;
  p.rank = rank;
  p.use = use;
  p.epoch = epoch;
  for (int r = 0; r < world; ++r) {
    if (!peer_recv[r] || (reinterpret_cast<uintptr_t>(peer_recv[r]) & 15u)) return FB_ERR_ARG;
    p.peer_rs[r] = static_cast<uint64_t*>(peer_recv[r]);
  }
  const int64_t threads = static_cast<int64_t>(m) * n / 2;
  const int64_t blocks = (threads + ar::kThreads - 1) / ar::kThreads;
  if (blocks >= (1ll << 31)) return FB_ERR_SHAPE;
  return launch_ex(ar::push_all_kernel, dim3(static_cast<unsigned>(blocks)), dim3(ar::kThreads), 0,
                   static_cast<cudaStream_t>(stream), 1, p);
}
